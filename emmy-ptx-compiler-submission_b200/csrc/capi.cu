// C-ABI plumbing shared by every family: version, thread-local error text,
// launch checks and the device status word.

#include "common.cuh"
#include "tma.cuh"

#include <mutex>
#include <string.h>

namespace emmy {

__device__ int g_device_status = 0;

namespace {
thread_local char t_error[512] = {0};
}

int set_error(int code, const char *fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(t_error, sizeof(t_error), fmt, ap);
  va_end(ap);
  return code;
}

void clear_error() { t_error[0] = 0; }

const char *last_error_text() { return t_error; }

namespace {
typedef int (*PFN_ctxGetCurrent)(void **ctx);
PFN_ctxGetCurrent ctx_get_current_fn() {
  static PFN_ctxGetCurrent fn = []() -> PFN_ctxGetCurrent {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      return reinterpret_cast<PFN_ctxGetCurrent>(p);
    return nullptr;
  }();
  return fn;
}

struct SymbolSlot {
  const void *symbol;
  int dev;
  void *ctx;
  void *addr;
};
std::mutex g_symbol_mutex;
SymbolSlot g_symbol_slots[256];
int g_symbol_used = 0;
}  // namespace

void *symbol_address(const void *symbol, int *rc) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    *rc = set_error(EMMY_ERR_CUDA, "no current device: %s", cudaGetErrorString(e));
    return nullptr;
  }
  // the context is part of the key: after a device reset the module is
  // loaded afresh and its symbols may move
  void *ctx = nullptr;
  if (auto get = ctx_get_current_fn()) get(&ctx);
  std::lock_guard<std::mutex> lock(g_symbol_mutex);
  for (int i = 0; i < g_symbol_used; ++i) {
    const SymbolSlot &s = g_symbol_slots[i];
    if (s.symbol == symbol && s.dev == dev && s.ctx == ctx) {
      *rc = EMMY_OK;
      return s.addr;
    }
  }
  void *p = nullptr;
  e = cudaGetSymbolAddress(&p, symbol);
  if (e != cudaSuccess || p == nullptr) {
    *rc = set_error(EMMY_ERR_CUDA, "cudaGetSymbolAddress: %s", cudaGetErrorString(e));
    return nullptr;
  }
  int slot = -1;
  for (int i = 0; i < g_symbol_used; ++i)
    if (g_symbol_slots[i].symbol == symbol && g_symbol_slots[i].dev == dev) slot = i;   // stale
  if (slot < 0 && g_symbol_used < 256) slot = g_symbol_used++;
  if (slot >= 0) g_symbol_slots[slot] = SymbolSlot{symbol, dev, ctx, p};
  *rc = EMMY_OK;
  return p;
}

int *device_status_ptr() {
  int rc = 0;
  return static_cast<int *>(symbol_address(reinterpret_cast<const void *>(&g_device_status), &rc));
}

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

int make_tensor_map(CUtensorMap *map, CUtensorMapDataType dtype, int rank, const void *base,
                    const uint64_t *dims, const uint64_t *strides_bytes, const uint32_t *box,
                    CUtensorMapSwizzle swizzle) {
  auto enc = tensor_map_encoder();
  if (!enc) return set_error(EMMY_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  cuuint32_t elem_strides[5] = {1, 1, 1, 1, 1};
  CUresult r = enc(map, dtype, (cuuint32_t)rank, const_cast<void *>(base),
                   reinterpret_cast<const cuuint64_t *>(dims),
                   reinterpret_cast<const cuuint64_t *>(strides_bytes),
                   reinterpret_cast<const cuuint32_t *>(box), elem_strides,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(EMMY_ERR_INVALID, "tensor map encode failed (%d)", (int)r);
  return EMMY_OK;
}

int check_launch(const char *what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess)
    return set_error(EMMY_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
  return EMMY_OK;
}

}  // namespace emmy

using namespace emmy;

extern "C" int emmy_version(void) { return 100; }

extern "C" const char *emmy_last_error(void) { return last_error_text(); }

extern "C" int emmy_get_device_status(int *code, void *stream) {
  clear_error();
  if (!code) return set_error(EMMY_ERR_INVALID, "emmy_get_device_status: null output");
  cudaStream_t st = as_stream(stream);
  int host = 0;
  cudaError_t e = cudaMemcpyFromSymbolAsync(&host, g_device_status, sizeof(int), 0,
                                            cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e != cudaSuccess)
    return set_error(EMMY_ERR_CUDA, "emmy_get_device_status: %s", cudaGetErrorString(e));
  *code = host;
  if (host != 0) {
    int zero = 0;
    e = cudaMemcpyToSymbolAsync(g_device_status, &zero, sizeof(int), 0,
                                cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (e != cudaSuccess)
      return set_error(EMMY_ERR_CUDA, "emmy_get_device_status: %s", cudaGetErrorString(e));
  }
  return EMMY_OK;
}

extern "C" int emmy_zero(void *ptr, size_t bytes, void *stream) {
  clear_error();
  if (bytes == 0) return EMMY_OK;
  if (!ptr) return set_error(EMMY_ERR_INVALID, "emmy_zero: null pointer");
  cudaError_t e = cudaMemsetAsync(ptr, 0, bytes, as_stream(stream));
  if (e != cudaSuccess) return set_error(EMMY_ERR_CUDA, "emmy_zero: %s", cudaGetErrorString(e));
  return EMMY_OK;
}

// ---------------------------------------------------------------------------
// Peer mappings of device buffers between the processes of one node (CUDA
// IPC), for kernels that write another GPU's memory over NVLink.  A buffer is
// exported as the handle of the allocation that holds it plus the offset into
// it (an allocator may hand out pieces of a larger allocation).

namespace {
typedef int (*PFN_getAddressRange)(unsigned long long *base, size_t *size, unsigned long long ptr);
PFN_getAddressRange address_range_fn() {
  static PFN_getAddressRange fn = nullptr;
  if (!fn) {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_getAddressRange>(p);
  }
  return fn;
}
}  // namespace

extern "C" int emmy_ipc_export(const void *ptr, void *handle, int64_t *offset) {
  clear_error();
  if (!ptr || !handle || !offset) return set_error(EMMY_ERR_INVALID, "emmy_ipc_export: null argument");
  auto range = address_range_fn();
  if (!range) return set_error(EMMY_ERR_CUDA, "cuMemGetAddressRange is unavailable");
  unsigned long long base = 0;
  size_t size = 0;
  if (range(&base, &size, reinterpret_cast<unsigned long long>(ptr)) != 0)
    return set_error(EMMY_ERR_INVALID, "emmy_ipc_export: not a device allocation");
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, reinterpret_cast<void *>(base));
  if (e != cudaSuccess) return set_error(EMMY_ERR_CUDA, "emmy_ipc_export: %s", cudaGetErrorString(e));
  memcpy(handle, &h, sizeof(h));
  *offset = (int64_t)(reinterpret_cast<unsigned long long>(ptr) - base);
  return EMMY_OK;
}

extern "C" int emmy_ipc_import(const void *handle, int64_t offset, void **peer_ptr,
                               void **peer_base) {
  clear_error();
  if (!handle || !peer_ptr || !peer_base || offset < 0)
    return set_error(EMMY_ERR_INVALID, "emmy_ipc_import: bad argument");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  void *base = nullptr;
  cudaError_t e = cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return set_error(EMMY_ERR_CUDA, "emmy_ipc_import: %s", cudaGetErrorString(e));
  *peer_base = base;
  *peer_ptr = static_cast<char *>(base) + offset;
  return EMMY_OK;
}

extern "C" int emmy_ipc_close(void *peer_base) {
  clear_error();
  if (!peer_base) return EMMY_OK;
  cudaError_t e = cudaIpcCloseMemHandle(peer_base);
  if (e != cudaSuccess) return set_error(EMMY_ERR_CUDA, "emmy_ipc_close: %s", cudaGetErrorString(e));
  return EMMY_OK;
}
