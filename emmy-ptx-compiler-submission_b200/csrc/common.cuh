// Shared host/device helpers for libemmyb200: status codes, error text,
// launch checks, warp reductions and streaming memory access.
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <stdint.h>
#include <stdio.h>
#include <stdarg.h>
#include <type_traits>

#include "../../include/emmy_b200.h"

namespace emmy {

// ---------------------------------------------------------------- host side

// Records the calling thread's last error message; returns `code`.
int set_error(int code, const char *fmt, ...);
void clear_error();
const char *last_error_text();

// Check the launch that was just queued; map a CUDA error to EMMY_ERR_CUDA.
int check_launch(const char *what);

inline cudaStream_t as_stream(void *s) { return reinterpret_cast<cudaStream_t>(s); }

inline bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

inline int sm_count() {
  static int cached[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return 148;
  if (!cached[dev]) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    cached[dev] = n > 0 ? n : 148;
  }
  return cached[dev];
}

// Attention on CUDA cores with one thread per query row (attention_rows.cu):
// -1 when there is no kernel for (d, dv), else the launch status.
int launch_attention_rows(const void *q, const void *k, const void *v, void *o,
                          const float *scale_div, int64_t batch, int64_t sq, int64_t sk,
                          int64_t d, int64_t dv, int in_f16, int out_f16, int k_transposed,
                          cudaStream_t st);

// Device address of one of this library's __device__ variables in the current
// device's current context (looked up with cudaGetSymbolAddress on first use
// in that context and cached; thread-safe).  Host code must pass this address
// to kernels, never the symbol itself, which on the host names a stand-in.
// Returns nullptr and sets *rc (with the error text) on failure.
void *symbol_address(const void *symbol, int *rc);

// Device address of the library's status word on the current device.  Kernels
// with bounded waits receive it as an argument and write a nonzero code there
// instead of hanging or trapping; emmy_get_device_status() reads and clears it.
int *device_status_ptr();

// ---------------------------------------------------------------- device side

// Seeds used by the reference for max/min folds (ptxc/ops.py:67-75).
constexpr float kMaxSeed = -1e30f;
constexpr float kMinSeed = 1e30f;

__device__ __forceinline__ float4 ld_stream4(const float *p) {
  return __ldcs(reinterpret_cast<const float4 *>(p));
}
__device__ __forceinline__ void st_stream4(float *p, float4 v) {
  __stcs(reinterpret_cast<float4 *>(p), v);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ float warp_min(float v) {
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) v = fminf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

}  // namespace emmy
