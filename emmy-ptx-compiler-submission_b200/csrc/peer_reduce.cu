// Reduce-scatter of split-K partials over peer memory: the exchange step of a
// matmul whose K is split across GPUs (the multi-GPU form of the reference's
// atomic split-K writes, reference ptxc/stmts.py:456-461).
//
// Every rank has run its K slice into a full-size partial C (the plain f32
// GEMM with in-GPU atomic split-K) in buffer `seq % 2` of a double-buffered
// pair that every rank has mapped (CUDA IPC).  This kernel then, on each rank:
//   1. publishes `seq` into every rank's flag word for this rank (a
//      system-scope release store over NVLink; every block stores it, so no
//      block depends on another being scheduled);
//   2. waits until its own flag words hold `seq` from every rank (system-scope
//      acquire loads, bounded: after the limit it records a status code and
//      returns without reading);
//   3. sums the `world` partials of the rows it owns (peer loads over NVLink)
//      into `out`.
// A rank's partials of step seq are read by the others during their step seq;
// its GEMM of step seq + 2 overwrites the same buffer only after its step
// seq + 1 wait has passed, which every other rank's step seq must have
// finished before publishing.  No host barrier, no NCCL call, no remote atomic.

#include "common.cuh"
#include "tma.cuh"

namespace emmy {

constexpr int kPeerMaxWorld = 8;
constexpr int kStatusPeerWait = 0x1301;

struct PeerReduceArgs {
  const float *parts[kPeerMaxWorld];          // every rank's partial buffer (this step's)
  long long *flags[kPeerMaxWorld];            // every rank's flag words [world]
  float *out;
  long long seq;
  long long row0, rows, n;                    // this rank's rows of C, columns
  int world, me;
};

__device__ __forceinline__ void st_release_sys(long long *p, long long v) {
  asm volatile("st.release.sys.global.b64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ long long ld_acquire_sys(const long long *p) {
  long long v;
  asm volatile("ld.acquire.sys.global.b64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__global__ void __launch_bounds__(256) peer_reduce_rows_kernel(const PeerReduceArgs a, int *status) {
  __shared__ int ready;
  if (threadIdx.x == 0) {
    // the GEMM before this kernel on the stream is complete: publish this step
    __threadfence_system();
    for (int r = 0; r < a.world; ++r) st_release_sys(a.flags[r] + a.me, a.seq);
    bool ok = true;
    const unsigned long long t0 = global_ns();
    for (int r = 0; ok && r < a.world; ++r) {
      while (ld_acquire_sys(a.flags[a.me] + r) < a.seq) {
        if (global_ns() - t0 > kWaitLimitNs) {
          atomicCAS(status, 0, kStatusPeerWait);
          ok = false;
          break;
        }
      }
    }
    ready = ok;
  }
  __syncthreads();
  if (!ready) return;
  // rows row0 .. row0 + rows of every partial, as float4 when the row pitch allows
  const int64_t total = a.rows * a.n;
  const int64_t base = a.row0 * a.n;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  if (a.n % 4 == 0) {
    const int64_t t4 = total / 4;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < t4; i += stride) {
      float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int r = 0; r < a.world; ++r) {
        const float4 v = *reinterpret_cast<const float4 *>(a.parts[r] + base + 4 * i);
        s.x += v.x; s.y += v.y; s.z += v.z; s.w += v.w;
      }
      *reinterpret_cast<float4 *>(a.out + 4 * i) = s;
    }
  } else {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += stride) {
      float s = 0.f;
      for (int r = 0; r < a.world; ++r) s += a.parts[r][base + i];
      a.out[i] = s;
    }
  }
}

}  // namespace emmy

using namespace emmy;

extern "C" int emmy_peer_reduce_rows(const float *const *parts, long long *const *flags, int world,
                                     int me, long long seq, int64_t row0, int64_t rows, int64_t n,
                                     float *out, void *stream) {
  clear_error();
  if (world < 1 || world > kPeerMaxWorld || me < 0 || me >= world)
    return set_error(EMMY_ERR_INVALID, "emmy_peer_reduce_rows: bad world / rank");
  if (row0 < 0 || rows < 0 || n < 0 || seq < 1)
    return set_error(EMMY_ERR_INVALID, "emmy_peer_reduce_rows: bad rows, columns or step");
  if (!parts || !flags || (rows > 0 && n > 0 && !out))
    return set_error(EMMY_ERR_INVALID, "emmy_peer_reduce_rows: null argument");
  PeerReduceArgs a{};
  for (int r = 0; r < world; ++r) {
    if (!parts[r] || !flags[r])
      return set_error(EMMY_ERR_INVALID, "emmy_peer_reduce_rows: null buffer of rank %d", r);
    if ((n % 4 == 0) && ((uintptr_t)(parts[r] + row0 * n) % 16) != 0)
      return set_error(EMMY_ERR_INVALID, "emmy_peer_reduce_rows: partial of rank %d not 16-byte aligned", r);
    a.parts[r] = parts[r];
    a.flags[r] = flags[r];
  }
  if ((n % 4 == 0) && rows > 0 && ((uintptr_t)out % 16) != 0)
    return set_error(EMMY_ERR_INVALID, "emmy_peer_reduce_rows: output not 16-byte aligned");
  a.out = out;
  a.seq = seq;
  a.row0 = row0;
  a.rows = rows;
  a.n = n;
  a.world = world;
  a.me = me;
  // enough blocks to stream the rows, at most two per SM (all resident: every
  // block waits on the flags)
  const int64_t work = (rows * n + 1023) / 1024;
  int64_t blocks = work < 1 ? 1 : work;
  const int64_t cap = 2 * (int64_t)sm_count();
  if (blocks > cap) blocks = cap;
  peer_reduce_rows_kernel<<<(unsigned)blocks, 256, 0, as_stream(stream)>>>(a, device_status_ptr());
  return check_launch("emmy_peer_reduce_rows");
}
