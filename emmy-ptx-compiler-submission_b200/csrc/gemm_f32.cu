// f32 and f64 GEMM / batched GEMM / split-K on sm_100a CUDA cores.
//
// Replaces the entry the reference emits for its tiled-matmul IR shape: a
// Tile over (m-block, n-block, m-lane, n-lane) axes, cp.async.cg 16-byte
// copies into double-buffered _a_smem/_b_smem, an inner Loop over the smem
// K-tile folding fma.rn into a per-thread register micro-tile, and direct (or,
// with a split-K Tile axis, red.global.add) writes (reference
// ptxc/stmts.py:663-725, 614-632, 1590-1623, 434-487; fixtures v_m_*, w_m_*).
//
// Here: a 128x128 CTA tile with BK = 16, 256 threads each owning an 8x8
// register tile (rows ty + 16*i, columns 4*tx + {0..3} and 64 + 4*tx + {0..3},
// which keeps every 128-bit shared load conflict-free), operands staged by TMA
// (cp.async.bulk.tensor) into a 4-stage shared-memory ring whose stages
// complete on mbarriers, one elected thread issuing the copies.  Products
// accumulate with fma in f32, as the reference's fused accumulate does.  A
// split-K launch gives each CTA a K range and combines partials with 128-bit
// vector atomics (red.global.add.v4.f32), the reference's atomic Write.
//
// f64 (the reference's fma.rn.f64 accumulate, ptxc/expr.py:1179-1309) runs
// the same kernel on doubles: BK = 8 keeps A's shared rows at 64 bytes, the
// 8x8 register tile holds 64 doubles (one CTA of 256 threads per SM), and
// split-K partials meet in f64 atomic adds.  The tcgen05 tensor cores have no
// f64 kind; DFMA on the CUDA cores is the f64 path.
//
// Shapes TMA cannot describe (K or N not a multiple of 16 bytes, unaligned
// bases) take a plain shared-memory tiled kernel instead.

#include "common.cuh"
#include "tma.cuh"

namespace emmy {

namespace gemm32 {
constexpr int BM = 128, BN = 128, STAGES = 4, THREADS = 256;
template <typename T> struct Cfg {
  static constexpr int BK = 64 / (int)sizeof(T);        // 64-byte rows of A in shared memory
  static constexpr int VK = 16 / (int)sizeof(T);        // elements per 16-byte shared load
  static constexpr int A_BYTES = BM * BK * (int)sizeof(T);
  static constexpr int B_BYTES = BK * BN * (int)sizeof(T);
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024;
};
}  // namespace gemm32

// 16-byte shared loads of VK consecutive elements, and four consecutive
// elements (one or two 16-byte loads).
__device__ __forceinline__ void lds_vk(const float *p, float v[4]) {
  const float4 a = *reinterpret_cast<const float4 *>(p);
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
}
__device__ __forceinline__ void lds_vk(const double *p, double v[2]) {
  const double2 a = *reinterpret_cast<const double2 *>(p);
  v[0] = a.x; v[1] = a.y;
}
__device__ __forceinline__ void lds4(const float *p, float v[4]) { lds_vk(p, v); }
__device__ __forceinline__ void lds4(const double *p, double v[4]) {
  lds_vk(p, v);
  lds_vk(p + 2, v + 2);
}
__device__ __forceinline__ float fma_t(float a, float b, float c) { return fmaf(a, b, c); }
__device__ __forceinline__ double fma_t(double a, double b, double c) { return fma(a, b, c); }

// acc[j] = fma(a, b[j], acc[j]) for j < 8.  For f32 on sm_100a this is four
// packed fma.rn.f32x2 (two lanes' fused multiply-adds per instruction, each
// rounded exactly as fmaf): the CUDA-core GEMM is issue-bound, and the packed
// form halves the FMA issue slots.
__device__ __forceinline__ void fma_row8(double acc[8], double a, const double b[8]) {
#pragma unroll
  for (int j = 0; j < 8; ++j) acc[j] = fma(a, b[j], acc[j]);
}
__device__ __forceinline__ void fma_row8(float acc[8], float a, const float b[8]) {
  unsigned long long ap;
  asm("mov.b64 %0, {%1, %1};" : "=l"(ap) : "f"(a));
#pragma unroll
  for (int p = 0; p < 4; ++p) {
    unsigned long long bp, cp;
    asm("mov.b64 %0, {%1, %2};" : "=l"(bp) : "f"(b[2 * p]), "f"(b[2 * p + 1]));
    asm("mov.b64 %0, {%1, %2};" : "=l"(cp) : "f"(acc[2 * p]), "f"(acc[2 * p + 1]));
    asm("fma.rn.f32x2 %0, %1, %2, %0;" : "+l"(cp) : "l"(ap), "l"(bp));
    asm("mov.b64 {%0, %1}, %2;" : "=f"(acc[2 * p]), "=f"(acc[2 * p + 1]) : "l"(cp));
  }
}
__device__ __forceinline__ void atomic_add4(float *dst, const float v[4]) {
  atomicAdd(reinterpret_cast<float4 *>(dst), make_float4(v[0], v[1], v[2], v[3]));
}
__device__ __forceinline__ void atomic_add4(double *dst, const double v[4]) {
#pragma unroll
  for (int j = 0; j < 4; ++j) atomicAdd(dst + j, v[j]);
}
__device__ __forceinline__ void st4(float *dst, const float v[4]) {
  *reinterpret_cast<float4 *>(dst) = make_float4(v[0], v[1], v[2], v[3]);
}
__device__ __forceinline__ void st4(double *dst, const double v[4]) {
  reinterpret_cast<double2 *>(dst)[0] = make_double2(v[0], v[1]);
  reinterpret_cast<double2 *>(dst)[1] = make_double2(v[2], v[3]);
}

enum GemmMode { GEMM_STORE = 0, GEMM_ACCUMULATE = 1, GEMM_ATOMIC = 2, GEMM_PEER = 3 };

// GEMM_PEER: a matmul and the reduce-scatter of its partial sums in one
// kernel.  Row m of this rank's partial product is stored (plain 16-byte
// stores; over NVLink when another GPU owns the row) into owner
// o = m / rows_per_rank's slot buffer, in slot `me`, row m % rows_per_rank:
// slots[o] is [world, rows_per_rank, N] and each rank writes only its own
// slot, so nothing needs zeroing and no remote atomics are issued.  The owner
// then sums its world slots (emmy_reduce_f32 over the slot axis).  With a K
// split inside the rank, the splits of a tile first meet in a local workspace
// (vector atomics); the last split to finish the tile (a per-tile arrival
// counter) stores the summed tile and clears the workspace tile and the
// counter for the next call, so each element crosses NVLink once.
struct PeerRows {
  void *rows[8];      // slot buffers of the owners, in this process's address space
  long long rows_per_rank;
  float *ws;          // M x N, zero between calls (the kernel leaves it zero)
  int *counters;      // one per 128 x 128 tile, zero between calls
  int me;             // this rank: the slot it writes
};

template <typename T>
__device__ __forceinline__ T *gemm_dst(T *Cb, const PeerRows &pr, int mode, int m, int n, int N) {
  if (mode == GEMM_PEER) {
    const int owner = (int)(m / pr.rows_per_rank);
    void *base = pr.rows[0];
#pragma unroll
    for (int r = 1; r < 8; ++r)            // a select chain: no local copy of the array
      if (owner == r) base = pr.rows[r];
    return static_cast<T *>(base) +
           ((int64_t)pr.me * pr.rows_per_rank + (m - owner * pr.rows_per_rank)) * N + n;
  }
  return Cb + (int64_t)m * N + n;
}

template <typename T>
__global__ void __launch_bounds__(gemm32::THREADS, sizeof(T) == 4 ? 2 : 1)
gemm_simt_tma_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                     const T *__restrict__ bias, T *__restrict__ C, int M, int N, int K,
                     int64_t c_batch_stride, int splits, int k_per_split, int epilogue, int mode,
                     const PeerRows peers, int *status) {
  using namespace gemm32;
  constexpr int BK = Cfg<T>::BK, VK = Cfg<T>::VK;
  constexpr int A_BYTES = Cfg<T>::A_BYTES, STAGE_BYTES = Cfg<T>::STAGE_BYTES;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char *smem = reinterpret_cast<unsigned char *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ __align__(8) uint64_t full[STAGES];

  const int tid = threadIdx.x;
  const int tx = tid & 15, ty = tid >> 4;
  const int m0 = blockIdx.x * BM, n0 = blockIdx.y * BN;
  const int batch = blockIdx.z / splits, split = blockIdx.z - batch * splits;
  const int kb = split * k_per_split;
  const int ke = min(K, kb + k_per_split);
  const int ntiles = ke > kb ? (ke - kb + BK - 1) / BK : 0;

  if (tid == 0) {
    prefetch_tensormap(&tmA);
    prefetch_tensormap(&tmB);
    for (int s = 0; s < STAGES; ++s) mbar_init(&full[s], 1);
    fence_barrier_init();
  }
  __syncthreads();

  auto issue = [&](int t) {
    const int s = t % STAGES;
    T *As = reinterpret_cast<T *>(smem + s * STAGE_BYTES);
    T *Bs = reinterpret_cast<T *>(smem + s * STAGE_BYTES + A_BYTES);
    mbar_expect_tx(&full[s], STAGE_BYTES);
    const int k = kb + t * BK;
    tma_load_3d(As, &tmA, &full[s], k, m0, batch);
    tma_load_3d(Bs, &tmB, &full[s], n0, k, batch);
  };
  if (tid == 0)
    for (int t = 0; t < STAGES - 1 && t < ntiles; ++t) issue(t);

  T acc[8][8];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[i][j] = T(0);

  int failed_at = -1;
  for (int t = 0; t < ntiles; ++t) {
    const int s = t % STAGES;
    if (tid == 0 && t + STAGES - 1 < ntiles) issue(t + STAGES - 1);
    const bool ok = mbar_wait(&full[s], (t / STAGES) & 1, status, kStatusMbarTimeout);
    const T *As = reinterpret_cast<const T *>(smem + s * STAGE_BYTES);
    const T *Bs = reinterpret_cast<const T *>(smem + s * STAGE_BYTES + A_BYTES);
#pragma unroll
    for (int kk = 0; kk < BK; kk += VK) {
      T a[8][VK];
#pragma unroll
      for (int i = 0; i < 8; ++i) lds_vk(As + (ty + 16 * i) * BK + kk, a[i]);
#pragma unroll
      for (int q = 0; q < VK; ++q) {
        T b[8];
        lds4(Bs + (kk + q) * BN + 4 * tx, b);
        lds4(Bs + (kk + q) * BN + 64 + 4 * tx, b + 4);
#pragma unroll
        for (int i = 0; i < 8; ++i) fma_row8(acc[i], a[i][q], b);
      }
    }
    // every thread is done with stage s before thread 0 refills it next trip;
    // the vote makes a timed-out wait a block-uniform exit
    if (__syncthreads_or(!ok)) {
      failed_at = t;
      break;
    }
  }
  if (failed_at >= 0) {
    // a copy never arrived: leave C untouched (the host sees EMMY_ERR_DEVICE);
    // before exiting, wait (bounded) for this CTA's copies still in flight
    if (tid == 0) {
      const int issued = min(ntiles, failed_at + STAGES);
      for (int u = failed_at; u < issued; ++u)
        mbar_wait(&full[u % STAGES], (u / STAGES) & 1, nullptr, 0);
    }
    __syncthreads();
    return;
  }

  T *Cb = C + (int64_t)batch * c_batch_stride;
  const bool peer_ws = mode == GEMM_PEER && splits > 1 && sizeof(T) == 4;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int m = m0 + ty + 16 * i;
    if (m >= M) continue;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int n = n0 + 64 * h + 4 * tx;
      if (n >= N) continue;
      T v[4] = {acc[i][4 * h], acc[i][4 * h + 1], acc[i][4 * h + 2], acc[i][4 * h + 3]};
      if ((epilogue & EMMY_EPI_BIAS) && bias && (mode < GEMM_ATOMIC || split == 0)) {
#pragma unroll
        for (int j = 0; j < 4; ++j) v[j] += (n + j < N) ? __ldg(bias + n + j) : T(0);
      }
      if (epilogue & EMMY_EPI_RELU) {
#pragma unroll
        for (int j = 0; j < 4; ++j) v[j] = fmax(v[j], T(0));
      }
      T *dst = peer_ws ? reinterpret_cast<T *>(peers.ws) + (int64_t)m * N + n
                       : gemm_dst(Cb, peers, mode, m, n, N);
      if (mode == GEMM_PEER && !peer_ws) {
        if (n + 3 < N) st4(dst, v);
        else
          for (int j = 0; j < 4 && n + j < N; ++j) dst[j] = v[j];
      } else if (peer_ws) {
        if (n + 3 < N) atomic_add4(dst, v);
        else
          for (int j = 0; j < 4 && n + j < N; ++j) atomicAdd(dst + j, v[j]);
      } else if (n + 3 < N) {
        if (mode == GEMM_ATOMIC) {
          atomic_add4(dst, v);
        } else if (mode == GEMM_ACCUMULATE) {
          T o[4];
#pragma unroll
          for (int j = 0; j < 4; ++j) o[j] = dst[j] + v[j];
          st4(dst, o);
        } else {
          st4(dst, v);
        }
      } else {
        for (int j = 0; j < 4 && n + j < N; ++j) {
          if (mode == GEMM_ATOMIC) atomicAdd(dst + j, v[j]);
          else if (mode == GEMM_ACCUMULATE) dst[j] += v[j];
          else dst[j] = v[j];
        }
      }
    }
  }
  if constexpr (sizeof(T) == 4) {
    if (peer_ws) {
      // the last split of this tile pushes the summed tile to its owner
      __shared__ int s_last;
      __syncthreads();
      const int tile = blockIdx.x + blockIdx.y * gridDim.x;
      if (tid == 0) {
        __threadfence();                                // this CTA's adds are visible
        s_last = atomicAdd(peers.counters + tile, 1) == splits - 1;
      }
      __syncthreads();
      if (s_last) {
        __threadfence();
#pragma unroll 1
        for (int i = 0; i < 8; ++i) {
          const int m = m0 + ty + 16 * i;
          if (m >= M) continue;
          for (int h = 0; h < 2; ++h) {
            const int n = n0 + 64 * h + 4 * tx;
            if (n >= N) continue;
            float *w = peers.ws + (int64_t)m * N + n;
            float *dst = gemm_dst(reinterpret_cast<float *>(Cb), peers, GEMM_PEER, m, n, N);
            if (n + 3 < N) {
              *reinterpret_cast<float4 *>(dst) = __ldcg(reinterpret_cast<const float4 *>(w));
              *reinterpret_cast<float4 *>(w) = make_float4(0.f, 0.f, 0.f, 0.f);
            } else {
              for (int j = 0; j < 4 && n + j < N; ++j) {
                dst[j] = __ldcg(w + j);
                w[j] = 0.f;
              }
            }
          }
        }
        if (tid == 0) peers.counters[tile] = 0;
      }
    }
  }
}

// Plain shared-memory tiled kernel for shapes TMA cannot describe.
// 64x64 CTA tile, 256 threads, 4x4 outputs per thread, BK = 16.
template <typename T>
__global__ void __launch_bounds__(256)
gemm_simt_plain_kernel(const T *__restrict__ A, const T *__restrict__ B,
                       const T *__restrict__ bias, T *__restrict__ C, int M, int N, int K,
                       int64_t sa, int64_t sb, int64_t sc, int splits, int k_per_split,
                       int epilogue, int mode, const PeerRows peers) {
  __shared__ T As[16][64 + 1];
  __shared__ T Bs[16][64 + 1];
  const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
  const int m0 = blockIdx.x * 64, n0 = blockIdx.y * 64;
  const int batch = blockIdx.z / splits, split = blockIdx.z - batch * splits;
  const int kb = split * k_per_split, ke = min(K, kb + k_per_split);
  const T *Ab = A + (int64_t)batch * sa;
  const T *Bb = B + (int64_t)batch * sb;
  T acc[4][4] = {};
  for (int k0 = kb; k0 < ke; k0 += 16) {
    for (int i = tid; i < 16 * 64; i += 256) {
      const int r = i / 16, c = i % 16;          // A tile: 64 rows x 16 k
      const int m = m0 + r, k = k0 + c;
      As[c][r] = (m < M && k < ke) ? Ab[(int64_t)m * K + k] : T(0);
      const int kr = i / 64, nc = i % 64;        // B tile: 16 k x 64 cols
      const int kk = k0 + kr, n = n0 + nc;
      Bs[kr][nc] = (kk < ke && n < N) ? Bb[(int64_t)kk * N + n] : T(0);
    }
    __syncthreads();
#pragma unroll
    for (int k = 0; k < 16; ++k)
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fma_t(As[k][ty + 16 * i], Bs[k][tx + 16 * j], acc[i][j]);
    __syncthreads();
  }
  T *Cb = C + (int64_t)batch * sc;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int m = m0 + ty + 16 * i;
    if (m >= M) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int n = n0 + tx + 16 * j;
      if (n >= N) continue;
      T v = acc[i][j];
      if ((epilogue & EMMY_EPI_BIAS) && bias && (mode < GEMM_ATOMIC || split == 0)) v += bias[n];
      if (epilogue & EMMY_EPI_RELU) v = fmax(v, T(0));
      T *dst = gemm_dst(Cb, peers, mode, m, n, N);
      if (mode == GEMM_PEER) *dst = v;
      else if (mode == GEMM_ATOMIC) atomicAdd(dst, v);
      else if (mode == GEMM_ACCUMULATE) *dst += v;
      else *dst = v;
    }
  }
}

}  // namespace emmy

using namespace emmy;

template <typename T>
static int gemm_simt(const char *name, const T *A, const T *B, const T *bias, T *C, int64_t batch,
                     int64_t M, int64_t N, int64_t K, int64_t a_batch_stride,
                     int64_t b_batch_stride, int64_t c_batch_stride, int splits, int accumulate,
                     int epilogue, void *stream, const PeerRows *peers = nullptr) {
  using namespace gemm32;
  constexpr int BK = Cfg<T>::BK, SMEM_BYTES = Cfg<T>::SMEM_BYTES;
  constexpr int ES = (int)sizeof(T), VEC = 16 / ES;
  clear_error();
  if (batch < 0 || M < 0 || N < 0 || K < 0 || splits < 0)
    return set_error(EMMY_ERR_INVALID, "%s: negative size", name);
  if (batch == 0 || M == 0 || N == 0) return EMMY_OK;
  if (!A || !B || !C) return set_error(EMMY_ERR_INVALID, "%s: null operand", name);
  if (M > INT32_MAX || N > INT32_MAX || K > INT32_MAX || batch > 65535)
    return set_error(EMMY_ERR_UNSUPPORTED, "%s: size beyond 32-bit tile indexing", name);
  if (epilogue & ~(EMMY_EPI_BIAS | EMMY_EPI_RELU))
    return set_error(EMMY_ERR_INVALID, "%s: unknown epilogue bits %d", name, epilogue);
  if ((epilogue & EMMY_EPI_RELU) && (splits > 1 || accumulate))
    return set_error(EMMY_ERR_INVALID, "%s: relu cannot follow a partial sum", name);
  cudaStream_t st = as_stream(stream);
  const int sms = sm_count();
  const int64_t mt = (M + BM - 1) / BM, nt = (N + BN - 1) / BN;
  // split count: the caller's, or enough K partitions to give every SM two
  // tiles.  A caller's split-K (> 1) whose grid would leave SMs short of two
  // CTAs is widened to fill them: the partials meet in atomic adds either way,
  // so only the (unordered) summation grouping changes.
  int sp = splits;
  const int64_t tiles_mn = mt * nt * batch;
  if (sp <= 0 || (sp > 1 && tiles_mn * sp < 2 * sms)) {
    const int want = sp;
    sp = 1;
    if (!accumulate && tiles_mn < 2 * sms) {
      sp = (int)((2 * sms + tiles_mn - 1) / tiles_mn);
      const int64_t kt = (K + BK - 1) / BK;
      if (sp > kt) sp = (int)(kt > 0 ? kt : 1);
      if (sp > 256) sp = 256;
    }
    if (sp < want) sp = want;
  }
  int64_t kps = (K + sp - 1) / sp;
  kps = (kps + BK - 1) / BK * BK;
  if (kps == 0) kps = BK;
  sp = (int)((K + kps - 1) / kps);
  if (sp < 1) sp = 1;
  const int mode = peers ? GEMM_PEER
                         : (sp > 1 ? GEMM_ATOMIC : (accumulate ? GEMM_ACCUMULATE : GEMM_STORE));
  const PeerRows pr = peers ? *peers : PeerRows{};
  if (batch > 1 && c_batch_stride < M * N)
    return set_error(EMMY_ERR_INVALID, "%s: batch stride of C overlaps its batches", name);
  if (mode == GEMM_ATOMIC && !accumulate) {
    const size_t elems = (size_t)((batch - 1) * c_batch_stride + M * N);
    cudaError_t e = cudaMemsetAsync(C, 0, elems * sizeof(T), st);
    if (e != cudaSuccess) return set_error(EMMY_ERR_CUDA, "%s: %s", name, cudaGetErrorString(e));
  }
  if ((int64_t)batch * sp > 65535)
    return set_error(EMMY_ERR_UNSUPPORTED, "%s: batch x splits beyond the grid limit", name);

  const bool tma_ok = K % VEC == 0 && N % 4 == 0 && aligned16(A) && aligned16(B) &&
                      aligned16(C) && (a_batch_stride * ES) % 16 == 0 &&
                      (b_batch_stride * ES) % 16 == 0 && (c_batch_stride % 4) == 0 && K > 0;
  const CUtensorMapDataType tdt =
      ES == 4 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_FLOAT64;
  if (tma_ok) {
    CUtensorMap ta, tb;
    const uint64_t adims[3] = {(uint64_t)K, (uint64_t)M, (uint64_t)batch};
    const uint64_t astr[2] = {(uint64_t)K * ES, (uint64_t)(batch > 1 ? a_batch_stride : M * K) * ES};
    const uint32_t abox[3] = {BK, BM, 1};
    const uint64_t bdims[3] = {(uint64_t)N, (uint64_t)K, (uint64_t)batch};
    const uint64_t bstr[2] = {(uint64_t)N * ES, (uint64_t)(batch > 1 ? b_batch_stride : K * N) * ES};
    const uint32_t bbox[3] = {BN, BK, 1};
    int rc = make_tensor_map(&ta, tdt, 3, A, adims, astr, abox,
                             CU_TENSOR_MAP_SWIZZLE_NONE);
    if (rc) return rc;
    rc = make_tensor_map(&tb, tdt, 3, B, bdims, bstr, bbox,
                         CU_TENSOR_MAP_SWIZZLE_NONE);
    if (rc) return rc;
    static bool attr_set[64] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && !attr_set[dev]) {
      cudaFuncSetAttribute(gemm_simt_tma_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           SMEM_BYTES);
      attr_set[dev] = true;
    }
    dim3 grid((unsigned)mt, (unsigned)nt, (unsigned)(batch * sp));
    gemm_simt_tma_kernel<T><<<grid, THREADS, SMEM_BYTES, st>>>(
        ta, tb, bias, C, (int)M, (int)N, (int)K, c_batch_stride, sp, (int)kps, epilogue, mode,
        pr, device_status_ptr());
    return check_launch(name);
  }
  if (peers && sp > 1) {
    // the plain kernel stores partial rows without a tile reduction: one split
    sp = 1;
    kps = K;
  }
  dim3 grid((unsigned)((M + 63) / 64), (unsigned)((N + 63) / 64), (unsigned)(batch * sp));
  gemm_simt_plain_kernel<T><<<grid, 256, 0, st>>>(A, B, bias, C, (int)M, (int)N, (int)K,
                                                  a_batch_stride, b_batch_stride, c_batch_stride,
                                                  sp, (int)kps, epilogue, mode, pr);
  return check_launch(name);
}

extern "C" int emmy_gemm_f32(const float *A, const float *B, const float *bias, float *C,
                             int64_t batch, int64_t M, int64_t N, int64_t K, int64_t a_batch_stride,
                             int64_t b_batch_stride, int64_t c_batch_stride, int splits,
                             int accumulate, int epilogue, void *stream) {
  return gemm_simt<float>("emmy_gemm_f32", A, B, bias, C, batch, M, N, K, a_batch_stride,
                          b_batch_stride, c_batch_stride, splits, accumulate, epilogue, stream);
}

extern "C" int emmy_gemm_f64(const double *A, const double *B, const double *bias, double *C,
                             int64_t batch, int64_t M, int64_t N, int64_t K, int64_t a_batch_stride,
                             int64_t b_batch_stride, int64_t c_batch_stride, int splits,
                             int accumulate, int epilogue, void *stream) {
  return gemm_simt<double>("emmy_gemm_f64", A, B, bias, C, batch, M, N, K, a_batch_stride,
                           b_batch_stride, c_batch_stride, splits, accumulate, epilogue, stream);
}


extern "C" int emmy_gemm_f32_rows_to_peers(const float *A, const float *B, const float *bias,
                                           float *const *rows, int64_t slot_floats, int world,
                                           int me, int64_t rows_per_rank, int64_t M, int64_t N,
                                           int64_t K, int splits, float *workspace,
                                           int *tile_counters, int64_t n_counters, void *stream) {
  clear_error();
  if (world < 1 || world > 8 || !rows || me < 0 || me >= world)
    return set_error(EMMY_ERR_INVALID, "emmy_gemm_f32_rows_to_peers: 1 to 8 row owners");
  if (rows_per_rank < 1 || rows_per_rank * world < M)
    return set_error(EMMY_ERR_INVALID, "emmy_gemm_f32_rows_to_peers: rows do not cover M");
  if (N < 0 || slot_floats < (int64_t)world * rows_per_rank * N)
    return set_error(EMMY_ERR_INVALID,
                     "emmy_gemm_f32_rows_to_peers: slot buffers of %lld floats, need world x "
                     "rows_per_rank x N = %lld", (long long)slot_floats,
                     (long long)world * rows_per_rank * N);
  if (!workspace || !tile_counters || n_counters < ((M + 63) / 64) * ((N + 63) / 64))
    return set_error(EMMY_ERR_INVALID, "emmy_gemm_f32_rows_to_peers: workspace or counters");
  PeerRows pr{};
  pr.rows_per_rank = rows_per_rank;
  pr.ws = workspace;
  pr.counters = tile_counters;
  pr.me = me;
  for (int r = 0; r < world; ++r) {
    if (!rows[r] && r * rows_per_rank < M)
      return set_error(EMMY_ERR_INVALID, "emmy_gemm_f32_rows_to_peers: null rows of owner %d", r);
    pr.rows[r] = rows[r];
  }
  return gemm_simt<float>("emmy_gemm_f32_rows_to_peers", A, B, bias, rows[0], 1, M, N, K, M * K,
                          K * N, M * N, splits, 0, bias ? EMMY_EPI_BIAS : 0, stream, &pr);
}