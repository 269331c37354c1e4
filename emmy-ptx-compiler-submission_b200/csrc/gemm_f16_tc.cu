// f16 GEMM / batched GEMM with f32 accumulation on the sm_100a tensor cores
// (tcgen05.mma, accumulator in tensor memory), with a fused bias + ReLU
// epilogue and f16 or f32 output.
//
// Replaces the entry the reference would emit for its tiled-matmul IR shape
// with f16 operands: the same cp.async staging and register micro-tile walk as
// the f32 fixtures, each f16 load widened to f32 for an fma.rn chain
// (reference ptxc/expr.py:168-180, ptxc/stmts.py:614-632, 663-725), followed by
// the epilogue Assigns and the converting Write (ptxc/stmts.py:434-487).
//
// Here: a persistent kernel, one CTA per SM, walking 128 x 256 output tiles.
//   warp 0      TMA producer: A [128 x 64] K-major and B [64 x 256] N-major
//               (row-major B as stored) into a 4-stage ring of 128-byte
//               swizzled shared memory (no multicast)
//   warp 1      one thread issues tcgen05.mma (M128 N256 K16), four per stage,
//               into one of two 256-column f32 TMEM accumulators, and commits
//               each stage back to the producer and each finished tile to the
//               epilogue
//   warps 2-5   epilogue: each warp drains its 32 TMEM lanes (one output row
//               per thread), adds the bias, applies ReLU, converts and stores,
//               then hands the accumulator back -- while the MMA warp already
//               fills the other accumulator with the next tile.
// Tiles are visited M-fastest within groups of 16 N-tiles, so concurrently
// running CTAs share B column panels in L2.  All mbarrier waits are bounded.

#include "common.cuh"
#include "tcgen05.cuh"

namespace emmy {

namespace gemm16 {
constexpr int BM = 128, BN = 256, BK = 64, STAGES = 4, THREADS = 192;
constexpr int A_BYTES = BM * BK * 2;                 // 16 KB
constexpr int B_BOX_BYTES = BK * 64 * 2;             // 8 KB: 64 k-rows x 64 n (128 B)
constexpr int B_BYTES = BK * BN * 2;                 // 32 KB
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024;
constexpr uint32_t TMEM_COLS = 512;                  // two 256-column accumulators
constexpr int GROUP_N = 16;                          // raster group width in N tiles
constexpr int kStatusGemmTimeout = 0x1101;
}  // namespace gemm16

struct TileCoord {
  int m0, n0, b;
};

// Tile t of (batch, mt, nt) tiles: batches outermost, then groups of GROUP_N
// N-tiles; inside a group M varies fastest.
__device__ __forceinline__ TileCoord gemm16_tile(int t, int mt, int nt) {
  using namespace gemm16;
  const int per_batch = mt * nt;
  const int b = t / per_batch;
  int r = t - b * per_batch;
  const int group = r / (mt * GROUP_N);
  const int first_n = group * GROUP_N;
  r -= group * mt * GROUP_N;
  const int m = r % mt;
  const int n = first_n + r / mt;
  return {m * BM, n * BN, b};
}

// One thread's accumulator row (its TMEM lane, 256 columns from `base`):
// bias, ReLU, convert, store.  tcgen05.ld is warp-collective, so every lane
// runs every chunk and only the stores are masked.
__device__ __forceinline__ void gemm16_drain_row(uint32_t base, int row, TileCoord tc, int M,
                                                 int N, int ktiles, const float *__restrict__ bias,
                                                 bool add_bias, bool relu, bool round16,
                                                 int out_f16, void *__restrict__ C,
                                                 int64_t c_batch_stride) {
#pragma unroll 1
  for (int c = 0; c < 256 / 32; ++c) {
    float v[32];
    __syncwarp();   // reconverge after the masked stores of the previous chunk
    tmem_ld32(base + c * 32, v);
    const int n = tc.n0 + c * 32;
    if (row >= M || n >= N) continue;
    if (ktiles == 0) {
#pragma unroll
      for (int k = 0; k < 32; ++k) v[k] = 0.f;
    }
    if (round16) {
#pragma unroll
      for (int k = 0; k < 32; ++k) v[k] = __half2float(__float2half_rn(v[k]));
    }
    if (add_bias) {
#pragma unroll
      for (int k = 0; k < 32; ++k) v[k] += (n + k < N) ? __ldg(bias + n + k) : 0.f;
    }
    if (relu) {
#pragma unroll
      for (int k = 0; k < 32; ++k) v[k] = fmaxf(v[k], 0.f);
    }
    const int64_t off = (int64_t)tc.b * c_batch_stride + (int64_t)row * N + n;
    if (out_f16) {
      __half *dst = reinterpret_cast<__half *>(C) + off;
      if (n + 32 <= N) {
#pragma unroll
        for (int p = 0; p < 4; ++p) {
          uint32_t w[4];
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            __half2 hh = __floats2half2_rn(v[8 * p + 2 * k], v[8 * p + 2 * k + 1]);
            w[k] = *reinterpret_cast<uint32_t *>(&hh);
          }
          *reinterpret_cast<uint4 *>(dst + 8 * p) = make_uint4(w[0], w[1], w[2], w[3]);
        }
      } else {
        for (int k = 0; k < 32 && n + k < N; ++k) dst[k] = __float2half_rn(v[k]);
      }
    } else {
      float *dst = reinterpret_cast<float *>(C) + off;
      if (n + 32 <= N) {
#pragma unroll
        for (int p = 0; p < 8; ++p)
          *reinterpret_cast<float4 *>(dst + 4 * p) =
              make_float4(v[4 * p], v[4 * p + 1], v[4 * p + 2], v[4 * p + 3]);
      } else {
        for (int k = 0; k < 32 && n + k < N; ++k) dst[k] = v[k];
      }
    }
  }
}

__global__ void __launch_bounds__(gemm16::THREADS, 1)
gemm_f16_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const float *__restrict__ bias, void *__restrict__ C, int M, int N, int K,
                   int batch, int64_t c_batch_stride, int out_f16, int epilogue, int *status) {
  using namespace gemm16;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char *smem = reinterpret_cast<unsigned char *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ __align__(8) uint64_t full[STAGES];
  __shared__ __align__(8) uint64_t empty[STAGES];
  __shared__ __align__(8) uint64_t acc_full[2];
  __shared__ __align__(8) uint64_t acc_empty[2];
  __shared__ uint32_t tmem_holder;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int mt = (M + BM - 1) / BM, nt = (N + BN - 1) / BN;
  const int tiles = mt * nt * batch;
  const int ktiles = (K + BK - 1) / BK;

  if (threadIdx.x == 0) {
    prefetch_tensormap(&tmA);
    prefetch_tensormap(&tmB);
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], 4);      // one arrival per epilogue warp
    }
    fence_barrier_init();
  }
  if (warp == 0) tmem_alloc(&tmem_holder, TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_holder;

  if (warp == 0) {
    if (lane == 0) {
      // TMA producer: one continuous stage sequence across all of this CTA's tiles
      int g = 0;
      bool ok = true;
      for (int t = blockIdx.x; ok && t < tiles; t += gridDim.x) {
        const TileCoord tc = gemm16_tile(t, mt, nt);
        for (int kt = 0; kt < ktiles; ++kt, ++g) {
          const int s = g % STAGES;
          if (g >= STAGES &&
              !mbar_wait(&empty[s], ((g / STAGES) - 1) & 1, status, kStatusGemmTimeout)) {
            ok = false;
            break;
          }
          unsigned char *sa = smem + s * STAGE_BYTES;
          unsigned char *sb = sa + A_BYTES;
          mbar_expect_tx(&full[s], STAGE_BYTES);
          tma_load_3d(sa, &tmA, &full[s], kt * BK, tc.m0, tc.b);
#pragma unroll
          for (int j = 0; j < BN / 64; ++j)
            tma_load_3d(sb + j * B_BOX_BYTES, &tmB, &full[s], tc.n0 + 64 * j, kt * BK, tc.b);
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) {
      // MMA issuer
      constexpr uint32_t idesc = f16_idesc(BM, BN, false, true);
      int g = 0, i = 0;
      bool ok = true;
      for (int t = blockIdx.x; ok && t < tiles; t += gridDim.x, ++i) {
        const int a = i & 1;
        if (i >= 2 && !mbar_wait(&acc_empty[a], ((i >> 1) - 1) & 1, status, kStatusGemmTimeout))
          break;
        tc_fence_after();
        const uint32_t acc = tmem + a * BN;
        // This thread runs only about one MMA ahead of the tensor core, and a
        // barrier wait between MMAs leaves the pipe empty for ~200 cycles, so
        // stages are taken two at a time: both waits, then eight MMAs back to
        // back (each stage is still released as soon as its own four are done).
        // Shared-memory operands written by TMA need no tcgen05 fence after
        // their barrier.
        for (int kt = 0; kt < ktiles; kt += 2) {
          const int n2 = kt + 1 < ktiles ? 2 : 1;
          for (int h = 0; h < n2; ++h)
            if (!mbar_wait(&full[(g + h) % STAGES], ((g + h) / STAGES) & 1, status,
                           kStatusGemmTimeout)) {
              ok = false;
              break;
            }
          if (!ok) break;
          for (int h = 0; h < n2; ++h, ++g) {
            const int s = g % STAGES;
            const uint32_t sa = smem_u32(smem + s * STAGE_BYTES);
            const uint32_t sb = sa + A_BYTES;
            // A: K-major, 128-byte rows, 8-row atoms 1024 B apart; a K16 step is 32 B
            const uint64_t da = sw128_desc(sa, 16, 1024);
            // B: N-major, 64-wide n atoms 8 KB apart, 8-row k atoms 1024 B apart; K16 = 2048 B
            const uint64_t db = sw128_desc(sb, B_BOX_BYTES, 1024);
#pragma unroll
            for (int kk = 0; kk < BK / 16; ++kk)
              mma_f16(acc, da + ((kk * 32) >> 4), db + ((kk * 2048) >> 4), idesc,
                      (kt + h > 0 || kk > 0) ? 1u : 0u);
            mma_commit(&empty[s]);
          }
        }
        if (!ok) break;
        mma_commit(&acc_full[a]);
      }
    }
    __syncwarp();
  } else {
    // epilogue warps 2..5: warp w reads TMEM lanes [32*(w%4), +32)
    const int q = warp & 3;
    const uint32_t lane_off = (uint32_t)(q * 32) << 16;
    const bool relu = epilogue & EMMY_EPI_RELU;
    const bool round16 = epilogue & EMMY_EPI_ROUND_F16;
    const bool add_bias = (epilogue & EMMY_EPI_BIAS) && bias != nullptr;
    int i = 0;
    for (int t = blockIdx.x; t < tiles; t += gridDim.x, ++i) {
      const int a = i & 1;
      const TileCoord tc = gemm16_tile(t, mt, nt);
      if (!mbar_wait(&acc_full[a], (i >> 1) & 1, status, kStatusGemmTimeout)) break;
      __syncwarp();
      tc_fence_after();
      gemm16_drain_row(tmem + lane_off + a * BN, tc.m0 + q * 32 + lane, tc, M, N, ktiles,
                       bias, add_bias, relu, round16, out_f16, C, c_batch_stride);
      // the accumulator's TMEM reads are complete (tcgen05.wait::ld in tmem_ld32)
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[a]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, TMEM_COLS);
}

// ---------------------------------------------------------------------------
// CTA-pair variant (tcgen05.mma.cta_group::2): the two CTAs of a cluster own a
// 256 x 256 output tile.  Each CTA stages its own 128 rows of A and its own
// 128 columns of B; one thread of CTA 0 issues M256 N256 K16 MMAs that read
// both CTAs' operands, and each CTA's tensor memory receives its 128 rows of
// the accumulator.  Per SM this halves the shared-memory operand traffic of
// the 128 x 256 single-CTA tile (which is shared-memory-bandwidth bound), and
// each CTA loads half of B.
//   warp 0 (both CTAs)   TMA producer for its own halves; transaction bytes
//                        are counted on CTA 0's stage barrier (no multicast)
//   warp 1 (CTA 0)       MMA issuer; stage and accumulator releases are
//                        committed to the barrier in each CTA
//   warps 2-5 (both)     epilogue of the CTA's 128 rows; the accumulator is
//                        handed back on CTA 0's barrier (8 arrivals)

namespace gemm16p {
constexpr int BM = 256, BMH = 128, BN = 256, BNH = 128, BK = 64, THREADS = 192;
constexpr int A_BYTES = BMH * BK * 2;                // 16 KB: this CTA's rows
constexpr int B_BOX_BYTES = BK * 64 * 2;             // 8 KB
constexpr int B_BYTES = BK * BNH * 2;                // 16 KB: this CTA's columns of one N half
constexpr int OUT_BOX_BYTES = 32 * 128;              // one warp's 32 rows x 128 B of C
constexpr int OUT_BYTES = 4 * 2 * OUT_BOX_BYTES;     // 4 epilogue warps, double-buffered
constexpr uint32_t TMEM_COLS = 512;
constexpr int kStatusGemmTimeout = 0x1102;
// NH: 256-column N halves per tile.  NH = 1: 256 x 256 tiles, two 256-column
// accumulators (the epilogue of one tile overlaps the next tile's products).
// NH = 2: 256 x 512 tiles, one 512-column accumulator; each stage carries the
// CTA's A rows once for two N = 256 products, so 24 KB of operands per
// product reach shared memory instead of 32 KB.
template <int NH>
struct PairCfg {
  static constexpr int TBN = BN * NH;                          // tile columns
  static constexpr int STAGE_BYTES = A_BYTES + NH * B_BYTES;
  static constexpr int STAGES = NH == 1 ? 6 : 4;
  static constexpr int NACC = 2 / NH;                          // accumulators
  static constexpr int ACC_COLS = BN * NH;
  static constexpr int GROUP_N = 8 / NH;                       // raster group width in tiles
  static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + OUT_BYTES + 1024;
  static_assert(NACC * ACC_COLS <= (int)TMEM_COLS, "tensor memory");
  static_assert(SMEM_BYTES <= 227 * 1024, "shared memory");
};
}  // namespace gemm16p

template <int NH>
__device__ __forceinline__ TileCoord gemm16p_tile(int t, int mt, int nt) {
  using namespace gemm16p;
  constexpr int GROUP_N = PairCfg<NH>::GROUP_N, BN = PairCfg<NH>::TBN;
  const int per_batch = mt * nt;
  const int b = t / per_batch;
  int r = t - b * per_batch;
  const int group = r / (mt * GROUP_N);
  const int first_n = group * GROUP_N;
  r -= group * mt * GROUP_N;
  const int m = r % mt;
  const int n = first_n + r / mt;
  return {m * BM, n * BN, b};
}

// One epilogue warp's 32 accumulator rows (TMEM lanes), ncols columns: bias,
// ReLU, convert, then stage 128-byte row pieces (64 f16 or 32 f32 columns) in
// shared memory with the 128-byte swizzle and write each 32-row box with one
// TMA store.  Coalesced writes, and TMA drops rows and columns outside C.
// Two staging buffers per warp: a buffer is refilled once the store issued
// from it two chunks earlier has finished reading it.
__device__ __forceinline__ void gemm16_drain_warp_tma(uint32_t tbase, int ncols, int lane, int row0,
                                                      TileCoord tc, int N,
                                                      const float *__restrict__ bias,
                                                      bool add_bias, bool relu, bool round16,
                                                      int out_f16, const CUtensorMap *tmC,
                                                      unsigned char *stage, int &seq) {
  const int step = out_f16 ? 64 : 32;                // columns per 128-byte row piece
#pragma unroll 1
  for (int c0 = 0; c0 < ncols; c0 += step, ++seq) {
    unsigned char *buf = stage + (seq & 1) * gemm16p::OUT_BOX_BYTES;
    if (seq >= 2 && lane == 0) bulk_wait_group_read<1>();
    __syncwarp();
    const int n = tc.n0 + c0;
    uint4 w[8];
    if (out_f16) {
      float v[64];
      tmem_ld64(tbase + c0, v);
      if (round16) {
#pragma unroll
        for (int k = 0; k < 64; ++k) v[k] = __half2float(__float2half_rn(v[k]));
      }
      if (add_bias) {
#pragma unroll
        for (int k = 0; k < 64; ++k) v[k] += (n + k < N) ? __ldg(bias + n + k) : 0.f;
      }
      if (relu) {
#pragma unroll
        for (int k = 0; k < 64; ++k) v[k] = fmaxf(v[k], 0.f);
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        uint32_t h[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          __half2 hh = __floats2half2_rn(v[8 * j + 2 * k], v[8 * j + 2 * k + 1]);
          h[k] = *reinterpret_cast<uint32_t *>(&hh);
        }
        w[j] = make_uint4(h[0], h[1], h[2], h[3]);
      }
    } else {
      float v[32];
      tmem_ld32(tbase + c0, v);
      if (round16) {
#pragma unroll
        for (int k = 0; k < 32; ++k) v[k] = __half2float(__float2half_rn(v[k]));
      }
      if (add_bias) {
#pragma unroll
        for (int k = 0; k < 32; ++k) v[k] += (n + k < N) ? __ldg(bias + n + k) : 0.f;
      }
      if (relu) {
#pragma unroll
        for (int k = 0; k < 32; ++k) v[k] = fmaxf(v[k], 0.f);
      }
#pragma unroll
      for (int j = 0; j < 8; ++j)
        w[j] = make_uint4(__float_as_uint(v[4 * j]), __float_as_uint(v[4 * j + 1]),
                          __float_as_uint(v[4 * j + 2]), __float_as_uint(v[4 * j + 3]));
    }
    // row `lane` of the box: 16-byte piece j at (j ^ (lane % 8)) * 16
#pragma unroll
    for (int j = 0; j < 8; ++j)
      *reinterpret_cast<uint4 *>(buf + lane * 128 + ((j ^ (lane & 7)) * 16)) = w[j];
    fence_proxy_async();                             // visible to the TMA (async proxy)
    __syncwarp();
    if (lane == 0) {
      tma_store_3d(tmC, buf, n, row0, tc.b);
      bulk_commit_group();
    }
  }
}

template <int NH>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(gemm16p::THREADS, 1)
gemm_f16_pair_kernel(const __grid_constant__ CUtensorMap tmA,
                     const __grid_constant__ CUtensorMap tmB,
                     const __grid_constant__ CUtensorMap tmC, const float *__restrict__ bias,
                     void *__restrict__ C, int M, int N, int K, int batch, int64_t c_batch_stride,
                     int out_f16, int epilogue, int *status) {
  using namespace gemm16p;
  using P = PairCfg<NH>;
  constexpr int STAGES = P::STAGES, STAGE_BYTES = P::STAGE_BYTES, NACC = P::NACC;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char *smem = reinterpret_cast<unsigned char *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ __align__(8) uint64_t full[STAGES];
  __shared__ __align__(8) uint64_t empty[STAGES];
  __shared__ __align__(8) uint64_t acc_full[NACC];
  __shared__ __align__(8) uint64_t acc_empty[NACC];
  __shared__ __align__(8) uint64_t mma_done;
  __shared__ uint32_t tmem_holder;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const int cluster = blockIdx.x >> 1, nclusters = gridDim.x >> 1;
  const int mt = (M + BM - 1) / BM, nt = (N + P::TBN - 1) / P::TBN;
  const int tiles = mt * nt * batch;
  const int ktiles = (K + BK - 1) / BK;

  if (threadIdx.x == 0) {
    prefetch_tensormap(&tmA);
    prefetch_tensormap(&tmB);
    prefetch_tensormap(&tmC);
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < NACC; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], 8);      // four epilogue warps in each CTA
    }
    mbar_init(&mma_done, 1);
    fence_barrier_init();
  }
  if (warp == 0) tmem_alloc_pair(&tmem_holder, TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  cluster_sync();       // both CTAs' barriers exist before any remote arrive
  tc_fence_after();
  const uint32_t tmem = tmem_holder;

  if (warp == 0) {
    if (lane == 0) {
      int g = 0;
      bool ok = true;
      for (int t = cluster; ok && t < tiles; t += nclusters) {
        const TileCoord tc = gemm16p_tile<NH>(t, mt, nt);
        for (int kt = 0; kt < ktiles; ++kt, ++g) {
          const int s = g % STAGES;
          if (g >= STAGES &&
              !mbar_wait(&empty[s], ((g / STAGES) - 1) & 1, status, kStatusGemmTimeout)) {
            ok = false;
            break;
          }
          unsigned char *sa = smem + s * STAGE_BYTES;
          unsigned char *sb = sa + A_BYTES;
          if (rank == 0) mbar_expect_tx(&full[s], 2 * STAGE_BYTES);
          const uint32_t leader_full = mapa_shared(smem_u32(&full[s]), 0);
          tma_load_3d_pair(sa, &tmA, leader_full, kt * BK, tc.m0 + BMH * (int)rank, tc.b);
          // per N half h: this CTA's 128 columns, as two 64-column boxes
#pragma unroll
          for (int h = 0; h < NH; ++h)
#pragma unroll
            for (int j = 0; j < BNH / 64; ++j)
              tma_load_3d_pair(sb + h * B_BYTES + j * B_BOX_BYTES, &tmB, leader_full,
                               tc.n0 + BN * h + BNH * (int)rank + 64 * j, kt * BK, tc.b);
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0 && rank == 0) {
      constexpr uint32_t idesc = f16_idesc(BM, BN, false, true);
      int g = 0, i = 0;
      bool ok = true;
      for (int t = cluster; ok && t < tiles; t += nclusters, ++i) {
        const int a = i % NACC;
        if (i >= NACC &&
            !mbar_wait(&acc_empty[a], ((i / NACC) - 1) & 1, status, kStatusGemmTimeout))
          break;
        tc_fence_after();
        const uint32_t acc = tmem + a * P::ACC_COLS;
        // two stages per barrier wait, then eight MMAs back to back; each stage
        // is released to both CTAs' producers as soon as its own four are done
        for (int kt = 0; kt < ktiles; kt += 2) {
          const int n2 = kt + 1 < ktiles ? 2 : 1;
          for (int h = 0; h < n2; ++h)
            if (!mbar_wait(&full[(g + h) % STAGES], ((g + h) / STAGES) & 1, status,
                           kStatusGemmTimeout)) {
              ok = false;
              break;
            }
          if (!ok) break;
          for (int h = 0; h < n2; ++h, ++g) {
            const int s = g % STAGES;
            const uint32_t sa = smem_u32(smem + s * STAGE_BYTES);
            const uint64_t da = sw128_desc(sa, 16, 1024);
#pragma unroll
            for (int kk = 0; kk < BK / 16; ++kk)
#pragma unroll
              for (int nh = 0; nh < NH; ++nh)
                mma_f16_pair(acc + nh * BN, da + ((kk * 32) >> 4),
                             sw128_desc(sa + A_BYTES + nh * B_BYTES, B_BOX_BYTES, 1024) +
                                 ((kk * 2048) >> 4),
                             idesc, (kt + h > 0 || kk > 0) ? 1u : 0u);
            mma_commit_pair(smem_u32(&empty[s]));
            mma_commit_pair(mapa_shared(smem_u32(&empty[s]), 1));
          }
        }
        if (!ok) break;
        mma_commit_pair(smem_u32(&acc_full[a]));
        mma_commit_pair(mapa_shared(smem_u32(&acc_full[a]), 1));
      }
      // every MMA issued has finished before the pair's tensor memory is freed
      mma_commit_pair(smem_u32(&mma_done));
      mbar_wait(&mma_done, 0, status, kStatusGemmTimeout);
    }
    __syncwarp();
  } else {
    const int q = warp & 3;
    const uint32_t lane_off = (uint32_t)(q * 32) << 16;
    const bool relu = epilogue & EMMY_EPI_RELU;
    const bool round16 = epilogue & EMMY_EPI_ROUND_F16;
    const bool add_bias = (epilogue & EMMY_EPI_BIAS) && bias != nullptr;
    unsigned char *stage = smem + STAGES * STAGE_BYTES + q * 2 * OUT_BOX_BYTES;
    int i = 0, seq = 0;
    for (int t = cluster; t < tiles; t += nclusters, ++i) {
      const int a = i % NACC;
      const TileCoord tc = gemm16p_tile<NH>(t, mt, nt);
      if (!mbar_wait(&acc_full[a], (i / NACC) & 1, status, kStatusGemmTimeout)) break;
      __syncwarp();
      tc_fence_after();
      gemm16_drain_warp_tma(tmem + lane_off + a * P::ACC_COLS, P::ACC_COLS, lane,
                            tc.m0 + BMH * (int)rank + q * 32, tc, N, bias, add_bias, relu,
                            round16, out_f16, &tmC, stage, seq);
      // the accumulator's TMEM reads are complete (tcgen05.wait::ld)
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if (rank == 0) mbar_arrive(&acc_empty[a]);
        else mbar_arrive_cluster(mapa_shared(smem_u32(&acc_empty[a]), 0));
      }
    }
    if (lane == 0) bulk_wait_group<0>();             // this warp's stores have landed
    __syncwarp();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();       // the peer is done with the pair's TMEM and barriers
  if (warp == 0) tmem_dealloc_pair(tmem, TMEM_COLS);
}

// CUDA-core fallback for shapes the TMA descriptors cannot take (K or N not a
// multiple of 8, unaligned bases): f16 loads widened to f32, fma accumulate.
__global__ void __launch_bounds__(256)
gemm_f16_plain_kernel(const __half *__restrict__ A, const __half *__restrict__ B,
                      const float *__restrict__ bias, void *__restrict__ C, int M, int N, int K,
                      int64_t sa, int64_t sb, int64_t sc, int out_f16, int epilogue) {
  __shared__ float As[16][64 + 1];
  __shared__ float Bs[16][64 + 1];
  const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
  const int m0 = blockIdx.x * 64, n0 = blockIdx.y * 64, b = blockIdx.z;
  const __half *Ab = A + (int64_t)b * sa;
  const __half *Bb = B + (int64_t)b * sb;
  float acc[4][4] = {};
  for (int k0 = 0; k0 < K; k0 += 16) {
    for (int i = tid; i < 16 * 64; i += 256) {
      const int r = i / 16, c = i % 16;
      As[c][r] = (m0 + r < M && k0 + c < K) ? __half2float(Ab[(int64_t)(m0 + r) * K + k0 + c]) : 0.f;
      const int kr = i / 64, nc = i % 64;
      Bs[kr][nc] = (k0 + kr < K && n0 + nc < N) ? __half2float(Bb[(int64_t)(k0 + kr) * N + n0 + nc]) : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int k = 0; k < 16; ++k)
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(As[k][ty + 16 * i], Bs[k][tx + 16 * j], acc[i][j]);
    __syncthreads();
  }
  for (int i = 0; i < 4; ++i) {
    const int m = m0 + ty + 16 * i;
    if (m >= M) continue;
    for (int j = 0; j < 4; ++j) {
      const int n = n0 + tx + 16 * j;
      if (n >= N) continue;
      float v = acc[i][j];
      if (epilogue & EMMY_EPI_ROUND_F16) v = __half2float(__float2half_rn(v));
      if ((epilogue & EMMY_EPI_BIAS) && bias) v += bias[n];
      if (epilogue & EMMY_EPI_RELU) v = fmaxf(v, 0.f);
      const int64_t off = (int64_t)b * sc + (int64_t)m * N + n;
      if (out_f16) reinterpret_cast<__half *>(C)[off] = __float2half_rn(v);
      else reinterpret_cast<float *>(C)[off] = v;
    }
  }
}

}  // namespace emmy

using namespace emmy;

namespace {

// One launch of the CTA-pair kernel: one cluster of two CTAs per two SMs,
// persistent over the tiles; C written by TMA stores of 32-row x 128-byte boxes.
template <int NH>
int launch_gemm16_pair(const CUtensorMap &ta, const CUtensorMap &tb, const float *bias, void *C,
                       int64_t M, int64_t N, int64_t K, int64_t batch, int out_f16, int epilogue,
                       cudaStream_t st) {
  using P = gemm16p::PairCfg<NH>;
  static bool attr_set[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr_set[dev]) {
    cudaFuncSetAttribute(gemm_f16_pair_kernel<NH>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         P::SMEM_BYTES);
    attr_set[dev] = true;
  }
  const int64_t ptiles = ((M + gemm16p::BM - 1) / gemm16p::BM) * ((N + P::TBN - 1) / P::TBN) * batch;
  const int64_t pairs = sm_count() / 2;
  const int clusters = (int)(ptiles < pairs ? ptiles : pairs);
  const uint64_t esize = out_f16 ? 2 : 4;
  CUtensorMap tc_map;
  const uint64_t cdims[3] = {(uint64_t)N, (uint64_t)M, (uint64_t)batch};
  const uint64_t cstr[2] = {(uint64_t)N * esize, (uint64_t)M * N * esize};
  const uint32_t cbox[3] = {(uint32_t)(128 / esize), 32, 1};
  const int rc = make_tensor_map(&tc_map, out_f16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                                  : CU_TENSOR_MAP_DATA_TYPE_FLOAT32,
                                 3, C, cdims, cstr, cbox, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  gemm_f16_pair_kernel<NH><<<2 * clusters, gemm16p::THREADS, P::SMEM_BYTES, st>>>(
      ta, tb, tc_map, bias, C, (int)M, (int)N, (int)K, (int)batch, M * N, out_f16, epilogue,
      device_status_ptr());
  return check_launch("emmy_gemm_f16 (tcgen05 pair)");
}

}  // namespace

extern "C" int emmy_gemm_f16(const void *A, const void *B, const float *bias, void *C,
                             int64_t batch, int64_t M, int64_t N, int64_t K, int out_dtype,
                             int epilogue, int accumulate, void *stream) {
  using namespace gemm16;
  clear_error();
  if (batch < 0 || M < 0 || N < 0 || K < 0)
    return set_error(EMMY_ERR_INVALID, "emmy_gemm_f16: negative size");
  if (batch == 0 || M == 0 || N == 0) return EMMY_OK;
  if (!A || !B || !C) return set_error(EMMY_ERR_INVALID, "emmy_gemm_f16: null operand");
  if (out_dtype != EMMY_DT_F32 && out_dtype != EMMY_DT_F16)
    return set_error(EMMY_ERR_INVALID, "emmy_gemm_f16: bad output dtype %d", out_dtype);
  if (accumulate)
    return set_error(EMMY_ERR_UNSUPPORTED, "emmy_gemm_f16: accumulating into C is not supported");
  if (epilogue & ~(EMMY_EPI_BIAS | EMMY_EPI_RELU | EMMY_EPI_ROUND_F16))
    return set_error(EMMY_ERR_INVALID, "emmy_gemm_f16: unknown epilogue bits %d", epilogue);
  if (M > INT32_MAX || N > INT32_MAX || K > INT32_MAX || batch > 65535)
    return set_error(EMMY_ERR_UNSUPPORTED, "emmy_gemm_f16: size beyond 32-bit tile indexing");
  cudaStream_t st = as_stream(stream);
  const int out_f16 = out_dtype == EMMY_DT_F16;
  const bool tma_ok = K % 8 == 0 && N % 8 == 0 && K > 0 && aligned16(A) && aligned16(B) &&
                      aligned16(C);
  if (tma_ok) {
    const int64_t tiles = ((M + BM - 1) / BM) * ((N + BN - 1) / BN) * batch;
    if (tiles > INT32_MAX) return set_error(EMMY_ERR_UNSUPPORTED, "emmy_gemm_f16: too many tiles");
    CUtensorMap ta, tb;
    const uint64_t adims[3] = {(uint64_t)K, (uint64_t)M, (uint64_t)batch};
    const uint64_t astr[2] = {(uint64_t)K * 2, (uint64_t)M * K * 2};
    const uint32_t abox[3] = {BK, BM, 1};
    const uint64_t bdims[3] = {(uint64_t)N, (uint64_t)K, (uint64_t)batch};
    const uint64_t bstr[2] = {(uint64_t)N * 2, (uint64_t)K * N * 2};
    const uint32_t bbox[3] = {64, BK, 1};
    int rc = make_tensor_map(&ta, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, A, adims, astr, abox,
                             CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
    rc = make_tensor_map(&tb, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, B, bdims, bstr, bbox,
                         CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
    static bool attr_set[64] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && !attr_set[dev]) {
      cudaFuncSetAttribute(gemm_f16_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           SMEM_BYTES);
      attr_set[dev] = true;
    }
    if (M >= gemm16p::BM) {
      // CTA pairs: 256 x 512 tiles when their rounds over the clusters take no
      // longer than those of 256 x 256 tiles (counted in 256 x 256 tile times),
      // else 256 x 256 tiles
      const int64_t pairs = sm_count() / 2;
      const int64_t mt = (M + gemm16p::BM - 1) / gemm16p::BM;
      const int64_t t1 = mt * ((N + 255) / 256) * batch, t2 = mt * ((N + 511) / 512) * batch;
      const int64_t r1 = (t1 + pairs - 1) / pairs, r2 = 2 * ((t2 + pairs - 1) / pairs);
      if (N > 256 && r2 <= r1)
        return launch_gemm16_pair<2>(ta, tb, bias, C, M, N, K, batch, out_f16, epilogue, st);
      return launch_gemm16_pair<1>(ta, tb, bias, C, M, N, K, batch, out_f16, epilogue, st);
    }
    const int grid = (int)(tiles < sm_count() ? tiles : sm_count());
    gemm_f16_tc_kernel<<<grid, THREADS, SMEM_BYTES, st>>>(ta, tb, bias, C, (int)M, (int)N, (int)K,
                                                          (int)batch, M * N, out_f16, epilogue,
                                                          device_status_ptr());
    return check_launch("emmy_gemm_f16 (tcgen05)");
  }
  dim3 grid((unsigned)((M + 63) / 64), (unsigned)((N + 63) / 64), (unsigned)batch);
  gemm_f16_plain_kernel<<<grid, 256, 0, st>>>(static_cast<const __half *>(A),
                                              static_cast<const __half *>(B), bias, C, (int)M,
                                              (int)N, (int)K, M * K, K * N, M * N, out_f16,
                                              epilogue);
  return check_launch("emmy_gemm_f16 (plain)");
}
