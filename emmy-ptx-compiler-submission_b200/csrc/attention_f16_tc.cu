// f16 attention-like chain with f32 softmax on the sm_100a tensor cores:
//   o = softmax(q k^T * recip(div)) v      per (batch, head), q/k/v/o [BH, S, D]
//
// Replaces the entry the reference emits for its attention IR shape (key loop
// over a head-dim dot loop, online max/sum with exp rescaling, a rescaled
// weighted sum of v and a final divide; reference ptxc/stmts.py:663-725,
// 564-611, 1311-1392, ptxc/expr.py:891-895), here with f16 operands as the
// benchmark configuration asks.
//
// One CTA owns 128 query rows of one (batch, head) and walks the keys in
// blocks of 64; up to D = 128 two CTAs share an SM, so one CTA's softmax runs
// while the other's tensor-core work does.  Warp roles:
//   warp 4      TMA producer: Q once, K blocks through a 2-stage ring (one
//               block ahead), V blocks through one buffer (no multicast;
//               128-byte swizzled boxes)
//   warp 5      one thread issues tcgen05.mma: S = Q K^T into TMEM (M128 x 64
//               keys), then, once P is ready, O += P V into TMEM (M128 x D)
//   warps 0-3   one query row per thread (TMEM lane): read the 64 scores once,
//               keep the running max m and sum l (base-2, scale folded in),
//               rescale the O row in TMEM when the max moves, write P as f16
//               into swizzled shared memory, and finally store O / l.
// Every mbarrier wait is bounded and reports through the device status word.

#include "common.cuh"
#include "tcgen05.cuh"

namespace emmy {

template <int D>
struct AttnCfg {
  static constexpr int BN = 64;                      // keys per block
  static constexpr int NKB = D / 64;                 // 64-wide head-dim blocks of Q and K
  static constexpr int NVB = D / 64;                 // 64-wide column blocks of V
  static constexpr int Q_BOX = 128 * 128;            // [128 rows][128 B]
  static constexpr int K_BOX = BN * 128;             // [BN keys][128 B]
  static constexpr int Q_BYTES = NKB * Q_BOX;
  static constexpr int K_BYTES = NKB * K_BOX;
  static constexpr int V_BYTES = NVB * K_BOX;
  static constexpr int P_BYTES = Q_BOX;              // [128 rows][64 keys] f16
  static constexpr int K_STAGES = 2;
  // Q | K stage 0 | K stage 1 | V | P, then the mbarriers
  static constexpr int BAR_OFF = Q_BYTES + K_STAGES * K_BYTES + V_BYTES + P_BYTES;
  static constexpr int SMEM = BAR_OFF + 128 + 1024;
  static constexpr uint32_t S_COL = 0;
  static constexpr uint32_t O_COL = 64;
  static constexpr uint32_t TMEM_COLS = O_COL + D <= 128 ? 128 : (O_COL + D <= 256 ? 256 : 512);
  static constexpr int THREADS = 192;
  static constexpr int MIN_BLOCKS = D <= 128 ? 2 : 1;   // two CTAs per SM overlap softmax and MMA
};

// status codes of the waits that can give up (first one recorded wins)
constexpr int kAttnWaitQ = 0x1201, kAttnWaitK = 0x1202, kAttnWaitP = 0x1203,
              kAttnWaitKEmpty = 0x1204, kAttnWaitS = 0x1205, kAttnWaitO = 0x1206,
              kAttnWaitOFinal = 0x1207, kAttnWaitV = 0x1208, kAttnWaitVEmpty = 0x1209;

template <int D>
__global__ void __launch_bounds__(192, AttnCfg<D>::MIN_BLOCKS)
attention_f16_tc_kernel(const __grid_constant__ CUtensorMap tmQ,
                        const __grid_constant__ CUtensorMap tmK,
                        const __grid_constant__ CUtensorMap tmV, void *__restrict__ O,
                        const float *__restrict__ scale_div, int S, int out_f16, int *status) {
  using C = AttnCfg<D>;
  constexpr int BN = C::BN;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char *smem = reinterpret_cast<unsigned char *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  unsigned char *sQ = smem;
  unsigned char *sK = sQ + C::Q_BYTES;                          // 2 stages
  unsigned char *sV = sK + C::K_STAGES * C::K_BYTES;
  unsigned char *sP = sV + C::V_BYTES;
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + C::BAR_OFF);
  uint64_t *q_full = bars + 0, *s_full = bars + 1, *p_full = bars + 2, *o_full = bars + 3;
  uint64_t *v_full = bars + 4, *v_empty = bars + 5, *k_full = bars + 6, *k_empty = bars + 8;
  uint32_t *tmem_holder = reinterpret_cast<uint32_t *>(bars + 10);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m0 = blockIdx.x * 128, bh = blockIdx.y;
  const int nblk = (S + BN - 1) / BN;

  if (threadIdx.x == 0) {
    prefetch_tensormap(&tmQ);
    prefetch_tensormap(&tmK);
    prefetch_tensormap(&tmV);
    mbar_init(q_full, 1);
    mbar_init(s_full, 1);
    mbar_init(p_full, 128);
    mbar_init(o_full, 1);
    mbar_init(v_full, 1);
    mbar_init(v_empty, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&k_empty[s], 1);
    }
    fence_barrier_init();
  }
  if (warp == 4) tmem_alloc(tmem_holder, C::TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;

  if (warp == 4) {
    if (lane == 0) {
      // TMA producer.  K runs one block ahead of V: K[j+1] is issued before
      // V[j] waits for the previous P V product to release the V buffer.
      auto load_k = [&](int j) -> bool {
        const int s = j & 1;
        if (j >= 2 && !mbar_wait(&k_empty[s], ((j >> 1) - 1) & 1, status, kAttnWaitKEmpty))
          return false;
        mbar_expect_tx(&k_full[s], C::K_BYTES);
        for (int kb = 0; kb < C::NKB; ++kb)
          tma_load_3d(sK + s * C::K_BYTES + kb * C::K_BOX, &tmK, &k_full[s], kb * 64, j * BN, bh);
        return true;
      };
      mbar_expect_tx(q_full, C::Q_BYTES);
      for (int kb = 0; kb < C::NKB; ++kb)
        tma_load_3d(sQ + kb * C::Q_BOX, &tmQ, q_full, kb * 64, m0, bh);
      bool ok = load_k(0);
      for (int j = 0; ok && j < nblk; ++j) {
        if (j + 1 < nblk && !load_k(j + 1)) break;
        if (j >= 1 && !mbar_wait(v_empty, (j - 1) & 1, status, kAttnWaitVEmpty)) break;
        mbar_expect_tx(v_full, C::V_BYTES);
        for (int vb = 0; vb < C::NVB; ++vb)
          tma_load_3d(sV + vb * C::K_BOX, &tmV, v_full, vb * 64, j * BN, bh);
      }
    }
    __syncwarp();
  } else if (warp == 5) {
    if (lane == 0) {
      constexpr uint32_t idesc_s = f16_idesc(128, BN, false, false);
      constexpr uint32_t idesc_o = f16_idesc(128, D, false, true);
      bool ok = mbar_wait(q_full, 0, status, kAttnWaitQ);
      const uint32_t qa = smem_u32(sQ);
      const uint32_t pa = smem_u32(sP);
      const uint32_t va = smem_u32(sV);
      for (int j = 0; ok && j < nblk; ++j) {
        const int s = j & 1;
        if (!mbar_wait(&k_full[s], (j >> 1) & 1, status, kAttnWaitK)) break;
        tc_fence_after();
        const uint32_t ka = smem_u32(sK + s * C::K_BYTES);
        // S = Q K^T: both operands K-major (head dim contiguous)
#pragma unroll
        for (int kb = 0; kb < C::NKB; ++kb)
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            mma_f16(tmem + C::S_COL, sw128_desc(qa + kb * C::Q_BOX + kk * 32, 16, 1024),
                    sw128_desc(ka + kb * C::K_BOX + kk * 32, 16, 1024), idesc_s,
                    (kb | kk) != 0 ? 1u : 0u);
        mma_commit(s_full);
        mma_commit(&k_empty[s]);
        if (!mbar_wait(p_full, j & 1, status, kAttnWaitP)) break;
        if (!mbar_wait(v_full, j & 1, status, kAttnWaitV)) break;
        tc_fence_after();
        // O += P V: P K-major over the 64 keys, V N-major (value columns contiguous)
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          mma_f16(tmem + C::O_COL, sw128_desc(pa + kk * 32, 16, 1024),
                  sw128_desc(va + kk * 16 * 128, C::K_BOX, 1024), idesc_o,
                  (j | kk) != 0 ? 1u : 0u);
        mma_commit(o_full);
        mma_commit(v_empty);
      }
    }
    __syncwarp();
  } else {
    // softmax / correction / epilogue: thread r owns query row m0 + r (TMEM lane r).
    // Scores are kept as t = s * scale * log2(e), so p = 2^(t - m).
    const int r = threadIdx.x;
    const uint32_t lane_base = tmem + ((uint32_t)(warp * 32) << 16);
    const float c = (scale_div ? 1.0f / __ldg(scale_div) : 1.0f) * 1.4426950408889634f;
    float m = -INFINITY, l = 0.f;
    for (int j = 0; j < nblk; ++j) {
      mbar_wait(s_full, j & 1, status, kAttnWaitS);
      __syncwarp();
      tc_fence_after();
      const int key0 = j * BN;
      float t[64];
      {
        float v0[32], v1[32];
        tmem_ld32(lane_base + C::S_COL, v0);
        tmem_ld32(lane_base + C::S_COL + 32, v1);
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          t[i] = key0 + i < S ? v0[i] * c : -INFINITY;
          t[32 + i] = key0 + 32 + i < S ? v1[i] * c : -INFINITY;
        }
      }
      float mb = t[0];
#pragma unroll
      for (int i = 1; i < 64; ++i) mb = fmaxf(mb, t[i]);
      const float m_new = fmaxf(m, mb);
      const float alpha = exp2f(m - m_new);
      if (j > 0) {
        // P and O are still in use by the previous block's P V product
        mbar_wait(o_full, (j - 1) & 1, status, kAttnWaitO);
        __syncwarp();
        tc_fence_after();
        // tcgen05.ld/st are warp-collective (.sync.aligned): the whole warp
        // rescales when any of its rows' max moved (alpha is 1 for the others)
        if (__any_sync(0xffffffffu, m_new > m)) {
#pragma unroll 1
          for (int cc = 0; cc < D / 32; ++cc) {
            float v[32];
            __syncwarp();
            tmem_ld32(lane_base + C::O_COL + cc * 32, v);
#pragma unroll
            for (int i = 0; i < 32; ++i) v[i] *= alpha;
            tmem_st32(lane_base + C::O_COL + cc * 32, v);
          }
        }
      }
      float ps = 0.f;
      uint32_t h[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const float p0 = exp2f(t[2 * i] - m_new);
        const float p1 = exp2f(t[2 * i + 1] - m_new);
        ps += p0 + p1;
        __half2 hh = __floats2half2_rn(p0, p1);
        h[i] = *reinterpret_cast<uint32_t *>(&hh);
      }
      // 64 keys = eight 16-byte chunks of this row's 128-byte line; chunk
      // index XOR (row % 8) is the 128-byte swizzle
      unsigned char *rowp = sP + r * 128;
#pragma unroll
      for (int q = 0; q < 8; ++q)
        *reinterpret_cast<uint4 *>(rowp + ((q ^ (r & 7)) * 16)) =
            make_uint4(h[4 * q], h[4 * q + 1], h[4 * q + 2], h[4 * q + 3]);
      l = l * alpha + ps;
      m = m_new;
      fence_proxy_async();      // P (generic-proxy writes) visible to the tensor core
      tc_fence_before();
      mbar_arrive(p_full);
    }
    // epilogue: O / l
    mbar_wait(o_full, (nblk - 1) & 1, status, kAttnWaitOFinal);
    __syncwarp();
    tc_fence_after();
    const float rl = 1.0f / l;
    const int row = m0 + r;
#pragma unroll 1
    for (int cc = 0; cc < D / 32; ++cc) {
      float v[32];
      __syncwarp();   // reconverge after the masked stores of the previous chunk
      tmem_ld32(lane_base + C::O_COL + cc * 32, v);
      if (row < S) {
        const int64_t off = ((int64_t)bh * S + row) * D + cc * 32;
        if (out_f16) {
          __half *dst = reinterpret_cast<__half *>(O) + off;
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            uint32_t w[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              __half2 hh = __floats2half2_rn(v[8 * q + 2 * i] * rl, v[8 * q + 2 * i + 1] * rl);
              w[i] = *reinterpret_cast<uint32_t *>(&hh);
            }
            *reinterpret_cast<uint4 *>(dst + 8 * q) = make_uint4(w[0], w[1], w[2], w[3]);
          }
        } else {
          float *dst = reinterpret_cast<float *>(O) + off;
#pragma unroll
          for (int q = 0; q < 8; ++q)
            *reinterpret_cast<float4 *>(dst + 4 * q) =
                make_float4(v[4 * q] * rl, v[4 * q + 1] * rl, v[4 * q + 2] * rl, v[4 * q + 3] * rl);
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 4) tmem_dealloc(tmem, C::TMEM_COLS);
}

// CUDA-core fallback (any head dim, pre-transposed k, S beyond one block of
// shared memory is refused): f16 in, f32 math, exact two-pass row softmax.
template <typename TOut>
__global__ void __launch_bounds__(256)
attention_f16_simt_kernel(const __half *__restrict__ q, const __half *__restrict__ k,
                          const __half *__restrict__ v, TOut *__restrict__ o,
                          const float *__restrict__ scale_div, int Sq, int Sk, int D, int Dv,
                          int k_transposed) {
  extern __shared__ float sh[];
  float *qs = sh;
  float *ps = sh + D;
  __shared__ float red[32];
  const int row = blockIdx.x, b = blockIdx.y;
  const float scale = scale_div ? 1.0f / __ldg(scale_div) : 1.0f;
  const __half *qr = q + ((int64_t)b * Sq + row) * D;
  const __half *kb = k + (int64_t)b * Sk * D;
  const __half *vb = v + (int64_t)b * Sk * Dv;
  for (int d = threadIdx.x; d < D; d += blockDim.x) qs[d] = __half2float(qr[d]);
  __syncthreads();
  float m = kMaxSeed;
  for (int j = threadIdx.x; j < Sk; j += blockDim.x) {
    float acc = 0.f;
    for (int d = 0; d < D; ++d)
      acc = fmaf(__half2float(k_transposed ? kb[(int64_t)d * Sk + j] : kb[(int64_t)j * D + d]),
                 qs[d], acc);
    ps[j] = acc * scale;
    m = fmaxf(m, ps[j]);
  }
  m = warp_max(m);
  const int w = threadIdx.x >> 5, l32 = threadIdx.x & 31, nw = blockDim.x >> 5;
  __syncthreads();
  if (l32 == 0) red[w] = m;
  __syncthreads();
  m = warp_max(l32 < nw ? red[l32] : -INFINITY);
  float l = 0.f;
  for (int j = threadIdx.x; j < Sk; j += blockDim.x) {
    const float p = __expf(ps[j] - m);
    ps[j] = p;
    l += p;
  }
  l = warp_sum(l);
  __syncthreads();
  if (l32 == 0) red[w] = l;
  __syncthreads();
  l = warp_sum(l32 < nw ? red[l32] : 0.f);
  const float rl = 1.0f / l;
  TOut *orow = o + ((int64_t)b * Sq + row) * Dv;
  for (int c = threadIdx.x; c < Dv; c += blockDim.x) {
    float acc = 0.f;
    for (int j = 0; j < Sk; ++j) acc = fmaf(ps[j], __half2float(vb[(int64_t)j * Dv + c]), acc);
    if constexpr (sizeof(TOut) == 2) orow[c] = __float2half_rn(acc * rl);
    else orow[c] = acc * rl;
  }
}

namespace {

template <int D>
int launch_attention_tc(const void *q, const void *k, const void *v, void *o,
                        const float *scale_div, int64_t batch, int64_t S, int out_f16,
                        cudaStream_t st) {
  using Cfg = AttnCfg<D>;
  CUtensorMap tq, tk, tv;
  const uint64_t dims[3] = {(uint64_t)D, (uint64_t)S, (uint64_t)batch};
  const uint64_t str[2] = {(uint64_t)D * 2, (uint64_t)S * D * 2};
  const uint32_t qbox[3] = {64, 128, 1};
  const uint32_t kbox[3] = {64, Cfg::BN, 1};
  int rc = make_tensor_map(&tq, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, q, dims, str, qbox,
                           CU_TENSOR_MAP_SWIZZLE_128B);
  if (!rc) rc = make_tensor_map(&tk, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, k, dims, str, kbox,
                                CU_TENSOR_MAP_SWIZZLE_128B);
  if (!rc) rc = make_tensor_map(&tv, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, v, dims, str, kbox,
                                CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  static bool attr_set[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr_set[dev]) {
    cudaFuncSetAttribute(attention_f16_tc_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         Cfg::SMEM);
    attr_set[dev] = true;
  }
  dim3 grid((unsigned)((S + 127) / 128), (unsigned)batch);
  attention_f16_tc_kernel<D><<<grid, Cfg::THREADS, Cfg::SMEM, st>>>(
      tq, tk, tv, o, scale_div, (int)S, out_f16, device_status_ptr());
  return check_launch("emmy_attention_f16 (tcgen05)");
}

}  // namespace

}  // namespace emmy

using namespace emmy;

extern "C" int emmy_attention_f16(const void *q, const void *k, const void *v, void *o,
                                  const float *scale_div, int64_t batch, int64_t sq, int64_t sk,
                                  int64_t d, int out_dtype, int k_transposed, void *stream) {
  clear_error();
  if (batch < 0 || sq < 0 || sk < 0 || d < 0)
    return set_error(EMMY_ERR_INVALID, "emmy_attention_f16: negative size");
  if (batch == 0 || sq == 0 || d == 0) return EMMY_OK;
  if (sk == 0) return set_error(EMMY_ERR_INVALID, "emmy_attention_f16: no keys");
  if (!q || !k || !v || !o) return set_error(EMMY_ERR_INVALID, "emmy_attention_f16: null operand");
  if (out_dtype != EMMY_DT_F32 && out_dtype != EMMY_DT_F16)
    return set_error(EMMY_ERR_INVALID, "emmy_attention_f16: bad output dtype");
  if (batch > 65535 || sq > INT32_MAX || sk > INT32_MAX)
    return set_error(EMMY_ERR_UNSUPPORTED, "emmy_attention_f16: grid too large");
  cudaStream_t st = as_stream(stream);
  const int out_f16 = out_dtype == EMMY_DT_F16;
  const bool tc = !k_transposed && sq == sk && aligned16(q) && aligned16(k) && aligned16(v) &&
                  aligned16(o) && (d == 64 || d == 128 || d == 256);
  if (tc) {
    if (d == 64) return launch_attention_tc<64>(q, k, v, o, scale_div, batch, sq, out_f16, st);
    if (d == 128) return launch_attention_tc<128>(q, k, v, o, scale_div, batch, sq, out_f16, st);
    return launch_attention_tc<256>(q, k, v, o, scale_div, batch, sq, out_f16, st);
  }
  const size_t smem = (size_t)(d + sk) * sizeof(float);
  if (smem > 200 * 1024)
    return set_error(EMMY_ERR_UNSUPPORTED, "emmy_attention_f16: %lld keys exceed shared memory",
                     (long long)sk);
  dim3 grid((unsigned)sq, (unsigned)batch);
  if (out_f16) {
    if (smem > 48 * 1024)
      cudaFuncSetAttribute(attention_f16_simt_kernel<__half>,
                           cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    attention_f16_simt_kernel<__half><<<grid, 256, smem, st>>>(
        static_cast<const __half *>(q), static_cast<const __half *>(k),
        static_cast<const __half *>(v), static_cast<__half *>(o), scale_div, (int)sq, (int)sk,
        (int)d, (int)d, k_transposed);
  } else {
    if (smem > 48 * 1024)
      cudaFuncSetAttribute(attention_f16_simt_kernel<float>,
                           cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    attention_f16_simt_kernel<float><<<grid, 256, smem, st>>>(
        static_cast<const __half *>(q), static_cast<const __half *>(k),
        static_cast<const __half *>(v), static_cast<float *>(o), scale_div, (int)sq, (int)sk,
        (int)d, (int)d, k_transposed);
  }
  return check_launch("emmy_attention_f16 (simt)");
}
