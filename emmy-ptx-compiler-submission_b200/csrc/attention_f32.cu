// f32 attention-like chain on sm_100a CUDA cores: out = softmax(q k^T * s) v.
//
// Replaces the entry the reference emits for the f32 attention fixtures
// (v_a_*, w_a_*): per output element a key loop with an inner head-dim dot
// loop, an online max/sum with exp rescaling and a rescaled weighted sum of v,
// divided by the sum at the end (reference ptxc/stmts.py:663-725, 564-611,
// 1311-1392; exp as ptxc/expr.py:891-895).  The scale s is recip(div) of the
// one-element constant the IR loads.
//
// Here one CTA owns one query row of one (batch, head): the q row is staged in
// shared memory, every thread scores a strided subset of the keys (f32 fma dot
// over the head dim), the row max and sum are reduced across the block, and
// each thread then produces output columns as the probability-weighted sum of
// v, read coalesced along the columns.  Scores stay in shared memory, so the
// row is exact two-pass softmax rather than the online rescaling.

#include "common.cuh"

namespace emmy {

__device__ __forceinline__ float block_max(float v, float *red) {
  v = warp_max(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31, nw = blockDim.x >> 5;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  return warp_max(l < nw ? red[l] : -INFINITY);
}

__device__ __forceinline__ float block_sum(float v, float *red) {
  v = warp_sum(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31, nw = blockDim.x >> 5;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  return warp_sum(l < nw ? red[l] : 0.f);
}

// q [B, Sq, D]; k [B, Sk, D] (or kt [B, D, Sk]); v [B, Sk, Dv]; o [B, Sq, Dv]
__global__ void __launch_bounds__(256)
attention_f32_kernel(const float *__restrict__ q, const float *__restrict__ k,
                     const float *__restrict__ v, float *__restrict__ o,
                     const float *__restrict__ scale_div, int Sq, int Sk, int D, int Dv,
                     int k_transposed) {
  extern __shared__ float sh[];
  float *qs = sh;              // D
  float *ps = sh + D;          // Sk scores, then probabilities
  __shared__ float red[32];
  const int row = blockIdx.x, b = blockIdx.y;
  const float scale = scale_div ? 1.0f / __ldg(scale_div) : 1.0f;
  const float *qr = q + ((int64_t)b * Sq + row) * D;
  const float *kb = k + (int64_t)b * Sk * D;
  const float *vb = v + (int64_t)b * Sk * Dv;
  for (int d = threadIdx.x; d < D; d += blockDim.x) qs[d] = __ldg(qr + d);
  __syncthreads();
  float m = kMaxSeed;
  for (int j = threadIdx.x; j < Sk; j += blockDim.x) {
    float acc = 0.f;
    if (k_transposed) {
      for (int d = 0; d < D; ++d) acc = fmaf(__ldg(kb + (int64_t)d * Sk + j), qs[d], acc);
    } else {
      const float *kr = kb + (int64_t)j * D;
      for (int d = 0; d < D; ++d) acc = fmaf(__ldg(kr + d), qs[d], acc);
    }
    const float s = acc * scale;
    ps[j] = s;
    m = fmaxf(m, s);
  }
  m = block_max(m, red);
  float l = 0.f;
  for (int j = threadIdx.x; j < Sk; j += blockDim.x) {
    const float p = __expf(ps[j] - m);
    ps[j] = p;
    l += p;
  }
  l = block_sum(l, red);      // also orders the ps writes before the reads below
  const float r = 1.0f / l;
  float *orow = o + ((int64_t)b * Sq + row) * Dv;
  for (int c = threadIdx.x; c < Dv; c += blockDim.x) {
    float acc = 0.f;
    for (int j = 0; j < Sk; ++j) acc = fmaf(ps[j], __ldg(vb + (int64_t)j * Dv + c), acc);
    orow[c] = acc * r;
  }
}

}  // namespace emmy

using namespace emmy;

extern "C" int emmy_attention_f32(const float *q, const float *k, const float *v, float *o,
                                  const float *scale_div, int64_t batch, int64_t sq, int64_t sk,
                                  int64_t d, int64_t dv, int k_transposed, void *stream) {
  clear_error();
  if (batch < 0 || sq < 0 || sk < 0 || d < 0 || dv < 0)
    return set_error(EMMY_ERR_INVALID, "emmy_attention_f32: negative size");
  if (batch == 0 || sq == 0 || dv == 0) return EMMY_OK;
  if (sk == 0) return set_error(EMMY_ERR_INVALID, "emmy_attention_f32: no keys");
  if (!q || !k || !v || !o) return set_error(EMMY_ERR_INVALID, "emmy_attention_f32: null operand");
  if (batch > 65535 || sq > INT32_MAX)
    return set_error(EMMY_ERR_UNSUPPORTED, "emmy_attention_f32: grid too large");
  // head dims up to 96 (d == dv): one thread per query row (any key count)
  const int rc = launch_attention_rows(q, k, v, o, scale_div, batch, sq, sk, d, dv, 0, 0,
                                       k_transposed, as_stream(stream));
  if (rc >= 0) return rc;
  const size_t smem = (size_t)(d + sk) * sizeof(float);
  if (smem > 200 * 1024)
    return set_error(EMMY_ERR_UNSUPPORTED, "emmy_attention_f32: %lld keys exceed shared memory",
                     (long long)sk);
  if (smem > 48 * 1024)
    cudaFuncSetAttribute(attention_f32_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)smem);
  dim3 grid((unsigned)sq, (unsigned)batch);
  attention_f32_kernel<<<grid, 256, smem, as_stream(stream)>>>(q, k, v, o, scale_div, (int)sq,
                                                               (int)sk, (int)d, (int)dv,
                                                               k_transposed);
  return check_launch("emmy_attention_f32");
}
