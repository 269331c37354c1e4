// Attention on CUDA cores for head dims the tcgen05 kernel does not take
// (D <= 96; f32 operands, pre-transposed keys, unaligned tensors).
//
// The reference emits this IR shape (reference ptxc/stmts.py:663-725 for the
// key Loop, :564-611 for the online max/sum Accum pair, :1311-1392 for the
// warp dot) as one thread per (query row, value column) walking every key.
// Here one thread owns a query row: q and the output accumulator sit in
// registers (D floats each), a 128-thread CTA stages 32 keys and their values
// at a time in shared memory (every thread reads the same element: a
// broadcast), computes the 32 scores, folds them into a running max / sum
// (rescaling the accumulator only when the tile raises the max), and adds the
// weighted values.  Work per (query, key): 2*D FMAs and one exp.

#include "common.cuh"

namespace emmy {

namespace {

constexpr int kRowsThreads = 128, kRowsKT = 32;

template <typename T> __device__ __forceinline__ float to_f(T v) { return float(v); }
template <> __device__ __forceinline__ float to_f<__half>(__half v) { return __half2float(v); }

template <typename TI, typename TO, int D>
__global__ void __launch_bounds__(kRowsThreads)
attention_rows_kernel(const TI *__restrict__ q, const TI *__restrict__ k, const TI *__restrict__ v,
                      TO *__restrict__ o, const float *__restrict__ scale_div, int Sq, int Sk,
                      int k_transposed) {
  static_assert(D % 4 == 0, "head dim in 16-byte groups");
  __shared__ float4 Ks[kRowsKT][D / 4];
  __shared__ float4 Vs[kRowsKT][D / 4];
  const int b = blockIdx.y;
  const int row = blockIdx.x * kRowsThreads + threadIdx.x;
  const bool live = row < Sq;
  const float c = scale_div ? 1.0f / __ldg(scale_div) : 1.0f;
  const TI *kb = k + (int64_t)b * Sk * D;
  const TI *vb = v + (int64_t)b * Sk * D;
  float qr[D], acc[D];
#pragma unroll
  for (int d = 0; d < D; ++d) {
    qr[d] = live ? to_f(q[((int64_t)b * Sq + row) * D + d]) : 0.f;
    acc[d] = 0.f;
  }
  float m = -INFINITY, l = 0.f;
  for (int k0 = 0; k0 < Sk; k0 += kRowsKT) {
    __syncthreads();                      // the previous tile is consumed
    for (int i = threadIdx.x; i < kRowsKT * D; i += kRowsThreads) {
      const int j = i / D, d = i - j * D, key = k0 + j;
      float kv = 0.f, vv = 0.f;
      if (key < Sk) {
        kv = to_f(k_transposed ? kb[(int64_t)d * Sk + key] : kb[(int64_t)key * D + d]);
        vv = to_f(vb[(int64_t)key * D + d]);
      }
      reinterpret_cast<float *>(&Ks[j][0])[d] = kv;
      reinterpret_cast<float *>(&Vs[j][0])[d] = vv;
    }
    __syncthreads();
    float s[kRowsKT];
    float mt = -INFINITY;
#pragma unroll
    for (int j = 0; j < kRowsKT; ++j) {
      float dot = 0.f;
#pragma unroll
      for (int d4 = 0; d4 < D / 4; ++d4) {
        const float4 kk = Ks[j][d4];           // one broadcast 16-byte load per 4 FMAs
        dot = fmaf(qr[4 * d4], kk.x, dot);
        dot = fmaf(qr[4 * d4 + 1], kk.y, dot);
        dot = fmaf(qr[4 * d4 + 2], kk.z, dot);
        dot = fmaf(qr[4 * d4 + 3], kk.w, dot);
      }
      s[j] = k0 + j < Sk ? dot * c : -INFINITY;
      mt = fmaxf(mt, s[j]);
    }
    if (mt > m) {                         // rescale only when the tile raises the max
      const float corr = __expf(m - mt);  // 0 on the first tile (m = -inf)
      l *= corr;
#pragma unroll
      for (int d = 0; d < D; ++d) acc[d] *= corr;
      m = mt;
    }
#pragma unroll
    for (int j = 0; j < kRowsKT; ++j) {
      const float p = __expf(s[j] - m);
      l += p;
#pragma unroll
      for (int d4 = 0; d4 < D / 4; ++d4) {
        const float4 vv = Vs[j][d4];
        acc[4 * d4] = fmaf(p, vv.x, acc[4 * d4]);
        acc[4 * d4 + 1] = fmaf(p, vv.y, acc[4 * d4 + 1]);
        acc[4 * d4 + 2] = fmaf(p, vv.z, acc[4 * d4 + 2]);
        acc[4 * d4 + 3] = fmaf(p, vv.w, acc[4 * d4 + 3]);
      }
    }
  }
  if (!live) return;
  const float rl = 1.0f / l;
  TO *orow = o + ((int64_t)b * Sq + row) * D;
#pragma unroll
  for (int d = 0; d < D; ++d) {
    if constexpr (sizeof(TO) == 2) orow[d] = __float2half_rn(acc[d] * rl);
    else orow[d] = acc[d] * rl;
  }
}

template <typename TI, typename TO, int D>
int launch_rows(const void *q, const void *k, const void *v, void *o, const float *scale_div,
                int64_t batch, int64_t sq, int64_t sk, int k_transposed, cudaStream_t st) {
  dim3 grid((unsigned)((sq + kRowsThreads - 1) / kRowsThreads), (unsigned)batch);
  attention_rows_kernel<TI, TO, D><<<grid, kRowsThreads, 0, st>>>(
      static_cast<const TI *>(q), static_cast<const TI *>(k), static_cast<const TI *>(v),
      static_cast<TO *>(o), scale_div, (int)sq, (int)sk, k_transposed);
  return check_launch("attention (rows)");
}

template <typename TI, typename TO>
int dispatch_rows(const void *q, const void *k, const void *v, void *o, const float *scale_div,
                  int64_t batch, int64_t sq, int64_t sk, int64_t d, int k_transposed,
                  cudaStream_t st) {
  switch (d) {
#define EMMY_ROWS_D(DD) \
    case DD: return launch_rows<TI, TO, DD>(q, k, v, o, scale_div, batch, sq, sk, k_transposed, st);
    EMMY_ROWS_D(8) EMMY_ROWS_D(16) EMMY_ROWS_D(24) EMMY_ROWS_D(32) EMMY_ROWS_D(48)
    EMMY_ROWS_D(64) EMMY_ROWS_D(80) EMMY_ROWS_D(96)
#undef EMMY_ROWS_D
    default: return -1;
  }
}

}  // namespace

// -1 when (d, dv) has no row-per-thread kernel; otherwise the launch status.
int launch_attention_rows(const void *q, const void *k, const void *v, void *o,
                          const float *scale_div, int64_t batch, int64_t sq, int64_t sk,
                          int64_t d, int64_t dv, int in_f16, int out_f16, int k_transposed,
                          cudaStream_t st) {
  if (d != dv || sq > INT32_MAX || sk > INT32_MAX || batch > 65535) return -1;
  if (in_f16) {
    if (out_f16) return dispatch_rows<__half, __half>(q, k, v, o, scale_div, batch, sq, sk, d, k_transposed, st);
    return dispatch_rows<__half, float>(q, k, v, o, scale_div, batch, sq, sk, d, k_transposed, st);
  }
  return dispatch_rows<float, float>(q, k, v, o, scale_div, batch, sq, sk, d, k_transposed, st);
}

}  // namespace emmy
