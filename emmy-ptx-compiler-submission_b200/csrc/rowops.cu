// Memory-bound row families on sm_100a: row reductions, rmsnorm / l2norm /
// layernorm and softmax.
//
// The reference emits, for each of these IR shapes, one thread per element slot
// with scalar 4-byte loads, a 5-level shfl.sync.bfly tree, shared slots and a
// TreeHalve, and reads a normalised row twice (reduce pass, then map pass)
// (reference ptxc/stmts.py:728-773, 1441-1568).  Here a row is read from HBM
// once with 128-bit streaming loads, held in registers, reduced with warp
// shuffles plus at most one shared-memory stage, and written once.  Rows too
// long for registers fall back to a two-read streaming kernel.
//
// Arithmetic follows the IR's op order (ptxc/expr.py:880-1089): recip is an
// IEEE division 1/x, sqrt is IEEE, exp is the fast exponential the reference
// also uses (ex2 of x*log2 e), and a squared-sum fold is an FMA as in the
// reference's fused accumulate (ptxc/stmts.py:614-632).

#include "common.cuh"

namespace emmy {

enum RowMode { MODE_SOFTMAX = 0, MODE_RMS = 1, MODE_L2 = 2, MODE_LN = 3 };

// ---------------------------------------------------------------------------
// group reductions: TPR threads cooperate on one row.  TPR == 32 is one warp
// (several rows per block); TPR > 32 is the whole block (one row per block).

template <int TPR>
__device__ __forceinline__ float group_sum(float v, float *red) {
  v = warp_sum(v);
  if constexpr (TPR > 32) {
    constexpr int W = TPR / 32;
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    __syncthreads();
    if (l == 0) red[w] = v;
    __syncthreads();
    v = warp_sum(l < W ? red[l] : 0.f);
  }
  return v;
}

// two sums reduced together (one shared-memory stage for both)
template <int TPR>
__device__ __forceinline__ void group_sum2(float &a, float &b, float *red) {
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) {
    a += __shfl_xor_sync(0xffffffffu, a, o);
    b += __shfl_xor_sync(0xffffffffu, b, o);
  }
  if constexpr (TPR > 32) {
    constexpr int W = TPR / 32;
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    __syncthreads();
    if (l == 0) {
      red[w] = a;
      red[16 + w] = b;
    }
    __syncthreads();
    a = l < W ? red[l] : 0.f;
    b = l < W ? red[16 + l] : 0.f;
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) {
      a += __shfl_xor_sync(0xffffffffu, a, o);
      b += __shfl_xor_sync(0xffffffffu, b, o);
    }
  }
}

template <int TPR>
__device__ __forceinline__ float group_max(float v, float *red) {
  v = warp_max(v);
  if constexpr (TPR > 32) {
    constexpr int W = TPR / 32;
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    __syncthreads();
    if (l == 0) red[w] = v;
    __syncthreads();
    v = warp_max(l < W ? red[l] : -INFINITY);
  }
  return v;
}

template <int TPR>
__device__ __forceinline__ float group_min(float v, float *red) {
  v = warp_min(v);
  if constexpr (TPR > 32) {
    constexpr int W = TPR / 32;
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    __syncthreads();
    if (l == 0) red[w] = v;
    __syncthreads();
    v = warp_min(l < W ? red[l] : INFINITY);
  }
  return v;
}

// ---------------------------------------------------------------------------
// register-resident row kernel: softmax, rms, l2, layernorm over rows of
// `cols` contiguous floats.  Each of the TPR threads owns NCH chunks of VEC
// consecutive elements: chunk c of thread t covers elements (c*TPR + t)*VEC.

// PREF: the weight (and, for layer norm, bias) elements a thread multiplies
// by are read into registers once, before its first row, when they number at
// most PREF per thread -- every row uses the same ones, and read after the
// row's reduction their L2 latency would sit on every row's path.
template <int MODE, int VEC, int TPR, int NCH, int PREF = 32>
__global__ void __launch_bounds__(TPR > 32 ? TPR : 256)
row_resident_kernel(const float *__restrict__ x, const float *__restrict__ w,
                    const float *__restrict__ b, float *__restrict__ y, int64_t rows,
                    int64_t cols, const float *__restrict__ eps_p,
                    const float *__restrict__ count_p) {
  constexpr int RPB = TPR > 32 ? 1 : 8;
  __shared__ float red[32];
  const int g = TPR > 32 ? 0 : (threadIdx.x >> 5);
  const int t = TPR > 32 ? threadIdx.x : (threadIdx.x & 31);
  float eps = 0.f, inv_count = 0.f;
  if constexpr (MODE == MODE_RMS || MODE == MODE_LN) {
    eps = eps_p ? __ldg(eps_p) : 0.f;
    inv_count = 1.0f / (count_p ? __ldg(count_p) : (float)cols);
  }
  constexpr bool PRE_W =
      (MODE == MODE_RMS || MODE == MODE_LN) && NCH * VEC * (MODE == MODE_LN ? 2 : 1) <= PREF;
  constexpr bool PRE_B = PRE_W && MODE == MODE_LN;
  float wv[PRE_W ? NCH : 1][VEC], bv[PRE_B ? NCH : 1][VEC];
  if constexpr (PRE_W) {
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      const int64_t idx = ((int64_t)c * TPR + t) * VEC;
#pragma unroll
      for (int k = 0; k < VEC; ++k) wv[c][k] = 1.f;
      if (w != nullptr && idx < cols) {
        if constexpr (VEC == 4) {
          const float4 q = __ldg(reinterpret_cast<const float4 *>(w + idx));
          wv[c][0] = q.x; wv[c][1] = q.y; wv[c][2] = q.z; wv[c][3] = q.w;
        } else {
          wv[c][0] = __ldg(w + idx);
        }
      }
      if constexpr (PRE_B) {
#pragma unroll
        for (int k = 0; k < VEC; ++k) bv[c][k] = 0.f;
        if (b != nullptr && idx < cols) {
          if constexpr (VEC == 4) {
            const float4 q = __ldg(reinterpret_cast<const float4 *>(b + idx));
            bv[c][0] = q.x; bv[c][1] = q.y; bv[c][2] = q.z; bv[c][3] = q.w;
          } else {
            bv[c][0] = __ldg(b + idx);
          }
        }
      }
    }
  }

  for (int64_t row = (int64_t)blockIdx.x * RPB + g; row < rows;
       row += (int64_t)gridDim.x * RPB) {
    const float *xr = x + row * cols;
    float *yr = y + row * cols;
    float v[NCH][VEC];
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      const int64_t idx = ((int64_t)c * TPR + t) * VEC;
      if (idx < cols) {
        if constexpr (VEC == 4) {
          float4 q = ld_stream4(xr + idx);
          v[c][0] = q.x; v[c][1] = q.y; v[c][2] = q.z; v[c][3] = q.w;
        } else {
          v[c][0] = __ldcs(xr + idx);
        }
      } else {
#pragma unroll
        for (int k = 0; k < VEC; ++k) v[c][k] = 0.f;
      }
    }

    if constexpr (MODE == MODE_SOFTMAX) {
      float m = kMaxSeed;
#pragma unroll
      for (int c = 0; c < NCH; ++c)
        if (((int64_t)c * TPR + t) * VEC < cols) {
#pragma unroll
          for (int k = 0; k < VEC; ++k) m = fmaxf(m, v[c][k]);
        }
      m = group_max<TPR>(m, red);
      float s = 0.f;
#pragma unroll
      for (int c = 0; c < NCH; ++c)
        if (((int64_t)c * TPR + t) * VEC < cols) {
#pragma unroll
          for (int k = 0; k < VEC; ++k) {
            v[c][k] = __expf(v[c][k] - m);
            s += v[c][k];
          }
        }
      s = group_sum<TPR>(s, red);
      const float r = 1.0f / s;
#pragma unroll
      for (int c = 0; c < NCH; ++c) {
        const int64_t idx = ((int64_t)c * TPR + t) * VEC;
        if (idx < cols) {
          if constexpr (VEC == 4) {
            st_stream4(yr + idx, make_float4(v[c][0] * r, v[c][1] * r, v[c][2] * r, v[c][3] * r));
          } else {
            __stcs(yr + idx, v[c][0] * r);
          }
        }
      }
    } else if constexpr (MODE == MODE_RMS || MODE == MODE_L2) {
      float s = 0.f;
#pragma unroll
      for (int c = 0; c < NCH; ++c)
#pragma unroll
        for (int k = 0; k < VEC; ++k) s = fmaf(v[c][k], v[c][k], s);
      s = group_sum<TPR>(s, red);
      float r;
      if constexpr (MODE == MODE_RMS) r = 1.0f / sqrtf(eps + s * inv_count);
      else r = 1.0f / sqrtf(s);
#pragma unroll
      for (int c = 0; c < NCH; ++c) {
        const int64_t idx = ((int64_t)c * TPR + t) * VEC;
        if (idx < cols) {
          float o[VEC];
#pragma unroll
          for (int k = 0; k < VEC; ++k) o[k] = v[c][k] * r;
          if (MODE == MODE_RMS && w != nullptr) {
            if constexpr (PRE_W) {
#pragma unroll
              for (int k = 0; k < VEC; ++k) o[k] *= wv[c][k];
            } else if constexpr (VEC == 4) {
              float4 q = __ldg(reinterpret_cast<const float4 *>(w + idx));
              o[0] *= q.x; o[1] *= q.y; o[2] *= q.z; o[3] *= q.w;
            } else {
              o[0] *= __ldg(w + idx);
            }
          }
          if constexpr (VEC == 4) st_stream4(yr + idx, make_float4(o[0], o[1], o[2], o[3]));
          else __stcs(yr + idx, o[0]);
        }
      }
    } else {  // MODE_LN: the IR's two moments in one pass, var = E[x^2] - mean^2
      float s = 0.f, q2 = 0.f;
#pragma unroll
      for (int c = 0; c < NCH; ++c)
#pragma unroll
        for (int k = 0; k < VEC; ++k) {
          s += v[c][k];
          q2 = fmaf(v[c][k], v[c][k], q2);
        }
      group_sum2<TPR>(s, q2, red);
      const float mean = s * inv_count;
#pragma unroll
      for (int c = 0; c < NCH; ++c)
#pragma unroll
        for (int k = 0; k < VEC; ++k) v[c][k] = v[c][k] - mean;
      // rounded op by op like the IR (mul, mul, sub, add: no contraction)
      const float var = __fsub_rn(__fmul_rn(q2, inv_count), __fmul_rn(mean, mean));
      const float r = 1.0f / sqrtf(__fadd_rn(var, eps));
#pragma unroll
      for (int c = 0; c < NCH; ++c) {
        const int64_t idx = ((int64_t)c * TPR + t) * VEC;
        if (idx < cols) {
          float o[VEC];
#pragma unroll
          for (int k = 0; k < VEC; ++k) o[k] = v[c][k] * r;
          if (w != nullptr) {
            if constexpr (PRE_W) {
#pragma unroll
              for (int k = 0; k < VEC; ++k) o[k] *= wv[c][k];
            } else if constexpr (VEC == 4) {
              float4 q = __ldg(reinterpret_cast<const float4 *>(w + idx));
              o[0] *= q.x; o[1] *= q.y; o[2] *= q.z; o[3] *= q.w;
            } else {
              o[0] *= __ldg(w + idx);
            }
          }
          if (b != nullptr) {
            if constexpr (PRE_B) {
#pragma unroll
              for (int k = 0; k < VEC; ++k) o[k] += bv[c][k];
            } else if constexpr (VEC == 4) {
              float4 q = __ldg(reinterpret_cast<const float4 *>(b + idx));
              o[0] += q.x; o[1] += q.y; o[2] += q.z; o[3] += q.w;
            } else {
              o[0] += __ldg(b + idx);
            }
          }
          if constexpr (VEC == 4) st_stream4(yr + idx, make_float4(o[0], o[1], o[2], o[3]));
          else __stcs(yr + idx, o[0]);
        }
      }
    }
  }
}

// ---------------------------------------------------------------------------
// streaming row kernel for rows longer than the register capacity: one block
// per row, the row is read twice (statistics, then the map pass).

template <int MODE>
__global__ void __launch_bounds__(1024)
row_stream_kernel(const float *__restrict__ x, const float *__restrict__ w,
                  const float *__restrict__ b, float *__restrict__ y, int64_t rows,
                  int64_t cols, const float *__restrict__ eps_p,
                  const float *__restrict__ count_p) {
  __shared__ float red[32];
  const int t = threadIdx.x;
  float eps = 0.f, inv_count = 0.f;
  if constexpr (MODE == MODE_RMS || MODE == MODE_LN) {
    eps = eps_p ? __ldg(eps_p) : 0.f;
    inv_count = 1.0f / (count_p ? __ldg(count_p) : (float)cols);
  }
  for (int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
    const float *xr = x + row * cols;
    float *yr = y + row * cols;
    if constexpr (MODE == MODE_SOFTMAX) {
      float m = kMaxSeed;
      for (int64_t i = t; i < cols; i += 1024) m = fmaxf(m, __ldg(xr + i));
      m = group_max<1024>(m, red);
      float s = 0.f;
      for (int64_t i = t; i < cols; i += 1024) s += __expf(__ldg(xr + i) - m);
      s = group_sum<1024>(s, red);
      const float r = 1.0f / s;
      for (int64_t i = t; i < cols; i += 1024) __stcs(yr + i, __expf(__ldcs(xr + i) - m) * r);
    } else if constexpr (MODE == MODE_RMS || MODE == MODE_L2) {
      float s = 0.f;
      for (int64_t i = t; i < cols; i += 1024) {
        float v = __ldg(xr + i);
        s = fmaf(v, v, s);
      }
      s = group_sum<1024>(s, red);
      float r;
      if constexpr (MODE == MODE_RMS) r = 1.0f / sqrtf(eps + s * inv_count);
      else r = 1.0f / sqrtf(s);
      for (int64_t i = t; i < cols; i += 1024) {
        float o = __ldcs(xr + i) * r;
        if (MODE == MODE_RMS && w != nullptr) o *= __ldg(w + i);
        __stcs(yr + i, o);
      }
    } else {
      float s = 0.f;
      for (int64_t i = t; i < cols; i += 1024) s += __ldg(xr + i);
      s = group_sum<1024>(s, red);
      const float mean = s * inv_count;
      float q2 = 0.f;
      for (int64_t i = t; i < cols; i += 1024) {
        float d = __ldg(xr + i) - mean;
        q2 = fmaf(d, d, q2);
      }
      q2 = group_sum<1024>(q2, red);
      const float r = 1.0f / sqrtf(q2 * inv_count + eps);
      for (int64_t i = t; i < cols; i += 1024) {
        float o = (__ldcs(xr + i) - mean) * r;
        if (w != nullptr) o *= __ldg(w + i);
        if (b != nullptr) o += __ldg(b + i);
        __stcs(yr + i, o);
      }
    }
  }
}

// ---------------------------------------------------------------------------
// reductions

template <int OP>
__device__ __forceinline__ float fold(float a, float v) {
  if constexpr (OP == EMMY_REDUCE_SUM) return a + v;
  else if constexpr (OP == EMMY_REDUCE_MAX) return fmaxf(a, v);
  else return fminf(a, v);
}
template <int OP>
__device__ __forceinline__ float seed() {
  if constexpr (OP == EMMY_REDUCE_SUM) return 0.f;
  else if constexpr (OP == EMMY_REDUCE_MAX) return kMaxSeed;
  else return kMinSeed;
}
template <int PRE>
__device__ __forceinline__ float premap(float v) {
  if constexpr (PRE == EMMY_PRE_SQUARE) return v * v;
  else if constexpr (PRE == EMMY_PRE_ABS) return fabsf(v);
  else return v;
}
template <int OP, int TPR>
__device__ __forceinline__ float group_fold(float v, float *red) {
  if constexpr (OP == EMMY_REDUCE_SUM) return group_sum<TPR>(v, red);
  else if constexpr (OP == EMMY_REDUCE_MAX) return group_max<TPR>(v, red);
  else return group_min<TPR>(v, red);
}
template <int OP, int PRE>
__device__ __forceinline__ float fold_in(float a, float v) {
  if constexpr (OP == EMMY_REDUCE_SUM && PRE == EMMY_PRE_SQUARE) return fmaf(v, v, a);
  else return fold<OP>(a, premap<PRE>(v));
}

// contiguous rows: y[row] = fold(x[row, :])
template <int OP, int PRE, int VEC, int TPR>
__global__ void __launch_bounds__(TPR > 32 ? TPR : 256)
reduce_rows_kernel(const float *__restrict__ x, float *__restrict__ y, int64_t rows, int64_t n,
                   const float *__restrict__ count_p) {
  constexpr int RPB = TPR > 32 ? 1 : 8;
  __shared__ float red[32];
  const int g = TPR > 32 ? 0 : (threadIdx.x >> 5);
  const int t = TPR > 32 ? threadIdx.x : (threadIdx.x & 31);
  const float inv_count = count_p ? 1.0f / __ldg(count_p) : 0.f;
  for (int64_t row = (int64_t)blockIdx.x * RPB + g; row < rows;
       row += (int64_t)gridDim.x * RPB) {
    const float *xr = x + row * n;
    float a0 = seed<OP>(), a1 = seed<OP>();
    int64_t i = (int64_t)t * VEC;
    constexpr int64_t STEP = (int64_t)TPR * VEC;
    for (; i + STEP < n; i += 2 * STEP) {
      if constexpr (VEC == 4) {
        float4 p = ld_stream4(xr + i), q = ld_stream4(xr + i + STEP);
        a0 = fold_in<OP, PRE>(a0, p.x); a0 = fold_in<OP, PRE>(a0, p.y);
        a0 = fold_in<OP, PRE>(a0, p.z); a0 = fold_in<OP, PRE>(a0, p.w);
        a1 = fold_in<OP, PRE>(a1, q.x); a1 = fold_in<OP, PRE>(a1, q.y);
        a1 = fold_in<OP, PRE>(a1, q.z); a1 = fold_in<OP, PRE>(a1, q.w);
      } else {
        float p = __ldcs(xr + i), q = __ldcs(xr + i + STEP);
        a0 = fold_in<OP, PRE>(a0, p);
        a1 = fold_in<OP, PRE>(a1, q);
      }
    }
    for (; i < n; i += STEP) {
      if constexpr (VEC == 4) {
        float4 p = ld_stream4(xr + i);
        a0 = fold_in<OP, PRE>(a0, p.x); a0 = fold_in<OP, PRE>(a0, p.y);
        a0 = fold_in<OP, PRE>(a0, p.z); a0 = fold_in<OP, PRE>(a0, p.w);
      } else {
        a0 = fold_in<OP, PRE>(a0, __ldcs(xr + i));
      }
    }
    float a = group_fold<OP, TPR>(fold<OP>(a0, a1), red);
    if (t == 0) y[row] = count_p ? a * inv_count : a;
  }
}

// strided view [outer, n, inner], inner > 1: one thread per (o, i) column,
// consecutive threads on consecutive i so every step is a coalesced row read.
template <int OP, int PRE>
__global__ void __launch_bounds__(256)
reduce_cols_kernel(const float *__restrict__ x, float *__restrict__ y, int64_t outer, int64_t n,
                   int64_t inner, const float *__restrict__ count_p) {
  const float inv_count = count_p ? 1.0f / __ldg(count_p) : 0.f;
  const int64_t total = outer * inner;
  for (int64_t c = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; c < total;
       c += (int64_t)gridDim.x * blockDim.x) {
    const int64_t o = c / inner, i = c - o * inner;
    const float *p = x + o * n * inner + i;
    float a0 = seed<OP>(), a1 = seed<OP>(), a2 = seed<OP>(), a3 = seed<OP>();
    int64_t j = 0;
    for (; j + 4 <= n; j += 4) {
      a0 = fold_in<OP, PRE>(a0, __ldg(p + (j + 0) * inner));
      a1 = fold_in<OP, PRE>(a1, __ldg(p + (j + 1) * inner));
      a2 = fold_in<OP, PRE>(a2, __ldg(p + (j + 2) * inner));
      a3 = fold_in<OP, PRE>(a3, __ldg(p + (j + 3) * inner));
    }
    for (; j < n; ++j) a0 = fold_in<OP, PRE>(a0, __ldg(p + j * inner));
    float a = fold<OP>(fold<OP>(a0, a1), fold<OP>(a2, a3));
    y[c] = count_p ? a * inv_count : a;
  }
}

// one long row split over many CTAs: partial folds into `part`, then a
// single-CTA finish.  Deterministic (fixed split, fixed tree).
template <int OP, int PRE>
__global__ void __launch_bounds__(1024)
reduce_long_partial_kernel(const float *__restrict__ x, int64_t n, int64_t chunk,
                           float *__restrict__ part) {
  __shared__ float red[32];
  const int64_t lo = (int64_t)blockIdx.x * chunk;
  const int64_t hi = min(n, lo + chunk);
  float a0 = seed<OP>(), a1 = seed<OP>();
  // chunk is a multiple of 4096 elements, so lo is 16-byte aligned whenever x is
  const bool vec = ((reinterpret_cast<uintptr_t>(x) & 15u) == 0);
  int64_t i = lo;
  if (vec) {
    for (i = lo + (int64_t)threadIdx.x * 4; i + 3 < hi; i += 4096) {
      float4 p = ld_stream4(x + i);
      a0 = fold_in<OP, PRE>(a0, p.x); a1 = fold_in<OP, PRE>(a1, p.y);
      a0 = fold_in<OP, PRE>(a0, p.z); a1 = fold_in<OP, PRE>(a1, p.w);
    }
    // the float4 sweep covers every complete group of 4; at most 3 remain
    for (int64_t k = lo + ((hi - lo) / 4) * 4 + threadIdx.x; k < hi; k += 1024)
      a0 = fold_in<OP, PRE>(a0, __ldcs(x + k));
  } else {
    for (i = lo + threadIdx.x; i < hi; i += 1024) a0 = fold_in<OP, PRE>(a0, __ldcs(x + i));
  }
  float a = group_fold<OP, 1024>(fold<OP>(a0, a1), red);
  if (threadIdx.x == 0) part[blockIdx.x] = a;
}

template <int OP>
__global__ void __launch_bounds__(1024)
reduce_long_finish_kernel(const float *__restrict__ part, int nparts, float *__restrict__ y,
                          const float *__restrict__ count_p) {
  __shared__ float red[32];
  float a = seed<OP>();
  for (int i = threadIdx.x; i < nparts; i += 1024) a = fold<OP>(a, part[i]);
  a = group_fold<OP, 1024>(a, red);
  if (threadIdx.x == 0) y[0] = count_p ? a * (1.0f / __ldg(count_p)) : a;
}

// ---------------------------------------------------------------------------
// strided softmax [outer, n, inner], inner > 1: one thread per column, an
// online max/sum pass then the map pass.
__global__ void __launch_bounds__(256)
softmax_cols_kernel(const float *__restrict__ x, float *__restrict__ y, int64_t outer, int64_t n,
                    int64_t inner) {
  const int64_t total = outer * inner;
  for (int64_t c = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; c < total;
       c += (int64_t)gridDim.x * blockDim.x) {
    const int64_t o = c / inner, i = c - o * inner;
    const float *p = x + o * n * inner + i;
    float *q = y + o * n * inner + i;
    float m = kMaxSeed, s = 0.f;
    for (int64_t j = 0; j < n; ++j) {
      const float v = __ldg(p + j * inner);
      const float gn = fmaxf(m, v);
      s = s * __expf(m - gn) + __expf(v - gn);
      m = gn;
    }
    const float r = 1.0f / s;
    for (int64_t j = 0; j < n; ++j) q[j * inner] = __expf(__ldg(p + j * inner) - m) * r;
  }
}

// ---------------------------------------------------------------------------
// host dispatch

namespace {

template <int MODE, int VEC, int TPR, int NCH, int PREF = 32>
void launch_resident(const float *x, const float *w, const float *b, float *y, int64_t rows,
                     int64_t cols, const float *eps, const float *count, cudaStream_t st) {
  constexpr int RPB = TPR > 32 ? 1 : 8;
  constexpr int threads = TPR > 32 ? TPR : 256;
  int64_t blocks = (rows + RPB - 1) / RPB;
  const int64_t cap = (int64_t)sm_count() * 64;  // grid-stride beyond ~64 CTAs per SM
  if (blocks > cap * 16) blocks = cap * 16;
  row_resident_kernel<MODE, VEC, TPR, NCH, PREF>
      <<<(unsigned)blocks, threads, 0, st>>>(x, w, b, y, rows, cols, eps, count);
}

template <int MODE>
int dispatch_row(const float *x, const float *w, const float *b, float *y, int64_t rows,
                 int64_t cols, const float *eps, const float *count, cudaStream_t st) {
  const bool v4 = (cols % 4 == 0) && aligned16(x) && aligned16(y) && (!w || aligned16(w)) &&
                  (!b || aligned16(b));
#define EMMY_ROW_CASE(V, T, N)                                                   \
  if (cols <= (int64_t)(V) * (T) * (N)) {                                        \
    launch_resident<MODE, V, T, N>(x, w, b, y, rows, cols, eps, count, st);      \
    return check_launch("row kernel");                                           \
  }
  // Capacities grow 128 .. 32768 floats.  Rows of 512-1024 floats use two
  // warps per row (64 threads, 8-16 floats each): measured faster on B200 than
  // one warp per row, whose 72-register layernorm variant limits occupancy.
  if (v4) {
    EMMY_ROW_CASE(4, 32, 1) EMMY_ROW_CASE(4, 32, 2) EMMY_ROW_CASE(4, 64, 2)
    EMMY_ROW_CASE(4, 64, 4) EMMY_ROW_CASE(4, 128, 4) EMMY_ROW_CASE(4, 128, 8)
    EMMY_ROW_CASE(4, 256, 8) EMMY_ROW_CASE(4, 512, 8) EMMY_ROW_CASE(4, 1024, 8)
  } else {
    EMMY_ROW_CASE(1, 32, 4) EMMY_ROW_CASE(1, 32, 8) EMMY_ROW_CASE(1, 64, 8)
    EMMY_ROW_CASE(1, 64, 16) EMMY_ROW_CASE(1, 128, 16) EMMY_ROW_CASE(1, 256, 16)
    EMMY_ROW_CASE(1, 512, 16) EMMY_ROW_CASE(1, 1024, 16)
  }
#undef EMMY_ROW_CASE
  int64_t blocks = rows < (int64_t)sm_count() * 8 ? rows : (int64_t)sm_count() * 8;
  row_stream_kernel<MODE><<<(unsigned)blocks, 1024, 0, st>>>(x, w, b, y, rows, cols, eps, count);
  return check_launch("row stream kernel");
}

template <int OP, int PRE>
int dispatch_reduce(const float *x, float *y, int64_t outer, int64_t n, int64_t inner,
                    const float *count, void *ws, size_t ws_bytes, cudaStream_t st) {
  if (inner > 1) {
    const int64_t total = outer * inner;
    int64_t blocks = (total + 255) / 256;
    const int64_t cap = (int64_t)sm_count() * 32;
    if (blocks > cap) blocks = cap;
    reduce_cols_kernel<OP, PRE><<<(unsigned)blocks, 256, 0, st>>>(x, y, outer, n, inner, count);
    return check_launch("column reduction");
  }
  if (outer == 1 && n > (1 << 16)) {
    const int64_t chunk_min = 4096 * 4;
    int64_t parts = (n + chunk_min - 1) / chunk_min;
    const int64_t maxparts = (int64_t)sm_count() * 2;
    if (parts > maxparts) parts = maxparts;
    int64_t chunk = (n + parts - 1) / parts;
    chunk = (chunk + 4095) / 4096 * 4096;
    parts = (n + chunk - 1) / chunk;
    if (ws != nullptr && ws_bytes >= (size_t)parts * sizeof(float) && parts > 1) {
      float *part = static_cast<float *>(ws);
      reduce_long_partial_kernel<OP, PRE><<<(unsigned)parts, 1024, 0, st>>>(x, n, chunk, part);
      int rc = check_launch("long reduction (partials)");
      if (rc) return rc;
      reduce_long_finish_kernel<OP><<<1, 1024, 0, st>>>(part, (int)parts, y, count);
      return check_launch("long reduction (finish)");
    }
  }
  const bool v4 = (n % 4 == 0) && aligned16(x);
  const int64_t per = n / (v4 ? 4 : 1);
  auto go = [&](auto vec_c, auto tpr_c) {
    constexpr int V = decltype(vec_c)::value, T = decltype(tpr_c)::value;
    constexpr int RPB = T > 32 ? 1 : 8;
    int64_t blocks = (outer + RPB - 1) / RPB;
    const int64_t cap = (int64_t)sm_count() * 64 * 16;
    if (blocks > cap) blocks = cap;
    reduce_rows_kernel<OP, PRE, V, T><<<(unsigned)blocks, T > 32 ? T : 256, 0, st>>>(x, y, outer, n, count);
  };
  using I4 = std::integral_constant<int, 4>;
  using I1 = std::integral_constant<int, 1>;
  const bool few_rows = outer < (int64_t)sm_count() * 4;
  if (v4) {
    if (per <= 256 || !few_rows) go(I4{}, std::integral_constant<int, 32>{});
    else if (per <= 4096) go(I4{}, std::integral_constant<int, 256>{});
    else go(I4{}, std::integral_constant<int, 1024>{});
  } else {
    if (per <= 1024 || !few_rows) go(I1{}, std::integral_constant<int, 32>{});
    else if (per <= 16384) go(I1{}, std::integral_constant<int, 256>{});
    else go(I1{}, std::integral_constant<int, 1024>{});
  }
  return check_launch("row reduction");
}

}  // namespace

}  // namespace emmy

using namespace emmy;

extern "C" size_t emmy_reduce_workspace_bytes(int64_t outer, int64_t n, int64_t inner) {
  if (outer != 1 || inner != 1 || n <= (1 << 16)) return 0;
  return (size_t)sm_count() * 2 * sizeof(float);
}

extern "C" int emmy_reduce_f32(const float *x, float *y, int64_t outer, int64_t n, int64_t inner,
                               int op, int pre, const float *count, void *workspace,
                               size_t workspace_bytes, void *stream) {
  clear_error();
  if (outer < 0 || n < 0 || inner < 1)
    return set_error(EMMY_ERR_INVALID, "emmy_reduce_f32: bad view [%lld, %lld, %lld]",
                     (long long)outer, (long long)n, (long long)inner);
  if (outer * inner == 0) return EMMY_OK;
  if (!x || !y) return set_error(EMMY_ERR_INVALID, "emmy_reduce_f32: null tensor pointer");
  if (op < 0 || op > 2 || pre < 0 || pre > 2)
    return set_error(EMMY_ERR_INVALID, "emmy_reduce_f32: bad op %d / pre %d", op, pre);
  cudaStream_t st = as_stream(stream);
#define EMMY_RED(O, P)                                                             \
  if (op == O && pre == P)                                                         \
    return dispatch_reduce<O, P>(x, y, outer, n, inner, count, workspace, workspace_bytes, st);
  EMMY_RED(0, 0) EMMY_RED(0, 1) EMMY_RED(0, 2)
  EMMY_RED(1, 0) EMMY_RED(1, 1) EMMY_RED(1, 2)
  EMMY_RED(2, 0) EMMY_RED(2, 1) EMMY_RED(2, 2)
#undef EMMY_RED
  return set_error(EMMY_ERR_INVALID, "emmy_reduce_f32: unreachable op");
}

extern "C" int emmy_rownorm_f32(const float *x, const float *w, const float *b, float *y,
                                int64_t rows, int64_t cols, const float *eps,
                                const float *count, int mode, void *stream) {
  clear_error();
  if (rows < 0 || cols < 0)
    return set_error(EMMY_ERR_INVALID, "emmy_rownorm_f32: negative size");
  if (rows == 0 || cols == 0) return EMMY_OK;
  if (!x || !y) return set_error(EMMY_ERR_INVALID, "emmy_rownorm_f32: null tensor pointer");
  cudaStream_t st = as_stream(stream);
  switch (mode) {
    case EMMY_NORM_RMS:
      return dispatch_row<MODE_RMS>(x, w, nullptr, y, rows, cols, eps, count, st);
    case EMMY_NORM_L2:
      return dispatch_row<MODE_L2>(x, nullptr, nullptr, y, rows, cols, eps, count, st);
    case EMMY_NORM_LAYER:
      return dispatch_row<MODE_LN>(x, w, b, y, rows, cols, eps, count, st);
    default:
      return set_error(EMMY_ERR_INVALID, "emmy_rownorm_f32: bad mode %d", mode);
  }
}

extern "C" int emmy_softmax_f32(const float *x, float *y, int64_t outer, int64_t n, int64_t inner,
                                void *stream) {
  clear_error();
  if (outer < 0 || n < 0 || inner < 1)
    return set_error(EMMY_ERR_INVALID, "emmy_softmax_f32: bad view");
  if (outer * n * inner == 0) return EMMY_OK;
  if (!x || !y) return set_error(EMMY_ERR_INVALID, "emmy_softmax_f32: null tensor pointer");
  cudaStream_t st = as_stream(stream);
  if (inner == 1)
    return dispatch_row<MODE_SOFTMAX>(x, nullptr, nullptr, y, outer, n, nullptr, nullptr, st);
  const int64_t total = outer * inner;
  int64_t blocks = (total + 255) / 256;
  const int64_t cap = (int64_t)sm_count() * 32;
  if (blocks > cap) blocks = cap;
  softmax_cols_kernel<<<(unsigned)blocks, 256, 0, st>>>(x, y, outer, n, inner);
  return check_launch("column softmax");
}

// ---------------------------------------------------------------------------
// Long-row reduction with no allocation at all.
//
// emmy_reduce_f32 splits one long row over many CTAs only when the caller
// hands it a device workspace for the per-CTA partials.  Some callers cannot
// allocate device memory at the point of the call: hosts whose device memory
// is owned by a pool or budget fixed at start-up, code running inside an
// allocator or pool callback that must not re-enter it, and latency-critical
// loops where an allocation's implicit device synchronisation is not
// acceptable.  emmy_reduce_f32_noalloc serves them by
// keeping the partials in a fixed array in the library's own device memory.

namespace emmy {

// Capacity of the partials array: one float per CTA, 4096 CTAs (16 KB held on
// every device that loads the library, for the life of the process).
constexpr int kNoallocParts = 4096;
// Each CTA of the split reduces a fixed 16384-element chunk, so the longest
// row this entry point accepts is kNoallocParts * kNoallocChunk elements.
constexpr int64_t kNoallocChunk = 16384;

static __device__ __align__(256) float g_noalloc_partials[kNoallocParts];

// Device address of g_noalloc_partials for the current device.  Host code may
// not pass the symbol itself to a kernel (on the host it names a stand-in, not
// device memory), so the address is looked up with cudaGetSymbolAddress, with
// the device current, on the first call in each device context (later calls
// reuse it; the lookup is thread-safe and repeated after a device reset).
static float *noalloc_partials_ptr(int *rc) {
  void *p = symbol_address(reinterpret_cast<const void *>(&g_noalloc_partials), rc);
  if (!p) {
    char why[256];
    snprintf(why, sizeof(why), "%s", last_error_text());
    set_error(*rc, "emmy_reduce_f32_noalloc: the address of the built-in scratch: %s", why);
  }
  return static_cast<float *>(p);
}

template <int OP, int PRE>
int noalloc_long(const float *x, float *y, int64_t n, const float *count, float *part,
                 cudaStream_t st) {
  const int64_t parts = (n + kNoallocChunk - 1) / kNoallocChunk;
  reduce_long_partial_kernel<OP, PRE><<<(unsigned)parts, 1024, 0, st>>>(x, n, kNoallocChunk, part);
  int rc = check_launch("emmy_reduce_f32_noalloc (partials)");
  if (rc) return rc;
  reduce_long_finish_kernel<OP><<<1, 1024, 0, st>>>(part, (int)parts, y, count);
  return check_launch("emmy_reduce_f32_noalloc (finish)");
}

}  // namespace emmy

extern "C" int emmy_reduce_f32_noalloc(const float *x, float *y, int64_t n, int op, int pre,
                                       const float *count, void *stream) {
  clear_error();
  if (n <= 0) return set_error(EMMY_ERR_INVALID, "emmy_reduce_f32_noalloc: row length %lld",
                               (long long)n);
  if (n > (int64_t)kNoallocParts * kNoallocChunk)
    return set_error(EMMY_ERR_INVALID,
                     "emmy_reduce_f32_noalloc: row of %lld elements exceeds the %lld-element "
                     "limit of the built-in scratch (use emmy_reduce_f32 with a workspace)",
                     (long long)n, (long long)kNoallocParts * kNoallocChunk);
  if (!x || !y) return set_error(EMMY_ERR_INVALID, "emmy_reduce_f32_noalloc: null tensor pointer");
  if (op < 0 || op > 2 || pre < 0 || pre > 2)
    return set_error(EMMY_ERR_INVALID, "emmy_reduce_f32_noalloc: bad op %d / pre %d", op, pre);
  int rc = EMMY_OK;
  float *part = noalloc_partials_ptr(&rc);
  if (!part) return rc;
  cudaStream_t st = as_stream(stream);
#define EMMY_NA(O, P) \
  if (op == O && pre == P) return noalloc_long<O, P>(x, y, n, count, part, st);
  EMMY_NA(0, 0) EMMY_NA(0, 1) EMMY_NA(0, 2)
  EMMY_NA(1, 0) EMMY_NA(1, 1) EMMY_NA(1, 2)
  EMMY_NA(2, 0) EMMY_NA(2, 1) EMMY_NA(2, 2)
#undef EMMY_NA
  return set_error(EMMY_ERR_INVALID, "emmy_reduce_f32_noalloc: unreachable op");
}
