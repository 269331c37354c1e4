// Row families for f16 and f64 tensors, and for any mix of f16 / f32 / f64
// inputs and outputs: reductions (sum, mean, max, min; squared or absolute
// pre-map), dot with a row-invariant vector, softmax, and rms / l2 / layer
// normalisation.
//
// The reference lowers these IR shapes dtype by dtype: an f16 load widens to
// f32, an f16-typed Assign rounds back to f16, an f64 chain stays f64
// (reference ptxc/expr.py:168-180, 226-277, 1179-1309; the fold
// ptxc/stmts.py:564-632).  Here every element is computed in the compute type
// TC -- double when any tensor or the accumulator is f64, else float -- and
// rounded once, at the store, to the output dtype.  That is at least as
// accurate as the reference's per-step f16 rounding, and within its checked
// tolerances.  The f32-only path (rowops.cu) stays the fast path for f32
// tensors; this one is written for dtype generality: 4-element vector loads
// (8 bytes of f16, 16 of f32, 32 of f64) when the rows are aligned for them,
// coalesced across the threads of a row, and the statistics passes re-read
// the row from L1/L2 for the map pass.
//
// Layout: x viewed as [outer, n, inner] row-major.  inner == 1: a warp per row
// (n <= 2048, or 8192 with vector loads) or a 256-thread block per row; inner > 1 (reductions and
// softmax over a strided axis): one thread per (outer, inner) column,
// consecutive threads on consecutive inner positions.

#include "common.cuh"

namespace emmy {
namespace rowt {

enum Mode { M_SUM = 0, M_MAX = 1, M_MIN = 2, M_SOFTMAX = 3, M_RMS = 4, M_L2 = 5, M_LN = 6, M_DOT = 7 };

struct Args {
  const void *x, *w, *b, *eps, *count;
  void *y;
  int xdt, wdt, ydt, cdt;
  int pre;                      // EMMY_PRE_* for the reductions
  int64_t outer, n, inner;
};

// Plain loads on purpose: the half-precision __ldg is a non-volatile inline
// asm statement, which the compiler may speculate out of an `if (ptr)` or a
// dtype switch -- a load through a null weight pointer that faulted.  A plain
// load is never speculated through a pointer not known to be valid.
template <typename TC> __device__ __forceinline__ TC ld(const void *p, int dt, int64_t i) {
  if (dt == EMMY_DT_F16) return TC(__half2float(static_cast<const __half *>(p)[i]));
  if (dt == EMMY_DT_F64) return TC(static_cast<const double *>(p)[i]);
  return TC(static_cast<const float *>(p)[i]);
}

__device__ __forceinline__ __half to_half(float v) { return __float2half_rn(v); }
__device__ __forceinline__ __half to_half(double v) { return __double2half(v); }

template <typename TC> __device__ __forceinline__ void st(void *p, int dt, int64_t i, TC v) {
  if (dt == EMMY_DT_F16) static_cast<__half *>(p)[i] = to_half(v);
  else if (dt == EMMY_DT_F64) static_cast<double *>(p)[i] = double(v);
  else static_cast<float *>(p)[i] = float(v);
}

template <typename TC> __device__ __forceinline__ TC fma_c(TC a, TC b, TC c);
template <> __device__ __forceinline__ float fma_c(float a, float b, float c) { return fmaf(a, b, c); }
template <> __device__ __forceinline__ double fma_c(double a, double b, double c) { return fma(a, b, c); }

// the reference's exp: the fast exponential for f32 (ex2 of x*log2 e,
// ptxc/expr.py:891-895); f64 keeps double precision
__device__ __forceinline__ float exp_c(float v) { return __expf(v); }

// Packed pairs of f32 (sm_100 sub / mul / add .f32x2, each lane rounded as
// its scalar form) and the base-2 exponential with subnormal results flushed,
// for the f16 softmax rows: e^(x - m) = 2^((x - m) log2 e), the subtract and
// the multiply on pairs, as __expf(x - m) computes it lane by lane.  A
// flushed p (below 2^-126) is 0 in the f16 output either way.
__device__ __forceinline__ uint64_t pk2(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void upk2(uint64_t r, float &lo, float &hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(r));
}
__device__ __forceinline__ uint64_t sub2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t mul2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t add2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ float ex2_ftz(float a) {
  float r;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(a));
  return r;
}
// e^(x - m) for the two halves of h, as a packed pair (m2 = (m, m),
// c2 = (log2 e, log2 e))
__device__ __forceinline__ uint64_t exp_pair(__half2 h, uint64_t m2, uint64_t c2) {
  const float2 f = __half22float2(h);
  float t0, t1;
  upk2(mul2(sub2(pk2(f.x, f.y), m2), c2), t0, t1);
  return pk2(ex2_ftz(t0), ex2_ftz(t1));
}
__device__ __forceinline__ double exp_c(double v) { return exp(v); }

template <typename TC> __device__ __forceinline__ TC max_seed() { return TC(-1e30); }
template <typename TC> __device__ __forceinline__ TC min_seed() { return TC(1e30); }

template <int MODE, typename TC> __device__ __forceinline__ TC seed() {
  if constexpr (MODE == M_MAX || MODE == M_SOFTMAX) return max_seed<TC>();
  else if constexpr (MODE == M_MIN) return min_seed<TC>();
  else return TC(0);
}

template <int MODE, typename TC> __device__ __forceinline__ TC combine(TC a, TC b) {
  if constexpr (MODE == M_MAX || MODE == M_SOFTMAX) return fmax(a, b);
  else if constexpr (MODE == M_MIN) return fmin(a, b);
  else return a + b;
}

// fold of one element into a reduction accumulator, with the pre-map
template <int MODE, typename TC> __device__ __forceinline__ TC fold(TC a, TC v, int pre) {
  if (pre == EMMY_PRE_SQUARE) {
    if constexpr (MODE == M_SUM) return fma_c(v, v, a);
    v = v * v;
  } else if (pre == EMMY_PRE_ABS) {
    v = fabs(v);
  }
  return combine<MODE, TC>(a, v);
}

template <int MODE, int TPR, typename TC> __device__ __forceinline__ TC group(TC v, TC *red) {
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) v = combine<MODE, TC>(v, __shfl_xor_sync(0xffffffffu, v, o));
  if constexpr (TPR > 32) {
    constexpr int W = TPR / 32;
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    __syncthreads();
    if (l == 0) red[w] = v;
    __syncthreads();
    v = l < W ? red[l] : seed<MODE == M_SOFTMAX ? M_MAX : MODE, TC>();
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) v = combine<MODE, TC>(v, __shfl_xor_sync(0xffffffffu, v, o));
  }
  return v;
}

// VEC consecutive elements (VEC = 4: one 8-byte f16, 16-byte f32 or two
// 16-byte f64 plain loads; the caller guarantees alignment)
template <typename TC, int VEC>
__device__ __forceinline__ void ldv(const void *p, int dt, int64_t i, TC v[VEC]) {
  if constexpr (VEC == 1) {
    v[0] = ld<TC>(p, dt, i);
  } else {
    if (dt == EMMY_DT_F16) {
      const uint2 u = *reinterpret_cast<const uint2 *>(static_cast<const __half *>(p) + i);
      const __half2 h0 = *reinterpret_cast<const __half2 *>(&u.x);
      const __half2 h1 = *reinterpret_cast<const __half2 *>(&u.y);
      v[0] = TC(__low2float(h0)); v[1] = TC(__high2float(h0));
      v[2] = TC(__low2float(h1)); v[3] = TC(__high2float(h1));
    } else if (dt == EMMY_DT_F64) {
      const double2 *q = reinterpret_cast<const double2 *>(static_cast<const double *>(p) + i);
      const double2 x0 = q[0], x1 = q[1];
      v[0] = TC(x0.x); v[1] = TC(x0.y); v[2] = TC(x1.x); v[3] = TC(x1.y);
    } else {
      const float4 x = *reinterpret_cast<const float4 *>(static_cast<const float *>(p) + i);
      v[0] = TC(x.x); v[1] = TC(x.y); v[2] = TC(x.z); v[3] = TC(x.w);
    }
  }
}

template <typename TC, int VEC>
__device__ __forceinline__ void stv(void *p, int dt, int64_t i, const TC v[VEC]) {
  if constexpr (VEC == 1) {
    st<TC>(p, dt, i, v[0]);
  } else {
    if (dt == EMMY_DT_F16) {
      __half2 h0 = __halves2half2(to_half(v[0]), to_half(v[1]));
      __half2 h1 = __halves2half2(to_half(v[2]), to_half(v[3]));
      uint2 u;
      u.x = *reinterpret_cast<unsigned *>(&h0);
      u.y = *reinterpret_cast<unsigned *>(&h1);
      *reinterpret_cast<uint2 *>(static_cast<__half *>(p) + i) = u;
    } else if (dt == EMMY_DT_F64) {
      double2 *q = reinterpret_cast<double2 *>(static_cast<double *>(p) + i);
      q[0] = make_double2(double(v[0]), double(v[1]));
      q[1] = make_double2(double(v[2]), double(v[3]));
    } else {
      *reinterpret_cast<float4 *>(static_cast<float *>(p) + i) =
          make_float4(float(v[0]), float(v[1]), float(v[2]), float(v[3]));
    }
  }
}

// inner == 1: TPR threads per row (a warp, 8 rows per block; or the block),
// VEC elements per thread per step
template <typename TC, int MODE, int TPR, int VEC>
__global__ void __launch_bounds__(256) rows_kernel(const Args a) {
  constexpr int RPB = TPR > 32 ? 1 : 256 / 32;
  __shared__ TC red[32];
  const int g = TPR > 32 ? 0 : (threadIdx.x >> 5);
  const int t = TPR > 32 ? threadIdx.x : (threadIdx.x & 31);
  const int64_t n = a.n;
  const int64_t i0 = (int64_t)t * VEC, step = (int64_t)TPR * VEC;
  TC eps = TC(0), inv_count = TC(0);
  if (a.eps) eps = ld<TC>(a.eps, a.cdt, 0);
  if (a.count) inv_count = TC(1) / ld<TC>(a.count, a.cdt, 0);
  else inv_count = TC(1) / TC(n);
  for (int64_t row = (int64_t)blockIdx.x * RPB + g; row < a.outer;
       row += (int64_t)gridDim.x * RPB) {
    const int64_t base = row * n;
    TC v[VEC];
    if constexpr (MODE == M_SUM || MODE == M_MAX || MODE == M_MIN) {
      TC acc = seed<MODE, TC>();
      for (int64_t i = i0; i < n; i += step) {
        ldv<TC, VEC>(a.x, a.xdt, base + i, v);
#pragma unroll
        for (int j = 0; j < VEC; ++j) acc = fold<MODE, TC>(acc, v[j], a.pre);
      }
      acc = group<MODE, TPR, TC>(acc, red);
      if (t == 0) st<TC>(a.y, a.ydt, row, a.count ? acc * inv_count : acc);
    } else if constexpr (MODE == M_DOT) {
      TC acc = TC(0), u[VEC];
      for (int64_t i = i0; i < n; i += step) {
        ldv<TC, VEC>(a.x, a.xdt, base + i, v);
        ldv<TC, VEC>(a.w, a.wdt, i, u);
#pragma unroll
        for (int j = 0; j < VEC; ++j) acc = fma_c(v[j], u[j], acc);
      }
      acc = group<M_SUM, TPR, TC>(acc, red);
      if (t == 0) st<TC>(a.y, a.ydt, row, acc);
    } else if constexpr (MODE == M_SOFTMAX) {
      TC m = max_seed<TC>();
      for (int64_t i = i0; i < n; i += step) {
        ldv<TC, VEC>(a.x, a.xdt, base + i, v);
#pragma unroll
        for (int j = 0; j < VEC; ++j) m = fmax(m, v[j]);
      }
      m = group<M_MAX, TPR, TC>(m, red);
      TC s = TC(0);
      for (int64_t i = i0; i < n; i += step) {
        ldv<TC, VEC>(a.x, a.xdt, base + i, v);
#pragma unroll
        for (int j = 0; j < VEC; ++j) s += exp_c(v[j] - m);
      }
      s = group<M_SUM, TPR, TC>(s, red);
      const TC r = TC(1) / s;
      for (int64_t i = i0; i < n; i += step) {
        ldv<TC, VEC>(a.x, a.xdt, base + i, v);
#pragma unroll
        for (int j = 0; j < VEC; ++j) v[j] = exp_c(v[j] - m) * r;
        stv<TC, VEC>(a.y, a.ydt, base + i, v);
      }
    } else if constexpr (MODE == M_RMS || MODE == M_L2) {
      TC s = TC(0), u[VEC];
      for (int64_t i = i0; i < n; i += step) {
        ldv<TC, VEC>(a.x, a.xdt, base + i, v);
#pragma unroll
        for (int j = 0; j < VEC; ++j) s = fma_c(v[j], v[j], s);
      }
      s = group<M_SUM, TPR, TC>(s, red);
      const TC r = MODE == M_RMS ? TC(1) / sqrt(eps + s * inv_count) : TC(1) / sqrt(s);
      for (int64_t i = i0; i < n; i += step) {
        ldv<TC, VEC>(a.x, a.xdt, base + i, v);
#pragma unroll
        for (int j = 0; j < VEC; ++j) v[j] = v[j] * r;
        if (MODE == M_RMS && a.w) {
          ldv<TC, VEC>(a.w, a.wdt, i, u);
#pragma unroll
          for (int j = 0; j < VEC; ++j) v[j] *= u[j];
        }
        stv<TC, VEC>(a.y, a.ydt, base + i, v);
      }
    } else {  // M_LN: mean, then the centred variance
      TC s = TC(0), u[VEC];
      for (int64_t i = i0; i < n; i += step) {
        ldv<TC, VEC>(a.x, a.xdt, base + i, v);
#pragma unroll
        for (int j = 0; j < VEC; ++j) s += v[j];
      }
      s = group<M_SUM, TPR, TC>(s, red);
      const TC mean = s * inv_count;
      TC q = TC(0);
      for (int64_t i = i0; i < n; i += step) {
        ldv<TC, VEC>(a.x, a.xdt, base + i, v);
#pragma unroll
        for (int j = 0; j < VEC; ++j) {
          const TC d = v[j] - mean;
          q = fma_c(d, d, q);
        }
      }
      q = group<M_SUM, TPR, TC>(q, red);
      const TC r = TC(1) / sqrt(q * inv_count + eps);
      for (int64_t i = i0; i < n; i += step) {
        ldv<TC, VEC>(a.x, a.xdt, base + i, v);
#pragma unroll
        for (int j = 0; j < VEC; ++j) v[j] = (v[j] - mean) * r;
        if (a.w) {
          ldv<TC, VEC>(a.w, a.wdt, i, u);
#pragma unroll
          for (int j = 0; j < VEC; ++j) v[j] *= u[j];
        }
        if (a.b) {
          ldv<TC, VEC>(a.b, a.wdt, i, u);
#pragma unroll
          for (int j = 0; j < VEC; ++j) v[j] += u[j];
        }
        stv<TC, VEC>(a.y, a.ydt, base + i, v);
      }
    }
  }
}

// inner > 1: one thread per (outer, inner) column; reductions and softmax
template <typename TC, int MODE>
__global__ void __launch_bounds__(256) cols_kernel(const Args a) {
  const int64_t total = a.outer * a.inner, n = a.n, inner = a.inner;
  TC inv_count = TC(0);
  if (a.count) inv_count = TC(1) / ld<TC>(a.count, a.cdt, 0);
  for (int64_t c = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; c < total;
       c += (int64_t)gridDim.x * blockDim.x) {
    const int64_t o = c / inner, i = c - o * inner;
    const int64_t base = o * n * inner + i;
    if constexpr (MODE == M_SOFTMAX) {
      TC m = max_seed<TC>();
      for (int64_t j = 0; j < n; ++j) m = fmax(m, ld<TC>(a.x, a.xdt, base + j * inner));
      TC s = TC(0);
      for (int64_t j = 0; j < n; ++j) s += exp_c(ld<TC>(a.x, a.xdt, base + j * inner) - m);
      const TC r = TC(1) / s;
      for (int64_t j = 0; j < n; ++j)
        st<TC>(a.y, a.ydt, base + j * inner, exp_c(ld<TC>(a.x, a.xdt, base + j * inner) - m) * r);
    } else {
      TC acc = seed<MODE, TC>();
      for (int64_t j = 0; j < n; ++j) acc = fold<MODE, TC>(acc, ld<TC>(a.x, a.xdt, base + j * inner), a.pre);
      st<TC>(a.y, a.ydt, c, a.count ? acc * inv_count : acc);
    }
  }
}

// f16 rows of 256 * CH * WPR elements held in registers, for softmax and
// rms / layer normalisation: WPR warps per row (one, or two for the longest
// rows, which would otherwise need ~180 registers a thread), each lane CH
// 16-byte pieces (8 halves) at piece lane + 32 k of its warp's part of the
// row, so the row is read from memory once (the kernel above reads it two or
// three times).  Same arithmetic as the kernel above in f32 (softmax: the max
// from the reference's -1e30 seed, e^(x - max), one correctly rounded
// 1 / sum; rms: 1 / sqrt(eps + sum(x^2) / n); layer norm: the mean, then
// the centred variance; weight and bias in their own dtype), rounded once to
// f16 at the store; only the summation order differs.
template <int MODE, int CH, int WPR>
__global__ void __launch_bounds__(256) rows_f16_resident_kernel(const Args a) {
  constexpr int N = 256 * CH * WPR, RPB = 8 / WPR;
  __shared__ float red[2][8];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int rib = warp / WPR, part = warp % WPR;      // row in block, part of the row
  const __half *x = static_cast<const __half *>(a.x);
  __half *y = static_cast<__half *>(a.y);
  float eps = 0.f, inv_count;
  if (a.eps) eps = ld<float>(a.eps, a.cdt, 0);
  if (a.count) inv_count = 1.0f / ld<float>(a.count, a.cdt, 0);
  else inv_count = 1.0f / float(N);
  int rcount = 0;                                     // reductions so far: exchange slot parity
  // a row's max or sum over its WPR warps, the same value in each.  Slots
  // alternate, so a slot is rewritten only after a barrier that every thread
  // passes once it has read the slot's previous value.
  auto allreduce = [&](float v, bool is_max) -> float {
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) {
      const float w = __shfl_xor_sync(0xffffffffu, v, o);
      v = is_max ? fmaxf(v, w) : v + w;
    }
    if constexpr (WPR > 1) {
      const int slot = rcount & 1;
      if (lane == 0) red[slot][warp] = v;
      __syncthreads();
      v = red[slot][rib * WPR];
#pragma unroll
      for (int w = 1; w < WPR; ++w)
        v = is_max ? fmaxf(v, red[slot][rib * WPR + w]) : v + red[slot][rib * WPR + w];
    }
    ++rcount;
    return v;
  };
  // every thread of the block runs the same number of iterations (the
  // barriers in allreduce), rows past the end doing no memory work
  for (int64_t r0 = (int64_t)blockIdx.x * RPB; r0 < a.outer; r0 += (int64_t)gridDim.x * RPB) {
    const int64_t row = r0 + rib;
    const bool live = row < a.outer;
    const int64_t piece0 = (int64_t)part * 32 * CH;   // this warp's first 8-element piece
    const uint4 *src = reinterpret_cast<const uint4 *>(x + row * N) + piece0;
    uint4 v[CH];
#pragma unroll
    for (int k = 0; k < CH; ++k) v[k] = live ? src[lane + 32 * k] : make_uint4(0, 0, 0, 0);
    float sc = 1.f, sh = 0.f;                         // y = x * sc - sh, before weight and bias
    if constexpr (MODE == M_SOFTMAX) {
      float m = max_seed<float>();
#pragma unroll
      for (int k = 0; k < CH; ++k) {
        const __half2 *h = reinterpret_cast<const __half2 *>(&v[k]);
#pragma unroll
        for (int q = 0; q < 4; ++q) m = fmaxf(m, fmaxf(__low2float(h[q]), __high2float(h[q])));
      }
      m = allreduce(m, true);
      const uint64_t c2 = pk2(1.4426950408889634f, 1.4426950408889634f), m2 = pk2(m, m);
      uint64_t s2[2] = {0ull, 0ull};
#pragma unroll
      for (int k = 0; k < CH; ++k) {
        const __half2 *h = reinterpret_cast<const __half2 *>(&v[k]);
#pragma unroll
        for (int q = 0; q < 4; ++q) s2[q & 1] = add2(s2[q & 1], exp_pair(h[q], m2, c2));
      }
      float s0, s1;
      upk2(add2(s2[0], s2[1]), s0, s1);
      const float s = allreduce(s0 + s1, false);
      sc = 1.0f / s;
      sh = m;                                         // softmax: e^(x - sh) * sc
    } else if constexpr (MODE == M_RMS) {
      float s = 0.f;
#pragma unroll
      for (int k = 0; k < CH; ++k) {
        const __half2 *h = reinterpret_cast<const __half2 *>(&v[k]);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float lo = __low2float(h[q]), hi = __high2float(h[q]);
          s = fmaf(lo, lo, s);
          s = fmaf(hi, hi, s);
        }
      }
      s = allreduce(s, false);
      sc = 1.0f / sqrtf(eps + s * inv_count);
    } else {                                          // M_LN
      float s = 0.f;
#pragma unroll
      for (int k = 0; k < CH; ++k) {
        const __half2 *h = reinterpret_cast<const __half2 *>(&v[k]);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          s += __low2float(h[q]);
          s += __high2float(h[q]);
        }
      }
      s = allreduce(s, false);
      const float mean = s * inv_count;
      float qv = 0.f;
#pragma unroll
      for (int k = 0; k < CH; ++k) {
        const __half2 *h = reinterpret_cast<const __half2 *>(&v[k]);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float d0 = __low2float(h[q]) - mean, d1 = __high2float(h[q]) - mean;
          qv = fmaf(d0, d0, qv);
          qv = fmaf(d1, d1, qv);
        }
      }
      qv = allreduce(qv, false);
      sc = 1.0f / sqrtf(qv * inv_count + eps);
      sh = mean;                                      // layer norm: (x - sh) * sc
    }
    if (live) {
      uint4 *dst = reinterpret_cast<uint4 *>(y + row * N) + piece0;
#pragma unroll
      for (int k = 0; k < CH; ++k) {
        const __half2 *h = reinterpret_cast<const __half2 *>(&v[k]);
        float o[8];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float lo = __low2float(h[q]), hi = __high2float(h[q]);
          if constexpr (MODE == M_SOFTMAX) {
            float p0, p1;
            upk2(exp_pair(h[q], pk2(sh, sh), pk2(1.4426950408889634f, 1.4426950408889634f)), p0,
                 p1);
            o[2 * q] = p0 * sc;
            o[2 * q + 1] = p1 * sc;
            (void)lo;
            (void)hi;
          } else if constexpr (MODE == M_RMS) {
            o[2 * q] = lo * sc;
            o[2 * q + 1] = hi * sc;
          } else {
            o[2 * q] = (lo - sh) * sc;
            o[2 * q + 1] = (hi - sh) * sc;
          }
        }
        if constexpr (MODE != M_SOFTMAX) {
          const int64_t e = (piece0 + lane + 32 * k) * 8;   // element index in the row
          float u[4];
          if (a.w) {
            ldv<float, 4>(a.w, a.wdt, e, u);
#pragma unroll
            for (int j = 0; j < 4; ++j) o[j] *= u[j];
            ldv<float, 4>(a.w, a.wdt, e + 4, u);
#pragma unroll
            for (int j = 0; j < 4; ++j) o[4 + j] *= u[j];
          }
          if (MODE == M_LN && a.b) {
            ldv<float, 4>(a.b, a.wdt, e, u);
#pragma unroll
            for (int j = 0; j < 4; ++j) o[j] += u[j];
            ldv<float, 4>(a.b, a.wdt, e + 4, u);
#pragma unroll
            for (int j = 0; j < 4; ++j) o[4 + j] += u[j];
          }
        }
        uint4 w;
        uint32_t *wq = reinterpret_cast<uint32_t *>(&w);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          __half2 hh = __floats2half2_rn(o[2 * q], o[2 * q + 1]);
          wq[q] = *reinterpret_cast<uint32_t *>(&hh);
        }
        dst[lane + 32 * k] = w;
      }
    }
  }
}

template <typename TC, int MODE>
void launch(const Args &a, cudaStream_t st) {
  const int sms = sm_count();
  if (a.inner > 1) {
    if constexpr (MODE == M_SUM || MODE == M_MAX || MODE == M_MIN || MODE == M_SOFTMAX) {
      int64_t blocks = (a.outer * a.inner + 255) / 256;
      if (blocks > (int64_t)sms * 32) blocks = (int64_t)sms * 32;
      cols_kernel<TC, MODE><<<(unsigned)blocks, 256, 0, st>>>(a);
    }
    return;
  }
  if constexpr ((MODE == M_SOFTMAX || MODE == M_RMS || MODE == M_LN) && sizeof(TC) == 4) {
    // f16 in and out, rows of 512, 1024, 2048 (and 4096 for softmax)
    // elements: the row in registers (weight and bias, when present, aligned
    // for 4-element loads)
    const int64_t ch = a.n / 256;
    auto wal = [&](const void *ptr) {
      const uintptr_t need = a.wdt == EMMY_DT_F16 ? 8 : (a.wdt == EMMY_DT_F64 ? 32 : 16);
      return ptr == nullptr || (reinterpret_cast<uintptr_t>(ptr) % need) == 0;
    };
    // (the norms' two-warp 4096 form needs 200+ registers and ran slower than
    // the general kernel: norms up to 2048)
    const bool ch_ok = ch == 2 || ch == 4 || ch == 8 || (ch == 16 && MODE == M_SOFTMAX);
    if (a.xdt == EMMY_DT_F16 && a.ydt == EMMY_DT_F16 && a.n % 256 == 0 && ch_ok &&
        aligned16(a.x) && aligned16(a.y) && wal(a.w) && wal(a.b)) {
      const int rpb = ch == 16 ? 4 : 8;                 // 4096: two warps per row
      int64_t blocks = (a.outer + rpb - 1) / rpb;
      if (blocks > (int64_t)sms * 16) blocks = (int64_t)sms * 16;
      switch (ch) {
        case 2: rows_f16_resident_kernel<MODE, 2, 1><<<(unsigned)blocks, 256, 0, st>>>(a); break;
        case 4: rows_f16_resident_kernel<MODE, 4, 1><<<(unsigned)blocks, 256, 0, st>>>(a); break;
        case 8: rows_f16_resident_kernel<MODE, 8, 1><<<(unsigned)blocks, 256, 0, st>>>(a); break;
        default:
          if constexpr (MODE == M_SOFTMAX)
            rows_f16_resident_kernel<MODE, 8, 2><<<(unsigned)blocks, 256, 0, st>>>(a);
          break;
      }
      return;
    }
  }
  // 4 elements per access when every row start is aligned for it
  auto al = [](const void *ptr, int dt) {
    const uintptr_t need = dt == EMMY_DT_F16 ? 8 : 16;
    return ptr == nullptr || (reinterpret_cast<uintptr_t>(ptr) % need) == 0;
  };
  const bool v4 = a.n % 4 == 0 && al(a.x, a.xdt) && al(a.y, a.ydt) && al(a.w, a.wdt) &&
                  al(a.b, a.wdt);
  const bool warp_rows = a.n <= (v4 ? 8192 : 2048);
  int64_t blocks = warp_rows ? (a.outer + 7) / 8 : a.outer;
  const int64_t cap = (int64_t)sms * (warp_rows ? 32 : 8);
  if (blocks > cap) blocks = cap;
#define EMMY_ROWT(TPR, V) rows_kernel<TC, MODE, TPR, V><<<(unsigned)blocks, 256, 0, st>>>(a)
  if (warp_rows) {
    if (v4) EMMY_ROWT(32, 4);
    else EMMY_ROWT(32, 1);
  } else {
    if (v4) EMMY_ROWT(256, 4);
    else EMMY_ROWT(256, 1);
  }
#undef EMMY_ROWT
}

template <typename TC>
void dispatch(const Args &a, int mode, cudaStream_t st) {
  switch (mode) {
    case M_SUM: launch<TC, M_SUM>(a, st); break;
    case M_MAX: launch<TC, M_MAX>(a, st); break;
    case M_MIN: launch<TC, M_MIN>(a, st); break;
    case M_SOFTMAX: launch<TC, M_SOFTMAX>(a, st); break;
    case M_RMS: launch<TC, M_RMS>(a, st); break;
    case M_L2: launch<TC, M_L2>(a, st); break;
    case M_LN: launch<TC, M_LN>(a, st); break;
    default: launch<TC, M_DOT>(a, st); break;
  }
}

}  // namespace rowt
}  // namespace emmy

using namespace emmy;

extern "C" int emmy_rowop(const void *x, int x_dtype, const void *w, const void *b, int wb_dtype,
                          void *y, int y_dtype, int64_t outer, int64_t n, int64_t inner, int mode,
                          int pre, const void *eps, const void *count, int const_dtype,
                          int compute_f64, void *stream) {
  using namespace rowt;
  clear_error();
  auto dt_ok = [](int dt) { return dt == EMMY_DT_F32 || dt == EMMY_DT_F16 || dt == EMMY_DT_F64; };
  if (outer < 0 || n < 0 || inner < 1) return set_error(EMMY_ERR_INVALID, "emmy_rowop: bad view");
  if (outer == 0) return EMMY_OK;
  if (n < 1) return set_error(EMMY_ERR_INVALID, "emmy_rowop: empty rows");
  if (!x || !y) return set_error(EMMY_ERR_INVALID, "emmy_rowop: null tensor");
  if (!dt_ok(x_dtype) || !dt_ok(y_dtype) || ((w || b) && !dt_ok(wb_dtype)) ||
      ((eps || count) && !dt_ok(const_dtype)))
    return set_error(EMMY_ERR_INVALID, "emmy_rowop: bad dtype");
  if (mode < M_SUM || mode > M_DOT) return set_error(EMMY_ERR_INVALID, "emmy_rowop: bad mode %d", mode);
  if (pre < EMMY_PRE_IDENTITY || pre > EMMY_PRE_ABS || (pre && mode > M_MIN))
    return set_error(EMMY_ERR_INVALID, "emmy_rowop: bad pre-map %d", pre);
  if (mode == M_DOT && !w) return set_error(EMMY_ERR_INVALID, "emmy_rowop: dot without a vector");
  if (inner > 1 && mode > M_SOFTMAX)
    return set_error(EMMY_ERR_UNSUPPORTED, "emmy_rowop: mode %d over a strided axis", mode);
  if (outer > INT64_MAX / n / inner) return set_error(EMMY_ERR_INVALID, "emmy_rowop: view overflows");
  Args a{};
  a.x = x; a.w = w; a.b = b; a.y = y; a.eps = eps; a.count = count;
  a.xdt = x_dtype; a.wdt = wb_dtype; a.ydt = y_dtype; a.cdt = const_dtype;
  a.pre = pre;
  a.outer = outer; a.n = n; a.inner = inner;
  cudaStream_t st = as_stream(stream);
  if (compute_f64) dispatch<double>(a, mode, st);
  else dispatch<float>(a, mode, st);
  return check_launch("emmy_rowop");
}
