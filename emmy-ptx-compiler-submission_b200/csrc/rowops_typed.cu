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
// tensors; this one trades 128-bit vector loads for dtype generality: loads
// are per element, coalesced across the threads of a row, and the statistics
// pass re-reads the row from L1/L2 for the map pass.
//
// Layout: x viewed as [outer, n, inner] row-major.  inner == 1: a warp per row
// (n <= 2048) or a 256-thread block per row; inner > 1 (reductions and
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

// inner == 1: TPR threads per row (a warp, 8 rows per block; or the block)
template <typename TC, int MODE, int TPR>
__global__ void __launch_bounds__(256) rows_kernel(const Args a) {
  constexpr int RPB = TPR > 32 ? 1 : 256 / 32;
  __shared__ TC red[32];
  const int g = TPR > 32 ? 0 : (threadIdx.x >> 5);
  const int t = TPR > 32 ? threadIdx.x : (threadIdx.x & 31);
  const int64_t n = a.n;
  TC eps = TC(0), inv_count = TC(0);
  if (a.eps) eps = ld<TC>(a.eps, a.cdt, 0);
  if (a.count) inv_count = TC(1) / ld<TC>(a.count, a.cdt, 0);
  else inv_count = TC(1) / TC(n);
  for (int64_t row = (int64_t)blockIdx.x * RPB + g; row < a.outer;
       row += (int64_t)gridDim.x * RPB) {
    const int64_t base = row * n;
    if constexpr (MODE == M_SUM || MODE == M_MAX || MODE == M_MIN) {
      TC acc = seed<MODE, TC>();
      for (int64_t i = t; i < n; i += TPR) acc = fold<MODE, TC>(acc, ld<TC>(a.x, a.xdt, base + i), a.pre);
      acc = group<MODE, TPR, TC>(acc, red);
      if (t == 0) st<TC>(a.y, a.ydt, row, a.count ? acc * inv_count : acc);
    } else if constexpr (MODE == M_DOT) {
      TC acc = TC(0);
      for (int64_t i = t; i < n; i += TPR)
        acc = fma_c(ld<TC>(a.x, a.xdt, base + i), ld<TC>(a.w, a.wdt, i), acc);
      acc = group<M_SUM, TPR, TC>(acc, red);
      if (t == 0) st<TC>(a.y, a.ydt, row, acc);
    } else if constexpr (MODE == M_SOFTMAX) {
      TC m = max_seed<TC>();
      for (int64_t i = t; i < n; i += TPR) m = fmax(m, ld<TC>(a.x, a.xdt, base + i));
      m = group<M_MAX, TPR, TC>(m, red);
      TC s = TC(0);
      for (int64_t i = t; i < n; i += TPR) s += exp_c(ld<TC>(a.x, a.xdt, base + i) - m);
      s = group<M_SUM, TPR, TC>(s, red);
      const TC r = TC(1) / s;
      for (int64_t i = t; i < n; i += TPR)
        st<TC>(a.y, a.ydt, base + i, exp_c(ld<TC>(a.x, a.xdt, base + i) - m) * r);
    } else if constexpr (MODE == M_RMS || MODE == M_L2) {
      TC s = TC(0);
      for (int64_t i = t; i < n; i += TPR) {
        const TC v = ld<TC>(a.x, a.xdt, base + i);
        s = fma_c(v, v, s);
      }
      s = group<M_SUM, TPR, TC>(s, red);
      const TC r = MODE == M_RMS ? TC(1) / sqrt(eps + s * inv_count) : TC(1) / sqrt(s);
      for (int64_t i = t; i < n; i += TPR) {
        TC o = ld<TC>(a.x, a.xdt, base + i) * r;
        if (MODE == M_RMS && a.w) o *= ld<TC>(a.w, a.wdt, i);
        st<TC>(a.y, a.ydt, base + i, o);
      }
    } else {  // M_LN: mean, then the centred variance
      TC s = TC(0);
      for (int64_t i = t; i < n; i += TPR) s += ld<TC>(a.x, a.xdt, base + i);
      s = group<M_SUM, TPR, TC>(s, red);
      const TC mean = s * inv_count;
      TC q = TC(0);
      for (int64_t i = t; i < n; i += TPR) {
        const TC d = ld<TC>(a.x, a.xdt, base + i) - mean;
        q = fma_c(d, d, q);
      }
      q = group<M_SUM, TPR, TC>(q, red);
      const TC r = TC(1) / sqrt(q * inv_count + eps);
      for (int64_t i = t; i < n; i += TPR) {
        TC o = (ld<TC>(a.x, a.xdt, base + i) - mean) * r;
        if (a.w) o *= ld<TC>(a.w, a.wdt, i);
        if (a.b) o += ld<TC>(a.b, a.wdt, i);
        st<TC>(a.y, a.ydt, base + i, o);
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
  if (a.n <= 2048) {
    int64_t blocks = (a.outer + 7) / 8;
    if (blocks > (int64_t)sms * 32) blocks = (int64_t)sms * 32;
    rows_kernel<TC, MODE, 32><<<(unsigned)blocks, 256, 0, st>>>(a);
  } else {
    int64_t blocks = a.outer;
    if (blocks > (int64_t)sms * 8) blocks = (int64_t)sms * 8;
    rows_kernel<TC, MODE, 256><<<(unsigned)blocks, 256, 0, st>>>(a);
  }
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
