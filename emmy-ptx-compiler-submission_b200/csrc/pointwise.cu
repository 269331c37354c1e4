// Pointwise (elementwise) family on sm_100a: out[i] = f(in_0[i], ..., scalars, immediates).
//
// Replaces the entry the reference emits for its pointwise IR shape: one
// thread per 1-4 elements, each element a chain of Loads, Assigns and a
// converting Write (reference ptxc/stmts.py:73-145 Load, :510-560 Assign,
// :434-487 Write; op spellings ptxc/expr.py:880-1089 and ptxc/ops.py:81-96).
// add/sub/mul/div/sqrt are rounded per op with no contraction, so chains the
// reference checks with rtol = atol = 0 stay bit-exact.  An f16-typed Assign
// computes in f32 and rounds to f16 (the matcher adds a round_f16 step).
//
// The matcher hands over the element's expression as a register program; one
// kernel evaluates it for every element.  The register file lives in shared
// memory (lane j of register r of thread t at [(r*VEC + j)*THREADS + t], no
// bank conflicts), scalar constants and immediates are written once per
// thread, and each instruction is decoded once per VEC elements.  Inputs and
// the output move as 16-byte (f32, f64) or 8-byte (f16) vectors when every
// pointer allows it; HBM traffic is then the algorithmic minimum.

#include <algorithm>

#include "common.cuh"
#include "pw_index.cuh"

namespace emmy {

constexpr int kPwMaxRegs = 32, kPwMaxInstr = 48, kPwMaxIn = 8, kPwThreads = 256;
constexpr int kPwSimpleGroups = 2;     // most 4-element groups per thread in the register kernel

enum PwOp {
  PW_COPY = 0, PW_ADD, PW_SUB, PW_MUL, PW_DIV, PW_MAX, PW_MIN, PW_NEG, PW_ABS, PW_EXP, PW_LOG,
  PW_SQRT, PW_RSQRT, PW_RECIP, PW_TANH, PW_SIGMOID, PW_RELU, PW_GT, PW_LT, PW_GE, PW_LE, PW_EQ,
  PW_WHERE, PW_ROUND_F16, PW_FMA, PW_LOG2, PW_LOG10, PW_COS, PW_SIN, PW_TAN, PW_ERF, PW_GELU,
  PW_GELU_TANH, PW_SOFTPLUS, PW_EXP2, PW_SILU, PW_POW, PW_FLOOR, PW_CEIL, PW_SIGN, PW_NE, PW_NOPS
};

struct PwProgram {
  PwIndex idx[kPwMaxIn];
  long long first;
  const void *inputs[kPwMaxIn];
  const void *scalars[kPwMaxIn];
  int in_dtype[kPwMaxIn];
  int sc_dtype[kPwMaxIn];
  double imm[kPwMaxIn];
  int n_in, n_sc, n_imm, n_instr, result_reg;
  signed char code[kPwMaxInstr][5];
};

// Correctly rounded arithmetic in both compute precisions (no FMA contraction).
__device__ __forceinline__ float add_rn(float a, float b) { return __fadd_rn(a, b); }
__device__ __forceinline__ double add_rn(double a, double b) { return __dadd_rn(a, b); }
__device__ __forceinline__ float sub_rn(float a, float b) { return __fsub_rn(a, b); }
__device__ __forceinline__ double sub_rn(double a, double b) { return __dsub_rn(a, b); }
__device__ __forceinline__ float mul_rn(float a, float b) { return __fmul_rn(a, b); }
__device__ __forceinline__ double mul_rn(double a, double b) { return __dmul_rn(a, b); }
__device__ __forceinline__ float div_rn(float a, float b) { return __fdiv_rn(a, b); }
__device__ __forceinline__ double div_rn(double a, double b) { return __ddiv_rn(a, b); }
__device__ __forceinline__ float fma_rn(float a, float b, float c) { return __fmaf_rn(a, b, c); }
__device__ __forceinline__ double fma_rn(double a, double b, double c) { return __fma_rn(a, b, c); }
__device__ __forceinline__ float sqrt_rn(float a) { return __fsqrt_rn(a); }
__device__ __forceinline__ double sqrt_rn(double a) { return __dsqrt_rn(a); }

// Ops whose library code is long stay out of line, so the dispatch below
// keeps a small instruction footprint.
template <typename T> __device__ __noinline__ T pw_slow(int op, T a, T b) {
  const T one = T(1), half = T(0.5);
  switch (op) {
    case PW_LOG2: return log2(a);
    case PW_LOG10: return log10(a);
    case PW_COS: return cos(a);
    case PW_SIN: return sin(a);
    case PW_TAN: return tan(a);
    case PW_ERF: return erf(a);
    case PW_GELU:        // x/2 * (1 + erf(x / sqrt 2))
      return mul_rn(mul_rn(half, a), add_rn(one, erf(mul_rn(a, T(0.7071067811865476)))));
    case PW_POW: return pow(a, b);
    case PW_SOFTPLUS: return add_rn(fmax(a, T(0)), log1p(exp(-fabs(a))));
    default: return T(0);
  }
}

// gelu with the tanh form in f32: x/2 * (1 + tanh(u)) = x / (1 + e^(-2u)),
// u = sqrt(2/pi) * (x + 0.044715 x^3).  One exponential (ex2) and one fast
// division instead of a tanh; no cancellation anywhere (1 + e^(-2u) >= 1).
// Relative error about |2u| * 2^-24 from the exponent's argument plus a few
// ulp, ~1e-6 where the result is not negligible, well inside the f32
// tolerance of the tanh form (the reference's own tanh is an approximation
// too: a Pade form near zero and the exp identity outside).  Limits: x = +inf
// gives +inf, x = -inf NaN (as the tanh form), x very negative 0.
__device__ __forceinline__ float gelu_tanh_f32(float x) {
  const float t = fmaf(0.044715f, __fmul_rn(__fmul_rn(x, x), x), x);
  const float e = __expf(-1.5957691216057308f * t);   // e^(-2 sqrt(2/pi) t)
  return __fdividef(x, 1.0f + e);
}

// gelu (tanh form) of a pair, the steps of gelu_tanh_f32 on packed f32x2
// lanes (each lane rounded as its scalar form; sm_100 mul / fma / add
// .f32x2), the exponential and the reciprocal on MUFU with subnormal results
// flushed: e < 2^-126 leaves 1 + e = 1 either way, and x / (1 + e) below
// 2^-126 rounds to 0 in any f16 output.
__device__ __forceinline__ uint64_t pk2(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void upk2(uint64_t r, float &lo, float &hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(r));
}
__device__ __forceinline__ uint64_t mul2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t fma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
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
__device__ __forceinline__ float rcp_ftz(float a) {
  float r;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(a));
  return r;
}
__device__ __forceinline__ uint64_t gelu_tanh_f32x2(uint64_t x) {
  const uint64_t t = fma2(pk2(0.044715f, 0.044715f), mul2(mul2(x, x), x), x);
  const uint64_t a = mul2(mul2(t, pk2(-1.5957691216057308f, -1.5957691216057308f)),
                          pk2(1.4426950408889634f, 1.4426950408889634f));
  float a0, a1;
  upk2(a, a0, a1);
  float d0, d1;
  upk2(add2(pk2(ex2_ftz(a0), ex2_ftz(a1)), pk2(1.0f, 1.0f)), d0, d1);
  return mul2(x, pk2(rcp_ftz(d0), rcp_ftz(d1)));
}

// One-step gelu (tanh form) on a contiguous f16 input with an f16 output: 8
// elements per 16-byte load and store, GS groups per thread loaded before any
// is computed, the pairs through gelu_tanh_f32x2.  n8 groups of 8.
template <int GS>
__global__ void __launch_bounds__(256)
gelu_tanh_f16x8_kernel(const uint4 *__restrict__ x, uint4 *__restrict__ y, int64_t n8) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t g0 = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; g0 < n8; g0 += GS * stride) {
    uint4 in[GS];
#pragma unroll
    for (int u = 0; u < GS; ++u) {
      const int64_t g = g0 + u * stride;
      if (g < n8) in[u] = __ldcs(x + g);
    }
#pragma unroll
    for (int u = 0; u < GS; ++u) {
      const int64_t g = g0 + u * stride;
      if (g >= n8) break;
      const uint32_t w[4] = {in[u].x, in[u].y, in[u].z, in[u].w};
      uint32_t o[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float2 f = __half22float2(*reinterpret_cast<const __half2 *>(&w[k]));
        float lo, hi;
        upk2(gelu_tanh_f32x2(pk2(f.x, f.y)), lo, hi);
        const __half2 h = __floats2half2_rn(lo, hi);
        o[k] = *reinterpret_cast<const uint32_t *>(&h);
      }
      __stcs(y + g, make_uint4(o[0], o[1], o[2], o[3]));
    }
  }
}

// One program step over the VEC lanes of this thread: RD[j*S] = op(RA[j*S], ...),
// S the lane stride (the shared-memory register file's, or 1 for registers).
template <typename T, int VEC, int S = kPwThreads>
__device__ __forceinline__ void pw_step(int op, T *RD, const T *RA, const T *RB, const T *RC) {
  const T zero = T(0), one = T(1), half = T(0.5);
#define PW_LANES(EXPR)                                                              \
  _Pragma("unroll") for (int j = 0; j < VEC; ++j) {                                 \
    const T a = RA[j * S], b = RB[j * S], c = RC[j * S];                            \
    (void)b; (void)c;                                                               \
    RD[j * S] = (EXPR);                                                             \
  }                                                                                 \
  break;
  switch (op) {
    case PW_COPY: PW_LANES(a)
    case PW_ADD: PW_LANES(add_rn(a, b))
    case PW_SUB: PW_LANES(sub_rn(a, b))
    case PW_MUL: PW_LANES(mul_rn(a, b))
    case PW_DIV: PW_LANES(div_rn(a, b))
    case PW_MAX: PW_LANES(fmax(a, b))       // maxNum, as max.f32 in the reference
    case PW_MIN: PW_LANES(fmin(a, b))
    case PW_NEG: PW_LANES(-a)
    case PW_ABS: PW_LANES(fabs(a))
    case PW_EXP: PW_LANES(exp(a))
    case PW_LOG: PW_LANES(log(a))
    case PW_SQRT: PW_LANES(sqrt_rn(a))
    case PW_RSQRT: PW_LANES(rsqrt(a))
    case PW_RECIP: PW_LANES(div_rn(one, a))
    case PW_TANH: PW_LANES(tanh(a))
    case PW_SIGMOID: PW_LANES(div_rn(one, add_rn(one, exp(-a))))
    case PW_RELU: PW_LANES(fmax(a, zero))
    case PW_GT: PW_LANES(a > b ? one : zero)
    case PW_LT: PW_LANES(a < b ? one : zero)
    case PW_GE: PW_LANES(a >= b ? one : zero)
    case PW_LE: PW_LANES(a <= b ? one : zero)
    case PW_EQ: PW_LANES(a == b ? one : zero)
    case PW_NE: PW_LANES(a != b ? one : zero)     // unordered: true when either is NaN (setp.neu)
    case PW_WHERE: PW_LANES(a != zero ? b : c)
    case PW_ROUND_F16: PW_LANES(T(__half2float(__float2half_rn(float(a)))))
    case PW_FMA: PW_LANES(fma_rn(a, b, c))
    case PW_GELU_TANH:   // x/2 * (1 + tanh(sqrt(2/pi) * (x + 0.044715 x^3)))
      if constexpr (sizeof(T) == 4) {
        PW_LANES(gelu_tanh_f32(a))
      } else {
        PW_LANES(mul_rn(mul_rn(half, a),
                        add_rn(one, tanh(mul_rn(fma_rn(T(0.044715), mul_rn(mul_rn(a, a), a), a),
                                                T(0.7978845608028654))))))
      }
    case PW_EXP2: PW_LANES(exp2(a))
    case PW_SILU: PW_LANES(div_rn(a, add_rn(one, exp(-a))))
    case PW_FLOOR: PW_LANES(floor(a))
    case PW_CEIL: PW_LANES(ceil(a))
    case PW_SIGN: PW_LANES(a > zero ? one : (a < zero ? -one : a))   // keeps +-0 and NaN
    default: PW_LANES(pw_slow<T>(op, a, b))
  }
#undef PW_LANES
}

template <typename T> __device__ __forceinline__ T pw_load1(const void *p, int dt, int64_t i) {
  if (dt == EMMY_DT_F16) return T(__half2float(static_cast<const __half *>(p)[i]));
  if (dt == EMMY_DT_F64) return T(static_cast<const double *>(p)[i]);
  return T(static_cast<const float *>(p)[i]);
}

// VEC = 4 consecutive elements from an aligned base (checked on the host).
template <typename T> __device__ __forceinline__ void pw_load4(const void *p, int dt, int64_t i, T v[4]) {
  if (dt == EMMY_DT_F16) {
    const uint2 u = __ldcs(reinterpret_cast<const uint2 *>(static_cast<const __half *>(p) + i));
    const __half2 h0 = *reinterpret_cast<const __half2 *>(&u.x);
    const __half2 h1 = *reinterpret_cast<const __half2 *>(&u.y);
    v[0] = T(__low2float(h0)); v[1] = T(__high2float(h0));
    v[2] = T(__low2float(h1)); v[3] = T(__high2float(h1));
  } else if (dt == EMMY_DT_F64) {
    const double2 *q = reinterpret_cast<const double2 *>(static_cast<const double *>(p) + i);
    const double2 a = __ldcs(q), b = __ldcs(q + 1);
    v[0] = T(a.x); v[1] = T(a.y); v[2] = T(b.x); v[3] = T(b.y);
  } else {
    const float4 a = __ldcs(reinterpret_cast<const float4 *>(static_cast<const float *>(p) + i));
    v[0] = T(a.x); v[1] = T(a.y); v[2] = T(a.z); v[3] = T(a.w);
  }
}

template <typename T> __device__ __forceinline__ void pw_store1(void *p, int dt, int64_t i, T v) {
  if (dt == EMMY_DT_F16) static_cast<__half *>(p)[i] = __float2half_rn(float(v));
  else if (dt == EMMY_DT_F64) static_cast<double *>(p)[i] = double(v);
  else static_cast<float *>(p)[i] = float(v);
}

template <typename T> __device__ __forceinline__ void pw_store4(void *p, int dt, int64_t i, const T v[4]) {
  if (dt == EMMY_DT_F16) {
    __half2 h0 = __floats2half2_rn(float(v[0]), float(v[1]));
    __half2 h1 = __floats2half2_rn(float(v[2]), float(v[3]));
    uint2 u;
    u.x = *reinterpret_cast<unsigned *>(&h0);
    u.y = *reinterpret_cast<unsigned *>(&h1);
    __stcs(reinterpret_cast<uint2 *>(static_cast<__half *>(p) + i), u);
  } else if (dt == EMMY_DT_F64) {
    double2 *q = reinterpret_cast<double2 *>(static_cast<double *>(p) + i);
    __stcs(q, make_double2(double(v[0]), double(v[1])));
    __stcs(q + 1, make_double2(double(v[2]), double(v[3])));
  } else {
    __stcs(reinterpret_cast<float4 *>(static_cast<float *>(p) + i),
           make_float4(float(v[0]), float(v[1]), float(v[2]), float(v[3])));
  }
}

// NIN >= 0: the input count is a compile-time constant and each thread loads
// all inputs of G groups before evaluating any of them (G * NIN vector loads
// in flight per thread).  NIN < 0: any input count, one group at a time.
// Element e of broadcast input k.
template <typename T> __device__ __forceinline__ T pw_load_bcast(const PwProgram &p, int k, int64_t e) {
  const PwIndex &x = p.idx[k];
  unsigned long long q = pw_div(x.div, (unsigned long long)(p.first + e));
  if (x.has_mod) q -= pw_div(x.mod, q) * x.mod.d;
  return pw_load1<T>(p.inputs[k], p.in_dtype[k], (int64_t)q);
}

// Elements e .. e+VEC-1 of a broadcast input: one quotient per group, the
// other lanes step from it (the quotient moves by at most one per lane when
// div >= VEC; smaller divisors divide per lane).
template <typename T, int VEC>
__device__ __forceinline__ void pw_bcast_group(const void *ptr, int dt, const PwIndex &x,
                                               long long first, int64_t e, int64_t n, T v[VEC]) {
  if (VEC > 1 && x.div.d == 1 && (!x.has_mod || x.mod.d >= (unsigned long long)VEC)) {
    // e % M: one remainder per group, consecutive lanes wrap at most once
    const unsigned long long x0 = (unsigned long long)(first + e);
    unsigned long long m0 = x0;
    if (x.has_mod) m0 = x0 - pw_div(x.mod, x0) * x.mod.d;
#pragma unroll
    for (int j = 0; j < VEC; ++j) {
      unsigned long long idx = m0 + j;
      if (x.has_mod && idx >= x.mod.d) idx -= x.mod.d;
      v[j] = e + j < n ? pw_load1<T>(ptr, dt, (int64_t)idx) : T(0);
    }
    return;
  }
  if (VEC == 1 || x.div.d < (unsigned long long)VEC) {
#pragma unroll
    for (int j = 0; j < VEC; ++j) {
      unsigned long long q = pw_div(x.div, (unsigned long long)(first + e + j));
      if (x.has_mod) q -= pw_div(x.mod, q) * x.mod.d;
      v[j] = e + j < n ? pw_load1<T>(ptr, dt, (int64_t)q) : T(0);
    }
    return;
  }
  const unsigned long long x0 = (unsigned long long)(first + e);
  const unsigned long long q0 = pw_div(x.div, x0);
  const unsigned long long r0 = x0 - q0 * x.div.d;
  unsigned long long m0 = q0;
  if (x.has_mod) m0 = q0 - pw_div(x.mod, q0) * x.mod.d;
  unsigned long long m1 = m0 + 1;
  if (x.has_mod && m1 == x.mod.d) m1 = 0;
#pragma unroll
  for (int j = 0; j < VEC; ++j) {
    const unsigned long long idx = r0 + j < x.div.d ? m0 : m1;
    v[j] = e + j < n ? pw_load1<T>(ptr, dt, (int64_t)idx) : T(0);
  }
}

template <typename T, int VEC>
__device__ __forceinline__ void pw_load_bcast_vec(const PwProgram &p, int k, int64_t e, int64_t n,
                                                  T v[VEC]) {
  pw_bcast_group<T, VEC>(p.inputs[k], p.in_dtype[k], p.idx[k], p.first, e, n, v);
}

// BC: some inputs are broadcast (read through PwIndex).
template <typename T, int VEC, int NIN, int G, bool BC = false>
__global__ void __launch_bounds__(kPwThreads)
pointwise_kernel(const PwProgram p, void *out, int out_dtype, int64_t n) {
  constexpr int S = kPwThreads;
  constexpr int NI = NIN < 0 ? 1 : (NIN == 0 ? 1 : NIN);
  extern __shared__ __align__(16) unsigned char pw_smem[];
  T *R = reinterpret_cast<T *>(pw_smem) + threadIdx.x;   // register r, lane j at R[(r*VEC+j)*S]
  for (int s = 0; s < p.n_sc; ++s) {
    const T v = pw_load1<T>(p.scalars[s], p.sc_dtype[s], 0);
#pragma unroll
    for (int j = 0; j < VEC; ++j) R[((p.n_in + s) * VEC + j) * S] = v;
  }
  for (int s = 0; s < p.n_imm; ++s) {
#pragma unroll
    for (int j = 0; j < VEC; ++j) R[((p.n_in + p.n_sc + s) * VEC + j) * S] = T(p.imm[s]);
  }
  const int n_in = NIN < 0 ? p.n_in : NIN;
  const int64_t groups = (n + VEC - 1) / VEC;
  const int64_t stride = (int64_t)gridDim.x * S;
  for (int64_t g0 = (int64_t)blockIdx.x * S + threadIdx.x; g0 < groups; g0 += stride * G) {
    T v[G][NI][VEC];
    if (NIN >= 0) {
#pragma unroll
      for (int q = 0; q < G; ++q) {
        const int64_t base = (g0 + q * stride) * VEC;
#pragma unroll
        for (int k = 0; k < NI; ++k) {
          if (k >= NIN) break;
          if (BC && p.idx[k].bcast) {
            pw_load_bcast_vec<T, VEC>(p, k, base, n, v[q][k]);
          } else if (VEC == 4 && base + VEC <= n) {
            pw_load4<T>(p.inputs[k], p.in_dtype[k], base, v[q][k]);
          } else {
#pragma unroll
            for (int j = 0; j < VEC; ++j)
              v[q][k][j] = base + j < n ? pw_load1<T>(p.inputs[k], p.in_dtype[k], base + j) : T(0);
          }
        }
      }
    }
#pragma unroll
    for (int q = 0; q < G; ++q) {
      const int64_t g = g0 + q * stride;
      if (g >= groups) break;
      const int64_t base = g * VEC;
      const bool full = base + VEC <= n;
      if (NIN >= 0) {
#pragma unroll
        for (int k = 0; k < NI; ++k) {
          if (k >= NIN) break;
#pragma unroll
          for (int j = 0; j < VEC; ++j) R[(k * VEC + j) * S] = v[q][k][j];
        }
      } else {
        for (int k = 0; k < n_in; ++k) {
          if (BC && p.idx[k].bcast) {
            T w[VEC];
            pw_load_bcast_vec<T, VEC>(p, k, base, n, w);
#pragma unroll
            for (int j = 0; j < VEC; ++j) R[(k * VEC + j) * S] = w[j];
          } else if (VEC == 4 && full) {
            T w[4];
            pw_load4<T>(p.inputs[k], p.in_dtype[k], base, w);
#pragma unroll
            for (int j = 0; j < VEC; ++j) R[(k * VEC + j) * S] = w[j];
          } else {
#pragma unroll
            for (int j = 0; j < VEC; ++j)
              R[(k * VEC + j) * S] =
                  base + j < n ? pw_load1<T>(p.inputs[k], p.in_dtype[k], base + j) : T(0);
          }
        }
      }
      for (int k = 0; k < p.n_instr; ++k) {
        const signed char *c = p.code[k];
        pw_step<T, VEC>(c[0], R + c[1] * VEC * S, R + c[2] * VEC * S, R + c[3] * VEC * S,
                        R + c[4] * VEC * S);
      }
      T o[VEC];
#pragma unroll
      for (int j = 0; j < VEC; ++j) o[j] = R[(p.result_reg * VEC + j) * S];
      if (VEC == 4 && full) {
        pw_store4<T>(out, out_dtype, base, o);
      } else {
#pragma unroll
        for (int j = 0; j < VEC; ++j)
          if (base + j < n) pw_store1<T>(out, out_dtype, base + j, o[j]);
      }
    }
  }
}

// One-step programs (the commonest pointwise shape: x op y, x op c, op x):
// operands straight from the loaded registers, no shared register file.
// Operand kinds: 0 = input tensor, 1 = one-element scalar tensor, 2 = immediate.
// Operand kinds: 0 = input tensor, 1 = one-element scalar tensor,
// 2 = immediate, 3 = broadcast input (read through idx).  `post` (>= 0) is a
// unary op applied to the step's result (x + b then ReLU).
struct PwSimple {
  const void *ptr[3];
  int dtype[3];
  int kind[3];
  // broadcast operand k read as b[(first + e) % M] with M and first multiples
  // of 4 and b 16-byte aligned: a 4-element group's values are b[m .. m+3]
  // for one m, read with one 16-byte load
  int row4[3];
  double imm[3];
  PwIndex idx[3];
  long long first;
  int nops, op, post;
};

template <typename T, bool BC>
__device__ __forceinline__ void pw_simple_operand_f32(const PwSimple &q, int k, int64_t base,
                                                      bool full, int64_t n, T v[4]) {
  if (q.kind[k] == 0) {
    const float *p = static_cast<const float *>(q.ptr[k]) + base;
    if (full) {
      const float4 a = __ldg(reinterpret_cast<const float4 *>(p));
      v[0] = T(a.x); v[1] = T(a.y); v[2] = T(a.z); v[3] = T(a.w);
    } else {
#pragma unroll
      for (int j = 0; j < 4; ++j) v[j] = base + j < n ? T(p[j]) : T(0);
    }
  } else if (BC && q.kind[k] == 3) {
    if (q.row4[k] && full) {
      const PwDiv &md = q.idx[k].mod;
      const unsigned long long x0 = (unsigned long long)(q.first + base);
      const unsigned long long m = x0 - pw_div(md, x0) * md.d;
      const float4 a = __ldg(reinterpret_cast<const float4 *>(static_cast<const float *>(q.ptr[k]) + m));
      v[0] = T(a.x); v[1] = T(a.y); v[2] = T(a.z); v[3] = T(a.w);
    } else {
      pw_bcast_group<T, 4>(q.ptr[k], EMMY_DT_F32, q.idx[k], q.first, base, n, v);
    }
  } else {
    const T c = q.kind[k] == 1 ? T(*static_cast<const float *>(q.ptr[k])) : T(q.imm[k]);
#pragma unroll
    for (int j = 0; j < 4; ++j) v[j] = c;
  }
}

template <typename T, bool BC>
__device__ __forceinline__ void pw_simple_operand(const PwSimple &q, int k, int64_t base, bool full,
                                                  int64_t n, T v[4]) {
  if (q.kind[k] == 0) {
    if (full) {
      pw_load4<T>(q.ptr[k], q.dtype[k], base, v);
    } else {
#pragma unroll
      for (int j = 0; j < 4; ++j) v[j] = base + j < n ? pw_load1<T>(q.ptr[k], q.dtype[k], base + j) : T(0);
    }
  } else if (BC && q.kind[k] == 3) {
    pw_bcast_group<T, 4>(q.ptr[k], q.dtype[k], q.idx[k], q.first, base, n, v);
  } else {
    const T c = q.kind[k] == 1 ? pw_load1<T>(q.ptr[k], q.dtype[k], 0) : T(q.imm[k]);
#pragma unroll
    for (int j = 0; j < 4; ++j) v[j] = c;
  }
}

// OPC >= 0 fixes the op at compile time (the six arithmetic ops, the common
// activations).  IO = 1 fixes every tensor operand and the output to f32, IO =
// 2 is a one-step program on one contiguous f16 input with an f16 output, IO =
// 0 reads each operand in its own dtype: a small kernel that stays at full
// occupancy.  OPC < 0 dispatches q.op at run time.
// The cheap unary ops a one-step program may be followed by.
template <typename T> __device__ __forceinline__ T pw_post(int op, T v) {
  switch (op) {
    case PW_RELU: return fmax(v, T(0));
    case PW_NEG: return -v;
    case PW_ABS: return fabs(v);
    case PW_ROUND_F16: return T(__half2float(__float2half_rn(float(v))));
    case PW_SQRT: return sqrt_rn(v);
    case PW_FLOOR: return floor(v);
    case PW_CEIL: return ceil(v);
    case PW_SIGN: return v > T(0) ? T(1) : (v < T(0) ? T(-1) : v);
    default: return v;                                  // PW_COPY
  }
}

// POST: 0 no unary step after the op, 1 one chosen at run time (q.post),
// 2 ReLU (the bias + ReLU shape, fixed at compile time); BC: some operand is
// a broadcast input; GS: 4-element groups per thread.
template <typename T, int OPC, int IO, int POST, bool BC, int GS>
__global__ void __launch_bounds__(kPwThreads)
pointwise_simple_kernel(const PwSimple q, void *out, int out_dtype, int64_t n) {
  // each thread takes GS 4-element groups a grid apart (coalesced), with
  // every group's operands loaded before any is computed
  const int64_t groups = (n + 3) / 4;
  const int64_t stride = (int64_t)gridDim.x * kPwThreads;
  for (int64_t g0 = (int64_t)blockIdx.x * kPwThreads + threadIdx.x; g0 < groups;
       g0 += GS * stride) {
    T a[GS][4], b[GS][4], c[GS][4];
#pragma unroll
    for (int u = 0; u < GS; ++u) {
      const int64_t base = (g0 + u * stride) * 4;
      if (base >= n) break;
      const bool full = base + 4 <= n;
      if (IO == 2 && full) {
        // one-step f16 program on a contiguous input (the only IO == 2 form)
        pw_load4<T>(q.ptr[0], EMMY_DT_F16, base, a[u]);
      } else if (IO == 1) {
        pw_simple_operand_f32<T, BC>(q, 0, base, full, n, a[u]);
        if (q.nops > 1) pw_simple_operand_f32<T, BC>(q, 1, base, full, n, b[u]);
        if (q.nops > 2) pw_simple_operand_f32<T, BC>(q, 2, base, full, n, c[u]);
      } else {
        pw_simple_operand<T, BC>(q, 0, base, full, n, a[u]);
        if (q.nops > 1) pw_simple_operand<T, BC>(q, 1, base, full, n, b[u]);
        if (q.nops > 2) pw_simple_operand<T, BC>(q, 2, base, full, n, c[u]);
      }
      if (q.nops < 2) {
#pragma unroll
        for (int j = 0; j < 4; ++j) b[u][j] = T(0);
      }
      if (q.nops < 3) {
#pragma unroll
        for (int j = 0; j < 4; ++j) c[u][j] = T(0);
      }
    }
#pragma unroll
    for (int u = 0; u < GS; ++u) {
      const int64_t base = (g0 + u * stride) * 4;
      if (base >= n) break;
      const bool full = base + 4 <= n;
      // registers in place of the shared-memory file (lane stride 1).  A
      // run-time op is dispatched once for the four lanes: a per-lane dispatch
      // would unroll four copies of every op's code.  A compile-time op is
      // applied lane by lane (measured faster for the streaming ops).
      T o[4];
      if (OPC >= 0) {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          T ra[1] = {a[u][j]}, rb[1] = {b[u][j]}, rc[1] = {c[u][j]}, rd[1];
          pw_step<T, 1, 1>(OPC, rd, ra, rb, rc);
          o[j] = rd[0];
        }
      } else {
        pw_step<T, 4, 1>(q.op, o, a[u], b[u], c[u]);
      }
      if (POST == 2) {
#pragma unroll
        for (int j = 0; j < 4; ++j) o[j] = fmax(o[j], T(0));
      } else if (POST == 1) {
#pragma unroll
        for (int j = 0; j < 4; ++j) o[j] = pw_post<T>(q.post, o[j]);
      }
      if (IO == 1) {
        float *dst = static_cast<float *>(out) + base;
        if (full) {
          *reinterpret_cast<float4 *>(dst) =
              make_float4(float(o[0]), float(o[1]), float(o[2]), float(o[3]));
        } else {
#pragma unroll
          for (int j = 0; j < 4; ++j)
            if (base + j < n) dst[j] = float(o[j]);
        }
      } else if (full) {
        pw_store4<T>(out, IO == 2 ? EMMY_DT_F16 : out_dtype, base, o);
      } else {
#pragma unroll
        for (int j = 0; j < 4; ++j)
          if (base + j < n) pw_store1<T>(out, out_dtype, base + j, o[j]);
      }
    }
  }
}

template <typename T, int VEC, int NIN, int G, bool BC = false>
void launch_pointwise(const PwProgram &p, int nregs, void *out, int out_dtype, int64_t n,
                      cudaStream_t st) {
  const int64_t groups = (n + VEC - 1) / VEC;
  // one pass: each thread takes G groups (their loads issued together) and the
  // grid covers the data once -- many short CTAs keep every SM streaming to
  // the end, where a capped grid-stride loop ran slower on B200
  int64_t blocks = (groups + (int64_t)kPwThreads * G - 1) / ((int64_t)kPwThreads * G);
  if (blocks > INT32_MAX) blocks = INT32_MAX;          // the grid-stride loop covers the rest
  const size_t smem = (size_t)nregs * VEC * kPwThreads * sizeof(T);
  if (smem > 48 * 1024)
    cudaFuncSetAttribute(pointwise_kernel<T, VEC, NIN, G, BC>,
                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  pointwise_kernel<T, VEC, NIN, G, BC><<<(unsigned)blocks, kPwThreads, smem, st>>>(p, out, out_dtype, n);
}

template <typename T, int VEC>
void dispatch_inputs(const PwProgram &p, int nregs, void *out, int out_dtype, int64_t n,
                     cudaStream_t st, bool bcast) {
  if (bcast) {
    switch (p.n_in) {
      case 2: launch_pointwise<T, VEC, 2, 2, true>(p, nregs, out, out_dtype, n, st); break;
      case 3: launch_pointwise<T, VEC, 3, 2, true>(p, nregs, out, out_dtype, n, st); break;
      default: launch_pointwise<T, VEC, -1, 1, true>(p, nregs, out, out_dtype, n, st); break;
    }
    return;
  }
  switch (p.n_in) {
    case 0: launch_pointwise<T, VEC, 0, 1>(p, nregs, out, out_dtype, n, st); break;
    case 1: launch_pointwise<T, VEC, 1, 2>(p, nregs, out, out_dtype, n, st); break;
    case 2: launch_pointwise<T, VEC, 2, 2>(p, nregs, out, out_dtype, n, st); break;
    case 3: launch_pointwise<T, VEC, 3, 2>(p, nregs, out, out_dtype, n, st); break;
    case 4: launch_pointwise<T, VEC, 4, 1>(p, nregs, out, out_dtype, n, st); break;
    default: launch_pointwise<T, VEC, -1, 1>(p, nregs, out, out_dtype, n, st); break;
  }
}

}  // namespace emmy

using namespace emmy;

template <typename T, int OPC, int IO, int POST, bool BC>
static void launch_simple_gs(const PwSimple &q, void *out, int out_dtype, int64_t n, unsigned gb,
                             cudaStream_t st, int gs) {
  if (gs > 1) pointwise_simple_kernel<T, OPC, IO, POST, BC, kPwSimpleGroups><<<gb, kPwThreads, 0, st>>>(q, out, out_dtype, n);
  else pointwise_simple_kernel<T, OPC, IO, POST, BC, 1><<<gb, kPwThreads, 0, st>>>(q, out, out_dtype, n);
}

template <typename T, int OPC, int IO>
static void launch_simple(const PwSimple &q, void *out, int out_dtype, int64_t n, unsigned gb,
                          cudaStream_t st, bool has_bc, int gs) {
  if (q.post == PW_RELU) {
    if (has_bc) launch_simple_gs<T, OPC, IO, 2, true>(q, out, out_dtype, n, gb, st, gs);
    else launch_simple_gs<T, OPC, IO, 2, false>(q, out, out_dtype, n, gb, st, gs);
  } else if (q.post >= 0) {
    if (has_bc) launch_simple_gs<T, OPC, IO, 1, true>(q, out, out_dtype, n, gb, st, gs);
    else launch_simple_gs<T, OPC, IO, 1, false>(q, out, out_dtype, n, gb, st, gs);
  } else {
    if (has_bc) launch_simple_gs<T, OPC, IO, 0, true>(q, out, out_dtype, n, gb, st, gs);
    else launch_simple_gs<T, OPC, IO, 0, false>(q, out, out_dtype, n, gb, st, gs);
  }
}

static int pointwise_impl(const void *const *inputs, const int *input_dtypes,
                          const int64_t *input_index, int n_inputs, const void *const *scalars,
                          const int *scalar_dtypes, int n_scalars, const double *immediates,
                          int n_imm, const int *program, int n_instr, int result_reg,
                          int compute_f64, void *out, int out_dtype, int64_t first, int64_t n,
                          void *stream) {
  clear_error();
  if (n < 0 || first < 0) return set_error(EMMY_ERR_INVALID, "emmy_pointwise: negative size");
  if (n == 0) return EMMY_OK;
  if (!out) return set_error(EMMY_ERR_INVALID, "emmy_pointwise: null output");
  if (n_inputs < 0 || n_inputs > kPwMaxIn || n_scalars < 0 || n_scalars > kPwMaxIn || n_imm < 0 ||
      n_imm > kPwMaxIn || n_instr < 1 || n_instr > kPwMaxInstr)
    return set_error(EMMY_ERR_INVALID, "emmy_pointwise: program has too many inputs or steps");
  if ((n_inputs && (!inputs || !input_dtypes)) || (n_scalars && (!scalars || !scalar_dtypes)) ||
      (n_imm && !immediates) || !program)
    return set_error(EMMY_ERR_INVALID, "emmy_pointwise: null argument array");
  const int nregs = n_inputs + n_scalars + n_imm + n_instr;
  if (nregs > kPwMaxRegs) return set_error(EMMY_ERR_INVALID, "emmy_pointwise: too many registers");
  if (result_reg < 0 || result_reg >= nregs)
    return set_error(EMMY_ERR_INVALID, "emmy_pointwise: bad result register");
  auto dt_ok = [](int dt) { return dt == EMMY_DT_F32 || dt == EMMY_DT_F16 || dt == EMMY_DT_F64; };
  if (!dt_ok(out_dtype)) return set_error(EMMY_ERR_INVALID, "emmy_pointwise: bad output dtype");
  PwProgram p{};
  p.n_in = n_inputs;
  p.n_sc = n_scalars;
  p.n_imm = n_imm;
  p.n_instr = n_instr;
  p.result_reg = result_reg;
  bool vec_ok = aligned16(out) || (out_dtype == EMMY_DT_F16 && ((uintptr_t)out & 7) == 0);
  bool bcast = false;
  p.first = first;
  for (int i = 0; i < n_inputs; ++i) {
    if (!inputs[i]) return set_error(EMMY_ERR_INVALID, "emmy_pointwise: null input %d", i);
    if (!dt_ok(input_dtypes[i])) return set_error(EMMY_ERR_INVALID, "emmy_pointwise: bad input dtype");
    p.inputs[i] = inputs[i];
    p.in_dtype[i] = input_dtypes[i];
    const int64_t dv = input_index ? input_index[3 * i] : 0;
    if (dv != 0) {
      // broadcast input: ((first + e) / div) % mod must stay inside its numel
      const int64_t md = input_index[3 * i + 1], numel = input_index[3 * i + 2];
      if (dv < 1 || dv >= (int64_t(1) << 62) || md < 0 || md >= (int64_t(1) << 62) || numel < 1)
        return set_error(EMMY_ERR_INVALID, "emmy_pointwise: bad index of input %d", i);
      const int64_t top = md > 0 ? std::min<int64_t>(md - 1, (first + n - 1) / dv) : (first + n - 1) / dv;
      if (top >= numel)
        return set_error(EMMY_ERR_INVALID, "emmy_pointwise: input %d read past its %lld elements", i,
                         (long long)numel);
      p.idx[i].bcast = 1;
      p.idx[i].div = make_div((unsigned long long)dv);
      p.idx[i].has_mod = md > 0;
      if (md > 0) p.idx[i].mod = make_div((unsigned long long)md);
      bcast = true;
      continue;
    }
    const uintptr_t need = input_dtypes[i] == EMMY_DT_F16 ? 8 : 16;
    vec_ok = vec_ok && ((uintptr_t)inputs[i] % need) == 0;
  }
  for (int i = 0; i < n_scalars; ++i) {
    if (!scalars[i]) return set_error(EMMY_ERR_INVALID, "emmy_pointwise: null scalar %d", i);
    if (!dt_ok(scalar_dtypes[i])) return set_error(EMMY_ERR_INVALID, "emmy_pointwise: bad scalar dtype");
    p.scalars[i] = scalars[i];
    p.sc_dtype[i] = scalar_dtypes[i];
  }
  for (int i = 0; i < n_imm; ++i) p.imm[i] = immediates[i];
  for (int k = 0; k < n_instr; ++k) {
    const int *c = program + 5 * k;
    if (c[0] < 0 || c[0] >= PW_NOPS)
      return set_error(EMMY_ERR_INVALID, "emmy_pointwise: unknown opcode %d", c[0]);
    // destinations are the temporaries (never an input, scalar or immediate)
    if (c[1] < n_inputs + n_scalars + n_imm || c[1] >= nregs)
      return set_error(EMMY_ERR_INVALID, "emmy_pointwise: step %d writes register %d", k, c[1]);
    for (int j = 2; j < 5; ++j)
      if (c[j] < 0 || c[j] >= nregs)
        return set_error(EMMY_ERR_INVALID, "emmy_pointwise: register %d out of range", c[j]);
    for (int j = 0; j < 5; ++j) p.code[k][j] = (signed char)c[j];
  }
  // the shared register file of a 4-wide double program with many registers
  // would not fit; such programs run one element per thread
  if ((size_t)nregs * 4 * kPwThreads * (compute_f64 ? 8 : 4) > 160 * 1024) vec_ok = false;
  cudaStream_t st = as_stream(stream);
  const int nleaf = n_inputs + n_scalars + n_imm;
  // Transcendental steps (exp, log, tanh, gelu, ...) are issue-bound; they
  // run faster in the general kernel, whose threads take two groups each.
  auto cheap = [](int op) {
    return op <= PW_ABS || (op >= PW_RELU && op <= PW_FMA) || op == PW_FLOOR || op == PW_CEIL ||
           op == PW_SIGN || op == PW_SQRT || op == PW_NE;
  };
  auto arity_of = [](int op) {
    return (op == PW_WHERE || op == PW_FMA) ? 3
           : (op == PW_ADD || op == PW_SUB || op == PW_MUL || op == PW_DIV || op == PW_MAX ||
              op == PW_MIN || op == PW_GT || op == PW_LT || op == PW_GE || op == PW_LE ||
              op == PW_EQ || op == PW_NE || op == PW_POW)
               ? 2
               : 1;
  };
  // one step on leaves, optionally followed by one unary step on its result
  // (the bias + ReLU shape): the register kernel
  const bool one = n_instr == 1 && result_reg == nleaf;
  const bool two = n_instr == 2 && result_reg == nleaf + 1 && arity_of(program[5]) == 1 &&
                   program[7] == nleaf && cheap(program[5]);
  bool leaves_only = true;
  for (int k = 0; k < arity_of(program[0]); ++k) leaves_only = leaves_only && program[2 + k] < nleaf;
  // the common activations also take the register kernel when every operand
  // and the output are f32, with the op fixed at compile time (measured: gelu
  // 122 -> 95 us, exp 105 -> 92 us on 2^26 elements; a run-time dispatch of
  // them per lane, or f16 operands, ran slower than the general kernel)
  auto all_f32 = [&]() {
    if (compute_f64 || out_dtype != EMMY_DT_F32) return false;
    for (int k = 0; k < arity_of(program[0]); ++k) {
      const int r = program[2 + k];
      if (r < n_inputs && input_dtypes[r] != EMMY_DT_F32) return false;
      if (r >= n_inputs && r < n_inputs + n_scalars && scalar_dtypes[r - n_inputs] != EMMY_DT_F32)
        return false;
    }
    return true;
  };
  // ... and, as one step on a contiguous f16 input with an f16 output, with
  // half loads and stores fixed at compile time
  auto all_f16_one = [&]() {
    return !compute_f64 && one && out_dtype == EMMY_DT_F16 && program[2] < n_inputs &&
           input_dtypes[program[2]] == EMMY_DT_F16 && !p.idx[program[2]].bcast;
  };
  auto activation = [](int op) { return op == PW_GELU_TANH || op == PW_SILU || op == PW_EXP; };
  auto compiled = [&](int op) { return activation(op) && (all_f32() || all_f16_one()); };
  if (vec_ok && (one || two) && leaves_only && (cheap(program[0]) || compiled(program[0]))) {
    const int op = program[0];
    const int arity = arity_of(op);
    PwSimple q{};
    q.op = op;
    q.nops = arity;
    q.post = two ? program[5] : -1;
    q.first = first;
    for (int k = 0; k < arity; ++k) {
      const int r = program[2 + k];
      if (r < n_inputs) {
        q.kind[k] = p.idx[r].bcast ? 3 : 0; q.ptr[k] = inputs[r]; q.dtype[k] = input_dtypes[r];
        q.idx[k] = p.idx[r];
        q.row4[k] = p.idx[r].bcast && p.idx[r].div.d == 1 && p.idx[r].has_mod &&
                    p.idx[r].mod.d % 4 == 0 && first % 4 == 0 && aligned16(inputs[r]);
      } else if (r < n_inputs + n_scalars) {
        q.kind[k] = 1; q.ptr[k] = scalars[r - n_inputs]; q.dtype[k] = scalar_dtypes[r - n_inputs];
      } else {
        q.kind[k] = 2; q.imm[k] = immediates[r - n_inputs - n_scalars];
      }
    }
    // two groups per thread unless two or more operands stream from HBM
    // (measured: 2 groups take a + b[e % M] from 118 to 99 us, unary
    // activations 5-20% faster; x + y 3% slower)
    int full_streams = 0;
    for (int k = 0; k < arity; ++k) full_streams += q.kind[k] == 0;
    const int gs = full_streams >= 2 ? 1 : kPwSimpleGroups;
    int64_t blocks = ((n + 3) / 4 + (int64_t)kPwThreads * gs - 1) / ((int64_t)kPwThreads * gs);
    if (blocks > INT32_MAX) blocks = INT32_MAX;
    const unsigned gb = (unsigned)blocks;
    bool f32io = !compute_f64 && out_dtype == EMMY_DT_F32;
    for (int k = 0; k < arity; ++k)
      if (q.kind[k] != 2 && q.dtype[k] != EMMY_DT_F32) f32io = false;
#define EMMY_PW_LAUNCH(T, OPC, IO) \
    launch_simple<T, OPC, IO>(q, out, out_dtype, n, gb, st, has_bc, gs)
    const bool has_bc = q.kind[0] == 3 || q.kind[1] == 3 || q.kind[2] == 3;
    if (compiled(op) && !f32io && op == PW_GELU_TANH && n % 8 == 0 && aligned16(q.ptr[0]) &&
        aligned16(out)) {
      // gelu on whole 8-element groups: 16-byte loads and stores, packed pairs;
      // eight groups (128 bytes) in flight per thread before any compute
      constexpr int GS = 8;
      const int64_t n8 = n / 8;
      int64_t blocks = (n8 + 256LL * GS - 1) / (256LL * GS);
      if (blocks > INT32_MAX) blocks = INT32_MAX;
      gelu_tanh_f16x8_kernel<GS><<<(unsigned)blocks, 256, 0, st>>>(
          static_cast<const uint4 *>(q.ptr[0]), static_cast<uint4 *>(out), n8);
    } else if (compiled(op) && !f32io) {               // one f16 step, no post, no broadcast
      switch (op) {
        case PW_GELU_TANH:
          pointwise_simple_kernel<float, PW_GELU_TANH, 2, 0, false, kPwSimpleGroups>
              <<<gb, kPwThreads, 0, st>>>(q, out, out_dtype, n);
          break;
        case PW_SILU:
          pointwise_simple_kernel<float, PW_SILU, 2, 0, false, kPwSimpleGroups>
              <<<gb, kPwThreads, 0, st>>>(q, out, out_dtype, n);
          break;
        default:
          pointwise_simple_kernel<float, PW_EXP, 2, 0, false, kPwSimpleGroups>
              <<<gb, kPwThreads, 0, st>>>(q, out, out_dtype, n);
          break;
      }
    } else if (compiled(op)) {                         // f32io holds here
      switch (op) {
        case PW_GELU_TANH: EMMY_PW_LAUNCH(float, PW_GELU_TANH, 1); break;
        case PW_SILU: EMMY_PW_LAUNCH(float, PW_SILU, 1); break;
        default: EMMY_PW_LAUNCH(float, PW_EXP, 1); break;
      }
    } else if (f32io) {
      switch (op) {
        case PW_ADD: EMMY_PW_LAUNCH(float, PW_ADD, 1); break;
        case PW_SUB: EMMY_PW_LAUNCH(float, PW_SUB, 1); break;
        case PW_MUL: EMMY_PW_LAUNCH(float, PW_MUL, 1); break;
        case PW_DIV: EMMY_PW_LAUNCH(float, PW_DIV, 1); break;
        case PW_MAX: EMMY_PW_LAUNCH(float, PW_MAX, 1); break;
        case PW_MIN: EMMY_PW_LAUNCH(float, PW_MIN, 1); break;
        default: EMMY_PW_LAUNCH(float, -1, 1); break;
      }
    } else if (compute_f64) {
      EMMY_PW_LAUNCH(double, -1, 0);
    } else {
      EMMY_PW_LAUNCH(float, -1, 0);
    }
#undef EMMY_PW_LAUNCH
    return check_launch("emmy_pointwise (one step)");
  }
  if (compute_f64) {
    if (vec_ok) dispatch_inputs<double, 4>(p, nregs, out, out_dtype, n, st, bcast);
    else dispatch_inputs<double, 1>(p, nregs, out, out_dtype, n, st, bcast);
  } else {
    if (vec_ok) dispatch_inputs<float, 4>(p, nregs, out, out_dtype, n, st, bcast);
    else dispatch_inputs<float, 1>(p, nregs, out, out_dtype, n, st, bcast);
  }
  return check_launch("emmy_pointwise");
}

extern "C" int emmy_pointwise(const void *const *inputs, const int *input_dtypes, int n_inputs,
                              const void *const *scalars, const int *scalar_dtypes, int n_scalars,
                              const double *immediates, int n_imm, const int *program, int n_instr,
                              int result_reg, int compute_f64, void *out, int out_dtype, int64_t n,
                              void *stream) {
  return pointwise_impl(inputs, input_dtypes, nullptr, n_inputs, scalars, scalar_dtypes, n_scalars,
                        immediates, n_imm, program, n_instr, result_reg, compute_f64, out, out_dtype,
                        0, n, stream);
}

extern "C" int emmy_pointwise_indexed(const void *const *inputs, const int *input_dtypes,
                                      const int64_t *input_index, int n_inputs,
                                      const void *const *scalars, const int *scalar_dtypes,
                                      int n_scalars, const double *immediates, int n_imm,
                                      const int *program, int n_instr, int result_reg,
                                      int compute_f64, void *out, int out_dtype, int64_t first,
                                      int64_t n, void *stream) {
  return pointwise_impl(inputs, input_dtypes, input_index, n_inputs, scalars, scalar_dtypes,
                        n_scalars, immediates, n_imm, program, n_instr, result_reg, compute_f64, out,
                        out_dtype, first, n, stream);
}
