// Integer pointwise programs on sm_100a: out[e] = f(in_0[e], ..., scalars,
// immediates) with the arithmetic on signed 64-bit values.
//
// Replaces what the reference emits for a pointwise IR whose Assigns are
// integer-typed (reference ptxc/stmts.py:509-560 Assign, ptxc/ops.py:98-117
// INT_BINARY, ptxc/expr.py:157-165 and 211-223 operand widening, 697-716
// div / rem, 815-877 predicates and where, 233-280 the converting store):
//   * every operand becomes an s64 value: an integer element is sign- or
//     zero-extended from its type (cvt.s64.s8 / .u8 / ... ), a float element
//     is truncated toward zero (cvt.rzi.s64.f16 / .f32 / .f64, which clamp to
//     the s64 range and take NaN to -2^63);
//   * add, sub and mul wrap modulo 2^64; div and rem are div.s64 / rem.s64
//     (toward zero); max, min and the comparisons are signed; xor is bitwise;
//     shifts are shl.b64 / shr.s64 by the low 32 bits of the count;
//   * comparisons and and / or / not give 0 or 1 (the reference's predicates;
//     its Assign sends bitwise_and / bitwise_or down that path too); where
//     selects on c != 0;
//   * the result is stored by the output's type: its low bits for an integer
//     output, cvt.rn.f64.s64 / cvt.rn.f32.s64 (then cvt.rn.f16.f32 for f16)
//     for a float output.
// The conversions are the PTX instructions the reference emits, written as
// inline PTX, so the two agree bit for bit.
//
// The program layout follows the float pointwise kernel: registers in shared
// memory (lane j of register r of thread t at [(r*VEC + j)*THREADS + t]),
// each instruction decoded once per four elements, inputs and the output
// moved as vectors of four elements (4 to 32 bytes) when the pointers allow.
// (Holding the s64 values in registers instead was measured slower: 70-122
// registers a thread leave too few warps to keep the loads in flight.)

#include <algorithm>
#include <type_traits>

#include "common.cuh"
#include "pw_index.cuh"
#include "tma.cuh"

namespace emmy {

constexpr int kPiThreads = 128, kPiVec = 4, kPiMaxRegs = 32, kPiMaxInstr = 48, kPiMaxIn = 8;

// opcodes shared with ptxc/match_pointwise.py (INT_OPCODES)
enum PiOp {
  PI_COPY, PI_ADD, PI_SUB, PI_MUL, PI_DIV, PI_REM, PI_SHL, PI_SHR, PI_XOR, PI_MAX, PI_MIN,
  PI_EQ, PI_NE, PI_GT, PI_LT, PI_GE, PI_LE, PI_LAND, PI_LOR, PI_LNOT, PI_WHERE, PI_NOPS
};

struct PiProgram {
  const void *inputs[kPiMaxIn];
  int in_dtype[kPiMaxIn];
  PwIndex idx[kPiMaxIn];
  const void *scalars[kPiMaxIn];
  int sc_dtype[kPiMaxIn];
  long long imm[kPiMaxIn];
  signed char code[kPiMaxInstr][5];
  long long first;
  int n_in, n_sc, n_imm, n_instr, result_reg;
};

// ---- operand conversions (the reference's cvt spellings) -------------------

__device__ __forceinline__ long long pi_rzi_f32(float x) {
  long long r;
  asm("cvt.rzi.s64.f32 %0, %1;" : "=l"(r) : "f"(x));
  return r;
}
__device__ __forceinline__ long long pi_rzi_f64(double x) {
  long long r;
  asm("cvt.rzi.s64.f64 %0, %1;" : "=l"(r) : "d"(x));
  return r;
}
__device__ __forceinline__ long long pi_rzi_f16(unsigned short h) {
  long long r;
  asm("cvt.rzi.s64.f16 %0, %1;" : "=l"(r) : "h"(h));
  return r;
}
__device__ __forceinline__ float pi_f32_of(long long v) {
  float r;
  asm("cvt.rn.f32.s64 %0, %1;" : "=f"(r) : "l"(v));
  return r;
}
__device__ __forceinline__ double pi_f64_of(long long v) {
  double r;
  asm("cvt.rn.f64.s64 %0, %1;" : "=d"(r) : "l"(v));
  return r;
}
__device__ __forceinline__ unsigned short pi_f16_of(long long v) {
  unsigned short r;
  asm("cvt.rn.f16.f32 %0, %1;" : "=h"(r) : "f"(pi_f32_of(v)));
  return r;
}

// element i of a buffer of type dt as an s64 value
__device__ __forceinline__ long long pi_load1(const void *p, int dt, int64_t i) {
  switch (dt) {
    case EMMY_DT_I8: return __ldg(static_cast<const signed char *>(p) + i);
    case EMMY_DT_U8: return __ldg(static_cast<const unsigned char *>(p) + i);
    case EMMY_DT_I16: return __ldg(static_cast<const short *>(p) + i);
    case EMMY_DT_U16: return __ldg(static_cast<const unsigned short *>(p) + i);
    case EMMY_DT_I32: return __ldg(static_cast<const int *>(p) + i);
    case EMMY_DT_U32: return __ldg(static_cast<const unsigned int *>(p) + i);
    case EMMY_DT_I64:
    case EMMY_DT_U64: return __ldg(static_cast<const long long *>(p) + i);
    case EMMY_DT_F16: return pi_rzi_f16(__ldg(static_cast<const unsigned short *>(p) + i));
    case EMMY_DT_F32: return pi_rzi_f32(__ldg(static_cast<const float *>(p) + i));
    default: return pi_rzi_f64(__ldg(static_cast<const double *>(p) + i));
  }
}

// a vector load: read-only global (GLOBAL) or shared memory
template <bool GLOBAL, typename V>
__device__ __forceinline__ V pi_ld(const V *q) {
  if constexpr (GLOBAL) return __ldg(q);
  else return *q;
}

// U groups of four elements of global (GLOBAL) or shared memory, group u at
// elements base + u * gstride .. + 3 (each group aligned for one or two vector
// loads), as values of type T (s64 values cut to T); lane 4u + j of v.  One
// switch on the type for all groups.
template <bool GLOBAL, int U, typename T, typename CONV>
__device__ __forceinline__ void pi_load_bytes(const void *p, int64_t base, int64_t gstride,
                                              T v[4 * U], const CONV &conv) {
#pragma unroll
  for (int u = 0; u < U; ++u) {
    const unsigned int w = pi_ld<GLOBAL>(reinterpret_cast<const unsigned int *>(
        static_cast<const unsigned char *>(p) + base + u * gstride));
#pragma unroll
    for (int j = 0; j < 4; ++j) v[4 * u + j] = conv((w >> (8 * j)) & 0xffu);
  }
}
template <bool GLOBAL, int U, typename T, typename CONV>
__device__ __forceinline__ void pi_load_halves(const void *p, int64_t base, int64_t gstride,
                                               T v[4 * U], const CONV &conv) {
#pragma unroll
  for (int u = 0; u < U; ++u) {
    const uint2 w = pi_ld<GLOBAL>(reinterpret_cast<const uint2 *>(
        static_cast<const unsigned short *>(p) + base + u * gstride));
    const unsigned int h[4] = {w.x & 0xffffu, w.x >> 16, w.y & 0xffffu, w.y >> 16};
#pragma unroll
    for (int j = 0; j < 4; ++j) v[4 * u + j] = conv(h[j]);
  }
}
template <bool GLOBAL, int U, typename T, typename CONV>
__device__ __forceinline__ void pi_load_words(const void *p, int64_t base, int64_t gstride,
                                              T v[4 * U], const CONV &conv) {
#pragma unroll
  for (int u = 0; u < U; ++u) {
    const uint4 w = pi_ld<GLOBAL>(reinterpret_cast<const uint4 *>(
        static_cast<const int *>(p) + base + u * gstride));
    const unsigned int x[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) v[4 * u + j] = conv(x[j]);
  }
}

// U groups of four elements of global (GLOBAL) or shared memory, group u at
// elements base + u * gstride .. + 3 (each group aligned for one or two vector
// loads), as values of type T (s64 values cut to T); lane 4u + j of v.  One
// switch on the type for all groups, each type's widening fixed in its case.
template <bool GLOBAL, int U, typename T>
__device__ __forceinline__ void pi_loadv(const void *p, int dt, int64_t base, int64_t gstride,
                                         T v[4 * U]) {
  switch (dt) {
    case EMMY_DT_I8:
      pi_load_bytes<GLOBAL, U>(p, base, gstride, v, [](unsigned int b) { return (T)(signed char)b; });
      break;
    case EMMY_DT_U8:
      pi_load_bytes<GLOBAL, U>(p, base, gstride, v, [](unsigned int b) { return (T)b; });
      break;
    case EMMY_DT_I16:
      pi_load_halves<GLOBAL, U>(p, base, gstride, v, [](unsigned int h) { return (T)(short)h; });
      break;
    case EMMY_DT_U16:
      pi_load_halves<GLOBAL, U>(p, base, gstride, v, [](unsigned int h) { return (T)h; });
      break;
    case EMMY_DT_F16:
      pi_load_halves<GLOBAL, U>(p, base, gstride, v,
                                [](unsigned int h) { return (T)pi_rzi_f16((unsigned short)h); });
      break;
    case EMMY_DT_I32:
      pi_load_words<GLOBAL, U>(p, base, gstride, v, [](unsigned int x) { return (T)(int)x; });
      break;
    case EMMY_DT_U32:
      pi_load_words<GLOBAL, U>(p, base, gstride, v, [](unsigned int x) { return (T)(long long)x; });
      break;
    case EMMY_DT_F32:
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const float4 w = pi_ld<GLOBAL>(reinterpret_cast<const float4 *>(
            static_cast<const float *>(p) + base + u * gstride));
        v[4 * u + 0] = (T)pi_rzi_f32(w.x); v[4 * u + 1] = (T)pi_rzi_f32(w.y);
        v[4 * u + 2] = (T)pi_rzi_f32(w.z); v[4 * u + 3] = (T)pi_rzi_f32(w.w);
      }
      break;
    case EMMY_DT_F64:
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const double2 *q = reinterpret_cast<const double2 *>(
            static_cast<const double *>(p) + base + u * gstride);
        const double2 a = pi_ld<GLOBAL>(q), b = pi_ld<GLOBAL>(q + 1);
        v[4 * u + 0] = (T)pi_rzi_f64(a.x); v[4 * u + 1] = (T)pi_rzi_f64(a.y);
        v[4 * u + 2] = (T)pi_rzi_f64(b.x); v[4 * u + 3] = (T)pi_rzi_f64(b.y);
      }
      break;
    default:                                           // I64, U64
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const longlong2 *q = reinterpret_cast<const longlong2 *>(
            static_cast<const long long *>(p) + base + u * gstride);
        const longlong2 a = pi_ld<GLOBAL>(q), b = pi_ld<GLOBAL>(q + 1);
        v[4 * u + 0] = (T)a.x; v[4 * u + 1] = (T)a.y; v[4 * u + 2] = (T)b.x; v[4 * u + 3] = (T)b.y;
      }
      break;
  }
}

// elements base .. base + 3 (aligned for one or two vector loads) of global
// (GLOBAL) or shared memory
template <bool GLOBAL = true>
__device__ __forceinline__ void pi_load4(const void *p, int dt, int64_t base, long long v[4]) {
  pi_loadv<GLOBAL, 1, long long>(p, dt, base, 0, v);
}

// ---- stores: the output's type decides (reference _cast_reg) ----------------

__device__ __forceinline__ void pi_store1(void *p, int dt, int64_t i, long long v) {
  const unsigned long long u = (unsigned long long)v;
  switch (dt) {
    case EMMY_DT_I8:
    case EMMY_DT_U8: static_cast<unsigned char *>(p)[i] = (unsigned char)u; break;
    case EMMY_DT_I16:
    case EMMY_DT_U16: static_cast<unsigned short *>(p)[i] = (unsigned short)u; break;
    case EMMY_DT_I32:
    case EMMY_DT_U32: static_cast<unsigned int *>(p)[i] = (unsigned int)u; break;
    case EMMY_DT_F16: static_cast<unsigned short *>(p)[i] = pi_f16_of(v); break;
    case EMMY_DT_F32: static_cast<float *>(p)[i] = pi_f32_of(v); break;
    case EMMY_DT_F64: static_cast<double *>(p)[i] = pi_f64_of(v); break;
    default: static_cast<unsigned long long *>(p)[i] = u; break;   // I64, U64
  }
}

// U groups of four elements, group u at base + u * gstride (each aligned for
// one or two vector stores); lane 4u + j of v (s64 values, or T values that
// stand for them).  One switch on the type for all groups.
template <int U, typename T>
__device__ __forceinline__ void pi_storev(void *p, int dt, int64_t base, int64_t gstride,
                                          const T v[4 * U]) {
  switch (dt) {
    case EMMY_DT_I8:
    case EMMY_DT_U8:
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const T *x = v + 4 * u;
        *reinterpret_cast<unsigned int *>(static_cast<unsigned char *>(p) + base + u * gstride) =
            ((unsigned int)x[0] & 0xffu) | ((unsigned int)x[1] & 0xffu) << 8 |
            ((unsigned int)x[2] & 0xffu) << 16 | ((unsigned int)x[3] & 0xffu) << 24;
      }
      break;
    case EMMY_DT_I16:
    case EMMY_DT_U16:
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const T *x = v + 4 * u;
        *reinterpret_cast<uint2 *>(static_cast<unsigned short *>(p) + base + u * gstride) =
            make_uint2(((unsigned int)x[0] & 0xffffu) | ((unsigned int)x[1] & 0xffffu) << 16,
                       ((unsigned int)x[2] & 0xffffu) | ((unsigned int)x[3] & 0xffffu) << 16);
      }
      break;
    case EMMY_DT_F16:
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const T *x = v + 4 * u;
        *reinterpret_cast<uint2 *>(static_cast<unsigned short *>(p) + base + u * gstride) =
            make_uint2((unsigned int)pi_f16_of(x[0]) | (unsigned int)pi_f16_of(x[1]) << 16,
                       (unsigned int)pi_f16_of(x[2]) | (unsigned int)pi_f16_of(x[3]) << 16);
      }
      break;
    case EMMY_DT_I32:
    case EMMY_DT_U32:
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const T *x = v + 4 * u;
        *reinterpret_cast<uint4 *>(static_cast<unsigned int *>(p) + base + u * gstride) =
            make_uint4((unsigned int)x[0], (unsigned int)x[1], (unsigned int)x[2], (unsigned int)x[3]);
      }
      break;
    case EMMY_DT_F32:
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const T *x = v + 4 * u;
        *reinterpret_cast<float4 *>(static_cast<float *>(p) + base + u * gstride) =
            make_float4(pi_f32_of(x[0]), pi_f32_of(x[1]), pi_f32_of(x[2]), pi_f32_of(x[3]));
      }
      break;
    case EMMY_DT_F64:
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const T *x = v + 4 * u;
        double2 *q = reinterpret_cast<double2 *>(static_cast<double *>(p) + base + u * gstride);
        q[0] = make_double2(pi_f64_of(x[0]), pi_f64_of(x[1]));
        q[1] = make_double2(pi_f64_of(x[2]), pi_f64_of(x[3]));
      }
      break;
    default:                                           // I64, U64
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const T *x = v + 4 * u;
        longlong2 *q = reinterpret_cast<longlong2 *>(static_cast<long long *>(p) + base + u * gstride);
        q[0] = make_longlong2((long long)x[0], (long long)x[1]);
        q[1] = make_longlong2((long long)x[2], (long long)x[3]);
      }
      break;
  }
}

__device__ __forceinline__ void pi_store4(void *p, int dt, int64_t base, const long long v[4]) {
  pi_storev<1, long long>(p, dt, base, 0, v);
}

// ---- one instruction over VEC lanes (lane stride S) -------------------------

__device__ __forceinline__ long long pi_div(long long a, long long b) {
  long long r;
  asm("div.s64 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ long long pi_rem(long long a, long long b) {
  long long r;
  asm("rem.s64 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ long long pi_shl(long long a, long long b) {
  long long r;
  asm("shl.b64 %0, %1, %2;" : "=l"(r) : "l"(a), "r"((unsigned int)b));
  return r;
}
__device__ __forceinline__ long long pi_shr(long long a, long long b) {
  long long r;
  asm("shr.s64 %0, %1, %2;" : "=l"(r) : "l"(a), "r"((unsigned int)b));
  return r;
}
// the same on 32-bit values (programs whose values the matcher proved to fit)
__device__ __forceinline__ int pi_div(int a, int b) {
  int r;
  asm("div.s32 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}
__device__ __forceinline__ int pi_rem(int a, int b) {
  int r;
  asm("rem.s32 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}
__device__ __forceinline__ int pi_shl(int a, int b) {
  int r;
  asm("shl.b32 %0, %1, %2;" : "=r"(r) : "r"(a), "r"((unsigned int)b));
  return r;
}
__device__ __forceinline__ int pi_shr(int a, int b) {
  int r;
  asm("shr.s32 %0, %1, %2;" : "=r"(r) : "r"(a), "r"((unsigned int)b));
  return r;
}

// One instruction over L lanes.  T: long long (s64, the reference's
// registers) or int (a program whose values the matcher proved to give the
// same bits on 32 bits).  Operand lane l is fa(l) / fb(l) / fc(l) and the
// result goes to put(l, value): the callers' operands are register arrays,
// shared-memory slots or one broadcast constant, all resolved at compile time.
template <typename T, int L, typename PUT, typename FA, typename FB, typename FC>
__device__ __forceinline__ void pi_apply(int op, const PUT &put, const FA &fa, const FB &fb,
                                         const FC &fc) {
  using U = typename std::make_unsigned<T>::type;
#define PI_LANES(EXPR)                                                            \
  _Pragma("unroll") for (int j = 0; j < L; ++j) {                                 \
    const T a = fa(j), b = fb(j), c = fc(j);                                      \
    (void)b; (void)c;                                                             \
    put(j, (T)(EXPR));                                                            \
  }                                                                               \
  break;
  switch (op) {
    case PI_COPY: PI_LANES(a)
    case PI_ADD: PI_LANES((T)((U)a + (U)b))
    case PI_SUB: PI_LANES((T)((U)a - (U)b))
    case PI_MUL: PI_LANES((T)((U)a * (U)b))
    case PI_DIV: PI_LANES(pi_div(a, b))
    case PI_REM: PI_LANES(pi_rem(a, b))
    case PI_SHL: PI_LANES(pi_shl(a, b))
    case PI_SHR: PI_LANES(pi_shr(a, b))
    case PI_XOR: PI_LANES(a ^ b)
    case PI_MAX: PI_LANES(a > b ? a : b)
    case PI_MIN: PI_LANES(a < b ? a : b)
    case PI_EQ: PI_LANES((T)(a == b))
    case PI_NE: PI_LANES((T)(a != b))
    case PI_GT: PI_LANES((T)(a > b))
    case PI_LT: PI_LANES((T)(a < b))
    case PI_GE: PI_LANES((T)(a >= b))
    case PI_LE: PI_LANES((T)(a <= b))
    case PI_LAND: PI_LANES((T)((a != 0) & (b != 0)))
    case PI_LOR: PI_LANES((T)((a != 0) | (b != 0)))
    case PI_LNOT: PI_LANES((T)(a == 0))
    default: PI_LANES(a != 0 ? b : c)                  // PI_WHERE
  }
#undef PI_LANES
}

// the same over register slots laid out with lane stride S
template <typename T, int VEC, int S>
__device__ __forceinline__ void pi_step(int op, T *RD, const T *RA, const T *RB, const T *RC) {
  pi_apply<T, VEC>(
      op, [&](int j, T v) { RD[j * S] = v; }, [&](int j) { return RA[j * S]; },
      [&](int j) { return RB[j * S]; }, [&](int j) { return RC[j * S]; });
}

// T: the register type (above).  VIO: every contiguous input and the output
// take vector loads / stores.  BC: some input is a broadcast (read through
// PwIndex).  Operands are widened to s64 as they load (as the reference does)
// and, for T = int, cut to their low 32 bits; results are sign-extended back
// to s64 for the store.
template <typename T, bool VIO, bool BC>
__global__ void __launch_bounds__(kPiThreads)
pointwise_int_kernel(const PiProgram p, void *out, int out_dtype, int64_t n) {
  constexpr int S = kPiThreads, VEC = kPiVec;
  extern __shared__ __align__(16) unsigned char pi_smem[];
  T *R = reinterpret_cast<T *>(pi_smem) + threadIdx.x;   // register r, lane j at R[(r*VEC+j)*S]
  for (int s = 0; s < p.n_sc; ++s) {
    const T v = (T)pi_load1(p.scalars[s], p.sc_dtype[s], 0);
#pragma unroll
    for (int j = 0; j < VEC; ++j) R[((p.n_in + s) * VEC + j) * S] = v;
  }
  for (int s = 0; s < p.n_imm; ++s) {
#pragma unroll
    for (int j = 0; j < VEC; ++j) R[((p.n_in + p.n_sc + s) * VEC + j) * S] = (T)p.imm[s];
  }
  const int64_t groups = (n + VEC - 1) / VEC;
  const int64_t stride = (int64_t)gridDim.x * S;
  for (int64_t g = (int64_t)blockIdx.x * S + threadIdx.x; g < groups; g += stride) {
    const int64_t base = g * VEC;
    const bool full = base + VEC <= n;
    for (int k = 0; k < p.n_in; ++k) {
      long long v[VEC];
      if (BC && p.idx[k].bcast) {
        const PwIndex &x = p.idx[k];
#pragma unroll
        for (int j = 0; j < VEC; ++j) {
          unsigned long long q = pw_div(x.div, (unsigned long long)(p.first + base + j));
          if (x.has_mod) q -= pw_div(x.mod, q) * x.mod.d;
          v[j] = base + j < n ? pi_load1(p.inputs[k], p.in_dtype[k], (int64_t)q) : 0;
        }
      } else if (VIO && full) {
        pi_load4(p.inputs[k], p.in_dtype[k], base, v);
      } else {
#pragma unroll
        for (int j = 0; j < VEC; ++j)
          v[j] = base + j < n ? pi_load1(p.inputs[k], p.in_dtype[k], base + j) : 0;
      }
#pragma unroll
      for (int j = 0; j < VEC; ++j) R[(k * VEC + j) * S] = (T)v[j];
    }
    for (int k = 0; k < p.n_instr; ++k) {
      const signed char *c = p.code[k];
      pi_step<T, VEC, S>(c[0], R + c[1] * VEC * S, R + c[2] * VEC * S, R + c[3] * VEC * S,
                         R + c[4] * VEC * S);
    }
    long long o[VEC];
#pragma unroll
    for (int j = 0; j < VEC; ++j) o[j] = (long long)R[(p.result_reg * VEC + j) * S];
    if (VIO && full) {
      pi_store4(out, out_dtype, base, o);
    } else {
#pragma unroll
      for (int j = 0; j < VEC; ++j)
        if (base + j < n) pi_store1(out, out_dtype, base + j, o[j]);
    }
  }
}

// Chain programs: every step reads the step before it (if it reads a step
// at all) plus inputs and constants -- max(x0 - x1, 0), ((x0 * x1) >> 3) ^ x2
// and the like.  The running value stays in registers (4 * U lanes a thread),
// so no shared register file; the inputs stream into shared memory by bulk
// copies (cp.async.bulk, no multicast) through a ring of `stages` chunks per
// CTA, which keeps many bytes in flight whatever the element width, and every
// step reads its input operands from the staged chunk.  Each step is decoded
// once per chunk and applied to all of the thread's lanes.  Persistent CTAs
// walk chunks of kPcThreads * 4 * U elements (group u of thread t: elements
// (u * kPcThreads + t) * 4 .. + 3); a last partial chunk is read from global
// memory directly.  Operand codes: -1 the previous step's value, 0..7 input
// k, 8 + j constant j (scalars, then immediates).
#ifndef EMMY_PC_GROUPS32
#define EMMY_PC_GROUPS32 4
#endif
#ifndef EMMY_PC_GROUPS64
#define EMMY_PC_GROUPS64 2
#endif
#ifndef EMMY_PC_RING_KB
#define EMMY_PC_RING_KB 72
#endif
constexpr int kPcThreads = 256, kPcMaxStages = 16;
constexpr int kStatusPcWait = 0x1401;

struct PiChain {
  const void *inputs[kPiMaxIn];
  int in_dtype[kPiMaxIn];
  int in_off[kPiMaxIn];                  // byte offset of input k in a staged chunk
  int in_bytes[kPiMaxIn];                // bytes of one chunk of input k
  const void *scalars[kPiMaxIn];
  int sc_dtype[kPiMaxIn];
  long long imm[kPiMaxIn];
  signed char code[kPiMaxInstr][4];      // op, then up to three operand codes
  int64_t n, nfull;                      // elements, full chunks
  int n_in, n_sc, n_imm, n_instr, stages, chunk_bytes;
};

__device__ __forceinline__ int pi_arity(int op) {
  return op == PI_WHERE ? 3 : (op == PI_COPY || op == PI_LNOT) ? 1 : 2;
}

template <typename T, int U, bool VO>
__global__ void __launch_bounds__(kPcThreads)
pointwise_int_chain_kernel(const __grid_constant__ PiChain p, void *out, int out_dtype,
                           int *status) {
  constexpr int L = kPiVec * U;                      // lanes a thread per chunk
  constexpr int CH = kPcThreads * L;                 // elements a chunk
  constexpr int GS = kPcThreads * kPiVec;            // element stride between groups
  extern __shared__ __align__(128) unsigned char pc_smem[];
  __shared__ uint64_t full[kPcMaxStages];
  __shared__ T kc[2 * kPiMaxIn];
  const int tid = threadIdx.x;
  if (tid < p.n_sc) kc[tid] = (T)pi_load1(p.scalars[tid], p.sc_dtype[tid], 0);
  else if (tid < p.n_sc + p.n_imm) kc[tid] = (T)p.imm[tid - p.n_sc];
  if (tid == 0) {
    for (int s = 0; s < p.stages; ++s) mbar_init(&full[s], 1);
    fence_barrier_init();
  }
  __syncthreads();
  const int64_t nchunks = (p.n + CH - 1) / CH;
  auto issue = [&](int64_t c, int s) {               // thread 0: chunk c into stage s
    unsigned char *dst = pc_smem + (size_t)s * p.chunk_bytes;
    mbar_expect_tx(&full[s], (uint32_t)p.chunk_bytes);
    for (int k = 0; k < p.n_in; ++k)
      bulk_load_1d(dst + p.in_off[k], static_cast<const unsigned char *>(p.inputs[k]) +
                   c * p.in_bytes[k], (uint32_t)p.in_bytes[k], &full[s]);
  };
  if (tid == 0)
    for (int s = 0; s < p.stages; ++s) {
      const int64_t c = blockIdx.x + (int64_t)s * gridDim.x;
      if (c < p.nfull) issue(c, s);
    }
  bool ok = true;
  int64_t i = 0;
  int s = 0;                                         // stage of chunk i, and its phase
  uint32_t phase = 0;
  for (;; ++i) {
    const int64_t c = blockIdx.x + i * gridDim.x;
    if (c >= nchunks) break;
    const bool staged = c < p.nfull;
    if (staged) ok = mbar_wait(&full[s], phase, status, kStatusPcWait);
    const int64_t base = c * CH + (int64_t)tid * kPiVec;   // the thread's first group
    if (ok && base < p.n) {
      const unsigned char *stage = pc_smem + (size_t)s * p.chunk_bytes;
      T acc[L];
#pragma unroll
      for (int l = 0; l < L; ++l) acc[l] = 0;
      // input d of this chunk into buf (from the stage, or global memory for
      // the partial chunk)
      auto fetch = [&](int d, T *buf) {
        if (staged) {
          pi_loadv<false, U, T>(stage + p.in_off[d], p.in_dtype[d], (int64_t)tid * kPiVec, GS, buf);
        } else {
#pragma unroll
          for (int u = 0; u < U; ++u)
#pragma unroll
            for (int j = 0; j < kPiVec; ++j) {
              const int64_t e = base + (int64_t)u * GS + j;
              buf[kPiVec * u + j] = e < p.n ? (T)pi_load1(p.inputs[d], p.in_dtype[d], e) : 0;
            }
        }
      };
      for (int k = 0; k < p.n_instr; ++k) {
        const int op = p.code[k][0];
        T a[3][L];
#pragma unroll
        for (int q = 0; q < 3; ++q) {
          if (q >= pi_arity(op)) {
#pragma unroll
            for (int l = 0; l < L; ++l) a[q][l] = 0;
            continue;
          }
          const int d = p.code[k][1 + q];
          if (d < 0) {
#pragma unroll
            for (int l = 0; l < L; ++l) a[q][l] = acc[l];
          } else if (d >= kPiMaxIn) {
            const T v = kc[d - kPiMaxIn];
#pragma unroll
            for (int l = 0; l < L; ++l) a[q][l] = v;
          } else {
            fetch(d, a[q]);
          }
        }
        pi_step<T, L, 1>(op, acc, a[0], a[1], a[2]);
      }
      if (VO && staged) {
        pi_storev<U, T>(out, out_dtype, base, GS, acc);
      } else {
#pragma unroll
        for (int u = 0; u < U; ++u)
#pragma unroll
          for (int j = 0; j < kPiVec; ++j) {
            const int64_t e = base + (int64_t)u * GS + j;
            if (e < p.n) pi_store1(out, out_dtype, e, (long long)acc[kPiVec * u + j]);
          }
      }
    }
    // every thread is done with stage s (and agrees whether a wait gave up)
    if (__syncthreads_or(!ok)) break;
    if (tid == 0) {
      const int64_t cn = blockIdx.x + (i + p.stages) * gridDim.x;
      if (cn < p.nfull) issue(cn, s);
    }
    if (++s == p.stages) {
      s = 0;
      phase ^= 1;
    }
  }
  if (!ok && tid == 0) {
    // a wait gave up: let the copies still in flight into this CTA's shared
    // memory land (each wait bounded) before the CTA exits
    for (int64_t j = i; j < i + p.stages; ++j) {
      const int64_t c = blockIdx.x + j * gridDim.x;
      if (c >= p.nfull) break;
      mbar_wait(&full[s], phase, nullptr, 0);
      if (++s == p.stages) {
        s = 0;
        phase ^= 1;
      }
    }
  }
}

// One-step programs (one op over contiguous inputs and constants: the
// commonest integer program) with the op fixed at compile time: operands in
// registers, no shared register file, two 4-element groups loaded per thread
// before any arithmetic.  Operand kinds: 0 contiguous input, 1 immediate,
// 2 one-element scalar tensor.
struct PiSimple {
  const void *ptr[3];
  int dtype[3];
  int kind[3];
  long long konst[3];
  int nops;
};

// G: 4-element groups per thread -- two on 32-bit values when at most one
// operand streams from memory, else one (s64 with two groups spills; two
// streams run faster with one, as in the float kernel)
template <typename T, int OP, bool VIO, int G>
__global__ void __launch_bounds__(256)
pointwise_int_simple_kernel(const PiSimple q, void *out, int out_dtype, int64_t n) {
  constexpr int VEC = kPiVec;
  const int64_t groups = (n + VEC - 1) / VEC;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  long long cval[3];
#pragma unroll
  for (int k = 0; k < 3; ++k)
    cval[k] = k >= q.nops ? 0 : q.kind[k] == 1 ? q.konst[k]
                              : q.kind[k] == 2 ? pi_load1(q.ptr[k], q.dtype[k], 0) : 0;
  for (int64_t g0 = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; g0 < groups;
       g0 += stride * G) {
    T v[G][3][VEC];
#pragma unroll
    for (int u = 0; u < G; ++u) {
      const int64_t base = (g0 + u * stride) * VEC;
      if (base >= n) break;
#pragma unroll
      for (int k = 0; k < 3; ++k) {
        long long w[VEC];
        if (k >= q.nops || q.kind[k] != 0) {
#pragma unroll
          for (int j = 0; j < VEC; ++j) w[j] = cval[k];
        } else if (VIO && base + VEC <= n) {
          pi_load4(q.ptr[k], q.dtype[k], base, w);
        } else {
#pragma unroll
          for (int j = 0; j < VEC; ++j)
            w[j] = base + j < n ? pi_load1(q.ptr[k], q.dtype[k], base + j) : 0;
        }
#pragma unroll
        for (int j = 0; j < VEC; ++j) v[u][k][j] = (T)w[j];
      }
    }
#pragma unroll
    for (int u = 0; u < G; ++u) {
      const int64_t base = (g0 + u * stride) * VEC;
      if (base >= n) break;
      T r[VEC];
      pi_step<T, VEC, 1>(OP, r, v[u][0], v[u][1], v[u][2]);
      long long o[VEC];
#pragma unroll
      for (int j = 0; j < VEC; ++j) o[j] = (long long)r[j];
      if (VIO && base + VEC <= n) {
        pi_store4(out, out_dtype, base, o);
      } else {
#pragma unroll
        for (int j = 0; j < VEC; ++j)
          if (base + j < n) pi_store1(out, out_dtype, base + j, o[j]);
      }
    }
  }
}

}  // namespace emmy

using namespace emmy;

namespace {

bool pi_dtype_ok(int dt) { return dt >= EMMY_DT_F32 && dt <= EMMY_DT_U64; }

int pi_elem_bytes(int dt) {
  switch (dt) {
    case EMMY_DT_I8: case EMMY_DT_U8: return 1;
    case EMMY_DT_I16: case EMMY_DT_U16: case EMMY_DT_F16: return 2;
    case EMMY_DT_I32: case EMMY_DT_U32: case EMMY_DT_F32: return 4;
    default: return 8;
  }
}

// four consecutive elements from an element index that is a multiple of 4
bool pi_vec_aligned(const void *p, int dt) {
  const uintptr_t need = std::min<uintptr_t>(16, 4 * (uintptr_t)pi_elem_bytes(dt));
  return ((uintptr_t)p % need) == 0;
}

}  // namespace

extern "C" int emmy_pointwise_int(const void *const *inputs, const int *input_dtypes,
                                  const int64_t *input_index, int n_inputs,
                                  const void *const *scalars, const int *scalar_dtypes,
                                  int n_scalars, const int64_t *immediates, int n_imm,
                                  const int *program, int n_instr, int result_reg, void *out,
                                  int out_dtype, int64_t first, int64_t n, int value_bits,
                                  void *stream) {
  clear_error();
  if (n < 0 || first < 0) return set_error(EMMY_ERR_INVALID, "emmy_pointwise_int: negative size");
  if (value_bits != 64 && value_bits != 32)
    return set_error(EMMY_ERR_INVALID, "emmy_pointwise_int: value_bits must be 64 or 32");
  if (n == 0) return EMMY_OK;
  if (!out) return set_error(EMMY_ERR_INVALID, "emmy_pointwise_int: null output");
  if (n_inputs < 0 || n_inputs > kPiMaxIn || n_scalars < 0 || n_scalars > kPiMaxIn || n_imm < 0 ||
      n_imm > kPiMaxIn || n_instr < 1 || n_instr > kPiMaxInstr)
    return set_error(EMMY_ERR_INVALID, "emmy_pointwise_int: program has too many inputs or steps");
  if ((n_inputs && (!inputs || !input_dtypes)) || (n_scalars && (!scalars || !scalar_dtypes)) ||
      (n_imm && !immediates) || !program)
    return set_error(EMMY_ERR_INVALID, "emmy_pointwise_int: null argument array");
  const int nregs = n_inputs + n_scalars + n_imm + n_instr;
  if (nregs > kPiMaxRegs) return set_error(EMMY_ERR_INVALID, "emmy_pointwise_int: too many registers");
  if (result_reg < 0 || result_reg >= nregs)
    return set_error(EMMY_ERR_INVALID, "emmy_pointwise_int: bad result register");
  if (!pi_dtype_ok(out_dtype)) return set_error(EMMY_ERR_INVALID, "emmy_pointwise_int: bad output dtype");
  PiProgram p{};
  p.n_in = n_inputs;
  p.n_sc = n_scalars;
  p.n_imm = n_imm;
  p.n_instr = n_instr;
  p.result_reg = result_reg;
  p.first = first;
  bool vio = pi_vec_aligned(out, out_dtype), bcast = false;
  for (int i = 0; i < n_inputs; ++i) {
    if (!inputs[i]) return set_error(EMMY_ERR_INVALID, "emmy_pointwise_int: null input %d", i);
    if (!pi_dtype_ok(input_dtypes[i]))
      return set_error(EMMY_ERR_INVALID, "emmy_pointwise_int: bad input dtype");
    p.inputs[i] = inputs[i];
    p.in_dtype[i] = input_dtypes[i];
    const int64_t dv = input_index ? input_index[3 * i] : 0;
    if (dv != 0) {
      // broadcast input: ((first + e) / div) % mod must stay inside its numel
      const int64_t md = input_index[3 * i + 1], numel = input_index[3 * i + 2];
      if (dv < 1 || dv >= (int64_t(1) << 62) || md < 0 || md >= (int64_t(1) << 62) || numel < 1)
        return set_error(EMMY_ERR_INVALID, "emmy_pointwise_int: bad index of input %d", i);
      const int64_t top = md > 0 ? std::min<int64_t>(md - 1, (first + n - 1) / dv) : (first + n - 1) / dv;
      if (top >= numel)
        return set_error(EMMY_ERR_INVALID, "emmy_pointwise_int: input %d read past its %lld elements",
                         i, (long long)numel);
      p.idx[i].bcast = 1;
      p.idx[i].div = make_div((unsigned long long)dv);
      p.idx[i].has_mod = md > 0;
      if (md > 0) p.idx[i].mod = make_div((unsigned long long)md);
      bcast = true;
      continue;
    }
    vio = vio && pi_vec_aligned(inputs[i], input_dtypes[i]);
  }
  for (int i = 0; i < n_scalars; ++i) {
    if (!scalars[i]) return set_error(EMMY_ERR_INVALID, "emmy_pointwise_int: null scalar %d", i);
    if (!pi_dtype_ok(scalar_dtypes[i]))
      return set_error(EMMY_ERR_INVALID, "emmy_pointwise_int: bad scalar dtype");
    p.scalars[i] = scalars[i];
    p.sc_dtype[i] = scalar_dtypes[i];
  }
  for (int i = 0; i < n_imm; ++i) p.imm[i] = immediates[i];
  for (int k = 0; k < n_instr; ++k) {
    const int *c = program + 5 * k;
    if (c[0] < 0 || c[0] >= PI_NOPS)
      return set_error(EMMY_ERR_INVALID, "emmy_pointwise_int: unknown opcode %d", c[0]);
    // destinations are the temporaries (never an input, scalar or immediate)
    if (c[1] < n_inputs + n_scalars + n_imm || c[1] >= nregs)
      return set_error(EMMY_ERR_INVALID, "emmy_pointwise_int: step %d writes register %d", k, c[1]);
    for (int j = 2; j < 5; ++j)
      if (c[j] < 0 || c[j] >= nregs)
        return set_error(EMMY_ERR_INVALID, "emmy_pointwise_int: register %d out of range", c[j]);
    for (int j = 0; j < 5; ++j) p.code[k][j] = (signed char)c[j];
  }
  const int64_t groups = (n + kPiVec - 1) / kPiVec;
  cudaStream_t st = as_stream(stream);
  // one step over contiguous inputs and constants: the op-specialised kernel
  const int nleaf = n_inputs + n_scalars + n_imm;
  auto arity = [](int op) { return op == PI_WHERE ? 3 : (op == PI_COPY || op == PI_LNOT) ? 1 : 2; };
  bool simple = !bcast && n_instr == 1 && result_reg == nleaf;
  for (int j = 0; simple && j < arity(program[0]); ++j) simple = program[2 + j] < nleaf;
  auto launch_simple = [&]() -> int {
    const int op = program[0];
    PiSimple q{};
    q.nops = arity(op);
    for (int j = 0; j < q.nops; ++j) {
      const int r = program[2 + j];
      if (r < n_inputs) {
        q.kind[j] = 0; q.ptr[j] = p.inputs[r]; q.dtype[j] = p.in_dtype[r];
      } else if (r < n_inputs + n_scalars) {
        q.kind[j] = 2; q.ptr[j] = p.scalars[r - n_inputs]; q.dtype[j] = p.sc_dtype[r - n_inputs];
      } else {
        q.kind[j] = 1; q.konst[j] = p.imm[r - n_inputs - n_scalars];
      }
    }
    int streams = 0;
    for (int j = 0; j < q.nops; ++j) streams += q.kind[j] == 0;
    const bool two = value_bits == 32 && streams <= 1;
    const int64_t G = two ? 2 : 1;
    int64_t sblocks = (groups + 256LL * G - 1) / (256LL * G);
    if (sblocks > INT32_MAX) sblocks = INT32_MAX;
    const unsigned sb = (unsigned)sblocks;
#define EMMY_PI_SIMPLE(OPC)                                                                          \
  case OPC:                                                                                          \
    if (value_bits == 32 && two) {                                                                   \
      if (vio) pointwise_int_simple_kernel<int, OPC, true, 2><<<sb, 256, 0, st>>>(q, out, out_dtype, n); \
      else pointwise_int_simple_kernel<int, OPC, false, 2><<<sb, 256, 0, st>>>(q, out, out_dtype, n); \
    } else if (value_bits == 32) {                                                                   \
      if (vio) pointwise_int_simple_kernel<int, OPC, true, 1><<<sb, 256, 0, st>>>(q, out, out_dtype, n); \
      else pointwise_int_simple_kernel<int, OPC, false, 1><<<sb, 256, 0, st>>>(q, out, out_dtype, n); \
    } else {                                                                                         \
      if (vio) pointwise_int_simple_kernel<long long, OPC, true, 1><<<sb, 256, 0, st>>>(q, out, out_dtype, n); \
      else pointwise_int_simple_kernel<long long, OPC, false, 1><<<sb, 256, 0, st>>>(q, out, out_dtype, n); \
    }                                                                                                \
    break;
    switch (op) {
      EMMY_PI_SIMPLE(PI_COPY) EMMY_PI_SIMPLE(PI_ADD) EMMY_PI_SIMPLE(PI_SUB) EMMY_PI_SIMPLE(PI_MUL)
      EMMY_PI_SIMPLE(PI_DIV) EMMY_PI_SIMPLE(PI_REM) EMMY_PI_SIMPLE(PI_SHL) EMMY_PI_SIMPLE(PI_SHR)
      EMMY_PI_SIMPLE(PI_XOR) EMMY_PI_SIMPLE(PI_MAX) EMMY_PI_SIMPLE(PI_MIN) EMMY_PI_SIMPLE(PI_EQ)
      EMMY_PI_SIMPLE(PI_NE) EMMY_PI_SIMPLE(PI_GT) EMMY_PI_SIMPLE(PI_LT) EMMY_PI_SIMPLE(PI_GE)
      EMMY_PI_SIMPLE(PI_LE) EMMY_PI_SIMPLE(PI_LAND) EMMY_PI_SIMPLE(PI_LOR) EMMY_PI_SIMPLE(PI_LNOT)
      default: EMMY_PI_SIMPLE(PI_WHERE)
    }
#undef EMMY_PI_SIMPLE
    return check_launch("emmy_pointwise_int (one step)");
  };
  // narrow streams (1- and 2-byte elements) go to the staged kernel below,
  // where bulk copies keep enough bytes in flight
  bool narrow = false;
  for (int i = 0; i < n_inputs; ++i) narrow = narrow || pi_elem_bytes(input_dtypes[i]) < 4;
  if (simple && !narrow) return launch_simple();
  // a chain program over 16-byte aligned contiguous inputs: the staged kernel
  // (four groups of four lanes a thread on 32-bit values, two on s64 ones)
  const int pc_groups = value_bits == 32 ? EMMY_PC_GROUPS32 : EMMY_PC_GROUPS64;
  const int64_t pc_chunk = (int64_t)kPcThreads * kPiVec * pc_groups;
  if (!bcast && n_inputs > 0 && (n_instr >= 2 || simple) && n >= pc_chunk) {
    PiChain c{};
    bool chain = true;
    int writer[kPiMaxRegs];
    for (int r = 0; r < kPiMaxRegs; ++r) writer[r] = -1;
    int chunk_bytes = 0;
    for (int k = 0; k < n_inputs; ++k) {
      chain = chain && ((uintptr_t)inputs[k] % 16) == 0;
      c.inputs[k] = p.inputs[k];
      c.in_dtype[k] = p.in_dtype[k];
      c.in_off[k] = chunk_bytes;
      c.in_bytes[k] = (int)pc_chunk * pi_elem_bytes(p.in_dtype[k]);
      chunk_bytes += c.in_bytes[k];
    }
    for (int k = 0; chain && k < n_instr; ++k) {
      const int *ins = program + 5 * k;
      c.code[k][0] = (signed char)ins[0];
      for (int q = 0; q < 3; ++q) {
        int d = 0;
        if (q < arity(ins[0])) {
          const int r = ins[2 + q];
          if (r < n_inputs) d = r;
          else if (r < nleaf) d = kPiMaxIn + (r - n_inputs);
          else if (k > 0 && writer[r] == k - 1) d = -1;
          else chain = false;                       // reads an older step: not a chain
        }
        c.code[k][1 + q] = (signed char)d;
      }
      writer[ins[1]] = k;
    }
    chain = chain && result_reg >= nleaf && writer[result_reg] == n_instr - 1 &&
            2 * chunk_bytes <= 192 * 1024;                 // two stages fit shared memory
    if (chain) {
      c.n = n;
      c.nfull = n / pc_chunk;
      c.n_in = n_inputs;
      c.n_sc = n_scalars;
      c.n_imm = n_imm;
      c.n_instr = n_instr;
      for (int k = 0; k < n_scalars; ++k) {
        c.scalars[k] = p.scalars[k];
        c.sc_dtype[k] = p.sc_dtype[k];
      }
      for (int k = 0; k < n_imm; ++k) c.imm[k] = p.imm[k];
      c.chunk_bytes = chunk_bytes;
      const int64_t nchunks = (n + pc_chunk - 1) / pc_chunk;
      const bool vo = pi_vec_aligned(out, out_dtype);
      auto go = [&](auto kern) {
        // the CTAs that the registers let reside on an SM share EMMY_PC_RING_KB
        // of staged chunks, two to sixteen stages each (72 KB measured as good
        // as 200 KB: past a few chunks in flight the issue rate bounds it)
        int per_sm = 1;
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kPcThreads, 0);
        per_sm = std::max(per_sm, 1);
        c.stages = std::max(2, std::min(kPcMaxStages, (EMMY_PC_RING_KB * 1024 / per_sm) / chunk_bytes));
        const size_t smem = (size_t)c.stages * chunk_bytes;
        // (the kernel's own barriers and constants take the static part)
        if (smem + 1024 > 48 * 1024)
          cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kPcThreads, smem);
        const unsigned grid =
            (unsigned)std::min<int64_t>(nchunks, (int64_t)std::max(per_sm, 1) * sm_count());
        kern<<<grid, kPcThreads, smem, st>>>(c, out, out_dtype, device_status_ptr());
      };
      if (value_bits == 32) {
        if (vo) go(pointwise_int_chain_kernel<int, EMMY_PC_GROUPS32, true>);
        else go(pointwise_int_chain_kernel<int, EMMY_PC_GROUPS32, false>);
      } else {
        if (vo) go(pointwise_int_chain_kernel<long long, EMMY_PC_GROUPS64, true>);
        else go(pointwise_int_chain_kernel<long long, EMMY_PC_GROUPS64, false>);
      }
      return check_launch("emmy_pointwise_int (chain)");
    }
  }
  if (simple) return launch_simple();
  const size_t smem = (size_t)nregs * kPiVec * kPiThreads * (value_bits / 8);
  int64_t blocks = (groups + kPiThreads - 1) / kPiThreads;
  if (blocks > INT32_MAX) blocks = INT32_MAX;             // the grid-stride loop covers the rest
  auto launch = [&](auto kern) {
    if (smem > 48 * 1024) cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    kern<<<(unsigned)blocks, kPiThreads, smem, st>>>(p, out, out_dtype, n);
  };
  if (value_bits == 32) {
    if (bcast) {
      if (vio) launch(pointwise_int_kernel<int, true, true>);
      else launch(pointwise_int_kernel<int, false, true>);
    } else {
      if (vio) launch(pointwise_int_kernel<int, true, false>);
      else launch(pointwise_int_kernel<int, false, false>);
    }
  } else if (bcast) {
    if (vio) launch(pointwise_int_kernel<long long, true, true>);
    else launch(pointwise_int_kernel<long long, false, true>);
  } else {
    if (vio) launch(pointwise_int_kernel<long long, true, false>);
    else launch(pointwise_int_kernel<long long, false, false>);
  }
  return check_launch("emmy_pointwise_int");
}
