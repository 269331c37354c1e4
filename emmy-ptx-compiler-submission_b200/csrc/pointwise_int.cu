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

// elements base .. base + 3 (aligned for one or two vector loads)
__device__ __forceinline__ void pi_load4(const void *p, int dt, int64_t base, long long v[4]) {
  switch (dt) {
    case EMMY_DT_I8:
    case EMMY_DT_U8: {
      const unsigned int w = __ldg(reinterpret_cast<const unsigned int *>(
          static_cast<const unsigned char *>(p) + base));
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const unsigned int b = (w >> (8 * j)) & 0xffu;
        v[j] = dt == EMMY_DT_I8 ? (long long)(signed char)b : (long long)b;
      }
      break;
    }
    case EMMY_DT_I16:
    case EMMY_DT_U16:
    case EMMY_DT_F16: {
      const uint2 w = __ldg(reinterpret_cast<const uint2 *>(
          static_cast<const unsigned short *>(p) + base));
      const unsigned int h[4] = {w.x & 0xffffu, w.x >> 16, w.y & 0xffffu, w.y >> 16};
#pragma unroll
      for (int j = 0; j < 4; ++j)
        v[j] = dt == EMMY_DT_I16   ? (long long)(short)h[j]
               : dt == EMMY_DT_U16 ? (long long)h[j]
                                   : pi_rzi_f16((unsigned short)h[j]);
      break;
    }
    case EMMY_DT_I32:
    case EMMY_DT_U32: {
      const uint4 w = __ldg(reinterpret_cast<const uint4 *>(static_cast<const int *>(p) + base));
      const unsigned int u[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
      for (int j = 0; j < 4; ++j)
        v[j] = dt == EMMY_DT_I32 ? (long long)(int)u[j] : (long long)u[j];
      break;
    }
    case EMMY_DT_F32: {
      const float4 w = __ldg(reinterpret_cast<const float4 *>(static_cast<const float *>(p) + base));
      v[0] = pi_rzi_f32(w.x); v[1] = pi_rzi_f32(w.y); v[2] = pi_rzi_f32(w.z); v[3] = pi_rzi_f32(w.w);
      break;
    }
    case EMMY_DT_F64: {
      const double2 *q = reinterpret_cast<const double2 *>(static_cast<const double *>(p) + base);
      const double2 a = __ldg(q), b = __ldg(q + 1);
      v[0] = pi_rzi_f64(a.x); v[1] = pi_rzi_f64(a.y); v[2] = pi_rzi_f64(b.x); v[3] = pi_rzi_f64(b.y);
      break;
    }
    default: {                                         // I64, U64
      const longlong2 *q = reinterpret_cast<const longlong2 *>(static_cast<const long long *>(p) + base);
      const longlong2 a = __ldg(q), b = __ldg(q + 1);
      v[0] = a.x; v[1] = a.y; v[2] = b.x; v[3] = b.y;
      break;
    }
  }
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

__device__ __forceinline__ void pi_store4(void *p, int dt, int64_t base, const long long v[4]) {
  unsigned long long u[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) u[j] = (unsigned long long)v[j];
  switch (dt) {
    case EMMY_DT_I8:
    case EMMY_DT_U8:
      *reinterpret_cast<unsigned int *>(static_cast<unsigned char *>(p) + base) =
          (unsigned int)(u[0] & 0xff) | (unsigned int)(u[1] & 0xff) << 8 |
          (unsigned int)(u[2] & 0xff) << 16 | (unsigned int)(u[3] & 0xff) << 24;
      break;
    case EMMY_DT_I16:
    case EMMY_DT_U16:
      *reinterpret_cast<uint2 *>(static_cast<unsigned short *>(p) + base) =
          make_uint2((unsigned int)(u[0] & 0xffff) | (unsigned int)(u[1] & 0xffff) << 16,
                     (unsigned int)(u[2] & 0xffff) | (unsigned int)(u[3] & 0xffff) << 16);
      break;
    case EMMY_DT_F16:
      *reinterpret_cast<uint2 *>(static_cast<unsigned short *>(p) + base) =
          make_uint2((unsigned int)pi_f16_of(v[0]) | (unsigned int)pi_f16_of(v[1]) << 16,
                     (unsigned int)pi_f16_of(v[2]) | (unsigned int)pi_f16_of(v[3]) << 16);
      break;
    case EMMY_DT_I32:
    case EMMY_DT_U32:
      *reinterpret_cast<uint4 *>(static_cast<unsigned int *>(p) + base) =
          make_uint4((unsigned int)u[0], (unsigned int)u[1], (unsigned int)u[2], (unsigned int)u[3]);
      break;
    case EMMY_DT_F32:
      *reinterpret_cast<float4 *>(static_cast<float *>(p) + base) =
          make_float4(pi_f32_of(v[0]), pi_f32_of(v[1]), pi_f32_of(v[2]), pi_f32_of(v[3]));
      break;
    case EMMY_DT_F64: {
      double2 *q = reinterpret_cast<double2 *>(static_cast<double *>(p) + base);
      q[0] = make_double2(pi_f64_of(v[0]), pi_f64_of(v[1]));
      q[1] = make_double2(pi_f64_of(v[2]), pi_f64_of(v[3]));
      break;
    }
    default: {                                         // I64, U64
      longlong2 *q = reinterpret_cast<longlong2 *>(static_cast<long long *>(p) + base);
      q[0] = make_longlong2(v[0], v[1]);
      q[1] = make_longlong2(v[2], v[3]);
      break;
    }
  }
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

// T: long long (s64, the reference's registers) or int (a program whose
// values the matcher proved to give the same bits on 32 bits).
template <typename T, int VEC, int S>
__device__ __forceinline__ void pi_step(int op, T *RD, const T *RA, const T *RB, const T *RC) {
  using U = typename std::make_unsigned<T>::type;
#define PI_LANES(EXPR)                                                            \
  _Pragma("unroll") for (int j = 0; j < VEC; ++j) {                               \
    const T a = RA[j * S], b = RB[j * S], c = RC[j * S];                          \
    (void)b; (void)c;                                                             \
    RD[j * S] = (EXPR);                                                           \
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
  if (simple) {
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
  }
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
