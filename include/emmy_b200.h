/*
 * emmy_b200.h -- C ABI of libemmyb200.so, the B200 (sm_100a) kernels that run
 * the kernel families the Emmy Kernel IR describes.
 *
 * The reference compiler turns one KernelOp into one PTX entry,
 *   .visible .entry <name>(.param .u64 param_<arg>, ...)   in meta "arg_order",
 * assembled and launched by the caller under the meta.json geometry
 * (reference ptxc/lower.py:549-595 assembles the module, ptxc/lower.py:616-648
 * declares one u64 pointer parameter per argument; tools/localrun.py:102-142
 * launches it).  Each function below replaces that entry for one family of IR
 * shapes.  Like the reference entries, every tensor and every one-element
 * "data" constant (eps, count, the attention divisor) arrives as a device
 * pointer; the launch geometry is chosen here, not taken from meta.json.
 *
 * Conventions
 *   - All pointers are device pointers on the current device.  The caller owns
 *     every buffer; the library allocates no device memory.
 *   - `stream` is a cudaStream_t (NULL = legacy default stream).  Calls are
 *     asynchronous and stream-ordered.
 *   - Return value: EMMY_OK (0) or an error code.  Argument checks run on the
 *     host before any launch; emmy_last_error() returns the message of the
 *     calling thread's last failure.  Nothing calls abort/exit/__trap.
 *   - int64 sizes; tensors are dense row-major unless a stride says otherwise.
 */
#ifndef EMMY_B200_H
#define EMMY_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define EMMY_OK 0
#define EMMY_ERR_INVALID 1      /* bad size, pointer, alignment or enum value */
#define EMMY_ERR_CUDA 2         /* a CUDA runtime call or launch failed */
#define EMMY_ERR_UNSUPPORTED 3  /* valid request this build has no kernel for */
#define EMMY_ERR_DEVICE 4       /* a kernel reported a device-side error */

/* reduction ops / pre-maps for emmy_reduce_f32 */
#define EMMY_REDUCE_SUM 0
#define EMMY_REDUCE_MAX 1
#define EMMY_REDUCE_MIN 2
#define EMMY_PRE_IDENTITY 0
#define EMMY_PRE_SQUARE 1
#define EMMY_PRE_ABS 2

/* row normalisation modes for emmy_rownorm_f32 */
#define EMMY_NORM_RMS 0
#define EMMY_NORM_L2 1
#define EMMY_NORM_LAYER 2

/* element dtypes */
#define EMMY_DT_F32 0
#define EMMY_DT_F16 1
#define EMMY_DT_F64 2
/* integer buffers (emmy_pointwise_int only) */
#define EMMY_DT_I8 3
#define EMMY_DT_U8 4
#define EMMY_DT_I16 5
#define EMMY_DT_U16 6
#define EMMY_DT_I32 7
#define EMMY_DT_U32 8
#define EMMY_DT_I64 9
#define EMMY_DT_U64 10

/* GEMM epilogue bits, applied in this order: round the f32 product to f16
 * (ROUND_F16; emmy_gemm_f16 only: the f16 intermediate of a matmul kernel
 * followed by a separate bias/ReLU kernel), add bias[n], ReLU. */
#define EMMY_EPI_BIAS 1
#define EMMY_EPI_RELU 2
#define EMMY_EPI_ROUND_F16 4

/* Library version (major*10000 + minor*100 + patch). */
int emmy_version(void);

/* Message of the calling thread's last failed call ("" if none). */
const char *emmy_last_error(void);

/* Read and clear the device status word that kernels with bounded waits set
 * (0 = no error).  Synchronises `stream` first. */
int emmy_get_device_status(int *code, void *stream);

/* Zero `bytes` bytes at `ptr` on `stream` (the meta.json "zero_outputs" step the
 * reference harness performs before an atomic split-K launch,
 * reference tools/prof.py:386 and ptxc/stmts.py:1626-1681). */
int emmy_zero(void *ptr, size_t bytes, void *stream);

/*
 * Reduction over the middle axis of the view x[outer, n, inner] into
 * y[outer, inner]:  y = fold_op(pre(x)) [* 1/count].
 * Replaces the entry the reference emits for the "cooperative reduction"
 * shape: a StridedLoop with an Accum, WarpShuffle, shared slots and a
 * TreeHalve, then a Cond(co == 0) write (reference ptxc/stmts.py:728-773,
 * 564-611, 1441-1568; fixtures v_r_*, w_r_*).  Seeds follow
 * ptxc/ops.py:67-75 (max starts at -1e30).  `count` (nullable) is the
 * one-element f32 buffer the IR divides by for a mean.  `workspace` (nullable)
 * lets a single long row (outer*inner == 1) be split over many CTAs;
 * emmy_reduce_workspace_bytes() gives its size.
 */
int emmy_reduce_f32(const float *x, float *y, int64_t outer, int64_t n, int64_t inner,
                    int op, int pre, const float *count, void *workspace,
                    size_t workspace_bytes, void *stream);
size_t emmy_reduce_workspace_bytes(int64_t outer, int64_t n, int64_t inner);

/*
 * Row normalisation of contiguous rows x[rows, cols] into y (same shape):
 *   RMS:   y = x * recip(sqrt(eps + sum(x*x) * recip(count))) [* w]
 *   L2:    y = x * recip(sqrt(sum(x*x)))
 *   LAYER: y = (x - mean) * recip(sqrt(var + eps)) [* w] [+ b]
 * Replaces the reduction-then-map entry of fixtures v_f_rms_512,
 * w_f_rms_2048, v_f_l2_256 (reference ptxc/stmts.py:728-773 for the two
 * StridedLoop passes) and the layernorm shape of
 * reference tools/specs/ln_specs.py:2-6.  w/b are [cols] (nullable); eps and
 * count are one-element f32 device buffers (nullable: eps 0, count = cols).
 */
int emmy_rownorm_f32(const float *x, const float *w, const float *b, float *y,
                     int64_t rows, int64_t cols, const float *eps, const float *count,
                     int mode, void *stream);

/*
 * Softmax over the middle axis of x[outer, n, inner] into y (same shape):
 *   y = exp(x - max) * recip(sum(exp(x - max))).
 * Replaces the online max/sum entry of fixtures v_f_softmax_*,
 * w_f_softmax_2048 (inner == 1) and w_f_softmax_dim0 (inner > 1)
 * (reference ptxc/stmts.py:564-611 for the rescaled Accum pair,
 * ptxc/expr.py:891-895 for exp).
 */
int emmy_softmax_f32(const float *x, float *y, int64_t outer, int64_t n, int64_t inner,
                     void *stream);

/*
 * Row families over f16 / f32 / f64 tensors in any mix, x viewed as
 * [outer, n, inner] (inner > 1: reductions and softmax only):
 *   mode 0/1/2  y[o, i] = sum / max / min over n of pre(x)   (pre: EMMY_PRE_*;
 *               count non-null: y = sum * 1/count, the IR's mean)
 *   mode 3      softmax over n
 *   mode 4/5/6  rms / l2 / layer normalisation of each row (w, b nullable;
 *               eps, count one-element buffers as in emmy_rownorm_f32)
 *   mode 7      y[o] = sum_j x[o, j] * w[j]  (dot with a row-invariant vector)
 * Dtypes are EMMY_DT_*: x_dtype, y_dtype, wb_dtype (w and b), const_dtype
 * (eps, count).  compute_f64 computes in double, else float; the result is
 * rounded once, at the store.  Replaces the entries the reference emits for
 * these IR shapes with f16 or f64 types (f16 widened to f32,
 * reference ptxc/expr.py:168-180; f64 arithmetic ptxc/expr.py:1179-1309).
 */
int emmy_rowop(const void *x, int x_dtype, const void *w, const void *b, int wb_dtype, void *y,
               int y_dtype, int64_t outer, int64_t n, int64_t inner, int mode, int pre,
               const void *eps, const void *count, int const_dtype, int compute_f64,
               void *stream);

/*
 * f64 matrix-vector product y[rows] = A[rows, cols] @ v[cols].
 * Replaces the entry the reference emits for the dot-with-vector reduction
 * shape (StridedLoop over a row with Load A, Load v, multiply, Accum add, then
 * the warp/tree combine; reference ptxc/stmts.py:728-773, 564-611 and the f64
 * arithmetic of ptxc/expr.py:1179-1309).  Products are fused into FMAs.
 */
int emmy_matvec_f64(const double *A, const double *v, double *y, int64_t rows, int64_t cols,
                    void *stream);

/*
 * f32 GEMM on CUDA cores: C[b] (+)= A[b] @ B[b] (+ bias[n]) (ReLU), A [M,K],
 * B [K,N], C [M,N] row-major, batch strides in elements.  `splits` K
 * partitions (0 = choose) are combined with atomic adds, the reference's
 * atomic Write of a split-K Tile axis; `accumulate` adds into C instead of
 * overwriting it.  Replaces the entry the reference emits for the tiled
 * matmul shape (reference ptxc/stmts.py:663-725, 614-632, 1590-1623,
 * 434-487; fixtures v_m_*, w_m_*).
 */
int emmy_gemm_f32(const float *A, const float *B, const float *bias, float *C, int64_t batch,
                  int64_t M, int64_t N, int64_t K, int64_t a_batch_stride,
                  int64_t b_batch_stride, int64_t c_batch_stride, int splits, int accumulate,
                  int epilogue, void *stream);

/*
 * f64 GEMM on CUDA cores (DFMA; the tensor cores have no f64 kind on sm_100a):
 * the emmy_gemm_f32 contract on doubles -- C[b] (+)= A[b] @ B[b] (+ bias[n])
 * (ReLU), split-K partials combined with f64 atomic adds.  Replaces the entry
 * the reference emits for the tiled matmul shape with f64 operands
 * (fma.rn.f64 accumulate, reference ptxc/expr.py:1179-1309, ptxc/stmts.py:614-632).
 */
int emmy_gemm_f64(const double *A, const double *B, const double *bias, double *C, int64_t batch,
                  int64_t M, int64_t N, int64_t K, int64_t a_batch_stride,
                  int64_t b_batch_stride, int64_t c_batch_stride, int splits, int accumulate,
                  int epilogue, void *stream);

/*
 * One rank's K slice of a matmul split across the GPUs of a node, fused with
 * the reduce-scatter of the partial sums: C_part = A[M, Kslice] @ B[Kslice, N]
 * (+ bias: pass it on one rank only, or it joins the sum once per rank) is
 * stored, row by row, into the owners' slot buffers.  Owner o (rows
 * [o * rows_per_rank, (o + 1) * rows_per_rank) of C) holds a slot buffer
 * rows[o] of [world, rows_per_rank, N] floats (slot_floats floats, checked to
 * be at least world * rows_per_rank * N); rank `me` writes only slot `me` of
 * each owner (plain 16-byte stores, over NVLink for another GPU's rows), so
 * nothing needs zeroing and no atomics cross NVLink.  The owner then sums its
 * `world` slots (emmy_reduce_f32 over the slot axis).  rows[] holds every
 * owner's buffer in this process's address space (emmy_ipc_import).  When the
 * K slice is split inside the rank (splits > 1, or splits = 0 and the library
 * widens the split to fill the GPU), the splits of each 128 x 128 tile first
 * sum in `workspace` (M x N floats, local) and the last split to arrive at
 * the tile (tile_counters: at least ceil(M / 64) * ceil(N / 64) ints) stores
 * it, so each element crosses NVLink once; workspace and counters must be
 * zero before the first call and are left zero.  The multi-GPU form of the
 * reference's atomic split-K Write (reference ptxc/stmts.py:456-461), one
 * kernel instead of GEMM + collective.
 */
int emmy_gemm_f32_rows_to_peers(const float *A, const float *B, const float *bias,
                                float *const *rows, int64_t slot_floats, int world, int me,
                                int64_t rows_per_rank, int64_t M, int64_t N, int64_t K,
                                int splits, float *workspace, int *tile_counters,
                                int64_t n_counters, void *stream);

/*
 * CUDA IPC for peer mappings between the processes of one node.  export: the
 * 64-byte handle of the allocation holding ptr and ptr's offset in it.
 * import: map a peer's handle; *peer_ptr = mapped base + offset, *peer_base
 * the base to pass to emmy_ipc_close.
 */
int emmy_ipc_export(const void *ptr, void *handle, int64_t *offset);
int emmy_ipc_import(const void *handle, int64_t offset, void **peer_ptr, void **peer_base);
int emmy_ipc_close(void *peer_base);

/*
 * Reduce-scatter of split-K partials over peer memory (the exchange after a
 * matmul whose K is split across GPUs; the multi-GPU form of the reference's
 * atomic split-K writes, ptxc/stmts.py:456-461).  parts[r]: rank r's full-size
 * [M, n] f32 partial of this step (mapped with emmy_ipc_import; this rank's
 * own at parts[me]); flags[r]: rank r's int64 flag words [world], zero before
 * the first step.  The kernel stores `seq` into flags[r][me] for every r
 * (system-scope release), waits until flags[me][q] >= seq for every q
 * (system-scope acquire, bounded: after the wait limit it records status 0x1301
 * in the device status word and writes nothing), then writes
 * out[i][:] = sum_r parts[r][row0 + i][:] for i < rows.  Launch it after the
 * GEMM that filled parts[me], on the same stream; seq starts at 1 and grows by
 * one per step, and each rank alternates two partial buffers by step parity
 * (a buffer of step s is rewritten at step s + 2, after every rank has passed
 * its wait of step s + 1, so no rank still reads it).  world <= 8.
 */
int emmy_peer_reduce_rows(const float *const *parts, long long *const *flags, int world, int me,
                          long long seq, int64_t row0, int64_t rows, int64_t n, float *out,
                          void *stream);

/*
 * f16 GEMM with f32 accumulation on the tcgen05 tensor cores:
 * C[b] = A[b] @ B[b] (+ bias[n]) (ReLU), A [M,K] f16, B [K,N] f16 row-major,
 * C [M,N] f32 or f16 (out_dtype), bias f32 (nullable), dense batches.
 * Replaces the entry the reference emits for the tiled matmul shape with f16
 * operands (f16 loads widened to f32, reference ptxc/expr.py:168-180, then
 * ptxc/stmts.py:614-632 and the converting Write, ptxc/stmts.py:434-487).
 * `accumulate` must be 0.
 */
int emmy_gemm_f16(const void *A, const void *B, const float *bias, void *C, int64_t batch,
                  int64_t M, int64_t N, int64_t K, int out_dtype, int epilogue, int accumulate,
                  void *stream);

/*
 * Attention-like chain, f32 on CUDA cores, per batch-head b:
 *   o[b] = softmax(q[b] @ k[b]^T * recip(*scale_div)) @ v[b]
 * q [B, Sq, D], k [B, Sk, D] (or, with k_transposed, kt [B, D, Sk]),
 * v [B, Sk, Dv], o [B, Sq, Dv]; scale_div (nullable: 1) is the one-element
 * divisor constant.  Replaces the entry the reference emits for the
 * matmul -> softmax -> reduce fixtures v_a_*, w_a_* (reference
 * ptxc/stmts.py:663-725, 564-611, 1311-1392).
 */
int emmy_attention_f32(const float *q, const float *k, const float *v, float *o,
                       const float *scale_div, int64_t batch, int64_t sq, int64_t sk, int64_t d,
                       int64_t dv, int k_transposed, void *stream);

/*
 * Attention-like chain, f16 in, f32 softmax and accumulation, per batch-head b:
 *   o[b] = softmax(q[b] @ k[b]^T * recip(*scale_div)) @ v[b]
 * q, k, v, o [B, S, D]; sq == sk with D a multiple of 8 up to 256 and
 * 16-byte aligned tensors run on the tcgen05 tensor cores (S = Q K^T and
 * O += P V accumulate in tensor memory; a D below 64 / 128 / 256 runs the
 * kernel of that width with the missing columns zero-filled); other shapes,
 * or k pre-transposed [B, D, Sk], run on CUDA cores; o f16 or f32.
 * Replaces the entry the reference emits for the attention IR shape
 * (reference ptxc/stmts.py:663-725, 564-611, 1311-1392) with f16 operands.
 */
int emmy_attention_f16(const void *q, const void *k, const void *v, void *o,
                       const float *scale_div, int64_t batch, int64_t sq, int64_t sk, int64_t d,
                       int out_dtype, int k_transposed, void *stream);

/*
 * Elementwise chain: out[i] = program(inputs[0][i], ..., *scalars[0], ..., immediates)
 * for i in [0, n).  Replaces the entry the reference emits for its pointwise
 * IR shape (reference ptxc/stmts.py:73-145, 434-487, 510-560; float ops
 * ptxc/expr.py:880-1089, ptxc/ops.py:81-96).
 * Registers: 0..n_inputs-1 hold the element of each input (EMMY_DT_*), then one
 * per one-element scalar tensor, then one per immediate, then one per program
 * step.  program holds n_instr rows {opcode, dst, a, b, c}; opcodes are the
 * table in ptxc/match_pointwise.py (OPCODES): 0 copy, 1 add, 2 subtract,
 * 3 multiply, 4 divide, 5 maximum, 6 minimum, 7 negative, 8 abs, 9 exp, 10 log,
 * 11 sqrt, 12 rsqrt, 13 reciprocal, 14 tanh, 15 sigmoid, 16 relu, 17 greater,
 * 18 less, 19 greater_equal, 20 less_equal, 21 equal, 22 where(a, b, c),
 * 23 round to f16, 24 fma, 25 log2, 26 log10, 27 cos, 28 sin, 29 tan, 30 erf,
 * 31 gelu, 32 gelu_tanh, 33 softplus, 34 exp2, 35 silu, 36 pow, 37 floor,
 * 38 ceil, 39 sign, 40 not_equal (unordered: true when either side is NaN).
 * Comparisons give 1 or 0.  compute_f64 selects double
 * arithmetic, else f32; add/subtract/multiply/divide/sqrt/fma are correctly
 * rounded and never contracted.  Limits: 8 inputs, 8 scalars, 8 immediates,
 * 48 steps, 32 registers in all.
 */
int emmy_pointwise(const void *const *inputs, const int *input_dtypes, int n_inputs,
                   const void *const *scalars, const int *scalar_dtypes, int n_scalars,
                   const double *immediates, int n_imm, const int *program, int n_instr,
                   int result_reg, int compute_f64, void *out, int out_dtype, int64_t n,
                   void *stream);

/*
 * emmy_pointwise with broadcast inputs (the bias of a matmul + bias + ReLU
 * chain, a per-row scale): input i is read at
 *   ((first + e) / div_i) % mod_i        (mod_i = 0: no modulo)
 * for element e of [0, n), or at e when div_i = 0 (contiguous, as in
 * emmy_pointwise).  input_index holds {div_i, mod_i, numel_i} per input;
 * numel_i bounds the broadcast reads (checked on the host).  first offsets
 * the element numbering, so a range [first, first + n) of a larger launch
 * (a shard, a pipeline chunk) reads the same broadcast elements.  The
 * reference reads such inputs through the decoded Tile axes
 * (ptxc/lower.py:787-812) at a flat index that is a row-major form of them
 * (ptxc/memory.py:150-186).
 */
int emmy_pointwise_indexed(const void *const *inputs, const int *input_dtypes,
                           const int64_t *input_index, int n_inputs,
                           const void *const *scalars, const int *scalar_dtypes, int n_scalars,
                           const double *immediates, int n_imm, const int *program, int n_instr,
                           int result_reg, int compute_f64, void *out, int out_dtype,
                           int64_t first, int64_t n, void *stream);

/*
 * Integer pointwise program: out[e] = program(inputs at e, scalars, immediates)
 * for e < n, evaluated on signed 64-bit values.  Replaces the entry the
 * reference emits for a pointwise IR whose Assigns are integer-typed
 * (ptxc/stmts.py:509-560, INT_BINARY in ptxc/ops.py:98-117, operand widening
 * ptxc/expr.py:157-165 and 211-223, div / rem :697-716, predicates and where
 * :815-877, the converting store :233-280).
 * Inputs, scalars and the output may be any EMMY_DT_* type.  An integer
 * element is sign- or zero-extended to s64, a float one truncated toward zero
 * (cvt.rzi.s64: clamped to the s64 range, NaN to -2^63); the result is stored as
 * its low bits (integer output) or rounded to nearest (float output; f16 via
 * f32).  input_index: NULL, or per input three int64 [div, mod, numel] --
 * div 0: contiguous, else the input is read at ((first + e) / div) % mod
 * (mod 0: no modulo) and every read must stay below numel.
 * program: n_instr rows of five ints [opcode, dst, a, b, c] over registers
 * 0..n_inputs-1 (inputs), then the scalars, the immediates and the
 * temporaries (dst must be a temporary; at most 32 registers, 48 steps, 8
 * inputs / scalars / immediates).  Opcodes: 0 copy, 1 add, 2 sub, 3 mul
 * (wrapping), 4 div, 5 rem (toward zero, as div.s64 / rem.s64; a zero divisor
 * gives an unspecified value), 6 shl, 7 shr (arithmetic; by the low 32 bits of
 * b, 64 or more: 0 / the sign), 8 xor, 9 max, 10 min, 11-16 eq ne gt lt ge le
 * (signed, 0 or 1), 17 and, 18 or (of b != 0 and a != 0), 19 not, 20 where
 * (a != 0 ? b : c).
 * value_bits: 64, or 32 when the caller has shown that the program gives the
 * same stored bits on 32-bit values: every value that must be exact (an
 * operand of a comparison, max, min, div, rem, shr, where's condition, a
 * logical op, or a result stored as a float or 64-bit integer) lies within
 * the int32 range, and every other value is used only through its low 32
 * bits (add, sub, mul, xor, shl, copy, a store to an integer of 32 bits or
 * fewer).  The matcher proves it by interval arithmetic over the inputs'
 * types and the immediates.
 * A chain program (each step reads only the step before it besides inputs
 * and constants; contiguous inputs on 16-byte boundaries; n >= 1024) runs
 * with its inputs staged in shared memory by bulk copies; a staging wait that
 * passes the library's wait limit records device status 0x1401
 * (emmy_get_device_status) and leaves the output incomplete.
 */
int emmy_pointwise_int(const void *const *inputs, const int *input_dtypes,
                       const int64_t *input_index, int n_inputs,
                       const void *const *scalars, const int *scalar_dtypes, int n_scalars,
                       const int64_t *immediates, int n_imm, const int *program, int n_instr,
                       int result_reg, void *out, int out_dtype, int64_t first, int64_t n,
                       int value_bits, void *stream);

/*
 * Long-row reduction that allocates nothing: y[0] = fold_op(pre(x[0..n))) [* 1/count].
 * No counterpart in the reference: it exists for callers that cannot allocate
 * device memory when they call -- hosts whose device memory is a pool or
 * budget fixed at start-up and owned by someone else, code that runs inside
 * an allocator or pool callback and must not re-enter it, and loops that
 * cannot afford an allocation's implicit device synchronisation.  The per-CTA partials live in a 4096-float array
 * inside the library (16 KB on every device that loads it, kept until exit).
 * Limit: n <= 4096 * 16384 = 67,108,864 elements; longer rows are rejected
 * with EMMY_ERR_INVALID (use emmy_reduce_f32 with a workspace instead).
 * The first call on a device looks up the array's device address; make that
 * first call before any stream capture.  Calls share the array, so calls
 * that overlap on the GPU (different streams, no ordering) race; every call
 * overwrites the partials it reads, so nothing needs clearing between calls.
 */
int emmy_reduce_f32_noalloc(const float *x, float *y, int64_t n, int op, int pre,
                            const float *count, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* EMMY_B200_H */
