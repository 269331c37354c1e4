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

/* output dtypes */
#define EMMY_DT_F32 0
#define EMMY_DT_F16 1

/* GEMM epilogue bits */
#define EMMY_EPI_BIAS 1
#define EMMY_EPI_RELU 2

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
 * f64 matrix-vector product y[rows] = A[rows, cols] @ v[cols].
 * Replaces the entry the reference emits for the dot-with-vector reduction
 * shape (StridedLoop over a row with Load A, Load v, multiply, Accum add, then
 * the warp/tree combine; reference ptxc/stmts.py:728-773, 564-611 and the f64
 * arithmetic of ptxc/expr.py:1179-1309).  Products are fused into FMAs.
 */
int emmy_matvec_f64(const double *A, const double *v, double *y, int64_t rows, int64_t cols,
                    void *stream);

#ifdef __cplusplus
}
#endif

#endif /* EMMY_B200_H */
