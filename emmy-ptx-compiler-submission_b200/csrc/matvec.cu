// f64 matrix-vector product y = A @ v on sm_100a (HBM-bound).
//
// In the IR this is the cooperative-reduction shape with a second load:
// StridedLoop over a row of A, Load A[row, j], Load v[j], multiply, Accum add,
// then the warp/tree combine and a Cond(co == 0) write (the dot-with-vector
// form of reference ptxc/stmts.py:728-773 and 564-611, in f64 as
// ptxc/expr.py:1179-1309 computes it).  Here one warp owns a row, streams it
// with 16-byte loads (two doubles per lane per step, four steps in flight) and
// reads v through the read-only path, where it stays L2-resident across rows.

#include "common.cuh"

namespace emmy {

__global__ void __launch_bounds__(256)
matvec_f64_kernel(const double *__restrict__ A, const double *__restrict__ v,
                  double *__restrict__ y, int64_t rows, int64_t cols, bool vec2) {
  const int lane = threadIdx.x & 31;
  const int64_t warps_total = (int64_t)gridDim.x * 8;
  for (int64_t row = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5); row < rows; row += warps_total) {
    const double *a = A + row * cols;
    double s0 = 0.0, s1 = 0.0, s2 = 0.0, s3 = 0.0;
    int64_t j = 0;
    if (vec2) {
      // 4 x 32 lanes x 2 doubles = 256 columns per step
      for (j = (int64_t)lane * 2; j + 192 + 1 < cols; j += 256) {
        const double2 p0 = __ldcs(reinterpret_cast<const double2 *>(a + j));
        const double2 p1 = __ldcs(reinterpret_cast<const double2 *>(a + j + 64));
        const double2 p2 = __ldcs(reinterpret_cast<const double2 *>(a + j + 128));
        const double2 p3 = __ldcs(reinterpret_cast<const double2 *>(a + j + 192));
        const double2 q0 = __ldg(reinterpret_cast<const double2 *>(v + j));
        const double2 q1 = __ldg(reinterpret_cast<const double2 *>(v + j + 64));
        const double2 q2 = __ldg(reinterpret_cast<const double2 *>(v + j + 128));
        const double2 q3 = __ldg(reinterpret_cast<const double2 *>(v + j + 192));
        s0 = fma(p0.x, q0.x, s0); s0 = fma(p0.y, q0.y, s0);
        s1 = fma(p1.x, q1.x, s1); s1 = fma(p1.y, q1.y, s1);
        s2 = fma(p2.x, q2.x, s2); s2 = fma(p2.y, q2.y, s2);
        s3 = fma(p3.x, q3.x, s3); s3 = fma(p3.y, q3.y, s3);
      }
      // remaining columns (fewer than 256), one double2 per lane per step
      for (; j + 1 < cols; j += 64) {
        const double2 p0 = __ldcs(reinterpret_cast<const double2 *>(a + j));
        const double2 q0 = __ldg(reinterpret_cast<const double2 *>(v + j));
        s0 = fma(p0.x, q0.x, s0); s0 = fma(p0.y, q0.y, s0);
      }
    } else {
      for (j = lane; j < cols; j += 32) s0 = fma(__ldcs(a + j), __ldg(v + j), s0);
    }
    double s = (s0 + s1) + (s2 + s3);
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (lane == 0) y[row] = s;
  }
}

// Long rows: one CTA of 256 threads per row.  All threads stride the row
// together with 16-byte loads (4 in flight each, 2048 doubles per step), then
// the partial dot products meet through warp shuffles and one shared-memory
// stage.  Many short-lived CTAs keep every SM busy to the end of the launch;
// one long-lived warp per row left the last wave of rows on a fraction of the
// GPU.
__global__ void __launch_bounds__(256)
matvec_f64_row_cta_kernel(const double *__restrict__ A, const double *__restrict__ v,
                          double *__restrict__ y, int64_t cols) {
  __shared__ double part[8];
  const int t = threadIdx.x;
  const double *a = A + (int64_t)blockIdx.x * cols;
  double s0 = 0.0, s1 = 0.0, s2 = 0.0, s3 = 0.0;
  int64_t j = (int64_t)t * 2;
  for (; j + 1536 + 1 < cols; j += 2048) {
    const double2 p0 = __ldcs(reinterpret_cast<const double2 *>(a + j));
    const double2 p1 = __ldcs(reinterpret_cast<const double2 *>(a + j + 512));
    const double2 p2 = __ldcs(reinterpret_cast<const double2 *>(a + j + 1024));
    const double2 p3 = __ldcs(reinterpret_cast<const double2 *>(a + j + 1536));
    const double2 q0 = __ldg(reinterpret_cast<const double2 *>(v + j));
    const double2 q1 = __ldg(reinterpret_cast<const double2 *>(v + j + 512));
    const double2 q2 = __ldg(reinterpret_cast<const double2 *>(v + j + 1024));
    const double2 q3 = __ldg(reinterpret_cast<const double2 *>(v + j + 1536));
    s0 = fma(p0.x, q0.x, s0); s0 = fma(p0.y, q0.y, s0);
    s1 = fma(p1.x, q1.x, s1); s1 = fma(p1.y, q1.y, s1);
    s2 = fma(p2.x, q2.x, s2); s2 = fma(p2.y, q2.y, s2);
    s3 = fma(p3.x, q3.x, s3); s3 = fma(p3.y, q3.y, s3);
  }
  for (; j + 1 < cols; j += 512) {
    const double2 p0 = __ldcs(reinterpret_cast<const double2 *>(a + j));
    const double2 q0 = __ldg(reinterpret_cast<const double2 *>(v + j));
    s0 = fma(p0.x, q0.x, s0); s0 = fma(p0.y, q0.y, s0);
  }
  double s = (s0 + s1) + (s2 + s3);
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if ((t & 31) == 0) part[t >> 5] = s;
  __syncthreads();
  if (t < 32) {
    s = t < 8 ? part[t] : 0.0;
#pragma unroll
    for (int o = 4; o >= 1; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (t == 0) y[blockIdx.x] = s;
  }
}

}  // namespace emmy

using namespace emmy;

extern "C" int emmy_matvec_f64(const double *A, const double *v, double *y, int64_t rows,
                               int64_t cols, void *stream) {
  clear_error();
  if (rows < 0 || cols < 0) return set_error(EMMY_ERR_INVALID, "emmy_matvec_f64: negative size");
  if (rows == 0) return EMMY_OK;
  if (!A || !v || !y) return set_error(EMMY_ERR_INVALID, "emmy_matvec_f64: null pointer");
  const bool vec2 = (cols % 2 == 0) && aligned16(A) && aligned16(v);
  if (vec2 && cols >= 4096 && rows <= INT32_MAX) {
    matvec_f64_row_cta_kernel<<<(unsigned)rows, 256, 0, as_stream(stream)>>>(A, v, y, cols);
    return check_launch("emmy_matvec_f64 (row CTA)");
  }
  int64_t blocks = (rows + 7) / 8;
  const int64_t cap = (int64_t)sm_count() * 8 * 16;
  if (blocks > cap) blocks = cap;
  matvec_f64_kernel<<<(unsigned)blocks, 256, 0, as_stream(stream)>>>(A, v, y, rows, cols, vec2);
  return check_launch("emmy_matvec_f64");
}
