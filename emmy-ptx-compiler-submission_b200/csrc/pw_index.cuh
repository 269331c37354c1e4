// Broadcast-input indexing shared by the float and integer pointwise kernels:
// a broadcast input is read at ((first + e) / div) % mod for element e, the
// quotients by multiply-shift (no hardware divide).
#pragma once

#include <stdint.h>

namespace emmy {

// A broadcast input is read at ((first + e) / div) % mod for element e (mod
// 0: no modulo).  The quotients use the round-up multiply-shift method for
// division by an invariant integer (Granlund & Montgomery, PLDI 1994, fig.
// 4.1): q = (t + ((x - t) >> 1)) >> (l - 1), t = mulhi(magic, x), l =
// ceil(log2 d), magic = floor(2^64 (2^l - d) / d) + 1; exact for all 64-bit x.
struct PwDiv {
  unsigned long long d, magic;
  int shift;                       // l - 1; -1 when d == 1
};

struct PwIndex {
  PwDiv div, mod;
  int bcast;                       // 0: input read at e (contiguous)
  int has_mod;
};

__host__ __device__ inline unsigned long long pw_div(const PwDiv &v, unsigned long long x) {
#ifdef __CUDA_ARCH__
  if (v.shift < 0) return x;
  const unsigned long long t = __umul64hi(v.magic, x);
  return (t + ((x - t) >> 1)) >> v.shift;
#else
  return x / v.d;
#endif
}

// Host: the multiply-shift constants for division by d (1 <= d < 2^62).
inline PwDiv make_div(unsigned long long d) {
  PwDiv v{};
  v.d = d;
  if (d == 1) {
    v.shift = -1;
    return v;
  }
  int l = 0;
  while ((1ull << l) < d) ++l;
  const unsigned __int128 num = ((unsigned __int128)((1ull << l) - d)) << 64;
  v.magic = (unsigned long long)(num / d) + 1;
  v.shift = l - 1;
  return v;
}

}  // namespace emmy
