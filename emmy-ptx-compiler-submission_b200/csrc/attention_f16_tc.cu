// f16 attention-like chain with f32 softmax on the sm_100a tensor cores:
//   o = softmax(q k^T * recip(div)) v      per (batch, head), q/k/v/o [BH, S, D]
//
// Replaces the entry the reference emits for its attention IR shape (key loop
// over a head-dim dot loop, online max/sum with exp rescaling, a rescaled
// weighted sum of v and a final divide; reference ptxc/stmts.py:663-725,
// 564-611, 1311-1392, ptxc/expr.py:891-895), here with f16 operands as the
// benchmark configuration asks.
//
// Persistent CTAs (as many as fit on the SMs, two per SM up to D = 128) walk
// the 128-query tiles t = blockIdx.x, blockIdx.x + gridDim.x, ... in (batch,
// head)-major order; each tile's keys go in blocks of 64 (128 at D = 256, see
// AttnCfg).  Warp roles (W = 4 softmax warps, 8 at D = 256):
//   warp W      TMA producer: the first tile's Q, then K and V blocks through
//               one ring in the order the MMA thread consumes them (K0, K1, V0,
//               K2, V1, ..., then the next tile's; no multicast, 128-byte
//               swizzle).  The next tile's Q is loaded by softmax thread 0 as
//               soon as the current tile's last score product is done (the
//               last reader of Q).
//   warp W + 1  one thread issues tcgen05.mma.  S = Q K^T goes to one of two
//               TMEM score buffers, one block ahead: S[g+1] is computed while
//               the softmax warps work on S[g].  O += P V (into TMEM, P read
//               from TMEM as the A operand) follows once P[g] is written.
//   warps 0..W-1 one query row per thread (TMEM lane; at D = 256 two threads
//               per row, each with half of the block): read the 64 scores,
//               exponentiate against the running max, write P as packed f16
//               over the first 32 columns of the same score buffer, keep the
//               running sum; at the end of a tile O / l, staged in shared
//               memory and written by TMA stores.
// g counts key blocks over all of a CTA's tiles, so the score buffers and
// their barriers simply continue from one tile into the next: the next tile's
// Q, K and V loads and its first score products overlap the current tile's
// last blocks and epilogue.  The next tile's first P V product (which starts
// O afresh) waits until the epilogue has read O out of TMEM.
// P[g] lives in score buffer g % 2 until O += P[g] V has read it; the next
// product into that buffer, S[g+2], is issued after that MMA by the same
// thread, and the tensor pipe runs one thread's MMAs in issue order.  So the
// softmax never waits for the previous P V product, except to rescale O.
// The running max is moved lazily: a row keeps its max until a block's max
// exceeds it by more than 2^8 (so P <= 256, well inside f16), and only then
// is its O row rescaled in TMEM.  The result is the same softmax; only the
// rounding differs from rescaling every block.
// Every mbarrier wait is bounded and reports through the device status word;
// on a timeout each role stops, in-flight TMA copies and MMAs are waited for
// (bounded), and TMEM is freed before the CTA exits.

#include "common.cuh"
#include "tcgen05.cuh"

namespace emmy {

// BN keys per block, HALVES softmax warps per TMEM lane quadrant (each taking
// BN / HALVES of a row's scores; with two, the halves exchange their block max
// through shared memory and add their sums at the end).  D = 256: 128-key
// blocks (score products at N = 128, the tensor core's full rate; N = 64 runs
// at 57% of it) -- one CTA fills an SM's tensor memory either way.  D <= 128:
// 64-key blocks and two CTAs per SM (128-key blocks would cost the second CTA:
// measured slower).
// DQ: the head dims the score product covers (K16 steps), a multiple of 16
// and at most D.  A head dim d below D runs the kernel of the next supported
// width: the tensor maps carry the real d, so TMA fills the columns d..D-1 of
// every Q, K and V box with zeros (they add nothing to the scores, and the O
// columns they produce are never stored), and the score product issues only
// ceil(d / 16) K16 steps.
// SLOTS_: depth of the K/V ring (0: the default below).
template <int D, int BN_, int HALVES_, int DQ_ = D, int SLOTS_ = 0>
struct AttnCfg {
  static constexpr int DQ = DQ_;                     // head dims the score product reads
  static constexpr int KSTEPS = DQ / 16;             // K16 steps of the score product
  static constexpr int BN = BN_;                     // keys per block
  static constexpr int HALVES = HALVES_;             // softmax warps per lane quadrant
  static constexpr int CPT = BN / HALVES;            // score columns per softmax thread
  static constexpr int SM_WARPS = 4 * HALVES;        // softmax warps
  static constexpr int NKB = D / 64;                 // 64-wide head-dim blocks of Q and K
  static constexpr int Q_BOX = 128 * 128;            // [128 rows][128 B]
  static constexpr int K_BOX = BN * 128;             // [BN keys][128 B]
  static constexpr int Q_BYTES = NKB * Q_BOX;
  static constexpr int SLOT_BYTES = NKB * K_BOX;     // one K or V block
  static constexpr int SLOTS = SLOTS_ ? SLOTS_ : (BN == 128 ? 2 : 3);
  // epilogue staging: one STAGE_ROWS-row x 128-byte box per softmax warp (16
  // rows where 32 would not leave two CTAs room for Q and the ring)
  static constexpr int STAGE_ROWS =
      HALVES > 1 || (Q_BYTES + SLOTS * SLOT_BYTES > 96 * 1024) ? 16 : 32;
  static constexpr int STAGE_BYTES = SM_WARPS * STAGE_ROWS * 128;
  // Q | ring slots | epilogue staging | half-row exchange, then the mbarriers
  static constexpr int STAGE_OFF = Q_BYTES + SLOTS * SLOT_BYTES;
  static constexpr int XCH_OFF = STAGE_OFF + STAGE_BYTES;
  static constexpr int XCH_BYTES = HALVES > 1 ? 3 * 2 * 128 * 4 : 0;   // max [2][2][128], sum [2][128]
  static constexpr int BAR_OFF = XCH_OFF + XCH_BYTES;
  // mbarriers: 12 fixed, full / empty per slot, 12 for the half-row
  // exchange, then the TMEM address word
  static constexpr int BAR_BYTES = ((12 + 2 * SLOTS + 12) * 8 + 8 + 63) / 64 * 64;
  static constexpr int SMEM = BAR_OFF + BAR_BYTES + 1024;
  // score buffers: three when they and O fit two CTAs' tensor memory (then
  // S runs two blocks ahead of the softmax), else two
  static constexpr int NSB = (HALVES == 1 && 3 * BN + D <= 256) ? 3 : 2;
  static constexpr uint32_t S_COL0 = 0;              // score buffer b at column b * BN
  static constexpr uint32_t O_COL = NSB * BN;
  static constexpr uint32_t TMEM_COLS = O_COL + D <= 256 ? 256 : 512;
  static constexpr int PRODUCER_WARP = SM_WARPS, MMA_WARP = SM_WARPS + 1;
  static constexpr int THREADS = 32 * (SM_WARPS + 2);
  static constexpr int MIN_BLOCKS = NSB * BN + D <= 256 ? 2 : 1;   // two CTAs per SM when TMEM allows
  static constexpr float RESCALE_LOG2 = 8.0f;        // lazy max threshold (P <= 2^8)
  static_assert(SMEM <= 227 * 1024, "shared memory");
  static_assert(DQ % 16 == 0 && DQ > 0 && DQ <= D, "score product width");
  static_assert(O_COL + D <= 512, "tensor memory");
};

// status codes of the waits that can give up (first one recorded wins)
constexpr int kAttnWaitQ = 0x1201, kAttnWaitSlot = 0x1202, kAttnWaitP = 0x1203,
              kAttnWaitEmpty = 0x1204, kAttnWaitS = 0x1205, kAttnWaitO = 0x1206,
              kAttnWaitOFinal = 0x1207, kAttnWaitDrain = 0x1208, kAttnWaitMma = 0x1209,
              kAttnWaitOFree = 0x120b, kAttnWaitHalf = 0x120c;

// D[tmem] (+)= A[tmem] x B[smem desc]: A is M x 16 f16, row m in TMEM lane m,
// two consecutive k packed per 32-bit column (8 columns per MMA).
__device__ __forceinline__ void mma_f16_tmem_a(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                               uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Store 16 consecutive 32-bit columns of this thread's TMEM lane (waits for completion).
__device__ __forceinline__ void tmem_st16_u(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
      "%14,%15,%16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15])
      : "memory");
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Packed pairs of f32 (sm_100 add / fma .f32x2: two lanes per
// instruction, each rounded as its scalar form).
__device__ __forceinline__ uint64_t pack2(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void unpack2(uint64_t r, float &lo, float &hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(r));
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
// the f16x2 of a pair (lo in the low half, as __floats2half2_rn(lo, hi))
__device__ __forceinline__ uint32_t f16x2_of(uint64_t p) {
  float lo, hi;
  unpack2(p, lo, hi);
  uint32_t h;
  asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(h) : "f"(hi), "f"(lo));
  return h;
}


template <int D, int BN_, int HALVES_, int DQ_, int SLOTS_>
__global__ void __launch_bounds__(AttnCfg<D, BN_, HALVES_, DQ_, SLOTS_>::THREADS,
                                  AttnCfg<D, BN_, HALVES_, DQ_, SLOTS_>::MIN_BLOCKS)
attention_f16_tc_kernel(const __grid_constant__ CUtensorMap tmQ,
                        const __grid_constant__ CUtensorMap tmK,
                        const __grid_constant__ CUtensorMap tmV,
                        const __grid_constant__ CUtensorMap tmO,
                        const float *__restrict__ scale_div, int S, int dv, int ntiles,
                        int out_f16, int *status) {
  using C = AttnCfg<D, BN_, HALVES_, DQ_, SLOTS_>;
  constexpr bool SPLIT = C::HALVES > 1;              // two softmax warps per row
  constexpr int BN = C::BN;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char *smem = reinterpret_cast<unsigned char *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  unsigned char *sQ = smem;
  unsigned char *sRing = sQ + C::Q_BYTES;
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + C::BAR_OFF);
  // per tile: q_full (Q landed), o_done (the tile's last P V product is
  // done), o_free (the epilogue has read O); per block: s_full / p_full
  // [g % NSB] (score buffer g % NSB holds S, then P), o_full [g % 2] (P V
  // product g done: two barriers, so with S two blocks ahead a wait for
  // product g - 1 is never two phases behind its barrier)
  constexpr int NSB = C::NSB;
  uint64_t *q_full = bars + 0, *o_done = bars + 1, *o_free = bars + 2, *mma_done = bars + 3;
  uint64_t *o_full = bars + 4;                       // [2]
  uint64_t *s_full = bars + 6, *p_full = bars + 9;   // [NSB] each (3 reserved)
  uint64_t *full = bars + 12, *empty = bars + 12 + C::SLOTS;   // [SLOTS] each
  // SPLIT: half-row exchange, per lane quadrant: block max [g % 2], tile sum
  uint64_t *xmax = bars + 12 + 2 * C::SLOTS, *xsum = xmax + 8;   // [4][2], [4]
  uint32_t *tmem_holder = reinterpret_cast<uint32_t *>(bars + 12 + 2 * C::SLOTS + 12);
  static_assert(NSB == 2 || !SPLIT, "the half-row exchange assumes two score buffers");

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nblk = (S + BN - 1) / BN;
  const int qtiles = (S + 127) / 128;
  // this CTA's tiles: blockIdx.x + i * gridDim.x for i < my_tiles
  const int my_tiles = blockIdx.x < ntiles ? (ntiles - 1 - blockIdx.x) / gridDim.x + 1 : 0;

  if (threadIdx.x == 0) {
    prefetch_tensormap(&tmQ);
    prefetch_tensormap(&tmK);
    prefetch_tensormap(&tmV);
    prefetch_tensormap(&tmO);
    mbar_init(q_full, 1);
    mbar_init(o_done, 1);
    mbar_init(o_free, 32 * C::SM_WARPS);
    mbar_init(&o_full[0], 1);
    mbar_init(&o_full[1], 1);
    mbar_init(mma_done, 1);
    for (int b = 0; b < NSB; ++b) {
      mbar_init(&s_full[b], 1);
      mbar_init(&p_full[b], 32 * C::SM_WARPS);
    }
    for (int s = 0; s < C::SLOTS; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    if (SPLIT) {
      for (int x = 0; x < 8; ++x) mbar_init(&xmax[x], 64);   // the two warps of a quadrant
      for (int x = 0; x < 4; ++x) mbar_init(&xsum[x], 64);
    }
    fence_barrier_init();
  }
  if (warp == C::PRODUCER_WARP) tmem_alloc(tmem_holder, C::TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;

  if (warp == C::PRODUCER_WARP) {
    if (lane == 0) {
      // TMA producer: ring item i goes to slot i % SLOTS once item i - SLOTS
      // has been consumed.  Per tile: K0 .. K[NSB-2], then per block j:
      // K[j+NSB-1] (if any), V[j] -- the order the MMA thread takes them.
      int issued = 0;
      auto load = [&](const CUtensorMap *map, int key_block, int bh) -> bool {
        const int slot = issued % C::SLOTS;
        if (issued >= C::SLOTS &&
            !mbar_wait(&empty[slot], ((issued / C::SLOTS) - 1) & 1, status, kAttnWaitEmpty))
          return false;
        mbar_expect_tx(&full[slot], C::SLOT_BYTES);
        for (int kb = 0; kb < C::NKB; ++kb)
          tma_load_3d(sRing + slot * C::SLOT_BYTES + kb * C::K_BOX, map, &full[slot], kb * 64,
                      key_block * BN, bh);
        ++issued;
        return true;
      };
      bool ok = true;
      if (my_tiles > 0) {
        const int bh = blockIdx.x / qtiles, m0 = (blockIdx.x - bh * qtiles) * 128;
        mbar_expect_tx(q_full, C::Q_BYTES);
        for (int kb = 0; kb < C::NKB; ++kb)
          tma_load_3d(sQ + kb * C::Q_BOX, &tmQ, q_full, kb * 64, m0, bh);
      }
      for (int i = 0; ok && i < my_tiles; ++i) {
        const int t = blockIdx.x + i * gridDim.x;
        const int bh = t / qtiles;
        for (int j = 0; ok && j < NSB - 1 && j < nblk; ++j) ok = load(&tmK, j, bh);
        for (int j = 0; ok && j < nblk; ++j) {
          if (j + NSB - 1 < nblk) ok = load(&tmK, j + NSB - 1, bh);
          if (ok) ok = load(&tmV, j, bh);
        }
      }
      // drain: every issued copy has landed before the CTA may exit (the
      // first Q with the MMA thread's wait or here; later ones by thread 0)
      if (my_tiles == 1) mbar_wait(q_full, 0, status, kAttnWaitDrain);
      for (int i = issued - C::SLOTS > 0 ? issued - C::SLOTS : 0; i < issued; ++i)
        mbar_wait(&full[i % C::SLOTS], (i / C::SLOTS) & 1, status, kAttnWaitDrain);
    }
    __syncwarp();
  } else if (warp == C::MMA_WARP) {
    if (lane == 0) {
      constexpr uint32_t idesc_s = f16_idesc(128, BN, false, false);
      constexpr uint32_t idesc_o = f16_idesc(128, D, false, true);
      const uint32_t qa = smem_u32(sQ);
      int taken = 0;
      // next ring item: wait until it has landed, return its shared address
      auto take = [&](uint32_t &addr) -> bool {
        const int slot = taken % C::SLOTS;
        if (!mbar_wait(&full[slot], (taken / C::SLOTS) & 1, status, kAttnWaitSlot)) return false;
        addr = smem_u32(sRing + slot * C::SLOT_BYTES);
        return true;
      };
      auto release = [&]() { mma_commit(&empty[taken % C::SLOTS]); ++taken; };
      // descriptors built once; a byte offset d inside a 1024-byte-aligned tile
      // adds d >> 4 to the start-address field
      const uint64_t dq = sw128_desc(qa, 16, 1024);
      auto issue_s = [&](int g, uint32_t ka) {
        // S[g % NSB] = Q K^T: both operands K-major (head dim contiguous)
        const uint64_t dk = sw128_desc(ka, 16, 1024);
#pragma unroll
        for (int ks = 0; ks < C::KSTEPS; ++ks) {
          const int kb = ks / 4, kk = ks % 4;
          mma_f16(tmem + C::S_COL0 + (g % NSB) * BN, dq + ((kb * C::Q_BOX + kk * 32) >> 4),
                  dk + ((kb * C::K_BOX + kk * 32) >> 4), idesc_s, ks != 0 ? 1u : 0u);
        }
        mma_commit(&s_full[g % NSB]);
      };
      // Q, K and V come from TMA: their barriers need no tcgen05 fence; P and
      // the rescaled O come from the softmax threads and do
      uint32_t ka = 0, va = 0;
      bool ok = true;
      int g = 0;                                   // key blocks over all tiles
      for (int i = 0; ok && i < my_tiles; ++i) {
        ok = mbar_wait(q_full, i & 1, status, kAttnWaitQ);
        // the tile's first NSB - 1 score products
        for (int j = 0; ok && j < NSB - 1 && j < nblk; ++j) {
          if (!(ok = take(ka))) break;
          issue_s(g + j, ka);
          release();
        }
        if (!ok) break;
        for (int j = 0; j < nblk; ++j, ++g) {
          if (j + NSB - 1 < nblk) {
            // S[g+NSB-1] into buffer (g-1) % NSB: its previous contents
            // (P[g-1]) were read by the P V product issued before it, and the
            // tensor pipe runs this thread's MMAs in issue order
            if (!(ok = take(ka))) break;
            issue_s(g + NSB - 1, ka);
            release();
          }
          // P[g] was published into score buffer g % NSB (one barrier per
          // buffer: P[g+NSB] cannot be published before S[g+NSB] is issued)
          if (!(ok = mbar_wait(&p_full[g % NSB], (g / NSB) & 1, status, kAttnWaitP) && take(va)))
            break;
          // the tile's first product overwrites O: the previous tile's
          // epilogue must have read it
          if (j == 0 && i > 0 && !(ok = mbar_wait(o_free, (i - 1) & 1, status, kAttnWaitOFree)))
            break;
          tc_fence_after();
          // O += P V: P from TMEM (16 keys = 8 columns per MMA; each softmax
          // thread's CPT keys packed into the first CPT / 2 of its CPT score
          // columns), V N-major (value columns contiguous)
#pragma unroll
          for (int kk = 0; kk < BN / 16; ++kk)
            mma_f16_tmem_a(tmem + C::O_COL,
                           tmem + C::S_COL0 + (g % NSB) * BN + (kk * 16 / C::CPT) * C::CPT +
                               (kk * 16 % C::CPT) / 2,
                           sw128_desc(va + kk * 16 * 128, C::K_BOX, 1024), idesc_o,
                           (j | kk) != 0 ? 1u : 0u);
          mma_commit(&o_full[g & 1]);
          release();
        }
        if (ok) mma_commit(o_done);
      }
      // every MMA this thread issued has finished before TMEM is freed
      mma_commit(mma_done);
      mbar_wait(mma_done, 0, status, kAttnWaitMma);
    }
    __syncwarp();
  } else {
    // softmax / epilogue.  Warp w reads TMEM lane quadrant w % 4: its thread
    // owns query row m0 + r, r = 32 * (w % 4) + lane, and of each block's
    // scores the CPT columns of half w / 4 (SPLIT) or all of them.  Scores are kept
    // as t = s * scale * log2(e), so p = 2^(t - m).
    const int quad = warp & 3, half = warp >> 2;
    const int r = quad * 32 + lane;
    const uint32_t lane_base = tmem + ((uint32_t)(quad * 32) << 16);
    const float c = (scale_div ? 1.0f / __ldg(scale_div) : 1.0f) * 1.4426950408889634f;
    const uint64_t c2 = pack2(c, c);
    unsigned char *stage = smem + C::STAGE_OFF + warp * (C::STAGE_ROWS * 128);   // this warp's box
    float *xch = reinterpret_cast<float *>(smem + C::XCH_OFF);   // SPLIT only
    constexpr int CPT = C::CPT;
    constexpr int OCOLS = D / C::HALVES;                 // O columns this warp rescales / writes
    bool ok = true;
    int g = 0, qloads = 0;
    for (int i = 0; ok && i < my_tiles; ++i) {
      const int t = blockIdx.x + i * gridDim.x;
      const int bh = t / qtiles, m0 = (t - bh * qtiles) * 128;
      float m = -INFINITY, l = 0.f;
      for (int j = 0; j < nblk; ++j, ++g) {
        ok = __all_sync(0xffffffffu, mbar_wait(&s_full[g % NSB], (g / NSB) & 1, status, kAttnWaitS));
        if (!ok) break;
        tc_fence_after();
        if (j + 1 == nblk && threadIdx.x == 0 && i + 1 < my_tiles) {
          // the tile's last score product is done, and with it every read of
          // Q: load the next tile's (its phase i + 1 of q_full cannot complete
          // before the MMA thread has waited for phase i)
          const int tn = t + gridDim.x;
          const int bhn = tn / qtiles, m0n = (tn - bhn * qtiles) * 128;
          mbar_expect_tx(q_full, C::Q_BYTES);
          for (int kb = 0; kb < C::NKB; ++kb)
            tma_load_3d(sQ + kb * C::Q_BOX, &tmQ, q_full, kb * 64, m0n, bhn);
          ++qloads;
        }
        const int key0 = j * BN + half * CPT;
        const uint32_t scol = C::S_COL0 + (g % NSB) * BN + half * CPT;   // this half's columns
        // raw scores v; t = v * c is folded into one FFMA below.  With c > 0 the
        // row max of t is c * max(v), with c < 0 it is c * min(v); masked keys
        // get the value whose t is -inf.
        float v[CPT];
        if constexpr (CPT == 64) tmem_ld64(lane_base + scol, v);
        else tmem_ld32(lane_base + scol, v);
        if (key0 + CPT > S) {
          const float far = c > 0.f ? -INFINITY : INFINITY;
#pragma unroll
          for (int k = 0; k < CPT; ++k)
            if (key0 + k >= S) v[k] = far;
        }
        // the block's row max of t: c * max(v) for c > 0, c * min(v) for c < 0
        auto block_max = [&]() -> float {
          float ext[8];
#pragma unroll
          for (int q = 0; q < 8; ++q) ext[q] = v[q];
          if (c > 0.f) {
#pragma unroll
            for (int k = 8; k < CPT; ++k) ext[k & 7] = fmaxf(ext[k & 7], v[k]);
#pragma unroll
            for (int w = 4; w >= 1; w >>= 1)
#pragma unroll
              for (int q = 0; q < w; ++q) ext[q] = fmaxf(ext[q], ext[q + w]);
          } else {
#pragma unroll
            for (int k = 8; k < CPT; ++k) ext[k & 7] = fminf(ext[k & 7], v[k]);
#pragma unroll
            for (int w = 4; w >= 1; w >>= 1)
#pragma unroll
              for (int q = 0; q < w; ++q) ext[q] = fminf(ext[q], ext[q + w]);
          }
          return ext[0] * c;
        };
        // p = 2^(v c - mu) for the pairs of this thread's scores (argument and
        // sums as packed pairs, the exponential on MUFU); P as packed f16 into
        // h; returns the sum of p
        uint32_t h[CPT / 2];
        auto exponentiate = [&](float mu) -> float {
          const uint64_t nm2 = pack2(-mu, -mu);
          uint64_t psum2[2] = {0ull, 0ull};
#pragma unroll
          for (int k = 0; k < CPT / 2; ++k) {
            const uint64_t t2 = fma2(pack2(v[2 * k], v[2 * k + 1]), c2, nm2);
            float t0, t1;
            unpack2(t2, t0, t1);
            const uint64_t p2 = pack2(ex2_approx(t0), ex2_approx(t1));
            psum2[k & 1] = add2(psum2[k & 1], p2);
            h[k] = f16x2_of(p2);
          }
          float ps0, ps1;
          unpack2(add2(psum2[0], psum2[1]), ps0, ps1);
          return ps0 + ps1;
        };
        // the row's block max over both halves (SPLIT): each half posts its
        // own, the quadrant's barrier for this block parity completes with
        // both.  A thread posts block g + 2 only after it has seen block g + 1,
        // for which its partner must have read block g, so one slot per parity
        // suffices and the barrier is never two phases ahead of a waiter.
        auto row_max = [&](float mine) -> float {
          if constexpr (SPLIT) {
            float *slot = xch + (g & 1) * 256;
            slot[half * 128 + r] = mine;
            mbar_arrive(&xmax[quad * 2 + (g & 1)]);
            ok = __all_sync(0xffffffffu, mbar_wait(&xmax[quad * 2 + (g & 1)], (g >> 1) & 1,
                                                   status, kAttnWaitHalf));
            return fmaxf(mine, slot[(half ^ 1) * 128 + r]);
          }
          return mine;
        };
        // Lazy max: the row max moves only when a block's max is more than
        // 2^8 above it (so P <= 2^8).  A tile's first block sets it.  Later
        // blocks are exponentiated against the running max while their max is
        // computed beside it (the two chains are independent), and a row
        // whose max does move -- rare after the first block -- redoes its
        // block against the new one.
        float mb, ps;
        if (j == 0) {
          mb = row_max(block_max());
          if (!ok) break;
          ps = exponentiate(mb);
        } else {
          ps = exponentiate(m);
          mb = row_max(block_max());
          if (!ok) break;
        }
        const bool move = mb > m + C::RESCALE_LOG2;
        const float m_use = move ? mb : m;
        const float alpha = move ? ex2_approx(m - mb) : 1.0f;
        if (j > 0 && move) ps = exponentiate(m_use);
        // tcgen05.ld/st are warp-collective (.sync.aligned): the whole warp
        // rescales when any of its rows moved its max (alpha is 1 for the others)
        if (j > 0 && __any_sync(0xffffffffu, move)) {
          // O is still being accumulated by P[g-1] V.  That product completes
          // phase (g-1) / 2 of o_full[(g-1) % 2], and the wait is unambiguous:
          // S[g] was issued after P[g-NSB] V, so its completion (waited above)
          // means every product up to g-NSB -- among them g-3, the previous
          // one on that barrier -- is done, and P[g+1] V has not been issued.
          ok = __all_sync(0xffffffffu,
                          mbar_wait(&o_full[(g - 1) & 1], ((g - 1) >> 1) & 1, status, kAttnWaitO));
          if (!ok) break;
          tc_fence_after();
#pragma unroll 1
          for (int cc = 0; cc < OCOLS / 32; ++cc) {
            float ov[32];
            __syncwarp();
            tmem_ld32(lane_base + C::O_COL + half * OCOLS + cc * 32, ov);
#pragma unroll
            for (int k = 0; k < 32; ++k) ov[k] *= alpha;
            tmem_st32(lane_base + C::O_COL + half * OCOLS + cc * 32, ov);
          }
        }
        // P over the first CPT / 2 of this half's score columns (already read)
        if constexpr (CPT == 64) tmem_st32_u(lane_base + scol, h);
        else tmem_st16_u(lane_base + scol, h);
        l = l * alpha + ps;                // this half's share of the row sum
        m = m_use;
        tc_fence_before();
        mbar_arrive(&p_full[g % NSB]);
      }
      if (!ok) break;
      if constexpr (SPLIT) {
        // the row sum: this half's share plus the partner's (one phase per tile)
        xch[512 + half * 128 + r] = l;
        mbar_arrive(&xsum[quad]);
        ok = __all_sync(0xffffffffu, mbar_wait(&xsum[quad], i & 1, status, kAttnWaitHalf));
        if (!ok) break;
        l += xch[512 + (half ^ 1) * 128 + r];
      }
      // epilogue: O / l, staged through this warp's box in STAGE_ROWS-row x
      // 128-byte swizzled pieces and written by TMA stores; rows beyond S are
      // dropped by the TMA.  Once O has been read out of TMEM, o_free lets the
      // next tile's first P V product start.
      ok = __all_sync(0xffffffffu, mbar_wait(o_done, i & 1, status, kAttnWaitOFinal));
      if (!ok) break;
      tc_fence_after();
      const float rl = 1.0f / l;
      const int step = out_f16 ? 64 : 32;               // columns per 128-byte row piece
      // pieces that hold real output columns (c < dv); TMA clips the last one
      const int c_top = (dv + step - 1) / step * step;
      const int c_end = (half + 1) * OCOLS < c_top ? (half + 1) * OCOLS : c_top;
#pragma unroll 1
      for (int c0 = half * OCOLS; c0 < c_end; c0 += step) {
        uint4 w[8];
        if (out_f16) {
          float v[64];
          tmem_ld64(lane_base + C::O_COL + c0, v);
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            uint32_t hq[4];
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              __half2 hh = __floats2half2_rn(v[8 * q + 2 * k] * rl, v[8 * q + 2 * k + 1] * rl);
              hq[k] = *reinterpret_cast<uint32_t *>(&hh);
            }
            w[q] = make_uint4(hq[0], hq[1], hq[2], hq[3]);
          }
        } else {
          float v[32];
          tmem_ld32(lane_base + C::O_COL + c0, v);
#pragma unroll
          for (int q = 0; q < 8; ++q)
            w[q] = make_uint4(__float_as_uint(v[4 * q] * rl), __float_as_uint(v[4 * q + 1] * rl),
                              __float_as_uint(v[4 * q + 2] * rl), __float_as_uint(v[4 * q + 3] * rl));
        }
        if (c0 + step >= c_end) {
          tc_fence_before();
          mbar_arrive(o_free);                          // O fully read out of TMEM
        }
        // the warp's 32 rows in 32 / STAGE_ROWS boxes; the box is free once
        // the previous TMA store has read it
#pragma unroll
        for (int hb = 0; hb < 32 / C::STAGE_ROWS; ++hb) {
          if (lane == 0) bulk_wait_group_read<0>();
          __syncwarp();
          const int row = lane - hb * C::STAGE_ROWS;
          if (row >= 0 && row < C::STAGE_ROWS) {
#pragma unroll
            for (int q = 0; q < 8; ++q)
              *reinterpret_cast<uint4 *>(stage + row * 128 + ((q ^ (row & 7)) * 16)) = w[q];
          }
          fence_proxy_async();
          __syncwarp();
          if (lane == 0) {
            tma_store_3d(&tmO, stage, c0, m0 + quad * 32 + hb * C::STAGE_ROWS, bh);
            bulk_commit_group();
          }
        }
      }
    }
    if (lane == 0) bulk_wait_group<0>();
    // the last Q this thread loaded has landed before the CTA may exit
    if (threadIdx.x == 0 && qloads > 0) mbar_wait(q_full, qloads & 1, status, kAttnWaitDrain);
    __syncwarp();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == C::PRODUCER_WARP) tmem_dealloc(tmem, C::TMEM_COLS);
}

// CUDA-core fallback (any head dim, pre-transposed k, S beyond one block of
// shared memory is refused): f16 in, f32 math, exact two-pass row softmax.
template <typename TOut>
__global__ void __launch_bounds__(256)
attention_f16_simt_kernel(const __half *__restrict__ q, const __half *__restrict__ k,
                          const __half *__restrict__ v, TOut *__restrict__ o,
                          const float *__restrict__ scale_div, int Sq, int Sk, int D, int Dv,
                          int k_transposed) {
  extern __shared__ float sh[];
  float *qs = sh;
  float *ps = sh + D;
  __shared__ float red[32];
  const int row = blockIdx.x, b = blockIdx.y;
  const float scale = scale_div ? 1.0f / __ldg(scale_div) : 1.0f;
  const __half *qr = q + ((int64_t)b * Sq + row) * D;
  const __half *kb = k + (int64_t)b * Sk * D;
  const __half *vb = v + (int64_t)b * Sk * Dv;
  for (int d = threadIdx.x; d < D; d += blockDim.x) qs[d] = __half2float(qr[d]);
  __syncthreads();
  float m = kMaxSeed;
  for (int j = threadIdx.x; j < Sk; j += blockDim.x) {
    float acc = 0.f;
    for (int d = 0; d < D; ++d)
      acc = fmaf(__half2float(k_transposed ? kb[(int64_t)d * Sk + j] : kb[(int64_t)j * D + d]),
                 qs[d], acc);
    ps[j] = acc * scale;
    m = fmaxf(m, ps[j]);
  }
  m = warp_max(m);
  const int w = threadIdx.x >> 5, l32 = threadIdx.x & 31, nw = blockDim.x >> 5;
  __syncthreads();
  if (l32 == 0) red[w] = m;
  __syncthreads();
  m = warp_max(l32 < nw ? red[l32] : -INFINITY);
  float l = 0.f;
  for (int j = threadIdx.x; j < Sk; j += blockDim.x) {
    const float p = __expf(ps[j] - m);
    ps[j] = p;
    l += p;
  }
  l = warp_sum(l);
  __syncthreads();
  if (l32 == 0) red[w] = l;
  __syncthreads();
  l = warp_sum(l32 < nw ? red[l32] : 0.f);
  const float rl = 1.0f / l;
  TOut *orow = o + ((int64_t)b * Sq + row) * Dv;
  for (int c = threadIdx.x; c < Dv; c += blockDim.x) {
    float acc = 0.f;
    for (int j = 0; j < Sk; ++j) acc = fmaf(ps[j], __half2float(vb[(int64_t)j * Dv + c]), acc);
    if constexpr (sizeof(TOut) == 2) orow[c] = __float2half_rn(acc * rl);
    else orow[c] = acc * rl;
  }
}

namespace {

// d: the real head dim (a multiple of 8, at most D); the maps carry it, so
// boxes reaching past it are zero-filled on load and clipped on store.
template <int D, int BN, int HALVES, int DQ, int SLOTS = 0>
int launch_attention_tc(const void *q, const void *k, const void *v, void *o,
                        const float *scale_div, int64_t batch, int64_t S, int64_t d,
                        int out_f16, cudaStream_t st) {
  using Cfg = AttnCfg<D, BN, HALVES, DQ, SLOTS>;
  CUtensorMap tq, tk, tv;
  const uint64_t dims[3] = {(uint64_t)d, (uint64_t)S, (uint64_t)batch};
  const uint64_t str[2] = {(uint64_t)d * 2, (uint64_t)S * d * 2};
  const uint32_t qbox[3] = {64, 128, 1};
  const uint32_t kbox[3] = {64, Cfg::BN, 1};
  int rc = make_tensor_map(&tq, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, q, dims, str, qbox,
                           CU_TENSOR_MAP_SWIZZLE_128B);
  if (!rc) rc = make_tensor_map(&tk, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, k, dims, str, kbox,
                                CU_TENSOR_MAP_SWIZZLE_128B);
  if (!rc) rc = make_tensor_map(&tv, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, v, dims, str, kbox,
                                CU_TENSOR_MAP_SWIZZLE_128B);
  // O written by TMA stores of STAGE_ROWS-row x 128-byte boxes
  CUtensorMap to;
  const uint64_t esize = out_f16 ? 2 : 4;
  const uint64_t ostr[2] = {(uint64_t)d * esize, (uint64_t)S * d * esize};
  const uint32_t obox[3] = {(uint32_t)(128 / esize), (uint32_t)Cfg::STAGE_ROWS, 1};
  if (!rc) rc = make_tensor_map(&to, out_f16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                             : CU_TENSOR_MAP_DATA_TYPE_FLOAT32,
                                3, o, dims, ostr, obox, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  static bool attr_set[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr_set[dev]) {
    cudaFuncSetAttribute(attention_f16_tc_kernel<D, BN, HALVES, DQ, SLOTS>,
                         cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM);
    attr_set[dev] = true;
  }
  // persistent CTAs: as many as are resident at once, each walking its tiles
  const int64_t ntiles = (S + 127) / 128 * batch;
  if (ntiles > INT32_MAX) return set_error(EMMY_ERR_INVALID, "emmy_attention_f16: too many query tiles");
  const int64_t slots = (int64_t)Cfg::MIN_BLOCKS * sm_count();
  const unsigned grid = (unsigned)(ntiles < slots ? ntiles : slots);
  attention_f16_tc_kernel<D, BN, HALVES, DQ, SLOTS><<<grid, Cfg::THREADS, Cfg::SMEM, st>>>(
      tq, tk, tv, to, scale_div, (int)S, (int)d, (int)ntiles, out_f16, device_status_ptr());
  return check_launch("emmy_attention_f16 (tcgen05)");
}

}  // namespace

}  // namespace emmy

using namespace emmy;

extern "C" int emmy_attention_f16(const void *q, const void *k, const void *v, void *o,
                                  const float *scale_div, int64_t batch, int64_t sq, int64_t sk,
                                  int64_t d, int out_dtype, int k_transposed, void *stream) {
  clear_error();
  if (batch < 0 || sq < 0 || sk < 0 || d < 0)
    return set_error(EMMY_ERR_INVALID, "emmy_attention_f16: negative size");
  if (batch == 0 || sq == 0 || d == 0) return EMMY_OK;
  if (sk == 0) return set_error(EMMY_ERR_INVALID, "emmy_attention_f16: no keys");
  if (!q || !k || !v || !o) return set_error(EMMY_ERR_INVALID, "emmy_attention_f16: null operand");
  if (out_dtype != EMMY_DT_F32 && out_dtype != EMMY_DT_F16)
    return set_error(EMMY_ERR_INVALID, "emmy_attention_f16: bad output dtype");
  if (batch > 65535 || sq > INT32_MAX || sk > INT32_MAX)
    return set_error(EMMY_ERR_UNSUPPORTED, "emmy_attention_f16: grid too large");
  cudaStream_t st = as_stream(stream);
  const int out_f16 = out_dtype == EMMY_DT_F16;
  // the tensor-core kernel: any head dim that is a multiple of 8 (16-byte rows
  // for TMA) up to 256, run by the kernel of the next width in {64, 128, 256}
  const bool tc = !k_transposed && sq == sk && aligned16(q) && aligned16(k) && aligned16(v) &&
                  aligned16(o) && d % 8 == 0 && d <= 256;
  if (tc) {
    // D = 256: 128-key blocks once there is more than one 64-key block.
    // (D = 128 with two softmax warps per row, 32 scores each, at two CTAs per
    // SM was measured slower: the per-block max exchange costs more than the
    // halved softmax work saves.)
    if (d <= 16)
      return launch_attention_tc<64, 64, 1, 16>(q, k, v, o, scale_div, batch, sq, d, out_f16, st);
    if (d <= 32)
      return launch_attention_tc<64, 64, 1, 32>(q, k, v, o, scale_div, batch, sq, d, out_f16, st);
    if (d <= 64)
      return launch_attention_tc<64, 64, 1, 64>(q, k, v, o, scale_div, batch, sq, d, out_f16, st);
    if (d <= 96)
      return launch_attention_tc<128, 64, 1, 96>(q, k, v, o, scale_div, batch, sq, d, out_f16,
                                                 st);
    if (d <= 128)
      return launch_attention_tc<128, 64, 1, 128>(q, k, v, o, scale_div, batch, sq, d, out_f16,
                                                  st);
    if (sq > 64)
      return launch_attention_tc<256, 128, 2, 256>(q, k, v, o, scale_div, batch, sq, d, out_f16,
                                                   st);
    return launch_attention_tc<256, 64, 1, 256>(q, k, v, o, scale_div, batch, sq, d, out_f16, st);
  }
  // head dims up to 96: one thread per query row (any key count)
  const int rc = launch_attention_rows(q, k, v, o, scale_div, batch, sq, sk, d, d, 1, out_f16,
                                       k_transposed, st);
  if (rc >= 0) return rc;
  const size_t smem = (size_t)(d + sk) * sizeof(float);
  if (smem > 200 * 1024)
    return set_error(EMMY_ERR_UNSUPPORTED, "emmy_attention_f16: %lld keys exceed shared memory",
                     (long long)sk);
  dim3 grid((unsigned)sq, (unsigned)batch);
  if (out_f16) {
    if (smem > 48 * 1024)
      cudaFuncSetAttribute(attention_f16_simt_kernel<__half>,
                           cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    attention_f16_simt_kernel<__half><<<grid, 256, smem, st>>>(
        static_cast<const __half *>(q), static_cast<const __half *>(k),
        static_cast<const __half *>(v), static_cast<__half *>(o), scale_div, (int)sq, (int)sk,
        (int)d, (int)d, k_transposed);
  } else {
    if (smem > 48 * 1024)
      cudaFuncSetAttribute(attention_f16_simt_kernel<float>,
                           cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    attention_f16_simt_kernel<float><<<grid, 256, smem, st>>>(
        static_cast<const __half *>(q), static_cast<const __half *>(k),
        static_cast<const __half *>(v), static_cast<float *>(o), scale_div, (int)sq, (int)sk,
        (int)d, (int)d, k_transposed);
  }
  return check_launch("emmy_attention_f16 (simt)");
}
