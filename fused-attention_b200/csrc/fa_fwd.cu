// Causal attention forward for sm_100a (B200): TMA + tcgen05 UMMA + TMEM, warp-specialised.
//
// Computes, per (batch, query head), O = softmax(Q K^T / sqrt(D) + causal mask) V and,
// optionally, the log2-domain row statistic LSE = m + log2(l) of the scaled scores
// (the quantity the reference's LSE-saving forward stores:
// attention/backward/fused_backward.py:60-62,169).  Online softmax in exp2 with the
// folded constant log2(e)/sqrt(D) follows attention/fused/fused.py:34-64; GQA (query head h
// reads K/V head h // (H / H_kv)) follows attention/gqa/fused_gqa.py:18,37-39.
//
// CTA work unit: two 128-row query tiles that read the SAME K/V head:
//   mode 0: q-tiles (2c, 2c+1) of one head          (MHA, odd GQA groups)
//   mode 1: q-tile i of query heads (2p, 2p+1)      (even GQA groups: K/V tile shared)
// Grid order: bands of up to 16 work units, every unit's heaviest tile pair first inside a band
// (see band_order), so the grid ends with its shortest CTAs.
// Warp roles (384 threads):
//   warps 0-3   softmax warpgroup of query tile 0: one thread = one query row = one TMEM lane,
//               holding the row's whole K/V tile of scores in registers (no exchange between
//               warpgroups, S read from TMEM once)
//   warps 4-7   softmax warpgroup of query tile 1
//   warp 8      TMA producer: Q tiles once, then the K ring (K(j) is freed once every tile's
//               Q K^T has read it, well before V(j) is freed, so K loads run ahead)
//   warp 9      UMMA issuer (the whole warp computes descriptors, one elected lane issues):
//               S_t = Q_t K_j^T into TMEM, O_t += P_t V_j with P_t read from TMEM
//   warp 10     TMA producer: the V ring
//   warp 11     idle
// Registers: the launch gives every thread 168; with 128-key tiles the producer/issuer warpgroup
// (warps 8-11) drops to 104 and the two softmax warpgroups, which hold 128 scores per thread, rise
// to 200 (4 x 32 x 104 + 8 x 32 x 200 = 384 x 168; neither side spills).  These are the only two
// budget changes: the increases can only be met from what the decrease frees, so nothing else may
// claim registers (a warp that raised its budget again at its end could take them first and leave
// a softmax warp waiting forever).  The teardown after the role branches runs under both budgets.
// TMEM (512 columns): S_0 | S_1 | O_0 | O_1, 128 columns each; P_t (16-bit) overwrites the first
// BN/2 columns of S_t once the row is in registers.  With 64-key tiles S_t takes 64 of the tile's
// 128 columns, so each tile has two S buffers and Q K^T runs two steps ahead of P V (O is then
// rescaled only after a per-tile "P V done" barrier).  The two tiles ping-pong: while one tile's
// warpgroup turns S into P, the tensor core runs the other tile's P V and next Q K^T.  P is
// published in two halves (keys [0, BN/2) and [BN/2, BN)), so the first half's P V runs while the
// second half is exponentiated; on interior tiles the first half uses the running max, and the
// new row max is computed alongside it instead of in front of it.
// exp2: most of every row on the MUFU unit (ex2.approx), a fixed share as a degree-3 polynomial on
// the FMA pipe (the MUFU unit alone needs as many cycles per tile as the tensor core: 16 results
// per clock and SM against 8192 FLOP per clock).
// O is rescaled in TMEM only when a row max grows by more than 2^8 (otherwise the stale max is
// kept, which is exact because numerator and denominator use the same offset).
#include "fa_internal.h"
#include "fa_sm100.cuh"

namespace fa {
namespace {

constexpr int kThreads = 384;
constexpr int kSoftmaxWarps = 8;    // 2 warpgroups: tile t = warp / 4
constexpr int kWarpProducerK = 8;   // Q tiles, then the K ring
constexpr int kWarpMma = 9;
constexpr int kWarpProducerV = 10;  // the V ring
constexpr int kBM = 128;
constexpr uint32_t kTmemCols = 512;
constexpr float kRescaleThreshold = 8.0f;  // log2 units: rescale O only if the max grows > 256x
constexpr int kLaunchRegs = 168;           // 65536 / 384, rounded down to the allocation unit of 8
constexpr int kRegsSoftmax = 200;
constexpr int kRegsOther = 104;
static_assert(4 * 32 * kRegsOther + 8 * 32 * kRegsSoftmax <= kThreads * kLaunchRegs, "register split");
constexpr int kSoftmaxCopy = 1;  // the softmax warpgroups' own copy of the bounded-wait loop

// Register split between the warpgroups: with 128-key tiles (a softmax thread holds 128 scores,
// and 168 registers spill).
template <int BN>
constexpr bool reg_split() {
#ifdef FA_FWD_REG_SPLIT
  return FA_FWD_REG_SPLIT != 0 && BN == 128;
#else
  return BN == 128;
#endif
}

// Of every 16 exp2 pairs on interior tiles, this many go to the FMA-pipe polynomial (measured
// best: 4 with 128-key tiles and the register split, +1-3 % over 3; 1 with 64-key tiles).
template <int BN>
constexpr int poly_pairs() {
#ifdef FA_FWD_POLY_PAIRS
  return FA_FWD_POLY_PAIRS;
#else
  return BN == 128 ? 4 : 1;
#endif
}

template <int D, int BN>
struct FwdCfg {
  // Shared-memory tiles are rows of swizzle chunks: 64 columns (128-byte rows, 128-byte swizzle)
  // for D = 64 and 128, one 32-column chunk (64-byte rows, 64-byte swizzle) for D = 32.
  static constexpr int kSwBytes = D >= 64 ? 128 : 64;
  static constexpr int kChunkCols = kSwBytes / 2;
  static constexpr uint32_t kLayout = D >= 64 ? kLayoutSw128 : kLayoutSw64;
  static constexpr int kSbo = 8 * kSwBytes;           // bytes between 8-row groups
  static constexpr int kKStepsPerChunk = kSwBytes / 32;  // 16-element UMMA K steps per row
  static constexpr int kChunks = D / kChunkCols;
  static constexpr int kQChunkBytes = kBM * kSwBytes;
  static constexpr int kKVChunkBytes = BN * kSwBytes;
  static constexpr int kQBytes = kBM * D * 2;
  static constexpr int kKVBytes = BN * D * 2;       // one K (or V) tile
  static constexpr int kBudget = 225 * 1024;
  static constexpr int kSlots = (kBudget - 2 * kQBytes) / kKVBytes;  // K + V ring slots that fit
  static constexpr int kVStages = (kSlots / 2) > 4 ? 4 : (kSlots / 2);
  static constexpr int kKStages = (kSlots - kVStages) > 4 ? 4 : (kSlots - kVStages);
  static_assert(kVStages >= 2 && kKStages >= 2, "need double-buffered K and V rings");
  static constexpr int kOffQ = 0;
  static constexpr int kOffK = 2 * kQBytes;
  static constexpr int kOffV = kOffK + kKStages * kKVBytes;
  static constexpr int kOffBar = kOffV + kVStages * kKVBytes;
  static constexpr int kSmemBytes = kOffBar + 256 + 1024;  // barriers + 1 KiB alignment slack
};

// barrier slots
enum : int {
  BAR_Q = 0,
  BAR_KFULL = 1,    // + K stage (4)
  BAR_KEMPTY = 5,   // + K stage (4)
  BAR_VFULL = 9,    // + V stage (4)
  BAR_VEMPTY = 13,  // + V stage (4)
  BAR_SFULL = 17,   // + tile (2)
  BAR_PFULLA = 19,  // + tile (2): P of the first half of the tile's keys is in TMEM
  BAR_OFULL = 21,   // + tile (2)
  BAR_DRAIN = 23,
  BAR_PFULLB = 24,  // + tile (2): P of the second half
  BAR_NEVER = 26,   // never arrived at (the failure-detection test build waits on it)
  BAR_SFULLB = 27,  // + tile (2): S in the tile's second buffer (64-key tiles)
  BAR_PVDONE = 29,  // + tile (2): the tile's P V of the step is done (64-key tiles)
  BAR_COUNT = 31
};

// 64-key tiles: S takes 64 of a tile's 128 TMEM columns, so each tile keeps two S buffers and the
// issuer runs Q K^T two steps ahead (S(j+2) into the buffer that P(j) V just read): the softmax
// warpgroup finds S(j+1) ready when it finishes P(j).
template <int BN>
constexpr bool s_double() {
  return BN == 64;
}

struct QTile {
  int bh;  // b * H + h (query head)
  int qt;  // 128-row query tile index
};

struct Work {
  QTile t[2];
  int ntiles;  // 1 or 2
  int bh_kv;   // b * H_kv + kv head
  int nkv[2];  // K/V tiles visible to each query tile
};

template <int BN>
__device__ __forceinline__ int kv_tiles_for(int qt, int S) {
  int last_row = min(qt * kBM + kBM - 1, S - 1);
  return last_row / BN + 1;
}

template <int BN>
__device__ __forceinline__ Work decode_work(const FwdParams& p, int item) {
  Work w;
  if (p.mode == 0) {
    const int ncp = (p.nq + 1) / 2;
    const UnitLevel ul = band_order(item, p.B * p.H, ncp, p.band);
    const int bh = ul.unit;
    const int c = ncp - 1 - ul.level;  // heavy (late) tile pairs first
    w.t[0] = {bh, 2 * c};
    w.t[1] = {bh, 2 * c + 1};
    w.ntiles = (2 * c + 1 < p.nq) ? 2 : 1;
    const int b = bh / p.H, h = bh - b * p.H;
    w.bh_kv = b * p.H_kv + h / p.group;
  } else {
    const int pairs_per_b = p.H / 2;
    const UnitLevel ul = band_order(item, p.B * pairs_per_b, p.nq, p.band);
    const int pi = ul.unit;
    const int i = p.nq - 1 - ul.level;
    const int b = pi / pairs_per_b, hp = pi - b * pairs_per_b;
    const int h = 2 * hp;
    w.t[0] = {b * p.H + h, i};
    w.t[1] = {b * p.H + h + 1, i};
    w.ntiles = 2;
    w.bh_kv = b * p.H_kv + h / p.group;
  }
  w.nkv[0] = kv_tiles_for<BN>(w.t[0].qt, p.S);
  w.nkv[1] = (w.ntiles == 2) ? kv_tiles_for<BN>(w.t[1].qt, p.S) : 0;
  return w;
}

// P = 2^(S * scale - m) for 32 columns of one row (masked entries, -inf, give 0; the polynomial
// pairs are only used on tiles without masked entries).  kPoly of the 16 pairs, spread over the
// chunk, take the polynomial; the rest go to MUFU ex2.
template <bool BF16, int kPoly>
__device__ __forceinline__ void softmax_chunk(const uint32_t (&r)[32], uint64_t scale2, uint64_t negm2,
                                              uint64_t (&sum2)[4], uint32_t (&pk)[16]) {
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const uint64_t x2 = ffma2(f2u(r[2 * i], r[2 * i + 1]), scale2, negm2);
    // polynomial pairs spread evenly over the chunk (i = 3, 7, 11, 15 for four of them)
    constexpr int kEvery = kPoly > 0 ? 16 / kPoly : 1;
    const bool poly = kPoly > 0 && i % kEvery == kEvery - 1;
    uint64_t p2;
    if (poly)
      p2 = exp2_poly2(x2);
    else
      p2 = f2(ex2_approx(f2lo(x2)), ex2_approx(f2hi(x2)));
    sum2[i & 3] = fadd2(sum2[i & 3], p2);
    pk[i] = pack2<BF16>(f2lo(p2), f2hi(p2));
  }
}

// Row max over NCH 32-column chunks: eight independent chains of the three-input max of sm_100
// (half the instructions of a two-input chain).
template <int NCH>
__device__ __forceinline__ float row_max(const uint32_t (&r)[NCH][32]) {
  float m8[8];
#pragma unroll
  for (int u = 0; u < 8; ++u) m8[u] = -INFINITY;
#pragma unroll
  for (int c = 0; c < NCH; ++c)
#pragma unroll
    for (int i = 0; i < 32; i += 2)
      m8[(c * 16 + i / 2) % 8] = fmax3(m8[(c * 16 + i / 2) % 8], __uint_as_float(r[c][i]), __uint_as_float(r[c][i + 1]));
  return fmaxf(fmax3(m8[0], m8[1], m8[2]), fmax3(m8[3], m8[4], fmax3(m8[5], m8[6], m8[7])));
}

// O row *= alpha in TMEM (D fp32 columns of this thread's lane).
template <int D>
__device__ __forceinline__ void rescale_o(uint32_t t_o, float alpha) {
#pragma unroll 1
  for (int c = 0; c < D / 32; ++c) {
    uint32_t o[32];
    tmem_ld32(t_o + c * 32, o);
    tmem_ld_wait(o);
#pragma unroll
    for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
    tmem_st32(t_o + c * 32, o);
  }
}

// S = Q K^T for one 128-row query tile: D/16 UMMAs, descriptors advanced by constant offsets
// (called by the whole issuer warp).
template <int D, int BN, bool BF16>
__device__ __forceinline__ void issue_qk(uint32_t d_tmem, uint64_t q_desc, uint64_t k_desc) {
  using C = FwdCfg<D, BN>;
  constexpr uint32_t IDESC = idesc_f16(BF16, kBM, BN, false, false);  // Q, K both K-major
  constexpr int KS = C::kKStepsPerChunk;
#pragma unroll
  for (int k = 0; k < D / 16; ++k) {
    umma_ss_w(d_tmem, desc_add(q_desc, (k / KS) * C::kQChunkBytes + (k % KS) * 32),
            desc_add(k_desc, (k / KS) * C::kKVChunkBytes + (k % KS) * 32), IDESC, k > 0 ? 1u : 0u);
  }
}

// O += P V over one half of the tile's keys (half = 0: keys [0, BN/2), 1: [BN/2, BN)): P (16-bit,
// keys in order, two per TMEM column) read from the first BN/2 columns of S as the A operand, V
// MN-major in shared memory.
template <int D, int BN, bool BF16>
__device__ __forceinline__ void issue_pv_half(uint32_t o_tmem, uint32_t p_tmem, uint64_t v_desc,
                                              uint32_t accumulate, int half) {
  constexpr uint32_t IDESC = idesc_f16(BF16, kBM, D, false, true);
  constexpr int kKeyStep = 16 * FwdCfg<D, BN>::kSwBytes;  // 16 key rows of V
  constexpr int kSteps = BN / 32;                          // 16-key UMMA steps per half
#pragma unroll
  for (int i = 0; i < kSteps; ++i) {
    const int k = half * kSteps + i;
    umma_ts_w(o_tmem, p_tmem + k * 8, desc_add(v_desc, k * kKeyStep), IDESC, (accumulate | k) ? 1u : 0u);
  }
}

template <int D, int BN, bool BF16>
__global__ void __launch_bounds__(kThreads, 1)
    fa_fwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                  const __grid_constant__ CUtensorMap tmV, const FwdParams p) {
  using C = FwdCfg<D, BN>;
  constexpr int KST = C::kKStages;
  constexpr int VST = C::kVStages;

  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* smem = smem_raw + (base - raw);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::kOffBar);
  volatile uint32_t* tmem_slot = reinterpret_cast<volatile uint32_t*>(smem + C::kOffBar + 8 * BAR_COUNT);
  volatile int* abort_slot = reinterpret_cast<volatile int*>(smem + C::kOffBar + 8 * BAR_COUNT + 4);
  const uint32_t bar0 = smem_u32(bars);
#define BAR(i) (bar0 + 8u * static_cast<uint32_t>(i))
  const uint32_t sQ = base + C::kOffQ;
  const uint32_t sK = base + C::kOffK;
  const uint32_t sV = base + C::kOffV;

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;

  // A failed CTA leaves a non-zero status word: every later CTA stops before touching TMEM.
  if (threadIdx.x == 0) *abort_slot = ld_status(p.status);
  __syncthreads();
  if (*abort_slot != 0) return;

  const Work w = decode_work<BN>(p, blockIdx.x);
  const int nmax = max(w.nkv[0], w.nkv[1]);

  if (threadIdx.x == 0) {
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
    mbar_init(BAR(BAR_Q), 1);
    for (int s = 0; s < 4; ++s) {
      mbar_init(BAR(BAR_KFULL + s), 1);
      mbar_init(BAR(BAR_KEMPTY + s), 1);
      mbar_init(BAR(BAR_VFULL + s), 1);
      mbar_init(BAR(BAR_VEMPTY + s), 1);
    }
    for (int t = 0; t < 2; ++t) {
      mbar_init(BAR(BAR_SFULL + t), 1);
      mbar_init(BAR(BAR_SFULLB + t), 1);
      mbar_init(BAR(BAR_PVDONE + t), 1);
      mbar_init(BAR(BAR_PFULLA + t), 128);
      mbar_init(BAR(BAR_PFULLB + t), 128);
      mbar_init(BAR(BAR_OFULL + t), 1);
    }
    mbar_init(BAR(BAR_DRAIN), 1);
    mbar_init(BAR(BAR_NEVER), 1);
    fence_barrier_init();
  }
  if (warp == 0) {
    tmem_alloc(smem_u32(const_cast<uint32_t*>(tmem_slot)), kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp >= kSoftmaxWarps) {
  if constexpr (reg_split<BN>()) regs_decrease<kRegsOther>();
  if (warp == kWarpProducerK) {
    // ------------------------------------------------------------ TMA: Q once, then the K ring
    if (lane == 0) {
      const uint64_t pol_q = policy_evict_first();
      const uint64_t pol_kv = policy_evict_last();
      mbar_arrive_expect_tx(BAR(BAR_Q), w.ntiles * C::kQBytes);
      for (int t = 0; t < w.ntiles; ++t)
        for (int c = 0; c < C::kChunks; ++c)
          tma_load_3d(sQ + t * C::kQBytes + c * C::kQChunkBytes, &tmQ, BAR(BAR_Q), c * C::kChunkCols,
                      w.t[t].qt * kBM, w.t[t].bh, pol_q);
      int issued = 0;
      for (int j = 0; j < nmax; ++j) {
        const int s = j % KST;
        if (!mbar_wait(BAR(BAR_KEMPTY + s), ((j / KST) & 1) ^ 1, p.status, kDevTimeoutKVEmpty)) break;
        mbar_arrive_expect_tx(BAR(BAR_KFULL + s), C::kKVBytes);
        for (int c = 0; c < C::kChunks; ++c)
          tma_load_3d(sK + s * C::kKVBytes + c * C::kKVChunkBytes, &tmK, BAR(BAR_KFULL + s), c * C::kChunkCols,
                      j * BN, w.bh_kv, pol_kv);
        ++issued;
      }
      // Never leave the CTA with a copy still writing into shared memory.
      drain_wait(BAR(BAR_Q), 0, p.status);
      for (int j = max(0, issued - KST); j < issued; ++j)
        drain_wait(BAR(BAR_KFULL + j % KST), (j / KST) & 1, p.status);
    }
    __syncwarp();
  } else if (warp == kWarpProducerV) {
    // ------------------------------------------------------------ TMA: the V ring
    if (lane == 0) {
      const uint64_t pol_kv = policy_evict_last();
      int issued = 0;
      for (int j = 0; j < nmax; ++j) {
        const int s = j % VST;
        if (!mbar_wait(BAR(BAR_VEMPTY + s), ((j / VST) & 1) ^ 1, p.status, kDevTimeoutKVEmpty)) break;
        mbar_arrive_expect_tx(BAR(BAR_VFULL + s), C::kKVBytes);
        for (int c = 0; c < C::kChunks; ++c)
          tma_load_3d(sV + s * C::kKVBytes + c * C::kKVChunkBytes, &tmV, BAR(BAR_VFULL + s), c * C::kChunkCols,
                      j * BN, w.bh_kv, pol_kv);
        ++issued;
      }
      for (int j = max(0, issued - VST); j < issued; ++j)
        drain_wait(BAR(BAR_VFULL + j % VST), (j / VST) & 1, p.status);
    }
    __syncwarp();
  } else if (warp == kWarpMma) {
    // ------------------------------------------------------------ UMMA issuer (whole warp;
    // elect.sync picks the one lane that issues each tcgen05 instruction)
    {
      const uint64_t dq0 = sdesc_sw(sQ, 16, C::kSbo, C::kLayout);
      const uint64_t dq1 = sdesc_sw(sQ + C::kQBytes, 16, C::kSbo, C::kLayout);
      const uint64_t dk0 = sdesc_sw(sK, 16, C::kSbo, C::kLayout);
      const uint64_t dv0 = sdesc_sw(sV, C::kKVChunkBytes, C::kSbo, C::kLayout);
      const uint32_t tS0 = tmem, tS1 = tmem + 128, tO0 = tmem + 256, tO1 = tmem + 384;
      const int n0 = w.nkv[0], n1 = w.nkv[1];
      if constexpr (s_double<BN>()) {
        // Two S buffers per tile: S(j) in buffer j % 2.  S(0) and S(1) up front, then in step j
        // P(j) V reads buffer j % 2 and S(j+2) is issued into it right behind.
        static_assert(KST >= 3, "S two steps ahead needs three K stages");
        bool ok = warp_all(mbar_wait(BAR(BAR_Q), 0, p.status, kDevTimeoutQ)) &&
                  warp_all(mbar_wait(BAR(BAR_KFULL + 0), 0, p.status, kDevTimeoutKV));
        if (ok) {
          tc_fence_after();
          issue_qk<D, BN, BF16>(tS0, dq0, dk0);
          umma_commit_w(BAR(BAR_SFULL + 0));
          if (n1 > 0) {
            issue_qk<D, BN, BF16>(tS1, dq1, dk0);
            umma_commit_w(BAR(BAR_SFULL + 1));
          }
          umma_commit_w(BAR(BAR_KEMPTY + 0));
          if (nmax > 1) {
            ok = warp_all(mbar_wait(BAR(BAR_KFULL + 1), 0, p.status, kDevTimeoutKV));
            if (ok) {
              tc_fence_after();
              const uint64_t dk1 = dk0 + static_cast<uint64_t>(C::kKVBytes >> 4);
              if (n0 > 1) {
                issue_qk<D, BN, BF16>(tS0 + 64, dq0, dk1);
                umma_commit_w(BAR(BAR_SFULLB + 0));
              }
              if (n1 > 1) {
                issue_qk<D, BN, BF16>(tS1 + 64, dq1, dk1);
                umma_commit_w(BAR(BAR_SFULLB + 1));
              }
              umma_commit_w(BAR(BAR_KEMPTY + 1));
            }
          }
        }
        for (int j = 0; ok && j < nmax; ++j) {
          const int vs = j % VST;
          const int ks2 = (j + 2) % KST;
          const uint32_t boff = (j & 1) * 64;
          const int sbar = (j & 1) ? BAR_SFULLB : BAR_SFULL;
          const uint64_t dvj = dv0 + static_cast<uint64_t>((vs * C::kKVBytes) >> 4);
          const uint64_t dk2 = dk0 + static_cast<uint64_t>((ks2 * C::kKVBytes) >> 4);
          FA_STALL_HERE(j, BAR(BAR_NEVER), p.status, ok)
          if (!(ok = warp_all(mbar_wait(BAR(BAR_VFULL + vs), (j / VST) & 1, p.status, kDevTimeoutKV)))) break;
          bool k_ready = false;
          bool issued_s = false;
          // tile 0
          if (j < n0) {
            if (!(ok = warp_all(mbar_wait(BAR(BAR_PFULLA + 0), j & 1, p.status, kDevTimeoutP)))) break;
            tc_fence_after();
            issue_pv_half<D, BN, BF16>(tO0, tS0 + boff, dvj, j > 0 ? 1u : 0u, 0);
            if (!(ok = warp_all(mbar_wait(BAR(BAR_PFULLB + 0), j & 1, p.status, kDevTimeoutP)))) break;
            tc_fence_after();
            issue_pv_half<D, BN, BF16>(tO0, tS0 + boff, dvj, 1u, 1);
            umma_commit_w(BAR(BAR_PVDONE + 0));
            if (j + 1 == n0) {
              umma_commit_w(BAR(BAR_OFULL + 0));
            } else if (j + 2 < n0) {
              if (!(ok = warp_all(mbar_wait(BAR(BAR_KFULL + ks2), ((j + 2) / KST) & 1, p.status, kDevTimeoutKV)))) break;
              tc_fence_after();
              k_ready = true;
              issue_qk<D, BN, BF16>(tS0 + boff, dq0, dk2);
              umma_commit_w(BAR(sbar + 0));
              issued_s = true;
            }
          }
          // tile 1
          if (j < n1) {
            if (!(ok = warp_all(mbar_wait(BAR(BAR_PFULLA + 1), j & 1, p.status, kDevTimeoutP)))) break;
            tc_fence_after();
            issue_pv_half<D, BN, BF16>(tO1, tS1 + boff, dvj, j > 0 ? 1u : 0u, 0);
            if (!(ok = warp_all(mbar_wait(BAR(BAR_PFULLB + 1), j & 1, p.status, kDevTimeoutP)))) break;
            tc_fence_after();
            issue_pv_half<D, BN, BF16>(tO1, tS1 + boff, dvj, 1u, 1);
            umma_commit_w(BAR(BAR_PVDONE + 1));
            if (j + 1 == n1) {
              umma_commit_w(BAR(BAR_OFULL + 1));
            } else if (j + 2 < n1) {
              if (!k_ready) {
                if (!(ok = warp_all(mbar_wait(BAR(BAR_KFULL + ks2), ((j + 2) / KST) & 1, p.status, kDevTimeoutKV)))) break;
                tc_fence_after();
              }
              issue_qk<D, BN, BF16>(tS1 + boff, dq1, dk2);
              umma_commit_w(BAR(sbar + 1));
              issued_s = true;
            }
          }
          if (issued_s) umma_commit_w(BAR(BAR_KEMPTY + ks2));  // K(j+2) read by every tile that needs it
          umma_commit_w(BAR(BAR_VEMPTY + vs));                 // V(j) read by every tile that needs it
        }
      } else {
        bool ok = warp_all(mbar_wait(BAR(BAR_Q), 0, p.status, kDevTimeoutQ)) &&
                  warp_all(mbar_wait(BAR(BAR_KFULL + 0), 0, p.status, kDevTimeoutKV));
        if (ok) {
          tc_fence_after();
          issue_qk<D, BN, BF16>(tS0, dq0, dk0);
          umma_commit_w(BAR(BAR_SFULL + 0));
          if (n1 > 0) {
            issue_qk<D, BN, BF16>(tS1, dq1, dk0);
            umma_commit_w(BAR(BAR_SFULL + 1));
          }
          umma_commit_w(BAR(BAR_KEMPTY + 0));
        }
        for (int j = 0; ok && j < nmax; ++j) {
          const int vs = j % VST;
          const int ks1 = (j + 1) % KST;
          const uint64_t dvj = dv0 + static_cast<uint64_t>((vs * C::kKVBytes) >> 4);
          const uint64_t dkn = dk0 + static_cast<uint64_t>((ks1 * C::kKVBytes) >> 4);
          FA_STALL_HERE(j, BAR(BAR_NEVER), p.status, ok)
          if (!(ok = warp_all(mbar_wait(BAR(BAR_VFULL + vs), (j / VST) & 1, p.status, kDevTimeoutKV)))) break;
          bool k_ready = false;
          bool issued_s = false;
          // tile 0
          if (j < n0) {
            if (!(ok = warp_all(mbar_wait(BAR(BAR_PFULLA + 0), j & 1, p.status, kDevTimeoutP)))) break;
            tc_fence_after();
            issue_pv_half<D, BN, BF16>(tO0, tS0, dvj, j > 0 ? 1u : 0u, 0);
            if (!(ok = warp_all(mbar_wait(BAR(BAR_PFULLB + 0), j & 1, p.status, kDevTimeoutP)))) break;
            tc_fence_after();
            issue_pv_half<D, BN, BF16>(tO0, tS0, dvj, 1u, 1);
            if (j + 1 == n0) {
              umma_commit_w(BAR(BAR_OFULL + 0));
            } else {
              if (!(ok = warp_all(mbar_wait(BAR(BAR_KFULL + ks1), ((j + 1) / KST) & 1, p.status, kDevTimeoutKV)))) break;
              tc_fence_after();
              k_ready = true;
              issue_qk<D, BN, BF16>(tS0, dq0, dkn);
              umma_commit_w(BAR(BAR_SFULL + 0));
              issued_s = true;
            }
          }
          // tile 1
          if (j < n1) {
            if (!(ok = warp_all(mbar_wait(BAR(BAR_PFULLA + 1), j & 1, p.status, kDevTimeoutP)))) break;
            tc_fence_after();
            issue_pv_half<D, BN, BF16>(tO1, tS1, dvj, j > 0 ? 1u : 0u, 0);
            if (!(ok = warp_all(mbar_wait(BAR(BAR_PFULLB + 1), j & 1, p.status, kDevTimeoutP)))) break;
            tc_fence_after();
            issue_pv_half<D, BN, BF16>(tO1, tS1, dvj, 1u, 1);
            if (j + 1 == n1) {
              umma_commit_w(BAR(BAR_OFULL + 1));
            } else {
              if (!k_ready) {
                if (!(ok = warp_all(mbar_wait(BAR(BAR_KFULL + ks1), ((j + 1) / KST) & 1, p.status, kDevTimeoutKV)))) break;
                tc_fence_after();
              }
              issue_qk<D, BN, BF16>(tS1, dq1, dkn);
              umma_commit_w(BAR(BAR_SFULL + 1));
              issued_s = true;
            }
          }
          if (issued_s) umma_commit_w(BAR(BAR_KEMPTY + ks1));  // K(j+1) read by every tile that needs it
          umma_commit_w(BAR(BAR_VEMPTY + vs));                 // V(j) read by every tile that needs it
        }
      }
      // All MMAs issued by this warp must finish before TMEM is released.
      umma_commit_w(BAR(BAR_DRAIN));
      drain_wait(BAR(BAR_DRAIN), 0, p.status);
    }
    __syncwarp();
  }
  } else {
    // ------------------------------------------------------------ softmax / epilogue
    // warpgroup t serves query tile t; a thread owns one row (TMEM lane) and its BN scores.
    if constexpr (reg_split<BN>()) regs_increase<kRegsSoftmax>();
    const int t = warp / 4;
    if (t < w.ntiles) {
      constexpr int NCH = BN / 32;  // 32-column chunks of a row
      const QTile tile = w.t[t];
      const int nkv = w.nkv[t];
      const int wq = warp % 4;  // TMEM lane quarter this warp may access
      const int row = wq * 32 + lane;
      const int qrow = tile.qt * kBM + row;
      const uint32_t lane_off = static_cast<uint32_t>(wq * 32) << 16;
      const uint32_t tS = tmem + t * 128 + lane_off;
      const uint32_t tO = tmem + 256 + t * 128 + lane_off;
      const float scale = p.scale_log2;
      float m_used = -INFINITY;
      float l = 0.f;
      bool ok = true;
      for (int j = 0; j < nkv; ++j) {
        // S(j): one buffer per tile, or (64-key tiles) buffer j % 2 of two
        const bool buf1 = s_double<BN>() && (j & 1);
        const uint32_t tSj = buf1 ? tS + 64 : tS;
        const int sbar = (buf1 ? BAR_SFULLB : BAR_SFULL) + t;
        const uint32_t sphase = s_double<BN>() ? (j >> 1) & 1 : j & 1;
        if (!(ok = warp_all(mbar_wait<kSoftmaxCopy>(BAR(sbar), sphase, p.status, kDevTimeoutS)))) break;
        tc_fence_after();
        uint32_t r[NCH][32];
#pragma unroll
        for (int c = 0; c < NCH; ++c) tmem_ld32(tSj + c * 32, r[c]);
#pragma unroll
        for (int c = 0; c < NCH; ++c) tmem_ld_wait(r[c]);
        const int kbase = j * BN;
        const bool masked = kbase + BN - 1 > tile.qt * kBM || kbase + BN > p.S;
        const uint64_t scale2 = f2(scale, scale);
        uint64_t sum2[4] = {0ull, 0ull, 0ull, 0ull};
        float alpha = 1.f;
        if (masked || j == 0) {
          // Diagonal or ragged tile, or the row's first tile: the exact row max first, then P.
          if (masked) {
#pragma unroll
            for (int c = 0; c < NCH; ++c)
#pragma unroll
              for (int i = 0; i < 32; ++i) {
                const int key = kbase + c * 32 + i;
                if (key > qrow || key >= p.S) r[c][i] = __float_as_uint(-INFINITY);
              }
          }
          const float mt = row_max<NCH>(r) * scale;
          const bool upd = mt > m_used + kRescaleThreshold;
          const float m_new = upd ? mt : m_used;
          alpha = ex2_approx(m_used - m_new);
          const uint64_t negm2 = f2(-m_new, -m_new);
#pragma unroll
          for (int c = 0; c < NCH; ++c) {
            uint32_t pk[16];
            softmax_chunk<BF16, 0>(r[c], scale2, negm2, sum2, pk);
            tmem_st16(tSj + c * 16, pk);
          }
          // Rescale the running O if any row's max moved.  P V of step j-1 must be complete: with
          // one S buffer it was issued before S_t(j), whose completion we waited for; with two,
          // its own barrier says so.
          if (s_double<BN>() && j > 0)
            if (!(ok = warp_all(mbar_wait<kSoftmaxCopy>(BAR(BAR_PVDONE + t), (j - 1) & 1, p.status, kDevTimeoutO)))) {
              tmem_st_wait();  // no TMEM store of this thread left in flight at teardown
              break;
            }
          if (j > 0 && __any_sync(0xffffffffu, upd)) rescale_o<D>(tO, alpha);
          m_used = m_new;
          tmem_st_wait();
          tc_fence_before();
          mbar_arrive(BAR(BAR_PFULLA + t));
          mbar_arrive(BAR(BAR_PFULLB + t));
        } else {
          // Interior tile: P of the first half of the keys with the running max m_used while the
          // new row max is computed alongside (off the S -> P critical path).  A row whose max
          // rose by more than the threshold redoes that half with the new max and rescales O
          // before anything is published; the second half then uses the settled max.
          uint64_t negm2 = f2(-m_used, -m_used);
#pragma unroll
          for (int c = 0; c < NCH / 2; ++c) {
            uint32_t pk[16];
            softmax_chunk<BF16, poly_pairs<BN>()>(r[c], scale2, negm2, sum2, pk);
            tmem_st16(tSj + c * 16, pk);
          }
          const float mt = row_max<NCH>(r) * scale;
          const bool upd = mt > m_used + kRescaleThreshold;
          if (s_double<BN>())  // P V of step j-1 is complete before O may be rescaled
            if (!(ok = warp_all(mbar_wait<kSoftmaxCopy>(BAR(BAR_PVDONE + t), (j - 1) & 1, p.status, kDevTimeoutO)))) {
              tmem_st_wait();  // no TMEM store of this thread left in flight at teardown
              break;
            }
          if (__any_sync(0xffffffffu, upd)) {
            const float m_new = upd ? mt : m_used;
            alpha = ex2_approx(m_used - m_new);
            negm2 = f2(-m_new, -m_new);
#pragma unroll
            for (int u = 0; u < 4; ++u) sum2[u] = 0ull;
#pragma unroll
            for (int c = 0; c < NCH / 2; ++c) {
              uint32_t pk[16];
              softmax_chunk<BF16, 0>(r[c], scale2, negm2, sum2, pk);
              tmem_st16(tSj + c * 16, pk);
            }
            rescale_o<D>(tO, alpha);
            m_used = m_new;
          }
          tmem_st_wait();
          tc_fence_before();
          mbar_arrive(BAR(BAR_PFULLA + t));
#pragma unroll
          for (int c = NCH / 2; c < NCH; ++c) {
            uint32_t pk[16];
            softmax_chunk<BF16, poly_pairs<BN>()>(r[c], scale2, negm2, sum2, pk);
            tmem_st16(tSj + c * 16, pk);
          }
          tmem_st_wait();
          tc_fence_before();
          mbar_arrive(BAR(BAR_PFULLB + t));
        }
        const uint64_t s01 = fadd2(fadd2(sum2[0], sum2[1]), fadd2(sum2[2], sum2[3]));
        l = l * alpha + (f2lo(s01) + f2hi(s01));
      }
      if (ok) ok = mbar_wait<kSoftmaxCopy>(BAR(BAR_OFULL + t), 0, p.status, kDevTimeoutO);
      ok = warp_all(ok);
      if (ok) {
        tc_fence_after();
        const float inv_l = 1.0f / l;
        uint8_t* orow = reinterpret_cast<uint8_t*>(p.o) + (static_cast<size_t>(tile.bh) * p.S + qrow) * (D * 2);
#pragma unroll 1
        for (int c = 0; c < D / 32; ++c) {
          uint32_t o[32];
          tmem_ld32(tO + c * 32, o);
          tmem_ld_wait(o);
          uint32_t pk[16];
#pragma unroll
          for (int i = 0; i < 16; ++i)
            pk[i] = pack2<BF16>(__uint_as_float(o[2 * i]) * inv_l, __uint_as_float(o[2 * i + 1]) * inv_l);
          if (qrow < p.S) {
            uint4* dst = reinterpret_cast<uint4*>(orow + c * 64);
#pragma unroll
            for (int v = 0; v < 4; ++v)
              dst[v] = make_uint4(pk[4 * v], pk[4 * v + 1], pk[4 * v + 2], pk[4 * v + 3]);
          }
        }
        if (p.lse != nullptr && qrow < p.S)
          p.lse[static_cast<size_t>(tile.bh) * p.S + qrow] = m_used + log2f(l);
      }
    }
  }
#undef BAR

  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

template <int D, int BN, bool BF16>
cudaError_t launch_fwd_t(const CUtensorMap& tmQ, const CUtensorMap& tmK, const CUtensorMap& tmV,
                         const FwdParams& p, cudaStream_t stream) {
  using C = FwdCfg<D, BN>;
  auto kern = fa_fwd_kernel<D, BN, BF16>;
  static std::atomic<bool> smem_set[64];
  cudaError_t e = opt_in_smem(kern, C::kSmemBytes, smem_set, reg_split<BN>() ? kLaunchRegs : 0);
  if (e != cudaSuccess) return e;
  kern<<<p.n_items, kThreads, C::kSmemBytes, stream>>>(tmQ, tmK, tmV, p);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_fwd(const CUtensorMap& tmQ, const CUtensorMap& tmK, const CUtensorMap& tmV,
                       const FwdParams& p, int D, int block_n, bool bf16, cudaStream_t stream) {
#define FA_FWD_CASE(DD, NN, BB)                                              \
  if (D == DD && block_n == NN && bf16 == BB)                                \
    return launch_fwd_t<DD, NN, BB>(tmQ, tmK, tmV, p, stream);
  FA_FWD_CASE(32, 64, false)
  FA_FWD_CASE(32, 128, false)
  FA_FWD_CASE(64, 64, false)
  FA_FWD_CASE(64, 128, false)
  FA_FWD_CASE(128, 64, false)
  FA_FWD_CASE(128, 128, false)
  FA_FWD_CASE(32, 64, true)
  FA_FWD_CASE(32, 128, true)
  FA_FWD_CASE(64, 64, true)
  FA_FWD_CASE(64, 128, true)
  FA_FWD_CASE(128, 64, true)
  FA_FWD_CASE(128, 128, true)
#undef FA_FWD_CASE
  return cudaErrorInvalidValue;
}

}  // namespace fa
