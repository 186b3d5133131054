// Backward-pass kernels for sm_100a.
//
// delta preprocess: delta[r] = sum_d dO[r, d] * O[r, d] in fp32 (the reference computes this
// with a torch expression on the host: attention/backward/fused_backward.py:175).
#include "fa_internal.h"
#include "fa_sm100.cuh"

namespace fa {
namespace {

// One 16-byte vector (8 elements) per thread; D / 8 threads share a row.
template <int D, bool BF16>
__global__ void __launch_bounds__(256) bwd_preprocess_kernel(const BwdParams p, long long rows) {
  constexpr int kTPR = D / 8;  // threads per row
  const long long gtid = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  const long long row = gtid / kTPR;
  const int part = static_cast<int>(gtid % kTPR);
  float acc = 0.f;
  if (row < rows) {
    const uint4 a = reinterpret_cast<const uint4*>(p.o)[row * kTPR + part];
    const uint4 b = reinterpret_cast<const uint4*>(p.dO)[row * kTPR + part];
    const uint32_t av[4] = {a.x, a.y, a.z, a.w};
    const uint32_t bv[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float2 fa, fb;
      if constexpr (BF16) {
        fa = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&av[i]));
        fb = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&bv[i]));
      } else {
        fa = __half22float2(*reinterpret_cast<const __half2*>(&av[i]));
        fb = __half22float2(*reinterpret_cast<const __half2*>(&bv[i]));
      }
      acc = fmaf(fa.x, fb.x, acc);
      acc = fmaf(fa.y, fb.y, acc);
    }
  }
#pragma unroll
  for (int off = kTPR / 2; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
  if (row < rows && part == 0) p.delta[row] = acc;
}

template <int D, bool BF16>
cudaError_t launch_pre_t(const BwdParams& p, cudaStream_t stream) {
  const long long rows = static_cast<long long>(p.B) * p.H * p.S;
  const long long threads = rows * (D / 8);
  const int block = 256;
  const long long grid = (threads + block - 1) / block;
  bwd_preprocess_kernel<D, BF16><<<static_cast<unsigned>(grid), block, 0, stream>>>(p, rows);
  return cudaGetLastError();
}

// ============================================================================ dK/dV and dQ
// Two atomic-free backward kernels on 128 x 128 tiles (every UMMA is M=128, N=128 or N=D).
//   dQ:    CTA = 128 query rows of one head (Q, dO resident); streams 128-key K and V tiles up
//          to the diagonal (reference loop: attention/backward/fused_backward.py:128-144).
//          TMEM: dQ | S | dP[0] | dP[1].  S is released as soon as both compute warpgroups have
//          read it, so S(s+1) runs on the tensor core while P(s) is being computed; dS overwrites
//          the first half of each warpgroup's own dP columns and feeds dQ += dS K from TMEM.
//   dK/dV: CTA = 128 keys of one K/V head (K, V resident); streams 128-row Q tiles (with their
//          LSE slices, 3-stage ring) and dO tiles (with their delta slices, 2-stage ring) of
//          every query head of the GQA group, from the diagonal on (reference loop:
//          attention/backward/fused_backward.py:81-103).  TMEM: dV | dK | S^T | dP^T.  P^T
//          overwrites S^T and dS^T overwrites dP^T, and both feed their UMMAs (dV += P^T dO,
//          dK += dS^T Q) straight from TMEM, which leaves the shared memory for a third Q stage:
//          Q(s) is held until dK(s), so with two stages the next tile's load was exposed.
// Warp roles (384 threads): warps 0-3 and 4-7 are two compute warpgroups splitting every tile's
// 128 columns (each thread: one TMEM lane = one row, 64 columns); warps 8 and 10 issue TMA
// loads; warp 9 issues the UMMAs (the whole warp runs the issue loop and one elected lane issues
// each tcgen05 instruction).  All warps run with the launch allocation of 168 registers per thread.
constexpr int kBwdThreads = 384;
constexpr int kBwdWarpLoadA = 8;
constexpr int kBwdWarpMma = 9;
constexpr int kBwdWarpLoadB = 10;
constexpr int kBT = 128;  // tile rows (outer and inner)
constexpr uint32_t kBwdTmemCols = 512;
constexpr int kSmemOptin = 232448;  // max dynamic shared memory per block on sm_100

// Of every 16 exp2 pairs, this many go to the FMA-pipe polynomial: 2 in the dK/dV kernel (3 %
// faster than none; it runs at the power cap, and the polynomial costs less energy than MUFU work),
// none in the dQ kernel (2 % slower with one or two).
#ifndef FA_DKDV_POLY_PAIRS
#define FA_DKDV_POLY_PAIRS 2
#endif
#ifndef FA_DQ_POLY_PAIRS
#define FA_DQ_POLY_PAIRS 0
#endif

// True for the polynomial pairs of a 16-pair group, spread evenly (none when kPoly == 0).
template <int kPoly>
__device__ __forceinline__ constexpr bool poly_pair(int i) {
  return kPoly > 0 && (i % 16) % (16 / (kPoly > 0 ? kPoly : 1)) == (16 / (kPoly > 0 ? kPoly : 1)) - 1;
}

// P = 2^(s * scale - m) for kN values (m given per pair), fp32 results, exp2 on MUFU ex2 except
// kPoly of every 16 pairs on the FMA-pipe polynomial.
template <int kN, int kPoly>
__device__ __forceinline__ void exp2_row(const uint32_t* s, const float* neg_m, float scale, float* out) {
  const uint64_t scale2 = f2(scale, scale);
#pragma unroll
  for (int i = 0; i < kN / 2; ++i) {
    const uint64_t x2 = ffma2(f2u(s[2 * i], s[2 * i + 1]), scale2, f2(neg_m[2 * i], neg_m[2 * i + 1]));
    const uint64_t p2 = poly_pair<kPoly>(i) ? exp2_poly2(x2)
                                                         : f2(ex2_approx(f2lo(x2)), ex2_approx(f2hi(x2)));
    out[2 * i] = f2lo(p2);
    out[2 * i + 1] = f2hi(p2);
  }
}

// P = 2^(s * scale - lse) for kN values with a per-value lse (read as float4 from shared memory,
// so each (x, y) / (z, w) half is a ready register pair): y = lse - s * scale in one packed FMA and
// 2^(-y) on MUFU, so no per-value negation is needed; kPoly of every 16 pairs instead take the
// FMA-pipe polynomial of x = -y.
template <int kN, int kPoly>
__device__ __forceinline__ void exp2_row_lse(const uint32_t* s, const float* lse, float scale, float* out) {
  const uint64_t nscale2 = f2(-scale, -scale);
#pragma unroll
  for (int c = 0; c < kN; c += 4) {
    const float4 l4 = *reinterpret_cast<const float4*>(lse + c);
    const uint64_t y0 = ffma2(f2u(s[c], s[c + 1]), nscale2, f2(l4.x, l4.y));
    const uint64_t y1 = ffma2(f2u(s[c + 2], s[c + 3]), nscale2, f2(l4.z, l4.w));
    if (poly_pair<kPoly>(c / 2)) {
      const uint64_t p2 = exp2_poly2(fsub2(0ull, y0));
      out[c] = f2lo(p2);
      out[c + 1] = f2hi(p2);
    } else {
      out[c] = ex2_neg_approx(f2lo(y0));
      out[c + 1] = ex2_neg_approx(f2hi(y0));
    }
    if (poly_pair<kPoly>(c / 2 + 1)) {
      const uint64_t p2 = exp2_poly2(fsub2(0ull, y1));
      out[c + 2] = f2lo(p2);
      out[c + 3] = f2hi(p2);
    } else {
      out[c + 2] = ex2_neg_approx(f2lo(y1));
      out[c + 3] = ex2_neg_approx(f2hi(y1));
    }
  }
}

// Store one 32-column fp32 chunk of an accumulator row as 16-bit values (64 bytes).
template <bool BF16>
__device__ __forceinline__ void store_row_chunk(uint8_t* dst, const uint32_t (&v)[32], float scale) {
  uint32_t pk[16];
#pragma unroll
  for (int i = 0; i < 16; ++i)
    pk[i] = pack2<BF16>(__uint_as_float(v[2 * i]) * scale, __uint_as_float(v[2 * i + 1]) * scale);
  uint4* d = reinterpret_cast<uint4*>(dst);
#pragma unroll
  for (int q = 0; q < 4; ++q) d[q] = make_uint4(pk[4 * q], pk[4 * q + 1], pk[4 * q + 2], pk[4 * q + 3]);
}

// Shared-memory geometry of a 128-row tile of head dim D: rows of swizzle chunks, 64 columns
// (128-byte rows, 128-byte swizzle) for D = 64 and 128, one 32-column chunk (64-byte rows,
// 64-byte swizzle) for D = 32.
template <int D>
struct BwdTile {
  static constexpr int kSwBytes = D >= 64 ? 128 : 64;
  static constexpr int kChunkCols = kSwBytes / 2;
  static constexpr int kChunks = D / kChunkCols;
  static constexpr int kChunkBytes = kBT * kSwBytes;  // one chunk of all 128 rows
  static constexpr uint32_t kLayout = D >= 64 ? kLayoutSw128 : kLayoutSw64;
  static constexpr int kSbo = 8 * kSwBytes;           // bytes between 8-row groups
  static constexpr int kKSteps = kSwBytes / 32;       // 16-element K steps per row
  static constexpr int kRowStep = 16 * kSwBytes;      // 16 rows: one K step of an MN-major operand
};

// K-major descriptor of a tile (A or B operand whose K dimension is the head dim).
template <int D>
__device__ __forceinline__ uint64_t kmajor_desc(uint32_t saddr) {
  return sdesc_sw(saddr, 16, BwdTile<D>::kSbo, BwdTile<D>::kLayout);
}
// MN-major descriptor of a tile (B operand whose N dimension is the head dim, K the 128 rows).
template <int D>
__device__ __forceinline__ uint64_t mnmajor_desc(uint32_t saddr) {
  return sdesc_sw(saddr, BwdTile<D>::kChunkBytes, BwdTile<D>::kSbo, BwdTile<D>::kLayout);
}

// Load a 128-row tile (all D columns) of head `bh`, rows [row0, row0 + 128), with TMA.
template <int D>
__device__ __forceinline__ void load_tile(uint32_t dst, const CUtensorMap* map, uint32_t bar, int row0, int bh,
                                          uint64_t policy) {
  using T = BwdTile<D>;
#pragma unroll
  for (int c = 0; c < T::kChunks; ++c)
    tma_load_3d(dst + c * T::kChunkBytes, map, bar, c * T::kChunkCols, row0, bh, policy);
}

// D[128 x 128] (+)= A[128 x D] * B[128 x D]^T, both K-major tiles of 128 rows (issued by a whole warp).
template <int D, bool BF16>
__device__ __forceinline__ void umma_rows_rows(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc) {
  using T = BwdTile<D>;
  constexpr uint32_t IDESC = idesc_f16(BF16, kBT, kBT, false, false);
#pragma unroll
  for (int k = 0; k < D / 16; ++k) {
    const uint32_t off = (k / T::kKSteps) * T::kChunkBytes + (k % T::kKSteps) * 32;
    umma_ss_w(d_tmem, desc_add(a_desc, off), desc_add(b_desc, off), IDESC, k > 0 ? 1u : 0u);
  }
}

// acc[128 x D] (+)= A[128 x 128] (16-bit in TMEM, K-major) * B[128 x D] (MN-major tile), issued by
// a whole warp.
// A is stored in two halves, one per compute warpgroup: K columns 0-63 packed in TMEM columns
// [a, a + 32), K columns 64-127 in [a + 64, a + 96) (each warpgroup writes into the first half of
// its own column range, so it never overwrites values the other warpgroup has yet to read).
template <int D, bool BF16>
__device__ __forceinline__ void umma_tmem_tile(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t acc) {
  constexpr uint32_t IDESC = idesc_f16(BF16, kBT, D, false, true);
#pragma unroll
  for (int k = 0; k < kBT / 16; ++k)
    umma_ts_w(d_tmem, a_tmem + (k / 4) * 64 + (k % 4) * 8, desc_add(b_desc, k * BwdTile<D>::kRowStep), IDESC,
            (acc | k) ? 1u : 0u);
}

struct BwdSmem {
  uint32_t base;
  uint8_t* ptr;
  uint32_t bar0;
  volatile uint32_t* tmem_slot;
  volatile int* abort_slot;
};

// Aligns the working area to 1 KiB inside the dynamic allocation; `ok` is false if the
// allocation's start leaves too little slack (never expected: the start is 1 KiB aligned).
template <int kUsed>
__device__ __forceinline__ BwdSmem bwd_smem(bool& ok) {
  extern __shared__ uint8_t smem_raw[];
  BwdSmem s;
  const uint32_t raw = smem_u32(smem_raw);
  s.base = (raw + 1023u) & ~1023u;
  ok = (s.base - raw) + kUsed <= static_cast<uint32_t>(kSmemOptin);
  s.ptr = smem_raw + (s.base - raw);
  s.bar0 = s.base + kUsed - 256;
  s.tmem_slot = reinterpret_cast<volatile uint32_t*>(s.ptr + kUsed - 256 + 8 * 28);
  s.abort_slot = reinterpret_cast<volatile int*>(s.ptr + kUsed - 256 + 8 * 28 + 4);
  return s;
}

// Common prologue: abort check, TMEM allocation.  Returns false (uniformly) if the CTA must stop.
__device__ __forceinline__ bool bwd_setup(const BwdSmem& sm, bool smem_ok, const BwdParams& p, uint32_t& tmem) {
  if (threadIdx.x == 0) {
    int st = ld_status(p.status);
    if (st == 0 && !smem_ok) {
      record_error(p.status, kDevSmemLayout, 0);
      st = kDevSmemLayout;
    }
    *sm.abort_slot = st;
  }
  __syncthreads();
  if (*sm.abort_slot != 0) return false;
  if (threadIdx.x / 32 == 0) {
    tmem_alloc(smem_u32(const_cast<uint32_t*>(sm.tmem_slot)), kBwdTmemCols);
    tmem_relinquish();
  }
  return true;
}

__device__ __forceinline__ void bwd_teardown(uint32_t tmem) {
  tc_fence_before();
  __syncthreads();
  if (threadIdx.x / 32 == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, kBwdTmemCols);
  }
}

// ---------------------------------------------------------------------------- dQ
template <int D>
struct DqCfg {
  static constexpr int kTile = kBT * D * 2;
  static constexpr int kBudget = kSmemOptin - 1024 - 256;
  static constexpr int kSlots = (kBudget - 2 * kTile) / kTile;
  static constexpr int kVStages = (kSlots / 2) > 4 ? 4 : (kSlots / 2);
  static constexpr int kKStages = (kSlots - kVStages) > 4 ? 4 : (kSlots - kVStages);
  static_assert(kKStages >= 2 && kVStages >= 2, "need double-buffered K and V rings");
  static constexpr int kOffQ = 0, kOffdO = kTile, kOffK = 2 * kTile;
  static constexpr int kOffV = kOffK + kKStages * kTile;
  static constexpr int kUsed = kOffV + kVStages * kTile + 256;
};

enum : int {
  DQ_OUTER = 0, DQ_KFULL = 1, DQ_KEMPTY = 5, DQ_VFULL = 9, DQ_VEMPTY = 13, DQ_SFULL = 17, DQ_SFREE = 18,
  DQ_DPFULL = 19 /* + 2 */, DQ_DSREADY = 21 /* + 2 */, DQ_ACC = 23, DQ_DRAIN = 24,
  DQ_NEVER = 25 /* never arrived at (failure-detection test build) */
};

template <int D, bool BF16>
__global__ void __launch_bounds__(kBwdThreads, 1)
    bwd_dq_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                  const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmdO,
                  const BwdParams p) {
  using C = DqCfg<D>;
  constexpr int KST = C::kKStages, VST = C::kVStages;
  bool smem_ok;
  const BwdSmem sm = bwd_smem<C::kUsed>(smem_ok);
#define BAR(i) (sm.bar0 + 8u * static_cast<uint32_t>(i))
  const uint32_t sQ = sm.base + C::kOffQ, sdO = sm.base + C::kOffdO;
  const uint32_t sK = sm.base + C::kOffK, sV = sm.base + C::kOffV;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;

  if (threadIdx.x == 0 && smem_ok) {
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
    tma_prefetch_desc(&tmdO);
    mbar_init(BAR(DQ_OUTER), 1);
    for (int s = 0; s < 4; ++s) {
      mbar_init(BAR(DQ_KFULL + s), 1);
      mbar_init(BAR(DQ_KEMPTY + s), 1);
      mbar_init(BAR(DQ_VFULL + s), 1);
      mbar_init(BAR(DQ_VEMPTY + s), 1);
    }
    mbar_init(BAR(DQ_SFULL), 1);
    mbar_init(BAR(DQ_SFREE), 256);
    mbar_init(BAR(DQ_DPFULL + 0), 1);
    mbar_init(BAR(DQ_DPFULL + 1), 1);
    mbar_init(BAR(DQ_DSREADY + 0), 256);
    mbar_init(BAR(DQ_DSREADY + 1), 256);
    mbar_init(BAR(DQ_ACC), 1);
    mbar_init(BAR(DQ_DRAIN), 1);
    mbar_init(BAR(DQ_NEVER), 1);
    fence_barrier_init();
  }
  uint32_t tmem;
  if (!bwd_setup(sm, smem_ok, p, tmem)) return;
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  tmem = *sm.tmem_slot;

  // work item: bands of heads, query tile descending (the longest rows first)
  const int nqt = (p.S + kBT - 1) / kBT;
  const UnitLevel ul = band_order(blockIdx.x, p.B * p.H, nqt, p.band);
  const int bh = ul.unit;
  const int i = nqt - 1 - ul.level;
  const int b = bh / p.H, h = bh - b * p.H;
  const int bkv = b * p.H_kv + h / p.group;
  const int nsteps = min(i * kBT + kBT - 1, p.S - 1) / kBT + 1;
  const uint32_t tDQ = tmem, tS = tmem + 128, tDP = tmem + 256;

  if (warp >= 8) {
    if (warp == kBwdWarpLoadA) {
      // ---------------- TMA: Q and dO once, then the K ring
      if (lane == 0) {
        const uint64_t pol_once = policy_evict_first();
        const uint64_t pol_shared = policy_evict_last();
        mbar_arrive_expect_tx(BAR(DQ_OUTER), 2 * C::kTile);
        load_tile<D>(sQ, &tmQ, BAR(DQ_OUTER), i * kBT, bh, pol_once);
        load_tile<D>(sdO, &tmdO, BAR(DQ_OUTER), i * kBT, bh, pol_once);
        int issued = 0;
        for (int s = 0; s < nsteps; ++s) {
          const int st = s % KST;
          if (!mbar_wait(BAR(DQ_KEMPTY + st), ((s / KST) & 1) ^ 1, p.status, kDevTimeoutBwd)) break;
          mbar_arrive_expect_tx(BAR(DQ_KFULL + st), C::kTile);
          load_tile<D>(sK + st * C::kTile, &tmK, BAR(DQ_KFULL + st), s * kBT, bkv, pol_shared);
          ++issued;
        }
        drain_wait(BAR(DQ_OUTER), 0, p.status);
        for (int s = max(0, issued - KST); s < issued; ++s) drain_wait(BAR(DQ_KFULL + s % KST), (s / KST) & 1, p.status);
      }
      __syncwarp();
    } else if (warp == kBwdWarpLoadB) {
      // ---------------- TMA: the V ring
      if (lane == 0) {
        const uint64_t pol_shared = policy_evict_last();
        int issued = 0;
        for (int s = 0; s < nsteps; ++s) {
          const int st = s % VST;
          if (!mbar_wait(BAR(DQ_VEMPTY + st), ((s / VST) & 1) ^ 1, p.status, kDevTimeoutBwd)) break;
          mbar_arrive_expect_tx(BAR(DQ_VFULL + st), C::kTile);
          load_tile<D>(sV + st * C::kTile, &tmV, BAR(DQ_VFULL + st), s * kBT, bkv, pol_shared);
          ++issued;
        }
        for (int s = max(0, issued - VST); s < issued; ++s) drain_wait(BAR(DQ_VFULL + s % VST), (s / VST) & 1, p.status);
      }
      __syncwarp();
    } else if (warp == kBwdWarpMma) {
      // ---------------- UMMA issuer
      {  // the whole warp runs the issue loop; one elected lane issues each tcgen05 op
        const uint64_t dQd = kmajor_desc<D>(sQ), dOd = kmajor_desc<D>(sdO);
        const uint64_t dKk = kmajor_desc<D>(sK), dVk = kmajor_desc<D>(sV);
        const uint64_t dKm = mnmajor_desc<D>(sK);
        bool ok = warp_all(mbar_wait(BAR(DQ_OUTER), 0, p.status, kDevTimeoutBwd)) &&
                  warp_all(mbar_wait(BAR(DQ_KFULL + 0), 0, p.status, kDevTimeoutBwd)) &&
                  warp_all(mbar_wait(BAR(DQ_VFULL + 0), 0, p.status, kDevTimeoutBwd));
        if (ok) {
          tc_fence_after();
          umma_rows_rows<D, BF16>(tS, dQd, dKk);  // S(0) = Q K_0^T
          umma_commit_w(BAR(DQ_SFULL));
          umma_rows_rows<D, BF16>(tDP, dOd, dVk);  // dP(0) = dO V_0^T
          umma_commit_w(BAR(DQ_DPFULL + 0));
          umma_commit_w(BAR(DQ_VEMPTY + 0));
        }
        for (int s = 0; ok && s < nsteps; ++s) {
          FA_STALL_HERE(s, BAR(DQ_NEVER), p.status, ok)
          if (s + 1 < nsteps) {
            const int k1 = (s + 1) % KST, v1 = (s + 1) % VST;
            if (!(ok = warp_all(mbar_wait(BAR(DQ_SFREE), s & 1, p.status, kDevTimeoutBwd)))) break;
            if (!(ok = warp_all(mbar_wait(BAR(DQ_KFULL + k1), ((s + 1) / KST) & 1, p.status, kDevTimeoutBwd)))) break;
            tc_fence_after();
            umma_rows_rows<D, BF16>(tS, dQd, desc_add(dKk, k1 * C::kTile));
            umma_commit_w(BAR(DQ_SFULL));
            if (!(ok = warp_all(mbar_wait(BAR(DQ_VFULL + v1), ((s + 1) / VST) & 1, p.status, kDevTimeoutBwd)))) break;
            tc_fence_after();
            umma_rows_rows<D, BF16>(tDP + 128 * ((s + 1) & 1), dOd, desc_add(dVk, v1 * C::kTile));
            umma_commit_w(BAR(DQ_DPFULL + ((s + 1) & 1)));
            umma_commit_w(BAR(DQ_VEMPTY + v1));
          }
          // dS(s) is ready.  One barrier per step parity: S(s+1) and dP(s+1) are already issued,
          // so the compute warps can finish step s+1 before the issuer looks, and a single
          // barrier would then be two phases ahead of the parity waited on.
          if (!(ok = warp_all(mbar_wait(BAR(DQ_DSREADY + (s & 1)), (s >> 1) & 1, p.status, kDevTimeoutBwd)))) break;
          tc_fence_after();
          umma_tmem_tile<D, BF16>(tDQ, tDP + 128 * (s & 1), desc_add(dKm, (s % KST) * C::kTile), s > 0 ? 1u : 0u);
          umma_commit_w(BAR(DQ_KEMPTY + s % KST));
        }
        if (ok) umma_commit_w(BAR(DQ_ACC));
        umma_commit_w(BAR(DQ_DRAIN));
        drain_wait(BAR(DQ_DRAIN), 0, p.status);
      }
      __syncwarp();
    }
  } else {
    // ---------------- compute warpgroups: warpgroup w owns columns [64 w, 64 w + 64)
    const int w = warp / 4, wq = warp % 4;
    const int row = wq * 32 + lane;
    const int qrow = i * kBT + row;
    const uint32_t lane_off = static_cast<uint32_t>(wq * 32) << 16;
    const size_t ridx = static_cast<size_t>(bh) * p.S + qrow;
    const float lse_r = qrow < p.S ? p.lse[ridx] : 0.f;
    const float del_r = qrow < p.S ? p.delta[ridx] : 0.f;
    float neg_lse[64];
#pragma unroll
    for (int c = 0; c < 64; ++c) neg_lse[c] = -lse_r;
    bool ok = true;
    for (int s = 0; s < nsteps; ++s) {
      if (!(ok = warp_all(mbar_wait(BAR(DQ_SFULL), s & 1, p.status, kDevTimeoutBwd)))) break;
      tc_fence_after();
      uint32_t sv[2][32];
      tmem_ld32(tS + lane_off + 64 * w, sv[0]);
      tmem_ld32(tS + lane_off + 64 * w + 32, sv[1]);
      tmem_ld_wait(sv[0]);
      tmem_ld_wait(sv[1]);
      tc_fence_before();
      mbar_arrive(BAR(DQ_SFREE));
      float pr[64];
      exp2_row<32, FA_DQ_POLY_PAIRS>(sv[0], neg_lse, p.scale_log2, pr);
      exp2_row<32, FA_DQ_POLY_PAIRS>(sv[1], neg_lse, p.scale_log2, pr + 32);
      const int k0 = s * kBT + 64 * w;
      if (k0 + 63 > i * kBT || k0 + 64 > p.S) {
#pragma unroll
        for (int c = 0; c < 64; ++c)
          if (k0 + c > qrow || k0 + c >= p.S) pr[c] = 0.f;
      }
      if (!(ok = warp_all(mbar_wait(BAR(DQ_DPFULL + (s & 1)), (s >> 1) & 1, p.status, kDevTimeoutBwd)))) break;
      tc_fence_after();
      const uint32_t tdp = tDP + 128 * (s & 1) + lane_off;
      uint32_t dp[2][32];
      tmem_ld32(tdp + 64 * w, dp[0]);
      tmem_ld32(tdp + 64 * w + 32, dp[1]);
      tmem_ld_wait(dp[0]);
      tmem_ld_wait(dp[1]);
#pragma unroll
      for (int h2 = 0; h2 < 2; ++h2) {
        uint32_t pk[16];
#pragma unroll
        for (int c2 = 0; c2 < 16; ++c2) {
          const uint64_t d2 = fadd2(f2u(dp[h2][2 * c2], dp[h2][2 * c2 + 1]), f2(-del_r, -del_r));
          const uint64_t ds = fmul2(f2(pr[32 * h2 + 2 * c2], pr[32 * h2 + 2 * c2 + 1]), d2);
          pk[c2] = pack2<BF16>(f2lo(ds), f2hi(ds));
        }
        tmem_st16(tdp + 64 * w + 16 * h2, pk);
      }
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(BAR(DQ_DSREADY + (s & 1)));
    }
    if (ok) ok = mbar_wait(BAR(DQ_ACC), 0, p.status, kDevTimeoutBwd);
    ok = warp_all(ok);
    if (ok) {
      tc_fence_after();
      uint8_t* orow = reinterpret_cast<uint8_t*>(p.dq) + ridx * (D * 2);
      if constexpr (D >= 64) {
        for (int c = w * (D / 64); c < (w + 1) * (D / 64); ++c) {  // 32-column chunks
          uint32_t v[32];
          tmem_ld32(tDQ + lane_off + c * 32, v);
          tmem_ld_wait(v);
          if (qrow < p.S) store_row_chunk<BF16>(orow + c * 64, v, p.sm_scale);
        }
      } else {  // D = 32: each warpgroup stores 16 columns (32 bytes) of its row
        uint32_t v[16];
        tmem_ld16(tDQ + lane_off + w * 16, v);
        tmem_ld_wait16(v);
        uint32_t pk[8];
#pragma unroll
        for (int i = 0; i < 8; ++i)
          pk[i] = pack2<BF16>(__uint_as_float(v[2 * i]) * p.sm_scale, __uint_as_float(v[2 * i + 1]) * p.sm_scale);
        if (qrow < p.S) {
          uint4* d = reinterpret_cast<uint4*>(orow + w * 32);
          d[0] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
          d[1] = make_uint4(pk[4], pk[5], pk[6], pk[7]);
        }
      }
    }
  }
#undef BAR
  bwd_teardown(tmem);
}

// ---------------------------------------------------------------------------- dK / dV
template <int D>
struct DkdvCfg {
  static constexpr int kTile = kBT * D * 2;
  static constexpr int kStat = kBT * 4;  // one LSE (or delta) slice of a query tile
  static constexpr int kBudget = kSmemOptin - 256;
  static constexpr int kDOStages = 2;    // dO is released after dS^T (before dK's Q), two stages suffice
  static constexpr int kQFit = (kBudget - 2 * kTile - kDOStages * (kTile + kStat)) / (kTile + kStat);
  static constexpr int kQStages = kQFit > 4 ? 4 : kQFit;  // Q is held until dK, so it gets more
  static_assert(kQStages >= 3, "need a triple-buffered Q ring");
  static constexpr int kOffK = 0, kOffV = kTile, kOffQ = 2 * kTile;
  static constexpr int kOffDO = kOffQ + kQStages * kTile;
  static constexpr int kOffLse = kOffDO + kDOStages * kTile;
  static constexpr int kOffDelta = kOffLse + kQStages * kStat;
  static constexpr int kUsed = kOffDelta + kDOStages * kStat + 256;
  static_assert(kUsed <= kSmemOptin, "shared memory budget");
};

enum : int {
  KV_OUTER = 0, KV_QFULL = 1 /* + Q stage (4) */, KV_QEMPTY = 5 /* + Q stage (4) */,
  KV_OFULL = 9 /* + dO stage (2) */, KV_OEMPTY = 11 /* + dO stage (2) */, KV_STFULL = 13,
  KV_PREADY = 14, KV_DPFULL = 15, KV_DSREADY = 16, KV_ACC = 17, KV_DRAIN = 18,
  KV_NEVER = 19 /* never arrived at (failure-detection test build) */
};

template <int D, bool BF16>
__global__ void __launch_bounds__(kBwdThreads, 1)
    bwd_dkdv_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                    const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmdO,
                    const BwdParams p) {
  using C = DkdvCfg<D>;
  constexpr int QST = C::kQStages, OST = C::kDOStages;
  bool smem_ok;
  const BwdSmem sm = bwd_smem<C::kUsed>(smem_ok);
#define BAR(i) (sm.bar0 + 8u * static_cast<uint32_t>(i))
  const uint32_t sK = sm.base + C::kOffK, sV = sm.base + C::kOffV;
  const uint32_t sQ = sm.base + C::kOffQ, sdO = sm.base + C::kOffDO;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;

  if (threadIdx.x == 0 && smem_ok) {
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
    tma_prefetch_desc(&tmdO);
    mbar_init(BAR(KV_OUTER), 1);
    for (int s = 0; s < 4; ++s) {
      mbar_init(BAR(KV_QFULL + s), 1);
      mbar_init(BAR(KV_QEMPTY + s), 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(BAR(KV_OFULL + s), 1);
      mbar_init(BAR(KV_OEMPTY + s), 1);
    }
    mbar_init(BAR(KV_STFULL), 1);
    mbar_init(BAR(KV_PREADY), 256);
    mbar_init(BAR(KV_DPFULL), 1);
    mbar_init(BAR(KV_DSREADY), 256);
    mbar_init(BAR(KV_ACC), 1);
    mbar_init(BAR(KV_DRAIN), 1);
    mbar_init(BAR(KV_NEVER), 1);
    fence_barrier_init();
  }
  uint32_t tmem;
  if (!bwd_setup(sm, smem_ok, p, tmem)) return;
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  tmem = *sm.tmem_slot;

  // work item: bands of (b, kv head), key tile ascending (tile 0 sees every query: heaviest first)
  const int nkt = (p.S + kBT - 1) / kBT;
  const UnitLevel ul = band_order(blockIdx.x, p.B * p.H_kv, nkt, p.band);
  const int bkv = ul.unit;
  const int j = ul.level;
  const int b = bkv / p.H_kv, g = bkv - b * p.H_kv;
  const int nqi = nkt - j;  // query tiles j .. nkt-1 see these keys
  const int nsteps = p.group * nqi;
  const uint32_t tDV = tmem, tDK = tmem + 128, tST = tmem + 256, tDPT = tmem + 384;

  if (warp >= 8) {
    if (warp == kBwdWarpLoadA) {
      // ---------------- TMA: K and V once, then the Q tiles with their LSE slices
      if (lane == 0) {
        const uint64_t pol_once = policy_evict_first();
        const uint64_t pol_shared = policy_evict_last();
        mbar_arrive_expect_tx(BAR(KV_OUTER), 2 * C::kTile);
        load_tile<D>(sK, &tmK, BAR(KV_OUTER), j * kBT, bkv, pol_once);
        load_tile<D>(sV, &tmV, BAR(KV_OUTER), j * kBT, bkv, pol_once);
        int issued = 0;
        for (int s = 0; s < nsteps; ++s) {
          const int st = s % QST;
          if (!mbar_wait(BAR(KV_QEMPTY + st), ((s / QST) & 1) ^ 1, p.status, kDevTimeoutBwd)) break;
          const int hh = s / nqi, it = j + (s - hh * nqi);
          const int bh = b * p.H + g * p.group + hh;
          const int rows = min(kBT, p.S - it * kBT);  // a multiple of 64 (S % 64 == 0)
          mbar_arrive_expect_tx(BAR(KV_QFULL + st), C::kTile + rows * 4);
          load_tile<D>(sQ + st * C::kTile, &tmQ, BAR(KV_QFULL + st), it * kBT, bh, pol_shared);
          bulk_load(sm.base + C::kOffLse + st * C::kStat, p.lse + static_cast<size_t>(bh) * p.S + it * kBT,
                    rows * 4, BAR(KV_QFULL + st));
          ++issued;
        }
        drain_wait(BAR(KV_OUTER), 0, p.status);
        for (int s = max(0, issued - QST); s < issued; ++s) drain_wait(BAR(KV_QFULL + s % QST), (s / QST) & 1, p.status);
      }
      __syncwarp();
    } else if (warp == kBwdWarpLoadB) {
      // ---------------- TMA: the dO tiles with their delta slices
      if (lane == 0) {
        const uint64_t pol_shared = policy_evict_last();
        int issued = 0;
        for (int s = 0; s < nsteps; ++s) {
          const int st = s % OST;
          if (!mbar_wait(BAR(KV_OEMPTY + st), ((s / OST) & 1) ^ 1, p.status, kDevTimeoutBwd)) break;
          const int hh = s / nqi, it = j + (s - hh * nqi);
          const int bh = b * p.H + g * p.group + hh;
          const int rows = min(kBT, p.S - it * kBT);
          mbar_arrive_expect_tx(BAR(KV_OFULL + st), C::kTile + rows * 4);
          load_tile<D>(sdO + st * C::kTile, &tmdO, BAR(KV_OFULL + st), it * kBT, bh, pol_shared);
          bulk_load(sm.base + C::kOffDelta + st * C::kStat, p.delta + static_cast<size_t>(bh) * p.S + it * kBT,
                    rows * 4, BAR(KV_OFULL + st));
          ++issued;
        }
        for (int s = max(0, issued - OST); s < issued; ++s) drain_wait(BAR(KV_OFULL + s % OST), (s / OST) & 1, p.status);
      }
      __syncwarp();
    } else if (warp == kBwdWarpMma) {
      // ---------------- UMMA issuer.  Per step s: dV += P^T(s) dO(s) (P^T read from TMEM where it
      // overwrote S^T(s)), then S^T(s+1) into the same columns, dK += dS^T(s) Q(s) (dS^T over
      // dP^T(s)), then dP^T(s+1).  Each barrier's next phase needs its waiter to have passed the
      // current one (S^T(s+1) follows PREADY(s), dP^T(s+1) follows DSREADY(s)), so no barrier can
      // run two phases ahead of the parity waited on.
      {  // the whole warp runs the issue loop; one elected lane issues each tcgen05 op
        const uint64_t dKd = kmajor_desc<D>(sK), dVd = kmajor_desc<D>(sV);
        const uint64_t dQk = kmajor_desc<D>(sQ), dOk = kmajor_desc<D>(sdO);
        const uint64_t dQm = mnmajor_desc<D>(sQ), dOm = mnmajor_desc<D>(sdO);
        bool ok = warp_all(mbar_wait(BAR(KV_OUTER), 0, p.status, kDevTimeoutBwd)) &&
                  warp_all(mbar_wait(BAR(KV_QFULL + 0), 0, p.status, kDevTimeoutBwd)) &&
                  warp_all(mbar_wait(BAR(KV_OFULL + 0), 0, p.status, kDevTimeoutBwd));
        if (ok) {
          tc_fence_after();
          umma_rows_rows<D, BF16>(tST, dKd, dQk);  // S^T(0) = K Q_0^T
          umma_commit_w(BAR(KV_STFULL));
          umma_rows_rows<D, BF16>(tDPT, dVd, dOk);  // dP^T(0) = V dO_0^T
          umma_commit_w(BAR(KV_DPFULL));
        }
        for (int s = 0; ok && s < nsteps; ++s) {
          const int qs = s % QST, os = s % OST;
          FA_STALL_HERE(s, BAR(KV_NEVER), p.status, ok)
          if (!(ok = warp_all(mbar_wait(BAR(KV_PREADY), s & 1, p.status, kDevTimeoutBwd)))) break;
          tc_fence_after();
          umma_tmem_tile<D, BF16>(tDV, tST, desc_add(dOm, os * C::kTile), s > 0 ? 1u : 0u);  // dV += P^T dO
          if (s + 1 < nsteps) {
            const int q1 = (s + 1) % QST;
            if (!(ok = warp_all(mbar_wait(BAR(KV_QFULL + q1), ((s + 1) / QST) & 1, p.status, kDevTimeoutBwd)))) break;
            tc_fence_after();
            umma_rows_rows<D, BF16>(tST, dKd, desc_add(dQk, q1 * C::kTile));  // S^T(s+1)
            umma_commit_w(BAR(KV_STFULL));
          }
          if (!(ok = warp_all(mbar_wait(BAR(KV_DSREADY), s & 1, p.status, kDevTimeoutBwd)))) break;
          tc_fence_after();
          umma_tmem_tile<D, BF16>(tDK, tDPT, desc_add(dQm, qs * C::kTile), s > 0 ? 1u : 0u);  // dK += dS^T Q
          umma_commit_w(BAR(KV_QEMPTY + qs));  // Q(s): read by S^T(s) and dK(s)
          // dO(s) stage: its tile is read by dP^T(s) and dV(s), its delta slice by the compute
          // warpgroups while they form dS^T(s), which DSREADY(s) has just confirmed is done.
          umma_commit_w(BAR(KV_OEMPTY + os));
          if (s + 1 < nsteps) {
            const int o1 = (s + 1) % OST;
            if (!(ok = warp_all(mbar_wait(BAR(KV_OFULL + o1), ((s + 1) / OST) & 1, p.status, kDevTimeoutBwd)))) break;
            tc_fence_after();
            umma_rows_rows<D, BF16>(tDPT, dVd, desc_add(dOk, o1 * C::kTile));  // dP^T(s+1)
            umma_commit_w(BAR(KV_DPFULL));
          }
        }
        if (ok) umma_commit_w(BAR(KV_ACC));
        umma_commit_w(BAR(KV_DRAIN));
        drain_wait(BAR(KV_DRAIN), 0, p.status);
      }
      __syncwarp();
    }
  } else {
    // ---------------- compute warpgroups: warpgroup w owns query columns [64 w, 64 w + 64)
    const int w = warp / 4, wq = warp % 4;
    const int row = wq * 32 + lane;
    const int key = j * kBT + row;
    const uint32_t lane_off = static_cast<uint32_t>(wq * 32) << 16;
    const float scale = p.scale_log2;
    bool ok = true;
    for (int s = 0; s < nsteps; ++s) {
      const int qs = s % QST, os = s % OST;
      const int hh = s / nqi, it = j + (s - hh * nqi);
      if (!(ok = warp_all(mbar_wait(BAR(KV_STFULL), s & 1, p.status, kDevTimeoutBwd)))) break;
      tc_fence_after();
      uint32_t sv[2][32];
      tmem_ld32(tST + lane_off + 64 * w, sv[0]);
      tmem_ld32(tST + lane_off + 64 * w + 32, sv[1]);
      tmem_ld_wait(sv[0]);
      tmem_ld_wait(sv[1]);
      const float* lse = reinterpret_cast<const float*>(sm.ptr + C::kOffLse + qs * C::kStat) + 64 * w;
      const float* del = reinterpret_cast<const float*>(sm.ptr + C::kOffDelta + os * C::kStat) + 64 * w;
      float pr[64];
      exp2_row_lse<32, FA_DKDV_POLY_PAIRS>(sv[0], lse, scale, pr);
      exp2_row_lse<32, FA_DKDV_POLY_PAIRS>(sv[1], lse + 32, scale, pr + 32);
      const int q0 = it * kBT + 64 * w;
      if (key > q0 || q0 + 64 > p.S) {  // some query of these 64 precedes the key, or lies past S
#pragma unroll
        for (int c = 0; c < 64; ++c)
          if (key > q0 + c || q0 + c >= p.S) pr[c] = 0.f;
      }
      // P^T -> TMEM over the first half of this warpgroup's own S^T columns (already read)
#pragma unroll
      for (int h2 = 0; h2 < 2; ++h2) {
        uint32_t pk[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) pk[i] = pack2<BF16>(pr[32 * h2 + 2 * i], pr[32 * h2 + 2 * i + 1]);
        tmem_st16(tST + lane_off + 64 * w + 16 * h2, pk);
      }
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(BAR(KV_PREADY));
      // dS^T = P^T (dP^T - delta) -> TMEM over dP^T.  On a ragged last query tile the delta
      // slice past S holds stale bytes: those queries (P = 0) read delta as 0, never 0 * NaN.
      const bool ragged = q0 + 64 > p.S;
      if (!(ok = warp_all(mbar_wait(BAR(KV_DPFULL), s & 1, p.status, kDevTimeoutBwd)))) break;
      tc_fence_after();
      uint32_t dp[2][32];
      tmem_ld32(tDPT + lane_off + 64 * w, dp[0]);
      tmem_ld32(tDPT + lane_off + 64 * w + 32, dp[1]);
      tmem_ld_wait(dp[0]);
      tmem_ld_wait(dp[1]);
#pragma unroll
      for (int h2 = 0; h2 < 2; ++h2) {
        uint32_t pk[16];
#pragma unroll
        for (int c4 = 0; c4 < 8; ++c4) {
          const int c = 32 * h2 + 4 * c4;
          float4 d4 = *reinterpret_cast<const float4*>(del + c);
          if (ragged) {
            d4.x = q0 + c < p.S ? d4.x : 0.f;
            d4.y = q0 + c + 1 < p.S ? d4.y : 0.f;
            d4.z = q0 + c + 2 < p.S ? d4.z : 0.f;
            d4.w = q0 + c + 3 < p.S ? d4.w : 0.f;
          }
          const uint64_t a = fmul2(f2(pr[c], pr[c + 1]),
                                   fsub2(f2u(dp[h2][4 * c4], dp[h2][4 * c4 + 1]), f2(d4.x, d4.y)));
          const uint64_t bb = fmul2(f2(pr[c + 2], pr[c + 3]),
                                    fsub2(f2u(dp[h2][4 * c4 + 2], dp[h2][4 * c4 + 3]), f2(d4.z, d4.w)));
          pk[2 * c4] = pack2<BF16>(f2lo(a), f2hi(a));
          pk[2 * c4 + 1] = pack2<BF16>(f2lo(bb), f2hi(bb));
        }
        tmem_st16(tDPT + lane_off + 64 * w + 16 * h2, pk);
      }
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(BAR(KV_DSREADY));
    }
    if (ok) ok = mbar_wait(BAR(KV_ACC), 0, p.status, kDevTimeoutBwd);
    ok = warp_all(ok);
    if (ok) {
      tc_fence_after();
      // warpgroup 0 writes dV rows, warpgroup 1 writes dK rows (scaled by 1/sqrt(D))
      void* out = (w == 0) ? p.dv : p.dk;
      const float osc = (w == 0) ? 1.0f : p.sm_scale;
      const uint32_t tacc = (w == 0 ? tDV : tDK) + lane_off;
      uint8_t* orow = reinterpret_cast<uint8_t*>(out) + (static_cast<size_t>(bkv) * p.S + key) * (D * 2);
#pragma unroll 1
      for (int c = 0; c < D / 32; ++c) {
        uint32_t v[32];
        tmem_ld32(tacc + c * 32, v);
        tmem_ld_wait(v);
        if (key < p.S) store_row_chunk<BF16>(orow + c * 64, v, osc);
      }
    }
  }
#undef BAR
  bwd_teardown(tmem);
}

template <int D, bool BF16>
cudaError_t launch_dkdv_t(const CUtensorMap& tmQ, const CUtensorMap& tmK, const CUtensorMap& tmV,
                          const CUtensorMap& tmdO, const BwdParams& p, cudaStream_t stream) {
  auto kern = bwd_dkdv_kernel<D, BF16>;
  static std::atomic<bool> smem_set[64];
  cudaError_t e = opt_in_smem(kern, kSmemOptin, smem_set);
  if (e != cudaSuccess) return e;
  const int nkt = (p.S + kBT - 1) / kBT;
  kern<<<p.B * p.H_kv * nkt, kBwdThreads, kSmemOptin, stream>>>(tmQ, tmK, tmV, tmdO, p);
  return cudaGetLastError();
}

template <int D, bool BF16>
cudaError_t launch_dq_t(const CUtensorMap& tmQ, const CUtensorMap& tmK, const CUtensorMap& tmV,
                        const CUtensorMap& tmdO, const BwdParams& p, cudaStream_t stream) {
  auto kern = bwd_dq_kernel<D, BF16>;
  static std::atomic<bool> smem_set[64];
  cudaError_t e = opt_in_smem(kern, kSmemOptin, smem_set);
  if (e != cudaSuccess) return e;
  const int nqt = (p.S + kBT - 1) / kBT;
  kern<<<p.B * p.H * nqt, kBwdThreads, kSmemOptin, stream>>>(tmQ, tmK, tmV, tmdO, p);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_bwd_preprocess(const BwdParams& p, bool bf16, cudaStream_t stream) {
  if (p.D == 32) return bf16 ? launch_pre_t<32, true>(p, stream) : launch_pre_t<32, false>(p, stream);
  if (p.D == 64) return bf16 ? launch_pre_t<64, true>(p, stream) : launch_pre_t<64, false>(p, stream);
  if (p.D == 128) return bf16 ? launch_pre_t<128, true>(p, stream) : launch_pre_t<128, false>(p, stream);
  return cudaErrorInvalidValue;
}

cudaError_t launch_bwd_dkdv(const CUtensorMap& tmQ, const CUtensorMap& tmK, const CUtensorMap& tmV,
                            const CUtensorMap& tmdO, const BwdParams& p, bool bf16, cudaStream_t stream) {
  if (p.D == 32) return bf16 ? launch_dkdv_t<32, true>(tmQ, tmK, tmV, tmdO, p, stream)
                             : launch_dkdv_t<32, false>(tmQ, tmK, tmV, tmdO, p, stream);
  if (p.D == 64) return bf16 ? launch_dkdv_t<64, true>(tmQ, tmK, tmV, tmdO, p, stream)
                             : launch_dkdv_t<64, false>(tmQ, tmK, tmV, tmdO, p, stream);
  if (p.D == 128) return bf16 ? launch_dkdv_t<128, true>(tmQ, tmK, tmV, tmdO, p, stream)
                              : launch_dkdv_t<128, false>(tmQ, tmK, tmV, tmdO, p, stream);
  return cudaErrorInvalidValue;
}

cudaError_t launch_bwd_dq(const CUtensorMap& tmQ, const CUtensorMap& tmK, const CUtensorMap& tmV,
                          const CUtensorMap& tmdO, const BwdParams& p, bool bf16, cudaStream_t stream) {
  if (p.D == 32) return bf16 ? launch_dq_t<32, true>(tmQ, tmK, tmV, tmdO, p, stream)
                             : launch_dq_t<32, false>(tmQ, tmK, tmV, tmdO, p, stream);
  if (p.D == 64) return bf16 ? launch_dq_t<64, true>(tmQ, tmK, tmV, tmdO, p, stream)
                             : launch_dq_t<64, false>(tmQ, tmK, tmV, tmdO, p, stream);
  if (p.D == 128) return bf16 ? launch_dq_t<128, true>(tmQ, tmK, tmV, tmdO, p, stream)
                              : launch_dq_t<128, false>(tmQ, tmK, tmV, tmdO, p, stream);
  return cudaErrorInvalidValue;
}

}  // namespace fa
