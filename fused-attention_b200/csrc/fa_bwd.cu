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
// Shared structure of the two atomic-free backward kernels.  A CTA keeps one 128-row OUTER tile
// resident in shared memory and streams 64-row INNER tiles through a TMA ring:
//   dK/dV: outer = 128 keys (K, V) of one K/V head; inner = 64-query tiles (Q, dO, lse, delta)
//          of every query head of the GQA group, for the query tiles that see those keys
//          (reference loop: attention/backward/fused_backward.py:81-103)
//   dQ:    outer = 128 queries (Q, dO) of one head; inner = 64-key tiles (K, V) up to the
//          diagonal (reference loop: attention/backward/fused_backward.py:128-144)
// Warp roles (384 threads): warps 0-3 / 4-7 = two compute warpgroups that take alternate inner
// steps, warp 8 = TMA producer, warp 9 = UMMA issuer.  TMEM (512 columns):
//   [0, D)            dV   (dK/dV kernel) | dQ (dQ kernel)
//   [128, 128 + D)    dK   (dK/dV kernel)
//   256 + 128 b       buffer b in {0, 1}: 64 columns of S (or S^T), then 64 columns of dP (dP^T).
// P^T (16-bit) overwrites the first 32 columns of S^T and dS (dS^T) the first 32 of dP (dP^T)
// once a thread has read its row, and feed the next UMMAs straight from TMEM.  While one
// warpgroup turns buffer b into P/dS, the tensor core computes the other buffer's S/dP and the
// previous step's accumulations, so neither side waits for the other in steady state.
constexpr int kBwdThreads = 384;
constexpr int kBwdWarpProducer = 8;
constexpr int kBwdWarpMma = 9;
constexpr int kBO = 128;  // outer tile rows
constexpr int kBI = 64;   // inner tile rows
constexpr uint32_t kBwdTmemCols = 512;

template <int D>
struct BwdCfg {
  static constexpr int kChunks = D / 64;
  static constexpr int kOuterChunk = kBO * 128;
  static constexpr int kInnerChunk = kBI * 128;
  static constexpr int kOuterBytes = kBO * D * 2;
  static constexpr int kInnerBytes = kBI * D * 2;
  static constexpr int kStatBytes = kBI * 4;
  static constexpr int kStageBytes = ((2 * kInnerBytes + 2 * kStatBytes) + 1023) / 1024 * 1024;
  static constexpr int kBudget = 225 * 1024;
  static constexpr int kStagesFit = (kBudget - 2 * kOuterBytes - 1024) / kStageBytes;
  static constexpr int kStages = kStagesFit > 4 ? 4 : kStagesFit;
  static_assert(kStages >= 2, "need a double-buffered inner ring");
  static constexpr int kOffOuterA = 0;              // K (dK/dV) or Q (dQ)
  static constexpr int kOffOuterB = kOuterBytes;    // V (dK/dV) or dO (dQ)
  static constexpr int kOffStages = 2 * kOuterBytes;
  // inside a stage: inner A (Q | K), inner B (dO | V), lse slice, delta slice
  static constexpr int kStInA = 0;
  static constexpr int kStInB = kInnerBytes;
  static constexpr int kStLse = 2 * kInnerBytes;
  static constexpr int kStDelta = 2 * kInnerBytes + kStatBytes;
  static constexpr int kOffBar = kOffStages + kStages * kStageBytes;
  static constexpr int kSmemBytes = kOffBar + 256 + 1024;
};

enum : int {
  BB_OUTER = 0,
  BB_SFULL = 1,   // + stage (4)
  BB_SEMPTY = 5,  // + stage (4)
  BB_MFULL = 9,   // + buffer (2): S / dP of a step are in TMEM
  BB_PFULL = 11,  // + buffer (2): P / dS of a step are in TMEM
  BB_ACC = 13,
  BB_DRAIN = 14,
  BB_COUNT = 15
};

struct BwdSmem {
  uint32_t base;
  uint8_t* ptr;
  uint64_t* bars;
  volatile uint32_t* tmem_slot;
  volatile int* abort_slot;
};

template <class C>
__device__ __forceinline__ BwdSmem bwd_smem() {
  extern __shared__ uint8_t smem_raw[];
  BwdSmem s;
  const uint32_t raw = smem_u32(smem_raw);
  s.base = (raw + 1023u) & ~1023u;
  s.ptr = smem_raw + (s.base - raw);
  s.bars = reinterpret_cast<uint64_t*>(s.ptr + C::kOffBar);
  s.tmem_slot = reinterpret_cast<volatile uint32_t*>(s.ptr + C::kOffBar + 8 * BB_COUNT);
  s.abort_slot = reinterpret_cast<volatile int*>(s.ptr + C::kOffBar + 8 * BB_COUNT + 4);
  return s;
}

// Common prologue: abort check, barrier init, TMEM allocation.  Returns false if this CTA
// must stop because an earlier CTA already failed (uniform across the CTA).
template <class C>
__device__ __forceinline__ bool bwd_setup(const BwdSmem& sm, const BwdParams& p, uint32_t& tmem) {
  if (threadIdx.x == 0) *sm.abort_slot = ld_status(p.status);
  __syncthreads();
  if (*sm.abort_slot != 0) return false;
  if (threadIdx.x == 0) {
    mbar_init(smem_u32(sm.bars + BB_OUTER), 1);
    for (int s = 0; s < 4; ++s) {
      mbar_init(smem_u32(sm.bars + BB_SFULL + s), 1);
      mbar_init(smem_u32(sm.bars + BB_SEMPTY + s), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(smem_u32(sm.bars + BB_MFULL + b), 1);
      mbar_init(smem_u32(sm.bars + BB_PFULL + b), 128);
    }
    mbar_init(smem_u32(sm.bars + BB_ACC), 1);
    mbar_init(smem_u32(sm.bars + BB_DRAIN), 1);
    fence_barrier_init();
  }
  if (threadIdx.x / 32 == 0) {
    tmem_alloc(smem_u32(const_cast<uint32_t*>(sm.tmem_slot)), kBwdTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  tmem = *sm.tmem_slot;
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

// Issue an M=128, N=64, K=D product of two K-major SW128 tiles (outer rows x inner rows);
// descriptors are precomputed bases advanced by constant offsets.
template <int D, class C>
__device__ __forceinline__ void umma_outer_inner(uint32_t d_tmem, uint64_t outer_desc,
                                                 uint64_t inner_desc, uint32_t idesc) {
#pragma unroll
  for (int k = 0; k < D / 16; ++k) {
    umma_ss(d_tmem, desc_add(outer_desc, (k / 4) * C::kOuterChunk + (k % 4) * 32),
            desc_add(inner_desc, (k / 4) * C::kInnerChunk + (k % 4) * 32), idesc, k > 0 ? 1u : 0u);
  }
}

// acc[128 x D] (+)= A[128 x 64] (16-bit, in TMEM) * B[64 x D] (inner tile, MN-major SW128).
template <int D, class C>
__device__ __forceinline__ void umma_tmem_inner(uint32_t d_tmem, uint32_t a_tmem, uint64_t inner_desc,
                                                uint32_t idesc, uint32_t accumulate) {
#pragma unroll
  for (int k = 0; k < kBI / 16; ++k)
    umma_ts(d_tmem, a_tmem + k * 8, desc_add(inner_desc, k * 2048), idesc, (accumulate | k) ? 1u : 0u);
}

// ---------------------------------------------------------------------------- dK / dV
template <int D, bool BF16>
__global__ void __launch_bounds__(kBwdThreads, 1)
    bwd_dkdv_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                    const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmdO,
                    const BwdParams p) {
  using C = BwdCfg<D>;
  constexpr int ST = C::kStages;
  constexpr uint32_t IDESC_SD = idesc_f16(BF16, kBO, kBI, false, false);
  constexpr uint32_t IDESC_ACC = idesc_f16(BF16, kBO, D, false, true);
  const BwdSmem sm = bwd_smem<C>();
  auto bar = [&](int i) -> uint32_t { return smem_u32(sm.bars + i); };
  const uint32_t sOA = sm.base + C::kOffOuterA, sOB = sm.base + C::kOffOuterB;
  auto stage = [&](int st) -> uint32_t { return sm.base + C::kOffStages + st * C::kStageBytes; };

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  uint32_t tmem;
  if (!bwd_setup<C>(sm, p, tmem)) return;

  // work item: (b, kv head) major, key tile ascending (tile 0 sees every query: heaviest first)
  const int nkt = (p.S + kBO - 1) / kBO;
  const int bkv = blockIdx.x / nkt;
  const int j = blockIdx.x - bkv * nkt;
  const int b = bkv / p.H_kv, g = bkv - b * p.H_kv;
  const int nqi_total = p.S / kBI;
  const int i_start = (j * kBO) / kBI;
  const int nqi = nqi_total - i_start;
  const int nsteps = p.group * nqi;

  if (warp == kBwdWarpProducer) {
    if (lane == 0) {
      const uint64_t pol_once = policy_evict_first();    // outer tile: read by this CTA only
      const uint64_t pol_shared = policy_evict_last();   // inner tiles: read by many CTAs
      mbar_arrive_expect_tx(bar(BB_OUTER), 2 * C::kOuterBytes);
      for (int c = 0; c < C::kChunks; ++c) {
        tma_load_3d(sOA + c * C::kOuterChunk, &tmK, bar(BB_OUTER), c * 64, j * kBO, bkv, pol_once);
        tma_load_3d(sOB + c * C::kOuterChunk, &tmV, bar(BB_OUTER), c * 64, j * kBO, bkv, pol_once);
      }
      int issued = 0;
      for (int s = 0; s < nsteps; ++s) {
        const int st = s % ST;
        if (!mbar_wait(bar(BB_SEMPTY + st), ((s / ST) & 1) ^ 1, p.status, kDevTimeoutBwd)) break;
        const int hh = s / nqi, i = i_start + (s - hh * nqi);
        const int bh = b * p.H + g * p.group + hh;
        const uint32_t sb = stage(st);
        mbar_arrive_expect_tx(bar(BB_SFULL + st), 2 * C::kInnerBytes + 2 * C::kStatBytes);
        for (int c = 0; c < C::kChunks; ++c) {
          tma_load_3d(sb + C::kStInA + c * C::kInnerChunk, &tmQ, bar(BB_SFULL + st), c * 64, i * kBI, bh, pol_shared);
          tma_load_3d(sb + C::kStInB + c * C::kInnerChunk, &tmdO, bar(BB_SFULL + st), c * 64, i * kBI, bh, pol_shared);
        }
        const size_t row0 = static_cast<size_t>(bh) * p.S + static_cast<size_t>(i) * kBI;
        bulk_load(sb + C::kStLse, p.lse + row0, C::kStatBytes, bar(BB_SFULL + st));
        bulk_load(sb + C::kStDelta, p.delta + row0, C::kStatBytes, bar(BB_SFULL + st));
        ++issued;
      }
      drain_wait(bar(BB_OUTER), 0, p.status);
      for (int s = max(0, issued - ST); s < issued; ++s)
        drain_wait(bar(BB_SFULL + s % ST), (s / ST) & 1, p.status);
    }
    __syncwarp();
  } else if (warp == kBwdWarpMma) {
    if (lane == 0) {
      // descriptors: outer K / V (K-major), inner Q / dO of stage 0 as K-major (S^T, dP^T) and
      // as MN-major B operands (dK, dV); stage st adds st * kStageBytes
      const uint64_t dK_ = sdesc_sw128(sOA, 16, 1024), dV_ = sdesc_sw128(sOB, 16, 1024);
      const uint64_t dQk = sdesc_sw128(stage(0) + C::kStInA, 16, 1024);
      const uint64_t dOk = sdesc_sw128(stage(0) + C::kStInB, 16, 1024);
      const uint64_t dQm = sdesc_sw128(stage(0) + C::kStInA, C::kInnerChunk, 1024);
      const uint64_t dOm = sdesc_sw128(stage(0) + C::kStInB, C::kInnerChunk, 1024);
      bool ok = mbar_wait(bar(BB_OUTER), 0, p.status, kDevTimeoutBwd) &&
                mbar_wait(bar(BB_SFULL + 0), 0, p.status, kDevTimeoutBwd);
      if (ok) {
        tc_fence_after();
        umma_outer_inner<D, C>(tmem + 256, dK_, dQk, IDESC_SD);       // S^T = K Q^T
        umma_outer_inner<D, C>(tmem + 256 + 64, dV_, dOk, IDESC_SD);  // dP^T = V dO^T
        umma_commit(bar(BB_MFULL + 0));
      }
      for (int s = 0; ok && s < nsteps; ++s) {
        const int st = s % ST, bf = s & 1;
        if (s + 1 < nsteps) {
          const int st1 = (s + 1) % ST, bf1 = (s + 1) & 1;
          if (!(ok = mbar_wait(bar(BB_SFULL + st1), ((s + 1) / ST) & 1, p.status, kDevTimeoutBwd))) break;
          tc_fence_after();
          const uint64_t so = static_cast<uint64_t>((st1 * C::kStageBytes) >> 4);
          umma_outer_inner<D, C>(tmem + 256 + 128 * bf1, dK_, dQk + so, IDESC_SD);
          umma_outer_inner<D, C>(tmem + 256 + 128 * bf1 + 64, dV_, dOk + so, IDESC_SD);
          umma_commit(bar(BB_MFULL + bf1));
        }
        if (!(ok = mbar_wait(bar(BB_PFULL + bf), (s >> 1) & 1, p.status, kDevTimeoutBwd))) break;
        tc_fence_after();
        const uint64_t so = static_cast<uint64_t>((st * C::kStageBytes) >> 4);
        const uint32_t acc = s > 0 ? 1u : 0u;
        umma_tmem_inner<D, C>(tmem + 0, tmem + 256 + 128 * bf, dOm + so, IDESC_ACC, acc);         // dV += P^T dO
        umma_tmem_inner<D, C>(tmem + 128, tmem + 256 + 128 * bf + 64, dQm + so, IDESC_ACC, acc);  // dK += dS^T Q
        umma_commit(bar(BB_SEMPTY + st));
      }
      if (ok) umma_commit(bar(BB_ACC));
      umma_commit(bar(BB_DRAIN));
      drain_wait(bar(BB_DRAIN), 0, p.status);
    }
    __syncwarp();
  } else if (warp < 8) {
    const int w = warp / 4;  // compute warpgroup: steps s with s % 2 == w
    const int wq = warp % 4;
    const int row = wq * 32 + lane;
    const int key = j * kBO + row;
    const uint32_t lane_off = static_cast<uint32_t>(wq * 32) << 16;
    const uint32_t tS = tmem + 256 + 128 * w + lane_off;
    const uint32_t tP = tS + 64;
    const float scale = p.scale_log2;
    bool ok = true;
    for (int s = w; s < nsteps; s += 2) {
      if (!(ok = mbar_wait(bar(BB_MFULL + w), (s >> 1) & 1, p.status, kDevTimeoutBwd))) break;
      tc_fence_after();
      const int st = s % ST;
      const int hh = s / nqi, i = i_start + (s - hh * nqi);
      uint32_t sv[2][32], dp[2][32];
      tmem_ld32(tS, sv[0]);
      tmem_ld32(tS + 32, sv[1]);
      tmem_ld32(tP, dp[0]);
      tmem_ld32(tP + 32, dp[1]);
      tmem_ld_wait(sv[0]);
      tmem_ld_wait(sv[1]);
      tmem_ld_wait(dp[0]);
      tmem_ld_wait(dp[1]);
      const float4* lse4 = reinterpret_cast<const float4*>(sm.ptr + C::kOffStages + st * C::kStageBytes + C::kStLse);
      const float4* del4 = reinterpret_cast<const float4*>(sm.ptr + C::kOffStages + st * C::kStageBytes + C::kStDelta);
      const int q0 = i * kBI;
      const bool need_mask = q0 < j * kBO + kBO;
#pragma unroll
      for (int h2 = 0; h2 < 2; ++h2) {
        uint32_t pk[16], dk[16];
#pragma unroll
        for (int c4 = 0; c4 < 8; ++c4) {
          const float4 l4 = lse4[h2 * 8 + c4];
          const float4 d4 = del4[h2 * 8 + c4];
          const float lv[4] = {l4.x, l4.y, l4.z, l4.w};
          const float dv[4] = {d4.x, d4.y, d4.z, d4.w};
          float pr[4], ds[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int c = c4 * 4 + e;
            float pv = ex2_approx(fmaf(__uint_as_float(sv[h2][c]), scale, -lv[e]));
            if (need_mask && key > q0 + h2 * 32 + c) pv = 0.f;
            pr[e] = pv;
            ds[e] = pv * (__uint_as_float(dp[h2][c]) - dv[e]);
          }
          pk[2 * c4] = pack2<BF16>(pr[0], pr[1]);
          pk[2 * c4 + 1] = pack2<BF16>(pr[2], pr[3]);
          dk[2 * c4] = pack2<BF16>(ds[0], ds[1]);
          dk[2 * c4 + 1] = pack2<BF16>(ds[2], ds[3]);
        }
        tmem_st16(tS + h2 * 16, pk);
        tmem_st16(tP + h2 * 16, dk);
      }
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(bar(BB_PFULL + w));
    }
    if (ok) ok = mbar_wait(bar(BB_ACC), 0, p.status, kDevTimeoutBwd);
    if (ok) {
      tc_fence_after();
      // warpgroup 0 writes dV rows, warpgroup 1 writes dK rows (scaled by 1/sqrt(D))
      void* out = (w == 0) ? p.dv : p.dk;
      const float osc = (w == 0) ? 1.0f : p.sm_scale;
      const uint32_t tacc = tmem + (w == 0 ? 0 : 128) + lane_off;
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
  bwd_teardown(tmem);
}

// ---------------------------------------------------------------------------- dQ
template <int D, bool BF16>
__global__ void __launch_bounds__(kBwdThreads, 1)
    bwd_dq_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                  const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmdO,
                  const BwdParams p) {
  using C = BwdCfg<D>;
  constexpr int ST = C::kStages;
  constexpr uint32_t IDESC_SD = idesc_f16(BF16, kBO, kBI, false, false);
  constexpr uint32_t IDESC_ACC = idesc_f16(BF16, kBO, D, false, true);
  const BwdSmem sm = bwd_smem<C>();
  auto bar = [&](int i) -> uint32_t { return smem_u32(sm.bars + i); };
  const uint32_t sOA = sm.base + C::kOffOuterA, sOB = sm.base + C::kOffOuterB;
  auto stage = [&](int st) -> uint32_t { return sm.base + C::kOffStages + st * C::kStageBytes; };

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  uint32_t tmem;
  if (!bwd_setup<C>(sm, p, tmem)) return;

  // work item: head major, query tile descending (the longest rows first)
  const int nqt = (p.S + kBO - 1) / kBO;
  const int bh = blockIdx.x / nqt;
  const int i = nqt - 1 - (blockIdx.x - bh * nqt);
  const int b = bh / p.H, h = bh - b * p.H;
  const int bkv = b * p.H_kv + h / p.group;
  const int last_row = min(i * kBO + kBO - 1, p.S - 1);
  const int nsteps = last_row / kBI + 1;

  if (warp == kBwdWarpProducer) {
    if (lane == 0) {
      const uint64_t pol_once = policy_evict_first();    // outer tile: read by this CTA only
      const uint64_t pol_shared = policy_evict_last();   // inner tiles: read by many CTAs
      mbar_arrive_expect_tx(bar(BB_OUTER), 2 * C::kOuterBytes);
      for (int c = 0; c < C::kChunks; ++c) {
        tma_load_3d(sOA + c * C::kOuterChunk, &tmQ, bar(BB_OUTER), c * 64, i * kBO, bh, pol_once);
        tma_load_3d(sOB + c * C::kOuterChunk, &tmdO, bar(BB_OUTER), c * 64, i * kBO, bh, pol_once);
      }
      int issued = 0;
      for (int s = 0; s < nsteps; ++s) {
        const int st = s % ST;
        if (!mbar_wait(bar(BB_SEMPTY + st), ((s / ST) & 1) ^ 1, p.status, kDevTimeoutBwd)) break;
        const uint32_t sb = stage(st);
        mbar_arrive_expect_tx(bar(BB_SFULL + st), 2 * C::kInnerBytes);
        for (int c = 0; c < C::kChunks; ++c) {
          tma_load_3d(sb + C::kStInA + c * C::kInnerChunk, &tmK, bar(BB_SFULL + st), c * 64, s * kBI, bkv, pol_shared);
          tma_load_3d(sb + C::kStInB + c * C::kInnerChunk, &tmV, bar(BB_SFULL + st), c * 64, s * kBI, bkv, pol_shared);
        }
        ++issued;
      }
      drain_wait(bar(BB_OUTER), 0, p.status);
      for (int s = max(0, issued - ST); s < issued; ++s)
        drain_wait(bar(BB_SFULL + s % ST), (s / ST) & 1, p.status);
    }
    __syncwarp();
  } else if (warp == kBwdWarpMma) {
    if (lane == 0) {
      const uint64_t dQ_ = sdesc_sw128(sOA, 16, 1024), dO_ = sdesc_sw128(sOB, 16, 1024);
      const uint64_t dKk = sdesc_sw128(stage(0) + C::kStInA, 16, 1024);
      const uint64_t dVk = sdesc_sw128(stage(0) + C::kStInB, 16, 1024);
      const uint64_t dKm = sdesc_sw128(stage(0) + C::kStInA, C::kInnerChunk, 1024);
      bool ok = mbar_wait(bar(BB_OUTER), 0, p.status, kDevTimeoutBwd) &&
                mbar_wait(bar(BB_SFULL + 0), 0, p.status, kDevTimeoutBwd);
      if (ok) {
        tc_fence_after();
        umma_outer_inner<D, C>(tmem + 256, dQ_, dKk, IDESC_SD);       // S = Q K^T
        umma_outer_inner<D, C>(tmem + 256 + 64, dO_, dVk, IDESC_SD);  // dP = dO V^T
        umma_commit(bar(BB_MFULL + 0));
      }
      for (int s = 0; ok && s < nsteps; ++s) {
        const int st = s % ST, bf = s & 1;
        if (s + 1 < nsteps) {
          const int st1 = (s + 1) % ST, bf1 = (s + 1) & 1;
          if (!(ok = mbar_wait(bar(BB_SFULL + st1), ((s + 1) / ST) & 1, p.status, kDevTimeoutBwd))) break;
          tc_fence_after();
          const uint64_t so = static_cast<uint64_t>((st1 * C::kStageBytes) >> 4);
          umma_outer_inner<D, C>(tmem + 256 + 128 * bf1, dQ_, dKk + so, IDESC_SD);
          umma_outer_inner<D, C>(tmem + 256 + 128 * bf1 + 64, dO_, dVk + so, IDESC_SD);
          umma_commit(bar(BB_MFULL + bf1));
        }
        if (!(ok = mbar_wait(bar(BB_PFULL + bf), (s >> 1) & 1, p.status, kDevTimeoutBwd))) break;
        tc_fence_after();
        const uint64_t so = static_cast<uint64_t>((st * C::kStageBytes) >> 4);
        umma_tmem_inner<D, C>(tmem + 0, tmem + 256 + 128 * bf + 64, dKm + so, IDESC_ACC, s > 0 ? 1u : 0u);  // dQ += dS K
        umma_commit(bar(BB_SEMPTY + st));
      }
      if (ok) umma_commit(bar(BB_ACC));
      umma_commit(bar(BB_DRAIN));
      drain_wait(bar(BB_DRAIN), 0, p.status);
    }
    __syncwarp();
  } else if (warp < 8) {
    const int w = warp / 4;
    const int wq = warp % 4;
    const int row = wq * 32 + lane;
    const int qrow = i * kBO + row;
    const uint32_t lane_off = static_cast<uint32_t>(wq * 32) << 16;
    const uint32_t tS = tmem + 256 + 128 * w + lane_off;
    const uint32_t tP = tS + 64;
    const float scale = p.scale_log2;
    const size_t ridx = static_cast<size_t>(bh) * p.S + qrow;
    const float lse_r = qrow < p.S ? p.lse[ridx] : 0.f;
    const float del_r = qrow < p.S ? p.delta[ridx] : 0.f;
    bool ok = true;
    for (int s = w; s < nsteps; s += 2) {
      if (!(ok = mbar_wait(bar(BB_MFULL + w), (s >> 1) & 1, p.status, kDevTimeoutBwd))) break;
      tc_fence_after();
      uint32_t sv[2][32], dp[2][32];
      tmem_ld32(tS, sv[0]);
      tmem_ld32(tS + 32, sv[1]);
      tmem_ld32(tP, dp[0]);
      tmem_ld32(tP + 32, dp[1]);
      tmem_ld_wait(sv[0]);
      tmem_ld_wait(sv[1]);
      tmem_ld_wait(dp[0]);
      tmem_ld_wait(dp[1]);
      const int k0 = s * kBI;
      const bool need_mask = k0 + kBI - 1 > i * kBO;
#pragma unroll
      for (int h2 = 0; h2 < 2; ++h2) {
        uint32_t dk[16];
#pragma unroll
        for (int c2 = 0; c2 < 16; ++c2) {
          float ds2[2];
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int c = 2 * c2 + e;
            float pv = ex2_approx(fmaf(__uint_as_float(sv[h2][c]), scale, -lse_r));
            if (need_mask && k0 + h2 * 32 + c > qrow) pv = 0.f;
            ds2[e] = pv * (__uint_as_float(dp[h2][c]) - del_r);
          }
          dk[c2] = pack2<BF16>(ds2[0], ds2[1]);
        }
        tmem_st16(tP + h2 * 16, dk);
      }
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(bar(BB_PFULL + w));
    }
    if (w == 0) {
      if (ok) ok = mbar_wait(bar(BB_ACC), 0, p.status, kDevTimeoutBwd);
      if (ok) {
        tc_fence_after();
        uint8_t* orow = reinterpret_cast<uint8_t*>(p.dq) + ridx * (D * 2);
#pragma unroll 1
        for (int c = 0; c < D / 32; ++c) {
          uint32_t v[32];
          tmem_ld32(tmem + lane_off + c * 32, v);
          tmem_ld_wait(v);
          if (qrow < p.S) store_row_chunk<BF16>(orow + c * 64, v, p.sm_scale);
        }
      }
    }
  }
  bwd_teardown(tmem);
}

template <int D, bool BF16>
cudaError_t launch_dkdv_t(const CUtensorMap& tmQ, const CUtensorMap& tmK, const CUtensorMap& tmV,
                          const CUtensorMap& tmdO, const BwdParams& p, cudaStream_t stream) {
  using C = BwdCfg<D>;
  auto kern = bwd_dkdv_kernel<D, BF16>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmemBytes);
  if (e != cudaSuccess) return e;
  const int nkt = (p.S + kBO - 1) / kBO;
  kern<<<p.B * p.H_kv * nkt, kBwdThreads, C::kSmemBytes, stream>>>(tmQ, tmK, tmV, tmdO, p);
  return cudaGetLastError();
}

template <int D, bool BF16>
cudaError_t launch_dq_t(const CUtensorMap& tmQ, const CUtensorMap& tmK, const CUtensorMap& tmV,
                        const CUtensorMap& tmdO, const BwdParams& p, cudaStream_t stream) {
  using C = BwdCfg<D>;
  auto kern = bwd_dq_kernel<D, BF16>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmemBytes);
  if (e != cudaSuccess) return e;
  const int nqt = (p.S + kBO - 1) / kBO;
  kern<<<p.B * p.H * nqt, kBwdThreads, C::kSmemBytes, stream>>>(tmQ, tmK, tmV, tmdO, p);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_bwd_preprocess(const BwdParams& p, bool bf16, cudaStream_t stream) {
  if (p.D == 64) return bf16 ? launch_pre_t<64, true>(p, stream) : launch_pre_t<64, false>(p, stream);
  if (p.D == 128) return bf16 ? launch_pre_t<128, true>(p, stream) : launch_pre_t<128, false>(p, stream);
  return cudaErrorInvalidValue;
}

cudaError_t launch_bwd_dkdv(const CUtensorMap& tmQ, const CUtensorMap& tmK, const CUtensorMap& tmV,
                            const CUtensorMap& tmdO, const BwdParams& p, bool bf16, cudaStream_t stream) {
  if (p.D == 64) return bf16 ? launch_dkdv_t<64, true>(tmQ, tmK, tmV, tmdO, p, stream)
                             : launch_dkdv_t<64, false>(tmQ, tmK, tmV, tmdO, p, stream);
  if (p.D == 128) return bf16 ? launch_dkdv_t<128, true>(tmQ, tmK, tmV, tmdO, p, stream)
                              : launch_dkdv_t<128, false>(tmQ, tmK, tmV, tmdO, p, stream);
  return cudaErrorInvalidValue;
}

cudaError_t launch_bwd_dq(const CUtensorMap& tmQ, const CUtensorMap& tmK, const CUtensorMap& tmV,
                          const CUtensorMap& tmdO, const BwdParams& p, bool bf16, cudaStream_t stream) {
  if (p.D == 64) return bf16 ? launch_dq_t<64, true>(tmQ, tmK, tmV, tmdO, p, stream)
                             : launch_dq_t<64, false>(tmQ, tmK, tmV, tmdO, p, stream);
  if (p.D == 128) return bf16 ? launch_dq_t<128, true>(tmQ, tmK, tmV, tmdO, p, stream)
                              : launch_dq_t<128, false>(tmQ, tmK, tmV, tmdO, p, stream);
  return cudaErrorInvalidValue;
}

}  // namespace fa
