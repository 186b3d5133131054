// Unfused causal attention on sm_100a: the reference's three-kernel baseline
// (attention/fused/unfused.py:27-116 and attention/gqa/unfused_gqa.py, MHA and GQA), with the
// score and probability matrices materialised in global memory:
//
//   1. unf_scores_kernel:  S = causal_mask(Q K^T / sqrt(D)), fp32 [B, H, N, N]
//   2. unf_softmax_kernel: P = row_softmax(S), 16-bit [B, H, N, N] (pass 1: row max and sum,
//                          pass 2: normalise and store)
//   3. unf_pv_kernel:      O = P V
//
// Only 128 x 128 tiles on or below the causal diagonal are computed, read or written (entries of
// a diagonal tile above the diagonal hold -inf in S and 0 in P); tiles strictly above it are never
// touched, as in the reference.  GQA: query head h reads K/V head h / (H / H_kv).
//
// The two GEMM kernels are TMA + tcgen05 kernels (one 128-row query tile per CTA): warp 0 loads
// tiles into a 3-stage shared-memory ring, warp 1 issues the UMMAs, warps 4-7 move the TMEM
// accumulator to global memory (one thread per row).  The scores kernel double-buffers S in TMEM
// so the Q K^T of tile j+1 runs while tile j is stored.  The softmax kernel is HBM-bound: one warp
// per row, 16-byte loads.  Waits are bounded like the fused kernels' (status word).
#include "fa_internal.h"
#include "fa_sm100.cuh"

namespace fa {
namespace {

constexpr int kUT = 128;       // tile rows / keys
constexpr int kUThreads = 256;  // warp 0 TMA, warp 1 UMMA, warps 4-7 epilogue
constexpr int kUStages = 3;
constexpr int kUEpiWarp0 = 4;

template <int D>
struct UnfTile {
  static constexpr int kSwBytes = D >= 64 ? 128 : 64;  // swizzle span of a D-column row chunk
  static constexpr int kChunkCols = kSwBytes / 2;
  static constexpr int kChunks = D / kChunkCols;
  static constexpr uint32_t kLayout = D >= 64 ? kLayoutSw128 : kLayoutSw64;
  static constexpr int kSbo = 8 * kSwBytes;
  static constexpr int kKSteps = kSwBytes / 32;        // 16-element K steps per chunk
  static constexpr int kChunkBytes = kUT * kSwBytes;   // one chunk of 128 rows
  static constexpr int kTile = kUT * D * 2;            // a 128-row tile of Q, K or V
};

struct UnfSmem {
  uint32_t base;
  uint32_t bar0;
  volatile uint32_t* tmem_slot;
  volatile int* abort_slot;
};

// 1 KiB-aligned working area, barriers and slots in its last 256 bytes.
template <int kUsed>
__device__ __forceinline__ UnfSmem unf_smem() {
  extern __shared__ uint8_t smem_raw[];
  UnfSmem s;
  const uint32_t raw = smem_u32(smem_raw);
  s.base = (raw + 1023u) & ~1023u;
  uint8_t* ptr = smem_raw + (s.base - raw);
  s.bar0 = s.base + kUsed - 256;
  s.tmem_slot = reinterpret_cast<volatile uint32_t*>(ptr + kUsed - 256 + 8 * 28);
  s.abort_slot = reinterpret_cast<volatile int*>(ptr + kUsed - 256 + 8 * 28 + 4);
  return s;
}

enum : int { U_FULL = 0 /* + stage (3) */, U_EMPTY = 3 /* + stage */, U_Q = 6, U_SFULL = 7 /* + 2 */,
             U_SFREE = 9 /* + 2 */, U_OFULL = 11, U_DRAIN = 12, U_NBARS = 13 };

// Shared prologue: abort check, barrier init, TMEM allocation.  Returns false (uniformly) when the
// status word already holds an error.
__device__ __forceinline__ bool unf_setup(const UnfSmem& sm, const int* status, uint32_t tmem_cols,
                                          uint32_t sfree_count) {
  if (threadIdx.x == 0) {
    *sm.abort_slot = ld_status(status);
    for (int i = 0; i < U_NBARS; ++i)
      mbar_init(sm.bar0 + 8u * i, (i == U_SFREE || i == U_SFREE + 1) ? sfree_count : 1u);
    fence_barrier_init();
  }
  __syncthreads();
  if (*sm.abort_slot != 0) return false;
  if (threadIdx.x / 32 == 0) {
    tmem_alloc(smem_u32(const_cast<uint32_t*>(sm.tmem_slot)), tmem_cols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  return true;
}

__device__ __forceinline__ void unf_teardown(uint32_t tmem, uint32_t cols) {
  tc_fence_before();
  __syncthreads();
  if (threadIdx.x / 32 == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, cols);
  }
}

// ---------------------------------------------------------------------------- 1. scores
template <int D, bool BF16>
__global__ void __launch_bounds__(kUThreads, 1)
    unf_scores_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                      const UnfParams p) {
  using T = UnfTile<D>;
  constexpr int kUsed = (1 + kUStages) * T::kTile + 256;
  const UnfSmem sm = unf_smem<kUsed>();
#define BAR(i) (sm.bar0 + 8u * static_cast<uint32_t>(i))
  const uint32_t sQ = sm.base, sK = sm.base + T::kTile;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int i = blockIdx.x, bh = blockIdx.y;
  const int b = bh / p.H, h = bh - b * p.H;
  const int bh_kv = b * p.H_kv + h / p.group;
  const int ntiles = i + 1;  // key tiles 0..i (128-key tiles, causal)
  if (!unf_setup(sm, p.status, 256, 128)) return;
  const uint32_t tmem = *sm.tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      const uint64_t pol = policy_evict_last();
      mbar_arrive_expect_tx(BAR(U_Q), T::kTile);
      for (int c = 0; c < T::kChunks; ++c)
        tma_load_3d(sQ + c * T::kChunkBytes, &tmQ, BAR(U_Q), c * T::kChunkCols, i * kUT, bh, pol);
      int issued = 0;
      for (int j = 0; j < ntiles; ++j) {
        const int st = j % kUStages;
        if (!mbar_wait(BAR(U_EMPTY + st), ((j / kUStages) & 1) ^ 1, p.status, kDevTimeoutKVEmpty)) break;
        mbar_arrive_expect_tx(BAR(U_FULL + st), T::kTile);
        for (int c = 0; c < T::kChunks; ++c)
          tma_load_3d(sK + st * T::kTile + c * T::kChunkBytes, &tmK, BAR(U_FULL + st), c * T::kChunkCols,
                      j * kUT, bh_kv, pol);
        ++issued;
      }
      drain_wait(BAR(U_Q), 0, p.status);
      for (int j = max(0, issued - kUStages); j < issued; ++j)
        drain_wait(BAR(U_FULL + j % kUStages), (j / kUStages) & 1, p.status);
    }
    __syncwarp();
  } else if (warp == 1) {
    constexpr uint32_t IDESC = idesc_f16(BF16, kUT, kUT, false, false);
    const uint64_t dq = sdesc_sw(sQ, 16, T::kSbo, T::kLayout);
    const uint64_t dk0 = sdesc_sw(sK, 16, T::kSbo, T::kLayout);
    bool ok = warp_all(mbar_wait(BAR(U_Q), 0, p.status, kDevTimeoutQ));
    for (int j = 0; ok && j < ntiles; ++j) {
      const int st = j % kUStages, sb = j & 1;
      if (!(ok = warp_all(mbar_wait(BAR(U_FULL + st), (j / kUStages) & 1, p.status, kDevTimeoutKV)))) break;
      if (!(ok = warp_all(mbar_wait(BAR(U_SFREE + sb), ((j >> 1) & 1) ^ 1, p.status, kDevTimeoutS)))) break;
      tc_fence_after();
      const uint64_t dk = desc_add(dk0, st * T::kTile);
#pragma unroll
      for (int k = 0; k < D / 16; ++k) {
        const uint32_t off = (k / T::kKSteps) * T::kChunkBytes + (k % T::kKSteps) * 32;
        umma_ss_w(tmem + sb * 128, desc_add(dq, off), desc_add(dk, off), IDESC, k > 0 ? 1u : 0u);
      }
      umma_commit_w(BAR(U_SFULL + sb));
      umma_commit_w(BAR(U_EMPTY + st));
    }
    umma_commit_w(BAR(U_DRAIN));
    drain_wait(BAR(U_DRAIN), 0, p.status);
    __syncwarp();
  } else if (warp >= kUEpiWarp0) {
    const int wq = warp % 4;
    const int row = i * kUT + wq * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>(wq * 32) << 16;
    float* srow = p.s + (static_cast<size_t>(bh) * p.N + row) * p.N;
    for (int j = 0; j < ntiles; ++j) {
      const int sb = j & 1;
      if (!warp_all(mbar_wait(BAR(U_SFULL + sb), (j >> 1) & 1, p.status, kDevTimeoutS))) break;
      tc_fence_after();
      uint32_t r[4][32];
#pragma unroll
      for (int c = 0; c < 4; ++c) tmem_ld32(tmem + lane_off + sb * 128 + c * 32, r[c]);
#pragma unroll
      for (int c = 0; c < 4; ++c) tmem_ld_wait(r[c]);
      tc_fence_before();
      mbar_arrive(BAR(U_SFREE + sb));
      if (row < p.N) {
        const int col0 = j * kUT;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
#pragma unroll
          for (int v = 0; v < 8; ++v) {
            float4 f;
            float* e = &f.x;
#pragma unroll
            for (int u = 0; u < 4; ++u) {
              const int col = col0 + c * 32 + v * 4 + u;
              e[u] = col > row ? -INFINITY : __uint_as_float(r[c][v * 4 + u]) * p.sm_scale;
            }
            const int col = col0 + c * 32 + v * 4;
            if (col < p.N) *reinterpret_cast<float4*>(srow + col) = f;
          }
        }
      }
    }
  }
#undef BAR
  unf_teardown(tmem, 256);
}

// ---------------------------------------------------------------------------- 2. softmax
// One warp per row r of tile i = r / 128: the row's 128 (i + 1) leading entries (capped at N) are
// read twice (max / sum, then normalise) and written as 16-bit P.  Lane l handles 4 consecutive
// entries per 128-entry step.
template <bool BF16>
__global__ void __launch_bounds__(256) unf_softmax_kernel(const UnfParams p, long long rows) {
  const long long gw = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) / 32;
  const int lane = threadIdx.x % 32;
  if (gw >= rows) return;
  const int r = static_cast<int>(gw % p.N);
  const int ncols = min(p.N, (r / kUT + 1) * kUT);
  const float* srow = p.s + gw * p.N;
  constexpr float kLog2e = 1.4426950408889634f;
  float m = -INFINITY, l = 0.f;
  for (int c = lane * 4; c < ncols; c += 128) {
    const float4 f = *reinterpret_cast<const float4*>(srow + c);
    const float mx = fmaxf(fmaxf(f.x, f.y), fmaxf(f.z, f.w));
    const float m_new = fmaxf(m, mx);
    if (m_new > -INFINITY) {
      const float base = m_new * kLog2e;
      l = l * ex2_approx(m * kLog2e - base) + ex2_approx(f.x * kLog2e - base) + ex2_approx(f.y * kLog2e - base) +
          ex2_approx(f.z * kLog2e - base) + ex2_approx(f.w * kLog2e - base);
      m = m_new;
    }
  }
  // combine the lanes' (max, sum) pairs
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    const float mo = __shfl_xor_sync(0xffffffffu, m, off);
    const float lo = __shfl_xor_sync(0xffffffffu, l, off);
    const float mn = fmaxf(m, mo);
    if (mn > -INFINITY) {
      l = l * ex2_approx((m - mn) * kLog2e) + lo * ex2_approx((mo - mn) * kLog2e);
      m = mn;
    }
  }
  const float inv_l = 1.0f / l;
  const float base = m * kLog2e;
  uint8_t* prow = reinterpret_cast<uint8_t*>(p.p) + gw * p.N * 2;
  for (int c = lane * 4; c < ncols; c += 128) {
    const float4 f = *reinterpret_cast<const float4*>(srow + c);
    uint2 out;
    out.x = pack2<BF16>(ex2_approx(f.x * kLog2e - base) * inv_l, ex2_approx(f.y * kLog2e - base) * inv_l);
    out.y = pack2<BF16>(ex2_approx(f.z * kLog2e - base) * inv_l, ex2_approx(f.w * kLog2e - base) * inv_l);
    *reinterpret_cast<uint2*>(prow + c * 2) = out;
  }
}

// ---------------------------------------------------------------------------- 3. P V
template <int D, bool BF16>
__global__ void __launch_bounds__(kUThreads, 1)
    unf_pv_kernel(const __grid_constant__ CUtensorMap tmP, const __grid_constant__ CUtensorMap tmV,
                  const UnfParams p) {
  using T = UnfTile<D>;
  constexpr int kPTile = kUT * kUT * 2;  // 128 x 128 16-bit P tile: two 64-column SW128 chunks
  constexpr int kStage = kPTile + T::kTile;
  constexpr int kUsed = kUStages * kStage + 256;
  const UnfSmem sm = unf_smem<kUsed>();
#define BAR(i) (sm.bar0 + 8u * static_cast<uint32_t>(i))
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int i = blockIdx.x, bh = blockIdx.y;
  const int b = bh / p.H, h = bh - b * p.H;
  const int bh_kv = b * p.H_kv + h / p.group;
  const int ntiles = i + 1;
  constexpr uint32_t kOCols = D < 32 ? 32 : D;
  if (!unf_setup(sm, p.status, kOCols, 1)) return;
  const uint32_t tmem = *sm.tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      const uint64_t pol = policy_evict_first();
      const uint64_t pol_v = policy_evict_last();
      int issued = 0;
      for (int j = 0; j < ntiles; ++j) {
        const int st = j % kUStages;
        if (!mbar_wait(BAR(U_EMPTY + st), ((j / kUStages) & 1) ^ 1, p.status, kDevTimeoutKVEmpty)) break;
        const uint32_t dst = sm.base + st * kStage;
        mbar_arrive_expect_tx(BAR(U_FULL + st), kStage);
        for (int c = 0; c < 2; ++c)
          tma_load_3d(dst + c * (kUT * 128), &tmP, BAR(U_FULL + st), j * kUT + c * 64, i * kUT, bh, pol);
        for (int c = 0; c < T::kChunks; ++c)
          tma_load_3d(dst + kPTile + c * T::kChunkBytes, &tmV, BAR(U_FULL + st), c * T::kChunkCols, j * kUT,
                      bh_kv, pol_v);
        ++issued;
      }
      for (int j = max(0, issued - kUStages); j < issued; ++j)
        drain_wait(BAR(U_FULL + j % kUStages), (j / kUStages) & 1, p.status);
    }
    __syncwarp();
  } else if (warp == 1) {
    constexpr uint32_t IDESC = idesc_f16(BF16, kUT, D, false, true);  // P K-major, V MN-major
    bool ok = true;
    for (int j = 0; ok && j < ntiles; ++j) {
      const int st = j % kUStages;
      if (!(ok = warp_all(mbar_wait(BAR(U_FULL + st), (j / kUStages) & 1, p.status, kDevTimeoutKV)))) break;
      tc_fence_after();
      const uint32_t base = sm.base + st * kStage;
      const uint64_t dp = sdesc_sw(base, 16, 1024, kLayoutSw128);
      const uint64_t dv = sdesc_sw(base + kPTile, T::kChunkBytes, T::kSbo, T::kLayout);
#pragma unroll
      for (int k = 0; k < kUT / 16; ++k)
        umma_ss_w(tmem, desc_add(dp, (k / 4) * (kUT * 128) + (k % 4) * 32), desc_add(dv, k * 16 * T::kSwBytes),
                  IDESC, (j | k) ? 1u : 0u);
      umma_commit_w(BAR(U_EMPTY + st));
    }
    if (ok) umma_commit_w(BAR(U_OFULL));
    umma_commit_w(BAR(U_DRAIN));
    drain_wait(BAR(U_DRAIN), 0, p.status);
    __syncwarp();
  } else if (warp >= kUEpiWarp0) {
    const int wq = warp % 4;
    const int row = i * kUT + wq * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>(wq * 32) << 16;
    if (warp_all(mbar_wait(BAR(U_OFULL), 0, p.status, kDevTimeoutO))) {
      tc_fence_after();
      uint8_t* orow = reinterpret_cast<uint8_t*>(p.o) + (static_cast<size_t>(bh) * p.N + row) * (D * 2);
#pragma unroll 1
      for (int c = 0; c < D / 32; ++c) {
        uint32_t v[32];
        tmem_ld32(tmem + lane_off + c * 32, v);
        tmem_ld_wait(v);
        uint32_t pk[16];
#pragma unroll
        for (int e = 0; e < 16; ++e) pk[e] = pack2<BF16>(__uint_as_float(v[2 * e]), __uint_as_float(v[2 * e + 1]));
        if (row < p.N) {
          uint4* dst = reinterpret_cast<uint4*>(orow + c * 64);
#pragma unroll
          for (int q = 0; q < 4; ++q) dst[q] = make_uint4(pk[4 * q], pk[4 * q + 1], pk[4 * q + 2], pk[4 * q + 3]);
        }
      }
    }
  }
#undef BAR
  unf_teardown(tmem, kOCols);
}

template <typename Kernel>
cudaError_t launch_tiles(Kernel kern, int smem, std::atomic<bool> (&done)[64], dim3 grid, cudaStream_t stream,
                         const CUtensorMap& a, const CUtensorMap& b, const UnfParams& p) {
  cudaError_t e = opt_in_smem(kern, smem, done);
  if (e != cudaSuccess) return e;
  kern<<<grid, kUThreads, smem, stream>>>(a, b, p);
  return cudaGetLastError();
}

template <int D, bool BF16>
cudaError_t launch_unfused_t(const CUtensorMap& tmQ, const CUtensorMap& tmK, const CUtensorMap& tmP,
                             const CUtensorMap& tmV, const UnfParams& p, cudaStream_t stream) {
  using T = UnfTile<D>;
  const dim3 grid((p.N + kUT - 1) / kUT, p.B * p.H);
  static std::atomic<bool> done_s[64], done_pv[64];
  cudaError_t e = launch_tiles(unf_scores_kernel<D, BF16>, (1 + kUStages) * T::kTile + 256 + 1024, done_s,
                               grid, stream, tmQ, tmK, p);
  if (e != cudaSuccess) return e;
  const long long rows = static_cast<long long>(p.B) * p.H * p.N;
  unf_softmax_kernel<BF16><<<static_cast<unsigned>((rows * 32 + 255) / 256), 256, 0, stream>>>(p, rows);
  if ((e = cudaGetLastError()) != cudaSuccess) return e;
  return launch_tiles(unf_pv_kernel<D, BF16>, kUStages * (kUT * kUT * 2 + T::kTile) + 256 + 1024, done_pv,
                      grid, stream, tmP, tmV, p);
}

}  // namespace

cudaError_t launch_unfused(const CUtensorMap& tmQ, const CUtensorMap& tmK, const CUtensorMap& tmP,
                           const CUtensorMap& tmV, const UnfParams& p, int D, bool bf16, cudaStream_t stream) {
#define FA_UNF_CASE(DD, BB) \
  if (D == DD && bf16 == BB) return launch_unfused_t<DD, BB>(tmQ, tmK, tmP, tmV, p, stream);
  FA_UNF_CASE(32, false)
  FA_UNF_CASE(64, false)
  FA_UNF_CASE(128, false)
  FA_UNF_CASE(32, true)
  FA_UNF_CASE(64, true)
  FA_UNF_CASE(128, true)
#undef FA_UNF_CASE
  return cudaErrorInvalidValue;
}

}  // namespace fa
