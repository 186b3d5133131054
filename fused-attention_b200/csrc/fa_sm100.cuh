// Device-side building blocks for the sm_100a attention kernels.
//
// Everything here is a thin inline-PTX wrapper around one Blackwell feature:
//   * mbarriers with BOUNDED waits (every wait gives up after FA_WAIT_TIMEOUT_NS and
//     records an error code in a device status word instead of hanging the GPU),
//   * TMA tiled loads (cp.async.bulk.tensor, no multicast anywhere in this library),
//   * tcgen05: TMEM alloc/dealloc, UMMA issue (A from SMEM or TMEM), commit, TMEM ld/st.
//
// Descriptor bit layouts follow the public PTX ISA "tcgen05 matrix descriptors" and
// "instruction descriptor" tables (the same fields CUTLASS names in
// cute/arch/mma_sm100_desc.hpp: SmemDescriptor / InstrDescriptor).
#pragma once

#include <cstdint>
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#ifndef FA_WAIT_TIMEOUT_NS
#define FA_WAIT_TIMEOUT_NS 2000000000ull  // 2 s: far above any legitimate pipeline wait
#endif
// Limit of the teardown waits for a CTA's own copies and UMMAs in flight (they always complete;
// this stays long even in the failure-detection test build, whose pipeline limit is short).
#ifndef FA_DRAIN_TIMEOUT_NS
#define FA_DRAIN_TIMEOUT_NS 2000000000ull
#endif

// Failure-detection test build only (the library built with -DFA_TEST_STALL_STEP=n, never the
// product library): at pipeline step n the UMMA issuer of every kernel waits on an mbarrier that
// nothing arrives at, so its bounded wait runs out and the kernel's abort path runs.
#ifdef FA_TEST_STALL_STEP
#define FA_STALL_HERE(step, bar, status, ok)                                              \
  if ((step) == FA_TEST_STALL_STEP) {                                                    \
    if (!((ok) = warp_all(mbar_wait((bar), 0, (status), kDevTestStall)))) break;         \
  }
#else
#define FA_STALL_HERE(step, bar, status, ok)
#endif

namespace fa {

// ---------------------------------------------------------------- status word codes
// The status word is int32[4] in device memory: [0] = first error code (0 = ok),
// [1] = blockIdx.x of the CTA that recorded it, [2] = role/detail, [3] = spare.
enum DeviceError : int {
  kDevOk = 0,
  kDevTimeoutQ = 101,       // waiting for the Q tile TMA
  kDevTimeoutKV = 102,      // MMA warp waiting for a K/V stage
  kDevTimeoutKVEmpty = 103, // producer waiting for a free K/V stage
  kDevTimeoutS = 104,       // softmax waiting for S = Q K^T
  kDevTimeoutP = 105,       // MMA warp waiting for P
  kDevTimeoutO = 106,       // epilogue waiting for the last P V
  kDevTimeoutDrain = 107,   // teardown waiting for in-flight copies / MMAs
  kDevTimeoutBwd = 108,     // backward pipeline wait
  kDevSmemLayout = 109,     // dynamic shared memory start leaves too little alignment slack
  kDevTestStall = 110,      // failure-detection test build: the injected wait ran out
  kDevAborted = 199,        // another CTA already failed; this one stopped early
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ int ld_status(const int* status) {
  int v;
  asm volatile("ld.volatile.global.s32 %0, [%1];" : "=r"(v) : "l"(status));
  return v;
}

__device__ __forceinline__ void record_error(int* status, int code, int detail) {
  if (atomicCAS(status, 0, code) == 0) {
    status[1] = static_cast<int>(blockIdx.x);
    status[2] = detail;
  }
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_async_shared() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Wait until the phase with the given parity has completed.  Returns false (after recording
// `code` in the status word, unless another CTA already failed) if the wait exceeds
// FA_WAIT_TIMEOUT_NS or if the status word shows that some CTA has already failed.
// The already-complete case is inlined; only a real wait calls the polling loop.  kCopy selects
// one of several identical copies of the loop: a kernel whose warpgroups run under different
// register budgets gives each budget its own copy (one callee cannot serve two budgets).
template <int kCopy = 0>
static __device__ __noinline__ bool mbar_wait_slow(uint32_t bar, uint32_t parity, int* status,
                                                   int code) {
  const uint64_t t0 = global_timer_ns();
  for (uint32_t it = 1;; ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((it & 63u) == 0) {
      if (ld_status(status) != 0) return false;
      if (global_timer_ns() - t0 > FA_WAIT_TIMEOUT_NS) {
        record_error(status, code, static_cast<int>(threadIdx.x));
        return false;
      }
    }
  }
}

template <int kCopy = 0>
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, int* status, int code) {
  if (mbar_try_wait(bar, parity)) return true;
  return mbar_wait_slow<kCopy>(bar, parity, status, code);
}

// Bounded wait used only while tearing down: ignores the abort flag so that copies and MMAs
// already in flight are always waited for (they complete on their own).
__device__ __forceinline__ void drain_wait(uint32_t bar, uint32_t parity, int* status) {
  if (mbar_try_wait(bar, parity)) return;
  const uint64_t t0 = global_timer_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (global_timer_ns() - t0 > FA_DRAIN_TIMEOUT_NS) {
      record_error(status, kDevTimeoutDrain, static_cast<int>(threadIdx.x));
      return;
    }
  }
}

// Warp-uniform result of a bounded wait: lanes of a warp must agree before warp-collective
// tcgen05 instructions, even in the (failure-only) case where their waits ended differently.
__device__ __forceinline__ bool warp_all(bool v) { return __all_sync(0xffffffffu, v) != 0; }

// ---------------------------------------------------------------- TMA
// L2 cache-policy operands for .L2::cache_hint (createpolicy results).
__device__ __forceinline__ uint64_t policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ uint64_t policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}

__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// 3-D tiled load: coordinates (x = head-dim column, y = sequence row, z = batch*head).
// x is always a multiple of the 32- or 64-column swizzle chunk here, i.e. 64- or 128-byte aligned.
__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap* map, uint32_t bar,
                                            int x, int y, int z, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%3, %4, %5}], [%2], %6;" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(x), "r"(y), "r"(z), "l"(policy)
      : "memory");
}

// Untiled bulk copy global -> shared (both 16-byte aligned, size a multiple of 16).
__device__ __forceinline__ void bulk_load(uint32_t dst, const void* src, uint32_t bytes,
                                          uint32_t bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
      "l"(src), "r"(bytes), "r"(bar)
      : "memory");
}

// ---------------------------------------------------------------- tcgen05: TMEM management
__device__ __forceinline__ void tmem_alloc(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// Per-warpgroup register budgets (every warp of a warpgroup executes the same instruction).  The
// increases draw on the registers the block was launched with: the budgets of all warpgroups
// must add up to at most threads x registers per thread at launch, which the launch checks.
template <int N>
__device__ __forceinline__ void regs_increase() {
  static_assert(N % 8 == 0 && N >= 24 && N <= 256, "register budget");
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(N));
}
template <int N>
__device__ __forceinline__ void regs_decrease() {
  static_assert(N % 8 == 0 && N >= 24 && N <= 256, "register budget");
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(N));
}

// ---------------------------------------------------------------- tcgen05: descriptors
// Shared-memory matrix descriptor, 128-byte swizzle (layout type 2), sm_100 version bit.
//   bits [0,14)  start address >> 4      bits [16,30) leading-dim byte offset >> 4
//   bits [32,46) stride-dim byte offset >> 4, bits [46,48) version = 1
//   bits [49,52) base offset = 0, bit 52 lbo mode = 0, bits [61,64) layout type
// K-major SW128 (rows of 128 B, 8-row atoms of 1 KiB): SBO = 1024, LBO unused.
// MN-major SW128: LBO = byte distance between 64-element MN chunks, SBO = byte distance
// between 8-row K groups (1024 for densely stacked rows).
// Swizzle-mode codes of the descriptor's [61,64) field.
constexpr uint32_t kLayoutSw128 = 2;  // 128-byte rows, 8-row (1 KiB) atoms
constexpr uint32_t kLayoutSw64 = 4;   // 64-byte rows, 8-row (512 B) atoms

__device__ __forceinline__ uint64_t sdesc_sw(uint32_t saddr, uint32_t lbo, uint32_t sbo, uint32_t layout) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32;
  d |= static_cast<uint64_t>(1) << 46;
  d |= static_cast<uint64_t>(layout) << 61;
  return d;
}

__device__ __forceinline__ uint64_t sdesc_sw128(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  return sdesc_sw(saddr, lbo, sbo, kLayoutSw128);
}

// Grid order: work item -> (unit, level), level 0 the heaviest.  Units come in bands of `band`;
// inside a band the items run level by level (every unit's heaviest tile first), and the bands
// follow each other.  Each band therefore ends with its lightest tiles, so the grid's tail is
// short CTAs, while only a band of units (and their K/V) is in flight at a time.
struct UnitLevel {
  int unit;
  int level;
};
__device__ __forceinline__ UnitLevel band_order(int item, int units, int levels, int band) {
  const int per_band = band * levels;
  const int b = item / per_band;
  const int first = b * band;
  const int size = min(band, units - first);
  const int r = item - b * per_band;
  return {first + r % size, r / size};
}

// Advance a descriptor's start address by `bytes` (a multiple of 16).  The start-address field
// is the low 14 bits of (address >> 4); shared-memory addresses stay below 256 KiB, so the add
// never carries into the next field.
__device__ __forceinline__ uint64_t desc_add(uint64_t desc, uint32_t bytes) {
  return desc + static_cast<uint64_t>(bytes >> 4);
}

// Instruction descriptor for kind::f16 with an fp32 accumulator.
//   [4,6) D format (1 = f32), [7,10) A format, [10,13) B format (0 = f16, 1 = bf16),
//   [15] A major (0 = K, 1 = MN), [16] B major, [17,23) N >> 3, [24,29) M >> 4.
__host__ __device__ constexpr uint32_t idesc_f16(bool bf16, int M, int N, bool a_mn, bool b_mn) {
  return (1u << 4) | ((bf16 ? 1u : 0u) << 7) | ((bf16 ? 1u : 0u) << 10) |
         ((a_mn ? 1u : 0u) << 15) | ((b_mn ? 1u : 0u) << 16) |
         (static_cast<uint32_t>(N >> 3) << 17) | (static_cast<uint32_t>(M >> 4) << 24);
}

// ---------------------------------------------------------------- tcgen05: MMA issue
// UMMA issue and commit, called by a whole warp with the same (warp-uniform) operands:
// elect.sync lets exactly one lane, always the lowest, issue the tcgen05 instruction, so every
// commit tracks that lane's MMAs.
//   umma_ss_w:     D[tmem] (+)= A[smem desc] * B[smem desc]^T
//   umma_ts_w:     D[tmem] (+)= A[tmem] * B[smem desc]  (A K-major, 2 x 16-bit per TMEM column)
//   umma_commit_w: arrive once on an mbarrier when every tcgen05 op issued so far is done.
// Descriptor arithmetic done by the whole warp stays on the uniform datapath: a loop in which one
// lane computed descriptors and issued measured 75.5 cycles per 128x128x16 UMMA with 16 busy
// warps on the SM, the warp-wide loop 64.8 (the UMMA's own rate).
__device__ __forceinline__ void umma_ss_w(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                          uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred pe, pa;\n\t"
      "elect.sync _|pe, 0xffffffff;\n\t"
      "setp.ne.b32 pa, %4, 0;\n\t"
      "@pe tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, pa;\n\t}\n" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate));
}
__device__ __forceinline__ void umma_ts_w(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                          uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred pe, pa;\n\t"
      "elect.sync _|pe, 0xffffffff;\n\t"
      "setp.ne.b32 pa, %4, 0;\n\t"
      "@pe tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, pa;\n\t}\n" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate));
}
__device__ __forceinline__ void umma_commit_w(uint32_t bar) {
  asm volatile(
      "{\n\t.reg .pred pe;\n\t"
      "elect.sync _|pe, 0xffffffff;\n\t"
      "@pe tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n\t}\n" ::"r"(bar)
      : "memory");
}

// ---------------------------------------------------------------- tcgen05: TMEM <-> registers
// 32x32b shape: thread t of the warp reads TMEM lane (lane_base + t), N consecutive 32-bit
// columns starting at the address's column.  A warp may only touch lanes
// [32*(warp_id % 4), 32*(warp_id % 4) + 32).
#define FA_R8(r, o) "=r"(r[o + 0]), "=r"(r[o + 1]), "=r"(r[o + 2]), "=r"(r[o + 3]), \
                    "=r"(r[o + 4]), "=r"(r[o + 5]), "=r"(r[o + 6]), "=r"(r[o + 7])
#define FA_W8(r, o) "r"(r[o + 0]), "r"(r[o + 1]), "r"(r[o + 2]), "r"(r[o + 3]), \
                    "r"(r[o + 4]), "r"(r[o + 5]), "r"(r[o + 6]), "r"(r[o + 7])
#define FA_D8(r, o) "+r"(r[o + 0]), "+r"(r[o + 1]), "+r"(r[o + 2]), "+r"(r[o + 3]), \
                    "+r"(r[o + 4]), "+r"(r[o + 5]), "+r"(r[o + 6]), "+r"(r[o + 7])

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : FA_R8(r, 0), FA_R8(r, 8), FA_R8(r, 16), FA_R8(r, 24)
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : FA_R8(r, 0), FA_R8(r, 8)
      : "r"(taddr));
}

// Wait for all outstanding tcgen05.ld of this thread.  The registers are threaded through
// as read-write operands so the compiler cannot hoist their uses above the wait.
__device__ __forceinline__ void tmem_ld_wait(uint32_t (&r)[32]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : FA_D8(r, 0), FA_D8(r, 8), FA_D8(r, 16), FA_D8(r, 24)
               :
               : "memory");
}
__device__ __forceinline__ void tmem_ld_wait16(uint32_t (&r)[16]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;" : FA_D8(r, 0), FA_D8(r, 8) : : "memory");
}

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
      FA_W8(r, 0), FA_W8(r, 8)
      : "memory");
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      FA_W8(r, 0), FA_W8(r, 8), FA_W8(r, 16), FA_W8(r, 24)
      : "memory");
}

__device__ __forceinline__ void tmem_st_wait() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// ---------------------------------------------------------------- math helpers
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// 2^(-x): the negation sits next to the ex2 so that it can become an operand modifier.
__device__ __forceinline__ float ex2_neg_approx(float x) {
  float y;
  asm("{\n\t.reg .f32 t;\n\tneg.f32 t, %1;\n\tex2.approx.ftz.f32 %0, t;\n\t}" : "=f"(y) : "f"(x));
  return y;
}

// ---- packed fp32 pairs (sm_100 f32x2 instructions: one issue slot for two lanes of math)
__device__ __forceinline__ uint64_t f2(float lo, float hi) {
  return (static_cast<uint64_t>(__float_as_uint(hi)) << 32) | __float_as_uint(lo);
}
__device__ __forceinline__ uint64_t f2u(uint32_t lo, uint32_t hi) {
  return (static_cast<uint64_t>(hi) << 32) | lo;
}
__device__ __forceinline__ float f2lo(uint64_t v) { return __uint_as_float(static_cast<uint32_t>(v)); }
__device__ __forceinline__ float f2hi(uint64_t v) { return __uint_as_float(static_cast<uint32_t>(v >> 32)); }
__device__ __forceinline__ uint64_t ffma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t fadd2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t fsub2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t fmul2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// 2^x for a pair of x <= 0 on the FMA pipe (no MUFU): x = n + f with n = round(x) (the 1.5 * 2^23
// addition leaves n in the low mantissa bits) and f in [-1/2, 1/2]; 2^f by a degree-3 polynomial
// fitted here to 2^f on [-1/2, 1/2] (relative-error least squares on Chebyshev nodes, reweighted
// towards the worst points: max relative error 7.5e-5, below half an fp16 ulp); 2^n is added to
// the result's exponent field.  x is clamped at -125 first: the polynomial's value lies in
// [2^-1/2, 2^1/2], so its exponent field is 126 or 127 and stays >= 1 (a normal number) after
// adding n >= -125.  Scores that far below the row maximum give at most 2^-124 instead of ~0,
// below anything a 16-bit P or the fp32 row sum can resolve next to the row's largest term (1).
__device__ __forceinline__ uint64_t exp2_poly2(uint64_t x2) {
  const float x0 = fmaxf(f2lo(x2), -125.f), x1 = fmaxf(f2hi(x2), -125.f);
  const uint64_t xc = f2(x0, x1);
  const uint64_t magic = f2(12582912.f, 12582912.f);
  const uint64_t j = fadd2(xc, magic);
  const uint64_t n = fsub2(j, magic);
  const uint64_t f = fsub2(xc, n);
  uint64_t p = ffma2(f2(0.05517164617776871f, 0.05517164617776871f), f,
                     f2(0.24261116981506348f, 0.24261116981506348f));
  p = ffma2(p, f, f2(0.6932609677314758f, 0.6932609677314758f));
  p = ffma2(p, f, f2(0.9999280571937561f, 0.9999280571937561f));
  const uint32_t lo = static_cast<uint32_t>(p) + (static_cast<uint32_t>(j) << 23);
  const uint32_t hi = static_cast<uint32_t>(p >> 32) + (static_cast<uint32_t>(j >> 32) << 23);
  return f2u(lo, hi);
}

// Pack two fp32 values into one 32-bit word of 16-bit floats (lo = first / lower k index).
template <bool kBf16>
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  uint32_t r;
  if constexpr (kBf16) {
    asm("cvt.rn.bf16x2.f32 %0, %2, %1;" : "=r"(r) : "f"(lo), "f"(hi));
  } else {
    asm("cvt.rn.f16x2.f32 %0, %2, %1;" : "=r"(r) : "f"(lo), "f"(hi));
  }
  return r;
}

}  // namespace fa
