// Host-side declarations shared by the C-ABI layer (fa_api.cu) and the kernel files.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <atomic>
#include <cstdint>

namespace fa {

// Parameters of one forward launch (plain values; tensor maps travel separately as
// __grid_constant__ kernel parameters).
struct FwdParams {
  void* o;            // [B, H, S, D] output, same dtype as q
  float* lse;         // [B, H, S] log2-domain LSE, or nullptr
  int* status;        // int32[4] device status word (see DeviceError)
  int S;              // sequence length (queries == keys)
  int H;              // query heads
  int H_kv;           // key/value heads
  int group;          // H / H_kv
  int B;              // batch
  int nq;             // number of 128-row query tiles = ceil(S / 128)
  int mode;           // 0: a CTA takes q-tiles (2c, 2c+1) of one head; 1: q-tile i of heads (2p, 2p+1)
  int n_items;        // grid size
  int band;           // work units (heads or head pairs) ordered heavy-first together
  float scale_log2;   // log2(e) / sqrt(D)
};

struct BwdParams {
  const void* q;
  const void* k;
  const void* v;
  const void* o;
  const void* dO;
  const float* lse;   // [B, H, S] log2 domain
  float* delta;       // [B, H, S] rowsum(dO * O) (written by the preprocess kernel)
  void* dq;
  void* dk;
  void* dv;
  int* status;
  int S, H, H_kv, group, B, D;
  int nq;             // ceil(S / 128)
  int n_items;
  int band;           // work units (heads) ordered heavy-first together
  float scale_log2;   // log2(e) / sqrt(D)
  float sm_scale;     // 1 / sqrt(D)
};

// Parameters of the unfused three-kernel baseline (scores, softmax, P V).
struct UnfParams {
  void* o;            // [B, H, N, D] output
  float* s;           // [B, H, N, N] fp32 scores (written by the scores kernel)
  void* p;            // [B, H, N, N] 16-bit probabilities (written by the softmax kernel)
  int* status;
  int N, H, H_kv, group, B;
  float sm_scale;     // 1 / sqrt(D)
};

// Work units (heads, head pairs) whose tiles are launched heavy-first together: up to 16 units,
// about 64 MiB of K/V at S = 8192, D = 128, so the heads in flight keep their K/V in the 126 MB L2.
#ifndef FA_WORK_BAND
#define FA_WORK_BAND 16
#endif
inline int work_band(long long units) {
  return units < FA_WORK_BAND ? static_cast<int>(units) : FA_WORK_BAND;
}

// Opt a kernel into `bytes` of dynamic shared memory once per device (the attribute is a
// per-function, per-device setting; setting it on every launch costs host time on short calls).
// `done` is the kernel's own flag array; devices past its size set the attribute every time.
template <typename Kernel>
inline cudaError_t opt_in_smem(Kernel kernel, int bytes, std::atomic<bool> (&done)[64],
                               int launch_regs = 0) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev >= 0 && dev < 64 && done[dev].load(std::memory_order_acquire)) return cudaSuccess;
  if (launch_regs > 0) {
    // A kernel that moves registers between its warpgroups at run time was written for exactly
    // this many registers per thread at launch; with fewer, its increases could never be met.
    cudaFuncAttributes attr;
    e = cudaFuncGetAttributes(&attr, kernel);
    if (e != cudaSuccess) return e;
    if (attr.numRegs != launch_regs) return cudaErrorInvalidKernelImage;
  }
  e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess && dev >= 0 && dev < 64) done[dev].store(true, std::memory_order_release);
  return e;
}

// Host helpers of the C-ABI layer (fa_api.cu), shared with fa_noalloc.cu.
// cuda_fail: records `e` as the text fa_last_cuda_error() returns and maps it to an FA_ERR_* code.
// check_device: FA_OK if the current device is compute capability 10.x, else FA_ERR_DEVICE (or the
// FA_ERR_* code of a failed runtime query).
int cuda_fail(cudaError_t e);
int check_device();

// Launchers implemented in the kernel translation units.  They return a cudaError_t.
cudaError_t launch_fwd(const CUtensorMap& tmQ, const CUtensorMap& tmK, const CUtensorMap& tmV,
                       const FwdParams& p, int D, int block_n, bool bf16, cudaStream_t stream);

cudaError_t launch_bwd_preprocess(const BwdParams& p, bool bf16, cudaStream_t stream);
cudaError_t launch_unfused(const CUtensorMap& tmQ, const CUtensorMap& tmK, const CUtensorMap& tmP,
                           const CUtensorMap& tmV, const UnfParams& p, int D, bool bf16, cudaStream_t stream);
cudaError_t launch_bwd_dkdv(const CUtensorMap& tmQ, const CUtensorMap& tmK, const CUtensorMap& tmV,
                            const CUtensorMap& tmdO, const BwdParams& p, bool bf16,
                            cudaStream_t stream);
cudaError_t launch_bwd_dq(const CUtensorMap& tmQ, const CUtensorMap& tmK, const CUtensorMap& tmV,
                          const CUtensorMap& tmdO, const BwdParams& p, bool bf16,
                          cudaStream_t stream);

}  // namespace fa
