// fa_bwd_noalloc: the backward pass for callers that cannot allocate device memory.
//
// The regular backward (fa_bwd_preprocess + fa_bwd_dkdv + fa_bwd_dq) needs a float32 scratch
// buffer `delta` of B*H*S rows that the caller allocates.  Some callers cannot do that: a plugin
// hosted inside a framework whose memory pool has already reserved nearly all of HBM (a raw
// cudaMalloc from the plugin then fails), or code on a latency-critical path that must not call
// cudaMalloc because it can synchronise the device and stall every other stream.  For them this
// file keeps the scratch in a file-scope __device__ array of fixed size, allocated once when the
// library's device code is loaded on a GPU and held by every GPU that loads the library until the
// process exits.  The caller still passes all inputs and outputs.
//
// Address of the array: the host-side name of the array is only a stand-in and is never passed to
// a kernel.  Every call made outside stream capture looks up the array's device address in the
// current CUDA context (cudaGetSymbolAddress, after the device check) and remembers it for that
// context; a call made while its stream is being captured uses the address remembered for the
// current context, so the first call in a context must come before any stream capture there (a
// captured call without one fails with FA_ERR_CUDA).  Because every uncaptured call looks the
// address up again, a context created after cudaDeviceReset, or a different context on the same
// device (a driver-API caller with its own cuCtxCreate), never runs with another context's
// address once it has made one uncaptured call.
//
// Sharing: every call on a device uses the same array and leaves its delta in it.  Nothing needs
// clearing first, because the preprocess kernel writes every row the two gradient kernels read.
// Calls whose work overlaps on the GPU (for example on two streams without ordering between them)
// race on the array and must not be issued.
#include <mutex>

#include "../../include/fa_sm100.h"
#include "fa_internal.h"

namespace {

__device__ __align__(256) float g_delta_scratch[FA_NOALLOC_MAX_ROWS];

using CtxGetCurrentFn = CUresult (*)(CUcontext*);

CtxGetCurrentFn ctx_get_current_fn() {
  static CtxGetCurrentFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuCtxGetCurrent", &p, 12000, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<CtxGetCurrentFn>(p);
  });
  return fn;
}

// Scratch addresses remembered per CUDA context (filled by uncaptured calls, read by captured ones).
constexpr int kCacheSlots = 64;
struct ScratchEntry {
  CUcontext ctx;
  float* ptr;
};
ScratchEntry g_cache[kCacheSlots];
int g_cache_next = 0;
std::mutex g_cache_mu;

int scratch_for_current_context(cudaStream_t stream, float** out) {
  cudaStreamCaptureStatus capture = cudaStreamCaptureStatusNone;
  cudaError_t e = cudaStreamIsCapturing(stream, &capture);
  if (e != cudaSuccess) return fa::cuda_fail(e);
  CtxGetCurrentFn get_ctx = ctx_get_current_fn();
  CUcontext ctx = nullptr;
  if (get_ctx == nullptr || get_ctx(&ctx) != CUDA_SUCCESS || ctx == nullptr) return FA_ERR_DRIVER;
  std::lock_guard<std::mutex> lock(g_cache_mu);
  int slot = -1;
  for (int i = 0; i < kCacheSlots; ++i)
    if (g_cache[i].ctx == ctx) slot = i;
  if (capture != cudaStreamCaptureStatusNone) {
    if (slot < 0) return fa::cuda_fail(cudaErrorStreamCaptureUnsupported);
    *out = g_cache[slot].ptr;
    return FA_OK;
  }
  void* p = nullptr;
  e = cudaGetSymbolAddress(&p, g_delta_scratch);
  if (e != cudaSuccess) return fa::cuda_fail(e);
  if (p == nullptr) return fa::cuda_fail(cudaErrorInvalidSymbol);
  if (slot < 0) {
    slot = g_cache_next;
    g_cache_next = (g_cache_next + 1) % kCacheSlots;
  }
  g_cache[slot] = {ctx, static_cast<float*>(p)};
  *out = static_cast<float*>(p);
  return FA_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

extern "C" int fa_bwd_noalloc(const void* q, const void* k, const void* v, const void* o,
                              const void* dO, const float* lse, void* dq, void* dk, void* dv,
                              int B, int H, int H_kv, int S, int D, int dtype, int tile_m,
                              int tile_n, int* dev_status, void* stream) {
  // Every check the three launches below would make, done before anything is enqueued.
  if (!q || !k || !v || !o || !dO || !lse || !dq || !dk || !dv || !dev_status) return FA_ERR_INVALID_ARG;
  if (B < 1 || H < 1 || H_kv < 1 || S < 1 || H % H_kv != 0) return FA_ERR_INVALID_ARG;
  if (static_cast<long long>(B) * H * S > FA_NOALLOC_MAX_ROWS) return FA_ERR_TOO_LARGE;
  if (dtype != FA_DTYPE_F16 && dtype != FA_DTYPE_BF16) return FA_ERR_UNSUPPORTED;
  if (D != 32 && D != 64 && D != 128) return FA_ERR_UNSUPPORTED;
  if ((tile_m != 64 && tile_m != 128) || (tile_n != 64 && tile_n != 128)) return FA_ERR_UNSUPPORTED;
  if (S % 64 != 0) return FA_ERR_UNSUPPORTED;
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(o) || !aligned16(dO) ||
      !aligned16(lse) || !aligned16(dq) || !aligned16(dk) || !aligned16(dv))
    return FA_ERR_ALIGNMENT;
  // The device check comes first: on a GPU that is not sm_100 the symbol lookup would fail with
  // a runtime error instead of the FA_ERR_DEVICE every other entry point returns.
  int rc = fa::check_device();
  if (rc != FA_OK) return rc;
  float* delta = nullptr;
  rc = scratch_for_current_context(static_cast<cudaStream_t>(stream), &delta);
  if (rc != FA_OK) return rc;
  rc = fa_bwd_preprocess(o, dO, delta, B, H, S, D, dtype, dev_status, stream);
  if (rc != FA_OK) return rc;
  rc = fa_bwd_dkdv(q, k, v, dO, lse, delta, dk, dv, B, H, H_kv, S, D, dtype, tile_m, tile_n,
                   dev_status, stream);
  if (rc != FA_OK) return rc;
  return fa_bwd_dq(q, k, v, dO, lse, delta, dq, B, H, H_kv, S, D, dtype, tile_m, tile_n,
                   dev_status, stream);
}
