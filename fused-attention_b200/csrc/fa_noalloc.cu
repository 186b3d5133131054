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
// Set-up: the first call on a device (with that device current) resolves the array's device
// address with cudaGetSymbolAddress and caches it; make that first call before any stream
// capture on the device.  The host-side name of the array is only a stand-in and is never passed
// to a kernel.
//
// Sharing: every call on a device uses the same array and leaves its delta in it.  Nothing needs
// clearing first, because the preprocess kernel writes every row the two gradient kernels read.
// Calls whose work overlaps on the GPU (for example on two streams without ordering between them)
// race on the array and must not be issued.
#include <mutex>

#include "../../include/fa_sm100.h"

namespace {

__device__ __align__(256) float g_delta_scratch[FA_NOALLOC_MAX_ROWS];

constexpr int kMaxDevices = 64;
float* g_scratch_ptr[kMaxDevices];
std::mutex g_scratch_mu;

// Device address of the scratch array on the current device (resolved once per device).
int scratch_for_current_device(float** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return FA_ERR_CUDA;
  if (dev < 0 || dev >= kMaxDevices) return FA_ERR_DEVICE;
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (g_scratch_ptr[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_delta_scratch) != cudaSuccess || p == nullptr) return FA_ERR_CUDA;
    g_scratch_ptr[dev] = static_cast<float*>(p);
  }
  *out = g_scratch_ptr[dev];
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
  float* delta = nullptr;
  int rc = scratch_for_current_device(&delta);
  if (rc != FA_OK) return rc;
  rc = fa_bwd_preprocess(o, dO, delta, B, H, S, D, dtype, dev_status, stream);
  if (rc != FA_OK) return rc;
  rc = fa_bwd_dkdv(q, k, v, dO, lse, delta, dk, dv, B, H, H_kv, S, D, dtype, tile_m, tile_n,
                   dev_status, stream);
  if (rc != FA_OK) return rc;
  return fa_bwd_dq(q, k, v, dO, lse, delta, dq, B, H, H_kv, S, D, dtype, tile_m, tile_n,
                   dev_status, stream);
}
