// C-ABI entry points of libfa_sm100.so (declared in include/fa_sm100.h).
//
// Host-side duties: argument validation (synchronous, before anything is enqueued), TMA tensor
// map encoding through the driver entry point (no link-time libcuda dependency), work-grid
// sizing, and the launch on the caller's stream.  Nothing here allocates device memory.
#include <atomic>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "../../include/fa_sm100.h"
#include "fa_internal.h"

namespace {
thread_local char g_last_cuda_error[256] = "";
}  // namespace

namespace fa {

int cuda_fail(cudaError_t e) {
  std::snprintf(g_last_cuda_error, sizeof(g_last_cuda_error), "%s: %s", cudaGetErrorName(e),
                cudaGetErrorString(e));
  // The error now lives in fa_last_cuda_error(); clear the runtime's (non-sticky) last-error
  // state so that a host framework does not report it again at an unrelated later call.
  (void)cudaGetLastError();
  return e == cudaErrorNotSupported ? FA_ERR_UNSUPPORTED : FA_ERR_CUDA;
}

int check_device() {
  // Per-device answer, cached: 0 unknown, 1 ok, 2 wrong arch (threads may race to fill an entry;
  // they all store the same value).
  static std::atomic<int> cached[64];
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e);
  const bool slot = dev >= 0 && dev < 64;
  const int known = slot ? cached[dev].load(std::memory_order_relaxed) : 0;
  if (known != 0) return known == 1 ? FA_OK : FA_ERR_DEVICE;
  int major = 0;
  e = cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
  if (e != cudaSuccess) return cuda_fail(e);
  const int ok = (major == 10) ? 1 : 2;
  if (slot) cached[dev].store(ok, std::memory_order_relaxed);
  return ok == 1 ? FA_OK : FA_ERR_DEVICE;
}

}  // namespace fa

namespace {

using fa::check_device;
using fa::cuda_fail;

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault,
                                         &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// Tensor map over a contiguous [BH, S, D] 16-bit tensor, boxes of 64 columns (128 B, the
// 128-byte swizzle span) x box_rows rows x 1 head.  Rows past S read as zero.
// Tensor maps encoded by this thread, reused when a call names the same tensor again (a map is a
// pure function of the address, shape, element type and box, so a hit is always valid).  Short
// calls spend a measurable part of their host time encoding three or four maps.
struct MapKey {
  const void* ptr;
  int bh, S, D, dtype, box_rows;
  bool operator==(const MapKey& o) const {
    return ptr == o.ptr && bh == o.bh && S == o.S && D == o.D && dtype == o.dtype && box_rows == o.box_rows;
  }
};
struct MapSlot {
  MapKey key;
  CUtensorMap map;
  bool used;
};
constexpr int kMapSlots = 16;
thread_local MapSlot t_maps[kMapSlots];
thread_local int t_map_next = 0;

int encode_map(CUtensorMap* m, const void* ptr, int bh, int S, int D, int dtype, int box_rows);

int make_map(CUtensorMap* m, const void* ptr, int bh, int S, int D, int dtype, int box_rows) {
  const MapKey key{ptr, bh, S, D, dtype, box_rows};
  for (int i = 0; i < kMapSlots; ++i)
    if (t_maps[i].used && t_maps[i].key == key) {
      *m = t_maps[i].map;
      return FA_OK;
    }
  const int rc = encode_map(m, ptr, bh, S, D, dtype, box_rows);
  if (rc == FA_OK) {
    MapSlot& slot = t_maps[t_map_next];
    t_map_next = (t_map_next + 1) % kMapSlots;
    slot.key = key;
    slot.map = *m;
    slot.used = true;
  }
  return rc;
}

int encode_map(CUtensorMap* m, const void* ptr, int bh, int S, int D, int dtype, int box_rows) {
  EncodeTiledFn enc = encode_fn();
  if (enc == nullptr) return FA_ERR_DRIVER;
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(D), static_cast<cuuint64_t>(S),
                        static_cast<cuuint64_t>(bh)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(D) * 2, static_cast<cuuint64_t>(S) * D * 2};
  // 64-column boxes (128-byte rows) with the 128-byte swizzle; D = 32 rows are 64 bytes, so
  // one 32-column box with the 64-byte swizzle.
  const bool narrow = D < 64;
  cuuint32_t box[3] = {narrow ? 32u : 64u, static_cast<cuuint32_t>(box_rows), 1u};
  cuuint32_t estr[3] = {1u, 1u, 1u};
  CUresult r = enc(m, dtype == FA_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                             : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                   3, const_cast<void*>(ptr), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, narrow ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? FA_OK : FA_ERR_DRIVER;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Argument checks that need no device: every entry point runs them (and its alignment checks)
// before check_device(), so a bad argument is reported the same way with or without a GPU.
int check_common(int B, int H, int H_kv, int S, int D, int dtype, int tile_m, int tile_n,
                 const int* dev_status) {
  if (B < 1 || H < 1 || H_kv < 1 || S < 1) return FA_ERR_INVALID_ARG;
  if (H % H_kv != 0) return FA_ERR_INVALID_ARG;
  if (dev_status == nullptr) return FA_ERR_INVALID_ARG;
  if (dtype != FA_DTYPE_F16 && dtype != FA_DTYPE_BF16) return FA_ERR_UNSUPPORTED;
  if (D != 32 && D != 64 && D != 128) return FA_ERR_UNSUPPORTED;
  if ((tile_m != 64 && tile_m != 128) || (tile_n != 64 && tile_n != 128)) return FA_ERR_UNSUPPORTED;
  // Every index the kernels form fits in 32 bits per head, 64 bits overall.
  if (static_cast<long long>(B) * H > (1LL << 30) || S > (1 << 24)) return FA_ERR_UNSUPPORTED;
  return FA_OK;
}

}  // namespace

extern "C" {

int fa_abi_version(void) { return FA_ABI_VERSION; }

const char* fa_strerror(int code) {
  switch (code) {
    case FA_OK: return "ok";
    case FA_ERR_INVALID_ARG: return "invalid argument (null pointer, non-positive size or H not divisible by H_kv)";
    case FA_ERR_UNSUPPORTED: return "unsupported configuration (D must be 32, 64 or 128, dtype f16/bf16, tiles 64/128)";
    case FA_ERR_ALIGNMENT: return "tensor base address is not 16-byte aligned";
    case FA_ERR_CUDA: return "CUDA runtime error (see fa_last_cuda_error)";
    case FA_ERR_DRIVER: return "cuTensorMapEncodeTiled unavailable or rejected the tensor";
    case FA_ERR_DEVICE: return "current device is not an sm_100 (B200) GPU";
    case FA_ERR_TOO_LARGE: return "B*H*S exceeds the static scratch of fa_bwd_noalloc (FA_NOALLOC_MAX_ROWS rows)";
    default: return "unknown error code";
  }
}

const char* fa_last_cuda_error(void) { return g_last_cuda_error; }

int fa_fwd(const void* q, const void* k, const void* v, void* o, float* lse, int B, int H,
           int H_kv, int S, int D, int dtype, int tile_m, int tile_n, int* dev_status,
           void* stream) {
  if (!q || !k || !v || !o) return FA_ERR_INVALID_ARG;
  int rc = check_common(B, H, H_kv, S, D, dtype, tile_m, tile_n, dev_status);
  if (rc != FA_OK) return rc;
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(o) ||
      (lse && (reinterpret_cast<uintptr_t>(lse) & 3u)))
    return FA_ERR_ALIGNMENT;
  if ((rc = check_device()) != FA_OK) return rc;

  CUtensorMap tmQ, tmK, tmV;
  if ((rc = make_map(&tmQ, q, B * H, S, D, dtype, 128)) != FA_OK) return rc;
  if ((rc = make_map(&tmK, k, B * H_kv, S, D, dtype, tile_n)) != FA_OK) return rc;
  if ((rc = make_map(&tmV, v, B * H_kv, S, D, dtype, tile_n)) != FA_OK) return rc;

  fa::FwdParams p{};
  p.o = o;
  p.lse = lse;
  p.status = dev_status;
  p.S = S;
  p.H = H;
  p.H_kv = H_kv;
  p.group = H / H_kv;
  p.B = B;
  p.nq = (S + 127) / 128;
  p.mode = (p.group % 2 == 0) ? 1 : 0;
  const long long items = p.mode == 0 ? static_cast<long long>(B) * H * ((p.nq + 1) / 2)
                                      : static_cast<long long>(B) * (H / 2) * p.nq;
  if (items > 0x7fffffffLL) return FA_ERR_UNSUPPORTED;
  p.n_items = static_cast<int>(items);
  p.band = fa::work_band(p.mode == 0 ? static_cast<long long>(B) * H : static_cast<long long>(B) * (H / 2));
  p.scale_log2 = 1.4426950408889634f / sqrtf(static_cast<float>(D));
  cudaError_t e = fa::launch_fwd(tmQ, tmK, tmV, p, D, tile_n, dtype == FA_DTYPE_BF16,
                                 static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? FA_OK : cuda_fail(e);
}

int fa_bwd_preprocess(const void* o, const void* dO, float* delta, int B, int H, int S, int D,
                      int dtype, int* dev_status, void* stream) {
  if (!o || !dO || !delta) return FA_ERR_INVALID_ARG;
  int rc = check_common(B, H, H, S, D, dtype, 128, 128, dev_status);
  if (rc != FA_OK) return rc;
  if (!aligned16(o) || !aligned16(dO) || (reinterpret_cast<uintptr_t>(delta) & 3u))
    return FA_ERR_ALIGNMENT;
  if ((rc = check_device()) != FA_OK) return rc;
  fa::BwdParams p{};
  p.o = o;
  p.dO = dO;
  p.delta = delta;
  p.status = dev_status;
  p.S = S;
  p.H = H;
  p.H_kv = H;
  p.group = 1;
  p.B = B;
  p.D = D;
  cudaError_t e = fa::launch_bwd_preprocess(p, dtype == FA_DTYPE_BF16, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? FA_OK : cuda_fail(e);
}

static int bwd_prepare(const void* q, const void* k, const void* v, const void* dO,
                       const float* lse, const float* delta, int B, int H, int H_kv, int S,
                       int D, int dtype, int tile_m, int tile_n, int* dev_status,
                       CUtensorMap* tmQ, CUtensorMap* tmK, CUtensorMap* tmV, CUtensorMap* tmdO,
                       fa::BwdParams* p, int q_rows, int kv_rows) {
  if (!q || !k || !v || !dO || !lse || !delta) return FA_ERR_INVALID_ARG;
  int rc = check_common(B, H, H_kv, S, D, dtype, tile_m, tile_n, dev_status);
  if (rc != FA_OK) return rc;
  // The backward streams whole 64-row tiles (and their lse / delta slices).
  if (S % 64 != 0) return FA_ERR_UNSUPPORTED;
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(dO) || !aligned16(lse) ||
      !aligned16(delta))
    return FA_ERR_ALIGNMENT;
  if ((rc = check_device()) != FA_OK) return rc;
  if ((rc = make_map(tmQ, q, B * H, S, D, dtype, q_rows)) != FA_OK) return rc;
  if ((rc = make_map(tmK, k, B * H_kv, S, D, dtype, kv_rows)) != FA_OK) return rc;
  if ((rc = make_map(tmV, v, B * H_kv, S, D, dtype, kv_rows)) != FA_OK) return rc;
  if ((rc = make_map(tmdO, dO, B * H, S, D, dtype, q_rows)) != FA_OK) return rc;
  p->q = q;
  p->k = k;
  p->v = v;
  p->dO = dO;
  p->lse = lse;
  p->delta = const_cast<float*>(delta);
  p->status = dev_status;
  p->S = S;
  p->H = H;
  p->H_kv = H_kv;
  p->group = H / H_kv;
  p->B = B;
  p->D = D;
  p->nq = (S + 127) / 128;
  p->scale_log2 = 1.4426950408889634f / sqrtf(static_cast<float>(D));
  p->sm_scale = 1.0f / sqrtf(static_cast<float>(D));
  return FA_OK;
}

int fa_bwd_dkdv(const void* q, const void* k, const void* v, const void* dO, const float* lse,
                const float* delta, void* dk, void* dv, int B, int H, int H_kv, int S, int D,
                int dtype, int tile_m, int tile_n, int* dev_status, void* stream) {
  if (!dk || !dv) return FA_ERR_INVALID_ARG;
  if (!aligned16(dk) || !aligned16(dv)) return FA_ERR_ALIGNMENT;
  CUtensorMap tmQ, tmK, tmV, tmdO;
  fa::BwdParams p{};
  int rc = bwd_prepare(q, k, v, dO, lse, delta, B, H, H_kv, S, D, dtype, tile_m, tile_n,
                       dev_status, &tmQ, &tmK, &tmV, &tmdO, &p, /*q_rows=*/128, /*kv_rows=*/128);
  if (rc != FA_OK) return rc;
  p.dk = dk;
  p.dv = dv;
  p.band = fa::work_band(static_cast<long long>(B) * H_kv);
  cudaError_t e = fa::launch_bwd_dkdv(tmQ, tmK, tmV, tmdO, p, dtype == FA_DTYPE_BF16,
                                      static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? FA_OK : cuda_fail(e);
}

int fa_bwd_dq(const void* q, const void* k, const void* v, const void* dO, const float* lse,
              const float* delta, void* dq, int B, int H, int H_kv, int S, int D, int dtype,
              int tile_m, int tile_n, int* dev_status, void* stream) {
  if (!dq) return FA_ERR_INVALID_ARG;
  if (!aligned16(dq)) return FA_ERR_ALIGNMENT;
  CUtensorMap tmQ, tmK, tmV, tmdO;
  fa::BwdParams p{};
  int rc = bwd_prepare(q, k, v, dO, lse, delta, B, H, H_kv, S, D, dtype, tile_m, tile_n,
                       dev_status, &tmQ, &tmK, &tmV, &tmdO, &p, /*q_rows=*/128, /*kv_rows=*/128);
  if (rc != FA_OK) return rc;
  p.dq = dq;
  p.band = fa::work_band(static_cast<long long>(B) * H);
  cudaError_t e = fa::launch_bwd_dq(tmQ, tmK, tmV, tmdO, p, dtype == FA_DTYPE_BF16,
                                    static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? FA_OK : cuda_fail(e);
}

int fa_unfused_fwd(const void* q, const void* k, const void* v, void* o, float* s_buf, void* p_buf,
                   int B, int H, int H_kv, int S, int D, int dtype, int* dev_status, void* stream) {
  if (!q || !k || !v || !o || !s_buf || !p_buf) return FA_ERR_INVALID_ARG;
  int rc = check_common(B, H, H_kv, S, D, dtype, 128, 128, dev_status);
  if (rc != FA_OK) return rc;
  // P rows must be 16-byte aligned for its tensor map; grid.y holds B * H.
  if (S % 8 != 0 || static_cast<long long>(B) * H > 65535) return FA_ERR_UNSUPPORTED;
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(o) || !aligned16(s_buf) ||
      !aligned16(p_buf))
    return FA_ERR_ALIGNMENT;
  if ((rc = check_device()) != FA_OK) return rc;
  CUtensorMap tmQ, tmK, tmP, tmV;
  if ((rc = make_map(&tmQ, q, B * H, S, D, dtype, 128)) != FA_OK) return rc;
  if ((rc = make_map(&tmK, k, B * H_kv, S, D, dtype, 128)) != FA_OK) return rc;
  if ((rc = make_map(&tmV, v, B * H_kv, S, D, dtype, 128)) != FA_OK) return rc;
  // P viewed as [B * H, S rows, S columns]: 64-column boxes of 128 rows (the score tiles' rows).
  if ((rc = make_map(&tmP, p_buf, B * H, S, S, dtype, 128)) != FA_OK) return rc;
  fa::UnfParams p{};
  p.o = o;
  p.s = s_buf;
  p.p = p_buf;
  p.status = dev_status;
  p.N = S;
  p.H = H;
  p.H_kv = H_kv;
  p.group = H / H_kv;
  p.B = B;
  p.sm_scale = 1.0f / sqrtf(static_cast<float>(D));
  cudaError_t e = fa::launch_unfused(tmQ, tmK, tmP, tmV, p, D, dtype == FA_DTYPE_BF16,
                                     static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? FA_OK : cuda_fail(e);
}

}  // extern "C"
