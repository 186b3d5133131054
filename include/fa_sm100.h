/* C ABI of the B200 (sm_100a) fused causal attention library, libfa_sm100.so.
 *
 * Every entry point:
 *   - takes DEVICE pointers to contiguous row-major tensors, plain integer sizes and a CUDA
 *     stream handle (cudaStream_t passed as void*; NULL = legacy default stream);
 *   - validates its arguments synchronously and returns FA_OK (0) or an FA_ERR_* code
 *     before anything is enqueued (fa_strerror() turns a code into text);
 *   - enqueues its kernels on `stream` and returns without synchronising the host;
 *   - allocates no device memory: all outputs and the scratch buffer `delta` belong to the
 *     caller.
 *
 * `dev_status` is a caller-owned int32[4] in device memory, zeroed before first use.  A kernel
 * whose internal pipeline wait exceeds its time limit stores an error code in dev_status[0]
 * (the CTA index in [1], the thread in [2]) and returns instead of hanging the GPU; later
 * launches that see a non-zero dev_status[0] exit immediately.  The caller reads it after a
 * stream synchronisation and resets it to zero.
 *
 * Layouts: q, o, dq, do = [B, H, S, D]; k, v, dk, dv = [B, H_kv, S, D] (H_kv divides H; query
 * head h reads K/V head h / (H / H_kv)); lse, delta = [B, H, S] float32.
 * dtype: FA_DTYPE_F16 or FA_DTYPE_BF16 (all 16-bit tensors share it); D in {32, 64, 128}.
 * Accumulation and softmax are float32.  lse is the log2-domain log-sum-exp of the scaled
 * scores:  lse[r] = log2( sum_{c <= r} 2^(log2(e) * q_r . k_c / sqrt(D)) ).
 */
#ifndef FA_SM100_H_
#define FA_SM100_H_

#ifdef __cplusplus
extern "C" {
#endif

#define FA_ABI_VERSION 1

#if defined(__GNUC__)
#define FA_API __attribute__((visibility("default")))
#else
#define FA_API
#endif

enum fa_status_code {
  FA_OK = 0,
  FA_ERR_INVALID_ARG = 1,  /* null pointer, non-positive size, H % H_kv != 0, ...       */
  FA_ERR_UNSUPPORTED = 2,  /* D, dtype or tile outside what the sm_100a kernels handle  */
  FA_ERR_ALIGNMENT = 3,    /* a tensor base address is not 16-byte aligned            */
  FA_ERR_CUDA = 4,         /* a CUDA runtime call failed (fa_last_cuda_error() has it) */
  FA_ERR_DRIVER = 5,       /* cuTensorMapEncodeTiled unavailable or rejected a tensor   */
  FA_ERR_DEVICE = 6,       /* current device is not compute capability 10.x (B200)      */
  FA_ERR_TOO_LARGE = 7     /* fa_bwd_noalloc: B*H*S exceeds FA_NOALLOC_MAX_ROWS         */
};

/* Capacity of fa_bwd_noalloc's static scratch: B*H*S float32 rows (16 MiB per GPU). */
#define FA_NOALLOC_MAX_ROWS (1 << 22)

enum fa_dtype { FA_DTYPE_F16 = 0, FA_DTYPE_BF16 = 1 };

/* ABI version of the loaded library (FA_ABI_VERSION at build time). */
FA_API int fa_abi_version(void);

/* Static description of an FA_ERR_* code. */
FA_API const char* fa_strerror(int code);

/* Text of the last CUDA runtime error seen by this thread inside the library. */
FA_API const char* fa_last_cuda_error(void);

/* Causal forward: o = softmax(q k^T / sqrt(D), causal) v, and lse when lse != NULL.
 * Replaces the kernel launch of attention/fused/fused.py:68-76 (fused_attention),
 * attention/gqa/fused_gqa.py:70-82 (fused_gqa_attention, H_kv < H) and the LSE-saving
 * forward attention/backward/fused_backward.py:26-62,161-170 (_forward).
 * tile_m, tile_n in {64, 128}: tile_n is the number of keys per K/V tile; the query side always
 * runs 128-row tcgen05 tiles (tile_m only takes part in the caller's divisibility contract). */
FA_API int fa_fwd(const void* q, const void* k, const void* v, void* o, float* lse,
           int B, int H, int H_kv, int S, int D, int dtype, int tile_m, int tile_n,
           int* dev_status, void* stream);

/* delta[b,h,r] = sum_d float(do[b,h,r,d]) * float(o[b,h,r,d]).
 * Replaces the host-side torch expression of attention/backward/fused_backward.py:175. */
FA_API int fa_bwd_preprocess(const void* o, const void* dO, float* delta,
                      int B, int H, int S, int D, int dtype, int* dev_status, void* stream);

/* dk, dv for every K/V head (summed over its query-head group, no atomics).
 * Replaces bwd_dkdv_kernel, attention/backward/fused_backward.py:66-107,180-181. */
FA_API int fa_bwd_dkdv(const void* q, const void* k, const void* v, const void* dO,
                const float* lse, const float* delta, void* dk, void* dv,
                int B, int H, int H_kv, int S, int D, int dtype, int tile_m, int tile_n,
                int* dev_status, void* stream);

/* dq.  Replaces bwd_dq_kernel, attention/backward/fused_backward.py:111-147,182-183. */
FA_API int fa_bwd_dq(const void* q, const void* k, const void* v, const void* dO,
              const float* lse, const float* delta, void* dq,
              int B, int H, int H_kv, int S, int D, int dtype, int tile_m, int tile_n,
              int* dev_status, void* stream);

/* Unfused causal forward, the reference's three-kernel baseline: s_buf = causal_mask(q k^T /
 * sqrt(D)) in float32, p_buf = row_softmax(s_buf) in the dtype of q, o = p_buf v.  Replaces the
 * three ct.launch calls of attention/fused/unfused.py:96-116 (unfused_attention) and
 * attention/gqa/unfused_gqa.py:99-128 (unfused_gqa_attention, H_kv < H).  s_buf and p_buf are
 * caller-owned [B, H, S, S] buffers; only their 128 x 128 tiles on or below the causal diagonal
 * are written (entries above the diagonal inside those tiles hold -inf and 0).  S % 8 == 0,
 * B * H <= 65535. */
FA_API int fa_unfused_fwd(const void* q, const void* k, const void* v, void* o, float* s_buf,
                          void* p_buf, int B, int H, int H_kv, int S, int D, int dtype,
                          int* dev_status, void* stream);

/* Whole backward (delta, dk/dv, dq) for callers that cannot allocate device memory: a plugin
 * inside a framework whose memory pool already holds nearly all of HBM, or a latency-critical
 * path that must not call cudaMalloc (it can synchronise the device).  No counterpart in the
 * reference.  Same tensors and rules as the three calls above, minus `delta`: the float32 delta
 * scratch lives in a static device array of FA_NOALLOC_MAX_ROWS rows that every GPU loading the
 * library holds until exit; larger problems (B*H*S > FA_NOALLOC_MAX_ROWS) return
 * FA_ERR_TOO_LARGE.  This call allocates nothing (no cudaMalloc/cudaFree).  A call made outside
 * stream capture looks up the array's address in the current CUDA context and remembers it; a
 * call made while its stream is captured uses the address remembered for the current context, so
 * make the first call in a context before any stream capture there (otherwise FA_ERR_CUDA).  After
 * cudaDeviceReset the next uncaptured call looks the address up again.
 * All calls on a device share the array: calls that overlap on the GPU race and must not be
 * issued; sequential calls need no clearing (every row is rewritten before it is read). */
FA_API int fa_bwd_noalloc(const void* q, const void* k, const void* v, const void* o,
                          const void* dO, const float* lse, void* dq, void* dk, void* dv,
                          int B, int H, int H_kv, int S, int D, int dtype, int tile_m, int tile_n,
                          int* dev_status, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* FA_SM100_H_ */
