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

}  // namespace

cudaError_t launch_bwd_preprocess(const BwdParams& p, bool bf16, cudaStream_t stream) {
  if (p.D == 64) return bf16 ? launch_pre_t<64, true>(p, stream) : launch_pre_t<64, false>(p, stream);
  if (p.D == 128) return bf16 ? launch_pre_t<128, true>(p, stream) : launch_pre_t<128, false>(p, stream);
  return cudaErrorInvalidValue;
}

cudaError_t launch_bwd_dkdv(const CUtensorMap&, const CUtensorMap&, const CUtensorMap&,
                            const CUtensorMap&, const BwdParams&, bool, cudaStream_t) {
  return cudaErrorNotSupported;
}

cudaError_t launch_bwd_dq(const CUtensorMap&, const CUtensorMap&, const CUtensorMap&,
                          const CUtensorMap&, const BwdParams&, bool, cudaStream_t) {
  return cudaErrorNotSupported;
}

}  // namespace fa
