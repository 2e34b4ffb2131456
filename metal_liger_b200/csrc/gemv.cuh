// HBM-streaming matrix-vector products for decoding (batch <= 2): a warp per
// weight row, every lane issuing kGemvBatch 16-byte weight loads before the
// first product uses one, the activations (batch x K bf16) in shared memory.
// Shared by the plain GEMV (gemv.cu) and the greedy head (lm_head.cu).
#pragma once

#include "common.cuh"

namespace ml {
namespace gemv {

constexpr int kThreads = 512;  // one CTA of 16 warps per SM
constexpr int kBatch = 16;     // 16-byte weight loads in flight per lane
constexpr int kMaxRows = 2;    // activation rows (sequences) per call

__device__ __forceinline__ float dot8_bf16(const uint4& a, const uint4& b, float acc) {
  const __nv_bfloat162* x = reinterpret_cast<const __nv_bfloat162*>(&a);
  const __nv_bfloat162* y = reinterpret_cast<const __nv_bfloat162*>(&b);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 fx = __bfloat1622float2(x[i]);
    const float2 fy = __bfloat1622float2(y[i]);
    acc = fmaf(fx.x, fy.x, acc);
    acc = fmaf(fx.y, fy.y, acc);
  }
  return acc;
}

// Stages rows [0, NB) of x (K bf16 each, pitch ld_x) into shared memory as
// 16-byte chunks [NB][K / 8].  Ends with __syncthreads().
template <int NB>
__device__ __forceinline__ void stage_rows(uint4* hs, const __nv_bfloat16* __restrict__ x,
                                           int64_t ld_x, int64_t nchunk) {
  for (int64_t i = threadIdx.x; i < NB * nchunk; i += blockDim.x) {
    const int b = (int)(i / nchunk);
    const int64_t c = i - b * nchunk;
    hs[i] = *reinterpret_cast<const uint4*>(x + b * ld_x + c * 8);
  }
  __syncthreads();
}

// acc[b] = this lane's share of dot(weight row, x row b); the caller sums
// the warp (warp_sum: a fixed butterfly).  Lane l takes chunks l, l + 32, ...
template <int NB>
__device__ __forceinline__ void row_dot(const uint4* __restrict__ wrow, const uint4* hs,
                                        int64_t nchunk, int lane, float (&acc)[NB]) {
#pragma unroll
  for (int b = 0; b < NB; ++b) acc[b] = 0.f;
  for (int64_t c0 = lane; c0 < nchunk; c0 += 32 * kBatch) {
    uint4 wv[kBatch];
#pragma unroll
    for (int u = 0; u < kBatch; ++u) {
      const int64_t c = c0 + 32 * u;
      if (c < nchunk) wv[u] = __ldcs(wrow + c);
    }
#pragma unroll
    for (int u = 0; u < kBatch; ++u) {
      const int64_t c = c0 + 32 * u;
      if (c < nchunk) {
#pragma unroll
        for (int b = 0; b < NB; ++b) acc[b] = dot8_bf16(wv[u], hs[b * nchunk + c], acc[b]);
      }
    }
  }
}

// Host: whether a call can take the GEMV kernels (16-byte rows, shared
// memory for the activations).
inline bool eligible(int64_t rows, int64_t K, int64_t ld_x, int64_t ld_w, const void* x,
                     const void* w) {
  return rows >= 1 && rows <= kMaxRows && K % 8 == 0 && ld_x % 8 == 0 && ld_w % 8 == 0 &&
         aligned16(x) && aligned16(w) && (size_t)rows * K * 2 <= 96 * 1024;
}

}  // namespace gemv
}  // namespace ml
