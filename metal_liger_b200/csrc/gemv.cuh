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

// RMSNorm of the staged activations in place, the decoder's input /
// post-attention norm fused into the projection that consumes it:
// hs[b] = bf16((x * r) * w) with r = rsqrt(mean(x^2) + eps), computed the
// way the RMSNorm forward kernel (rms_norm.cu, rms_fwd_vec / rms_fwd_ring)
// computes a row laid out as `tpr` threads of `nv` 16-byte vectors — thread
// t squares vectors t, t + tpr, ... in element order with fmaf, the row
// group sums by shuffles (tpr < 32) or by warp butterflies and then the
// warps' partials in warp order — so the fused product equals RMSNorm
// followed by the GEMV bit for bit.  Needs tpr <= blockDim.x.  Ends with
// __syncthreads().
template <int NB>
__device__ __forceinline__ void rmsnorm_rows(uint4* hs, int64_t nchunk,
                                             const __nv_bfloat16* __restrict__ nw, float eps,
                                             int tpr, int nv) {
  __shared__ float red[32];
  __shared__ float tot_s;
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const float inv_h = 1.f / (float)(nchunk * 8);
#pragma unroll
  for (int b = 0; b < NB; ++b) {
    const uint4* row = hs + b * nchunk;
    float ss = 0.f;
    if (t < tpr) {
      for (int i = 0; i < nv; ++i) {
        const int64_t v = (int64_t)i * tpr + t;
        if (v < nchunk) {
          const uint4 c = row[v];
          const __nv_bfloat162* e = reinterpret_cast<const __nv_bfloat162*>(&c);
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const float2 f = __bfloat1622float2(e[j]);
            ss = fmaf(f.x, f.x, ss);
            ss = fmaf(f.y, f.y, ss);
          }
        }
      }
    }
    if (tpr < 32) {
      for (int o = tpr >> 1; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
      if (t == 0) tot_s = ss;
    } else {
      ss = warp_sum(ss);
      if (lane == 0 && warp < (tpr >> 5)) red[warp] = ss;
    }
    __syncthreads();
    float tot;
    if (tpr < 32) {
      tot = tot_s;
    } else {
      tot = 0.f;
      for (int i = 0; i < (tpr >> 5); ++i) tot += red[i];  // warp order, as the norm kernel
    }
    const float r = rsqrtf(fmaf(tot, inv_h, eps));
    for (int64_t c = t; c < nchunk; c += blockDim.x) {
      uint4 xv = hs[b * nchunk + c];
      const uint4 wv = *reinterpret_cast<const uint4*>(nw + c * 8);
      __nv_bfloat162* xe = reinterpret_cast<__nv_bfloat162*>(&xv);
      const __nv_bfloat162* we = reinterpret_cast<const __nv_bfloat162*>(&wv);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 fx = __bfloat1622float2(xe[j]);
        const float2 fw = __bfloat1622float2(we[j]);
        xe[j] = __floats2bfloat162_rn((fx.x * r) * fw.x, (fx.y * r) * fw.y);
      }
      hs[b * nchunk + c] = xv;
    }
    __syncthreads();  // red / tot_s reused by the next row; hs complete
  }
}

// Host: the RMSNorm forward kernel's row layout for a bf16 row of K
// elements (the same rms_row_split call as rms_norm.cu's pick_cfg with
// backward = false): `nv` 16-byte vectors on each of `tpr` threads.  False
// when that kernel takes its scalar path for such a row (then there is
// nothing to mirror).
inline bool rms_row_layout(int64_t K, int* tpr, int* nv) {
  if (K % 8 != 0) return false;
  return rms_row_split(K / 8, rms_one_vec_limit(2, /*backward=*/false), nv, tpr);
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
