// Fused linear cross-entropy (FLCE) on sm_100a.
//
// Same result as the reference's _FusedLinearCrossEntropyFunction
// (ops/fused_linear_cross_entropy.py:82-185): loss = sum over non-ignored
// rows of (lse - logit[label]) / max(#non-ignored, 1), dX = P W, dW = P^T h
// with P = (softmax - onehot) * mask / max(#non-ignored, 1); the bias gets no
// gradient.  The reference walks the VOCAB in chunks twice (forward for the
// online max/sum-exp, backward recomputing every logit chunk: 8*H*V FLOPs per
// token).  Here the TOKENS are chunked and every logit is computed once:
//
//   per token chunk c (rows [r0, r0+C)):
//     1. logits GEMM (tcgen05, 128x256 tiles) with a fused epilogue that
//        writes E = exp(logit - tile_max) in bf16, the per-(row, vocab tile)
//        (max, sum E), and the target logit picked when the label falls in
//        the tile — the [C, V] fp32 logits never exist;
//     2. flce_lse: merge the tile partials into lse, the per-row loss, and a
//        per-(row, tile) factor f = exp(tile_max - lse) * mask / n_valid;
//     3. flce_transform: P = E * f - onehot * mask / n_valid, in place (bf16);
//     4. dX slabs (+)= P W      (tcgen05, split-K slabs, fp32),
//        dW      (+)= P^T h_c  (tcgen05, both operands MN-major, fp32).
//   loss = sum(row_loss) / max(n_valid, 1)   (fixed-order reduction)
//
// The gradients are therefore produced in the forward at grad_output = 1;
// ml_flce_backward multiplies them by the real grad_output and casts, which
// is exact because they are linear in it.  6*H*V FLOPs per token in total.
#include "gemm.cuh"
#include "p2p.cuh"

#include <algorithm>

namespace ml {
namespace flce {
namespace {

constexpr int kTileV = 256;  // vocab columns per logits tile (GEMM BN)

inline size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

struct Layout {
  int64_t chunk = 0, ldE = 0, n_tiles = 0;
  size_t off_E = 0, off_pm = 0, off_ps = 0, off_tgt = 0, off_rowloss = 0, off_cnt = 0, total = 0;
};

Layout layout(int64_t n, int64_t v, int64_t chunk) {
  Layout L;
  L.chunk = std::max<int64_t>(1, std::min(chunk, n));
  L.ldE = (v + 7) / 8 * 8;
  L.n_tiles = (v + kTileV - 1) / kTileV;
  size_t off = 0;
  L.off_E = off;
  off = align256(off + (size_t)L.chunk * L.ldE * 2);
  L.off_pm = off;
  off = align256(off + (size_t)L.n_tiles * L.chunk * 4);
  L.off_ps = off;
  off = align256(off + (size_t)L.n_tiles * L.chunk * 4);
  L.off_tgt = off;
  off = align256(off + (size_t)L.chunk * 4);
  L.off_rowloss = off;
  off = align256(off + (size_t)n * 4);
  L.off_cnt = off;
  off = align256(off + 16);
  L.total = off;
  return L;
}

// Split-K slabs for the dX GEMM.  Its (m, n) tiles are few (rows/256 x h/256
// on the CTA-pair kernel), so their last wave over the SM pairs can be mostly
// empty (8192 x 2048: 256 tiles on 74 pairs = 3.46 waves, 86% busy).  Pick the
// split count (1..4) whose units fill whole waves best; a split is taken only
// if it gains more than 2% of wave efficiency.
int dx_slabs(int64_t chunk_rows, int64_t h, int64_t v) {
  const int64_t kb = (v + 63) / 64;
  if (kb < 64) return 1;
  const int64_t tiles = ((chunk_rows + 255) / 256) * ((h + 255) / 256);
  const int64_t slots = std::max(1, num_sms() / 2);
  auto eff = [&](int64_t s) {
    const int64_t units = tiles * s;
    const int64_t waves = (units + slots - 1) / slots;
    return (double)units / (double)(waves * slots);
  };
  int64_t best = 1;
  double best_eff = eff(1);
  for (int64_t s = 2; s <= 4 && s <= kb / 32; ++s) {
    if (eff(s) > best_eff + 0.02) {
      best = s;
      best_eff = eff(s);
    }
  }
  // the split count gemm::launch will actually use for this request
  const int64_t per = (kb + best - 1) / best;
  return (int)((kb + per - 1) / per);
}

// n_valid = #(labels != ignore), stored as float; cnt[1] = 1 / max(n_valid, 1).
__global__ void __launch_bounds__(1024)
flce_count(const int64_t* __restrict__ labels, int64_t n, int64_t ignore, float* cnt) {
  __shared__ unsigned long long part[32];
  unsigned long long c = 0;
  for (int64_t i = threadIdx.x; i < n; i += blockDim.x) c += labels[i] != ignore ? 1ull : 0ull;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) c += __shfl_xor_sync(0xffffffffu, c, o);
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = c;
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned long long t = 0;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) t += part[w];
    cnt[0] = (float)t;
    cnt[1] = 1.f / fmaxf((float)t, 1.f);
  }
}

// Per row of the chunk: merge (tile max, tile sum) into lse; row loss; and
// f[t][r] = exp(m_t - lse) * mask * scale written over part_m.
// Block = 32 rows x 8 tile-lanes: reads are coalesced across rows.
__global__ void __launch_bounds__(256)
flce_lse(float* __restrict__ part_m, const float* __restrict__ part_s,
         const float* __restrict__ tgt, const int64_t* __restrict__ labels, int64_t rows,
         int64_t n_tiles, int64_t ignore, const float* __restrict__ cnt,
         float* __restrict__ row_loss, float* __restrict__ lse_out) {
  __shared__ float sm[8][33], ss[8][33], s_lse[32];
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  const int64_t r = (int64_t)blockIdx.x * 32 + tx;
  float M = -INFINITY, S = 0.f;
  if (r < rows) {
    for (int64_t t = ty; t < n_tiles; t += 8) {
      const float m = part_m[t * rows + r];
      const float s = part_s[t * rows + r];
      if (m > M) {
        S = S * __expf(M - m) + s;
        M = m;
      } else {
        S += s * __expf(m - M);
      }
    }
  }
  sm[ty][tx] = M;
  ss[ty][tx] = S;
  __syncthreads();
  if (ty == 0) {
    float MM = -INFINITY, SS = 0.f;
    for (int k = 0; k < 8; ++k) {  // fixed order
      const float m = sm[k][tx], s = ss[k][tx];
      if (s == 0.f) continue;
      if (m > MM) {
        SS = SS * __expf(MM - m) + s;
        MM = m;
      } else {
        SS += s * __expf(m - MM);
      }
    }
    const float lse = MM + __logf(SS);
    s_lse[tx] = lse;
    if (r < rows) {
      const bool valid = labels[r] != ignore;
      row_loss[r] = valid ? (lse - tgt[r]) : 0.f;
      if (lse_out) lse_out[r] = lse;
    }
  }
  __syncthreads();
  if (r < rows) {
    const float lse = s_lse[tx];
    const float scale = labels[r] != ignore ? cnt[1] : 0.f;
    for (int64_t t = ty; t < n_tiles; t += 8) {
      const float m = part_m[t * rows + r];
      part_m[t * rows + r] = __expf(m - lse) * scale;
    }
  }
}

// P = E * f[tile][row] - onehot(label) * scale, in place, 8 bf16 per step.
// Column c of E holds vocabulary id label_base + c.
__global__ void __launch_bounds__(256)
flce_transform(__nv_bfloat16* __restrict__ E, int64_t ldE, int64_t rows, int64_t vocab,
               const float* __restrict__ f, const int64_t* __restrict__ labels, int64_t ignore,
               const float* __restrict__ scale_ptr, int64_t label_base) {
  // Rows over blocks (grid-stride), 16-byte vectors of a row over threads, 4
  // vectors in flight per thread: no per-element index division, one label
  // and scale per row, one tile factor per 32 vectors (from L1).
  constexpr int U = 4;
  const int64_t vpr = (vocab + 7) / 8;  // vectors per row
  const float scale = scale_ptr[0];
  for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
    const int64_t lab0 = labels[r];
    const float sub = lab0 != ignore ? scale : 0.f;
    const int64_t lab = lab0 != ignore ? lab0 - label_base : (int64_t)-1;
    __nv_bfloat16* row = E + r * ldE;
    for (int64_t base = threadIdx.x; base < vpr; base += (int64_t)blockDim.x * U) {
      Vec16<__nv_bfloat16> v[U];
      float fr[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int64_t vi = base + (int64_t)u * blockDim.x;
        if (vi < vpr && vi * 8 + 8 <= vocab) {
          v[u] = *reinterpret_cast<const Vec16<__nv_bfloat16>*>(row + vi * 8);
          fr[u] = f[((vi * 8) / kTileV) * rows + r];
        }
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int64_t vi = base + (int64_t)u * blockDim.x;
        if (vi >= vpr) continue;
        const int64_t c0 = vi * 8;
        if (c0 + 8 <= vocab) {
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            float x = __bfloat162float(v[u].v[j]) * fr[u];
            if (lab == c0 + j) x -= sub;
            v[u].v[j] = __float2bfloat16_rn(x);
          }
          *reinterpret_cast<Vec16<__nv_bfloat16>*>(row + c0) = v[u];
        } else {  // ragged last vector of the row
          const float fl = f[(c0 / kTileV) * rows + r];
          for (int j = 0; c0 + j < vocab; ++j) {
            float x = __bfloat162float(row[c0 + j]) * fl;
            if (lab == c0 + j) x -= sub;
            row[c0 + j] = __float2bfloat16_rn(x);
          }
        }
      }
    }
  }
}

// Vocabulary-sharded path, phase 1: merge this shard's tile partials into a
// per-row (max, sum exp(logit - max)).  Block = 32 rows x 8 tile-lanes.
__global__ void __launch_bounds__(256)
flce_merge_tiles(const float* __restrict__ part_m, const float* __restrict__ part_s,
                 int64_t rows, int64_t n_tiles, float* __restrict__ row_m,
                 float* __restrict__ row_s) {
  __shared__ float sm[8][33], ss[8][33];
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  const int64_t r = (int64_t)blockIdx.x * 32 + tx;
  float M = -INFINITY, S = 0.f;
  if (r < rows) {
    for (int64_t t = ty; t < n_tiles; t += 8) {
      const float m = part_m[t * rows + r];
      const float s = part_s[t * rows + r];
      if (m > M) {
        S = S * __expf(M - m) + s;
        M = m;
      } else {
        S += s * __expf(m - M);
      }
    }
  }
  sm[ty][tx] = M;
  ss[ty][tx] = S;
  __syncthreads();
  if (ty == 0 && r < rows) {
    float MM = -INFINITY, SS = 0.f;
    for (int k = 0; k < 8; ++k) {
      const float m = sm[k][tx], s = ss[k][tx];
      if (s == 0.f) continue;
      if (m > MM) {
        SS = SS * __expf(MM - m) + s;
        MM = m;
      } else {
        SS += s * __expf(m - MM);
      }
    }
    row_m[r] = MM;
    row_s[r] = SS;
  }
}

// Vocabulary-sharded path, phase 2: f[t][r] = exp(m_t - lse_r) * mask * scale,
// written over part_m, from the GLOBAL per-row log-sum-exp.
__global__ void __launch_bounds__(256)
flce_factors(float* __restrict__ part_m, int64_t rows, int64_t n_tiles,
             const float* __restrict__ lse, const int64_t* __restrict__ labels, int64_t ignore,
             const float* __restrict__ scale_ptr) {
  const int64_t total = rows * n_tiles;
  const float scale = scale_ptr[0];
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i % rows;
    const float sc = labels[r] != ignore ? scale : 0.f;
    part_m[i] = __expf(part_m[i] - lse[r]) * sc;
  }
}

// loss = sum(row_loss) / max(n_valid, 1); one CTA, fixed order.
__global__ void __launch_bounds__(1024)
flce_loss(const float* __restrict__ row_loss, int64_t n, const float* __restrict__ cnt,
          float* __restrict__ loss) {
  __shared__ float part[32];
  float s = 0.f;
  for (int64_t i = threadIdx.x; i < n; i += blockDim.x) s += row_loss[i];
  s = warp_sum(s);
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) t += part[w];
    loss[0] = t * cnt[1];
  }
}

// dst[i] = cast(g * sum_s src[s][i]) for i < n.
template <typename T>
__global__ void __launch_bounds__(256)
scale_cast(const float* __restrict__ src, int slabs, int64_t slab_stride, int64_t n,
           const float* __restrict__ g, T* __restrict__ dst) {
  const float gv = g != nullptr ? g[0] : 1.f;
  const int64_t nv = n / 4;
  const bool vec = (reinterpret_cast<uintptr_t>(src) & 15) == 0 && (slab_stride & 3) == 0;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < (vec ? nv : n);
       i += (int64_t)gridDim.x * blockDim.x) {
    if (vec) {
      float4 a = __ldcs(reinterpret_cast<const float4*>(src) + i);
      for (int s = 1; s < slabs; ++s) {
        const float4 b = __ldcs(reinterpret_cast<const float4*>(src + s * slab_stride) + i);
        a.x += b.x;
        a.y += b.y;
        a.z += b.z;
        a.w += b.w;
      }
      dst[4 * i + 0] = from_f32<T>(a.x * gv);
      dst[4 * i + 1] = from_f32<T>(a.y * gv);
      dst[4 * i + 2] = from_f32<T>(a.z * gv);
      dst[4 * i + 3] = from_f32<T>(a.w * gv);
    } else {
      float a = src[i];
      for (int s = 1; s < slabs; ++s) a += src[s * slab_stride + i];
      dst[i] = from_f32<T>(a * gv);
    }
  }
  if (vec) {
    for (int64_t i = nv * 4 + (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x) {
      float a = src[i];
      for (int s = 1; s < slabs; ++s) a += src[s * slab_stride + i];
      dst[i] = from_f32<T>(a * gv);
    }
  }
}

int launch_scale_cast(const float* src, int slabs, int64_t stride, int64_t n, const float* g,
                      void* dst, int dtype, cudaStream_t st) {
  if (n == 0) return ML_OK;
  const int grid = (int)std::min<int64_t>((n / 4 + 255) / 256 + 1, (int64_t)num_sms() * 8);
  switch (dtype) {
    case ML_DTYPE_F32:
      scale_cast<float><<<grid, 256, 0, st>>>(src, slabs, stride, n, g, static_cast<float*>(dst));
      break;
    case ML_DTYPE_BF16:
      scale_cast<__nv_bfloat16><<<grid, 256, 0, st>>>(src, slabs, stride, n, g,
                                                      static_cast<__nv_bfloat16*>(dst));
      break;
    case ML_DTYPE_F16:
      scale_cast<__half><<<grid, 256, 0, st>>>(src, slabs, stride, n, g, static_cast<__half*>(dst));
      break;
    default:
      set_error("flce: bad output dtype %d", dtype);
      return ML_ERR_INVALID_ARG;
  }
  ML_CHECK_LAUNCH("flce scale_cast");
  return ML_OK;
}

}  // namespace
}  // namespace flce
}  // namespace ml

using namespace ml;

extern "C" int ml_flce_dx_slabs(int64_t n, int64_t h, int64_t v, int64_t chunk_tokens) {
  if (n <= 0 || h <= 0 || v <= 0) return 1;
  const int64_t chunk = std::max<int64_t>(1, std::min(chunk_tokens > 0 ? chunk_tokens : n, n));
  return flce::dx_slabs(chunk, h, v);
}

extern "C" size_t ml_flce_workspace_bytes(int64_t n, int64_t h, int64_t v, int64_t chunk_tokens) {
  (void)h;
  if (n <= 0 || v <= 0) return 256;
  return flce::layout(n, v, chunk_tokens > 0 ? chunk_tokens : n).total;
}

extern "C" int ml_flce_forward(const void* hidden, const void* weight, const void* bias,
                               int bias_dtype, const int64_t* labels, int64_t n, int64_t h,
                               int64_t v, int64_t ignore_index, int64_t chunk_tokens, float* loss,
                               float* lse, float* dx_slabs, float* dw_acc, void* workspace,
                               size_t workspace_bytes, void* stream) {
  ML_CHECK_ARG(n >= 0 && h > 0 && v > 0, "flce_forward: bad sizes n=%lld h=%lld v=%lld",
               (long long)n, (long long)h, (long long)v);
  ML_CHECK_ARG(h % 8 == 0, "flce_forward: hidden size must be a multiple of 8 (TMA row pitch)");
  ML_CHECK_ARG(loss != nullptr, "flce_forward: null loss");
  ML_CHECK_ARG(bias == nullptr || (bias_dtype >= 0 && bias_dtype <= 2), "flce_forward: bias dtype");
  ML_CHECK_ARG(v < (int64_t)1 << 31 && n < (int64_t)1 << 31, "flce_forward: sizes too large");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (n == 0) {
    ML_CHECK_CUDA(cudaMemsetAsync(loss, 0, sizeof(float), st), "flce_forward: memset");
    if (dw_acc) ML_CHECK_CUDA(cudaMemsetAsync(dw_acc, 0, (size_t)v * h * 4, st), "memset dW");
    return ML_OK;
  }
  ML_CHECK_ARG(hidden && weight && labels, "flce_forward: null input");
  const int64_t chunk = chunk_tokens > 0 ? chunk_tokens : n;
  const flce::Layout L = flce::layout(n, v, chunk);
  ML_CHECK_ARG(workspace != nullptr && ((uintptr_t)workspace & 255) == 0,
               "flce_forward: workspace must be 256-byte aligned");
  ML_CHECK_ARG(workspace_bytes >= L.total, "flce_forward: workspace too small (%zu < %zu)",
               workspace_bytes, L.total);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  __nv_bfloat16* E = reinterpret_cast<__nv_bfloat16*>(ws + L.off_E);
  float* pm = reinterpret_cast<float*>(ws + L.off_pm);
  float* ps = reinterpret_cast<float*>(ws + L.off_ps);
  float* tgt = reinterpret_cast<float*>(ws + L.off_tgt);
  float* row_loss = reinterpret_cast<float*>(ws + L.off_rowloss);
  float* cnt = reinterpret_cast<float*>(ws + L.off_cnt);
  const int slabs = flce::dx_slabs(L.chunk, h, v);

  flce::flce_count<<<1, 1024, 0, st>>>(labels, n, ignore_index, cnt);
  ML_CHECK_LAUNCH("flce_count");

  const __nv_bfloat16* hid = static_cast<const __nv_bfloat16*>(hidden);
  for (int64_t r0 = 0; r0 < n; r0 += L.chunk) {
    const int64_t rows = std::min(L.chunk, n - r0);
    ML_CHECK_CUDA(cudaMemsetAsync(tgt, 0, (size_t)rows * 4, st), "flce: memset tgt");
    // 1. logits GEMM + softmax-partials epilogue
    gemm::Problem g1;
    g1.M = rows;
    g1.N = v;
    g1.nseg = 1;
    g1.seg[0].a = {hid + r0 * h, rows, h, h};
    g1.seg[0].b = {weight, v, h, h};
    g1.seg[0].K = h;
    g1.epi = gemm::EPI_FLCE;
    g1.bn = 256;
    g1.D = E;
    g1.ldd = L.ldE;
    g1.labels = labels + r0;
    g1.ignore_index = ignore_index;
    g1.part_m = pm;
    g1.part_s = ps;
    g1.tgt = tgt;
    g1.bias = bias;
    g1.bias_dtype = bias_dtype;
    g1.raster = 0;  // M-tiles fastest: each W tile is read from HBM once
    int rc = gemm::launch(g1, st);
    if (rc) return rc;
    // 2. lse, row loss, per-(row, tile) factors
    flce::flce_lse<<<(unsigned)((rows + 31) / 32), 256, 0, st>>>(
        pm, ps, tgt, labels + r0, rows, L.n_tiles, ignore_index, cnt, row_loss + r0,
        lse ? lse + r0 : nullptr);
    ML_CHECK_LAUNCH("flce_lse");
    if (dx_slabs == nullptr && dw_acc == nullptr) continue;
    // 3. P = softmax - onehot (scaled), in place
    {
      const int grid = (int)std::min<int64_t>(rows, (int64_t)1 << 20);  // a row per block
      flce::flce_transform<<<grid, 256, 0, st>>>(E, L.ldE, rows, v, pm, labels + r0,
                                                 ignore_index, cnt + 1, 0);
      ML_CHECK_LAUNCH("flce_transform");
    }
    // 4a. dX slabs = P W  (A = P [rows, V] K-major, B = W stored [V, H]: N-major)
    if (dx_slabs != nullptr) {
      gemm::Problem g2;
      g2.M = rows;
      g2.N = h;
      g2.nseg = 1;
      g2.seg[0].a = {E, rows, v, L.ldE};
      g2.seg[0].b = {weight, v, h, h};
      g2.seg[0].K = v;
      g2.b_mn = true;
      g2.epi = gemm::EPI_PARTIAL;
      g2.splits = slabs;
      g2.D = dx_slabs + r0 * h;
      g2.ldd = h;
      g2.split_stride = n * h;
      g2.raster = 1;
      rc = gemm::launch(g2, st);
      if (rc) return rc;
    }
    // 4b. dW (+)= P^T h_c  (A = P stored [rows, V]: M-major; B = h_c stored [rows, H]: N-major)
    if (dw_acc != nullptr) {
      gemm::Problem g3;
      g3.M = v;
      g3.N = h;
      g3.nseg = 1;
      g3.seg[0].a = {E, rows, v, L.ldE};
      g3.seg[0].b = {hid + r0 * h, rows, h, h};
      g3.seg[0].K = rows;
      g3.a_mn = true;
      g3.b_mn = true;
      g3.epi = gemm::EPI_STORE;
      g3.d_f32 = true;
      g3.D = dw_acc;
      g3.ldd = h;
      g3.beta = r0 > 0 ? 1.f : 0.f;
      g3.raster = 1;
      rc = gemm::launch(g3, st);
      if (rc) return rc;
    }
  }
  flce::flce_loss<<<1, 1024, 0, st>>>(row_loss, n, cnt, loss);
  ML_CHECK_LAUNCH("flce_loss");
  return ML_OK;
}

extern "C" int ml_flce_backward(const float* grad_output, const float* dx_slabs, int slabs,
                                void* dhidden, int dh_dtype, int64_t n, int64_t h,
                                const float* dw_acc, void* dweight, int dw_dtype, int64_t v,
                                void* stream) {
  ML_CHECK_ARG(n >= 0 && h > 0 && v >= 0, "flce_backward: bad sizes");
  ML_CHECK_ARG(slabs >= 1 && slabs <= 16, "flce_backward: bad slab count %d", slabs);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (dhidden != nullptr) {
    ML_CHECK_ARG(dx_slabs != nullptr, "flce_backward: dhidden requested without dx_slabs");
    int rc = flce::launch_scale_cast(dx_slabs, slabs, n * h, n * h, grad_output, dhidden,
                                     dh_dtype, st);
    if (rc) return rc;
  }
  if (dweight != nullptr) {
    ML_CHECK_ARG(dw_acc != nullptr, "flce_backward: dweight requested without dw_acc");
    int rc = flce::launch_scale_cast(dw_acc, 1, 0, v * h, grad_output, dweight, dw_dtype, st);
    if (rc) return rc;
  }
  return ML_OK;
}

extern "C" int ml_flce_count_valid(const int64_t* labels, int64_t n, int64_t ignore_index,
                                   float* out, void* stream) {
  ML_CHECK_ARG(n >= 0 && out != nullptr && (n == 0 || labels != nullptr),
               "flce_count_valid: bad arguments");
  flce::flce_count<<<1, 1024, 0, static_cast<cudaStream_t>(stream)>>>(labels, n, ignore_index,
                                                                      out);
  ML_CHECK_LAUNCH("flce_count_valid");
  return ML_OK;
}

namespace ml {
namespace flce {
// dW [v_local, h] (+)= P^T hidden for a (softmax - onehot) * scale chunk P
// held in the workspace (both operands read in place: MN-major).
int shard_dw_gemm(const void* hidden, const __nv_bfloat16* E, int64_t ldE, int64_t rows,
                  int64_t h, int64_t v_local, float* dw, int dw_accumulate, cudaStream_t st) {
  gemm::Problem g3;
  g3.M = v_local;
  g3.N = h;
  g3.nseg = 1;
  g3.seg[0].a = {E, rows, v_local, ldE};
  g3.seg[0].b = {hidden, rows, h, h};
  g3.seg[0].K = rows;
  g3.a_mn = true;
  g3.b_mn = true;
  g3.epi = gemm::EPI_STORE;
  g3.d_f32 = true;
  g3.D = dw;
  g3.ldd = h;
  g3.beta = dw_accumulate ? 1.f : 0.f;
  g3.raster = 1;
  return gemm::launch(g3, st);
}
}  // namespace flce
}  // namespace ml

extern "C" size_t ml_flce_shard_workspace_bytes(int64_t rows, int64_t v_local) {
  if (rows <= 0 || v_local <= 0) return 256;
  return flce::layout(rows, v_local, rows).total;
}

extern "C" int ml_flce_shard_stats(const void* hidden, const void* weight, const void* bias,
                                   int bias_dtype, const int64_t* labels, int64_t rows, int64_t h,
                                   int64_t v_local, int64_t vocab_offset, int64_t ignore_index,
                                   float* row_max, float* row_sum, float* row_tgt,
                                   void* workspace, size_t workspace_bytes, void* stream) {
  ML_CHECK_ARG(rows > 0 && h > 0 && v_local > 0 && vocab_offset >= 0,
               "flce_shard_stats: bad sizes");
  ML_CHECK_ARG(h % 8 == 0, "flce_shard_stats: hidden size must be a multiple of 8");
  ML_CHECK_ARG(hidden && weight && labels && row_max && row_sum && row_tgt,
               "flce_shard_stats: null pointer");
  const flce::Layout L = flce::layout(rows, v_local, rows);
  ML_CHECK_ARG(workspace != nullptr && ((uintptr_t)workspace & 255) == 0 &&
                   workspace_bytes >= L.total,
               "flce_shard_stats: workspace must be 256-byte aligned and >= %zu bytes", L.total);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  float* pm = reinterpret_cast<float*>(ws + L.off_pm);
  float* ps = reinterpret_cast<float*>(ws + L.off_ps);
  ML_CHECK_CUDA(cudaMemsetAsync(row_tgt, 0, (size_t)rows * 4, st), "flce_shard_stats: memset");
  gemm::Problem g1;
  g1.M = rows;
  g1.N = v_local;
  g1.nseg = 1;
  g1.seg[0].a = {hidden, rows, h, h};
  g1.seg[0].b = {weight, v_local, h, h};
  g1.seg[0].K = h;
  g1.epi = gemm::EPI_FLCE;
  g1.bn = 256;
  g1.D = ws + L.off_E;
  g1.ldd = L.ldE;
  g1.labels = labels;
  g1.label_base = vocab_offset;
  g1.ignore_index = ignore_index;
  g1.part_m = pm;
  g1.part_s = ps;
  g1.tgt = row_tgt;
  g1.bias = bias;
  g1.bias_dtype = bias_dtype;
  int rc = gemm::launch(g1, st);
  if (rc) return rc;
  flce::flce_merge_tiles<<<(unsigned)((rows + 31) / 32), 256, 0, st>>>(pm, ps, rows, L.n_tiles,
                                                                       row_max, row_sum);
  ML_CHECK_LAUNCH("flce_merge_tiles");
  return ML_OK;
}

extern "C" int ml_flce_shard_grads(const void* hidden, const void* weight, const int64_t* labels,
                                   int64_t rows, int64_t h, int64_t v_local, int64_t vocab_offset,
                                   int64_t ignore_index, const float* lse, const float* scale,
                                   float* dx, float* dw, int dw_accumulate, void* workspace,
                                   size_t workspace_bytes, void* stream) {
  ML_CHECK_ARG(rows > 0 && h > 0 && v_local > 0 && vocab_offset >= 0,
               "flce_shard_grads: bad sizes");
  ML_CHECK_ARG(hidden && weight && labels && lse && scale, "flce_shard_grads: null pointer");
  const flce::Layout L = flce::layout(rows, v_local, rows);
  ML_CHECK_ARG(workspace != nullptr && ((uintptr_t)workspace & 255) == 0 &&
                   workspace_bytes >= L.total,
               "flce_shard_grads: workspace must be 256-byte aligned and >= %zu bytes", L.total);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  __nv_bfloat16* E = reinterpret_cast<__nv_bfloat16*>(ws + L.off_E);
  float* pm = reinterpret_cast<float*>(ws + L.off_pm);
  {
    const int64_t total = rows * L.n_tiles;
    const int grid = (int)std::min<int64_t>((total + 255) / 256, (int64_t)num_sms() * 8);
    flce::flce_factors<<<grid, 256, 0, st>>>(pm, rows, L.n_tiles, lse, labels, ignore_index,
                                             scale);
    ML_CHECK_LAUNCH("flce_factors");
  }
  {
    const int grid = (int)std::min<int64_t>(rows, (int64_t)1 << 20);  // a row per block
    flce::flce_transform<<<grid, 256, 0, st>>>(E, L.ldE, rows, v_local, pm, labels, ignore_index,
                                               scale, vocab_offset);
    ML_CHECK_LAUNCH("flce_transform");
  }
  if (dx != nullptr) {
    gemm::Problem g2;
    g2.M = rows;
    g2.N = h;
    g2.nseg = 1;
    g2.seg[0].a = {E, rows, v_local, L.ldE};
    g2.seg[0].b = {weight, v_local, h, h};
    g2.seg[0].K = v_local;
    g2.b_mn = true;
    g2.epi = gemm::EPI_STORE;
    g2.d_f32 = true;
    g2.D = dx;
    g2.ldd = h;
    g2.raster = 1;
    int rc = gemm::launch(g2, st);
    if (rc) return rc;
  }
  if (dw != nullptr) return flce::shard_dw_gemm(hidden, E, L.ldE, rows, h, v_local, dw,
                                                 dw_accumulate, st);
  return ML_OK;
}

extern "C" int ml_flce_shard_grads_dw(const void* hidden, int64_t rows, int64_t h,
                                      int64_t v_local, float* dw, int dw_accumulate,
                                      void* workspace, size_t workspace_bytes, void* stream) {
  ML_CHECK_ARG(rows > 0 && h > 0 && v_local > 0, "flce_shard_grads_dw: bad sizes");
  ML_CHECK_ARG(hidden && dw, "flce_shard_grads_dw: null pointer");
  const flce::Layout L = flce::layout(rows, v_local, rows);
  ML_CHECK_ARG(workspace != nullptr && ((uintptr_t)workspace & 255) == 0 &&
                   workspace_bytes >= L.total,
               "flce_shard_grads_dw: workspace must be 256-byte aligned and >= %zu bytes",
               L.total);
  const __nv_bfloat16* E =
      reinterpret_cast<const __nv_bfloat16*>(static_cast<uint8_t*>(workspace) + L.off_E);
  return flce::shard_dw_gemm(hidden, E, L.ldE, rows, h, v_local, dw, dw_accumulate,
                             static_cast<cudaStream_t>(stream));
}

// Vocabulary-parallel dX through peer memory: dX = P W of this rank's shard
// (P: the transformed exponentials that ml_flce_shard_grads left in the
// shard workspace, rows x v_local), every output tile stored by the GEMM's
// epilogue straight into its row owner's receive slot for this rank
// (p2p.cu); then this rank's arrive flag is raised on every rank.  Followed
// by ml_flce_p2p_reduce and ml_flce_p2p_finish with the same epoch.
extern "C" int ml_flce_shard_dx_p2p(const void* weight, int64_t rows, int64_t h, int64_t v_local,
                                    const void* shard_ws, size_t shard_ws_bytes, int64_t chunk_cap,
                                    int world, int rank, void* const* peer_ws, int64_t epoch,
                                    void* stream) {
  ML_CHECK_ARG(weight && shard_ws, "flce_shard_dx_p2p: null pointer");
  ML_CHECK_ARG(rows > 0 && rows <= chunk_cap && h > 0 && h % 8 == 0 && v_local > 0 && epoch > 0,
               "flce_shard_dx_p2p: bad sizes (rows %lld, chunk %lld, h %lld)", (long long)rows,
               (long long)chunk_cap, (long long)h);
  const flce::Layout L = flce::layout(rows, v_local, rows);
  ML_CHECK_ARG(((uintptr_t)shard_ws & 255) == 0 && shard_ws_bytes >= L.total,
               "flce_shard_dx_p2p: shard workspace must be 256-byte aligned and >= %zu bytes",
               L.total);
  p2p::Peers pe;
  if (int rc = p2p::check_peers(world, rank, peer_ws, pe)) return rc;
  const p2p::XLayout X = p2p::xlayout(world, chunk_cap, h);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const __nv_bfloat16* E =
      reinterpret_cast<const __nv_bfloat16*>(static_cast<const uint8_t*>(shard_ws) + L.off_E);
  gemm::Problem g;
  g.M = rows;
  g.N = h;
  g.nseg = 1;
  g.seg[0].a = {E, rows, v_local, L.ldE};
  g.seg[0].b = {weight, v_local, h, h};
  g.seg[0].K = v_local;
  g.b_mn = true;
  g.epi = gemm::EPI_STORE;
  g.d_f32 = true;
  g.ldd = h;
  g.raster = 1;
  g.peer_n = world;
  g.peer_me = rank;
  g.peer_rows = X.rows_per_owner;
  for (int r = 0; r < world; ++r)
    g.peer_dst[r] = reinterpret_cast<float*>(pe.ws[r] + X.off_recv);
  if (int rc = gemm::launch(g, st)) return rc;
  return p2p::launch_signal(pe, world, rank, 0, epoch, st);
}
