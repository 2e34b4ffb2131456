// Decode-step attention for the static-KV generator: one query token per
// sequence against the first `len` positions of the static KV cache, with
// grouped-query heads read in place (no repeat_kv copies) and the length read
// from device memory (the captured decode step advances it), so the step
// needs no mask.  Split-K over the keys ("flash decoding"): each warp takes
// 32 positions of one (sequence, kv head) for all G query heads of that group
// and writes their partials (max, sum-exp, unnormalised output); a second
// kernel merges the partials in order.  Caches of up to 256 positions run as
// one launch: a CTA per (sequence, kv head) keeps all its partials in shared
// memory and merges them itself, bitwise the two-kernel result; inside the
// generator's fused decoder layers that CTA also prepares its q, k and v rows
// first (decode_qk_attn_single), one launch for prep and attention.
//
// Math: o = sum_j softmax_j(scale * q.k_j) v_j with fp32 scores, exponents
// and accumulation over bf16 q, K, V — the computation of the reference's
// attention on one query row (transformers' SDPA path).
#include "common.cuh"

#include <cmath>

namespace ml {
namespace {

constexpr int kWarps = 4;      // warps per CTA
constexpr int kChunk = 32;     // key positions per warp (one per lane): one partial
constexpr int kMaxGroup = 16;  // query heads per kv head
constexpr int kMaxDim = 256;   // head dimension, a multiple of 32
constexpr int kMaxGD = 32;     // G * D / 32: output registers per lane

struct DecodeArgs {
  const __nv_bfloat16* q;  // [B, Hq, 1, D] at strides (sq_b, sq_h), D contiguous
  const __nv_bfloat16* k;  // [B, Hkv, L, D] contiguous
  const __nv_bfloat16* v;
  const int64_t* pos;      // device: valid keys = *pos + len_offset
  int64_t len_offset;
  int64_t sq_b, sq_h;
  int B, Hq, Hkv, L, D;
  float scale;
  float* part_m;           // [nchunk][B * Hq]
  float* part_l;           // [nchunk][B * Hq]
  float* part_o;           // [nchunk][B * Hq][D]
  __nv_bfloat16* out;      // [B, 1, Hq, D]
};

// One warp = one partial over 32 key positions (a position per lane) for
// every query head of one (sequence, kv head): the lane loads its whole K row
// (all 16-byte loads issued before use) and forms the G scores; per head the
// warp takes max / sum-exp with shuffles; then P.V walks the 32 positions
// with the V row read coalesced (a lane owns DPL = D/32 output dimensions of
// every head) and the probabilities broadcast by shuffle.  G and DPL are
// template parameters so every per-lane array stays in registers.
//
// The partial of slot c goes to pm / pl [c * stride + row0 + g] and po
// [(c * stride + row0 + g) * D + d]: the global workspace (two-kernel path)
// or this CTA's shared memory (single-launch path).  Every thread of the CTA
// must call this (it loads q into `qs` behind a __syncthreads).
template <int G, int DPL, bool kQReady = false>
__device__ __forceinline__ void attn_partial(const DecodeArgs& a, int c, float* qs, float* pm,
                                             float* pl, float* po, int64_t stride,
                                             int64_t row0) {
  constexpr int D = 32 * DPL;
  constexpr int NCH = D / 8;            // 16-byte chunks of a K row
  constexpr bool kPrefetchV = DPL <= 4;  // V fragments of all 32 positions in registers
  const int lane = threadIdx.x & 31;
  const int b = blockIdx.y / a.Hkv, kvh = blockIdx.y % a.Hkv;
  const int nslot = (a.L + kChunk - 1) / kChunk;
  const int64_t j0 = (int64_t)c * kChunk;
  const int64_t kv_base = ((int64_t)b * a.Hkv + kvh) * a.L * D;
  // K row and V fragments first: their addresses depend only on this warp's
  // slot, not on the filled length, so all loads of the step overlap.
  const int64_t j = j0 + lane;
  const bool in_cache = c < nslot && j < a.L;
  uint4 kv[NCH <= 16 ? NCH : 16];
  if (in_cache) {
    const uint4* krow = reinterpret_cast<const uint4*>(a.k + kv_base + j * D);
#pragma unroll
    for (int u = 0; u < (NCH <= 16 ? NCH : 16); ++u) kv[u] = krow[u];
  }
  __nv_bfloat162 vfrag[kPrefetchV ? kChunk : 1][DPL / 2];
  if constexpr (kPrefetchV) {
    if (c < nslot) {
      const __nv_bfloat16* vbase = a.v + kv_base + j0 * D + lane * DPL;
#pragma unroll
      for (int kk = 0; kk < kChunk; ++kk)
        if (j0 + kk < a.L) {
#pragma unroll
          for (int e = 0; e < DPL / 2; ++e)
            vfrag[kk][e] = *reinterpret_cast<const __nv_bfloat162*>(vbase + (int64_t)kk * D + 2 * e);
        }
    }
  }
  const int64_t n = min((int64_t)a.L, *a.pos + a.len_offset);
  if (!kQReady) {  // else the caller has filled qs (and synchronised)
    for (int i = threadIdx.x; i < G * D; i += blockDim.x) {
      const int g = i / D, d = i - g * D;
      qs[i] = __bfloat162float(a.q[(int64_t)b * a.sq_b + (int64_t)(kvh * G + g) * a.sq_h + d]);
    }
  }
  __syncthreads();
  if (c >= nslot) return;  // warps past the last partial slot
  const int64_t slot0 = (int64_t)c * stride + row0;
  if (j0 >= n) {  // past the filled positions: empty partials
    if (lane < G) {
      pm[slot0 + lane] = -INFINITY;
      pl[slot0 + lane] = 0.f;
    }
    return;
  }
  const bool valid = j < n;
  float s[G];
#pragma unroll
  for (int g = 0; g < G; ++g) s[g] = 0.f;
  if (valid) {
    const uint4* krow = reinterpret_cast<const uint4*>(a.k + kv_base + j * D);
#pragma unroll
    for (int h0 = 0; h0 < NCH; h0 += 16) {
      constexpr int U = NCH < 16 ? NCH : 16;
      if (h0 > 0) {  // second half of a 256-wide row
#pragma unroll
        for (int u = 0; u < U; ++u) kv[u] = krow[h0 + u];
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const __nv_bfloat162* k2 = reinterpret_cast<const __nv_bfloat162*>(&kv[u]);
        const int d0 = (h0 + u) * 8;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 kf = __bfloat1622float2(k2[e]);
#pragma unroll
          for (int g = 0; g < G; ++g) {
            s[g] = fmaf(qs[g * D + d0 + 2 * e], kf.x, s[g]);
            s[g] = fmaf(qs[g * D + d0 + 2 * e + 1], kf.y, s[g]);
          }
        }
      }
    }
  }
  float p[G];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    const float sc = valid ? s[g] * a.scale : -INFINITY;
    const float m = warp_max(sc);
    p[g] = valid ? __expf(sc - m) : 0.f;
    const float l = warp_sum(p[g]);
    if (lane == 0) {
      pm[slot0 + g] = m;
      pl[slot0 + g] = l;
    }
  }
  float o[G][DPL];
#pragma unroll
  for (int g = 0; g < G; ++g)
#pragma unroll
    for (int e = 0; e < DPL; ++e) o[g][e] = 0.f;
  const int cnt = (int)min((int64_t)kChunk, n - j0);
  const __nv_bfloat16* vbase = a.v + kv_base + j0 * D + lane * DPL;
#pragma unroll
  for (int kk = 0; kk < kChunk; ++kk) {
    if (kk < cnt) {
      float vf[DPL];
#pragma unroll
      for (int e = 0; e < DPL / 2; ++e) {
        const float2 f = kPrefetchV
            ? __bfloat1622float2(vfrag[kPrefetchV ? kk : 0][e])
            : __bfloat1622float2(
                  *reinterpret_cast<const __nv_bfloat162*>(vbase + (int64_t)kk * D + 2 * e));
        vf[2 * e] = f.x;
        vf[2 * e + 1] = f.y;
      }
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const float pk = __shfl_sync(0xffffffffu, p[g], kk);
#pragma unroll
        for (int e = 0; e < DPL; ++e) o[g][e] = fmaf(pk, vf[e], o[g][e]);
      }
    }
  }
#pragma unroll
  for (int g = 0; g < G; ++g) {
    float* dst = po + (slot0 + g) * D + lane * DPL;
#pragma unroll
    for (int e = 0; e < DPL; ++e) dst[e] = o[g][e];
  }
}

template <int G, int DPL>
__global__ void __launch_bounds__(32 * kWarps)
decode_attn_chunk(const __grid_constant__ DecodeArgs a) {
  __shared__ float qs[G * 32 * DPL];
  const int b = blockIdx.y / a.Hkv, kvh = blockIdx.y % a.Hkv;
  const int c = blockIdx.x * kWarps + (threadIdx.x >> 5);  // partial index
  attn_partial<G, DPL>(a, c, qs, a.part_m, a.part_l, a.part_o, (int64_t)a.B * a.Hq,
                       (int64_t)b * a.Hq + kvh * G);
}

// out[b, 0, h, :] = sum_c e^(m_c - M) o_c / sum_c e^(m_c - M) l_c over the
// partials that hold keys (l_c > 0).  A warp per (b, h): lane c reads
// partial c's (m, l) (32 partials per pass), one warp max and one warp sum
// give M and the denominator, then each lane adds its D/32 output dimensions
// of every partial with the weights broadcast by shuffle (the partials'
// loads are independent, so they overlap).  Fixed order: deterministic.
// merge_row merges the partials of one row held at pm / pl / po (layout of
// attn_partial) into dst[lane * DPL ...]; one warp.
template <int DPL>
__device__ __forceinline__ void merge_row(const float* pm, const float* pl, const float* po,
                                          int64_t stride, int64_t row, int nchunk, int D,
                                          __nv_bfloat16* dst) {
  const int lane = threadIdx.x & 31;
  float M = -INFINITY;
  for (int c0 = 0; c0 < nchunk; c0 += 32) {
    const int c = c0 + lane;
    if (c < nchunk && pl[c * stride + row] > 0.f)
      M = fmaxf(M, pm[c * stride + row]);
  }
  M = warp_max(M);
  float L = 0.f;
  float o[DPL];
#pragma unroll
  for (int e = 0; e < DPL; ++e) o[e] = 0.f;
  for (int c0 = 0; c0 < nchunk; c0 += 32) {
    const int c = c0 + lane;
    float w = 0.f, wl = 0.f;
    if (c < nchunk) {
      const float l = pl[c * stride + row];
      if (l > 0.f) {
        w = __expf(pm[c * stride + row] - M);
        wl = w * l;
      }
    }
    L += warp_sum(wl);
    const int cn = min(32, nchunk - c0);
#pragma unroll 8
    for (int k = 0; k < 32; ++k) {
      if (k >= cn) break;
      const float wk = __shfl_sync(0xffffffffu, w, k);
      if (wk > 0.f) {
        const float* src = po + ((int64_t)(c0 + k) * stride + row) * D + lane * DPL;
#pragma unroll
        for (int e = 0; e < DPL; ++e) o[e] = fmaf(wk, src[e], o[e]);
      }
    }
  }
  const float inv = L > 0.f ? 1.f / L : 0.f;
  dst += lane * DPL;
#pragma unroll
  for (int e = 0; e < DPL; ++e) dst[e] = __float2bfloat16_rn(o[e] * inv);
}

template <int DPL>
__global__ void __launch_bounds__(256) decode_attn_merge(const __grid_constant__ DecodeArgs a,
                                                         int nchunk) {
  const int64_t row = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  if (row >= (int64_t)a.B * a.Hq) return;
  // rows are b * Hq + h, the layout of out [B, 1, Hq, D]
  merge_row<DPL>(a.part_m, a.part_l, a.part_o, (int64_t)a.B * a.Hq, row, nchunk, a.D,
                 a.out + row * a.D);
}

// Single launch for caches of up to kFusedSlots * 32 positions: one CTA per
// (sequence, kv head) holds every slot's partial in shared memory (a warp per
// slot, attn_partial) and its warps merge them (merge_row, a warp per query
// head of the group) — the two-kernel path's arithmetic in its order, so
// the output is bitwise the same, without the workspace round trip and the
// second launch.
constexpr int kFusedSlots = 8;

template <int G, int DPL>
__global__ void __launch_bounds__(32 * kFusedSlots)
decode_attn_single(const __grid_constant__ DecodeArgs a) {
  constexpr int D = 32 * DPL;
  __shared__ float qs[G * D];
  __shared__ float sm_m[kFusedSlots * G], sm_l[kFusedSlots * G];
  __shared__ float sm_o[kFusedSlots * G * D];
  const int warp = threadIdx.x >> 5;
  const int b = blockIdx.y / a.Hkv, kvh = blockIdx.y % a.Hkv;
  attn_partial<G, DPL>(a, warp, qs, sm_m, sm_l, sm_o, G, 0);
  __syncthreads();
  const int nslot = (a.L + kChunk - 1) / kChunk;  // <= kFusedSlots (host check)
  for (int g = warp; g < G; g += kFusedSlots) {
    const int64_t h = (int64_t)kvh * G + g;
    merge_row<DPL>(sm_m, sm_l, sm_o, G, g, nslot, D, a.out + ((int64_t)b * a.Hq + h) * D);
  }
}

// Decode-step q/k preparation for Qwen3-style attention, one warp per head
// row of the single new token: q and k rows get the per-head RMSNorm
// (y = bf16((x * rrms) * w), the fused RMSNorm's rounding) and then RoPE from
// the model's own cos/sin (y1 = a1*c1 - a2*s1, y2 = a2*c2 + a1*s2 in fp32,
// rounded once: the fused RoPE's arithmetic, partner half by shuffle); q goes
// to q_out [B, Hq, D], k to the K cache and the v row unchanged to the V
// cache, both at position *pos.  Replaces the two per-head norms, RoPE and
// the two cache writes of a decode step (five launches) with one.
struct QkPrep {
  const __nv_bfloat16* q;  // [B, Hq * D]
  const __nv_bfloat16* k;  // [B, Hkv * D]
  const __nv_bfloat16* v;  // [B, Hkv * D]
  const void* wq;
  const void* wk;
  int w_dtype;
  float eps_q, eps_k;
  const void* cos;         // [B, (1,) D] at batch stride cs_b
  const void* sin;
  int cs_dtype;
  int64_t cs_b;
  __nv_bfloat16* q_out;    // [B, Hq, D]
  __nv_bfloat16* k_cache;  // [B, Hkv, L, D]
  __nv_bfloat16* v_cache;
  const int64_t* pos;
  int B, Hq, Hkv, L;
};

// Row r of sequence b (q rows 0..Hq-1, k rows, v rows), one warp; k and v
// rows index the caches at p, so they need p inside [0, L).  A q row (whose
// cos/sin are per sequence, not per cache slot) goes to q_out, or, with q_f32, to
// q_f32[0, D) as the bf16-rounded values in fp32 (what a kernel loading
// q_out would see).
template <int EPL>
__device__ __forceinline__ void prep_row(const QkPrep& a, int b, int r, int64_t p,
                                         float* q_f32) {
  constexpr int D = 32 * EPL;
  const int lane = threadIdx.x & 31;
  const int d0 = lane * EPL;
  if (r >= a.Hq + a.Hkv) {  // v row: copy into the cache
    const int h = r - a.Hq - a.Hkv;
    const __nv_bfloat16* src = a.v + ((int64_t)b * a.Hkv + h) * D + d0;
    __nv_bfloat16* dst = a.v_cache + (((int64_t)b * a.Hkv + h) * a.L + p) * D + d0;
#pragma unroll
    for (int e = 0; e < EPL; ++e) dst[e] = src[e];
    return;
  }
  const bool is_q = r < a.Hq;
  const int h = is_q ? r : r - a.Hq;
  const __nv_bfloat16* src = is_q ? a.q + ((int64_t)b * a.Hq + h) * D + d0
                                  : a.k + ((int64_t)b * a.Hkv + h) * D + d0;
  const void* w = is_q ? a.wq : a.wk;
  float x[EPL];
  float ss = 0.f;
#pragma unroll
  for (int e = 0; e < EPL; ++e) {
    x[e] = __bfloat162float(src[e]);
    ss = fmaf(x[e], x[e], ss);
  }
  ss = warp_sum(ss);
  const float rr = rsqrtf(ss * (1.f / (float)D) + (is_q ? a.eps_q : a.eps_k));
  float y[EPL], yp[EPL];
#pragma unroll
  for (int e = 0; e < EPL; ++e)
    y[e] = __bfloat162float(__float2bfloat16_rn((x[e] * rr) * load_as_f32(w, d0 + e, a.w_dtype)));
#pragma unroll
  for (int e = 0; e < EPL; ++e) yp[e] = __shfl_xor_sync(0xffffffffu, y[e], 16);
  const bool first_half = lane < 16;
  float o[EPL];
#pragma unroll
  for (int e = 0; e < EPL; ++e) {
    const int d = d0 + e;
    const float c = load_as_f32(a.cos, (int64_t)b * a.cs_b + d, a.cs_dtype);
    const float sn = load_as_f32(a.sin, (int64_t)b * a.cs_b + d, a.cs_dtype);
    // first half: a1 = y, a2 = partner; second half: a2 = y, a1 = partner
    o[e] = first_half ? y[e] * c - yp[e] * sn : y[e] * c + yp[e] * sn;
  }
  if (is_q && q_f32 != nullptr) {
#pragma unroll
    for (int e = 0; e < EPL; ++e) q_f32[d0 + e] = __bfloat162float(__float2bfloat16_rn(o[e]));
    return;
  }
  __nv_bfloat16* dst = is_q ? a.q_out + ((int64_t)b * a.Hq + h) * D + d0
                            : a.k_cache + (((int64_t)b * a.Hkv + h) * a.L + p) * D + d0;
#pragma unroll
  for (int e = 0; e < EPL; ++e) dst[e] = __float2bfloat16_rn(o[e]);
}

template <int EPL>
__global__ void __launch_bounds__(256) decode_qk_prep(const __grid_constant__ QkPrep a) {
  const int64_t row = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int per_b = a.Hq + 2 * a.Hkv;
  if (row >= (int64_t)a.B * per_b) return;
  const int64_t p = *a.pos;
  const int r = (int)(row % per_b);
  // A q row is prepared for any position (as decode_qk_attn_single does);
  // the k and v rows are written only at a position inside the cache.
  if (r >= a.Hq && (p < 0 || p >= a.L)) return;
  prep_row<EPL>(a, (int)(row / per_b), r, p, nullptr);
}

// q/k preparation and the single-launch attention in one kernel, a CTA per
// (sequence, kv head): its warps first prepare the group's G q rows (into
// shared memory, as the bf16 values q_out would hold), the k row and the v
// row (into the caches at *pos); after a barrier, which makes the new cache
// row visible to the whole CTA, the slot warps and the merge run as in
// decode_attn_single.  Bitwise decode_qk_prep followed by the attention.
template <int G, int DPL>
__global__ void __launch_bounds__(32 * kFusedSlots)
decode_qk_attn_single(const __grid_constant__ QkPrep qp, const __grid_constant__ DecodeArgs a) {
  constexpr int D = 32 * DPL;
  __shared__ float qs[G * D];
  __shared__ float sm_m[kFusedSlots * G], sm_l[kFusedSlots * G];
  __shared__ float sm_o[kFusedSlots * G * D];
  const int warp = threadIdx.x >> 5;
  const int b = blockIdx.y / a.Hkv, kvh = blockIdx.y % a.Hkv;
  const int64_t p = *qp.pos;
  const bool in_cache = p >= 0 && p < qp.L;
  for (int r = warp; r < G + 2; r += kFusedSlots) {
    if (r < G)
      prep_row<DPL>(qp, b, kvh * G + r, p, qs + r * D);
    else if (in_cache)  // the k row, then the v row, of this kv head
      prep_row<DPL>(qp, b, r == G ? qp.Hq + kvh : qp.Hq + qp.Hkv + kvh, p, nullptr);
  }
  __syncthreads();
  attn_partial<G, DPL, true>(a, warp, qs, sm_m, sm_l, sm_o, G, 0);
  __syncthreads();
  const int nslot = (a.L + kChunk - 1) / kChunk;  // <= kFusedSlots (host check)
  for (int g = warp; g < G; g += kFusedSlots) {
    const int64_t h = (int64_t)kvh * G + g;
    merge_row<DPL>(sm_m, sm_l, sm_o, G, g, nslot, D, a.out + ((int64_t)b * a.Hq + h) * D);
  }
}

}  // namespace
}  // namespace ml

using namespace ml;

extern "C" int ml_decode_qk_norm_rope_bf16(
    const void* q, const void* k, const void* v, const void* wq, const void* wk, int w_dtype,
    float eps_q, float eps_k, const void* cos, const void* sin, int cs_dtype, int64_t cs_b,
    int64_t batch, int64_t q_heads, int64_t kv_heads, int64_t max_len, int64_t head_dim,
    void* q_out, void* k_cache, void* v_cache, const int64_t* pos, void* stream) {
  ML_CHECK_ARG(batch > 0 && q_heads > 0 && kv_heads > 0 && max_len > 0,
               "decode_qk_norm_rope: bad sizes");
  ML_CHECK_ARG(head_dim == 64 || head_dim == 128 || head_dim == 256,
               "decode_qk_norm_rope: head_dim %lld not in {64, 128, 256}", (long long)head_dim);
  ML_CHECK_ARG(q && k && v && wq && wk && cos && sin && q_out && k_cache && v_cache && pos,
               "decode_qk_norm_rope: null pointer");
  ML_CHECK_ARG((w_dtype >= 0 && w_dtype <= 2) && (cs_dtype >= 0 && cs_dtype <= 2),
               "decode_qk_norm_rope: bad dtype codes");
  QkPrep a;
  a.q = static_cast<const __nv_bfloat16*>(q);
  a.k = static_cast<const __nv_bfloat16*>(k);
  a.v = static_cast<const __nv_bfloat16*>(v);
  a.wq = wq;
  a.wk = wk;
  a.w_dtype = w_dtype;
  a.eps_q = eps_q;
  a.eps_k = eps_k;
  a.cos = cos;
  a.sin = sin;
  a.cs_dtype = cs_dtype;
  a.cs_b = cs_b;
  a.q_out = static_cast<__nv_bfloat16*>(q_out);
  a.k_cache = static_cast<__nv_bfloat16*>(k_cache);
  a.v_cache = static_cast<__nv_bfloat16*>(v_cache);
  a.pos = pos;
  a.B = (int)batch;
  a.Hq = (int)q_heads;
  a.Hkv = (int)kv_heads;
  a.L = (int)max_len;
  const int64_t rows = batch * (q_heads + 2 * kv_heads);
  const unsigned grid = (unsigned)((rows * 32 + 255) / 256);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (head_dim == 64) decode_qk_prep<2><<<grid, 256, 0, st>>>(a);
  else if (head_dim == 128) decode_qk_prep<4><<<grid, 256, 0, st>>>(a);
  else decode_qk_prep<8><<<grid, 256, 0, st>>>(a);
  ML_CHECK_LAUNCH("decode_qk_norm_rope");
  return ML_OK;
}

extern "C" size_t ml_decode_attention_workspace_bytes(int64_t batch, int64_t q_heads,
                                                      int64_t max_len, int64_t head_dim) {
  if (batch <= 0 || q_heads <= 0 || max_len <= 0 || head_dim <= 0) return 0;
  const int64_t nchunk = (max_len + kChunk - 1) / kChunk;
  if (nchunk <= kFusedSlots) return 0;  // one launch, partials in shared memory
  return (size_t)nchunk * batch * q_heads * (2 + head_dim) * sizeof(float);
}

extern "C" int ml_decode_attention_bf16(const void* q, int64_t sq_b, int64_t sq_h,
                                        const void* k_cache, const void* v_cache,
                                        const int64_t* pos, int64_t len_offset, int64_t batch,
                                        int64_t q_heads, int64_t kv_heads, int64_t max_len,
                                        int64_t head_dim, float scale, void* out, void* workspace,
                                        size_t workspace_bytes, void* stream) {
  ML_CHECK_ARG(batch > 0 && q_heads > 0 && kv_heads > 0 && max_len > 0,
               "decode_attention: bad sizes");
  ML_CHECK_ARG(q_heads % kv_heads == 0 && q_heads / kv_heads <= kMaxGroup,
               "decode_attention: %lld query heads per kv head (at most %d)",
               (long long)(q_heads / std::max<int64_t>(kv_heads, 1)), kMaxGroup);
  ML_CHECK_ARG(head_dim % 32 == 0 && head_dim <= kMaxDim,
               "decode_attention: head_dim %lld must be a multiple of 32 up to %d",
               (long long)head_dim, kMaxDim);
  ML_CHECK_ARG((q_heads / kv_heads) * head_dim <= 32 * kMaxGD,
               "decode_attention: query heads per kv head x head_dim above %d", 32 * kMaxGD);
  ML_CHECK_ARG(q && k_cache && v_cache && pos && out, "decode_attention: null pointer");
  ML_CHECK_ARG(aligned16(k_cache) && aligned16(v_cache),
               "decode_attention: KV buffers must be 16-byte aligned");
  ML_CHECK_ARG(batch * kv_heads <= 65535 && max_len < ((int64_t)1 << 31),
               "decode_attention: too many sequences x kv heads");
  const int nchunk = (int)((max_len + kChunk - 1) / kChunk);
  const bool single = nchunk <= kFusedSlots;
  ML_CHECK_ARG(single || (workspace && workspace_bytes >= ml_decode_attention_workspace_bytes(
                                                              batch, q_heads, max_len, head_dim)),
               "decode_attention: workspace too small");
  DecodeArgs a;
  a.q = static_cast<const __nv_bfloat16*>(q);
  a.k = static_cast<const __nv_bfloat16*>(k_cache);
  a.v = static_cast<const __nv_bfloat16*>(v_cache);
  a.pos = pos;
  a.len_offset = len_offset;
  a.sq_b = sq_b;
  a.sq_h = sq_h;
  a.B = (int)batch;
  a.Hq = (int)q_heads;
  a.Hkv = (int)kv_heads;
  a.L = (int)max_len;
  a.D = (int)head_dim;
  a.scale = scale;
  a.part_m = single ? nullptr : static_cast<float*>(workspace);
  a.part_l = single ? nullptr : a.part_m + (int64_t)nchunk * batch * q_heads;
  a.part_o = single ? nullptr : a.part_l + (int64_t)nchunk * batch * q_heads;
  a.out = static_cast<__nv_bfloat16*>(out);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int G = (int)(q_heads / kv_heads);
  const dim3 grid((nchunk + kWarps - 1) / kWarps, (unsigned)(batch * kv_heads));
  const int dpl = (int)(head_dim / 32);
#define ML_DA_CASE(G_, DPL_)                                               \
  if (G == G_ && dpl == DPL_) {                                            \
    if (single)                                                            \
      decode_attn_single<G_, DPL_>                                         \
          <<<dim3(1, (unsigned)(batch * kv_heads)), 32 * kFusedSlots, 0, st>>>(a); \
    else                                                                   \
      decode_attn_chunk<G_, DPL_><<<grid, 32 * kWarps, 0, st>>>(a);        \
    launched = true;                                                       \
  }
  bool launched = false;
  ML_DA_CASE(1, 2) ML_DA_CASE(1, 4) ML_DA_CASE(1, 8)
  ML_DA_CASE(2, 2) ML_DA_CASE(2, 4) ML_DA_CASE(2, 8)
  ML_DA_CASE(4, 2) ML_DA_CASE(4, 4) ML_DA_CASE(4, 8)
  ML_DA_CASE(8, 2) ML_DA_CASE(8, 4)
  ML_DA_CASE(16, 2)
#undef ML_DA_CASE
  if (!launched) {
    set_error("decode_attention: %d query heads per kv head with head_dim %lld is not built "
              "(G in {1, 2, 4, 8, 16}, head_dim in {64, 128, 256}, G * head_dim <= 1024)",
              G, (long long)head_dim);
    return ML_ERR_INVALID_ARG;
  }
  ML_CHECK_LAUNCH("decode_attention(chunk)");
  if (single) return ML_OK;
  const int64_t warps = batch * q_heads;
  const unsigned mgrid = (unsigned)((warps * 32 + 255) / 256);
  if (dpl == 2) decode_attn_merge<2><<<mgrid, 256, 0, st>>>(a, nchunk);
  else if (dpl == 4) decode_attn_merge<4><<<mgrid, 256, 0, st>>>(a, nchunk);
  else decode_attn_merge<8><<<mgrid, 256, 0, st>>>(a, nchunk);
  ML_CHECK_LAUNCH("decode_attention(merge)");
  return ML_OK;
}

extern "C" int ml_decode_qk_attention_bf16(
    const void* q, const void* k, const void* v, const void* wq, const void* wk, int w_dtype,
    float eps_q, float eps_k, const void* cos, const void* sin, int cs_dtype, int64_t cs_b,
    int64_t batch, int64_t q_heads, int64_t kv_heads, int64_t max_len, int64_t head_dim,
    void* k_cache, void* v_cache, const int64_t* pos, float scale, void* out, void* stream) {
  ML_CHECK_ARG(batch > 0 && q_heads > 0 && kv_heads > 0 && max_len > 0,
               "decode_qk_attention: bad sizes");
  ML_CHECK_ARG(head_dim == 64 || head_dim == 128 || head_dim == 256,
               "decode_qk_attention: head_dim %lld not in {64, 128, 256}", (long long)head_dim);
  ML_CHECK_ARG(q && k && v && wq && wk && cos && sin && k_cache && v_cache && pos && out,
               "decode_qk_attention: null pointer");
  ML_CHECK_ARG((w_dtype >= 0 && w_dtype <= 2) && (cs_dtype >= 0 && cs_dtype <= 2),
               "decode_qk_attention: bad dtype codes");
  ML_CHECK_ARG(q_heads % kv_heads == 0, "decode_qk_attention: %lld query heads for %lld kv heads",
               (long long)q_heads, (long long)kv_heads);
  ML_CHECK_ARG((max_len + kChunk - 1) / kChunk <= kFusedSlots,
               "decode_qk_attention: a cache of %lld positions (at most %d; longer caches take "
               "ml_decode_qk_norm_rope_bf16 and ml_decode_attention_bf16)",
               (long long)max_len, kChunk * kFusedSlots);
  ML_CHECK_ARG(aligned16(k_cache) && aligned16(v_cache),
               "decode_qk_attention: KV buffers must be 16-byte aligned");
  ML_CHECK_ARG(batch * kv_heads <= 65535, "decode_qk_attention: too many sequences x kv heads");
  QkPrep qp;
  qp.q = static_cast<const __nv_bfloat16*>(q);
  qp.k = static_cast<const __nv_bfloat16*>(k);
  qp.v = static_cast<const __nv_bfloat16*>(v);
  qp.wq = wq;
  qp.wk = wk;
  qp.w_dtype = w_dtype;
  qp.eps_q = eps_q;
  qp.eps_k = eps_k;
  qp.cos = cos;
  qp.sin = sin;
  qp.cs_dtype = cs_dtype;
  qp.cs_b = cs_b;
  qp.q_out = nullptr;  // q stays in shared memory
  qp.k_cache = static_cast<__nv_bfloat16*>(k_cache);
  qp.v_cache = static_cast<__nv_bfloat16*>(v_cache);
  qp.pos = pos;
  qp.B = (int)batch;
  qp.Hq = (int)q_heads;
  qp.Hkv = (int)kv_heads;
  qp.L = (int)max_len;
  DecodeArgs a;
  memset(&a, 0, sizeof(a));
  a.q = nullptr;  // taken from shared memory
  a.k = static_cast<const __nv_bfloat16*>(k_cache);
  a.v = static_cast<const __nv_bfloat16*>(v_cache);
  a.pos = pos;
  a.len_offset = 1;  // the new token's position is attended to
  a.B = (int)batch;
  a.Hq = (int)q_heads;
  a.Hkv = (int)kv_heads;
  a.L = (int)max_len;
  a.D = (int)head_dim;
  a.scale = scale;
  a.out = static_cast<__nv_bfloat16*>(out);
  const int G = (int)(q_heads / kv_heads);
  const int dpl = (int)(head_dim / 32);
  const dim3 grid(1, (unsigned)(batch * kv_heads));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  bool launched = false;
#define ML_QA_CASE(G_, DPL_)                                                           \
  if (G == G_ && dpl == DPL_) {                                                        \
    decode_qk_attn_single<G_, DPL_><<<grid, 32 * kFusedSlots, 0, st>>>(qp, a);         \
    launched = true;                                                                   \
  }
  ML_QA_CASE(1, 2) ML_QA_CASE(1, 4) ML_QA_CASE(1, 8)
  ML_QA_CASE(2, 2) ML_QA_CASE(2, 4) ML_QA_CASE(2, 8)
  ML_QA_CASE(4, 2) ML_QA_CASE(4, 4) ML_QA_CASE(4, 8)
  ML_QA_CASE(8, 2) ML_QA_CASE(8, 4)
  ML_QA_CASE(16, 2)
#undef ML_QA_CASE
  if (!launched) {
    set_error("decode_qk_attention: %d query heads per kv head with head_dim %lld is not built "
              "(G in {1, 2, 4, 8, 16}, head_dim in {64, 128, 256}, G * head_dim <= 1024)",
              G, (long long)head_dim);
    return ML_ERR_INVALID_ARG;
  }
  ML_CHECK_LAUNCH("decode_qk_attention");
  return ML_OK;
}
