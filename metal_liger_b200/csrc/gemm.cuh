// Persistent, warp-specialised tcgen05 GEMM for sm_100a (bf16 in, fp32 accumulate).
//
//   D[M, N] = alpha * sum_seg A_seg[M, K_seg] * B_seg[N, K_seg]^T  (+ epilogue)
//
// Each operand is given as a row-major bf16 matrix that is either "K-major"
// (K contiguous: A as [M, K], B as [N, K]) or "MN-major" (M or N contiguous:
// A as [K, M], B as [K, N]); both layouts are fed to the tensor core directly
// through 128-byte-swizzled TMA tiles, so no operand is ever transposed in
// memory.  Up to kMaxSeg K-segments (each with its own A/B tensors) are
// accumulated into one accumulator — this is how LoRA's rank-r term joins the
// base-weight product in the same TMEM tile, and how dQ*Wq + dK*Wk + dV*Wv
// becomes one GEMM.
//
// CTA = 6 warps: warp 0 issues TMA loads into a STAGES-deep shared-memory
// ring, warp 1 allocates TMEM and issues tcgen05.mma (M=128, N=BN, K=16) from
// one thread, warps 2-5 drain the fp32 accumulator (tcgen05.ld) and run the
// epilogue.  The accumulator is double-buffered in TMEM (2*BN columns) so the
// epilogue of tile i overlaps the MMAs of tile i+1.  The grid is persistent
// (<= one CTA per SM) and walks tiles in an L2-friendly raster.
//
// Every mbarrier wait is bounded (see sm100::mbar_wait_bounded): on timeout
// the CTA records an error in the library's device error word, all roles drain and the
// kernel frees its TMEM and returns.
#pragma once

#include "common.cuh"
#include "sm100.cuh"

namespace ml {
namespace gemm {

constexpr int BM = 128;
constexpr int BK = 64;       // one 128-byte swizzle row of bf16
constexpr int kMaxSeg = 4;
constexpr int kMaxPeers = 8;  // ranks a peer-mode store epilogue can address
constexpr int kThreads = 192;

enum Epi : int {
  EPI_STORE = 0,        // D = alpha*acc (+ beta*D), D bf16 or fp32
  EPI_PARTIAL = 1,      // split-K: fp32 partial [split][M][ldd] = alpha*acc
  EPI_FLCE = 2,         // fused linear-cross-entropy logits epilogue (BN = 256)
  EPI_ARGMAX = 3,       // greedy decoding head: per tile, the row's largest logit (rounded
                        // to the logit dtype) and the first column holding it
  EPI_SWIGLU = 4,       // split-B gate|up tile (BN = 256): gate, up and h = silu(gate) * up
                        // stored (bf16) from one accumulator
  EPI_DSWIGLU = 5,      // dH tile: d_gate, d_up of SwiGLU from dH and the stored gate / up
};

// Wait sites recorded in the device error word.
enum Site : int { SITE_PROD_EMPTY = 1, SITE_MMA_TEMPTY = 2, SITE_MMA_FULL = 3, SITE_EPI = 4,
                  SITE_DRAIN = 5, SITE_SELFTEST = 6 };

struct alignas(64) Params {
  CUtensorMap tma_a[kMaxSeg];
  CUtensorMap tma_b[kMaxSeg];
  // b_split: the B tile's columns [0, BN/2) come from tma_b and [BN/2, BN)
  // from tma_b2, both at rows [nt BN/2, nt BN/2 + BN/2) of their matrices
  // (K-major B only) — two weights whose matching rows share one tile.
  CUtensorMap tma_b2[kMaxSeg];
  int b_split;
  int seg_kb[kMaxSeg];     // k-blocks (of BK) per segment
  int nseg;
  // m_groups > 1 (1-SM kernel only): independent products stacked along M.
  // Group g takes m-tiles [grp_mt0[g], grp_mt0[g + 1]) with its own tensor
  // maps tma_a[g] / tma_b[g] and the K range all groups share; its output
  // rows start at row grp_row0[g] of D and it has grp_m[g] valid rows.
  int m_groups;
  int grp_mt0[kMaxSeg + 1];
  int grp_row0[kMaxSeg];
  int grp_m[kMaxSeg];
  int M, N;
  int m_tiles, n_tiles, splits, kb_per_split, kb_total;
  int raster;              // 0: M-tiles fastest, 1: N-tiles fastest
  int group_m;             // raster 0 only: N-tile groups of this many M-tiles (0 = all)
  int epi;
  int d_f32;               // EPI_STORE: 1 = fp32 output, 0 = bf16 output
  int vec_ok;              // output pointer/ld allow 16-byte stores
  void* D;
  int64_t ldd;
  int64_t split_stride;    // EPI_PARTIAL: elements between split slabs
  float alpha;
  float beta;              // EPI_STORE with fp32 D: D = alpha*acc + beta*D (beta in {0,1})
  // EPI_FLCE
  const int64_t* labels;   // labels for rows [0, M) (already offset to the chunk)
  int64_t label_base;      // vocabulary id of logit column 0 (vocab-sharded logits)
  int64_t ignore_index;
  float* part_m;           // [n_tiles][M] tile max of the logits row
  float* part_s;           // [n_tiles][M] sum exp(logit - tile max)
  float* tgt;              // [M] target logit
  int64_t vocab;           // valid logit columns (= N)
  const void* bias;        // optional [vocab] logit bias (EPI_FLCE, EPI_ARGMAX)
  int bias_dtype;
  // EPI_ARGMAX (also uses part_m, vocab, bias)
  int* part_i;             // [n_tiles][M] first column of the tile's row maximum
  int logit_dtype;         // ML_DTYPE_* the logits are rounded to before comparing
  // EPI_SWIGLU: D = gate, D2 = up, D3 = h.  EPI_DSWIGLU: D = d_gate, D2 = d_up,
  // aux1 = gate, aux2 = up (inputs).  All bf16 [M, N] at pitch ldd.
  void* D2;
  void* D3;
  const void* aux1;
  const void* aux2;
  // EPI_STORE fp32, peer mode (peer_n > 0): output row r goes to rank
  // o = r / peer_rows, into the receive slot that rank keeps for this one:
  // peer_dst[o] + (peer_me * peer_rows + r - o * peer_rows) * ldd — plain
  // stores into another GPU's memory (mapped here), issued tile by tile
  // while the GEMM runs.
  int peer_n;
  int peer_me;
  int peer_rows;
  float* peer_dst[kMaxPeers];
  int* err;                // device error word (bounded-wait timeouts)
};

__device__ __forceinline__ void decode_unit(const Params& p, int unit, int& mt, int& nt, int& sp) {
  const int tiles = p.m_tiles * p.n_tiles;
  sp = unit / tiles;
  int t = unit - sp * tiles;
  if (p.raster == 1) {
    mt = t / p.n_tiles;
    nt = t - mt * p.n_tiles;
  } else if (p.group_m > 0 && p.group_m < p.m_tiles) {
    // groups of group_m M-tiles sweep all N-tiles before moving on
    const int per_group = p.group_m * p.n_tiles;
    const int g = t / per_group;
    const int r = t - g * per_group;
    const int gm0 = g * p.group_m;
    const int gsize = min(p.group_m, p.m_tiles - gm0);
    nt = r / gsize;
    mt = gm0 + (r - nt * gsize);
  } else {
    nt = t / p.m_tiles;
    mt = t - nt * p.m_tiles;
  }
}

__device__ __forceinline__ int group_of(const Params& p, int mt) {
  int g = 0;
  while (g + 1 < p.m_groups && mt >= p.grp_mt0[g + 1]) ++g;
  return g;
}

__device__ __forceinline__ void locate_kb(const Params& p, int kb, int& seg, int& kl) {
  seg = 0;
  kl = kb;
#pragma unroll
  for (int s = 0; s < kMaxSeg - 1; ++s) {
    if (seg < p.nseg - 1 && kl >= p.seg_kb[seg]) {
      kl -= p.seg_kb[seg];
      ++seg;
    }
  }
}

template <int BN>
struct Cfg {
  static constexpr int STAGES = BN == 256 ? 4 : (BN == 128 ? 6 : 8);
  static constexpr uint32_t A_BYTES = BM * BK * 2;
  static constexpr uint32_t B_BYTES = BN * BK * 2;
  static constexpr uint32_t STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr uint32_t TMEM_COLS = 2 * BN < 32 ? 32 : 2 * BN;
  static constexpr size_t SMEM = 1024 /*align slack*/ + (size_t)STAGES * STAGE_BYTES + 256;
};

// ---------------------------------------------------------------------------
// epilogue helpers
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t pack_bf16x2(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

// Store 32 consecutive columns [col0, col0+32) of one output row.
__device__ __forceinline__ void store_row32(const Params& p, float (&v)[32], int64_t row,
                                            int col0, float* __restrict__ partial_base) {
  const int N = p.N;
  if (p.epi == EPI_PARTIAL) {
    float* dst = partial_base + row * p.ldd + col0;
    if (p.vec_ok && col0 + 32 <= N) {
#pragma unroll
      for (int j = 0; j < 32; j += 4)
        *reinterpret_cast<float4*>(dst + j) =
            make_float4(v[j] * p.alpha, v[j + 1] * p.alpha, v[j + 2] * p.alpha, v[j + 3] * p.alpha);
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (col0 + j < N) dst[j] = v[j] * p.alpha;
    }
    return;
  }
  if (p.d_f32) {
    float* dst;
    if (p.peer_n > 0) {
      const int o = (int)(row / p.peer_rows);
      dst = p.peer_dst[o] + ((int64_t)p.peer_me * p.peer_rows + row - (int64_t)o * p.peer_rows) *
                                p.ldd + col0;
    } else {
      dst = static_cast<float*>(p.D) + row * p.ldd + col0;
    }
    if (p.vec_ok && col0 + 32 <= N) {
#pragma unroll
      for (int j = 0; j < 32; j += 4) {
        float4 o = make_float4(v[j] * p.alpha, v[j + 1] * p.alpha, v[j + 2] * p.alpha,
                               v[j + 3] * p.alpha);
        if (p.beta != 0.f) {
          const float4 old = *reinterpret_cast<const float4*>(dst + j);
          o.x += old.x;
          o.y += old.y;
          o.z += old.z;
          o.w += old.w;
        }
        *reinterpret_cast<float4*>(dst + j) = o;
      }
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (col0 + j < N) dst[j] = v[j] * p.alpha + (p.beta != 0.f ? dst[j] : 0.f);
    }
  } else {
    __nv_bfloat16* dst = static_cast<__nv_bfloat16*>(p.D) + row * p.ldd + col0;
    if (p.vec_ok && col0 + 32 <= N) {
#pragma unroll
      for (int j = 0; j < 32; j += 8) {
        uint4 o;
        o.x = pack_bf16x2(v[j] * p.alpha, v[j + 1] * p.alpha);
        o.y = pack_bf16x2(v[j + 2] * p.alpha, v[j + 3] * p.alpha);
        o.z = pack_bf16x2(v[j + 4] * p.alpha, v[j + 5] * p.alpha);
        o.w = pack_bf16x2(v[j + 6] * p.alpha, v[j + 7] * p.alpha);
        *reinterpret_cast<uint4*>(dst + j) = o;
      }
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (col0 + j < N) dst[j] = __float2bfloat16_rn(v[j] * p.alpha);
    }
  }
}

__device__ __forceinline__ void add_bias32(const Params& p, float (&v)[32], int col0) {
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    const int col = col0 + j;
    if (col < p.vocab) v[j] += load_as_f32(p.bias, col, p.bias_dtype);
  }
}

// Logit value as a model whose logits have dtype `dt` would hold it.
__device__ __forceinline__ float round_logit(float v, int dt) {
  if (dt == ML_DTYPE_BF16) return __bfloat162float(__float2bfloat16_rn(v));
  if (dt == ML_DTYPE_F16) return __half2float(__float2half_rn(v));
  return v;
}

// torch.argmax order: NaN above every number, then larger values, then the
// earlier column.
__device__ __forceinline__ bool argmax_better(float a, int ca, float b, int cb) {
  const bool na = a != a, nb = b != b;
  if (na != nb) return na;
  if (!na && a != b) return a > b;
  return ca < cb;
}

// 8 bf16 from 8 floats (round to nearest even), as one 16-byte word.
__device__ __forceinline__ uint4 pack8_bf16(const float* v) {
  uint4 o;
  o.x = pack_bf16x2(v[0], v[1]);
  o.y = pack_bf16x2(v[2], v[3]);
  o.z = pack_bf16x2(v[4], v[5]);
  o.w = pack_bf16x2(v[6], v[7]);
  return o;
}

__device__ __forceinline__ float bf16r(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }

__device__ __forceinline__ void unpack8_bf16(const uint4& w, float* v) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&w);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float2 f = __bfloat1622float2(h[j]);
    v[2 * j] = f.x;
    v[2 * j + 1] = f.y;
  }
}

// EPI_SWIGLU, one 256-wide split-B tile: accumulator columns [0, 128) are
// gate and [128, 256) up for intermediate columns [128 nt, 128 nt + 128).
// gate and up are rounded to bf16 as the unfused projections store them, and
// h is computed from those stored values exactly as the SwiGLU kernel does.
__device__ __forceinline__ void swiglu_tile(const Params& p, uint32_t taddr, int64_t row,
                                            bool row_ok, int nt) {
  constexpr int HALF = 128;
  const int col_base = nt * HALF;
  __nv_bfloat16* dg = static_cast<__nv_bfloat16*>(p.D) + row * p.ldd;
  __nv_bfloat16* du = static_cast<__nv_bfloat16*>(p.D2) + row * p.ldd;
  __nv_bfloat16* dh = static_cast<__nv_bfloat16*>(p.D3) + row * p.ldd;
#pragma unroll 1
  for (int c = 0; c < HALF / 32; ++c) {
    float g[32], u[32];
    sm100::tmem_ld_32x32b_x32(taddr + c * 32, g);
    sm100::tmem_ld_32x32b_x32(taddr + HALF + c * 32, u);
    const int col0 = col_base + c * 32;
    if (!row_ok || col0 >= p.N) continue;
    float h[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      g[j] = bf16r(g[j] * p.alpha);
      u[j] = bf16r(u[j] * p.alpha);
      h[j] = swiglu_fwd(g[j], u[j]);
    }
    if (p.vec_ok && col0 + 32 <= p.N) {
#pragma unroll
      for (int j = 0; j < 32; j += 8) {
        *reinterpret_cast<uint4*>(dg + col0 + j) = pack8_bf16(g + j);
        *reinterpret_cast<uint4*>(du + col0 + j) = pack8_bf16(u + j);
        *reinterpret_cast<uint4*>(dh + col0 + j) = pack8_bf16(h + j);
      }
    } else {
      for (int j = 0; j < 32 && col0 + j < p.N; ++j) {
        dg[col0 + j] = __float2bfloat16_rn(g[j]);
        du[col0 + j] = __float2bfloat16_rn(u[j]);
        dh[col0 + j] = __float2bfloat16_rn(h[j]);
      }
    }
  }
}

// EPI_DSWIGLU: the accumulator is dH; dH is rounded to bf16 (as the unfused
// path stores it) and the SwiGLU backward is applied with the stored gate /
// up, written as d_gate (D) and d_up (D2): dH never reaches memory.  The
// gate / up words of the next 32 columns are loaded before the current ones
// are used, so one chunk of loads is always in flight behind the math.
template <int BN>
__device__ __forceinline__ void dswiglu_tile(const Params& p, uint32_t taddr, int64_t row,
                                             bool row_ok, int nt) {
  const int col_base = nt * BN;
  const __nv_bfloat16* gin = static_cast<const __nv_bfloat16*>(p.aux1) + row * p.ldd;
  const __nv_bfloat16* uin = static_cast<const __nv_bfloat16*>(p.aux2) + row * p.ldd;
  __nv_bfloat16* dgo = static_cast<__nv_bfloat16*>(p.D) + row * p.ldd;
  __nv_bfloat16* duo = static_cast<__nv_bfloat16*>(p.D2) + row * p.ldd;
  auto full_chunk = [&](int c) { return row_ok && p.vec_ok && col_base + c * 32 + 32 <= p.N; };
  uint4 gw[4], uw[4];
  if (full_chunk(0)) {
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      gw[q] = *reinterpret_cast<const uint4*>(gin + col_base + q * 8);
      uw[q] = *reinterpret_cast<const uint4*>(uin + col_base + q * 8);
    }
  }
#pragma unroll 1
  for (int c = 0; c < BN / 32; ++c) {
    float v[32];
    sm100::tmem_ld_32x32b_x32(taddr + c * 32, v);
    const int col0 = col_base + c * 32;
    uint4 gn[4], un[4];
    const bool next = c + 1 < BN / 32 && full_chunk(c + 1);
    if (next) {
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        gn[q] = *reinterpret_cast<const uint4*>(gin + col0 + 32 + q * 8);
        un[q] = *reinterpret_cast<const uint4*>(uin + col0 + 32 + q * 8);
      }
    }
    if (full_chunk(c)) {
      float g[32], u[32], dg[32], du[32];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        unpack8_bf16(gw[q], g + 8 * q);
        unpack8_bf16(uw[q], u + 8 * q);
      }
#pragma unroll
      for (int j = 0; j < 32; ++j) swiglu_bwd(g[j], u[j], bf16r(v[j] * p.alpha), dg[j], du[j]);
#pragma unroll
      for (int j = 0; j < 32; j += 8) {
        *reinterpret_cast<uint4*>(dgo + col0 + j) = pack8_bf16(dg + j);
        *reinterpret_cast<uint4*>(duo + col0 + j) = pack8_bf16(du + j);
      }
    } else if (row_ok) {
      for (int j = 0; j < 32 && col0 + j < p.N; ++j) {
        float dg, du;
        swiglu_bwd(__bfloat162float(gin[col0 + j]), __bfloat162float(uin[col0 + j]),
                   bf16r(v[j] * p.alpha), dg, du);
        dgo[col0 + j] = __float2bfloat16_rn(dg);
        duo[col0 + j] = __float2bfloat16_rn(du);
      }
    }
    if (next) {
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        gw[q] = gn[q];
        uw[q] = un[q];
      }
    }
  }
}

// Drains one accumulator tile (this thread's TMEM lane = output row `row`,
// BN fp32 columns starting at `taddr`) through the selected epilogue.
template <int BN>
__device__ __forceinline__ void epilogue_tile(const Params& p, uint32_t taddr, int64_t row,
                                              bool row_ok, int nt, int sp) {
  if (p.epi == EPI_FLCE) {
    if constexpr (BN == 256) {
      constexpr float kLog2e = 1.4426950408889634f;
      const int col_base = nt * BN;
      const int64_t label = row_ok ? p.labels[row] : p.ignore_index;
      const int64_t lrel =
          label == p.ignore_index ? (int64_t)-1 : label - p.label_base - col_base;
      // Tiles inside the vocabulary (all but the last) skip the per-column
      // bounds checks; the target column is picked only in the one chunk
      // that holds it; max and sum run as four independent chains.  Every
      // instruction saved here is an issue slot left to the producer and
      // MMA warps, which share the SM's schedulers with these warps.
      const bool full = col_base + BN <= p.vocab;
      const int tchunk = (lrel >= 0 && lrel < BN) ? (int)(lrel >> 5) : -1;
      const int tcol = (int)(lrel & 31);
      float m = -INFINITY;
      float tgt = 0.f;
      bool has_tgt = false;
#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
        float v[32];
        sm100::tmem_ld_32x32b_x32(taddr + c * 32, v);
        if (p.bias != nullptr) add_bias32(p, v, col_base + c * 32);
        if (full) {
          float m1 = -INFINITY, m2 = -INFINITY, m3 = -INFINITY;
#pragma unroll
          for (int j = 0; j < 32; j += 4) {
            m = fmaxf(m, v[j]);
            m1 = fmaxf(m1, v[j + 1]);
            m2 = fmaxf(m2, v[j + 2]);
            m3 = fmaxf(m3, v[j + 3]);
          }
          m = fmaxf(fmaxf(m, m1), fmaxf(m2, m3));
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if (col_base + c * 32 + j < p.vocab) m = fmaxf(m, v[j]);
        }
        if (c == tchunk) {
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if (j == tcol) tgt = v[j];
          has_tgt = true;
        }
      }
      const float mb = m * kLog2e;
      float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
        float v[32];
        sm100::tmem_ld_32x32b_x32(taddr + c * 32, v);
        const int col0 = col_base + c * 32;
        if (p.bias != nullptr) add_bias32(p, v, col0);
        if (full) {
#pragma unroll
          for (int j = 0; j < 32; j += 4) {
            v[j] = sm100::fast_exp2(fmaf(v[j], kLog2e, -mb));
            v[j + 1] = sm100::fast_exp2(fmaf(v[j + 1], kLog2e, -mb));
            v[j + 2] = sm100::fast_exp2(fmaf(v[j + 2], kLog2e, -mb));
            v[j + 3] = sm100::fast_exp2(fmaf(v[j + 3], kLog2e, -mb));
            s0 += v[j];
            s1 += v[j + 1];
            s2 += v[j + 2];
            s3 += v[j + 3];
          }
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const float e =
                (col0 + j < p.vocab) ? sm100::fast_exp2(fmaf(v[j], kLog2e, -mb)) : 0.f;
            s0 += e;
            v[j] = e;
          }
        }
        if (row_ok) {
          __nv_bfloat16* dst = static_cast<__nv_bfloat16*>(p.D) + row * p.ldd + col0;
          if (p.vec_ok && col0 + 32 <= p.vocab) {
#pragma unroll
            for (int j = 0; j < 32; j += 8) {
              uint4 o;
              o.x = pack_bf16x2(v[j], v[j + 1]);
              o.y = pack_bf16x2(v[j + 2], v[j + 3]);
              o.z = pack_bf16x2(v[j + 4], v[j + 5]);
              o.w = pack_bf16x2(v[j + 6], v[j + 7]);
              *reinterpret_cast<uint4*>(dst + j) = o;
            }
          } else {
            for (int j = 0; j < 32; ++j)
              if (col0 + j < p.vocab) dst[j] = __float2bfloat16_rn(v[j]);
          }
        }
      }
      const float s = (s0 + s1) + (s2 + s3);
      if (row_ok) {
        p.part_m[(int64_t)nt * p.M + row] = m;
        p.part_s[(int64_t)nt * p.M + row] = s;
        if (has_tgt) p.tgt[row] = tgt;
      }
    }
  } else if (p.epi == EPI_ARGMAX) {
    const int col_base = nt * BN;
    float best = 0.f;
    int best_col = -1;
#pragma unroll 1
    for (int c = 0; c < BN / 32; ++c) {
      float v[32];
      sm100::tmem_ld_32x32b_x32(taddr + c * 32, v);
      if (p.bias != nullptr) add_bias32(p, v, col_base + c * 32);
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        const int col = col_base + c * 32 + j;
        const float x = round_logit(v[j], p.logit_dtype);
        if (col < p.vocab && (best_col < 0 || argmax_better(x, col, best, best_col))) {
          best = x;
          best_col = col;
        }
      }
    }
    if (row_ok) {
      p.part_m[(int64_t)nt * p.M + row] = best;
      p.part_i[(int64_t)nt * p.M + row] = best_col;
    }
  } else if (p.epi == EPI_SWIGLU) {
    if constexpr (BN == 256) swiglu_tile(p, taddr, row, row_ok, nt);
  } else if (p.epi == EPI_DSWIGLU) {
    dswiglu_tile<BN>(p, taddr, row, row_ok, nt);
  } else {
    float* partial_base = nullptr;
    if (p.epi == EPI_PARTIAL) partial_base = static_cast<float*>(p.D) + (int64_t)sp * p.split_stride;
#pragma unroll 1
    for (int c = 0; c < BN / 32; ++c) {
      float v[32];
      sm100::tmem_ld_32x32b_x32(taddr + c * 32, v);
      const int col0 = nt * BN + c * 32;
      if (row_ok && col0 < p.N) store_row32(p, v, row, col0, partial_base);
    }
  }
}

// ---------------------------------------------------------------------------
// the kernel
// ---------------------------------------------------------------------------
template <int BN, bool A_MN, bool B_MN>
__global__ void __launch_bounds__(kThreads, 1) gemm_kernel(const __grid_constant__ Params p) {
  using C = Cfg<BN>;
  constexpr int STAGES = C::STAGES;
  constexpr uint32_t IDESC = sm100::idesc_bf16_f32(BM, BN, A_MN, B_MN);
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * C::A_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * C::STAGE_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      sm100::mbar_init(&full[s], 1);
      sm100::mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      sm100::mbar_init(&tfull[b], 1);
      sm100::mbar_init(&tempty[b], 4);
    }
    *abort_flag = 0;
    sm100::fence_barrier_init();
    sm100::fence_proxy_async_smem();
  }
  if (warp == 0 && lane == 0) {
    for (int s = 0; s < p.nseg; ++s) {
      sm100::tma_prefetch_desc(&p.tma_a[s]);
      sm100::tma_prefetch_desc(&p.tma_b[s]);
    }
  }
  if (warp == 1) {
    sm100::tmem_alloc(tmem_slot, C::TMEM_COLS);
    sm100::tmem_relinquish();
  }
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const int num_units = p.m_tiles * p.n_tiles * p.splits;
  // Launched as a programmatic dependent: the set-up above overlaps the
  // previous kernel's tail; no operand, output or FLCE statistic is touched
  // before that kernel has completed.
  pdl_wait();

  if (warp == 0) {
    // ------------------------------ producer ------------------------------
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int inflight = 0;  // stages issued but not yet known to be consumed
      bool ok = true;
      for (int unit = blockIdx.x; unit < num_units && ok; unit += gridDim.x) {
        int mt, nt, sp;
        decode_unit(p, unit, mt, nt, sp);
        const int kb0 = sp * p.kb_per_split;
        const int kb1 = min(p.kb_total, kb0 + p.kb_per_split);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!sm100::mbar_wait_bounded(&empty[stage], phase ^ 1u, abort_flag, p.err, SITE_PROD_EMPTY)) {
            ok = false;
            break;
          }
          inflight = min(inflight + 1, STAGES);
          int seg, kl;
          int a_row = mt * BM;  // M coordinate of the A tile in its tensor
          if (p.m_groups > 1) {
            seg = group_of(p, mt);
            kl = kb;
            a_row = (mt - p.grp_mt0[seg]) * BM;
          } else {
            locate_kb(p, kb, seg, kl);
          }
          const int kx = kl * BK;
          uint64_t* bar = &full[stage];
          sm100::mbar_arrive_expect_tx(bar, C::STAGE_BYTES);
          uint8_t* a_dst = sA + stage * C::A_BYTES;
          uint8_t* b_dst = sB + stage * C::B_BYTES;
          if constexpr (!A_MN) {
            sm100::tma_load_2d(a_dst, &p.tma_a[seg], bar, kx, a_row);
          } else {
            sm100::tma_load_2d(a_dst, &p.tma_a[seg], bar, a_row, kx);
            sm100::tma_load_2d(a_dst + 64 * BK * 2, &p.tma_a[seg], bar, a_row + 64, kx);
          }
          if constexpr (!B_MN) {
            if (p.b_split) {
              sm100::tma_load_2d(b_dst, &p.tma_b[seg], bar, kx, nt * (BN / 2));
              sm100::tma_load_2d(b_dst + (BN / 2) * BK * 2, &p.tma_b2[seg], bar, kx,
                                 nt * (BN / 2));
            } else {
              sm100::tma_load_2d(b_dst, &p.tma_b[seg], bar, kx, nt * BN);
            }
          } else {
#pragma unroll
            for (int c = 0; c < BN / 64; ++c)
              sm100::tma_load_2d(b_dst + c * 64 * BK * 2, &p.tma_b[seg], bar, nt * BN + c * 64,
                                 kx);
          }
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (!ok) {
        // Drain: let every issued copy land before the CTA exits (bounded).
        int s = stage, ph = phase;
        for (int i = 0; i < inflight; ++i) {
          if (--s < 0) {
            s = STAGES - 1;
            ph ^= 1;
          }
          const uint64_t t0 = sm100::globaltimer_ns();
          while (!sm100::mbar_try_wait(&full[s], ph) &&
                 sm100::globaltimer_ns() - t0 < 1000000000ull) {
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------ MMA issuer -----------------------------
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int unit = blockIdx.x; unit < num_units && ok; unit += gridDim.x) {
        int mt, nt, sp;
        decode_unit(p, unit, mt, nt, sp);
        const int kb0 = sp * p.kb_per_split;
        const int kb1 = min(p.kb_total, kb0 + p.kb_per_split);
        if (!sm100::mbar_wait_bounded(&tempty[acc], acc_phase ^ 1u, abort_flag, p.err, SITE_MMA_TEMPTY)) {
          ok = false;
          break;
        }
        sm100::tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(acc * BN);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!sm100::mbar_wait_bounded(&full[stage], phase, abort_flag, p.err, SITE_MMA_FULL)) {
            ok = false;
            break;
          }
          sm100::tc_fence_after();
          const uint32_t a_base = sm100::smem_u32(sA + stage * C::A_BYTES);
          const uint32_t b_base = sm100::smem_u32(sB + stage * C::B_BYTES);
          // one descriptor per operand and stage; each K = 16 step advances its
          // start-address field (address / 16) by 2048 / 16 (MN-major) or
          // 32 / 16 (K-major), which stays inside the 14-bit field
          const uint64_t ad0 = A_MN ? sm100::sdesc_sw128(a_base, 64 * BK * 2, 1024)
                                    : sm100::sdesc_sw128(a_base, 16, 1024);
          const uint64_t bd0 = B_MN ? sm100::sdesc_sw128(b_base, 64 * BK * 2, 1024)
                                    : sm100::sdesc_sw128(b_base, 16, 1024);
          constexpr uint64_t kAStep = A_MN ? 2048 / 16 : 32 / 16;
          constexpr uint64_t kBStep = B_MN ? 2048 / 16 : 32 / 16;
#pragma unroll
          for (int k = 0; k < BK / 16; ++k)
            sm100::umma_bf16(d_tmem, ad0 + k * kAStep, bd0 + k * kBStep, IDESC,
                        (kb > kb0 || k > 0) ? 1u : 0u);
          sm100::umma_commit(&empty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        sm100::umma_commit(&tfull[acc]);
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1u;
      }
    }
  } else {
    // ------------------------------ epilogue -------------------------------
    const int ew = warp & 3;                 // TMEM sub-partition of this warp
    const int rloc = ew * 32 + lane;         // row within the tile
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int unit = blockIdx.x; unit < num_units; unit += gridDim.x) {
      int mt, nt, sp;
      decode_unit(p, unit, mt, nt, sp);
      bool ok = sm100::mbar_wait_bounded(&tfull[acc], acc_phase, abort_flag, p.err, SITE_EPI);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      sm100::tc_fence_after();
      const uint32_t taddr = tmem_base + ((uint32_t)(ew * 32) << 16) + (uint32_t)(acc * BN);
      int64_t row = (int64_t)mt * BM + rloc;
      bool row_ok = row < p.M;
      if (p.m_groups > 1) {
        const int g = group_of(p, mt);
        const int lr = (mt - p.grp_mt0[g]) * BM + rloc;
        row = (int64_t)p.grp_row0[g] + lr;
        row_ok = lr < p.grp_m[g];
      }
      epilogue_tile<BN>(p, taddr, row, row_ok, nt, sp);
      sm100::tc_fence_before();
      __syncwarp();
      if (lane == 0) sm100::mbar_arrive(&tempty[acc]);
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1u;
    }
    // peer mode: this thread's stores into other GPUs are visible system-wide
    // before the grid completes
    if (p.peer_n > 0) __threadfence_system();
  }

  // A programmatic dependent (e.g. the split-K reduction) may begin launching.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  if (warp == 1) sm100::tmem_dealloc(tmem_base, C::TMEM_COLS);
}

// ---------------------------------------------------------------------------
// 2-SM variant: a cluster of 2 CTAs computes 256 x 256 tiles with
// tcgen05.mma.cta_group::2 (M = 256 split 128/128 across the pair's TMEM,
// N = 256 with each CTA holding half of B).  Per CTA and k-block only
// 16 KB of A and 16 KB of B cross into shared memory (vs 16 + 32 KB for the
// 1-SM 128 x 256 tile), which is what lets the tensor cores run near peak.
// Protocol: both CTAs' producers load their own halves with the pair form of
// the TMA load, completing bytes on the LEADER's full barrier (the leader
// arms it with the pair's total); the leader's single MMA thread issues the
// pair MMA and its commits arrive on the empty / TMEM-full barriers of both
// CTAs; each CTA drains its own 128 accumulator rows and arrives on the
// leader's TMEM-empty barrier.
// ---------------------------------------------------------------------------
// BN = 256 (each CTA holds 128 columns of B) or 128 (64 columns): the
// narrower tile fills the SM pairs better when 256-wide tiles would leave a
// mostly empty last wave.
template <int BN>
struct PairCfg {
  static constexpr int STAGES = BN == 256 ? 6 : 8;
  static constexpr uint32_t A_BYTES = 128 * BK * 2;        // this CTA's 128 rows of A
  static constexpr uint32_t B_BYTES = (BN / 2) * BK * 2;   // this CTA's BN/2 rows/cols of B
  static constexpr uint32_t STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr uint32_t TMEM_COLS = 2 * BN;            // two fp32 accumulators
  static constexpr size_t SMEM = 1024 + (size_t)STAGES * STAGE_BYTES + 256;
};

template <int BN, bool A_MN, bool B_MN>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
gemm_pair_kernel(const __grid_constant__ Params p) {
  static_assert(BN == 128 || BN == 256, "pair tile width");
  using C = PairCfg<BN>;
  constexpr int STAGES = C::STAGES;
  constexpr int BH = BN / 2;  // columns of B per CTA
  constexpr uint32_t IDESC = sm100::idesc_bf16_f32(256, BN, A_MN, B_MN);
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * C::A_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * C::STAGE_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = sm100::cluster_ctarank();
  const bool leader = rank == 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      sm100::mbar_init(&full[s], 1);   // used in the leader: its producer's arrive + tx
      sm100::mbar_init(&empty[s], 1);  // one commit (issued to both CTAs) per phase
    }
    for (int b = 0; b < 2; ++b) {
      sm100::mbar_init(&tfull[b], 1);
      sm100::mbar_init(&tempty[b], 8);  // 4 epilogue warps x 2 CTAs (leader's copy)
    }
    *abort_flag = 0;
    sm100::fence_barrier_init();
    sm100::fence_proxy_async_smem();
  }
  if (warp == 0 && lane == 0) {
    for (int s = 0; s < p.nseg; ++s) {
      sm100::tma_prefetch_desc(&p.tma_a[s]);
      sm100::tma_prefetch_desc(&p.tma_b[s]);
    }
  }
  if (warp == 1) {
    sm100::tmem_alloc_pair(tmem_slot, C::TMEM_COLS);
    sm100::tmem_relinquish_pair();
  }
  sm100::tc_fence_before();
  __syncthreads();
  sm100::cluster_sync();  // barriers of both CTAs initialised before any remote use
  sm100::tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const int num_units = p.m_tiles * p.n_tiles * p.splits;
  const int cluster_id = blockIdx.x >> 1;
  const int nclusters = gridDim.x >> 1;
  pdl_wait();  // programmatic dependent (see gemm_kernel)

  if (warp == 0) {
    // --------------------------- producer (both CTAs) ------------------------
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int inflight = 0;
      bool ok = true;
      for (int unit = cluster_id; unit < num_units && ok; unit += nclusters) {
        int mt, nt, sp;
        decode_unit(p, unit, mt, nt, sp);
        const int kb0 = sp * p.kb_per_split;
        const int kb1 = min(p.kb_total, kb0 + p.kb_per_split);
        const int m0 = mt * 256 + (int)rank * 128;
        const int n0 = nt * BN + (int)rank * BH;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!sm100::mbar_wait_bounded(&empty[stage], phase ^ 1u, abort_flag, p.err,
                                        SITE_PROD_EMPTY)) {
            ok = false;
            break;
          }
          inflight = min(inflight + 1, STAGES);
          int seg, kl;
          locate_kb(p, kb, seg, kl);
          const int kx = kl * BK;
          if (leader) sm100::mbar_arrive_expect_tx(&full[stage], 2 * C::STAGE_BYTES);
          const uint32_t bar = sm100::mapa_shared(sm100::smem_u32(&full[stage]), 0);
          uint8_t* a_dst = sA + stage * C::A_BYTES;
          uint8_t* b_dst = sB + stage * C::B_BYTES;
          if constexpr (!A_MN) {
            sm100::tma_load_2d_pair(a_dst, &p.tma_a[seg], bar, kx, m0);
          } else {
            sm100::tma_load_2d_pair(a_dst, &p.tma_a[seg], bar, m0, kx);
            sm100::tma_load_2d_pair(a_dst + 64 * BK * 2, &p.tma_a[seg], bar, m0 + 64, kx);
          }
          if constexpr (!B_MN) {
            if (p.b_split)  // this CTA's half of the tile: the first or the second matrix
              sm100::tma_load_2d_pair(b_dst, rank ? &p.tma_b2[seg] : &p.tma_b[seg], bar, kx,
                                      nt * BH);
            else
              sm100::tma_load_2d_pair(b_dst, &p.tma_b[seg], bar, kx, n0);
          } else {
#pragma unroll
            for (int c = 0; c < BH / 64; ++c)
              sm100::tma_load_2d_pair(b_dst + c * 64 * BK * 2, &p.tma_b[seg], bar, n0 + 64 * c, kx);
          }
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (!ok && leader) {
        // Drain (bounded): let every copy this pair issued land before exit.
        int s = stage, ph = phase;
        for (int i = 0; i < inflight; ++i) {
          if (--s < 0) {
            s = STAGES - 1;
            ph ^= 1;
          }
          const uint64_t t0 = sm100::globaltimer_ns();
          while (!sm100::mbar_try_wait(&full[s], ph) &&
                 sm100::globaltimer_ns() - t0 < 1000000000ull) {
          }
        }
      }
    }
  } else if (warp == 1) {
    // --------------------------- MMA issuer (leader) -------------------------
    if (lane == 0 && leader) {
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int unit = cluster_id; unit < num_units && ok; unit += nclusters) {
        int mt, nt, sp;
        decode_unit(p, unit, mt, nt, sp);
        const int kb0 = sp * p.kb_per_split;
        const int kb1 = min(p.kb_total, kb0 + p.kb_per_split);
        if (!sm100::mbar_wait_bounded(&tempty[acc], acc_phase ^ 1u, abort_flag, p.err,
                                      SITE_MMA_TEMPTY)) {
          ok = false;
          break;
        }
        sm100::tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(acc * BN);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!sm100::mbar_wait_bounded(&full[stage], phase, abort_flag, p.err, SITE_MMA_FULL)) {
            ok = false;
            break;
          }
          sm100::tc_fence_after();
          const uint32_t a_base = sm100::smem_u32(sA + stage * C::A_BYTES);
          const uint32_t b_base = sm100::smem_u32(sB + stage * C::B_BYTES);
          // one descriptor per operand and stage; each K = 16 step advances its
          // start-address field (address / 16) by 2048 / 16 (MN-major) or
          // 32 / 16 (K-major), which stays inside the 14-bit field
          const uint64_t ad0 = A_MN ? sm100::sdesc_sw128(a_base, 64 * BK * 2, 1024)
                                    : sm100::sdesc_sw128(a_base, 16, 1024);
          const uint64_t bd0 = B_MN ? sm100::sdesc_sw128(b_base, 64 * BK * 2, 1024)
                                    : sm100::sdesc_sw128(b_base, 16, 1024);
          constexpr uint64_t kAStep = A_MN ? 2048 / 16 : 32 / 16;
          constexpr uint64_t kBStep = B_MN ? 2048 / 16 : 32 / 16;
#pragma unroll
          for (int k = 0; k < BK / 16; ++k)
            sm100::umma_bf16_pair(d_tmem, ad0 + k * kAStep, bd0 + k * kBStep, IDESC,
                        (kb > kb0 || k > 0) ? 1u : 0u);
          sm100::umma_commit_pair(&empty[stage], 0x3);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        sm100::umma_commit_pair(&tfull[acc], 0x3);
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1u;
      }
    }
  } else {
    // --------------------------- epilogue (both CTAs) ------------------------
    const int ew = warp & 3;
    const int rloc = ew * 32 + lane;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int unit = cluster_id; unit < num_units; unit += nclusters) {
      int mt, nt, sp;
      decode_unit(p, unit, mt, nt, sp);
      bool ok = sm100::mbar_wait_bounded(&tfull[acc], acc_phase, abort_flag, p.err, SITE_EPI);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      sm100::tc_fence_after();
      const uint32_t taddr = tmem_base + ((uint32_t)(ew * 32) << 16) + (uint32_t)(acc * BN);
      const int64_t row = (int64_t)mt * 256 + (int64_t)rank * 128 + rloc;
      epilogue_tile<BN>(p, taddr, row, row < p.M, nt, sp);
      sm100::tc_fence_before();
      __syncwarp();
      if (lane == 0) sm100::mbar_arrive_cluster(sm100::mapa_shared(sm100::smem_u32(&tempty[acc]), 0));
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1u;
    }
    if (p.peer_n > 0) __threadfence_system();  // peer mode (see gemm_kernel)
  }

  // A programmatic dependent (e.g. the split-K reduction) may begin launching.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  sm100::tc_fence_before();
  __syncthreads();
  sm100::cluster_sync();  // no CTA leaves while its peer may still signal it
  sm100::tc_fence_after();
  if (warp == 1) sm100::tmem_dealloc_pair(tmem_base, C::TMEM_COLS);
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------

// Row-major bf16 matrix [rows, cols] with leading dimension `ld` (elements).
struct Mat {
  const void* ptr = nullptr;
  int64_t rows = 0, cols = 0, ld = 0;
};

// One K-segment: logical A [M, K], logical B [N, K].
//   a_mn = false: A stored as [M, K] (K contiguous); true: stored as [K, M].
//   b_mn = false: B stored as [N, K];                true: stored as [K, N].
struct Seg {
  Mat a, b;
  Mat b2;  // Problem::b_split: the matrix of the second half of every B tile
  int64_t K = 0;
};

struct Problem {
  int64_t M = 0, N = 0;
  Seg seg[kMaxSeg];
  int nseg = 0;
  bool a_mn = false, b_mn = false;
  int epi = EPI_STORE;
  bool d_f32 = false;
  void* D = nullptr;
  int64_t ldd = 0;
  float alpha = 1.f, beta = 0.f;
  int splits = 1;      // EPI_PARTIAL only
  int raster = 0;
  int group_m = 0;
  int bn = 0;          // 0 = choose
  int pair = -1;       // CTA-pair kernel: -1 = process default, else a ml_gemm_set_cta_pair mode
  int max_ctas = 0;    // 0 = SM count
  // FLCE
  const int64_t* labels = nullptr;
  int64_t label_base = 0;
  int64_t ignore_index = -100;
  float* part_m = nullptr;
  float* part_s = nullptr;
  float* tgt = nullptr;
  const void* bias = nullptr;
  int bias_dtype = 0;
  int64_t split_stride = 0;   // EPI_PARTIAL; 0 = M * ldd
  // EPI_ARGMAX
  int* part_i = nullptr;
  int logit_dtype = 0;
  // m_groups > 1: seg[g] is an independent product (A of grp_m[g] rows,
  // B, one K shared by all groups), stacked along M in D; M = sum grp_m.
  // Runs on the 1-SM kernel.
  int m_groups = 1;
  int64_t grp_m[kMaxSeg] = {};
  // b_split (K-major B, 256-wide tiles): N is the width of each of the two
  // B matrices; tile n holds their rows [128 n, 128 n + 128) side by side
  bool b_split = false;
  // EPI_SWIGLU / EPI_DSWIGLU outputs and inputs (see Params)
  void* D2 = nullptr;
  void* D3 = nullptr;
  const void* aux1 = nullptr;
  const void* aux2 = nullptr;
  // EPI_STORE fp32 peer mode (see Params): D unused; peer_dst[0..peer_n)
  int peer_n = 0;
  int peer_me = 0;
  int64_t peer_rows = 0;
  float* peer_dst[kMaxPeers] = {};
};

// Builds tensor maps, picks the tile width and launches.  Returns ML_OK or an
// error code (message via set_error).
int launch(const Problem& pr, cudaStream_t stream);

// Tile width the launcher would use for N (64, 128 or 256).
int pick_bn(int64_t N);

// Device address of the library's error word on the current device.
int* device_error_word();

// Split-K helper: out[M, N] (fp32, row pitch ldo) = alpha * A B^T via
// `splits` fp32 partial slabs in `partial` (>= splits*M*N floats) and a
// fixed-order reduction.  pr.epi / pr.D / pr.splits are filled in here.
int launch_splitk(Problem pr, int splits, float* out, int64_t ldo, float* partial,
                  size_t partial_bytes, cudaStream_t stream);
// Same with the output type chosen: fp32 (out_f32) or bf16.
int launch_splitk_to(Problem pr, int splits, void* out, bool out_f32, int64_t ldo,
                     float* partial, size_t partial_bytes, cudaStream_t stream);

// Split count launch_splitk would pick to fill the GPU for these sizes.
int auto_splits(int64_t M, int64_t N, int64_t K);

}  // namespace gemm
}  // namespace ml
