// Rotary position embedding (rotate-half convention) for sm_100a.
//
// Computes out = x*cos + rotate_half(x)*(sign*sin) with rotate_half([a,b]) =
// [-b, a], the expression of the reference's _apply_rotary_fused
// (ops/fused_rope.py:67-75); sign = -1 is the reference's backward
// (ops/fused_rope.py:50-57).  Element d < D/2 uses cos[d]/sin[d] and element
// d + D/2 uses cos[d+D/2]/sin[d+D/2], exactly as the broadcast expression
// does, so tables whose halves differ give the reference's answer too.
//
// Launch shape: work units of (batch, 16 positions, 8 heads of q|k), taken in
// contiguous ranges by a grid of ~4 waves.  Each thread owns one position and
// 16 bytes of each half of the head dim, keeps that position's cos/sin for
// its frequencies in registers (recompute mode: fp32 pos*inv_freq, sincosf,
// so HBM never sees a table) and rotates 4 head rows per step with all loads
// in flight together.  Each row half is a coalesced 16-byte-per-thread access.
#include "common.cuh"

#include <algorithm>

namespace ml {
namespace {

constexpr int kPos = 16;       // positions per work unit (one per thread group)
constexpr int kHeads = 8;      // heads per work unit
constexpr int kBatch = 4;      // rows per thread with loads in flight together
constexpr int kThreads = 256;  // upper bound; positions per unit shrink for wide rows
constexpr int kMaxHeadDim = 512;

struct RopeView {
  const void* in;
  void* out;
  int64_t heads;
  int64_t is[4];
  int64_t os[4];
};

struct RopeArgs {
  RopeView t[2];
  int ntensors;
  int64_t batch, seq, head_dim;
  // table mode
  const void* cos;
  const void* sin;
  int cs_dtype;
  int64_t cs[3];
  // recompute mode
  const int64_t* positions;
  int64_t pos_sb;
  const float* inv_freq;
  float scaling;
  float sign;
};

template <typename T, int N>
__device__ __forceinline__ void load_n(const T* p, float* f) {
  if constexpr (N * sizeof(T) % 16 == 0) {
#pragma unroll
    for (int c = 0; c < (int)(N * sizeof(T) / 16); ++c) {
      Vec16<T> v = ld_vec_stream(p + c * Vec16<T>::N);
#pragma unroll
      for (int j = 0; j < Vec16<T>::N; ++j) f[c * Vec16<T>::N + j] = to_f32(v.v[j]);
    }
  } else {
#pragma unroll
    for (int j = 0; j < N; ++j) f[j] = to_f32(p[j]);
  }
}

template <typename T, int N>
__device__ __forceinline__ void store_n(T* p, const float* f) {
  if constexpr (N * sizeof(T) % 16 == 0) {
#pragma unroll
    for (int c = 0; c < (int)(N * sizeof(T) / 16); ++c) {
      Vec16<T> v;
#pragma unroll
      for (int j = 0; j < Vec16<T>::N; ++j) v.v[j] = from_f32<T>(f[c * Vec16<T>::N + j]);
      st_vec_stream(p + c * Vec16<T>::N, v);
    }
  } else {
#pragma unroll
    for (int j = 0; j < N; ++j) p[j] = from_f32<T>(f[j]);
  }
}

// sin/cos of x for 16-bit outputs: reduce x to r in [-pi, pi] with a
// two-constant Cody-Waite step (2*pi = kTwoPiHi + kTwoPiLo, the first exactly
// representable in fp32), then evaluate with the SFU sin/cos, whose absolute
// error on [-pi, pi] is ~4e-7 -- far below bf16/fp16 resolution.
constexpr float kInvTwoPi = 0.15915494309189535f;
constexpr float kTwoPiHi = 6.28318548202514648f;
constexpr float kTwoPiLo = -1.7484556000744883e-07f;

__device__ __forceinline__ void sincos_reduced(float x, float* s, float* c) {
  const float k = rintf(x * kInvTwoPi);
  float r = fmaf(-k, kTwoPiHi, x);
  r = fmaf(-k, kTwoPiLo, r);
  *s = __sinf(r);
  *c = __cosf(r);
}

// Work unit = (batch, block of kPos positions, block of kHeads heads of the
// concatenated [q heads..., k heads...] list).  A CTA of kPos*TPH threads owns
// one position per thread group; each thread owns VEC frequencies, so it
// evaluates its 2*VEC cos/sin values once per position block (in registers,
// no shared memory, no barrier) and applies them to every head row of the
// unit.  CTAs take contiguous ranges of units (head blocks fastest), so cos/sin
// are recomputed only when the position block changes.
template <int N, typename T>
struct Raw {  // N elements of T kept packed in registers
  T v[N];
};

template <typename T, int N>
__device__ __forceinline__ void load_raw(const T* p, Raw<N, T>& r) {
  if constexpr (N * sizeof(T) % 16 == 0) {
#pragma unroll
    for (int c = 0; c < (int)(N * sizeof(T) / 16); ++c)
      *reinterpret_cast<int4*>(&r.v[c * (16 / sizeof(T))]) =
          __ldcs(reinterpret_cast<const int4*>(p) + c);
  } else {
#pragma unroll
    for (int j = 0; j < N; ++j) r.v[j] = p[j];
  }
}

template <typename Tin, typename Tout, int VEC, bool TABLE>
__global__ void __launch_bounds__(kThreads) rope_kernel(const RopeArgs a, int64_t units_per_cta,
                                                        int npos) {
  pdl_wait();  // a programmatic dependent: inputs may come from the previous kernel
  pdl_release();
  const int64_t D = a.head_dim;
  const int64_t half = D >> 1;
  const int tph = (int)(half / VEC);           // threads per row
  const int pgrp = threadIdx.x / tph;          // position within the block
  const int lane = threadIdx.x % tph;
  if (pgrp >= npos) return;
  const int64_t d0 = (int64_t)lane * VEC;
  const int64_t heads_total = a.t[0].heads + (a.ntensors > 1 ? a.t[1].heads : 0);
  const int64_t hblocks = (heads_total + kHeads - 1) / kHeads;
  const int64_t pblocks = (a.seq + npos - 1) / npos;
  const int64_t units = a.batch * pblocks * hblocks;
  const int64_t u0 = (int64_t)blockIdx.x * units_per_cta;
  const int64_t u1 = u0 + units_per_cta < units ? u0 + units_per_cta : units;
  const float sign = a.sign;
  // cos/sin of this thread's frequencies at its position; the recompute mode
  // has identical halves, so only the table mode keeps two sets.
  float c1[VEC], s1[VEC];
  float c2[TABLE ? VEC : 1], s2[TABLE ? VEC : 1];
  int64_t cached = -1;
  for (int64_t u = u0; u < u1; ++u) {
    const int64_t bp = u / hblocks;            // (batch, position block)
    const int64_t hb = u - bp * hblocks;
    const int64_t b = bp / pblocks;
    const int64_t s = (bp - b * pblocks) * npos + pgrp;
    const bool pos_ok = s < a.seq;
    if (bp != cached) {
      cached = bp;
      if (pos_ok) {
        if constexpr (TABLE) {
          const int64_t base = b * a.cs[0] + s * a.cs[1];
#pragma unroll
          for (int j = 0; j < VEC; ++j) {
            c1[j] = load_as_f32(a.cos, base + (d0 + j) * a.cs[2], a.cs_dtype);
            c2[j] = load_as_f32(a.cos, base + (d0 + j + half) * a.cs[2], a.cs_dtype);
            s1[j] = sign * load_as_f32(a.sin, base + (d0 + j) * a.cs[2], a.cs_dtype);
            s2[j] = sign * load_as_f32(a.sin, base + (d0 + j + half) * a.cs[2], a.cs_dtype);
          }
        } else {
          const int64_t pos = a.positions != nullptr ? a.positions[b * a.pos_sb + s] : s;
#pragma unroll
          for (int j = 0; j < VEC; ++j) {
            float sv, cv;
            const float ang = (float)pos * a.inv_freq[d0 + j];
            if constexpr (sizeof(Tout) == 2)
              sincos_reduced(ang, &sv, &cv);
            else
              sincosf(ang, &sv, &cv);
            c1[j] = cv * a.scaling;
            s1[j] = sign * sv * a.scaling;
          }
        }
      }
    }
    if (!pos_ok) continue;
    // rows of this unit: heads [hb*kHeads, ...) of the concatenated list
    const int64_t h_begin = hb * kHeads;
    const int64_t h_end = h_begin + kHeads < heads_total ? h_begin + kHeads : heads_total;
#pragma unroll 1
    for (int64_t h0 = h_begin; h0 < h_end; h0 += kBatch) {
      Raw<VEC, Tin> x1[kBatch], x2[kBatch];
#pragma unroll
      for (int q = 0; q < kBatch; ++q) {
        const int64_t hh = h0 + q;
        if (hh < h_end) {
          const int ti = hh < a.t[0].heads ? 0 : 1;
          const RopeView& v = a.t[ti];
          const int64_t h = ti == 0 ? hh : hh - a.t[0].heads;
          const Tin* xr = static_cast<const Tin*>(v.in) + b * v.is[0] + h * v.is[1] + s * v.is[2];
          load_raw<Tin, VEC>(xr + d0, x1[q]);
          load_raw<Tin, VEC>(xr + half + d0, x2[q]);
        }
      }
#pragma unroll
      for (int q = 0; q < kBatch; ++q) {
        const int64_t hh = h0 + q;
        if (hh < h_end) {
          const int ti = hh < a.t[0].heads ? 0 : 1;
          const RopeView& v = a.t[ti];
          const int64_t h = ti == 0 ? hh : hh - a.t[0].heads;
          float y1[VEC], y2[VEC];
#pragma unroll
          for (int j = 0; j < VEC; ++j) {
            const float a1 = to_f32(x1[q].v[j]);
            const float a2 = to_f32(x2[q].v[j]);
            if constexpr (TABLE) {
              y1[j] = a1 * c1[j] - a2 * s1[j];
              y2[j] = a2 * c2[j] + a1 * s2[j];
            } else {
              y1[j] = a1 * c1[j] - a2 * s1[j];
              y2[j] = a2 * c1[j] + a1 * s1[j];
            }
          }
          Tout* yr = static_cast<Tout*>(v.out) + b * v.os[0] + h * v.os[1] + s * v.os[2];
          store_n<Tout, VEC>(yr + d0, y1);
          store_n<Tout, VEC>(yr + half + d0, y2);
        }
      }
    }
  }
}

template <typename Tin, typename Tout>
int launch(const RopeArgs& a, bool vec_ok, cudaStream_t st) {
  constexpr int V = 16 / sizeof(Tin);
  const int vec = vec_ok ? V : 1;
  const int64_t half = a.head_dim / 2;
  const int tph = (int)(half / vec);
  if (tph > kThreads) {
    set_error("rope: head_dim too large for the launch shape");
    return ML_ERR_UNSUPPORTED;
  }
  const int npos = std::max(1, std::min(kPos, kThreads / tph));
  const int threads = std::max(32, (tph * npos + 31) / 32 * 32);
  const int64_t heads_total = a.t[0].heads + (a.ntensors > 1 ? a.t[1].heads : 0);
  const int64_t units = a.batch * ((a.seq + npos - 1) / npos) * ((heads_total + kHeads - 1) / kHeads);
  int per_sm = 0;
  const bool table = a.cos != nullptr;
  const void* kfn = table ? (vec_ok ? (const void*)rope_kernel<Tin, Tout, V, true>
                                    : (const void*)rope_kernel<Tin, Tout, 1, true>)
                          : (vec_ok ? (const void*)rope_kernel<Tin, Tout, V, false>
                                    : (const void*)rope_kernel<Tin, Tout, 1, false>);
  cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kfn, threads, 0);
  per_sm = std::max(per_sm, 1);
  // Each CTA takes a contiguous range of units.  Ranges are whole position
  // blocks (all head blocks of a position block) when that still leaves >= 2
  // waves, so cos/sin are evaluated once per position; otherwise single units.
  const int64_t hblocks = (heads_total + kHeads - 1) / kHeads;
  const int64_t slots = (int64_t)num_sms() * per_sm;
  int64_t per_cta = units / hblocks >= 2 * slots ? hblocks : 1;
  while (per_cta > 1 && (units + per_cta - 1) / per_cta < 2 * slots) per_cta /= 2;
  int64_t ctas = (units + per_cta - 1) / per_cta;
  // Launched as a programmatic dependent (PDL): the CTAs are scheduled while
  // the previous kernel drains and wait for it before their first load.
  auto k = table ? (vec_ok ? rope_kernel<Tin, Tout, V, true> : rope_kernel<Tin, Tout, 1, true>)
                 : (vec_ok ? rope_kernel<Tin, Tout, V, false> : rope_kernel<Tin, Tout, 1, false>);
  ML_CHECK_CUDA(launch_pdl(k, dim3((unsigned)ctas), dim3(threads), 0, st, a, per_cta, npos),
                "rope launch");
  return ML_OK;
}

bool view_vec_ok(const RopeView& v, int64_t half, int in_elt, int out_elt) {
  const int vin = 16 / in_elt;
  // The output side stores VEC(in) elements per half: VEC*out_elt bytes must
  // be a multiple of 16 (true for all supported pairs) and aligned.
  if (half % vin != 0) return false;
  if (!aligned16(v.in) || !aligned16(v.out)) return false;
  for (int i = 0; i < 3; ++i) {
    if ((v.is[i] * in_elt) % 16 != 0) return false;
    if ((v.os[i] * out_elt) % 16 != 0) return false;
  }
  if (((half * out_elt) % 16) != 0) return false;
  return true;
}

int dtype_size(int d) { return d == ML_DTYPE_F32 ? 4 : 2; }

}  // namespace
}  // namespace ml

using namespace ml;

extern "C" int ml_rope(const ml_rope_tensor* q, const ml_rope_tensor* k, int in_dtype,
                       int out_dtype, int64_t batch, int64_t seq, int64_t head_dim,
                       const void* cos, const void* sin, int cs_dtype, const int64_t* cs_strides,
                       const int64_t* positions, int64_t pos_stride_batch, const float* inv_freq,
                       float scaling, int sin_sign, void* stream) {
  ML_CHECK_ARG(q != nullptr, "rope: q view is required");
  ML_CHECK_ARG(batch >= 0 && seq >= 0, "rope: negative sizes");
  ML_CHECK_ARG(head_dim > 0 && head_dim % 2 == 0 && head_dim <= kMaxHeadDim,
               "rope: head_dim must be even and in [2, %d], got %lld", kMaxHeadDim,
               (long long)head_dim);
  ML_CHECK_ARG(sin_sign == 1 || sin_sign == -1, "rope: sin_sign must be +1 or -1");
  ML_CHECK_ARG(in_dtype >= 0 && in_dtype <= 2 && out_dtype >= 0 && out_dtype <= 2,
               "rope: bad dtype codes");
  if (cos != nullptr) {
    ML_CHECK_ARG(sin != nullptr && cs_strides != nullptr, "rope: table mode needs sin and strides");
    ML_CHECK_ARG(cs_dtype >= 0 && cs_dtype <= 2, "rope: bad cos/sin dtype");
  } else {
    ML_CHECK_ARG(inv_freq != nullptr, "rope: recompute mode needs inv_freq");
  }
  RopeArgs a{};
  const ml_rope_tensor* views[2] = {q, k};
  a.ntensors = 0;
  for (int i = 0; i < 2; ++i) {
    const ml_rope_tensor* v = views[i];
    if (v == nullptr || v->heads == 0) continue;
    ML_CHECK_ARG(v->heads > 0 && v->in && v->out, "rope: bad tensor view %d", i);
    ML_CHECK_ARG(v->in_strides[3] == 1 && v->out_strides[3] == 1,
                 "rope: the head_dim stride must be 1");
    RopeView& rv = a.t[a.ntensors++];
    rv.in = v->in;
    rv.out = v->out;
    rv.heads = v->heads;
    for (int j = 0; j < 4; ++j) {
      rv.is[j] = v->in_strides[j];
      rv.os[j] = v->out_strides[j];
    }
  }
  if (a.ntensors == 0 || batch == 0 || seq == 0) return ML_OK;
  a.batch = batch;
  a.seq = seq;
  a.head_dim = head_dim;
  a.cos = cos;
  a.sin = sin;
  a.cs_dtype = cs_dtype;
  if (cs_strides) {
    a.cs[0] = cs_strides[0];
    a.cs[1] = cs_strides[1];
    a.cs[2] = cs_strides[2];
  }
  a.positions = positions;
  a.pos_sb = pos_stride_batch;
  a.inv_freq = inv_freq;
  a.scaling = scaling;
  a.sign = (float)sin_sign;
  const int64_t half = head_dim / 2;
  bool vec_ok = true;
  for (int i = 0; i < a.ntensors; ++i)
    vec_ok = vec_ok && view_vec_ok(a.t[i], half, dtype_size(in_dtype), dtype_size(out_dtype));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (in_dtype == out_dtype) {
    switch (in_dtype) {
      case ML_DTYPE_F32: return launch<float, float>(a, vec_ok, st);
      case ML_DTYPE_BF16: return launch<__nv_bfloat16, __nv_bfloat16>(a, vec_ok, st);
      case ML_DTYPE_F16: return launch<__half, __half>(a, vec_ok, st);
    }
  } else if (out_dtype == ML_DTYPE_F32) {
    switch (in_dtype) {
      case ML_DTYPE_BF16: return launch<__nv_bfloat16, float>(a, vec_ok, st);
      case ML_DTYPE_F16: return launch<__half, float>(a, vec_ok, st);
    }
  } else if (in_dtype == ML_DTYPE_F32) {
    // Narrowing output (caller asked for it explicitly).
    switch (out_dtype) {
      case ML_DTYPE_BF16: return launch<float, __nv_bfloat16>(a, vec_ok, st);
      case ML_DTYPE_F16: return launch<float, __half>(a, vec_ok, st);
    }
  }
  set_error("rope: unsupported dtype pair (%d -> %d)", in_dtype, out_dtype);
  return ML_ERR_UNSUPPORTED;
}
