// Rotary position embedding (rotate-half convention) for sm_100a.
//
// Computes out = x*cos + rotate_half(x)*(sign*sin) with rotate_half([a,b]) =
// [-b, a], the expression of the reference's _apply_rotary_fused
// (ops/fused_rope.py:67-75); sign = -1 is the reference's backward
// (ops/fused_rope.py:50-57).  Element d < D/2 uses cos[d]/sin[d] and element
// d + D/2 uses cos[d+D/2]/sin[d+D/2], exactly as the broadcast expression
// does, so tables whose halves differ give the reference's answer too.
//
// Launch shape: one CTA per (batch, tile of kPos positions).  The CTA first
// materialises cos/sin for its positions in shared memory (in recompute mode
// from fp32 pos*inv_freq, so HBM never sees a table), then streams every
// head row of q and k for those positions: each row is split into
// 16-byte vectors of the first and second half, so one thread holds the
// (d, d+D/2) pairs it rotates.  Reads/writes are fully coalesced per row.
#include "common.cuh"

#include <algorithm>

namespace ml {
namespace {

constexpr int kPos = 8;        // positions per CTA
constexpr int kThreads = 256;
constexpr int kMaxHeadDim = 512;  // 2*kPos*512*4 B = 32 KB of shared memory

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

// VEC = elements of each half handled per thread (16 bytes of Tin, or 1 for
// the scalar path).
template <typename Tin, typename Tout, int VEC>
__global__ void __launch_bounds__(kThreads) rope_kernel(const RopeArgs a) {
  extern __shared__ float smem_cs[];  // [2][kPos][head_dim]
  const int64_t D = a.head_dim;
  float* cs_base = smem_cs;
  float* sn_base = smem_cs + kPos * D;
#define cs_s(p, d) cs_base[(p) * D + (d)]
#define sn_s(p, d) sn_base[(p) * D + (d)]
  const int64_t half = D >> 1;
  const int64_t tiles = (a.seq + kPos - 1) / kPos;
  const int64_t b = blockIdx.x / tiles;
  const int64_t s0 = (blockIdx.x % tiles) * kPos;
  const int np = (int)(a.seq - s0 < kPos ? a.seq - s0 : kPos);

  // 1) cos/sin for this CTA's positions.
  if (a.cos != nullptr) {
    for (int idx = threadIdx.x; idx < np * D; idx += blockDim.x) {
      const int p = idx / (int)D;
      const int64_t d = idx % D;
      const int64_t off = b * a.cs[0] + (s0 + p) * a.cs[1] + d * a.cs[2];
      cs_s(p, d) = load_as_f32(a.cos, off, a.cs_dtype);
      sn_s(p, d) = load_as_f32(a.sin, off, a.cs_dtype);
    }
  } else {
    for (int idx = threadIdx.x; idx < np * half; idx += blockDim.x) {
      const int p = idx / (int)half;
      const int64_t i = idx % half;
      const int64_t s = s0 + p;
      const int64_t pos = a.positions != nullptr ? a.positions[b * a.pos_sb + s] : s;
      const float ang = (float)pos * a.inv_freq[i];
      float sv, cv;
      sincosf(ang, &sv, &cv);
      cv *= a.scaling;
      sv *= a.scaling;
      cs_s(p, i) = cv;
      cs_s(p, i + half) = cv;
      sn_s(p, i) = sv;
      sn_s(p, i + half) = sv;
    }
  }
  __syncthreads();

  // 2) rotate every (tensor, head, position) row.
  const int tph = (int)(half / VEC);  // threads per row
  const int slots = blockDim.x / tph; // rows in flight per CTA step
  const int slot = threadIdx.x / tph;
  const int lane = threadIdx.x % tph;
  if (slot >= slots) return;
  const int64_t d0 = (int64_t)lane * VEC;
  const float sign = a.sign;
  for (int ti = 0; ti < a.ntensors; ++ti) {
    const RopeView& v = a.t[ti];
    const int64_t nrows = v.heads * np;
    const Tin* in = static_cast<const Tin*>(v.in);
    Tout* out = static_cast<Tout*>(v.out);
    for (int64_t r = slot; r < nrows; r += slots) {
      const int64_t h = r / np;
      const int p = (int)(r % np);
      const int64_t s = s0 + p;
      const Tin* xr = in + b * v.is[0] + h * v.is[1] + s * v.is[2];
      Tout* yr = out + b * v.os[0] + h * v.os[1] + s * v.os[2];
      float x1[VEC], x2[VEC], y1[VEC], y2[VEC];
      load_n<Tin, VEC>(xr + d0, x1);
      load_n<Tin, VEC>(xr + half + d0, x2);
#pragma unroll
      for (int j = 0; j < VEC; ++j) {
        const int64_t d = d0 + j;
        y1[j] = x1[j] * cs_s(p, d) - x2[j] * (sign * sn_s(p, d));
        y2[j] = x2[j] * cs_s(p, d + half) + x1[j] * (sign * sn_s(p, d + half));
      }
      store_n<Tout, VEC>(yr + d0, y1);
      store_n<Tout, VEC>(yr + half + d0, y2);
    }
  }
#undef cs_s
#undef sn_s
}

template <typename Tin, typename Tout>
int launch(const RopeArgs& a, bool vec_ok, cudaStream_t st) {
  const int64_t tiles = (a.seq + kPos - 1) / kPos;
  const int64_t grid = a.batch * tiles;
  if (grid > 0x7fffffff) {
    set_error("rope: grid too large");
    return ML_ERR_INVALID_ARG;
  }
  constexpr int V = 16 / sizeof(Tin);
  const size_t smem = 2 * kPos * (size_t)a.head_dim * sizeof(float);
  if (vec_ok)
    rope_kernel<Tin, Tout, V><<<(unsigned)grid, kThreads, smem, st>>>(a);
  else
    rope_kernel<Tin, Tout, 1><<<(unsigned)grid, kThreads, smem, st>>>(a);
  ML_CHECK_LAUNCH("rope");
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
