// Shared device/host helpers for the metal_liger_b200 CUDA library.
//
// Every kernel in this library is compiled for sm_100a only.  Host launchers
// are plain `extern "C"` functions (see include/metal_liger_b200.h) that take
// raw device pointers, sizes and a cudaStream_t, and return an int status
// (0 = ok).  The last error message is kept per host thread and can be read
// with ml_last_error().
#pragma once

#include <mutex>
#include <utility>

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>
#include <stdio.h>
#include <stdarg.h>

#include "../../include/metal_liger_b200.h"

namespace ml {

// ---------------------------------------------------------------------------
// Error reporting (host)
// ---------------------------------------------------------------------------
void set_error(const char* fmt, ...);

#define ML_CHECK_ARG(cond, ...)                                              \
  do {                                                                       \
    if (!(cond)) {                                                           \
      ::ml::set_error(__VA_ARGS__);                                          \
      return ML_ERR_INVALID_ARG;                                             \
    }                                                                        \
  } while (0)

#define ML_CHECK_LAUNCH(what)                                                \
  do {                                                                       \
    cudaError_t _e = cudaGetLastError();                                     \
    if (_e != cudaSuccess) {                                                 \
      ::ml::set_error("%s: CUDA launch failed: %s", what,                    \
                      cudaGetErrorString(_e));                               \
      return ML_ERR_CUDA;                                                    \
    }                                                                        \
  } while (0)

#define ML_CHECK_CUDA(call, what)                                            \
  do {                                                                       \
    cudaError_t _e = (call);                                                 \
    if (_e != cudaSuccess) {                                                 \
      ::ml::set_error("%s: %s", what, cudaGetErrorString(_e));               \
      return ML_ERR_CUDA;                                                    \
    }                                                                        \
  } while (0)

int num_sms();  // SM count of the current device (cached per device)

inline bool aligned16(const void* p) {
  return (reinterpret_cast<uintptr_t>(p) & 15u) == 0;
}

// RMSNorm row split, shared by the RMSNorm kernels (rms_norm.cu) and the
// decode GEMVs that replay the norm on their staged activations (gemv.cu),
// which must match it bit for bit: a row of `nvec` 16-byte vectors goes to
// `tpr` threads holding `nv` vectors each.  One vector per thread while
// nvec <= one_vec_limit, else the fewest of 2/4/8 that keep a row within
// kRmsMaxThreads threads; sub-warp groups of 4/8/16 threads for short rows,
// whole warps above.  False when no vector layout fits (scalar path).
constexpr int kRmsMaxThreads = 256;  // vector path: per-thread registers hold 2 rows (prefetch)

// Rows up to this many vectors take one vector per thread.  Measured on B200
// (bf16 [16384, 4096]): the forward is faster with two vectors per thread on
// 256 threads (4.4 vs 2.8 TB/s), the backward with one on 512 threads and
// the ring kernel (2.9 vs 2.6 TB/s).
constexpr int64_t rms_one_vec_limit(int elem_bytes, bool backward) {
  return (elem_bytes == 2 && backward) ? 512 : 256;
}

inline bool rms_row_split(int64_t nvec, int64_t one_vec_limit, int* nv_out, int* tpr_out) {
  int nv = 1;
  if (nvec > one_vec_limit)
    while ((nvec + nv - 1) / nv > kRmsMaxThreads && nv < 8) nv *= 2;
  const int64_t per = (nvec + nv - 1) / nv;
  int64_t tpr;
  if (per <= 4) tpr = 4;
  else if (per <= 8) tpr = 8;
  else if (per <= 16) tpr = 16;
  else tpr = (per + 31) / 32 * 32;
  if (tpr > (nv == 1 ? 512 : kRmsMaxThreads)) return false;
  *nv_out = nv;
  *tpr_out = (int)tpr;
  return true;
}

// ---------------------------------------------------------------------------
// Element access (device): load/store one element of a runtime dtype as fp32.
// ---------------------------------------------------------------------------
__device__ __forceinline__ float to_f32(float v) { return v; }
__device__ __forceinline__ float to_f32(__nv_bfloat16 v) { return __bfloat162float(v); }
__device__ __forceinline__ float to_f32(__half v) { return __half2float(v); }

template <typename T> __device__ __forceinline__ T from_f32(float v);
template <> __device__ __forceinline__ float from_f32<float>(float v) { return v; }
template <> __device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float v) {
  return __float2bfloat16_rn(v);
}
template <> __device__ __forceinline__ __half from_f32<__half>(float v) {
  return __float2half_rn(v);
}

__device__ __forceinline__ float load_as_f32(const void* p, int64_t i, int dtype) {
  switch (dtype) {
    case ML_DTYPE_F32: return static_cast<const float*>(p)[i];
    case ML_DTYPE_BF16: return __bfloat162float(static_cast<const __nv_bfloat16*>(p)[i]);
    default: return __half2float(static_cast<const __half*>(p)[i]);
  }
}

__device__ __forceinline__ void store_from_f32(void* p, int64_t i, int dtype, float v) {
  switch (dtype) {
    case ML_DTYPE_F32: static_cast<float*>(p)[i] = v; break;
    case ML_DTYPE_BF16: static_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v); break;
    default: static_cast<__half*>(p)[i] = __float2half_rn(v); break;
  }
}

// 16-byte vector of T: VEC = 16 / sizeof(T) elements.
template <typename T>
struct alignas(16) Vec16 {
  static constexpr int N = 16 / sizeof(T);
  T v[N];
};

template <typename T>
__device__ __forceinline__ Vec16<T> ld_vec(const T* p) {
  Vec16<T> r;
  *reinterpret_cast<int4*>(&r) = __ldg(reinterpret_cast<const int4*>(p));
  return r;
}

// Streaming load: data read exactly once (evict-first in L1/L2).
template <typename T>
__device__ __forceinline__ Vec16<T> ld_vec_stream(const T* p) {
  Vec16<T> r;
  *reinterpret_cast<int4*>(&r) = __ldcs(reinterpret_cast<const int4*>(p));
  return r;
}

template <typename T>
__device__ __forceinline__ void st_vec(T* p, const Vec16<T>& v) {
  *reinterpret_cast<int4*>(p) = *reinterpret_cast<const int4*>(&v);
}

template <typename T>
__device__ __forceinline__ void st_vec_stream(T* p, const Vec16<T>& v) {
  __stcs(reinterpret_cast<int4*>(p), *reinterpret_cast<const int4*>(&v));
}

// SwiGLU arithmetic (reference ops/fused_swiglu.py:26-50, fp32), shared by
// the elementwise kernels (swiglu.cu) and the GEMM epilogues that apply it to
// a fresh accumulator tile (gemm.cuh), so both round identically.
// sigmoid(g) = 1 / (1 + e^-g) with the SFU exponential and reciprocal (2 ulp
// each); the quotient tends to exactly 0 for large negative g.
__device__ __forceinline__ float swiglu_sigmoid(float g) {
  return __fdividef(1.f, 1.f + __expf(-g));
}
// h = silu(g) * u
__device__ __forceinline__ float swiglu_fwd(float g, float u) {
  const float s = swiglu_sigmoid(g);
  return (g * s) * u;
}
// d_gate = d u s (1 + g (1 - s)),  d_up = d silu(g)
__device__ __forceinline__ void swiglu_bwd(float g, float u, float d, float& dg, float& du) {
  const float s = swiglu_sigmoid(g);
  du = d * (g * s);
  dg = d * u * s * (1.f + g * (1.f - s));
}

// Programmatic dependent launch (PDL).  A kernel launched with launch_pdl
// may be scheduled while the previous kernel on the stream is still
// draining; it must call pdl_wait() before its first access to global
// memory that an earlier kernel may have written (the wait returns once the
// previous grid has completed and its writes are visible).  pdl_release()
// lets the next programmatic dependent start launching: every CTA calls it
// once, right after its own pdl_wait(), so the next kernel's CTAs fill the SMs
// as this grid's CTAs retire.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_release() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                       cudaStream_t st, Args&&... args) {
  cudaLaunchConfig_t lc = {};
  lc.gridDim = grid;
  lc.blockDim = block;
  lc.dynamicSmemBytes = smem;
  lc.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  lc.attrs = attr;
  lc.numAttrs = 1;
  return cudaLaunchKernelEx(&lc, kernel, std::forward<Args>(args)...);
}

// Runs a setup step (a kernel attribute, an occupancy query) once per CUDA
// device — the current one — and returns its cached result: kernel
// attributes belong to the device context they were set in.
template <typename T>
class PerDevice {
 public:
  template <typename F>
  T get(F&& fn) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDev) dev = 0;
    std::lock_guard<std::mutex> lock(mu_);
    if (!done_[dev]) {
      val_[dev] = fn();
      done_[dev] = true;
    }
    return val_[dev];
  }

 private:
  static constexpr int kMaxDev = 64;
  std::mutex mu_;
  bool done_[kMaxDev] = {};
  T val_[kMaxDev] = {};
};

// Shared-window address of a generic pointer to shared memory.
__device__ __forceinline__ uint32_t smem_u32_of(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

}  // namespace ml
