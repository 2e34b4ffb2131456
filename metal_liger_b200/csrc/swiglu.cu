// SwiGLU forward/backward for sm_100a.
//
// Math follows the reference's _FusedSwiGLUFunction (ops/fused_swiglu.py:26-50)
// and its Metal kernels (kernels/swiglu.metal:17-56): fp32 arithmetic, output
// cast to the input dtype.  Unlike the reference autograd Function (which
// saves an extra fp32 sigmoid tensor, ops/fused_swiglu.py:34), the backward
// recomputes sigmoid from gate, so only gate/up are kept between passes.
//
// Launch shape: grid-stride over 16-byte vectors (8 bf16 / 4 fp32 per
// thread per step), grid = SM count x resident CTAs; streaming loads/stores
// because every byte is touched exactly once.  Launched as programmatic
// dependents (PDL): the CTAs are scheduled while the previous kernel drains
// and wait for it before their first load.  A scalar tail handles n not a
// multiple of the vector width or unaligned pointers.
#include "common.cuh"

#include <algorithm>

namespace ml {
namespace {

template <typename T, int UNROLL>
__global__ void __launch_bounds__(256)
swiglu_fwd_kernel(const T* __restrict__ gate, const T* __restrict__ up, T* __restrict__ out,
                  int64_t n, bool vec_ok) {
  constexpr int VEC = 16 / sizeof(T);
  const int64_t nthreads = (int64_t)gridDim.x * blockDim.x;
  const int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  pdl_wait();  // launched as a programmatic dependent: inputs may come from the previous kernel
  pdl_release();
  int64_t done = 0;
  if (vec_ok) {
    const int64_t nvec = n / VEC;
    // UNROLL independent vectors per thread per step keeps enough bytes in flight.
    for (int64_t base = tid; base < nvec; base += nthreads * UNROLL) {
      Vec16<T> g[UNROLL], u[UNROLL];
#pragma unroll
      for (int k = 0; k < UNROLL; ++k) {
        const int64_t v = base + k * nthreads;
        if (v < nvec) {
          g[k] = ld_vec_stream(gate + v * VEC);
          u[k] = ld_vec_stream(up + v * VEC);
        }
      }
#pragma unroll
      for (int k = 0; k < UNROLL; ++k) {
        const int64_t v = base + k * nthreads;
        if (v < nvec) {
          Vec16<T> o;
#pragma unroll
          for (int j = 0; j < VEC; ++j) {
            o.v[j] = from_f32<T>(swiglu_fwd(to_f32(g[k].v[j]), to_f32(u[k].v[j])));
          }
          st_vec_stream(out + v * VEC, o);
        }
      }
    }
    done = nvec * VEC;
  }
  for (int64_t i = done + tid; i < n; i += nthreads) {
    out[i] = from_f32<T>(swiglu_fwd(to_f32(gate[i]), to_f32(up[i])));
  }
}

template <typename T, int UNROLL>
__global__ void __launch_bounds__(256)
swiglu_bwd_kernel(const T* __restrict__ gate, const T* __restrict__ up,
                  const T* __restrict__ dout, T* __restrict__ dgate, T* __restrict__ dup,
                  int64_t n, bool vec_ok) {
  constexpr int VEC = 16 / sizeof(T);
  const int64_t nthreads = (int64_t)gridDim.x * blockDim.x;
  const int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  pdl_wait();
  pdl_release();
  int64_t done = 0;
  if (vec_ok) {
    const int64_t nvec = n / VEC;
    for (int64_t base = tid; base < nvec; base += nthreads * UNROLL) {
      Vec16<T> g[UNROLL], u[UNROLL], d[UNROLL];
#pragma unroll
      for (int k = 0; k < UNROLL; ++k) {
        const int64_t v = base + k * nthreads;
        if (v < nvec) {
          g[k] = ld_vec_stream(gate + v * VEC);
          u[k] = ld_vec_stream(up + v * VEC);
          d[k] = ld_vec_stream(dout + v * VEC);
        }
      }
#pragma unroll
      for (int k = 0; k < UNROLL; ++k) {
        const int64_t v = base + k * nthreads;
        if (v < nvec) {
          Vec16<T> og, ou;
#pragma unroll
          for (int j = 0; j < VEC; ++j) {
            float dg, du;
            swiglu_bwd(to_f32(g[k].v[j]), to_f32(u[k].v[j]), to_f32(d[k].v[j]), dg, du);
            ou.v[j] = from_f32<T>(du);
            og.v[j] = from_f32<T>(dg);
          }
          st_vec_stream(dgate + v * VEC, og);
          st_vec_stream(dup + v * VEC, ou);
        }
      }
    }
    done = nvec * VEC;
  }
  for (int64_t i = done + tid; i < n; i += nthreads) {
    float dg, du;
    swiglu_bwd(to_f32(gate[i]), to_f32(up[i]), to_f32(dout[i]), dg, du);
    dup[i] = from_f32<T>(du);
    dgate[i] = from_f32<T>(dg);
  }
}

template <typename K>
int elementwise_grid(K kernel, int64_t n, int vec) {
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, 256, 0) != cudaSuccess ||
      per_sm <= 0)
    per_sm = 4;
  int64_t want = (n / vec + 255) / 256;
  int64_t grid = std::min<int64_t>((int64_t)num_sms() * per_sm, std::max<int64_t>(want, 1));
  return static_cast<int>(grid);
}

constexpr int kUnroll = 2;

template <typename T>
int launch_fwd(const void* gate, const void* up, void* out, int64_t n, cudaStream_t st) {
  constexpr int VEC = 16 / sizeof(T);
  const bool vec_ok = aligned16(gate) && aligned16(up) && aligned16(out);
  auto k = swiglu_fwd_kernel<T, kUnroll>;
  const int grid = elementwise_grid(k, n, VEC * kUnroll);
  ML_CHECK_CUDA(launch_pdl(k, dim3(grid), dim3(256), 0, st, static_cast<const T*>(gate),
                           static_cast<const T*>(up), static_cast<T*>(out), n, vec_ok),
                "swiglu_forward launch");
  return ML_OK;
}

template <typename T>
int launch_bwd(const void* gate, const void* up, const void* dout, void* dgate, void* dup,
               int64_t n, cudaStream_t st) {
  constexpr int VEC = 16 / sizeof(T);
  const bool vec_ok = aligned16(gate) && aligned16(up) && aligned16(dout) && aligned16(dgate) &&
                      aligned16(dup);
  auto k = swiglu_bwd_kernel<T, kUnroll>;
  const int grid = elementwise_grid(k, n, VEC * kUnroll);
  ML_CHECK_CUDA(launch_pdl(k, dim3(grid), dim3(256), 0, st, static_cast<const T*>(gate),
                           static_cast<const T*>(up), static_cast<const T*>(dout),
                           static_cast<T*>(dgate), static_cast<T*>(dup), n, vec_ok),
                "swiglu_backward launch");
  return ML_OK;
}

}  // namespace
}  // namespace ml

using namespace ml;

extern "C" int ml_swiglu_forward(const void* gate, const void* up, void* out, int64_t n, int dtype,
                                 void* stream) {
  ML_CHECK_ARG(n >= 0, "swiglu_forward: negative size");
  if (n == 0) return ML_OK;
  ML_CHECK_ARG(gate && up && out, "swiglu_forward: null pointer");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  switch (dtype) {
    case ML_DTYPE_F32: return launch_fwd<float>(gate, up, out, n, st);
    case ML_DTYPE_BF16: return launch_fwd<__nv_bfloat16>(gate, up, out, n, st);
    case ML_DTYPE_F16: return launch_fwd<__half>(gate, up, out, n, st);
  }
  set_error("swiglu_forward: bad dtype code %d", dtype);
  return ML_ERR_INVALID_ARG;
}

extern "C" int ml_swiglu_backward(const void* gate, const void* up, const void* dout, void* dgate,
                                  void* dup, int64_t n, int dtype, void* stream) {
  ML_CHECK_ARG(n >= 0, "swiglu_backward: negative size");
  if (n == 0) return ML_OK;
  ML_CHECK_ARG(gate && up && dout && dgate && dup, "swiglu_backward: null pointer");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  switch (dtype) {
    case ML_DTYPE_F32: return launch_bwd<float>(gate, up, dout, dgate, dup, n, st);
    case ML_DTYPE_BF16: return launch_bwd<__nv_bfloat16>(gate, up, dout, dgate, dup, n, st);
    case ML_DTYPE_F16: return launch_bwd<__half>(gate, up, dout, dgate, dup, n, st);
  }
  set_error("swiglu_backward: bad dtype code %d", dtype);
  return ML_ERR_INVALID_ARG;
}
