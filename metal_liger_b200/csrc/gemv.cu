// Decode-time linear layers: y[b, n] = sum_k x[b, k] * W[n, k] (+ bias[n])
// for one or two activation rows, HBM-streaming (gemv.cuh).  The greedy
// generator routes the decoder's bf16 nn.Linear calls through this while it
// decodes (one token per sequence per step), where a tensor-core tile would
// be 1/128 useful and the step is a pass over the weights.
//
// Rows of W go to warps round-robin with the CTA index fastest, so even a
// 1,024-row projection spreads its rows over every SM (each busy warp keeps
// 8 KB of one row in flight: 8 MB across the GPU for hidden 4096).
//
// A decoder layer's decode step runs as four of these launches around the
// attention kernels: the input RMSNorm fused into the q/k/v GEMV's
// activation staging, the residual add into the o projection's epilogue, the
// post-attention RMSNorm into the gate/up/SwiGLU GEMV and the residual add
// into the down projection's — each bitwise the unfused ops.
#include "gemv.cuh"

#include <cstring>

namespace ml {
namespace {

template <int NB, typename TO>
__global__ void __launch_bounds__(gemv::kThreads)
gemv_rows(const __nv_bfloat16* __restrict__ x, int64_t ld_x,
          const __nv_bfloat16* __restrict__ weight, int64_t ld_w, const void* __restrict__ bias,
          int bias_dtype, const __nv_bfloat16* __restrict__ residual, int64_t ld_r, int64_t K,
          int64_t N, TO* __restrict__ y, int64_t ld_y) {
  extern __shared__ uint4 hs[];  // [NB][K / 8] activation chunks
  const int64_t nchunk = K / 8;
  gemv::stage_rows<NB>(hs, x, ld_x, nchunk);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t total = (int64_t)gridDim.x * (blockDim.x >> 5);
  for (int64_t r = (int64_t)warp * gridDim.x + blockIdx.x; r < N; r += total) {
    float acc[NB];
    gemv::row_dot<NB>(reinterpret_cast<const uint4*>(weight + r * ld_w), hs, nchunk, lane, acc);
#pragma unroll
    for (int b = 0; b < NB; ++b) {
      float v = warp_sum(acc[b]);
      if (bias != nullptr) v += load_as_f32(bias, r, bias_dtype);
      // The decoder's `residual + proj(x)`: the projection rounded to bf16,
      // then torch's bf16 add (both operands to fp32, one rounding).
      if (residual != nullptr)
        v = __bfloat162float(__float2bfloat16_rn(v)) + __bfloat162float(residual[b * ld_r + r]);
      if (lane == 0) y[b * ld_y + r] = from_f32<TO>(v);
    }
  }
}

// SwiGLU MLP input side for decoding: h[b, i] = silu(gate) * up with
// gate = bf16(x . Wg[i]), up = bf16(x . Wu[i]) — one launch instead of two
// GEMVs and the activation kernel, and neither gate nor up is stored.  Each
// warp takes row i of both weights, 8 chunks of each in flight per lane per
// batch, in the same chunk order as row_dot (so gate and up are bitwise the
// two GEMVs' outputs), and the activation is the SwiGLU kernel's expression
// ((g * sigmoid(g)) * u, sigmoid = 1 / (1 + e^-g) on the SFU), so the fused
// step equals GEMV, GEMV, swiglu_forward bit for bit.  With `nw` the staged
// activations are first RMSNorm'd (gemv::rmsnorm_rows: the post-attention
// norm, bitwise the RMSNorm kernel's output).
__device__ __forceinline__ float sigmoid_sfu(float g) { return __fdividef(1.f, 1.f + __expf(-g)); }

template <int NB>
__global__ void __launch_bounds__(gemv::kThreads)
gemv_swiglu_rows(const __nv_bfloat16* __restrict__ x, int64_t ld_x,
                 const __nv_bfloat16* __restrict__ nw, float eps, int ntpr, int nnv,
                 const __nv_bfloat16* __restrict__ wg, int64_t ld_g,
                 const __nv_bfloat16* __restrict__ wu, int64_t ld_u, int64_t K, int64_t I,
                 __nv_bfloat16* __restrict__ y, int64_t ld_y) {
  constexpr int kHalf = gemv::kBatch / 2;
  extern __shared__ uint4 hs[];
  const int64_t nchunk = K / 8;
  gemv::stage_rows<NB>(hs, x, ld_x, nchunk);
  if (nw != nullptr) gemv::rmsnorm_rows<NB>(hs, nchunk, nw, eps, ntpr, nnv);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t total = (int64_t)gridDim.x * (blockDim.x >> 5);
  for (int64_t r = (int64_t)warp * gridDim.x + blockIdx.x; r < I; r += total) {
    const uint4* grow = reinterpret_cast<const uint4*>(wg + r * ld_g);
    const uint4* urow = reinterpret_cast<const uint4*>(wu + r * ld_u);
    float ag[NB], au[NB];
#pragma unroll
    for (int b = 0; b < NB; ++b) ag[b] = au[b] = 0.f;
    for (int64_t c0 = lane; c0 < nchunk; c0 += 32 * kHalf) {
      uint4 gv[kHalf], uv[kHalf];
#pragma unroll
      for (int u = 0; u < kHalf; ++u) {
        const int64_t c = c0 + 32 * u;
        if (c < nchunk) {
          gv[u] = __ldcs(grow + c);
          uv[u] = __ldcs(urow + c);
        }
      }
#pragma unroll
      for (int u = 0; u < kHalf; ++u) {
        const int64_t c = c0 + 32 * u;
        if (c < nchunk) {
#pragma unroll
          for (int b = 0; b < NB; ++b) {
            ag[b] = gemv::dot8_bf16(gv[u], hs[b * nchunk + c], ag[b]);
            au[b] = gemv::dot8_bf16(uv[u], hs[b * nchunk + c], au[b]);
          }
        }
      }
    }
#pragma unroll
    for (int b = 0; b < NB; ++b) {
      const float g = __bfloat162float(__float2bfloat16_rn(warp_sum(ag[b])));
      const float u = __bfloat162float(__float2bfloat16_rn(warp_sum(au[b])));
      if (lane == 0) y[b * ld_y + r] = __float2bfloat16_rn((g * sigmoid_sfu(g)) * u);
    }
  }
}

// Up to kMaxMats projections of the same activations in one launch (q, k
// and v of an attention block): their rows are concatenated in one row space
// and each warp row writes to its own matrix's output.  With `norm_w` the
// staged activations are first RMSNorm'd (the block's input norm).
constexpr int kMaxMats = 4;
struct MultiArgs {
  const __nv_bfloat16* w[kMaxMats];
  const void* bias[kMaxMats];
  void* y[kMaxMats];
  int64_t ld_w[kMaxMats], ld_y[kMaxMats], first[kMaxMats + 1];  // first[i]: row offset of matrix i
  const __nv_bfloat16* norm_w;  // NULL: no norm
  float eps;
  int ntpr, nnv;                // the RMSNorm kernel's row layout (gemv::rms_row_layout)
  int nmat;
  int bias_dtype;
};

template <int NB, typename TO>
__global__ void __launch_bounds__(gemv::kThreads)
gemv_multi_rows(const __nv_bfloat16* __restrict__ x, int64_t ld_x, int64_t K,
                const __grid_constant__ MultiArgs a) {
  extern __shared__ uint4 hs[];
  const int64_t nchunk = K / 8;
  gemv::stage_rows<NB>(hs, x, ld_x, nchunk);
  if (a.norm_w != nullptr) gemv::rmsnorm_rows<NB>(hs, nchunk, a.norm_w, a.eps, a.ntpr, a.nnv);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t total = (int64_t)gridDim.x * (blockDim.x >> 5);
  const int64_t R = a.first[a.nmat];
  for (int64_t r = (int64_t)warp * gridDim.x + blockIdx.x; r < R; r += total) {
    int m = 0;
#pragma unroll
    for (int i = 1; i < kMaxMats; ++i)
      if (i < a.nmat && r >= a.first[i]) m = i;
    const int64_t rr = r - a.first[m];
    float acc[NB];
    gemv::row_dot<NB>(reinterpret_cast<const uint4*>(a.w[m] + rr * a.ld_w[m]), hs, nchunk, lane,
                      acc);
#pragma unroll
    for (int b = 0; b < NB; ++b) {
      float v = warp_sum(acc[b]);
      if (a.bias[m] != nullptr) v += load_as_f32(a.bias[m], rr, a.bias_dtype);
      if (lane == 0) static_cast<TO*>(a.y[m])[b * a.ld_y[m] + rr] = from_f32<TO>(v);
    }
  }
}

template <int NB, typename TO>
int launch_rows(const void* x, int64_t ld_x, const void* w, int64_t ld_w, const void* bias,
                int bias_dtype, const void* residual, int64_t ld_r, int64_t K, int64_t N, void* y,
                int64_t ld_y, cudaStream_t st) {
  auto k = gemv_rows<NB, TO>;
  const size_t smem = (size_t)NB * K * 2;
  if (smem > 48 * 1024) {
    static PerDevice<cudaError_t> attr;
    ML_CHECK_CUDA(attr.get([&] {
                    return cudaFuncSetAttribute((const void*)k,
                                                cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                96 * 1024);
                  }),
                  "gemv_bf16: smem attribute");
  }
  // One CTA per SM (or per row when there are fewer rows): rows reach the
  // warps with the CTA index fastest, so every SM gets a share.
  const int grid = (int)std::max<int64_t>(1, std::min<int64_t>(num_sms(), N));
  k<<<grid, gemv::kThreads, smem, st>>>(static_cast<const __nv_bfloat16*>(x), ld_x,
                                        static_cast<const __nv_bfloat16*>(w), ld_w, bias,
                                        bias_dtype, static_cast<const __nv_bfloat16*>(residual),
                                        ld_r, K, N, static_cast<TO*>(y), ld_y);
  ML_CHECK_LAUNCH("gemv_bf16");
  return ML_OK;
}

}  // namespace
}  // namespace ml

namespace ml {
namespace {

// Checks and launch shared by ml_gemv_bf16 and ml_gemv_residual_bf16.
int gemv_entry(const char* what, const void* x, int64_t ld_x, const void* weight, int64_t ld_w,
               const void* bias, int bias_dtype, const void* residual, int64_t ld_r,
               int64_t batch, int64_t K, int64_t N, void* y, int y_dtype, int64_t ld_y,
               void* stream) {
  ML_CHECK_ARG(batch >= 0 && K > 0 && N > 0, "%s: bad sizes batch=%lld K=%lld N=%lld", what,
               (long long)batch, (long long)K, (long long)N);
  if (batch == 0) return ML_OK;
  ML_CHECK_ARG(x && weight && y, "%s: null pointer", what);
  ML_CHECK_ARG(gemv::eligible(batch, K, ld_x, ld_w, x, weight),
               "%s: needs 1-2 rows, K and row pitches multiples of 8, 16-byte aligned "
               "bases and rows*K*2 <= 96 KiB (batch=%lld K=%lld)",
               what, (long long)batch, (long long)K);
  ML_CHECK_ARG(y_dtype == ML_DTYPE_BF16 || y_dtype == ML_DTYPE_F32,
               "%s: output dtype %d is neither bf16 nor fp32", what, y_dtype);
  ML_CHECK_ARG(bias == nullptr || bias_dtype == ML_DTYPE_F32 || bias_dtype == ML_DTYPE_BF16 ||
                   bias_dtype == ML_DTYPE_F16,
               "%s: bad bias dtype %d", what, bias_dtype);
  ML_CHECK_ARG(ld_y >= N, "%s: output pitch %lld below N %lld", what, (long long)ld_y,
               (long long)N);
  ML_CHECK_ARG(residual == nullptr || (y_dtype == ML_DTYPE_BF16 && ld_r >= N),
               "%s: a residual needs a bf16 output and a pitch of at least N", what);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (y_dtype == ML_DTYPE_BF16)
    return batch == 1 ? launch_rows<1, __nv_bfloat16>(x, ld_x, weight, ld_w, bias, bias_dtype,
                                                      residual, ld_r, K, N, y, ld_y, st)
                      : launch_rows<2, __nv_bfloat16>(x, ld_x, weight, ld_w, bias, bias_dtype,
                                                      residual, ld_r, K, N, y, ld_y, st);
  return batch == 1 ? launch_rows<1, float>(x, ld_x, weight, ld_w, bias, bias_dtype, nullptr, 0,
                                            K, N, y, ld_y, st)
                    : launch_rows<2, float>(x, ld_x, weight, ld_w, bias, bias_dtype, nullptr, 0,
                                            K, N, y, ld_y, st);
}

// Norm operand checks shared by the fused-RMSNorm entries; fills the row
// layout the RMSNorm kernel would use (0, 0 without a norm).
int norm_args(const char* what, const void* norm_w, int64_t K, float eps, int* tpr, int* nv) {
  *tpr = 0;
  *nv = 0;
  if (norm_w == nullptr) return ML_OK;
  ML_CHECK_ARG(aligned16(norm_w), "%s: norm weight not 16-byte aligned", what);
  ML_CHECK_ARG(eps >= 0.f, "%s: negative eps", what);
  ML_CHECK_ARG(gemv::rms_row_layout(K, tpr, nv),
               "%s: no vector RMSNorm layout for a %lld-element row", what, (long long)K);
  return ML_OK;
}

int swiglu_entry(const char* what, const void* x, int64_t ld_x, const void* norm_w, float eps,
                 const void* w_gate, int64_t ld_g, const void* w_up, int64_t ld_u, int64_t batch,
                 int64_t K, int64_t inter, void* y, int64_t ld_y, void* stream) {
  ML_CHECK_ARG(batch >= 0 && K > 0 && inter > 0, "%s: bad sizes batch=%lld K=%lld inter=%lld",
               what, (long long)batch, (long long)K, (long long)inter);
  if (batch == 0) return ML_OK;
  ML_CHECK_ARG(x && w_gate && w_up && y, "%s: null pointer", what);
  ML_CHECK_ARG(gemv::eligible(batch, K, ld_x, ld_g, x, w_gate) &&
                   gemv::eligible(batch, K, ld_x, ld_u, x, w_up),
               "%s: needs 1-2 rows, K and row pitches multiples of 8, 16-byte "
               "aligned bases and rows*K*2 <= 96 KiB (batch=%lld K=%lld)",
               what, (long long)batch, (long long)K);
  ML_CHECK_ARG(ld_y >= inter, "%s: output pitch %lld below %lld", what, (long long)ld_y,
               (long long)inter);
  int tpr, nv;
  const int rc = norm_args(what, norm_w, K, eps, &tpr, &nv);
  if (rc != ML_OK) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const size_t smem = (size_t)batch * K * 2;
  const int grid = (int)std::max<int64_t>(1, std::min<int64_t>(num_sms(), inter));
  auto run = [&](auto kernel) -> int {
    if (smem > 48 * 1024)
      ML_CHECK_CUDA(cudaFuncSetAttribute((const void*)kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, 96 * 1024),
                    what);
    kernel<<<grid, gemv::kThreads, smem, st>>>(
        static_cast<const __nv_bfloat16*>(x), ld_x, static_cast<const __nv_bfloat16*>(norm_w),
        eps, tpr, nv, static_cast<const __nv_bfloat16*>(w_gate), ld_g,
        static_cast<const __nv_bfloat16*>(w_up), ld_u, K, inter,
        static_cast<__nv_bfloat16*>(y), ld_y);
    ML_CHECK_LAUNCH(what);
    return ML_OK;
  };
  return batch == 1 ? run(gemv_swiglu_rows<1>) : run(gemv_swiglu_rows<2>);
}

int multi_entry(const char* what, const void* x, int64_t ld_x, const void* norm_w, float eps,
                int nmat, const void* const* weight, const int64_t* ld_w, const int64_t* n,
                const void* const* bias, int bias_dtype, int64_t batch, int64_t K,
                void* const* y, const int64_t* ld_y, int y_dtype, void* stream) {
  ML_CHECK_ARG(nmat >= 1 && nmat <= kMaxMats, "%s: %d matrices (1-%d)", what, nmat, kMaxMats);
  ML_CHECK_ARG(batch >= 0 && K > 0, "%s: bad sizes batch=%lld K=%lld", what, (long long)batch,
               (long long)K);
  if (batch == 0) return ML_OK;
  ML_CHECK_ARG(x && weight && ld_w && n && y && ld_y, "%s: null pointer", what);
  ML_CHECK_ARG(y_dtype == ML_DTYPE_BF16 || y_dtype == ML_DTYPE_F32,
               "%s: output dtype %d is neither bf16 nor fp32", what, y_dtype);
  ML_CHECK_ARG(bias == nullptr || bias_dtype == ML_DTYPE_F32 || bias_dtype == ML_DTYPE_BF16 ||
                   bias_dtype == ML_DTYPE_F16,
               "%s: bad bias dtype %d", what, bias_dtype);
  MultiArgs a;
  memset(&a, 0, sizeof(a));
  const int rc = norm_args(what, norm_w, K, eps, &a.ntpr, &a.nnv);
  if (rc != ML_OK) return rc;
  a.norm_w = static_cast<const __nv_bfloat16*>(norm_w);
  a.eps = eps;
  a.nmat = nmat;
  a.bias_dtype = bias_dtype;
  a.first[0] = 0;
  for (int i = 0; i < nmat; ++i) {
    ML_CHECK_ARG(weight[i] && y[i] && n[i] > 0, "%s: matrix %d is empty or null", what, i);
    ML_CHECK_ARG(gemv::eligible(batch, K, ld_x, ld_w[i], x, weight[i]),
                 "%s: matrix %d: needs 1-2 rows, K and row pitches multiples of 8, "
                 "16-byte aligned bases and rows*K*2 <= 96 KiB", what, i);
    ML_CHECK_ARG(ld_y[i] >= n[i], "%s: output %d pitch below its rows", what, i);
    a.w[i] = static_cast<const __nv_bfloat16*>(weight[i]);
    a.bias[i] = bias != nullptr ? bias[i] : nullptr;
    a.y[i] = y[i];
    a.ld_w[i] = ld_w[i];
    a.ld_y[i] = ld_y[i];
    a.first[i + 1] = a.first[i] + n[i];
  }
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const size_t smem = (size_t)batch * K * 2;
  const int grid = (int)std::max<int64_t>(1, std::min<int64_t>(num_sms(), a.first[nmat]));
  auto run = [&](auto kernel) -> int {
    if (smem > 48 * 1024)
      ML_CHECK_CUDA(cudaFuncSetAttribute((const void*)kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, 96 * 1024),
                    what);
    kernel<<<grid, gemv::kThreads, smem, st>>>(static_cast<const __nv_bfloat16*>(x), ld_x, K, a);
    ML_CHECK_LAUNCH(what);
    return ML_OK;
  };
  if (y_dtype == ML_DTYPE_BF16)
    return batch == 1 ? run(gemv_multi_rows<1, __nv_bfloat16>)
                      : run(gemv_multi_rows<2, __nv_bfloat16>);
  return batch == 1 ? run(gemv_multi_rows<1, float>) : run(gemv_multi_rows<2, float>);
}

}  // namespace
}  // namespace ml

using namespace ml;

extern "C" int ml_gemv_bf16(const void* x, int64_t ld_x, const void* weight, int64_t ld_w,
                            const void* bias, int bias_dtype, int64_t batch, int64_t K, int64_t N,
                            void* y, int y_dtype, int64_t ld_y, void* stream) {
  return gemv_entry("gemv_bf16", x, ld_x, weight, ld_w, bias, bias_dtype, nullptr, 0, batch, K,
                    N, y, y_dtype, ld_y, stream);
}

extern "C" int ml_gemv_residual_bf16(const void* x, int64_t ld_x, const void* weight,
                                     int64_t ld_w, const void* bias, int bias_dtype,
                                     const void* residual, int64_t ld_r, int64_t batch,
                                     int64_t K, int64_t N, void* y, int64_t ld_y, void* stream) {
  return gemv_entry("gemv_residual_bf16", x, ld_x, weight, ld_w, bias, bias_dtype, residual,
                    ld_r, batch, K, N, y, ML_DTYPE_BF16, ld_y, stream);
}

extern "C" int ml_gemv_swiglu_bf16(const void* x, int64_t ld_x, const void* w_gate, int64_t ld_g,
                                   const void* w_up, int64_t ld_u, int64_t batch, int64_t K,
                                   int64_t inter, void* y, int64_t ld_y, void* stream) {
  return swiglu_entry("gemv_swiglu_bf16", x, ld_x, nullptr, 0.f, w_gate, ld_g, w_up, ld_u, batch,
                      K, inter, y, ld_y, stream);
}

extern "C" int ml_gemv_rmsnorm_swiglu_bf16(const void* x, int64_t ld_x, const void* norm_weight,
                                           float eps, const void* w_gate, int64_t ld_g,
                                           const void* w_up, int64_t ld_u, int64_t batch,
                                           int64_t K, int64_t inter, void* y, int64_t ld_y,
                                           void* stream) {
  ML_CHECK_ARG(norm_weight != nullptr, "gemv_rmsnorm_swiglu_bf16: null norm weight");
  return swiglu_entry("gemv_rmsnorm_swiglu_bf16", x, ld_x, norm_weight, eps, w_gate, ld_g, w_up,
                      ld_u, batch, K, inter, y, ld_y, stream);
}

extern "C" int ml_gemv_multi_bf16(const void* x, int64_t ld_x, int nmat, const void* const* weight,
                                  const int64_t* ld_w, const int64_t* n, const void* const* bias,
                                  int bias_dtype, int64_t batch, int64_t K, void* const* y,
                                  const int64_t* ld_y, int y_dtype, void* stream) {
  return multi_entry("gemv_multi_bf16", x, ld_x, nullptr, 0.f, nmat, weight, ld_w, n, bias,
                     bias_dtype, batch, K, y, ld_y, y_dtype, stream);
}

extern "C" int ml_gemv_rmsnorm_multi_bf16(const void* x, int64_t ld_x, const void* norm_weight,
                                          float eps, int nmat, const void* const* weight,
                                          const int64_t* ld_w, const int64_t* n,
                                          const void* const* bias, int bias_dtype, int64_t batch,
                                          int64_t K, void* const* y, const int64_t* ld_y,
                                          int y_dtype, void* stream) {
  ML_CHECK_ARG(norm_weight != nullptr, "gemv_rmsnorm_multi_bf16: null norm weight");
  return multi_entry("gemv_rmsnorm_multi_bf16", x, ld_x, norm_weight, eps, nmat, weight, ld_w, n,
                     bias, bias_dtype, batch, K, y, ld_y, y_dtype, stream);
}
