// Decode-time linear layers: y[b, n] = sum_k x[b, k] * W[n, k] (+ bias[n])
// for one or two activation rows, HBM-streaming (gemv.cuh).  The greedy
// generator routes the decoder's bf16 nn.Linear calls through this while it
// decodes (one token per sequence per step), where a tensor-core tile would
// be 1/128 useful and the step is a pass over the weights.
//
// Rows of W go to warps round-robin with the CTA index fastest, so even a
// 1,024-row projection spreads its rows over every SM (each busy warp keeps
// 8 KB of one row in flight: 8 MB across the GPU for hidden 4096).
#include "gemv.cuh"

namespace ml {
namespace {

template <int NB, typename TO>
__global__ void __launch_bounds__(gemv::kThreads)
gemv_rows(const __nv_bfloat16* __restrict__ x, int64_t ld_x,
          const __nv_bfloat16* __restrict__ weight, int64_t ld_w, const void* __restrict__ bias,
          int bias_dtype, int64_t K, int64_t N, TO* __restrict__ y, int64_t ld_y) {
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
      if (lane == 0) y[b * ld_y + r] = from_f32<TO>(v);
    }
  }
}

template <int NB, typename TO>
int launch_rows(const void* x, int64_t ld_x, const void* w, int64_t ld_w, const void* bias,
                int bias_dtype, int64_t K, int64_t N, void* y, int64_t ld_y, cudaStream_t st) {
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
                                        bias_dtype, K, N, static_cast<TO*>(y), ld_y);
  ML_CHECK_LAUNCH("gemv_bf16");
  return ML_OK;
}

}  // namespace
}  // namespace ml

using namespace ml;

extern "C" int ml_gemv_bf16(const void* x, int64_t ld_x, const void* weight, int64_t ld_w,
                            const void* bias, int bias_dtype, int64_t batch, int64_t K, int64_t N,
                            void* y, int y_dtype, int64_t ld_y, void* stream) {
  ML_CHECK_ARG(batch >= 0 && K > 0 && N > 0, "gemv_bf16: bad sizes batch=%lld K=%lld N=%lld",
               (long long)batch, (long long)K, (long long)N);
  if (batch == 0) return ML_OK;
  ML_CHECK_ARG(x && weight && y, "gemv_bf16: null pointer");
  ML_CHECK_ARG(gemv::eligible(batch, K, ld_x, ld_w, x, weight),
               "gemv_bf16: needs 1-2 rows, K and row pitches multiples of 8, 16-byte aligned "
               "bases and rows*K*2 <= 96 KiB (batch=%lld K=%lld)",
               (long long)batch, (long long)K);
  ML_CHECK_ARG(y_dtype == ML_DTYPE_BF16 || y_dtype == ML_DTYPE_F32,
               "gemv_bf16: output dtype %d is neither bf16 nor fp32", y_dtype);
  ML_CHECK_ARG(bias == nullptr || bias_dtype == ML_DTYPE_F32 || bias_dtype == ML_DTYPE_BF16 ||
                   bias_dtype == ML_DTYPE_F16,
               "gemv_bf16: bad bias dtype %d", bias_dtype);
  ML_CHECK_ARG(ld_y >= N, "gemv_bf16: output pitch %lld below N %lld", (long long)ld_y,
               (long long)N);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (y_dtype == ML_DTYPE_BF16)
    return batch == 1 ? launch_rows<1, __nv_bfloat16>(x, ld_x, weight, ld_w, bias, bias_dtype, K,
                                                      N, y, ld_y, st)
                      : launch_rows<2, __nv_bfloat16>(x, ld_x, weight, ld_w, bias, bias_dtype, K,
                                                      N, y, ld_y, st);
  return batch == 1
             ? launch_rows<1, float>(x, ld_x, weight, ld_w, bias, bias_dtype, K, N, y, ld_y, st)
             : launch_rows<2, float>(x, ld_x, weight, ld_w, bias, bias_dtype, K, N, y, ld_y, st);
}
