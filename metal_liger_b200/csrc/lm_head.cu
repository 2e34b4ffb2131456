// Greedy decoding head for the static-KV generator: next token = argmax over
// the vocabulary of hidden . W^T, without materialising the logits.
//
// Follows the reference's decode step (generation.py:99-126): logits =
// model(...).logits[:, -1, :] in the model's dtype, next = torch.argmax(
// logits, -1).  Here the lm_head product runs on the tcgen05 GEMM core with
// the EPI_ARGMAX epilogue: each tile's accumulator rows are rounded to the
// logit dtype (what the reference's logits hold) and reduced to (max, first
// column of it) per row; a one-warp-per-row kernel then reduces the tiles in
// the same order torch.argmax uses (NaN first, then value, then the lower
// index), so the choice is exactly argmax of the dtype-rounded fp32 logits.
// Decode is HBM-bound on W: one pass over [vocab, hidden] bf16 per step.
#include "gemm.cuh"
#include "gemv.cuh"

namespace ml {
namespace {

// index[r] / value[r] = torch.argmax order over the n_tiles candidates of
// row r.  One warp per row; lanes take every 32nd tile, then the warp reduces
// with the same total order (deterministic: no order of evaluation matters).
__global__ void argmax_reduce(const float* __restrict__ part_m, const int* __restrict__ part_i,
                              int n_tiles, int rows, int64_t* __restrict__ index,
                              float* __restrict__ value) {
  // Launched as a programmatic dependent of the GEMM that wrote the tiles.
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int warp = (int)((blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5);
  const int lane = threadIdx.x & 31;
  if (warp >= rows) return;
  float best = 0.f;
  int col = -1;
  for (int t = lane; t < n_tiles; t += 32) {
    const float x = part_m[(int64_t)t * rows + warp];
    const int c = part_i[(int64_t)t * rows + warp];
    if (c >= 0 && (col < 0 || gemm::argmax_better(x, c, best, col))) {
      best = x;
      col = c;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float xb = __shfl_xor_sync(0xffffffffu, best, o);
    const int cb = __shfl_xor_sync(0xffffffffu, col, o);
    if (cb >= 0 && (col < 0 || gemm::argmax_better(xb, cb, best, col))) {
      best = xb;
      col = cb;
    }
  }
  if (lane == 0) {
    index[warp] = col;
    if (value != nullptr) value[warp] = best;
  }
}

// Batch <= 2 (single-sequence greedy decoding): an HBM-streaming GEMV with
// the same argmax, no tensor cores.  At M = 1 the 128-row MMA tile is 1/128
// useful and the 256-column vocabulary tiles fall in 4 + 1/74 waves over 148
// SMs (a nearly empty fifth wave), while this kernel splits the vocabulary
// rows evenly over the SMs and streams each weight row once with 16-byte
// loads (16 per lane for hidden 4096, all in flight before use).  The hidden
// rows sit in shared memory as bf16; products are exact in fp32 and summed
// per lane, then across the warp by a fixed butterfly.  Each CTA writes one
// (max, column) candidate per sequence; argmax_reduce picks among CTAs.
template <int NB>
__global__ void __launch_bounds__(gemv::kThreads)
gemv_argmax(const __nv_bfloat16* __restrict__ hidden, int64_t ld_h,
            const __nv_bfloat16* __restrict__ weight, int64_t ld_w, const void* __restrict__ bias,
            int bias_dtype, int64_t H, int64_t V, int logit_dtype, float* __restrict__ part_m,
            int* __restrict__ part_i) {
  extern __shared__ uint4 hs[];  // [NB][H / 8] hidden chunks
  __shared__ float cand_v[gemv::kThreads / 32][NB];
  __shared__ int cand_c[gemv::kThreads / 32][NB];
  const int64_t nchunk = H / 8;
  gemv::stage_rows<NB>(hs, hidden, ld_h, nchunk);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nwarps = blockDim.x >> 5;
  const int64_t per = (V + gridDim.x - 1) / gridDim.x;
  const int64_t r0 = (int64_t)blockIdx.x * per;
  const int64_t r1 = r0 + per < V ? r0 + per : V;
  float best[NB];
  int col[NB];
#pragma unroll
  for (int b = 0; b < NB; ++b) {
    best[b] = 0.f;
    col[b] = -1;
  }
  for (int64_t r = r0 + warp; r < r1; r += nwarps) {
    const uint4* wrow = reinterpret_cast<const uint4*>(weight + r * ld_w);
    float acc[NB];
    gemv::row_dot<NB>(wrow, hs, nchunk, lane, acc);
#pragma unroll
    for (int b = 0; b < NB; ++b) {
      float v = warp_sum(acc[b]);
      if (bias != nullptr) v += load_as_f32(bias, r, bias_dtype);
      v = gemm::round_logit(v, logit_dtype);
      if (col[b] < 0 || gemm::argmax_better(v, (int)r, best[b], col[b])) {
        best[b] = v;
        col[b] = (int)r;
      }
    }
  }
  if (lane == 0) {
#pragma unroll
    for (int b = 0; b < NB; ++b) {
      cand_v[warp][b] = best[b];
      cand_c[warp][b] = col[b];
    }
  }
  __syncthreads();
  if (threadIdx.x < NB) {
    const int b = threadIdx.x;
    float bv = 0.f;
    int bc = -1;
    for (int w = 0; w < nwarps; ++w) {
      const int c = cand_c[w][b];
      if (c >= 0 && (bc < 0 || gemm::argmax_better(cand_v[w][b], c, bv, bc))) {
        bv = cand_v[w][b];
        bc = c;
      }
    }
    part_m[(int64_t)blockIdx.x * NB + b] = bv;
    part_i[(int64_t)blockIdx.x * NB + b] = bc;
  }
}

int64_t max_tiles(int64_t vocab) { return (vocab + 63) / 64; }

}  // namespace
}  // namespace ml

namespace ml {
namespace {
int launch_reduce(const float* part_m, const int* part_i, int n_tiles, int batch,
                  int64_t* index, float* value, cudaStream_t st) {
  cudaLaunchConfig_t lc = {};
  const int threads = 256;
  lc.gridDim = dim3(static_cast<unsigned>((batch * 32 + threads - 1) / threads), 1, 1);
  lc.blockDim = dim3(threads, 1, 1);
  lc.dynamicSmemBytes = 0;
  lc.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  lc.attrs = attr;
  lc.numAttrs = 1;
  ML_CHECK_CUDA(cudaLaunchKernelEx(&lc, argmax_reduce, part_m, part_i, n_tiles, batch, index,
                                   value),
                "lm_head_argmax(reduce)");
  return ML_OK;
}
}  // namespace
}  // namespace ml

using namespace ml;

extern "C" size_t ml_lm_head_argmax_workspace_bytes(int64_t batch, int64_t vocab) {
  if (batch <= 0 || vocab <= 0) return 0;
  return (size_t)max_tiles(vocab) * (size_t)batch * (sizeof(float) + sizeof(int)) + 16;
}

extern "C" int ml_lm_head_argmax(const void* hidden, int64_t ld_hidden, const void* weight,
                                 int64_t ld_weight, const void* bias, int bias_dtype,
                                 int64_t batch, int64_t hidden_size, int64_t vocab,
                                 int logit_dtype, int64_t* index, float* value, void* workspace,
                                 size_t workspace_bytes, void* stream) {
  ML_CHECK_ARG(batch >= 0 && hidden_size > 0 && vocab > 0,
               "lm_head_argmax: bad sizes batch=%lld hidden=%lld vocab=%lld", (long long)batch,
               (long long)hidden_size, (long long)vocab);
  ML_CHECK_ARG(vocab < ((int64_t)1 << 31), "lm_head_argmax: vocab %lld too large",
               (long long)vocab);
  ML_CHECK_ARG(logit_dtype == ML_DTYPE_F32 || logit_dtype == ML_DTYPE_BF16 ||
                   logit_dtype == ML_DTYPE_F16,
               "lm_head_argmax: bad logit dtype %d", logit_dtype);
  if (batch == 0) return ML_OK;
  ML_CHECK_ARG(hidden && weight && index, "lm_head_argmax: null pointer");
  ML_CHECK_ARG(bias == nullptr || bias_dtype == ML_DTYPE_F32 || bias_dtype == ML_DTYPE_BF16 ||
                   bias_dtype == ML_DTYPE_F16,
               "lm_head_argmax: bad bias dtype %d", bias_dtype);
  ML_CHECK_ARG(ld_hidden >= hidden_size && ld_weight >= hidden_size,
               "lm_head_argmax: row pitches (%lld, %lld) below hidden %lld",
               (long long)ld_hidden, (long long)ld_weight, (long long)hidden_size);
  const int64_t n_tiles_max = max_tiles(vocab);
  ML_CHECK_ARG(workspace != nullptr && aligned16(workspace) &&
                   workspace_bytes >= ml_lm_head_argmax_workspace_bytes(batch, vocab),
               "lm_head_argmax: workspace must be 16-byte aligned and >= %zu bytes",
               ml_lm_head_argmax_workspace_bytes(batch, vocab));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  float* part_m = static_cast<float*>(workspace);
  int* part_i = reinterpret_cast<int*>(part_m + n_tiles_max * batch);

  const int sms = num_sms();
  if (gemv::eligible(batch, hidden_size, ld_hidden, ld_weight, hidden, weight) &&
      n_tiles_max >= sms) {
    const size_t smem = (size_t)batch * hidden_size * 2;
    auto launch_gemv = [&](auto kernel) -> int {
      if (smem > 48 * 1024)
        ML_CHECK_CUDA(cudaFuncSetAttribute((const void*)kernel,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           96 * 1024),
                      "lm_head_argmax: smem attribute");
      kernel<<<sms, gemv::kThreads, smem, st>>>(
          static_cast<const __nv_bfloat16*>(hidden), ld_hidden,
          static_cast<const __nv_bfloat16*>(weight), ld_weight, bias, bias_dtype, hidden_size,
          vocab, logit_dtype, part_m, part_i);
      ML_CHECK_LAUNCH("lm_head_argmax(gemv)");
      return ML_OK;
    };
    if (int rc = batch == 1 ? launch_gemv(gemv_argmax<1>) : launch_gemv(gemv_argmax<2>))
      return rc;
    return launch_reduce(part_m, part_i, sms, (int)batch, index, value, st);
  }

  gemm::Problem pr;
  pr.M = batch;
  pr.N = vocab;
  pr.nseg = 1;
  pr.seg[0].a = {hidden, batch, hidden_size, ld_hidden};
  pr.seg[0].b = {weight, vocab, hidden_size, ld_weight};
  pr.seg[0].K = hidden_size;
  // The tile width is fixed here so the reduction knows the tile count
  // whatever GEMM kernel the launcher picks.  (Narrower tiles fill the last
  // wave better for Qwen3-VL's 151,936 columns but were measured slower:
  // batch 8, 245 us at 256 columns vs 498 us at 64.)
  const int bn = gemm::pick_bn(vocab);
  pr.bn = bn;
  pr.epi = gemm::EPI_ARGMAX;
  pr.part_m = part_m;
  pr.part_i = part_i;
  pr.bias = bias;
  pr.bias_dtype = bias_dtype;
  pr.logit_dtype = logit_dtype;
  if (int rc = gemm::launch(pr, st)) return rc;
  return launch_reduce(part_m, part_i, (int)((vocab + bn - 1) / bn), (int)batch, index, value,
                       st);
}

