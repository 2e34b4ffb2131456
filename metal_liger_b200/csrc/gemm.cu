// Host side of the tcgen05 GEMM: tensor-map encoding, tile-width choice,
// kernel instantiations, split-K reduction and the generic C-ABI GEMM entry.
#include "gemm.cuh"

#include <algorithm>
#include <atomic>
#include <initializer_list>
#include <mutex>

namespace ml {
namespace gemm {

// Device-wide error word written by bounded waits that gave up (0 = none).
__device__ int g_device_error = 0;

int* device_error_word() {
  static std::mutex mu;
  static int* cache[64] = {nullptr};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  std::lock_guard<std::mutex> lock(mu);
  if (cache[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_device_error) != cudaSuccess) return nullptr;
    cache[dev] = static_cast<int*>(p);
  }
  return cache[dev];
}

namespace {

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// 2-D bf16 tensor map over a row-major matrix: inner extent `inner`
// (contiguous), outer extent `outer`, row pitch `ld` elements; box
// {64, box_outer} with 128-byte swizzle; out-of-range elements read as zero.
int make_map(CUtensorMap* map, const void* ptr, int64_t inner, int64_t outer, int64_t ld,
             int box_outer, const char* what) {
  EncodeTiledFn enc = encode_fn();
  if (enc == nullptr) {
    set_error("%s: cuTensorMapEncodeTiled unavailable from the driver", what);
    return ML_ERR_CUDA;
  }
  if (ptr == nullptr || !aligned16(ptr)) {
    set_error("%s: operand pointer must be non-null and 16-byte aligned", what);
    return ML_ERR_INVALID_ARG;
  }
  if (inner <= 0 || outer <= 0 || ld < inner || (ld * 2) % 16 != 0) {
    set_error("%s: bad operand shape (inner=%lld outer=%lld ld=%lld; ld must be a multiple of 8)",
              what, (long long)inner, (long long)outer, (long long)ld);
    return ML_ERR_INVALID_ARG;
  }
  cuuint64_t gdim[2] = {(cuuint64_t)inner, (cuuint64_t)outer};
  cuuint64_t gstride[1] = {(cuuint64_t)(ld * 2)};
  cuuint32_t box[2] = {64u, (cuuint32_t)box_outer};
  cuuint32_t estride[2] = {1u, 1u};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), gdim, gstride,
                   box, estride, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("%s: cuTensorMapEncodeTiled failed (%d)", what, (int)r);
    return ML_ERR_CUDA;
  }
  return ML_OK;
}

template <int BN, bool A_MN, bool B_MN>
int launch_t(const Params& prm, int grid, cudaStream_t st) {
  auto k = gemm_kernel<BN, A_MN, B_MN>;
  const size_t smem = Cfg<BN>::SMEM;
  static PerDevice<cudaError_t> attr;
  const cudaError_t attr_err = attr.get([&] {
    return cudaFuncSetAttribute((const void*)k, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                (int)smem);
  });
  if (attr_err != cudaSuccess) {
    set_error("gemm: cudaFuncSetAttribute failed: %s", cudaGetErrorString(attr_err));
    return ML_ERR_CUDA;
  }
  ML_CHECK_CUDA(launch_pdl(k, dim3(grid), dim3(kThreads), smem, st, prm), "gemm_kernel");
  return ML_OK;
}

std::atomic<int> g_pair_mode{-1};
// SMs every GEMM leaves free (ml_gemm_set_reserved_sms): its persistent grid
// then stops short of the whole GPU, so a kernel on another stream — an
// NCCL collective overlapping the GEMM — finds SMs to run on.
std::atomic<int> g_reserved_sms{0};

template <int BN, bool A_MN, bool B_MN>
int launch_pair_t(const Params& prm, int64_t units, int max_ctas, cudaStream_t st) {
  auto k = gemm_pair_kernel<BN, A_MN, B_MN>;
  const size_t smem = PairCfg<BN>::SMEM;
  // Per device: the smem attribute, then how many CTA pairs fit at once (GPC
  // boundaries can leave an SM unpaired); -1 = the attribute failed.
  static PerDevice<int> setup;
  const int resident_pairs = setup.get([&]() -> int {
    if (cudaFuncSetAttribute((const void*)k, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)smem) != cudaSuccess) {
      cudaGetLastError();
      return -1;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * (unsigned)(num_sms() / 2), 1, 1);
    cfg.blockDim = dim3(kThreads, 1, 1);
    cfg.dynamicSmemBytes = smem;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, (const void*)k, &cfg) != cudaSuccess || n <= 0) {
      cudaGetLastError();
      n = num_sms() / 2;
    }
    return n;
  });
  const cudaError_t attr_err = resident_pairs < 0 ? cudaErrorInvalidValue : cudaSuccess;
  if (attr_err != cudaSuccess) {
    set_error("gemm(pair): cudaFuncSetAttribute failed: %s", cudaGetErrorString(attr_err));
    return ML_ERR_CUDA;
  }
  int64_t pairs = std::min<int64_t>(units, resident_pairs);
  if (max_ctas > 0) pairs = std::min<int64_t>(pairs, max_ctas / 2);
  const int grid = 2 * (int)std::max<int64_t>(pairs, 1);
  ML_CHECK_CUDA(launch_pdl(k, dim3(grid), dim3(kThreads), smem, st, prm), "gemm_pair_kernel");
  return ML_OK;
}

template <int BN>
int launch_pair_bn(const Params& prm, bool a_mn, bool b_mn, int64_t units, int max_ctas,
                   cudaStream_t st) {
  if (!a_mn && !b_mn) return launch_pair_t<BN, false, false>(prm, units, max_ctas, st);
  if (!a_mn && b_mn) return launch_pair_t<BN, false, true>(prm, units, max_ctas, st);
  if (a_mn && !b_mn) return launch_pair_t<BN, true, false>(prm, units, max_ctas, st);
  return launch_pair_t<BN, true, true>(prm, units, max_ctas, st);
}

int launch_pair(const Params& prm, int bn, bool a_mn, bool b_mn, int64_t units, int max_ctas,
                cudaStream_t st) {
  return bn == 256 ? launch_pair_bn<256>(prm, a_mn, b_mn, units, max_ctas, st)
                   : launch_pair_bn<128>(prm, a_mn, b_mn, units, max_ctas, st);
}

// Tile choice, from B200 measurements of both kernels over the shapes of
// this library (bf16, 64-deep k-blocks).  In isolation (short bursts at full
// clock) the CTA-pair kernel with 256 x 256 tiles is 8-28% faster on large
// problems (8192^3: 1.47 vs 1.35 PFLOP/s; FLCE logits / dW shapes: +27%; the
// 1-SM 128 x 256 tile is limited by shared-memory bandwidth) and 3-7% slower
// on a few waves (4096^3).  Inside a long training step, which runs under the
// 1 kW power cap, the pair kernel is the faster one at every size measured:
// it moves fewer shared-memory and L2 bytes per FLOP, so the cap leaves it a
// higher clock (Qwen3-VL-8B LoRA step: 163.6 ms with the pair kernel on every
// GEMM it can take vs 171.0 ms with the burst-tuned split).  So the pair
// kernel takes every GEMM with 256-wide tiles and more than 128 rows.  Its
// 128-wide tile is smem-bound (about half the 256-wide throughput) and is
// used only when forced.
// `mode` (ml_gemm_set_cta_pair): -1 auto, 0 1-SM only, 1 pair when possible,
// 2 / 3 pair with 256 / 128-wide tiles only (tuning and tests).
struct TileChoice {
  int bn;
  bool pair;
};

TileChoice choose_tile(const Problem& pr, int mode) {
  const int one_bn = pr.bn ? pr.bn : pick_bn(pr.N);
  const bool pair_ok = mode != 0 && pr.M > BM;
  const bool w256 = pr.bn ? pr.bn == 256 : pr.N > 128;
  const bool w128 = pr.bn ? pr.bn == 128 : (pr.N > 64 && pr.epi != EPI_FLCE);
  if (mode == 3) return w128 && pair_ok ? TileChoice{128, true} : TileChoice{one_bn, false};
  if (mode == 1 || mode == 2) {
    if (pair_ok && w256) return {256, true};
    if (pair_ok && w128 && mode == 1) return {128, true};
    return {one_bn, false};
  }
  if (mode == 0 || !pair_ok || !w256) return {one_bn, false};
  return {256, true};
}

template <int BN>
int launch_bn(const Params& prm, bool a_mn, bool b_mn, int grid, cudaStream_t st) {
  if (!a_mn && !b_mn) return launch_t<BN, false, false>(prm, grid, st);
  if (!a_mn && b_mn) return launch_t<BN, false, true>(prm, grid, st);
  if (a_mn && !b_mn) return launch_t<BN, true, false>(prm, grid, st);
  return launch_t<BN, true, true>(prm, grid, st);
}
}  // namespace

int pick_bn(int64_t N) {
  if (N > 128) return 256;
  if (N > 64) return 128;
  return 64;
}

int launch(const Problem& pr, cudaStream_t st) {
  if (pr.M <= 0 || pr.N <= 0 || pr.nseg <= 0 || pr.nseg > kMaxSeg) {
    set_error("gemm: bad problem (M=%lld N=%lld nseg=%d)", (long long)pr.M, (long long)pr.N,
              pr.nseg);
    return ML_ERR_INVALID_ARG;
  }
  const bool grouped = pr.m_groups > 1;
  if (grouped) {
    if (pr.m_groups > kMaxSeg || pr.nseg != pr.m_groups || pr.b_split ||
        (pr.epi != EPI_PARTIAL && pr.epi != EPI_STORE)) {
      set_error("gemm: grouped GEMM needs 2..%d groups, one segment each, a store or "
                "partial epilogue", kMaxSeg);
      return ML_ERR_INVALID_ARG;
    }
    int64_t total = 0;
    for (int g = 0; g < pr.m_groups; ++g) {
      if (pr.grp_m[g] <= 0 || pr.seg[g].K != pr.seg[0].K) {
        set_error("gemm: grouped GEMM needs rows in every group and one K for all");
        return ML_ERR_INVALID_ARG;
      }
      total += pr.grp_m[g];
    }
    if (total != pr.M) {
      set_error("gemm: grouped GEMM rows do not add up to M");
      return ML_ERR_INVALID_ARG;
    }
  }
  const int mode = grouped ? 0 : (pr.pair >= 0 ? pr.pair : g_pair_mode.load(std::memory_order_relaxed));
  const TileChoice tc = choose_tile(pr, mode);
  const int bn = tc.bn;
  const bool pair = tc.pair;
  if (bn != 64 && bn != 128 && bn != 256) {
    set_error("gemm: bad tile width %d", bn);
    return ML_ERR_INVALID_ARG;
  }
  if (pr.epi == EPI_FLCE && bn != 256) {
    set_error("gemm: the FLCE epilogue needs 256-wide tiles");
    return ML_ERR_INVALID_ARG;
  }
  if ((pr.b_split || pr.epi == EPI_SWIGLU) &&
      (!pr.b_split || pr.epi != EPI_SWIGLU || bn != 256 || pr.b_mn)) {
    set_error("gemm: the SwiGLU epilogue takes split K-major B operands on 256-wide tiles");
    return ML_ERR_INVALID_ARG;
  }
  if ((pr.epi == EPI_SWIGLU && (pr.D == nullptr || pr.D2 == nullptr || pr.D3 == nullptr)) ||
      (pr.epi == EPI_DSWIGLU && (pr.D == nullptr || pr.D2 == nullptr || pr.aux1 == nullptr ||
                                 pr.aux2 == nullptr))) {
    set_error("gemm: SwiGLU epilogue with a null output or input");
    return ML_ERR_INVALID_ARG;
  }
  Params prm;
  memset(&prm, 0, sizeof(prm));
  int kb_total = 0;
  for (int s = 0; s < pr.nseg; ++s) {
    const Seg& g = pr.seg[s];
    if (g.K <= 0) {
      set_error("gemm: segment %d has K=%lld", s, (long long)g.K);
      return ML_ERR_INVALID_ARG;
    }
    int rc;
    // A: logical [M, K] (a grouped GEMM's group s: its own grp_m[s] rows)
    const int64_t am = grouped ? pr.grp_m[s] : pr.M;
    if (!pr.a_mn)
      rc = make_map(&prm.tma_a[s], g.a.ptr, g.K, am, g.a.ld, BM, "gemm A (K-major)");
    else
      rc = make_map(&prm.tma_a[s], g.a.ptr, am, g.K, g.a.ld, BK, "gemm A (M-major)");
    if (rc) return rc;
    // B: logical [N, K]; each CTA of a pair loads 128 of the tile's 256 rows.
    // Split B: two [N, K] matrices, half a tile's rows from each.
    if (pr.b_split) {
      rc = make_map(&prm.tma_b[s], g.b.ptr, g.K, pr.N, g.b.ld, bn / 2, "gemm B (split, first)");
      if (rc) return rc;
      rc = make_map(&prm.tma_b2[s], g.b2.ptr, g.K, pr.N, g.b2.ld, bn / 2,
                    "gemm B (split, second)");
    } else if (!pr.b_mn) {
      rc = make_map(&prm.tma_b[s], g.b.ptr, g.K, pr.N, g.b.ld, pair ? bn / 2 : bn,
                    "gemm B (K-major)");
    } else {
      rc = make_map(&prm.tma_b[s], g.b.ptr, pr.N, g.K, g.b.ld, BK, "gemm B (N-major)");
    }
    if (rc) return rc;
    prm.seg_kb[s] = (int)((g.K + BK - 1) / BK);
    kb_total += prm.seg_kb[s];
  }
  prm.nseg = pr.nseg;
  prm.M = (int)pr.M;
  prm.N = (int)pr.N;
  prm.m_tiles = (int)((pr.M + (pair ? 2 * BM : BM) - 1) / (pair ? 2 * BM : BM));
  prm.m_groups = grouped ? pr.m_groups : 1;
  if (grouped) {
    kb_total = prm.seg_kb[0];  // the groups share one K range
    int mt = 0, row = 0;
    for (int g = 0; g < pr.m_groups; ++g) {
      prm.grp_mt0[g] = mt;
      prm.grp_row0[g] = row;
      prm.grp_m[g] = (int)pr.grp_m[g];
      mt += (int)((pr.grp_m[g] + BM - 1) / BM);
      row += (int)pr.grp_m[g];
    }
    prm.grp_mt0[pr.m_groups] = mt;
    prm.m_tiles = mt;
  }
  const int tile_n = pr.b_split ? bn / 2 : bn;  // columns of N per tile
  prm.n_tiles = (int)((pr.N + tile_n - 1) / tile_n);
  prm.b_split = pr.b_split ? 1 : 0;
  int splits = std::max(1, std::min(pr.splits, kb_total));
  const int kb_per = (kb_total + splits - 1) / splits;
  splits = (kb_total + kb_per - 1) / kb_per;
  if (pr.epi != EPI_PARTIAL && splits != 1) {
    set_error("gemm: split-K needs the partial epilogue");
    return ML_ERR_INVALID_ARG;
  }
  prm.splits = splits;
  prm.kb_per_split = kb_per;
  prm.kb_total = kb_total;
  prm.raster = pr.raster;
  prm.group_m = pr.group_m;
  if (pr.raster == 0 && pr.group_m == 0 && prm.n_tiles > 1) {
    // M-fastest raster re-reads all of A once per N-tile column.  When A does
    // not fit comfortably in L2, sweep the N-tiles in groups of M-tiles whose
    // A rows stay resident, so A is read from HBM about once and B once per
    // group.  Group size, from ncu DRAM counts on the LoRA shapes: with short
    // K (A rows of a 256-row tile <= 4 MB) up to ~48 MB of A per group cuts
    // the B sweeps (gate/up 16384 x 12288 x 4160: 1.18 -> 0.85 GB per launch,
    // less DRAM energy under the power cap); with long K the larger groups
    // thrash L2 (dX 16384 x 4096 x 24640: 3.9 -> 6.2 GB), so ~16 MB.
    int64_t k_total = 0;
    for (int s = 0; s < pr.nseg; ++s) k_total += pr.seg[s].K;
    const int64_t a_bytes_per_mtile = (int64_t)(pair ? 2 * BM : BM) * k_total * 2;
    if ((int64_t)prm.m_tiles * a_bytes_per_mtile > ((int64_t)48 << 20)) {
      const int64_t target = a_bytes_per_mtile <= ((int64_t)4 << 20) ? ((int64_t)48 << 20)
                                                                         : ((int64_t)16 << 20);
      const int64_t g = std::max<int64_t>(1, target / a_bytes_per_mtile);
      prm.group_m = (int)std::min<int64_t>(g, prm.m_tiles);
    }
  }
  prm.epi = pr.epi;
  prm.d_f32 = pr.d_f32 ? 1 : 0;
  prm.D = pr.D;
  prm.ldd = pr.ldd;
  prm.alpha = pr.alpha;
  prm.beta = pr.beta;
  const bool bf16_out = (pr.epi == EPI_STORE && !pr.d_f32) || pr.epi == EPI_FLCE ||
                        pr.epi == EPI_SWIGLU || pr.epi == EPI_DSWIGLU;
  const int elt = bf16_out ? 2 : 4;
  prm.vec_ok = aligned16(pr.D) && ((pr.ldd * elt) % 16 == 0);
  for (const void* q : std::initializer_list<const void*>{pr.D2, pr.D3, pr.aux1, pr.aux2})
    if (q != nullptr && !aligned16(q)) prm.vec_ok = 0;
  prm.D2 = pr.D2;
  prm.D3 = pr.D3;
  prm.aux1 = pr.aux1;
  prm.aux2 = pr.aux2;
  prm.peer_n = 0;
  if (pr.peer_n > 0) {
    if (pr.epi != EPI_STORE || !pr.d_f32 || pr.beta != 0.f || pr.peer_n > kMaxPeers ||
        pr.peer_me < 0 || pr.peer_me >= pr.peer_n || pr.peer_rows <= 0 ||
        pr.peer_rows * pr.peer_n < pr.M || pr.peer_rows > 0x7fffffff) {
      set_error("gemm: bad peer-store request");
      return ML_ERR_INVALID_ARG;
    }
    prm.vec_ok = (pr.ldd * 4) % 16 == 0;
    for (int o = 0; o < pr.peer_n; ++o) {
      if (pr.peer_dst[o] == nullptr) {
        set_error("gemm: null peer destination %d", o);
        return ML_ERR_INVALID_ARG;
      }
      if (!aligned16(pr.peer_dst[o])) prm.vec_ok = 0;
      prm.peer_dst[o] = pr.peer_dst[o];
    }
    prm.peer_n = pr.peer_n;
    prm.peer_me = pr.peer_me;
    prm.peer_rows = (int)pr.peer_rows;
  }
  prm.labels = pr.labels;
  prm.label_base = pr.label_base;
  prm.ignore_index = pr.ignore_index;
  prm.part_m = pr.part_m;
  prm.part_s = pr.part_s;
  prm.tgt = pr.tgt;
  prm.vocab = pr.N;
  prm.bias = pr.bias;
  prm.bias_dtype = pr.bias_dtype;
  prm.part_i = pr.part_i;
  prm.logit_dtype = pr.logit_dtype;
  prm.split_stride = pr.split_stride ? pr.split_stride : pr.M * pr.ldd;
  prm.err = device_error_word();
  const int64_t units = (int64_t)prm.m_tiles * prm.n_tiles * prm.splits;
  if (units > 0x7fffffff) {
    set_error("gemm: problem too large");
    return ML_ERR_INVALID_ARG;
  }
  int max_ctas = pr.max_ctas;
  const int reserved = g_reserved_sms.load(std::memory_order_relaxed);
  if (reserved > 0) {
    const int avail = std::max(2, num_sms() - reserved);
    max_ctas = max_ctas > 0 ? std::min(max_ctas, avail) : avail;
  }
  if (pair) return launch_pair(prm, bn, pr.a_mn, pr.b_mn, units, max_ctas, st);
  int grid = (int)std::min<int64_t>(units, max_ctas > 0 ? max_ctas : num_sms());
  grid = std::max(grid, 1);
  switch (bn) {
    case 64: return launch_bn<64>(prm, pr.a_mn, pr.b_mn, grid, st);
    case 128: return launch_bn<128>(prm, pr.a_mn, pr.b_mn, grid, st);
    default: return launch_bn<256>(prm, pr.a_mn, pr.b_mn, grid, st);
  }
}

}  // namespace gemm

namespace {

// D[m, n] = sum_s partial[s][m][n] (+ beta * D), fixed summation order.
__global__ void splitk_reduce(const float* __restrict__ part, int splits, int64_t M, int64_t N,
                              int64_t ldp, void* __restrict__ D, int64_t ldd, int d_f32,
                              float beta) {
  // Launched as a programmatic dependent of the GEMM that wrote `part`; the
  // next programmatic dependent may start launching once this wait returns.
  pdl_wait();
  pdl_release();
  const int64_t total = M * N;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t m = i / N, n = i - (i / N) * N;
    float s = 0.f;
    for (int k = 0; k < splits; ++k) s += part[((int64_t)k * M + m) * ldp + n];
    if (d_f32) {
      float* d = static_cast<float*>(D) + m * ldd + n;
      *d = s + (beta != 0.f ? *d : 0.f);
    } else {
      __nv_bfloat16* d = static_cast<__nv_bfloat16*>(D) + m * ldd + n;
      *d = __float2bfloat16_rn(s + (beta != 0.f ? __bfloat162float(*d) : 0.f));
    }
  }
}

}  // namespace

namespace gemm {

// Split count for a GEMM with fewer tiles than SMs: the s in [1, 16] (each
// split keeping >= 4 k-blocks) whose tiles * s units keep the largest share
// of SM slots busy over whole waves; ties go to the smaller s.  E.g. 32 tiles
// on 148 SMs: s = 9 (288 units, 97% of two waves) rather than s = 10 (320
// units, a third wave 16% full).
int auto_splits(int64_t M, int64_t N, int64_t K) {
  const int bn = pick_bn(N);
  const int64_t tiles = ((M + BM - 1) / BM) * ((N + bn - 1) / bn);
  const int64_t kb = (K + BK - 1) / BK;
  const int64_t sms = num_sms();
  if (tiles >= sms || kb < 8) return 1;
  int64_t best = 1;
  double best_busy = 0.0;
  const int64_t smax = std::max<int64_t>(1, std::min<int64_t>(16, kb / 4));
  for (int64_t s = 1; s <= smax; ++s) {
    const int64_t per = (kb + s - 1) / s;
    const int64_t actual = (kb + per - 1) / per;  // what launch() will run
    const int64_t units = tiles * actual;
    const int64_t waves = (units + sms - 1) / sms;
    const double busy = (double)units / (double)(waves * sms);
    if (busy > best_busy + 1e-9) {
      best_busy = busy;
      best = actual;
    }
  }
  return (int)best;
}

int launch_splitk(Problem pr, int splits, float* out, int64_t ldo, float* partial,
                  size_t partial_bytes, cudaStream_t st) {
  return launch_splitk_to(pr, splits, out, true, ldo, partial, partial_bytes, st);
}

int launch_splitk_to(Problem pr, int splits, void* out, bool out_f32, int64_t ldo,
                     float* partial, size_t partial_bytes, cudaStream_t st) {
  if (splits <= 1) {
    pr.epi = EPI_STORE;
    pr.d_f32 = out_f32;
    pr.D = out;
    pr.ldd = ldo;
    pr.splits = 1;
    return launch(pr, st);
  }
  if (partial == nullptr ||
      partial_bytes < (size_t)splits * (size_t)pr.M * (size_t)pr.N * sizeof(float)) {
    set_error("gemm split-K: partial buffer too small");
    return ML_ERR_INVALID_ARG;
  }
  pr.epi = EPI_PARTIAL;
  pr.splits = splits;
  pr.D = partial;
  pr.ldd = pr.N;
  pr.split_stride = pr.M * pr.N;
  pr.d_f32 = true;
  int rc = launch(pr, st);
  if (rc) return rc;
  const int64_t total = pr.M * pr.N;
  int grid = (int)std::min<int64_t>((total + 255) / 256, (int64_t)num_sms() * 8);
  // Programmatic dependent launch: the reduction's launch overlaps the GEMM's
  // tail; it waits (griddepcontrol.wait) for the GEMM grid before reading.
  cudaLaunchConfig_t lc = {};
  lc.gridDim = dim3((unsigned)std::max(grid, 1), 1, 1);
  lc.blockDim = dim3(256, 1, 1);
  lc.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  lc.attrs = attr;
  lc.numAttrs = 1;
  ML_CHECK_CUDA(cudaLaunchKernelEx(&lc, splitk_reduce, (const float*)partial, splits, pr.M, pr.N,
                                   (int64_t)pr.N, out, ldo, out_f32 ? 1 : 0, 0.f),
                "gemm split-K reduce");
  return ML_OK;
}

}  // namespace gemm

namespace {

int choose_splits(int64_t m, int64_t n, int64_t k_total, int bn) {
  const int64_t tiles = ((m + gemm::BM - 1) / gemm::BM) * ((n + bn - 1) / bn);
  const int64_t kb = (k_total + gemm::BK - 1) / gemm::BK;
  const int sms = num_sms();
  if (tiles * 2 > sms || kb < 16) return 1;
  int64_t s = std::min<int64_t>((sms + tiles - 1) / tiles, kb / 8);
  return (int)std::max<int64_t>(1, std::min<int64_t>(s, 16));
}

}  // namespace
}  // namespace ml

namespace ml {
namespace gemm {
namespace {

// Self-test of the bounded-wait path the tcgen05 kernels use: one thread
// waits on an mbarrier phase that nothing completes, through
// sm100::mbar_wait_bounded with the limit shortened to `limit_ns`; the wait
// gives up, records (SITE_SELFTEST << 8) | ML_ERR_TIMEOUT in the device error
// word, and the kernel returns normally (no trap, the context stays usable).
__global__ void selftest_bounded_wait(uint64_t limit_ns, int* err) {
  __shared__ __align__(8) uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    sm100::mbar_init(&bar, 1);
    abort_flag = 0;
    sm100::fence_barrier_init();
  }
  __syncthreads();
  if (threadIdx.x == 0)
    (void)sm100::mbar_wait_bounded(&bar, 0, &abort_flag, err, SITE_SELFTEST, limit_ns);
}

}  // namespace
}  // namespace gemm
}  // namespace ml

using namespace ml;

extern "C" int ml_selftest_bounded_wait(int64_t limit_us, void* stream) {
  ML_CHECK_ARG(limit_us >= 1000 && limit_us <= 1000000,
               "selftest_bounded_wait: limit %lld us outside [1 ms, 1 s]", (long long)limit_us);
  int* err = gemm::device_error_word();
  if (err == nullptr) {
    set_error("selftest_bounded_wait: device error word unavailable");
    return ML_ERR_CUDA;
  }
  gemm::selftest_bounded_wait<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(
      (uint64_t)limit_us * 1000ull, err);
  ML_CHECK_LAUNCH("selftest_bounded_wait");
  return ML_OK;
}

extern "C" int ml_device_error(void* stream) {
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int h = 0;
  ML_CHECK_CUDA(cudaStreamSynchronize(st), "device_error: sync");
  ML_CHECK_CUDA(cudaMemcpyFromSymbol(&h, gemm::g_device_error, sizeof(int)), "device_error: read");
  if (h != 0) {
    const int zero = 0;
    ML_CHECK_CUDA(cudaMemcpyToSymbol(gemm::g_device_error, &zero, sizeof(int)),
                  "device_error: clear");
  }
  return h;
}

extern "C" size_t ml_gemm_bf16_workspace_bytes(int64_t m, int64_t n, int64_t k_total) {
  if (m <= 0 || n <= 0 || k_total <= 0) return 0;
  const int s = choose_splits(m, n, k_total, gemm::pick_bn(n));
  return s > 1 ? (size_t)s * (size_t)m * (size_t)n * sizeof(float) : 0;
}

extern "C" int ml_gemm_set_reserved_sms(int n, int* previous) {
  ML_CHECK_ARG(n >= 0 && n <= 128, "gemm_set_reserved_sms: n must be in [0, 128]");
  const int old = gemm::g_reserved_sms.exchange(n);
  if (previous) *previous = old;
  return ML_OK;
}

extern "C" int ml_gemm_set_cta_pair(int mode, int* previous) {
  ML_CHECK_ARG(mode >= -1 && mode <= 3, "gemm_set_cta_pair: mode must be in [-1, 3]");
  const int old = gemm::g_pair_mode.exchange(mode);
  if (previous) *previous = old;
  return ML_OK;
}

extern "C" int ml_gemm_bf16(int64_t m, int64_t n, const ml_gemm_segment* segs, int nseg, void* d,
                            int d_dtype, int64_t ldd, float alpha, float beta, void* workspace,
                            size_t workspace_bytes, void* stream) {
  ML_CHECK_ARG(m >= 0 && n >= 0, "gemm: negative sizes");
  ML_CHECK_ARG(nseg >= 1 && nseg <= gemm::kMaxSeg, "gemm: nseg must be in [1, %d]",
               gemm::kMaxSeg);
  ML_CHECK_ARG(segs != nullptr, "gemm: null segment list");
  ML_CHECK_ARG(d_dtype == ML_DTYPE_F32 || d_dtype == ML_DTYPE_BF16,
               "gemm: output dtype must be f32 or bf16");
  ML_CHECK_ARG(beta == 0.f || beta == 1.f, "gemm: beta must be 0 or 1");
  ML_CHECK_ARG(ldd >= n, "gemm: ldd < n");
  if (m == 0 || n == 0) return ML_OK;
  ML_CHECK_ARG(d != nullptr, "gemm: null output");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  gemm::Problem pr;
  pr.M = m;
  pr.N = n;
  pr.nseg = nseg;
  pr.a_mn = segs[0].a.mn_major != 0;
  pr.b_mn = segs[0].b.mn_major != 0;
  int64_t k_total = 0;
  for (int s = 0; s < nseg; ++s) {
    ML_CHECK_ARG((segs[s].a.mn_major != 0) == pr.a_mn && (segs[s].b.mn_major != 0) == pr.b_mn,
                 "gemm: all segments must share operand majorness");
    ML_CHECK_ARG(segs[s].k >= 0, "gemm: negative k");
    pr.seg[s].a.ptr = segs[s].a.ptr;
    pr.seg[s].a.ld = segs[s].a.ld;
    pr.seg[s].b.ptr = segs[s].b.ptr;
    pr.seg[s].b.ld = segs[s].b.ld;
    pr.seg[s].K = segs[s].k;
    k_total += segs[s].k;
  }
  if (k_total == 0 || std::all_of(segs, segs + nseg, [](const ml_gemm_segment& g) {
        return g.k == 0;
      })) {
    set_error("gemm: K == 0 is not supported (scale or clear D instead)");
    return ML_ERR_INVALID_ARG;
  }
  // drop empty segments
  int w = 0;
  for (int s = 0; s < nseg; ++s)
    if (pr.seg[s].K > 0) pr.seg[w++] = pr.seg[s];
  pr.nseg = w;
  pr.d_f32 = d_dtype == ML_DTYPE_F32;
  pr.D = d;
  pr.ldd = ldd;
  pr.alpha = alpha;
  pr.beta = beta;
  const int bn = gemm::pick_bn(n);
  int splits = choose_splits(m, n, k_total, bn);
  if (splits > 1 &&
      (workspace == nullptr || !aligned16(workspace) ||
       workspace_bytes < (size_t)splits * (size_t)m * (size_t)n * sizeof(float)))
    splits = 1;
  if (splits == 1) {
    pr.epi = gemm::EPI_STORE;
    if (!pr.d_f32 && beta != 0.f) {
      set_error("gemm: beta=1 needs an fp32 output");
      return ML_ERR_INVALID_ARG;
    }
    return gemm::launch(pr, st);
  }
  pr.epi = gemm::EPI_PARTIAL;
  pr.splits = splits;
  pr.D = workspace;
  pr.ldd = n;
  pr.d_f32 = true;
  pr.beta = 0.f;
  int rc = gemm::launch(pr, st);
  if (rc) return rc;
  const int64_t total = m * n;
  int grid = (int)std::min<int64_t>((total + 255) / 256, (int64_t)num_sms() * 8);
  splitk_reduce<<<std::max(grid, 1), 256, 0, st>>>(static_cast<const float*>(workspace), splits, m,
                                                    n, n, d, ldd, d_dtype == ML_DTYPE_F32,
                                                    beta);
  ML_CHECK_LAUNCH("gemm split-K reduce");
  return ML_OK;
}
