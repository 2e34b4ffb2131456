// Peer memory between the GPUs of one node (one process per GPU) and the
// vocabulary-parallel FLCE's dX exchange over it.
//
// The vocabulary-parallel FLCE leaves every rank with a partial dX for the
// chunk's token rows (its vocabulary shard's P_shard W_shard); the full dX is
// their sum.  Instead of a separate all-reduce after the dX GEMM, each rank
// owns a block of rows, and the dX GEMM's epilogue stores every output tile
// straight into the owner's receive slot for this rank (peer-mode store
// epilogue, gemm.cuh): the reduce-scatter traffic crosses NVLink tile by tile
// while the GEMM runs.  The owner then sums its slots in rank order and
// writes the reduced rows into every rank's gather buffer (the all-gather,
// plain stores again); flags in each rank's exchange buffer, written with
// release stores and read with acquire loads at system scope, order the
// phases.  Every wait is bounded (%globaltimer): a wait that gives up records
// ML_ERR_TIMEOUT in the device error word (ml_device_error) and the kernel
// returns; nothing traps or hangs.
//
// The per-row softmax statistics are merged the same way: every rank stores
// its (max, sum-exp, target) rows into every rank's stats slots, and each
// rank merges all of them in rank order (the same result on every rank).
//
// Exchange buffer of each rank (ml_flce_p2p_workspace_bytes):
//   [0, 256)           int64 arrive[kMaxPeers], done[kMaxPeers], stats[kMaxPeers]
//                      (epochs)
//   recv               fp32 [world][rows_per_owner][h]  (slot per source rank)
//   gather             fp32 [chunk_cap][h]               (the reduced chunk)
//   stats              fp32 [2][world][3][chunk_cap]     (by epoch parity: a
//                      rank may store chunk c + 1's rows while a slower one
//                      still merges chunk c's)
// rows_per_owner = ceil(chunk_cap / world) rounded up to a multiple of 256,
// so a 256-row GEMM tile never straddles two owners.
#include "p2p.cuh"

#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>

namespace ml {
namespace p2p {

XLayout xlayout(int world, int64_t chunk_cap, int64_t h) {
  XLayout L;
  const int64_t per = (chunk_cap + world - 1) / world;
  L.rows_per_owner = (per + 255) / 256 * 256;
  L.off_recv = 256;
  L.off_gather = L.off_recv + (size_t)world * L.rows_per_owner * h * 4;
  L.off_stats = L.off_gather + (size_t)chunk_cap * h * 4;
  L.total = L.off_stats + (size_t)2 * world * 3 * chunk_cap * 4;
  return L;
}

namespace {

constexpr uint64_t kWaitNs = 2000000000ull;  // 2 s per wait
constexpr int kSiteArrive = 7, kSiteDone = 8, kSiteStats = 9;

__device__ __forceinline__ void st_release_sys(int64_t* p, int64_t v) {
  asm volatile("st.release.sys.global.b64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ int64_t ld_acquire_sys(const int64_t* p) {
  int64_t v;
  asm volatile("ld.acquire.sys.global.b64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// Spins until flags[0..n) all reach `epoch` or the bound passes.
__device__ bool wait_flags(const int64_t* flags, int n, int64_t epoch, int* err, int site) {
  const uint64_t t0 = sm100::globaltimer_ns();
  for (int s = 0; s < n; ++s) {
    while (ld_acquire_sys(flags + s) < epoch) {
      if (sm100::globaltimer_ns() - t0 > kWaitNs) {
        if (err != nullptr) atomicCAS(err, 0, (site << 8) | ML_ERR_TIMEOUT);
        return false;
      }
    }
  }
  return true;
}

// flags[slot] of every rank (arrive: slot = this rank) = epoch.
__global__ void signal_k(const __grid_constant__ Peers pe, int world, int me, int which,
                         int64_t epoch) {
  const int t = threadIdx.x;
  __threadfence_system();
  if (t < world) {
    int64_t* flags = reinterpret_cast<int64_t*>(pe.ws[t]) + which * kMax;
    st_release_sys(flags + me, epoch);
  }
}

// The owner's phase: wait for every source's arrive flag, sum the slots of
// this rank's rows in rank order, write the sums into every rank's gather
// buffer.
__global__ void __launch_bounds__(256) reduce_gather_k(const __grid_constant__ Peers pe, int world,
                                                       int me, int64_t rows, int64_t h,
                                                       int64_t rows_per_owner, size_t off_recv,
                                                       size_t off_gather, int64_t epoch,
                                                       int* err) {
  __shared__ int ok;
  if (threadIdx.x == 0) {
    const int64_t* arrive = reinterpret_cast<const int64_t*>(pe.ws[me]);
    ok = wait_flags(arrive, world, epoch, err, kSiteArrive) ? 1 : 0;
  }
  __syncthreads();
  if (!ok) return;
  const int64_t r0 = (int64_t)me * rows_per_owner;
  const int64_t r1 = rows < r0 + rows_per_owner ? rows : r0 + rows_per_owner;
  const int64_t nr = r1 > r0 ? r1 - r0 : 0;
  const int64_t n4 = nr * h / 4;
  const size_t slot4 = (size_t)rows_per_owner * h / 4;
  const float4* recv = reinterpret_cast<const float4*>(pe.ws[me] + off_recv);
  // kU independent vectors per thread per step: enough loads in flight for
  // a grid that shares the SMs with the concurrent dW GEMM
  constexpr int kU = 4;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t base = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; base < n4;
       base += stride * kU) {
    float4 acc[kU];
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      const int64_t i = base + u * stride;
      if (i < n4) acc[u] = __ldcg(recv + i);
    }
    for (int s = 1; s < world; ++s) {
#pragma unroll
      for (int u = 0; u < kU; ++u) {
        const int64_t i = base + u * stride;
        if (i < n4) {
          const float4 v = __ldcg(recv + (size_t)s * slot4 + i);
          acc[u].x += v.x;
          acc[u].y += v.y;
          acc[u].z += v.z;
          acc[u].w += v.w;
        }
      }
    }
    for (int p = 0; p < world; ++p) {
      float4* dst = reinterpret_cast<float4*>(pe.ws[p] + off_gather) + (size_t)r0 * h / 4;
#pragma unroll
      for (int u = 0; u < kU; ++u) {
        const int64_t i = base + u * stride;
        if (i < n4) dst[i] = acc[u];
      }
    }
  }
  __threadfence_system();
}

// Waits for every owner's done flag (this rank's gather buffer is complete).
__global__ void wait_done_k(const int64_t* done, int world, int64_t epoch, int* err) {
  if (threadIdx.x == 0) wait_flags(done, world, epoch, err, kSiteDone);
}

// This rank's (max, sum-exp, target) rows into slot `me` of every rank.
__global__ void __launch_bounds__(256) stats_put_k(const __grid_constant__ Peers pe, int world,
                                                   int me, const float* __restrict__ m,
                                                   const float* __restrict__ s,
                                                   const float* __restrict__ t, int64_t rows,
                                                   int64_t chunk_cap, size_t off_set) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < rows;
       i += (int64_t)gridDim.x * blockDim.x) {
    const float v[3] = {m[i], s[i], t[i]};
    for (int p = 0; p < world; ++p) {
      float* slot = reinterpret_cast<float*>(pe.ws[p] + off_set) + (size_t)me * 3 * chunk_cap;
#pragma unroll
      for (int k = 0; k < 3; ++k) slot[(size_t)k * chunk_cap + i] = v[k];
    }
  }
  __threadfence_system();
}

// Waits for every rank's stats rows, merges them in rank order:
// max = max_r m_r, sum = sum_r s_r exp(m_r - max), target = sum_r t_r.
__global__ void __launch_bounds__(256) stats_merge_k(const uint8_t* __restrict__ own, int world,
                                                     int64_t rows, int64_t chunk_cap,
                                                     size_t off_set, int64_t epoch,
                                                     float* __restrict__ out_m,
                                                     float* __restrict__ out_s,
                                                     float* __restrict__ out_t, int* err) {
  __shared__ int ok;
  if (threadIdx.x == 0) {
    const int64_t* flags = reinterpret_cast<const int64_t*>(own) + 2 * kMax;
    ok = wait_flags(flags, world, epoch, err, kSiteStats) ? 1 : 0;
  }
  __syncthreads();
  if (!ok) return;
  const float* slots = reinterpret_cast<const float*>(own + off_set);
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < rows;
       i += (int64_t)gridDim.x * blockDim.x) {
    float mg = -INFINITY;
    for (int r = 0; r < world; ++r) mg = fmaxf(mg, __ldcg(slots + (size_t)r * 3 * chunk_cap + i));
    float sg = 0.f, tg = 0.f;
    for (int r = 0; r < world; ++r) {
      const float* sl = slots + (size_t)r * 3 * chunk_cap;
      const float mr = __ldcg(sl + i);
      const float sr = __ldcg(sl + chunk_cap + i);
      sg += sr == 0.f ? 0.f : sr * expf(mr - mg);
      tg += __ldcg(sl + 2 * chunk_cap + i);
    }
    out_m[i] = mg;
    out_s[i] = sg;
    out_t[i] = tg;
  }
}

}  // namespace

int launch_signal(const Peers& pe, int world, int me, int which, int64_t epoch, cudaStream_t st) {
  signal_k<<<1, 32, 0, st>>>(pe, world, me, which, epoch);
  ML_CHECK_LAUNCH("flce_p2p(signal)");
  return ML_OK;
}

int check_peers(int world, int rank, void* const* peer_ws, Peers& pe) {
  ML_CHECK_ARG(world >= 1 && world <= kMax && rank >= 0 && rank < world,
               "flce_p2p: rank %d of world %d (at most %d ranks)", rank, world, kMax);
  ML_CHECK_ARG(peer_ws != nullptr, "flce_p2p: null peer table");
  for (int r = 0; r < kMax; ++r) pe.ws[r] = nullptr;
  for (int r = 0; r < world; ++r) {
    ML_CHECK_ARG(peer_ws[r] != nullptr && ((uintptr_t)peer_ws[r] & 255) == 0,
                 "flce_p2p: exchange buffer of rank %d is null or not 256-byte aligned", r);
    pe.ws[r] = static_cast<uint8_t*>(peer_ws[r]);
  }
  return ML_OK;
}

}  // namespace p2p
}  // namespace ml

using namespace ml;

extern "C" int ml_p2p_alloc(size_t bytes, void** out) {
  ML_CHECK_ARG(out != nullptr && bytes > 0, "p2p_alloc: bad arguments");
  *out = nullptr;
  void* p = nullptr;
  ML_CHECK_CUDA(cudaMalloc(&p, bytes), "p2p_alloc: cudaMalloc");
  const cudaError_t e = cudaMemset(p, 0, bytes);
  if (e != cudaSuccess) {
    cudaFree(p);
    set_error("p2p_alloc: cudaMemset: %s", cudaGetErrorString(e));
    return ML_ERR_CUDA;
  }
  *out = p;
  return ML_OK;
}

extern "C" int ml_p2p_free(void* p) {
  if (p != nullptr) ML_CHECK_CUDA(cudaFree(p), "p2p_free");
  return ML_OK;
}

extern "C" size_t ml_p2p_handle_bytes(void) { return sizeof(cudaIpcMemHandle_t); }

extern "C" int ml_p2p_export(const void* base, void* handle_out) {
  ML_CHECK_ARG(base != nullptr && handle_out != nullptr, "p2p_export: null pointer");
  cudaIpcMemHandle_t hd;
  ML_CHECK_CUDA(cudaIpcGetMemHandle(&hd, const_cast<void*>(base)), "p2p_export");
  std::memcpy(handle_out, &hd, sizeof(hd));
  return ML_OK;
}

extern "C" int ml_p2p_import(const void* handle, void** out) {
  ML_CHECK_ARG(handle != nullptr && out != nullptr, "p2p_import: null pointer");
  cudaIpcMemHandle_t hd;
  std::memcpy(&hd, handle, sizeof(hd));
  *out = nullptr;
  ML_CHECK_CUDA(cudaIpcOpenMemHandle(out, hd, cudaIpcMemLazyEnablePeerAccess), "p2p_import");
  return ML_OK;
}

extern "C" int ml_p2p_close(void* p) {
  if (p != nullptr) ML_CHECK_CUDA(cudaIpcCloseMemHandle(p), "p2p_close");
  return ML_OK;
}

extern "C" size_t ml_flce_p2p_workspace_bytes(int world, int64_t chunk_cap, int64_t h) {
  if (world < 1 || world > p2p::kMax || chunk_cap <= 0 || h <= 0) return 0;
  return p2p::xlayout(world, chunk_cap, h).total;
}

// The owner's phase: waits for every rank's tiles of this chunk (arrive
// flags), sums this rank's rows in rank order into every rank's gather
// buffer and raises this rank's done flag on every rank.
extern "C" int ml_flce_p2p_reduce(int64_t rows, int64_t h, int64_t chunk_cap, int world, int rank,
                                  void* const* peer_ws, int64_t epoch, void* stream) {
  ML_CHECK_ARG(rows > 0 && rows <= chunk_cap && h > 0 && h % 8 == 0 && epoch > 0,
               "flce_p2p_reduce: bad sizes");
  p2p::Peers pe;
  if (int rc = p2p::check_peers(world, rank, peer_ws, pe)) return rc;
  const p2p::XLayout X = p2p::xlayout(world, chunk_cap, h);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // this rank's rows: a grid of up to two CTAs per SM (the owner phase runs
  // beside the dW GEMM, whose one CTA per SM leaves room for them)
  const int64_t r0 = (int64_t)rank * X.rows_per_owner;
  const int64_t nr = std::max<int64_t>(0, std::min<int64_t>(rows, r0 + X.rows_per_owner) - r0);
  const int grid = (int)std::max<int64_t>(
      1, std::min<int64_t>((nr * h / 4 + 1023) / 1024, (int64_t)2 * num_sms()));
  p2p::reduce_gather_k<<<grid, 256, 0, st>>>(pe, world, rank, rows, h, X.rows_per_owner,
                                           X.off_recv, X.off_gather, epoch,
                                           gemm::device_error_word());
  ML_CHECK_LAUNCH("flce_p2p_reduce");
  return p2p::launch_signal(pe, world, rank, 1, epoch, st);
}

// Waits for every owner's done flag, then copies the chunk's reduced dX
// (rows x h fp32, from this rank's gather buffer) to dx_out.
extern "C" int ml_flce_p2p_finish(int64_t rows, int64_t h, int64_t chunk_cap, int world, int rank,
                                  void* const* peer_ws, int64_t epoch, float* dx_out,
                                  void* stream) {
  ML_CHECK_ARG(dx_out != nullptr, "flce_p2p_finish: null output");
  ML_CHECK_ARG(rows > 0 && rows <= chunk_cap && h > 0 && h % 8 == 0 && epoch > 0,
               "flce_p2p_finish: bad sizes");
  p2p::Peers pe;
  if (int rc = p2p::check_peers(world, rank, peer_ws, pe)) return rc;
  const p2p::XLayout X = p2p::xlayout(world, chunk_cap, h);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int64_t* done = reinterpret_cast<const int64_t*>(pe.ws[rank]) + p2p::kMax;
  p2p::wait_done_k<<<1, 32, 0, st>>>(done, world, epoch, gemm::device_error_word());
  ML_CHECK_LAUNCH("flce_p2p_finish(wait)");
  ML_CHECK_CUDA(cudaMemcpyAsync(dx_out, pe.ws[rank] + X.off_gather, (size_t)rows * h * 4,
                                cudaMemcpyDeviceToDevice, st),
                "flce_p2p_finish(copy)");
  return ML_OK;
}

// The statistics exchange of one chunk, in two calls (a rank's merge waits
// for every rank's put): this rank's [rows] max / sum-exp / target into its
// slot on every rank, then this rank's stats flag on every rank ...
extern "C" int ml_flce_p2p_stats_put(const float* row_max, const float* row_sum,
                                     const float* row_tgt, int64_t rows, int64_t h,
                                     int64_t chunk_cap, int world, int rank, void* const* peer_ws,
                                     int64_t epoch, void* stream) {
  ML_CHECK_ARG(row_max && row_sum && row_tgt, "flce_p2p_stats_put: null pointer");
  ML_CHECK_ARG(rows > 0 && rows <= chunk_cap && h > 0 && epoch > 0,
               "flce_p2p_stats_put: bad sizes");
  p2p::Peers pe;
  if (int rc = p2p::check_peers(world, rank, peer_ws, pe)) return rc;
  const p2p::XLayout X = p2p::xlayout(world, chunk_cap, h);
  const size_t off_set = X.off_stats + (size_t)(epoch & 1) * world * 3 * chunk_cap * 4;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int grid = (int)std::min<int64_t>((rows + 255) / 256, 64);
  p2p::stats_put_k<<<grid, 256, 0, st>>>(pe, world, rank, row_max, row_sum, row_tgt, rows,
                                          chunk_cap, off_set);
  ML_CHECK_LAUNCH("flce_p2p_stats_put");
  return p2p::launch_signal(pe, world, rank, 2, epoch, st);
}

// ... and the merge: waits for every rank's stats flag and writes the merged
// [rows] max, sum-exp (relative to that max) and target logit.
extern "C" int ml_flce_p2p_stats_merge(int64_t rows, int64_t h, int64_t chunk_cap, int world,
                                       int rank, void* const* peer_ws, int64_t epoch,
                                       float* out_max, float* out_sum, float* out_tgt,
                                       void* stream) {
  ML_CHECK_ARG(out_max && out_sum && out_tgt, "flce_p2p_stats_merge: null output");
  ML_CHECK_ARG(rows > 0 && rows <= chunk_cap && h > 0 && epoch > 0,
               "flce_p2p_stats_merge: bad sizes");
  p2p::Peers pe;
  if (int rc = p2p::check_peers(world, rank, peer_ws, pe)) return rc;
  const p2p::XLayout X = p2p::xlayout(world, chunk_cap, h);
  const size_t off_set = X.off_stats + (size_t)(epoch & 1) * world * 3 * chunk_cap * 4;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int grid = (int)std::min<int64_t>((rows + 255) / 256, 64);
  p2p::stats_merge_k<<<grid, 256, 0, st>>>(pe.ws[rank], world, rows, chunk_cap, off_set, epoch,
                                            out_max, out_sum, out_tgt, gemm::device_error_word());
  ML_CHECK_LAUNCH("flce_p2p_stats_merge");
  return ML_OK;
}
