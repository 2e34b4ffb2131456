// RMSNorm forward/backward for sm_100a.
//
// Follows the math of the reference's _FusedRMSNormFunction
// (ops/fused_rms_norm.py:30-60) and the Metal kernels it was meant to drive
// (kernels/rms_norm.metal:22-200): fp32 accumulation, rrms saved per row,
// analytic VJP with no recompute of x_norm.
//
// Launch shape (B200-first): the row is held in registers, read once with
// 16-byte vector loads.  A CTA holds G row-groups of TPR threads; each group
// owns one row per iteration and reduces it with warp shuffles plus one
// shared-memory exchange.  The grid is persistent (a multiple of the SM
// count), so the backward's dweight partials are one fp32 row per CTA,
// reduced deterministically by a second small kernel — never a [rows, hidden]
// per-row buffer like the reference's Metal host code (csrc/rms_norm_metal.mm:182,211).
#include "common.cuh"

#include <algorithm>
#include <atomic>
#include <mutex>

namespace ml {
namespace {

constexpr int kMaxThreads = kRmsMaxThreads;

// Backward CTA size: when a thread's share of two rows (current + prefetch)
// fits in ~80 registers the CTA holds three 256-thread row groups and runs one
// per SM, so the dweight partials (one row per CTA) number about the SM count.
// Larger shares keep 256-thread CTAs (three groups would not fit an SM).
template <typename TX>
__host__ __device__ constexpr int bwd_max_threads(int nv) {
  return nv == 1 ? 512 : (nv == 2 && sizeof(TX) == 4) ? 768 : kMaxThreads;
}
// One vector per thread: 512-thread CTAs, two per SM (<= 64 registers), so
// twice the rows are in flight of a single CTA per SM.
__host__ __device__ constexpr int bwd_min_blocks(int nv) { return nv == 1 ? 2 : 1; }

// Forward CTA size: one vector per thread allows 512-thread rows (16-bit
// rows of up to 4096 elements); two vectors per thread run two or three row
// groups in a 512-thread CTA (fp32 [8192, 2048]: 22.6 us against 24.6 us with
// one 256-thread row per CTA, same results bit for bit); wider shares keep
// 256 threads.
__host__ __device__ constexpr int fwd_max_threads(int nv) { return nv <= 2 ? 512 : kMaxThreads; }

struct RowCfg {
  int nv = 0;       // 16-byte vectors per thread per row
  int tpr = 0;      // threads per row (4, 8, 16, or a multiple of 32)
  int groups = 0;   // rows in flight per CTA
  bool vec = false; // false -> generic scalar kernels
};

// Rows of up to 32 vectors get sub-warp groups (4/8/16 lanes, reduced with
// shuffles alone: the per-head q/k norm has 16 vectors per bf16 row), so no
// lane idles.  16-bit rows of 257-512 vectors (hidden 4096 bf16) take one
// vector per thread on 512 threads instead of two on 256: two 8-element
// vectors per thread and row cost ~160 registers (one CTA of 8 warps per
// SM), one costs ~80.
template <typename TX>
RowCfg pick_cfg(int64_t hidden, const void* a, const void* b, const void* c, const void* d,
                bool backward) {
  RowCfg cfg;
  constexpr int VEC = 16 / sizeof(TX);
  if (hidden % VEC != 0 || !aligned16(a) || !aligned16(b) || !aligned16(c) || !aligned16(d))
    return cfg;
  const int64_t nvec = hidden / VEC;
  int nv, tpr;
  if (!rms_row_split(nvec, rms_one_vec_limit((int)sizeof(TX), backward), &nv, &tpr)) return cfg;
  cfg.nv = nv;
  cfg.tpr = tpr;
  const int max_groups = tpr < 32 ? 32 : 8;  // named barriers are only needed for tpr >= 32
  const int cta_threads = (!backward && nv == 2) ? fwd_max_threads(nv) : kMaxThreads;
  cfg.groups = std::max(1, std::min<int>(max_groups, cta_threads / cfg.tpr));
  cfg.vec = true;
  return cfg;
}

// Reduce `v` (and optionally `v2`) over the TPR threads of this thread's row
// group.  `red` is a [2][32][2] shared array double-buffered by `buf` so one
// barrier per row suffices.  Each row group synchronises on its own named
// barrier (id 1 + group), so groups never wait for one another.
__device__ __forceinline__ void group_barrier(int tpr) {
  if (tpr == (int)blockDim.x) {
    __syncthreads();
  } else {
    const int id = 1 + (int)threadIdx.x / tpr;
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(tpr) : "memory");
  }
}

__device__ __forceinline__ float2 group_sum2(float v, float v2, float (*red)[32][2], int buf,
                                            int tpr) {
  if (tpr < 32) {  // sub-warp group aligned within its warp: shuffles alone
    for (int o = tpr >> 1; o > 0; o >>= 1) {
      v += __shfl_xor_sync(0xffffffffu, v, o);
      v2 += __shfl_xor_sync(0xffffffffu, v2, o);
    }
    return make_float2(v, v2);
  }
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  v = warp_sum(v);
  v2 = warp_sum(v2);
  if (lane == 0) {
    red[buf][warp][0] = v;
    red[buf][warp][1] = v2;
  }
  group_barrier(tpr);
  const int wpg = tpr >> 5;                 // warps per group
  const int first = (warp / wpg) * wpg;     // first warp of my group
  float s = 0.f, s2 = 0.f;
  for (int i = 0; i < wpg; ++i) {           // fixed order: deterministic
    s += red[buf][first + i][0];
    s2 += red[buf][first + i][1];
  }
  return make_float2(s, s2);
}

template <typename TW, int VEC>
__device__ __forceinline__ void load_weight(const TW* w, int64_t col, int64_t hidden, float* out) {
#pragma unroll
  for (int j = 0; j < VEC; ++j) out[j] = (col + j < hidden) ? to_f32(w[col + j]) : 0.f;
}

// ------------------------------- forward ----------------------------------
template <typename TX, typename TW, int NV>
__global__ void __launch_bounds__(fwd_max_threads(NV))
rms_fwd_vec(const TX* __restrict__ x, const TW* __restrict__ w, TX* __restrict__ y,
            float* __restrict__ rrms, int64_t rows, int64_t hidden, float eps, int tpr,
            int groups) {
  constexpr int VEC = 16 / sizeof(TX);
  __shared__ float red[2][32][2];
  const int g = threadIdx.x / tpr;
  const int t = threadIdx.x % tpr;
  // launched as a programmatic dependent: x and w may come from the previous kernel
  pdl_wait();
  pdl_release();
  float wr[NV][VEC];
#pragma unroll
  for (int i = 0; i < NV; ++i) load_weight<TW, VEC>(w, (int64_t)(i * tpr + t) * VEC, hidden, wr[i]);

  const int64_t row_stride = (int64_t)gridDim.x * groups;
  const int64_t niter = (rows + row_stride - 1) / row_stride;
  const float inv_h = 1.f / (float)hidden;
  int64_t row = (int64_t)blockIdx.x * groups + g;
  // Software pipeline: the next row's loads are in flight while this row is
  // reduced and written.
  Vec16<TX> xv[NV], xn[NV];
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int64_t col = (int64_t)(i * tpr + t) * VEC;
    if (row < rows && col < hidden) xv[i] = ld_vec_stream(x + row * hidden + col);
  }
  int buf = 0;
  for (int64_t it = 0; it < niter; ++it, row += row_stride) {
    const bool active = row < rows;
    const int64_t nrow = row + row_stride;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int64_t col = (int64_t)(i * tpr + t) * VEC;
      if (nrow < rows && col < hidden) xn[i] = ld_vec_stream(x + nrow * hidden + col);
    }
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int64_t col = (int64_t)(i * tpr + t) * VEC;
      if (active && col < hidden) {
#pragma unroll
        for (int j = 0; j < VEC; ++j) {
          const float f = to_f32(xv[i].v[j]);
          ss = fmaf(f, f, ss);
        }
      }
    }
    const float tot = group_sum2(ss, 0.f, red, buf, tpr).x;
    buf ^= 1;
    if (active) {
      const float r = rsqrtf(fmaf(tot, inv_h, eps));
      if (t == 0 && rrms != nullptr) rrms[row] = r;
#pragma unroll
      for (int i = 0; i < NV; ++i) {
        const int64_t col = (int64_t)(i * tpr + t) * VEC;
        if (col < hidden) {
          Vec16<TX> o;
#pragma unroll
          for (int j = 0; j < VEC; ++j)
            o.v[j] = from_f32<TX>((to_f32(xv[i].v[j]) * r) * wr[i][j]);
          st_vec_stream(y + row * hidden + col, o);
        }
      }
    }
#pragma unroll
    for (int i = 0; i < NV; ++i) xv[i] = xn[i];
  }
}

// ---------------------- ring-prefetch variants (NV = 1) ----------------------
// With one 16-byte vector per thread and row, the register double buffer of
// the kernels above keeps only ~16 B per thread in flight and each row
// iteration waits out a full memory latency.  These variants stream the rows
// through a per-group ring of S slots in shared memory with cp.async (every
// thread copies, and later reads, only its own vectors, so no barrier guards
// the ring); S - 1 rows are in flight while one is reduced.
__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32_of(dst)), "l"(src)
               : "memory");
}
__device__ __forceinline__ void cp_async4(void* dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32_of(dst)), "l"(src)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

constexpr int kRingStages = 6;

template <typename TX, typename TW, int S>
__global__ void __launch_bounds__(512)
rms_fwd_ring(const TX* __restrict__ x, const TW* __restrict__ w, TX* __restrict__ y,
             float* __restrict__ rrms, int64_t rows, int64_t hidden, float eps, int tpr,
             int groups) {
  constexpr int VEC = 16 / sizeof(TX);
  __shared__ float red[2][32][2];
  extern __shared__ __align__(16) uint8_t ring_raw[];
  const int g = threadIdx.x / tpr;
  const int t = threadIdx.x % tpr;
  Vec16<TX>* ring = reinterpret_cast<Vec16<TX>*>(ring_raw) + (size_t)g * S * tpr;
  const int64_t col = (int64_t)t * VEC;
  const bool has_col = col < hidden;
  pdl_wait();
  pdl_release();
  float wr[VEC];
  load_weight<TW, VEC>(w, col, hidden, wr);
  const int64_t row_stride = (int64_t)gridDim.x * groups;
  const int64_t niter = (rows + row_stride - 1) / row_stride;
  const float inv_h = 1.f / (float)hidden;
  const int64_t row0 = (int64_t)blockIdx.x * groups + g;
  auto issue = [&](int64_t r, int slot) {
    if (r < rows && has_col) cp_async16(&ring[slot * tpr + t], x + r * hidden + col);
    cp_async_commit();
  };
#pragma unroll
  for (int j = 0; j < S - 1; ++j) issue(row0 + j * row_stride, j);
  int buf = 0;
  for (int64_t it = 0; it < niter; ++it) {
    const int64_t row = row0 + it * row_stride;
    issue(row + (S - 1) * row_stride, (int)((it + S - 1) % S));
    cp_async_wait<S - 1>();
    const bool active = row < rows && has_col;
    Vec16<TX> xv;
    float ss = 0.f;
    if (active) {
      xv = ring[(int)(it % S) * tpr + t];
#pragma unroll
      for (int j = 0; j < VEC; ++j) {
        const float f = to_f32(xv.v[j]);
        ss = fmaf(f, f, ss);
      }
    }
    const float tot = group_sum2(ss, 0.f, red, buf, tpr).x;
    buf ^= 1;
    if (row < rows) {
      const float r = rsqrtf(fmaf(tot, inv_h, eps));
      if (t == 0 && rrms != nullptr) rrms[row] = r;
      if (has_col) {
        Vec16<TX> o;
#pragma unroll
        for (int j = 0; j < VEC; ++j) o.v[j] = from_f32<TX>((to_f32(xv.v[j]) * r) * wr[j]);
        st_vec_stream(y + row * hidden + col, o);
      }
    }
  }
  cp_async_wait<0>();
}

// Generic path: any hidden size / alignment.  One CTA per row (grid-stride),
// two passes over the row (the second hits L1/L2).
template <typename TX, typename TW>
__global__ void __launch_bounds__(256)
rms_fwd_generic(const TX* __restrict__ x, const TW* __restrict__ w, TX* __restrict__ y,
                float* __restrict__ rrms, int64_t rows, int64_t hidden, float eps) {
  __shared__ float red[2][32][2];
  pdl_wait();
  pdl_release();
  int buf = 0;
  for (int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
    const TX* xr = x + row * hidden;
    float ss = 0.f;
    for (int64_t c = threadIdx.x; c < hidden; c += blockDim.x) {
      const float f = to_f32(xr[c]);
      ss = fmaf(f, f, ss);
    }
    const float tot = group_sum2(ss, 0.f, red, buf, blockDim.x).x;
    buf ^= 1;
    const float r = rsqrtf(tot / (float)hidden + eps);
    if (threadIdx.x == 0 && rrms != nullptr) rrms[row] = r;
    for (int64_t c = threadIdx.x; c < hidden; c += blockDim.x)
      y[row * hidden + c] = from_f32<TX>((to_f32(xr[c]) * r) * to_f32(w[c]));
  }
}

// ------------------------------- backward ---------------------------------
// Writes dx and one fp32 dweight partial row per CTA into `partial`
// ([gridDim.x, hidden]).  Row groups of a CTA fold their partials together
// through shared memory (fixed order) before the single store.
template <typename TX, typename TW, int NV>
__global__ void __launch_bounds__(bwd_max_threads<TX>(NV), bwd_min_blocks(NV))
rms_bwd_vec(const TX* __restrict__ x, const TW* __restrict__ w, const float* __restrict__ rrms,
            const TX* __restrict__ dy, TX* __restrict__ dx, float* __restrict__ partial,
            int64_t rows, int64_t hidden, float eps, int tpr, int groups) {
  constexpr int VEC = 16 / sizeof(TX);
  __shared__ float red[2][32][2];
  extern __shared__ float fold[];  // [groups][hidden] when groups > 1
  const int g = threadIdx.x / tpr;
  const int t = threadIdx.x % tpr;
  // launched as a programmatic dependent: every input, and the partials the
  // previous call's reduction reads, belong to earlier kernels until this wait
  pdl_wait();
  float wr[NV][VEC];
  float acc[NV][VEC];
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    load_weight<TW, VEC>(w, (int64_t)(i * tpr + t) * VEC, hidden, wr[i]);
#pragma unroll
    for (int j = 0; j < VEC; ++j) acc[i][j] = 0.f;
  }
  const int64_t row_stride = (int64_t)gridDim.x * groups;
  const int64_t niter = (rows + row_stride - 1) / row_stride;
  const float inv_h = 1.f / (float)hidden;
  int64_t row = (int64_t)blockIdx.x * groups + g;
  Vec16<TX> xv[NV], gv[NV], xn[NV], gn[NV];
  // The saved rrms of the next row is fetched with that row's data, so no
  // load sits on the critical path between the reduction and the stores.
  float rv = (rrms != nullptr && row < rows) ? __ldg(rrms + row) : 0.f;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int64_t col = (int64_t)(i * tpr + t) * VEC;
    if (row < rows && col < hidden) {
      xv[i] = ld_vec_stream(x + row * hidden + col);
      gv[i] = ld_vec_stream(dy + row * hidden + col);
    }
  }
  int buf = 0;
  for (int64_t it = 0; it < niter; ++it, row += row_stride) {
    const bool active = row < rows;
    const int64_t nrow = row + row_stride;
    const float rn = (rrms != nullptr && nrow < rows) ? __ldg(rrms + nrow) : 0.f;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int64_t col = (int64_t)(i * tpr + t) * VEC;
      if (nrow < rows && col < hidden) {
        xn[i] = ld_vec_stream(x + nrow * hidden + col);
        gn[i] = ld_vec_stream(dy + nrow * hidden + col);
      }
    }
    float ss = 0.f, gwx = 0.f;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int64_t col = (int64_t)(i * tpr + t) * VEC;
      if (active && col < hidden) {
#pragma unroll
        for (int j = 0; j < VEC; ++j) {
          const float xf = to_f32(xv[i].v[j]);
          ss = fmaf(xf, xf, ss);
          gwx = fmaf(to_f32(gv[i].v[j]) * wr[i][j], xf, gwx);
        }
      }
    }
    const float2 sums = group_sum2(ss, gwx, red, buf, tpr);
    buf ^= 1;
    if (active) {
      const float r = rrms != nullptr ? rv : rsqrtf(fmaf(sums.x, inv_h, eps));
      const float c = (sums.y * inv_h) * (r * r * r);
#pragma unroll
      for (int i = 0; i < NV; ++i) {
        const int64_t col = (int64_t)(i * tpr + t) * VEC;
        if (col < hidden) {
          Vec16<TX> o;
#pragma unroll
          for (int j = 0; j < VEC; ++j) {
            const float xf = to_f32(xv[i].v[j]);
            const float gf = to_f32(gv[i].v[j]);
            o.v[j] = from_f32<TX>((gf * wr[i][j]) * r - xf * c);
            acc[i][j] = fmaf(gf, xf * r, acc[i][j]);
          }
          st_vec_stream(dx + row * hidden + col, o);
        }
      }
    }
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      xv[i] = xn[i];
      gv[i] = gn[i];
    }
    rv = rn;
  }
  // The dweight reduction kernel may start launching now; it waits for this
  // grid to finish (griddepcontrol.wait) before reading the partials.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  // Fold the row groups' partials (fixed order) and store one row per CTA.
  if (groups > 1) {
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int64_t col = (int64_t)(i * tpr + t) * VEC;
#pragma unroll
      for (int j = 0; j < VEC; ++j)
        if (col + j < hidden) fold[(int64_t)g * hidden + col + j] = acc[i][j];
    }
    __syncthreads();
    for (int64_t c = threadIdx.x; c < hidden; c += blockDim.x) {
      float s = 0.f;
      for (int k = 0; k < groups; ++k) s += fold[(int64_t)k * hidden + c];
      partial[(int64_t)blockIdx.x * hidden + c] = s;
    }
  } else {
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int64_t col = (int64_t)(i * tpr + t) * VEC;
#pragma unroll
      for (int j = 0; j < VEC; ++j)
        if (col + j < hidden) partial[(int64_t)blockIdx.x * hidden + col + j] = acc[i][j];
    }
  }
}

// Backward, ring-prefetch variant: x, dY and the saved rrms of the next
// S - 1 rows stream into shared memory while the current row is reduced; a
// thread owns NV 16-byte vectors of the row (vector i at columns
// (i * tpr + t) * VEC: each vector of the row is contiguous over the
// threads).  Dynamic shared memory: [groups][S][NV][tpr] x vectors, the
// same for dY, [groups][S][tpr] rrms words, and the [groups][hidden]
// dweight fold — after the ring when NV = 1, over the ring's own memory
// (free once the last row is read) when NV > 1.  NV = 2 lets a 16-bit row of
// 4096 run on 256 threads, so three rows are reduced at once per SM where
// one vector per thread (512 threads per row) fits two.
template <typename TX, typename TW, int S, int NV>
__global__ void __launch_bounds__(NV == 1 ? 512 : 768)
rms_bwd_ring(const TX* __restrict__ x, const TW* __restrict__ w, const float* __restrict__ rrms,
             const TX* __restrict__ dy, TX* __restrict__ dx, float* __restrict__ partial,
             int64_t rows, int64_t hidden, float eps, int tpr, int groups) {
  constexpr int VEC = 16 / sizeof(TX);
  constexpr bool kFoldOverRing = NV > 1;
  __shared__ float red[2][32][2];
  extern __shared__ __align__(16) uint8_t ring_raw[];
  const int g = threadIdx.x / tpr;
  const int t = threadIdx.x % tpr;
  const int nthreads = tpr * groups;
  Vec16<TX>* ringx = reinterpret_cast<Vec16<TX>*>(ring_raw) + (size_t)g * S * NV * tpr;
  Vec16<TX>* ringg = reinterpret_cast<Vec16<TX>*>(ring_raw) + (size_t)(groups + g) * S * NV * tpr;
  float* ringr = reinterpret_cast<float*>(reinterpret_cast<Vec16<TX>*>(ring_raw) +
                                          (size_t)2 * groups * S * NV * tpr) +
                 (size_t)g * S * tpr;
  float* fold = kFoldOverRing
                    ? reinterpret_cast<float*>(ring_raw)
                    : reinterpret_cast<float*>(ring_raw + (size_t)2 * groups * S * NV * tpr * 16 +
                                               (size_t)groups * S * tpr * 4);
  pdl_wait();  // programmatic dependent (see rms_bwd_vec)
  int64_t colv[NV];
  bool hasv[NV];
  float wr[NV][VEC], acc[NV][VEC];
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    colv[i] = (int64_t)(i * tpr + t) * VEC;
    hasv[i] = colv[i] < hidden;
    load_weight<TW, VEC>(w, colv[i], hidden, wr[i]);
#pragma unroll
    for (int j = 0; j < VEC; ++j) acc[i][j] = 0.f;
  }
  const int64_t row_stride = (int64_t)gridDim.x * groups;
  const int64_t niter = (rows + row_stride - 1) / row_stride;
  const float inv_h = 1.f / (float)hidden;
  const int64_t row0 = (int64_t)blockIdx.x * groups + g;
  auto issue = [&](int64_t r, int slot) {
    if (r < rows) {
#pragma unroll
      for (int i = 0; i < NV; ++i) {
        if (hasv[i]) {
          cp_async16(&ringx[(slot * NV + i) * tpr + t], x + r * hidden + colv[i]);
          cp_async16(&ringg[(slot * NV + i) * tpr + t], dy + r * hidden + colv[i]);
        }
      }
      if (rrms != nullptr) cp_async4(&ringr[slot * tpr + t], rrms + r);
    }
    cp_async_commit();
  };
#pragma unroll
  for (int j = 0; j < S - 1; ++j) issue(row0 + j * row_stride, j);
  int buf = 0;
  for (int64_t it = 0; it < niter; ++it) {
    const int64_t row = row0 + it * row_stride;
    issue(row + (S - 1) * row_stride, (int)((it + S - 1) % S));
    cp_async_wait<S - 1>();
    const int slot = (int)(it % S);
    const bool active = row < rows;
    Vec16<TX> xv[NV], gv[NV];
    float ss = 0.f, gwx = 0.f;
    if (active) {
#pragma unroll
      for (int i = 0; i < NV; ++i) {
        if (!hasv[i]) continue;
        xv[i] = ringx[(slot * NV + i) * tpr + t];
        gv[i] = ringg[(slot * NV + i) * tpr + t];
#pragma unroll
        for (int j = 0; j < VEC; ++j) {
          const float xf = to_f32(xv[i].v[j]);
          ss = fmaf(xf, xf, ss);
          gwx = fmaf(to_f32(gv[i].v[j]) * wr[i][j], xf, gwx);
        }
      }
    }
    const float2 sums = group_sum2(ss, gwx, red, buf, tpr);
    buf ^= 1;
    if (active) {
      const float r = rrms != nullptr ? ringr[slot * tpr + t] : rsqrtf(fmaf(sums.x, inv_h, eps));
      const float c = (sums.y * inv_h) * (r * r * r);
#pragma unroll
      for (int i = 0; i < NV; ++i) {
        if (!hasv[i]) continue;
        Vec16<TX> o;
#pragma unroll
        for (int j = 0; j < VEC; ++j) {
          const float xf = to_f32(xv[i].v[j]);
          const float gf = to_f32(gv[i].v[j]);
          o.v[j] = from_f32<TX>((gf * wr[i][j]) * r - xf * c);
          acc[i][j] = fmaf(gf, xf * r, acc[i][j]);
        }
        st_vec_stream(dx + row * hidden + colv[i], o);
      }
    }
  }
  cp_async_wait<0>();
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  if (kFoldOverRing) __syncthreads();  // every group is done with the ring
  // Fold the row groups' partials (fixed order) and store one row per CTA.
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    if (!hasv[i]) continue;
#pragma unroll
    for (int j = 0; j < VEC; ++j)
      if (colv[i] + j < hidden) fold[(int64_t)g * hidden + colv[i] + j] = acc[i][j];
  }
  __syncthreads();
  for (int64_t c = threadIdx.x; c < hidden; c += nthreads) {
    float sum = 0.f;
    for (int k = 0; k < groups; ++k) sum += fold[(int64_t)k * hidden + c];
    partial[(int64_t)blockIdx.x * hidden + c] = sum;
  }
}

template <typename TX, typename TW>
__global__ void __launch_bounds__(256)
rms_bwd_generic(const TX* __restrict__ x, const TW* __restrict__ w, const float* __restrict__ rrms,
                const TX* __restrict__ dy, TX* __restrict__ dx, float* __restrict__ partial,
                int64_t rows, int64_t hidden, float eps) {
  __shared__ float red[2][32][2];
  // Per-CTA dweight partial lives directly in `partial` (this CTA's row):
  // each column is owned by exactly one thread, so no races.
  float* prow = partial + (int64_t)blockIdx.x * hidden;
  pdl_wait();  // programmatic dependent (see rms_bwd_vec)
  for (int64_t c = threadIdx.x; c < hidden; c += blockDim.x) prow[c] = 0.f;
  int buf = 0;
  for (int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
    const TX* xr = x + row * hidden;
    const TX* gr = dy + row * hidden;
    float ss = 0.f, gwx = 0.f;
    for (int64_t c = threadIdx.x; c < hidden; c += blockDim.x) {
      const float xf = to_f32(xr[c]);
      ss = fmaf(xf, xf, ss);
      gwx = fmaf(to_f32(gr[c]) * to_f32(w[c]), xf, gwx);
    }
    const float2 sums = group_sum2(ss, gwx, red, buf, blockDim.x);
    buf ^= 1;
    const float r = rrms != nullptr ? rrms[row] : rsqrtf(sums.x / (float)hidden + eps);
    const float cc = (sums.y / (float)hidden) * (r * r * r);
    for (int64_t c = threadIdx.x; c < hidden; c += blockDim.x) {
      const float xf = to_f32(xr[c]);
      const float gf = to_f32(gr[c]);
      dx[row * hidden + c] = from_f32<TX>((gf * to_f32(w[c])) * r - xf * cc);
      prow[c] = fmaf(gf, xf * r, prow[c]);
    }
  }
}

// Second stage: dweight[c] = sum_p partial[p][c], fixed summation order.
// Block = 32 columns x 32 part-lanes; each lane sums every 32nd part (about
// ten independent loads for a full grid, all in flight at once), then lane
// sums are added in order through shared memory.
constexpr int kReduceLanes = 32;

template <typename TW>
__global__ void __launch_bounds__(32 * kReduceLanes)
rms_dw_reduce(const float* __restrict__ partial, int parts, int64_t hidden, TW* __restrict__ dw) {
  __shared__ float s[kReduceLanes][33];
  // Launched as a programmatic dependent of the backward kernel: wait until
  // that grid has completed and its partials are visible.
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  const int64_t c = (int64_t)blockIdx.x * 32 + tx;
  float acc = 0.f;
  if (c < hidden) {
#pragma unroll 8
    for (int p = ty; p < parts; p += kReduceLanes) acc += partial[(int64_t)p * hidden + c];
  }
  s[ty][tx] = acc;
  __syncthreads();
  if (ty == 0 && c < hidden) {
    float tot = 0.f;
#pragma unroll
    for (int k = 0; k < kReduceLanes; ++k) tot += s[k][tx];
    dw[c] = from_f32<TW>(tot);
  }
}

int occupancy_grid(const void* kernel, int threads, size_t smem, int64_t work_ctas) {
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, threads, smem) != cudaSuccess ||
      per_sm <= 0)
    per_sm = 1;
  int64_t grid = (int64_t)num_sms() * per_sm;
  if (work_ctas < grid) grid = work_ctas;
  return static_cast<int>(std::max<int64_t>(grid, 1));
}

// Fewest CTAs (<= max_grid) that still need the same number of row
// iterations as max_grid: every CTA then does equal work and the last
// iteration is not a partial wave.
int64_t balanced_grid(int64_t work, int64_t max_grid) {
  max_grid = std::max<int64_t>(max_grid, 1);
  const int64_t iters = (work + max_grid - 1) / max_grid;
  return std::max<int64_t>(1, (work + iters - 1) / std::max<int64_t>(iters, 1));
}

// Grid used by the backward; the workspace size is derived from it, so the
// two must agree.  It depends only on sizes and the device's SM count.
constexpr int kBwdCtasPerSm = 4;
constexpr int kGenericGrid = 4;  // CTAs per SM for the generic kernels

int64_t bwd_grid_upper_bound(int64_t rows) {
  int64_t g = (int64_t)num_sms() * std::max(kBwdCtasPerSm, kGenericGrid);
  return std::max<int64_t>(1, std::min<int64_t>(g, rows));
}

template <typename TX, typename TW>
int launch_fwd(const void* x, const void* w, void* y, float* rrms, int64_t rows, int64_t hidden,
               float eps, cudaStream_t st) {
  const TX* xp = static_cast<const TX*>(x);
  const TW* wp = static_cast<const TW*>(w);
  TX* yp = static_cast<TX*>(y);
  RowCfg cfg = pick_cfg<TX>(hidden, x, y, x, y, false);
  // Sub-warp rows (the per-head q/k norm) stream through the cp.async ring:
  // 1.8x the register-prefetch kernel on [131072, 128] bf16.
  if (cfg.vec && cfg.nv == 1 && cfg.tpr < 32) {
    constexpr int S = kRingStages;
    cfg.groups = std::max(1, std::min(cfg.tpr < 32 ? 32 : 8, 512 / cfg.tpr));
    const int threads = cfg.tpr * cfg.groups;
    const size_t smem = (size_t)cfg.groups * S * cfg.tpr * 16;
    auto k = rms_fwd_ring<TX, TW, S>;
    static PerDevice<cudaError_t> attr;
    ML_CHECK_CUDA(attr.get([&] {
                    return cudaFuncSetAttribute(
                        (const void*)k, cudaFuncAttributeMaxDynamicSharedMemorySize, 96 * 1024);
                  }),
                  "rms_norm_forward: smem attribute");
    const int64_t work = (rows + cfg.groups - 1) / cfg.groups;
    const int grid = (int)balanced_grid(work, occupancy_grid((const void*)k, threads, smem, work));
    ML_CHECK_CUDA(launch_pdl(k, dim3(grid), dim3(threads), smem, st, xp, wp, yp, rrms, rows,
                             hidden, eps, cfg.tpr, cfg.groups),
                  "rms_norm_forward");
  } else if (cfg.vec) {
    const int threads = cfg.tpr * cfg.groups;
    const int64_t work = (rows + cfg.groups - 1) / cfg.groups;
#define ML_FWD_CASE(NV_)                                                                   \
  case NV_: {                                                                              \
    auto k = rms_fwd_vec<TX, TW, NV_>;                                                     \
    int grid = (int)balanced_grid(work, occupancy_grid((const void*)k, threads, 0, work)); \
    ML_CHECK_CUDA(launch_pdl(k, dim3(grid), dim3(threads), 0, st, xp, wp, yp, rrms, rows, \
                             hidden, eps, cfg.tpr, cfg.groups),                          \
                  "rms_norm_forward");                                                   \
    break;                                                                                 \
  }
    switch (cfg.nv) {
      ML_FWD_CASE(1)
      ML_FWD_CASE(2)
      ML_FWD_CASE(4)
      ML_FWD_CASE(8)
      default: set_error("rms_norm_forward: bad config"); return ML_ERR_INVALID_ARG;
    }
#undef ML_FWD_CASE
  } else {
    int grid = static_cast<int>(std::min<int64_t>(rows, (int64_t)num_sms() * kGenericGrid));
    ML_CHECK_CUDA(launch_pdl(rms_fwd_generic<TX, TW>, dim3(std::max(grid, 1)), dim3(256), 0, st,
                             xp, wp, yp, rrms, rows, hidden, eps),
                  "rms_norm_forward");
  }
  ML_CHECK_LAUNCH("rms_norm_forward");
  return ML_OK;
}

// Process-wide override of the backward's vectors per thread (0 = measured
// default; ml_rms_norm_set_bwd_vectors, a tuning and test knob).
std::atomic<int> g_bwd_nv{0};

template <typename TX, typename TW>
int launch_bwd(const void* x, const void* w, const float* rrms, const void* dy, void* dx, void* dw,
               float eps, float* partial, size_t partial_bytes, int64_t rows, int64_t hidden,
               cudaStream_t st) {
  const TX* xp = static_cast<const TX*>(x);
  const TW* wp = static_cast<const TW*>(w);
  const TX* gp = static_cast<const TX*>(dy);
  TX* dxp = static_cast<TX*>(dx);
  RowCfg cfg = pick_cfg<TX>(hidden, x, dy, dx, x, true);
  const int force_nv = g_bwd_nv.load(std::memory_order_relaxed);
  if (force_nv > 0 && cfg.vec) {
    // the same row split with the vectors per thread forced (rows whose split
    // does not fit a CTA keep the default)
    const int64_t nvec = hidden / (16 / (int64_t)sizeof(TX));
    const int64_t per = (nvec + force_nv - 1) / force_nv;
    const int64_t tpr = per <= 4 ? 4 : per <= 8 ? 8 : per <= 16 ? 16 : (per + 31) / 32 * 32;
    if (tpr <= (force_nv == 1 ? 512 : kMaxThreads)) {
      cfg.nv = force_nv;
      cfg.tpr = (int)tpr;
    }
  }
  if (cfg.vec)
    cfg.groups = std::max(1, std::min(cfg.tpr < 32 ? 32 : 8,
                                      bwd_max_threads<TX>(cfg.nv) / cfg.tpr));
  int grid = 0;
  const int64_t max_parts = static_cast<int64_t>(partial_bytes / (sizeof(float) * (size_t)hidden));
  // 16-bit rows of 257-512 vectors (hidden 2056-4096): the ring with two
  // vectors per thread, three row groups of 256 threads per CTA, one CTA
  // per SM (the layout knob still selects the others).
  const bool ring2 = cfg.vec && force_nv == 0 && sizeof(TX) == 2 && cfg.nv == 1 &&
                     cfg.tpr > 256 && cfg.tpr <= 512;
  if (ring2) {
    constexpr int S = 4, NV = 2, kGroups = 3;
    cfg.nv = NV;
    cfg.tpr = 256;
    cfg.groups = kGroups;
    const size_t ring_bytes = (size_t)kGroups * S * cfg.tpr * (2 * NV * 16 + 4);
    const size_t smem = std::max(ring_bytes, (size_t)kGroups * hidden * sizeof(float));
    const int threads = cfg.tpr * cfg.groups;
    auto k = rms_bwd_ring<TX, TW, S, NV>;
    static PerDevice<cudaError_t> attr;
    ML_CHECK_CUDA(attr.get([&] {
                    return cudaFuncSetAttribute(
                        (const void*)k, cudaFuncAttributeMaxDynamicSharedMemorySize, 210 * 1024);
                  }),
                  "rms_norm_backward: smem attribute");
    const int64_t work = (rows + cfg.groups - 1) / cfg.groups;
    const int per_sm = std::min<int>(
        kBwdCtasPerSm, occupancy_grid((const void*)k, threads, smem, 1 << 30) / num_sms());
    grid = static_cast<int>(balanced_grid(
        work, std::min<int64_t>((int64_t)num_sms() * std::max(per_sm, 1), max_parts)));
    ML_CHECK_CUDA(launch_pdl(k, dim3(grid), dim3(threads), smem, st, xp, wp, rrms, gp, dxp,
                             partial, rows, hidden, eps, cfg.tpr, cfg.groups),
                  "rms_norm_backward");
  } else if (cfg.vec && cfg.nv == 1) {
    constexpr int S = 4;
    cfg.groups = std::max(1, std::min(cfg.tpr < 32 ? 32 : 8, 512 / cfg.tpr));
    size_t smem = (size_t)cfg.groups * S * cfg.tpr * (2 * 16 + 4) +
                  (size_t)cfg.groups * hidden * sizeof(float);
    while (smem > 112 * 1024 && cfg.groups > 1) {
      cfg.groups /= 2;
      smem = (size_t)cfg.groups * S * cfg.tpr * (2 * 16 + 4) +
             (size_t)cfg.groups * hidden * sizeof(float);
    }
    const int threads = cfg.tpr * cfg.groups;
    auto k = rms_bwd_ring<TX, TW, S, 1>;
    static PerDevice<cudaError_t> attr;
    ML_CHECK_CUDA(attr.get([&] {
                    return cudaFuncSetAttribute(
                        (const void*)k, cudaFuncAttributeMaxDynamicSharedMemorySize, 112 * 1024);
                  }),
                  "rms_norm_backward: smem attribute");
    const int64_t work = (rows + cfg.groups - 1) / cfg.groups;
    const int per_sm = std::min<int>(
        kBwdCtasPerSm, occupancy_grid((const void*)k, threads, smem, 1 << 30) / num_sms());
    grid = static_cast<int>(balanced_grid(
        work, std::min<int64_t>((int64_t)num_sms() * std::max(per_sm, 1), max_parts)));
    ML_CHECK_CUDA(launch_pdl(k, dim3(grid), dim3(threads), smem, st, xp, wp, rrms, gp, dxp,
                             partial, rows, hidden, eps, cfg.tpr, cfg.groups),
                  "rms_norm_backward");
  } else if (cfg.vec) {
    const int threads = cfg.tpr * cfg.groups;
    size_t smem = cfg.groups > 1 ? (size_t)cfg.groups * hidden * sizeof(float) : 0;
    if (smem > 96 * 1024) {  // fold buffer too large: one row group per CTA
      cfg.groups = 1;
      smem = 0;
    }
    const int threads_eff = cfg.tpr * cfg.groups;
    (void)threads;
    const int64_t work = (rows + cfg.groups - 1) / cfg.groups;
#define ML_BWD_CASE(NV_)                                                                     \
  case NV_: {                                                                                \
    auto k = rms_bwd_vec<TX, TW, NV_>;                                                       \
    if (smem > 48 * 1024)                                                                    \
      ML_CHECK_CUDA(cudaFuncSetAttribute((const void*)k,                                     \
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,        \
                                         (int)smem),                                         \
                    "rms_norm_backward: smem attribute");                                    \
    const int per_sm = std::min<int>(                                                        \
        kBwdCtasPerSm, occupancy_grid((const void*)k, threads_eff, smem, 1 << 30) / num_sms()); \
    grid = static_cast<int>(balanced_grid(                                                   \
        work, std::min<int64_t>((int64_t)num_sms() * std::max(per_sm, 1), max_parts)));      \
    ML_CHECK_CUDA(launch_pdl(k, dim3(grid), dim3(threads_eff), smem, st, xp, wp, rrms, gp,  \
                             dxp, partial, rows, hidden, eps, cfg.tpr, cfg.groups),          \
                  "rms_norm_backward");                                                      \
    break;                                                                                   \
  }
    switch (cfg.nv) {
      ML_BWD_CASE(1)
      ML_BWD_CASE(2)
      ML_BWD_CASE(4)
      ML_BWD_CASE(8)
      default: set_error("rms_norm_backward: bad config"); return ML_ERR_INVALID_ARG;
    }
#undef ML_BWD_CASE
  } else {
    grid = static_cast<int>(std::min<int64_t>(
        std::min<int64_t>(rows, (int64_t)num_sms() * kGenericGrid), max_parts));
    grid = std::max(grid, 1);
    ML_CHECK_CUDA(launch_pdl(rms_bwd_generic<TX, TW>, dim3(grid), dim3(256), 0, st, xp, wp, rrms,
                             gp, dxp, partial, rows, hidden, eps),
                  "rms_norm_backward");
  }
  ML_CHECK_LAUNCH("rms_norm_backward");
  // Programmatic dependent launch: the reduction's launch overlaps the tail
  // of the backward grid instead of following it.
  cudaLaunchConfig_t lc = {};
  lc.gridDim = dim3(static_cast<unsigned>((hidden + 31) / 32), 1, 1);
  lc.blockDim = dim3(32 * kReduceLanes, 1, 1);
  lc.dynamicSmemBytes = 0;
  lc.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  lc.attrs = attr;
  lc.numAttrs = 1;
  ML_CHECK_CUDA(cudaLaunchKernelEx(&lc, rms_dw_reduce<TW>, (const float*)partial, grid, hidden,
                                   static_cast<TW*>(dw)),
                "rms_norm_backward(dweight reduce)");
  return ML_OK;
}

#define ML_DISPATCH_XW(XD, WD, FN, ...)                                             \
  [&]() -> int {                                                                    \
    switch ((XD) * 3 + (WD)) {                                                      \
      case ML_DTYPE_F32 * 3 + ML_DTYPE_F32: return FN<float, float>(__VA_ARGS__);   \
      case ML_DTYPE_F32 * 3 + ML_DTYPE_BF16: return FN<float, __nv_bfloat16>(__VA_ARGS__); \
      case ML_DTYPE_F32 * 3 + ML_DTYPE_F16: return FN<float, __half>(__VA_ARGS__);  \
      case ML_DTYPE_BF16 * 3 + ML_DTYPE_F32: return FN<__nv_bfloat16, float>(__VA_ARGS__); \
      case ML_DTYPE_BF16 * 3 + ML_DTYPE_BF16:                                       \
        return FN<__nv_bfloat16, __nv_bfloat16>(__VA_ARGS__);                       \
      case ML_DTYPE_BF16 * 3 + ML_DTYPE_F16: return FN<__nv_bfloat16, __half>(__VA_ARGS__); \
      case ML_DTYPE_F16 * 3 + ML_DTYPE_F32: return FN<__half, float>(__VA_ARGS__);  \
      case ML_DTYPE_F16 * 3 + ML_DTYPE_BF16: return FN<__half, __nv_bfloat16>(__VA_ARGS__); \
      case ML_DTYPE_F16 * 3 + ML_DTYPE_F16: return FN<__half, __half>(__VA_ARGS__); \
    }                                                                               \
    set_error("unsupported dtype pair (%d, %d)", (int)(XD), (int)(WD));             \
    return ML_ERR_INVALID_ARG;                                                      \
  }()

bool valid_dtype(int d) { return d == ML_DTYPE_F32 || d == ML_DTYPE_BF16 || d == ML_DTYPE_F16; }

// ---------------------------------------------------------------------------
// Scratch for ml_rms_norm_backward_noalloc: a file-scope device array, so the
// entry point never allocates.  Every GPU that loads this library holds it
// (4 MiB) until the process exits.
// ---------------------------------------------------------------------------
constexpr size_t kNoAllocScratchFloats = size_t(1) << 20;
static __device__ __align__(256) float g_rms_bwd_scratch[kNoAllocScratchFloats];

// Device address of g_rms_bwd_scratch on the current device.  Looked up once
// per device (with that device current) and cached; host code must never pass
// the symbol itself to a kernel, since on the host it only names a stand-in.
float* noalloc_scratch() {
  static std::mutex mu;
  static float* cache[64] = {nullptr};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
    set_error("rms_norm_backward_noalloc: no current CUDA device");
    return nullptr;
  }
  std::lock_guard<std::mutex> lock(mu);
  if (cache[dev] == nullptr) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_rms_bwd_scratch);
    if (e != cudaSuccess || p == nullptr) {
      set_error("rms_norm_backward_noalloc: cudaGetSymbolAddress failed: %s",
                cudaGetErrorString(e));
      return nullptr;
    }
    cache[dev] = static_cast<float*>(p);
  }
  return cache[dev];
}

}  // namespace
}  // namespace ml

using namespace ml;

extern "C" int ml_rms_norm_forward(const void* x, int x_dtype, const void* weight, int w_dtype,
                                   void* y, float* rrms, int64_t rows, int64_t hidden, float eps,
                                   void* stream) {
  ML_CHECK_ARG(valid_dtype(x_dtype) && valid_dtype(w_dtype),
               "rms_norm_forward: bad dtype codes (%d, %d)", x_dtype, w_dtype);
  ML_CHECK_ARG(rows >= 0 && hidden > 0, "rms_norm_forward: bad sizes rows=%lld hidden=%lld",
               (long long)rows, (long long)hidden);
  if (rows == 0) return ML_OK;
  ML_CHECK_ARG(x && weight && y, "rms_norm_forward: null pointer");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  return ML_DISPATCH_XW(x_dtype, w_dtype, launch_fwd, x, weight, y, rrms, rows, hidden, eps, st);
}

extern "C" size_t ml_rms_norm_backward_workspace_bytes(int64_t rows, int64_t hidden) {
  if (rows <= 0 || hidden <= 0) return 0;
  return (size_t)bwd_grid_upper_bound(rows) * (size_t)hidden * sizeof(float);
}

extern "C" int ml_rms_norm_set_bwd_vectors(int nv, int* previous) {
  ML_CHECK_ARG(nv == 0 || nv == 1 || nv == 2 || nv == 4 || nv == 8,
               "rms_norm_set_bwd_vectors: nv must be 0, 1, 2, 4 or 8");
  const int old = g_bwd_nv.exchange(nv);
  if (previous) *previous = old;
  return ML_OK;
}

extern "C" int ml_rms_norm_backward(const void* x, int x_dtype, const void* weight, int w_dtype,
                                    const float* rrms, const void* dy, void* dx, void* dweight,
                                    float eps, void* workspace, size_t workspace_bytes,
                                    int64_t rows, int64_t hidden, void* stream) {
  ML_CHECK_ARG(valid_dtype(x_dtype) && valid_dtype(w_dtype),
               "rms_norm_backward: bad dtype codes (%d, %d)", x_dtype, w_dtype);
  ML_CHECK_ARG(rows >= 0 && hidden > 0, "rms_norm_backward: bad sizes rows=%lld hidden=%lld",
               (long long)rows, (long long)hidden);
  ML_CHECK_ARG(weight && dweight, "rms_norm_backward: null weight/dweight");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (rows == 0) {
    // Empty input: dweight is an empty sum.
    const size_t wbytes = (size_t)hidden * (w_dtype == ML_DTYPE_F32 ? 4 : 2);
    ML_CHECK_CUDA(cudaMemsetAsync(dweight, 0, wbytes, st), "rms_norm_backward: memset");
    return ML_OK;
  }
  ML_CHECK_ARG(x && dy && dx, "rms_norm_backward: null pointer");
  ML_CHECK_ARG(workspace != nullptr && aligned16(workspace),
               "rms_norm_backward: workspace must be a non-null 16-byte aligned pointer");
  ML_CHECK_ARG(workspace_bytes >= (size_t)hidden * sizeof(float),
               "rms_norm_backward: workspace too small (%zu bytes)", workspace_bytes);
  return ML_DISPATCH_XW(x_dtype, w_dtype, launch_bwd, x, weight, rrms, dy, dx, dweight, eps,
                        static_cast<float*>(workspace), workspace_bytes, rows, hidden, st);
}

extern "C" int ml_rms_norm_backward_noalloc(const void* x, int x_dtype, const void* weight,
                                            int w_dtype, const float* rrms, const void* dy,
                                            void* dx, void* dweight, float eps, int64_t rows,
                                            int64_t hidden, void* stream) {
  ML_CHECK_ARG(valid_dtype(x_dtype) && valid_dtype(w_dtype),
               "rms_norm_backward_noalloc: bad dtype codes (%d, %d)", x_dtype, w_dtype);
  ML_CHECK_ARG(rows >= 0 && hidden > 0,
               "rms_norm_backward_noalloc: bad sizes rows=%lld hidden=%lld", (long long)rows,
               (long long)hidden);
  ML_CHECK_ARG((size_t)hidden <= kNoAllocScratchFloats,
               "rms_norm_backward_noalloc: hidden=%lld exceeds the static scratch limit of %zu "
               "columns; use ml_rms_norm_backward with a workspace",
               (long long)hidden, kNoAllocScratchFloats);
  ML_CHECK_ARG(weight && dweight, "rms_norm_backward_noalloc: null weight/dweight");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (rows == 0) {
    const size_t wbytes = (size_t)hidden * (w_dtype == ML_DTYPE_F32 ? 4 : 2);
    ML_CHECK_CUDA(cudaMemsetAsync(dweight, 0, wbytes, st), "rms_norm_backward_noalloc: memset");
    return ML_OK;
  }
  ML_CHECK_ARG(x && dy && dx, "rms_norm_backward_noalloc: null pointer");
  float* scratch = noalloc_scratch();
  if (scratch == nullptr) return ML_ERR_CUDA;
  // Every partial row the reduction reads is written earlier in this same
  // call, so the scratch needs no clearing between calls.
  return ML_DISPATCH_XW(x_dtype, w_dtype, launch_bwd, x, weight, rrms, dy, dx, dweight, eps,
                        scratch, kNoAllocScratchFloats * sizeof(float), rows, hidden, st);
}
