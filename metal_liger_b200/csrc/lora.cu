// Fused LoRA QKV and LoRA MLP (forward + backward) on sm_100a.
//
// Same results as the reference's _LoRA_QKV / _LoRA_MLP (ops/fused_lora.py:85-266):
//   y_i   = X W_i^T + s_i (X A_i^T) B_i^T
//   dA_i  = s_i (dY_i B_i)^T X,  dB_i = s_i dY_i^T (X A_i^T)   (fp32 results)
//   dX    = sum_i dY_i W_i + s_i (dY_i B_i) A_i                (frozen W: no dW)
// and for the MLP the SwiGLU in between (h = silu(gate) * up in fp32).
//
// Every product runs on the tcgen05 GEMM.  The rank-r terms never get their
// own pass over the big tensors: the adapters' A matrices are stacked into
// one [64, in] operand so a single skinny GEMM yields U = X [A_q;A_k;A_v]^T
// for all of them, and the low-rank update is folded into the base GEMM as
// one extra 64-wide K-segment ([X | U] [W | s B_pad]^T), accumulating in the
// same TMEM tile.  In the backward, dX = dQ Wq + dK Wk + dV Wv + G (s A) is a
// single 4-segment GEMM with G = [dQ Bq | dK Bk | dV Bv] (one 3-segment GEMM),
// and the dA/dB products are split-K GEMMs over the token dimension reading
// X / dY in their stored layout (MN-major operands, no transposes).
// Small pack kernels build the padded, scaled rank operands (<= 64 x out).
#include "gemm.cuh"

#include <algorithm>
#include <atomic>
#include <initializer_list>
#include <vector>

extern "C" int ml_swiglu_forward(const void* gate, const void* up, void* out, int64_t n, int dtype,
                                 void* stream);
extern "C" int ml_swiglu_backward(const void* gate, const void* up, const void* dout, void* dgate,
                                  void* dup, int64_t n, int dtype, void* stream);

namespace ml {
namespace lora {
namespace {

constexpr int kSlot = 64;  // padded rank width shared by the adapters of one call
using bf16 = __nv_bfloat16;

// SwiGLU inside the MLP's GEMMs (1, the default) or as separate elementwise
// passes (0): process-wide, read once per call (ml_lora_set_mlp_swiglu_fusion).
std::atomic<int> g_mlp_swiglu_fused{1};

inline size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

// Carves 256-byte-aligned buffers out of the caller's workspace; in dry mode
// it only measures, so sizing and use share one code path.
struct Arena {
  uint8_t* base = nullptr;
  size_t off = 0;
  bool dry = true;
  template <typename T>
  T* take(size_t count) {
    off = align256(off);
    T* p = dry ? nullptr : reinterpret_cast<T*>(base + off);
    off += count * sizeof(T);
    return p;
  }
};

// ------------------------------ pack kernels -------------------------------
// The rank operands of one call (stacked A's, slot-padded B's, their
// transposes, scaled copies) are assembled by ONE launch: every element of
// every destination operand is written exactly once — the value of the
// adapter block covering it, else 0 — so no memset precedes it.
constexpr int kMaxPieces = 3;
constexpr int kMaxOperands = 6;

// dst(r0 + i, c0 + j) = scale * src[i * cols + j]   (trans = 0: src is [rows, cols])
// dst(r0 + i, c0 + j) = scale * src[j * rows + i]   (trans = 1: src is [cols, rows])
struct Piece {
  const void* src;
  int64_t r0, c0, rows, cols;
  float scale;
  int dt;
  int trans;
};

struct Operand {
  bf16* dst;
  int64_t ld, rows, cols;
  int npieces;
  Piece p[kMaxPieces];
};

struct Assembly {
  Operand op[kMaxOperands];
  int64_t start[kMaxOperands + 1];  // prefix sums of rows * cols
  int nops;
};

// One thread per 8 consecutive destination elements of a row (every operand
// width is a multiple of 8), written as one 16-byte store; 32-bit index math
// (the host checks the total fits).
__global__ void __launch_bounds__(256) assemble_k(const __grid_constant__ Assembly a) {
  pdl_wait();  // a programmatic dependent: the pieces may come from the previous kernel
  pdl_release();
  const int e8 = blockIdx.x * blockDim.x + threadIdx.x;  // index of an 8-element chunk
  if (e8 >= (int)(a.start[a.nops] >> 3)) return;
  const int e = e8 << 3;
  int k = 0;
  while (k + 1 < a.nops && e >= (int)a.start[k + 1]) ++k;
  const Operand& o = a.op[k];
  const int local = e - (int)a.start[k];
  const int cols = (int)o.cols;
  const int r = local / cols, c0 = local - r * cols;
  Vec16<bf16> out;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const int c = c0 + j;
    float v = 0.f;
    for (int q = 0; q < o.npieces; ++q) {
      const Piece& pc = o.p[q];
      const int i = r - (int)pc.r0, jj = c - (int)pc.c0;
      if (i >= 0 && i < (int)pc.rows && jj >= 0 && jj < (int)pc.cols)
        v = pc.scale * load_as_f32(pc.src,
                                   pc.trans ? (int64_t)jj * pc.rows + i : (int64_t)i * pc.cols + jj,
                                   pc.dt);
    }
    out.v[j] = __float2bfloat16_rn(v);
  }
  *reinterpret_cast<Vec16<bf16>*>(o.dst + (int64_t)r * o.ld + c0) = out;
}

// Scatter of the fp32 [n, 64] skinny-GEMM results into the per-adapter
// gradients, several adapters per launch.  The results arrive as the
// split-K GEMM's `splits` partial slabs (split_stride floats apart), summed
// here in slab order — the sum a separate reduction kernel would form, so
// none is launched:
//   trans = 0 (dB): dst[i * cols + j] = scale * sum_s src[s][i * 64 + off + j]   dst [rows, cols = r]
//   trans = 1 (dA): dst[i * cols + j] = scale * sum_s src[s][j * 64 + off + i]   dst [rows = r, cols]
struct UnpackJob {
  void* dst;         // in the adapter parameter's dtype (dt)
  const float* src;
  int64_t rows, cols, off;
  int64_t split_stride;
  int splits;
  float scale;
  int trans;
  int dt;
};

constexpr int kMaxUnpack = 6;

struct Unpacks {
  UnpackJob j[kMaxUnpack];
  int64_t start[kMaxUnpack + 1];
  int n;
};

__global__ void unpack_k(const __grid_constant__ Unpacks u) {
  pdl_wait();  // a programmatic dependent: the slabs come from the previous GEMM
  pdl_release();
  const int64_t total = u.start[u.n];
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total;
       e += (int64_t)gridDim.x * blockDim.x) {
    int k = 0;
    while (k + 1 < u.n && e >= u.start[k + 1]) ++k;
    const UnpackJob& jb = u.j[k];
    const int64_t local = e - u.start[k];
    const int64_t i = local / jb.cols, j = local - (local / jb.cols) * jb.cols;
    const int64_t at = jb.trans ? j * kSlot + jb.off + i : i * kSlot + jb.off + j;
    float acc = 0.f;
    for (int sp = 0; sp < jb.splits; ++sp) acc += jb.src[sp * jb.split_stride + at];
    store_from_f32(jb.dst, local, jb.dt, jb.scale * acc);
  }
}

inline int egrid(int64_t n) {
  return (int)std::max<int64_t>(1, std::min<int64_t>((n + 255) / 256, (int64_t)num_sms() * 8));
}

#define LORA_LAUNCH(kernel, n, ...)                                        \
  do {                                                                     \
    if ((n) > 0) {                                                         \
      kernel<<<egrid(n), 256, 0, st>>>(__VA_ARGS__);                       \
      ML_CHECK_LAUNCH(#kernel);                                            \
    }                                                                      \
  } while (0)

#define LORA_TRY(call)          \
  do {                                \
    int _rc = (call);                 \
    if (_rc != ML_OK) return _rc;     \
  } while (0)

int zero(void* p, size_t bytes, cudaStream_t st) {
  ML_CHECK_CUDA(cudaMemsetAsync(p, 0, bytes, st), "lora: memset");
  return ML_OK;
}

Piece piece(const void* src, int dt, int64_t r0, int64_t c0, int64_t rows, int64_t cols,
            float scale, bool trans) {
  Piece p;
  p.src = src;
  p.dt = dt;
  p.r0 = r0;
  p.c0 = c0;
  p.rows = rows;
  p.cols = cols;
  p.scale = scale;
  p.trans = trans ? 1 : 0;
  return p;
}

// Collects the operands of one call and launches assemble_k once.
struct Assembler {
  Assembly a{};
  int add(bf16* dst, int64_t rows, int64_t cols, std::initializer_list<Piece> pieces) {
    if (a.nops >= kMaxOperands || pieces.size() > (size_t)kMaxPieces) {
      set_error("lora: too many rank operands in one assembly");
      return ML_ERR_INVALID_ARG;
    }
    Operand& o = a.op[a.nops];
    o.dst = dst;
    o.ld = cols;
    o.rows = rows;
    o.cols = cols;
    o.npieces = 0;
    for (const Piece& p : pieces) o.p[o.npieces++] = p;
    a.start[a.nops + 1] = a.start[a.nops] + rows * cols;
    ++a.nops;
    return ML_OK;
  }
  int launch(cudaStream_t st) {
    const int64_t n = a.start[a.nops];
    if (n == 0) return ML_OK;
    if (n >= ((int64_t)1 << 31)) {
      set_error("lora: rank operands too large (%lld elements)", (long long)n);
      return ML_ERR_INVALID_ARG;
    }
    for (int k = 0; k < a.nops; ++k)
      if (a.op[k].cols % 8 != 0 || a.op[k].ld % 8 != 0 ||
          (reinterpret_cast<uintptr_t>(a.op[k].dst) & 15) != 0) {
        set_error("lora: rank operand %d is not 16-byte granular", k);
        return ML_ERR_INVALID_ARG;
      }
    const int64_t chunks = n / 8;
    ML_CHECK_CUDA(launch_pdl(assemble_k, dim3((unsigned)((chunks + 255) / 256)), dim3(256), 0,
                             st, a),
                  "lora: assemble rank operands");
    return ML_OK;
  }
};

// The split-K partial slabs of one skinny product (summed by unpack_k).
struct Partials {
  const float* ptr = nullptr;
  int splits = 1;
  int64_t split_stride = 0;
};

struct Unpacker {
  Unpacks u{};
  // `p` holds `p.splits` partial slabs of `p.split_stride` floats each.
  int add(void* dst, int dt, const Partials& p, int64_t rows, int64_t cols, int64_t off,
          float scale, bool trans) {
    if (u.n >= kMaxUnpack) {
      set_error("lora: too many gradient scatters in one launch");
      return ML_ERR_INVALID_ARG;
    }
    UnpackJob& j = u.j[u.n];
    j.dst = dst;
    j.src = p.ptr;
    j.splits = p.splits;
    j.split_stride = p.split_stride;
    j.rows = rows;
    j.cols = cols;
    j.off = off;
    j.scale = scale;
    j.trans = trans ? 1 : 0;
    j.dt = dt;
    u.start[u.n + 1] = u.start[u.n] + rows * cols;
    ++u.n;
    return ML_OK;
  }
  int launch(cudaStream_t st) {
    const int64_t n = u.start[u.n];
    if (n == 0) return ML_OK;
    ML_CHECK_CUDA(launch_pdl(unpack_k, dim3(egrid(n)), dim3(256), 0, st, u),
                  "lora: scatter adapter gradients");
    return ML_OK;
  }
};

// One K-segment: A [M, K] / B [N, K] logical views.
gemm::Seg seg(const void* a, int64_t lda, const void* b, int64_t ldb, int64_t k) {
  gemm::Seg s;
  s.a.ptr = a;
  s.a.ld = lda;
  s.b.ptr = b;
  s.b.ld = ldb;
  s.K = k;
  return s;
}

// D[M, N] (bf16, pitch ldd) = sum of segments (at most gemm::kMaxSeg).
int gemm_bf16(int64_t M, int64_t N, const gemm::Seg* segs, size_t nseg, bool a_mn, bool b_mn,
              void* D, int64_t ldd, cudaStream_t st) {
  if (nseg == 0 || nseg > (size_t)gemm::kMaxSeg) {
    set_error("lora: %zu GEMM segments (1..%d supported)", nseg, gemm::kMaxSeg);
    return ML_ERR_INVALID_ARG;
  }
  gemm::Problem p;
  p.M = M;
  p.N = N;
  p.nseg = 0;
  for (size_t i = 0; i < nseg; ++i) p.seg[p.nseg++] = segs[i];
  p.a_mn = a_mn;
  p.b_mn = b_mn;
  p.epi = gemm::EPI_STORE;
  p.d_f32 = false;
  p.D = D;
  p.ldd = ldd;
  return gemm::launch(p, st);
}

int gemm_bf16(int64_t M, int64_t N, std::initializer_list<gemm::Seg> segs, bool a_mn, bool b_mn,
              void* D, int64_t ldd, cudaStream_t st) {
  return gemm_bf16(M, N, segs.begin(), segs.size(), a_mn, b_mn, D, ldd, st);
}

int gemm_bf16(int64_t M, int64_t N, const std::vector<gemm::Seg>& segs, bool a_mn, bool b_mn,
              void* D, int64_t ldd, cudaStream_t st) {
  return gemm_bf16(M, N, segs.data(), segs.size(), a_mn, b_mn, D, ldd, st);
}

size_t skinny_partial_floats(int64_t M, int64_t K) {
  return (size_t)gemm::auto_splits(M, kSlot, K) * (size_t)M * kSlot;
}

// One A^T-style skinny product over the token dimension: [M, 64] fp32 from
// A (MN-major, M columns) and B (MN-major, 64 columns), K = tokens.
struct Skinny {
  int64_t M;
  gemm::Seg s;
};

// Up to gemm::kMaxSeg skinny products sharing K, stacked along M in ONE
// grouped split-K GEMM launch and left as its partial slabs in `partial`
// (skinny_partial_floats(sum M, K) floats) for unpack_k to sum: no reduction
// launch.  outs[g] locates product g's rows in the slabs.
int gemm_skinny_partials(std::initializer_list<Skinny> parts, float* partial, Partials* outs,
                         cudaStream_t st) {
  gemm::Problem p;
  p.N = kSlot;
  p.a_mn = true;
  p.b_mn = true;
  p.epi = gemm::EPI_PARTIAL;
  int g = 0;
  int64_t total = 0;
  for (const Skinny& q : parts) {
    if (g == gemm::kMaxSeg) {
      set_error("lora: more than %d skinny products in one launch", gemm::kMaxSeg);
      return ML_ERR_INVALID_ARG;
    }
    p.seg[g] = q.s;
    p.grp_m[g] = q.M;
    total += q.M;
    ++g;
  }
  p.nseg = g;
  p.m_groups = g;
  p.M = total;
  p.splits = gemm::auto_splits(total, kSlot, p.seg[0].K);
  p.D = partial;
  p.ldd = kSlot;
  p.split_stride = total * kSlot;
  int64_t row = 0;
  for (int i = 0; i < g; ++i) {
    outs[i].ptr = partial + row * kSlot;
    outs[i].splits = p.splits;
    outs[i].split_stride = total * kSlot;
    row += p.grp_m[i];
  }
  return gemm::launch(p, st);
}

// out[T, 64] bf16 = sum of segments: the rank projections (U = X A^T,
// G = dY B).  With few tokens the 128-row tiles do not cover the GPU, so the
// reduction over K is split (fixed-order fp32 reduce) when the caller's
// partial buffer (skinny_partial_floats(T, K)) allows.
int rank_proj(int64_t T, const gemm::Seg* segs, size_t nseg, bf16* out, float* part,
              size_t part_floats, cudaStream_t st) {
  int64_t K = 0;
  for (size_t i = 0; i < nseg; ++i) K += segs[i].K;
  const int splits = gemm::auto_splits(T, kSlot, K);
  if (splits <= 1 || part == nullptr || part_floats < (size_t)splits * (size_t)T * kSlot)
    return gemm_bf16(T, kSlot, segs, nseg, false, false, out, kSlot, st);
  if (nseg == 0 || nseg > (size_t)gemm::kMaxSeg) {
    set_error("lora: %zu GEMM segments (1..%d supported)", nseg, gemm::kMaxSeg);
    return ML_ERR_INVALID_ARG;
  }
  gemm::Problem p;
  p.M = T;
  p.N = kSlot;
  p.nseg = 0;
  for (size_t i = 0; i < nseg; ++i) p.seg[p.nseg++] = segs[i];
  p.a_mn = false;
  p.b_mn = false;
  return gemm::launch_splitk_to(p, splits, out, false, kSlot, part, part_floats * 4, st);
}

int rank_proj(int64_t T, std::initializer_list<gemm::Seg> segs, bf16* out, float* part,
              size_t part_floats, cudaStream_t st) {
  return rank_proj(T, segs.begin(), segs.size(), out, part, part_floats, st);
}

int rank_proj(int64_t T, const std::vector<gemm::Seg>& segs, bf16* out, float* part,
              size_t part_floats, cudaStream_t st) {
  return rank_proj(T, segs.data(), segs.size(), out, part, part_floats, st);
}

inline size_t esize(int dtype) { return dtype == ML_DTYPE_F32 ? 4 : 2; }

bool valid_proj(const ml_lora_proj& p) {
  return p.w && p.a && p.b && p.out_features > 0 && p.a_dtype >= 0 && p.a_dtype <= 2 &&
         p.b_dtype >= 0 && p.b_dtype <= 2;
}

// --------------------------- QKV (1-3 projections) -------------------------
// `np` projections of one input X (Q/K/V: np = 3; a single LoRA linear such as
// o_proj: np = 1).  Adapter i owns rank slot [i r, (i + 1) r) of the 64-wide
// rank operands, so np * r <= 64.
int qkv_forward(const bf16* x, int64_t T, int64_t H, int64_t r, int np, const ml_lora_proj* pj,
                void* const* out, bf16* u, Arena& ar, cudaStream_t st) {
  bf16* acat = ar.take<bf16>((size_t)kSlot * H);
  bf16* bpad[3] = {};
  for (int i = 0; i < np; ++i) bpad[i] = ar.take<bf16>((size_t)pj[i].out_features * kSlot);
  const size_t rpf = skinny_partial_floats(T, H);
  float* rpart = ar.take<float>(rpf);
  if (ar.dry) return ML_OK;
  // acat = [A_0; A_1; ...] (rows i r ..), bpad_i = s_i B_i in columns [i r, (i + 1) r)
  Assembler as;
  {
    Piece pa[3];
    for (int i = 0; i < np; ++i) pa[i] = piece(pj[i].a, pj[i].a_dtype, i * r, 0, r, H, 1.f, false);
    if (np == 1) LORA_TRY(as.add(acat, kSlot, H, {pa[0]}));
    if (np == 2) LORA_TRY(as.add(acat, kSlot, H, {pa[0], pa[1]}));
    if (np == 3) LORA_TRY(as.add(acat, kSlot, H, {pa[0], pa[1], pa[2]}));
  }
  for (int i = 0; i < np; ++i) {
    const int64_t o = pj[i].out_features;
    LORA_TRY(as.add(bpad[i], o, kSlot,
                    {piece(pj[i].b, pj[i].b_dtype, 0, i * r, o, r, pj[i].scaling, false)}));
  }
  LORA_TRY(as.launch(st));
  // U = X [A_0; A_1; ...]^T   [T, 64]
  LORA_TRY(rank_proj(T, {seg(x, H, acat, H, H)}, u, rpart, rpf, st));
  // y_i = [X | U] [W_i | s_i B_i (in its slot)]^T
  for (int i = 0; i < np; ++i) {
    const int64_t o = pj[i].out_features;
    LORA_TRY(gemm_bf16(T, o, {seg(x, H, pj[i].w, H, H), seg(u, kSlot, bpad[i], kSlot, kSlot)},
                       false, false, out[i], o, st));
  }
  return ML_OK;
}

int qkv_backward(const bf16* x, const bf16* u, int64_t T, int64_t H, int64_t r, int np,
                 const ml_lora_proj* pj, const void* const* dy, bf16* dx, void* const* da,
                 void* const* db, Arena& ar, cudaStream_t st) {
  int64_t osum = 0;
  for (int i = 0; i < np; ++i) osum += pj[i].out_features;
  bf16* bt[3] = {};
  for (int i = 0; i < np; ++i) bt[i] = ar.take<bf16>((size_t)kSlot * pj[i].out_features);
  bf16* acat_s = ar.take<bf16>((size_t)kSlot * H);
  bf16* G = ar.take<bf16>((size_t)T * kSlot);
  // split-K partial slabs of dA (X^T G) and of every dB (dY_i^T U), one
  // grouped launch, summed by unpack_k
  float* dABp = ar.take<float>(skinny_partial_floats(H + osum, T));
  const size_t pf = skinny_partial_floats(T, osum);
  float* part = ar.take<float>(pf);
  if (ar.dry) return ML_OK;
  // bt_i = B_i^T in rows [i r, (i + 1) r); acat_s = [s_0 A_0; s_1 A_1; ...]
  Assembler as;
  for (int i = 0; i < np; ++i) {
    const int64_t o = pj[i].out_features;
    LORA_TRY(as.add(bt[i], kSlot, o, {piece(pj[i].b, pj[i].b_dtype, i * r, 0, r, o, 1.f, true)}));
  }
  {
    Piece pa[3];
    for (int i = 0; i < np; ++i)
      pa[i] = piece(pj[i].a, pj[i].a_dtype, i * r, 0, r, H, pj[i].scaling, false);
    if (np == 1) LORA_TRY(as.add(acat_s, kSlot, H, {pa[0]}));
    if (np == 2) LORA_TRY(as.add(acat_s, kSlot, H, {pa[0], pa[1]}));
    if (np == 3) LORA_TRY(as.add(acat_s, kSlot, H, {pa[0], pa[1], pa[2]}));
  }
  LORA_TRY(as.launch(st));
  // G = [dY_0 B_0 | dY_1 B_1 | ...]   [T, 64]
  std::vector<gemm::Seg> gsegs, xsegs;
  for (int i = 0; i < np; ++i) {
    const int64_t o = pj[i].out_features;
    gsegs.push_back(seg(dy[i], o, bt[i], o, o));
    xsegs.push_back(seg(dy[i], o, pj[i].w, H, o));
  }
  xsegs.push_back(seg(G, kSlot, acat_s, H, kSlot));
  LORA_TRY(rank_proj(T, gsegs, G, part, pf, st));
  // dX = sum_i dY_i W_i + G (s A)   — one accumulator, W read in place (N-major)
  LORA_TRY(gemm_bf16(T, H, xsegs, false, true, dx, H, st));
  // dA_i = s_i (X^T G)[:, slot_i]^T ;  dB_i = s_i dY_i^T U[:, slot_i]
  Partials pp[4];  // [0] = dA, [1 + i] = dB_i
  {
    const Skinny a{H, seg(x, H, G, kSlot, T)};
    Skinny b[3];
    for (int i = 0; i < np; ++i) {
      const int64_t o = pj[i].out_features;
      b[i] = {o, seg(dy[i], o, u, kSlot, T)};
    }
    if (np == 1) LORA_TRY(gemm_skinny_partials({a, b[0]}, dABp, pp, st));
    if (np == 2) LORA_TRY(gemm_skinny_partials({a, b[0], b[1]}, dABp, pp, st));
    if (np == 3) LORA_TRY(gemm_skinny_partials({a, b[0], b[1], b[2]}, dABp, pp, st));
  }
  Unpacker un;
  for (int i = 0; i < np; ++i) {
    LORA_TRY(un.add(da[i], pj[i].a_dtype, pp[0], r, H, i * r, pj[i].scaling, true));
    LORA_TRY(un.add(db[i], pj[i].b_dtype, pp[1 + i], pj[i].out_features, r, i * r,
                    pj[i].scaling, false));
  }
  return un.launch(st);
}

// ------------------------------- MLP --------------------------------------
// With the SwiGLU fused into the GEMMs (the default):
//  * forward: ONE GEMM produces gate, up and h.  Its 256-wide tiles take B
//    rows [128 n, 128 n + 128) of [Wg | s_g Bg] for the first half and of
//    [Wu | s_u Bu] for the second (two tensor maps, no weight copy), so the
//    accumulator holds gate and up of the same 128 intermediate columns and
//    the epilogue writes gate, up (saved for the backward) and
//    h = silu(gate) * up from the bf16-rounded values — the separate SwiGLU
//    pass, which re-read gate and up, is gone;
//  * backward: the dH GEMM's epilogue applies the SwiGLU backward with the
//    saved gate / up and writes d_gate / d_up — dH never reaches memory.
// Both round exactly where the unfused path stores bf16 tensors, so their
// outputs are bitwise those of the unfused kernels.
// pj[0] = gate (I x H), pj[1] = up (I x H), pj[2] = down (H x I).
int mlp_forward(const bf16* x, int64_t T, int64_t H, int64_t I, int64_t r,
                const ml_lora_proj* pj, bf16* gate, bf16* up, bf16* h, bf16* out, bf16* u1,
                bf16* u2, Arena& ar, cudaStream_t st) {
  const bool fused = g_mlp_swiglu_fused.load(std::memory_order_relaxed) != 0;
  bf16* acat = ar.take<bf16>((size_t)kSlot * H);   // rows [0,r) = Ag, [r,2r) = Au
  bf16* bgp = ar.take<bf16>((size_t)I * kSlot);     // cols [0,r) = s_g Bg
  bf16* bup = ar.take<bf16>((size_t)I * kSlot);     // cols [r,2r) = s_u Bu
  bf16* ad = ar.take<bf16>((size_t)kSlot * I);      // rows [0,r) = Ad
  bf16* bdp = ar.take<bf16>((size_t)H * kSlot);     // cols [0,r) = s_d Bd
  const size_t rpf = std::max(skinny_partial_floats(T, H), skinny_partial_floats(T, I));
  float* rpart = ar.take<float>(rpf);
  if (ar.dry) return ML_OK;
  Assembler as;
  LORA_TRY(as.add(acat, kSlot, H,
                  {piece(pj[0].a, pj[0].a_dtype, 0, 0, r, H, 1.f, false),
                   piece(pj[1].a, pj[1].a_dtype, r, 0, r, H, 1.f, false)}));
  LORA_TRY(as.add(bgp, I, kSlot, {piece(pj[0].b, pj[0].b_dtype, 0, 0, I, r, pj[0].scaling, false)}));
  LORA_TRY(as.add(bup, I, kSlot, {piece(pj[1].b, pj[1].b_dtype, 0, r, I, r, pj[1].scaling, false)}));
  LORA_TRY(as.add(ad, kSlot, I, {piece(pj[2].a, pj[2].a_dtype, 0, 0, r, I, 1.f, false)}));
  LORA_TRY(as.add(bdp, H, kSlot, {piece(pj[2].b, pj[2].b_dtype, 0, 0, H, r, pj[2].scaling, false)}));
  LORA_TRY(as.launch(st));
  // U1 = X [Ag; Au]^T
  LORA_TRY(rank_proj(T, {seg(x, H, acat, H, H)}, u1, rpart, rpf, st));
  if (fused) {
    // gate | up = [X | U1] [W | s B]^T of both projections, h in the epilogue
    gemm::Problem p;
    p.M = T;
    p.N = I;
    p.nseg = 2;
    p.seg[0] = seg(x, H, pj[0].w, H, H);
    p.seg[0].b2 = {pj[1].w, I, H, H};
    p.seg[1] = seg(u1, kSlot, bgp, kSlot, kSlot);
    p.seg[1].b2 = {bup, I, kSlot, kSlot};
    p.b_split = true;
    p.bn = 256;
    p.epi = gemm::EPI_SWIGLU;
    p.D = gate;
    p.D2 = up;
    p.D3 = h;
    p.ldd = I;
    LORA_TRY(gemm::launch(p, st));
  } else {
    // gate / up = [X | U1] [W | s B]^T
    LORA_TRY(gemm_bf16(T, I, {seg(x, H, pj[0].w, H, H), seg(u1, kSlot, bgp, kSlot, kSlot)},
                       false, false, gate, I, st));
    LORA_TRY(gemm_bf16(T, I, {seg(x, H, pj[1].w, H, H), seg(u1, kSlot, bup, kSlot, kSlot)},
                       false, false, up, I, st));
    // h = silu(gate) * up (fp32 math)
    LORA_TRY(ml_swiglu_forward(gate, up, h, T * I, ML_DTYPE_BF16, st));
  }
  // U2 = h Ad^T ; out = [h | U2] [Wd | s Bd]^T
  LORA_TRY(rank_proj(T, {seg(h, I, ad, I, I)}, u2, rpart, rpf, st));
  LORA_TRY(gemm_bf16(T, H, {seg(h, I, pj[2].w, I, I), seg(u2, kSlot, bdp, kSlot, kSlot)}, false,
                     false, out, H, st));
  return ML_OK;
}

int mlp_backward(const bf16* x, const bf16* gate, const bf16* up, const bf16* h, const bf16* u1,
                 const bf16* u2, int64_t T, int64_t H, int64_t I, int64_t r,
                 const ml_lora_proj* pj, const bf16* dy, bf16* dx, void* const* da,
                 void* const* db, Arena& ar, cudaStream_t st) {
  const bool fused = g_mlp_swiglu_fused.load(std::memory_order_relaxed) != 0;
  bf16* bdT = ar.take<bf16>((size_t)kSlot * H);     // rows [0,r) = Bd^T
  bf16* ads = ar.take<bf16>((size_t)kSlot * I);     // rows [0,r) = s_d Ad
  bf16* bgT = ar.take<bf16>((size_t)kSlot * I);     // rows [0,r) = Bg^T
  bf16* buT = ar.take<bf16>((size_t)kSlot * I);     // rows [r,2r) = Bu^T
  bf16* acs = ar.take<bf16>((size_t)kSlot * H);     // rows [0,r) = s_g Ag, [r,2r) = s_u Au
  bf16* Gd = ar.take<bf16>((size_t)T * kSlot);
  bf16* Ggu = ar.take<bf16>((size_t)T * kSlot);
  bf16* dH = fused ? nullptr : ar.take<bf16>((size_t)T * I);
  bf16* dgate = ar.take<bf16>((size_t)T * I);
  bf16* dup = ar.take<bf16>((size_t)T * I);
  // split-K partial slabs of the adapter-gradient products in two grouped
  // launches, summed by unpack_k: the down adapter's [h^T G_d; dY^T U2] and
  // the gate/up adapters' [X^T G_gu; d_gate^T U1; d_up^T U1]
  float* down_p = ar.take<float>(skinny_partial_floats(I + H, T));
  float* gu_p = ar.take<float>(skinny_partial_floats(H + 2 * I, T));
  const size_t pf = std::max(skinny_partial_floats(T, H), skinny_partial_floats(T, 2 * I));
  float* part = ar.take<float>(pf);
  if (ar.dry) return ML_OK;
  Assembler as;
  LORA_TRY(as.add(bdT, kSlot, H, {piece(pj[2].b, pj[2].b_dtype, 0, 0, r, H, 1.f, true)}));
  LORA_TRY(as.add(ads, kSlot, I, {piece(pj[2].a, pj[2].a_dtype, 0, 0, r, I, pj[2].scaling, false)}));
  LORA_TRY(as.add(bgT, kSlot, I, {piece(pj[0].b, pj[0].b_dtype, 0, 0, r, I, 1.f, true)}));
  LORA_TRY(as.add(buT, kSlot, I, {piece(pj[1].b, pj[1].b_dtype, r, 0, r, I, 1.f, true)}));
  LORA_TRY(as.add(acs, kSlot, H,
                  {piece(pj[0].a, pj[0].a_dtype, 0, 0, r, H, pj[0].scaling, false),
                   piece(pj[1].a, pj[1].a_dtype, r, 0, r, H, pj[1].scaling, false)}));
  LORA_TRY(as.launch(st));
  // G_d = dY Bd ; dH = dY Wd + G_d (s_d Ad)      (Wd stored [H, I]: N-major)
  LORA_TRY(rank_proj(T, {seg(dy, H, bdT, H, H)}, Gd, part, pf, st));
  if (fused) {
    // d_gate, d_up from the dH accumulator and the saved gate / up
    gemm::Problem p;
    p.M = T;
    p.N = I;
    p.nseg = 2;
    p.seg[0] = seg(dy, H, pj[2].w, I, H);
    p.seg[1] = seg(Gd, kSlot, ads, I, kSlot);
    p.b_mn = true;
    p.epi = gemm::EPI_DSWIGLU;
    p.D = dgate;
    p.D2 = dup;
    p.aux1 = gate;
    p.aux2 = up;
    p.ldd = I;
    LORA_TRY(gemm::launch(p, st));
  } else {
    LORA_TRY(gemm_bf16(T, I, {seg(dy, H, pj[2].w, I, H), seg(Gd, kSlot, ads, I, kSlot)}, false,
                       true, dH, I, st));
  }
  // down adapter grads: dA_d = s_d (h^T G_d)^T, dB_d = s_d dY^T U2
  Partials pd[2], pgu[3];  // {dA_d, dB_d}, {dA_gu, dB_g, dB_u}
  LORA_TRY(gemm_skinny_partials({{I, seg(h, I, Gd, kSlot, T)}, {H, seg(dy, H, u2, kSlot, T)}},
                                down_p, pd, st));
  // SwiGLU backward (sigmoid recomputed), unless the dH GEMM applied it
  if (!fused) LORA_TRY(ml_swiglu_backward(gate, up, dH, dgate, dup, T * I, ML_DTYPE_BF16, st));
  // G_gu = [d_gate Bg | d_up Bu]
  LORA_TRY(rank_proj(T, {seg(dgate, I, bgT, I, I), seg(dup, I, buT, I, I)}, Ggu, part, pf, st));
  // dX = d_gate Wg + d_up Wu + G_gu (s A)        (Wg/Wu stored [I, H]: N-major)
  LORA_TRY(gemm_bf16(T, H,
                     {seg(dgate, I, pj[0].w, H, I), seg(dup, I, pj[1].w, H, I),
                      seg(Ggu, kSlot, acs, H, kSlot)},
                     false, true, dx, H, st));
  // gate/up adapter grads
  LORA_TRY(gemm_skinny_partials({{H, seg(x, H, Ggu, kSlot, T)},
                                 {I, seg(dgate, I, u1, kSlot, T)},
                                 {I, seg(dup, I, u1, kSlot, T)}},
                                gu_p, pgu, st));
  Unpacker un;
  LORA_TRY(un.add(da[2], pj[2].a_dtype, pd[0], r, I, 0, pj[2].scaling, true));
  LORA_TRY(un.add(db[2], pj[2].b_dtype, pd[1], H, r, 0, pj[2].scaling, false));
  LORA_TRY(un.add(da[0], pj[0].a_dtype, pgu[0], r, H, 0, pj[0].scaling, true));
  LORA_TRY(un.add(da[1], pj[1].a_dtype, pgu[0], r, H, r, pj[1].scaling, true));
  LORA_TRY(un.add(db[0], pj[0].b_dtype, pgu[1], I, r, 0, pj[0].scaling, false));
  LORA_TRY(un.add(db[1], pj[1].b_dtype, pgu[2], I, r, r, pj[1].scaling, false));
  return un.launch(st);
}

int check_ws(const Arena& need, size_t have, void* ws, const char* what) {
  if (ws == nullptr || ((uintptr_t)ws & 255) != 0) {
    set_error("%s: workspace must be a non-null 256-byte aligned pointer", what);
    return ML_ERR_INVALID_ARG;
  }
  if (have < need.off) {
    set_error("%s: workspace too small (%zu < %zu bytes)", what, have, need.off);
    return ML_ERR_INVALID_ARG;
  }
  return ML_OK;
}

}  // namespace
}  // namespace lora
}  // namespace ml

using namespace ml;
using lora::Arena;

#define LORA_ARGCHECK_COMMON(what, NP)                                                       \
  ML_CHECK_ARG(tokens >= 0 && in_features > 0 && rank > 0, what ": bad sizes");              \
  ML_CHECK_ARG(in_features % 8 == 0, what ": in_features must be a multiple of 8");          \
  ML_CHECK_ARG((NP) >= 1 && (NP) <= 3, what ": nproj must be 1, 2 or 3");                    \
  ML_CHECK_ARG((NP) * rank <= lora::kSlot, what ": nproj * rank = %lld > 64 is not supported", \
               (long long)((NP) * rank));                                                    \
  ML_CHECK_ARG(proj != nullptr, what ": null projections");                                   \
  for (int _i = 0; _i < (NP); ++_i)                                                           \
    ML_CHECK_ARG(lora::valid_proj(proj[_i]) && proj[_i].out_features % 8 == 0,                \
                 what ": projection %d is invalid (null pointer, bad dtype, or out_features " \
                 "not a multiple of 8)", _i);

extern "C" size_t ml_lora_linear_workspace_bytes(int64_t tokens, int64_t in_features, int nproj,
                                                 const ml_lora_proj* proj, int backward) {
  if (tokens <= 0 || in_features <= 0 || proj == nullptr || nproj < 1 || nproj > 3) return 256;
  Arena ar;
  const int64_t r = 1;
  if (backward)
    lora::qkv_backward(nullptr, nullptr, tokens, in_features, r, nproj, proj, nullptr, nullptr,
                       nullptr, nullptr, ar, nullptr);
  else
    lora::qkv_forward(nullptr, tokens, in_features, r, nproj, proj, nullptr, nullptr, ar, nullptr);
  return std::max<size_t>(ar.off, 256);
}

extern "C" int ml_lora_linear_forward(const void* x, int64_t tokens, int64_t in_features,
                                      int64_t rank, int nproj, const ml_lora_proj* proj,
                                      void* const* out, void* u, void* workspace,
                                      size_t workspace_bytes, void* stream) {
  LORA_ARGCHECK_COMMON("lora_linear_forward", nproj)
  if (tokens == 0) return ML_OK;
  ML_CHECK_ARG(x && out && u, "lora_linear_forward: null pointer");
  for (int i = 0; i < nproj; ++i) ML_CHECK_ARG(out[i], "lora_linear_forward: null output %d", i);
  Arena need;
  lora::qkv_forward(nullptr, tokens, in_features, rank, nproj, proj, nullptr, nullptr, need,
                    nullptr);
  int rc = lora::check_ws(need, workspace_bytes, workspace, "lora_linear_forward");
  if (rc) return rc;
  Arena ar;
  ar.base = static_cast<uint8_t*>(workspace);
  ar.dry = false;
  return lora::qkv_forward(static_cast<const __nv_bfloat16*>(x), tokens, in_features, rank,
                           nproj, proj, out, static_cast<__nv_bfloat16*>(u), ar,
                           static_cast<cudaStream_t>(stream));
}

extern "C" int ml_lora_linear_backward(const void* x, const void* u, int64_t tokens,
                                       int64_t in_features, int64_t rank, int nproj,
                                       const ml_lora_proj* proj, const void* const* dy, void* dx,
                                       void* const* da, void* const* db, void* workspace,
                                       size_t workspace_bytes, void* stream) {
  LORA_ARGCHECK_COMMON("lora_linear_backward", nproj)
  ML_CHECK_ARG(dy && da && db, "lora_linear_backward: null pointer arrays");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (tokens == 0) {
    for (int i = 0; i < nproj; ++i) {
      ML_CHECK_CUDA(cudaMemsetAsync(da[i], 0, (size_t)rank * in_features * lora::esize(proj[i].a_dtype),
                                    st),
                    "memset dA");
      ML_CHECK_CUDA(cudaMemsetAsync(db[i], 0,
                                    (size_t)proj[i].out_features * rank * lora::esize(proj[i].b_dtype),
                                    st),
                    "memset dB");
    }
    return ML_OK;
  }
  ML_CHECK_ARG(x && u && dx, "lora_linear_backward: null pointer");
  for (int i = 0; i < nproj; ++i)
    ML_CHECK_ARG(dy[i] && da[i] && db[i], "lora_linear_backward: null pointer for projection %d",
                 i);
  Arena need;
  lora::qkv_backward(nullptr, nullptr, tokens, in_features, rank, nproj, proj, nullptr, nullptr,
                     nullptr, nullptr, need, nullptr);
  int rc = lora::check_ws(need, workspace_bytes, workspace, "lora_linear_backward");
  if (rc) return rc;
  Arena ar;
  ar.base = static_cast<uint8_t*>(workspace);
  ar.dry = false;
  return lora::qkv_backward(static_cast<const __nv_bfloat16*>(x),
                            static_cast<const __nv_bfloat16*>(u), tokens, in_features, rank,
                            nproj, proj, dy, static_cast<__nv_bfloat16*>(dx), da, db, ar, st);
}

extern "C" size_t ml_lora_qkv_workspace_bytes(int64_t tokens, int64_t in_features,
                                              const ml_lora_proj* proj, int backward) {
  return ml_lora_linear_workspace_bytes(tokens, in_features, 3, proj, backward);
}

extern "C" int ml_lora_qkv_forward(const void* x, int64_t tokens, int64_t in_features,
                                   int64_t rank, const ml_lora_proj* proj, void* const* out,
                                   void* u, void* workspace, size_t workspace_bytes,
                                   void* stream) {
  return ml_lora_linear_forward(x, tokens, in_features, rank, 3, proj, out, u, workspace,
                                workspace_bytes, stream);
}

extern "C" int ml_lora_qkv_backward(const void* x, const void* u, int64_t tokens,
                                    int64_t in_features, int64_t rank, const ml_lora_proj* proj,
                                    const void* const* dy, void* dx, void* const* da,
                                    void* const* db, void* workspace, size_t workspace_bytes,
                                    void* stream) {
  return ml_lora_linear_backward(x, u, tokens, in_features, rank, 3, proj, dy, dx, da, db,
                                 workspace, workspace_bytes, stream);
}

#define LORA_MLP_CHECK(what)                                                                   \
  ML_CHECK_ARG(tokens >= 0 && hidden > 0 && inter > 0 && rank > 0, what ": bad sizes");        \
  ML_CHECK_ARG(hidden % 8 == 0 && inter % 8 == 0, what ": sizes must be multiples of 8");      \
  ML_CHECK_ARG(2 * rank <= lora::kSlot, what ": rank %lld > 32 is not supported",              \
               (long long)rank);                                                                \
  ML_CHECK_ARG(proj != nullptr && lora::valid_proj(proj[0]) && lora::valid_proj(proj[1]) &&    \
                   lora::valid_proj(proj[2]),                                                  \
               what ": invalid projections");                                                  \
  ML_CHECK_ARG(proj[0].out_features == inter && proj[1].out_features == inter &&               \
                   proj[2].out_features == hidden,                                             \
               what ": projection shapes do not match hidden/intermediate");

extern "C" int ml_lora_set_mlp_swiglu_fusion(int enable, int* previous) {
  ML_CHECK_ARG(enable == 0 || enable == 1, "lora_set_mlp_swiglu_fusion: enable must be 0 or 1");
  const int old = lora::g_mlp_swiglu_fused.exchange(enable);
  if (previous) *previous = old;
  return ML_OK;
}

extern "C" size_t ml_lora_mlp_workspace_bytes(int64_t tokens, int64_t hidden, int64_t inter,
                                              int backward) {
  if (tokens <= 0 || hidden <= 0 || inter <= 0) return 256;
  Arena ar;
  ml_lora_proj dummy[3] = {};
  if (backward)
    lora::mlp_backward(nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, tokens, hidden,
                       inter, 1, dummy, nullptr, nullptr, nullptr, nullptr, ar, nullptr);
  else
    lora::mlp_forward(nullptr, tokens, hidden, inter, 1, dummy, nullptr, nullptr, nullptr,
                      nullptr, nullptr, nullptr, ar, nullptr);
  return std::max<size_t>(ar.off, 256);
}

extern "C" int ml_lora_mlp_forward(const void* x, int64_t tokens, int64_t hidden, int64_t inter,
                                   int64_t rank, const ml_lora_proj* proj, void* gate, void* up,
                                   void* h, void* out, void* u1, void* u2, void* workspace,
                                   size_t workspace_bytes, void* stream) {
  LORA_MLP_CHECK("lora_mlp_forward")
  if (tokens == 0) return ML_OK;
  ML_CHECK_ARG(x && gate && up && h && out && u1 && u2, "lora_mlp_forward: null pointer");
  Arena need;
  ml_lora_proj dummy[3] = {};
  lora::mlp_forward(nullptr, tokens, hidden, inter, 1, dummy, nullptr, nullptr, nullptr, nullptr,
                    nullptr, nullptr, need, nullptr);
  int rc = lora::check_ws(need, workspace_bytes, workspace, "lora_mlp_forward");
  if (rc) return rc;
  Arena ar;
  ar.base = static_cast<uint8_t*>(workspace);
  ar.dry = false;
  using b = __nv_bfloat16;
  return lora::mlp_forward(static_cast<const b*>(x), tokens, hidden, inter, rank, proj,
                           static_cast<b*>(gate), static_cast<b*>(up), static_cast<b*>(h),
                           static_cast<b*>(out), static_cast<b*>(u1), static_cast<b*>(u2), ar,
                           static_cast<cudaStream_t>(stream));
}

extern "C" int ml_lora_mlp_backward(const void* x, const void* gate, const void* up,
                                    const void* h, const void* u1, const void* u2, int64_t tokens,
                                    int64_t hidden, int64_t inter, int64_t rank,
                                    const ml_lora_proj* proj, const void* dy, void* dx,
                                    void* const* da, void* const* db, void* workspace,
                                    size_t workspace_bytes, void* stream) {
  LORA_MLP_CHECK("lora_mlp_backward")
  ML_CHECK_ARG(da && db, "lora_mlp_backward: null pointer arrays");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (tokens == 0) {
    const int64_t in_f[3] = {hidden, hidden, inter};
    for (int i = 0; i < 3; ++i) {
      ML_CHECK_CUDA(cudaMemsetAsync(da[i], 0, (size_t)rank * in_f[i] * lora::esize(proj[i].a_dtype),
                                    st),
                    "memset dA");
      ML_CHECK_CUDA(cudaMemsetAsync(db[i], 0,
                                    (size_t)proj[i].out_features * rank * lora::esize(proj[i].b_dtype),
                                    st),
                    "memset dB");
    }
    return ML_OK;
  }
  ML_CHECK_ARG(x && gate && up && h && u1 && u2 && dy && dx, "lora_mlp_backward: null pointer");
  Arena need;
  ml_lora_proj dummy[3] = {};
  lora::mlp_backward(nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, tokens, hidden, inter,
                     1, dummy, nullptr, nullptr, nullptr, nullptr, need, nullptr);
  int rc = lora::check_ws(need, workspace_bytes, workspace, "lora_mlp_backward");
  if (rc) return rc;
  Arena ar;
  ar.base = static_cast<uint8_t*>(workspace);
  ar.dry = false;
  using b = __nv_bfloat16;
  return lora::mlp_backward(static_cast<const b*>(x), static_cast<const b*>(gate),
                            static_cast<const b*>(up), static_cast<const b*>(h),
                            static_cast<const b*>(u1), static_cast<const b*>(u2), tokens, hidden,
                            inter, rank, proj, static_cast<const b*>(dy), static_cast<b*>(dx), da,
                            db, ar, st);
}
