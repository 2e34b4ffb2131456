/*
 * metal_liger_b200 — C ABI of the B200 (sm_100a) fused-op library.
 *
 * This is the drop-in boundary that replaces the reference's native layer:
 * the Objective-C++/Metal functions declared in csrc/metal_liger_ops.h and
 * bound by csrc/bindings.mm, plus the pure-ATen hot paths of ops/*.py that
 * never had a native kernel (RoPE, chunked fused linear cross-entropy, fused
 * LoRA).  Each entry point cites the reference interface it replaces.
 *
 * Conventions (all entry points):
 *   - pointers are DEVICE pointers owned by the caller (inputs borrowed,
 *     outputs written in place); nothing here allocates device memory unless
 *     the comment says so;
 *   - sizes are element counts; strides are in elements;
 *   - `stream` is a cudaStream_t passed as void* (NULL = legacy default
 *     stream); work is only enqueued, never synchronised;
 *   - the return value is ML_OK (0) or an ML_ERR_* code; the message of the
 *     last failure on the calling host thread is returned by ml_last_error().
 *     Argument errors are detected on the host before anything is enqueued.
 */
#ifndef METAL_LIGER_B200_H_
#define METAL_LIGER_B200_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define ML_API __attribute__((visibility("default")))
#else
#define ML_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* Element types accepted by the dtype arguments. */
enum {
  ML_DTYPE_F32 = 0,
  ML_DTYPE_BF16 = 1,
  ML_DTYPE_F16 = 2
};

/* Status codes. */
enum {
  ML_OK = 0,
  ML_ERR_INVALID_ARG = 1, /* bad shape / dtype / alignment / null pointer */
  ML_ERR_CUDA = 2,        /* a CUDA runtime call or kernel launch failed */
  ML_ERR_UNSUPPORTED = 3, /* valid request this build does not implement */
  ML_ERR_TIMEOUT = 4      /* a bounded device-side wait gave up */
};

/* Library version as 10000*major + 100*minor + patch. */
ML_API int ml_version(void);

/* Message describing the last failure on this host thread ("" if none). */
ML_API const char* ml_last_error(void);

/* ------------------------------------------------------------------------
 * RMSNorm
 * ------------------------------------------------------------------------ */

/*
 * y = (x * rsqrt(mean(x^2, -1) + eps) * weight).to(x dtype), computed in fp32,
 * and rrms[row] = rsqrt(mean(x^2) + eps) in fp32.
 * x, y: [rows, hidden] contiguous, dtype x_dtype; weight: [hidden], w_dtype.
 * rrms: [rows] fp32 (may be NULL when not needed).
 * Replaces metal_rms_norm_forward (reference csrc/metal_liger_ops.h:14-18,
 * csrc/rms_norm_metal.mm:110-160) and the math of
 * _FusedRMSNormFunction.forward (ops/fused_rms_norm.py:30-41).
 */
ML_API int ml_rms_norm_forward(const void* x, int x_dtype, const void* weight, int w_dtype,
                        void* y, float* rrms, int64_t rows, int64_t hidden, float eps,
                        void* stream);

/* Bytes of device scratch ml_rms_norm_backward needs for these sizes. */
ML_API size_t ml_rms_norm_backward_workspace_bytes(int64_t rows, int64_t hidden);

/*
 * dx = g*w*r - x*mean(g*w*x)*r^3 (per row, to x dtype) and
 * dweight = sum_rows(g * x * r) (to w dtype), all arithmetic in fp32, where
 * r = rrms[row] if rrms != NULL else rsqrt(mean(x^2)+eps) recomputed from x.
 * dy has x_dtype.  dweight is reduced deterministically in two stages
 * through `workspace` (>= ml_rms_norm_backward_workspace_bytes bytes, 16-byte
 * aligned); no [rows, hidden] per-row buffer is formed.
 * Replaces metal_rms_norm_backward (reference csrc/metal_liger_ops.h:20-25,
 * csrc/rms_norm_metal.mm:164-213) and _FusedRMSNormFunction.backward
 * (ops/fused_rms_norm.py:43-60).
 */
ML_API int ml_rms_norm_backward(const void* x, int x_dtype, const void* weight, int w_dtype,
                         const float* rrms, const void* dy, void* dx, void* dweight,
                         float eps, void* workspace, size_t workspace_bytes,
                         int64_t rows, int64_t hidden, void* stream);

/*
 * Process-wide override of the RMSNorm backward's row layout: every row is
 * split over threads holding nv 16-byte vectors each (1 = one vector per
 * thread, streamed through a shared-memory ring; 2, 4, 8 = register rows),
 * where the split fits a CTA; 0 (the default) uses the measured choice per
 * shape.  Results are identical up to the order of the row reduction.  The
 * previous setting is stored to *previous when non-NULL.  A tuning and test
 * knob with no reference counterpart.
 */
ML_API int ml_rms_norm_set_bwd_vectors(int nv, int* previous);

/*
 * Allocation-free ml_rms_norm_backward: same arguments and results, minus the
 * workspace.  It has no counterpart in the reference; it exists for callers
 * that cannot allocate device memory at call time -- hosts whose memory
 * planner owns all device memory after start-up (fixed arenas), and hot loops
 * that must not pay the implicit device synchronisation cudaMalloc/cudaFree
 * can cause.  The dweight partials live in a static device array of 4 MiB
 * (1,048,576 floats) that every GPU which loads this library keeps until the
 * process exits; hidden must be <= 1,048,576 (larger returns
 * ML_ERR_INVALID_ARG), rows are unlimited.  The first call on each device
 * looks up the array's device address with that device current; make that
 * first call before any stream capture.  All calls share the one array, so
 * calls whose work overlaps on the GPU (other streams, other host threads on
 * the same device) race and must be serialised by the caller.  Each call
 * writes every scratch element it reads, so nothing needs clearing between
 * calls.  Calls no cudaMalloc, cudaFree or other allocating routine.
 */
ML_API int ml_rms_norm_backward_noalloc(const void* x, int x_dtype, const void* weight,
                                        int w_dtype, const float* rrms, const void* dy, void* dx,
                                        void* dweight, float eps, int64_t rows, int64_t hidden,
                                        void* stream);

/* ------------------------------------------------------------------------
 * SwiGLU
 * ------------------------------------------------------------------------ */

/*
 * out = (silu(gate) * up).to(dtype), fp32 arithmetic; n elements, all three
 * buffers contiguous with the same dtype.
 * Replaces metal_swiglu_forward (reference csrc/metal_liger_ops.h:28-31,
 * csrc/swiglu_metal.mm:66-105) and _FusedSwiGLUFunction.forward
 * (ops/fused_swiglu.py:26-35).
 */
ML_API int ml_swiglu_forward(const void* gate, const void* up, void* out, int64_t n, int dtype,
                      void* stream);

/*
 * dgate = dout*up*s*(1 + gate*(1-s)), dup = dout*gate*s with s = sigmoid(gate)
 * recomputed in fp32 (nothing beyond gate/up is saved by the forward).
 * Replaces metal_swiglu_backward (reference csrc/metal_liger_ops.h:33-36,
 * csrc/swiglu_metal.mm:109-143) and _FusedSwiGLUFunction.backward
 * (ops/fused_swiglu.py:37-50).
 */
ML_API int ml_swiglu_backward(const void* gate, const void* up, const void* dout, void* dgate,
                       void* dup, int64_t n, int dtype, void* stream);

/* ------------------------------------------------------------------------
 * RoPE (rotate-half convention)
 * ------------------------------------------------------------------------ */

/* One [batch, heads, seq, head_dim] view to rotate (strides in elements; the
 * head_dim stride must be 1, the others are free, e.g. a transpose view). */
typedef struct ml_rope_tensor {
  const void* in;
  void* out;
  int64_t heads;
  int64_t in_strides[4];  /* batch, head, seq, dim */
  int64_t out_strides[4]; /* batch, head, seq, dim */
} ml_rope_tensor;

/*
 * out = in*cos + rotate_half(in)*(sin_sign*sin) for q and (optionally) k in
 * one launch; rotate_half([a, b]) = [-b, a].  sin_sign = +1 is the forward
 * rotation, -1 the reference's backward (inverse) rotation.
 * Angles come from one of two sources:
 *   table mode  (cos != NULL): cos/sin element (b, s, d) is read at
 *     b*cs_strides[0] + s*cs_strides[1] + d*cs_strides[2] (use stride 0 to
 *     broadcast, e.g. a [seq, head_dim] table), dtype cs_dtype;
 *   recompute mode (cos == NULL): angle = float(pos) * inv_freq[d mod D/2],
 *     pos = positions[b*pos_stride_batch + s] (or s when positions == NULL),
 *     cos/sin evaluated in fp32 in-kernel and multiplied by `scaling`.
 * in_dtype / out_dtype may differ (torch type promotion of the reference's
 * x*cos expression).  All arithmetic is fp32.
 * Replaces _FusedRoPEFunction.forward/backward and _apply_rotary_fused
 * (reference ops/fused_rope.py:22-57, :67-75) and apply_fused_rotary
 * (ops/fused_rope.py:110-127); the reference has no native RoPE.
 */
ML_API int ml_rope(const ml_rope_tensor* q, const ml_rope_tensor* k, int in_dtype, int out_dtype,
            int64_t batch, int64_t seq, int64_t head_dim,
            const void* cos, const void* sin, int cs_dtype, const int64_t* cs_strides,
            const int64_t* positions, int64_t pos_stride_batch, const float* inv_freq,
            float scaling, int sin_sign, void* stream);


/* ------------------------------------------------------------------------
 * Dense bf16 GEMM on the tcgen05 tensor cores (the building block of the
 * FLCE and LoRA paths; the reference uses ATen matmul/addmm there,
 * ops/fused_lora.py:69-82,142-165 and ops/fused_linear_cross_entropy.py:44,78-79)
 * ------------------------------------------------------------------------ */

/* A row-major bf16 operand.  For A (logical [M, K]): mn_major = 0 means it is
 * stored as [M, K] (K contiguous), 1 means stored as [K, M].  For B (logical
 * [N, K]): 0 = stored [N, K], 1 = stored [K, N].  ld = row pitch in elements
 * (multiple of 8); ptr must be 16-byte aligned. */
typedef struct ml_gemm_operand {
  const void* ptr;
  int64_t ld;
  int mn_major;
} ml_gemm_operand;

/* One K-segment: the segments' products are summed into one accumulator. */
typedef struct ml_gemm_segment {
  ml_gemm_operand a;
  ml_gemm_operand b;
  int64_t k;
} ml_gemm_segment;

/* Scratch bytes ml_gemm_bf16 can use for split-K partials (0 = none needed). */
ML_API size_t ml_gemm_bf16_workspace_bytes(int64_t m, int64_t n, int64_t k_total);

/*
 * D[m, n] = alpha * sum_s A_s[m, k_s] * B_s[n, k_s]^T  (+ D if beta == 1),
 * bf16 operands, fp32 accumulation, D fp32 or bf16 (beta = 1 needs fp32 D)
 * with row pitch ldd.  1 <= nseg <= 4; all segments share operand majorness.
 * Uses split-K (deterministic, fixed-order reduction) when the workspace
 * allows and the tile count is small.
 */
ML_API int ml_gemm_bf16(int64_t m, int64_t n, const ml_gemm_segment* segs, int nseg, void* d,
                        int d_dtype, int64_t ldd, float alpha, float beta, void* workspace,
                        size_t workspace_bytes, void* stream);

/*
 * Process-wide choice of GEMM kernel: -1 = automatic (default: the 2-SM
 * CTA-pair kernel (tcgen05 cta_group::2, 256 rows x 256 or 128 columns per
 * pair) or the 1-SM kernel, whichever fills the SMs best for the shape),
 * 0 = 1-SM kernel only, 1 = CTA pair whenever the shape allows, 2 / 3 = CTA
 * pair with 256- / 128-wide tiles only.  Applies to every GEMM in this
 * library (plain, FLCE, LoRA).  The previous mode is stored to *previous
 * when non-NULL.  A tuning and test knob with no reference counterpart.
 */
ML_API int ml_gemm_set_cta_pair(int mode, int* previous);

/*
 * Process-wide number of SMs (0-128) every GEMM of this library leaves free
 * while it is set: the persistent GEMM grid then stops short of the whole
 * GPU, so a kernel on another stream (an NCCL collective the GEMM is meant
 * to overlap) can be scheduled next to it instead of after it.  Read at
 * launch time; 0 (the default) uses every SM.  The previous value is stored
 * to *previous when non-NULL.  No reference counterpart (the reference is
 * single-device).
 */
ML_API int ml_gemm_set_reserved_sms(int n, int* previous);

/* ------------------------------------------------------------------------
 * Fused linear cross-entropy
 * ------------------------------------------------------------------------ */

/* Number of fp32 [n, h] slabs ml_flce_forward writes for dhidden (split-K). */
ML_API int ml_flce_dx_slabs(int64_t n, int64_t h, int64_t v, int64_t chunk_tokens);

/* Device scratch bytes ml_flce_forward needs (256-byte aligned buffer). */
ML_API size_t ml_flce_workspace_bytes(int64_t n, int64_t h, int64_t v, int64_t chunk_tokens);

/*
 * Mean cross-entropy of logits = hidden @ weight^T (+ bias) over rows whose
 * label != ignore_index, without materialising the [n, v] logits:
 *   loss[0] = sum_r (lse_r - logit_r[label_r]) / max(#valid, 1)
 * hidden [n, h] and weight [v, h] are bf16 row-major (h a multiple of 8);
 * bias [v] (optional, bias_dtype) gets no gradient; labels int64 [n].
 * When dx_slabs / dw_acc are non-NULL the gradients for grad_output = 1 are
 * produced in the same pass (each logit is computed once):
 *   dx_slabs: ml_flce_dx_slabs(...) fp32 slabs of [n, h] that sum to dhidden;
 *   dw_acc:   fp32 [v, h] dweight.
 * lse (optional) receives the per-row log-sum-exp.  Tokens are processed in
 * chunks of chunk_tokens rows (<= 0: all rows); the result does not depend
 * on it.  workspace: >= ml_flce_workspace_bytes(...), 256-byte aligned.
 * Replaces _FusedLinearCrossEntropyFunction.forward/backward
 * (reference ops/fused_linear_cross_entropy.py:39-185), which has no native
 * kernel in the reference.
 */
ML_API int ml_flce_forward(const void* hidden, const void* weight, const void* bias,
                           int bias_dtype, const int64_t* labels, int64_t n, int64_t h, int64_t v,
                           int64_t ignore_index, int64_t chunk_tokens, float* loss, float* lse,
                           float* dx_slabs, float* dw_acc, void* workspace,
                           size_t workspace_bytes, void* stream);

/*
 * Backward of ml_flce_forward: dhidden = grad_output[0] * sum(dx_slabs) cast to
 * dh_dtype, dweight = grad_output[0] * dw_acc cast to dw_dtype (either output
 * may be NULL).  grad_output is a device fp32 scalar.
 */
ML_API int ml_flce_backward(const float* grad_output, const float* dx_slabs, int slabs,
                            void* dhidden, int dh_dtype, int64_t n, int64_t h,
                            const float* dw_acc, void* dweight, int dw_dtype, int64_t v,
                            void* stream);

/* --- vocabulary-parallel FLCE (weight sharded by vocabulary rows) -------- */

/* out[0] = #(labels != ignore_index), out[1] = 1 / max(out[0], 1) (fp32, device). */
ML_API int ml_flce_count_valid(const int64_t* labels, int64_t n, int64_t ignore_index, float* out,
                               void* stream);

/* Workspace bytes shared by ml_flce_shard_stats / _grads for one token chunk. */
ML_API size_t ml_flce_shard_workspace_bytes(int64_t rows, int64_t v_local);

/*
 * Phase 1 for one token chunk on one vocabulary shard (weight rows
 * [vocab_offset, vocab_offset + v_local) of the full lm_head): per row the
 * shard's logit max, sum exp(logit - max) and the target logit (0 when the
 * label lies outside the shard).  The shard's exp(logit - tile max) values
 * stay in `workspace` for phase 2.  The caller merges the three [rows]
 * vectors across ranks (max, then rescaled sum; target by sum) into the
 * global log-sum-exp.  Same math as _chunked_forward_pass
 * (reference ops/fused_linear_cross_entropy.py:39-55), split by vocabulary.
 */
ML_API int ml_flce_shard_stats(const void* hidden, const void* weight, const void* bias,
                               int bias_dtype, const int64_t* labels, int64_t rows, int64_t h,
                               int64_t v_local, int64_t vocab_offset, int64_t ignore_index,
                               float* row_max, float* row_sum, float* row_tgt, void* workspace,
                               size_t workspace_bytes, void* stream);

/*
 * Phase 2: with the GLOBAL per-row log-sum-exp `lse` and `scale` (device
 * scalar, 1/max(#valid,1)), form this shard's (softmax - onehot) * scale and
 * write dx [rows, h] fp32 (this shard's partial dhidden, to be summed across
 * ranks) and dw [v_local, h] fp32 (this shard's dweight; accumulated when
 * dw_accumulate != 0).  Either output may be NULL.  Same math as
 * _chunked_backward_pass (reference ops/fused_linear_cross_entropy.py:57-80).
 */
ML_API int ml_flce_shard_grads(const void* hidden, const void* weight, const int64_t* labels,
                               int64_t rows, int64_t h, int64_t v_local, int64_t vocab_offset,
                               int64_t ignore_index, const float* lse, const float* scale,
                               float* dx, float* dw, int dw_accumulate, void* workspace,
                               size_t workspace_bytes, void* stream);

/*
 * Phase 2 split in two: after ml_flce_shard_grads ran with dw == NULL (it
 * leaves the (softmax - onehot) * scale chunk in `workspace`), this runs the
 * shard's dW GEMM alone, so a caller can start the all-reduce of dx before
 * it and overlap the two.  Same arguments and layout as above.
 */
ML_API int ml_flce_shard_grads_dw(const void* hidden, int64_t rows, int64_t h, int64_t v_local,
                                  float* dw, int dw_accumulate, void* workspace,
                                  size_t workspace_bytes, void* stream);

/* --- peer memory between the node's GPUs (one process per GPU) ----------
 * A device buffer from ml_p2p_alloc (cudaMalloc'd, zeroed) is exported as an
 * opaque handle of ml_p2p_handle_bytes() bytes, passed to the other ranks by
 * the caller (the process group), and mapped there with ml_p2p_import
 * (peer access enabled on demand); ml_p2p_close unmaps, ml_p2p_free frees. */
ML_API int ml_p2p_alloc(size_t bytes, void** out);
ML_API int ml_p2p_free(void* ptr);
ML_API size_t ml_p2p_handle_bytes(void);
ML_API int ml_p2p_export(const void* base, void* handle_out);
ML_API int ml_p2p_import(const void* handle, void** out);
ML_API int ml_p2p_close(void* ptr);

/*
 * The vocabulary-parallel dX without a collective library: every rank keeps
 * an exchange buffer of ml_flce_p2p_workspace_bytes(world, chunk_cap, h)
 * bytes (ml_p2p_alloc) mapped on every other rank; `peer_ws` lists the
 * world buffers as mapped on this GPU (own included), indexed by rank.
 * Rank r owns the chunk's rows [r R, r R + R), R = ceil(chunk_cap / world)
 * rounded up to a multiple of 256.  Per chunk, with an epoch that starts at
 * 1 and grows by one per chunk, identical on every rank:
 *   ml_flce_shard_dx_p2p  after ml_flce_shard_grads(dx = dw = NULL) on the
 *                         same shard workspace: the shard's dX GEMM, whose
 *                         epilogue stores each fp32 tile into its row owner's
 *                         receive slot for this rank (plain stores into peer
 *                         memory, overlapping the math), then an arrive flag
 *                         on every rank;
 *   ml_flce_p2p_reduce    waits for every rank's arrive flag, sums this
 *                         rank's rows over the ranks in rank order and writes
 *                         them into every rank's gather buffer, then a done
 *                         flag on every rank;
 *   ml_flce_p2p_finish    waits for every owner's done flag and copies the
 *                         chunk's summed dX (rows x h fp32) to dx_out.
 * Waits are bounded (2 s): one that gives up records ML_ERR_TIMEOUT in the
 * device error word (ml_device_error).  Replaces the NCCL all-reduce of the
 * shard's partial dX; the result is bit for bit independent of the ranks'
 * timing (fixed summation order).  world <= 8, h a multiple of 8.
 */
ML_API size_t ml_flce_p2p_workspace_bytes(int world, int64_t chunk_cap, int64_t h);
ML_API int ml_flce_shard_dx_p2p(const void* weight, int64_t rows, int64_t h, int64_t v_local,
                                const void* shard_ws, size_t shard_ws_bytes, int64_t chunk_cap,
                                int world, int rank, void* const* peer_ws, int64_t epoch,
                                void* stream);
ML_API int ml_flce_p2p_reduce(int64_t rows, int64_t h, int64_t chunk_cap, int world, int rank,
                              void* const* peer_ws, int64_t epoch, void* stream);
ML_API int ml_flce_p2p_finish(int64_t rows, int64_t h, int64_t chunk_cap, int world, int rank,
                              void* const* peer_ws, int64_t epoch, float* dx_out, void* stream);

/*
 * The chunk's softmax statistics through the same buffers (replacing the two
 * all-reduces of ml_flce_shard_stats' outputs), same epoch as the chunk's dX:
 *   ml_flce_p2p_stats_put    this rank's [rows] max / sum-exp / target logit
 *                            into its slot on every rank, then a stats flag;
 *   ml_flce_p2p_stats_merge  waits for every rank's flag and writes, per row,
 *                            max = max_r max_r, sum = sum_r sum_r exp(max_r -
 *                            max), target = sum_r target_r, over the ranks in
 *                            rank order (identical on every rank).
 */
ML_API int ml_flce_p2p_stats_put(const float* row_max, const float* row_sum,
                                 const float* row_tgt, int64_t rows, int64_t h,
                                 int64_t chunk_cap, int world, int rank, void* const* peer_ws,
                                 int64_t epoch, void* stream);
ML_API int ml_flce_p2p_stats_merge(int64_t rows, int64_t h, int64_t chunk_cap, int world,
                                   int rank, void* const* peer_ws, int64_t epoch, float* out_max,
                                   float* out_sum, float* out_tgt, void* stream);

/* ------------------------------------------------------------------------
 * Fused LoRA QKV / MLP
 * ------------------------------------------------------------------------ */

/* One LoRA-adapted projection y = x W^T + scaling * (x A^T) B^T. */
typedef struct ml_lora_proj {
  const void* w;         /* frozen base weight [out_features, in_features], bf16 */
  const void* a;         /* lora_A [rank, in_features], dtype a_dtype */
  const void* b;         /* lora_B [out_features, rank], dtype b_dtype */
  int a_dtype;
  int b_dtype;
  int64_t out_features;
  float scaling;
} ml_lora_proj;

/* Workspace bytes (256-byte aligned buffer) for ml_lora_qkv_forward
 * (backward = 0) or ml_lora_qkv_backward (backward = 1). */
ML_API size_t ml_lora_qkv_workspace_bytes(int64_t tokens, int64_t in_features,
                                          const ml_lora_proj* proj, int backward);

/*
 * Q, K, V for proj[0..2] sharing one input x [tokens, in_features] (bf16):
 * out[i] [tokens, out_i] bf16.  Also writes u [tokens, 64] bf16, the stacked
 * x A_i^T (adapter i in columns [i*rank, (i+1)*rank)) that the backward
 * reuses.  rank <= 21.  Replaces _LoRA_QKV.forward (reference
 * ops/fused_lora.py:96-119) and _lora_linear (:69-82).
 */
ML_API int ml_lora_qkv_forward(const void* x, int64_t tokens, int64_t in_features, int64_t rank,
                               const ml_lora_proj* proj, void* const* out, void* u,
                               void* workspace, size_t workspace_bytes, void* stream);

/*
 * Backward of ml_lora_qkv_forward for upstream dy[0..2] (bf16): dx [tokens,
 * in] bf16 = sum_i dy_i W_i + s_i (dy_i B_i) A_i (one GEMM), and per adapter
 * da[i] [rank, in] = s_i (dy_i B_i)^T x, db[i] [out_i, rank] = s_i dy_i^T u_i,
 * accumulated in fp32 and written in the adapter's own dtype (proj[i].a_dtype
 * / b_dtype) — the value autograd gives the parameter after the reference's
 * fp32 `.float()` result.  W gets no gradient.  Replaces _LoRA_QKV.backward
 * (reference ops/fused_lora.py:121-171).
 */
ML_API int ml_lora_qkv_backward(const void* x, const void* u, int64_t tokens, int64_t in_features,
                                int64_t rank, const ml_lora_proj* proj, const void* const* dy,
                                void* dx, void* const* da, void* const* db, void* workspace,
                                size_t workspace_bytes, void* stream);

/*
 * The same pair for 1 to 3 LoRA projections of one input (nproj * rank <= 64):
 * ml_lora_qkv_* are these with nproj = 3.  nproj = 1 is a single fused LoRA
 * linear (o_proj): y = x W^T + s (x A^T) B^T with the rank term folded into
 * the base GEMM, and dx / dA / dB as above.  The reference describes this
 * single-projection form ("LoRA_W", ops/fused_lora.py:26) and falls back to
 * PEFT's unfused modules (ops/fused_lora.py:69-82) for it.
 */
ML_API size_t ml_lora_linear_workspace_bytes(int64_t tokens, int64_t in_features, int nproj,
                                             const ml_lora_proj* proj, int backward);
ML_API int ml_lora_linear_forward(const void* x, int64_t tokens, int64_t in_features,
                                  int64_t rank, int nproj, const ml_lora_proj* proj,
                                  void* const* out, void* u, void* workspace,
                                  size_t workspace_bytes, void* stream);
ML_API int ml_lora_linear_backward(const void* x, const void* u, int64_t tokens,
                                   int64_t in_features, int64_t rank, int nproj,
                                   const ml_lora_proj* proj, const void* const* dy, void* dx,
                                   void* const* da, void* const* db, void* workspace,
                                   size_t workspace_bytes, void* stream);

/*
 * Process-wide choice for the MLP entry points below: 1 (default) applies the
 * SwiGLU inside the GEMMs — the forward's gate and up projections run as one
 * GEMM whose epilogue also writes h = silu(gate) * up, and the backward's dH
 * GEMM writes d_gate / d_up directly (dH is never stored); 0 runs the
 * projections and the SwiGLU as separate passes.  Results are bitwise the
 * same; the backward workspace is smaller with 1 (no dH buffer), so query
 * ml_lora_mlp_workspace_bytes after setting it.  The previous setting is
 * stored to *previous when non-NULL.  A tuning and test knob with no
 * reference counterpart (the reference computes the SwiGLU between its
 * matmuls, ops/fused_lora.py:195-197, :235-244).
 */
ML_API int ml_lora_set_mlp_swiglu_fusion(int enable, int* previous);

/* Workspace bytes for the MLP entry points (backward = 0 or 1). */
ML_API size_t ml_lora_mlp_workspace_bytes(int64_t tokens, int64_t hidden, int64_t inter,
                                          int backward);

/*
 * LoRA SwiGLU MLP, proj = {gate [inter x hidden], up [inter x hidden],
 * down [hidden x inter]}: gate, up [tokens, inter]; h = silu(gate) * up (fp32
 * math, bf16 out); out [tokens, hidden] = down(h).  u1 / u2 [tokens, 64]
 * receive x [Ag;Au]^T and h Ad^T for the backward.  rank <= 32.  Replaces
 * _LoRA_MLP.forward (reference ops/fused_lora.py:182-207).
 */
ML_API int ml_lora_mlp_forward(const void* x, int64_t tokens, int64_t hidden, int64_t inter,
                               int64_t rank, const ml_lora_proj* proj, void* gate, void* up,
                               void* h, void* out, void* u1, void* u2, void* workspace,
                               size_t workspace_bytes, void* stream);

/*
 * Backward of ml_lora_mlp_forward: dx [tokens, hidden] bf16 and da[i]
 * [rank, in_i], db[i] [out_i, rank] for gate, up, down (fp32 accumulation,
 * written in each adapter's dtype as above).  Replaces _LoRA_MLP.backward
 * (reference ops/fused_lora.py:209-266).
 */
ML_API int ml_lora_mlp_backward(const void* x, const void* gate, const void* up, const void* h,
                                const void* u1, const void* u2, int64_t tokens, int64_t hidden,
                                int64_t inter, int64_t rank, const ml_lora_proj* proj,
                                const void* dy, void* dx, void* const* da, void* const* db,
                                void* workspace, size_t workspace_bytes, void* stream);

/*
 * Greedy decoding head: index[b] = argmax over v < vocab of the logit
 * round_to(logit_dtype, sum_k hidden[b, k] * weight[v, k] (+ bias[v])), the
 * products accumulated in fp32 on the tcgen05 GEMM core and never stored;
 * value[b] (optional) = that logit.  Ties and NaN follow torch.argmax (NaN
 * first, then the lowest index).  hidden [batch, hidden_size] and weight
 * [vocab, hidden_size] are bf16 with row pitches ld_hidden / ld_weight
 * (elements, multiples of 8; 16-byte aligned bases); logit_dtype is the
 * dtype the model's logits have (ML_DTYPE_BF16 for a bf16 lm_head); bias is
 * optional ([vocab], bias_dtype).  workspace >=
 * ml_lm_head_argmax_workspace_bytes(batch, vocab), 16-byte aligned.
 * Replaces the reference's greedy step of MetalLigerGenerator.generate,
 * logits = model(...).logits[:, -1, :]; argmax(logits, -1)
 * (generation.py:99-101,118-122), without the [batch, vocab] logits.
 */
ML_API size_t ml_lm_head_argmax_workspace_bytes(int64_t batch, int64_t vocab);
ML_API int ml_lm_head_argmax(const void* hidden, int64_t ld_hidden, const void* weight,
                             int64_t ld_weight, const void* bias, int bias_dtype, int64_t batch,
                             int64_t hidden_size, int64_t vocab, int logit_dtype, int64_t* index,
                             float* value, void* workspace, size_t workspace_bytes,
                             void* stream);

/*
 * Decode-time linear layer: y[b, n] = sum_k x[b, k] * weight[n, k] (+ bias[n])
 * for batch = 1 or 2 activation rows (bf16, pitch ld_x), weight [N, K] bf16
 * (pitch ld_w), fp32 accumulation, y (pitch ld_y) in y_dtype (ML_DTYPE_BF16
 * or ML_DTYPE_F32).  K and the pitches are multiples of 8, bases 16-byte
 * aligned, batch * K * 2 <= 96 KiB.  An HBM-streaming kernel (one pass over
 * the weight) for the generator's decode steps; no reference counterpart
 * (the reference's decode runs the model's nn.Linear modules,
 * generation.py:109-115).
 */
ML_API int ml_gemv_bf16(const void* x, int64_t ld_x, const void* weight, int64_t ld_w,
                        const void* bias, int bias_dtype, int64_t batch, int64_t K, int64_t N,
                        void* y, int y_dtype, int64_t ld_y, void* stream);

/*
 * ml_gemv_bf16 for nmat (1-4) projections of the same activations in one
 * launch (q, k and v of an attention block): for each i, y[i][b, n] =
 * sum_k x[b, k] * weight[i][n, k] (+ bias[i][n]) for n < n[i], output pitch
 * ld_y[i]; bias is NULL or an array of nmat pointers (entries may be NULL).
 * The layout rules of ml_gemv_bf16 hold for every matrix.
 */
ML_API int ml_gemv_multi_bf16(const void* x, int64_t ld_x, int nmat, const void* const* weight,
                              const int64_t* ld_w, const int64_t* n, const void* const* bias,
                              int bias_dtype, int64_t batch, int64_t K, void* const* y,
                              const int64_t* ld_y, int y_dtype, void* stream);

/*
 * Decode-step attention (no reference counterpart; the reference's decode
 * runs the model's attention over its growing cache, generation.py:109-115):
 * out[b, 0, h, :] = sum_{j < n} softmax_j(scale * q[b, h] . k[b, h / G, j])
 * v[b, h / G, j] with n = min(max_len, *pos + len_offset) read from device
 * memory, G = q_heads / kv_heads (<= 16).  q is [B, q_heads, 1, head_dim] at
 * element strides (sq_b, sq_h), head_dim contiguous; k_cache / v_cache
 * [B, kv_heads, max_len, head_dim] contiguous bf16; out [B, 1, q_heads,
 * head_dim] bf16; head_dim a multiple of 32 up to 256; fp32 scores and
 * accumulation; workspace >= ml_decode_attention_workspace_bytes, which is 0
 * for caches of at most 256 positions (one launch, the partials in shared
 * memory: workspace may then be NULL).
 */
ML_API size_t ml_decode_attention_workspace_bytes(int64_t batch, int64_t q_heads,
                                                  int64_t max_len, int64_t head_dim);
ML_API int ml_decode_attention_bf16(const void* q, int64_t sq_b, int64_t sq_h,
                                    const void* k_cache, const void* v_cache,
                                    const int64_t* pos, int64_t len_offset, int64_t batch,
                                    int64_t q_heads, int64_t kv_heads, int64_t max_len,
                                    int64_t head_dim, float scale, void* out, void* workspace,
                                    size_t workspace_bytes, void* stream);

/*
 * Decode-step q/k preparation for Qwen3-style attention (no reference
 * counterpart; it replaces, for the single new token, the per-head q_norm /
 * k_norm RMSNorms, RoPE and the two cache writes): q [B, q_heads * D] and
 * k [B, kv_heads * D] rows get RMSNorm with weights wq / wk (eps_q / eps_k;
 * y = bf16((x * rrms) * w)) and RoPE with the model's cos / sin ([B, D] at
 * batch stride cs_b, dtype cs_dtype; rotate-half, fp32, one rounding); q goes
 * to q_out [B, q_heads, D], k to k_cache [B, kv_heads, max_len, D] at position
 * *pos (device) and v [B, kv_heads * D] unchanged to v_cache at *pos.
 * head_dim is 64, 128 or 256; q, k, v, caches and q_out bf16.
 */
ML_API int ml_decode_qk_norm_rope_bf16(
    const void* q, const void* k, const void* v, const void* wq, const void* wk, int w_dtype,
    float eps_q, float eps_k, const void* cos, const void* sin, int cs_dtype, int64_t cs_b,
    int64_t batch, int64_t q_heads, int64_t kv_heads, int64_t max_len, int64_t head_dim,
    void* q_out, void* k_cache, void* v_cache, const int64_t* pos, void* stream);

/*
 * ml_decode_qk_norm_rope_bf16 followed by ml_decode_attention_bf16 (len_offset
 * 1: the new token's position is attended to) in one launch, bit for bit the
 * two calls, for caches of at most 256 positions (max_len <= 256) and the
 * head shapes ml_decode_attention_bf16 builds; q stays on chip (no q_out), k
 * and v go to the caches at *pos, out [B, 1, q_heads, head_dim] bf16.  No
 * workspace.  No reference counterpart (the reference's decode runs the
 * block's norms, RoPE, cache update and attention module by module,
 * generation.py:109-115).
 */
ML_API int ml_decode_qk_attention_bf16(
    const void* q, const void* k, const void* v, const void* wq, const void* wk, int w_dtype,
    float eps_q, float eps_k, const void* cos, const void* sin, int cs_dtype, int64_t cs_b,
    int64_t batch, int64_t q_heads, int64_t kv_heads, int64_t max_len, int64_t head_dim,
    void* k_cache, void* v_cache, const int64_t* pos, float scale, void* out, void* stream);

/*
 * Decode-time SwiGLU MLP input side: y[b, i] = bf16(silu(g) * u) with
 * g = bf16(x[b] . w_gate[i]), u = bf16(x[b] . w_up[i]) (fp32 accumulation;
 * bitwise equal to two ml_gemv_bf16 calls and ml_swiglu_forward), for
 * batch = 1 or 2; w_gate / w_up [inter, K] bf16; the same layout rules as
 * ml_gemv_bf16.  One pass over both weights, gate and up never stored.  No
 * reference counterpart (the reference's decode runs gate_proj, up_proj and
 * the activation separately, ops/fused_swiglu.py:71-75).
 */
ML_API int ml_gemv_swiglu_bf16(const void* x, int64_t ld_x, const void* w_gate, int64_t ld_g,
                               const void* w_up, int64_t ld_u, int64_t batch, int64_t K,
                               int64_t inter, void* y, int64_t ld_y, void* stream);

/*
 * The decoder layer's decode step fused around the GEMVs (no reference
 * counterpart; the reference's decode runs the layer's modules one by one,
 * generation.py:109-115, through transformers' decoder layer: input norm,
 * attention, residual add, post-attention norm, MLP, residual add).
 *
 * ml_gemv_residual_bf16: y[b, n] = bf16(bf16(x[b] . weight[n] (+ bias[n])) +
 * residual[b, n]) — ml_gemv_bf16 followed by the bf16 residual add, bit for
 * bit; residual [batch, N] bf16 at pitch ld_r (NULL: plain bf16 GEMV), not
 * overlapping y; y bf16.
 *
 * ml_gemv_rmsnorm_multi_bf16 / ml_gemv_rmsnorm_swiglu_bf16: ml_gemv_multi_bf16
 * / ml_gemv_swiglu_bf16 of the RMSNorm'd activations bf16((x * rrms) * w),
 * norm_weight [K] bf16 (16-byte aligned), bitwise equal to
 * ml_rms_norm_forward (bf16 x and weight, 16-byte aligned rows) followed by
 * the GEMV; K a multiple of 8 up to 16,384 (the RMSNorm kernel's vector row
 * layouts).
 */
ML_API int ml_gemv_residual_bf16(const void* x, int64_t ld_x, const void* weight, int64_t ld_w,
                                 const void* bias, int bias_dtype, const void* residual,
                                 int64_t ld_r, int64_t batch, int64_t K, int64_t N, void* y,
                                 int64_t ld_y, void* stream);
ML_API int ml_gemv_rmsnorm_multi_bf16(const void* x, int64_t ld_x, const void* norm_weight,
                                      float eps, int nmat, const void* const* weight,
                                      const int64_t* ld_w, const int64_t* n,
                                      const void* const* bias, int bias_dtype, int64_t batch,
                                      int64_t K, void* const* y, const int64_t* ld_y,
                                      int y_dtype, void* stream);
ML_API int ml_gemv_rmsnorm_swiglu_bf16(const void* x, int64_t ld_x, const void* norm_weight,
                                       float eps, const void* w_gate, int64_t ld_g,
                                       const void* w_up, int64_t ld_u, int64_t batch, int64_t K,
                                       int64_t inter, void* y, int64_t ld_y, void* stream);

/*
 * Self-test of the bounded device-side waits (no reference counterpart):
 * enqueues on `stream` a one-warp kernel whose mbarrier wait can never
 * complete, bounded to limit_us (1,000 - 1,000,000 us); the wait gives up and
 * records (6 << 8) | ML_ERR_TIMEOUT in the device error word, which
 * ml_device_error then returns.  Nothing faults, traps or hangs.
 */
ML_API int ml_selftest_bounded_wait(int64_t limit_us, void* stream);

/* Synchronises `stream`, then returns and clears the device error word set
 * by a bounded wait inside a tcgen05 kernel that gave up ((site << 8) |
 * ML_ERR_TIMEOUT), or 0.  A negative-free ML_ERR_CUDA is returned if the
 * synchronisation itself fails. */
ML_API int ml_device_error(void* stream);

#ifdef __cplusplus
}  /* extern "C" */
#endif

#endif  /* METAL_LIGER_B200_H_ */
