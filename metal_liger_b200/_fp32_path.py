"""fp32-accurate mode of the GEMM-based ops (LoRA, FLCE) for fp32 inputs.

The tcgen05 GEMM multiplies bf16 operands.  For fp32 inputs each operand is
split into three bf16 parts that together carry its 24-bit significand,

    a = a_hi + a_mid + a_lo,   a_hi = bf16(a), a_mid = bf16(a - a_hi),
                               a_lo = bf16(a - a_hi - a_mid),

and a b is taken as the six products down to order 2^-16 relative (hi.hi,
hi.mid, mid.hi, hi.lo, lo.hi, mid.mid; the dropped ones are ~2^-24), in two
ml_gemm_bf16 launches of three K-segments on one fp32 accumulator.  fp32
inputs thus get fp32-level products — the reference computes these ops in the
input dtype, and its own LoRA test checks fp32 results at atol 1e-4 /
rtol 1e-3 (tests/test_fused_ops.py:233-241).
Every GEMM is this library's; the few elementwise steps between them
(row log-sum-exp, softmax rows, sums) are torch CUDA ops.  bf16 inputs never
come here: they take the fused single-pass kernels.
"""

from __future__ import annotations

import torch
from torch import Tensor

from metal_liger_b200 import _C

F32 = torch.float32
BF16 = torch.bfloat16


def _pitched(t: Tensor) -> Tensor:
    """2-D bf16 view whose row pitch is a multiple of 8 elements and whose data
    pointer is 16-byte aligned (TMA rules); copies only when needed."""
    if t.stride(1) == 1 and t.stride(0) % 8 == 0 and t.data_ptr() % 16 == 0:
        return t
    r, c = t.shape
    buf = torch.zeros(r, (c + 7) // 8 * 8, dtype=t.dtype, device=t.device)
    buf[:, :c] = t
    return buf[:, :c]


def _split3(t: Tensor):
    hi = t.to(BF16)
    r1 = t - hi.to(F32)
    mid = r1.to(BF16)
    lo = (r1 - mid.to(F32)).to(BF16)
    return _pitched(hi), _pitched(mid), _pitched(lo)


def _gemm3(pairs, M, N, K, a_mn, b_mn, out, beta, stream):
    lib = _C.load()
    segs = (_C.GemmSegment * 3)()
    for i, (x, y) in enumerate(pairs):
        segs[i].a.ptr = x.data_ptr()
        segs[i].a.ld = x.stride(0)
        segs[i].a.mn_major = int(a_mn)
        segs[i].b.ptr = y.data_ptr()
        segs[i].b.ld = y.stride(0)
        segs[i].b.mn_major = int(b_mn)
        segs[i].k = K
    ws_bytes = int(lib.ml_gemm_bf16_workspace_bytes(M, N, 3 * K))
    ws = torch.empty(max(ws_bytes, 16), dtype=torch.uint8, device=out.device)
    _C.call("ml_gemm_bf16", M, N, segs, 3, out.data_ptr(), _C.dtype_code(F32), out.stride(0),
            1.0, float(beta), ws.data_ptr(), ws_bytes, stream)


def mm3(a: Tensor, b: Tensor, a_mn: bool = False, b_mn: bool = False) -> Tensor:
    """fp32 A @ B^T for A logical [M, K], B logical [N, K] with ~fp32 accuracy.

    Storage: A is [M, K] (K-major) or, with a_mn, [K, M]; B is [N, K] or, with
    b_mn, [K, N] — transposed operands are read in place, never copied.
    """
    a = a.to(F32)
    b = b.to(F32)
    M, K = (a.shape[1], a.shape[0]) if a_mn else (a.shape[0], a.shape[1])
    N, Kb = (b.shape[1], b.shape[0]) if b_mn else (b.shape[0], b.shape[1])
    if K != Kb:
        raise RuntimeError(f"mm3: inner sizes differ ({K} vs {Kb})")
    out = torch.empty((M, N), dtype=F32, device=a.device)
    if M == 0 or N == 0:
        return out
    if K == 0:
        return out.zero_()
    a_hi, a_mid, a_lo = _split3(a)
    b_hi, b_mid, b_lo = _split3(b)
    st = _C.stream_of(a)
    _gemm3(((a_hi, b_hi), (a_hi, b_mid), (a_mid, b_hi)), M, N, K, a_mn, b_mn, out, 0.0, st)
    _gemm3(((a_hi, b_lo), (a_lo, b_hi), (a_mid, b_mid)), M, N, K, a_mn, b_mn, out, 1.0, st)
    return out


# ------------------------------- LoRA ------------------------------------
# Formulas of the reference's _LoRA_QKV / _LoRA_MLP (ops/fused_lora.py:96-266)
# with every product through mm3.  U (x A_i^T of each adapter, in rank slot
# [i r, (i + 1) r) of a [T, 64] fp32 tensor) is kept for the backward like the
# bf16 path keeps its bf16 U.

def _slot(u: Tensor, i: int, r: int) -> Tensor:
    return u[:, i * r:(i + 1) * r]


def lora_proj_forward(x2: Tensor, projs, r: int):
    """projs: [(W, A, B, s)]; returns ([Y_i fp32 [T, out_i]], U fp32 [T, 64])."""
    T = x2.shape[0]
    u = torch.zeros((T, 64), dtype=F32, device=x2.device)
    outs = []
    for i, (w, a, b, s) in enumerate(projs):
        ui = mm3(x2, a)
        u[:, i * r:(i + 1) * r] = ui
        outs.append(mm3(x2, w) + float(s) * mm3(ui, b))
    return outs, u


def lora_proj_backward(x2: Tensor, u: Tensor, projs, r: int, dys):
    """Returns (dX fp32 [T, in], [(dA_i fp32 [r, in], dB_i fp32 [out_i, r])])."""
    dx = None
    grads = []
    for i, ((w, a, b, s), dy) in enumerate(zip(projs, dys)):
        s = float(s)
        dy = dy.to(F32)
        g = mm3(dy, b, b_mn=True)                      # dY B        [T, r]
        da = s * mm3(g, x2, a_mn=True, b_mn=True)      # s G^T X     [r, in]
        db = s * mm3(dy, _slot(u, i, r), a_mn=True, b_mn=True)  # s dY^T U  [out, r]
        term = mm3(dy, w, b_mn=True) + s * mm3(g, a, b_mn=True)
        dx = term if dx is None else dx + term
        grads.append((da, db))
    return dx, grads


def lora_mlp_forward(x2: Tensor, gp, up, dp, r: int):
    """Returns (out, gate, up, h, u1, u2), all fp32."""
    from metal_liger_b200 import _torch_library  # noqa: F401  (ops registered)

    (go, uo), u1 = lora_proj_forward(x2, [gp, up], r)
    h = torch.ops.metal_liger.swiglu_forward(go, uo, "")
    (out,), u2 = lora_proj_forward(h, [dp], r)
    return out, go, uo, h, u1, u2


def lora_mlp_backward(x2, gate, up, h, u1, u2, gp, upp, dp, r: int, dy):
    """Returns (dX, [(dA, dB) for gate, up, down]), all fp32."""
    dh, ((dad, dbd),) = lora_proj_backward(h, u2, [dp], r, [dy])
    dgate, dup = torch.ops.metal_liger.swiglu_backward(gate, up, dh.contiguous(), "")
    dx, ((dag, dbg), (dau, dbu)) = lora_proj_backward(x2, u1, [gp, upp], r, [dgate, dup])
    return dx, [(dag, dbg), (dau, dbu), (dad, dbd)]


# -------------------------------- FLCE -----------------------------------
# The reference's chunked algorithm (ops/fused_linear_cross_entropy.py:39-185)
# in fp32, chunked over tokens so that a chunk of logits stays under ~1 GB.

def flce_forward(hidden: Tensor, weight: Tensor, labels: Tensor, bias, ignore_index: int,
                 chunk_size: int, need_dx: bool, need_dw: bool):
    """(loss, dx [1, N, H] fp32 or empty, dw [V, H] fp32 or empty), gradients
    at grad_output = 1."""
    h2 = hidden.reshape(-1, hidden.shape[-1]).to(F32)
    w = weight.to(F32)
    lab = labels.reshape(-1).to(torch.int64)
    N, H = h2.shape
    V = w.shape[0]
    dev = h2.device
    mask = lab != ignore_index
    n_valid = mask.sum().to(F32)
    scale = 1.0 / torch.clamp(n_valid, min=1.0)
    dx = torch.zeros((1, N, H) if need_dx else (0,), dtype=F32, device=dev)
    dw = torch.zeros((V, H) if need_dw else (0,), dtype=F32, device=dev)
    total = torch.zeros((), dtype=F32, device=dev)
    rows = max(1, min(int(chunk_size) if chunk_size and chunk_size > 0 else N,
                      (1 << 28) // max(V, 1)))
    for r0 in range(0, N, rows):
        r1 = min(N, r0 + rows)
        hc, lc, mc = h2[r0:r1], lab[r0:r1], mask[r0:r1]
        logits = mm3(hc, w)
        if bias is not None:
            logits = logits + bias.to(F32)
        lse = torch.logsumexp(logits, dim=-1)
        safe = torch.where(mc, lc, torch.zeros_like(lc))
        tgt = logits.gather(1, safe[:, None])[:, 0]
        total = total + ((lse - tgt) * mc.to(F32)).sum()
        if need_dx or need_dw:
            p = torch.exp(logits - lse[:, None]) * (mc.to(F32) * scale)[:, None]
            rows_idx = torch.arange(r1 - r0, device=dev)
            p[rows_idx, safe] -= mc.to(F32) * scale
            if need_dx:
                dx[0, r0:r1] = mm3(p, w, b_mn=True)                  # P W
            if need_dw:
                dw += mm3(p, hc, a_mn=True, b_mn=True)               # P^T h
    return total * scale, dx, dw
