"""``metal_liger::`` custom operators backed by the sm_100a CUDA library.

Mirrors the reference's torch.library registration (_torch_library.py:26-86)
with two deliberate differences:

* the ``torch.library.Library`` object is held at module scope.  The
  reference builds it as a temporary inside ``torch.library.define(...,
  lib=torch.library.Library(...))`` (_torch_library.py:47,66), so its ops
  vanish again and a second registration raises; here registration happens
  once at import and ``register_metal_liger_ops()`` is idempotent;
* kernels are registered for the ``CUDA`` dispatch key (the reference used
  ``mps``, _torch_library.py:50,69).  No CPU kernel is registered: calling an
  op with CPU tensors raises, there is no fallback.

The reference schemas ``rms_norm_forward(Tensor x, Tensor weight, float eps,
str kernel_dir) -> (Tensor, Tensor)`` and ``swiglu_forward(Tensor gate, Tensor
up, str kernel_dir) -> Tensor`` are kept verbatim; ``kernel_dir`` is accepted
and ignored (kernels are compiled ahead of time).  The other ops extend the
surface to the rest of the hot path.
"""

from __future__ import annotations

import ctypes
import logging

import torch
from torch import Tensor

from metal_liger_b200 import _C

logger = logging.getLogger(__name__)

NAMESPACE = "metal_liger"
_LIB = torch.library.Library(NAMESPACE, "DEF")  # module scope: keeps the ops alive
_REGISTERED = False


def _contig(t: Tensor) -> Tensor:
    return t if t.is_contiguous() else t.contiguous()


# ---------------------------------------------------------------------------
# RMSNorm
# ---------------------------------------------------------------------------

def rms_norm_forward_cuda(x: Tensor, weight: Tensor, eps: float, kernel_dir: str = ""):
    """(y, rrms) with y = x*rsqrt(mean(x^2)+eps)*w in fp32, rrms of shape x.shape[:-1]."""
    _C.require_cuda("rms_norm_forward", x, weight)
    if x.dim() < 1 or weight.dim() != 1 or weight.shape[0] != x.shape[-1]:
        raise RuntimeError(
            f"rms_norm_forward: weight {tuple(weight.shape)} does not match x {tuple(x.shape)}")
    x = _contig(x)
    weight = _contig(weight)
    hidden = x.shape[-1]
    rows = x.numel() // hidden if hidden else 0
    y = torch.empty_like(x, memory_format=torch.contiguous_format)
    rrms = torch.empty(x.shape[:-1], dtype=torch.float32, device=x.device)
    _C.call("ml_rms_norm_forward", _C.ptr(x), _C.dtype_code(x), _C.ptr(weight),
            _C.dtype_code(weight), _C.ptr(y), _C.ptr(rrms), rows, hidden, float(eps),
            _C.stream_of(x))
    return y, rrms


def rms_norm_backward_cuda(x: Tensor, weight: Tensor, grad_out: Tensor, eps: float,
                           kernel_dir: str = "", rrms: Tensor | None = None):
    """(dx, dweight); uses the saved fp32 ``rrms`` when given, else recomputes it."""
    _C.require_cuda("rms_norm_backward", x, weight, grad_out, rrms)
    if grad_out.shape != x.shape:
        raise RuntimeError("rms_norm_backward: grad_out shape differs from x")
    x = _contig(x)
    weight = _contig(weight)
    grad_out = _contig(grad_out.to(x.dtype))
    hidden = x.shape[-1]
    rows = x.numel() // hidden if hidden else 0
    if rrms is not None:
        rrms = _contig(rrms.to(torch.float32))
        if rrms.numel() != rows:
            raise RuntimeError("rms_norm_backward: rrms has the wrong number of rows")
    dx = torch.empty_like(x, memory_format=torch.contiguous_format)
    dw = torch.empty_like(weight, memory_format=torch.contiguous_format)
    lib = _C.load()
    ws_bytes = int(lib.ml_rms_norm_backward_workspace_bytes(rows, hidden))
    ws = torch.empty(max(ws_bytes // 4, 4), dtype=torch.float32, device=x.device)
    _C.call("ml_rms_norm_backward", _C.ptr(x), _C.dtype_code(x), _C.ptr(weight),
            _C.dtype_code(weight), _C.ptr(rrms), _C.ptr(grad_out), _C.ptr(dx), _C.ptr(dw),
            float(eps), _C.ptr(ws), ws.numel() * 4, rows, hidden, _C.stream_of(x))
    return dx, dw


# ---------------------------------------------------------------------------
# SwiGLU
# ---------------------------------------------------------------------------

def swiglu_forward_cuda(gate: Tensor, up: Tensor, kernel_dir: str = "") -> Tensor:
    _C.require_cuda("swiglu_forward", gate, up)
    if gate.shape != up.shape:
        raise RuntimeError("MetalLiger SwiGLU: gate and up must match")
    gate = _contig(gate)
    up = _contig(up.to(gate.dtype))
    out = torch.empty_like(gate, memory_format=torch.contiguous_format)
    _C.call("ml_swiglu_forward", _C.ptr(gate), _C.ptr(up), _C.ptr(out), gate.numel(),
            _C.dtype_code(gate), _C.stream_of(gate))
    return out


def swiglu_backward_cuda(gate: Tensor, up: Tensor, grad_out: Tensor, kernel_dir: str = ""):
    _C.require_cuda("swiglu_backward", gate, up, grad_out)
    if gate.shape != up.shape or grad_out.shape != gate.shape:
        raise RuntimeError("MetalLiger SwiGLU backward: gate, up and grad_out must match")
    up_dtype = up.dtype
    gate = _contig(gate)
    up = _contig(up.to(gate.dtype))
    grad_out = _contig(grad_out.to(gate.dtype))
    dgate = torch.empty_like(gate, memory_format=torch.contiguous_format)
    dup = torch.empty_like(gate, memory_format=torch.contiguous_format)
    _C.call("ml_swiglu_backward", _C.ptr(gate), _C.ptr(up), _C.ptr(grad_out), _C.ptr(dgate),
            _C.ptr(dup), gate.numel(), _C.dtype_code(gate), _C.stream_of(gate))
    return dgate, dup.to(up_dtype)


# ---------------------------------------------------------------------------
# RoPE
# ---------------------------------------------------------------------------

def _as_bhsd(x: Tensor, name: str) -> Tensor:
    if x.dim() == 4:
        return x
    if x.dim() == 3:
        return x.unsqueeze(0)
    raise RuntimeError(f"{name}: expected a [batch, heads, seq, head_dim] tensor, got {x.dim()}-D")


def _rope_view(x: Tensor, out: Tensor) -> _C.RopeTensor:
    v = _C.RopeTensor()
    v.inp = x.data_ptr()
    v.out = out.data_ptr()
    v.heads = x.shape[1]
    for i in range(4):
        v.in_strides[i] = x.stride(i)
        v.out_strides[i] = out.stride(i)
    return v


def _prep_rope_input(x: Tensor, name: str) -> Tensor:
    x = _as_bhsd(x, name)
    if x.stride(-1) != 1:
        x = x.contiguous()
    return x


def _cs_strides(cos: Tensor, sin: Tensor, shape: torch.Size):
    """Broadcast cos/sin to ``shape`` ([B,H,S,D]); returns (cos, sin, strides[b,s,d])."""
    ce = cos.expand(shape) if cos.dim() <= 4 else None
    se = sin.expand(shape) if sin.dim() <= 4 else None
    if ce is None or se is None:
        raise RuntimeError("rope: cos/sin must broadcast to x")
    if ce.stride(1) != 0 or se.stride(1) != 0:
        # Tables that vary per head cannot share the per-position cache.
        if torch.equal(ce[:, :1].expand(shape), ce) and torch.equal(se[:, :1].expand(shape), se):
            ce = ce[:, :1].contiguous().expand(shape)
            se = se[:, :1].contiguous().expand(shape)
        else:
            raise RuntimeError("rope: cos/sin that vary across heads are not supported")
    if (ce.stride(0), ce.stride(2), ce.stride(3)) != (se.stride(0), se.stride(2), se.stride(3)):
        ce = ce[:, :1].contiguous().expand(shape)
        se = se[:, :1].contiguous().expand(shape)
    if se.dtype != ce.dtype:
        se = se.to(ce.dtype)
        se = se[:, :1].contiguous().expand(shape)
        ce = ce[:, :1].contiguous().expand(shape)
    strides = (ctypes.c_int64 * 3)(ce.stride(0), ce.stride(2), ce.stride(3))
    return ce, se, strides


def _rope_launch(tensors, cos, sin, sign, positions=None, inv_freq=None, scaling=1.0,
                 out_dtype=None):
    first = tensors[0]
    B, _, S, D = first.shape
    for t in tensors[1:]:
        if t.shape[0] != B or t.shape[2] != S or t.shape[3] != D:
            raise RuntimeError("rope: q and k must agree on batch, seq and head_dim")
        if t.dtype != first.dtype:
            raise RuntimeError("rope: q and k must have the same dtype")
    in_dtype = first.dtype
    if out_dtype is None:
        out_dtype = in_dtype
    # Outputs take the input's memory layout when it is dense (e.g. q as the
    # [B, H, S, D] transpose of a [B, S, H, D] projection, as in HF attention):
    # the gradient then flows back in the projection's own layout and needs no
    # copy before the q/k norm and projection backward.
    outs = [torch.empty_like(t, dtype=out_dtype) for t in tensors]
    views = [_rope_view(t, o) for t, o in zip(tensors, outs)]
    qv = ctypes.pointer(views[0])
    kv = ctypes.pointer(views[1]) if len(views) > 1 else None
    if cos is not None:
        ce, se, strides = _cs_strides(cos, sin, first.shape)
        _C.call("ml_rope", qv, kv, _C.dtype_code(in_dtype), _C.dtype_code(out_dtype), B, S, D,
                ce.data_ptr(), se.data_ptr(), _C.dtype_code(ce), strides, None, 0, None, 1.0,
                int(sign), _C.stream_of(first))
    else:
        pos_ptr, pos_sb = None, 0
        if positions is not None:
            positions = positions.to(device=first.device, dtype=torch.int64)
            if positions.dim() == 1:
                positions = positions.unsqueeze(0)
            if positions.shape[-1] != S or positions.shape[0] not in (1, B):
                raise RuntimeError("rope: position_ids must be [batch, seq] or [seq]")
            positions = positions.contiguous()
            pos_sb = 0 if positions.shape[0] == 1 else positions.stride(0)
            pos_ptr = positions.data_ptr()
        inv = inv_freq.to(device=first.device, dtype=torch.float32).contiguous()
        if inv.numel() != D // 2:
            raise RuntimeError(f"rope: inv_freq must have head_dim/2 = {D // 2} entries")
        _C.call("ml_rope", qv, kv, _C.dtype_code(in_dtype), _C.dtype_code(out_dtype), B, S, D,
                None, None, 0, None, pos_ptr, pos_sb, inv.data_ptr(), float(scaling), int(sign),
                _C.stream_of(first))
        # keep temporaries alive until the launch is enqueued (it is, by now)
        del positions, inv
    return outs


def rope_apply_cuda(x: Tensor, cos: Tensor, sin: Tensor, sin_sign: int) -> Tensor:
    _C.require_cuda("rope_apply", x, cos, sin)
    orig_dim = x.dim()
    xv = _prep_rope_input(x, "rope_apply")
    out_dtype = torch.promote_types(torch.promote_types(x.dtype, cos.dtype), sin.dtype)
    (y,) = _rope_launch([xv], cos, sin, sin_sign, out_dtype=out_dtype)
    return y if orig_dim == 4 else y.squeeze(0)


def rope_apply_qk_cuda(q: Tensor, k: Tensor, cos: Tensor, sin: Tensor, sin_sign: int):
    _C.require_cuda("rope_apply_qk", q, k, cos, sin)
    qv = _prep_rope_input(q, "rope_apply_qk")
    kv = _prep_rope_input(k, "rope_apply_qk")
    out_dtype = torch.promote_types(torch.promote_types(q.dtype, cos.dtype), sin.dtype)
    yq, yk = _rope_launch([qv, kv], cos, sin, sin_sign, out_dtype=out_dtype)
    if q.dim() == 3:
        yq, yk = yq.squeeze(0), yk.squeeze(0)
    return yq, yk


def rope_apply_pos_cuda(x: Tensor, position_ids: Tensor | None, inv_freq: Tensor,
                        scaling: float, sin_sign: int) -> Tensor:
    _C.require_cuda("rope_apply_pos", x, position_ids, inv_freq)
    orig_dim = x.dim()
    xv = _prep_rope_input(x, "rope_apply_pos")
    (y,) = _rope_launch([xv], None, None, sin_sign, positions=position_ids, inv_freq=inv_freq,
                        scaling=scaling)
    return y if orig_dim == 4 else y.squeeze(0)


def rope_apply_qk_pos_cuda(q: Tensor, k: Tensor, position_ids: Tensor | None, inv_freq: Tensor,
                           scaling: float, sin_sign: int):
    _C.require_cuda("rope_apply_qk_pos", q, k, position_ids, inv_freq)
    qv = _prep_rope_input(q, "rope_apply_qk_pos")
    kv = _prep_rope_input(k, "rope_apply_qk_pos")
    yq, yk = _rope_launch([qv, kv], None, None, sin_sign, positions=position_ids,
                          inv_freq=inv_freq, scaling=scaling)
    if q.dim() == 3:
        yq, yk = yq.squeeze(0), yk.squeeze(0)
    return yq, yk


# ---------------------------------------------------------------------------
# Fused linear cross-entropy
# ---------------------------------------------------------------------------

def _bf16_2d(t: Tensor, cols: int) -> Tensor:
    t = t.reshape(-1, cols)
    if t.dtype != torch.bfloat16:
        t = t.to(torch.bfloat16)
    return _contig(t)


# The tcgen05 paths read 2-D operands with TMA, whose row pitch must be a
# multiple of 16 bytes (8 bf16).  Other sizes are zero-padded to the next
# multiple of 8 (the added rows/columns contribute zero products, and the
# padding is sliced off the results), so every shape the reference accepts
# works; multiples of 8 (all Qwen3-VL shapes) take no copies.
def _p8(n: int) -> int:
    return (n + 7) // 8 * 8


def _pad2(t: Tensor, rows: int, cols: int) -> Tensor:
    """Zero-padded [rows, cols] copy of 2-D ``t`` (``t`` itself when it has that shape)."""
    if t.shape[0] == rows and t.shape[1] == cols:
        return t
    out = torch.zeros((rows, cols), dtype=t.dtype, device=t.device)
    out[:t.shape[0], :t.shape[1]] = t
    return out


def _pad_proj(w: Tensor, a: Tensor, b: Tensor, fin8: int):
    """Pads one adapter (W [out, in], A [r, in], B [out, r]) to in = fin8,
    out = multiple of 8."""
    o8 = _p8(w.shape[0])
    r = a.shape[0]
    return _pad2(w, o8, fin8), _pad2(a, r, fin8), _pad2(b, o8, r)


def flce_forward_cuda(hidden: Tensor, weight: Tensor, labels: Tensor, bias: Tensor | None,
                      ignore_index: int, chunk_size: int, need_dx: bool, need_dw: bool):
    """(loss, dx_slabs, dw_acc): loss and, when requested, the fp32 gradients at
    grad_output = 1 (dx as split-K slabs [s, N, H], dw [V, H]).

    bf16/fp16 inputs run the fused kernels with bf16 operands; fp32 inputs take
    the fp32-accurate path (three-part bf16 splits, six GEMM products, _fp32_path.py).
    """
    _C.require_cuda("flce_forward", hidden, weight, labels, bias)
    H = hidden.shape[-1]
    if _fp32_mode(hidden):
        from metal_liger_b200 import _fp32_path as F
        if weight.dim() != 2 or weight.shape[1] != H:
            raise RuntimeError(
                f"flce_forward: weight {tuple(weight.shape)} does not match hidden {H}")
        return F.flce_forward(hidden, weight, labels, bias, int(ignore_index), int(chunk_size),
                              need_dx, need_dw)
    if weight.dim() != 2 or weight.shape[1] != H:
        raise RuntimeError(f"flce_forward: weight {tuple(weight.shape)} does not match hidden {H}")
    if H % 8:
        H8 = _p8(H)
        h2 = hidden.reshape(-1, H)
        loss, dx, dw = flce_forward_cuda(_pad2(h2, h2.shape[0], H8), _pad2(weight, weight.shape[0], H8),
                                         labels, bias, ignore_index, chunk_size, need_dx, need_dw)
        if dx.numel():
            dx = dx[..., :H].contiguous()
        if dw.numel():
            dw = dw[:, :H].contiguous()
        return loss, dx, dw
    h2 = _bf16_2d(hidden, H)
    w2 = _bf16_2d(weight, H)
    lab = _contig(labels.reshape(-1).to(torch.int64))
    N, V = h2.shape[0], w2.shape[0]
    if lab.numel() != N:
        raise RuntimeError(f"flce_forward: {lab.numel()} labels for {N} rows")
    b = None
    if bias is not None:
        b = _contig(bias.reshape(-1))
        if b.numel() != V:
            raise RuntimeError("flce_forward: bias must have vocab entries")
    lib = _C.load()
    chunk = int(chunk_size) if chunk_size and chunk_size > 0 else N
    slabs = int(lib.ml_flce_dx_slabs(N, H, V, chunk))
    dev = hidden.device
    loss = torch.empty((), dtype=torch.float32, device=dev)
    dx = torch.empty((slabs, N, H) if need_dx else (0,), dtype=torch.float32, device=dev)
    dw = torch.empty((V, H) if need_dw else (0,), dtype=torch.float32, device=dev)
    ws_bytes = int(lib.ml_flce_workspace_bytes(N, H, V, chunk))
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
    _C.call("ml_flce_forward", _C.ptr(h2), _C.ptr(w2), _C.ptr(b),
            _C.dtype_code(b) if b is not None else 0, _C.ptr(lab), N, H, V, int(ignore_index),
            chunk, _C.ptr(loss), None, _C.ptr(dx) if need_dx else None,
            _C.ptr(dw) if need_dw else None, _C.ptr(ws), ws_bytes, _C.stream_of(hidden))
    return loss, dx, dw


_CODE_TO_DTYPE = {0: torch.float32, 1: torch.bfloat16, 2: torch.float16}


def flce_backward_cuda(grad_output: Tensor, dx_slabs: Tensor, dw_acc: Tensor, dh_dtype: int,
                       dw_dtype: int):
    """(dhidden [N, H], dweight [V, H]) = grad_output * saved gradients, cast."""
    _C.require_cuda("flce_backward", grad_output, dx_slabs, dw_acc)
    g = _contig(grad_output.reshape(1).to(torch.float32))
    dev = grad_output.device
    dh = torch.empty(0, device=dev)
    dwt = torch.empty(0, device=dev)
    n = h = v = 0
    slabs = 1
    if dx_slabs.numel():
        slabs, n, h = dx_slabs.shape
        dh = torch.empty((n, h), dtype=_CODE_TO_DTYPE[dh_dtype], device=dev)
    if dw_acc.numel():
        v, h = dw_acc.shape
        dwt = torch.empty((v, h), dtype=_CODE_TO_DTYPE[dw_dtype], device=dev)
    if dx_slabs.numel() or dw_acc.numel():
        _C.call("ml_flce_backward", _C.ptr(g), _C.ptr(dx_slabs) if dx_slabs.numel() else None,
                slabs, _C.ptr(dh) if dh.numel() else None, dh_dtype, n, max(h, 1),
                _C.ptr(dw_acc) if dw_acc.numel() else None, _C.ptr(dwt) if dwt.numel() else None,
                dw_dtype, v, _C.stream_of(grad_output))
    return dh, dwt


# ---------------------------------------------------------------------------
# Fused LoRA
# ---------------------------------------------------------------------------

def _lora_proj(w: Tensor, a: Tensor, b: Tensor, scaling: float, keep: list) -> _C.LoraProj:
    w = _contig(w if w.dtype == torch.bfloat16 else w.to(torch.bfloat16))
    a = _contig(a)
    b = _contig(b)
    keep += [w, a, b]
    p = _C.LoraProj()
    p.w, p.a, p.b = w.data_ptr(), a.data_ptr(), b.data_ptr()
    p.a_dtype, p.b_dtype = _C.dtype_code(a), _C.dtype_code(b)
    p.out_features = w.shape[0]
    p.scaling = float(scaling)
    return p


def _ptr_array(tensors):
    arr = (ctypes.c_void_p * len(tensors))()
    for i, t in enumerate(tensors):
        arr[i] = t.data_ptr()
    return arr


def _check_rank(a_list, b_list, in_list):
    r = a_list[0].shape[0]
    for a, b, fin in zip(a_list, b_list, in_list):
        if a.dim() != 2 or b.dim() != 2 or a.shape[0] != r or b.shape[1] != r or a.shape[1] != fin:
            raise RuntimeError("lora: A must be [rank, in] and B [out, rank] with one shared rank")
    return r


def _fp32_mode(x: Tensor) -> bool:
    """fp32 inputs take the fp32-accurate path (three-part bf16 splits, six GEMM products, _fp32_path.py)."""
    return x.dtype == torch.float32


def lora_qkv_forward_cuda(x, qw, qa, qb, kw, ka, kb, vw, va, vb, scaling):
    _C.require_cuda("lora_qkv_forward", x, qw, qa, qb, kw, ka, kb, vw, va, vb)
    H = x.shape[-1]
    if _fp32_mode(x):
        from metal_liger_b200 import _fp32_path as F
        r = _check_rank((qa, ka, va), (qb, kb, vb), (H, H, H))
        outs, u = F.lora_proj_forward(x.reshape(-1, H), [(qw, qa, qb, scaling[0]),
                                                         (kw, ka, kb, scaling[1]),
                                                         (vw, va, vb, scaling[2])], r)
        return outs[0], outs[1], outs[2], u
    if H % 8 or any(w.shape[0] % 8 for w in (qw, kw, vw)):
        H8 = _p8(H)
        x2 = x.reshape(-1, H)
        pq, pk, pv = (_pad_proj(w, a, b, H8) for w, a, b in ((qw, qa, qb), (kw, ka, kb),
                                                             (vw, va, vb)))
        q, k, v, u = lora_qkv_forward_cuda(_pad2(x2, x2.shape[0], H8), *pq, *pk, *pv, scaling)
        return (q[:, :qw.shape[0]].contiguous(), k[:, :kw.shape[0]].contiguous(),
                v[:, :vw.shape[0]].contiguous(), u)
    x2 = _bf16_2d(x, H)
    T = x2.shape[0]
    keep: list = []
    projs = (_C.LoraProj * 3)()
    ws_ = (qw, kw, vw)
    r = _check_rank((qa, ka, va), (qb, kb, vb), (H, H, H))
    for i, (w, a, b) in enumerate(((qw, qa, qb), (kw, ka, kb), (vw, va, vb))):
        if w.shape[1] != H:
            raise RuntimeError("lora_qkv_forward: weight in_features differ from x")
        projs[i] = _lora_proj(w, a, b, scaling[i], keep)
    dev = x.device
    outs = [torch.empty((T, w.shape[0]), dtype=torch.bfloat16, device=dev) for w in ws_]
    u = torch.empty((T, 64), dtype=torch.bfloat16, device=dev)
    lib = _C.load()
    nbytes = int(lib.ml_lora_qkv_workspace_bytes(T, H, projs, 0))
    ws = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    _C.call("ml_lora_qkv_forward", _C.ptr(x2), T, H, r, projs, _ptr_array(outs), _C.ptr(u),
            _C.ptr(ws), nbytes, _C.stream_of(x))
    outs = [o.to(x.dtype) for o in outs]
    return outs[0], outs[1], outs[2], u


def lora_qkv_backward_cuda(x, u, qw, qa, qb, kw, ka, kb, vw, va, vb, scaling, dq, dk, dv):
    _C.require_cuda("lora_qkv_backward", x, u, qw, qa, qb, kw, ka, kb, vw, va, vb, dq, dk, dv)
    H = x.shape[-1]
    if u.dtype == torch.float32:
        from metal_liger_b200 import _fp32_path as F
        r = _check_rank((qa, ka, va), (qb, kb, vb), (H, H, H))
        projs = [(qw, qa, qb, scaling[0]), (kw, ka, kb, scaling[1]), (vw, va, vb, scaling[2])]
        dys = [d.reshape(-1, w.shape[0]) for d, w in ((dq, qw), (dk, kw), (dv, vw))]
        dx, grads = F.lora_proj_backward(x.reshape(-1, H).float(), u, projs, r, dys)
        flat = []
        for (da, db), (_, a, b, _) in zip(grads, projs):
            flat += [da.to(a.dtype), db.to(b.dtype)]
        return (dx.to(x.dtype).view(x.shape), *flat)
    if H % 8 or any(w.shape[0] % 8 for w in (qw, kw, vw)):
        H8 = _p8(H)
        x2 = x.reshape(-1, H)
        T = x2.shape[0]
        trip = ((qw, qa, qb, dq), (kw, ka, kb, dk), (vw, va, vb, dv))
        padded = [_pad_proj(w, a, b, H8) for w, a, b, _ in trip]
        dys = [_pad2(d.reshape(T, w.shape[0]), T, _p8(w.shape[0])) for w, _, _, d in trip]
        res = lora_qkv_backward_cuda(_pad2(x2, T, H8), u, *padded[0], *padded[1], *padded[2],
                                     scaling, *dys)
        dx = res[0][:, :H].reshape(x.shape)
        grads = []
        for i, (w, _, _, _) in enumerate(trip):
            grads += [res[1 + 2 * i][:, :H].contiguous(), res[2 + 2 * i][:w.shape[0]].contiguous()]
        return (dx.contiguous(), *grads)
    x2 = _bf16_2d(x, H)
    T = x2.shape[0]
    keep: list = []
    projs = (_C.LoraProj * 3)()
    r = _check_rank((qa, ka, va), (qb, kb, vb), (H, H, H))
    for i, (w, a, b) in enumerate(((qw, qa, qb), (kw, ka, kb), (vw, va, vb))):
        projs[i] = _lora_proj(w, a, b, scaling[i], keep)
    dys = [_bf16_2d(d, w.shape[0]) for d, w in ((dq, qw), (dk, kw), (dv, vw))]
    dev = x.device
    dx = torch.empty((T, H), dtype=torch.bfloat16, device=dev)
    # adapter gradients in the adapters' own dtypes (fp32 accumulation inside)
    das = [torch.empty((r, H), dtype=a.dtype, device=dev) for a in (qa, ka, va)]
    dbs = [torch.empty((w.shape[0], r), dtype=b.dtype, device=dev)
           for w, b in ((qw, qb), (kw, kb), (vw, vb))]
    lib = _C.load()
    nbytes = int(lib.ml_lora_qkv_workspace_bytes(T, H, projs, 1))
    ws = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    _C.call("ml_lora_qkv_backward", _C.ptr(x2), _C.ptr(_contig(u)), T, H, r, projs,
            _ptr_array(dys), _C.ptr(dx), _ptr_array(das), _ptr_array(dbs), _C.ptr(ws), nbytes,
            _C.stream_of(x))
    return (dx.to(x.dtype).view(x.shape), das[0], dbs[0], das[1], dbs[1], das[2], dbs[2])


def lora_linear_forward_cuda(x, w, a, b, scaling):
    _C.require_cuda("lora_linear_forward", x, w, a, b)
    H = x.shape[-1]
    if _fp32_mode(x):
        from metal_liger_b200 import _fp32_path as F
        r = _check_rank((a,), (b,), (H,))
        (y,), u = F.lora_proj_forward(x.reshape(-1, H), [(w, a, b, scaling)], r)
        return y, u
    if w.dim() == 2 and (H % 8 or w.shape[0] % 8):
        x2 = x.reshape(-1, H)
        y, u = lora_linear_forward_cuda(_pad2(x2, x2.shape[0], _p8(H)),
                                        *_pad_proj(w, a, b, _p8(H)), scaling)
        return y[:, :w.shape[0]].contiguous(), u
    x2 = _bf16_2d(x, H)
    T = x2.shape[0]
    if w.dim() != 2 or w.shape[1] != H:
        raise RuntimeError("lora_linear_forward: weight must be [out, in] with in == x.shape[-1]")
    r = _check_rank((a,), (b,), (H,))
    keep: list = []
    projs = (_C.LoraProj * 1)()
    projs[0] = _lora_proj(w, a, b, scaling, keep)
    dev = x.device
    out = torch.empty((T, w.shape[0]), dtype=torch.bfloat16, device=dev)
    u = torch.empty((T, 64), dtype=torch.bfloat16, device=dev)
    lib = _C.load()
    nbytes = int(lib.ml_lora_linear_workspace_bytes(T, H, 1, projs, 0))
    ws = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    _C.call("ml_lora_linear_forward", _C.ptr(x2), T, H, r, 1, projs, _ptr_array([out]),
            _C.ptr(u), _C.ptr(ws), nbytes, _C.stream_of(x))
    return out.to(x.dtype), u


def lora_linear_backward_cuda(x, u, w, a, b, scaling, dy):
    _C.require_cuda("lora_linear_backward", x, u, w, a, b, dy)
    H = x.shape[-1]
    if u.dtype == torch.float32:
        from metal_liger_b200 import _fp32_path as F
        r = _check_rank((a,), (b,), (H,))
        dx, ((da, db),) = F.lora_proj_backward(x.reshape(-1, H).float(), u, [(w, a, b, scaling)],
                                               r, [dy.reshape(-1, w.shape[0])])
        return dx.to(x.dtype).view(x.shape), da.to(a.dtype), db.to(b.dtype)
    if w.dim() == 2 and (H % 8 or w.shape[0] % 8):
        x2 = x.reshape(-1, H)
        T = x2.shape[0]
        o8 = _p8(w.shape[0])
        dxp, dap, dbp = lora_linear_backward_cuda(
            _pad2(x2, T, _p8(H)), u, *_pad_proj(w, a, b, _p8(H)), scaling,
            _pad2(dy.reshape(T, w.shape[0]), T, o8))
        return (dxp[:, :H].reshape(x.shape).contiguous(), dap[:, :H].contiguous(),
                dbp[:w.shape[0]].contiguous())
    x2 = _bf16_2d(x, H)
    T = x2.shape[0]
    r = _check_rank((a,), (b,), (H,))
    keep: list = []
    projs = (_C.LoraProj * 1)()
    projs[0] = _lora_proj(w, a, b, scaling, keep)
    dys = [_bf16_2d(dy, w.shape[0])]
    dev = x.device
    dx = torch.empty((T, H), dtype=torch.bfloat16, device=dev)
    da = torch.empty((r, H), dtype=a.dtype, device=dev)
    db = torch.empty((w.shape[0], r), dtype=b.dtype, device=dev)
    lib = _C.load()
    nbytes = int(lib.ml_lora_linear_workspace_bytes(T, H, 1, projs, 1))
    ws = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    _C.call("ml_lora_linear_backward", _C.ptr(x2), _C.ptr(_contig(u)), T, H, r, 1, projs,
            _ptr_array(dys), _C.ptr(dx), _ptr_array([da]), _ptr_array([db]), _C.ptr(ws), nbytes,
            _C.stream_of(x))
    return dx.to(x.dtype).view(x.shape), da, db


def lora_mlp_forward_cuda(x, gw, ga, gb, uw, ua, ub, dw, da, db, scaling):
    _C.require_cuda("lora_mlp_forward", x, gw, ga, gb, uw, ua, ub, dw, da, db)
    H = x.shape[-1]
    if _fp32_mode(x):
        from metal_liger_b200 import _fp32_path as F
        inter = gw.shape[0]
        r = _check_rank((ga, ua, da), (gb, ub, db), (H, H, inter))
        out, g_, u_, h, u1, u2 = F.lora_mlp_forward(
            x.reshape(-1, H), (gw, ga, gb, scaling[0]), (uw, ua, ub, scaling[1]),
            (dw, da, db, scaling[2]), r)
        return out.view(x.shape), g_, u_, h, u1, u2
    inter = gw.shape[0]
    if H % 8 or inter % 8:
        H8, I8 = _p8(H), _p8(inter)
        x2 = x.reshape(-1, H)
        out, g_, u_, h, u1, u2 = lora_mlp_forward_cuda(
            _pad2(x2, x2.shape[0], H8), *_pad_proj(gw, ga, gb, H8), *_pad_proj(uw, ua, ub, H8),
            *_pad_proj(dw, da, db, I8), scaling)
        return (out[:, :H].reshape(x.shape).contiguous(), g_[:, :inter].contiguous(),
                u_[:, :inter].contiguous(), h[:, :inter].contiguous(), u1, u2)
    x2 = _bf16_2d(x, H)
    T = x2.shape[0]
    if uw.shape[0] != inter or dw.shape != (H, inter) or gw.shape[1] != H or uw.shape[1] != H:
        raise RuntimeError("lora_mlp_forward: gate/up must be [inter, hidden], down [hidden, inter]")
    r = _check_rank((ga, ua, da), (gb, ub, db), (H, H, inter))
    keep: list = []
    projs = (_C.LoraProj * 3)()
    for i, (w, a, b) in enumerate(((gw, ga, gb), (uw, ua, ub), (dw, da, db))):
        projs[i] = _lora_proj(w, a, b, scaling[i], keep)
    dev = x.device
    bf = torch.bfloat16
    gate = torch.empty((T, inter), dtype=bf, device=dev)
    up = torch.empty((T, inter), dtype=bf, device=dev)
    h = torch.empty((T, inter), dtype=bf, device=dev)
    out = torch.empty((T, H), dtype=bf, device=dev)
    u1 = torch.empty((T, 64), dtype=bf, device=dev)
    u2 = torch.empty((T, 64), dtype=bf, device=dev)
    lib = _C.load()
    nbytes = int(lib.ml_lora_mlp_workspace_bytes(T, H, inter, 0))
    ws = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    _C.call("ml_lora_mlp_forward", _C.ptr(x2), T, H, inter, r, projs, _C.ptr(gate), _C.ptr(up),
            _C.ptr(h), _C.ptr(out), _C.ptr(u1), _C.ptr(u2), _C.ptr(ws), nbytes, _C.stream_of(x))
    return out.to(x.dtype).view(x.shape), gate, up, h, u1, u2


def lora_mlp_backward_cuda(x, gate, up, h, u1, u2, gw, ga, gb, uw, ua, ub, dw, da, db, scaling,
                           dy):
    _C.require_cuda("lora_mlp_backward", x, gate, up, h, u1, u2, gw, ga, gb, uw, ua, ub, dw, da,
                    db, dy)
    H = x.shape[-1]
    if u1.dtype == torch.float32:
        from metal_liger_b200 import _fp32_path as F
        inter = gw.shape[0]
        r = _check_rank((ga, ua, da), (gb, ub, db), (H, H, inter))
        projs = ((gw, ga, gb, scaling[0]), (uw, ua, ub, scaling[1]), (dw, da, db, scaling[2]))
        dx, grads = F.lora_mlp_backward(x.reshape(-1, H).float(), gate, up, h, u1, u2, *projs, r,
                                        dy.reshape(-1, H))
        flat = []
        for (ga_, gb_), (_, a, b, _) in zip(grads, projs):
            flat += [ga_.to(a.dtype), gb_.to(b.dtype)]
        return (dx.to(x.dtype).view(x.shape), *flat)
    inter = gw.shape[0]
    if H % 8 or inter % 8:
        H8, I8 = _p8(H), _p8(inter)
        x2 = x.reshape(-1, H)
        T = x2.shape[0]
        res = lora_mlp_backward_cuda(
            _pad2(x2, T, H8), _pad2(gate.reshape(T, inter), T, I8),
            _pad2(up.reshape(T, inter), T, I8), _pad2(h.reshape(T, inter), T, I8), u1, u2,
            *_pad_proj(gw, ga, gb, H8), *_pad_proj(uw, ua, ub, H8), *_pad_proj(dw, da, db, I8),
            scaling, _pad2(dy.reshape(T, H), T, H8))
        cut = ((H, inter), (H, inter), (inter, H))    # (in, out) of gate, up, down
        grads = []
        for i, (fin, fout) in enumerate(cut):
            grads += [res[1 + 2 * i][:, :fin].contiguous(), res[2 + 2 * i][:fout].contiguous()]
        return (res[0][:, :H].reshape(x.shape).contiguous(), *grads)
    x2 = _bf16_2d(x, H)
    T = x2.shape[0]
    r = _check_rank((ga, ua, da), (gb, ub, db), (H, H, inter))
    keep: list = []
    projs = (_C.LoraProj * 3)()
    for i, (w, a, b) in enumerate(((gw, ga, gb), (uw, ua, ub), (dw, da, db))):
        projs[i] = _lora_proj(w, a, b, scaling[i], keep)
    dy2 = _bf16_2d(dy, H)
    dev = x.device
    dx = torch.empty((T, H), dtype=torch.bfloat16, device=dev)
    das = [torch.empty((r, fin), dtype=a.dtype, device=dev)
           for fin, a in ((H, ga), (H, ua), (inter, da))]
    dbs = [torch.empty((fo, r), dtype=b.dtype, device=dev)
           for fo, b in ((inter, gb), (inter, ub), (H, db))]
    lib = _C.load()
    nbytes = int(lib.ml_lora_mlp_workspace_bytes(T, H, inter, 1))
    ws = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    _C.call("ml_lora_mlp_backward", _C.ptr(x2), _C.ptr(_contig(gate)), _C.ptr(_contig(up)),
            _C.ptr(_contig(h)), _C.ptr(_contig(u1)), _C.ptr(_contig(u2)), T, H, inter, r, projs,
            _C.ptr(dy2), _C.ptr(dx), _ptr_array(das), _ptr_array(dbs), _C.ptr(ws), nbytes,
            _C.stream_of(x))
    return (dx.to(x.dtype).view(x.shape), das[0], dbs[0], das[1], dbs[1], das[2], dbs[2])


# ---------------------------------------------------------------------------
# Registration
# ---------------------------------------------------------------------------

def lm_head_argmax_cuda(hidden: Tensor, weight: Tensor, bias: Tensor | None, logit_dtype: int):
    """Greedy decoding head: (index int64 [B], value fp32 [B]) of the largest
    logit of each row of hidden [B, H] against weight [V, H] (bf16), the
    logits rounded to the dtype ``logit_dtype`` (an ML_DTYPE_* code) and never
    stored; ties and NaN as torch.argmax."""
    _C.require_cuda("lm_head_argmax", hidden, weight, bias)
    if hidden.dtype != torch.bfloat16 or weight.dtype != torch.bfloat16:
        raise RuntimeError("lm_head_argmax: hidden and weight must be bfloat16")
    if hidden.dim() != 2 or weight.dim() != 2 or hidden.shape[1] != weight.shape[1]:
        raise RuntimeError(f"lm_head_argmax: shapes {tuple(hidden.shape)} x "
                           f"{tuple(weight.shape)} do not match")
    B, H = hidden.shape
    V = weight.shape[0]
    if hidden.stride(1) != 1 or hidden.stride(0) % 8 or hidden.data_ptr() % 16:
        hidden = hidden.contiguous()
    weight = _contig(weight)
    if bias is not None:
        bias = _contig(bias)
    index = torch.empty(B, dtype=torch.int64, device=hidden.device)
    value = torch.empty(B, dtype=torch.float32, device=hidden.device)
    if B == 0:
        return index, value
    lib = _C.load()
    ws_bytes = int(lib.ml_lm_head_argmax_workspace_bytes(B, V))
    ws = torch.empty(max(ws_bytes, 16), dtype=torch.uint8, device=hidden.device)
    _C.call("ml_lm_head_argmax", _C.ptr(hidden), hidden.stride(0), _C.ptr(weight),
            weight.stride(0), _C.ptr(bias), _C.dtype_code(bias) if bias is not None else 0,
            B, H, V, int(logit_dtype), _C.ptr(index), _C.ptr(value), _C.ptr(ws), ws_bytes,
            _C.stream_of(hidden))
    return index, value


def _gemv_rows(name: str, x: Tensor, K: int) -> tuple[int, Tensor]:
    rows = x.numel() // K if K else 0
    if rows > 2:
        raise RuntimeError(f"{name}: {rows} rows; the GEMV path takes at most 2")
    x2 = x.reshape(rows, K)
    if x2.stride(-1) != 1 or (rows > 1 and x2.stride(0) % 8) or x2.data_ptr() % 16:
        x2 = x2.contiguous()
    return rows, x2


def _norm_weight(name: str, norm_weight: Tensor, K: int) -> Tensor:
    if norm_weight.dtype != torch.bfloat16 or norm_weight.shape != (K,):
        raise RuntimeError(f"{name}: the norm weight must be bf16 [{K}]")
    norm_weight = norm_weight.contiguous()
    if norm_weight.data_ptr() % 16:
        norm_weight = norm_weight.clone()
    return norm_weight


def _gemv(name: str, x: Tensor, weight: Tensor, bias: Tensor | None,
          residual: Tensor | None = None) -> Tensor:
    _C.require_cuda(name, x, weight, bias, residual)
    if x.dtype != torch.bfloat16 or weight.dtype != torch.bfloat16:
        raise RuntimeError(f"{name}: x and weight must be bfloat16")
    K = x.shape[-1]
    if weight.dim() != 2 or weight.shape[1] != K:
        raise RuntimeError(f"{name}: weight {tuple(weight.shape)} does not match x "
                           f"{tuple(x.shape)}")
    rows, x2 = _gemv_rows(name, x, K)
    weight = _contig(weight)
    if bias is not None:
        bias = _contig(bias)
    N = weight.shape[0]
    if residual is not None:
        if residual.dtype != torch.bfloat16 or residual.numel() != rows * N or \
                residual.shape[-1] != N:
            raise RuntimeError(f"{name}: residual {tuple(residual.shape)} is not bf16 "
                               f"[..., {N}] with {rows} rows")
        residual = residual.reshape(rows, N).contiguous()
    y = torch.empty((rows, N), dtype=torch.bfloat16, device=x.device)
    if rows:
        ld_x = x2.stride(0) if rows > 1 else K
        bdt = _C.dtype_code(bias) if bias is not None else 0
        if residual is None:
            _C.call("ml_gemv_bf16", _C.ptr(x2), ld_x, _C.ptr(weight), weight.stride(0),
                    _C.ptr(bias), bdt, rows, K, N, _C.ptr(y), _C.dtype_code(torch.bfloat16), N,
                    _C.stream_of(x))
        else:
            _C.call("ml_gemv_residual_bf16", _C.ptr(x2), ld_x, _C.ptr(weight), weight.stride(0),
                    _C.ptr(bias), bdt, _C.ptr(residual), N, rows, K, N, _C.ptr(y), N,
                    _C.stream_of(x))
    return y.reshape(*x.shape[:-1], N)


def gemv_cuda(x: Tensor, weight: Tensor, bias: Tensor | None):
    """Decode-time linear layer for 1-2 activation rows: x [..., K] bf16 with
    at most 2 rows, weight [N, K] bf16 -> [..., N] bf16 (fp32 accumulation,
    one HBM pass over the weight)."""
    return _gemv("gemv", x, weight, bias)


def gemv_residual_cuda(x: Tensor, weight: Tensor, bias: Tensor | None, residual: Tensor):
    """residual + gemv(x, weight, bias) in one launch, bit for bit the two
    ops (the decoder layer's `residual + o_proj(...)` / `+ down_proj(...)`)."""
    return _gemv("gemv_residual", x, weight, bias, residual)


def _gemv_swiglu(name: str, x: Tensor, norm_weight: Tensor | None, eps: float, w_gate: Tensor,
                 w_up: Tensor) -> Tensor:
    _C.require_cuda(name, x, w_gate, w_up, norm_weight)
    if x.dtype != torch.bfloat16 or w_gate.dtype != torch.bfloat16 or w_up.dtype != torch.bfloat16:
        raise RuntimeError(f"{name}: x and the weights must be bfloat16")
    K = x.shape[-1]
    if w_gate.shape != w_up.shape or w_gate.dim() != 2 or w_gate.shape[1] != K:
        raise RuntimeError(f"{name}: weights {tuple(w_gate.shape)} / {tuple(w_up.shape)} "
                           f"do not match x {tuple(x.shape)}")
    rows, x2 = _gemv_rows(name, x, K)
    if norm_weight is not None:
        norm_weight = _norm_weight(name, norm_weight, K)
    w_gate, w_up = _contig(w_gate), _contig(w_up)
    inter = w_gate.shape[0]
    y = torch.empty((rows, inter), dtype=torch.bfloat16, device=x.device)
    if rows:
        ld_x = x2.stride(0) if rows > 1 else K
        if norm_weight is None:
            _C.call("ml_gemv_swiglu_bf16", _C.ptr(x2), ld_x, _C.ptr(w_gate), w_gate.stride(0),
                    _C.ptr(w_up), w_up.stride(0), rows, K, inter, _C.ptr(y), inter,
                    _C.stream_of(x))
        else:
            _C.call("ml_gemv_rmsnorm_swiglu_bf16", _C.ptr(x2), ld_x, _C.ptr(norm_weight),
                    float(eps), _C.ptr(w_gate), w_gate.stride(0), _C.ptr(w_up), w_up.stride(0),
                    rows, K, inter, _C.ptr(y), inter, _C.stream_of(x))
    return y.reshape(*x.shape[:-1], inter)


def gemv_swiglu_cuda(x: Tensor, w_gate: Tensor, w_up: Tensor):
    """Decode-time SwiGLU input side for 1-2 rows: silu(x W_g^T) * (x W_u^T),
    bf16, equal bit for bit to gemv, gemv and swiglu_forward."""
    return _gemv_swiglu("gemv_swiglu", x, None, 0.0, w_gate, w_up)


def gemv_rmsnorm_swiglu_cuda(x: Tensor, norm_weight: Tensor, eps: float, w_gate: Tensor,
                             w_up: Tensor):
    """gemv_swiglu of rms_norm_forward(x, norm_weight, eps) in one launch, bit
    for bit the two ops (the decoder layer's post-attention norm and MLP
    input side)."""
    return _gemv_swiglu("gemv_rmsnorm_swiglu", x, norm_weight, eps, w_gate, w_up)


def _gemv_multi(name: str, x: Tensor, norm_weight: Tensor | None, eps: float,
                weights: list[Tensor], biases: list[Tensor | None]):
    import ctypes

    _C.require_cuda(name, x, *weights, *[b for b in biases if b is not None], norm_weight)
    if not 1 <= len(weights) <= 4 or (biases and len(biases) != len(weights)):
        raise RuntimeError(f"{name}: 1-4 weights, and one bias entry per weight if any")
    K = x.shape[-1]
    if x.dtype != torch.bfloat16 or any(w.dtype != torch.bfloat16 or w.dim() != 2 or
                                        w.shape[1] != K for w in weights):
        raise RuntimeError(f"{name}: bf16 x [..., K] and bf16 weights [N_i, K]")
    rows, x2 = _gemv_rows(name, x, K)
    if norm_weight is not None:
        norm_weight = _norm_weight(name, norm_weight, K)
    weights = [_contig(w) for w in weights]
    biases = [None if b is None else _contig(b) for b in (biases or [None] * len(weights))]
    bdt = {b.dtype for b in biases if b is not None}
    if len(bdt) > 1:
        raise RuntimeError(f"{name}: biases of different dtypes")
    outs = [torch.empty((rows, w.shape[0]), dtype=torch.bfloat16, device=x.device)
            for w in weights]
    if rows:
        m = len(weights)
        P = ctypes.c_void_p * m
        I64 = ctypes.c_int64 * m
        mats = (m, P(*[w.data_ptr() for w in weights]), I64(*[w.stride(0) for w in weights]),
                I64(*[w.shape[0] for w in weights]),
                P(*[0 if b is None else b.data_ptr() for b in biases]) if bdt else None,
                _C.dtype_code(bdt.pop()) if bdt else 0, rows, K,
                P(*[o.data_ptr() for o in outs]), I64(*[o.shape[1] for o in outs]),
                _C.dtype_code(torch.bfloat16))
        ld_x = x2.stride(0) if rows > 1 else K
        if norm_weight is None:
            _C.call("ml_gemv_multi_bf16", _C.ptr(x2), ld_x, *mats, _C.stream_of(x))
        else:
            _C.call("ml_gemv_rmsnorm_multi_bf16", _C.ptr(x2), ld_x, _C.ptr(norm_weight),
                    float(eps), *mats, _C.stream_of(x))
    return [o.reshape(*x.shape[:-1], o.shape[1]) for o in outs]


def gemv_multi_cuda(x: Tensor, weights: list[Tensor], biases: list[Tensor | None]):
    """Several decode-time projections of the same 1-2 activation rows in one
    launch (q, k and v): [x W_i^T (+ b_i)] as bf16 tensors [..., N_i]."""
    return _gemv_multi("gemv_multi", x, None, 0.0, weights, biases)


def gemv_rmsnorm_multi_cuda(x: Tensor, norm_weight: Tensor, eps: float, weights: list[Tensor],
                            biases: list[Tensor | None]):
    """gemv_multi of rms_norm_forward(x, norm_weight, eps) in one launch, bit
    for bit the two ops (the decoder layer's input norm and q/k/v)."""
    return _gemv_multi("gemv_rmsnorm_multi", x, norm_weight, eps, weights, biases)


def decode_attention_cuda(q: Tensor, k_cache: Tensor, v_cache: Tensor, pos: Tensor,
                          len_offset: int, scale: float):
    """One decode step of attention: q [B, Hq, 1, D] against the first
    ``pos + len_offset`` positions (pos: an int64 device tensor) of the static
    caches k/v [B, Hkv, L, D]; returns [B, 1, Hq, D] bf16."""
    _C.require_cuda("decode_attention", q, k_cache, v_cache, pos)
    if q.dtype != torch.bfloat16 or k_cache.dtype != torch.bfloat16 or \
            v_cache.dtype != torch.bfloat16:
        raise RuntimeError("decode_attention: bf16 q and caches")
    if q.dim() != 4 or q.shape[2] != 1 or k_cache.dim() != 4 or k_cache.shape != v_cache.shape:
        raise RuntimeError(f"decode_attention: q {tuple(q.shape)} must be [B, Hq, 1, D] and the "
                           f"caches equal [B, Hkv, L, D]")
    B, Hq, _, D = q.shape
    Bk, Hkv, L, Dk = k_cache.shape
    if Bk != B or Dk != D or pos.dtype != torch.int64:
        raise RuntimeError("decode_attention: batch / head_dim mismatch or non-int64 position")
    if q.stride(3) != 1:
        q = q.contiguous()
    k_cache, v_cache = _contig(k_cache), _contig(v_cache)
    out = torch.empty((B, 1, Hq, D), dtype=torch.bfloat16, device=q.device)
    lib = _C.load()
    # caches of up to 8 chunks run as one launch that needs no workspace
    nbytes = int(lib.ml_decode_attention_workspace_bytes(B, Hq, L, D))
    ws = torch.empty(nbytes, dtype=torch.uint8, device=q.device) if nbytes else None
    _C.call("ml_decode_attention_bf16", _C.ptr(q), q.stride(0), q.stride(1), _C.ptr(k_cache),
            _C.ptr(v_cache), _C.ptr(pos), int(len_offset), B, Hq, Hkv, L, D, float(scale),
            _C.ptr(out), _C.ptr(ws), nbytes, _C.stream_of(q))
    return out


def decode_qk_norm_rope_cuda(q: Tensor, k: Tensor, v: Tensor, wq: Tensor, wk: Tensor,
                             eps_q: float, eps_k: float, cos: Tensor, sin: Tensor,
                             k_cache: Tensor, v_cache: Tensor, pos: Tensor):
    """Decode step, one new token per sequence: per-head RMSNorm + RoPE of q
    ([B, 1, Hq*D]) and k, k and v written into the caches [B, Hkv, L, D] at
    the device position ``pos``; returns q as [B, Hq, 1, D] bf16."""
    _C.require_cuda("decode_qk_norm_rope", q, k, v, wq, wk, cos, sin, k_cache, v_cache, pos)
    B, Hkv, L, D = k_cache.shape
    if any(t.dtype != torch.bfloat16 for t in (q, k, v, k_cache, v_cache)):
        raise RuntimeError("decode_qk_norm_rope: bf16 q, k, v and caches")
    if q.numel() % (B * D) or k.numel() != B * Hkv * D or v.numel() != B * Hkv * D:
        raise RuntimeError("decode_qk_norm_rope: q/k/v sizes do not match the caches")
    if v_cache.shape != k_cache.shape or not (k_cache.is_contiguous() and v_cache.is_contiguous()):
        raise RuntimeError("decode_qk_norm_rope: contiguous caches of equal shape")
    if pos.dtype != torch.int64 or wq.numel() != D or wk.numel() != D:
        raise RuntimeError("decode_qk_norm_rope: int64 position and [D] norm weights")
    Hq = q.numel() // (B * D)
    q, k, v = _contig(q), _contig(k), _contig(v)
    cos2 = _contig(cos.reshape(B, -1))
    sin2 = _contig(sin.reshape(B, -1))
    if cos2.shape[1] != D or sin2.shape != cos2.shape:
        raise RuntimeError("decode_qk_norm_rope: cos/sin must be [B, (1,) D]")
    wq, wk = _contig(wq), _contig(wk)
    if wk.dtype != wq.dtype:
        wk = wk.to(wq.dtype)
    q_out = torch.empty((B, Hq, 1, D), dtype=torch.bfloat16, device=q.device)
    _C.call("ml_decode_qk_norm_rope_bf16", _C.ptr(q), _C.ptr(k), _C.ptr(v), _C.ptr(wq),
            _C.ptr(wk), _C.dtype_code(wq), float(eps_q), float(eps_k), _C.ptr(cos2),
            _C.ptr(sin2), _C.dtype_code(cos2), D, B, Hq, Hkv, L, D, _C.ptr(q_out),
            _C.ptr(k_cache), _C.ptr(v_cache), _C.ptr(pos), _C.stream_of(q))
    return q_out


def decode_qk_attention_cuda(q: Tensor, k: Tensor, v: Tensor, wq: Tensor, wk: Tensor,
                             eps_q: float, eps_k: float, cos: Tensor, sin: Tensor,
                             k_cache: Tensor, v_cache: Tensor, pos: Tensor, scale: float):
    """decode_qk_norm_rope followed by decode_attention(..., len_offset=1) in
    one launch, bit for bit the two ops, for caches of at most 256 positions;
    returns [B, 1, Hq, D] bf16."""
    _C.require_cuda("decode_qk_attention", q, k, v, wq, wk, cos, sin, k_cache, v_cache, pos)
    B, Hkv, L, D = k_cache.shape
    if any(t.dtype != torch.bfloat16 for t in (q, k, v, k_cache, v_cache)):
        raise RuntimeError("decode_qk_attention: bf16 q, k, v and caches")
    if q.numel() % (B * D) or k.numel() != B * Hkv * D or v.numel() != B * Hkv * D:
        raise RuntimeError("decode_qk_attention: q/k/v sizes do not match the caches")
    if v_cache.shape != k_cache.shape or not (k_cache.is_contiguous() and v_cache.is_contiguous()):
        raise RuntimeError("decode_qk_attention: contiguous caches of equal shape")
    if pos.dtype != torch.int64 or wq.numel() != D or wk.numel() != D:
        raise RuntimeError("decode_qk_attention: int64 position and [D] norm weights")
    Hq = q.numel() // (B * D)
    q, k, v = _contig(q), _contig(k), _contig(v)
    cos2 = _contig(cos.reshape(B, -1))
    sin2 = _contig(sin.reshape(B, -1))
    if cos2.shape[1] != D or sin2.shape != cos2.shape:
        raise RuntimeError("decode_qk_attention: cos/sin must be [B, (1,) D]")
    wq, wk = _contig(wq), _contig(wk)
    if wk.dtype != wq.dtype:
        wk = wk.to(wq.dtype)
    out = torch.empty((B, 1, Hq, D), dtype=torch.bfloat16, device=q.device)
    _C.call("ml_decode_qk_attention_bf16", _C.ptr(q), _C.ptr(k), _C.ptr(v), _C.ptr(wq),
            _C.ptr(wk), _C.dtype_code(wq), float(eps_q), float(eps_k), _C.ptr(cos2),
            _C.ptr(sin2), _C.dtype_code(cos2), D, B, Hq, Hkv, L, D, _C.ptr(k_cache),
            _C.ptr(v_cache), _C.ptr(pos), float(scale), _C.ptr(out), _C.stream_of(q))
    return out


_SCHEMAS = {
    "decode_qk_norm_rope": "decode_qk_norm_rope(Tensor q, Tensor k, Tensor v, Tensor wq, "
                           "Tensor wk, float eps_q, float eps_k, Tensor cos, Tensor sin, "
                           "Tensor(a!) k_cache, Tensor(b!) v_cache, Tensor pos) -> Tensor",
    "decode_qk_attention": "decode_qk_attention(Tensor q, Tensor k, Tensor v, Tensor wq, "
                           "Tensor wk, float eps_q, float eps_k, Tensor cos, Tensor sin, "
                           "Tensor(a!) k_cache, Tensor(b!) v_cache, Tensor pos, float scale) "
                           "-> Tensor",
    "decode_attention": "decode_attention(Tensor q, Tensor k_cache, Tensor v_cache, Tensor pos, "
                        "int len_offset, float scale) -> Tensor",
    "gemv_multi": "gemv_multi(Tensor x, Tensor[] weights, Tensor?[] biases) -> Tensor[]",
    "gemv_swiglu": "gemv_swiglu(Tensor x, Tensor w_gate, Tensor w_up) -> Tensor",
    "gemv": "gemv(Tensor x, Tensor weight, Tensor? bias) -> Tensor",
    "gemv_residual": "gemv_residual(Tensor x, Tensor weight, Tensor? bias, Tensor residual) "
                     "-> Tensor",
    "gemv_rmsnorm_multi": "gemv_rmsnorm_multi(Tensor x, Tensor norm_weight, float eps, "
                          "Tensor[] weights, Tensor?[] biases) -> Tensor[]",
    "gemv_rmsnorm_swiglu": "gemv_rmsnorm_swiglu(Tensor x, Tensor norm_weight, float eps, "
                           "Tensor w_gate, Tensor w_up) -> Tensor",
    "lm_head_argmax": "lm_head_argmax(Tensor hidden, Tensor weight, Tensor? bias, "
                      "int logit_dtype) -> (Tensor, Tensor)",
    "rms_norm_forward": "rms_norm_forward(Tensor x, Tensor weight, float eps, str kernel_dir) "
                        "-> (Tensor, Tensor)",
    "rms_norm_backward": "rms_norm_backward(Tensor x, Tensor weight, Tensor grad_out, float eps, "
                         "str kernel_dir, Tensor? rrms=None) -> (Tensor, Tensor)",
    "swiglu_forward": "swiglu_forward(Tensor gate, Tensor up, str kernel_dir) -> Tensor",
    "swiglu_backward": "swiglu_backward(Tensor gate, Tensor up, Tensor grad_out, str kernel_dir) "
                       "-> (Tensor, Tensor)",
    "rope_apply": "rope_apply(Tensor x, Tensor cos, Tensor sin, int sin_sign) -> Tensor",
    "rope_apply_qk": "rope_apply_qk(Tensor q, Tensor k, Tensor cos, Tensor sin, int sin_sign) "
                     "-> (Tensor, Tensor)",
    "rope_apply_pos": "rope_apply_pos(Tensor x, Tensor? position_ids, Tensor inv_freq, "
                      "float scaling, int sin_sign) -> Tensor",
    "rope_apply_qk_pos": "rope_apply_qk_pos(Tensor q, Tensor k, Tensor? position_ids, "
                         "Tensor inv_freq, float scaling, int sin_sign) -> (Tensor, Tensor)",
    "flce_forward": "flce_forward(Tensor hidden, Tensor weight, Tensor labels, Tensor? bias, "
                    "int ignore_index, int chunk_size, bool need_dx, bool need_dw) "
                    "-> (Tensor, Tensor, Tensor)",
    "flce_backward": "flce_backward(Tensor grad_output, Tensor dx_slabs, Tensor dw_acc, "
                     "int dh_dtype, int dw_dtype) -> (Tensor, Tensor)",
    "lora_qkv_forward": "lora_qkv_forward(Tensor x, Tensor qw, Tensor qa, Tensor qb, Tensor kw, "
                        "Tensor ka, Tensor kb, Tensor vw, Tensor va, Tensor vb, float[] scaling) "
                        "-> (Tensor, Tensor, Tensor, Tensor)",
    "lora_qkv_backward": "lora_qkv_backward(Tensor x, Tensor u, Tensor qw, Tensor qa, Tensor qb, "
                         "Tensor kw, Tensor ka, Tensor kb, Tensor vw, Tensor va, Tensor vb, "
                         "float[] scaling, Tensor dq, Tensor dk, Tensor dv) -> (Tensor, Tensor, "
                         "Tensor, Tensor, Tensor, Tensor, Tensor)",
    "lora_linear_forward": "lora_linear_forward(Tensor x, Tensor w, Tensor a, Tensor b, "
                           "float scaling) -> (Tensor, Tensor)",
    "lora_linear_backward": "lora_linear_backward(Tensor x, Tensor u, Tensor w, Tensor a, "
                            "Tensor b, float scaling, Tensor dy) -> (Tensor, Tensor, Tensor)",
    "lora_mlp_forward": "lora_mlp_forward(Tensor x, Tensor gw, Tensor ga, Tensor gb, Tensor uw, "
                        "Tensor ua, Tensor ub, Tensor dw, Tensor da, Tensor db, float[] scaling) "
                        "-> (Tensor, Tensor, Tensor, Tensor, Tensor, Tensor)",
    "lora_mlp_backward": "lora_mlp_backward(Tensor x, Tensor gate, Tensor up, Tensor h, Tensor u1, "
                         "Tensor u2, Tensor gw, Tensor ga, Tensor gb, Tensor uw, Tensor ua, "
                         "Tensor ub, Tensor dw, Tensor da, Tensor db, float[] scaling, Tensor dy) "
                         "-> (Tensor, Tensor, Tensor, Tensor, Tensor, Tensor, Tensor)",
}

_CUDA_IMPLS = {
    "decode_qk_norm_rope": decode_qk_norm_rope_cuda,
    "decode_attention": decode_attention_cuda,
    "gemv_multi": gemv_multi_cuda,
    "gemv_swiglu": gemv_swiglu_cuda,
    "gemv": gemv_cuda,
    "decode_qk_attention": decode_qk_attention_cuda,
    "gemv_residual": gemv_residual_cuda,
    "gemv_rmsnorm_multi": gemv_rmsnorm_multi_cuda,
    "gemv_rmsnorm_swiglu": gemv_rmsnorm_swiglu_cuda,
    "lm_head_argmax": lm_head_argmax_cuda,
    "rms_norm_forward": rms_norm_forward_cuda,
    "rms_norm_backward": rms_norm_backward_cuda,
    "swiglu_forward": swiglu_forward_cuda,
    "swiglu_backward": swiglu_backward_cuda,
    "rope_apply": rope_apply_cuda,
    "rope_apply_qk": rope_apply_qk_cuda,
    "rope_apply_pos": rope_apply_pos_cuda,
    "rope_apply_qk_pos": rope_apply_qk_pos_cuda,
    "flce_forward": flce_forward_cuda,
    "flce_backward": flce_backward_cuda,
    "lora_qkv_forward": lora_qkv_forward_cuda,
    "lora_qkv_backward": lora_qkv_backward_cuda,
    "lora_linear_forward": lora_linear_forward_cuda,
    "lora_linear_backward": lora_linear_backward_cuda,
    "lora_mlp_forward": lora_mlp_forward_cuda,
    "lora_mlp_backward": lora_mlp_backward_cuda,
}


def _promote3(a, b, c):
    return torch.promote_types(torch.promote_types(a.dtype, b.dtype), c.dtype)


def _fake_impls():
    def rms_fwd(x, weight, eps, kernel_dir):
        return (torch.empty_like(x),
                torch.empty(x.shape[:-1], dtype=torch.float32, device=x.device))

    def rms_bwd(x, weight, grad_out, eps, kernel_dir, rrms=None):
        return torch.empty_like(x), torch.empty_like(weight)

    def swi_fwd(gate, up, kernel_dir):
        return torch.empty_like(gate)

    def swi_bwd(gate, up, grad_out, kernel_dir):
        return torch.empty_like(gate), torch.empty_like(up)

    def rope(x, cos, sin, sin_sign):
        return torch.empty(x.shape, dtype=_promote3(x, cos, sin), device=x.device)

    def rope_qk(q, k, cos, sin, sin_sign):
        dt = _promote3(q, cos, sin)
        return (torch.empty(q.shape, dtype=dt, device=q.device),
                torch.empty(k.shape, dtype=dt, device=k.device))

    def rope_pos(x, position_ids, inv_freq, scaling, sin_sign):
        return torch.empty(x.shape, dtype=x.dtype, device=x.device)

    def rope_qk_pos(q, k, position_ids, inv_freq, scaling, sin_sign):
        return (torch.empty(q.shape, dtype=q.dtype, device=q.device),
                torch.empty(k.shape, dtype=k.dtype, device=k.device))

    def flce_fwd(hidden, weight, labels, bias, ignore_index, chunk_size, need_dx, need_dw):
        H = hidden.shape[-1]
        N = hidden.numel() // H
        V = weight.shape[0]
        dev = hidden.device
        slabs = 1  # shape-only estimate for tracing
        return (torch.empty((), dtype=torch.float32, device=dev),
                torch.empty((slabs, N, H) if need_dx else (0,), dtype=torch.float32, device=dev),
                torch.empty((V, H) if need_dw else (0,), dtype=torch.float32, device=dev))

    def flce_bwd(grad_output, dx_slabs, dw_acc, dh_dtype, dw_dtype):
        dev = grad_output.device
        dh = (torch.empty(dx_slabs.shape[1:], dtype=_CODE_TO_DTYPE[dh_dtype], device=dev)
              if dx_slabs.dim() == 3 else torch.empty(0, device=dev))
        dw = (torch.empty(dw_acc.shape, dtype=_CODE_TO_DTYPE[dw_dtype], device=dev)
              if dw_acc.dim() == 2 else torch.empty(0, device=dev))
        return dh, dw

    def _u_dtype(x):
        return torch.float32 if x.dtype == torch.float32 else torch.bfloat16

    def lqkv_fwd(x, qw, qa, qb, kw, ka, kb, vw, va, vb, scaling):
        T = x.numel() // x.shape[-1]
        mk = lambda w: torch.empty((T, w.shape[0]), dtype=x.dtype, device=x.device)  # noqa: E731
        return mk(qw), mk(kw), mk(vw), torch.empty((T, 64), dtype=_u_dtype(x), device=x.device)

    def lqkv_bwd(x, u, qw, qa, qb, kw, ka, kb, vw, va, vb, scaling, dq, dk, dv):
        r, H = qa.shape
        return (torch.empty_like(x), torch.empty_like(qa), torch.empty_like(qb),
                torch.empty_like(ka), torch.empty_like(kb), torch.empty_like(va),
                torch.empty_like(vb))

    def llin_fwd(x, w, a, b, scaling):
        T = x.numel() // x.shape[-1]
        return (torch.empty((T, w.shape[0]), dtype=x.dtype, device=x.device),
                torch.empty((T, 64), dtype=_u_dtype(x), device=x.device))

    def llin_bwd(x, u, w, a, b, scaling, dy):
        return torch.empty_like(x), torch.empty_like(a), torch.empty_like(b)

    def lmlp_fwd(x, gw, ga, gb, uw, ua, ub, dw, da, db, scaling):
        T = x.numel() // x.shape[-1]
        inter = gw.shape[0]
        dt = _u_dtype(x)
        bf = lambda *s: torch.empty(s, dtype=dt, device=x.device)  # noqa: E731
        return (torch.empty_like(x), bf(T, inter), bf(T, inter), bf(T, inter), bf(T, 64),
                bf(T, 64))

    def lmlp_bwd(x, gate, up, h, u1, u2, gw, ga, gb, uw, ua, ub, dw, da, db, scaling, dy):
        return (torch.empty_like(x), torch.empty_like(ga), torch.empty_like(gb),
                torch.empty_like(ua), torch.empty_like(ub), torch.empty_like(da),
                torch.empty_like(db))

    def lm_argmax(hidden, weight, bias, logit_dtype):
        B = hidden.shape[0]
        return (torch.empty(B, dtype=torch.int64, device=hidden.device),
                torch.empty(B, dtype=torch.float32, device=hidden.device))

    def gemv_fake(x, weight, bias):
        return torch.empty((*x.shape[:-1], weight.shape[0]), dtype=x.dtype, device=x.device)

    def gemv_swiglu_fake(x, w_gate, w_up):
        return torch.empty((*x.shape[:-1], w_gate.shape[0]), dtype=x.dtype, device=x.device)

    def gemv_multi_fake(x, weights, biases):
        return [torch.empty((*x.shape[:-1], w.shape[0]), dtype=x.dtype, device=x.device)
                for w in weights]

    def gemv_residual_fake(x, weight, bias, residual):
        return torch.empty((*x.shape[:-1], weight.shape[0]), dtype=x.dtype, device=x.device)

    def gemv_rmsnorm_multi_fake(x, norm_weight, eps, weights, biases):
        return [torch.empty((*x.shape[:-1], w.shape[0]), dtype=x.dtype, device=x.device)
                for w in weights]

    def gemv_rmsnorm_swiglu_fake(x, norm_weight, eps, w_gate, w_up):
        return torch.empty((*x.shape[:-1], w_gate.shape[0]), dtype=x.dtype, device=x.device)

    def decode_qk_attention_fake(q, k, v, wq, wk, eps_q, eps_k, cos, sin, k_cache, v_cache, pos,
                                 scale):
        B, Hkv, L, D = k_cache.shape
        return torch.empty((B, 1, q.numel() // (B * D), D), dtype=q.dtype, device=q.device)

    def decode_attention_fake(q, k_cache, v_cache, pos, len_offset, scale):
        B, Hq, _, D = q.shape
        return torch.empty((B, 1, Hq, D), dtype=q.dtype, device=q.device)

    def decode_qk_fake(q, k, v, wq, wk, eps_q, eps_k, cos, sin, k_cache, v_cache, pos):
        B, Hkv, L, D = k_cache.shape
        return torch.empty((B, q.numel() // (B * D), 1, D), dtype=q.dtype, device=q.device)

    return {
        "decode_qk_norm_rope": decode_qk_fake,
        "decode_attention": decode_attention_fake,
        "gemv_multi": gemv_multi_fake,
        "gemv_swiglu": gemv_swiglu_fake,
        "gemv": gemv_fake,
        "decode_qk_attention": decode_qk_attention_fake,
        "gemv_residual": gemv_residual_fake,
        "gemv_rmsnorm_multi": gemv_rmsnorm_multi_fake,
        "gemv_rmsnorm_swiglu": gemv_rmsnorm_swiglu_fake,
        "lm_head_argmax": lm_argmax,
        "lora_qkv_forward": lqkv_fwd,
        "lora_qkv_backward": lqkv_bwd,
        "lora_linear_forward": llin_fwd,
        "lora_linear_backward": llin_bwd,
        "lora_mlp_forward": lmlp_fwd,
        "lora_mlp_backward": lmlp_bwd,
        "flce_forward": flce_fwd,
        "flce_backward": flce_bwd,
        "rms_norm_forward": rms_fwd,
        "rms_norm_backward": rms_bwd,
        "swiglu_forward": swi_fwd,
        "swiglu_backward": swi_bwd,
        "rope_apply": rope,
        "rope_apply_qk": rope_qk,
        "rope_apply_pos": rope_pos,
        "rope_apply_qk_pos": rope_qk_pos,
    }


def _register_all() -> None:
    fakes = _fake_impls()
    for name, schema in _SCHEMAS.items():
        _LIB.define(schema)
        _LIB.impl(name, _CUDA_IMPLS[name], "CUDA")
        torch.library.register_fake(f"{NAMESPACE}::{name}", fakes[name], lib=_LIB)


def register_metal_liger_ops() -> bool:
    """Register the ``metal_liger::`` ops (idempotent).  Returns True when registered.

    Mirrors reference _torch_library.py:26-86.  Registration does not load the
    CUDA library; the first op call does, and raises if it is missing.
    """
    global _REGISTERED
    if _REGISTERED:
        return True
    _register_all()
    _REGISTERED = True
    logger.debug("metal_liger_b200: registered %d metal_liger:: ops", len(_SCHEMAS))
    return True


def registered_op_names() -> list[str]:
    return list(_SCHEMAS)
