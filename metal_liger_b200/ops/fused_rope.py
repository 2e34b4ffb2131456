"""Fused rotary position embedding on B200 — drop-in for ops/fused_rope.py.

Keeps the reference's names and signatures (`_FusedRoPEFunction.apply(x, cos,
sin)`, `_rotate_half`, `_apply_rotary_fused`, `MetalLigerRoPE`,
`apply_fused_rotary`; reference ops/fused_rope.py:22-127) and adds the
in-kernel recompute the reference's docstring describes but never implements
(ops/fused_rope.py:10-14): `apply_fused_rotary_from_positions` takes
position ids and ``inv_freq`` and evaluates cos/sin in fp32 inside the kernel,
so no cos/sin table is read from HBM.

Both q and k are rotated by ONE kernel launch in `apply_fused_rotary*`.  The
backward is the reference's inverse rotation, x*cos + rotate_half(x)*(-sin)
(ops/fused_rope.py:50-57).  Strided [B, H, S, D] views (e.g. the
``transpose(1, 2)`` HF attention produces) are read in place.
"""

from typing import Optional

import torch
import torch.nn as nn

import metal_liger_b200._torch_library  # noqa: F401  (registers metal_liger:: ops)


def _fill_missing_grads(meta, *grads):
    """Autograd passes None for an unused output; rotate zeros in its place."""
    out = []
    for (shape, dtype, device), g in zip(meta, grads):
        out.append(torch.zeros(shape, dtype=dtype, device=device) if g is None else g)
    return out


class _FusedRoPEFunction(torch.autograd.Function):
    """out = x*cos + rotate_half(x)*sin for one tensor (reference signature)."""

    @staticmethod
    def forward(ctx, x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor):
        out = torch.ops.metal_liger.rope_apply(x, cos, sin, 1)
        ctx.save_for_backward(cos, sin)
        ctx.x_dtype = x.dtype
        return out

    @staticmethod
    def backward(ctx, grad_output: torch.Tensor):
        cos, sin = ctx.saved_tensors
        grad_x = torch.ops.metal_liger.rope_apply(grad_output, cos, sin, -1)
        return grad_x.to(ctx.x_dtype), None, None


class _FusedRoPEQKFunction(torch.autograd.Function):
    """q and k rotated with the same cos/sin tables in a single launch."""

    @staticmethod
    def forward(ctx, q, k, cos, sin):
        q_out, k_out = torch.ops.metal_liger.rope_apply_qk(q, k, cos, sin, 1)
        ctx.save_for_backward(cos, sin)
        ctx.dtypes = (q.dtype, k.dtype)
        ctx.out_meta = ((q_out.shape, q_out.dtype, q_out.device),
                        (k_out.shape, k_out.dtype, k_out.device))
        return q_out, k_out

    @staticmethod
    def backward(ctx, dq, dk):
        cos, sin = ctx.saved_tensors
        dq, dk = _fill_missing_grads(ctx.out_meta, dq, dk)
        gq, gk = torch.ops.metal_liger.rope_apply_qk(dq, dk, cos, sin, -1)
        return gq.to(ctx.dtypes[0]), gk.to(ctx.dtypes[1]), None, None


class _FusedRoPEPosFunction(torch.autograd.Function):
    """q and k rotated with cos/sin recomputed in-kernel from positions."""

    @staticmethod
    def forward(ctx, q, k, position_ids, inv_freq, scaling):
        q_out, k_out = torch.ops.metal_liger.rope_apply_qk_pos(
            q, k, position_ids, inv_freq, float(scaling), 1)
        ctx.save_for_backward(position_ids if position_ids is not None else torch.empty(0),
                              inv_freq)
        ctx.has_pos = position_ids is not None
        ctx.scaling = float(scaling)
        ctx.out_meta = ((q_out.shape, q_out.dtype, q_out.device),
                        (k_out.shape, k_out.dtype, k_out.device))
        return q_out, k_out

    @staticmethod
    def backward(ctx, dq, dk):
        pos, inv_freq = ctx.saved_tensors
        dq, dk = _fill_missing_grads(ctx.out_meta, dq, dk)
        gq, gk = torch.ops.metal_liger.rope_apply_qk_pos(
            dq.contiguous() if dq.stride(-1) != 1 else dq,
            dk.contiguous() if dk.stride(-1) != 1 else dk,
            pos if ctx.has_pos else None, inv_freq, ctx.scaling, -1)
        return gq, gk, None, None, None


def _rotate_half(x: torch.Tensor) -> torch.Tensor:
    """Rotate half of the hidden dims: [x1, x2] -> [-x2, x1] (reference helper,
    ops/fused_rope.py:60-64; plain tensor expression, not a kernel)."""
    x1 = x[..., : x.shape[-1] // 2]
    x2 = x[..., x.shape[-1] // 2:]
    return torch.cat((-x2, x1), dim=-1)


def _apply_rotary_fused(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """x*cos + rotate_half(x)*sin in one sm_100a kernel (reference ops/fused_rope.py:67-75)."""
    return torch.ops.metal_liger.rope_apply(x, cos, sin, 1)


class MetalLigerRoPE(nn.Module):
    """Wraps a rotary-embedding module; forwards its (cos, sin) unchanged
    (reference ops/fused_rope.py:78-107: Qwen3-VL applies the rotation inside
    attention, so this wrapper is a pass-through)."""

    def __init__(self, original_rope: nn.Module):
        super().__init__()
        self._original = original_rope
        if hasattr(original_rope, "dim"):
            self.dim = original_rope.dim
        if hasattr(original_rope, "max_position_embeddings"):
            self.max_position_embeddings = original_rope.max_position_embeddings
        if hasattr(original_rope, "base"):
            self.base = original_rope.base
        if hasattr(original_rope, "inv_freq"):
            self.register_buffer("inv_freq", original_rope.inv_freq, persistent=False)

    def forward(self, x, position_ids=None, **kwargs):
        result = self._original(x, position_ids=position_ids, **kwargs)
        if isinstance(result, tuple) and len(result) == 2:
            cos, sin = result
            return cos, sin
        return result


def apply_fused_rotary(q: torch.Tensor, k: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor):
    """Rotate q and k with precomputed cos/sin (reference ops/fused_rope.py:110-127).

    q: [batch, q_heads, seq, head_dim], k: [batch, kv_heads, seq, head_dim];
    cos/sin broadcastable to them ([seq, head_dim] or [batch, 1, seq, head_dim]).
    Returns (q_rot, k_rot); one kernel launch for both.
    """
    return _FusedRoPEQKFunction.apply(q, k, cos, sin)


def rope_inv_freq(head_dim: int, theta: float, device=None) -> torch.Tensor:
    """inv_freq = 1 / theta^(arange(0, D, 2)/D) in fp32, the HF rotary formula."""
    exps = torch.arange(0, head_dim, 2, dtype=torch.int64).float() / head_dim
    return (1.0 / (theta ** exps)).to(device=device, dtype=torch.float32)


def apply_fused_rotary_from_positions(q: torch.Tensor, k: torch.Tensor,
                                      position_ids: Optional[torch.Tensor],
                                      inv_freq: Optional[torch.Tensor] = None,
                                      theta: float = 10000.0,
                                      attention_scaling: float = 1.0):
    """Rotate q and k with cos/sin recomputed in-kernel (fp32) from positions.

    angle[b, s, i] = float(position_ids[b, s]) * inv_freq[i], both halves of the
    head dim sharing inv_freq (HF's ``cat(freqs, freqs)``); cos/sin are scaled by
    ``attention_scaling``.  ``position_ids`` may be None (positions 0..S-1).
    Outputs keep q/k's dtype.
    """
    if inv_freq is None:
        inv_freq = rope_inv_freq(q.shape[-1], theta, device=q.device)
    return _FusedRoPEPosFunction.apply(q, k, position_ids, inv_freq, attention_scaling)
