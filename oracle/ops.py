"""CPU oracle: a plain restatement of the reference's hot-path algorithms.

TEST INFRASTRUCTURE ONLY.  Nothing in the product (``metal_liger_b200``)
imports this module; only ``tests/``, ``__graft_entry__.smoke()`` and
``bench.py`` (its CPU-baseline / ``--impl reference`` arm) use it, as the
checker or the timed CPU baseline — never as the thing measured or shipped.

Each function restates the math of the reference file:line it cites
(paths relative to the krrish-v/metal_liger package root) with torch CPU
tensor arithmetic in fp32, the precision the reference computes in.  The
functions take an optional ``dtype`` so tests can also evaluate them in fp64.
It is pinned against fixtures produced by running the reference itself
(tests/golden/make_golden.py); see tests/test_oracle_golden.py.
"""

from __future__ import annotations

import math

import torch

F32 = torch.float32


def _up(t: torch.Tensor | None, dtype=F32):
    return None if t is None else t.to(dtype)


# ---------------------------------------------------------------------------
# RMSNorm — reference ops/fused_rms_norm.py:30-60
# ---------------------------------------------------------------------------

def rms_norm_forward(x, weight, eps, dtype=F32):
    """ops/fused_rms_norm.py:31-41: rrms = rsqrt(mean(x^2)+eps); y = (x*rrms*w).to(x.dtype)."""
    xf = _up(x, dtype)
    var = (xf * xf).mean(dim=-1, keepdim=True)
    rrms = torch.rsqrt(var + eps)
    y = (xf * rrms) * _up(weight, dtype)
    return y.to(x.dtype) if dtype == F32 else y, rrms.squeeze(-1)


def rms_norm_backward(x, weight, rrms, grad_out, dtype=F32):
    """ops/fused_rms_norm.py:43-60: dx = g*w*r - x*mean(g*w*x)*r^3; dw = sum(g*x*r)."""
    g = _up(grad_out, dtype)
    xf = _up(x, dtype)
    wf = _up(weight, dtype)
    r = _up(rrms, dtype).unsqueeze(-1)
    gw = g * wf
    mean_gwx = (gw * xf).mean(dim=-1, keepdim=True)
    dx = gw * r - xf * mean_gwx * r.pow(3)
    dw = (g * (xf * r)).reshape(-1, x.shape[-1]).sum(0)
    if dtype == F32:
        return dx.to(x.dtype), dw.to(weight.dtype)
    return dx, dw


# ---------------------------------------------------------------------------
# SwiGLU — reference ops/fused_swiglu.py:26-50
# ---------------------------------------------------------------------------

def swiglu_forward(gate, up, dtype=F32):
    """ops/fused_swiglu.py:27-35: out = (g*sigmoid(g)*u).to(gate.dtype)."""
    g = _up(gate, dtype)
    s = torch.sigmoid(g)
    out = (g * s) * _up(up, dtype)
    return out.to(gate.dtype) if dtype == F32 else out


def swiglu_backward(gate, up, grad_out, dtype=F32):
    """ops/fused_swiglu.py:38-50: du = go*g*s; dg = go*u*s*(1+g*(1-s))."""
    g = _up(gate, dtype)
    u = _up(up, dtype)
    d = _up(grad_out, dtype)
    s = torch.sigmoid(g)
    du = d * (g * s)
    dg = d * u * s * (1.0 + g * (1.0 - s))
    if dtype == F32:
        return dg.to(gate.dtype), du.to(up.dtype)
    return dg, du


# ---------------------------------------------------------------------------
# RoPE — reference ops/fused_rope.py:22-75
# ---------------------------------------------------------------------------

def rotate_half(x):
    """ops/fused_rope.py:60-64: [x1, x2] -> [-x2, x1]."""
    h = x.shape[-1] // 2
    return torch.cat((-x[..., h:], x[..., :h]), dim=-1)


def rope_apply(x, cos, sin, dtype=F32):
    """ops/fused_rope.py:67-75: x*cos + rotate_half(x)*sin (fp32 arithmetic here)."""
    xf = _up(x, dtype)
    return xf * _up(cos, dtype) + rotate_half(xf) * _up(sin, dtype)


def rope_backward(grad_out, cos, sin, dtype=F32):
    """ops/fused_rope.py:50-57: the same rotation with -sin."""
    return rope_apply(grad_out, cos, -_up(sin, dtype), dtype)


def rope_inv_freq(head_dim, theta):
    """HF rotary: inv_freq = 1 / theta^(arange(0, D, 2)/D), fp32."""
    exps = torch.arange(0, head_dim, 2, dtype=torch.int64).float() / head_dim
    return 1.0 / (theta ** exps)


def rope_cos_sin(position_ids, inv_freq, scaling=1.0):
    """cos/sin [B, S, D] in fp32 from positions (HF's cat(freqs, freqs))."""
    freqs = position_ids.to(F32)[..., None] * inv_freq.to(F32)
    emb = torch.cat((freqs, freqs), dim=-1)
    return emb.cos() * scaling, emb.sin() * scaling


# ---------------------------------------------------------------------------
# Chunked fused linear cross-entropy —
# reference ops/fused_linear_cross_entropy.py:39-185
# ---------------------------------------------------------------------------

def flce_forward(hidden, weight, labels, bias=None, ignore_index=-100, chunk_size=8192,
                 dtype=F32):
    """ops/fused_linear_cross_entropy.py:93-157.

    Online max / sum-exp over vocab chunks (:39-55), lse = m + log(s) (:123),
    target logit by a row dot with W[label] (:135-141), masked mean with the
    count clamped to >= 1 (:143-149).  Returns (loss, lse, mask).
    """
    h = _up(hidden, dtype)
    w = _up(weight, dtype)
    n, v = h.shape[0], w.shape[0]
    run_max = torch.full((n,), float("-inf"), dtype=dtype, device=h.device)
    run_sum = torch.zeros(n, dtype=dtype, device=h.device)
    for start in range(0, v, chunk_size):
        end = min(start + chunk_size, v)
        logits = h @ w[start:end].t()
        if bias is not None:
            logits = logits + _up(bias[start:end], dtype)
        new_max = torch.maximum(run_max, logits.max(dim=-1).values)
        run_sum = run_sum * torch.exp(run_max - new_max) + \
            torch.exp(logits - new_max[:, None]).sum(dim=-1)
        run_max = new_max
    lse = run_max + torch.log(run_sum)
    mask = labels != ignore_index
    safe = torch.where(mask, labels, torch.zeros_like(labels))
    tgt = (h * w[safe]).sum(dim=-1)
    if bias is not None:
        tgt = tgt + _up(bias, dtype)[safe]
    tok = (lse - tgt) * mask.to(dtype)
    loss = tok.sum() / torch.clamp(mask.to(dtype).sum(), min=1.0)
    return loss, lse, mask


def flce_backward(hidden, weight, labels, lse, mask, grad_output=1.0, bias=None,
                  chunk_size=8192, dtype=F32):
    """ops/fused_linear_cross_entropy.py:57-80, :159-185.

    Per vocab chunk: recompute logits, P = exp(l - lse), P[label] -= 1,
    P *= mask * grad / max(sum(mask), 1); dX += P @ W_c; dW_c += P^T @ h.
    The bias gets no gradient (:184-185).  Returns (dX, dW) in the input dtypes
    (fp32/fp64 when dtype != fp32 is requested).
    """
    h = _up(hidden, dtype)
    w = _up(weight, dtype)
    n, v = h.shape[0], w.shape[0]
    num_valid = torch.clamp(mask.to(dtype).sum(), min=1.0)
    go = grad_output if torch.is_tensor(grad_output) else torch.tensor(grad_output)
    go = go.to(h.device)
    scale = go.to(dtype) / num_valid
    fmask = mask.to(dtype)[:, None]
    dx = torch.zeros_like(h)
    dw = torch.zeros_like(w)
    for start in range(0, v, chunk_size):
        end = min(start + chunk_size, v)
        logits = h @ w[start:end].t()
        if bias is not None:
            logits = logits + _up(bias[start:end], dtype)
        p = torch.exp(logits - lse.to(dtype)[:, None])
        cls = torch.arange(start, end, dtype=labels.dtype, device=labels.device)[None, :]
        p = torch.where(labels[:, None] == cls, p - 1.0, p)
        p = p * fmask * scale
        dx += p @ w[start:end]
        dw[start:end] += p.t() @ h
    if dtype == F32:
        return dx.to(hidden.dtype), dw.to(weight.dtype)
    return dx, dw


# ---------------------------------------------------------------------------
# Fused LoRA — reference ops/fused_lora.py:69-266
# ---------------------------------------------------------------------------

def _store(t, store_dtype):
    """Round ``t`` to the dtype the reference stores that intermediate in (no-op
    when ``store_dtype`` is None)."""
    return t if store_dtype is None else t.to(store_dtype).to(t.dtype)


def lora_linear(x, w, a, b, s, store_dtype=None):
    """ops/fused_lora.py:69-82: x W^T + s (x A^T) B^T, in x's dtype.

    ``store_dtype`` rounds the rank projection x A^T where the reference holds it
    as a tensor of the input dtype."""
    dt = x.dtype
    out = x @ w.t()
    if a is not None and b is not None:
        out = out + _store(x @ a.to(dt).t(), store_dtype) @ b.to(dt).t() * s
    return out


def _lora_grads(dy, x, a, b, s, store_dtype=None):
    """ops/fused_lora.py:142-149: dA = s (dY B)^T X ; dB = s dY^T (X A^T), as fp32."""
    dt = dy.dtype
    ac, bc = a.to(dt), b.to(dt)
    da = (_store(dy @ bc, store_dtype).t() @ x * s).float()
    db = (dy.t() @ _store(x @ ac.t(), store_dtype) * s).float()
    return da, db


def _lora_dx(dy, w, a, b, s, store_dtype=None):
    """ops/fused_lora.py:155-161: dY W + s (dY B) A."""
    dt = dy.dtype
    return dy @ w + _store(dy @ b.to(dt), store_dtype) @ a.to(dt) * s


# The reference evaluates in the input dtype.  Tests evaluate the same
# algorithm with fp32 products (``dtype=torch.float32``); ``store_dtype``
# then rounds every intermediate the reference keeps as a tensor of the input
# dtype -- x A^T, dY B, gate, up, h, dH, d_gate, d_up -- so the comparison
# measures accumulation differences, not the reference's own storage
# quantisation.

def lora_qkv_forward(x, q, k, v, dtype=None, store_dtype=None):
    """ops/fused_lora.py:96-119.  q/k/v are (W, A, B, s) tuples.  Returns Q, K, V."""
    cast = (lambda t: t) if dtype is None else (lambda t: t.to(dtype))
    xf = cast(x).reshape(-1, x.shape[-1])
    outs = []
    for (w, a, b, s) in (q, k, v):
        outs.append(lora_linear(xf, cast(w), cast(a), cast(b), s, store_dtype)
                    .view(*x.shape[:-1], -1))
    return tuple(outs)


def lora_qkv_backward(x, q, k, v, dq, dk, dv, dtype=None, store_dtype=None):
    """ops/fused_lora.py:121-171.  Returns (dX, [(dA, dB) for q, k, v])."""
    cast = (lambda t: t) if dtype is None else (lambda t: t.to(dtype))
    xf = cast(x).reshape(-1, x.shape[-1])
    dx = None
    grads = []
    for (w, a, b, s), dy in zip((q, k, v), (dq, dk, dv)):
        dyf = cast(dy).reshape(-1, dy.shape[-1])
        grads.append(_lora_grads(dyf, xf, cast(a), cast(b), s, store_dtype))
        term = _lora_dx(dyf, cast(w), cast(a), cast(b), s, store_dtype)
        dx = term if dx is None else dx + term
    return dx.view(*x.shape), grads


def lora_w_forward(x, p, dtype=None, store_dtype=None):
    """One LoRA projection p = (W, A, B, s) of x: the per-projection step of
    ops/fused_lora.py:96-119 (the single-projection form of ops/fused_lora.py:26)."""
    return lora_qkv_forward(x, p, p, p, dtype, store_dtype)[0]


def lora_w_backward(x, p, dy, dtype=None, store_dtype=None):
    """Backward of lora_w_forward: the per-projection terms of
    ops/fused_lora.py:142-161.  Returns (dX, (dA, dB))."""
    cast = (lambda t: t) if dtype is None else (lambda t: t.to(dtype))
    w, a, b, s = p
    xf = cast(x).reshape(-1, x.shape[-1])
    dyf = cast(dy).reshape(-1, dy.shape[-1])
    da, db = _lora_grads(dyf, xf, cast(a), cast(b), s, store_dtype)
    dx = _lora_dx(dyf, cast(w), cast(a), cast(b), s, store_dtype)
    return dx.view(*x.shape), (da, db)


def lora_mlp_forward(x, g, u, d, dtype=None, store_dtype=None):
    """ops/fused_lora.py:182-207: gate/up LoRA linears, h = silu(gate)*up (fp32 math,
    cast to x dtype), down LoRA linear.  Returns (out, gate, up, h)."""
    cast = (lambda t: t) if dtype is None else (lambda t: t.to(dtype))
    xf = cast(x).reshape(-1, x.shape[-1])
    gw, ga, gb, gs = g
    uw, ua, ub, us = u
    dw, da, db, ds = d
    gate = _store(lora_linear(xf, cast(gw), cast(ga), cast(gb), gs, store_dtype), store_dtype)
    up = _store(lora_linear(xf, cast(uw), cast(ua), cast(ub), us, store_dtype), store_dtype)
    gf = gate.float()
    h = _store((gf * torch.sigmoid(gf) * up.float()).to(xf.dtype), store_dtype)
    out = lora_linear(h, cast(dw), cast(da), cast(db), ds, store_dtype)
    return out.view(*x.shape[:-1], -1), gate, up, h


def lora_mlp_backward(x, g, u, d, dy, dtype=None, store_dtype=None):
    """ops/fused_lora.py:209-266.  Returns (dX, [(dA, dB) for gate, up, down])."""
    cast = (lambda t: t) if dtype is None else (lambda t: t.to(dtype))
    _, gate, up, h = lora_mlp_forward(x, g, u, d, dtype, store_dtype)
    xf = cast(x).reshape(-1, x.shape[-1])
    dyf = cast(dy).reshape(-1, dy.shape[-1])
    gw, ga, gb, gs = (cast(t) if torch.is_tensor(t) else t for t in g)
    uw, ua, ub, us = (cast(t) if torch.is_tensor(t) else t for t in u)
    dw, da, db, ds = (cast(t) if torch.is_tensor(t) else t for t in d)
    dt = dyf.dtype
    d_da, d_db = _lora_grads(dyf, h, da, db, ds, store_dtype)
    dh = _store(dyf @ dw + _store(dyf @ db.to(dt), store_dtype) @ da.to(dt) * ds, store_dtype)
    gf, uf = gate.float(), up.float()
    sg = torch.sigmoid(gf)
    dhf = dh.float()
    d_gate = _store((dhf * uf * sg * (1.0 + gf * (1.0 - sg))).to(dt), store_dtype)
    d_up = _store((dhf * (gf * sg)).to(dt), store_dtype)
    g_grads = _lora_grads(d_gate, xf, ga, gb, gs, store_dtype)
    u_grads = _lora_grads(d_up, xf, ua, ub, us, store_dtype)
    dx = _lora_dx(d_gate, gw, ga, gb, gs, store_dtype) + \
        _lora_dx(d_up, uw, ua, ub, us, store_dtype)
    return dx.view(*x.shape), [g_grads, u_grads, (d_da, d_db)]


def flops_flce(n, h, v):
    """Algorithmic FLOPs of one FLCE fwd+bwd (logits, dX, dW GEMMs once each)."""
    return 6.0 * n * h * v


def ceil_div(a, b):
    return -(-a // b)


__all__ = [name for name in dir() if not name.startswith("_") and name not in ("math", "torch")]
