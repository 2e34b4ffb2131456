"""Fused LoRA QKV + MLP on B200 — drop-in for the reference's ops/fused_lora.py.

Same public names, signatures and results as the reference
(ops/fused_lora.py:43-421): ``_get_lora_params``, ``_lora_linear``,
``_LoRA_QKV.apply(X, QW,QA,QB,QS, KW,KA,KB,KS, VW,VA,VB,VS)``,
``_LoRA_MLP.apply(X, GW,GA,GB,GS, UW,UA,UB,US, DW,DA,DB,DS)``,
``apply_fused_lora_qkv``, ``apply_fused_lora_mlp`` and ``patch_fused_lora``;
plus ``_LoRA_W`` / ``apply_fused_lora_linear`` for a single LoRA projection.

Each Function is two ``metal_liger::`` ops (forward, backward) that run every
product on the tcgen05 GEMM: the rank-r update is an extra K-segment of the
base-weight GEMM (one TMEM accumulator per output tile), dX for Q/K/V (or
gate/up) is ONE GEMM over the concatenated K dimension, and the A/B
gradients are split-K GEMMs over the tokens.  X is saved once (as in the
reference), plus the tiny [tokens, 64] rank projections so the backward does
not recompute them.  A/B gradients are accumulated in fp32 and returned in
the adapters' own dtype — the value autograd assigns after the reference's
fp32 ``.float()`` result, without a separate cast kernel per adapter; the
frozen base weights get no gradient.
"""

import logging
import types

import torch
import torch.nn as nn

import metal_liger_b200._torch_library  # noqa: F401  (registers metal_liger:: ops)

logger = logging.getLogger(__name__)


def _get_lora_params(linear):
    """(W, A, B, scaling) of the first adapter of a PEFT LoRA Linear, else 4 Nones
    (reference ops/fused_lora.py:43-66)."""
    if not hasattr(linear, "lora_A"):
        return None, None, None, None
    adapters = list(linear.lora_A.keys())
    if not adapters:
        return None, None, None, None
    name = adapters[0]
    W = linear.base_layer.weight if hasattr(linear, "base_layer") else linear.weight
    A = linear.lora_A[name].weight
    B = linear.lora_B[name].weight
    return W, A, B, linear.scaling[name]


def _lora_linear(X, W, A, B, scaling):
    """x W^T + s (x A^T) B^T as a plain tensor expression (reference helper,
    ops/fused_lora.py:69-82).  The fused Functions below do not use it."""
    import torch.nn.functional as F

    out = F.linear(X, W)
    if A is not None and B is not None:
        out = out + F.linear(F.linear(X, A.to(X.dtype)), B.to(X.dtype)) * scaling
    return out


def _zeros_for(grad, ref):
    return torch.zeros_like(ref) if grad is None else grad


class _LoRA_QKV(torch.autograd.Function):
    """Q, K, V LoRA projections of one input; X saved once for all three."""

    @staticmethod
    def forward(ctx, X, QW, QA, QB, QS, KW, KA, KB, KS, VW, VA, VB, VS):
        scal = [float(QS), float(KS), float(VS)]
        Q, K, V, U = torch.ops.metal_liger.lora_qkv_forward(X, QW, QA, QB, KW, KA, KB, VW, VA, VB,
                                                            scal)
        ctx.save_for_backward(X, U, QW, QA, QB, KW, KA, KB, VW, VA, VB)
        ctx.scal = scal
        lead = X.shape[:-1]
        return Q.view(*lead, -1), K.view(*lead, -1), V.view(*lead, -1)

    @staticmethod
    def backward(ctx, dQ, dK, dV):
        X, U, QW, QA, QB, KW, KA, KB, VW, VA, VB = ctx.saved_tensors
        lead = X.shape[:-1]
        dQ = _zeros_for(dQ, torch.empty(*lead, QW.shape[0], dtype=X.dtype, device=X.device))
        dK = _zeros_for(dK, torch.empty(*lead, KW.shape[0], dtype=X.dtype, device=X.device))
        dV = _zeros_for(dV, torch.empty(*lead, VW.shape[0], dtype=X.dtype, device=X.device))
        dX, dQA, dQB, dKA, dKB, dVA, dVB = torch.ops.metal_liger.lora_qkv_backward(
            X, U, QW, QA, QB, KW, KA, KB, VW, VA, VB, ctx.scal, dQ, dK, dV)
        return (dX,
                None, dQA, dQB, None,
                None, dKA, dKB, None,
                None, dVA, dVB, None)


class _LoRA_MLP(torch.autograd.Function):
    """gate/up/down LoRA SwiGLU MLP; saves X, gate, up, h (as the reference)."""

    @staticmethod
    def forward(ctx, X, GW, GA, GB, GS, UW, UA, UB, US, DW, DA, DB, DS):
        scal = [float(GS), float(US), float(DS)]
        out, gate, up, h, u1, u2 = torch.ops.metal_liger.lora_mlp_forward(
            X, GW, GA, GB, UW, UA, UB, DW, DA, DB, scal)
        ctx.save_for_backward(X, gate, up, h, u1, u2, GW, GA, GB, UW, UA, UB, DW, DA, DB)
        ctx.scal = scal
        return out

    @staticmethod
    def backward(ctx, dY):
        (X, gate, up, h, u1, u2, GW, GA, GB, UW, UA, UB, DW, DA, DB) = ctx.saved_tensors
        dX, dGA, dGB, dUA, dUB, dDA, dDB = torch.ops.metal_liger.lora_mlp_backward(
            X, gate, up, h, u1, u2, GW, GA, GB, UW, UA, UB, DW, DA, DB, ctx.scal, dY)
        return (dX,
                None, dGA, dGB, None,
                None, dUA, dUB, None,
                None, dDA, dDB, None)


class _LoRA_W(torch.autograd.Function):
    """One LoRA linear y = X W^T + s (X A^T) B^T with the rank term folded into
    the base GEMM (the single-projection form the reference describes as
    "LoRA_W", ops/fused_lora.py:26, and leaves to PEFT).  Saves X and the
    [tokens, 64] rank projection; A/B gradients in the adapters' dtype
    (fp32 accumulation), W frozen."""

    @staticmethod
    def forward(ctx, X, W, A, B, S):
        s = float(S)
        Y, U = torch.ops.metal_liger.lora_linear_forward(X, W, A, B, s)
        ctx.save_for_backward(X, U, W, A, B)
        ctx.s = s
        return Y.view(*X.shape[:-1], -1)

    @staticmethod
    def backward(ctx, dY):
        X, U, W, A, B = ctx.saved_tensors
        dX, dA, dB = torch.ops.metal_liger.lora_linear_backward(X, U, W, A, B, ctx.s,
                                                                dY.contiguous())
        return dX, None, dA, dB, None


def apply_fused_lora_linear(linear, X: torch.Tensor) -> torch.Tensor:
    """A single PEFT LoRA linear (e.g. o_proj) through one fused op; falls back
    to the module itself when it carries no adapter."""
    W, A, B, S = _get_lora_params(linear)
    if A is None:
        return linear(X)
    return _LoRA_W.apply(X, W, A, B, S)


def apply_fused_lora_qkv(attn_module, X: torch.Tensor):
    """(Q, K, V) of an attention module's q/k/v_proj in one fused op; falls back
    to the modules themselves when any projection is not LoRA
    (reference ops/fused_lora.py:269-295)."""
    QW, QA, QB, QS = _get_lora_params(attn_module.q_proj)
    KW, KA, KB, KS = _get_lora_params(attn_module.k_proj)
    VW, VA, VB, VS = _get_lora_params(attn_module.v_proj)
    if QA is None or KA is None or VA is None:
        return attn_module.q_proj(X), attn_module.k_proj(X), attn_module.v_proj(X)
    return _LoRA_QKV.apply(X, QW, QA, QB, QS, KW, KA, KB, KS, VW, VA, VB, VS)


def apply_fused_lora_mlp(mlp_module, X: torch.Tensor) -> torch.Tensor:
    """down(silu(gate(X)) * up(X)) with all three LoRA projections fused; falls
    back to the module when any projection is not LoRA
    (reference ops/fused_lora.py:298-320)."""
    GW, GA, GB, GS = _get_lora_params(mlp_module.gate_proj)
    UW, UA, UB, US = _get_lora_params(mlp_module.up_proj)
    DW, DA, DB, DS = _get_lora_params(mlp_module.down_proj)
    if GA is None or UA is None or DA is None:
        return mlp_module(X)
    return _LoRA_MLP.apply(X, GW, GA, GB, GS, UW, UA, UB, US, DW, DA, DB, DS)


def _find_layers_list(module, depth=0):
    """First child named 'layers' with children, searched up to 6 levels deep
    (reference ops/fused_lora.py:347-356)."""
    if depth > 6:
        return None
    for name, child in module.named_children():
        if name == "layers" and len(list(child.children())) > 0:
            return child
        found = _find_layers_list(child, depth + 1)
        if found is not None:
            return found
    return None


def _has_lora(module, names):
    return all(hasattr(module, n) and _get_lora_params(getattr(module, n))[1] is not None
               for n in names)


def patch_fused_lora(model: nn.Module, fuse_o_proj: bool = False) -> int:
    """Route every decoder layer's q/k/v and gate/up/down LoRA projections
    through the fused Functions (reference ops/fused_lora.py:323-421).
    ``fuse_o_proj=True`` (a B200 extension, off by default as in the
    reference) also routes a LoRA ``o_proj`` through ``_LoRA_W``.

    The module tree is not modified: the attention forward is wrapped so that,
    for the duration of one call, q_proj/k_proj/v_proj are shadowed in the
    instance ``__dict__`` by callables returning the fused results (Python
    finds ``__dict__`` before ``_modules``); the MLP's ``forward`` is replaced
    on the instance.  ``state_dict`` keys and values are unchanged.  Returns
    the number of patched modules.
    """
    # A PEFT wrapper's HF model (reference ops/fused_lora.py:344).  A plain HF
    # PreTrainedModel also has ``base_model`` (its inner backbone, without a
    # ``.model``): search it from the model itself then.
    base = getattr(getattr(model, "base_model", None), "model", None) or model
    layers = _find_layers_list(base)
    if layers is None:
        logger.warning("MetalLiger fused LoRA: could not find transformer layers")
        return 0
    patched = 0
    for layer in layers:
        attn = getattr(layer, "self_attn", None)
        mlp = getattr(layer, "mlp", None)
        if attn is not None and _has_lora(attn, ("q_proj", "k_proj", "v_proj")):
            original = attn.forward

            def fused_attn_forward(self_attn, hidden_states, *args, _orig=original, **kwargs):
                q, k, v = apply_fused_lora_qkv(self_attn, hidden_states)
                self_attn.__dict__["q_proj"] = lambda _x, _t=q: _t
                self_attn.__dict__["k_proj"] = lambda _x, _t=k: _t
                self_attn.__dict__["v_proj"] = lambda _x, _t=v: _t
                try:
                    return _orig(hidden_states, *args, **kwargs)
                finally:
                    for n in ("q_proj", "k_proj", "v_proj"):
                        self_attn.__dict__.pop(n, None)

            attn.forward = types.MethodType(fused_attn_forward, attn)
            attn._metal_liger_fused_lora = True
            patched += 1
        o_proj = getattr(attn, "o_proj", None) if attn is not None else None
        if fuse_o_proj and o_proj is not None and _get_lora_params(o_proj)[1] is not None:
            def fused_o_forward(self_linear, x):
                return apply_fused_lora_linear(self_linear, x)

            o_proj.forward = types.MethodType(fused_o_forward, o_proj)
            o_proj._metal_liger_fused_lora = True
            patched += 1
        if mlp is not None and _has_lora(mlp, ("gate_proj", "up_proj", "down_proj")):
            def fused_mlp_forward(self_mlp, x):
                return apply_fused_lora_mlp(self_mlp, x)

            mlp.forward = types.MethodType(fused_mlp_forward, mlp)
            mlp._metal_liger_fused_lora = True
            patched += 1
    logger.info("MetalLiger fused LoRA: activated on %d modules", patched)
    return patched
