"""Model patching for HuggingFace Qwen3-VL-style models — drop-in for patch.py.

``apply_metal_liger_to_qwen3vl(model, fuse_rms_norm=True, fuse_swiglu=True,
fuse_rope=False, fuse_cross_entropy=False, fuse_lora=True,
use_optimized_generator=False)`` keeps the reference's signature, flags and
behaviour (reference patch.py:181-240):

* every decoder layer's ``input_layernorm`` / ``post_attention_layernorm`` and
  the final norm become ``MetalLigerRMSNorm`` sharing the original weight
  storage (so ``state_dict`` keys and values are unchanged);
* every MLP with a ``gate_proj`` is wrapped in ``MetalLigerSwiGLU``;
* PEFT LoRA projections are routed through the fused LoRA Functions by
  ``patch_fused_lora`` (which never touches ``_modules``);
* ``fuse_rope`` only logs that the fused functions are available
  (``apply_fused_rotary*``), as the reference does;
* ``fuse_cross_entropy`` (the reference only logs it) routes the causal-LM
  loss through ``MetalLigerFusedLinearCrossEntropy``: in training mode, when
  ``labels`` are given, the model's forward runs with its ``lm_head`` shadowed
  by a capture of the hidden states, and the loss over HF's shifted labels
  (``ignore_index=-100``) comes from the fused op, so the ``[B*S, V]`` logits
  are never formed (the output's ``logits`` is None).

Layers are located through the same PEFT / VL nesting paths the reference
tries (patch.py:27-89).
"""

import inspect
import logging
import types

import torch
import torch.nn as nn
import torch.nn.functional as F

from metal_liger_b200.generation import patch_generator
from metal_liger_b200.ops.fused_lora import patch_fused_lora
from metal_liger_b200.ops.fused_rms_norm import MetalLigerRMSNorm
from metal_liger_b200.ops.fused_rope import apply_fused_rotary
from metal_liger_b200.ops.fused_swiglu import MetalLigerSwiGLU

logger = logging.getLogger(__name__)


def _walk(obj, path):
    for name in path:
        obj = getattr(obj, name, None)
        if obj is None:
            return None
    return obj


# Attribute paths to the decoder layer list, most specific first
# (reference patch.py:36-54).
_LAYER_PATHS = (
    ("base_model", "model", "model", "language_model", "layers"),
    ("base_model", "model", "model", "layers"),
    ("model", "language_model", "layers"),
    ("model", "layers"),
    ("layers",),
    ("module", "model", "layers"),
)

# Parents of the final norm (reference patch.py:69-81 and :146-154).
_NORM_PARENTS = (
    ("base_model", "model", "model", "language_model"),
    ("model", "language_model"),
    ("base_model", "model", "model"),
    ("model",),
)


def _find_layers(model: nn.Module):
    for path in _LAYER_PATHS:
        try:
            layers = _walk(model, path)
            if layers is not None and len(layers) > 0:
                return layers
        except (AttributeError, TypeError):
            continue
    return None


def _find_final_norm(model: nn.Module):
    """(parent, norm) of the final RMSNorm, or (None, None)."""
    for path in _NORM_PARENTS:
        parent = _walk(model, path)
        norm = getattr(parent, "norm", None) if parent is not None else None
        if norm is not None and hasattr(norm, "weight"):
            return parent, norm
    return None, None


def _fused_norm_like(old: nn.Module) -> MetalLigerRMSNorm:
    eps = getattr(old, "variance_epsilon", getattr(old, "eps", 1e-6))
    return MetalLigerRMSNorm(hidden_size=old.weight.shape[0], eps=eps, weight=old.weight.data)


def _replace_rms_norms(model: nn.Module) -> int:
    layers = _find_layers(model)
    if layers is None:
        logger.warning("MetalLiger: could not find transformer layers for RMSNorm patching")
        return 0
    count = 0
    for layer in layers:
        for attr in ("input_layernorm", "post_attention_layernorm"):
            if hasattr(layer, attr):
                setattr(layer, attr, _fused_norm_like(getattr(layer, attr)))
                count += 1
    parent, norm = _find_final_norm(model)
    if parent is not None:
        parent.norm = _fused_norm_like(norm)
        count += 1
    return count


def _replace_mlps(model: nn.Module) -> int:
    layers = _find_layers(model)
    if layers is None:
        return 0
    count = 0
    for layer in layers:
        if hasattr(layer, "mlp") and hasattr(layer.mlp, "gate_proj"):
            layer.mlp = MetalLigerSwiGLU(layer.mlp)
            count += 1
    return count


def _replace_qk_norms(model: nn.Module) -> int:
    """Per-head q_norm / k_norm of every attention block -> MetalLigerRMSNorm."""
    layers = _find_layers(model)
    if layers is None:
        return 0
    count = 0
    for layer in layers:
        attn = getattr(layer, "self_attn", None)
        for attr in ("q_norm", "k_norm"):
            norm = getattr(attn, attr, None) if attn is not None else None
            if norm is not None and hasattr(norm, "weight"):
                setattr(attn, attr, _fused_norm_like(norm))
                count += 1
    return count


def _fused_rotary_pos_emb(q, k, cos, sin, position_ids=None, unsqueeze_dim=1):
    """HF ``apply_rotary_pos_emb`` signature, computed by the fused RoPE kernel
    (q and k in one launch; strided [B, H, S, D] views read in place)."""
    return apply_fused_rotary(q, k, cos.unsqueeze(unsqueeze_dim), sin.unsqueeze(unsqueeze_dim))


def _patch_attention_rope(model: nn.Module) -> int:
    """Rebind ``apply_rotary_pos_emb`` in the modeling module(s) of the model's
    attention classes to the fused kernel.  Returns the number of modules
    rebound (the originals are kept as ``_metal_liger_original_rope``)."""
    import sys

    layers = _find_layers(model)
    if layers is None:
        return 0
    done = 0
    seen = set()
    for layer in layers:
        attn = getattr(layer, "self_attn", None)
        if attn is None:
            continue
        mod = sys.modules.get(type(attn).__module__)
        if mod is None or id(mod) in seen or not hasattr(mod, "apply_rotary_pos_emb"):
            continue
        seen.add(id(mod))
        if getattr(mod, "apply_rotary_pos_emb") is not _fused_rotary_pos_emb:
            mod._metal_liger_original_rope = mod.apply_rotary_pos_emb
            mod.apply_rotary_pos_emb = _fused_rotary_pos_emb
        done += 1
    return done


def restore_attention_rope(model: nn.Module) -> int:
    """Undo ``fuse_rope_in_attention``: put back the modeling module's original
    ``apply_rotary_pos_emb``.  The rebinding is per modeling module, so it also
    reaches other models of the same class in the process; this restores them
    all.  Returns the number of modules restored."""
    import sys

    layers = _find_layers(model)
    if layers is None:
        return 0
    done = 0
    for layer in layers:
        attn = getattr(layer, "self_attn", None)
        mod = sys.modules.get(type(attn).__module__) if attn is not None else None
        orig = getattr(mod, "_metal_liger_original_rope", None) if mod is not None else None
        if orig is not None and mod.apply_rotary_pos_emb is _fused_rotary_pos_emb:
            mod.apply_rotary_pos_emb = orig
            done += 1
    return done


# Owners of the lm_head whose forward takes ``labels``: a PEFT wrapper's HF
# model, a DDP-style ``module``, or the model itself (deepest first, since
# PEFT wrappers forward unknown attributes to the model they wrap).
_LM_PATHS = (("base_model", "model"), ("module",), ())


def _find_causal_lm(model: nn.Module):
    for path in _LM_PATHS:
        obj = _walk(model, path) if path else model
        head = getattr(obj, "lm_head", None) if obj is not None else None
        if not isinstance(head, nn.Linear) or hasattr(head, "lora_A"):
            continue
        fwd = obj.__dict__.get("_metal_liger_original_forward", obj.forward)
        try:
            params = inspect.signature(fwd).parameters
        except (TypeError, ValueError):
            continue
        if "labels" in params:
            return obj
    return None


class _HiddenCapture(nn.Module):
    """Stands in for the lm_head during one forward: keeps the hidden states
    it is given and returns an empty [..., 0] tensor in place of the logits."""

    def __init__(self):
        super().__init__()
        self.hidden = None

    def forward(self, hidden_states):
        self.hidden = hidden_states
        return hidden_states.new_empty(*hidden_states.shape[:-1], 0)


def causal_lm_loss(hidden, lm_head, labels=None, shift_labels=None, num_items_in_batch=None,
                   ignore_index=-100, chunk_size=8192):
    """HF's causal-LM loss (transformers ``ForCausalLMLoss``: labels shifted by
    one, the last position ignored; a mean over the non-ignored tokens, or a
    sum divided by ``num_items_in_batch`` when that is given) computed by the
    fused linear cross-entropy from the final hidden states."""
    from metal_liger_b200.ops.fused_linear_cross_entropy import MetalLigerFusedLinearCrossEntropy

    if shift_labels is None:
        shift_labels = F.pad(labels, (0, 1), value=ignore_index)[..., 1:]
    shift_labels = shift_labels.reshape(-1).to(hidden.device)
    loss = MetalLigerFusedLinearCrossEntropy(lm_head, ignore_index=ignore_index,
                                             chunk_size=chunk_size)(
        hidden.reshape(-1, hidden.shape[-1]), shift_labels)
    if num_items_in_batch is not None:
        n_valid = (shift_labels != ignore_index).sum().to(loss.dtype)
        if torch.is_tensor(num_items_in_batch):
            num_items_in_batch = num_items_in_batch.to(loss.device)
        loss = loss * n_valid / num_items_in_batch
    return loss


def _fused_ce_forward(self, *args, **kwargs):
    """The causal LM's forward with the loss from the fused linear
    cross-entropy (training mode with labels); otherwise the original."""
    orig = self.__dict__["_metal_liger_original_forward"]
    if args:  # positional arguments by the original forward's parameter names
        sig = inspect.signature(orig)
        named = {}
        for name, val in sig.bind_partial(*args, **kwargs).arguments.items():
            kind = sig.parameters[name].kind
            if kind is inspect.Parameter.VAR_POSITIONAL:
                return orig(*args, **kwargs)
            if kind is inspect.Parameter.VAR_KEYWORD:
                named.update(val)
            else:
                named[name] = val
        kwargs = named
    labels = kwargs.get("labels")
    shift_labels = kwargs.get("shift_labels")
    keep = kwargs.get("logits_to_keep", 0)
    if (not self.training or (labels is None and shift_labels is None)
            or not (isinstance(keep, int) and keep == 0)):
        return orig(**kwargs)
    kwargs = dict(kwargs)
    kwargs["labels"] = None
    kwargs.pop("shift_labels", None)
    capture = _HiddenCapture()
    object.__setattr__(self, "lm_head", capture)  # shadows _modules["lm_head"]
    try:
        out = orig(**kwargs)
    finally:
        self.__dict__.pop("lm_head", None)
    if capture.hidden is None:
        raise RuntimeError("fuse_cross_entropy: the model's forward did not call its lm_head")
    loss = causal_lm_loss(capture.hidden, self.lm_head, labels, shift_labels,
                          kwargs.get("num_items_in_batch"))
    if isinstance(out, tuple):
        return (loss,) + tuple(out[1:])
    fields = {k: v for k, v in out.items() if k not in ("loss", "logits")}
    return type(out)(loss=loss, **fields)


def _patch_cross_entropy(model: nn.Module) -> int:
    lm = _find_causal_lm(model)
    if lm is None:
        return 0
    if "_metal_liger_original_forward" not in lm.__dict__:
        lm.__dict__["_metal_liger_original_forward"] = lm.forward
        lm.forward = types.MethodType(_fused_ce_forward, lm)
    return 1


def restore_cross_entropy(model: nn.Module) -> int:
    """Undo ``fuse_cross_entropy``: the causal LM's original forward again."""
    lm = _find_causal_lm(model)
    if lm is None or "_metal_liger_original_forward" not in lm.__dict__:
        return 0
    lm.__dict__.pop("forward", None)
    lm.__dict__.pop("_metal_liger_original_forward")
    return 1


def apply_metal_liger_to_qwen3vl(
    model: nn.Module,
    fuse_rms_norm: bool = True,
    fuse_swiglu: bool = True,
    fuse_rope: bool = False,
    fuse_cross_entropy: bool = False,
    fuse_lora: bool = True,
    use_optimized_generator: bool = False,
    *,
    fuse_qk_norm: bool = False,
    fuse_rope_in_attention: bool = False,
    fuse_lora_o_proj: bool = False,
) -> nn.Module:
    """Apply the fused B200 ops to a Qwen3-VL (or similar) model in place; returns it.

    The positional flags are the reference's.  The keyword-only flags are B200
    extensions, off by default so the default patch matches the reference:
    ``fuse_qk_norm`` swaps the per-head q_norm/k_norm for the fused RMSNorm,
    ``fuse_rope_in_attention`` rebinds the attention module's
    ``apply_rotary_pos_emb`` to the fused RoPE, and ``fuse_lora_o_proj``
    routes a LoRA o_proj through the fused single-projection op.
    """
    stats = {}
    if fuse_rms_norm:
        stats["rms_norm"] = _replace_rms_norms(model)
        logger.info("MetalLiger: replaced %d RMSNorm layers with fused versions",
                    stats["rms_norm"])
    if fuse_qk_norm:
        stats["qk_norm"] = _replace_qk_norms(model)
    if fuse_rope_in_attention:
        stats["rope_in_attention"] = _patch_attention_rope(model)
    if fuse_swiglu:
        stats["swiglu"] = _replace_mlps(model)
        logger.info("MetalLiger: replaced %d MLP layers with fused SwiGLU", stats["swiglu"])
    if fuse_lora:
        stats["fused_lora"] = patch_fused_lora(model, fuse_o_proj=fuse_lora_o_proj)
        logger.info("MetalLiger: fused LoRA QKV+MLP on %d modules", stats["fused_lora"])
    if use_optimized_generator:
        patch_generator(model)
        stats["generator"] = "optimized"
    if fuse_rope:
        logger.info("MetalLiger: fused RoPE — use apply_fused_rotary() / "
                    "apply_fused_rotary_from_positions()")
        stats["rope"] = "available"
    if fuse_cross_entropy:
        stats["cross_entropy"] = _patch_cross_entropy(model)
        if stats["cross_entropy"]:
            logger.info("MetalLiger: causal-LM loss routed through the fused linear "
                        "cross-entropy (training mode with labels)")
        else:
            logger.warning("MetalLiger: no lm_head with a labels-taking forward found; use "
                           "MetalLigerFusedLinearCrossEntropy in the trainer")
    total = sum(v for v in stats.values() if isinstance(v, int))
    logger.info("MetalLiger: %d total layers patched. Details: %s", total, stats)
    return model
