"""The patcher on the real HuggingFace Qwen3-VL text decoder (transformers'
``Qwen3VLTextModel``, random init, small shape): loss and LoRA gradients of
the patched model agree with the unpatched one.

Both runs are bf16 end to end; they round at different points (fused kernels
keep fp32 inside each op), so the comparison is at bf16 tolerance: the loss
within 1e-2 relative, every LoRA gradient within 5e-2 relative Frobenius.
"""

import copy
import sys

import pytest
import torch
import torch.nn as nn

pytestmark = pytest.mark.gpu
DEV = "cuda"


class _CausalLM(nn.Module):
    """HF CausalLM nesting (``model.model.layers``, ``model.model.norm``)."""

    def __init__(self, text_model, vocab, hidden):
        super().__init__()
        self.model = text_model
        self.lm_head = nn.Linear(hidden, vocab, bias=False, device=DEV, dtype=torch.bfloat16)


def _build(seed=0, layers=2):
    from transformers.models.qwen3_vl.configuration_qwen3_vl import Qwen3VLTextConfig
    from transformers.models.qwen3_vl.modeling_qwen3_vl import Qwen3VLTextModel

    from metal_liger_b200.lora_adapters import inject_lora

    cfg = Qwen3VLTextConfig(hidden_size=256, intermediate_size=512, num_hidden_layers=layers,
                            num_attention_heads=4, num_key_value_heads=2, head_dim=64,
                            vocab_size=1000, rms_norm_eps=1e-6,
                            rope_parameters={"rope_type": "default", "rope_theta": 5e6,
                                             "mrope_section": [12, 10, 10]})
    cfg._attn_implementation = "sdpa"
    torch.manual_seed(seed)
    with torch.device(DEV):
        text = Qwen3VLTextModel(cfg).to(torch.bfloat16)
    model = _CausalLM(text, 1000, 256)
    n = inject_lora(model, r=16, alpha=32, init_std=0.05)
    assert n == 7 * layers
    return model


def _run(model, ids, labels, fused_loss):
    from metal_liger_b200.lora_adapters import lora_parameters
    from metal_liger_b200.ops.fused_linear_cross_entropy import MetalLigerFusedLinearCrossEntropy

    h = model.model(input_ids=ids, use_cache=False).last_hidden_state
    w = model.lm_head.weight
    if fused_loss:
        loss = MetalLigerFusedLinearCrossEntropy(model.lm_head, ignore_index=-100)(h, labels)
    else:
        logits = h.float() @ w.float().t()
        loss = torch.nn.functional.cross_entropy(logits.view(-1, logits.shape[-1]),
                                                 labels.view(-1), ignore_index=-100)
    loss.backward()
    grads = {n: p.grad.float().clone() for n, p in model.named_parameters() if p.requires_grad}
    assert len(grads) == len(lora_parameters(model))
    return loss.detach().float().item(), grads


def test_patched_qwen3vl_text_decoder_matches_unpatched():
    from metal_liger_b200 import apply_metal_liger_to_qwen3vl

    base = _build()
    patched = copy.deepcopy(base)
    g = torch.Generator(device=DEV).manual_seed(3)
    ids = torch.randint(0, 1000, (2, 96), generator=g, device=DEV)
    labels = torch.roll(ids, -1, dims=1)
    labels[:, -1] = -100
    ref_loss, ref_grads = _run(base, ids, labels, fused_loss=False)

    attn_mod = sys.modules[type(base.model.layers[0].self_attn).__module__]
    original_rope = attn_mod.apply_rotary_pos_emb
    try:
        apply_metal_liger_to_qwen3vl(patched, fuse_qk_norm=True, fuse_rope_in_attention=True,
                                     fuse_lora_o_proj=True)
        # As in the reference (patch.py:110-114), replacement norms wrap the old
        # weight's data in a new Parameter, which is trainable; freeze them again
        # so both runs train the same adapter set.
        for n, p in patched.named_parameters():
            if "lora_" not in n:
                p.requires_grad_(False)
        from metal_liger_b200.ops.fused_rms_norm import MetalLigerRMSNorm
        layer = patched.model.layers[0]
        assert isinstance(layer.input_layernorm, MetalLigerRMSNorm)
        assert isinstance(layer.self_attn.q_norm, MetalLigerRMSNorm)
        assert isinstance(patched.model.norm, MetalLigerRMSNorm)
        assert getattr(layer.self_attn, "_metal_liger_fused_lora", False)
        assert getattr(layer.self_attn.o_proj, "_metal_liger_fused_lora", False)
        assert attn_mod.apply_rotary_pos_emb is not original_rope
        loss, grads = _run(patched, ids, labels, fused_loss=True)
    finally:
        attn_mod.apply_rotary_pos_emb = original_rope

    assert abs(loss - ref_loss) <= 1e-2 * abs(ref_loss), (loss, ref_loss)
    assert ref_grads.keys() == grads.keys()
    for name, ref in ref_grads.items():
        got = grads[name]
        rel = ((got - ref).norm() / ref.norm().clamp(min=1e-30)).item()
        assert rel <= 5e-2, f"{name}: relative Frobenius error {rel:.3e}"


def _build_vl(seed=0, layers=2, vocab=32000):
    """A small transformers Qwen3VLForConditionalGeneration (text decoder +
    a one-block vision tower that text-only inputs never run), bf16, with
    PEFT-layout LoRA on the decoder's q/k/v/o/gate/up/down."""
    from transformers.models.qwen3_vl.configuration_qwen3_vl import Qwen3VLConfig
    from transformers.models.qwen3_vl.modeling_qwen3_vl import Qwen3VLForConditionalGeneration

    from metal_liger_b200.lora_adapters import inject_lora

    cfg = Qwen3VLConfig(
        text_config=dict(hidden_size=256, intermediate_size=512, num_hidden_layers=layers,
                         num_attention_heads=4, num_key_value_heads=2, head_dim=64,
                         vocab_size=vocab, rms_norm_eps=1e-6,
                         rope_parameters={"rope_type": "default", "rope_theta": 5e6,
                                          "mrope_section": [12, 10, 10]}),
        vision_config=dict(depth=1, hidden_size=64, intermediate_size=128, num_heads=2,
                           out_hidden_size=256, deepstack_visual_indexes=[0]))
    cfg._attn_implementation = "sdpa"
    torch.manual_seed(seed)
    with torch.device(DEV):
        model = Qwen3VLForConditionalGeneration(cfg).to(torch.bfloat16)
    assert inject_lora(model, r=16, alpha=32, init_std=0.05) == 7 * layers
    return model


def _train_once(model, ids, labels):
    from metal_liger_b200.lora_adapters import lora_parameters

    model.train()
    torch.cuda.synchronize()
    base = torch.cuda.memory_allocated()
    torch.cuda.reset_peak_memory_stats()
    out = model(input_ids=ids, labels=labels)
    out.loss.backward()
    torch.cuda.synchronize()
    peak = torch.cuda.max_memory_allocated() - base
    grads = {n: p.grad.float().clone() for n, p in model.named_parameters() if p.requires_grad}
    assert len(grads) == len(lora_parameters(model))
    return out, grads, peak


def test_fuse_cross_entropy_matches_hf_loss_and_lowers_peak_memory():
    """fuse_cross_entropy=True: model(input_ids, labels=...) takes its loss from
    the fused linear cross-entropy (HF's shift, ignore_index -100) and never
    forms the [B*S, V] logits.  Loss within 1e-2 relative and LoRA gradients
    within 5e-2 relative Frobenius of the unpatched HF model (both bf16); the
    step's peak device memory is lower."""
    from metal_liger_b200 import apply_metal_liger_to_qwen3vl

    base = _build_vl()
    patched = copy.deepcopy(base)
    g = torch.Generator(device=DEV).manual_seed(4)
    ids = torch.randint(0, 32000, (2, 512), generator=g, device=DEV)
    labels = ids.clone()
    labels[:, :16] = -100  # e.g. a masked prompt
    ref_out, ref_grads, ref_peak = _train_once(base, ids, labels)
    assert ref_out.logits is not None

    attn_mod = sys.modules[type(base.model.language_model.layers[0].self_attn).__module__]
    original_rope = attn_mod.apply_rotary_pos_emb
    try:
        apply_metal_liger_to_qwen3vl(patched, fuse_cross_entropy=True, fuse_qk_norm=True,
                                     fuse_rope_in_attention=True, fuse_lora_o_proj=True)
        for n, p in patched.named_parameters():
            if "lora_" not in n:
                p.requires_grad_(False)
        out, grads, peak = _train_once(patched, ids, labels)
    finally:
        attn_mod.apply_rotary_pos_emb = original_rope
    assert out.logits is None
    loss, ref_loss = out.loss.float().item(), ref_out.loss.float().item()
    assert abs(loss - ref_loss) <= 1e-2 * abs(ref_loss), (loss, ref_loss)
    assert ref_grads.keys() == grads.keys()
    for name, ref in ref_grads.items():
        rel = ((grads[name] - ref).norm() / ref.norm().clamp(min=1e-30)).item()
        assert rel <= 5e-2, f"{name}: relative Frobenius error {rel:.3e}"
    # HF's loss holds the bf16 logits, their fp32 copy and the softmax
    # gradient ([1024, 32000] each); the fused op holds none of them
    assert peak < ref_peak - 100 * 2**20, (peak, ref_peak)
