"""Patcher structure on CPU: the same modules are swapped as in the reference, and
state_dict keys and values are unchanged (checkpoint compatibility)."""

import torch

from metal_liger_b200 import apply_metal_liger_to_qwen3vl
from metal_liger_b200.ops.fused_rms_norm import MetalLigerRMSNorm
from metal_liger_b200.ops.fused_swiglu import MetalLigerSwiGLU
from metal_liger_b200.patch import _find_layers
from peft_stub import make_model


def test_patch_counts_and_state_dict_unchanged(caplog):
    model = make_model(n_layers=3)
    before = {k: v.clone() for k, v in model.state_dict().items()}
    caplog.set_level("INFO")
    out = apply_metal_liger_to_qwen3vl(model)
    assert out is model
    after = model.state_dict()
    assert list(before) == list(after)
    for k in before:
        assert torch.equal(before[k], after[k]), k
    layers = _find_layers(model)
    assert len(layers) == 3
    for layer in layers:
        assert isinstance(layer.input_layernorm, MetalLigerRMSNorm)
        assert isinstance(layer.post_attention_layernorm, MetalLigerRMSNorm)
        assert isinstance(layer.mlp, MetalLigerSwiGLU)
        assert getattr(layer.self_attn, "_metal_liger_fused_lora", False)
        assert getattr(layer.mlp, "_metal_liger_fused_lora", False)
    assert isinstance(model.base_model.model.model.language_model.norm, MetalLigerRMSNorm)
    text = caplog.text
    assert "replaced 7 RMSNorm" in text and "replaced 3 MLP" in text
    assert "fused LoRA QKV+MLP on 6 modules" in text


def test_rms_norm_shares_weight_storage():
    model = make_model(n_layers=1)
    w = model.base_model.model.model.language_model.layers[0].input_layernorm.weight
    apply_metal_liger_to_qwen3vl(model, fuse_swiglu=False, fuse_lora=False)
    w2 = model.base_model.model.model.language_model.layers[0].input_layernorm.weight
    assert w2.data_ptr() == w.data_ptr()


def test_flags_off_leave_model_alone():
    model = make_model(n_layers=1)
    apply_metal_liger_to_qwen3vl(model, fuse_rms_norm=False, fuse_swiglu=False, fuse_lora=False,
                                 fuse_rope=True, fuse_cross_entropy=True)
    layer = model.base_model.model.model.language_model.layers[0]
    assert not isinstance(layer.input_layernorm, MetalLigerRMSNorm)
    assert not hasattr(layer.self_attn, "_metal_liger_fused_lora")


def test_non_peft_model_paths():
    model = make_model(n_layers=2).base_model.model  # bare Qwen3-VL-shaped model
    apply_metal_liger_to_qwen3vl(model, fuse_lora=False)
    assert isinstance(model.model.language_model.norm, MetalLigerRMSNorm)


def test_extension_flags_on_hf_qwen3vl_text_model():
    """The keyword-only B200 extensions on transformers' Qwen3VLTextModel (CPU,
    structure only): q/k norms swapped, o_proj routed through _LoRA_W, the
    attention module's rotary function rebound (and restored here)."""
    import sys

    from transformers.models.qwen3_vl.configuration_qwen3_vl import Qwen3VLTextConfig
    from transformers.models.qwen3_vl.modeling_qwen3_vl import Qwen3VLTextModel

    from metal_liger_b200.lora_adapters import LoraLinear, inject_lora, lora_parameters

    cfg = Qwen3VLTextConfig(hidden_size=64, intermediate_size=128, num_hidden_layers=2,
                            num_attention_heads=2, num_key_value_heads=1, head_dim=32,
                            vocab_size=100)
    holder = torch.nn.Module()
    holder.model = Qwen3VLTextModel(cfg)
    assert inject_lora(holder, r=4, alpha=8) == 14
    assert len(lora_parameters(holder)) == 28
    assert all(not p.requires_grad for n, p in holder.named_parameters() if "lora_" not in n)
    keys = set(holder.state_dict())
    mod = sys.modules[type(holder.model.layers[0].self_attn).__module__]
    original = mod.apply_rotary_pos_emb
    try:
        apply_metal_liger_to_qwen3vl(holder, fuse_qk_norm=True, fuse_rope_in_attention=True,
                                     fuse_lora_o_proj=True)
        assert mod.apply_rotary_pos_emb is not original
        assert mod._metal_liger_original_rope is original
    finally:
        mod.apply_rotary_pos_emb = original
    for layer in holder.model.layers:
        assert isinstance(layer.self_attn.q_norm, MetalLigerRMSNorm)
        assert isinstance(layer.self_attn.k_norm, MetalLigerRMSNorm)
        assert isinstance(layer.self_attn.o_proj, LoraLinear)
        assert layer.self_attn.o_proj._metal_liger_fused_lora
        assert isinstance(layer.mlp, MetalLigerSwiGLU)
    assert isinstance(holder.model.norm, MetalLigerRMSNorm)
    assert set(holder.state_dict()) == keys
