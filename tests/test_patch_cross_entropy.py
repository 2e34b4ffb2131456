"""``fuse_cross_entropy`` wiring on CPU: the patched causal LM's training loss is
HF's loss (labels shifted by one, ignore_index -100, mean over valid tokens or
sum / num_items_in_batch), computed from the captured hidden states.

The fused op needs a GPU, so here ``MetalLigerFusedLinearCrossEntropy`` is
replaced by a differentiable torch stand-in (test code, not the product); the
GPU test in test_gpu_hf_qwen3vl.py runs the real kernel.  Checked: loss and
gradients equal the unpatched model's, logits are not returned, eval mode
and label-less calls keep the original forward, the lm_head stays registered
(state_dict unchanged) and the patch can be undone.
"""

import copy

import pytest
import torch
import torch.nn as nn
import torch.nn.functional as F

V = 300


class _StandInFLCE(nn.Module):
    calls = 0

    def __init__(self, lm_head, ignore_index=-100, chunk_size=8192):
        super().__init__()
        self.lm_head = lm_head
        self.ignore_index = ignore_index

    def forward(self, hidden, labels):
        type(self).calls += 1
        logits = hidden.float() @ self.lm_head.weight.float().t()
        return F.cross_entropy(logits, labels, ignore_index=self.ignore_index)


@pytest.fixture
def stand_in(monkeypatch):
    import metal_liger_b200.ops.fused_linear_cross_entropy as flce

    _StandInFLCE.calls = 0
    monkeypatch.setattr(flce, "MetalLigerFusedLinearCrossEntropy", _StandInFLCE)
    return _StandInFLCE


def _model(seed=0):
    from transformers.models.qwen3_vl.configuration_qwen3_vl import Qwen3VLConfig
    from transformers.models.qwen3_vl.modeling_qwen3_vl import Qwen3VLForConditionalGeneration

    cfg = Qwen3VLConfig(
        text_config=dict(hidden_size=64, intermediate_size=128, num_hidden_layers=2,
                         num_attention_heads=4, num_key_value_heads=2, head_dim=16,
                         vocab_size=V, rope_parameters={"rope_type": "default",
                                                        "rope_theta": 5e6,
                                                        "mrope_section": [4, 2, 2]}),
        vision_config=dict(depth=1, hidden_size=32, intermediate_size=64, num_heads=2,
                           out_hidden_size=64, deepstack_visual_indexes=[0]))
    torch.manual_seed(seed)
    return Qwen3VLForConditionalGeneration(cfg)


def _patch(model):
    from metal_liger_b200 import apply_metal_liger_to_qwen3vl

    return apply_metal_liger_to_qwen3vl(model, fuse_rms_norm=False, fuse_swiglu=False,
                                        fuse_lora=False, fuse_cross_entropy=True)


def _data():
    g = torch.Generator().manual_seed(1)
    ids = torch.randint(0, V, (2, 10), generator=g)
    labels = ids.clone()
    labels[0, :3] = -100
    return ids, labels


def test_training_loss_and_grads_equal_hf(stand_in):
    base = _model()
    fused = _patch(copy.deepcopy(base))
    ids, labels = _data()
    base.train()
    fused.train()
    ref = base(input_ids=ids, labels=labels)
    out = fused(input_ids=ids, labels=labels)
    assert stand_in.calls == 1
    assert out.logits is None and ref.logits.shape == (2, 10, V)
    assert torch.allclose(out.loss, ref.loss, rtol=1e-6, atol=1e-7)
    ref.loss.backward()
    out.loss.backward()
    gb = dict(base.named_parameters())
    for name, p in fused.named_parameters():
        if gb[name].grad is None:
            assert p.grad is None
            continue
        assert torch.allclose(p.grad, gb[name].grad, rtol=1e-5, atol=1e-7), name


def test_positional_ids_and_num_items_in_batch(stand_in):
    base = _model()
    fused = _patch(copy.deepcopy(base))
    ids, labels = _data()
    fused.train()
    base.train()
    n_items = torch.tensor(40.0)
    out = fused(ids, labels=labels, num_items_in_batch=n_items)
    logits = base(input_ids=ids).logits
    shift = F.pad(labels, (0, 1), value=-100)[..., 1:].reshape(-1)
    ref = F.cross_entropy(logits.float().reshape(-1, V), shift, ignore_index=-100,
                          reduction="sum") / n_items
    assert stand_in.calls == 1
    assert torch.allclose(out.loss, ref, rtol=1e-5, atol=1e-7)


def test_eval_and_labelless_calls_keep_the_original_forward(stand_in):
    fused = _patch(_model())
    ids, labels = _data()
    fused.eval()
    out = fused(input_ids=ids, labels=labels)
    assert out.logits.shape == (2, 10, V) and out.loss is not None
    fused.train()
    out = fused(input_ids=ids)
    assert out.logits.shape == (2, 10, V) and out.loss is None
    assert stand_in.calls == 0


def test_state_dict_unchanged_and_restore(stand_in):
    from metal_liger_b200.patch import restore_cross_entropy

    base = _model()
    fused = _patch(copy.deepcopy(base))
    ids, labels = _data()
    fused.train()
    fused(input_ids=ids, labels=labels)
    assert "lm_head" in fused._modules and "lm_head" not in fused.__dict__
    sd0, sd1 = base.state_dict(), fused.state_dict()
    assert sd0.keys() == sd1.keys()
    for k in sd0:
        assert torch.equal(sd0[k], sd1[k]), k
    assert restore_cross_entropy(fused) == 1
    assert "forward" not in fused.__dict__
    assert fused(input_ids=ids, labels=labels).logits is not None
    assert restore_cross_entropy(fused) == 0


def test_model_without_lm_head_is_left_alone():
    from metal_liger_b200.patch import _patch_cross_entropy

    m = nn.Sequential(nn.Linear(4, 4))
    assert _patch_cross_entropy(m) == 0
    assert "forward" not in m.__dict__
