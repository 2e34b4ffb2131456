"""Static-KV generator host logic on CPU: the cache against transformers'
DynamicCache on a small Qwen3-VL text decoder, the decode loop against the
oracle's restatement of the reference loop (oracle/generation.py), and the
patch_generator / patcher-flag semantics (reference generation.py:131-164,
patch.py:221-224).

The fused greedy head is a CUDA kernel; here a test-only subclass swaps it
for torch.argmax over the same logits, so these tests check the cache and the
loop, and tests/test_gpu_generation.py checks the kernel.
"""

import pytest
import torch
import torch.nn as nn

from oracle import generation as OG


class _CausalLM(nn.Module):
    def __init__(self, text_model, vocab, hidden, dtype):
        super().__init__()
        self.model = text_model
        self.config = text_model.config
        self.lm_head = nn.Linear(hidden, vocab, bias=False, dtype=dtype)

    def generate(self, *a, **k):  # stands in for transformers' generate()
        return "original"


def _model(dtype=torch.bfloat16, layers=2, seed=0):
    from transformers.models.qwen3_vl.configuration_qwen3_vl import Qwen3VLTextConfig
    from transformers.models.qwen3_vl.modeling_qwen3_vl import Qwen3VLTextModel

    cfg = Qwen3VLTextConfig(hidden_size=128, intermediate_size=256, num_hidden_layers=layers,
                            num_attention_heads=4, num_key_value_heads=2, head_dim=32,
                            vocab_size=300, rms_norm_eps=1e-6,
                            rope_parameters={"rope_type": "default", "rope_theta": 5e6,
                                             "mrope_section": [6, 5, 5]})
    cfg._attn_implementation = "sdpa"
    torch.manual_seed(seed)
    text = Qwen3VLTextModel(cfg).to(dtype)
    m = _CausalLM(text, 300, 128, dtype)
    with torch.no_grad():
        m.lm_head.weight.normal_(0, 0.5)
    return m.eval()


class _TorchHeadGenerator:
    """MetalLigerGenerator with torch.argmax standing in for the CUDA head."""

    @staticmethod
    def make(model):
        from metal_liger_b200.generation import MetalLigerGenerator

        class G(MetalLigerGenerator):
            def _greedy(self, h):
                return torch.argmax(self.head(h), dim=-1)

            def _logits(self, h):
                return self.head(h)

        return G(model)


def test_static_cache_matches_dynamic_cache():
    from transformers.cache_utils import DynamicCache

    from metal_liger_b200.generation import MetalLigerStaticCache

    m = _model(torch.float32)
    ids = torch.randint(0, 300, (2, 7), generator=torch.Generator().manual_seed(1))
    sc = MetalLigerStaticCache(m, 2, 12)
    assert sc.key_cache.shape == (2, 2, 2, 12, 32)
    dc = DynamicCache()
    with torch.no_grad():
        a = m.model(input_ids=ids, past_key_values=sc, use_cache=True).last_hidden_state
        b = m.model(input_ids=ids, past_key_values=dc, use_cache=True).last_hidden_state
        sc.seen_tokens += 7
        assert sc.get_seq_length() == 7 and dc.get_seq_length() == 7
        torch.testing.assert_close(a, b, rtol=1e-5, atol=1e-5)
        for step in range(3):
            tok = torch.tensor([[3 + step], [11 * step]])
            a = m.model(input_ids=tok, past_key_values=sc, use_cache=True).last_hidden_state
            b = m.model(input_ids=tok, past_key_values=dc, use_cache=True).last_hidden_state
            sc.seen_tokens += 1
            torch.testing.assert_close(a, b, rtol=1e-5, atol=1e-5)
    # the filled prefix holds exactly what the dynamic cache holds
    k_dyn = dc.layers[1].keys
    torch.testing.assert_close(sc.key_cache[1, :, :, :10], k_dyn, rtol=0, atol=0)
    with pytest.raises(RuntimeError, match="exceed max_seq_len"):
        sc.update(torch.zeros(2, 2, 3, 32), torch.zeros(2, 2, 3, 32), 0)


@pytest.mark.parametrize("eos", [None, "first"])
def test_greedy_loop_matches_reference_loop(eos):
    m = _model()
    ids = torch.randint(0, 300, (2, 5), generator=torch.Generator().manual_seed(2))
    ref = OG.generate(m, ids, max_new_tokens=9)
    eos_id = None
    if eos == "first":  # stop once both rows emitted this token (rows stop together)
        eos_id = int(ref[0, 5])
        ref = OG.generate(m, ids, max_new_tokens=9, eos_token_id=eos_id)
    got = _TorchHeadGenerator.make(m).generate(ids, max_new_tokens=9, eos_token_id=eos_id)
    assert got.dtype == ids.dtype
    assert torch.equal(got, ref)


@pytest.mark.parametrize("eos", [None, "late"])
def test_static_decode_steps_match_reference_loop(eos):
    """The self-advancing decode step (the one replayed on a CUDA graph on the
    GPU; here run eagerly): device-side position, in-place KV write, boolean
    mask over the full static buffers, token written to the output buffer."""
    m = _model()
    ids = torch.randint(0, 300, (2, 5), generator=torch.Generator().manual_seed(12))
    ref = OG.generate(m, ids, max_new_tokens=12)
    eos_id = None
    if eos == "late":
        eos_id = int(ref[1, 9])
        ref = OG.generate(m, ids, max_new_tokens=12, eos_token_id=eos_id)
    got = _TorchHeadGenerator.make(m).generate(ids, max_new_tokens=12, eos_token_id=eos_id,
                                               cuda_graph=True)
    assert torch.equal(got, ref)


def _qwen3_text_model(seed=0):
    """A plain (non multimodal-RoPE) decoder: transformers' Qwen3ForCausalLM."""
    from transformers.models.qwen3.configuration_qwen3 import Qwen3Config
    from transformers.models.qwen3.modeling_qwen3 import Qwen3ForCausalLM

    cfg = Qwen3Config(hidden_size=128, intermediate_size=256, num_hidden_layers=2,
                      num_attention_heads=4, num_key_value_heads=2, head_dim=32, vocab_size=300,
                      rms_norm_eps=1e-6, tie_word_embeddings=False)
    cfg._attn_implementation = "sdpa"
    torch.manual_seed(seed)
    m = Qwen3ForCausalLM(cfg).to(torch.bfloat16)
    with torch.no_grad():
        m.lm_head.weight.normal_(0, 0.5)
    return m.eval()


def test_static_decode_on_a_plain_decoder():
    """A decoder with 1-D RoPE positions: the static step passes [B, 1]
    positions from the device scalar; tokens equal the reference loop's."""
    m = _qwen3_text_model()
    ids = torch.randint(0, 300, (2, 5), generator=torch.Generator().manual_seed(21))
    ref = OG.generate(m, ids, max_new_tokens=10)
    g = _TorchHeadGenerator.make(m)
    assert not g._mrope
    assert torch.equal(g.generate(ids, max_new_tokens=10, cuda_graph=True), ref)
    assert torch.equal(g.generate(ids, max_new_tokens=10, cuda_graph=False), ref)


def test_decode_attention_falls_back_outside_the_captured_step():
    """The registered decode attention is transformers' SDPA whenever no decode
    position is set (prefill, eager calls) or the shapes are not one query
    token per sequence."""
    from transformers.integrations.sdpa_attention import sdpa_attention_forward

    from metal_liger_b200 import generation as G

    class _Attn(torch.nn.Module):
        num_key_value_groups = 2
        is_causal = True

    mod = _Attn()
    gen = torch.Generator().manual_seed(3)
    q = torch.randn(1, 4, 3, 32, generator=gen)
    k = torch.randn(1, 2, 3, 32, generator=gen)
    v = torch.randn(1, 2, 3, 32, generator=gen)
    assert G._DECODE_POS[0] is None
    a, _ = G._decode_attention_forward(mod, q, k, v, None, scaling=0.2)
    b, _ = sdpa_attention_forward(mod, q, k, v, None, scaling=0.2)
    torch.testing.assert_close(a, b)
    from transformers import AttentionInterface
    assert AttentionInterface._global_mapping[G._DECODE_ATTN] is G._decode_attention_forward


def test_sampling_rule_matches_reference():
    """temperature != 1 samples; temperature 1 with top_p 1 is greedy, as in
    the reference (generation.py:118-123)."""
    m = _model()
    ids = torch.randint(0, 300, (1, 4), generator=torch.Generator().manual_seed(3))
    g = _TorchHeadGenerator.make(m)
    greedy = OG.generate(m, ids, max_new_tokens=6)
    assert torch.equal(g.generate(ids, max_new_tokens=6, temperature=1.0, top_p=1.0), greedy)
    assert torch.equal(g.generate(ids, max_new_tokens=6, temperature=0), greedy)
    torch.manual_seed(5)
    a = g.generate(ids, max_new_tokens=6, temperature=0.7)
    torch.manual_seed(5)
    b = OG.generate(m, ids, max_new_tokens=6, temperature=0.7)
    assert a.shape == b.shape == (1, 10)
    assert torch.equal(a[:, :5], greedy[:, :5])  # the first token is always the argmax
    assert torch.equal(a, b)  # same logits, same draws


def test_patch_generator_semantics():
    from metal_liger_b200.generation import patch_generator

    m = _model()
    m.train()
    assert patch_generator(m) is m and m.generate() == "original"  # skipped while training
    m.eval()
    patch_generator(m)
    assert m._orig_generate() == "original"
    assert m.generate.__func__.__qualname__ == "MetalLigerGenerator.generate"
    m2 = _model()
    m2.train()
    patch_generator(m2, force=True)
    assert m2.generate.__func__.__qualname__ == "MetalLigerGenerator.generate"
    fp32 = _model(torch.float32)
    with pytest.raises(TypeError, match="bfloat16"):
        patch_generator(fp32)


def test_patcher_flag_installs_the_generator():
    from metal_liger_b200.patch import apply_metal_liger_to_qwen3vl

    m = _model()
    apply_metal_liger_to_qwen3vl(m, fuse_rms_norm=False, fuse_swiglu=False, fuse_lora=False,
                                 use_optimized_generator=True)
    assert m.generate.__func__.__qualname__ == "MetalLigerGenerator.generate"
    m2 = _model()
    m2.train()
    apply_metal_liger_to_qwen3vl(m2, fuse_rms_norm=False, fuse_swiglu=False, fuse_lora=False,
                                 use_optimized_generator=True)
    assert m2.generate() == "original"
