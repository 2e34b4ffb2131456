"""Fused greedy head (metal_liger::lm_head_argmax, the tcgen05 GEMM with the
argmax epilogue) and the static-KV generator on the GPU.

The head's choice is an index, so it is checked exactly: the oracle
(oracle/generation.py:argmax_rounded) forms fp64 logits, rounds them to fp32
and then to the logit dtype, and takes torch.argmax.  The kernel accumulates
in fp32 in another order, so a logit within one fp32 rounding of a
logit-dtype rounding boundary may land one ulp (of the logit dtype) away from
the oracle's (fp32 logits: a few fp32 ulps, bounded here by 1e-5 relative);
the tests therefore require (a) the logit the kernel picked to be the
oracle's maximum up to that tolerance, and (b) the same index wherever the
oracle's best logit beats the runner-up by more than twice the tolerance.  Exact ties
(duplicate vocabulary rows) and NaN follow torch.argmax: the lowest index.
"""

import pytest
import torch
import torch.nn as nn

from oracle import generation as OG
from metal_liger_b200 import _torch_library  # noqa: F401  (registers metal_liger:: ops)

pytestmark = pytest.mark.gpu
DEV = "cuda"
CODES = {torch.float32: 0, torch.bfloat16: 1, torch.float16: 2}


def _ulp(x: torch.Tensor, dt: torch.dtype) -> torch.Tensor:
    mant = {torch.bfloat16: 8, torch.float16: 11, torch.float32: 24}[dt]
    e = torch.floor(torch.log2(x.abs().clamp(min=1e-30)))
    return torch.pow(2.0, e - (mant - 1))


def _check(idx, val, hidden, weight, dt, bias=None):
    ridx, rval, logits = OG.argmax_rounded(hidden.cpu(), weight.cpu(), dt,
                                           None if bias is None else bias.cpu())
    idx, val = idx.cpu(), val.cpu()
    picked = logits.gather(1, idx[:, None])[:, 0]
    # one ulp of the logit dtype, or (fp32 logits) the fp32 accumulation-order
    # difference, 1e-5 relative
    tol = torch.maximum(_ulp(rval, dt), 1e-5 * rval.abs().clamp(min=1.0))
    assert torch.all((rval - picked) <= tol), "kernel picked a logit below the maximum"
    top2 = logits.topk(2, dim=1).values
    clear = (top2[:, 0] - top2[:, 1]) > 2 * tol
    assert torch.equal(idx[clear], ridx[clear]), "index differs on a clearly separated row"
    assert torch.all((val - rval).abs() <= tol)


@pytest.mark.parametrize("B,H,V,dt", [
    (1, 4096, 151936, torch.bfloat16),   # Qwen3-VL-8B lm_head, one sequence (GEMV kernel)
    (2, 520, 20000, torch.bfloat16),     # GEMV kernel, hidden not a multiple of 256
    (2, 2048, 151936, torch.float32),    # GEMV kernel, fp32 logits
    (1, 256, 1001, torch.bfloat16),      # small vocabulary: tensor-core path at batch 1
    (3, 256, 1001, torch.bfloat16),      # ragged vocabulary tile
    (16, 512, 5000, torch.float16),
    (8, 128, 100, torch.float32),        # vocabulary narrower than one tile
    (130, 256, 3000, torch.bfloat16),    # two row tiles (CTA-pair kernel by default)
])
def test_lm_head_argmax_against_oracle(B, H, V, dt):
    g = torch.Generator(device=DEV).manual_seed(B * 7 + V)
    hidden = torch.randn(B, H, generator=g, device=DEV).bfloat16()
    weight = (torch.randn(V, H, generator=g, device=DEV) * 0.05).bfloat16()
    idx, val = torch.ops.metal_liger.lm_head_argmax(hidden, weight, None, CODES[dt])
    assert idx.dtype == torch.int64 and idx.shape == (B,)
    _check(idx, val, hidden, weight, dt)


def test_lm_head_argmax_bias_strided_ties_and_nan():
    g = torch.Generator(device=DEV).manual_seed(3)
    H, V = 256, 2048
    full = torch.randn(4, 3, H, generator=g, device=DEV).bfloat16()
    hidden = full[:, -1, :]                                  # strided rows, as h[:, -1, :]
    # the GEMV kernel (batch <= 2) with the same bias, on a vocabulary large
    # enough to take it
    w_big = (torch.randn(30000, H, generator=g, device=DEV) * 0.05).bfloat16()
    b_big = torch.randn(30000, generator=g, device=DEV).bfloat16()
    i2, v2 = torch.ops.metal_liger.lm_head_argmax(hidden[:2], w_big, b_big, 1)
    _check(i2, v2, hidden[:2], w_big, torch.bfloat16, b_big.float())
    weight = (torch.randn(V, H, generator=g, device=DEV) * 0.05).bfloat16()
    bias = torch.randn(V, generator=g, device=DEV) * 0.1
    idx, val = torch.ops.metal_liger.lm_head_argmax(hidden, weight, bias, 1)
    _check(idx, val, hidden, weight, torch.bfloat16, bias)
    # exact ties: the row that wins for sequence 0 is duplicated at a higher
    # and a lower index; the lowest copy must win
    win = int(idx[0])
    w2 = weight.clone()
    lo, hi = (win // 2, min(V - 1, win + 700))
    w2[hi] = weight[win]
    w2[lo] = weight[win]
    idx2, _ = torch.ops.metal_liger.lm_head_argmax(hidden, w2, None, 1)
    assert int(idx2[0]) == min(lo, win)
    # NaN logits win, first NaN first (torch.argmax)
    w3 = weight.clone()
    w3[1500] = float("nan")
    w3[900] = float("nan")
    idx3, _ = torch.ops.metal_liger.lm_head_argmax(hidden, w3, None, 1)
    assert idx3.tolist() == [900] * 4
    wb = w_big.clone()
    wb[29000] = float("nan")
    wb[12345] = float("nan")
    idx4, _ = torch.ops.metal_liger.lm_head_argmax(hidden[:1], wb, None, 1)
    assert idx4.tolist() == [12345]
    win = int(torch.ops.metal_liger.lm_head_argmax(hidden[:1], w_big, None, 1)[0][0])
    wt = w_big.clone()
    wt[win // 3] = w_big[win]
    assert int(torch.ops.metal_liger.lm_head_argmax(hidden[:1], wt, None, 1)[0][0]) == win // 3


def test_lm_head_argmax_errors_and_empty():
    w = torch.randn(64, 32, device=DEV).bfloat16()
    with pytest.raises(RuntimeError, match="bfloat16"):
        torch.ops.metal_liger.lm_head_argmax(torch.randn(2, 32, device=DEV), w, None, 1)
    with pytest.raises(RuntimeError, match="do not match"):
        torch.ops.metal_liger.lm_head_argmax(torch.randn(2, 16, device=DEV).bfloat16(), w,
                                             None, 1)
    idx, val = torch.ops.metal_liger.lm_head_argmax(torch.empty(0, 32, device=DEV).bfloat16(),
                                                    w, None, 1)
    assert idx.shape == (0,) and val.shape == (0,)


class _CausalLM(nn.Module):
    def __init__(self, text_model, vocab, hidden):
        super().__init__()
        self.model = text_model
        self.config = text_model.config
        self.lm_head = nn.Linear(hidden, vocab, bias=False, device=DEV, dtype=torch.bfloat16)


def _model(seed=0, layers=2, vocab=1000):
    from transformers.models.qwen3_vl.configuration_qwen3_vl import Qwen3VLTextConfig
    from transformers.models.qwen3_vl.modeling_qwen3_vl import Qwen3VLTextModel

    cfg = Qwen3VLTextConfig(hidden_size=256, intermediate_size=512, num_hidden_layers=layers,
                            num_attention_heads=4, num_key_value_heads=2, head_dim=64,
                            vocab_size=vocab, rms_norm_eps=1e-6,
                            rope_parameters={"rope_type": "default", "rope_theta": 5e6,
                                             "mrope_section": [12, 10, 10]})
    cfg._attn_implementation = "sdpa"
    torch.manual_seed(seed)
    with torch.device(DEV):
        text = Qwen3VLTextModel(cfg).to(torch.bfloat16)
    m = _CausalLM(text, vocab, 256)
    with torch.no_grad():
        m.lm_head.weight.normal_(0, 0.5)
    return m.eval()


@pytest.mark.parametrize("graph", [False, True], ids=["eager", "cuda_graph"])
def test_generator_matches_reference_loop(graph):
    """Greedy tokens equal the reference loop's (oracle loop on the same GPU
    model with transformers' DynamicCache and the model's own lm_head); where
    they part, the reference's two best logits at that step are within one
    bf16 ulp of each other (a rounding-order near-tie), never further.  The
    CUDA-graph decode replays one captured, self-advancing step per token."""
    from metal_liger_b200.generation import MetalLigerGenerator

    m = _model()
    ids = torch.randint(0, 1000, (3, 6), generator=torch.Generator().manual_seed(4)).to(DEV)
    got = MetalLigerGenerator(m).generate(ids, max_new_tokens=24, cuda_graph=graph)
    ref = OG.generate(m, ids, max_new_tokens=24)
    assert got.shape == ref.shape == (3, 30)
    _same_or_near_tie(m, got, ref)


def _same_or_near_tie(m, got, ref):
    """Sequences equal, or the first difference sits where the reference's two
    best logits are within one bf16 ulp (a rounding-order near-tie)."""
    assert got.shape == ref.shape
    for b in range(got.shape[0]):
        diff = (got[b] != ref[b]).nonzero()
        if diff.numel() == 0:
            continue
        t = int(diff[0])
        with torch.no_grad():
            h = m.model(input_ids=ref[b:b + 1, :t]).last_hidden_state[:, -1]
            logits = m.lm_head(h).float()[0]
        top2 = logits.topk(2).values
        assert float(top2[0] - top2[1]) <= float(_ulp(top2[0:1], torch.bfloat16)[0]), \
            f"row {b} diverges at {t} without a near-tie"


def test_decode_graph_is_reused_across_calls():
    """The captured step and its buffers are kept per (batch, length): a second
    call replays it from the first decode token, a call with another prompt
    length but the same total length reuses it, and the returned ids are
    copies (a later call does not change them)."""
    from metal_liger_b200.generation import MetalLigerGenerator

    m = _model(seed=3)
    g = MetalLigerGenerator(m)
    gen = torch.Generator().manual_seed(11)
    ids1 = torch.randint(0, 1000, (2, 6), generator=gen).to(DEV)
    ids2 = torch.randint(0, 1000, (2, 9), generator=gen).to(DEV)
    a = g.generate(ids1, max_new_tokens=20)
    a_copy = a.clone()
    assert len(g._states) == 1 and next(iter(g._states.values())).graph is not None
    b = g.generate(ids1, max_new_tokens=20)
    assert torch.equal(a, b)
    c = g.generate(ids2, max_new_tokens=17)               # same total length 26
    assert len(g._states) == 1
    _same_or_near_tie(m, c, OG.generate(m, ids2, max_new_tokens=17))
    assert torch.equal(a, a_copy)
    d = g.generate(ids1[:1], max_new_tokens=20)           # another batch: a second state
    assert len(g._states) == 2
    _same_or_near_tie(m, d, OG.generate(m, ids1[:1], max_new_tokens=20))


def test_generator_eos_sampling_and_patch():
    from metal_liger_b200.generation import patch_generator

    m = _model(seed=1)
    ids = torch.randint(0, 1000, (1, 5), generator=torch.Generator().manual_seed(6)).to(DEV)
    patch_generator(m)
    out = m.generate(ids, max_new_tokens=8)
    assert out.shape == (1, 13) and torch.equal(out[:, :5], ids)
    eos = int(out[0, 7])
    stopped = m.generate(ids, max_new_tokens=8, eos_token_id=eos)
    first = int((out[0, 5:] == eos).nonzero()[0]) + 5
    assert torch.equal(stopped, out[:, :first + 1])
    torch.manual_seed(0)
    sampled = m.generate(ids, max_new_tokens=8, temperature=0.8)
    assert sampled.shape == (1, 13) and int(sampled.max()) < 1000 and int(sampled.min()) >= 0
    assert int(sampled[0, 5]) == int(out[0, 5])  # the first token is always the argmax


def test_cuda_graph_decode_stops_at_eos_like_the_eager_loop():
    """End of sequence found inside a chunk of graph replays: the output is
    cut exactly where the eager loop (and the reference) stops."""
    from metal_liger_b200.generation import MetalLigerGenerator

    m = _model(seed=2)
    g = MetalLigerGenerator(m)
    ids = torch.randint(0, 1000, (1, 4), generator=torch.Generator().manual_seed(9)).to(DEV)
    full = g.generate(ids, max_new_tokens=40, cuda_graph=False)
    eos = int(full[0, 4 + 9])              # a token produced after the graph warm-up
    first = int((full[0, 4:] == eos).nonzero()[0]) + 4
    eager = g.generate(ids, max_new_tokens=40, eos_token_id=eos, cuda_graph=False)
    graph = g.generate(ids, max_new_tokens=40, eos_token_id=eos, cuda_graph=True)
    assert torch.equal(eager, full[:, :first + 1])
    assert torch.equal(graph, eager)


@pytest.mark.parametrize("rows,K,N", [(1, 4096, 1024), (2, 4096, 12288), (1, 12288, 4096),
                                      (2, 520, 7), (1, 64, 300)])
def test_gemv_against_fp32_reference(rows, K, N):
    """Decode-time linear layer: fp32 accumulation of bf16 products, output
    rounded to bf16 once, so within one bf16 rounding of the fp32 result."""
    g = torch.Generator(device=DEV).manual_seed(rows * K + N)
    x = torch.randn(rows, 1, K, generator=g, device=DEV).bfloat16()
    w = (torch.randn(N, K, generator=g, device=DEV) * 0.02).bfloat16()
    b = torch.randn(N, generator=g, device=DEV).bfloat16()
    y = torch.ops.metal_liger.gemv(x, w, b)
    assert y.shape == (rows, 1, N) and y.dtype == torch.bfloat16
    ref = x.float().reshape(rows, K) @ w.float().t() + b.float()
    got = y.float().reshape(rows, N)
    tol = 2.0 ** -8 * ref.abs() + 1e-3 * ref.abs().max()
    assert torch.all((got - ref).abs() <= tol), float((got - ref).abs().max())
    y0 = torch.ops.metal_liger.gemv(x, w, None)
    torch.testing.assert_close(y0.float().reshape(rows, N), (x.float().reshape(rows, K)
                                                              @ w.float().t()),
                               rtol=2 ** -7, atol=1e-3)


def test_gemv_rejects_more_than_two_rows():
    w = torch.randn(64, 32, device=DEV).bfloat16()
    with pytest.raises(RuntimeError, match="at most 2"):
        torch.ops.metal_liger.gemv(torch.randn(3, 32, device=DEV).bfloat16(), w, None)


@pytest.mark.parametrize("rows,K,I", [(1, 4096, 12288), (2, 512, 1000), (1, 64, 33)])
def test_gemv_swiglu_equals_gemv_gemv_swiglu(rows, K, I):
    """The fused decode MLP input side is the unfused decode path bit for bit."""
    g = torch.Generator(device=DEV).manual_seed(rows + K + I)
    x = torch.randn(rows, K, generator=g, device=DEV).bfloat16()
    wg = (torch.randn(I, K, generator=g, device=DEV) * 0.05).bfloat16()
    wu = (torch.randn(I, K, generator=g, device=DEV) * 0.05).bfloat16()
    ops = torch.ops.metal_liger
    fused = ops.gemv_swiglu(x, wg, wu)
    unfused = ops.swiglu_forward(ops.gemv(x, wg, None), ops.gemv(x, wu, None), "")
    assert torch.equal(fused, unfused)


def test_generator_on_the_patched_model():
    """Inference patch (fused RMSNorm, q/k norm, SwiGLU MLP, RoPE in attention):
    the CUDA-graph decode (GEMV projections, fused gate/up/activation) against
    the eager loop of the same generator and against the reference loop."""
    from metal_liger_b200 import apply_metal_liger_to_qwen3vl
    from metal_liger_b200.generation import MetalLigerGenerator

    from metal_liger_b200.patch import restore_attention_rope

    m = _model(seed=5)
    apply_metal_liger_to_qwen3vl(m, fuse_lora=False, fuse_qk_norm=True,
                                 fuse_rope_in_attention=True)
    try:
        for p in m.parameters():
            p.requires_grad_(False)
        ids = torch.randint(0, 1000, (2, 7), generator=torch.Generator().manual_seed(13)).to(DEV)
        g = MetalLigerGenerator(m)
        graph = g.generate(ids, max_new_tokens=30)
        eager = g.generate(ids, max_new_tokens=30, cuda_graph=False)
        _same_or_near_tie(m, graph, eager)
        _same_or_near_tie(m, graph, OG.generate(m, ids, max_new_tokens=30))
    finally:
        # the RoPE rebinding is per modeling module (process-wide): undo it
        restore_attention_rope(m)


@pytest.mark.parametrize("rows", [1, 2])
def test_gemv_multi_equals_separate_gemvs(rows):
    """q, k, v in one launch: each output is the single GEMV's bit for bit,
    with and without biases."""
    g = torch.Generator(device=DEV).manual_seed(40 + rows)
    K = 1024
    x = torch.randn(rows, 1, K, generator=g, device=DEV).bfloat16()
    ws = [(torch.randn(n, K, generator=g, device=DEV) * 0.03).bfloat16() for n in (512, 128, 128)]
    bs = [torch.randn(w.shape[0], generator=g, device=DEV).bfloat16() for w in ws]
    ops = torch.ops.metal_liger
    for biases in ([None, None, None], bs, [bs[0], None, bs[2]]):
        outs = ops.gemv_multi(x, ws, biases)
        assert [tuple(o.shape) for o in outs] == [(rows, 1, w.shape[0]) for w in ws]
        for o, w, b in zip(outs, ws, biases):
            assert torch.equal(o, ops.gemv(x, w, b))


@pytest.mark.parametrize("B,Hq,Hkv,L,D,n", [(1, 32, 8, 192, 128, 150), (2, 4, 2, 300, 64, 300),
                                            (1, 8, 8, 64, 128, 1), (3, 8, 2, 260, 256, 129),
                                            (2, 16, 1, 100, 64, 77), (2, 8, 2, 1024, 128, 777)])
def test_decode_attention_against_fp32_reference(B, Hq, Hkv, L, D, n):
    """Decode-step attention over the first n = pos + 1 cache positions (read
    from device memory), grouped-query heads in place, against fp32 softmax
    attention over the same positions."""
    g = torch.Generator(device=DEV).manual_seed(B * L + n)
    q = torch.randn(B, 1, Hq, D, generator=g, device=DEV).bfloat16().transpose(1, 2)
    k = torch.randn(B, Hkv, L, D, generator=g, device=DEV).bfloat16()
    v = torch.randn(B, Hkv, L, D, generator=g, device=DEV).bfloat16()
    pos = torch.tensor([n - 1], dtype=torch.int64, device=DEV)
    scale = D ** -0.5
    out = torch.ops.metal_liger.decode_attention(q, k, v, pos, 1, scale)
    assert out.shape == (B, 1, Hq, D) and out.dtype == torch.bfloat16
    G = Hq // Hkv
    kk = k[:, :, :n].float().repeat_interleave(G, dim=1)
    vv = v[:, :, :n].float().repeat_interleave(G, dim=1)
    att = torch.softmax((q.float() @ kk.transpose(-1, -2)) * scale, dim=-1)
    ref = (att @ vv).transpose(1, 2)
    torch.testing.assert_close(out.float(), ref, rtol=2e-2, atol=1e-2)
    pos.fill_(n - 2 if n > 1 else 0)                      # the length follows the device value
    out2 = torch.ops.metal_liger.decode_attention(q, k, v, pos, 1, scale)
    m = max(n - 1, 1)
    att2 = torch.softmax((q.float() @ kk[:, :, :m].transpose(-1, -2)) * scale, dim=-1)
    torch.testing.assert_close(out2.float(), (att2 @ vv[:, :, :m]).transpose(1, 2), rtol=2e-2,
                               atol=1e-2)



def test_decode_attention_rejects_unsupported_groups():
    """Query heads per kv head x head_dim above 1024 is refused (the generator
    then keeps transformers' attention)."""
    q = torch.randn(1, 16, 1, 256, device=DEV).bfloat16()
    k = torch.randn(1, 1, 64, 256, device=DEV).bfloat16()
    pos = torch.zeros(1, dtype=torch.int64, device=DEV)
    with pytest.raises(RuntimeError, match="above 1024"):
        torch.ops.metal_liger.decode_attention(q, k, k, pos, 1, 0.0625)


@pytest.mark.parametrize("B,Hq,Hkv,D", [(1, 32, 8, 128), (2, 4, 2, 64), (1, 8, 4, 256)])
def test_decode_qk_norm_rope_against_the_unfused_ops(B, Hq, Hkv, D):
    """One new token: per-head RMSNorm (this library's) + RoPE (this library's,
    with the model's cos/sin) of q and k, k/v written into the caches at the
    device position; the fused kernel against the separate ops at bf16
    rounding (one ulp), the untouched cache positions unchanged."""
    from metal_liger_b200.ops.fused_rope import apply_fused_rotary

    g = torch.Generator(device=DEV).manual_seed(B * Hq + D)
    L, p = 40, 17
    q = torch.randn(B, 1, Hq * D, generator=g, device=DEV).bfloat16()
    k = torch.randn(B, 1, Hkv * D, generator=g, device=DEV).bfloat16()
    v = torch.randn(B, 1, Hkv * D, generator=g, device=DEV).bfloat16()
    wq = (1 + 0.1 * torch.randn(D, generator=g, device=DEV)).bfloat16()
    wk = (1 + 0.1 * torch.randn(D, generator=g, device=DEV)).bfloat16()
    ang = torch.rand(B, 1, D // 2, generator=g, device=DEV) * 6.0
    cos = torch.cat([ang.cos(), ang.cos()], -1).bfloat16()
    sin = torch.cat([ang.sin(), ang.sin()], -1).bfloat16()
    kc = torch.randn(B, Hkv, L, D, generator=g, device=DEV).bfloat16()
    vc = torch.randn(B, Hkv, L, D, generator=g, device=DEV).bfloat16()
    kc0, vc0 = kc.clone(), vc.clone()
    pos = torch.tensor([p], dtype=torch.int64, device=DEV)
    ops = torch.ops.metal_liger
    q4 = ops.decode_qk_norm_rope(q, k, v, wq, wk, 1e-6, 1e-5, cos, sin, kc, vc, pos)
    assert q4.shape == (B, Hq, 1, D)
    qn = ops.rms_norm_forward(q.view(B, 1, Hq, D), wq, 1e-6, "")[0].transpose(1, 2)
    kn = ops.rms_norm_forward(k.view(B, 1, Hkv, D), wk, 1e-5, "")[0].transpose(1, 2)
    qr, kr = apply_fused_rotary(qn, kn, cos.unsqueeze(1), sin.unsqueeze(1))
    ulp = 2.0 ** -7
    assert torch.allclose(q4.float(), qr.float(), rtol=ulp, atol=ulp)
    assert torch.allclose(kc[:, :, p].float(), kr[:, :, 0].float(), rtol=ulp, atol=ulp)
    assert torch.equal(vc[:, :, p], v.view(B, Hkv, D))
    keep = torch.ones(L, dtype=torch.bool)
    keep[p] = False
    assert torch.equal(kc[:, :, keep], kc0[:, :, keep]) and torch.equal(vc[:, :, keep], vc0[:, :, keep])


@pytest.mark.parametrize("rows,K,N", [(1, 4096, 4096), (2, 12288, 4096), (1, 1024, 1000)])
def test_gemv_residual_equals_gemv_then_add(rows, K, N):
    """The o / down projection with the decoder's residual add in its
    epilogue: gemv followed by the bf16 add, bit for bit, with and without a
    bias."""
    g = torch.Generator(device=DEV).manual_seed(rows * 7 + K + N)
    x = torch.randn(rows, 1, K, generator=g, device=DEV).bfloat16()
    w = (torch.randn(N, K, generator=g, device=DEV) * 0.02).bfloat16()
    b = torch.randn(N, generator=g, device=DEV).bfloat16()
    res = torch.randn(rows, 1, N, generator=g, device=DEV).bfloat16()
    ops = torch.ops.metal_liger
    for bias in (None, b):
        y = ops.gemv_residual(x, w, bias, res)
        assert y.shape == (rows, 1, N)
        assert torch.equal(y, res + ops.gemv(x, w, bias))


@pytest.mark.parametrize("K", [4096, 2048, 8192, 16384, 1000, 256, 128, 64])
@pytest.mark.parametrize("rows", [1, 2])
def test_gemv_rmsnorm_multi_equals_norm_then_gemv_multi(rows, K):
    """The decoder's input RMSNorm fused into the q/k/v GEMV's activation
    staging: equal bit for bit to this library's RMSNorm kernel followed by
    gemv_multi, for every RMSNorm row layout (two to eight vectors per thread
    on 256 threads, one per thread, sub-warp rows)."""
    g = torch.Generator(device=DEV).manual_seed(rows * 31 + K)
    x = (torch.randn(rows, 1, K, generator=g, device=DEV) * 3).bfloat16()
    nw = (1 + 0.1 * torch.randn(K, generator=g, device=DEV)).bfloat16()
    ws = [(torch.randn(n, K, generator=g, device=DEV) * 0.03).bfloat16() for n in (256, 64, 64)]
    bs = [torch.randn(w.shape[0], generator=g, device=DEV).bfloat16() for w in ws]
    ops = torch.ops.metal_liger
    xn = ops.rms_norm_forward(x, nw, 1e-6, "")[0]
    for biases in ([None, None, None], bs):
        fused = ops.gemv_rmsnorm_multi(x, nw, 1e-6, ws, biases)
        for f, u in zip(fused, ops.gemv_multi(xn, ws, biases)):
            assert torch.equal(f, u)


@pytest.mark.parametrize("rows,K,I", [(1, 4096, 12288), (2, 2048, 1000), (1, 128, 96)])
def test_gemv_rmsnorm_swiglu_equals_norm_then_gemv_swiglu(rows, K, I):
    """The post-attention RMSNorm fused into the gate/up/SwiGLU GEMV: equal
    bit for bit to the RMSNorm kernel followed by gemv_swiglu."""
    g = torch.Generator(device=DEV).manual_seed(rows + K * 3 + I)
    x = (torch.randn(rows, 1, K, generator=g, device=DEV) * 2).bfloat16()
    nw = (1 + 0.1 * torch.randn(K, generator=g, device=DEV)).bfloat16()
    wg = (torch.randn(I, K, generator=g, device=DEV) * 0.05).bfloat16()
    wu = (torch.randn(I, K, generator=g, device=DEV) * 0.05).bfloat16()
    ops = torch.ops.metal_liger
    fused = ops.gemv_rmsnorm_swiglu(x, nw, 1e-5, wg, wu)
    unfused = ops.gemv_swiglu(ops.rms_norm_forward(x, nw, 1e-5, "")[0], wg, wu)
    assert torch.equal(fused, unfused)


def test_fused_rmsnorm_gemv_rejects_bad_operands():
    ops = torch.ops.metal_liger
    x = torch.randn(1, 1, 256, device=DEV).bfloat16()
    w = torch.randn(64, 256, device=DEV).bfloat16()
    with pytest.raises(RuntimeError, match="norm weight"):
        ops.gemv_rmsnorm_swiglu(x, torch.ones(256, device=DEV), 1e-6, w, w)  # fp32
    with pytest.raises(RuntimeError, match="norm weight"):
        ops.gemv_rmsnorm_multi(x, torch.ones(128, device=DEV).bfloat16(), 1e-6, [w], [None])
    with pytest.raises(RuntimeError, match="residual"):
        ops.gemv_residual(x, w, None, torch.randn(1, 1, 65, device=DEV).bfloat16())


def test_fused_decoder_layers_equal_the_unfused_decode_path(monkeypatch):
    """The CUDA-graph decode with whole decoder layers fused (the norms in the
    q/k/v and gate/up GEMVs, the residual adds in the o and down GEMVs)
    produces exactly the tokens of the decode path with the layers unfused
    (RMSNorm kernels, the attention block patch, GEMVs and torch residual
    adds): every fused op equals its unfused composition bit for bit."""
    from metal_liger_b200 import apply_metal_liger_to_qwen3vl, generation
    from metal_liger_b200.generation import MetalLigerGenerator
    from metal_liger_b200.patch import restore_attention_rope

    m = _model(seed=9, layers=3)
    apply_metal_liger_to_qwen3vl(m, fuse_lora=False, fuse_qk_norm=True,
                                 fuse_rope_in_attention=True)
    calls = []
    real = generation._decode_layer_forward

    def counting(layer, cache, pos):
        fwd = real(layer, cache, pos)

        def wrapped(*a, **k):
            calls.append(1)
            return fwd(*a, **k)
        return wrapped

    try:
        for p in m.parameters():
            p.requires_grad_(False)
        ids = torch.randint(0, 1000, (2, 5), generator=torch.Generator().manual_seed(21)).to(DEV)
        monkeypatch.setattr(generation, "_decode_layer_forward", counting)
        fused = MetalLigerGenerator(m).generate(ids, max_new_tokens=20)
        assert calls, "the fused decoder-layer path did not run"
        monkeypatch.setattr(generation, "_FUSED_LAYER_TYPES", ())
        unfused = MetalLigerGenerator(m).generate(ids, max_new_tokens=20)
        assert torch.equal(fused, unfused)
    finally:
        restore_attention_rope(m)


@pytest.mark.parametrize("G,D", [(4, 128), (16, 64), (1, 256), (2, 256)])
def test_decode_attention_single_launch_equals_split_merge(G, D):
    """Caches of up to 256 positions take the single-launch kernel (every
    slot's partial and their merge in one CTA's shared memory), longer ones
    the chunk and merge kernels.  Over the same filled positions both give
    the same output bit for bit (same partials, merged in the same order)."""
    B, Hkv, n = 2, 2, 200
    Hq = G * Hkv
    g = torch.Generator(device=DEV).manual_seed(G * 1000 + D)
    q = torch.randn(B, Hq, 1, D, generator=g, device=DEV).bfloat16()
    k_long = torch.randn(B, Hkv, 320, D, generator=g, device=DEV).bfloat16()
    v_long = torch.randn(B, Hkv, 320, D, generator=g, device=DEV).bfloat16()
    k_short = k_long[:, :, :256].contiguous()
    v_short = v_long[:, :, :256].contiguous()
    pos = torch.tensor([n - 1], dtype=torch.int64, device=DEV)
    ops = torch.ops.metal_liger
    single = ops.decode_attention(q, k_short, v_short, pos, 1, D ** -0.5)
    split = ops.decode_attention(q, k_long, v_long, pos, 1, D ** -0.5)
    assert torch.equal(single, split)


@pytest.mark.parametrize("B,Hq,Hkv,D,L,p", [(1, 32, 8, 128, 192, 150), (2, 4, 2, 64, 256, 255),
                                            (1, 16, 1, 64, 100, 0), (2, 8, 4, 256, 64, 40),
                                            (3, 8, 1, 128, 200, 77)])
def test_decode_qk_attention_equals_prep_then_attention(B, Hq, Hkv, D, L, p):
    """q/k norm + RoPE + cache write and the attention in one launch: the
    output and both caches bit for bit those of decode_qk_norm_rope followed
    by decode_attention."""
    g = torch.Generator(device=DEV).manual_seed(B * Hq + D + L + p)
    q = torch.randn(B, 1, Hq * D, generator=g, device=DEV).bfloat16()
    k = torch.randn(B, 1, Hkv * D, generator=g, device=DEV).bfloat16()
    v = torch.randn(B, 1, Hkv * D, generator=g, device=DEV).bfloat16()
    wq = (1 + 0.1 * torch.randn(D, generator=g, device=DEV)).bfloat16()
    wk = (1 + 0.1 * torch.randn(D, generator=g, device=DEV)).bfloat16()
    ang = torch.rand(B, 1, D // 2, generator=g, device=DEV) * 6.0
    cos = torch.cat([ang.cos(), ang.cos()], -1).bfloat16()
    sin = torch.cat([ang.sin(), ang.sin()], -1).bfloat16()
    kc = torch.randn(B, Hkv, L, D, generator=g, device=DEV).bfloat16()
    vc = torch.randn(B, Hkv, L, D, generator=g, device=DEV).bfloat16()
    kc2, vc2 = kc.clone(), vc.clone()
    pos = torch.tensor([p], dtype=torch.int64, device=DEV)
    ops = torch.ops.metal_liger
    fused = ops.decode_qk_attention(q, k, v, wq, wk, 1e-6, 1e-5, cos, sin, kc, vc, pos,
                                    D ** -0.5)
    q4 = ops.decode_qk_norm_rope(q, k, v, wq, wk, 1e-6, 1e-5, cos, sin, kc2, vc2, pos)
    ref = ops.decode_attention(q4, kc2, vc2, pos, 1, D ** -0.5)
    assert torch.equal(kc, kc2) and torch.equal(vc, vc2)
    assert torch.equal(fused, ref)


def test_decode_qk_attention_rejects_long_caches():
    ops = torch.ops.metal_liger
    B, Hkv, D = 1, 2, 64
    kc = torch.zeros(B, Hkv, 257, D, device=DEV).bfloat16()
    x = torch.zeros(B, 1, 4 * D, device=DEV).bfloat16()
    kv = torch.zeros(B, 1, Hkv * D, device=DEV).bfloat16()
    w = torch.ones(D, device=DEV).bfloat16()
    cs = torch.ones(B, 1, D, device=DEV).bfloat16()
    pos = torch.zeros(1, dtype=torch.int64, device=DEV)
    with pytest.raises(RuntimeError, match="at most 256"):
        ops.decode_qk_attention(x, kv, kv, w, w, 1e-6, 1e-6, cs, cs, kc, kc.clone(), pos, 0.125)


@pytest.mark.parametrize("p", [40, 41, -1])
def test_decode_prep_outside_the_cache_writes_q_only(p):
    """A device position outside [0, L): both forms still prepare q (norm +
    RoPE) and leave both caches untouched, and the one-launch attention stays
    bit for bit the prep kernel followed by the attention."""
    from metal_liger_b200.ops.fused_rope import apply_fused_rotary

    B, Hq, Hkv, D, L = 2, 8, 2, 64, 40
    g = torch.Generator(device=DEV).manual_seed(71 + p)
    q = torch.randn(B, 1, Hq * D, generator=g, device=DEV).bfloat16()
    k = torch.randn(B, 1, Hkv * D, generator=g, device=DEV).bfloat16()
    v = torch.randn(B, 1, Hkv * D, generator=g, device=DEV).bfloat16()
    wq = (1 + 0.1 * torch.randn(D, generator=g, device=DEV)).bfloat16()
    wk = (1 + 0.1 * torch.randn(D, generator=g, device=DEV)).bfloat16()
    ang = torch.rand(B, 1, D // 2, generator=g, device=DEV) * 6.0
    cos = torch.cat([ang.cos(), ang.cos()], -1).bfloat16()
    sin = torch.cat([ang.sin(), ang.sin()], -1).bfloat16()
    kc = torch.randn(B, Hkv, L, D, generator=g, device=DEV).bfloat16()
    vc = torch.randn(B, Hkv, L, D, generator=g, device=DEV).bfloat16()
    kc0, vc0 = kc.clone(), vc.clone()
    kc2, vc2 = kc.clone(), vc.clone()
    pos = torch.tensor([p], dtype=torch.int64, device=DEV)
    ops = torch.ops.metal_liger
    q4 = ops.decode_qk_norm_rope(q, k, v, wq, wk, 1e-6, 1e-5, cos, sin, kc2, vc2, pos)
    assert torch.equal(kc2, kc0) and torch.equal(vc2, vc0)
    qn = ops.rms_norm_forward(q.view(B, 1, Hq, D), wq, 1e-6, "")[0].transpose(1, 2)
    kn = ops.rms_norm_forward(k.view(B, 1, Hkv, D), wk, 1e-5, "")[0].transpose(1, 2)
    qr, _ = apply_fused_rotary(qn, kn, cos.unsqueeze(1), sin.unsqueeze(1))
    ulp = 2.0 ** -7
    assert torch.allclose(q4.float(), qr.float(), rtol=ulp, atol=ulp)
    if p >= 0:  # the attention reads min(p + 1, L) positions
        fused = ops.decode_qk_attention(q, k, v, wq, wk, 1e-6, 1e-5, cos, sin, kc, vc, pos,
                                        D ** -0.5)
        assert torch.equal(kc, kc0) and torch.equal(vc, vc0)
        assert torch.equal(fused, ops.decode_attention(q4, kc2, vc2, pos, 1, D ** -0.5))
