"""RoPE CUDA parity: reference fixtures, strided views, BASELINE config 1 (in-kernel cos/sin)."""

import pytest
import torch

from conftest import golden_names, load_golden
from oracle import ops as O
from tolerances import assert_close

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.mark.parametrize("name", golden_names("rope_"))
def test_against_reference_fixture(name):
    from metal_liger_b200.ops.fused_rope import _FusedRoPEFunction
    d = load_golden(name)
    x = d["x"].to(DEV).requires_grad_(True)
    y = _FusedRoPEFunction.apply(x, d["cos"].to(DEV), d["sin"].to(DEV))
    y.backward(d["dy"].to(DEV))
    assert y.dtype == d["y"].dtype, (y.dtype, d["y"].dtype)
    assert x.grad.dtype == d["dx"].dtype
    if d["y"].dtype == torch.float32:
        assert_close(y.detach().cpu(), d["y"], rtol=1e-5, atol=1e-6, what="y")
        assert_close(x.grad.cpu(), d["dx"], rtol=1e-5, atol=1e-6, what="dx")
    # and always against the fp32 oracle at the dtype's tolerance
    ry = O.rope_apply(d["x"], d["cos"], d["sin"])
    rdx = O.rope_backward(d["dy"], d["cos"], d["sin"])
    assert_close(y.detach().cpu(), ry, dtype=d["y"].dtype, what="y vs oracle")
    assert_close(x.grad.cpu(), rdx, dtype=d["dx"].dtype, what="dx vs oracle")


def test_reference_test_case_and_inverse():
    """tests/test_fused_ops.py:156-188 — and a real check that bwd inverts fwd."""
    from metal_liger_b200.ops.fused_rope import _apply_rotary_fused, _rotate_half
    seq, dim = 128, 64
    freqs = 1.0 / (10000.0 ** (torch.arange(0, dim, 2).float() / dim))
    ang = torch.arange(seq).float()[:, None] * freqs[None, :]
    cos, sin = torch.cos(ang).repeat(1, 2).to(DEV), torch.sin(ang).repeat(1, 2).to(DEV)
    x = torch.randn(2, 8, seq, dim, device=DEV)
    ref = x * cos + _rotate_half(x) * sin
    out = _apply_rotary_fused(x, cos, sin)
    assert torch.allclose(ref, out, atol=1e-6)
    back = torch.ops.metal_liger.rope_apply(out, cos, sin, -1)
    assert torch.allclose(back, x, atol=1e-5)


def test_qk_single_launch_on_transposed_views():
    """HF passes q/k as transpose(1, 2) views of [B, S, H, D]; read them in place."""
    from metal_liger_b200.ops.fused_rope import apply_fused_rotary
    B, S, Hq, Hk, D = 2, 24, 6, 2, 128
    qs = torch.randn(B, S, Hq, D, device=DEV, dtype=torch.bfloat16)
    ks = torch.randn(B, S, Hk, D, device=DEV, dtype=torch.bfloat16)
    q = qs.transpose(1, 2).requires_grad_(True)
    k = ks.transpose(1, 2).requires_grad_(True)
    q.retain_grad()
    k.retain_grad()
    pos = torch.arange(S).expand(B, S)
    inv = O.rope_inv_freq(D, 5e6)
    cos, sin = O.rope_cos_sin(pos, inv)
    cos, sin = cos[:, None].to(DEV, torch.bfloat16), sin[:, None].to(DEV, torch.bfloat16)
    qr, kr = apply_fused_rotary(q, k, cos, sin)
    dq, dk = torch.randn_like(qr), torch.randn_like(kr)
    torch.autograd.backward([qr, kr], [dq, dk])
    for got, x, what in ((qr, q, "q"), (kr, k, "k")):
        ref = O.rope_apply(x.detach().cpu(), cos.cpu(), sin.cpu())
        assert_close(got.detach().cpu(), ref, dtype=torch.bfloat16, what=what)
    assert_close(q.grad.cpu(), O.rope_backward(dq.cpu(), cos.cpu(), sin.cpu()),
                 dtype=torch.bfloat16, what="dq")
    assert_close(k.grad.cpu(), O.rope_backward(dk.cpu(), cos.cpu(), sin.cpu()),
                 dtype=torch.bfloat16, what="dk")


@pytest.mark.parametrize("D", [2, 6, 64, 96, 128, 256])
def test_head_dims_and_scalar_path(D):
    from metal_liger_b200.ops.fused_rope import apply_fused_rotary_from_positions
    q = torch.randn(2, 3, 11, D, device=DEV)
    k = torch.randn(2, 1, 11, D, device=DEV)
    pos = torch.randint(0, 5000, (2, 11))
    qr, kr = apply_fused_rotary_from_positions(q, k, pos.to(DEV), theta=10000.0)
    cos, sin = O.rope_cos_sin(pos, O.rope_inv_freq(D, 10000.0))
    cos, sin = cos[:, None], sin[:, None]
    # fp32 angles up to ~5000 rad: allow a few ulp of the angle in cos/sin
    assert_close(qr.cpu(), O.rope_apply(q.cpu(), cos, sin), rtol=1e-4, atol=2e-4, what="q")
    assert_close(kr.cpu(), O.rope_apply(k.cpu(), cos, sin), rtol=1e-4, atol=2e-4, what="k")


def test_baseline_config_c2_full_size():
    """BASELINE configs[1] RoPE: q [8,16,2048,128], k [8,8,2048,128] bf16, positions
    0..2047, theta 5e6, cos/sin recomputed in-kernel; fwd + bwd."""
    from metal_liger_b200.ops.fused_rope import apply_fused_rotary_from_positions
    g = torch.Generator(device=DEV).manual_seed(1236)
    q = torch.randn(8, 16, 2048, 128, generator=g, device=DEV).bfloat16().requires_grad_(True)
    k = torch.randn(8, 8, 2048, 128, generator=g, device=DEV).bfloat16().requires_grad_(True)
    pos = torch.arange(2048, device=DEV).expand(8, 2048)
    qr, kr = apply_fused_rotary_from_positions(q, k, pos, theta=5e6)
    dq = torch.randn(qr.shape, generator=g, device=DEV).bfloat16()
    dk = torch.randn(kr.shape, generator=g, device=DEV).bfloat16()
    torch.autograd.backward([qr, kr], [dq, dk])
    cos, sin = O.rope_cos_sin(pos.cpu(), O.rope_inv_freq(128, 5e6))
    cos, sin = cos[:, None].to(DEV), sin[:, None].to(DEV)
    for got, exp, what in ((qr, O.rope_apply(q.detach(), cos, sin), "q"),
                           (kr, O.rope_apply(k.detach(), cos, sin), "k"),
                           (q.grad, O.rope_backward(dq, cos, sin), "dq"),
                           (k.grad, O.rope_backward(dk, cos, sin), "dk")):
        assert got.dtype == torch.bfloat16
        diff = (got.float() - exp).abs()
        bad = diff > 1e-2 + 2e-2 * exp.abs()
        assert not bad.any(), f"{what}: {int(bad.sum())} elements out of tolerance"


def test_bad_inputs_raise():
    x = torch.randn(1, 2, 4, 7, device=DEV)  # odd head_dim
    with pytest.raises(RuntimeError):
        torch.ops.metal_liger.rope_apply(x, torch.ones(4, 7, device=DEV),
                                         torch.ones(4, 7, device=DEV), 1)


@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float16])
def test_16bit_large_positions_accuracy(dt):
    """16-bit inputs evaluate cos/sin after a two-constant range reduction to
    [-pi, pi]; check against the fp32 oracle (torch cos/sin) for positions up to
    1e5, where an unreduced fast sin/cos would be visibly wrong."""
    from metal_liger_b200.ops.fused_rope import apply_fused_rotary_from_positions
    g = torch.Generator().manual_seed(5)
    q = torch.randn(2, 4, 64, 128, generator=g).to(dt)
    k = torch.randn(2, 2, 64, 128, generator=g).to(dt)
    pos = torch.randint(0, 100_000, (2, 64), generator=g)
    qr, kr = apply_fused_rotary_from_positions(q.to(DEV), k.to(DEV), pos.to(DEV), theta=10000.0)
    cos, sin = O.rope_cos_sin(pos, O.rope_inv_freq(128, 10000.0))
    cos, sin = cos[:, None], sin[:, None]
    rq = O.rope_apply(q, cos, sin)
    assert_close(qr.cpu(), rq, dtype=dt, what="q")
    # the error budget is dominated by the 16-bit output rounding, not cos/sin
    err = (qr.float().cpu() - rq).abs().max().item()
    assert err <= 2.0 ** -7 * rq.abs().max().item(), err
