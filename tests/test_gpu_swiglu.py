"""SwiGLU CUDA parity: reference fixtures, reference-test shapes, BASELINE config 1."""

import pytest
import torch
import torch.nn.functional as F

from conftest import golden_names, load_golden
from oracle import ops as O
from tolerances import assert_close

pytestmark = pytest.mark.gpu
DEV = "cuda"


def run_fused(gate, up, dy):
    from metal_liger_b200.ops.fused_swiglu import fused_swiglu
    gl = gate.detach().clone().to(DEV).requires_grad_(True)
    ul = up.detach().clone().to(DEV).requires_grad_(True)
    out = fused_swiglu(gl, ul)
    out.backward(dy.to(DEV))
    torch.cuda.synchronize()
    return out.detach(), gl.grad, ul.grad


@pytest.mark.parametrize("name", golden_names("swiglu_"))
def test_against_reference_fixture(name):
    d = load_golden(name)
    out, dg, du = run_fused(d["gate"], d["up"], d["dy"])
    dt = d["gate"].dtype
    kw = dict(rtol=1e-5, atol=1e-6) if dt == torch.float32 else {}
    assert_close(out.cpu(), d["out"].float(), dtype=dt, what="out", **kw)
    assert_close(dg.cpu(), d["dgate"].float(), dtype=dt, what="dgate", **kw)
    assert_close(du.cpu(), d["dup"].float(), dtype=dt, what="dup", **kw)


def test_reference_test_shapes():
    """tests/test_fused_ops.py:94-136: fwd [4,128,5120], bwd [2,16,512] vs F.silu(g)*u."""
    g = torch.Generator().manual_seed(3)
    gate = torch.randn(4, 128, 5120, generator=g)
    up = torch.randn(4, 128, 5120, generator=g)
    out, _, _ = run_fused(gate, up, torch.zeros_like(gate))
    assert torch.allclose(F.silu(gate) * up, out.cpu(), atol=1e-5, rtol=1e-4)
    gate = torch.randn(2, 16, 512, generator=g, requires_grad=True)
    up = torch.randn(2, 16, 512, generator=g, requires_grad=True)
    (F.silu(gate) * up).sum().backward()
    _, dg, du = run_fused(gate, up, torch.ones(2, 16, 512))
    assert torch.allclose(gate.grad, dg.cpu(), atol=1e-4, rtol=1e-3)
    assert torch.allclose(up.grad, du.cpu(), atol=1e-4, rtol=1e-3)


def test_baseline_config_c2_full_size():
    """BASELINE configs[1] SwiGLU: gate/up [8,2048,6144] bf16 ~N(0,1), dY ~N(0,1).

    The fp32 oracle runs on the GPU here (it is plain tensor math) to keep the
    test fast; it is the same code the CPU pin checks against the reference.
    """
    g = torch.Generator(device=DEV).manual_seed(1235)
    gate = torch.randn(8, 2048, 6144, generator=g, device=DEV).bfloat16()
    up = torch.randn(8, 2048, 6144, generator=g, device=DEV).bfloat16()
    dy = torch.randn(8, 2048, 6144, generator=g, device=DEV).bfloat16()
    out, dg, du = run_fused(gate, up, dy)
    ref = O.swiglu_forward(gate, up, dtype=torch.float64)
    rdg, rdu = O.swiglu_backward(gate, up, dy, dtype=torch.float64)
    for got, exp, what in ((out, ref, "out"), (dg, rdg, "dgate"), (du, rdu, "dup")):
        assert got.dtype == torch.bfloat16
        diff = (got.double() - exp).abs()
        bad = diff > 1e-2 + 2e-2 * exp.abs()
        assert not bad.any(), f"{what}: {int(bad.sum())} elements out of tolerance"
    del gate, up, dy, out, dg, du, ref, rdg, rdu
    torch.cuda.empty_cache()


@pytest.mark.parametrize("n", [1, 7, 8, 9, 4097, 65537])
@pytest.mark.parametrize("dt", [torch.float32, torch.bfloat16, torch.float16])
def test_ragged_sizes(n, dt):
    g = torch.Generator().manual_seed(n)
    gate = (3 * torch.randn(n, generator=g)).to(dt)
    up = torch.randn(n, generator=g).to(dt)
    dy = torch.randn(n, generator=g).to(dt)
    out, dg, du = run_fused(gate, up, dy)
    ro = O.swiglu_forward(gate, up)
    rdg, rdu = O.swiglu_backward(gate, up, dy)
    kw = dict(rtol=1e-5, atol=1e-6) if dt == torch.float32 else {}
    assert_close(out.cpu(), ro.float(), dtype=dt, what="out", **kw)
    assert_close(dg.cpu(), rdg.float(), dtype=dt, what="dgate", **kw)
    assert_close(du.cpu(), rdu.float(), dtype=dt, what="dup", **kw)


def test_extreme_gate_values():
    gate = torch.tensor([-1e4, -100.0, -20.0, 0.0, 20.0, 100.0, 1e4, float("-inf")], device=DEV)
    up = torch.ones_like(gate)
    out, dg, du = run_fused(gate, up, torch.ones_like(gate))
    assert torch.isfinite(out[:-1]).all()
    ref = O.swiglu_forward(gate.cpu(), up.cpu())
    assert_close(out[:-1].cpu(), ref[:-1], rtol=1e-5, atol=1e-6, what="out")


def test_unaligned_views():
    base = torch.randn(1 + 4099, device=DEV, dtype=torch.bfloat16)
    gate = base[1:]            # 2-byte offset: not 16-byte aligned
    up = torch.randn(4099, device=DEV, dtype=torch.bfloat16)
    from metal_liger_b200.ops.fused_swiglu import fused_swiglu
    out = fused_swiglu(gate, up)
    ref = O.swiglu_forward(gate.cpu(), up.cpu())
    assert_close(out.cpu(), ref.float(), dtype=torch.bfloat16, what="out")


def test_ext_mirror_and_module():
    from metal_liger_b200 import metal_liger_ext as ext
    from metal_liger_b200.ops.fused_swiglu import MetalLigerSwiGLU
    gate = torch.randn(64, 96, device=DEV)
    up = torch.randn(64, 96, device=DEV)
    dy = torch.randn(64, 96, device=DEV)
    out = ext.swiglu_forward(gate, up, "")
    dg, du = ext.swiglu_backward(gate, up, dy, "")
    assert_close(out.cpu(), O.swiglu_forward(gate.cpu(), up.cpu()), rtol=1e-5, atol=1e-6)
    rdg, rdu = O.swiglu_backward(gate.cpu(), up.cpu(), dy.cpu())
    assert_close(dg.cpu(), rdg, rtol=1e-5, atol=1e-6)
    assert_close(du.cpu(), rdu, rtol=1e-5, atol=1e-6)

    class MLP(torch.nn.Module):
        def __init__(self):
            super().__init__()
            self.gate_proj = torch.nn.Linear(16, 32, bias=False)
            self.up_proj = torch.nn.Linear(16, 32, bias=False)
            self.down_proj = torch.nn.Linear(32, 16, bias=False)

    mlp = MLP().to(DEV)
    x = torch.randn(4, 16, device=DEV)
    fused = MetalLigerSwiGLU(mlp)
    ref = mlp.down_proj(F.silu(mlp.gate_proj(x)) * mlp.up_proj(x))
    assert_close(fused(x).detach().cpu(), ref.detach().cpu(), rtol=1e-5, atol=1e-5)
