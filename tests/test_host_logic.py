"""Host-side logic that needs no GPU: op registration, fake kernels, no-fallback policy."""

import sys

import pytest
import torch

import metal_liger_b200 as ml
from metal_liger_b200 import _torch_library as tl


def test_registration_is_idempotent():
    assert ml.register_metal_liger_ops() is True
    assert ml.register_metal_liger_ops() is True
    for name in tl.registered_op_names():
        assert hasattr(torch.ops.metal_liger, name)


def test_reference_schemas_kept():
    s = str(torch.ops.metal_liger.rms_norm_forward.default._schema)
    assert "Tensor x, Tensor weight, float eps, str kernel_dir" in s
    s = str(torch.ops.metal_liger.swiglu_forward.default._schema)
    assert "Tensor gate, Tensor up, str kernel_dir" in s


def test_fake_shapes_on_meta():
    x = torch.empty(3, 5, 16, device="meta", dtype=torch.bfloat16)
    w = torch.empty(16, device="meta")
    y, rrms = torch.ops.metal_liger.rms_norm_forward(x, w, 1e-6, "")
    assert y.shape == x.shape and y.dtype == x.dtype
    assert rrms.shape == (3, 5) and rrms.dtype == torch.float32
    q = torch.empty(2, 4, 8, 32, device="meta", dtype=torch.bfloat16)
    cos = torch.empty(8, 32, device="meta", dtype=torch.float32)
    out = torch.ops.metal_liger.rope_apply(q, cos, cos, 1)
    assert out.dtype == torch.float32  # torch promotion of x*cos, as in the reference


def test_fused_decode_op_fakes_on_meta():
    """The decoder-layer decode ops (fused norm / residual GEMVs, q/k prep +
    attention) propagate shapes on the meta device, as graph tracers need."""
    ops = torch.ops.metal_liger
    m = dict(device="meta", dtype=torch.bfloat16)
    x = torch.empty(2, 1, 64, **m)
    nw = torch.empty(64, **m)
    w1, w2 = torch.empty(48, 64, **m), torch.empty(16, 64, **m)
    assert ops.gemv_residual(x, w1, None, torch.empty(2, 1, 48, **m)).shape == (2, 1, 48)
    outs = ops.gemv_rmsnorm_multi(x, nw, 1e-6, [w1, w2], [None, None])
    assert [tuple(o.shape) for o in outs] == [(2, 1, 48), (2, 1, 16)]
    assert ops.gemv_rmsnorm_swiglu(x, nw, 1e-6, w1, w1).shape == (2, 1, 48)
    kc = torch.empty(2, 2, 40, 32, **m)
    q, kv = torch.empty(2, 1, 4 * 32, **m), torch.empty(2, 1, 2 * 32, **m)
    cs = torch.empty(2, 1, 32, **m)
    w = torch.empty(32, **m)
    pos = torch.empty(1, device="meta", dtype=torch.int64)
    out = ops.decode_qk_attention(q, kv, kv, w, w, 1e-6, 1e-6, cs, cs, kc, kc, pos, 0.2)
    assert out.shape == (2, 1, 4, 32)


@pytest.mark.parametrize("call", [
    lambda: torch.ops.metal_liger.gemv_residual(
        torch.randn(1, 64).bfloat16(), torch.randn(8, 64).bfloat16(), None,
        torch.randn(1, 8).bfloat16()),
    lambda: torch.ops.metal_liger.gemv_rmsnorm_swiglu(
        torch.randn(1, 64).bfloat16(), torch.ones(64).bfloat16(), 1e-6,
        torch.randn(8, 64).bfloat16(), torch.randn(8, 64).bfloat16()),
    lambda: torch.ops.metal_liger.gemv_rmsnorm_multi(
        torch.randn(1, 64).bfloat16(), torch.ones(64).bfloat16(), 1e-6,
        [torch.randn(8, 64).bfloat16()], [None]),
    lambda: torch.ops.metal_liger.rms_norm_forward(torch.randn(2, 8), torch.ones(8), 1e-6, ""),
    lambda: torch.ops.metal_liger.swiglu_forward(torch.randn(8), torch.randn(8), ""),
    lambda: ml.ops.fused_swiglu.fused_swiglu(torch.randn(8), torch.randn(8)),
])
def test_cpu_tensors_fail_loudly(call):
    with pytest.raises((NotImplementedError, RuntimeError)):
        call()


def test_install_alias():
    ml.install_as_metal_liger()
    import metal_liger  # noqa: F401
    assert sys.modules["metal_liger"] is ml
    from metal_liger.ops.fused_rms_norm import MetalLigerRMSNorm
    assert MetalLigerRMSNorm is ml.MetalLigerRMSNorm
    for k in [k for k in sys.modules if k == "metal_liger" or k.startswith("metal_liger.")]:
        del sys.modules[k]


def test_rms_module_repr_and_params():
    m = ml.MetalLigerRMSNorm(16, eps=1e-5)
    assert m.weight.shape == (16,)
    assert "hidden_size=16" in repr(m)


def test_lora_fakes_return_adapter_dtypes():
    x = torch.empty(2, 8, 64, device="meta", dtype=torch.bfloat16)
    w = torch.empty(32, 64, device="meta", dtype=torch.bfloat16)
    a = torch.empty(4, 64, device="meta", dtype=torch.bfloat16)
    b = torch.empty(32, 4, device="meta", dtype=torch.float32)
    y, u = torch.ops.metal_liger.lora_linear_forward(x, w, a, b, 2.0)
    assert y.shape == (16, 32) and u.shape == (16, 64)
    dx, da, db = torch.ops.metal_liger.lora_linear_backward(x, u, w, a, b, 2.0, y)
    assert dx.shape == x.shape and da.dtype == a.dtype and db.dtype == b.dtype
