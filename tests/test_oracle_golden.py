"""Pin the CPU oracle against fixtures produced by the reference itself.

tests/golden/*.pt were written by tests/golden/make_golden.py, which runs the
reference's own autograd Functions (ops/*.py) on seeded inputs.  Here the
oracle (oracle/ops.py) is run on the same inputs and must reproduce them.
"""

import pytest
import torch
import torch.nn.functional as F

from conftest import golden_names, load_golden
from oracle import ops as O
from tolerances import assert_close


@pytest.mark.parametrize("name", golden_names("rms_"))
def test_rms_norm(name):
    d = load_golden(name)
    y, rrms = O.rms_norm_forward(d["x"], d["w"], float(d["eps"]))
    assert_close(y, d["y"], rtol=1e-5, atol=1e-5, what=f"{name} y")
    dx, dw = O.rms_norm_backward(d["x"], d["w"], rrms, d["dy"])
    assert_close(dx, d["dx"], rtol=1e-5, atol=1e-5, what=f"{name} dx")
    assert_close(dw, d["dw"], rtol=1e-4, atol=1e-4, what=f"{name} dw")


@pytest.mark.parametrize("name", golden_names("swiglu_"))
def test_swiglu(name):
    d = load_golden(name)
    out = O.swiglu_forward(d["gate"], d["up"])
    assert_close(out, d["out"], rtol=1e-5, atol=1e-6, what=f"{name} out")
    dg, du = O.swiglu_backward(d["gate"], d["up"], d["dy"])
    assert_close(dg, d["dgate"], rtol=1e-5, atol=1e-6, what=f"{name} dgate")
    assert_close(du, d["dup"], rtol=1e-5, atol=1e-6, what=f"{name} dup")


@pytest.mark.parametrize("name", golden_names("rope_"))
def test_rope(name):
    d = load_golden(name)
    y = O.rope_apply(d["x"], d["cos"], d["sin"])
    # The reference computes in the promoted dtype (bf16 inputs stay bf16);
    # the oracle computes in fp32, so compare at the dtype's tolerance.
    assert_close(y, d["y"].float(), dtype=d["y"].dtype, what=f"{name} y")
    dx = O.rope_backward(d["dy"], d["cos"], d["sin"])
    assert_close(dx, d["dx"].float(), dtype=d["dx"].dtype, what=f"{name} dx")


@pytest.mark.parametrize("name", golden_names("flce_"))
def test_flce(name):
    d = load_golden(name)
    bias = d.get("bias")
    loss, lse, mask = O.flce_forward(d["hidden"], d["weight"], d["labels"], bias, -100,
                                     int(d["chunk"]))
    assert_close(loss, d["loss"], rtol=1e-5, atol=1e-6, what=f"{name} loss")
    dx, dw = O.flce_backward(d["hidden"], d["weight"], d["labels"], lse, mask,
                             d["grad_output"], bias, int(d["chunk"]))
    assert_close(dx, d["dhidden"], rtol=1e-4, atol=1e-7, norm_rtol=1e-5, what=f"{name} dX")
    assert_close(dw, d["dweight"], rtol=1e-4, atol=1e-7, norm_rtol=1e-5, what=f"{name} dW")
    # bookkeeping is exact
    assert int(mask.sum()) == int((d["labels"] != -100).sum())


def test_flce_matches_cross_entropy():
    d = load_golden("flce_f32_bias")
    logits = d["hidden"] @ d["weight"].t() + d["bias"]
    ref = F.cross_entropy(logits.double(), d["labels"], ignore_index=-100)
    loss, _, _ = O.flce_forward(d["hidden"], d["weight"], d["labels"], d["bias"], -100, 128)
    assert abs(loss.item() - ref.item()) <= 1e-5 * abs(ref.item())


def test_flce_all_ignored_is_exactly_zero():
    d = load_golden("flce_f32_allign")
    assert d["loss"].item() == 0.0
    loss, _, _ = O.flce_forward(d["hidden"], d["weight"], d["labels"], None, -100, 128)
    assert loss.item() == 0.0


def _lora_tuple(d, name):
    return (d[f"{name}_w"], d[f"{name}_a"], d[f"{name}_b"], float(d["s"]))


@pytest.mark.parametrize("name", golden_names("lora_qkv"))
def test_lora_qkv(name):
    d = load_golden(name)
    q, k, v = (_lora_tuple(d, n) for n in ("q", "k", "v"))
    Q, K, V = O.lora_qkv_forward(d["x"], q, k, v)
    for got, key in ((Q, "Q"), (K, "K"), (V, "V")):
        assert_close(got, d[key], rtol=1e-5, atol=1e-5, what=f"{name} {key}")
    dx, grads = O.lora_qkv_backward(d["x"], q, k, v, d["dq"], d["dk"], d["dv"])
    assert_close(dx, d["dx"], rtol=1e-5, atol=1e-5, what=f"{name} dX")
    for (da, db), n in zip(grads, ("q", "k", "v")):
        assert_close(da, d[f"{n}_da"], rtol=1e-5, atol=1e-5, what=f"{name} d{n}A")
        assert_close(db, d[f"{n}_db"], rtol=1e-5, atol=1e-5, what=f"{name} d{n}B")


def test_lora_mlp():
    d = load_golden("lora_mlp_f32")
    g, u, dn = (_lora_tuple(d, n) for n in ("gate", "up", "down"))
    out, _, _, _ = O.lora_mlp_forward(d["x"], g, u, dn)
    assert_close(out, d["out"], rtol=1e-5, atol=1e-5, what="mlp out")
    dx, grads = O.lora_mlp_backward(d["x"], g, u, dn, d["dy"])
    assert_close(dx, d["dx"], rtol=1e-5, atol=1e-5, what="mlp dX")
    for (da, db), n in zip(grads, ("gate", "up", "down")):
        assert_close(da, d[f"{n}_da"], rtol=1e-5, atol=1e-5, what=f"mlp d{n}A")
        assert_close(db, d[f"{n}_db"], rtol=1e-5, atol=1e-5, what=f"mlp d{n}B")


def test_lora_qkv_matches_autograd():
    """The reference test's own check (tests/test_fused_ops.py:198-240), via the oracle."""
    d = load_golden("lora_qkv_f32")
    x = d["x"].clone().requires_grad_(True)
    params = {n: [d[f"{n}_w"].clone(), d[f"{n}_a"].clone().requires_grad_(True),
                  d[f"{n}_b"].clone().requires_grad_(True)] for n in ("q", "k", "v")}
    s = float(d["s"])
    outs = [x @ p[0].t() + (x @ p[1].t()) @ p[2].t() * s for p in params.values()]
    torch.autograd.backward(outs, [d["dq"], d["dk"], d["dv"]])
    assert_close(x.grad, d["dx"], rtol=1e-4, atol=1e-4, what="autograd dX")
    assert_close(params["q"][1].grad, d["q_da"], rtol=1e-4, atol=1e-4, what="autograd dQA")
