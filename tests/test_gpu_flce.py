"""Fused linear cross-entropy CUDA parity.

bf16 inputs run the fused kernels (bf16 operands, fp32 accumulation) and are
compared at the bf16 tolerance against an fp32 reference of the same inputs:
2e-2 relative / 1e-2 absolute element-wise, plus a relative Frobenius bound
(the gradients are scaled by 1/n_valid and would pass any absolute bound);
the loss at 1e-4 relative.  fp32 inputs (the reference fixtures) take the
fp32-accurate path (three-part bf16 splits, six GEMM products) and are held to 1e-5 relative on
the loss and 1e-4 relative Frobenius on the gradients.  Ignore counts are
exact (the all-ignored loss is exactly 0).
"""

import pytest
import torch
import torch.nn.functional as F

from conftest import golden_names, load_golden
from oracle import ops as O
from tolerances import assert_close

pytestmark = pytest.mark.gpu
DEV = "cuda"


def run_flce(hidden, weight, labels, bias=None, chunk=8192, grad_output=1.0, need=(True, True)):
    from metal_liger_b200.ops.fused_linear_cross_entropy import _FusedLinearCrossEntropyFunction
    h = hidden.detach().clone().to(DEV).requires_grad_(need[0])
    w = weight.detach().clone().to(DEV).requires_grad_(need[1])
    b = bias.to(DEV) if bias is not None else None
    loss = _FusedLinearCrossEntropyFunction.apply(h, w, labels.to(DEV), b, -100, chunk)
    go = torch.as_tensor(grad_output, dtype=torch.float32, device=DEV)
    loss.backward(go)
    torch.cuda.synchronize()
    return loss.detach(), h.grad, w.grad


def check_grads(dx, dw, rdx, rdw, norm=2e-2, what=""):
    assert_close(dx, rdx.float(), dtype=torch.bfloat16, norm_rtol=norm, what=f"{what} dX")
    assert_close(dw, rdw.float(), dtype=torch.bfloat16, norm_rtol=norm, what=f"{what} dW")


@pytest.mark.parametrize("name", golden_names("flce_"))
def test_against_reference_fixture(name):
    d = load_golden(name)
    loss, dx, dw = run_flce(d["hidden"], d["weight"], d["labels"], d.get("bias"),
                            chunk=int(d["chunk"]), grad_output=d["grad_output"].item())
    if name.endswith("allign"):
        assert loss.item() == 0.0
        assert dx.abs().max().item() == 0.0 and dw.abs().max().item() == 0.0
        return
    assert abs(loss.item() - d["loss"].item()) <= 1e-5 * abs(d["loss"].item())
    assert dx.dtype == torch.float32 and dw.dtype == torch.float32
    for got, exp, what in ((dx.cpu(), d["dhidden"], "dX"), (dw.cpu(), d["dweight"], "dW")):
        rel = ((got - exp.float()).norm() / exp.float().norm()).item()
        assert rel <= 1e-4, f"{name} {what}: relative Frobenius error {rel:.3e}"
        assert torch.allclose(got, exp.float(), rtol=1e-3, atol=1e-6), f"{name} {what}"


def _bf16_case(n, h, v, seed, ignore_frac=0.1):
    g = torch.Generator().manual_seed(seed)
    hid = torch.randn(n, h, generator=g).bfloat16()
    w = (0.02 * torch.randn(v, h, generator=g)).bfloat16()
    lab = torch.randint(0, v, (n,), generator=g)
    k = int(round(ignore_frac * n))
    lab[torch.randperm(n, generator=g)[:k]] = -100
    return hid, w, lab


@pytest.mark.parametrize("n,h,v,chunk", [(1000, 256, 5000, 384), (130, 64, 300, 8192),
                                         (256, 128, 2048, 100),
                                         (77, 100, 1001, 32)])   # hidden not a multiple of 8
def test_bf16_against_oracle(n, h, v, chunk, pair_mode):
    hid, w, lab = _bf16_case(n, h, v, seed=n + v)
    loss, dx, dw = run_flce(hid, w, lab, chunk=chunk, grad_output=0.75)
    rl, lse, mask = O.flce_forward(hid, w, lab, None, -100, 4096)
    rdx, rdw = O.flce_backward(hid, w, lab, lse, mask, 0.75, None, 4096)
    assert abs(loss.item() - rl.item()) <= 1e-4 * abs(rl.item())
    assert dx.dtype == torch.bfloat16 and dw.dtype == torch.bfloat16
    check_grads(dx.cpu(), dw.cpu(), rdx, rdw, what="bf16")
    # F.cross_entropy agrees too
    ref = F.cross_entropy((hid.float() @ w.float().t()), lab, ignore_index=-100)
    assert abs(loss.item() - ref.item()) <= 1e-4 * abs(ref.item())


def test_result_independent_of_chunk():
    hid, w, lab = _bf16_case(777, 128, 3001, seed=5)
    l1, dx1, dw1 = run_flce(hid, w, lab, chunk=100)
    l2, dx2, dw2 = run_flce(hid, w, lab, chunk=8192)
    assert abs(l1.item() - l2.item()) <= 1e-6 * abs(l2.item())
    assert_close(dx1.float(), dx2.float(), rtol=1e-2, atol=1e-6, norm_rtol=1e-3, what="dX")
    assert_close(dw1.float(), dw2.float(), rtol=1e-2, atol=1e-6, norm_rtol=1e-3, what="dW")


def test_no_grad_variants_and_bias():
    hid, w, lab = _bf16_case(200, 64, 1000, seed=9)
    bias = 0.1 * torch.randn(1000)
    loss, dx, dw = run_flce(hid, w, lab, bias=bias, need=(True, False))
    assert dw is None
    rl, lse, mask = O.flce_forward(hid, w, lab, bias, -100, 512)
    rdx, rdw = O.flce_backward(hid, w, lab, lse, mask, 1.0, bias, 512)
    assert abs(loss.item() - rl.item()) <= 1e-4 * abs(rl.item())
    assert_close(dx.cpu(), rdx.float(), dtype=torch.bfloat16, norm_rtol=2e-2, what="dX")
    loss2, dx2, dw2 = run_flce(hid, w, lab, bias=bias, need=(False, True))
    assert dx2 is None and loss2.item() == loss.item()
    assert_close(dw2.cpu(), rdw.float(), dtype=torch.bfloat16, norm_rtol=2e-2, what="dW")


def test_ignore_bookkeeping_exact():
    hid, w, lab = _bf16_case(300, 64, 500, seed=11, ignore_frac=0.5)
    lab[:10] = -100
    loss, dx, dw = run_flce(hid, w, lab)
    ignored = lab == -100
    assert dx[ignored.to(DEV)].abs().max().item() == 0.0  # ignored rows get no gradient
    rl, _, mask = O.flce_forward(hid, w, lab, None, -100, 512)
    assert int(mask.sum()) == int((~ignored).sum())
    assert abs(loss.item() - rl.item()) <= 1e-4 * abs(rl.item())


def _gpu_reference(hid, w, lab):
    """The pinned oracle (oracle.ops.flce_forward / flce_backward, the
    reference's vocab-chunked algorithm in fp32) evaluated on the GPU's
    tensors, TF32 off.  Returns (loss, dX, dW) in fp32."""
    torch.backends.cuda.matmul.allow_tf32 = False
    hf, wf = hid.float(), w.float()
    loss, lse, mask = O.flce_forward(hf, wf, lab, None, -100, 8192)
    dx, dw = O.flce_backward(hf, wf, lab, lse, mask, 1.0, None, 8192)
    return loss, dx, dw


def test_baseline_config_c3_full_size():
    """hidden [16384,2048] ~N(0,1), W [151936,2048] ~N(0,0.02) bf16,
    labels uniform with 10% = -100, mean over non-ignored, chunk 8192 tokens."""
    torch.backends.cuda.matmul.allow_tf32 = False
    g = torch.Generator(device=DEV).manual_seed(1236)
    n, h, v = 16384, 2048, 151936
    hid = torch.randn(n, h, generator=g, device=DEV).bfloat16()
    w = (0.02 * torch.randn(v, h, generator=g, device=DEV)).bfloat16()
    lab = torch.randint(0, v, (n,), generator=g, device=DEV)
    lab[torch.randperm(n, generator=g, device=DEV)[: n // 10]] = -100
    loss, dx, dw = run_flce(hid, w, lab, chunk=8192)
    rl, rdx, rdw = _gpu_reference(hid, w, lab)
    assert abs(loss.item() - rl.item()) <= 1e-4 * abs(rl.item()), (loss.item(), rl.item())
    for got, ref, what in ((dx, rdx, "dX"), (dw, rdw, "dW")):
        diff = (got.float() - ref).abs()
        bad = diff > 1e-2 + 2e-2 * ref.abs()
        assert not bad.any(), f"{what}: {int(bad.sum())} elements out of tolerance"
        # the gradients carry 1/n_valid, so also hold the absolute term to
        # 1e-2 of the tensor's largest magnitude rather than 1e-2 outright
        bad = diff > 1e-2 * ref.abs().max() + 2e-2 * ref.abs()
        assert not bad.any(), f"{what}: {int(bad.sum())} elements out of the scaled tolerance"
        rel = (got.float() - ref).norm() / ref.norm()
        assert rel.item() < 2e-2, f"{what}: relative Frobenius error {rel.item():.3e}"
    # size-independent property: each valid row of P sums to zero, so the
    # column sums of dW = P^T h vanish (up to rounding)
    colsum = dw.float().sum(0)
    assert colsum.norm().item() <= 1e-2 * dw.float().norm().item()
    del hid, w, dx, dw, rdx, rdw
    torch.cuda.empty_cache()


def test_module_matches_function():
    from metal_liger_b200.ops.fused_linear_cross_entropy import MetalLigerFusedLinearCrossEntropy
    lm_head = torch.nn.Linear(64, 700, bias=False).to(DEV).bfloat16()
    mod = MetalLigerFusedLinearCrossEntropy(lm_head)
    hs = torch.randn(2, 50, 64, device=DEV).bfloat16()
    lab = torch.randint(0, 700, (2, 50), device=DEV)
    loss = mod(hs, lab)
    ref = F.cross_entropy((hs.float().reshape(-1, 64) @ lm_head.weight.float().t()),
                          lab.reshape(-1), ignore_index=-100)
    assert abs(loss.item() - ref.item()) <= 1e-4 * ref.item()


def test_fp32_inputs_take_the_accurate_path():
    """fp32 hidden/weight: three-part bf16 splits (six GEMM products) give ~fp32 products; compared
    with the fp32 torch reference (TF32 off) at 1e-5 / 1e-4."""
    torch.backends.cuda.matmul.allow_tf32 = False
    g = torch.Generator(device=DEV).manual_seed(21)
    n, h, v = 1000, 256, 5000
    hid = torch.randn(n, h, generator=g, device=DEV)
    w = 0.05 * torch.randn(v, h, generator=g, device=DEV)
    lab = torch.randint(0, v, (n,), generator=g, device=DEV)
    lab[:100] = -100
    loss, dx, dw = run_flce(hid, w, lab, chunk=384)
    rl, rdx, rdw = _gpu_reference(hid, w, lab)
    assert abs(loss.item() - rl.item()) <= 1e-5 * abs(rl.item()), (loss.item(), rl.item())
    for got, ref, what in ((dx, rdx, "dX"), (dw, rdw, "dW")):
        rel = ((got - ref).norm() / ref.norm()).item()
        assert rel <= 1e-4, f"{what}: relative Frobenius error {rel:.3e}"
