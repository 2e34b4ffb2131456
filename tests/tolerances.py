"""Tolerances used by the parity tests (from the path's stated contract).

* fp32 paths: 1e-5 relative (plus a small absolute floor for values near 0);
* bf16 paths: 2e-2 relative / 1e-2 absolute against an fp32 reference;
* integer/bookkeeping quantities (ignore counts, masks): bit-exact.

``assert_close_rel`` also checks the relative Frobenius error, which keeps
tests meaningful when element values are far below the absolute floor.
"""

import torch

FP32_RTOL, FP32_ATOL = 1e-5, 1e-6
BF16_RTOL, BF16_ATOL = 2e-2, 1e-2


def tol_for(dtype):
    if dtype in (torch.bfloat16, torch.float16):
        return BF16_RTOL, BF16_ATOL
    return FP32_RTOL, FP32_ATOL


def rel_err(a, b):
    a = a.double()
    b = b.double()
    den = b.norm().item()
    return (a - b).norm().item() / (den if den > 0 else 1.0)


def assert_close(actual, expected, dtype=None, rtol=None, atol=None, norm_rtol=None, what=""):
    dtype = dtype or actual.dtype
    r, a = tol_for(dtype)
    rtol = r if rtol is None else rtol
    atol = a if atol is None else atol
    act = actual.detach().float().cpu()
    exp = expected.detach().float().cpu()
    assert act.shape == exp.shape, f"{what}: shape {tuple(act.shape)} != {tuple(exp.shape)}"
    diff = (act - exp).abs()
    bad = diff > atol + rtol * exp.abs()
    assert not bad.any(), (
        f"{what}: {int(bad.sum())} / {bad.numel()} elements out of tolerance "
        f"(rtol={rtol}, atol={atol}); max abs diff {diff.max().item():.3e}")
    if norm_rtol is not None:
        e = rel_err(act, exp)
        assert e <= norm_rtol, f"{what}: relative Frobenius error {e:.3e} > {norm_rtol}"
