"""Vocabulary-parallel FLCE on 2+ GPUs (NCCL) against the single-GPU FLCE.

Needs at least two CUDA devices; skipped otherwise (the 1-GPU round-end run
skips it; the host logic is covered by tests/test_vocab_parallel.py on CPU).
"""

import pytest
import torch

from vp_helpers import free_port, run_ranks

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs >= 2 GPUs")]


def _problem(device):
    g = torch.Generator(device=device).manual_seed(11)
    n, h, v = 3000, 512, 20011
    hid = torch.randn(n, h, generator=g, device=device).bfloat16()
    w = (0.02 * torch.randn(v, h, generator=g, device=device)).bfloat16()
    lab = torch.randint(0, v, (n,), generator=g, device=device)
    lab[::10] = -100
    return hid, w, lab


def _rank_fn(rank, world, chunk):
    from metal_liger_b200.ops.fused_linear_cross_entropy import (
        _VocabParallelFLCEFunction, shard_lm_head)
    dev = torch.device("cuda", rank)
    hid, w, lab = _problem(dev)
    ws, off = shard_lm_head(w, rank, world)
    h = hid.clone().requires_grad_(True)
    wsh = ws.clone().requires_grad_(True)
    loss = _VocabParallelFLCEFunction.apply(h, wsh, lab, None, off, -100, chunk, None)
    loss.backward(torch.tensor(1.5, device=dev))
    torch.cuda.synchronize()
    return {"loss": loss.item(), "dx": h.grad.float().cpu(), "dw": wsh.grad.float().cpu(),
            "off": off}


@pytest.mark.parametrize("chunk", [1024, 8192])
def test_two_gpu_vocab_parallel_matches_single_gpu(chunk):
    from metal_liger_b200.ops.fused_linear_cross_entropy import _FusedLinearCrossEntropyFunction
    world = min(torch.cuda.device_count(), 2)
    res = run_ranks(_rank_fn, world, free_port(), "nccl", 60, chunk)
    for r in range(world):
        assert not isinstance(res[r], str), res[r]
    hid, w, lab = _problem(torch.device("cuda", 0))
    h = hid.clone().requires_grad_(True)
    wf = w.clone().requires_grad_(True)
    loss = _FusedLinearCrossEntropyFunction.apply(h, wf, lab, None, -100, chunk)
    loss.backward(torch.tensor(1.5, device="cuda:0"))
    for r in range(world):
        assert abs(res[r]["loss"] - loss.item()) <= 1e-5 * abs(loss.item())
        rel = (res[r]["dx"] - h.grad.float().cpu()).norm() / h.grad.float().norm().cpu()
        assert rel.item() < 1e-2, rel.item()
    dw = torch.cat([res[r]["dw"] for r in range(world)])
    rel = (dw - wf.grad.float().cpu()).norm() / wf.grad.float().norm().cpu()
    assert rel.item() < 1e-2, rel.item()
