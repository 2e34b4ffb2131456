"""Vocabulary-parallel FLCE on 2+ GPUs against the single-GPU FLCE, with the
partial dX summed by NCCL or through peer memory (the dX GEMM storing into
the row owners' buffers; every rank then holds the bitwise same dX).

Needs at least two CUDA devices; skipped otherwise (the 1-GPU round-end run
skips it; the host logic is covered by tests/test_vocab_parallel.py on CPU
and the peer-memory exchange's kernels by tests/test_gpu_flce_p2p.py, which
emulates the ranks on one GPU).
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


def _rank_fn(rank, world, chunk, exchange="nccl"):
    import metal_liger_b200.ops.fused_linear_cross_entropy as F
    from metal_liger_b200.ops.fused_linear_cross_entropy import (
        _VocabParallelFLCEFunction, shard_lm_head)
    F.VP_DX_EXCHANGE = exchange
    dev = torch.device("cuda", rank)
    hid, w, lab = _problem(dev)
    ws, off = shard_lm_head(w, rank, world)
    h = hid.clone().requires_grad_(True)
    wsh = ws.clone().requires_grad_(True)
    loss = _VocabParallelFLCEFunction.apply(h, wsh, lab, None, off, -100, chunk, None)
    loss.backward(torch.tensor(1.5, device=dev))
    torch.cuda.synchronize()
    from metal_liger_b200 import _C
    return {"loss": loss.item(), "dx": h.grad.float().cpu(), "dw": wsh.grad.float().cpu(),
            "off": off, "err": int(_C.load().ml_device_error(None))}


@pytest.mark.parametrize("exchange", ["nccl", "p2p"])
@pytest.mark.parametrize("chunk", [1024, 8192])
def test_two_gpu_vocab_parallel_matches_single_gpu(chunk, exchange):
    from metal_liger_b200.ops.fused_linear_cross_entropy import _FusedLinearCrossEntropyFunction
    world = min(torch.cuda.device_count(), 2)
    res = run_ranks(_rank_fn, world, free_port(), "nccl", 60, chunk, exchange)
    for r in range(world):
        assert not isinstance(res[r], str), res[r]
        assert res[r]["err"] == 0, hex(res[r]["err"])
    # every rank ends with the same summed dX
    for r in range(1, world):
        if exchange == "p2p":
            assert torch.equal(res[r]["dx"], res[0]["dx"])
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
