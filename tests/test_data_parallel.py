"""Token-row data-parallel LoRA training step on CPU ranks (gloo, world size 2).

The C5 training step averages the adapter gradients over the ranks with
``metal_liger_b200.data_parallel.all_reduce_gradients`` (one all-reduce of
the flattened gradients).  Two ranks, each on half the token rows, must end
with the gradients — and, after an AdamW step, the adapter weights — of one
process stepping on the concatenated batch.  The shard phase is either a
PEFT-layout LoRA model run by autograd or the oracle's restatement of the
reference's fused LoRA QKV backward (ops/fused_lora.py:121-171).  A rank that
leaves before the collective must make its peer fail with an error, not hang.
"""

import pytest
import torch

from oracle import ops as O
from vp_helpers import free_port, run_ranks

T, H, OUT, R = 16, 24, 20, 4


def _model(seed=0):
    import torch.nn as nn

    from metal_liger_b200.lora_adapters import inject_lora

    torch.manual_seed(seed)
    m = nn.Sequential()
    m.add_module("q_proj", nn.Linear(H, OUT, bias=False))
    m.add_module("act", nn.Tanh())
    m.add_module("o_proj", nn.Linear(OUT, H, bias=False))
    inject_lora(m, r=R, alpha=8.0, targets=("q_proj", "o_proj"), init_std=0.3)
    return m


def _batch():
    g = torch.Generator().manual_seed(1)
    return torch.randn(T, H, generator=g), torch.randn(T, H, generator=g)


def _train_step(model, x, y):
    from metal_liger_b200.lora_adapters import lora_parameters

    loss = ((model(x) - y) ** 2).mean()
    loss.backward()
    return lora_parameters(model)


def _dp_rank(rank, world):
    from metal_liger_b200.data_parallel import all_reduce_gradients

    model = _model()
    x, y = _batch()
    rows = slice(rank * T // world, (rank + 1) * T // world)
    params = _train_step(model, x[rows], y[rows])
    n = all_reduce_gradients(params, check_sizes=True)
    grads = [p.grad.clone() for p in params]
    opt = torch.optim.AdamW(params, lr=1e-2)
    opt.step()
    return {"n": n, "grads": grads, "weights": [p.detach().clone() for p in params]}


def test_two_ranks_match_one_process_on_the_concatenated_batch():
    res = run_ranks(_dp_rank, 2, free_port(), "gloo", 30)
    for r in (0, 1):
        assert not isinstance(res[r], str), res[r]
    model = _model()
    x, y = _batch()
    params = _train_step(model, x, y)
    ref_grads = [p.grad.clone() for p in params]
    torch.optim.AdamW(params, lr=1e-2).step()
    assert res[0]["n"] == sum(p.numel() for p in params)
    for r in (0, 1):
        for got, ref in zip(res[r]["grads"], ref_grads):
            assert torch.allclose(got, ref, rtol=1e-5, atol=1e-7)
        for got, ref in zip(res[r]["weights"], params):
            assert torch.allclose(got, ref.detach(), rtol=1e-5, atol=1e-7)
    # both ranks hold bit-identical results (the same all-reduce output)
    for a, b in zip(res[0]["weights"], res[1]["weights"]):
        assert torch.equal(a, b)


def _qkv_problem():
    g = torch.Generator().manual_seed(5)
    x = torch.randn(T, H, generator=g)

    def proj(o):
        return (0.2 * torch.randn(o, H, generator=g), 0.3 * torch.randn(R, H, generator=g),
                0.3 * torch.randn(o, R, generator=g), 2.0)

    q, k, v = proj(OUT), proj(8), proj(8)
    dq = torch.randn(T, OUT, generator=g)
    dk = torch.randn(T, 8, generator=g)
    dv = torch.randn(T, 8, generator=g)
    return x, q, k, v, dq, dk, dv


def _oracle_rank(rank, world):
    """The shard phase is the oracle's LoRA QKV backward on this rank's rows,
    for a mean loss over those rows; the exchange is the package's."""
    from metal_liger_b200.data_parallel import all_reduce_gradients

    x, q, k, v, dq, dk, dv = _qkv_problem()
    n = T // world
    rows = slice(rank * n, (rank + 1) * n)
    _, grads = O.lora_qkv_backward(x[rows], q, k, v, dq[rows] / n, dk[rows] / n, dv[rows] / n)
    params = []
    for da, db in grads:
        for gtensor in (da, db):
            p = torch.nn.Parameter(torch.zeros_like(gtensor))
            p.grad = gtensor.clone()
            params.append(p)
    all_reduce_gradients(params)
    return [p.grad for p in params]


def test_oracle_shard_phase_matches_full_batch_oracle():
    res = run_ranks(_oracle_rank, 2, free_port(), "gloo", 30)
    for r in (0, 1):
        assert not isinstance(res[r], str), res[r]
    x, q, k, v, dq, dk, dv = _qkv_problem()
    _, grads = O.lora_qkv_backward(x, q, k, v, dq / T, dk / T, dv / T)
    ref = [g for pair in grads for g in pair]
    for r in (0, 1):
        for got, exp in zip(res[r], ref):
            assert torch.allclose(got, exp, rtol=1e-5, atol=1e-7)


def _leaver(rank, world):
    from metal_liger_b200.data_parallel import all_reduce_gradients

    if rank == 1:
        return "left"  # leaves between steps: never joins the gradient all-reduce
    model = _model()
    x, y = _batch()
    all_reduce_gradients(_train_step(model, x[:T // 2], y[:T // 2]))
    return "completed"


def test_rank_that_leaves_makes_peer_fail_not_hang():
    res = run_ranks(_leaver, 2, free_port(), "gloo", 5)
    assert res[1] == "left"
    assert isinstance(res[0], str) and res[0].startswith("ERROR"), res[0]


def _mismatch(rank, world):
    from metal_liger_b200.data_parallel import all_reduce_gradients

    p = torch.nn.Parameter(torch.zeros(4 + rank))
    p.grad = torch.ones(4 + rank)
    try:
        all_reduce_gradients([p], check_sizes=True)
    except RuntimeError as exc:
        return "raised: " + str(exc)
    return "reduced"


def test_mismatched_gradient_sets_raise_on_every_rank():
    res = run_ranks(_mismatch, 2, free_port(), "gloo", 30)
    for r in (0, 1):
        assert isinstance(res[r], str) and res[r].startswith("raised"), res[r]


@pytest.mark.parametrize("average", [True, False])
def test_single_rank_group_is_identity_or_sum(average):
    res = run_ranks(_single, 1, free_port(), "gloo", 30, average)
    assert not isinstance(res[0], str), res[0]
    assert torch.equal(res[0], torch.arange(6.0))


def _single(rank, world, average):
    from metal_liger_b200.data_parallel import all_reduce_gradients

    p = torch.nn.Parameter(torch.zeros(6))
    p.grad = torch.arange(6.0)
    all_reduce_gradients([p], average=average)
    return p.grad
