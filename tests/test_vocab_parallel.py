"""Vocabulary-parallel FLCE host logic on CPU ranks (gloo, world size 2).

The collective orchestration (shard offsets, MAX/SUM merge of the per-row
statistics, dX all-reduce, local dW shards) runs with oracle-based shard
phases; the result must equal the single-process oracle.  A rank that leaves
before the collectives must make the other rank fail with an error, not hang.
"""

import pytest
import torch

from oracle import ops as O
from vp_helpers import OraclePhases, free_port, run_ranks


def _problem():
    g = torch.Generator().manual_seed(3)
    n, h, v = 40, 16, 101
    hid = torch.randn(n, h, generator=g)
    w = 0.3 * torch.randn(v, h, generator=g)
    lab = torch.randint(0, v, (n,), generator=g)
    lab[::7] = -100
    return hid, w, lab


def _rank_fn(rank, world, chunk, exchange="allreduce"):
    import metal_liger_b200.ops.fused_linear_cross_entropy as F
    from metal_liger_b200.ops.fused_linear_cross_entropy import shard_lm_head, \
        vocab_parallel_flce
    F.VP_STATS_EXCHANGE = exchange
    hid, w, lab = _problem()
    ws, off = shard_lm_head(w, rank, world)
    loss, dx, dw = vocab_parallel_flce(hid, ws, lab, off, chunk_size=chunk,
                                       phases=OraclePhases())
    return {"loss": loss, "dx": dx, "dw": dw, "off": off}


@pytest.mark.parametrize("exchange", ["allreduce", "allgather"])
@pytest.mark.parametrize("chunk", [16, 4096])
def test_gloo_two_ranks_match_single_process_oracle(chunk, exchange):
    """Both ways of merging the per-row statistics (two all-reduces, or one
    all-gather merged in rank order) give the single-process result."""
    res = run_ranks(_rank_fn, 2, free_port(), "gloo", 30, chunk, exchange)
    for r in (0, 1):
        assert not isinstance(res[r], str), res[r]
    hid, w, lab = _problem()
    rl, lse, mask = O.flce_forward(hid, w, lab, None, -100, 32)
    rdx, rdw = O.flce_backward(hid, w, lab, lse, mask, 1.0, None, 32)
    for r in (0, 1):
        assert torch.allclose(res[r]["loss"], rl, rtol=1e-5, atol=1e-6)
        assert torch.allclose(res[r]["dx"], rdx, rtol=1e-4, atol=1e-6)
    dw = torch.cat([res[0]["dw"], res[1]["dw"]])
    assert res[1]["off"] == res[0]["dw"].shape[0]
    assert torch.allclose(dw, rdw, rtol=1e-4, atol=1e-6)


def _leaver(rank, world):
    from metal_liger_b200.ops.fused_linear_cross_entropy import shard_lm_head, \
        vocab_parallel_flce
    if rank == 1:
        return "left"  # never joins the collectives
    hid, w, lab = _problem()
    ws, off = shard_lm_head(w, rank, world)
    vocab_parallel_flce(hid, ws, lab, off, chunk_size=16, phases=OraclePhases())
    return "completed"


def test_rank_that_leaves_makes_peer_fail_not_hang():
    res = run_ranks(_leaver, 2, free_port(), "gloo", 5)
    assert res[1] == "left"
    assert isinstance(res[0], str) and res[0].startswith("ERROR"), res[0]


def test_shard_split_covers_vocab():
    from metal_liger_b200.ops.fused_linear_cross_entropy import shard_lm_head
    w = torch.zeros(151936, 1)
    for world in (1, 2, 4, 8, 3):
        total = 0
        for r in range(world):
            s, off = shard_lm_head(w, r, world)
            assert off == total
            total += s.shape[0]
        assert total == 151936
