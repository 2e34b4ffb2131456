"""The vocabulary-parallel FLCE's peer-memory exchanges (softmax statistics
and dX), its ranks emulated on one GPU.

Each emulated rank has its own exchange buffer (all on this GPU, so the
"peer" stores are local) and its own vocabulary shard; the phases run in an
order where every wait finds its flags already set by earlier launches on
the stream (all ranks' statistics puts before any merge; all ranks' dX GEMMs,
then all owners' reductions, then all finishes), so no kernel waits on a
later one.  Every rank's merged statistics must be identical and equal the
rank-order merge.  The exchanged dX must equal,
bit for bit and on every rank, the rank-order sum of the shards' partial dX
from the plain shard GEMM (what the NCCL path all-reduces), for ragged
chunks and row blocks that leave an owner empty.  A wait whose flags nothing
sets must give up and report ML_ERR_TIMEOUT through the device error word.
"""

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _buffers(world, chunk, h):
    from metal_liger_b200 import _C

    lib = _C.load()
    nbytes = int(lib.ml_flce_p2p_workspace_bytes(world, chunk, h))
    assert nbytes > 0
    bufs = []
    for _ in range(world):
        p = ctypes.c_void_p()
        _C.call("ml_p2p_alloc", nbytes, ctypes.byref(p))
        bufs.append(p.value)
    return bufs, (ctypes.c_void_p * world)(*bufs)


def _free(bufs):
    from metal_liger_b200 import _C

    torch.cuda.synchronize()
    for b in bufs:
        _C.call("ml_p2p_free", b)


def _problem(n, h, v, seed):
    g = torch.Generator(device=DEV).manual_seed(seed)
    hid = torch.randn(n, h, generator=g, device=DEV).bfloat16()
    w = (0.02 * torch.randn(v, h, generator=g, device=DEV)).bfloat16()
    lab = torch.randint(0, v, (n,), generator=g, device=DEV)
    lab[::7] = -100
    return hid, w, lab


@pytest.mark.parametrize("world,n,h,v,chunk", [(2, 1000, 256, 3001, 600),
                                               (3, 1500, 128, 2000, 512),
                                               (4, 2048, 512, 5003, 2048),
                                               (8, 2304, 256, 4001, 2304)])
def test_exchange_equals_rank_order_sum_of_partials(world, n, h, v, chunk):
    from metal_liger_b200 import _C
    from metal_liger_b200.ops.fused_linear_cross_entropy import CudaShardPhases, shard_lm_head

    hid, w, lab = _problem(n, h, v, seed=world * 100 + n)
    phases = CudaShardPhases()
    cnt = phases.count(lab, -100)
    shards = [shard_lm_head(w, r, world) for r in range(world)]
    bufs, table = _buffers(world, chunk, h)
    st = torch.cuda.current_stream().cuda_stream
    out = [torch.full((n, h), float("nan"), device=DEV) for _ in range(world)]
    expect = torch.empty(n, h, device=DEV)
    epoch = 0
    try:
        for r0 in range(0, n, chunk):
            r1 = min(n, r0 + chunk)
            rows = r1 - r0
            hc, lc = hid[r0:r1], lab[r0:r1]
            stats = [phases.stats(hc, ws, None, lc, off, -100) for ws, off in shards]
            mg = torch.stack([m for m, _, _, _ in stats]).amax(0)
            sg = sum(s * torch.exp(m - mg) for m, s, _, _ in stats)
            tg = sum(t for _, _, t, _ in stats)
            epoch += 1
            # the statistics through peer memory: every rank's merge identical,
            # and equal to the rank-order merge above
            for r, (m, s_, t, _) in enumerate(stats):
                _C.call("ml_flce_p2p_stats_put", m.data_ptr(), s_.data_ptr(), t.data_ptr(), rows,
                        h, chunk, world, r, table, epoch, st)
            merged = []
            for r in range(world):
                out3 = [torch.empty(rows, device=DEV) for _ in range(3)]
                _C.call("ml_flce_p2p_stats_merge", rows, h, chunk, world, r, table, epoch,
                        *(o.data_ptr() for o in out3), st)
                merged.append(out3)
            for r in range(world):
                for a, b in zip(merged[r], merged[0]):
                    assert torch.equal(a, b), f"rank {r} merged statistics differ"
            assert torch.equal(merged[0][0], mg)
            assert torch.allclose(merged[0][1], sg, rtol=1e-6, atol=0)
            assert torch.allclose(merged[0][2], tg, rtol=1e-6, atol=1e-6)
            lse = (merged[0][0] + torch.log(merged[0][1])).contiguous()
            parts = []
            for (ws, off), (_, _, _, state) in zip(shards, stats):
                part = torch.empty(rows, h, device=DEV)
                phases.grads(state, hc, ws, lc, off, -100, lse, cnt[1:2], part, None, False)
                parts.append(part)
            acc = parts[0].clone()
            for part in parts[1:]:
                acc += part
            expect[r0:r1] = acc
            for r, ((ws, off), (_, _, _, state)) in enumerate(zip(shards, stats)):
                _C.call("ml_flce_shard_dx_p2p", ws.data_ptr(), rows, h, ws.shape[0],
                        state.data_ptr(), state.numel(), chunk, world, r, table, epoch, st)
            for r in range(world):
                _C.call("ml_flce_p2p_reduce", rows, h, chunk, world, r, table, epoch, st)
            for r in range(world):
                _C.call("ml_flce_p2p_finish", rows, h, chunk, world, r, table, epoch,
                        out[r][r0:r1].data_ptr(), st)
        torch.cuda.synchronize()
        assert _C.load().ml_device_error(None) == 0
        for r in range(world):
            assert torch.equal(out[r], expect), f"rank {r}"
    finally:
        _free(bufs)


def test_wait_with_no_arrivals_gives_up_and_reports_timeout():
    from metal_liger_b200 import _C

    lib = _C.load()
    assert lib.ml_device_error(None) == 0
    bufs, table = _buffers(2, 512, 128)
    try:
        st = torch.cuda.current_stream().cuda_stream
        # nothing raised epoch 1's arrive flags: the owner's wait runs out (2 s)
        _C.call("ml_flce_p2p_reduce", 512, 128, 512, 2, 0, table, 1, st)
        torch.cuda.synchronize()
        assert lib.ml_device_error(None) == (7 << 8) | 4
        assert lib.ml_device_error(None) == 0
        # the context stays usable
        x = torch.ones(4, device=DEV)
        assert float((x + x).sum()) == 8.0
    finally:
        _free(bufs)


def test_bad_arguments_are_refused_before_launch():
    from metal_liger_b200 import _C

    lib = _C.load()
    table = (ctypes.c_void_p * 2)(None, None)
    assert lib.ml_flce_p2p_reduce(512, 128, 512, 2, 0, table, 1, None) != 0
    assert lib.ml_flce_p2p_workspace_bytes(9, 512, 128) == 0
    assert lib.ml_flce_p2p_workspace_bytes(2, 0, 128) == 0
