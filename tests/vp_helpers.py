"""Test helpers for the vocabulary-parallel FLCE: oracle-based shard phases (CPU)
and a multi-process runner.  Test infrastructure only."""

import io
import os
import socket
import traceback

import torch


class OraclePhases:
    """ml_flce_shard_stats / _grads restated with the oracle's fp32 torch math."""

    def count(self, labels, ignore_index):
        n = (labels != ignore_index).sum().to(torch.float32)
        return torch.stack([n, 1.0 / torch.clamp(n, min=1.0)])

    def stats(self, hidden, weight, bias, labels, vocab_offset, ignore_index):
        logits = hidden.float() @ weight.float().t()
        if bias is not None:
            logits = logits + bias.float()
        m = logits.max(dim=-1).values
        s = torch.exp(logits - m[:, None]).sum(dim=-1)
        rel = labels - vocab_offset
        inside = (labels != ignore_index) & (rel >= 0) & (rel < weight.shape[0])
        t = torch.where(inside, logits.gather(1, rel.clamp(0, weight.shape[0] - 1)[:, None])[:, 0],
                        torch.zeros_like(m))
        return m, s, t, logits

    def grads(self, state, hidden, weight, labels, vocab_offset, ignore_index, lse, scale,
              dx_out, dw_out, dw_accumulate):
        mask = (labels != ignore_index).to(torch.float32)
        p = torch.exp(state - lse[:, None]) * (mask * scale)[:, None]
        rel = labels - vocab_offset
        inside = (labels != ignore_index) & (rel >= 0) & (rel < weight.shape[0])
        idx = torch.nonzero(inside)[:, 0]
        p[idx, rel[idx]] -= scale
        self._p = p
        if dx_out is not None:
            dx_out.copy_(p @ weight.float())
        if dw_out is not None:
            self.grads_dw(state, hidden, weight, dw_out, dw_accumulate)

    def grads_dw(self, state, hidden, weight, dw_out, dw_accumulate):
        g = self._p.t() @ hidden.float()
        if dw_accumulate:
            dw_out += g
        else:
            dw_out.copy_(g)


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def run_ranks(fn, world, port, backend, timeout_s, *args):
    """Spawn `world` processes running fn(rank, world, *args); returns per-rank results
    (or the formatted exception)."""
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_entry, args=(fn, r, world, port, backend, timeout_s, q, args))
             for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    for _ in range(world):
        rank, res = q.get(timeout=120)
        if isinstance(res, bytes):
            res = torch.load(io.BytesIO(res), weights_only=False)
        results[rank] = res
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    return results


def _entry(fn, rank, world, port, backend, timeout_s, q, args):
    import datetime

    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    try:
        kw = {}
        if backend == "nccl":
            torch.cuda.set_device(rank)
            kw["device_id"] = torch.device("cuda", rank)
        dist.init_process_group(backend, rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=timeout_s), **kw)
        res = fn(rank, world, *args)
        # results travel as serialised bytes: tensors put on the queue would be
        # shared through file descriptors that vanish when this process exits
        buf = io.BytesIO()
        torch.save(res, buf)
        q.put((rank, buf.getvalue()))
        dist.destroy_process_group()
    except Exception:  # report, never hang the parent
        q.put((rank, "ERROR: " + traceback.format_exc()))
