"""Fused linear + cross-entropy on B200 — drop-in for ops/fused_linear_cross_entropy.py.

Same names and signatures as the reference (`_FusedLinearCrossEntropyFunction.apply(
hidden, weight, labels, bias=None, ignore_index=-100, chunk_size=8192)`,
`MetalLigerFusedLinearCrossEntropy(lm_head, ignore_index, chunk_size)`;
reference ops/fused_linear_cross_entropy.py:82-230) and the same result: the
mean cross-entropy over non-ignored rows, no gradient for the bias.

How it runs (one ``metal_liger::flce_forward`` call): the tokens are processed
in chunks of ``chunk_size`` rows; per chunk one tcgen05 logits GEMM writes
exp(logit - tile max) with fused per-tile max / sum-exp / target-logit
epilogues, a small kernel merges them into the log-sum-exp, the buffer is
turned into (softmax - onehot) / n_valid in place, and two more tcgen05 GEMMs
read it for dX = P W and dW += P^T h.  Every logit is computed once (the
reference recomputes all of them in backward) and the [N, V] logits never
exist.  The gradients are formed during the forward at grad_output = 1 and
scaled by the real grad_output in backward (they are linear in it).

``chunk_size`` is the token-chunk length here (the reference's argument of
the same name chunks the vocabulary); results do not depend on it.  Inputs
enter the tensor cores as bf16.
"""

import torch
import torch.nn as nn

import metal_liger_b200._torch_library  # noqa: F401  (registers metal_liger:: ops)
from metal_liger_b200._C import DTYPE_CODES


class _FusedLinearCrossEntropyFunction(torch.autograd.Function):
    """Chunked linear + cross-entropy that never materialises the full logits."""

    @staticmethod
    def forward(ctx, hidden: torch.Tensor, weight: torch.Tensor, labels: torch.Tensor,
                bias: torch.Tensor = None, ignore_index: int = -100, chunk_size: int = 8192):
        need_dx = bool(ctx.needs_input_grad[0])
        need_dw = bool(ctx.needs_input_grad[1])
        loss, dx, dw = torch.ops.metal_liger.flce_forward(
            hidden, weight, labels, bias, int(ignore_index), int(chunk_size), need_dx, need_dw)
        ctx.save_for_backward(dx, dw)
        ctx.hidden_shape = hidden.shape
        ctx.codes = (DTYPE_CODES.get(hidden.dtype, 0), DTYPE_CODES.get(weight.dtype, 0))
        return loss

    @staticmethod
    def backward(ctx, grad_output: torch.Tensor):
        dx, dw = ctx.saved_tensors
        gh, gw = torch.ops.metal_liger.flce_backward(grad_output, dx, dw, ctx.codes[0],
                                                     ctx.codes[1])
        grad_hidden = gh.view(ctx.hidden_shape) if ctx.needs_input_grad[0] else None
        grad_weight = gw if ctx.needs_input_grad[1] else None
        return grad_hidden, grad_weight, None, None, None, None


class MetalLigerFusedLinearCrossEntropy(nn.Module):
    """Fused lm_head + cross-entropy loss (reference ops/fused_linear_cross_entropy.py:188-230).

    Args:
        lm_head: the language-model head linear layer (its weight/bias are shared)
        ignore_index: label to ignore (default -100)
        chunk_size: token-chunk length (default 8192)
    """

    def __init__(self, lm_head: nn.Linear, ignore_index: int = -100, chunk_size: int = 8192):
        super().__init__()
        self.weight = lm_head.weight
        self.bias = lm_head.bias
        self.ignore_index = ignore_index
        self.chunk_size = chunk_size

    def forward(self, hidden_states: torch.Tensor, labels: torch.Tensor) -> torch.Tensor:
        batch_seq = (hidden_states.shape[0] * hidden_states.shape[1]
                     if hidden_states.ndim == 3 else hidden_states.shape[0])
        hidden_flat = hidden_states.reshape(batch_seq, -1)
        labels_flat = labels.reshape(-1)
        return _FusedLinearCrossEntropyFunction.apply(
            hidden_flat, self.weight, labels_flat, self.bias, self.ignore_index, self.chunk_size)


# ---------------------------------------------------------------------------
# Vocabulary-parallel FLCE (lm_head sharded by vocabulary rows across ranks)
# ---------------------------------------------------------------------------

def shard_lm_head(weight: torch.Tensor, rank: int, world: int):
    """(weight[v0:v1], v0): this rank's contiguous vocabulary shard (row split as even as
    possible; earlier ranks get the remainder)."""
    v = weight.shape[0]
    base, rem = divmod(v, world)
    v0 = rank * base + min(rank, rem)
    v1 = v0 + base + (1 if rank < rem else 0)
    return weight[v0:v1], v0


class CudaShardPhases:
    """The two per-chunk phases on this GPU (ml_flce_shard_stats / _grads)."""

    def count(self, labels, ignore_index):
        from metal_liger_b200 import _C
        out = torch.empty(2, dtype=torch.float32, device=labels.device)
        _C.call("ml_flce_count_valid", labels.data_ptr(), labels.numel(), int(ignore_index),
                out.data_ptr(), _C.stream_of(labels))
        return out

    def stats(self, hidden, weight, bias, labels, vocab_offset, ignore_index):
        from metal_liger_b200 import _C
        rows, h = hidden.shape
        v_local = weight.shape[0]
        lib = _C.load()
        nbytes = int(lib.ml_flce_shard_workspace_bytes(rows, v_local))
        ws = torch.empty(nbytes, dtype=torch.uint8, device=hidden.device)
        m = torch.empty(rows, dtype=torch.float32, device=hidden.device)
        s = torch.empty_like(m)
        t = torch.empty_like(m)
        _C.call("ml_flce_shard_stats", hidden.data_ptr(), weight.data_ptr(),
                bias.data_ptr() if bias is not None else None,
                _C.dtype_code(bias) if bias is not None else 0, labels.data_ptr(), rows, h,
                v_local, int(vocab_offset), int(ignore_index), m.data_ptr(), s.data_ptr(),
                t.data_ptr(), ws.data_ptr(), nbytes, _C.stream_of(hidden))
        return m, s, t, ws

    def grads(self, state, hidden, weight, labels, vocab_offset, ignore_index, lse, scale,
              dx_out, dw_out, dw_accumulate):
        from metal_liger_b200 import _C
        rows, h = hidden.shape
        _C.call("ml_flce_shard_grads", hidden.data_ptr(), weight.data_ptr(), labels.data_ptr(),
                rows, h, weight.shape[0], int(vocab_offset), int(ignore_index), lse.data_ptr(),
                scale.data_ptr(), dx_out.data_ptr() if dx_out is not None else None,
                dw_out.data_ptr() if dw_out is not None else None, int(dw_accumulate),
                state.data_ptr(), state.numel(), _C.stream_of(hidden))

    def grads_dw(self, state, hidden, weight, dw_out, dw_accumulate):
        """The dW GEMM alone, after grads(..., dw_out=None, ...) on the same state."""
        from metal_liger_b200 import _C
        rows, h = hidden.shape
        _C.call("ml_flce_shard_grads_dw", hidden.data_ptr(), rows, h, weight.shape[0],
                dw_out.data_ptr(), int(dw_accumulate), state.data_ptr(), state.numel(),
                _C.stream_of(hidden))


# How the vocabulary-parallel FLCE runs its collectives (process-wide):
# * VP_STATS_EXCHANGE: "allreduce" merges the per-row statistics with two
#   all-reduces (MAX of the maxima, then SUM of the rescaled sums and target
#   logits); "allgather" gathers every rank's (max, sum, target) in one
#   collective and merges them locally in rank order.
# * VP_OVERLAP_SMS: SMs the GEMMs leave free while a chunk's asynchronous dX
#   all-reduce may be in flight, so the collective's kernels run beside the
#   dW GEMM instead of after it (0: the GEMMs take every SM).
VP_STATS_EXCHANGE = "allreduce"
VP_OVERLAP_SMS = 0
# * VP_DX_EXCHANGE: "nccl" sums each chunk's partial dX with an asynchronous
#   NCCL all-reduce that overlaps the chunk's dW GEMM; "p2p" exchanges it
#   through peer memory without a collective library: the dX GEMM's epilogue
#   stores every tile into its row owner's buffer on the owning GPU while the
#   GEMM runs, then each owner sums its rows in rank order and writes them to
#   every rank (ml_flce_shard_dx_p2p / ml_flce_p2p_reduce / ml_flce_p2p_finish),
#   the owner's phase on a side stream beside the dW GEMM; the statistics go
#   through the same buffers (ml_flce_p2p_stats_put / _merge), so the step
#   uses no collective at all.  Its waits are bounded: one that gives up (a
#   rank that never arrives) leaves ML_ERR_TIMEOUT in the device error word,
#   which _C.load().ml_device_error(None) reads and clears.
VP_DX_EXCHANGE = "nccl"


class PeerExchange:
    """The p2p dX exchange's buffers for one (process group, device, chunk
    capacity, hidden size): one ml_p2p_alloc buffer per rank, exported once
    and mapped on every other rank (handles exchanged through the process
    group), plus the side stream of the owners' phase and the epoch counter
    every rank advances identically (one per chunk)."""

    _cache: dict = {}

    @classmethod
    def get(cls, group, device, chunk_cap, h):
        import torch.distributed as dist

        key = (id(group) if group is not None else None, dist.get_rank(group), device.index,
               int(chunk_cap), int(h))
        ex = cls._cache.get(key)
        if ex is None:
            ex = cls(group, device, int(chunk_cap), int(h))
            cls._cache[key] = ex
        return ex

    def __init__(self, group, device, chunk_cap, h):
        import ctypes

        import torch.distributed as dist
        from metal_liger_b200 import _C

        lib = _C.load()
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.chunk_cap, self.h = chunk_cap, h
        nbytes = int(lib.ml_flce_p2p_workspace_bytes(self.world, chunk_cap, h))
        if nbytes == 0:
            raise RuntimeError(f"vocab-parallel FLCE p2p exchange: unsupported world size "
                               f"{self.world} (at most 8) or sizes")
        with torch.cuda.device(device):
            base = ctypes.c_void_p()
            _C.call("ml_p2p_alloc", nbytes, ctypes.byref(base))
            hb = int(lib.ml_p2p_handle_bytes())
            handle = (ctypes.c_uint8 * hb)()
            _C.call("ml_p2p_export", base, handle)
            handles = [None] * self.world
            dist.all_gather_object(handles, bytes(handle), group=group)
            ptrs, self.imported = [], []
            for r, hnd in enumerate(handles):
                if r == self.rank:
                    ptrs.append(base.value)
                    continue
                buf = (ctypes.c_uint8 * hb).from_buffer_copy(hnd)
                out = ctypes.c_void_p()
                _C.call("ml_p2p_import", buf, ctypes.byref(out))
                ptrs.append(out.value)
                self.imported.append(out.value)
            self.stream = torch.cuda.Stream(device)
        self.base = base.value
        self.table = (ctypes.c_void_p * self.world)(*ptrs)
        self.epoch = 0


def _merge_stats(m, s, t, group, phases):
    """Global (max, sum exp(logit - max), target logit) per row from every
    rank's shard statistics."""
    import torch.distributed as dist

    if VP_STATS_EXCHANGE == "allgather":
        world = dist.get_world_size(group)
        mine = torch.stack([m, s, t])
        if dist.get_backend(group) == "nccl":
            every = torch.empty((world,) + tuple(mine.shape), dtype=mine.dtype,
                                device=mine.device)
            dist.all_gather_into_tensor(every, mine, group=group)
        else:
            parts = [torch.empty_like(mine) for _ in range(world)]
            dist.all_gather(parts, mine, group=group)
            every = torch.stack(parts)
        mg = every[:, 0].amax(dim=0)
        sg = (every[:, 1] * torch.exp(every[:, 0] - mg)).sum(dim=0)
        return mg, sg, every[:, 2].sum(dim=0)
    mg = m.clone()
    dist.all_reduce(mg, op=dist.ReduceOp.MAX, group=group)
    st = torch.stack([s * torch.exp(m - mg), t])
    dist.all_reduce(st, op=dist.ReduceOp.SUM, group=group)
    return mg, st[0], st[1]


def _leave_sms_for_collectives(phases, pending):
    import contextlib

    if VP_OVERLAP_SMS <= 0 or not pending or not isinstance(phases, CudaShardPhases):
        return contextlib.nullcontext()
    from metal_liger_b200 import _C
    return _C.gemm_reserved_sms(VP_OVERLAP_SMS)


def _p2p_stats(ex, m, s, t, h):
    """The chunk's (max, sum-exp, target) merged over the ranks through peer
    memory (rank order; the same on every rank), for epoch ex.epoch."""
    from metal_liger_b200 import _C

    rows = m.numel()
    st = torch.cuda.current_stream(m.device).cuda_stream
    _C.call("ml_flce_p2p_stats_put", m.data_ptr(), s.data_ptr(), t.data_ptr(), rows, h,
            ex.chunk_cap, ex.world, ex.rank, ex.table, ex.epoch, st)
    mg, sg, tg = torch.empty_like(m), torch.empty_like(s), torch.empty_like(t)
    _C.call("ml_flce_p2p_stats_merge", rows, h, ex.chunk_cap, ex.world, ex.rank, ex.table,
            ex.epoch, mg.data_ptr(), sg.data_ptr(), tg.data_ptr(), st)
    return mg, sg, tg


def _p2p_dx(ex, state, weight_shard, rows, h, dx_rows, previous):
    """One chunk's dX through peer memory (epoch ex.epoch, set by the
    chunk's statistics exchange): the dX GEMM with the peer-store epilogue on
    the current stream (after the previous chunk's exchange, whose owners must
    be done reading their receive slots), the owners' phase on the exchange's
    side stream, writing the summed rows into `dx_rows`."""
    from metal_liger_b200 import _C

    main = torch.cuda.current_stream(dx_rows.device)
    if previous is not None:
        main.wait_event(previous)
    _C.call("ml_flce_shard_dx_p2p", weight_shard.data_ptr(), rows, h, weight_shard.shape[0],
            state.data_ptr(), state.numel(), ex.chunk_cap, ex.world, ex.rank, ex.table,
            ex.epoch, main.cuda_stream)
    ex.stream.wait_stream(main)
    _C.call("ml_flce_p2p_reduce", rows, h, ex.chunk_cap, ex.world, ex.rank, ex.table, ex.epoch,
            ex.stream.cuda_stream)
    _C.call("ml_flce_p2p_finish", rows, h, ex.chunk_cap, ex.world, ex.rank, ex.table, ex.epoch,
            dx_rows.data_ptr(), ex.stream.cuda_stream)


def vocab_parallel_flce(hidden, weight_shard, labels, vocab_offset, bias_shard=None,
                        ignore_index=-100, chunk_size=8192, group=None, phases=None,
                        need_dx=True, need_dw=True):
    """Vocabulary-parallel fused linear cross-entropy; every rank calls it with the
    same hidden/labels and its own contiguous vocabulary shard of the lm_head.

    Per token chunk: each rank computes its shard's per-row (max, sum-exp,
    target logit); two all-reduces (MAX of the maxima, then SUM of the
    rescaled sums and target logits) give the global log-sum-exp; each rank
    then forms its shard's (softmax - onehot)/n_valid and produces its partial
    dX (summed across ranks with an all-reduce that overlaps the next chunk)
    and its own dW shard, which never leaves the rank.

    Returns (loss, dx [N, H] fp32 or None, dw_shard [V_local, H] fp32 or None),
    the gradients at grad_output = 1.
    """
    import torch.distributed as dist

    phases = phases or CudaShardPhases()
    hidden = hidden.reshape(-1, hidden.shape[-1])
    if hidden.dtype != torch.bfloat16 and isinstance(phases, CudaShardPhases):
        hidden = hidden.to(torch.bfloat16)
    if weight_shard.dtype != torch.bfloat16 and isinstance(phases, CudaShardPhases):
        weight_shard = weight_shard.to(torch.bfloat16)
    hidden = hidden.contiguous()
    weight_shard = weight_shard.contiguous()
    h_in = hidden.shape[1]
    if h_in % 8 and isinstance(phases, CudaShardPhases):
        # TMA row pitch: zero-pad the hidden size to a multiple of 8 (zero
        # columns add nothing to the logits; sliced off the gradients below)
        from metal_liger_b200._torch_library import _p8, _pad2
        hidden = _pad2(hidden, hidden.shape[0], _p8(h_in))
        weight_shard = _pad2(weight_shard, weight_shard.shape[0], _p8(h_in))
    labels = labels.reshape(-1).to(torch.int64).contiguous()
    n, h = hidden.shape
    dev = hidden.device
    cnt = phases.count(labels, ignore_index)
    row_loss = torch.zeros(n, dtype=torch.float32, device=dev)
    dx = torch.zeros((n, h), dtype=torch.float32, device=dev) if need_dx else None
    dw = (torch.zeros((weight_shard.shape[0], h), dtype=torch.float32, device=dev)
          if need_dw else None)
    chunk = int(chunk_size) if chunk_size and chunk_size > 0 else n
    pending = []
    ex = None
    if (need_dx and VP_DX_EXCHANGE == "p2p" and isinstance(phases, CudaShardPhases)
            and dist.get_backend(group) == "nccl"):
        ex = PeerExchange.get(group, dev, chunk, h)
    exchanged = None  # event: the previous chunk's p2p exchange is complete
    for r0 in range(0, n, chunk):
        r1 = min(n, r0 + chunk)
        hc, lc = hidden[r0:r1], labels[r0:r1]
        with _leave_sms_for_collectives(phases, pending):
            m, s, t, state = phases.stats(hc, weight_shard, bias_shard, lc, vocab_offset,
                                          ignore_index)
        if ex is not None:
            ex.epoch += 1
            mg, sg, tg = _p2p_stats(ex, m, s, t, h)
        else:
            mg, sg, tg = _merge_stats(m, s, t, group, phases)
        lse = mg + torch.log(sg)
        mask = (lc != ignore_index).to(torch.float32)
        row_loss[r0:r1] = (lse - tg) * mask
        if ex is not None:
            phases.grads(state, hc, weight_shard, lc, vocab_offset, ignore_index,
                         lse.contiguous(), cnt[1:2], None, None, r0 > 0)
            _p2p_dx(ex, state, weight_shard, r1 - r0, h, dx[r0:r1], exchanged)
            exchanged = ex.stream.record_event()
        else:
            # dX first, so its all-reduce runs while this chunk's dW GEMM does
            phases.grads(state, hc, weight_shard, lc, vocab_offset, ignore_index,
                         lse.contiguous(), cnt[1:2], dx[r0:r1] if need_dx else None, None,
                         r0 > 0)
            if need_dx:
                pending.append(dist.all_reduce(dx[r0:r1], op=dist.ReduceOp.SUM, group=group,
                                               async_op=True))
        if need_dw:
            with _leave_sms_for_collectives(phases, pending):
                phases.grads_dw(state, hc, weight_shard, dw, r0 > 0)
    for work in pending:
        work.wait()
    if exchanged is not None:
        torch.cuda.current_stream(dev).wait_event(exchanged)
    loss = row_loss.sum() * cnt[1]
    if h != h_in:
        dx = dx[:, :h_in].contiguous() if dx is not None else None
        dw = dw[:, :h_in].contiguous() if dw is not None else None
    return loss, dx, dw


class _VocabParallelFLCEFunction(torch.autograd.Function):
    """Autograd wrapper of vocab_parallel_flce (gradients formed in forward)."""

    @staticmethod
    def forward(ctx, hidden, weight_shard, labels, bias_shard, vocab_offset, ignore_index,
                chunk_size, group):
        need_dx = bool(ctx.needs_input_grad[0])
        need_dw = bool(ctx.needs_input_grad[1])
        loss, dx, dw = vocab_parallel_flce(hidden, weight_shard, labels, vocab_offset,
                                           bias_shard, ignore_index, chunk_size, group,
                                           need_dx=need_dx, need_dw=need_dw)
        empty = torch.empty(0, device=hidden.device)
        ctx.save_for_backward(dx.unsqueeze(0) if dx is not None else empty,
                              dw if dw is not None else empty)
        ctx.hidden_shape = hidden.shape
        ctx.codes = (DTYPE_CODES.get(hidden.dtype, 0), DTYPE_CODES.get(weight_shard.dtype, 0))
        return loss

    @staticmethod
    def backward(ctx, grad_output):
        dx, dw = ctx.saved_tensors
        gh, gw = torch.ops.metal_liger.flce_backward(grad_output, dx, dw, ctx.codes[0],
                                                     ctx.codes[1])
        grad_hidden = gh.view(ctx.hidden_shape) if ctx.needs_input_grad[0] else None
        grad_weight = gw if ctx.needs_input_grad[1] else None
        return grad_hidden, grad_weight, None, None, None, None, None, None


class VocabParallelFusedLinearCrossEntropy(nn.Module):
    """lm_head + cross-entropy with the lm_head split by vocabulary across a process
    group: holds this rank's shard (``weight_shard`` = rows [vocab_offset,
    vocab_offset + V_local) of the full head).  The loss is the full-vocabulary
    mean cross-entropy, identical on every rank."""

    def __init__(self, weight_shard: nn.Parameter, vocab_offset: int, bias_shard=None,
                 ignore_index: int = -100, chunk_size: int = 8192, group=None):
        super().__init__()
        self.weight = weight_shard
        self.bias = bias_shard
        self.vocab_offset = vocab_offset
        self.ignore_index = ignore_index
        self.chunk_size = chunk_size
        self.group = group

    def forward(self, hidden_states: torch.Tensor, labels: torch.Tensor) -> torch.Tensor:
        hidden_flat = hidden_states.reshape(-1, hidden_states.shape[-1])
        return _VocabParallelFLCEFunction.apply(hidden_flat, self.weight, labels.reshape(-1),
                                                self.bias, self.vocab_offset, self.ignore_index,
                                                self.chunk_size, self.group)
