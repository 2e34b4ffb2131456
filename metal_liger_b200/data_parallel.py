"""Token-row data parallelism for LoRA training: the gradient all-reduce.

Every rank runs the same model on its own rows of the batch; the trainable
(adapter) gradients are then averaged over the ranks with ONE collective on
one flat buffer, so every rank takes the same optimizer step.  With equal row
counts per rank and a mean loss per rank, the averaged gradient equals the
gradient of the mean loss over the concatenated batch.  The frozen base
weights get no gradient and never cross the wire.

The reference has no distributed code; this is the data-parallel exchange of
the full training step (a LoRA model patched with this package's fused ops),
run over NCCL on GPUs and over gloo in the CPU tests.
"""

from __future__ import annotations

from typing import Iterable

import torch
import torch.distributed as dist


def all_reduce_gradients(params: Iterable[torch.nn.Parameter], group=None,
                         average: bool = True, check_sizes: bool = False) -> int:
    """Sum (average=True: mean) the ``.grad`` of ``params`` over the ranks of
    ``group`` in place, with one all-reduce of the flattened gradients.

    Every rank must pass the same parameters in the same order, each with a
    gradient.  ``check_sizes`` first compares the flat sizes across ranks
    (two small all-reduces and a host synchronisation) and raises on a
    mismatch instead of reducing mismatched buffers; the training step leaves
    it off so the host never waits for the device.  Returns the number of
    gradient elements reduced.
    """
    grads = [p.grad for p in params if p.grad is not None]
    if not grads:
        return 0
    world = dist.get_world_size(group)
    flat = torch._utils._flatten_dense_tensors(grads)
    if check_sizes:
        n = torch.tensor([flat.numel(), -flat.numel()], dtype=torch.int64, device=flat.device)
        dist.all_reduce(n, op=dist.ReduceOp.MAX, group=group)
        if int(n[0].item()) != -int(n[1].item()):
            raise RuntimeError(f"all_reduce_gradients: ranks hold different gradient sizes "
                               f"({-int(n[1].item())} vs {int(n[0].item())} elements)")
    dist.all_reduce(flat, group=group)
    if average and world > 1:
        flat.div_(world)
    # one multi-tensor copy back (a copy per parameter would be ~500 launches
    # for a LoRA-adapted 36-layer model)
    torch._foreach_copy_(grads, list(torch._utils._unflatten_dense_tensors(flat, grads)))
    return int(flat.numel())
