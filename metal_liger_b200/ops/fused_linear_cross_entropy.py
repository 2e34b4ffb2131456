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
