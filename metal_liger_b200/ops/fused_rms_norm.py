"""Fused RMSNorm on B200 — drop-in for the reference's ops/fused_rms_norm.py.

Same classes and signatures as the reference (`_FusedRMSNormFunction`,
`MetalLigerRMSNorm`, ops/fused_rms_norm.py:22-82).  Forward and backward each
run as one sm_100a kernel (plus a tiny deterministic dweight reduction) through
the ``metal_liger::rms_norm_*`` ops; the forward saves x, weight and the fp32
per-row ``rrms`` exactly as the reference does (ops/fused_rms_norm.py:39).
"""

import torch
import torch.nn as nn

import metal_liger_b200._torch_library  # noqa: F401  (registers metal_liger:: ops)


class _FusedRMSNormFunction(torch.autograd.Function):
    """y = x * weight * rsqrt(mean(x^2) + eps), fp32 math, output in x.dtype.

    Backward (reference ops/fused_rms_norm.py:43-60):
        dx = g*w*r - x*mean(g*w*x)*r^3,   dweight = sum_rows(g * x * r)
    """

    @staticmethod
    def forward(ctx, x: torch.Tensor, weight: torch.Tensor, eps: float):
        y, rrms = torch.ops.metal_liger.rms_norm_forward(x, weight, float(eps), "")
        ctx.save_for_backward(x, weight, rrms)
        ctx.eps = eps
        return y

    @staticmethod
    def backward(ctx, grad_output: torch.Tensor):
        x, weight, rrms = ctx.saved_tensors
        grad_x, grad_weight = torch.ops.metal_liger.rms_norm_backward(
            x, weight, grad_output, float(ctx.eps), "", rrms)
        if not ctx.needs_input_grad[1]:
            grad_weight = None
        return grad_x, grad_weight, None


class MetalLigerRMSNorm(nn.Module):
    """Drop-in replacement for nn.RMSNorm / transformers RMSNorm
    (reference ops/fused_rms_norm.py:63-82)."""

    def __init__(self, hidden_size: int, eps: float = 1e-6, weight: torch.Tensor = None):
        super().__init__()
        self.eps = eps
        self.hidden_size = hidden_size
        if weight is not None:
            self.weight = nn.Parameter(weight)
        else:
            self.weight = nn.Parameter(torch.ones(hidden_size))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return _FusedRMSNormFunction.apply(x, self.weight, self.eps)

    def extra_repr(self) -> str:
        return f"hidden_size={self.hidden_size}, eps={self.eps}, fused=MetalLiger-B200"
