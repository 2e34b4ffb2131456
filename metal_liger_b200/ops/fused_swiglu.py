"""Fused SwiGLU on B200 — drop-in for the reference's ops/fused_swiglu.py.

Same names as the reference (`_FusedSwiGLUFunction`, `fused_swiglu`,
`MetalLigerSwiGLU`, ops/fused_swiglu.py:18-75).  One elementwise sm_100a
kernel each way.  The reference saves gate, up AND an fp32 sigmoid tensor
(ops/fused_swiglu.py:34); here only gate and up are saved and the backward
recomputes sigmoid in registers, which is free on a bandwidth-bound op.
"""

import torch
import torch.nn as nn

import metal_liger_b200._torch_library  # noqa: F401  (registers metal_liger:: ops)


class _FusedSwiGLUFunction(torch.autograd.Function):
    """out = silu(gate) * up in fp32, cast to gate.dtype."""

    @staticmethod
    def forward(ctx, gate: torch.Tensor, up: torch.Tensor):
        out = torch.ops.metal_liger.swiglu_forward(gate, up, "")
        ctx.save_for_backward(gate, up)
        return out

    @staticmethod
    def backward(ctx, grad_output: torch.Tensor):
        gate, up = ctx.saved_tensors
        grad_gate, grad_up = torch.ops.metal_liger.swiglu_backward(gate, up, grad_output, "")
        return grad_gate, grad_up


def fused_swiglu(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    """Functional: SiLU(gate) * up in a single fused op."""
    return _FusedSwiGLUFunction.apply(gate, up)


class MetalLigerSwiGLU(nn.Module):
    """Drop-in for a SwiGLU MLP block — fuses the activation step only
    (reference ops/fused_swiglu.py:58-75)."""

    def __init__(self, original_mlp: nn.Module):
        super().__init__()
        self.gate_proj = original_mlp.gate_proj
        self.up_proj = original_mlp.up_proj
        self.down_proj = original_mlp.down_proj

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        gate = self.gate_proj(x)
        up = self.up_proj(x)
        activated = _FusedSwiGLUFunction.apply(gate, up)
        return self.down_proj(activated)

    def extra_repr(self) -> str:
        return "fused=MetalLiger-B200"
