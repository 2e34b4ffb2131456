"""Fused ops (B200 / sm_100a) with the reference's module layout (ops/__init__.py)."""
from metal_liger_b200.ops.fused_rms_norm import MetalLigerRMSNorm
from metal_liger_b200.ops.fused_swiglu import MetalLigerSwiGLU
from metal_liger_b200.ops.fused_rope import MetalLigerRoPE
from metal_liger_b200.ops.fused_linear_cross_entropy import MetalLigerFusedLinearCrossEntropy
