"""metal_liger_b200 — B200-native (sm_100a) fused training ops with metal_liger's API.

Drop-in for the reference package ``metal_liger`` (v0.3.0, __init__.py:24-60):
the same public names, re-implemented as hand-written CUDA kernels for B200
behind a C ABI (``include/metal_liger_b200.h``), exposed as ``metal_liger::``
torch custom ops and the reference's autograd Functions.

    import metal_liger_b200 as metal_liger
    model = metal_liger.apply_metal_liger_to_qwen3vl(model)

``metal_liger_b200.install_as_metal_liger()`` additionally aliases the package
under the name ``metal_liger`` so unmodified ``from metal_liger... import``
code resolves to it.
"""

import sys as _sys

__version__ = "0.1.0"
REFERENCE_VERSION = "0.3.0"

from metal_liger_b200._torch_library import register_metal_liger_ops

register_metal_liger_ops()

from metal_liger_b200.ops.fused_rms_norm import MetalLigerRMSNorm  # noqa: E402
from metal_liger_b200.ops.fused_swiglu import MetalLigerSwiGLU  # noqa: E402
from metal_liger_b200.ops.fused_rope import MetalLigerRoPE  # noqa: E402
from metal_liger_b200.ops.fused_linear_cross_entropy import (  # noqa: E402
    MetalLigerFusedLinearCrossEntropy,
)
from metal_liger_b200.ops.fused_lora import (  # noqa: E402
    apply_fused_lora_qkv,
    apply_fused_lora_mlp,
    apply_fused_lora_linear,
    patch_fused_lora,
)
from metal_liger_b200.patch import apply_metal_liger_to_qwen3vl  # noqa: E402
from metal_liger_b200._compile import apply_compile  # noqa: E402

__all__ = [
    "MetalLigerRMSNorm",
    "MetalLigerSwiGLU",
    "MetalLigerRoPE",
    "MetalLigerFusedLinearCrossEntropy",
    "apply_metal_liger_to_qwen3vl",
    "apply_fused_lora_qkv",
    "apply_fused_lora_mlp",
    "apply_fused_lora_linear",
    "patch_fused_lora",
    "apply_compile",
    "register_metal_liger_ops",
    "install_as_metal_liger",
]


def install_as_metal_liger() -> None:
    """Alias this package (and its submodules) as ``metal_liger`` in sys.modules."""
    import importlib

    mods = ["", ".ops", ".ops.fused_rms_norm", ".ops.fused_swiglu", ".ops.fused_rope",
            "._torch_library", "._compile", ".generation", ".metal_liger_ext"]
    for extra in ("ops.fused_linear_cross_entropy", "ops.fused_lora", "patch"):
        try:
            importlib.import_module(f"metal_liger_b200.{extra}")
            mods.append("." + extra)
        except ImportError:
            pass
    for m in mods:
        mod = importlib.import_module("metal_liger_b200" + m)
        _sys.modules["metal_liger" + m] = mod
