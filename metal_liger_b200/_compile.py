"""Layer-level torch.compile helpers of the reference (_compile.py) — not on this path.

The reference's own README reports no throughput benefit from them
(README.md:34-36), and on B200 the fused ops are already single kernels, so
only the deprecated entry point is kept, as the same no-op
(reference _compile.py:369-379).
"""

import logging

import torch.nn as nn

logger = logging.getLogger(__name__)


def apply_compile(model: nn.Module, **kwargs) -> nn.Module:
    """Deprecated no-op kept for API compatibility; returns ``model`` unchanged."""
    logger.warning("MetalLiger: apply_compile() is deprecated and does nothing. Skipping compile.")
    return model
