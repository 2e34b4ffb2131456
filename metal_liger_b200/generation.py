"""Static-KV generator of the reference (generation.py:18-164) — out of scope here.

Generation is an inference side path, disabled by default in the reference's
patcher (patch.py:188).  The name is kept so imports resolve; calling it raises.
"""

import torch.nn as nn


def patch_generator(model: nn.Module) -> nn.Module:
    raise NotImplementedError(
        "metal_liger_b200 implements the fused training-op path only; the MPS static-KV "
        "generator (use_optimized_generator=True) is not provided")
