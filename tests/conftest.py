"""Shared pytest configuration.

Markers:
  gpu  — needs a CUDA device (B200 / sm_100a); skipped when none is present.
         The driver runs `-m gpu` on a B200 and `-m "not gpu"` on a CPU host.
"""

import os
import sys
from pathlib import Path

import pytest
import torch

ROOT = Path(__file__).resolve().parent.parent
GOLDEN = Path(__file__).resolve().parent / "golden"
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

os.environ.setdefault("TORCHDYNAMO_DISABLE", "1")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: test needs a CUDA GPU (sm_100a)")


def pytest_collection_modifyitems(config, items):
    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device on this host")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


def load_golden(name: str) -> dict:
    return torch.load(GOLDEN / f"{name}.pt", weights_only=True)


def golden_names(prefix: str) -> list[str]:
    return sorted(p.stem for p in GOLDEN.glob(f"{prefix}*.pt"))


@pytest.fixture(scope="session")
def cuda_lib():
    """The built CUDA library (loads it; fails loudly if missing)."""
    from metal_liger_b200 import _C
    return _C.load()


@pytest.fixture(params=[0, 1, 3], ids=["1sm", "pair", "pair128"])
def pair_mode(request):
    """Run a GPU test with every GEMM on the 1-SM kernel, with the 2-SM (CTA
    pair) kernel forced wherever the tile shape allows, and with the pair
    kernel's 128-wide tiles forced."""
    from metal_liger_b200 import _C

    with _C.gemm_cta_pair(request.param):
        yield request.param
