"""The C-ABI library loads and exports every entry point include/*.h declares.

No GPU work is issued: only pure-host entry points and argument validation
paths that return before anything is enqueued.
"""

import ctypes
import re
import subprocess
from pathlib import Path

import pytest

from metal_liger_b200 import _C

ROOT = Path(__file__).resolve().parent.parent


def declared_symbols():
    names = set()
    for hdr in (ROOT / "include").glob("*.h"):
        text = hdr.read_text()
        names.update(re.findall(r"ML_API\s+[\w\s\*]+?\b(ml_\w+)\s*\(", text))
    return sorted(names)


def test_header_declares_entry_points():
    names = declared_symbols()
    assert "ml_rms_norm_forward" in names and "ml_rope" in names
    assert len(names) >= 8


def test_library_exports_every_declared_symbol(cuda_lib):
    missing = [n for n in declared_symbols() if not hasattr(cuda_lib, n)]
    assert not missing, f"declared in include/*.h but not exported: {missing}"


def test_nm_exports_match_header():
    out = subprocess.run(["nm", "-D", "--defined-only", str(_C.LIB_PATH)], capture_output=True,
                         text=True, check=True).stdout
    exported = set(re.findall(r"\bT (ml_\w+)", out))
    assert set(declared_symbols()) <= exported
    # nothing beyond the header leaks out of the library (hidden visibility)
    assert exported <= set(declared_symbols()), exported - set(declared_symbols())


def test_ctypes_signatures_cover_header():
    assert set(declared_symbols()) == set(_C.SIGNATURES), \
        set(declared_symbols()) ^ set(_C.SIGNATURES)


def test_version_and_error_string(cuda_lib):
    assert cuda_lib.ml_version() >= 100
    assert isinstance(cuda_lib.ml_last_error(), (bytes, type(None)))


def test_invalid_args_rejected_on_host(cuda_lib):
    # negative size -> INVALID_ARG before any CUDA call
    assert cuda_lib.ml_swiglu_forward(None, None, None, -1, 0, None) == 1
    assert b"negative" in cuda_lib.ml_last_error()
    # bad dtype code
    assert cuda_lib.ml_rms_norm_forward(None, 7, None, 0, None, None, 4, 8, 1e-6, None) == 1
    # odd head_dim for RoPE
    q = _C.RopeTensor()
    assert cuda_lib.ml_rope(ctypes.byref(q), None, 1, 1, 1, 1, 63, None, None, 0, None, None, 0,
                            None, 1.0, 1, None) == 1
    assert b"head_dim" in cuda_lib.ml_last_error()


def test_empty_inputs_are_noops(cuda_lib):
    assert cuda_lib.ml_swiglu_forward(None, None, None, 0, 1, None) == 0
    assert cuda_lib.ml_rms_norm_forward(None, 0, None, 0, None, None, 0, 8, 1e-6, None) == 0


def test_python_raises_with_library_message():
    with pytest.raises(RuntimeError, match="status 1"):
        _C.check(1, "probe")


def test_gemm_kernel_mode_knob(cuda_lib):
    prev = ctypes.c_int(-7)
    assert cuda_lib.ml_gemm_set_cta_pair(0, ctypes.byref(prev)) == 0
    assert prev.value == -1  # process default: automatic
    assert cuda_lib.ml_gemm_set_cta_pair(5, None) == 1
    assert b"mode" in cuda_lib.ml_last_error()
    assert cuda_lib.ml_gemm_set_cta_pair(-1, ctypes.byref(prev)) == 0
    assert prev.value == 0


def test_lora_linear_rejects_bad_projection_counts(cuda_lib):
    projs = (_C.LoraProj * 3)()
    for i in range(3):
        projs[i].w = projs[i].a = projs[i].b = 16
        projs[i].out_features = 64
    # four projections, and three of rank 32 (3 x 32 > the 64-wide rank slot)
    assert cuda_lib.ml_lora_linear_forward(16, 8, 64, 8, 4, projs, None, 16, None, 0, None) == 1
    assert b"nproj" in cuda_lib.ml_last_error()
    assert cuda_lib.ml_lora_linear_forward(16, 8, 64, 32, 3, projs, None, 16, None, 0, None) == 1
    assert b"64" in cuda_lib.ml_last_error()
