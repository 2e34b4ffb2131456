"""ctypes binding of the C ABI in ``include/metal_liger_b200.h``.

The shared library is built in-tree by ``metal_liger_b200._build`` (nvcc,
sm_100a only).  There is no fallback: if the library is missing or a call
fails, a ``RuntimeError`` is raised with the library's own message.  This
module replaces the reference's pybind module ``metal_liger_ext``
(csrc/bindings.mm:10-33); the tensor-level API lives in
``metal_liger_b200.metal_liger_ext`` and ``metal_liger_b200._torch_library``.
"""

from __future__ import annotations

import contextlib
import ctypes
import os
import threading
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().parent / "lib" / "libmetal_liger_b200.so"

DTYPE_CODES = {torch.float32: 0, torch.bfloat16: 1, torch.float16: 2}

ML_OK = 0
ML_ERR_TIMEOUT = 4

c_void_p = ctypes.c_void_p
c_int = ctypes.c_int
c_int64 = ctypes.c_int64
c_float = ctypes.c_float
c_size_t = ctypes.c_size_t


class RopeTensor(ctypes.Structure):
    """Mirror of ``ml_rope_tensor``."""

    _fields_ = [
        ("inp", c_void_p),
        ("out", c_void_p),
        ("heads", c_int64),
        ("in_strides", c_int64 * 4),
        ("out_strides", c_int64 * 4),
    ]


class GemmOperand(ctypes.Structure):
    """Mirror of ``ml_gemm_operand``."""

    _fields_ = [("ptr", c_void_p), ("ld", c_int64), ("mn_major", c_int)]


class GemmSegment(ctypes.Structure):
    """Mirror of ``ml_gemm_segment``."""

    _fields_ = [("a", GemmOperand), ("b", GemmOperand), ("k", c_int64)]


class LoraProj(ctypes.Structure):
    """Mirror of ``ml_lora_proj``."""

    _fields_ = [("w", c_void_p), ("a", c_void_p), ("b", c_void_p), ("a_dtype", c_int),
                ("b_dtype", c_int), ("out_features", c_int64), ("scaling", c_float)]


# name -> (restype, argtypes).  Kept in the same order as the header.
SIGNATURES: dict[str, tuple[object, list[object]]] = {
    "ml_version": (c_int, []),
    "ml_last_error": (ctypes.c_char_p, []),
    "ml_rms_norm_forward": (c_int, [c_void_p, c_int, c_void_p, c_int, c_void_p, c_void_p,
                                    c_int64, c_int64, c_float, c_void_p]),
    "ml_rms_norm_backward_workspace_bytes": (c_size_t, [c_int64, c_int64]),
    "ml_rms_norm_backward": (c_int, [c_void_p, c_int, c_void_p, c_int, c_void_p, c_void_p,
                                     c_void_p, c_void_p, c_float, c_void_p, c_size_t, c_int64,
                                     c_int64, c_void_p]),
    "ml_rms_norm_backward_noalloc": (c_int, [c_void_p, c_int, c_void_p, c_int, c_void_p,
                                             c_void_p, c_void_p, c_void_p, c_float, c_int64,
                                             c_int64, c_void_p]),
    "ml_swiglu_forward": (c_int, [c_void_p, c_void_p, c_void_p, c_int64, c_int, c_void_p]),
    "ml_swiglu_backward": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int64,
                                   c_int, c_void_p]),
    "ml_rope": (c_int, [ctypes.POINTER(RopeTensor), ctypes.POINTER(RopeTensor), c_int, c_int,
                        c_int64, c_int64, c_int64, c_void_p, c_void_p, c_int,
                        ctypes.POINTER(c_int64), c_void_p, c_int64, c_void_p, c_float, c_int,
                        c_void_p]),
    "ml_gemm_bf16_workspace_bytes": (c_size_t, [c_int64, c_int64, c_int64]),
    "ml_gemm_bf16": (c_int, [c_int64, c_int64, ctypes.POINTER(GemmSegment), c_int, c_void_p, c_int,
                             c_int64, c_float, c_float, c_void_p, c_size_t, c_void_p]),
    "ml_gemm_set_cta_pair": (c_int, [c_int, ctypes.POINTER(c_int)]),
    "ml_lora_set_mlp_swiglu_fusion": (c_int, [c_int, ctypes.POINTER(c_int)]),
    "ml_gemm_set_reserved_sms": (c_int, [c_int, ctypes.POINTER(c_int)]),
    "ml_rms_norm_set_bwd_vectors": (c_int, [c_int, ctypes.POINTER(c_int)]),
    "ml_selftest_bounded_wait": (c_int, [c_int64, c_void_p]),
    "ml_lm_head_argmax_workspace_bytes": (c_size_t, [c_int64, c_int64]),
    "ml_gemv_bf16": (c_int, [c_void_p, c_int64, c_void_p, c_int64, c_void_p, c_int, c_int64,
                             c_int64, c_int64, c_void_p, c_int, c_int64, c_void_p]),
    "ml_gemv_multi_bf16": (c_int, [c_void_p, c_int64, c_int, c_void_p, c_void_p, c_void_p,
                                   c_void_p, c_int, c_int64, c_int64, c_void_p, c_void_p, c_int,
                                   c_void_p]),
    "ml_decode_attention_workspace_bytes": (c_size_t, [c_int64, c_int64, c_int64, c_int64]),
    "ml_decode_attention_bf16": (c_int, [c_void_p, c_int64, c_int64, c_void_p, c_void_p, c_void_p,
                                         c_int64, c_int64, c_int64, c_int64, c_int64, c_int64,
                                         ctypes.c_float, c_void_p, c_void_p, c_size_t, c_void_p]),
    "ml_decode_qk_norm_rope_bf16": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                            c_int, ctypes.c_float, ctypes.c_float, c_void_p,
                                            c_void_p, c_int, c_int64, c_int64, c_int64, c_int64,
                                            c_int64, c_int64, c_void_p, c_void_p, c_void_p,
                                            c_void_p, c_void_p]),
    "ml_decode_qk_attention_bf16": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                            c_int, ctypes.c_float, ctypes.c_float, c_void_p,
                                            c_void_p, c_int, c_int64, c_int64, c_int64, c_int64,
                                            c_int64, c_int64, c_void_p, c_void_p, c_void_p,
                                            ctypes.c_float, c_void_p, c_void_p]),
    "ml_gemv_swiglu_bf16": (c_int, [c_void_p, c_int64, c_void_p, c_int64, c_void_p, c_int64,
                                    c_int64, c_int64, c_int64, c_void_p, c_int64, c_void_p]),
    "ml_gemv_residual_bf16": (c_int, [c_void_p, c_int64, c_void_p, c_int64, c_void_p, c_int,
                                      c_void_p, c_int64, c_int64, c_int64, c_int64, c_void_p,
                                      c_int64, c_void_p]),
    "ml_gemv_rmsnorm_multi_bf16": (c_int, [c_void_p, c_int64, c_void_p, ctypes.c_float, c_int,
                                           c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int64,
                                           c_int64, c_void_p, c_void_p, c_int, c_void_p]),
    "ml_gemv_rmsnorm_swiglu_bf16": (c_int, [c_void_p, c_int64, c_void_p, ctypes.c_float,
                                            c_void_p, c_int64, c_void_p, c_int64, c_int64,
                                            c_int64, c_int64, c_void_p, c_int64, c_void_p]),
    "ml_lm_head_argmax": (c_int, [c_void_p, c_int64, c_void_p, c_int64, c_void_p, c_int, c_int64,
                                  c_int64, c_int64, c_int, c_void_p, c_void_p, c_void_p,
                                  c_size_t, c_void_p]),
    "ml_flce_dx_slabs": (c_int, [c_int64, c_int64, c_int64, c_int64]),
    "ml_flce_workspace_bytes": (c_size_t, [c_int64, c_int64, c_int64, c_int64]),
    "ml_flce_forward": (c_int, [c_void_p, c_void_p, c_void_p, c_int, c_void_p, c_int64, c_int64,
                                c_int64, c_int64, c_int64, c_void_p, c_void_p, c_void_p, c_void_p,
                                c_void_p, c_size_t, c_void_p]),
    "ml_flce_backward": (c_int, [c_void_p, c_void_p, c_int, c_void_p, c_int, c_int64, c_int64,
                                 c_void_p, c_void_p, c_int, c_int64, c_void_p]),
    "ml_flce_count_valid": (c_int, [c_void_p, c_int64, c_int64, c_void_p, c_void_p]),
    "ml_flce_shard_workspace_bytes": (c_size_t, [c_int64, c_int64]),
    "ml_flce_shard_stats": (c_int, [c_void_p, c_void_p, c_void_p, c_int, c_void_p, c_int64, c_int64,
                                    c_int64, c_int64, c_int64, c_void_p, c_void_p, c_void_p,
                                    c_void_p, c_size_t, c_void_p]),
    "ml_flce_shard_grads": (c_int, [c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int64,
                                    c_int64, c_int64, c_void_p, c_void_p, c_void_p, c_void_p,
                                    c_int, c_void_p, c_size_t, c_void_p]),
    "ml_flce_shard_grads_dw": (c_int, [c_void_p, c_int64, c_int64, c_int64, c_void_p, c_int,
                                       c_void_p, c_size_t, c_void_p]),
    "ml_p2p_alloc": (c_int, [c_size_t, ctypes.POINTER(c_void_p)]),
    "ml_p2p_free": (c_int, [c_void_p]),
    "ml_p2p_handle_bytes": (c_size_t, []),
    "ml_p2p_export": (c_int, [c_void_p, c_void_p]),
    "ml_p2p_import": (c_int, [c_void_p, ctypes.POINTER(c_void_p)]),
    "ml_p2p_close": (c_int, [c_void_p]),
    "ml_flce_p2p_workspace_bytes": (c_size_t, [c_int, c_int64, c_int64]),
    "ml_flce_shard_dx_p2p": (c_int, [c_void_p, c_int64, c_int64, c_int64, c_void_p, c_size_t,
                                     c_int64, c_int, c_int, ctypes.POINTER(c_void_p), c_int64,
                                     c_void_p]),
    "ml_flce_p2p_reduce": (c_int, [c_int64, c_int64, c_int64, c_int, c_int,
                                   ctypes.POINTER(c_void_p), c_int64, c_void_p]),
    "ml_flce_p2p_finish": (c_int, [c_int64, c_int64, c_int64, c_int, c_int,
                                   ctypes.POINTER(c_void_p), c_int64, c_void_p, c_void_p]),
    "ml_flce_p2p_stats_put": (c_int, [c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int64,
                                      c_int, c_int, ctypes.POINTER(c_void_p), c_int64, c_void_p]),
    "ml_flce_p2p_stats_merge": (c_int, [c_int64, c_int64, c_int64, c_int, c_int,
                                        ctypes.POINTER(c_void_p), c_int64, c_void_p, c_void_p,
                                        c_void_p, c_void_p]),
    "ml_lora_qkv_workspace_bytes": (c_size_t, [c_int64, c_int64, ctypes.POINTER(LoraProj), c_int]),
    "ml_lora_qkv_forward": (c_int, [c_void_p, c_int64, c_int64, c_int64, ctypes.POINTER(LoraProj),
                                    ctypes.POINTER(c_void_p), c_void_p, c_void_p, c_size_t,
                                    c_void_p]),
    "ml_lora_qkv_backward": (c_int, [c_void_p, c_void_p, c_int64, c_int64, c_int64,
                                     ctypes.POINTER(LoraProj), ctypes.POINTER(c_void_p), c_void_p,
                                     ctypes.POINTER(c_void_p), ctypes.POINTER(c_void_p), c_void_p,
                                     c_size_t, c_void_p]),
    "ml_lora_linear_workspace_bytes": (c_size_t, [c_int64, c_int64, c_int,
                                                  ctypes.POINTER(LoraProj), c_int]),
    "ml_lora_linear_forward": (c_int, [c_void_p, c_int64, c_int64, c_int64, c_int,
                                       ctypes.POINTER(LoraProj), ctypes.POINTER(c_void_p),
                                       c_void_p, c_void_p, c_size_t, c_void_p]),
    "ml_lora_linear_backward": (c_int, [c_void_p, c_void_p, c_int64, c_int64, c_int64, c_int,
                                        ctypes.POINTER(LoraProj), ctypes.POINTER(c_void_p),
                                        c_void_p, ctypes.POINTER(c_void_p),
                                        ctypes.POINTER(c_void_p), c_void_p, c_size_t,
                                        c_void_p]),
    "ml_lora_mlp_workspace_bytes": (c_size_t, [c_int64, c_int64, c_int64, c_int]),
    "ml_lora_mlp_forward": (c_int, [c_void_p, c_int64, c_int64, c_int64, c_int64,
                                    ctypes.POINTER(LoraProj), c_void_p, c_void_p, c_void_p,
                                    c_void_p, c_void_p, c_void_p, c_void_p, c_size_t, c_void_p]),
    "ml_lora_mlp_backward": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                     c_int64, c_int64, c_int64, c_int64, ctypes.POINTER(LoraProj),
                                     c_void_p, c_void_p, ctypes.POINTER(c_void_p),
                                     ctypes.POINTER(c_void_p), c_void_p, c_size_t, c_void_p]),
    "ml_device_error": (c_int, [c_void_p]),
}

_lib = None
_lock = threading.Lock()


def load() -> ctypes.CDLL:
    """Load the CUDA library (once).  Raises if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not LIB_PATH.exists():
            raise RuntimeError(
                f"metal_liger_b200: CUDA library not found at {LIB_PATH}. Build it with "
                "`python -m metal_liger_b200._build` (nvcc, sm_100a). There is no CPU fallback.")
        lib = ctypes.CDLL(str(LIB_PATH), mode=os.RTLD_NOW | getattr(os, "RTLD_LOCAL", 0))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib


def last_error() -> str:
    msg = load().ml_last_error()
    return msg.decode(errors="replace") if msg else ""


def check(status: int, what: str) -> None:
    if status != ML_OK:
        raise RuntimeError(f"metal_liger_b200 {what} failed (status {status}): {last_error()}")


def call(name: str, *args) -> int:
    """Invoke an entry point and raise on a non-zero status."""
    fn = getattr(load(), name)
    status = fn(*args)
    check(status, name)
    return status


def dtype_code(t: torch.Tensor | torch.dtype) -> int:
    dt = t if isinstance(t, torch.dtype) else t.dtype
    try:
        return DTYPE_CODES[dt]
    except KeyError:
        raise RuntimeError(f"metal_liger_b200: unsupported dtype {dt}") from None


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def stream_of(t: torch.Tensor) -> int:
    """Raw cudaStream_t of torch's current stream on ``t``'s device."""
    return torch.cuda.current_stream(t.device).cuda_stream


def require_cuda(name: str, *tensors: torch.Tensor | None) -> None:
    dev = None
    for t in tensors:
        if t is None:
            continue
        if t.device.type != "cuda":
            raise RuntimeError(
                f"metal_liger_b200 {name}: tensors must be on a CUDA device, got {t.device} "
                "(there is no CPU fallback)")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise RuntimeError(f"metal_liger_b200 {name}: tensors on different devices")


@contextlib.contextmanager
def gemm_cta_pair(mode: int):
    """Select the 2-SM GEMM kernel process-wide for the duration of a block:
    -1 automatic, 0 never, 1 whenever the tile shape allows."""
    prev = ctypes.c_int(-1)
    call("ml_gemm_set_cta_pair", int(mode), ctypes.byref(prev))
    try:
        yield
    finally:
        call("ml_gemm_set_cta_pair", prev.value, None)


@contextlib.contextmanager
def gemm_reserved_sms(n: int):
    """Leave `n` SMs free of this library's GEMMs for the duration of a block
    (for kernels on other streams that should overlap them)."""
    prev = ctypes.c_int(0)
    call("ml_gemm_set_reserved_sms", int(n), ctypes.byref(prev))
    try:
        yield
    finally:
        call("ml_gemm_set_reserved_sms", prev.value, None)


@contextlib.contextmanager
def lora_mlp_swiglu_fusion(enable: bool):
    """Run the LoRA MLP with the SwiGLU inside its GEMMs (True, the default)
    or as separate elementwise passes (False) for the duration of a block."""
    prev = ctypes.c_int(1)
    call("ml_lora_set_mlp_swiglu_fusion", 1 if enable else 0, ctypes.byref(prev))
    try:
        yield
    finally:
        call("ml_lora_set_mlp_swiglu_fusion", prev.value, None)


def exported_symbols() -> list[str]:
    return list(SIGNATURES)
