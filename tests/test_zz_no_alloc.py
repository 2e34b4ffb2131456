"""GPU check of ml_rms_norm_backward_noalloc, the allocation-free entry point.

Some callers cannot allocate device memory when they call into this library
(a host whose memory planner owns all device memory after start-up, or a hot
loop that must not risk the implicit device synchronisation of
cudaMalloc/cudaFree).  For them the RMSNorm backward keeps its dweight
partials in a static device array instead of a caller-provided workspace.
This test calls it through the C ABI twice in a row (different shapes, so the
second call runs on the first call's leftover scratch) and checks each result
against the workspace-based ml_rms_norm_backward at the suite's tolerances.
The file name sorts last so a stop-at-first-failure run reaches it after every
other test; it also passes on its own in a fresh process.
"""

import ctypes

import pytest
import torch

from metal_liger_b200 import _C
from tolerances import assert_close

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _workspace_backward(lib, x, w, rrms, dy, eps):
    rows, hidden = x.shape
    dx = torch.empty_like(x)
    dw = torch.empty_like(w)
    ws_bytes = int(lib.ml_rms_norm_backward_workspace_bytes(rows, hidden))
    ws = torch.empty(max(ws_bytes // 4, 4), dtype=torch.float32, device=DEV)
    st = torch.cuda.current_stream().cuda_stream
    rc = lib.ml_rms_norm_backward(x.data_ptr(), _C.dtype_code(x), w.data_ptr(), _C.dtype_code(w),
                                  rrms.data_ptr(), dy.data_ptr(), dx.data_ptr(), dw.data_ptr(),
                                  eps, ws.data_ptr(), ws.numel() * 4, rows, hidden, st)
    assert rc == 0, _C.last_error()
    return dx, dw


def _noalloc_backward(lib, x, w, rrms, dy, eps):
    rows, hidden = x.shape
    dx = torch.empty_like(x)
    dw = torch.empty_like(w)
    st = torch.cuda.current_stream().cuda_stream
    rc = lib.ml_rms_norm_backward_noalloc(x.data_ptr(), _C.dtype_code(x), w.data_ptr(),
                                          _C.dtype_code(w), rrms.data_ptr(), dy.data_ptr(),
                                          dx.data_ptr(), dw.data_ptr(), eps, rows, hidden, st)
    assert rc == 0, _C.last_error()
    return dx, dw


def _inputs(rows, hidden, xd, wd, seed):
    g = torch.Generator(device=DEV).manual_seed(seed)
    x = torch.randn(rows, hidden, generator=g, device=DEV).to(xd)
    w = (1 + 0.1 * torch.randn(hidden, generator=g, device=DEV)).to(wd)
    dy = torch.randn(rows, hidden, generator=g, device=DEV).to(xd)
    rrms = torch.empty(rows, dtype=torch.float32, device=DEV)
    y = torch.empty_like(x)
    lib = _C.load()
    rc = lib.ml_rms_norm_forward(x.data_ptr(), _C.dtype_code(x), w.data_ptr(), _C.dtype_code(w),
                                 y.data_ptr(), rrms.data_ptr(), rows, hidden, 1e-6,
                                 torch.cuda.current_stream().cuda_stream)
    assert rc == 0, _C.last_error()
    return x, w, rrms, dy


def test_noalloc_matches_workspace_entry_point_on_two_calls_in_a_row():
    lib = _C.load()
    cases = [((4096, 2048), torch.float32, torch.float32),   # BASELINE hidden, fp32
             ((777, 1000), torch.bfloat16, torch.float32)]   # ragged, mixed dtypes
    for i, ((rows, hidden), xd, wd) in enumerate(cases):
        x, w, rrms, dy = _inputs(rows, hidden, xd, wd, seed=10 + i)
        ref_dx, ref_dw = _workspace_backward(lib, x, w, rrms, dy, 1e-6)
        dx, dw = _noalloc_backward(lib, x, w, rrms, dy, 1e-6)
        torch.cuda.synchronize()
        if xd == torch.float32:
            assert_close(dx, ref_dx, rtol=1e-5, atol=1e-6, what=f"call {i} dx")
        else:
            assert_close(dx, ref_dx.float(), dtype=xd, what=f"call {i} dx")
        scale = ref_dw.float().abs().max().item()
        assert_close(dw, ref_dw, rtol=1e-5, atol=1e-5 * scale, norm_rtol=1e-5,
                     what=f"call {i} dweight")


def test_noalloc_rejects_rows_wider_than_its_scratch():
    lib = _C.load()
    too_wide = (1 << 20) + 1
    rc = lib.ml_rms_norm_backward_noalloc(None, 0, None, 0, None, None, None, None, 1e-6, 1,
                                          too_wide, None)
    assert rc == 1
    assert b"static scratch" in lib.ml_last_error()
