"""tcgen05 GEMM core (ml_gemm_bf16) against a torch fp32 matmul of the same bf16 inputs.

Covers every operand-majorness combination, ragged M/N/K (TMA zero-fill at the
edges), multiple K-segments in one accumulator, bf16/fp32 outputs, beta=1
accumulation and the split-K path.
"""

import ctypes

import pytest
import torch

from metal_liger_b200 import _C
from tolerances import assert_close

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _operand(logical, mn_major):
    """Store a logical [rows, K] operand K-major ([rows, K]) or MN-major ([K, rows]).

    TMA needs a row pitch that is a multiple of 16 bytes, so the storage is
    padded to a multiple of 8 columns and a view of the valid part is returned.
    """
    t = logical.t() if mn_major else logical
    r, c = t.shape
    pad = (c + 7) // 8 * 8
    buf = torch.zeros(r, pad, dtype=t.dtype, device=t.device)
    buf[:, :c] = t
    return buf[:, :c]


def run_gemm(segs, m, n, out_dtype=torch.float32, alpha=1.0, beta=0.0, d_init=None,
             a_mn=False, b_mn=False):
    """segs: list of (A [m, k], B [n, k]) bf16 logical operands."""
    lib = _C.load()
    keep = []
    arr = (_C.GemmSegment * len(segs))()
    for i, (a, b) in enumerate(segs):
        sa = _operand(a, a_mn)
        sb = _operand(b, b_mn)
        keep += [sa, sb]
        arr[i].a.ptr = sa.data_ptr()
        arr[i].a.ld = sa.stride(0)
        arr[i].a.mn_major = int(a_mn)
        arr[i].b.ptr = sb.data_ptr()
        arr[i].b.ld = sb.stride(0)
        arr[i].b.mn_major = int(b_mn)
        arr[i].k = a.shape[1]
    d = d_init.clone() if d_init is not None else torch.empty(m, n, dtype=out_dtype, device=DEV)
    k_total = sum(a.shape[1] for a, _ in segs)
    ws_bytes = int(lib.ml_gemm_bf16_workspace_bytes(m, n, k_total))
    ws = torch.empty(max(ws_bytes // 4, 4), dtype=torch.float32, device=DEV)
    rc = lib.ml_gemm_bf16(m, n, arr, len(segs), d.data_ptr(), _C.dtype_code(d), d.stride(0),
                          alpha, beta, ws.data_ptr(), ws.numel() * 4,
                          torch.cuda.current_stream().cuda_stream)
    assert rc == 0, _C.last_error()
    torch.cuda.synchronize()
    assert lib.ml_device_error(None) == 0
    return d, ws_bytes


def reference(segs, alpha=1.0):
    out = None
    for a, b in segs:
        t = a.float() @ b.float().t()
        out = t if out is None else out + t
    return out * alpha


def rand(*shape, seed=0, scale=1.0):
    g = torch.Generator(device=DEV).manual_seed(seed)
    return (scale * torch.randn(*shape, generator=g, device=DEV)).bfloat16()


@pytest.mark.parametrize("a_mn,b_mn", [(False, False), (True, False), (False, True), (True, True)])
@pytest.mark.parametrize("m,n,k", [(128, 256, 64), (256, 256, 512), (300, 200, 96), (77, 40, 130)])
def test_single_segment(a_mn, b_mn, m, n, k, pair_mode):
    a = rand(m, k, seed=1)
    b = rand(n, k, seed=2)
    d, _ = run_gemm([(a, b)], m, n, a_mn=a_mn, b_mn=b_mn)
    ref = reference([(a, b)])
    assert_close(d, ref, rtol=1e-4, atol=1e-4 * ref.abs().max().item(), what="D")


@pytest.mark.parametrize("a_mn,b_mn", [(False, False), (False, True), (True, True)])
def test_multi_segment_accumulates_in_one_tile(a_mn, b_mn, pair_mode):
    m, n = 384, 512
    segs = [(rand(m, 256, seed=3), rand(n, 256, seed=4)),
            (rand(m, 64, seed=5), rand(n, 64, seed=6)),
            (rand(m, 100, seed=7), rand(n, 100, seed=8))]
    d, _ = run_gemm(segs, m, n, a_mn=a_mn, b_mn=b_mn, alpha=0.5)
    ref = reference(segs, alpha=0.5)
    assert_close(d, ref, rtol=1e-4, atol=1e-4 * ref.abs().max().item(), what="D")


def test_bf16_output_and_beta_accumulate(pair_mode):
    m, n, k = 256, 384, 320
    a, b = rand(m, k, seed=9), rand(n, k, seed=10)
    d, _ = run_gemm([(a, b)], m, n, out_dtype=torch.bfloat16)
    ref = reference([(a, b)])
    assert_close(d, ref, dtype=torch.bfloat16, what="bf16 D")
    init = torch.randn(m, n, device=DEV)
    d2, _ = run_gemm([(a, b)], m, n, beta=1.0, d_init=init, alpha=2.0)
    assert_close(d2, init + 2.0 * ref, rtol=1e-4, atol=1e-4 * ref.abs().max().item() * 2,
                 what="beta=1 D")


def test_split_k_path():
    m, n, k = 128, 64, 16384  # one tile, long K -> split-K with a fixed-order reduction
    a, b = rand(m, k, seed=11), rand(n, k, seed=12)
    d, ws_bytes = run_gemm([(a, b)], m, n, a_mn=True, b_mn=True)
    assert ws_bytes > 0, "expected the split-K path"
    ref = reference([(a, b)])
    assert_close(d, ref, rtol=1e-4, atol=1e-4 * ref.abs().max().item(), what="split-K D")
    d_again, _ = run_gemm([(a, b)], m, n, a_mn=True, b_mn=True)
    assert torch.equal(d, d_again), "split-K reduction must be deterministic"


def test_split_k_pair_tiles(pair_mode):
    m, n, k = 512, 256, 8192  # few tiles, long K -> split-K on 256 x 256 tiles
    a, b = rand(m, k, seed=15), rand(n, k, seed=16)
    d, ws_bytes = run_gemm([(a, b)], m, n, a_mn=True, b_mn=True)
    ref = reference([(a, b)])
    assert_close(d, ref, rtol=1e-4, atol=1e-4 * ref.abs().max().item(), what="split-K D")
    d_again, _ = run_gemm([(a, b)], m, n, a_mn=True, b_mn=True)
    assert torch.equal(d, d_again), "split-K reduction must be deterministic"


@pytest.mark.parametrize("a_mn,b_mn", [(False, False), (True, True)])
def test_ragged_many_pair_tiles(a_mn, b_mn, pair_mode):
    # more tiles than SM pairs (persistent loop) with ragged M/N/K edges
    m, n, k = 2500, 3000, 200
    a, b = rand(m, k, seed=17), rand(n, k, seed=18)
    d, _ = run_gemm([(a, b)], m, n, a_mn=a_mn, b_mn=b_mn)
    ref = reference([(a, b)])
    assert_close(d, ref, rtol=1e-4, atol=1e-4 * ref.abs().max().item(), what="D")


def test_large_square(pair_mode):
    m = n = k = 4096
    a, b = rand(m, k, seed=13), rand(n, k, seed=14)
    d, _ = run_gemm([(a, b)], m, n, out_dtype=torch.bfloat16)
    ref = reference([(a, b)])
    assert_close(d, ref, dtype=torch.bfloat16, norm_rtol=5e-3, what="4096^3 D")


@pytest.mark.parametrize("reserve", [16, 100])
def test_reserved_sms_give_the_same_result(reserve, pair_mode):
    """A GEMM launched while SMs are reserved for other streams
    (ml_gemm_set_reserved_sms) runs on a smaller persistent grid and writes
    exactly the same D; the setting is restored afterwards."""
    m, n, k = 1024, 768, 512
    a, b = rand(m, k, seed=21), rand(n, k, seed=22)
    d0, _ = run_gemm([(a, b)], m, n)
    with _C.gemm_reserved_sms(reserve):
        d1, _ = run_gemm([(a, b)], m, n)
    assert torch.equal(d0, d1)
    prev = ctypes.c_int(-1)
    _C.call("ml_gemm_set_reserved_sms", 0, ctypes.byref(prev))
    assert prev.value == 0


def test_bad_arguments_rejected():
    lib = _C.load()
    arr = (_C.GemmSegment * 1)()
    a = rand(64, 60, seed=1)  # ld 60 is not a multiple of 8
    arr[0].a.ptr = a.data_ptr()
    arr[0].a.ld = 60
    arr[0].b.ptr = a.data_ptr()
    arr[0].b.ld = 60
    arr[0].k = 60
    d = torch.empty(64, 64, device=DEV)
    rc = lib.ml_gemm_bf16(64, 64, arr, 1, d.data_ptr(), 0, 64, 1.0, 0.0, None, 0,
                          torch.cuda.current_stream().cuda_stream)
    assert rc == 1 and b"multiple of 8" in lib.ml_last_error()


def test_bounded_wait_gives_up_and_reports():
    """The bounded mbarrier wait of the tcgen05 kernels, made to run out on
    purpose (a phase nothing completes, 20 ms limit): the kernel returns, the
    device error word holds (site 6 << 8) | ML_ERR_TIMEOUT, reading it clears
    it, and the context stays usable (a GEMM runs and checks after it)."""
    lib = _C.load()
    st = torch.cuda.current_stream().cuda_stream
    assert lib.ml_device_error(st) == 0
    assert lib.ml_selftest_bounded_wait(20000, st) == 0
    assert lib.ml_device_error(st) == (6 << 8) | 4
    assert lib.ml_device_error(st) == 0
    assert lib.ml_selftest_bounded_wait(10, st) != 0      # limits below 1 ms are refused
    a = torch.randn(256, 128, device=DEV).bfloat16()
    b = torch.randn(192, 128, device=DEV).bfloat16()
    d, _ = run_gemm([(a, b)], 256, 192)
    torch.testing.assert_close(d.float(), reference([(a, b)]), rtol=2e-2, atol=2e-1)
