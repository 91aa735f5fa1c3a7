"""The allocation-free entry point camoe_wkv7_fwd_bwd_noalloc.

It serves callers that cannot create device allocations (a host whose device
memory belongs to another runtime's pooled allocator, or a training step that
must not let cudaMalloc synchronise the device): it runs the forward and the
backward in one call and keeps the state checkpoint in a library-owned device
array instead of a caller buffer.  It launches the same kernels on the same
inputs as the ordinary entry points (camoe_wkv7_fwd + camoe_wkv7_bwd), so its
results must equal theirs bit for bit, on consecutive calls that reuse the
array.  The test buffers themselves are allocated by torch; the entry point
allocates nothing.

This file is collected last so that, if it fails, a run that stops at the first
failure has already run every other test.
"""
import ctypes

import numpy as np
import pytest
import torch

from camoe_b200 import _lib, ops
from camoe_b200.inputs import make_inputs

NAMES = ("r", "w", "k", "v", "a", "b")
SCRATCH_BYTES = 64 << 20  # CAMOE_WKV7_NOALLOC_SCRATCH_BYTES


@pytest.fixture(autouse=True)
def _no_device_timeouts():
    """Every bounded device-side wait must have completed (no timed-out kernel)."""
    if not torch.cuda.is_available():
        yield
        return
    before = _lib.lib().camoe_wkv7_device_errors()
    yield
    assert _lib.lib().camoe_wkv7_device_errors() == before


def entry():
    f = _lib.lib().camoe_wkv7_fwd_bwd_noalloc
    vp, i64, ci = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int
    f.argtypes = [vp] * 16 + [i64] * 5 + [ci, ci, ci, vp]
    f.restype = ci
    return f


def test_noalloc_rejects_problems_larger_than_its_scratch():
    # 4097 chains x one 16-step chunk needs more than 64 MiB of checkpoint and
    # workspace; rejected before any device work
    p = ctypes.c_void_p(256)
    args = [p] * 7 + [None] + [p] * 8
    st = entry()(*args, 4097, 16, 1, 0, 1, 64, _lib.DTYPE_BF16, _lib.ALGO_AUTO, None)
    assert st == _lib.ERR_WORKSPACE
    st = entry()(*args, 1, 16, 1, 0, 1, 32, _lib.DTYPE_BF16, _lib.ALGO_AUTO, None)
    assert st == _lib.ERR_UNSUPPORTED
    # sequence lengths whose byte counts would overflow 64-bit arithmetic are
    # rejected by the chunk-count bound, never wrapped into a small size
    for T in (1 << 62, (1 << 63) - 1):
        for algo in (_lib.ALGO_CHUNKED, _lib.ALGO_SCAN):
            st = entry()(*args, 1, T, 1, 0, 1, 64, _lib.DTYPE_BF16, algo, None)
            assert st == _lib.ERR_WORKSPACE, (T, algo)
    st = entry()(*args, 0x7fffffff, (1 << 40), 1, 0, 1, 64, _lib.DTYPE_BF16,
                 _lib.ALGO_AUTO, None)
    assert st == _lib.ERR_WORKSPACE


def _bits(t):
    """The tensor's bytes as an integer array (bit-for-bit comparison)."""
    t = t.contiguous().cpu()
    return (t.view(torch.int16) if t.element_size() == 2 else t.view(torch.int32)).numpy()


@pytest.mark.gpu
@pytest.mark.parametrize("dtype,algo", [(torch.bfloat16, "chunked"), (torch.bfloat16, "scan"),
                                        (torch.float32, "scan")],
                         ids=["bf16-chunked", "bf16-scan", "fp32-scan"])
def test_noalloc_matches_ordinary_entry_points_on_consecutive_calls(dtype, algo):
    f = entry()
    # calls in a row with different problems: each reuses the scratch that still
    # holds the previous call's checkpoint; the largest uses nearly all of it; the
    # last works on heads [3, 7) of 11 in place
    cases = [(2, 96, 4, 0, 4, 31, True), (1, 200, 3, 0, 3, 32, False),
             (2, 1024, 14, 0, 14, 33, True), (2, 80, 11, 3, 4, 34, True)]
    for B, T, H, h0, hc, seed, with_dsa in cases:
        need = ops.ckpt_bytes(B, T, hc, dtype, algo) + ops.work_bytes(B, T, hc, dtype, algo)
        assert need + 256 <= SCRATCH_BYTES
        inp = make_inputs(B, T, H, 64, seed=seed, with_dsa=with_dsa)
        xs = [inp[n].to(dtype).cuda() for n in NAMES]
        dy = inp["dy"].to(dtype).cuda()
        dsa = inp["dsa"].cuda() if with_dsa else None
        y0, sa0, ck = ops.wkv7_forward(*xs, algo=algo, h0=h0, h_count=hc, zero_rest=True)
        g0 = ops.wkv7_backward(*xs, dy, dsa, ck, algo=algo, h0=h0, h_count=hc, zero_rest=True)
        y1 = torch.zeros_like(xs[0])
        sa1 = torch.zeros(xs[0].shape, dtype=torch.float32, device="cuda")
        g1 = [torch.zeros_like(xs[0]) for _ in range(6)]
        stream = torch.cuda.current_stream().cuda_stream
        st = f(*[x.data_ptr() for x in xs], dy.data_ptr(), None if dsa is None else dsa.data_ptr(),
               y1.data_ptr(), sa1.data_ptr(), *[t.data_ptr() for t in g1],
               B, T, H, h0, hc, 64, ops.dtype_code(dtype), ops.algo_code(algo), stream)
        assert st == 0, _lib.lib().camoe_wkv7_strerror(st)
        torch.cuda.synchronize()
        for name, a, b in zip(("y", "sa", "dr", "dw", "dk", "dv", "da", "db"),
                              [y0, sa0, *g0], [y1, sa1, *g1]):
            np.testing.assert_array_equal(_bits(b), _bits(a), err_msg=f"{name} {B, T, H, h0, hc}")
