"""C ABI checks that need no GPU: the library loads, exports every function
the header declares, and rejects bad arguments before touching the device."""
import ctypes
import os
import re

import pytest

from camoe_b200 import _lib

INCLUDE = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include")
HEADER = os.path.join(INCLUDE, "camoe_wkv7.h")
HEADERS = [os.path.join(INCLUDE, h) for h in ("camoe_wkv7.h", "camoe_timemix.h")]


def _sources():
    return "\n".join(re.sub(r"/\*.*?\*/", "", open(h).read(), flags=re.S) for h in HEADERS)


def header_functions():
    return sorted(set(re.findall(r"\b(camoe_(?:wkv7|tm)_\w+)\s*\(", _sources())))


def test_header_declares_expected_entry_points():
    names = header_functions()
    for n in _lib.EXPORTS + _lib.TM_EXPORTS:
        assert n in names


def header_param_counts():
    out = {}
    for name, params in re.findall(r"\b(camoe_(?:wkv7|tm)_\w+)\s*\(([^)]*)\)\s*;", _sources()):
        params = params.strip()
        out[name] = 0 if params in ("", "void") else params.count(",") + 1
    return out


def test_bindings_declare_the_header_argument_counts():
    """Every function the ctypes binding calls has argtypes of the header's arity
    (an unset argtypes would pass 64-bit pointers and sizes as C ints)."""
    lib = _lib.lib()
    counts = header_param_counts()
    for name in _lib.EXPORTS + _lib.TM_EXPORTS:
        f = getattr(lib, name)
        assert f.argtypes is not None, name
        assert len(f.argtypes) == counts[name], name


def test_library_exports_every_header_function():
    lib = _lib.lib()
    for name in header_functions():
        assert hasattr(lib, name), name


def test_version_and_strerror():
    lib = _lib.lib()
    assert lib.camoe_wkv7_version() >= 10000
    for code in range(7):
        assert lib.camoe_wkv7_strerror(code)
    assert b"unknown" in lib.camoe_wkv7_strerror(99)


def test_ckpt_bytes_fits_the_reference_checkpoint_tensor():
    lib = _lib.lib()
    for dtype in (_lib.DTYPE_BF16, _lib.DTYPE_FP32):
        for algo in (_lib.ALGO_AUTO, _lib.ALGO_SCAN, _lib.ALGO_CHUNKED):
            if dtype == _lib.DTYPE_FP32 and algo == _lib.ALGO_CHUNKED:
                assert lib.camoe_wkv7_ckpt_bytes(4, 4096, 16, 64, dtype, algo) == 0
                continue
            for B, T, H in ((1, 64, 2), (8, 1024, 16), (4, 4096, 16), (2, 65536, 32)):
                got = lib.camoe_wkv7_ckpt_bytes(B, T, H, 64, dtype, algo)
                ref = B * H * (T // 16) * 64 * 64 * 4  # camoe/backbone.py:87
                assert 0 < got <= ref
    assert lib.camoe_wkv7_ckpt_bytes(1, 64, 1, 32, 0, 0) == 0   # N != 64
    assert lib.camoe_wkv7_ckpt_bytes(1, 64, 1, 64, 7, 0) == 0   # bad dtype
    assert lib.camoe_wkv7_ckpt_bytes(0, 64, 1, 64, 0, 0) == 0   # empty


def _fwd(B=1, T=16, H=1, h0=0, hc=1, N=64, dtype=0, algo=0, ptr=16, ckpt=None, nbytes=0):
    lib = _lib.lib()
    p = ctypes.c_void_p(ptr)
    return lib.camoe_wkv7_fwd(p, p, p, p, p, p, p, p, ckpt, nbytes, B, T, H, h0, hc, N,
                              dtype, algo, None)


def test_work_bytes():
    lib = _lib.lib()
    assert lib.camoe_wkv7_work_bytes(4, 4096, 16, 64, _lib.DTYPE_FP32, _lib.ALGO_SCAN) == 0
    assert lib.camoe_wkv7_work_bytes(4, 4096, 16, 64, _lib.DTYPE_BF16, _lib.ALGO_CHUNKED) > 0
    assert lib.camoe_wkv7_work_bytes(4, 4096, 16, 32, _lib.DTYPE_BF16, _lib.ALGO_CHUNKED) == 0


def test_fwd_argument_errors_need_no_device():
    assert _fwd(N=32) == _lib.ERR_UNSUPPORTED
    assert _fwd(B=-1) == _lib.ERR_INVALID_ARG
    assert _fwd(H=2, h0=1, hc=2) == _lib.ERR_INVALID_ARG     # head range past H_total
    assert _fwd(dtype=5) == _lib.ERR_UNSUPPORTED
    assert _fwd(dtype=1, algo=2) == _lib.ERR_UNSUPPORTED     # chunked is bf16 only
    assert _fwd(algo=9) == _lib.ERR_UNSUPPORTED
    assert _fwd(ptr=0) == _lib.ERR_INVALID_ARG               # null pointers
    assert _fwd(ptr=24) == _lib.ERR_ALIGNMENT                # 8-byte aligned only
    assert _fwd(ckpt=ctypes.c_void_p(16), nbytes=10) == _lib.ERR_WORKSPACE
    # empty work returns before any device call
    assert _fwd(B=0) == _lib.OK
    assert _fwd(T=0) == _lib.OK
    assert _fwd(hc=0) == _lib.OK


def test_bwd_argument_errors_need_no_device():
    lib = _lib.lib()
    p = ctypes.c_void_p(16)

    def bwd(ckpt=p, nbytes=1 << 40, dsa=None, work=p, wbytes=1 << 40, **kw):
        g = dict(B=1, T=32, H=1, h0=0, hc=1, N=64, dtype=0, algo=0)
        g.update(kw)
        return lib.camoe_wkv7_bwd(p, p, p, p, p, p, p, dsa, ckpt, nbytes, work, wbytes,
                                  p, p, p, p, p, p, g["B"], g["T"], g["H"], g["h0"], g["hc"],
                                  g["N"], g["dtype"], g["algo"], None)

    assert bwd(ckpt=None) == _lib.ERR_INVALID_ARG
    assert bwd(nbytes=100) == _lib.ERR_WORKSPACE
    assert bwd(work=None) == _lib.ERR_INVALID_ARG            # chunked needs a workspace
    assert bwd(wbytes=100) == _lib.ERR_WORKSPACE
    assert bwd(work=ctypes.c_void_p(24)) == _lib.ERR_ALIGNMENT
    assert bwd(dsa=ctypes.c_void_p(20)) == _lib.ERR_ALIGNMENT
    assert bwd(N=128) == _lib.ERR_UNSUPPORTED
    assert bwd(B=0) == _lib.OK


def test_fwd_state_argument_errors_need_no_device():
    lib = _lib.lib()
    p = ctypes.c_void_p(16)

    def fst(s0=ctypes.c_void_p(1 << 20), s_out=ctypes.c_void_p(1 << 30), ptr=p, work=None,
            wbytes=0, **kw):
        g = dict(B=2, T=32, H=4, h0=0, hc=4, N=64, dtype=0, algo=0)
        g.update(kw)
        return lib.camoe_wkv7_fwd_state(ptr, ptr, ptr, ptr, ptr, ptr, ptr, ptr, s0, s_out,
                                        work, wbytes, g["B"], g["T"], g["H"], g["h0"], g["hc"],
                                        g["N"], g["dtype"], g["algo"], None)

    assert fst(N=32) == _lib.ERR_UNSUPPORTED
    assert fst(dtype=1, algo=2) == _lib.ERR_UNSUPPORTED
    assert fst(H=2, h0=1, hc=2) == _lib.ERR_INVALID_ARG
    assert fst(s0=ctypes.c_void_p(1 << 20 | 8)) == _lib.ERR_ALIGNMENT
    assert fst(s_out=ctypes.c_void_p(1 << 30 | 4)) == _lib.ERR_ALIGNMENT
    # partially overlapping start and final state arrays (2*4*16 KiB each)
    assert fst(s_out=ctypes.c_void_p((1 << 20) + 4096)) == _lib.ERR_INVALID_ARG
    assert fst(s0=ctypes.c_void_p((1 << 30) - 16384)) == _lib.ERR_INVALID_ARG
    assert fst(ptr=ctypes.c_void_p(0)) == _lib.ERR_INVALID_ARG
    assert fst(ptr=ctypes.c_void_p(24)) == _lib.ERR_ALIGNMENT
    need = lib.camoe_wkv7_state_work_bytes(2, 32, 4, 64, 0, 0)
    assert need == 2 * 4 * 2 * 9472      # one key-side record per chunk and chain
    assert lib.camoe_wkv7_state_work_bytes(2, 16, 4, 64, 0, 0) == 0      # decode kernel
    assert lib.camoe_wkv7_state_work_bytes(2, 32, 4, 64, 1, 0) == 0      # fp32 scan
    assert lib.camoe_wkv7_state_work_bytes(2, 16, 4, 64, 0, 2) > 0       # forced chunked
    assert fst(work=ctypes.c_void_p(1 << 40), wbytes=need - 1) == _lib.ERR_WORKSPACE
    assert fst(work=ctypes.c_void_p((1 << 40) + 8), wbytes=need) == _lib.ERR_ALIGNMENT
    # nothing to do: no device call
    assert fst(B=0) == _lib.OK
    assert fst(T=0, s_out=ctypes.c_void_p(1 << 20)) == _lib.OK   # in place, no step
    assert fst(T=0, s_out=None) == _lib.OK


def test_carry_argument_errors_need_no_device():
    lib = _lib.lib()
    p = ctypes.c_void_p(16)
    s = ctypes.c_void_p(1 << 30)

    def fc(s0=s, s_out=None, **kw):
        g = dict(B=1, T=32, H=1, h0=0, hc=1, N=64, dtype=0, algo=0)
        g.update(kw)
        return lib.camoe_wkv7_fwd_carry(p, p, p, p, p, p, p, p, s0, s_out, None, 0, g["B"],
                                        g["T"], g["H"], g["h0"], g["hc"], g["N"], g["dtype"],
                                        g["algo"], None)

    def bc(s0=s, ds_out=None, ds0=None, **kw):
        g = dict(B=1, T=32, H=1, h0=0, hc=1, N=64, dtype=0, algo=0)
        g.update(kw)
        return lib.camoe_wkv7_bwd_carry(p, p, p, p, p, p, p, None, s0, ds_out, ds0, p, 1 << 40,
                                        p, 1 << 40, p, p, p, p, p, p, g["B"], g["T"], g["H"],
                                        g["h0"], g["hc"], g["N"], g["dtype"], g["algo"], None)

    assert fc(T=40) == _lib.ERR_SHAPE                 # not a whole number of chunks
    assert fc(T=0) == _lib.ERR_SHAPE                  # nothing to carry the state through
    assert fc(s0=ctypes.c_void_p((1 << 30) + 4)) == _lib.ERR_ALIGNMENT
    assert fc(s0=None, s_out=ctypes.c_void_p(8)) == _lib.ERR_ALIGNMENT
    assert fc(N=32) == _lib.ERR_UNSUPPORTED
    assert fc(B=0) == _lib.OK
    assert bc(T=24) == _lib.ERR_SHAPE
    assert bc(s0=None, ds0=s, T=0) == _lib.ERR_SHAPE
    assert bc(ds_out=ctypes.c_void_p(40)) == _lib.ERR_ALIGNMENT
    assert bc(ds0=ctypes.c_void_p(4)) == _lib.ERR_ALIGNMENT
    assert bc(hc=0) == _lib.OK

    def key_null(ds0, dtype, algo):
        n = None
        return lib.camoe_wkv7_bwd_carry(p, p, p, p, p, p, p, None, s, None, ds0, p, 1 << 40, p,
                                        1 << 40, n, n, n, p, n, n, 1, 32, 1, 0, 1, 64, dtype,
                                        algo, None)

    # dv and ds0 only: chunked path with ds0 given; the scan or no ds0 need all six
    assert key_null(None, 0, 2) == _lib.ERR_INVALID_ARG
    assert key_null(s, 1, 0) == _lib.ERR_INVALID_ARG      # fp32 resolves to the scan
    assert key_null(s, 0, 1) == _lib.ERR_INVALID_ARG


def test_fwd_value_argument_errors_need_no_device():
    lib = _lib.lib()
    p = ctypes.c_void_p(16)

    def fv(ckpt=p, nbytes=1 << 40, s0=None, dtype=0, T=32, B=1):
        return lib.camoe_wkv7_fwd_value(p, p, p, p, p, p, p, p, s0, None, ckpt, nbytes, B, T, 1,
                                        0, 1, 64, dtype, None)

    assert fv(dtype=1) == _lib.ERR_UNSUPPORTED       # chunked records are bf16 only
    assert fv(ckpt=None) == _lib.ERR_INVALID_ARG     # the records live in the checkpoint
    assert fv(nbytes=100) == _lib.ERR_WORKSPACE
    assert fv(T=0, s0=p) == _lib.ERR_SHAPE
    assert fv(T=24, s0=p) == _lib.ERR_SHAPE
    assert fv(B=0) == _lib.OK


def test_seg_chain_argument_errors_need_no_device():
    lib = _lib.lib()
    p = ctypes.c_void_p(16)

    def sc(st=p, tr=p, lo=p, B=2, P=4, H=4, h0=0, hc=4, backward=0):
        return lib.camoe_wkv7_seg_chain(st, tr, lo, B, P, H, h0, hc, backward, None)

    assert sc(P=0) == _lib.ERR_INVALID_ARG
    assert sc(h0=2, hc=3) == _lib.ERR_INVALID_ARG         # head range past H_total
    assert sc(backward=2) == _lib.ERR_INVALID_ARG
    assert sc(tr=None) == _lib.ERR_INVALID_ARG
    assert sc(lo=ctypes.c_void_p(40)) == _lib.ERR_ALIGNMENT
    # nothing to chain: no device call
    assert sc(P=1) == _lib.OK
    assert sc(B=0) == _lib.OK
    assert sc(hc=0) == _lib.OK


def test_error_raises_camoe_error():
    with pytest.raises(_lib.CamoeError) as ei:
        _lib.check(_lib.ERR_ALIGNMENT)
    assert ei.value.status == _lib.ERR_ALIGNMENT


def test_test_hooks_reject_out_of_range_arguments():
    """The wait-limit hook validates before touching any device state."""
    lib = _lib.lib()
    assert lib.camoe_wkv7_test_hooks(999, -1) == _lib.ERR_INVALID_ARG
    assert lib.camoe_wkv7_test_hooks(_lib.DEFAULT_WAIT_LIMIT + 1, -1) == _lib.ERR_INVALID_ARG
    assert lib.camoe_wkv7_test_hooks(_lib.DEFAULT_WAIT_LIMIT, -2) == _lib.ERR_INVALID_ARG


def test_lora_wgrad_argument_errors_need_no_device():
    """Shape, null and alignment errors return before any CUDA call."""
    lib = _lib.lib()
    fake, odd = ctypes.c_void_p(1 << 20), ctypes.c_void_p((1 << 20) + 8)
    call = (lambda big, thin, dw, out_cd, work, nw, R, C, D:
            lib.camoe_tm_lora_wgrad(big, thin, dw, out_cd, work, nw, R, C, D, None))
    assert lib.camoe_tm_lora_work_bytes(8192, 1024, 160) == 16 * 1024 * 160 * 4
    assert lib.camoe_tm_lora_work_bytes(5, 128, 64) == 1 * 128 * 64 * 4
    assert call(fake, fake, fake, 1, fake, 1 << 30, 64, 1024, 48) == _lib.ERR_UNSUPPORTED  # D % 32
    assert call(fake, fake, fake, 1, fake, 1 << 30, 64, 1024, 32) == _lib.ERR_UNSUPPORTED  # D < 64
    assert call(fake, fake, fake, 1, fake, 1 << 30, 64, 192, 64) == _lib.ERR_UNSUPPORTED   # C % 128
    assert call(fake, fake, fake, 1, fake, 1 << 30, 64, 1024, 288) == _lib.ERR_UNSUPPORTED  # D > 256
    assert call(fake, fake, fake, 2, fake, 1 << 30, 64, 1024, 64) == _lib.ERR_INVALID_ARG
    assert call(None, fake, fake, 1, fake, 1 << 30, 64, 1024, 64) == _lib.ERR_INVALID_ARG
    assert call(odd, fake, fake, 1, fake, 1 << 30, 64, 1024, 64) == _lib.ERR_ALIGNMENT
    assert call(fake, fake, fake, 1, None, 1 << 30, 64, 1024, 64) == _lib.ERR_INVALID_ARG
    assert call(fake, fake, fake, 1, fake, 16, 64, 1024, 64) == _lib.ERR_WORKSPACE


def test_lora_work_bytes_matches_the_python_sizing():
    from camoe_b200 import timemix
    lib = _lib.lib()
    for R in (1, 5, 63, 64, 65, 1000, 1024, 1025, 8192, 100000):
        for C, D in ((1024, 64), (128, 160), (2048, 256)):
            assert lib.camoe_tm_lora_work_bytes(R, C, D) == timemix.lora_work_bytes(R, C, D)
