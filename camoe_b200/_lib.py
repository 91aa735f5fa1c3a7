"""ctypes binding of the C ABI in include/camoe_wkv7.h (libcamoe_wkv7.so).

There is no fallback: if the library is missing or fails to load, every op
raises.  The library is built in-tree by camoe_b200.build.
"""
from __future__ import annotations

import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libcamoe_wkv7.so")

DTYPE_BF16, DTYPE_FP32 = 0, 1
ALGO_AUTO, ALGO_SCAN, ALGO_CHUNKED = 0, 1, 2
ALGOS = {"auto": ALGO_AUTO, "scan": ALGO_SCAN, "chunked": ALGO_CHUNKED}

OK, ERR_INVALID_ARG, ERR_UNSUPPORTED, ERR_SHAPE, ERR_ALIGNMENT, ERR_WORKSPACE, ERR_CUDA = range(7)

EXPORTS = ("camoe_wkv7_version", "camoe_wkv7_strerror", "camoe_wkv7_last_cuda_error",
           "camoe_wkv7_device_errors", "camoe_wkv7_ckpt_bytes", "camoe_wkv7_work_bytes",
           "camoe_wkv7_fwd", "camoe_wkv7_bwd", "camoe_wkv7_fwd_state",
           "camoe_wkv7_state_work_bytes", "camoe_wkv7_wind_fwd", "camoe_wkv7_wind_bwd",
           "camoe_wkv7_fwd_carry", "camoe_wkv7_bwd_carry", "camoe_wkv7_seg_chain",
           "camoe_wkv7_fwd_value", "camoe_wkv7_test_hooks")
# the kernels' default wait limit (clock cycles), restored by tests that lower it
DEFAULT_WAIT_LIMIT = 2000000000


# include/camoe_timemix.h: fused elementwise kernels of the time mix
TM_EXPORTS = ("camoe_tm_work_bytes", "camoe_tm_mix_fwd", "camoe_tm_mix_fwd_prev",
              "camoe_tm_mix_bwd", "camoe_tm_prep_fwd",
              "camoe_tm_prep_bwd", "camoe_tm_post_fwd", "camoe_tm_post_bwd", "camoe_tm_lnsa_fwd",
              "camoe_tm_lnsa_bwd", "camoe_tm_lora_work_bytes", "camoe_tm_lora_wgrad")


class CamoeError(RuntimeError):
    """A non-zero status from the C ABI."""

    def __init__(self, status: int, message: str):
        super().__init__(f"camoe_wkv7 error {status}: {message}")
        self.status = status


_lib = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise ImportError(f"{LIB_PATH} is missing; build it with `python -m camoe_b200.build` "
                          "(the operator has no CPU fallback)")
    l = ctypes.CDLL(LIB_PATH)
    i64, vp, ci, sz = ctypes.c_int64, ctypes.c_void_p, ctypes.c_int, ctypes.c_size_t
    l.camoe_wkv7_version.restype = ci
    l.camoe_wkv7_version.argtypes = []
    l.camoe_wkv7_strerror.restype = ctypes.c_char_p
    l.camoe_wkv7_strerror.argtypes = [ci]
    l.camoe_wkv7_last_cuda_error.restype = ci
    l.camoe_wkv7_last_cuda_error.argtypes = []
    l.camoe_wkv7_device_errors.restype = ctypes.c_uint
    l.camoe_wkv7_device_errors.argtypes = []
    l.camoe_wkv7_ckpt_bytes.restype = sz
    l.camoe_wkv7_ckpt_bytes.argtypes = [i64, i64, i64, ci, ci, ci]
    l.camoe_wkv7_work_bytes.restype = sz
    l.camoe_wkv7_work_bytes.argtypes = [i64, i64, i64, ci, ci, ci]
    l.camoe_wkv7_fwd.restype = ci
    l.camoe_wkv7_fwd.argtypes = [vp] * 9 + [sz] + [i64] * 5 + [ci, ci, ci, vp]
    l.camoe_wkv7_fwd_state.restype = ci
    l.camoe_wkv7_fwd_state.argtypes = [vp] * 11 + [sz] + [i64] * 5 + [ci, ci, ci, vp]
    l.camoe_wkv7_state_work_bytes.restype = sz
    l.camoe_wkv7_state_work_bytes.argtypes = [i64, i64, i64, ci, ci, ci]
    l.camoe_wkv7_bwd.restype = ci
    l.camoe_wkv7_bwd.argtypes = [vp] * 9 + [sz, vp, sz] + [vp] * 6 + [i64] * 5 + [ci, ci, ci, vp]
    l.camoe_tm_work_bytes.restype = sz
    l.camoe_wkv7_fwd_carry.restype = ci
    l.camoe_wkv7_fwd_carry.argtypes = [vp] * 11 + [sz] + [i64] * 5 + [ci, ci, ci, vp]
    l.camoe_wkv7_bwd_carry.restype = ci
    l.camoe_wkv7_bwd_carry.argtypes = [vp] * 12 + [sz, vp, sz] + [vp] * 6 + [i64] * 5 + \
        [ci, ci, ci, vp]
    l.camoe_wkv7_fwd_value.restype = ci
    l.camoe_wkv7_fwd_value.argtypes = [vp] * 11 + [sz] + [i64] * 5 + [ci, ci, vp]
    l.camoe_wkv7_test_hooks.restype = ci
    l.camoe_wkv7_test_hooks.argtypes = [ctypes.c_longlong, ci]
    l.camoe_wkv7_seg_chain.restype = ci
    l.camoe_wkv7_seg_chain.argtypes = [vp] * 3 + [i64] * 5 + [ci, vp]
    l.camoe_tm_work_bytes.argtypes = [i64] * 3
    l.camoe_tm_mix_fwd.argtypes = [vp, ci, vp, vp] + [i64] * 3 + [vp]
    l.camoe_tm_mix_fwd_prev.argtypes = [vp, ci, vp, vp, vp] + [i64] * 3 + [vp]
    l.camoe_tm_mix_bwd.argtypes = [vp, ci, vp, vp, vp, vp, vp, sz] + [i64] * 3 + [vp]
    l.camoe_tm_prep_fwd.argtypes = [vp] * 12 + [i64] * 3 + [vp]
    l.camoe_tm_prep_bwd.argtypes = [vp] * 26 + [sz] + [i64] * 3 + [vp]
    l.camoe_tm_post_fwd.argtypes = [vp] * 9 + [i64] * 3 + [vp]
    l.camoe_tm_post_bwd.argtypes = [vp] * 16 + [sz] + [i64] * 3 + [vp]
    l.camoe_tm_lnsa_fwd.argtypes = [vp] * 4 + [i64] * 3 + [vp]
    l.camoe_tm_lnsa_bwd.argtypes = [vp] * 6 + [sz] + [i64] * 3 + [vp]
    l.camoe_tm_lora_wgrad.argtypes = [vp, vp, vp, ci, vp, sz] + [i64] * 3 + [vp]
    for n in TM_EXPORTS[1:]:
        getattr(l, n).restype = ci
    l.camoe_tm_lora_work_bytes.restype = sz
    l.camoe_tm_lora_work_bytes.argtypes = [i64] * 3
    # the wind op's entry points take the ClampW ones' argument types
    l.camoe_wkv7_wind_fwd.restype = ci
    l.camoe_wkv7_wind_fwd.argtypes = l.camoe_wkv7_fwd.argtypes
    l.camoe_wkv7_wind_bwd.restype = ci
    l.camoe_wkv7_wind_bwd.argtypes = l.camoe_wkv7_bwd.argtypes
    _lib = l
    return l


def check(status: int) -> None:
    if status != OK:
        l = lib()
        msg = l.camoe_wkv7_strerror(status).decode()
        if status == ERR_CUDA:
            msg += f" (cudaError {l.camoe_wkv7_last_cuda_error()})"
        raise CamoeError(status, msg)
