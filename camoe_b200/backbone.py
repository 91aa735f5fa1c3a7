"""Drop-in replacement for the WKV-7 op section of the reference's
``camoe/backbone.py`` (lines 14-131).

Same module-level names and call contract:

* ``HEAD_SIZE``, ``CHUNK_LEN``, ``W_SCALE``, ``USE_CUDA``, ``RUN_CUDA_RWKV7``,
  ``CUDA_KERNEL_EXPECTS_FP32`` (camoe/backbone.py:15-20);
* ``init_rwkv7_cuda()`` (camoe/backbone.py:22) — loads the prebuilt sm_100a
  library instead of JIT-compiling, binds ``RUN_CUDA_RWKV7`` and registers the
  reference's torch ops ``torch.ops.rwkv7_clampw.forward/backward`` with the
  reference's argument lists (camoe/cuda/rwkv7_clampw.cpp:12-28).  Unlike the
  reference (camoe/backbone.py:130-131) a failure raises: there is no silent
  CPU fallback;
* ``RWKV7_ClampW`` — the autograd Function (camoe/backbone.py:75-102):
  ``forward(ctx, r, w, k, v, a, b) -> (y, sa)`` with the same assertions, and
  ``backward(ctx, dy, dsa)``, which takes the gradient of both outputs (the
  reference's ``backward(ctx, dy)`` cannot be called by autograd for a
  two-output Function);
* ``RUN_CUDA_RWKV7(r, w, k, v, a, b)`` on ``[B, T, C]`` tensors returning
  ``(y, sa)`` in the caller's dtype (camoe/backbone.py:104-121);
* ``RWKV7_ClampW_State`` — the same op over a piece of a longer sequence:
  start state in, final state out, gradients through both (no counterpart in
  the reference, whose op always starts from zero);
* the reference's second op, ``torch.ops.wind_backstepping.forward/backward``
  (camoe/cuda/wkv7_op.cpp:18-21, decay exp(-exp(w))), registered by
  ``init_rwkv7_cuda`` too, and ``WindBackstepping``, its autograd Function.

Environment flags read by ``init_rwkv7_cuda`` as in the reference:
``CAMOE_FORCE_FP32_KERNEL=1`` selects fp32 inputs and the fp32-exact scan.
``CAMOE_DISABLE_FAST_MATH`` is accepted and has no effect (the kernels always
use accurate ``expf``).  ``CAMOE_WKV7_ALGO`` (auto|scan|chunked) picks the
algorithm for bf16.
"""
from __future__ import annotations

import math
import os

import torch

from . import _lib, ops

HEAD_SIZE = 64
CHUNK_LEN = 16
USE_CUDA = False
RUN_CUDA_RWKV7 = None
CUDA_KERNEL_EXPECTS_FP32 = False
W_SCALE = -math.exp(-0.5)

_ALGO = "auto"
_TORCH_LIB = None


class RWKV7_ClampW(torch.autograd.Function):
    """y, sa = RWKV7_ClampW.apply(r, w, k, v, a, b) on [B, T, H, 64] tensors."""

    @staticmethod
    def forward(ctx, r, w, k, v, a, b):
        B, T, H, C = r.shape
        assert T % CHUNK_LEN == 0
        expected_dtype = torch.float32 if CUDA_KERNEL_EXPECTS_FP32 else torch.bfloat16
        assert all(i.dtype == expected_dtype for i in [r, w, k, v, a, b]), "RWKV7 kernel dtype mismatch"
        assert all(i.is_contiguous() for i in [r, w, k, v, a, b]), "RWKV7 kernel needs contiguous tensors"
        needs_ckpt = any(ctx.needs_input_grad)
        y, sa, ckpt = ops.wkv7_forward(r, w, k, v, a, b, algo=_ALGO, save_ckpt=needs_ckpt)
        ctx.set_materialize_grads(False)
        ctx.save_for_backward(r, w, k, v, a, b, ckpt)
        return y, sa

    @staticmethod
    def backward(ctx, dy, dsa):
        r, w, k, v, a, b, ckpt = ctx.saved_tensors
        expected_dtype = r.dtype
        if dy is None:
            dy = torch.zeros_like(r)
        assert dy.dtype == expected_dtype, "RWKV7 backward dtype mismatch"
        dy = dy.contiguous()
        if dsa is not None:
            dsa = dsa.to(torch.float32).contiguous()
        grads = ops.wkv7_backward(r, w, k, v, a, b, dy, dsa, ckpt, algo=_ALGO)
        return grads


class WindBackstepping(torch.autograd.Function):
    """y, sa = WindBackstepping.apply(w, q, k, v, z, a): the reference's
    wind_backstepping op (decay exp(-exp(w)), camoe/cuda/wkv7_cuda.cu; bound
    by camoe/cuda/wkv7_op.cpp:18-21, no Python wrapper in the reference) as an
    autograd Function on [B, T, H, 64] tensors, gradients of y and sa."""

    @staticmethod
    def forward(ctx, w, q, k, v, z, a):
        assert q.shape[1] % CHUNK_LEN == 0
        assert all(i.is_contiguous() for i in [w, q, k, v, z, a]), "wind kernel needs contiguous tensors"
        y, sa, ckpt = ops.wkv7_forward(q, w, k, v, z, a, algo=_ALGO,
                                       save_ckpt=any(ctx.needs_input_grad), decay="wind")
        ctx.set_materialize_grads(False)
        ctx.save_for_backward(w, q, k, v, z, a, ckpt)
        return y, sa

    @staticmethod
    def backward(ctx, dy, dsa):
        w, q, k, v, z, a, ckpt = ctx.saved_tensors
        dy = torch.zeros_like(q) if dy is None else dy.contiguous()
        if dsa is not None:
            dsa = dsa.to(torch.float32).contiguous()
        dq, dw, dk, dv, dz, da = ops.wkv7_backward(q, w, k, v, z, a, dy, dsa, ckpt, algo=_ALGO,
                                                   decay="wind")
        return dw, dq, dk, dv, dz, da


class RWKV7_ClampW_State(torch.autograd.Function):
    """y, sa, sT = RWKV7_ClampW_State.apply(r, w, k, v, a, b, s0): the ClampW op
    over one piece of a longer sequence, starting from the state ``s0``
    ([B, H, 64, 64] fp32, element [b, h, i, j] = S[i][j], i the value index)
    and returning its final state ``sT``, differentiable in all seven inputs.
    Carrying ``sT`` into the next piece (detached or not) trains over
    sequences longer than one call (truncated BPTT).  T must be a multiple of
    16.  The reference has no carried state: its op always starts from zero
    (camoe/cuda/rwkv7_clampw.cu:28)."""

    @staticmethod
    def forward(ctx, r, w, k, v, a, b, s0):
        B, T, H, C = r.shape
        assert T % CHUNK_LEN == 0
        assert all(i.is_contiguous() for i in [r, w, k, v, a, b, s0]), \
            "RWKV7 kernel needs contiguous tensors"
        sT = torch.empty_like(s0)
        needs_ckpt = any(ctx.needs_input_grad)
        y, sa, ckpt = ops.wkv7_forward(r, w, k, v, a, b, algo=_ALGO, save_ckpt=needs_ckpt,
                                       s0=s0, s_out=sT)
        ctx.set_materialize_grads(False)
        ctx.save_for_backward(r, w, k, v, a, b, s0, ckpt)
        return y, sa, sT

    @staticmethod
    def backward(ctx, dy, dsa, dsT):
        r, w, k, v, a, b, s0, ckpt = ctx.saved_tensors
        dy = torch.zeros_like(r) if dy is None else dy.to(r.dtype).contiguous()
        if dsa is not None:
            dsa = dsa.to(torch.float32).contiguous()
        if dsT is not None:
            dsT = dsT.to(torch.float32).contiguous()
        ds0 = torch.empty_like(s0)
        grads = ops.wkv7_backward(r, w, k, v, a, b, dy, dsa, ckpt, algo=_ALGO, s0=s0,
                                  ds_out=dsT, ds0=ds0)
        return tuple(grads) + (ds0,)


def _run_cuda(r, w, k, v, a, b):
    B, T, HC = r.shape
    H = HC // HEAD_SIZE
    orig_dtype = r.dtype
    target_dtype = torch.float32 if CUDA_KERNEL_EXPECTS_FP32 else torch.bfloat16
    r, w, k, v, a, b = [x.to(dtype=target_dtype).contiguous().view(B, T, H, HEAD_SIZE)
                        for x in [r, w, k, v, a, b]]
    out, sa = RWKV7_ClampW.apply(r, w, k, v, a, b)
    out = out.view(B, T, HC).to(orig_dtype)
    sa = sa.view(B, T, HC).to(orig_dtype)
    return out, sa


def _register_torch_ops():
    """torch.ops.rwkv7_clampw.forward/backward with the reference's arguments
    (camoe/cuda/rwkv7_clampw.cpp:12-28): outputs preallocated by the caller and
    written in place; ``s`` is the [B, H, T/16, 64, 64] fp32 checkpoint tensor
    the reference allocates (camoe/backbone.py:87), used here as the
    checkpoint buffer; ``sa`` is not read by backward (states are recomputed)."""
    global _TORCH_LIB
    if _TORCH_LIB is not None:
        return
    try:
        lib = torch.library.Library("rwkv7_clampw", "DEF")
    except RuntimeError:  # namespace already defined (e.g. by the reference extension)
        return
    lib.define("forward(Tensor r, Tensor w, Tensor k, Tensor v, Tensor a, Tensor b, "
               "Tensor(a!) y, Tensor(b!) s, Tensor(c!) sa) -> ()")
    lib.define("backward(Tensor r, Tensor w, Tensor k, Tensor v, Tensor a, Tensor b, Tensor dy, "
               "Tensor s, Tensor sa, Tensor(a!) dr, Tensor(b!) dw, Tensor(c!) dk, Tensor(d!) dv, "
               "Tensor(e!) da, Tensor(f!) db) -> ()")

    def fwd_impl(r, w, k, v, a, b, y, s, sa):
        ops.wkv7_forward(r, w, k, v, a, b, algo=_ALGO, y=y, sa=sa, ckpt=s.view(torch.uint8))

    def bwd_impl(r, w, k, v, a, b, dy, s, sa, dr, dw, dk, dv, da, db):
        ops.wkv7_backward(r, w, k, v, a, b, dy, None, s.view(torch.uint8), algo=_ALGO,
                          grads=(dr, dw, dk, dv, da, db))

    lib.impl("forward", fwd_impl, "CUDA")
    lib.impl("backward", bwd_impl, "CUDA")
    _TORCH_LIB = lib
    _register_wind_ops()


_WIND_LIB = None


def _register_wind_ops():
    """torch.ops.wind_backstepping.forward/backward with the reference's
    arguments (camoe/cuda/wkv7_op.cpp:18-21): (w, q, k, v, z, a) inputs,
    outputs preallocated and written in place, ``s`` the checkpoint buffer."""
    global _WIND_LIB
    if _WIND_LIB is not None:
        return
    try:
        lib = torch.library.Library("wind_backstepping", "DEF")
    except RuntimeError:  # namespace already defined
        return
    lib.define("forward(Tensor w, Tensor q, Tensor k, Tensor v, Tensor z, Tensor a, "
               "Tensor(a!) y, Tensor(b!) s, Tensor(c!) sa) -> ()")
    lib.define("backward(Tensor w, Tensor q, Tensor k, Tensor v, Tensor z, Tensor a, Tensor dy, "
               "Tensor s, Tensor sa, Tensor(a!) dw, Tensor(b!) dq, Tensor(c!) dk, Tensor(d!) dv, "
               "Tensor(e!) dz, Tensor(f!) da) -> ()")

    def fwd_impl(w, q, k, v, z, a, y, s, sa):
        ops.wkv7_forward(q, w, k, v, z, a, algo=_ALGO, y=y, sa=sa, ckpt=s.view(torch.uint8),
                         decay="wind")

    def bwd_impl(w, q, k, v, z, a, dy, s, sa, dw, dq, dk, dv, dz, da):
        ops.wkv7_backward(q, w, k, v, z, a, dy, None, s.view(torch.uint8), algo=_ALGO,
                          grads=(dq, dw, dk, dv, dz, da), decay="wind")

    lib.impl("forward", fwd_impl, "CUDA")
    lib.impl("backward", bwd_impl, "CUDA")
    _WIND_LIB = lib


def init_rwkv7_cuda():
    """Load the sm_100a WKV-7 library and bind ``RUN_CUDA_RWKV7``.  Raises on failure."""
    global USE_CUDA, RUN_CUDA_RWKV7, CUDA_KERNEL_EXPECTS_FP32, _ALGO
    force_fp32_kernel = os.environ.get("CAMOE_FORCE_FP32_KERNEL", "0") == "1"
    _ALGO = os.environ.get("CAMOE_WKV7_ALGO", "auto")
    if _ALGO not in _lib.ALGOS:
        raise ValueError(f"CAMOE_WKV7_ALGO must be one of {sorted(_lib.ALGOS)}, got {_ALGO!r}")
    _lib.lib()  # raises ImportError when the library is missing
    _register_torch_ops()
    CUDA_KERNEL_EXPECTS_FP32 = force_fp32_kernel
    RUN_CUDA_RWKV7 = _run_cuda
    USE_CUDA = True
