"""Torch-level calls of the WKV-7 ClampW C ABI.

These functions take [B, T, H, 64] CUDA tensors, allocate the outputs with
torch (the C ABI itself allocates nothing) and launch on the current CUDA
stream.  Heads [h0, h0 + h_count) of the given tensors are processed in
place; the rest of the outputs is left unwritten (zero-filled when
``zero_rest`` is set), which is how the multi-GPU launcher shards heads
without copies.
"""
from __future__ import annotations

import torch

from . import _lib
from ._lib import ALGO_AUTO, ALGOS, DTYPE_BF16, DTYPE_FP32, check

HEAD_SIZE = 64


def dtype_code(dt: torch.dtype) -> int:
    if dt == torch.bfloat16:
        return DTYPE_BF16
    if dt == torch.float32:
        return DTYPE_FP32
    raise TypeError(f"WKV-7 op supports bfloat16 and float32 inputs, got {dt}")


def algo_code(algo) -> int:
    if isinstance(algo, str):
        return ALGOS[algo]
    return int(algo)


def _check_inputs(xs, names):
    ref = xs[0]
    if ref.dim() != 4 or ref.shape[-1] != HEAD_SIZE:
        raise ValueError(f"expected [B, T, H, {HEAD_SIZE}] tensors, got {tuple(ref.shape)}")
    for x, n in zip(xs, names):
        if not x.is_cuda:
            raise ValueError(f"{n} must be a CUDA tensor (the op has no CPU path)")
        if x.shape != ref.shape:
            raise ValueError(f"{n} has shape {tuple(x.shape)}, expected {tuple(ref.shape)}")
        if x.dtype != ref.dtype:
            raise TypeError(f"{n} has dtype {x.dtype}, expected {ref.dtype}")
        if not x.is_contiguous():
            raise ValueError(f"{n} must be contiguous")
        if x.device != ref.device:
            raise ValueError(f"{n} is on {x.device}, expected {ref.device}")


def _stream_ptr(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def ckpt_bytes(B: int, T: int, h_count: int, dtype: torch.dtype, algo="auto") -> int:
    return int(_lib.lib().camoe_wkv7_ckpt_bytes(B, T, h_count, HEAD_SIZE, dtype_code(dtype),
                                                algo_code(algo)))


def work_bytes(B: int, T: int, h_count: int, dtype: torch.dtype, algo="auto") -> int:
    return int(_lib.lib().camoe_wkv7_work_bytes(B, T, h_count, HEAD_SIZE, dtype_code(dtype),
                                                algo_code(algo)))


DECAYS = ("clampw", "wind")


def _check_carry(states, B, H, device, decay):
    given = {n: s for n, s in states.items() if s is not None}
    if given and decay != "clampw":
        raise ValueError("carried states are supported for the ClampW decay only")
    for n, s in given.items():
        _check_state(s, B, H, device, n)
    return bool(given)


def wkv7_forward(r, w, k, v, a, b, *, algo="auto", save_ckpt: bool = True, h0: int = 0,
                 h_count: int | None = None, y=None, sa=None, ckpt=None, zero_rest=False,
                 decay: str = "clampw", s0=None, s_out=None):
    """Forward.  Returns (y, sa, ckpt); ckpt is None when save_ckpt is False.
    ``decay="wind"`` runs the wind_backstepping op (decay exp(-exp(w))), whose
    (q, z, a) are passed here as (r, a, b).

    Training across calls (ClampW, T a multiple of 16): ``s0`` ([B, H, 64, 64]
    fp32) is the state the sequence starts from and ``s_out`` receives its
    final state; the checkpoint then serves ``wkv7_backward(..., s0=s0)``."""
    if decay not in DECAYS:
        raise ValueError(f"decay must be one of {DECAYS}, got {decay!r}")
    _check_inputs((r, w, k, v, a, b), "rwkvab")
    B, T, H, N = r.shape
    hc = H - h0 if h_count is None else h_count
    alloc = torch.zeros if zero_rest else torch.empty
    if y is None:
        y = alloc(B, T, H, N, dtype=r.dtype, device=r.device)
    if sa is None:
        sa = alloc(B, T, H, N, dtype=torch.float32, device=r.device)
    nbytes = 0
    if save_ckpt:
        nbytes = ckpt_bytes(B, T, hc, r.dtype, algo)
        if ckpt is None:
            ckpt = torch.empty(max(nbytes, 16), dtype=torch.uint8, device=r.device)
        else:
            nbytes = ckpt.numel() * ckpt.element_size()
    else:
        ckpt = None
    carry = _check_carry({"s0": s0, "s_out": s_out}, B, H, r.device, decay)
    ptr = (lambda t: None if t is None else t.data_ptr())
    if carry:
        st = _lib.lib().camoe_wkv7_fwd_carry(
            *(x.data_ptr() for x in (r, w, k, v, a, b)), y.data_ptr(), sa.data_ptr(), ptr(s0),
            ptr(s_out), ptr(ckpt), nbytes, B, T, H, h0, hc, N, dtype_code(r.dtype),
            algo_code(algo), _stream_ptr(r.device))
        check(st)
        return y, sa, ckpt
    if decay == "wind":  # the wind op's argument order: (w, q, k, v, z, a)
        fn, ins = _lib.lib().camoe_wkv7_wind_fwd, (w, r, k, v, a, b)
    else:
        fn, ins = _lib.lib().camoe_wkv7_fwd, (r, w, k, v, a, b)
    st = fn(*(x.data_ptr() for x in ins),
            y.data_ptr(), sa.data_ptr(), ptr(ckpt), nbytes,
            B, T, H, h0, hc, N, dtype_code(r.dtype), algo_code(algo), _stream_ptr(r.device))
    check(st)
    return y, sa, ckpt


def wkv7_forward_value(r, w, k, v, a, b, ckpt, *, h0: int = 0, h_count: int | None = None,
                       y=None, sa=None, s0=None, s_out=None):
    """The value pass of a chunked training forward alone (bf16): ``ckpt``
    holds the key-side records an earlier ``wkv7_forward`` of the same r, w,
    k, a, b (and geometry) wrote; ``v`` and the start state ``s0`` may differ.
    Writes y, sa, ``s_out`` and the checkpoint's states.  Returns (y, sa)."""
    _check_inputs((r, w, k, v, a, b), "rwkvab")
    B, T, H, N = r.shape
    hc = H - h0 if h_count is None else h_count
    _check_carry({"s0": s0, "s_out": s_out}, B, H, r.device, "clampw")
    if y is None:
        y = torch.empty_like(r)
    if sa is None:
        sa = torch.empty(B, T, H, N, dtype=torch.float32, device=r.device)
    ptr = (lambda t: None if t is None else t.data_ptr())
    st = _lib.lib().camoe_wkv7_fwd_value(
        *(x.data_ptr() for x in (r, w, k, v, a, b)), y.data_ptr(), sa.data_ptr(), ptr(s0),
        ptr(s_out), ckpt.data_ptr(), ckpt.numel() * ckpt.element_size(), B, T, H, h0, hc, N,
        dtype_code(r.dtype), _stream_ptr(r.device))
    check(st)
    return y, sa


def _check_state(s, B, H, device, name):
    if s.dtype != torch.float32 or tuple(s.shape) != (B, H, HEAD_SIZE, HEAD_SIZE) \
            or not s.is_contiguous() or s.device != device:
        raise ValueError(f"{name} must be a contiguous float32 [B, H, {HEAD_SIZE}, {HEAD_SIZE}] "
                         f"tensor on {device}, got {tuple(s.shape)} {s.dtype} on {s.device}")


def state_work_bytes(B: int, T: int, h_count: int, dtype: torch.dtype, algo="auto") -> int:
    return int(_lib.lib().camoe_wkv7_state_work_bytes(B, T, h_count, HEAD_SIZE,
                                                      dtype_code(dtype), algo_code(algo)))


def _use_workspace(work, chains: int, device: torch.device) -> bool:
    if work is None or isinstance(work, str):
        # "auto": the fused kernel runs one CTA per chain, so with fewer chains
        # than about 3/4 of the SMs the two-kernel path (key side over every SM)
        # is faster: B200, T=4096, 64 chains 192 us vs 316 us; 128 chains at
        # T=1024 the fused kernel wins, 87 us vs 96 us
        sms = torch.cuda.get_device_properties(device).multi_processor_count
        return 4 * chains < 3 * sms
    return bool(work)


def wkv7_forward_state(r, w, k, v, a, b, state=None, *, algo="auto", h0: int = 0,
                       h_count: int | None = None, y=None, sa=None, out_state=None,
                       inplace: bool = False, zero_rest=False, work="auto"):
    """Stateful inference forward: every chain starts from ``state`` ([B, H, 64, 64]
    fp32, element [b, h, i, j] = S[i][j] with i the value index; None = zero) and
    its state after the last step is returned.  With ``inplace`` the final state
    overwrites ``state``; otherwise it goes to ``out_state`` (allocated when not
    given).  Any T.  ``work``: a uint8 workspace tensor, True / False to allocate
    one or run without, or "auto" (a workspace when there are fewer chains than
    3/4 of the SM count).  Returns (y, sa, final_state)."""
    _check_inputs((r, w, k, v, a, b), "rwkvab")
    B, T, H, N = r.shape
    hc = H - h0 if h_count is None else h_count
    wneed = state_work_bytes(B, T, hc, r.dtype, algo)
    if isinstance(work, torch.Tensor):
        wt = work
    elif wneed > 0 and _use_workspace(work, B * hc, r.device):
        wt = torch.empty(wneed, dtype=torch.uint8, device=r.device)
    else:
        wt = None
    if state is not None:
        _check_state(state, B, H, r.device, "state")
    if inplace:
        if state is None:
            raise ValueError("inplace needs a state tensor")
        out_state = state
    elif out_state is None:
        out_state = (torch.zeros if zero_rest else torch.empty)(B, H, N, N, dtype=torch.float32,
                                                                device=r.device)
    else:
        _check_state(out_state, B, H, r.device, "out_state")
    alloc = torch.zeros if zero_rest else torch.empty
    if y is None:
        y = alloc(B, T, H, N, dtype=r.dtype, device=r.device)
    if sa is None:
        sa = alloc(B, T, H, N, dtype=torch.float32, device=r.device)
    st = _lib.lib().camoe_wkv7_fwd_state(
        r.data_ptr(), w.data_ptr(), k.data_ptr(), v.data_ptr(), a.data_ptr(), b.data_ptr(),
        y.data_ptr(), sa.data_ptr(), None if state is None else state.data_ptr(),
        out_state.data_ptr(), None if wt is None else wt.data_ptr(),
        0 if wt is None else wt.numel() * wt.element_size(), B, T, H, h0, hc, N,
        dtype_code(r.dtype), algo_code(algo), _stream_ptr(r.device))
    check(st)
    return y, sa, out_state


def wkv7_decode_step(r, w, k, v, a, b, state):
    """One generated token for every sequence: inputs [B, H, 64] (or [B, 1, H, 64]),
    ``state`` [B, H, 64, 64] fp32 updated in place.  Returns (y, sa) shaped like r."""
    shape = r.shape
    xs = [x.reshape(x.shape[0], 1, x.shape[-2], x.shape[-1]) for x in (r, w, k, v, a, b)]
    y, sa, _ = wkv7_forward_state(*xs, state, inplace=True)
    return y.reshape(shape), sa.reshape(shape)


def wkv7_backward(r, w, k, v, a, b, dy, dsa, ckpt, *, algo="auto", h0: int = 0,
                  h_count: int | None = None, grads=None, zero_rest=False, work=None,
                  decay: str = "clampw", s0=None, ds_out=None, ds0=None,
                  ds0_only: bool = False):
    """Backward.  ``dsa`` (fp32) may be None.  Returns (dr, dw, dk, dv, da, db).
    ``work`` is the scratch workspace (allocated here when not given).  ``decay``
    as in wkv7_forward (the gradients keep the (r, w, k, v, a, b) order).

    Training across calls (ClampW, T a multiple of 16): ``s0`` is the start
    state the forward was given, ``ds_out`` the gradient of its final state
    (None = zero) and ``ds0`` ([B, H, 64, 64] fp32) receives the gradient of
    the start state.  ``ds0_only`` (chunked path, ``ds0`` given) computes only
    ``ds0`` and dv, skipping the key-side pass; the other five gradients are
    left unwritten."""
    if decay not in DECAYS:
        raise ValueError(f"decay must be one of {DECAYS}, got {decay!r}")
    _check_inputs((r, w, k, v, a, b, dy), "rwkvab" + "y")
    B, T, H, N = r.shape
    hc = H - h0 if h_count is None else h_count
    if dsa is not None:
        if dsa.dtype != torch.float32 or dsa.shape != r.shape or not dsa.is_contiguous() \
                or dsa.device != r.device:
            raise ValueError("dsa must be a contiguous float32 tensor shaped like the inputs")
    if grads is None:
        alloc = torch.zeros if zero_rest else torch.empty
        grads = tuple(alloc(B, T, H, N, dtype=r.dtype, device=r.device) for _ in range(6))
    nbytes = 0 if ckpt is None else ckpt.numel() * ckpt.element_size()
    wneed = work_bytes(B, T, hc, r.dtype, algo)
    if work is None and wneed > 0:
        work = torch.empty(wneed, dtype=torch.uint8, device=r.device)
    wbytes = 0 if work is None else work.numel() * work.element_size()
    dr, dw, dk, dv, da, db = grads
    if ds0_only and ds0 is None:
        raise ValueError("ds0_only needs ds0")
    if _check_carry({"s0": s0, "ds_out": ds_out, "ds0": ds0}, B, H, r.device, decay):
        ptr = (lambda t: None if t is None else t.data_ptr())
        outs = [g.data_ptr() for g in grads]
        if ds0_only:
            outs = [None, None, None, outs[3], None, None]
        st = _lib.lib().camoe_wkv7_bwd_carry(
            *(x.data_ptr() for x in (r, w, k, v, a, b)), dy.data_ptr(), ptr(dsa), ptr(s0),
            ptr(ds_out), ptr(ds0), ptr(ckpt), nbytes, ptr(work), wbytes,
            *outs, B, T, H, h0, hc, N, dtype_code(r.dtype), algo_code(algo),
            _stream_ptr(r.device))
        check(st)
        return grads
    if decay == "wind":  # (w, q, k, v, z, a) in, (dw, dq, dk, dv, dz, da) out
        fn, ins, outs = _lib.lib().camoe_wkv7_wind_bwd, (w, r, k, v, a, b), (dw, dr, dk, dv, da, db)
    else:
        fn, ins, outs = _lib.lib().camoe_wkv7_bwd, (r, w, k, v, a, b), (dr, dw, dk, dv, da, db)
    st = fn(*(x.data_ptr() for x in ins),
            dy.data_ptr(), None if dsa is None else dsa.data_ptr(),
            None if ckpt is None else ckpt.data_ptr(), nbytes,
            None if work is None else work.data_ptr(), wbytes,
            *(g.data_ptr() for g in outs), B, T, H, h0, hc, N, dtype_code(r.dtype),
            algo_code(algo), _stream_ptr(r.device))
    check(st)
    return grads
