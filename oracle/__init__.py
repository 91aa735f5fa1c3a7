"""CPU oracle for the WKV-7 ClampW recurrence — TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline leg of
``bench.py`` may import this package, and only as the result to compare against
(or as the timed CPU baseline).  The ``camoe_b200`` product path never imports it.

Contents:

* ``fwd`` / ``bwd`` / ``fwd_state`` / ``bwd_state`` — ctypes bindings of ``wkv7_oracle.c`` (a plain-C
  restatement of ``camoe/backbone.py:264-294`` and of the gradient formulas of
  ``camoe/cuda/rwkv7_clampw.cu:83-170``), in float64 (ground truth) or float32
  (reference precision), OpenMP over (batch, head) chains.
* ``RefOp`` — the reference's own ClampW (or wind_backstepping) CUDA op,
  compiled by ``oracle/Makefile`` from the reference's sources into
  ``oracle/_ref/``; the GPU parity tests call it with device pointers.
* ``torch_reference`` — a float64 torch restatement of the same recurrence
  whose gradients come from autograd; an independent cross-check of ``bwd``.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_DIR = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_DIR, "_build", "libwkv7_oracle.so")
_REF_DIR = os.path.join(_DIR, "_ref")

W_SCALE = -0.6065306597126334  # -exp(-1/2), camoe/backbone.py:20

_lib = None


def build(ref: bool = False) -> None:
    """Compile the oracle (and, with ``ref=True``, the reference op) via make."""
    targets = ["all"] + (["ref"] if ref else [])
    subprocess.run(["make", "-s", "-C", _DIR] + targets, check=True)


def _load():
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(_LIB_PATH):
        build()
    lib = ctypes.CDLL(_LIB_PATH)
    i64, fp, ci = ctypes.c_int64, ctypes.c_void_p, ctypes.c_int
    for suf in ("f64", "f32"):
        f = getattr(lib, f"wkv7_oracle_fwd_{suf}")
        f.argtypes = [i64] * 4 + [fp] * 8 + [ci, ci]
        f.restype = ci
        g = getattr(lib, f"wkv7_oracle_bwd_{suf}")
        g.argtypes = [i64] * 5 + [fp] * 14 + [ci, ci]
        g.restype = ci
        gs = getattr(lib, f"wkv7_oracle_bwd_state_{suf}")
        gs.argtypes = [i64] * 5 + [fp] * 17 + [ci, ci]
        gs.restype = ci
        h = getattr(lib, f"wkv7_oracle_fwd_state_{suf}")
        h.argtypes = [i64] * 4 + [fp] * 10 + [ci, ci]
        h.restype = ci
    lib.wkv7_oracle_decay.argtypes = [ctypes.c_double]
    lib.wkv7_oracle_decay.restype = ctypes.c_double
    _lib = lib
    return lib


def _f32(x) -> np.ndarray:
    if hasattr(x, "detach"):  # torch tensor
        x = x.detach().float().cpu().numpy()
    return np.ascontiguousarray(x, dtype=np.float32)


def _ptr(x: np.ndarray | None):
    return None if x is None else x.ctypes.data_as(ctypes.c_void_p)


def default_threads() -> int:
    return max(1, len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else os.cpu_count() or 1)


DECAYS = {"clampw": 0, "wind": 1}


def fwd(r, w, k, v, a, b, precision: str = "f64", threads: int | None = None,
        decay: str = "clampw"):
    """Forward recurrence.  Inputs [B,T,H,N] (numpy or torch); returns (y, sa) float32.
    ``decay="wind"`` applies the wind_backstepping decay exp(-exp(w)) (then r, a,
    b are that op's q, z, a)."""
    r, w, k, v, a, b = (_f32(x) for x in (r, w, k, v, a, b))
    B, T, H, N = r.shape
    y = np.empty_like(r)
    sa = np.empty_like(r)
    fn = getattr(_load(), f"wkv7_oracle_fwd_{precision}")
    rc = fn(B, T, H, N, *map(_ptr, (r, w, k, v, a, b, y, sa)), DECAYS[decay],
            threads or default_threads())
    if rc != 0:
        raise RuntimeError(f"oracle forward failed with code {rc}")
    return y, sa


def fwd_state(r, w, k, v, a, b, s0=None, precision: str = "f64", threads: int | None = None,
              decay: str = "clampw"):
    """Forward from the start state ``s0`` ([B,H,N,N], element [b,h,i,j] = S[i][j]
    with i the value index; None = zero).  Returns (y, sa, s_final) float32."""
    r, w, k, v, a, b = (_f32(x) for x in (r, w, k, v, a, b))
    B, T, H, N = r.shape
    s0 = None if s0 is None else _f32(s0).reshape(B, H, N, N)
    y = np.empty_like(r)
    sa = np.empty_like(r)
    sT = np.empty((B, H, N, N), dtype=np.float32)
    fn = getattr(_load(), f"wkv7_oracle_fwd_state_{precision}")
    rc = fn(B, T, H, N, *map(_ptr, (r, w, k, v, a, b, s0, y, sa, sT)), DECAYS[decay],
            threads or default_threads())
    if rc != 0:
        raise RuntimeError(f"oracle stateful forward failed with code {rc}")
    return y, sa, sT


def bwd(r, w, k, v, a, b, dy, dsa=None, precision: str = "f64", ckpt: int = 64,
        threads: int | None = None, decay: str = "clampw"):
    """Exact gradients (dr, dw, dk, dv, da, db) of sum(dy*y) + sum(dsa*sa), float32."""
    r, w, k, v, a, b, dy = (_f32(x) for x in (r, w, k, v, a, b, dy))
    dsa = None if dsa is None else _f32(dsa)
    B, T, H, N = r.shape
    outs = [np.empty_like(r) for _ in range(6)]
    fn = getattr(_load(), f"wkv7_oracle_bwd_{precision}")
    rc = fn(B, T, H, N, ckpt, *map(_ptr, (r, w, k, v, a, b, dy, dsa)), *map(_ptr, outs),
            DECAYS[decay], threads or default_threads())
    if rc != 0:
        raise RuntimeError(f"oracle backward failed with code {rc}")
    return tuple(outs)


def bwd_state(r, w, k, v, a, b, dy, dsa=None, s0=None, dsT=None, precision: str = "f64",
              ckpt: int = 64, threads: int | None = None, decay: str = "clampw"):
    """``bwd`` for a sequence carried across calls: the forward started from
    ``s0`` ([B,H,N,N], None = zero) and ``dsT`` is the gradient of its final
    state (None = zero).  Returns (dr, dw, dk, dv, da, db, ds0), ds0 the
    gradient of the start state."""
    r, w, k, v, a, b, dy = (_f32(x) for x in (r, w, k, v, a, b, dy))
    B, T, H, N = r.shape
    dsa = None if dsa is None else _f32(dsa)
    s0 = None if s0 is None else _f32(s0).reshape(B, H, N, N)
    dsT = None if dsT is None else _f32(dsT).reshape(B, H, N, N)
    outs = [np.empty_like(r) for _ in range(6)]
    ds0 = np.empty((B, H, N, N), dtype=np.float32)
    fn = getattr(_load(), f"wkv7_oracle_bwd_state_{precision}")
    rc = fn(B, T, H, N, ckpt, *map(_ptr, (r, w, k, v, a, b, dy, dsa, s0, dsT, ds0)),
            *map(_ptr, outs), DECAYS[decay], threads or default_threads())
    if rc != 0:
        raise RuntimeError(f"oracle backward failed with code {rc}")
    return tuple(outs) + (ds0,)


def decay(w_in: float) -> float:
    return _load().wkv7_oracle_decay(float(w_in))


def torch_reference(r, w, k, v, a, b, dy=None, dsa=None, s0=None, decay: str = "clampw",
                    dsT=None):
    """Float64 torch restatement of camoe/backbone.py:264-294 returning (y, sa);
    with dy given, also the six input gradients from autograd (sa-gradient dsa
    optional).  ``s0`` ([B,H,N,N], default zero) is the start state.  Small
    sizes only: it loops over time in Python."""
    import torch

    xs = [torch.as_tensor(np.asarray(_f32(x)), dtype=torch.float64).requires_grad_(dy is not None)
          for x in (r, w, k, v, a, b)]
    rr, ww, kk, vv, aa, bb = xs
    B, T, H, N = rr.shape
    dec = torch.exp(-torch.exp(ww)) if decay == "wind" else torch.exp(W_SCALE / (1.0 + torch.exp(-ww)))
    S0 = None if s0 is None else torch.as_tensor(_f32(s0), dtype=torch.float64).reshape(
        B, H, N, N).requires_grad_(dy is not None)
    S = torch.zeros(B, H, N, N, dtype=torch.float64) if S0 is None else S0
    ys, sas = [], []
    for t in range(T):
        sa = (S * aa[:, t].unsqueeze(-2)).sum(-1)
        S = S * dec[:, t].unsqueeze(-2) + sa.unsqueeze(-1) * bb[:, t].unsqueeze(-2) \
            + vv[:, t].unsqueeze(-1) * kk[:, t].unsqueeze(-2)
        ys.append((S * rr[:, t].unsqueeze(-2)).sum(-1))
        sas.append(sa)
    y = torch.stack(ys, 1)
    sa = torch.stack(sas, 1)
    if dy is None:
        return y.detach().numpy(), sa.detach().numpy()
    loss = (y * torch.as_tensor(_f32(dy), dtype=torch.float64)).sum()
    if dsa is not None:
        loss = loss + (sa * torch.as_tensor(_f32(dsa), dtype=torch.float64)).sum()
    if dsT is not None:
        loss = loss + (S * torch.as_tensor(_f32(dsT), dtype=torch.float64).reshape(B, H, N, N)).sum()
    grads = torch.autograd.grad(loss, xs + ([S0] if S0 is not None else []))
    return (y.detach().numpy(), sa.detach().numpy()) + tuple(g.numpy() for g in grads)


class RefOp:
    """The reference's ClampW CUDA op, or with ``decay="wind"`` its
    wind_backstepping op (built from its sources into oracle/_ref/), called with
    device pointers.  Arguments are in the ClampW order (r, w, k, v, a, b) for
    both; the wind op's own order (w, q, k, v, z, a) is applied here.  It
    launches on the legacy default stream and validates nothing, so callers
    synchronise and pass T % 16 == 0."""

    _NAMES = {("clampw", False): "librwkv7_clampw_ref_bf16.so",
              ("clampw", True): "librwkv7_clampw_ref_fp32.so",
              ("wind", False): "libwind_ref_bf16.so", ("wind", True): "libwind_ref_fp32.so"}

    def __init__(self, fp32: bool = False, decay: str = "clampw"):
        path = os.path.join(_REF_DIR, self._NAMES[(decay, fp32)])
        if not os.path.exists(path):
            raise FileNotFoundError(f"{path} not built (make -C oracle ref)")
        self.wind = decay == "wind"
        self.lib = ctypes.CDLL(path)
        ci, fp = ctypes.c_int, ctypes.c_void_p
        pre = "ref_wind" if self.wind else "ref_clampw"
        self._fwd = getattr(self.lib, pre + "_fwd")
        self._bwd = getattr(self.lib, pre + "_bwd")
        self._fwd.argtypes = [ci] * 3 + [fp] * 9
        self._fwd.restype = ci
        self._bwd.argtypes = [ci] * 3 + [fp] * 15
        self._bwd.restype = ci

    @staticmethod
    def available(fp32: bool = False, decay: str = "clampw") -> bool:
        return os.path.exists(os.path.join(_REF_DIR, RefOp._NAMES[(decay, fp32)]))

    def forward(self, r, w, k, v, a, b, y, s, sa):
        B, T, H, _ = r.shape
        ins = (w, r, k, v, a, b) if self.wind else (r, w, k, v, a, b)
        rc = self._fwd(B, T, H, *[x.data_ptr() for x in ins + (y, s, sa)])
        if rc != 0:
            raise RuntimeError(f"reference forward failed: cuda error {rc}")

    def backward(self, r, w, k, v, a, b, dy, s, sa, dr, dw, dk, dv, da, db):
        B, T, H, _ = r.shape
        if self.wind:
            ptrs = (w, r, k, v, a, b, dy, s, sa, dw, dr, dk, dv, da, db)
        else:
            ptrs = (r, w, k, v, a, b, dy, s, sa, dr, dw, dk, dv, da, db)
        rc = self._bwd(B, T, H, *[x.data_ptr() for x in ptrs])
        if rc != 0:
            raise RuntimeError(f"reference backward failed: cuda error {rc}")
