"""Time-segmented WKV-7 ClampW for a few long sequences.

The sequential value passes of the chunked op give each (b, h) chain one
group of CTAs that walks its chunks in order.  With few chains per GPU (the
long-context problem B=2 T=65536 H=32 split over 8 GPUs leaves 2 sequences x
4 heads = 8 chains per GPU) most SMs idle while each chain walks its 4096
chunks.  Here every chain is cut into P segments of T/P steps that run as
independent chains -- the [B, T, H, 64] tensors viewed as [B*P, T/P, H, 64],
no copy -- joined through their states.  The state map of a segment is
affine, S_end = S_start A + C, so

1. every segment's transition A (its final state from an identity start with
   v = 0) and its final state C from a zero start come from two forwards over
   all segments at once (on the chunked path the key-side pass, which does not
   depend on v or the start state, runs once for these and step 3:
   ``camoe_wkv7_fwd_value``);
2. the start states S_g = S_{g-1} A_{g-1} + C_{g-1}, S_0 = s0, come from one
   launch that chains the P - 1 products per chain (``camoe_wkv7_seg_chain``);
3. the training forward of every segment starts from its S_g
   (``camoe_wkv7_fwd_carry``).

The backward mirrors it: every segment's start-state gradient D_g with no
gradient at its end (``camoe_wkv7_bwd_carry``), the end gradients
E_{g-1} = E_g A_g^T + D_g with E_{P-1} = ds_out (the same chain launch, run
backwards), then the backward of every segment with E_g at its end.  That is
three forward passes and one and a half backward passes over the sequence (the
first backward runs only the value pass), at P times the parallelism: it pays
when B * h_count * P CTA groups fill the GPU where B * h_count do not.

The reference runs every chain from t = 0 to T in one pass
(camoe/cuda/rwkv7_clampw.cu:36 forward, :93 backward); the results are the
same recurrence up to rounding (the transitions are formed through the same
chunked kernels).
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from . import _lib, ops
from ._lib import check
from .ops import HEAD_SIZE, _check_inputs, _check_state, _stream_ptr

NAMES = "rwkvab"


@dataclass
class Saved:
    """What the backward needs from a segmented forward."""
    xs: tuple             # r, w, k, v, a, b viewed as [B*P, T/P, H, 64]
    shape: tuple          # (B, T, H, 64)
    segments: int
    h0: int
    h_count: int
    starts: torch.Tensor  # [B*P, H, 64, 64] fp32: the start state of every segment
    trans: torch.Tensor   # [B*P, H, 64, 64] fp32: every segment's transition A
    ckpt: torch.Tensor
    algo: str


def auto_segments(chains: int, T: int, sms: int, min_len: int = 2048) -> int:
    """Segments per chain: the largest power of two P with 2 * chains * P <=
    sms (up to sms / 2 chain segments the value passes run two CTAs per
    segment, one per SM, so every segment still gets its SMs) and segments of
    at least ``min_len`` steps; 1 when that P is below 4.  The segmented step
    walks 3/P of the chain's chunks in value forwards and 2/P in value
    backwards, at two CTAs per segment, against all of them once each at up
    to four CTAs per chain in one pass; per chunk on B200 that is
    (3 x 0.41 + 2 x 0.52) / P us against 0.34 + 0.43 us, a gain only from
    P > 2.9.  B200 (148 SMs), the long-context share of 8 chains at
    T=65536: P = 8, measured fastest of 4, 8 and 16."""
    P = 1
    while 2 * chains * 2 * P <= sms and T % (16 * 2 * P) == 0 and T // (2 * P) >= min_len:
        P *= 2
    return P if P >= 4 else 1


def _view(x: torch.Tensor, P: int) -> torch.Tensor:
    B, T, H, N = x.shape
    return x.view(B * P, T // P, H, N)


def _states(BP: int, H: int, device) -> torch.Tensor:
    return torch.zeros(BP, H, HEAD_SIZE, HEAD_SIZE, dtype=torch.float32, device=device)


class Buffers:
    """Device buffers of a segmented forward + backward, allocated and filled
    once so that a step launches only the op's kernels and the two chain
    kernels: no allocation and no fill or copy kernels (unless a start state,
    a final-state gradient, ``s_out`` or ``ds0`` is passed, which are copied).
    Every step overwrites them, so one Buffers serves one forward/backward pair
    at a time, in stream order.

    Holds, for B sequences of T steps cut into P segments (heads [h0, h0 +
    h_count) of H): the segments' start states (row 0 kept at zero), their
    transitions and zero-start final states, the identity start of the
    transition pass, v = 0 over the head range, the end-state gradients (the
    last kept at zero), and the checkpoint and backward workspace."""

    def __init__(self, B: int, T: int, H: int, P: int, *, h0: int = 0,
                 h_count: int | None = None, device=None, dtype=torch.bfloat16, algo="auto"):
        hc = H - h0 if h_count is None else h_count
        N = HEAD_SIZE
        BP, Ts = B * P, T // P
        self.key = (B, T, H, P, h0, hc, dtype, algo)
        self.starts, self.trans, self.local = (_states(BP, H, device) for _ in range(3))
        self.ends = _states(BP, H, device)
        self.eye = _states(BP, H, device)
        self.eye[:, h0:h0 + hc] = torch.eye(N, device=device)
        self.vz = torch.zeros(BP, Ts, H, N, dtype=dtype, device=device)
        self.ckpt = torch.empty(max(ops.ckpt_bytes(BP, Ts, hc, dtype, algo), 16),
                                dtype=torch.uint8, device=device)
        self.work = torch.empty(max(ops.work_bytes(BP, Ts, hc, dtype, algo), 16),
                                dtype=torch.uint8, device=device)
        self.starts_dirty = False  # row 0 of starts holds a start state, not zero
        self.ends_dirty = False    # the last row of ends holds a gradient, not zero

    def check(self, B, T, H, P, h0, hc, dtype, algo):
        if (B, T, H, P, h0, hc, dtype, algo) != self.key:
            raise ValueError(f"Buffers made for {self.key}, called with "
                             f"{(B, T, H, P, h0, hc, dtype, algo)}")


def seg_chain(states, trans, local, B: int, P: int, h0: int, h_count: int, backward: bool):
    """camoe_wkv7_seg_chain on [B*P, H, 64, 64] fp32 tensors (see the header)."""
    for t, n in ((states, "states"), (trans, "trans"), (local, "local")):
        if t.dtype != torch.float32 or not t.is_contiguous() or t.dim() != 4 \
                or t.shape[0] != B * P or t.shape[2:] != (HEAD_SIZE, HEAD_SIZE):
            raise ValueError(f"{n} must be a contiguous float32 [B*P, H, 64, 64] tensor, "
                             f"got {tuple(t.shape)} {t.dtype}")
    H = states.shape[1]
    check(_lib.lib().camoe_wkv7_seg_chain(states.data_ptr(), trans.data_ptr(), local.data_ptr(),
                                          B, P, H, h0, h_count, int(backward),
                                          _stream_ptr(states.device)))


def wkv7_forward_segmented(r, w, k, v, a, b, segments: int, *, h0: int = 0,
                           h_count: int | None = None, s0=None, s_out=None, y=None, sa=None,
                           algo="auto", bufs: Buffers | None = None):
    """Training forward with every chain cut into ``segments`` pieces of equal
    length (T a multiple of 16 x segments).  ``s0`` ([B, H, 64, 64] fp32, None
    = zero) is the state the sequences start from and ``s_out`` receives their
    final states.  Heads [h0, h0 + h_count) are processed, in place.  ``bufs``
    (a ``Buffers`` of the same geometry) replaces every per-call allocation and
    fill.  Returns (y, sa, saved); ``saved`` feeds ``wkv7_backward_segmented``."""
    _check_inputs((r, w, k, v, a, b), NAMES)
    B, T, H, N = r.shape
    P = int(segments)
    if P < 1 or T % (16 * P) != 0:
        raise ValueError(f"T={T} must be a multiple of 16 x segments (segments={segments})")
    hc = H - h0 if h_count is None else h_count
    if h0 < 0 or hc < 0 or h0 + hc > H:
        raise ValueError(f"head range [{h0}, {h0 + hc}) outside H={H}")
    dev = r.device
    for s, n in ((s0, "s0"), (s_out, "s_out")):
        if s is not None:
            _check_state(s, B, H, dev, n)
    hs = slice(h0, h0 + hc)
    if y is None:
        y = torch.empty_like(r)
    if sa is None:
        sa = torch.empty(r.shape, dtype=torch.float32, device=dev)
    xs = tuple(_view(x, P) for x in (r, w, k, v, a, b))
    yv, sav = _view(y, P), _view(sa, P)
    BP = B * P
    if bufs is not None:
        bufs.check(B, T, H, P, h0, hc, r.dtype, algo)
        starts, trans = bufs.starts, bufs.trans
    else:
        starts, trans = _states(BP, H, dev), _states(BP, H, dev)
    sv = starts.view(B, P, H, N, N)
    if s0 is not None:
        sv[:, 0, hs] = s0[:, hs]
        if bufs is not None:
            bufs.starts_dirty = True
    elif bufs is not None and bufs.starts_dirty:
        sv[:, 0, hs] = 0.0
        bufs.starts_dirty = False
    fin = _states(BP, H, dev) if s_out is not None else None
    # the chunked path runs the key-side pass once, into the checkpoint, and
    # the value pass three times over it
    chunked = r.dtype == torch.bfloat16 and algo in ("auto", "chunked")
    ckpt = None if bufs is None else bufs.ckpt
    if P > 1:
        # 1. transitions (identity start, v = 0) and zero-start final states
        if bufs is not None:
            local, eye, vzv = bufs.local, bufs.eye, bufs.vz
        else:
            local = _states(BP, H, dev)
            eye = _states(BP, H, dev)
            eye[:, hs] = torch.eye(N, device=dev)
            vz = torch.empty_like(v)
            vz[:, :, hs].zero_()
            vzv = _view(vz, P)
        xz = (xs[0], xs[1], xs[2], vzv, xs[4], xs[5])
        if chunked:
            _, _, ckpt = ops.wkv7_forward(*xz, algo=algo, h0=h0, h_count=hc, y=yv, sa=sav, s0=eye,
                                          s_out=trans, ckpt=ckpt)
            ops.wkv7_forward_value(*xs, ckpt, h0=h0, h_count=hc, y=yv, sa=sav, s_out=local)
        else:
            ops.wkv7_forward_state(*xz, eye, algo=algo, h0=h0, h_count=hc, y=yv, sa=sav,
                                   out_state=trans)
            ops.wkv7_forward_state(*xs, None, algo=algo, h0=h0, h_count=hc, y=yv, sa=sav,
                                   out_state=local)
        # 2. the start state of every segment
        seg_chain(starts, trans, local, B, P, h0, hc, backward=False)
    # 3. the training forward of every segment from its start state
    if chunked and P > 1:
        ops.wkv7_forward_value(*xs, ckpt, h0=h0, h_count=hc, y=yv, sa=sav, s0=starts, s_out=fin)
    else:
        _, _, ckpt = ops.wkv7_forward(*xs, algo=algo, h0=h0, h_count=hc, y=yv, sa=sav,
                                      s0=starts, s_out=fin, ckpt=ckpt)
    if s_out is not None:
        s_out[:, hs] = fin.view(B, P, H, N, N)[:, P - 1, hs]
    saved = Saved(xs, (B, T, H, N), P, h0, hc, starts, trans, ckpt, algo)
    return y, sa, saved


def wkv7_backward_segmented(saved: Saved, dy, dsa=None, *, ds_out=None, ds0=None, grads=None,
                            bufs: Buffers | None = None):
    """Backward of ``wkv7_forward_segmented``.  ``dsa`` (fp32) may be None;
    ``ds_out`` is the gradient of the final states (None = zero) and ``ds0``
    ([B, H, 64, 64] fp32) receives the gradient of the start states.  ``bufs``
    as in the forward.  Returns (dr, dw, dk, dv, da, db)."""
    B, T, H, N = saved.shape
    P, h0, hc = saved.segments, saved.h0, saved.h_count
    hs = slice(h0, h0 + hc)
    ref = saved.xs[0]
    dev = ref.device
    if tuple(dy.shape) != (B, T, H, N) or not dy.is_contiguous() or dy.dtype != ref.dtype:
        raise ValueError("dy must be a contiguous tensor shaped and typed like the inputs")
    if dsa is not None and (tuple(dsa.shape) != (B, T, H, N) or dsa.dtype != torch.float32
                            or not dsa.is_contiguous()):
        raise ValueError("dsa must be a contiguous float32 tensor shaped like the inputs")
    for s, n in ((ds_out, "ds_out"), (ds0, "ds0")):
        if s is not None:
            _check_state(s, B, H, dev, n)
    if grads is None:
        grads = tuple(torch.empty(B, T, H, N, dtype=ref.dtype, device=dev) for _ in range(6))
    gv = tuple(_view(g, P) for g in grads)
    dyv = _view(dy, P)
    dsav = None if dsa is None else _view(dsa, P)
    BP, Ts = B * P, T // P
    if bufs is not None:
        bufs.check(B, T, H, P, h0, hc, ref.dtype, saved.algo)
        work, ends = bufs.work, bufs.ends
    else:
        wneed = ops.work_bytes(BP, Ts, hc, ref.dtype, saved.algo)
        work = torch.empty(max(wneed, 16), dtype=torch.uint8, device=dev) if wneed > 0 else None
        ends = _states(BP, H, dev)
    if ds_out is not None:
        ends.view(B, P, H, N, N)[:, P - 1, hs] = ds_out[:, hs]
        if bufs is not None:
            bufs.ends_dirty = True
    elif bufs is not None and bufs.ends_dirty:
        ends.view(B, P, H, N, N)[:, P - 1, hs] = 0.0
        bufs.ends_dirty = False
    kw = dict(algo=saved.algo, h0=h0, h_count=hc, grads=gv, work=work, s0=saved.starts)
    if P > 1:
        # start-state gradients with no gradient at the segment ends (the value
        # pass alone on the chunked path), then the end gradients
        local = bufs.local if bufs is not None else _states(BP, H, dev)
        chunked = ref.dtype == torch.bfloat16 and saved.algo in ("auto", "chunked")
        ops.wkv7_backward(*saved.xs, dyv, dsav, saved.ckpt, ds0=local, ds0_only=chunked, **kw)
        seg_chain(ends, saved.trans, local, B, P, h0, hc, backward=True)
    first = _states(BP, H, dev) if ds0 is not None else None
    ops.wkv7_backward(*saved.xs, dyv, dsav, saved.ckpt, ds_out=ends, ds0=first, **kw)
    if ds0 is not None:
        ds0[:, hs] = first.view(B, P, H, N, N)[:, 0, hs]
    return grads


class SegmentedClampW(torch.autograd.Function):
    """y, sa = SegmentedClampW.apply(r, w, k, v, a, b, segments): the
    ``RWKV7_ClampW`` Function with every chain cut into ``segments`` pieces
    (same inputs, outputs and gradients, up to rounding)."""

    @staticmethod
    def forward(ctx, r, w, k, v, a, b, segments):
        y, sa, saved = wkv7_forward_segmented(r, w, k, v, a, b, segments)
        ctx.set_materialize_grads(False)
        ctx.saved = saved
        return y, sa

    @staticmethod
    def backward(ctx, dy, dsa):
        saved = ctx.saved
        ref = saved.xs[0]
        dy = torch.zeros(saved.shape, dtype=ref.dtype, device=ref.device) if dy is None \
            else dy.to(ref.dtype).contiguous()
        if dsa is not None:
            dsa = dsa.to(torch.float32).contiguous()
        grads = wkv7_backward_segmented(saved, dy, dsa)
        return tuple(grads) + (None,)
