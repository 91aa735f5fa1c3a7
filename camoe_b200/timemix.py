"""RWKV-7 time mix with the WKV-7 op and its elementwise neighbours fused.

``RWKV7TimeMix`` is a drop-in for the reference's ``RWKV7_TimeMix``
(camoe/backbone.py:134-373): same constructor arguments, the same parameter
names and shapes (a state_dict loads either way), the same
``forward(x, v_first=None) -> (out, v_first, state_representation)``.

What runs:

* projections (receptance, key, value, output) and the LoRA products: bf16
  GEMMs (cuBLAS through torch), weights cast from the fp32 parameters per
  call as autocast does, their gradients written by the GEMMs in fp32
  (``MatmulBf16Fn``); the two LoRA hidden activations (tanh for the decay,
  sigmoid for the gate, on [B, T, D] with D <= 160) are torch ops;
* everything else is four fused CUDA kernels (include/camoe_timemix.h), each
  one pass over HBM, and the WKV-7 op itself:
  ``mix`` (token shift and six mixes, backbone.py:316-323) before the GEMMs,
  ``prep`` (decay, value residual, in-context rate, key normalisation and the
  op's a/b, :326-343) between the GEMMs and the op, ``lnsa`` (the LayerNorm of
  sa, :348) and ``post`` (GroupNorm, bonus and gate, :359-367) after it.
  ``prep -> op -> lnsa/post`` is one autograd Function, so the op's gradients
  and the epilogue's gradients of r, k', v' are added inside the prep backward
  kernel instead of in separate passes.

Numerics: fp32 arithmetic in every kernel, bf16 activations (the reference
under bf16 autocast rounds the same tensors except sa before ``ln_sa``, which
here is normalised in fp32) and fp32 parameters.  The reference's debugging
switches (CAMOE_NAN_DEBUG, CAMOE_SANITIZE_TIMEMIX_OUT) and its torch fallback
path are not reproduced.
"""
from __future__ import annotations

import ctypes
import math

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import _lib, ops
from ._lib import check

HEAD_SIZE = 64
_BF = torch.bfloat16


def lora_dims(C: int) -> dict:
    """LoRA ranks of the RWKV-7 time mix for width C (camoe/backbone.py:177-181)."""
    def r(f):
        return max(32, int(round((f * C ** 0.5) / 32) * 32))
    return {"decay": r(2.5), "aaa": r(2.5), "mv": r(1.7), "gate": r(5.0)}


def _p(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream(t):
    return torch.cuda.current_stream(t.device).cuda_stream


def _work(B, T, C, device):
    n = int(_lib.lib().camoe_tm_work_bytes(B, T, C))
    return torch.empty(max(n, 16), dtype=torch.uint8, device=device), n


def lora_work_bytes(R: int, C: int, D: int) -> int:
    """camoe_tm_lora_work_bytes(R, C, D) without the call: one fp32 [C, D] partial
    sum per slice of 64-row stages, at most 16 slices (lora_tc.cu)."""
    return min(16, max(1, -(-R // 64))) * C * D * 4


def _weight_grad(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """a^T b in fp32 for 2-D bf16 a [R, m], b [R, n]: the weight gradient of a
    product.  Where one side is a LoRA rank (a multiple of 32 from 64 to 256)
    and the other a multiple of 128, the tcgen05 kernel camoe_tm_lora_wgrad
    reduces over the R rows (include/camoe_timemix.h); the square projections
    stay with cuBLAS."""
    R, m = a.shape
    n = b.shape[1]
    if a.is_cuda and a.dtype == _BF and b.dtype == _BF and R > 0:
        rank = (lambda d: d % 32 == 0 and 64 <= d <= 256)
        big = None
        if m % 128 == 0 and rank(n):
            big, thin, C, D, out_cd = a, b, m, n, 1   # [m][n] = [C][D]
        elif n % 128 == 0 and rank(m):
            big, thin, C, D, out_cd = b, a, n, m, 0   # [m][n] = [D][C]
        if big is not None:
            big, thin = big.contiguous(), thin.contiguous()
            nw = lora_work_bytes(R, C, D)
            # one allocation (host time counts when the step is dispatched eagerly):
            # the partial sums, then the gradient
            buf = torch.empty(nw + 4 * m * n, dtype=torch.uint8, device=a.device)
            dw = buf[nw:].view(torch.float32).view(m, n)
            check(_lib.lib().camoe_tm_lora_wgrad(big.data_ptr(), thin.data_ptr(), dw.data_ptr(),
                                                 out_cd, buf.data_ptr(), nw, R, C, D,
                                                 torch.cuda.current_stream(a.device).cuda_stream))
            return dw
    return torch.mm(a.t(), b, out_dtype=torch.float32)


class MatmulBf16Fn(torch.autograd.Function):
    """x @ w (or x @ w^T for ``F.linear``'s layout) with the fp32 parameter w
    cast to bf16 per call, as autocast casts it for the reference's
    projections and LoRA products.  The backward writes w's gradient in fp32
    directly (``_weight_grad``: the LoRA ranks' tcgen05 kernel, else a cuBLAS
    GEMM with fp32 output), where autocast's path writes it in bf16 and
    converts it with one more kernel per weight; the input's gradient stays
    bf16."""

    @staticmethod
    def forward(ctx, x, w, transposed: bool):
        wb = w.to(_BF)
        ctx.transposed = transposed
        ctx.save_for_backward(x, wb)
        return x @ (wb.t() if transposed else wb)

    @staticmethod
    def backward(ctx, dy):
        x, wb = ctx.saved_tensors
        dx = dw = None
        if ctx.needs_input_grad[0]:
            dx = dy @ (wb if ctx.transposed else wb.t())
        if ctx.needs_input_grad[1]:
            x2, dy2 = x.reshape(-1, x.shape[-1]), dy.reshape(-1, dy.shape[-1])
            dw = _weight_grad(dy2, x2) if ctx.transposed else _weight_grad(x2, dy2)
        return dx, dw, None


class Mix6Fn(torch.autograd.Function):
    """(xr, xw, xk, xv, xa, xg) = x + (shift(x) - x) * mix[m] (bf16 outputs)."""

    @staticmethod
    def forward(ctx, x, mix):
        B, T, C = x.shape
        x = x.contiguous()
        mix = mix.float().contiguous()
        outs = [torch.empty(B, T, C, dtype=_BF, device=x.device) for _ in range(6)]
        ptrs = (ctypes.c_void_p * 6)(*[o.data_ptr() for o in outs])
        code = {_BF: 0, torch.float32: 1}.get(x.dtype)
        if code is None:
            raise TypeError(f"time-mix input must be bfloat16 or float32, got {x.dtype}")
        check(_lib.lib().camoe_tm_mix_fwd(_p(x), code, _p(mix), ptrs, B, T, C, _stream(x)))
        ctx.save_for_backward(x, mix)
        ctx.code = code
        return tuple(outs)

    @staticmethod
    def backward(ctx, *douts):
        x, mix = ctx.saved_tensors
        B, T, C = x.shape
        ds = [torch.zeros(B, T, C, dtype=_BF, device=x.device) if d is None
              else d.to(_BF).contiguous() for d in douts]
        ptrs = (ctypes.c_void_p * 6)(*[d.data_ptr() for d in ds])
        dx = torch.empty_like(x)
        dmix = torch.empty(6, C, dtype=torch.float32, device=x.device)
        work, nw = _work(B, T, C, x.device)
        check(_lib.lib().camoe_tm_mix_bwd(_p(x), ctx.code, _p(mix), ptrs, _p(dx), _p(dmix),
                                          _p(work), nw, B, T, C, _stream(x)))
        return dx, dmix


class Wkv7BlockFn(torch.autograd.Function):
    """prep -> WKV-7 op -> (post, lnsa) between the projection GEMMs and the
    output GEMM.  Inputs are [B, T, C] bf16 activations (vl and v_first None
    for layer 0) and fp32 parameters; returns (z, state_representation)."""

    @staticmethod
    def forward(ctx, r, wl, k, v, vl, al, v_first, g, prep_par, r_k, lnx_w, lnx_b, lnsa_w,
                lnsa_b, algo):
        B, T, C = r.shape
        H = C // HEAD_SIZE
        acts = [t.contiguous() if t is not None else None for t in (r, wl, k, v, vl, al, v_first, g)]
        r, wl, k, v, vl, al, v_first, g = acts
        L = _lib.lib()
        dev = r.device
        op_in = [torch.empty(B, T, C, dtype=_BF, device=dev) for _ in range(5)]
        w_op, k_op, v_op, a_op, b_op = op_in
        check(L.camoe_tm_prep_fwd(_p(wl), _p(k), _p(v), _p(vl), _p(al), _p(v_first),
                                  _p(prep_par), *[_p(t) for t in op_in], B, T, C, _stream(r)))
        as4 = (lambda t: t.view(B, T, H, HEAD_SIZE))
        needs_ckpt = any(ctx.needs_input_grad)
        y, sa, ckpt = ops.wkv7_forward(as4(r), as4(w_op), as4(k_op), as4(v_op), as4(a_op),
                                       as4(b_op), algo=algo, save_ckpt=needs_ckpt)
        y = y.view(B, T, C)
        sa = sa.view(B, T, C)
        srep = torch.empty(B, T, C, dtype=torch.float32, device=dev)
        check(L.camoe_tm_lnsa_fwd(_p(sa), _p(lnsa_w), _p(lnsa_b), _p(srep), B, T, C, _stream(r)))
        z = torch.empty(B, T, C, dtype=_BF, device=dev)
        check(L.camoe_tm_post_fwd(_p(y), _p(r), _p(k_op), _p(v_op), _p(g), _p(r_k), _p(lnx_w),
                                  _p(lnx_b), _p(z), B, T, C, _stream(r)))
        ctx.set_materialize_grads(False)
        ctx.algo = algo
        ctx.vres = vl is not None
        ctx.save_for_backward(r, wl, k, v, vl, al, v_first, g, prep_par, r_k, lnx_w, lnx_b,
                              lnsa_w, w_op, k_op, v_op, a_op, b_op, y, sa, ckpt)
        return z, srep

    @staticmethod
    def backward(ctx, dz, dsrep):
        (r, wl, k, v, vl, al, v_first, g, prep_par, r_k, lnx_w, lnx_b, lnsa_w, w_op, k_op, v_op,
         a_op, b_op, y, sa, ckpt) = ctx.saved_tensors
        B, T, C = r.shape
        H = C // HEAD_SIZE
        dev = r.device
        L = _lib.lib()
        st = _stream(r)
        work, nw = _work(B, T, C, dev)
        e = (lambda dt=_BF: torch.empty(B, T, C, dtype=dt, device=dev))
        dz = torch.zeros(B, T, C, dtype=_BF, device=dev) if dz is None else dz.to(_BF).contiguous()
        dy, dr_epi, dk_epi, dv_epi, dg = e(), e(), e(), e(), e()
        dpost = torch.empty(3, C, dtype=torch.float32, device=dev)
        check(L.camoe_tm_post_bwd(_p(dz), _p(y), _p(r), _p(k_op), _p(v_op), _p(g), _p(r_k),
                                  _p(lnx_w), _p(lnx_b), _p(dy), _p(dr_epi), _p(dk_epi),
                                  _p(dv_epi), _p(dg), _p(dpost), _p(work), nw, B, T, C, st))
        dsa = None
        dlnsa = torch.zeros(2, C, dtype=torch.float32, device=dev)
        if dsrep is not None:
            dsrep = dsrep.float().contiguous()
            dsa = e(torch.float32)
            check(L.camoe_tm_lnsa_bwd(_p(dsrep), _p(sa), _p(lnsa_w), _p(dsa), _p(dlnsa),
                                      _p(work), nw, B, T, C, st))
        as4 = (lambda t: t.view(B, T, H, HEAD_SIZE))
        g_op = ops.wkv7_backward(as4(r), as4(w_op), as4(k_op), as4(v_op), as4(a_op), as4(b_op),
                                 as4(dy), None if dsa is None else as4(dsa), ckpt, algo=ctx.algo)
        dr_op, dw_op, dk_op, dv_op, da_op, db_op = (t.view(B, T, C) for t in g_op)
        dr, dwl, dk, dv, dal = e(), e(), e(), e(), e()
        dvl = e() if ctx.vres else None
        dvf = e() if ctx.vres else None
        dprep = torch.empty(5, C, dtype=torch.float32, device=dev)
        check(L.camoe_tm_prep_bwd(_p(dr_op), _p(dr_epi), _p(dw_op), _p(dk_op), _p(dk_epi),
                                  _p(dv_op), _p(dv_epi), _p(da_op), _p(db_op), None, _p(wl),
                                  _p(k), _p(v), _p(vl), _p(al), _p(v_first), _p(prep_par),
                                  _p(dr), _p(dwl), _p(dk), _p(dv), _p(dvl), _p(dal), _p(dvf),
                                  _p(dprep), _p(work), nw, B, T, C, st))
        return (dr, dwl, dk, dv, dvl, dal, dvf, dg, dprep, dpost[2].view(H, HEAD_SIZE),
                dpost[0], dpost[1], dlnsa[0], dlnsa[1], None)


def _ortho(shape, scale):
    x = torch.empty(*shape)
    gain = math.sqrt(shape[0] / shape[1]) if shape[0] > shape[1] else 1.0
    nn.init.orthogonal_(x, gain=gain * scale)
    return x


class RWKV7TimeMix(nn.Module):
    """Fused RWKV-7 time mix.  ``algo`` picks the WKV-7 algorithm ("auto":
    chunked tensor-core path for bf16)."""

    def __init__(self, n_embd: int, n_layer: int, layer_id: int, head_size: int = 64,
                 algo: str = "auto"):
        super().__init__()
        if head_size != HEAD_SIZE or n_embd % HEAD_SIZE != 0:
            raise ValueError(f"head size must be {HEAD_SIZE} and divide n_embd")
        C, H, N = n_embd, n_embd // head_size, head_size
        self.layer_id, self.n_layer, self.head_size, self.n_head, self.n_embd = (
            layer_id, n_layer, head_size, H, n_embd)
        self.algo = algo
        self.ln_sa = nn.LayerNorm(C)
        d = lora_dims(C)
        # the RWKV-7 initialisation the reference uses (camoe/backbone.py:154-224)
        with torch.no_grad():
            r01 = layer_id / max(n_layer - 1, 1)
            r10 = 1.0 - layer_id / n_layer
            ddd = (torch.arange(C, dtype=torch.float32) / C).view(1, 1, C)
            for name, p in (("x_r", 0.2), ("x_w", 0.9), ("x_k", 0.7), ("x_v", 0.7), ("x_a", 0.9),
                            ("x_g", 0.2)):
                setattr(self, name, nn.Parameter(1.0 - torch.pow(ddd, p * r10)))
            n = torch.arange(C, dtype=torch.float32)
            linear = n / (C - 1) - 0.5
            zz = ((n % N) - (N - 1) / 2) / ((N - 1) / 2)
            zigzag = zz * zz.abs()
            www = -6 + 6 * (n / (C - 1)) ** (1 + r01 ** 0.3)
            self.w0 = nn.Parameter((www + 0.5 + zigzag * 2.5).view(1, 1, C))
            self.w1 = nn.Parameter(torch.zeros(C, d["decay"]))
            self.w2 = nn.Parameter(_ortho((d["decay"], C), 0.1))
            self.a0 = nn.Parameter((-0.19 + zigzag * 0.3 + linear * 0.4).view(1, 1, C))
            self.a1 = nn.Parameter(torch.zeros(C, d["aaa"]))
            self.a2 = nn.Parameter(_ortho((d["aaa"], C), 0.1))
            self.v0 = nn.Parameter((0.73 - linear * 0.4).view(1, 1, C))
            self.v1 = nn.Parameter(torch.zeros(C, d["mv"]))
            self.v2 = nn.Parameter(_ortho((d["mv"], C), 0.1))
            self.g1 = nn.Parameter(torch.zeros(C, d["gate"]))
            self.g2 = nn.Parameter(_ortho((d["gate"], C), 0.1))
            self.k_k = nn.Parameter((0.71 - linear * 0.1).view(1, 1, C))
            self.k_a = nn.Parameter(torch.full((1, 1, C), 1.02))
            self.r_k = nn.Parameter(torch.full((H, N), -0.04))
        self.receptance = nn.Linear(C, C, bias=False)
        self.key = nn.Linear(C, C, bias=False)
        self.value = nn.Linear(C, C, bias=False)
        self.output = nn.Linear(C, C, bias=False)
        self.ln_x = nn.GroupNorm(H, C, eps=64e-5)
        with torch.no_grad():
            s = C ** -0.5
            self.receptance.weight.uniform_(-0.5 * s, 0.5 * s)
            self.key.weight.uniform_(-0.05 * s, 0.05 * s)
            self.value.weight.uniform_(-0.5 * s, 0.5 * s)
            self.output.weight.zero_()

    def forward(self, x: torch.Tensor, v_first: torch.Tensor | None = None):
        B, T, C = x.shape
        mix = torch.cat([getattr(self, n).view(1, C) for n in
                         ("x_r", "x_w", "x_k", "x_v", "x_a", "x_g")])
        xr, xw, xk, xv, xa, xg = Mix6Fn.apply(x, mix)
        L = (lambda t, m: MatmulBf16Fn.apply(t, m.weight, True))  # F.linear(t, bf16(W))
        P = (lambda t, w: MatmulBf16Fn.apply(t, w, False))         # t @ bf16(w)
        r = L(xr, self.receptance)
        k = L(xk, self.key)
        v = L(xv, self.value)
        wl = P(torch.tanh(P(xw, self.w1)), self.w2)
        al = P(P(xa, self.a1), self.a2)
        g = P(torch.sigmoid(P(xg, self.g1)), self.g2)
        if self.layer_id == 0:
            vl = vf = None
        else:
            if v_first is None:
                raise ValueError("layers after the first need v_first")
            vl = P(P(xv, self.v1), self.v2)
            vf = v_first.to(_BF)
        prep_par = torch.cat([t.view(1, C) for t in (self.w0, self.v0, self.a0, self.k_k, self.k_a)])
        z, srep = Wkv7BlockFn.apply(r, wl, k, v, vl, al, vf, g, prep_par, self.r_k,
                                    self.ln_x.weight, self.ln_x.bias, self.ln_sa.weight,
                                    self.ln_sa.bias, self.algo)
        out = L(z, self.output)
        if self.layer_id == 0:
            v_first = v
        return out, v_first, srep

    @torch.no_grad()
    def forward_state(self, x: torch.Tensor, v_first: torch.Tensor | None = None, state=None):
        """Inference over steps [t0, t0 + T) of each sequence, carrying the
        layer's state across calls, so that generating a token costs one step
        instead of a pass over the whole context (the reference re-runs the
        prefix for every token, eval.py:212).  ``state`` is None at t0 = 0 or
        the (x_prev, wkv) returned by the previous call: x_prev [B, C] the last
        step of x (the token shift's input), wkv [B, H, 64, 64] fp32 the WKV
        state.  Returns (out, v_first, state_representation, new_state); the
        outputs equal ``forward`` over the concatenated steps.  ``v_first``
        (layers > 0) covers the same steps as x."""
        B, T, C = x.shape
        H = C // HEAD_SIZE
        dev = x.device
        L = _lib.lib()
        st = _stream(x)
        x = x.contiguous()
        code = {_BF: 0, torch.float32: 1}.get(x.dtype)
        if code is None:
            raise TypeError(f"time-mix input must be bfloat16 or float32, got {x.dtype}")
        x_prev, wkv = (None, None) if state is None else state
        if x_prev is not None:
            x_prev = x_prev.to(x.dtype).contiguous()
            if tuple(x_prev.shape) != (B, C):
                raise ValueError(f"state x_prev must be [B, C] = [{B}, {C}]")
        mix = torch.cat([getattr(self, n).view(1, C) for n in
                         ("x_r", "x_w", "x_k", "x_v", "x_a", "x_g")]).float().contiguous()
        xs = [torch.empty(B, T, C, dtype=_BF, device=dev) for _ in range(6)]
        ptrs = (ctypes.c_void_p * 6)(*[t.data_ptr() for t in xs])
        check(L.camoe_tm_mix_fwd_prev(_p(x), code, _p(x_prev), _p(mix), ptrs, B, T, C, st))
        xr, xw, xk, xv, xa, xg = xs
        W = (lambda m: m.weight.to(_BF))
        P = (lambda t: t.to(_BF))
        r = F.linear(xr, W(self.receptance)).contiguous()
        k = F.linear(xk, W(self.key)).contiguous()
        v = F.linear(xv, W(self.value)).contiguous()
        wl = (torch.tanh(xw @ P(self.w1)) @ P(self.w2)).contiguous()
        al = ((xa @ P(self.a1)) @ P(self.a2)).contiguous()
        g = (torch.sigmoid(xg @ P(self.g1)) @ P(self.g2)).contiguous()
        if self.layer_id == 0:
            vl = vf = None
        else:
            if v_first is None:
                raise ValueError("layers after the first need v_first")
            vl = ((xv @ P(self.v1)) @ P(self.v2)).contiguous()
            vf = v_first.to(_BF).contiguous()
        prep_par = torch.cat([t.view(1, C) for t in (self.w0, self.v0, self.a0, self.k_k,
                                                      self.k_a)]).float().contiguous()
        op_in = [torch.empty(B, T, C, dtype=_BF, device=dev) for _ in range(5)]
        check(L.camoe_tm_prep_fwd(_p(wl), _p(k), _p(v), _p(vl), _p(al), _p(vf), _p(prep_par),
                                  *[_p(t) for t in op_in], B, T, C, st))
        w_op, k_op, v_op, a_op, b_op = op_in
        as4 = (lambda t: t.view(B, T, H, HEAD_SIZE))
        y, sa, wkv_new = ops.wkv7_forward_state(as4(r), as4(w_op), as4(k_op), as4(v_op),
                                                as4(a_op), as4(b_op), wkv, algo=self.algo)
        y, sa = y.view(B, T, C), sa.view(B, T, C)
        # fp32 parameter copies held here until the launches are queued
        ln_w, ln_b, r_k, gx, bx = (t.float().contiguous() for t in (
            self.ln_sa.weight, self.ln_sa.bias, self.r_k, self.ln_x.weight, self.ln_x.bias))
        srep = torch.empty(B, T, C, dtype=torch.float32, device=dev)
        check(L.camoe_tm_lnsa_fwd(_p(sa), _p(ln_w), _p(ln_b), _p(srep), B, T, C, st))
        z = torch.empty(B, T, C, dtype=_BF, device=dev)
        check(L.camoe_tm_post_fwd(_p(y), _p(r), _p(k_op), _p(v_op), _p(g), _p(r_k), _p(gx),
                                  _p(bx), _p(z), B, T, C, st))
        out = F.linear(z, W(self.output))
        if self.layer_id == 0:
            v_first = v
        return out, v_first, srep, (x[:, -1].contiguous(), wkv_new)
