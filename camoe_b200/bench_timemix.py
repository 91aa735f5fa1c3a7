"""Timings of the fused RWKV-7 time mix (camoe_b200.timemix) on one GPU.

    python -m camoe_b200.bench_timemix [--batch 8 --seq 1024 --embd 1024 --layer 2]

Prints JSON lines:

* ``layer``: one time-mix layer, forward + backward (eagerly dispatched, and
  replayed from a CUDA graph to show the device time), through the fused module
  and through the same layer computed op by op as the reference's
  ``RWKV7_TimeMix.forward`` does (camoe/backbone.py:311-371, restated below as
  ``eager_forward``, the unfused baseline) under bf16 autocast, with this
  package's WKV-7 op behind ``RUN_CUDA_RWKV7`` in both, so the difference is
  the fusion of everything around the op.
* ``decode``: one generated token through one layer with the state carried
  (``RWKV7TimeMix.forward_state``), against re-running the layer over the
  whole context as the reference's generation loop does (B=64 sequences).
* ``kernel``: each fused kernel alone, CUDA-event time per launch (L2 flushed
  before each) against its algorithmic bytes (each input read once, each
  output written once) and the measured HBM bandwidth.

Seeded synthetic inputs and parameters; timing with CUDA events after warm-up.
"""
from __future__ import annotations

import argparse
import ctypes
import json

import torch
import torch.nn.functional as F

from . import _lib, backbone, timemix
from .bench_state import hbm_peak_gbs

BF = torch.bfloat16


def eager_forward(m, x, v_first):
    """The reference's time-mix forward, op for op (camoe/backbone.py:311-371),
    using the module's parameters; the unfused baseline."""
    B, T, C = x.shape
    H = m.n_head
    with torch.autocast("cuda", dtype=BF):
        xx = F.pad(x, (0, 0, 1, -1)) - x
        xr, xw, xk = x + xx * m.x_r, x + xx * m.x_w, x + xx * m.x_k
        xv, xa, xg = x + xx * m.x_v, x + xx * m.x_a, x + xx * m.x_g
        r = m.receptance(xr)
        w = -F.softplus(-(m.w0 + torch.tanh(xw @ m.w1) @ m.w2)) - 0.5
        k = m.key(xk)
        v = m.value(xv)
        if m.layer_id == 0:
            v_first = v.clone()
        else:
            v = v + (v_first - v) * torch.sigmoid(m.v0 + (xv @ m.v1) @ m.v2)
        a = torch.sigmoid(m.a0 + (xa @ m.a1) @ m.a2)
        g = torch.sigmoid(xg @ m.g1) @ m.g2
        kk = F.normalize((k * m.k_k).view(B, T, H, -1), dim=-1, p=2.0).view(B, T, C)
        k = k * (1 + (a - 1) * m.k_a)
        x_att, sa = backbone.RUN_CUDA_RWKV7(r, w, k, v, -kk, kk * a)
        srep = m.ln_sa(sa)
        x_att = m.ln_x(x_att.view(B * T, C)).view(B, T, C)
        x_att = x_att + ((r.view(B, T, H, -1) * k.view(B, T, H, -1) * m.r_k).sum(dim=-1, keepdim=True)
                         * v.view(B, T, H, -1)).view(B, T, C)
        out = m.output(x_att * g)
    return out, v_first, srep


def time_ms(fn, steps, warmup=3):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        fn()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / steps


def time_flushed_us(fn, steps, flush):
    """Mean CUDA-event time of single launches, each after writing a buffer
    larger than L2 (so inputs come from HBM)."""
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(steps)]
    for e0, e1 in ev:
        flush.zero_()
        flush.sum()  # read it back: L2 left holding clean lines, no write-back during fn
        e0.record()
        fn()
        e1.record()
    torch.cuda.synchronize()
    return sum(e0.elapsed_time(e1) for e0, e1 in ev) * 1e3 / steps


def time_graph_ms(fn, steps):
    """fn captured once in a CUDA graph (after warm-up on a side stream) and
    replayed: device time without Python dispatch."""
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for _ in range(3):
            fn()
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        fn()
    return time_ms(g.replay, steps)


def bench_layer(B, T, C, layer, steps):
    torch.manual_seed(0)
    m = timemix.RWKV7TimeMix(C, 12, layer).cuda()
    with torch.no_grad():  # non-zero LoRA inputs and output projection, as after training
        for n in ("w1", "a1", "v1", "g1"):
            getattr(m, n).normal_(0, 0.1)
        m.output.weight.normal_(0, C ** -0.5)
    x = torch.randn(B, T, C, device="cuda", dtype=BF).requires_grad_(True)
    vf = None if layer == 0 else (0.5 * torch.randn(B, T, C, device="cuda", dtype=BF)).requires_grad_(True)
    d_out = torch.randn(B, T, C, device="cuda", dtype=BF)
    d_srep = torch.randn(B, T, C, device="cuda")

    def step(fwd):
        out, _, srep = fwd(m, x, vf)
        torch.autograd.backward([out, srep], [d_out, d_srep.to(srep.dtype)])

    backbone.init_rwkv7_cuda()
    fused = time_ms(lambda: step(lambda mm, xx, vv: mm(xx, vv)), steps)
    eager = time_ms(lambda: step(eager_forward), steps)
    fused_g = time_graph_ms(lambda: step(lambda mm, xx, vv: mm(xx, vv)), steps)
    eager_g = time_graph_ms(lambda: step(eager_forward), steps)
    fwd_fused = time_ms(lambda: m(x.detach(), None if vf is None else vf.detach()), steps)
    with torch.no_grad():
        fwd_eager = time_ms(lambda: eager_forward(m, x, vf), steps)
    return {"workload": f"time mix layer {layer}: B={B} T={T} C={C} H={C // 64}, bf16, fwd+bwd",
            "metric": "timemix_layer_tokens_per_s",
            "fused": {"ms": round(fused, 3), "tokens_per_s": round(B * T / fused * 1e3),
                      "fwd_ms": round(fwd_fused, 3), "graph_ms": round(fused_g, 3)},
            "eager": {"ms": round(eager, 3), "tokens_per_s": round(B * T / eager * 1e3),
                      "fwd_ms": round(fwd_eager, 3), "graph_ms": round(eager_g, 3)},
            "speedup": round(eager / fused, 2), "speedup_graph": round(eager_g / fused_g, 2)}


def bench_decode(B, ctx, C, layer, steps):
    """Per generated token, one time-mix layer: forward_state on one step with
    the carried state (eager, and replayed from a CUDA graph), against what the
    reference's generation loop does per token, a forward over the whole
    context (eval.py:212)."""
    torch.manual_seed(0)
    m = timemix.RWKV7TimeMix(C, 12, layer).cuda()
    x = torch.randn(B, ctx, C, device="cuda", dtype=BF)
    vf = None if layer == 0 else torch.randn(B, ctx, C, device="cuda", dtype=BF)
    with torch.no_grad():
        _, _, _, state = m.forward_state(x, vf)
    x1 = x[:, -1:].contiguous()
    v1 = None if vf is None else vf[:, -1:].contiguous()
    holder = {"s": state}

    def token():
        o, _, _, holder["s"] = m.forward_state(x1, v1, holder["s"])

    step_ms = time_ms(token, steps)
    step_graph_ms = time_graph_ms(token, steps)
    with torch.no_grad():
        full_ms = time_ms(lambda: m(x, vf), max(3, steps // 10))
    return {"workload": f"time mix layer {layer} decode: B={B} context {ctx} C={C}, bf16, "
                        "one generated token",
            "metric": "decode_ms_per_token",
            "stateful": {"ms": round(step_ms, 4), "graph_ms": round(step_graph_ms, 4)},
            "rerun_context": {"ms": round(full_ms, 3)},
            "speedup_graph": round(full_ms / step_graph_ms, 1)}


def bench_kernels(B, T, C, steps):
    L = _lib.lib()
    n = B * T * C
    st = torch.cuda.current_stream().cuda_stream
    P = (lambda t: None if t is None else ctypes.c_void_p(t.data_ptr()))
    bf = (lambda: torch.randn(B, T, C, device="cuda", dtype=BF))
    f32 = (lambda: torch.randn(B, T, C, device="cuda"))
    vec = (lambda k: torch.rand(k, C, device="cuda"))
    nw = int(L.camoe_tm_work_bytes(B, T, C))
    work = torch.empty(nw, dtype=torch.uint8, device="cuda")
    peak, kind = hbm_peak_gbs()
    x, six, dsix = bf(), [bf() for _ in range(6)], [bf() for _ in range(6)]
    arr = (lambda ts: (ctypes.c_void_p * 6)(*[t.data_ptr() for t in ts]))
    ins = [bf() for _ in range(6)]           # wl, k, v, vl, al, v_first
    outs5 = [bf() for _ in range(5)]
    grads9 = [bf() for _ in range(9)]
    outs7 = [bf() for _ in range(7)]
    y, r, ko, vo, g, z, dz = (bf() for _ in range(7))
    sa, srep, dsrep, dsa = f32(), f32(), f32(), f32()
    dx = bf()
    par5, par6, par3, par2 = vec(5), vec(6), vec(3), vec(2)
    dpar = vec(6)  # parameter-gradient output (never an input)
    calls = {
        # name: (launch, algorithmic bytes per launch)
        "mix_fwd": (lambda: L.camoe_tm_mix_fwd(P(x), 0, P(par6), arr(six), B, T, C, st), 14 * n),
        "mix_bwd": (lambda: L.camoe_tm_mix_bwd(P(x), 0, P(par6), arr(dsix), P(dx), P(dpar), P(work),
                                               nw, B, T, C, st), 16 * n),
        "prep_fwd": (lambda: L.camoe_tm_prep_fwd(*[P(t) for t in ins], P(par5),
                                                 *[P(t) for t in outs5], B, T, C, st), 22 * n),
        "prep_bwd": (lambda: L.camoe_tm_prep_bwd(*[P(t) for t in grads9], None,
                                                 *[P(t) for t in ins], P(par5),
                                                 *[P(t) for t in outs7], P(dpar), P(work), nw,
                                                 B, T, C, st), 44 * n),
        "post_fwd": (lambda: L.camoe_tm_post_fwd(P(y), P(r), P(ko), P(vo), P(g), P(par3), P(par3[1]),
                                                 P(par3[2]), P(z), B, T, C, st), 12 * n),
        "post_bwd": (lambda: L.camoe_tm_post_bwd(P(dz), P(y), P(r), P(ko), P(vo), P(g), P(par3),
                                                 P(par3[1]), P(par3[2]), *[P(t) for t in outs5],
                                                 P(dpar), P(work), nw, B, T, C, st), 22 * n),
        "lnsa_fwd": (lambda: L.camoe_tm_lnsa_fwd(P(sa), P(par2[0]), P(par2[1]), P(srep), B, T, C,
                                                 st), 8 * n),
        "lnsa_bwd": (lambda: L.camoe_tm_lnsa_bwd(P(dsrep), P(sa), P(par2[0]), P(dsa), P(dpar),
                                                 P(work), nw, B, T, C, st), 12 * n),
    }
    lines = []
    flush = torch.empty(64 << 20, dtype=torch.float32, device="cuda")  # 256 MB, twice the L2
    for name, (fn, nbytes) in calls.items():
        assert fn() == 0, name
        us = time_flushed_us(fn, steps, flush)
        gbs = nbytes / us / 1e3
        lines.append({"kernel": name, "workload": f"B={B} T={T} C={C}", "us": round(us, 2),
                      "bytes": nbytes, "achieved_gbs": round(gbs, 1), "peak_gbs": peak,
                      "frac": round(gbs / peak, 3), "peak_kind": kind})
    return lines


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--batch", type=int, default=8)
    ap.add_argument("--seq", type=int, default=1024)
    ap.add_argument("--embd", type=int, default=1024)
    ap.add_argument("--layer", type=int, default=2)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--no-layer", action="store_true")
    args = ap.parse_args()
    if not args.no_layer:
        print(json.dumps(bench_layer(args.batch, args.seq, args.embd, args.layer, args.steps)))
        print(json.dumps(bench_decode(64, args.seq, args.embd, args.layer, 5 * args.steps)))
    for line in bench_kernels(args.batch, args.seq, args.embd, args.steps):
        print(json.dumps(line))


if __name__ == "__main__":
    main()
