"""Timings of the long-context problem's 8-GPU share on one GPU: the
one-pass op against the time-segmented path (camoe_b200.segmented).

    python -m camoe_b200.bench_long [--segments 4,8,16,32] [--steps 10]

Workload: B=2 T=65536 H=32 N=64 bf16 (C=2048), w_in ~ N(2, 0.5), the rest as
camoe_b200.inputs.make_inputs draws it, generated on the GPU from a seeded
generator; one GPU's share of the (b, head-group) split over 8 GPUs is the
heads [0, 4) of both sequences, 8 chains, read and written in place through
the head range.  Each step is one forward and one backward (all six
gradients) over the share; inputs (7 x 268 MB) exceed L2, so no flush.

Prints one JSON line per variant: ms per step, tokens/s of the share
(B x T), and the HBM roofline fraction of the share's 44 algorithmic bytes
per (b, t, h, i) element.  Timing: CUDA events on the launching stream after
warm-up.
"""
from __future__ import annotations

import argparse
import json

import torch

from . import ops, segmented
from .bench_state import hbm_peak_gbs

ELEM_BYTES = 18 + 26  # forward + backward algorithmic bytes per element


def make_share(B=2, T=65536, H=32, seed=0):
    gen = torch.Generator(device="cuda").manual_seed(seed)
    shp = (B, T, H, 64)
    r, k, v, u, dy, w, kk = (torch.randn(shp, generator=gen, device="cuda") for _ in range(7))
    w = 2.0 + 0.5 * w
    kk = torch.nn.functional.normalize(kk, dim=-1, p=2.0)
    xs = [t.to(torch.bfloat16).contiguous() for t in (r, w, k, v, -kk, kk * torch.sigmoid(u))]
    return xs, dy.to(torch.bfloat16)


def time_steps(step, steps: int, warmup: int = 3) -> float:
    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(steps):
        step()
    end.record()
    torch.cuda.synchronize()
    return start.elapsed_time(end) / steps


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--segments", default="4,8,16,32")
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--heads", type=int, default=4, help="heads per GPU (h_count)")
    args = ap.parse_args()
    B, T, H = 2, 65536, 32
    h0, hc = 0, args.heads
    xs, dy = make_share(B, T, H)
    y = torch.zeros_like(xs[0])
    sa = torch.zeros(xs[0].shape, device="cuda")
    grads = tuple(torch.zeros_like(xs[0]) for _ in range(6))
    wb = ops.work_bytes(B, T, hc, torch.bfloat16)
    work = torch.empty(max(wb, 16), dtype=torch.uint8, device="cuda")
    ckpt = torch.empty(max(ops.ckpt_bytes(B, T, hc, torch.bfloat16), 16), dtype=torch.uint8,
                       device="cuda")
    hbm, kind = hbm_peak_gbs()
    elems = B * T * hc * 64

    def report(name, ms, extra=None):
        gbs = ELEM_BYTES * elems / (ms / 1e3) / 1e9
        line = {"workload": f"long_b2_t65536 share: B={B} T={T} heads {h0}..{h0 + hc - 1} of {H}",
                "variant": name, "ms_per_step": ms, "tokens_per_s": B * T / (ms / 1e3),
                "hbm_gbs": gbs, "roofline_frac": gbs / hbm, "peak": hbm, "peak_kind": kind}
        line.update(extra or {})
        print(json.dumps(line), flush=True)

    def one_pass():
        ops.wkv7_forward(*xs, h0=h0, h_count=hc, y=y, sa=sa, ckpt=ckpt)
        ops.wkv7_backward(*xs, dy, None, ckpt, h0=h0, h_count=hc, grads=grads, work=work)

    report("one pass", time_steps(one_pass, args.steps))
    for P in (int(p) for p in args.segments.split(",") if p):
        def seg_step(P=P):
            _, _, saved = segmented.wkv7_forward_segmented(*xs, P, h0=h0, h_count=hc, y=y, sa=sa)
            segmented.wkv7_backward_segmented(saved, dy, grads=grads)

        report(f"{P} segments", time_steps(seg_step, args.steps), {"segments": P})


if __name__ == "__main__":
    main()
