"""Timings of the stateful forward (camoe_wkv7_fwd_state) on one GPU.

    python -m camoe_b200.bench_state [--decode-batch 1024] [--heads 16] [--steps 50]

Prints one JSON line per workload:

* ``decode``: one generated token for B sequences of H heads, the state
  ([B, H, 64, 64] fp32) updated in place by the decode-step kernel.  The step
  is captured in a CUDA graph (``steps`` launches per replay) so the number is
  the kernel's, not Python's.  Its cost is the state: 32 KiB of HBM traffic
  per chain (16 KiB read, 16 KiB written) plus 1 KiB of inputs and outputs,
  so the roofline is HBM bandwidth.  The state (B*H*16 KiB) is larger than L2
  for B >= 512 at H = 16.
* ``prefill``: a prompt of T tokens from a given start state to the final
  state (bf16), through the fused one-CTA-per-chain kernel and through the
  two-kernel path with a workspace.

Inputs are seeded synthetic data (camoe_b200.inputs.make_inputs).  Timing:
CUDA events on the launching stream after warm-up.
"""
from __future__ import annotations

import argparse
import json
import os

import torch

from . import ops
from .inputs import make_inputs

NAMES = ("r", "w", "k", "v", "a", "b")
STATE_BYTES = 64 * 64 * 4


def hbm_peak_gbs() -> tuple[float, str]:
    path = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))),
                        "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, "fallback"


def bench_decode(B: int, H: int, dtype: torch.dtype, steps: int, reps: int) -> dict:
    inp = make_inputs(B, 1, H, seed=0)
    xs = [inp[n].to(dtype).cuda()[:, 0].contiguous() for n in NAMES]
    state = torch.randn(B, H, 64, 64, device="cuda")
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for _ in range(3):
            ops.wkv7_decode_step(*xs, state)
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for _ in range(steps):
            ops.wkv7_decode_step(*xs, state)
    for _ in range(3):
        graph.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        graph.replay()
    e1.record()
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / (reps * steps)
    esz = torch.tensor([], dtype=dtype).element_size()
    chains = B * H
    # per chain: state read + written, six inputs read, y (dtype) and sa (fp32) written
    algo_bytes = chains * (2 * STATE_BYTES + 64 * (6 * esz + esz + 4))
    peak, kind = hbm_peak_gbs()
    gbs = algo_bytes / us / 1e3
    return {"workload": f"decode: B={B} H={H} one token, {str(dtype).split('.')[-1]} inputs, "
                        f"fp32 state {chains * STATE_BYTES / 2**20:.0f} MiB",
            "metric": "decode_tokens_per_s", "value": round(B / us * 1e6),
            "us_per_step": round(us, 2),
            "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": peak,
                         "unit": "GB/s", "frac": round(gbs / peak, 3), "peak_kind": kind,
                         "bytes_per_step": algo_bytes},
            "timing": f"CUDA graph of {steps} steps, {reps} replays"}


def bench_prefill(B: int, T: int, H: int, reps: int) -> dict:
    inp = make_inputs(B, T, H, seed=0)
    xs = [inp[n].to(torch.bfloat16).cuda() for n in NAMES]
    state = torch.randn(B, H, 64, 64, device="cuda")
    y = torch.empty_like(xs[0])
    sa = torch.empty(xs[0].shape, device="cuda")
    wt = torch.empty(max(ops.state_work_bytes(B, T, H, torch.bfloat16), 16), dtype=torch.uint8,
                     device="cuda")
    out = {"workload": f"prefill: B={B} T={T} H={H} bf16 from a start state",
           "metric": "prefill_tokens_per_s"}
    for name, work in (("fused", False), ("workspace", wt)):
        def run():
            ops.wkv7_forward_state(*xs, state, inplace=True, work=work, y=y, sa=sa)
        for _ in range(3):
            run()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            run()
        e1.record()
        torch.cuda.synchronize()
        us = e0.elapsed_time(e1) * 1e3 / reps
        out[name] = {"us": round(us, 1), "tokens_per_s": round(B * T / us * 1e6)}
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--decode-batch", type=int, default=1024)
    ap.add_argument("--heads", type=int, default=16)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--reps", type=int, default=10)
    ap.add_argument("--prefill", default="4x4096,8x1024", help="BxT list for the prefill lines")
    args = ap.parse_args()
    for dt in (torch.bfloat16, torch.float32):
        print(json.dumps(bench_decode(args.decode_batch, args.heads, dt, args.steps, args.reps)))
    for bt in filter(None, args.prefill.split(",")):
        B, T = (int(x) for x in bt.split("x"))
        print(json.dumps(bench_prefill(B, T, args.heads, args.reps)))


if __name__ == "__main__":
    main()
