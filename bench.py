"""Benchmark of the WKV-7 ClampW forward+backward on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload NAME] [--algo auto|scan|chunked]

One step = one forward and one backward of the op over one batch of seeded
synthetic inputs (bf16, [B, T, H, 64]) resident in HBM.  The default workload
is B=4 sequences of T=4096 per GPU with H=16 heads of 64 (C=1024): the per-GPU
share of the B=32 batch sharded over 8 GPUs; each rank runs its own batch
shard with no collective (weak scaling).  Inputs per step (7 x 32 MiB) are
larger than the 126 MB L2, so no flush is needed between steps.

For N > 1 run one process per GPU under torch.distributed.run; the reported
time is the max over ranks of the CUDA-event time of the K timed steps.

``--split`` (strong scaling) takes the workload as the whole problem and
splits its B x H chains over the ranks as camoe_b200.launcher does (batch
shards, else (batch, head-group) shards read in place through the head
range); a shard of few long chains runs time-segmented
(camoe_b200.segmented.auto_segments).  E.g. ``--workload long_b2_t65536
--split`` under 8 ranks: 8 chains of 65536 steps per GPU.  Inputs are drawn on
the GPU from a seeded generator.

``--impl reference`` times the CPU oracle port of the reference's recurrence
(fp32, every host thread) on a bounded sample of the same workload; it prints
the same JSON line with "impl": "reference".
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import statistics
import subprocess
import sys
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

from camoe_b200 import ops  # noqa: E402
from camoe_b200.inputs import WORKLOADS, make_inputs  # noqa: E402

METRIC = "WKV-7 fwd+bwd tokens/s per GPU and % HBM roofline at 1/2/4/8 B200"
NAMES = ("r", "w", "k", "v", "a", "b")
# algorithmic bytes per (b, t, h, i) element: forward reads 6 bf16 inputs and
# writes y (bf16) and sa (fp32); backward reads 7 bf16 inputs and writes 6 bf16
# gradients.
FWD_BYTES, BWD_BYTES = 6 * 2 + 2 + 4, 7 * 2 + 6 * 2
FALLBACK_HBM_GBS = 6650.0


def profiled_traffic(workload: str, kernels: list[str]):
    """DRAM bytes (read + write) per launch of `kernels`, summed, from the committed
    ncu launch-list summary of this workload (profiles/launches_<workload>.md), or
    None when there is no such capture."""
    path = os.path.join(ROOT, "profiles", f"launches_{workload}.md")
    try:
        with open(path) as f:
            line = next(l for l in f if l.startswith("traffic-per-launch-bytes:"))
    except (OSError, StopIteration):
        return None
    per = dict(kv.split("=") for kv in line.split(":", 1)[1].split())
    try:
        return sum(int(per[k]) for k in kernels)
    except KeyError:
        return None


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.proc = None
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "50", "-i", str(gpu_index)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=10)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out, _ = self.proc.communicate()
        sm, smax, reasons, power = [], [], set(), []
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for line in out.strip().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax.append(float(parts[2]))
                power.append(float(parts[3]))
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        loaded = [s for s in sm if smax and s > 0.5 * max(smax)] or sm
        return {"sm_mhz": statistics.median(loaded) if loaded else None,
                "sm_max_mhz": max(smax) if smax else None,
                "reasons": sorted(reasons), "samples": len(sm),
                "power_w_max": max(power) if power else None}


def dist_setup(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    elif torch.cuda.is_available():
        torch.cuda.set_device(local)
    return world, rank, local


def barrier(world, local):
    if world > 1:
        import torch.distributed as dist
        dist.barrier(device_ids=[local])


def max_over_ranks(x: float, world: int, local: int) -> float:
    if world == 1:
        return x
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device=f"cuda:{local}")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def cpu_baseline(wl: dict, budget_s: float = 15.0, seed: int = 0):
    """Time the CPU oracle (fp32, all host threads) on a bounded sample of the
    workload: B and H as configured, T truncated to fit ~budget_s."""
    import oracle

    threads = oracle.default_threads()
    B, H, N, T = wl["B"], wl["H"], wl["N"], wl["T"]

    def run(t_len):
        inp = make_inputs(B, t_len, H, N, seed=seed, w_mu=wl["w_mu"], w_sigma=wl["w_sigma"])
        xs = [inp[n] for n in NAMES]
        t0 = time.perf_counter()
        oracle.fwd(*xs, precision="f32", threads=threads)
        oracle.bwd(*xs, inp["dy"], precision="f32", ckpt=16, threads=threads)
        return time.perf_counter() - t0

    t_probe = min(T, 64)
    dt = run(t_probe)
    t_len = T
    est = dt * T / t_probe
    if est > budget_s:
        t_len = max(16, int(T * budget_s / est) // 16 * 16)
    dt = run(t_len)
    tokens = B * t_len
    return {"value": tokens / dt, "unit": "tokens/s", "cores": threads, "kind": "port",
            "sample": f"B={B} T={t_len} (of {T}) H={H} N={N} fp32 fwd+bwd, C oracle "
                      f"(restatement of camoe/backbone.py:264-294 + rwkv7_clampw.cu:83-170), "
                      f"{threads} threads, {dt:.2f} s"}


def run_reference(args, wl, world, rank):
    if rank != 0:
        return
    cb = cpu_baseline(wl, budget_s=float(os.environ.get("CAMOE_CPU_BUDGET_S", "12")))
    line = {"impl": "reference", "metric": METRIC, "value": cb["value"], "unit": "tokens/s",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": 1e3 * wl["B"] * wl["T"] / cb["value"], "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": config_of(args, wl, world), "cpu_baseline": cb,
            "e2e": {"value": cb["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def run_split(args, wl, world, rank, local):
    """Strong scaling: the workload is the whole problem, split over the ranks."""
    import torch.nn.functional as F

    from camoe_b200 import launcher, segmented

    dev = torch.device("cuda", local)
    B, T, H, N = wl["B"], wl["T"], wl["H"], wl["N"]
    sh = launcher.plan_shards(B, H, world)[rank]
    nb, hc = sh.b1 - sh.b0, sh.h1 - sh.h0
    gen = torch.Generator(device=dev).manual_seed(1000 + rank)
    shp = (nb, T, H, N)
    r, k, v, u, dy, w, kk = (torch.randn(shp, generator=gen, device=dev) for _ in range(7))
    w = wl["w_mu"] + wl["w_sigma"] * w
    kk = F.normalize(kk, dim=-1, p=2.0)
    xs = [t.to(torch.bfloat16).contiguous() for t in (r, w, k, v, -kk, kk * torch.sigmoid(u))]
    dy = dy.to(torch.bfloat16)
    del r, k, v, u, w, kk
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    P = segmented.auto_segments(nb * hc, T, sms) if args.segments == "auto" else int(args.segments)
    y = torch.zeros_like(xs[0])
    sa = torch.zeros(xs[0].shape, dtype=torch.float32, device=dev)
    grads = tuple(torch.zeros_like(xs[0]) for _ in range(6))
    ckpt = torch.empty(max(ops.ckpt_bytes(nb, T, hc, torch.bfloat16), 16), dtype=torch.uint8,
                       device=dev)
    work = torch.empty(max(ops.work_bytes(nb, T, hc, torch.bfloat16), 16), dtype=torch.uint8,
                       device=dev)
    stream = torch.cuda.current_stream(dev)

    def step(ev=None):
        if ev is not None:
            ev[0].record(stream)
        if P > 1:
            _, _, saved = segmented.wkv7_forward_segmented(*xs, P, h0=sh.h0, h_count=hc, y=y,
                                                           sa=sa)
            if ev is not None:
                ev[1].record(stream)
            segmented.wkv7_backward_segmented(saved, dy, grads=grads)
        else:
            ops.wkv7_forward(*xs, h0=sh.h0, h_count=hc, y=y, sa=sa, ckpt=ckpt)
            if ev is not None:
                ev[1].record(stream)
            ops.wkv7_backward(*xs, dy, None, ckpt, h0=sh.h0, h_count=hc, grads=grads, work=work)
        if ev is not None:
            ev[2].record(stream)

    clocks = ClockSampler(local)
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(dev)
    barrier(world, local)
    torch.cuda.synchronize(dev)
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(args.steps)]
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for kk_ in range(args.steps):
        step(evs[kk_])
    end.record(stream)
    torch.cuda.synchronize(dev)
    barrier(world, local)
    torch.cuda.synchronize(dev)
    clk = clocks.stop()
    ms = max_over_ranks(start.elapsed_time(end), world, local)
    fwd_ms = max_over_ranks(sum(e[0].elapsed_time(e[1]) for e in evs) / args.steps, world, local)
    bwd_ms = max_over_ranks(sum(e[1].elapsed_time(e[2]) for e in evs) / args.steps, world, local)
    step_ms = ms / args.steps
    value = B * T * args.steps / (ms / 1e3)
    hbm, peak_kind = peaks()
    shard_elems = nb * T * hc * N
    step_gbs = (FWD_BYTES + BWD_BYTES) * shard_elems / (step_ms / 1e3) / 1e9
    bwd_gbs = BWD_BYTES * shard_elems / (bwd_ms / 1e3) / 1e9
    if rank == 0:
        line = {"metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": step_ms,
                "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
                "dtype": "bf16", "data": "synthetic (seeded randn drawn on the GPU)",
                "config": {"workload": f"{args.workload} split: B={B} T={T} H={H} N={N} bf16 "
                                       f"WKV-7 ClampW fwd+bwd over {world} GPU(s), {nb} "
                                       f"sequence(s) x {hc} heads per GPU",
                           "model": "WKV-7 ClampW op", "global_batch": B, "seq_len": T,
                           "heads": H, "head_size": N, "segments_per_chain": P,
                           "parallelism": f"{world} (batch, head-group) shards, no collective",
                           "l2": "inputs larger than L2, no flush",
                           "w_in": f"N({wl['w_mu']},{wl['w_sigma']})"},
                "roofline": {"bound": "hbm", "kernel": "backward of one GPU's shard",
                             "achieved": bwd_gbs, "peak": hbm, "peak_kind": peak_kind,
                             "unit": "GB/s", "frac": bwd_gbs / hbm, "traffic": None,
                             "fwd_ms": fwd_ms, "bwd_ms": bwd_ms, "step_achieved": step_gbs,
                             "step_frac": step_gbs / hbm},
                "clocks": clk,
                "gpu_launches": (9 if P > 1 else 4) * args.steps,
                "tokens_per_s_per_gpu": value / world}
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


def config_of(args, wl, world):
    return {"workload": f"{args.workload}: B={wl['B']}/GPU T={wl['T']} H={wl['H']} N={wl['N']} "
                        f"bf16 WKV-7 ClampW fwd+bwd", "model": "WKV-7 ClampW op",
            "global_batch": wl["B"] * world, "seq_len": wl["T"], "heads": wl["H"],
            "head_size": wl["N"], "parallelism": f"dp{world} (batch shards, no collective)",
            "algo": args.algo, "l2": "inputs larger than L2 (7 x 32 MiB per step), no flush",
            "w_in": f"N({wl['w_mu']},{wl['w_sigma']})"}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=300)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="shard_b4_t4096", choices=sorted(WORKLOADS))
    ap.add_argument("--algo", default="auto", choices=["auto", "scan", "chunked"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--split", action="store_true",
                    help="strong scaling: split the workload's chains over the ranks")
    ap.add_argument("--segments", default="auto", help="with --split: segments per chain")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    wl = WORKLOADS[args.workload]

    if args.impl == "reference":
        world = int(os.environ.get("WORLD_SIZE", "1"))
        rank = int(os.environ.get("RANK", "0"))
        run_reference(args, wl, world, rank)
        return

    world, rank, local = dist_setup(args)
    if args.split:
        run_split(args, wl, world, rank, local)
        return
    dev = torch.device("cuda", local)
    B, T, H, N = wl["B"], wl["T"], wl["H"], wl["N"]
    inp = make_inputs(B, T, H, N, seed=1000 + rank, w_mu=wl["w_mu"], w_sigma=wl["w_sigma"],
                      dtype=torch.bfloat16)
    xs = [inp[n].to(dev) for n in NAMES]
    dy = inp["dy"].to(dev)
    stream = torch.cuda.current_stream(dev)

    # preallocated outputs: the timed step is exactly one fwd + one bwd launch pair
    y, sa, ckpt = ops.wkv7_forward(*xs, algo=args.algo)
    wb = ops.work_bytes(B, T, H, torch.bfloat16, args.algo)
    work = torch.empty(max(wb, 16), dtype=torch.uint8, device=dev)
    grads = ops.wkv7_backward(*xs, dy, None, ckpt, algo=args.algo, work=work)

    def step(ev=None):
        if ev is not None:
            ev[0].record(stream)
        ops.wkv7_forward(*xs, algo=args.algo, y=y, sa=sa, ckpt=ckpt)
        if ev is not None:
            ev[1].record(stream)
        ops.wkv7_backward(*xs, dy, None, ckpt, algo=args.algo, grads=grads, work=work)
        if ev is not None:
            ev[2].record(stream)

    clocks = ClockSampler(local) if rank == 0 or world > 1 else None
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(dev)
    barrier(world, local)
    torch.cuda.synchronize(dev)
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(args.steps)]
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for k in range(args.steps):
        step(evs[k])
    end.record(stream)
    torch.cuda.synchronize(dev)
    barrier(world, local)
    torch.cuda.synchronize(dev)
    clk = clocks.stop() if clocks is not None else None

    ms_local = start.elapsed_time(end)
    fwd_ms = sum(e[0].elapsed_time(e[1]) for e in evs) / args.steps
    bwd_ms = sum(e[1].elapsed_time(e[2]) for e in evs) / args.steps
    ms = max_over_ranks(ms_local, world, local)
    tokens_per_rank = B * T
    value = tokens_per_rank * world * args.steps / (ms / 1e3)
    elems = B * T * H * N

    hbm, peak_kind = peaks()
    kern = "bwd" if bwd_ms >= fwd_ms else "fwd"
    k_ms = bwd_ms if kern == "bwd" else fwd_ms
    k_bytes = (BWD_BYTES if kern == "bwd" else FWD_BYTES) * elems
    achieved = k_bytes / (k_ms / 1e3) / 1e9
    step_ms = ms / args.steps
    step_gbs = (FWD_BYTES + BWD_BYTES) * elems / (step_ms / 1e3) / 1e9
    kname = {"fwd": "forward (keyside_kernel + value_fwd_kernel)",
             "bwd": "backward (value_bwd_kernel + keyside_bwd_kernel)"}[kern]
    traffic = None
    if args.algo == "scan":
        kname = f"scan_{kern}_kernel"
    else:
        traffic = profiled_traffic(args.workload,
                                   ["value_bwd_kernel", "keyside_bwd_kernel"] if kern == "bwd"
                                   else ["keyside_kernel", "value_fwd_kernel"])
    roofline = {"bound": "hbm", "kernel": kname, "achieved": achieved,
                "peak": hbm, "peak_kind": peak_kind, "unit": "GB/s", "frac": achieved / hbm,
                "traffic": traffic,
                "traffic_source": (f"profiles/launches_{args.workload}.md (ncu dram__bytes_read.sum"
                                   " + dram__bytes_write.sum per launch)") if traffic else None,
                "algorithmic_bytes_per_launch": k_bytes,
                "launch_ms": k_ms, "fwd_ms": fwd_ms, "bwd_ms": bwd_ms,
                "step_achieved": step_gbs, "step_frac": step_gbs / hbm,
                "bytes_per_element": {"fwd": FWD_BYTES, "bwd": BWD_BYTES}}

    e2e = None
    if not args.no_e2e:
        e2e = measure_e2e(args, xs, dy, dev, stream, world, local)

    cb = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cb = cpu_baseline(wl, budget_s=float(os.environ.get("CAMOE_CPU_BUDGET_S", "12")))

    if rank == 0:
        line = {"metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": step_ms,
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
                "dtype": "bf16", "data": "synthetic (seeded randn, distributions of the op's "
                                         "workloads)",
                "config": config_of(args, wl, world), "roofline": roofline,
                "cpu_baseline": cb, "clocks": clk, "e2e": e2e,
                "gpu_launches": (4 if args.algo in ("auto", "chunked") else 2) * args.steps,
                "tokens_per_s_per_gpu": value / world}
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


def measure_e2e(args, xs, dy, dev, stream, world, local):
    """Same metric through the public autograd API with host buffers: every step
    copies its inputs from pinned host memory and reads every output back.

    Steps are pipelined as an input pipeline would run them: step k+1's inputs go
    host -> device on one copy stream (into the other of two device buffers) and
    step k's outputs go device -> host on a second copy stream while the op runs
    on the compute stream, so both PCIe directions overlap the compute.  The timed
    region starts before the first input copy and ends after the last output copy."""
    from camoe_b200 import backbone

    os.environ.setdefault("CAMOE_WKV7_ALGO", args.algo)
    backbone.init_rwkv7_cuda()
    host_in = [x.cpu().pin_memory() for x in xs] + [dy.cpu().pin_memory()]
    n_out = 8
    host_out = [torch.empty(xs[0].shape, dtype=torch.bfloat16 if i != 1 else torch.float32,
                            pin_memory=True) for i in range(n_out)]
    h2d = sum(t.numel() * t.element_size() for t in host_in)
    d2h = sum(t.numel() * t.element_size() for t in host_out)
    bufs = [[torch.empty_like(h, device=dev) for h in host_in] for _ in range(2)]
    up, down = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    freed = [torch.cuda.Event(), torch.cuda.Event()]  # compute done with buffer b
    landed = [torch.cuda.Event(), torch.cuda.Event()]  # inputs of buffer b on the device
    computed = torch.cuda.Event()

    def copy_in(k):
        b = k % 2
        with torch.cuda.stream(up):
            if k >= 2:
                up.wait_event(freed[b])
            for d, h in zip(bufs[b], host_in):
                d.copy_(h, non_blocking=True)
            landed[b].record(up)

    def step(k, last):
        b = k % 2
        stream.wait_event(landed[b])
        ins = [t.detach().requires_grad_(True) for t in bufs[b][:6]]
        y, sa = backbone.RWKV7_ClampW.apply(*ins)
        torch.autograd.backward([y], [bufs[b][6]])
        outs = [y, sa] + [t.grad for t in ins]
        freed[b].record(stream)
        if not last:
            copy_in(k + 1)
        computed.record(stream)
        with torch.cuda.stream(down):
            down.wait_event(computed)
            for h, o in zip(host_out, outs):
                h.copy_(o, non_blocking=True)
                o.record_stream(down)

    def run(n):
        copy_in(0)
        for k in range(n):
            step(k, k == n - 1)

    steps = max(3, min(args.steps, 20))
    run(2)
    torch.cuda.synchronize(dev)
    barrier(world, local)
    s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s0.record(stream)
    up.wait_stream(stream)
    run(steps)
    stream.wait_stream(down)
    s1.record(stream)
    torch.cuda.synchronize(dev)
    barrier(world, local)
    ms = max_over_ranks(s0.elapsed_time(s1), world, local)
    tokens = xs[0].shape[0] * xs[0].shape[1] * world * steps
    return {"value": tokens / (ms / 1e3), "unit": "tokens/s", "h2d_bytes_per_step": h2d,
            "d2h_bytes_per_step": d2h, "steps": steps,
            "api": "camoe_b200.backbone.RWKV7_ClampW.apply + autograd backward",
            "pipelining": "inputs of step k+1 and outputs of step k copied on two streams "
                          "while step k computes"}


if __name__ == "__main__":
    main()
