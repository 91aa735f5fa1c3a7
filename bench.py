"""Benchmark of the WKV-7 ClampW forward+backward on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload NAME] [--algo auto|scan|chunked]

One step = one forward and one backward of the op over one batch of seeded
synthetic inputs (bf16, [B, T, H, 64]) resident in HBM.  The default workload
is B=4 sequences of T=4096 per GPU with H=16 heads of 64 (C=1024): the per-GPU
share of the B=32 batch sharded over 8 GPUs; each rank runs its own batch
shard with no collective (weak scaling).  Inputs per step (7 x 32 MiB) are
larger than the 126 MB L2, so no flush is needed between steps.

Timing: W warm-up steps, then R blocks of exactly K steps, each block
bracketed by a barrier and a device synchronisation on both sides and timed
with CUDA events on the launching stream (max over ranks).  ``ms_per_step`` is
the median block / K; the nvidia-smi clock sampler runs across all blocks, so
it sees the timed region even when one block is a few milliseconds.  R is at
least ``--blocks`` and grows until the blocks cover ``--min-timed-s``.

For N > 1 run one process per GPU under torch.distributed.run.

Workloads of the op (``--workload``): ``shard_b4_t4096`` (default),
``layer_b8_t1024`` (the single-GPU layer shape), ``long_b2_t65536`` (the
long-context problem; with ``--split`` it is split over the ranks as
camoe_b200.launcher does, a shard of few long chains running time-segmented;
with ``--share-heads H`` one GPU times the one-pass op against the
time-segmented path on heads [0, H) of both sequences, ``--segments`` listing
the segment counts).  Other workloads print their own lines:
``decode_b1024_h16`` (one generated token through the decode-step kernel,
bf16 and fp32, and prefills from a start state), ``timemix_b8_t1024_c1024``
(the fused time mix: layer forward+backward against the op-by-op layer, a
stateful decode token, and each fused kernel, and the tcgen05 LoRA weight
gradient per rank, alone against HBM bandwidth).

``--impl reference`` times the CPU oracle port of the reference's recurrence
(fp32, every host thread) on a bounded sample of the same workload and prints
the same JSON line with "impl": "reference"; on a GPU box it adds, as an extra
key, the reference's own CUDA op (built from its sources into oracle/_ref)
timed on the same workload in bf16 and fp32.
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
OTHER_WORKLOADS = ("decode_b1024_h16", "timemix_b8_t1024_c1024", "train_step_c4")
# the op's calls in one train step of the 0.4B CaMoE configuration: 12 RWKV-7
# layers at C=1024, B=8 sequences of T=1024; each layer's attention stage runs
# under activation checkpointing (camoe/system.py:317-324), so the op runs a
# forward, a recompute forward and a backward per layer
C4 = dict(layers=12, B=8, T=1024, H=16, N=64)
# kernels of this repository (their names all sit in the camoe namespace)
OWN_KERNEL_TAG = "camoe::"


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
                 "-lms", "20", "-i", str(gpu_index)],
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


def count_launches(fn, dev) -> dict:
    """Kernel launches of one call of `fn`, read from the CUDA activity trace
    (torch.profiler): this repository's kernels, other kernels (library and
    torch fills), and memory copies/sets.  Run outside any timed region."""
    try:
        from torch.autograd import DeviceType
        from torch.profiler import ProfilerActivity, profile
        torch.cuda.synchronize(dev)
        with profile(activities=[ProfilerActivity.CUDA]) as prof:
            fn()
            torch.cuda.synchronize(dev)
        own, other, mem = 0, 0, 0
        names = set()
        for e in prof.events():
            if e.device_type != DeviceType.CUDA:
                continue
            n = e.name
            if n.startswith("Memcpy") or n.startswith("Memset"):
                mem += 1
            elif OWN_KERNEL_TAG in n:
                own += 1
                names.add(n.split("(")[0].replace("void ", ""))
            else:
                other += 1
        return {"own": own, "other_kernels": other, "memcpy_memset": mem,
                "own_kernels": sorted(names), "source": "torch.profiler CUDA activity"}
    except Exception as e:  # pragma: no cover - tracing unavailable
        return {"own": None, "source": f"unavailable: {type(e).__name__}: {e}"}


def timed_blocks(step, K, dev, stream, world, local, min_blocks, min_total_s, phases=True):
    """Run blocks of exactly K steps, each bracketed by barrier + synchronize and
    timed with CUDA events on `stream`.  With `phases`, `step(ev)` records
    ev[0..2] around its forward and backward.  Returns (block ms list (max over
    ranks), mean fwd ms, mean bwd ms; the last two None without phases)."""
    blocks, fwd, bwd = [], [], []
    t_start = time.perf_counter()
    while True:
        evs = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(K)]
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize(dev)
        barrier(world, local)
        torch.cuda.synchronize(dev)
        start.record(stream)
        for k in range(K):
            step(evs[k] if phases else None)
        end.record(stream)
        torch.cuda.synchronize(dev)
        barrier(world, local)
        torch.cuda.synchronize(dev)
        blocks.append(start.elapsed_time(end))
        if phases:
            fwd += [e[0].elapsed_time(e[1]) for e in evs]
            bwd += [e[1].elapsed_time(e[2]) for e in evs]
        # every rank takes the same decision: on the max over ranks of the elapsed time
        elapsed = max_over_ranks(time.perf_counter() - t_start, world, local)
        if len(blocks) >= min_blocks and elapsed >= min_total_s:
            break
    blocks = [max_over_ranks(b, world, local) for b in blocks]
    if not phases:
        return blocks, None, None
    return (blocks, max_over_ranks(statistics.fmean(fwd), world, local),
            max_over_ranks(statistics.fmean(bwd), world, local))


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


def reference_cuda_op(wl: dict, steps: int, warmup: int) -> dict:
    """The reference's own ClampW CUDA op (camoe/cuda/rwkv7_clampw.cu, built from
    its sources with the flags of camoe/backbone.py:49-59 into oracle/_ref),
    timed fwd+bwd on the workload with CUDA events, bf16 and fp32 inputs."""
    import oracle

    if not torch.cuda.is_available():
        return {"unavailable": "no CUDA device"}
    B, T, H, N = wl["B"], wl["T"], wl["H"], wl["N"]
    out = {"source": "camoe/cuda/rwkv7_clampw.cu built from the reference's sources "
                     "(oracle/Makefile ref), launched through its cuda_forward/cuda_backward",
           "workload": f"B={B} T={T} H={H} N={N}"}
    inp = make_inputs(B, T, H, N, seed=0, w_mu=wl["w_mu"], w_sigma=wl["w_sigma"])
    dev = torch.device("cuda", 0)
    for fp32 in (False, True):
        key = "fp32" if fp32 else "bf16"
        if not oracle.RefOp.available(fp32=fp32):
            out[key] = {"unavailable": "oracle/_ref not built (make -C oracle ref)"}
            continue
        dt = torch.float32 if fp32 else torch.bfloat16
        op = oracle.RefOp(fp32=fp32)
        xs = [inp[n].to(dt).to(dev) for n in NAMES]
        dy = inp["dy"].to(dt).to(dev)
        y = torch.empty_like(xs[0])
        sa = torch.empty(xs[0].shape, dtype=torch.float32, device=dev)
        s = torch.empty(B, H, T // 16, N, N, dtype=torch.float32, device=dev)
        gs = [torch.empty_like(xs[0]) for _ in range(6)]
        # it launches on the legacy default stream: time there
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
        for _ in range(warmup):
            op.forward(*xs, y, s, sa)
            op.backward(*xs, dy, s, sa, *gs)
        torch.cuda.synchronize(dev)
        fwd, bwd = [], []
        for _ in range(steps):
            ev[0].record(torch.cuda.default_stream(dev))
            op.forward(*xs, y, s, sa)
            ev[1].record(torch.cuda.default_stream(dev))
            op.backward(*xs, dy, s, sa, *gs)
            ev[2].record(torch.cuda.default_stream(dev))
            torch.cuda.synchronize(dev)
            fwd.append(ev[0].elapsed_time(ev[1]))
            bwd.append(ev[1].elapsed_time(ev[2]))
        ms = statistics.median(f + b for f, b in zip(fwd, bwd))
        out[key] = {"ms_per_step": ms, "fwd_ms": statistics.median(fwd),
                    "bwd_ms": statistics.median(bwd), "tokens_per_s": B * T / (ms / 1e3),
                    "steps": steps}
        del xs, dy, y, sa, s, gs
        torch.cuda.empty_cache()
    return out


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
    if torch.cuda.is_available() and not args.no_reference_gpu:
        try:
            line["reference_cuda_op"] = reference_cuda_op(wl, steps=min(max(args.steps, 3), 10),
                                                          warmup=2)
        except Exception as e:  # reported, never fatal for the CPU arm
            line["reference_cuda_op"] = {"unavailable": f"{type(e).__name__}: {e}"}
    print(json.dumps(line), flush=True)


def make_gpu_inputs(B, T, H, N, dev, w_mu, w_sigma, seed):
    """The make_inputs distributions, drawn on the GPU (for sizes where the CPU
    generator would take long)."""
    import torch.nn.functional as F

    gen = torch.Generator(device=dev).manual_seed(seed)
    shp = (B, T, H, N)
    r, k, v, u, dy, w, kk = (torch.randn(shp, generator=gen, device=dev) for _ in range(7))
    w = w_mu + w_sigma * w
    kk = F.normalize(kk, dim=-1, p=2.0)
    xs = [t.to(torch.bfloat16).contiguous() for t in (r, w, k, v, -kk, kk * torch.sigmoid(u))]
    return xs, dy.to(torch.bfloat16)


def run_split(args, wl, world, rank, local):
    """Strong scaling: the workload is the whole problem, split over the ranks."""
    from camoe_b200 import launcher, segmented

    dev = torch.device("cuda", local)
    B, T, H, N = wl["B"], wl["T"], wl["H"], wl["N"]
    sh = launcher.plan_shards(B, H, world)[rank]
    nb, hc = sh.b1 - sh.b0, sh.h1 - sh.h0
    xs, dy = make_gpu_inputs(nb, T, H, N, dev, wl["w_mu"], wl["w_sigma"], 1000 + rank)
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
    seg_bufs = segmented.Buffers(nb, T, H, P, h0=sh.h0, h_count=hc, device=dev) if P > 1 else None

    def step(ev=None):
        if ev is not None:
            ev[0].record(stream)
        if P > 1:
            _, _, saved = segmented.wkv7_forward_segmented(*xs, P, h0=sh.h0, h_count=hc, y=y,
                                                           sa=sa, bufs=seg_bufs)
            if ev is not None:
                ev[1].record(stream)
            segmented.wkv7_backward_segmented(saved, dy, grads=grads, bufs=seg_bufs)
        else:
            ops.wkv7_forward(*xs, h0=sh.h0, h_count=hc, y=y, sa=sa, ckpt=ckpt)
            if ev is not None:
                ev[1].record(stream)
            ops.wkv7_backward(*xs, dy, None, ckpt, h0=sh.h0, h_count=hc, grads=grads, work=work)
        if ev is not None:
            ev[2].record(stream)

    for _ in range(args.warmup):
        step()
    launches = count_launches(step, dev)
    clocks = ClockSampler(local)
    blocks, fwd_ms, bwd_ms = timed_blocks(step, args.steps, dev, stream, world, local,
                                          args.blocks, args.min_timed_s)
    clk = clocks.stop()
    ms = statistics.median(blocks)
    step_ms = ms / args.steps
    value = B * T / (step_ms / 1e3)
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
                "timing": timing_note(blocks, args.steps),
                "roofline": {"bound": "hbm", "kernel": "backward of one GPU's shard",
                             "achieved": bwd_gbs, "peak": hbm, "peak_kind": peak_kind,
                             "unit": "GB/s", "frac": bwd_gbs / hbm, "traffic": None,
                             "fwd_ms": fwd_ms, "bwd_ms": bwd_ms, "step_achieved": step_gbs,
                             "step_frac": step_gbs / hbm},
                "clocks": clk,
                "gpu_launches": None if launches["own"] is None else launches["own"] * args.steps,
                "launches_per_step": launches,
                "tokens_per_s_per_gpu": value / world}
        print(json.dumps(line), flush=True)


def run_long_share(args, wl, dev):
    """One GPU's share of the long-context split (heads [0, H) of both
    sequences, read and written in place through the head range): the one-pass
    op against the time-segmented path for each segment count."""
    from camoe_b200 import segmented

    B, T, H, N = wl["B"], wl["T"], wl["H"], wl["N"]
    h0, hc = 0, args.share_heads
    xs, dy = make_gpu_inputs(B, T, H, N, dev, wl["w_mu"], wl["w_sigma"], 0)
    y = torch.zeros_like(xs[0])
    sa = torch.zeros(xs[0].shape, dtype=torch.float32, device=dev)
    grads = tuple(torch.zeros_like(xs[0]) for _ in range(6))
    work = torch.empty(max(ops.work_bytes(B, T, hc, torch.bfloat16), 16), dtype=torch.uint8,
                       device=dev)
    ckpt = torch.empty(max(ops.ckpt_bytes(B, T, hc, torch.bfloat16), 16), dtype=torch.uint8,
                       device=dev)
    hbm, kind = peaks()
    elems = B * T * hc * N
    stream = torch.cuda.current_stream(dev)
    for P in (int(p) for p in args.segments.split(",") if p):
        if P == 1:
            def step(ev=None):
                ops.wkv7_forward(*xs, h0=h0, h_count=hc, y=y, sa=sa, ckpt=ckpt)
                ops.wkv7_backward(*xs, dy, None, ckpt, h0=h0, h_count=hc, grads=grads, work=work)
        else:
            bufs = segmented.Buffers(B, T, H, P, h0=h0, h_count=hc, device=dev)

            def step(ev=None, P=P, bufs=bufs):
                _, _, saved = segmented.wkv7_forward_segmented(*xs, P, h0=h0, h_count=hc, y=y,
                                                               sa=sa, bufs=bufs)
                segmented.wkv7_backward_segmented(saved, dy, grads=grads, bufs=bufs)
        for _ in range(args.warmup):
            step()
        launches = count_launches(step, dev)
        blocks, _, _ = timed_blocks(step, args.steps, dev, stream, 1, 0, args.blocks,
                                    args.min_timed_s, phases=False)
        ms = statistics.median(blocks) / args.steps
        gbs = (FWD_BYTES + BWD_BYTES) * elems / (ms / 1e3) / 1e9
        print(json.dumps({
            "workload": f"{args.workload} share: B={B} T={T} heads {h0}..{h0 + hc - 1} of {H}",
            "variant": "one pass" if P == 1 else f"{P} segments", "segments": P,
            "ms_per_step": ms, "tokens_per_s": B * T / (ms / 1e3), "hbm_gbs": gbs,
            "roofline_frac": gbs / hbm, "peak": hbm, "peak_kind": kind,
            "launches_per_step": launches, "timing": timing_note(blocks, args.steps)}),
            flush=True)


def timing_note(blocks, K):
    return {"blocks": len(blocks), "steps_per_block": K,
            "block_ms_median": statistics.median(blocks), "block_ms_min": min(blocks),
            "block_ms_max": max(blocks),
            "protocol": "each block of exactly K steps bracketed by barrier + synchronize, "
                        "CUDA events on the launching stream, max over ranks; "
                        "ms_per_step = median block / K"}


def config_of(args, wl, world):
    return {"workload": f"{args.workload}: B={wl['B']}/GPU T={wl['T']} H={wl['H']} N={wl['N']} "
                        f"{args.dtype} WKV-7 ClampW fwd+bwd", "model": "WKV-7 ClampW op",
            "global_batch": wl["B"] * world, "seq_len": wl["T"], "heads": wl["H"],
            "head_size": wl["N"], "parallelism": f"dp{world} (batch shards, no collective)",
            "algo": args.algo, "l2": "inputs larger than L2 (7 x 32 MiB per step), no flush",
            "w_in": f"N({wl['w_mu']},{wl['w_sigma']})"}


def run_op(args, wl, world, rank, local):
    dev = torch.device("cuda", local)
    B, T, H, N = wl["B"], wl["T"], wl["H"], wl["N"]
    dt = torch.float32 if args.dtype == "fp32" else torch.bfloat16
    inp = make_inputs(B, T, H, N, seed=1000 + rank, w_mu=wl["w_mu"], w_sigma=wl["w_sigma"],
                      dtype=dt)
    xs = [inp[n].to(dev) for n in NAMES]
    dy = inp["dy"].to(dev)
    stream = torch.cuda.current_stream(dev)

    # preallocated outputs: the timed step is exactly one fwd + one bwd call
    y, sa, ckpt = ops.wkv7_forward(*xs, algo=args.algo)
    wb = ops.work_bytes(B, T, H, dt, args.algo)
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

    for _ in range(args.warmup):
        step()
    scan = args.algo == "scan" or dt == torch.float32
    launches = {"own": 2 if scan else 4, "source": "static (--no-trace)"} \
        if args.no_trace else count_launches(step, dev)
    clocks = ClockSampler(local)
    blocks, fwd_ms, bwd_ms = timed_blocks(step, args.steps, dev, stream, world, local,
                                          args.blocks, args.min_timed_s)
    clk = clocks.stop()

    ms = statistics.median(blocks)
    step_ms = ms / args.steps
    value = B * T * world / (step_ms / 1e3)
    elems = B * T * H * N
    hbm, peak_kind = peaks()
    kern = "bwd" if bwd_ms >= fwd_ms else "fwd"
    k_ms = bwd_ms if kern == "bwd" else fwd_ms
    # fp32 inputs and outputs (sa is fp32 either way) double the bf16 element bytes
    fwd_b, bwd_b = (FWD_BYTES, BWD_BYTES) if dt == torch.bfloat16 else (6 * 4 + 4 + 4, 13 * 4)
    k_bytes = (bwd_b if kern == "bwd" else fwd_b) * elems
    achieved = k_bytes / (k_ms / 1e3) / 1e9
    step_gbs = (fwd_b + bwd_b) * elems / (step_ms / 1e3) / 1e9
    kname = {"fwd": "forward (keyside_kernel + value_fwd_kernel)",
             "bwd": "backward (value_bwd_kernel + keyside_bwd_kernel)"}[kern]
    traffic = None
    if scan:
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
                "bytes_per_element": {"fwd": fwd_b, "bwd": bwd_b}}

    e2e = None
    if not args.no_e2e and dt == torch.bfloat16:  # the autograd API's default (bf16) path
        e2e = measure_e2e(args, xs, dy, dev, stream, world, local)

    cb = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cb = cpu_baseline(wl, budget_s=float(os.environ.get("CAMOE_CPU_BUDGET_S", "12")))

    if rank == 0:
        own = launches.get("own")
        line = {"metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": step_ms,
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
                "dtype": args.dtype, "data": "synthetic (seeded randn, distributions of the "
                                             "op's workloads)",
                "config": config_of(args, wl, world), "roofline": roofline,
                "timing": timing_note(blocks, args.steps),
                "cpu_baseline": cb, "clocks": clk, "e2e": e2e,
                "gpu_launches": None if own is None else own * args.steps,
                "launches_per_step": launches,
                "tokens_per_s_per_gpu": value / world}
        print(json.dumps(line), flush=True)


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


# ---------------------------------------------------------------------------
# Other workloads: the decode step and prefill (stateful forward), the fused
# time mix.  One JSON line per measurement; CUDA events on the launching stream
# after warm-up.
# ---------------------------------------------------------------------------

STATE_BYTES = 64 * 64 * 4


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


def capture(fn, reps=1):
    """fn captured in a CUDA graph (`reps` calls) after warm-up on a side stream."""
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for _ in range(3):
            fn()
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for _ in range(reps):
            fn()
    return g


def bench_decode(B, H, dtype, steps, reps):
    """One generated token for B sequences of H heads, the [B, H, 64, 64] fp32
    state updated in place by the decode-step kernel, `steps` tokens per CUDA
    graph replay.  Its cost is the state: 32 KiB of HBM traffic per chain plus
    1 KiB of inputs and outputs, so the roofline is HBM bandwidth (the state is
    larger than L2 for B >= 512 at H = 16)."""
    inp = make_inputs(B, 1, H, seed=0)
    xs = [inp[n].to(dtype).cuda()[:, 0].contiguous() for n in NAMES]
    state = torch.randn(B, H, 64, 64, device="cuda")
    graph = capture(lambda: ops.wkv7_decode_step(*xs, state), steps)
    ms = time_ms(graph.replay, reps)
    us = ms * 1e3 / steps
    esz = torch.tensor([], dtype=dtype).element_size()
    chains = B * H
    # per chain: state read + written, six inputs read, y (dtype) and sa (fp32) written
    algo_bytes = chains * (2 * STATE_BYTES + 64 * (6 * esz + esz + 4))
    peak, kind = peaks()
    gbs = algo_bytes / us / 1e3
    return {"workload": f"decode: B={B} H={H} one token, {str(dtype).split('.')[-1]} inputs, "
                        f"fp32 state {chains * STATE_BYTES / 2**20:.0f} MiB",
            "metric": "decode_tokens_per_s", "value": round(B / us * 1e6),
            "us_per_step": round(us, 2),
            "roofline": {"bound": "hbm", "kernel": "step_fwd_kernel", "achieved": round(gbs, 1),
                         "peak": peak, "unit": "GB/s", "frac": round(gbs / peak, 3),
                         "peak_kind": kind, "bytes_per_step": algo_bytes},
            "timing": f"CUDA graph of {steps} steps, {reps} replays"}


def bench_prefill(B, T, H, reps):
    """A prompt of T tokens from a given start state to the final state (bf16),
    through the fused one-CTA-per-chain kernel and through the two-kernel path
    with a workspace."""
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
        us = 1e3 * time_ms(lambda: ops.wkv7_forward_state(*xs, state, inplace=True, work=work,
                                                          y=y, sa=sa), reps)
        out[name] = {"us": round(us, 1), "tokens_per_s": round(B * T / us * 1e6)}
    return out


def op_share_c4(fwd, bwd, steps, warmup):
    """Time `steps` train steps' worth of op calls (C4): per layer fwd(l) twice
    (forward, recompute) then bwd(l), layers in order forward and reverse in
    backward as autograd runs them.  CUDA events on the current stream."""
    L = C4["layers"]

    def step():
        for l in range(L):
            fwd(l)
        for l in reversed(range(L)):
            fwd(l)  # the activation-checkpoint recompute of layer l
            bwd(l)

    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        step()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / steps
    tokens = C4["B"] * C4["T"]
    return {"ms_per_step": ms, "tokens_per_s": tokens / (ms / 1e3)}


def c4_inputs(dt, dev):
    B, T, H, N = C4["B"], C4["T"], C4["H"], C4["N"]
    layers = []
    for l in range(C4["layers"]):
        inp = make_inputs(B, T, H, N, seed=100 + l, dtype=dt)
        layers.append(([inp[n].to(dev) for n in NAMES], inp["dy"].to(dev)))
    return layers


def run_train_step_c4(args):
    """Our op on the call pattern of one 0.4B CaMoE train step (C4), bf16
    through the chunked kernels and fp32 through the scan."""
    dev = torch.device("cuda", 0)
    B, T, H, N = C4["B"], C4["T"], C4["H"], C4["N"]
    for dt in (torch.bfloat16, torch.float32):
        layers = c4_inputs(dt, dev)
        state = []
        for xs, dy in layers:
            y, sa, ck = ops.wkv7_forward(*xs)
            g = ops.wkv7_backward(*xs, dy, sa, ck)
            state.append((y, sa, ck, g))
        work = torch.empty(max(ops.work_bytes(B, T, H, dt), 16), dtype=torch.uint8, device=dev)

        def fwd(l):
            xs, _ = layers[l]
            y, sa, ck, _ = state[l]
            ops.wkv7_forward(*xs, y=y, sa=sa, ckpt=ck)

        def bwd(l):
            xs, dy = layers[l]
            _, sa, ck, g = state[l]
            # the dsa the layer's ln_sa sends back is an input of the backward
            ops.wkv7_backward(*xs, dy, sa, ck, grads=g, work=work)

        r = op_share_c4(fwd, bwd, max(args.steps // 4, 3), 2)
        print(json.dumps({
            "workload": f"train_step_c4 op share: {C4['layers']} layers x (forward, recompute "
                        f"forward, backward with dsa), B={B} T={T} H={H} N={N}, "
                        f"{str(dt).split('.')[-1]} inputs",
            "metric": "camoe_c4_op_tokens_per_s", "impl": "ours",
            "algo": "chunked" if dt == torch.bfloat16 else "scan", **r}), flush=True)
        del layers, state, work
        torch.cuda.empty_cache()


def reference_train_step_c4(args):
    """The reference's own CUDA op (oracle/_ref) on the same call pattern (C4);
    its backward takes no dsa (camoe/cuda/rwkv7_clampw.cpp:19-23)."""
    import oracle

    dev = torch.device("cuda", 0)
    B, T, H, N = C4["B"], C4["T"], C4["H"], C4["N"]
    for fp32 in (False, True):
        dt = torch.float32 if fp32 else torch.bfloat16
        if not oracle.RefOp.available(fp32=fp32):
            print(json.dumps({"workload": "train_step_c4 op share", "impl": "reference",
                              "unavailable": "oracle/_ref not built"}), flush=True)
            continue
        op = oracle.RefOp(fp32=fp32)
        layers = c4_inputs(dt, dev)
        state = []
        for xs, _ in layers:
            state.append((torch.empty_like(xs[0]),
                          torch.empty(B, H, T // 16, N, N, dtype=torch.float32, device=dev),
                          torch.empty(xs[0].shape, dtype=torch.float32, device=dev),
                          [torch.empty_like(xs[0]) for _ in range(6)]))

        def fwd(l):
            y, s, sa, _ = state[l]
            op.forward(*layers[l][0], y, s, sa)

        def bwd(l):
            y, s, sa, g = state[l]
            op.backward(*layers[l][0], layers[l][1], s, sa, *g)

        # it launches on the legacy default stream, which the events also use
        r = op_share_c4(fwd, bwd, 2, 1)
        print(json.dumps({
            "workload": f"train_step_c4 op share: {C4['layers']} layers x (forward, recompute "
                        f"forward, backward), B={B} T={T} H={H} N={N}, "
                        f"{str(dt).split('.')[-1]} inputs",
            "metric": "camoe_c4_op_tokens_per_s", "impl": "reference",
            "source": "camoe/cuda/rwkv7_clampw.cu built from the reference's sources", **r}),
            flush=True)
        del layers, state
        torch.cuda.empty_cache()


def run_decode(args):
    for dt in (torch.bfloat16, torch.float32):
        print(json.dumps(bench_decode(1024, 16, dt, 50, 10)), flush=True)
    for B, T in ((4, 4096), (8, 1024), (2, 16384)):
        print(json.dumps(bench_prefill(B, T, 16, 10)), flush=True)


def eager_timemix(m, x, v_first):
    """The reference's time-mix forward, op for op (camoe/backbone.py:311-371),
    with the module's parameters and this package's op behind RUN_CUDA_RWKV7:
    the unfused baseline of the fused layer."""
    import torch.nn.functional as F

    from camoe_b200 import backbone

    B, T, C = x.shape
    H = m.n_head
    with torch.autocast("cuda", dtype=torch.bfloat16):
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


def run_timemix(args, B=8, T=1024, C=1024, layer=2, steps=20):
    """The fused time mix: one layer forward + backward (dispatched eagerly, and
    replayed from a CUDA graph) against the same layer op by op; one decode token
    with the state carried against re-running the layer over the context (what
    the reference's generation loop does per token, eval.py:212); and each fused
    kernel, and the tcgen05 LoRA weight gradient per rank, alone (L2 flushed
    before each launch) against HBM bandwidth."""
    import ctypes

    from camoe_b200 import _lib, backbone, timemix

    BF = torch.bfloat16
    backbone.init_rwkv7_cuda()
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

    fused = time_ms(lambda: step(lambda mm, xx, vv: mm(xx, vv)), steps)
    eager = time_ms(lambda: step(eager_timemix), steps)
    fused_g = time_ms(capture(lambda: step(lambda mm, xx, vv: mm(xx, vv))).replay, steps)
    eager_g = time_ms(capture(lambda: step(eager_timemix)).replay, steps)
    print(json.dumps({
        "workload": f"time mix layer {layer}: B={B} T={T} C={C} H={C // 64}, bf16, fwd+bwd",
        "metric": "timemix_layer_tokens_per_s",
        "fused": {"ms": round(fused, 3), "tokens_per_s": round(B * T / fused * 1e3),
                  "graph_ms": round(fused_g, 3)},
        "eager": {"ms": round(eager, 3), "tokens_per_s": round(B * T / eager * 1e3),
                  "graph_ms": round(eager_g, 3)},
        "speedup": round(eager / fused, 2), "speedup_graph": round(eager_g / fused_g, 2)}),
        flush=True)

    # one generated token, B=64 sequences, context T
    Bd = 64
    xd = torch.randn(Bd, T, C, device="cuda", dtype=BF)
    vd = None if layer == 0 else torch.randn(Bd, T, C, device="cuda", dtype=BF)
    with torch.no_grad():
        _, _, _, state = m.forward_state(xd, vd)
    x1 = xd[:, -1:].contiguous()
    v1 = None if vd is None else vd[:, -1:].contiguous()
    holder = {"s": state}

    def token():
        _, _, _, holder["s"] = m.forward_state(x1, v1, holder["s"])

    with torch.no_grad():
        tok_ms = time_ms(token, 5 * steps)
        tok_g = time_ms(capture(token).replay, 5 * steps)
        full_ms = time_ms(lambda: m(xd, vd), max(3, steps // 2))
    print(json.dumps({
        "workload": f"time mix layer {layer} decode: B={Bd} context {T} C={C}, bf16, one token",
        "metric": "decode_ms_per_token",
        "stateful": {"ms": round(tok_ms, 4), "graph_ms": round(tok_g, 4)},
        "rerun_context": {"ms": round(full_ms, 3)},
        "speedup_graph": round(full_ms / tok_g, 1)}), flush=True)

    # each fused kernel alone
    L = _lib.lib()
    n = B * T * C
    st = torch.cuda.current_stream().cuda_stream
    P = (lambda t: None if t is None else ctypes.c_void_p(t.data_ptr()))
    bf = (lambda: torch.randn(B, T, C, device="cuda", dtype=BF))
    f32 = (lambda: torch.randn(B, T, C, device="cuda"))
    vec = (lambda k: torch.rand(k, C, device="cuda"))
    nw = int(L.camoe_tm_work_bytes(B, T, C))
    work = torch.empty(nw, dtype=torch.uint8, device="cuda")
    peak, kind = peaks()
    xk, six, dsix = bf(), [bf() for _ in range(6)], [bf() for _ in range(6)]
    arr = (lambda ts: (ctypes.c_void_p * 6)(*[t.data_ptr() for t in ts]))
    ins = [bf() for _ in range(6)]           # wl, k, v, vl, al, v_first
    outs5 = [bf() for _ in range(5)]
    grads9 = [bf() for _ in range(9)]
    outs7 = [bf() for _ in range(7)]
    y, r, ko, vo, g, z, dz = (bf() for _ in range(7))
    sa, srep, dsrep, dsa = f32(), f32(), f32(), f32()
    dx = bf()
    par6, par5, par3, par2 = vec(6), vec(5), vec(3), vec(2)
    dpar = vec(6)  # parameter-gradient output (never an input)
    calls = {
        # name: (launch, algorithmic bytes per launch)
        "mix_fwd": (lambda: L.camoe_tm_mix_fwd(P(xk), 0, P(par6), arr(six), B, T, C, st), 14 * n),
        "mix_bwd": (lambda: L.camoe_tm_mix_bwd(P(xk), 0, P(par6), arr(dsix), P(dx), P(dpar),
                                               P(work), nw, B, T, C, st), 16 * n),
        "prep_fwd": (lambda: L.camoe_tm_prep_fwd(*[P(t) for t in ins], P(par5),
                                                 *[P(t) for t in outs5], B, T, C, st), 22 * n),
        "prep_bwd": (lambda: L.camoe_tm_prep_bwd(*[P(t) for t in grads9], None,
                                                 *[P(t) for t in ins], P(par5),
                                                 *[P(t) for t in outs7], P(dpar), P(work), nw,
                                                 B, T, C, st), 44 * n),
        "post_fwd": (lambda: L.camoe_tm_post_fwd(P(y), P(r), P(ko), P(vo), P(g), P(par3),
                                                 P(par3[1]), P(par3[2]), P(z), B, T, C, st),
                     12 * n),
        "post_bwd": (lambda: L.camoe_tm_post_bwd(P(dz), P(y), P(r), P(ko), P(vo), P(g), P(par3),
                                                 P(par3[1]), P(par3[2]), *[P(t) for t in outs5],
                                                 P(dpar), P(work), nw, B, T, C, st), 22 * n),
        "lnsa_fwd": (lambda: L.camoe_tm_lnsa_fwd(P(sa), P(par2[0]), P(par2[1]), P(srep), B, T,
                                                 C, st), 8 * n),
        "lnsa_bwd": (lambda: L.camoe_tm_lnsa_bwd(P(dsrep), P(sa), P(par2[0]), P(dsa), P(dpar),
                                                 P(work), nw, B, T, C, st), 12 * n),
    }
    # the LoRA weight gradients (tcgen05): bytes = the [R, C] and [R, D] bf16
    # operands read once and the fp32 [C, D] gradient written once, R = B T
    R = B * T
    lw = {}
    for D in sorted(set(timemix.lora_dims(C).values())):
        if D % 32 or not 64 <= D <= 256:
            continue
        lw[D] = (torch.randn(R, D, device="cuda", dtype=BF), torch.empty(C, D, device="cuda"),
                 int(L.camoe_tm_lora_work_bytes(R, C, D)))
        lw[D] += (torch.empty(lw[D][2], dtype=torch.uint8, device="cuda"),)
        calls[f"lora_wgrad_d{D}"] = (
            (lambda D=D: L.camoe_tm_lora_wgrad(P(xk), P(lw[D][0]), P(lw[D][1]), 1, P(lw[D][3]),
                                               lw[D][2], R, C, D, st)),
            R * C * 2 + R * D * 2 + C * D * 4)
    flush = torch.empty(64 << 20, dtype=torch.float32, device="cuda")  # 256 MB, twice the L2
    for name, (fn, nbytes) in calls.items():
        assert fn() == 0, name
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
              for _ in range(steps)]
        for e0, e1 in ev:
            flush.zero_()
            flush.sum()  # read back: L2 holds clean lines, no write-back during fn
            e0.record()
            fn()
            e1.record()
        torch.cuda.synchronize()
        us = sum(e0.elapsed_time(e1) for e0, e1 in ev) * 1e3 / steps
        gbs = nbytes / us / 1e3
        print(json.dumps({"kernel": name, "workload": f"B={B} T={T} C={C}", "us": round(us, 2),
                          "bytes": nbytes, "achieved_gbs": round(gbs, 1), "peak_gbs": peak,
                          "frac": round(gbs / peak, 3), "peak_kind": kind}), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--blocks", type=int, default=10, help="minimum timed blocks of --steps")
    ap.add_argument("--min-timed-s", type=float, default=1.0,
                    help="add blocks until the timed blocks cover this many seconds")
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="shard_b4_t4096",
                    choices=sorted(WORKLOADS) + list(OTHER_WORKLOADS))
    ap.add_argument("--algo", default="auto", choices=["auto", "scan", "chunked"])
    ap.add_argument("--dtype", default="bf16", choices=["bf16", "fp32"],
                    help="input dtype of the op workloads (fp32 runs the fp32-exact scan)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-trace", action="store_true",
                    help="skip the traced launch count (e.g. under ncu, which owns the counters)")
    ap.add_argument("--no-reference-gpu", action="store_true",
                    help="--impl reference: skip timing the reference's CUDA op")
    ap.add_argument("--split", action="store_true",
                    help="strong scaling: split the workload's chains over the ranks")
    ap.add_argument("--segments", default="auto",
                    help="with --split: segments per chain; with --share-heads: a list")
    ap.add_argument("--share-heads", type=int, default=0,
                    help="time one GPU's share (heads [0, H) of every sequence), one pass "
                         "against the time-segmented path")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)

    if args.workload in OTHER_WORKLOADS:
        torch.cuda.set_device(0)
        if args.workload == "train_step_c4" and args.impl == "reference":
            reference_train_step_c4(args)
            return
        {"decode_b1024_h16": run_decode, "timemix_b8_t1024_c1024": run_timemix,
         "train_step_c4": run_train_step_c4}[args.workload](args)
        return
    wl = WORKLOADS[args.workload]
    if args.impl == "reference":
        world = int(os.environ.get("WORLD_SIZE", "1"))
        rank = int(os.environ.get("RANK", "0"))
        run_reference(args, wl, world, rank)
        return

    world, rank, local = dist_setup(args)
    try:
        if args.share_heads:
            if args.segments == "auto":
                args.segments = "1,4,8,16"
            run_long_share(args, wl, torch.device("cuda", local))
        elif args.split:
            run_split(args, wl, world, rank, local)
        else:
            run_op(args, wl, world, rank, local)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
