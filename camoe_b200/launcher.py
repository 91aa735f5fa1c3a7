"""One-process-per-GPU sharding of the WKV-7 op.

The op is independent per (batch, head) chain, so a multi-GPU job is a
partition of the B x H chains with no exchange on the data path:

* batch shards when B is a multiple of the world size (contiguous batch
  slices, every head): e.g. B=32 over 8 GPUs -> 4 sequences per GPU;
* (batch, head-group) shards when the world size is a multiple of B and H
  divides evenly: e.g. B=2, H=32 over 8 GPUs -> 1 sequence x 8 heads per GPU,
  processed in place through the C ABI's head range (no copy).

``run`` spawns one process per rank (torch.multiprocessing, ``spawn``), sets
up a process group (NCCL on GPUs, gloo on CPU) with a short timeout, runs the
per-shard function and gathers every shard's outputs back to the caller on
the host (outside any timed region).  A rank that raises or does not finish
within ``timeout`` makes ``run`` raise instead of hanging.
"""
from __future__ import annotations

import datetime
import os
import queue
import shutil
import tempfile
import time
import traceback
from dataclasses import dataclass

import torch

NAMES = ("r", "w", "k", "v", "a", "b")
OUT_NAMES = ("y", "sa", "dr", "dw", "dk", "dv", "da", "db")


@dataclass(frozen=True)
class Shard:
    b0: int
    b1: int  # batch range [b0, b1)
    h0: int
    h1: int  # head range [h0, h1)

    @property
    def chains(self) -> int:
        return (self.b1 - self.b0) * (self.h1 - self.h0)


def plan_shards(B: int, H: int, world: int) -> list[Shard]:
    """Partition B x H chains over `world` ranks (equal sizes, no collective)."""
    if world < 1:
        raise ValueError("world must be >= 1")
    if B % world == 0:
        per = B // world
        return [Shard(r * per, (r + 1) * per, 0, H) for r in range(world)]
    if world % B == 0 and H % (world // B) == 0:
        groups = world // B
        hp = H // groups
        return [Shard(r // groups, r // groups + 1, (r % groups) * hp, (r % groups + 1) * hp)
                for r in range(world)]
    raise ValueError(f"cannot split B={B} x H={H} chains evenly over {world} ranks")


def cuda_shard_fn(inputs: dict, shard: Shard, device: torch.device, segments="auto") -> dict:
    """Forward + backward of one shard on `device` through the C ABI (head range
    in place).  A shard of few long chains (bf16) runs time-segmented
    (camoe_b200.segmented): ``segments`` "auto" picks the count from the
    chain count, the length and the SM count; an int forces it."""
    from . import ops, segmented

    sl = slice(shard.b0, shard.b1)
    xs = [inputs[n][sl].to(device) for n in NAMES]
    dy = inputs["dy"][sl].to(device)
    dsa = inputs["dsa"][sl].to(device) if inputs.get("dsa") is not None else None
    hc = shard.h1 - shard.h0
    T = xs[0].shape[1]
    P = segments
    if segments == "auto":
        P = 1
        if xs[0].dtype == torch.bfloat16:
            sms = torch.cuda.get_device_properties(device).multi_processor_count
            P = segmented.auto_segments(shard.chains, T, sms)
    if P > 1:
        y = torch.zeros_like(xs[0])
        sa = torch.zeros(xs[0].shape, dtype=torch.float32, device=device)
        grads = tuple(torch.zeros_like(xs[0]) for _ in range(6))
        _, _, saved = segmented.wkv7_forward_segmented(*xs, P, h0=shard.h0, h_count=hc, y=y,
                                                       sa=sa)
        segmented.wkv7_backward_segmented(saved, dy, dsa, grads=grads)
    else:
        y, sa, ck = ops.wkv7_forward(*xs, h0=shard.h0, h_count=hc, zero_rest=True)
        grads = ops.wkv7_backward(*xs, dy, dsa, ck, h0=shard.h0, h_count=hc, zero_rest=True)
    torch.cuda.synchronize(device)
    hs = slice(shard.h0, shard.h1)
    out = {"y": y, "sa": sa}
    out.update(dict(zip(OUT_NAMES[2:], grads)))
    return {n: t[:, :, hs].cpu() for n, t in out.items()}


def _to_wire(t: torch.Tensor):
    """(bf16 flag, numpy array) of a CPU tensor; bf16 travels as its int16 bit pattern."""
    t = t.contiguous()
    if t.dtype == torch.bfloat16:
        return True, t.view(torch.int16).numpy()
    return False, t.numpy()


def _from_wire(is_bf16: bool, a) -> torch.Tensor:
    t = torch.from_numpy(a)
    return t.view(torch.bfloat16) if is_bf16 else t


def _worker(rank, world, init_method, backend, inputs, shards, shard_fn, results, timeout_s):
    import torch.distributed as dist
    try:
        os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
        if backend == "nccl":
            torch.cuda.set_device(rank)
            device = torch.device("cuda", rank)
        else:
            device = torch.device("cpu")
            # one node: gloo on the loopback device, so that its choice of
            # interface does not depend on the host name resolving
            os.environ.setdefault("GLOO_SOCKET_IFNAME", "lo")
        dist.init_process_group(backend, init_method=init_method, rank=rank,
                                world_size=world, timeout=datetime.timedelta(seconds=timeout_s))
        out = shard_fn(inputs, shards[rank], device)
        dist.barrier()  # every rank finished its shard
        # plain arrays, pickled by value: a tensor would travel as a shared-memory
        # handle that the parent can no longer open once this process has exited
        results.put((rank, "ok", {n: _to_wire(t) for n, t in out.items()}))
        dist.destroy_process_group()
    except Exception:  # reported to the parent, which raises
        results.put((rank, "error", traceback.format_exc()))


def run(inputs: dict, world: int, backend: str = "nccl", shard_fn=None,
        timeout: float = 120.0) -> dict:
    """Run `shard_fn` (default: the CUDA op) on `world` ranks and gather the outputs.

    `inputs` holds CPU tensors r, w, k, v, a, b, dy [, dsa] of shape [B, T, H, 64].
    Returns dict of full [B, T, H, 64] CPU tensors y, sa, dr, dw, dk, dv, da, db.
    """
    import torch.multiprocessing as mp

    B, T, H, N = inputs["r"].shape
    shards = plan_shards(B, H, world)
    fn = shard_fn or cuda_shard_fn
    ctx = mp.get_context("spawn")
    results = ctx.Queue()
    # rendezvous through a file in a private directory: no port to race for
    rdv_dir = tempfile.mkdtemp(prefix="camoe_rdv_")
    init_method = "file://" + os.path.join(rdv_dir, "store")
    procs = [ctx.Process(target=_worker, args=(r, world, init_method, backend, inputs, shards,
                                                 fn, results, timeout), daemon=True)
             for r in range(world)]
    for p in procs:
        p.start()
    got, errors = {}, []
    # one deadline for the whole job, not one per result
    limit = timeout + 10.0
    deadline = time.monotonic() + limit
    try:
        while len(got) + len(errors) < world:
            try:
                left = max(deadline - time.monotonic(), 0.0)
                rank, status, payload = results.get(timeout=left)
            except queue.Empty:
                raise TimeoutError(f"ranks {sorted(set(range(world)) - set(got))} did not finish "
                                   f"within {limit:.0f} s")
            if status == "ok":
                got[rank] = {n: _from_wire(*x) for n, x in payload.items()}
            else:
                errors.append((rank, payload))
                break
    finally:
        for p in procs:
            p.join(timeout=5.0)
            if p.is_alive():
                p.kill()
                p.join(timeout=5.0)
        shutil.rmtree(rdv_dir, ignore_errors=True)
    if errors:
        rank, tb = errors[0]
        raise RuntimeError(f"rank {rank} failed:\n{tb}")
    full = {n: torch.zeros(B, T, H, N, dtype=got[0][n].dtype) for n in OUT_NAMES}
    for rank, sh in enumerate(shards):
        for n in OUT_NAMES:
            full[n][sh.b0:sh.b1, :, sh.h0:sh.h1] = got[rank][n]
    return full
