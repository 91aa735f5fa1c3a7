"""Multi-rank sharding of the op, on CPU with gloo (world size 2).

The shard function here is the CPU oracle on the shard's chains, so the test
checks the partition, the per-rank dispatch and the gather: the gathered
result must equal the single-process oracle result bit for bit (chains are
independent).  Failures of a rank are made on the host (an exception, a rank
that stalls) and must surface as errors, never as a hang.
"""
import time

import numpy as np
import pytest
import torch

import oracle
from camoe_b200 import launcher
from camoe_b200.inputs import make_inputs

NAMES = ("r", "w", "k", "v", "a", "b")


def oracle_shard(inputs, shard, device):
    sl, hs = slice(shard.b0, shard.b1), slice(shard.h0, shard.h1)
    xs = [inputs[n][sl, :, hs].contiguous() for n in NAMES]
    dsa = inputs.get("dsa")
    y, sa = oracle.fwd(*xs, threads=1)
    g = oracle.bwd(*xs, inputs["dy"][sl, :, hs], None if dsa is None else dsa[sl, :, hs],
                   threads=1)
    return {n: torch.from_numpy(v) for n, v in zip(launcher.OUT_NAMES, (y, sa) + g)}


def failing_shard(inputs, shard, device):
    if shard.b0 == 1:
        raise RuntimeError("injected failure on the second rank")
    return oracle_shard(inputs, shard, device)


def stalling_shard(inputs, shard, device):
    if shard.b0 == 1:
        time.sleep(60)
    return oracle_shard(inputs, shard, device)


def test_plan_shards():
    assert launcher.plan_shards(32, 16, 8) == [launcher.Shard(4 * r, 4 * r + 4, 0, 16) for r in range(8)]
    sh = launcher.plan_shards(2, 32, 8)
    assert [(s.b0, s.h0, s.h1) for s in sh] == [(r // 4, (r % 4) * 8, (r % 4) * 8 + 8) for r in range(8)]
    assert sum(s.chains for s in sh) == 64
    assert launcher.plan_shards(4, 16, 1) == [launcher.Shard(0, 4, 0, 16)]
    with pytest.raises(ValueError):
        launcher.plan_shards(3, 5, 2)


def test_auto_segments():
    from camoe_b200.segmented import auto_segments
    assert auto_segments(8, 65536, 148) == 8      # long-context share: 64 segments, 128 CTAs
    assert auto_segments(16, 65536, 148) == 4
    assert auto_segments(64, 65536, 148) == 1     # the chains fill the GPU already
    assert auto_segments(64, 4096, 148) == 1
    assert auto_segments(32, 65536, 148) == 1     # P = 2 would be slower than one pass
    assert auto_segments(8, 8192, 148) == 4       # segments of at least 2048 steps
    assert auto_segments(8, 4096, 148) == 1
    assert auto_segments(8, 2048, 148) == 1
    assert auto_segments(1, 65536 + 16, 148) == 1  # T must split into whole chunks


@pytest.mark.parametrize("B,H", [(2, 2), (1, 4)], ids=["batch-shards", "head-groups"])
def test_two_ranks_gloo_match_single_process(B, H):
    inp = make_inputs(B, 32, H, 64, seed=3, with_dsa=True)
    full = launcher.run(inp, world=2, backend="gloo", shard_fn=oracle_shard, timeout=60)
    y, sa = oracle.fwd(*[inp[n] for n in NAMES])
    g = oracle.bwd(*[inp[n] for n in NAMES], inp["dy"], inp["dsa"])
    for n, want in zip(launcher.OUT_NAMES, (y, sa) + g):
        np.testing.assert_array_equal(full[n].numpy(), want, err_msg=n)


def test_rank_failure_is_reported():
    inp = make_inputs(2, 16, 1, 64, seed=4)
    t0 = time.time()
    with pytest.raises(RuntimeError, match="rank 1 failed"):
        launcher.run(inp, world=2, backend="gloo", shard_fn=failing_shard, timeout=20)
    assert time.time() - t0 < 60


def test_stalled_rank_times_out():
    inp = make_inputs(2, 16, 1, 64, seed=5)
    t0 = time.time()
    with pytest.raises((TimeoutError, RuntimeError)):
        launcher.run(inp, world=2, backend="gloo", shard_fn=stalling_shard, timeout=5)
    assert time.time() - t0 < 60
