"""The one-process-per-GPU launcher on the real op: sharded results must equal
the single-process results bit for bit (chains are independent)."""
import numpy as np
import pytest
import torch

from camoe_b200 import launcher, ops
from camoe_b200.inputs import make_inputs

pytestmark = pytest.mark.gpu
NAMES = ("r", "w", "k", "v", "a", "b")


@pytest.mark.parametrize("B,H", [(2, 4), (1, 4)], ids=["batch-shards", "head-groups"])
def test_launcher_matches_single_process(B, H):
    world = min(2, torch.cuda.device_count())
    if B % world and world % B:
        pytest.skip("shape does not split over the available GPUs")
    inp = make_inputs(B, 64, H, 64, seed=9, with_dsa=True, dtype=torch.bfloat16)
    inp["dsa"] = inp["dsa"].float()
    full = launcher.run(inp, world=world, backend="nccl", timeout=120)
    xs = [inp[n].cuda() for n in NAMES]
    y, sa, ck = ops.wkv7_forward(*xs)
    g = ops.wkv7_backward(*xs, inp["dy"].cuda(), inp["dsa"].cuda(), ck)
    torch.cuda.synchronize()
    for n, want in zip(launcher.OUT_NAMES, (y, sa) + tuple(g)):
        np.testing.assert_array_equal(full[n].float().numpy(), want.float().cpu().numpy(), err_msg=n)


def test_segmented_shard_matches_one_pass():
    """cuda_shard_fn with a forced segment count on a head-group shard: the
    same outputs as the one-pass shard within the bf16 tolerance."""
    from helpers import TOL_BF16, nrel
    inp = make_inputs(1, 512, 4, 64, seed=10, with_dsa=True, dtype=torch.bfloat16)
    inp["dsa"] = inp["dsa"].float()
    shard = launcher.Shard(0, 1, 1, 3)
    dev = torch.device("cuda", 0)
    one = launcher.cuda_shard_fn(inp, shard, dev, segments=1)
    seg = launcher.cuda_shard_fn(inp, shard, dev, segments=4)
    for n in launcher.OUT_NAMES:
        assert nrel(seg[n].float().numpy(), one[n].float().numpy()) < TOL_BF16, n
