"""GPU parity of the WKV-7 op against the CPU oracle and the reference's own
CUDA op (built from the reference's sources into oracle/_ref/).

Tolerance: norm-relative max error max|x - ref| / max|ref| per output tensor,
1e-4 for fp32 inputs (fp32-exact scan) and 2e-2 for bf16, the oracle being
evaluated in float64 on the same (bf16-rounded) inputs.
"""
import numpy as np
import pytest
import torch

import oracle
from camoe_b200 import ops
from camoe_b200.inputs import make_inputs
from helpers import GRADS, TOL_BF16, TOL_FP32, nrel

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _no_device_timeouts():
    """Every bounded device-side wait must have completed (no timed-out kernel)."""
    from camoe_b200 import _lib
    before = _lib.lib().camoe_wkv7_device_errors()
    yield
    assert _lib.lib().camoe_wkv7_device_errors() == before

NAMES = ("r", "w", "k", "v", "a", "b")
# (dtype, algo) pairs of the product path
PATHS = [(torch.float32, "scan"), (torch.bfloat16, "scan"), (torch.bfloat16, "chunked")]
PATH_IDS = ["fp32-scan", "bf16-scan", "bf16-chunked"]

SHAPES = {
    # name: (B, T, H, seed, w_mu, w_sigma)
    "small": (1, 64, 2, 0, 0.0, 1.0),
    "ragged_t40": (2, 40, 1, 2, 0.0, 1.0),
    "single_chunk": (3, 16, 1, 3, 0.0, 1.0),
    "t17": (1, 17, 2, 6, 0.0, 1.0),
    "t5": (2, 5, 3, 7, 0.0, 1.0),
    "extreme_decay": (1, 48, 1, 4, 0.0, 6.0),
    "slow_decay": (1, 256, 2, 1, 2.0, 0.5),
    "layer_b8_t1024": (8, 1024, 16, 0, 0.0, 1.0),
    # 64 chains: the chunked backward splits each chain's state rows over two CTAs
    "rows_split2_b4_t200": (4, 200, 16, 8, 0.0, 1.0),
}


def tol_for(dtype):
    return TOL_FP32 if dtype == torch.float32 else TOL_BF16


def run_op(inp, dtype, algo, with_dsa=False, h0=0, hc=None):
    xs = {n: inp[n].to(dtype).cuda() for n in NAMES + ("dy",)}
    dsa = inp["dsa"].cuda() if with_dsa else None
    y, sa, ck = ops.wkv7_forward(*[xs[n] for n in NAMES], algo=algo, h0=h0, h_count=hc,
                                 zero_rest=True)
    grads = ops.wkv7_backward(*[xs[n] for n in NAMES], xs["dy"], dsa, ck, algo=algo, h0=h0,
                              h_count=hc, zero_rest=True)
    torch.cuda.synchronize()
    return [t.float().cpu().numpy() for t in (y, sa) + tuple(grads)]


def oracle_outputs(inp, dtype, with_dsa=False):
    xs = [inp[n].to(dtype).float() for n in NAMES + ("dy",)]
    y, sa = oracle.fwd(*xs[:6])
    grads = oracle.bwd(*xs, inp["dsa"] if with_dsa else None)
    return [y, sa, *grads]


def compare(got, want, tol, label=""):
    errs = {n: nrel(g, w) for n, g, w in zip(("y", "sa") + GRADS, got, want)}
    bad = {n: e for n, e in errs.items() if not e < tol}
    assert not bad, f"{label} errors above {tol}: {bad} (all: {errs})"
    return errs


@pytest.mark.parametrize("dtype,algo", PATHS, ids=PATH_IDS)
@pytest.mark.parametrize("shape", list(SHAPES), ids=list(SHAPES))
def test_matches_oracle(shape, dtype, algo):
    B, T, H, seed, mu, sig = SHAPES[shape]
    inp = make_inputs(B, T, H, 64, seed=seed, w_mu=mu, w_sigma=sig)
    compare(run_op(inp, dtype, algo), oracle_outputs(inp, dtype), tol_for(dtype), shape)


@pytest.mark.parametrize("dtype,algo", PATHS, ids=PATH_IDS)
@pytest.mark.parametrize("B,T,H", [(2, 96, 3), (4, 80, 16), (8, 67, 16)],
                         ids=["rows_split4", "rows_split2", "rows_whole"])
def test_external_sa_gradient(dtype, algo, B, T, H):
    inp = make_inputs(B, T, H, 64, seed=21, with_dsa=True)
    compare(run_op(inp, dtype, algo, with_dsa=True), oracle_outputs(inp, dtype, True),
            tol_for(dtype), "dsa")


@pytest.mark.parametrize("dtype,algo", PATHS, ids=PATH_IDS)
def test_head_range_matches_full_run_bitwise(dtype, algo):
    inp = make_inputs(2, 64, 8, 64, seed=5, with_dsa=True)
    full = run_op(inp, dtype, algo, with_dsa=True)
    part = run_op(inp, dtype, algo, with_dsa=True, h0=3, hc=4)
    for f, p in zip(full, part):
        np.testing.assert_array_equal(p[:, :, 3:7], f[:, :, 3:7])
        assert not np.any(p[:, :, :3]) and not np.any(p[:, :, 7:])


@pytest.mark.parametrize("dtype,algo", PATHS, ids=PATH_IDS)
def test_deterministic(dtype, algo):
    inp = make_inputs(2, 128, 4, 64, seed=8, with_dsa=True)
    a = run_op(inp, dtype, algo, with_dsa=True)
    b = run_op(inp, dtype, algo, with_dsa=True)
    for x, y in zip(a, b):
        np.testing.assert_array_equal(x, y)


@pytest.mark.parametrize("dtype,algo", PATHS, ids=PATH_IDS)
def test_long_sequence(dtype, algo):
    # a long chain: the state is carried across 512 chunks
    inp = make_inputs(1, 8192, 2, 64, seed=13, w_mu=2.0, w_sigma=0.5)
    compare(run_op(inp, dtype, algo), oracle_outputs(inp, dtype), tol_for(dtype), "long")


@pytest.mark.parametrize("fp32", [False, True], ids=["bf16", "fp32"])
@pytest.mark.parametrize("shape", ["small", "extreme_decay", "layer_b8_t1024"])
def test_matches_reference_cuda_op(shape, fp32):
    """Against the reference's own op (camoe/cuda/rwkv7_clampw.cu) on the same inputs."""
    if not oracle.RefOp.available(fp32):
        pytest.skip("reference op not built (make -C oracle ref)")
    ref = oracle.RefOp(fp32)
    B, T, H, seed, mu, sig = SHAPES[shape]
    dtype = torch.float32 if fp32 else torch.bfloat16
    inp = make_inputs(B, T, H, 64, seed=seed, w_mu=mu, w_sigma=sig)
    xs = [inp[n].to(dtype).cuda() for n in NAMES]
    dy = inp["dy"].to(dtype).cuda()
    y = torch.empty_like(xs[0])
    s = torch.empty(B, H, T // 16, 64, 64, dtype=torch.float32, device="cuda")
    sa = torch.empty(B, T, H, 64, dtype=torch.float32, device="cuda")
    grads = [torch.empty_like(xs[0]) for _ in range(6)]
    torch.cuda.synchronize()
    ref.forward(*xs, y, s, sa)
    ref.backward(*xs, dy, s, sa, *grads)
    torch.cuda.synchronize()
    want = [t.float().cpu().numpy() for t in [y, sa] + grads]
    algos = ["scan"] if fp32 else ["scan", "chunked"]
    for algo in algos:
        got = run_op(inp, dtype, algo)
        # the reference reverses its state through 1/w, so its own fp32 error
        # exceeds the fp32 bar at strong decay; compare fp32 at 1e-3
        compare(got, want, 1e-3 if fp32 else TOL_BF16, f"ref-{algo}")
