"""GPU parity of the wind_backstepping decay variant (decay exp(-exp(w)),
camoe/cuda/wkv7_cuda.cu) against the CPU oracle and against the reference's
own wind op (built from its sources into oracle/_ref/ by oracle/Makefile).

Inputs come from camoe_b200.inputs.make_inputs(decay="wind"): w_in =
-softplus(-x) - 1/2, what RWKV-7's time mix feeds the op (camoe/backbone.py:326),
so every decay is at least exp(-e^{-1/2}) = 0.545.  Tolerance: norm-relative max
error per output tensor, 1e-4 for fp32 (scan) and 2e-2 for bf16, the oracle in
float64 on the same rounded inputs.
"""
import pytest
import torch

import oracle
from camoe_b200 import _lib, ops
from camoe_b200.inputs import make_inputs
from helpers import GRADS, TOL_BF16, TOL_FP32, nrel

pytestmark = pytest.mark.gpu

NAMES = ("r", "w", "k", "v", "a", "b")
PATHS = [(torch.float32, "scan"), (torch.bfloat16, "scan"), (torch.bfloat16, "chunked")]
PATH_IDS = ["fp32-scan", "bf16-scan", "bf16-chunked"]
SHAPES = {
    # name: (B, T, H, seed, w_mu, w_sigma)
    "small": (1, 64, 2, 0, 0.0, 1.0),
    "ragged_t40": (2, 40, 1, 2, 0.0, 1.0),
    "fast_decay": (1, 48, 2, 4, 3.0, 1.0),   # most decays near the 0.545 bound
    "slow_decay": (1, 256, 2, 1, -3.0, 1.0),
    "layer_b8_t1024": (8, 1024, 16, 0, 0.0, 1.0),
    "rows_split2_b4_t200": (4, 200, 16, 8, 0.0, 1.0),
}


@pytest.fixture(autouse=True)
def _no_device_timeouts():
    before = _lib.lib().camoe_wkv7_device_errors()
    yield
    assert _lib.lib().camoe_wkv7_device_errors() == before


def inputs(shape, with_dsa=False):
    B, T, H, seed, mu, sig = SHAPES[shape]
    return make_inputs(B, T, H, seed=seed, w_mu=mu, w_sigma=sig, decay="wind", with_dsa=with_dsa)


def run_op(inp, dtype, algo, with_dsa=False):
    xs = [inp[n].to(dtype).cuda() for n in NAMES]
    dy = inp["dy"].to(dtype).cuda()
    dsa = inp["dsa"].cuda() if with_dsa else None
    y, sa, ck = ops.wkv7_forward(*xs, algo=algo, decay="wind")
    grads = ops.wkv7_backward(*xs, dy, dsa, ck, algo=algo, decay="wind")
    torch.cuda.synchronize()
    return [t.float().cpu().numpy() for t in (y, sa) + tuple(grads)]


def compare(got, want, tol, label):
    errs = {n: nrel(g, w) for n, g, w in zip(("y", "sa") + GRADS, got, want)}
    bad = {n: e for n, e in errs.items() if not e < tol}
    assert not bad, f"{label}: errors above {tol}: {bad} (all: {errs})"


@pytest.mark.parametrize("dtype,algo", PATHS, ids=PATH_IDS)
@pytest.mark.parametrize("shape", list(SHAPES), ids=list(SHAPES))
def test_wind_matches_oracle(shape, dtype, algo):
    inp = inputs(shape, with_dsa=True)
    xs = [inp[n].to(dtype).float() for n in NAMES + ("dy",)]
    y, sa = oracle.fwd(*xs[:6], decay="wind")
    grads = oracle.bwd(*xs, inp["dsa"], decay="wind")
    got = run_op(inp, dtype, algo, with_dsa=True)
    compare(got, [y, sa, *grads], TOL_FP32 if dtype == torch.float32 else TOL_BF16,
            f"{shape} {algo}")


@pytest.mark.parametrize("fp32", [False, True], ids=["bf16", "fp32"])
@pytest.mark.parametrize("shape", ["small", "fast_decay", "layer_b8_t1024"])
def test_wind_matches_reference_cuda_op(shape, fp32):
    """Against the reference's own wind_backstepping op on the same inputs."""
    if not oracle.RefOp.available(fp32, decay="wind"):
        pytest.skip("reference wind op not built (make -C oracle ref)")
    ref = oracle.RefOp(fp32, decay="wind")
    inp = inputs(shape)
    B, T, H = inp["r"].shape[:3]
    dtype = torch.float32 if fp32 else torch.bfloat16
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
    for algo in (["scan"] if fp32 else ["scan", "chunked"]):
        got = run_op(inp, dtype, algo)
        # the reference reverses its state through 1/w (wkv7_cuda.cu:91-94), so
        # its own fp32 error exceeds the fp32 bar; compare fp32 at 1e-3
        compare(got, want, 1e-3 if fp32 else TOL_BF16, f"ref-{algo}")


def test_wind_torch_ops_and_autograd_function():
    """torch.ops.wind_backstepping.forward/backward (reference argument order,
    camoe/cuda/wkv7_op.cpp:18-21) and the WindBackstepping autograd Function
    give the ops-level results bit for bit."""
    from camoe_b200 import backbone
    backbone.init_rwkv7_cuda()
    inp = inputs("small")
    B, T, H = inp["r"].shape[:3]
    r, w, k, v, a, b = (inp[n].to(torch.bfloat16).cuda() for n in NAMES)
    dy = inp["dy"].to(torch.bfloat16).cuda()
    y0, sa0, ck = ops.wkv7_forward(r, w, k, v, a, b, decay="wind")
    g0 = ops.wkv7_backward(r, w, k, v, a, b, dy, None, ck, decay="wind")
    y, sa = torch.empty_like(r), torch.empty(r.shape, device="cuda")
    s = torch.empty(B, H, T // 16, 64, 64, device="cuda")
    torch.ops.wind_backstepping.forward(w, r, k, v, a, b, y, s, sa)
    dw, dq, dk, dv, dz, da = (torch.empty_like(r) for _ in range(6))
    torch.ops.wind_backstepping.backward(w, r, k, v, a, b, dy, s, sa, dw, dq, dk, dv, dz, da)
    torch.cuda.synchronize()
    assert torch.equal(y, y0) and torch.equal(sa, sa0)
    for got, want in zip((dq, dw, dk, dv, dz, da), g0):
        assert torch.equal(got, want)
    leaves = [x.clone().requires_grad_(True) for x in (w, r, k, v, a, b)]
    ya, saa = backbone.WindBackstepping.apply(*leaves)
    ya.backward(dy)
    assert torch.equal(ya.detach(), y0)
    for leaf, want in zip(leaves, (g0[1], g0[0], g0[2], g0[3], g0[4], g0[5])):
        assert torch.equal(leaf.grad, want)
