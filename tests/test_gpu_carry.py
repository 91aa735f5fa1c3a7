"""GPU parity of training across calls (camoe_wkv7_fwd_carry / _bwd_carry and
the RWKV7_ClampW_State autograd Function): a start state in, the final state
out, and the gradient of the start state out of the backward, against the CPU
oracle (fwd_state / bwd_state, whose torch-autograd check is in
test_oracle.py).

The reference has no carried state (its op starts from zero,
camoe/cuda/rwkv7_clampw.cu:28); with s0 = 0 and no final-state gradient the
carried calls are the reference's op, which test_zero_state_is_the_plain_op
checks.  Start states are real ones (the oracle's state after a random
prefix); the final-state gradients are Gaussian, scaled like the state.

Tolerance: norm-relative max error per output tensor, 1e-4 for fp32 inputs
(scan) and 2e-2 for bf16, the oracle in float64 on the same rounded inputs.
"""
import numpy as np
import pytest
import torch

import oracle
from camoe_b200 import _lib, backbone, ops
from camoe_b200.inputs import make_inputs
from helpers import GRADS, TOL_BF16, TOL_FP32, nrel

pytestmark = pytest.mark.gpu

NAMES = ("r", "w", "k", "v", "a", "b")
PATHS = [(torch.float32, "scan"), (torch.bfloat16, "scan"), (torch.bfloat16, "chunked")]
PATH_IDS = ["fp32-scan", "bf16-scan", "bf16-chunked"]
SHAPES = {
    # name: (B, T, H, seed): one chunk, the checkpoint's first stored chunk,
    # and many chunks over many chains
    "t16": (2, 16, 3, 1),
    "t48": (1, 48, 2, 2),
    "t256": (2, 256, 4, 3),
    "b8_t1024": (8, 1024, 16, 4),
}


@pytest.fixture(autouse=True)
def _no_device_timeouts():
    before = _lib.lib().camoe_wkv7_device_errors()
    yield
    assert _lib.lib().camoe_wkv7_device_errors() == before


def tol_for(dtype):
    return TOL_FP32 if dtype == torch.float32 else TOL_BF16


def states(B, H, seed):
    """A start state (the oracle's state after 48 random steps) and a final-
    state gradient, [B, H, 64, 64] float32."""
    pre = make_inputs(B, 48, H, seed=1000 + seed)
    s0 = oracle.fwd_state(*[pre[n] for n in NAMES])[2]
    dsT = np.random.default_rng(seed).standard_normal(s0.shape).astype(np.float32)
    return s0, dsT * float(np.abs(s0).max())


def run_carry(xs, dy, dsa, s0, dsT, algo):
    B, T, H, _ = xs[0].shape
    sT = torch.empty(B, H, 64, 64, device="cuda")
    y, sa, ck = ops.wkv7_forward(*xs, algo=algo, s0=s0, s_out=sT)
    ds0 = torch.empty(B, H, 64, 64, device="cuda")
    grads = ops.wkv7_backward(*xs, dy, dsa, ck, algo=algo, s0=s0, ds_out=dsT, ds0=ds0)
    torch.cuda.synchronize()
    return y, sa, sT, grads, ds0


@pytest.mark.parametrize("dtype,algo", PATHS, ids=PATH_IDS)
@pytest.mark.parametrize("shape", list(SHAPES), ids=list(SHAPES))
def test_carry_matches_oracle(shape, dtype, algo):
    B, T, H, seed = SHAPES[shape]
    inp = make_inputs(B, T, H, seed=seed, with_dsa=True)
    s0, dsT = states(B, H, seed)
    xs = [inp[n].to(dtype).cuda() for n in NAMES]
    y, sa, sT, grads, ds0 = run_carry(xs, inp["dy"].to(dtype).cuda(), inp["dsa"].cuda(),
                                      torch.from_numpy(s0).cuda(), torch.from_numpy(dsT).cuda(),
                                      algo)
    rx = [inp[n].to(dtype).float() for n in NAMES + ("dy",)]
    yw, saw, sw = oracle.fwd_state(*rx[:6], s0=s0)
    gw = oracle.bwd_state(*rx, inp["dsa"], s0=s0, dsT=dsT)
    got = [y, sa, sT] + list(grads) + [ds0]
    errs = {n: nrel(g.float().cpu().numpy(), w)
            for n, g, w in zip(("y", "sa", "sT") + GRADS + ("ds0",), got, [yw, saw, sw, *gw])}
    bad = {n: e for n, e in errs.items() if not e < tol_for(dtype)}
    assert not bad, f"{shape} {algo}: errors above {tol_for(dtype)}: {bad} (all: {errs})"


@pytest.mark.parametrize("dtype,algo", PATHS, ids=PATH_IDS)
def test_split_gradients_equal_one_pass(dtype, algo):
    """Forward [0, T1) -> state -> [T1, T); backward [T1, T) first, its ds0
    handed to [0, T1) as ds_out: the concatenated gradients equal the one-pass
    backward's (and the oracle's)."""
    B, T, H, T1 = 2, 160, 4, 64
    inp = make_inputs(B, T, H, seed=7)
    xs = [inp[n].to(dtype).cuda() for n in NAMES]
    dy = inp["dy"].to(dtype).cuda()
    first = [x[:, :T1].contiguous() for x in xs]
    second = [x[:, T1:].contiguous() for x in xs]
    s1 = torch.empty(B, H, 64, 64, device="cuda")
    ya, saa, cka = ops.wkv7_forward(*first, algo=algo, s_out=s1)
    yb, sab, ckb = ops.wkv7_forward(*second, algo=algo, s0=s1)
    ds1 = torch.empty_like(s1)
    gb = ops.wkv7_backward(*second, dy[:, T1:].contiguous(), None, ckb, algo=algo, s0=s1,
                           ds0=ds1)
    ga = ops.wkv7_backward(*first, dy[:, :T1].contiguous(), None, cka, algo=algo, ds_out=ds1)
    y, sa, ck = ops.wkv7_forward(*xs, algo=algo)
    g = ops.wkv7_backward(*xs, dy, None, ck, algo=algo)
    torch.cuda.synchronize()
    tol = tol_for(dtype)
    want = oracle.bwd(*[inp[n].to(dtype).float() for n in NAMES + ("dy",)], None)
    for n, a, b_, one, w in zip(GRADS, ga, gb, g, want):
        cat = torch.cat([a, b_], 1).float().cpu().numpy()
        assert nrel(cat, one.float().cpu().numpy()) < tol, n
        assert nrel(cat, w) < tol, n
    assert nrel(torch.cat([ya, yb], 1).float().cpu().numpy(), y.float().cpu().numpy()) < tol
    assert nrel(torch.cat([saa, sab], 1).cpu().numpy(), sa.cpu().numpy()) < tol


def test_ds0_only_skips_the_key_side():
    """ds0_only (chunked): ds0 and dv bit for bit those of the full carried
    backward; the other five gradient buffers are not written."""
    B, T, H = 2, 96, 3
    inp = make_inputs(B, T, H, seed=12)
    xs = [inp[n].to(torch.bfloat16).cuda() for n in NAMES]
    dy = inp["dy"].to(torch.bfloat16).cuda()
    s0, dsT = (torch.from_numpy(x).cuda() for x in states(B, H, 12))
    y, sa, ck = ops.wkv7_forward(*xs, algo="chunked", s0=s0)
    full0 = torch.empty_like(s0)
    g_full = ops.wkv7_backward(*xs, dy, None, ck, algo="chunked", s0=s0, ds_out=dsT, ds0=full0)
    only0 = torch.empty_like(s0)
    marks = tuple(torch.full_like(xs[0], 3.0) for _ in range(6))
    ops.wkv7_backward(*xs, dy, None, ck, algo="chunked", s0=s0, ds_out=dsT, ds0=only0,
                      grads=marks, ds0_only=True)
    torch.cuda.synchronize()
    assert torch.equal(only0, full0) and torch.equal(marks[3], g_full[3])
    for i in (0, 1, 2, 4, 5):
        assert (marks[i] == 3.0).all()


def test_value_pass_reuses_the_key_side_records():
    """camoe_wkv7_fwd_value over a checkpoint written by a forward with another
    v and start state gives bit for bit the outputs, final state and (through
    the backward) gradients of a full forward with its own v and start state."""
    B, T, H = 2, 96, 3
    inp = make_inputs(B, T, H, seed=13)
    xs = [inp[n].to(torch.bfloat16).cuda() for n in NAMES]
    dy = inp["dy"].to(torch.bfloat16).cuda()
    s0, _ = (torch.from_numpy(x).cuda() for x in states(B, H, 13))
    other = list(xs)
    other[3] = (xs[3].float() * -0.5).to(torch.bfloat16)
    s_a, s_b = torch.empty_like(s0), torch.empty_like(s0)
    y0, sa0, ck0 = ops.wkv7_forward(*xs, algo="chunked", s0=s0, s_out=s_a)
    _, _, ck1 = ops.wkv7_forward(*other, algo="chunked")
    y1, sa1 = ops.wkv7_forward_value(*xs, ck1, s0=s0, s_out=s_b)
    g0 = ops.wkv7_backward(*xs, dy, None, ck0, algo="chunked", s0=s0)
    g1 = ops.wkv7_backward(*xs, dy, None, ck1, algo="chunked", s0=s0)
    torch.cuda.synchronize()
    assert torch.equal(y0, y1) and torch.equal(sa0, sa1) and torch.equal(s_a, s_b)
    for a, b_ in zip(g0, g1):
        assert torch.equal(a, b_)


@pytest.mark.parametrize("dtype,algo", PATHS, ids=PATH_IDS)
def test_zero_state_is_the_plain_op(dtype, algo):
    """s0 = 0 and ds_out = 0 give the plain op's outputs and gradients."""
    B, T, H = 2, 64, 3
    inp = make_inputs(B, T, H, seed=8)
    xs = [inp[n].to(dtype).cuda() for n in NAMES]
    dy = inp["dy"].to(dtype).cuda()
    z = torch.zeros(B, H, 64, 64, device="cuda")
    y0, sa0, ck0 = ops.wkv7_forward(*xs, algo=algo)
    g0 = ops.wkv7_backward(*xs, dy, None, ck0, algo=algo)
    y1, sa1, sT, g1, ds0 = run_carry(xs, dy, None, z, z.clone(), algo)
    for a, b_ in zip((y0, sa0) + tuple(g0), (y1, sa1) + tuple(g1)):
        assert nrel(b_.float().cpu().numpy(), a.float().cpu().numpy()) < 1e-6
    assert torch.isfinite(sT).all() and torch.isfinite(ds0).all()


@pytest.mark.parametrize("dtype,algo", [(torch.float32, "scan"), (torch.bfloat16, "chunked")],
                         ids=["fp32-scan", "bf16-chunked"])
def test_autograd_function_over_pieces(dtype, algo, monkeypatch):
    """RWKV7_ClampW_State over three pieces with the state carried (not
    detached): one loss.backward() gives every input, and the first piece's
    start state, the gradient of one pass over the whole sequence."""
    monkeypatch.setattr(backbone, "_ALGO", algo)
    B, T, H, P = 2, 192, 2, 3
    inp = make_inputs(B, T, H, seed=9)
    s0np = states(B, H, 9)[0]
    leaves = [inp[n].to(dtype).cuda().requires_grad_(True) for n in NAMES]
    s0 = torch.from_numpy(s0np).cuda().requires_grad_(True)
    dy = inp["dy"].to(dtype).cuda()
    L = T // P
    state, loss = s0, 0
    for i in range(P):
        piece = [x[:, i * L:(i + 1) * L].contiguous() for x in leaves]
        y, sa, state = backbone.RWKV7_ClampW_State.apply(*piece, state)
        loss = loss + (y.float() * dy[:, i * L:(i + 1) * L].float()).sum()
    loss.backward()
    torch.cuda.synchronize()
    rx = [inp[n].to(dtype).float() for n in NAMES + ("dy",)]
    want = oracle.bwd_state(*rx, None, s0=s0np)
    tol = tol_for(dtype)
    for n, leaf, w in zip(GRADS + ("ds0",), leaves + [s0], want):
        assert nrel(leaf.grad.float().cpu().numpy(), w) < tol, n
