"""GPU parity of the time-segmented path (camoe_b200.segmented): every chain
cut into P pieces joined through their transitions.

* outputs and all six gradients against the CPU oracle (the reference's
  recurrence in one pass, float64) for P = 1, 2, 4, 8, on the bf16 chunked and
  fp32 scan paths, with a dsa input;
* a start state, a final-state gradient and the start-state gradient against
  the oracle's fwd_state / bwd_state;
* head ranges: only heads [h0, h0 + h_count) are written;
* the segment-chain kernel against torch.matmul in float64;
* the long-context shard (B=2 T=65536 H=32, heads 4..7, w_in ~ N(2, 0.5)) cut
  into 16 segments against the one-pass op on the same inputs;
* the autograd Function against RWKV7_ClampW.

Tolerance: norm-relative max error per output tensor, 1e-4 for fp32 inputs
(scan) and 2e-2 for bf16, as for the one-pass op.
"""
import numpy as np
import pytest
import torch

import oracle
from camoe_b200 import _lib, backbone, ops, segmented
from camoe_b200.inputs import make_inputs
from helpers import GRADS, TOL_BF16, TOL_FP32, nrel

pytestmark = pytest.mark.gpu

NAMES = ("r", "w", "k", "v", "a", "b")
PATHS = [(torch.bfloat16, "chunked"), (torch.float32, "scan")]
PATH_IDS = ["bf16-chunked", "fp32-scan"]


@pytest.fixture(autouse=True)
def _no_device_timeouts():
    before = _lib.lib().camoe_wkv7_device_errors()
    yield
    assert _lib.lib().camoe_wkv7_device_errors() == before


def tol_for(dtype):
    return TOL_FP32 if dtype == torch.float32 else TOL_BF16


def np_of(t):
    return t.float().cpu().numpy()


@pytest.mark.parametrize("dtype,algo", PATHS, ids=PATH_IDS)
@pytest.mark.parametrize("P", [1, 2, 4, 8])
def test_segmented_matches_oracle(P, dtype, algo):
    B, T, H = 2, 256, 3
    inp = make_inputs(B, T, H, seed=40 + P, with_dsa=True)
    xs = [inp[n].to(dtype).cuda() for n in NAMES]
    y, sa, saved = segmented.wkv7_forward_segmented(*xs, P, algo=algo)
    grads = segmented.wkv7_backward_segmented(saved, inp["dy"].to(dtype).cuda(),
                                              inp["dsa"].cuda())
    torch.cuda.synchronize()
    rx = [inp[n].to(dtype).float() for n in NAMES + ("dy",)]
    want = list(oracle.fwd(*rx[:6])) + list(oracle.bwd(*rx, inp["dsa"]))
    errs = {n: nrel(np_of(g), w) for n, g, w in zip(("y", "sa") + GRADS, [y, sa, *grads], want)}
    bad = {n: e for n, e in errs.items() if not e < tol_for(dtype)}
    assert not bad, f"P={P} {algo}: errors above {tol_for(dtype)}: {bad} (all: {errs})"


@pytest.mark.parametrize("dtype,algo", PATHS, ids=PATH_IDS)
def test_segmented_carries_states(dtype, algo):
    """s0 in, final state out, final-state gradient in, start-state gradient
    out, with 4 segments, against the oracle's stateful forward and backward."""
    B, T, H, P = 2, 128, 2, 4
    inp = make_inputs(B, T, H, seed=50)
    g = np.random.default_rng(50)
    pre = make_inputs(B, 48, H, seed=51)
    s0 = oracle.fwd_state(*[pre[n] for n in NAMES])[2]
    dsT = (g.standard_normal(s0.shape) * np.abs(s0).max()).astype(np.float32)
    xs = [inp[n].to(dtype).cuda() for n in NAMES]
    sT = torch.empty(B, H, 64, 64, device="cuda")
    ds0 = torch.empty(B, H, 64, 64, device="cuda")
    y, sa, saved = segmented.wkv7_forward_segmented(*xs, P, s0=torch.from_numpy(s0).cuda(),
                                                    s_out=sT, algo=algo)
    grads = segmented.wkv7_backward_segmented(saved, inp["dy"].to(dtype).cuda(),
                                              ds_out=torch.from_numpy(dsT).cuda(), ds0=ds0)
    torch.cuda.synchronize()
    rx = [inp[n].to(dtype).float() for n in NAMES + ("dy",)]
    yw, saw, sw = oracle.fwd_state(*rx[:6], s0=s0)
    gw = oracle.bwd_state(*rx, None, s0=s0, dsT=dsT)
    names = ("y", "sa", "sT") + GRADS + ("ds0",)
    errs = {n: nrel(np_of(a), w) for n, a, w in zip(names, [y, sa, sT, *grads, ds0],
                                                     [yw, saw, sw, *gw])}
    bad = {n: e for n, e in errs.items() if not e < tol_for(dtype)}
    assert not bad, f"{algo}: errors above {tol_for(dtype)}: {bad} (all: {errs})"


def test_segmented_head_range_writes_only_its_heads():
    B, T, H, h0, hc, P = 2, 128, 5, 1, 3, 4
    xs = [make_inputs(B, T, H, seed=60)[n].to(torch.bfloat16).cuda() for n in NAMES]
    dy = make_inputs(B, T, H, seed=61)["dy"].to(torch.bfloat16).cuda()
    y = torch.zeros_like(xs[0])
    sa = torch.zeros(xs[0].shape, device="cuda")
    grads = tuple(torch.zeros_like(xs[0]) for _ in range(6))
    _, _, saved = segmented.wkv7_forward_segmented(*xs, P, h0=h0, h_count=hc, y=y, sa=sa)
    segmented.wkv7_backward_segmented(saved, dy, grads=grads)
    yf, saf, ck = ops.wkv7_forward(*xs)
    gf = ops.wkv7_backward(*xs, dy, None, ck)
    torch.cuda.synchronize()
    hs = slice(h0, h0 + hc)
    for got, full in zip((y, sa) + grads, (yf, saf) + tuple(gf)):
        assert nrel(np_of(got[:, :, hs]), np_of(full[:, :, hs])) < TOL_BF16
        assert (got[:, :, :h0] == 0).all() and (got[:, :, h0 + hc:] == 0).all()


@pytest.mark.parametrize("backward", [False, True])
def test_seg_chain_kernel_against_matmul(backward):
    B, P, H, h0, hc = 3, 6, 4, 1, 2
    g = torch.Generator().manual_seed(7)
    states = torch.randn(B * P, H, 64, 64, generator=g)
    trans = torch.randn(B * P, H, 64, 64, generator=g) / 8
    local = torch.randn(B * P, H, 64, 64, generator=g)
    st = states.cuda()
    segmented.seg_chain(st, trans.cuda(), local.cuda(), B, P, h0, hc, backward)
    torch.cuda.synchronize()
    want = states.double().view(B, P, H, 64, 64).clone()
    A, C = trans.double().view(B, P, H, 64, 64), local.double().view(B, P, H, 64, 64)
    hs = slice(h0, h0 + hc)
    if backward:
        for gi in range(P - 1, 0, -1):
            want[:, gi - 1, hs] = want[:, gi, hs] @ A[:, gi, hs].transpose(-1, -2) + C[:, gi, hs]
    else:
        for gi in range(1, P):
            want[:, gi, hs] = want[:, gi - 1, hs] @ A[:, gi - 1, hs] + C[:, gi - 1, hs]
    got = st.cpu().double().view(B, P, H, 64, 64)
    assert torch.equal(got[:, :, :h0], want[:, :, :h0].float().double())
    assert torch.equal(got[:, :, h0 + hc:], want[:, :, h0 + hc:].float().double())
    assert float((got - want).abs().max() / want.abs().max()) < 1e-5


def test_segmented_long_context_shard_equals_one_pass():
    """One GPU's share of the long-context problem (B=2 T=65536 H=32, heads
    4..7), 16 segments of 4096 steps, against the one-pass chunked op."""
    B, T, H, h0, hc, P = 2, 65536, 32, 4, 4, 16
    gen = torch.Generator(device="cuda").manual_seed(3)
    shp = (B, T, H, 64)
    r, k, v, u, dy, w, kk = (torch.randn(shp, generator=gen, device="cuda") for _ in range(7))
    w = 2.0 + 0.5 * w
    kk = torch.nn.functional.normalize(kk, dim=-1, p=2.0)
    xs = [t.to(torch.bfloat16).contiguous() for t in (r, w, k, v, -kk, kk * torch.sigmoid(u))]
    dy = dy.to(torch.bfloat16)
    del r, k, v, u, w, kk
    y, sa, saved = segmented.wkv7_forward_segmented(*xs, P, h0=h0, h_count=hc)
    grads = segmented.wkv7_backward_segmented(saved, dy)
    del saved
    y1, sa1, ck = ops.wkv7_forward(*xs, h0=h0, h_count=hc)
    g1 = ops.wkv7_backward(*xs, dy, None, ck, h0=h0, h_count=hc)
    del ck
    torch.cuda.synchronize()
    hs = slice(h0, h0 + hc)
    for n, a, b_ in zip(("y", "sa") + GRADS, (y, sa) + tuple(grads), (y1, sa1) + tuple(g1)):
        a, b_ = a[:, :, hs].float(), b_[:, :, hs].float()
        e = float((a - b_).abs().max() / b_.abs().max())
        assert e < TOL_BF16, f"{n}: {e:.3g}"


def test_autograd_function_equals_rwkv7_clampw():
    B, T, H, P = 2, 192, 2, 3
    inp = make_inputs(B, T, H, seed=70)
    leaves = [[inp[n].to(torch.bfloat16).cuda().requires_grad_(True) for n in NAMES]
              for _ in range(2)]
    dy = inp["dy"].to(torch.bfloat16).cuda()
    y0, _ = backbone.RWKV7_ClampW.apply(*leaves[0])
    y0.backward(dy)
    y1, _ = segmented.SegmentedClampW.apply(*leaves[1], P)
    y1.backward(dy)
    torch.cuda.synchronize()
    assert nrel(np_of(y1.detach()), np_of(y0.detach())) < TOL_BF16
    for n, a, b_ in zip(GRADS, leaves[1], leaves[0]):
        assert nrel(np_of(a.grad), np_of(b_.grad)) < TOL_BF16, n


@pytest.mark.parametrize("dtype,algo", PATHS, ids=PATH_IDS)
def test_preallocated_buffers_are_bit_identical_over_consecutive_steps(dtype, algo):
    """segmented.Buffers (no allocation or fill inside a step) gives the
    per-call allocations' results bit for bit, over consecutive steps that
    alternate a start state / final-state gradient with none (the kept-zero
    rows of the buffers must be restored)."""
    B, T, H, P, h0, hc = 2, 256, 5, 4, 1, 3
    inp = make_inputs(B, T, H, seed=71, with_dsa=True)
    xs = [inp[n].to(dtype).cuda() for n in NAMES]
    dy = inp["dy"].to(dtype).cuda()
    dsa = inp["dsa"].cuda()
    g = torch.Generator().manual_seed(72)
    s0 = (0.3 * torch.randn(B, H, 64, 64, generator=g)).cuda()
    dso = (0.3 * torch.randn(B, H, 64, 64, generator=g)).cuda()
    bufs = segmented.Buffers(B, T, H, P, h0=h0, h_count=hc, device=xs[0].device, dtype=dtype,
                             algo=algo)
    for with_state in (True, False, True, False):
        st = dict(s0=s0) if with_state else {}
        ds = dict(ds_out=dso) if with_state else {}
        outs = []
        for b in (None, bufs):
            y = torch.zeros_like(xs[0])
            sa = torch.zeros(xs[0].shape, dtype=torch.float32, device="cuda")
            grads = tuple(torch.zeros_like(xs[0]) for _ in range(6))
            _, _, saved = segmented.wkv7_forward_segmented(*xs, P, h0=h0, h_count=hc, y=y, sa=sa,
                                                           algo=algo, bufs=b, **st)
            segmented.wkv7_backward_segmented(saved, dy, dsa, grads=grads, bufs=b, **ds)
            outs.append((y, sa) + grads)
        torch.cuda.synchronize()
        for name, a, c in zip(("y", "sa") + GRADS, *outs):
            assert torch.equal(a, c), (name, with_state)
