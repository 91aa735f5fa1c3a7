"""GPU parity of the stateful forward (camoe_wkv7_fwd_state): start state in,
final state out, and the decode-step kernel, against the CPU oracle.

The reference has no stateful call (it recomputes the whole prefix for every
generated token, eval.py:212); its recurrence with S_{-1} = s0 is the oracle's
fwd_state, whose zero-state case is pinned to the reference like fwd.  The
start states are real ones: the oracle's final state after a random prefix.

Tolerance: norm-relative max error per output tensor (y, sa, final state),
1e-4 for fp32 inputs and 2e-2 for bf16, the oracle in float64 on the same
(rounded) inputs.
"""
import numpy as np
import pytest
import torch

import oracle
from camoe_b200 import _lib, ops
from camoe_b200.inputs import make_inputs
from helpers import TOL_BF16, TOL_FP32, nrel

pytestmark = pytest.mark.gpu

NAMES = ("r", "w", "k", "v", "a", "b")
# (dtype, algo, work): work False = the fused chunked kernel, True = the
# key-side pass into a workspace, then the value pass
PATHS = [(torch.float32, "scan", False), (torch.bfloat16, "scan", False),
         (torch.bfloat16, "chunked", False), (torch.bfloat16, "chunked", True),
         (torch.float32, "auto", "auto"), (torch.bfloat16, "auto", "auto")]
PATH_IDS = ["fp32-scan", "bf16-scan", "bf16-chunked-fused", "bf16-chunked-work", "fp32-auto",
            "bf16-auto"]

# (B, T, H, seed): decode steps (T <= 16 runs the step kernel under scan/auto),
# ragged and whole chunks, and a multi-chunk prefill
SHAPES = {
    "decode_t1": (4, 1, 16, 11),
    "t5": (2, 5, 3, 12),
    "t16": (3, 16, 2, 13),
    "t17": (1, 17, 2, 14),
    "ragged_t40": (2, 40, 3, 15),
    "prefill_t256": (2, 256, 4, 16),
}


@pytest.fixture(autouse=True)
def _no_device_timeouts():
    before = _lib.lib().camoe_wkv7_device_errors()
    yield
    assert _lib.lib().camoe_wkv7_device_errors() == before


def tol_for(dtype):
    return TOL_FP32 if dtype == torch.float32 else TOL_BF16


def start_state(B, H, seed, T0=48):
    """The oracle's state after T0 random steps (a realistic magnitude)."""
    pre = make_inputs(B, T0, H, seed=1000 + seed)
    return oracle.fwd_state(*[pre[n] for n in NAMES])[2]


def rounded(inp, dtype):
    return [inp[n].to(dtype).float() for n in NAMES]


def to_dev(inp, dtype):
    return [inp[n].to(dtype).cuda() for n in NAMES]


def check(got, want, tol, label):
    errs = {n: nrel(g, w) for n, g, w in zip(("y", "sa", "state"), got, want)}
    bad = {n: e for n, e in errs.items() if not e < tol}
    assert not bad, f"{label}: errors above {tol}: {bad} (all: {errs})"


@pytest.mark.parametrize("dtype,algo,work", PATHS, ids=PATH_IDS)
@pytest.mark.parametrize("shape", list(SHAPES), ids=list(SHAPES))
def test_state_matches_oracle(shape, dtype, algo, work):
    B, T, H, seed = SHAPES[shape]
    inp = make_inputs(B, T, H, seed=seed)
    s0 = start_state(B, H, seed)
    want = oracle.fwd_state(*rounded(inp, dtype), s0=s0)
    y, sa, sT = ops.wkv7_forward_state(*to_dev(inp, dtype), torch.from_numpy(s0).cuda(), algo=algo,
                                       work=work)
    torch.cuda.synchronize()
    got = [y.float().cpu().numpy(), sa.cpu().numpy(), sT.cpu().numpy()]
    check(got, want, tol_for(dtype), f"{shape} {dtype} {algo}")


@pytest.mark.parametrize("dtype,algo,work", PATHS[:4], ids=PATH_IDS[:4])
def test_zero_state_equals_stateless_forward(dtype, algo, work):
    """s0 = None gives bit-for-bit the outputs of camoe_wkv7_fwd (same kernels)."""
    for (B, T, H) in ((2, 40, 3), (1, 7, 2), (2, 128, 16)):
        xs = to_dev(make_inputs(B, T, H, seed=T), dtype)
        # the workspace path runs the training forward's kernels
        y0, sa0, _ = ops.wkv7_forward(*xs, algo=algo, save_ckpt=work is True)
        y1, sa1, sT = ops.wkv7_forward_state(*xs, None, algo=algo, work=work)
        torch.cuda.synchronize()
        assert torch.equal(y0, y1) and torch.equal(sa0, sa1)
        assert torch.isfinite(sT).all()


@pytest.mark.parametrize("dtype,algo,work", PATHS[:4], ids=PATH_IDS[:4])
def test_split_sequence_equals_one_pass(dtype, algo, work):
    """Forward over [0, T1) then over [T1, T) from its final state equals one
    forward over [0, T) (outputs within tolerance of the one-pass oracle)."""
    B, T, H, T1 = 2, 96, 3, 48
    inp = make_inputs(B, T, H, seed=21)
    xs = to_dev(inp, dtype)
    ya, saa, s1 = ops.wkv7_forward_state(*[x[:, :T1].contiguous() for x in xs], None, algo=algo,
                                         work=work)
    yb, sab, s2 = ops.wkv7_forward_state(*[x[:, T1:].contiguous() for x in xs], s1, algo=algo,
                                         work=work)
    torch.cuda.synchronize()
    want = oracle.fwd_state(*rounded(inp, dtype))
    got = [torch.cat([ya, yb], 1).float().cpu().numpy(), torch.cat([saa, sab], 1).cpu().numpy(),
           s2.cpu().numpy()]
    check(got, want, tol_for(dtype), f"split {dtype} {algo}")


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16], ids=["fp32", "bf16"])
def test_prefill_then_decode_loop(dtype):
    """Prefill a 64-step prompt (chunked for bf16), then 16 single-token decode
    steps updating the state in place: y of every decoded token and the final
    state match the oracle's one pass over all 80 steps."""
    B, T0, n_dec, H = 3, 64, 16, 8
    inp = make_inputs(B, T0 + n_dec, H, seed=31)
    xs = to_dev(inp, dtype)
    _, _, state = ops.wkv7_forward_state(*[x[:, :T0].contiguous() for x in xs], None)
    ys, sas = [], []
    for t in range(T0, T0 + n_dec):
        y, sa = ops.wkv7_decode_step(*[x[:, t].contiguous() for x in xs], state)
        ys.append(y)
        sas.append(sa)
    torch.cuda.synchronize()
    yw, saw, sw = oracle.fwd_state(*rounded(inp, dtype))
    got = [torch.stack(ys, 1).float().cpu().numpy(), torch.stack(sas, 1).cpu().numpy(),
           state.cpu().numpy()]
    check(got, [yw[:, T0:], saw[:, T0:], sw], tol_for(dtype), f"decode {dtype}")


@pytest.mark.parametrize("dtype,algo,work", PATHS[:4], ids=PATH_IDS[:4])
def test_inplace_equals_out_of_place(dtype, algo, work):
    B, T, H = 2, 33, 4
    xs = to_dev(make_inputs(B, T, H, seed=41), dtype)
    s0 = torch.from_numpy(start_state(B, H, 41)).cuda()
    y0, sa0, s_out = ops.wkv7_forward_state(*xs, s0, algo=algo, work=work)
    s_in = s0.clone()
    y1, sa1, s_same = ops.wkv7_forward_state(*xs, s_in, algo=algo, inplace=True, work=work)
    torch.cuda.synchronize()
    assert s_same.data_ptr() == s_in.data_ptr()
    assert torch.equal(y0, y1) and torch.equal(sa0, sa1) and torch.equal(s_out, s_in)


@pytest.mark.parametrize("dtype,algo,work", PATHS[:4], ids=PATH_IDS[:4])
def test_head_range_touches_only_its_states(dtype, algo, work):
    """A head slice [h0, h0 + hc) reads and writes only those heads' states,
    and its outputs equal the full run's bit for bit."""
    B, T, H, h0, hc = 2, 40, 6, 2, 3
    xs = to_dev(make_inputs(B, T, H, seed=51), dtype)
    s0 = torch.from_numpy(start_state(B, H, 51)).cuda()
    yf, saf, sf = ops.wkv7_forward_state(*xs, s0, algo=algo, work=work)
    out = torch.full_like(s0, 7.0)
    y, sa, _ = ops.wkv7_forward_state(*xs, s0, algo=algo, h0=h0, h_count=hc, out_state=out,
                                      zero_rest=True, work=work)
    torch.cuda.synchronize()
    sl = slice(h0, h0 + hc)
    assert torch.equal(out[:, sl], sf[:, sl])
    assert (out[:, :h0] == 7.0).all() and (out[:, h0 + hc:] == 7.0).all()
    assert torch.equal(y[:, :, sl], yf[:, :, sl]) and torch.equal(sa[:, :, sl], saf[:, :, sl])


def test_zero_steps_copy_or_clear_the_state():
    B, H, h0, hc = 2, 4, 1, 2
    xs = to_dev(make_inputs(B, 0, H, seed=0), torch.bfloat16)
    s0 = torch.randn(B, H, 64, 64, device="cuda")
    out = torch.full_like(s0, 3.0)
    ops.wkv7_forward_state(*xs, s0, h0=h0, h_count=hc, out_state=out)
    torch.cuda.synchronize()
    assert torch.equal(out[:, h0:h0 + hc], s0[:, h0:h0 + hc])
    assert (out[:, :h0] == 3.0).all() and (out[:, h0 + hc:] == 3.0).all()
    ops.wkv7_forward_state(*xs, None, h0=h0, h_count=hc, out_state=out)
    torch.cuda.synchronize()
    assert (out[:, h0:h0 + hc] == 0).all() and (out[:, :h0] == 3.0).all()


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16], ids=["fp32", "bf16"])
def test_decode_batch_of_many_chains(dtype):
    """The decode-step kernel over 2048 chains (B=128, H=16), one token."""
    B, H = 128, 16
    inp = make_inputs(B, 1, H, seed=61)
    s0 = np.ascontiguousarray(
        np.random.default_rng(61).standard_normal((B, H, 64, 64)).astype(np.float32))
    want = oracle.fwd_state(*rounded(inp, dtype), s0=s0)
    state = torch.from_numpy(s0).cuda()
    y, sa = ops.wkv7_decode_step(*[x[:, 0] for x in to_dev(inp, dtype)], state)
    torch.cuda.synchronize()
    got = [y.float().cpu().numpy()[:, None], sa.cpu().numpy()[:, None], state.cpu().numpy()]
    check(got, want, tol_for(dtype), f"decode batch {dtype}")
