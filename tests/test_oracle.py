"""The CPU oracle, pinned against the reference's own recurrence.

The golden vectors were produced by the reference's fallback recurrence
(camoe/backbone.py:250-294) with torch.autograd gradients
(tests/golden/make_golden.py).  A second, independent restatement in float64
torch (oracle.torch_reference) cross-checks the external-sa-gradient path,
which the reference cannot exercise (its autograd backward drops dsa).
"""
import math

import numpy as np
import pytest

import oracle
from camoe_b200.inputs import make_inputs
from helpers import GRADS, golden_cases, input_digest, load_golden, nrel

CASES = golden_cases()


def test_golden_cases_present():
    assert len(CASES) >= 5


@pytest.mark.parametrize("path", CASES, ids=lambda p: p.split("/")[-1][:-4])
@pytest.mark.parametrize("precision", ["f64", "f32"])
def test_oracle_matches_reference_golden(path, precision):
    z, inp = load_golden(path)
    assert input_digest(inp) == str(z["input_sha256"]), "input generator drifted"
    args = [inp[n] for n in ("r", "w", "k", "v", "a", "b")]
    y, sa = oracle.fwd(*args, precision=precision)
    grads = oracle.bwd(*args, inp["dy"], precision=precision, ckpt=16)
    # the golden values are float32 autograd through a float32 loop; sa is the
    # reference's own per-step row sum (camoe/backbone.py:284), captured
    tol = 2e-5
    assert nrel(y, z["y"]) < tol
    assert nrel(sa, z["sa"]) < tol
    for n, g in zip(GRADS, grads):
        assert nrel(g, z[n]) < tol, n


def test_oracle_sa_and_dsa_against_torch_autograd():
    inp = make_inputs(2, 24, 2, 64, seed=11, with_dsa=True)
    args = [inp[n] for n in ("r", "w", "k", "v", "a", "b")]
    ref = oracle.torch_reference(*args, dy=inp["dy"], dsa=inp["dsa"])
    y, sa = oracle.fwd(*args)
    grads = oracle.bwd(*args, inp["dy"], inp["dsa"], ckpt=5)
    assert nrel(y, ref[0]) < 1e-6
    assert nrel(sa, ref[1]) < 1e-6
    for n, g, gr in zip(GRADS, grads, ref[2:]):
        assert nrel(g, gr) < 1e-6, n


@pytest.mark.parametrize("ckpt", [1, 3, 16, 64, 1000])
def test_oracle_checkpoint_interval_does_not_change_gradients(ckpt):
    inp = make_inputs(1, 50, 1, 64, seed=5, with_dsa=True)
    args = [inp[n] for n in ("r", "w", "k", "v", "a", "b", "dy", "dsa")]
    base = oracle.bwd(*args, ckpt=7)
    other = oracle.bwd(*args, ckpt=ckpt)
    for g0, g1 in zip(base, other):
        np.testing.assert_array_equal(g0, g1)


def test_oracle_decay_range():
    # w = exp(-e^{-1/2} sigmoid(x)) lies in (exp(-e^{-1/2}), 1)
    lo = math.exp(-math.exp(-0.5))
    assert abs(oracle.decay(0.0) - math.exp(-math.exp(-0.5) / 2)) < 1e-15
    assert lo < oracle.decay(30.0) < lo + 1e-9
    assert 1 - 1e-9 < oracle.decay(-30.0) < 1.0


def test_oracle_empty_inputs():
    inp = make_inputs(1, 0, 1, 64, seed=0)
    args = [inp[n] for n in ("r", "w", "k", "v", "a", "b")]
    y, sa = oracle.fwd(*args)
    assert y.shape == (1, 0, 1, 64)
    grads = oracle.bwd(*args, inp["dy"])
    assert all(g.shape == (1, 0, 1, 64) for g in grads)


def test_oracle_chains_are_independent():
    # results for (b, h) must not depend on the other chains in the batch
    inp = make_inputs(2, 32, 3, 64, seed=9)
    args = [inp[n] for n in ("r", "w", "k", "v", "a", "b")]
    y, sa = oracle.fwd(*args)
    one = [x[1:2, :, 2:3].contiguous() for x in args]
    y1, sa1 = oracle.fwd(*one)
    np.testing.assert_array_equal(y[1:2, :, 2:3], y1)
    np.testing.assert_array_equal(sa[1:2, :, 2:3], sa1)


def test_oracle_state_forward_zero_start_equals_fwd():
    inp = make_inputs(2, 37, 3, seed=5)
    xs = [inp[n] for n in ("r", "w", "k", "v", "a", "b")]
    y, sa = oracle.fwd(*xs)
    y1, sa1, sT = oracle.fwd_state(*xs)
    assert np.array_equal(y, y1) and np.array_equal(sa, sa1)
    assert sT.shape == (2, 3, 64, 64) and np.isfinite(sT).all()


def test_oracle_state_forward_against_torch_with_start_state():
    """The start state enters the recurrence as S_{-1}: checked against the
    independent float64 torch restatement."""
    inp = make_inputs(2, 24, 2, seed=6)
    xs = [inp[n] for n in ("r", "w", "k", "v", "a", "b")]
    s0 = np.random.default_rng(6).standard_normal((2, 2, 64, 64)).astype(np.float32)
    y, sa, _ = oracle.fwd_state(*xs, s0=s0)
    yt, sat = oracle.torch_reference(*xs, s0=s0)
    assert nrel(y, yt) < 1e-6 and nrel(sa, sat) < 1e-6


@pytest.mark.parametrize("T1", [1, 16, 23])
def test_oracle_state_split_identity(T1):
    """A forward over [0, T1) then over [T1, T) from its final state equals one
    forward over [0, T)."""
    inp = make_inputs(2, 40, 3, seed=7)
    xs = [inp[n] for n in ("r", "w", "k", "v", "a", "b")]
    y, sa, sT = oracle.fwd_state(*xs)
    ya, saa, s1 = oracle.fwd_state(*[x[:, :T1] for x in xs])
    yb, sab, s2 = oracle.fwd_state(*[x[:, T1:] for x in xs], s0=s1)
    assert nrel(np.concatenate([ya, yb], 1), y) < 1e-5
    assert nrel(np.concatenate([saa, sab], 1), sa) < 1e-5
    assert nrel(s2, sT) < 1e-5


def test_oracle_wind_decay_against_torch_autograd():
    """The wind_backstepping decay exp(-exp(w)) (camoe/cuda/wkv7_cuda.cu:21,66-67,108):
    forward and all six gradients of the C oracle against float64 torch autograd."""
    inp = make_inputs(1, 40, 2, seed=8, decay="wind", with_dsa=True)
    xs = [inp[n] for n in ("r", "w", "k", "v", "a", "b")]
    y, sa = oracle.fwd(*xs, decay="wind")
    grads = oracle.bwd(*xs, inp["dy"], inp["dsa"], decay="wind", ckpt=16)
    ref = oracle.torch_reference(*xs, dy=inp["dy"], dsa=inp["dsa"], decay="wind")
    for name, got, want in zip(("y", "sa") + GRADS, (y, sa) + grads, ref):
        assert nrel(got, want) < 1e-6, name
    # the decay differs from ClampW's on the same inputs
    y_c, _ = oracle.fwd(*xs)
    assert nrel(y_c, y) > 1e-3


def test_wind_inputs_are_in_the_bounded_decay_range():
    inp = make_inputs(2, 64, 4, seed=9, decay="wind", w_sigma=3.0)
    assert float(inp["w"].max()) <= -0.5
    lo = math.exp(-math.exp(-0.5))
    dec = np.exp(-np.exp(inp["w"].numpy().astype(np.float64)))
    assert dec.min() >= lo - 1e-12 and dec.max() < 1


def test_oracle_state_gradients_against_torch_autograd():
    """The backward of a sequence carried across calls: with a start state and
    a gradient of the final state, all six gradients and the gradient of the
    start state against float64 torch autograd."""
    inp = make_inputs(2, 24, 2, seed=9, with_dsa=True)
    xs = [inp[n] for n in ("r", "w", "k", "v", "a", "b")]
    g = np.random.default_rng(9)
    s0 = g.standard_normal((2, 2, 64, 64)).astype(np.float32)
    dsT = g.standard_normal((2, 2, 64, 64)).astype(np.float32)
    got = oracle.bwd_state(*xs, inp["dy"], inp["dsa"], s0=s0, dsT=dsT, ckpt=8)
    want = oracle.torch_reference(*xs, dy=inp["dy"], dsa=inp["dsa"], s0=s0, dsT=dsT)[2:]
    for name, a, b in zip(GRADS + ("ds0",), got, want):
        assert nrel(a, b) < 1e-6, name
    # without states it is bwd
    plain = oracle.bwd(*xs, inp["dy"], inp["dsa"])
    zero = oracle.bwd_state(*xs, inp["dy"], inp["dsa"])
    for a, b in zip(plain, zero[:6]):
        assert np.array_equal(a, b)


def test_oracle_state_gradient_split_identity():
    """Gradients of one pass over [0, T) equal those of [0, T1) and [T1, T)
    with the state carried forward and its gradient carried back."""
    T, T1 = 48, 16
    inp = make_inputs(1, T, 2, seed=10)
    xs = [inp[n] for n in ("r", "w", "k", "v", "a", "b")]
    full = oracle.bwd(*xs, inp["dy"])
    first = [x[:, :T1] for x in xs]
    second = [x[:, T1:] for x in xs]
    _, _, s1 = oracle.fwd_state(*first)
    g2 = oracle.bwd_state(*second, inp["dy"][:, T1:], s0=s1)
    g1 = oracle.bwd_state(*first, inp["dy"][:, :T1], dsT=g2[6])
    for name, f, a, b in zip(GRADS, full, g1[:6], g2[:6]):
        assert nrel(np.concatenate([a, b], 1), f) < 1e-5, name


def test_oracle_segment_map_is_affine():
    """The algebra of the time-segmented path, on the oracle: a stretch's final
    state is S_end = s0 A + C, with A the final state from the identity with
    v = 0 and C the final state from zero; its start-state gradient is
    ds0 = dsT A^T + D, with D the start-state gradient when dsT = 0."""
    inp = make_inputs(1, 40, 2, seed=11)
    xs = [inp[n] for n in ("r", "w", "k", "v", "a", "b")]
    g = np.random.default_rng(11)
    s0 = g.standard_normal((1, 2, 64, 64)).astype(np.float32)
    dsT = g.standard_normal((1, 2, 64, 64)).astype(np.float32)
    eye = np.broadcast_to(np.eye(64, dtype=np.float32), (1, 2, 64, 64)).copy()
    xz = list(xs)
    xz[3] = np.zeros_like(xs[3])
    A = oracle.fwd_state(*xz, s0=eye)[2].astype(np.float64)
    C = oracle.fwd_state(*xs)[2].astype(np.float64)
    S = oracle.fwd_state(*xs, s0=s0)[2]
    assert nrel(S, s0.astype(np.float64) @ A + C) < 1e-6
    D = oracle.bwd_state(*xs, inp["dy"], s0=s0)[6].astype(np.float64)
    ds0 = oracle.bwd_state(*xs, inp["dy"], s0=s0, dsT=dsT)[6]
    assert nrel(ds0, dsT.astype(np.float64) @ np.swapaxes(A, -1, -2) + D) < 1e-6
