"""The WKV-7 op at its call site inside the reference's own CaMoE train step
(tests/golden/make_camoe_step_golden.py): the CPU oracle, given the inputs the
reference model passed to ``RUN_CUDA_RWKV7`` (camoe/backbone.py:347) and the
gradients the rest of the model sent back (dy from the ln_x / output path, dsa
from ln_sa -> state_representation -> bridge and experts), reproduces the
reference recurrence's y, sa and six input gradients.  This pins the oracle on
real-model activations, which the GPU replay (test_gpu_camoe_step.py) then
compares the op against."""
import os

import numpy as np
import pytest

import oracle
from helpers import GOLDEN_DIR, GRADS, nrel

PATH = os.path.join(GOLDEN_DIR, "camoe_step_c128_l2.npz")


def calls():
    z = np.load(PATH)
    B, T, C = (int(x) for x in z["shape"])
    H = C // 64
    out = []
    for layer in range(int(z["n_layer"])):
        g = (lambda n: z[f"l{layer}_{n}"].reshape(B, T, H, 64))
        out.append({n: g(n) for n in ("r", "w", "k", "v", "a", "b", "y", "sa", "dy", "dsa") + GRADS})
    return out


def test_fixture_covers_every_gradient_path():
    for c in calls():
        for n in ("dy", "dsa") + GRADS:
            assert np.abs(c[n]).max() > 0, n


@pytest.mark.parametrize("layer", [0, 1])
def test_oracle_reproduces_the_reference_at_the_model_call_site(layer):
    c = calls()[layer]
    xs = [c[n].astype(np.float32) for n in "rwkvab"]
    y, sa = oracle.fwd(*xs)
    grads = oracle.bwd(*xs, c["dy"], c["dsa"])
    # the reference ran its float32 loop; the oracle is float64
    tol = 2e-5
    assert nrel(y, c["y"]) < tol
    assert nrel(sa, c["sa"]) < tol
    for n, g in zip(GRADS, grads):
        assert nrel(g, c[n]) < tol, n
