"""The op as a drop-in at the reference model's call site, on the GPU.

Replays the calls that the reference's own CaMoE train step
(camoe/system.py:304-355 with train.py:726-774; recorded by
tests/golden/make_camoe_step_golden.py, 2 layers at C=128) makes to
``RUN_CUDA_RWKV7(r, w, k, v, -kk, kk*a)`` (camoe/backbone.py:347), through
``camoe_b200.backbone.RUN_CUDA_RWKV7`` -- the reference's [B, T, C] calling
convention, dtype casts and autograd Function -- with the recorded gradients
of y and sa fed to ``backward``, as the model's autograd graph does.  The
activation-checkpoint recompute calls the op again with the same inputs; the
replay does so too and checks that both calls agree bit for bit.

* bf16 kernel (the default): every output and gradient against the oracle on
  the bf16-rounded inputs, and against the reference recurrence's values,
  within 2e-2 norm-relative error;
* fp32 kernel (CAMOE_FORCE_FP32_KERNEL=1): against the reference recurrence's
  values within 1e-4.
"""
import numpy as np
import pytest
import torch

import oracle
from camoe_b200 import _lib, backbone
from helpers import GRADS, TOL_BF16, TOL_FP32, nrel
from test_camoe_step_golden import calls

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _no_device_timeouts():
    before = _lib.lib().camoe_wkv7_device_errors()
    yield
    assert _lib.lib().camoe_wkv7_device_errors() == before


def replay(c, monkeypatch, fp32):
    monkeypatch.setenv("CAMOE_FORCE_FP32_KERNEL", "1" if fp32 else "0")
    backbone.init_rwkv7_cuda()
    B, T, H, N = c["r"].shape
    outs = []
    for _ in range(2):  # the forward, then the activation-checkpoint recompute
        xs = [torch.from_numpy(c[n].reshape(B, T, H * N)).cuda().requires_grad_(True)
              for n in "rwkvab"]
        y, sa = backbone.RUN_CUDA_RWKV7(*xs)
        assert y.dtype == torch.float32 and sa.dtype == torch.float32  # the caller's dtype
        dy = torch.from_numpy(c["dy"].reshape(B, T, H * N)).cuda()
        dsa = torch.from_numpy(c["dsa"].reshape(B, T, H * N)).cuda()
        torch.autograd.backward([y, sa], [dy, dsa])
        torch.cuda.synchronize()
        outs.append([t.detach().cpu().numpy().reshape(B, T, H, N)
                     for t in [y, sa] + [x.grad for x in xs]])
    for a, b in zip(*outs):
        np.testing.assert_array_equal(a, b)
    return outs[0]


@pytest.mark.parametrize("layer", [0, 1])
def test_bf16_op_at_the_model_call_site(layer, monkeypatch):
    c = calls()[layer]
    got = replay(c, monkeypatch, fp32=False)
    rounded = [torch.from_numpy(c[n]).to(torch.bfloat16).float().numpy() for n in "rwkvab"]
    want = list(oracle.fwd(*rounded)) + list(oracle.bwd(*rounded, c["dy"], c["dsa"]))
    for name, g, w in zip(("y", "sa") + GRADS, got, want):
        assert nrel(g, w) < TOL_BF16, (name, "oracle")
        assert nrel(g, c[name]) < TOL_BF16, (name, "reference")


@pytest.mark.parametrize("layer", [0, 1])
def test_fp32_op_at_the_model_call_site(layer, monkeypatch):
    c = calls()[layer]
    try:
        got = replay(c, monkeypatch, fp32=True)
    finally:
        monkeypatch.setenv("CAMOE_FORCE_FP32_KERNEL", "0")
        backbone.init_rwkv7_cuda()
    for name, g in zip(("y", "sa") + GRADS, got):
        assert nrel(g, c[name]) < TOL_FP32, name
