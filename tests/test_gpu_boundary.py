"""The reference-facing boundary on the GPU: the autograd Function and
RUN_CUDA_RWKV7 wrapper of camoe_b200.backbone, the torch.ops.rwkv7_clampw
mirror, and error behaviour (errors raise; nothing traps the device)."""
import numpy as np
import pytest
import torch

import oracle
from camoe_b200 import CamoeError, backbone, ops
from camoe_b200.inputs import make_inputs
from helpers import GRADS, TOL_BF16, TOL_FP32, nrel

pytestmark = pytest.mark.gpu
NAMES = ("r", "w", "k", "v", "a", "b")


@pytest.fixture(autouse=True)
def _init(monkeypatch):
    monkeypatch.delenv("CAMOE_FORCE_FP32_KERNEL", raising=False)
    monkeypatch.delenv("CAMOE_WKV7_ALGO", raising=False)
    backbone.init_rwkv7_cuda()
    yield
    monkeypatch.delenv("CAMOE_FORCE_FP32_KERNEL", raising=False)
    backbone.init_rwkv7_cuda()


@pytest.mark.parametrize("fp32", [False, True], ids=["bf16", "fp32"])
def test_run_cuda_wrapper_autograd_both_outputs(fp32, monkeypatch):
    """RUN_CUDA_RWKV7 on [B, T, C] fp32 tensors as RWKV7_TimeMix calls it
    (camoe/backbone.py:347), gradients flowing from both y and sa."""
    if fp32:
        monkeypatch.setenv("CAMOE_FORCE_FP32_KERNEL", "1")
        backbone.init_rwkv7_cuda()
    B, T, H = 2, 64, 3
    inp = make_inputs(B, T, H, 64, seed=3, with_dsa=True)
    dt = torch.float32 if fp32 else torch.bfloat16
    xs = [inp[n].to(dt).float().reshape(B, T, H * 64).cuda().requires_grad_(True) for n in NAMES]
    y, sa = backbone.RUN_CUDA_RWKV7(*xs)
    assert y.dtype == torch.float32 and sa.dtype == torch.float32
    gy = inp["dy"].to(dt).float().reshape(B, T, H * 64).cuda()
    gsa = inp["dsa"].reshape(B, T, H * 64).cuda()
    ((y * gy).sum() + (sa * gsa).sum()).backward()
    want_y, want_sa = oracle.fwd(*[x.detach().cpu().view(B, T, H, 64) for x in xs])
    want_g = oracle.bwd(*[x.detach().cpu().view(B, T, H, 64) for x in xs],
                        gy.cpu().view(B, T, H, 64), inp["dsa"])
    tol = TOL_FP32 if fp32 else TOL_BF16
    assert nrel(y.detach().cpu().view(B, T, H, 64), want_y) < tol
    assert nrel(sa.detach().cpu().view(B, T, H, 64), want_sa) < tol
    for n, x, w in zip(GRADS, xs, want_g):
        assert nrel(x.grad.cpu().view(B, T, H, 64), w) < tol, n


def test_only_y_used_in_loss():
    B, T, H = 1, 32, 2
    inp = make_inputs(B, T, H, 64, seed=4)
    xs = [inp[n].to(torch.bfloat16).cuda().requires_grad_(True) for n in NAMES]
    y, sa = backbone.RWKV7_ClampW.apply(*xs)
    (y.float() * inp["dy"].cuda()).sum().backward()
    want = oracle.bwd(*[x.detach().float().cpu() for x in xs], inp["dy"].to(torch.bfloat16).float())
    for n, x, w in zip(GRADS, xs, want):
        assert nrel(x.grad.float().cpu(), w) < TOL_BF16, n


def test_no_grad_forward_skips_checkpoint():
    inp = make_inputs(1, 32, 2, 64, seed=4)
    xs = [inp[n].to(torch.bfloat16).cuda() for n in NAMES]
    with torch.no_grad():
        y, sa = backbone.RWKV7_ClampW.apply(*xs)
    want_y, want_sa = oracle.fwd(*[x.float().cpu() for x in xs])
    assert nrel(y.float().cpu(), want_y) < TOL_BF16
    assert nrel(sa.cpu(), want_sa) < TOL_BF16


def test_function_asserts_like_the_reference():
    inp = make_inputs(1, 24, 1, 64, seed=1)  # T % 16 != 0
    xs = [inp[n].to(torch.bfloat16).cuda() for n in NAMES]
    with pytest.raises(AssertionError):
        backbone.RWKV7_ClampW.apply(*xs)
    inp = make_inputs(1, 32, 1, 64, seed=1)
    xs = [inp[n].cuda() for n in NAMES]  # fp32 while the kernel expects bf16
    with pytest.raises(AssertionError):
        backbone.RWKV7_ClampW.apply(*xs)


def test_torch_ops_mirror_of_reference_binding():
    B, T, H = 2, 48, 2
    inp = make_inputs(B, T, H, 64, seed=7)
    xs = [inp[n].to(torch.bfloat16).cuda() for n in NAMES]
    dy = inp["dy"].to(torch.bfloat16).cuda()
    y = torch.empty_like(xs[0])
    s = torch.empty(B, H, T // 16, 64, 64, dtype=torch.float32, device="cuda")
    sa = torch.empty(B, T, H, 64, dtype=torch.float32, device="cuda")
    torch.ops.rwkv7_clampw.forward(*xs, y, s, sa)
    grads = [torch.empty_like(xs[0]) for _ in range(6)]
    torch.ops.rwkv7_clampw.backward(*xs, dy, s, sa, *grads)
    torch.cuda.synchronize()
    ref = [inp[n].to(torch.bfloat16).float() for n in NAMES]
    want_y, want_sa = oracle.fwd(*ref)
    want_g = oracle.bwd(*ref, dy.float().cpu())
    assert nrel(y.float().cpu(), want_y) < TOL_BF16
    assert nrel(sa.cpu(), want_sa) < TOL_BF16
    for n, g, w in zip(GRADS, grads, want_g):
        assert nrel(g.float().cpu(), w) < TOL_BF16, n


def test_errors_raise_without_device_fault():
    inp = make_inputs(1, 32, 1, 64, seed=2)
    xs = [inp[n].to(torch.bfloat16).cuda() for n in NAMES]
    # a contiguous view whose data pointer is only 2-byte aligned
    flat = torch.empty(xs[0].numel() + 1, dtype=torch.bfloat16, device="cuda")
    bad = flat[1:].view_as(xs[0])
    with pytest.raises(CamoeError) as ei:
        ops.wkv7_forward(bad, *xs[1:])
    assert ei.value.status == 4
    with pytest.raises(CamoeError):
        ops.wkv7_forward(*xs, algo="chunked", h0=0, h_count=5)  # head range past H
    with pytest.raises(CamoeError):  # fp32 has no chunked path
        ops.wkv7_forward(*[x.float() for x in xs], algo="chunked")
    with pytest.raises(ValueError):
        ops.wkv7_forward(*[x.cpu() for x in xs])
    # the context is still healthy afterwards
    y, sa, _ = ops.wkv7_forward(*xs, algo="scan")
    torch.cuda.synchronize()
    assert torch.isfinite(y.float()).all()


def test_empty_inputs():
    for B, T, H in ((0, 32, 2), (2, 0, 2)):
        xs = [torch.zeros(B, T, H, 64, dtype=torch.bfloat16, device="cuda") for _ in NAMES]
        y, sa, ck = ops.wkv7_forward(*xs)
        g = ops.wkv7_backward(*xs, torch.zeros_like(xs[0]), None, ck)
        assert y.shape == (B, T, H, 64) and all(t.shape == (B, T, H, 64) for t in g)


@pytest.mark.parametrize("decay", ["clampw", "wind"])
def test_first_call_on_a_fresh_thread(decay):
    """The op's first CUDA call on a thread (as on a framework's backward worker
    thread, before anything else there touched the device) gives the main
    thread's results: the chunked path binds the device's context before it
    encodes its TMA descriptors.  All buffers come from the main thread."""
    import threading

    B, T, H = 2, 64, 3
    inp = make_inputs(B, T, H, 64, seed=12, decay=decay)
    xs = [inp[n].to(torch.bfloat16).cuda() for n in NAMES]
    dy = inp["dy"].to(torch.bfloat16).cuda()
    y0, sa0, ck0 = ops.wkv7_forward(*xs, decay=decay)
    g0 = ops.wkv7_backward(*xs, dy, None, ck0, decay=decay)
    y, sa, ck = torch.empty_like(y0), torch.empty_like(sa0), torch.empty_like(ck0)
    grads = tuple(torch.empty_like(g) for g in g0)
    work = torch.empty(max(ops.work_bytes(B, T, H, torch.bfloat16), 16), dtype=torch.uint8,
                       device="cuda")
    torch.cuda.synchronize()
    errors = []

    def run():
        try:
            ops.wkv7_forward(*xs, y=y, sa=sa, ckpt=ck, decay=decay)
            ops.wkv7_backward(*xs, dy, None, ck, grads=grads, work=work, decay=decay)
        except Exception as e:  # reported on the main thread
            errors.append(e)

    th = threading.Thread(target=run)
    th.start()
    th.join()
    torch.cuda.synchronize()
    assert not errors, errors
    assert torch.equal(y, y0) and torch.equal(sa, sa0)
    for g, w in zip(grads, g0):
        assert torch.equal(g, w)
