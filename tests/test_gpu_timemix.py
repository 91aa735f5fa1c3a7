"""GPU numerics of the fused time mix (camoe_b200/timemix.py,
include/camoe_timemix.h).

* Each fused kernel, forward and backward (input and parameter gradients),
  against a plain PyTorch fp32 statement of the same reference lines with
  autograd, on the same bf16-rounded inputs.  Tolerance: norm-relative max
  error 1e-2 for bf16 outputs (one bf16 rounding of the result), 1e-4 for fp32
  outputs and parameter gradients (fp32 sums in a different order).
* The whole module against golden vectors of the reference's own
  RWKV7_TimeMix (tests/golden/make_timemix_golden.py: float64 on the CPU):
  outputs, the input gradients and every parameter gradient.  Tolerance 3e-2:
  bf16 activations and GEMMs across eight chained products (the op alone is
  held to 2e-2).
"""
import ctypes
import os
import sys

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from camoe_b200 import _lib, timemix
from helpers import GOLDEN_DIR, nrel

sys.path.insert(0, GOLDEN_DIR)
from make_timemix_golden import CASES, digest, grad_projection, timemix_inputs, timemix_params  # noqa: E402

pytestmark = pytest.mark.gpu
BF = torch.bfloat16
W_SCALE = -float(np.exp(-0.5))


@pytest.fixture(autouse=True)
def _no_device_timeouts():
    before = _lib.lib().camoe_wkv7_device_errors()
    yield
    assert _lib.lib().camoe_wkv7_device_errors() == before


def rnd(*shape, scale=1.0, seed=0, dtype=BF):
    g = torch.Generator().manual_seed(seed)
    return (scale * torch.randn(*shape, generator=g)).to(dtype).cuda()


def p(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def stream():
    return torch.cuda.current_stream().cuda_stream


def work(B, T, C):
    n = int(_lib.lib().camoe_tm_work_bytes(B, T, C))
    return torch.empty(n, dtype=torch.uint8, device="cuda"), n


def close(got, want, tol, name):
    e = nrel(got.detach().float().cpu().numpy(), want.detach().float().cpu().numpy())
    assert e < tol, f"{name}: {e:.3g} >= {tol}"


# C = 320: 40 threads of 8 columns (a full warp and a partial one), 160 of 2
SHAPES = [(2, 40, 128), (1, 17, 1024), (3, 16, 2048), (1, 5, 64), (2, 9, 320)]


@pytest.mark.parametrize("xdt", [BF, torch.float32], ids=["bf16", "fp32"])
@pytest.mark.parametrize("B,T,C", SHAPES)
def test_mix_kernel(B, T, C, xdt):
    x = rnd(B, T, C, seed=1, dtype=xdt)
    mix = torch.rand(6, C, generator=torch.Generator().manual_seed(2)).cuda()
    outs = [torch.empty(B, T, C, dtype=BF, device="cuda") for _ in range(6)]
    L = _lib.lib()
    ptr6 = (lambda ts: (ctypes.c_void_p * 6)(*[t.data_ptr() for t in ts]))
    assert L.camoe_tm_mix_fwd(p(x), 0 if xdt == BF else 1, p(mix), ptr6(outs), B, T, C, stream()) == 0
    xr = x.float().requires_grad_(True)
    mr = mix.clone().requires_grad_(True)
    xx = F.pad(xr, (0, 0, 1, -1)) - xr          # backbone.py:316 (ZeroPad2d((0, 0, 1, -1)))
    want = [xr + xx * mr[m] for m in range(6)]
    for m in range(6):
        close(outs[m], want[m], 1e-2, f"mix out {m}")
    douts = [rnd(B, T, C, seed=10 + m) for m in range(6)]
    dx = torch.empty_like(x)
    dmix = torch.empty(6, C, device="cuda")
    w, nw = work(B, T, C)
    assert L.camoe_tm_mix_bwd(p(x), 0 if xdt == BF else 1, p(mix), ptr6(douts), p(dx), p(dmix),
                              p(w), nw, B, T, C, stream()) == 0
    torch.autograd.backward(want, [d.float() for d in douts])
    close(dx, xr.grad, 1e-2 if xdt == BF else 1e-4, "dx")
    close(dmix, mr.grad, 1e-4, "dmix")


def prep_ref(wl, k, v, vl, al, vf, par, H):
    """camoe/backbone.py:326-343 in fp32 (as the reference computes them)."""
    w0, v0, a0, k_k, k_a = par
    w = -F.softplus(-(w0 + wl)) - 0.5
    if vl is not None:
        v = v + (vf - v) * torch.sigmoid(v0 + vl)
    a = torch.sigmoid(a0 + al)
    B, T, C = k.shape
    kk = F.normalize((k * k_k).view(B, T, H, -1), dim=-1, p=2.0).view(B, T, C)
    k = k * (1 + (a - 1) * k_a)
    return w, k, v, -kk, kk * a


@pytest.mark.parametrize("vres", [False, True], ids=["layer0", "layer_gt0"])
@pytest.mark.parametrize("B,T,C", SHAPES)
def test_prep_kernel(B, T, C, vres):
    H = C // 64
    ins = {n: rnd(B, T, C, seed=20 + i) for i, n in enumerate(("wl", "k", "v", "vl", "al", "vf"))}
    if not vres:
        ins["vl"] = ins["vf"] = None
    g = torch.Generator().manual_seed(3)
    par = torch.stack([-2 + torch.randn(C, generator=g), 0.5 + 0.3 * torch.randn(C, generator=g),
                       0.3 * torch.randn(C, generator=g), 0.71 + 0.1 * torch.randn(C, generator=g),
                       1.02 + 0.1 * torch.randn(C, generator=g)]).cuda()
    outs = [torch.empty(B, T, C, dtype=BF, device="cuda") for _ in range(5)]
    L = _lib.lib()
    assert L.camoe_tm_prep_fwd(*[p(ins[n]) for n in ("wl", "k", "v", "vl", "al", "vf")], p(par),
                               *[p(o) for o in outs], B, T, C, stream()) == 0
    leaves = {n: (t.float().requires_grad_(True) if t is not None else None) for n, t in ins.items()}
    parl = par.clone().requires_grad_(True)
    want = prep_ref(leaves["wl"], leaves["k"], leaves["v"], leaves["vl"], leaves["al"],
                    leaves["vf"], list(parl), H)
    for name, got, w in zip(("w", "k'", "v'", "a", "b"), outs, want):
        close(got, w, 1e-2, name)
    # gradients: op grads for (r, w, k', v', a, b), epilogue grads for (r, k', v')
    gops = [rnd(B, T, C, seed=40 + i) for i in range(6)]
    gepi = [rnd(B, T, C, seed=50 + i) for i in range(3)]
    dvfo = rnd(B, T, C, seed=60) if not vres else None
    outs_g = [torch.empty(B, T, C, dtype=BF, device="cuda") for _ in range(5)]
    dvl = torch.empty(B, T, C, dtype=BF, device="cuda") if vres else None
    dvf = torch.empty(B, T, C, dtype=BF, device="cuda") if vres else None
    dpar = torch.empty(5, C, device="cuda")
    w, nw = work(B, T, C)
    dr, dwl, dk, dv, dal = outs_g
    assert L.camoe_tm_prep_bwd(p(gops[0]), p(gepi[0]), p(gops[1]), p(gops[2]), p(gepi[1]),
                               p(gops[3]), p(gepi[2]), p(gops[4]), p(gops[5]), p(dvfo),
                               *[p(ins[n]) for n in ("wl", "k", "v", "vl", "al", "vf")], p(par),
                               p(dr), p(dwl), p(dk), p(dv), p(dvl), p(dal), p(dvf), p(dpar),
                               p(w), nw, B, T, C, stream()) == 0
    gsum = [gops[1].float(), gops[2].float() + gepi[1].float(), gops[3].float() + gepi[2].float(),
            gops[4].float(), gops[5].float()]
    loss = sum((o * gg).sum() for o, gg in zip(want, gsum))
    if not vres:
        loss = loss + (leaves["v"] * dvfo.float()).sum()   # v_first = v in layer 0
    loss.backward()
    close(dr, gops[0].float() + gepi[0].float(), 1e-2, "dr")
    close(dwl, leaves["wl"].grad, 1e-2, "dwl")
    close(dk, leaves["k"].grad, 1e-2, "dk")
    close(dv, leaves["v"].grad, 1e-2, "dv")
    close(dal, leaves["al"].grad, 1e-2, "dal")
    if vres:
        close(dvl, leaves["vl"].grad, 1e-2, "dvl")
        close(dvf, leaves["vf"].grad, 1e-2, "dv_first")
        close(dpar, parl.grad, 1e-4, "dparams")
    else:
        keep = [0, 2, 3, 4]  # v0 unused in layer 0
        close(dpar[keep], parl.grad[keep], 1e-4, "dparams")
        assert float(dpar[1].abs().max()) == 0.0


def post_ref(y, r, ko, vo, g, r_k, gamma, beta, H):
    """camoe/backbone.py:359-367 in fp32."""
    B, T, C = y.shape
    x = F.group_norm(y.view(B * T, C), H, gamma, beta, eps=64e-5).view(B, T, C)
    x = x + ((r.view(B, T, H, -1) * ko.view(B, T, H, -1) * r_k).sum(-1, keepdim=True)
             * vo.view(B, T, H, -1)).view(B, T, C)
    return x * g


@pytest.mark.parametrize("B,T,C", SHAPES)
def test_post_kernel(B, T, C):
    H = C // 64
    y, r, ko, vo, g = (rnd(B, T, C, seed=70 + i) for i in range(5))
    gen = torch.Generator().manual_seed(4)
    r_k = (-0.04 + 0.1 * torch.randn(H, 64, generator=gen)).cuda()
    gamma = (1 + 0.1 * torch.randn(C, generator=gen)).cuda()
    beta = (0.1 * torch.randn(C, generator=gen)).cuda()
    z = torch.empty(B, T, C, dtype=BF, device="cuda")
    L = _lib.lib()
    assert L.camoe_tm_post_fwd(p(y), p(r), p(ko), p(vo), p(g), p(r_k), p(gamma), p(beta), p(z),
                               B, T, C, stream()) == 0
    lv = [t.float().requires_grad_(True) for t in (y, r, ko, vo, g)]
    lp = [t.clone().requires_grad_(True) for t in (r_k, gamma, beta)]
    want = post_ref(*lv, *lp, H)
    close(z, want, 1e-2, "z")
    dz = rnd(B, T, C, seed=80)
    outs = [torch.empty(B, T, C, dtype=BF, device="cuda") for _ in range(5)]
    dpar = torch.empty(3, C, device="cuda")
    w, nw = work(B, T, C)
    assert L.camoe_tm_post_bwd(p(dz), p(y), p(r), p(ko), p(vo), p(g), p(r_k), p(gamma), p(beta),
                               *[p(o) for o in outs], p(dpar), p(w), nw, B, T, C, stream()) == 0
    want.backward(dz.float())
    for name, got, leaf in zip(("dy", "dr", "dk'", "dv'", "dg"), outs, lv):
        close(got, leaf.grad, 1e-2, name)
    close(dpar[0], lp[1].grad, 1e-4, "dgamma")
    close(dpar[1], lp[2].grad, 1e-4, "dbeta")
    close(dpar[2].view(H, 64), lp[0].grad, 1e-4, "dr_k")


@pytest.mark.parametrize("B,T,C", SHAPES)
def test_lnsa_kernel(B, T, C):
    sa = rnd(B, T, C, scale=3.0, seed=90, dtype=torch.float32) + 0.5
    gen = torch.Generator().manual_seed(5)
    wt = (1 + 0.1 * torch.randn(C, generator=gen)).cuda()
    bs = (0.1 * torch.randn(C, generator=gen)).cuda()
    out = torch.empty_like(sa)
    L = _lib.lib()
    assert L.camoe_tm_lnsa_fwd(p(sa), p(wt), p(bs), p(out), B, T, C, stream()) == 0
    sl = sa.clone().requires_grad_(True)
    wl_, bl = wt.clone().requires_grad_(True), bs.clone().requires_grad_(True)
    want = F.layer_norm(sl, (C,), wl_, bl, eps=1e-5)
    close(out, want, 1e-4, "ln_sa")
    dout = rnd(B, T, C, seed=91, dtype=torch.float32)
    dsa = torch.empty_like(sa)
    dpar = torch.empty(2, C, device="cuda")
    w, nw = work(B, T, C)
    assert L.camoe_tm_lnsa_bwd(p(dout), p(sa), p(wt), p(dsa), p(dpar), p(w), nw, B, T, C,
                               stream()) == 0
    want.backward(dout)
    close(dsa, sl.grad, 1e-4, "dsa")
    close(dpar[0], wl_.grad, 1e-4, "dweight")
    close(dpar[1], bl.grad, 1e-4, "dbias")


def test_backward_kernels_are_deterministic():
    B, T, C = 2, 48, 256
    y, r, ko, vo, g, dz = (rnd(B, T, C, seed=100 + i) for i in range(6))
    H = C // 64
    r_k, gamma, beta = torch.randn(H, 64).cuda(), torch.randn(C).cuda(), torch.randn(C).cuda()
    L = _lib.lib()
    w, nw = work(B, T, C)
    res = []
    for _ in range(2):
        outs = [torch.empty(B, T, C, dtype=BF, device="cuda") for _ in range(5)]
        dpar = torch.empty(3, C, device="cuda")
        assert L.camoe_tm_post_bwd(p(dz), p(y), p(r), p(ko), p(vo), p(g), p(r_k), p(gamma),
                                   p(beta), *[p(o) for o in outs], p(dpar), p(w), nw, B, T, C,
                                   stream()) == 0
        res.append([o.clone() for o in outs] + [dpar.clone()])
    for a, b in zip(*res):
        assert torch.equal(a, b)


# --------------------------------------------------------------------------
# the whole module against the reference module (float64 golden vectors)

def load_case(name):
    z = np.load(os.path.join(GOLDEN_DIR, name + ".npz"))
    B, T, C, n_layer, layer_id, seed = (int(v) for v in z["shape"])
    params = timemix_params(C, seed)
    inp = timemix_inputs(B, T, C, layer_id, seed)
    assert digest(params) == str(z["params_digest"]) and digest(inp) == str(z["inputs_digest"])
    return z, (B, T, C, n_layer, layer_id), params, inp


@pytest.mark.parametrize("xdt", [torch.float32, BF], ids=["x_fp32", "x_bf16"])
@pytest.mark.parametrize("case", sorted(CASES))
def test_module_matches_reference_module(case, xdt):
    z, (B, T, C, n_layer, layer_id), params, inp = load_case(case)
    tol = 3e-2
    mod = timemix.RWKV7TimeMix(C, n_layer, layer_id).cuda()
    mod.load_state_dict({k: torch.from_numpy(v) for k, v in params.items()})
    x = torch.from_numpy(inp["x"]).to(xdt).cuda().requires_grad_(True)
    vf = None
    if layer_id > 0:
        vf = torch.from_numpy(inp["v_first"]).to(BF).cuda().requires_grad_(True)
    out, vf_out, srep = mod(x, vf)
    close(out, torch.from_numpy(z["out"]), tol, "out")
    close(srep, torch.from_numpy(z["srep"]), tol, "state_representation")
    close(vf_out, torch.from_numpy(z["v_first_out"]), tol, "v_first")
    loss = (out.float() * torch.from_numpy(inp["d_out"]).cuda()).sum() + \
        (srep * torch.from_numpy(inp["d_srep"]).cuda()).sum()
    if layer_id == 0:
        loss = loss + (vf_out.float() * torch.from_numpy(inp["d_vf"]).cuda()).sum()
    loss.backward()
    close(x.grad, torch.from_numpy(z["grad_x"]), tol, "dx")
    if vf is not None:
        close(vf.grad, torch.from_numpy(z["grad_v_first"]), tol, "dv_first")
    checked = 0
    for k, prm in mod.named_parameters():
        if "grad_" + k in z.files:
            close(prm.grad.view(z["grad_" + k].shape), torch.from_numpy(z["grad_" + k]), tol, k)
            checked += 1
        elif "pgrad_" + k in z.files:
            got = grad_projection(prm.grad.detach().cpu().numpy())
            close(torch.from_numpy(got), torch.from_numpy(z["pgrad_" + k]), tol, k)
            checked += 1
        else:  # unused by this layer (v0, v1, v2 in layer 0)
            assert prm.grad is None or float(prm.grad.abs().max()) == 0.0, k
    assert checked >= 24


def _graph(fn):
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for _ in range(2):
            fn()
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        fn()
    return g


def test_op_forward_backward_replays_from_a_cuda_graph():
    """The op's forward and backward (chunked path: TMA descriptors, workspace
    and checkpoint from the caching allocator) captured in a CUDA graph and
    replayed give the eager results bit for bit."""
    from camoe_b200 import ops
    from camoe_b200.inputs import make_inputs
    inp = make_inputs(2, 256, 8, seed=7)
    xs = [inp[n].to(BF).cuda() for n in ("r", "w", "k", "v", "a", "b")]
    dy = inp["dy"].to(BF).cuda()
    y0, sa0, ck0 = ops.wkv7_forward(*xs)
    g0 = ops.wkv7_backward(*xs, dy, None, ck0)
    res = {}

    def step():
        y, sa, ck = ops.wkv7_forward(*xs)
        res["out"] = (y, sa) + tuple(ops.wkv7_backward(*xs, dy, None, ck))

    g = _graph(step)
    for t in res["out"]:
        t.zero_()
    g.replay()
    torch.cuda.synchronize()
    for got, want in zip(res["out"], (y0, sa0) + tuple(g0)):
        assert torch.equal(got, want)


def test_layer_replays_from_a_cuda_graph():
    """One fused time-mix layer, forward and backward, captured and replayed
    (as bench.py --workload timemix_b8_t1024_c1024 times it) matches the eager layer."""
    B, T, C = 2, 64, 256
    torch.manual_seed(3)
    m = timemix.RWKV7TimeMix(C, 4, 1).cuda()
    x = torch.randn(B, T, C, device="cuda", dtype=BF, requires_grad=True)
    vf = torch.randn(B, T, C, device="cuda", dtype=BF)
    d_out = torch.randn(B, T, C, device="cuda", dtype=BF)

    def step():
        x.grad = None
        out, _, srep = m(x, vf)
        torch.autograd.backward([out, srep], [d_out, torch.ones_like(srep)])
        return out

    out0 = step().detach().clone()
    gx0 = x.grad.detach().clone()
    res = {}

    def capt():
        res["out"] = step()

    g = _graph(capt)
    g.replay()
    torch.cuda.synchronize()
    close(res["out"], out0, 1e-3, "graph out")
    close(x.grad, gx0, 1e-3, "graph dx")


@pytest.mark.parametrize("layer_id", [0, 2])
def test_forward_state_prefill_then_decode_equals_one_pass(layer_id):
    """RWKV7TimeMix.forward_state: a 32-step prefill, then 16 single-token calls
    carrying (x_prev, wkv), give forward()'s outputs over all 48 steps."""
    B, T0, n, C = 2, 32, 16, 256
    torch.manual_seed(11)
    m = timemix.RWKV7TimeMix(C, 4, layer_id).cuda()
    with torch.no_grad():  # non-zero LoRA inputs and output projection
        for name in ("w1", "a1", "v1", "g1"):
            getattr(m, name).normal_(0, 0.1)
        m.output.weight.normal_(0, C ** -0.5)
    x = torch.randn(B, T0 + n, C, device="cuda", dtype=BF)
    vf = None if layer_id == 0 else torch.randn(B, T0 + n, C, device="cuda", dtype=BF)
    with torch.no_grad():
        out, vf_out, srep = m(x, vf)
    o1, v1, s1, state = m.forward_state(x[:, :T0], None if vf is None else vf[:, :T0])
    outs, srs, vfs = [o1], [s1], [v1]
    for t in range(T0, T0 + n):
        o, v_, s_, state = m.forward_state(x[:, t:t + 1], None if vf is None else vf[:, t:t + 1],
                                           state)
        outs.append(o)
        srs.append(s_)
        vfs.append(v_)
    torch.cuda.synchronize()
    close(torch.cat(outs, 1), out, 2e-2, "out")
    close(torch.cat(srs, 1), srep, 2e-2, "state_representation")
    close(torch.cat(vfs, 1), vf_out, 2e-2, "v_first")
    assert state[0].shape == (B, C) and state[1].shape == (B, C // 64, 64, 64)


# R = 5 and 1000: ragged last stages (rows past R load as zeros); D = 96 and
# 160 padded to 128 and 192 columns; D = 256 the largest rank; C = 128 one tile
@pytest.mark.parametrize("R,C,D,out_cd", [(5, 128, 96, 0), (1000, 128, 64, 1),
                                          (200, 256, 256, 1), (8192, 1024, 160, 1),
                                          (8192, 1024, 64, 0)])
def test_lora_wgrad(R, C, D, out_cd):
    """camoe_tm_lora_wgrad (tcgen05) against the product in float64, bit-identical
    on a second call (fixed-order reduction), and no bounded wait ran out."""
    g = torch.Generator().manual_seed(R + D)
    big = torch.randn(R, C, generator=g).to(BF).cuda()
    thin = torch.randn(R, D, generator=g).to(BF).cuda()
    L = _lib.lib()
    errs = L.camoe_wkv7_device_errors()
    nw = int(L.camoe_tm_lora_work_bytes(R, C, D))
    work = torch.empty(max(nw, 16), dtype=torch.uint8, device="cuda")
    outs = []
    for _ in range(2):
        dw = torch.full((C, D) if out_cd else (D, C), float("nan"), device="cuda")
        assert L.camoe_tm_lora_wgrad(p(big), p(thin), p(dw), out_cd, p(work), nw, R, C, D,
                                     stream()) == 0
        outs.append(dw)
    torch.cuda.synchronize()
    want = big.double().t() @ thin.double()
    close(outs[0], want if out_cd else want.t(), 1e-5, "dw")
    assert torch.equal(outs[0], outs[1])
    assert L.camoe_wkv7_device_errors() == errs


def test_weight_grad_routes_lora_shapes():
    """The time mix's weight gradients: LoRA shapes through the kernel, both
    orientations, and a square projection and a rank of 32 through cuBLAS,
    all against float64."""
    g = torch.Generator().manual_seed(7)
    for m, n in ((1024, 64), (160, 1024), (1024, 1024), (1024, 32)):
        a = torch.randn(3000, m, generator=g).to(BF).cuda()
        b = torch.randn(3000, n, generator=g).to(BF).cuda()
        got = timemix._weight_grad(a, b)
        assert got.dtype == torch.float32 and got.shape == (m, n)
        close(got, a.double().t() @ b.double(), 1e-5, f"{m}x{n}")
