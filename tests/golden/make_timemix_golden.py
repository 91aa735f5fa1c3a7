"""Golden vectors of the whole RWKV-7 time mix, from the REFERENCE module.

Builds the reference's ``RWKV7_TimeMix`` (camoe/backbone.py:134-373, imported
from the reference checkout), sets every parameter to seeded values
(``timemix_params``: the reference initialises the LoRA inputs and the output
projection to zero, which would leave those gradient paths untested), and
runs its own forward in float64 on the CPU with its WKV-7 call
(``RUN_CUDA_RWKV7``, backbone.py:347) bound to a float64 torch statement of
the op's recurrence (the reference's fallback recurrence does not return
``sa``, which ``ln_sa`` needs).  Gradients come from torch.autograd of
    sum(out * d_out) + sum(state_representation * d_srep) [+ sum(v_first_out * d_vf)]
with respect to x, v_first (layers > 0) and every parameter.

Stored per case: the outputs and all gradients (float32), the matrix
gradients as projections (``grad_projection``).  Parameters and
inputs are regenerated from the seed by ``timemix_params`` / ``timemix_inputs``
(imported by the tests), with a checksum stored and checked.

Usage (needs the reference checkout, so it runs only in the build container):
    python tests/golden/make_timemix_golden.py [/path/to/reference]
"""
import hashlib
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))

CASES = {
    # name: (B, T, C, n_layer, layer_id, seed)
    "timemix_layer0_c128": (1, 32, 128, 4, 0, 0),
    "timemix_layer2_c128": (1, 32, 128, 4, 2, 1),
}
PROJ = 8  # random directions a matrix gradient is stored along


def grad_projection(g):
    """A 2-D gradient [m, n] stored as g @ P, P a seeded [n, PROJ] Gaussian
    matrix (the same for every n): a weight gradient that is wrong anywhere
    changes it, at PROJ/n of the size."""
    P = np.random.default_rng(5000 + g.shape[1]).standard_normal((g.shape[1], PROJ))
    return (np.asarray(g, dtype=np.float64) @ P).astype(np.float32)

def lora_dims(C):
    def r(f):
        return max(32, int(round((f * C ** 0.5) / 32) * 32))
    return {"decay": r(2.5), "aaa": r(2.5), "mv": r(1.7), "gate": r(5.0)}


def timemix_params(C, seed):
    """Seeded parameter values with the reference's names and shapes."""
    g = np.random.default_rng(1000 + seed)
    H, N = C // 64, 64
    d = lora_dims(C)
    n = (lambda *s: g.standard_normal(s).astype(np.float32))
    p = {}
    for m in ("x_r", "x_w", "x_k", "x_v", "x_a", "x_g"):
        p[m] = g.uniform(0.0, 1.0, (1, 1, C)).astype(np.float32)
    p["w0"] = (-2.0 + 1.5 * n(1, 1, C)).astype(np.float32)
    p["a0"] = (0.3 * n(1, 1, C)).astype(np.float32)
    p["v0"] = (0.5 + 0.3 * n(1, 1, C)).astype(np.float32)
    p["k_k"] = (0.71 + 0.1 * n(1, 1, C)).astype(np.float32)
    p["k_a"] = (1.02 + 0.1 * n(1, 1, C)).astype(np.float32)
    p["r_k"] = (-0.04 + 0.1 * n(H, N)).astype(np.float32)
    for a, b, key in (("w1", "w2", "decay"), ("a1", "a2", "aaa"), ("v1", "v2", "mv"),
                      ("g1", "g2", "gate")):
        p[a] = (0.1 * n(C, d[key])).astype(np.float32)
        p[b] = (0.1 * n(d[key], C)).astype(np.float32)
    for lin in ("receptance", "key", "value", "output"):
        p[lin + ".weight"] = (C ** -0.5 * n(C, C)).astype(np.float32)
    for ln in ("ln_x", "ln_sa"):
        p[ln + ".weight"] = (1.0 + 0.1 * n(C)).astype(np.float32)
        p[ln + ".bias"] = (0.1 * n(C)).astype(np.float32)
    return p


def timemix_inputs(B, T, C, layer_id, seed):
    """x, v_first (layers > 0) and the output gradients, float32."""
    g = np.random.default_rng(2000 + seed)
    n = (lambda *s: g.standard_normal(s).astype(np.float32))
    out = {"x": n(B, T, C), "d_out": n(B, T, C), "d_srep": n(B, T, C)}
    if layer_id > 0:
        out["v_first"] = (0.5 * n(B, T, C)).astype(np.float32)
    else:
        out["d_vf"] = n(B, T, C)
    return out


def digest(arrays):
    h = hashlib.sha256()
    for k in sorted(arrays):
        h.update(k.encode())
        h.update(np.ascontiguousarray(arrays[k], dtype=np.float32).tobytes())
    return h.hexdigest()


def op64(r, w, k, v, a, b):
    """Float64 WKV-7 ClampW recurrence on [B, T, C] tensors -> (y, sa), the
    recurrence of camoe/backbone.py:264-294 with sa returned."""
    import torch
    B, T, C = r.shape
    H = C // 64
    rr, ww, kk, vv, aa, bb = (t.reshape(B, T, H, 64) for t in (r, w, k, v, a, b))
    dec = torch.exp(-np.exp(-0.5) * torch.sigmoid(ww))
    S = torch.zeros(B, H, 64, 64, dtype=r.dtype)
    ys, sas = [], []
    for t in range(T):
        sa = (S * aa[:, t].unsqueeze(-2)).sum(-1)
        S = S * dec[:, t].unsqueeze(-2) + sa.unsqueeze(-1) * bb[:, t].unsqueeze(-2) \
            + vv[:, t].unsqueeze(-1) * kk[:, t].unsqueeze(-2)
        ys.append((S * rr[:, t].unsqueeze(-2)).sum(-1))
        sas.append(sa)
    return torch.stack(ys, 1).reshape(B, T, C), torch.stack(sas, 1).reshape(B, T, C)


def main():
    import torch
    ref_root = sys.argv[1] if len(sys.argv) > 1 else "/root/reference"
    sys.path.insert(0, ref_root)
    import camoe.backbone as rb

    torch.set_num_threads(max(1, os.cpu_count() or 1))
    rb.USE_CUDA = True
    rb.RUN_CUDA_RWKV7 = op64
    os.environ["CAMOE_FORCE_TIMEMIX_FALLBACK"] = "0"
    for name, (B, T, C, n_layer, layer_id, seed) in CASES.items():
        mod = rb.RWKV7_TimeMix(C, n_layer, layer_id, 64).double()
        params = timemix_params(C, seed)
        sd = mod.state_dict()
        assert set(sd) == set(params), sorted(set(sd) ^ set(params))
        mod.load_state_dict({k: torch.from_numpy(v).double() for k, v in params.items()})
        inp = timemix_inputs(B, T, C, layer_id, seed)
        x = torch.from_numpy(inp["x"]).double().requires_grad_(True)
        vf = None
        if layer_id > 0:
            vf = torch.from_numpy(inp["v_first"]).double().requires_grad_(True)
        out, vf_out, srep = mod(x, vf)
        loss = (out * torch.from_numpy(inp["d_out"]).double()).sum() + \
            (srep * torch.from_numpy(inp["d_srep"]).double()).sum()
        if layer_id == 0:
            loss = loss + (vf_out * torch.from_numpy(inp["d_vf"]).double()).sum()
        loss.backward()
        rec = {"shape": np.array([B, T, C, n_layer, layer_id, seed]),
               "params_digest": np.array(digest(params)),
               "inputs_digest": np.array(digest(inp)),
               "out": out.detach().float().numpy(), "srep": srep.detach().float().numpy(),
               "v_first_out": vf_out.detach().float().numpy(),
               "grad_x": x.grad.float().numpy()}
        if vf is not None:
            rec["grad_v_first"] = vf.grad.float().numpy()
        for k, p in mod.named_parameters():
            if p.grad is None:  # v0, v1, v2 are unused in layer 0
                continue
            gk = p.grad.numpy()
            if gk.ndim == 2 and k != "r_k":
                rec["pgrad_" + k] = grad_projection(gk)
            else:
                rec["grad_" + k] = gk.astype(np.float32)
        np.savez_compressed(os.path.join(HERE, name + ".npz"), **rec)
        print(name, "max|out| %.3g max|srep| %.3g" % (float(out.detach().abs().max()),
                                                      float(srep.detach().abs().max())))


if __name__ == "__main__":
    main()
