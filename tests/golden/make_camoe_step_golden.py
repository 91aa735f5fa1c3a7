"""Golden vectors of the WKV-7 op at its call site inside the REFERENCE's own
CaMoE train step.

Builds the reference's ``CaMoE_System`` (camoe/system.py:358-540, imported
from the reference checkout) at a tiny size -- the 0.4B configuration of
camoe/config.py:172-260 with n_embd=128 (2 heads of 64), 2 layers, a 512-token
vocabulary, prefix_len 8 and low_rank_dim 16; 6 RWKV + 2 Transformer experts,
top-2 routing, gradient checkpointing of the attention stage on -- and runs one
training step as train.py:726-774 does: ``model(x)``, ``compute_losses``,
``backward``.  The op's call site, ``RUN_CUDA_RWKV7(r, w, k, v, -kk, kk*a)``
in ``RWKV7_TimeMix.forward`` (camoe/backbone.py:345-348), is bound to a
recorder around the reference's own CPU recurrence ``_run_torch_fallback``
(camoe/backbone.py:250-294), with sa captured from its per-step row sums as
make_golden.py does, so the model runs the CUDA path's semantics (sa feeds
``ln_sa`` -> state_representation -> bridge and experts) on the CPU.

The time mix's output projection and LoRA input matrices are drawn from a
seeded normal distribution first (at initialisation the output projection is
zero, camoe/backbone.py:89, so no gradient would reach y).

Recorded per call: the six inputs as the model passes them ([B, T, C] fp32),
y and sa; for the calls that receive gradients, the gradients of y and sa
flowing back from the rest of the model (dy, dsa) and the six input
gradients.  The activation-checkpoint recompute (camoe/system.py:317-324)
calls the op a second time per layer; its inputs are checked to equal the
first call's and are not stored again.  ``torch.compile`` (used by the
reference's bridge, critic and experts) is disabled while generating, which
changes no arithmetic.

Usage (needs the reference checkout, so it runs only in the build container):
    TORCHDYNAMO_DISABLE=1 python tests/golden/make_camoe_step_golden.py [/path/to/reference]
"""
import os
import sys

import numpy as np
import torch
from torch.overrides import TorchFunctionMode

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "camoe_step_c128_l2.npz")
SEED = 7
B, T = 1, 64
SIZES = dict(n_embd=128, n_layer=2, vocab_size=512, prefix_len=8, low_rank_dim=16)


class RowSums(TorchFunctionMode):
    """Keeps the result of every ``Tensor.sum(dim=-1)`` (still in the graph)."""

    def __init__(self):
        super().__init__()
        self.sums = []

    def __torch_function__(self, func, types, args=(), kwargs=None):
        kwargs = kwargs or {}
        out = func(*args, **kwargs)
        if func is torch.Tensor.sum and kwargs.get("dim") == -1:
            self.sums.append(out)
        return out


def main():
    if os.environ.get("TORCHDYNAMO_DISABLE") != "1":
        sys.exit("run with TORCHDYNAMO_DISABLE=1 (the reference compiles its modules)")
    ref_root = sys.argv[1] if len(sys.argv) > 1 else "/root/reference"
    sys.path.insert(0, ref_root)
    import camoe.backbone as bb
    from camoe.config import CONFIG_04B
    from camoe.system import CaMoE_System

    calls = []
    fallback = bb.RWKV7_TimeMix._run_torch_fallback

    class RecordedOp(torch.autograd.Function):
        @staticmethod
        def forward(ctx, r, w, k, v, a, b):
            Bn, Tn, C = r.shape
            # the inner graph keeps its own saved tensors (identity hooks), so the
            # activation checkpoint does not recompute the layer again to unpack them
            with torch.enable_grad(), torch.autograd.graph.saved_tensors_hooks(lambda t: t,
                                                                              lambda t: t):
                xs = [t.detach().requires_grad_(True) for t in (r, w, k, v, a, b)]
                rs = RowSums()
                with rs:
                    y = fallback(*xs, C // 64, 64)
                # per step: sa_t (camoe/backbone.py:284), then y_t (:290)
                assert len(rs.sums) == 2 * Tn
                sa = torch.stack(rs.sums[0::2], dim=1).reshape(Bn, Tn, C)
            ctx.xs, ctx.outs, ctx.idx = xs, (y, sa), len(calls)
            calls.append({"inputs": [t.detach().clone() for t in (r, w, k, v, a, b)],
                          "y": y.detach().clone(), "sa": sa.detach().clone()})
            return y.detach().clone(), sa.detach().clone()

        @staticmethod
        def backward(ctx, dy, dsa):
            gs = torch.autograd.grad(ctx.outs, ctx.xs, grad_outputs=(dy, dsa))
            calls[ctx.idx].update(dy=dy.detach().clone(), dsa=dsa.detach().clone(),
                                  grads=[g.detach().clone() for g in gs])
            return gs

    bb.USE_CUDA = True
    bb.RUN_CUDA_RWKV7 = lambda r, w, k, v, a, b: RecordedOp.apply(r, w, k, v, a, b)

    cfg = dict(CONFIG_04B)
    cfg.update(SIZES)
    torch.manual_seed(SEED)
    model = CaMoE_System(cfg)
    # move the time mix off its initialisation, as after some training: the
    # output projection starts at zero (camoe/backbone.py:89), which would make
    # the gradient of y exactly zero, and the LoRA inputs start at zero
    gp = torch.Generator().manual_seed(SEED + 2)
    with torch.no_grad():
        for blk in model.blocks:
            att = blk.att
            att.output.weight.copy_(torch.randn(att.output.weight.shape, generator=gp)
                                    * cfg["n_embd"] ** -0.5)
            for n in ("w1", "a1", "v1", "g1"):
                prm = getattr(att, n)
                prm.copy_(0.1 * torch.randn(prm.shape, generator=gp))
    model.train()
    g = torch.Generator().manual_seed(SEED + 1)
    idx = torch.randint(0, cfg["vocab_size"], (B, T + 1), generator=g)
    x, y = idx[:, :-1], idx[:, 1:]
    logits, info = model(x, step=0, phase="normal")
    total, _, main_loss, critic, aux = model.compute_losses(logits, y, info)
    total.backward()

    L = cfg["n_layer"]
    assert len(calls) == 2 * L, f"expected a forward and a recompute call per layer, got {len(calls)}"
    out = {"seed": SEED, "shape": np.array([B, T, cfg["n_embd"]]), "n_layer": L,
           "tokens": idx.numpy(), "total_loss": float(total.detach()),
           "main_loss": float(main_loss.detach())}
    with_grad = [c for c in calls if "dy" in c]
    assert len(with_grad) == L, "one call per layer receives the gradients"
    for layer in range(L):
        # the backward recomputes the layers last to first
        fwd, rec = calls[layer], calls[2 * L - 1 - layer]
        for a_, b_ in zip(fwd["inputs"], rec["inputs"]):
            assert torch.equal(a_, b_), "the recompute must see the forward's inputs"
        assert torch.equal(fwd["y"], rec["y"]) and torch.equal(fwd["sa"], rec["sa"])
        gc = fwd if "dy" in fwd else rec
        pre = f"l{layer}_"
        for n, t in zip("rwkvab", fwd["inputs"]):
            out[pre + n] = t.numpy()
        out[pre + "y"], out[pre + "sa"] = fwd["y"].numpy(), fwd["sa"].numpy()
        out[pre + "dy"], out[pre + "dsa"] = gc["dy"].numpy(), gc["dsa"].numpy()
        for n, t in zip(("dr", "dw", "dk", "dv", "da", "db"), gc["grads"]):
            out[pre + n] = t.numpy()
    np.savez_compressed(OUT, **out)
    print(OUT, {k: (float(np.abs(v).max()) if isinstance(v, np.ndarray) and v.dtype.kind == "f"
                    else v) for k, v in out.items() if not k.endswith(("_r", "_w", "_k", "_v"))})


if __name__ == "__main__":
    main()
