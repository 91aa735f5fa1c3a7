"""Generate the golden vectors under tests/golden/ from the REFERENCE itself.

Runs the reference's own CPU recurrence ``RWKV7_TimeMix._run_torch_fallback``
(camoe/backbone.py:250-294, imported from the reference checkout) in float32
and takes the six input gradients from torch.autograd through it.  The
recurrence computes ``sa`` at every step (camoe/backbone.py:284) but returns
only y, so ``sa`` is captured from the reference's own calls: a
TorchFunctionMode records the result of every ``Tensor.sum(dim=-1)`` made
inside the function, which per step are sa_t (:284) and then y_t (:290).  The
reference has no tests or stored vectors for this op, so these fixtures are
what pins the oracle (tests/test_oracle.py) to the reference's behaviour.

Inputs are not stored: they are regenerated from the seed with
camoe_b200.inputs.make_inputs, and a checksum of them is stored and checked.

Usage (needs the reference checkout, so it runs only in the build container):
    python tests/golden/make_golden.py [/path/to/reference]
"""
import hashlib
import os
import sys

import numpy as np
import torch
from torch.overrides import TorchFunctionMode

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
from camoe_b200.inputs import make_inputs  # noqa: E402

CASES = {
    # name: (B, T, H, seed, w_mu, w_sigma)
    "cpu_small_seed0": (1, 64, 2, 0, 0.0, 1.0),        # the op's CPU-sized workload
    "slow_decay_seed1": (1, 64, 1, 1, 2.0, 0.5),       # long-context decay distribution
    "ragged_t40_seed2": (2, 40, 1, 2, 0.0, 1.0),       # T not a multiple of 16
    "single_chunk_seed3": (3, 16, 1, 3, 0.0, 1.0),     # one 16-step chunk, B > 1
    "extreme_decay_seed4": (1, 48, 1, 4, 0.0, 6.0),    # decays at both clamps
}


def input_digest(inp: dict) -> str:
    h = hashlib.sha256()
    for n in ("r", "w", "k", "v", "a", "b", "dy"):
        h.update(np.ascontiguousarray(inp[n].numpy(), dtype=np.float32).tobytes())
    return h.hexdigest()


class RowSumRecorder(TorchFunctionMode):
    """Records the output of every ``Tensor.sum(dim=-1)`` call made under it."""

    def __init__(self):
        super().__init__()
        self.sums = []

    def __torch_function__(self, func, types, args=(), kwargs=None):
        kwargs = kwargs or {}
        out = func(*args, **kwargs)
        if func is torch.Tensor.sum and kwargs.get("dim") == -1:
            self.sums.append(out.detach().clone())
        return out


def main():
    ref_root = sys.argv[1] if len(sys.argv) > 1 else "/root/reference"
    sys.path.insert(0, ref_root)
    from camoe.backbone import RWKV7_TimeMix  # the reference's fallback recurrence

    torch.set_num_threads(max(1, os.cpu_count() or 1))
    for name, (B, T, H, seed, mu, sig) in CASES.items():
        N = 64
        inp = make_inputs(B, T, H, N, seed=seed, w_mu=mu, w_sigma=sig)
        xs = [inp[n].reshape(B, T, H * N).clone().requires_grad_(True)
              for n in ("r", "w", "k", "v", "a", "b")]
        rec = RowSumRecorder()
        with rec:
            y = RWKV7_TimeMix._run_torch_fallback(*xs, H, N)
        assert len(rec.sums) == 2 * T, "expected the sa and y row sums of every step"
        sa = torch.stack(rec.sums[0::2], dim=1)  # [B, T, H, N]: sa_t of :284
        y_rows = torch.stack(rec.sums[1::2], dim=1)  # y_t of :290, a check of the capture
        assert torch.equal(y_rows.reshape(B, T, H * N), y.detach())
        (y * inp["dy"].reshape(B, T, H * N)).sum().backward()
        out = {"y": y.detach().reshape(B, T, H, N).numpy(), "sa": sa.numpy()}
        for n, x in zip(("dr", "dw", "dk", "dv", "da", "db"), xs):
            out[n] = x.grad.reshape(B, T, H, N).numpy()
        np.savez_compressed(os.path.join(HERE, f"{name}.npz"),
                            shape=np.array([B, T, H, N]), seed=seed, w_mu=mu, w_sigma=sig,
                            input_sha256=input_digest(inp), **out)
        print(name, {k: float(np.abs(v).max()) for k, v in out.items()})


if __name__ == "__main__":
    main()
