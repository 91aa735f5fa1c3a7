"""Shared test helpers: error metrics and fixture loading."""
import glob
import os

import numpy as np

GOLDEN_DIR = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
GRADS = ("dr", "dw", "dk", "dv", "da", "db")

# Norm-relative max error bars: max|x - ref| / max|ref| per output tensor.
TOL_FP32 = 1e-4
TOL_BF16 = 2e-2


def nrel(x, ref) -> float:
    x = np.asarray(x, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    denom = np.abs(ref).max()
    if denom == 0:
        return float(np.abs(x).max())
    return float(np.abs(x - ref).max() / denom)


def golden_cases():
    """The op's fixtures (make_golden.py); the time mix (timemix_*) and the
    CaMoE train-step call site (camoe_step_*) have their own."""
    return sorted(f for f in glob.glob(os.path.join(GOLDEN_DIR, "*.npz"))
                  if not os.path.basename(f).startswith(("timemix_", "camoe_step_")))


def load_golden(path):
    import torch  # noqa: F401  (make_inputs needs torch)
    from camoe_b200.inputs import make_inputs

    z = np.load(path)
    B, T, H, N = (int(v) for v in z["shape"])
    inp = make_inputs(B, T, H, N, seed=int(z["seed"]), w_mu=float(z["w_mu"]),
                      w_sigma=float(z["w_sigma"]))
    return z, inp


def input_digest(inp) -> str:
    import hashlib
    h = hashlib.sha256()
    for n in ("r", "w", "k", "v", "a", "b", "dy"):
        h.update(np.ascontiguousarray(inp[n].numpy(), dtype=np.float32).tobytes())
    return h.hexdigest()
