"""Seeded synthetic inputs for the WKV-7 ClampW op.

The distributions follow the op's workloads: r, k, v, u, dy, w_in and kk are
standard normal draws of shape [B, T, H*N], made in that order from one CPU
``torch.Generator`` seeded with ``seed``; ``w_in = mu + sigma * w_in``; kk is
L2-normalised per head; then ``a = -kk`` and ``b = kk * sigmoid(u)``, which is
how ``RWKV7_TimeMix.forward`` builds the op's a/b arguments
(camoe/backbone.py:340-347).  The state starts at zero.
"""
from __future__ import annotations

import torch

NAMES = ("r", "w", "k", "v", "a", "b")


def make_inputs(B: int, T: int, H: int, N: int = 64, seed: int = 0, w_mu: float = 0.0,
                w_sigma: float = 1.0, dtype: torch.dtype = torch.float32,
                device: str | torch.device = "cpu", with_dsa: bool = False,
                decay: str = "clampw") -> dict:
    """Return dict(r, w, k, v, a, b, dy[, dsa]) of [B, T, H, N] contiguous tensors.

    ``w`` is the raw decay input w_in (the op applies exp(-e^{-1/2} sigmoid(w_in))).
    With ``decay="wind"`` it is -softplus(-x) - 1/2 of the same draw x, the input
    RWKV-7's time mix gives a decay exp(-exp(w_in)) (camoe/backbone.py:326).
    Values are drawn in float32 on the CPU and then cast, so every dtype and
    device sees the same numbers up to rounding.
    """
    g = torch.Generator().manual_seed(seed)
    C = H * N

    def randn():
        return torch.randn(B, T, C, generator=g, dtype=torch.float32)

    r, k, v, u, dy, w_in, kk = (randn() for _ in range(7))
    w_in = w_mu + w_sigma * w_in
    if decay == "wind":
        w_in = -torch.nn.functional.softplus(-w_in) - 0.5
    kk = torch.nn.functional.normalize(kk.view(B, T, H, N), dim=-1, p=2.0)
    a = -kk
    b = kk * torch.sigmoid(u.view(B, T, H, N))
    out = {"r": r.view(B, T, H, N), "w": w_in.view(B, T, H, N), "k": k.view(B, T, H, N),
           "v": v.view(B, T, H, N), "a": a, "b": b, "dy": dy.view(B, T, H, N)}
    if with_dsa:
        out["dsa"] = torch.randn(B, T, C, generator=g, dtype=torch.float32).view(B, T, H, N)
    return {n: x.to(dtype=dtype if n != "dsa" else torch.float32).contiguous().to(device)
            for n, x in out.items()}


# Named workloads of the op (sizes of one GPU's share where a workload is sharded).
WORKLOADS = {
    "cpu_small": dict(B=1, T=64, H=2, N=64, w_mu=0.0, w_sigma=1.0),
    "layer_b8_t1024": dict(B=8, T=1024, H=16, N=64, w_mu=0.0, w_sigma=1.0),
    "shard_b4_t4096": dict(B=4, T=4096, H=16, N=64, w_mu=0.0, w_sigma=1.0),
    "long_b2_t65536": dict(B=2, T=65536, H=32, N=64, w_mu=2.0, w_sigma=0.5),
}
