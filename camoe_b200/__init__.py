"""B200-native (sm_100a) WKV-7 ClampW operator for CaMoE's RWKV-7 TimeMix.

Public entry points:

* ``camoe_b200.backbone`` — drop-in for the op section of the reference's
  camoe/backbone.py (``init_rwkv7_cuda``, ``RWKV7_ClampW``, ``RUN_CUDA_RWKV7``).
* ``camoe_b200.ops`` — ``wkv7_forward`` / ``wkv7_backward`` on [B, T, H, 64]
  CUDA tensors (any T, head ranges, algorithm choice).
* ``camoe_b200.launcher`` — one-process-per-GPU batch/head sharding.
* ``include/camoe_wkv7.h`` — the C ABI underneath, for non-Python callers.
"""
from . import ops  # noqa: F401
from ._lib import CamoeError  # noqa: F401

__all__ = ["ops", "CamoeError"]
