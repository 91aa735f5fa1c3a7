"""CPU checks of the fused time mix: module layout against the reference's
RWKV7_TimeMix (parameter names and shapes as in the golden vectors made from
the reference module), the golden fixtures themselves, the initialisation,
and C-ABI argument validation that needs no device."""
import ctypes
import os
import sys

import numpy as np
import pytest
import torch

from camoe_b200 import _lib, timemix
from helpers import GOLDEN_DIR

sys.path.insert(0, GOLDEN_DIR)
from make_timemix_golden import CASES, digest, timemix_inputs, timemix_params  # noqa: E402


@pytest.mark.parametrize("case", sorted(CASES))
def test_golden_fixture_and_state_dict_layout(case):
    z = np.load(os.path.join(GOLDEN_DIR, case + ".npz"))
    B, T, C, n_layer, layer_id, seed = (int(v) for v in z["shape"])
    params = timemix_params(C, seed)
    assert digest(params) == str(z["params_digest"])
    assert digest(timemix_inputs(B, T, C, layer_id, seed)) == str(z["inputs_digest"])
    mod = timemix.RWKV7TimeMix(C, n_layer, layer_id)
    sd = mod.state_dict()
    assert set(sd) == set(params)                      # the reference's names
    for k, v in params.items():
        assert tuple(sd[k].shape) == v.shape, k        # and shapes
    mod.load_state_dict({k: torch.from_numpy(v) for k, v in params.items()})
    for k in sd:
        if k.startswith("v") and layer_id == 0 and k in ("v0", "v1", "v2"):
            assert "grad_" + k not in z.files and "pgrad_" + k not in z.files
        else:
            assert ("grad_" + k in z.files) or ("pgrad_" + k in z.files), k


def test_initialisation_follows_rwkv7():
    C, n_layer = 256, 6
    m0 = timemix.RWKV7TimeMix(C, n_layer, 0)
    m5 = timemix.RWKV7TimeMix(C, n_layer, 5)
    d = timemix.lora_dims(C)
    assert m0.w1.shape == (C, d["decay"]) and m0.g2.shape == (d["gate"], C)
    assert d == {"decay": 32, "aaa": 32, "mv": 32, "gate": 64}  # Python round(2.5) == 2
    assert timemix.lora_dims(1024) == {"decay": 64, "aaa": 64, "mv": 64, "gate": 160}
    for m in (m0, m5):
        assert float(m.output.weight.abs().max()) == 0.0     # zero output projection
        for n in ("w1", "a1", "v1", "g1"):
            assert float(getattr(m, n).abs().max()) == 0.0   # zero LoRA inputs
        assert float(m.k_a.min()) == pytest.approx(1.02) and float(m.r_k.max()) == pytest.approx(-0.04)
        assert float(m.receptance.weight.abs().max()) <= 0.5 * C ** -0.5
    # token-shift mixes 1 - (c / C)^(p (1 - layer / n_layer)), p = 0.2 for x_r
    c = torch.arange(C, dtype=torch.float32) / C
    for m, lid in ((m0, 0), (m5, 5)):
        want = 1.0 - torch.pow(c, 0.2 * (1.0 - lid / n_layer))
        assert torch.allclose(m.x_r.detach().view(C), want)
    assert float(m0.ln_x.eps) == 64e-5


def test_timemix_abi_rejects_bad_arguments_without_a_device():
    L = _lib.lib()
    p = ctypes.c_void_p(16)
    outs = (ctypes.c_void_p * 6)(*([16] * 6))
    assert L.camoe_tm_work_bytes(2, 40, 100) == 0                       # C not a multiple of 64
    assert L.camoe_tm_work_bytes(2, 40, 128) > 0
    assert L.camoe_tm_mix_fwd(p, 0, p, outs, 2, 40, 96, None) == _lib.ERR_UNSUPPORTED
    assert L.camoe_tm_mix_fwd(p, 0, p, outs, 2, 40, 4096, None) == _lib.ERR_UNSUPPORTED
    assert L.camoe_tm_mix_fwd(p, 7, p, outs, 2, 40, 128, None) == _lib.ERR_UNSUPPORTED
    assert L.camoe_tm_mix_fwd(None, 0, p, outs, 2, 40, 128, None) == _lib.ERR_INVALID_ARG
    assert L.camoe_tm_mix_fwd(ctypes.c_void_p(24), 0, p, outs, 2, 40, 128, None) == _lib.ERR_ALIGNMENT
    assert L.camoe_tm_mix_fwd(p, 0, p, outs, 0, 40, 128, None) == _lib.OK   # empty: no launch
    # the carried token-shift row is optional but must be aligned when given
    assert L.camoe_tm_mix_fwd_prev(p, 0, ctypes.c_void_p(40), p, outs, 2, 40, 128, None) == _lib.ERR_ALIGNMENT
    assert L.camoe_tm_mix_fwd_prev(p, 0, None, p, outs, 0, 40, 128, None) == _lib.OK
    assert L.camoe_tm_lnsa_fwd(p, p, p, p, -1, 4, 128, None) == _lib.ERR_INVALID_ARG
    # prep: value-residual inputs come as a pair
    assert L.camoe_tm_prep_fwd(p, p, p, p, p, None, p, p, p, p, p, p, 2, 40, 128, None) == _lib.ERR_INVALID_ARG
    # backward: workspace too small
    args = [p] * 15
    assert L.camoe_tm_post_bwd(*args, p, 8, 2, 40, 128, None) == _lib.ERR_WORKSPACE
    assert L.camoe_tm_post_bwd(*args, None, 1 << 30, 2, 40, 128, None) == _lib.ERR_INVALID_ARG
