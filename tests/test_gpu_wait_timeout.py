"""A bounded device wait that runs out returns instead of hanging.

Every pipeline wait of the chunked kernels gives up after a limit, counts the
event (camoe_wkv7_device_errors) and makes the kernel's roles leave their
loops (camoe_b200/csrc/wkv7_sync.cuh).  Here the test hook lowers the limit to
a few milliseconds and makes the forward's value-pass producer withhold one
pair of chunks, so that every role's next wait runs out on a tiny problem.
The call must return (no hang, no fault), the error counter must grow, and
the next ordinary call must be correct with no further timeouts.  Nothing here
traps, asserts on the device or reads out of bounds: the withheld pair simply
never arrives.
"""
import pytest
import torch

import oracle
from camoe_b200 import _lib, ops
from camoe_b200.inputs import make_inputs
from helpers import TOL_BF16, nrel

pytestmark = pytest.mark.gpu

NAMES = ("r", "w", "k", "v", "a", "b")
SHORT_LIMIT = 4_000_000  # clock cycles: about 2 ms at 1.9 GHz


def hooks(limit, skip):
    _lib.check(_lib.lib().camoe_wkv7_test_hooks(limit, skip))


def test_withheld_chunk_pair_times_out_and_the_next_call_is_correct():
    inp = make_inputs(1, 256, 1, seed=91)  # 16 chunks = 8 pairs, one chain
    xs = [inp[n].to(torch.bfloat16).cuda() for n in NAMES]
    L = _lib.lib()
    torch.cuda.synchronize()
    before = L.camoe_wkv7_device_errors()
    try:
        hooks(SHORT_LIMIT, 1)
        ops.wkv7_forward(*xs, algo="chunked")
        torch.cuda.synchronize()  # returns: the waits ran out instead of spinning
    finally:
        hooks(_lib.DEFAULT_WAIT_LIMIT, -1)
    after = L.camoe_wkv7_device_errors()
    assert after != 0xFFFFFFFF
    assert after > before, "the withheld pair must have made waits run out"

    # the context is still usable and the op correct, with no new timeouts
    y, sa, ck = ops.wkv7_forward(*xs, algo="chunked")
    dy = inp["dy"].to(torch.bfloat16).cuda()
    grads = ops.wkv7_backward(*xs, dy, None, ck, algo="chunked")
    torch.cuda.synchronize()
    assert L.camoe_wkv7_device_errors() == after
    rx = [inp[n].to(torch.bfloat16).float() for n in NAMES + ("dy",)]
    want = list(oracle.fwd(*rx[:6])) + list(oracle.bwd(*rx))
    got = [t.float().cpu().numpy() for t in (y, sa) + tuple(grads)]
    for name, g, w in zip(("y", "sa", "dr", "dw", "dk", "dv", "da", "db"), got, want):
        assert nrel(g, w) < TOL_BF16, name
