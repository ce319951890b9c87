"""Failure detection on the device without a GPU fault (needs a B200).

Every wait inside the selection kernel is bounded.  Here the bound is set to 1 ns, so the waits
that do not succeed at once run out: the kernel must unwind cleanly (no trap, no hang), record
the expiry in the device error word, and leave the context usable -- the next normal call on
the same device runs to the right answer and reports no error.
"""
import ctypes

import pytest
import torch

from sta import _lib as L
from sta import core
from sta.core import Geometry
from sta.synth import SynthSpec, make_inputs, rope_inv_freq

pytestmark = pytest.mark.gpu


def test_expired_wait_reports_timeout_and_context_survives():
    H, Hk, N, D, T = 8, 2, 4096, 128, 64
    q, k, _ = make_inputs(SynthSpec(n_heads=H, n_kv_heads=Hk, seq_len=N, head_dim=D,
                                    n_planted=16, seed=11, dtype=torch.bfloat16))
    q, k = q[0].cuda(), k[0].cuda()
    g = Geometry(rope_inv_freq(D, 1e4), 1.0, 1.0)
    tau = torch.full((H,), 5.0)
    assert core.device_error() == 0  # clean start (the read also clears the word)
    good = core.select(q, k, tau, g, tile=T)
    torch.cuda.synchronize()
    assert core.device_error() == 0

    core.select(q, k, tau, g, tile=T, wait_limit_ns=1)
    torch.cuda.synchronize()  # the kernel returned: it unwound instead of hanging
    lib = L.lib()
    code = L.c_i32(0)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    rc = lib.sta_device_error(stream, ctypes.byref(code))
    assert rc == 4, "STA_ERR_TIMEOUT expected"
    assert code.value in (101, 102, 103, 104), code.value
    assert core.device_error() == 0  # the read cleared it

    again = core.select(q, k, tau, g, tile=T)
    torch.cuda.synchronize()
    assert core.device_error() == 0
    for key in ("row_max", "row_count", "votes"):
        assert torch.equal(again[key], good[key]), key
