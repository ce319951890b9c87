"""The allocation-free entry point (sta_shared_forward_static) against sta_shared_forward.

It serves hosts that cannot allocate device memory (their runtime owns all allocations, or
they run under a fixed budget): scratch comes from a fixed array the library reserves at load
time.  This file is collected last on purpose; the test must pass alone in a fresh process and
after the rest of the suite.
"""
import ctypes
import math

import pytest
import torch

from sta import _lib as L
from sta import core
from sta.core import Geometry
from sta.synth import SynthSpec, make_inputs, yarn_inv_freq

pytestmark = pytest.mark.gpu


def _args(q, k, v, out, tau, invf, ms, st, T, k_max):
    a = L.ForwardArgs()
    a.q, a.q_stride_h, a.q_stride_n = q.data_ptr(), q.stride(0), q.stride(1)
    a.k, a.k_stride_h, a.k_stride_n = k.data_ptr(), k.stride(0), k.stride(1)
    a.v, a.v_stride_h, a.v_stride_n = v.data_ptr(), v.stride(0), v.stride(1)
    a.out = out.data_ptr()
    a.dtype = L.STA_DTYPE_BF16
    a.batch, a.n_heads, a.n_kv_heads, a.n, a.d = 1, q.shape[0], k.shape[0], q.shape[1], q.shape[2]
    a.tau = tau.data_ptr()
    a.inv_freq_a, a.pos_scale_a, a.rope_scale_a = invf.data_ptr(), 1.0, ms
    a.inv_freq_c, a.pos_scale_c, a.rope_scale_c = invf.data_ptr(), 1.0, ms
    a.sm_scale = 1.0 / math.sqrt(q.shape[2])
    a.pct, a.n_global, a.n_local, a.tile, a.k_max = 30.0, 32, 32, T, k_max
    for name in ("shared_size", "kept_size", "chosen", "overflow", "kpct_meas", "overflow20"):
        setattr(a, name, st[name].data_ptr())
    return a


def test_static_scratch_entry_point_matches_workspace_entry_point():
    lib = L.lib()
    H, Hk, N, D, T, k_max = 8, 2, 3072, 128, 64, 512
    q, k, v = make_inputs(SynthSpec(n_heads=H, n_kv_heads=Hk, seq_len=N, head_dim=D,
                                    n_planted=24, seed=77, dtype=torch.bfloat16))
    dev = torch.device("cuda")
    q, k, v = q[0].to(dev), k[0].to(dev), v[0].to(dev)
    invf, ms = yarn_inv_freq(D, 5e5, 4.0, 1024)
    tau = torch.full((H,), 5.0, device=dev)
    invf_d = invf.to(dev)
    # reference result through the workspace entry point
    ref, ref_st, _ = core.forward("shared", q[None], k[None], v[None], tau, Geometry(invf, 1.0, ms),
                                  Geometry(invf, 1.0, ms), tile=T, k_max=k_max)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    nt = (N + T - 1) // T
    for call in range(2):  # two calls in a row share (and reuse) the static scratch
        out = torch.full((H, N, D), float("nan"), dtype=torch.bfloat16, device=dev)
        st = {n: torch.full((H, nt), -7, dtype=torch.int32, device=dev)
              for n in ("shared_size", "kept_size", "chosen", "kpct_meas")}
        st["overflow"] = torch.full((H, nt), 7, dtype=torch.uint8, device=dev)
        st["overflow20"] = torch.full((H, nt), 7, dtype=torch.uint8, device=dev)
        a = _args(q, k, v, out, tau, invf_d, ms, st, T, k_max)
        rc = lib.sta_shared_forward_static(ctypes.byref(a), stream)
        assert rc == 0, lib.sta_last_error()
        torch.cuda.synchronize()
        err = (out.float() - ref[0].float()).abs()
        assert torch.isfinite(out.float()).all()
        assert err.max().item() <= 2e-2 and err.mean().item() <= 1e-3, (call, err.max().item())
        for n in st:
            assert torch.equal(st[n], ref_st[n][0]), n


def test_static_scratch_rejects_oversize_problem():
    lib = L.lib()
    dev = torch.device("cuda")
    H, N, D = 1, 65536, 128   # one kv head needs > 64 MiB of scratch at k_max 2048
    x = torch.zeros((H, N, D), dtype=torch.bfloat16, device=dev)
    invf = torch.ones(D // 2, device=dev)
    tau = torch.ones(H, device=dev)
    nt = N // 64
    st = {n: torch.zeros((H, nt), dtype=torch.int32, device=dev)
          for n in ("shared_size", "kept_size", "chosen", "kpct_meas")}
    st["overflow"] = torch.zeros((H, nt), dtype=torch.uint8, device=dev)
    st["overflow20"] = torch.zeros((H, nt), dtype=torch.uint8, device=dev)
    a = _args(x, x, x, x, tau, invf, 1.0, st, 64, 2048)
    rc = lib.sta_shared_forward_static(ctypes.byref(a), None)
    assert rc == 5
    assert b"64 MiB" in lib.sta_last_error()
