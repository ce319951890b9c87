"""Screened Kernel A scoring (one fp16 tensor-core product per pair, exact rescoring of the pairs
a proven bound leaves undecided) against the exact three-product kernel and the oracle.

The two kernels define the exact score by different fp32 summation orders (tensor-core
accumulation vs a fixed FMA chain), so they may disagree only on pairs whose score lies within
about 1e-5 (relative) of the threshold; the oracle check counts disagreements against the
oracle's own 1e-3 boundary band."""
import math

import numpy as np
import pytest
import torch

from oracle import sta_oracle as oracle
from sta import core
from sta.core import Geometry
from sta.synth import SynthSpec, make_inputs, rope_inv_freq, yarn_inv_freq

pytestmark = pytest.mark.gpu


def cu(x):
    return x.cuda()


def _votes(res, H, N, T):
    return core.expand_compact(res["votes"], H, N, T).cpu().numpy().astype(np.int32)


@pytest.mark.parametrize("H,Hk,N,D,T,yarn", [(8, 2, 4096, 128, 64, True), (4, 4, 1500, 64, 64, False),
                                             (4, 2, 2048, 128, 32, True)])
def test_screened_equals_exact_kernel(H, Hk, N, D, T, yarn):
    q, k, _ = make_inputs(SynthSpec(n_heads=H, n_kv_heads=Hk, seq_len=N, head_dim=D, n_planted=16,
                                    seed=11, dtype=torch.bfloat16))
    if yarn:
        invf, ms = yarn_inv_freq(D, 5e5, 4.0, 1024)
        g = Geometry(invf, 1.0, ms)
    else:
        g = Geometry(rope_inv_freq(D, 1e4), 0.5, 1.0)
    tau = torch.full((H,), 5.0)
    bits = T == 32
    a = core.select(cu(q[0]), cu(k[0]), tau, g, tile=T, bits=bits, screen=True)
    b = core.select(cu(q[0]), cu(k[0]), tau, g, tile=T, bits=bits, screen=False)
    torch.cuda.synchronize()
    assert core.device_error() == 0
    ma, mb = a["row_max"].cpu().numpy(), b["row_max"].cpu().numpy()
    np.testing.assert_allclose(ma, mb, rtol=1e-5, atol=1e-5)
    va, vb = _votes(a, H, N, T), _votes(b, H, N, T)
    nd = int(np.abs(va - vb).sum())
    assert nd <= max(2, va.sum() // 100000), nd
    ca, cb = a["row_count"].cpu().numpy(), b["row_count"].cpu().numpy()
    assert int(np.abs(ca - cb).sum()) <= max(2, ca.sum() // 100000)


def test_screened_vs_oracle_with_degenerate_rows():
    """Rows of zero queries (every score ties at 0: every key is a max candidate and lies on the
    tau = 0 threshold) and large-norm queries, against the oracle; tau = 0 keeps every row's
    own maximum (the candidates' exact scores are the same FMA chain in both passes)."""
    H, N, D, T = 2, 640, 128, 64
    q, k, _ = make_inputs(SynthSpec(n_heads=H, n_kv_heads=H, seq_len=N, head_dim=D, n_planted=8,
                                    seed=5, dtype=torch.bfloat16))
    q = q.clone()
    q[0, 0, 100:164] = 0
    q[0, 1, 300:310] *= 40
    g = Geometry(rope_inv_freq(D, 1e4))
    for tau_v in (5.0, 0.0):
        tau = torch.full((H,), tau_v)
        res = core.select(cu(q[0]), cu(k[0]), tau, g, tile=T, screen=True)
        torch.cuda.synchronize()
        assert core.device_error() == 0
        o = oracle.select_vote(q[0].float().numpy(), k[0].float().numpy(), tau.numpy(),
                               g.inv_freq.numpy(), 1.0, 1.0, 1.0 / math.sqrt(D), T)
        np.testing.assert_allclose(res["row_max"].cpu().numpy(), o["m"], rtol=2e-5, atol=2e-4)
        v = _votes(res, H, N, T)
        assert int(np.abs(v - o["votes"]).sum()) <= o["boundary"]
        rc = res["row_count"].cpu().numpy()
        if tau_v == 0.0:
            assert int(rc.min()) >= 1
            # zero queries: every causal key ties at score 0 and is kept
            assert (rc[0, 100:164] == np.arange(101, 165)).all()


def test_screened_dca_planes():
    """Dual Chunk Attention selection geometry (three query planes) through the screened kernel
    equals the exact kernel."""
    H, Hk, N, D = 4, 2, 2304, 128
    q, k, _ = make_inputs(SynthSpec(n_heads=H, n_kv_heads=Hk, seq_len=N, head_dim=D, n_planted=8,
                                    seed=3, dtype=torch.bfloat16))
    g = Geometry(rope_inv_freq(D, 1e4), 1.0, 1.0, dca=(768, 256))
    tau = torch.full((H,), 5.0)
    a = core.select(cu(q[0]), cu(k[0]), tau, g, tile=64, screen=True)
    b = core.select(cu(q[0]), cu(k[0]), tau, g, tile=64, screen=False)
    torch.cuda.synchronize()
    np.testing.assert_allclose(a["row_max"].cpu().numpy(), b["row_max"].cpu().numpy(),
                               rtol=1e-5, atol=1e-5)
    assert int(np.abs(_votes(a, H, N, 64) - _votes(b, H, N, 64)).sum()) <= 2


@pytest.mark.parametrize("T,screen", [(64, False), (128, False), (64, True)])
def test_vote_histograms_match_votes(T, screen):
    """Kernel A's per-tile histograms of nonzero votes (consumed by the shared-path selection in
    place of a pass over the votes) equal a bincount of the votes it wrote."""
    H, Hk, N, D = 4, 2, 1800, 128
    q, k, _ = make_inputs(SynthSpec(n_heads=H, n_kv_heads=Hk, seq_len=N, head_dim=D, n_planted=8,
                                    seed=21, dtype=torch.bfloat16))
    res = core.select(cu(q[0]), cu(k[0]), torch.full((H,), 5.0), Geometry(rope_inv_freq(D, 1e4)),
                      tile=T, vote_hist=True, screen=screen)
    torch.cuda.synchronize()
    v = _votes(res, H, N, T)
    hist = res["vote_hist"].cpu().numpy()
    nt = (N + T - 1) // T
    for h in range(H):
        for t in range(nt):
            want = np.bincount(v[h, t][v[h, t] > 0], minlength=T + 1)
            want[0] = 0
            assert (hist[h, t] == want).all(), (h, t)
