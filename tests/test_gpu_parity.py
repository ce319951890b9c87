"""CUDA path vs the oracle / the reference's golden outputs (needs a B200).

Parity bar (from the benchmark contract): integer / index outputs of the selection bit-exact
for identical votes; Kernel A's keep decisions exact except pairs whose score lies within 1e-3
of the threshold (counted by the oracle); outputs within max-abs 1e-4 (fp32) or max-abs 2e-2 /
mean-abs 1e-3 (bf16).
"""
import glob
import json
import math
import os

import numpy as np
import pytest
import torch

from conftest import oracle

import sta  # noqa: F401
from sta import core
from sta.core import Geometry
from sta import shared_selection_exact_2 as ex2
from sta import shared_selection_exact as ex1
from sta import shared_selection_hybrid_exact as hyb
from sta import shared_selection_perquery as pq
from sta import pqstream_kernel as pqs
from sta.synth import SynthSpec, make_inputs, rope_inv_freq, yarn_inv_freq

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
FIX = sorted(glob.glob(os.path.join(HERE, "golden", "*.npz")))
DEV = "cuda"
BAND = 1e-3
F32_TOL = 1e-4
BF16_MAX, BF16_MEAN = 2e-2, 1e-3


def load(name):
    z = np.load(os.path.join(HERE, "golden", name + ".npz"))
    meta = json.loads(str(z["meta"]))
    return meta, {k: z[k] for k in z.files if k != "meta"}


def cu(x, dtype=None):
    if isinstance(x, torch.Tensor):
        t = x.to(DEV)
    else:
        t = torch.from_numpy(np.ascontiguousarray(x)).to(DEV)
    return t.to(dtype) if dtype is not None else t


def names(pattern):
    return [os.path.basename(p)[:-4] for p in FIX if pattern in os.path.basename(p)]


def assert_close_out(got, ref, dtype):
    ref = np.asarray(ref, np.float32)
    got = got.float().cpu().numpy()
    ok = np.isfinite(ref)
    assert np.isfinite(got[ok]).all(), "non-finite output where the reference is finite"
    err = np.abs(got[ok] - ref[ok])
    if dtype == torch.float32:
        assert err.max() <= F32_TOL, err.max()
    else:
        assert err.max() <= BF16_MAX and err.mean() <= BF16_MEAN, (err.max(), err.mean())


def device_sel(q, k, tau, g, T, wmode=0, bits=False):
    """Kernel A's own outputs on the device, as dense numpy arrays (H, nt, N) for the oracle's
    ``sel`` argument: the oracle then selects and attends on the device's keep decisions, which
    isolates the float threshold boundary from everything downstream of it."""
    q, k = cu(q), cu(k)
    H, N = q.shape[0], q.shape[1]
    r = core.select(q, k, tau, g, tile=T, wmode=wmode, bits=bits)
    torch.cuda.synchronize()
    assert core.device_error() == 0
    out = {"votes": core.expand_compact(r["votes"], H, N, T).cpu().numpy().astype(np.int32)}
    if wmode:
        out["wvotes"] = core.expand_compact(r["wvotes"], H, N, T).cpu().numpy()
    if bits:
        out["bits"] = core.expand_compact(r["bits"], H, N, T).cpu().numpy().view(np.uint32)
    return out


def assert_bf16_out(got, ref, what=""):
    """north_star's bf16 bar on every element: max-abs 2e-2 and mean-abs 1e-3."""
    got = got.float().cpu().numpy() if isinstance(got, torch.Tensor) else got
    assert np.isfinite(got).all(), what
    err = np.abs(got - ref)
    assert err.max() <= BF16_MAX and err.mean() <= BF16_MEAN, (what, err.max(), err.mean())


# ---------------------------------------------------------------------------------------------
# Kernel A (tcgen05 select) vs oracle
# ---------------------------------------------------------------------------------------------
SELECT_CASES = [
    # H, Hkv, N, D, T, dtype, wmode, bits, pos_scale, seed
    (2, 2, 300, 64, 64, torch.float32, 0, False, 0.5, 1),
    (2, 2, 256, 128, 32, torch.float32, 2, True, 1.0, 2),
    (4, 2, 384, 128, 64, torch.bfloat16, 1, False, 1.0, 3),
    (2, 1, 200, 64, 32, torch.bfloat16, 2, True, 0.75, 4),
    (1, 1, 129, 128, 64, torch.float32, 0, False, 1.0, 5),
    (2, 2, 1000, 128, 128, torch.bfloat16, 0, False, 1.0, 6),
]


@pytest.mark.parametrize("case", SELECT_CASES, ids=[f"sel{i}" for i in range(len(SELECT_CASES))])
def test_select_vs_oracle(case):
    H, Hk, N, D, T, dt, wmode, want_bits, ps, seed = case
    q, k, v = make_inputs(SynthSpec(n_heads=H, n_kv_heads=Hk, seq_len=N, head_dim=D,
                                    n_planted=8, n_planted_queries=16, seed=seed, dtype=dt))
    tau = torch.full((H,), 5.0)
    invf = rope_inv_freq(D, 1e4)
    g = Geometry(invf, ps, 1.0)
    res = core.select(cu(q[0]), cu(k[0]), tau, g, tile=T, wmode=wmode, bits=want_bits)
    torch.cuda.synchronize()
    assert core.device_error() == 0
    kx = k[0].float().repeat_interleave(H // Hk, 0).numpy()
    o = oracle.select_vote(q[0].float().numpy(), kx, tau.numpy(), invf.numpy(), ps, 1.0,
                           1.0 / math.sqrt(D), T, wmode=wmode, want_bits=want_bits)
    np.testing.assert_allclose(res["row_max"].cpu().numpy(), o["m"], rtol=2e-5, atol=2e-4)
    votes = core.expand_compact(res["votes"], H, N, T).cpu().numpy().astype(np.int32)
    diff = int(np.abs(votes - o["votes"]).sum())
    assert diff <= o["boundary"], (diff, o["boundary"])
    rc = res["row_count"].cpu().numpy()
    assert int(np.abs(rc - o["row_counts"]).sum()) <= o["boundary"]
    if wmode:
        wv = core.expand_compact(res["wvotes"], H, N, T).cpu().numpy()
        np.testing.assert_allclose(wv, o["wvotes"], rtol=1e-3, atol=2e-3)
    if want_bits:
        b = core.expand_compact(res["bits"], H, N, T).cpu().numpy().view(np.uint32)
        nb = sum(bin(int(x)).count("1") for x in (b ^ o["bits"]).ravel() if x)
        assert nb <= o["boundary"]


def test_select_tau_zero_keeps_argmax():
    """Both passes issue identical tensor-core sequences: with tau = 0 every real query keeps
    at least its own maximum key."""
    H, N, D = 2, 700, 128
    q, k, _ = make_inputs(SynthSpec(n_heads=H, n_kv_heads=H, seq_len=N, head_dim=D, seed=9,
                                    dtype=torch.bfloat16))
    res = core.select(cu(q[0]), cu(k[0]), torch.zeros(H), Geometry(rope_inv_freq(D, 1e4)),
                      tile=64)
    assert int(res["row_count"].min()) >= 1


# ---------------------------------------------------------------------------------------------
# selection stage: bit-exact on the reference's own votes
# ---------------------------------------------------------------------------------------------
@pytest.mark.parametrize("name", names("shared"))
def test_build_sets_bit_exact_on_reference_votes(name):
    meta, a = load(name)
    H, N, T = meta["H"], meta["N"], meta["T"]
    votes = core.compact_from_dense(cu(a["votes"].astype(np.uint8)), T)
    wv = None
    if meta["select_score"] != "freq":
        wv = core.compact_from_dense(cu(a["wvotes"].astype(np.float32)), T)
    o = core.build_sets(votes, wv, H, N, tile=T, k_max=meta["k_max"], n_global=meta["n_global"],
                        n_local=meta["n_local"], pct=meta["pct"], pos_scale=meta["pos_scale_c"],
                        select_score=meta["select_score"], measure=meta["measure"])
    np.testing.assert_array_equal(o["idx"].cpu().numpy(), a["idx"])
    np.testing.assert_array_equal(o["newpos_k"].cpu().numpy(), a["newpos_k"])
    np.testing.assert_array_equal(o["newpos_q"].cpu().numpy(), a["newpos_q"])
    np.testing.assert_array_equal(o["shared_size"].cpu().numpy(), a["shared_size"])
    np.testing.assert_array_equal(o["kept_size"].cpu().numpy(), a["kept_size"])
    np.testing.assert_array_equal(o["chosen"].cpu().numpy(), a["kpct"])
    np.testing.assert_array_equal(o["overflow"].cpu().numpy(), a["overflow"])
    np.testing.assert_array_equal(o["kpct_meas"].cpu().numpy(), a["kpct_meas"])
    np.testing.assert_array_equal(o["overflow20"].cpu().numpy(), a["overflow20"])


@pytest.mark.parametrize("name", names("pq_union"))
def test_build_sets_pq_bit_exact_on_reference_votes(name):
    meta, a = load(name)
    H, N = meta["H"], meta["N"]
    votes = core.compact_from_dense(cu(a["votes"].astype(np.uint8)), 32)
    bits = core.compact_from_dense(cu(a["bits"].astype(np.int32)), 32)
    wv = None
    if meta["select_score"] != "freq":
        wv = core.compact_from_dense(cu(a["wvotes"].astype(np.float32)), 32)
    o = core.build_sets_pq(votes, wv, bits, H, N, k_max=meta["k_max"],
                           select_score=meta["select_score"])
    for key in ("idx", "newpos_k", "newpos_q", "mask"):
        np.testing.assert_array_equal(o[key].cpu().numpy(), a[key], err_msg=key)
    np.testing.assert_array_equal(o["usize"].cpu().numpy(), a["usize"])
    np.testing.assert_array_equal(o["kept_size"].cpu().numpy(), a["kept_size"])
    np.testing.assert_array_equal(o["overflow"].cpu().numpy(), a["overflow"])


# ---------------------------------------------------------------------------------------------
# Kernel C on the reference's own sets
# ---------------------------------------------------------------------------------------------
@pytest.mark.parametrize("name", names("shared") + names("pq_union"))
def test_gather_attend_on_reference_sets(name):
    meta, a = load(name)
    T = meta["T"]
    is_pq = meta["kind"] == "pq"
    g = Geometry(torch.from_numpy(a["inv_freq_c"]), 1.0,
                 1.0 if is_pq else meta["rope_scale_c"])
    out = core.gather_attend(cu(a["q"]), cu(a["k"]), cu(a["v"]), cu(a["idx"]),
                             cu(a["newpos_k"]), cu(a["newpos_q"]), g, tile=T,
                             mask=cu(a["mask"]) if is_pq else None)
    assert_close_out(out, a["out"], torch.float32)


# ---------------------------------------------------------------------------------------------
# end to end through the reference call surfaces
# ---------------------------------------------------------------------------------------------
@pytest.mark.parametrize("name", names("shared"))
def test_shared_end_to_end_vs_reference(name):
    meta, a = load(name)
    q, k, v = (cu(a[x])[None] for x in ("q", "k", "v"))
    tau = torch.from_numpy(a["tau"])
    kw = dict(pct=meta["pct"], n_global=meta["n_global"], n_local=meta["n_local"],
              tile=meta["T"], k_max=meta["k_max"], measure=meta["measure"])
    if meta["geom"] == "hybrid":
        res = hyb.shared_pi_attention(q, k, v, tau, torch.from_numpy(a["inv_freq_a"]),
                                      meta["pos_scale_a"], meta["rope_scale_a"],
                                      torch.from_numpy(a["inv_freq_c"]), meta["pos_scale_c"],
                                      meta["rope_scale_c"], select_score=meta["select_score"], **kw)
    elif meta["module"] == "shared_selection_triton_exact":
        res = ex1.shared_pi_attention(q, k, v, tau, torch.from_numpy(a["inv_freq_a"]),
                                      meta["pos_scale_a"], rope_scale=meta["rope_scale_a"], **kw)
    else:
        res = ex2.shared_pi_attention(q, k, v, tau, torch.from_numpy(a["inv_freq_a"]),
                                      meta["pos_scale_a"], rope_scale=meta["rope_scale_a"],
                                      select_score=meta["select_score"], **kw)
    out = res[0][0]
    assert out.dtype == torch.float32 and out.shape == q.shape[1:]
    assert res[1].dtype == torch.int64 and res[4].dtype == torch.bool
    T = meta["T"]
    sm = 1.0 / math.sqrt(meta["D"])
    wmode = {"freq": 0, "margin": 1, "expmass": 2}[meta["select_score"]]
    # every tile: the oracle on the device's own votes (selection bit-exact, outputs 1e-4)
    ga = Geometry(torch.from_numpy(a["inv_freq_a"]), meta["pos_scale_a"], meta["rope_scale_a"])
    dsel = device_sel(a["q"], a["k"], torch.from_numpy(a["tau"]), ga, T, wmode)
    o = oracle.shared_attention(a["q"], a["k"], a["v"], a["tau"], a["inv_freq_a"],
                                meta["pos_scale_a"], meta["rope_scale_a"], a["inv_freq_c"],
                                meta["pos_scale_c"], meta["rope_scale_c"], sm_scale=sm,
                                sel=dsel, select_score=meta["select_score"], **kw)
    for j in range(1, 7):
        np.testing.assert_array_equal(res[j].cpu().numpy(), np.asarray(o[j]).astype(
            res[j].cpu().numpy().dtype), err_msg=f"stat {j}")
    assert_close_out(out, o[0], torch.float32)
    # tiles that no boundary pair touches: the reference's own outputs, exactly
    sel = oracle.select_vote(a["q"], a["k"], a["tau"], a["inv_freq_a"], meta["pos_scale_a"],
                             meta["rope_scale_a"], sm, T)
    clean = sel["near_tiles"] == 0
    assert clean.any()
    for got, key in ((res[1], "shared_size"), (res[2], "kept_size"), (res[3], "kpct"),
                     (res[4], "overflow")):
        np.testing.assert_array_equal(got.cpu().numpy()[clean],
                                      a[key].astype(got.cpu().numpy().dtype)[clean], err_msg=key)
    N = meta["N"]
    got = out.cpu().numpy()
    for h, t in zip(*np.nonzero(clean)):
        r0, r1 = t * T, min((t + 1) * T, N)
        assert np.abs(got[h, r0:r1] - a["out"][h, r0:r1]).max() <= F32_TOL, (h, t)


@pytest.mark.parametrize("name", names("pq_union"))
def test_pq_union_end_to_end_vs_reference(name):
    meta, a = load(name)
    q, k, v = (cu(a[x])[None] for x in ("q", "k", "v"))
    out, usize, kept, ovf = pq.shared_pq_attention(
        q, k, v, torch.from_numpy(a["tau"]), torch.from_numpy(a["inv_freq_a"]),
        torch.from_numpy(a["inv_freq_c"]), meta["pos_scale_a"], meta["rope_scale_a"],
        k_max=meta["k_max"], select_score=meta["select_score"])
    np.testing.assert_array_equal(usize.cpu().numpy(), a["usize"])
    np.testing.assert_array_equal(kept.cpu().numpy(), a["kept_size"])
    assert_close_out(out[0], a["out"], torch.float32)
    assert_close_out(out[0], a["out_torch_golden"], torch.float32)


@pytest.mark.parametrize("name", names("pqstream"))
def test_pqstream_end_to_end_vs_reference(name):
    meta, a = load(name)
    q, k, v = (cu(a[x])[None] for x in ("q", "k", "v"))
    out, span, kept, blocks, skipped = pqs.pqstream_attention(
        q, k, v, torch.from_numpy(a["tau"]), torch.from_numpy(a["inv_freq_a"]),
        torch.from_numpy(a["inv_freq_c"]), meta["pos_scale_a"], meta["rope_scale_a"],
        block_n=meta["block_n"], pos_advance=meta["pos_advance"], use_skip=meta["use_skip"])
    np.testing.assert_array_equal(span.cpu().numpy(), a["span"])
    np.testing.assert_array_equal(kept.cpu().numpy(), a["kept"])
    np.testing.assert_array_equal(blocks.cpu().numpy(), a["blocks"])
    np.testing.assert_array_equal(skipped.cpu().numpy(), a["skipped"])
    ok = np.isfinite(a["out"])
    got = out[0].float().cpu().numpy()
    assert np.abs(got[ok] - a["out"][ok]).max() <= F32_TOL


# ---------------------------------------------------------------------------------------------
# bf16 / GQA / larger shapes against the oracle (the interpreter cannot run bf16)
# ---------------------------------------------------------------------------------------------
BF16_CASES = [
    # H, Hkv, N, D, T, geom, select_score, k_max, seed
    (4, 1, 1024, 128, 64, "yarn", "freq", 256, 40),
    (2, 2, 777, 64, 32, "pi", "expmass", 200, 41),
    (4, 4, 1536, 128, 64, "pi", "freq", 2048, 42),
]


@pytest.mark.parametrize("case", BF16_CASES, ids=[f"bf16_{i}" for i in range(len(BF16_CASES))])
def test_shared_bf16_gqa_vs_oracle(case):
    H, Hk, N, D, T, geom, score, k_max, seed = case
    q, k, v = make_inputs(SynthSpec(n_heads=H, n_kv_heads=Hk, seq_len=N, head_dim=D,
                                    n_planted=16, seed=seed, dtype=torch.bfloat16))
    tau = torch.full((H,), 5.0)
    if geom == "yarn":
        invf, rs = yarn_inv_freq(D, 5e5, 4.0, 256)
        ps = 1.0
    else:
        invf, rs, ps = rope_inv_freq(D, 1e4), 1.0, 0.5
    res = ex2.shared_pi_attention(cu(q), cu(k), cu(v), tau, invf, ps, rope_scale=rs, tile=T,
                                  k_max=k_max, select_score=score)
    G = H // Hk
    qx, kx, vx = (x[0].float().numpy() for x in (q, k, v))
    kx, vx = np.repeat(kx, G, 0), np.repeat(vx, G, 0)
    wmode = {"freq": 0, "margin": 1, "expmass": 2}[score]
    dsel = device_sel(q[0], k[0], tau, Geometry(invf, ps, rs), T, wmode)
    own = oracle.select_vote(qx, kx, tau.numpy(), invf.numpy(), ps, rs, 1.0 / math.sqrt(D), T,
                             wmode=wmode)
    assert int(np.abs(dsel["votes"] - own["votes"]).sum()) <= own["boundary"]
    o = oracle.shared_attention(qx, kx, vx, tau.numpy(), invf.numpy(), ps, rs, invf.numpy(), ps,
                                rs, tile=T, k_max=k_max, select_score=score, v_is_bf16=True,
                                sel=dsel)
    np.testing.assert_array_equal(res[2].cpu().numpy(), o[2])
    np.testing.assert_array_equal(res[1].cpu().numpy(), o[1])
    assert_bf16_out(res[0][0], o[0])


def test_pq_bf16_vs_oracle():
    H, N, D = 2, 640, 128
    q, k, v = make_inputs(SynthSpec(n_heads=H, n_kv_heads=H, seq_len=N, head_dim=D, seed=50,
                                    dtype=torch.bfloat16))
    tau = torch.full((H,), 5.0)
    invf = rope_inv_freq(D, 1e4)
    out, usize, kept, ovf = pq.shared_pq_attention(cu(q), cu(k), cu(v), tau, invf, invf,
                                                   0.5, 1.0, k_max=256)
    dsel = device_sel(q[0], k[0], tau, Geometry(invf, 0.5, 1.0), 32, wmode=2, bits=True)
    o = oracle.pq_attention(*(x[0].float().numpy() for x in (q, k, v)), tau.numpy(),
                            invf.numpy(), invf.numpy(), 0.5, 1.0, k_max=256, v_is_bf16=True,
                            sel=dsel)
    np.testing.assert_array_equal(usize.cpu().numpy(), o[1])
    np.testing.assert_array_equal(kept.cpu().numpy(), o[2])
    assert_bf16_out(out[0], o[0])


def test_pqstream_bf16_vs_oracle():
    H, N, D = 2, 600, 128
    q, k, v = make_inputs(SynthSpec(n_heads=H, n_kv_heads=1, seq_len=N, head_dim=D, seed=51,
                                    dtype=torch.bfloat16))
    tau = torch.full((H,), 5.0)
    invf = rope_inv_freq(D, 1e4)
    out, span, kept, _, _ = pqs.pqstream_attention(cu(q), cu(k), cu(v), tau, invf, invf, 0.5,
                                                    block_n=64)
    kx = np.repeat(k[0].float().numpy(), H, 0)
    vx = np.repeat(v[0].float().numpy(), H, 0)
    dsel = device_sel(q[0], k[0], tau, Geometry(invf, 0.5, 1.0), 32, bits=True)
    nt = (N + 31) // 32
    kb = {(h, t): dsel["bits"][h, t] for h in range(H) for t in range(nt)}
    o = oracle.pqstream_attention(q[0].float().numpy(), kx, vx, tau.numpy(), invf.numpy(),
                                  invf.numpy(), 0.5, block_n=64, v_is_bf16=True, keep_bits=kb)
    np.testing.assert_array_equal(span.cpu().numpy(), o[1])
    np.testing.assert_array_equal(kept.cpu().numpy(), o[2])
    assert_bf16_out(out[0], o[0])


def test_pqstream_tau_inf_full_is_dense_rope():
    """Invariant oracle of pqstream_kernel.py:301-307: tau=+inf with pos_advance='full'
    reproduces native-RoPE dense causal attention."""
    H, N, D = 2, 320, 64
    q, k, v = make_inputs(SynthSpec(n_heads=H, n_kv_heads=H, seq_len=N, head_dim=D, seed=52))
    invf = rope_inv_freq(D, 1e4)
    out, *_ = pqs.pqstream_attention(cu(q), cu(k), cu(v), torch.full((H,), float("inf")), invf,
                                     invf, pos_advance="full")
    ref = oracle.dense_rope_attention(q[0].numpy(), k[0].numpy(), v[0].numpy(), invf.numpy())
    assert np.abs(out[0].cpu().numpy() - ref).max() <= 2e-4


def test_errors_are_loud():
    q = torch.zeros((1, 2, 64, 64), device=DEV, dtype=torch.float16)
    with pytest.raises(TypeError):
        ex2.shared_pi_attention(q, q, q, torch.ones(2), rope_inv_freq(64, 1e4))
    q = torch.zeros((1, 2, 64, 64), device=DEV)
    with pytest.raises(ValueError, match="q_pos_base must be 0"):
        ex2.shared_pi_attention(q, q, q, torch.ones(2), rope_inv_freq(64, 1e4), q_pos_base=3)
    with pytest.raises((ValueError, RuntimeError)):
        ex2.shared_pi_attention(q, q, q, torch.ones(2), rope_inv_freq(64, 1e4), tile=48)


# ---------------------------------------------------------------------------------------------
# chunk_exact
# ---------------------------------------------------------------------------------------------
@pytest.mark.parametrize("name", [n for n in names("chunk") if n.startswith("chunk_")])
def test_build_sets_chunk_on_reference_votes(name):
    from test_oracle import chunk_tiles_without_ties
    meta, a = load(name)
    H, N, C = meta["H"], meta["N"], meta["chunk_size"]
    votes = core.compact_from_dense(cu(a["votes"].astype(np.uint8)), 32)
    wv = None
    if meta["select_score"] != "freq":
        wv = core.compact_from_dense(cu(a["wvotes"].astype(np.float32)), 32)
    n_chunk = oracle.derive_n_chunk(meta["k_max"], C, 32, 32, 32)
    o = core.build_sets_chunk(votes, wv, H, N, k_max=meta["k_max"], chunk_size=C,
                              n_chunk=n_chunk, select_score=meta["select_score"],
                              chunk_agg=meta["chunk_agg"])
    idx = o["idx"].cpu().numpy()
    exact = chunk_tiles_without_ties(a, meta, n_chunk, idx)
    for key in ("idx", "newpos_k", "newpos_q", "mask", "usize", "kept_size"):
        np.testing.assert_array_equal(o[key].cpu().numpy()[exact], a[key][exact], err_msg=key)
    # identical to the oracle everywhere (same tie rule)
    ws = a.get("wvotes") if meta["select_score"] != "freq" else None
    ref = oracle.build_sets_chunk(a["votes"], ws, 32, 32, 32, meta["k_max"], C, n_chunk,
                                  select_score=meta["select_score"], chunk_agg=meta["chunk_agg"])
    np.testing.assert_array_equal(idx, ref[0])
    np.testing.assert_array_equal(o["kept_size"].cpu().numpy(), ref[5])


@pytest.mark.parametrize("name", [n for n in names("chunk") if n.startswith("chunk_")])
def test_chunk_end_to_end_vs_reference(name):
    from sta import shared_selection_chunked as ch
    meta, a = load(name)
    q, k, v = (cu(a[x])[None] for x in ("q", "k", "v"))
    out, usize, kept = ch.shared_chunk_attention(
        q, k, v, torch.from_numpy(a["tau"]), torch.from_numpy(a["inv_freq_a"]),
        torch.from_numpy(a["inv_freq_c"]), meta["pos_scale_a"], meta["rope_scale_a"],
        k_max=meta["k_max"], chunk_size=meta["chunk_size"], select_score=meta["select_score"],
        chunk_agg=meta["chunk_agg"])
    np.testing.assert_array_equal(usize.cpu().numpy(), a["usize"])
    np.testing.assert_array_equal(kept.cpu().numpy(), a["kept_size"])
    res = oracle.chunk_attention(a["q"], a["k"], a["v"], a["tau"], a["inv_freq_a"],
                                 a["inv_freq_c"], meta["pos_scale_a"], meta["rope_scale_a"],
                                 k_max=meta["k_max"], chunk_size=meta["chunk_size"],
                                 select_score=meta["select_score"], chunk_agg=meta["chunk_agg"])
    assert_close_out(out[0], res[0], torch.float32)
    if meta["select_score"] != "freq":      # no chunk-mass ties: the reference's own output
        assert_close_out(out[0], a["out"], torch.float32)


def test_chunk_bf16_gqa_vs_oracle():
    from sta import shared_selection_chunked as ch
    H, Hk, N, D = 4, 2, 1024, 128
    q, k, v = make_inputs(SynthSpec(n_heads=H, n_kv_heads=Hk, seq_len=N, head_dim=D, seed=60,
                                    dtype=torch.bfloat16))
    tau = torch.full((H,), 5.0)
    invf = rope_inv_freq(D, 1e4)
    out, usize, kept = ch.shared_chunk_attention(cu(q), cu(k), cu(v), tau, invf, invf, 0.5,
                                                 k_max=512)
    G = H // Hk
    dsel = device_sel(q[0], k[0], tau, Geometry(invf, 0.5, 1.0), 32, wmode=2)
    res = oracle.chunk_attention(q[0].float().numpy(), np.repeat(k[0].float().numpy(), G, 0),
                                 np.repeat(v[0].float().numpy(), G, 0), tau.numpy(),
                                 invf.numpy(), invf.numpy(), 0.5, k_max=512, v_is_bf16=True,
                                 sel=dsel)
    np.testing.assert_array_equal(usize.cpu().numpy(), res[1])
    np.testing.assert_array_equal(kept.cpu().numpy(), res[2])
    assert_bf16_out(out[0], res[0])
    assert int(kept.max()) <= 512


# ---------------------------------------------------------------------------------------------
# Dual Chunk Attention selection geometry (hybrid: DCA select, PI attend)
# ---------------------------------------------------------------------------------------------
@pytest.mark.parametrize("D,T,dt", [(64, 64, torch.float32), (128, 64, torch.bfloat16),
                                    (128, 32, torch.bfloat16)])
def test_dca_select_and_hybrid_vs_oracle(D, T, dt):
    H, Hk, N = 4, 2, 1100          # chunk_len 256: every chunk relation, ragged tail
    s_, w_ = 320, 64
    q, k, v = make_inputs(SynthSpec(n_heads=H, n_kv_heads=Hk, seq_len=N, head_dim=D, seed=70,
                                    n_planted=16, dtype=dt))
    tau = torch.full((H,), 5.0)
    invf = rope_inv_freq(D, 1e4)
    ms = oracle.dca_mscale(N, 512)
    res = hyb.shared_pi_attention(cu(q), cu(k), cu(v), tau, invf, 1.0, ms, invf, 0.5, 1.0,
                                  tile=T, k_max=512, dca_chunk_size=s_, dca_local_window=w_)
    G = H // Hk
    qx, kx, vx = q[0].float().numpy(), np.repeat(k[0].float().numpy(), G, 0), \
        np.repeat(v[0].float().numpy(), G, 0)
    dsel = device_sel(q[0], k[0], tau, Geometry(invf, 1.0, ms, (s_, w_)), T)
    own = oracle.select_vote(qx, kx, tau.numpy(), invf.numpy(), 1.0, ms, 1.0 / math.sqrt(D), T,
                             dca=(s_, w_))
    assert int(np.abs(dsel["votes"] - own["votes"]).sum()) <= own["boundary"]
    o = oracle.shared_attention(qx, kx, vx, tau.numpy(), invf.numpy(), 1.0, ms, invf.numpy(), 0.5,
                                1.0, tile=T, k_max=512, v_is_bf16=dt == torch.bfloat16,
                                dca_a=(s_, w_), sel=dsel)
    np.testing.assert_array_equal(res[2].cpu().numpy(), o[2])
    np.testing.assert_array_equal(res[1].cpu().numpy(), o[1])
    if dt == torch.float32:
        assert_close_out(res[0][0], o[0], torch.float32)
    else:
        assert_bf16_out(res[0][0], o[0])


def test_cfg2_fallback_clusters_vs_oracle():
    """Config-2 inputs (YaRN, GQA, bf16) at S = 8192 with its dense query clusters: the graded
    tiles 80 / 100 and the flat tile 64 drive the 30 -> 25 -> 20 % fallback.  On these seeds the
    oracle picks 30 % on some heads, 25 % and 20 % on others, and leaves the rest unresolved;
    the device selection must make the same pick and keep the same keys on those tiles."""
    from sta.synth import make_config_inputs
    q, k, v, c = make_config_inputs(2, seq_len=8192, n_heads=8)
    H, N, D, T = 8, 8192, 128, 64
    invf, rs = yarn_inv_freq(D, 5e5, 4.0, 8192)
    tau = torch.full((H,), 5.0)
    out, ssz, ksz, kpct, ovf, kmeas, ovf20 = ex2.shared_pi_attention(
        cu(q), cu(k), cu(v), tau, invf, 1.0, rope_scale=rs, tile=T, k_max=2048)
    tiles = [64, 80, 100]
    qx, kx, vx = (x[0].float().numpy() for x in (q, k, v))
    kx, vx = np.repeat(kx, H // 2, 0), np.repeat(vx, H // 2, 0)
    sm = 1.0 / math.sqrt(D)
    sel = oracle.select_vote(qx, kx, tau.numpy(), invf.numpy(), 1.0, rs, sm, T, tiles=tiles)
    dev = core.select(cu(q[0]), cu(k[0]), tau, Geometry(invf, 1.0, rs), tile=T)
    votes = core.expand_compact(dev["votes"], H, N, T).cpu().numpy().astype(np.int32)
    diff = sum(int(np.abs(votes[:, t] - sel["votes"][:, t]).sum()) for t in tiles)
    assert diff <= sel["boundary"], (diff, sel["boundary"])
    # selection bit-exact on the device's own votes (isolates the float boundary)
    seen = set()
    nt = N // T
    idx = np.full((H, nt, 2048), N, np.int32)
    npk = np.zeros((H, nt, 2048), np.float32)
    npq = np.zeros((H, nt, T), np.float32)
    for t in tiles:
        s = oracle.build_sets(votes[:, t:t + 1], 1.0, 32, 32, 30.0, T, 2048, q_pos_base=t * T)
        idx[:, t], npk[:, t], npq[:, t] = s[0][:, 0], s[1][:, 0], s[2][:, 0]
        seen |= set(int(x) for x in s[5][:, 0])
        np.testing.assert_array_equal(kpct[:, t].cpu().numpy(), s[5][:, 0])
        np.testing.assert_array_equal(ksz[:, t].cpu().numpy(), s[4][:, 0])
        np.testing.assert_array_equal(ssz[:, t].cpu().numpy(), s[3][:, 0])
        np.testing.assert_array_equal(ovf20[:, t].cpu().numpy(), s[8][:, 0])
    assert {0, 20, 25, 30} <= seen, seen
    ref = oracle.gather_attn(qx, kx, vx, invf.numpy(), idx, npk, npq, sm, rs, T,
                             v_is_bf16=True, tiles=tiles)
    for t in tiles:
        got = out[0, :, t * T:(t + 1) * T].float().cpu().numpy()
        err = np.abs(got - ref[:, t * T:(t + 1) * T])
        assert err.mean() <= BF16_MEAN and err.max() <= BF16_MAX, (t, err.max(), err.mean())


SLAB_CASES = [
    # variant, H, Hkv, N, D, T, dtype, geometry, extra kwargs
    ("shared", 4, 2, 1000, 128, 64, torch.bfloat16, "yarn", {}),
    ("shared", 2, 2, 700, 64, 32, torch.float32, "pi", {"select_score": "expmass"}),
    ("shared", 4, 2, 1100, 128, 64, torch.bfloat16, "dca", {}),
    ("pq_union", 4, 2, 900, 128, 32, torch.bfloat16, "yarn", {"select_score": "expmass"}),
    ("pq_stream", 4, 2, 900, 128, 32, torch.bfloat16, "yarn", {"select_score": "expmass"}),
    ("chunk", 2, 2, 800, 64, 32, torch.float32, "pi", {"n_chunk": 8}),
]


@pytest.mark.parametrize("case", SLAB_CASES, ids=[f"slab_{c[0]}_{c[7]}" for c in SLAB_CASES])
def test_query_slabs_reproduce_whole_sequence(case):
    """The single-sequence multi-GPU unit: slabs of query positions [s, e), each called with
    k / v truncated to e keys and q_pos_base = s, reproduce the whole-sequence call bit for bit
    (every query tile's result depends only on its own queries and the keys before them)."""
    from sta.partition import slab_edges
    variant, H, Hk, N, D, T, dt, geom, extra = case
    q, k, v = make_inputs(SynthSpec(n_heads=H, n_kv_heads=Hk, seq_len=N, head_dim=D,
                                    n_planted=16, seed=80, dtype=dt))
    tau = torch.full((H,), 5.0)
    if geom == "yarn":
        invf, rs = yarn_inv_freq(D, 5e5, 4.0, 256)
        ga = Geometry(invf, 1.0, rs)
    elif geom == "dca":
        invf, rs = rope_inv_freq(D, 1e4), 1.0
        ga = Geometry(invf, 1.0, 1.05, (320, 64))
    else:
        invf, rs = rope_inv_freq(D, 1e4), 1.0
        ga = Geometry(invf, 0.5, 1.0)
    gc = Geometry(invf, 0.5 if geom != "yarn" else 1.0, rs) if variant == "shared" else \
        Geometry(rope_inv_freq(D, 5e5 if geom == "yarn" else 1e4))
    kw = dict(tile=T, k_max=256, keep_sets=variant != "pq_stream", **extra)
    qd, kd, vd = cu(q), cu(k), cu(v)
    out, st, sets = core.forward(variant, qd, kd, vd, tau, ga, gc, **kw)
    edges = slab_edges(N, 3, attend_weight=128.0)
    assert len(set(edges)) == 4 and all(e % 128 == 0 for e in edges[:-1])
    for s0, s1 in zip(edges, edges[1:]):
        o2, st2, sets2 = core.forward(variant, qd[:, :, s0:s1].contiguous(), kd[:, :, :s1],
                                      vd[:, :, :s1], tau, ga, gc, q_pos_base=s0, **kw)
        assert torch.equal(o2, out[:, :, s0:s1]), (s0, s1)
        t0, t1 = s0 // T, (s1 + T - 1) // T
        for name, x in st2.items():
            ref = st[name][..., s0:s1] if name == "kept" else st[name][..., t0:t1]
            assert torch.equal(x, ref), (name, s0, s1)
        for name, x in sets2.items():
            if name == "idx":  # padding sentinel = the call's key count
                x = torch.where(x == s1, torch.full_like(x, N), x)
            assert torch.equal(x, sets[name][:, :, t0:t1]), (name, s0, s1)
    assert core.device_error() == 0


@pytest.mark.parametrize("variant", ["shared", "pq_union", "pq_stream"])
def test_forward_host_pipeline_equals_device_call(variant):
    """Host buffers in, host output back, transfers overlapped by kv-head group: the result is
    the device call's, bit for bit (every stage is independent per kv head)."""
    H, Hk, N, D = 8, 4, 640, 128
    q, k, v = make_inputs(SynthSpec(batch=2, n_heads=H, n_kv_heads=Hk, seq_len=N, head_dim=D,
                                    seed=90, n_planted=16, dtype=torch.bfloat16))
    tau = torch.full((H,), 5.0)
    invf, rs = yarn_inv_freq(D, 5e5, 4.0, 256)
    ga = Geometry(invf, 1.0, rs)
    gc = ga if variant == "shared" else Geometry(rope_inv_freq(D, 5e5))
    T = 64 if variant == "shared" else 32
    kw = dict(tile=T, k_max=256, select_score="freq" if variant == "shared" else "expmass")
    ref, st_ref, _ = core.forward(variant, cu(q), cu(k), cu(v), tau, ga, gc, **kw)
    out_h, st = core.forward_host(variant, q, k, v, tau, ga, gc, groups=2, **kw)
    torch.cuda.synchronize()
    assert not out_h.is_cuda
    assert torch.equal(out_h, ref.cpu())
    # a single kv head: the groups run over its q heads
    k1, v1 = k[:, :1].contiguous(), v[:, :1].contiguous()
    q1 = q[:, :2].contiguous()
    ref1, _, _ = core.forward(variant, cu(q1), cu(k1), cu(v1), tau[:2], ga, gc, **kw)
    out1, _ = core.forward_host(variant, q1, k1, v1, tau[:2], ga, gc, groups=[1, 1], **kw)
    torch.cuda.synchronize()
    assert torch.equal(out1, ref1.cpu())
    for name, x in st_ref.items():
        if torch.is_tensor(x):
            assert torch.equal(st[name], x), name


# ---------------------------------------------------------------------------------------------
# decode (one query per head against the cache) vs the reference's torch decode rules
# ---------------------------------------------------------------------------------------------
@pytest.mark.parametrize("name", names("decode_"))
def test_decode_vs_reference(name):
    meta, a = load(name)
    M, D = meta["M"], meta["D"]
    q, k, v = cu(a["q"])[None], cu(a["k"])[None], cu(a["v"])[None]
    mode = meta["mode"]
    ga = Geometry(torch.from_numpy(a["inv_freq_a"]), meta["pos_scale"], meta["rope_scale"])
    gc = Geometry(torch.from_numpy(a["inv_freq_c"]), meta["pos_scale"], meta["rope_scale_c"])
    out, st, sets = core.decode(mode, q, k, v, torch.from_numpy(a["tau"]), ga, gc,
                                n_global=meta["n_global"], n_local=meta["n_local"],
                                k_max=meta["k_max"], pct_decode=meta["pct_decode"],
                                block_n=meta["block_n"], keep_sets=True,
                                chunk_size=meta.get("chunk_size", 16),
                                n_chunk=meta.get("n_chunk", 0),
                                chunk_agg=meta.get("chunk_agg", "sum"),
                                select_score=meta.get("select_score", "expmass"))
    cap = min(sets["idx"].shape[-1], a["idx"].shape[1])
    np.testing.assert_array_equal(sets["idx"][0, :, :cap].cpu().numpy(), a["idx"][:, :cap])
    np.testing.assert_array_equal(sets["newpos_k"][0, :, :cap].cpu().numpy(),
                                  a["newpos_k"][:, :cap])
    np.testing.assert_array_equal(sets["newpos_q"][0].cpu().numpy(), a["newpos_q"])
    assert np.abs(out[0].cpu().numpy() - a["out"]).max() <= F32_TOL


@pytest.mark.parametrize("mode", ["pi", "rank", "stream", "chunk"])
def test_decode_bf16_gqa_vs_oracle(mode):
    H, Hk, M, D = 8, 2, 3001, 128
    q, k, v = make_inputs(SynthSpec(n_heads=H, n_kv_heads=Hk, seq_len=M, head_dim=D, seed=95,
                                    n_planted=32, dtype=torch.bfloat16))
    tau = torch.full((H,), 8.0)
    invf, rs = yarn_inv_freq(D, 5e5, 4.0, 1024)
    ga = Geometry(invf, 1.0, rs)
    gc = Geometry(invf, 1.0, rs) if mode == "pi" else Geometry(rope_inv_freq(D, 5e5))
    kw = dict(n_global=32, n_local=32, k_max=160, block_n=32, chunk_size=16, n_chunk=4)
    out, st, sets = core.decode(mode, cu(q[:, :, M - 1]), cu(k), cu(v), tau, ga, gc,
                                keep_sets=True, **kw)
    G = H // Hk
    qx = q[0, :, M - 1].float().numpy()
    kx = np.repeat(k[0].float().numpy(), G, 0)
    vx = np.repeat(v[0].float().numpy(), G, 0)
    sm = 1.0 / math.sqrt(D)
    if mode == "pi":
        o = oracle.decode_pi(qx, kx, vx, tau.numpy(), invf.numpy(), 1.0, rs, sm, 32, 32, 160)
    elif mode == "rank":
        o = oracle.decode_rank(qx, kx, vx, tau.numpy(), invf.numpy(), gc.inv_freq.numpy(), 1.0,
                               rs, sm, 32, 32, 160)
    elif mode == "chunk":
        o = oracle.decode_chunk(qx, kx, vx, tau.numpy(), invf.numpy(), gc.inv_freq.numpy(), 1.0,
                                rs, sm, 32, 32, 160, 16, 4)
    else:
        o = oracle.decode_stream(qx, kx, vx, tau.numpy(), invf.numpy(), gc.inv_freq.numpy(),
                                 1.0, rs, sm, 32, 32, 32)
    idx = sets["idx"][0].cpu().numpy()
    same = (idx == o[1][:, :idx.shape[1]]).all(1)
    assert same.sum() >= H - 1, same          # a boundary key may flip on one head
    err = np.abs(out[0].float().cpu().numpy() - o[0])[same]
    assert err.max() <= BF16_MAX and err.mean() <= BF16_MEAN, (err.max(), err.mean())
    assert int(st["kept"].min()) >= 64        # the forced keys at least


TINY = [1, 5, 33, 64, 65, 130, 257]


@pytest.mark.parametrize("N", TINY)
def test_tiny_sequences_vs_oracle(N):
    """Sequences shorter than one selection block / tile, and just past the boundaries (the
    reference supports ragged N down to a single token)."""
    H, D = 2, 64
    q, k, v = make_inputs(SynthSpec(n_heads=H, n_kv_heads=H, seq_len=N, head_dim=D, seed=100 + N,
                                    n_planted=min(4, max(N - 1, 0)), n_planted_queries=4))
    tau = torch.full((H,), 5.0)
    invf = rope_inv_freq(D, 1e4)
    res = ex2.shared_pi_attention(cu(q), cu(k), cu(v), tau, invf, 0.5, tile=64, k_max=64)
    qx, kx, vx = (x[0].float().numpy() for x in (q, k, v))
    o = oracle.shared_attention(qx, kx, vx, tau.numpy(), invf.numpy(), 0.5, 1.0, invf.numpy(),
                                0.5, 1.0, tile=64, k_max=64)
    assert np.abs(res[0][0].cpu().numpy() - o[0]).max() <= F32_TOL
    np.testing.assert_array_equal(res[2].cpu().numpy(), o[2])
    out, usize, kept, ovf = pq.shared_pq_attention(cu(q), cu(k), cu(v), tau, invf, invf, 0.5, 1.0,
                                                   k_max=96)
    o2 = oracle.pq_attention(qx, kx, vx, tau.numpy(), invf.numpy(), invf.numpy(), 0.5, 1.0,
                             k_max=96)
    assert np.abs(out[0].cpu().numpy() - o2[0]).max() <= F32_TOL
    out3, span, kept3, _, _ = pqs.pqstream_attention(cu(q), cu(k), cu(v), tau, invf, invf, 0.5)
    o3 = oracle.pqstream_attention(qx, kx, vx, tau.numpy(), invf.numpy(), invf.numpy(), 0.5)
    assert np.abs(out3[0].cpu().numpy() - o3[0]).max() <= F32_TOL
    np.testing.assert_array_equal(kept3.cpu().numpy().reshape(o3[2].shape), o3[2])


def test_full_length_properties_cfg2_shape():
    """Config-2 geometry at its full sequence length (32k; 8 of the 32 q heads), checked through
    size-independent properties: query slabs reproduce the whole call bit for bit, every query
    keeps its own argmax at tau = 0, and the selection outputs are well formed (slots ascending
    and in range, positions non-decreasing, the fallback honoured)."""
    from sta.synth import make_config_inputs
    q, k, v, c = make_config_inputs(2, n_heads=8)
    H, N, D, T = 8, c["S"], c["D"], c["T"]
    invf, rs = yarn_inv_freq(D, 5e5, 4.0, 8192)
    g = Geometry(invf, 1.0, rs)
    tau = torch.full((H,), 5.0)
    qd, kd, vd = cu(q), cu(k), cu(v)
    kw = dict(tile=T, k_max=2048, keep_sets=True)
    out, st, sets = core.forward("shared", qd, kd, vd, tau, g, g, **kw)
    s0 = 16384
    o2, st2, _ = core.forward("shared", qd[:, :, s0:].contiguous(), kd, vd, tau, g, g,
                              q_pos_base=s0, **kw)
    assert torch.equal(o2, out[:, :, s0:])
    assert torch.equal(st2["kept_size"], st["kept_size"][..., s0 // T:])
    idx = sets["idx"][0]
    valid = idx < N
    assert bool(((idx[..., 1:] > idx[..., :-1]) | ~valid[..., 1:]).all())   # ascending
    npk = sets["newpos_k"][0]
    assert bool(((npk[..., 1:] >= npk[..., :-1]) | ~valid[..., 1:]).all())  # monotone positions
    ks, ch = st["kept_size"][0], st["chosen"][0]
    assert bool((ks[ch > 0] <= 2048).all())                                  # fitted picks fit
    assert int(((ch > 0) & (ch < 30)).sum()) > 0                             # fallback exercised
    sel = core.select(qd[0], kd[0], torch.zeros(H), g, tile=T)
    assert int(sel["row_count"].min()) >= 1                                  # argmax kept
    assert core.device_error() == 0
