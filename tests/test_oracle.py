"""Pin the CPU oracle against the golden fixtures produced by the reference implementation.

The fixtures (tests/golden/*.npz, made by tests/golden/make_golden.py) hold the reference's own
Triton kernels' outputs, run through the Triton interpreter.  Integer / index outputs of the
selection must match bit-exactly when the oracle's selection is fed the reference's votes;
Kernel A's votes must match except where a score sits within 1e-3 of its threshold; outputs
match within the fp32 / bf16 tolerances the parity protocol states.
"""
import glob
import json
import math
import os

import numpy as np
import pytest

from conftest import oracle

HERE = os.path.dirname(os.path.abspath(__file__))
FIXTURES = sorted(glob.glob(os.path.join(HERE, "golden", "*.npz")))


def load(path):
    z = np.load(path)
    meta = json.loads(str(z["meta"]))
    return meta, {k: z[k] for k in z.files if k != "meta"}


def ids(paths):
    return [os.path.basename(p)[:-4] for p in paths]


def out_tol(meta):
    return (2e-2, 1e-3) if meta["dtype"] == "bfloat16" else (1e-4, 1e-5)


def test_fixtures_present():
    assert len(FIXTURES) >= 10


@pytest.mark.parametrize("path", [p for p in FIXTURES if "shared" in p],
                         ids=ids([p for p in FIXTURES if "shared" in p]))
def test_shared_selection_bit_exact(path):
    """_build_sets restatement == reference selection, fed the reference's votes."""
    meta, a = load(path)
    ws = a.get("wvotes") if meta["select_score"] != "freq" else None
    sets = oracle.build_sets(a["votes"], meta["pos_scale_c"], meta["n_global"],
                             meta["n_local"], meta["pct"], meta["T"], meta["k_max"],
                             measure=meta["measure"], wvotes=ws,
                             select_score=meta["select_score"])
    np.testing.assert_array_equal(sets[0], a["idx"])
    np.testing.assert_array_equal(sets[1], a["newpos_k"])
    np.testing.assert_array_equal(sets[2], a["newpos_q"])
    np.testing.assert_array_equal(sets[3], a["shared_size"])
    np.testing.assert_array_equal(sets[4], a["kept_size"])
    np.testing.assert_array_equal(sets[5], a["kpct"])
    np.testing.assert_array_equal(sets[6], a["overflow"].astype(bool))
    np.testing.assert_array_equal(sets[7], a["kpct_meas"])
    np.testing.assert_array_equal(sets[8], a["overflow20"].astype(bool))


@pytest.mark.parametrize("path", [p for p in FIXTURES if "shared" in p],
                         ids=ids([p for p in FIXTURES if "shared" in p]))
def test_shared_votes_and_output(path):
    meta, a = load(path)
    wmode = {"freq": 0, "margin": 1, "expmass": 2}[meta["select_score"]]
    sel = oracle.select_vote(a["q"], a["k"], a["tau"], a["inv_freq_a"], meta["pos_scale_a"],
                             meta["rope_scale_a"], 1.0 / np.sqrt(meta["D"]), meta["T"],
                             wmode=wmode)
    diff = int((sel["votes"] != a["votes"]).sum())
    assert diff <= sel["boundary"], (diff, sel["boundary"])
    if wmode:
        np.testing.assert_allclose(sel["wvotes"], a["wvotes"], rtol=1e-4, atol=1e-4)
    res = oracle.shared_attention(
        a["q"], a["k"], a["v"], a["tau"], a["inv_freq_a"], meta["pos_scale_a"],
        meta["rope_scale_a"], a["inv_freq_c"], meta["pos_scale_c"], meta["rope_scale_c"],
        pct=meta["pct"], n_global=meta["n_global"], n_local=meta["n_local"], tile=meta["T"],
        k_max=meta["k_max"], block_k=meta["block_k"], measure=meta["measure"],
        select_score=meta["select_score"], v_is_bf16=meta["dtype"] == "bfloat16")
    if diff == 0:
        np.testing.assert_array_equal(res[-1]["idx"], a["idx"])
    mx, mean = out_tol(meta)
    err = np.abs(res[0] - a["out"])
    assert err.max() <= mx and err.mean() <= mean, (err.max(), err.mean())


@pytest.mark.parametrize("path", [p for p in FIXTURES if "pq_union" in p],
                         ids=ids([p for p in FIXTURES if "pq_union" in p]))
def test_pq_union(path):
    meta, a = load(path)
    ws = a.get("wvotes") if meta["select_score"] != "freq" else None
    sets = oracle.build_sets_pq(a["votes"], a["bits"], ws, meta["n_global"], meta["n_local"],
                                32, meta["k_max"], select_score=meta["select_score"])
    # ties at the truncation cut are implementation-defined in the reference (torch.topk):
    # compare index sets exactly only for tiles without an exact tie at the cut
    np.testing.assert_array_equal(sets[4], a["usize"])
    np.testing.assert_array_equal(sets[5], a["kept_size"])
    np.testing.assert_array_equal(sets[6], a["overflow"].astype(bool))
    np.testing.assert_array_equal(sets[0], a["idx"])
    np.testing.assert_array_equal(sets[1], a["newpos_k"])
    np.testing.assert_array_equal(sets[2], a["newpos_q"])
    np.testing.assert_array_equal(sets[3], a["mask"])
    wmode = {"freq": 0, "margin": 1, "expmass": 2}[meta["select_score"]]
    sel = oracle.select_vote(a["q"], a["k"], a["tau"], a["inv_freq_a"], meta["pos_scale_a"],
                             meta["rope_scale_a"], 1.0 / np.sqrt(meta["D"]), 32, wmode=wmode,
                             want_bits=True)
    diff = int((sel["bits"].view(np.int32) != a["bits"]).sum())
    assert diff <= sel["boundary"]
    res = oracle.pq_attention(a["q"], a["k"], a["v"], a["tau"], a["inv_freq_a"], a["inv_freq_c"],
                              meta["pos_scale_a"], meta["rope_scale_a"], k_max=meta["k_max"],
                              select_score=meta["select_score"],
                              v_is_bf16=meta["dtype"] == "bfloat16")
    mx, mean = out_tol(meta)
    for ref in (a["out"], a["out_torch_golden"]):
        err = np.abs(res[0] - ref)
        assert err.max() <= mx and err.mean() <= mean, (err.max(), err.mean())


@pytest.mark.parametrize("path", [p for p in FIXTURES if "pqstream" in p],
                         ids=ids([p for p in FIXTURES if "pqstream" in p]))
def test_pqstream(path):
    meta, a = load(path)
    out, span, kept, blocks, skipped = oracle.pqstream_attention(
        a["q"], a["k"], a["v"], a["tau"], a["inv_freq_a"], a["inv_freq_c"], meta["pos_scale_a"],
        meta["rope_scale_a"], block_n=meta["block_n"], pos_advance=meta["pos_advance"],
        use_skip=meta["use_skip"], v_is_bf16=meta["dtype"] == "bfloat16")
    np.testing.assert_array_equal(span, a["span"])
    np.testing.assert_array_equal(kept, a["kept"])
    np.testing.assert_array_equal(blocks, a["blocks"])
    np.testing.assert_array_equal(skipped, a["skipped"])
    mx, mean = out_tol(meta)
    ok = np.isfinite(a["out"])
    err = np.abs(res_or(out)[ok] - a["out"][ok])
    assert err.max() <= mx and err.mean() <= mean, (err.max(), err.mean())


def res_or(x):
    return x


def test_dca_position_rule():
    """dca_kernel._selfcheck known answers (dca_kernel.py:670-701), restated."""
    k_t, q_t, qc_t, L = oracle.dca_position_tables(3072, 512, 8192 + 512)
    assert L == 2560
    assert q_t.min() == 0 and q_t.max() == L - 1
    assert qc_t[0] == L and qc_t[-1] == 3072
    assert int((qc_t < 3072).sum()) == 512
    assert k_t.max() == L - 1
    assert qc_t[0] - k_t[L - 1] == 1.0
    assert qc_t.max() - k_t.min() < 4096
    assert abs(oracle.dca_mscale(8192, 4096) - (0.05 * np.log(2.0) + 1)) < 1e-12
    assert oracle.dca_mscale(4096, 4096) == 1.0


@pytest.mark.parametrize("path", [p for p in FIXTURES if os.path.basename(p).startswith("chunk_")],
                         ids=ids([p for p in FIXTURES if os.path.basename(p).startswith("chunk_")]))
def test_chunk(path):
    meta, a = load(path)
    ws = a.get("wvotes") if meta["select_score"] != "freq" else None
    n_chunk = oracle.derive_n_chunk(meta["k_max"], meta["chunk_size"], 32, 32, 32)
    sets = oracle.build_sets_chunk(a["votes"], ws, 32, 32, 32, meta["k_max"], meta["chunk_size"],
                                   n_chunk, select_score=meta["select_score"],
                                   chunk_agg=meta["chunk_agg"])
    exact = chunk_tiles_without_ties(a, meta, n_chunk, sets[0])
    for i, key in enumerate(("idx", "newpos_k", "newpos_q", "mask", "usize", "kept_size")):
        np.testing.assert_array_equal(sets[i][exact], a[key][exact], err_msg=key)
    if not exact.all():
        return
    res = oracle.chunk_attention(a["q"], a["k"], a["v"], a["tau"], a["inv_freq_a"],
                                 a["inv_freq_c"], meta["pos_scale_a"], meta["rope_scale_a"],
                                 k_max=meta["k_max"], chunk_size=meta["chunk_size"],
                                 select_score=meta["select_score"], chunk_agg=meta["chunk_agg"])
    for ref in (a["out"], a["out_torch_golden"]):
        err = np.abs(res[0] - ref)
        assert err.max() <= 1e-4, err.max()


def chunk_tiles_without_ties(a, meta, n_chunk, idx):
    """Tiles whose chunk selection does not depend on a tie at the top-n_chunk cut.  In the
    other tiles the two selections may differ, but only inside the tied group: same number of
    chunks, every difference a chunk whose mass equals the cut (checked here)."""
    votes = a["votes"]
    H, nt, N = votes.shape
    C = meta["chunk_size"]
    nC = (N + C - 1) // C
    if meta["select_score"] == "freq" or "wvotes" not in a:
        rv = votes.astype(np.float32)
    else:
        rv = a["wvotes"].astype(np.float32)
    pad = nC * C - N
    mass = np.pad(np.where(votes > 0, rv, 0), ((0, 0), (0, 0), (0, pad))).reshape(H, nt, nC, C).sum(-1)
    forced, vis = oracle.forced_chunk_mask(nt, nC, C, N, 32, 32, 32)
    exact = np.ones((H, nt), bool)
    for h in range(H):
        for t in range(nt):
            cand = np.nonzero(vis[t] & ~forced[t])[0]
            if len(cand) <= n_chunk:
                continue
            cut = np.sort(mass[h, t, cand])[::-1][n_chunk - 1]
            ties = set(cand[mass[h, t, cand] == cut].tolist())
            if len(ties) <= 1:
                continue
            ours = set((idx[h, t][idx[h, t] < N] // C).tolist())
            ref = set((a["idx"][h, t][a["idx"][h, t] < N] // C).tolist())
            assert len(ours) == len(ref)
            assert (ours ^ ref) <= ties
            exact[h, t] = ours == ref
    return exact


def test_dca_positions_match_reference_tables():
    """The DCA selection geometry's positions reproduce the reference's ChunkLlama tables:
    cos/sin(position * inv_freq) * mscale for keys, same-chunk and previous/older-chunk queries."""
    meta, a = load(os.path.join(HERE, "golden", "dca_tables_s320_w64.npz"))
    n = meta["seq_len"]
    kpos, qi, qs, qo, L = oracle.dca_positions(n, meta["chunk_size"], meta["local_window"])
    invf = a["inv_freq"].astype(np.float32)
    ms = np.float32(meta["mscale"])

    def tab(pos):
        ang = pos.astype(np.float32)[:, None] * invf[None, :]
        c, s = np.cos(ang).astype(np.float32) * ms, np.sin(ang).astype(np.float32) * ms
        return np.concatenate([c, c], -1), np.concatenate([s, s], -1)

    kc, ks = tab(kpos)
    np.testing.assert_allclose(kc, a["k_cos"][:n], atol=2e-6)
    np.testing.assert_allclose(ks, a["k_sin"][:n], atol=2e-6)
    qc, qsn = tab(qi[:L])
    np.testing.assert_allclose(qc, a["q_cos"], atol=2e-6)
    np.testing.assert_allclose(qsn, a["q_sin"], atol=2e-6)
    sc, ss = tab(qs[:L])                       # previous-chunk queries (qc table by offset)
    np.testing.assert_allclose(sc, a["qc_cos"], atol=2e-6)
    oc, _ = tab(qo[:1])                        # older chunks: the qc table at offset L - 1
    np.testing.assert_allclose(oc[0], a["qc_cos"][L - 1], atol=2e-6)


# ---------------------------------------------------------------------------------------------
# decode: the oracle's per-query rules against the reference's torch decode paths
# ---------------------------------------------------------------------------------------------
def _decode_case(name):
    z = np.load(os.path.join(HERE, "golden", name + ".npz"))
    meta = json.loads(str(z["meta"]))
    return meta, {k: z[k] for k in z.files if k != "meta"}


def run_decode_oracle(meta, a):
    sm = 1.0 / math.sqrt(meta["D"])
    if meta["mode"] == "pi":
        return oracle.decode_pi(a["q"], a["k"], a["v"], a["tau"], a["inv_freq_a"],
                                meta["pos_scale"], meta["rope_scale"], sm, meta["n_global"],
                                meta["n_local"], meta["k_max"], meta["pct_decode"])
    if meta["mode"] == "rank":
        return oracle.decode_rank(a["q"], a["k"], a["v"], a["tau"], a["inv_freq_a"],
                                  a["inv_freq_c"], meta["pos_scale"], meta["rope_scale"], sm,
                                  meta["n_global"], meta["n_local"], meta["k_max"])
    if meta["mode"] == "chunk":
        return oracle.decode_chunk(a["q"], a["k"], a["v"], a["tau"], a["inv_freq_a"],
                                   a["inv_freq_c"], meta["pos_scale"], meta["rope_scale"], sm,
                                   meta["n_global"], meta["n_local"], meta["k_max"],
                                   meta["chunk_size"], meta["n_chunk"], meta["select_score"],
                                   meta["chunk_agg"])
    return oracle.decode_stream(a["q"], a["k"], a["v"], a["tau"], a["inv_freq_a"],
                                a["inv_freq_c"], meta["pos_scale"], meta["rope_scale"], sm,
                                meta["n_global"], meta["n_local"], meta["block_n"])


@pytest.mark.parametrize("name", sorted(os.path.basename(p)[:-4] for p in
                                        glob.glob(os.path.join(HERE, "golden", "decode_*.npz"))))
def test_decode_oracle_matches_reference(name):
    meta, a = _decode_case(name)
    out, idx, npk, npq = run_decode_oracle(meta, a)
    # the stream rule pads its slot buffer to a multiple of 1024 (pqstream_kernel.py:756-757):
    # compare the common slots, the rest must be padding
    cap = min(a["idx"].shape[1], idx.shape[1])
    np.testing.assert_array_equal(idx[:, :cap], a["idx"][:, :cap])
    np.testing.assert_array_equal(npk[:, :cap], a["newpos_k"][:, :cap])
    assert (a["idx"][:, cap:] == meta["M"]).all() and (idx[:, cap:] == meta["M"]).all()
    np.testing.assert_array_equal(npq, a["newpos_q"])
    assert np.abs(out - a["out"]).max() <= 1e-5


def test_decode_rules_reduce_to_dense_attention_at_tau_inf():
    """Invariant of every decode rule: tau = +inf keeps every cached key; with positions that
    preserve the query-key distances (PI at pos_scale 1 = identity, dense ranks over all keys
    = the positions, streamed positions = minus the distance to the query) each equals the
    last row of dense causal RoPE attention."""
    rng = np.random.default_rng(3)
    H, M, D = 2, 97, 32
    q = rng.standard_normal((H, M, D)).astype(np.float32)
    k = rng.standard_normal((H, M, D)).astype(np.float32)
    v = rng.standard_normal((H, M, D)).astype(np.float32)
    invf = (1.0 / (1e4 ** (np.arange(0, D, 2, dtype=np.float32) / D))).astype(np.float32)
    tau = np.full(H, np.inf, np.float32)
    sm = 1.0 / math.sqrt(D)
    dense = oracle.dense_rope_attention(q, k, v, invf)[:, M - 1]
    outs = [oracle.decode_pi(q[:, M - 1], k, v, tau, invf, 1.0, 1.0, sm, 32, 32, 4 * M)[0],
            oracle.decode_rank(q[:, M - 1], k, v, tau, invf, invf, 1.0, 1.0, sm, 32, 32, 4 * M)[0],
            oracle.decode_stream(q[:, M - 1], k, v, tau, invf, invf, 1.0, 1.0, sm, 32, 32, 16)[0],
            oracle.decode_chunk(q[:, M - 1], k, v, tau, invf, invf, 1.0, 1.0, sm, 32, 32, 4 * M,
                                16, 64)[0]]
    for o in outs:
        assert np.abs(o - dense).max() <= 1e-4


def test_prefill_rules_reduce_to_dense_attention_at_tau_inf():
    """Invariant of the prefill paths: tau = +inf with a budget that keeps everything (pct 100,
    k_max >= N, every chunk) and positions that preserve distances (pos_scale 1 for the shared
    path; dense ranks over all keys = the positions for PQ-Union and chunk_exact) equals dense
    causal RoPE attention -- the property the GPU hook tests rely on."""
    rng = np.random.default_rng(4)
    H, N, D = 2, 150, 32
    q = rng.standard_normal((H, N, D)).astype(np.float32)
    k = rng.standard_normal((H, N, D)).astype(np.float32)
    v = rng.standard_normal((H, N, D)).astype(np.float32)
    invf = (1.0 / (1e4 ** (np.arange(0, D, 2, dtype=np.float32) / D))).astype(np.float32)
    tau = np.full(H, np.inf, np.float32)
    dense = oracle.dense_rope_attention(q, k, v, invf)
    shared = oracle.shared_attention(q, k, v, tau, invf, 1.0, 1.0, invf, 1.0, 1.0, pct=100.0,
                                     tile=32, k_max=4 * N)[0]
    pqu = oracle.pq_attention(q, k, v, tau, invf, invf, k_max=4 * N)[0]
    chk = oracle.chunk_attention(q, k, v, tau, invf, invf, k_max=4 * N, n_chunk=64)[0]
    for o in (shared, pqu, chk):
        assert np.abs(o - dense).max() <= 1e-4


def cfg0_inputs_sha256(q, k, v):
    import hashlib
    h = hashlib.sha256()
    for x in (q, k, v):
        h.update(x.contiguous().numpy().tobytes())
    return h.hexdigest()


def test_oracle_matches_reference_at_config0():
    """Benchmark config 0 at its own shape (fixture made by the unmodified reference under the
    Triton interpreter): votes equal except boundary pairs, the selection bit-exact on the
    reference's votes, stats and outputs equal on every tile without boundary pairs."""
    import json
    import math
    from sta.synth import config_geometry, make_config_inputs
    q, k, v, c = make_config_inputs(0)
    z = np.load(os.path.join(HERE, "golden", "config0_f32.npz"))
    meta = json.loads(str(z["meta"]))
    assert cfg0_inputs_sha256(q, k, v) == meta["inputs_sha256"]
    ga, _ = config_geometry(c)
    qx, kx, vx = (x[0].numpy() for x in (q, k, v))
    invf = ga["inv_freq"].numpy()
    T, N = c["T"], c["S"]
    sm = 1.0 / math.sqrt(c["D"])
    tau = np.full(c["H"], c["tau"], np.float32)
    sel = oracle.select_vote(qx, kx, tau, invf, 1.0, 1.0, sm, T)
    assert int(np.abs(sel["votes"] - z["votes"]).sum()) <= sel["boundary"]
    s = oracle.build_sets(z["votes"], 1.0, 32, 32, c["pct"], T, c["k_max"])
    np.testing.assert_array_equal(s[0], z["idx"])
    np.testing.assert_array_equal(s[4], z["kept_size"])
    o = oracle.shared_attention(qx, kx, vx, tau, invf, 1.0, 1.0, invf, 1.0, 1.0, tile=T,
                                k_max=c["k_max"])
    clean = sel["near_tiles"] == 0
    assert clean.sum() >= clean.size // 2
    np.testing.assert_array_equal(o[2][clean], z["kept_size"][clean])
    for h, t in zip(*np.nonzero(clean)):
        r0, r1 = t * T, min((t + 1) * T, N)
        assert np.abs(o[0][h, r0:r1] - z["out"][h, r0:r1]).max() <= 1e-4, (h, t)


def test_oracle_dense_dca_matches_reference():
    """Dense DCA (the reference's dca_forward prefill on a one-layer Llama, its three blocks
    merged by log-sum-exp) equals one softmax over all causal keys with per-relation query
    rotations."""
    import json
    z = np.load(os.path.join(HERE, "golden", "dca_dense_gqa_f32.npz"))
    meta = json.loads(str(z["meta"]))
    G = meta["H"] // meta["Hkv"]
    k = np.repeat(z["k"], G, 0)
    v = np.repeat(z["v"], G, 0)
    o = oracle.dca_dense_attention(z["q"], k, v, meta["chunk_size"], meta["local_window"],
                                   z["inv_freq"], meta["mscale"], meta["sm_scale"])
    err = np.abs(o - z["out"])
    assert err.max() <= 1e-4, err.max()
