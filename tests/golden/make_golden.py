"""Generate the golden fixtures in this directory from the REFERENCE implementation.

Runs the reference repository's own Triton kernels on the CPU through the Triton interpreter
(``TRITON_INTERPRET=1``) on small seeded inputs and stores inputs + outputs as ``.npz``.  The
reference is imported read-only from the checkout given by ``--ref``; it is NOT needed
at test time -- the committed fixtures are.

Intermediate tensors (Kernel A's votes / wvotes / bits, and the selection outputs) are captured
by wrapping the reference module's host selection function for the duration of one call.

    TRITON_INTERPRET=1 python tests/golden/make_golden.py --ref <reference checkout>
"""
from __future__ import annotations

import argparse
import json
import os
import sys

os.environ.setdefault("TRITON_INTERPRET", "1")

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(REPO, "sparse-thresholded-attention_b200"))

from sta.synth import SynthSpec, make_inputs, rope_inv_freq, yarn_inv_freq  # noqa: E402


def _np(x):
    if isinstance(x, torch.Tensor):
        if x.dtype == torch.bfloat16:
            x = x.float()
        return x.detach().cpu().numpy()
    return np.asarray(x)


class Capture:
    """Wrap ``module.<name>`` so that its inputs and outputs are recorded."""

    def __init__(self, module, name):
        self.module, self.name = module, name
        self.orig = getattr(module, name)
        self.args = self.kwargs = self.result = None

    def __enter__(self):
        def wrapped(*args, **kwargs):
            self.args, self.kwargs = args, kwargs
            self.result = self.orig(*args, **kwargs)
            return self.result
        setattr(self.module, self.name, wrapped)
        return self

    def __exit__(self, *exc):
        setattr(self.module, self.name, self.orig)


def inputs(H, N, D, seed, dtype, planted=8, Hkv=None):
    spec = SynthSpec(batch=1, n_heads=H, n_kv_heads=Hkv or H, seq_len=N, head_dim=D,
                     n_planted=planted, n_planted_queries=16, seed=seed, dtype=dtype)
    q, k, v = make_inputs(spec)
    return q, k, v


ONLY = None


def save(name, meta, arrays):
    if ONLY and ONLY not in name:
        return
    path = os.path.join(HERE, name + ".npz")
    out = {k: _np(v) for k, v in arrays.items()}
    for k, v in list(out.items()):
        if v.dtype == np.int64:
            out[k] = v.astype(np.int32)
        if v.dtype == np.bool_:
            out[k] = v.astype(np.uint8)
    np.savez_compressed(path, meta=np.array(json.dumps(meta)), **out)
    print("wrote", path, {k: v.shape for k, v in out.items()})


def gen_shared(ref, mod_name, case, H, N, D, T, k_max, seed, dtype, select_score="freq",
               geom="pi", pos_scale=1.0, tau_val=5.0, pct=30.0, measure=False, block_n=64,
               block_k=64, n_global=32, n_local=32, planted=8):
    mod = __import__(mod_name)
    q, k, v = inputs(H, N, D, seed, dtype, planted=planted)
    tau = torch.full((H,), float(tau_val))
    meta = dict(kind="shared", module=mod_name, H=H, N=N, D=D, T=T, k_max=k_max, seed=seed,
                dtype=str(dtype).replace("torch.", ""), select_score=select_score, geom=geom,
                pct=pct, measure=measure, block_n=block_n, block_k=block_k,
                n_global=n_global, n_local=n_local)
    if geom == "hybrid":
        invf_a, att = yarn_inv_freq(D, 5e5, 4.0, 256)
        invf_c = rope_inv_freq(D, 1e4)
        meta.update(pos_scale_a=1.0, rope_scale_a=att, pos_scale_c=pos_scale, rope_scale_c=1.0)
        with Capture(mod, "_build_sets") as cap:
            res = mod.shared_pi_attention(q, k, v, tau, invf_a, 1.0, att, invf_c, pos_scale, 1.0,
                                          pct=pct, n_global=n_global, n_local=n_local, tile=T,
                                          k_max=k_max, block_n=block_n, block_k=block_k,
                                          measure=measure, select_score=select_score)
    else:
        if geom == "yarn":
            invf, att = yarn_inv_freq(D, 5e5, 4.0, 256)
            rs, ps = att, 1.0
        else:
            invf, rs, ps = rope_inv_freq(D, 1e4), 1.0, pos_scale
        invf_a = invf_c = invf
        meta.update(pos_scale_a=ps, rope_scale_a=rs, pos_scale_c=ps, rope_scale_c=rs)
        kw = dict(pos_scale=ps, pct=pct, rope_scale=rs, n_global=n_global, n_local=n_local,
                  tile=T, k_max=k_max, block_n=block_n, block_k=block_k, measure=measure)
        if mod_name != "shared_selection_triton_exact":
            kw["select_score"] = select_score
        with Capture(mod, "_build_sets") as cap:
            res = mod.shared_pi_attention(q, k, v, tau, invf, **kw)
    votes = cap.args[0]
    wvotes = cap.kwargs.get("wvotes")
    sets = cap.result
    arrays = dict(q=q[0], k=k[0], v=v[0], tau=tau, inv_freq_a=invf_a, inv_freq_c=invf_c,
                  out=res[0][0], shared_size=res[1], kept_size=res[2], kpct=res[3],
                  overflow=res[4], kpct_meas=res[5], overflow20=res[6], votes=votes,
                  idx=sets[0], newpos_k=sets[1], newpos_q=sets[2])
    if wvotes is not None and wvotes.shape[-1] == N:
        arrays["wvotes"] = wvotes
    save(case, meta, arrays)


def gen_cfg0(case):
    """Benchmark config 0 exactly (sta.synth.config(0): fp32, H = Hkv = 4, S 1024, D 64, tile 64,
    tau 5, top 30 %, cap 2048, plain RoPE theta 1e4, seed 0, 32 planted keys per head) through
    the reference's shared_pi_attention (shared_selection_triton_exact_2.py:432-486).  The
    inputs are regenerated by sta.synth at test time; the fixture stores their SHA-256."""
    import hashlib
    from sta.synth import config_geometry, make_config_inputs
    mod = __import__("shared_selection_triton_exact_2")
    q, k, v, c = make_config_inputs(0)
    ga, _ = config_geometry(c)
    tau = torch.full((c["H"],), float(c["tau"]))
    with Capture(mod, "_build_sets") as cap:
        res = mod.shared_pi_attention(q, k, v, tau, ga["inv_freq"], pos_scale=ga["pos_scale"],
                                      pct=c["pct"], rope_scale=ga["rope_scale"], tile=c["T"],
                                      k_max=c["k_max"])
    h = hashlib.sha256()
    for x in (q, k, v):
        h.update(x.contiguous().numpy().tobytes())
    meta = dict(kind="shared", module="shared_selection_triton_exact_2", config=0, H=c["H"],
                N=c["S"], S=c["S"], D=c["D"], T=c["T"], k_max=c["k_max"], seed=c["seed"],
                pct=c["pct"], tau=c["tau"], inputs_sha256=h.hexdigest())
    sets = cap.result
    save(case, meta, dict(out=res[0][0], shared_size=res[1], kept_size=res[2], kpct=res[3],
                          overflow=res[4], votes=cap.args[0], idx=sets[0]))


def gen_dca_dense(case, H, Hkv, N, D, chunk_size, pretrain_len, local_window, seed):
    """The reference's dense DCA attention (dca_forward prefill, dca_kernel.py:447-487) on a
    one-layer random-init Llama patched by the reference's own patch_model_with_dca.  On the
    CPU the reference takes its PyTorch block path (_fa_block's fallback, fp32) and merges the
    three blocks by log-sum-exp.  Stores the layer's raw q / k / v (projection outputs, before
    any rotation) and the attention output (the input of o_proj)."""
    from transformers import LlamaConfig, LlamaForCausalLM
    dca = __import__("dca_kernel")
    torch.manual_seed(seed)
    cfg = LlamaConfig(hidden_size=H * D, num_attention_heads=H, num_key_value_heads=Hkv,
                      head_dim=D, num_hidden_layers=1, intermediate_size=64, vocab_size=64,
                      max_position_embeddings=pretrain_len, rope_theta=10000.0)
    model = LlamaForCausalLM(cfg).float().eval()
    originals = dca.patch_model_with_dca(model, chunk_size, pretrain_len, local_window)
    attn = model.model.layers[0].self_attn
    cap = {}
    hooks = [attn.q_proj.register_forward_hook(lambda m, i, o: cap.__setitem__("q", o)),
             attn.k_proj.register_forward_hook(lambda m, i, o: cap.__setitem__("k", o)),
             attn.v_proj.register_forward_hook(lambda m, i, o: cap.__setitem__("v", o)),
             attn.o_proj.register_forward_pre_hook(lambda m, i: cap.__setitem__("out", i[0]))]
    x = torch.randn(1, N, H * D) * 2.0
    with torch.no_grad():
        attn(x, position_embeddings=None, attention_mask=None)
    for h in hooks:
        h.remove()
    dca.unpatch_model(originals)
    q = cap["q"].view(1, N, H, D).transpose(1, 2)[0]
    k = cap["k"].view(1, N, Hkv, D).transpose(1, 2)[0]
    v = cap["v"].view(1, N, Hkv, D).transpose(1, 2)[0]
    out = cap["out"].view(1, N, H, D).transpose(1, 2)[0]
    inv_freq = 1.0 / (10000 ** (torch.arange(0, D, 2).float() / D))
    meta = dict(kind="dca_dense", H=H, Hkv=Hkv, N=N, D=D, chunk_size=chunk_size,
                pretrain_len=pretrain_len, local_window=local_window, seed=seed,
                mscale=dca.get_mscale(N / pretrain_len), sm_scale=float(attn.scaling))
    save(case, meta, dict(q=q, k=k, v=v, out=out, inv_freq=inv_freq))


def gen_pq(case, H, N, D, k_max, seed, dtype, select_score="expmass", geom="pi",
           pos_scale=1.0, tau_val=5.0, planted=8):
    mod = __import__("shared_selection_triton_perquery")
    q, k, v = inputs(H, N, D, seed, dtype, planted=planted)
    tau = torch.full((H,), float(tau_val))
    invf_c = rope_inv_freq(D, 1e4)
    if geom == "yarn":
        invf_a, rs = yarn_inv_freq(D, 5e5, 4.0, 256)
        ps = 1.0
    else:
        invf_a, rs, ps = invf_c, 1.0, pos_scale
    meta = dict(kind="pq", H=H, N=N, D=D, T=32, k_max=k_max, seed=seed,
                dtype=str(dtype).replace("torch.", ""), select_score=select_score, geom=geom,
                pos_scale_a=ps, rope_scale_a=rs, n_global=32, n_local=32, block_k=64)
    with Capture(mod, "_build_sets_pq") as cap:
        res = mod.shared_pq_attention(q, k, v, tau, invf_a, invf_c, pos_scale_a=ps,
                                      rope_scale_a=rs, k_max=k_max, select_score=select_score)
    golden = mod.pq_attention_torch(q, k, v, tau, invf_a, invf_c, pos_scale_a=ps,
                                    rope_scale_a=rs, k_max=k_max, select_score=select_score)
    votes, bits, wvotes = cap.args[0], cap.args[1], cap.args[2]
    sets = cap.result
    arrays = dict(q=q[0], k=k[0], v=v[0], tau=tau, inv_freq_a=invf_a, inv_freq_c=invf_c,
                  out=res[0][0], out_torch_golden=golden[0], usize=res[1], kept_size=res[2],
                  overflow=res[3], votes=votes, bits=bits.view(torch.int32), idx=sets[0],
                  newpos_k=sets[1], newpos_q=sets[2], mask=sets[3])
    if wvotes.shape[-1] == N:
        arrays["wvotes"] = wvotes
    save(case, meta, arrays)


def gen_pqstream(case, H, N, D, seed, dtype, block_n=32, pos_advance="max", use_skip=True,
                 geom="pi", pos_scale=1.0, tau_val=5.0, planted=8):
    mod = __import__("pqstream_kernel")
    q, k, v = inputs(H, N, D, seed, dtype, planted=planted)
    tau = torch.full((H,), float(tau_val))
    invf_c = rope_inv_freq(D, 1e4)
    if geom == "yarn":
        invf_a, rs = yarn_inv_freq(D, 5e5, 4.0, 256)
        ps = 1.0
    else:
        invf_a, rs, ps = invf_c, 1.0, pos_scale
    meta = dict(kind="pqstream", H=H, N=N, D=D, T=32, seed=seed,
                dtype=str(dtype).replace("torch.", ""), geom=geom, pos_scale_a=ps,
                rope_scale_a=rs, n_global=32, n_local=32, block_n=block_n,
                pos_advance=pos_advance, use_skip=use_skip, tau=tau_val)
    out, span, kept, blocks, skipped = mod.pqstream_attention(
        q, k, v, tau, invf_a, invf_c, pos_scale_a=ps, rope_scale_a=rs, block_n=block_n,
        pos_advance=pos_advance, use_skip=use_skip)
    golden = mod.pqstream_attention_torch(q, k, v, tau, invf_a, invf_c, pos_scale_a=ps,
                                          rope_scale_a=rs, block_n=block_n,
                                          pos_advance=pos_advance)
    save(case, meta, dict(q=q[0], k=k[0], v=v[0], tau=tau, inv_freq_a=invf_a,
                          inv_freq_c=invf_c, out=out[0], out_torch_golden=golden[0], span=span,
                          kept=kept, blocks=blocks, skipped=skipped))


def install_chunk_shim():
    """The reference's chunked module imports `chunk_recall_core.forced_chunk_mask`, which the
    reference repository does not ship.  Its own golden (chunk_attention_torch,
    shared_selection_triton_chunked.py:378-384) restates the rule inline; this test-only shim
    returns the same (forced, visible) masks, shape (nt, nC), so the module can be imported."""
    import types
    shim = types.ModuleType("chunk_recall_core")

    def forced_chunk_mask(nt, nC, C, N, T, n_global, n_local, q_pos_base, dev):
        c = torch.arange(nC, device=dev)
        t = torch.arange(nt, device=dev)
        r0 = q_pos_base + t * T
        last_q = (q_pos_base + (t + 1) * T).clamp(max=N) - 1
        vis = c[None, :] * C <= last_q[:, None]
        glob = (c < (n_global + C - 1) // C)[None, :]
        lo = (r0 - n_local + 1).clamp(min=0) // C
        hi = last_q // C
        loc = (c[None, :] >= lo[:, None]) & (c[None, :] <= hi[:, None])
        return (glob | loc) & vis, vis

    shim.forced_chunk_mask = forced_chunk_mask
    sys.modules["chunk_recall_core"] = shim


def gen_chunk(case, H, N, D, k_max, seed, dtype, select_score="expmass", chunk_size=16,
              chunk_agg="sum", tau_val=5.0, planted=8):
    install_chunk_shim()
    mod = __import__("shared_selection_triton_chunked")
    q, k, v = inputs(H, N, D, seed, dtype, planted=planted)
    tau = torch.full((H,), float(tau_val))
    invf = rope_inv_freq(D, 1e4)
    meta = dict(kind="chunk", H=H, N=N, D=D, T=32, k_max=k_max, seed=seed,
                dtype=str(dtype).replace("torch.", ""), select_score=select_score,
                chunk_size=chunk_size, chunk_agg=chunk_agg, pos_scale_a=0.5, rope_scale_a=1.0,
                n_global=32, n_local=32, block_k=64)
    with Capture(mod, "_build_sets_chunk") as cap:
        res = mod.shared_chunk_attention(q, k, v, tau, invf, invf, pos_scale_a=0.5,
                                         k_max=k_max, chunk_size=chunk_size,
                                         select_score=select_score, chunk_agg=chunk_agg)
    golden = mod.chunk_attention_torch(q, k, v, tau, invf, invf, pos_scale_a=0.5, k_max=k_max,
                                       chunk_size=chunk_size, select_score=select_score,
                                       chunk_agg=chunk_agg)
    votes, wvotes = cap.args[0], cap.args[1]
    sets = cap.result
    arrays = dict(q=q[0], k=k[0], v=v[0], tau=tau, inv_freq_a=invf, inv_freq_c=invf,
                  out=res[0][0], out_torch_golden=golden[0], usize=res[1], kept_size=res[2],
                  votes=votes, idx=sets[0], newpos_k=sets[1], newpos_q=sets[2], mask=sets[3])
    if wvotes.shape[-1] == N:
        arrays["wvotes"] = wvotes
    save(case, meta, arrays)


def gen_dca_tables(case, chunk_size, local_window, pretrain, seq_len, dim=64):
    """The reference's ChunkLlama rotary tables (dca_kernel.py:176-269) for a small setting."""
    mod = __import__("dca_kernel")
    mod._DCA_CHUNK_SIZE, mod._DCA_LOCAL_WINDOW = chunk_size, local_window
    rot = mod.ChunkLlamaRotaryEmbedding(dim=dim, max_position_embeddings=pretrain, base=10000)
    rot._set_cos_sin_cache(seq_len=seq_len, device=None, dtype=torch.float32)
    meta = dict(kind="dca_tables", chunk_size=chunk_size, local_window=local_window,
                pretrain=pretrain, seq_len=seq_len, dim=dim, mscale=rot._last_mscale)
    save(case, meta, dict(inv_freq=rot.inv_freq, q_cos=rot.q_cos_cached, q_sin=rot.q_sin_cached,
                          qc_cos=rot.qc_cos_cached, qc_sin=rot.qc_sin_cached,
                          k_cos=rot.k_cos_cached, k_sin=rot.k_sin_cached))


def gen_decode(case, mode, H, M, D, seed, k_max=64, pct_decode=100.0, block_n=32, pos_scale=1.0,
               rope_scale=1.0, geom="pi", tau_val=5.0, chunk_size=16, n_chunk=4,
               select_score="expmass", chunk_agg="sum"):
    """One decode step of the reference's torch decode paths: the query at position M-1 against
    the cache 0..M-1 (selection sets + attention output)."""
    q, k, v = inputs(H, M, D, seed, torch.float32, planted=8)
    qd, K, V = q[0, :, M - 1].contiguous(), k[0].contiguous(), v[0].contiguous()
    tau = torch.full((H,), float(tau_val))
    invf = rope_inv_freq(D, 1e4)
    sm = 1.0 / D ** 0.5
    if geom == "yarn":
        invf, rope_scale = yarn_inv_freq(D, 5e5, 4.0, 128)
    ng, nl, qpos = 32, 32, M - 1
    if mode == "pi":
        ref = __import__("shared_selection_triton_exact")
        idx, npk, npq = ref._decode_build_sets(qd, K, tau, invf, qpos, pos_scale, rope_scale, sm,
                                               ng, nl, k_max, pct_decode)
        out = ref._decode_attend_torch(qd, K, V, idx, npk, npq, invf, rope_scale, sm)
        invf_c, rs_c = invf, rope_scale
    elif mode == "rank":
        ref = __import__("shared_selection_triton_perquery")
        idx, npk, npq = ref._decode_build_sets_pq(qd, K, tau, invf, qpos, pos_scale, rope_scale,
                                                  sm, ng, nl, k_max)
        invf_c, rs_c = rope_inv_freq(D, 1e4), 1.0
        out = ref._decode_attend_torch_pq(qd, K, V, idx, npk, npq, invf_c, sm)
    elif mode == "chunk":
        install_chunk_shim()
        ref = __import__("shared_selection_triton_chunked")
        pq = __import__("shared_selection_triton_perquery")
        idx, npk, npq = ref._decode_build_sets_chunk(qd, K, tau, invf, qpos, pos_scale,
                                                     rope_scale, sm, ng, nl, k_max, chunk_size,
                                                     n_chunk, select_score=select_score,
                                                     chunk_agg=chunk_agg)
        invf_c, rs_c = rope_inv_freq(D, 1e4), 1.0
        out = pq._decode_attend_torch_pq(qd, K, V, idx, npk, npq, invf_c, sm)
    else:
        ref = __import__("pqstream_kernel")
        idx, npk, npq = ref._decode_build_sets_pqs(qd, K, tau, invf, qpos, pos_scale, rope_scale,
                                                   sm, ng, nl, block_n)
        invf_c, rs_c = rope_inv_freq(D, 1e4), 1.0
        out = ref._decode_attend_torch(qd, K, V, idx, npk, npq, invf_c, sm)
    meta = dict(kind="decode", mode=mode, H=H, M=M, D=D, seed=seed, k_max=k_max,
                pct_decode=pct_decode, block_n=block_n, pos_scale=pos_scale,
                rope_scale=float(rope_scale), rope_scale_c=float(rs_c), n_global=ng, n_local=nl,
                tau=float(tau_val), chunk_size=chunk_size, n_chunk=n_chunk,
                select_score=select_score, chunk_agg=chunk_agg)
    save(case, meta, dict(q=qd, k=K, v=V, tau=tau, inv_freq_a=invf, inv_freq_c=invf_c, idx=idx,
                          newpos_k=npk, newpos_q=npq, out=out))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", required=True,
                    help="directory of the reference checkout (its modules are imported)")
    ap.add_argument("--only", default=None, help="generate only cases whose name contains this")
    args = ap.parse_args()
    global ONLY
    ONLY = args.only
    sys.path.insert(0, args.ref)
    torch.set_num_threads(os.cpu_count() or 1)
    # fp32 only: the Triton interpreter does not evaluate bf16 arithmetic faithfully (numpy has
    # no bf16; its bf16 outputs come back as ~1e10 garbage), so bf16 parity is anchored on the
    # fp32-pinned oracle instead.
    f32 = torch.float32
    # shared path: PI freq, ragged N, small k_max to drive the 30->25->20 fallback + truncation
    gen_shared(None, "shared_selection_triton_exact_2", "shared_pi_freq_f32", 2, 300, 64, 64, 160,
               11, f32, pos_scale=0.5, measure=True)
    gen_shared(None, "shared_selection_triton_exact", "shared_exact_sort_f32", 2, 256, 64, 32, 96,
               12, f32, pos_scale=0.75)
    gen_shared(None, "shared_selection_triton_exact_2", "shared_pi_margin_f32", 2, 320, 64, 64,
               200, 13, f32, select_score="margin", pos_scale=0.5)
    gen_shared(None, "shared_selection_triton_exact_2", "shared_pi_expmass_f32", 2, 320, 64, 64,
               200, 14, f32, select_score="expmass", pos_scale=0.5)
    gen_shared(None, "shared_selection_triton_YaRN_exact", "shared_yarn_freq_f32", 2, 288, 64, 32,
               128, 15, f32, geom="yarn")
    gen_shared(None, "shared_selection_triton_hybrid_exact", "shared_hybrid_expmass_f32", 2, 288,
               64, 32, 128, 16, f32, geom="hybrid", pos_scale=0.5, select_score="expmass")
    gen_shared(None, "shared_selection_triton_exact_2", "shared_pi_freq_tau1_f32", 2, 256, 64, 64,
               2048, 18, f32, tau_val=1.0)
    # benchmark config 0 at its own shape
    gen_cfg0("config0_f32")
    # dense Dual Chunk Attention (dca_kernel.py), GQA, three chunk relations, ragged tail
    gen_dca_dense("dca_dense_gqa_f32", 4, 2, 700, 64, 320, 512, 64, 61)
    # PQ-Union: overflow-forcing k_max, expmass and freq ranking, yarn select geometry
    gen_pq("pq_union_expmass_f32", 2, 288, 64, 160, 21, f32)
    gen_pq("pq_union_freq_f32", 2, 256, 64, 4096, 22, f32, select_score="freq")
    gen_pq("pq_union_yarn_f32", 2, 256, 64, 128, 23, f32, geom="yarn")
    # PQ-Stream: max / full advance, skip on/off, ragged N, BN 32 and 64
    # Dual Chunk Attention position tables (the DCA selection geometry's position rule)
    gen_dca_tables("dca_tables_s320_w64", 320, 64, 1024, 2048)
    # chunk_exact: chunk-granular selection, exact static budget
    gen_chunk("chunk_expmass_f32", 2, 384, 64, 256, 41, f32)
    gen_chunk("chunk_freq_f32", 2, 320, 64, 192, 42, f32, select_score="freq")
    gen_chunk("chunk_mean_c32_f32", 2, 384, 64, 384, 43, f32, chunk_size=32, chunk_agg="mean")
    gen_pqstream("pqstream_max_f32", 2, 300, 64, 31, f32)
    gen_pqstream("pqstream_full_f32", 2, 256, 64, 32, f32, pos_advance="full")
    gen_pqstream("pqstream_bn64_f32", 2, 288, 64, 33, f32, block_n=64, geom="yarn")
    gen_pqstream("pqstream_noskip_f32", 2, 256, 64, 34, f32, use_skip=False, pos_scale=0.5)
    # decode: one query per head against the cache (the reference's torch decode rules)
    gen_decode("decode_pi_cap_f32", "pi", 3, 700, 64, 51, k_max=96, pos_scale=0.5, tau_val=12.0)
    gen_decode("decode_pi_pct_f32", "pi", 2, 523, 128, 52, k_max=4096, pct_decode=50.0,
               tau_val=12.0)
    gen_decode("decode_pi_yarn_f32", "pi", 2, 640, 64, 53, k_max=128, geom="yarn")
    gen_decode("decode_rank_cap_f32", "rank", 3, 700, 64, 54, k_max=80, pos_scale=0.5,
               tau_val=12.0)
    gen_decode("decode_stream_bn32_f32", "stream", 2, 777, 64, 55, tau_val=9.0)
    gen_decode("decode_chunk_expmass_f32", "chunk", 3, 650, 64, 57, k_max=256, tau_val=12.0,
               n_chunk=6)
    # (freq ranking ties whole groups of chunks; torch.topk orders ties arbitrarily, so the
    # pinned cases rank by exp(s - m))
    gen_decode("decode_chunk_mean_c32_f32", "chunk", 2, 500, 64, 58, k_max=256, tau_val=20.0,
               n_chunk=1, chunk_size=32, chunk_agg="mean")
    gen_decode("decode_stream_bn64_f32", "stream", 2, 600, 128, 56, block_n=64, geom="yarn",
               tau_val=9.0)


if __name__ == "__main__":
    main()
