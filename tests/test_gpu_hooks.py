"""The HuggingFace attention hooks on a tiny random-init Llama (needs a B200).

Invariant used as the check: with tau = +inf every causal key passes the threshold, pct = 100
keeps the whole pooled set, k_max >= N caps nothing and pos_scale = 1 leaves positions
unchanged, so thresholded attention IS dense causal RoPE attention; the patched model must
reproduce the unpatched model's logits, and greedy decoding must produce the same tokens.
"""
import math

import pytest
import torch

pytestmark = pytest.mark.gpu


def tiny_llama(seed=0, n_kv=2):
    from transformers import LlamaConfig, LlamaForCausalLM
    torch.manual_seed(seed)
    cfg = LlamaConfig(vocab_size=211, hidden_size=256, intermediate_size=512,
                      num_hidden_layers=2, num_attention_heads=4, num_key_value_heads=n_kv,
                      head_dim=64, max_position_embeddings=4096, rope_theta=10000.0,
                      attn_implementation="eager")
    return LlamaForCausalLM(cfg).cuda().float().eval()


def set_tau(model, value):
    for layer in model.model.layers:
        sa = layer.self_attn
        sa.tau_head_vec = torch.full((model.config.num_attention_heads,), value,
                                     device="cuda")


@pytest.mark.parametrize("modname", ["shared_selection_exact_2", "shared_selection_exact"])
def test_hook_prefill_and_decode_match_dense_at_tau_inf(modname):
    import importlib
    import transformers.models.llama.modeling_llama as ml
    mod = importlib.import_module("sta." + modname)
    orig_forward = ml.LlamaAttention.forward
    model = tiny_llama()
    ids = torch.randint(0, 211, (1, 192), generator=torch.Generator().manual_seed(1)).cuda()
    with torch.no_grad():
        ref_logits = model(ids).logits
        ref_gen = model.generate(ids, max_new_tokens=3, do_sample=False)
    try:
        set_tau(model, math.inf)
        mod.install_shared_pi_forward(model, pct=100.0, context_window=4096, tile=64,
                                      k_max=512)
        with torch.no_grad():
            logits = model(ids).logits
            gen = model.generate(ids, max_new_tokens=3, do_sample=False)
        assert torch.isfinite(logits).all()
        err = (logits - ref_logits).abs().max().item()
        assert err <= 1e-3, err
        assert torch.equal(gen, ref_gen)
        sa = model.model.layers[0].self_attn
        assert sa.spi_last_kept.shape == (4, 3)
        # every tile keeps all of its causal keys plus the in-tile future of its local block
        assert int(sa.spi_last_kept[:, -1].min()) >= 192
    finally:
        ml.LlamaAttention.forward = orig_forward


def test_hook_threshold_selects_and_matches_oracle():
    """At a finite tau the hook's attention output (the input of o_proj) equals the oracle's
    shared thresholded attention of the layer's own q / k / v (captured at the projections),
    run on the device's Kernel A votes with the geometry the hook freezes at prefill."""
    import numpy as np
    import transformers.models.llama.modeling_llama as ml
    from conftest import oracle
    from sta import core
    from sta import shared_selection_exact_2 as st
    from sta.core import Geometry
    orig_forward = ml.LlamaAttention.forward
    model = tiny_llama(seed=3)
    N, H, Hk, D = 512, 4, 2, 64
    ids = torch.randint(0, 211, (1, N), generator=torch.Generator().manual_seed(2)).cuda()
    sa = model.model.layers[1].self_attn
    cap = {}
    hooks = [sa.q_proj.register_forward_hook(lambda m, i, o: cap.__setitem__("q", o)),
             sa.k_proj.register_forward_hook(lambda m, i, o: cap.__setitem__("k", o)),
             sa.v_proj.register_forward_hook(lambda m, i, o: cap.__setitem__("v", o)),
             sa.o_proj.register_forward_pre_hook(lambda m, i: cap.__setitem__("out", i[0]))]
    try:
        set_tau(model, 0.5)
        st.install_shared_pi_forward(model, pct=30.0, tile=64, k_max=256)
        with torch.no_grad():
            out = model(ids).logits
        assert torch.isfinite(out).all()
        assert int(sa.spi_last_kept[:, -1].max()) < N
        q = cap["q"].view(1, N, H, D).transpose(1, 2)[0].contiguous()
        k = cap["k"].view(1, N, Hk, D).transpose(1, 2)[0].contiguous()
        v = cap["v"].view(1, N, Hk, D).transpose(1, 2)[0].contiguous()
        got = cap["out"].view(1, N, H, D).transpose(1, 2)[0].cpu().numpy()
        inv_a, ps_a, rs_a = sa.spi_sel
        ps = sa.spi_pos_scale
        ps_a = ps if ps_a is None else ps_a
        tau = torch.full((H,), 0.5)
        votes = core.select(q, k, tau, Geometry(inv_a.cpu(), ps_a, rs_a), tile=64)["votes"]
        dense = core.expand_compact(votes, H, N, 64).cpu().numpy().astype(np.int32)
        G = H // Hk
        qx = q.cpu().numpy()
        kx = np.repeat(k.cpu().numpy(), G, 0)
        vx = np.repeat(v.cpu().numpy(), G, 0)
        inv_c, ps_c, rs_c = sa.spi_att
        ps_c = ps if ps_c is None else ps_c
        o = oracle.shared_attention(qx, kx, vx, tau.numpy(), inv_a.cpu().numpy(), ps_a, rs_a,
                                    inv_c.cpu().numpy(), ps_c, rs_c, pct=30.0,
                                    sm_scale=sa.scaling, tile=64, k_max=256,
                                    sel={"votes": dense})
        assert np.abs(got - o[0]).max() <= 1e-4
        np.testing.assert_array_equal(sa.spi_last_kept.cpu().numpy(), o[2])
    finally:
        for h in hooks:
            h.remove()
        ml.LlamaAttention.forward = orig_forward


@pytest.mark.parametrize("modname,installer,kw", [
    ("shared_selection_perquery", "install_shared_pi_forward", dict(k_max=512)),
    ("shared_selection_chunked", "install_shared_pi_forward", dict(k_max=512, chunk_size=16)),
    ("pqstream_kernel", "install_pqstream_forward", dict()),
])
def test_per_query_hooks_prefill_and_decode_match_dense_at_tau_inf(modname, installer, kw):
    """tau = +inf keeps every causal key; with positions that reproduce the native ones (dense
    ranks over all keys = the positions themselves; PQ-Stream 'full' with every key kept gives
    relative positions, which RoPE does not distinguish) the hooks equal dense attention."""
    import importlib
    import transformers.models.llama.modeling_llama as ml
    mod = importlib.import_module("sta." + modname)
    orig_forward = ml.LlamaAttention.forward
    model = tiny_llama(seed=5)
    ids = torch.randint(0, 211, (1, 160), generator=torch.Generator().manual_seed(4)).cuda()
    with torch.no_grad():
        ref_logits = model(ids).logits
        ref_gen = model.generate(ids, max_new_tokens=3, do_sample=False)
    try:
        set_tau(model, math.inf)
        if modname == "pqstream_kernel":
            kw = dict(kw, pos_advance="full")
        if modname == "shared_selection_chunked":
            kw = dict(kw, n_chunk=4096 // 16)
        getattr(mod, installer)(model, context_window=4096, **kw)
        with torch.no_grad():
            logits = model(ids).logits
            gen = model.generate(ids, max_new_tokens=3, do_sample=False)
        assert torch.isfinite(logits).all()
        err = (logits - ref_logits).abs().max().item()
        assert err <= 1e-3, err
        assert torch.equal(gen, ref_gen)
    finally:
        ml.LlamaAttention.forward = orig_forward
