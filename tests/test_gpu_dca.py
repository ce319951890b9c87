"""Dense Dual Chunk Attention kernel (sta_dca_forward) vs the reference and the oracle (B200).

Bar: fp32 inputs within 1e-4 of the reference's own output (tests/golden/dca_dense_gqa_f32.npz,
the reference's dca_forward on a one-layer Llama) and of the float64 oracle; bf16 inputs within
max-abs 2e-2 / mean-abs 1e-3 of the oracle.
"""
import json
import math
import os

import numpy as np
import pytest
import torch

from conftest import oracle

from sta import core
from sta import dca_kernel as dk
from sta.synth import SynthSpec, make_inputs, rope_inv_freq

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
F32_TOL = 1e-4
BF16_MAX, BF16_MEAN = 2e-2, 1e-3


def fixture():
    z = np.load(os.path.join(HERE, "golden", "dca_dense_gqa_f32.npz"))
    return json.loads(str(z["meta"])), z


def test_dense_dca_fp32_matches_reference_output():
    meta, z = fixture()
    q, k, v = (torch.from_numpy(z[x]).cuda()[None] for x in ("q", "k", "v"))
    out = core.dca_dense(q, k, v, torch.from_numpy(z["inv_freq"]),
                         chunk_size=meta["chunk_size"], local_window=meta["local_window"],
                         rope_scale=meta["mscale"], sm_scale=meta["sm_scale"])
    torch.cuda.synchronize()
    assert core.device_error() == 0
    err = np.abs(out[0].cpu().numpy() - z["out"])
    assert err.max() <= F32_TOL, err.max()


@pytest.mark.parametrize("D,Hk,N", [(128, 2, 1100), (64, 1, 777), (128, 4, 300)])
def test_dense_dca_bf16_vs_oracle(D, Hk, N):
    H = 4
    q, k, v = make_inputs(SynthSpec(n_heads=H, n_kv_heads=Hk, seq_len=N, head_dim=D,
                                    n_planted=8, seed=90 + D + N, dtype=torch.bfloat16))
    s_, w_ = 320, 64
    invf = rope_inv_freq(D, 1e4)
    ms = dk.get_mscale(N / 512)
    out = dk.dca_attention(q.cuda(), k.cuda(), v.cuda(), invf, chunk_size=s_, local_window=w_,
                           rope_scale=ms)
    torch.cuda.synchronize()
    assert core.device_error() == 0
    G = H // Hk
    o = oracle.dca_dense_attention(q[0].float().numpy(), np.repeat(k[0].float().numpy(), G, 0),
                                   np.repeat(v[0].float().numpy(), G, 0), s_, w_, invf.numpy(),
                                   ms)
    err = np.abs(out[0].float().cpu().numpy() - o)
    assert err.max() <= BF16_MAX and err.mean() <= BF16_MEAN, (err.max(), err.mean())


def test_plain_causal_rope_attention_fp32_vs_oracle():
    """chunk_size 0: ordinary causal attention with RoPE at the true positions."""
    H, N, D = 2, 300, 64
    q, k, v = make_inputs(SynthSpec(n_heads=H, n_kv_heads=H, seq_len=N, head_dim=D, seed=95))
    invf = rope_inv_freq(D, 1e4)
    out = core.dca_dense(q.cuda(), k.cuda(), v.cuda(), invf, chunk_size=0, local_window=0)
    ref = oracle.dense_rope_attention(q[0].numpy(), k[0].numpy(), v[0].numpy(), invf.numpy())
    assert np.abs(out[0].cpu().numpy() - ref).max() <= F32_TOL


def test_dense_dca_query_slab_reproduces_whole_call():
    H, Hk, N, D = 4, 2, 900, 128
    q, k, v = make_inputs(SynthSpec(n_heads=H, n_kv_heads=Hk, seq_len=N, head_dim=D, seed=96,
                                    dtype=torch.bfloat16))
    q, k, v = q.cuda(), k.cuda(), v.cuda()
    invf = rope_inv_freq(D, 1e4)
    kw = dict(chunk_size=320, local_window=64, rope_scale=1.05)
    whole = core.dca_dense(q, k, v, invf, **kw)
    for base in (256, 768):
        part = core.dca_dense(q[:, :, base:].contiguous(), k, v, invf, q_pos_base=base, **kw)
        assert torch.equal(part, whole[:, :, base:])


def _tiny_llama(meta):
    from transformers import LlamaConfig, LlamaForCausalLM
    torch.manual_seed(meta["seed"])
    H, Hkv, D = meta["H"], meta["Hkv"], meta["D"]
    cfg = LlamaConfig(hidden_size=H * D, num_attention_heads=H, num_key_value_heads=Hkv,
                      head_dim=D, num_hidden_layers=1, intermediate_size=64, vocab_size=64,
                      max_position_embeddings=meta["pretrain_len"], rope_theta=10000.0)
    model = LlamaForCausalLM(cfg).float().eval()
    x = torch.randn(1, meta["N"], H * D) * 2.0
    return model, x


def test_patched_llama_attention_matches_reference_and_decodes():
    """install_dca_forward on the same one-layer Llama (same seed and input) reproduces the
    reference's attention output; one decode step equals the kernel on the 128-row slab."""
    from transformers import DynamicCache
    meta, z = fixture()
    model, x = _tiny_llama(meta)
    model = model.cuda()
    x = x.cuda()
    originals = dk.install_dca_forward(model, chunk_size=meta["chunk_size"],
                                       context_window=meta["pretrain_len"],
                                       local_window=meta["local_window"])
    try:
        attn = model.model.layers[0].self_attn
        cap = {}
        h = attn.o_proj.register_forward_pre_hook(lambda m, i: cap.__setitem__("out", i[0]))
        cache = DynamicCache()
        with torch.no_grad():
            attn(x, position_embeddings=None, attention_mask=None, past_key_values=cache)
            N, H, D = meta["N"], meta["H"], meta["D"]
            out = cap["out"].view(1, N, H, D).transpose(1, 2)[0].cpu().numpy()
            assert np.abs(out - z["out"]).max() <= F32_TOL
            # decode one token: the kernel on the slab that holds position N
            x1 = torch.randn(1, 1, H * D, device="cuda")
            attn(x1, position_embeddings=None, attention_mask=None, past_key_values=cache)
            got = cap["out"].view(1, 1, H, D)[0, 0]
            k_all = cache.layers[0].keys if hasattr(cache, "layers") else cache.key_cache[0]
            v_all = cache.layers[0].values if hasattr(cache, "layers") else cache.value_cache[0]
            q1 = attn.q_proj(x1).view(1, 1, H, D).transpose(1, 2)
            base = (N // 128) * 128
            slab = torch.zeros((1, H, N + 1 - base, D), device="cuda")
            slab[:, :, -1] = q1[:, :, 0]
            ref = core.dca_dense(slab, k_all, v_all, torch.from_numpy(z["inv_freq"]),
                                 chunk_size=meta["chunk_size"], local_window=meta["local_window"],
                                 rope_scale=meta["mscale"], sm_scale=meta["sm_scale"],
                                 q_pos_base=base)[0, :, -1]
            assert torch.allclose(got, ref, atol=1e-6, rtol=0)
        h.remove()
    finally:
        dk.unpatch_model(originals)
