"""HuggingFace Llama attention hooks (``install_shared_pi_forward`` and friends).

Mirror of the reference hooks (shared_selection_triton_exact_2.py:658-767, the YaRN / hybrid /
perquery / pqstream variants): the patched ``LlamaAttention.forward`` projects q/k/v, stores RAW
k/v in the KV cache, freezes the PI position scale at prefill and routes the prefill through
the B200 op.  Differences: k/v are passed GQA-native (no ``repeat_kv`` copy).

Decode (past_len > 0) and the per-query prefill mode run the reference's per-query rule
(threshold + optional top-pct + forced global/local/self + k_max cap by score + PI reposition,
shared_selection_triton_exact.py:464-560) on the device: ``sta.core.decode``, one launch sequence
per query position, GQA-native.
"""
from __future__ import annotations

import torch


def _check_device_waits():
    """Raise when a bounded device wait of the prefill kernels expired (the launches return
    before the kernels run, so such a failure only shows in the device error word; reading it
    synchronises the stream once per prefill call)."""
    from .core import device_error
    code = device_error()
    if code:
        raise RuntimeError(f"thresholded attention: a bounded device wait expired (code {code}); "
                           "the layer output is incomplete")


def _rope_theta(cfg):
    theta = 10000.0
    rp = getattr(cfg, "rope_parameters", None) or getattr(cfg, "rope_scaling", None)
    if isinstance(rp, dict) and rp.get("rope_theta"):
        theta = float(rp["rope_theta"])
    elif getattr(cfg, "rope_theta", None):
        theta = float(cfg.rope_theta)
    return theta


def _base_inv_freq(model):
    cfg = model.config
    hd = getattr(cfg, "head_dim", None) or (cfg.hidden_size // cfg.num_attention_heads)
    th = _rope_theta(cfg)
    return 1.0 / (th ** (torch.arange(0, hd, 2, dtype=torch.float32) / hd))


def make_shared_installer(geom, attention_fn, select_score=False, hybrid=False):
    """Build ``install_shared_pi_forward`` for a shared-selection module.
    geom: "pi" (base frequencies, pos_scale = min(1, W/L)), "yarn" (the model's YaRN
    frequencies + mscale, raw positions) or "hybrid" (YaRN select, PI attend)."""

    def install_shared_pi_forward(model, pct=30.0, context_window=4096, n_global=32,
                                  n_local=32, tile=32, k_max=1024, block_n=32, block_k=32,
                                  max_len=None, pct_decode=100.0, decode_backend="torch",
                                  select_backend="torch", prefill_mode="shared",
                                  measure=False, select_score="freq", apply_mscale=True):
        import transformers.models.llama.modeling_llama as ml
        rotary = model.model.rotary_emb
        inv_rot = rotary.inv_freq.detach().float()
        att_scale = float(getattr(rotary, "attention_scaling", 1.0))
        base = _base_inv_freq(model)
        for li, layer in enumerate(model.model.layers):
            sa = layer.self_attn
            dev = sa.q_proj.weight.device
            if geom == "pi":
                sa.spi_sel = (inv_rot.to(dev), None, att_scale)
                sa.spi_att = (inv_rot.to(dev), None, att_scale)
            elif geom == "yarn":
                rs = att_scale if apply_mscale else 1.0
                sa.spi_sel = (inv_rot.to(dev), 1.0, rs)
                sa.spi_att = (inv_rot.to(dev), 1.0, rs)
            else:  # hybrid
                rs = att_scale if apply_mscale else 1.0
                sa.spi_sel = (inv_rot.to(dev), 1.0, rs)
                sa.spi_att = (base.to(dev), None, 1.0)
            sa.spi_pct, sa.spi_W = pct, context_window
            sa.spi_ng, sa.spi_nl, sa.spi_tile, sa.spi_kmax = n_global, n_local, tile, k_max
            sa.spi_layer_idx = getattr(sa, "layer_idx", li)
            sa.spi_max_len = max_len
            sa.spi_pos_scale = None
            sa.spi_pct_decode = pct_decode
            sa.spi_measure = measure
            sa.spi_select_score = select_score
            sa.spi_prefill_mode = prefill_mode

        def spi_forward(self, hidden_states, position_embeddings=None, attention_mask=None,
                        past_key_values=None, **kwargs):
            B, N, _ = hidden_states.shape
            hs = (B, N, -1, self.head_dim)
            q = self.q_proj(hidden_states).view(hs).transpose(1, 2)
            k = self.k_proj(hidden_states).view(hs).transpose(1, 2)
            v = self.v_proj(hidden_states).view(hs).transpose(1, 2)
            cache = past_key_values if past_key_values is not None else kwargs.get("past_key_value")
            past_len = 0
            if cache is not None:
                try:
                    past_len = int(cache.get_seq_length(self.spi_layer_idx))
                except TypeError:
                    past_len = int(cache.get_seq_length())
                k, v = cache.update(k, v, self.spi_layer_idx)
            if past_len == 0:
                L = self.spi_max_len if self.spi_max_len is not None else N
                self.spi_pos_scale = min(1.0, self.spi_W / float(L))
            ps = self.spi_pos_scale
            inv_a, psa, rsa = self.spi_sel
            inv_c, psc, rsc = self.spi_att
            psa = ps if psa is None else psa
            psc = ps if psc is None else psc
            if past_len == 0 and self.spi_prefill_mode == "shared":
                from .core import Geometry
                from ._surface import shared_attention
                res = shared_attention(q, k, v, self.tau_head_vec, Geometry(inv_a, psa, rsa),
                                       Geometry(inv_c, psc, rsc), pct=self.spi_pct,
                                       sm_scale=self.scaling, n_global=self.spi_ng,
                                       n_local=self.spi_nl, tile=self.spi_tile,
                                       k_max=self.spi_kmax, measure=self.spi_measure,
                                       select_score=self.spi_select_score)
                out = res[0]
                (self.spi_last_shared, self.spi_last_kept, self.spi_last_kpct,
                 self.spi_last_overflow, self.spi_last_kpct_meas,
                 self.spi_last_overflow20) = res[1:]
                _check_device_waits()
            else:
                from .core import Geometry, decode
                outs = []
                for i in range(N):
                    P = past_len + i
                    o, _, _ = decode("pi", q[:, :, i], k[:, :, :P + 1], v[:, :, :P + 1],
                                     self.tau_head_vec, Geometry(inv_a, psa, rsa),
                                     Geometry(inv_c, psc, rsc), n_global=self.spi_ng,
                                     n_local=self.spi_nl, k_max=self.spi_kmax,
                                     pct_decode=self.spi_pct_decode, sm_scale=self.scaling)
                    outs.append(o[0])
                out = torch.stack(outs, 1).unsqueeze(0)
            attn = out.transpose(1, 2).reshape(B, N, -1).contiguous()
            return self.o_proj(attn), None

        ml.LlamaAttention.forward = spi_forward

    return install_shared_pi_forward


# ---------------------------------------------------------------------------------------------
# Per-query-selection families: PQ-Union, chunk_exact, PQ-Stream
# ---------------------------------------------------------------------------------------------
def _pq_geometry(model, select_geom, apply_mscale):
    """Selection / attend geometry of the per-query families
    (shared_selection_triton_perquery.py:798-830): 'pi' selects with the base frequencies at
    compressed positions (pos_scale frozen at prefill), 'yarn' with the model's YaRN frequencies
    (+ mscale) at raw positions; the attend geometry is always base RoPE, rope_scale 1."""
    if select_geom not in ("pi", "yarn"):
        raise AssertionError(f"select_geom must be pi|yarn, got {select_geom!r}")
    rotary = model.model.rotary_emb
    inv_rot = rotary.inv_freq.detach().float()
    att_scale = float(getattr(rotary, "attention_scaling", 1.0))
    base = _base_inv_freq(model)
    if select_geom == "yarn":
        return inv_rot, (att_scale if apply_mscale else 1.0), base
    return base, 1.0, base


def _install_per_query(kind, model, prefix, cfg):
    """Patch LlamaAttention.forward for one per-query family.  ``kind``: 'pq' | 'chunk' |
    'stream'; ``prefix``: the attribute prefix the reference uses ('spi' or 'pqs')."""
    import transformers.models.llama.modeling_llama as ml
    inv_a, rs_a, inv_c = _pq_geometry(model, cfg["select_geom"], cfg["apply_mscale"])
    for li, layer in enumerate(model.model.layers):
        sa = layer.self_attn
        dev = sa.q_proj.weight.device
        setattr(sa, f"{prefix}_inv_freq_a", inv_a.to(dev))
        setattr(sa, f"{prefix}_rope_scale_a", rs_a)
        setattr(sa, f"{prefix}_inv_freq_c", inv_c.to(dev))
        setattr(sa, f"{prefix}_geom", cfg["select_geom"])
        setattr(sa, f"{prefix}_W", cfg["context_window"])
        setattr(sa, f"{prefix}_ng", cfg["n_global"])
        setattr(sa, f"{prefix}_nl", cfg["n_local"])
        setattr(sa, f"{prefix}_tile", cfg["tile"])
        setattr(sa, f"{prefix}_block_n", cfg["block_n"])
        setattr(sa, f"{prefix}_block_k", cfg["block_k"])
        setattr(sa, f"{prefix}_layer_idx", getattr(sa, "layer_idx", li))
        setattr(sa, f"{prefix}_max_len", cfg["max_len"])
        setattr(sa, f"{prefix}_pos_scale_a", None)
        setattr(sa, f"{prefix}_decode_backend", cfg["decode_backend"])
        setattr(sa, f"{prefix}_select_backend", cfg["select_backend"])
        setattr(sa, f"{prefix}_prefill_mode", cfg["prefill_mode"])
        for key in ("k_max", "select_score", "measure", "chunk_size", "n_chunk", "chunk_agg",
                    "pos_advance", "use_skip", "num_warps"):
            if key in cfg:
                name = {"k_max": "kmax", "pos_advance": "advance"}.get(key, key)
                setattr(sa, f"{prefix}_{name}", cfg[key])
    shared_mode = {"pq": "shared", "chunk": "shared", "stream": "stream"}[kind]

    def per_query_forward(self, hidden_states, position_embeddings=None, attention_mask=None,
                          past_key_values=None, **kwargs):
        g = lambda n: getattr(self, f"{prefix}_{n}")  # noqa: E731
        B, N, _ = hidden_states.shape
        hs = (B, N, -1, self.head_dim)
        q = self.q_proj(hidden_states).view(hs).transpose(1, 2)
        k = self.k_proj(hidden_states).view(hs).transpose(1, 2)
        v = self.v_proj(hidden_states).view(hs).transpose(1, 2)
        cache = past_key_values if past_key_values is not None else kwargs.get("past_key_value")
        past_len = 0
        if cache is not None:
            try:
                past_len = int(cache.get_seq_length(g("layer_idx")))
            except TypeError:
                past_len = int(cache.get_seq_length())
            k, v = cache.update(k, v, g("layer_idx"))
        if past_len == 0:
            if g("geom") == "yarn":
                setattr(self, f"{prefix}_pos_scale_a", 1.0)
            else:
                L = g("max_len") if g("max_len") is not None else N
                setattr(self, f"{prefix}_pos_scale_a", min(1.0, g("W") / float(L)))
        ps = g("pos_scale_a")
        from .core import Geometry, decode
        if past_len == 0 and g("prefill_mode") == shared_mode:
            args = (q, k, v, self.tau_head_vec, g("inv_freq_a"), g("inv_freq_c"))
            kw = dict(pos_scale_a=ps, rope_scale_a=g("rope_scale_a"), sm_scale=self.scaling,
                      n_global=g("ng"), n_local=g("nl"), tile=g("tile"), block_n=g("block_n"))
            if kind == "pq":
                from .shared_selection_perquery import shared_pq_attention
                out, usize, kept, ovf = shared_pq_attention(*args, k_max=g("kmax"),
                                                            select_score=g("select_score"), **kw)
                self.spi_last_usize, self.spi_last_kept, self.spi_last_overflow = usize, kept, ovf
            elif kind == "chunk":
                from .shared_selection_chunked import shared_chunk_attention
                out, usize, kept = shared_chunk_attention(
                    *args, k_max=g("kmax"), chunk_size=g("chunk_size"), n_chunk=g("n_chunk"),
                    select_score=g("select_score"), chunk_agg=g("chunk_agg"), **kw)
                self.spi_last_usize, self.spi_last_kept = usize, kept
            else:
                from .pqstream_kernel import pqstream_attention
                out, span, kept, blocks, skipped = pqstream_attention(
                    *args, pos_advance=g("advance"), use_skip=g("use_skip"), **kw)
                self.pqs_last_span, self.pqs_last_kept = span, kept
                self.pqs_last_skipped = skipped
            _check_device_waits()
        else:
            # decode, or the per-query prefill mode: one device decode call per query position
            mode = {"pq": "rank", "chunk": "chunk", "stream": "stream"}[kind]
            ga = Geometry(g("inv_freq_a"), ps, g("rope_scale_a"))
            gc = Geometry(g("inv_freq_c"), 1.0, 1.0)
            extra = {}
            if kind == "chunk":
                extra = dict(chunk_size=g("chunk_size"), n_chunk=g("n_chunk"),
                             chunk_agg=g("chunk_agg"), select_score=g("select_score"))
            outs = []
            for i in range(N):
                P = past_len + i
                o, _, _ = decode(mode, q[:, :, i], k[:, :, :P + 1], v[:, :, :P + 1],
                                 self.tau_head_vec, ga, gc, n_global=g("ng"), n_local=g("nl"),
                                 k_max=getattr(self, f"{prefix}_kmax", 0) or 0,
                                 block_n=g("block_n"), sm_scale=self.scaling, **extra)
                outs.append(o[0])
            out = torch.stack(outs, 1).unsqueeze(0)
        attn = out.transpose(1, 2).reshape(B, N, -1).contiguous()
        return self.o_proj(attn), None

    ml.LlamaAttention.forward = per_query_forward


def install_pq_forward(model, pct=30.0, context_window=4096, n_global=32, n_local=32, tile=32,
                       k_max=4096, block_n=32, block_k=32, max_len=None, pct_decode=100.0,
                       decode_backend="torch", select_backend="torch", prefill_mode="shared",
                       measure=False, select_score="expmass", select_geom="pi",
                       apply_mscale=True):
    """PQ-Union hooks (shared_selection_triton_perquery.py:784-830).  pct / pct_decode are
    accepted and ignored, as in the reference (full union / full per-query set)."""
    if n_global + n_local > k_max:
        raise AssertionError(f"decode forced set (n_global={n_global} + n_local={n_local}) "
                             f"exceeds k_max={k_max}")
    _install_per_query("pq", model, "spi", dict(
        context_window=context_window, n_global=n_global, n_local=n_local, tile=tile,
        k_max=k_max, block_n=block_n, block_k=block_k, max_len=max_len,
        decode_backend=decode_backend, select_backend=select_backend, prefill_mode=prefill_mode,
        measure=measure, select_score=select_score, select_geom=select_geom,
        apply_mscale=apply_mscale))


def install_chunk_forward(model, pct=30.0, context_window=4096, n_global=32, n_local=32, tile=32,
                          k_max=4096, block_n=32, block_k=32, max_len=None, pct_decode=100.0,
                          decode_backend="triton", select_backend="triton", prefill_mode="shared",
                          measure=False, select_score="expmass", select_geom="pi",
                          apply_mscale=True, chunk_size=16, n_chunk=None, chunk_agg="sum"):
    """chunk_exact hooks (shared_selection_triton_chunked.py:488-560); n_chunk None derives the
    budget that fills k_max exactly."""
    from .shared_selection_chunked import derive_n_chunk
    if chunk_agg not in ("sum", "mean"):
        raise AssertionError(f"chunk_agg must be sum|mean, got {chunk_agg!r}")
    if n_chunk is None:
        n_chunk = derive_n_chunk(k_max, chunk_size, n_global, n_local, tile)
    _install_per_query("chunk", model, "spi", dict(
        context_window=context_window, n_global=n_global, n_local=n_local, tile=tile,
        k_max=k_max, block_n=block_n, block_k=block_k, max_len=max_len,
        decode_backend=decode_backend, select_backend=select_backend, prefill_mode=prefill_mode,
        measure=measure, select_score=select_score, select_geom=select_geom,
        apply_mscale=apply_mscale, chunk_size=chunk_size, n_chunk=n_chunk, chunk_agg=chunk_agg))


def install_pqstream_forward(model, context_window=4096, n_global=32, n_local=32, tile=32,
                             block_n=32, block_k=32, max_len=None, decode_backend="torch",
                             select_backend="torch", prefill_mode="stream", select_geom="pi",
                             apply_mscale=True, pos_advance="max", use_skip=True, num_warps=None,
                             pct=None, pct_decode=None, k_max=None, select_score=None,
                             measure=False, **_unused):
    """PQ-Stream hooks (pqstream_kernel.py:834-997); pct / pct_decode / k_max / select_score /
    measure are accepted and ignored, as in the reference (no budget, no ranking)."""
    if pos_advance not in ("max", "full"):
        raise AssertionError(f"pos_advance must be max|full, got {pos_advance!r}")
    if prefill_mode == "shared":
        prefill_mode = "stream"
    _install_per_query("stream", model, "pqs", dict(
        context_window=context_window, n_global=n_global, n_local=n_local, tile=tile,
        block_n=block_n, block_k=block_k, max_len=max_len, decode_backend=decode_backend,
        select_backend=select_backend, prefill_mode=prefill_mode, select_geom=select_geom,
        apply_mscale=apply_mscale, pos_advance=pos_advance, use_skip=use_skip,
        num_warps=num_warps))
