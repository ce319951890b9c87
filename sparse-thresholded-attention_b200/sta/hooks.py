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

import math

import torch


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
