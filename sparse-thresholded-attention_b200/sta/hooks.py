"""HuggingFace Llama attention hooks (``install_shared_pi_forward`` and friends).

Mirror of the reference hooks (shared_selection_triton_exact_2.py:658-767, the YaRN / hybrid /
perquery / pqstream variants): the patched ``LlamaAttention.forward`` projects q/k/v, stores RAW
k/v in the KV cache, freezes the PI position scale at prefill and routes the prefill through
the B200 op.  Differences: k/v are passed GQA-native (no ``repeat_kv`` copy).

Decode (past_len > 0) is not on the accelerated path: it runs the reference's per-query torch
rule (threshold + forced global/local/self + k_max cap by score + reposition) in torch, exactly
as the reference's default ``decode_backend="torch"`` does.
"""
from __future__ import annotations

import math

import torch


def _rope(x, pos, inv_freq, rope_scale):
    half = x.shape[-1] // 2
    ang = pos[..., None].to(torch.float32) * inv_freq.to(torch.float32)
    c = torch.cos(ang) * rope_scale
    s = torch.sin(ang) * rope_scale
    x1, x2 = x[..., :half].float(), x[..., half:].float()
    return torch.cat([x1 * c - x2 * s, x2 * c + x1 * s], dim=-1)


@torch.no_grad()
def decode_step(q, K, V, tau, q_pos, sel, att, n_global, n_local, k_max, pct_decode=100.0,
                reposition="pi", sm_scale=None):
    """One decode query per head (torch).  q (H,D); K, V (H,M,D) (GQA already expanded).
    sel / att: (inv_freq, pos_scale, rope_scale) of the selection and attend geometries.
    reposition: "pi" (newpos = rank + cummax(pos*pos_scale_c - rank)) or "rank" (dense ranks)."""
    H, M, D = K.shape
    dev = K.device
    if sm_scale is None:
        sm_scale = 1.0 / math.sqrt(D)
    ia, psa, rsa = sel
    ic, psc, rsc = att
    pos = torch.arange(M, device=dev)
    qs = _rope(q, torch.tensor(float(q_pos) * psa, device=dev), ia.to(dev), rsa)
    ks = _rope(K, pos.float() * psa, ia.to(dev), rsa)
    score = torch.einsum("hd,hmd->hm", qs, ks) * sm_scale
    m = score.max(-1).values
    keep = score >= (m - tau.to(dev).float())[:, None]
    forced = torch.zeros(M, dtype=torch.bool, device=dev)
    forced[:min(n_global, M)] = True
    forced[max(0, q_pos - n_local + 1):q_pos + 1] = True
    forced[q_pos] = True
    if pct_decode < 100.0:
        n_pass = keep.sum(-1)
        b = torch.ceil(pct_decode / 100.0 * n_pass).clamp(min=1).long()
        sp = torch.where(keep, score, torch.full_like(score, -math.inf))
        cut = torch.gather(torch.sort(sp, -1, descending=True).values, -1,
                           (b - 1).clamp(0, M - 1)[:, None])
        keep = keep & (score >= cut)
    kp = keep | forced[None]
    nf = int(forced.sum())
    bud = k_max - nf
    nonf = kp & ~forced[None]
    snf = torch.where(nonf, score, torch.full_like(score, -math.inf))
    ci = min(max(bud - 1, 0), M - 1)
    cutc = torch.sort(snf, -1, descending=True).values[:, ci:ci + 1]
    kept_nf = nonf & (score >= cutc) if bud > 0 else torch.zeros_like(nonf)
    final = torch.where((kp.sum(-1) > k_max)[:, None], forced[None] | kept_nf, kp)
    rank0 = (final.int().cumsum(-1) - 1).float()
    if reposition == "pi":
        cr = torch.where(final, pos.float()[None] * psc - rank0, torch.full_like(rank0, -math.inf))
        newpos = rank0 + torch.cummax(cr, -1).values
    else:
        newpos = rank0
    out = torch.empty((H, D), dtype=q.dtype, device=dev)
    for h in range(H):
        kk = final[h].nonzero().squeeze(-1)
        qr = _rope(q[h], newpos[h, q_pos], ic.to(dev), rsc)
        kr = _rope(K[h, kk], newpos[h, kk], ic.to(dev), rsc)
        a = torch.softmax((kr @ qr) * sm_scale, -1)
        out[h] = (a[:, None] * V[h, kk].float()).sum(0).to(q.dtype)
    return out


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
                G = q.shape[1] // k.shape[1]
                Kf = k[0].repeat_interleave(G, 0)
                Vf = v[0].repeat_interleave(G, 0)
                outs = []
                for i in range(N):
                    P = past_len + i
                    outs.append(decode_step(q[0, :, i], Kf[:, :P + 1], Vf[:, :P + 1],
                                            self.tau_head_vec, P, (inv_a, psa, rsa),
                                            (inv_c, psc, rsc), self.spi_ng, self.spi_nl,
                                            self.spi_kmax, self.spi_pct_decode, "pi",
                                            self.scaling))
                out = torch.stack(outs, 1).unsqueeze(0)
            attn = out.transpose(1, 2).reshape(B, N, -1).contiguous()
            return self.o_proj(attn), None

        ml.LlamaAttention.forward = spi_forward

    return install_shared_pi_forward
