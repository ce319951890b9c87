"""Dense Dual Chunk Attention (ChunkLlama) on the B200 kernel -- drop-in for the reference's
``dca_kernel.py`` (``patch_model_with_dca`` / ``unpatch_model`` / ``install_dca_forward`` /
``get_mscale``).

The reference's attention core (dca_kernel.py:447-487) runs three flash-attention calls per
query segment (intra / succ / inter) and merges them by log-sum-exp; here one fused kernel
(``sta_dca_forward``) runs one online softmax over all causal keys, each key block scored with
the query rotation of its chunk relation.  ``dca_attention`` is the functional op; the patched
``LlamaAttention.forward`` routes prefill through it and decodes with the same kernel on the
128-row query slab that holds the new token.

Differences in execution only: the KV cache stores RAW keys (the reference stores keys already
rotated at j mod chunk_len); k / v keep their kv-head count (no ``repeat_kv`` copy).
"""
from __future__ import annotations

import math
from typing import Any, Dict

import torch

from . import core


def get_mscale(scale: float = 1.0) -> float:
    """ChunkLlama's length scaling of cos / sin (dca_kernel.py:166-170): 0.05 ln(scale) + 1."""
    if scale <= 1:
        return 1.0
    return 0.05 * math.log(scale) + 1.0


def flash_attn_status() -> str:
    """Which attention path runs (the reference reports flash-attn vs its PyTorch fallback)."""
    return "B200 fused dense-DCA kernel (tcgen05), no fallback"


def dca_attention(q, k, v, inv_freq, *, chunk_size: int, local_window: int,
                  rope_scale: float = 1.0, sm_scale=None, q_pos_base: int = 0):
    """Dense DCA attention of RAW q (Z, H, Nq, D) against RAW k / v (Z, Hkv, N, D),
    Nq = N - q_pos_base.  Keys rotate at j mod L (L = chunk_size - local_window), queries at the
    intra / succ / inter positions by chunk relation; cos / sin carry ``rope_scale``."""
    if not (0 < local_window < chunk_size):
        raise AssertionError(f"need 0 < w({local_window}) < s({chunk_size})")
    return core.dca_dense(q, k, v, inv_freq, chunk_size=chunk_size, local_window=local_window,
                          rope_scale=rope_scale, sm_scale=sm_scale, q_pos_base=q_pos_base)


def _base_inv_freq(module, dim):
    cfg = getattr(module, "config", None)
    theta = 10000.0
    rp = getattr(cfg, "rope_parameters", None) or getattr(cfg, "rope_scaling", None)
    if isinstance(rp, dict) and rp.get("rope_theta"):
        theta = float(rp["rope_theta"])
    elif getattr(cfg, "rope_theta", None):
        theta = float(cfg.rope_theta)
    theta = float(int(theta))  # the reference builds its tables from int(base)
    return 1.0 / (theta ** (torch.arange(0, dim, 2, dtype=torch.float32) / dim))


def _make_forward(chunk_size: int, pretrain_len: int, local_window: int):
    s, c, w = chunk_size, pretrain_len, local_window

    def dca_forward(self, hidden_states, position_embeddings=None, attention_mask=None,
                    past_key_values=None, **kwargs):
        bsz, q_len, _ = hidden_states.shape
        if past_key_values is None:
            past_key_values = kwargs.get("past_key_value", None)
        D = self.head_dim
        scale = float(getattr(self, "scaling", None) or (1.0 / math.sqrt(D)))
        q = self.q_proj(hidden_states).view(bsz, q_len, -1, D).transpose(1, 2)
        k = self.k_proj(hidden_states).view(bsz, q_len, -1, D).transpose(1, 2)
        v = self.v_proj(hidden_states).view(bsz, q_len, -1, D).transpose(1, 2)
        start_pos = 0
        if past_key_values is not None and hasattr(past_key_values, "get_seq_length"):
            try:
                start_pos = int(past_key_values.get_seq_length(self.layer_idx))
            except TypeError:
                start_pos = int(past_key_values.get_seq_length())
        if not (start_pos == 0 or q_len == 1):
            raise AssertionError(
                f"dca_forward: chunked prefill is unsupported (start_pos={start_pos}, "
                f"q_len={q_len}). Prefill must be a single pass over an empty cache; decode "
                "must be one token.")
        kv_seq_len = start_pos + q_len
        # mscale follows the reference's table rule (dca_kernel.py:194-241): tables built at the
        # pretraining length (mscale 1), rebuilt with mscale(len / c) and 512 positions of
        # headroom whenever a call's sequence outgrows them, otherwise kept as they are
        if not hasattr(self, "_dca_max_len"):
            self._dca_max_len, self._dca_mscale = c, 1.0
        if kv_seq_len > self._dca_max_len:
            self._dca_mscale = get_mscale(kv_seq_len / c)
            self._dca_max_len = kv_seq_len + 512
        if past_key_values is not None and hasattr(past_key_values, "update"):
            k, v = past_key_values.update(k, v, self.layer_idx)
        invf = getattr(self, "_dca_inv_freq", None)
        if invf is None or invf.device != q.device:
            invf = _base_inv_freq(self, D).to(q.device)
            self._dca_inv_freq = invf
        kw = dict(chunk_size=s, local_window=w, rope_scale=self._dca_mscale, sm_scale=scale)
        if q_len > 1:
            out = dca_attention(q, k, v, invf, **kw)
        else:
            P = k.shape[2] - 1                      # the new token's position
            base = (P // 128) * 128                 # the 128-row slab that holds it
            slab = torch.zeros((bsz, q.shape[1], P + 1 - base, D), dtype=q.dtype, device=q.device)
            slab[:, :, -1] = q[:, :, 0]
            out = dca_attention(slab, k, v, invf, q_pos_base=base, **kw)[:, :, -1:]
        attn = out.transpose(1, 2).reshape(bsz, q_len, -1).contiguous()
        return self.o_proj(attn), None

    return dca_forward


def _is_patchable_llama(module) -> bool:
    required = ("q_proj", "k_proj", "v_proj", "o_proj", "head_dim", "layer_idx")
    if not all(hasattr(module, a) for a in required):
        return False
    return hasattr(module, "num_heads") or (
        hasattr(module, "config") and hasattr(module.config, "num_attention_heads"))


def patch_model_with_dca(model, chunk_size: int, pretrain_len: int,
                         local_window: int) -> Dict[str, Any]:
    """Class-level patch of every Llama attention forward (dca_kernel.py:541-624).  Returns
    the ``originals`` dict for ``unpatch_model``; raises if no attention layer was found."""
    import transformers.models.llama.modeling_llama as _llama_mod
    assert 0 < local_window < chunk_size, f"need 0 < w({local_window}) < s({chunk_size})"
    assert chunk_size < pretrain_len, f"need s({chunk_size}) < c({pretrain_len})"
    if (chunk_size - local_window) % 128:
        raise ValueError("this build needs chunk_size - local_window to be a multiple of 128")
    n_patched = sum(1 for _, m in model.named_modules() if _is_patchable_llama(m))
    if n_patched == 0:
        raise RuntimeError(
            "patch_model_with_dca patched 0 attention layers -- the model would have run DENSE. "
            "Check that this is a Llama-style model and that the attention modules expose "
            "q_proj/k_proj/v_proj/o_proj/head_dim/layer_idx.")
    for _, m in model.named_modules():  # fresh tables, as the reference's new rotary modules
        for a in ("_dca_mscale", "_dca_max_len", "_dca_inv_freq"):
            if hasattr(m, a):
                delattr(m, a)
    fwd = _make_forward(chunk_size, pretrain_len, local_window)
    originals: Dict[str, Any] = {}
    for cls_name in ("LlamaAttention", "LlamaFlashAttention2", "LlamaSdpaAttention"):
        cls = getattr(_llama_mod, cls_name, None)
        if cls is not None:
            originals[cls_name] = cls.forward
            cls.forward = fwd
    originals["_model"] = model
    originals["_n_patched"] = n_patched
    return originals


def unpatch_model(originals: Dict[str, Any]) -> None:
    """Restore the attention forwards saved by ``patch_model_with_dca``."""
    import transformers.models.llama.modeling_llama as _llama_mod
    for cls_name in ("LlamaAttention", "LlamaFlashAttention2", "LlamaSdpaAttention"):
        if cls_name in originals:
            cls = getattr(_llama_mod, cls_name, None)
            if cls is not None:
                cls.forward = originals[cls_name]
    model = originals.get("_model")
    if model is not None:
        for _, m in model.named_modules():
            for a in ("_dca_mscale", "_dca_max_len", "_dca_inv_freq"):
                if hasattr(m, a):
                    delattr(m, a)


def install_dca_forward(model, chunk_size: int = 3072, context_window: int = 4096,
                        local_window: int = 512) -> Dict[str, Any]:
    """Same name and defaults as the reference's wrapper (dca_kernel.py:660-664)."""
    return patch_model_with_dca(model, chunk_size, context_window, local_window)
