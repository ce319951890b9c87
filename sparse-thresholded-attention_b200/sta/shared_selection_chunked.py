"""Drop-in for ``shared_selection_triton_chunked`` (chunk_exact): selection at chunk
granularity with an exact static budget.  ``shared_chunk_attention`` keeps the reference
signature and return tuple (shared_selection_triton_chunked.py:249-320); the budget helpers
``n_forced_chunks`` / ``derive_n_chunk`` (:114-146) and the measurement accessors
``get_chunk_stats`` / ``reset_chunk_stats`` (:72-110) keep their names.

The forced-chunk rule is the one the reference's own golden restates (chunked.py:378-384);
the reference module imports it from ``chunk_recall_core``, which the reference does not ship.
Ties among equal chunk masses at the top-n_chunk cut keep the lowest chunk indices (the
reference's ``torch.topk`` order among ties is implementation-defined).
"""
from __future__ import annotations

from ._surface import _check_prefill
from .core import Geometry, forward


def _fresh():
    return {"cells": 0, "cap_cnt": None, "tot_cnt": None, "slots": None}


_CHUNK_STATS = {"prefill": _fresh(), "decode": _fresh()}


def reset_chunk_stats():
    _CHUNK_STATS["prefill"] = _fresh()
    _CHUNK_STATS["decode"] = _fresh()


def get_chunk_stats():
    """Cells processed and slots gathered since the last reset (recall fields need the
    per-key passer masks, which this build does not materialise: reported as 0)."""
    def ph(d):
        tot = d["cells"]
        slt = float(d["slots"].item()) if d["slots"] is not None else 0.0
        return {"cells": tot, "recall_count": 0.0, "utilisation": 0.0,
                "slots_per_cell": (slt / tot) if tot else 0.0}
    return {"prefill": ph(_CHUNK_STATS["prefill"]), "decode": ph(_CHUNK_STATS["decode"])}


def n_forced_chunks(chunk_size, n_global, n_local, tile):
    """Worst-case number of chunks the forced global + local sets occupy."""
    C = chunk_size
    return (n_global + C - 1) // C + (n_local + tile - 1 + C - 1) // C + 1


def derive_n_chunk(k_max, chunk_size, n_global, n_local, tile):
    """Chunks to select so that forced + selected fill k_max exactly."""
    C = chunk_size
    assert k_max % C == 0, f"k_max={k_max} must be divisible by chunk_size={C}"
    nf = n_forced_chunks(C, n_global, n_local, tile)
    n = k_max // C - nf
    assert n > 0, (f"chunk_size={C} leaves no budget: forced needs {nf} chunks ({nf * C} slots) "
                   f"of k_max={k_max}.")
    return n


def shared_chunk_attention(q, k, v, tau, inv_freq_a, inv_freq_c, pos_scale_a=1.0, rope_scale_a=1.0,
                           sm_scale=None, n_global=32, n_local=32, tile=32, k_max=4096,
                           chunk_size=16, n_chunk=None, block_n=64, block_k=64, q_pos_base=0,
                           select_score="expmass", chunk_agg="sum", measure=False):
    """Returns (out, usize, kept_size)."""
    if n_chunk is None:
        n_chunk = derive_n_chunk(k_max, chunk_size, n_global, n_local, tile)
    nf = n_forced_chunks(chunk_size, n_global, n_local, tile)
    N = q.shape[2]
    nC_total = (N + chunk_size - 1) // chunk_size
    bound = min(nC_total, nf + n_chunk) * chunk_size
    assert bound <= k_max, (f"budget overflow: min(nC={nC_total}, {nf} forced + {n_chunk} "
                            f"selected) * {chunk_size} = {bound} > k_max={k_max}")
    _check_prefill(q_pos_base)
    if chunk_agg not in ("sum", "mean"):
        raise KeyError(chunk_agg)
    out, st, _ = forward("chunk", q, k, v, tau, Geometry(inv_freq_a, pos_scale_a, rope_scale_a),
                         Geometry(inv_freq_c, 1.0, 1.0), sm_scale=sm_scale, n_global=n_global,
                         n_local=n_local, tile=tile, k_max=k_max, select_score=select_score,
                         chunk_size=chunk_size, n_chunk=n_chunk, chunk_agg=chunk_agg)
    usize, kept = st["usize"], st["kept_size"]
    if q.shape[0] == 1:
        usize, kept = usize[0], kept[0]
    if measure:
        d = _CHUNK_STATS["prefill"]
        d["cells"] += kept.numel()
        s = kept.double().sum()
        d["slots"] = s if d["slots"] is None else d["slots"] + s
    return out, usize, kept


def install_shared_pi_forward(*args, **kwargs):
    """The chunk_exact HuggingFace hook (shared_selection_triton_chunked.py:488); see
    ``sta.hooks.install_chunk_forward``."""
    from .hooks import install_chunk_forward
    return install_chunk_forward(*args, **kwargs)
