"""Drop-in for ``pqstream_kernel`` (PQ-Stream): per-query threshold sets with streamed block
positions, no k_max.  ``pqstream_attention`` keeps the reference signature and return tuple
(pqstream_kernel.py:498-564); the span / kept / skip counters keep the reference accessors
(get_overflow_stats / reset_overflow_stats / reset_span_stats, :89-154)."""
from __future__ import annotations

from .core import Geometry, forward

ADV_MAX = 0
ADV_FULL = 1
_ADV = {"max": ADV_MAX, "full": ADV_FULL}


def _fresh():
    return {"cells": 0, "span_sum": None, "span_max": None, "kept_sum": None, "rows": 0,
            "blocks": None, "skipped": None}


_STATS = {"prefill": _fresh(), "decode": _fresh()}


def reset_overflow_stats():
    _STATS["prefill"] = _fresh()
    _STATS["decode"] = _fresh()


reset_span_stats = reset_overflow_stats


def _phase_stats(d):
    tot = d["cells"]
    ssum = float(d["span_sum"].item()) if d["span_sum"] is not None else 0.0
    smax = float(d["span_max"].item()) if d["span_max"] is not None else 0.0
    ksum = float(d["kept_sum"].item()) if d["kept_sum"] is not None else 0.0
    blk = int(d["blocks"].item()) if d["blocks"] is not None else 0
    skp = int(d["skipped"].item()) if d["skipped"] is not None else 0
    return {"total_cells": tot, "span_mean": (ssum / tot) if tot else 0.0, "span_max": smax,
            "kept_mean": (ksum / d["rows"]) if d["rows"] else 0.0, "blocks": blk,
            "skipped": skp, "skip_frac": (skp / blk) if blk else 0.0, "overflow_cells": 0,
            "overflow_frac": 0.0}


def get_overflow_stats():
    return {"prefill": _phase_stats(_STATS["prefill"]), "decode": _phase_stats(_STATS["decode"])}


def _acc(dst, key, val, reduce="sum"):
    if dst[key] is None:
        dst[key] = val
    elif reduce == "max":
        dst[key] = dst[key].maximum(val)
    else:
        dst[key] = dst[key] + val


def _stats_accumulate(span, kept, blocks, skipped, phase="prefill"):
    d = _STATS[phase]
    d["cells"] += span.numel()
    d["rows"] += kept.numel()
    _acc(d, "span_sum", span.double().sum())
    _acc(d, "span_max", span.max(), reduce="max")
    _acc(d, "kept_sum", kept.double().sum())
    _acc(d, "blocks", blocks.long().sum())
    _acc(d, "skipped", skipped.long().sum())


def pqstream_attention(q, k, v, tau, inv_freq_a, inv_freq_c, pos_scale_a=1.0, rope_scale_a=1.0,
                       sm_scale=None, n_global=32, n_local=32, tile=32, block_n=32,
                       pos_advance="max", q_pos_base=0, use_skip=True, num_warps=None):
    """Returns (out, span, kept, blocks, skipped).  num_warps is accepted and ignored."""
    if tile != 32:
        raise AssertionError("BLOCK_M is fixed at 32 by the tile convention")
    if q_pos_base != 0:
        raise AssertionError(f"pqstream prefill expects q_pos_base == 0, got {q_pos_base}")
    if block_n < tile - 1:
        raise AssertionError(f"block_n={block_n} < tile-1={tile - 1}")
    if pos_advance not in _ADV:
        raise KeyError(pos_advance)
    if block_n not in (32, 64):
        raise NotImplementedError("block_n must be 32 or 64")
    out, st, _ = forward("pq_stream", q, k, v, tau, Geometry(inv_freq_a, pos_scale_a, rope_scale_a),
                         Geometry(inv_freq_c, 1.0, 1.0), sm_scale=sm_scale, n_global=n_global,
                         n_local=n_local, tile=32, k_max=0, block_n=block_n,
                         pos_advance=pos_advance, use_skip=use_skip)
    span, kept, blocks, skipped = st["span"], st["kept"], st["blocks"], st["skipped"]
    if q.shape[0] == 1:
        span, kept, blocks, skipped = span[0], kept[0], blocks[0], skipped[0]
    _stats_accumulate(span, kept, blocks, skipped)
    return out, span, kept, blocks, skipped


def install_pqstream_forward(*args, **kwargs):
    """The PQ-Stream HuggingFace hook (pqstream_kernel.py:834); see
    ``sta.hooks.install_pqstream_forward``."""
    from .hooks import install_pqstream_forward as f
    return f(*args, **kwargs)


install_shared_pi_forward = install_pqstream_forward   # the reference's alias (:998)
