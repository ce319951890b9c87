"""Drop-in for ``shared_selection_triton_perquery`` (PQ-Union, "pq_exact"): per-query key sets
via the tile's full union + forced keys, dense-rank positions and a per-query slot bitmask.

``shared_pq_attention`` keeps the reference signature and return tuple
(shared_selection_triton_perquery.py:459-525); the measurement-only overflow counters keep the
reference accessors (get_overflow_stats / reset_overflow_stats, :56-110)."""
from __future__ import annotations

from ._surface import _check_prefill
from .core import Geometry, forward


def _fresh():
    return {"cells": 0, "overflow": None, "union_sum": None, "union_max": None}


_OVF_STATS = {"prefill": _fresh(), "decode": _fresh()}


def reset_overflow_stats():
    _OVF_STATS["prefill"] = _fresh()
    _OVF_STATS["decode"] = _fresh()


def _phase_stats(d):
    tot = d["cells"]
    ovf = int(d["overflow"].item()) if d["overflow"] is not None else 0
    usum = int(d["union_sum"].item()) if d["union_sum"] is not None else 0
    umax = int(d["union_max"].item()) if d["union_max"] is not None else 0
    return {"total_cells": tot, "overflow_cells": ovf,
            "overflow_frac": (ovf / tot) if tot else 0.0,
            "union_mean": (usum / tot) if tot else 0.0, "union_max": umax}


def get_overflow_stats():
    """Cumulative since the last reset: how often |union U forced| exceeded k_max, plus
    union-size statistics.  One host sync here, none during the run."""
    return {"prefill": _phase_stats(_OVF_STATS["prefill"]),
            "decode": _phase_stats(_OVF_STATS["decode"])}


def _ovf_accumulate(overflow, usize, phase="prefill"):
    d = _OVF_STATS[phase]
    d["cells"] += overflow.numel()
    ov, us, um = overflow.sum(), usize.long().sum(), usize.max()
    if d["overflow"] is None:
        d["overflow"], d["union_sum"], d["union_max"] = ov, us, um
    else:
        d["overflow"] = d["overflow"] + ov
        d["union_sum"] = d["union_sum"] + us
        d["union_max"] = d["union_max"].maximum(um)


def shared_pq_attention(q, k, v, tau, inv_freq_a, inv_freq_c, pos_scale_a=1.0, rope_scale_a=1.0,
                        sm_scale=None, n_global=32, n_local=32, tile=32, k_max=4096,
                        block_n=64, block_k=64, q_pos_base=0, select_score="expmass"):
    """Returns (out, usize, kept_size, overflow).  tile must be 32."""
    if tile != 32:
        raise AssertionError("pq_exact packs per-query keep bits into int32 -> tile must be 32")
    if n_global + n_local + tile - 1 > k_max:
        raise AssertionError(f"forced set ({n_global + n_local + tile - 1}) exceeds k_max={k_max}")
    _check_prefill(q_pos_base)
    out, st, _ = forward("pq_union", q, k, v, tau, Geometry(inv_freq_a, pos_scale_a, rope_scale_a),
                         Geometry(inv_freq_c, 1.0, 1.0), sm_scale=sm_scale, n_global=n_global,
                         n_local=n_local, tile=32, k_max=k_max, select_score=select_score)
    usize, kept, ovf = st["usize"], st["kept_size"], st["overflow"].bool()
    if q.shape[0] == 1:
        usize, kept, ovf = usize[0], kept[0], ovf[0]
    _ovf_accumulate(ovf, usize)
    return out, usize, kept, ovf


def install_shared_pi_forward(*args, **kwargs):
    """The PQ-Union HuggingFace hook (shared_selection_triton_perquery.py:784); see
    ``sta.hooks.install_pq_forward``."""
    from .hooks import install_pq_forward
    return install_pq_forward(*args, **kwargs)
