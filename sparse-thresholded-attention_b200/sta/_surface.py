"""Shared implementation behind the reference-compatible module surfaces.

Each public module of this package mirrors one reference module's prefill call surface (same
function names, positional order, defaults and return tuples) and routes it to libsta.so.
"""
from __future__ import annotations

import math

import torch

from . import core
from .core import Geometry


def _batch(q, k, v):
    if q.dim() != 4:
        raise ValueError("q, k, v must be (Z, H, N, D)")
    return q.shape[0]


_Q_POS_BASE_MSG = ("q_pos_base must be 0 here: every reference prefill call passes 0 with q and k "
                   "covering the same positions 0..N-1.  Query slabs (q holding positions "
                   "q_pos_base..N-1 against all N keys) are sta.core.forward(..., q_pos_base=...)")


def _check_prefill(q_pos_base):
    """Raise ValueError unless q_pos_base == 0 (see _Q_POS_BASE_MSG)."""
    if int(q_pos_base) != 0:
        raise ValueError(_Q_POS_BASE_MSG)


def shared_attention(q, k, v, tau, ga: Geometry, gc: Geometry, pct=30.0, sm_scale=None,
                     n_global=32, n_local=32, tile=32, k_max=1024, q_pos_base=0, measure=False,
                     select_score="freq"):
    """Shared-selection prefill (Kernel A -> selection -> Kernel C) for one or two geometries.
    Returns the reference's 7-tuple (out, shared_size, kept_size, kpct, overflow, kpct_meas,
    overflow20) with the reference's dtypes (int64 sizes, int32 pct, bool flags)."""
    _check_prefill(q_pos_base)
    if select_score not in ("freq", "margin", "expmass"):
        raise KeyError(select_score)
    Z = _batch(q, k, v)
    out, st, _ = core.forward("shared", q, k, v, tau, ga, gc, sm_scale=sm_scale, pct=pct,
                              n_global=n_global, n_local=n_local, tile=tile, k_max=k_max,
                              select_score=select_score, measure=measure)
    shared = st["shared_size"].long()
    kept = st["kept_size"].long()
    kpct = st["chosen"]
    ovf = st["overflow"].bool()
    kpm = st["kpct_meas"]
    ovf20 = st["overflow20"].bool()
    if Z == 1:
        shared, kept, kpct, ovf, kpm, ovf20 = (x[0] for x in (shared, kept, kpct, ovf, kpm, ovf20))
    if measure:
        _measure_report(kpct, ovf, ovf20, pct, k_max)
    return out, shared, kept, kpct, ovf, kpm, ovf20


def _measure_report(chosen, orig_overflow, overflow20, pct, k_max):
    """Host-side prints of the reference's measure=True mode (exact_2.py:374-383)."""
    adjusted = orig_overflow & (chosen > 0)
    if bool(adjusted.any()):
        vals, counts = torch.unique(chosen[adjusted].cpu(), return_counts=True)
        summary = ", ".join(f"{int(a)}%:{int(b)}" for a, b in zip(vals, counts))
        print(f"Adjusted top-pct to fit k_max={k_max}: {summary} (requested {pct:g}%).",
              flush=True)
    if bool(overflow20.any()):
        start = max(0, int(round(pct)))
        steps = [start] + [c for c in (25, 20) if c < start]
        print(f"WARNING: {int(overflow20.sum().item())} (head,tile) sets still exceed "
              f"k_max={k_max} even at top {steps[-1]}%; gather will truncate those tiles.",
              flush=True)


def default_sm_scale(q):
    return 1.0 / math.sqrt(q.shape[-1])
