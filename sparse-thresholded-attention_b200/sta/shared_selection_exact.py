"""Drop-in for ``shared_selection_triton_exact`` (the original exact-max shared-PI kernel,
frequency voting only).  ``shared_pi_attention`` keeps the reference signature and return
tuple (shared_selection_triton_exact.py:376-423)."""
from __future__ import annotations

from ._surface import shared_attention
from .core import Geometry
from .hooks import make_shared_installer


def shared_pi_attention(q, k, v, tau, inv_freq, pos_scale=1.0, pct=30.0, sm_scale=None,
                        rope_scale=1.0, n_global=32, n_local=32, tile=32, k_max=1024,
                        block_n=64, block_k=64, q_pos_base=0, measure=False):
    """q,k,v: (1,H,N,D) RAW.  Returns (out, shared_size, kept_size, kpct, overflow, kpct_meas,
    overflow20)."""
    g = Geometry(inv_freq, pos_scale, rope_scale)
    return shared_attention(q, k, v, tau, g, g, pct=pct, sm_scale=sm_scale, n_global=n_global,
                            n_local=n_local, tile=tile, k_max=k_max, q_pos_base=q_pos_base,
                            measure=measure, select_score="freq")


install_shared_pi_forward = make_shared_installer("pi", shared_pi_attention)
