"""Drop-in for ``shared_selection_triton_hybrid_exact``: selection (Kernel A) in one geometry
(YaRN), repositioning + attention in another (PI).  ``shared_pi_attention`` keeps the hybrid
signature (shared_selection_triton_hybrid_exact.py:450-510)."""
from __future__ import annotations

from ._surface import shared_attention
from .core import Geometry
from .hooks import make_shared_installer


def shared_pi_attention(q, k, v, tau,
                        inv_freq_a, pos_scale_a, rope_scale_a,
                        inv_freq_c, pos_scale_c, rope_scale_c,
                        pct=30.0, sm_scale=None, n_global=32, n_local=32, tile=32, k_max=1024,
                        block_n=64, block_k=64, q_pos_base=0, measure=False, select_score="freq",
                        dca_chunk_size=None, dca_local_window=None):
    """Kernel A scores with (inv_freq_a, pos_scale_a, rope_scale_a); the selection's PI
    repositioning and Kernel C use (inv_freq_c, pos_scale_c, rope_scale_c).

    Extension: with dca_chunk_size / dca_local_window the selection geometry uses Dual Chunk
    Attention position ids (ChunkLlama's rule, dca_kernel.py:194-231) instead of positions x
    pos_scale_a; chunk_size - local_window must be a multiple of 256."""
    dca = None if dca_chunk_size is None else (int(dca_chunk_size), int(dca_local_window))
    return shared_attention(q, k, v, tau, Geometry(inv_freq_a, pos_scale_a, rope_scale_a, dca),
                            Geometry(inv_freq_c, pos_scale_c, rope_scale_c), pct=pct,
                            sm_scale=sm_scale, n_global=n_global, n_local=n_local, tile=tile,
                            k_max=k_max, q_pos_base=q_pos_base, measure=measure,
                            select_score=select_score)


install_shared_pi_forward = make_shared_installer("hybrid", shared_pi_attention,
                                                  select_score=True, hybrid=True)
