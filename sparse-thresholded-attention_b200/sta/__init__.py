"""sta -- B200-native (sm_100a) exact-max thresholded attention prefill.

Host-side mirror of the reference repository's prefill call surfaces, backed by libsta.so
(hand-written CUDA for sm_100a behind a C ABI, include/sta.h):

    sta.shared_selection_exact          <- shared_selection_triton_exact
    sta.shared_selection_exact_2        <- shared_selection_triton_exact_2
    sta.shared_selection_yarn_exact     <- shared_selection_triton_YaRN_exact
    sta.shared_selection_hybrid_exact   <- shared_selection_triton_hybrid_exact
    sta.shared_selection_perquery       <- shared_selection_triton_perquery (PQ-Union)
    sta.pqstream_kernel                 <- pqstream_kernel (PQ-Stream)
    sta.shared_selection_chunked        <- shared_selection_triton_chunked (chunk_exact)
    sta.hooks                           the HuggingFace attention hooks of every family
    sta.core                            forward / forward_host / decode and the stage calls
    sta.partition                       multi-GPU units (kv-head ranges, query slabs)
"""
from . import core  # noqa: F401
from ._lib import lib  # noqa: F401
from .core import Geometry  # noqa: F401

__all__ = ["core", "lib", "Geometry"]
