"""Drop-in for ``shared_selection_triton_YaRN_exact``: the exact_2 kernel with YaRN positions
everywhere (raw positions, YaRN NTK-by-parts frequencies, mscale as rope_scale).  Same call
surface as exact_2 (shared_selection_triton_YaRN_exact.py:442-496); the hook reads the YaRN
frequencies and mscale from a yarn-loaded model's rotary embedding (:681-690)."""
from __future__ import annotations

from .hooks import make_shared_installer
from .shared_selection_exact_2 import shared_pi_attention  # noqa: F401  (identical surface)

install_shared_pi_forward = make_shared_installer("yarn", shared_pi_attention, select_score=True)
