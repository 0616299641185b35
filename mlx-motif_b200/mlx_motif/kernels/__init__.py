"""CUDA (sm_100a) kernels of the Motif decode hot path, with the reference's operator surface.

Same exports as ``src/mlx_motif/kernels/__init__.py:21-50``. Every op calls
the in-tree C-ABI library; ``MLX_MOTIF_DISABLE_KERNELS=1`` (read at import)
routes each op to its ``*_reference`` twin, a torch composition used only as
a correctness mode.

    attention.py — sdpa_dual_v, sdpa_dual_v_q4  (shared-QK dual-V SDPA)
    gda.py       — gda_post, gda_post_split     (GDA post-attention reduction)
    mlp.py       — polynorm, polynorm_mul, _dequant_probe
"""

from .attention import (
    sdpa_dual_v,
    sdpa_dual_v_q4,
    sdpa_dual_v_q4_reference,
    sdpa_dual_v_reference,
)
from .gda import (
    gda_post,
    gda_post_reference,
    gda_post_split,
    gda_post_split_reference,
)
from .mlp import (
    _dequant_probe,  # noqa: F401 — test helper, not in __all__ (as in the reference)
    polynorm,
    polynorm_mul,
    polynorm_reference,
)

__all__ = [
    "polynorm",
    "polynorm_reference",
    "polynorm_mul",
    "gda_post",
    "gda_post_reference",
    "gda_post_split",
    "gda_post_split_reference",
    "sdpa_dual_v",
    "sdpa_dual_v_reference",
    "sdpa_dual_v_q4",
    "sdpa_dual_v_q4_reference",
]
