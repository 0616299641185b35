"""mlx_motif on B200: the Motif GDA decode hot path as sm_100a CUDA kernels.

Drop-in for the reference's operator layer (``mlx_motif.kernels``), 4-slot
cache API (``mlx_motif.cache``) and quantized linear, plus a CUDA-graph
decode engine (``mlx_motif.model.MotifDecoder``). All compute runs in the
in-tree C-ABI library ``libmotif_b200.so`` (``include/motif_b200.h``).
"""

from . import _native  # noqa: F401  (loads the CUDA library; raises if it is missing)
from .cache import MotifGroupedKVCache, MotifGroupedQuantizedKVCache, MotifVanillaKVCache  # noqa: F401
from .linear import QuantizedLinear, quantized_matmul  # noqa: F401
from .quantization import dequantize, quantize  # noqa: F401

__version__ = "0.1.0"
