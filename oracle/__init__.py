"""CPU oracle for the Motif decode hot path (TEST INFRASTRUCTURE ONLY).

This package is the checker, never the product: only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline legs may import
it. The product path (``mlx_motif``) never imports it and fails loudly when
its CUDA library is missing.

Parity status (see ``motif_oracle`` for the per-function citations):
  * PolyNorm: pinned against the reference's only numeric golden vector
    (``tests/fixtures/motif_parity_cases.json`` -> ``polynorm_reference_2x3``,
    copied under ``tests/golden/``).
  * Affine dequantize: pinned by the reference's own bit-extract kernel
    (``src/mlx_motif/kernels/mlp.py:176-198``), which its tests hold equal to
    ``mx.dequantize`` (``tests/test_dequant_probe.py:21-38``).
  * Affine quantize (``mx.quantize``, MLX 0.31.2, not vendored): parity
    UNPINNED against MLX. The restated algorithm is documented in
    ``motif_oracle.quantize``; the CUDA kernels are bit-exact to it.
  * SDPA, RoPE, RMSNorm, quantized matmul (MLX / mlx-lm internals): restated
    from their published definitions; checked by tolerance, parity unpinned
    beyond the reference's own tolerance tests.
"""

from .motif_oracle import *  # noqa: F401,F403
