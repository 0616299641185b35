"""MLX-layout affine group quantization on the GPU (``mx.quantize`` / ``mx.dequantize`` stand-ins).

``quantize`` packs the last axis into (data uint32, scales, biases) exactly as
the reference's 4-slot cache and ``nn.QuantizedLinear`` store it
(``cache.py:430-436``, ``model.py:1047``); ``dequantize`` inverts it with the
bit-extract formula of ``kernels/mlp.py:176-198``. Both call the C ABI
(``motif_quantize`` / ``motif_dequantize``).

Quantizer: per group, scale = max((max−min)/(2^bits−1), 1e-7) signed towards
the larger-magnitude edge, bias = that edge (or 0 when it rounds to code 0),
codes = clamp(round((w − bias)/scale)), IEEE fp32 throughout.
"""

from __future__ import annotations

import torch

from ._native import check, contiguous, dtype_code, lib, ptr, stream


def quantize(w: torch.Tensor, group_size: int = 64, bits: int = 4):
    """(…, D) -> (data (…, D·bits/32) uint32, scales (…, D/g), biases (…, D/g))."""
    *lead, D = w.shape
    if D % group_size:
        raise ValueError(f"last axis {D} is not a multiple of group_size {group_size}")
    rows = w.numel() // D if D else 0
    wc = contiguous(w)
    data = torch.empty((*lead, D * bits // 32), dtype=torch.uint32, device=w.device)
    scales = torch.empty((*lead, D // group_size), dtype=w.dtype, device=w.device)
    biases = torch.empty_like(scales)
    if rows:
        check(lib.motif_quantize(dtype_code(w), bits, group_size, ptr(wc), rows, D, ptr(data), ptr(scales),
                                 ptr(biases), stream(w.device)), "quantize")
    return data, scales, biases


def dequantize(data: torch.Tensor, scales: torch.Tensor, biases: torch.Tensor, group_size: int = 64,
               bits: int = 4) -> torch.Tensor:
    """Inverse of :func:`quantize`; output dtype = scales.dtype."""
    from .kernels.mlp import _dequant_probe

    return _dequant_probe(data, scales, biases, group_size=group_size, bits=bits)
