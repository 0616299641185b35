"""PolyNorm (and its fused ·up form) plus the dequant probe (test helper).

Operator surface of ``src/mlx_motif/kernels/mlp.py``: ``polynorm``
(``mlp.py:119-157``), ``polynorm_reference`` (``mlp.py:108-116``) and
``_dequant_probe`` (``mlp.py:213-255``). The kernels are ``motif_polynorm``,
``motif_polynorm_mul`` and ``motif_dequantize`` of the C ABI.
"""

from __future__ import annotations

import torch

from ._common import _DISABLE, check, contiguous, dtype_code, lib, ptr, stream


def polynorm_reference(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor, eps: float) -> torch.Tensor:
    """Torch composition of ``mlp.py:108-116`` (powers in fp32, result in x.dtype)."""
    xf = x.float()
    w = weight.float().reshape(-1)
    b = bias.float().reshape(-1)

    def _rms(z):
        return z * torch.rsqrt(torch.mean(z * z, dim=-1, keepdim=True) + eps)

    x2 = xf * xf
    x3 = x2 * xf
    return (w[0] * _rms(x3) + w[1] * _rms(x2) + w[2] * _rms(xf) + b[0]).to(x.dtype)


def polynorm(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    """Fused PolyNorm over the last axis: `x` (..., D), `weight` (3,), `bias` (1,)."""
    if _DISABLE:
        return polynorm_reference(x, weight, bias, eps)
    *lead, D = x.shape
    rows = x.numel() // D if D else 0
    if rows == 0:
        return torch.zeros_like(x)
    xc = contiguous(x)
    w = contiguous(weight.to(device=x.device, dtype=x.dtype).reshape(-1))
    b = contiguous(bias.to(device=x.device, dtype=x.dtype).reshape(-1))
    y = torch.empty_like(xc)
    check(lib.motif_polynorm(dtype_code(x), ptr(xc), ptr(w), ptr(b), float(eps), rows, D, ptr(y),
                             stream(x.device)), "polynorm")
    return y


def polynorm_mul(gate: torch.Tensor, up: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor,
                 eps: float = 1e-6) -> torch.Tensor:
    """``polynorm(gate) * up`` in one pass (the MotifMLP activation, ``model.py:267-268``)."""
    if _DISABLE:
        return polynorm_reference(gate, weight, bias, eps) * up
    assert gate.shape == up.shape, "gate and up must have the same shape"
    *lead, D = gate.shape
    rows = gate.numel() // D if D else 0
    if rows == 0:
        return torch.zeros_like(gate)
    g = contiguous(gate)
    u = contiguous(up)
    w = contiguous(weight.to(device=gate.device, dtype=gate.dtype).reshape(-1))
    b = contiguous(bias.to(device=gate.device, dtype=gate.dtype).reshape(-1))
    y = torch.empty_like(g)
    check(lib.motif_polynorm_mul(dtype_code(g), ptr(g), ptr(u), D, ptr(w), ptr(b), float(eps), rows, D,
                                 ptr(y), stream(gate.device)), "polynorm_mul")
    return y


def _dequant_probe(data: torch.Tensor, scales: torch.Tensor, biases: torch.Tensor,
                   group_size: int = 64, bits: int = 4) -> torch.Tensor:
    """Dequantize an MLX affine triple; output dtype = scales.dtype, last axis D."""
    *lead, n_uint = data.shape
    D = n_uint * (32 // bits)
    assert D % 32 == 0 and D % group_size == 0
    rows = data.numel() // n_uint if n_uint else 0
    y = torch.empty((*lead, D), dtype=scales.dtype, device=data.device)
    if rows == 0:
        return y
    d = contiguous(data)
    s = contiguous(scales)
    b = contiguous(biases)
    check(lib.motif_dequantize(dtype_code(s), bits, group_size, ptr(d), ptr(s), ptr(b), rows, D, ptr(y),
                               stream(data.device)), "dequantize")
    return y
