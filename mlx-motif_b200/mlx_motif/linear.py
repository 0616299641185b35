"""Affine-quantized linear (the ``nn.QuantizedLinear`` / ``mx.quantized_matmul`` of the reference).

Weights keep MLX's layout — ``weight`` (N, K·bits/32) uint32, ``scales`` and
``biases`` (N, K/group_size) — so a fused qkv weight is the row concatenation
``fuse_qkv`` builds (``model.py:1017-1079``). ``y = x · dequant(W)ᵀ`` runs the
``motif_quantized_linear`` kernel: an HBM-streaming GEMV for decode rows.
"""

from __future__ import annotations

import torch

from ._native import check, contiguous, dtype_code, lib, ptr, stream


def quantized_matmul(x: torch.Tensor, w: torch.Tensor, scales: torch.Tensor, biases: torch.Tensor,
                     transpose: bool = True, group_size: int = 64, bits: int = 4,
                     out: torch.Tensor | None = None, workspace: torch.Tensor | None = None) -> torch.Tensor:
    """x (…, K) · dequant(w)ᵀ -> (…, N)."""
    if not transpose:
        raise NotImplementedError("only the transposed (nn.QuantizedLinear) form is implemented")
    N = w.shape[0]
    K = w.shape[1] * (32 // bits)
    assert x.shape[-1] == K, f"x last axis {x.shape[-1]} != in_dim {K}"
    lead = x.shape[:-1]
    M = x.numel() // K if K else 0
    xc = contiguous(x)
    y = out if out is not None else torch.empty((*lead, N), dtype=x.dtype, device=x.device)
    ws_bytes = lib.motif_quantized_linear_workspace_bytes(max(M, 1), N, K, bits, group_size)
    if workspace is None or workspace.numel() < ws_bytes:
        # zero-filled: the split-K tile counters must start at zero (the kernel re-zeroes them)
        workspace = torch.zeros(max(ws_bytes, 16), dtype=torch.uint8, device=x.device)
    check(lib.motif_quantized_linear(dtype_code(x), bits, group_size, ptr(xc), M, K, ptr(w), ptr(scales),
                                     ptr(biases), N, ptr(y), ptr(workspace), ws_bytes, stream(x.device)),
          "quantized_linear")
    return y


class QuantizedLinear:
    """Holder of one quantized weight (weight, scales, biases) with MLX's attribute names."""

    def __init__(self, weight: torch.Tensor, scales: torch.Tensor, biases: torch.Tensor, group_size: int = 64,
                 bits: int = 4):
        self.weight = contiguous(weight)
        self.scales = contiguous(scales)
        self.biases = contiguous(biases)
        self.group_size = group_size
        self.bits = bits

    @property
    def in_dim(self) -> int:
        return self.weight.shape[1] * (32 // self.bits)

    @property
    def out_dim(self) -> int:
        return self.weight.shape[0]

    def nbytes(self) -> int:
        return sum(t.numel() * t.element_size() for t in (self.weight, self.scales, self.biases))

    def __call__(self, x: torch.Tensor, out: torch.Tensor | None = None,
                 workspace: torch.Tensor | None = None) -> torch.Tensor:
        return quantized_matmul(x, self.weight, self.scales, self.biases, True, self.group_size, self.bits,
                                out=out, workspace=workspace)
