"""Shared helpers for the operator modules: the disable flag, scalar/λ arrays, workspaces.

Mirrors ``src/mlx_motif/kernels/_common.py``: ``_DISABLE`` is read once at
import from ``MLX_MOTIF_DISABLE_KERNELS`` (correctness-only mode that routes
each op to its ``*_reference`` twin, written here as a torch composition on the
inputs' device). The default path is always the CUDA library.
"""

from __future__ import annotations

import torch

from .._native import _DISABLE, check, contiguous, dtype_code, lib, ptr, stream  # noqa: F401


def as_f32_device(value, device) -> torch.Tensor:
    """λ / scalar inputs as a contiguous fp32 device vector (the kernels read fp32)."""
    if isinstance(value, torch.Tensor):
        return contiguous(value.to(device=device, dtype=torch.float32).reshape(-1))
    return torch.tensor([float(v) for v in (value if isinstance(value, (list, tuple)) else [value])],
                        dtype=torch.float32, device=device)


def workspace(nbytes: int, device) -> torch.Tensor:
    """Scratch memory from torch's caching allocator (stream-ordered reuse)."""
    return torch.empty(max(int(nbytes), 16), dtype=torch.uint8, device=device)


def kv_len_args(kv_len, cap: int):
    """(host kv_len, device pointer) for an int or a 1-element int32 CUDA tensor."""
    if isinstance(kv_len, torch.Tensor):
        if kv_len.dtype != torch.int32 or not kv_len.is_cuda or kv_len.numel() != 1:
            raise TypeError("a device kv_len must be a 1-element int32 CUDA tensor")
        return 0, kv_len.data_ptr()
    kv_len = int(cap if kv_len is None else kv_len)
    return kv_len, None
