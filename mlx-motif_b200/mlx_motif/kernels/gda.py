"""GDA post-attention reduction: ``gda_post_split`` and ``gda_post``.

Operator surface of ``src/mlx_motif/kernels/gda.py``: ``gda_post_split``
(223-282), ``gda_post`` (285-341) and their references (207-220, 108-124).
``lambda_full`` may hold the reference's single per-layer λ or, as an
extension, one λ per noise group or per origin head.
"""

from __future__ import annotations

import torch

from ._common import _DISABLE, as_f32_device, check, contiguous, dtype_code, lib, ptr, stream


def _lam_per_head(lambda_full, q_origin: int, gr: int, device) -> torch.Tensor:
    lam = as_f32_device(lambda_full, device)
    if lam.numel() == 1:
        return lam.expand(q_origin)
    if lam.numel() == q_origin // gr:
        return lam.repeat_interleave(gr)
    return lam


def gda_post_split_reference(attn_o, attn_n, subln_weight, lambda_full, lambda_init, gr, eps):
    """Torch composition of ``gda.py:207-220`` (fp32 math, result in attn_o.dtype)."""
    o = attn_o.float()
    n = attn_n.float().repeat_interleave(gr, dim=1)
    lam = _lam_per_head(lambda_full, o.shape[1], gr, o.device).reshape(1, -1, 1, 1)
    diff = o - lam * n
    rms_inv = torch.rsqrt(torch.mean(diff * diff, dim=-1, keepdim=True) + eps)
    return (diff * rms_inv * subln_weight.float() * (1.0 - lambda_init)).to(attn_o.dtype)


def gda_post_reference(merged, subln_weight, lambda_full, lambda_init, q_groups, gr, eps):
    """Torch composition of ``gda.py:108-124``."""
    q_origin = q_groups * gr
    return gda_post_split_reference(merged[:, :q_origin], merged[:, q_origin:], subln_weight, lambda_full,
                                    lambda_init, gr, eps)


def gda_post_split(attn_o: torch.Tensor, attn_n: torch.Tensor, subln_weight: torch.Tensor, lambda_full,
                   lambda_init: float, gr: int, eps: float = 1e-5) -> torch.Tensor:
    """(o − λ·n)·rsqrt(mean d² + eps)·w·(1 − λ_init) on split inputs.

    attn_o (B, q_origin, S, 2d), attn_n (B, q_groups, S, 2d) -> (B, q_origin, S, 2d).
    """
    if _DISABLE:
        return gda_post_split_reference(attn_o, attn_n, subln_weight, lambda_full, lambda_init, gr, eps)
    B, q_origin, S, channels = attn_o.shape
    _, q_groups, _, _ = attn_n.shape
    assert q_origin == q_groups * gr, f"q_origin={q_origin} != q_groups({q_groups}) * gr({gr})"
    o = contiguous(attn_o)
    n = contiguous(attn_n.to(attn_o.dtype))
    w = contiguous(subln_weight.to(device=o.device, dtype=o.dtype).reshape(-1))
    lam = as_f32_device(lambda_full, o.device)
    y = torch.empty_like(o)
    check(lib.motif_gda_post_split(dtype_code(o), ptr(o), ptr(n), ptr(w), ptr(lam), lam.numel(),
                                   float(lambda_init), B, q_groups, gr, S, channels, float(eps), ptr(y),
                                   stream(o.device)), "gda_post_split")
    return y


def gda_post(merged: torch.Tensor, subln_weight: torch.Tensor, lambda_full, lambda_init: float, q_groups: int,
             gr: int, eps: float = 1e-5) -> torch.Tensor:
    """The same reduction on a concatenated (B, q_origin + q_groups, S, 2d) input."""
    if _DISABLE:
        return gda_post_reference(merged, subln_weight, lambda_full, lambda_init, q_groups, gr, eps)
    B, q_heads, S, channels = merged.shape
    q_origin = q_groups * gr
    assert q_heads == q_origin + q_groups, f"q_heads={q_heads} expected {q_origin}+{q_groups}"
    m = contiguous(merged)
    w = contiguous(subln_weight.to(device=m.device, dtype=m.dtype).reshape(-1))
    lam = as_f32_device(lambda_full, m.device)
    y = torch.empty((B, q_origin, S, channels), dtype=m.dtype, device=m.device)
    check(lib.motif_gda_post(dtype_code(m), ptr(m), ptr(w), ptr(lam), lam.numel(), float(lambda_init), B,
                             q_groups, gr, S, channels, float(eps), ptr(y), stream(m.device)), "gda_post")
    return y
