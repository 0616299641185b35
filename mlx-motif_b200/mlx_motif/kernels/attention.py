"""Shared-QK dual-V decode attention: ``sdpa_dual_v`` and ``sdpa_dual_v_q4``.

Operator surface of ``src/mlx_motif/kernels/attention.py``: ``sdpa_dual_v``
(190-260), ``sdpa_dual_v_q4`` (510-645) and their references (181-187,
473-507). Same shapes, runtime ``kv_len`` over a full-capacity buffer, and the
same shape contract and assertion messages. ``kv_len`` may also be a
1-element int32 CUDA tensor (read on the device, so the call can sit in a
captured CUDA graph).

The kernels (``motif_sdpa_dual_v`` / ``motif_sdpa_dual_v_q``) are split-KV:
one CTA per (batch, kv head, KV chunk) serving all GQA heads of that kv head,
partials merged by a second kernel.
"""

from __future__ import annotations

import torch

from ._common import _DISABLE, check, contiguous, dtype_code, kv_len_args, lib, ptr, stream, workspace

_MAX_SPLITS = 64


def _sdpa_f32(q, k, v, scale):
    s = torch.matmul(q.float(), k.float().transpose(-1, -2)) * scale
    if s.shape[-1] == 0:
        return torch.zeros(q.shape[:-1] + (v.shape[-1],), device=q.device)
    return torch.matmul(torch.softmax(s, dim=-1), v.float())


def sdpa_dual_v_reference(q, k, v1, v2, scale):
    """cat(SDPA(q,k,v1), SDPA(q,k,v2), axis=-1) as a torch composition (``attention.py:181-187``)."""
    return torch.cat([_sdpa_f32(q, k, v1, scale), _sdpa_f32(q, k, v2, scale)], dim=-1).to(q.dtype)


def sdpa_dual_v(q: torch.Tensor, k: torch.Tensor, v1: torch.Tensor, v2: torch.Tensor, scale: float,
                kv_len=None) -> torch.Tensor:
    """Shared-QK, dual-V SDPA with native GQA broadcast.

    q (B, H_q, 1, D); k, v1, v2 (B, H_kv, KV_cap, D). Each H_q/H_kv consecutive
    Q heads share one (K, V*) head. Returns (B, H_q, 1, 2·D) =
    cat([SDPA(q,k,v1), SDPA(q,k,v2)], axis=-1); rows >= kv_len are never read.
    """
    if kv_len is None:
        kv_len = k.shape[2]
    if _DISABLE:
        n = int(kv_len.item()) if isinstance(kv_len, torch.Tensor) else int(kv_len)
        k, v1, v2 = k[..., :n, :], v1[..., :n, :], v2[..., :n, :]
        gqa = q.shape[1] // k.shape[1]
        if gqa > 1:
            k, v1, v2 = (t.repeat_interleave(gqa, dim=1) for t in (k, v1, v2))
        return sdpa_dual_v_reference(q, k, v1, v2, scale)

    B, H_q, S_q, D = q.shape
    _, H_kv, KV_cap, _ = k.shape
    assert S_q == 1, "sdpa_dual_v is decode-only"
    assert D % 32 == 0, f"D={D} must be a multiple of 32"
    assert H_q % H_kv == 0, f"H_q={H_q} must be a multiple of H_kv={H_kv}"
    assert v1.shape == v2.shape == (B, H_kv, KV_cap, D), "v1,v2 must match (B, H_kv, KV_cap, D)"
    assert k.shape[-1] == D, "K head_dim must match Q"
    n_host, n_dev = kv_len_args(kv_len, KV_cap)
    if n_dev is None:
        assert 0 <= n_host <= KV_cap, f"kv_len={n_host} must be in [0, {KV_cap}]"
    qc, kc, v1c, v2c = (contiguous(t) for t in (q, k, v1.to(q.dtype), v2.to(q.dtype)))
    y = torch.empty((B, H_q, 1, 2 * D), dtype=q.dtype, device=q.device)
    ws_bytes = lib.motif_sdpa_dual_v_workspace_bytes(B, H_q, D, _MAX_SPLITS)
    ws = workspace(ws_bytes, q.device)
    check(lib.motif_sdpa_dual_v(dtype_code(q), ptr(qc), ptr(kc), ptr(v1c), ptr(v2c), float(scale), B, H_q,
                                H_kv, KV_cap, D, n_host, n_dev, ptr(y), ptr(ws), ws_bytes, stream(q.device)),
          "sdpa_dual_v")
    return y


def _dequantize_triple(t, group_size, bits, dtype):
    from .mlp import _dequant_probe

    return _dequant_probe(t[0], t[1], t[2], group_size=group_size, bits=bits).to(dtype)


def sdpa_dual_v_q4_reference(q, k_q, v1_q, v2_q, scale, group_size: int = 64, bits: int = 4, kv_len=None):
    """Dequantize K, V1, V2 then run the dual-V reference (``attention.py:473-507``)."""
    if kv_len is not None:
        n = int(kv_len.item()) if isinstance(kv_len, torch.Tensor) else int(kv_len)
        k_q, v1_q, v2_q = (tuple(x[..., :n, :] for x in t) for t in (k_q, v1_q, v2_q))
    k, v1, v2 = (_dequantize_triple(t, group_size, bits, q.dtype) for t in (k_q, v1_q, v2_q))
    gqa = q.shape[1] // k.shape[1]
    if gqa > 1:
        k, v1, v2 = (t.repeat_interleave(gqa, dim=1) for t in (k, v1, v2))
    return sdpa_dual_v_reference(q, k, v1, v2, scale)


def sdpa_dual_v_q4(q: torch.Tensor, k_q: tuple, v1_q: tuple, v2_q: tuple, scale: float, group_size: int = 64,
                   bits: int = 4, kv_len=None) -> torch.Tensor:
    """Quantized-input shared-QK, dual-V SDPA decode kernel.

    k_q, v1_q, v2_q: ``(data uint32, scales, biases)`` triples of (B, H_kv,
    KV_cap, D) tensors in the MLX affine layout. Returns (B, H_q, 1, 2·D).
    """
    if _DISABLE:
        return sdpa_dual_v_q4_reference(q, k_q, v1_q, v2_q, scale, group_size, bits, kv_len)
    k_data, k_scales, k_biases = k_q
    v1_data, v1_scales, v1_biases = v1_q
    v2_data, v2_scales, v2_biases = v2_q
    B, H_q, S_q, D = q.shape
    _, H_kv, KV_cap, n_uint = k_data.shape
    if kv_len is None:
        kv_len = KV_cap
    el_per_int = 32 // bits
    assert n_uint * el_per_int == D, (
        f"k_data last axis = {n_uint} ⇒ packed D = {n_uint * el_per_int}, expected {D}"
    )
    assert S_q == 1, "sdpa_dual_v_q4 is decode-only"
    assert D % 32 == 0
    assert D % group_size == 0
    assert H_q % H_kv == 0
    assert bits in (4, 8)
    n_host, n_dev = kv_len_args(kv_len, KV_cap)
    if n_dev is None:
        assert 0 <= n_host <= KV_cap, f"kv_len={n_host} must be in [0, {KV_cap}]"
    # The C ABI enforces the packed lane->word->group contract of attention.py:565-608
    # ((32/bits) % (D/32) == 0 and group_size % (D/32) == 0) and raises AssertionError.
    parts = [contiguous(t) for t in (q, k_data, k_scales, k_biases, v1_data, v1_scales, v1_biases, v2_data,
                                     v2_scales, v2_biases)]
    y = torch.empty((B, H_q, 1, 2 * D), dtype=q.dtype, device=q.device)
    ws_bytes = lib.motif_sdpa_dual_v_workspace_bytes(B, H_q, D, _MAX_SPLITS)
    ws = workspace(ws_bytes, q.device)
    check(lib.motif_sdpa_dual_v_q(dtype_code(q), bits, group_size, *(ptr(t) for t in parts), float(scale), B, H_q,
                                  H_kv, KV_cap, D, n_host, n_dev, ptr(y), ptr(ws), ws_bytes, stream(q.device)),
          "sdpa_dual_v_q4")
    return y
