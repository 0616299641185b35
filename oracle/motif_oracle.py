"""CPU restatement of the reference's decode hot path (TEST INFRASTRUCTURE ONLY).

Every function below restates one reference function (numpy, float64 inside an
op, rounded to the reference's storage dtype at the op boundary) and cites the
file:line of the reference it follows. Paths are relative to the reference
project root (junhoyeo/mlx-motif).

Nothing in the product package imports this module: it is the checker used by
``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline legs of
``bench.py``.

Third-party arithmetic the reference calls but does not vendor (MLX 0.31.2 /
mlx-lm 0.29.1, pinned at ``uv.lock:461-462,491-492``) is restated from its
published definition:
  * ``mx.quantize`` / ``mx.dequantize``: affine group quantization
    (``quantize``/``dequantize`` below). Dequantize is pinned by the
    reference's bit-extract probe; quantize is parity UNPINNED against MLX.
  * ``mx.fast.scaled_dot_product_attention``: softmax(q k^T * scale) v.
  * ``mx.fast.rope`` with ``traditional=False``: rotate (x[i], x[i + D/2]).
  * ``mx.fast.rms_norm``: x * rsqrt(mean(x^2) + eps) * w.
  * ``mx.quantized_matmul``: y = sum_g s_g * sum_k x_k q_k + b_g * sum_k x_k.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np

__all__ = [
    "round_half_away",
    "polynorm_reference",
    "polynorm_mul_reference",
    "gda_post_split_reference",
    "gda_post_reference",
    "sdpa_dual_v_reference",
    "causal_gqa_sdpa",
    "grouped_prompt_attention_reference",
    "sdpa_dual_v_q4_reference",
    "dequantize",
    "quantize",
    "quantized_matmul",
    "rope_inv_freq",
    "rope",
    "rms_norm",
    "lambda_init_for_layer",
    "lambda_full",
    "origin_first_perm",
    "OracleGroupedKVCache",
    "OracleGroupedQuantizedKVCache",
    "OracleArgs",
    "make_synthetic_weights",
    "GroupedDecodeOracle",
    "shard_weights_tp",
    "vanilla_v_paired_to_slab_perm",
    "vanilla_v_slab_to_paired_perm",
    "OracleVanillaKVCache",
    "vanilla_attention_reference",
    "OracleVanillaArgs",
    "make_synthetic_weights_vanilla",
    "VanillaDecodeOracle",
]


def _f64(a) -> np.ndarray:
    return np.asarray(a).astype(np.float64)


def round_half_away(x: np.ndarray) -> np.ndarray:
    """Round half away from zero, exactly (the Metal/CUDA ``round`` rule).

    ``x - trunc(x)`` is exact in binary floating point, so no double rounding.
    """
    x = np.asarray(x)
    t = np.trunc(x)
    frac = x - t
    return t + np.where(np.abs(frac) >= 0.5, np.sign(x), 0).astype(x.dtype)


# --------------------------------------------------------------------------- #
# PolyNorm — src/mlx_motif/kernels/mlp.py:108-116 (reference), 21-93 (kernel)
# --------------------------------------------------------------------------- #


def polynorm_reference(x, weight, bias, eps: float = 1e-6) -> np.ndarray:
    """w0*rms(x^3) + w1*rms(x^2) + w2*rms(x) + b over the last axis.

    Follows ``kernels/mlp.py:108-116`` with the powers formed in float64.
    The reference forms x^6 in the input dtype (fp16 overflows for
    |x| > ~6.3); its Metal kernel (``mlp.py:30-39``) and the B200 kernel
    accumulate in fp32, which is what this restatement models.
    """
    xf = _f64(x)
    w = _f64(weight).reshape(-1)
    b = _f64(bias).reshape(-1)

    def _rms(z):
        return z / np.sqrt(np.mean(z * z, axis=-1, keepdims=True) + eps)

    x2 = xf * xf
    x3 = x2 * xf
    return w[0] * _rms(x3) + w[1] * _rms(x2) + w[2] * _rms(xf) + b[0]


def polynorm_mul_reference(gate, up, weight, bias, eps: float = 1e-6, out_dtype=np.float16):
    """``act_fn(gate_proj(x)) * up_proj(x)`` of ``model.py:267-268``.

    The reference materialises polynorm(gate) in the activation dtype, then
    multiplies by ``up`` in that dtype; both roundings are modelled.
    """
    act = polynorm_reference(gate, weight, bias, eps).astype(out_dtype)
    return (_f64(act) * _f64(up)).astype(out_dtype)


# --------------------------------------------------------------------------- #
# GDA post reduction — src/mlx_motif/kernels/gda.py:108-124, 207-220
# --------------------------------------------------------------------------- #


def _lambda_per_origin_head(lambda_full, q_origin: int, gr: int) -> np.ndarray:
    """Broadcast λ to one value per origin head.

    The reference λ is one per-layer scalar (``model.py:462-470``; the kernel
    reads ``lambda_full[0]``, ``gda.py:152``). A vector of length q_groups
    (one per noise group) or q_origin (one per origin head) is accepted as an
    extension for per-head λ.
    """
    lam = _f64(lambda_full).reshape(-1)
    if lam.size == 1:
        return np.full((q_origin,), lam[0])
    if lam.size == q_origin // gr:
        return np.repeat(lam, gr)
    if lam.size == q_origin:
        return lam
    raise ValueError(f"lambda_full must have 1, {q_origin // gr} or {q_origin} values; got {lam.size}")


def gda_post_split_reference(attn_o, attn_n, subln_weight, lambda_full, lambda_init, gr, eps=1e-5):
    """(o - λ·repeat(n, gr)) * rsqrt(mean(d^2) + eps) * w * (1 - λ_init).

    ``gda.py:207-220``: attn_o (B, q_origin, S, 2d), attn_n (B, q_groups, S, 2d).
    """
    o = _f64(attn_o)
    n = np.repeat(_f64(attn_n), gr, axis=1)
    lam = _lambda_per_origin_head(lambda_full, o.shape[1], gr)[None, :, None, None]
    diff = o - lam * n
    rms_inv = 1.0 / np.sqrt(np.mean(diff * diff, axis=-1, keepdims=True) + eps)
    return diff * rms_inv * _f64(subln_weight) * (1.0 - lambda_init)


def gda_post_reference(merged, subln_weight, lambda_full, lambda_init, q_groups, gr, eps=1e-5):
    """``gda.py:108-124``: the same reduction on a concatenated (origin | noise) input."""
    q_origin = q_groups * gr
    m = np.asarray(merged)
    return gda_post_split_reference(
        m[:, :q_origin], m[:, q_origin:], subln_weight, lambda_full, lambda_init, gr, eps
    )


# --------------------------------------------------------------------------- #
# Dual-V SDPA — src/mlx_motif/kernels/attention.py:181-187, 217-229
# --------------------------------------------------------------------------- #


def _sdpa(q, k, v, scale):
    """softmax(q k^T * scale) v in float64 (q (B,H,S,D), k/v (B,H,N,D))."""
    s = np.einsum("bhsd,bhnd->bhsn", q, k) * scale
    if s.shape[-1] == 0:
        return np.zeros(q.shape[:-1] + (v.shape[-1],))
    s = s - s.max(axis=-1, keepdims=True)
    p = np.exp(s)
    p = p / p.sum(axis=-1, keepdims=True)
    return np.einsum("bhsn,bhnd->bhsd", p, v)


def _sdpa_causal(q, k, v, scale, offset):
    """``mx.fast.scaled_dot_product_attention`` with mlx-lm's causal mask for a prompt block
    (``create_causal_mask``: query i sits at position offset + i and sees keys 0 .. offset + i),
    float64; q (B,H,S,D), k/v (B,H,N,D)."""
    S, N = q.shape[2], k.shape[2]
    s = np.einsum("bhsd,bhnd->bhsn", q, k) * scale
    mask = np.arange(N)[None, :] <= (offset + np.arange(S))[:, None]
    s = np.where(mask[None, None], s, -np.inf)
    s = s - s.max(axis=-1, keepdims=True)
    p = np.exp(s)
    p = p / p.sum(axis=-1, keepdims=True)
    return np.einsum("bhsn,bhnd->bhsd", p, v)


def causal_gqa_sdpa(q, k, v, scale, offset):
    """Native-GQA causal SDPA (q head i reads kv head i // (Hq // Hkv)), float64."""
    qf, kf, vf = _f64(q), _f64(k), _f64(v)
    rep = qf.shape[1] // kf.shape[1]
    if rep > 1:
        kf = np.repeat(kf, rep, axis=1)
        vf = np.repeat(vf, rep, axis=1)
    return _sdpa_causal(qf, kf, vf, scale, offset)


def grouped_prompt_attention_reference(q_origin, q_noise, k1, k2, v1, v2, scale, offset):
    """The prompt branch of ``_forward_grouped`` (``model.py:769-807``): four per-slab causal
    SDPAs, each rounded to fp16 (MLX materialises fp16 arrays), concatenated on the channel
    axis: attn_origin = [SDPA(q1,k1,v1) | SDPA(q1,k1,v2)], attn_noise the same with (q2, k2).
    q_* (B, H, S, D); k/v (B, G, N, D) holding the cache rows [0, offset + S)."""
    f16 = np.float16

    def pair(q, k):
        return np.concatenate([causal_gqa_sdpa(q, k, v, scale, offset).astype(f16) for v in (v1, v2)], axis=-1)

    return pair(q_origin, k1), pair(q_noise, k2)


def sdpa_dual_v_reference(q, k, v1, v2, scale, kv_len=None):
    """cat[SDPA(q,k,v1), SDPA(q,k,v2)] with GQA repeat and a live-length slice.

    ``attention.py:217-229`` (slice to kv_len, ``mx.repeat`` over heads) then
    ``attention.py:181-187`` (two SDPAs, concat on the channel axis).
    """
    if kv_len is None:
        kv_len = np.asarray(k).shape[2]
    qf = _f64(q)
    kf = _f64(np.asarray(k)[..., :kv_len, :])
    v1f = _f64(np.asarray(v1)[..., :kv_len, :])
    v2f = _f64(np.asarray(v2)[..., :kv_len, :])
    gqa = qf.shape[1] // kf.shape[1]
    if gqa > 1:
        kf = np.repeat(kf, gqa, axis=1)
        v1f = np.repeat(v1f, gqa, axis=1)
        v2f = np.repeat(v2f, gqa, axis=1)
    a1 = _sdpa(qf, kf, v1f, scale)
    a2 = _sdpa(qf, kf, v2f, scale)
    return np.concatenate([a1, a2], axis=-1)


# --------------------------------------------------------------------------- #
# Affine group quantization (MLX mx.quantize / mx.dequantize)
# --------------------------------------------------------------------------- #


def dequantize(data, scales, biases, group_size: int = 64, bits: int = 4, out_dtype=None):
    """``scale[g] * ((data[ch // EL] >> (ch % EL)·bits) & mask) + bias[g]``.

    Follows the reference's bit-extract kernel ``kernels/mlp.py:176-198``:
    little-endian packing, EL = 32/bits values per uint32, no zero-point,
    arithmetic in fp32 and one rounding to the output dtype (the scales'
    dtype by default, as ``mlp.py:224`` states).
    """
    data = np.asarray(data, dtype=np.uint32)
    el = 32 // bits
    mask = np.uint32((1 << bits) - 1)
    D = data.shape[-1] * el
    shifts = (np.arange(el, dtype=np.uint32) * np.uint32(bits))
    raw = (data[..., :, None] >> shifts) & mask
    raw = raw.reshape(*data.shape[:-1], D).astype(np.float32)
    s = np.repeat(np.asarray(scales).astype(np.float32), group_size, axis=-1)
    b = np.repeat(np.asarray(biases).astype(np.float32), group_size, axis=-1)
    out = s * raw + b
    dt = np.asarray(scales).dtype if out_dtype is None else out_dtype
    return out.astype(dt)


def quantize(w, group_size: int = 64, bits: int = 4):
    """Affine group quantization of the last axis -> (data uint32, scales, biases).

    Restates MLX's published affine quantizer (MLX 0.31.2, not vendored in the
    reference; call sites ``cache.py:399-402,498``). All arithmetic is IEEE
    fp32 on the fp32-widened input; parity against MLX is UNPINNED.

    Per group of ``group_size`` values:
      n_bins = 2^bits - 1
      scale  = max((w_max - w_min) / n_bins, 1e-7)
      if |w_min| > |w_max|: edge = w_min            else: edge = w_max, scale = -scale
      q0     = round(edge / scale)                    (round half away from zero)
      if q0 == 0: bias = 0                            else: scale = edge / q0, bias = edge
      code   = clamp(round((w - bias) / scale), 0, n_bins)
    Scales and biases are stored in the input dtype (round to nearest even);
    codes pack little-endian, 32/bits per uint32.
    """
    w = np.asarray(w)
    out_dtype = w.dtype
    D = w.shape[-1]
    if D % group_size != 0:
        raise ValueError(f"last axis {D} is not a multiple of group_size {group_size}")
    if bits not in (2, 3, 4, 6, 8) or (32 % bits) != 0:
        raise ValueError(f"bits={bits} not supported (need 32 % bits == 0)")
    n_bins = np.float32((1 << bits) - 1)
    eps = np.float32(1e-7)
    wf = w.astype(np.float32).reshape(*w.shape[:-1], D // group_size, group_size)
    w_max = wf.max(axis=-1)
    w_min = wf.min(axis=-1)
    with np.errstate(divide="ignore", invalid="ignore"):
        scale = np.maximum((w_max - w_min) / n_bins, eps).astype(np.float32)
        side = np.abs(w_min) > np.abs(w_max)
        scale = np.where(side, scale, -scale).astype(np.float32)
        edge = np.where(side, w_min, w_max).astype(np.float32)
        q0 = round_half_away((edge / scale).astype(np.float32))
        at_zero = q0 == 0
        scale = np.where(at_zero, scale, (edge / np.where(at_zero, 1, q0)).astype(np.float32)).astype(np.float32)
        bias = np.where(at_zero, np.float32(0), edge).astype(np.float32)
        t = ((wf - bias[..., None]) / scale[..., None]).astype(np.float32)
    codes = np.clip(round_half_away(t), 0, n_bins).astype(np.uint32)
    el = 32 // bits
    codes = codes.reshape(*w.shape[:-1], D // el, el)
    shifts = np.arange(el, dtype=np.uint32) * np.uint32(bits)
    data = np.bitwise_or.reduce(codes << shifts, axis=-1).astype(np.uint32)
    return data, scale.astype(out_dtype), bias.astype(out_dtype)


def sdpa_dual_v_q4_reference(q, k_q, v1_q, v2_q, scale, group_size=64, bits=4, kv_len=None):
    """Dequantize K, V1, V2 then run the dual-V reference (``attention.py:473-507``)."""
    if kv_len is not None:
        k_q = tuple(np.asarray(x)[..., :kv_len, :] for x in k_q)
        v1_q = tuple(np.asarray(x)[..., :kv_len, :] for x in v1_q)
        v2_q = tuple(np.asarray(x)[..., :kv_len, :] for x in v2_q)
    k = dequantize(*k_q, group_size=group_size, bits=bits)
    v1 = dequantize(*v1_q, group_size=group_size, bits=bits)
    v2 = dequantize(*v2_q, group_size=group_size, bits=bits)
    return sdpa_dual_v_reference(q, k, v1, v2, scale)


def quantized_matmul(x, data, scales, biases, group_size: int = 64, bits: int = 4):
    """``x @ dequant(W)^T`` with W stored (N, K/EL) uint32 + (N, K/g) scales/biases.

    The layout is the one ``nn.QuantizedLinear`` holds (``model.py:1047``:
    ``in_dim = weight.shape[1] * (32 // bits)``; rows concatenate on axis 0 in
    ``fuse_qkv``, ``model.py:1069-1071``). Arithmetic restates MLX's affine
    quantized matmul: per group g, ``s_g * sum_k x_k q_k + b_g * sum_k x_k``,
    here in float64.
    """
    x = _f64(x)
    data = np.asarray(data, dtype=np.uint32)
    N = data.shape[0]
    el = 32 // bits
    K = data.shape[1] * el
    mask = np.uint32((1 << bits) - 1)
    shifts = np.arange(el, dtype=np.uint32) * np.uint32(bits)
    q = ((data[:, :, None] >> shifts) & mask).reshape(N, K).astype(np.float64)
    ng = K // group_size
    xg = x.reshape(*x.shape[:-1], ng, group_size)
    qg = q.reshape(N, ng, group_size)
    dots = np.einsum("...gk,ngk->...ng", xg, qg)
    xs = xg.sum(axis=-1)  # (..., ng)
    s = _f64(scales)
    b = _f64(biases)
    return np.einsum("...ng,ng->...n", dots, s) + np.einsum("...g,ng->...n", xs, b)


# --------------------------------------------------------------------------- #
# RoPE / RMSNorm / λ — mlx-lm initialize_rope (model.py:414-420), model.py:389,462-470
# --------------------------------------------------------------------------- #


def rope_inv_freq(dims: int, base: float = 10000.0) -> np.ndarray:
    """fp32 inverse frequencies 2^(-(i / (dims/2)) * log2(base)), i < dims/2, formed in
    float64 and rounded once to fp32 (mlx-lm's non-traditional RoPE frequencies)."""
    half = dims // 2
    return np.array([2.0 ** (-(i / half) * math.log2(base)) for i in range(half)], np.float64).astype(np.float32)


def rope(x, offset: int, base: float = 10000.0, inv_freq=None) -> np.ndarray:
    """Non-traditional RoPE (``traditional=False``, ``model.py:417``).

    x (B, H, S, D): pairs (x[i], x[i + D/2]) rotate by θ = (offset + s)·inv_freq[i]
    with θ formed in fp32 (as the device kernel forms it) and cos/sin in float64.
    """
    xf = _f64(x)
    D = xf.shape[-1]
    half = D // 2
    if inv_freq is None:
        inv_freq = rope_inv_freq(D, base)
    S = xf.shape[-2]
    pos = (np.arange(S, dtype=np.float32) + np.float32(offset)).astype(np.float32)
    theta = (pos[:, None] * inv_freq[None, :]).astype(np.float32).astype(np.float64)
    c, s = np.cos(theta), np.sin(theta)
    x1, x2 = xf[..., :half], xf[..., half:]
    return np.concatenate([x1 * c - x2 * s, x1 * s + x2 * c], axis=-1)


def rms_norm(x, weight, eps: float = 1e-6) -> np.ndarray:
    """``nn.RMSNorm``: x * rsqrt(mean(x^2) + eps) * w over the last axis."""
    xf = _f64(x)
    return xf / np.sqrt(np.mean(xf * xf, axis=-1, keepdims=True) + eps) * _f64(weight)


def lambda_init_for_layer(layer_idx: int) -> float:
    """``model.py:389``: λ_init = 0.8 − 0.6·exp(−0.3·(layer_idx − 1))."""
    return 0.8 - 0.6 * math.exp(-0.3 * (layer_idx - 1))


def lambda_full(lq1, lk1, lq2, lk2, lam_init: float) -> np.float32:
    """``model.py:462-470``: exp(Σ lq1·lk1) − exp(Σ lq2·lk2) + λ_init in fp32."""
    f = np.float32
    l1 = np.exp(f(np.sum(np.asarray(lq1, f) * np.asarray(lk1, f), dtype=f)))
    l2 = np.exp(f(np.sum(np.asarray(lq2, f) * np.asarray(lk2, f), dtype=f)))
    return f(l1 - l2 + f(lam_init))


def origin_first_perm(q_groups: int, gr: int, d: int) -> np.ndarray:
    """``model.py:994-1015``: row permutation from the HF head stripes
    [g0_o1..g0_o<gr>, g0_n, g1_o1, ..] to origin-first [all origin | all noise]."""
    heads = [g * (gr + 1) + p for g in range(q_groups) for p in range(gr)]
    heads += [g * (gr + 1) + gr for g in range(q_groups)]
    return np.concatenate([np.arange(h * d, (h + 1) * d) for h in heads]).astype(np.int64)


# --------------------------------------------------------------------------- #
# 4-slot KV caches — src/mlx_motif/cache.py:178-545
# --------------------------------------------------------------------------- #


class _OracleGroupedBase:
    """Offset / growth bookkeeping of ``MotifGroupedKVCacheBase`` (``cache.py:178-300``)."""

    step = 256

    def is_trimmable(self):
        return True

    def trim(self, n):  # cache.py:221-224
        n = min(self.offset, n)
        self.offset -= n
        return n

    @staticmethod
    def _assert_uniform_heads(k1, k2, v1, v2):  # cache.py:283-300
        h1 = k1.shape[1]
        if not (k2.shape[1] == v1.shape[1] == v2.shape[1] == h1):
            raise ValueError(
                "4-slot grouped KV cache requires k1/k2/v1/v2 to share a head count; "
                f"got k1={h1}, k2={k2.shape[1]}, v1={v1.shape[1]}, v2={v2.shape[1]}"
            )

    def _grow(self, B, H, S, D, dtype):  # cache.py:245-265
        prev = self.offset
        if self.k1 is None or (prev + S) > self._slot_capacity(self.k1):
            new_len = ((self.step + S - 1) // self.step) * self.step
            if self.k1 is not None:
                slots = [self.k1, self.k2, self.v1, self.v2]
                if prev % self.step != 0:
                    slots = [self._trim_slot(s, prev) for s in slots]
                fresh = self._init_storage(B, H, new_len, D, dtype)
                self.k1, self.k2, self.v1, self.v2 = (self._expand_slot(s, fresh) for s in slots)
            else:
                self.k1, self.k2, self.v1, self.v2 = (
                    self._init_storage(B, H, new_len, D, dtype) for _ in range(4)
                )


class OracleGroupedKVCache(_OracleGroupedBase):
    """fp16 4-slot cache (``cache.py:303-404``)."""

    def __init__(self):
        self.k1 = self.k2 = self.v1 = self.v2 = None
        self.offset = 0

    def _slot_capacity(self, slot):
        return slot.shape[2]

    def _init_storage(self, B, H, n, D, dtype):
        return np.zeros((B, H, n, D), dtype)

    def _trim_slot(self, slot, prev):
        return slot[..., :prev, :]

    def _expand_slot(self, slot, fresh):
        return np.concatenate([slot, fresh], axis=2)

    def update_and_fetch_4(self, k1, k2, v1, v2):  # cache.py:337-360
        self._assert_uniform_heads(k1, k2, v1, v2)
        B, H, S, D = k1.shape
        prev = self.offset
        self._grow(B, H, S, D, k1.dtype)
        for slot, new in ((self.k1, k1), (self.k2, k2), (self.v1, v1), (self.v2, v2)):
            slot[..., prev : prev + S, :] = new
        self.offset += S
        return self.k1, self.k2, self.v1, self.v2

    @property
    def state(self):  # cache.py:366-376
        if self.offset == 0 or self.k1 is None:
            return self.k1, self.k2, self.v1, self.v2
        o = self.offset
        return tuple(s[..., :o, :] for s in (self.k1, self.k2, self.v1, self.v2))


class OracleGroupedQuantizedKVCache(_OracleGroupedBase):
    """Quantized 4-slot cache (``cache.py:407-545``): one batched quantize per write."""

    def __init__(self, group_size: int = 64, bits: int = 8):
        self.k1 = self.k2 = self.v1 = self.v2 = None
        self.offset = 0
        self.group_size = group_size
        self.bits = bits

    def _slot_capacity(self, slot):
        return slot[0].shape[2]

    def _init_storage(self, B, H, n, D, dtype):  # cache.py:430-436
        el = 32 // self.bits
        return (
            np.zeros((B, H, n, D // el), np.uint32),
            np.zeros((B, H, n, D // self.group_size), dtype),
            np.zeros((B, H, n, D // self.group_size), dtype),
        )

    def _trim_slot(self, slot, prev):
        return tuple(x[..., :prev, :] for x in slot)

    def _expand_slot(self, slot, fresh):
        return tuple(np.concatenate([slot[i], fresh[i]], axis=-2) for i in range(3))

    def _update_4(self, k1, k2, v1, v2):  # cache.py:485-512
        self._assert_uniform_heads(k1, k2, v1, v2)
        B, H, S, D = k1.shape
        prev = self.offset
        self._grow(B, H, S, D, k1.dtype)
        fresh = np.concatenate([k1, k2, v1, v2], axis=1)
        qd, qs, qb = quantize(fresh, self.group_size, self.bits)
        for i, slot in enumerate((self.k1, self.k2, self.v1, self.v2)):
            h0, h1 = i * H, (i + 1) * H
            slot[0][..., prev : prev + S, :] = qd[:, h0:h1]
            slot[1][..., prev : prev + S, :] = qs[:, h0:h1]
            slot[2][..., prev : prev + S, :] = qb[:, h0:h1]
        self.offset += S

    def update_and_fetch_4_quantized(self, k1, k2, v1, v2):  # cache.py:467-483
        self._update_4(k1, k2, v1, v2)
        return self.k1, self.k2, self.v1, self.v2

    def update_and_fetch_4(self, k1, k2, v1, v2):  # cache.py:448-465
        self._update_4(k1, k2, v1, v2)
        o = self.offset

        def _deq(slot):
            return dequantize(*(x[..., :o, :] for x in slot), group_size=self.group_size, bits=self.bits)

        return _deq(self.k1), _deq(self.k2), _deq(self.v1), _deq(self.v2)


# --------------------------------------------------------------------------- #
# Grouped decoder (12.7B-class GDA) — model.py:563-837, 845-905
# --------------------------------------------------------------------------- #


@dataclass
class OracleArgs:
    """Shape of a grouped (GDA) Motif decoder; defaults are the 12.7B-class config."""

    hidden_size: int = 4096
    num_hidden_layers: int = 48
    intermediate_size: int = 14336
    num_noise_heads: int = 8  # q_groups
    grouped_ratio: int = 3  # origin heads per group
    kv_heads_per_slot: int = 8  # k1/k2/v1/v2 heads each (num_key_value_heads = 2x)
    head_dim: int = 128
    vocab_size: int = 219520
    rms_norm_eps: float = 1e-6
    attn_rms_norm_eps: float = 1e-5
    rope_theta: float = 10000.0
    group_size: int = 64
    bits: int = 4

    @property
    def q_origin(self):
        return self.num_noise_heads * self.grouped_ratio

    @property
    def q_heads(self):
        return self.num_noise_heads * (self.grouped_ratio + 1)

    @property
    def qkv_out(self):
        d = self.head_dim
        return self.q_heads * d + 2 * self.kv_heads_per_slot * d + 2 * self.kv_heads_per_slot * d


def _q_linear(rng, n_out, n_in, std, group_size, bits):
    w = (rng.standard_normal((n_out, n_in), dtype=np.float32) * std).astype(np.float16)
    return quantize(w, group_size, bits)


def make_synthetic_weights(args: OracleArgs, seed: int = 0, std: float = 0.02) -> dict:
    """Random-init weights (std 0.02) with every linear quantized by ``quantize``.

    Layout per layer (the reference's fused-QKV layout, ``model.py:1017-1079``):
      qkv  (q_heads*d + 2*Hkv*d + 2*Hkv*d, H/EL) with Q rows origin-first
      o    (H, q_origin*2d/EL), gate/up (I, H/EL), down (H, I/EL)
    Norm weights are 1 + N(0, 0.02) in fp16; λ parameters N(0, 0.1) in fp32.
    """
    rng = np.random.default_rng(seed)
    g, b = args.group_size, args.bits
    H, I, d = args.hidden_size, args.intermediate_size, args.head_dim
    f16 = np.float16

    def norm_w(n):
        return (1.0 + 0.02 * rng.standard_normal(n)).astype(f16)

    layers = []
    for li in range(args.num_hidden_layers):
        lam_init = lambda_init_for_layer(li)
        lp = [rng.standard_normal(d).astype(np.float32) * 0.1 for _ in range(4)]
        layers.append(
            dict(
                input_norm=norm_w(H),
                post_norm=norm_w(H),
                qkv=_q_linear(rng, args.qkv_out, H, std, g, b),
                o=_q_linear(rng, H, args.q_origin * 2 * d, std, g, b),
                gate=_q_linear(rng, I, H, std, g, b),
                up=_q_linear(rng, I, H, std, g, b),
                down=_q_linear(rng, H, I, std, g, b),
                subln=norm_w(2 * d),
                lambda_init=lam_init,
                lambda_full=np.array([lambda_full(*lp, lam_init)], np.float32),
                polynorm_w=np.array([1 / 3, 1 / 3, 1 / 3], f16),
                polynorm_b=np.zeros((1,), f16),
            )
        )
    return dict(
        embed=(rng.standard_normal((args.vocab_size, H), dtype=np.float32) * std).astype(f16),
        final_norm=norm_w(H),
        lm_head=_q_linear(rng, args.vocab_size, H, std, g, b),
        layers=layers,
    )


class GroupedDecodeOracle:
    """Batch-1 decode through the DUAL_V / QUANT_SDPA path of ``_forward_grouped``.

    One ``step(token)`` follows ``Model.__call__`` (``model.py:896-905``) ->
    ``MotifModel`` (858-879) -> ``MotifDecoderLayer`` (845-855) with
    ``_forward_grouped`` (563-837) on the fused, origin-first QKV and the
    4-slot cache, then ``MotifMLP`` (267-268). Every op output is rounded to
    fp16, the reference's activation dtype.
    """

    def __init__(self, args: OracleArgs, weights: dict, cache: str = "fp16"):
        self.args = args
        self.w = weights
        if cache == "fp16":
            self.caches = [OracleGroupedKVCache() for _ in range(args.num_hidden_layers)]
        elif cache in ("q4", "q8"):
            bits = 4 if cache == "q4" else 8
            self.caches = [
                OracleGroupedQuantizedKVCache(group_size=64, bits=bits)
                for _ in range(args.num_hidden_layers)
            ]
        else:
            raise ValueError(cache)
        self.cache_kind = cache
        self.inv_freq = rope_inv_freq(args.head_dim, args.rope_theta)

    def _lin(self, x, triple):
        a = self.args
        return quantized_matmul(x, *triple, group_size=a.group_size, bits=a.bits).astype(np.float16)

    def layer(self, li: int, h: np.ndarray) -> np.ndarray:
        a = self.args
        L = self.w["layers"][li]
        f16 = np.float16
        d, G, gr, Hk = a.head_dim, a.num_noise_heads, a.grouped_ratio, a.kv_heads_per_slot
        cache = self.caches[li]
        x = rms_norm(h, L["input_norm"], a.rms_norm_eps).astype(f16)
        qkv = self._lin(x, L["qkv"])  # (1, qkv_out)
        qd = a.q_heads * d
        kd = 2 * Hk * d
        q = qkv[..., :qd].reshape(1, 1, a.q_heads, d).transpose(0, 2, 1, 3)
        k = qkv[..., qd : qd + kd].reshape(1, 1, 2 * Hk, d).transpose(0, 2, 1, 3)
        v = qkv[..., qd + kd :].reshape(1, 1, 2 * Hk, d).transpose(0, 2, 1, 3)
        off = cache.offset
        q = rope(q, off, inv_freq=self.inv_freq).astype(f16)
        k = rope(k, off, inv_freq=self.inv_freq).astype(f16)
        k1, k2 = k[:, 0::2], k[:, 1::2]  # model.py:625-627 with k_ratio = 1
        v1, v2 = v[:, 0::2], v[:, 1::2]  # model.py:628-630
        q1, q2 = q[:, : G * gr], q[:, G * gr :]  # model.py:673-675
        scale = d ** -0.5
        if self.cache_kind == "fp16":
            K1, K2, V1, V2 = cache.update_and_fetch_4(k1, k2, v1, v2)
            n = cache.offset
            ao = sdpa_dual_v_reference(q1, K1, V1, V2, scale, n).astype(f16)
            an = sdpa_dual_v_reference(q2, K2, V1, V2, scale, n).astype(f16)
        else:
            K1, K2, V1, V2 = cache.update_and_fetch_4_quantized(k1, k2, v1, v2)
            n = cache.offset
            gs, bits = cache.group_size, cache.bits
            ao = sdpa_dual_v_q4_reference(q1, K1, V1, V2, scale, gs, bits, n).astype(f16)
            an = sdpa_dual_v_q4_reference(q2, K2, V1, V2, scale, gs, bits, n).astype(f16)
        out = gda_post_split_reference(
            ao, an, L["subln"], L["lambda_full"], L["lambda_init"], gr, a.attn_rms_norm_eps
        ).astype(f16)
        out = out.transpose(0, 2, 1, 3).reshape(1, -1)
        o = self._lin(out, L["o"])
        h = (h.astype(np.float32) + o.astype(np.float32)).astype(f16)
        x2 = rms_norm(h, L["post_norm"], a.rms_norm_eps).astype(f16)
        gt = self._lin(x2, L["gate"])
        up = self._lin(x2, L["up"])
        act = polynorm_mul_reference(gt, up, L["polynorm_w"], L["polynorm_b"], 1e-6)
        dn = self._lin(act, L["down"])
        return (h.astype(np.float32) + dn.astype(np.float32)).astype(f16)

    def step(self, token: int):
        """One decode step -> (logits fp16 (V,), argmax token)."""
        h = self.w["embed"][int(token)][None, :].astype(np.float16)
        for li in range(self.args.num_hidden_layers):
            h = self.layer(li, h)
        hn = rms_norm(h, self.w["final_norm"], self.args.rms_norm_eps).astype(np.float16)
        logits = self._lin(hn, self.w["lm_head"])[0]
        return logits, int(np.argmax(logits.astype(np.float32)))


# --------------------------------------------------------------------------- #
# Tensor-parallel sharding of the synthetic weights (host logic; no reference
# counterpart — the reference is single-device).
# --------------------------------------------------------------------------- #


def shard_weights_tp(args: OracleArgs, weights: dict, rank: int, world: int) -> dict:
    """Column/row-parallel shard of one rank, by noise group and MLP columns.

    qkv: the rank keeps its q_groups/world groups of origin and noise Q heads
    and its kv heads of every slot; o: the matching input columns; gate/up:
    rows [r*I/w, (r+1)*I/w); down: the matching input columns. Embedding,
    norms and lm_head stay replicated.
    """
    G, gr, d, Hk = args.num_noise_heads, args.grouped_ratio, args.head_dim, args.kv_heads_per_slot
    if G % world or Hk % world or args.intermediate_size % world:
        raise ValueError("q_groups, kv heads and intermediate size must divide the TP world size")
    gpr = G // world  # groups per rank
    kpr = Hk // world  # kv heads per slot per rank
    el = 32 // args.bits
    gs = args.group_size
    I = args.intermediate_size
    ipr = I // world

    def rows(triple, idx):
        return tuple(np.ascontiguousarray(t[idx]) for t in triple)

    def cols(triple, c0, c1):
        dta, s, b = triple
        return (
            np.ascontiguousarray(dta[:, c0 // el : c1 // el]),
            np.ascontiguousarray(s[:, c0 // gs : c1 // gs]),
            np.ascontiguousarray(b[:, c0 // gs : c1 // gs]),
        )

    qo0 = rank * gpr * gr
    origin_rows = np.arange(qo0 * d, (qo0 + gpr * gr) * d)
    noise_base = G * gr * d
    noise_rows = noise_base + np.arange(rank * gpr * d, (rank + 1) * gpr * d)
    kbase = G * (gr + 1) * d
    # k heads are interleaved k1/k2 pairs (head 2j -> k1[j], 2j+1 -> k2[j]).
    k_rows = kbase + np.arange(2 * rank * kpr * d, 2 * (rank + 1) * kpr * d)
    vbase = kbase + 2 * Hk * d
    v_rows = vbase + np.arange(2 * rank * kpr * d, 2 * (rank + 1) * kpr * d)
    qkv_idx = np.concatenate([origin_rows, noise_rows, k_rows, v_rows])

    out_layers = []
    for L in weights["layers"]:
        c0 = rank * gpr * gr * 2 * d
        c1 = (rank + 1) * gpr * gr * 2 * d
        lam = np.asarray(L["lambda_full"]).reshape(-1)
        if lam.size == G * gr:
            lam = lam[qo0 : qo0 + gpr * gr]
        elif lam.size == G:
            lam = lam[rank * gpr : (rank + 1) * gpr]
        out_layers.append(
            dict(
                L,
                qkv=rows(L["qkv"], qkv_idx),
                o=cols(L["o"], c0, c1),
                gate=rows(L["gate"], np.arange(rank * ipr, (rank + 1) * ipr)),
                up=rows(L["up"], np.arange(rank * ipr, (rank + 1) * ipr)),
                down=cols(L["down"], rank * ipr, (rank + 1) * ipr),
                lambda_full=lam.astype(np.float32),
            )
        )
    return dict(weights, layers=out_layers)


# --------------------------------------------------------------------------- #
# Vanilla decoder (2.6B-class, ungrouped differential attention) —
# model.py:486-559 (_forward_vanilla), 450-454 (_init_vanilla), cache.py:55-175
# --------------------------------------------------------------------------- #


def vanilla_v_paired_to_slab_perm(n_kv_heads: int) -> np.ndarray:
    """``cache.py:55-69``: head index of the paired V order [v0_a, v0_b, v1_a, ...] that lands
    at slab position p of [va_0 .. va_{H-1}, vb_0 .. vb_{H-1}]: 2·(p mod H) + p div H."""
    h = n_kv_heads
    return np.array([2 * (p % h) + (p // h) for p in range(2 * h)], np.int64)


def vanilla_v_slab_to_paired_perm(n_kv_heads: int) -> np.ndarray:
    """``cache.py:72-82``: the inverse permutation, (q mod 2)·H + q div 2."""
    h = n_kv_heads
    return np.array([(q % 2) * h + (q // 2) for q in range(2 * h)], np.int64)


class OracleVanillaKVCache:
    """``MotifVanillaKVCache`` (``cache.py:85-175``) on mlx-lm ``KVCache`` semantics: keys in the
    projection's stripe order, values in slab order, appended along the sequence axis;
    ``update_and_fetch`` returns the whole live cache."""

    V_HEAD_ORDER = "slab"

    def __init__(self):
        self.keys = None
        self.values = None
        self.offset = 0

    def update_and_fetch(self, k, v):
        if self.keys is None:
            self.keys, self.values = np.array(k), np.array(v)
        else:
            self.keys = np.concatenate([self.keys, k], axis=2)
            self.values = np.concatenate([self.values, v], axis=2)
        self.offset += k.shape[2]
        return self.keys, self.values

    def hf_ordered_values(self):  # cache.py:160-175
        if self.values is None:
            return None
        perm = vanilla_v_slab_to_paired_perm(self.values.shape[1] // 2)
        return self.values[:, perm, : self.offset, :]

    @property
    def meta_state(self):
        return (self.V_HEAD_ORDER,)


def _gqa_sdpa(q, k, v, scale):
    """``mx.fast.scaled_dot_product_attention`` with native GQA: q head i reads kv head i // n_rep;
    a block of S > 1 queries (the last S cache positions) gets the causal mask."""
    S, N = np.asarray(q).shape[2], np.asarray(k).shape[2]
    return causal_gqa_sdpa(q, k, v, scale, N - S)


def vanilla_attention_reference(q, k, v_paired, cache, lam, lam_init, subln_w, eps=1e-5, kv_dtype=np.float16):
    """``_forward_vanilla`` (``model.py:486-559``) from the roped projections to the o_proj input.

    q (B, 2H, S, d) and k (B, 2Hk, S, d) after RoPE, v (B, 2Hk, S, d) in the projection's paired
    order; ``cache`` an ``OracleVanillaKVCache``. V goes to slab order (line 514), the cache
    appends (521), the stripes split (528-533), four SDPAs run (548-551), and
    (o1 − λ·o2) per slab, SubLN and the (1 − λ_init) scale follow (553-557), each op
    rounded to fp16 as MLX's fp16 arrays are. Returns (B, H, S, 2d) fp16. ``kv_dtype``: the
    element type the cache holds (fp16; float32 for rows dequantized from a q4/q8 cache, whose
    values the quantized SDPA reads in fp32).
    """
    f16 = np.float16
    B, two_h, S, d = q.shape
    H, Hk = two_h // 2, k.shape[1] // 2
    v = np.asarray(v_paired)[:, vanilla_v_paired_to_slab_perm(Hk)]
    K, V = cache.update_and_fetch(np.asarray(k, kv_dtype), np.asarray(v, kv_dtype))
    kv = K.shape[2]
    va, vb = V[:, :Hk], V[:, Hk:]
    q_ = np.asarray(q).reshape(B, H, 2, S, d)
    k_ = K.reshape(B, Hk, 2, kv, d)
    q1, q2 = q_[:, :, 0], q_[:, :, 1]
    k1, k2 = k_[:, :, 0], k_[:, :, 1]
    scale = d ** -0.5
    o1a, o1b = (_gqa_sdpa(q1, k1, vs, scale).astype(f16) for vs in (va, vb))
    o2a, o2b = (_gqa_sdpa(q2, k2, vs, scale).astype(f16) for vs in (va, vb))
    lam16 = np.float16(np.asarray(lam, np.float32).reshape(-1)[0])

    def diff(o1, o2):  # fp16 ops: the product, then the difference, each rounded
        return (o1.astype(np.float32) - (lam16.astype(np.float32) * o2.astype(np.float32)).astype(f16)).astype(f16)

    out = np.concatenate([diff(o1a, o2a), diff(o1b, o2b)], axis=-1)
    out = rms_norm(out, subln_w, eps).astype(f16)
    scale_out = np.float16(1.0 - lam_init)  # a Python float meets an fp16 array: cast to fp16
    return (out.astype(np.float32) * np.float32(scale_out)).astype(f16)


@dataclass
class OracleVanillaArgs:
    """Shape of a vanilla (2.6B-class) Motif decoder; defaults are config[3]."""

    hidden_size: int = 2048
    num_hidden_layers: int = 32
    intermediate_size: int = 8192
    num_attention_heads: int = 16  # halved to 8 effective differential heads
    num_key_value_heads: int = 4  # halved to 2
    head_dim: int = 128
    vocab_size: int = 219520
    rms_norm_eps: float = 1e-6
    attn_rms_norm_eps: float = 1e-5
    rope_theta: float = 10000.0
    group_size: int = 64
    bits: int = 4

    @property
    def H(self):  # model.py:452
        return self.num_attention_heads // 2

    @property
    def Hk(self):  # model.py:453
        return self.num_key_value_heads // 2

    @property
    def qkv_out(self):
        d = self.head_dim
        return 2 * self.H * d + 2 * self.Hk * d + 2 * self.Hk * d


def make_synthetic_weights_vanilla(args: OracleVanillaArgs, seed: int = 0, std: float = 0.02) -> dict:
    """Random-init vanilla weights: per layer one fused [q | k | v] linear (rows of q_proj,
    k_proj and v_proj stacked; v in the projection's paired order), o (hidden, 2H·d), the
    PolyNorm MLP, SubLN over 2d and one λ per layer."""
    rng = np.random.default_rng(seed)
    g, b = args.group_size, args.bits
    Hd, I, d = args.hidden_size, args.intermediate_size, args.head_dim
    f16 = np.float16

    def norm_w(n):
        return (1.0 + 0.02 * rng.standard_normal(n)).astype(f16)

    layers = []
    for li in range(args.num_hidden_layers):
        lam_init = lambda_init_for_layer(li)
        lp = [rng.standard_normal(d).astype(np.float32) * 0.1 for _ in range(4)]
        layers.append(
            dict(
                input_norm=norm_w(Hd),
                post_norm=norm_w(Hd),
                qkv=_q_linear(rng, args.qkv_out, Hd, std, g, b),
                o=_q_linear(rng, Hd, 2 * args.H * d, std, g, b),
                gate=_q_linear(rng, I, Hd, std, g, b),
                up=_q_linear(rng, I, Hd, std, g, b),
                down=_q_linear(rng, Hd, I, std, g, b),
                subln=norm_w(2 * d),
                lambda_init=lam_init,
                lambda_full=np.array([lambda_full(*lp, lam_init)], np.float32),
                polynorm_w=np.array([1 / 3, 1 / 3, 1 / 3], f16),
                polynorm_b=np.zeros((1,), f16),
            )
        )
    return dict(
        embed=(rng.standard_normal((args.vocab_size, Hd), dtype=np.float32) * std).astype(f16),
        final_norm=norm_w(Hd),
        lm_head=_q_linear(rng, args.vocab_size, Hd, std, g, b),
        layers=layers,
    )


class VanillaDecodeOracle:
    """Batch-1 decode of the vanilla model: ``MotifDecoderLayer`` (``model.py:845-855``) with
    ``_forward_vanilla`` (486-559) on an ``OracleVanillaKVCache``, the PolyNorm MLP (267-268),
    final norm and lm_head (858-905); every op rounded to fp16."""

    def __init__(self, args: OracleVanillaArgs, weights: dict):
        self.args = args
        self.w = weights
        self.caches = [OracleVanillaKVCache() for _ in range(args.num_hidden_layers)]
        self.inv_freq = rope_inv_freq(args.head_dim, args.rope_theta)

    def _lin(self, x, triple):
        a = self.args
        return quantized_matmul(x, *triple, group_size=a.group_size, bits=a.bits).astype(np.float16)

    def layer(self, li: int, h: np.ndarray) -> np.ndarray:
        a = self.args
        L = self.w["layers"][li]
        f16 = np.float16
        d, H, Hk = a.head_dim, a.H, a.Hk
        cache = self.caches[li]
        x = rms_norm(h, L["input_norm"], a.rms_norm_eps).astype(f16)
        qkv = self._lin(x, L["qkv"])
        qd, kd = 2 * H * d, 2 * Hk * d
        q = qkv[..., :qd].reshape(1, 1, 2 * H, d).transpose(0, 2, 1, 3)
        k = qkv[..., qd : qd + kd].reshape(1, 1, 2 * Hk, d).transpose(0, 2, 1, 3)
        v = qkv[..., qd + kd :].reshape(1, 1, 2 * Hk, d).transpose(0, 2, 1, 3)
        off = cache.offset
        q = rope(q, off, inv_freq=self.inv_freq).astype(f16)
        k = rope(k, off, inv_freq=self.inv_freq).astype(f16)
        out = vanilla_attention_reference(q, k, v, cache, L["lambda_full"], L["lambda_init"], L["subln"],
                                          a.attn_rms_norm_eps)
        out = out.transpose(0, 2, 1, 3).reshape(1, -1)
        o = self._lin(out, L["o"])
        h = (h.astype(np.float32) + o.astype(np.float32)).astype(f16)
        x2 = rms_norm(h, L["post_norm"], a.rms_norm_eps).astype(f16)
        act = polynorm_mul_reference(self._lin(x2, L["gate"]), self._lin(x2, L["up"]), L["polynorm_w"],
                                     L["polynorm_b"], 1e-6)
        dn = self._lin(act, L["down"])
        return (h.astype(np.float32) + dn.astype(np.float32)).astype(f16)

    def step(self, token: int):
        """One decode step -> (logits fp16 (V,), argmax token)."""
        h = self.w["embed"][int(token)][None, :].astype(np.float16)
        for li in range(self.args.num_hidden_layers):
            h = self.layer(li, h)
        hn = rms_norm(h, self.w["final_norm"], self.args.rms_norm_eps).astype(np.float16)
        logits = self._lin(hn, self.w["lm_head"])[0]
        return logits, int(np.argmax(logits.astype(np.float32)))
