"""4-slot KV caches for grouped differential attention (k1, k2, v1, v2) on the GPU.

API of ``src/mlx_motif/cache.py``: ``MotifGroupedKVCache`` (303-404) and
``MotifGroupedQuantizedKVCache`` (407-545) with ``update_and_fetch_4``,
``update_and_fetch_4_quantized``, ``offset``, ``step``, ``trim``,
``is_trimmable``, ``state`` / ``meta_state``, ``make_mask`` and
``to_quantized``; ``MotifVanillaKVCache`` (85-175); and mlx-lm's stock
``KVCache`` for a grouped model run without the 4-slot cache. Fetches return the FULL row-contiguous capacity buffers;
consumers bound reads by ``offset`` (the attention kernels take it as
``kv_len``).

Writes go through ``motif_kv4_append``: a copy for the fp16 cache, or one
batched affine quantize of all four slots for the quantized cache (codes,
scales and biases bit-identical to quantizing each slot separately, since
groups never cross the head axis).

Capacity: by default slots grow in ``step``-row increments like the reference
(``cache.py:245-265``). Passing ``max_size`` preallocates the whole capacity
once, rounded up to whole ``step`` blocks, so the buffers never move — the
form a captured CUDA graph needs.
"""

from __future__ import annotations

import torch

from ._native import check, dtype_code, lib, motif_kv4_slots, ptr, stream


def create_causal_mask(N: int, offset: int = 0, window_size: int | None = None) -> torch.Tensor:
    """Boolean (N, offset+N) causal mask (True = attend), mlx-lm's convention."""
    rinds = torch.arange(offset + N)
    linds = torch.arange(offset, offset + N)
    mask = linds[:, None] >= rinds[None]
    if window_size is not None:
        mask = mask & (linds[:, None] < rinds[None] + window_size)
    return mask


def create_attention_mask(N: int, offset: int = 0, return_array: bool = False, window_size: int | None = None):
    """mlx-lm cache-module contract: None for one query row, "causal" or an explicit array otherwise."""
    if N == 1:
        return None
    if return_array:
        return create_causal_mask(N, offset, window_size)
    return "causal"


def _slots_struct(slots, bits: int, group_size: int, B: int, H: int, cap: int, D: int) -> motif_kv4_slots:
    s = motif_kv4_slots()
    for i, slot in enumerate(slots):
        if bits == 16:
            s.data[i] = ptr(slot)
            s.scales[i] = None
            s.biases[i] = None
        else:
            s.data[i] = ptr(slot[0])
            s.scales[i] = ptr(slot[1])
            s.biases[i] = ptr(slot[2])
    s.bits = bits
    s.group_size = group_size
    s.batch = B
    s.heads = H
    s.capacity = cap
    s.head_dim = D
    return s


class MotifGroupedKVCacheBase:
    """Offset bookkeeping and storage growth shared by both 4-slot caches (``cache.py:178-300``)."""

    step = 256

    def update_and_fetch(self, keys, values):
        raise NotImplementedError(
            "MotifGroupedKVCacheBase subclasses require the model to call "
            "update_and_fetch_4 directly — the 1-slot path is intentionally unsupported."
        )

    def is_trimmable(self):
        return True

    def trim(self, n):
        n = min(self.offset, n)
        self.offset -= n
        return n

    def make_mask(self, N, return_array: bool = False, window_size=None):
        return create_attention_mask(N, offset=self.offset, return_array=return_array, window_size=window_size)

    @staticmethod
    def _assert_uniform_heads(k1, k2, v1, v2) -> None:
        h1 = k1.shape[1]
        if not (k2.shape[1] == v1.shape[1] == v2.shape[1] == h1):
            raise ValueError(
                "4-slot grouped KV cache requires k1/k2/v1/v2 to share a head "
                f"count; got k1={h1}, k2={k2.shape[1]}, v1={v1.shape[1]}, "
                f"v2={v2.shape[1]}. This happens with k_ratio > 1, which the "
                "4-slot cache does not support."
            )

    def _grow(self, B: int, H: int, S: int, D: int, dtype, device) -> None:
        prev = self.offset
        if self.k1 is not None and prev + S <= self._slot_capacity(self.k1):
            return
        if self.max_size is not None:
            # Whole `step`-row blocks, the reference's growth unit: every capacity is then a
            # multiple of 256, which the tensor-core decode step's q4 tiles (four rows of scales
            # per 16-byte line) and 128-row TMA boxes rely on. Reads stay bounded by the offset.
            cap = -(-self.max_size // self.step) * self.step
            if self.k1 is None and prev + S <= cap:
                self.k1, self.k2, self.v1, self.v2 = (
                    self._init_storage(B, H, cap, D, dtype, device) for _ in range(4)
                )
                return
            raise ValueError(f"cache capacity {cap} exceeded (offset {prev} + {S} rows)")
        new_len = ((self.step + S - 1) // self.step) * self.step
        if self.k1 is None:
            self.k1, self.k2, self.v1, self.v2 = (
                self._init_storage(B, H, new_len, D, dtype, device) for _ in range(4)
            )
            return
        slots = [self.k1, self.k2, self.v1, self.v2]
        if prev % self.step != 0:
            slots = [self._trim_slot(s, prev) for s in slots]
        fresh = self._init_storage(B, H, new_len, D, dtype, device)
        self.k1, self.k2, self.v1, self.v2 = (self._expand_slot(s, fresh) for s in slots)

    def slots_struct(self) -> motif_kv4_slots:
        """C-ABI view of the four slots (valid until the next growth)."""
        return self._struct()


class MotifGroupedKVCache(MotifGroupedKVCacheBase):
    """fp16/bf16 4-slot cache; each slot (B, H, capacity, D)."""

    def __init__(self, max_size: int | None = None):
        self.k1 = self.k2 = self.v1 = self.v2 = None
        self.offset = 0
        self.max_size = max_size

    def _slot_capacity(self, slot) -> int:
        return slot.shape[2]

    def _init_storage(self, B, H, n, D, dtype, device):
        return torch.zeros((B, H, n, D), dtype=dtype, device=device)

    def _trim_slot(self, slot, prev):
        return slot[..., :prev, :].contiguous()

    def _expand_slot(self, slot, fresh):
        return torch.cat([slot, fresh], dim=2)

    def _struct(self):
        B, H, cap, D = self.k1.shape
        return _slots_struct((self.k1, self.k2, self.v1, self.v2), 16, 64, B, H, cap, D)

    def update_and_fetch_4(self, k1, k2, v1, v2):
        """Append the 4 incoming slices; return the FULL capacity buffers (``cache.py:337-360``)."""
        self._assert_uniform_heads(k1, k2, v1, v2)
        B, H, S, D = k1.shape
        prev = self.offset
        self._grow(B, H, S, D, k1.dtype, k1.device)
        ins = [t.to(self.k1.dtype).contiguous() for t in (k1, k2, v1, v2)]
        s = self._struct()
        check(lib.motif_kv4_append(dtype_code(self.k1), s, *(ptr(t) for t in ins), S, prev, None,
                                   stream(k1.device)), "kv4_append")
        self.offset += S
        return self.k1, self.k2, self.v1, self.v2

    @property
    def state(self):
        if self.offset == 0 or self.k1 is None:
            return self.k1, self.k2, self.v1, self.v2
        o = self.offset
        return tuple(t[..., :o, :] for t in (self.k1, self.k2, self.v1, self.v2))

    @state.setter
    def state(self, v):
        self.k1, self.k2, self.v1, self.v2 = (t.contiguous() if t is not None else None for t in v)

    @property
    def meta_state(self):
        return (str(self.offset),)

    @meta_state.setter
    def meta_state(self, v):
        self.offset = int(v[0])

    def to_quantized(self, group_size: int = 64, bits: int = 8) -> "MotifGroupedQuantizedKVCache":
        """Switch to the quantized variant (``cache.py:394-404``)."""
        from .quantization import quantize

        new = MotifGroupedQuantizedKVCache(group_size=group_size, bits=bits)
        if self.offset > 0:
            o = self.offset
            new.k1, new.k2, new.v1, new.v2 = (
                quantize(t[..., :o, :].contiguous(), group_size, bits) for t in (self.k1, self.k2, self.v1, self.v2)
            )
            new.offset = self.offset
        return new


class MotifGroupedQuantizedKVCache(MotifGroupedKVCacheBase):
    """4-slot quantized cache: each slot a (data uint32, scales, biases) triple."""

    def __init__(self, group_size: int = 64, bits: int = 8, max_size: int | None = None):
        self.k1 = self.k2 = self.v1 = self.v2 = None
        self.offset = 0
        self.group_size = group_size
        self.bits = bits
        self.max_size = max_size

    def _slot_capacity(self, slot) -> int:
        return slot[0].shape[2]

    def _init_storage(self, B, H, n, D, dtype, device):
        el = 32 // self.bits
        return (
            torch.zeros((B, H, n, D // el), dtype=torch.uint32, device=device),
            torch.zeros((B, H, n, D // self.group_size), dtype=dtype, device=device),
            torch.zeros((B, H, n, D // self.group_size), dtype=dtype, device=device),
        )

    def _trim_slot(self, slot, prev):
        return tuple(x[..., :prev, :].contiguous() for x in slot)

    def _expand_slot(self, slot, fresh):
        return tuple(torch.cat([slot[i], fresh[i]], dim=-2) for i in range(3))

    def _struct(self):
        B, H, cap, _ = self.k1[0].shape
        D = self.k1[1].shape[-1] * self.group_size
        return _slots_struct((self.k1, self.k2, self.v1, self.v2), self.bits, self.group_size, B, H, cap, D)

    def _update_4(self, k1, k2, v1, v2):
        """One batched quantize of all four slots written at [offset, offset+S) (``cache.py:485-512``)."""
        self._assert_uniform_heads(k1, k2, v1, v2)
        B, H, S, D = k1.shape
        prev = self.offset
        self._grow(B, H, S, D, k1.dtype, k1.device)
        ins = [t.to(self.k1[1].dtype).contiguous() for t in (k1, k2, v1, v2)]
        s = self._struct()
        check(lib.motif_kv4_append(dtype_code(self.k1[1]), s, *(ptr(t) for t in ins), S, prev, None,
                                   stream(k1.device)), "kv4_append")
        self.offset += S

    def update_and_fetch_4(self, k1, k2, v1, v2):
        """Quantize and append; return dequantized live slices (``cache.py:448-465``)."""
        from .quantization import dequantize

        self._update_4(k1, k2, v1, v2)
        o = self.offset

        def _deq(slot):
            return dequantize(*(x[..., :o, :].contiguous() for x in slot), group_size=self.group_size,
                              bits=self.bits)

        return _deq(self.k1), _deq(self.k2), _deq(self.v1), _deq(self.v2)

    def update_and_fetch_4_quantized(self, k1, k2, v1, v2):
        """Quantize and append; return each slot's FULL capacity triple (``cache.py:467-483``)."""
        self._update_4(k1, k2, v1, v2)
        return self.k1, self.k2, self.v1, self.v2

    @property
    def state(self):
        if self.offset == 0 or self.k1 is None:
            return self.k1, self.k2, self.v1, self.v2
        o = self.offset
        return tuple(tuple(x[..., :o, :] for x in slot) for slot in (self.k1, self.k2, self.v1, self.v2))

    @state.setter
    def state(self, v):
        self.k1, self.k2, self.v1, self.v2 = (
            tuple(x.contiguous() for x in slot) if slot is not None else None for slot in v
        )

    @property
    def meta_state(self):
        return tuple(map(str, (self.offset, self.group_size, self.bits)))

    @meta_state.setter
    def meta_state(self, v):
        self.offset, self.group_size, self.bits = map(int, v)


# --------------------------------------------------------------------------- #
# Vanilla (ungrouped) differential attention cache — cache.py:55-175
# --------------------------------------------------------------------------- #


def vanilla_v_paired_to_slab_perm(n_kv_heads: int) -> torch.Tensor:
    """Head index of the projection's paired V order ``[v0_a, v0_b, v1_a, ...]`` that lands at slab
    position p of ``[va_0 .. va_{H-1}, vb_0 .. vb_{H-1}]``: 2·(p mod H) + p div H (``cache.py:55-69``)."""
    h = n_kv_heads
    return torch.tensor([2 * (p % h) + (p // h) for p in range(2 * h)], dtype=torch.int64)


def vanilla_v_slab_to_paired_perm(n_kv_heads: int) -> torch.Tensor:
    """The inverse permutation, slab -> paired: (q mod 2)·H + q div 2 (``cache.py:72-82``)."""
    h = n_kv_heads
    return torch.tensor([(q % 2) * h + (q // 2) for q in range(2 * h)], dtype=torch.int64)


class MotifVanillaKVCache(MotifGroupedKVCache):
    """KV cache of the vanilla (2.6B-class) differential attention path (``cache.py:85-175``).

    Reference view (mlx-lm ``KVCache`` semantics): ``keys`` (B, 2·Hk, offset, d) in the k
    projection's stripe order [k1_0, k2_0, k1_1, ...] and ``values`` (B, 2·Hk, offset, d) in SLAB
    order [va_0 .. va_{Hk-1}, vb_0 .. vb_{Hk-1}]; ``update_and_fetch(keys, values)`` takes the new
    rows in those orders and returns the whole live cache. ``meta_state`` carries the "slab"
    marker and a restore with another (or no) marker raises; ``hf_ordered_values`` gives V in
    the paired order.

    Device layout: the 4-slot form with Hk heads per slot — k1 (even k heads), k2 (odd), va, vb
    — so the one-launch decode step (``motif_vanilla_decode_step``) reads each slot as a
    row-contiguous (Hk, capacity, d) array. ``keys``/``values`` are gathered copies.
    """

    V_HEAD_ORDER = "slab"

    def update_and_fetch(self, keys, values):
        if keys.shape[1] % 2 or keys.shape[1] != values.shape[1]:
            raise ValueError(f"vanilla cache: keys {tuple(keys.shape)} / values {tuple(values.shape)} need "
                             "an even, equal head count (2·Hk)")
        hk = keys.shape[1] // 2
        self.update_and_fetch_4(keys[:, 0::2], keys[:, 1::2], values[:, :hk], values[:, hk:])
        return self.keys, self.values

    @property
    def keys(self):
        if self.k1 is None:
            return None
        o = self.offset
        B, hk, _, D = self.k1.shape
        return torch.stack([self.k1[:, :, :o], self.k2[:, :, :o]], dim=2).reshape(B, 2 * hk, o, D)

    @property
    def values(self):
        if self.v1 is None:
            return None
        o = self.offset
        return torch.cat([self.v1[:, :, :o], self.v2[:, :, :o]], dim=1)

    def hf_ordered_values(self):
        """The live V in the projection's paired order (a gathered copy), or None when empty."""
        v = self.values
        if v is None:
            return None
        return v[:, vanilla_v_slab_to_paired_perm(v.shape[1] // 2).to(v.device)]

    @property
    def state(self):
        return self.keys, self.values

    @state.setter
    def state(self, v):
        keys, values = v
        B, h2, n, D = keys.shape
        hk = h2 // 2
        cap = max(n, self.max_size or 0)
        if self.max_size is not None:  # preallocated: whole step blocks, as _grow allocates
            cap = -(-cap // self.step) * self.step
        self.k1, self.k2, self.v1, self.v2 = (
            self._init_storage(B, hk, cap, D, keys.dtype, keys.device) for _ in range(4)
        )
        for dst, src in zip((self.k1, self.k2, self.v1, self.v2),
                            (keys[:, 0::2], keys[:, 1::2], values[:, :hk], values[:, hk:])):
            dst[:, :, :n].copy_(src)
        self.offset = n

    @property
    def meta_state(self):
        return (self.V_HEAD_ORDER,)

    @meta_state.setter
    def meta_state(self, v):
        marker = None
        if isinstance(v, (tuple, list)):
            marker = v[0] if len(v) else None
        elif v not in (None, ""):
            marker = v
        if marker is None:
            raise ValueError("MotifVanillaKVCache.from_state: state carries no V head-order marker; the "
                             f"vanilla path stores V in slab order (expected {self.V_HEAD_ORDER!r})")
        if marker != self.V_HEAD_ORDER:
            raise ValueError(f"MotifVanillaKVCache.from_state: V head-order marker mismatch — got {marker!r}, "
                             f"expected {self.V_HEAD_ORDER!r}")

    @classmethod
    def from_state(cls, state, meta_state, max_size: int | None = None) -> "MotifVanillaKVCache":
        """mlx-lm ``_BaseCache.from_state``: state first, then the marker check."""
        c = cls(max_size=max_size)
        c.state = state
        c.meta_state = meta_state
        return c


# --------------------------------------------------------------------------- #
# Stock single-slot cache (mlx-lm KVCache) for the grouped model without the 4-slot cache
# --------------------------------------------------------------------------- #


class KVCache:
    """mlx-lm's stock ``KVCache`` contract: ``keys``/``values`` (B, n_kv_heads, capacity, D) in the
    projection's head order, ``update_and_fetch(keys, values)`` returns the live rows, ``offset``,
    ``step``-row growth, ``trim``, ``state``/``meta_state``.

    The reference's ``make_cache`` hands a grouped model this cache when
    ``MLX_MOTIF_4SLOT_CACHE=0`` (``model.py:983-989``); its attention then slices k1 = heads[0::2],
    k2 = heads[1::2] (and v1/v2 alike) from the fetched buffers (``model.py:670-683``). Here the
    kernels read those slices in place: with k_ratio 1 the even and odd heads are k1 and k2, so
    ``slots_struct`` describes the buffers as four slots of n_kv_heads/2 heads and capacity
    2·capacity whose rows [0, capacity) are exactly the sliced heads' rows (slot k2 starts one
    head later). Appends, the decode step and the attention kernels then work unchanged, and
    every read stays below ``offset``.
    """

    step = 256

    def __init__(self, max_size: int | None = None):
        self.keys = self.values = None
        self.offset = 0
        self.max_size = max_size

    def is_trimmable(self):
        return True

    def trim(self, n):
        n = min(self.offset, n)
        self.offset -= n
        return n

    def make_mask(self, N, return_array: bool = False, window_size=None):
        return create_attention_mask(N, offset=self.offset, return_array=return_array, window_size=window_size)

    @staticmethod
    def _alloc(B: int, H2: int, cap: int, D: int, dtype, device) -> torch.Tensor:
        """Zeroed (B, H2, cap, D) storage followed by one spare head of padding: the odd-head slot
        of ``slots_struct`` begins one head into the buffer, so its last head's view (capacity
        2·cap) ends one head past the buffer; the padding keeps that span allocated."""
        flat = torch.zeros(B * H2 * cap * D + cap * D, dtype=dtype, device=device)
        return flat[: B * H2 * cap * D].view(B, H2, cap, D)

    def _grow(self, B: int, H2: int, S: int, D: int, dtype, device) -> None:
        prev = self.offset
        if self.keys is not None and prev + S <= self.keys.shape[2]:
            return
        if self.max_size is not None:
            cap = -(-self.max_size // self.step) * self.step
            if self.keys is None and prev + S <= cap:
                self.keys = self._alloc(B, H2, cap, D, dtype, device)
                self.values = self._alloc(B, H2, cap, D, dtype, device)
                return
            raise ValueError(f"cache capacity {cap} exceeded (offset {prev} + {S} rows)")
        new_len = ((self.step + S - 1) // self.step) * self.step
        cap = new_len if self.keys is None else prev + new_len
        keys = self._alloc(B, H2, cap, D, dtype, device)
        values = self._alloc(B, H2, cap, D, dtype, device)
        if self.keys is not None:
            keys[..., :prev, :].copy_(self.keys[..., :prev, :])
            values[..., :prev, :].copy_(self.values[..., :prev, :])
        self.keys, self.values = keys, values

    def slots_struct(self) -> motif_kv4_slots:
        """The four-slot view of the kernels (valid until the next growth): k1 = even key heads,
        k2 = odd key heads, v1 = even value heads, v2 = odd value heads."""
        B, H2, cap, D = self.keys.shape
        s = _slots_struct((self.keys, self.keys, self.values, self.values), 16, 64, B, H2 // 2, 2 * cap, D)
        row_bytes = cap * D * self.keys.element_size()
        s.data[1] = s.data[1] + row_bytes
        s.data[3] = s.data[3] + row_bytes
        return s

    def update_and_fetch(self, keys, values):
        """Append (B, n_kv_heads, S, D) keys/values at ``offset``; return the live rows."""
        B, H2, S, D = keys.shape
        if H2 % 2 or values.shape != keys.shape:
            raise ValueError(f"KVCache: keys {tuple(keys.shape)} / values {tuple(values.shape)} need an even, "
                             "equal head count")
        prev = self.offset
        self._grow(B, H2, S, D, keys.dtype, keys.device)
        ins = [t.to(self.keys.dtype).contiguous() for t in (keys[:, 0::2], keys[:, 1::2], values[:, 0::2],
                                                               values[:, 1::2])]
        check(lib.motif_kv4_append(dtype_code(self.keys), self.slots_struct(), *(ptr(t) for t in ins), S, prev,
                                   None, stream(keys.device)), "kv4_append")
        self.offset += S
        return self.keys[..., : self.offset, :], self.values[..., : self.offset, :]

    @property
    def state(self):
        if self.keys is None:
            return None, None
        return self.keys[..., : self.offset, :], self.values[..., : self.offset, :]

    @state.setter
    def state(self, v):
        keys, values = v
        B, H2, n, D = keys.shape
        cap = max(n, self.max_size or 0)
        cap = -(-cap // self.step) * self.step
        self.keys = self._alloc(B, H2, cap, D, keys.dtype, keys.device)
        self.values = self._alloc(B, H2, cap, D, keys.dtype, keys.device)
        self.keys[..., :n, :].copy_(keys)
        self.values[..., :n, :].copy_(values)
        self.offset = n

    @property
    def meta_state(self):
        return ""

    @meta_state.setter
    def meta_state(self, v):
        if v not in (None, ""):
            raise ValueError(f"KVCache carries no meta state; got {v!r}")
