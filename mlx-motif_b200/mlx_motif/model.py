"""Motif GDA decoder on B200: config, path resolution and the CUDA-graph decode engine.

Host-side mirror of ``src/mlx_motif/model.py``:
  * ``ModelArgs`` with the reference's validation rules (``model.py:48-204``).
  * ``AttnPath`` / ``_resolve_attention_path`` (``model.py:288-344``), same
    truth table and env flags (``MLX_MOTIF_QUANT_SDPA``, ``MLX_MOTIF_DUAL_V``).
  * λ helpers (``model.py:389, 462-470``) and the origin-first Q permutation
    of ``fuse_qkv`` (``model.py:994-1015``).
  * ``MotifDecoder``: batch-1 decode of the grouped (12.7B-class) model
    through the DUAL_V / QUANT_SDPA path of ``_forward_grouped``
    (``model.py:563-837``) and ``MotifDecoderLayer`` (845-855). One decode
    step is a fixed sequence of C-ABI kernels captured once into a CUDA graph;
    the position and KV length live in device memory, so the graph replays at
    every length and the greedy token never leaves the GPU.

Per layer the step launches: fused-qkv GEMV, RoPE+4-slot append, fused
dual-V attention + GDA post (2 kernels), o_proj GEMV, residual+RMSNorm,
fused gate|up GEMV, PolyNorm·up, down GEMV, residual+RMSNorm.
"""

from __future__ import annotations

import contextlib
import enum
import math
import os
from dataclasses import dataclass

import torch

from ._native import check, lib, motif_linear_io, ptr, stream
from .cache import KVCache, MotifGroupedKVCache, MotifGroupedQuantizedKVCache, MotifVanillaKVCache
from .linear import QuantizedLinear
from .quantization import quantize

# MOTIF_NVTX=1: NVTX ranges around every op a decoder launches (per layer and op name) and around
# graph replays and prompt blocks, for Nsight timelines. Ranges are host-side markers: a replayed
# CUDA graph shows as one "decode_step" range, its kernels inside it.
_NVTX = os.environ.get("MOTIF_NVTX", "0") not in ("", "0")


def nvtx_range(name: str):
    """An NVTX range named ``name`` while MOTIF_NVTX is set, else a no-op context."""
    if not _NVTX:
        return contextlib.nullcontext()
    return torch.cuda.nvtx.range(name)

# --------------------------------------------------------------------------- #
# Config (model.py:48-204)
# --------------------------------------------------------------------------- #


@dataclass
class ModelArgs:
    model_type: str = "motif"
    hidden_size: int = 4096
    num_hidden_layers: int = 48
    intermediate_size: int = 14336
    num_attention_heads: int = 32
    num_key_value_heads: int = 16
    vocab_size: int = 219520
    rms_norm_eps: float = 1e-6
    rope_theta: float = 10000.0
    max_position_embeddings: int = 32768
    head_dim: int | None = 128
    num_noise_heads: int | None = 8
    k_ratio: int = 1
    attn_rms_norm_eps: float = 1e-5
    tie_word_embeddings: bool = False
    fused_rope: bool = False
    # The reference's remaining config fields (model.py:65-76), accepted so its configs construct;
    # MotifDecoder rejects the values its decode path does not implement.
    rope_scaling: dict | None = None
    hidden_act: str = "poly_norm"
    use_bias: bool = False
    expanded: bool = False
    sliding_window: int | None = None
    use_sliding_window: bool = False
    max_window_layers: int | None = None
    bos_token_id: int | None = None
    eos_token_id: int | None = None

    @classmethod
    def from_dict(cls, params: dict) -> "ModelArgs":
        """The fields of ``params`` that ModelArgs has (unknown keys ignored, as mlx-lm's
        ``BaseModelArgs.from_dict``); absent optional fields take the reference's defaults
        (head_dim and num_noise_heads None, max_position_embeddings 8192), not this class's
        12.7B-class ones."""
        import dataclasses

        names = {f.name for f in dataclasses.fields(cls)}
        kw = {k: v for k, v in params.items() if k in names}
        for k, v in (("head_dim", None), ("num_noise_heads", None), ("max_position_embeddings", 8192)):
            kw.setdefault(k, v)
        return cls(**kw)

    def __post_init__(self) -> None:
        for name in ("hidden_size", "num_hidden_layers", "intermediate_size", "num_attention_heads",
                     "num_key_value_heads", "vocab_size", "max_position_embeddings"):
            v = getattr(self, name)
            if type(v) is not int:
                raise ValueError(f"{name} must be an integer; got {v!r}")
            if v <= 0:
                raise ValueError(f"{name} must be greater than zero; got {v}")
        if self.head_dim is not None:
            if type(self.head_dim) is not int:
                raise ValueError(f"head_dim must be an integer; got {self.head_dim!r}")
            if self.head_dim <= 0:
                raise ValueError(f"head_dim must be greater than zero; got {self.head_dim}")
        elif self.hidden_size < self.num_attention_heads:
            raise ValueError("derived head_dim must be greater than zero")
        elif self.hidden_size % self.num_attention_heads:
            raise ValueError("hidden_size must be divisible by num_attention_heads when head_dim is omitted")
        if self.is_grouped:
            self._validate_grouped()
        else:
            self._validate_vanilla()

    def _validate_vanilla(self) -> None:
        if self.num_attention_heads % 2:
            raise ValueError("num_attention_heads must be even for vanilla differential attention")
        if self.num_key_value_heads % 2:
            raise ValueError("num_key_value_heads must be even for vanilla differential attention")
        if self.num_attention_heads % self.num_key_value_heads:
            raise ValueError("num_attention_heads must be divisible by num_key_value_heads")
        if self.head_dim is not None and self.head_dim * self.num_attention_heads != self.hidden_size:
            raise ValueError("head_dim * num_attention_heads must equal hidden_size for vanilla attention")

    def _validate_grouped(self) -> None:
        if type(self.num_noise_heads) is not int:
            raise ValueError(f"num_noise_heads must be an integer when provided; got {self.num_noise_heads!r}")
        if self.num_noise_heads <= 0:
            raise ValueError("num_noise_heads must be greater than zero")
        if type(self.k_ratio) is not int:
            raise ValueError(f"k_ratio must be an integer; got {self.k_ratio!r}")
        if self.k_ratio < 1:
            raise ValueError(f"k_ratio must be greater than or equal to 1 for grouped attention; got {self.k_ratio}")
        if self.num_attention_heads <= self.num_noise_heads:
            raise ValueError("num_attention_heads must be greater than num_noise_heads for grouped attention")
        if self.num_attention_heads % self.num_noise_heads:
            raise ValueError("num_attention_heads must be divisible by num_noise_heads")
        width = self.k_ratio + 1
        if self.num_key_value_heads < width:
            raise ValueError(f"num_key_value_heads must be at least k_ratio + 1 for grouped attention; "
                             f"got {self.num_key_value_heads} and {self.k_ratio}")
        if self.num_key_value_heads % width:
            raise ValueError(f"num_key_value_heads must be divisible by k_ratio + 1; "
                             f"got {self.num_key_value_heads} and {self.k_ratio}")
        k_noise = self.num_key_value_heads // width
        if self.num_noise_heads % k_noise:
            raise ValueError("num_noise_heads must be divisible by num_key_value_heads / (k_ratio + 1)")
        if (self.num_attention_heads // self.num_noise_heads - 1) % self.k_ratio:
            raise ValueError("the grouped attention ratio must be divisible by k_ratio")

    @property
    def is_grouped(self) -> bool:
        return self.num_noise_heads is not None

    # Derived attention dims: grouped (MotifAttention._init_grouped, model.py:424-447) and
    # vanilla (_init_vanilla, model.py:450-454: H = heads / 2, Hk = kv heads / 2).
    @property
    def d(self) -> int:
        return self.head_dim or self.hidden_size // self.num_attention_heads

    @property
    def grouped_ratio(self) -> int:
        """Grouped: origin heads per noise head. Vanilla: q pairs per kv pair (n_rep = H / Hk)."""
        if not self.is_grouped:
            return self.num_attention_heads // self.num_key_value_heads
        return (self.num_attention_heads - self.num_noise_heads) // self.num_noise_heads

    @property
    def q_heads(self) -> int:
        if not self.is_grouped:
            return self.num_attention_heads
        return (self.grouped_ratio + 1) * self.num_noise_heads

    @property
    def q_origin(self) -> int:
        """Rows of the attention output (each 2·d wide): gr·G grouped, H vanilla."""
        if not self.is_grouped:
            return self.num_attention_heads // 2
        return self.grouped_ratio * self.num_noise_heads

    @property
    def k_noise_heads(self) -> int:
        return self.num_key_value_heads // (self.k_ratio + 1)

    @property
    def kv_repeat(self) -> int:
        if not self.is_grouped:
            return 1
        return self.num_noise_heads // self.k_noise_heads

    @property
    def qkv_out(self) -> int:
        return self.q_heads * self.d + self.num_key_value_heads * self.d + 2 * self.k_noise_heads * self.d


# --------------------------------------------------------------------------- #
# Path resolution (model.py:288-344)
# --------------------------------------------------------------------------- #


class AttnPath(enum.Enum):
    QUANT_SDPA = "sdpa_dual_v_q4"
    DUAL_V = "sdpa_dual_v"
    FALLBACK = "stacked_sdpa"


def _resolve_attention_path(cache, S: int, kv_repeat: int, kr: int, fused_rope: bool, env=os.environ) -> AttnPath:
    """First match wins: QUANT_SDPA (quantized 4-slot cache), DUAL_V, else FALLBACK."""
    falsy = ("0", "", "false", "False")
    decode_ok = S == 1 and kv_repeat == 1 and kr == 1
    if (decode_ok and not fused_rope and isinstance(cache, MotifGroupedQuantizedKVCache)
            and env.get("MLX_MOTIF_QUANT_SDPA", "1") not in falsy):
        return AttnPath.QUANT_SDPA
    if decode_ok and not fused_rope and env.get("MLX_MOTIF_DUAL_V", "1") not in falsy:
        return AttnPath.DUAL_V
    return AttnPath.FALLBACK


def make_cache(args: ModelArgs, max_size: int | None = None, env=os.environ) -> list:
    """One cache per layer, chosen by ``MLX_MOTIF_4SLOT_CACHE`` as ``Model.make_cache`` does
    (``model.py:922-991``): unset or "1" -> ``MotifGroupedKVCache`` (4 fp16 slots), "q4"/"4" and
    "q8"/"8" -> ``MotifGroupedQuantizedKVCache`` (group 64), "0"/""/"false"/"off" -> the stock
    ``KVCache``; a vanilla model always gets ``MotifVanillaKVCache``. A grouped model with
    k_ratio > 1 cannot use the 4-slot caches: an explicit request raises ``ValueError``, the
    default quietly falls back to the stock cache. ``max_size`` preallocates (graph-safe)."""
    raw = env.get("MLX_MOTIF_4SLOT_CACHE")
    explicit = raw is not None
    val = (raw if explicit else "1").lower()
    use_4slot = val not in ("0", "", "false", "off")
    if use_4slot and args.is_grouped and args.k_ratio != 1:
        if explicit:
            raise ValueError(
                "MLX_MOTIF_4SLOT_CACHE is not supported with k_ratio > 1 "
                f"(got k_ratio={args.k_ratio}): the 4-slot grouped KV cache allocates every slot with k1's "
                "head count, which differs from k2/v1/v2 when k_ratio > 1. Unset MLX_MOTIF_4SLOT_CACHE for "
                "this model configuration.")
        use_4slot = False
    caches = []
    for _ in range(args.num_hidden_layers):
        if not args.is_grouped:
            caches.append(MotifVanillaKVCache(max_size=max_size))
        elif not use_4slot:
            caches.append(KVCache(max_size=max_size))
        elif val in ("q4", "4"):
            caches.append(MotifGroupedQuantizedKVCache(group_size=64, bits=4, max_size=max_size))
        elif val in ("q8", "8"):
            caches.append(MotifGroupedQuantizedKVCache(group_size=64, bits=8, max_size=max_size))
        else:
            caches.append(MotifGroupedKVCache(max_size=max_size))
    return caches


def decode_attention_mode(args: ModelArgs, cache, env=os.environ) -> tuple[AttnPath, str]:
    """The grouped decode step's path (``_resolve_attention_path`` with S = 1) and the launches
    that realise it: "fused" for QUANT_SDPA and for DUAL_V on fp16 rows (fp16 or stock cache),
    "bridge" for DUAL_V or FALLBACK on a packed cache (its rows dequantized to fp16 first, as
    ``update_and_fetch_4`` returns them, ``cache.py:448-465``), "two_call" for FALLBACK on fp16
    rows. MOTIF_FUSED_ATTN=0 turns "fused" into "two_call" (for comparisons)."""
    path = _resolve_attention_path(cache, 1, args.kv_repeat, args.k_ratio, args.fused_rope, env=env)
    packed = isinstance(cache, MotifGroupedQuantizedKVCache)
    if path is AttnPath.FALLBACK:
        mode = "bridge" if packed else "two_call"
    elif path is AttnPath.DUAL_V and packed:
        mode = "bridge"
    else:
        mode = "fused"
    if mode == "fused" and env.get("MOTIF_FUSED_ATTN", "1") == "0":
        mode = "two_call"
    return path, mode


def cache_kind(cache) -> str:
    """The decoder's name for a cache object: "fp16", "q4", "q8" or "stock"."""
    if isinstance(cache, MotifGroupedQuantizedKVCache):
        return f"q{cache.bits}"
    if isinstance(cache, KVCache):
        return "stock"
    if isinstance(cache, MotifGroupedKVCache):
        return "fp16"
    raise TypeError(f"not a cache of this package: {type(cache).__name__}")


# --------------------------------------------------------------------------- #
# λ and the origin-first permutation
# --------------------------------------------------------------------------- #


def lambda_init_for_layer(layer_idx: int) -> float:
    """λ_init = 0.8 − 0.6·exp(−0.3·(layer_idx − 1)) (``model.py:389``)."""
    return 0.8 - 0.6 * math.exp(-0.3 * (layer_idx - 1))


def lambda_full(lq1, lk1, lq2, lk2, lam_init: float) -> torch.Tensor:
    """exp(Σ lq1·lk1) − exp(Σ lq2·lk2) + λ_init in fp32 (``model.py:462-470``)."""
    l1 = torch.exp(torch.sum(lq1.float() * lk1.float(), dim=-1))
    l2 = torch.exp(torch.sum(lq2.float() * lk2.float(), dim=-1))
    return (l1 - l2 + lam_init).reshape(1).float()


def origin_first_perm(q_groups: int, gr: int, d: int) -> torch.Tensor:
    """Row permutation HF head stripes -> [origin heads | noise heads] (``model.py:994-1015``)."""
    heads = [g * (gr + 1) + p for g in range(q_groups) for p in range(gr)]
    heads += [g * (gr + 1) + gr for g in range(q_groups)]
    return torch.cat([torch.arange(h * d, (h + 1) * d) for h in heads])


def rope_inv_freq(dims: int, base: float, device) -> torch.Tensor:
    """fp32 inverse frequencies 2^(−(i/(dims/2))·log2 base), i < dims/2 (non-traditional RoPE).

    Formed in float64 and rounded once to fp32, so every caller gets the same table.
    """
    half = dims // 2
    vals = [2.0 ** (-(i / half) * math.log2(base)) for i in range(half)]
    return torch.tensor(vals, dtype=torch.float64).to(torch.float32).to(device)


# --------------------------------------------------------------------------- #
# Tensor-parallel shard plan (no reference counterpart: the reference is single-device)
# --------------------------------------------------------------------------- #


def tp_shard_plan(args: ModelArgs, rank: int, world: int) -> dict:
    """Which rows/columns of each global weight rank `rank` of `world` keeps.

    Attention is split by GDA group (each group's gr origin heads, its noise
    head and its kv head of every slot stay on one rank, so attention and
    gda_post need no exchange); o_proj keeps the matching input columns;
    gate/up keep rows [r·I/w, (r+1)·I/w) and down the matching columns. The
    two row-parallel outputs (o_proj, down_proj) are summed across ranks. The
    lm_head keeps vocabulary rows [r·V/w, (r+1)·V/w); the greedy token is the
    largest of the ranks' packed argmax keys (one int64 MAX all-reduce).
    """
    G, gr, d, Hk, I = args.num_noise_heads, args.grouped_ratio, args.d, args.k_noise_heads, args.intermediate_size
    if G % world or Hk % world or I % world or G != Hk:
        raise ValueError(f"TP {world}: q_groups {G}, kv heads {Hk} and intermediate {I} must split evenly")
    gpr, kpr, ipr = G // world, Hk // world, I // world
    qo0 = rank * gpr * gr
    qkv_rows = torch.cat([
        torch.arange(qo0 * d, (qo0 + gpr * gr) * d),  # origin heads of my groups
        G * gr * d + torch.arange(rank * gpr * d, (rank + 1) * gpr * d),  # my noise heads
        G * (gr + 1) * d + torch.arange(2 * rank * kpr * d, 2 * (rank + 1) * kpr * d),  # (k1,k2) pairs
        G * (gr + 1) * d + 2 * Hk * d + torch.arange(2 * rank * kpr * d, 2 * (rank + 1) * kpr * d),  # (v1,v2)
    ])
    V = args.vocab_size
    if V % world:
        raise ValueError(f"TP {world}: vocab {V} must split evenly")
    vpr = V // world
    return dict(
        qkv_rows=qkv_rows,
        o_cols=(rank * gpr * gr * 2 * d, (rank + 1) * gpr * gr * 2 * d),
        mlp_rows=(rank * ipr, (rank + 1) * ipr),
        vocab_rows=(rank * vpr, (rank + 1) * vpr),
    )


# --------------------------------------------------------------------------- #
# Decode engine
# --------------------------------------------------------------------------- #


def _ql(triple, device) -> QuantizedLinear:
    import numpy as np

    d, s, b = triple
    if isinstance(d, np.ndarray):
        d = torch.from_numpy(d.view(np.int32)).view(torch.uint32)
        s = torch.from_numpy(s)
        b = torch.from_numpy(b)
    return QuantizedLinear(d.to(device), s.to(device), b.to(device))


def _t(a, device, dtype=None) -> torch.Tensor:
    import numpy as np

    if isinstance(a, np.ndarray):
        a = torch.from_numpy(np.ascontiguousarray(a))
    a = torch.as_tensor(a)
    return a.to(device=device, dtype=dtype or a.dtype).contiguous()


class MotifDecoder:
    """Batch-1 greedy decoder of the Motif model on one GPU (or one TP rank).

    Grouped configs (``num_noise_heads`` set) run ``_forward_grouped``'s DUAL_V /
    QUANT_SDPA path; vanilla configs (``num_noise_heads`` None, the 2.6B class)
    run ``_forward_vanilla`` (``model.py:486-559``) on a ``MotifVanillaKVCache``
    (one GPU; its 4-slot form holds k1, k2 and the two V slabs).

    ``cache``: "fp16" (4-slot fp16 rows), "q4"/"q8" (packed 4-slot cache, group 64),
    "stock" (mlx-lm's single-slot ``KVCache``), or None to take the kind ``make_cache``
    picks from ``MLX_MOTIF_4SLOT_CACHE`` (the reference's default: 4-slot fp16).
    ``max_seq`` is the preallocated KV capacity (rounded up to whole 256-row steps).

    The attention of each decode step follows ``_resolve_attention_path`` (``model.py:302-344``,
    ``MLX_MOTIF_QUANT_SDPA`` / ``MLX_MOTIF_DUAL_V``), as ``_forward_grouped`` does at
    ``model.py:608-614`` and ``716-768``:
      * QUANT_SDPA (packed cache) and DUAL_V (fp16 or stock cache): the one-launch step
        ``motif_gda_decode_step`` (RoPE, append, dual-V attention over the cache as stored,
        gda_post_split);
      * DUAL_V on a packed cache (``MLX_MOTIF_QUANT_SDPA=0``): the dequant bridge — RoPE + the
        quantized append, the slots dequantized to fp16 rows (``update_and_fetch_4``'s bridge,
        ``cache.py:448-465``), then the split-KV attention on those rows;
      * FALLBACK (``MLX_MOTIF_DUAL_V=0``, or ``fused_rope``): separate launches — RoPE + append,
        then the split-KV attention and merge (over the dequantized rows for a packed cache).
    With a process group ``tp_group`` the weights passed in must already be this rank's shard
    (q groups and MLP columns); the engine all-reduces the o_proj and down_proj outputs and the
    PolyNorm statistics.
    """

    def __init__(self, args: ModelArgs, weights: dict, cache: str | None = None, max_seq: int = 4096,
                 device="cuda", tp_group=None):
        if args.hidden_act != "poly_norm" or args.use_bias or args.rope_scaling is not None or args.use_sliding_window:
            raise ValueError("MotifDecoder implements hidden_act='poly_norm', bias-free linears, unscaled RoPE and "
                             f"full attention (got hidden_act={args.hidden_act!r}, use_bias={args.use_bias}, "
                             f"rope_scaling={args.rope_scaling!r}, use_sliding_window={args.use_sliding_window})")
        self.vanilla = not args.is_grouped
        if self.vanilla:
            if tp_group is not None:
                raise ValueError("the vanilla decode path runs on one GPU (no tensor parallelism)")
            if args.grouped_ratio not in (1, 2, 4) or args.d != 128:
                raise ValueError(f"vanilla decode step built for n_rep 1, 2, 4 and head_dim 128 "
                                 f"(got n_rep {args.grouped_ratio}, head_dim {args.d})")
        elif args.k_ratio != 1 or args.kv_repeat != 1:
            raise ValueError("MotifDecoder runs the grouped DUAL_V/QUANT_SDPA decode path "
                             "(num_noise_heads set, k_ratio == 1, kv_repeat == 1)")
        self.args = args
        self.device = torch.device(device)
        self.tp_group = tp_group
        self.tp = 1 if tp_group is None else torch.distributed.get_world_size(tp_group)
        a = args
        self.gr = a.grouped_ratio  # vanilla: n_rep, the q pairs of one kv pair
        self.d = a.d
        self.kv_heads = a.k_noise_heads // self.tp
        if self.vanilla:
            self.q_groups = self.kv_heads
            self.q_heads = 2 * self.q_groups * self.gr  # q1/q2 stripes interleaved
        else:
            self.q_groups = a.num_noise_heads // self.tp
            self.q_heads = self.q_groups * (self.gr + 1)
        self.q_origin = self.q_groups * self.gr
        self.inter = a.intermediate_size // self.tp
        self.H = a.hidden_size
        self.V = a.vocab_size
        self.max_seq = max_seq
        if cache is None:
            cache = "fp16" if self.vanilla else cache_kind(make_cache(args, env=os.environ)[0])
        if cache not in ("fp16", "q4", "q8", "stock") or (cache == "stock" and self.vanilla):
            raise ValueError(f"cache must be fp16, q4, q8 (or stock for a grouped model); got {cache!r}")
        self.cache_kind = cache
        dev = self.device

        self.embed = _t(weights["embed"], dev, torch.float16)
        self.final_norm = _t(weights["final_norm"], dev, torch.float16)
        self.lm_head = weights["lm_head"] if isinstance(weights["lm_head"], QuantizedLinear) else _ql(weights["lm_head"], dev)
        # Under TP the lm_head is this rank's vocabulary shard, rows [v0, v0 + V_local).
        self.V_local = self.lm_head.out_dim
        rank = 0 if tp_group is None else torch.distributed.get_rank(tp_group)
        self.v0 = rank * self.V_local
        if self.V_local * self.tp != a.vocab_size:
            raise ValueError(f"lm_head rows {self.V_local} x TP {self.tp} != vocab {a.vocab_size}")
        self.layers = []
        for L in weights["layers"]:
            if "gate_up" in L:
                gate_up = L["gate_up"]
            else:
                g, u = _ql(L["gate"], dev), _ql(L["up"], dev)
                gate_up = QuantizedLinear(torch.cat([g.weight, u.weight]), torch.cat([g.scales, u.scales]),
                                          torch.cat([g.biases, u.biases]))
            self.layers.append(dict(
                input_norm=_t(L["input_norm"], dev, torch.float16),
                post_norm=_t(L["post_norm"], dev, torch.float16),
                qkv=L["qkv"] if isinstance(L["qkv"], QuantizedLinear) else _ql(L["qkv"], dev),
                o=L["o"] if isinstance(L["o"], QuantizedLinear) else _ql(L["o"], dev),
                gate_up=gate_up,
                down=L["down"] if isinstance(L["down"], QuantizedLinear) else _ql(L["down"], dev),
                subln=_t(L["subln"], dev, torch.float16),
                lambda_full=_t(L["lambda_full"], dev, torch.float32).reshape(-1),
                lambda_init=float(L["lambda_init"]),
                polynorm_w=_t(L.get("polynorm_w", [1 / 3, 1 / 3, 1 / 3]), dev, torch.float16),
                polynorm_b=_t(L.get("polynorm_b", [0.0]), dev, torch.float16),
            ))
        self._check_shapes()

        # KV caches: preallocated capacity (buffers never move; graph-safe).
        if cache == "fp16":
            kind = MotifVanillaKVCache if self.vanilla else MotifGroupedKVCache
            self.caches = [kind(max_size=max_seq) for _ in self.layers]
        elif cache == "stock":
            self.caches = [KVCache(max_size=max_seq) for _ in self.layers]
        else:
            bits = 4 if cache == "q4" else 8
            self.caches = [MotifGroupedQuantizedKVCache(64, bits, max_size=max_seq) for _ in self.layers]
        for c in self.caches:
            c._grow(1, (2 if cache == "stock" else 1) * self.kv_heads, 1, self.d, torch.float16, dev)
        self._slots = [c.slots_struct() for c in self.caches]
        self._resolve_attn_mode()

        f16 = torch.float16
        H, d = self.H, self.d
        # Residual stream ping-pong: the qkv prologue reads h_a and writes h_b, the gate|up
        # prologue reads h_b and writes h_a (a kernel never overwrites what its CTAs read).
        self.h_a = torch.zeros(H, dtype=f16, device=dev)
        self.h_b = torch.zeros(H, dtype=f16, device=dev)
        self.x = torch.zeros(H, dtype=f16, device=dev)  # scratch input vector (timing helpers)
        self.qkv = torch.zeros(self.layers[0]["qkv"].out_dim, dtype=f16, device=dev)
        self.q = torch.zeros(self.q_heads * d, dtype=f16, device=dev)
        self.attn = torch.zeros(self.q_origin * 2 * d, dtype=f16, device=dev)
        self.o = torch.zeros(H, dtype=f16, device=dev)
        self.gu = torch.zeros(2 * self.inter, dtype=f16, device=dev)
        self.act = torch.zeros(self.inter, dtype=f16, device=dev)
        self.dn = torch.zeros(H, dtype=f16, device=dev)
        # PolyNorm statistics of the gate rows: one (Σg², Σg⁴, Σg⁶) triplet per 16-row tile.
        self.stats_tiles = self.inter // 16
        self.stats = torch.zeros(self.stats_tiles * 3, dtype=torch.float32, device=dev)
        self.stats_sum = torch.zeros(3, dtype=torch.float32, device=dev)
        self.logits = torch.zeros(self.V_local, dtype=f16, device=dev)
        self.amax_key = torch.zeros(1, dtype=torch.int64, device=dev)  # TP: this rank's argmax key
        self.token = torch.zeros(1, dtype=torch.int32, device=dev)
        # pos_len[0] = position of the token being decoded, pos_len[1] = kv_len after its append.
        self.pos_len = torch.tensor([0, 1], dtype=torch.int32, device=dev)
        self._one_one = torch.ones(2, dtype=torch.int32, device=dev)
        self.inv_freq = rope_inv_freq(d, a.rope_theta, dev)
        self.scale = d ** -0.5
        lin_ws = max(lib.motif_linear_fused_workspace_bytes(ql.out_dim, ql.in_dim)
                     for L in self.layers for ql in (L["qkv"], L["o"], L["gate_up"], L["down"]))
        lin_ws = max(lin_ws, lib.motif_linear_fused_workspace_bytes(self.V_local, H))
        # short row blocks (speculative verify, prompt tails): chunks of 2..8 rows share one weight pass
        lin_ws = max([lin_ws] + [lib.motif_quantized_linear_workspace_bytes(m, ql.out_dim, ql.in_dim, 4, 64)
                                 for m in range(2, 9)
                                 for ql in [self.lm_head] + [L[n] for L in self.layers
                                                             for n in ("qkv", "o", "gate_up", "down")]])
        if self.inter % 16:
            raise ValueError("intermediate size per rank must be a multiple of 16")
        self.lin_ws = torch.zeros(max(lin_ws, 16), dtype=torch.uint8, device=dev)
        if self.fused_attn:
            self.attn_ws_bytes = lib.motif_gda_decode_step_workspace_bytes(self.q_heads, d, 64)
        else:
            self.attn_ws_bytes = lib.motif_gda_decode_attention_workspace_bytes(self.q_heads, d, 64)
        self.attn_ws = torch.zeros(self.attn_ws_bytes, dtype=torch.uint8, device=dev)
        self._bridge = None
        if self.attn_mode == "bridge":  # fp16 rows of the dequant bridge, shared by the layers in turn
            from .cache import _slots_struct

            cap = self._slots[0].capacity
            self._bridge = [torch.zeros((1, self.kv_heads, cap, d), dtype=f16, device=dev) for _ in range(4)]
            self._bridge_slots = _slots_struct(self._bridge, 16, 64, 1, self.kv_heads, cap, d)
        self.argmax_ws_bytes = lib.motif_argmax_workspace_bytes(self.V_local)
        self.argmax_ws = torch.zeros(self.argmax_ws_bytes, dtype=torch.uint8, device=dev)
        self.offset = 0  # host mirror of pos_len[0]
        # Sampling of the head: 0 = greedy (fused argmax); > 0 = temperature (set_sampling).
        self.temperature = 0.0
        self.seed = 0
        self.stream_id = 0
        self._graphs: dict[bool, torch.cuda.CUDAGraph] = {}
        # row-block forwards (the speculative verify) captured per (rows, logits buffer)
        self._row_graphs: dict[tuple, torch.cuda.CUDAGraph] = {}
        self._rows_seen: set = set()
        self._rows_ids = torch.zeros(128, dtype=torch.int32, device=dev)
        self.pinned_in = torch.zeros(1, dtype=torch.int32).pin_memory()
        self.pinned_out = torch.zeros(1, dtype=torch.int32).pin_memory()
        # Tensor parallelism exchanges the row-parallel outputs and the PolyNorm statistics through
        # peer memory inside the GEMVs (MOTIF_TP_NCCL=1: NCCL all-reduces instead).
        self.tp_exchange = self.tp_group is not None and os.environ.get("MOTIF_TP_NCCL", "0") != "1"
        # MOTIF_TP_KEY_EXCHANGE=1: the head's token keys meet over the same buffers (rows below
        # 2^24 - 1) instead of an NCCL MAX all-reduce.
        self.key_exchange = (self.tp_exchange and self.V < (1 << 24) - 1
                             and os.environ.get("MOTIF_TP_KEY_EXCHANGE", "0") == "1")
        self._xbuf = None
        if self.tp_exchange:
            self._setup_exchange()

    # ------------------------------------------------------------------ #
    def _resolve_attn_mode(self) -> None:
        """The decode step's attention launches: "fused" (one launch), "two_call" (RoPE + append,
        then the split-KV attention and merge) or "bridge" (two_call over fp16 rows dequantized
        from a packed cache), from ``_resolve_attention_path`` (vanilla models: "fused").
        MOTIF_FUSED_ATTN=0 turns "fused" into "two_call" (for comparisons)."""
        self.attn_path, mode = (None, "fused") if self.vanilla else decode_attention_mode(self.args, self.caches[0])
        self.attn_mode = mode
        self.fused_attn = mode == "fused"
        # kernels per layer: one step / RoPE+append, split attention, merge / + four dequantizes
        self.attn_launches = {"fused": 1, "two_call": 3, "bridge": 7}[mode]

    def make_cache(self) -> list:
        """Fresh caches for this decoder's model as the environment asks (``Model.make_cache``,
        ``model.py:922-991``), preallocated to this decoder's capacity."""
        return make_cache(self.args, max_size=self.max_seq, env=os.environ)

    def _check_shapes(self) -> None:
        L0 = self.layers[0]
        d = self.d
        exp_qkv = self.q_heads * d + 4 * self.kv_heads * d
        if L0["qkv"].out_dim != exp_qkv or L0["qkv"].in_dim != self.H:
            raise ValueError(f"qkv weight ({L0['qkv'].out_dim}, {L0['qkv'].in_dim}) != ({exp_qkv}, {self.H})")
        if L0["o"].in_dim != self.q_origin * 2 * d or L0["o"].out_dim != self.H:
            raise ValueError("o_proj shape mismatch")
        if L0["gate_up"].out_dim != 2 * self.inter or L0["down"].in_dim != self.inter:
            raise ValueError("MLP shape mismatch")

    @property
    def weight_bytes(self) -> int:
        """Packed weight bytes streamed per token (every linear + lm_head)."""
        n = self.lm_head.nbytes()
        for L in self.layers:
            n += sum(L[k].nbytes() for k in ("qkv", "o", "gate_up", "down"))
        return n

    def weights_dict(self) -> dict:
        """The device weights in the constructor's format (share them with another cache kind)."""
        return dict(embed=self.embed, final_norm=self.final_norm, lm_head=self.lm_head,
                    layers=[dict(L) for L in self.layers])

    def attention_kernel(self) -> str:
        """Which kernel the fused decode step launches for this decoder's caches: "tcgen05" (the
        tensor-core long-cache step) or "split" (the CUDA-core split-KV step); from
        ``motif_decode_step_kernel``, so it is the library's own choice, not a re-derivation."""
        k = lib.motif_decode_step_kernel(self._slots[0])
        if k < 0:
            check(-k, "decode_step_kernel")
        return {1: "split", 2: "tcgen05"}[k]

    def kv_bytes_per_token(self, kv_len: int) -> int:
        """KV-cache bytes the attention reads at one step (4 slots, all layers)."""
        d = self.d
        per_row = 2 * d if self.cache_kind in ("fp16", "stock") else \
            (d * (4 if self.cache_kind == "q4" else 8) // 8 + 4 * d // 64)
        return len(self.layers) * 4 * self.kv_heads * kv_len * per_row

    # ------------------------------------------------------------------ #
    def _setup_exchange(self) -> None:
        """One peer-visible buffer per rank (CUDA IPC) holding, for the two layer parities, every
        rank's o_proj and down_proj partial rows and PolyNorm tile statistics, each value as an
        8-byte (fp32, exchange number) pair, and for the two step parities every rank's greedy /
        sampled token key (motif_argmax_key_exchange). Ranks trade the IPC handles over the
        process group and open each other's buffers."""
        import ctypes as C

        W, H = self.tp, self.H
        me = torch.distributed.get_rank(self.tp_group)
        ntl = self.inter // 16
        part = W * H * 8
        off = dict(o=0, dn=2 * part, st=4 * part)
        off["key"] = off["st"] + 2 * W * ntl * 3 * 8
        total = off["key"] + 2 * W * 8
        ptr = C.c_void_p()
        handle = (C.c_char * lib.motif_ipc_handle_bytes())()
        check(lib.motif_ipc_alloc(total, C.byref(ptr), handle), "ipc_alloc")
        handles = [None] * W
        torch.distributed.all_gather_object(handles, bytes(handle), group=self.tp_group)
        peers = []
        for r in range(W):
            if r == me:
                peers.append(ptr.value)
            else:
                q = C.c_void_p()
                check(lib.motif_ipc_open(handles[r], C.byref(q)), "ipc_open")
                peers.append(q.value)
        self._xbuf, self._xpeers, self._xoff, self._xme, self._xntl = ptr.value, peers, off, me, ntl
        self._xbytes = total
        # every rank's key area, for the head's token exchange
        self._key_slots = (C.c_void_p * W)(*[base + off["key"] for base in peers])

    def _x_slot(self, kind: str, par: int, src: int) -> int:
        """Byte offset of source rank src's slot of exchange `kind` ("o", "dn", "st") at parity par."""
        W, H = self.tp, self.H
        if kind == "st":
            return self._xoff["st"] + (par * W + src) * self._xntl * 3 * 8
        return self._xoff[kind] + (par * W + src) * H * 8

    def _x_producer(self, io, out: str, layer: int) -> None:
        """io stores its rows (out "o"/"dn") or tile statistics ("st") of `layer` into every rank."""
        io.tp_world, io.tp_seq, io.tp_tag = self.tp, self.pos_len.data_ptr(), layer
        for r, base in enumerate(self._xpeers):
            if out == "st":
                io.tp_stats[r] = base + self._x_slot("st", layer & 1, self._xme)
            else:
                io.tp_out[r] = base + self._x_slot(out, layer & 1, self._xme)

    def _x_consumer(self, io, layer: int, kind: str) -> None:
        """io reads exchange `kind` of `layer`: the ranks' rows ("o"/"dn": its residual delta is their
        sum) or tile statistics ("st")."""
        io.tp_world, io.tp_seq, io.tp_tag = self.tp, self.pos_len.data_ptr(), layer
        if kind == "st":
            io.tp_stats_in = self._xbuf + self._x_slot("st", layer & 1, 0)
        else:
            io.tp_in = self._xbuf + self._x_slot(kind, layer & 1, 0)

    def _tp_reset_flags(self) -> None:
        """After the position is rewound every rank zeroes its exchange buffer between two
        barriers, so no pair can still carry the number of a step that is about to run again."""
        if not self.tp_exchange:
            return
        torch.cuda.synchronize(self.device)
        torch.distributed.barrier(group=self.tp_group)
        check(lib.motif_ipc_zero(self._xbuf, self._xbytes, stream(self.device)), "ipc_zero")
        torch.cuda.synchronize(self.device)
        torch.distributed.barrier(group=self.tp_group)

    _TP_WAIT_BYTE = 65504  # the GEMV workspace's int64 of exchange-read nanoseconds (CTA 0)
    _ERR_BYTE = 65532  # the GEMV workspace's error word (exchange waits that ran out)

    def exchange_read_ns(self, reset: bool = False) -> int:
        """Nanoseconds CTA 0 of the consuming GEMVs spent reading exchanged values (waits for the
        peers included) since the last reset; 0 without a peer-memory exchange."""
        if not self.tp_exchange:
            return 0
        word = self.lin_ws[self._TP_WAIT_BYTE:self._TP_WAIT_BYTE + 8].view(torch.int64)
        v = int(word.item())
        if reset:
            word.zero_()
        return v

    def release_exchange(self) -> None:
        """Close the peers' buffers and free this rank's (call on every rank, after a barrier)."""
        if self._xbuf is None:
            return
        torch.cuda.synchronize(self.device)
        for r, base in enumerate(self._xpeers):
            if r != self._xme:
                check(lib.motif_ipc_close(base), "ipc_close")
        check(lib.motif_ipc_free(self._xbuf), "ipc_free")
        self._xbuf = None

    def _allreduce(self, t: torch.Tensor) -> None:
        if self.tp_group is not None:
            torch.distributed.all_reduce(t, group=self.tp_group)

    def _io(self, mode: int, **kw) -> motif_linear_io:
        io = motif_linear_io()
        io.mode = mode
        for k, v in kw.items():
            setattr(io, k, v)
        return io

    def _build_plan(self) -> None:
        """Fixed C-ABI argument structs of every fused linear of a step (pointers never move)."""
        eps = self.args.rms_norm_eps
        I = self.inter
        gp = self.gu.data_ptr()
        tp = self.tp_group is not None
        X = self.tp_exchange
        plan = []
        for li, L in enumerate(self.layers):
            if li == 0:
                qkv_io = self._io(1, token=ptr(self.token), embed=ptr(self.embed), vocab=self.V,
                                  h_out=ptr(self.h_b), norm_w=ptr(L["input_norm"]), eps=eps)
            elif X:  # residual delta = the ranks' down_proj partials of the previous layer
                qkv_io = self._io(1, h_in=ptr(self.h_a), h_out=ptr(self.h_b), norm_w=ptr(L["input_norm"]), eps=eps)
                self._x_consumer(qkv_io, li - 1, "dn")
            else:
                qkv_io = self._io(1, h_in=ptr(self.h_a), delta=ptr(self.dn), h_out=ptr(self.h_b),
                                  norm_w=ptr(L["input_norm"]), eps=eps)
            o_io = self._io(0, x=ptr(self.attn))
            if X:
                self._x_producer(o_io, "o", li)
                gu_io = self._io(1, h_in=ptr(self.h_b), h_out=ptr(self.h_a), norm_w=ptr(L["post_norm"]), eps=eps,
                                 stats_rows=I)
                self._x_consumer(gu_io, li, "o")
                self._x_producer(gu_io, "st", li)
                dn_io = self._io(2, gate=gp, up=gp + 2 * I, stats=ptr(self.stats), stats_count=self.tp * self._xntl,
                                 poly_w=ptr(L["polynorm_w"]), poly_b=ptr(L["polynorm_b"]), poly_eps=1e-6,
                                 poly_dim=self.args.intermediate_size)
                self._x_consumer(dn_io, li, "st")
                self._x_producer(dn_io, "dn", li)
            else:
                gu_io = self._io(1, h_in=ptr(self.h_b), delta=ptr(self.o), h_out=ptr(self.h_a),
                                 norm_w=ptr(L["post_norm"]), eps=eps, stats_out=ptr(self.stats), stats_rows=I)
                stats_src, stats_n = (self.stats_sum, 1) if tp else (self.stats, self.stats_tiles)
                dn_io = self._io(2, gate=gp, up=gp + 2 * I, stats=ptr(stats_src), stats_count=stats_n,
                                 poly_w=ptr(L["polynorm_w"]), poly_b=ptr(L["polynorm_b"]), poly_eps=1e-6,
                                 poly_dim=self.args.intermediate_size)
            plan.append((qkv_io, o_io, gu_io, dn_io))
        # The lm_head GEMV also picks the greedy token and advances pos_len (MOTIF_FUSED_ARGMAX=0: separate
        # argmax launches).
        self.fused_argmax = (tp and self.temperature == 0) or (
            os.environ.get("MOTIF_FUSED_ARGMAX", "1") != "0" and self.temperature == 0)
        if tp and self.temperature == 0:  # this rank's key; the ranks' keys are combined by an all-reduce
            extra = dict(argmax_key_out=ptr(self.amax_key), argmax_row_offset=self.v0)
        elif tp:  # temperature: this rank's logits shard, then its Gumbel-max key (motif_sample_key)
            extra = {}
        elif self.fused_argmax:
            extra = dict(argmax_out=ptr(self.token), pos_len_inc=ptr(self.pos_len))
        else:
            extra = {}
        if X:
            head_io = self._io(1, h_in=ptr(self.h_a), norm_w=ptr(self.final_norm), eps=eps, **extra)
            self._x_consumer(head_io, len(self.layers) - 1, "dn")
        else:
            head_io = self._io(1, h_in=ptr(self.h_a), delta=ptr(self.dn), norm_w=ptr(self.final_norm), eps=eps,
                               **extra)
        self._plan = (plan, head_io)

    def _linear(self, io, ql: QuantizedLinear, out: torch.Tensor, st: int) -> None:
        check(lib.motif_linear_fused(io, ptr(ql.weight), ptr(ql.scales), ptr(ql.biases), ql.out_dim, ql.in_dim,
                                     ptr(out), ptr(self.lin_ws), self.lin_ws.numel(), st), "linear_fused")

    def _launch_step(self, with_head: bool) -> None:
        """Enqueue one decode step on the current stream (no host sync, no allocation).

        Per layer: qkv GEMV (prologue: [embedding +] residual + input RMSNorm), RoPE + 4-slot
        append, dual-V attention + GDA post (2 kernels), o_proj GEMV, gate|up GEMV (prologue:
        residual + post-attention RMSNorm; epilogue: PolyNorm statistics), down GEMV (prologue:
        PolyNorm·up). Head: lm_head GEMV (prologue: residual + final norm; epilogue: greedy token and
        position advance, or a separate argmax when MOTIF_FUSED_ARGMAX=0).
        """
        if getattr(self, "_plan", None) is None:
            self._build_plan()
        plan, head_io = self._plan
        st = stream(self.device)
        pos_p = self.pos_len.data_ptr()
        kvl_p = pos_p + 4
        tp = self.tp_group is not None
        for li, L in enumerate(self.layers):
            with nvtx_range(f"layer {li}"):
                self._launch_layer(li, L, plan[li], st, pos_p, kvl_p, tp)
        with nvtx_range("head"):
            self._head(with_head, head_io, st)

    def _launch_layer(self, li: int, L: dict, ios, st: int, pos_p: int, kvl_p: int, tp: bool) -> None:
        """One layer of ``_launch_step``."""
        qkv_io, o_io, gu_io, dn_io = ios
        with nvtx_range("qkv"):
            self._linear(qkv_io, L["qkv"], self.qkv, st)
        with nvtx_range("attention"):
            if self.vanilla:
                check(lib.motif_vanilla_decode_step(ptr(self.qkv), ptr(self.inv_freq), self._slots[li], pos_p,
                                                    self.scale, self.kv_heads, self.gr, ptr(L["subln"]),
                                                    ptr(L["lambda_full"]), L["lambda_init"],
                                                    self.args.attn_rms_norm_eps, ptr(self.attn), ptr(self.attn_ws),
                                                    self.attn_ws_bytes, st), "vanilla_decode_step")
            elif self.fused_attn:
                check(lib.motif_gda_decode_step(ptr(self.qkv), ptr(self.inv_freq), self._slots[li], pos_p, self.scale,
                                                self.q_groups, self.gr, ptr(L["subln"]), ptr(L["lambda_full"]),
                                                L["lambda_full"].numel(), L["lambda_init"],
                                                self.args.attn_rms_norm_eps, ptr(self.attn), ptr(self.attn_ws),
                                                self.attn_ws_bytes, st), "gda_decode_step")
            else:
                check(lib.motif_rope_qkv_append(ptr(self.qkv), ptr(self.inv_freq), self.q_heads, self._slots[li],
                                                pos_p, ptr(self.q), st), "rope_qkv_append")
                slots = self._slots[li]
                if self.attn_mode == "bridge":
                    slots = self._dequant_bridge(li, st)
                check(lib.motif_gda_decode_attention(ptr(self.q), slots, self.scale, self.q_groups, self.gr,
                                                     0, kvl_p, ptr(L["subln"]), ptr(L["lambda_full"]),
                                                     L["lambda_full"].numel(), L["lambda_init"],
                                                     self.args.attn_rms_norm_eps, ptr(self.attn), ptr(self.attn_ws),
                                                     self.attn_ws_bytes, st), "gda_decode_attention")
        with nvtx_range("o_proj"):
            self._linear(o_io, L["o"], self.o, st)
            if not self.tp_exchange:
                self._allreduce(self.o)
        with nvtx_range("gate_up"):
            self._linear(gu_io, L["gate_up"], self.gu, st)
            if tp and not self.tp_exchange:
                # Full-row PolyNorm statistics across ranks (12 bytes over NCCL).
                torch.sum(self.stats.view(-1, 3), dim=0, out=self.stats_sum)
                self._allreduce(self.stats_sum)
        with nvtx_range("down"):
            self._linear(dn_io, L["down"], self.dn, st)
            if not self.tp_exchange:
                self._allreduce(self.dn)

    def _dequant_bridge(self, li: int, st: int):
        """Layer li's packed slots dequantized to fp16 rows in the shared bridge buffers (every
        capacity row, so the launch does not depend on the length; rows past the length are
        zeros and never read) — the fetch of ``update_and_fetch_4`` on a quantized cache."""
        c = self.caches[li]
        rows = self.kv_heads * self._slots[li].capacity
        for i, slot in enumerate((c.k1, c.k2, c.v1, c.v2)):
            data, scales, biases = slot
            check(lib.motif_dequantize(0, c.bits, c.group_size, ptr(data), ptr(scales), ptr(biases), rows, self.d,
                                       ptr(self._bridge[i]), st), "dequantize")
        return self._bridge_slots

    def _head(self, with_head: bool, head_io, st: int) -> None:
        """lm_head + greedy token + position advance (one launch when the argmax is fused)."""
        if with_head:
            self._linear(head_io, self.lm_head, self.logits, st)
            if self.tp_group is not None:
                if self.temperature > 0:  # this shard's Gumbel-max key, noise drawn per global index
                    check(lib.motif_sample_key(ptr(self.logits), self.V_local, self.temperature, self.seed,
                                               ptr(self.pos_len), 0, self.stream_id, self.v0, ptr(self.amax_key), st),
                          "sample_key")
                if self.key_exchange:  # the ranks' keys meet over peer memory
                    import ctypes as C

                    check(lib.motif_argmax_key_exchange(ptr(self.amax_key), C.cast(self._key_slots, C.c_void_p),
                                                        self.tp, self._xme, ptr(self.pos_len), ptr(self.token),
                                                        ptr(self.pos_len), ptr(self.lin_ws) + self._ERR_BYTE, st),
                          "argmax_key_exchange")
                    return
                torch.distributed.all_reduce(self.amax_key, op=torch.distributed.ReduceOp.MAX, group=self.tp_group)
                check(lib.motif_argmax_key_decode(ptr(self.amax_key), ptr(self.token), ptr(self.pos_len), st),
                      "argmax_key_decode")
                return
            if self.fused_argmax:
                return  # the GEMV wrote the token and advanced pos_len
            if self.temperature > 0:  # Gumbel-max draw from softmax(logits / T); advances pos_len
                check(lib.motif_sample(ptr(self.logits), 1, self.V_local, self.V_local, self.temperature, self.seed,
                                       ptr(self.pos_len), 0, self.stream_id, ptr(self.token), ptr(self.pos_len), st),
                      "sample")
                return
            check(lib.motif_argmax(0, ptr(self.logits), self.V_local, ptr(self.token), ptr(self.argmax_ws),
                                   self.argmax_ws_bytes, st), "argmax")
        self.pos_len.add_(self._one_one)

    # ------------------------------------------------------------------ #
    def _graph(self, with_head: bool) -> torch.cuda.CUDAGraph:
        g = self._graphs.get(with_head)
        if g is None:
            # Warm up once outside capture (function attributes, NCCL comm init), then restore state.
            saved = (self.pos_len.clone(), self.token.clone())
            self._launch_step(with_head)
            self.pos_len.copy_(saved[0])
            self.token.copy_(saved[1])
            torch.cuda.synchronize(self.device)
            self._tp_reset_flags()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                self._launch_step(with_head)
            self._graphs[with_head] = g
        return g

    def set_sampling(self, temperature: float, seed: int = 0, stream_id: int = 0) -> None:
        """Head mode for the following steps: greedy (temperature 0) or a Gumbel-max draw from
        softmax(logits / temperature), seeded and counted by position (``motif_sample``; under
        tensor parallelism each rank draws the noise of its vocabulary shard by global index,
        ``motif_sample_key``, and the ranks' keys meet in the MAX all-reduce of the greedy head,
        so the draw equals one GPU's)."""
        self.temperature = float(temperature)
        self.seed = int(seed)
        self.stream_id = int(stream_id)
        self._plan = None
        self._graphs.clear()

    def release_graphs(self) -> None:
        """Drop every captured CUDA graph (decode steps and row blocks). Under tensor parallelism
        the graphs hold NCCL calls, so every rank calls this before the process group is
        destroyed."""
        self._graphs.clear()
        self._row_graphs.clear()
        self._rows_seen.clear()

    def rewind(self, offset: int) -> None:
        """Drop cache rows at and after ``offset`` (the reference cache's ``trim``): the next step
        writes position ``offset``."""
        if not 0 <= offset <= self.offset:
            raise ValueError(f"rewind to {offset} outside [0, {self.offset}]")
        self.offset = offset
        for c in self.caches:
            c.offset = offset
        self.pos_len.copy_(torch.tensor([offset, offset + 1], dtype=torch.int32))
        self._tp_reset_flags()

    def reset(self) -> None:
        self.pos_len.copy_(torch.tensor([0, 1], dtype=torch.int32))
        self.offset = 0
        for c in self.caches:
            c.offset = 0
        self._tp_reset_flags()

    def _bump_host(self, n: int = 1) -> None:
        self.offset += n
        for c in self.caches:
            c.offset = self.offset

    def step_device(self, with_head: bool = True) -> None:
        """One decode step from ``self.token`` (device); the argmax lands back in ``self.token``."""
        if self.offset >= self.max_seq:
            raise ValueError(f"KV capacity {self.max_seq} exhausted")
        with nvtx_range("decode_step"):
            self._graph(with_head).replay()
        self._bump_host()

    def step_eager(self, with_head: bool = True) -> None:
        """Same step launched kernel by kernel (no graph) — for debugging and tests."""
        if self.offset >= self.max_seq:
            raise ValueError(f"KV capacity {self.max_seq} exhausted")
        self._launch_step(with_head)
        self._bump_host()

    # Row blocks of at least this many prompt rows run the tensor-core GEMMs; shorter blocks of at
    # least min_rows_block rows run the multi-row GEMV (one weight pass per 8 rows). A prompt tail
    # shorter than that takes the decode step, one graph launch per token.
    min_block_rows = 128
    min_rows_block = 4

    def prefill(self, ids, chunk: int | None = None, batched: bool | None = None) -> None:
        """Ingest a prompt. All rows but the last run as blocks of up to ``chunk`` rows
        (default 2048, mlx-lm's prefill step) through the prompt path (q4 GEMMs on the tensor
        cores, or the multi-row GEMV below ``min_block_rows`` rows, and causal prompt attention);
        the last token, and a remainder shorter than ``min_rows_block``, take the decode step,
        which also yields the first greedy token.
        ``batched=False`` (or MOTIF_BATCHED_PREFILL=0, or tensor parallelism) runs every row
        through the decode step."""
        ids_d = torch.as_tensor(ids, dtype=torch.int32).reshape(-1).to(self.device)
        n = ids_d.numel()
        if batched is None:
            batched = os.environ.get("MOTIF_BATCHED_PREFILL", "1") != "0"
        batched = batched and self._block_ok()
        chunk = chunk or 2048
        i = 0
        if batched:
            while n - 1 - i >= self.min_rows_block:
                S = min(chunk, n - 1 - i)
                self._prefill_block(ids_d[i : i + S])
                i += S
        for j in range(i, n):
            self.token.copy_(ids_d[j : j + 1])
            self.step_device(with_head=(j == n - 1))

    def _block_ok(self) -> bool:
        """The prompt path's contract: head_dim 128 (the prompt attention and its combine)."""
        return self.d == 128

    def _gemm_ok(self) -> bool:
        """The tensor-core GEMM's shapes (k % 512, n % 128) for every linear of a layer; blocks
        of other shapes run the multi-row GEMV."""
        lins = [L[k] for L in self.layers for k in ("qkv", "o", "gate_up", "down")]
        return self.d == 128 and all(ql.in_dim % 512 == 0 and ql.out_dim % 128 == 0 for ql in lins)

    def _block_buffers(self, S: int) -> dict:
        b = getattr(self, "_blk", None)
        if b is not None and b["S"] >= S:
            return b
        f16, dev, d = torch.float16, self.device, self.d
        L0 = self.layers[0]
        b = dict(
            S=S,
            h=torch.empty((S, self.H), dtype=f16, device=dev),
            x=torch.empty((S, self.H), dtype=f16, device=dev),
            tmp=torch.empty((S, self.H), dtype=f16, device=dev),
            qkv=torch.empty((S, L0["qkv"].out_dim), dtype=f16, device=dev),
            q=torch.empty((self.q_heads, S, d), dtype=f16, device=dev),
            o=torch.empty((S, self.q_heads, 2 * d), dtype=f16, device=dev),
            attn=torch.empty((S, self.q_origin * 2 * d), dtype=f16, device=dev),
            gu=torch.empty((S, 2 * self.inter), dtype=f16, device=dev),
            act=torch.empty((S, self.inter), dtype=f16, device=dev),
            err=torch.zeros(1, dtype=torch.int32, device=dev),
        )
        if self.tp_group is not None:  # PolyNorm statistics and the lm_head shard's rows
            b["stats"] = torch.empty((S, 3), dtype=torch.float32, device=dev)
            b["logits"] = torch.empty((S, self.V_local), dtype=f16, device=dev)
            b["gathered"] = torch.empty(self.tp * S * self.V_local, dtype=f16, device=dev)
        self._blk = b
        self._row_graphs.clear()  # captured row blocks point at the old buffers
        return b

    def _attn_slots(self, li: int, rows: int):
        """The fp16 4-slot view the prompt attention reads: the cache itself, or (q4/q8 cache) its
        rows [0, rows) dequantized into a scratch fp16 cache — the reference's prompt path also
        attends over the dequantized fetch (cache.py:448-465)."""
        if self.cache_kind in ("fp16", "stock"):
            return self._slots[li]
        from .cache import _slots_struct

        c = self.caches[li]
        G, d = self.kv_heads, self.d
        cap = ((rows + 63) // 64) * 64
        sc = getattr(self, "_deq_scratch", None)
        if sc is None or sc[0].shape[2] < cap:
            sc = [torch.zeros((1, G, cap, d), dtype=torch.float16, device=self.device) for _ in range(4)]
            self._deq_scratch = sc
        cap = sc[0].shape[2]
        st = stream(self.device)
        el = 32 // c.bits
        for i, slot in enumerate((c.k1, c.k2, c.v1, c.v2)):
            data, scales, biases = slot
            ccap = data.shape[2]
            for g in range(G):
                check(lib.motif_dequantize(0, c.bits, c.group_size, data.data_ptr() + g * ccap * (d // el) * 4,
                                           scales.data_ptr() + g * ccap * (d // c.group_size) * 2,
                                           biases.data_ptr() + g * ccap * (d // c.group_size) * 2, rows, d,
                                           sc[i].data_ptr() + g * cap * d * 2, st), "dequantize")
        return _slots_struct(sc, 16, 64, 1, G, cap, d)

    def _prefill_block(self, ids_d: torch.Tensor, logits_out: torch.Tensor | None = None) -> None:
        """One block of S rows at positions [offset, offset + S): per layer input norm, qkv linear,
        RoPE + cache append, causal attention over the cache + combine, o_proj (+ residual), post
        norm, gate|up, PolyNorm·up, down (+ residual) — ``MotifDecoderLayer`` (model.py:845-855)
        over the block. Blocks of at least 128 rows run the tcgen05 GEMMs with the residual
        fused; shorter blocks (the speculative verify, prompt tails) run the multi-row q4 GEMV,
        which streams the weights once per 8 rows, and fold the residual into the next norm. With ``logits_out`` (S, V) the final norm and lm_head run
        for every row (model.py:858-905); otherwise only the K/V rows stay (in the cache)."""
        S = ids_d.numel()
        if self.offset + S + 1 > self.max_seq:
            raise ValueError(f"KV capacity {self.max_seq} exhausted by a {S}-row block at {self.offset}")
        with nvtx_range(f"prompt block {S} rows"):
            b = self._launch_block(ids_d, logits_out, device_offset=False)
        self._bump_host(S)
        self.pos_len.copy_(torch.tensor([self.offset, self.offset + 1], dtype=torch.int32))
        if int(b["err"].item()) != 0:
            raise RuntimeError("prompt block: a tensor-core pipeline wait timed out")

    def _launch_block(self, ids_d: torch.Tensor, logits_out: torch.Tensor | None, device_offset: bool) -> dict:
        """The launches of ``_prefill_block``. With ``device_offset`` the rows' positions are read
        from ``pos_len[0]`` at run time (a CUDA graph replayed at every offset; the split attention
        is shaped for the largest offset the capacity allows) and ``pos_len`` advances on the device."""
        S = ids_d.numel()
        off = self.offset
        b = self._block_buffers(S)
        a = self.args
        st = stream(self.device)
        H, d, I = self.H, self.d, self.inter
        eps = a.rms_norm_eps
        h, x, tmp = b["h"][:S], b["x"][:S], b["tmp"][:S]
        qkv, o, attn = b["qkv"][:S], b["o"][:S], b["attn"][:S]
        q = b["q"].view(-1)[: self.q_heads * S * d].view(self.q_heads, S, d)  # head-major, contiguous
        gu, act, err = b["gu"][:S], b["act"][:S], b["err"]
        mode = 1 if self.vanilla else 0
        tp = self.tp_group is not None
        big = S >= self.min_block_rows and self._gemm_ok()
        # one GPU: the GEMM epilogue adds the residual; otherwise the row-parallel partials are
        # all-reduced (tensor parallelism) and the residual is folded into the next norm
        fuse = big and not tp
        split_ws = None
        wsb = lib.motif_prefill_attention_split_workspace_bytes(S, self.q_heads)
        if wsb:
            split_ws = getattr(self, "_split_ws", None)
            if split_ws is None or split_ws.numel() < wsb:
                split_ws = self._split_ws = torch.empty(wsb, dtype=torch.uint8, device=self.device)
                self._row_graphs.clear()
        off_dev = ptr(self.pos_len) if device_offset else None
        attn_off = self.max_seq - S - 1 if device_offset else off  # device offset: the launch's bound

        def lin(xin, ql, out, residual=None):
            if big:
                check(lib.motif_q4_gemm(ptr(xin), S, ql.in_dim, ptr(ql.weight), ptr(ql.scales), ptr(ql.biases),
                                        ql.out_dim, ptr(out), ptr(residual) if residual is not None else None,
                                        ptr(err), st), "q4_gemm")
            else:
                check(lib.motif_quantized_linear(0, 4, 64, ptr(xin), S, ql.in_dim, ptr(ql.weight), ptr(ql.scales),
                                                 ptr(ql.biases), ql.out_dim, ptr(out), ptr(self.lin_ws),
                                                 self.lin_ws.numel(), st), "quantized_linear")

        def norm_after(residual_out, w):
            # fused: the residual was added in the GEMM epilogue; else h += residual_out, then the norm
            if fuse:
                check(lib.motif_rms_norm(0, ptr(h), ptr(w), eps, S, H, ptr(x), st), "rms_norm")
            else:
                check(lib.motif_add_rms_norm(0, ptr(h), ptr(residual_out), ptr(w), eps, S, H, ptr(x), st),
                      "add_rms_norm")

        for li, L in enumerate(self.layers):
            if li == 0:
                check(lib.motif_embed_rms_norm_rows(0, ptr(ids_d), S, ptr(self.embed), self.V, H,
                                                    ptr(L["input_norm"]), eps, ptr(h), ptr(x), st), "embed rows")
            else:
                norm_after(tmp, L["input_norm"])
            lin(x, L["qkv"], qkv)
            check(lib.motif_rope_qkv_append_rows(ptr(qkv), S, ptr(self.inv_freq), self.q_heads, self._slots[li],
                                                 off, off_dev, ptr(q), st), "rope rows")
            slots = self._attn_slots(li, off + S)
            if split_ws is not None:  # a short block over a longer cache: split-KV
                check(lib.motif_prefill_attention_split(ptr(q), S, self.q_heads, slots, attn_off, off_dev, mode,
                                                        self.gr, self.scale, ptr(o), ptr(split_ws), split_ws.numel(),
                                                        ptr(err), st), "prefill_attention")
            else:
                check(lib.motif_prefill_attention(ptr(q), S, self.q_heads, slots, off, mode, self.gr, self.scale,
                                                  ptr(o), ptr(err), st), "prefill_attention")
            check(lib.motif_prefill_post(ptr(o), S, self.q_heads, mode, self.q_groups, self.gr, ptr(L["subln"]),
                                         ptr(L["lambda_full"]), L["lambda_full"].numel(), L["lambda_init"],
                                         a.attn_rms_norm_eps, ptr(attn), st), "prefill_post")
            lin(attn, L["o"], h if fuse else tmp, residual=h if fuse else None)
            if tp:
                self._allreduce(tmp)
            norm_after(tmp, L["post_norm"])
            lin(x, L["gate_up"], gu)
            if tp:  # PolyNorm's means run over the whole intermediate row: sum the ranks' statistics
                stats = b["stats"][:S]
                check(lib.motif_polynorm_row_stats(0, ptr(gu), 2 * I, S, I, ptr(stats), st), "polynorm stats")
                self._allreduce(stats)
                check(lib.motif_polynorm_mul_stats(0, ptr(gu), ptr(gu) + 2 * I, 2 * I, ptr(L["polynorm_w"]),
                                                   ptr(L["polynorm_b"]), 1e-6, S, I, ptr(stats),
                                                   a.intermediate_size, ptr(act), st), "polynorm_mul_stats")
            else:
                check(lib.motif_polynorm_mul(0, ptr(gu), ptr(gu) + 2 * I, 2 * I, ptr(L["polynorm_w"]),
                                             ptr(L["polynorm_b"]), 1e-6, S, I, ptr(act), st), "polynorm_mul")
            lin(act, L["down"], h if fuse else tmp, residual=h if fuse else None)
            if tp:
                self._allreduce(tmp)
        if logits_out is not None:
            norm_after(tmp, self.final_norm)
            ql = self.lm_head
            local = b["logits"][:S] if tp else logits_out  # this rank's vocabulary shard
            check(lib.motif_quantized_linear(0, 4, 64, ptr(x), S, ql.in_dim, ptr(ql.weight), ptr(ql.scales),
                                             ptr(ql.biases), ql.out_dim, ptr(local), ptr(self.lin_ws),
                                             self.lin_ws.numel(), st), "lm_head rows")
            if tp:  # rank r holds vocabulary rows [r·V/tp, (r+1)·V/tp): gather them into (S, V)
                gathered = b["gathered"][: self.tp * S * self.V_local]
                torch.distributed.all_gather_into_tensor(gathered, local.reshape(-1), group=self.tp_group)
                logits_out.view(S, self.tp, self.V_local).copy_(gathered.view(self.tp, S, self.V_local).transpose(0, 1))
        if device_offset:
            self.pos_len.add_(S)
        return b

    def forward_rows(self, ids, logits_out: torch.Tensor | None = None) -> torch.Tensor:
        """Feed a block of tokens at the current position and return their logits (S, V) fp16 (the
        whole vocabulary, gathered from the ranks under tensor parallelism): the batched
        ``[1, S]`` forward of a speculative verify. The cache advances by S."""
        ids_d = torch.as_tensor(ids, dtype=torch.int32).reshape(-1).to(self.device)
        S = ids_d.numel()
        if logits_out is None:
            logits_out = torch.empty((S, self.V_local * self.tp), dtype=torch.float16, device=self.device)
        key = (S, logits_out.data_ptr())
        if not self._rows_graph_ok(S) or key not in self._rows_seen:
            self._rows_seen.add(key)  # the first call runs eagerly (attributes, buffers), the next captures
            self._prefill_block(ids_d, logits_out)
            return logits_out
        if self.offset + S + 1 > self.max_seq:
            raise ValueError(f"KV capacity {self.max_seq} exhausted by a {S}-row block at {self.offset}")
        g = self._row_graphs.get(key)
        if g is None:
            torch.cuda.synchronize(self.device)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                self._launch_block(self._rows_ids[:S], logits_out, device_offset=True)
            self._row_graphs[key] = g
        self._rows_ids[:S].copy_(ids_d)
        g.replay()
        self._bump_host(S)
        return logits_out

    def _rows_graph_ok(self, S: int) -> bool:
        """A row block replays as a CUDA graph when its launches take no host-side offset: an fp16
        cache (a quantized cache is dequantized up to the block's rows) and a short block (the
        multi-row GEMV and split attention path) on one GPU; under tensor parallelism row blocks
        run eagerly. MOTIF_ROWS_GRAPH=0 keeps every call eager."""
        return (self.cache_kind == "fp16" and self.tp_group is None and 1 <= S < min(self.min_block_rows, 129)
                and os.environ.get("MOTIF_ROWS_GRAPH", "1") != "0")

    def check_rows_error(self) -> None:
        """Raise if a graph-replayed row block's pipeline wait timed out (its error word is read
        here, not after every replay)."""
        b = getattr(self, "_blk", None)
        if b is not None and int(b["err"].item()) != 0:
            raise RuntimeError("row block: a tensor-core pipeline wait timed out")

    def ingest(self, ids) -> None:
        """Append tokens to the cache without producing a next token (blocks of ``min_rows_block``
        or more through the prompt path, the rest through the decode step without its head)."""
        ids_d = torch.as_tensor(ids, dtype=torch.int32).reshape(-1).to(self.device)
        n, i = ids_d.numel(), 0
        if self._block_ok():
            while n - i >= self.min_rows_block:
                S = min(2048, n - i)
                self._prefill_block(ids_d[i : i + S])
                i += S
        for j in range(i, n):
            self.token.copy_(ids_d[j : j + 1])
            self.step_device(with_head=False)

    def decode_host(self, token: int) -> int:
        """Public per-token API with host buffers: H2D token, one graph replay, D2H argmax, sync."""
        self.pinned_in[0] = int(token)
        self.token.copy_(self.pinned_in, non_blocking=True)
        self.step_device(with_head=True)
        self.pinned_out.copy_(self.token, non_blocking=True)
        torch.cuda.current_stream(self.device).synchronize()
        return int(self.pinned_out[0])

    def generate(self, prompt_ids, n_tokens: int) -> list[int]:
        """Greedy generation: prefill the prompt, then n_tokens argmax steps (device-resident)."""
        self.prefill(prompt_ids)
        out = [int(self.token.item())]
        toks = []
        for _ in range(n_tokens - 1):
            self.step_device(with_head=True)
            toks.append(self.token.clone())
        out += [int(t.item()) for t in toks]
        return out

    def fill_cache_synthetic(self, n: int, seed: int = 0, std: float = 0.5) -> None:
        """Fill the first n cache rows of every layer with N(0,1)·std keys/values (a stand-in
        for a long prompt's KV; decode cost does not depend on the values) and set the position."""
        if n >= self.max_seq:
            raise ValueError("synthetic fill must leave room to decode")
        gen = torch.Generator(device=self.device)
        gen.manual_seed(seed)
        for c in self.caches:
            if self.cache_kind == "stock":
                for buf in (c.keys, c.values):
                    buf[:, :, :n].copy_((torch.randn((1, 2 * self.kv_heads, n, self.d), generator=gen,
                                                     device=self.device) * std).half())
                continue
            for slot_name in ("k1", "k2", "v1", "v2"):
                rows = torch.randn((1, self.kv_heads, n, self.d), generator=gen, device=self.device) * std
                rows = rows.half()
                slot = getattr(c, slot_name)
                if self.cache_kind == "fp16":
                    slot[:, :, :n].copy_(rows)
                else:
                    dq, sc, bi = quantize(rows, 64, c.bits)
                    slot[0][:, :, :n].copy_(dq)
                    slot[1][:, :, :n].copy_(sc)
                    slot[2][:, :, :n].copy_(bi)
        self.pos_len[0] = n
        self.pos_len[1] = n + 1
        self.offset = n
        for c in self.caches:
            c.offset = n
        self._tp_reset_flags()

    # ------------------------------------------------------------------ #
    @classmethod
    def random(cls, args: ModelArgs, seed: int = 0, std: float = 0.02, cache: str = "fp16", max_seq: int = 4096,
               device="cuda", tp_group=None, rank: int = 0, world: int = 1) -> "MotifDecoder":
        """Random-init weights (std 0.02) generated and quantized (q4, g64) on the GPU.

        With TP, every rank draws the same global tensors layer by layer (same seed)
        and keeps its shard, so the sharded model equals the unsharded one.
        """
        dev = torch.device(device)
        gen = torch.Generator(device=dev)
        gen.manual_seed(seed)
        f16 = torch.float16
        a = args
        H, I, d = a.hidden_size, a.intermediate_size, a.d

        def randn(*shape):
            return (torch.randn(shape, generator=gen, device=dev, dtype=torch.float32) * std).to(f16)

        def qlin(w):
            return QuantizedLinear(*quantize(w, 64, 4))

        def norm_w(n):
            return (1.0 + 0.02 * torch.randn(n, generator=gen, device=dev)).to(f16)

        plan = tp_shard_plan(args, rank, world) if world > 1 else None
        layers = []
        for li in range(a.num_hidden_layers):
            qkv = randn(a.qkv_out, H)
            o = randn(H, a.q_origin * 2 * d)
            gate = randn(I, H)
            up = randn(I, H)
            down = randn(H, I)
            if world > 1:
                qkv = qkv.index_select(0, plan["qkv_rows"].to(dev))
                o = o[:, plan["o_cols"][0]:plan["o_cols"][1]].contiguous()
                r0, r1 = plan["mlp_rows"]
                gate = gate[r0:r1].contiguous()
                up = up[r0:r1].contiguous()
                down = down[:, r0:r1].contiguous()
            lam_init = lambda_init_for_layer(li)
            lp = [torch.randn(d, generator=gen, device=dev) * 0.1 for _ in range(4)]
            layers.append(dict(
                input_norm=norm_w(H), post_norm=norm_w(H),
                qkv=qlin(qkv), o=qlin(o), gate_up=qlin(torch.cat([gate, up])), down=qlin(down),
                subln=norm_w(2 * d), lambda_init=lam_init, lambda_full=lambda_full(*lp, lam_init),
                polynorm_w=torch.full((3,), 1 / 3, dtype=f16, device=dev),
                polynorm_b=torch.zeros(1, dtype=f16, device=dev),
            ))
            del qkv, o, gate, up, down
        embed = randn(a.vocab_size, H)
        final_norm = norm_w(H)
        head = randn(a.vocab_size, H)
        if world > 1:
            head = head[plan["vocab_rows"][0]:plan["vocab_rows"][1]].contiguous()
        weights = dict(embed=embed, final_norm=final_norm, lm_head=qlin(head), layers=layers)
        return cls(args, weights, cache=cache, max_seq=max_seq, device=dev, tp_group=tp_group)


def motif_12_7b_args(**overrides) -> ModelArgs:
    """12.7B-class grouped config of the bench (8 KV heads per slot; see ModelArgs defaults)."""
    return ModelArgs(**overrides)
