"""Host-side logic on CPU: ModelArgs validation, the attention-path truth table,
λ helpers, the tensor-parallel shard plan, and a world-size-2 gloo run of the
TP decode algorithm (oracle math, real torch.distributed collectives)."""

from __future__ import annotations

import os

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle as O


def test_model_args_validation():
    from mlx_motif.model import ModelArgs

    a = ModelArgs()
    assert (a.grouped_ratio, a.q_heads, a.q_origin, a.k_noise_heads, a.kv_repeat, a.qkv_out) == (3, 32, 24, 8, 1,
                                                                                                   8192)
    with pytest.raises(ValueError, match="hidden_size must be greater than zero"):
        ModelArgs(hidden_size=0)
    with pytest.raises(ValueError, match="must be an integer"):
        ModelArgs(num_hidden_layers=2.0)
    with pytest.raises(ValueError, match="greater than num_noise_heads"):
        ModelArgs(num_attention_heads=8, num_noise_heads=8)
    with pytest.raises(ValueError, match="divisible by num_noise_heads"):
        ModelArgs(num_attention_heads=30, num_noise_heads=8)
    with pytest.raises(ValueError, match="k_ratio"):
        ModelArgs(k_ratio=0)
    with pytest.raises(ValueError, match=r"divisible by k_ratio \+ 1"):
        ModelArgs(num_key_value_heads=15)
    with pytest.raises(ValueError, match="even"):
        ModelArgs(num_noise_heads=None, num_attention_heads=15, num_key_value_heads=15, head_dim=None,
                  hidden_size=30)
    lit = ModelArgs(num_key_value_heads=8)  # BASELINE's literal "8 KV heads" reading
    assert lit.kv_repeat == 2


_TINY_GROUPED = dict(model_type="motif", hidden_size=64, num_hidden_layers=2, intermediate_size=128,
                     num_attention_heads=10, num_key_value_heads=4, num_noise_heads=2, k_ratio=1, vocab_size=128,
                     max_position_embeddings=64, head_dim=16, tie_word_embeddings=False, hidden_act="poly_norm")
_TINY_VANILLA = dict(model_type="motif", hidden_size=64, num_hidden_layers=2, intermediate_size=128,
                     num_attention_heads=4, num_key_value_heads=4, num_noise_heads=None, vocab_size=128,
                     max_position_embeddings=64, head_dim=16, tie_word_embeddings=True, hidden_act="poly_norm")


@pytest.mark.parametrize("base,overrides,message", [
    (_TINY_GROUPED, {"num_attention_heads": 0}, "num_attention_heads must be greater than zero"),
    (_TINY_GROUPED, {"num_key_value_heads": 0}, "num_key_value_heads must be greater than zero"),
    (_TINY_GROUPED, {"num_noise_heads": 0}, "num_noise_heads must be greater than zero"),
    (_TINY_GROUPED, {"k_ratio": -1}, "k_ratio must be greater than or equal to 1"),
    (_TINY_GROUPED, {"num_key_value_heads": 1, "k_ratio": 1}, r"num_key_value_heads must be at least k_ratio \+ 1"),
    (_TINY_GROUPED, {"num_hidden_layers": -3}, "num_hidden_layers must be greater than zero"),
    (_TINY_GROUPED, {"max_position_embeddings": 0}, "max_position_embeddings must be greater than zero"),
    (_TINY_GROUPED, {"hidden_size": 1, "head_dim": None}, "derived head_dim must be greater than zero"),
    (_TINY_VANILLA, {"num_attention_heads": 3}, "num_attention_heads must be even"),
    (_TINY_VANILLA, {"num_key_value_heads": 3}, "num_key_value_heads must be even"),
    (_TINY_VANILLA, {"num_attention_heads": 6, "num_key_value_heads": 4},
     "num_attention_heads must be divisible by num_key_value_heads"),
    (_TINY_VANILLA, {"head_dim": 8}, r"head_dim \* num_attention_heads must equal hidden_size"),
    (_TINY_GROUPED, {"num_attention_heads": 9}, "num_attention_heads must be divisible by num_noise_heads"),
    (_TINY_GROUPED, {"num_key_value_heads": 5}, r"num_key_value_heads must be divisible by k_ratio \+ 1"),
    (_TINY_GROUPED, {"hidden_size": 65, "head_dim": None}, "hidden_size must be divisible by num_attention_heads"),
    (_TINY_GROUPED, {"k_ratio": 3, "num_key_value_heads": 8}, "grouped attention ratio must be divisible by k_ratio"),
])
def test_model_args_rejections_carry_the_reference_messages(base, overrides, message):
    """The structural and head-topology rejections of the reference's tests/test_model.py:72-139,
    with the message fragments its tests match."""
    from mlx_motif.model import ModelArgs

    with pytest.raises(ValueError, match=message):
        ModelArgs(**dict(base, **overrides))


def test_resolve_attention_path_truth_table():
    from mlx_motif.cache import MotifGroupedKVCache, MotifGroupedQuantizedKVCache
    from mlx_motif.model import AttnPath, _resolve_attention_path

    q, f = MotifGroupedQuantizedKVCache(64, 4), MotifGroupedKVCache()
    R = _resolve_attention_path
    assert R(q, 1, 1, 1, False, env={}) is AttnPath.QUANT_SDPA
    assert R(q, 1, 1, 1, False, env={"MLX_MOTIF_QUANT_SDPA": "0"}) is AttnPath.DUAL_V
    assert R(q, 1, 1, 1, False, env={"MLX_MOTIF_QUANT_SDPA": "0", "MLX_MOTIF_DUAL_V": "false"}) is AttnPath.FALLBACK
    assert R(f, 1, 1, 1, False, env={}) is AttnPath.DUAL_V
    assert R(f, 5, 1, 1, False, env={}) is AttnPath.FALLBACK
    assert R(f, 1, 2, 1, False, env={}) is AttnPath.FALLBACK
    assert R(q, 1, 1, 2, False, env={}) is AttnPath.FALLBACK
    assert R(q, 1, 1, 1, True, env={}) is AttnPath.FALLBACK
    assert R(None, 1, 1, 1, False, env={}) is AttnPath.DUAL_V


def test_make_cache_env_routing():
    """MLX_MOTIF_4SLOT_CACHE picks the cache as the reference's Model.make_cache does
    (model.py:922-991): 4-slot fp16 by default, q4/q8 packed, the stock cache when off; a vanilla
    model always gets the slab-ordered cache; k_ratio > 1 raises on an explicit request and quietly
    takes the stock cache otherwise."""
    from mlx_motif.cache import KVCache, MotifGroupedKVCache, MotifGroupedQuantizedKVCache, MotifVanillaKVCache
    from mlx_motif.model import ModelArgs, cache_kind, make_cache

    g = ModelArgs(num_hidden_layers=3)
    cases = {None: (MotifGroupedKVCache, "fp16"), "1": (MotifGroupedKVCache, "fp16"),
             "true": (MotifGroupedKVCache, "fp16"), "q4": (MotifGroupedQuantizedKVCache, "q4"),
             "4": (MotifGroupedQuantizedKVCache, "q4"), "Q8": (MotifGroupedQuantizedKVCache, "q8"),
             "8": (MotifGroupedQuantizedKVCache, "q8"), "0": (KVCache, "stock"), "": (KVCache, "stock"),
             "false": (KVCache, "stock"), "OFF": (KVCache, "stock")}
    for val, (cls, kind) in cases.items():
        env = {} if val is None else {"MLX_MOTIF_4SLOT_CACHE": val}
        caches = make_cache(g, env=env)
        assert len(caches) == 3 and all(type(c) is cls for c in caches), val
        assert cache_kind(caches[0]) == kind
        if kind in ("q4", "q8"):
            assert caches[0].group_size == 64 and caches[0].bits == int(kind[1])
    v = ModelArgs(hidden_size=2048, num_hidden_layers=2, intermediate_size=8192, num_attention_heads=16,
                  num_key_value_heads=4, num_noise_heads=None)
    for val in (None, "q4", "0"):
        env = {} if val is None else {"MLX_MOTIF_4SLOT_CACHE": val}
        assert all(type(c) is MotifVanillaKVCache for c in make_cache(v, env=env))
    kr2 = ModelArgs(num_attention_heads=40, num_key_value_heads=24, num_noise_heads=8, k_ratio=2)
    assert all(type(c) is KVCache for c in make_cache(kr2, env={}))
    for val in ("1", "q4", "q8"):
        with pytest.raises(ValueError, match="not supported with k_ratio > 1"):
            make_cache(kr2, env={"MLX_MOTIF_4SLOT_CACHE": val})
    assert all(type(c) is KVCache for c in make_cache(kr2, env={"MLX_MOTIF_4SLOT_CACHE": "0"}))


def test_decode_attention_mode_follows_the_resolved_path():
    """The decoder's attention launches per resolved path: one fused launch for QUANT_SDPA and
    for DUAL_V on fp16 rows; the dequant bridge for DUAL_V/FALLBACK on a packed cache; RoPE/append
    + split attention for FALLBACK on fp16 rows."""
    from mlx_motif.cache import KVCache, MotifGroupedKVCache, MotifGroupedQuantizedKVCache
    from mlx_motif.model import AttnPath, ModelArgs, decode_attention_mode

    a = ModelArgs(num_hidden_layers=1)
    q, f, s = MotifGroupedQuantizedKVCache(64, 4), MotifGroupedKVCache(), KVCache()
    M = decode_attention_mode
    assert M(a, q, env={}) == (AttnPath.QUANT_SDPA, "fused")
    assert M(a, q, env={"MLX_MOTIF_QUANT_SDPA": "0"}) == (AttnPath.DUAL_V, "bridge")
    assert M(a, q, env={"MLX_MOTIF_QUANT_SDPA": "0", "MLX_MOTIF_DUAL_V": "0"}) == (AttnPath.FALLBACK, "bridge")
    assert M(a, q, env={"MLX_MOTIF_DUAL_V": "0"}) == (AttnPath.QUANT_SDPA, "fused")
    for c in (f, s):
        assert M(a, c, env={}) == (AttnPath.DUAL_V, "fused")
        assert M(a, c, env={"MLX_MOTIF_DUAL_V": "False"}) == (AttnPath.FALLBACK, "two_call")
        assert M(a, c, env={"MOTIF_FUSED_ATTN": "0"}) == (AttnPath.DUAL_V, "two_call")
    assert M(ModelArgs(num_hidden_layers=1, fused_rope=True), f, env={}) == (AttnPath.FALLBACK, "two_call")


def test_lambda_helpers_match_oracle():
    from mlx_motif.model import lambda_full, lambda_init_for_layer, origin_first_perm

    for li in (0, 1, 7, 47):
        assert lambda_init_for_layer(li) == O.lambda_init_for_layer(li)
    rng = np.random.default_rng(0)
    lp = [rng.standard_normal(128).astype(np.float32) * 0.1 for _ in range(4)]
    got = lambda_full(*(torch.from_numpy(x) for x in lp), 0.65)
    np.testing.assert_allclose(got.numpy(), O.lambda_full(*lp, 0.65), rtol=1e-6)
    np.testing.assert_array_equal(origin_first_perm(8, 3, 128).numpy(), O.origin_first_perm(8, 3, 128))


@pytest.mark.parametrize("world", [2, 4, 8])
def test_tp_shard_plan_matches_oracle_sharding(world):
    from mlx_motif.model import ModelArgs, tp_shard_plan

    oa = O.OracleArgs(hidden_size=128, num_hidden_layers=1, intermediate_size=512, vocab_size=64)
    ma = ModelArgs(hidden_size=128, num_hidden_layers=1, intermediate_size=512, vocab_size=64)
    w = O.make_synthetic_weights(oa, seed=0)
    for rank in range(world):
        sh = O.shard_weights_tp(oa, w, rank, world)["layers"][0]
        plan = tp_shard_plan(ma, rank, world)
        L = w["layers"][0]
        np.testing.assert_array_equal(L["qkv"][0][plan["qkv_rows"].numpy()], sh["qkv"][0])
        c0, c1 = plan["o_cols"]
        np.testing.assert_array_equal(L["o"][0][:, c0 // 8:c1 // 8], sh["o"][0])
        r0, r1 = plan["mlp_rows"]
        np.testing.assert_array_equal(L["gate"][0][r0:r1], sh["gate"][0])
        np.testing.assert_array_equal(L["down"][1][:, r0 // 64:r1 // 64], sh["down"][1])
        v0, v1 = plan["vocab_rows"]
        assert (v0, v1) == (rank * 64 // world, (rank + 1) * 64 // world)


# ---------------------------------------------------------------- gloo TP decode
def _tp_layer(args, L, h, cache, rank, world, inv_freq):
    """One decode layer on this rank's shard; all-reduces where the engine does."""
    f16 = np.float16
    d, gr = args.head_dim, args.grouped_ratio
    G = args.num_noise_heads // world
    Hk = args.kv_heads_per_slot // world
    lin = lambda x, t: O.quantized_matmul(x, *t, 64, 4).astype(f16)  # noqa: E731
    x = O.rms_norm(h, L["input_norm"]).astype(f16)
    qkv = lin(x, L["qkv"])
    qd, kd = G * (gr + 1) * d, 2 * Hk * d
    q = qkv[..., :qd].reshape(1, 1, -1, d).transpose(0, 2, 1, 3)
    k = qkv[..., qd:qd + kd].reshape(1, 1, -1, d).transpose(0, 2, 1, 3)
    v = qkv[..., qd + kd:].reshape(1, 1, -1, d).transpose(0, 2, 1, 3)
    off = cache.offset
    q = O.rope(q, off, inv_freq=inv_freq).astype(f16)
    k = O.rope(k, off, inv_freq=inv_freq).astype(f16)
    K1, K2, V1, V2 = cache.update_and_fetch_4(k[:, 0::2], k[:, 1::2], v[:, 0::2], v[:, 1::2])
    n = cache.offset
    ao = O.sdpa_dual_v_reference(q[:, :G * gr], K1, V1, V2, d ** -0.5, n).astype(f16)
    an = O.sdpa_dual_v_reference(q[:, G * gr:], K2, V1, V2, d ** -0.5, n).astype(f16)
    out = O.gda_post_split_reference(ao, an, L["subln"], L["lambda_full"], L["lambda_init"], gr).astype(f16)
    o = torch.from_numpy(O.quantized_matmul(out.transpose(0, 2, 1, 3).reshape(1, -1), *L["o"], 64, 4))
    dist.all_reduce(o)  # row-parallel o_proj
    h = (h.astype(np.float32) + o.numpy().astype(f16).astype(np.float32)).astype(f16)
    x2 = O.rms_norm(h, L["post_norm"]).astype(f16)
    g = lin(x2, L["gate"]).astype(np.float64)
    u = lin(x2, L["up"])
    g2 = g * g
    stats = torch.tensor([g2.sum(), (g2 * g2).sum(), (g2 ** 3).sum()], dtype=torch.float64)
    dist.all_reduce(stats)  # PolyNorm statistics over the full intermediate row
    r2, r4, r6 = (1.0 / np.sqrt(stats.numpy() / args.intermediate_size + 1e-6))
    w = L["polynorm_w"].astype(np.float64)
    act = (w[0] * g2 * g * r6 + w[1] * g2 * r4 + w[2] * g * r2).astype(f16)
    act = (act.astype(np.float64) * u.astype(np.float64)).astype(f16)
    dn = torch.from_numpy(O.quantized_matmul(act, *L["down"], 64, 4))
    dist.all_reduce(dn)  # row-parallel down_proj
    return (h.astype(np.float32) + dn.numpy().astype(f16).astype(np.float32)).astype(f16)


def _tp_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        args = O.OracleArgs(hidden_size=128, num_hidden_layers=2, intermediate_size=256, num_noise_heads=8,
                            grouped_ratio=3, kv_heads_per_slot=8, head_dim=128, vocab_size=64)
        w = O.shard_weights_tp(args, O.make_synthetic_weights(args, seed=3, std=0.05), rank, world)
        caches = [O.OracleGroupedKVCache() for _ in range(args.num_hidden_layers)]
        inv = O.rope_inv_freq(128)
        logits_seq = []
        for tok in (1, 7, 9):
            h = w["embed"][tok][None, :].astype(np.float16)
            for li, L in enumerate(w["layers"]):
                h = _tp_layer(args, L, h, caches[li], rank, world, inv)
            hn = O.rms_norm(h, w["final_norm"]).astype(np.float16)
            logits_seq.append(O.quantized_matmul(hn, *w["lm_head"], 64, 4).astype(np.float16)[0])
        if rank == 0:
            q.put(np.stack(logits_seq))
    finally:
        dist.destroy_process_group()


def test_tp2_gloo_decode_equals_single_rank():
    """Sharded decode over 2 gloo ranks (all-reduce after o_proj, down_proj and of the
    PolyNorm statistics) reproduces the unsharded oracle decode."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29500 + (os.getpid() % 1000)
    procs = [ctx.Process(target=_tp_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    tp_logits = q.get(timeout=240)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    args = O.OracleArgs(hidden_size=128, num_hidden_layers=2, intermediate_size=256, num_noise_heads=8,
                        grouped_ratio=3, kv_heads_per_slot=8, head_dim=128, vocab_size=64)
    ref = O.GroupedDecodeOracle(args, O.make_synthetic_weights(args, seed=3, std=0.05))
    for i, tok in enumerate((1, 7, 9)):
        logits, _ = ref.step(tok)
        np.testing.assert_allclose(tp_logits[i].astype(np.float32), logits.astype(np.float32), atol=2e-2, rtol=2e-2)


# ---------------------------------------------------------------- vocabulary-parallel argmax
def _argmax_key(v: np.ndarray, row0: int) -> np.ndarray:
    """The packed key of the lm_head epilogue (argmax_key_out): order-preserving fp32 bits of the
    fp16 value (NaN as -inf) above the inverted global row, top bit flipped for int64 order."""
    f = v.astype(np.float32).copy()
    f[np.isnan(f)] = -np.inf
    b = f.view(np.uint32).astype(np.uint64)
    hi = np.where(b & 0x80000000, ~b & 0xFFFFFFFF, b | 0x80000000)
    rows = np.arange(row0, row0 + len(v), dtype=np.uint64)
    key = (hi << np.uint64(32)) | (np.uint64(0xFFFFFFFF) - rows)
    return (key ^ np.uint64(1 << 63)).view(np.int64)


def _key_worker(rank, world, port, logits, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        n = len(logits) // world
        k = torch.tensor([_argmax_key(logits[rank * n:(rank + 1) * n], rank * n).max()])
        dist.all_reduce(k, op=dist.ReduceOp.MAX)
        u = int(k.item()) ^ (1 << 63) if int(k.item()) >= 0 else (int(k.item()) + (1 << 64)) ^ (1 << 63)
        q.put(0 if u == 0 else 0xFFFFFFFF - (u & 0xFFFFFFFF))
    finally:
        dist.destroy_process_group()


def test_vocab_parallel_argmax_keys_over_gloo():
    """Shard keys combined by an int64 MAX all-reduce give the first index of the global maximum,
    with NaN ranked below everything (ties across shards and inside one shard)."""
    rng = np.random.default_rng(11)
    logits = rng.standard_normal(64).astype(np.float16)
    logits[[9, 40, 41]] = np.float16(3.5)  # tie across shards and within shard 1: index 9 wins
    logits[[2, 50]] = np.float16("nan")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 30500 + (os.getpid() % 500)
    procs = [ctx.Process(target=_key_worker, args=(r, 2, port, logits, q)) for r in range(2)]
    for p in procs:
        p.start()
    toks = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert toks == [9, 9]


def test_nvtx_ranges_follow_the_env_switch(monkeypatch):
    """MOTIF_NVTX off: the decoder's op ranges are no-op contexts; on: each opens an NVTX range
    with its name (the launches inside are the same either way)."""
    import contextlib

    import mlx_motif.model as M

    monkeypatch.setattr(M, "_NVTX", False)
    assert isinstance(M.nvtx_range("qkv"), contextlib.nullcontext)
    opened = []

    def fake_range(name):
        opened.append(name)
        return contextlib.nullcontext()

    monkeypatch.setattr(M, "_NVTX", True)
    monkeypatch.setattr(torch.cuda.nvtx, "range", fake_range)
    with M.nvtx_range("layer 0"):
        with M.nvtx_range("qkv"):
            pass
    assert opened == ["layer 0", "qkv"]


def test_key_exchange_packing_keeps_the_token():
    """The packing motif_argmax_key_exchange applies to each rank's key — value bits above a step
    number (bits 24..31) above 2^24 - 1 - row — keeps the largest key's token: over random
    vocabulary shards, ties across shards included, the largest packed key decodes to the row
    the plain keys' MAX names."""
    import struct

    def key_of(val, row):
        b = struct.unpack("<I", struct.pack("<f", val))[0]
        hi = (~b & 0xFFFFFFFF) if (b & 0x80000000) else (b | 0x80000000)
        return (hi << 32) | (0xFFFFFFFF - row)

    def pack(k, number):
        row = 0xFFFFFFFF - (k & 0xFFFFFFFF)
        return (k & 0xFFFFFFFF00000000) | (number << 24) | (0xFFFFFF - row)

    rng = np.random.default_rng(3)
    for _ in range(3000):
        world = int(rng.integers(1, 9))
        vocab = int(rng.integers(world, 219521))
        shard = vocab // world
        vals = np.round(rng.normal(0, 3, world), int(rng.integers(1, 7))).astype(np.float32).tolist()
        if rng.random() < 0.3:
            vals = [vals[0]] * world
        rows = [r * shard + int(rng.integers(0, shard)) for r in range(world)]
        keys = [key_of(v, w) for v, w in zip(vals, rows)]
        want = 0xFFFFFFFF - (max(keys) & 0xFFFFFFFF)
        number = int(rng.integers(1, 256))
        assert 0xFFFFFF - (max(pack(k, number) for k in keys) & 0xFFFFFF) == want


def test_reference_config_fixtures_construct_model_args():
    """The reference's own tiny config fixtures (copied by tests/golden/make_golden.py) build
    ModelArgs — every field of its config, activation and bias included — with the shape
    expectations its parity-fixture test checks (tests/test_swift_parity_fixtures.py:24-44), and
    ModelArgs.from_dict gives the same arguments."""
    import json
    from pathlib import Path

    from mlx_motif.model import ModelArgs

    cases = json.loads((Path(__file__).parent / "golden" / "model_configs.json").read_text())["configs"]
    assert len(cases) == 2
    for case in cases:
        args = ModelArgs(**case["python"])
        want = case["expectations"]
        assert args.is_grouped is want["is_grouped"]
        assert (args.head_dim or args.hidden_size // args.num_attention_heads) == want["effective_head_dim"]
        if args.is_grouped:
            assert args.num_attention_heads // args.num_noise_heads == want["origin_heads_per_noise_head"]
            assert args.num_key_value_heads // args.num_noise_heads == want["kv_heads_per_group"]
        assert ModelArgs.from_dict(dict(case["python"], unknown_key=1)) == args


@pytest.mark.parametrize("field,value", [("hidden_act", "silu"), ("use_bias", True),
                                         ("rope_scaling", {"type": "linear", "factor": 2.0}),
                                         ("use_sliding_window", True)])
def test_decoder_rejects_config_values_it_does_not_implement(field, value):
    """ModelArgs takes every reference config field; the decoder names the ones whose values its
    decode path does not implement instead of running something else."""
    from mlx_motif.model import ModelArgs, MotifDecoder

    with pytest.raises(ValueError, match=field):
        MotifDecoder(ModelArgs(**{field: value}), {}, device="cpu")


def test_make_mask_follows_the_mlx_lm_contract():
    """cache.make_mask(N, return_array=..., window_size=...) as mlx-lm calls it (the reference's
    tests/test_grouped_cache.py:16-45): None for one query, "causal" for several, an explicit
    (N, offset + N) boolean mask on request, and a sliding window that keeps the last
    window_size keys of every query."""
    from mlx_motif.cache import KVCache, MotifGroupedKVCache, MotifGroupedQuantizedKVCache

    cache = MotifGroupedKVCache()
    cache.offset = 3
    assert cache.make_mask(1, return_array=False, window_size=None) is None
    assert cache.make_mask(4, return_array=False, window_size=None) == "causal"
    mask = cache.make_mask(4, return_array=True, window_size=None)
    assert tuple(mask.shape) == (4, 7)
    q = torch.arange(4)[:, None] + 3
    k = torch.arange(7)[None, :]
    assert torch.equal(mask, k <= q)
    assert torch.equal(cache.make_mask(4, return_array=True, window_size=2), (k <= q) & (k > q - 2))
    qcache = MotifGroupedQuantizedKVCache(group_size=64, bits=8)
    qcache.offset = 2
    assert qcache.make_mask(1, return_array=False, window_size=None) is None
    assert qcache.make_mask(5, return_array=False, window_size=None) == "causal"
    stock = KVCache()
    stock.offset = 2
    assert tuple(stock.make_mask(3, return_array=True, window_size=None).shape) == (3, 5)
