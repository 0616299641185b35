"""CPU checks of the oracle itself: the reference's golden vector and the
properties the reference's tests assert (no GPU)."""

from __future__ import annotations

import json
from pathlib import Path

import numpy as np
import pytest

import oracle as O

GOLDEN = Path(__file__).resolve().parent / "golden"


def test_polynorm_golden_vector():
    """Reference fixture component_checks[polynorm_reference_2x3] (expected to 1e-6 there)."""
    case = json.loads((GOLDEN / "polynorm_reference_2x3.json").read_text())
    got = O.polynorm_reference(np.array(case["input"]), case["weight"], case["bias"], case["eps"])
    np.testing.assert_allclose(got, np.array(case["expected"]), atol=1e-12, rtol=0)


def _rand(rng, shape, scale=0.1):
    return (rng.standard_normal(shape) * scale).astype(np.float16)


@pytest.mark.parametrize("bits,tol", [(4, 0.5), (8, 0.05)])
def test_quantize_roundtrip_tolerance(bits, tol):
    """tests/test_grouped_cache.py:111-129 bounds (q4 0.5, q8 0.05)."""
    rng = np.random.default_rng(0)
    x = _rand(rng, (1, 8, 5, 128))
    d, s, b = O.quantize(x, 64, bits)
    assert d.dtype == np.uint32 and d.shape == (1, 8, 5, 128 * bits // 32)
    assert s.shape == b.shape == (1, 8, 5, 2) and s.dtype == np.float16
    y = O.dequantize(d, s, b, 64, bits)
    np.testing.assert_allclose(y.astype(np.float32), x.astype(np.float32), atol=tol, rtol=tol)


@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("gs", [32, 64, 128])
def test_quantize_error_within_one_step(bits, gs):
    """The zero-preserving edge adjustment (scale = edge / q0) can shrink the step so
    the far edge clips by at most one code; everything else is within half a step."""
    rng = np.random.default_rng(1)
    x = rng.standard_normal((7, 256)).astype(np.float32)
    d, s, b = O.quantize(x, gs, bits)
    y = O.dequantize(d, s, b, gs, bits).astype(np.float64)
    step = np.repeat(np.abs(s.astype(np.float64)), gs, axis=-1)
    assert np.all(np.abs(y - x) <= 1.0 * step * (1 + 1e-5) + 1e-6)


def test_quantize_edge_groups():
    """Constant, zero and sign-dominated groups quantize to exact reconstructions of the edge."""
    g = np.zeros((4, 64), np.float16)
    g[1] = 0.75
    g[2] = np.linspace(-2, 0.5, 64)
    g[3] = np.linspace(-0.5, 3, 64)
    d, s, b = O.quantize(g, 64, 4)
    y = O.dequantize(d, s, b, 64, 4).astype(np.float32)
    assert np.all(y[0] == 0)
    assert np.all(y[1] == np.float32(0.75))
    assert y[2].min() == np.float32(-2.0)  # negative edge is the bias: exact
    assert y[3].max() == pytest.approx(3.0, abs=1e-3)  # positive edge: scale < 0, bias = w_max


def test_round_half_away():
    x = np.array([0.5, 1.5, 2.5, -0.5, -1.5, 0.49999997, 2.4999998], np.float32)
    np.testing.assert_array_equal(O.round_half_away(x), np.array([1, 2, 3, -1, -2, 0, 2], np.float32))


@pytest.mark.parametrize("bits", [4, 8])
def test_batched_quantize_equals_per_slot(bits):
    """tests/test_grouped_cache.py:167-210: one batched quantize == four per-slot quantizes."""
    rng = np.random.default_rng(2)
    H, D = 8, 128
    cache = O.OracleGroupedQuantizedKVCache(64, bits)
    steps = [tuple(_rand(rng, (1, H, S, D)) for _ in range(4)) for S in (5, 1, 1, 1)]
    for st in steps:
        live = cache.update_and_fetch_4_quantized(*st)
    o = cache.offset
    assert o == 8
    for i, slot in enumerate(live):
        ref = O.quantize(np.concatenate([st_[i] for st_ in steps], axis=2), 64, bits)
        for comp_ref, comp in zip(ref, slot):
            np.testing.assert_array_equal(comp_ref, comp[..., :o, :])


def test_cache_growth_and_state():
    cache = O.OracleGroupedKVCache()
    cache.step = 4
    rng = np.random.default_rng(3)
    for _ in range(10):
        out = cache.update_and_fetch_4(*(_rand(rng, (1, 2, 1, 32)) for _ in range(4)))
    assert cache.offset == 10 and out[0].shape[2] == 12
    assert all(t.shape[2] == 10 for t in cache.state)
    assert cache.trim(3) == 3 and cache.offset == 7


def test_sdpa_dual_v_reference_properties():
    rng = np.random.default_rng(4)
    q = rng.standard_normal((1, 6, 1, 64))
    k = rng.standard_normal((1, 2, 40, 64))
    v = rng.standard_normal((1, 2, 40, 64))
    out = O.sdpa_dual_v_reference(q, k, v, v, 0.125, kv_len=17)
    np.testing.assert_allclose(out[..., :64], out[..., 64:])
    poisoned = k.copy()
    poisoned[..., 17:, :] = 1e4
    np.testing.assert_allclose(O.sdpa_dual_v_reference(q, poisoned, v, v, 0.125, kv_len=17), out)
    rep = O.sdpa_dual_v_reference(q, np.repeat(k, 3, 1), np.repeat(v, 3, 1), np.repeat(v, 3, 1), 0.125, 17)
    np.testing.assert_allclose(rep, out)


def test_gda_post_merged_equals_split():
    rng = np.random.default_rng(5)
    o = rng.standard_normal((2, 8, 3, 40))
    n = rng.standard_normal((2, 2, 3, 40))
    w = rng.standard_normal(40)
    a = O.gda_post_split_reference(o, n, w, np.array([0.4321]), 0.65, 4, 1e-5)
    b = O.gda_post_reference(np.concatenate([o, n], axis=1), w, np.array([0.4321]), 0.65, 2, 4, 1e-5)
    np.testing.assert_allclose(a, b)
    per_group = O.gda_post_split_reference(o, n, w, np.array([0.4321, 0.4321]), 0.65, 4, 1e-5)
    np.testing.assert_allclose(a, per_group)


@pytest.mark.parametrize("offset", [0, 5])
def test_rope_before_split_equals_after(offset):
    """tests/test_grouped_cache.py:338-369: RoPE is per head, so split order is irrelevant."""
    rng = np.random.default_rng(6)
    k = rng.standard_normal((1, 4, 4, 128)).astype(np.float16)
    full = O.rope(k, offset)
    np.testing.assert_array_equal(full[:, 0::2], O.rope(k[:, 0::2], offset))
    np.testing.assert_array_equal(full[:, 1::2], O.rope(k[:, 1::2], offset))


def test_quantized_matmul_matches_dequantized_product():
    rng = np.random.default_rng(7)
    w = (rng.standard_normal((48, 256)) * 0.02).astype(np.float16)
    tri = O.quantize(w, 64, 4)
    x = rng.standard_normal((3, 256)).astype(np.float16)
    ref = x.astype(np.float64) @ O.dequantize(*tri, 64, 4, out_dtype=np.float64).T
    np.testing.assert_allclose(O.quantized_matmul(x, *tri, 64, 4), ref, rtol=1e-10, atol=1e-10)


def test_origin_first_perm():
    p = O.origin_first_perm(2, 3, 4)
    heads = p.reshape(-1, 4)[:, 0] // 4
    assert list(heads) == [0, 1, 2, 4, 5, 6, 3, 7]


def test_tiny_decoder_oracle_runs_and_is_causal():
    args = O.OracleArgs(hidden_size=128, num_hidden_layers=2, intermediate_size=256, num_noise_heads=2,
                        grouped_ratio=3, kv_heads_per_slot=2, head_dim=128, vocab_size=97)
    w = O.make_synthetic_weights(args, seed=0)
    dec = O.GroupedDecodeOracle(args, w)
    logits0, t0 = dec.step(5)
    logits1, _ = dec.step(t0)
    assert logits0.shape == (97,) and np.isfinite(logits1).all()
    dec2 = O.GroupedDecodeOracle(args, w)
    np.testing.assert_array_equal(dec2.step(5)[0], logits0)
