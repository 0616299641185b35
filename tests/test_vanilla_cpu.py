"""CPU checks of the vanilla (2.6B-class) path's host side and oracle: the V head-order
permutations and ``MotifVanillaKVCache``'s state/marker rules (the behaviour of the
reference's ``tests/test_vanilla_slab_cache.py``), the vanilla ModelArgs dims, and the
oracle's slab-ordered attention against a paired-order restatement."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle as O


@pytest.mark.parametrize("hk", [1, 2, 4, 8])
def test_perms_round_trip_and_match_oracle(hk):
    from mlx_motif.cache import vanilla_v_paired_to_slab_perm, vanilla_v_slab_to_paired_perm

    p, inv = vanilla_v_paired_to_slab_perm(hk), vanilla_v_slab_to_paired_perm(hk)
    assert p[inv].tolist() == list(range(2 * hk)) and inv[p].tolist() == list(range(2 * hk))
    assert p.tolist() == O.vanilla_v_paired_to_slab_perm(hk).tolist()
    assert inv.tolist() == O.vanilla_v_slab_to_paired_perm(hk).tolist()
    # the model's reorder (reshape(B, Hk, 2, S, d), slot-major transpose) is the same permutation
    B, S, d = 2, 3, 8
    paired = torch.randn(B, 2 * hk, S, d)
    slab_ref = paired.reshape(B, hk, 2, S, d).transpose(1, 2).reshape(B, 2 * hk, S, d)
    assert torch.equal(paired[:, p], slab_ref)


def _cache_from(keys, values, **kw):
    from mlx_motif.cache import MotifVanillaKVCache

    return MotifVanillaKVCache.from_state((keys, values), ("slab",), **kw)


def test_vanilla_cache_state_views_and_markers():
    from mlx_motif.cache import MotifVanillaKVCache, vanilla_v_paired_to_slab_perm

    B, hk, S, d = 1, 3, 5, 16
    paired = torch.arange(B * 2 * hk * S * d, dtype=torch.float32).reshape(B, 2 * hk, S, d)
    slab = paired[:, vanilla_v_paired_to_slab_perm(hk)]
    keys = torch.randn(B, 2 * hk, S, d)
    c = _cache_from(keys, slab, max_size=32)
    assert c.offset == S and c.meta_state == ("slab",)
    assert torch.equal(c.keys, keys) and torch.equal(c.values, slab)
    assert torch.equal(c.hf_ordered_values(), paired)
    # device form: k1/k2 = even/odd k heads, v1/v2 = the two slabs, capacity preallocated in
    # whole 256-row steps
    assert c.k1.shape == (B, hk, 256, d)
    assert torch.equal(c.k1[:, :, :S], keys[:, 0::2]) and torch.equal(c.k2[:, :, :S], keys[:, 1::2])
    assert torch.equal(c.v1[:, :, :S], slab[:, :hk]) and torch.equal(c.v2[:, :, :S], slab[:, hk:])
    # the oracle cache gives the same HF view
    oc = O.OracleVanillaKVCache()
    oc.update_and_fetch(keys.numpy(), slab.numpy())
    assert np.array_equal(oc.hf_ordered_values(), paired.numpy())
    c.trim(2)
    assert c.offset == S - 2 and c.keys.shape[2] == S - 2
    for bad in (("paired",), ("hf",)):
        with pytest.raises(ValueError, match="V head-order marker mismatch"):
            MotifVanillaKVCache.from_state((keys, slab), bad)
    for bad in ((), ""):
        with pytest.raises(ValueError, match="no V head-order marker"):
            MotifVanillaKVCache.from_state((keys, slab), bad)
    assert MotifVanillaKVCache().hf_ordered_values() is None


def test_vanilla_model_args_dims():
    """config[3] (2.6B-class): 16 q heads -> H = 8 differential heads, 4 kv heads -> Hk = 2,
    n_rep 4, fused qkv rows (16 + 4 + 4)·128, attention output H·2d = hidden."""
    from mlx_motif.model import ModelArgs

    a = ModelArgs(hidden_size=2048, num_hidden_layers=32, intermediate_size=8192, num_attention_heads=16,
                  num_key_value_heads=4, num_noise_heads=None)
    assert not a.is_grouped
    assert (a.q_heads, a.q_origin, a.k_noise_heads, a.grouped_ratio, a.kv_repeat) == (16, 8, 2, 4, 1)
    assert a.qkv_out == 3072 == O.OracleVanillaArgs().qkv_out
    assert a.q_origin * 2 * a.d == a.hidden_size
    with pytest.raises(ValueError, match="even"):
        ModelArgs(hidden_size=384, num_attention_heads=3, num_key_value_heads=2, num_noise_heads=None)


def test_vanilla_oracle_matches_paired_restatement():
    """The slab-ordered oracle attention equals a direct paired-order computation: pair i of
    kv group g = i // n_rep attends q1_i over k1_g and q2_i over k2_g, each against the value
    pair [v_2g | v_2g+1] (the projection's paired heads), then (o1 - λ·o2) · SubLN · (1 - λ_init)."""
    rng = np.random.default_rng(0)
    hk, n_rep, d, n = 2, 4, 16, 9
    H = hk * n_rep
    f16 = np.float16
    q = rng.standard_normal((1, 2 * H, 1, d)).astype(f16)
    k = rng.standard_normal((1, 2 * hk, n, d)).astype(f16)
    v = rng.standard_normal((1, 2 * hk, n, d)).astype(f16)  # paired order
    sub = (1 + 0.02 * rng.standard_normal(2 * d)).astype(f16)
    lam, lam_init = np.array([0.3], np.float32), 0.5
    got = O.vanilla_attention_reference(q, k, v, O.OracleVanillaKVCache(), lam, lam_init, sub)
    want = np.zeros((1, H, 1, 2 * d))
    qf, kf, vf = (x.astype(np.float64) for x in (q, k, v))
    for i in range(H):
        g = i // n_rep
        vp = np.concatenate([vf[0, 2 * g], vf[0, 2 * g + 1]], axis=-1)  # (n, 2d)

        def att(qh, kh):
            s = (qh @ kh.T) * d ** -0.5
            p = np.exp(s - s.max())
            return (p / p.sum()) @ vp

        o1, o2 = att(qf[0, 2 * i], kf[0, 2 * g]), att(qf[0, 2 * i + 1], kf[0, 2 * g + 1])
        diff = o1 - 0.3 * o2
        y = diff / np.sqrt(np.mean(diff * diff) + 1e-5) * sub.astype(np.float64)
        want[0, i] = y * (1 - lam_init)
    np.testing.assert_allclose(got.astype(np.float64), want, atol=2e-2, rtol=2e-2)


def test_vanilla_decode_oracle_is_deterministic():
    a = O.OracleVanillaArgs(hidden_size=256, num_hidden_layers=2, intermediate_size=256, num_attention_heads=2,
                            num_key_value_heads=2, head_dim=128, vocab_size=300)
    w = O.make_synthetic_weights_vanilla(a, seed=1)
    t1 = [O.VanillaDecodeOracle(a, w).step(5)[1] for _ in range(2)]
    assert t1[0] == t1[1]
    orc = O.VanillaDecodeOracle(a, w)
    for t in (5, 6, 7):
        orc.step(t)
    assert all(c.offset == 3 for c in orc.caches)
    assert orc.caches[0].values.shape == (1, 2, 3, 128)
