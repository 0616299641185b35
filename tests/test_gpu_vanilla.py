"""GPU parity of the vanilla (2.6B-class, ungrouped differential attention) decode path:
the one-launch attention step against the oracle's ``_forward_vanilla`` restatement
(``model.py:486-559``), its cache writes against the two-call RoPE/append kernel, the
``MotifVanillaKVCache`` API (``cache.py:85-175``, the behaviour ``tests/test_vanilla_slab_cache.py``
checks) and greedy decode of a small vanilla model."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle as O
from conftest import assert_close
from test_gpu_kernels import down, rounded, up

pytestmark = pytest.mark.gpu


def _make_cache(kind, Hk, hist, cap, dev):
    from mlx_motif.cache import MotifGroupedKVCache, MotifGroupedQuantizedKVCache

    pos = hist[0].shape[2]
    if kind == "fp16":
        c = MotifGroupedKVCache(max_size=cap)
        if pos:
            c.update_and_fetch_4(*(up(h) for h in hist))
    else:
        c = MotifGroupedQuantizedKVCache(64, 4 if kind == "q4" else 8, max_size=cap)
        if pos:
            c.update_and_fetch_4_quantized(*(up(h) for h in hist))
    if not pos:
        c._grow(1, Hk, 1, 128, torch.float16, dev)
    return c


def _slot_rows(cache, kind, n):
    """The first n rows of the four slots as float arrays (dequantized in fp32 for q4/q8)."""
    out = []
    for slot in (cache.k1, cache.k2, cache.v1, cache.v2):
        if kind == "fp16":
            out.append(down(slot[..., :n, :]))
        else:
            d, s, b = (x[..., :n, :].cpu() for x in slot)
            out.append(O.dequantize(d.numpy().view(np.uint32), s.float().numpy(), b.float().numpy(), 64,
                                    cache.bits, out_dtype=np.float32))
    return out


CASES = [("fp16", n_rep, kv) for n_rep in (1, 2, 4) for kv in (1, 37, 3000)]
CASES += [("q4", 4, 200), ("q8", 4, 200), ("q4", 2, 3000), ("fp16", 4, 200)]


@pytest.mark.parametrize("kind,n_rep,kv_len", CASES)
def test_vanilla_decode_step_matches_oracle(cuda, kind, n_rep, kv_len):
    """motif_vanilla_decode_step == oracle RoPE, slab-ordered cache append, four SDPAs,
    (o1 - λ·o2), SubLN and the (1 - λ_init) scale; its cache writes equal the two-call
    RoPE/append kernel's bit for bit; a repeated launch gives the same output."""
    from mlx_motif import _native as N
    from mlx_motif.model import rope_inv_freq

    rng = np.random.default_rng(7 * kv_len + n_rep)
    Hk, d, cap = 2, 128, 4096
    H = Hk * n_rep
    pos = kv_len - 1
    hist = [rounded(rng.standard_normal((1, Hk, pos, d)) * 0.5, "float16") for _ in range(4)]
    qkv = rounded(rng.standard_normal((2 * H + 4 * Hk) * d), "float16")
    ca, cb = _make_cache(kind, Hk, hist, cap, cuda), _make_cache(kind, Hk, hist, cap, cuda)
    inv = rope_inv_freq(d, 10000.0, cuda)
    pos_t = torch.tensor([pos, kv_len], dtype=torch.int32, device=cuda)
    subln = rounded(1 + 0.02 * rng.standard_normal(2 * d), "float16")
    lam, lam_init = np.array([0.41], np.float32), 0.35
    tq, t_sub, t_lam = up(qkv), up(subln), torch.tensor(lam, device=cuda)
    wsb = N.lib.motif_gda_decode_step_workspace_bytes(2 * H, d, 64)
    ws = torch.zeros(wsb, dtype=torch.uint8, device=cuda)
    outs = []
    for _ in range(2):
        out = torch.full((H * 2 * d,), float("nan"), dtype=torch.float16, device=cuda)
        N.check(N.lib.motif_vanilla_decode_step(tq.data_ptr(), inv.data_ptr(), ca.slots_struct(), pos_t.data_ptr(),
                                                d ** -0.5, Hk, n_rep, t_sub.data_ptr(), t_lam.data_ptr(), lam_init,
                                                1e-5, out.data_ptr(), ws.data_ptr(), wsb, N.stream()),
                "vanilla_decode_step")
        torch.cuda.synchronize()
        outs.append(out)
    assert torch.equal(outs[0], outs[1]), "repeated step differs (counters not reset?)"
    assert torch.equal(ws[:256], torch.zeros(256, dtype=torch.uint8, device=cuda))
    # the same layout through the two-call RoPE/append kernel: identical cache rows
    q_out = torch.empty(2 * H * d, dtype=torch.float16, device=cuda)
    N.check(N.lib.motif_rope_qkv_append(tq.data_ptr(), inv.data_ptr(), 2 * H, cb.slots_struct(), pos_t.data_ptr(),
                                        q_out.data_ptr(), N.stream()))
    torch.cuda.synchronize()
    for n in ("k1", "k2", "v1", "v2"):
        a, b = getattr(ca, n), getattr(cb, n)
        for x, y in (zip(a, b) if isinstance(a, tuple) else [(a, b)]):
            assert torch.equal(x[..., :kv_len, :], y[..., :kv_len, :]), f"cache slot {n} differs"
    # ---- oracle, on the kernel's own stored rows (the new row included)
    k1, k2, va, vb = _slot_rows(ca, kind, kv_len)
    K = np.stack([k1, k2], axis=2).reshape(1, 2 * Hk, kv_len, d)  # stripe order
    V_paired = np.concatenate([va, vb], axis=1)[:, O.vanilla_v_slab_to_paired_perm(Hk)]
    q = qkv[: 2 * H * d].reshape(1, 2 * H, 1, d)
    qr = O.rope(q, pos).astype(np.float16)
    assert_close(down(q_out).reshape(qr.shape), qr, "float16", what="roped q")
    kv_dtype = np.float16 if kind == "fp16" else np.float32
    ref = O.vanilla_attention_reference(qr, K, V_paired, O.OracleVanillaKVCache(), lam, lam_init, subln, 1e-5,
                                        kv_dtype=kv_dtype)
    assert_close(down(outs[0]), ref.reshape(-1).astype(np.float64), "float16", what="vanilla attention step")


def test_vanilla_decode_step_rejects_bad_contract(cuda):
    from mlx_motif import _native as N
    from mlx_motif.cache import MotifGroupedKVCache

    c = MotifGroupedKVCache(max_size=64)
    c._grow(1, 2, 1, 128, torch.float16, cuda)
    t = torch.zeros(4096, dtype=torch.float16, device=cuda)
    ws = torch.zeros(1 << 16, dtype=torch.uint8, device=cuda)
    rc = N.lib.motif_vanilla_decode_step(t.data_ptr(), t.data_ptr(), c.slots_struct(), t.data_ptr(), 0.1, 2, 3,
                                         t.data_ptr(), t.data_ptr(), 0.2, 1e-5, t.data_ptr(), ws.data_ptr(),
                                         ws.numel(), N.stream())
    assert rc == N.ERR_BAD_CONTRACT and b"n_rep=3" in N.lib.motif_last_error()
    rc = N.lib.motif_vanilla_decode_step(t.data_ptr(), t.data_ptr(), c.slots_struct(), t.data_ptr(), 0.1, 4, 2,
                                         t.data_ptr(), t.data_ptr(), 0.2, 1e-5, t.data_ptr(), ws.data_ptr(),
                                         ws.numel(), N.stream())
    assert rc == N.ERR_BAD_CONTRACT and b"kv heads per slot" in N.lib.motif_last_error()


# ---------------------------------------------------------------- MotifVanillaKVCache API
def test_vanilla_cache_update_and_fetch_orders():
    """keys come back in stripe order, values in slab order; hf_ordered_values restores the
    projection's paired order; state + meta_state round-trip (reference tests of
    ``MotifVanillaKVCache``, ``tests/test_vanilla_slab_cache.py:119-190``)."""
    from mlx_motif.cache import MotifVanillaKVCache, vanilla_v_paired_to_slab_perm

    B, Hk, S, d = 1, 3, 5, 128
    g = torch.Generator(device="cuda").manual_seed(3)
    paired = torch.randn((B, 2 * Hk, S, d), generator=g, device="cuda").half()
    slab = paired[:, vanilla_v_paired_to_slab_perm(Hk).cuda()]
    k = torch.randn((B, 2 * Hk, S, d), generator=g, device="cuda").half()
    cache = MotifVanillaKVCache()
    K, V = cache.update_and_fetch(k[:, :, :2], slab[:, :, :2])
    K, V = cache.update_and_fetch(k[:, :, 2:], slab[:, :, 2:])
    assert cache.offset == S
    assert torch.equal(K, k) and torch.equal(V, slab)
    assert torch.equal(cache.hf_ordered_values(), paired)
    assert cache.meta_state == ("slab",)
    r = MotifVanillaKVCache.from_state(cache.state, cache.meta_state)
    assert r.offset == S and torch.equal(r.keys, k) and torch.equal(r.values, slab)
    with pytest.raises(ValueError, match="V head-order marker mismatch"):
        MotifVanillaKVCache.from_state(cache.state, ("paired",))
    with pytest.raises(ValueError, match="no V head-order marker"):
        MotifVanillaKVCache.from_state(cache.state, ())
    # the 4-slot device form the decode step reads
    assert torch.equal(cache.k1[:, :, :S], k[:, 0::2]) and torch.equal(cache.v2[:, :, :S], slab[:, Hk:])


# ---------------------------------------------------------------- whole vanilla decoder
def _vanilla_args(n_rep):
    heads = 4 if n_rep < 4 else 8
    kv = heads // n_rep
    return O.OracleVanillaArgs(hidden_size=heads * 128, num_hidden_layers=3, intermediate_size=512,
                               num_attention_heads=heads, num_key_value_heads=kv, head_dim=128, vocab_size=1000)


def _to_model_args(a):
    from mlx_motif.model import ModelArgs

    return ModelArgs(hidden_size=a.hidden_size, num_hidden_layers=a.num_hidden_layers,
                     intermediate_size=a.intermediate_size, num_attention_heads=a.num_attention_heads,
                     num_key_value_heads=a.num_key_value_heads, vocab_size=a.vocab_size, head_dim=a.head_dim,
                     num_noise_heads=None)


@pytest.mark.parametrize("n_rep", [1, 2, 4])
def test_vanilla_decoder_matches_oracle(cuda, n_rep):
    """Greedy decode of a 3-layer vanilla model: every token and the last logits equal the
    oracle's fp16 forward (prefill through the decode path, then generated steps)."""
    from mlx_motif.cache import MotifVanillaKVCache
    from mlx_motif.model import MotifDecoder

    a = _vanilla_args(n_rep)
    w = O.make_synthetic_weights_vanilla(a, seed=n_rep, std=0.05)
    dec = MotifDecoder(_to_model_args(a), w, cache="fp16", max_seq=64, device=cuda)
    assert dec.vanilla and all(isinstance(c, MotifVanillaKVCache) for c in dec.caches)
    orc = O.VanillaDecodeOracle(a, w)
    prompt = [5, 17, 3]
    for t in prompt:
        logits, tok = orc.step(t)
    toks_o = [tok]
    for _ in range(4):
        logits, tok = orc.step(toks_o[-1])
        toks_o.append(tok)
    toks = dec.generate(prompt, 5)
    assert toks == toks_o, f"device {toks} != oracle {toks_o}"
    assert_close(down(dec.logits), logits.astype(np.float64), "float16", atol=1e-2, rtol=2e-2,
                 what="final logits")
    # the caches hold the reference's view: stripe-ordered keys, slab-ordered values
    c = dec.caches[1]
    assert c.keys.shape == (1, 2 * a.Hk, len(prompt) + 4, 128)
    assert c.values.shape == c.keys.shape


def test_vanilla_decoder_quantized_cache_runs(cuda):
    """q8 4-slot cache under the vanilla step: greedy tokens equal the fp16-cache decoder's
    on a short prompt (quantization error far below the logit margins of this model)."""
    from mlx_motif.model import MotifDecoder

    a = _vanilla_args(4)
    w = O.make_synthetic_weights_vanilla(a, seed=9, std=0.05)
    ref = MotifDecoder(_to_model_args(a), w, cache="fp16", max_seq=64, device=cuda).generate([1, 2], 4)
    q8 = MotifDecoder(_to_model_args(a), w, cache="q8", max_seq=64, device=cuda).generate([1, 2], 4)
    assert q8 == ref
