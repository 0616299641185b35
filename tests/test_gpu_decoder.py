"""GPU parity of the decode-step pieces and of the whole decoder against the oracle:
quantized linear, RoPE, norms, argmax, 4-slot cache API, the fused layer
attention, and greedy decode of a small GDA model (graph and eager)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle as O
from conftest import assert_close
from test_gpu_kernels import down, rounded, up

pytestmark = pytest.mark.gpu


# ---------------------------------------------------------------- quantized linear
@pytest.mark.parametrize("N,K", [(8192, 4096), (4096, 6144), (28672, 4096), (4096, 14336), (16, 128),
                                 (100, 384), (257, 1280), (1000, 4096)])
def test_quantized_linear_matches_oracle(cuda, N, K):
    from mlx_motif.linear import quantized_matmul
    from mlx_motif.quantization import quantize

    rng = np.random.default_rng(N + K)
    w = rounded(rng.standard_normal((N, K)) * 0.02, "float16")
    x = rounded(rng.standard_normal((1, K)), "float16")
    d, s, b = quantize(up(w), 64, 4)
    got = quantized_matmul(up(x), d, s, b, group_size=64, bits=4)
    ref = O.quantized_matmul(x, d.cpu().numpy().view(np.uint32), down(s), down(b), 64, 4)
    assert_close(down(got), ref, "float16", what=f"q4 linear {N}x{K}")


@pytest.mark.parametrize("bits,gs", [(8, 64), (4, 32), (4, 128)])
def test_quantized_linear_general_path(cuda, bits, gs):
    from mlx_motif.linear import quantized_matmul
    from mlx_motif.quantization import quantize

    rng = np.random.default_rng(3)
    w = rounded(rng.standard_normal((300, 512)) * 0.02, "float16")
    x = rounded(rng.standard_normal((3, 512)), "float16")
    d, s, b = quantize(up(w), gs, bits)
    got = quantized_matmul(up(x), d, s, b, group_size=gs, bits=bits)
    ref = O.quantized_matmul(x, d.cpu().numpy().view(np.uint32), down(s), down(b), gs, bits)
    assert_close(down(got), ref, "float16", what="general linear")


def test_quantized_linear_multi_row_uses_fast_path(cuda):
    from mlx_motif.linear import quantized_matmul
    from mlx_motif.quantization import quantize

    rng = np.random.default_rng(4)
    w = rounded(rng.standard_normal((512, 4096)) * 0.02, "float16")
    x = rounded(rng.standard_normal((5, 4096)), "float16")
    d, s, b = quantize(up(w), 64, 4)
    got = quantized_matmul(up(x), d, s, b)
    ref = O.quantized_matmul(x, d.cpu().numpy().view(np.uint32), down(s), down(b), 64, 4)
    assert_close(down(got), ref, "float16", what="5-row linear")


@pytest.mark.parametrize("M", [2, 3, 5, 8, 9, 17])
@pytest.mark.parametrize("N,K", [(2048, 2048), (16384, 2048), (2048, 8192), (1000, 4096), (100, 512)])
def test_quantized_linear_row_chunks_match_oracle(cuda, M, N, K):
    """2..127 rows run the multi-row GEMV (chunks of up to 8 rows, one weight pass per chunk);
    the same workspace serves two calls in a row (split-tile counters return to zero)."""
    from mlx_motif.linear import quantized_matmul
    from mlx_motif.quantization import quantize

    rng = np.random.default_rng(M * 131 + N + K)
    w = rounded(rng.standard_normal((N, K)) * 0.02, "float16")
    x = rounded(rng.standard_normal((M, K)), "float16")
    d, s, b = quantize(up(w), 64, 4)
    ref = O.quantized_matmul(x, d.cpu().numpy().view(np.uint32), down(s), down(b), 64, 4)
    from mlx_motif._native import lib

    ws = torch.zeros(max(lib.motif_quantized_linear_workspace_bytes(M, N, K, 4, 64), 16), dtype=torch.uint8,
                     device="cuda")
    for call in range(2):
        got = quantized_matmul(up(x), d, s, b, workspace=ws)
        assert_close(down(got), ref, "float16", what=f"{M}-row linear {N}x{K} call {call}")


@pytest.mark.parametrize("M", [3, 5, 37, 163])
@pytest.mark.parametrize("N,K", [(4096, 768), (4096, 1792)])
def test_quantized_linear_rows_of_tp8_shard_shapes(cuda, M, N, K):
    """Row blocks of the 8-way tensor-parallel o and down shards (k = 768, 1792: not multiples of
    512, so neither the multi-row GEMV nor the GEMM takes them): a few rows run the one-row GEMV,
    a longer block the general kernel in one launch; both match the oracle."""
    from mlx_motif._native import lib
    from mlx_motif.linear import quantized_matmul
    from mlx_motif.quantization import quantize

    rng = np.random.default_rng(M * 7 + K)
    w = rounded(rng.standard_normal((N, K)) * 0.02, "float16")
    x = rounded(rng.standard_normal((M, K)), "float16")
    d, s, b = quantize(up(w), 64, 4)
    ref = O.quantized_matmul(x, d.cpu().numpy().view(np.uint32), down(s), down(b), 64, 4)
    ws = torch.zeros(max(lib.motif_quantized_linear_workspace_bytes(M, N, K, 4, 64), 16), dtype=torch.uint8,
                     device="cuda")
    got = quantized_matmul(up(x), d, s, b, workspace=ws)
    assert_close(down(got), ref, "float16", what=f"{M}-row linear {N}x{K}")


# ---------------------------------------------------------------- rope / norms / argmax
@pytest.mark.parametrize("offset", [0, 5, 16000])
def test_rope_matches_oracle(cuda, offset):
    from mlx_motif import _native as N
    from mlx_motif.model import rope_inv_freq

    rng = np.random.default_rng(5)
    x = rounded(rng.standard_normal((1, 16, 3, 128)), "float16")
    inv = rope_inv_freq(128, 10000.0, cuda)
    np.testing.assert_array_equal(inv.cpu().numpy(), O.rope_inv_freq(128, 10000.0))
    tx = up(x)
    y = torch.empty_like(tx)
    N.check(N.lib.motif_rope(0, tx.data_ptr(), 1, 16, 3, 128, offset, None, inv.data_ptr(), y.data_ptr(),
                             N.stream()))
    assert_close(down(y), O.rope(x, offset), "float16", what="rope")


def test_norms_and_embedding(cuda):
    from mlx_motif import _native as N

    rng = np.random.default_rng(6)
    H = 4096
    x = rounded(rng.standard_normal((2, H)), "float16")
    dl = rounded(rng.standard_normal((2, H)), "float16")
    w = rounded(1 + 0.02 * rng.standard_normal(H), "float16")
    tx, td, tw = up(x), up(dl), up(w)
    y = torch.empty_like(tx)
    N.check(N.lib.motif_rms_norm(0, tx.data_ptr(), tw.data_ptr(), 1e-6, 2, H, y.data_ptr(), N.stream()))
    assert_close(down(y), O.rms_norm(x, w, 1e-6), "float16", what="rms_norm")
    h = tx.clone()
    N.check(N.lib.motif_add_rms_norm(0, h.data_ptr(), td.data_ptr(), tw.data_ptr(), 1e-6, 2, H, y.data_ptr(),
                                     N.stream()))
    hs = (x.astype(np.float32) + dl.astype(np.float32)).astype(np.float16)
    np.testing.assert_array_equal(down(h), hs.astype(np.float32))
    assert_close(down(y), O.rms_norm(hs, w, 1e-6), "float16", what="add_rms_norm")
    table = rounded(rng.standard_normal((50, H)), "float16")
    tt = up(table)
    tok = torch.tensor([37], dtype=torch.int32, device=cuda)
    hh = torch.empty(H, dtype=torch.float16, device=cuda)
    yy = torch.empty(H, dtype=torch.float16, device=cuda)
    N.check(N.lib.motif_embed_rms_norm(0, tok.data_ptr(), tt.data_ptr(), 50, H, tw.data_ptr(), 1e-6,
                                       hh.data_ptr(), yy.data_ptr(), N.stream()))
    np.testing.assert_array_equal(down(hh), table[37])
    assert_close(down(yy), O.rms_norm(table[37], w, 1e-6), "float16", what="embed")


@pytest.mark.parametrize("n", [1, 97, 219520])
def test_argmax_first_index_of_max(cuda, n):
    from mlx_motif import _native as N

    rng = np.random.default_rng(n)
    v = rounded(rng.standard_normal(n), "float16")
    if n > 10:
        m = v.max()
        v[n // 3] = m
        v[n // 2] = m  # ties resolve to the first index
    tv = up(v)
    out = torch.zeros(1, dtype=torch.int32, device=cuda)
    ws_b = N.lib.motif_argmax_workspace_bytes(n)
    ws = torch.empty(ws_b, dtype=torch.uint8, device=cuda)
    N.check(N.lib.motif_argmax(0, tv.data_ptr(), n, out.data_ptr(), ws.data_ptr(), ws_b, N.stream()))
    assert int(out.item()) == int(np.argmax(v))


# ---------------------------------------------------------------- 4-slot caches
def test_fp16_cache_update_and_fetch(cuda):
    from mlx_motif.cache import MotifGroupedKVCache

    rng = np.random.default_rng(0)
    cache = MotifGroupedKVCache()
    xs = [up(rng.standard_normal((1, 8, 5, 128)) * 0.1) for _ in range(4)]
    out = cache.update_and_fetch_4(*xs)
    assert all(t.shape == (1, 8, 256, 128) for t in out) and cache.offset == 5
    ys = [up(rng.standard_normal((1, 8, 1, 128)) * 0.1) for _ in range(4)]
    out = cache.update_and_fetch_4(*ys)
    assert cache.offset == 6
    for slot, a, b in zip(out, xs, ys):
        assert torch.equal(slot[..., :5, :], a) and torch.equal(slot[..., 5:6, :], b)
    assert all(t.shape == (1, 8, 6, 128) for t in cache.state)
    cache.step = 4
    small = MotifGroupedKVCache()
    small.step = 4
    for _ in range(10):
        small.update_and_fetch_4(*(up(rng.standard_normal((1, 4, 1, 32))) for _ in range(4)))
    assert small.offset == 10 and small.k1.shape[2] == 12


def test_cache_head_mismatch_fails_fast(cuda):
    from mlx_motif.cache import MotifGroupedKVCache, MotifGroupedQuantizedKVCache

    for cache in (MotifGroupedKVCache(), MotifGroupedQuantizedKVCache(64, 8)):
        k1 = torch.zeros(1, 4, 1, 128, dtype=torch.float16, device=cuda)
        k2 = torch.zeros(1, 2, 1, 128, dtype=torch.float16, device=cuda)
        with pytest.raises(ValueError, match="share a head count"):
            cache.update_and_fetch_4(k1, k2, k2, k2)


@pytest.mark.parametrize("bits", [4, 8])
def test_quantized_cache_batched_write_bit_exact(cuda, bits):
    """Batched GPU write == oracle's per-slot quantize, bit for bit (codes, scales, biases, rows)."""
    from mlx_motif.cache import MotifGroupedQuantizedKVCache

    rng = np.random.default_rng(1)
    steps = [[rounded(rng.standard_normal((1, 8, S, 128)) * 0.1, "float16") for _ in range(4)] for S in (5, 1, 1, 1)]
    cache = MotifGroupedQuantizedKVCache(64, bits)
    for st in steps:
        live = cache.update_and_fetch_4_quantized(*(up(t) for t in st))
    o = cache.offset
    assert o == 8 and all(c.shape[2] == 256 for slot in live for c in slot)
    for i, slot in enumerate(live):
        ref = O.quantize(np.concatenate([s[i] for s in steps], axis=2).astype(np.float16), 64, bits)
        np.testing.assert_array_equal(slot[0][..., :o, :].cpu().numpy().view(np.uint32), ref[0])
        np.testing.assert_array_equal(down(slot[1][..., :o, :]), ref[1].astype(np.float32))
        np.testing.assert_array_equal(down(slot[2][..., :o, :]), ref[2].astype(np.float32))
    deq = MotifGroupedQuantizedKVCache(64, bits)
    for st in steps:
        out = deq.update_and_fetch_4(*(up(t) for t in st))
    tol = {4: 0.5, 8: 0.05}[bits]
    full = np.concatenate([s[0] for s in steps], axis=2)
    np.testing.assert_allclose(down(out[0]), full.astype(np.float32), atol=tol, rtol=tol)


@pytest.mark.parametrize("bits", [4, 8])
def test_quantized_cache_state_roundtrip(cuda, bits):
    from mlx_motif.cache import MotifGroupedKVCache, MotifGroupedQuantizedKVCache

    rng = np.random.default_rng(2)
    cache = MotifGroupedQuantizedKVCache(64, bits)
    for _ in range(3):
        t = up(rng.standard_normal((1, 4, 1, 128)) * 0.1)
        cache.update_and_fetch_4(t, t, t, t)
    saved = cache.state
    assert all(a.shape[2] == 3 for slot in saved for a in slot)
    restored = MotifGroupedQuantizedKVCache()
    restored.meta_state = cache.meta_state
    restored.state = saved
    assert (restored.offset, restored.group_size, restored.bits) == (3, 64, bits)
    tb = up(rng.standard_normal((1, 4, 1, 128)) * 0.1)
    out = restored.update_and_fetch_4(tb, tb, tb, tb)
    assert all(x.shape == (1, 4, 4, 128) for x in out) and restored.offset == 4
    plain = MotifGroupedKVCache()
    xs = [up(rng.standard_normal((1, 8, 7, 128)) * 0.1) for _ in range(4)]
    plain.update_and_fetch_4(*xs)
    qc = plain.to_quantized(64, 8)
    assert qc.offset == 7
    out = qc.update_and_fetch_4(xs[0][..., :1, :], xs[1][..., :1, :], xs[2][..., :1, :], xs[3][..., :1, :])
    assert all(t.shape == (1, 8, 8, 128) for t in out)
    assert cache.trim(2) == 2 and cache.offset == 1 and cache.is_trimmable()


@pytest.mark.parametrize("N_rows,K", [(1000, 512), (219520 // 8, 4096), (300, 384)])
def test_linear_fused_argmax_epilogue(cuda, N_rows, K):
    """argmax_out / pos_len_inc of motif_linear_fused: the first index of the largest fp16 output
    (rows 5 and 13 tie), a NaN output never wins, equal to motif_argmax on the written outputs,
    pos_len advanced by one per launch, state reset between launches (TMA path for K % 512 == 0,
    register path otherwise)."""
    from mlx_motif import _native as N
    from mlx_motif.quantization import quantize

    rng = np.random.default_rng(N_rows + K)
    w = rng.standard_normal((N_rows, K)).astype(np.float32) * 0.02
    w[5] = w[13] = 1.0  # same 16-row tile: identical accumulation order, so an exact tie
    q = quantize(up(rounded(w, "float16")), 64, 4)
    q[1][3, 0] = float("nan")  # row 3's output is NaN
    x = up(rounded(np.abs(rng.standard_normal(K)) * 0.01, "float16"))
    y = torch.empty(N_rows, dtype=torch.float16, device=cuda)
    tok = torch.full((1,), -1, dtype=torch.int32, device=cuda)
    pos_len = torch.tensor([10, 11], dtype=torch.int32, device=cuda)
    ws = torch.zeros(N.lib.motif_linear_fused_workspace_bytes(N_rows, K), dtype=torch.uint8, device=cuda)
    io = N.motif_linear_io()
    io.mode, io.x, io.argmax_out, io.pos_len_inc = 0, x.data_ptr(), tok.data_ptr(), pos_len.data_ptr()
    ref = torch.empty(1, dtype=torch.int32, device=cuda)
    aws = torch.empty(N.lib.motif_argmax_workspace_bytes(N_rows), dtype=torch.uint8, device=cuda)
    for i in range(2):
        tok.fill_(-1)
        _fused(N, io, q, y, ws)
        N.check(N.lib.motif_argmax(0, y.data_ptr(), N_rows, ref.data_ptr(), aws.data_ptr(), aws.numel(), N.stream()))
        torch.cuda.synchronize()
        assert torch.isnan(y[3]).item()
        assert int(tok.item()) == 5 == int(ref.item()), (int(tok.item()), int(ref.item()))
        assert pos_len.tolist() == [11 + i, 12 + i]


# ---------------------------------------------------------------- fused decode layer attention
@pytest.mark.parametrize("cache_kind", ["fp16", "q4", "q8"])
@pytest.mark.parametrize("kv_len", [1, 37, 200, 3000])
def test_fused_rope_append_and_gda_attention(cuda, cache_kind, kv_len):
    """rope_qkv_append + gda_decode_attention == oracle rope, cache write, two sdpa_dual_v and
    gda_post_split (model.py:589-768) for the 12.7B-class head layout (gr=3, 8 groups)."""
    from mlx_motif import _native as N
    from mlx_motif.cache import MotifGroupedKVCache, MotifGroupedQuantizedKVCache
    from mlx_motif.model import rope_inv_freq

    rng = np.random.default_rng(kv_len)
    G, gr, d, cap = 8, 3, 128, 4096
    qh = G * (gr + 1)
    pos = kv_len - 1
    hist = [rounded(rng.standard_normal((1, G, pos, d)) * 0.5, "float16") for _ in range(4)]
    qkv = rounded(rng.standard_normal(qh * d + 4 * G * d), "float16")
    if cache_kind == "fp16":
        cache = MotifGroupedKVCache(max_size=cap)
    else:
        cache = MotifGroupedQuantizedKVCache(64, 4 if cache_kind == "q4" else 8, max_size=cap)
    if pos:
        cache.update_and_fetch_4(*(up(h) for h in hist)) if cache_kind == "fp16" else \
            cache.update_and_fetch_4_quantized(*(up(h) for h in hist))
    else:
        cache._grow(1, G, 1, d, torch.float16, cuda)
    slots = cache.slots_struct()
    inv = rope_inv_freq(d, 10000.0, cuda)
    pos_t = torch.tensor([pos, kv_len], dtype=torch.int32, device=cuda)
    q_out = torch.empty(qh * d, dtype=torch.float16, device=cuda)
    tq = up(qkv)
    N.check(N.lib.motif_rope_qkv_append(tq.data_ptr(), inv.data_ptr(), qh, slots, pos_t.data_ptr(),
                                        q_out.data_ptr(), N.stream()))
    subln = rounded(1 + 0.02 * rng.standard_normal(2 * d), "float16")
    lam = np.array([0.37], np.float32)
    out = torch.empty(G * gr * 2 * d, dtype=torch.float16, device=cuda)
    ws_b = N.lib.motif_gda_decode_attention_workspace_bytes(qh, d, 64)
    ws = torch.empty(ws_b, dtype=torch.uint8, device=cuda)
    t_sub, t_lam = up(subln), torch.tensor(lam, device=cuda)
    N.check(N.lib.motif_gda_decode_attention(q_out.data_ptr(), slots, d ** -0.5, G, gr, 0, pos_t.data_ptr() + 4,
                                             t_sub.data_ptr(), t_lam.data_ptr(), 1, 0.8, 1e-5, out.data_ptr(),
                                             ws.data_ptr(), ws_b, N.stream()))
    # ---- oracle
    q = qkv[: qh * d].reshape(1, qh, 1, d)
    k = qkv[qh * d: qh * d + 2 * G * d].reshape(1, 2 * G, 1, d)
    v = qkv[qh * d + 2 * G * d:].reshape(1, 2 * G, 1, d)
    qr = O.rope(q, pos).astype(np.float16)
    kr = O.rope(k, pos).astype(np.float16)
    assert_close(down(q_out).reshape(qr.shape), qr, "float16", what="roped q")
    new = [kr[:, 0::2], kr[:, 1::2], v[:, 0::2], v[:, 1::2]]
    if cache_kind == "fp16":
        oc = O.OracleGroupedKVCache()
        if pos:
            oc.update_and_fetch_4(*hist)
        K1, K2, V1, V2 = oc.update_and_fetch_4(*[n.astype(np.float16) for n in new])
        # the appended rows match the oracle's roped fp16 values to one fp16 ulp
        for i, slot in enumerate((cache.k1, cache.k2, cache.v1, cache.v2)):
            assert_close(down(slot[..., pos, :]), new[i][..., 0, :], "float16", what=f"slot {i} row")
        ao = O.sdpa_dual_v_reference(qr[:, : G * gr], K1, V1, V2, d ** -0.5, kv_len).astype(np.float16)
        an = O.sdpa_dual_v_reference(qr[:, G * gr:], K2, V1, V2, d ** -0.5, kv_len).astype(np.float16)
    else:
        bits = cache.bits
        # use the kernel's own stored rows as the history (bit-exact quantized state)
        trip = [tuple(x[..., :kv_len, :].cpu() for x in slot) for slot in (cache.k1, cache.k2, cache.v1, cache.v2)]
        trip = [(t[0].numpy().view(np.uint32), t[1].float().numpy(), t[2].float().numpy()) for t in trip]
        # the appended row quantizes the roped fp16 values exactly like the oracle quantizer
        for i in range(4):
            rq = O.quantize(new[i].astype(np.float16), 64, bits)
            kern_row = trip[i][0][..., pos:pos + 1, :]
            mism = (kern_row != rq[0]).mean()
            assert mism <= 0.02, f"slot {i}: {mism:.3f} of codes differ (RoPE rounding can flip a few)"
        ao = O.sdpa_dual_v_q4_reference(qr[:, : G * gr], trip[0], trip[2], trip[3], d ** -0.5, 64, bits).astype(np.float16)
        an = O.sdpa_dual_v_q4_reference(qr[:, G * gr:], trip[1], trip[2], trip[3], d ** -0.5, 64, bits).astype(np.float16)
    ref = O.gda_post_split_reference(ao, an, subln, lam, 0.8, gr, 1e-5).astype(np.float16)
    assert_close(down(out), ref.reshape(-1).astype(np.float64), "float16", what="fused attention")


@pytest.mark.parametrize("cache_kind", ["fp16", "q4", "q8", "q4g32"])
@pytest.mark.parametrize("kv_len", [1, 37, 200, 3000])
def test_gda_decode_step_equals_two_call_path(cuda, cache_kind, kv_len):
    """motif_gda_decode_step (one launch) == motif_rope_qkv_append + motif_gda_decode_attention
    bit for bit: the attention output and every slot of the cache (codes, scales, biases);
    a repeated launch gives the same output (its per-group counters reset)."""
    from mlx_motif import _native as N
    from mlx_motif.cache import MotifGroupedKVCache, MotifGroupedQuantizedKVCache
    from mlx_motif.model import rope_inv_freq

    rng = np.random.default_rng(100 + kv_len)
    G, gr, d, cap = 8, 3, 128, 4096
    qh = G * (gr + 1)
    pos = kv_len - 1
    hist = [up(rounded(rng.standard_normal((1, G, pos, d)) * 0.5, "float16")) for _ in range(4)]
    tq = up(rounded(rng.standard_normal(qh * d + 4 * G * d), "float16"))

    def make():
        if cache_kind == "fp16":
            c = MotifGroupedKVCache(max_size=cap)
            if pos:
                c.update_and_fetch_4(*hist)
        else:
            gs = 32 if cache_kind == "q4g32" else 64
            c = MotifGroupedQuantizedKVCache(gs, 8 if cache_kind == "q8" else 4, max_size=cap)
            if pos:
                c.update_and_fetch_4_quantized(*hist)
        if not pos:
            c._grow(1, G, 1, d, torch.float16, cuda)
        return c

    ca, cb = make(), make()
    inv = rope_inv_freq(d, 10000.0, cuda)
    pos_t = torch.tensor([pos, kv_len], dtype=torch.int32, device=cuda)
    t_sub = up(rounded(1 + 0.02 * rng.standard_normal(2 * d), "float16"))
    t_lam = torch.tensor(rng.uniform(0.1, 0.6, G * gr).astype(np.float32), device=cuda)
    # two-call path on cache a
    q_out = torch.empty(qh * d, dtype=torch.float16, device=cuda)
    sa = ca.slots_struct()
    N.check(N.lib.motif_rope_qkv_append(tq.data_ptr(), inv.data_ptr(), qh, sa, pos_t.data_ptr(), q_out.data_ptr(),
                                        N.stream()))
    ref = torch.empty(G * gr * 2 * d, dtype=torch.float16, device=cuda)
    ws_b = N.lib.motif_gda_decode_attention_workspace_bytes(qh, d, 64)
    ws = torch.zeros(ws_b, dtype=torch.uint8, device=cuda)
    N.check(N.lib.motif_gda_decode_attention(q_out.data_ptr(), sa, d ** -0.5, G, gr, 0, pos_t.data_ptr() + 4,
                                             t_sub.data_ptr(), t_lam.data_ptr(), G * gr, 0.8, 1e-5, ref.data_ptr(),
                                             ws.data_ptr(), ws_b, N.stream()))
    # one launch on cache b, twice
    sb = cb.slots_struct()
    fb = N.lib.motif_gda_decode_step_workspace_bytes(qh, d, 64)
    fws = torch.zeros(fb, dtype=torch.uint8, device=cuda)
    outs = []
    for _ in range(2):
        out = torch.full((G * gr * 2 * d,), float("nan"), dtype=torch.float16, device=cuda)
        N.check(N.lib.motif_gda_decode_step(tq.data_ptr(), inv.data_ptr(), sb, pos_t.data_ptr(), d ** -0.5, G, gr,
                                            t_sub.data_ptr(), t_lam.data_ptr(), G * gr, 0.8, 1e-5, out.data_ptr(),
                                            fws.data_ptr(), fb, N.stream()), "gda_decode_step")
        torch.cuda.synchronize()
        outs.append(out)
    assert torch.equal(outs[0], ref), "fused step differs from the two-call path"
    assert torch.equal(outs[1], ref), "repeated fused step differs (counters not reset?)"
    assert torch.equal(fws[:256], torch.zeros(256, dtype=torch.uint8, device=cuda))
    names = ("k1", "k2", "v1", "v2")
    for n in names:
        a, b = getattr(ca, n), getattr(cb, n)
        for x, y in (zip(a, b) if isinstance(a, tuple) else [(a, b)]):
            assert torch.equal(x[..., :kv_len, :], y[..., :kv_len, :]), f"cache slot {n} differs"


# ---------------------------------------------------------------- whole decoder
def _tiny_args():
    return O.OracleArgs(hidden_size=256, num_hidden_layers=3, intermediate_size=512, num_noise_heads=8,
                        grouped_ratio=3, kv_heads_per_slot=8, head_dim=128, vocab_size=1000)


def _to_model_args(a):
    from mlx_motif.model import ModelArgs

    return ModelArgs(hidden_size=a.hidden_size, num_hidden_layers=a.num_hidden_layers,
                     intermediate_size=a.intermediate_size, num_attention_heads=a.q_heads,
                     num_key_value_heads=2 * a.kv_heads_per_slot, vocab_size=a.vocab_size,
                     head_dim=a.head_dim, num_noise_heads=a.num_noise_heads)


@pytest.mark.parametrize("cache_kind", ["fp16", "q4", "q8"])
def test_decoder_matches_oracle(cuda, cache_kind):
    """Greedy decode of a 3-layer GDA model: logits within tolerance of the oracle at every
    step (the oracle is fed the GPU's token so the trajectories stay aligned); tokens agree."""
    from mlx_motif.model import MotifDecoder

    oa = _tiny_args()
    w = O.make_synthetic_weights(oa, seed=1, std=0.05)
    dec = MotifDecoder(_to_model_args(oa), w, cache=cache_kind, max_seq=512, device=cuda)
    orc = O.GroupedDecodeOracle(oa, w, cache=cache_kind)
    prompt = [3, 17, 256, 999, 5, 42]
    agree = 0
    tok = None
    for i in range(len(prompt) + 10):
        t_in = prompt[i] if i < len(prompt) else tok
        dec.token.fill_(int(t_in))
        dec.step_device(with_head=True)
        logits_ref, tok_ref = orc.step(t_in)
        got = down(dec.logits)
        # Quantized caches: a value one fp16 ulp apart upstream (GEMV order, RoPE rounding) can
        # sit on a quantization boundary and flip a code by one step (1/15 of a group's range
        # at 4 bits), which moves that row's attention output visibly. The reference bounds its
        # own q4-cache logits only loosely (tests/test_model.py:262-290, within 5.0 of fp16), so
        # the quantized caches get a wider but still tight band here.
        atol = {"fp16": 2e-3, "q8": 2e-2, "q4": 1e-1}[cache_kind]
        rtol = 2e-2 if cache_kind != "fp16" else 1e-2
        assert_close(got, logits_ref.astype(np.float64), "float16", atol=atol, rtol=rtol, what=f"step {i} logits")
        tok = int(dec.token.item())
        agree += int(tok == tok_ref)
    assert agree >= 14, f"greedy agreement {agree}/16"


def test_decoder_graph_equals_eager(cuda):
    from mlx_motif.model import MotifDecoder

    oa = _tiny_args()
    w = O.make_synthetic_weights(oa, seed=2, std=0.05)
    a = MotifDecoder(_to_model_args(oa), w, max_seq=256, device=cuda)
    b = MotifDecoder(_to_model_args(oa), w, max_seq=256, device=cuda)
    for t in (7, 8, 9):
        a.token.fill_(t)
        b.token.fill_(t)
        a.step_device()
        b.step_eager()
        assert torch.equal(a.logits, b.logits) and torch.equal(a.token, b.token)
    assert a.offset == 3 and int(a.pos_len[0]) == 3 and int(a.pos_len[1]) == 4


def test_decoder_with_nvtx_ranges_equals_without(cuda, monkeypatch):
    """MOTIF_NVTX ranges around every op change no launch: the same logits and tokens, eager
    and graph-replayed."""
    import mlx_motif.model as M

    oa = _tiny_args()
    w = O.make_synthetic_weights(oa, seed=2, std=0.05)
    plain = M.MotifDecoder(_to_model_args(oa), w, max_seq=256, device=cuda)
    monkeypatch.setattr(M, "_NVTX", True)
    marked = M.MotifDecoder(_to_model_args(oa), w, max_seq=256, device=cuda)
    for t in (7, 8, 9):
        plain.token.fill_(t)
        marked.token.fill_(t)
        plain.step_eager()
        (marked.step_eager if t == 7 else marked.step_device)()
        assert torch.equal(plain.logits, marked.logits) and torch.equal(plain.token, marked.token)


def test_decoder_host_api_and_generate(cuda):
    from mlx_motif.model import MotifDecoder

    oa = _tiny_args()
    w = O.make_synthetic_weights(oa, seed=3, std=0.05)
    a = MotifDecoder(_to_model_args(oa), w, max_seq=256, device=cuda)
    toks = a.generate([1, 2, 3], 5)
    b = MotifDecoder(_to_model_args(oa), w, max_seq=256, device=cuda)
    b.prefill([1, 2])
    t = b.decode_host(3)
    seq = [t]
    for _ in range(4):
        t = b.decode_host(t)
        seq.append(t)
    assert seq == toks


# ---------------------------------------------------------------- fused decode linear
def _fused(N_, io, ql, out, ws):
    N_.check(N_.lib.motif_linear_fused(io, ql[0].data_ptr(), ql[1].data_ptr(), ql[2].data_ptr(), ql[0].shape[0],
                                       ql[0].shape[1] * 8, out.data_ptr(), ws.data_ptr(), ws.numel(), N_.stream()))


def test_linear_fused_modes_match_oracle(cuda):
    """mode 1 (embedding/residual + RMSNorm prologue, h_out), stats epilogue, mode 2
    (PolyNorm·up prologue from tile statistics), repeated calls bit-identical."""
    from mlx_motif import _native as N
    from mlx_motif.quantization import quantize

    rng = np.random.default_rng(31)
    H, I, V = 4096, 14336, 64
    h = rounded(rng.standard_normal(H), "float16")
    dl = rounded(rng.standard_normal(H) * 0.5, "float16")
    nw = rounded(1 + 0.02 * rng.standard_normal(H), "float16")
    emb = rounded(rng.standard_normal((V, H)), "float16")
    wgu = rounded(rng.standard_normal((2 * I, H)) * 0.02, "float16")
    wd = rounded(rng.standard_normal((H, I)) * 0.02, "float16")
    gu_q = quantize(up(wgu), 64, 4)
    d_q = quantize(up(wd), 64, 4)
    ws = torch.zeros(max(N.lib.motif_linear_fused_workspace_bytes(2 * I, H),
                         N.lib.motif_linear_fused_workspace_bytes(H, I)), dtype=torch.uint8, device=cuda)
    th, tdl, tnw, temb = up(h), up(dl), up(nw), up(emb)
    h_out = torch.empty(H, dtype=torch.float16, device=cuda)
    gu = torch.empty(2 * I, dtype=torch.float16, device=cuda)
    stats = torch.zeros(I // 16 * 3, dtype=torch.float32, device=cuda)
    io = N.motif_linear_io()
    io.mode, io.h_in, io.delta, io.h_out, io.norm_w, io.eps = 1, th.data_ptr(), tdl.data_ptr(), h_out.data_ptr(), \
        tnw.data_ptr(), 1e-6
    io.stats_out, io.stats_rows = stats.data_ptr(), I
    _fused(N, io, gu_q, gu, ws)
    hs = (h.astype(np.float32) + dl.astype(np.float32)).astype(np.float16)
    np.testing.assert_array_equal(down(h_out), hs.astype(np.float32))
    xn = O.rms_norm(hs, nw, 1e-6).astype(np.float16)
    trip_np = lambda t: (t[0].cpu().numpy().view(np.uint32), down(t[1]), down(t[2]))  # noqa: E731
    ref_gu = O.quantized_matmul(xn, *trip_np(gu_q), 64, 4)
    assert_close(down(gu), ref_gu, "float16", what="gate|up (mode 1)")
    g16 = down(gu)[:I].astype(np.float64)
    st = stats.view(-1, 3).sum(0).cpu().numpy()
    np.testing.assert_allclose(st, [np.sum(g16 ** 2), np.sum(g16 ** 4), np.sum(g16 ** 6)], rtol=1e-4)
    # mode 2: PolyNorm(gate)·up -> down
    pw = up([1 / 3, 1 / 3, 1 / 3])
    pb = up([0.0])
    dn = torch.empty(H, dtype=torch.float16, device=cuda)
    io2 = N.motif_linear_io()
    io2.mode, io2.gate, io2.up = 2, gu.data_ptr(), gu.data_ptr() + 2 * I
    io2.stats, io2.stats_count, io2.poly_w, io2.poly_b, io2.poly_eps, io2.poly_dim = stats.data_ptr(), I // 16, \
        pw.data_ptr(), pb.data_ptr(), 1e-6, I
    _fused(N, io2, d_q, dn, ws)
    act = O.polynorm_mul_reference(down(gu)[:I], down(gu)[I:], [1 / 3] * 3, [0.0], 1e-6)
    ref_dn = O.quantized_matmul(act, *trip_np(d_q), 64, 4)
    assert_close(down(dn), ref_dn, "float16", what="down (mode 2)")
    again = torch.empty_like(dn)
    _fused(N, io2, d_q, again, ws)
    assert torch.equal(again, dn), "split-K reduction must be deterministic and its counters reset"
    # embedding gather prologue
    tok = torch.tensor([17], dtype=torch.int32, device=cuda)
    io3 = N.motif_linear_io()
    io3.mode, io3.token, io3.embed, io3.vocab, io3.norm_w, io3.eps, io3.h_out = 1, tok.data_ptr(), temb.data_ptr(), \
        V, tnw.data_ptr(), 1e-6, h_out.data_ptr()
    _fused(N, io3, gu_q, gu, ws)
    np.testing.assert_array_equal(down(h_out), emb[17])
    ref3 = O.quantized_matmul(O.rms_norm(emb[17], nw, 1e-6).astype(np.float16), *trip_np(gu_q), 64, 4)
    assert_close(down(gu), ref3, "float16", what="embedding prologue")
