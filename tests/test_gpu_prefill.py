"""GPU parity of the prefill (prompt-length) path against the oracle: the tcgen05 q4 GEMM
(the reference's mx.quantized_matmul behind every nn.QuantizedLinear of a prompt forward,
model.py:1047-1079)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle as O
from conftest import assert_close
from test_gpu_kernels import down, rounded, up

pytestmark = pytest.mark.gpu


def _qweights(rng, n, k):
    w = (rng.standard_normal((n, k)) * 0.02).astype(np.float16)
    return O.quantize(w, 64, 4)


def _dev_triple(tr, dev):
    d, s, b = tr
    return (torch.from_numpy(np.ascontiguousarray(d).view(np.int32)).to(dev), torch.from_numpy(s).to(dev),
            torch.from_numpy(b).to(dev))


@pytest.mark.parametrize("M,N,K", [(128, 256, 512), (300, 384, 1024), (129, 128, 2048), (1000, 3072, 2048),
                                   (517, 2048, 8192), (1000, 16384, 512), (1100, 38400, 512)])
def test_q4_gemm_matches_oracle(cuda, M, N, K):
    """motif_q4_gemm (tcgen05) == oracle quantized_matmul (fp64 of the dequantized weights),
    fp16 tolerance; rows past M are never written; the error word stays 0. The last two shapes
    fill a whole wave with 256-row CTAs (two row tiles per B tile, ragged last pair)."""
    from mlx_motif import _native as N_

    rng = np.random.default_rng(M + N + K)
    x = rounded(rng.standard_normal((M, K)), "float16")
    tr = _qweights(rng, N, K)
    wd, ws, wb = _dev_triple(tr, cuda)
    tx = up(x)
    y = torch.full((M + 3, N), 7.0, dtype=torch.float16, device=cuda)
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    N_.check(N_.lib.motif_q4_gemm(tx.data_ptr(), M, K, wd.data_ptr(), ws.data_ptr(), wb.data_ptr(), N, y.data_ptr(),
                                  None, err.data_ptr(), N_.stream()), "q4_gemm")
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    ref = O.quantized_matmul(x, *tr, group_size=64, bits=4)
    assert_close(down(y[:M]), ref, "float16", what=f"q4 gemm {M}x{N}x{K}")
    assert torch.all(y[M:] == 7.0), "rows past M written"


def test_q4_gemm_residual_and_linear_routing(cuda):
    """With a residual the epilogue adds it in fp16 after rounding the product (the reference's
    h + linear(x)); motif_quantized_linear routes m >= 128 to the same GEMM."""
    from mlx_motif import _native as N_

    M, N, K = 256, 512, 1024
    rng = np.random.default_rng(5)
    x = rounded(rng.standard_normal((M, K)), "float16")
    res = rounded(rng.standard_normal((M, N)), "float16")
    tr = _qweights(rng, N, K)
    wd, ws, wb = _dev_triple(tr, cuda)
    tx, tres = up(x), up(res)
    y = torch.empty((M, N), dtype=torch.float16, device=cuda)
    N_.check(N_.lib.motif_q4_gemm(tx.data_ptr(), M, K, wd.data_ptr(), ws.data_ptr(), wb.data_ptr(), N, y.data_ptr(),
                                  tres.data_ptr(), None, N_.stream()), "q4_gemm")
    y2 = torch.empty((M, N), dtype=torch.float16, device=cuda)
    N_.check(N_.lib.motif_quantized_linear(0, 4, 64, tx.data_ptr(), M, K, wd.data_ptr(), ws.data_ptr(),
                                           wb.data_ptr(), N, y2.data_ptr(), None, 0, N_.stream()), "linear")
    torch.cuda.synchronize()
    lin = O.quantized_matmul(x, *tr, group_size=64, bits=4).astype(np.float16)
    assert_close(down(y2), lin, "float16", what="quantized_linear m=256")
    ref = (lin.astype(np.float32) + res.astype(np.float32)).astype(np.float16)
    # the product may round differently by one fp16 ulp before the add
    assert_close(down(y), ref, "float16", atol=4e-3, what="gemm + residual")
    assert torch.equal((y2.float() + tres.float()).half(), y), "residual epilogue != fp16(linear) + residual"


def test_q4_gemm_rejects_outside_contract(cuda):
    from mlx_motif import _native as N_

    t = torch.zeros(1 << 20, dtype=torch.float16, device=cuda)
    p = t.data_ptr()
    assert N_.lib.motif_q4_gemm(p, 64, 512, p, p, p, 256, p, None, None, N_.stream()) == N_.ERR_BAD_CONTRACT
    assert N_.lib.motif_q4_gemm(p, 128, 576, p, p, p, 256, p, None, None, N_.stream()) == N_.ERR_BAD_CONTRACT
    assert N_.lib.motif_q4_gemm(p, 128, 512, p, p, p, 200, p, None, None, N_.stream()) == N_.ERR_BAD_CONTRACT


# ---------------------------------------------------------------- batched RoPE + append
@pytest.mark.parametrize("bits", [16, 4])
def test_rope_qkv_append_rows_equals_row_by_row(cuda, bits):
    """motif_rope_qkv_append_rows over a block of rows == motif_rope_qkv_append one row at a time,
    bit for bit: q (head-major) and every cache slot (codes, scales and biases for q4)."""
    from mlx_motif import _native as N_
    from mlx_motif.cache import MotifGroupedKVCache, MotifGroupedQuantizedKVCache
    from mlx_motif.model import rope_inv_freq

    G, qh, d, S, off, cap = 2, 8, 128, 37, 5, 128
    rng = np.random.default_rng(bits)
    qkv = up(rounded(rng.standard_normal((S, (qh + 4 * G) * d)), "float16"))
    inv = rope_inv_freq(d, 10000.0, cuda)

    def make():
        c = MotifGroupedKVCache(max_size=cap) if bits == 16 else MotifGroupedQuantizedKVCache(64, 4, max_size=cap)
        c._grow(1, G, 1, d, torch.float16, cuda)
        return c

    ca, cb = make(), make()
    qa = torch.empty((qh, S, d), dtype=torch.float16, device=cuda)
    N_.check(N_.lib.motif_rope_qkv_append_rows(qkv.data_ptr(), S, inv.data_ptr(), qh, ca.slots_struct(), off, None,
                                               qa.data_ptr(), N_.stream()), "rope rows")
    qb = torch.empty((qh, S, d), dtype=torch.float16, device=cuda)
    row_q = torch.empty((qh, d), dtype=torch.float16, device=cuda)
    for s in range(S):
        pos = torch.tensor([off + s], dtype=torch.int32, device=cuda)
        N_.check(N_.lib.motif_rope_qkv_append(qkv[s].data_ptr(), inv.data_ptr(), qh, cb.slots_struct(),
                                              pos.data_ptr(), row_q.data_ptr(), N_.stream()))
        qb[:, s].copy_(row_q)
    torch.cuda.synchronize()
    assert torch.equal(qa, qb)
    for n in ("k1", "k2", "v1", "v2"):
        a, b = getattr(ca, n), getattr(cb, n)
        for x, y in (zip(a, b) if isinstance(a, tuple) else [(a, b)]):
            assert torch.equal(x, y), f"slot {n} differs"


# ---------------------------------------------------------------- prompt attention
def _filled_cache(rng, G, n, cap, dev):
    from mlx_motif.cache import MotifGroupedKVCache

    c = MotifGroupedKVCache(max_size=cap)
    rows = [rounded(rng.standard_normal((1, G, n, 128)) * 0.5, "float16") for _ in range(4)]
    c.update_and_fetch_4(*(up(r) for r in rows))
    return c, rows


@pytest.mark.parametrize("S,off", [(1, 0), (100, 0), (300, 0), (130, 77), (64, 1000)])
def test_prefill_attention_grouped_matches_oracle(cuda, S, off):
    """motif_prefill_attention (tcgen05, mode 0) == the four per-slab causal SDPAs of
    _forward_grouped's prompt branch (model.py:769-807), and motif_prefill_post ==
    gda_post_split over every row."""
    from mlx_motif import _native as N_

    G, gr, d = 2, 3, 128
    qh = G * (gr + 1)
    rng = np.random.default_rng(S + off)
    cache, (k1, k2, v1, v2) = _filled_cache(rng, G, off + S, 2048, cuda)
    q = rounded(rng.standard_normal((qh, S, d)), "float16")  # head-major, origin-first
    tq = up(q)
    o = torch.full((S, qh, 2 * d), float("nan"), dtype=torch.float16, device=cuda)
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    N_.check(N_.lib.motif_prefill_attention(tq.data_ptr(), S, qh, cache.slots_struct(), off, 0, gr, d ** -0.5,
                                            o.data_ptr(), err.data_ptr(), N_.stream()), "prefill_attention")
    subln = rounded(1 + 0.02 * rng.standard_normal(2 * d), "float16")
    lam = np.array([0.37], np.float32)
    y = torch.empty((S, G * gr, 2 * d), dtype=torch.float16, device=cuda)
    t_sub, t_lam = up(subln), torch.tensor(lam, device=cuda)
    N_.check(N_.lib.motif_prefill_post(o.data_ptr(), S, qh, 0, G, gr, t_sub.data_ptr(), t_lam.data_ptr(), 1, 0.8,
                                       1e-5, y.data_ptr(), N_.stream()), "prefill_post")
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    ao, an = O.grouped_prompt_attention_reference(q[None, : G * gr], q[None, G * gr:], k1, k2, v1, v2, d ** -0.5, off)
    got = down(o).transpose(1, 0, 2)[None]  # (1, qh, S, 256)
    assert_close(got[:, : G * gr], ao.astype(np.float64), "float16", what="origin heads")
    assert_close(got[:, G * gr:], an.astype(np.float64), "float16", what="noise heads")
    # the post on the kernel's own attention rows
    ref = O.gda_post_split_reference(got[:, : G * gr], got[:, G * gr:], subln, lam, 0.8, gr, 1e-5)
    assert_close(down(y).transpose(1, 0, 2)[None], ref.astype(np.float16).astype(np.float64), "float16",
                 what="gda post rows")


@pytest.mark.parametrize("G,S,off", [(8, 5, 800), (8, 1, 300), (8, 17, 2000), (8, 128, 1000), (8, 3, 190),
                                     (2, 5, 830), (8, 64, 255)])
def test_prefill_attention_split_matches_oracle(cuda, G, S, off):
    """motif_prefill_attention_split (key tiles divided among CTAs per head, fp32 partial
    states merged by a second kernel) == the oracle's per-slab causal SDPAs, and == the
    one-CTA-per-head launch within fp16 rounding; rows whose first visible key lies in a
    later split (the block's own causal tail) included."""
    from mlx_motif import _native as N_

    gr, d = 3, 128
    qh = G * (gr + 1)
    rng = np.random.default_rng(7 * S + off + G)
    cache, (k1, k2, v1, v2) = _filled_cache(rng, G, off + S, 4096, cuda)
    tq = up(rounded(rng.standard_normal((qh, S, d)), "float16"))
    q = down(tq)
    ws_bytes = N_.lib.motif_prefill_attention_split_workspace_bytes(S, qh)
    assert ws_bytes > 0
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=cuda)
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    outs = []
    for split in (True, False):
        o = torch.full((S, qh, 2 * d), float("nan"), dtype=torch.float16, device=cuda)
        if split:
            N_.check(N_.lib.motif_prefill_attention_split(tq.data_ptr(), S, qh, cache.slots_struct(), off, None, 0, gr,
                                                          d ** -0.5, o.data_ptr(), ws.data_ptr(), ws_bytes,
                                                          err.data_ptr(), N_.stream()), "prefill_attention_split")
        else:
            N_.check(N_.lib.motif_prefill_attention(tq.data_ptr(), S, qh, cache.slots_struct(), off, 0, gr,
                                                    d ** -0.5, o.data_ptr(), err.data_ptr(), N_.stream()),
                     "prefill_attention")
        outs.append(o)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    ao, an = O.grouped_prompt_attention_reference(q[None, : G * gr], q[None, G * gr:], k1, k2, v1, v2, d ** -0.5, off)
    got = down(outs[0]).transpose(1, 0, 2)[None]
    assert_close(got[:, : G * gr], ao.astype(np.float64), "float16", what="split: origin heads")
    assert_close(got[:, G * gr:], an.astype(np.float64), "float16", what="split: noise heads")
    assert_close(down(outs[0]), down(outs[1]).astype(np.float64), "float16", what="split vs one CTA per head")


@pytest.mark.parametrize("n_rep,S,off", [(4, 200, 0), (4, 129, 300), (2, 64, 0), (1, 257, 5)])
def test_prefill_attention_vanilla_matches_oracle(cuda, n_rep, S, off):
    """mode 1 + the vanilla combine == _forward_vanilla's prompt attention (model.py:486-559):
    four per-slab causal SDPAs with native GQA, (o1 − λ·o2), SubLN, (1 − λ_init)."""
    from mlx_motif import _native as N_

    Hk, d = 2, 128
    H = Hk * n_rep
    qh = 2 * H
    rng = np.random.default_rng(10 * n_rep + S)
    cache, (k1, k2, va, vb) = _filled_cache(rng, Hk, off + S, 1024, cuda)
    q = rounded(rng.standard_normal((qh, S, d)), "float16")
    tq = up(q)
    o = torch.empty((S, qh, 2 * d), dtype=torch.float16, device=cuda)
    N_.check(N_.lib.motif_prefill_attention(tq.data_ptr(), S, qh, cache.slots_struct(), off, 1, n_rep, d ** -0.5,
                                            o.data_ptr(), None, N_.stream()), "prefill_attention")
    subln = rounded(1 + 0.02 * rng.standard_normal(2 * d), "float16")
    lam, lam_init = np.array([0.41], np.float32), 0.35
    y = torch.empty((S, H, 2 * d), dtype=torch.float16, device=cuda)
    N_.check(N_.lib.motif_prefill_post(o.data_ptr(), S, qh, 1, Hk, n_rep, up(subln).data_ptr(),
                                       torch.tensor(lam, device=cuda).data_ptr(), 1, lam_init, 1e-5, y.data_ptr(),
                                       N_.stream()), "prefill_post")
    torch.cuda.synchronize()
    # oracle: keys in stripe order, values in the projection's paired order, the new rows last
    K = np.stack([k1, k2], axis=2).reshape(1, 2 * Hk, off + S, d)
    V_paired = np.concatenate([va, vb], axis=1)[:, O.vanilla_v_slab_to_paired_perm(Hk)]
    oc = O.OracleVanillaKVCache()
    if off:
        oc.update_and_fetch(K[:, :, :off].astype(np.float16),
                            np.concatenate([va, vb], axis=1)[:, :, :off].astype(np.float16))
    ref = O.vanilla_attention_reference(q[None], K[:, :, off:], V_paired[:, :, off:], oc, lam, lam_init, subln, 1e-5)
    assert_close(down(y), ref[0].transpose(1, 0, 2).astype(np.float64), "float16", what="vanilla prompt attention")


# ---------------------------------------------------------------- whole-model prompt ingestion
def _grouped_model(cache, seed=0):
    from mlx_motif.model import ModelArgs, MotifDecoder

    a = ModelArgs(hidden_size=512, num_hidden_layers=3, intermediate_size=1024, num_attention_heads=32,
                  num_key_value_heads=16, num_noise_heads=8, vocab_size=1024)
    return MotifDecoder.random(a, seed=seed, std=0.05, cache=cache, max_seq=1024)


def _vanilla_model(n_rep, seed=0):
    from mlx_motif.model import ModelArgs, MotifDecoder

    heads = 8 if n_rep == 4 else 4
    a = ModelArgs(hidden_size=heads * 128, num_hidden_layers=3, intermediate_size=1024, num_attention_heads=heads,
                  num_key_value_heads=heads // n_rep, num_noise_heads=None, vocab_size=1024)
    return MotifDecoder.random(a, seed=seed, std=0.05, cache="fp16", max_seq=1024)


@pytest.mark.parametrize("kind", ["grouped-fp16", "grouped-q4", "grouped-q8", "vanilla-4", "vanilla-1"])
def test_batched_prefill_matches_stepwise(cuda, kind):
    """A prompt ingested in tensor-core row blocks (chunks of 128, so several blocks with a
    nonzero cache offset, the chunked-prefill case; the 43-row tail runs the multi-row GEMV)
    leaves the same cache and greedy continuation as feeding it through the decode step one
    token at a time: K/V rows within fp16 tolerance, identical greedy tokens, close final logits."""
    _compare_prefill(kind, 300, 128)


@pytest.mark.parametrize("kind", ["grouped-fp16", "grouped-q4", "vanilla-4"])
def test_short_prompt_row_block_matches_stepwise(cuda, kind):
    """A 37-token prompt: one 36-row block on the multi-row GEMV (chunks of 7 and 8 rows), then
    the decode step for the last token, against the all-decode-step ingestion."""
    _compare_prefill(kind, 37, None)


def _compare_prefill(kind, n, chunk):
    def make():
        if kind.startswith("grouped"):
            return _grouped_model(kind.split("-")[1], seed=3)
        return _vanilla_model(int(kind.split("-")[1]), seed=3)

    prompt = np.random.default_rng(1).integers(0, 1024, n).tolist()
    a, b = make(), make()
    assert a._block_ok()
    a.prefill(prompt, chunk=chunk, batched=True)
    b.prefill(prompt, batched=False)
    assert a.offset == b.offset == len(prompt)
    assert int(a.token.item()) == int(b.token.item())
    # A q4 cache flips a code wherever a row sits on a rounding boundary; the flip (one
    # quantization step, range/15) then propagates through the later layers.
    lt = {"q4": 0.15, "q8": 0.05}.get(kind.split("-")[1], 2e-2)
    assert_close(down(a.logits), down(b.logits), "float16", atol=lt, rtol=2e-2, what="first-token logits")
    ca, cb = a.caches[-1], b.caches[-1]
    for slot in ("k1", "k2", "v1", "v2"):
        x, y = getattr(ca, slot), getattr(cb, slot)
        if isinstance(x, tuple):  # quantized: the rows agree but for boundary flips of single codes
            from mlx_motif.quantization import dequantize

            dx = dequantize(*(t[..., :n, :].contiguous() for t in x), group_size=64, bits=ca.bits).float()
            dy = dequantize(*(t[..., :n, :].contiguous() for t in y), group_size=64, bits=cb.bits).float()
            rel = ((dx - dy).abs().mean() / dy.abs().mean()).item()
            assert rel <= 0.05, f"last-layer {slot}: mean |difference| is {rel:.3f} of mean |value|"
        else:
            assert_close(down(x[..., :n, :]), down(y[..., :n, :]), "float16", atol=2e-2, rtol=2e-2,
                         what=f"last-layer {slot} rows")
    ta = [int(a.token.item())]
    tb = [int(b.token.item())]
    for _ in range(6):
        a.step_device()
        b.step_device()
        ta.append(int(a.token.item()))
        tb.append(int(b.token.item()))
    assert ta == tb


def test_batched_prefill_vanilla_matches_oracle(cuda):
    """Vanilla prompt of 140 tokens through one 139-row tensor-core block + the decode step ==
    the oracle's token-by-token _forward_vanilla: the same first greedy token, logits within
    tolerance."""
    from mlx_motif.model import ModelArgs, MotifDecoder

    a = O.OracleVanillaArgs(hidden_size=1024, num_hidden_layers=2, intermediate_size=512, num_attention_heads=8,
                            num_key_value_heads=2, head_dim=128, vocab_size=512)
    w = O.make_synthetic_weights_vanilla(a, seed=4, std=0.05)
    ma = ModelArgs(hidden_size=1024, num_hidden_layers=2, intermediate_size=512, num_attention_heads=8,
                   num_key_value_heads=2, vocab_size=512, num_noise_heads=None)
    dec = MotifDecoder(ma, w, cache="fp16", max_seq=256, device=cuda)
    prompt = np.random.default_rng(2).integers(0, 512, 140).tolist()
    dec.prefill(prompt, batched=True)
    orc = O.VanillaDecodeOracle(a, w)
    for t in prompt:
        logits, tok = orc.step(t)
    assert int(dec.token.item()) == tok
    assert_close(down(dec.logits), logits.astype(np.float64), "float16", atol=2e-2, rtol=2e-2, what="logits")
