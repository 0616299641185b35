"""GPU parity of the tensor-core decode step used for long fp16 caches (capacity at or above
MOTIF_LONG_ATTN_MIN_CAP, default 2048): the same contract as the CUDA-core step — RoPE + append
of the new row, split-KV attention, merge with the differential combine — checked against the
oracle, against the CUDA-core step on the same inputs, and for bit-identical cache writes."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle as O
from conftest import assert_close
from test_gpu_kernels import down, rounded, up

pytestmark = pytest.mark.gpu


def _run_step(N, mode, tq, inv, slots, pos_t, d, G, gr, t_sub, t_lam, lam_len, out, ws, wb):
    if mode == "gda":
        return N.lib.motif_gda_decode_step(tq.data_ptr(), inv.data_ptr(), slots, pos_t.data_ptr(), d ** -0.5, G, gr,
                                           t_sub.data_ptr(), t_lam.data_ptr(), lam_len, 0.8, 1e-5, out.data_ptr(),
                                           ws.data_ptr(), wb, N.stream())
    return N.lib.motif_vanilla_decode_step(tq.data_ptr(), inv.data_ptr(), slots, pos_t.data_ptr(), d ** -0.5, G, gr,
                                           t_sub.data_ptr(), t_lam.data_ptr(), 0.35, 1e-5, out.data_ptr(),
                                           ws.data_ptr(), wb, N.stream())


@pytest.mark.parametrize("kind", ["fp16", "q4"])
@pytest.mark.parametrize("mode,gr", [("gda", 3), ("vanilla", 4), ("vanilla", 1)])
@pytest.mark.parametrize("kv_len", [1, 130, 3000, 16000])
def test_long_decode_step_matches_oracle_and_short_path(cuda, monkeypatch, kind, mode, gr, kv_len):
    from mlx_motif import _native as N
    from mlx_motif.cache import MotifGroupedKVCache, MotifGroupedQuantizedKVCache
    from mlx_motif.model import rope_inv_freq

    d, cap = 128, 16384
    G = 8 if mode == "gda" else 2
    qh = G * (gr + 1) if mode == "gda" else 2 * G * gr
    out_heads = G * gr
    rng = np.random.default_rng(kv_len + 7 * gr)
    pos = kv_len - 1
    hist = [rounded(rng.standard_normal((1, G, pos, d)) * 0.5, "float16") for _ in range(4)]
    qkv = rounded(rng.standard_normal(qh * d + 4 * G * d), "float16")

    def make():
        if kind == "fp16":
            c = MotifGroupedKVCache(max_size=cap)
            if pos:
                c.update_and_fetch_4(*(up(h) for h in hist))
        else:
            c = MotifGroupedQuantizedKVCache(64, 4, max_size=cap)
            if pos:
                c.update_and_fetch_4_quantized(*(up(h) for h in hist))
        if not pos:
            c._grow(1, G, 1, d, torch.float16, cuda)
        return c

    inv = rope_inv_freq(d, 10000.0, cuda)
    pos_t = torch.tensor([pos, kv_len], dtype=torch.int32, device=cuda)
    subln = rounded(1 + 0.02 * rng.standard_normal(2 * d), "float16")
    lam = np.array([0.37], np.float32)
    tq, t_sub, t_lam = up(qkv), up(subln), torch.tensor(lam, device=cuda)
    wb = N.lib.motif_gda_decode_step_workspace_bytes(qh, d, 64)
    outs, caches = {}, {}
    for path, min_cap in (("long", "0"), ("short", str(1 << 40))):
        monkeypatch.setenv("MOTIF_LONG_ATTN_MIN_CAP", min_cap)
        c = make()
        ws = torch.zeros(wb, dtype=torch.uint8, device=cuda)
        res = []
        for _ in range(2):
            out = torch.full((out_heads * 2 * d,), float("nan"), dtype=torch.float16, device=cuda)
            N.check(_run_step(N, mode, tq, inv, c.slots_struct(), pos_t, d, G, gr, t_sub, t_lam, 1, out, ws, wb),
                    path)
            torch.cuda.synchronize()
            res.append(out)
        assert torch.equal(res[0], res[1]), f"{path}: repeated step differs"
        assert torch.equal(ws[:256], torch.zeros(256, dtype=torch.uint8, device=cuda)), f"{path}: control words"
        outs[path], caches[path] = res[0], c
    for n in ("k1", "k2", "v1", "v2"):
        a, b = getattr(caches["long"], n), getattr(caches["short"], n)
        for x, y in (zip(a, b) if isinstance(a, tuple) else [(a, b)]):
            assert torch.equal(x[..., :kv_len, :], y[..., :kv_len, :]), f"cache slot {n} differs"
    assert_close(down(outs["long"]), down(outs["short"]), "float16", what="long vs short step")
    # oracle on the stored rows (dequantized in fp32 for q4, as the quantized SDPA reads them)
    c = caches["long"]

    def rows(n):
        t = getattr(c, n)
        if kind == "fp16":
            return down(t[..., :kv_len, :])
        dd, ss, bb = (x[..., :kv_len, :].cpu() for x in t)
        return O.dequantize(dd.numpy().view(np.uint32), ss.float().numpy(), bb.float().numpy(), 64, 4,
                            out_dtype=np.float32)

    k1, k2, v1, v2 = (rows(n) for n in ("k1", "k2", "v1", "v2"))
    if mode == "gda":
        q = qkv[: qh * d].reshape(1, qh, 1, d)
        qr = O.rope(q, pos).astype(np.float16)
        ao = O.sdpa_dual_v_reference(qr[:, : G * gr], k1, v1, v2, d ** -0.5, kv_len).astype(np.float16)
        an = O.sdpa_dual_v_reference(qr[:, G * gr:], k2, v1, v2, d ** -0.5, kv_len).astype(np.float16)
        ref = O.gda_post_split_reference(ao, an, subln, lam, 0.8, gr, 1e-5).astype(np.float16)
    else:
        q = qkv[: qh * d].reshape(1, qh, 1, d)
        qr = O.rope(q, pos).astype(np.float16)
        K = np.stack([k1, k2], axis=2).reshape(1, 2 * G, kv_len, d)
        V_paired = np.concatenate([v1, v2], axis=1)[:, O.vanilla_v_slab_to_paired_perm(G)]
        ref = O.vanilla_attention_reference(qr, K, V_paired, O.OracleVanillaKVCache(), lam, 0.35, subln, 1e-5,
                                            kv_dtype=np.float16 if kind == "fp16" else np.float32)
    assert_close(down(outs["long"]), ref.reshape(-1).astype(np.float64), "float16", what="long step vs oracle")


def test_q4_cache_of_unrounded_length_takes_tensor_core_step(cuda, monkeypatch):
    """A q4 cache sized like the bench's p16k run (16000 prompt rows + warm-up + steps + margin
    = 16033 rows, not a multiple of 4) is preallocated in whole 256-row steps, so the decode step
    takes the tensor-core kernel (reported by motif_decode_step_kernel), and its output matches the
    CUDA-core split step on the same cache."""
    from mlx_motif import _native as N
    from mlx_motif.cache import MotifGroupedQuantizedKVCache
    from mlx_motif.model import rope_inv_freq

    monkeypatch.delenv("MOTIF_LONG_ATTN_MIN_CAP", raising=False)
    G, gr, d, kv_len = 8, 3, 128, 16000
    qh = G * (gr + 1)
    rng = np.random.default_rng(5)
    c = MotifGroupedQuantizedKVCache(64, 4, max_size=16033)
    c.update_and_fetch_4_quantized(*(up(rounded(rng.standard_normal((1, G, kv_len - 1, d)) * 0.5, "float16"))
                                     for _ in range(4)))
    assert c.k1[0].shape[2] == 16128
    assert N.lib.motif_decode_step_kernel(c.slots_struct()) == N.ATTN_KERNEL_TCGEN05
    inv = rope_inv_freq(d, 10000.0, cuda)
    pos_t = torch.tensor([kv_len - 1, kv_len], dtype=torch.int32, device=cuda)
    tq = up(rounded(rng.standard_normal(qh * d + 4 * G * d), "float16"))
    t_sub = up(rounded(1 + 0.02 * rng.standard_normal(2 * d), "float16"))
    t_lam = torch.tensor([0.37], dtype=torch.float32, device=cuda)
    wb = N.lib.motif_gda_decode_step_workspace_bytes(qh, d, 64)
    outs = {}
    for path, min_cap in (("tcgen05", None), ("split", str(1 << 40))):
        if min_cap is None:
            monkeypatch.delenv("MOTIF_LONG_ATTN_MIN_CAP", raising=False)
        else:
            monkeypatch.setenv("MOTIF_LONG_ATTN_MIN_CAP", min_cap)
        want = N.ATTN_KERNEL_TCGEN05 if path == "tcgen05" else N.ATTN_KERNEL_SPLIT
        assert N.lib.motif_decode_step_kernel(c.slots_struct()) == want
        ws = torch.zeros(wb, dtype=torch.uint8, device=cuda)
        out = torch.full((G * gr * 2 * d,), float("nan"), dtype=torch.float16, device=cuda)
        N.check(_run_step(N, "gda", tq, inv, c.slots_struct(), pos_t, d, G, gr, t_sub, t_lam, 1, out, ws, wb), path)
        torch.cuda.synchronize()
        outs[path] = out
    assert_close(down(outs["tcgen05"]), down(outs["split"]), "float16", what="tcgen05 vs split step at 16033")
