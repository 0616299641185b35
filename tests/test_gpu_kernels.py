"""GPU parity of the operator kernels against the CPU oracle.

Shapes, seeds-style inputs, poisoned padding and contract rejections follow
the reference's tests (tests/test_kernels*.py, tests/test_dequant_probe.py);
every call goes through the C ABI via ``mlx_motif.kernels``.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle as O
from conftest import assert_close

pytestmark = pytest.mark.gpu

DT = {"float16": torch.float16, "bfloat16": torch.bfloat16, "float32": torch.float32}


def up(a, dtype="float16", dev="cuda"):
    t = torch.from_numpy(np.ascontiguousarray(np.asarray(a, dtype=np.float32)))
    return t.to(dev).to(DT[dtype])


def down(t):
    return t.float().cpu().numpy()


def rounded(a, dtype):
    """The CPU copy of exactly what was uploaded (inputs rounded to the kernel dtype)."""
    return down(up(a, dtype, "cpu"))


# ---------------------------------------------------------------- polynorm
@pytest.mark.parametrize("shape", [(2, 4, 16), (1, 1, 64), (3, 7, 256), (1, 1, 4096), (1, 1, 14336)])
@pytest.mark.parametrize("dtype", ["float32", "float16", "bfloat16"])
def test_polynorm_matches_oracle(cuda, shape, dtype):
    from mlx_motif.kernels import polynorm

    rng = np.random.default_rng(0)
    x = rounded(rng.standard_normal(shape), dtype)
    w = rounded([0.4, 0.3, 0.3], dtype)
    b = rounded([0.05], dtype)
    got = polynorm(up(x, dtype), up(w, dtype), up(b, dtype), 1e-6)
    assert got.dtype == DT[dtype] and got.shape == shape
    assert_close(down(got), O.polynorm_reference(x, w, b, 1e-6), dtype, what="polynorm")


def test_polynorm_golden_on_gpu(cuda):
    import json
    from pathlib import Path

    from mlx_motif.kernels import polynorm

    case = json.loads((Path(__file__).parent / "golden" / "polynorm_reference_2x3.json").read_text())
    got = polynorm(up(case["input"], "float32"), up(case["weight"], "float32"), up(case["bias"], "float32"),
                   case["eps"])
    np.testing.assert_allclose(down(got), np.array(case["expected"]), atol=1e-6, rtol=1e-6)


@pytest.mark.parametrize("dim", [64, 1000, 14336])
def test_polynorm_mul_matches_oracle(cuda, dim):
    from mlx_motif.kernels import polynorm_mul

    rng = np.random.default_rng(1)
    g = rounded(rng.standard_normal((3, dim)), "float16")
    u = rounded(rng.standard_normal((3, dim)), "float16")
    w = rounded([1 / 3, 1 / 3, 1 / 3], "float16")
    b = rounded([0.0], "float16")
    got = polynorm_mul(up(g), up(u), up(w), up(b), 1e-6)
    ref = O.polynorm_mul_reference(g, u, w, b, 1e-6)
    assert_close(down(got), ref.astype(np.float64), "float16", what="polynorm_mul")


# ---------------------------------------------------------------- gda post
@pytest.mark.parametrize("B,q_groups,gr,S,d", [(1, 8, 4, 1, 128), (1, 8, 3, 1, 128), (1, 8, 4, 32, 128),
                                               (2, 4, 4, 1, 128), (1, 2, 4, 1, 64)])
@pytest.mark.parametrize("dtype", ["float32", "float16", "bfloat16"])
def test_gda_post_split_matches_oracle(cuda, B, q_groups, gr, S, d, dtype):
    from mlx_motif.kernels import gda_post, gda_post_split

    rng = np.random.default_rng(0)
    C = 2 * d
    o = rounded(rng.standard_normal((B, q_groups * gr, S, C)), dtype)
    n = rounded(rng.standard_normal((B, q_groups, S, C)), dtype)
    w = rounded(rng.standard_normal(C), dtype)
    lam = np.array([0.4321], np.float32)
    ref = O.gda_post_split_reference(o, n, w, lam, 0.65, gr, 1e-5)
    got = gda_post_split(up(o, dtype), up(n, dtype), up(w, dtype), torch.tensor(lam, device=cuda), 0.65, gr, 1e-5)
    assert_close(down(got), ref, dtype, what="gda_post_split")
    merged = np.concatenate([o, n], axis=1)
    got2 = gda_post(up(merged, dtype), up(w, dtype), torch.tensor(lam, device=cuda), 0.65, q_groups, gr, 1e-5)
    assert_close(down(got2), ref, dtype, what="gda_post")


@pytest.mark.parametrize("d", [192, 20, 17])
def test_gda_post_split_edge_channels(cuda, d):
    from mlx_motif.kernels import gda_post_split

    rng = np.random.default_rng(1)
    o = rng.standard_normal((1, 8, 3, 2 * d)).astype(np.float32)
    n = rng.standard_normal((1, 2, 3, 2 * d)).astype(np.float32)
    w = rng.standard_normal(2 * d).astype(np.float32)
    ref = O.gda_post_split_reference(o, n, w, [0.4321], 0.65, 4, 1e-5)
    got = gda_post_split(up(o, "float32"), up(n, "float32"), up(w, "float32"), 0.4321, 0.65, 4, 1e-5)
    assert_close(down(got), ref, "float32", what="gda edge")


@pytest.mark.parametrize("lam_len", [8, 24])
def test_gda_post_split_per_head_lambda(cuda, lam_len):
    """Per-head λ extension (config[0]: λ ~ U(0.1, 0.9)), checked against the oracle."""
    from mlx_motif.kernels import gda_post_split

    rng = np.random.default_rng(2)
    o = rounded(rng.standard_normal((1, 24, 1, 256)), "float16")
    n = rounded(rng.standard_normal((1, 8, 1, 256)), "float16")
    w = rounded(np.ones(256), "float16")
    lam = rng.uniform(0.1, 0.9, lam_len).astype(np.float32)
    ref = O.gda_post_split_reference(o, n, w, lam, 0.8, 3, 1e-5)
    got = gda_post_split(up(o), up(n), up(w), torch.tensor(lam, device=cuda), 0.8, 3, 1e-5)
    assert_close(down(got), ref, "float16", what="gda per-head λ")


# ---------------------------------------------------------------- sdpa_dual_v
@pytest.mark.parametrize("B,H,KV,d", [(1, 8, 1, 128), (1, 8, 16, 128), (1, 40, 64, 128), (1, 40, 256, 128),
                                      (1, 8, 17, 128), (2, 16, 64, 64), (1, 8, 5000, 128)])
@pytest.mark.parametrize("dtype", ["float32", "float16", "bfloat16"])
def test_sdpa_dual_v_matches_oracle(cuda, B, H, KV, d, dtype):
    from mlx_motif.kernels import sdpa_dual_v

    rng = np.random.default_rng(0)
    q = rounded(rng.standard_normal((B, H, 1, d)) * 0.1, dtype)
    k = rounded(rng.standard_normal((B, H, KV, d)) * 0.1, dtype)
    v1 = rounded(rng.standard_normal((B, H, KV, d)) * 0.5, dtype)
    v2 = rounded(rng.standard_normal((B, H, KV, d)) * 0.5, dtype)
    scale = d ** -0.5
    got = sdpa_dual_v(up(q, dtype), up(k, dtype), up(v1, dtype), up(v2, dtype), scale)
    assert got.shape == (B, H, 1, 2 * d)
    assert_close(down(got), O.sdpa_dual_v_reference(q, k, v1, v2, scale), dtype, what="sdpa_dual_v")


@pytest.mark.parametrize("B,H_q,H_kv,KV,d", [(1, 32, 8, 64, 128), (1, 16, 8, 32, 128), (1, 32, 4, 100, 128),
                                             (2, 32, 8, 17, 128), (1, 24, 8, 1024, 128), (1, 40, 8, 300, 128)])
@pytest.mark.parametrize("dtype", ["float32", "float16", "bfloat16"])
def test_sdpa_dual_v_gqa(cuda, B, H_q, H_kv, KV, d, dtype):
    from mlx_motif.kernels import sdpa_dual_v

    rng = np.random.default_rng(0)
    q = rounded(rng.standard_normal((B, H_q, 1, d)) * 0.1, dtype)
    k = rounded(rng.standard_normal((B, H_kv, KV, d)) * 0.1, dtype)
    v1 = rounded(rng.standard_normal((B, H_kv, KV, d)) * 0.5, dtype)
    v2 = rounded(rng.standard_normal((B, H_kv, KV, d)) * 0.5, dtype)
    scale = d ** -0.5
    got = sdpa_dual_v(up(q, dtype), up(k, dtype), up(v1, dtype), up(v2, dtype), scale)
    assert_close(down(got), O.sdpa_dual_v_reference(q, k, v1, v2, scale), dtype, what="gqa")


@pytest.mark.parametrize("B,H_q,H_kv,cap,kv_len,d", [(1, 8, 8, 256, 1, 128), (1, 8, 8, 256, 17, 128),
                                                     (1, 32, 8, 256, 100, 128), (1, 40, 8, 512, 385, 128),
                                                     (2, 16, 8, 256, 200, 64), (1, 24, 8, 4096, 3000, 128)])
@pytest.mark.parametrize("dtype", ["float32", "float16", "bfloat16"])
def test_sdpa_dual_v_runtime_kv_len_poisoned(cuda, B, H_q, H_kv, cap, kv_len, d, dtype):
    """Rows past kv_len hold 1e4: any read past the live region diverges loudly."""
    from mlx_motif.kernels import sdpa_dual_v

    rng = np.random.default_rng(7)
    q = rounded(rng.standard_normal((B, H_q, 1, d)) * 0.1, dtype)
    k = rounded(rng.standard_normal((B, H_kv, cap, d)) * 0.1, dtype)
    v1 = rounded(rng.standard_normal((B, H_kv, cap, d)) * 0.5, dtype)
    v2 = rounded(rng.standard_normal((B, H_kv, cap, d)) * 0.5, dtype)
    for t in (k, v1, v2):
        t[..., kv_len:, :] = 1e4
    scale = d ** -0.5
    ref = O.sdpa_dual_v_reference(q, k, v1, v2, scale, kv_len)
    got = sdpa_dual_v(up(q, dtype), up(k, dtype), up(v1, dtype), up(v2, dtype), scale, kv_len=kv_len)
    assert_close(down(got), ref, dtype, what="poisoned kv_len")
    # Device-resident kv_len (the graph-capture form) gives the same result.
    dev_len = torch.tensor([kv_len], dtype=torch.int32, device=cuda)
    got_d = sdpa_dual_v(up(q, dtype), up(k, dtype), up(v1, dtype), up(v2, dtype), scale, kv_len=dev_len)
    assert_close(down(got_d), ref, dtype, what="device kv_len")


def test_sdpa_dual_v_growing_kv_len(cuda):
    from mlx_motif.kernels import sdpa_dual_v

    rng = np.random.default_rng(11)
    B, H_q, H_kv, cap, d = 1, 32, 8, 256, 128
    q = rounded(rng.standard_normal((B, H_q, 1, d)) * 0.1, "float16")
    k = rounded(rng.standard_normal((B, H_kv, cap, d)) * 0.1, "float16")
    v1 = rounded(rng.standard_normal((B, H_kv, cap, d)) * 0.5, "float16")
    v2 = rounded(rng.standard_normal((B, H_kv, cap, d)) * 0.5, "float16")
    tq, tk, t1, t2 = up(q), up(k), up(v1), up(v2)
    for kv_len in (0, 1, 2, 31, 32, 33, 100, 255, 256):
        got = sdpa_dual_v(tq, tk, t1, t2, d ** -0.5, kv_len=kv_len)
        ref = O.sdpa_dual_v_reference(q, k, v1, v2, d ** -0.5, kv_len) if kv_len else np.zeros((B, H_q, 1, 2 * d))
        assert_close(down(got), ref, "float16", what=f"kv_len={kv_len}")


# ---------------------------------------------------------------- quantization
@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("group_size", [32, 64, 128])
@pytest.mark.parametrize("D", [64, 128, 256])
@pytest.mark.parametrize("dtype", ["float16", "bfloat16", "float32"])
def test_quantize_bit_exact_and_dequant(cuda, bits, group_size, D, dtype):
    """Codes, scales and biases bit-identical to the oracle quantizer; dequantize identical."""
    if D % group_size:
        pytest.skip("D not a multiple of group_size")
    from mlx_motif.kernels import _dequant_probe
    from mlx_motif.quantization import quantize

    rng = np.random.default_rng(0)
    x = rounded(rng.standard_normal((2, 5, 7, D)), dtype)
    x[0, 0, 0] = 0.0  # all-zero group
    x[0, 0, 1] = 0.75  # constant group
    tx = up(x, dtype)
    d, s, b = quantize(tx, group_size, bits)
    xd = x.astype(np.float16) if dtype == "float16" else x
    if dtype == "bfloat16":
        # numpy has no bf16: quantize the exact fp32 values, then compare the rounded scales.
        rd, rs, rb = O.quantize(x.astype(np.float32), group_size, bits)
        np.testing.assert_array_equal(d.cpu().numpy().view(np.uint32), rd)
        np.testing.assert_array_equal(down(s), rounded(rs, "bfloat16"))
        np.testing.assert_array_equal(down(b), rounded(rb, "bfloat16"))
    else:
        rd, rs, rb = O.quantize(xd.astype(np.float16 if dtype == "float16" else np.float32), group_size, bits)
        np.testing.assert_array_equal(d.cpu().numpy().view(np.uint32), rd)
        np.testing.assert_array_equal(down(s), rs.astype(np.float32))
        np.testing.assert_array_equal(down(b), rb.astype(np.float32))
    probe = _dequant_probe(d, s, b, group_size=group_size, bits=bits)
    ref = O.dequantize(d.cpu().numpy().view(np.uint32), down(s), down(b), group_size, bits, out_dtype=np.float32)
    np.testing.assert_array_equal(down(probe), rounded(ref, dtype))


# ---------------------------------------------------------------- sdpa_dual_v_q4
_Q_SHAPES = [(1, 4, 4, 16, 128), (1, 4, 4, 128, 128), (1, 4, 4, 300, 128), (1, 4, 4, 1024, 128),
             (2, 4, 4, 64, 128), (1, 8, 4, 64, 128), (1, 16, 4, 64, 128), (1, 40, 8, 256, 128),
             (1, 40, 8, 1024, 128), (1, 24, 8, 2048, 128)]


def _q_inputs(rng, B, H_q, H_kv, KV, d, bits, dtype, gs=64):
    from mlx_motif.quantization import quantize

    q = rounded(rng.standard_normal((B, H_q, 1, d)), dtype)
    raw = [rounded(rng.standard_normal((B, H_kv, KV, d)), dtype) for _ in range(3)]
    trip = [quantize(up(t, dtype), gs, bits) for t in raw]
    return q, trip


def _np_triple(t):
    return (t[0].cpu().numpy().view(np.uint32), down(t[1]), down(t[2]))


@pytest.mark.parametrize("B,H_q,H_kv,KV,d", _Q_SHAPES)
@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("dtype", ["float16", "bfloat16"])
def test_sdpa_dual_v_q4_matches_oracle(cuda, B, H_q, H_kv, KV, d, bits, dtype):
    from mlx_motif.kernels import sdpa_dual_v_q4

    rng = np.random.default_rng(0)
    q, (kq, v1q, v2q) = _q_inputs(rng, B, H_q, H_kv, KV, d, bits, dtype)
    scale = d ** -0.5
    got = sdpa_dual_v_q4(up(q, dtype), kq, v1q, v2q, scale, group_size=64, bits=bits)
    assert got.shape == (B, H_q, 1, 2 * d) and got.dtype == DT[dtype]
    ref = O.sdpa_dual_v_q4_reference(q, _np_triple(kq), _np_triple(v1q), _np_triple(v2q), scale, 64, bits)
    # The reference dequantizes K/V to the activation dtype before SDPA; the kernel keeps
    # the fp32 dequant in registers. fp16: north-star tolerance; bf16: the reference's 5e-2.
    assert_close(down(got), ref, dtype, what="sdpa_dual_v_q4")


def test_sdpa_dual_v_q4_concatenated_layout(cuda):
    from mlx_motif.kernels import sdpa_dual_v_q4
    from mlx_motif.quantization import quantize

    rng = np.random.default_rng(0)
    q = up(rng.standard_normal((1, 4, 1, 128)))
    kq = quantize(up(rng.standard_normal((1, 4, 64, 128))), 64, 4)
    vq = quantize(up(rng.standard_normal((1, 4, 64, 128))), 64, 4)
    same = sdpa_dual_v_q4(q, kq, vq, vq, 128 ** -0.5)
    assert torch.equal(same[..., :128], same[..., 128:])
    vo = quantize(up(rng.standard_normal((1, 4, 64, 128))), 64, 4)
    diff = sdpa_dual_v_q4(q, kq, vq, vo, 128 ** -0.5)
    assert not torch.allclose(diff[..., :128], diff[..., 128:], atol=1e-3)


@pytest.mark.parametrize("B,H_q,H_kv,cap,kv_len,d", [(1, 8, 8, 256, 1, 128), (1, 8, 8, 256, 100, 128),
                                                     (1, 32, 8, 256, 100, 128), (1, 40, 8, 512, 385, 128)])
@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("dtype", ["float16", "bfloat16"])
def test_sdpa_dual_v_q4_runtime_kv_len_poisoned(cuda, B, H_q, H_kv, cap, kv_len, d, bits, dtype):
    from mlx_motif.kernels import sdpa_dual_v_q4
    from mlx_motif.quantization import quantize

    rng = np.random.default_rng(9)
    q = rounded(rng.standard_normal((B, H_q, 1, d)), dtype)
    full = rounded(rng.standard_normal((B, H_kv, cap, d)), dtype)
    full[..., kv_len:, :] = 1e3
    tf = up(full, dtype)
    kq, v1q, v2q = quantize(tf, 64, bits), quantize(tf * 0.5, 64, bits), quantize(tf * -0.25, 64, bits)
    got = sdpa_dual_v_q4(up(q, dtype), kq, v1q, v2q, d ** -0.5, 64, bits, kv_len=kv_len)
    ref = O.sdpa_dual_v_q4_reference(q, _np_triple(kq), _np_triple(v1q), _np_triple(v2q), d ** -0.5, 64, bits,
                                     kv_len)
    assert_close(down(got), ref, dtype, what="q4 poisoned")


def test_sdpa_dual_v_q4_growing_kv_len(cuda):
    from mlx_motif.kernels import sdpa_dual_v_q4
    from mlx_motif.quantization import quantize

    rng = np.random.default_rng(13)
    q = up(rng.standard_normal((1, 32, 1, 128)))
    full = up(rng.standard_normal((1, 8, 256, 128)))
    kq, v1q, v2q = quantize(full, 64, 4), quantize(full * 0.5, 64, 4), quantize(full * -0.25, 64, 4)
    qn = down(q)
    for kv_len in (1, 31, 32, 33, 100, 255, 256):
        got = sdpa_dual_v_q4(q, kq, v1q, v2q, 128 ** -0.5, 64, 4, kv_len=kv_len)
        ref = O.sdpa_dual_v_q4_reference(qn, _np_triple(kq), _np_triple(v1q), _np_triple(v2q), 128 ** -0.5, 64,
                                         4, kv_len)
        assert_close(down(got), ref, "float16", what=f"kv_len={kv_len}")


@pytest.mark.parametrize("D,bits", [(256, 8), (512, 4)])
def test_sdpa_dual_v_q4_rejects_out_of_contract_head_dim(cuda, D, bits):
    from mlx_motif.kernels import sdpa_dual_v_q4
    from mlx_motif.quantization import quantize

    q = torch.randn(1, 4, 1, D, device=cuda, dtype=torch.float16)
    kq = quantize(torch.randn(1, 4, 64, D, device=cuda, dtype=torch.float16), 128, bits)
    with pytest.raises(AssertionError, match=r"D/32 <= 32/bits"):
        sdpa_dual_v_q4(q, kq, kq, kq, D ** -0.5, group_size=128, bits=bits)


@pytest.mark.parametrize("D,bits", [(96, 8), (96, 4), (160, 4)])
def test_sdpa_dual_v_q4_rejects_word_straddling_head_dim(cuda, D, bits):
    from mlx_motif.kernels import sdpa_dual_v_q4
    from mlx_motif.quantization import quantize

    q = torch.randn(1, 4, 1, D, device=cuda, dtype=torch.float16)
    kq = quantize(torch.randn(1, 4, 64, D, device=cuda, dtype=torch.float16), 32, bits)
    with pytest.raises(AssertionError, match=r"qk_per_thread \| EL_PER_INT"):
        sdpa_dual_v_q4(q, kq, kq, kq, D ** -0.5, group_size=32, bits=bits)


@pytest.mark.parametrize("group_size", [32, 64, 128])
@pytest.mark.parametrize("bits", [4, 8])
def test_sdpa_dual_v_q4_accepts_shipped_shape_boundaries(cuda, group_size, bits):
    from mlx_motif.kernels import sdpa_dual_v_q4

    rng = np.random.default_rng(0)
    q, (kq, v1q, v2q) = _q_inputs(rng, 1, 4, 4, 64, 128, bits, "float16", gs=group_size)
    got = sdpa_dual_v_q4(up(q), kq, v1q, v2q, 128 ** -0.5, group_size=group_size, bits=bits)
    ref = O.sdpa_dual_v_q4_reference(q, _np_triple(kq), _np_triple(v1q), _np_triple(v2q), 128 ** -0.5,
                                     group_size, bits)
    assert_close(down(got), ref, "float16", what="boundaries")
