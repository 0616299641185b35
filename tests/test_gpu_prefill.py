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
                                   (517, 2048, 8192)])
def test_q4_gemm_matches_oracle(cuda, M, N, K):
    """motif_q4_gemm (tcgen05) == oracle quantized_matmul (fp64 of the dequantized weights),
    fp16 tolerance; rows past M are never written; the error word stays 0."""
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
