"""The allocation-free attention entry point (``motif_sdpa_dual_v_static``).

It serves callers that cannot allocate device memory — a plugin whose memory
belongs to its host framework's allocator, or a hot path that must not pay
cudaMalloc's device-wide synchronisation — by keeping the split-KV partials in one
static device array instead of a caller workspace. These tests call it through
the C ABI and hold it to the regular ``motif_sdpa_dual_v`` (which takes a
caller workspace) on two calls in a row, then check the size limit.

The file is named to be collected last, so a run that stops at the first
failure has already run every other test.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import assert_close

pytestmark = pytest.mark.gpu


def _inputs(rng, B, H_q, H_kv, cap, D, dev):
    q = torch.from_numpy(rng.standard_normal((B, H_q, 1, D)).astype(np.float32) * 0.3).half().to(dev)
    k, v1, v2 = (torch.from_numpy(rng.standard_normal((B, H_kv, cap, D)).astype(np.float32) * 0.5).half().to(dev)
                 for _ in range(3))
    return q, k, v1, v2


def _regular(N, q, k, v1, v2, kv_len, dev):
    B, H_q, _, D = q.shape
    H_kv, cap = k.shape[1], k.shape[2]
    y = torch.empty((B, H_q, 1, 2 * D), dtype=torch.float16, device=dev)
    ws_bytes = N.lib.motif_sdpa_dual_v_workspace_bytes(B, H_q, D, 64)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
    N.check(N.lib.motif_sdpa_dual_v(0, q.data_ptr(), k.data_ptr(), v1.data_ptr(), v2.data_ptr(), D ** -0.5, B, H_q,
                                    H_kv, cap, D, kv_len, None, y.data_ptr(), ws.data_ptr(), ws_bytes, N.stream()))
    return y


def _static(N, q, k, v1, v2, kv_len, dev):
    B, H_q, _, D = q.shape
    H_kv, cap = k.shape[1], k.shape[2]
    y = torch.empty((B, H_q, 1, 2 * D), dtype=torch.float16, device=dev)
    N.check(N.lib.motif_sdpa_dual_v_static(0, q.data_ptr(), k.data_ptr(), v1.data_ptr(), v2.data_ptr(), D ** -0.5,
                                           B, H_q, H_kv, cap, D, kv_len, None, y.data_ptr(), N.stream()))
    return y


def test_static_scratch_entry_matches_workspace_entry_twice(cuda):
    from mlx_motif import _native as N

    assert N.lib.motif_sdpa_dual_v_static_scratch_bytes() == 4 << 20
    rng = np.random.default_rng(21)
    # Two calls in a row with different shapes and lengths: the second reuses the
    # array the first one left behind (nothing in it needs to start at zero).
    for (B, H_q, H_kv, cap, D, kv_len) in [(1, 24, 8, 2048, 128, 1500), (2, 16, 4, 1024, 64, 333)]:
        q, k, v1, v2 = _inputs(rng, B, H_q, H_kv, cap, D, cuda)
        got = _static(N, q, k, v1, v2, kv_len, cuda)
        ref = _regular(N, q, k, v1, v2, kv_len, cuda)
        torch.cuda.synchronize()
        assert_close(got.float().cpu().numpy(), ref.float().cpu().numpy(), "float16",
                     what=f"static vs workspace entry B={B} H_q={H_q} kv_len={kv_len}")


def test_static_scratch_entry_rejects_shapes_beyond_the_array(cuda):
    from mlx_motif import _native as N

    q = torch.zeros(8, dtype=torch.float16, device=cuda)
    # 16 x 128 query rows at D=128 need 16*128*258*4*2 bytes (~4.2 MB) for two splits.
    rc = N.lib.motif_sdpa_dual_v_static(0, q.data_ptr(), q.data_ptr(), q.data_ptr(), q.data_ptr(), 0.1, 16, 128, 16,
                                        64, 128, 64, None, q.data_ptr(), N.stream())
    assert rc == N.ERR_WORKSPACE
    assert b"static array" in N.lib.motif_last_error()
