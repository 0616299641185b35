"""The C-ABI library loads, exports every symbol include/*.h declares, and rejects bad
arguments with status codes before touching a GPU (runs on CPU)."""

from __future__ import annotations

import ctypes as C
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent


def _declared():
    names = set()
    for h in (ROOT / "include").glob("*.h"):
        names |= set(re.findall(r"^MOTIF_API\s+[\w\s\*]+?\b(motif_\w+)\s*\(", h.read_text(), flags=re.M))
    return names


def test_library_exports_every_declared_symbol():
    from mlx_motif import _native as N

    declared = _declared()
    assert len(declared) >= 20
    lib = C.CDLL(str(N.LIB_PATH))
    missing = [n for n in sorted(declared) if not hasattr(lib, n)]
    assert not missing, f"declared but not exported: {missing}"
    assert declared == set(N.SIGNATURES), "ctypes signature table and header disagree"


def test_status_strings_and_version():
    from mlx_motif import _native as N

    assert N.lib.motif_abi_version() == 3  # motif_argmax_key_exchange added
    assert N.lib.motif_status_string(0) == b"ok"
    assert N.lib.motif_status_string(3) == b"shape outside kernel contract"


def test_null_and_shape_errors_need_no_gpu():
    from mlx_motif import _native as N

    rc = N.lib.motif_polynorm(0, None, None, None, 1e-6, 1, 8, None, None)
    assert rc == N.ERR_NULL and b"null" in N.lib.motif_last_error()
    rc = N.lib.motif_sdpa_dual_v_q(0, 8, 128, 1, 1, 1, 1, 1, 1, 1, 1, 1, 1, 0.1, 1, 4, 4, 64, 256, 64, None, 1,
                                   None, 0, None)
    assert rc == N.ERR_BAD_CONTRACT
    assert b"D/32 <= 32/bits" in N.lib.motif_last_error()
    rc = N.lib.motif_sdpa_dual_v_q(0, 4, 32, 1, 1, 1, 1, 1, 1, 1, 1, 1, 1, 0.1, 1, 4, 4, 64, 96, 64, None, 1,
                                   None, 0, None)
    assert rc == N.ERR_BAD_CONTRACT and b"qk_per_thread | EL_PER_INT" in N.lib.motif_last_error()
    rc = N.lib.motif_sdpa_dual_v(0, 1, 1, 1, 1, 0.1, 1, 6, 4, 64, 128, 10, None, 1, None, 0, None)
    assert rc == N.ERR_BAD_CONTRACT and b"multiple of H_kv" in N.lib.motif_last_error()
    rc = N.lib.motif_sdpa_dual_v(0, 1, 1, 1, 1, 0.1, 1, 8, 4, 64, 128, 65, None, 1, None, 0, None)
    assert rc == N.ERR_BAD_SHAPE and b"kv_len=65" in N.lib.motif_last_error()
    rc = N.lib.motif_quantize(0, 3, 64, 1, 1, 64, 1, 1, 1, None)
    assert rc == N.ERR_DTYPE
    rc = N.lib.motif_gda_post_split(0, 1, 1, 1, 1, 5, 0.5, 1, 8, 3, 1, 256, 1e-5, 1, None)
    assert rc == N.ERR_BAD_SHAPE and b"lambda_full has 5 values" in N.lib.motif_last_error()
    rc = N.lib.motif_argmax(0, 1, 100, 1, 1, 0, None)
    assert rc == N.ERR_WORKSPACE


def test_python_layer_maps_contract_errors_to_assertion():
    from mlx_motif import _native as N

    with pytest.raises(AssertionError, match="qk_per_thread"):
        N.check(N.lib.motif_sdpa_dual_v_q(0, 4, 32, 1, 1, 1, 1, 1, 1, 1, 1, 1, 1, 0.1, 1, 4, 4, 64, 96, 64, None,
                                          1, None, 0, None), "sdpa_dual_v_q4")
    with pytest.raises(ValueError):
        N.check(N.ERR_NULL)
    with pytest.raises(N.MotifError):
        N.check(N.ERR_CUDA)


def test_workspace_queries():
    from mlx_motif import _native as N

    assert N.lib.motif_sdpa_dual_v_workspace_bytes(1, 32, 128, 10) == 4 * 32 * 10 * 258
    assert N.lib.motif_quantized_linear_workspace_bytes(1, 4096, 14336, 4, 64) > 0
    # stream-K: tiles split across warps need partials + counters, a single K block never does
    assert N.lib.motif_quantized_linear_workspace_bytes(1, 219520, 4096, 4, 64) > 0
    assert N.lib.motif_quantized_linear_workspace_bytes(1, 4096, 512, 4, 64) == 0
    assert N.lib.motif_linear_fused_workspace_bytes(8192, 4096) > 0
    assert N.lib.motif_argmax_workspace_bytes(219520) >= 8


def _fake_slots(bits: int, capacity: int, heads: int = 8, base: int = 1 << 20):
    """A 4-slot view over fake, 16-byte aligned addresses (the query never dereferences them)."""
    from mlx_motif import _native as N

    s = N.motif_kv4_slots()
    for i in range(4):
        s.data[i] = base + i * (1 << 28)
        s.scales[i] = None if bits == 16 else base + (4 + i) * (1 << 28)
        s.biases[i] = None if bits == 16 else base + (8 + i) * (1 << 28)
    s.bits, s.group_size, s.batch, s.heads, s.capacity, s.head_dim = bits, 64, 1, heads, capacity, 128
    return s


def test_decode_step_kernel_query(monkeypatch):
    """The decode step's kernel choice, answered without a GPU: the tensor-core step for long fp16
    caches and for q4 caches whose capacity is a multiple of 4; the CUDA-core split step below
    the length threshold, for q8, and for a q4 capacity the tensor-core tiles cannot address."""
    from mlx_motif import _native as N

    monkeypatch.delenv("MOTIF_LONG_ATTN_MIN_CAP", raising=False)
    q = N.lib.motif_decode_step_kernel
    assert q(_fake_slots(16, 16128)) == N.ATTN_KERNEL_TCGEN05
    assert q(_fake_slots(4, 16128)) == N.ATTN_KERNEL_TCGEN05
    assert q(_fake_slots(4, 16033)) == N.ATTN_KERNEL_SPLIT  # a raw, unrounded capacity
    assert q(_fake_slots(8, 16128)) == N.ATTN_KERNEL_SPLIT
    assert q(_fake_slots(16, 512)) == N.ATTN_KERNEL_SPLIT
    bad = _fake_slots(16, 4096)
    bad.data[2] = (1 << 20) + 8  # not 16-byte aligned: no TMA
    assert q(bad) == N.ATTN_KERNEL_SPLIT
    monkeypatch.setenv("MOTIF_LONG_ATTN_MIN_CAP", "0")
    assert q(_fake_slots(16, 512)) == N.ATTN_KERNEL_TCGEN05
    wrong = _fake_slots(16, 4096)
    wrong.head_dim = 64
    assert q(wrong) < 0
    assert q(None) == -N.ERR_NULL


def test_preallocated_capacity_rounds_to_whole_steps():
    """max_size preallocation rounds the capacity up to whole 256-row steps (the reference's
    growth unit), so a bench or decoder sizing the cache as prompt + steps + margin (16033 rows)
    still gets a capacity the tensor-core q4 step takes."""
    import torch

    from mlx_motif.cache import MotifGroupedKVCache, MotifGroupedQuantizedKVCache

    c = MotifGroupedQuantizedKVCache(64, 4, max_size=16033)
    c._grow(1, 8, 1, 128, torch.float16, "cpu")
    assert c.k1[0].shape == (1, 8, 16128, 16) and c.k1[1].shape == (1, 8, 16128, 2)
    f = MotifGroupedKVCache(max_size=256)
    f._grow(1, 8, 1, 128, torch.float16, "cpu")
    assert f.k1.shape[2] == 256
    with pytest.raises(ValueError, match="capacity 256 exceeded"):
        f.offset = 200
        f.k1 = None
        f._grow(1, 8, 100, 128, torch.float16, "cpu")
