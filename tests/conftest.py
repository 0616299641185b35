"""Test configuration: import paths, the `gpu` marker, shared tolerances.

`-m "not gpu"` runs the oracle checks, host logic and the C-ABI load/export
checks on CPU; `-m gpu` runs the CUDA parity tests (they call the C ABI
through the `mlx_motif` package and compare with the CPU oracle).
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent
PKG = ROOT / "mlx-motif_b200"
for p in (str(ROOT), str(PKG)):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")
    lib = PKG / "mlx_motif" / "libmotif_b200.so"
    if not lib.exists():
        sys.path.insert(0, str(PKG))
        import build_native

        build_native.build()


# North-star tolerance for fp16 outputs: max-abs 2e-3 / rel 1e-2 (elementwise
# |got - ref| <= atol + rtol·|ref|). bf16 and fp32 use the reference's own
# test tolerances (5e-2 and 1e-4).
TOL = {"float16": (2e-3, 1e-2), "bfloat16": (5e-2, 5e-2), "float32": (1e-4, 1e-4)}


def assert_close(got, ref, dtype_name: str, atol=None, rtol=None, what: str = ""):
    a, r = TOL[dtype_name]
    atol = a if atol is None else atol
    rtol = r if rtol is None else rtol
    got = np.asarray(got, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    assert got.shape == ref.shape, f"{what}: shape {got.shape} != {ref.shape}"
    err = np.abs(got - ref)
    bound = atol + rtol * np.abs(ref)
    bad = err > bound
    assert not bad.any(), (
        f"{what}: {int(bad.sum())} of {bad.size} outside atol={atol} rtol={rtol}; "
        f"max abs err {err.max():.3e}, worst excess {(err - bound).max():.3e}"
    )


@pytest.fixture(scope="session")
def cuda():
    import torch

    if not torch.cuda.is_available():
        pytest.fail("no CUDA device: GPU tests need a B200 (sm_100a)")
    return torch.device("cuda:0")


@pytest.fixture(autouse=True)
def _short_attention_path_by_default(monkeypatch, request):
    """Tests written for the CUDA-core decode step (bit-exact comparisons) keep it at every cache
    capacity; the long-cache tensor-core step has its own tests, which set the threshold."""
    if "long_attn" not in request.node.nodeid and "bench" not in request.node.nodeid:
        monkeypatch.setenv("MOTIF_LONG_ATTN_MIN_CAP", str(1 << 40))
