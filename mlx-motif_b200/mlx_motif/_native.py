"""ctypes binding of the in-tree CUDA library (``libmotif_b200.so``).

The library is the only compute path of this package: if it is missing or
fails to load, importing ``mlx_motif`` raises immediately (there is no CPU or
eager fallback). Build it with ``python mlx-motif_b200/build_native.py``.

Status codes from the C ABI become Python exceptions with the reference's
error classes: shape-contract violations raise ``AssertionError`` (the
reference asserts its contracts, e.g. ``kernels/attention.py:556-608``),
other misuse ``ValueError``/``TypeError``, CUDA failures ``RuntimeError``.
"""

from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().parent / "libmotif_b200.so"

OK, ERR_NULL, ERR_BAD_SHAPE, ERR_BAD_CONTRACT, ERR_DTYPE, ERR_CUDA, ERR_WORKSPACE = range(7)
F16, BF16, F32 = 0, 1, 2
ATTN_KERNEL_SPLIT, ATTN_KERNEL_TCGEN05 = 1, 2
ATTN_KERNEL_NAMES = {ATTN_KERNEL_SPLIT: "split", ATTN_KERNEL_TCGEN05: "tcgen05"}

_DTYPE_CODES = {torch.float16: F16, torch.bfloat16: BF16, torch.float32: F32}


class motif_kv4_slots(C.Structure):  # noqa: N801 — mirrors the C struct name
    _fields_ = [
        ("data", C.c_void_p * 4),
        ("scales", C.c_void_p * 4),
        ("biases", C.c_void_p * 4),
        ("bits", C.c_int32),
        ("group_size", C.c_int32),
        ("batch", C.c_int64),
        ("heads", C.c_int64),
        ("capacity", C.c_int64),
        ("head_dim", C.c_int64),
    ]


class motif_linear_io(C.Structure):  # noqa: N801 — mirrors the C struct name
    _fields_ = [
        ("mode", C.c_int32),
        ("x", C.c_void_p),
        ("h_in", C.c_void_p),
        ("token", C.c_void_p),
        ("embed", C.c_void_p),
        ("vocab", C.c_int64),
        ("delta", C.c_void_p),
        ("h_out", C.c_void_p),
        ("norm_w", C.c_void_p),
        ("eps", C.c_float),
        ("gate", C.c_void_p),
        ("up", C.c_void_p),
        ("stats", C.c_void_p),
        ("stats_count", C.c_int64),
        ("poly_w", C.c_void_p),
        ("poly_b", C.c_void_p),
        ("poly_eps", C.c_float),
        ("poly_dim", C.c_int64),
        ("stats_out", C.c_void_p),
        ("stats_rows", C.c_int64),
        ("argmax_out", C.c_void_p),
        ("pos_len_inc", C.c_void_p),
        ("argmax_key_out", C.c_void_p),
        ("argmax_row_offset", C.c_int64),
        ("tp_world", C.c_int32),
        ("tp_seq", C.c_void_p),
        ("tp_tag", C.c_int32),
        ("tp_out", C.c_void_p * 8),
        ("tp_stats", C.c_void_p * 8),
        ("tp_in", C.c_void_p),
        ("tp_stats_in", C.c_void_p),
    ]


_P, _I, _L, _F, _S = C.c_void_p, C.c_int, C.c_int64, C.c_float, C.c_size_t
_KV = C.POINTER(motif_kv4_slots)
_IO = C.POINTER(motif_linear_io)

# name -> (restype, argtypes); every symbol of include/motif_b200.h.
SIGNATURES = {
    "motif_status_string": (C.c_char_p, [_I]),
    "motif_last_error": (C.c_char_p, []),
    "motif_abi_version": (_I, []),
    "motif_polynorm": (_I, [_I, _P, _P, _P, _F, _L, _L, _P, _P]),
    "motif_polynorm_mul": (_I, [_I, _P, _P, _L, _P, _P, _F, _L, _L, _P, _P]),
    "motif_gda_post_split": (_I, [_I, _P, _P, _P, _P, _L, _F, _L, _L, _L, _L, _L, _F, _P, _P]),
    "motif_gda_post": (_I, [_I, _P, _P, _P, _L, _F, _L, _L, _L, _L, _L, _F, _P, _P]),
    "motif_sdpa_dual_v_workspace_bytes": (_S, [_L, _L, _L, _L]),
    "motif_sdpa_dual_v": (_I, [_I, _P, _P, _P, _P, _F, _L, _L, _L, _L, _L, _L, _P, _P, _P, _S, _P]),
    "motif_sdpa_dual_v_static_scratch_bytes": (_S, []),
    "motif_sdpa_dual_v_static": (_I, [_I, _P, _P, _P, _P, _F, _L, _L, _L, _L, _L, _L, _P, _P, _P]),
    "motif_sdpa_dual_v_q": (
        _I,
        [_I, _I, _I, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _F, _L, _L, _L, _L, _L, _L, _P, _P, _P, _S, _P],
    ),
    "motif_gda_decode_attention_workspace_bytes": (_S, [_L, _L, _L]),
    "motif_gda_decode_step_workspace_bytes": (_S, [_L, _L, _L]),
    "motif_gda_decode_step": (
        _I,
        [_P, _P, _KV, _P, _F, _L, _L, _P, _P, _L, _F, _F, _P, _P, _S, _P],
    ),
    "motif_q4_gemm": (_I, [_P, _L, _L, _P, _P, _P, _L, _P, _P, _P, _P]),
    "motif_sample": (_I, [_P, _L, _L, _L, _F, C.c_uint64, _P, _L, C.c_uint32, _P, _P, _P]),
    "motif_speculative_accept": (_I, [_P, _P, _L, _P, _L, _L, _F, C.c_uint64, _P, _L, _P, _P]),
    "motif_sample_key": (_I, [_P, _L, _F, C.c_uint64, _P, _L, C.c_uint32, _L, _P, _P]),
    "motif_embed_rms_norm_rows": (_I, [_I, _P, _L, _P, _L, _L, _P, _F, _P, _P, _P]),
    "motif_rope_qkv_append_rows": (_I, [_P, _L, _P, _L, _KV, _L, _P, _P, _P]),
    "motif_prefill_attention": (_I, [_P, _L, _L, _KV, _L, _I, _L, _F, _P, _P, _P]),
    "motif_polynorm_row_stats": (_I, [_I, _P, _L, _L, _L, _P, _P]),
    "motif_polynorm_mul_stats": (_I, [_I, _P, _P, _L, _P, _P, _F, _L, _L, _P, _L, _P, _P]),
    "motif_prefill_attention_split_workspace_bytes": (_S, [_L, _L]),
    "motif_prefill_attention_split": (_I, [_P, _L, _L, _KV, _L, _P, _I, _L, _F, _P, _P, _S, _P, _P]),
    "motif_prefill_post": (_I, [_P, _L, _L, _I, _L, _L, _P, _P, _L, _F, _F, _P, _P]),
    "motif_vanilla_decode_step": (
        _I,
        [_P, _P, _KV, _P, _F, _L, _L, _P, _P, _F, _F, _P, _P, _S, _P],
    ),
    "motif_decode_step_kernel": (_I, [_KV]),
    "motif_gda_decode_attention": (
        _I,
        [_P, _KV, _F, _L, _L, _L, _P, _P, _P, _L, _F, _F, _P, _P, _S, _P],
    ),
    "motif_quantize": (_I, [_I, _I, _I, _P, _L, _L, _P, _P, _P, _P]),
    "motif_dequantize": (_I, [_I, _I, _I, _P, _P, _P, _L, _L, _P, _P]),
    "motif_kv4_append": (_I, [_I, _KV, _P, _P, _P, _P, _L, _L, _P, _P]),
    "motif_rope_qkv_append": (_I, [_P, _P, _L, _KV, _P, _P, _P]),
    "motif_rope": (_I, [_I, _P, _L, _L, _L, _L, _L, _P, _P, _P, _P]),
    "motif_quantized_linear_workspace_bytes": (_S, [_L, _L, _L, _I, _I]),
    "motif_quantized_linear": (_I, [_I, _I, _I, _P, _L, _L, _P, _P, _P, _L, _P, _P, _S, _P]),
    "motif_linear_fused_workspace_bytes": (_S, [_L, _L]),
    "motif_linear_fused": (_I, [_IO, _P, _P, _P, _L, _L, _P, _P, _S, _P]),
    "motif_rms_norm": (_I, [_I, _P, _P, _F, _L, _L, _P, _P]),
    "motif_add_rms_norm": (_I, [_I, _P, _P, _P, _F, _L, _L, _P, _P]),
    "motif_embed_rms_norm": (_I, [_I, _P, _P, _L, _L, _P, _F, _P, _P, _P]),
    "motif_argmax_workspace_bytes": (_S, [_L]),
    "motif_argmax": (_I, [_I, _P, _L, _P, _P, _S, _P]),
    "motif_argmax_key_decode": (_I, [_P, _P, _P, _P]),
    "motif_argmax_key_exchange": (_I, [_P, _P, _I, _I, _P, _P, _P, _P, _P]),
    "motif_ipc_handle_bytes": (_S, []),
    "motif_ipc_alloc": (_I, [_S, C.POINTER(C.c_void_p), _P]),
    "motif_ipc_open": (_I, [_P, C.POINTER(C.c_void_p)]),
    "motif_ipc_close": (_I, [_P]),
    "motif_ipc_zero": (_I, [_P, _S, _P]),
    "motif_ipc_free": (_I, [_P]),
}


def _load():
    if not LIB_PATH.exists():
        raise ImportError(
            f"mlx_motif: CUDA library {LIB_PATH} is missing. Build it with "
            "`python mlx-motif_b200/build_native.py` (nvcc, sm_100a). There is no CPU fallback."
        )
    lib = C.CDLL(str(LIB_PATH))
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


lib = _load()


class MotifError(RuntimeError):
    """A CUDA-side failure reported by the C ABI."""


def check(rc: int, what: str = "") -> None:
    """Raise the reference-style exception for a non-OK status code."""
    if rc == OK:
        return
    msg = (lib.motif_last_error() or b"").decode(errors="replace")
    text = f"{what}: {msg}" if what else msg
    if rc in (ERR_BAD_CONTRACT, ERR_BAD_SHAPE):
        raise AssertionError(text)
    if rc in (ERR_NULL, ERR_WORKSPACE):
        raise ValueError(text)
    if rc == ERR_DTYPE:
        raise TypeError(text)
    raise MotifError(text)


def dtype_code(t: torch.Tensor) -> int:
    try:
        return _DTYPE_CODES[t.dtype]
    except KeyError:
        raise TypeError(f"unsupported dtype {t.dtype}; expected float16, bfloat16 or float32") from None


def ptr(t: torch.Tensor | None) -> int | None:
    """Device pointer of a CUDA tensor (None stays NULL)."""
    if t is None:
        return None
    if not t.is_cuda:
        raise ValueError("mlx_motif kernels take CUDA tensors (got a CPU tensor)")
    return t.data_ptr()


def stream(device: torch.device | None = None) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def contiguous(t: torch.Tensor) -> torch.Tensor:
    return t if t.is_contiguous() else t.contiguous()


def kernels_disabled() -> bool:
    """``MLX_MOTIF_DISABLE_KERNELS`` (read once at import, as ``kernels/_common.py:10``)."""
    return _DISABLE


_DISABLE = os.environ.get("MLX_MOTIF_DISABLE_KERNELS", "0") not in ("0", "", "false", "False")
