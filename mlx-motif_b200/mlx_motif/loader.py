"""MLX-format Motif checkpoints -> ``MotifDecoder``.

Reads what the reference's converter writes and its loader consumes
(``src/mlx_motif/loader.py:96-124``, ``convert.py:246-279``): ``config.json``
with a ``quantization`` block (``group_size``, ``bits``), and ``model.safetensors``
or shards listed in ``model.safetensors.index.json``. Every ``nn.Linear`` is an
MLX affine-quantized triple ``<name>.weight`` (uint32 words), ``.scales``,
``.biases``; embeddings and norms are dense; the λ vectors are fp32
(``convert.py:246-249``). Parameter names follow the reference modules
(``model.py:212-231, 385-458, 845-905``).

The safetensors container is parsed directly (an 8-byte little-endian header
length, a JSON header of ``{name: {dtype, shape, data_offsets}}``, then the raw
bytes), so no extra package is needed; tensors are memory-mapped and copied once
to the device.

Fusion mirrors ``Model.fuse_qkv`` (``model.py:994-1079``): q, k and v rows are
concatenated into one linear, and for the grouped model the q rows are permuted
from the checkpoint's head stripes ``[g0_o1 .. g0_o<gr>, g0_n, g1_o1, ..]`` to
origin-first. gate and up are concatenated the same way (one GEMV). Scales,
biases, embeddings and norms are held in fp16, the decoder's activation type.
"""

from __future__ import annotations

import json
import struct
from pathlib import Path

import numpy as np
import torch

from .model import ModelArgs, MotifDecoder, origin_first_perm

_DTYPES = {
    "F16": (np.float16, None),
    "BF16": (np.uint16, torch.bfloat16),
    "F32": (np.float32, None),
    "U32": (np.uint32, None),
    "I32": (np.int32, None),
    "U8": (np.uint8, None),
    "I64": (np.int64, None),
}
_NAMES = {np.dtype(np.float16): "F16", np.dtype(np.float32): "F32", np.dtype(np.uint32): "U32",
          np.dtype(np.int32): "I32", np.dtype(np.uint8): "U8", np.dtype(np.int64): "I64"}


def read_safetensors(path) -> dict[str, torch.Tensor]:
    """All tensors of one safetensors file as CPU torch tensors (bf16 kept as bf16)."""
    path = Path(path)
    with open(path, "rb") as f:
        n = struct.unpack("<Q", f.read(8))[0]
        header = json.loads(f.read(n))
    base = 8 + n
    raw = np.memmap(path, dtype=np.uint8, mode="r")
    out = {}
    for name, meta in header.items():
        if name == "__metadata__":
            continue
        np_dtype, torch_view = _DTYPES[meta["dtype"]]
        b, e = meta["data_offsets"]
        arr = np.array(raw[base + b : base + e]).view(np_dtype).reshape(meta["shape"])
        t = torch.from_numpy(arr)
        out[name] = t.view(torch_view) if torch_view is not None else t
    return out


def write_safetensors(path, tensors: dict[str, torch.Tensor], metadata: dict | None = None) -> None:
    """Write CPU tensors in the safetensors layout (bf16 supported)."""
    header, chunks, off = {}, [], 0
    for name, t in tensors.items():
        t = t.detach().contiguous().cpu()
        if t.dtype == torch.bfloat16:
            arr, code = t.view(torch.uint16).numpy(), "BF16"
        else:
            arr = t.numpy()
            code = _NAMES[arr.dtype]
        data = arr.tobytes()
        header[name] = {"dtype": code, "shape": list(arr.shape), "data_offsets": [off, off + len(data)]}
        chunks.append(data)
        off += len(data)
    if metadata:
        header["__metadata__"] = {str(k): str(v) for k, v in metadata.items()}
    hb = json.dumps(header).encode()
    hb += b" " * ((8 - len(hb) % 8) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(hb)))
        f.write(hb)
        for c in chunks:
            f.write(c)


def load_tensors(model_dir) -> dict[str, torch.Tensor]:
    """``model.safetensors`` or every shard named by ``model.safetensors.index.json``."""
    d = Path(model_dir)
    index = d / "model.safetensors.index.json"
    if index.exists():
        files = sorted(set(json.loads(index.read_text())["weight_map"].values()))
    else:
        files = sorted(p.name for p in d.glob("*.safetensors"))
    if not files:
        raise FileNotFoundError(f"no safetensors files in {d}")
    tensors = {}
    for fn in files:
        tensors.update(read_safetensors(d / fn))
    return {k: v for k, v in tensors.items() if "rotary_emb.inv_freq" not in k and "rope.inv_freq" not in k}


def args_from_config(cfg: dict) -> ModelArgs:
    """``ModelArgs`` from a converted ``config.json`` (unknown keys ignored, as ``ModelArgs.from_dict``)."""
    return ModelArgs.from_dict(cfg)


def _f16(t: torch.Tensor) -> torch.Tensor:
    return t.to(torch.float16)


def _triple(tensors: dict, prefix: str):
    w = tensors[prefix + ".weight"]
    if w.dtype not in (torch.int32, torch.uint32):
        raise ValueError(f"{prefix}: expected a quantized linear (uint32 weight), got {w.dtype}")
    return w.view(torch.int32), _f16(tensors[prefix + ".scales"]), _f16(tensors[prefix + ".biases"])


def _cat(*triples):
    return tuple(torch.cat([t[i] for t in triples], dim=0) for i in range(3))


def decoder_weights(tensors: dict, args: ModelArgs) -> dict:
    """Checkpoint tensors -> the ``MotifDecoder`` weights dict (CPU tensors): fused, origin-first qkv,
    fused gate|up, fp16 scales/biases/norms/embedding, λ_full from the four λ vectors."""
    from .model import lambda_full, lambda_init_for_layer

    layers = []
    d = args.d
    for i in range(args.num_hidden_layers):
        p = f"model.layers.{i}."
        q = _triple(tensors, p + "self_attn.q_proj")
        if args.is_grouped:
            perm = origin_first_perm(args.num_noise_heads, args.grouped_ratio, d)
            q = tuple(t[perm] for t in q)
        qkv = _cat(q, _triple(tensors, p + "self_attn.k_proj"), _triple(tensors, p + "self_attn.v_proj"))
        gate_up = _cat(_triple(tensors, p + "mlp.gate_proj"), _triple(tensors, p + "mlp.up_proj"))
        lam_init = lambda_init_for_layer(i)
        lq = [tensors[p + f"self_attn.lambda_{n}"].float() for n in ("q1", "k1", "q2", "k2")]
        layers.append(dict(
            input_norm=_f16(tensors[p + "input_layernorm.weight"]),
            post_norm=_f16(tensors[p + "post_attention_layernorm.weight"]),
            qkv=qkv,
            o=_triple(tensors, p + "self_attn.o_proj"),
            gate_up=gate_up,
            down=_triple(tensors, p + "mlp.down_proj"),
            subln=_f16(tensors[p + "self_attn.subln.weight"]),
            lambda_init=lam_init,
            lambda_full=lambda_full(*lq, lam_init),
            polynorm_w=_f16(tensors.get(p + "mlp.act_fn.weight", torch.full((3,), 1 / 3))),
            polynorm_b=_f16(tensors.get(p + "mlp.act_fn.bias", torch.zeros(1))),
        ))
    if "lm_head.weight" in tensors:
        lm_head = _triple(tensors, "lm_head")
    else:
        raise NotImplementedError("tied word embeddings: the lm_head GEMV needs a q4 lm_head "
                                  "(the checkpoint keeps only the dense embedding)")
    return dict(embed=_f16(tensors["model.embed_tokens.weight"]), final_norm=_f16(tensors["model.norm.weight"]),
                lm_head=lm_head, layers=layers)


def load(path, device="cuda", cache: str = "fp16", max_seq: int = 4096) -> MotifDecoder:
    """Load a converted MLX Motif checkpoint directory into a ``MotifDecoder`` (the reference's
    ``load(path, fuse_qkv=True)`` model half; tokenization stays with the caller)."""
    d = Path(path)
    cfg = json.loads((d / "config.json").read_text())
    q = cfg.get("quantization") or {}
    if q.get("bits") != 4 or q.get("group_size") != 64:
        raise ValueError(f"the decode kernels take q4 group-64 linears; checkpoint has {q}")
    args = args_from_config(cfg)
    weights = decoder_weights(load_tensors(d), args)
    from .linear import QuantizedLinear

    dev = torch.device(device)

    def ql(t):
        return QuantizedLinear(t[0].view(torch.uint32).to(dev), t[1].to(dev), t[2].to(dev))

    for L in weights["layers"]:
        for k in ("qkv", "o", "gate_up", "down"):
            L[k] = ql(L[k])
    weights["lm_head"] = ql(weights["lm_head"])
    return MotifDecoder(args, weights, cache=cache, max_seq=max_seq, device=dev)
