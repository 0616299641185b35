"""CPU checks of the MLX checkpoint loader: the safetensors container round trip (bf16, uint32,
fp32), config parsing, and the parameter-name mapping with fuse_qkv's origin-first q order
(``model.py:994-1079``), on a checkpoint written in the reference's names and layouts."""

from __future__ import annotations

import numpy as np
import torch

import oracle as O
from golden.checkpoint_fixture import build_checkpoint


def _args():
    return O.OracleArgs(hidden_size=256, num_hidden_layers=2, intermediate_size=512, num_noise_heads=8,
                        grouped_ratio=3, kv_heads_per_slot=8, head_dim=128, vocab_size=300)


def test_safetensors_round_trip(tmp_path):
    from mlx_motif.loader import read_safetensors, write_safetensors

    t = {"a": torch.randn(3, 5).to(torch.bfloat16), "b": torch.arange(12, dtype=torch.int32).view(torch.uint32)
         .reshape(3, 4), "c": torch.randn(7), "d": torch.randn(2, 2).half()}
    write_safetensors(tmp_path / "x.safetensors", t, metadata={"format": "mlx"})
    r = read_safetensors(tmp_path / "x.safetensors")
    assert set(r) == set(t)
    for k in t:
        assert r[k].dtype == t[k].dtype and r[k].shape == t[k].shape
        assert torch.equal(r[k].view(torch.uint8) if k != "b" else r[k].view(torch.int32),
                           t[k].view(torch.uint8) if k != "b" else t[k].view(torch.int32))


def test_checkpoint_mapping_and_fusion(tmp_path):
    from mlx_motif.loader import args_from_config, decoder_weights, load_tensors

    a = _args()
    w = build_checkpoint(tmp_path, O, a, seed=3)
    import json

    args = args_from_config(json.loads((tmp_path / "config.json").read_text()))
    assert args.is_grouped and args.q_heads == 32 and args.grouped_ratio == 3 and args.qkv_out == w["layers"][0]["qkv"][0].shape[0]
    tensors = load_tensors(tmp_path)
    dw = decoder_weights(tensors, args)
    for L, ref in zip(dw["layers"], w["layers"]):
        # fused qkv codes equal the oracle's origin-first fused rows bit for bit
        assert np.array_equal(L["qkv"][0].numpy(), ref["qkv"][0].view(np.int32))
        # scales/biases went bf16 -> fp16: within bf16 precision of the originals
        np.testing.assert_allclose(L["qkv"][1].float().numpy(), ref["qkv"][1].astype(np.float32), rtol=1e-2)
        gu = np.concatenate([ref["gate"][0], ref["up"][0]]).view(np.int32)
        assert np.array_equal(L["gate_up"][0].numpy(), gu)
        assert np.array_equal(L["down"][0].numpy(), ref["down"][0].view(np.int32))
        np.testing.assert_allclose(L["lambda_full"].numpy(), ref["lambda_full"], rtol=1e-6)
    assert dw["embed"].dtype == torch.float16 and dw["embed"].shape == (300, 256)
