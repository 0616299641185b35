"""A checkpoint written in the reference's MLX layout (un-fused projections, head-stripe q order,
separate gate/up, λ vectors) loads into a decoder whose logits match the oracle's forward of the
same weights at every greedy step."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle as O
from conftest import assert_close
from golden.checkpoint_fixture import build_checkpoint
from test_gpu_kernels import down

pytestmark = pytest.mark.gpu


def test_loaded_checkpoint_decodes_like_the_oracle(cuda, tmp_path):
    from mlx_motif.loader import load

    oa = O.OracleArgs(hidden_size=256, num_hidden_layers=3, intermediate_size=512, num_noise_heads=8,
                      grouped_ratio=3, kv_heads_per_slot=8, head_dim=128, vocab_size=1000)
    w = build_checkpoint(tmp_path, O, oa, seed=2, dense_dtype=torch.float16)
    dec = load(tmp_path, device=cuda, cache="fp16", max_seq=256)
    orc = O.GroupedDecodeOracle(oa, w, cache="fp16")
    prompt = [7, 99, 512, 3]
    tok = None
    for i in range(len(prompt) + 6):
        t_in = prompt[i] if i < len(prompt) else tok
        dec.token.fill_(int(t_in))
        dec.step_device(with_head=True)
        logits_ref, tok_ref = orc.step(t_in)
        assert_close(down(dec.logits), logits_ref.astype(np.float64), "float16", what=f"step {i} logits")
        tok = int(dec.token.item())
        assert tok == tok_ref


def test_loader_rejects_other_quantization(tmp_path):
    import json

    from mlx_motif.loader import load

    (tmp_path / "config.json").write_text(json.dumps({"hidden_size": 256, "quantization": {"bits": 8,
                                                                                          "group_size": 64}}))
    with pytest.raises(ValueError, match="q4 group-64"):
        load(tmp_path)
