"""Build a small MLX-format Motif checkpoint directory from the oracle's synthetic weights, in the
reference's parameter names and layouts (un-fused q/k/v in the checkpoint's head-stripe q order,
separate gate/up, fp32 λ vectors, bf16 or fp16 dense tensors), for the loader tests."""

from __future__ import annotations

import json

import numpy as np
import torch


def _lam_vectors(rng, d):
    return [(rng.standard_normal(d) * 0.1).astype(np.float32) for _ in range(4)]


def build_checkpoint(out_dir, O, args, seed: int = 0, dense_dtype=torch.bfloat16):
    """Write config.json + two safetensors shards + index; return the oracle weights that the
    checkpoint encodes (λ_full recomputed from the λ vectors written)."""
    from mlx_motif.loader import write_safetensors
    from mlx_motif.model import origin_first_perm

    w = O.make_synthetic_weights(args, seed=seed, std=0.05)
    rng = np.random.default_rng(seed + 1)
    d = args.head_dim
    G, gr = args.num_noise_heads, args.grouped_ratio
    qd = (gr + 1) * G * d
    kd = 2 * args.kv_heads_per_slot * d
    inv = torch.argsort(origin_first_perm(G, gr, d)).numpy()  # origin-first -> head stripes

    def trip(name, t, out):
        dd, ss, bb = t
        out[name + ".weight"] = torch.from_numpy(np.ascontiguousarray(dd).view(np.uint32))
        out[name + ".scales"] = torch.from_numpy(np.ascontiguousarray(ss)).to(dense_dtype)
        out[name + ".biases"] = torch.from_numpy(np.ascontiguousarray(bb)).to(dense_dtype)

    shards = [{}, {}]
    for i, L in enumerate(w["layers"]):
        t = shards[i % 2]
        p = f"model.layers.{i}."
        dq, sq, bq = L["qkv"]
        q = (dq[:qd][inv], sq[:qd][inv], bq[:qd][inv])
        k = (dq[qd:qd + kd], sq[qd:qd + kd], bq[qd:qd + kd])
        v = (dq[qd + kd:], sq[qd + kd:], bq[qd + kd:])
        trip(p + "self_attn.q_proj", q, t)
        trip(p + "self_attn.k_proj", k, t)
        trip(p + "self_attn.v_proj", v, t)
        trip(p + "self_attn.o_proj", L["o"], t)
        trip(p + "mlp.gate_proj", L["gate"], t)
        trip(p + "mlp.up_proj", L["up"], t)
        trip(p + "mlp.down_proj", L["down"], t)
        lv = _lam_vectors(rng, d)
        for n, a in zip(("q1", "k1", "q2", "k2"), lv):
            t[p + f"self_attn.lambda_{n}"] = torch.from_numpy(a)
        L["lambda_full"] = np.array([O.lambda_full(*lv, L["lambda_init"])], np.float32)
        t[p + "self_attn.subln.weight"] = torch.from_numpy(L["subln"]).to(dense_dtype)
        t[p + "input_layernorm.weight"] = torch.from_numpy(L["input_norm"]).to(dense_dtype)
        t[p + "post_attention_layernorm.weight"] = torch.from_numpy(L["post_norm"]).to(dense_dtype)
        t[p + "mlp.act_fn.weight"] = torch.from_numpy(L["polynorm_w"]).to(dense_dtype)
        t[p + "mlp.act_fn.bias"] = torch.from_numpy(L["polynorm_b"]).to(dense_dtype)
    t = shards[0]
    t["model.embed_tokens.weight"] = torch.from_numpy(w["embed"]).to(dense_dtype)
    t["model.norm.weight"] = torch.from_numpy(w["final_norm"]).to(dense_dtype)
    trip("lm_head", w["lm_head"], shards[1])
    weight_map = {}
    for si, sh in enumerate(shards):
        fn = f"model-{si + 1:05d}-of-00002.safetensors"
        write_safetensors(out_dir / fn, sh, metadata={"format": "mlx"})
        weight_map.update({k: fn for k in sh})
    (out_dir / "model.safetensors.index.json").write_text(json.dumps({"weight_map": weight_map}))
    cfg = dict(model_type="motif", hidden_size=args.hidden_size, num_hidden_layers=args.num_hidden_layers,
               intermediate_size=args.intermediate_size, num_attention_heads=args.q_heads,
               num_key_value_heads=2 * args.kv_heads_per_slot, num_noise_heads=G, k_ratio=1,
               vocab_size=args.vocab_size, head_dim=d, rms_norm_eps=args.rms_norm_eps,
               attn_rms_norm_eps=args.attn_rms_norm_eps, rope_theta=args.rope_theta,
               tie_word_embeddings=False, quantization={"group_size": 64, "bits": 4})
    (out_dir / "config.json").write_text(json.dumps(cfg))
    return w
