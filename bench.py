#!/usr/bin/env python
"""Decode benchmark of the 12.7B-class q4 GDA model on B200 (one JSON line on stdout).

Headline (BASELINE.json metric, config[1]): greedy decode tok/s after a
164-token random prompt, random-init weights (std 0.02, q4 group 64, fp16
scales/biases), fp16 4-slot KV cache, batch 1. A "step" is one decode token:
one replay of the captured CUDA graph (48 layers + lm_head + argmax); the
next input token never leaves the GPU. Weights (6.85 GB) are far larger than
L2, so every step streams them from HBM (no flush needed).

Also reported in the same line:
  e2e           the same metric through the public per-token API
                (``MotifDecoder.decode_host``): pinned-host token -> device,
                one replay, argmax -> pinned host, sync, every step.
  roofline      dominant kernel = the q4 GEMV (``motif_quantized_linear``):
                algorithmic bytes (packed weights + scales + biases + x + y)
                of one step's 193 GEMV launches / their CUDA-event time.
  extra.p16k_*  config[2]: decode at a 16000-token context (KV cache filled
                with synthetic N(0,1)·0.5 rows), q4 and fp16 4-slot caches,
                with the attention kernels' HBM GB/s.
  extra.vanilla_2p6b_p3204  config[3]: the 2.6B-class vanilla model ingests a
                3204-token prompt (tensor-core blocks), then greedy decode, one GPU.
  extra.speculative  config[4]: that model drafts K=4 tokens per cycle for the
                12.7B-class target (one [1, K+1] verify forward per cycle,
                rejection sampling at T=0.7), 800-token prompt, 256 tokens.
  cpu_baseline  the CPU oracle (numpy restatement of the reference path) on
                one full-size layer, scaled to a token.

Multi-GPU (``torchrun --nproc-per-node N``): tensor parallel over N ranks
(GDA groups and MLP columns sharded, NCCL all-reduce after o_proj and
down_proj, PolyNorm statistics all-reduced); the timed region is the max over
ranks; the token stream is shared, so value = tokens/s of the one stream
(scaling "strong": the model is fixed while N grows).

``--impl reference`` times the reference's CPU implementation of the path
(the oracle port: MLX is not installable here) on the host cores.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
for _p in (str(ROOT), str(ROOT / "mlx-motif_b200")):
    if _p not in sys.path:
        sys.path.insert(0, _p)

METRIC = "12.7B-class q4 decode tok/s at p164 (config[1]); p16k in extra"
PROMPT_LEN = 164


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=128)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--cache", choices=["fp16", "q4", "q8"], default="fp16")
    ap.add_argument("--no-long", action="store_true", help="skip the p16k extras")
    ap.add_argument("--no-vanilla", action="store_true", help="skip the config[3] 2.6B vanilla extra")
    ap.add_argument("--no-spec", action="store_true", help="skip the config[4] speculative extra")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--layers", type=int, default=48, help="(debug) model depth; 48 is the benchmark")
    ap.add_argument("--prompt", type=int, default=164, help="prompt length (164 = config[1])")
    ap.add_argument("--vocab", type=int, default=219520, help="(profiling) vocabulary size; 219520 is the benchmark")
    ap.add_argument("--kernel-case", choices=["gemm", "prefill_attn", "long_q4", "long_fp16", "rows_gemv", "verify"],
                    default=None,
                    help="(profiling) run one small case --steps times and exit: the prompt GEMM "
                         "(3204 x 16384 x 2048), a 2048-row vanilla prompt-attention block, the long-cache "
                         "decode step at 16000 rows (q4 / fp16 cache), the 5-row GEMV on the 12.7B-class "
                         "gate|up shape, or the speculative verify (a 5-row forward of the 12.7B-class model "
                         "at an 800-row cache; the last one inside cudaProfilerStart/Stop)")
    ap.add_argument("--profile", action="store_true",
                    help="profiler window only: cudaProfilerStart/Stop around the timed steps, then exit "
                         "(for `ncu --profile-from-start off`)")
    return ap.parse_args()


# --------------------------------------------------------------------------- #
# clocks during the timed region
# --------------------------------------------------------------------------- #
class ClockSampler:
    QUERY = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines: list[str] = []
        self.t0 = self.t1 = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                 "-lms", "20"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            threading.Thread(target=self._read, daemon=True).start()
            time.sleep(0.15)
        except OSError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append((time.time(), line.strip()))

    def mark(self, which: str):
        setattr(self, which, time.time())

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"], "samples": 0}
        time.sleep(0.1)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        rows = []
        for ts, line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 10:
                continue
            rows.append((ts, parts))
        inside = [r for r in rows if self.t0 is not None and self.t0 - 0.02 <= r[0] <= self.t1 + 0.02]
        use = inside or rows
        if not use:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"], "samples": 0}
        sm = [float(p[2]) for _, p in use if p[2].replace(".", "").isdigit()]
        smax = [float(p[3]) for _, p in use if p[3].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for _, p in use for i in range(4) if p[6 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(smax) if smax else None,
                "reasons": reasons, "samples": len(use), "samples_inside_timed_region": len(inside)}


# --------------------------------------------------------------------------- #
# distributed plumbing
# --------------------------------------------------------------------------- #
def dist_setup(n_gpus: int):
    import torch

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != n_gpus:
        raise SystemExit(f"--gpus {n_gpus} but WORLD_SIZE={world}: launch N>1 with torchrun")
    group = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180),
                                device_id=torch.device("cuda", local))
        group = dist.group.WORLD
    return rank, world, local, group


def max_over_ranks(v: float, world: int) -> float:
    if world == 1:
        return v
    import torch
    import torch.distributed as dist

    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world: int):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


# --------------------------------------------------------------------------- #
# CPU legs: whole decode tokens of the numpy oracle on the host cores
# --------------------------------------------------------------------------- #
class CpuOracleTokens:
    """Whole config[1] decode tokens through the numpy oracle (the CPU restatement of the
    reference's ``*_reference`` path): 48 full-size GDA layers, each with its own fp16 4-slot
    cache filled to the p164 prompt, the final norm and the full 219520 x 4096 q4 lm_head, every
    quantized matmul split over a thread pool of all host cores.

    One layer's weights (235M q4 weights, 132 MB, drawn once) serve all 48 layers, so building
    the sample takes seconds instead of minutes; the per-token work (every layer's GEMVs, the
    attention over its own cache, the lm_head) is that of the real model. The lm_head's codes are
    random words with small scales (its values do not matter for timing)."""

    def __init__(self, threads: int, kv_len: int = PROMPT_LEN):
        import concurrent.futures as cf

        import numpy as np

        import oracle as O

        self.threads = threads
        self.kv_len = kv_len
        one = O.OracleArgs(num_hidden_layers=1, vocab_size=1000)
        w = O.make_synthetic_weights(one, seed=0)
        rng = np.random.default_rng(0)
        V, H = 219520, one.hidden_size
        lm = (rng.integers(0, 1 << 32, (V, H // 8), dtype=np.uint32),
              (rng.random((V, H // 64)) * 1e-3).astype(np.float16),
              (rng.standard_normal((V, H // 64)) * 1e-3).astype(np.float16))
        self.layer_weights = sum(w["layers"][0][k][0].size * 8 for k in ("qkv", "o", "gate", "up", "down"))
        args = O.OracleArgs(num_hidden_layers=48, vocab_size=V)
        weights = dict(embed=w["embed"], final_norm=w["final_norm"], lm_head=lm, layers=[w["layers"][0]] * 48)
        self.orc = O.GroupedDecodeOracle(args, weights)
        d = one.head_dim
        for c in self.orc.caches:  # the prompt's KV rows
            c.update_and_fetch_4(*((rng.standard_normal((1, 8, kv_len, d)) * 0.5).astype(np.float16)
                                   for _ in range(4)))
        self.pool = cf.ThreadPoolExecutor(threads) if threads > 1 else None
        self.token = 1
        self._impl = O.motif_oracle.quantized_matmul  # the oracle's own matmul, applied per chunk

    def _qmm(self, x, data, scales, biases, group_size=64, bits=4):
        """The oracle's quantized matmul over row chunks (at most 4096 rows each, so the float64
        unpack of the lm_head stays a few hundred MB per thread) on the pool."""
        import numpy as np

        n = data.shape[0]
        step = min(4096, -(-n // self.threads))
        cuts = list(range(0, n, step)) + [n]
        f = self._impl
        if self.pool is None:
            parts = [f(x, data[a:b], scales[a:b], biases[a:b], group_size, bits) for a, b in zip(cuts[:-1], cuts[1:])]
        else:
            parts = list(self.pool.map(lambda ab: f(x, data[ab[0]:ab[1]], scales[ab[0]:ab[1]], biases[ab[0]:ab[1]],
                                                    group_size, bits), list(zip(cuts[:-1], cuts[1:]))))
        return np.concatenate(parts, axis=-1)

    def token_seconds(self) -> float:
        """Wall seconds of one decode token (the oracle's step: embedding row, 48 layers, norm,
        lm_head, argmax); the next token is the argmax."""
        import oracle.motif_oracle as M

        orig = M.quantized_matmul
        M.quantized_matmul = self._qmm
        try:
            t0 = time.perf_counter()
            _, tok = self.orc.step(self.token % 1000)
            dt = time.perf_counter() - t0
        finally:
            M.quantized_matmul = orig
        self.token = tok
        return dt

    def describe(self, n_tokens: int) -> str:
        return (f"{n_tokens} whole decode token(s) of the numpy oracle (CPU restatement of the reference's "
                f"*_reference path): 48 full-size GDA layers ({self.layer_weights / 1e6:.0f}M q4 weights each; one "
                f"layer's weights shared by all 48, each layer with its own fp16 4-slot cache from kv_len "
                f"{self.kv_len}), final norm and the 219520x4096 q4 lm_head, matmuls on {self.threads} "
                f"thread(s)")

    def close(self):
        if self.pool:
            self.pool.shutdown()


def cpu_baseline(threads: int, tokens: int = 2) -> dict:
    """The cpu_baseline leg: one untimed token, then `tokens` timed whole tokens (~10-30 s)."""
    s = CpuOracleTokens(threads)
    s.token_seconds()
    secs = [s.token_seconds() for _ in range(tokens)]
    out = {"value": len(secs) / sum(secs), "unit": "tok/s", "cores": threads, "kind": "port",
           "sample": s.describe(len(secs))}
    s.close()
    return out


# --------------------------------------------------------------------------- #
# B200 arm
# --------------------------------------------------------------------------- #
def _graph_time(fn, reps: int = 5) -> float:
    """Best CUDA-event time (ms) of replaying a graph that captured fn() once."""
    import torch

    fn()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        fn()
    g.replay()
    torch.cuda.synchronize()
    st = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    best = math.inf
    for _ in range(reps):
        e0.record(st)
        g.replay()
        e1.record(st)
        e1.synchronize()
        best = min(best, e0.elapsed_time(e1))
    del g
    return best


def time_gemvs(model) -> dict:
    """CUDA-event time of one step's q4 GEMV launches (every layer's qkv, o, gate|up, down + lm_head),
    replayed from a CUDA graph so host launch cost is excluded. Bytes: every linear's packed
    weights, scales and biases plus its x and y vectors."""
    import torch

    lins = [(L[k], inp) for L in model.layers for k, inp in
            (("qkv", model.x), ("o", model.attn), ("gate_up", model.x), ("down", model.act))]
    lins.append((model.lm_head, model.x))
    outs = {id(q): torch.empty(q.out_dim, dtype=torch.float16, device=model.device) for q, _ in lins}
    alg = sum(q.nbytes() + 2 * q.in_dim + 2 * q.out_dim for q, _ in lins)

    def run():
        for q, inp in lins:
            q(inp[: q.in_dim], out=outs[id(q)], workspace=model.lin_ws)

    best = _graph_time(run)
    n = len(lins)
    return {"launches": n, "ms_total": best, "ms_per_launch": best / n, "bytes_total": alg,
            "bytes_per_launch": alg / n, "gbs": alg / (best / 1e3) / 1e9,
            "kernel": "q4_gemv_tma_kernel (motif_quantized_linear, one launch per linear)"}


def time_attention(model) -> dict:
    """CUDA-event time (graph replay) of the 48 layers' attention step at the current kv_len: the
    one-launch RoPE + cache append + dual-V attention + GDA merge (motif_gda_decode_step), or the
    attention alone when the model runs the two-call path."""
    from mlx_motif._native import check, lib, ptr, stream

    kv_len = int(model.pos_len[1].item())
    pos_p = model.pos_len.data_ptr()
    kvl_p = pos_p + 4

    def run():
        st = stream(model.device)
        for li, L in enumerate(model.layers):
            if model.fused_attn:
                # writes row pos from the last qkv: the slot the next decode step overwrites
                check(lib.motif_gda_decode_step(ptr(model.qkv), ptr(model.inv_freq), model._slots[li], pos_p,
                                                model.scale, model.q_groups, model.gr, ptr(L["subln"]),
                                                ptr(L["lambda_full"]), L["lambda_full"].numel(), L["lambda_init"],
                                                1e-5, ptr(model.attn), ptr(model.attn_ws), model.attn_ws_bytes, st))
            else:
                check(lib.motif_gda_decode_attention(ptr(model.q), model._slots[li], model.scale, model.q_groups,
                                                     model.gr, 0, kvl_p, ptr(L["subln"]), ptr(L["lambda_full"]),
                                                     L["lambda_full"].numel(), L["lambda_init"], 1e-5,
                                                     ptr(model.attn), ptr(model.attn_ws), model.attn_ws_bytes, st))

    best = _graph_time(run)
    kv_bytes = model.kv_bytes_per_token(kv_len)
    return {"kv_len": kv_len, "ms_48_layers": best, "bytes": kv_bytes, "gbs": kv_bytes / (best / 1e3) / 1e9}


def read_traffic() -> float | None:
    """ncu DRAM bytes per q4-GEMV launch, from the committed profile summary (None if absent)."""
    p = ROOT / "profiles" / "q4_gemv_decode_step.txt"
    if not p.exists():
        return None
    for line in p.read_text().splitlines():
        if line.startswith("traffic_bytes_per_launch:"):
            try:
                return float(line.split(":", 1)[1].split()[0])
            except ValueError:
                return None
    return None


def peaks() -> tuple[float, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def bf16_peak_tflops() -> float:
    """Dense bf16 tensor peak for a kernel timed alone (burst figure), else the fallback."""
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        return float(json.loads(p.read_text())["bf16_tflops"])
    return 1590.0


def run_b200(a) -> None:
    import numpy as np
    import torch

    from mlx_motif.model import ModelArgs, MotifDecoder

    rank, world, local, group = dist_setup(a.gpus)
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    global PROMPT_LEN
    PROMPT_LEN = a.prompt
    margin = a.warmup * 2 + a.steps * 2 + 16
    args = ModelArgs(num_hidden_layers=a.layers, vocab_size=a.vocab)
    t_init = time.time()
    model = MotifDecoder.random(args, seed=0, cache=a.cache, max_seq=PROMPT_LEN + margin + 8, device=dev,
                                tp_group=group, rank=rank, world=world)
    torch.cuda.synchronize()
    t_init = time.time() - t_init
    prompt = np.random.default_rng(0).integers(0, args.vocab_size, PROMPT_LEN).tolist()
    model.prefill(prompt)  # warm-up: first-call setup (function attributes, buffers, the decode graph)
    model.reset()
    prefill_ms = timed_prefill(model, prompt)
    for _ in range(a.warmup):
        model.step_device()
    torch.cuda.synchronize()
    barrier(world)

    if a.profile:
        torch.cuda.cudart().cudaProfilerStart()
        for _ in range(a.steps):
            model.step_device()
        torch.cuda.synchronize()
        torch.cuda.cudart().cudaProfilerStop()
        if rank == 0:
            print(json.dumps({"profile_steps": a.steps, "kernels_per_step": model_launches(model)}))
        return

    sampler = ClockSampler(local) if rank == 0 else None
    if sampler:
        sampler.start()
    torch.cuda.synchronize()
    model.exchange_read_ns(reset=True)
    st = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier(world)
    torch.cuda.synchronize()
    if sampler:
        sampler.mark("t0")
    e0.record(st)
    for _ in range(a.steps):
        model.step_device()
    e1.record(st)
    torch.cuda.synchronize()
    if sampler:
        sampler.mark("t1")
    barrier(world)
    ms = max_over_ranks(e0.elapsed_time(e1), world)
    xchg_ms = max_over_ranks(model.exchange_read_ns() / 1e6 / a.steps, world)
    clocks = sampler.stop() if sampler else None
    value = a.steps / (ms / 1e3)
    launches = model_launches(model) * a.steps
    kv_mid = PROMPT_LEN + a.warmup + a.steps // 2
    bytes_per_step = model.weight_bytes * world + model.kv_bytes_per_token(kv_mid) * world

    # ---- e2e through the public per-token API (host buffers) ----
    tok = int(model.token.item())
    for _ in range(a.warmup):
        tok = model.decode_host(tok)
    barrier(world)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(a.steps):
        tok = model.decode_host(tok)
    e2e_s = max_over_ranks(time.perf_counter() - t0, world)
    e2e = {"value": a.steps / e2e_s, "unit": "tok/s", "h2d_bytes_per_step": 4, "d2h_bytes_per_step": 4}

    # ---- dominant kernel roofline (q4 GEMV), measured live ----
    gem = time_gemvs(model)
    peak, peak_kind = peaks()
    traffic = read_traffic()
    roofline = {"bound": "hbm", "kernel": gem["kernel"] + f", all {gem['launches']} launches of a step",
                "achieved": round(gem["gbs"], 1), "peak": peak, "peak_kind": peak_kind, "unit": "GB/s",
                "frac": round(gem["gbs"] / peak, 4), "traffic": traffic,
                "bytes_per_launch": round(gem["bytes_per_launch"]), "ms_per_launch": round(gem["ms_per_launch"], 5)}
    attn_p164 = time_attention(model)
    attn_p164["attention_kernel"] = model.attention_kernel()
    step_frac = bytes_per_step / world / (ms / a.steps / 1e3) / 1e9 / peak

    extra = {"weights_gb": round(model.weight_bytes * world / 1e9, 3), "init_s": round(t_init, 1),
             "step_hbm_gbs_per_gpu": round(bytes_per_step / world / (ms / a.steps / 1e3) / 1e9, 1),
             "step_frac_of_peak": round(step_frac, 4), "attention_p164": attn_p164,
             "prefill_p164": {"ms": round(prefill_ms, 3), "tok_s": round(PROMPT_LEN / (prefill_ms / 1e3), 1),
                              "path": prefill_path(model, PROMPT_LEN)},
             "gemv": {k: (round(v, 4) if isinstance(v, float) else v) for k, v in gem.items()}}
    if world > 1:
        extra["tp_exchange"] = {
            "read_ms_per_step": round(xchg_ms, 4), "share_of_step": round(xchg_ms / (ms / a.steps), 4),
            "note": "time CTA 0 of the consuming GEMVs spent reading the peers' exchanged rows and PolyNorm "
                    "statistics (waits for slower ranks included), summed over the exchanges of a step, max "
                    "over ranks"}

    # ---- config[2]: p16k with q4 and fp16 caches ----
    if not a.no_long:
        weights = model.weights_dict()
        model.release_graphs()  # graphs may hold NCCL calls: released before the communicator
        del model
        model = None
        torch.cuda.empty_cache()
        for kind in ("q4", "fp16"):
            m = MotifDecoder(args, weights, cache=kind, max_seq=16000 + a.warmup + a.steps + 8, device=dev,
                             tp_group=group)
            pre = None
            if world == 1:  # real prompt ingestion (tensor-core blocks of 2048 rows)
                long_prompt = np.random.default_rng(1).integers(0, args.vocab_size, 16000).tolist()
                pms = timed_prefill(m, long_prompt)
                pre = {"ms": round(pms, 2), "tok_s": round(16000 / (pms / 1e3), 1),
                       "tflops": round(prefill_flops(m, 16000) / (pms / 1e3) / 1e12, 1)}
            else:  # synthetic rows stand in for the prompt's KV (keeps the multi-GPU run short)
                m.fill_cache_synthetic(16000, seed=1)
                m.token.fill_(1)
            for _ in range(a.warmup):
                m.step_device()
            torch.cuda.synchronize()
            barrier(world)
            e0.record(st)
            for _ in range(a.steps):
                m.step_device()
            e1.record(st)
            torch.cuda.synchronize()
            barrier(world)
            lms = max_over_ranks(e0.elapsed_time(e1), world)
            att = time_attention(m)
            extra[f"p16k_{kind}"] = {
                "tok_s": round(a.steps / (lms / 1e3), 2), "ms_per_step": round(lms / a.steps, 4),
                "attention_kernel": m.attention_kernel(), "cache_capacity": int(m._slots[0].capacity),
                "attention_gbs": round(att["gbs"], 1), "attention_frac": round(att["gbs"] / peak, 4),
                "attention_ms_per_step": round(att["ms_48_layers"], 4),
                "peak_hbm_bytes": int(torch.cuda.max_memory_allocated(dev)),
                "prefill_16000": pre,
            }
            m.release_graphs()
            del m
            torch.cuda.empty_cache()

    # ---- config[3]: the 2.6B-class vanilla decoder (one GPU: the vanilla path has no TP) ----
    if world == 1 and not a.no_vanilla:
        if model is not None:
            model.release_graphs()
            del model
            model = None
            torch.cuda.empty_cache()
        van = ModelArgs(hidden_size=2048, num_hidden_layers=32, intermediate_size=8192, num_attention_heads=16,
                        num_key_value_heads=4, num_noise_heads=None, vocab_size=a.vocab)
        ctx = 3204
        m = MotifDecoder.random(van, seed=0, cache="fp16", max_seq=ctx + a.warmup + a.steps + 8, device=dev)
        vprompt = np.random.default_rng(2).integers(0, van.vocab_size, ctx).tolist()
        m.prefill(vprompt)  # warm-up: first-call setup (function attributes, block buffers, graphs)
        m.reset()
        vpms = timed_prefill(m, vprompt)
        for _ in range(a.warmup):
            m.step_device()
        torch.cuda.synchronize()
        e0.record(st)
        for _ in range(a.steps):
            m.step_device()
        e1.record(st)
        torch.cuda.synchronize()
        vms = e0.elapsed_time(e1)
        vb = m.weight_bytes + m.kv_bytes_per_token(ctx + a.warmup + a.steps // 2)
        vflops = prefill_flops(m, ctx)
        extra["vanilla_2p6b_p3204"] = {
            "workload": "config[3]: 2.6B-class vanilla q4 (32L, H2048, 16 q / 4 kv heads, I8192, V219520), "
                        "3204 random prompt ids ingested in tensor-core blocks (2048 + 1155 rows + 1 decode "
                        "step), then greedy decode, fp16 4-slot cache",
            "prefill": {"ms": round(vpms, 2), "tok_s": round(ctx / (vpms / 1e3), 1),
                        "tflops": round(vflops / (vpms / 1e3) / 1e12, 1),
                        "frac_of_bf16_peak": round(vflops / (vpms / 1e3) / 1e12 / bf16_peak_tflops(), 4)},
            "tok_s": round(a.steps / (vms / 1e3), 2), "ms_per_step": round(vms / a.steps, 4),
            "weights_gb": round(m.weight_bytes / 1e9, 3),
            "step_hbm_gbs": round(vb / (vms / a.steps / 1e3) / 1e9, 1),
            "kernels_per_step": model_launches(m),
        }
        # ---- config[4]: speculative decoding, this 2.6B-class draft + the 12.7B-class target ----
        m.release_graphs()
        del m
        torch.cuda.empty_cache()
        if not a.no_spec:
            extra["speculative"] = speculative_extra(a, args, van, dev, st, e0, e1, group, rank, world)

    # config[4] under tensor parallelism (target sharded, draft replicated)
    if world > 1 and not a.no_spec:
        if model is not None:
            model.release_graphs()
            del model
            model = None
            torch.cuda.empty_cache()
        van = ModelArgs(hidden_size=2048, num_hidden_layers=32, intermediate_size=8192, num_attention_heads=16,
                        num_key_value_heads=4, num_noise_heads=None, vocab_size=a.vocab)
        extra["speculative"] = speculative_extra(a, args, van, dev, st, e0, e1, group, rank, world)

    cpu = None
    if rank == 0 and world == 1 and not a.no_cpu_baseline:
        cpu = cpu_baseline(threads=os.cpu_count() or 1)

    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "tok/s", "n_gpus": world, "steps": a.steps,
            "warmup": a.warmup, "ms_per_step": round(ms / a.steps, 4), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "fp16 activations, q4 g64 weights, fp32 accumulate",
            "data": "synthetic: random-init weights (std 0.02) and random prompt ids",
            "config": {"workload": f"config[1]: 12.7B-class GDA q4, p{PROMPT_LEN} prompt then greedy decode, "
                                   f"{a.cache} 4-slot cache, batch 1",
                       "model": "motif-12.7B-class (48L, H4096, 24+8 q heads, 8 kv/slot, I14336, V219520)",
                       "global_batch": 1, "seq_len": PROMPT_LEN, "parallelism": f"tp{world}" if world > 1 else "single",
                       "l2": "inputs larger than L2: 6.85 GB of weights stream from HBM every step"},
            "e2e": e2e, "gpu_launches": launches,
            "roofline": roofline, "cpu_baseline": cpu, "clocks": clocks, "extra": extra,
        }
        print(json.dumps(line), flush=True)
    if model is not None:
        model.release_graphs()
    torch.cuda.synchronize()
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()


def prefill_path(model, n: int) -> str:
    """How MotifDecoder.prefill ingests an n-token prompt on this model (one GPU or a TP rank)."""
    rows = n - 1
    if rows < model.min_rows_block or not model._block_ok():
        return "decode steps"
    big = rows >= model.min_block_rows and model._gemm_ok()
    kind = "tensor-core q4 GEMMs" if big else "multi-row q4 GEMVs (the shard shapes leave the GEMM contract)"
    tp = f", tensor parallel over {model.tp} ranks with NCCL all-reduces" if model.tp > 1 else ""
    return f"one {rows}-row block ({kind}{tp}) + the decode step for the last token"


def prefill_flops(model, n: int) -> float:
    """Algorithmic FLOPs of ingesting an n-token prompt: every linear (2 per weight per row)
    plus the causal attention of all query heads (q·k over d and p·[v1|v2] over 2d, for the
    n(n+1)/2 visible pairs). The lm_head runs for the last row only."""
    lin = sum(L[k].out_dim * L[k].in_dim for L in model.layers for k in ("qkv", "o", "gate_up", "down"))
    pairs = n * (n + 1) / 2
    attn = len(model.layers) * model.q_heads * pairs * 2 * (model.d + 2 * model.d)
    return 2.0 * lin * n + attn + 2.0 * model.lm_head.out_dim * model.lm_head.in_dim


def speculative_extra(a, args, van, dev, st, e0, e1, group, rank, world) -> dict:
    """config[4]: the 2.6B-class draft (a replica on every rank) and the 12.7B-class target (sharded
    under tensor parallelism); tok/s over the generated tokens, max over ranks."""
    import numpy as np
    import torch

    from mlx_motif.model import MotifDecoder
    from mlx_motif.speculative import SpeculativeDecoder

    par = "1 GPU" if world == 1 else f"TP{world}, draft replicated"
    n_prompt, n_gen, K, T = 800, 256, 4, 0.7
    cap = n_prompt + n_gen + 2 * K + 16
    draft = MotifDecoder.random(van, seed=0, cache="fp16", max_seq=cap, device=dev)
    target = MotifDecoder.random(args, seed=0, cache="fp16", max_seq=cap, device=dev, tp_group=group, rank=rank,
                                 world=world)
    sprompt = np.random.default_rng(4).integers(0, args.vocab_size, n_prompt).tolist()
    spec = SpeculativeDecoder(target, draft, k=K, temperature=T, seed=0)
    spec.generate(sprompt, 16)  # warm-up: graphs, buffers
    spec.stats = {k2: 0 for k2 in spec.stats}
    torch.cuda.synchronize()
    barrier(world)
    t0 = time.perf_counter()
    toks = spec.generate(sprompt, n_gen)
    torch.cuda.synchronize()
    wall = max_over_ranks(time.perf_counter() - t0, world)
    st_ = spec.stats
    # one [1, K+1] verify forward (multi-row GEMVs, logits for every row) against one decode
    # step of the target; both rewound so the cache stays at the same length
    vids = torch.as_tensor(sprompt[: K + 1], dtype=torch.int32, device=dev)
    plog = torch.empty((K + 1, target.V_local * target.tp), dtype=torch.float16, device=dev)
    base = target.offset

    def verify_once():
        target.forward_rows(vids, plog)
        target.rewind(base)

    def step_once():
        target.step_device(with_head=True)
        target.rewind(base)

    rows_ms = {}
    for name, fn in (("verify_forward_ms", verify_once), ("decode_step_ms", step_once)):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        barrier(world)
        e0.record(st)
        for _ in range(10):
            fn()
        e1.record(st)
        torch.cuda.synchronize()
        rows_ms[name] = round(max_over_ranks(e0.elapsed_time(e1), world) / 10, 3)
    out = {
        "workload": f"config[4]: draft 2.6B-class vanilla q4, target 12.7B-class GDA q4 ({par}), K=4, "
                    "temperature 0.7, top-p 1.0, 800 random prompt ids, 256 generated tokens; wall time "
                    "includes both prompts' ingestion",
        "tok_s": round(len(toks) / wall, 2), "seconds": round(wall, 3),
        "acceptance": round(st_["accepted"] / max(1, st_["drafted"]), 4),
        "target_forwards": st_["target_forwards"], "cycles": st_["cycles"],
        **rows_ms,
        "note": "draft and target are independent random-init models, so few draft tokens match "
                "the target's distribution; the verify forward streams the target's weights once for "
                "its K+1 rows (multi-row GEMV); on one GPU the verify replays a CUDA graph (positions "
                "read from the device offset), under TP it runs eagerly with NCCL all-reduces; "
                "verify_forward_ms and decode_step_ms also cover the host's rewind between calls "
                "(under TP: a device sync, two barriers and the exchange reset)",
    }
    target.release_graphs()  # graphs may hold NCCL calls: released before the communicator
    torch.cuda.synchronize()
    barrier(world)
    del spec, draft, target
    torch.cuda.empty_cache()
    return out


def timed_prefill(model, prompt) -> float:
    """CUDA-event milliseconds of model.prefill(prompt) on the current stream (tensor-core row
    blocks, then the last token through the decode step)."""
    import torch

    st = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    e0.record(st)
    model.prefill(prompt)
    e1.record(st)
    torch.cuda.synchronize()
    return e0.elapsed_time(e1)


def model_launches(model) -> int:
    """Kernels of this library per decode step with the head: per layer the four q4 GEMVs (norms,
    residuals and PolyNorm fused into their prologues) and the attention step (one fused launch, or
    RoPE/append + split-KV + combine, plus four dequantizes on the bridge path), then the lm_head GEMV (its epilogue picks the token, or two
    argmax kernels; torch's position increment in that case is not counted)."""
    per_layer = 4 + model.attn_launches
    if model.tp_group is not None:
        head = 2  # vocabulary shard GEMV + key decode (the all-reduce is NCCL's)
    else:
        head = 1 + (0 if model.fused_argmax else 2)
    return len(model.layers) * per_layer + head


# --------------------------------------------------------------------------- #
# reference arm: the CPU oracle port
# --------------------------------------------------------------------------- #
def run_kernel_case(a) -> None:
    """Small single-kernel workloads for ncu captures (one GPU; nothing is timed here)."""
    import os

    import numpy as np
    import torch

    from mlx_motif import _native as N
    from mlx_motif.cache import MotifGroupedKVCache, MotifGroupedQuantizedKVCache
    from mlx_motif.model import rope_inv_freq
    from mlx_motif.quantization import quantize

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    g = torch.Generator(device=dev).manual_seed(0)
    reps = a.steps
    if a.kernel_case == "gemm":
        M, n, k = 3204, 16384, 2048
        d, s, b = quantize((torch.randn((n, k), generator=g, device=dev) * 0.02).half(), 64, 4)
        x = torch.randn((M, k), generator=g, device=dev).half()
        y = torch.empty((M, n), dtype=torch.float16, device=dev)
        for _ in range(reps):
            N.check(N.lib.motif_q4_gemm(x.data_ptr(), M, k, d.data_ptr(), s.data_ptr(), b.data_ptr(), n, y.data_ptr(),
                                        None, None, N.stream()), "q4_gemm")
    elif a.kernel_case == "rows_gemv":
        M, n, k = 5, 28672, 4096
        d, s, b = quantize((torch.randn((n, k), generator=g, device=dev) * 0.02).half(), 64, 4)
        x = torch.randn((M, k), generator=g, device=dev).half()
        y = torch.empty((M, n), dtype=torch.float16, device=dev)
        wb = N.lib.motif_quantized_linear_workspace_bytes(M, n, k, 4, 64)
        ws = torch.zeros(max(wb, 16), dtype=torch.uint8, device=dev)
        for _ in range(reps):
            N.check(N.lib.motif_quantized_linear(0, 4, 64, x.data_ptr(), M, k, d.data_ptr(), s.data_ptr(),
                                                 b.data_ptr(), n, y.data_ptr(), ws.data_ptr(), wb, N.stream()),
                    "quantized_linear")
    elif a.kernel_case == "verify":
        from mlx_motif.model import ModelArgs, MotifDecoder

        m = MotifDecoder.random(ModelArgs(num_hidden_layers=a.layers, vocab_size=a.vocab), seed=0, cache="fp16",
                                max_seq=1024, device=dev)
        ids = np.random.default_rng(4).integers(0, a.vocab, 800).tolist()
        m.ingest(ids)
        rows = torch.as_tensor(ids[:5], dtype=torch.int32, device=dev)
        logits = torch.empty((5, m.V_local), dtype=torch.float16, device=dev)
        base = m.offset
        for i in range(reps):
            last = i == reps - 1
            if last:
                torch.cuda.synchronize()
                torch.cuda.profiler.start()
            m.forward_rows(rows, logits)
            if last:
                torch.cuda.synchronize()
                torch.cuda.profiler.stop()
            m.rewind(base)
    elif a.kernel_case == "prefill_attn":
        S, Hk, n_rep = 2048, 2, 4
        qh = 2 * Hk * n_rep
        c = MotifGroupedKVCache(max_size=4096)
        c.update_and_fetch_4(*(torch.randn((1, Hk, S, 128), generator=g, device=dev).half() * 0.5 for _ in range(4)))
        q = torch.randn((qh, S, 128), generator=g, device=dev).half()
        o = torch.empty((S, qh, 256), dtype=torch.float16, device=dev)
        for _ in range(reps):
            N.check(N.lib.motif_prefill_attention(q.data_ptr(), S, qh, c.slots_struct(), 0, 1, n_rep, 128 ** -0.5,
                                                  o.data_ptr(), None, N.stream()), "prefill_attention")
    else:
        os.environ["MOTIF_LONG_ATTN_MIN_CAP"] = "0"
        G, gr, d_, L = 8, 3, 128, 16000
        qh = G * (gr + 1)
        if a.kernel_case == "long_q4":
            c = MotifGroupedQuantizedKVCache(64, 4, max_size=L + 64)
            c.update_and_fetch_4_quantized(*(torch.randn((1, G, L - 1, d_), generator=g, device=dev).half() * 0.5
                                             for _ in range(4)))
        else:
            c = MotifGroupedKVCache(max_size=L + 64)
            c.update_and_fetch_4(*(torch.randn((1, G, L - 1, d_), generator=g, device=dev).half() * 0.5
                                   for _ in range(4)))
        inv = rope_inv_freq(d_, 10000.0, dev)
        pos = torch.tensor([L - 1, L], dtype=torch.int32, device=dev)
        tq = torch.randn(qh * d_ + 4 * G * d_, generator=g, device=dev).half()
        sub = torch.ones(2 * d_, device=dev).half()
        lam = torch.tensor([0.3], device=dev)
        out = torch.empty(G * gr * 2 * d_, device=dev).half()
        wb = N.lib.motif_gda_decode_step_workspace_bytes(qh, d_, 64)
        ws = torch.zeros(wb, dtype=torch.uint8, device=dev)
        for _ in range(reps):
            N.check(N.lib.motif_gda_decode_step(tq.data_ptr(), inv.data_ptr(), c.slots_struct(), pos.data_ptr(),
                                                d_ ** -0.5, G, gr, sub.data_ptr(), lam.data_ptr(), 1, 0.8, 1e-5,
                                                out.data_ptr(), ws.data_ptr(), wb, N.stream()), "decode step")
    torch.cuda.synchronize()
    print(json.dumps({"kernel_case": a.kernel_case, "launches": reps}))


def run_reference(a) -> None:
    """Reference arm: whole config[1] decode tokens of the oracle port on all host cores (MLX, the
    reference's runtime, is not installable in this image). W untimed warm-up tokens, then up to
    K timed tokens; it stops early (reporting the tokens done) after ~120 s of timed work so the
    run stays within a few minutes. Under torchrun only rank 0 runs."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    sampler = CpuOracleTokens(threads)
    for _ in range(a.warmup):
        sampler.token_seconds()
    secs = []
    for _ in range(a.steps):
        secs.append(sampler.token_seconds())
        if sum(secs) > 120:
            break
    value = len(secs) / sum(secs)
    line = {
        "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": a.gpus, "steps": len(secs),
        "warmup": a.warmup, "ms_per_step": 1e3 / value, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "fp16 storage, float64 compute", "data": "synthetic",
        "impl": "reference",
        "config": {"workload": f"config[1]: 12.7B-class GDA q4, p{PROMPT_LEN}, fp16 4-slot cache, batch 1",
                   "model": "motif-12.7B-class", "global_batch": 1, "seq_len": PROMPT_LEN,
                   "parallelism": "host cores"},
        "cpu_baseline": {"value": value, "unit": "tok/s", "cores": threads, "kind": "port",
                         "sample": sampler.describe(len(secs)) + " (MLX, the reference's own runtime, is not "
                                                                 "installable in this image; the oracle port "
                                                                 "stands in)"},
        "e2e": {"value": value, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    sampler.close()
    print(json.dumps(line), flush=True)


def main():
    a = parse_args()
    if a.impl == "reference":
        run_reference(a)
    elif a.kernel_case:
        run_kernel_case(a)
    else:
        run_b200(a)


if __name__ == "__main__":
    main()
