"""Tensor-parallel decode on 2, 4 and 8 GPUs: the sharded MotifDecoder (GDA groups, MLP
columns and the lm_head's vocabulary split over ranks; the row-parallel outputs and the
PolyNorm statistics exchanged through peer memory inside the GEMVs, or all-reduced by NCCL;
the packed argmax keys combined by one all-reduce) produces the same greedy tokens as the
unsharded model built from the same seed. Each case is skipped without enough GPUs."""

from __future__ import annotations

import os
from datetime import timedelta

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

PROMPT = [3, 17, 29, 5]
N_TOKENS = 8


def _watchdog():
    """A worker that is still running after 240 s prints every thread's stack and exits, so a
    stuck rank shows where it stopped and the test fails instead of waiting for good."""
    import faulthandler
    import sys

    faulthandler.dump_traceback_later(240, exit=True, file=sys.stderr)


def _collect(procs, q):
    """Each worker's result; the workers are joined, and killed if they do not finish."""
    try:
        got = dict(q.get(timeout=300) for _ in procs)
        for p in procs:
            p.join(timeout=120)
            assert p.exitcode == 0
        return got
    finally:
        for p in procs:
            if p.is_alive():
                p.kill()
                p.join(timeout=30)


def _args():
    from mlx_motif.model import ModelArgs

    return ModelArgs(hidden_size=512, num_hidden_layers=3, intermediate_size=1024, num_attention_heads=32,
                     num_key_value_heads=16, vocab_size=2048, head_dim=128, num_noise_heads=8)


def _head_env(head: str) -> None:
    """How the ranks' token keys meet: "key" over peer memory, "allreduce" by NCCL MAX."""
    os.environ["MOTIF_TP_KEY_EXCHANGE"] = "1" if head == "key" else "0"


def _worker(rank, world, port, q, exchange="peer"):
    import torch.distributed as dist
    from mlx_motif.model import MotifDecoder

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    _watchdog()
    if exchange == "nccl":
        os.environ["MOTIF_TP_NCCL"] = "1"
    _head_env("key" if exchange == "peer-key" else "allreduce")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        m = MotifDecoder.random(_args(), seed=5, std=0.05, max_seq=64, device=f"cuda:{rank}",
                                tp_group=dist.group.WORLD, rank=rank, world=world)
        toks = m.generate(PROMPT, N_TOKENS)
        m.reset()
        again = m.generate(PROMPT, N_TOKENS)  # rewound position: the exchange flags were reset
        m.release_graphs()  # graphs holding NCCL calls go before the process group
        torch.cuda.synchronize()
        dist.barrier()
        m.release_exchange()
        q.put((rank, (toks, again)))
    finally:
        dist.destroy_process_group()


def _sample_worker(rank, world, port, q, head="allreduce"):
    import torch.distributed as dist
    from mlx_motif.model import MotifDecoder

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    _watchdog()
    _head_env(head)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        m = MotifDecoder.random(_args(), seed=5, std=0.05, max_seq=64, device=f"cuda:{rank}",
                                tp_group=dist.group.WORLD, rank=rank, world=world)
        m.set_sampling(0.8, seed=21)
        toks = m.generate(PROMPT, N_TOKENS)
        m.release_graphs()
        torch.cuda.synchronize()
        dist.barrier()
        m.release_exchange()
        q.put((rank, toks))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,head", [(2, "allreduce"), (4, "allreduce"), (8, "allreduce"), (2, "key"), (4, "key"),
                                        (8, "key")])
def test_tp_temperature_sampling_equals_single_gpu(world, head):
    """Temperature sampling under tensor parallelism (each rank's Gumbel-max key over its
    vocabulary shard, noise drawn per global index, combined by the MAX all-reduce or over peer
    memory) draws the same tokens as one GPU with the same seed."""
    from mlx_motif.model import MotifDecoder

    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29880 + (os.getpid() % 40) + 5 * world + (2 if head == "key" else 0)
    procs = [ctx.Process(target=_sample_worker, args=(r, world, port, q, head)) for r in range(world)]
    for p in procs:
        p.start()
    got = _collect(procs, q)
    ref = MotifDecoder.random(_args(), seed=5, std=0.05, max_seq=64, device="cuda:0")
    ref.set_sampling(0.8, seed=21)
    want = ref.generate(PROMPT, N_TOKENS)
    for r in range(world):
        assert got[r] == want, f"rank {r}: TP{world} sampled {got[r]}, one GPU {want}"


@pytest.mark.parametrize("world,exchange", [(2, "peer"), (2, "nccl"), (4, "peer"), (8, "peer"), (2, "peer-key"),
                                            (4, "peer-key"), (8, "peer-key")])
def test_tp_decode_equals_single_gpu(world, exchange):
    """Peer-memory exchange inside the GEMVs (default) and the NCCL all-reduce path; "peer-key"
    also moves the token keys onto peer memory (motif_argmax_key_exchange)."""
    from mlx_motif.model import MotifDecoder

    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29600 + (os.getpid() % 300) + 11 * world + {"peer": 0, "nccl": 7, "peer-key": 3}[exchange]
    procs = [ctx.Process(target=_worker, args=(r, world, port, q, exchange)) for r in range(world)]
    for p in procs:
        p.start()
    got = _collect(procs, q)
    ref = MotifDecoder.random(_args(), seed=5, std=0.05, max_seq=64, device="cuda:0").generate(PROMPT, N_TOKENS)
    for r in range(1, world):
        assert got[r] == got[0], f"rank {r} disagrees on the greedy tokens"
    assert got[0][0] == ref, f"TP{world} tokens {got[0][0]} != single-GPU tokens {ref}"
    assert got[0][1] == ref, f"TP{world} tokens after reset() differ"


ROW_PROMPT = [(7 + 13 * i) % 2048 for i in range(170)]  # 170 ids inside the vocabulary
VERIFY_IDS = [5, 900, 17, 3, 44]


def _draft_args():
    from mlx_motif.model import ModelArgs

    return ModelArgs(hidden_size=512, num_hidden_layers=2, intermediate_size=1024, num_attention_heads=4,
                     num_key_value_heads=2, num_noise_heads=None, vocab_size=2048)


def _rows_worker(rank, world, port, q):
    import torch.distributed as dist
    from mlx_motif.model import MotifDecoder
    from mlx_motif.speculative import SpeculativeDecoder

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    _watchdog()
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        dev = f"cuda:{rank}"
        m = MotifDecoder.random(_args(), seed=5, std=0.05, max_seq=256, device=dev, tp_group=dist.group.WORLD,
                                rank=rank, world=world)
        m.prefill(ROW_PROMPT)  # a 169-row block: GEMMs (TP2) or the multi-row GEMV (TP4, TP8), all-reduced
        first = int(m.token.item())
        rows = m.forward_rows(VERIFY_IDS).float().cpu().numpy()
        draft = MotifDecoder.random(_draft_args(), seed=12, std=0.05, max_seq=256, device=dev)
        spec = SpeculativeDecoder(m, draft, k=4, temperature=0.0)
        toks = spec.generate(ROW_PROMPT[:40], 12)
        m.release_graphs()
        torch.cuda.synchronize()
        dist.barrier()
        m.release_exchange()
        q.put((rank, (first, rows, toks)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4, 8])
def test_tp_row_blocks_and_speculative_verify(world):
    """Prompt ingestion in row blocks and the [1, K+1] verify under tensor parallelism (NCCL
    all-reduce of the row-parallel outputs and of the PolyNorm statistics, the lm_head shards
    gathered) agree with one GPU; speculative greedy decoding with a replicated draft
    reproduces the single-GPU greedy tokens on every rank."""
    from mlx_motif.model import MotifDecoder

    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29950 + (os.getpid() % 40) + 3 * world
    procs = [ctx.Process(target=_rows_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = _collect(procs, q)
    ref = MotifDecoder.random(_args(), seed=5, std=0.05, max_seq=256, device="cuda:0")
    ref.prefill(ROW_PROMPT)
    first = int(ref.token.item())
    rows = ref.forward_rows(VERIFY_IDS).float().cpu().numpy()
    ref.reset()  # generate() prefills at the current position
    greedy = ref.generate(ROW_PROMPT[:40], 12)
    for r in range(world):
        assert got[r][0] == first, f"rank {r}: first token {got[r][0]} != {first}"
        err = float(abs(got[r][1] - rows).max())
        assert err < 5e-2, f"rank {r}: verify logits differ by {err}"
        assert got[r][2] == greedy, f"rank {r}: speculative tokens {got[r][2]} != greedy {greedy}"
