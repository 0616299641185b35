"""GPU tests of the sampling and speculative-decoding path: Gumbel-max sampling draws from
softmax(l/T) (greedy at T = 0); the acceptance kernel keeps the target distribution (the
speculative-sampling identity, checked by frequency), reduces to argmax matching at T = 0 and
accepts everything when draft and target agree; the [1, K+1] row-block forward matches the
decode step; speculative greedy decoding reproduces the target's greedy tokens."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import assert_close
from test_gpu_kernels import down

pytestmark = pytest.mark.gpu


def _sample(N, logits, T, seed=0, pos=0, rows=None):
    rows = rows or logits.shape[0]
    tok = torch.zeros(rows, dtype=torch.int32, device=logits.device)
    N.check(N.lib.motif_sample(logits.data_ptr(), rows, logits.shape[1], logits.shape[1], T, seed, None, pos, 0,
                               tok.data_ptr(), None, N.stream()), "sample")
    return tok


def test_sample_greedy_and_distribution(cuda):
    from mlx_motif import _native as N

    l = torch.tensor([[0.5, 2.0, -1.0, 2.0, 1.0, 0.0, -3.0, 1.5]], dtype=torch.float16, device=cuda)
    assert _sample(N, l, 0.0).item() == 1  # first index of the maximum
    T, rows = 0.7, 40000
    big = l.repeat(rows, 1)
    counts = np.bincount(_sample(N, big, T, seed=5).cpu().numpy(), minlength=8) / rows
    p = torch.softmax(l.float()[0] / T, 0).cpu().numpy()
    assert np.abs(counts - p).max() < 0.01, (counts, p)
    # fresh draws at another position, same distribution
    c2 = np.bincount(_sample(N, big, T, seed=5, pos=7).cpu().numpy(), minlength=8) / rows
    assert np.abs(c2 - p).max() < 0.01 and not np.array_equal(c2, counts)


def _accept(N, p, q, draft, T, pos=0, seed=3):
    out = torch.zeros(2, dtype=torch.int32, device=p.device)
    N.check(N.lib.motif_speculative_accept(p.data_ptr(), q.data_ptr() if q is not None else None, p.shape[1],
                                           draft.data_ptr(), draft.numel(), p.shape[1], T, seed, None, pos,
                                           out.data_ptr(), N.stream()), "accept")
    return out.tolist()


@pytest.mark.parametrize("shards", [2, 4, 8])
@pytest.mark.parametrize("T", [0.0, 0.7, 1.3])
def test_sample_key_over_vocabulary_shards_equals_whole_row(cuda, shards, T):
    """Tensor-parallel sampling: each shard's motif_sample_key (noise drawn per global index), the
    largest key over the shards (the int64 MAX all-reduce) and motif_argmax_key_decode give the
    token motif_sample draws from the whole row, at every position tried."""
    from mlx_motif import _native as N

    V = 219520
    g = torch.Generator(device=cuda).manual_seed(shards)
    logits = (torch.randn((1, V), generator=g, device=cuda) * 2).half()
    per = V // shards
    keys = torch.zeros(shards, dtype=torch.int64, device=cuda)
    tok = torch.zeros(1, dtype=torch.int32, device=cuda)
    for pos in (0, 5, 163):
        want = _sample(N, logits, T, seed=11, pos=pos).item()
        for r in range(shards):
            N.check(N.lib.motif_sample_key(logits.data_ptr() + 2 * r * per, per, T, 11, None, pos, 0, r * per,
                                           keys[r:].data_ptr(), N.stream()), "sample_key")
        best = keys.max().reshape(1).contiguous()
        N.check(N.lib.motif_argmax_key_decode(best.data_ptr(), tok.data_ptr(), None, N.stream()), "key_decode")
        torch.cuda.synchronize()
        assert tok.item() == want, f"pos {pos}: shards give {tok.item()}, the whole row {want}"


def test_speculative_accept_rules(cuda):
    from mlx_motif import _native as N

    g = torch.Generator(device=cuda).manual_seed(0)
    K, V = 4, 64
    p = (torch.randn((K + 1, V), generator=g, device=cuda) * 2).half()
    am = p.float().argmax(1)
    # greedy: accept while the draft equals the argmax, then the argmax of that row
    draft = am[:K].clone().int()
    draft[2] = (draft[2] + 1) % V
    assert _accept(N, p, None, draft, 0.0) == [2, int(am[2])]
    assert _accept(N, p, None, am[:K].int(), 0.0) == [K, int(am[K])]
    # draft distribution == target distribution: every draft token is accepted
    q = p[:K].clone()
    for pos in range(20):
        assert _accept(N, p, q, torch.randint(0, V, (K,), device=cuda, dtype=torch.int32), 0.7, pos=pos)[0] == K


def test_speculative_sampling_keeps_the_target_distribution(cuda):
    """K = 1: draw x from q, accept with min(1, p/q), else resample from max(0, p − q): the emitted
    token is distributed as p (frequency check over many positions)."""
    from mlx_motif import _native as N

    V, T, trials = 6, 0.7, 12000
    lp = torch.tensor([[1.0, 0.2, -0.5, 2.0, 0.0, -1.0], [0.0] * 6], dtype=torch.float16, device=cuda)
    lq = torch.tensor([[0.0, 1.5, 0.5, 0.5, -1.0, 0.3]], dtype=torch.float16, device=cuda)
    p = torch.softmax(lp.float()[0] / T, 0).cpu().numpy()
    qd = torch.softmax(lq.float()[0] / T, 0).cpu().numpy()
    rng = np.random.default_rng(1)
    xs = rng.choice(V, size=trials, p=qd / qd.sum())
    emitted = np.zeros(V)
    d = torch.zeros(1, dtype=torch.int32, device=cuda)
    for t in range(trials):
        d.fill_(int(xs[t]))
        n, y = _accept(N, lp, lq, d, T, pos=t)
        emitted[int(xs[t]) if n == 1 else y] += 1
    freq = emitted / trials
    assert np.abs(freq - p).max() < 0.02, (freq, p)


def _models(cuda):
    from mlx_motif.model import ModelArgs, MotifDecoder

    tgt = MotifDecoder.random(ModelArgs(hidden_size=512, num_hidden_layers=3, intermediate_size=1024,
                                        num_attention_heads=32, num_key_value_heads=16, num_noise_heads=8,
                                        vocab_size=1024), seed=11, std=0.05, cache="fp16", max_seq=512, device=cuda)
    dft = MotifDecoder.random(ModelArgs(hidden_size=512, num_hidden_layers=2, intermediate_size=1024,
                                        num_attention_heads=4, num_key_value_heads=2, num_noise_heads=None,
                                        vocab_size=1024), seed=12, std=0.05, cache="fp16", max_seq=512, device=cuda)
    return tgt, dft


def test_row_block_forward_matches_decode_steps(cuda):
    tgt, _ = _models(cuda)
    ids = [5, 900, 17, 3, 44]
    tgt.ingest([1, 2, 3, 4, 5, 6, 7])
    rows = tgt.forward_rows(ids)
    ref = []
    tgt.rewind(7)
    for t in ids:
        tgt.token.fill_(t)
        tgt.step_device(with_head=True)
        ref.append(down(tgt.logits))
    assert_close(down(rows), np.stack(ref), "float16", atol=1e-2, rtol=2e-2, what="verify rows vs decode steps")


def test_row_block_graph_replays_match_eager(cuda):
    """forward_rows replays a captured CUDA graph after its first (eager) call: the rows'
    positions come from the device offset, so one graph serves every offset; logits match the
    eager launches within tolerance (the split attention may be cut differently, so later layers
    differ by rounding), the first layer's K/V rows are written identically at the device offset,
    and the host and device offsets advance by the block."""
    tgt, _ = _models(cuda)
    rng = np.random.default_rng(8)
    tgt.ingest(rng.integers(0, 1024, 300).tolist())
    ids = [5, 900, 17, 3, 44]
    ids_d = torch.tensor(ids, dtype=torch.int32, device=cuda)
    out_g = torch.empty((5, tgt.V_local), dtype=torch.float16, device=cuda)
    out_e = torch.empty_like(out_g)
    tgt.forward_rows(ids, out_g)  # first call (at 300): eager
    for base in (290, 250, 100, 37):  # rewind only moves back
        tgt.rewind(base)
        tgt.forward_rows(ids, out_g)  # graph
        assert tgt.offset == base + 5 and tgt.pos_len.tolist() == [base + 5, base + 6]
        slots = ("k1", "k2", "v1", "v2")
        kv_g = [[getattr(c, n)[..., base:base + 5, :].clone() for n in slots] for c in (tgt.caches[0], tgt.caches[-1])]
        tgt.rewind(base)
        tgt._prefill_block(ids_d, out_e)
        kv_e = [[getattr(c, n)[..., base:base + 5, :] for n in slots] for c in (tgt.caches[0], tgt.caches[-1])]
        assert all(torch.equal(x, y) for x, y in zip(kv_g[0], kv_e[0])), f"first-layer rows differ at {base}"
        for x, y in zip(kv_g[1], kv_e[1]):
            assert_close(down(x), down(y).astype(np.float64), "float16", atol=2e-2, rtol=2e-2,
                         what=f"last-layer rows at {base}")
        assert_close(down(out_g), down(out_e).astype(np.float64), "float16", atol=1e-2, rtol=2e-2,
                     what=f"graph vs eager at {base}")
    tgt.check_rows_error()
    assert len(tgt._row_graphs) == 1


def test_speculative_greedy_equals_target_greedy(cuda):
    from mlx_motif.speculative import SpeculativeDecoder

    tgt, dft = _models(cuda)
    prompt = [3, 77, 512, 9, 140]
    ref = tgt.generate(prompt, 24)
    spec = SpeculativeDecoder(tgt, dft, k=4, temperature=0.0)
    got = spec.generate(prompt, 24)
    assert got == ref  # an unrelated draft is (nearly) always rejected: one target forward per token


def test_self_draft_accepts_every_token(cuda):
    """A draft with the target's own weights (separate caches) proposes the target's argmaxes: all K
    accepted each cycle, K + 1 tokens per target forward, output equal to the target's greedy."""
    from mlx_motif.model import MotifDecoder
    from mlx_motif.speculative import SpeculativeDecoder

    tgt, _ = _models(cuda)
    twin = MotifDecoder(tgt.args, tgt.weights_dict(), cache="fp16", max_seq=512, device=cuda)
    prompt = [3, 77, 512, 9, 140]
    ref = tgt.generate(prompt, 25)
    spec = SpeculativeDecoder(tgt, twin, k=4, temperature=0.0)
    assert spec.generate(prompt, 25) == ref
    assert spec.stats["target_forwards"] == 5 and spec.stats["accepted"] == 20


def test_speculative_sampling_runs_and_self_draft_accepts_all(cuda):
    from mlx_motif.speculative import SpeculativeDecoder

    tgt, dft = _models(cuda)
    spec = SpeculativeDecoder(tgt, dft, k=4, temperature=0.7, seed=3)
    toks = spec.generate([3, 77, 512], 40)
    assert len(toks) == 40 and all(0 <= t < 1024 for t in toks)
    s = spec.stats
    assert s["cycles"] == s["target_forwards"] and 0 <= s["accepted"] <= s["drafted"]
