"""Speculative decoding: a small draft decoder proposes K tokens, the target verifies them in one
batched ``[1, K+1]`` forward, and rejection sampling keeps the target's distribution.

Mirrors the reference's speculative loop (``swift/Sources/MotifKit/MotifSpeculativeDecoding.swift``
108-400): a persistent draft KV cache trimmed on rejection, K draft tokens per cycle sampled at
the same temperature as the target, one verify forward over ``[last, x_1 .. x_K]``, acceptance of
x_i with probability min(1, p_i(x_i) / q_i(x_i)), a replacement drawn from max(0, p_i − q_i) at
the first rejection, and a bonus token from p_K when all K are accepted. At temperature 0 the
rule accepts while the draft equals the target's argmax, so the output equals the target's
greedy decode.

Under tensor parallelism the target is sharded and the draft is replicated on every rank: each
rank runs the same draft steps (same seed, same kernels), the verify gathers the full vocabulary
rows, and the acceptance kernel draws the same tokens everywhere, so the ranks stay in step with
no extra exchange.

Device work per cycle: K draft decode steps (CUDA graphs, sampling in the head), one target
row-block forward with logits (a CUDA graph after its first call), one acceptance kernel; the host
reads back two int32 and the row block's error word per cycle.
"""

from __future__ import annotations

import torch

from ._native import check, lib, ptr, stream
from .model import MotifDecoder


class SpeculativeDecoder:
    def __init__(self, target: MotifDecoder, draft: MotifDecoder, k: int = 4, temperature: float = 0.7,
                 seed: int = 0):
        if draft.tp_group is not None:
            raise ValueError("the draft runs on one GPU (under tensor parallelism every rank holds a replica)")
        V = target.V_local * target.tp  # the verify gathers the target's vocabulary shards
        if V != draft.V_local:
            raise ValueError(f"target vocabulary {V} != draft vocabulary {draft.V_local}")
        if not 1 <= k <= 16:
            raise ValueError("k must be in 1..16")
        self.target, self.draft, self.k = target, draft, k
        self.temperature = float(temperature)
        self.seed = int(seed)
        dev = target.device
        self.q_logits = torch.empty((k, draft.V_local), dtype=torch.float16, device=dev)
        self.p_logits = torch.empty((k + 1, V), dtype=torch.float16, device=dev)
        self.draft_tokens = torch.zeros(k, dtype=torch.int32, device=dev)
        self.verify_ids = torch.zeros(k + 1, dtype=torch.int32, device=dev)
        self.result = torch.zeros(2, dtype=torch.int32, device=dev)
        self.result_host = torch.zeros(2, dtype=torch.int32).pin_memory()
        self.stats = {"cycles": 0, "drafted": 0, "accepted": 0, "target_forwards": 0}
        draft.set_sampling(self.temperature, seed=self.seed, stream_id=1)

    def generate(self, prompt_ids, n_tokens: int) -> list[int]:
        """Ingest the prompt into both models, then generate ``n_tokens`` tokens (the first one
        sampled from the target's distribution after the prompt)."""
        t, dft, k = self.target, self.draft, self.k
        prompt = [int(x) for x in prompt_ids]
        t.reset()
        dft.reset()
        # both caches hold prompt[:-1]; `last` is the committed token not yet in either cache
        t.ingest(prompt[:-1])
        dft.ingest(prompt[:-1])
        last = prompt[-1]
        out: list[int] = []
        st = stream(t.device)
        while len(out) < n_tokens:
            base = t.offset
            # K draft tokens: draft steps on last, x_1 .. x_{K-1}
            dft.token.fill_(last)
            for i in range(k):
                dft.step_device(with_head=True)
                self.q_logits[i].copy_(dft.logits)
                self.draft_tokens[i : i + 1].copy_(dft.token)
            # verify [last, x_1 .. x_K] in one target forward
            self.verify_ids[0] = last
            self.verify_ids[1:].copy_(self.draft_tokens)
            t.forward_rows(self.verify_ids, self.p_logits)
            check(lib.motif_speculative_accept(ptr(self.p_logits), ptr(self.q_logits), self.p_logits.shape[1],
                                               ptr(self.draft_tokens), k, self.p_logits.shape[1], self.temperature,
                                               self.seed,
                                               None, base, ptr(self.result), st), "speculative_accept")
            self.result_host.copy_(self.result)
            t.check_rows_error()
            n_acc, nxt = int(self.result_host[0]), int(self.result_host[1])
            accepted = self.draft_tokens[:n_acc].tolist()
            # target: rows of last and x_1 .. x_n are valid
            t.rewind(base + n_acc + 1)
            if n_acc < k:
                dft.rewind(base + n_acc + 1)
            else:  # the draft never ran x_K: feed it before the next cycle
                dft.token.fill_(accepted[-1])
                dft.step_device(with_head=False)
            out.extend(accepted + [nxt])
            last = nxt
            s = self.stats
            s["cycles"] += 1
            s["drafted"] += k
            s["accepted"] += n_acc
            s["target_forwards"] += 1
        return out[:n_tokens]
