"""Dual-model greedy-exact speculative decoding on two resident engines.

Restates ``run_dual_model_speculative_request``
(``experiments/models/qwen_explicit_runtime_loop.py:651-916``) for a batch of
sequences whose cursors move independently on the device:

1. the draft engine consumes each sequence's current token and proposes k
   tokens greedily (k decode steps: inputs current, d1 .. d(k-1));
2. the target engine verifies ``[current, d1..dk]`` in one pass (M = B·(k+1),
   greedy token after every position, ``qwen_explicit_runtime_loop.py:804-811``);
3. ``ls_spec_accept`` keeps the longest agreeing prefix, takes the target's
   token after it as the next current token (correction or bonus), rolls both
   cursors back (target ``base + 1 + n``, draft ``base + min(n + 1, k)``) and
   appends the committed tokens to a per-sequence log (``:813-866``).

A whole cycle is one CUDA-graph replay once captured; nothing returns to the
host until :meth:`tokens` reads the log.  As in the reference, the token the
prefill produces is the first ``current`` and is not itself emitted.
"""

from __future__ import annotations

import torch

from .engine import DecodeEngine


class SpeculativeDecoder:
    def __init__(self, draft: DecodeEngine, target: DecodeEngine, proposal_len: int, max_new_tokens: int,
                 use_graph: bool = True):
        if draft.B != target.B:
            raise ValueError("draft and target engines must hold the same batch")
        if proposal_len < 1:
            raise ValueError("proposal_len must be positive")
        if target.B * (proposal_len + 1) > target.T:
            raise ValueError(f"verify of {target.B} x {proposal_len + 1} tokens exceeds the target's "
                             f"{target.T}-token step")
        self.draft, self.target = draft, target
        self.B = target.B
        self.k = proposal_len
        self.cap = max_new_tokens
        dev = target.rt.device
        self.out = torch.zeros(self.B, max_new_tokens, device=dev, dtype=torch.int64)
        self.out_len = torch.zeros(self.B, device=dev, dtype=torch.int32)
        self.use_graph = use_graph
        self.graphs: dict[int, torch.cuda.CUDAGraph] = {}

    def prefill(self, prompt_ids: torch.Tensor) -> torch.Tensor:
        """Prefill both models; returns the target's first greedy token per sequence (the first current)."""
        first = self.target.prefill(prompt_ids)
        self.draft.prefill(prompt_ids)
        self.target.next_ids.copy_(first)
        self.out_len.zero_()
        return first

    def _cycle(self, k: int) -> None:
        d, t = self.draft, self.target
        ids = t.verify_inputs(k)
        ids[:, 0].copy_(t.next_ids)
        d.arenas.ids[:self.B].copy_(t.next_ids)
        for i in range(k):
            d._forward(1, head=True)  # greedy proposal into the draft's ids, cursor + 1
            ids[:, i + 1].copy_(d.arenas.ids[:self.B])
        t._verify_once(k, draft_cache_pos=d.kv.cache_pos, out_tokens=self.out, out_len=self.out_len)

    def _capture(self, k: int) -> None:
        d, t = self.draft, self.target
        saved = [x.clone() for x in (d.kv.cache_pos, t.kv.cache_pos, d.arenas.ids, t.arenas.ids, t.next_ids,
                                     self.out, self.out_len)]
        self._cycle(k)  # eager warm-up
        torch.cuda.synchronize()
        for dst, src in zip((d.kv.cache_pos, t.kv.cache_pos, d.arenas.ids, t.arenas.ids, t.next_ids, self.out,
                             self.out_len), saved):
            dst.copy_(src)
        graph = torch.cuda.CUDAGraph()
        stream = torch.cuda.Stream()
        stream.wait_stream(torch.cuda.current_stream())
        with torch.cuda.graph(graph, stream=stream):
            self._cycle(k)
        torch.cuda.current_stream().wait_stream(stream)
        torch.cuda.synchronize()
        self.graphs[k] = graph

    def cycle(self, k: int | None = None) -> None:
        """Enqueue one draft-propose / target-verify / accept cycle (no host sync)."""
        k = self.k if k is None else k
        for eng in (self.draft, self.target):
            if max(eng.kv.sequence_lens) + k + 1 > eng.S:
                raise ValueError("KV cache is full")
        if self.use_graph:
            if k not in self.graphs:
                self._capture(k)
            self.graphs[k].replay()
        else:
            self._cycle(k)
        # conservative host bounds until sync_cursors()
        self.draft.kv.sequence_lens = [n + k for n in self.draft.kv.sequence_lens]
        self.target.kv.sequence_lens = [n + k + 1 for n in self.target.kv.sequence_lens]

    def sync_cursors(self) -> None:
        self.draft.sync_cursors()
        self.target.sync_cursors()

    def tokens(self) -> list[list[int]]:
        """The committed tokens of each sequence so far (reads the device log)."""
        lens = self.out_len.tolist()
        out = self.out.cpu()
        return [out[b, :lens[b]].tolist() for b in range(self.B)]

    def generate(self, prompt_ids: torch.Tensor, max_new_tokens: int | None = None) -> list[list[int]]:
        """Prefill, then cycle until every sequence has ``max_new_tokens`` committed.

        Near the end the proposal length shrinks to the tokens still missing
        (``min(k, remaining)``, ``qwen_explicit_runtime_loop.py:741``), computed
        from the sequence that has the most left; this reads the log length
        each cycle (one small host sync).
        """
        n_new = self.cap if max_new_tokens is None else min(max_new_tokens, self.cap)
        self.prefill(prompt_ids)
        while True:
            have = min(self.out_len.tolist())
            if have >= n_new:
                break
            self.cycle(min(self.k, n_new - have))
            self.sync_cursors()
        return [t[:n_new] for t in self.tokens()]
