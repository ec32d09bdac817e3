"""Speculative verify on the device against the reference.

* ``ls_spec_accept`` against a Python restatement of the reference's
  accept / reject loop (``qwen_explicit_runtime_loop.py:813-866``), with
  planted agreeing prefixes of every length.
* The dual-model loop (draft engine proposes, target engine verifies, device
  accept) reproduces the reference's own token streams on the tiny stack
  (``tests/golden/tiny_stack.pt``: a distinct random draft, and the target as
  its own draft), eager and as one CUDA graph per cycle.
* A batched verify pass (B 4, k 4, M 20, tcgen05 linears) returns, at every
  position, the oracle's greedy token for the same inputs.
"""

from __future__ import annotations

import pytest
import torch

from leanstack_b200 import kernels as K
from leanstack_b200 import synth
from leanstack_b200.config import TINY, TINY_DRAFT
from leanstack_b200.engine import DecodeEngine
from leanstack_b200.leanserve import materialize_from_tensors
from leanstack_b200.speculative import SpeculativeDecoder
from oracle import qwen_oracle as qo

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _gold(golden_dir, name):
    return torch.load(golden_dir / name, weights_only=False)


def test_spec_accept_matches_reference_rule():
    B, k, cap = 9, 4, 7
    gen = torch.Generator().manual_seed(5)
    verdict = torch.randint(0, 1000, (B, k + 1), generator=gen)
    ids = torch.randint(0, 1000, (B, k + 1), generator=gen)
    for b in range(B):  # sequence b agrees on its first min(b, k) proposals
        n = min(b, k)
        ids[b, 1:1 + n] = verdict[b, :n]
        if n < k:
            ids[b, 1 + n] = verdict[b, n] + 1
    pos = torch.arange(B, dtype=torch.int32) * 10 + 100
    dpos = pos + k
    out = torch.full((B, cap), -1, dtype=torch.int64)
    out_len = torch.tensor([0, 0, 0, 0, 0, 5, 6, 7, 1], dtype=torch.int32)
    d_ids, d_ver, d_pos, d_dpos = ids.to(DEV), verdict.to(DEV), pos.to(DEV), dpos.to(DEV)
    d_out, d_len = out.to(DEV), out_len.to(DEV)
    nxt = torch.empty(B, dtype=torch.int64, device=DEV)
    acc = torch.empty(B, dtype=torch.int32, device=DEV)
    K.spec_accept(d_ids, d_ver, B, k, next_ids=nxt, accepted=acc, cache_pos=d_pos, draft_cache_pos=d_dpos,
                  out_tokens=d_out, out_len=d_len)
    torch.cuda.synchronize()
    for b in range(B):
        n = 0
        committed = []
        for i in range(k):  # the reference's loop
            if ids[b, 1 + i] != verdict[b, i]:
                committed.append(int(verdict[b, i]))
                break
            committed.append(int(ids[b, 1 + i]))
            n += 1
        if n == k:
            committed.append(int(verdict[b, k]))
        assert int(acc[b]) == n == min(b, k)
        assert int(nxt[b]) == committed[-1] == int(d_ids[b, 0])
        assert int(d_pos[b]) == int(pos[b]) + n + 1
        assert int(d_dpos[b]) == int(pos[b]) + min(n + 1, k)
        start = int(out_len[b])
        want = (out[b, :start].tolist() + committed)[:cap]
        assert int(d_len[b]) == len(want)
        assert d_out[b, :len(want)].tolist() == want


@pytest.mark.parametrize("use_graph", [False, True])
def test_dual_model_speculative_matches_reference_streams(golden_dir, use_graph):
    gold = _gold(golden_dir, "tiny_stack.pt")
    prompt = gold["greedy"]["prompt"]
    tgt = materialize_from_tensors(TINY, synth.synth_checkpoint(TINY, 3, device=DEV), device=DEV)
    drf = materialize_from_tensors(TINY_DRAFT, synth.synth_checkpoint(TINY_DRAFT, 4, device=DEV), device=DEV)
    S = prompt.shape[1] + 24 + 4 + 8
    for name, draft_rt in (("spec_distinct", drf), ("spec_self", tgt)):
        t_eng = DecodeEngine(tgt, batch_size=1, max_seq_len=S, linear_backend="cuda_core", use_graph=use_graph)
        d_eng = DecodeEngine(draft_rt, batch_size=1, max_seq_len=S, linear_backend="cuda_core",
                             use_graph=use_graph)
        spec = SpeculativeDecoder(d_eng, t_eng, proposal_len=4, max_new_tokens=24, use_graph=use_graph)
        got = spec.generate(prompt)[0]
        print(name, got)
        assert got == gold[name]["tokens"].tolist(), name
        assert K.device_error() == 0


def test_batched_verify_pass_matches_oracle():
    B, k, P = 4, 4, 19
    t = synth.synth_checkpoint(TINY, 3, device=DEV)
    rt = materialize_from_tensors(TINY, t, device=DEV)
    orc = qo.OracleModel.from_checkpoint(TINY, {n: v.cpu() for n, v in t.items()})
    prompt = synth.token_ids((B, P), TINY.vocab_size, 21, "verify/prompt")
    eng = DecodeEngine(rt, batch_size=B, max_seq_len=64, linear_backend="tc")
    first = eng.prefill(prompt).cpu()
    props = synth.token_ids((B, k), TINY.vocab_size, 22, "verify/props")
    # plant agreement: sequence b proposes the oracle's own greedy continuation for b tokens
    kv = orc.new_kv(B, 64)
    pc = orc.rope(64)
    qo.stack_forward(orc, qo.embed(orc, prompt), kv, pc)
    cur = first.view(B, 1)
    kv2 = orc.new_kv(B, 64)
    qo.stack_forward(orc, qo.embed(orc, prompt), kv2, pc)
    greedy = []
    for _ in range(k):
        h = qo.stack_forward(orc, qo.embed(orc, cur), kv2, pc)
        cur = qo.greedy_token(orc, h).view(B, 1)
        greedy.append(cur.view(-1))
    greedy = torch.stack(greedy, 1)
    for b in range(B):
        props[b, :b] = greedy[b, :b]
    inp = eng.verify_inputs(k)
    inp[:, 0].copy_(first.to(DEV))
    inp[:, 1:].copy_(props.to(DEV))
    ids_in = torch.cat([first.view(B, 1), props], 1)
    eng.verify_step(k)
    verdict = eng.verdict[:B * (k + 1)].view(B, k + 1).cpu()
    h = qo.stack_forward(orc, qo.embed(orc, ids_in), kv, pc)
    want = torch.stack([qo.greedy_token(orc, h[:, i:i + 1]).view(B) for i in range(k + 1)], 1)
    assert torch.equal(verdict, want), (verdict, want)
    acc = eng.accepted.cpu().tolist()
    for b in range(B):
        n = 0
        while n < k and int(props[b, n]) == int(want[b, n]):
            n += 1
        assert acc[b] == n
    lens = eng.sync_cursors()
    assert lens == [P + acc[b] + 1 for b in range(B)]
