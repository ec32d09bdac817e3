"""Tensor-parallel partition math on CPU (gloo, world size 2).

Each rank cuts the TINY checkpoint with ``leanstack_b200.tp``, runs one decoder
layer on its shard with the oracle's torch ops (fp32 partials for the row-split
o_proj / down_proj, summed by a gloo all-reduce, rounded once), and the result
must match the oracle's unsharded layer.  The head's argmax keys are reduced
with a MAX all-reduce and must pick the oracle's greedy token, lowest id on
ties across shards.  No GPU is used.
"""

from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp
import torch.nn.functional as F

from leanstack_b200 import synth, tp
from leanstack_b200.config import QWEN3_4B, TINY
from oracle import qwen_oracle as qo


def test_local_geometry_and_divisibility():
    g8 = tp.local_geometry(QWEN3_4B, 8)
    assert (g8.num_attention_heads, g8.num_key_value_heads, g8.intermediate_size) == (4, 1, 1216)
    assert g8.hidden_size == QWEN3_4B.hidden_size and g8.vocab_size == QWEN3_4B.vocab_size
    assert g8.num_key_value_groups == QWEN3_4B.num_key_value_groups
    s = tp.shard_info(QWEN3_4B, 3, 8)
    assert (s.vocab_offset, s.vocab_rows) == (3 * 18992, 18992)
    with pytest.raises(ValueError):
        tp.local_geometry(QWEN3_4B, 3)


def test_shards_reassemble_to_the_checkpoint():
    g = TINY
    full = synth.synth_layer(g, 0, 5)
    world = 2
    shards = [tp.shard_layer_tensors(full, g, 0, r, world) for r in range(world)]
    p = "model.layers.0."
    for name in ("self_attn.q_proj.weight", "self_attn.k_proj.weight", "self_attn.v_proj.weight",
                 "mlp.gate_proj.weight", "mlp.up_proj.weight"):
        assert torch.equal(torch.cat([s[p + name] for s in shards], 0), full[p + name])
    for name in ("self_attn.o_proj.weight", "mlp.down_proj.weight"):
        assert torch.equal(torch.cat([s[p + name] for s in shards], 1), full[p + name])
    # The re-fused gate_up of a rank is [gate_r; up_r], not a slice of [gate; up].
    w0 = qo.fuse_layer(shards[0], 0).gate_up_proj
    i_loc = g.intermediate_size // world
    assert torch.equal(w0[:i_loc], full[p + "mlp.gate_proj.weight"][:i_loc])
    assert torch.equal(w0[i_loc:], full[p + "mlp.up_proj.weight"][:i_loc])


def test_argmax_key_order():
    gen = torch.Generator().manual_seed(3)
    vals = (torch.randn(400, generator=gen) * 4).bfloat16().float().tolist() + [0.0, -0.0, 1.5, 1.5, -3.0]
    ids = torch.randint(0, 151936, (len(vals),), generator=gen).tolist()
    for i in range(len(vals)):
        for j in range(0, len(vals), 7):
            a = (vals[i], -ids[i])
            b = (vals[j], -ids[j])
            ka, kb = tp.argmax_key(vals[i], ids[i]), tp.argmax_key(vals[j], ids[j])
            assert (ka > kb) == (a > b) and (ka == kb) == (a == b), (vals[i], ids[i], vals[j], ids[j])
        assert tp.argmax_key_id(tp.argmax_key(vals[i], ids[i])) == ids[i]
    assert tp.argmax_key(-0.0, 7) == tp.argmax_key(0.0, 7)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _tp_layer(m: qo.OracleModel, w: qo.LayerWeights, hidden, kv, cos, sin, mask, comm: tp.TPComm):
    eps = m.rms_norm_eps
    xn = qo.rmsnorm(hidden, w.input_layernorm, eps)
    q, k, v = qo.qkv_project(xn, w, m.num_attention_heads, m.num_key_value_heads, m.head_dim, cos, sin, eps)
    kv.append(0, k, v)
    k, v = kv.get(0)
    attn = qo.attention(q, k, v, mask, m.head_dim ** -0.5)
    part = attn.float() @ w.o_proj.float().t()
    comm.all_reduce_sum(part)
    h = hidden + part.to(hidden.dtype)
    n = qo.rmsnorm(h, w.post_attention_layernorm, eps)
    gu = F.linear(n, w.gate_up_proj)
    i_loc = w.gate_up_proj.shape[0] // 2
    g_, u = torch.split(gu, (i_loc, i_loc), dim=-1)
    part2 = (F.silu(g_) * u).float() @ w.down_proj.float().t()
    comm.all_reduce_sum(part2)
    return h + part2.to(hidden.dtype)


def _worker(rank: int, world: int, port: int, q: mp.Queue) -> None:
    try:
        _work(rank, world, port, q)
    except BaseException as e:  # report instead of leaving the parent waiting
        q.put((rank, "error", repr(e)))
        raise


def _work(rank: int, world: int, port: int, q: mp.Queue) -> None:
    import datetime

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        torch.set_num_threads(2)
        g = TINY
        tensors = synth.synth_checkpoint(g, 9)
        comm = tp.TPComm(rank, world)
        full = qo.OracleModel.from_checkpoint(g, tensors, layer_indices=[0])
        local_g = tp.local_geometry(g, world)
        shard = tp.shard_info(g, rank, world)
        local = qo.OracleModel.from_checkpoint(local_g, tp.shard_checkpoint(tensors, g, rank, world, [0]),
                                               layer_indices=[0])
        past, q_len, batch, S = 37, 3, 2, 64
        cos, sin = full.rope(S)
        gen = torch.Generator().manual_seed(1)
        hidden = torch.randn(batch, q_len, g.hidden_size, generator=gen).bfloat16()
        k_past = torch.randn(batch, g.num_key_value_heads, past, g.head_dim, generator=gen).bfloat16()
        v_past = torch.randn(batch, g.num_key_value_heads, past, g.head_dim, generator=gen).bfloat16()
        c, s = cos[past:past + q_len].unsqueeze(0), sin[past:past + q_len].unsqueeze(0)
        mask = qo.decode_mask(q_len, past + q_len, torch.bfloat16)

        kv_full = full.new_kv(batch, S)
        kv_full.append(0, k_past, v_past)
        ref = qo.layer_forward(full, 0, full.layers[0], hidden, kv_full, c, s, mask)

        hk = local_g.num_key_value_heads
        kv_loc = local.new_kv(batch, S)
        kv_loc.append(0, k_past[:, rank * hk:(rank + 1) * hk].contiguous(),
                      v_past[:, rank * hk:(rank + 1) * hk].contiguous())
        out = _tp_layer(local, local.layers[0], hidden, kv_loc, c, s, mask, comm)

        # Greedy head: vocab shards -> keys -> MAX all-reduce.
        hn = qo.rmsnorm(out[:, -1], full.final_norm, g.rms_norm_eps)
        logits = F.linear(hn, full.lm_head)                       # [B, V] bf16, as the oracle head
        lo = shard.vocab_offset
        logits_tied = logits.clone()
        logits_tied[:, 5] = 50.0                                   # the same best logit in both shards:
        logits_tied[:, g.vocab_size - 3] = 50.0                    # the lowest id (5) must win
        got = []
        for lg in (logits, logits_tied):
            loc = lg[:, lo:lo + shard.vocab_rows].float()
            best = loc.max(dim=1).values
            keys = torch.tensor([tp.argmax_key(best[b].item(), lo + int((loc[b] == best[b]).nonzero()[0]))
                                 for b in range(batch)], dtype=torch.int64)
            comm.all_reduce_max(keys)
            got.append(([tp.argmax_key_id(int(k)) for k in keys], lg.float().argmax(dim=1).tolist()))
        q.put((rank, (out.float() - ref.float()).abs().max().item(), ref.float().abs().max().item(),
               (out == ref).float().mean().item(), got))
    finally:
        dist.destroy_process_group()


def test_tp_layer_and_head_match_unsharded_oracle_world2():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=240) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    errors = [r for r in results if r[1] == "error"]
    assert not errors, errors
    assert all(p.exitcode == 0 for p in procs)
    for rank, err, ref_max, exact, got in results:
        assert err <= 2e-2 * max(1.0, ref_max), (rank, err)
        assert exact > 0.97, (rank, exact)
        for ids, want in got:
            assert ids == want, (rank, ids, want)
