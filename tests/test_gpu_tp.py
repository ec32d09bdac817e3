"""Tensor-parallel decode engine on 2 GPUs (NCCL), against the single-GPU engine.

Each rank runs in its own process on its own GPU with its shard of the same
seeded checkpoint.  The TP engine's greedy tokens must equal the single-GPU
engine's (fp32 partial sums differ only in summation order) and its last hidden
rows must agree within the north-star bound.  Both the eager step and the
CUDA-graph step (NCCL captured in the graph) are checked, for the CUDA-core
(batch 1) and tensor-core (batch 4) linears, each with NCCL and with the
one-shot all-reduce over peer memory (fused into the CUDA-core linear; a
kernel after the tcgen05 GEMM's fp32 partials), whose results must equal the
NCCL path's bit for bit at world size 2.  Skipped with fewer than 2 GPUs.
"""

from __future__ import annotations

import datetime
import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu

WORLD = 2
CASES = ((1, "cuda_core", False), (1, "cuda_core", True), (4, "tc", False), (4, "tc", True))


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _run(rank: int, port: int, q) -> None:
    import torch.distributed as dist

    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
        torch.cuda.set_device(rank)
        dist.init_process_group("nccl", rank=rank, world_size=WORLD, timeout=datetime.timedelta(seconds=120))
        from leanstack_b200 import kernels as K
        from leanstack_b200 import synth, tp
        from leanstack_b200.config import TINY
        from leanstack_b200.engine import DecodeEngine
        from leanstack_b200.leanserve import materialize_from_tensors

        dev = torch.device("cuda", rank)
        g = TINY
        out = {}
        for batch, backend, p2p in CASES:
            prompt = synth.token_ids((batch, 24), g.vocab_size, 3, "tp/prompt")
            rt, shard = tp.materialize_tp_shard(g, synth.synth_checkpoint(g, 3, device=dev), rank, WORLD, device=dev)
            comm = tp.TPComm(rank, WORLD)
            if p2p:
                comm.enable_p2p(g.hidden_size)
            for use_graph in (False, True):
                eng = DecodeEngine(rt, batch_size=batch, max_seq_len=128, linear_backend=backend, tp=comm,
                                   shard=shard, use_graph=use_graph)
                toks = eng.generate(prompt, 12).cpu()
                rows = eng.last_head_rows().float().cpu()
                out[(batch, backend, p2p, use_graph)] = (toks, rows)
                eng.graph = None
                del eng
            assert K.device_error() == 0
            comm.close()
            if rank == 0 and (batch, backend, "single") not in out:
                full = materialize_from_tensors(g, synth.synth_checkpoint(g, 3, device=dev), device=dev,
                                                free_source=True)
                e1 = DecodeEngine(full, batch_size=batch, max_seq_len=128, linear_backend=backend)
                out[(batch, backend, "single")] = (e1.generate(prompt, 12).cpu(), e1.last_head_rows().float().cpu())
                del e1
        torch.cuda.synchronize()
        q.put((rank, out))
    except BaseException as e:  # report to the parent instead of leaving it waiting
        q.put((rank, repr(e)))
        raise
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


def test_tp2_engine_matches_single_gpu_engine():
    if torch.cuda.device_count() < WORLD:
        pytest.skip(f"needs {WORLD} GPUs")
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_run, args=(r, port, q)) for r in range(WORLD)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=600) for _ in range(WORLD))
    for p in procs:
        p.join(timeout=120)
    for r, v in res.items():
        assert not isinstance(v, str), f"rank {r}: {v}"
    out0, out1 = res[0], res[1]
    for batch, backend, p2p in CASES:
        ref_toks, ref_rows = out0[(batch, backend, "single")]
        for use_graph in (False, True):
            toks0, rows0 = out0[(batch, backend, p2p, use_graph)]
            toks1, rows1 = out1[(batch, backend, p2p, use_graph)]
            assert torch.equal(toks0, toks1), "ranks disagree"
            assert torch.equal(rows0, rows1), "ranks hold different residual streams"
            same = (toks0 == ref_toks).float().mean().item()
            assert same >= 0.9, (batch, backend, p2p, use_graph, toks0.tolist(), ref_toks.tolist())
            assert torch.equal(toks0[:, :4], ref_toks[:, :4])
            err = (rows0 - ref_rows).abs().max().item()
            if torch.equal(toks0, ref_toks):
                assert err <= 2e-2 * max(1.0, ref_rows.abs().max().item()), err
            if p2p:  # two fp32 partials sum the same way on either path
                assert torch.equal(toks0, out0[(batch, backend, False, use_graph)][0])
                assert torch.equal(rows0, out0[(batch, backend, False, use_graph)][1])
