#!/usr/bin/env python
"""Per-kernel timing at the Qwen3-4B decode shapes (CUDA events, cold weights).

``python microbench.py [--kernels a,b] [--reps N] [--m 1] [--seq 600]``

Each kernel runs over ``--copies`` distinct weight sets (more bytes than the
126 MB L2), rotating between them, so every launch streams its weights from
HBM.  Prints one JSON line per kernel: average launch time, algorithmic bytes
per launch and GB/s.  This is also the small case used for ncu captures.
"""

from __future__ import annotations

import argparse
import json
import sys
from pathlib import Path

import torch

sys.path.insert(0, str(Path(__file__).resolve().parent))

from leanstack_b200 import kernels as K  # noqa: E402
from leanstack_b200 import synth  # noqa: E402
from leanstack_b200.config import QWEN3_4B  # noqa: E402


def _events():
    return torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)


def _time(fn, reps: int) -> float:
    """Average device time of ``fn`` over ``reps`` back-to-back launches captured
    in one CUDA graph (no host launch overhead between them, as in the decode step)."""
    fn(0)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())
    with torch.cuda.graph(graph, stream=stream):
        for i in range(reps):
            fn(i)
    torch.cuda.current_stream().wait_stream(stream)
    graph.replay()
    torch.cuda.synchronize()
    a, b = _events()
    a.record()
    graph.replay()
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b) / 1000.0 / reps


def profile_step(kind: str) -> int:
    """Random-init Qwen3-4B, prompt through ``prefill_full``, one captured step
    replayed once untimed, then timed twice (CUDA events) inside NVTX 'step'."""
    from leanstack_b200.engine import DecodeEngine
    from leanstack_b200.leanserve import materialize_from_tensors

    g = QWEN3_4B
    dev = torch.device("cuda")
    rt = materialize_from_tensors(g, synth.synth_checkpoint(g, 1, device=dev), device=dev, free_source=True)
    B, cached, k = {"bs1": (1, 512, 0), "bs32": (32, 2048, 0), "verify": (16, 1024, 4)}[kind]
    if kind == "bs1":  # config 2: static KV of 4096 positions, the default (CUDA-core) backend
        eng = DecodeEngine(rt, batch_size=B, max_seq_len=4096)
    else:
        eng = DecodeEngine(rt, batch_size=B, max_seq_len=cached + 64, linear_backend="tc")
    eng.prefill_full(synth.token_ids((B, cached), g.vocab_size, 1, f"mb/step/{kind}"))
    if kind in ("bs1", "bs32"):
        eng.capture()
        step = eng.decode_step
    else:
        inp = eng.verify_inputs(k)
        props = synth.token_ids((B, k), g.vocab_size, 1, "mb/step/props").to(dev)

        def step():
            inp[:, 1:].copy_(props)
            eng.verify_step(k)
    step()
    torch.cuda.synchronize()
    a, b = _events()
    torch.cuda.nvtx.range_push("step")
    a.record()
    for _ in range(2):
        step()
    b.record()
    torch.cuda.nvtx.range_pop()
    torch.cuda.synchronize()
    print(json.dumps({"step": kind, "batch": B, "cached": cached, "ms_per_step": a.elapsed_time(b) / 2,
                      "launches_per_step": eng.kernel_launches_per_step() if kind != "verify" else None}))
    return 0


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--kernels", default="qkv,attention,oproj,gateup,down,lmhead,qknorm,embed")
    ap.add_argument("--reps", type=int, default=20)
    ap.add_argument("--m", type=int, default=1)
    ap.add_argument("--seq", type=int, default=600, help="cached positions for attention")
    ap.add_argument("--copies", type=int, default=4)
    ap.add_argument("--batch", type=int, default=1, help="sequences of the prefill_attn case")
    ap.add_argument("--step", choices=("bs1", "bs32", "verify"), default=None,
                    help="instead of kernels: one whole captured step of Qwen3-4B (config 3 bs32 decode over 2048 "
                         "cached, or the config-4 verify pass), two replays inside the NVTX range 'step' "
                         "(for `ncu --nvtx --nvtx-include step/`)")
    args = ap.parse_args(argv)
    if args.step:
        return profile_step(args.step)
    g = QWEN3_4B
    dev = torch.device("cuda")
    m, H, I = args.m, g.hidden_size, g.intermediate_size
    C = args.copies

    def w(shape, name):
        return [synth.normal(shape, 0.02, c, name, device=dev) for c in range(C)]

    x = synth.normal((m, H), 1.0, 0, "mb/x", device=dev)
    nw = synth.norm_weight((H,), 0, "mb/nw", device=dev)
    out = {}
    wanted = set(args.kernels.split(","))
    if "qkv" in wanted or "qknorm" in wanted:
        qkv_w = w((g.qkv_dim, H), "mb/qkv")
        qn = synth.norm_weight((g.head_dim,), 0, "mb/qn", device=dev)
        cos, sin = (torch.randn(4096, 64, device=dev).bfloat16() for _ in range(2))
        scratch = torch.empty(m, g.qkv_dim, device=dev, dtype=torch.bfloat16)
        q = torch.empty(m, g.num_attention_heads, g.head_dim, device=dev, dtype=torch.bfloat16)
        kc = torch.zeros(m, g.num_key_value_heads, 4096, g.head_dim, device=dev, dtype=torch.bfloat16)
        vc = torch.zeros_like(kc)
        pos = torch.full((m,), 100, device=dev, dtype=torch.int32)
        if "qkv" in wanted:
            t = _time(lambda i: K.linear(x, qkv_w[i % C], norm_w=nw, out=scratch), args.reps)
            out["qkv(norm+gemv)"] = (t, g.qkv_dim * H * 2)
        if "qknorm" in wanted:
            from leanstack_b200 import _native as nat

            def qk(i):
                nat.call("ls_rmsnorm_qkv_rope_kvappend", x.data_ptr(), m, 1, H, nw.data_ptr(), 1e-6,
                         qkv_w[i % C].data_ptr(), g.num_attention_heads, g.num_key_value_heads, g.head_dim,
                         qn.data_ptr(), qn.data_ptr(), cos.data_ptr(), sin.data_ptr(), 4096, 0, pos.data_ptr(), 0,
                         kc.data_ptr(), vc.data_ptr(), 4096, None, None, scratch.data_ptr(), q.data_ptr(),
                         torch.cuda.current_stream().cuda_stream)
            t = _time(qk, args.reps)
            out["qkv+qknorm_rope_append (2 kernels)"] = (t, g.qkv_dim * H * 2)
    if "attention" in wanted:
        S = 4096
        kcs = [synth.normal((m, g.num_key_value_heads, S, g.head_dim), 1.0, c, "mb/k", device=dev) for c in range(2)]
        vcs = [synth.normal((m, g.num_key_value_heads, S, g.head_dim), 1.0, c, "mb/v", device=dev) for c in range(2)]
        q = synth.normal((m, g.num_attention_heads, g.head_dim), 1.0, 0, "mb/q", device=dev)
        pos = torch.full((m,), args.seq - 1, device=dev, dtype=torch.int32)
        ws = torch.zeros(K.attention_workspace_bytes(m, 1, 32, 8, 128, S), device=dev, dtype=torch.uint8)
        o = torch.empty(m, g.q_dim, device=dev, dtype=torch.bfloat16)
        t = _time(lambda i: K.decode_attention(q, kcs[i % 2], vcs[i % 2], m, 1, 32, 8, 128, S, 128 ** -0.5,
                                               cache_pos=pos, out=o, workspace=ws), args.reps)
        out[f"attention(seq={args.seq})"] = (t, m * args.seq * g.kv_dim * 2 * 2)
    if "verify_attn" in wanted:  # verify pass: --batch sequences x --m new tokens over --seq cached positions
        B, Q, S = args.batch, m, 2048
        kcs = [synth.normal((B, g.num_key_value_heads, S, g.head_dim), 1.0, c, "mb/vk", device=dev) for c in range(2)]
        vcs = [synth.normal((B, g.num_key_value_heads, S, g.head_dim), 1.0, c, "mb/vv", device=dev) for c in range(2)]
        q = synth.normal((B * Q, g.num_attention_heads, g.head_dim), 1.0, 0, "mb/vq", device=dev)
        pos = torch.full((B,), args.seq, device=dev, dtype=torch.int32)
        o = torch.empty(B * Q, g.q_dim, device=dev, dtype=torch.bfloat16)
        t = _time(lambda i: K.decode_attention(q, kcs[i % 2], vcs[i % 2], B, Q, 32, 8, 128, S, 128 ** -0.5,
                                               cache_pos=pos, out=o), args.reps)
        out[f"verify_attn(B={B},q={Q},seq={args.seq})"] = (t, B * (args.seq + Q) * g.kv_dim * 2 * 2)
    if "prefill_attn" in wanted:  # causal attention of --m prompt tokens per sequence, batch --batch
        B, P = args.batch, m
        kc = synth.normal((B, g.num_key_value_heads, P, g.head_dim), 1.0, 0, "mb/pk", device=dev)
        vc = synth.normal((B, g.num_key_value_heads, P, g.head_dim), 1.0, 0, "mb/pv", device=dev)
        q = synth.normal((B * P, g.num_attention_heads, g.head_dim), 1.0, 0, "mb/pq", device=dev)
        o = torch.empty(B * P, g.q_dim, device=dev, dtype=torch.bfloat16)
        ws = torch.zeros(max(256, K.attention_workspace_bytes(B, P, 32, 8, 128, P)), device=dev, dtype=torch.uint8)
        t = _time(lambda i: K.decode_attention(q, kc, vc, B, P, 32, 8, 128, P, 128 ** -0.5, uniform_past=0, out=o,
                                               workspace=ws), args.reps)
        flops = 4.0 * B * g.num_attention_heads * (P * (P + 1) / 2) * g.head_dim
        print(json.dumps({"kernel": f"prefill_attention(batch={B}, len={P})", "us": round(t * 1e6, 2),
                          "tflops": round(flops / t / 1e12, 1)}), flush=True)
    if "oproj" in wanted:
        ow = w((H, g.q_dim), "mb/o")
        a = synth.normal((m, g.q_dim), 1.0, 0, "mb/a", device=dev)
        h = torch.empty(m, H, device=dev, dtype=torch.bfloat16)
        t = _time(lambda i: K.oproj_residual(a, ow[i % C], x, out=h), args.reps)
        out["oproj+residual"] = (t, H * g.q_dim * 2)
    if "gateup" in wanted:
        guw = w((2 * I, H), "mb/gu")
        act = torch.empty(m, I, device=dev, dtype=torch.bfloat16)
        t = _time(lambda i: K.gateup_silu(x, nw, guw[i % C], 1e-6, out=act), args.reps)
        out["norm+gateup+silu"] = (t, 2 * I * H * 2)
    if "down" in wanted:
        dw = w((H, I), "mb/d")
        act = synth.normal((m, I), 1.0, 0, "mb/act", device=dev)
        h = torch.empty(m, H, device=dev, dtype=torch.bfloat16)
        t = _time(lambda i: K.down_residual(act, dw[i % C], x, out=h), args.reps)
        out["down+residual"] = (t, H * I * 2)
    if "lmhead" in wanted:
        lm = synth.normal((g.vocab_size, H), 0.02, 0, "mb/lm", device=dev)
        ids = torch.empty(m, device=dev, dtype=torch.int64)
        ws = torch.zeros(K.lmhead_workspace_bytes(m, g.vocab_size), device=dev, dtype=torch.uint8)
        t = _time(lambda i: K.lmhead_argmax(x, nw, lm, 1e-6, out_ids=ids, workspace=ws), args.reps)
        out["norm+lmhead+argmax"] = (t, g.vocab_size * H * 2)
    if "embed" in wanted:
        emb = synth.normal((g.vocab_size, H), 0.02, 0, "mb/emb", device=dev)
        ids = torch.tensor([5] * m, device=dev)
        xe = torch.empty(m, H, device=dev, dtype=torch.bfloat16)
        t = _time(lambda i: K.embed_gather(ids, emb, out=xe), args.reps)
        out["embed"] = (t, m * H * 2)
    big = {k for k in wanted if k.startswith("big_")}
    if big:  # large-M prefill GEMM; --m is the token count (e.g. 4096)
        def big_case(name, n_rows, k_dim, epi):
            wts = w((n_rows, k_dim), "mb/big" + name)
            xa = synth.normal((m, k_dim), 1.0, 0, "mb/bx" + name, device=dev)
            n_out = n_rows // 2 if epi == K.EPI_SILU_MUL else n_rows
            res = synth.normal((m, n_out), 1.0, 0, "mb/bres" + name, device=dev)
            o = torch.empty(m, n_out, device=dev, dtype=torch.bfloat16)
            t = _time(lambda i: K.gemm_big(xa, wts[i % C], epilogue=epi, residual=res, out=o), args.reps)
            out[f"big_{name}(m={m})"] = (t, 2.0 * m * n_rows * k_dim)  # FLOPs, not bytes
        if "big_qkv" in big:
            big_case("qkv", g.qkv_dim, H, K.EPI_STORE)
        if "big_gateup" in big:
            big_case("gateup", 2 * I, H, K.EPI_SILU_MUL)
        if "big_oproj" in big:
            big_case("oproj", H, g.q_dim, K.EPI_RESIDUAL)
        if "big_down" in big:
            big_case("down", H, I, K.EPI_RESIDUAL)
    tc = {k for k in wanted if k.startswith("tc_")}
    if tc:
        def tc_case(name, n_rows, k_dim, epi, n_out, extra=None):
            ws_ = torch.zeros(K.gemm_workspace_bytes(m, k_dim, n_out, epi), device=dev, dtype=torch.uint8)
            wts = w((n_rows, k_dim), "mb/" + name)
            xa = synth.normal((m, k_dim), 1.0, 0, "mb/xa" + name, device=dev)
            res = synth.normal((m, n_out), 1.0, 0, "mb/res" + name, device=dev)
            o = torch.empty(m, n_out, device=dev, dtype=torch.bfloat16)
            t = _time(lambda i: K.gemm_tc(xa, wts[i % C], epilogue=epi, residual=res, out=o, workspace=ws_),
                      args.reps)
            out[f"tc_{name}(m={m})"] = (t, n_rows * k_dim * 2)
            tl = [K.gemm_tc_tile_weight(t_, silu=epi == K.EPI_SILU_MUL) for t_ in wts]
            t = _time(lambda i: K.gemm_tc(xa, wts[i % C], epilogue=epi, residual=res, out=o, workspace=ws_,
                                          tiled=tl[i % C]), args.reps)
            out[f"tc_tiled_{name}(m={m})"] = (t, n_rows * k_dim * 2)
            del tl
            if epi in (K.EPI_STORE, K.EPI_RESIDUAL) and n_out != g.vocab_size:
                # split-partial form: the GEMM alone, and for the residual
                # linears the pair (GEMM + residual/RMSNorm consumer) against
                # (residual GEMM + RMSNorm)
                part = torch.empty(K.gemm_splits(m, k_dim, n_out) * m * n_out, device=dev)
                t = _time(lambda i: K.gemm_tc_splits(xa, wts[i % C], part), args.reps)
                out[f"tc_split_{name}(m={m})"] = (t, n_rows * k_dim * 2)
                if epi == K.EPI_RESIDUAL:
                    s_ = K.gemm_splits(m, k_dim, n_out)
                    xn_ = torch.empty_like(o)

                    def pair_new(i):
                        K.gemm_tc_splits(xa, wts[i % C], part)
                        K.residual_rmsnorm_splits(part, s_, res, out_residual=o, norm_w=nw[:n_out], eps=1e-6,
                                                  out_norm=xn_)

                    def pair_old(i):
                        K.gemm_tc(xa, wts[i % C], epilogue=epi, residual=res, out=o, workspace=ws_)
                        K.rmsnorm(o, nw[:n_out], 1e-6, out=xn_)
                    out[f"tc_pair_split_{name}+norm(m={m})"] = (_time(pair_new, args.reps), n_rows * k_dim * 2)
                    out[f"tc_pair_reduce_{name}+norm(m={m})"] = (_time(pair_old, args.reps), n_rows * k_dim * 2)
        if "tc_qkv" in tc:
            tc_case("qkv", g.qkv_dim, H, K.EPI_STORE, g.qkv_dim)
        if "tc_oproj" in tc:
            tc_case("oproj", H, g.q_dim, K.EPI_RESIDUAL, H)
        if "tc_gateup" in tc:
            tc_case("gateup", 2 * I, H, K.EPI_SILU_MUL, I)
            # plain [2I, H] linear with whole-K tiles (split-partial form) + the SiLU*up combine
            wts = w((2 * I, H), "mb/gateup")
            xa = synth.normal((m, H), 1.0, 0, "mb/xagateup", device=dev)
            s_ = K.gemm_splits(m, H, 2 * I)
            part = torch.empty(s_ * m * 2 * I, device=dev)
            act = torch.empty(m, I, device=dev, dtype=torch.bfloat16)
            out[f"tc_split_gateup(m={m})"] = (_time(lambda i: K.gemm_tc_splits(xa, wts[i % C], part), args.reps),
                                              2 * I * H * 2)

            def gu_pair(i):
                K.gemm_tc_splits(xa, wts[i % C], part)
                K.silu_mul_splits(part, s_, m, I, out=act)
            out[f"tc_pair_split_gateup+silu(m={m})"] = (_time(gu_pair, args.reps), 2 * I * H * 2)
        if "tc_down" in tc:
            tc_case("down", H, I, K.EPI_RESIDUAL, H)
        if "tc_lmhead" in tc:
            tc_case("lmhead_logits", g.vocab_size, H, K.EPI_STORE, g.vocab_size)
    if "rmsnorm" in wanted:
        xr = synth.normal((m, H), 1.0, 0, "mb/xr", device=dev)
        yr = torch.empty_like(xr)
        t = _time(lambda i: K.rmsnorm(xr, nw, 1e-6, out=yr), args.reps)
        out["rmsnorm"] = (t, 2 * m * H * 2)
    for name, (t, nbytes) in out.items():
        if name.startswith("big_"):
            print(json.dumps({"kernel": name, "m": m, "us": round(t * 1e6, 2), "flops": nbytes,
                              "tflops": round(nbytes / t / 1e12, 1)}))
            continue
        print(json.dumps({"kernel": name, "m": m, "us": round(t * 1e6, 2), "bytes": nbytes,
                          "gbs": round(nbytes / t / 1e9, 1)}))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
