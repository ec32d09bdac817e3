#!/usr/bin/env python
"""Benchmark: Qwen3-4B BF16 greedy decode tok/s on B200.

Workload: random-init Qwen3-4B (36 layers, 2560 hidden, tied 151936 vocab,
seeded synthetic weights), batch 1, 512 uniform-random prompt ids (seed 1),
static KV cache of 4096 positions.  One step = one greedy decode token: the
whole 36-layer stack + final norm + lm_head + argmax, replayed as one CUDA
graph.  Each step streams 8.05 GB of weights (> 126 MB L2), so no L2 flush is
needed between steps.

Arms:
* default: the native path (libleanb200.so).  ``value`` = tokens / device time
  (CUDA events, max over ranks); ``e2e`` = the same through the public engine
  API with the step's input token copied from pinned host memory and the
  result read back every step; ``roofline`` = the dominant kernel (fused
  post-norm + gate_up + SiLU*up) timed with CUDA events; ``cpu_baseline`` = the
  CPU oracle (the reference's eager torch path restated) on this host's cores.
* ``--impl reference``: the reference's CPU implementation of the path (the
  oracle port; the reference cannot travel to the GPU box) timed alone.

Multi-GPU (torchrun, N > 1): Megatron tensor parallelism over the N GPUs
(``--parallel tp``, the default; ``scaling: strong``): column-split QKV and
gate_up, row-split o_proj and down_proj with an NCCL all-reduce of their fp32
partials, a vocab-split greedy head with a MAX all-reduce of argmax keys.  The
same bs1 sequence is decoded by all ranks; ``value`` is its tok/s.
``--parallel replicas`` runs N independent bs1 replicas instead (weak scaling).
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import torch

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))

from leanstack_b200 import synth  # noqa: E402
from leanstack_b200.config import QWEN3_4B  # noqa: E402

METRIC = "Qwen3-4B BF16 greedy decode tok/s (bs1, 512-token prompt, static KV 4096)"
WORKLOAD = "cfg2: Qwen3-4B random-init, batch 1, 512 uniform prompt ids, greedy decode"
SEED = 1
PROMPT = 512
MAX_SEQ = 4096


def parse_args():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=256)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-sample-seconds", type=float, default=12.0)
    ap.add_argument("--e2e-steps", type=int, default=64)
    ap.add_argument("--linear-backend", choices=("auto", "tc", "cuda_core"), default="auto",
                    help="tensor-core (tcgen05) or CUDA-core streaming linears for the decode step")
    ap.add_argument("--parallel", choices=("tp", "replicas"), default="tp",
                    help="with N > 1 GPUs: tensor parallelism (one sequence) or independent replicas")
    ap.add_argument("--batched", default="8,32,64",
                    help="comma-separated batch sizes of the config-3 batched-decode section ('' to skip)")
    ap.add_argument("--batched-cached", type=int, default=2048, help="cached positions per sequence (config 3)")
    ap.add_argument("--batched-steps", type=int, default=128)
    ap.add_argument("--no-verify", action="store_true", help="skip the config-4 speculative-verify section")
    ap.add_argument("--no-prefill", action="store_true", help="skip the config-5 prefill section")
    ap.add_argument("--prefill-batch", type=int, default=16)
    ap.add_argument("--prefill-len", type=int, default=4096)
    ap.add_argument("--allreduce", choices=("fused", "nccl"), default="fused",
                    help="tensor parallelism: fused one-shot P2P all-reduce in the CUDA-core linears, or NCCL")
    return ap.parse_args()


def measured_peaks() -> dict:
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": float(d["hbm_gbs"]), "bf16_tflops": float(d["bf16_tflops"]),
                "bf16_tflops_sustained": float(d.get("bf16_tflops_sustained", d["bf16_tflops"])), "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


class ClockSampler:
    """nvidia-smi clock / throttle sampling during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.path = None

    def start(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100", "-f", self.path], stdout=subprocess.DEVNULL, stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        time.sleep(0.3)

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.2)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        rows = []
        for line in Path(self.path).read_text().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 9:
                rows.append(parts)
        os.unlink(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


# ---------------------------------------------------------------------------
# distributed plumbing
# ---------------------------------------------------------------------------

def dist_setup(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch.distributed as dist

        if args.impl == "ours":
            torch.cuda.set_device(local)
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300))
        else:
            dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=900))
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def max_over_ranks(value: float, world: int) -> float:
    if world == 1:
        return value
    import torch.distributed as dist

    t = torch.tensor([value], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ---------------------------------------------------------------------------
# CPU oracle (reference path restated) — the timed CPU baseline
# ---------------------------------------------------------------------------

def cpu_info(threads: int) -> dict:
    """Host CPU model, the bf16 matrix/vector extensions it offers, and the threads used."""
    model, flags = "unknown", set()
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name") and model == "unknown":
                model = line.split(":", 1)[1].strip()
            elif line.startswith("flags") and not flags:
                flags = set(line.split(":", 1)[1].split())
    except OSError:
        pass
    wanted = ("amx_bf16", "amx_tile", "avx512_bf16", "avx512f")
    return {"model": model, "bf16_flags": [f for f in wanted if f in flags], "threads": threads,
            "logical_cpus": os.cpu_count()}


def cpu_decode_rate(tensors_cpu: dict, budget_s: float, min_steps: int = 1, warmup: int = 3):
    """Time full-model bs1 decode steps of the CPU oracle (bf16, all host cores).

    One model and KV cache serve the warm-up and the timed sample, and the
    sample runs until both ``min_steps`` steps and ``budget_s`` seconds are done,
    so every caller times the same steady state.  The KV cache holds 512
    seeded positions (a prefill on the CPU would take minutes and is not part of
    the timed metric).  Returns (tok/s, steps, threads, seconds).
    """
    from oracle import qwen_oracle as qo

    torch.set_num_threads(os.cpu_count() or 1)
    g = QWEN3_4B
    m = qo.OracleModel.from_checkpoint(g, tensors_cpu, precision="bf16")
    kv = m.new_kv(1, MAX_SEQ)
    kv.key_cache[:, :, :, :PROMPT] = synth.normal((g.num_hidden_layers, 1, g.num_key_value_heads, PROMPT, g.head_dim),
                                                  1.0, SEED, "bench/cpu_k")
    kv.value_cache[:, :, :, :PROMPT] = synth.normal((g.num_hidden_layers, 1, g.num_key_value_heads, PROMPT,
                                                     g.head_dim), 1.0, SEED, "bench/cpu_v")
    kv.set_all(PROMPT)
    pc = m.rope(MAX_SEQ)
    tok = torch.tensor([[1]])
    with torch.inference_mode():
        for _ in range(max(1, warmup)):
            hidden = qo.stack_forward(m, qo.embed(m, tok), kv, pc)
            tok = qo.greedy_token(m, hidden).view(1, 1)
        steps = 0
        t0 = time.perf_counter()
        while True:
            hidden = qo.stack_forward(m, qo.embed(m, tok), kv, pc)
            tok = qo.greedy_token(m, hidden).view(1, 1)
            steps += 1
            el = time.perf_counter() - t0
            if steps >= min_steps and el >= budget_s:
                break
    return steps / el, steps, torch.get_num_threads(), el


def cpu_sample_text(steps: int, el: float) -> str:
    return (f"{steps} full-model bs1 decode steps ({el:.1f} s, after 3 warm-up steps) over a 512-position KV "
            f"cache: CPU oracle (the reference's eager torch path restated), bf16")


def bench_config() -> dict:
    """The workload description both arms print (identical dicts)."""
    return {"workload": WORKLOAD, "model": "Qwen3-4B (random init)", "global_batch": 1, "seq_len": PROMPT,
            "max_seq": MAX_SEQ, "l2": "not flushed: each step streams 8.05 GB of weights (> 126 MB L2)"}


def cpu_checkpoint():
    """Synthesize the 4B checkpoint (on the GPU when present: same values) and bring it to the host."""
    dev = "cuda" if torch.cuda.is_available() else "cpu"
    t = synth.synth_checkpoint(QWEN3_4B, SEED, device=dev)
    return {k: v.to("cpu") for k, v in t.items()}


def run_reference(args, world, rank):
    if rank != 0:
        barrier(world)
        return 0
    tensors = cpu_checkpoint()
    torch.cuda.empty_cache() if torch.cuda.is_available() else None
    # the same steady-state sample as the native arm's cpu_baseline: W warm-up
    # steps, then at least K steps and at least --cpu-sample-seconds
    rate, steps, threads, el = cpu_decode_rate(tensors, args.cpu_sample_seconds, min_steps=args.steps,
                                               warmup=max(3, args.warmup))
    line = {
        "impl": "reference", "metric": METRIC, "value": rate, "unit": "tok/s", "n_gpus": args.gpus,
        "steps": steps, "warmup": args.warmup, "ms_per_step": 1000.0 * el / steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded random-init weights, uniform ids)",
        "config": bench_config(),
        "cpu_baseline": {"value": rate, "unit": "tok/s", "cores": threads, "kind": "port",
                         "sample": cpu_sample_text(steps, el), "cpu": cpu_info(threads)},
        "e2e": {"value": rate, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    barrier(world)
    return 0


# ---------------------------------------------------------------------------
# native arm
# ---------------------------------------------------------------------------

def _timed(fn, steps: int, warmup: int, world: int) -> float:
    """Seconds for ``steps`` calls of ``fn`` after ``warmup`` (CUDA events, max over ranks)."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    barrier(world)
    stream = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        fn()
    e1.record(stream)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    barrier(world)
    return max_over_ranks(ms, world) / 1000.0


def run_layer_linears(rt, eng, peaks) -> dict:
    """BASELINE config 1's per-linear figures: each decode linear at M = 1 (the
    engine's CUDA-core kernels with their fused prologues / epilogues), timed
    with CUDA events over a CUDA graph of launches that walk the 36 resident
    layers, so every launch streams its own weights from HBM and no host
    launch cost sits between them.  GB/s = (weight + input + output bytes) / time."""
    from leanstack_b200 import kernels as K

    g = QWEN3_4B
    a = eng.arenas
    H, I, Q = g.hidden_size, eng.g.intermediate_size, eng.g.q_dim
    qkv_out = torch.empty(1, eng.g.qkv_dim, device=rt.device, dtype=torch.bfloat16)
    attn = torch.zeros(1, Q, device=rt.device, dtype=torch.bfloat16)
    ws = torch.zeros(K.lmhead_workspace_bytes(1, eng.vocab_rows), device=rt.device, dtype=torch.uint8)
    ids = torch.empty(1, device=rt.device, dtype=torch.int64)
    cases = {
        "qkv (input norm + QKV)": (lambda L: K.linear(a.h[:1], L.attention.qkv_proj_weight,
                                                      norm_w=L.input_layernorm_weight, eps=g.rms_norm_eps,
                                                      out=qkv_out),
                                   eng.g.qkv_dim * H * 2 + H * 2 + eng.g.qkv_dim * 2, len(rt.layers)),
        "o_proj + residual": (lambda L: K.oproj_residual(attn, L.attention.o_proj_weight, a.h[:1], out=a.x[:1]),
                              H * Q * 2 + Q * 2 + 2 * H * 2, len(rt.layers)),
        "gate_up + SiLU*up (post norm)": (lambda L: K.gateup_silu(a.h[:1], L.post_attention_layernorm_weight,
                                                                   L.mlp.gate_up_proj_weight, g.rms_norm_eps,
                                                                   out=a.act[:1]),
                                          2 * I * H * 2 + H * 2 + I * 2, len(rt.layers)),
        "down + residual": (lambda L: K.down_residual(a.act[:1], L.mlp.down_proj_weight, a.h[:1], out=a.x[:1]),
                            H * I * 2 + I * 2 + 2 * H * 2, len(rt.layers)),
        "lm_head + argmax (final norm)": (lambda L: K.lmhead_argmax(a.h[:1], rt.final_norm_weight, rt.lm_head_weight,
                                                                     g.rms_norm_eps, out_ids=ids, workspace=ws),
                                          eng.vocab_rows * H * 2 + H * 2 + 8, 1),
    }
    out = {}
    for name, (fn, nbytes, n_layers) in cases.items():
        # launches over n_layers distinct layers captured in one CUDA graph, as
        # in the decode step: no host launch cost between them
        laps = 1 if n_layers > 1 else 8
        for L in rt.layers[:2]:
            fn(L)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.graph(graph, stream=side):
            for _ in range(laps):
                for L in rt.layers[:n_layers]:
                    fn(L)
        torch.cuda.current_stream().wait_stream(side)
        graph.replay()
        torch.cuda.synchronize()
        reps = 4
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            graph.replay()
        e1.record()
        torch.cuda.synchronize()
        del graph
        per = e0.elapsed_time(e1) / 1000.0 / (reps * laps * n_layers)
        out[name] = {"us": per * 1e6, "bytes": nbytes, "gbs": nbytes / per / 1e9,
                     "hbm_frac": nbytes / per / 1e9 / peaks["hbm_gbs"]}
    return out


def run_batched(rt, comm, shard, batch: int, cached: int, steps: int, warmup: int, world: int, peaks) -> dict:
    """``batch`` sequences with ``cached`` prompt positions each, greedy decode."""
    from leanstack_b200.engine import DecodeEngine

    g = QWEN3_4B
    eng = DecodeEngine(rt, batch_size=batch, max_seq_len=cached + warmup + steps + 8, tp=comm, shard=shard)
    eng.prefill(synth.token_ids((batch, cached), g.vocab_size, SEED, f"cfg3/prompt{batch}"))
    eng.capture()
    t = _timed(eng.decode_step, steps, warmup, world)
    gl = eng.g
    kv_bytes = batch * (cached + warmup + steps // 2) * gl.kv_bytes_per_token()
    step_bytes = g.num_hidden_layers * gl.layer_weight_bytes() + eng.vocab_rows * g.hidden_size * 2 + kv_bytes
    out = {"batch": batch, "cached_per_seq": cached, "steps": steps, "tok_per_s": batch * steps / t,
           "ms_per_step": 1000.0 * t / steps, "linear_backend": eng.backend,
           "step_bytes_per_gpu": step_bytes, "step_frac_of_hbm": step_bytes / (t / steps) / 1e9 / peaks["hbm_gbs"],
           "kv_share_of_bytes": kv_bytes / step_bytes}
    eng.graph = None
    del eng
    torch.cuda.empty_cache()
    return out


def run_prefill(rt, comm, shard, batch: int, plen: int, decode_steps: int, world: int, peaks) -> dict:
    """one-pass prefill of ``batch`` x ``plen`` uniform prompt ids (M = batch * plen
    large-M tcgen05 GEMMs), then ``decode_steps`` greedy steps at that batch."""
    from leanstack_b200.engine import DecodeEngine

    g = QWEN3_4B
    eng = DecodeEngine(rt, batch_size=batch, max_seq_len=plen + decode_steps + 16, linear_backend="tc", tp=comm,
                       shard=shard)
    eng.prefill_full(synth.token_ids((batch, 128), g.vocab_size, SEED, "cfg5/warm"))  # warm-up pass
    torch.cuda.synchronize()
    eng.reset()
    prompt = synth.token_ids((batch, plen), g.vocab_size, SEED, "cfg5/prompt")
    barrier(world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    eng.prefill_full(prompt)
    e1.record()
    torch.cuda.synchronize()
    t = max_over_ranks(e0.elapsed_time(e1) / 1000.0, world)
    eng.capture()
    td = _timed(eng.decode_step, decode_steps, 2, world)
    gl = eng.g
    lin_params = gl.qkv_dim * g.hidden_size + g.hidden_size * gl.q_dim + 2 * gl.intermediate_size * g.hidden_size + \
        g.hidden_size * gl.intermediate_size
    flops = 2.0 * batch * plen * lin_params * g.num_hidden_layers * world  # whole job (all ranks)
    out = {"batch": batch, "prompt_len": plen, "m": batch * plen, "prefill_s": t,
           "prefill_tok_per_s": batch * plen / t, "linear_tflops": flops / t / 1e12,
           "linear_tensor_frac_per_gpu": flops / world / t / 1e12 / peaks["bf16_tflops_sustained"],
           "tensor_peak": "bf16_tflops_sustained (a prefill pass runs for most of a second)",
           "decode_steps": decode_steps, "decode_tok_per_s": batch * decode_steps / td,
           "attention": "causal prefill attention on tcgen05 (prefill_attention_tc_kernel: S and O in TMEM)"}
    eng.graph = None
    del eng
    torch.cuda.empty_cache()
    return out


def run_verify(rt, comm, shard, steps: int, warmup: int, world: int, peaks) -> dict:
    """target verify at batch 16, k = 4 uniform proposals, 1024 cached (M = 80)."""
    from leanstack_b200 import kernels as K
    from leanstack_b200.engine import DecodeEngine

    g = QWEN3_4B
    B, k, cached = 16, 4, 1024
    eng = DecodeEngine(rt, batch_size=B, max_seq_len=cached + (warmup + steps + 2) * (k + 1) + 8,
                       linear_backend="tc", tp=comm, shard=shard)
    eng.prefill(synth.token_ids((B, cached), g.vocab_size, SEED, "cfg4/prompt"))
    props = synth.token_ids((warmup + steps + 1, B, k), g.vocab_size, SEED, "cfg4/proposals").to(rt.device)
    inp = eng.verify_inputs(k)
    it = iter(range(props.shape[0]))

    def step():
        inp[:, 1:].copy_(props[next(it)])
        eng.verify_step(k)

    step()  # capture
    pos0 = None
    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    pos0 = eng.kv.cache_pos.clone()
    t = _timed(step, steps, 0, world)
    committed = int((eng.kv.cache_pos - pos0).sum().item())
    eng.sync_cursors()
    # the dominant verify GEMM alone: gate_up + SiLU*up at M = 80 on tcgen05
    gl = eng.g
    m = B * (k + 1)
    layer = rt.layers[0]
    xs = eng.xn[:m]
    reps = 8
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)

    def gate_up(w):  # what the verify step runs: whole-K linear + SiLU*up combine, or the paired GEMM
        if eng.gu_plain:
            s_ = K.gemm_tc_splits(xs, w, eng.tc_part)
            K.silu_mul_splits(eng.tc_part, s_, m, gl.intermediate_size, out=eng.arenas.act[:m])
        else:
            K.gemm_tc(xs, w, epilogue=K.EPI_SILU_MUL, out=eng.arenas.act[:m], workspace=eng.tc_ws)
    gate_up(layer.mlp.gate_up_proj_weight)
    torch.cuda.synchronize()
    e0.record()
    for i in range(reps):
        for lay in rt.layers:
            gate_up(lay.mlp.gate_up_proj_weight)
    e1.record()
    torch.cuda.synchronize()
    per = e0.elapsed_time(e1) / 1000.0 / (reps * len(rt.layers))
    w_bytes = 2 * gl.intermediate_size * g.hidden_size * 2
    flops = 2.0 * m * 2 * gl.intermediate_size * g.hidden_size
    out = {"batch": B, "proposal_len": k, "m": m, "cached_per_seq": cached, "steps": steps,
           "verify_steps_per_s": steps / t, "ms_per_verify": 1000.0 * t / steps,
           "positions_per_s": steps * m / t, "committed_tok_per_s": committed / t,
           "proposals": "uniform random ids (accept rate ~0)",
           "dominant_gemm": {"kernel": ("gemm_tc_kernel<SPLIT_F32> whole-K gate_up + silu_mul_splits (M=80)"
                                        if eng.gu_plain else "gemm_tc_kernel<SILU_MUL> (gate_up + SiLU*up, M=80)"),
                             "us": per * 1e6,
                             "gbs": w_bytes / per / 1e9, "hbm_frac": w_bytes / per / 1e9 / peaks["hbm_gbs"],
                             "tflops": flops / per / 1e12,
                             "tensor_frac": flops / per / 1e12 / peaks.get("bf16_tflops", 1663.3),
                             "hbm_bound_tensor_frac": (peaks["hbm_gbs"] * 1e9 * flops / w_bytes) / 1e12
                             / peaks.get("bf16_tflops", 1663.3)}}
    for gph in eng.verify_graphs.values():
        del gph
    eng.verify_graphs.clear()
    del eng
    torch.cuda.empty_cache()
    return out

def run_draft_cycle(rt, steps: int, warmup: int, world: int, peaks) -> dict:
    """BASELINE config 4 with the draft model in the loop: a random-init
    Qwen3-0.6B-geometry draft (28 layers, hidden 1024, 16 / 8 heads,
    intermediate 3072) decoding 16 sequences over 1024 cached positions, and
    whole speculative cycles (k = 4 draft steps, one M = 80 target verify, the
    device accept; one CUDA-graph replay per cycle)."""
    from leanstack_b200.config import QWEN3_06B_DRAFT
    from leanstack_b200.engine import DecodeEngine
    from leanstack_b200.leanserve import materialize_from_tensors
    from leanstack_b200.speculative import SpeculativeDecoder

    gd = QWEN3_06B_DRAFT
    B, k, cached = 16, 4, 1024
    rt_d = materialize_from_tensors(gd, synth.synth_checkpoint(gd, SEED, device=rt.device), device=rt.device,
                                    free_source=True)
    S = cached + (warmup + steps + 2) * (k + 1) + 16
    prompt = synth.token_ids((B, cached), gd.vocab_size, SEED, "cfg4d/prompt")
    # the draft alone: bs16 greedy decode
    drf = DecodeEngine(rt_d, batch_size=B, max_seq_len=S, linear_backend="tc")
    drf.prefill_full(prompt)
    drf.capture()
    td = _timed(drf.decode_step, steps, warmup, world)
    draft_bytes = gd.num_hidden_layers * gd.layer_weight_bytes() + gd.lm_head_bytes() + \
        B * (cached + warmup + steps // 2) * gd.kv_bytes_per_token()
    out = {"draft": "Qwen3-0.6B geometry (random init)", "batch": B, "cached_per_seq": cached,
           "draft_decode_tok_per_s": B * steps / td, "draft_ms_per_step": 1000.0 * td / steps,
           "draft_step_frac_of_hbm": draft_bytes / (td / steps) / 1e9 / peaks["hbm_gbs"]}
    drf.graph = None
    del drf
    # whole cycles: draft proposes k, target verifies k + 1, device accept
    tgt = DecodeEngine(rt, batch_size=B, max_seq_len=S, linear_backend="tc")
    drf = DecodeEngine(rt_d, batch_size=B, max_seq_len=S, linear_backend="tc")
    spec = SpeculativeDecoder(drf, tgt, k, (warmup + steps + 2) * (k + 1))
    first = tgt.prefill_full(prompt)
    drf.prefill_full(prompt)
    tgt.next_ids.copy_(first)
    spec.out_len.zero_()
    tc = _timed(spec.cycle, steps, warmup, world)
    committed = int(spec.out_len.sum().item())
    spec.sync_cursors()
    out.update({"proposal_len": k, "cycles": steps, "ms_per_cycle": 1000.0 * tc / steps,
                "cycles_per_s": steps / tc,
                "committed_tok_per_s_incl_warmup_cycles": committed / (tc * (steps + warmup) / steps),
                "accepted_per_cycle": committed / (B * (steps + warmup)) - 1.0,
                "proposals": "the draft's greedy tokens (two unrelated random-init models: acceptance ~0)"})
    spec.graphs.clear()
    for g_ in tgt.verify_graphs.values():
        del g_
    tgt.verify_graphs.clear()
    del spec, tgt, drf, rt_d
    torch.cuda.empty_cache()
    return out


def run_ours(args, world, rank, local):
    from leanstack_b200 import kernels as K
    from leanstack_b200 import tp as tpm
    from leanstack_b200.engine import DecodeEngine
    from leanstack_b200.leanserve import materialize_from_tensors

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    g = QWEN3_4B
    peaks = measured_peaks()
    tp_mode = world > 1 and args.parallel == "tp"
    tensors = synth.synth_checkpoint(g, SEED, device=dev)
    if tp_mode:
        rt, shard = tpm.materialize_tp_shard(g, tensors, rank, world, device=dev)
        comm = tpm.TPComm(rank, world)
        if args.allreduce == "fused":
            comm.enable_p2p(g.hidden_size)
    else:
        rt = materialize_from_tensors(g, tensors, device=dev, free_source=True)
        shard = comm = None
    del tensors
    torch.cuda.empty_cache()
    prompt = synth.token_ids((1, PROMPT), g.vocab_size, SEED, "cfg2/prompt")
    eng = DecodeEngine(rt, batch_size=1, max_seq_len=MAX_SEQ, linear_backend=args.linear_backend, tp=comm,
                       shard=shard)
    eng.prefill(prompt)
    eng.capture()
    total_steps = args.warmup + args.steps + args.e2e_steps + 2
    if PROMPT + total_steps > eng.S:
        raise SystemExit(f"--warmup + --steps + --e2e-steps exceed the {MAX_SEQ}-position cache")

    for _ in range(args.warmup):
        eng.decode_step()
    torch.cuda.synchronize()
    barrier(world)
    clocks = ClockSampler(local)
    clocks.start()
    stream = torch.cuda.current_stream()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    ev0.record(stream)
    for _ in range(args.steps):
        eng.decode_step()
    ev1.record(stream)
    torch.cuda.synchronize()
    clk = clocks.stop()
    elapsed_ms = ev0.elapsed_time(ev1)
    barrier(world)
    elapsed_ms = max_over_ranks(elapsed_ms, world)
    ms_per_step = elapsed_ms / args.steps
    seqs = 1 if tp_mode else world  # sequences decoded by the whole job
    value = seqs * args.steps * eng.B / (elapsed_ms / 1000.0)

    # --- e2e through the public API: host ids in, host ids out, every step ---
    pin_in = torch.empty((1,), dtype=torch.int64, pin_memory=True)
    pin_out = torch.empty((1,), dtype=torch.int64, pin_memory=True)
    pin_out.copy_(eng.current_ids.cpu())
    torch.cuda.synchronize()
    barrier(world)
    t0 = time.perf_counter()
    for _ in range(args.e2e_steps):
        pin_in.copy_(pin_out)
        eng.current_ids.copy_(pin_in, non_blocking=True)
        eng.decode_step()
        pin_out.copy_(eng.current_ids, non_blocking=True)
        stream.synchronize()
    e2e_s = time.perf_counter() - t0
    e2e_s = max_over_ranks(e2e_s, world)
    e2e = {"value": seqs * args.e2e_steps / e2e_s, "unit": "tok/s", "h2d_bytes_per_step": 8,
           "d2h_bytes_per_step": 8, "steps": args.e2e_steps}

    # --- roofline of the dominant kernel: gate_up + SiLU*up (with its norm on the CUDA-core path) ---
    a = eng.arenas
    reps = 4
    ev2, ev3 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if eng.backend == "tc":
        kernel_name = "gemm_tc_kernel<SILU_MUL> (tcgen05 gate_up + SiLU*up, M=1)"
        xn = eng.xn[:1]

        def dominant(layer):
            K.gemm_tc(xn, layer.mlp.gate_up_proj_weight, epilogue=K.EPI_SILU_MUL, out=a.act[:1], workspace=eng.tc_ws)
    else:
        kernel_name = "linear_small_m<1,SILU_MUL,norm> (post-norm + gate_up + SiLU*up, M=1)"

        def dominant(layer):
            K.gateup_silu(a.h[:1], layer.post_attention_layernorm_weight, layer.mlp.gate_up_proj_weight,
                          g.rms_norm_eps, out=a.act[:1])
    ev2.record(stream)
    for _ in range(reps):
        for layer in rt.layers:
            dominant(layer)
    ev3.record(stream)
    torch.cuda.synchronize()
    per_launch_s = ev2.elapsed_time(ev3) / 1000.0 / (reps * len(rt.layers))
    gl = eng.g  # this rank's geometry (intermediate split under tensor parallelism)
    gu_bytes = 2 * gl.intermediate_size * g.hidden_size * 2 + g.hidden_size * 2 * 2 + gl.intermediate_size * 2
    achieved = gu_bytes / per_launch_s / 1e9
    traffic = None
    tp = REPO / "profiles" / "traffic.json"
    if tp.exists() and not tp_mode:
        traffic = json.loads(tp.read_text()).get("gateup_silu_per_launch_bytes")
    # per-GPU step bytes: this rank's weight shard, vocab shard of the head and KV heads
    step_bytes = g.num_hidden_layers * gl.layer_weight_bytes() + eng.vocab_rows * g.hidden_size * 2 + \
        (PROMPT + args.warmup + args.steps // 2) * gl.kv_bytes_per_token()
    roofline = {"kernel": kernel_name, "bound": "hbm",
                "achieved": achieved, "peak": peaks["hbm_gbs"], "unit": "GB/s", "frac": achieved / peaks["hbm_gbs"],
                "traffic": traffic, "algorithmic_bytes_per_launch": gu_bytes,
                "avg_launch_us": per_launch_s * 1e6, "peak_source": f"{peaks['source']} (MEASURED_PEAKS.json copy)",
                "step_achieved_gbs": step_bytes / (ms_per_step / 1000.0) / 1e9,
                "step_frac": step_bytes / (ms_per_step / 1000.0) / 1e9 / peaks["hbm_gbs"],
                "step_bytes": step_bytes}

    # --- config 3 (batched decode) and config 4 (speculative verify) sections ---
    extra = {}
    if not tp_mode and eng.backend != "tc":
        extra["cfg1_linears_m1"] = run_layer_linears(rt, eng, peaks)
    for bs in [int(x) for x in args.batched.split(",") if x.strip()]:
        extra[f"bs{bs}"] = run_batched(rt, comm, shard, bs, args.batched_cached, args.batched_steps, 4, world,
                                       peaks)
    if not args.no_verify:
        extra["verify_cfg4"] = run_verify(rt, comm, shard, 64, 4, world, peaks)
        if not tp_mode:
            extra["draft_cycle_cfg4"] = run_draft_cycle(rt, 64, 4, world, peaks)
    if not args.no_prefill:
        extra["prefill_cfg5"] = run_prefill(rt, comm, shard, args.prefill_batch, args.prefill_len, 64, world, peaks)

    # --- CPU baseline (rank 0, N == 1 only) ---
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        tensors_cpu = cpu_checkpoint()
        rate, steps, threads, el = cpu_decode_rate(tensors_cpu, args.cpu_sample_seconds)
        del tensors_cpu
        cpu = {"value": rate, "unit": "tok/s", "cores": threads, "kind": "port",
               "sample": cpu_sample_text(steps, el), "cpu": cpu_info(threads)}

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True,
            "scaling": "strong" if tp_mode else "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded random-init weights, uniform ids)",
            "config": {**bench_config(), "global_batch": seqs},
            "parallelism": (f"tp{world}" + ("" if args.allreduce == "nccl" else " fused-allreduce")
                            if tp_mode else f"replicas x{world}") if world > 1 else "single GPU",
            "linear_backend": eng.backend,
            "e2e": e2e, "roofline": roofline, "cpu_baseline": cpu, "clocks": clk,
            "gpu_launches": args.steps * eng.kernel_launches_per_step(),
        }
        if tp_mode:
            line["collectives_per_step"] = eng.collectives_per_step()
        line.update(extra)
        print(json.dumps(line), flush=True)
    barrier(world)
    eng.graph = None  # release the graph (it holds NCCL work) before the process group goes
    torch.cuda.synchronize()
    if comm is not None:
        comm.close()
    return 0


def main() -> int:
    args = parse_args()
    world, rank, local = dist_setup(args)
    try:
        if args.impl == "reference":
            return run_reference(args, world, rank)
        return run_ours(args, world, rank, local)
    finally:
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()


if __name__ == "__main__":
    sys.exit(main())
