"""Measure how far the reference's own code paths agree on the config-2 stream.

Run in the build container, where the reference source tree is present::

    python tests/golden/make_stream_paths.py --reference-src <reference>/src

``stream_4b.pt`` holds the first 64 greedy tokens of random-init Qwen3-4B as
the reference's decode driver produces them on the CPU: ``run_semantic_stack_decode``,
whose layers are the bs1 vector forms (``torch.mv`` linears,
``src/leanstack/runtime/qwen_explicit.py:1247-1272``).  The reference also owns
a general layer, ``semantic_qwen_layer_forward`` (``:1211-1244``), the one its
prefill and verify drivers run, with the same rounding points but
``F.linear`` in place of ``torch.mv``.  On the CPU the two reach different bf16
GEMV kernels whose fp32 sums run in a different order.

This script replays the fixture's prompt and, teacher-forced, its 64 tokens
through (a) the reference's general layer, (b) the oracle's restatement of
the vector path, and (c) the oracle's restatements of both paths with one ulp
of noise: in every attention output, a seeded random fraction f (1e-2, 1e-3,
1e-4) of the bf16 elements get their last mantissa bit flipped.  It stores the tokens each
predicts in ``stream_4b_paths.json``.  (b) must equal the fixture (it pins the
oracle on the whole stream); (a) shows which steps the reference's own
arithmetic decides differently when only the summation order of its linears
changes; (c) measures how many of the stream's near-tie steps one ulp of noise
in one attention output in ten thousand is enough to flip.
"""

from __future__ import annotations

import argparse
import json
import os
import platform
import sys
import time
from pathlib import Path

os.environ.setdefault("TORCHDYNAMO_DISABLE", "1")
os.environ.setdefault("LEANSTACK_SEMANTIC_LOGITS_BACKEND", "torch")

import torch  # noqa: E402

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]
sys.path.insert(0, str(REPO))
sys.path.insert(0, str(HERE))

import make_golden as mg  # noqa: E402
from leanstack_b200 import synth  # noqa: E402
from leanstack_b200.config import QWEN3_4B  # noqa: E402
from oracle import qwen_oracle as qo  # noqa: E402


def _cpu_model() -> str:
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return platform.processor()


def reference_general_path(qe, leanserve, tensors, gold) -> list[int]:
    g = QWEN3_4B
    cfg = mg._serve_config(leanserve, g)
    layers = tuple(mg._ref_layer(qe, g, tensors, i) for i in range(g.num_hidden_layers))
    embed = tensors["model.embed_tokens.weight"]
    rt = qe.QwenSemanticStackRuntime(
        model_path=Path("synthetic"), config=cfg, layer_indices=tuple(range(g.num_hidden_layers)),
        embed_tokens_weight=embed, layers=layers, rope_inv_freq=mg._inv_freq(g), attention_scaling=1.0,
        final_norm_weight=tensors["model.norm.weight"], lm_head_weight=embed, device=torch.device("cpu"),
        dtype=torch.bfloat16)
    max_seq = 4096
    pc = qe.build_qwen_position_cache(rt.rope_inv_freq, 1.0, max_seq_len=max_seq, dtype=torch.bfloat16)
    want = gold["tokens"].tolist()
    with torch.inference_mode():
        hidden, cache = qe.run_semantic_stack_prefill(rt, gold["prompt"], max_seq_len=max_seq, position_cache=pc)
        got = [int(qe.select_semantic_greedy_token(rt, hidden))]
        for step in range(1, len(want)):
            past = cache.get_seq_length()
            pe = qe.slice_qwen_position_embeddings(pc, start=past, length=1)
            hidden = torch.nn.functional.embedding(torch.tensor([[want[step - 1]]]), rt.embed_tokens_weight)
            for layer in rt.layers:
                hidden = qe.semantic_qwen_layer_forward(
                    config=rt.config, layer=layer, rope_inv_freq=rt.rope_inv_freq,
                    attention_scaling=rt.attention_scaling, hidden_states=hidden, position_ids=None,
                    attention_mask=None, kv_cache=cache, position_embeddings=pe)
            got.append(int(qe.select_semantic_greedy_token(rt, hidden)))
    return got


def perturbed_sdpa(fraction: float):
    """``sdpa`` whose bf16 output has the last mantissa bit flipped in a seeded
    random ``fraction`` of its elements (one ulp, sign kept)."""
    exact = qo.sdpa

    def run(*args, **kwargs):
        out = exact(*args, **kwargs)
        gen = torch.Generator().manual_seed(out.numel())
        flip = torch.rand(out.shape, generator=gen) < fraction
        bits = out.contiguous().view(torch.int16)
        return torch.where(flip, bits ^ 1, bits).view(torch.bfloat16)

    return run


def oracle_path(tensors, gold, vector: bool = True, noise: float = 0.0) -> list[int]:
    """Teacher-forced stream of the oracle: the decode driver's vector form
    (``vector``) or the general layer with the torch head (``F.linear``)."""
    if noise:
        saved, qo.sdpa = qo.sdpa, perturbed_sdpa(noise)
        try:
            return oracle_path(tensors, gold, vector)
        finally:
            qo.sdpa = saved
    m = qo.OracleModel.from_checkpoint(QWEN3_4B, tensors)
    kv, pc = m.new_kv(1, 4096), m.rope(4096)
    want = gold["tokens"].tolist()

    def head(h):
        return int(qo.greedy_logits_vector(m, h).argmax()) if vector else int(qo.greedy_token(m, h)[0])

    with torch.inference_mode():
        hidden = qo.stack_forward(m, qo.embed(m, gold["prompt"]), kv, pc)
        got = [head(hidden)]
        for step in range(1, len(want)):
            ids = torch.tensor([[want[step - 1]]])
            hidden = qo.decode_step_vector(m, ids, kv, pc) if vector else qo.stack_forward(m, qo.embed(m, ids), kv, pc)
            got.append(head(hidden))
    return got


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference-src", required=True)
    args = ap.parse_args()
    torch.set_num_threads(os.cpu_count())
    qe, _kvc, leanserve, _pack, _spec, _loop = mg._import_reference(Path(args.reference_src))
    gold = torch.load(HERE / "stream_4b.pt", weights_only=False)
    t0 = time.time()
    tensors = synth.synth_checkpoint(QWEN3_4B, 1)
    for k, v in gold["weights_sample"].items():
        assert synth.tensor_digest(tensors[k]) == v, k
    print(f"weights in {time.time() - t0:.1f}s", flush=True)
    want = gold["tokens"].tolist()
    t0 = time.time()
    general = reference_general_path(qe, leanserve, tensors, gold)
    print(f"reference general path in {time.time() - t0:.1f}s", flush=True)
    t0 = time.time()
    vector = oracle_path(tensors, gold)
    print(f"oracle vector path in {time.time() - t0:.1f}s", flush=True)
    noisy = {}
    for path in ("vector", "general"):
        for f in (1e-2, 1e-3, 1e-4):
            t0 = time.time()
            noisy[f"{path} {f:g}"] = oracle_path(tensors, gold, vector=path == "vector", noise=f)
            print(f"oracle {path} path with 1-ulp noise in {f:g} of attention outputs in {time.time() - t0:.1f}s",
                  flush=True)

    def mismatches(tokens):
        return [i for i, (a, b) in enumerate(zip(tokens, want)) if a != b]

    mism = mismatches(general)
    out = {
        "meta": {"torch": torch.__version__, "cpu": _cpu_model(), "threads": torch.get_num_threads(),
                 "generated_by": "tests/golden/make_stream_paths.py", "teacher_forced": True},
        "fixture_tokens": want,
        "reference_general_path_tokens": general,
        "reference_general_path_mismatches": mism,
        "oracle_vector_path_tokens": vector,
        "oracle_vector_path_mismatches": mismatches(vector),
        "attention_noise_tokens": noisy,
        "attention_noise_mismatches": {k: mismatches(v) for k, v in noisy.items()},
    }
    (HERE / "stream_4b_paths.json").write_text(json.dumps(out, indent=1) + "\n")
    print(json.dumps({k: v for k, v in out.items() if "mismatches" in k or k == "meta"}))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
