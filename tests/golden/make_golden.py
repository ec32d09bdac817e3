"""Generate the golden fixtures by running the reference itself on seeded inputs.

Run in the build container, where the reference source tree is present::

    python tests/golden/make_golden.py --reference-src <reference>/src [--skip-4b]

It imports the reference's eager semantic runtime (``leanstack.runtime.
qwen_explicit``, ``leanstack.runtime.kv_cache``, ``leanstack.pack``,
``leanstack.leanserve`` and the dual-model loop in
``experiments/models/qwen_explicit_runtime_loop.py``) with
``TORCHDYNAMO_DISABLE=1`` and ``LEANSTACK_SEMANTIC_LOGITS_BACKEND=torch``, feeds
it inputs from ``leanstack_b200.synth`` (bit-identical on CPU and GPU) and saves
the outputs, plus digests of every input, as ``tests/golden/*.pt``.  The GPU
box does not have the reference; the tests only read these files.
"""

from __future__ import annotations

import argparse
import importlib.util
import json
import os
import sys
import tempfile
import time
from pathlib import Path

os.environ.setdefault("TORCHDYNAMO_DISABLE", "1")
os.environ.setdefault("LEANSTACK_SEMANTIC_LOGITS_BACKEND", "torch")

import torch  # noqa: E402

REPO = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(REPO))

from leanstack_b200 import synth  # noqa: E402
from leanstack_b200.config import QWEN3_4B, TINY, TINY_DRAFT  # noqa: E402

OUT = Path(__file__).resolve().parent


def _import_reference(src: Path):
    sys.path.insert(0, str(src))
    from leanstack.runtime import qwen_explicit as qe
    from leanstack.runtime import kv_cache as kvc
    from leanstack import leanserve, pack
    from leanstack.config import ModelSpec
    loop_path = src.parent / "experiments" / "models" / "qwen_explicit_runtime_loop.py"
    spec = importlib.util.spec_from_file_location("ref_runtime_loop", loop_path)
    loop = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(loop)
    return qe, kvc, leanserve, pack, ModelSpec, loop


def _serve_config(leanserve, g):
    return leanserve.QwenServeConfig(
        vocab_size=g.vocab_size, hidden_size=g.hidden_size, intermediate_size=g.intermediate_size,
        num_hidden_layers=g.num_hidden_layers, num_attention_heads=g.num_attention_heads,
        num_key_value_heads=g.num_key_value_heads, max_position_embeddings=g.max_position_embeddings,
        head_dim=g.head_dim, rms_norm_eps=g.rms_norm_eps, rope_parameters={"rope_theta": g.rope_theta},
    )


def _ref_layer(qe, g, tensors, layer_idx):
    """Build the reference's QwenSemanticLayerRuntime from HF-named tensors."""
    p = f"model.layers.{layer_idx}."
    t = lambda n: tensors[p + n].contiguous()  # noqa: E731
    q, k, v = t("self_attn.q_proj.weight"), t("self_attn.k_proj.weight"), t("self_attn.v_proj.weight")
    gate, up = t("mlp.gate_proj.weight"), t("mlp.up_proj.weight")
    return qe.QwenSemanticLayerRuntime(
        layer_idx=layer_idx,
        input_layernorm_weight=t("input_layernorm.weight"),
        attention=qe.QwenSemanticAttentionRuntime(
            layer_idx=layer_idx, q_proj_weight=q, k_proj_weight=k, v_proj_weight=v,
            qkv_proj_weight=torch.cat((q, k, v), 0).contiguous(),
            q_proj_out_dim=q.shape[0], k_proj_out_dim=k.shape[0],
            num_attention_heads=g.num_attention_heads, num_key_value_heads=g.num_key_value_heads,
            num_key_value_groups=g.num_key_value_groups, head_dim=g.head_dim,
            attention_scale=g.head_dim ** -0.5, o_proj_weight=t("self_attn.o_proj.weight"),
            q_norm_weight=t("self_attn.q_norm.weight"), k_norm_weight=t("self_attn.k_norm.weight"),
        ),
        post_attention_layernorm_weight=t("post_attention_layernorm.weight"),
        mlp=qe.QwenSemanticMlpRuntime(
            gate_proj_weight=gate, up_proj_weight=up, gate_up_proj_weight=torch.cat((gate, up), 0).contiguous(),
            gate_proj_out_dim=gate.shape[0], down_proj_weight=t("mlp.down_proj.weight"),
        ),
    )


def _inv_freq(g):
    return 1.0 / (g.rope_theta ** (torch.arange(0, g.head_dim, 2, dtype=torch.float32) / g.head_dim))


def _digests(tensors: dict) -> dict:
    return {k: synth.tensor_digest(v) for k, v in sorted(tensors.items())}


def _layer_inputs(g, seed, batch, past, q_len, tag):
    """Seeded hidden input and pre-filled KV for a single-layer case."""
    x = synth.normal((batch, q_len, g.hidden_size), 1.0, seed, f"{tag}/x")
    kc = synth.normal((batch, g.num_key_value_heads, past, g.head_dim), 1.0, seed, f"{tag}/k_cache")
    vc = synth.normal((batch, g.num_key_value_heads, past, g.head_dim), 1.0, seed, f"{tag}/v_cache")
    return x, kc, vc


def gen_layer_cases(qe, kvc, leanserve):
    g = QWEN3_4B
    seed = 0
    tensors = synth.synth_layer(g, 0, seed)
    cfg = _serve_config(leanserve, g)
    layer = _ref_layer(qe, g, tensors, 0)
    eps = g.rms_norm_eps
    out = {"weights": _digests(tensors)}

    # --- cfg1: bs1 decode at position 512 over 512 cached positions (vector path) ---
    past = 512
    x, kc, vc = _layer_inputs(g, seed, 1, past, 1, "cfg1")
    kv = qe.build_qwen_kv_cache(cfg, max_seq_len=1024, device=torch.device("cpu"), dtype=torch.bfloat16,
                                batch_size=1, cache_kind="static")
    kv.key_cache[0, :, :, :past] = kc
    kv.value_cache[0, :, :, :past] = vc
    kv.layer_seq_lens[0] = past
    kv.max_layer_seq_len = past
    pc = qe.build_qwen_position_cache(_inv_freq(g), 1.0, max_seq_len=1024, dtype=torch.bfloat16)
    cos, sin = qe.slice_qwen_position_embeddings(pc, start=past, length=1)
    att = layer.attention
    xv = x.reshape(-1)
    xn = qe.qwen_rmsnorm_vector(xv, layer.input_layernorm_weight, eps)
    q, k, v = qe._semantic_attention_qkv_vector_eager(
        xn, att.qkv_proj_weight, att.q_proj_out_dim, att.k_proj_out_dim, att.num_attention_heads,
        att.num_key_value_heads, att.head_dim, att.q_norm_weight, att.k_norm_weight, cos, sin, eps)
    K, V = kv.append_and_get(0, k, v)
    attn = qe.sdpa_qwen_attention_forward(q, K, V, None, scaling=g.head_dim ** -0.5,
                                          num_key_value_groups=g.num_key_value_groups).reshape(-1)
    o = qe._semantic_decode_attention_output_vector_eager(q, K, V, att.o_proj_weight, att.attention_scale,
                                                          att.num_key_value_groups)
    h = xv + o
    y = qe._semantic_mlp_epilogue_vector_eager(h, layer.post_attention_layernorm_weight,
                                               layer.mlp.gate_up_proj_weight, layer.mlp.gate_proj_out_dim,
                                               layer.mlp.down_proj_weight, eps)
    # the whole-layer entry point must agree with the pieces
    kv.layer_seq_lens[0] = past
    y_full = qe.semantic_qwen_decode_layer_forward(layer, x, kv, (cos, sin), eps).reshape(-1)
    assert torch.equal(y_full, y), "reference decode layer disagrees with its own pieces"
    out["cfg1"] = {
        "inputs": _digests({"x": x, "k_cache": kc, "v_cache": vc}),
        "past": past, "xn": xn, "q": q.reshape(-1), "k": k.reshape(-1), "v": v.reshape(-1),
        "attn": attn, "o_proj": o, "h": h, "out": y,
    }

    # --- verify: B=2, 64 cached, Q=5 with the decode mask (general path) ---
    for tag, batch, past, q_len in (("verify", 2, 64, 5), ("prefill", 2, 0, 16)):
        x, kc, vc = _layer_inputs(g, seed, batch, past, q_len, tag)
        kv = qe.build_qwen_kv_cache(cfg, max_seq_len=256, device=torch.device("cpu"), dtype=torch.bfloat16,
                                    batch_size=batch, cache_kind="static")
        if past:
            kv.key_cache[0, :, :, :past] = kc
            kv.value_cache[0, :, :, :past] = vc
            kv.layer_seq_lens[0] = past
            kv.max_layer_seq_len = past
        pc = qe.build_qwen_position_cache(_inv_freq(g), 1.0, max_seq_len=256, dtype=torch.bfloat16)
        pos = qe.slice_qwen_position_embeddings(pc, start=past, length=q_len)
        mask = qe.build_decode_attention_mask(q_len, past + q_len, torch.device("cpu"), torch.bfloat16) if past else None
        y = qe.semantic_qwen_layer_forward(config=cfg, layer=layer, rope_inv_freq=_inv_freq(g), attention_scaling=1.0,
                                           hidden_states=x, position_ids=None, attention_mask=mask, kv_cache=kv,
                                           position_embeddings=pos)
        Kn, Vn = kv.get(0)
        out[tag] = {
            "inputs": _digests({"x": x, "k_cache": kc, "v_cache": vc}),
            "batch": batch, "past": past, "q_len": q_len, "out": y,
            "k_new": Kn[:, :, past:].contiguous(), "v_new": Vn[:, :, past:].contiguous(),
        }
    return out


class _StubTokenizer:
    def decode(self, ids, skip_special_tokens=True):
        return " ".join(str(int(i)) for i in (ids.tolist() if hasattr(ids, "tolist") else ids))


def _write_hf_checkpoint(g, tensors, root: Path):
    from safetensors.torch import save_file
    root.mkdir(parents=True, exist_ok=True)
    save_file({k: v.contiguous() for k, v in tensors.items()}, str(root / "model.safetensors"))
    cfg = {
        "architectures": ["Qwen3ForCausalLM"], "model_type": "qwen3", "vocab_size": g.vocab_size,
        "hidden_size": g.hidden_size, "intermediate_size": g.intermediate_size,
        "num_hidden_layers": g.num_hidden_layers, "num_attention_heads": g.num_attention_heads,
        "num_key_value_heads": g.num_key_value_heads, "head_dim": g.head_dim,
        "max_position_embeddings": g.max_position_embeddings, "rms_norm_eps": g.rms_norm_eps,
        "rope_theta": g.rope_theta, "tie_word_embeddings": True, "torch_dtype": "bfloat16",
        "hidden_act": "silu", "attention_bias": False,
    }
    (root / "config.json").write_text(json.dumps(cfg), encoding="utf-8")


def _model_spec(ModelSpec, g):
    return ModelSpec(
        key=g.key, family="Qwen-family", loader_hint="synthetic", dtype="bfloat16", kv_layout="static",
        required_kernels=(), semantic_model_id=None, num_hidden_layers=g.num_hidden_layers,
        hidden_size=g.hidden_size, intermediate_size=g.intermediate_size,
        num_attention_heads=g.num_attention_heads, num_key_value_heads=g.num_key_value_heads,
        head_dim=g.head_dim, vocab_size=g.vocab_size, max_position_embeddings=g.max_position_embeddings,
    )


def gen_tiny(qe, leanserve, pack, ModelSpec, loop):
    """Tiny stacks through the reference's own pack -> materialize -> decode path."""
    out = {}
    runtimes = {}
    with tempfile.TemporaryDirectory() as tmp:
        for g, seed in ((TINY, 3), (TINY_DRAFT, 4)):
            tensors = synth.synth_checkpoint(g, seed)
            ckpt, pdir = Path(tmp) / f"{g.key}-hf", Path(tmp) / f"{g.key}-pack"
            _write_hf_checkpoint(g, tensors, ckpt)
            pack.build_qwen_leanpack(model=_model_spec(ModelSpec, g), model_path=ckpt, output_dir=pdir)
            rt = leanserve.materialize_qwen_full_semantic_runtime_from_leanpack(pdir, device="cpu", dtype="bfloat16")
            runtimes[g.key] = rt
            out[f"{g.key}_weights"] = _digests(tensors)

        tgt = runtimes[TINY.key]
        prompt = synth.token_ids((1, 24), TINY.vocab_size, 3, "tiny/prompt")
        new = 32
        max_seq = prompt.shape[1] + new
        pc = qe.build_qwen_position_cache(tgt.rope_inv_freq, 1.0, max_seq_len=max_seq, dtype=torch.bfloat16)
        with torch.inference_mode():
            hidden, cache = qe.run_semantic_stack_prefill(tgt, prompt, max_seq_len=max_seq, position_cache=pc)
            prefill_last = hidden[0, -1].clone()
            tok = qe.select_semantic_greedy_token(tgt, hidden)
            toks = [int(tok)]
            for _ in range(new - 1):
                hidden, cache = qe.run_semantic_stack_decode(tgt, tok, cache, position_cache=pc)
                tok = qe.select_semantic_greedy_token(tgt, hidden)
                toks.append(int(tok))
        out["greedy"] = {"prompt": prompt, "tokens": torch.tensor(toks), "prefill_last_hidden": prefill_last}

        spec = {}
        for name, draft_key in (("spec_distinct", TINY_DRAFT.key), ("spec_self", TINY.key)):
            res = loop.run_dual_model_speculative_request(
                draft_runtime=runtimes[draft_key], verifier_runtime=tgt, tokenizer=_StubTokenizer(),
                input_ids=prompt, device=torch.device("cpu"), page_size=16, max_new_tokens=24,
                proposal_len=4, stop_token_ids=())
            s = res["speculative_summary"]
            spec[name] = {"tokens": torch.tensor(res["generated_token_ids"]), "cycles": s["cycles"],
                          "accepted": s["accepted_proposal_tokens"], "proposed": s["proposed_tokens"],
                          "bonus": s["bonus_tokens"]}
        out.update(spec)
    return out


def gen_4b_stream(qe, leanserve, steps: int):
    """cfg2: full random-init Qwen3-4B, 512 uniform prompt ids, greedy stream."""
    g = QWEN3_4B
    seed = 1
    t0 = time.time()
    tensors = synth.synth_checkpoint(g, seed)
    print(f"  synthesized 4B weights in {time.time() - t0:.1f}s", flush=True)
    cfg = _serve_config(leanserve, g)
    layers = tuple(_ref_layer(qe, g, tensors, i) for i in range(g.num_hidden_layers))
    embed = tensors["model.embed_tokens.weight"]
    rt = qe.QwenSemanticStackRuntime(
        model_path=Path("synthetic"), config=cfg, layer_indices=tuple(range(g.num_hidden_layers)),
        embed_tokens_weight=embed, layers=layers, rope_inv_freq=_inv_freq(g), attention_scaling=1.0,
        final_norm_weight=tensors["model.norm.weight"], lm_head_weight=embed, device=torch.device("cpu"),
        dtype=torch.bfloat16)
    prompt = synth.token_ids((1, 512), g.vocab_size, seed, "cfg2/prompt")
    max_seq = 4096
    pc = qe.build_qwen_position_cache(rt.rope_inv_freq, 1.0, max_seq_len=max_seq, dtype=torch.bfloat16)
    toks, margins, top5 = [], [], []

    def head(hidden):
        logits = qe._semantic_greedy_head_vector_eager  # noqa: F841 (documents which head)
        last = qe.last_hidden_vector(hidden)
        n = qe.qwen_rmsnorm_vector(last, rt.final_norm_weight, cfg.rms_norm_eps)
        lg = torch.mv(rt.lm_head_weight, n)
        tk = qe.select_semantic_greedy_token(rt, hidden)
        assert int(tk) == int(lg.argmax()), "torch head disagrees with mv+argmax"
        v, i = lg.float().topk(5)
        margins.append(float(v[0] - v[1]))
        top5.append(torch.stack([v, i.float()]))
        return tk

    with torch.inference_mode():
        t0 = time.time()
        hidden, cache = qe.run_semantic_stack_prefill(rt, prompt, max_seq_len=max_seq, position_cache=pc)
        print(f"  prefill 512 in {time.time() - t0:.1f}s", flush=True)
        prefill_last = hidden[0, -1].clone()
        tok = head(hidden)
        toks.append(int(tok))
        t0 = time.time()
        for _ in range(steps - 1):
            hidden, cache = qe.run_semantic_stack_decode(rt, tok, cache, position_cache=pc)
            tok = head(hidden)
            toks.append(int(tok))
        print(f"  {steps - 1} decode steps in {time.time() - t0:.1f}s", flush=True)
    return {"prompt": prompt, "tokens": torch.tensor(toks), "margins": torch.tensor(margins),
            "top5": torch.stack(top5), "prefill_last_hidden": prefill_last,
            "weights_sample": _digests({k: tensors[k] for k in ("model.embed_tokens.weight",
                                                                "model.layers.0.self_attn.q_proj.weight",
                                                                "model.layers.35.mlp.down_proj.weight",
                                                                "model.norm.weight")})}


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference-src", required=True)
    ap.add_argument("--skip-4b", action="store_true")
    ap.add_argument("--steps", type=int, default=64)
    args = ap.parse_args()
    torch.set_num_threads(os.cpu_count())
    qe, kvc, leanserve, pack, ModelSpec, loop = _import_reference(Path(args.reference_src))
    meta = {"torch": torch.__version__, "generated_by": "tests/golden/make_golden.py"}
    t0 = time.time()
    layer = gen_layer_cases(qe, kvc, leanserve)
    torch.save({"meta": meta, **layer}, OUT / "layer_4b.pt")
    print(f"layer cases done in {time.time() - t0:.1f}s", flush=True)
    t0 = time.time()
    tiny = gen_tiny(qe, leanserve, pack, ModelSpec, loop)
    torch.save({"meta": meta, **tiny}, OUT / "tiny_stack.pt")
    print(f"tiny cases done in {time.time() - t0:.1f}s", flush=True)
    if not args.skip_4b:
        t0 = time.time()
        stream = gen_4b_stream(qe, leanserve, args.steps)
        torch.save({"meta": meta, **stream}, OUT / "stream_4b.pt")
        print(f"4B stream done in {time.time() - t0:.1f}s", flush=True)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
