"""Pin the CPU oracle against fixtures produced by running the reference itself.

``tests/golden/make_golden.py`` ran the reference's eager semantic runtime on
seeded inputs; here the oracle (``oracle/qwen_oracle.py``) recomputes the same
cases from the same seeds and must agree bit for bit.  The input digests also
pin the synthetic generator, so the GPU tests that regenerate the inputs on the
device see exactly the reference's inputs.
"""

from __future__ import annotations

import torch

from leanstack_b200 import synth
from leanstack_b200.config import QWEN3_4B, TINY, TINY_DRAFT
from oracle import qwen_oracle as qo


def _load(golden_dir, name):
    return torch.load(golden_dir / name, weights_only=False)


def _layer_model(tensors):
    g = QWEN3_4B
    return _one_layer(tensors, "bf16")


def _one_layer(tensors, precision):
    g = QWEN3_4B
    return qo.OracleModel.from_checkpoint(
        g, {**tensors, "model.embed_tokens.weight": torch.zeros(1, g.hidden_size, dtype=torch.bfloat16),
            "model.norm.weight": torch.ones(g.hidden_size, dtype=torch.bfloat16)},
        precision=precision, layer_indices=[0])


def _inputs(tag, batch, past, q_len, seed=0):
    g = QWEN3_4B
    x = synth.normal((batch, q_len, g.hidden_size), 1.0, seed, f"{tag}/x")
    kc = synth.normal((batch, g.num_key_value_heads, past, g.head_dim), 1.0, seed, f"{tag}/k_cache")
    vc = synth.normal((batch, g.num_key_value_heads, past, g.head_dim), 1.0, seed, f"{tag}/v_cache")
    return x, kc, vc


def test_synthetic_inputs_match_reference_run(golden_dir):
    gold = _load(golden_dir, "layer_4b.pt")
    tensors = synth.synth_layer(QWEN3_4B, 0, 0)
    assert {k: synth.tensor_digest(v) for k, v in sorted(tensors.items())} == gold["weights"]
    x, kc, vc = _inputs("cfg1", 1, 512, 1)
    assert gold["cfg1"]["inputs"] == {"k_cache": synth.tensor_digest(kc), "v_cache": synth.tensor_digest(vc),
                                      "x": synth.tensor_digest(x)}


def test_oracle_cfg1_decode_layer_bit_exact(golden_dir):
    gold = _load(golden_dir, "layer_4b.pt")
    g = QWEN3_4B
    tensors = synth.synth_layer(g, 0, 0)
    m = _layer_model(tensors)
    w = m.layers[0]
    c = gold["cfg1"]
    past = c["past"]
    x, kc, vc = _inputs("cfg1", 1, past, 1)
    kv = m.new_kv(1, 1024)
    kv.key_cache[0, :, :, :past] = kc
    kv.value_cache[0, :, :, :past] = vc
    kv.set_all(past)
    cos, sin = m.rope(1024)
    cos, sin = cos[past:past + 1][None], sin[past:past + 1][None]
    xn = qo.rmsnorm(x, w.input_layernorm, g.rms_norm_eps)
    assert torch.equal(xn.reshape(-1), c["xn"])
    q, k, v = qo.qkv_project(xn, w, g.num_attention_heads, g.num_key_value_heads, g.head_dim, cos, sin,
                             g.rms_norm_eps)
    assert torch.equal(q.reshape(-1), c["q"])
    assert torch.equal(k.reshape(-1), c["k"])
    assert torch.equal(v.reshape(-1), c["v"])
    kv.append(0, k, v)
    K, V = kv.get(0)
    attn = qo.attention(q, K, V, None, g.head_dim ** -0.5)
    assert torch.equal(attn.reshape(-1), c["attn"])
    kv.set_all(past)
    y = qo.layer_forward(m, 0, w, x, kv, cos, sin, None)
    assert torch.equal(y.reshape(-1), c["out"])
    # the decode driver's mv form of the same layer
    kv.set_all(past)
    yv = qo.decode_layer_vector(m, 0, w, x, kv, cos, sin)
    assert torch.equal(yv.reshape(-1), c["out"])


def test_stream_paths_record(golden_dir):
    """``stream_4b_paths.json`` (made by ``tests/golden/make_stream_paths.py``
    from the reference itself): the oracle's restatement of the decode driver
    reproduced all 64 teacher-forced tokens of the reference's config-2 stream;
    the reference's own general layer, which differs only in the order of its
    linears' fp32 sums, decided six of them differently (each at a top-2 gap
    of at most 2 bf16 ulps), and one flipped bit in 1e-2 .. 1e-4 of the
    attention outputs flips four to eight (each at a gap of at most 3 ulps)."""
    import json

    gold = _load(golden_dir, "stream_4b.pt")
    paths = json.loads((golden_dir / "stream_4b_paths.json").read_text())
    want = gold["tokens"].tolist()
    assert paths["fixture_tokens"] == want
    assert paths["oracle_vector_path_tokens"] == want
    gen = paths["reference_general_path_tokens"]
    mism = [i for i, (a, b) in enumerate(zip(gen, want)) if a != b]
    assert mism == paths["reference_general_path_mismatches"] == [16, 23, 30, 46, 53, 54]
    margins = gold["margins"].tolist()
    assert all(margins[i] <= 2 * 2 ** -5 for i in mism)
    # the disagreeing token is one of the reference's top two each time
    top5 = gold["top5"]
    assert all(gen[i] in (int(top5[i][1][0]), int(top5[i][1][1])) for i in mism)
    # one ulp of noise in 1e-2 .. 1e-4 of the attention outputs flips only near-tie
    # steps too (top-2 gap at most 3 bf16 ulps at the logits' magnitude, 4 .. 8)
    noise = paths["attention_noise_mismatches"]
    assert set(noise) == {f"{p} {f}" for p in ("vector", "general") for f in ("0.01", "0.001", "0.0001")}
    for f, toks in paths["attention_noise_tokens"].items():
        steps = [i for i, (a, b) in enumerate(zip(toks, want)) if a != b]
        assert steps == noise[f] and 0 < len(steps) <= 10
        assert all(margins[i] <= 3 * 2 ** -5 for i in steps)


def test_oracle_verify_and_prefill_layer_bit_exact(golden_dir):
    gold = _load(golden_dir, "layer_4b.pt")
    g = QWEN3_4B
    m = _layer_model(synth.synth_layer(g, 0, 0))
    for tag in ("verify", "prefill"):
        c = gold[tag]
        b, past, q_len = c["batch"], c["past"], c["q_len"]
        x, kc, vc = _inputs(tag, b, past, q_len)
        kv = m.new_kv(b, 256)
        if past:
            kv.key_cache[0, :, :, :past] = kc
            kv.value_cache[0, :, :, :past] = vc
            kv.set_all(past)
        pc = m.rope(256)
        y = qo.stack_forward(m, x, kv, pc)
        assert torch.equal(y, c["out"]), tag
        K, V = kv.get(0)
        assert torch.equal(K[:, :, past:], c["k_new"]), tag
        assert torch.equal(V[:, :, past:], c["v_new"]), tag


def test_oracle_tiny_stack_greedy_and_speculative(golden_dir):
    gold = _load(golden_dir, "tiny_stack.pt")
    tgt_t = synth.synth_checkpoint(TINY, 3)
    drf_t = synth.synth_checkpoint(TINY_DRAFT, 4)
    assert {k: synth.tensor_digest(v) for k, v in sorted(tgt_t.items())} == gold[f"{TINY.key}_weights"]
    tgt = qo.OracleModel.from_checkpoint(TINY, tgt_t)
    drf = qo.OracleModel.from_checkpoint(TINY_DRAFT, drf_t)
    prompt = gold["greedy"]["prompt"]
    toks, _ = qo.greedy_generate(tgt, prompt, 32, prompt.shape[1] + 32)
    assert toks[0].tolist() == gold["greedy"]["tokens"].tolist()
    for name, draft in (("spec_distinct", drf), ("spec_self", tgt)):
        ids, stats = qo.dual_model_speculative(draft, tgt, prompt, 24, 4)
        assert ids == gold[name]["tokens"].tolist(), name
        assert stats["cycles"] == gold[name]["cycles"], name
        assert stats["accepted"] == gold[name]["accepted"], name
        assert stats["bonus"] == gold[name]["bonus"], name


def test_fp32_oracle_close_to_bf16_reference(golden_dir):
    """The fp32 oracle (tolerance baseline) stays within 2e-2 of the reference's bf16 layer."""
    gold = _load(golden_dir, "layer_4b.pt")
    g = QWEN3_4B
    tensors = synth.synth_layer(g, 0, 0)
    m = _layer_model(tensors)
    m32 = _one_layer(tensors, "fp32")
    c = gold["cfg1"]
    past = c["past"]
    x, kc, vc = _inputs("cfg1", 1, past, 1)
    kv = m32.new_kv(1, 1024)
    kv.key_cache[0, :, :, :past] = kc.float()
    kv.value_cache[0, :, :, :past] = vc.float()
    kv.set_all(past)
    cos, sin = m32.rope(1024)
    y = qo.layer_forward(m32, 0, m32.layers[0], x.float(), kv, cos[past:past + 1][None], sin[past:past + 1][None],
                         None)
    err = (y.reshape(-1) - c["out"].float()).abs().max().item()
    print("bf16 reference vs fp32 oracle, max abs err", err, "max |y|", y.abs().max().item())
    assert err <= 2e-2 * max(1.0, y.abs().max().item()), err
    del m
