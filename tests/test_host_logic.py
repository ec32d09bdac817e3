"""Host-side logic on the CPU: KV cursor protocol, buffer planning, the
synthetic generator, geometry constants and leanpack read/write."""

from __future__ import annotations

import pytest
import torch

from leanstack_b200 import synth
from leanstack_b200.config import QWEN3_06B_DRAFT, QWEN3_4B, TINY
from leanstack_b200.kv_cache import KVPageLayout, StaticKVBlockManager
from leanstack_b200.leanserve import build_resident_buffer_plan, load_leanpack_artifact


def _kv(batch=2, layers=3, max_seq=32):
    layout = KVPageLayout(num_layers=layers, num_key_value_heads=2, head_dim=128, page_size=16, max_seq_len=max_seq,
                          batch_size=batch, dtype=torch.bfloat16, device=torch.device("cpu"))
    return StaticKVBlockManager(layout)


def test_geometry_matches_reference_registry():
    # src/leanstack/model_registry.py:6-93 and tests/test_active_contract.py:11-21
    g = QWEN3_4B
    assert (g.num_hidden_layers, g.hidden_size, g.intermediate_size) == (36, 2560, 9728)
    assert (g.num_attention_heads, g.num_key_value_heads, g.head_dim, g.vocab_size) == (32, 8, 128, 151936)
    # tests/test_hot_kernel_cases.py:17-28: projection shapes (K, N)
    assert (g.hidden_size, g.q_dim) == (2560, 4096)
    assert (g.hidden_size, g.kv_dim) == (2560, 1024)
    assert (g.q_dim, g.hidden_size) == (4096, 2560)
    assert (g.hidden_size, g.intermediate_size) == (2560, 9728)
    assert (g.intermediate_size, g.hidden_size) == (9728, 2560)
    assert g.kv_bytes_per_token() == 147456
    assert abs(g.num_hidden_layers * g.layer_weight_bytes() / 1e9 - 7.267) < 0.01
    assert abs(g.lm_head_bytes() / 1e9 - 0.778) < 0.001
    d = QWEN3_06B_DRAFT
    assert (d.num_hidden_layers, d.hidden_size, d.intermediate_size, d.q_dim) == (28, 1024, 3072, 2048)


def test_kv_cursor_protocol_matches_reference():
    kv = _kv()
    k = torch.randn(2, 2, 3, 128).bfloat16()
    kv.append(0, k, k)
    assert kv.get_layer_seq_length(0) == 3 and kv.get_seq_length() == 3
    K_, V_ = kv.get(0)
    assert K_.shape == (2, 2, 3, 128) and torch.equal(K_, k)
    snap = kv.snapshot_cursor()
    kv.append(0, k, k)
    assert kv.get_layer_seq_length(0) == 6
    kv.restore_cursor(kv.cursor_after_tokens(snap, 1))
    assert kv.layer_seq_lens[0] == 4 and kv.max_layer_seq_len == 4
    assert kv.page_table(0) == (0,)
    assert kv.summary()["cache_kind"] == "static"
    with pytest.raises(ValueError, match="token_count must be non-negative"):
        kv.cursor_after_tokens(snap, -1)


def test_kv_overflow_and_shape_errors():
    kv = _kv(max_seq=4)
    k = torch.zeros(2, 2, 3, 128, dtype=torch.bfloat16)
    kv.append(1, k, k)
    with pytest.raises(ValueError, match="cache overflow"):
        kv.append(1, k, k)
    with pytest.raises(ValueError, match="batch_size"):
        kv.append(0, torch.zeros(1, 2, 1, 128, dtype=torch.bfloat16), torch.zeros(1, 2, 1, 128, dtype=torch.bfloat16))
    with pytest.raises(ValueError, match="same shape"):
        kv.append(0, k, k[:, :, :2])


def test_per_sequence_cursors():
    kv = _kv(batch=3)
    kv.set_sequence_lens([5, 7, 6])
    assert kv.cache_pos.tolist() == [5, 7, 6]
    assert kv.get_seq_length() == 7
    kv.note_advanced(2)
    assert kv.sequence_lens == [7, 9, 8]
    with pytest.raises(ValueError):
        kv.set_sequence_lens([1, 2])
    with pytest.raises(ValueError):
        kv.set_sequence_lens([0, 0, 99])


def test_buffer_plan_bytes():
    plan = build_resident_buffer_plan(QWEN3_4B, weights_bytes=8_045_000_000, batch_size=1, max_seq_len=4096,
                                      max_tokens_per_step=8)
    assert plan.kv_cache_bytes == 4096 * 147456
    assert plan.scratch.tokens == 8
    assert plan.resident_bytes > plan.weights_bytes + plan.kv_cache_bytes
    plan = build_resident_buffer_plan(QWEN3_4B, weights_bytes=0, batch_size=32, max_seq_len=2177, max_tokens_per_step=32)
    assert plan.max_seq_len == 2192  # rounded up to the 16-token page


def test_synth_is_deterministic_and_distributed():
    a = synth.normal((4096,), 0.02, 5, "w")
    b = synth.normal((4096,), 0.02, 5, "w")
    c = synth.normal((4096,), 0.02, 6, "w")
    assert torch.equal(a, b) and not torch.equal(a, c)
    big = synth.normal((1 << 20,), 1.0, 0, "x").float()
    assert abs(big.mean().item()) < 0.01 and abs(big.std().item() - 1.0) < 0.01
    n = synth.norm_weight((1 << 16,), 0, "n").float()
    assert abs(n.mean().item() - 1.0) < 1e-3 and abs(n.std().item() - 0.01) < 1e-3
    ids = synth.token_ids((10000,), 151936, 1, "ids")
    assert ids.min() >= 0 and ids.max() < 151936 and ids.unique().numel() > 9000


def test_leanpack_roundtrip(tmp_path):
    from leanstack_b200.pack import write_qwen_leanpack

    tensors = synth.synth_checkpoint(TINY, 3)
    write_qwen_leanpack(TINY, tensors, tmp_path / "pack")
    art = load_leanpack_artifact(tmp_path / "pack")
    g = art.geometry()
    assert (g.hidden_size, g.num_hidden_layers, g.intermediate_size) == (512, 2, 1536)
    assert art.lm_head_is_tied()
    got = art.load("layer-001.safetensors", ("layers.1.attention.qkv_proj.weight",), "cpu", torch.bfloat16)
    want = torch.cat([tensors[f"model.layers.1.self_attn.{n}_proj.weight"] for n in "qkv"], 0)
    assert torch.equal(got["layers.1.attention.qkv_proj.weight"], want)
