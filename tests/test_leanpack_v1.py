"""leanpack/v1 (per-rank shard files, offset-mapped loading, one copy of a tied
head) on the CPU: the writer's layout and the mapped runtime against the
in-memory materializers it replaces."""

from __future__ import annotations

import json

import pytest
import torch

from leanstack_b200 import synth
from leanstack_b200 import tp as tpm
from leanstack_b200.config import TINY
from leanstack_b200.leanserve import map_leanpack_v1_rank, materialize_from_leanpack_v1, materialize_from_tensors
from leanstack_b200.pack import V1_ALIGN, v1_rank_file, write_qwen_leanpack, write_qwen_leanpack_v1


def _runtime_tensors(rt) -> dict[str, torch.Tensor]:
    out = {"embed": rt.embed_tokens_weight, "final_norm": rt.final_norm_weight, "lm_head": rt.lm_head_weight}
    for i, layer in enumerate(rt.layers):
        att, mlp = layer.attention, layer.mlp
        out.update({f"{i}.in": layer.input_layernorm_weight, f"{i}.post": layer.post_attention_layernorm_weight,
                    f"{i}.qkv": att.qkv_proj_weight, f"{i}.o": att.o_proj_weight, f"{i}.qn": att.q_norm_weight,
                    f"{i}.kn": att.k_norm_weight, f"{i}.gu": mlp.gate_up_proj_weight, f"{i}.down": mlp.down_proj_weight,
                    f"{i}.q": att.q_proj_weight, f"{i}.gate": mlp.gate_proj_weight})
    return out


def _assert_same_runtime(a, b):
    ta, tb = _runtime_tensors(a), _runtime_tensors(b)
    assert ta.keys() == tb.keys()
    for k in ta:
        assert ta[k].shape == tb[k].shape, k
        assert torch.equal(ta[k], tb[k]), k
    assert (a.config.num_attention_heads, a.config.num_key_value_heads, a.config.intermediate_size) == \
        (b.config.num_attention_heads, b.config.num_key_value_heads, b.config.intermediate_size)


def test_v1_single_rank_layout_and_roundtrip(tmp_path):
    tensors = synth.synth_checkpoint(TINY, 5)
    m = write_qwen_leanpack_v1(TINY, tensors, tmp_path / "pack")
    assert m["format_version"] == "leanpack/v1" and m["tensor_parallel"]["world"] == 1
    assert [f["file"] for f in m["files"]] == [v1_rank_file(0, 1)]
    on_disk = json.loads((tmp_path / "pack" / "manifest.json").read_text())
    assert on_disk["tensors"] == m["tensors"]
    stored = [e for e in m["tensors"] if not e.get("view_of")]
    # every tensor on a 4096-byte boundary, extents disjoint and in order
    ends = 0
    for e in stored:
        assert e["offset_bytes"] % V1_ALIGN == 0 and e["offset_bytes"] >= ends
        ends = e["offset_bytes"] + e["size_bytes"]
    assert m["files"][0]["size_bytes"] == ends == (tmp_path / "pack" / v1_rank_file(0, 1)).stat().st_size
    # a tied head is stored once: its entry is a row range of the embedding
    head = next(e for e in m["tensors"] if e["name"] == "lm_head.weight")
    assert head["view_of"] == "model.embed_tokens.weight" and head["size_bytes"] == 0
    assert (head["row_offset"], head["rows"]) == (0, TINY.vocab_size)
    payload = sum(e["size_bytes"] for e in stored)
    assert payload == sum(t.numel() * 2 for t in tensors.values())  # each source byte once, nothing more
    # mapped views are zero-copy and equal the fused serving tensors
    _, views = map_leanpack_v1_rank(tmp_path / "pack", 0)
    base = {v.untyped_storage().data_ptr() for v in views.values()}
    assert len(base) == 1
    want_qkv = torch.cat([tensors[f"model.layers.1.self_attn.{n}_proj.weight"] for n in "qkv"], 0)
    assert torch.equal(views["layers.1.attention.qkv_proj.weight"], want_qkv)
    want_gu = torch.cat([tensors["model.layers.0.mlp.gate_proj.weight"], tensors["model.layers.0.mlp.up_proj.weight"]])
    assert torch.equal(views["layers.0.mlp.gate_up_proj.weight"], want_gu)
    rt, shard, tiles = materialize_from_leanpack_v1(tmp_path / "pack", device="cpu")
    assert tiles is None and (shard.rank, shard.world, shard.vocab_offset) == (0, 1, 0)
    _assert_same_runtime(rt, materialize_from_tensors(TINY, dict(tensors), device="cpu"))
    assert rt.lm_head_weight.data_ptr() == rt.embed_tokens_weight.data_ptr()  # the tied head is a view


@pytest.mark.parametrize("tied", [True, False])
def test_v1_tensor_parallel_shards_match_materialize_tp_shard(tmp_path, tied):
    tensors = synth.synth_checkpoint(TINY, 6)
    if not tied:
        tensors["lm_head.weight"] = synth.normal((TINY.vocab_size, TINY.hidden_size), 0.02, 6, "lm_head")
    world = 2
    m = write_qwen_leanpack_v1(TINY, tensors, tmp_path / "pack", world=world)
    assert [f["file"] for f in m["files"]] == [v1_rank_file(r, world) for r in range(world)]
    for r in range(world):
        rt, shard, _ = materialize_from_leanpack_v1(tmp_path / "pack", rank=r, device="cpu")
        ref, ref_shard = tpm.materialize_tp_shard(TINY, dict(tensors), r, world, device="cpu")
        assert shard == ref_shard
        _assert_same_runtime(rt, ref)
        head = next(e for e in m["tensors"] if e["name"] == "lm_head.weight" and e["rank"] == r)
        assert bool(head.get("view_of")) == tied
        if not tied:
            assert head["shape"] == [TINY.vocab_size // world, TINY.hidden_size]


def test_v1_rejects_bad_artifacts(tmp_path):
    tensors = synth.synth_checkpoint(TINY, 7)
    write_qwen_leanpack(TINY, tensors, tmp_path / "v0")
    with pytest.raises(ValueError, match="not a leanpack/v1"):
        map_leanpack_v1_rank(tmp_path / "v0")
    write_qwen_leanpack_v1(TINY, tensors, tmp_path / "v1", world=2)
    with pytest.raises(ValueError, match="outside"):
        map_leanpack_v1_rank(tmp_path / "v1", rank=2)
    with open(tmp_path / "v1" / v1_rank_file(1, 2), "ab") as fh:  # a truncated or appended file is refused
        fh.write(b"\0" * 16)
    with pytest.raises(ValueError, match="bytes on disk"):
        map_leanpack_v1_rank(tmp_path / "v1", rank=1)
    with pytest.raises(FileExistsError):
        write_qwen_leanpack_v1(TINY, tensors, tmp_path / "v1")
    with pytest.raises(ValueError):
        write_qwen_leanpack_v1(TINY, tensors, tmp_path / "v3", world=3)  # 2 kv heads do not split 3 ways
