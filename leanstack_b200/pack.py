"""leanpack/v0 writer for in-memory checkpoints.

Writes the on-disk layout the reference's packer produces and its
materializer reads (``src/leanstack/pack.py:226-375``): ``embeddings.
safetensors``, one ``layer-NNN.safetensors`` per layer holding the fused
``attention.qkv_proj`` (q; k; v rows) and ``mlp.gate_up_proj`` (gate; up rows)
plus the norms, o_proj and down_proj, ``output.safetensors`` with the final
norm and lm_head, and a ``manifest.json`` with geometry, hyper-parameters and a
per-tensor index.  The format is kept identical so packs are interchangeable
with the reference's; only the code is new.
"""

from __future__ import annotations

import json
from datetime import datetime, timezone
from pathlib import Path

import torch

from .config import QwenGeometry


def _entries(file_name: str, tensors: dict[str, torch.Tensor], roles: dict[str, str], sources: dict[str, list[str]]):
    out = []
    offset = 0
    for name, t in tensors.items():
        size = t.numel() * t.element_size()
        out.append({"name": name, "file": file_name, "role": roles[name], "dtype": str(t.dtype).replace("torch.", ""),
                    "shape": list(t.shape), "numel": int(t.numel()), "logical_offset_bytes": offset,
                    "size_bytes": size, "source_tensors": sources[name]})
        offset += size
    return out


def write_qwen_leanpack(geometry: QwenGeometry, tensors: dict[str, torch.Tensor], output_dir, *,
                        model_key: str | None = None, overwrite: bool = False) -> dict:
    from safetensors.torch import save_file

    root = Path(output_dir)
    if root.exists() and any(root.iterdir()) and not overwrite:
        raise FileExistsError(f"output_dir already exists: {root}")
    root.mkdir(parents=True, exist_ok=True)
    g = geometry
    files, entries = [], []

    def group(file_name, group_tensors, roles, sources):
        group_tensors = {k: v.detach().to("cpu").contiguous() for k, v in group_tensors.items()}
        save_file(group_tensors, str(root / file_name))
        files.append({"file": file_name, "tensor_count": len(group_tensors),
                      "size_bytes": (root / file_name).stat().st_size})
        entries.extend(_entries(file_name, group_tensors, roles, sources))

    e = "model.embed_tokens.weight"
    group("embeddings.safetensors", {e: tensors[e]}, {e: "embedding"}, {e: [e]})
    for i in range(g.num_hidden_layers):
        p, q = f"model.layers.{i}.", f"layers.{i}."
        qkv_src = [p + "self_attn.q_proj.weight", p + "self_attn.k_proj.weight", p + "self_attn.v_proj.weight"]
        gu_src = [p + "mlp.gate_proj.weight", p + "mlp.up_proj.weight"]
        layer = {
            q + "input_layernorm.weight": (tensors[p + "input_layernorm.weight"], "input_layernorm",
                                           [p + "input_layernorm.weight"]),
            q + "attention.qkv_proj.weight": (torch.cat([tensors[s] for s in qkv_src], 0), "attention_qkv_fused",
                                              qkv_src),
            q + "attention.o_proj.weight": (tensors[p + "self_attn.o_proj.weight"], "attention_output_projection",
                                            [p + "self_attn.o_proj.weight"]),
            q + "attention.q_norm.weight": (tensors[p + "self_attn.q_norm.weight"], "attention_q_norm",
                                            [p + "self_attn.q_norm.weight"]),
            q + "attention.k_norm.weight": (tensors[p + "self_attn.k_norm.weight"], "attention_k_norm",
                                            [p + "self_attn.k_norm.weight"]),
            q + "post_attention_layernorm.weight": (tensors[p + "post_attention_layernorm.weight"],
                                                    "post_attention_layernorm",
                                                    [p + "post_attention_layernorm.weight"]),
            q + "mlp.gate_up_proj.weight": (torch.cat([tensors[s] for s in gu_src], 0), "mlp_gate_up_fused", gu_src),
            q + "mlp.down_proj.weight": (tensors[p + "mlp.down_proj.weight"], "mlp_down_projection",
                                         [p + "mlp.down_proj.weight"]),
        }
        group(f"layer-{i:03d}.safetensors", {k: v[0] for k, v in layer.items()}, {k: v[1] for k, v in layer.items()},
              {k: v[2] for k, v in layer.items()})
    lm_src = "lm_head.weight" if "lm_head.weight" in tensors else "model.embed_tokens.weight"
    group("output.safetensors", {"model.norm.weight": tensors["model.norm.weight"], "lm_head.weight": tensors[lm_src]},
          {"model.norm.weight": "final_norm", "lm_head.weight": "lm_head"},
          {"model.norm.weight": ["model.norm.weight"], "lm_head.weight": [lm_src]})
    manifest = {
        "format_version": "leanpack/v0",
        "created_at_utc": datetime.now(timezone.utc).isoformat(),
        "model_key": model_key or g.key,
        "semantic_model_id": None,
        "source_model_path": "<in-memory>",
        "target_gpu": "B200 / sm_100a",
        "dtype": "bfloat16",
        "geometry": {
            "num_hidden_layers": g.num_hidden_layers, "hidden_size": g.hidden_size,
            "intermediate_size": g.intermediate_size, "num_attention_heads": g.num_attention_heads,
            "num_key_value_heads": g.num_key_value_heads, "head_dim": g.head_dim, "vocab_size": g.vocab_size,
            "max_position_embeddings": g.max_position_embeddings,
        },
        "model_hparams": {"rms_norm_eps": g.rms_norm_eps, "rope_theta": g.rope_theta},
        "exact_prompt_buckets": [], "buckets": [], "speculative_modes": [], "draft_heads": [],
        "required_kernels": [], "backend_policy": [], "files": files, "tensors": entries,
    }
    (root / "manifest.json").write_text(json.dumps(manifest, indent=2) + "\n", encoding="utf-8")
    return manifest


# ---------------------------------------------------------------------------
# leanpack/v1: the B200 serving format
# ---------------------------------------------------------------------------
#
# What v0 does not give (the reference's own list: no physical tiling on disk,
# no direct mmap-style offset loading), v1 adds:
#
#   manifest.json              format "leanpack/v1": geometry, hyper-parameters,
#                              tensor-parallel world, per-tensor index with the
#                              exact byte offset of every tensor in its file
#   rank-RR-of-WW.bin          one flat file per tensor-parallel rank holding
#                              that rank's Megatron shard: QKV rows of its heads,
#                              its re-fused [gate_r; up_r] rows, its column
#                              slices of o_proj / down, the replicated norms and
#                              embedding, and (untied heads only) its vocab rows
#                              of lm_head
#
# Every tensor starts on a 4096-byte boundary, so a loader maps the file and
# takes zero-copy views at the recorded offsets.  A tied head is stored once:
# the lm_head entry is a view (row range) of the embedding, with no bytes of
# its own.  Optionally the packer also stores each linear's pre-tiled tcgen05
# image (the 16 KB shared-memory tiles ls_gemm_tc_tile_weight writes), which
# the engine's tensor-core path streams with plain bulk copies.

V1_FORMAT = "leanpack/v1"
V1_ALIGN = 4096

_LINEARS = (("attention.qkv_proj.weight", False), ("attention.o_proj.weight", False),
            ("mlp.gate_up_proj.weight", True), ("mlp.down_proj.weight", False))


def v1_rank_file(rank: int, world: int) -> str:
    return f"rank-{rank:02d}-of-{world:02d}.bin"


def _serving_layer(local: dict[str, torch.Tensor], i: int) -> list[tuple[str, torch.Tensor, str, list[str]]]:
    """Fused serving tensors of layer ``i`` from Hugging Face-named (possibly sharded) tensors."""
    p, q = f"model.layers.{i}.", f"layers.{i}."
    qkv_src = [p + "self_attn.q_proj.weight", p + "self_attn.k_proj.weight", p + "self_attn.v_proj.weight"]
    gu_src = [p + "mlp.gate_proj.weight", p + "mlp.up_proj.weight"]
    one = lambda s: local[s]  # noqa: E731
    return [
        (q + "input_layernorm.weight", one(p + "input_layernorm.weight"), "input_layernorm",
         [p + "input_layernorm.weight"]),
        (q + "attention.qkv_proj.weight", torch.cat([local[s] for s in qkv_src], 0), "attention_qkv_fused", qkv_src),
        (q + "attention.o_proj.weight", one(p + "self_attn.o_proj.weight"), "attention_output_projection",
         [p + "self_attn.o_proj.weight"]),
        (q + "attention.q_norm.weight", one(p + "self_attn.q_norm.weight"), "attention_q_norm",
         [p + "self_attn.q_norm.weight"]),
        (q + "attention.k_norm.weight", one(p + "self_attn.k_norm.weight"), "attention_k_norm",
         [p + "self_attn.k_norm.weight"]),
        (q + "post_attention_layernorm.weight", one(p + "post_attention_layernorm.weight"),
         "post_attention_layernorm", [p + "post_attention_layernorm.weight"]),
        (q + "mlp.gate_up_proj.weight", torch.cat([local[s] for s in gu_src], 0), "mlp_gate_up_fused", gu_src),
        (q + "mlp.down_proj.weight", one(p + "mlp.down_proj.weight"), "mlp_down_projection",
         [p + "mlp.down_proj.weight"]),
    ]


def write_qwen_leanpack_v1(geometry: QwenGeometry, tensors: dict[str, torch.Tensor], output_dir, *,
                           world: int = 1, tc_tiles: bool = False, model_key: str | None = None,
                           overwrite: bool = False) -> dict:
    """Write a leanpack/v1 artifact with one shard file per tensor-parallel rank.

    ``tensors`` are Hugging Face-named (``model.layers.N.self_attn.q_proj.weight``
    ...), as ``write_qwen_leanpack`` takes them.  ``tc_tiles`` additionally
    stores each linear's tcgen05 tile image; producing it runs the tiling
    kernel, so it needs a CUDA device.
    """
    from .tp import check_divisible, local_geometry, shard_checkpoint, shard_info

    g = geometry
    if world < 1:
        raise ValueError("world must be >= 1")
    check_divisible(g, world)
    root = Path(output_dir)
    if root.exists() and any(root.iterdir()) and not overwrite:
        raise FileExistsError(f"output_dir already exists: {root}")
    root.mkdir(parents=True, exist_ok=True)
    if tc_tiles and not torch.cuda.is_available():
        raise RuntimeError("tc_tiles needs a CUDA device to run the tiling kernel")
    files, entries, ranks = [], [], []
    for r in range(world):
        local = shard_checkpoint(tensors, g, r, world)
        shard = shard_info(g, r, world)
        lg = local_geometry(g, world)
        items: list[tuple[str, torch.Tensor, str, list[str]]] = [
            ("model.embed_tokens.weight", local["model.embed_tokens.weight"], "embedding",
             ["model.embed_tokens.weight"])]
        for i in range(g.num_hidden_layers):
            items += _serving_layer(local, i)
        items.append(("model.norm.weight", local["model.norm.weight"], "final_norm", ["model.norm.weight"]))
        tied = "lm_head.weight" not in local
        if not tied:
            items.append(("lm_head.weight", local["lm_head.weight"], "lm_head", ["lm_head.weight"]))
        extra: dict[str, dict] = {}
        if tc_tiles:
            from . import kernels as K

            layer_items = {name: t for name, t, _, _ in items}
            for i in range(g.num_hidden_layers):
                for base, silu in _LINEARS:
                    name = f"layers.{i}.{base}"
                    w = layer_items[name].to("cuda", torch.bfloat16).contiguous()
                    img = K.gemm_tc_tile_weight(w, silu=silu).cpu()
                    tname = name.removesuffix(".weight") + ".tc_tiled"
                    items.append((tname, img, "tc_tile_image", [name]))
                    extra[tname] = {"layout": "tc_tiled", "tiled_from": name, "silu": silu}
        file_name = v1_rank_file(r, world)
        offset = 0
        with open(root / file_name, "wb") as fh:
            for name, t, role, sources in items:
                t = t.detach().to("cpu").contiguous()
                pad = (-offset) % V1_ALIGN
                if pad:
                    fh.write(b"\0" * pad)
                    offset += pad
                raw = t.view(torch.uint8).reshape(-1).numpy()
                fh.write(raw.tobytes())
                entry = {"name": name, "rank": r, "file": file_name, "role": role,
                         "dtype": str(t.dtype).replace("torch.", ""), "shape": list(t.shape), "layout": "row_major",
                         "offset_bytes": offset, "size_bytes": int(raw.size), "source_tensors": sources}
                entry.update(extra.get(name, {}))
                entries.append(entry)
                offset += int(raw.size)
        if tied:
            entries.append({"name": "lm_head.weight", "rank": r, "file": file_name, "role": "lm_head",
                            "dtype": "bfloat16", "shape": [shard.vocab_rows, g.hidden_size], "layout": "row_major",
                            "view_of": "model.embed_tokens.weight", "row_offset": shard.vocab_offset,
                            "rows": shard.vocab_rows, "offset_bytes": None, "size_bytes": 0,
                            "source_tensors": ["model.embed_tokens.weight"]})
        files.append({"file": file_name, "rank": r, "size_bytes": offset,
                      "tensor_count": sum(1 for e in entries if e["rank"] == r)})
        ranks.append({"rank": r, "vocab_offset": shard.vocab_offset, "vocab_rows": shard.vocab_rows,
                      "local_geometry": {"num_attention_heads": lg.num_attention_heads,
                                         "num_key_value_heads": lg.num_key_value_heads,
                                         "intermediate_size": lg.intermediate_size}})
    manifest = {
        "format_version": V1_FORMAT,
        "created_at_utc": datetime.now(timezone.utc).isoformat(),
        "model_key": model_key or g.key,
        "source_model_path": "<in-memory>",
        "target_gpu": "B200 / sm_100a",
        "dtype": "bfloat16",
        "alignment_bytes": V1_ALIGN,
        "geometry": {
            "num_hidden_layers": g.num_hidden_layers, "hidden_size": g.hidden_size,
            "intermediate_size": g.intermediate_size, "num_attention_heads": g.num_attention_heads,
            "num_key_value_heads": g.num_key_value_heads, "head_dim": g.head_dim, "vocab_size": g.vocab_size,
            "max_position_embeddings": g.max_position_embeddings,
        },
        "model_hparams": {"rms_norm_eps": g.rms_norm_eps, "rope_theta": g.rope_theta},
        "tensor_parallel": {"world": world, "scheme": "megatron: qkv by heads and [gate_r; up_r] column-split, "
                                                        "o_proj / down row-split, embedding and norms replicated, "
                                                        "lm_head vocab-split"},
        "tc_tiles": bool(tc_tiles),
        "ranks": ranks,
        "files": files,
        "tensors": entries,
    }
    (root / "manifest.json").write_text(json.dumps(manifest, indent=2) + "\n", encoding="utf-8")
    return manifest
