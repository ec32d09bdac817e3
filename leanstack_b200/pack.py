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
