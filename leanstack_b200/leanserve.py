"""Materializer and resident buffer planner (the reference's ``leanserve.py``).

* ``materialize_qwen_full_semantic_runtime_from_leanpack`` /
  ``materialize_qwen_semantic_stack_from_leanpack`` keep the reference's
  signatures (``src/leanstack/leanserve.py:470-548``) and return a
  ``QwenSemanticStackRuntime`` with the same fields, read from a leanpack/v0
  directory (``manifest.json`` + ``embeddings`` / ``layer-NNN`` / ``output``
  safetensors, ``src/leanstack/pack.py:226-375``).  A tied lm_head is kept
  resident once (the reference loads it twice, ``leanserve.py:509-517``).
* ``materialize_from_tensors`` builds the same runtime from Hugging Face-named
  tensors already in memory (the synthetic checkpoints of the benchmarks).
* ``ResidentBufferPlan`` is no longer descriptive only (reference
  ``leanserve.py:331-377``): ``allocate_arenas`` hands out the KV and
  activation arenas that the engine and the kernels write into.
"""

from __future__ import annotations

import json
from dataclasses import dataclass, field
from pathlib import Path

import torch

from .config import QwenGeometry
from .kv_cache import KVPageLayout, StaticKVBlockManager
from .qwen_explicit import (QwenSemanticAttentionRuntime, QwenSemanticLayerRuntime, QwenSemanticMlpRuntime,
                            QwenSemanticStackRuntime)


def resolve_torch_dtype(name) -> torch.dtype:
    if isinstance(name, torch.dtype):
        return name
    table = {"bfloat16": torch.bfloat16, "float16": torch.float16, "float32": torch.float32}
    if name not in table:
        raise ValueError(f"unsupported dtype: {name}")
    return table[name]


def rope_inv_freq(geometry: QwenGeometry, device) -> torch.Tensor:
    """``1 / theta^(arange(0, D, 2) / D)`` in fp32 (``leanserve.py:492-496``)."""
    d = geometry.head_dim
    return 1.0 / (geometry.rope_theta ** (torch.arange(0, d, 2, device=device, dtype=torch.float32) / d))


def _layer_runtime(g: QwenGeometry, layer_idx: int, t: dict[str, torch.Tensor]) -> QwenSemanticLayerRuntime:
    qkv = t["qkv"]
    gate_up = t["gate_up"]
    q_w, k_w, v_w = torch.split(qkv, (g.q_dim, g.kv_dim, g.kv_dim), dim=0)
    gate_w, up_w = torch.split(gate_up, (g.intermediate_size, g.intermediate_size), dim=0)
    return QwenSemanticLayerRuntime(
        layer_idx=layer_idx,
        input_layernorm_weight=t["input_layernorm"],
        attention=QwenSemanticAttentionRuntime(
            layer_idx=layer_idx, q_proj_weight=q_w, k_proj_weight=k_w, v_proj_weight=v_w, qkv_proj_weight=qkv,
            q_proj_out_dim=g.q_dim, k_proj_out_dim=g.kv_dim, num_attention_heads=g.num_attention_heads,
            num_key_value_heads=g.num_key_value_heads, num_key_value_groups=g.num_key_value_groups,
            head_dim=g.head_dim, attention_scale=g.head_dim ** -0.5, o_proj_weight=t["o_proj"],
            q_norm_weight=t["q_norm"], k_norm_weight=t["k_norm"]),
        post_attention_layernorm_weight=t["post_attention_layernorm"],
        mlp=QwenSemanticMlpRuntime(gate_proj_weight=gate_w, up_proj_weight=up_w, gate_up_proj_weight=gate_up,
                                   gate_proj_out_dim=g.intermediate_size, down_proj_weight=t["down_proj"]),
    )


def materialize_from_tensors(geometry: QwenGeometry, tensors: dict[str, torch.Tensor], device="cuda:0",
                             dtype="bfloat16", layer_indices=None, include_output_head: bool = True,
                             free_source: bool = False) -> QwenSemanticStackRuntime:
    """Build the runtime from Hugging Face-named tensors (fusing qkv and gate_up as leanpack does)."""
    dev = torch.device(device)
    dt = resolve_torch_dtype(dtype)
    g = geometry
    idx = tuple(range(g.num_hidden_layers)) if layer_indices is None else tuple(layer_indices)
    layers = []
    for i in idx:
        p = f"model.layers.{i}."
        get = (tensors.pop if free_source else tensors.__getitem__)
        q, k, v = get(p + "self_attn.q_proj.weight"), get(p + "self_attn.k_proj.weight"), get(p + "self_attn.v_proj.weight")
        gate, up = get(p + "mlp.gate_proj.weight"), get(p + "mlp.up_proj.weight")
        t = {
            "qkv": torch.cat((q, k, v), 0).to(dev, dt).contiguous(),
            "gate_up": torch.cat((gate, up), 0).to(dev, dt).contiguous(),
            "o_proj": get(p + "self_attn.o_proj.weight").to(dev, dt).contiguous(),
            "down_proj": get(p + "mlp.down_proj.weight").to(dev, dt).contiguous(),
            "q_norm": get(p + "self_attn.q_norm.weight").to(dev, dt).contiguous(),
            "k_norm": get(p + "self_attn.k_norm.weight").to(dev, dt).contiguous(),
            "input_layernorm": get(p + "input_layernorm.weight").to(dev, dt).contiguous(),
            "post_attention_layernorm": get(p + "post_attention_layernorm.weight").to(dev, dt).contiguous(),
        }
        del q, k, v, gate, up
        layers.append(_layer_runtime(g, i, t))
    embed = tensors["model.embed_tokens.weight"].to(dev, dt).contiguous()
    final_norm = lm_head = None
    if include_output_head:
        final_norm = tensors["model.norm.weight"].to(dev, dt).contiguous()
        lm = tensors.get("lm_head.weight")
        lm_head = embed if lm is None else lm.to(dev, dt).contiguous()
    return QwenSemanticStackRuntime(
        model_path=Path("<in-memory>"), config=g, layer_indices=idx, embed_tokens_weight=embed,
        layers=tuple(layers), rope_inv_freq=rope_inv_freq(g, dev), attention_scaling=1.0,
        final_norm_weight=final_norm, lm_head_weight=lm_head, device=dev, dtype=dt)


# ---------------------------------------------------------------------------
# leanpack/v0 reader
# ---------------------------------------------------------------------------

@dataclass
class LeanPackArtifact:
    root: Path
    manifest: dict

    @property
    def tensor_index(self) -> dict[str, dict]:
        return {e["name"]: e for e in self.manifest.get("tensors", [])}

    def geometry(self) -> QwenGeometry:
        geo = self.manifest.get("geometry") or {}
        hp = self.manifest.get("model_hparams") or {}
        if not geo:
            raise ValueError("leanpack manifest has no geometry")
        return QwenGeometry(
            key=str(self.manifest.get("model_key", "leanpack")),
            num_hidden_layers=int(geo["num_hidden_layers"]), hidden_size=int(geo["hidden_size"]),
            intermediate_size=int(geo["intermediate_size"]), num_attention_heads=int(geo["num_attention_heads"]),
            num_key_value_heads=int(geo["num_key_value_heads"]), head_dim=int(geo["head_dim"]),
            vocab_size=int(geo["vocab_size"]), max_position_embeddings=int(geo.get("max_position_embeddings", 32768)),
            rms_norm_eps=float(hp.get("rms_norm_eps", 1e-6)), rope_theta=float(hp.get("rope_theta", 1_000_000.0)))

    def load(self, file_name: str, names, device, dtype) -> dict[str, torch.Tensor]:
        from safetensors import safe_open

        out = {}
        with safe_open(str(self.root / file_name), framework="pt", device="cpu") as fh:
            for n in names:
                out[n] = fh.get_tensor(n).to(device=device, dtype=dtype).contiguous()
        return out

    def lm_head_is_tied(self) -> bool:
        entry = self.tensor_index.get("lm_head.weight")
        return bool(entry) and entry.get("source_tensors") == ["model.embed_tokens.weight"]


def load_leanpack_artifact(path_or_dir) -> LeanPackArtifact:
    root = Path(path_or_dir)
    if root.name == "manifest.json":
        root = root.parent
    return LeanPackArtifact(root=root, manifest=json.loads((root / "manifest.json").read_text(encoding="utf-8")))


def materialize_qwen_semantic_stack_from_leanpack(pack_dir, *, model=None, layer_indices=None, device="cuda:0",
                                                  dtype="bfloat16", include_output_head: bool = False):
    """Reference signature (``leanserve.py:470-530``)."""
    art = load_leanpack_artifact(pack_dir)
    if model is not None and art.manifest.get("model_key") not in (None, getattr(model, "key", None)):
        raise ValueError(f"leanpack model_key mismatch: manifest={art.manifest.get('model_key')} "
                         f"requested={getattr(model, 'key', None)}")
    g = art.geometry()
    dev, dt = torch.device(device), resolve_torch_dtype(dtype)
    idx = tuple(range(g.num_hidden_layers)) if not layer_indices else tuple(layer_indices)
    for i in idx:
        if i < 0 or i >= g.num_hidden_layers:
            raise ValueError(f"layer index {i} out of range for num_hidden_layers={g.num_hidden_layers}")
    embed = art.load("embeddings.safetensors", ("model.embed_tokens.weight",), dev, dt)["model.embed_tokens.weight"]
    layers = []
    for i in idx:
        p = f"layers.{i}."
        names = {"input_layernorm": "input_layernorm.weight", "qkv": "attention.qkv_proj.weight",
                 "o_proj": "attention.o_proj.weight", "q_norm": "attention.q_norm.weight",
                 "k_norm": "attention.k_norm.weight", "post_attention_layernorm": "post_attention_layernorm.weight",
                 "gate_up": "mlp.gate_up_proj.weight", "down_proj": "mlp.down_proj.weight"}
        raw = art.load(f"layer-{i:03d}.safetensors", tuple(p + v for v in names.values()), dev, dt)
        layers.append(_layer_runtime(g, i, {k: raw[p + v] for k, v in names.items()}))
    final_norm = lm_head = None
    if include_output_head:
        if art.lm_head_is_tied():
            final_norm = art.load("output.safetensors", ("model.norm.weight",), dev, dt)["model.norm.weight"]
            lm_head = embed
        else:
            out = art.load("output.safetensors", ("model.norm.weight", "lm_head.weight"), dev, dt)
            final_norm, lm_head = out["model.norm.weight"], out["lm_head.weight"]
    return QwenSemanticStackRuntime(
        model_path=art.root, config=g, layer_indices=idx, embed_tokens_weight=embed, layers=tuple(layers),
        rope_inv_freq=rope_inv_freq(g, dev), attention_scaling=1.0, final_norm_weight=final_norm,
        lm_head_weight=lm_head, device=dev, dtype=dt)


def materialize_qwen_full_semantic_runtime_from_leanpack(pack_dir, *, model=None, device="cuda:0",
                                                         dtype="bfloat16", include_output_head: bool = True):
    """Reference signature (``leanserve.py:533-548``)."""
    return materialize_qwen_semantic_stack_from_leanpack(pack_dir, model=model, layer_indices=None, device=device,
                                                         dtype=dtype, include_output_head=include_output_head)


# ---------------------------------------------------------------------------
# leanpack/v1 reader (format written by pack.write_qwen_leanpack_v1)
# ---------------------------------------------------------------------------

_DTYPES = {"bfloat16": torch.bfloat16, "float16": torch.float16, "float32": torch.float32, "uint8": torch.uint8}


def map_leanpack_v1_rank(pack_dir, rank: int = 0) -> tuple[dict, dict[str, torch.Tensor]]:
    """Map rank ``rank``'s shard file and return ``(manifest, {name: CPU view})``.

    The file is memory-mapped (copy-on-write, nothing is read until touched) and
    every stored tensor is a zero-copy view at its recorded offset.  The tied
    head's entry is left out: it is a row range of the embedding, see
    :func:`materialize_from_leanpack_v1`.
    """
    root = Path(pack_dir)
    if root.name == "manifest.json":
        root = root.parent
    manifest = json.loads((root / "manifest.json").read_text(encoding="utf-8"))
    if manifest.get("format_version") != "leanpack/v1":
        raise ValueError(f"not a leanpack/v1 artifact: {manifest.get('format_version')!r}")
    world = int(manifest["tensor_parallel"]["world"])
    if not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside the pack's tensor-parallel world of {world}")
    finfo = next(f for f in manifest["files"] if f["rank"] == rank)
    path = root / finfo["file"]
    size = path.stat().st_size
    if size != finfo["size_bytes"]:
        raise ValueError(f"{path.name}: {size} bytes on disk, manifest says {finfo['size_bytes']}")
    align = int(manifest.get("alignment_bytes", 1))
    blob = torch.from_file(str(path), shared=False, size=size, dtype=torch.uint8)
    views: dict[str, torch.Tensor] = {}
    for e in manifest["tensors"]:
        if e["rank"] != rank or e.get("view_of"):
            continue
        off, n = int(e["offset_bytes"]), int(e["size_bytes"])
        if off % align or off + n > size:
            raise ValueError(f"{e['name']}: bad extent [{off}, {off + n}) in a {size}-byte file")
        dt = _DTYPES[e["dtype"]]
        views[e["name"]] = blob[off:off + n].view(dt).view(e["shape"])
    return manifest, views


def materialize_from_leanpack_v1(pack_dir, *, rank: int = 0, device="cuda:0", dtype="bfloat16"):
    """Build rank ``rank``'s runtime from a leanpack/v1 artifact.

    Returns ``(runtime, shard, tc_tiles)``: the runtime in the rank's local
    geometry (whole model when the pack has one rank), its
    :class:`~leanstack_b200.tp.TPShard` (vocab range of its head), and, when the
    pack holds tile images, one ``{"qkv", "o", "gu", "down"}`` dict per layer of
    device tensors for ``DecodeEngine(tc_tiles=...)`` (else None).
    """
    from .tp import local_geometry, shard_info

    manifest, views = map_leanpack_v1_rank(pack_dir, rank)
    art = LeanPackArtifact(root=Path(pack_dir), manifest=manifest)
    g = art.geometry()
    world = int(manifest["tensor_parallel"]["world"])
    lg = local_geometry(g, world)
    shard = shard_info(g, rank, world)
    dev, dt = torch.device(device), resolve_torch_dtype(dtype)
    put = lambda name: views[name].to(dev, dt).contiguous()  # noqa: E731
    names = {"input_layernorm": "input_layernorm.weight", "qkv": "attention.qkv_proj.weight",
             "o_proj": "attention.o_proj.weight", "q_norm": "attention.q_norm.weight",
             "k_norm": "attention.k_norm.weight", "post_attention_layernorm": "post_attention_layernorm.weight",
             "gate_up": "mlp.gate_up_proj.weight", "down_proj": "mlp.down_proj.weight"}
    layers = []
    for i in range(g.num_hidden_layers):
        layers.append(_layer_runtime(lg, i, {k: put(f"layers.{i}.{v}") for k, v in names.items()}))
    embed = put("model.embed_tokens.weight")
    head = next(e for e in manifest["tensors"] if e["rank"] == rank and e["name"] == "lm_head.weight")
    if head.get("view_of"):
        lm = embed[int(head["row_offset"]):int(head["row_offset"]) + int(head["rows"])]
    else:
        lm = put("lm_head.weight")
    rt = QwenSemanticStackRuntime(
        model_path=art.root, config=lg, layer_indices=tuple(range(g.num_hidden_layers)), embed_tokens_weight=embed,
        layers=tuple(layers), rope_inv_freq=rope_inv_freq(g, dev), attention_scaling=1.0,
        final_norm_weight=put("model.norm.weight"), lm_head_weight=lm, device=dev, dtype=dt)
    tiles = None
    if manifest.get("tc_tiles"):
        keys = {"attention.qkv_proj": "qkv", "attention.o_proj": "o", "mlp.gate_up_proj": "gu",
                "mlp.down_proj": "down"}
        tiles = [{k: views[f"layers.{i}.{base}.tc_tiled"].to(dev) for base, k in keys.items()}
                 for i in range(g.num_hidden_layers)]
    return rt, shard, tiles


# ---------------------------------------------------------------------------
# Resident buffer planner
# ---------------------------------------------------------------------------

@dataclass(frozen=True)
class ScratchPlan:
    """Per-step activation arenas for ``tokens`` tokens in flight (``leanserve.py:52-68``)."""

    tokens: int
    hidden_state_bytes: int
    qkv_projection_bytes: int
    attention_output_bytes: int
    mlp_activation_bytes: int
    logits_bytes: int

    @property
    def total_bytes(self) -> int:
        return (self.hidden_state_bytes + self.qkv_projection_bytes + self.attention_output_bytes
                + self.mlp_activation_bytes + self.logits_bytes)


@dataclass(frozen=True)
class ResidentBufferPlan:
    weights_bytes: int
    batch_size: int
    max_seq_len: int
    kv_cache_bytes: int
    scratch: ScratchPlan
    page_size: int = 16

    @property
    def resident_bytes(self) -> int:
        return self.weights_bytes + self.kv_cache_bytes + self.scratch.total_bytes


def runtime_weight_bytes(rt: QwenSemanticStackRuntime) -> int:
    seen, total = set(), 0
    tensors = [rt.embed_tokens_weight, rt.final_norm_weight, rt.lm_head_weight]
    for layer in rt.layers:
        a, m = layer.attention, layer.mlp
        tensors += [layer.input_layernorm_weight, a.qkv_proj_weight, a.o_proj_weight, a.q_norm_weight,
                    a.k_norm_weight, layer.post_attention_layernorm_weight, m.gate_up_proj_weight,
                    m.down_proj_weight]
    for t in tensors:
        if t is None or t.data_ptr() in seen:
            continue
        seen.add(t.data_ptr())
        total += t.numel() * t.element_size()
    return total


def build_resident_buffer_plan(geometry: QwenGeometry, *, weights_bytes: int, batch_size: int, max_seq_len: int,
                               max_tokens_per_step: int, page_size: int = 16, dtype_bytes: int = 2) -> ResidentBufferPlan:
    g = geometry
    kv_tokens = (max_seq_len + page_size - 1) // page_size * page_size
    kv = batch_size * g.num_hidden_layers * 2 * g.kv_dim * kv_tokens * dtype_bytes
    t = max_tokens_per_step
    scratch = ScratchPlan(
        tokens=t,
        hidden_state_bytes=2 * t * g.hidden_size * dtype_bytes,
        qkv_projection_bytes=t * (g.qkv_dim + g.q_dim) * dtype_bytes,
        attention_output_bytes=t * g.q_dim * dtype_bytes,
        mlp_activation_bytes=t * g.intermediate_size * dtype_bytes,
        logits_bytes=batch_size * 8,
    )
    return ResidentBufferPlan(weights_bytes=weights_bytes, batch_size=batch_size, max_seq_len=kv_tokens,
                              kv_cache_bytes=kv, scratch=scratch, page_size=page_size)


@dataclass
class Arenas:
    """The resident buffers one engine instance writes into."""

    kv: StaticKVBlockManager
    x: torch.Tensor          # [T, H] residual stream
    h: torch.Tensor          # [T, H] post-attention residual
    qkv: torch.Tensor        # [T, qkv_dim] raw projection
    q: torch.Tensor          # [T, Hq, D] rotated q
    attn: torch.Tensor       # [T, Hq*D]
    act: torch.Tensor        # [T, I]
    ids: torch.Tensor        # [T] int64 token ids of the step
    head_rows: torch.Tensor  # [B, H] last position per sequence (prefill head input)
    extra: dict = field(default_factory=dict)


def allocate_arenas(plan: ResidentBufferPlan, geometry: QwenGeometry, device, dtype=torch.bfloat16) -> Arenas:
    g = geometry
    t = plan.scratch.tokens
    dev = torch.device(device)
    layout = KVPageLayout(num_layers=g.num_hidden_layers, num_key_value_heads=g.num_key_value_heads,
                          head_dim=g.head_dim, page_size=plan.page_size, max_seq_len=plan.max_seq_len,
                          batch_size=plan.batch_size, dtype=dtype, device=dev)
    kv = StaticKVBlockManager(layout)

    def z(*shape, dt=dtype):
        return torch.zeros(shape, device=dev, dtype=dt)

    return Arenas(kv=kv, x=z(t, g.hidden_size), h=z(t, g.hidden_size), qkv=z(t, g.qkv_dim),
                  q=z(t, g.num_attention_heads, g.head_dim), attn=z(t, g.q_dim), act=z(t, g.intermediate_size),
                  ids=z(t, dt=torch.int64), head_rows=z(plan.batch_size, g.hidden_size))
