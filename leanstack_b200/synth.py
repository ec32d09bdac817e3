"""Seeded synthetic inputs that are bit-identical on the CPU and on the GPU.

The benchmark configurations use random-init Qwen3 weights (``N(0, 0.02)``
linears, ``1 + N(0, 0.01)`` norm weights), ``N(0, 1)`` activations and KV
entries, and uniform-random token ids.  ``torch.randn`` gives different values
on CPU and CUDA, so it cannot feed both the CPU oracle and the GPU kernels.
Instead every value here is a table lookup driven by an integer hash:

* ``hash(i) = mix32(mix32(i) ^ key)`` with a 32-bit bijective mixer; ``key`` is
  the CRC32 of ``"<seed>/<tensor name>"``.  Integer ops are exact on both
  devices.
* the top 16 bits select one of 65,536 normal quantiles
  ``sqrt(2) * erfinv(2 (j + 0.5) / 65536 - 1)``; the table is computed once in
  float64 on the CPU, scaled, rounded to bf16 and copied to the device.

So a tensor depends only on (seed, name, shape), never on the device, and the
GPU can regenerate the 8 GB of Qwen3-4B weights in well under a second.
"""

from __future__ import annotations

import zlib
from functools import lru_cache

import torch

from .config import QwenGeometry

_MASK32 = 0xFFFFFFFF
_CHUNK = 1 << 24


def stream_key(seed: int, name: str) -> int:
    return zlib.crc32(f"{int(seed)}/{name}".encode("utf-8")) & _MASK32


def _mix32(x: torch.Tensor) -> torch.Tensor:
    # x is int64 holding values in [0, 2^32); both multipliers are < 2^31 so no
    # product leaves the non-negative int64 range.
    x = x ^ (x >> 16)
    x = (x * 0x7FEB352D) & _MASK32
    x = x ^ (x >> 15)
    x = (x * 0x5BD1E995) & _MASK32
    x = x ^ (x >> 16)
    return x


def hash_stream(start: int, count: int, key: int, device) -> torch.Tensor:
    idx = torch.arange(start, start + count, device=device, dtype=torch.int64) & _MASK32
    return _mix32(_mix32(idx) ^ key)


@lru_cache(maxsize=None)
def _unit_quantiles() -> torch.Tensor:
    j = torch.arange(65536, dtype=torch.float64)
    p = (j + 0.5) / 65536.0
    return torch.erfinv(2.0 * p - 1.0) * (2.0 ** 0.5)


@lru_cache(maxsize=None)
def _normal_table_cpu(std: float) -> torch.Tensor:
    return (_unit_quantiles() * float(std)).to(torch.float32).to(torch.bfloat16)


@lru_cache(maxsize=None)
def _norm_weight_table_cpu(std: float) -> torch.Tensor:
    return (1.0 + _normal_table_cpu(std).to(torch.float32)).to(torch.bfloat16)


_DEVICE_TABLES: dict = {}


def _table(kind: str, std: float, device) -> torch.Tensor:
    device = torch.device(device)
    cache_key = (kind, float(std), str(device))
    table = _DEVICE_TABLES.get(cache_key)
    if table is None:
        cpu = _normal_table_cpu(std) if kind == "normal" else _norm_weight_table_cpu(std)
        table = cpu.to(device)
        _DEVICE_TABLES[cache_key] = table
    return table


def _fill_from_table(out: torch.Tensor, table: torch.Tensor, key: int) -> torch.Tensor:
    flat = out.view(-1)
    n = flat.numel()
    for start in range(0, n, _CHUNK):
        count = min(_CHUNK, n - start)
        h = hash_stream(start, count, key, flat.device)
        flat[start:start + count] = table[h >> 16]
    return out


def normal(shape, std: float, seed: int, name: str, device="cpu") -> torch.Tensor:
    """bf16 tensor with values from the ``N(0, std)`` quantile table."""
    out = torch.empty(tuple(shape), dtype=torch.bfloat16, device=device)
    return _fill_from_table(out, _table("normal", std, device), stream_key(seed, name))


def norm_weight(shape, seed: int, name: str, device="cpu", std: float = 0.01) -> torch.Tensor:
    """bf16 RMSNorm weight ``1 + N(0, std)``."""
    out = torch.empty(tuple(shape), dtype=torch.bfloat16, device=device)
    return _fill_from_table(out, _table("norm", std, device), stream_key(seed, name))


def token_ids(shape, vocab_size: int, seed: int, name: str, device="cpu") -> torch.Tensor:
    """Uniform-random token ids in ``[0, vocab_size)`` (int64)."""
    out = torch.empty(tuple(shape), dtype=torch.int64, device=device)
    flat = out.view(-1)
    n = flat.numel()
    key = stream_key(seed, name)
    for start in range(0, n, _CHUNK):
        count = min(_CHUNK, n - start)
        flat[start:start + count] = hash_stream(start, count, key, flat.device) % int(vocab_size)
    return out


# ---------------------------------------------------------------------------
# Whole-checkpoint helpers (Hugging Face tensor names, as a Qwen3 checkpoint
# directory would hold them; the reference reads these names in
# src/leanstack/runtime/qwen_explicit.py:187-211).
# ---------------------------------------------------------------------------

LINEAR_STD = 0.02


def layer_tensor_shapes(geometry: QwenGeometry, layer_idx: int) -> dict[str, tuple[int, ...]]:
    g = geometry
    p = f"model.layers.{layer_idx}."
    return {
        f"{p}input_layernorm.weight": (g.hidden_size,),
        f"{p}self_attn.q_proj.weight": (g.q_dim, g.hidden_size),
        f"{p}self_attn.k_proj.weight": (g.kv_dim, g.hidden_size),
        f"{p}self_attn.v_proj.weight": (g.kv_dim, g.hidden_size),
        f"{p}self_attn.o_proj.weight": (g.hidden_size, g.q_dim),
        f"{p}self_attn.q_norm.weight": (g.head_dim,),
        f"{p}self_attn.k_norm.weight": (g.head_dim,),
        f"{p}post_attention_layernorm.weight": (g.hidden_size,),
        f"{p}mlp.gate_proj.weight": (g.intermediate_size, g.hidden_size),
        f"{p}mlp.up_proj.weight": (g.intermediate_size, g.hidden_size),
        f"{p}mlp.down_proj.weight": (g.hidden_size, g.intermediate_size),
    }


def synth_tensor(name: str, shape, seed: int, device="cpu") -> torch.Tensor:
    if name.endswith("norm.weight"):
        return norm_weight(shape, seed, name, device=device)
    return normal(shape, LINEAR_STD, seed, name, device=device)


def synth_layer(geometry: QwenGeometry, layer_idx: int, seed: int, device="cpu") -> dict[str, torch.Tensor]:
    return {
        name: synth_tensor(name, shape, seed, device)
        for name, shape in layer_tensor_shapes(geometry, layer_idx).items()
    }


def synth_embedding(geometry: QwenGeometry, seed: int, device="cpu") -> torch.Tensor:
    return normal((geometry.vocab_size, geometry.hidden_size), LINEAR_STD, seed,
                  "model.embed_tokens.weight", device=device)


def synth_final_norm(geometry: QwenGeometry, seed: int, device="cpu") -> torch.Tensor:
    return norm_weight((geometry.hidden_size,), seed, "model.norm.weight", device=device)


def synth_checkpoint(geometry: QwenGeometry, seed: int, device="cpu") -> dict[str, torch.Tensor]:
    """All tensors of a tied-embedding Qwen3 checkpoint under HF names."""
    out = {"model.embed_tokens.weight": synth_embedding(geometry, seed, device)}
    for layer_idx in range(geometry.num_hidden_layers):
        out.update(synth_layer(geometry, layer_idx, seed, device))
    out["model.norm.weight"] = synth_final_norm(geometry, seed, device)
    if not geometry.tie_word_embeddings:
        out["lm_head.weight"] = normal((geometry.vocab_size, geometry.hidden_size), LINEAR_STD, seed,
                                       "lm_head.weight", device=device)
    return out


def tensor_digest(t: torch.Tensor) -> str:
    """Order-sensitive 64-bit digest of a tensor's bytes (for pinning inputs)."""
    import hashlib

    data = t.detach().to("cpu").contiguous().view(torch.uint8).numpy().tobytes()
    return hashlib.blake2b(data, digest_size=8).hexdigest()
