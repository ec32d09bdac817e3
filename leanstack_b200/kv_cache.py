"""Static resident KV cache with the reference's manager protocol.

``StaticKVBlockManager`` keeps the reference's API (``src/leanstack/runtime/
kv_cache.py:207-318``: append / get / append_and_get / get_seq_length /
get_layer_seq_length / page_table / summary / snapshot_* / restore_* /
cursor_after_tokens) and its arena layout ``[L, B, Hkv, max_seq, D]``, but the
arenas are allocated once by the buffer planner and reused across requests,
and it adds what the batched hot path needs:

* per-sequence cursors (``sequence_lens``), mirrored on the device as the int32
  ``cache_pos`` tensor that the kernels read, so a batch can hold ragged
  sequences (speculative acceptance differs per sequence);
* ``advance`` / ``set_sequence_lens`` to move both views together.

The per-layer cursors of the reference stay for protocol compatibility: the
layer-at-a-time dispatch path advances one layer at a time, the engine moves
all layers at once.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch


@dataclass(frozen=True)
class KVPageLayout:
    """Same fields and checks as the reference (``kv_cache.py:8-34``)."""

    num_layers: int
    num_key_value_heads: int
    head_dim: int
    page_size: int
    max_seq_len: int
    batch_size: int
    dtype: torch.dtype
    device: torch.device

    def __post_init__(self) -> None:
        if self.page_size <= 0:
            raise ValueError("page_size must be positive")
        if self.max_seq_len <= 0:
            raise ValueError("max_seq_len must be positive")
        if self.batch_size <= 0:
            raise ValueError("batch_size must be positive")

    @property
    def num_pages(self) -> int:
        return (self.max_seq_len + self.page_size - 1) // self.page_size

    def pages_for_tokens(self, token_count: int) -> int:
        if token_count <= 0:
            return 0
        return (token_count + self.page_size - 1) // self.page_size

    def arena_shape(self) -> tuple[int, int, int, int, int]:
        return (self.num_layers, self.batch_size, self.num_key_value_heads, self.max_seq_len, self.head_dim)

    def arena_bytes(self) -> int:
        n = 1
        for d in self.arena_shape():
            n *= d
        return 2 * n * torch.tensor([], dtype=self.dtype).element_size()


@dataclass
class StaticKVCacheSnapshot:
    key_cache: torch.Tensor
    value_cache: torch.Tensor
    layer_seq_lens: list[int]
    max_layer_seq_len: int
    sequence_lens: list[int]


@dataclass(frozen=True)
class StaticKVCursorSnapshot:
    layer_seq_lens: tuple[int, ...]
    max_layer_seq_len: int
    sequence_lens: tuple[int, ...] = ()


class StaticKVBlockManager:
    def __init__(self, layout: KVPageLayout, key_cache: torch.Tensor | None = None,
                 value_cache: torch.Tensor | None = None):
        self.layout = layout
        shape = layout.arena_shape()
        if key_cache is None:
            key_cache = torch.zeros(shape, device=layout.device, dtype=layout.dtype)
        if value_cache is None:
            value_cache = torch.zeros(shape, device=layout.device, dtype=layout.dtype)
        if tuple(key_cache.shape) != shape or tuple(value_cache.shape) != shape:
            raise ValueError(f"arena shape mismatch: expected {shape}")
        self.key_cache = key_cache
        self.value_cache = value_cache
        self.layer_seq_lens = [0 for _ in range(layout.num_layers)]
        self.max_layer_seq_len = 0
        self.sequence_lens = [0 for _ in range(layout.batch_size)]
        self.cache_pos = torch.zeros((layout.batch_size,), device=layout.device, dtype=torch.int32)

    # -- reference protocol ------------------------------------------------
    def _check_states(self, key_states: torch.Tensor, value_states: torch.Tensor) -> int:
        if key_states.shape != value_states.shape:
            raise ValueError("key/value states must have the same shape")
        batch_size, num_heads, token_count, head_dim = key_states.shape
        if batch_size != self.layout.batch_size:
            raise ValueError(f"expected batch_size={self.layout.batch_size}, got {batch_size}")
        if num_heads != self.layout.num_key_value_heads:
            raise ValueError(f"expected num_key_value_heads={self.layout.num_key_value_heads}, got {num_heads}")
        if head_dim != self.layout.head_dim:
            raise ValueError(f"expected head_dim={self.layout.head_dim}, got {head_dim}")
        return token_count

    def reserve(self, layer_idx: int, token_count: int) -> int:
        """Check room for ``token_count`` more tokens in a layer; return its cursor."""
        start = self.layer_seq_lens[layer_idx]
        end = start + token_count
        if end > self.layout.max_seq_len:
            raise ValueError(
                f"cache overflow for layer {layer_idx}: requested {end} tokens with "
                f"max_seq_len={self.layout.max_seq_len}")
        return start

    def advance_layer(self, layer_idx: int, token_count: int) -> None:
        end = self.reserve(layer_idx, token_count) + token_count
        self.layer_seq_lens[layer_idx] = end
        self.max_layer_seq_len = max(self.max_layer_seq_len, end)

    def append(self, layer_idx: int, key_states: torch.Tensor, value_states: torch.Tensor) -> None:
        token_count = self._check_states(key_states, value_states)
        start = self.reserve(layer_idx, token_count)
        self.key_cache[layer_idx, :, :, start:start + token_count].copy_(key_states)
        self.value_cache[layer_idx, :, :, start:start + token_count].copy_(value_states)
        self.advance_layer(layer_idx, token_count)
        if layer_idx == self.layout.num_layers - 1:
            # a full layer pass finished: every sequence now holds the same count
            self.set_sequence_lens([self.layer_seq_lens[layer_idx]] * self.layout.batch_size, align_layers=False)

    def append_and_get(self, layer_idx: int, key_states: torch.Tensor, value_states: torch.Tensor):
        self.append(layer_idx, key_states, value_states)
        return self.get(layer_idx)

    def get(self, layer_idx: int):
        seq_len = self.layer_seq_lens[layer_idx]
        return (self.key_cache[layer_idx, :, :, :seq_len, :], self.value_cache[layer_idx, :, :, :seq_len, :])

    def get_layer_seq_length(self, layer_idx: int) -> int:
        return self.layer_seq_lens[layer_idx]

    def get_seq_length(self) -> int:
        return self.max_layer_seq_len

    def page_table(self, layer_idx: int) -> tuple[int, ...]:
        return tuple(range(self.layout.pages_for_tokens(self.get_layer_seq_length(layer_idx))))

    def summary(self) -> dict:
        seq_len = self.get_seq_length()
        return {
            "cache_kind": "static",
            "page_size": self.layout.page_size,
            "num_pages": self.layout.num_pages,
            "used_pages": self.layout.pages_for_tokens(seq_len),
            "allocated_pages": self.layout.pages_for_tokens(seq_len),
            "seq_len": seq_len,
            "sequence_lens": list(self.sequence_lens),
        }

    def snapshot_state(self) -> StaticKVCacheSnapshot:
        return StaticKVCacheSnapshot(self.key_cache.clone(), self.value_cache.clone(), list(self.layer_seq_lens),
                                     int(self.max_layer_seq_len), list(self.sequence_lens))

    def restore_state(self, snapshot: StaticKVCacheSnapshot) -> None:
        self.key_cache.copy_(snapshot.key_cache)
        self.value_cache.copy_(snapshot.value_cache)
        self.layer_seq_lens = list(snapshot.layer_seq_lens)
        self.max_layer_seq_len = int(snapshot.max_layer_seq_len)
        self.set_sequence_lens(snapshot.sequence_lens)

    def snapshot_cursor(self) -> StaticKVCursorSnapshot:
        return StaticKVCursorSnapshot(tuple(int(n) for n in self.layer_seq_lens), int(self.max_layer_seq_len),
                                      tuple(int(n) for n in self.sequence_lens))

    def restore_cursor(self, snapshot: StaticKVCursorSnapshot) -> None:
        seq = snapshot.sequence_lens or (int(snapshot.max_layer_seq_len),) * self.layout.batch_size
        self.set_sequence_lens(seq, align_layers=False)
        self.layer_seq_lens = list(snapshot.layer_seq_lens)
        self.max_layer_seq_len = int(snapshot.max_layer_seq_len)

    def cursor_after_tokens(self, snapshot: StaticKVCursorSnapshot, token_count: int) -> StaticKVCursorSnapshot:
        if token_count < 0:
            raise ValueError("token_count must be non-negative")
        return StaticKVCursorSnapshot(
            tuple(int(n) + token_count for n in snapshot.layer_seq_lens),
            int(snapshot.max_layer_seq_len) + token_count,
            tuple(int(n) + token_count for n in snapshot.sequence_lens),
        )

    # -- batched hot path ---------------------------------------------------
    def set_sequence_lens(self, lens, align_layers: bool = True) -> None:
        """Set every sequence's cursor (host and device); by default align the layer cursors to the longest."""
        lens = [int(n) for n in lens]
        if len(lens) != self.layout.batch_size:
            raise ValueError(f"expected {self.layout.batch_size} lengths, got {len(lens)}")
        if any(n < 0 or n > self.layout.max_seq_len for n in lens):
            raise ValueError(f"sequence length outside [0, {self.layout.max_seq_len}]: {lens}")
        self.sequence_lens = lens
        self.cache_pos.copy_(torch.tensor(lens, dtype=torch.int32), non_blocking=False)
        if align_layers:
            top = max(lens)
            self.layer_seq_lens = [top] * self.layout.num_layers
            self.max_layer_seq_len = top

    def note_advanced(self, token_count: int) -> None:
        """Record on the host that a device step advanced every sequence by ``token_count``."""
        self.sequence_lens = [n + token_count for n in self.sequence_lens]
        top = max(self.sequence_lens)
        if top > self.layout.max_seq_len:
            raise ValueError(f"cache overflow: {top} tokens with max_seq_len={self.layout.max_seq_len}")
        self.layer_seq_lens = [top] * self.layout.num_layers
        self.max_layer_seq_len = top

    def reset(self) -> None:
        self.set_sequence_lens([0] * self.layout.batch_size)
