"""Model geometry for the decode hot path.

The geometry constants restate the reference's model registry
(``src/leanstack/model_registry.py:6-93`` for Qwen3-4B-Base and ``:94-128``
for the Qwen3-0.6B-Base draft) and the leanserve serve config
(``src/leanstack/leanserve.py:36-49``).  Only the fields the hot path reads are
kept; the control-plane policy strings of the registry are out of scope.
"""

from __future__ import annotations

from dataclasses import asdict, dataclass, field


@dataclass(frozen=True)
class QwenGeometry:
    """Shape of one Qwen3 decoder stack.

    Mirrors ``QwenServeConfig`` (``src/leanstack/leanserve.py:36-49``): the
    attribute names are the Hugging Face / reference names so that code written
    against the reference's ``runtime.config`` reads the same fields.
    """

    key: str
    num_hidden_layers: int
    hidden_size: int
    intermediate_size: int
    num_attention_heads: int
    num_key_value_heads: int
    head_dim: int
    vocab_size: int
    max_position_embeddings: int = 32768
    rms_norm_eps: float = 1e-6
    rope_theta: float = 1_000_000.0
    tie_word_embeddings: bool = True
    rope_parameters: dict = field(default_factory=dict)

    def __post_init__(self) -> None:
        if not self.rope_parameters:
            object.__setattr__(self, "rope_parameters", {"rope_theta": float(self.rope_theta)})
        if self.num_attention_heads % self.num_key_value_heads != 0:
            raise ValueError("num_attention_heads must be a multiple of num_key_value_heads")

    # Derived sizes -----------------------------------------------------
    @property
    def q_dim(self) -> int:
        return self.num_attention_heads * self.head_dim

    @property
    def kv_dim(self) -> int:
        return self.num_key_value_heads * self.head_dim

    @property
    def qkv_dim(self) -> int:
        return self.q_dim + 2 * self.kv_dim

    @property
    def num_key_value_groups(self) -> int:
        return self.num_attention_heads // self.num_key_value_heads

    def layer_weight_bytes(self, dtype_bytes: int = 2) -> int:
        """Bytes one decoder layer streams per decode step (linears + norms)."""
        h, i = self.hidden_size, self.intermediate_size
        linears = self.qkv_dim * h + h * self.q_dim + 2 * i * h + h * i
        norms = 2 * h + 2 * self.head_dim
        return (linears + norms) * dtype_bytes

    def lm_head_bytes(self, dtype_bytes: int = 2) -> int:
        return self.vocab_size * self.hidden_size * dtype_bytes

    def kv_bytes_per_token(self, dtype_bytes: int = 2) -> int:
        """K and V bytes per cached position across all layers (147,456 B for 4B)."""
        return self.num_hidden_layers * 2 * self.kv_dim * dtype_bytes

    def as_dict(self) -> dict:
        return asdict(self)


# Qwen3-4B-Base (model_registry.py:6-93).
QWEN3_4B = QwenGeometry(
    key="qwen3-4b",
    num_hidden_layers=36,
    hidden_size=2560,
    intermediate_size=9728,
    num_attention_heads=32,
    num_key_value_heads=8,
    head_dim=128,
    vocab_size=151936,
)

# Qwen3-0.6B-Base draft (model_registry.py:94-128).  q_dim (2048) differs from
# hidden_size (1024), which the kernels must handle.
QWEN3_06B_DRAFT = QwenGeometry(
    key="qwen3-0.6b",
    num_hidden_layers=28,
    hidden_size=1024,
    intermediate_size=3072,
    num_attention_heads=16,
    num_key_value_heads=8,
    head_dim=128,
    vocab_size=151936,
)

# Small geometries for fast parity tests.  head_dim stays 128 (the kernels are
# specialised for it); every other dimension is a small multiple of 128.
TINY = QwenGeometry(
    key="tiny",
    num_hidden_layers=2,
    hidden_size=512,
    intermediate_size=1536,
    num_attention_heads=4,
    num_key_value_heads=2,
    head_dim=128,
    vocab_size=4096,
    max_position_embeddings=2048,
)

TINY_DRAFT = QwenGeometry(
    key="tiny-draft",
    num_hidden_layers=2,
    hidden_size=256,
    intermediate_size=768,
    num_attention_heads=4,
    num_key_value_heads=2,
    head_dim=128,
    vocab_size=4096,
    max_position_embeddings=2048,
)

GEOMETRIES = {g.key: g for g in (QWEN3_4B, QWEN3_06B_DRAFT, TINY, TINY_DRAFT)}


def get_geometry(key: str) -> QwenGeometry:
    try:
        return GEOMETRIES[key]
    except KeyError as exc:
        raise ValueError(f"unknown geometry {key!r}; known: {sorted(GEOMETRIES)}") from exc
