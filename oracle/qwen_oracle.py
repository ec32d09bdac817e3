"""CPU oracle for the Qwen3 decode hot path — TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline /
reference arm may import this module, and only as the checker or the timed CPU
baseline.  The product path (``leanstack_b200``) never calls it.

What it is: a restatement, in eager PyTorch on the CPU, of the arithmetic of
the reference's "semantic" Qwen3 runtime (``src/leanstack/runtime/
qwen_explicit.py``) and its static KV cache (``src/leanstack/runtime/
kv_cache.py``).  Each function cites the reference lines it follows.  Two
precisions:

* ``"bf16"`` mirrors the reference: every tensor is bf16, so each torch op
  rounds its result to bf16 exactly where the reference's ops do (after every
  linear, RMSNorm, RoPE multiply/subtract, SiLU, multiply, residual add and
  attention).  This is the token-parity oracle.
* ``"fp32"`` runs the same formulas on fp32 tensors (bf16 weights and inputs
  upcast).  This is the "fp32-accumulated reference" that the ≤2e-2
  max-abs-error criterion is measured against.

Pinning: ``tests/golden/make_golden.py`` runs the reference itself (imported
from its source tree in the build container) on the same seeded inputs and
stores its outputs as fixtures; ``tests/test_oracle_golden.py`` checks this
module against them bit for bit.  The reference's own tests pin shapes only
(``tests/test_hot_kernel_cases.py:17-28``, ``tests/test_active_contract.py:11-21``).
"""

from __future__ import annotations

from dataclasses import dataclass, field

import torch
import torch.nn.functional as F

BF16 = torch.bfloat16


def _dt(precision: str) -> torch.dtype:
    if precision == "bf16":
        return BF16
    if precision == "fp32":
        return torch.float32
    raise ValueError(f"unknown precision {precision!r}")


# ---------------------------------------------------------------------------
# Elementwise pieces
# ---------------------------------------------------------------------------

def rmsnorm(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    """``F.rms_norm`` over the last dim (``qwen_explicit.py:621-633``).

    For bf16 input torch computes ``bf16((x * rsqrt(mean(x^2) + eps)) * w)``
    in fp32 with a single rounding.
    """
    return F.rms_norm(x, normalized_shape=(x.shape[-1],), weight=weight.to(x.dtype), eps=eps)


def rope_inv_freq(head_dim: int, theta: float) -> torch.Tensor:
    """``1 / theta^(arange(0, D, 2)/D)`` in fp32 (``qwen_explicit.py:465-469``)."""
    return 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.float32) / head_dim))


def rope_cache(inv_freq: torch.Tensor, max_seq_len: int, dtype: torch.dtype,
               attention_scaling: float = 1.0) -> tuple[torch.Tensor, torch.Tensor]:
    """cos/sin table ``[max_seq_len, D/2]`` (``qwen_explicit.py:664-676``).

    Angles are fp32 products ``pos * inv_freq``; cos/sin are taken in fp32 and
    rounded to the model dtype (bf16), exactly as the reference's position cache.
    """
    pos = torch.arange(max_seq_len, dtype=torch.float32, device=inv_freq.device)
    freqs = torch.outer(pos, inv_freq.float())
    return ((freqs.cos() * attention_scaling).to(dtype), (freqs.sin() * attention_scaling).to(dtype))


def apply_rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """NeoX-half rotation ``[x1 c - x2 s, x2 c + x1 s]`` (``qwen_explicit.py:690-716``).

    ``x`` is ``[B, H, Q, D]``; ``cos``/``sin`` are ``[B or 1, Q, D/2]``.  In bf16
    every product and the sum/difference round separately, as in the reference.
    """
    c = cos.unsqueeze(1)
    s = sin.unsqueeze(1)
    x1, x2 = x.chunk(2, dim=-1)
    return torch.cat((x1 * c - x2 * s, x2 * c + x1 * s), dim=-1)


# ---------------------------------------------------------------------------
# Layer pieces (general B x Q path; the bs1 vector path is the same arithmetic)
# ---------------------------------------------------------------------------

@dataclass
class LayerWeights:
    """One decoder layer in the leanpack fused layout (``pack.py:271-285``)."""

    input_layernorm: torch.Tensor
    qkv_proj: torch.Tensor          # [Hq*D + 2*Hkv*D, H]
    o_proj: torch.Tensor            # [H, Hq*D]
    q_norm: torch.Tensor            # [D]
    k_norm: torch.Tensor            # [D]
    post_attention_layernorm: torch.Tensor
    gate_up_proj: torch.Tensor      # [2*I, H]
    down_proj: torch.Tensor         # [H, I]

    def to(self, dtype: torch.dtype) -> "LayerWeights":
        return LayerWeights(**{k: v.to(dtype) for k, v in self.__dict__.items()})


def fuse_layer(tensors: dict[str, torch.Tensor], layer_idx: int) -> LayerWeights:
    """Fuse HF per-projection tensors the way leanpack does (``pack.py:271-285``)."""
    p = f"model.layers.{layer_idx}."
    return LayerWeights(
        input_layernorm=tensors[f"{p}input_layernorm.weight"],
        qkv_proj=torch.cat((tensors[f"{p}self_attn.q_proj.weight"], tensors[f"{p}self_attn.k_proj.weight"],
                            tensors[f"{p}self_attn.v_proj.weight"]), dim=0).contiguous(),
        o_proj=tensors[f"{p}self_attn.o_proj.weight"],
        q_norm=tensors[f"{p}self_attn.q_norm.weight"],
        k_norm=tensors[f"{p}self_attn.k_norm.weight"],
        post_attention_layernorm=tensors[f"{p}post_attention_layernorm.weight"],
        gate_up_proj=torch.cat((tensors[f"{p}mlp.gate_proj.weight"], tensors[f"{p}mlp.up_proj.weight"]),
                               dim=0).contiguous(),
        down_proj=tensors[f"{p}mlp.down_proj.weight"],
    )


def qkv_project(xn: torch.Tensor, w: LayerWeights, hq: int, hkv: int, d: int, cos, sin, eps: float):
    """Fused QKV projection, per-head q/k RMSNorm, RoPE (``qwen_explicit.py:733-770``).

    ``xn`` is the normed hidden ``[B, Q, H]``; returns q ``[B, Hq, Q, D]`` and
    k, v ``[B, Hkv, Q, D]``.
    """
    b, q_len, _ = xn.shape
    qkv = F.linear(xn, w.qkv_proj.to(xn.dtype))
    q, k, v = torch.split(qkv, (hq * d, hkv * d, hkv * d), dim=-1)
    q = rmsnorm(q.reshape(b, q_len, hq, d), w.q_norm, eps).transpose(1, 2)
    k = rmsnorm(k.reshape(b, q_len, hkv, d), w.k_norm, eps).transpose(1, 2)
    v = v.reshape(b, q_len, hkv, d).transpose(1, 2)
    return apply_rope(q, cos, sin), apply_rope(k, cos, sin), v


def decode_mask(query_len: int, total_len: int, dtype: torch.dtype, device="cpu") -> torch.Tensor:
    """Additive mask: key j visible to query i iff ``j <= past + i`` (``qwen_explicit.py:551-563``)."""
    past = total_len - query_len
    qpos = torch.arange(query_len, device=device).unsqueeze(1)
    kpos = torch.arange(total_len, device=device).unsqueeze(0)
    mask = torch.zeros((query_len, total_len), dtype=dtype, device=device)
    mask = mask.masked_fill(~(kpos <= past + qpos), torch.finfo(dtype).min)
    return mask[None, None]


def sdpa(*args, **kwargs) -> torch.Tensor:
    """``F.scaled_dot_product_attention``, the reference's attention op.

    Every attention of the oracle goes through this name, so a measurement
    script can wrap it (``tests/golden/make_stream_paths.py`` perturbs its
    output by one ulp in a few elements to measure how sensitive a greedy
    stream is to such noise).
    """
    return F.scaled_dot_product_attention(*args, **kwargs)


def attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, mask, scale: float) -> torch.Tensor:
    """GQA scaled-dot-product attention (``qwen_explicit.py:1000-1039``).

    Decode (Q == 1) runs unmasked; Q == S runs causal; otherwise the additive
    ``mask`` applies.  Returns ``[B, Q, Hq*D]``.
    """
    q_len, kv_len = q.shape[-2], k.shape[-2]
    is_decode = q_len == 1 and kv_len >= 1
    causal = (not is_decode) and q_len == kv_len
    out = sdpa(
        q, k, v,
        attn_mask=None if (causal or is_decode) else mask,
        dropout_p=0.0, is_causal=causal, scale=scale, enable_gqa=True,
    )
    b = q.shape[0]
    return out.transpose(1, 2).reshape(b, q_len, -1)


def post_attention_mlp(attn: torch.Tensor, residual: torch.Tensor, w: LayerWeights, eps: float) -> torch.Tensor:
    """o_proj + residual, post-norm, gate_up, SiLU*up, down + residual (``qwen_explicit.py:809-852``)."""
    dt = attn.dtype
    h = residual + F.linear(attn, w.o_proj.to(dt))
    n = rmsnorm(h, w.post_attention_layernorm, eps)
    gu = F.linear(n, w.gate_up_proj.to(dt))
    inter = w.gate_up_proj.shape[0] // 2
    g, u = torch.split(gu, (inter, inter), dim=-1)
    return h + F.linear(F.silu(g) * u, w.down_proj.to(dt))


# ---------------------------------------------------------------------------
# Static KV cache (kv_cache.py:207-318), generalised to per-sequence cursors
# ---------------------------------------------------------------------------

@dataclass
class OracleKV:
    """``[L, B, Hkv, S_max, D]`` K and V arenas with per-layer cursors.

    Mirrors ``StaticKVBlockManager`` (``kv_cache.py:207-318``): ``append``
    writes at the layer's cursor and ``get`` returns the live prefix.
    """

    key_cache: torch.Tensor
    value_cache: torch.Tensor
    layer_seq_lens: list[int] = field(default_factory=list)

    @classmethod
    def empty(cls, layers: int, batch: int, hkv: int, max_seq: int, d: int, dtype, device="cpu") -> "OracleKV":
        shape = (layers, batch, hkv, max_seq, d)
        return cls(torch.zeros(shape, dtype=dtype, device=device), torch.zeros(shape, dtype=dtype, device=device),
                   [0] * layers)

    def append(self, layer: int, k: torch.Tensor, v: torch.Tensor) -> None:
        start = self.layer_seq_lens[layer]
        end = start + k.shape[2]
        if end > self.key_cache.shape[3]:
            raise ValueError(f"cache overflow for layer {layer}: requested {end} tokens")
        self.key_cache[layer, :, :, start:end] = k
        self.value_cache[layer, :, :, start:end] = v
        self.layer_seq_lens[layer] = end

    def get(self, layer: int):
        n = self.layer_seq_lens[layer]
        return self.key_cache[layer, :, :, :n], self.value_cache[layer, :, :, :n]

    def seq_len(self) -> int:
        return max(self.layer_seq_lens, default=0)

    def set_all(self, n: int) -> None:
        self.layer_seq_lens = [int(n)] * len(self.layer_seq_lens)


# ---------------------------------------------------------------------------
# Layer and stack drivers
# ---------------------------------------------------------------------------

@dataclass
class OracleModel:
    """A materialized stack in oracle form (fields follow ``QwenSemanticStackRuntime``,
    ``qwen_explicit.py:132-145``)."""

    hidden_size: int
    num_attention_heads: int
    num_key_value_heads: int
    head_dim: int
    intermediate_size: int
    rms_norm_eps: float
    rope_theta: float
    embed_tokens: torch.Tensor
    layers: list[LayerWeights]
    final_norm: torch.Tensor
    lm_head: torch.Tensor
    precision: str = "bf16"

    @property
    def dtype(self) -> torch.dtype:
        return _dt(self.precision)

    @classmethod
    def from_checkpoint(cls, geometry, tensors: dict[str, torch.Tensor], precision: str = "bf16",
                        layer_indices=None) -> "OracleModel":
        dt = _dt(precision)
        idx = range(geometry.num_hidden_layers) if layer_indices is None else layer_indices
        embed = tensors["model.embed_tokens.weight"]
        lm = tensors.get("lm_head.weight", embed)
        return cls(
            hidden_size=geometry.hidden_size,
            num_attention_heads=geometry.num_attention_heads,
            num_key_value_heads=geometry.num_key_value_heads,
            head_dim=geometry.head_dim,
            intermediate_size=geometry.intermediate_size,
            rms_norm_eps=geometry.rms_norm_eps,
            rope_theta=geometry.rope_theta,
            embed_tokens=embed.to(dt),
            layers=[fuse_layer(tensors, i).to(dt) for i in idx],
            final_norm=tensors["model.norm.weight"].to(dt),
            lm_head=lm.to(dt),
            precision=precision,
        )

    @property
    def device(self) -> torch.device:
        return self.embed_tokens.device

    def new_kv(self, batch: int, max_seq: int) -> OracleKV:
        return OracleKV.empty(len(self.layers), batch, self.num_key_value_heads, max_seq, self.head_dim, self.dtype,
                              self.device)

    def rope(self, max_seq: int):
        """Position cache on the model's device (the reference builds it where the model lives)."""
        return rope_cache(rope_inv_freq(self.head_dim, self.rope_theta).to(self.device), max_seq, self.dtype)


def layer_forward(m: OracleModel, layer_idx: int, w: LayerWeights, hidden: torch.Tensor, kv: OracleKV | None,
                  cos: torch.Tensor, sin: torch.Tensor, mask) -> torch.Tensor:
    """One decoder layer, general path (``qwen_explicit.py:1211-1244`` with ``:1093-1144``).

    The bs1 vector path (``:1247-1272``) performs the same roundings, so it is
    not restated separately.
    """
    eps = m.rms_norm_eps
    residual = hidden
    xn = rmsnorm(hidden, w.input_layernorm, eps)
    q, k, v = qkv_project(xn, w, m.num_attention_heads, m.num_key_value_heads, m.head_dim, cos, sin, eps)
    if kv is not None:
        kv.append(layer_idx, k, v)
        k, v = kv.get(layer_idx)
    attn = attention(q, k, v, mask, m.head_dim ** -0.5)
    return post_attention_mlp(attn, residual, w, eps)


def stack_forward(m: OracleModel, hidden: torch.Tensor, kv: OracleKV, position_cache) -> torch.Tensor:
    """Run all layers over ``hidden [B, Q, H]`` at the cache's current cursor.

    Covers prefill (``run_semantic_stack_prefill``, ``qwen_explicit.py:1455-1491``:
    empty cache, causal), decode (``:1617-1644``, Q == 1) and verify
    (``:1676-1717``: Q > 1 over a non-empty cache with the decode mask).
    """
    q_len = hidden.shape[1]
    past = kv.seq_len()
    cos_c, sin_c = position_cache
    cos = cos_c[past:past + q_len].unsqueeze(0)
    sin = sin_c[past:past + q_len].unsqueeze(0)
    mask = decode_mask(q_len, past + q_len, m.dtype, hidden.device) if (q_len > 1 and past > 0) else None
    for i, w in enumerate(m.layers):
        hidden = layer_forward(m, i, w, hidden, kv, cos, sin, mask)
    return hidden


def decode_layer_vector(m: OracleModel, layer_idx: int, w: LayerWeights, hidden: torch.Tensor, kv: OracleKV,
                        cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """One layer of the bs1 decode path (``semantic_qwen_decode_layer_forward``,
    ``qwen_explicit.py:1247-1272``, with ``:1147-1177``, ``:773-806``, ``:886-913``,
    ``:932-949``).

    Same rounding points as :func:`layer_forward`, but every linear is a
    ``torch.mv`` on a flat vector, the form the reference's decode driver runs.
    On the CPU ``mv`` and ``F.linear`` reach different bf16 kernels whose fp32
    sums differ in order, so the two paths are separate restatements.
    """
    eps = m.rms_norm_eps
    hq, hkv, d = m.num_attention_heads, m.num_key_value_heads, m.head_dim
    residual = hidden.reshape(-1)
    xn = rmsnorm(residual.view(1, -1), w.input_layernorm, eps).view(-1)
    qkv = torch.mv(w.qkv_proj, xn)
    q, k, v = torch.split(qkv, (hq * d, hkv * d, hkv * d), dim=0)
    q = rmsnorm(q.view(1, hq, d), w.q_norm, eps).view(1, hq, 1, d)
    k = rmsnorm(k.view(1, hkv, d), w.k_norm, eps).view(1, hkv, 1, d)
    v = v.view(1, hkv, 1, d)
    q, k = apply_rope(q, cos, sin), apply_rope(k, cos, sin)
    kv.append(layer_idx, k, v)
    keys, values = kv.get(layer_idx)
    attn = sdpa(q, keys, values, dropout_p=0.0, is_causal=False, scale=d ** -0.5, enable_gqa=hq != hkv)
    h = residual + torch.mv(w.o_proj, attn.reshape(-1))
    n = rmsnorm(h.view(1, -1), w.post_attention_layernorm, eps).view(-1)
    gu = torch.mv(w.gate_up_proj, n)
    g, u = torch.split(gu, (m.intermediate_size, gu.shape[0] - m.intermediate_size), dim=0)
    return (h + torch.mv(w.down_proj, F.silu(g) * u)).view(1, 1, -1)


def decode_step_vector(m: OracleModel, ids: torch.Tensor, kv: OracleKV, position_cache) -> torch.Tensor:
    """``run_semantic_stack_decode`` for one sequence and one token (``qwen_explicit.py:1617-1644``)."""
    past = kv.seq_len()
    cos_c, sin_c = position_cache
    cos, sin = cos_c[past:past + 1].unsqueeze(0), sin_c[past:past + 1].unsqueeze(0)
    hidden = embed(m, ids.view(1, 1).to(m.device))
    for i, w in enumerate(m.layers):
        hidden = decode_layer_vector(m, i, w, hidden, kv, cos, sin)
    return hidden


def greedy_logits_vector(m: OracleModel, hidden: torch.Tensor) -> torch.Tensor:
    """The bs1 torch head: ``mv(lm_head, rmsnorm(last))`` (``qwen_explicit.py:952-960``, ``:1814-1832``)."""
    last = hidden[0, -1]
    n = rmsnorm(last.view(1, -1), m.final_norm, m.rms_norm_eps).view(-1)
    return torch.mv(m.lm_head, n)


def embed(m: OracleModel, ids: torch.Tensor) -> torch.Tensor:
    return F.embedding(ids, m.embed_tokens)


def greedy_logits(m: OracleModel, hidden_last: torch.Tensor) -> torch.Tensor:
    """Final RMSNorm + lm_head logits of the last position (``qwen_explicit.py:952-960``)."""
    n = rmsnorm(hidden_last, m.final_norm, m.rms_norm_eps)
    return F.linear(n, m.lm_head)


def greedy_token(m: OracleModel, hidden: torch.Tensor) -> torch.Tensor:
    """Torch greedy head: argmax of (bf16) logits, lowest index on ties.

    ``hidden`` is ``[B, Q, H]``; the last position of each sequence is used
    (``qwen_explicit.py:1814-1832`` with ``LEANSTACK_SEMANTIC_LOGITS_BACKEND=torch``).
    Returns ``[B]`` int64.
    """
    logits = greedy_logits(m, hidden[:, -1, :])
    return logits.argmax(dim=-1)


def top2_margin(m: OracleModel, hidden: torch.Tensor) -> list[float]:
    """Gap between the best and second-best logit per sequence (fp32 of the logits)."""
    logits = greedy_logits(m, hidden[:, -1, :]).float()
    top = logits.topk(2, dim=-1).values
    return (top[:, 0] - top[:, 1]).tolist()


def greedy_generate(m: OracleModel, prompt_ids: torch.Tensor, new_tokens: int, max_seq: int,
                    with_margins: bool = False):
    """Prefill then ``new_tokens`` greedy steps (``runtime_loop.py:264-352``).

    The first token comes from the prefill's last position; every further
    token from one decode step.  Returns ``(tokens [B, new_tokens], margins)``.
    """
    b = prompt_ids.shape[0]
    kv = m.new_kv(b, max_seq)
    pc = m.rope(max_seq)
    hidden = stack_forward(m, embed(m, prompt_ids), kv, pc)
    tokens, margins = [], []
    tok = greedy_token(m, hidden)
    for step in range(new_tokens):
        tokens.append(tok)
        if with_margins:
            margins.append(top2_margin(m, hidden))
        if step == new_tokens - 1:
            break
        hidden = stack_forward(m, embed(m, tok.view(b, 1)), kv, pc)
        tok = greedy_token(m, hidden)
    return torch.stack(tokens, dim=1), margins


# ---------------------------------------------------------------------------
# Dual-model speculative decode (runtime_loop.py:651-916), batch 1
# ---------------------------------------------------------------------------

def dual_model_speculative(draft: OracleModel, target: OracleModel, prompt_ids: torch.Tensor,
                           max_new_tokens: int, proposal_len: int, max_seq: int | None = None):
    """Greedy-exact draft/verify loop for one sequence (``runtime_loop.py:651-916``).

    Each cycle: the draft consumes the current token and proposes
    ``k`` tokens greedily; the target verifies ``[current, d1..dk]`` in one
    pass; the longest agreeing prefix is accepted, the first disagreement is
    replaced by the target's token (or a bonus token is appended when all
    agree); both caches roll back to ``base + 1 + accepted``.
    Returns ``(generated ids, stats)``.
    """
    assert prompt_ids.shape[0] == 1
    max_seq = max_seq or prompt_ids.shape[1] + max_new_tokens + proposal_len + 1
    dkv, tkv = draft.new_kv(1, max_seq), target.new_kv(1, max_seq)
    dpc, tpc = draft.rope(max_seq), target.rope(max_seq)
    stack_forward(draft, embed(draft, prompt_ids), dkv, dpc)
    th = stack_forward(target, embed(target, prompt_ids), tkv, tpc)
    current = int(greedy_token(target, th)[0])
    generated: list[int] = []
    stats = {"cycles": 0, "proposed": 0, "accepted": 0, "bonus": 0}
    while len(generated) < max_new_tokens:
        stats["cycles"] += 1
        k = min(proposal_len, max_new_tokens - len(generated))
        dbase, tbase = dkv.seq_len(), tkv.seq_len()
        proposals: list[int] = []
        tok = current
        for _ in range(k):
            dh = stack_forward(draft, embed(draft, torch.tensor([[tok]])), dkv, dpc)
            tok = int(greedy_token(draft, dh)[0])
            proposals.append(tok)
        stats["proposed"] += len(proposals)
        ids = torch.tensor([[current] + proposals])
        vh = stack_forward(target, embed(target, ids), tkv, tpc)
        # one head call per position, as runtime_loop.py:805-812 does
        verdict = [int(greedy_token(target, vh[:, pos:pos + 1, :])[0]) for pos in range(vh.shape[1])]
        committed: list[int] = []
        accepted = 0
        mismatch = False
        for i, p in enumerate(proposals):
            if p != verdict[i]:
                mismatch = True
                committed.append(verdict[i])
                dkv.set_all(dbase + 1 + i)
                tkv.set_all(tbase + 1 + i)
                current = verdict[i]
                break
            committed.append(p)
            accepted += 1
        stats["accepted"] += accepted
        if not mismatch:
            bonus = verdict[len(proposals)]
            if len(generated) + len(committed) < max_new_tokens:
                committed.append(bonus)
                stats["bonus"] += 1
            current = bonus
        for t in committed:
            if len(generated) >= max_new_tokens:
                break
            generated.append(int(t))
    return generated, stats
