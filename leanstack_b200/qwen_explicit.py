"""Drop-in for the reference's semantic runtime dispatch (``qwen_explicit.py``).

Same dataclasses, helper names, argument meanings and return shapes as the
reference's kernel-dispatch surface (``src/leanstack/runtime/qwen_explicit.py``:
dataclasses ``:79-145``, dispatch table ``:963-971``, layer forwards
``:1211-1272``, stack drivers ``:1455-1738``, greedy head ``:1814-1832``), so
the leanserve materializer and the request / speculative loops drive it
unchanged.  Every numeric op runs in libleanb200.so on the current CUDA
stream; there is no CPU path (a CPU tensor raises).

Differences from the reference, all deliberate:
* no ``torch.compile`` wrapper and no silent fallback (reference ``:578-604``,
  ``:1821-1826``): a kernel error raises;
* the decode layer fuses the input RMSNorm into the QKV projection, the
  residual add into o_proj / down, and appends K/V from inside the QKV kernel;
  rounding points are the reference's;
* the general (B x Q) path runs all B * Q tokens of a layer at once and picks
  the linear kernel by token count m: the CUDA-core streaming kernels with the
  norm fused in for m <= 8, the tcgen05 weight-streaming GEMM for m <= 128 and
  the persistent large-M tcgen05 GEMM above (prefill); attention applies the
  reference's causal / decode-mask visibility from the cache cursor and moves
  to the tcgen05 prefill kernel at 256 query rows per kv head.  These are the
  kernels and call order of ``DecodeEngine``'s steps, so both give the same
  bits.
"""

from __future__ import annotations

import os
from dataclasses import dataclass
from pathlib import Path
from typing import Any

import torch

from . import kernels as K
from .kv_cache import KVPageLayout, StaticKVBlockManager

SMALL_M = 8      # largest token count of one CUDA-core linear launch
TC_MAX_M = 128   # largest token count of one weight-streaming tcgen05 GEMM launch


@dataclass
class QwenSemanticAttentionRuntime:
    layer_idx: int
    q_proj_weight: torch.Tensor
    k_proj_weight: torch.Tensor
    v_proj_weight: torch.Tensor
    qkv_proj_weight: torch.Tensor
    q_proj_out_dim: int
    k_proj_out_dim: int
    num_attention_heads: int
    num_key_value_heads: int
    num_key_value_groups: int
    head_dim: int
    attention_scale: float
    o_proj_weight: torch.Tensor
    q_norm_weight: torch.Tensor
    k_norm_weight: torch.Tensor


@dataclass
class QwenSemanticMlpRuntime:
    gate_proj_weight: torch.Tensor
    up_proj_weight: torch.Tensor
    gate_up_proj_weight: torch.Tensor
    gate_proj_out_dim: int
    down_proj_weight: torch.Tensor


@dataclass
class QwenSemanticLayerRuntime:
    layer_idx: int
    input_layernorm_weight: torch.Tensor
    attention: QwenSemanticAttentionRuntime
    post_attention_layernorm_weight: torch.Tensor
    mlp: QwenSemanticMlpRuntime


@dataclass
class QwenSemanticStackRuntime:
    model_path: Path
    config: Any
    layer_indices: tuple[int, ...]
    embed_tokens_weight: torch.Tensor
    layers: tuple[QwenSemanticLayerRuntime, ...]
    rope_inv_freq: torch.Tensor
    attention_scaling: float
    final_norm_weight: torch.Tensor | None
    lm_head_weight: torch.Tensor | None
    device: torch.device
    dtype: torch.dtype


KVCacheManager = StaticKVBlockManager


def normalize_stop_token_ids(stop_token_ids) -> tuple[int, ...]:
    """Stop ids as a tuple of ints: None -> (), one int -> (id,) (``qwen_explicit.py:1868-1873``)."""
    if stop_token_ids is None:
        return ()
    if isinstance(stop_token_ids, int):
        return (int(stop_token_ids),)
    return tuple(int(t) for t in stop_token_ids)


def resolve_semantic_logits_backend() -> str:
    """Kept for interface parity (``qwen_explicit.py:150-151``); every value selects the native head."""
    return os.environ.get("LEANSTACK_SEMANTIC_LOGITS_BACKEND", "auto").strip().lower()


# ---------------------------------------------------------------------------
# Position cache (host arithmetic, identical to the reference's, then resident)
# ---------------------------------------------------------------------------

def build_qwen_position_cache(rope_inv_freq: torch.Tensor, attention_scaling: float, max_seq_len: int,
                              dtype: torch.dtype) -> tuple[torch.Tensor, torch.Tensor]:
    """bf16 cos/sin table ``[max_seq_len, D/2]`` (``qwen_explicit.py:664-676``).

    Angles and cos/sin are computed on the CPU in fp32 exactly as the reference
    does, then copied to the inverse-frequency tensor's device.
    """
    if max_seq_len <= 0:
        raise ValueError("max_seq_len must be positive")
    inv = rope_inv_freq.detach().to("cpu", torch.float32)
    pos = torch.arange(max_seq_len, dtype=torch.float32)
    freqs = torch.outer(pos, inv)
    cos = (freqs.cos() * attention_scaling).to(dtype)
    sin = (freqs.sin() * attention_scaling).to(dtype)
    return cos.to(rope_inv_freq.device), sin.to(rope_inv_freq.device)


def slice_qwen_position_embeddings(position_cache, start: int, length: int):
    if length <= 0:
        raise ValueError("length must be positive")
    cos_cache, sin_cache = position_cache
    return cos_cache.narrow(0, start, length).unsqueeze(0), sin_cache.narrow(0, start, length).unsqueeze(0)


def build_decode_attention_mask(query_len: int, total_len: int, device, dtype) -> torch.Tensor:
    """The reference's additive verify mask (``qwen_explicit.py:551-563``).

    The native attention applies the same rule (key j visible to query i iff
    j <= past + i) from the cursors, so the mask is only built for callers that
    inspect it.
    """
    past_len = total_len - query_len
    q = torch.arange(query_len, device=device).unsqueeze(1)
    k = torch.arange(total_len, device=device).unsqueeze(0)
    mask = torch.zeros((query_len, total_len), device=device, dtype=dtype)
    return mask.masked_fill(~(k <= past_len + q), torch.finfo(dtype).min).unsqueeze(0).unsqueeze(0)


def build_qwen_kv_cache(config, max_seq_len: int, device, dtype, page_size: int = 16, batch_size: int = 1,
                        cache_kind: str = "auto") -> StaticKVBlockManager:
    """Static cache factory (``qwen_explicit.py:1066-1090``).  Only the static kind exists here."""
    if cache_kind not in {"auto", "static"}:
        raise ValueError(f"unsupported cache_kind: {cache_kind} (the paged cache is out of scope)")
    head_dim = getattr(config, "head_dim", config.hidden_size // config.num_attention_heads)
    layout = KVPageLayout(num_layers=config.num_hidden_layers, num_key_value_heads=config.num_key_value_heads,
                          head_dim=head_dim, page_size=page_size, max_seq_len=max_seq_len, batch_size=batch_size,
                          dtype=dtype, device=torch.device(device))
    return StaticKVBlockManager(layout)


def _cos_sin_table(cos: torch.Tensor, sin: torch.Tensor):
    """Flatten a ``[1, Q, D/2]`` position slice into a ``[Q, D/2]`` table."""
    half = cos.shape[-1]
    return cos.reshape(-1, half).contiguous(), sin.reshape(-1, half).contiguous()


# ---------------------------------------------------------------------------
# Dispatch helpers (the reference's table at qwen_explicit.py:963-971)
# ---------------------------------------------------------------------------

def qwen_rmsnorm(hidden_states: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    return K.rmsnorm(hidden_states.contiguous(), weight, eps)


def qwen_rmsnorm_vector(hidden_states: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    return qwen_rmsnorm(hidden_states.reshape(1, -1), weight, eps).view(-1)


def _linear_routed(x: torch.Tensor, w: torch.Tensor, *, norm_w: torch.Tensor | None = None, eps: float = 1e-6,
                   epilogue: int = K.EPI_STORE, residual: torch.Tensor | None = None) -> torch.Tensor:
    """``epilogue(w @ rmsnorm?(x))`` for x ``[m, k]``, on the kernel family for m.

    m <= 8: CUDA-core streaming linear with the RMSNorm in its prologue;
    m <= 128: RMSNorm kernel, then the tcgen05 weight-streaming GEMM in the
    split-partial form with the engine's consumers (residual add, SiLU*up
    combine; the q/k norm takes the QKV partials in ``_qkv``), giving the
    engine's bits;
    larger: RMSNorm kernel, then the persistent large-M tcgen05 GEMM.
    """
    m = x.shape[0]
    if m <= SMALL_M:
        return K.linear(x, w, norm_w=norm_w, eps=eps, epilogue=epilogue, residual=residual)
    xn = K.rmsnorm(x, norm_w, eps) if norm_w is not None else x
    if m <= TC_MAX_M:
        if epilogue == K.EPI_RESIDUAL:  # split partials + residual consumer, the engine's kernels
            part = torch.empty(K.gemm_splits(m, w.shape[1], w.shape[0]) * m * w.shape[0], device=x.device,
                               dtype=torch.float32)
            s = K.gemm_tc_splits(xn, w, part)
            out = torch.empty(m, w.shape[0], device=x.device, dtype=x.dtype)
            K.residual_rmsnorm_splits(part, s, residual, out_residual=out)
            return out
        if epilogue == K.EPI_SILU_MUL and K.gate_up_plain(m, w.shape[1], w.shape[0]):
            part = torch.empty(K.gemm_splits(m, w.shape[1], w.shape[0]) * m * w.shape[0], device=x.device,
                               dtype=torch.float32)
            s = K.gemm_tc_splits(xn, w, part)
            act = torch.empty(m, w.shape[0] // 2, device=x.device, dtype=x.dtype)
            K.silu_mul_splits(part, s, m, w.shape[0] // 2, out=act)
            return act
        return K.gemm_tc(xn, w, epilogue=epilogue, residual=residual)
    return K.gemm_big(xn, w, epilogue=epilogue, residual=residual)


def _qkv(hidden: torch.Tensor, batch: int, q_len: int, qkv_w, hq, hkv, d, qn, kn, cos, sin, eps, input_norm=None,
         kv: StaticKVBlockManager | None = None, layer_idx: int = 0, past: int = 0):
    cos_t, sin_t = _cos_sin_table(cos, sin)
    m = batch * q_len
    x = hidden.reshape(m, -1).contiguous()
    if SMALL_M < m <= TC_MAX_M:  # the engine's kernels: QKV split partials summed by the q/k norm
        xn = K.rmsnorm(x, input_norm, eps) if input_norm is not None else x
        part = torch.empty(K.gemm_splits(m, x.shape[1], qkv_w.shape[0]) * m * qkv_w.shape[0], device=x.device,
                           dtype=torch.float32)
        s = K.gemm_tc_splits(xn, qkv_w, part)
        if kv is not None:
            q = K.qk_norm_rope_splits(part, s, batch, q_len, hq, hkv, d, qn, kn, cos_t, sin_t, eps=eps,
                                      uniform_past=past, rope_offset=past, k_cache=kv.key_cache[layer_idx],
                                      v_cache=kv.value_cache[layer_idx], max_seq=kv.layout.max_seq_len,
                                      q_out=torch.empty((m, hq, d), device=x.device, dtype=x.dtype))
            return q, None, None
        k_out = torch.empty((m, hkv, d), device=x.device, dtype=x.dtype)
        v_out = torch.empty((m, hkv, d), device=x.device, dtype=x.dtype)
        q = K.qk_norm_rope_splits(part, s, batch, q_len, hq, hkv, d, qn, kn, cos_t, sin_t, eps=eps, k_out=k_out,
                                  v_out=v_out, q_out=torch.empty((m, hq, d), device=x.device, dtype=x.dtype))
        return q, k_out, v_out
    if m > SMALL_M:
        qkv = _linear_routed(x, qkv_w, norm_w=input_norm, eps=eps)
        if kv is not None:
            q = K.qk_norm_rope(qkv, batch, q_len, hq, hkv, d, qn, kn, cos_t, sin_t, eps=eps, uniform_past=past,
                               rope_offset=past, k_cache=kv.key_cache[layer_idx], v_cache=kv.value_cache[layer_idx],
                               max_seq=kv.layout.max_seq_len)
            return q, None, None
        k_out = torch.empty((m, hkv, d), device=x.device, dtype=x.dtype)
        v_out = torch.empty((m, hkv, d), device=x.device, dtype=x.dtype)
        q = K.qk_norm_rope(qkv, batch, q_len, hq, hkv, d, qn, kn, cos_t, sin_t, eps=eps, k_out=k_out, v_out=v_out)
        return q, k_out, v_out
    if kv is not None:
        q = K.qkv_rope_append(x, batch, q_len, qkv_w, hq, hkv, d, qn, kn, cos_t, sin_t, input_norm_w=input_norm,
                              eps=eps, uniform_past=past, rope_offset=past, k_cache=kv.key_cache[layer_idx],
                              v_cache=kv.value_cache[layer_idx], max_seq=kv.layout.max_seq_len)
        return q, None, None
    k_out = torch.empty((m, hkv, d), device=x.device, dtype=x.dtype)
    v_out = torch.empty((m, hkv, d), device=x.device, dtype=x.dtype)
    q = K.qkv_rope_append(x, batch, q_len, qkv_w, hq, hkv, d, qn, kn, cos_t, sin_t, input_norm_w=input_norm,
                          eps=eps, k_out=k_out, v_out=v_out)
    return q, k_out, v_out


def _semantic_attention_qkv_vector(hidden_states, qkv_proj_weight, q_proj_out_dim, k_proj_out_dim,
                                   num_attention_heads, num_key_value_heads, head_dim, q_norm_weight, k_norm_weight,
                                   cos, sin, rms_norm_eps):
    """bs1 fused QKV + q/k norm + RoPE (``qwen_explicit.py:773-806``) -> q [1,Hq,1,D], k, v [1,Hkv,1,D]."""
    q, k, v = _qkv(hidden_states, 1, 1, qkv_proj_weight, num_attention_heads, num_key_value_heads, head_dim,
                   q_norm_weight, k_norm_weight, cos, sin, rms_norm_eps)
    return (q.view(1, num_attention_heads, 1, head_dim), k.view(1, num_key_value_heads, 1, head_dim),
            v.view(1, num_key_value_heads, 1, head_dim))


def _semantic_attention_qkv(hidden_states, qkv_proj_weight, q_proj_out_dim, k_proj_out_dim, num_attention_heads,
                            num_key_value_heads, head_dim, q_norm_weight, k_norm_weight, cos, sin, rms_norm_eps):
    """General fused QKV (``qwen_explicit.py:733-770``) -> q [B,Hq,Q,D], k, v [B,Hkv,Q,D]."""
    b, q_len, _ = hidden_states.shape
    q, k, v = _qkv(hidden_states, b, q_len, qkv_proj_weight, num_attention_heads, num_key_value_heads, head_dim,
                   q_norm_weight, k_norm_weight, cos, sin, rms_norm_eps)
    return (q.view(b, q_len, num_attention_heads, head_dim).transpose(1, 2),
            k.view(b, q_len, num_key_value_heads, head_dim).transpose(1, 2),
            v.view(b, q_len, num_key_value_heads, head_dim).transpose(1, 2))


def _attend(q_bhqd: torch.Tensor, key_states: torch.Tensor, value_states: torch.Tensor, scale: float) -> torch.Tensor:
    """Attention of q ``[B, Hq, Q, D]`` over ``[B, Hkv, S, D]`` keys with the causal-suffix rule."""
    b, hq, q_len, d = q_bhqd.shape
    hkv, seq = key_states.shape[1], key_states.shape[2]
    if key_states.stride(3) != 1 or key_states.stride(2) != d or key_states.stride(1) % d:
        raise ValueError("key/value views must be [B, Hkv, S, D] slices with contiguous rows")
    if value_states.stride() != key_states.stride():
        raise ValueError("key and value views must share a layout")
    max_seq = key_states.stride(1) // d
    if key_states.stride(0) != hkv * max_seq * d:
        raise ValueError("batch stride of the key view must be Hkv * max_seq * D")
    q = q_bhqd.transpose(1, 2).contiguous()
    return K.decode_attention(q, key_states, value_states, b, q_len, hq, hkv, d, max_seq, scale,
                              uniform_past=seq - q_len)


def _semantic_decode_attention_output_vector(query_states, key_states, value_states, o_proj_weight,
                                             attention_scale, num_key_value_groups):
    """bs1 SDPA + o_proj (``qwen_explicit.py:886-913``) -> [H]."""
    attn = _attend(query_states, key_states, value_states, attention_scale)
    return K.linear(attn, o_proj_weight).view(-1)


def _semantic_decode_attention_output(query_states, key_states, value_states, o_proj_weight, attention_scale,
                                      num_key_value_groups):
    """General SDPA + o_proj (``qwen_explicit.py:855-883``) -> [B, Q, H]."""
    b, _, q_len, _ = query_states.shape
    attn = _attend(query_states, key_states, value_states, attention_scale)
    return _linear_routed(attn, o_proj_weight).view(b, q_len, -1)


def sdpa_qwen_attention_forward(query_states, key_states, value_states, attention_mask, scaling,
                                num_key_value_groups):
    """GQA attention (``qwen_explicit.py:1000-1039``) -> [B, Q, Hq, D].

    The mask argument is accepted for interface parity; visibility comes from
    the rule key j <= (S - Q) + i, which is what the reference's decode mask
    and causal prefill both encode.
    """
    b, hq, q_len, d = query_states.shape
    attn = _attend(query_states, key_states, value_states, scaling)
    return attn.view(b, q_len, hq, d)


def _semantic_mlp_epilogue_vector(hidden_states, post_attention_layernorm_weight, gate_up_proj_weight,
                                  gate_proj_out_dim, down_proj_weight, rms_norm_eps):
    """``r + down(silu(g) * u)`` of the normed h (``qwen_explicit.py:932-949``) -> [H]."""
    h = hidden_states.reshape(1, -1).contiguous()
    act = K.gateup_silu(h, post_attention_layernorm_weight, gate_up_proj_weight, rms_norm_eps)
    return K.down_residual(act, down_proj_weight, h).view(-1)


def _semantic_mlp_epilogue(hidden_states, post_attention_layernorm_weight, gate_up_proj_weight, gate_proj_out_dim,
                           down_proj_weight, rms_norm_eps):
    shape = hidden_states.shape
    h = hidden_states.reshape(-1, shape[-1]).contiguous()
    act = _linear_routed(h, gate_up_proj_weight, norm_w=post_attention_layernorm_weight, eps=rms_norm_eps,
                         epilogue=K.EPI_SILU_MUL)
    return _linear_routed(act, down_proj_weight, epilogue=K.EPI_RESIDUAL, residual=h).view(shape)


def _semantic_post_attention_mlp(attention_output, residual, o_proj_weight, post_attention_layernorm_weight,
                                 gate_up_proj_weight, gate_proj_out_dim, down_proj_weight, rms_norm_eps):
    """o_proj + residual, then the MLP epilogue (``qwen_explicit.py:809-852``)."""
    shape = residual.shape
    res = residual.reshape(-1, shape[-1]).contiguous()
    h = _linear_routed(attention_output.reshape(res.shape[0], -1).contiguous(), o_proj_weight,
                       epilogue=K.EPI_RESIDUAL, residual=res)
    act = _linear_routed(h, gate_up_proj_weight, norm_w=post_attention_layernorm_weight, eps=rms_norm_eps,
                         epilogue=K.EPI_SILU_MUL)
    return _linear_routed(act, down_proj_weight, epilogue=K.EPI_RESIDUAL, residual=h).view(shape)


def _semantic_greedy_head_vector(hidden_states, final_norm_weight, lm_head_weight, rms_norm_eps):
    """Final RMSNorm + lm_head + argmax (``qwen_explicit.py:952-960``) -> [1, 1] int64."""
    ids = K.lmhead_argmax(hidden_states.reshape(1, -1).contiguous(), final_norm_weight, lm_head_weight,
                          rms_norm_eps)
    return ids.view(1, 1)


# ---------------------------------------------------------------------------
# Layer forwards
# ---------------------------------------------------------------------------

def semantic_qwen_decode_layer_forward(layer: QwenSemanticLayerRuntime, hidden_states: torch.Tensor,
                                       kv_cache: StaticKVBlockManager, position_embeddings, rms_norm_eps: float):
    """One bs1 decode layer (``qwen_explicit.py:1247-1272``) with fused norm / append / residuals."""
    att, mlp = layer.attention, layer.mlp
    residual = hidden_states.reshape(1, -1).contiguous()
    cos, sin = position_embeddings
    past = kv_cache.reserve(att.layer_idx, 1)
    q, _, _ = _qkv(residual, 1, 1, att.qkv_proj_weight, att.num_attention_heads, att.num_key_value_heads,
                   att.head_dim, att.q_norm_weight, att.k_norm_weight, cos, sin, rms_norm_eps,
                   input_norm=layer.input_layernorm_weight, kv=kv_cache, layer_idx=att.layer_idx, past=past)
    kv_cache.advance_layer(att.layer_idx, 1)
    ks, vs = kv_cache.get(att.layer_idx)
    attn = _attend(q.view(1, 1, att.num_attention_heads, att.head_dim).transpose(1, 2), ks, vs,
                   att.attention_scale)
    h = K.oproj_residual(attn, att.o_proj_weight, residual)
    act = K.gateup_silu(h, layer.post_attention_layernorm_weight, mlp.gate_up_proj_weight, rms_norm_eps)
    return K.down_residual(act, mlp.down_proj_weight, h).view(1, 1, -1)


def semantic_qwen_layer_forward(config, layer: QwenSemanticLayerRuntime, rope_inv_freq, attention_scaling,
                                hidden_states: torch.Tensor, position_ids, attention_mask,
                                kv_cache: StaticKVBlockManager | None = None, position_embeddings=None):
    """General layer over ``[B, Q, H]`` (``qwen_explicit.py:1211-1244``).

    All B * Q tokens go through the layer together: the K/V of the Q new
    positions land at the layer cursor, and query i of each sequence attends
    every key up to its own position -- the reference's causal prefill and
    decode-mask visibility.  The linears run on the kernel family for
    m = B * Q (``_linear_routed``).
    """
    if kv_cache is None:
        raise ValueError("the native general path needs a KV cache (the reference's cache-less path is unused)")
    if position_embeddings is None:
        raise ValueError("position_embeddings are required")
    att, mlp = layer.attention, layer.mlp
    eps = config.rms_norm_eps
    b, q_len, hidden = hidden_states.shape
    cos_all, sin_all = position_embeddings
    residual = hidden_states.reshape(b * q_len, hidden).contiguous()
    past = kv_cache.reserve(att.layer_idx, q_len)
    q, _, _ = _qkv(residual, b, q_len, att.qkv_proj_weight, att.num_attention_heads, att.num_key_value_heads,
                   att.head_dim, att.q_norm_weight, att.k_norm_weight, cos_all, sin_all, eps,
                   input_norm=layer.input_layernorm_weight, kv=kv_cache, layer_idx=att.layer_idx, past=past)
    kv_cache.advance_layer(att.layer_idx, q_len)
    ks, vs = kv_cache.get(att.layer_idx)
    attn = _attend(q.view(b, q_len, att.num_attention_heads, att.head_dim).transpose(1, 2), ks, vs,
                   att.attention_scale)
    h = _linear_routed(attn, att.o_proj_weight, epilogue=K.EPI_RESIDUAL, residual=residual)
    act = _linear_routed(h, mlp.gate_up_proj_weight, norm_w=layer.post_attention_layernorm_weight, eps=eps,
                         epilogue=K.EPI_SILU_MUL)
    return _linear_routed(act, mlp.down_proj_weight, epilogue=K.EPI_RESIDUAL, residual=h).view(b, q_len, hidden)


# ---------------------------------------------------------------------------
# Stack drivers
# ---------------------------------------------------------------------------

def _embed(runtime: QwenSemanticStackRuntime, input_ids: torch.Tensor) -> torch.Tensor:
    ids = input_ids.to(runtime.device).contiguous()
    out = K.embed_gather(ids.view(-1), runtime.embed_tokens_weight)
    return out.view(*ids.shape, -1)


def _position_cache(runtime, position_cache, total_len):
    return position_cache or build_qwen_position_cache(runtime.rope_inv_freq, runtime.attention_scaling,
                                                       max_seq_len=total_len, dtype=runtime.dtype)


def run_semantic_stack_prefill_from_hidden(runtime: QwenSemanticStackRuntime, hidden_states: torch.Tensor,
                                           page_size: int = 16, max_seq_len: int | None = None,
                                           position_cache=None, kv_cache: StaticKVBlockManager | None = None):
    """Prefill (``qwen_explicit.py:1494-1521``).  ``kv_cache`` may be a resident arena to reuse."""
    b, seq_len, _ = hidden_states.shape
    if kv_cache is None:
        kv_cache = build_qwen_kv_cache(runtime.config, max_seq_len=max_seq_len or seq_len, device=runtime.device,
                                       dtype=runtime.dtype, page_size=page_size, batch_size=b)
    pc = _position_cache(runtime, position_cache, max_seq_len or seq_len)
    pos = slice_qwen_position_embeddings(pc, start=kv_cache.get_seq_length(), length=seq_len)
    for layer in runtime.layers:
        hidden_states = semantic_qwen_layer_forward(runtime.config, layer, runtime.rope_inv_freq,
                                                    runtime.attention_scaling, hidden_states, None, None, kv_cache,
                                                    pos)
    kv_cache.set_sequence_lens([kv_cache.get_seq_length()] * b)
    return hidden_states, kv_cache


def run_semantic_stack_prefill(runtime: QwenSemanticStackRuntime, input_ids: torch.Tensor, page_size: int = 16,
                               max_seq_len: int | None = None, position_cache=None,
                               kv_cache: StaticKVBlockManager | None = None):
    """Prefill from token ids (``qwen_explicit.py:1455-1491``)."""
    return run_semantic_stack_prefill_from_hidden(runtime, _embed(runtime, input_ids), page_size=page_size,
                                                  max_seq_len=max_seq_len, position_cache=position_cache,
                                                  kv_cache=kv_cache)


def run_semantic_stack_decode_from_hidden(runtime: QwenSemanticStackRuntime, hidden_states: torch.Tensor,
                                          kv_cache: StaticKVBlockManager, position_cache=None):
    """Decode one token per sequence (``qwen_explicit.py:1647-1673``)."""
    b, q_len, _ = hidden_states.shape
    past = kv_cache.get_seq_length()
    pc = _position_cache(runtime, position_cache, past + q_len)
    pos = slice_qwen_position_embeddings(pc, start=past, length=q_len)
    eps = runtime.config.rms_norm_eps
    if b == 1 and q_len == 1:
        for layer in runtime.layers:
            hidden_states = semantic_qwen_decode_layer_forward(layer, hidden_states, kv_cache, pos, eps)
    else:
        for layer in runtime.layers:
            hidden_states = semantic_qwen_layer_forward(runtime.config, layer, runtime.rope_inv_freq,
                                                        runtime.attention_scaling, hidden_states, None, None,
                                                        kv_cache, pos)
    kv_cache.set_sequence_lens([kv_cache.get_seq_length()] * kv_cache.layout.batch_size)
    return hidden_states, kv_cache


def run_semantic_stack_decode(runtime: QwenSemanticStackRuntime, input_ids: torch.Tensor,
                              kv_cache: StaticKVBlockManager, position_cache=None):
    """``run_semantic_stack_decode`` (``qwen_explicit.py:1617-1644``)."""
    return run_semantic_stack_decode_from_hidden(runtime, _embed(runtime, input_ids), kv_cache, position_cache)


def run_semantic_stack_verify_from_hidden(runtime: QwenSemanticStackRuntime, hidden_states: torch.Tensor,
                                          kv_cache: StaticKVBlockManager, position_cache=None):
    """Verify k+1 tokens in one pass (``qwen_explicit.py:1676-1717``)."""
    q_len = hidden_states.shape[1]
    if q_len <= 0:
        raise ValueError("verify path requires at least one token")
    return run_semantic_stack_decode_from_hidden(runtime, hidden_states, kv_cache, position_cache)


def run_semantic_stack_verify_tokens(runtime: QwenSemanticStackRuntime, input_ids: torch.Tensor,
                                     kv_cache: StaticKVBlockManager, position_cache=None):
    """``run_semantic_stack_verify_tokens`` (``qwen_explicit.py:1720-1738``)."""
    return run_semantic_stack_verify_from_hidden(runtime, _embed(runtime, input_ids), kv_cache, position_cache)


def last_hidden_vector(hidden_states: torch.Tensor) -> torch.Tensor:
    return hidden_states[:, -1, :].reshape(-1)


def select_semantic_greedy_token(runtime: QwenSemanticStackRuntime, hidden_states: torch.Tensor) -> torch.Tensor:
    """Greedy token of the last position (``qwen_explicit.py:1814-1832``) -> LongTensor [1, 1].

    bf16-rounded logits, lowest index on ties: the reference's torch head.
    """
    if runtime.final_norm_weight is None or runtime.lm_head_weight is None:
        raise ValueError("runtime does not include model.norm and lm_head")
    return _semantic_greedy_head_vector(last_hidden_vector(hidden_states).contiguous(), runtime.final_norm_weight,
                                        runtime.lm_head_weight, runtime.config.rms_norm_eps)


def select_semantic_greedy_tokens(runtime: QwenSemanticStackRuntime, hidden_states: torch.Tensor) -> torch.Tensor:
    """Greedy token of the last position of every sequence of a batch -> LongTensor [B]."""
    b = hidden_states.shape[0]
    rows = hidden_states[:, -1, :].contiguous()
    out = torch.empty((b,), device=rows.device, dtype=torch.int64)
    for s in range(0, b, SMALL_M):
        e = min(b, s + SMALL_M)
        K.lmhead_argmax(rows[s:e], runtime.final_norm_weight, runtime.lm_head_weight, runtime.config.rms_norm_eps,
                        out_ids=out[s:e])
    return out
