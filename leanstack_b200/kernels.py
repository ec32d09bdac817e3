"""Torch-tensor front end of the C ABI.

Each function takes CUDA tensors, checks dtype / device / layout, and enqueues
the kernel on torch's current stream.  Outputs are written into caller tensors
when given (the engine passes its resident arenas) and allocated otherwise (the
reference-style dispatch helpers return fresh tensors, as the reference does).
"""

from __future__ import annotations

import ctypes

import torch

from . import _native as nat
from ._native import EPI_RESIDUAL, EPI_SILU_MUL, EPI_SPLIT_F32, EPI_STORE, EPI_STORE_F32  # noqa: F401

BF16 = torch.bfloat16


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _check(t: torch.Tensor, name: str, dtype=BF16, contiguous: bool = True) -> None:
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"{name} must be a tensor")
    if t.device.type != "cuda":
        raise ValueError(f"{name} must be a CUDA tensor (got {t.device}); there is no CPU path")
    if t.dtype != dtype:
        raise TypeError(f"{name} must be {dtype}, got {t.dtype}")
    if contiguous and not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")


def sm_count() -> int:
    v = ctypes.c_int(0)
    nat.call("ls_sm_count", ctypes.byref(v))
    return v.value


def device_error(clear: bool = True) -> int:
    v = ctypes.c_int(0)
    nat.call("ls_get_device_error", ctypes.byref(v), int(clear))
    return v.value


def set_wait_limit_ns(ns: int) -> None:
    """Limit of every bounded device wait on the current device (default 2 s)."""
    nat.call("ls_set_wait_limit_ns", int(ns))


def wait_limit_ns() -> int:
    v = ctypes.c_int64(0)
    nat.call("ls_get_wait_limit_ns", ctypes.byref(v))
    return v.value


def embed_gather(ids: torch.Tensor, embed: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    _check(ids, "ids", torch.int64)
    _check(embed, "embed")
    m = ids.numel()
    if out is None:
        out = torch.empty((m, embed.shape[1]), device=embed.device, dtype=BF16)
    nat.call("ls_embed_gather", ids.data_ptr(), m, embed.data_ptr(), embed.shape[0], embed.shape[1],
             out.data_ptr(), _stream())
    return out


def rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float, out: torch.Tensor | None = None) -> torch.Tensor:
    _check(x, "x")
    _check(w, "w")
    n = x.shape[-1]
    m = x.numel() // n
    if out is None:
        out = torch.empty_like(x)
    nat.call("ls_rmsnorm", x.data_ptr(), m, n, w.data_ptr(), float(eps), out.data_ptr(), _stream())
    return out


def linear(x: torch.Tensor, w: torch.Tensor, *, norm_w: torch.Tensor | None = None, eps: float = 1e-6,
           epilogue: int = EPI_STORE, residual: torch.Tensor | None = None,
           out: torch.Tensor | None = None) -> torch.Tensor:
    """``out = epilogue(w @ rmsnorm?(x))`` for x ``[m, k]`` with m <= 8."""
    _check(x, "x")
    _check(w, "w")
    k = x.shape[-1]
    m = x.numel() // k
    n = w.shape[0]
    if w.shape[1] != k:
        raise ValueError(f"weight in-features {w.shape[1]} != activation width {k}")
    if norm_w is not None:
        _check(norm_w, "norm_w")
    if residual is not None:
        _check(residual, "residual")
    cols = n // 2 if epilogue == EPI_SILU_MUL else n
    if out is None:
        out = torch.empty((*x.shape[:-1], cols), device=x.device,
                          dtype=torch.float32 if epilogue == EPI_STORE_F32 else BF16)
    nat.call("ls_linear_bf16", x.data_ptr(), m, k, _ptr(norm_w), float(eps), w.data_ptr(), n, int(epilogue),
             _ptr(residual), out.data_ptr(), _stream())
    return out


def qkv_rope_append(x: torch.Tensor, batch: int, q_len: int, qkv_w: torch.Tensor, num_heads: int,
                    num_kv_heads: int, head_dim: int, q_norm_w: torch.Tensor, k_norm_w: torch.Tensor,
                    cos: torch.Tensor, sin: torch.Tensor, *, input_norm_w: torch.Tensor | None = None,
                    eps: float = 1e-6, cache_pos: torch.Tensor | None = None, uniform_past: int = 0,
                    rope_offset: int = 0,
                    k_cache: torch.Tensor | None = None, v_cache: torch.Tensor | None = None, max_seq: int = 0,
                    k_out: torch.Tensor | None = None, v_out: torch.Tensor | None = None,
                    qkv_scratch: torch.Tensor | None = None, q_out: torch.Tensor | None = None):
    """Input RMSNorm + QKV projection + q/k norm + RoPE + KV append (one C call)."""
    _check(x, "x")
    _check(qkv_w, "qkv_w")
    _check(cos, "cos")
    _check(sin, "sin")
    m = batch * q_len
    hidden = x.shape[-1]
    if cache_pos is not None:
        _check(cache_pos, "cache_pos", torch.int32)
    dev = x.device
    if qkv_scratch is None:
        qkv_scratch = torch.empty((m, qkv_w.shape[0]), device=dev, dtype=BF16)
    if q_out is None:
        q_out = torch.empty((m, num_heads, head_dim), device=dev, dtype=BF16)
    nat.call("ls_rmsnorm_qkv_rope_kvappend", x.data_ptr(), batch, q_len, hidden, _ptr(input_norm_w), float(eps),
             qkv_w.data_ptr(), num_heads, num_kv_heads, head_dim, q_norm_w.data_ptr(), k_norm_w.data_ptr(),
             cos.data_ptr(), sin.data_ptr(), cos.shape[0], int(rope_offset), _ptr(cache_pos), int(uniform_past),
             _ptr(k_cache),
             _ptr(v_cache), int(max_seq), _ptr(k_out), _ptr(v_out), qkv_scratch.data_ptr(), q_out.data_ptr(),
             _stream())
    return q_out


def qk_norm_rope(qkv: torch.Tensor, batch: int, q_len: int, num_heads: int, num_kv_heads: int, head_dim: int,
                 q_norm_w: torch.Tensor, k_norm_w: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, *,
                 eps: float = 1e-6, cache_pos: torch.Tensor | None = None, uniform_past: int = 0,
                 rope_offset: int = 0, k_cache: torch.Tensor | None = None, v_cache: torch.Tensor | None = None,
                 max_seq: int = 0, k_out: torch.Tensor | None = None, v_out: torch.Tensor | None = None,
                 q_out: torch.Tensor | None = None) -> torch.Tensor:
    """q/k RMSNorm + RoPE + K/V append on a precomputed fused projection ``qkv [m, (Hq+2Hkv) D]``."""
    _check(qkv, "qkv")
    m = batch * q_len
    if cache_pos is not None:
        _check(cache_pos, "cache_pos", torch.int32)
    if q_out is None:
        q_out = torch.empty((m, num_heads, head_dim), device=qkv.device, dtype=BF16)
    nat.call("ls_qk_norm_rope_kvappend", qkv.data_ptr(), batch, q_len, num_heads, num_kv_heads, head_dim,
             q_norm_w.data_ptr(), k_norm_w.data_ptr(), float(eps), cos.data_ptr(), sin.data_ptr(), cos.shape[0],
             int(rope_offset), _ptr(cache_pos), int(uniform_past), _ptr(k_cache), _ptr(v_cache), int(max_seq),
             _ptr(k_out), _ptr(v_out), q_out.data_ptr(), _stream())
    return q_out


def qk_norm_rope_splits(part: torch.Tensor, splits: int, batch: int, q_len: int, num_heads: int,
                        num_kv_heads: int, head_dim: int, q_norm_w: torch.Tensor, k_norm_w: torch.Tensor,
                        cos: torch.Tensor, sin: torch.Tensor, *, eps: float = 1e-6,
                        cache_pos: torch.Tensor | None = None, uniform_past: int = 0, rope_offset: int = 0,
                        k_cache: torch.Tensor | None = None, v_cache: torch.Tensor | None = None, max_seq: int = 0,
                        k_out: torch.Tensor | None = None, v_out: torch.Tensor | None = None,
                        q_out: torch.Tensor) -> torch.Tensor:
    """:func:`qk_norm_rope` on the split fp32 partials of the QKV projection (``gemm_tc_splits``)."""
    _check(part, "part", torch.float32)
    m = batch * q_len
    if part.numel() < splits * m * (num_heads + 2 * num_kv_heads) * head_dim:
        raise ValueError("split partials smaller than splits x m x qkv_dim")
    if cache_pos is not None:
        _check(cache_pos, "cache_pos", torch.int32)
    nat.call("ls_qk_norm_rope_kvappend_splits", part.data_ptr(), splits, batch, q_len, num_heads, num_kv_heads,
             head_dim, q_norm_w.data_ptr(), k_norm_w.data_ptr(), float(eps), cos.data_ptr(), sin.data_ptr(),
             cos.shape[0], int(rope_offset), _ptr(cache_pos), int(uniform_past), _ptr(k_cache), _ptr(v_cache),
             int(max_seq), _ptr(k_out), _ptr(v_out), q_out.data_ptr(), _stream())
    return q_out


def argmax_workspace_bytes(m: int, n: int) -> int:
    v = ctypes.c_int64(0)
    nat.call("ls_argmax_rows_workspace_bytes", m, n, ctypes.byref(v))
    return v.value


def argmax_rows(logits: torch.Tensor, *, out_ids: torch.Tensor | None = None,
                workspace: torch.Tensor | None = None) -> torch.Tensor:
    """Row argmax of bf16 logits ``[m, n]``, lowest index on ties -> int64 ``[m]``."""
    _check(logits, "logits")
    n = logits.shape[-1]
    m = logits.numel() // n
    if out_ids is None:
        out_ids = torch.empty((m,), device=logits.device, dtype=torch.int64)
    if workspace is None:
        workspace = torch.zeros(argmax_workspace_bytes(m, n), device=logits.device, dtype=torch.uint8)
    nat.call("ls_argmax_rows", logits.data_ptr(), m, n, out_ids.data_ptr(), workspace.data_ptr(), workspace.numel(),
             _stream())
    return out_ids


def attention_workspace_bytes(batch: int, q_len: int, num_heads: int, num_kv_heads: int, head_dim: int,
                              max_seq: int) -> int:
    v = ctypes.c_int64(0)
    nat.call("ls_decode_attention_workspace_bytes", batch, q_len, num_heads, num_kv_heads, head_dim, max_seq,
             ctypes.byref(v))
    return v.value


def decode_attention(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, batch: int, q_len: int,
                     num_heads: int, num_kv_heads: int, head_dim: int, max_seq: int, scale: float, *,
                     cache_pos: torch.Tensor | None = None, uniform_past: int = 0,
                     out: torch.Tensor | None = None, workspace: torch.Tensor | None = None) -> torch.Tensor:
    """GQA attention over a ``[batch, Hkv, max_seq, D]`` cache slice.

    ``k_cache`` may be a strided view whose base pointer starts the slice; its
    sequence stride must equal ``head_dim`` and the (b, h) stride
    ``max_seq * head_dim``.
    """
    _check(q, "q")
    for name, t in (("k_cache", k_cache), ("v_cache", v_cache)):
        if t.dtype != BF16 or t.device.type != "cuda":
            raise TypeError(f"{name} must be a bf16 CUDA tensor")
    m = batch * q_len
    if out is None:
        out = torch.empty((m, num_heads * head_dim), device=q.device, dtype=BF16)
    need = attention_workspace_bytes(batch, q_len, num_heads, num_kv_heads, head_dim, max_seq)
    if workspace is None:
        workspace = torch.zeros(max(need, 256), device=q.device, dtype=torch.uint8)
    nat.call("ls_decode_attention", q.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), _ptr(cache_pos),
             int(uniform_past), batch, q_len, num_heads, num_kv_heads, head_dim, max_seq, float(scale),
             out.data_ptr(), workspace.data_ptr(), workspace.numel(), _stream())
    return out


def decode_attention_qkv(qkv: torch.Tensor, batch: int, num_heads: int, num_kv_heads: int, head_dim: int,
                         q_norm_w: torch.Tensor, k_norm_w: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor,
                         k_cache: torch.Tensor, v_cache: torch.Tensor, max_seq: int, scale: float, *,
                         eps: float = 1e-6, cache_pos: torch.Tensor | None = None, uniform_past: int = 0,
                         rope_offset: int = 0, out: torch.Tensor | None = None) -> torch.Tensor:
    """One decode token per sequence from the raw fused projection ``qkv [batch, (Hq+2Hkv) D]``:
    :func:`qk_norm_rope` (q/k norm, RoPE, K/V append at ``cache_pos``) and :func:`decode_attention`
    in one launch, with the same bits as the two."""
    _check(qkv, "qkv")
    for name, t in (("k_cache", k_cache), ("v_cache", v_cache)):
        if t.dtype != BF16 or t.device.type != "cuda":
            raise TypeError(f"{name} must be a bf16 CUDA tensor")
    if cache_pos is not None:
        _check(cache_pos, "cache_pos", torch.int32)
    if out is None:
        out = torch.empty((batch, num_heads * head_dim), device=qkv.device, dtype=BF16)
    nat.call("ls_decode_attention_qkv", qkv.data_ptr(), batch, num_heads, num_kv_heads, head_dim,
             q_norm_w.data_ptr(), k_norm_w.data_ptr(), float(eps), cos.data_ptr(), sin.data_ptr(), cos.shape[0],
             int(rope_offset), _ptr(cache_pos), int(uniform_past), k_cache.data_ptr(), v_cache.data_ptr(),
             int(max_seq), float(scale), out.data_ptr(), _stream())
    return out


def oproj_residual(attn: torch.Tensor, o_w: torch.Tensor, residual: torch.Tensor,
                   out: torch.Tensor | None = None) -> torch.Tensor:
    _check(attn, "attn")
    _check(o_w, "o_w")
    _check(residual, "residual")
    k = attn.shape[-1]
    m = attn.numel() // k
    if out is None:
        out = torch.empty_like(residual)
    nat.call("ls_oproj_residual", attn.data_ptr(), m, k, o_w.data_ptr(), o_w.shape[0], residual.data_ptr(),
             out.data_ptr(), _stream())
    return out


def gateup_silu(h: torch.Tensor, post_norm_w: torch.Tensor | None, gate_up_w: torch.Tensor, eps: float,
                out: torch.Tensor | None = None) -> torch.Tensor:
    _check(h, "h")
    _check(gate_up_w, "gate_up_w")
    hidden = h.shape[-1]
    m = h.numel() // hidden
    inter = gate_up_w.shape[0] // 2
    if out is None:
        out = torch.empty((*h.shape[:-1], inter), device=h.device, dtype=BF16)
    nat.call("ls_rmsnorm_gateup_silu", h.data_ptr(), m, hidden, _ptr(post_norm_w), float(eps),
             gate_up_w.data_ptr(), inter, out.data_ptr(), _stream())
    return out


def down_residual(act: torch.Tensor, down_w: torch.Tensor, residual: torch.Tensor,
                  out: torch.Tensor | None = None) -> torch.Tensor:
    _check(act, "act")
    _check(down_w, "down_w")
    _check(residual, "residual")
    inter = act.shape[-1]
    m = act.numel() // inter
    if out is None:
        out = torch.empty_like(residual)
    nat.call("ls_down_residual", act.data_ptr(), m, inter, down_w.data_ptr(), down_w.shape[0],
             residual.data_ptr(), out.data_ptr(), _stream())
    return out


def lmhead_workspace_bytes(m: int, vocab: int) -> int:
    v = ctypes.c_int64(0)
    nat.call("ls_lmhead_workspace_bytes", m, vocab, ctypes.byref(v))
    return v.value


def lmhead_argmax(h: torch.Tensor, final_norm_w: torch.Tensor | None, lm_head_w: torch.Tensor, eps: float, *,
                  out_ids: torch.Tensor | None = None, workspace: torch.Tensor | None = None) -> torch.Tensor:
    _check(h, "h")
    _check(lm_head_w, "lm_head_w")
    hidden = h.shape[-1]
    m = h.numel() // hidden
    vocab = lm_head_w.shape[0]
    if out_ids is None:
        out_ids = torch.empty((m,), device=h.device, dtype=torch.int64)
    need = lmhead_workspace_bytes(m, vocab)
    if workspace is None:
        workspace = torch.zeros(need, device=h.device, dtype=torch.uint8)
    nat.call("ls_lmhead_argmax", h.data_ptr(), m, hidden, _ptr(final_norm_w), float(eps), lm_head_w.data_ptr(),
             vocab, out_ids.data_ptr(), workspace.data_ptr(), workspace.numel(), _stream())
    return out_ids


def lmhead_argmax_keys(h: torch.Tensor, final_norm_w: torch.Tensor | None, lm_head_shard: torch.Tensor, eps: float,
                       vocab_offset: int, *, out_keys: torch.Tensor | None = None,
                       workspace: torch.Tensor | None = None) -> torch.Tensor:
    """Greedy head over one vocab shard; int64 keys (see ``tp.argmax_key``) per row."""
    _check(h, "h")
    _check(lm_head_shard, "lm_head_shard")
    hidden = h.shape[-1]
    m = h.numel() // hidden
    rows = lm_head_shard.shape[0]
    if out_keys is None:
        out_keys = torch.empty((m,), device=h.device, dtype=torch.int64)
    need = lmhead_workspace_bytes(m, rows)
    if workspace is None:
        workspace = torch.zeros(need, device=h.device, dtype=torch.uint8)
    nat.call("ls_lmhead_argmax_keys", h.data_ptr(), m, hidden, _ptr(final_norm_w), float(eps),
             lm_head_shard.data_ptr(), rows, int(vocab_offset), out_keys.data_ptr(), workspace.data_ptr(),
             workspace.numel(), _stream())
    return out_keys


def argmax_rows_keys(logits: torch.Tensor, vocab_offset: int, *, out_keys: torch.Tensor | None = None,
                     workspace: torch.Tensor | None = None) -> torch.Tensor:
    _check(logits, "logits")
    m, n = logits.shape
    if out_keys is None:
        out_keys = torch.empty((m,), device=logits.device, dtype=torch.int64)
    if workspace is None:
        workspace = torch.zeros(argmax_workspace_bytes(m, n), device=logits.device, dtype=torch.uint8)
    nat.call("ls_argmax_rows_keys", logits.data_ptr(), m, n, int(vocab_offset), out_keys.data_ptr(),
             workspace.data_ptr(), workspace.numel(), _stream())
    return out_keys


def argmax_keys_to_ids(keys: torch.Tensor, *, out_ids: torch.Tensor | None = None) -> torch.Tensor:
    _check(keys, "keys", torch.int64)
    if out_ids is None:
        out_ids = torch.empty_like(keys)
    nat.call("ls_argmax_keys_to_ids", keys.data_ptr(), keys.numel(), out_ids.data_ptr(), _stream())
    return out_ids


def gemm_workspace_bytes(m: int, k: int, n: int, epilogue: int) -> int:
    v = ctypes.c_int64(0)
    nat.call("ls_gemm_bf16_tcgen05_workspace_bytes", m, k, n, int(epilogue), ctypes.byref(v))
    return v.value


def gemm_tc(x: torch.Tensor, w: torch.Tensor, *, epilogue: int = EPI_STORE, residual: torch.Tensor | None = None,
            out: torch.Tensor | None = None, workspace: torch.Tensor | None = None,
            tiled: torch.Tensor | None = None) -> torch.Tensor:
    """tcgen05 weight-streaming GEMM: ``out = epilogue(x @ w.T)`` for x ``[m, k]``, 1 <= m <= 128."""
    _check(x, "x")
    _check(w, "w")
    k = x.shape[-1]
    m = x.numel() // k
    n = w.shape[0] // 2 if epilogue == EPI_SILU_MUL else w.shape[0]
    if w.shape[1] != k:
        raise ValueError(f"weight in-features {w.shape[1]} != activation width {k}")
    if residual is not None:
        _check(residual, "residual")
    if out is None:
        out = torch.empty((*x.shape[:-1], n), device=x.device,
                          dtype=torch.float32 if epilogue == EPI_STORE_F32 else BF16)
    need = gemm_workspace_bytes(m, k, n, epilogue)
    if workspace is None:
        workspace = torch.zeros(need, device=x.device, dtype=torch.uint8)
    if tiled is not None:  # the weight's pre-tiled copy (gemm_tc_tile_weight); ``w`` gives the shape only
        nat.call("ls_gemm_bf16_tcgen05_tiled", x.data_ptr(), m, k, tiled.data_ptr(), n, int(epilogue),
                 _ptr(residual), out.data_ptr(), workspace.data_ptr(), workspace.numel(), _stream())
    else:
        nat.call("ls_gemm_bf16_tcgen05", x.data_ptr(), m, k, w.data_ptr(), n, int(epilogue), _ptr(residual),
                 out.data_ptr(), workspace.data_ptr(), workspace.numel(), _stream())
    return out


def gemm_splits(m: int, k: int, n: int) -> int:
    """k-splits of the ``EPI_SPLIT_F32`` form of :func:`gemm_tc` (its output is ``[splits, m, n]`` fp32)."""
    v = ctypes.c_int64(0)
    nat.call("ls_gemm_bf16_tcgen05_splits", m, k, n, ctypes.byref(v))
    return v.value


def gemm_tc_splits(x: torch.Tensor, w: torch.Tensor, out: torch.Tensor, *,
                   tiled: torch.Tensor | None = None) -> int:
    """tcgen05 GEMM with the split-partial epilogue: ``out[:splits*m*n]`` (fp32,
    viewed as ``[splits, m, n]``) receives one unrounded partial of ``x @ w.T``
    per k-split; returns ``splits``.  The consumer adds them in split order."""
    _check(x, "x")
    _check(w, "w")
    _check(out, "out", torch.float32)
    k = x.shape[-1]
    m = x.numel() // k
    n = w.shape[0]
    if w.shape[1] != k:
        raise ValueError(f"weight in-features {w.shape[1]} != activation width {k}")
    s = gemm_splits(m, k, n)
    if out.numel() < s * m * n:
        raise ValueError(f"split output holds {out.numel()} floats, needs {s} x {m} x {n}")
    if tiled is not None:
        nat.call("ls_gemm_bf16_tcgen05_tiled", x.data_ptr(), m, k, tiled.data_ptr(), n, EPI_SPLIT_F32, None,
                 out.data_ptr(), None, 0, _stream())
    else:
        nat.call("ls_gemm_bf16_tcgen05", x.data_ptr(), m, k, w.data_ptr(), n, EPI_SPLIT_F32, None, out.data_ptr(),
                 None, 0, _stream())
    return s


def residual_rmsnorm_splits(part: torch.Tensor, splits: int, residual: torch.Tensor, *, out_residual: torch.Tensor,
                            norm_w: torch.Tensor | None = None, eps: float = 1e-6,
                            out_norm: torch.Tensor | None = None) -> None:
    """``out_residual = bf16(residual + bf16(sum_s part[s]))`` over ``[m, n]`` rows,
    then (with ``norm_w``) ``out_norm = rmsnorm(out_residual) * norm_w``."""
    _check(part, "part", torch.float32)
    _check(residual, "residual")
    _check(out_residual, "out_residual")
    n = residual.shape[-1]
    m = residual.numel() // n
    if part.numel() < splits * m * n:
        raise ValueError("split partials smaller than splits x m x n")
    if (norm_w is None) != (out_norm is None):
        raise ValueError("norm_w and out_norm come together")
    nat.call("ls_residual_rmsnorm_splits", part.data_ptr(), splits, m, n, residual.data_ptr(), _ptr(norm_w),
             float(eps), out_residual.data_ptr(), _ptr(out_norm), _stream())


def gate_up_plain(m: int, k: int, n_rows: int) -> bool:
    """Whether the fused gate_up linear ``[n_rows = 2I, k]`` runs as a plain
    linear in the split-partial form followed by :func:`silu_mul_splits`
    (whole-K tiles when its 128-row tiles cover the SMs, else k-splits on two
    CTAs per SM) instead of the paired SiLU epilogue: when I is a multiple of
    128, so that the paired pre-tiled image is also the plain one."""
    del m, k
    return (n_rows // 2) % 128 == 0


def silu_mul_splits(part: torch.Tensor, splits: int, m: int, intermediate: int, *, out: torch.Tensor) -> None:
    """``out[m, I] = bf16(bf16(silu(bf16(g))) * bf16(u))`` from the split partials
    ``part [splits, m, 2I]`` of the gate_up projection run as a plain linear."""
    _check(part, "part", torch.float32)
    _check(out, "out")
    if part.numel() < splits * m * 2 * intermediate or out.numel() < m * intermediate:
        raise ValueError("silu_mul_splits: buffers smaller than the shapes")
    nat.call("ls_silu_mul_splits", part.data_ptr(), splits, m, intermediate, out.data_ptr(), _stream())


def gemm_big(x: torch.Tensor, w: torch.Tensor, *, epilogue: int = EPI_STORE, residual: torch.Tensor | None = None,
             out: torch.Tensor | None = None) -> torch.Tensor:
    """Large-M tcgen05 GEMM (prefill): ``out = epilogue(x @ w.T)`` for x ``[m, k]`` with m in the thousands."""
    _check(x, "x")
    _check(w, "w")
    k = x.shape[-1]
    m = x.numel() // k
    n = w.shape[0] // 2 if epilogue == EPI_SILU_MUL else w.shape[0]
    if w.shape[1] != k:
        raise ValueError(f"weight in-features {w.shape[1]} != activation width {k}")
    if residual is not None:
        _check(residual, "residual")
    if out is None:
        out = torch.empty((*x.shape[:-1], n), device=x.device,
                          dtype=torch.float32 if epilogue == EPI_STORE_F32 else BF16)
    nat.call("ls_gemm_bf16_tcgen05_big", x.data_ptr(), m, k, w.data_ptr(), n, int(epilogue), _ptr(residual),
             out.data_ptr(), _stream())
    return out


def gemm_tc_tile_weight(w: torch.Tensor, silu: bool = False) -> torch.Tensor:
    """Tile a ``[N, K]`` weight for :func:`gemm_tc` (``tiled=``): 16 KB MMA-image tiles (uint8 buffer)."""
    _check(w, "w")
    nbytes = ctypes.c_int64(0)
    nat.call("ls_gemm_tc_tiled_bytes", w.shape[0], w.shape[1], int(bool(silu)), ctypes.byref(nbytes))
    out = torch.empty(nbytes.value, device=w.device, dtype=torch.uint8)
    nat.call("ls_gemm_tc_tile_weight", w.data_ptr(), w.shape[0], w.shape[1], int(bool(silu)), out.data_ptr(),
             _stream())
    return out


def linear_allreduce_residual(x: torch.Tensor, w: torch.Tensor, residual: torch.Tensor, exchange,
                              out: torch.Tensor | None = None) -> torch.Tensor:
    """Row-split linear + fused one-shot all-reduce over the ranks + residual (``ls_linear_allreduce_residual``).

    ``exchange``: a :class:`leanstack_b200.tp.P2PExchange` (every rank calls with the same m)."""
    _check(x, "x")
    _check(w, "w")
    _check(residual, "residual")
    k = x.shape[-1]
    m = x.numel() // k
    n = w.shape[0]
    if out is None:
        out = torch.empty_like(residual)
    nat.call("ls_linear_allreduce_residual", x.data_ptr(), m, k, w.data_ptr(), n, residual.data_ptr(),
             out.data_ptr(), ctypes.byref(exchange.desc), _stream())
    return out


def allreduce_residual_f32(part: torch.Tensor, residual: torch.Tensor, exchange,
                           out: torch.Tensor | None = None) -> torch.Tensor:
    """One-shot all-reduce over the ranks of fp32 partials ``part [m, n]`` plus the
    residual epilogue (``ls_allreduce_residual_f32``): ``bf16(res + bf16(sum))``."""
    _check(part, "part", torch.float32)
    _check(residual, "residual")
    n = part.shape[-1]
    m = part.numel() // n
    if out is None:
        out = torch.empty_like(residual)
    nat.call("ls_allreduce_residual_f32", part.data_ptr(), m, n, residual.data_ptr(), out.data_ptr(),
             ctypes.byref(exchange.desc), _stream())
    return out


def allreduce_residual_splits(part: torch.Tensor, splits: int, residual: torch.Tensor, exchange, *,
                              out: torch.Tensor) -> torch.Tensor:
    """:func:`allreduce_residual_f32` over split partials ``part [splits, m, n]``
    (each rank adds its splits in order first)."""
    _check(part, "part", torch.float32)
    _check(residual, "residual")
    n = residual.shape[-1]
    m = residual.numel() // n
    if part.numel() < splits * m * n:
        raise ValueError("split partials smaller than splits x m x n")
    nat.call("ls_allreduce_residual_splits", part.data_ptr(), splits, m, n, residual.data_ptr(), out.data_ptr(),
             ctypes.byref(exchange.desc), _stream())
    return out


def sum_splits_f32(part: torch.Tensor, splits: int, n: int, *, out: torch.Tensor) -> torch.Tensor:
    """``out[:n] = sum_s part[s * n : (s + 1) * n]`` in split order (fp32)."""
    _check(part, "part", torch.float32)
    _check(out, "out", torch.float32)
    if part.numel() < splits * n or out.numel() < n:
        raise ValueError("sum_splits_f32: buffers smaller than the shapes")
    nat.call("ls_sum_splits_f32", part.data_ptr(), splits, n, out.data_ptr(), _stream())
    return out


def residual_add_f32(residual: torch.Tensor, y: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """``out = bf16(residual + bf16(y))`` for an fp32 ``y`` (after a tensor-parallel all-reduce)."""
    _check(residual, "residual")
    _check(y, "y", torch.float32)
    if out is None:
        out = torch.empty_like(residual)
    nat.call("ls_residual_add_f32", residual.data_ptr(), y.data_ptr(), residual.numel(), out.data_ptr(), _stream())
    return out


def spec_accept(ids: torch.Tensor, verdict: torch.Tensor, batch: int, k: int, *,
                next_ids: torch.Tensor | None = None, accepted: torch.Tensor | None = None,
                cache_pos: torch.Tensor | None = None, draft_cache_pos: torch.Tensor | None = None,
                out_tokens: torch.Tensor | None = None, out_len: torch.Tensor | None = None) -> None:
    """Greedy-exact accept / reject of a verify pass (see ``ls_spec_accept``); updates ``ids[:, 0]``."""
    _check(ids, "ids", torch.int64)
    _check(verdict, "verdict", torch.int64)
    if ids.numel() < batch * (k + 1) or verdict.numel() < batch * (k + 1):
        raise ValueError("ids / verdict must hold batch * (k + 1) tokens")
    if next_ids is not None:
        _check(next_ids, "next_ids", torch.int64)
    if accepted is not None:
        _check(accepted, "accepted", torch.int32)
    for name, t in (("cache_pos", cache_pos), ("draft_cache_pos", draft_cache_pos), ("out_len", out_len)):
        if t is not None:
            _check(t, name, torch.int32)
    cap = 0
    if out_tokens is not None:
        _check(out_tokens, "out_tokens", torch.int64)
        if out_tokens.dim() != 2 or out_tokens.shape[0] != batch:
            raise ValueError("out_tokens must be [batch, capacity]")
        cap = out_tokens.shape[1]
    nat.call("ls_spec_accept", ids.data_ptr(), verdict.data_ptr(), batch, k, _ptr(next_ids), _ptr(accepted),
             _ptr(cache_pos), _ptr(draft_cache_pos), _ptr(out_tokens), _ptr(out_len), cap, _stream())


def advance_cursors(cache_pos: torch.Tensor, q_len: int, delta: torch.Tensor | None = None) -> None:
    _check(cache_pos, "cache_pos", torch.int32)
    nat.call("ls_advance_cursors", cache_pos.data_ptr(), _ptr(delta), cache_pos.numel(), int(q_len), _stream())
