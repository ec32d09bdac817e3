"""Resident decode engine: arenas from the buffer planner + a CUDA-graph step.

This is the serving fast path behind the reference-shaped API.  One engine
owns, for a fixed (batch, max_seq): the KV arenas, the activation arenas, the
position cache, the kernel workspaces and one captured CUDA graph of a whole
decode step (embedding gather, 36 x 5 layer kernels, greedy head, cursor
advance).  Every kernel reads the per-sequence cursors from the device
(``cache_pos``), so the captured graph stays valid as the sequences grow and
the host only replays it.

Token flow: the step's input ids live in ``arenas.ids[:B]``; the greedy head
writes the next ids back into the same slots, so consecutive replays decode
autoregressively with no host round trip.

Tensor parallelism (``tp`` given, world > 1): the runtime is this rank's shard
(``tp.materialize_tp_shard``).  o_proj and down_proj write fp32 partials that
one NCCL all-reduce sums before the residual-add kernel; the head reduces its
vocab shard to int64 argmax keys and a MAX all-reduce picks the token.  The
collectives are captured into the step's CUDA graph with the kernels.
"""

from __future__ import annotations

import torch

from . import kernels as K
from .leanserve import allocate_arenas, build_resident_buffer_plan, runtime_weight_bytes
from .qwen_explicit import QwenSemanticStackRuntime, build_qwen_position_cache
from .tp import TPComm, TPShard

SMALL_M = 8      # largest token count of the CUDA-core linear kernels
TC_MAX_M = 128   # largest token count of one tcgen05 GEMM launch
BACKENDS = ("auto", "tc", "cuda_core")


def resolve_backend(backend: str, batch_size: int, tensor_parallel: bool = False) -> str:
    """``auto``: on one GPU, tensor cores from 2 sequences on and CUDA-core
    streaming for one; under tensor parallelism (row-split linears through the
    fused peer all-reduce of the CUDA-core kernel), tensor cores from 6.

    Measured on Qwen3-4B decode steps with 2048 cached positions (tok/s,
    CUDA-core / tcgen05), one GPU, split-partial GEMMs summed by the next
    kernel and whole-K gate_up: B 1 388 / 383, 2 610 / 680, 3 926 / 1082,
    4 1111 / 1418, 5 1228 / 1722, 6 1330 / 2025, 8 1524 / 2644.  Before those
    GEMM forms (the tensor-parallel ones still reduce inside the GEMM): B 5
    1229 / 1186, 6 1328 / 1413.
    """
    if backend not in BACKENDS:
        raise ValueError(f"unknown linear backend {backend!r}; choose from {BACKENDS}")
    if backend == "auto":
        return "tc" if batch_size >= (6 if tensor_parallel else 2) else "cuda_core"
    return backend


class DecodeEngine:
    def __init__(self, runtime: QwenSemanticStackRuntime, batch_size: int, max_seq_len: int,
                 max_tokens_per_step: int | None = None, use_graph: bool = True, linear_backend: str = "auto",
                 tp: TPComm | None = None, shard: TPShard | None = None,
                 tc_tiles: list[dict] | None = None):
        if runtime.final_norm_weight is None or runtime.lm_head_weight is None:
            raise ValueError("the engine needs the output head (include_output_head=True)")
        self.tp = tp if (tp is not None and tp.world > 1) else None
        if self.tp is not None and shard is None:
            raise ValueError("a tensor-parallel engine needs its TPShard")
        self.vocab_offset = shard.vocab_offset if self.tp is not None else 0
        self.vocab_rows = runtime.lm_head_weight.shape[0]
        self.backend = resolve_backend(linear_backend, batch_size, self.tp is not None)
        limit = TC_MAX_M if self.backend == "tc" else SMALL_M
        if batch_size < 1 or batch_size > limit:
            raise ValueError(f"batch_size {batch_size}: the {self.backend} step handles 1..{limit} sequences")
        if max_tokens_per_step is None:
            max_tokens_per_step = limit
        self.rt = runtime
        self.g = g = runtime.config
        self.B = batch_size
        self.max_seq = max_seq_len
        self.T = min(limit, max(max_tokens_per_step, batch_size)) // batch_size * batch_size
        self.plan = build_resident_buffer_plan(g, weights_bytes=runtime_weight_bytes(runtime), batch_size=batch_size,
                                               max_seq_len=max_seq_len, max_tokens_per_step=self.T)
        self.arenas = allocate_arenas(self.plan, g, runtime.device, runtime.dtype)
        self.kv = self.arenas.kv
        self.S = self.kv.layout.max_seq_len
        self.cos, self.sin = build_qwen_position_cache(runtime.rope_inv_freq, runtime.attention_scaling, self.S,
                                                       runtime.dtype)
        dev = runtime.device
        ws = max(K.attention_workspace_bytes(batch_size, q, g.num_attention_heads, g.num_key_value_heads, g.head_dim,
                                             self.S) for q in range(1, self.T // batch_size + 1))
        self.attn_ws = torch.zeros(max(ws, 256), device=dev, dtype=torch.uint8)
        self.gu_plain = False
        if self.backend == "tc":
            T = self.T
            row_epi = K.EPI_STORE_F32 if self.tp is not None else K.EPI_RESIDUAL
            shapes = [(T, g.hidden_size, g.qkv_dim, K.EPI_STORE), (T, g.q_dim, g.hidden_size, row_epi),
                      (T, g.hidden_size, g.intermediate_size, K.EPI_SILU_MUL),
                      (T, g.intermediate_size, g.hidden_size, row_epi),
                      (batch_size, g.hidden_size, self.vocab_rows, K.EPI_STORE)]
            self.tc_ws = torch.zeros(max(K.gemm_workspace_bytes(*s_) for s_ in shapes), device=dev, dtype=torch.uint8)
            self.xn = torch.zeros(T, g.hidden_size, device=dev, dtype=runtime.dtype)
            self.logits = torch.zeros(T, self.vocab_rows, device=dev, dtype=runtime.dtype)
            self.lm_ws = torch.zeros(K.argmax_workspace_bytes(T, self.vocab_rows), device=dev, dtype=torch.uint8)
            # Split fp32 partials of QKV / o_proj / down (one GPU): the GEMMs
            # leave the cross-split sum to the next kernel (q/k norm, residual +
            # RMSNorm) instead of reducing behind a grid-wide wait.
            # gate_up as a plain [2I, H] linear (whole-K tiles when its 128-row
            # tiles cover the SMs, else k-splits) followed by the SiLU*up
            # combine; else the paired SiLU epilogue.
            self.gu_plain = K.gate_up_plain(T, g.hidden_size, 2 * g.intermediate_size)
            # Split fp32 partials of QKV / o_proj / down / gate_up: the GEMMs
            # leave the cross-split sum to the next kernel (q/k norm, residual +
            # RMSNorm, SiLU*up, or the tensor-parallel all-reduce) instead of
            # reducing behind a grid-wide wait.  Shapes are this rank's shard.
            rt0 = runtime.layers[0]
            shapes_ = [(g.hidden_size, rt0.attention.qkv_proj_weight.shape[0]),
                       (rt0.attention.o_proj_weight.shape[1], g.hidden_size),
                       (rt0.mlp.down_proj_weight.shape[1], g.hidden_size)]
            if self.gu_plain:
                shapes_.append((g.hidden_size, rt0.mlp.gate_up_proj_weight.shape[0]))
            part = max(K.gemm_splits(mm, k_, n_) * mm * n_
                       for mm in range(batch_size, T + 1, batch_size) for k_, n_ in shapes_)
            self.tc_part = torch.zeros(part, device=dev, dtype=torch.float32)
        else:
            self.lm_ws = torch.zeros(K.lmhead_workspace_bytes(self.T, self.vocab_rows), device=dev,
                                     dtype=torch.uint8)
        if self.tp is not None:
            self.part = torch.zeros(self.T, g.hidden_size, device=dev, dtype=torch.float32)
            self.keys = torch.zeros(self.T, device=dev, dtype=torch.int64)
        # speculative verify: the target's token after every input position, and per-sequence results
        self.verdict = torch.zeros(self.T, device=dev, dtype=torch.int64)
        self.next_ids = torch.zeros(batch_size, device=dev, dtype=torch.int64)
        self.accepted = torch.zeros(batch_size, device=dev, dtype=torch.int32)
        self.verify_graphs: dict[int, torch.cuda.CUDAGraph] = {}
        # Pre-tiled tcgen05 weight images per layer ({"qkv", "o", "gu", "down"},
        # e.g. from a leanpack/v1 artifact): the tensor-core linears stream them
        # with plain bulk copies instead of TMA tensor maps.
        if tc_tiles is not None and len(tc_tiles) != len(runtime.layers):
            raise ValueError(f"tc_tiles has {len(tc_tiles)} layers, the runtime {len(runtime.layers)}")
        self.tc_tiles = tc_tiles
        self.use_graph = use_graph
        self.graph: torch.cuda.CUDAGraph | None = None

    # ------------------------------------------------------------------
    def _forward(self, q_len: int, head, advance: bool = True) -> None:
        """Enqueue one step of ``q_len`` tokens per sequence on the current stream.

        ``head``: falsy (no head), ``True`` / ``"last"`` (greedy token of each
        sequence's last position into ``ids[:B]``) or ``"all"`` (greedy token
        after every position into ``verdict[:m]``, the verify pass).
        ``advance``: move the device cursors by ``q_len`` at the end.
        """
        B, g, a, rt = self.B, self.g, self.arenas, self.rt
        m = B * q_len
        eps = g.rms_norm_eps
        kv = self.kv
        tc = self.backend == "tc"
        split = tc and self.tp is None  # one GPU: the residual linears' partials go to the residual consumer
        part = self.tc_part if tc else None
        s_down = 0
        K.embed_gather(a.ids[:m], rt.embed_tokens_weight, out=a.x[:m])
        for li, layer in enumerate(rt.layers):
            att, mlp = layer.attention, layer.mlp
            tt = self.tc_tiles[li] if (tc and self.tc_tiles is not None) else {}
            # QKV projection (with the input RMSNorm) into a.qkv
            if tc:
                if li == 0 or self.tp is not None:
                    K.rmsnorm(a.x[:m], layer.input_layernorm_weight, eps, out=self.xn[:m])
                else:  # the previous layer's down residual (one GPU), then this layer's input norm
                    K.residual_rmsnorm_splits(part, s_down, a.h[:m], out_residual=a.x[:m],
                                              norm_w=layer.input_layernorm_weight, eps=eps, out_norm=self.xn[:m])
                s_qkv = K.gemm_tc_splits(self.xn[:m], att.qkv_proj_weight, part, tiled=tt.get("qkv"))
                K.qk_norm_rope_splits(part, s_qkv, B, q_len, g.num_attention_heads, g.num_key_value_heads,
                                      g.head_dim, att.q_norm_weight, att.k_norm_weight, self.cos, self.sin, eps=eps,
                                      cache_pos=kv.cache_pos, k_cache=kv.key_cache[li], v_cache=kv.value_cache[li],
                                      max_seq=self.S, q_out=a.q[:m])
            else:
                K.linear(a.x[:m], att.qkv_proj_weight, norm_w=layer.input_layernorm_weight, eps=eps,
                         out=a.qkv[:m])
                if q_len == 1:  # q/k norm, RoPE, K/V append and attention in one launch
                    K.decode_attention_qkv(a.qkv[:m], B, g.num_attention_heads, g.num_key_value_heads, g.head_dim,
                                           att.q_norm_weight, att.k_norm_weight, self.cos, self.sin,
                                           kv.key_cache[li], kv.value_cache[li], self.S, att.attention_scale,
                                           eps=eps, cache_pos=kv.cache_pos, out=a.attn[:m])
                else:
                    K.qk_norm_rope(a.qkv[:m], B, q_len, g.num_attention_heads, g.num_key_value_heads, g.head_dim,
                                   att.q_norm_weight, att.k_norm_weight, self.cos, self.sin, eps=eps,
                                   cache_pos=kv.cache_pos, k_cache=kv.key_cache[li], v_cache=kv.value_cache[li],
                                   max_seq=self.S, q_out=a.q[:m])
            if tc or q_len != 1:
                K.decode_attention(a.q[:m], kv.key_cache[li], kv.value_cache[li], B, q_len, g.num_attention_heads,
                                   g.num_key_value_heads, g.head_dim, self.S, att.attention_scale,
                                   cache_pos=kv.cache_pos, out=a.attn[:m], workspace=self.attn_ws)
            if self.tp is not None:
                self._row_split(a.attn[:m], att.o_proj_weight, a.x[:m], a.h[:m], tc, tt.get("o"))
                if tc:
                    K.rmsnorm(a.h[:m], layer.post_attention_layernorm_weight, eps, out=self.xn[:m])
                    self._gate_up(self.xn[:m], mlp.gate_up_proj_weight, a.act[:m], tt.get("gu"))
                else:
                    K.gateup_silu(a.h[:m], layer.post_attention_layernorm_weight, mlp.gate_up_proj_weight, eps,
                                  out=a.act[:m])
                self._row_split(a.act[:m], mlp.down_proj_weight, a.h[:m], a.x[:m], tc, tt.get("down"))
            elif split:
                s_o = K.gemm_tc_splits(a.attn[:m], att.o_proj_weight, part, tiled=tt.get("o"))
                K.residual_rmsnorm_splits(part, s_o, a.x[:m], out_residual=a.h[:m],
                                          norm_w=layer.post_attention_layernorm_weight, eps=eps, out_norm=self.xn[:m])
                self._gate_up(self.xn[:m], mlp.gate_up_proj_weight, a.act[:m], tt.get("gu"))
                s_down = K.gemm_tc_splits(a.act[:m], mlp.down_proj_weight, part, tiled=tt.get("down"))
            else:
                K.oproj_residual(a.attn[:m], att.o_proj_weight, a.x[:m], out=a.h[:m])
                K.gateup_silu(a.h[:m], layer.post_attention_layernorm_weight, mlp.gate_up_proj_weight, eps,
                              out=a.act[:m])
                K.down_residual(a.act[:m], mlp.down_proj_weight, a.h[:m], out=a.x[:m])
        normed = False
        if split:  # the last layer's down residual (+ the final norm when the head takes every row)
            normed = bool(head) and (head == "all" or q_len == 1)
            K.residual_rmsnorm_splits(part, s_down, a.h[:m], out_residual=a.x[:m],
                                      norm_w=rt.final_norm_weight if normed else None, eps=eps,
                                      out_norm=self.xn[:m] if normed else None)
        if head:
            if head == "all":
                rows, n, dest = a.x[:m], m, self.verdict[:m]
            elif q_len == 1:
                rows, n, dest = a.x[:B], B, a.ids[:B]
            else:
                a.head_rows.copy_(a.x[:m].view(B, q_len, -1)[:, -1])
                rows, n, dest = a.head_rows, B, a.ids[:B]
            self._head(rows, n, dest, tc, normed=normed)
        if advance:
            K.advance_cursors(kv.cache_pos, q_len)

    def _head(self, rows: torch.Tensor, n: int, dest: torch.Tensor, tc: bool, normed: bool = False) -> None:
        """Greedy head over ``rows [n, H]``: final norm, lm_head (this rank's vocab shard), argmax into ``dest``.
        ``normed``: ``xn[:n]`` already holds the final norm of ``rows`` (tensor-core path)."""
        rt, eps = self.rt, self.g.rms_norm_eps
        self._head_rows = rows
        if self.tp is not None:
            keys = self.keys[:n]
            if tc:
                K.rmsnorm(rows, rt.final_norm_weight, eps, out=self.xn[:n])
                K.gemm_tc(self.xn[:n], rt.lm_head_weight, out=self.logits[:n], workspace=self.tc_ws)
                K.argmax_rows_keys(self.logits[:n], self.vocab_offset, out_keys=keys, workspace=self.lm_ws)
            else:
                K.lmhead_argmax_keys(rows, rt.final_norm_weight, rt.lm_head_weight, eps, self.vocab_offset,
                                     out_keys=keys, workspace=self.lm_ws)
            self.tp.all_reduce_max(keys)
            K.argmax_keys_to_ids(keys, out_ids=dest)
        elif tc:
            if not normed:
                K.rmsnorm(rows, rt.final_norm_weight, eps, out=self.xn[:n])
            K.gemm_tc(self.xn[:n], rt.lm_head_weight, out=self.logits[:n], workspace=self.tc_ws)
            K.argmax_rows(self.logits[:n], out_ids=dest, workspace=self.lm_ws)
        else:
            K.lmhead_argmax(rows, rt.final_norm_weight, rt.lm_head_weight, eps, out_ids=dest, workspace=self.lm_ws)

    def prefill_full(self, prompt_ids: torch.Tensor) -> torch.Tensor:
        """Prefill ``[B, P]`` prompts in one pass per layer.

        All B·P tokens go through each layer together: the linears run as
        large-M tcgen05 GEMMs (``ls_gemm_bf16_tcgen05_big``), attention runs
        causally over each sequence (the decode kernel with q_len = P), and the
        K/V of every position land in the cache.  Activations for the pass are
        allocated for its duration.  Returns the first greedy token per
        sequence ``[B]``; the cursors advance by P.
        """
        if prompt_ids.dim() != 2 or prompt_ids.shape[0] != self.B:
            raise ValueError(f"prompt_ids must be [{self.B}, P]")
        B, P = prompt_ids.shape
        if len(set(self.kv.sequence_lens)) != 1 or self.kv.sequence_lens[0] + P > self.S:
            raise ValueError("prefill_full needs equal cursors and room for the prompt")
        g, rt, a, kv = self.g, self.rt, self.arenas, self.kv
        dev, dt, eps, m = rt.device, rt.dtype, g.rms_norm_eps, B * P
        ids = prompt_ids.to(dev, torch.int64).reshape(-1)
        x = torch.empty(m, g.hidden_size, device=dev, dtype=dt)
        h = torch.empty_like(x)
        xn = torch.empty_like(x)
        qkv = torch.empty(m, g.qkv_dim, device=dev, dtype=dt)
        q = torch.empty(m, g.num_attention_heads, g.head_dim, device=dev, dtype=dt)
        attn = torch.empty(m, g.q_dim, device=dev, dtype=dt)
        act = torch.empty(m, g.intermediate_size, device=dev, dtype=dt)
        part = torch.empty(m, g.hidden_size, device=dev, dtype=torch.float32) if self.tp is not None else None

        def row_split(inp, w, res, out):
            if self.tp is None:
                K.gemm_big(inp, w, epilogue=K.EPI_RESIDUAL, residual=res, out=out)
            else:
                K.gemm_big(inp, w, epilogue=K.EPI_STORE_F32, out=part)
                self.tp.all_reduce_sum(part)
                K.residual_add_f32(res, part, out=out)

        K.embed_gather(ids, rt.embed_tokens_weight, out=x)
        for li, layer in enumerate(rt.layers):
            att, mlp = layer.attention, layer.mlp
            K.rmsnorm(x, layer.input_layernorm_weight, eps, out=xn)
            K.gemm_big(xn, att.qkv_proj_weight, out=qkv)
            K.qk_norm_rope(qkv, B, P, g.num_attention_heads, g.num_key_value_heads, g.head_dim, att.q_norm_weight,
                           att.k_norm_weight, self.cos, self.sin, eps=eps, cache_pos=kv.cache_pos,
                           k_cache=kv.key_cache[li], v_cache=kv.value_cache[li], max_seq=self.S, q_out=q)
            K.decode_attention(q, kv.key_cache[li], kv.value_cache[li], B, P, g.num_attention_heads,
                               g.num_key_value_heads, g.head_dim, self.S, att.attention_scale,
                               cache_pos=kv.cache_pos, out=attn, workspace=self.attn_ws)
            row_split(attn, att.o_proj_weight, x, h)
            K.rmsnorm(h, layer.post_attention_layernorm_weight, eps, out=xn)
            K.gemm_big(xn, mlp.gate_up_proj_weight, epilogue=K.EPI_SILU_MUL, out=act)
            row_split(act, mlp.down_proj_weight, h, x)
        a.head_rows.copy_(x.view(B, P, -1)[:, -1])
        self._head(a.head_rows, B, a.ids[:B], self.backend == "tc")
        K.advance_cursors(kv.cache_pos, P)
        kv.note_advanced(P)
        return a.ids[:B].clone()

    def _gate_up(self, xn: torch.Tensor, w: torch.Tensor, act: torch.Tensor, tiled: torch.Tensor | None) -> None:
        """act = SiLU(gate) * up on the tensor cores: plain split-partial linear +
        combine (the paired tile image is the plain one when I % 128 == 0), or
        the paired SiLU epilogue."""
        m = xn.shape[0]
        if self.gu_plain:
            s_gu = K.gemm_tc_splits(xn, w, self.tc_part, tiled=tiled)
            K.silu_mul_splits(self.tc_part, s_gu, m, w.shape[0] // 2, out=act)
        else:
            K.gemm_tc(xn, w, epilogue=K.EPI_SILU_MUL, out=act, workspace=self.tc_ws, tiled=tiled)

    def _row_split(self, x: torch.Tensor, w: torch.Tensor, residual: torch.Tensor, out: torch.Tensor,
                   tc: bool, tiled: torch.Tensor | None = None) -> None:
        """Row-split linear of tensor parallelism: fp32 partial, all-reduce, residual add.
        On the tensor cores the GEMM leaves its k-split partials; they are added
        in split order on each rank (inside the fused all-reduce, or by a sum
        kernel before NCCL), then across ranks."""
        if not tc and self.tp.p2p is not None:  # fused one-shot all-reduce in the linear's epilogue
            K.linear_allreduce_residual(x, w, residual, self.tp.p2p, out=out)
            return
        part = self.part[:x.shape[0]]
        if tc:
            s = K.gemm_tc_splits(x, w, self.tc_part, tiled=tiled)
            if self.tp.p2p_tc is not None:  # one-shot all-reduce of the partials + residual, over peer memory
                K.allreduce_residual_splits(self.tc_part, s, residual, self.tp.p2p_tc, out=out)
                return
            K.sum_splits_f32(self.tc_part, s, part.numel(), out=part)
        else:
            K.linear(x, w, epilogue=K.EPI_STORE_F32, out=part)
        if self.tp.p2p_tc is not None:  # one-shot all-reduce of the partials + residual, over peer memory
            K.allreduce_residual_f32(part, residual, self.tp.p2p_tc, out=out)
            return
        self.tp.all_reduce_sum(part)
        K.residual_add_f32(residual, part, out=out)

    # ------------------------------------------------------------------
    def reset(self) -> None:
        self.kv.reset()

    def prefill(self, prompt_ids: torch.Tensor) -> torch.Tensor:
        """Run ``prompt_ids [B, P]`` through the stack; returns the first greedy token per sequence ``[B]``.

        The prompt runs in chunks of ``T // B`` tokens per sequence; the head
        runs once, on the last position.
        """
        if prompt_ids.dim() != 2 or prompt_ids.shape[0] != self.B:
            raise ValueError(f"prompt_ids must be [{self.B}, P]")
        ids = prompt_ids.to(self.rt.device, torch.int64)
        P = ids.shape[1]
        start = self.kv.sequence_lens[0]
        if start + P > self.S:
            raise ValueError(f"prompt of {P} tokens does not fit: cursor {start}, max_seq {self.S}")
        chunk = max(1, self.T // self.B)
        for c0 in range(0, P, chunk):
            c1 = min(P, c0 + chunk)
            q = c1 - c0
            self.arenas.ids[:self.B * q].copy_(ids[:, c0:c1].reshape(-1))
            self._forward(q, head=(c1 == P))
            self.kv.note_advanced(q)
        return self.arenas.ids[:self.B].clone()

    def set_next_ids(self, ids: torch.Tensor) -> None:
        self.arenas.ids[:self.B].copy_(ids.reshape(-1).to(self.arenas.ids.device))

    def _decode_once(self) -> None:
        self._forward(1, head=True)

    def capture(self) -> None:
        """Capture one decode step (q_len 1 + head + cursor advance) as a CUDA graph."""
        a = self.arenas
        saved_pos = self.kv.cache_pos.clone()
        saved_ids = a.ids[:self.B].clone()
        self._decode_once()  # eager warm-up: sets kernel attributes, resolves symbols
        torch.cuda.synchronize()
        self.kv.cache_pos.copy_(saved_pos)
        a.ids[:self.B].copy_(saved_ids)
        graph = torch.cuda.CUDAGraph()
        stream = torch.cuda.Stream()
        stream.wait_stream(torch.cuda.current_stream())
        with torch.cuda.graph(graph, stream=stream):
            self._decode_once()
        torch.cuda.current_stream().wait_stream(stream)
        torch.cuda.synchronize()
        self.graph = graph

    # ------------------------------------------------------------------
    # speculative verify (runtime_loop.py:651-916)
    # ------------------------------------------------------------------
    def _verify_once(self, k: int, draft_cache_pos: torch.Tensor | None = None,
                     out_tokens: torch.Tensor | None = None, out_len: torch.Tensor | None = None) -> None:
        self._forward(k + 1, head="all", advance=False)
        K.spec_accept(self.arenas.ids, self.verdict, self.B, k, next_ids=self.next_ids, accepted=self.accepted,
                      cache_pos=self.kv.cache_pos, draft_cache_pos=draft_cache_pos, out_tokens=out_tokens,
                      out_len=out_len)

    def verify_inputs(self, k: int) -> torch.Tensor:
        """View ``[B, k + 1]`` of the verify input ids: column 0 holds each
        sequence's current token (kept by the accept kernel), columns 1..k the
        proposals the caller writes before :meth:`verify_step`."""
        return self.arenas.ids[:self.B * (k + 1)].view(self.B, k + 1)

    def verify_step(self, k: int) -> None:
        """One target verify pass over ``[current, d1..dk]`` per sequence plus the
        greedy-exact accept / reject, all on the device (graph replay once captured).

        Results: ``next_ids [B]`` (the next current token), ``accepted [B]``
        (proposals kept), the cursors moved by ``accepted + 1``, ``verdict``.
        The host's cursor mirror is not updated (that would need a sync); call
        :meth:`sync_cursors` to refresh it.
        """
        if self.B * (k + 1) > self.T:
            raise ValueError(f"verify of {self.B} x {k + 1} tokens exceeds the {self.T}-token step")
        if max(self.kv.sequence_lens) + k + 1 > self.S:
            raise ValueError("KV cache is full")
        if self.use_graph and k not in self.verify_graphs:
            a = self.arenas
            saved = (self.kv.cache_pos.clone(), a.ids.clone())
            self._verify_once(k)  # eager warm-up
            torch.cuda.synchronize()
            self.kv.cache_pos.copy_(saved[0])
            a.ids.copy_(saved[1])
            graph = torch.cuda.CUDAGraph()
            stream = torch.cuda.Stream()
            stream.wait_stream(torch.cuda.current_stream())
            with torch.cuda.graph(graph, stream=stream):
                self._verify_once(k)
            torch.cuda.current_stream().wait_stream(stream)
            torch.cuda.synchronize()
            self.verify_graphs[k] = graph
        if self.use_graph:
            self.verify_graphs[k].replay()
        else:
            self._verify_once(k)
        # conservative host bound until the next sync_cursors()
        self.kv.sequence_lens = [n + k + 1 for n in self.kv.sequence_lens]
        self._unsynced = True

    def sync_cursors(self) -> list[int]:
        """Read the device cursors back (a host sync) into the host mirror."""
        lens = [int(v) for v in self.kv.cache_pos.tolist()]
        self.kv.set_sequence_lens(lens)
        self._unsynced = False
        return lens

    def decode_step(self) -> None:
        """Enqueue one decode step (graph replay when captured)."""
        if self.kv.sequence_lens[0] + 1 > self.S:
            raise ValueError("KV cache is full")
        if self.use_graph and self.graph is None:
            self.capture()
        if self.graph is not None:
            self.graph.replay()
        else:
            self._decode_once()
        self.kv.note_advanced(1)

    def last_head_rows(self) -> torch.Tensor:
        """The final-layer hidden rows ``[B, H]`` the greedy head consumed in the last step."""
        return self._head_rows

    @property
    def current_ids(self) -> torch.Tensor:
        return self.arenas.ids[:self.B]

    def generate(self, prompt_ids: torch.Tensor, new_tokens: int) -> torch.Tensor:
        """Prefill then greedy-decode; returns ``[B, new_tokens]`` (first token from the prefill)."""
        first = self.prefill(prompt_ids)
        out = [first]
        for _ in range(new_tokens - 1):
            self.decode_step()
            out.append(self.current_ids.clone())
        return torch.stack(out, dim=1)

    def kernel_launches_per_step(self) -> int:
        """Kernels one decode step launches (embedding, layers, head, cursor advance)."""
        per_layer = (9 if self.gu_plain else 8) if self.backend == "tc" else 5  # CUDA cores: attention takes the q/k norm
        head = 3 if self.backend == "tc" else 1
        if self.tp is not None:  # + all-reduce / residual-add kernels after each row-split linear, + keys-to-ids
            if self.tp.p2p is None or self.backend == "tc":
                per_layer += 2
            if self.tp.p2p is None and self.backend == "tc":  # + the local split sums before NCCL
                per_layer += 2
            head += 1
        return 1 + per_layer * len(self.rt.layers) + head + 1

    def collectives_per_step(self) -> int:
        """NCCL all-reduces one decode step issues (0 on one GPU; the fused
        all-reduce of the CUDA-core linears is not counted)."""
        if self.tp is None:
            return 0
        fused = self.tp.p2p is not None  # CUDA-core: in the linear; tensor cores: one-shot kernel after it
        return (0 if fused else 2 * len(self.rt.layers)) + 1
