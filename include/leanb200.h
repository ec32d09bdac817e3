/*
 * leanb200.h — C ABI of libleanb200.so, the B200 (sm_100a) kernels behind the
 * leanstack decode hot path.
 *
 * Every entry point takes raw device pointers, int64 sizes and a CUDA stream
 * (passed as void*), enqueues its work on that stream, and returns an
 * ls_status code.  Nothing here allocates device memory: outputs and
 * workspaces are caller-provided (the resident arenas of the buffer planner).
 * Errors are returned as codes, never by aborting; ls_last_error() describes
 * the most recent failure of the calling thread.  Every call is valid inside
 * CUDA stream capture.
 *
 * Tensor layouts (bf16 unless stated, row-major, innermost dimension last):
 *   hidden / residual     [m, hidden]                 m = batch * q_len tokens
 *   weights               [out_features, in_features] (torch nn.Linear layout)
 *   fused qkv weight      [(Hq + 2*Hkv) * D, hidden]  rows: q heads, k heads, v heads
 *   fused gate_up weight  [2 * I, hidden]             rows: gate, then up
 *   q (rotated)           [m, Hq, D]
 *   attention output      [m, Hq * D]
 *   K / V cache (1 layer) [batch, Hkv, max_seq, D]
 *   rope cos / sin        [rope_len, D / 2]           the reference's bf16 position cache; row r
 *                         holds position rope_offset + r
 *   cache_pos             int32 [batch] on device:    cached positions of each sequence
 *                         before this call; token i of sequence b sits at
 *                         position cache_pos[b] + i and attends keys 0..cache_pos[b]+i.
 *                         Where an entry point also takes uniform_past, cache_pos may be
 *                         NULL and every sequence then uses cache_pos[b] = uniform_past
 *                         (the reference's per-layer host cursor, kv_cache.py:219).
 */
#ifndef LEANB200_H
#define LEANB200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define LS_ABI_VERSION 1

typedef enum ls_status {
  LS_OK = 0,
  LS_ERR_INVALID_ARGUMENT = 1,  /* null pointer, non-positive size */
  LS_ERR_UNSUPPORTED_SHAPE = 2, /* shape outside what the kernels implement */
  LS_ERR_MISALIGNED = 3,        /* pointer not 16-byte aligned / size not a multiple of 8 */
  LS_ERR_WORKSPACE = 4,         /* workspace null or too small */
  LS_ERR_CUDA = 5,              /* a CUDA runtime call failed */
  LS_ERR_KV_OVERFLOW = 6,       /* a KV position beyond max_seq (device-detected) */
  LS_ERR_TIMEOUT = 7,           /* a bounded device-side wait ran out */
  LS_ERR_NOT_SUPPORTED = 8      /* feature not available on this device */
} ls_status;

/* Exchange regions of the fused one-shot tensor-parallel all-reduce: every
 * rank's region (its own at index `rank`), mapped into this process with
 * ls_ipc_open.  Region layout: per-(source rank, CTA) flags, per-CTA call
 * counters, then two slots of [world][max_rows][width] fp32 partials. */
#define LS_MAX_TP_RANKS 8
typedef struct ls_p2p_exchange {
  void* peer[LS_MAX_TP_RANKS];
  int32_t rank;
  int32_t world;
  int32_t max_ctas;
  int32_t max_rows;
  int64_t width;
  unsigned long long* trace;  /* optional (NULL): per CTA 4 globaltimer stamps of the last call, for profiling */
} ls_p2p_exchange;

/* Epilogues of ls_linear_bf16. */
typedef enum ls_epilogue {
  LS_EPI_STORE = 0,     /* out = bf16(W x) */
  LS_EPI_RESIDUAL = 1,  /* out = bf16(residual + bf16(W x)) */
  LS_EPI_SILU_MUL = 2,  /* W = [gate; up] (2I rows): out[I] = bf16(bf16(silu(bf16 g)) * bf16 u) */
  LS_EPI_STORE_F32 = 4, /* out (float*) = W x unrounded: the partial of a tensor-parallel row-split linear */
  LS_EPI_SPLIT_F32 = 8  /* tcgen05 GEMM only: out (float*) = [splits][m][n] per-split unrounded sums of W x
                           (ls_gemm_bf16_tcgen05_splits); the consumer adds them in split order */
} ls_epilogue;

typedef void* ls_stream_t; /* a cudaStream_t */

/* Library version (LS_ABI_VERSION) and the last error message of this thread. */
int ls_version(void);
const char* ls_last_error(void);

/* Read (and optionally clear) the device-side error flag that kernels set when
 * they skip an out-of-range access or a bounded wait runs out (LS_ERR_TIMEOUT
 * in the low byte, the wait site above it).  Synchronizes the current device.
 * No counterpart in the reference, whose eager torch path has no device-side
 * waits; its nearest failure handling is the ValueError cursor checks of
 * src/leanstack/runtime/kv_cache.py:100-103. */
int ls_get_device_error(int* code, int clear);

/* Limit, in ns, of every bounded spin-wait in the kernels (mbarrier waits,
 * split-K counters, the fused all-reduce's peer wait, the persistent step's
 * grid barrier) on the current device; 2 s by default, 1 us .. 60 s accepted.
 * A wait that runs out records LS_ERR_TIMEOUT, the kernel drains and returns,
 * and the context stays usable.  Synchronizes the device first.  For failure
 * tests and for callers that must learn of a lost peer sooner. */
int ls_set_wait_limit_ns(int64_t ns);
int ls_get_wait_limit_ns(int64_t* ns);

/* Number of SMs of the current device (grid sizing is a multiple of it). */
int ls_sm_count(int* out);

/*
 * x[m] = embed[ids[m]] — the embedding lookup of run_semantic_stack_decode
 * (reference: src/leanstack/runtime/qwen_explicit.py:1623, F.embedding).
 * ids: int64 [m] on device.
 */
int ls_embed_gather(const int64_t* ids, int64_t m, const void* embed, int64_t vocab, int64_t hidden,
                    void* out, ls_stream_t stream);

/*
 * Skinny linear on the CUDA cores for m <= 8 activation rows, with an optional
 * RMSNorm prologue over x (norm_w == NULL: none) and one of ls_epilogue.
 * For LS_EPI_SILU_MUL, n is the number of weight rows (2I) and out has n/2
 * columns.  Replaces the torch.mv / F.linear calls of the reference's
 * dispatch helpers (src/leanstack/runtime/qwen_explicit.py:787, :913, :942-948).
 */
int ls_linear_bf16(const void* x, int64_t m, int64_t k, const void* norm_w, float eps, const void* w, int64_t n,
                   int epilogue, const void* residual, void* out, ls_stream_t stream);

/*
 * Input RMSNorm + fused QKV projection + per-head q/k RMSNorm + NeoX RoPE +
 * KV append, for m = batch * q_len tokens.
 * Replaces _semantic_attention_qkv_vector / _semantic_attention_qkv
 * (src/leanstack/runtime/qwen_explicit.py:733-806) followed by
 * StaticKVBlockManager.append (src/leanstack/runtime/kv_cache.py:222-243).
 *   input_norm_w  NULL if x is already normed (the reference helper's input)
 *   k_cache/v_cache  layer slice [batch, Hkv, max_seq, D], or NULL to skip the append
 *   k_out/v_out   optional [m, Hkv, D] copies of the rotated k and raw v (NULL: skip)
 *   qkv_scratch   [m, (Hq + 2 Hkv) D] raw projection (caller workspace)
 *   q_out         [m, Hq, D] normed + rotated q
 */
int ls_rmsnorm_qkv_rope_kvappend(const void* x, int64_t batch, int64_t q_len, int64_t hidden,
                                 const void* input_norm_w, float eps, const void* qkv_w, int64_t num_heads,
                                 int64_t num_kv_heads, int64_t head_dim, const void* q_norm_w,
                                 const void* k_norm_w, const void* rope_cos, const void* rope_sin,
                                 int64_t rope_len, int64_t rope_offset, const int32_t* cache_pos,
                                 int64_t uniform_past, void* k_cache,
                                 void* v_cache, int64_t max_seq, void* k_out, void* v_out, void* qkv_scratch,
                                 void* q_out, ls_stream_t stream);

/* Large-M GEMM for prefill (m in the thousands; config 5: m = 65536):
 * out[m, n] = epilogue(x[m, k] . W[n, k]^T) with the epilogues of
 * ls_gemm_bf16_tcgen05, replacing the F.linear calls of the prefill layer
 * (src/leanstack/runtime/qwen_explicit.py:809-829, :1093-1144).  Persistent
 * tcgen05 kernel: 128 weight rows x 256 activation rows per tile (128 for
 * SILU_MUL), the whole K per tile, tiles visited in L2-sized bands.  No
 * workspace.  k a multiple of 8. */
int ls_gemm_bf16_tcgen05_big(const void* x, int64_t m, int64_t k, const void* w, int64_t n, int epilogue,
                             const void* residual, void* out, ls_stream_t stream);

/* The same GEMM over weights pre-tiled once by ls_gemm_tc_tile_weight (the
 * leanpack-v1 tile layout): [ceil(n/128)][ceil(k/64)] tiles of 128 rows x 64 k,
 * each the 16 KB shared-memory image the MMA reads (128-byte swizzle), rows
 * past n and columns past k zero; for SILU_MUL the gate half is tiled first,
 * then the up half.  Every weight tile arrives as one contiguous bulk copy
 * instead of a 128-row strided TMA box.  n_rows as in the untiled call (2n for
 * SILU_MUL). */
int ls_gemm_tc_tiled_bytes(int64_t n_rows, int64_t k, int silu, int64_t* bytes);
int ls_gemm_tc_tile_weight(const void* w, int64_t n_rows, int64_t k, int silu, void* out, ls_stream_t stream);
int ls_gemm_bf16_tcgen05_tiled(const void* x, int64_t m, int64_t k, const void* w_tiled, int64_t n, int epilogue,
                               const void* residual, void* out, void* workspace, int64_t workspace_bytes,
                               ls_stream_t stream);

/*
 * The second half of ls_rmsnorm_qkv_rope_kvappend on a precomputed fused
 * projection qkv [m, (Hq + 2 Hkv) D]: per-head q/k RMSNorm, NeoX RoPE and the
 * K/V append (src/leanstack/runtime/qwen_explicit.py:793-806, :690-716;
 * src/leanstack/runtime/kv_cache.py:222-243).  Used after
 * ls_gemm_bf16_tcgen05 computes the projection for larger batches.
 */
int ls_qk_norm_rope_kvappend(const void* qkv, int64_t batch, int64_t q_len, int64_t num_heads, int64_t num_kv_heads,
                             int64_t head_dim, const void* q_norm_w, const void* k_norm_w, float eps,
                             const void* rope_cos, const void* rope_sin, int64_t rope_len, int64_t rope_offset,
                             const int32_t* cache_pos, int64_t uniform_past, void* k_cache, void* v_cache,
                             int64_t max_seq, void* k_out, void* v_out, void* q_out, ls_stream_t stream);
/* The same on the split fp32 partials of the QKV projection
 * (ls_gemm_bf16_tcgen05 with LS_EPI_SPLIT_F32): qkv = bf16(sum over the
 * splits in order) first, the rounding of the reference's F.linear
 * (src/leanstack/runtime/qwen_explicit.py:748). */
int ls_qk_norm_rope_kvappend_splits(const float* qkv_part, int64_t splits, int64_t batch, int64_t q_len,
                                    int64_t num_heads, int64_t num_kv_heads, int64_t head_dim, const void* q_norm_w,
                                    const void* k_norm_w, float eps, const void* rope_cos, const void* rope_sin,
                                    int64_t rope_len, int64_t rope_offset, const int32_t* cache_pos,
                                    int64_t uniform_past, void* k_cache, void* v_cache, int64_t max_seq, void* k_out,
                                    void* v_out, void* q_out, ls_stream_t stream);

/*
 * Row-wise argmax of bf16 logits [m, n] (lowest index on ties): the
 * reference's `logits.argmax(dim=-1)` (src/leanstack/runtime/qwen_explicit.py:960)
 * for logits produced by ls_gemm_bf16_tcgen05.  out_ids: int64 [m].
 * workspace: ls_argmax_rows_workspace_bytes() bytes, zero-filled once.
 */
int ls_argmax_rows(const void* logits, int64_t m, int64_t n, int64_t* out_ids, void* workspace,
                   int64_t workspace_bytes, ls_stream_t stream);
int ls_argmax_rows_workspace_bytes(int64_t m, int64_t n, int64_t* bytes);

/*
 * GQA attention of q [m, Hq, D] over the cache (keys 0..cache_pos[b]+i for
 * token i of sequence b).  Below 256 query rows per (sequence, kv head) the
 * keys are split over the sequence on the tensor cores and merged inside a
 * thread-block cluster: decode (q_len 1, unmasked) and verify (q_len k+1 with
 * the decode mask of src/leanstack/runtime/qwen_explicit.py:551-563).  From
 * 256 rows (prefill, causal) a CTA owns 128 rows and walks the keys once with
 * tcgen05 products (S and O in tensor memory).  Replaces the SDPA calls at
 * src/leanstack/runtime/qwen_explicit.py:886-903 and :1000-1039.  Cache
 * positions past cache_pos[b] + q_len are never read into the result.
 * workspace: ls_decode_attention_workspace_bytes() bytes (currently 0; the
 * argument is kept so that a caller's buffer plan stays valid).
 */
int ls_decode_attention(const void* q, const void* k_cache, const void* v_cache, const int32_t* cache_pos,
                        int64_t uniform_past, int64_t batch, int64_t q_len, int64_t num_heads, int64_t num_kv_heads, int64_t head_dim,
                        int64_t max_seq, float scale, void* out, void* workspace, int64_t workspace_bytes,
                        ls_stream_t stream);
int ls_decode_attention_workspace_bytes(int64_t batch, int64_t q_len, int64_t num_heads, int64_t num_kv_heads,
                                        int64_t head_dim, int64_t max_seq, int64_t* bytes);
/* One decode token per sequence from the raw fused projection qkv [batch,
 * (Hq + 2 Hkv) D] (bf16, as ls_linear_bf16 writes it): the per-head q/k
 * RMSNorm and NeoX RoPE of ls_qk_norm_rope_kvappend (bit for bit), the K/V
 * append at cache_pos[b], and the attention of ls_decode_attention over keys
 * 0..cache_pos[b], in one launch.  Replaces, for the bs1 / small-batch decode
 * step, src/leanstack/runtime/qwen_explicit.py:733-806 (q/k norm, RoPE),
 * src/leanstack/runtime/kv_cache.py:247-254 (append_and_get) and the SDPA at
 * qwen_explicit.py:886-903.  num_heads / num_kv_heads <= 16; q is not written
 * out.  A position outside the cache or the rope table sets
 * LS_ERR_KV_OVERFLOW on the device and appends nothing.  The kernel starts
 * under programmatic dependent launch and reads cache_pos, the cache rows
 * before it, the rope table and the norm weights before it waits for the
 * previous kernel in the stream; only qkv is read after the wait.  So those
 * must not be written by a kernel that may still run when this one starts
 * (a kernel that lets its dependents launch before it ends). */
int ls_decode_attention_qkv(const void* qkv, int64_t batch, int64_t num_heads, int64_t num_kv_heads,
                            int64_t head_dim, const void* q_norm_w, const void* k_norm_w, float eps,
                            const void* rope_cos, const void* rope_sin, int64_t rope_len, int64_t rope_offset,
                            const int32_t* cache_pos, int64_t uniform_past, void* k_cache, void* v_cache,
                            int64_t max_seq, float scale, void* out, ls_stream_t stream);

/* h = residual + bf16(o_w attn): o_proj with the residual epilogue
 * (src/leanstack/runtime/qwen_explicit.py:913 and :1262, :819-820). */
int ls_oproj_residual(const void* attn, int64_t m, int64_t k, const void* o_w, int64_t n, const void* residual,
                      void* out, ls_stream_t stream);

/* act = silu(gate) * up of the post-attention-normed h
 * (src/leanstack/runtime/qwen_explicit.py:932-947, :821-828). */
int ls_rmsnorm_gateup_silu(const void* h, int64_t m, int64_t hidden, const void* post_norm_w, float eps,
                           const void* gate_up_w, int64_t intermediate, void* out, ls_stream_t stream);

/* out = residual + bf16(down_w act) (src/leanstack/runtime/qwen_explicit.py:947-949, :829). */
int ls_down_residual(const void* act, int64_t m, int64_t intermediate, const void* down_w, int64_t hidden,
                     const void* residual, void* out, ls_stream_t stream);

/*
 * Greedy head: final RMSNorm + lm_head + argmax over the bf16-rounded logits,
 * lowest index on ties, for each of m rows.  out_ids: int64 [m] on device.
 * Replaces select_semantic_greedy_token's torch head
 * (src/leanstack/runtime/qwen_explicit.py:952-960, :1814-1832) and the cuTile
 * cutile_logits_argmax (src/leanstack/runtime/cutile_logits.py:37-69).
 * workspace: ls_lmhead_workspace_bytes() bytes, zero-filled once before first use.
 */
int ls_lmhead_argmax(const void* h, int64_t m, int64_t hidden, const void* final_norm_w, float eps,
                     const void* lm_head_w, int64_t vocab, int64_t* out_ids, void* workspace,
                     int64_t workspace_bytes, ls_stream_t stream);
int ls_lmhead_workspace_bytes(int64_t m, int64_t vocab, int64_t* bytes);

/* ls_lmhead_argmax without a caller workspace; it allocates no device memory.
 * No counterpart in the reference: it is for callers that cannot allocate on
 * the token-selection path (an FFI host with no device allocator of its own, or
 * a server whose HBM plan is fixed at start-up).  Its scratch is a fixed 16 KiB
 * array per device inside this library; a call that would need more (m rows x
 * head-grid CTAs) fails with LS_ERR_WORKSPACE.  Every call looks up the
 * array's device address (host-side, no allocation); the first call that sees
 * an address on a device clears the arrival counter and waits for that on
 * `stream`: make it before any stream capture and let it finish before other
 * calls on the device start.  Calls that overlap on the GPU share the scratch
 * and race: serialise them on one stream. */
int ls_lmhead_argmax_noalloc(const void* h, int64_t m, int64_t hidden, const void* final_norm_w, float eps,
                             const void* lm_head_w, int64_t vocab, int64_t* out_ids, ls_stream_t stream);

/*
 * Weight-streaming GEMM on the tcgen05 tensor cores for 1 <= m <= 128
 * activation rows (larger batches run as several launches): out[m, n] = epilogue(x[m, k] . w[n, k]^T) with epilogue one
 * of ls_epilogue.  For LS_EPI_SILU_MUL, w is the fused [2 n, k] gate_up matrix
 * and out is [m, n].  This is the batched-decode / speculative-verify form of
 * the reference's F.linear calls (src/leanstack/runtime/qwen_explicit.py:748,
 * :819-829) and of the cuTile GEMM it benchmarks
 * (experiments/cutile/qwen_bf16_hot_kernels.py:19-36).  workspace:
 * ls_gemm_bf16_tcgen05_workspace_bytes() bytes, zero-filled once before first
 * use (tile counters are left at zero).
 */
int ls_gemm_bf16_tcgen05(const void* x, int64_t m, int64_t k, const void* w, int64_t n, int epilogue,
                         const void* residual, void* out, void* workspace, int64_t workspace_bytes,
                         ls_stream_t stream);
int ls_gemm_bf16_tcgen05_workspace_bytes(int64_t m, int64_t k, int64_t n, int epilogue, int64_t* bytes);
/* Number of k-splits of the LS_EPI_SPLIT_F32 form: its out holds splits * m * n
 * floats and the call needs no workspace (NULL is accepted).  The split form
 * leaves the cross-split sum to the next kernel (ls_residual_rmsnorm_splits,
 * ls_qk_norm_rope_kvappend_splits) instead of reducing partials inside the
 * GEMM behind a grid-wide wait: the decode step's QKV, o_proj and down. */
int ls_gemm_bf16_tcgen05_splits(int64_t m, int64_t k, int64_t n, int64_t* splits);

/* Fused one-shot all-reduce over NVLink peer memory (no counterpart in the
 * reference, which runs on one GPU; it replaces the NCCL all-reduce of the
 * tensor-parallel row-split o_proj / down_proj, whose reference-side linear +
 * residual is src/leanstack/runtime/qwen_explicit.py:1262 and :819-829).
 * out = bf16(residual + bf16(sum over ranks of W_r x_r)), m <= 8 rows: each CTA
 * computes its slice of the fp32 partial and stores every value into every
 * rank's region together with the CTA's call number (one 8-byte plain peer
 * store per value and rank, no multicast), then polls its own elements until
 * every rank's call number matches (bounded by the wait limit, then
 * LS_ERR_TIMEOUT in the device error flag) and sums in rank order, so every
 * rank holds the same bits.  All ranks must issue the same sequence of these
 * calls with the same m, and each rank must own its GPU.  Regions hold up to
 * 128 rows. */
int ls_p2p_region_bytes(int64_t max_rows, int64_t width, int64_t max_ctas, int64_t* bytes);
int ls_p2p_alloc(int64_t bytes, void** region);   /* cudaMalloc + zero, at set-up */
int ls_p2p_free(void* region);
int ls_ipc_get_handle(void* region, void* handle64);  /* 64-byte cudaIpcMemHandle_t */
int ls_ipc_open(const void* handle64, void** region);
int ls_ipc_close(void* region);
int ls_linear_allreduce_residual(const void* x, int64_t m, int64_t k, const void* w, int64_t n,
                                 const void* residual, void* out, const ls_p2p_exchange* ex, ls_stream_t stream);
/* The same one-shot all-reduce for partials another kernel wrote: part is the
 * fp32 [m, n] partial of this rank's row-split linear (the tcgen05 GEMM's
 * LS_EPI_STORE_F32 output, 1 <= m <= ex->max_rows), out = bf16(residual +
 * bf16(sum over ranks in rank order)).  Replaces an NCCL all-reduce of the
 * partials plus ls_residual_add_f32 (the reference's o_proj / down residual,
 * src/leanstack/runtime/qwen_explicit.py:819-829).  Fixed grid of 128 CTAs:
 * use an exchange of its own (not shared with ls_linear_allreduce_residual),
 * with max_ctas >= 128. */
int ls_allreduce_residual_f32(const float* part, int64_t m, int64_t n, const void* residual, void* out,
                              const ls_p2p_exchange* ex, ls_stream_t stream);
/* The same over the split partials of a row-split linear run in the
 * LS_EPI_SPLIT_F32 form (part = [splits][m][n]): each rank adds its splits in
 * order, then the ranks' sums are exchanged and added in rank order. */
int ls_allreduce_residual_splits(const float* part, int64_t splits, int64_t m, int64_t n, const void* residual,
                                 void* out, const ls_p2p_exchange* ex, ls_stream_t stream);
/* out[i] = sum over the splits of part[s][i] (n elements per split), in split
 * order: the local sum before an NCCL all-reduce of a row-split linear's
 * split partials (no counterpart in the reference, which runs on one GPU). */
int ls_sum_splits_f32(const float* part, int64_t splits, int64_t n, float* out, ls_stream_t stream);

/* Tensor-parallel greedy head.  Each rank holds a vocab shard (rows
 * [vocab_offset, vocab_offset + vocab_rows) of lm_head) and writes, per row, an
 * int64 key of its best (bf16 logit, vocab id): a signed MAX over the ranks'
 * keys (one all-reduce of m int64) selects the largest logit and, on equal
 * logits, the lowest id -- the tie rule of torch.argmax in
 * select_semantic_greedy_token (src/leanstack/runtime/qwen_explicit.py:952-960).
 * ls_argmax_keys_to_ids turns the reduced keys back into ids. */
int ls_lmhead_argmax_keys(const void* h, int64_t m, int64_t hidden, const void* final_norm_w, float eps,
                          const void* lm_head_w, int64_t vocab_rows, int64_t vocab_offset, int64_t* out_keys,
                          void* workspace, int64_t workspace_bytes, ls_stream_t stream);
int ls_argmax_rows_keys(const void* logits, int64_t m, int64_t n, int64_t vocab_offset, int64_t* out_keys,
                        void* workspace, int64_t workspace_bytes, ls_stream_t stream);
int ls_argmax_keys_to_ids(const int64_t* keys, int64_t m, int64_t* out_ids, ls_stream_t stream);

/* out = bf16(residual + bf16(y)) over n elements, y fp32: the residual epilogue
 * of o_proj / down applied after the tensor-parallel all-reduce of their
 * fp32 partials (src/leanstack/runtime/qwen_explicit.py:819-829, :1262). */
int ls_residual_add_f32(const void* residual, const float* y, int64_t n, void* out, ls_stream_t stream);

/* Standalone RMSNorm over the last dim, bf16((x * rsqrt(mean(x^2) + eps)) * w),
 * for m rows of length n (src/leanstack/runtime/qwen_explicit.py:621-637). */
int ls_rmsnorm(const void* x, int64_t m, int64_t n, const void* w, float eps, void* out, ls_stream_t stream);

/* Residual add of a linear's split partials (LS_EPI_SPLIT_F32), then RMSNorm:
 * out_residual = bf16(residual + bf16(sum over the splits of part[s][m][n]))
 * (the o_proj / down residual of src/leanstack/runtime/qwen_explicit.py:819-829,
 * :852) and, when norm_w is not NULL, out_norm = the RMSNorm of out_residual
 * (:621-637), the post-attention / next input / final norm that follows. */
int ls_residual_rmsnorm_splits(const float* part, int64_t splits, int64_t m, int64_t n, const void* residual,
                               const void* norm_w, float eps, void* out_residual, void* out_norm,
                               ls_stream_t stream);

/* SiLU(gate) * up over the split partials of the fused gate_up projection run
 * as a plain [2I, k] linear (LS_EPI_SPLIT_F32, part = [splits][m][2I]):
 * act[m, I] = bf16(bf16(silu(bf16(g))) * bf16(u)), the MLP epilogue of
 * src/leanstack/runtime/qwen_explicit.py:932-949.  With whole-K tiles (one
 * split when the gate_up rows give at least one 128-row tile per SM) the
 * GEMM needs no cross-CTA reduction at all. */
int ls_silu_mul_splits(const float* part, int64_t splits, int64_t m, int64_t intermediate, void* act,
                       ls_stream_t stream);

/* cache_pos[b] += delta[b] (delta NULL: += q_len): moves the device cursors
 * after a step, the device-side counterpart of the reference's host cursor
 * bookkeeping (src/leanstack/runtime/kv_cache.py:239-245, :298-318). */
int ls_advance_cursors(int32_t* cache_pos, const int32_t* delta, int64_t batch, int64_t q_len, ls_stream_t stream);

/* Greedy-exact accept / reject after a speculative verify pass, on the device
 * (experiments/models/qwen_explicit_runtime_loop.py:804-862).  ids: int64
 * [batch, k+1] = [current, d1..dk] per sequence (the verify input); verdict:
 * int64 [batch, k+1], the target's greedy token after each input position.
 * Per sequence: n = length of the prefix with d(i+1) == verdict[i]; the next
 * current token is verdict[n] (correction, or bonus when n == k), written to
 * next_ids[b] and to ids[b][0]; accepted[b] = n; cache_pos[b] += n + 1 (the
 * verifier cursor rollback of :836-838); draft_cache_pos[b] -= k - min(n+1, k)
 * (the draft consumed current, d1..d(k-1) while proposing and keeps current
 * plus the accepted proposals, :833); the committed tokens d1..dn, next are
 * appended to out_tokens[b][out_len[b]...] up to out_cap (:856-866).  Every
 * output pointer may be NULL. */
int ls_spec_accept(int64_t* ids, const int64_t* verdict, int64_t batch, int64_t k, int64_t* next_ids,
                   int32_t* accepted, int32_t* cache_pos, int32_t* draft_cache_pos, int64_t* out_tokens,
                   int32_t* out_len, int64_t out_cap, ls_stream_t stream);

#ifdef LEANB200_PROFILING
/* Measurement hooks, compiled only into a library built with
 * -DLEANB200_PROFILING (python -m leanstack_b200.build --profiling); the
 * release library exports none of them. */
/* NVLink latency probe of the exchange: `iters` flag round trips between rank 0 and
 * rank 1 through two 4-byte words (my_flag in this rank's region, peer_flag in
 * the other's, both zero and unused by the all-reduce), one thread, bounded
 * waits.  times_dev (device, 2 x u64): total ns, and 1 if a wait gave up. */
int ls_p2p_pingpong(void* my_flag, void* peer_flag, int rank, int iters, unsigned long long* times_dev,
                    ls_stream_t stream);
/* Profiling hook of ls_linear_bf16 and the fused head / all-reduce forms: with a
 * non-NULL device buffer of grid x 5 u64, every launch records per CTA the
 * globaltimer at start, after the PDL wait, after the activation prologue,
 * after the weight stream, and at the end.  NULL turns it off. */
int ls_linear_set_trace(void* buffer);
/* Profiling hook of ls_gemm_bf16_tcgen05(_tiled): with a non-NULL device buffer
 * of grid x 8 u64, each launch records per CTA the globaltimer at start, when
 * the first stage landed, after the last MMA issue, after the epilogue, and
 * for the first and the last split tile when its contributors were complete
 * and when this CTA's share was reduced (0 where there is none).  NULL turns
 * it off. */
int ls_gemm_tc_set_trace(void* buffer);
#endif /* LEANB200_PROFILING */

#ifdef __cplusplus
}
#endif

#endif /* LEANB200_H */
