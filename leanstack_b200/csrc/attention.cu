// Attention-side kernels of the decode / verify hot path (head_dim 128).
//
// 1. qk_norm_rope_append: per token and head, the q/k RMSNorm over head_dim,
//    the NeoX-half rotary embedding and the K/V append into the static cache
//    (reference: src/leanstack/runtime/qwen_explicit.py:733-806 and :690-716,
//    src/leanstack/runtime/kv_cache.py:222-243).  Rounding follows the
//    reference's bf16 torch ops: norm = bf16((x * r) * w); each RoPE product
//    and the sum / difference round to bf16.
// 2. decode_attention: the launcher of the tensor-core split-KV attention
//    (attention_tc.cu): GQA attention of the m = batch * q_len new tokens over
//    the cache.  Token i of sequence b sees keys 0 .. cache_pos[b] + i, which is
//    both the unmasked decode case (q_len 1) and the verify mask of
//    qwen_explicit.py:551-563.
#include "common.cuh"

namespace lsb {

constexpr int kHeadDim = 128;

struct QkRopeParams {
  const __nv_bfloat16* qkv;  // [M, (Hq + 2 Hkv) D], or null: the split partials below
  const float* part;         // [splits][M][(Hq + 2 Hkv) D] fp32 (tcgen05 GEMM, LS_EPI_SPLIT_F32)
  int splits;
  const __nv_bfloat16* q_norm_w;
  const __nv_bfloat16* k_norm_w;
  const __nv_bfloat16* cos;  // [rope_len, D/2]
  const __nv_bfloat16* sin;
  const int* cache_pos;      // [B] or null (then uniform_past)
  int uniform_past;
  __nv_bfloat16* q_out;      // [M, Hq, D]
  __nv_bfloat16* k_cache;    // [B, Hkv, S, D] or null
  __nv_bfloat16* v_cache;
  __nv_bfloat16* k_out;      // [M, Hkv, D] or null
  __nv_bfloat16* v_out;
  int* err;
  int q_len, Hq, Hkv, rope_len, rope_offset, max_seq;
  float eps;
};

// PART: the projection comes as split fp32 partials (p.part), else as bf16
// (p.qkv); two instances, so the bf16 one (prefill, one row per token and
// head over 65k tokens) keeps its registers low and its occupancy high.
template <bool PART>
__global__ void __launch_bounds__(128) qk_norm_rope_append_kernel(QkRopeParams p) {
  grid_dep_wait();
  grid_dep_launch();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int h = blockIdx.y * 4 + warp;
  if (h >= p.Hq + p.Hkv) return;
  const int t = blockIdx.x;
  const int b = t / p.q_len, i = t - b * p.q_len;
  const int pos = (p.cache_pos ? p.cache_pos[b] : p.uniform_past) + i;
  const bool is_q = h < p.Hq;
  const int hk = h - p.Hq;
  const int qkv_dim = (p.Hq + 2 * p.Hkv) * kHeadDim;
  const int e0 = lane * 4;
  // Four bf16 elements of the projection at column col of token t: loaded, or
  // the split partials summed in split order and rounded once.
  auto load4 = [&](int col) -> uint2 {
    if (!PART) return *reinterpret_cast<const uint2*>(p.qkv + (size_t)t * qkv_dim + col);
    const size_t slab = (size_t)gridDim.x * qkv_dim;
    const float* q = p.part + (size_t)t * qkv_dim + col;
    float4 a = __ldcg(reinterpret_cast<const float4*>(q));
    // Eight splits' loads in flight at a time, added in split order.
    for (int j0 = 1; j0 < p.splits; j0 += 8) {
      float4 v[8];
#pragma unroll
      for (int u = 0; u < 8; ++u)
        if (j0 + u < p.splits) v[u] = __ldcg(reinterpret_cast<const float4*>(q + (j0 + u) * slab));
#pragma unroll
      for (int u = 0; u < 8; ++u)
        if (j0 + u < p.splits) {
          a.x += v[u].x;
          a.y += v[u].y;
          a.z += v[u].z;
          a.w += v[u].w;
        }
    }
    __nv_bfloat162 lo = __floats2bfloat162_rn(a.x, a.y), hi = __floats2bfloat162_rn(a.z, a.w);
    return make_uint2(*reinterpret_cast<uint32_t*>(&lo), *reinterpret_cast<uint32_t*>(&hi));
  };

  const int row = pos - p.rope_offset;  // row of the cos/sin table
  if (pos < 0 || row < 0 || row >= p.rope_len || (!is_q && (p.k_cache != nullptr) && pos >= p.max_seq)) {
    if (lane == 0) raise_device_error(p.err, LS_ERR_KV_OVERFLOW);
    return;
  }

  const uint2 raw_u = load4(h * kHeadDim + e0);
  // A key head's V columns, fetched before the norm so both loads overlap.
  const uint2 v_u = is_q ? make_uint2(0u, 0u) : load4((h + p.Hkv) * kHeadDim + e0);
  const __nv_bfloat16* nw = is_q ? p.q_norm_w : p.k_norm_w;
  const uint2 w_u = *reinterpret_cast<const uint2*>(nw + e0);
  const int idx = lane < 16 ? e0 : e0 - kHeadDim / 2;
  const uint2 c_u = *reinterpret_cast<const uint2*>(p.cos + (size_t)row * (kHeadDim / 2) + idx);
  const uint2 s_u = *reinterpret_cast<const uint2*>(p.sin + (size_t)row * (kHeadDim / 2) + idx);
  const uint2 packed = head_norm_rope(raw_u, w_u, c_u, s_u, p.eps, lane);
  if (is_q) {
    *reinterpret_cast<uint2*>(p.q_out + ((size_t)t * p.Hq + h) * kHeadDim + e0) = packed;
    return;
  }
  if (p.k_cache) {
    const size_t off = (((size_t)b * p.Hkv + hk) * p.max_seq + pos) * kHeadDim + e0;
    *reinterpret_cast<uint2*>(p.k_cache + off) = packed;
    *reinterpret_cast<uint2*>(p.v_cache + off) = v_u;
  }
  if (p.k_out) {
    const size_t off = ((size_t)t * p.Hkv + hk) * kHeadDim + e0;
    *reinterpret_cast<uint2*>(p.k_out + off) = packed;
    *reinterpret_cast<uint2*>(p.v_out + off) = v_u;
  }
}

}  // namespace lsb

namespace lsb_host {
using namespace lsb;

static cudaLaunchConfig_t pdl_config(dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                                     cudaLaunchAttribute* attr) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cfg;
}

int launch_qk_norm_rope(const void* qkv, const float* part, int64_t splits, int64_t batch, int64_t q_len, int64_t hq, int64_t hkv, const void* qn,
                        const void* kn, const void* cos, const void* sin, int64_t rope_len, int64_t rope_offset,
                        const int32_t* cache_pos, int64_t uniform_past, void* k_cache, void* v_cache, int64_t max_seq, void* k_out, void* v_out, void* q_out,
                        float eps, cudaStream_t stream) {
  QkRopeParams p = {};
  p.qkv = static_cast<const __nv_bfloat16*>(qkv);
  p.part = part;
  p.splits = (int)splits;
  p.q_norm_w = static_cast<const __nv_bfloat16*>(qn);
  p.k_norm_w = static_cast<const __nv_bfloat16*>(kn);
  p.cos = static_cast<const __nv_bfloat16*>(cos);
  p.sin = static_cast<const __nv_bfloat16*>(sin);
  p.cache_pos = cache_pos;
  p.uniform_past = (int)uniform_past;
  p.q_out = static_cast<__nv_bfloat16*>(q_out);
  p.k_cache = static_cast<__nv_bfloat16*>(k_cache);
  p.v_cache = static_cast<__nv_bfloat16*>(v_cache);
  p.k_out = static_cast<__nv_bfloat16*>(k_out);
  p.v_out = static_cast<__nv_bfloat16*>(v_out);
  p.q_len = (int)q_len;
  p.Hq = (int)hq;
  p.Hkv = (int)hkv;
  p.rope_len = (int)rope_len;
  p.rope_offset = (int)rope_offset;
  p.max_seq = (int)max_seq;
  p.eps = eps;
  p.err = device_error_ptr();
  const int m = (int)(batch * q_len);
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = pdl_config(dim3(m, (unsigned)((hq + hkv + 3) / 4)), dim3(128), 0, stream, attr);
  cudaError_t e = qkv ? cudaLaunchKernelEx(&cfg, qk_norm_rope_append_kernel<false>, p)
                      : cudaLaunchKernelEx(&cfg, qk_norm_rope_append_kernel<true>, p);
  if (e != cudaSuccess) return set_error(LS_ERR_CUDA, "qk_norm_rope launch: %s", cudaGetErrorString(e));
  return LS_OK;
}

int attention_workspace_bytes(int64_t batch, int64_t q_len, int64_t hq, int64_t hkv, int64_t max_seq,
                              int64_t* bytes) {
  (void)batch, (void)q_len, (void)hq, (void)hkv, (void)max_seq;
  *bytes = 0;  // splits merge through distributed shared memory (attention_tc.cu)
  return LS_OK;
}

int launch_decode_attention_tc(const void* q, const void* k_cache, const void* v_cache, const int32_t* cache_pos,
                               int64_t uniform_past, int64_t batch, int64_t q_len, int64_t hq, int64_t hkv,
                               int64_t max_seq, float scale, void* out, cudaStream_t stream);

int launch_prefill_attention_tc(const void* q, const void* k_cache, const void* v_cache, const int32_t* cache_pos,
                                int64_t uniform_past, int64_t batch, int64_t q_len, int64_t hq, int64_t hkv,
                                int64_t max_seq, float scale, void* out, cudaStream_t stream);

// Query rows per (sequence, kv head) from which the 128-row tcgen05 prefill
// kernel (one pass over the keys per 128 rows) replaces the split-KV kernel.
constexpr int64_t kPrefillRows = 256;

int launch_decode_attention(const void* q, const void* k_cache, const void* v_cache, const int32_t* cache_pos,
                            int64_t uniform_past, int64_t batch, int64_t q_len, int64_t hq, int64_t hkv,
                            int64_t max_seq, float scale, void* out, void* workspace, int64_t workspace_bytes,
                            cudaStream_t stream) {
  (void)workspace;
  (void)workspace_bytes;
  if (q_len * (hq / hkv) >= kPrefillRows)
    return launch_prefill_attention_tc(q, k_cache, v_cache, cache_pos, uniform_past, batch, q_len, hq, hkv, max_seq,
                                       scale, out, stream);
  return launch_decode_attention_tc(q, k_cache, v_cache, cache_pos, uniform_past, batch, q_len, hq, hkv, max_seq,
                                    scale, out, stream);
}

}  // namespace lsb_host
