// Attention-side kernels of the decode / verify hot path (head_dim 128).
//
// 1. qk_norm_rope_append: per token and head, the q/k RMSNorm over head_dim,
//    the NeoX-half rotary embedding and the K/V append into the static cache
//    (reference: src/leanstack/runtime/qwen_explicit.py:733-806 and :690-716,
//    src/leanstack/runtime/kv_cache.py:222-243).  Rounding follows the
//    reference's bf16 torch ops: norm = bf16((x * r) * w); each RoPE product
//    and the sum / difference round to bf16.
// 2. decode_attention: GQA attention of the m = batch * q_len new tokens over
//    the cache, split over the sequence (flash-decoding).  Token i of sequence
//    b sees keys 0 .. cache_pos[b] + i, which is both the unmasked decode case
//    (q_len 1) and the verify mask of qwen_explicit.py:551-563.  Softmax runs in
//    fp32 (base-2 exponent); the last CTA of each (sequence, kv head) merges
//    the splits and writes bf16.
#include "common.cuh"

namespace lsb {

constexpr int kHeadDim = 128;

struct QkRopeParams {
  const __nv_bfloat16* qkv;  // [M, (Hq + 2 Hkv) D]
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
  const __nv_bfloat16* src = p.qkv + (size_t)t * qkv_dim + (size_t)h * kHeadDim;
  const int e0 = lane * 4;

  const int row = pos - p.rope_offset;  // row of the cos/sin table
  if (pos < 0 || row < 0 || row >= p.rope_len || (!is_q && (p.k_cache != nullptr) && pos >= p.max_seq)) {
    if (lane == 0) raise_device_error(p.err, LS_ERR_KV_OVERFLOW);
    return;
  }

  const uint2 raw_u = *reinterpret_cast<const uint2*>(src + e0);
  float raw[4] = {bf16_lo(raw_u.x), bf16_hi(raw_u.x), bf16_lo(raw_u.y), bf16_hi(raw_u.y)};
  float ss = raw[0] * raw[0] + raw[1] * raw[1] + raw[2] * raw[2] + raw[3] * raw[3];
  ss = warp_sum(ss);
  const float r = rsqrtf(ss / (float)kHeadDim + p.eps);
  const __nv_bfloat16* nw = is_q ? p.q_norm_w : p.k_norm_w;
  const uint2 w_u = *reinterpret_cast<const uint2*>(nw + e0);
  const float wv[4] = {bf16_lo(w_u.x), bf16_hi(w_u.x), bf16_lo(w_u.y), bf16_hi(w_u.y)};
  float n[4], other[4], o[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) n[j] = round_bf16((raw[j] * r) * wv[j]);
#pragma unroll
  for (int j = 0; j < 4; ++j) other[j] = __shfl_xor_sync(0xffffffffu, n[j], 16);
  const bool first_half = lane < 16;
  const int idx = first_half ? e0 : e0 - kHeadDim / 2;
  const uint2 c_u = *reinterpret_cast<const uint2*>(p.cos + (size_t)row * (kHeadDim / 2) + idx);
  const uint2 s_u = *reinterpret_cast<const uint2*>(p.sin + (size_t)row * (kHeadDim / 2) + idx);
  const float c[4] = {bf16_lo(c_u.x), bf16_hi(c_u.x), bf16_lo(c_u.y), bf16_hi(c_u.y)};
  const float s[4] = {bf16_lo(s_u.x), bf16_hi(s_u.x), bf16_lo(s_u.y), bf16_hi(s_u.y)};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    if (first_half) o[j] = round_bf16(round_bf16(n[j] * c[j]) - round_bf16(other[j] * s[j]));
    else o[j] = round_bf16(round_bf16(n[j] * c[j]) + round_bf16(other[j] * s[j]));
  }
  __nv_bfloat162 lo2 = __floats2bfloat162_rn(o[0], o[1]);
  __nv_bfloat162 hi2 = __floats2bfloat162_rn(o[2], o[3]);
  uint2 packed = make_uint2(*reinterpret_cast<uint32_t*>(&lo2), *reinterpret_cast<uint32_t*>(&hi2));
  if (is_q) {
    *reinterpret_cast<uint2*>(p.q_out + ((size_t)t * p.Hq + h) * kHeadDim + e0) = packed;
    return;
  }
  const uint2 v_u = *reinterpret_cast<const uint2*>(src + (size_t)p.Hkv * kHeadDim + e0);
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

// ---------------------------------------------------------------------------
// Split-KV decode / verify attention
//
// Grid (splits, Hkv * RG, B) with thread-block clusters of `splits` CTAs along
// x: the splits of one (sequence, kv head, row group) form one cluster.  Each
// CTA runs an online softmax over its share of the keys, leaves its partial
// (max, sum, output) in its own shared memory, and cluster rank 0 merges the
// partials through distributed shared memory after a cluster barrier.  No
// global workspace, fences or atomics are involved.
// ---------------------------------------------------------------------------
constexpr int kAttnWarps = 4;
constexpr int kAttnThreads = kAttnWarps * 32;
constexpr int kRT = 4;        // query rows per CTA
constexpr int kUK = 4;        // keys per warp per iteration (loads in flight)
constexpr int kMinChunk = 16; // keys per split at least
constexpr int kMaxSplits = 16;

struct AttnParams {
  const __nv_bfloat16* q;        // [M, Hq, D]
  const __nv_bfloat16* k_cache;  // [B, Hkv, S, D]
  const __nv_bfloat16* v_cache;
  const int* cache_pos;          // [B] or null (then uniform_past)
  int uniform_past;
  __nv_bfloat16* out;            // [M, Hq * D]
  int* err;
  int q_len, Hq, Hkv, G, R, RG, splits, max_seq;
  float scale_log2;
};

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\nbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ float ld_dsmem_f32(const float* local, uint32_t rank) {
  uint32_t remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(smem_u32(local)), "r"(rank));
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(remote) : "memory");
  return v;
}

__global__ void __launch_bounds__(kAttnThreads) decode_attention_kernel(AttnParams p) {
  __shared__ float sm_m[kAttnWarps][kRT];
  __shared__ float sm_l[kAttnWarps][kRT];
  __shared__ __align__(16) float sm_o[kAttnWarps][kRT][kHeadDim];
  // This CTA's merged partial, read by cluster rank 0.
  __shared__ float part_m[kRT], part_l[kRT];
  __shared__ __align__(16) float part_o[kRT][kHeadDim];

  grid_dep_wait();
  grid_dep_launch();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int b = blockIdx.z;
  const int y = blockIdx.y;
  const int hkv = y / p.RG, rg = y - hkv * p.RG;
  const int s = (int)cluster_rank();  // split index == rank in the cluster
  const int cp = p.cache_pos ? p.cache_pos[b] : p.uniform_past;
  int L = cp + p.q_len;  // keys visible to the last token of this sequence
  if (L > p.max_seq || cp < 0) {
    if (threadIdx.x == 0 && s == 0) raise_device_error(p.err, LS_ERR_KV_OVERFLOW);
    L = min(max(L, 1), p.max_seq);
  }
  int chunk = (L + p.splits - 1) / p.splits;
  chunk = max(chunk, kMinChunk);
  const int j0 = min(s * chunk, L), j1 = min(j0 + chunk, L);  // empty for idle splits
  const int r0 = rg * kRT;
  const int nrows = min(kRT, p.R - r0);

  float qf[kRT][4];
  int lim[kRT];
#pragma unroll
  for (int rr = 0; rr < kRT; ++rr) {
    const int r = r0 + rr;
    if (rr < nrows) {
      const int i = r / p.G, g = r - (r / p.G) * p.G;
      const int t = b * p.q_len + i;
      const uint2 u = *reinterpret_cast<const uint2*>(p.q + ((size_t)t * p.Hq + hkv * p.G + g) * kHeadDim + lane * 4);
      qf[rr][0] = bf16_lo(u.x) * p.scale_log2;
      qf[rr][1] = bf16_hi(u.x) * p.scale_log2;
      qf[rr][2] = bf16_lo(u.y) * p.scale_log2;
      qf[rr][3] = bf16_hi(u.y) * p.scale_log2;
      lim[rr] = cp + i;  // last visible key
    } else {
      qf[rr][0] = qf[rr][1] = qf[rr][2] = qf[rr][3] = 0.f;
      lim[rr] = -1;
    }
  }
  float m[kRT], l[kRT], o[kRT][4];
#pragma unroll
  for (int rr = 0; rr < kRT; ++rr) {
    m[rr] = -INFINITY;
    l[rr] = 0.f;
    o[rr][0] = o[rr][1] = o[rr][2] = o[rr][3] = 0.f;
  }
  const size_t head_base = ((size_t)b * p.Hkv + hkv) * p.max_seq;
  const __nv_bfloat16* kb = p.k_cache + head_base * kHeadDim + lane * 4;
  const __nv_bfloat16* vb = p.v_cache + head_base * kHeadDim + lane * 4;

  for (int jb = j0 + warp; jb < j1; jb += kAttnWarps * kUK) {
    uint2 kv[kUK], vv[kUK];
#pragma unroll
    for (int u = 0; u < kUK; ++u) {
      const int j = jb + u * kAttnWarps;
      if (j < j1) {
        kv[u] = *reinterpret_cast<const uint2*>(kb + (size_t)j * kHeadDim);
        vv[u] = *reinterpret_cast<const uint2*>(vb + (size_t)j * kHeadDim);
      } else {
        kv[u] = make_uint2(0, 0);
        vv[u] = make_uint2(0, 0);
      }
    }
#pragma unroll
    for (int u = 0; u < kUK; ++u) {
      const int j = jb + u * kAttnWarps;
      if (j >= j1) break;
      const float k0 = bf16_lo(kv[u].x), k1 = bf16_hi(kv[u].x), k2 = bf16_lo(kv[u].y), k3 = bf16_hi(kv[u].y);
      const float v0 = bf16_lo(vv[u].x), v1 = bf16_hi(vv[u].x), v2 = bf16_lo(vv[u].y), v3 = bf16_hi(vv[u].y);
#pragma unroll
      for (int rr = 0; rr < kRT; ++rr) {
        float d = qf[rr][0] * k0;
        d = fmaf(qf[rr][1], k1, d);
        d = fmaf(qf[rr][2], k2, d);
        d = fmaf(qf[rr][3], k3, d);
        d = warp_sum(d);
        if (j <= lim[rr]) {
          const float mn = fmaxf(m[rr], d);
          const float corr = exp2f(m[rr] - mn);
          const float pr = exp2f(d - mn);
          l[rr] = fmaf(l[rr], corr, pr);
          o[rr][0] = fmaf(o[rr][0], corr, pr * v0);
          o[rr][1] = fmaf(o[rr][1], corr, pr * v1);
          o[rr][2] = fmaf(o[rr][2], corr, pr * v2);
          o[rr][3] = fmaf(o[rr][3], corr, pr * v3);
          m[rr] = mn;
        }
      }
    }
  }

  // Merge the warps of this CTA into part_*.
#pragma unroll
  for (int rr = 0; rr < kRT; ++rr) {
    if (lane == 0) { sm_m[warp][rr] = m[rr]; sm_l[warp][rr] = l[rr]; }
    *reinterpret_cast<float4*>(&sm_o[warp][rr][lane * 4]) = make_float4(o[rr][0], o[rr][1], o[rr][2], o[rr][3]);
  }
  __syncthreads();
  if (threadIdx.x < kRT) {
    const int rr = threadIdx.x;
    float mx = -INFINITY;
    for (int w = 0; w < kAttnWarps; ++w) mx = fmaxf(mx, sm_m[w][rr]);
    float ls = 0.f;
    if (mx != -INFINITY)
      for (int w = 0; w < kAttnWarps; ++w) ls += sm_l[w][rr] * exp2f(sm_m[w][rr] - mx);
    part_m[rr] = mx;
    part_l[rr] = ls;
  }
  __syncthreads();
  const int d = threadIdx.x;  // kAttnThreads == kHeadDim: one dimension per thread
#pragma unroll
  for (int rr = 0; rr < kRT; ++rr) {
    float acc = 0.f;
    const float mx = part_m[rr];
    if (mx != -INFINITY)
      for (int w = 0; w < kAttnWarps; ++w) acc += sm_o[w][rr][d] * exp2f(sm_m[w][rr] - mx);
    part_o[rr][d] = acc;
  }

  auto store_row = [&](int rr, float value) {
    const int r = r0 + rr;
    const int i = r / p.G, g = r - (r / p.G) * p.G;
    const int t = b * p.q_len + i;
    p.out[((size_t)t * p.Hq + hkv * p.G + g) * kHeadDim + d] = f_to_bf16(value);
  };

  if (p.splits == 1) {
    __syncthreads();
    for (int rr = 0; rr < nrows; ++rr) store_row(rr, part_o[rr][d] / part_l[rr]);
    return;
  }
  cluster_sync_all();  // every split's partial is in its shared memory
  if (s == 0) {
    for (int rr = 0; rr < nrows; ++rr) {
      float mx = -INFINITY;
      for (int c = 0; c < p.splits; ++c) mx = fmaxf(mx, ld_dsmem_f32(&part_m[rr], (uint32_t)c));
      float ls = 0.f, acc = 0.f;
      for (int c = 0; c < p.splits; ++c) {
        const float mc = ld_dsmem_f32(&part_m[rr], (uint32_t)c);
        if (mc == -INFINITY) continue;
        const float w = exp2f(mc - mx);
        ls += ld_dsmem_f32(&part_l[rr], (uint32_t)c) * w;
        acc += ld_dsmem_f32(&part_o[rr][d], (uint32_t)c) * w;
      }
      store_row(rr, acc / ls);
    }
  }
  cluster_sync_all();  // keep every CTA's shared memory alive until rank 0 has read it
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
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  return cfg;
}

int launch_qk_norm_rope(const void* qkv, int64_t batch, int64_t q_len, int64_t hq, int64_t hkv, const void* qn,
                        const void* kn, const void* cos, const void* sin, int64_t rope_len, int64_t rope_offset,
                        const int32_t* cache_pos, int64_t uniform_past, void* k_cache, void* v_cache, int64_t max_seq, void* k_out, void* v_out, void* q_out,
                        float eps, cudaStream_t stream) {
  QkRopeParams p = {};
  p.qkv = static_cast<const __nv_bfloat16*>(qkv);
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
  cudaError_t e = cudaLaunchKernelEx(&cfg, qk_norm_rope_append_kernel, p);
  if (e != cudaSuccess) return set_error(LS_ERR_CUDA, "qk_norm_rope launch: %s", cudaGetErrorString(e));
  return LS_OK;
}

struct AttnPlan {
  int G, R, RG, splits;
};

// Splits per (sequence, kv head, row group): a power of two up to 16, enough
// for about two CTAs per SM, and no more than the cache has 16-key chunks.
static AttnPlan attn_plan(int64_t batch, int64_t q_len, int64_t hq, int64_t hkv, int64_t max_seq) {
  AttnPlan pl;
  pl.G = (int)(hq / hkv);
  pl.R = (int)(q_len * pl.G);
  pl.RG = (pl.R + kRT - 1) / kRT;
  const int64_t pairs = batch * hkv * pl.RG;
  int splits = 1;
  while (splits < kMaxSplits && pairs * splits < 2 * (int64_t)sm_count() &&
         (int64_t)(splits * 2) * kMinChunk <= max_seq)
    splits *= 2;
  pl.splits = splits;
  return pl;
}

int attention_workspace_bytes(int64_t batch, int64_t q_len, int64_t hq, int64_t hkv, int64_t max_seq,
                              int64_t* bytes) {
  (void)attn_plan(batch, q_len, hq, hkv, max_seq);
  *bytes = 0;  // partials are merged through distributed shared memory
  return LS_OK;
}

int launch_decode_attention(const void* q, const void* k_cache, const void* v_cache, const int32_t* cache_pos,
                            int64_t uniform_past, int64_t batch, int64_t q_len, int64_t hq, int64_t hkv,
                            int64_t max_seq, float scale, void* out, void* workspace, int64_t workspace_bytes,
                            cudaStream_t stream) {
  (void)workspace;
  (void)workspace_bytes;
  AttnPlan pl = attn_plan(batch, q_len, hq, hkv, max_seq);
  AttnParams p = {};
  p.q = static_cast<const __nv_bfloat16*>(q);
  p.k_cache = static_cast<const __nv_bfloat16*>(k_cache);
  p.v_cache = static_cast<const __nv_bfloat16*>(v_cache);
  p.cache_pos = cache_pos;
  p.uniform_past = (int)uniform_past;
  p.out = static_cast<__nv_bfloat16*>(out);
  p.q_len = (int)q_len;
  p.Hq = (int)hq;
  p.Hkv = (int)hkv;
  p.G = pl.G;
  p.R = pl.R;
  p.RG = pl.RG;
  p.splits = pl.splits;
  p.max_seq = (int)max_seq;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.err = device_error_ptr();
  static bool nonportable_set = false;
  if (pl.splits > 8 && !nonportable_set) {
    cudaError_t e = cudaFuncSetAttribute(decode_attention_kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    if (e != cudaSuccess) return set_error(LS_ERR_CUDA, "cluster size attribute: %s", cudaGetErrorString(e));
    nonportable_set = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(pl.splits, (unsigned)(hkv * pl.RG), (unsigned)batch);
  cfg.blockDim = dim3(kAttnThreads);
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  int na = 0;
  attr[na].id = cudaLaunchAttributeClusterDimension;
  attr[na].val.clusterDim.x = pl.splits;
  attr[na].val.clusterDim.y = 1;
  attr[na].val.clusterDim.z = 1;
  ++na;
  if (pdl_enabled()) {
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  cudaError_t e = cudaLaunchKernelEx(&cfg, decode_attention_kernel, p);
  if (e != cudaSuccess) return set_error(LS_ERR_CUDA, "decode_attention launch: %s", cudaGetErrorString(e));
  return LS_OK;
}

}  // namespace lsb_host
