// Split-KV decode / verify attention on the tensor cores (mma.sync m16n8k16, bf16).
//
// Same contract as the CUDA-core kernel in attention.cu (reference:
// src/leanstack/runtime/qwen_explicit.py:886-903, :1000-1039, mask :551-563):
// for every sequence b, kv head h and query row r = (token i, group member g)
// of that head, attend over keys 0 .. cache_pos[b] + i of the static cache.
//
// Layout of the work:
//  * A CTA owns up to 16 query rows of one (sequence, kv head) -- the MMA's M
//    dimension: the G = Hq/Hkv heads sharing the kv head, times the q_len
//    tokens -- and one split of the keys.  The splits of one (sequence, kv head,
//    row group) form a thread-block cluster.
//  * Each of the 4 warps streams 16-key blocks of K and V through a private
//    3-stage cp.async ring in shared memory (XOR-swizzled 16-byte chunks, so
//    ldmatrix reads are free of bank conflicts) and keeps its own online
//    softmax: S = Q K^T (16 MMAs per block), P = exp2(S - m) in fp32, O += P V
//    with P split into two bf16 terms (hi + lo, 32 MMAs per block) so that the
//    probabilities keep about 16 bits instead of bf16's 8.
//  * Merge: the 4 warps combine in shared memory; then every CTA of the cluster
//    sends each slice of 128/splits output dimensions to the CTA that owns it
//    (remote shared-memory stores), one cluster barrier, and every CTA merges
//    its slice over the splits and writes bf16.  No global workspace.
//
// HBM traffic per (sequence, kv head): 512 bytes per visible key (K and V,
// head_dim 128, bf16), read once; Q and the output are noise.
#include "common.cuh"

namespace lsb {

constexpr int kTaHeadDim = 128;
constexpr int kTaWarps = 4;
constexpr int kTaThreads = kTaWarps * 32;
constexpr int kTaRows = 16;   // query rows per CTA (MMA M)
constexpr int kTaKeys = 16;   // keys per block
constexpr int kTaStages = 3;
constexpr int kTaTileBytes = kTaKeys * kTaHeadDim * 2;        // 4 KB: one K or V tile
constexpr int kTaStageBytes = 2 * kTaTileBytes;               // K + V
constexpr int kTaRingBytes = kTaWarps * kTaStages * kTaStageBytes;  // 96 KB
constexpr int kTaMaxSplits = 16;
constexpr int kTaMergeBytes = kTaWarps * kTaRows * (kTaHeadDim + 2) * 4;  // reuses the ring
constexpr int kTaRecvBytes = kTaRows * kTaHeadDim * 4 + 2 * kTaMaxSplits * kTaRows * 4;
constexpr int kTaSmemBytes = kTaRingBytes + kTaRecvBytes;
constexpr int kTaQStageBytes = kTaRows * kTaHeadDim * 2;  // fused mode: the CTA's normalised query rows
static_assert(kTaMergeBytes <= kTaRingBytes, "merge buffers must fit in the ring");

struct TaParams {
  const __nv_bfloat16* q;        // [M, Hq, D]
  const __nv_bfloat16* k_cache;  // [B, Hkv, S, D]
  const __nv_bfloat16* v_cache;
  const int* cache_pos;          // [B] or null (then uniform_past)
  int uniform_past;
  __nv_bfloat16* out;            // [M, Hq * D]
  int* err;
  int q_len, Hq, Hkv, G, R, RG, splits, max_seq;
  float scale_log2;
  // Fused q/k norm + RoPE + K/V append (q_len 1): when qkv is set, q is formed
  // here from the raw projection and the new token's K/V row goes into the
  // cache and, from registers, into the shared-memory tile that holds it.
  const __nv_bfloat16* qkv;      // [B, (Hq + 2 Hkv) D] or null
  const __nv_bfloat16* q_norm_w;
  const __nv_bfloat16* k_norm_w;
  const __nv_bfloat16* cos;      // [rope_len, D/2]
  const __nv_bfloat16* sin;
  __nv_bfloat16* k_store;        // the caches, writable
  __nv_bfloat16* v_store;
  int rope_len, rope_offset;
  float eps;
};

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void mma_bf16(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}
__device__ __forceinline__ uint32_t ta_cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void ta_cluster_arrive_relaxed() {
  asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
}
__device__ __forceinline__ void ta_cluster_wait() { asm volatile("barrier.cluster.wait.aligned;" ::: "memory"); }
__device__ __forceinline__ void ta_cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\nbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ void ta_st_remote(const void* local, uint32_t rank, float v) {
  uint32_t remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(smem_u32(local)), "r"(rank));
  asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(remote), "f"(v) : "memory");
}

// Byte offset of 16-byte chunk `chunk` (0..15) of key row `key` (0..15) in a tile.
__device__ __forceinline__ uint32_t ta_swz(int key, int chunk) {
  return (uint32_t)(key * (kTaHeadDim * 2) + ((chunk ^ (key & 7)) << 4));
}

template <bool FUSED>
__global__ void __launch_bounds__(kTaThreads) decode_attention_tc_kernel(TaParams p) {
  extern __shared__ __align__(128) unsigned char ta_smem[];
  float* recv_o = reinterpret_cast<float*>(ta_smem + kTaRingBytes);  // [splits][16][128/splits]
  float* recv_m = recv_o + kTaRows * kTaHeadDim;                      // [kTaMaxSplits][16]
  float* recv_l = recv_m + kTaMaxSplits * kTaRows;

  if (p.splits > 1) ta_cluster_arrive_relaxed();  // this CTA is running
  // Fused mode waits for the previous kernel (the QKV projection) only before
  // reading the raw projection: cache_pos, the cache rows before it, the rope
  // table and the norm weights are written by no kernel that can still be
  // running (the cursor and accept kernels let their dependents start only at
  // their own end), so the first K/V copies go out under the projection's tail.
  if (!FUSED) grid_dep_wait();
  grid_dep_launch();

  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g8 = lane >> 2, t4 = lane & 3;
  const int b = blockIdx.z;
  const int hkv = blockIdx.y / p.RG, rg = blockIdx.y - hkv * p.RG;
  const int s = p.splits > 1 ? (int)ta_cluster_rank() : 0;
  const int cp = p.cache_pos ? (FUSED ? __ldcg(p.cache_pos + b) : p.cache_pos[b]) : p.uniform_past;
  int L = cp + p.q_len;
  if (L > p.max_seq || cp < 0) {
    if (threadIdx.x == 0 && s == 0) raise_device_error(p.err, LS_ERR_KV_OVERFLOW);
    L = min(max(L, 0), p.max_seq);
  }
  // Keys of this split, in whole 16-key blocks.
  const int nblk_all = (L + kTaKeys - 1) / kTaKeys;
  const int blk_per = (nblk_all + p.splits - 1) / p.splits;
  const int blk0 = min(s * blk_per, nblk_all), blk1 = min(blk0 + blk_per, nblk_all);
  const int r0 = rg * kTaRows;
  const int nrows = min(kTaRows, p.R - r0);
  // Fused mode (q_len 1): the new token's key (position cp) is not in the
  // cache yet, so the copies stop before it; its tile row is written from
  // registers by the warp that owns its block.
  constexpr bool fused = FUSED;
  const int Lcopy = fused ? min(L, max(cp, 0)) : L;
  const int e0 = lane * 4;  // fused mode: the 4 head dims this lane normalises
  const size_t qkv_dim = (size_t)(p.Hq + 2 * p.Hkv) * kTaHeadDim;
  const int rrow = cp - p.rope_offset;
  const bool rope_ok = fused && cp >= 0 && rrow >= 0 && rrow < p.rope_len;
  if (fused && !rope_ok && threadIdx.x == 0 && s == 0) raise_device_error(p.err, LS_ERR_KV_OVERFLOW);

  const size_t head_base = ((size_t)b * p.Hkv + hkv) * p.max_seq * kTaHeadDim;
  const __nv_bfloat16* kbase = p.k_cache + head_base;
  const __nv_bfloat16* vbase = p.v_cache + head_base;
  const uint32_t ring = smem_u32(ta_smem) + warp * kTaStages * kTaStageBytes;

  // This warp's blocks: blk0 + warp, blk0 + warp + 4, ...
  const int nb = (blk1 - blk0 - warp + kTaWarps - 1) / kTaWarps;  // may be <= 0
  auto load_block = [&](int n, int stage) {
    const int kb = (blk0 + warp + n * kTaWarps) * kTaKeys;
    const uint32_t st = ring + stage * kTaStageBytes;
#pragma unroll
    for (int it = 0; it < 8; ++it) {
      const int c = lane + 32 * it;
      const int r = c >> 4, cc = c & 15;
      const int j = kb + r;
      const bool ok = j < Lcopy;
      const size_t off = (size_t)(ok ? j : 0) * kTaHeadDim + cc * 8;
      const uint32_t so = ta_swz(r, cc);
      cp_async16(st + so, kbase + off, ok ? 16u : 0u);
      cp_async16(st + kTaTileBytes + so, vbase + off, ok ? 16u : 0u);
    }
  };

  float o[16][4];
#pragma unroll
  for (int nt = 0; nt < 16; ++nt) o[nt][0] = o[nt][1] = o[nt][2] = o[nt][3] = 0.f;
  float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.f, 0.f};

#pragma unroll
  for (int st = 0; st < kTaStages; ++st) {
    if (st < nb) load_block(st, st);
    cp_async_commit();
  }

  // Fused mode: the normalised, rotated query rows into shared memory (warp w
  // forms rows w, w + 4, ...), and the new token's K (normalised, rotated) and
  // V rows in the registers of the warp whose block holds position cp; that
  // warp also appends them to the cache.
  __nv_bfloat16* qs = reinterpret_cast<__nv_bfloat16*>(ta_smem + kTaSmemBytes);
  int n_new = -1;
  uint2 knew = make_uint2(0u, 0u), vnew = make_uint2(0u, 0u);
  if (fused) {
    const __nv_bfloat16* xt = p.qkv + (size_t)b * qkv_dim;
    const int idx = lane < 16 ? e0 : e0 - kTaHeadDim / 2;
    uint2 c_u = make_uint2(0u, 0u), s_u = make_uint2(0u, 0u);
    if (rope_ok) {
      c_u = *reinterpret_cast<const uint2*>(p.cos + (size_t)rrow * (kTaHeadDim / 2) + idx);
      s_u = *reinterpret_cast<const uint2*>(p.sin + (size_t)rrow * (kTaHeadDim / 2) + idx);
    }
    const uint2 wk = *reinterpret_cast<const uint2*>(p.k_norm_w + e0);
    const uint2 wq = *reinterpret_cast<const uint2*>(p.q_norm_w + e0);
    grid_dep_wait();  // the raw projection is the previous kernel's output
    const int blk_new = cp / kTaKeys;
    if (rope_ok && cp < p.max_seq && blk_new >= blk0 && blk_new < blk1 && (blk_new - blk0) % kTaWarps == warp) {
      n_new = (blk_new - blk0) / kTaWarps;
      const uint2 rk = *reinterpret_cast<const uint2*>(xt + (size_t)(p.Hq + hkv) * kTaHeadDim + e0);
      vnew = *reinterpret_cast<const uint2*>(xt + (size_t)(p.Hq + p.Hkv + hkv) * kTaHeadDim + e0);
      knew = head_norm_rope(rk, wk, c_u, s_u, p.eps, lane);
      if (rg == 0) {
        const size_t off = (((size_t)b * p.Hkv + hkv) * p.max_seq + cp) * kTaHeadDim + e0;
        *reinterpret_cast<uint2*>(p.k_store + off) = knew;
        *reinterpret_cast<uint2*>(p.v_store + off) = vnew;
      }
    }
    for (int r = warp; r < nrows; r += kTaWarps) {  // q_len 1: row r0 + r is query head hkv * G + r0 + r
      const uint2 rq = *reinterpret_cast<const uint2*>(xt + (size_t)(hkv * p.G + r0 + r) * kTaHeadDim + e0);
      const uint2 o = rope_ok ? head_norm_rope(rq, wq, c_u, s_u, p.eps, lane) : make_uint2(0u, 0u);
      *reinterpret_cast<uint2*>(qs + r * kTaHeadDim + e0) = o;
    }
    __syncthreads();
  }

  // Q fragments (A operand, rows g8 and g8 + 8, 8 k-steps of 16 dims) and the
  // last key each of the two rows may see.
  uint32_t qa[8][4];
  int lim[2];
#pragma unroll
  for (int hr = 0; hr < 2; ++hr) {
    const int row = r0 + g8 + 8 * hr;
    const bool valid = row < p.R;
    const int i = valid ? row / p.G : 0;
    const int gq = valid ? row - i * p.G : 0;
    lim[hr] = valid ? cp + i : -1;
    const __nv_bfloat16* qp = fused ? qs + (size_t)(row - r0) * kTaHeadDim
                                    : p.q + ((size_t)(b * p.q_len + i) * p.Hq + hkv * p.G + gq) * kTaHeadDim;
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
      qa[ks][hr] = valid ? *reinterpret_cast<const uint32_t*>(qp + ks * 16 + 2 * t4) : 0u;
      qa[ks][2 + hr] = valid ? *reinterpret_cast<const uint32_t*>(qp + ks * 16 + 8 + 2 * t4) : 0u;
    }
  }

  for (int n = 0; n < nb; ++n) {
    cp_async_wait<kTaStages - 1>();
    __syncwarp();
    const int stage = n % kTaStages;
    const uint32_t stK = ring + stage * kTaStageBytes;
    const uint32_t stV = stK + kTaTileBytes;
    const int jb = (blk0 + warp + n * kTaWarps) * kTaKeys;
    if (fused && n == n_new) {  // fused mode: the new token's K / V row over the tile's zero-filled row
      const uint32_t o = ta_swz(cp - jb, lane >> 1) + (lane & 1) * 8;
      asm volatile("st.shared.v2.u32 [%0], {%1, %2};" ::"r"(stK + o), "r"(knew.x), "r"(knew.y) : "memory");
      asm volatile("st.shared.v2.u32 [%0], {%1, %2};" ::"r"(stV + o), "r"(vnew.x), "r"(vnew.y) : "memory");
      __syncwarp();
    }

    // S = Q K^T for 16 keys (two n-tiles of 8 keys).
    float sc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
    {
      const int key = (lane & 7) + ((lane >> 4) << 3);
      const int csel = (lane >> 3) & 1;
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) {
        uint32_t b00, b01, b10, b11;
        ldsm_x4(stK + ta_swz(key, 2 * ks + csel), b00, b01, b10, b11);
        mma_bf16(sc[0], qa[ks], b00, b01);
        mma_bf16(sc[1], qa[ks], b10, b11);
      }
    }
    // Online softmax (base 2) of rows g8 (hr 0) and g8 + 8 (hr 1).
    float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int hr = e >> 1;
        const int j = jb + nt * 8 + 2 * t4 + (e & 1);
        float v = sc[nt][e] * p.scale_log2;
        if (j >= L || j > lim[hr]) v = -INFINITY;
        sc[nt][e] = v;
        mx[hr] = fmaxf(mx[hr], v);
      }
    float corr[2];
#pragma unroll
    for (int hr = 0; hr < 2; ++hr) {
      mx[hr] = fmaxf(mx[hr], __shfl_xor_sync(0xffffffffu, mx[hr], 1));
      mx[hr] = fmaxf(mx[hr], __shfl_xor_sync(0xffffffffu, mx[hr], 2));
      const float mn = fmaxf(m_run[hr], mx[hr]);
      corr[hr] = (mn == -INFINITY) ? 1.f : exp2f(m_run[hr] - mn);
      m_run[hr] = mn;
    }
    float ps[2] = {0.f, 0.f};
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int hr = e >> 1;
        const float pv = (m_run[hr] == -INFINITY) ? 0.f : exp2f(sc[nt][e] - m_run[hr]);
        sc[nt][e] = pv;
        ps[hr] += pv;
      }
#pragma unroll
    for (int hr = 0; hr < 2; ++hr) l_run[hr] = l_run[hr] * corr[hr] + ps[hr];
#pragma unroll
    for (int nt = 0; nt < 16; ++nt) {
      o[nt][0] *= corr[0];
      o[nt][1] *= corr[0];
      o[nt][2] *= corr[1];
      o[nt][3] *= corr[1];
    }
    // P as A operands: hi = bf16(p), lo = bf16(p - hi).
    uint32_t ahi[4], alo[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {  // a0: row g8 keys 2t..; a1: row g8+8; a2, a3: keys 8 + 2t..
      const float x0 = sc[q >> 1][(q & 1) * 2], x1 = sc[q >> 1][(q & 1) * 2 + 1];
      const float h0 = round_bf16(x0), h1 = round_bf16(x1);
      ahi[q] = pack_bf16(h0, h1);
      alo[q] = pack_bf16(x0 - h0, x1 - h1);
    }
    // O += P V over 16 n-tiles of 8 dims.
    {
      const int key = (lane & 7) + (((lane >> 3) & 1) << 3);
      const int csel = lane >> 4;
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        uint32_t v0, v1, v2, v3;
        ldsm_x4_t(stV + ta_swz(key, 2 * c + csel), v0, v1, v2, v3);
        mma_bf16(o[2 * c], ahi, v0, v1);
        mma_bf16(o[2 * c], alo, v0, v1);
        mma_bf16(o[2 * c + 1], ahi, v2, v3);
        mma_bf16(o[2 * c + 1], alo, v2, v3);
      }
    }
    __syncwarp();
    if (n + kTaStages < nb) load_block(n + kTaStages, stage);
    cp_async_commit();
  }
  cp_async_wait<0>();
#pragma unroll
  for (int hr = 0; hr < 2; ++hr) {
    l_run[hr] += __shfl_xor_sync(0xffffffffu, l_run[hr], 1);
    l_run[hr] += __shfl_xor_sync(0xffffffffu, l_run[hr], 2);
  }
  __syncthreads();  // every warp is done with its ring: reuse it for the merge

  // ---- merge the 4 warps of this CTA ----
  float* wm = reinterpret_cast<float*>(ta_smem);       // [4][16]
  float* wl = wm + kTaWarps * kTaRows;                 // [4][16]
  float* wo = wl + kTaWarps * kTaRows;                 // [4][16][128]
  if (t4 == 0) {
    wm[warp * kTaRows + g8] = m_run[0];
    wm[warp * kTaRows + g8 + 8] = m_run[1];
    wl[warp * kTaRows + g8] = l_run[0];
    wl[warp * kTaRows + g8 + 8] = l_run[1];
  }
#pragma unroll
  for (int nt = 0; nt < 16; ++nt) {
    const int d = nt * 8 + 2 * t4;
    float* w0 = wo + ((size_t)warp * kTaRows + g8) * kTaHeadDim + d;
    float* w1 = wo + ((size_t)warp * kTaRows + g8 + 8) * kTaHeadDim + d;
    *reinterpret_cast<float2*>(w0) = make_float2(o[nt][0], o[nt][1]);
    *reinterpret_cast<float2*>(w1) = make_float2(o[nt][2], o[nt][3]);
  }
  __syncthreads();
  if (p.splits > 1) ta_cluster_wait();  // every CTA of the cluster has started: remote stores are safe

  const int d = threadIdx.x;  // one output dimension per thread (kTaThreads == kTaHeadDim)
  const int w = kTaHeadDim / p.splits;  // dims each cluster CTA finishes
  for (int r = 0; r < nrows; ++r) {
    float mx = -INFINITY;
#pragma unroll
    for (int k = 0; k < kTaWarps; ++k) mx = fmaxf(mx, wm[k * kTaRows + r]);
    float ls = 0.f, acc = 0.f;
    if (mx != -INFINITY) {
#pragma unroll
      for (int k = 0; k < kTaWarps; ++k) {
        const float sc = exp2f(wm[k * kTaRows + r] - mx);
        ls += wl[k * kTaRows + r] * sc;
        acc += wo[((size_t)k * kTaRows + r) * kTaHeadDim + d] * sc;
      }
    }
    if (p.splits == 1) {
      const int row = r0 + r;
      const int i = row / p.G, gq = row - (row / p.G) * p.G;
      p.out[((size_t)(b * p.q_len + i) * p.Hq + hkv * p.G + gq) * kTaHeadDim + d] = f_to_bf16(acc / ls);
    } else {
      const int owner = d / w;
      ta_st_remote(recv_o + ((size_t)s * kTaRows + r) * w + (d - owner * w), (uint32_t)owner, acc);
      if (d < p.splits) {  // this CTA's (max, sum) of row r to every CTA of the cluster
        ta_st_remote(recv_m + s * kTaRows + r, (uint32_t)d, mx);
        ta_st_remote(recv_l + s * kTaRows + r, (uint32_t)d, ls);
      }
    }
  }
  if (p.splits == 1) return;
  ta_cluster_sync();  // release this CTA's remote stores, acquire the others'

  for (int idx = threadIdx.x; idx < nrows * w; idx += kTaThreads) {
    const int r = idx / w, dd = idx - r * w;
    float mx = -INFINITY;
    for (int c = 0; c < p.splits; ++c) mx = fmaxf(mx, recv_m[c * kTaRows + r]);
    float ls = 0.f, acc = 0.f;
    for (int c = 0; c < p.splits; ++c) {
      const float mc = recv_m[c * kTaRows + r];
      if (mc == -INFINITY) continue;
      const float sc = exp2f(mc - mx);
      ls += recv_l[c * kTaRows + r] * sc;
      acc += recv_o[((size_t)c * kTaRows + r) * w + dd] * sc;
    }
    const int row = r0 + r;
    const int i = row / p.G, gq = row - (row / p.G) * p.G;
    p.out[((size_t)(b * p.q_len + i) * p.Hq + hkv * p.G + gq) * kTaHeadDim + s * w + dd] = f_to_bf16(acc / ls);
  }
}

}  // namespace lsb

namespace lsb_host {
using namespace lsb;

struct TaPlan {
  int G, R, RG, splits;
};

// Splits per (sequence, kv head, 16-row group): a power of two up to 16, until
// there are about as many CTAs as SMs, keeping at least 32 cache positions a
// split.  Measured on Qwen3-4B decode steps: at batch 1 (8 pairs) 16 and 8
// splits tie and fewer are slower; at batch 32 (256 pairs) one split (no
// cluster) is 5% faster than two and 9% faster than four.
static TaPlan ta_plan(int64_t batch, int64_t q_len, int64_t hq, int64_t hkv, int64_t max_seq) {
  TaPlan pl;
  pl.G = (int)(hq / hkv);
  pl.R = (int)(q_len * pl.G);
  pl.RG = (pl.R + kTaRows - 1) / kTaRows;
  const int64_t pairs = batch * hkv * pl.RG;
  int splits = 1;
  while (splits < kTaMaxSplits && pairs * splits < (int64_t)sm_count() && (int64_t)splits * 2 * 32 <= max_seq)
    splits *= 2;
  pl.splits = splits;
  return pl;
}

template <bool FUSED>
static int launch_ta(const TaParams& p, const TaPlan& pl, int64_t batch, int64_t hkv, cudaStream_t stream) {
  constexpr size_t smem = kTaSmemBytes + (FUSED ? kTaQStageBytes : 0);
  static bool attrs_set = false;
  if (!attrs_set) {
    cudaError_t e =
        cudaFuncSetAttribute(decode_attention_tc_kernel<FUSED>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(decode_attention_tc_kernel<FUSED>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    if (e != cudaSuccess) return set_error(LS_ERR_CUDA, "attention_tc attributes: %s", cudaGetErrorString(e));
    attrs_set = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(pl.splits, (unsigned)(hkv * pl.RG), (unsigned)batch);
  cfg.blockDim = dim3(kTaThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = pl.splits;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  cudaError_t e = cudaLaunchKernelEx(&cfg, decode_attention_tc_kernel<FUSED>, p);
  if (e != cudaSuccess) return set_error(LS_ERR_CUDA, "decode_attention_tc launch: %s", cudaGetErrorString(e));
  return LS_OK;
}

static TaParams ta_params(const TaPlan& pl, const void* k_cache, const void* v_cache, const int32_t* cache_pos,
                          int64_t uniform_past, int64_t q_len, int64_t hq, int64_t hkv, int64_t max_seq, float scale,
                          void* out) {
  TaParams p = {};
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
  return p;
}

int launch_decode_attention_tc(const void* q, const void* k_cache, const void* v_cache, const int32_t* cache_pos,
                               int64_t uniform_past, int64_t batch, int64_t q_len, int64_t hq, int64_t hkv,
                               int64_t max_seq, float scale, void* out, cudaStream_t stream) {
  const TaPlan pl = ta_plan(batch, q_len, hq, hkv, max_seq);
  if ((int64_t)hkv * pl.RG > 65535)
    return set_error(LS_ERR_UNSUPPORTED_SHAPE, "decode_attention: %lld kv heads x %d row groups exceed the grid",
                     (long long)hkv, pl.RG);
  TaParams p = ta_params(pl, k_cache, v_cache, cache_pos, uniform_past, q_len, hq, hkv, max_seq, scale, out);
  p.q = static_cast<const __nv_bfloat16*>(q);
  return launch_ta<false>(p, pl, batch, hkv, stream);
}

// One decode token per sequence (q_len 1) straight from the raw fused QKV
// projection: q/k RMSNorm + RoPE, the K/V append at cache_pos[b], and the
// attention, in one launch (the kernel's fused mode).
int launch_decode_attention_qkv(const void* qkv, int64_t batch, int64_t hq, int64_t hkv, const void* qn,
                                const void* kn, float eps, const void* cos, const void* sin, int64_t rope_len,
                                int64_t rope_offset, const int32_t* cache_pos, int64_t uniform_past, void* k_cache,
                                void* v_cache, int64_t max_seq, float scale, void* out, cudaStream_t stream) {
  const TaPlan pl = ta_plan(batch, 1, hq, hkv, max_seq);
  if (pl.RG != 1)
    return set_error(LS_ERR_UNSUPPORTED_SHAPE, "decode_attention_qkv: %d query heads per kv head (at most %d)",
                     pl.G, kTaRows);
  TaParams p = ta_params(pl, k_cache, v_cache, cache_pos, uniform_past, 1, hq, hkv, max_seq, scale, out);
  p.qkv = static_cast<const __nv_bfloat16*>(qkv);
  p.q_norm_w = static_cast<const __nv_bfloat16*>(qn);
  p.k_norm_w = static_cast<const __nv_bfloat16*>(kn);
  p.cos = static_cast<const __nv_bfloat16*>(cos);
  p.sin = static_cast<const __nv_bfloat16*>(sin);
  p.k_store = static_cast<__nv_bfloat16*>(k_cache);
  p.v_store = static_cast<__nv_bfloat16*>(v_cache);
  p.rope_len = (int)rope_len;
  p.rope_offset = (int)rope_offset;
  p.eps = eps;
  return launch_ta<true>(p, pl, batch, hkv, stream);
}

}  // namespace lsb_host
