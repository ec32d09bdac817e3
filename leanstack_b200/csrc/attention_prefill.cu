// Causal GQA attention for long query blocks (prefill, config 5) on the legacy
// mma.sync tensor path.  The default is the tcgen05 kernel in gemm_tc.cu
// (prefill_attention_tc_kernel, 2.6x faster at config 5); this one is kept as
// an option (LEANB200_PREFILL_ATTN=mma) and as its cross-check.
//
// Same contract as the split-KV kernel (attention_tc.cu): query row r =
// (token i, group member g) of kv head h in sequence b sees keys
// 0 .. cache_pos[b] + i (qwen_explicit.py:551-563, :1000-1039).  When the
// rows of one (sequence, kv head) number in the hundreds, splitting the keys
// is the wrong shape: every 16-row group would stream the whole cache again.
// Here a CTA owns 128 consecutive rows (8 warps x 16 = MMA M per warp) and
// streams each 64-key K/V tile ONCE through a shared cp.async ring; every warp
// runs its own online softmax over the tile (S = Q K^T and O += P V with
// mma.sync m16n8k16, P split into bf16 hi + lo as in the decode kernel) and
// the CTA visits only the keys its last row can see.  No merge is needed: a
// CTA sees all keys of its rows.
#include "common.cuh"

namespace lsb {

constexpr int kPaHeadDim = 128;
constexpr int kPaWarps = 8;
constexpr int kPaThreads = kPaWarps * 32;
constexpr int kPaRows = kPaWarps * 16;
constexpr int kPaKeys = 64;                                  // keys per ring stage
constexpr int kPaStages = 2;
constexpr int kPaTileBytes = kPaKeys * kPaHeadDim * 2;       // 16 KB: K or V of one stage
constexpr int kPaSmemBytes = kPaStages * 2 * kPaTileBytes;   // 64 KB

struct PaParams {
  const __nv_bfloat16* q;        // [M, Hq, D]
  const __nv_bfloat16* k_cache;  // [B, Hkv, S, D]
  const __nv_bfloat16* v_cache;
  const int* cache_pos;          // [B] or null (then uniform_past)
  int uniform_past;
  __nv_bfloat16* out;            // [M, Hq * D]
  int* err;
  int q_len, Hq, Hkv, G, R, max_seq;
  float scale_log2;
};

__device__ __forceinline__ void pa_cp_async16(uint32_t dst, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}
__device__ __forceinline__ void pa_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void pa_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ void pa_ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void pa_ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                             uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void pa_mma(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t pa_pack(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}
// Byte offset of 16-byte chunk `chunk` of key row `key` in a [keys][128] bf16 tile (XOR swizzle).
__device__ __forceinline__ uint32_t pa_swz(int key, int chunk) {
  return (uint32_t)(key * (kPaHeadDim * 2) + ((chunk ^ (key & 7)) << 4));
}

__global__ void __launch_bounds__(kPaThreads, 1) prefill_attention_kernel(PaParams p) {
  extern __shared__ __align__(128) unsigned char pa_smem[];
  grid_dep_wait();
  grid_dep_launch();
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g8 = lane >> 2, t4 = lane & 3;
  const int b = blockIdx.z, hkv = blockIdx.y;
  // Row blocks in reverse order: the last rows see the most keys, so the
  // longest blocks start first and the short ones fill the tail.
  const int r0 = (gridDim.x - 1 - blockIdx.x) * kPaRows;
  const int cp = p.cache_pos ? p.cache_pos[b] : p.uniform_past;
  int L = cp + p.q_len;
  if (L > p.max_seq || cp < 0) {
    if (tid == 0 && blockIdx.x == 0) raise_device_error(p.err, LS_ERR_KV_OVERFLOW);
    L = min(max(L, 0), p.max_seq);
  }
  // Keys the CTA's last row can see.
  const int r_last = min(r0 + kPaRows, p.R) - 1;
  const int L_blk = min(L, cp + r_last / p.G + 1);
  const int ntiles = (L_blk + kPaKeys - 1) / kPaKeys;

  // This warp's 16 rows: lane holds rows g8 and g8 + 8 (A-fragment rows).
  uint32_t qa[8][4];
  int lim[2];
  int wmax = -1;  // the last key any row of this warp sees
#pragma unroll
  for (int hr = 0; hr < 2; ++hr) {
    const int row = r0 + warp * 16 + g8 + 8 * hr;
    const bool valid = row < p.R;
    const int i = valid ? row / p.G : 0;
    const int gq = valid ? row - i * p.G : 0;
    const __nv_bfloat16* qp = p.q + ((size_t)(b * p.q_len + i) * p.Hq + hkv * p.G + gq) * kPaHeadDim;
    lim[hr] = valid ? cp + i : -1;
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
      qa[ks][hr] = valid ? *reinterpret_cast<const uint32_t*>(qp + ks * 16 + 2 * t4) : 0u;
      qa[ks][2 + hr] = valid ? *reinterpret_cast<const uint32_t*>(qp + ks * 16 + 8 + 2 * t4) : 0u;
    }
  }
  {
    const int wr_last = min(r0 + warp * 16 + 15, p.R - 1);
    wmax = wr_last >= r0 + warp * 16 ? cp + wr_last / p.G : -1;
  }

  const size_t head_base = ((size_t)b * p.Hkv + hkv) * p.max_seq * kPaHeadDim;
  const __nv_bfloat16* kbase = p.k_cache + head_base;
  const __nv_bfloat16* vbase = p.v_cache + head_base;
  const uint32_t ring = smem_u32(pa_smem);
  auto load_tile = [&](int kt, int stage) {
    const uint32_t st = ring + stage * 2 * kPaTileBytes;
    for (int c = tid; c < kPaKeys * 16; c += kPaThreads) {
      const int r = c >> 4, cc = c & 15;
      const int j = kt * kPaKeys + r;
      const bool ok = j < L_blk;
      const size_t off = (size_t)(ok ? j : 0) * kPaHeadDim + cc * 8;
      const uint32_t so = pa_swz(r, cc);
      pa_cp_async16(st + so, kbase + off, ok ? 16u : 0u);
      pa_cp_async16(st + kPaTileBytes + so, vbase + off, ok ? 16u : 0u);
    }
  };

  float o[16][4];
#pragma unroll
  for (int nt = 0; nt < 16; ++nt) o[nt][0] = o[nt][1] = o[nt][2] = o[nt][3] = 0.f;
  float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.f, 0.f};

#pragma unroll
  for (int st = 0; st < kPaStages; ++st) {
    if (st < ntiles) load_tile(st, st);
    pa_commit();
  }
  for (int kt = 0; kt < ntiles; ++kt) {
    pa_wait<kPaStages - 1>();
    __syncthreads();
    const int stage = kt % kPaStages;
    const uint32_t stK = ring + stage * 2 * kPaTileBytes;
    const uint32_t stV = stK + kPaTileBytes;
    if (kt * kPaKeys <= wmax) {  // some row of this warp sees part of this tile
#pragma unroll
      for (int half = 0; half < 2; ++half) {  // 32 keys at a time
        const int kb0 = half * 32;
        const int jb = kt * kPaKeys + kb0;
        if (jb > wmax) break;
        float sc[4][4];
#pragma unroll
        for (int nt = 0; nt < 4; ++nt) sc[nt][0] = sc[nt][1] = sc[nt][2] = sc[nt][3] = 0.f;
        {
          const int csel = (lane >> 3) & 1;
#pragma unroll
          for (int pr = 0; pr < 2; ++pr) {  // n-tile pairs: keys kb0 + 16 pr .. + 15
            const int key = kb0 + pr * 16 + (lane & 7) + ((lane >> 4) << 3);
#pragma unroll
            for (int ks = 0; ks < 8; ++ks) {
              uint32_t b00, b01, b10, b11;
              pa_ldsm_x4(stK + pa_swz(key, 2 * ks + csel), b00, b01, b10, b11);
              pa_mma(sc[2 * pr], qa[ks], b00, b01);
              pa_mma(sc[2 * pr + 1], qa[ks], b10, b11);
            }
          }
        }
        float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
        for (int nt = 0; nt < 4; ++nt)
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int hr = e >> 1;
            const int j = jb + nt * 8 + 2 * t4 + (e & 1);
            float v = sc[nt][e] * p.scale_log2;
            if (j >= L_blk || j > lim[hr]) v = -INFINITY;
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
        for (int nt = 0; nt < 4; ++nt)
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
        // O += P V over the 32 keys: two k-steps of 16 keys.
#pragma unroll
        for (int kk = 0; kk < 2; ++kk) {
          uint32_t ahi[4], alo[4];
#pragma unroll
          for (int q = 0; q < 4; ++q) {  // a0: row g8 keys 2t..; a1: row g8+8; a2, a3: keys 8 + 2t..
            const int nt = 2 * kk + (q >> 1);
            const float x0 = sc[nt][(q & 1) * 2], x1 = sc[nt][(q & 1) * 2 + 1];
            const float h0 = round_bf16(x0), h1 = round_bf16(x1);
            ahi[q] = pa_pack(h0, h1);
            alo[q] = pa_pack(x0 - h0, x1 - h1);
          }
          const int key = kb0 + kk * 16 + (lane & 7) + (((lane >> 3) & 1) << 3);
          const int csel = lane >> 4;
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            uint32_t v0, v1, v2, v3;
            pa_ldsm_x4_t(stV + pa_swz(key, 2 * c + csel), v0, v1, v2, v3);
            pa_mma(o[2 * c], ahi, v0, v1);
            pa_mma(o[2 * c], alo, v0, v1);
            pa_mma(o[2 * c + 1], ahi, v2, v3);
            pa_mma(o[2 * c + 1], alo, v2, v3);
          }
        }
      }
    }
    __syncthreads();  // every warp is done with this stage
    if (kt + kPaStages < ntiles) load_tile(kt + kPaStages, stage);
    pa_commit();
  }
  pa_wait<0>();

#pragma unroll
  for (int hr = 0; hr < 2; ++hr) {
    l_run[hr] += __shfl_xor_sync(0xffffffffu, l_run[hr], 1);
    l_run[hr] += __shfl_xor_sync(0xffffffffu, l_run[hr], 2);
  }
#pragma unroll
  for (int hr = 0; hr < 2; ++hr) {
    const int row = r0 + warp * 16 + g8 + 8 * hr;
    if (row >= p.R) continue;
    const int i = row / p.G, gq = row - (row / p.G) * p.G;
    __nv_bfloat16* op = p.out + ((size_t)(b * p.q_len + i) * p.Hq + hkv * p.G + gq) * kPaHeadDim;
    const float inv = 1.f / l_run[hr];
#pragma unroll
    for (int nt = 0; nt < 16; ++nt) {
      const float y0 = o[nt][2 * hr] * inv, y1 = o[nt][2 * hr + 1] * inv;
      *reinterpret_cast<__nv_bfloat162*>(op + nt * 8 + 2 * t4) = __floats2bfloat162_rn(y0, y1);
    }
  }
}

}  // namespace lsb

namespace lsb_host {
using namespace lsb;

int launch_prefill_attention(const void* q, const void* k_cache, const void* v_cache, const int32_t* cache_pos,
                             int64_t uniform_past, int64_t batch, int64_t q_len, int64_t hq, int64_t hkv,
                             int64_t max_seq, float scale, void* out, cudaStream_t stream) {
  PaParams p = {};
  p.q = static_cast<const __nv_bfloat16*>(q);
  p.k_cache = static_cast<const __nv_bfloat16*>(k_cache);
  p.v_cache = static_cast<const __nv_bfloat16*>(v_cache);
  p.cache_pos = cache_pos;
  p.uniform_past = (int)uniform_past;
  p.out = static_cast<__nv_bfloat16*>(out);
  p.q_len = (int)q_len;
  p.Hq = (int)hq;
  p.Hkv = (int)hkv;
  p.G = (int)(hq / hkv);
  p.R = (int)(q_len * p.G);
  p.max_seq = (int)max_seq;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.err = device_error_ptr();
  const int row_blocks = (p.R + kPaRows - 1) / kPaRows;
  if (hkv > 65535 || batch > 65535)
    return set_error(LS_ERR_UNSUPPORTED_SHAPE, "prefill_attention: %lld kv heads / %lld sequences", (long long)hkv,
                     (long long)batch);
  static bool attr_done = false;
  if (!attr_done) {
    cudaError_t e = cudaFuncSetAttribute(prefill_attention_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         kPaSmemBytes);
    if (e != cudaSuccess) return set_error(LS_ERR_CUDA, "prefill_attention attribute: %s", cudaGetErrorString(e));
    attr_done = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)row_blocks, (unsigned)hkv, (unsigned)batch);
  cfg.blockDim = dim3(kPaThreads);
  cfg.dynamicSmemBytes = kPaSmemBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  cudaError_t e = cudaLaunchKernelEx(&cfg, prefill_attention_kernel, p);
  return e == cudaSuccess ? LS_OK : set_error(LS_ERR_CUDA, "prefill_attention launch: %s", cudaGetErrorString(e));
}

}  // namespace lsb_host
