// One whole bs1 decode step as a single persistent kernel.
//
// At batch 1 every linear reads each weight byte once and does one FMA with
// it, so the step is a stream of 8 GB of weights through 148 SMs.  Launching
// ~220 kernels per token pays each kernel's ramp-up and tail (the weight
// stream stops between kernels).  This kernel keeps one 1024-thread CTA per SM
// resident for the whole step (cooperative launch) and runs the phases of all
// layers back to back, separated by grid-wide barriers:
//
//   per layer:  QKV    input RMSNorm (every CTA, redundant) + fused QKV rows
//               ATTN   q/k RMSNorm + RoPE + K/V append + split-KV attention;
//                      the last split of each kv head merges the partials
//               O      o_proj rows + residual
//               GU     post-attention RMSNorm + gate/up row pairs + SiLU*up
//               DOWN   down rows + residual
//   then:       HEAD   final RMSNorm + lm_head rows + argmax; the last CTA
//                      writes the token id and advances the cursor.
//
// Before a CTA arrives at a barrier it prefetches (into L2) the first bytes of
// its slice of the next phase's weights, so the HBM stream does not drain while
// the grid synchronises.  Data written by other CTAs is read through L2
// (ld.global.cg): L1 is not coherent across SMs.  Rounding points are the
// reference's (see linear_small_m.cu and attention.cu).  Every barrier and
// counter wait is bounded; on a timeout the kernel records LS_ERR_TIMEOUT and
// every CTA leaves at its next barrier.
#include "common.cuh"

namespace lsb {

constexpr int kDsThreads = 1024;
constexpr int kDsWarps = kDsThreads / 32;
constexpr int kDsGranule = 256;   // bf16 per warp-wide 512-byte load
constexpr int kDsUnroll = 8;      // 16-byte loads in flight per lane
constexpr int kDsAttnWarps = 8;   // warps that run the attention of one work item
constexpr int kDsMaxRows = 4;     // query rows per kv head (GQA group) supported
constexpr int kDsHeadDim = 128;
constexpr uint32_t kDsPrefetch = 32 * 1024;

struct DsLayer {
  const __nv_bfloat16* ln_w;     // [H]
  const __nv_bfloat16* qkv_w;    // [(Hq + 2 Hkv) D, H]
  const __nv_bfloat16* qn_w;     // [D]
  const __nv_bfloat16* kn_w;     // [D]
  const __nv_bfloat16* o_w;      // [H, Hq D]
  const __nv_bfloat16* post_w;   // [H]
  const __nv_bfloat16* gu_w;     // [2 I, H]
  const __nv_bfloat16* down_w;   // [H, I]
  __nv_bfloat16* k_cache;        // [Hkv, S, D] (batch 1)
  __nv_bfloat16* v_cache;
};

struct DsParams {
  const DsLayer* layers;            // [L] in device memory
  const __nv_bfloat16* embed;       // [V, H]
  const __nv_bfloat16* final_norm;  // [H]
  const __nv_bfloat16* lm_head;     // [V, H]
  const __nv_bfloat16* rope_cos;    // [S, D/2]
  const __nv_bfloat16* rope_sin;
  int64_t* ids;                     // [1] in: this step's token, out: the next token
  int* cache_pos;                   // [1]
  __nv_bfloat16* x;                 // [H] residual stream
  __nv_bfloat16* h;                 // [H]
  __nv_bfloat16* qkv;               // [(Hq + 2 Hkv) D]
  __nv_bfloat16* attn;              // [Hq D]
  __nv_bfloat16* act;               // [I]
  float* attn_part;                 // [Hkv][splits][rows][D + 2]
  unsigned int* head_counters;      // [Hkv] zero between steps
  float* best_val;                  // [grid]
  int* best_idx;                    // [grid]
  unsigned int* barrier;            // zeroed before every launch
  unsigned int* head_counter;       // [1] zero between steps
  int* err;
  unsigned long long* trace;        // optional: per barrier and CTA, globaltimer at arrival and at release
  int L, H, I, Hq, Hkv, V, S, splits;
  float eps, scale_log2;
};

// ---------------------------------------------------------------------------
// Grid barrier (all CTAs resident: cooperative launch).  Returns false when
// the step was aborted (a bounded wait ran out somewhere).
// ---------------------------------------------------------------------------
__device__ __forceinline__ unsigned int ld_acquire_u32(const unsigned int* p) {
  unsigned int v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ bool ds_grid_sync(const DsParams& p, unsigned int& gen, int* s_abort) {
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned long long* tr =
        p.trace ? p.trace + ((size_t)(gen / gridDim.x) * gridDim.x + blockIdx.x) * 2 : nullptr;
    if (tr) tr[0] = global_timer_ns();
    gen += gridDim.x;
    __threadfence();
    atomicAdd(p.barrier, 1u);
    const WaitClock clk(p.err);
    while (ld_acquire_u32(p.barrier) < gen) {
      if (ld_acquire_u32(p.barrier + 1) != 0u) {  // another CTA aborted
        *s_abort = 1;
        break;
      }
      if (clk.expired()) {
        raise_device_error(p.err, 7 | (16 << 8));
        atomicExch(p.barrier + 1, 1u);
        *s_abort = 1;
        break;
      }
    }
    __threadfence();
    if (tr) tr[1] = global_timer_ns();
  } else {
    gen += gridDim.x;
  }
  __syncthreads();
  return *(volatile int*)s_abort == 0;
}

__device__ __forceinline__ uint4 ldcg16(const void* ptr) { return __ldcg(reinterpret_cast<const uint4*>(ptr)); }

// Load a bf16 vector written by other CTAs into shared memory, optionally
// RMS-normalised with weight w: xs = bf16((v * rsqrt(mean(v^2) + eps)) * w).
__device__ void ds_load_vec(const __nv_bfloat16* v, int n, const __nv_bfloat16* w, float eps, __nv_bfloat16* xs,
                            float* red) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nv = n >> 3;
  float r = 1.f;
  if (w) {
    float ss = 0.f;
    for (int i = tid; i < nv; i += kDsThreads) {
      float f[8];
      unpack8(ldcg16(v + i * 8), f);
#pragma unroll
      for (int j = 0; j < 8; ++j) ss = fmaf(f[j], f[j], ss);
    }
    ss = warp_sum(ss);
    if (lane == 0) red[warp] = ss;
    __syncthreads();
    if (warp == 0) {
      float t = lane < kDsWarps ? red[lane] : 0.f;
      t = warp_sum(t);
      if (lane == 0) red[kDsWarps] = rsqrtf(t / (float)n + eps);
    }
    __syncthreads();
    r = red[kDsWarps];
  }
  for (int i = tid; i < nv; i += kDsThreads) {
    const uint4 raw = ldcg16(v + i * 8);
    if (w) {
      float f[8], wf[8];
      unpack8(raw, f);
      unpack8(ldg16(w + i * 8), wf);
      uint4 o;
      uint32_t* op = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        __nv_bfloat162 pr = __floats2bfloat162_rn((f[2 * j] * r) * wf[2 * j], (f[2 * j + 1] * r) * wf[2 * j + 1]);
        op[j] = *reinterpret_cast<uint32_t*>(&pr);
      }
      *reinterpret_cast<uint4*>(xs + i * 8) = o;
    } else {
      *reinterpret_cast<uint4*>(xs + i * 8) = raw;
    }
  }
  __syncthreads();
}

// Unit range [u0, u1) of CTA c when `units` are split evenly over the grid.
__device__ __forceinline__ void ds_range(int units, int& u0, int& u1) {
  u0 = (int)(((int64_t)units * blockIdx.x) / gridDim.x);
  u1 = (int)(((int64_t)units * (blockIdx.x + 1)) / gridDim.x);
}

// L2 prefetch of the first bytes of this CTA's rows [u0, u1) of W (and of the
// paired up rows when pair_offset_rows > 0).
__device__ __forceinline__ void ds_prefetch_rows(const __nv_bfloat16* w, int K, int units, int pair_offset_rows) {
  if (threadIdx.x != 0) return;
  int u0, u1;
  ds_range(units, u0, u1);
  const size_t range = (size_t)(u1 - u0) * K * 2;
  const uint32_t pf = (uint32_t)(range < kDsPrefetch ? range : kDsPrefetch);
  const char* a = reinterpret_cast<const char*>(w + (size_t)u0 * K);
  for (uint32_t off = 0; off < pf; off += 16384) prefetch_l2(a + off, min(16384u, pf - off));
  if (pair_offset_rows > 0) {
    const char* b = reinterpret_cast<const char*>(w + ((size_t)u0 + pair_offset_rows) * K);
    for (uint32_t off = 0; off < pf; off += 16384) prefetch_l2(b + off, min(16384u, pf - off));
  }
}

enum { DS_STORE = 0, DS_RESIDUAL = 1, DS_SILU = 2, DS_ARGMAX = 3 };

// One GEMV phase: this CTA's rows of W (K wide) against xs (smem), the
// reference's rounding in the epilogue.  RPU = 2 pairs row u with row u + N/2.
template <int EPI>
__device__ void ds_gemv(const __nv_bfloat16* W, int N, int K, const __nv_bfloat16* xs, float* segbuf, int seg_cap,
                        const __nv_bfloat16* residual, __nv_bfloat16* out, float* best_v, int* best_i) {
  constexpr int RPU = (EPI == DS_SILU) ? 2 : 1;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int units = (EPI == DS_SILU) ? N / 2 : N;
  int u0, u1;
  ds_range(units, u0, u1);
  const int P = u1 - u0, R = P * RPU;
  const int gpr = (K + kDsGranule - 1) / kDsGranule;
  const int total = R * gpr;
  const int g_begin = (int)(((int64_t)total * warp) / kDsWarps);
  const int g_end = (int)(((int64_t)total * (warp + 1)) / kDsWarps);
  const int t_first = g_begin / gpr;
  int g = g_begin;
  while (g < g_end) {
    const int t = g / gpr;
    const int kg0 = g - t * gpr;
    const int seg = min(g_end, (t + 1) * gpr) - g;
    const int row = (RPU == 2) ? ((t < P) ? (u0 + t) : (u0 + (t - P) + N / 2)) : (u0 + t);
    const __nv_bfloat16* wrow = W + (size_t)row * K;
    float a = 0.f;
    for (int kk = 0; kk < seg; kk += kDsUnroll) {
      uint4 wv[kDsUnroll];
      bool ok[kDsUnroll];
#pragma unroll
      for (int u = 0; u < kDsUnroll; ++u) {
        const int k = (kg0 + kk + u) * kDsGranule + lane * 8;
        ok[u] = (kk + u < seg) && (k < K);
        wv[u] = ok[u] ? ldg_stream(wrow + k) : make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int u = 0; u < kDsUnroll; ++u) {
        if (ok[u]) {
          const int k = (kg0 + kk + u) * kDsGranule + lane * 8;
          a = dot8(wv[u], *reinterpret_cast<const uint4*>(xs + k), a);
        }
      }
    }
    a = warp_sum(a);
    if (lane == 0 && t - t_first < seg_cap) segbuf[warp * seg_cap + (t - t_first)] = a;
    g += seg;
  }
  // Rows [s_wr0[w], s_wr1[w]] of warp w (empty: r0 > r1), once per call instead of per output.
  __shared__ int s_wr0[kDsWarps], s_wr1[kDsWarps];
  if (tid < kDsWarps) {
    const int wb = (int)(((int64_t)total * tid) / kDsWarps);
    const int we = (int)(((int64_t)total * (tid + 1)) / kDsWarps);
    s_wr0[tid] = wb < we ? wb / gpr : 1;
    s_wr1[tid] = wb < we ? (we - 1) / gpr : 0;
  }
  __syncthreads();
  auto row_sum = [&](int t) -> float {
    float s = 0.f;
#pragma unroll 4
    for (int w = 0; w < kDsWarps; ++w) {
      const int f = s_wr0[w];
      if (t >= f && t <= s_wr1[w]) s += segbuf[w * seg_cap + (t - f)];
    }
    return s;
  };
  if (EPI == DS_ARGMAX) {
    float best = -INFINITY;
    int besti = 0x7fffffff;
    for (int t = tid; t < P; t += kDsThreads) {
      const float v = round_bf16(row_sum(t));
      if (v > best || (v == best && u0 + t < besti)) { best = v; besti = u0 + t; }
    }
    *best_v = best;
    *best_i = besti;
  } else {
    for (int t = tid; t < P; t += kDsThreads) {
      const int u = u0 + t;
      if (EPI == DS_STORE) {
        out[u] = f_to_bf16(row_sum(t));
      } else if (EPI == DS_RESIDUAL) {
        out[u] = f_to_bf16(bf16_to_f(__ldcg(residual + u)) + round_bf16(row_sum(t)));
      } else {
        const float gt = round_bf16(row_sum(t));
        const float up = round_bf16(row_sum(P + t));
        out[u] = f_to_bf16(round_bf16(gt / (1.0f + expf(-gt))) * up);
      }
    }
  }
  __syncthreads();
}

// Shared memory of the step kernel.
struct DsSmem {
  __nv_bfloat16 xs[16384];                        // activation vector (<= 16384 wide)
  float segbuf[kDsWarps * 64];                    // per-warp row partials
  float red[kDsWarps + 1];
  // attention
  float q[kDsMaxRows][kDsHeadDim];                // normed + rotated query rows (fp32)
  float knew[kDsHeadDim], vnew[kDsHeadDim];       // the new token's k (rotated) and v
  float wm[kDsAttnWarps][kDsMaxRows], wl[kDsAttnWarps][kDsMaxRows];
  float wo[kDsAttnWarps][kDsMaxRows][kDsHeadDim];
  float bv[kDsWarps];
  int bi[kDsWarps];
  int abort_flag;
  int is_last;
};

// RMSNorm over one head (128 values, one warp) + NeoX RoPE at position pos,
// with the reference's bf16 rounding; lane holds elements 4*lane .. 4*lane+3.
__device__ __forceinline__ void ds_norm_rope_head(const __nv_bfloat16* src, const __nv_bfloat16* nw, float eps,
                                                  const __nv_bfloat16* cos_row, const __nv_bfloat16* sin_row,
                                                  float out[4]) {
  const int lane = threadIdx.x & 31;
  const int e0 = lane * 4;
  const uint2 raw_u = __ldcg(reinterpret_cast<const uint2*>(src + e0));
  const float raw[4] = {bf16_lo(raw_u.x), bf16_hi(raw_u.x), bf16_lo(raw_u.y), bf16_hi(raw_u.y)};
  float ss = raw[0] * raw[0] + raw[1] * raw[1] + raw[2] * raw[2] + raw[3] * raw[3];
  ss = warp_sum(ss);
  const float r = rsqrtf(ss / (float)kDsHeadDim + eps);
  const uint2 w_u = *reinterpret_cast<const uint2*>(nw + e0);
  const float wv[4] = {bf16_lo(w_u.x), bf16_hi(w_u.x), bf16_lo(w_u.y), bf16_hi(w_u.y)};
  float n[4], other[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) n[j] = round_bf16((raw[j] * r) * wv[j]);
#pragma unroll
  for (int j = 0; j < 4; ++j) other[j] = __shfl_xor_sync(0xffffffffu, n[j], 16);
  const bool first = lane < 16;
  const int idx = first ? e0 : e0 - kDsHeadDim / 2;
  const uint2 c_u = *reinterpret_cast<const uint2*>(cos_row + idx);
  const uint2 s_u = *reinterpret_cast<const uint2*>(sin_row + idx);
  const float c[4] = {bf16_lo(c_u.x), bf16_hi(c_u.x), bf16_lo(c_u.y), bf16_hi(c_u.y)};
  const float s[4] = {bf16_lo(s_u.x), bf16_hi(s_u.x), bf16_lo(s_u.y), bf16_hi(s_u.y)};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    if (first) out[j] = round_bf16(round_bf16(n[j] * c[j]) - round_bf16(other[j] * s[j]));
    else out[j] = round_bf16(round_bf16(n[j] * c[j]) + round_bf16(other[j] * s[j]));
  }
}

// Attention phase work item (kv head h, split s) for the single new token at pos.
__device__ void ds_attention_item(const DsParams& p, const DsLayer& ly, int hkv, int s, int pos, DsSmem& sm) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int G = p.Hq / p.Hkv;
  const __nv_bfloat16* cos_row = p.rope_cos + (size_t)pos * (kDsHeadDim / 2);
  const __nv_bfloat16* sin_row = p.rope_sin + (size_t)pos * (kDsHeadDim / 2);
  // q rows of this group and the new k / v (warps 0..G-1: q heads, warp G: k, warp G+1: v)
  if (warp < G) {
    float o[4];
    ds_norm_rope_head(p.qkv + (size_t)(hkv * G + warp) * kDsHeadDim, ly.qn_w, p.eps, cos_row, sin_row, o);
#pragma unroll
    for (int j = 0; j < 4; ++j) sm.q[warp][lane * 4 + j] = o[j] * p.scale_log2;
  } else if (warp == G) {
    float o[4];
    ds_norm_rope_head(p.qkv + (size_t)(p.Hq + hkv) * kDsHeadDim, ly.kn_w, p.eps, cos_row, sin_row, o);
#pragma unroll
    for (int j = 0; j < 4; ++j) sm.knew[lane * 4 + j] = o[j];
    if (s == 0) {
      __nv_bfloat162 lo2 = __floats2bfloat162_rn(o[0], o[1]);
      __nv_bfloat162 hi2 = __floats2bfloat162_rn(o[2], o[3]);
      *reinterpret_cast<uint2*>(ly.k_cache + ((size_t)hkv * p.S + pos) * kDsHeadDim + lane * 4) =
          make_uint2(*reinterpret_cast<uint32_t*>(&lo2), *reinterpret_cast<uint32_t*>(&hi2));
    }
  } else if (warp == G + 1) {
    const uint2 v_u = __ldcg(reinterpret_cast<const uint2*>(p.qkv + (size_t)(p.Hq + p.Hkv + hkv) * kDsHeadDim +
                                                             lane * 4));
    sm.vnew[lane * 4 + 0] = bf16_lo(v_u.x);
    sm.vnew[lane * 4 + 1] = bf16_hi(v_u.x);
    sm.vnew[lane * 4 + 2] = bf16_lo(v_u.y);
    sm.vnew[lane * 4 + 3] = bf16_hi(v_u.y);
    if (s == 0) *reinterpret_cast<uint2*>(ly.v_cache + ((size_t)hkv * p.S + pos) * kDsHeadDim + lane * 4) = v_u;
  }
  __syncthreads();
  const int L = pos + 1;
  int chunk = (L + p.splits - 1) / p.splits;
  chunk = max(chunk, 16);
  const int j0 = min(s * chunk, L), j1 = min(j0 + chunk, L);
  if (warp < kDsAttnWarps) {
    float qf[kDsMaxRows][4];
    float m[kDsMaxRows], l[kDsMaxRows], o[kDsMaxRows][4];
#pragma unroll
    for (int r = 0; r < kDsMaxRows; ++r) {
      m[r] = -INFINITY;
      l[r] = 0.f;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        o[r][j] = 0.f;
        qf[r][j] = r < G ? sm.q[r][lane * 4 + j] : 0.f;
      }
    }
    const __nv_bfloat16* kb = ly.k_cache + (size_t)hkv * p.S * kDsHeadDim + lane * 4;
    const __nv_bfloat16* vb = ly.v_cache + (size_t)hkv * p.S * kDsHeadDim + lane * 4;
    for (int j = j0 + warp; j < j1; j += kDsAttnWarps) {
      float k4[4], v4[4];
      if (j == pos) {
#pragma unroll
        for (int e = 0; e < 4; ++e) { k4[e] = sm.knew[lane * 4 + e]; v4[e] = sm.vnew[lane * 4 + e]; }
      } else {
        const uint2 ku = *reinterpret_cast<const uint2*>(kb + (size_t)j * kDsHeadDim);
        const uint2 vu = *reinterpret_cast<const uint2*>(vb + (size_t)j * kDsHeadDim);
        k4[0] = bf16_lo(ku.x); k4[1] = bf16_hi(ku.x); k4[2] = bf16_lo(ku.y); k4[3] = bf16_hi(ku.y);
        v4[0] = bf16_lo(vu.x); v4[1] = bf16_hi(vu.x); v4[2] = bf16_lo(vu.y); v4[3] = bf16_hi(vu.y);
      }
#pragma unroll
      for (int r = 0; r < kDsMaxRows; ++r) {
        if (r >= G) break;
        float d = qf[r][0] * k4[0];
        d = fmaf(qf[r][1], k4[1], d);
        d = fmaf(qf[r][2], k4[2], d);
        d = fmaf(qf[r][3], k4[3], d);
        d = warp_sum(d);
        const float mn = fmaxf(m[r], d);
        const float corr = exp2f(m[r] - mn);
        const float pr = exp2f(d - mn);
        l[r] = fmaf(l[r], corr, pr);
#pragma unroll
        for (int e = 0; e < 4; ++e) o[r][e] = fmaf(o[r][e], corr, pr * v4[e]);
        m[r] = mn;
      }
    }
#pragma unroll
    for (int r = 0; r < kDsMaxRows; ++r) {
      if (r >= G) break;
      if (lane == 0) { sm.wm[warp][r] = m[r]; sm.wl[warp][r] = l[r]; }
#pragma unroll
      for (int e = 0; e < 4; ++e) sm.wo[warp][r][lane * 4 + e] = o[r][e];
    }
  }
  __syncthreads();
  // merge the attention warps into this item's partial (thread = (row, dim))
  float* part = p.attn_part + (((size_t)hkv * p.splits + s) * kDsMaxRows) * (kDsHeadDim + 2);
  for (int e = tid; e < G * kDsHeadDim; e += kDsThreads) {
    const int r = e / kDsHeadDim, d = e - r * kDsHeadDim;
    float mx = -INFINITY;
    for (int w = 0; w < kDsAttnWarps; ++w) mx = fmaxf(mx, sm.wm[w][r]);
    float ls = 0.f, acc = 0.f;
    if (mx != -INFINITY)
      for (int w = 0; w < kDsAttnWarps; ++w) {
        const float sc = exp2f(sm.wm[w][r] - mx);
        ls += sm.wl[w][r] * sc;
        acc += sm.wo[w][r][d] * sc;
      }
    part[r * (kDsHeadDim + 2) + d] = acc;
    if (d == 0) {
      part[r * (kDsHeadDim + 2) + kDsHeadDim] = mx;
      part[r * (kDsHeadDim + 2) + kDsHeadDim + 1] = ls;
    }
  }
  __threadfence();
  __syncthreads();
  if (tid == 0) sm.is_last = atomicAdd(p.head_counters + hkv, 1u) == (unsigned int)p.splits - 1;
  __syncthreads();
  if (!sm.is_last) return;
  __threadfence();
  // The last split of this kv head merges all splits and writes the G query heads.
  const float* base = p.attn_part + ((size_t)hkv * p.splits * kDsMaxRows) * (kDsHeadDim + 2);
  for (int e = tid; e < G * kDsHeadDim; e += kDsThreads) {
    const int r = e / kDsHeadDim, d = e - r * kDsHeadDim;
    float mx = -INFINITY;
    for (int sp = 0; sp < p.splits; ++sp)
      mx = fmaxf(mx, __ldcg(base + ((size_t)sp * kDsMaxRows + r) * (kDsHeadDim + 2) + kDsHeadDim));
    float ls = 0.f, acc = 0.f;
    for (int sp = 0; sp < p.splits; ++sp) {
      const float* ent = base + ((size_t)sp * kDsMaxRows + r) * (kDsHeadDim + 2);
      const float ms = __ldcg(ent + kDsHeadDim);
      if (ms == -INFINITY) continue;
      const float sc = exp2f(ms - mx);
      ls += __ldcg(ent + kDsHeadDim + 1) * sc;
      acc += __ldcg(ent + d) * sc;
    }
    p.attn[(size_t)(hkv * G + r) * kDsHeadDim + d] = f_to_bf16(acc / ls);
  }
  if (tid == 0) p.head_counters[hkv] = 0u;
}

__global__ void __launch_bounds__(kDsThreads, 1) decode_step_kernel(DsParams p) {
  extern __shared__ __align__(16) unsigned char ds_smem_raw[];
  DsSmem& sm = *reinterpret_cast<DsSmem*>(ds_smem_raw);
  const int tid = threadIdx.x;
  unsigned int gen = 0;
  if (tid == 0) sm.abort_flag = 0;
  __syncthreads();
  const int pos = p.cache_pos[0];
  const int64_t token = p.ids[0];
  const int qkv_rows = (p.Hq + 2 * p.Hkv) * kDsHeadDim;
  const int qdim = p.Hq * kDsHeadDim;
  if (pos < 0 || pos >= p.S || token < 0 || token >= p.V) {
    if (tid == 0 && blockIdx.x == 0) raise_device_error(p.err, LS_ERR_KV_OVERFLOW);
    return;  // every CTA sees the same values and leaves together
  }
  const int seg_cap = 64;

  for (int li = 0; li < p.L; ++li) {
    const DsLayer ly = p.layers[li];
    // ---- QKV: input RMSNorm + fused projection ----
    const __nv_bfloat16* xin = (li == 0) ? (p.embed + (size_t)token * p.H) : p.x;
    if (li == 0 && blockIdx.x == 0) {
      for (int i = tid; i < p.H / 8; i += kDsThreads)
        *reinterpret_cast<uint4*>(p.x + i * 8) = ldg16(xin + i * 8);
    }
    ds_load_vec(xin, p.H, ly.ln_w, p.eps, sm.xs, sm.red);
    ds_gemv<DS_STORE>(ly.qkv_w, qkv_rows, p.H, sm.xs, sm.segbuf, seg_cap, nullptr, p.qkv, nullptr, nullptr);
    ds_prefetch_rows(ly.o_w, qdim, p.H, 0);
    if (!ds_grid_sync(p, gen, &sm.abort_flag)) return;
    // ---- ATTN ----
    for (int item = blockIdx.x; item < p.Hkv * p.splits; item += gridDim.x)
      ds_attention_item(p, ly, item / p.splits, item % p.splits, pos, sm);
    if (!ds_grid_sync(p, gen, &sm.abort_flag)) return;
    // ---- O: o_proj + residual ----
    ds_load_vec(p.attn, qdim, nullptr, 0.f, sm.xs, sm.red);
    ds_gemv<DS_RESIDUAL>(ly.o_w, p.H, qdim, sm.xs, sm.segbuf, seg_cap, p.x, p.h, nullptr, nullptr);
    ds_prefetch_rows(ly.gu_w, p.H, p.I, p.I);
    if (!ds_grid_sync(p, gen, &sm.abort_flag)) return;
    // ---- GU: post-attention RMSNorm + gate/up + SiLU*up ----
    ds_load_vec(p.h, p.H, ly.post_w, p.eps, sm.xs, sm.red);
    ds_gemv<DS_SILU>(ly.gu_w, 2 * p.I, p.H, sm.xs, sm.segbuf, seg_cap, nullptr, p.act, nullptr, nullptr);
    ds_prefetch_rows(ly.down_w, p.I, p.H, 0);
    if (!ds_grid_sync(p, gen, &sm.abort_flag)) return;
    // ---- DOWN + residual ----
    ds_load_vec(p.act, p.I, nullptr, 0.f, sm.xs, sm.red);
    ds_gemv<DS_RESIDUAL>(ly.down_w, p.H, p.I, sm.xs, sm.segbuf, seg_cap, p.h, p.x, nullptr, nullptr);
    if (li + 1 < p.L) ds_prefetch_rows(p.layers[li + 1].qkv_w, p.H, qkv_rows, 0);
    else ds_prefetch_rows(p.lm_head, p.H, p.V, 0);
    if (!ds_grid_sync(p, gen, &sm.abort_flag)) return;
  }
  // ---- HEAD: final RMSNorm + lm_head + argmax ----
  ds_load_vec(p.x, p.H, p.final_norm, p.eps, sm.xs, sm.red);
  float best = -INFINITY;
  int besti = 0x7fffffff;
  ds_gemv<DS_ARGMAX>(p.lm_head, p.V, p.H, sm.xs, sm.segbuf, seg_cap, nullptr, nullptr, &best, &besti);
  {
    const int lane = tid & 31, warp = tid >> 5;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, best, o);
      const int oi = __shfl_xor_sync(0xffffffffu, besti, o);
      if (ov > best || (ov == best && oi < besti)) { best = ov; besti = oi; }
    }
    if (lane == 0) { sm.bv[warp] = best; sm.bi[warp] = besti; }
    __syncthreads();
    if (tid == 0) {
      for (int w = 1; w < kDsWarps; ++w)
        if (sm.bv[w] > best || (sm.bv[w] == best && sm.bi[w] < besti)) { best = sm.bv[w]; besti = sm.bi[w]; }
      p.best_val[blockIdx.x] = best;
      p.best_idx[blockIdx.x] = besti;
      __threadfence();
      sm.is_last = atomicAdd(p.head_counter, 1u) == gridDim.x - 1;
    }
    __syncthreads();
    if (sm.is_last && tid == 0) {
      __threadfence();
      float bb = -INFINITY;
      int bj = 0x7fffffff;
      for (int c = 0; c < (int)gridDim.x; ++c) {
        const float v = __ldcg(p.best_val + c);
        const int j = __ldcg(p.best_idx + c);
        if (v > bb || (v == bb && j < bj)) { bb = v; bj = j; }
      }
      p.ids[0] = (int64_t)bj;
      p.cache_pos[0] = pos + 1;
      *p.head_counter = 0u;
    }
  }
}

}  // namespace lsb

namespace lsb_host {
// Profiling hook: when set, every barrier of the next decode_step launches
// records (arrival, release) globaltimer stamps per CTA into this buffer.
#ifdef LEANB200_PROFILING
static unsigned long long* g_ds_trace = nullptr;
#endif
}  // namespace lsb_host

namespace lsb_host {
using namespace lsb;

size_t decode_step_smem() { return sizeof(DsSmem); }

int decode_step_splits(int hkv) {
  int splits = 1;
  while (splits < 32 && hkv * splits * 2 <= sm_count()) splits *= 2;
  return splits;
}

int launch_decode_step(const DsParams& p, cudaStream_t stream) {
  static int configured[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  const size_t smem = sizeof(DsSmem);
  if (dev >= 0 && dev < 64 && !configured[dev]) {
    cudaError_t e = cudaFuncSetAttribute(decode_step_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return set_error(LS_ERR_CUDA, "decode_step smem attribute: %s", cudaGetErrorString(e));
    configured[dev] = 1;
  }
  cudaError_t e = cudaMemsetAsync(p.barrier, 0, 2 * sizeof(unsigned int), stream);  // arrivals, abort flag
  if (e != cudaSuccess) return set_error(LS_ERR_CUDA, "decode_step barrier reset: %s", cudaGetErrorString(e));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(sm_count());
  cfg.blockDim = dim3(kDsThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  e = cudaLaunchKernelEx(&cfg, decode_step_kernel, p);
  if (e != cudaSuccess) return set_error(LS_ERR_CUDA, "decode_step launch: %s", cudaGetErrorString(e));
  return LS_OK;
}

static size_t align256(size_t v) { return (v + 255) / 256 * 256; }

struct DsWorkspace {
  size_t barrier, head_counters, best_val, best_idx, attn_part, total;
};

static DsWorkspace ds_workspace(int hkv, int splits, int grid) {
  DsWorkspace w;
  w.barrier = 0;  // [0] arrivals, [1] abort flag, [2] head argmax counter
  w.head_counters = 256;
  w.best_val = w.head_counters + align256((size_t)hkv * 4);
  w.best_idx = w.best_val + align256((size_t)grid * 4);
  w.attn_part = w.best_idx + align256((size_t)grid * 4);
  w.total = w.attn_part + align256((size_t)hkv * splits * kDsMaxRows * (kDsHeadDim + 2) * 4);
  return w;
}

int decode_step_workspace_bytes(int64_t hkv, int64_t* bytes) {
  *bytes = (int64_t)ds_workspace((int)hkv, decode_step_splits((int)hkv), sm_count()).total;
  return LS_OK;
}

// Largest per-warp segment count over the phases (must fit the segbuf).
static int ds_max_segs(int units, int rpu, int K, int grid) {
  const int gpr = (K + kDsGranule - 1) / kDsGranule;
  const int per_cta = (units + grid - 1) / grid;
  const int total = per_cta * rpu * gpr;
  const int range = (total + kDsWarps - 1) / kDsWarps;
  return range / gpr + 2;
}

int decode_step(const void* layers, int64_t L, int64_t H, int64_t I, int64_t hq, int64_t hkv, int64_t head_dim,
                int64_t vocab, int64_t max_seq, float eps, const void* embed, const void* final_norm,
                const void* lm_head, const void* cos, const void* sin, int64_t* ids, int32_t* cache_pos, void* x,
                void* h, void* qkv, void* attn, void* act, void* workspace, int64_t workspace_bytes,
                cudaStream_t stream) {
  if (head_dim != kDsHeadDim) return set_error(LS_ERR_UNSUPPORTED_SHAPE, "decode_step: head_dim must be 128");
  if (hq % hkv || hq / hkv > kDsMaxRows || hq / hkv + 2 > kDsWarps)
    return set_error(LS_ERR_UNSUPPORTED_SHAPE, "decode_step: GQA group of %lld rows unsupported", (long long)(hq / hkv));
  const int64_t qdim = hq * head_dim;
  if (H > 16384 || I > 16384 || qdim > 16384 || H % 8 || I % 8)
    return set_error(LS_ERR_UNSUPPORTED_SHAPE, "decode_step: vectors wider than 16384 or not multiples of 8");
  const int grid = sm_count();
  const int splits = decode_step_splits((int)hkv);
  const int segs[] = {ds_max_segs((int)((hq + 2 * hkv) * head_dim), 1, (int)H, grid),
                      ds_max_segs((int)H, 1, (int)qdim, grid), ds_max_segs((int)I, 2, (int)H, grid),
                      ds_max_segs((int)H, 1, (int)I, grid), ds_max_segs((int)vocab, 1, (int)H, grid)};
  for (int sgs : segs)
    if (sgs > 64) return set_error(LS_ERR_UNSUPPORTED_SHAPE, "decode_step: %d row segments per warp (max 64)", sgs);
  const DsWorkspace w = ds_workspace((int)hkv, splits, grid);
  if (!workspace || workspace_bytes < (int64_t)w.total)
    return set_error(LS_ERR_WORKSPACE, "decode_step: workspace needs %zu bytes", w.total);
  char* ws = static_cast<char*>(workspace);
  DsParams p = {};
  p.layers = static_cast<const DsLayer*>(layers);
  p.embed = static_cast<const __nv_bfloat16*>(embed);
  p.final_norm = static_cast<const __nv_bfloat16*>(final_norm);
  p.lm_head = static_cast<const __nv_bfloat16*>(lm_head);
  p.rope_cos = static_cast<const __nv_bfloat16*>(cos);
  p.rope_sin = static_cast<const __nv_bfloat16*>(sin);
  p.ids = ids;
  p.cache_pos = cache_pos;
  p.x = static_cast<__nv_bfloat16*>(x);
  p.h = static_cast<__nv_bfloat16*>(h);
  p.qkv = static_cast<__nv_bfloat16*>(qkv);
  p.attn = static_cast<__nv_bfloat16*>(attn);
  p.act = static_cast<__nv_bfloat16*>(act);
  p.barrier = reinterpret_cast<unsigned int*>(ws + w.barrier);
  p.head_counter = reinterpret_cast<unsigned int*>(ws + w.barrier) + 2;
  p.head_counters = reinterpret_cast<unsigned int*>(ws + w.head_counters);
  p.best_val = reinterpret_cast<float*>(ws + w.best_val);
  p.best_idx = reinterpret_cast<int*>(ws + w.best_idx);
  p.attn_part = reinterpret_cast<float*>(ws + w.attn_part);
  p.err = device_error_ptr();
#ifdef LEANB200_PROFILING
  p.trace = g_ds_trace;
#endif
  p.L = (int)L;
  p.H = (int)H;
  p.I = (int)I;
  p.Hq = (int)hq;
  p.Hkv = (int)hkv;
  p.V = (int)vocab;
  p.S = (int)max_seq;
  p.splits = splits;
  p.eps = eps;
  p.scale_log2 = (1.0f / sqrtf((float)head_dim)) * 1.4426950408889634f;
  return launch_decode_step(p, stream);
}

}  // namespace lsb_host

#ifdef LEANB200_PROFILING
extern "C" int ls_decode_step_set_trace(void* buffer) {
  lsb_host::g_ds_trace = static_cast<unsigned long long*>(buffer);
  return LS_OK;
}
#endif
