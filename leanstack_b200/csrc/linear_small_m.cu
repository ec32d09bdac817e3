// Skinny-M linear layers on the CUDA cores: y[m, n] = sum_k W[n, k] * x[m, k]
// for m <= 8 activation rows (bs1 decode and small batches).
//
// These layers are HBM-bound: every weight byte is used m times, so the
// kernel's only job is to stream W at full bandwidth.  Design:
//   * grid = 2 CTAs per SM, each CTA owns a contiguous, balanced range of
//     output "units" (a row, or a gate/up row pair for the SiLU epilogue), so
//     every SM streams the same number of bytes;
//   * the CTA's rows are cut into 512-byte granules (32 lanes x 16 B) and the
//     flat granule list is split evenly over the warps; a warp issues U
//     independent 16-byte streaming loads before it consumes any of them;
//   * the (optionally RMS-normalised) activations sit in shared memory as bf16;
//   * per-row partial sums meet in shared memory, then the epilogue applies
//     the reference's bf16 rounding points.
//
// Rounding follows the reference's torch ops (src/leanstack/runtime/
// qwen_explicit.py): F.rms_norm gives bf16((x * r) * w) with r in fp32; mv /
// linear accumulate in fp32 and round once; the residual add, SiLU and the
// gate*up product each round to bf16 (:809-852, :932-949).  The argmax
// epilogue reproduces torch.argmax over bf16 logits (lowest index on ties).
#include <cstdlib>

#include "common.cuh"

namespace lsb {

constexpr int kLinThreads = 512;
constexpr int kLinWarps = kLinThreads / 32;
constexpr int kGranule = 256;  // bf16 elements per warp-wide 512-byte load
constexpr uint32_t kPrefetchBytes = 64 * 1024;  // per CTA and weight range, issued before the PDL wait

enum { EPI_STORE = 0, EPI_RESIDUAL = 1, EPI_SILU_MUL = 2, EPI_ARGMAX = 3, EPI_STORE_F32 = 4, EPI_AR_RESIDUAL = 5 };

struct LinearParams {
  const __nv_bfloat16* x;      // [M, K]
  const __nv_bfloat16* norm_w; // [K] or null
  const __nv_bfloat16* w;      // [N, K]
  const __nv_bfloat16* residual;  // [M, N] (EPI_RESIDUAL)
  __nv_bfloat16* out;          // [M, N] or [M, N/2]
  float eps;
  int K;
  int N;        // weight rows
  int units;    // N, or N/2 for EPI_SILU_MUL
  int max_local_units;  // ceil(units / gridDim.x)
  int max_segs;         // row segments one warp can touch
  // EPI_ARGMAX
  float* part_val;       // [M, gridDim.x]
  int* part_idx;         // [M, gridDim.x]
  unsigned int* counter; // 1 int, zero between calls
  int64_t* out_ids;      // [M]: winning row index, or its argmax_key when out_keys
  int64_t id_offset;     // added to the winning row index (vocab shard offset)
  int out_keys;
  // EPI_AR_RESIDUAL: tensor-parallel exchange regions
  P2PExchange ex;
  int* err;
  unsigned long long* trace;  // optional profiling: per CTA 5 globaltimer stamps
};

template <int M>
struct LinUnroll { static constexpr int value = (M <= 2) ? 8 : ((M <= 4) ? 6 : 4); };

template <int M>
struct LinMinBlocks { static constexpr int value = (M <= 4) ? 2 : 1; };

template <int M, int EPI, bool NORM>
__global__ void __launch_bounds__(kLinThreads, LinMinBlocks<M>::value) linear_small_m_kernel(LinearParams p) {
  constexpr int U = LinUnroll<M>::value;
  constexpr int RPU = (EPI == EPI_SILU_MUL) ? 2 : 1;  // weight rows per unit
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const int K = p.K;
  __nv_bfloat16* xs = reinterpret_cast<__nv_bfloat16*>(smem_raw);  // [M, K]
  const int k_pad = (K + 7) & ~7;
  // Per-warp partial sums, one slot per (row segment, activation row): each
  // warp covers a contiguous granule range, so it touches each row at most
  // once; rows are then summed over warps in a fixed order (deterministic).
  float* segbuf = reinterpret_cast<float*>(smem_raw + ((size_t)M * k_pad * 2 + 15) / 16 * 16);
  __shared__ float red[kLinWarps][M];
  __shared__ float rscale[M];

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int G = gridDim.x;
  const int u0 = (int)(((int64_t)p.units * blockIdx.x) / G);
  const int u1 = (int)(((int64_t)p.units * (blockIdx.x + 1)) / G);
  const int P = u1 - u0;            // units owned by this CTA
  const int R = P * RPU;            // weight rows owned by this CTA
  const int ms = p.max_segs;

  unsigned long long* tr = p.trace ? p.trace + (size_t)blockIdx.x * 5 : nullptr;
  if (tr && tid == 0) tr[0] = global_timer_ns();
  // Weights do not depend on the previous kernel: start pulling this CTA's
  // first weight bytes into L2, let the next kernel launch, and only then wait
  // (PDL) for the activations the previous kernel writes.
  if (tid == 0 && P > 0) {
    const size_t range = (size_t)P * K * 2;
    const uint32_t pf = (uint32_t)(range < kPrefetchBytes ? range : kPrefetchBytes);
    const char* base = reinterpret_cast<const char*>(p.w + (size_t)u0 * K);
    for (uint32_t off = 0; off < pf; off += 16384) prefetch_l2(base + off, min(16384u, pf - off));
    if (RPU == 2) {
      const char* up = reinterpret_cast<const char*>(p.w + ((size_t)u0 + p.N / 2) * K);
      for (uint32_t off = 0; off < pf; off += 16384) prefetch_l2(up + off, min(16384u, pf - off));
    }
  }
  // The norm weight does not depend on the previous kernel either: this
  // thread's first 16-byte vector of it is loaded before the wait.
  const int kvec = K >> 3;  // 16-byte vectors per activation row
  const uint4 nw0 = (NORM && tid < kvec) ? ldg16(p.norm_w + tid * 8) : make_uint4(0, 0, 0, 0);
  grid_dep_launch();
  grid_dep_wait();
  if (tr && tid == 0) tr[1] = global_timer_ns();
  __shared__ uint32_t s_epoch;
  if (EPI == EPI_AR_RESIDUAL && tid == 0) {  // per-CTA call counter of the fused all-reduce
    uint32_t* ctr = reinterpret_cast<uint32_t*>(p.ex.peer[p.ex.rank] + p2p_ctr_offset(p.ex.max_ctas)) + blockIdx.x;
    s_epoch = *ctr + 1u;
    *ctr = s_epoch;
  }

  // ---- prologue: (optional) RMSNorm of the M activation rows into smem ----
  if (NORM) {
    // x is read from L2 once: the vectors of the first pass stay in registers
    // for the second (one vector per thread and row covers K <= 4096).
    constexpr int XC = (M <= 2) ? M : 1;
    uint4 xc[XC];
    float ss[M];
#pragma unroll
    for (int m = 0; m < M; ++m) ss[m] = 0.f;
    for (int v = tid; v < kvec; v += kLinThreads) {
#pragma unroll
      for (int m = 0; m < M; ++m) {
        float f[8];
        const uint4 xv = ldg16(p.x + (size_t)m * K + v * 8);
        if (M <= 2 && v == tid) xc[m < XC ? m : 0] = xv;
        unpack8(xv, f);
#pragma unroll
        for (int j = 0; j < 8; ++j) ss[m] = fmaf(f[j], f[j], ss[m]);
      }
    }
#pragma unroll
    for (int m = 0; m < M; ++m) {
      float s = warp_sum(ss[m]);
      if (lane == 0) red[warp][m] = s;
    }
    __syncthreads();
    if (tid < M) {
      float s = 0.f;
      for (int w = 0; w < kLinWarps; ++w) s += red[w][tid];
      rscale[tid] = rsqrtf(s / (float)K + p.eps);
    }
    __syncthreads();
    for (int v = tid; v < kvec; v += kLinThreads) {
      float wf[8];
      unpack8(v == tid ? nw0 : ldg16(p.norm_w + v * 8), wf);
#pragma unroll
      for (int m = 0; m < M; ++m) {
        float f[8];
        unpack8((M <= 2 && v == tid) ? xc[m < XC ? m : 0] : ldg16(p.x + (size_t)m * K + v * 8), f);
        const float r = rscale[m];
        uint4 o;
        uint32_t* op = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          __nv_bfloat162 pr = __floats2bfloat162_rn((f[2 * j] * r) * wf[2 * j], (f[2 * j + 1] * r) * wf[2 * j + 1]);
          op[j] = *reinterpret_cast<uint32_t*>(&pr);
        }
        *reinterpret_cast<uint4*>(xs + (size_t)m * K + v * 8) = o;
      }
    }
  } else {
    for (int v = tid; v < M * kvec; v += kLinThreads) {
      const int m = v / kvec, c = v - m * kvec;
      *reinterpret_cast<uint4*>(xs + (size_t)m * K + c * 8) = ldg16(p.x + (size_t)m * K + c * 8);
    }
  }
  // The residual of this thread's first output, loaded now so that the
  // epilogue does not wait for it (written by an earlier kernel: after the wait).
  float res0 = 0.f;
  if (EPI == EPI_RESIDUAL && tid < M * P) {
    const int m = tid / P, t = tid - m * P;
    res0 = bf16_to_f(p.residual[(size_t)m * p.N + u0 + t]);
  }
  __syncthreads();

  if (tr && tid == 0) tr[2] = global_timer_ns();
  // ---- main loop: stream this CTA's weight rows ----
  const int gpr = (K + kGranule - 1) / kGranule;  // granules per row
  const int total = R * gpr;
  const int g_begin = (int)(((int64_t)total * warp) / kLinWarps);
  const int g_end = (int)(((int64_t)total * (warp + 1)) / kLinWarps);
  const int half_rows = p.N / 2;
  const int t_first = g_begin / gpr;
  int g = g_begin;
  while (g < g_end) {
    const int t = g / gpr;                    // local row
    const int kg0 = g - t * gpr;
    const int seg = min(g_end, (t + 1) * gpr) - g;
    int row;
    if (RPU == 2) row = (t < P) ? (u0 + t) : (u0 + (t - P) + half_rows);
    else row = u0 + t;
    const __nv_bfloat16* wrow = p.w + (size_t)row * K;
    float a[M];
#pragma unroll
    for (int m = 0; m < M; ++m) a[m] = 0.f;
    for (int kk = 0; kk < seg; kk += U) {
      uint4 wv[U];
      bool ok[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int k = (kg0 + kk + u) * kGranule + lane * 8;
        ok[u] = (kk + u < seg) && (k < K);
        wv[u] = ok[u] ? ldg_stream(wrow + k) : make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        if (ok[u]) {
          const int k = (kg0 + kk + u) * kGranule + lane * 8;
#pragma unroll
          for (int m = 0; m < M; ++m) {
            const uint4 xv = *reinterpret_cast<const uint4*>(xs + (size_t)m * K + k);
            a[m] = dot8(wv[u], xv, a[m]);
          }
        }
      }
    }
#pragma unroll
    for (int m = 0; m < M; ++m) {
      const float s = warp_sum(a[m]);
      if (lane == 0) segbuf[((size_t)warp * ms + (t - t_first)) * M + m] = s;
    }
    g += seg;
  }
  __syncthreads();

  if (tr && tid == 0) tr[3] = global_timer_ns();
  // Sum of local row t for activation row m over the warps that cover it, in
  // warp order.  Warp w streams granules [gb(w), gb(w + 1)) of the CTA's flat
  // granule list, so the covering warps follow from arithmetic: the first is
  // the last warp starting at or before the row's first granule, and usually
  // one or two warps contribute.  Reading shared memory only for those keeps
  // the epilogue's memory instructions few: each one queues behind the
  // sibling CTA's weight loads in the SM's memory-instruction queue (measured
  // at gate_up: ~2.4 us for a single store while the sibling streams).
  auto gb = [&](int w) -> int { return (int)(((int64_t)total * w) / kLinWarps); };
  auto row_sum = [&](int m, int t) -> float {
    float s = 0.f;
    const int g0 = t * gpr, g1 = g0 + gpr;
    int w = (int)(((int64_t)kLinWarps * (g0 + 1) + total - 1) / total) - 1;
    for (w = w < 0 ? 0 : w; w < kLinWarps; ++w) {
      const int wb = gb(w), we = gb(w + 1);
      if (wb >= g1) break;
      if (wb < we && we > g0) s += segbuf[((size_t)w * ms + (t - wb / gpr)) * M + m];
    }
    return s;
  };
  // ---- epilogue ----
  if (EPI == EPI_STORE_F32) {  // unrounded fp32 partial (tensor-parallel row-split linears)
    for (int i = tid; i < M * P; i += kLinThreads) {
      const int m = i / P, t = i - m * P;
      reinterpret_cast<float*>(p.out)[(size_t)m * p.N + u0 + t] = row_sum(m, t);
    }
  } else if (EPI == EPI_AR_RESIDUAL) {
    // Fused one-shot all-reduce of the row-split partials (see ls_linear_allreduce_residual).
    // Every fp32 partial travels to every rank together with this CTA's call
    // number in one 8-byte store; a reader polls its own elements until the
    // call number matches, so no fence, flag or barrier sits between the push
    // and the sum.
    const P2PExchange& ex = p.ex;
    unsigned char* mine = ex.peer[ex.rank];
    const uint32_t epoch = s_epoch;  // this CTA's call number, read in the prologue
    unsigned long long* trace = ex.trace ? ex.trace + (size_t)blockIdx.x * 4 : nullptr;
    if (trace && tid == 0) trace[0] = global_timer_ns();
    const size_t slot_base = (size_t)(epoch & 1u) * LS_MAX_TP_RANKS * ex.max_rows * ex.width;
    const size_t recv_off = p2p_recv_offset(ex.max_ctas);
    for (int i = tid; i < M * P; i += kLinThreads) {
      const int m = i / P, t = i - m * P;
      const float v = row_sum(m, t);
      const size_t off = slot_base + ((size_t)ex.rank * ex.max_rows + m) * ex.width + u0 + t;
      for (int q = 0; q < ex.world; ++q)
        st_pair_sys(reinterpret_cast<uint2*>(ex.peer[q] + recv_off) + off, __float_as_uint(v), epoch);
    }
    if (trace && tid == 0) trace[1] = global_timer_ns();
    const uint2* recv = reinterpret_cast<const uint2*>(mine + recv_off) + slot_base;
    // One wait limit for the whole CTA: once any element gives up, every
    // thread skips its remaining waits (sticky abort), so a vanished peer costs
    // one limit, not one per element.
    __shared__ int s_ar_abort;
    if (tid == 0) s_ar_abort = 0;
    __syncthreads();
    const WaitClock clk(p.err);
    for (int i = tid; i < M * P; i += kLinThreads) {
      const int m = i / P, t = i - m * P;
      float y = 0.f;
      for (int q = 0; q < ex.world; ++q) {
        const uint2* src = recv + ((size_t)q * ex.max_rows + m) * ex.width + u0 + t;
        uint2 v = ld_pair_sys(src);
        while (v.y != epoch) {
          if (*reinterpret_cast<volatile int*>(&s_ar_abort)) break;
          if (clk.expired()) {
            raise_device_error(p.err, LS_ERR_TIMEOUT | (0x30 << 8));
            s_ar_abort = 1;
            break;
          }
          v = ld_pair_sys(src);
        }
        y += __uint_as_float(v.x);
      }
      const size_t o = (size_t)m * p.N + u0 + t;
      p.out[o] = f_to_bf16(bf16_to_f(p.residual[o]) + round_bf16(y));
    }
    if (trace && tid == 0) {
      trace[2] = global_timer_ns();
      trace[3] = trace[2];
    }
  } else if (EPI == EPI_STORE || EPI == EPI_RESIDUAL) {
    for (int i = tid; i < M * P; i += kLinThreads) {
      const int m = i / P, t = i - m * P;
      const size_t o = (size_t)m * p.N + u0 + t;
      float y = row_sum(m, t);
      if (EPI == EPI_RESIDUAL) y = (i == tid ? res0 : bf16_to_f(p.residual[o])) + round_bf16(y);
      p.out[o] = f_to_bf16(y);
    }
  } else if (EPI == EPI_SILU_MUL) {
    for (int i = tid; i < M * P; i += kLinThreads) {
      const int m = i / P, t = i - m * P;
      const float gt = round_bf16(row_sum(m, t));
      const float up = round_bf16(row_sum(m, P + t));
      const float act = round_bf16(gt / (1.0f + expf(-gt)));
      p.out[(size_t)m * half_rows + u0 + t] = f_to_bf16(act * up);
    }
  } else {  // EPI_ARGMAX: per activation row, best bf16 logit, lowest index on ties
    __shared__ float bv[kLinWarps];
    __shared__ int bi[kLinWarps];
    __shared__ bool is_last;
    for (int m = 0; m < M; ++m) {
      float best = -INFINITY;
      int besti = 0x7fffffff;
      for (int t = tid; t < P; t += kLinThreads) {
        const float v = round_bf16(row_sum(m, t));
        const int idx = u0 + t;
        if (v > best || (v == best && idx < besti)) { best = v; besti = idx; }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, best, o);
        const int oi = __shfl_xor_sync(0xffffffffu, besti, o);
        if (ov > best || (ov == best && oi < besti)) { best = ov; besti = oi; }
      }
      if (lane == 0) { bv[warp] = best; bi[warp] = besti; }
      __syncthreads();
      if (tid == 0) {
        for (int w = 1; w < kLinWarps; ++w)
          if (bv[w] > best || (bv[w] == best && bi[w] < besti)) { best = bv[w]; besti = bi[w]; }
        p.part_val[(size_t)m * G + blockIdx.x] = best;
        p.part_idx[(size_t)m * G + blockIdx.x] = besti;
      }
      __syncthreads();
    }
    if (tid == 0) {
      __threadfence();
      const unsigned int prev = atomicAdd(p.counter, 1u);
      is_last = (prev == (unsigned int)G - 1);
    }
    __syncthreads();
    if (is_last) {
      __threadfence();
      for (int m = 0; m < M; ++m) {
        float best = -INFINITY;
        int besti = 0x7fffffff;
        for (int c = tid; c < G; c += kLinThreads) {
          const float v = __ldcg(p.part_val + (size_t)m * G + c);
          const int idx = __ldcg(p.part_idx + (size_t)m * G + c);
          if (v > best || (v == best && idx < besti)) { best = v; besti = idx; }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
          const float ov = __shfl_xor_sync(0xffffffffu, best, o);
          const int oi = __shfl_xor_sync(0xffffffffu, besti, o);
          if (ov > best || (ov == best && oi < besti)) { best = ov; besti = oi; }
        }
        if (lane == 0) { bv[warp] = best; bi[warp] = besti; }
        __syncthreads();
        if (tid == 0) {
          for (int w = 1; w < kLinWarps; ++w)
            if (bv[w] > best || (bv[w] == best && bi[w] < besti)) { best = bv[w]; besti = bi[w]; }
          const int64_t id = (int64_t)besti + p.id_offset;
          p.out_ids[m] = p.out_keys ? argmax_key(best, id) : id;
        }
        __syncthreads();
      }
      if (tid == 0) *p.counter = 0u;
    }
  }
  if (tr) {
    __syncthreads();
    if (tid == 0) tr[4] = global_timer_ns();
  }
}

}  // namespace lsb

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
namespace lsb_host {

using namespace lsb;

// Two 512-thread CTAs per SM: 32 warps with 8 loads of 512 B in flight each
// keep ~128 KB per SM in flight, what the measured 6 TB/s needs (one CTA per
// SM reached only 4.5 TB/s on the lm_head).  m > 4 needs more registers and
// runs one CTA per SM.
#ifdef LEANB200_PROFILING
// Profiling hook (ls_linear_set_trace): when set, every launch records per CTA
// (start, after the PDL wait, after the prologue, after the main loop, end).
static unsigned long long* g_lin_trace = nullptr;
#endif

static int linear_grid(int units, int m) {
  const int g = (m <= 4 ? 2 : 1) * sm_count();
  return units < g ? units : g;
}

static int linear_max_segs(int K, int rpu, int max_local) {
  const int gpr = (K + kGranule - 1) / kGranule;
  const int total = max_local * rpu * gpr;
  const int range = (total + kLinWarps - 1) / kLinWarps;
  return range / gpr + 2;
}

static size_t linear_smem(int M, int K, int max_segs) {
  const size_t k_pad = (size_t)((K + 7) & ~7);
  return ((size_t)M * k_pad * 2 + 15) / 16 * 16 + (size_t)kLinWarps * max_segs * M * sizeof(float);
}

template <int M, int EPI, bool NORM>
static int launch_linear_t(LinearParams p, int grid, size_t smem, cudaStream_t stream) {
  auto kern = linear_small_m_kernel<M, EPI, NORM>;
  // Raise the dynamic shared-memory limit once per device (not inside every
  // launch, so captured steps contain launches only).
  static int configured[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (smem > 48 * 1024 && dev >= 0 && dev < 64 && (int)smem > configured[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return set_error(LS_ERR_CUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
    configured[dev] = (int)smem;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kLinThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, p);
  if (e != cudaSuccess) return set_error(LS_ERR_CUDA, "linear launch: %s", cudaGetErrorString(e));
  return LS_OK;
}

template <int EPI, bool NORM>
static int dispatch_m(int M, LinearParams p, int grid, size_t smem, cudaStream_t s) {
  switch (M) {
    case 1: return launch_linear_t<1, EPI, NORM>(p, grid, smem, s);
    case 2: return launch_linear_t<2, EPI, NORM>(p, grid, smem, s);
    case 3: return launch_linear_t<3, EPI, NORM>(p, grid, smem, s);
    case 4: return launch_linear_t<4, EPI, NORM>(p, grid, smem, s);
    case 5: return launch_linear_t<5, EPI, NORM>(p, grid, smem, s);
    case 6: return launch_linear_t<6, EPI, NORM>(p, grid, smem, s);
    case 7: return launch_linear_t<7, EPI, NORM>(p, grid, smem, s);
    case 8: return launch_linear_t<8, EPI, NORM>(p, grid, smem, s);
    default: return set_error(LS_ERR_UNSUPPORTED_SHAPE, "linear: m=%d outside 1..8", M);
  }
}

static int launch_linear_impl(const void* x, int64_t m, int64_t k, const void* norm_w, float eps, const void* w,
                              int64_t n, int epi, const void* residual, void* out, cudaStream_t stream,
                              float* part_val, int* part_idx, unsigned int* counter, int64_t* out_ids,
                              int grid_override, int64_t id_offset, bool out_keys,
                              const P2PExchange* ex = nullptr) {
  if (!x || !w || (epi != EPI_ARGMAX && !out)) return set_error(LS_ERR_INVALID_ARGUMENT, "linear: null pointer");
  if (m < 1 || m > 8) return set_error(LS_ERR_UNSUPPORTED_SHAPE, "linear: m=%lld outside 1..8", (long long)m);
  if (k < 8 || n < 1 || k > 32768 || n > (int64_t)1 << 30)
    return set_error(LS_ERR_UNSUPPORTED_SHAPE, "linear: k=%lld n=%lld", (long long)k, (long long)n);
  if (k % 8) return set_error(LS_ERR_MISALIGNED, "linear: k=%lld not a multiple of 8", (long long)k);
  if (!aligned16(x) || !aligned16(w) || (norm_w && !aligned16(norm_w)))
    return set_error(LS_ERR_MISALIGNED, "linear: x/w/norm_w must be 16-byte aligned");
  if ((epi == EPI_RESIDUAL || epi == EPI_AR_RESIDUAL) && !residual)
    return set_error(LS_ERR_INVALID_ARGUMENT, "linear: residual is null");
  if (epi == EPI_AR_RESIDUAL && (!ex || norm_w)) return set_error(LS_ERR_INVALID_ARGUMENT, "linear: bad all-reduce call");
  if (epi == EPI_SILU_MUL && (n % 2)) return set_error(LS_ERR_UNSUPPORTED_SHAPE, "linear: gate_up rows odd");
  LinearParams p = {};
  p.x = static_cast<const __nv_bfloat16*>(x);
  p.norm_w = static_cast<const __nv_bfloat16*>(norm_w);
  p.w = static_cast<const __nv_bfloat16*>(w);
  p.residual = static_cast<const __nv_bfloat16*>(residual);
  p.out = static_cast<__nv_bfloat16*>(out);
  p.eps = eps;
  p.K = (int)k;
  p.N = (int)n;
  p.units = (epi == EPI_SILU_MUL) ? (int)(n / 2) : (int)n;
  const int grid = grid_override > 0 ? grid_override : linear_grid(p.units, (int)m);
  p.max_local_units = (p.units + grid - 1) / grid;
  const int rpu = (epi == EPI_SILU_MUL) ? 2 : 1;
  p.max_segs = linear_max_segs((int)k, rpu, p.max_local_units);
  p.part_val = part_val;
  p.part_idx = part_idx;
  p.counter = counter;
  p.out_ids = out_ids;
  p.id_offset = id_offset;
  p.out_keys = out_keys ? 1 : 0;
  p.err = device_error_ptr();
#ifdef LEANB200_PROFILING
  p.trace = g_lin_trace;
#endif
  if (epi == EPI_AR_RESIDUAL) {
    p.ex = *ex;
    const int g_ar = grid_override > 0 ? grid_override : linear_grid(p.units, (int)m);
    if (g_ar > ex->max_ctas || m > ex->max_rows || n != ex->width)
      return set_error(LS_ERR_UNSUPPORTED_SHAPE, "linear all-reduce: grid %d / m %lld / n %lld beyond the exchange "
                       "region (%d CTAs, %d rows, width %d)", g_ar, (long long)m, (long long)n, ex->max_ctas,
                       ex->max_rows, ex->width);
  }
  const size_t smem = linear_smem((int)m, (int)k, p.max_segs);
  if (smem > 200 * 1024)
    return set_error(LS_ERR_UNSUPPORTED_SHAPE, "linear: m=%lld k=%lld needs %zu B of shared memory", (long long)m,
                     (long long)k, smem);
  const bool norm = norm_w != nullptr;
  switch (epi) {
    case EPI_STORE: return norm ? dispatch_m<EPI_STORE, true>((int)m, p, grid, smem, stream)
                                : dispatch_m<EPI_STORE, false>((int)m, p, grid, smem, stream);
    case EPI_RESIDUAL: return norm ? dispatch_m<EPI_RESIDUAL, true>((int)m, p, grid, smem, stream)
                                   : dispatch_m<EPI_RESIDUAL, false>((int)m, p, grid, smem, stream);
    case EPI_SILU_MUL: return norm ? dispatch_m<EPI_SILU_MUL, true>((int)m, p, grid, smem, stream)
                                   : dispatch_m<EPI_SILU_MUL, false>((int)m, p, grid, smem, stream);
    case EPI_ARGMAX: return norm ? dispatch_m<EPI_ARGMAX, true>((int)m, p, grid, smem, stream)
                                 : dispatch_m<EPI_ARGMAX, false>((int)m, p, grid, smem, stream);
    case EPI_STORE_F32: return norm ? dispatch_m<EPI_STORE_F32, true>((int)m, p, grid, smem, stream)
                                    : dispatch_m<EPI_STORE_F32, false>((int)m, p, grid, smem, stream);
    case EPI_AR_RESIDUAL: return dispatch_m<EPI_AR_RESIDUAL, false>((int)m, p, grid, smem, stream);
    default: return set_error(LS_ERR_INVALID_ARGUMENT, "linear: unknown epilogue %d", epi);
  }
}

int launch_linear(const void* x, int64_t m, int64_t k, const void* norm_w, float eps, const void* w, int64_t n,
                  int epi, const void* residual, void* out, cudaStream_t stream, float* part_val, int* part_idx,
                  unsigned int* counter, int64_t* out_ids, int grid_override) {
  return launch_linear_impl(x, m, k, norm_w, eps, w, n, epi, residual, out, stream, part_val, part_idx, counter,
                            out_ids, grid_override, 0, false);
}

// Greedy head over one vocab shard: out_keys[m] = argmax_key(best logit, shard row + vocab_offset).
int launch_lmhead_keys(const void* h, int64_t m, int64_t k, const void* norm_w, float eps, const void* w,
                       int64_t rows, int64_t vocab_offset, int64_t* out_keys, cudaStream_t stream, float* part_val,
                       int* part_idx, unsigned int* counter, int grid) {
  return launch_linear_impl(h, m, k, norm_w, eps, w, rows, EPI_ARGMAX, nullptr, nullptr, stream, part_val, part_idx,
                            counter, out_keys, grid, vocab_offset, true);
}

int launch_linear_allreduce(const void* x, int64_t m, int64_t k, const void* w, int64_t n, const void* residual,
                            void* out, const P2PExchange* ex, cudaStream_t stream) {
  return launch_linear_impl(x, m, k, nullptr, 0.f, w, n, EPI_AR_RESIDUAL, residual, out, stream, nullptr, nullptr,
                            nullptr, nullptr, 0, 0, false, ex);
}

int lmhead_grid(int64_t vocab, int64_t m) { return linear_grid((int)vocab, (int)m); }

}  // namespace lsb_host

#ifdef LEANB200_PROFILING
extern "C" int ls_linear_set_trace(void* buffer) {
  lsb_host::g_lin_trace = static_cast<unsigned long long*>(buffer);
  return LS_OK;
}
#endif
