// Weight-streaming linear layers for m <= 4 activation rows, fed by bulk TMA.
//
// y[m, n] = sum_k W[n, k] * x[m, k] is HBM-bound at decode batch sizes: every
// weight byte is used m times.  This kernel keeps the DRAM pipe full with
// bulk copies instead of per-thread loads:
//   * one CTA per SM owns a balanced, contiguous range of output units (a row,
//     or a gate/up row pair for the SiLU epilogue);
//   * a producer warp streams whole weight rows into a ring of shared-memory
//     stages with cp.async.bulk (completion tracked by mbarriers), so ~100 KB
//     per SM is in flight with almost no registers;
//   * under programmatic dependent launch the producer fills the ring BEFORE
//     the kernel waits for its predecessor: weights never depend on the
//     previous kernel, only the activations do;
//   * eight consumer warps dot each stage against the (optionally
//     RMS-normalised) activations held in shared memory; per-row partial sums
//     are combined over warps in a fixed order, so results are deterministic;
//   * the epilogues apply the reference's bf16 rounding points (see
//     linear_small_m.cu) and the argmax epilogue ends with a last-CTA
//     reduction across the grid.
#include "common.cuh"

namespace lsb {

constexpr int kStreamWarps = 8;                         // consumer warps
constexpr int kStreamConsumers = kStreamWarps * 32;
constexpr int kStreamThreads = kStreamConsumers + 32;   // + one producer warp
constexpr int kStreamGranule = 256;                     // bf16 per warp-wide 512-byte read
constexpr int kStreamMaxStages = 8;

enum { SEPI_STORE = 0, SEPI_RESIDUAL = 1, SEPI_SILU_MUL = 2, SEPI_ARGMAX = 3 };

struct StreamParams {
  const __nv_bfloat16* x;
  const __nv_bfloat16* norm_w;
  const __nv_bfloat16* w;
  const __nv_bfloat16* residual;
  __nv_bfloat16* out;
  float eps;
  int K, N, units;
  int rows_per_chunk;  // whole weight rows per stage
  int stages;
  int stage_bytes;     // rows_per_chunk * K * 2 rounded up to 128
  int max_segs;        // row segments one warp can touch in one chunk
  float* part_val;
  int* part_idx;
  unsigned int* counter;
  int64_t* out_ids;
  int* err;
};

__host__ __device__ inline size_t stream_align(size_t v, size_t a) { return (v + a - 1) / a * a; }

template <int M, int EPI, bool NORM>
__global__ void __launch_bounds__(kStreamThreads, 1) linear_stream_kernel(StreamParams p) {
  constexpr int RPU = (EPI == SEPI_SILU_MUL) ? 2 : 1;
  extern __shared__ __align__(128) unsigned char smem[];
  const int K = p.K, RC = p.rows_per_chunk, NS = p.stages, MS = p.max_segs;
  unsigned char* stage_base = smem;
  __nv_bfloat16* xs = reinterpret_cast<__nv_bfloat16*>(smem + (size_t)NS * p.stage_bytes);
  float* segbuf = reinterpret_cast<float*>(reinterpret_cast<unsigned char*>(xs) + stream_align((size_t)M * K * 2, 16));
  float* gbuf = segbuf + 2 * kStreamWarps * MS * M;
  uint64_t* full = reinterpret_cast<uint64_t*>(stream_align(reinterpret_cast<size_t>(gbuf + RC * M), 8));
  uint64_t* empty = full + NS;
  __shared__ float red[kStreamWarps][M];
  __shared__ float rscale[M];
  __shared__ float bv[kStreamWarps];
  __shared__ int bi[kStreamWarps];
  __shared__ int aborted;
  __shared__ bool is_last;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int G = gridDim.x;
  const int u0 = (int)(((int64_t)p.units * blockIdx.x) / G);
  const int u1 = (int)(((int64_t)p.units * (blockIdx.x + 1)) / G);
  const int P = u1 - u0;
  const int blocks = (P + RC - 1) / RC;
  const int n_chunks = blocks * RPU;
  const int half_rows = p.N / 2;

  if (tid == 0) {
    for (int s = 0; s < NS; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    aborted = 0;
    mbar_fence_init();
  }
  __syncthreads();
  grid_dep_launch();

  // ---------------- producer: stream whole weight rows into the ring ----------------
  if (warp == kStreamWarps) {
    if (lane == 0) {
      for (int c = 0; c < n_chunks; ++c) {
        const int s = c % NS;
        if (c >= NS && !mbar_wait(&empty[s], ((c / NS) - 1) & 1, p.err)) break;
        if (*(volatile int*)&aborted) break;
        const int j = c / RPU, half = c - j * RPU;
        const int r_begin = u0 + j * RC;
        const int nrows = min(u1, r_begin + RC) - r_begin;
        const uint32_t bytes = (uint32_t)nrows * K * 2;
        mbar_arrive_expect_tx(&full[s], bytes);
        bulk_g2s(stage_base + (size_t)s * p.stage_bytes, p.w + (size_t)(r_begin + half * half_rows) * K, bytes,
                 &full[s]);
      }
    }
    return;
  }

  // ---------------- consumers ----------------
  grid_dep_wait();  // activations come from the previous kernel
  const int kvec = K >> 3;
  if (NORM) {
    float ss[M];
#pragma unroll
    for (int m = 0; m < M; ++m) ss[m] = 0.f;
    for (int v = tid; v < kvec; v += kStreamConsumers) {
#pragma unroll
      for (int m = 0; m < M; ++m) {
        float f[8];
        unpack8(ldg16(p.x + (size_t)m * K + v * 8), f);
#pragma unroll
        for (int q = 0; q < 8; ++q) ss[m] = fmaf(f[q], f[q], ss[m]);
      }
    }
#pragma unroll
    for (int m = 0; m < M; ++m) {
      const float t = warp_sum(ss[m]);
      if (lane == 0) red[warp][m] = t;
    }
    named_bar_sync(1, kStreamConsumers);
    if (tid < M) {
      float t = 0.f;
      for (int w = 0; w < kStreamWarps; ++w) t += red[w][tid];
      rscale[tid] = rsqrtf(t / (float)K + p.eps);
    }
    named_bar_sync(1, kStreamConsumers);
    for (int v = tid; v < kvec; v += kStreamConsumers) {
      float wf[8];
      unpack8(ldg16(p.norm_w + v * 8), wf);
#pragma unroll
      for (int m = 0; m < M; ++m) {
        float f[8];
        unpack8(ldg16(p.x + (size_t)m * K + v * 8), f);
        const float r = rscale[m];
        uint4 o;
        uint32_t* op = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          __nv_bfloat162 pr = __floats2bfloat162_rn((f[2 * q] * r) * wf[2 * q], (f[2 * q + 1] * r) * wf[2 * q + 1]);
          op[q] = *reinterpret_cast<uint32_t*>(&pr);
        }
        *reinterpret_cast<uint4*>(xs + (size_t)m * K + v * 8) = o;
      }
    }
  } else {
    for (int v = tid; v < M * kvec; v += kStreamConsumers) {
      const int m = v / kvec, q = v - m * kvec;
      *reinterpret_cast<uint4*>(xs + (size_t)m * K + q * 8) = ldg16(p.x + (size_t)m * K + q * 8);
    }
  }
  named_bar_sync(1, kStreamConsumers);

  const int gpr = (K + kStreamGranule - 1) / kStreamGranule;
  float best_v[M];
  int best_i[M];
#pragma unroll
  for (int m = 0; m < M; ++m) {
    best_v[m] = -INFINITY;
    best_i[m] = 0x7fffffff;
  }

  for (int c = 0; c < n_chunks; ++c) {
    const int s = c % NS;
    const int j = c / RPU, half = c - j * RPU;
    const int r_begin = u0 + j * RC;
    const int nrows = min(u1, r_begin + RC) - r_begin;
    // A timed-out wait marks the CTA aborted; every consumer still reaches the
    // named barrier below, then all of them leave together.
    const bool have = mbar_wait(&full[s], (c / NS) & 1, p.err);
    if (!have) aborted = 1;
    const __nv_bfloat16* wst = reinterpret_cast<const __nv_bfloat16*>(stage_base + (size_t)s * p.stage_bytes);
    float* sb = segbuf + (c & 1) * kStreamWarps * MS * M;
    const int total = nrows * gpr;
    const int g_begin = (int)(((int64_t)total * warp) / kStreamWarps);
    const int g_end = (int)(((int64_t)total * (warp + 1)) / kStreamWarps);
    const int t_first = g_begin / gpr;
    int g = have ? g_begin : g_end;
    while (g < g_end) {
      const int t = g / gpr;
      const int kg0 = g - t * gpr;
      const int seg = min(g_end, (t + 1) * gpr) - g;
      float a[M];
#pragma unroll
      for (int m = 0; m < M; ++m) a[m] = 0.f;
      const __nv_bfloat16* wrow = wst + (size_t)t * K;
#pragma unroll 2
      for (int kk = 0; kk < seg; ++kk) {
        const int k = (kg0 + kk) * kStreamGranule + lane * 8;
        if (k < K) {
          const uint4 wv = *reinterpret_cast<const uint4*>(wrow + k);
#pragma unroll
          for (int m = 0; m < M; ++m) a[m] = dot8(wv, *reinterpret_cast<const uint4*>(xs + (size_t)m * K + k), a[m]);
        }
      }
#pragma unroll
      for (int m = 0; m < M; ++m) {
        const float v = warp_sum(a[m]);
        if (lane == 0) sb[((size_t)warp * MS + (t - t_first)) * M + m] = v;
      }
      g += seg;
    }
    named_bar_sync(1, kStreamConsumers);
    if (*(volatile int*)&aborted) break;
    if (tid == 0) mbar_arrive(&empty[s]);  // the stage may be refilled

    for (int i = tid; i < M * nrows; i += kStreamConsumers) {
      const int m = i / nrows, t = i - m * nrows;
      const int lo = t * gpr, hi = lo + gpr;
      float y = 0.f;
      for (int w = 0; w < kStreamWarps; ++w) {
        const int wb = (int)(((int64_t)total * w) / kStreamWarps);
        const int we = (int)(((int64_t)total * (w + 1)) / kStreamWarps);
        if (wb < we && wb < hi && we > lo) y += sb[((size_t)w * MS + (t - wb / gpr)) * M + m];
      }
      const int u = r_begin + t;
      if (EPI == SEPI_STORE) {
        p.out[(size_t)m * p.N + u] = f_to_bf16(y);
      } else if (EPI == SEPI_RESIDUAL) {
        const size_t o = (size_t)m * p.N + u;
        p.out[o] = f_to_bf16(bf16_to_f(p.residual[o]) + round_bf16(y));
      } else if (EPI == SEPI_SILU_MUL) {
        if (half == 0) {
          gbuf[t * M + m] = round_bf16(y);
        } else {
          const float gt = gbuf[t * M + m];
          const float act = round_bf16(gt / (1.0f + expf(-gt)));
          p.out[(size_t)m * half_rows + u] = f_to_bf16(act * round_bf16(y));
        }
      } else {  // argmax over bf16 logits, lowest index on ties
        const float v = round_bf16(y);
#pragma unroll
        for (int mm = 0; mm < M; ++mm) {
          if (mm == m && (v > best_v[mm] || (v == best_v[mm] && u < best_i[mm]))) {
            best_v[mm] = v;
            best_i[mm] = u;
          }
        }
      }
    }
  }

  if (EPI == SEPI_ARGMAX) {
    for (int m = 0; m < M; ++m) {
      float best = best_v[m];
      int besti = best_i[m];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, best, o);
        const int oi = __shfl_xor_sync(0xffffffffu, besti, o);
        if (ov > best || (ov == best && oi < besti)) { best = ov; besti = oi; }
      }
      if (lane == 0) { bv[warp] = best; bi[warp] = besti; }
      named_bar_sync(1, kStreamConsumers);
      if (tid == 0) {
        for (int w = 1; w < kStreamWarps; ++w)
          if (bv[w] > best || (bv[w] == best && bi[w] < besti)) { best = bv[w]; besti = bi[w]; }
        p.part_val[(size_t)m * G + blockIdx.x] = best;
        p.part_idx[(size_t)m * G + blockIdx.x] = besti;
      }
      named_bar_sync(1, kStreamConsumers);
    }
    if (tid == 0) {
      __threadfence();
      const unsigned int prev = atomicAdd(p.counter, 1u);
      is_last = (prev == (unsigned int)G - 1);
    }
    named_bar_sync(1, kStreamConsumers);
    if (is_last) {
      __threadfence();
      for (int m = 0; m < M; ++m) {
        float best = -INFINITY;
        int besti = 0x7fffffff;
        for (int c = tid; c < G; c += kStreamConsumers) {
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
        named_bar_sync(1, kStreamConsumers);
        if (tid == 0) {
          for (int w = 1; w < kStreamWarps; ++w)
            if (bv[w] > best || (bv[w] == best && bi[w] < besti)) { best = bv[w]; besti = bi[w]; }
          p.out_ids[m] = (int64_t)besti;
        }
        named_bar_sync(1, kStreamConsumers);
      }
      if (tid == 0) *p.counter = 0u;
    }
  }
}

}  // namespace lsb

namespace lsb_host {
using namespace lsb;

struct StreamPlan {
  int grid, rows_per_chunk, stages, stage_bytes, max_segs;
  size_t smem;
  bool ok;
};

static StreamPlan stream_plan(int M, int K, int N, int epi) {
  StreamPlan pl = {};
  const int rpu = (epi == SEPI_SILU_MUL) ? 2 : 1;
  const int units = (epi == SEPI_SILU_MUL) ? N / 2 : N;
  const int g = sm_count();
  pl.grid = units < g ? units : g;
  const int row_bytes = K * 2;
  pl.rows_per_chunk = row_bytes >= 32768 ? 1 : 32768 / row_bytes;
  const int max_local = (units + pl.grid - 1) / pl.grid;
  if (pl.rows_per_chunk > max_local) pl.rows_per_chunk = max_local;
  pl.stage_bytes = (int)stream_align((size_t)pl.rows_per_chunk * row_bytes, 128);
  int stages = (96 * 1024) / pl.stage_bytes;
  if (stages > kStreamMaxStages) stages = kStreamMaxStages;
  if (stages < 2) stages = 2;
  pl.stages = stages;
  const int gpr = (K + kStreamGranule - 1) / kStreamGranule;
  const int total = pl.rows_per_chunk * gpr;
  const int range = (total + kStreamWarps - 1) / kStreamWarps;
  pl.max_segs = range / gpr + 2;
  pl.smem = (size_t)pl.stages * pl.stage_bytes + stream_align((size_t)M * K * 2, 16) +
            (size_t)2 * kStreamWarps * pl.max_segs * M * 4 + (size_t)pl.rows_per_chunk * M * 4 + 8 +
            (size_t)2 * pl.stages * 8;
  pl.ok = row_bytes <= 65536 && pl.smem <= 200 * 1024 && rpu >= 1;
  return pl;
}

bool stream_supported(int64_t m, int64_t k, int64_t n, int epi) {
  if (m < 1 || m > 4 || k % 8 || k > 32768) return false;
  return stream_plan((int)m, (int)k, (int)n, epi).ok;
}

int stream_grid(int64_t m, int64_t k, int64_t n, int epi) { return stream_plan((int)m, (int)k, (int)n, epi).grid; }

template <int M, int EPI, bool NORM>
static int launch_stream_t(const StreamParams& p, const StreamPlan& pl, cudaStream_t stream) {
  auto kern = linear_stream_kernel<M, EPI, NORM>;
  static int configured[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && (int)pl.smem > configured[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)pl.smem);
    if (e != cudaSuccess) return set_error(LS_ERR_CUDA, "cudaFuncSetAttribute(stream): %s", cudaGetErrorString(e));
    configured[dev] = (int)pl.smem;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(pl.grid);
  cfg.blockDim = dim3(kStreamThreads);
  cfg.dynamicSmemBytes = pl.smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, p);
  if (e != cudaSuccess) return set_error(LS_ERR_CUDA, "linear_stream launch: %s", cudaGetErrorString(e));
  return LS_OK;
}

template <int EPI, bool NORM>
static int stream_dispatch_m(int M, const StreamParams& p, const StreamPlan& pl, cudaStream_t s) {
  switch (M) {
    case 1: return launch_stream_t<1, EPI, NORM>(p, pl, s);
    case 2: return launch_stream_t<2, EPI, NORM>(p, pl, s);
    case 3: return launch_stream_t<3, EPI, NORM>(p, pl, s);
    case 4: return launch_stream_t<4, EPI, NORM>(p, pl, s);
    default: return set_error(LS_ERR_UNSUPPORTED_SHAPE, "linear_stream: m=%d", M);
  }
}

int launch_linear_stream(const void* x, int64_t m, int64_t k, const void* norm_w, float eps, const void* w, int64_t n,
                         int epi, const void* residual, void* out, cudaStream_t stream, float* part_val,
                         int* part_idx, unsigned int* counter, int64_t* out_ids) {
  const StreamPlan pl = stream_plan((int)m, (int)k, (int)n, epi);
  if (!pl.ok) return set_error(LS_ERR_UNSUPPORTED_SHAPE, "linear_stream: plan does not fit (m=%lld k=%lld)",
                               (long long)m, (long long)k);
  StreamParams p = {};
  p.x = static_cast<const __nv_bfloat16*>(x);
  p.norm_w = static_cast<const __nv_bfloat16*>(norm_w);
  p.w = static_cast<const __nv_bfloat16*>(w);
  p.residual = static_cast<const __nv_bfloat16*>(residual);
  p.out = static_cast<__nv_bfloat16*>(out);
  p.eps = eps;
  p.K = (int)k;
  p.N = (int)n;
  p.units = (epi == SEPI_SILU_MUL) ? (int)(n / 2) : (int)n;
  p.rows_per_chunk = pl.rows_per_chunk;
  p.stages = pl.stages;
  p.stage_bytes = pl.stage_bytes;
  p.max_segs = pl.max_segs;
  p.part_val = part_val;
  p.part_idx = part_idx;
  p.counter = counter;
  p.out_ids = out_ids;
  p.err = device_error_ptr();
  const bool norm = norm_w != nullptr;
  switch (epi) {
    case SEPI_STORE: return norm ? stream_dispatch_m<SEPI_STORE, true>((int)m, p, pl, stream)
                                 : stream_dispatch_m<SEPI_STORE, false>((int)m, p, pl, stream);
    case SEPI_RESIDUAL: return norm ? stream_dispatch_m<SEPI_RESIDUAL, true>((int)m, p, pl, stream)
                                    : stream_dispatch_m<SEPI_RESIDUAL, false>((int)m, p, pl, stream);
    case SEPI_SILU_MUL: return norm ? stream_dispatch_m<SEPI_SILU_MUL, true>((int)m, p, pl, stream)
                                    : stream_dispatch_m<SEPI_SILU_MUL, false>((int)m, p, pl, stream);
    case SEPI_ARGMAX: return norm ? stream_dispatch_m<SEPI_ARGMAX, true>((int)m, p, pl, stream)
                                  : stream_dispatch_m<SEPI_ARGMAX, false>((int)m, p, pl, stream);
    default: return set_error(LS_ERR_INVALID_ARGUMENT, "linear_stream: unknown epilogue %d", epi);
  }
}

}  // namespace lsb_host
