// Skinny-M linears (1 <= m <= 8) on the tensor cores over pre-tiled weights.
//
// Weight layout ("gemv tiles", written once by ls_gemv_tile_weight):
//   unit u = 8 consecutive output rows (for the SiLU epilogue: 8 gate rows and
//   the 8 matching up rows, gate half first); each half is K/32 tiles of
//   8 rows x 32 k = 512 bytes, and within a tile lane l (g = l/4, t = l%4)
//   holds the 16 bytes
//     W[8u+g][32j+2t, +1], W[8u+g][32j+2t+8, +9], W[8u+g][32j+16+2t, +1], W[8u+g][32j+16+2t+8, +9]
//   -- exactly the B fragments of two mma.m16n8k16 k-steps.  Tiles are stored
//   unit-major, so the whole matrix is one sequence of 512-byte tiles.
//
// Kernel: the tile sequence is cut into equal contiguous ranges, one per CTA
// and within it one per warp (perfect balance, every warp streams one
// contiguous stretch of memory with 16-byte loads, 8 in flight per lane).
// Per tile a warp issues one LDG.128 per lane and two MMAs whose A operand is
// the activation rows (M <= 8 of the 16 MMA rows) kept in shared memory in
// fragment order.  Per (unit, half) a warp keeps one fp32 C fragment; partials
// are summed over warps in warp order, and a unit split between CTAs is
// finished by the last CTA to arrive, which adds the CTAs' partials in CTA
// order: the result does not depend on timing.
//
// Epilogues as in the reference's decode path (qwen_explicit.py:913-949,
// :1247-1272): STORE, RESIDUAL (bf16(res + bf16(y))), SILU_MUL
// (bf16(bf16(silu(bf16 g)) * bf16 u)); optional RMSNorm prologue.
#include "common.cuh"

namespace lsb {

constexpr int kGvThreads = 512;
constexpr int kGvWarps = kGvThreads / 32;
constexpr int kGvUnroll = 8;
constexpr int kGvMaxSegs = 8;   // (unit, half) segments one warp may touch, beyond which the shape is rejected
constexpr int kGvMaxUnits = 16; // units one CTA may touch
enum { GV_STORE = 0, GV_RESIDUAL = 1, GV_SILU = 2 };

struct GemvParams {
  const __nv_bfloat16* x;         // [M, K]
  const __nv_bfloat16* norm_w;    // [K] or null
  const uint4* w;                 // tiled weights
  const __nv_bfloat16* residual;  // [M, N]
  __nv_bfloat16* out;             // [M, N] (N = output rows)
  float* part;                    // [G][2][RPU][M][8] partials of CTA-boundary units
  unsigned int* counter;          // [units], zero between calls (after a fixed-size partials region,
                                  // so calls of any shape can share one workspace)
  float eps;
  int K, N, units, kp;            // kp = K / 32 (tiles per half)
  int tiles;                      // units * RPU * kp (< 2^31)
};

__device__ __forceinline__ void gv_mma(float (&d)[4], uint32_t a0, uint32_t a2, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(0u), "r"(a2), "r"(0u), "r"(b0), "r"(b1));
}

__device__ __forceinline__ int gv_cta_begin(int tiles, int c, int G) { return (int)((long long)tiles * c / G); }

// CTA whose tile range contains tile x.
__device__ __forceinline__ int gv_cta_of(int tiles, int x, int G) {
  int c = (int)(((long long)x * G) / tiles);
  while (c + 1 < G && gv_cta_begin(tiles, c + 1, G) <= x) ++c;
  while (c > 0 && gv_cta_begin(tiles, c, G) > x) --c;
  return c;
}

template <int M, int EPI, bool NORM>
__global__ void __launch_bounds__(kGvThreads, 2) gemv_mma_kernel(GemvParams p) {
  constexpr int RPU = (EPI == GV_SILU) ? 2 : 1;
  extern __shared__ __align__(16) unsigned char gv_smem[];
  uint4* xf = reinterpret_cast<uint4*>(gv_smem);                          // [kp][M][4] fragment order
  float* segbuf = reinterpret_cast<float*>(gv_smem + (size_t)p.kp * M * 4 * 16);  // [warps][kGvMaxSegs][M][8]
  __shared__ float red[kGvWarps][M];
  __shared__ float rscale[M];
  __shared__ int s_last[2], s_lo[2], s_hi[2];
  __shared__ int s_wf[kGvWarps], s_wl[kGvWarps];             // first / last segment of each warp
  __shared__ float ysum[kGvMaxUnits * (EPI == GV_SILU ? 2 : 1) * M * 8];

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g8 = lane >> 2, t4 = lane & 3;
  const int G = gridDim.x;
  const int c_begin = gv_cta_begin(p.tiles, blockIdx.x, G), c_end = gv_cta_begin(p.tiles, blockIdx.x + 1, G);
  const int w_begin = c_begin + (c_end - c_begin) * warp / kGvWarps;
  const int w_end = c_begin + (c_end - c_begin) * (warp + 1) / kGvWarps;
  if (lane == 0) {
    s_wf[warp] = w_end > w_begin ? w_begin / p.kp : 1;  // empty range: first > last
    s_wl[warp] = w_end > w_begin ? (w_end - 1) / p.kp : 0;
  }

  // Start this warp's first weight tiles toward L2 before waiting on the previous kernel.
  if (lane == 0 && w_end > w_begin) {
    const int n = min(w_end - w_begin, 32);
    prefetch_l2(p.w + (size_t)w_begin * 32, (uint32_t)(n * 512));
  }
  grid_dep_launch();
  grid_dep_wait();

  // ---- activations into shared memory in A-fragment order (optional RMSNorm) ----
  const int K = p.K;
  if (NORM) {
    float ss[M];
#pragma unroll
    for (int m = 0; m < M; ++m) ss[m] = 0.f;
    for (int v = tid; v < (K >> 3); v += kGvThreads) {
#pragma unroll
      for (int m = 0; m < M; ++m) {
        float f[8];
        unpack8(ldg16(p.x + (size_t)m * K + v * 8), f);
#pragma unroll
        for (int j = 0; j < 8; ++j) ss[m] = fmaf(f[j], f[j], ss[m]);
      }
    }
#pragma unroll
    for (int m = 0; m < M; ++m) {
      const float s = warp_sum(ss[m]);
      if (lane == 0) red[warp][m] = s;
    }
    __syncthreads();
    if (tid < M) {
      float s = 0.f;
      for (int w = 0; w < kGvWarps; ++w) s += red[w][tid];
      rscale[tid] = rsqrtf(s / (float)K + p.eps);
    }
    __syncthreads();
  }
  for (int i = tid; i < p.kp * M * 4; i += kGvThreads) {
    const int tt = i & 3, m = (i >> 2) % M, j = (i >> 2) / M;
    const int kb = 32 * j + 2 * tt;
    const int ks[4] = {kb, kb + 8, kb + 16, kb + 24};
    uint32_t v[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const __nv_bfloat162 raw = *reinterpret_cast<const __nv_bfloat162*>(p.x + (size_t)m * K + ks[q]);
      if (NORM) {
        const __nv_bfloat162 wv = *reinterpret_cast<const __nv_bfloat162*>(p.norm_w + ks[q]);
        const float r = rscale[m];
        const __nv_bfloat162 o = __floats2bfloat162_rn((__low2float(raw) * r) * __low2float(wv),
                                                       (__high2float(raw) * r) * __high2float(wv));
        v[q] = *reinterpret_cast<const uint32_t*>(&o);
      } else {
        v[q] = *reinterpret_cast<const uint32_t*>(&raw);
      }
    }
    xf[i] = make_uint4(v[0], v[1], v[2], v[3]);
  }
  __syncthreads();

  // ---- main loop: this warp's tiles, one (unit, half) segment at a time ----
  const int kp = p.kp;
  const int seg_first = w_begin / kp;
  int tt = w_begin;
  while (tt < w_end) {
    const int seg = tt / kp;
    const int s_end = min(w_end, (seg + 1) * kp);
    const uint4* wseg = p.w + (size_t)seg * kp * 32 + lane;  // tile j of this segment: wseg[j * 32]
    const uint4* xseg = xf + g8 * 4 + t4;                      // k-pair j: xseg[j * M * 4]
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    for (int j0 = tt - seg * kp; j0 < s_end - seg * kp; j0 += kGvUnroll) {
      const int jn = s_end - seg * kp - j0;  // tiles left in this segment
      uint4 b[kGvUnroll];
#pragma unroll
      for (int u = 0; u < kGvUnroll; ++u)
        b[u] = (u < jn) ? ldg_stream(reinterpret_cast<const __nv_bfloat16*>(wseg + (size_t)(j0 + u) * 32))
                        : make_uint4(0, 0, 0, 0);
#pragma unroll
      for (int u = 0; u < kGvUnroll; ++u) {
        if (u < jn) {
          const int j = j0 + u;
          uint4 a = make_uint4(0, 0, 0, 0);
          if (g8 < M) a = xseg[j * M * 4];
          gv_mma(acc, a.x, a.y, b[u].x, b[u].y);
          gv_mma(acc, a.z, a.w, b[u].z, b[u].w);
        }
      }
    }
    const int ls = (int)(seg - seg_first);
    if (g8 < M && ls < kGvMaxSegs) {
      float* d = segbuf + (((size_t)warp * kGvMaxSegs + ls) * M + g8) * 8 + 2 * t4;
      d[0] = acc[0];
      d[1] = acc[1];
    }
    tt = s_end;
  }
  __syncthreads();

  // ---- CTA reduction over warps (warp order), per (unit, half, m, row) ----
  const int cseg0 = c_begin / kp, cseg1 = (c_end - 1) / kp;  // segments this CTA touches
  const int cu0 = cseg0 / RPU, cu1 = cseg1 / RPU;             // units this CTA touches
  const int nu = cu1 - cu0 + 1;                               // <= kGvMaxUnits (checked on the host)
  const int unit_tiles = RPU * kp;
  {
    // ysum[unit - cu0][half][m][n]: the CTA's sum of warp partials, in warp order.
    const int total = nu * RPU * M * 8;
    for (int i = tid; i < total; i += kGvThreads) {
      const int n = i & 7, m = (i >> 3) % M, uh = (i >> 3) / M;  // uh = (unit - cu0) * RPU + half
      const int seg = cu0 * RPU + uh;
      float acc = 0.f;
      if (seg >= cseg0 && seg <= cseg1) {
#pragma unroll 1
        for (int w = 0; w < kGvWarps; ++w) {
          const int f = s_wf[w], l = s_wl[w];
          if (seg >= f && seg <= l) acc += segbuf[(((size_t)w * kGvMaxSegs + (seg - f)) * M + m) * 8 + n];
        }
      }
      ysum[i] = acc;
    }
  }
  __syncthreads();
  auto epilogue = [&](int u, int m, int n, float y0, float y1) {
    const size_t o = (size_t)m * p.N + (size_t)u * 8 + n;
    if (EPI == GV_STORE) {
      p.out[o] = f_to_bf16(y0);
    } else if (EPI == GV_RESIDUAL) {
      p.out[o] = f_to_bf16(bf16_to_f(p.residual[o]) + round_bf16(y0));
    } else {
      const float gt = round_bf16(y0), up = round_bf16(y1);
      p.out[o] = f_to_bf16(round_bf16(gt / (1.0f + expf(-gt))) * up);
    }
  };
  auto whole = [&](int u) { return u * unit_tiles >= c_begin && (u + 1) * unit_tiles <= c_end; };
  // Units inside this CTA's range: finish directly.  Units at either end that
  // are shared with a neighbour: publish this CTA's partial (slot 0 for the
  // first unit, 1 for the last).
  for (int i = tid; i < nu * M * 8; i += kGvThreads) {
    const int n = i & 7, m = (i >> 3) % M, ul = (i >> 3) / M, u = cu0 + ul;
    const float y0 = ysum[((ul * RPU) * M + m) * 8 + n];
    const float y1 = RPU == 2 ? ysum[((ul * RPU + 1) * M + m) * 8 + n] : 0.f;
    if (whole(u)) {
      epilogue(u, m, n, y0, y1);
    } else {
      const int slot = (u == cu0) ? 0 : 1;
      float* dst = p.part + (((size_t)blockIdx.x * 2 + slot) * RPU * M + m) * 8 + n;
      dst[0] = y0;
      if (RPU == 2) dst[M * 8] = y1;
    }
  }
  const bool shared0 = !whole(cu0), shared1 = (nu > 1) && !whole(cu1);
  if (!shared0 && !shared1) return;
  __threadfence();
  __syncthreads();
  if (tid < 2) {
    const bool sh = tid == 0 ? shared0 : shared1;
    int last = 0;
    if (sh) {
      const int u = tid == 0 ? cu0 : cu1;
      const int c_lo = gv_cta_of(p.tiles, u * unit_tiles, G);
      const int c_hi = gv_cta_of(p.tiles, (u + 1) * unit_tiles - 1, G);
      last = atomicAdd(p.counter + u, 1u) == (unsigned int)(c_hi - c_lo) ? 1 : 0;
      if (last) {
        s_lo[tid] = c_lo;
        s_hi[tid] = c_hi;
      }
    }
    s_last[tid] = last;
  }
  __syncthreads();
  for (int e = 0; e < 2; ++e) {
    if (!s_last[e]) continue;  // uniform across the CTA
    __threadfence();
    const int u = e == 0 ? cu0 : cu1;
    for (int i = tid; i < M * 8; i += kGvThreads) {  // every CTA sharing unit u has published: sum in CTA order
      const int m = i >> 3, n = i & 7;
      float y0 = 0.f, y1 = 0.f;
      for (int c = s_lo[e]; c <= s_hi[e]; ++c) {
        const int sl = (gv_cta_begin(p.tiles, c, G) / unit_tiles == u) ? 0 : 1;  // u is c's first or last unit
        const float* src = p.part + (((size_t)c * 2 + sl) * RPU * M + m) * 8 + n;
        y0 += __ldcg(src);
        if (RPU == 2) y1 += __ldcg(src + M * 8);
      }
      epilogue(u, m, n, y0, y1);
    }
    if (tid == 0) p.counter[u] = 0u;
  }
}

// Pre-tiling: W [N, K] row-major bf16 -> gemv tiles (see the layout above).
// silu: rows [0, N/2) are gate rows and [N/2, N) the matching up rows.
__global__ void gemv_tile_kernel(const __nv_bfloat16* w, int N, int K, int silu, uint4* out) {
  const int kp = K / 32;
  const int rpu = silu ? 2 : 1;
  const long long tiles = (long long)(N / 8) * kp;  // == units * rpu * kp
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < tiles * 32;
       i += (long long)gridDim.x * blockDim.x) {
    const long long tile = i >> 5;
    const int lane = (int)(i & 31), g = lane >> 2, t = lane & 3;
    const long long seg = tile / kp;
    const int j = (int)(tile - seg * kp);
    const long long unit = seg / rpu;
    const int half = (int)(seg - unit * rpu);
    const long long row = half ? (N / 2 + unit * 8 + g) : (unit * 8 + g);
    const __nv_bfloat16* r = w + row * K + 32 * j + 2 * t;
    uint32_t v[4];
    const int off[4] = {0, 8, 16, 24};
#pragma unroll
    for (int q = 0; q < 4; ++q) v[q] = *reinterpret_cast<const uint32_t*>(r + off[q]);
    out[i] = make_uint4(v[0], v[1], v[2], v[3]);
  }
}

}  // namespace lsb

namespace lsb_host {
using namespace lsb;

static size_t gv_smem_bytes(int M, int K) {
  return (size_t)(K / 32) * M * 4 * 16 + (size_t)kGvWarps * kGvMaxSegs * M * 8 * 4;
}

template <int M, int EPI, bool NORM>
static int launch_gv(const GemvParams& p, int grid, size_t smem, cudaStream_t stream) {
  static bool attr_done = false;
  if (!attr_done) {
    cudaError_t e =
        cudaFuncSetAttribute(gemv_mma_kernel<M, EPI, NORM>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    if (e != cudaSuccess) return set_error(LS_ERR_CUDA, "gemv_mma attribute: %s", cudaGetErrorString(e));
    attr_done = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kGvThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  cudaError_t e = cudaLaunchKernelEx(&cfg, gemv_mma_kernel<M, EPI, NORM>, p);
  return e == cudaSuccess ? LS_OK : set_error(LS_ERR_CUDA, "gemv_mma launch: %s", cudaGetErrorString(e));
}

template <int EPI, bool NORM>
static int gv_dispatch(int M, const GemvParams& p, int grid, size_t smem, cudaStream_t s) {
  switch (M) {
    case 1: return launch_gv<1, EPI, NORM>(p, grid, smem, s);
    case 2: return launch_gv<2, EPI, NORM>(p, grid, smem, s);
    case 3: return launch_gv<3, EPI, NORM>(p, grid, smem, s);
    case 4: return launch_gv<4, EPI, NORM>(p, grid, smem, s);
    case 5: return launch_gv<5, EPI, NORM>(p, grid, smem, s);
    case 6: return launch_gv<6, EPI, NORM>(p, grid, smem, s);
    case 7: return launch_gv<7, EPI, NORM>(p, grid, smem, s);
    case 8: return launch_gv<8, EPI, NORM>(p, grid, smem, s);
    default: return set_error(LS_ERR_UNSUPPORTED_SHAPE, "gemv_mma: m=%d outside 1..8", M);
  }
}

static int gv_grid() { return 2 * sm_count(); }

// Partials region sized for the largest call (m 8, two halves), then the counters.
static int64_t gv_part_bytes() { return ((int64_t)gv_grid() * 2 * 2 * 8 * 8 * 4 + 255) / 256 * 256; }

int gemv_workspace_bytes(int64_t m, int64_t n_rows, int epi, int64_t* bytes) {
  (void)m;
  const int rpu = epi == GV_SILU ? 2 : 1;
  const int64_t units = n_rows / (8 * rpu);
  *bytes = gv_part_bytes() + units * 4;
  return LS_OK;
}

int launch_gemv_mma(const void* x, int64_t m, int64_t k, const void* norm_w, float eps, const void* w_tiled,
                    int64_t n_rows, int epi, const void* residual, void* out, void* workspace,
                    int64_t workspace_bytes, cudaStream_t stream) {
  if (!x || !w_tiled || !out || !workspace) return set_error(LS_ERR_INVALID_ARGUMENT, "gemv_mma: null pointer");
  if (m < 1 || m > 8) return set_error(LS_ERR_UNSUPPORTED_SHAPE, "gemv_mma: m=%lld outside 1..8", (long long)m);
  if (epi < GV_STORE || epi > GV_SILU) return set_error(LS_ERR_INVALID_ARGUMENT, "gemv_mma: epilogue %d", epi);
  const int rpu = epi == GV_SILU ? 2 : 1;
  if (k < 32 || k % 32 || k > 16384 || n_rows % (8 * rpu) || n_rows < 8 * rpu || n_rows > (1 << 30))
    return set_error(LS_ERR_UNSUPPORTED_SHAPE, "gemv_mma: k=%lld (multiple of 32, <= 16384), n=%lld (multiple of %d)",
                     (long long)k, (long long)n_rows, 8 * rpu);
  if (epi == GV_RESIDUAL && !residual) return set_error(LS_ERR_INVALID_ARGUMENT, "gemv_mma: residual is null");
  if (!aligned16(w_tiled) || !aligned16(x)) return set_error(LS_ERR_MISALIGNED, "gemv_mma: x / weights not aligned");
  int64_t need = 0;
  gemv_workspace_bytes(m, n_rows, epi, &need);
  if (workspace_bytes < need)
    return set_error(LS_ERR_WORKSPACE, "gemv_mma: workspace needs %lld bytes", (long long)need);
  GemvParams p = {};
  p.x = static_cast<const __nv_bfloat16*>(x);
  p.norm_w = static_cast<const __nv_bfloat16*>(norm_w);
  p.w = static_cast<const uint4*>(w_tiled);
  p.residual = static_cast<const __nv_bfloat16*>(residual);
  p.out = static_cast<__nv_bfloat16*>(out);
  p.eps = eps;
  p.K = (int)k;
  p.N = (int)(n_rows / rpu);
  p.units = (int)(n_rows / (8 * rpu));
  p.kp = (int)(k / 32);
  const long long tiles = (long long)p.units * rpu * p.kp;
  const int grid = gv_grid();
  if (tiles >= (1ll << 31) || tiles < grid)
    return set_error(LS_ERR_UNSUPPORTED_SHAPE, "gemv_mma: %lld tiles outside [%d, 2^31)", tiles, grid);
  p.tiles = (int)tiles;
  // Each warp may touch at most kGvMaxSegs (unit, half) segments.
  const long long per_warp = (p.tiles / grid + 1) / kGvWarps + 1;
  const long long per_cta = p.tiles / grid + 1;
  if (per_warp / p.kp + 2 > kGvMaxSegs || per_cta / (rpu * p.kp) + 2 > kGvMaxUnits)
    return set_error(LS_ERR_UNSUPPORTED_SHAPE, "gemv_mma: k=%lld too short for %lld rows", (long long)k,
                     (long long)n_rows);
  p.part = static_cast<float*>(workspace);
  p.counter = reinterpret_cast<unsigned int*>(static_cast<char*>(workspace) + gv_part_bytes());
  const size_t smem = gv_smem_bytes((int)m, (int)k);
  if (smem > 200 * 1024) return set_error(LS_ERR_UNSUPPORTED_SHAPE, "gemv_mma: %zu B of shared memory", smem);
  const bool norm = norm_w != nullptr;
  switch (epi) {
    case GV_STORE: return norm ? gv_dispatch<GV_STORE, true>((int)m, p, grid, smem, stream)
                               : gv_dispatch<GV_STORE, false>((int)m, p, grid, smem, stream);
    case GV_RESIDUAL: return norm ? gv_dispatch<GV_RESIDUAL, true>((int)m, p, grid, smem, stream)
                                  : gv_dispatch<GV_RESIDUAL, false>((int)m, p, grid, smem, stream);
    default: return norm ? gv_dispatch<GV_SILU, true>((int)m, p, grid, smem, stream)
                         : gv_dispatch<GV_SILU, false>((int)m, p, grid, smem, stream);
  }
}

int launch_gemv_tile(const void* w, int64_t n, int64_t k, int silu, void* out, cudaStream_t stream) {
  if (!w || !out) return set_error(LS_ERR_INVALID_ARGUMENT, "gemv_tile: null pointer");
  if (k % 32 || n % (silu ? 16 : 8) || k <= 0 || n <= 0)
    return set_error(LS_ERR_UNSUPPORTED_SHAPE, "gemv_tile: n=%lld k=%lld", (long long)n, (long long)k);
  if (!aligned16(out)) return set_error(LS_ERR_MISALIGNED, "gemv_tile: output not aligned");
  gemv_tile_kernel<<<4 * sm_count(), 256, 0, stream>>>(static_cast<const __nv_bfloat16*>(w), (int)n, (int)k,
                                                        silu, static_cast<uint4*>(out));
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? LS_OK : set_error(LS_ERR_CUDA, "gemv_tile launch: %s", cudaGetErrorString(e));
}

}  // namespace lsb_host

using namespace lsb_host;

extern "C" {

int ls_gemv_tile_weight(const void* w, int64_t n_rows, int64_t k, int silu, void* out, ls_stream_t stream) {
  return launch_gemv_tile(w, n_rows, k, silu, out, (cudaStream_t)stream);
}

int ls_gemv_workspace_bytes(int64_t m, int64_t n_rows, int epilogue, int64_t* bytes) {
  if (!bytes || m < 1 || m > 8 || n_rows < 1 || epilogue < 0 || epilogue > 2)
    return set_error(LS_ERR_INVALID_ARGUMENT, "ls_gemv_workspace_bytes: bad arguments");
  return gemv_workspace_bytes(m, n_rows, epilogue, bytes);
}

int ls_gemv_bf16(const void* x, int64_t m, int64_t k, const void* norm_w, float eps, const void* w_tiled,
                 int64_t n_rows, int epilogue, const void* residual, void* out, void* workspace,
                 int64_t workspace_bytes, ls_stream_t stream) {
  return launch_gemv_mma(x, m, k, norm_w, eps, w_tiled, n_rows, epilogue, residual, out, workspace, workspace_bytes,
                         (cudaStream_t)stream);
}

}  // extern "C"
