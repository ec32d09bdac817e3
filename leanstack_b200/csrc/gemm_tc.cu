// Weight-streaming GEMM on the 5th-generation tensor cores (tcgen05 + TMEM + TMA).
//
// Y[b, n] = sum_k X[b, k] * W[n, k] for the decode / verify shapes: few
// activation rows (b < 256) against large weight matrices that are read once.
// The product is computed transposed ("swap AB"): the weight tile is the MMA's
// A operand (128 rows = MMA M), the activations are the B operand (MMA N = the
// batch rounded up to 16), and the fp32 accumulator D[n, b] lives in TMEM with
// one TMEM lane per weight row.
//
// Work split ("stream-K"): the (128-row tile, 64-wide k-block) units of the
// whole matrix are divided evenly over one CTA per SM, so every SM streams the
// same number of weight bytes whatever the shape.  A tile whose k-blocks are
// split between CTAs is finished by its last contributor, which sums the fp32
// partials of all contributors in CTA order (deterministic).  The split-partial
// epilogue (SPLIT_F32, below) skips that reduction: with fewer tiles than SMs
// its grid is tile-aligned on two CTAs per SM (each with a ring cut to fit
// beside the other), with more it is one whole-K CTA per tile, and the next
// kernel adds the partials.
//
// Warp roles (6 warps): warp 4 issues TMA loads of weight and activation
// k-blocks into a shared-memory ring (128-byte swizzle, the canonical K-major
// UMMA layout); warp 5 issues tcgen05.mma (one elected thread) and commits
// stage releases and accumulator completion to mbarriers; warps 0-3 drain TMEM
// with tcgen05.ld and run the epilogue.  Under programmatic dependent launch
// the producer loads the first weight stages before waiting on the previous
// kernel (weights never depend on it; activations do).
//
// Epilogues follow the reference's bf16 rounding points
// (src/leanstack/runtime/qwen_explicit.py:809-852, :913, :932-949): STORE
// rounds the fp32 sum once; RESIDUAL adds the rounded product to the residual
// and rounds again; SILU_MUL pairs gate tile t with up tile t (two TMEM
// accumulators) and rounds after the projection, after SiLU and after the
// product.  Every mbarrier wait is bounded (LS_ERR_TIMEOUT).
// The file also holds the large-M prefill GEMM (gemm_big_kernel) and the causal
// prefill attention on tcgen05 (prefill_attention_tc_kernel), which share the
// TMA, UMMA-descriptor and TMEM helpers below.
#include <cuda.h>

#include "common.cuh"

namespace lsb {

constexpr int kTcTileN = 128;   // weight rows per tile (MMA M)
constexpr int kTcBlockK = 64;   // K per stage: one 128-byte swizzle atom of bf16
constexpr int kTcThreads = 192;
constexpr int kTcEpiThreads = 128;
constexpr int kTcMaxStages = 16;
// Tile counters sit in a fixed-size region at the start of the workspace, so
// one workspace can serve GEMMs of different shapes: partials of one call never
// land on another call's counters.
constexpr int kTcMaxTiles = 2048;
constexpr size_t kTcCounterBytes = (size_t)2 * kTcMaxTiles * sizeof(unsigned int);

// TEPI_SPLIT_F32: no reduction in the kernel.  The grid is tile-aligned (every
// CTA holds the k-range of exactly one tile) and CTA j of a tile's splits
// writes its unrounded fp32 sum to out[j][b][n]; the consumer kernel adds the
// splits in order j = 0, 1, ... and applies the epilogue itself (bit-identical
// to the in-kernel reduction of the same split count).
enum { TEPI_STORE = 0, TEPI_RESIDUAL = 1, TEPI_SILU_MUL = 2, TEPI_STORE_F32 = 4, TEPI_SPLIT_F32 = 8 };

struct TcParams {
  const __nv_bfloat16* residual;  // [B, N]
  __nv_bfloat16* out;             // [B, N]
  float* partial;                 // [grid][2 slots][accs][BN][128]
  unsigned int* counters;         // [2][tiles]: arrivals, departures; zero between calls
  int* err;
  int B;          // activation rows
  int BN;         // MMA N (B rounded up to 16)
  int N;          // output columns
  int tiles;      // ceil(N / 128)
  int kblocks;    // ceil(K / 64)
  int stages;
  int stage_bytes;
  int acc_buffers;  // 2: the MMA fills one TMEM accumulator while the epilogue drains the other
  uint32_t tmem_cols;
  // Pre-tiled weights (ls_gemm_tc_tile_weight): tile (t, kb) is the 16 KB
  // shared-memory image at w_tiled[(t * kblocks + kb) * 16 KB]; null: TMA maps.
  const unsigned char* w_tiled;
  const unsigned char* w2_tiled;
  unsigned long long* trace;  // optional profiling: per CTA 8 globaltimer stamps
  int aligned;  // N % 8 == 0 and out / residual 16-byte aligned: vector stores, bulk residual rows
};

__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t saddr) {
  // K-major, 128-byte swizzle: 8-row groups 1024 B apart (SBO), LBO unused,
  // descriptor version 1, layout type 2 (SWIZZLE_128B).
  return (uint64_t)((saddr >> 4) & 0x3FFF) | (1ull << 16) | (64ull << 32) | (1ull << 46) | (2ull << 61);
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void umma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(
          tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate));
}

__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float v[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// First unit of CTA c and the CTA that owns unit u (units split evenly).
__device__ __forceinline__ long long tc_unit_begin(long long U, int G, int c) { return U * c / G; }
__device__ __forceinline__ int tc_unit_owner(long long U, int G, long long u) {
  return (int)(((u + 1) * G + U - 1) / U - 1);
}

// Spin (bounded) until a global counter reaches `target`.
__device__ __forceinline__ bool wait_counter(const unsigned int* ctr, unsigned int target, int* err, int site) {
  const WaitClock clk(err);
  while (true) {
    unsigned int v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(ctr) : "memory");
    if (v >= target) return true;
    if (clk.expired()) {
      raise_device_error(err, 7 /* LS_ERR_TIMEOUT */ | (site << 8));
      return false;
    }
    __nanosleep(64);
  }
}

template <int EPI>
__device__ __forceinline__ float tc_apply(const TcParams& p, size_t o, float y, float y2) {
  if (EPI == TEPI_STORE || EPI == TEPI_STORE_F32) return y;
  if (EPI == TEPI_RESIDUAL) return bf16_to_f(p.residual[o]) + round_bf16(y);
  const float g = round_bf16(y);
  return round_bf16(g / (1.0f + expf(-g))) * round_bf16(y2);
}

template <int EPI>
__device__ __forceinline__ void tc_store(const TcParams& p, size_t o, float v) {
  if (EPI == TEPI_STORE_F32) reinterpret_cast<float*>(p.out)[o] = v;
  else p.out[o] = f_to_bf16(v);
}

// One contributor's share of a split tile's reduction: output columns
// [b0, b1) x the tile's 128 weight rows, summed over the partials of CTAs
// c_lo..c_hi in CTA order.  Work items are (column, 4-row quad) pairs read as
// float4; the partials of up to kRedC contributors x kRedI items are loaded
// before any is added, so one L2 round trip serves 16 float4 loads per thread.
template <int EPI>
__device__ __forceinline__ void tc_reduce_tile(const TcParams& p, int t, int c_lo, int c_hi, int b0, int b1,
                                               long long U, int G, int KB) {
  constexpr int ACCS = (EPI == TEPI_SILU_MUL) ? 2 : 1;
  constexpr int kRedI = 4 / ACCS;  // items per batch
  constexpr int kRedC = 4;         // contributors per load round
  const int items = (b1 - b0) * (kTcTileN / 4);
  const size_t part_stride = (size_t)ACCS * p.BN * kTcTileN;  // floats per partial slot
  for (int it0 = threadIdx.x; it0 < items; it0 += kTcEpiThreads * kRedI) {
    float4 y[kRedI][ACCS];
#pragma unroll
    for (int i = 0; i < kRedI; ++i)
#pragma unroll
      for (int a = 0; a < ACCS; ++a) y[i][a] = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int c0 = c_lo; c0 <= c_hi; c0 += kRedC) {
      float4 v[kRedC][kRedI][ACCS];
#pragma unroll
      for (int cu = 0; cu < kRedC; ++cu) {
        const int c = c0 + cu;
        if (c > c_hi) break;
        const int sl = (t == (int)(tc_unit_begin(U, G, c) / KB)) ? 0 : 1;
        const float* part = p.partial + ((size_t)c * 2 + sl) * part_stride;
#pragma unroll
        for (int i = 0; i < kRedI; ++i) {
          const int it = it0 + i * kTcEpiThreads;
          if (it < items) {
            const int b = b0 + it / (kTcTileN / 4), row0 = (it % (kTcTileN / 4)) * 4;
#pragma unroll
            for (int a = 0; a < ACCS; ++a)
              v[cu][i][a] = __ldcg(reinterpret_cast<const float4*>(part + ((size_t)a * p.BN + b) * kTcTileN + row0));
          }
        }
      }
#pragma unroll
      for (int cu = 0; cu < kRedC; ++cu) {
        if (c0 + cu > c_hi) break;
#pragma unroll
        for (int i = 0; i < kRedI; ++i)
#pragma unroll
          for (int a = 0; a < ACCS; ++a) {
            y[i][a].x += v[cu][i][a].x;
            y[i][a].y += v[cu][i][a].y;
            y[i][a].z += v[cu][i][a].z;
            y[i][a].w += v[cu][i][a].w;
          }
      }
    }
#pragma unroll
    for (int i = 0; i < kRedI; ++i) {
      const int it = it0 + i * kTcEpiThreads;
      if (it >= items) continue;
      const int b = b0 + it / (kTcTileN / 4);
      const int n0 = t * kTcTileN + (it % (kTcTileN / 4)) * 4;
      const float ya[4] = {y[i][0].x, y[i][0].y, y[i][0].z, y[i][0].w};
      const float yb[4] = {y[i][ACCS - 1].x, y[i][ACCS - 1].y, y[i][ACCS - 1].z, y[i][ACCS - 1].w};
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        if (n0 + q < p.N) {
          const size_t o = (size_t)b * p.N + n0 + q;
          tc_store<EPI>(p, o, tc_apply<EPI>(p, o, ya[q], yb[q]));
        }
      }
    }
  }
}

// Output of one reduced element with the residual value already loaded.
template <int EPI>
__device__ __forceinline__ float tc_apply_r(float y, float y2, float r) {
  if (EPI == TEPI_STORE || EPI == TEPI_STORE_F32) return y;
  if (EPI == TEPI_RESIDUAL) return r + round_bf16(y);
  const float g = round_bf16(y);
  return round_bf16(g / (1.0f + expf(-g))) * round_bf16(y2);
}

__device__ __forceinline__ void red_release_gpu(unsigned int* ctr, unsigned int v) {
  asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(ctr), "r"(v) : "memory");
}

// Deferred stream-K reduction of the (at most two) split tiles this CTA
// contributed to.  Each contributor of a tile owns a slice [b0, b1) of its
// activation columns and sums the fp32 partials of all contributors for that
// slice in CTA order (deterministic).  Shares are taken last tile first: its
// other contributor (the next CTA) wrote its part at the start of its
// mainloop, so it is complete as soon as this CTA's own part is.
//
// The idle stage ring serves as two staging regions.  One thread waits for a
// tile's contributors and pulls their partial columns (and, for RESIDUAL, the
// residual rows) in with bulk async copies; the next job's copies are in
// flight while the 128 epilogue threads sum the current one.  Shapes whose
// jobs do not fit fall back to tc_reduce_tile (direct float4 loads).
constexpr int kTcMaxRedJobs = 16;

template <int EPI>
__device__ __forceinline__ void tc_stream_k_fixup(const TcParams& p, long long U, int G, int KB, long long ub,
                                                  long long ue, int cta, unsigned char* area, size_t area_bytes,
                                                  uint64_t* bars, volatile int* abort,
                                                  unsigned long long* tr) {
  constexpr int ACCS = (EPI == TEPI_SILU_MUL) ? 2 : 1;
  constexpr uint32_t kColBytes = kTcTileN * 4;  // one activation column of one partial
  constexpr uint32_t kResBytes = kTcTileN * 2;  // one residual row segment
  const bool res_bulk = (EPI == TEPI_RESIDUAL) && p.aligned;
  const int tid = threadIdx.x;
  int sh_t[2], sh_lo[2], sh_hi[2], sh_b0[2], sh_b1[2];
  int ns = 0;
  const int t_first = (int)(ub / KB), t_last = (int)((ue - 1) / KB);
  for (int w = 0; w < 2; ++w) {
    const int t = w == 0 ? t_last : t_first;
    if (w == 1 && t_first == t_last) break;
    const long long tile_begin = (long long)t * KB, tile_end = tile_begin + KB;
    const int c_lo = tc_unit_owner(U, G, tile_begin), c_hi = tc_unit_owner(U, G, tile_end - 1);
    const int nc = c_hi - c_lo + 1;
    if (nc == 1) continue;  // a whole tile: written by the epilogue
    const int j = cta - c_lo;
    sh_t[ns] = t;
    sh_lo[ns] = c_lo;
    sh_hi[ns] = c_hi;
    sh_b0[ns] = (int)(((long long)p.B * j) / nc);
    sh_b1[ns] = (int)(((long long)p.B * (j + 1)) / nc);
    ++ns;
  }
  const size_t part_stride = (size_t)ACCS * p.BN * kTcTileN;  // floats per partial slot
  const size_t half = (area_bytes / 2) & ~(size_t)1023;
  // Jobs: (share, first column, columns), in order.
  int jb_s[kTcMaxRedJobs], jb_c0[kTcMaxRedJobs], jb_cn[kTcMaxRedJobs];
  int nj = 0;
  bool staged = true;
  for (int s = 0; s < ns && staged; ++s) {
    const int nc = sh_hi[s] - sh_lo[s] + 1;
    const size_t per_col = (size_t)nc * ACCS * kColBytes + (res_bulk ? kResBytes : 0);
    int chunk = (int)(half / per_col);
    if (chunk < 1) {
      staged = false;
      break;
    }
    for (int c0 = sh_b0[s]; c0 < sh_b1[s]; c0 += chunk) {
      if (nj == kTcMaxRedJobs) {
        staged = false;
        break;
      }
      jb_s[nj] = s;
      jb_c0[nj] = c0;
      jb_cn[nj] = min(chunk, sh_b1[s] - c0);
      ++nj;
    }
  }

  if (!staged) {
    for (int s = 0; s < ns; ++s) {
      const int nc = sh_hi[s] - sh_lo[s] + 1;
      if (sh_b1[s] <= sh_b0[s]) continue;
      if (tid == 0 && !wait_counter(p.counters + sh_t[s], (unsigned int)nc, p.err, 5 + s)) *abort = 1;
      named_bar_sync(1, kTcEpiThreads);
      if (*abort) return;
      tc_reduce_tile<EPI>(p, sh_t[s], sh_lo[s], sh_hi[s], sh_b0[s], sh_b1[s], U, G, KB);
    }
  } else {
    // Thread 0: wait for the job's tile (first job of a share only), then
    // start its copies into region (job & 1).  On a timeout it arrives without
    // copies so that nobody waits on the region's barrier for nothing.
    auto issue = [&](int jj) {
      const int s = jb_s[jj], t = sh_t[s], c_lo = sh_lo[s], c_hi = sh_hi[s], nc = c_hi - c_lo + 1;
      uint64_t* bar = bars + (jj & 1);
      unsigned char* region = area + (size_t)(jj & 1) * half;
      if ((jj == 0 || jb_s[jj - 1] != s) && !*abort) {
        if (!wait_counter(p.counters + t, (unsigned int)nc, p.err, 5 + s)) *abort = 1;
        if (tr) tr[4 + 2 * s] = global_timer_ns();
      }
      if (*abort) {
        mbar_arrive(bar);
        return;
      }
      const int c0 = jb_c0[jj], cn = jb_cn[jj];
      const uint32_t seg_bytes = (uint32_t)cn * kColBytes;
      const int n_first = t * kTcTileN;
      const uint32_t res_row = (uint32_t)min(kTcTileN, p.N - n_first) * 2;
      // Partials were published with generic stores and a release; the
      // acquire above orders them before these bulk (async-proxy) reads, as
      // does the proxy fence for this CTA's generic reads of the region.
      asm volatile("fence.proxy.async.global;" ::: "memory");
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      mbar_arrive_expect_tx(bar, (uint32_t)(nc * ACCS) * seg_bytes + (res_bulk ? (uint32_t)cn * res_row : 0u));
      for (int c = c_lo; c <= c_hi; ++c) {
        const int sl = (t == (int)(tc_unit_begin(U, G, c) / KB)) ? 0 : 1;
        const float* part = p.partial + ((size_t)c * 2 + sl) * part_stride;
        for (int a = 0; a < ACCS; ++a)
          bulk_g2s(region + (size_t)((c - c_lo) * ACCS + a) * seg_bytes, part + ((size_t)a * p.BN + c0) * kTcTileN,
                   seg_bytes, bar);
      }
      if (res_bulk) {
        unsigned char* rdst = region + (size_t)nc * ACCS * seg_bytes;
        for (int bl = 0; bl < cn; ++bl)
          bulk_g2s(rdst + (size_t)bl * kResBytes, p.residual + (size_t)(c0 + bl) * p.N + n_first, res_row, bar);
      }
    };
    if (tid == 0) {
      if (nj > 0) issue(0);
      if (nj > 1) issue(1);
    }
    uint32_t phase[2] = {0u, 0u};
    for (int jj = 0; jj < nj; ++jj) {
      const int r = jj & 1;
      if (!mbar_wait(bars + r, phase[r], p.err, 7)) *abort = 1;
      phase[r] ^= 1u;
      named_bar_sync(1, kTcEpiThreads);
      if (*abort) return;
      const int s = jb_s[jj], t = sh_t[s], nc = sh_hi[s] - sh_lo[s] + 1;
      const int c0 = jb_c0[jj], cn = jb_cn[jj];
      const float* sm = reinterpret_cast<const float*>(area + (size_t)r * half);
      const __nv_bfloat16* smr = reinterpret_cast<const __nv_bfloat16*>(area + (size_t)r * half +
                                                                         (size_t)nc * ACCS * cn * kColBytes);
      const int items = cn * (kTcTileN / 4);
      for (int it = tid; it < items; it += kTcEpiThreads) {
        const int bl = it / (kTcTileN / 4), row0 = (it % (kTcTileN / 4)) * 4;
        float4 y[ACCS];
#pragma unroll
        for (int a = 0; a < ACCS; ++a) y[a] = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int c = 0; c < nc; ++c) {
#pragma unroll
          for (int a = 0; a < ACCS; ++a) {
            const float4 v = *reinterpret_cast<const float4*>(sm + ((size_t)(c * ACCS + a) * cn + bl) * kTcTileN + row0);
            y[a].x += v.x;
            y[a].y += v.y;
            y[a].z += v.z;
            y[a].w += v.w;
          }
        }
        const int b = c0 + bl;
        const int n0 = t * kTcTileN + row0;
        const size_t o = (size_t)b * p.N + n0;
        const float ya[4] = {y[0].x, y[0].y, y[0].z, y[0].w};
        const float yb[4] = {y[ACCS - 1].x, y[ACCS - 1].y, y[ACCS - 1].z, y[ACCS - 1].w};
        float rv[4] = {0.f, 0.f, 0.f, 0.f};
        if (EPI == TEPI_RESIDUAL) {
#pragma unroll
          for (int q = 0; q < 4; ++q)
            if (n0 + q < p.N) rv[q] = bf16_to_f(res_bulk ? smr[bl * kTcTileN + row0 + q] : p.residual[o + q]);
        }
        float ov[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) ov[q] = tc_apply_r<EPI>(ya[q], yb[q], rv[q]);
        if (p.aligned && n0 + 3 < p.N) {
          if (EPI == TEPI_STORE_F32) {
            *reinterpret_cast<float4*>(reinterpret_cast<float*>(p.out) + o) = make_float4(ov[0], ov[1], ov[2], ov[3]);
          } else {
            __nv_bfloat162 lo = __floats2bfloat162_rn(ov[0], ov[1]), hi = __floats2bfloat162_rn(ov[2], ov[3]);
            uint2 pk;
            pk.x = *reinterpret_cast<uint32_t*>(&lo);
            pk.y = *reinterpret_cast<uint32_t*>(&hi);
            *reinterpret_cast<uint2*>(p.out + o) = pk;
          }
        } else {
#pragma unroll
          for (int q = 0; q < 4; ++q)
            if (n0 + q < p.N) tc_store<EPI>(p, o + q, ov[q]);
        }
      }
      named_bar_sync(1, kTcEpiThreads);  // region r is free again
      if (tr && tid == 0 && (jj + 1 == nj || jb_s[jj + 1] != s)) tr[5 + 2 * s] = global_timer_ns();
      if (tid == 0 && jj + 2 < nj) issue(jj + 2);
    }
  }
  // Departures: the last contributor of a tile to leave resets its counters
  // for the next call.  Contributors without columns leave without waiting:
  // some contributor with columns saw every arrival before it left.
  if (tid == 0 && !*abort) {
    unsigned int prev[2] = {0u, 0u};
    for (int s = 0; s < ns; ++s) prev[s] = atomicAdd(p.counters + p.tiles + sh_t[s], 1u);
    for (int s = 0; s < ns; ++s) {
      if (prev[s] == (unsigned int)(sh_hi[s] - sh_lo[s])) {
        p.counters[sh_t[s]] = 0u;
        p.counters[p.tiles + sh_t[s]] = 0u;
      }
    }
  }
}

template <int EPI>
__global__ void __launch_bounds__(kTcThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_w2,
                   const __grid_constant__ CUtensorMap tm_x, TcParams p) {
  constexpr bool SILU = (EPI == TEPI_SILU_MUL);
  constexpr int ACCS = SILU ? 2 : 1;
  constexpr uint32_t kWBytes = kTcTileN * kTcBlockK * 2;  // 16 KB per weight tile
  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<size_t>(smem_raw) + 1023) & ~size_t(1023));
  const int NS = p.stages;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + (size_t)NS * p.stage_bytes);
  uint64_t* empty = full + NS;
  uint64_t* acc_full = empty + NS;   // [2]
  uint64_t* acc_empty = acc_full + 2;  // [2]
  uint64_t* red_bar = acc_empty + 2;    // [2] stream-K reduction copies
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(red_bar + 2);
  __shared__ int s_abort;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = gridDim.x, cta = blockIdx.x;
  const int KB = p.kblocks;
  const long long U = (long long)p.tiles * KB;
  const long long ub = tc_unit_begin(U, G, cta), ue = tc_unit_begin(U, G, cta + 1);
  const uint32_t x_bytes = (uint32_t)p.BN * kTcBlockK * 2;
  const uint32_t idesc = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(p.BN >> 3) << 17) |
                         ((uint32_t)(kTcTileN >> 4) << 24);
  const int nbuf = p.acc_buffers;
  const uint32_t acc_cols = (uint32_t)(p.BN * ACCS);

  if (threadIdx.x == 0) {
    for (int s = 0; s < NS; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], kTcEpiThreads);
    }
    mbar_init(&red_bar[0], 1);
    mbar_init(&red_bar[1], 1);
    s_abort = 0;
    mbar_fence_init();
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(p.tmem_cols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  grid_dep_launch();
  const uint32_t tmem = *tmem_slot;
  unsigned long long* tr = p.trace ? p.trace + (size_t)cta * 8 : nullptr;
  if (tr && threadIdx.x == 0) tr[0] = global_timer_ns();

  if (warp == 4) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      const long long n_units = ue - ub;
      const long long pre = n_units < NS ? n_units : NS;
      // Weights first (independent of the previous kernel), then activations.
      auto load_w = [&](unsigned char* st, int t, int kb, uint64_t* bar) {
        if (p.w_tiled) {
          const size_t off = ((size_t)t * KB + kb) * kWBytes;
          bulk_g2s(st, p.w_tiled + off, kWBytes, bar);
          if (SILU) bulk_g2s(st + kWBytes, p.w2_tiled + off, kWBytes, bar);
        } else {
          tma_load_2d(st, &tm_w, kb * kTcBlockK, t * kTcTileN, bar);
          if (SILU) tma_load_2d(st + kWBytes, &tm_w2, kb * kTcBlockK, t * kTcTileN, bar);
        }
      };
      for (long long i = 0; i < pre; ++i) {
        const long long u = ub + i;
        const int t = (int)(u / KB), kb = (int)(u % KB);
        unsigned char* st = smem + (size_t)i * p.stage_bytes;
        mbar_arrive_expect_tx(&full[i], kWBytes * ACCS + x_bytes);
        load_w(st, t, kb, &full[i]);
      }
      grid_dep_wait();
      for (long long i = 0; i < pre; ++i) {
        const long long u = ub + i;
        const int kb = (int)(u % KB);
        tma_load_2d(smem + (size_t)i * p.stage_bytes + kWBytes * ACCS, &tm_x, kb * kTcBlockK, 0, &full[i]);
      }
      for (long long i = pre; i < n_units; ++i) {
        const int s = (int)(i % NS);
        if (!mbar_wait(&empty[s], (uint32_t)((i / NS) - 1) & 1u, p.err, 1)) {
          s_abort = 1;
          break;
        }
        const long long u = ub + i;
        const int t = (int)(u / KB), kb = (int)(u % KB);
        unsigned char* st = smem + (size_t)s * p.stage_bytes;
        mbar_arrive_expect_tx(&full[s], kWBytes * ACCS + x_bytes);
        load_w(st, t, kb, &full[s]);
        tma_load_2d(st + kWBytes * ACCS, &tm_x, kb * kTcBlockK, 0, &full[s]);
      }
    }
  } else if (warp == 5) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      long long i = 0;
      int seg = 0;
      long long u = ub;
      while (u < ue && !*(volatile int*)&s_abort) {
        const long long tile_end = (u / KB + 1) * KB;
        const long long seg_end = ue < tile_end ? ue : tile_end;
        const int a = seg % nbuf;
        if (seg >= nbuf && !mbar_wait(&acc_empty[a], (uint32_t)((seg / nbuf) - 1) & 1u, p.err, 2)) {
          s_abort = 1;
          break;
        }
        tc_fence_after();
        const uint32_t acc_tmem = tmem + (uint32_t)a * acc_cols;
        for (long long v = u; v < seg_end; ++v, ++i) {
          const int s = (int)(i % NS);
          if (!mbar_wait(&full[s], (uint32_t)(i / NS) & 1u, p.err, 3)) {
            s_abort = 1;
            break;
          }
          if (tr && i == 0) tr[1] = global_timer_ns();
          tc_fence_after();
          const uint32_t sw = smem_u32(smem + (size_t)s * p.stage_bytes);
          const uint32_t sx = sw + kWBytes * ACCS;
#pragma unroll
          for (int kk = 0; kk < kTcBlockK / 16; ++kk) {
            const uint32_t acc = (v != u || kk > 0) ? 1u : 0u;
            const uint64_t bdesc = umma_desc_sw128(sx + kk * 32);
            umma_f16(acc_tmem, umma_desc_sw128(sw + kk * 32), bdesc, idesc, acc);
            if (SILU)
              umma_f16(acc_tmem + (uint32_t)p.BN, umma_desc_sw128(sw + kWBytes + kk * 32), bdesc, idesc, acc);
          }
          umma_commit(&empty[s]);  // the stage is free once these MMAs have read it
        }
        umma_commit(&acc_full[a]);  // accumulator buffer a holds this segment
        ++seg;
        u = seg_end;
      }
      if (tr) tr[2] = global_timer_ns();
    }
  } else {
    // ---------------- epilogue (warps 0-3: TMEM lanes 0-127) ----------------
    grid_dep_wait();
    const int row = warp * 32 + lane;  // weight row within the tile = TMEM lane
    const uint32_t lane_off = (uint32_t)(warp * 32) << 16;
    int seg = 0;
    long long u = ub;
    while (u < ue) {
      const int t = (int)(u / KB);
      const long long tile_begin = (long long)t * KB, tile_end = tile_begin + KB;
      const long long seg_end = ue < tile_end ? ue : tile_end;
      const bool whole = (u == tile_begin && seg_end == tile_end);
      const int a = seg % nbuf;
      if (!mbar_wait(&acc_full[a], (uint32_t)(seg / nbuf) & 1u, p.err, 4)) s_abort = 1;
      named_bar_sync(1, kTcEpiThreads);
      if (*(volatile int*)&s_abort) break;
      tc_fence_after();
      const uint32_t acc_addr = tmem + lane_off + (uint32_t)a * acc_cols;
      const int n = t * kTcTileN + row;
      const int slot = (t == (int)(ub / KB)) ? 0 : 1;
      float* mypart = p.partial + (((size_t)cta * 2 + slot) * ACCS * p.BN) * kTcTileN;
      const int split = (EPI == TEPI_SPLIT_F32) ? cta - tc_unit_owner(U, G, tile_begin) : 0;
      for (int cb = 0; cb < p.BN; cb += 16) {
        float v[16], w2[16];
        tmem_ld16(acc_addr + (uint32_t)cb, v);
        if (SILU) tmem_ld16(acc_addr + (uint32_t)(p.BN + cb), w2);
        if (EPI == TEPI_SPLIT_F32) {
          if (n < p.N) {
            float* dst = reinterpret_cast<float*>(p.out) + (size_t)split * p.B * p.N + n;
#pragma unroll
            for (int j = 0; j < 16; ++j)
              if (cb + j < p.B) dst[(size_t)(cb + j) * p.N] = v[j];
          }
        } else if (whole) {
          if (n < p.N) {
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              const int b = cb + j;
              if (b < p.B) {
                const size_t o = (size_t)b * p.N + n;
                tc_store<EPI>(p, o, tc_apply<EPI>(p, o, v[j], SILU ? w2[j] : 0.f));
              }
            }
          }
        } else {
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            mypart[(size_t)(cb + j) * kTcTileN + row] = v[j];
            if (SILU) mypart[((size_t)p.BN + cb + j) * kTcTileN + row] = w2[j];
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&acc_empty[a]);  // the MMA warp may reuse this accumulator buffer
      if (!whole && EPI != TEPI_SPLIT_F32) {
        // Publish this contributor's partial; the reduction waits until the
        // whole mainloop is done (below), so no CTA ever waits mid-stream.
        named_bar_sync(1, kTcEpiThreads);
        if (threadIdx.x == 0) red_release_gpu(p.counters + t, 1u);
      }
      ++seg;
      u = seg_end;
    }

    if (tr && threadIdx.x == 0) tr[3] = global_timer_ns();
    // ---- deferred stream-K reduction of this CTA's partial tiles ----
    if (EPI != TEPI_SPLIT_F32 && !*(volatile int*)&s_abort)
      tc_stream_k_fixup<EPI>(p, U, G, KB, ub, ue, cta, smem, (size_t)NS * p.stage_bytes, red_bar, &s_abort, tr);
  }

  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(p.tmem_cols) : "memory");
  }
}


// ---------------------------------------------------------------------------
// Large-M GEMM (prefill, config 5): out[M, N] = epilogue(x[M, K] . w[N, K]^T)
// for M in the thousands.  Persistent CTAs walk output tiles of 128 weight
// rows (MMA M, operand A) x BN activation rows (MMA N, operand B: 256, or 128
// for the SiLU pair whose gate and up tiles share one activation tile), each
// over the whole K: no split-K, no partials.  Tiles are visited in bands of
// kBgGroup activation tiles so that a band's activations and the weight tiles
// in use stay in L2.  Warp roles as in gemm_tc_kernel; two TMEM accumulators
// (512 columns) let the epilogue of one tile overlap the MMAs of the next.
// ---------------------------------------------------------------------------
constexpr int kBgGroup = 16;

struct BgParams {
  const __nv_bfloat16* residual;  // [M, N]
  void* out;                      // [M, N] bf16 (fp32 for STORE_F32)
  int* err;
  int M, N, tiles_n, tiles_m, kblocks, BN, stages, stage_bytes;
  uint32_t tmem_cols;  // 2 accumulators x BN x (1 or 2) columns
  int vec_epi;         // N % 16 == 0 and 16-byte aligned out / residual: row-vector epilogue through smem
};
constexpr int kBgStageCols = 16;                          // activation columns per epilogue chunk
constexpr int kBgEpiBytes = kBgStageCols * kTcTileN * 4;  // fp32 staging of one chunk: 8 KB

__device__ __forceinline__ void bg_tile(int i, const BgParams& p, int& tn, int& tm) {
  const int band_tiles = kBgGroup * p.tiles_n;
  const int band = i / band_tiles, j = i - band * band_tiles;
  const int gm = min(kBgGroup, p.tiles_m - band * kBgGroup);
  tm = band * kBgGroup + j % gm;
  tn = j / gm;
}

template <int EPI>
__global__ void __launch_bounds__(kTcThreads, 1)
    gemm_big_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_w2,
                    const __grid_constant__ CUtensorMap tm_x, BgParams p) {
  constexpr bool SILU = (EPI == TEPI_SILU_MUL);
  constexpr int ACCS = SILU ? 2 : 1;
  constexpr uint32_t kWBytes = kTcTileN * kTcBlockK * 2;
  extern __shared__ unsigned char bg_smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<size_t>(bg_smem_raw) + 1023) & ~size_t(1023));
  const int NS = p.stages;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + (size_t)NS * p.stage_bytes);
  uint64_t* empty = full + NS;
  uint64_t* acc_full = empty + NS;
  uint64_t* acc_empty = acc_full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
  float* epi_stage = reinterpret_cast<float*>(smem + (size_t)NS * p.stage_bytes + 1024);  // [16][128]
  __shared__ int s_abort;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int total = p.tiles_n * p.tiles_m;
  const int KB = p.kblocks;
  const uint32_t x_bytes = (uint32_t)p.BN * kTcBlockK * 2;
  const uint32_t idesc = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(p.BN >> 3) << 17) |
                         ((uint32_t)(kTcTileN >> 4) << 24);
  const uint32_t acc_cols = (uint32_t)(p.BN * ACCS);

  if (threadIdx.x == 0) {
    for (int st = 0; st < NS; ++st) {
      mbar_init(&full[st], 1);
      mbar_init(&empty[st], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], kTcEpiThreads);
    }
    s_abort = 0;
    mbar_fence_init();
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(p.tmem_cols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  grid_dep_launch();
  const uint32_t tmem = *tmem_slot;

  if (warp == 4) {
    if (lane == 0) {  // TMA producer
      grid_dep_wait();
      long long it = 0;
      for (int i = blockIdx.x; i < total && !*(volatile int*)&s_abort; i += gridDim.x) {
        int tn, tm;
        bg_tile(i, p, tn, tm);
        for (int kb = 0; kb < KB; ++kb, ++it) {
          const int st = (int)(it % NS);
          if (it >= NS && !mbar_wait(&empty[st], (uint32_t)((it / NS) - 1) & 1u, p.err, 17)) {
            s_abort = 1;
            break;
          }
          unsigned char* sp = smem + (size_t)st * p.stage_bytes;
          mbar_arrive_expect_tx(&full[st], kWBytes * ACCS + x_bytes);
          tma_load_2d(sp, &tm_w, kb * kTcBlockK, tn * kTcTileN, &full[st]);
          if (SILU) tma_load_2d(sp + kWBytes, &tm_w2, kb * kTcBlockK, tn * kTcTileN, &full[st]);
          tma_load_2d(sp + kWBytes * ACCS, &tm_x, kb * kTcBlockK, tm * p.BN, &full[st]);
        }
      }
    }
  } else if (warp == 5) {
    if (lane == 0) {  // MMA issuer
      long long it = 0;
      int lt = 0;
      for (int i = blockIdx.x; i < total && !*(volatile int*)&s_abort; i += gridDim.x, ++lt) {
        const int a = lt & 1;
        if (lt >= 2 && !mbar_wait(&acc_empty[a], (uint32_t)((lt >> 1) - 1) & 1u, p.err, 18)) {
          s_abort = 1;
          break;
        }
        tc_fence_after();
        const uint32_t acc_tmem = tmem + (uint32_t)a * acc_cols;
        for (int kb = 0; kb < KB; ++kb, ++it) {
          const int st = (int)(it % NS);
          if (!mbar_wait(&full[st], (uint32_t)(it / NS) & 1u, p.err, 19)) {
            s_abort = 1;
            break;
          }
          tc_fence_after();
          const uint32_t sw = smem_u32(smem + (size_t)st * p.stage_bytes);
          const uint32_t sx = sw + kWBytes * ACCS;
#pragma unroll
          for (int kk = 0; kk < kTcBlockK / 16; ++kk) {
            const uint32_t acc = (kb > 0 || kk > 0) ? 1u : 0u;
            const uint64_t bdesc = umma_desc_sw128(sx + kk * 32);
            umma_f16(acc_tmem, umma_desc_sw128(sw + kk * 32), bdesc, idesc, acc);
            if (SILU) umma_f16(acc_tmem + (uint32_t)p.BN, umma_desc_sw128(sw + kWBytes + kk * 32), bdesc, idesc, acc);
          }
          umma_commit(&empty[st]);
        }
        umma_commit(&acc_full[a]);
      }
    }
  } else {  // epilogue: warps 0-3 own TMEM lanes 0-127 (= weight rows of the tile)
    grid_dep_wait();
    const int row = warp * 32 + lane;
    const uint32_t lane_off = (uint32_t)(warp * 32) << 16;
    int lt = 0;
    for (int i = blockIdx.x; i < total; i += gridDim.x, ++lt) {
      int tn, tm;
      bg_tile(i, p, tn, tm);
      const int a = lt & 1;
      if (!mbar_wait(&acc_full[a], (uint32_t)(lt >> 1) & 1u, p.err, 20)) s_abort = 1;
      named_bar_sync(1, kTcEpiThreads);
      if (*(volatile int*)&s_abort) break;
      tc_fence_after();
      const uint32_t acc_addr = tmem + lane_off + (uint32_t)a * acc_cols;
      const int n = tn * kTcTileN + row;
      for (int cb = 0; cb < p.BN; cb += 16) {
        float v[16], w2[16];
        tmem_ld16(acc_addr + (uint32_t)cb, v);
        if (SILU) tmem_ld16(acc_addr + (uint32_t)(p.BN + cb), w2);
        if (p.vec_epi) {
          // Stage the chunk as [16 activation rows][128 weight rows] (SiLU*up
          // already formed), then each thread writes 16 consecutive outputs of
          // one activation row with 16-byte vectors (and loads the residual
          // the same way): 8 threads per row, whole 256-byte row segments.
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            float y = v[j];
            if (SILU) {
              const float g = round_bf16(v[j]);
              y = round_bf16(g / (1.0f + expf(-g))) * round_bf16(w2[j]);
            }
            epi_stage[j * kTcTileN + row] = y;
          }
          named_bar_sync(1, kTcEpiThreads);
          {
            const int jj = threadIdx.x >> 3, part = threadIdx.x & 7;
            const int b = tm * p.BN + cb + jj;
            const int n0 = tn * kTcTileN + part * 16;
            if (b < p.M && n0 < p.N) {
              const float4* src = reinterpret_cast<const float4*>(epi_stage + jj * kTcTileN + part * 16);
              float y[16];
#pragma unroll
              for (int q = 0; q < 4; ++q) {
                const float4 f = src[q];
                y[4 * q] = f.x, y[4 * q + 1] = f.y, y[4 * q + 2] = f.z, y[4 * q + 3] = f.w;
              }
              const size_t o = (size_t)b * p.N + n0;
              if (EPI == TEPI_RESIDUAL) {
                float r[16];
                unpack8(ldg16(p.residual + o), r);
                unpack8(ldg16(p.residual + o + 8), r + 8);
#pragma unroll
                for (int q = 0; q < 16; ++q) y[q] = r[q] + round_bf16(y[q]);
              }
              if (EPI == TEPI_STORE_F32) {
                float4* dst = reinterpret_cast<float4*>(reinterpret_cast<float*>(p.out) + o);
#pragma unroll
                for (int q = 0; q < 4; ++q) dst[q] = make_float4(y[4 * q], y[4 * q + 1], y[4 * q + 2], y[4 * q + 3]);
              } else {
                uint4 pk[2];
                uint32_t* pw = reinterpret_cast<uint32_t*>(pk);
#pragma unroll
                for (int q = 0; q < 8; ++q) {
                  __nv_bfloat162 h2 = __floats2bfloat162_rn(y[2 * q], y[2 * q + 1]);
                  pw[q] = *reinterpret_cast<uint32_t*>(&h2);
                }
                uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(p.out) + o);
                dst[0] = pk[0];
                dst[1] = pk[1];
              }
            }
          }
          named_bar_sync(1, kTcEpiThreads);  // the staging buffer is free again
          continue;
        }
        if (n < p.N) {
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const int b = tm * p.BN + cb + j;
            if (b < p.M) {
              const size_t o = (size_t)b * p.N + n;
              float y = v[j];
              if (EPI == TEPI_RESIDUAL) y = bf16_to_f(p.residual[o]) + round_bf16(y);
              if (SILU) {
                const float g = round_bf16(v[j]);
                y = round_bf16(g / (1.0f + expf(-g))) * round_bf16(w2[j]);
              }
              if (EPI == TEPI_STORE_F32) reinterpret_cast<float*>(p.out)[o] = y;
              else reinterpret_cast<__nv_bfloat16*>(p.out)[o] = f_to_bf16(y);
            }
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&acc_empty[a]);
    }
  }

  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(p.tmem_cols) : "memory");
  }
}

}  // namespace lsb

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
namespace lsb_host {
using namespace lsb;

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
  }
  return fn;
}

// 2-D bf16 tensor map over a row-major [rows, cols] matrix, box [box_rows, 64], 128-byte swizzle.
static int make_map(CUtensorMap* map, const void* base, int64_t rows, int64_t cols, int box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return set_error(LS_ERR_NOT_SUPPORTED, "cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)cols * 2};
  cuuint32_t box[2] = {(cuuint32_t)kTcBlockK, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(LS_ERR_INVALID_ARGUMENT, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return LS_OK;
}

struct TcPlan {
  int grid, BN, tiles, kblocks, stages, stage_bytes, accs, acc_buffers;
  int splits;  // CTAs per tile on a tile-aligned grid (TEPI_SPLIT_F32)
  uint32_t tmem_cols;
  size_t smem, counter_bytes, partial_bytes;
};

// Shared memory given to the stage ring.  Under load the HBM round trip is a
// few microseconds, so the bytes in flight per SM (stages x tile bytes) set the
// stream rate; 112 KB measured best (64 to 208 KB swept).
static int tc_stage_budget_kb() { return 112; }

#ifdef LEANB200_PROFILING
// Profiling hook (ls_gemm_tc_set_trace): per CTA 8 stamps: start, first stage
// landed, last MMA issued, epilogue done, then for the first and the last
// split tile: counter complete, share reduced (0 where there is none).
static unsigned long long* g_tc_trace = nullptr;
#endif

static TcPlan tc_plan(int64_t m, int64_t k, int64_t n_out, int epi) {
  TcPlan pl = {};
  pl.accs = (epi == TEPI_SILU_MUL) ? 2 : 1;
  pl.BN = (int)((m + 15) / 16 * 16);
  pl.tiles = (int)((n_out + kTcTileN - 1) / kTcTileN);
  pl.kblocks = (int)((k + kTcBlockK - 1) / kTcBlockK);
  const int64_t units = (int64_t)pl.tiles * pl.kblocks;
  const int sms = sm_count();
  pl.stage_bytes = (int)(((size_t)kTcTileN * kTcBlockK * 2 * pl.accs + (size_t)pl.BN * kTcBlockK * 2 + 1023) / 1024 *
                         1024);
  int stages = (int)(((size_t)tc_stage_budget_kb() * 1024) / pl.stage_bytes);
  if (stages > kTcMaxStages) stages = kTcMaxStages;
  // At least four stages: with two or three of the large stages of the wider
  // SiLU pairs (M 48-128: 40-48 KB each) the ring ran dry between HBM round
  // trips (gate_up at M 80: 39.7 -> 35.9 us; verify pass 5.57 -> 5.32 ms,
  // bs32 step 5543 -> 5700 tok/s).
  if (stages < 4) stages = 4;
  pl.stages = stages;
  // Two accumulator buffers while they fit in 256 TMEM columns (half the SM's
  // TMEM, so a co-resident CTA of the next kernel can always allocate).
  pl.acc_buffers = (2 * pl.BN * pl.accs <= 256) ? 2 : 1;
  uint32_t cols = 32;
  while (cols < (uint32_t)(pl.acc_buffers * pl.BN * pl.accs)) cols <<= 1;
  pl.tmem_cols = cols;
  pl.smem = 1024 + (size_t)pl.stages * pl.stage_bytes + (size_t)(2 * pl.stages + 6) * 8 + 16;
  pl.grid = (int)(units < sms ? units : sms);
  // Fewer tiles than SMs: with the grid a multiple of the tile count, the even
  // split of the unit list falls on tile boundaries, so every CTA holds a
  // k-range of exactly one tile and reduces one share (split-K).  Taken when
  // it keeps at least 90% of the SMs streaming (Qwen3-4B: QKV 48 tiles -> 144
  // CTAs, o_proj / down 20 tiles -> 140), or with the next multiple when that
  // is at most 5% above the SM count and two CTAs fit on one SM, so that the
  // few SMs that run two CTAs need no second wave (gate_up, 76 pair tiles ->
  // 152 CTAs at M <= 32: 28.4 -> 25.9 us at M 16; at M 80 the 126 KB ring
  // does not fit twice and the extra CTAs ran as a second wave, 38% slower).
  // Under full stream-K the CTAs that hold pieces of two split tiles reduce
  // both, one after the other, and set the end of the kernel (measured tail
  // after the last MMA: 8-11 us at M 8-80).
  // The split-partial epilogue always takes the tile-aligned grid (with one
  // CTA per tile when there are more tiles than SMs): its consumer needs every
  // tile split the same way.
  const bool split_out = (epi == TEPI_SPLIT_F32);
  if (pl.tiles >= sms && split_out) {
    // One CTA per whole-K tile.  Up to twice the SM count, two CTAs share an
    // SM, so the ring is cut until two fit (at least two stages).
    pl.grid = pl.tiles;
    while (pl.stages > 2 && 2 * (1024 + (size_t)pl.stages * pl.stage_bytes + (size_t)(2 * pl.stages + 6) * 8 + 16 +
                                 1024) > (size_t)228 * 1024)
      --pl.stages;
    pl.smem = 1024 + (size_t)pl.stages * pl.stage_bytes + (size_t)(2 * pl.stages + 6) * 8 + 16;
  }
  if (pl.tiles < sms && split_out) {
    // Two CTAs per SM (twice the splits), each with a ring cut to fit beside
    // the other: a CTA's stream rate is bound by the bytes its ring keeps in
    // flight, so an SM with two streams about twice as fast.
    int st = pl.stages;
    auto smem_of = [&](int stages) {
      return 1024 + (size_t)stages * pl.stage_bytes + (size_t)(2 * stages + 6) * 8 + 16;
    };
    while (st > 3 && 2 * (smem_of(st) + 1024) > (size_t)228 * 1024) --st;
    const int per2 = (2 * sms) / pl.tiles < pl.kblocks ? (2 * sms) / pl.tiles : pl.kblocks;
    if (2 * (smem_of(st) + 1024) <= (size_t)228 * 1024 && per2 > sms / pl.tiles) {
      pl.stages = st;
      pl.smem = smem_of(st);
      pl.grid = pl.tiles * per2;
    }
  }
  if (pl.tiles < sms && pl.grid <= sms) {
    const int per_tile = sms / pl.tiles < pl.kblocks ? sms / pl.tiles : pl.kblocks;
    const int g = pl.tiles * per_tile;
    const int g_up = pl.tiles * (per_tile + 1);
    if (per_tile + 1 <= pl.kblocks && (int64_t)g_up * 100 <= (int64_t)sms * 105 &&
        2 * (pl.smem + 1024) <= (size_t)228 * 1024)
      pl.grid = g_up;
    else if ((int64_t)g * 10 >= (int64_t)sms * 9 || split_out)
      pl.grid = g;
  }
  pl.splits = pl.grid / pl.tiles;
  pl.counter_bytes = split_out ? 0 : kTcCounterBytes;
  pl.partial_bytes = split_out ? 0 : (size_t)pl.grid * 2 * pl.accs * pl.BN * kTcTileN * 4;
  return pl;
}

int tc_split_count(int64_t m, int64_t k, int64_t n_out, int64_t* splits) {
  *splits = tc_plan(m, k, n_out, TEPI_SPLIT_F32).splits;
  return LS_OK;
}

int tc_workspace_bytes(int64_t m, int64_t k, int64_t n_out, int epi, int64_t* bytes) {
  TcPlan pl = tc_plan(m, k, n_out, epi);
  *bytes = (int64_t)(pl.counter_bytes + pl.partial_bytes);
  return LS_OK;
}

template <int EPI>
static int launch_tc_t(const CUtensorMap& w, const CUtensorMap& w2, const CUtensorMap& x, const TcParams& p,
                       const TcPlan& pl, cudaStream_t stream) {
  auto kern = gemm_tc_kernel<EPI>;
  static int configured[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && (int)pl.smem > configured[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)pl.smem);
    if (e != cudaSuccess) return set_error(LS_ERR_CUDA, "cudaFuncSetAttribute(gemm_tc): %s", cudaGetErrorString(e));
    configured[dev] = (int)pl.smem;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(pl.grid);
  cfg.blockDim = dim3(kTcThreads);
  cfg.dynamicSmemBytes = pl.smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, w, w2, x, p);
  if (e != cudaSuccess) return set_error(LS_ERR_CUDA, "gemm_tc launch: %s", cudaGetErrorString(e));
  return LS_OK;
}

// out[m, n_out] = epilogue(x[m, k] . w^T); for SILU_MUL w is [2 n_out, k] (gate rows, then up rows).
int64_t tc_tiled_bytes(int64_t n_out, int64_t k, int silu);

int launch_gemm_tc(const void* x, int64_t m, int64_t k, const void* w, int64_t n_out, int epi, const void* residual,
                   void* out, void* workspace, int64_t workspace_bytes, cudaStream_t stream,
                   const void* w_tiled) {
  if (!x || !(w || w_tiled) || !out) return set_error(LS_ERR_INVALID_ARGUMENT, "gemm_tc: null pointer");
  // m <= 128 keeps every CTA at <= 256 TMEM columns, so any two CTAs that
  // share an SM can both allocate (a blocked allocation would stall the
  // stream-K reduction of the CTA holding the columns).
  if (m < 1 || m > 128) return set_error(LS_ERR_UNSUPPORTED_SHAPE, "gemm_tc: m=%lld outside 1..128", (long long)m);
  if (k < 8 || k % 8 || n_out < 1) return set_error(LS_ERR_MISALIGNED, "gemm_tc: k=%lld must be a positive multiple of 8",
                                                    (long long)k);
  if (!aligned16(x) || (!w_tiled && !aligned16(w)) || (workspace && !aligned16(workspace)))
    return set_error(LS_ERR_MISALIGNED, "gemm_tc: x, w and the workspace must be 16-byte aligned");
  if (epi == TEPI_RESIDUAL && !residual) return set_error(LS_ERR_INVALID_ARGUMENT, "gemm_tc: residual is null");
  TcPlan pl = tc_plan(m, k, n_out, epi);
  if (pl.tmem_cols > 256) return set_error(LS_ERR_UNSUPPORTED_SHAPE, "gemm_tc: m=%lld too wide for TMEM", (long long)m);
  if (pl.tiles > kTcMaxTiles)
    return set_error(LS_ERR_UNSUPPORTED_SHAPE, "gemm_tc: n=%lld has more than %d row tiles", (long long)n_out,
                     kTcMaxTiles);
  if (epi == TEPI_SPLIT_F32 && !aligned16(out))
    return set_error(LS_ERR_MISALIGNED, "gemm_tc: split partial output must be 16-byte aligned");
  if (epi != TEPI_SPLIT_F32 && (!workspace || workspace_bytes < (int64_t)(pl.counter_bytes + pl.partial_bytes)))
    return set_error(LS_ERR_WORKSPACE, "gemm_tc: workspace needs %zu bytes", pl.counter_bytes + pl.partial_bytes);
  if (!w_tiled && epi == TEPI_SILU_MUL && ((n_out * k * 2) % 16))
    return set_error(LS_ERR_MISALIGNED, "gemm_tc: up-projection view misaligned");
  CUtensorMap mw, mw2, mx;
  int rc = 0;
  if (w_tiled) {
    if (!aligned16(w_tiled)) return set_error(LS_ERR_MISALIGNED, "gemm_tc: tiled weights not 16-byte aligned");
    memset(&mw, 0, sizeof(mw));
    mw2 = mw;
  } else {
    rc = make_map(&mw, w, n_out, k, kTcTileN);
    if (rc) return rc;
    if (epi == TEPI_SILU_MUL) {
      rc = make_map(&mw2, static_cast<const __nv_bfloat16*>(w) + n_out * k, n_out, k, kTcTileN);
      if (rc) return rc;
    } else {
      mw2 = mw;
    }
  }
  rc = make_map(&mx, x, m, k, pl.BN);
  if (rc) return rc;
  TcParams p = {};
  p.residual = static_cast<const __nv_bfloat16*>(residual);
  p.out = static_cast<__nv_bfloat16*>(out);
  p.counters = workspace ? static_cast<unsigned int*>(workspace) : nullptr;
  p.partial = workspace ? reinterpret_cast<float*>(static_cast<char*>(workspace) + pl.counter_bytes) : nullptr;
  p.err = device_error_ptr();
  p.B = (int)m;
  p.BN = pl.BN;
  p.N = (int)n_out;
  p.tiles = pl.tiles;
  p.kblocks = pl.kblocks;
  p.stages = pl.stages;
  p.stage_bytes = pl.stage_bytes;
  p.acc_buffers = pl.acc_buffers;
  p.tmem_cols = pl.tmem_cols;
  p.w_tiled = static_cast<const unsigned char*>(w_tiled);
#ifdef LEANB200_PROFILING
  p.trace = g_tc_trace;
#endif
  p.aligned = (n_out % 8 == 0) && aligned16(out) && (!residual || aligned16(residual)) ? 1 : 0;
  p.w2_tiled = w_tiled ? p.w_tiled + tc_tiled_bytes(n_out, k, 0) : nullptr;
  switch (epi) {
    case TEPI_STORE: return launch_tc_t<TEPI_STORE>(mw, mw2, mx, p, pl, stream);
    case TEPI_RESIDUAL: return launch_tc_t<TEPI_RESIDUAL>(mw, mw2, mx, p, pl, stream);
    case TEPI_SILU_MUL: return launch_tc_t<TEPI_SILU_MUL>(mw, mw2, mx, p, pl, stream);
    case TEPI_STORE_F32: return launch_tc_t<TEPI_STORE_F32>(mw, mw2, mx, p, pl, stream);
    case TEPI_SPLIT_F32: return launch_tc_t<TEPI_SPLIT_F32>(mw, mw2, mx, p, pl, stream);
    default: return set_error(LS_ERR_INVALID_ARGUMENT, "gemm_tc: unknown epilogue %d", epi);
  }
}


template <int EPI>
static int launch_big_t(const CUtensorMap& w, const CUtensorMap& w2, const CUtensorMap& x, const BgParams& p,
                        int grid, size_t smem, cudaStream_t stream) {
  auto kern = gemm_big_kernel<EPI>;
  static int configured[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && (int)smem > configured[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return set_error(LS_ERR_CUDA, "cudaFuncSetAttribute(gemm_big): %s", cudaGetErrorString(e));
    configured[dev] = (int)smem;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kTcThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, w, w2, x, p);
  return e == cudaSuccess ? LS_OK : set_error(LS_ERR_CUDA, "gemm_big launch: %s", cudaGetErrorString(e));
}

// Large-M GEMM (see gemm_big_kernel); any m >= 1, k a multiple of 8.
int launch_gemm_big(const void* x, int64_t m, int64_t k, const void* w, int64_t n_out, int epi, const void* residual,
                    void* out, cudaStream_t stream) {
  if (!x || !w || !out) return set_error(LS_ERR_INVALID_ARGUMENT, "gemm_big: null pointer");
  if (m < 1 || m > (1ll << 30) || n_out < 1 || k < 8 || k % 8)
    return set_error(LS_ERR_UNSUPPORTED_SHAPE, "gemm_big: m=%lld k=%lld n=%lld", (long long)m, (long long)k,
                     (long long)n_out);
  if (!aligned16(x) || !aligned16(w)) return set_error(LS_ERR_MISALIGNED, "gemm_big: x and w must be 16-byte aligned");
  if (epi == TEPI_RESIDUAL && !residual) return set_error(LS_ERR_INVALID_ARGUMENT, "gemm_big: residual is null");
  const bool silu = epi == TEPI_SILU_MUL;
  if (silu && ((n_out * k * 2) % 16)) return set_error(LS_ERR_MISALIGNED, "gemm_big: up-projection view misaligned");
  BgParams p = {};
  // Non-SiLU epilogues with long K (o_proj, down): two CTAs per SM on
  // 128 x 128 tiles, 3 x 32 KB rings and 256 TMEM columns each, so that two
  // producer / MMA pipelines share the SM and cover the latency of operands
  // that miss L2 (a 128 x 256 tile of down needs 7.5 MB over its K).
  const bool two_per_sm = !silu && k >= 4096;
  p.BN = (silu || two_per_sm) ? 128 : 256;
  p.M = (int)m;
  p.N = (int)n_out;
  p.tiles_n = (int)((n_out + kTcTileN - 1) / kTcTileN);
  p.tiles_m = (int)((m + p.BN - 1) / p.BN);
  p.kblocks = (int)((k + kTcBlockK - 1) / kTcBlockK);
  p.stage_bytes = (silu ? 2 : 1) * kTcTileN * kTcBlockK * 2 + p.BN * kTcBlockK * 2;
  p.stages = two_per_sm ? 3 : 4;
  p.tmem_cols = two_per_sm ? 256u : 512u;
  p.residual = static_cast<const __nv_bfloat16*>(residual);
  p.out = out;
  p.err = device_error_ptr();
  const long long total = (long long)p.tiles_n * p.tiles_m;
  if (total > (1ll << 31) - 1) return set_error(LS_ERR_UNSUPPORTED_SHAPE, "gemm_big: too many tiles");
  const int cap = (two_per_sm ? 2 : 1) * sm_count();
  const int grid = (int)(total < cap ? total : cap);
  p.vec_epi = (n_out % 16 == 0) && aligned16(out) && (!residual || aligned16(residual)) ? 1 : 0;
  const size_t smem = 1024 + (size_t)p.stages * p.stage_bytes + 1024 + (size_t)kBgEpiBytes;
  CUtensorMap mw, mw2, mx;
  int rc = make_map(&mw, w, n_out, k, kTcTileN);
  if (rc) return rc;
  if (silu) {
    rc = make_map(&mw2, static_cast<const __nv_bfloat16*>(w) + n_out * k, n_out, k, kTcTileN);
    if (rc) return rc;
  } else {
    mw2 = mw;
  }
  rc = make_map(&mx, x, m, k, p.BN);
  if (rc) return rc;
  switch (epi) {
    case TEPI_STORE: return launch_big_t<TEPI_STORE>(mw, mw2, mx, p, grid, smem, stream);
    case TEPI_RESIDUAL: return launch_big_t<TEPI_RESIDUAL>(mw, mw2, mx, p, grid, smem, stream);
    case TEPI_SILU_MUL: return launch_big_t<TEPI_SILU_MUL>(mw, mw2, mx, p, grid, smem, stream);
    case TEPI_STORE_F32: return launch_big_t<TEPI_STORE_F32>(mw, mw2, mx, p, grid, smem, stream);
    default: return set_error(LS_ERR_INVALID_ARGUMENT, "gemm_big: unknown epilogue %d", epi);
  }
}

// Pre-tiling for the tcgen05 GEMM: W [N, K] -> [ceil(N/128)][ceil(K/64)] tiles
// of 128 rows x 64 k, each the 16 KB shared-memory image the MMA reads
// (K-major, 128-byte swizzle: 16-byte chunk c of row r at r * 128 + ((c ^ (r % 8)) * 16));
// rows >= N and k >= K are zero.  silu: the gate half [0, N/2) and the up half
// [N/2, N) are tiled separately, gate tiles first.
}  // namespace lsb_host

namespace lsb {
__global__ void tc_tile_kernel(const __nv_bfloat16* w, int N, int K, int tiles, int kblocks, uint4* out) {
  const long long chunks = (long long)tiles * kblocks * 128 * 8;  // 16-byte chunks
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < chunks;
       i += (long long)gridDim.x * blockDim.x) {
    const int c = (int)(i & 7);
    const int r = (int)((i >> 3) & 127);
    const long long tk = i >> 10;  // tile index t * kblocks + kb
    const int kb = (int)(tk % kblocks), t = (int)(tk / kblocks);
    const int row = t * 128 + r, k0 = kb * 64 + c * 8;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (row < N && k0 < K) v = *reinterpret_cast<const uint4*>(w + (size_t)row * K + k0);
    out[(tk << 10) + r * 8 + (c ^ (r & 7))] = v;
  }
}
}  // namespace lsb

namespace lsb_host {
int64_t tc_tiled_bytes(int64_t n_out, int64_t k, int silu) {
  const int64_t tiles = (n_out + kTcTileN - 1) / kTcTileN, kb = (k + kTcBlockK - 1) / kTcBlockK;
  return (silu ? 2 : 1) * tiles * kb * (int64_t)kTcTileN * kTcBlockK * 2;
}

int launch_tc_tile(const void* w, int64_t n_rows, int64_t k, int silu, void* out, cudaStream_t stream) {
  if (!w || !out || n_rows < 1 || k < 8 || k % 8 || (silu && n_rows % 2))
    return set_error(LS_ERR_INVALID_ARGUMENT, "gemm_tc_tile: bad arguments");
  if (!aligned16(w) || !aligned16(out)) return set_error(LS_ERR_MISALIGNED, "gemm_tc_tile: not 16-byte aligned");
  const int64_t n_out = silu ? n_rows / 2 : n_rows;
  const int tiles = (int)((n_out + kTcTileN - 1) / kTcTileN), kb = (int)((k + kTcBlockK - 1) / kTcBlockK);
  const int parts = silu ? 2 : 1;
  for (int h = 0; h < parts; ++h) {
    const __nv_bfloat16* src = static_cast<const __nv_bfloat16*>(w) + (size_t)h * n_out * k;
    uint4* dst = reinterpret_cast<uint4*>(static_cast<char*>(out) + (size_t)h * tc_tiled_bytes(n_out, k, 0));
    tc_tile_kernel<<<4 * sm_count(), 256, 0, stream>>>(src, (int)n_out, (int)k, tiles, kb, dst);
  }
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? LS_OK : set_error(LS_ERR_CUDA, "gemm_tc_tile launch: %s", cudaGetErrorString(e));
}

}  // namespace lsb_host

#ifdef LEANB200_PROFILING
extern "C" int ls_gemm_tc_set_trace(void* buffer) {
  lsb_host::g_tc_trace = static_cast<unsigned long long*>(buffer);
  return LS_OK;
}
#endif

// ---------------------------------------------------------------------------
// Causal GQA prefill attention on tcgen05 (config 5).
//
// Same contract as prefill_attention_kernel (attention_prefill.cu): query row
// r = (token i, group member g) of kv head h in sequence b sees keys
// 0 .. cache_pos[b] + i (src/leanstack/runtime/qwen_explicit.py:551-563,
// :1000-1039).  A CTA owns 128 consecutive rows of one (sequence, kv head)
// (the MMA's M) and walks 128-key tiles of the cache:
//   * warp 4 streams K and V tiles with TMA (128-byte swizzle) into a 2-stage
//     ring; the rows of one (b, h) are contiguous [S, 128] strips;
//   * warp 5 issues S = Q K^T into TMEM columns [0, 128) (Q and K K-major),
//     then O += P V into columns [128, 256) with V as an MN-major B operand
//     (the cache's [key][dim] layout read as dims x keys: 64-dim halves 16 KB
//     apart, 8-key groups 1 KB apart), and S of the next tile while the
//     softmax of the current one runs;
//   * warps 0-7 run the softmax, two threads per row: warps w and w + 4 read
//     TMEM lanes 32 (w % 4) .. + 31 (row = lane) and own keys / output dims
//     [0, 64) and [64, 128) respectively.  Both take the maximum over the
//     whole 128-score row (exact and order-free, so they agree) and
//     exponentiate their own half: online softmax in fp32 (exp2 of the
//     log2-scaled scores), P split into bf16 hi + lo (about 16 bits of the
//     probability, as the mma.sync kernels do) written to shared memory in the
//     K-major layout, O rescaled in TMEM when the row maximum grows, and
//     finally O / l stored as bf16 (the two halves' row sums added once).
// V rows past the last visible key are zeroed in shared memory before the PV
// product: the cache beyond a sequence's length is the caller's memory and may
// hold anything, and 0 x NaN is NaN.  Every wait is bounded (LS_ERR_TIMEOUT).
// ---------------------------------------------------------------------------
namespace lsb {

constexpr int kPtRows = 128;   // query rows per CTA (MMA M)
constexpr int kPtKeys = 64;    // keys per tile (S's N, PV's K)
constexpr int kPtQHalf = 16384;              // Q: two 64-dim halves of [128 rows x 64] bf16
constexpr int kPtKvHalf = 8192;              // K or V tile: two 64-dim halves of [64 keys x 64] bf16
constexpr int kPtP = 8192 * 2;               // one P tile [128 rows x 64 keys] bf16 = 16 KB (hi or lo)
constexpr int kPtQ = 0;
constexpr int kPtPbuf = 2 * kPtQHalf;        // P buffers: 2 x (hi, lo)
constexpr int kPtRing = kPtPbuf + 2 * 2 * kPtP;
constexpr int kPtStage = 4 * kPtKvHalf;      // K + V of one tile: 32 KB
constexpr int kPtStages = 3;
constexpr int kPtBars = kPtRing + kPtStages * kPtStage;  // 196608
constexpr int kPtSmem = 1024 + kPtBars + 128;
constexpr int kPtThreads = 320;  // 8 softmax warps, TMA warp 8, MMA warp 9
constexpr int kPtSoft = 256;
// The row maximum used for the exponent only moves (and O is rescaled) when a
// score exceeds it by more than 2^8: P stays <= 256, well inside what the
// bf16 hi + lo split represents to about 16 bits.
constexpr float kPtRescaleLog2 = 8.f;

struct PtParams {
  const __nv_bfloat16* q;  // [M, Hq, D]
  const int* cache_pos;    // [B] or null (then uniform_past)
  int uniform_past;
  __nv_bfloat16* out;      // [M, Hq * D]
  int* err;
  int q_len, Hq, Hkv, G, R, max_seq;
  float scale_log2;
};

__device__ __forceinline__ uint64_t umma_desc_sw128_mn(uint32_t saddr, uint32_t lbo_bytes) {
  // MN-major, 128-byte swizzle: 64-element MN chunks lbo_bytes apart (LBO),
  // 8-row K groups 1024 B apart (SBO), descriptor version 1, SWIZZLE_128B.
  return (uint64_t)((saddr >> 4) & 0x3FFF) | ((uint64_t)(lbo_bytes >> 4) << 16) | (64ull << 32) | (1ull << 46) |
         (2ull << 61);
}

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const float v[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
          taddr),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])), "r"(__float_as_uint(v[3])),
      "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])), "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])),
      "r"(__float_as_uint(v[8])), "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])),
      "r"(__float_as_uint(v[11])), "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])),
      "r"(__float_as_uint(v[14])), "r"(__float_as_uint(v[15]))
      : "memory");
}
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
// 2^x with the hardware's approximate exp2 (MUFU); 2^-inf = 0.  The softmax
// probabilities are rounded to about 16 bits afterwards.
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Byte offset of 16-byte chunk c of row r in a K-major tile stored as 64-wide
// halves of `half` bytes each (128-byte swizzle; c >> 3 selects the half).
__device__ __forceinline__ uint32_t pt_off(int r, int c, int half) {
  return (uint32_t)((c >> 3) * half + r * 128 + (((c & 7) ^ (r & 7)) << 4));
}

__global__ void __launch_bounds__(kPtThreads, 1)
    prefill_attention_tc_kernel(const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_v,
                                PtParams p) {
  extern __shared__ unsigned char pt_smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<size_t>(pt_smem_raw) + 1023) & ~size_t(1023));
  uint64_t* kv_full = reinterpret_cast<uint64_t*>(smem + kPtBars);
  uint64_t* kv_empty = kv_full + kPtStages;
  uint64_t* q_full = kv_empty + kPtStages;
  uint64_t* s_full = q_full + 1;
  uint64_t* s_free = s_full + 1;
  uint64_t* p_full = s_free + 1;  // [2]: one per P buffer
  uint64_t* o_done = p_full + 2;  // [2]: the PV product that read P buffer b is complete
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(o_done + 2);
  __shared__ int s_abort;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int b = blockIdx.z, hkv = blockIdx.y;
  const int r0 = (gridDim.x - 1 - blockIdx.x) * kPtRows;  // longest row blocks first

  if (threadIdx.x == 0) {
    for (int s = 0; s < kPtStages; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    mbar_init(q_full, kPtSoft);
    mbar_init(s_full, 1);
    mbar_init(s_free, kPtSoft);
    for (int u = 0; u < 2; ++u) {
      mbar_init(&p_full[u], kPtSoft);
      mbar_init(&o_done[u], 1);
    }
    s_abort = 0;
    mbar_fence_init();
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(256)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tS = tmem, tO = tmem + 128;  // S: columns [0, 64); O: [128, 256)

  // The cache and the queries are written by the previous kernel.
  grid_dep_wait();
  grid_dep_launch();
  const int cp = p.cache_pos ? p.cache_pos[b] : p.uniform_past;
  int L = cp + p.q_len;
  if (L > p.max_seq || cp < 0) {
    if (threadIdx.x == 0 && blockIdx.x == 0) raise_device_error(p.err, LS_ERR_KV_OVERFLOW);
    L = min(max(L, 0), p.max_seq);
  }
  const int r_last = min(r0 + kPtRows, p.R) - 1;
  const int L_blk = min(L, cp + r_last / p.G + 1);
  const int ntiles = L_blk > 0 ? (L_blk + kPtKeys - 1) / kPtKeys : 0;
  const int kv_row0 = (b * p.Hkv + hkv) * p.max_seq;

  if (warp == 8) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      for (int kt = 0; kt < ntiles && !*(volatile int*)&s_abort; ++kt) {
        const int s = kt % kPtStages;
        if (kt >= kPtStages && !mbar_wait(&kv_empty[s], (uint32_t)((kt / kPtStages) - 1) & 1u, p.err, 0x21)) {
          s_abort = 1;
          break;
        }
        unsigned char* st = smem + kPtRing + s * kPtStage;
        mbar_arrive_expect_tx(&kv_full[s], kPtStage);
        const int y = kv_row0 + kt * kPtKeys;
        tma_load_2d(st, &tm_k, 0, y, &kv_full[s]);
        tma_load_2d(st + kPtKvHalf, &tm_k, 64, y, &kv_full[s]);
        tma_load_2d(st + 2 * kPtKvHalf, &tm_v, 0, y, &kv_full[s]);
        tma_load_2d(st + 3 * kPtKvHalf, &tm_v, 64, y, &kv_full[s]);
      }
    }
  } else if (warp == 9) {
    // ---------------- MMA issuer ----------------
    if (lane == 0 && ntiles > 0) {
      constexpr uint32_t idesc_s = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(kPtKeys >> 3) << 17) |
                                   ((uint32_t)(kPtRows >> 4) << 24);
      constexpr uint32_t idesc_pv = (1u << 4) | (1u << 7) | (1u << 10) | (1u << 16) | ((uint32_t)(128 >> 3) << 17) |
                                    ((uint32_t)(kPtRows >> 4) << 24);  // B (V) MN-major; N = 128 dims
      const uint32_t sQ = smem_u32(smem + kPtQ);
      auto issue_s = [&](int kt) -> bool {
        const int s = kt % kPtStages;
        if (!mbar_wait(&kv_full[s], (uint32_t)(kt / kPtStages) & 1u, p.err, 0x22)) return false;
        if (kt > 0 && !mbar_wait(s_free, (uint32_t)(kt - 1) & 1u, p.err, 0x23)) return false;
        tc_fence_after();
        const uint32_t sK = smem_u32(smem + kPtRing + s * kPtStage);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint32_t qo = (uint32_t)((kk >> 2) * kPtQHalf + (kk & 3) * 32);
          const uint32_t ko = (uint32_t)((kk >> 2) * kPtKvHalf + (kk & 3) * 32);
          umma_f16(tS, umma_desc_sw128(sQ + qo), umma_desc_sw128(sK + ko), idesc_s, kk > 0 ? 1u : 0u);
        }
        umma_commit(s_full);
        return true;
      };
      bool ok = mbar_wait(q_full, 0u, p.err, 0x24) && issue_s(0);
      for (int kt = 0; ok && kt < ntiles; ++kt) {
        if (kt + 1 < ntiles && !issue_s(kt + 1)) {
          ok = false;
          break;
        }
        const int u = kt & 1;
        if (!mbar_wait(&p_full[u], (uint32_t)(kt >> 1) & 1u, p.err, 0x25)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t sPh = smem_u32(smem + kPtPbuf + u * 2 * kPtP), sPl = sPh + kPtP;
        const uint32_t sV = smem_u32(smem + kPtRing + (kt % kPtStages) * kPtStage + 2 * kPtKvHalf);
#pragma unroll
        for (int kk = 0; kk < kPtKeys / 16; ++kk) {
          const uint64_t bdesc = umma_desc_sw128_mn(sV + kk * 2048, kPtKvHalf);
          umma_f16(tO, umma_desc_sw128(sPh + kk * 32), bdesc, idesc_pv, (kt > 0 || kk > 0) ? 1u : 0u);
          umma_f16(tO, umma_desc_sw128(sPl + kk * 32), bdesc, idesc_pv, 1u);
        }
        umma_commit(&o_done[u]);
        umma_commit(&kv_empty[kt % kPtStages]);
      }
      if (!ok) s_abort = 1;
    }
  } else {
    // ---------------- softmax / epilogue: warps 0-7, two threads per query row ----------------
    const int quad = warp & 3, ch = warp >> 2;  // TMEM lane quadrant; key / dim half
    const int r = quad * 32 + lane;
    const int row = r0 + r;
    const bool valid = row < p.R;
    const int i = valid ? row / p.G : 0;
    const int gq = valid ? row - i * p.G : 0;
    const int lim = valid ? cp + i : -1;
    const uint32_t lane_off = (uint32_t)(quad * 32) << 16;
    constexpr int kHalfKeys = kPtKeys / 2;  // 32 keys of each tile per thread
    const int own = ch * kHalfKeys, other = (1 - ch) * kHalfKeys;
    {  // this thread's half of the Q row into shared memory (zeros for rows past the end)
      const uint4* qp = reinterpret_cast<const uint4*>(p.q + ((size_t)(b * p.q_len + i) * p.Hq + hkv * p.G + gq) * 128);
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        const uint4 v = valid ? qp[ch * 8 + c] : make_uint4(0, 0, 0, 0);
        *reinterpret_cast<uint4*>(smem + kPtQ + pt_off(r, ch * 8 + c, kPtQHalf)) = v;
      }
      fence_proxy_async_smem();
      mbar_arrive(q_full);
    }
    float m_run = -INFINITY, l_half = 0.f;
    bool ok = true;
    for (int kt = 0; kt < ntiles; ++kt) {
      // Wait results are made warp-uniform: the tcgen05.ld / st below are
      // warp-collective and must not be reached by part of a warp.
      if (!__all_sync(0xffffffffu, mbar_wait(s_full, (uint32_t)kt & 1u, p.err, 0x26))) {
        ok = false;
        break;
      }
      tc_fence_after();
      const int j0 = kt * kPtKeys;
      float sv[kHalfKeys], t[kHalfKeys];
#pragma unroll
      for (int c = 0; c < kHalfKeys / 16; ++c) {
        tmem_ld16(tS + lane_off + (uint32_t)(other + c * 16), t + c * 16);
        tmem_ld16(tS + lane_off + (uint32_t)(own + c * 16), sv + c * 16);
      }
      tc_fence_before();
      mbar_arrive(s_free);  // S is in registers: the next tile's QK^T may overwrite it
      // Both threads of a row take the maximum over the whole row (the same raw
      // scores in another order; max is exact and order-free, and the scale is
      // positive, so the scaled maximum is that of the scaled scores).  Tiles
      // every row of the warp sees in full skip the causal mask.
      const bool full = __all_sync(0xffffffffu, j0 + kPtKeys - 1 <= lim);
      float mraw = -INFINITY;
      if (full) {
#pragma unroll
        for (int e = 0; e < kHalfKeys; ++e) mraw = fmaxf(mraw, fmaxf(t[e], sv[e]));
      } else {
#pragma unroll
        for (int e = 0; e < kHalfKeys; ++e) {
          mraw = fmaxf(mraw, (j0 + other + e > lim) ? -INFINITY : t[e]);
          mraw = fmaxf(mraw, (j0 + own + e > lim) ? -INFINITY : sv[e]);
        }
      }
      const float mt = (mraw == -INFINITY) ? -INFINITY : mraw * p.scale_log2;
      bool resc = false;
      float corr = 1.f;
      if (m_run == -INFINITY) {
        m_run = mt;  // first visible keys of this row: nothing accumulated yet
      } else if (mt > m_run + kPtRescaleLog2) {
        corr = ex2_approx(m_run - mt);
        m_run = mt;
        resc = true;
      }
      float ps = 0.f;
      if (m_run == -INFINITY) {
#pragma unroll
        for (int e = 0; e < kHalfKeys; ++e) sv[e] = 0.f;
      } else if (full) {
#pragma unroll
        for (int e = 0; e < kHalfKeys; ++e) {
          const float pv = ex2_approx(fmaf(sv[e], p.scale_log2, -m_run));
          sv[e] = pv;
          ps += pv;
        }
      } else {
#pragma unroll
        for (int e = 0; e < kHalfKeys; ++e) {
          const float pv = (j0 + own + e > lim) ? 0.f : ex2_approx(fmaf(sv[e], p.scale_log2, -m_run));
          sv[e] = pv;
          ps += pv;
        }
      }
      l_half = l_half * corr + ps;
      const int u = kt & 1;
      // P buffer u was last read by PV(kt - 2).
      if (kt >= 2 && !__all_sync(0xffffffffu, mbar_wait(&o_done[u], (uint32_t)((kt >> 1) - 1) & 1u, p.err, 0x27))) {
        ok = false;
        break;
      }
      // O is rescaled once every PV product so far is in it (PV(kt - 1)); the
      // whole warp joins when any of its rows needs it (corr is 1 for the others).
      if (__any_sync(0xffffffffu, resc)) {
        if (!__all_sync(0xffffffffu, mbar_wait(&o_done[u ^ 1], (uint32_t)((kt - 1) >> 1) & 1u, p.err, 0x2a))) {
          ok = false;
          break;
        }
        tc_fence_after();
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          float ov[16];
          tmem_ld16(tO + lane_off + (uint32_t)(ch * 64 + c * 16), ov);
#pragma unroll
          for (int e = 0; e < 16; ++e) ov[e] *= corr;
          tmem_st16(tO + lane_off + (uint32_t)(ch * 64 + c * 16), ov);
        }
        tmem_st_wait();
      }
      unsigned char* ph = smem + kPtPbuf + u * 2 * kPtP;
#pragma unroll
      for (int c = 0; c < kHalfKeys / 8; ++c) {
        uint32_t hi[4], lo[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float x0 = sv[c * 8 + 2 * e], x1 = sv[c * 8 + 2 * e + 1];
          const float h0 = round_bf16(x0), h1 = round_bf16(x1);
          __nv_bfloat162 hv = __floats2bfloat162_rn(h0, h1), lv = __floats2bfloat162_rn(x0 - h0, x1 - h1);
          hi[e] = *reinterpret_cast<uint32_t*>(&hv);
          lo[e] = *reinterpret_cast<uint32_t*>(&lv);
        }
        const int chunk = ch * (kHalfKeys / 8) + c;  // 8 keys per 16-byte chunk, 8 chunks per 64-key row
        *reinterpret_cast<uint4*>(ph + pt_off(r, chunk, kPtP)) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
        *reinterpret_cast<uint4*>(ph + kPtP + pt_off(r, chunk, kPtP)) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
      }
      if (j0 + kPtKeys > L_blk) {
        // Last tile: zero the V rows past the last visible key; thread (r < 64,
        // half ch) clears dims [64 ch, 64 ch + 64) of key j0 + r.
        const int s = kt % kPtStages;
        if (!__all_sync(0xffffffffu, mbar_wait(&kv_full[s], (uint32_t)(kt / kPtStages) & 1u, p.err, 0x28))) {
          ok = false;
          break;
        }
        if (r < kPtKeys && j0 + r >= L_blk) {
          unsigned char* vt = smem + kPtRing + s * kPtStage + 2 * kPtKvHalf;
#pragma unroll
          for (int c = 0; c < 8; ++c)
            *reinterpret_cast<uint4*>(vt + pt_off(r, ch * 8 + c, kPtKvHalf)) = make_uint4(0, 0, 0, 0);
        }
      }
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(&p_full[u]);
    }
    // Epilogue: O / l as bf16, l = the two halves' sums (added in a fixed order).
    // Every softmax thread reaches the named barrier, on error paths too.
    const int ul = (ntiles - 1) & 1;
    const bool fin = __all_sync(0xffffffffu, ok && ntiles > 0 &&
                                                 mbar_wait(&o_done[ul], (uint32_t)((ntiles - 1) >> 1) & 1u, p.err, 0x29));
    float* lsum = reinterpret_cast<float*>(smem + kPtPbuf);  // P is no longer read once the last PV is done
    if (fin) {
      tc_fence_after();
      lsum[ch * kPtRows + r] = l_half;
    }
    named_bar_sync(1, kPtSoft);
    if (fin) {
      const float l = lsum[r] + lsum[kPtRows + r];
      const float inv = l > 0.f ? 1.f / l : 0.f;
      uint4* op = reinterpret_cast<uint4*>(p.out + ((size_t)(b * p.q_len + i) * p.Hq + hkv * p.G + gq) * 128 + ch * 64);
      // Every lane loads (warp-collective tcgen05.ld); only valid rows store.
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        float ov[16];
        tmem_ld16(tO + lane_off + (uint32_t)(ch * 64 + c * 16), ov);
        uint32_t pk[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          __nv_bfloat162 v2 = __floats2bfloat162_rn(ov[2 * e] * inv, ov[2 * e + 1] * inv);
          pk[e] = *reinterpret_cast<uint32_t*>(&v2);
        }
        if (valid) {
          op[2 * c] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
          op[2 * c + 1] = make_uint4(pk[4], pk[5], pk[6], pk[7]);
        }
      }
    } else if (!ok) {
      s_abort = 1;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(256) : "memory");
  }
}

}  // namespace lsb

namespace lsb_host {

// Causal prefill attention on tcgen05 (see prefill_attention_tc_kernel).
int launch_prefill_attention_tc(const void* q, const void* k_cache, const void* v_cache, const int32_t* cache_pos,
                                int64_t uniform_past, int64_t batch, int64_t q_len, int64_t hq, int64_t hkv,
                                int64_t max_seq, float scale, void* out, cudaStream_t stream) {
  const int64_t kv_rows = batch * hkv * max_seq;
  if (hkv > 65535 || batch > 65535 || kv_rows + kPtKeys > (1ll << 31) || q_len * hq > (1ll << 31))
    return set_error(LS_ERR_UNSUPPORTED_SHAPE, "prefill_attention_tc: %lld sequences x %lld kv heads x %lld positions",
                     (long long)batch, (long long)hkv, (long long)max_seq);
  PtParams p = {};
  p.q = static_cast<const __nv_bfloat16*>(q);
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
  CUtensorMap mk, mv;
  int rc = make_map(&mk, k_cache, kv_rows, 128, kPtKeys);  // boxes of 64 dims x 64 keys
  if (rc) return rc;
  rc = make_map(&mv, v_cache, kv_rows, 128, kPtKeys);
  if (rc) return rc;
  static int configured[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !configured[dev]) {
    cudaError_t e = cudaFuncSetAttribute(prefill_attention_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         kPtSmem);
    if (e != cudaSuccess) return set_error(LS_ERR_CUDA, "prefill_attention_tc attribute: %s", cudaGetErrorString(e));
    configured[dev] = 1;
  }
  const int row_blocks = (int)((p.R + kPtRows - 1) / kPtRows);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)row_blocks, (unsigned)hkv, (unsigned)batch);
  cfg.blockDim = dim3(kPtThreads);
  cfg.dynamicSmemBytes = kPtSmem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, prefill_attention_tc_kernel, mk, mv, p);
  return e == cudaSuccess ? LS_OK : set_error(LS_ERR_CUDA, "prefill_attention_tc launch: %s", cudaGetErrorString(e));
}

}  // namespace lsb_host
