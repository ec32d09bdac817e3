// C ABI of libleanb200.so: argument checking, error reporting and the small
// glue kernels (embedding gather, cursor advance).  The heavy kernels live in
// linear_small_m.cu and attention.cu.
#include <cstdarg>
#include <cstddef>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>

#include "common.cuh"

namespace lsb {
// The device status block: the error flag kernels raise, and the limit of
// their bounded waits (ls_set_wait_limit_ns).  Kernels receive &error.
__device__ DeviceStatus g_device_status = {0, 0, kDefaultWaitNs};

__global__ void embed_gather_kernel(const int64_t* ids, const __nv_bfloat16* embed, int64_t vocab, int hidden,
                                    __nv_bfloat16* out, int* err) {
  grid_dep_wait();
  const int m = blockIdx.x;  // one token per grid column (up to 2^31 - 1 tokens)
  const int64_t id = ids[m];
  const int vec = hidden >> 3;
  if (id < 0 || id >= vocab) {
    if (threadIdx.x == 0 && blockIdx.y == 0) raise_device_error(err, LS_ERR_INVALID_ARGUMENT);
    return;
  }
  for (int v = blockIdx.y * blockDim.x + threadIdx.x; v < vec; v += gridDim.y * blockDim.x)
    reinterpret_cast<uint4*>(out + (size_t)m * hidden)[v] =
        reinterpret_cast<const uint4*>(embed + (size_t)id * hidden)[v];
}

// One CTA per row: y = bf16((x * rsqrt(mean(x^2) + eps)) * w).  Rows whose
// length is a multiple of 8 (16-byte aligned) go through 16-byte vectors, one
// 8-column group per thread (norm_threads); the second pass re-reads x from
// L1.  The sum of squares is taken per thread over its groups, then over the
// lanes of a warp, then over the warps in order -- the order
// residual_norm_splits_kernel uses with the same launch, so the two give
// identical bits.  Launched with programmatic dependent launch: the next
// kernel may start its own prologue (weight prefetch) at once.
constexpr int kNormThreads = 256;     // scalar path
constexpr int kNormMaxThreads = 1024;
static inline int norm_threads(int64_t n, int vec) {
  if (!vec) return kNormThreads;
  const int64_t t = (n / 8 + 31) / 32 * 32;
  return (int)(t < 32 ? 32 : (t > kNormMaxThreads ? kNormMaxThreads : t));
}
__global__ void __launch_bounds__(kNormMaxThreads) rmsnorm_kernel(const __nv_bfloat16* x, int n, const __nv_bfloat16* w,
                                                                  float eps, __nv_bfloat16* out, int vec) {
  grid_dep_launch();
  grid_dep_wait();
  __shared__ float red[kNormMaxThreads / 32];
  const __nv_bfloat16* xr = x + (size_t)blockIdx.x * n;
  __nv_bfloat16* orow = out + (size_t)blockIdx.x * n;
  const int nt = blockDim.x;
  float ss = 0.f;
  if (vec) {
    for (int v = threadIdx.x; v < n / 8; v += nt) {
      float f[8];
      unpack8(ldg16(xr + v * 8), f);
#pragma unroll
      for (int j = 0; j < 8; ++j) ss = fmaf(f[j], f[j], ss);
    }
  } else {
    for (int i = threadIdx.x; i < n; i += nt) {
      const float v = bf16_to_f(xr[i]);
      ss = fmaf(v, v, ss);
    }
  }
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
  for (int i = 0; i < nt / 32; ++i) tot += red[i];
  const float r = rsqrtf(tot / (float)n + eps);
  if (vec) {
    for (int v = threadIdx.x; v < n / 8; v += nt) {
      float f[8], g[8];
      unpack8(ldg16(xr + v * 8), f);
      unpack8(ldg16(w + v * 8), g);
      uint4 o;
      uint32_t* op = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        __nv_bfloat162 pr = __floats2bfloat162_rn((f[2 * j] * r) * g[2 * j], (f[2 * j + 1] * r) * g[2 * j + 1]);
        op[j] = *reinterpret_cast<uint32_t*>(&pr);
      }
      *reinterpret_cast<uint4*>(orow + v * 8) = o;
    }
  } else {
    for (int i = threadIdx.x; i < n; i += nt)
      orow[i] = f_to_bf16((bf16_to_f(xr[i]) * r) * bf16_to_f(w[i]));
  }
}

// Residual add of split fp32 partials, then RMSNorm (one CTA per row):
// h = bf16(residual + bf16(sum_j part[j])), the splits added in order j = 0,
// 1, ... (the order of the GEMM's in-kernel reduction), and, when w is not
// null, y = bf16((h * rsqrt(mean(h^2) + eps)) * w) with the sum of squares
// taken in rmsnorm_kernel's order, so both paths give identical bits.
__global__ void __launch_bounds__(kNormMaxThreads) residual_norm_splits_kernel(const float* part, int splits, int m,
                                                                                 int n, const __nv_bfloat16* residual,
                                                                                 const __nv_bfloat16* w, float eps,
                                                                                 __nv_bfloat16* out_res,
                                                                                 __nv_bfloat16* out_norm) {
  grid_dep_launch();
  grid_dep_wait();
  __shared__ float red[kNormMaxThreads / 32];
  const size_t slab = (size_t)m * n;
  const float* pr = part + (size_t)blockIdx.x * n;
  const __nv_bfloat16* rr = residual + (size_t)blockIdx.x * n;
  __nv_bfloat16* hr = out_res + (size_t)blockIdx.x * n;
  const int nv = n / 8;
  // Thread t owns the 8-column groups t, t + blockDim, ... (one group when the
  // launch gives a thread per group); the first group's h stays in registers.
  uint4 h0 = make_uint4(0, 0, 0, 0);
  float ss = 0.f;
  for (int v = threadIdx.x; v < nv; v += blockDim.x) {
    float4 a0 = __ldcg(reinterpret_cast<const float4*>(pr + v * 8));
    float4 a1 = __ldcg(reinterpret_cast<const float4*>(pr + v * 8 + 4));
    for (int j = 1; j < splits; ++j) {
      const float4 b0 = __ldcg(reinterpret_cast<const float4*>(pr + j * slab + v * 8));
      const float4 b1 = __ldcg(reinterpret_cast<const float4*>(pr + j * slab + v * 8 + 4));
      a0.x += b0.x, a0.y += b0.y, a0.z += b0.z, a0.w += b0.w;
      a1.x += b1.x, a1.y += b1.y, a1.z += b1.z, a1.w += b1.w;
    }
    const float y[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
    float f[8];
    unpack8(ldg16(rr + v * 8), f);
    uint4 o;
    uint32_t* op = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      __nv_bfloat162 pr2 = __floats2bfloat162_rn(f[2 * j] + round_bf16(y[2 * j]), f[2 * j + 1] + round_bf16(y[2 * j + 1]));
      op[j] = *reinterpret_cast<uint32_t*>(&pr2);
    }
    *reinterpret_cast<uint4*>(hr + v * 8) = o;
    if (v == threadIdx.x) h0 = o;
    float h[8];
    unpack8(o, h);
#pragma unroll
    for (int j = 0; j < 8; ++j) ss = fmaf(h[j], h[j], ss);
  }
  if (!out_norm) return;
  // Sum of squares in rmsnorm_kernel's order (same launch shape).
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
  const int nw = (blockDim.x + 31) / 32;
  for (int i = 0; i < nw; ++i) tot += red[i];
  const float r = rsqrtf(tot / (float)n + eps);
  __nv_bfloat16* orow = out_norm + (size_t)blockIdx.x * n;
  for (int v = threadIdx.x; v < nv; v += blockDim.x) {
    float f[8], g[8];
    unpack8(v == threadIdx.x ? h0 : *reinterpret_cast<const uint4*>(hr + v * 8), f);  // own stores above
    unpack8(ldg16(w + v * 8), g);
    uint4 o;
    uint32_t* op = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      __nv_bfloat162 pr2 = __floats2bfloat162_rn((f[2 * j] * r) * g[2 * j], (f[2 * j + 1] * r) * g[2 * j + 1]);
      op[j] = *reinterpret_cast<uint32_t*>(&pr2);
    }
    *reinterpret_cast<uint4*>(orow + v * 8) = o;
  }
}

// SiLU(gate) * up from the split fp32 partials of the gate_up projection run
// as a plain [2I, K] GEMM (LS_EPI_SPLIT_F32): g = bf16(sum_j part[j][b][i]),
// u = bf16(sum_j part[j][b][I + i]), act = bf16(bf16(silu(g)) * u) -- the
// rounding points of the reference's MLP (qwen_explicit.py:932-949) and of
// the GEMM's paired SiLU epilogue.  Four outputs per thread.
__global__ void silu_mul_splits_kernel(const float* part, int splits, int m, int inter, __nv_bfloat16* act) {
  grid_dep_launch();
  grid_dep_wait();
  const int q = inter / 4;
  const size_t slab = (size_t)m * 2 * inter;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < (int64_t)m * q;
       e += (int64_t)gridDim.x * blockDim.x) {
    const int b = (int)(e / q), i = (int)(e - (int64_t)b * q) * 4;
    const float* pg = part + (size_t)b * 2 * inter + i;
    float4 g = __ldcg(reinterpret_cast<const float4*>(pg));
    float4 u = __ldcg(reinterpret_cast<const float4*>(pg + inter));
    for (int j = 1; j < splits; ++j) {
      const float4 g2 = __ldcg(reinterpret_cast<const float4*>(pg + j * slab));
      const float4 u2 = __ldcg(reinterpret_cast<const float4*>(pg + j * slab + inter));
      g.x += g2.x, g.y += g2.y, g.z += g2.z, g.w += g2.w;
      u.x += u2.x, u.y += u2.y, u.z += u2.z, u.w += u2.w;
    }
    const float gv[4] = {g.x, g.y, g.z, g.w}, uv[4] = {u.x, u.y, u.z, u.w};
    float o[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float gr = round_bf16(gv[j]);
      o[j] = round_bf16(gr / (1.0f + expf(-gr))) * round_bf16(uv[j]);
    }
    __nv_bfloat162 lo = __floats2bfloat162_rn(o[0], o[1]), hi = __floats2bfloat162_rn(o[2], o[3]);
    *reinterpret_cast<uint2*>(act + (size_t)b * inter + i) =
        make_uint2(*reinterpret_cast<uint32_t*>(&lo), *reinterpret_cast<uint32_t*>(&hi));
  }
}

// out[i] = sum_j part[j][i] over the splits in order: the local sum of a
// tensor-parallel row-split linear's split partials before an NCCL all-reduce
// (the order the fused peer all-reduce uses, so both give the same bits).
__global__ void sum_splits_kernel(const float* part, int splits, int64_t n, float* out) {
  grid_dep_launch();
  grid_dep_wait();
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    float v = part[i];
    for (int j = 1; j < splits; ++j) v += part[(size_t)j * n + i];
    out[i] = v;
  }
}

// Row argmax over bf16 logits: grid (chunks, m); each CTA reduces one chunk of
// one row, the last CTA of the row reduces the chunk winners.
constexpr int kArgmaxThreads = 256;
__global__ void __launch_bounds__(kArgmaxThreads) argmax_rows_kernel(const __nv_bfloat16* logits, int n, int chunks,
                                                                     float* part_val, int* part_idx,
                                                                     unsigned int* counters, int64_t* out_ids,
                                                                     int64_t id_offset, int out_keys) {
  grid_dep_wait();
  __shared__ float bv[kArgmaxThreads / 32];
  __shared__ int bi[kArgmaxThreads / 32];
  __shared__ bool is_last;
  const int row = blockIdx.y, c = blockIdx.x;
  const int lo = (int)(((long long)n * c) / chunks), hi = (int)(((long long)n * (c + 1)) / chunks);
  const __nv_bfloat16* r = logits + (size_t)row * n;
  float best = -INFINITY;
  int besti = 0x7fffffff;
  for (int i = lo + threadIdx.x; i < hi; i += kArgmaxThreads) {
    const float v = bf16_to_f(r[i]);
    if (v > best || (v == best && i < besti)) { best = v; besti = i; }
  }
  auto reduce = [&]() {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, best, o);
      const int oi = __shfl_xor_sync(0xffffffffu, besti, o);
      if (ov > best || (ov == best && oi < besti)) { best = ov; besti = oi; }
    }
    if ((threadIdx.x & 31) == 0) { bv[threadIdx.x >> 5] = best; bi[threadIdx.x >> 5] = besti; }
    __syncthreads();
    if (threadIdx.x == 0)
      for (int w = 1; w < kArgmaxThreads / 32; ++w)
        if (bv[w] > best || (bv[w] == best && bi[w] < besti)) { best = bv[w]; besti = bi[w]; }
  };
  reduce();
  if (threadIdx.x == 0) {
    part_val[(size_t)row * chunks + c] = best;
    part_idx[(size_t)row * chunks + c] = besti;
    __threadfence();
    is_last = atomicAdd(counters + row, 1u) == (unsigned int)chunks - 1;
  }
  __syncthreads();
  if (!is_last) return;
  __threadfence();
  best = -INFINITY;
  besti = 0x7fffffff;
  for (int i = threadIdx.x; i < chunks; i += kArgmaxThreads) {
    const float v = __ldcg(part_val + (size_t)row * chunks + i);
    const int idx = __ldcg(part_idx + (size_t)row * chunks + i);
    if (v > best || (v == best && idx < besti)) { best = v; besti = idx; }
  }
  __syncthreads();
  reduce();
  if (threadIdx.x == 0) {
    const int64_t id = (int64_t)besti + id_offset;
    out_ids[row] = out_keys ? argmax_key(best, id) : id;
    counters[row] = 0u;
  }
}

// ids[i] = the vocab id carried by the winning key of row i.
__global__ void argmax_keys_to_ids_kernel(const int64_t* keys, int64_t m, int64_t* ids) {
  grid_dep_wait();
  for (int64_t i = threadIdx.x; i < m; i += blockDim.x) ids[i] = argmax_key_id(keys[i]);
}

// out = bf16(residual + bf16(y)) for fp32 y: the residual epilogue applied
// after a tensor-parallel all-reduce of row-split partials.
__global__ void residual_add_kernel(const __nv_bfloat16* residual, const float* y, __nv_bfloat16* out, int64_t n) {
  grid_dep_wait();
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    out[i] = f_to_bf16(bf16_to_f(residual[i]) + round_bf16(y[i]));
}

__global__ void advance_cursors_kernel(int* cache_pos, const int* delta, int batch, int q_len) {
  grid_dep_wait();
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b < batch) cache_pos[b] += delta ? delta[b] : q_len;
}
// Greedy-exact accept / reject of one speculative verify step, per sequence b:
// ids[b] = [current, d1..dk] went through the target, verdict[b][i] is the
// target's greedy token after input position i.  Accept the longest prefix of
// proposals with d(i+1) == verdict[i]; the next current token is the target's
// token after the last accepted position (the correction, or the bonus when
// all k agree); the cursor keeps current + the accepted proposals.
// The draft model consumed current, d1..d(k-1) while proposing; it keeps
// current and the accepted proposals: min(n + 1, k) of its k new positions.
// The tokens the cycle commits (d1..dn, then the next current) are appended to
// a per-sequence output log of capacity out_cap.
__global__ void spec_accept_kernel(int64_t* ids, const int64_t* verdict, int batch, int k, int64_t* next_ids,
                                   int32_t* accepted, int32_t* cache_pos, int32_t* draft_cache_pos,
                                   int64_t* out_tokens, int32_t* out_len, int out_cap) {
  grid_dep_wait();
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= batch) return;
  int64_t* in = ids + (size_t)b * (k + 1);
  const int64_t* v = verdict + (size_t)b * (k + 1);
  int n = 0;
  while (n < k && in[1 + n] == v[n]) ++n;
  const int64_t next = v[n];
  if (next_ids) next_ids[b] = next;
  if (accepted) accepted[b] = n;
  if (cache_pos) cache_pos[b] += n + 1;
  if (draft_cache_pos) draft_cache_pos[b] -= k - min(n + 1, k);
  if (out_tokens && out_len) {
    int len = out_len[b];
    int64_t* o = out_tokens + (size_t)b * out_cap;
    for (int i = 0; i < n && len < out_cap; ++i) o[len++] = in[1 + i];
    if (len < out_cap) o[len++] = next;
    out_len[b] = len;
  }
  in[0] = next;  // the next step's first input token
}
}  // namespace lsb

namespace lsb_host {

static thread_local char g_last_error[512] = "";

int set_error(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return code;
}

int sm_count() {
  static int cached[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) dev = 0;
  if (cached[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    cached[dev] = n;
  }
  return cached[dev];
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int* device_error_ptr() {
  static int* cached[64] = {nullptr};
  static std::mutex mu;
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return nullptr;
  std::lock_guard<std::mutex> lock(mu);
  if (!cached[dev]) {
    void* ptr = nullptr;
    if (cudaGetSymbolAddress(&ptr, lsb::g_device_status) == cudaSuccess)
      cached[dev] = &static_cast<lsb::DeviceStatus*>(ptr)->error;
  }
  return cached[dev];
}

// Defined in the kernel translation units.
int launch_linear(const void* x, int64_t m, int64_t k, const void* norm_w, float eps, const void* w, int64_t n,
                  int epi, const void* residual, void* out, cudaStream_t stream, float* part_val, int* part_idx,
                  unsigned int* counter, int64_t* out_ids, int grid_override);
int lmhead_grid(int64_t vocab, int64_t m);
int launch_lmhead_keys(const void* h, int64_t m, int64_t k, const void* norm_w, float eps, const void* w,
                       int64_t rows, int64_t vocab_offset, int64_t* out_keys, cudaStream_t stream, float* part_val,
                       int* part_idx, unsigned int* counter, int grid);
int launch_qk_norm_rope(const void* qkv, const float* part, int64_t splits, int64_t batch, int64_t q_len, int64_t hq, int64_t hkv, const void* qn,
                        const void* kn, const void* cos, const void* sin, int64_t rope_len, int64_t rope_offset,
                        const int32_t* cache_pos, int64_t uniform_past, void* k_cache, void* v_cache, int64_t max_seq, void* k_out, void* v_out, void* q_out,
                        float eps, cudaStream_t stream);
int attention_workspace_bytes(int64_t batch, int64_t q_len, int64_t hq, int64_t hkv, int64_t max_seq,
                              int64_t* bytes);
int launch_decode_attention(const void* q, const void* k_cache, const void* v_cache, const int32_t* cache_pos,
                            int64_t uniform_past, int64_t batch, int64_t q_len, int64_t hq, int64_t hkv, int64_t max_seq, float scale,
                            void* out, void* workspace, int64_t workspace_bytes, cudaStream_t stream);
int launch_decode_attention_qkv(const void* qkv, int64_t batch, int64_t hq, int64_t hkv, const void* qn,
                                const void* kn, float eps, const void* cos, const void* sin, int64_t rope_len,
                                int64_t rope_offset, const int32_t* cache_pos, int64_t uniform_past, void* k_cache,
                                void* v_cache, int64_t max_seq, float scale, void* out, cudaStream_t stream);

int tc_workspace_bytes(int64_t m, int64_t k, int64_t n_out, int epi, int64_t* bytes);
int tc_split_count(int64_t m, int64_t k, int64_t n_out, int64_t* splits);
int launch_gemm_tc(const void* x, int64_t m, int64_t k, const void* w, int64_t n_out, int epi, const void* residual,
                   void* out, void* workspace, int64_t workspace_bytes, cudaStream_t stream,
                   const void* w_tiled = nullptr);
int64_t tc_tiled_bytes(int64_t n_out, int64_t k, int silu);
int launch_gemm_big(const void* x, int64_t m, int64_t k, const void* w, int64_t n_out, int epi, const void* residual,
                    void* out, cudaStream_t stream);
int launch_tc_tile(const void* w, int64_t n_rows, int64_t k, int silu, void* out, cudaStream_t stream);

}  // namespace lsb_host

using namespace lsb_host;

#define LS_REQUIRE(cond, code, ...) \
  do {                              \
    if (!(cond)) return set_error(code, __VA_ARGS__); \
  } while (0)

extern "C" {

int ls_version(void) { return LS_ABI_VERSION; }

const char* ls_last_error(void) { return g_last_error; }

int ls_sm_count(int* out) {
  LS_REQUIRE(out, LS_ERR_INVALID_ARGUMENT, "ls_sm_count: out is null");
  *out = sm_count();
  return LS_OK;
}

int ls_get_device_error(int* code, int clear) {
  LS_REQUIRE(code, LS_ERR_INVALID_ARGUMENT, "ls_get_device_error: code is null");
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return set_error(LS_ERR_CUDA, "device synchronize: %s", cudaGetErrorString(e));
  int v = 0;
  e = cudaMemcpyFromSymbol(&v, lsb::g_device_status, sizeof(int), offsetof(lsb::DeviceStatus, error));
  if (e != cudaSuccess) return set_error(LS_ERR_CUDA, "read device error: %s", cudaGetErrorString(e));
  *code = v;
  if (clear && v) {
    int zero = 0;
    e = cudaMemcpyToSymbol(lsb::g_device_status, &zero, sizeof(int), offsetof(lsb::DeviceStatus, error));
    if (e != cudaSuccess) return set_error(LS_ERR_CUDA, "clear device error: %s", cudaGetErrorString(e));
  }
  return LS_OK;
}

int ls_set_wait_limit_ns(int64_t ns) {
  LS_REQUIRE(ns >= 1000 && ns <= 60ll * 1000000000ll, LS_ERR_INVALID_ARGUMENT,
             "ls_set_wait_limit_ns: %lld ns outside [1 us, 60 s]", (long long)ns);
  cudaError_t e = cudaDeviceSynchronize();  // no kernel of the old limit still waiting
  const unsigned long long v = (unsigned long long)ns;
  if (e == cudaSuccess)
    e = cudaMemcpyToSymbol(lsb::g_device_status, &v, sizeof(v), offsetof(lsb::DeviceStatus, wait_limit_ns));
  if (e != cudaSuccess) return set_error(LS_ERR_CUDA, "ls_set_wait_limit_ns: %s", cudaGetErrorString(e));
  return LS_OK;
}

int ls_get_wait_limit_ns(int64_t* ns) {
  LS_REQUIRE(ns, LS_ERR_INVALID_ARGUMENT, "ls_get_wait_limit_ns: ns is null");
  unsigned long long v = 0;
  cudaError_t e =
      cudaMemcpyFromSymbol(&v, lsb::g_device_status, sizeof(v), offsetof(lsb::DeviceStatus, wait_limit_ns));
  if (e != cudaSuccess) return set_error(LS_ERR_CUDA, "ls_get_wait_limit_ns: %s", cudaGetErrorString(e));
  *ns = (int64_t)v;
  return LS_OK;
}

int ls_embed_gather(const int64_t* ids, int64_t m, const void* embed, int64_t vocab, int64_t hidden, void* out,
                    ls_stream_t stream) {
  LS_REQUIRE(ids && embed && out, LS_ERR_INVALID_ARGUMENT, "ls_embed_gather: null pointer");
  LS_REQUIRE(m > 0 && m < (1ll << 31) && vocab > 0 && hidden > 0 && hidden <= (1 << 20), LS_ERR_INVALID_ARGUMENT,
             "ls_embed_gather: bad sizes");
  LS_REQUIRE(hidden % 8 == 0 && aligned16(embed) && aligned16(out), LS_ERR_MISALIGNED,
             "ls_embed_gather: hidden must be a multiple of 8 and pointers 16-byte aligned");
  const int vec = (int)(hidden / 8);
  const int threads = 128;
  const int blocks = (vec + threads - 1) / threads;
  lsb::embed_gather_kernel<<<dim3((unsigned)m, blocks), threads, 0, (cudaStream_t)stream>>>(
      ids, static_cast<const __nv_bfloat16*>(embed), vocab, (int)hidden, static_cast<__nv_bfloat16*>(out),
      device_error_ptr());
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? LS_OK : set_error(LS_ERR_CUDA, "embed_gather launch: %s", cudaGetErrorString(e));
}

int ls_linear_bf16(const void* x, int64_t m, int64_t k, const void* norm_w, float eps, const void* w, int64_t n,
                   int epilogue, const void* residual, void* out, ls_stream_t stream) {
  LS_REQUIRE((epilogue >= LS_EPI_STORE && epilogue <= LS_EPI_SILU_MUL) || epilogue == LS_EPI_STORE_F32,
             LS_ERR_INVALID_ARGUMENT, "ls_linear_bf16: unknown epilogue %d", epilogue);
  return launch_linear(x, m, k, norm_w, eps, w, n, epilogue, residual, out, (cudaStream_t)stream, nullptr, nullptr,
                       nullptr, nullptr, 0);
}

int ls_rmsnorm_qkv_rope_kvappend(const void* x, int64_t batch, int64_t q_len, int64_t hidden,
                                 const void* input_norm_w, float eps, const void* qkv_w, int64_t num_heads,
                                 int64_t num_kv_heads, int64_t head_dim, const void* q_norm_w,
                                 const void* k_norm_w, const void* rope_cos, const void* rope_sin,
                                 int64_t rope_len, int64_t rope_offset, const int32_t* cache_pos,
                                 int64_t uniform_past, void* k_cache,
                                 void* v_cache, int64_t max_seq, void* k_out, void* v_out, void* qkv_scratch,
                                 void* q_out, ls_stream_t stream) {
  LS_REQUIRE(x && qkv_w && q_norm_w && k_norm_w && rope_cos && rope_sin && qkv_scratch && q_out,
             LS_ERR_INVALID_ARGUMENT, "ls_rmsnorm_qkv_rope_kvappend: null pointer");
  LS_REQUIRE(head_dim == 128, LS_ERR_UNSUPPORTED_SHAPE, "head_dim=%lld (only 128 is implemented)",
             (long long)head_dim);
  LS_REQUIRE(batch > 0 && q_len > 0 && num_heads > 0 && num_kv_heads > 0 && num_heads % num_kv_heads == 0,
             LS_ERR_INVALID_ARGUMENT, "ls_rmsnorm_qkv_rope_kvappend: bad head counts / sizes");
  LS_REQUIRE(rope_len > 0, LS_ERR_INVALID_ARGUMENT, "rope_len must be positive");
  LS_REQUIRE(rope_offset >= 0, LS_ERR_INVALID_ARGUMENT, "rope_offset must be non-negative");
  LS_REQUIRE(cache_pos || (uniform_past >= rope_offset && uniform_past + q_len <= rope_offset + rope_len),
             LS_ERR_KV_OVERFLOW, "positions %lld..%lld outside the rope table rows %lld..%lld",
             (long long)uniform_past, (long long)(uniform_past + q_len - 1), (long long)rope_offset,
             (long long)(rope_offset + rope_len - 1));
  LS_REQUIRE(cache_pos || !k_cache || uniform_past + q_len <= max_seq, LS_ERR_KV_OVERFLOW,
             "cache overflow: %lld tokens with max_seq=%lld", (long long)(uniform_past + q_len), (long long)max_seq);
  LS_REQUIRE((k_cache == nullptr) == (v_cache == nullptr) && (k_out == nullptr) == (v_out == nullptr),
             LS_ERR_INVALID_ARGUMENT, "k/v cache and k/v out come in pairs");
  LS_REQUIRE(!k_cache || max_seq > 0, LS_ERR_INVALID_ARGUMENT, "max_seq must be positive");
  const int64_t m = batch * q_len;
  LS_REQUIRE(m <= 65535, LS_ERR_UNSUPPORTED_SHAPE, "too many tokens for the small-m path: %lld", (long long)m);
  const int64_t qkv_dim = (num_heads + 2 * num_kv_heads) * head_dim;
  int rc = launch_linear(x, m, hidden, input_norm_w, eps, qkv_w, qkv_dim, 0, nullptr, qkv_scratch,
                         (cudaStream_t)stream, nullptr, nullptr, nullptr, nullptr, 0);
  if (rc) return rc;
  return launch_qk_norm_rope(qkv_scratch, nullptr, 0, batch, q_len, num_heads, num_kv_heads, q_norm_w, k_norm_w, rope_cos,
                             rope_sin, rope_len, rope_offset, cache_pos, uniform_past, k_cache, v_cache, max_seq, k_out, v_out, q_out, eps,
                             (cudaStream_t)stream);
}

int ls_decode_attention_workspace_bytes(int64_t batch, int64_t q_len, int64_t num_heads, int64_t num_kv_heads,
                                        int64_t head_dim, int64_t max_seq, int64_t* bytes) {
  LS_REQUIRE(bytes, LS_ERR_INVALID_ARGUMENT, "bytes is null");
  LS_REQUIRE(head_dim == 128, LS_ERR_UNSUPPORTED_SHAPE, "head_dim=%lld (only 128 is implemented)",
             (long long)head_dim);
  LS_REQUIRE(batch > 0 && q_len > 0 && num_kv_heads > 0 && num_heads % num_kv_heads == 0 && max_seq > 0,
             LS_ERR_INVALID_ARGUMENT, "bad attention sizes");
  return attention_workspace_bytes(batch, q_len, num_heads, num_kv_heads, max_seq, bytes);
}

int ls_decode_attention(const void* q, const void* k_cache, const void* v_cache, const int32_t* cache_pos,
                        int64_t uniform_past, int64_t batch, int64_t q_len, int64_t num_heads, int64_t num_kv_heads,
                        int64_t head_dim, int64_t max_seq, float scale, void* out, void* workspace,
                        int64_t workspace_bytes, ls_stream_t stream) {
  LS_REQUIRE(q && k_cache && v_cache && out, LS_ERR_INVALID_ARGUMENT, "ls_decode_attention: null pointer");
  LS_REQUIRE(cache_pos || (uniform_past >= 0 && uniform_past + q_len <= max_seq), LS_ERR_KV_OVERFLOW,
             "uniform_past=%lld + q_len=%lld beyond max_seq=%lld", (long long)uniform_past, (long long)q_len,
             (long long)max_seq);
  LS_REQUIRE(head_dim == 128, LS_ERR_UNSUPPORTED_SHAPE, "head_dim=%lld (only 128 is implemented)",
             (long long)head_dim);
  LS_REQUIRE(batch > 0 && batch <= 65535 && q_len > 0 && num_kv_heads > 0 && num_heads % num_kv_heads == 0 &&
                 max_seq > 0,
             LS_ERR_INVALID_ARGUMENT, "ls_decode_attention: bad sizes");
  LS_REQUIRE(aligned16(q) && aligned16(k_cache) && aligned16(v_cache) && aligned16(out), LS_ERR_MISALIGNED,
             "ls_decode_attention: pointers must be 16-byte aligned");
  return launch_decode_attention(q, k_cache, v_cache, cache_pos, uniform_past, batch, q_len, num_heads, num_kv_heads, max_seq,
                                 scale, out, workspace, workspace_bytes, (cudaStream_t)stream);
}

int ls_decode_attention_qkv(const void* qkv, int64_t batch, int64_t num_heads, int64_t num_kv_heads,
                            int64_t head_dim, const void* q_norm_w, const void* k_norm_w, float eps,
                            const void* rope_cos, const void* rope_sin, int64_t rope_len, int64_t rope_offset,
                            const int32_t* cache_pos, int64_t uniform_past, void* k_cache, void* v_cache,
                            int64_t max_seq, float scale, void* out, ls_stream_t stream) {
  LS_REQUIRE(qkv && q_norm_w && k_norm_w && rope_cos && rope_sin && k_cache && v_cache && out,
             LS_ERR_INVALID_ARGUMENT, "ls_decode_attention_qkv: null pointer");
  LS_REQUIRE(head_dim == 128, LS_ERR_UNSUPPORTED_SHAPE, "head_dim=%lld (only 128 is implemented)",
             (long long)head_dim);
  LS_REQUIRE(batch > 0 && batch <= 65535 && num_kv_heads > 0 && num_heads % num_kv_heads == 0 &&
                 num_heads / num_kv_heads <= 16 && max_seq > 0 && max_seq < (1ll << 31),
             LS_ERR_INVALID_ARGUMENT, "ls_decode_attention_qkv: bad sizes");
  LS_REQUIRE(rope_len > 0 && rope_offset >= 0, LS_ERR_INVALID_ARGUMENT, "bad rope table");
  LS_REQUIRE(cache_pos || (uniform_past >= rope_offset && uniform_past < rope_offset + rope_len &&
                           uniform_past < max_seq),
             LS_ERR_KV_OVERFLOW, "uniform_past=%lld outside the cache or the rope table", (long long)uniform_past);
  LS_REQUIRE(aligned16(qkv) && aligned16(q_norm_w) && aligned16(k_norm_w) && aligned16(rope_cos) &&
                 aligned16(rope_sin) && aligned16(k_cache) && aligned16(v_cache) && aligned16(out),
             LS_ERR_MISALIGNED, "ls_decode_attention_qkv: pointers must be 16-byte aligned");
  return launch_decode_attention_qkv(qkv, batch, num_heads, num_kv_heads, q_norm_w, k_norm_w, eps, rope_cos, rope_sin,
                                     rope_len, rope_offset, cache_pos, uniform_past, k_cache, v_cache, max_seq, scale,
                                     out, (cudaStream_t)stream);
}

int ls_oproj_residual(const void* attn, int64_t m, int64_t k, const void* o_w, int64_t n, const void* residual,
                      void* out, ls_stream_t stream) {
  LS_REQUIRE(residual, LS_ERR_INVALID_ARGUMENT, "ls_oproj_residual: residual is null");
  return launch_linear(attn, m, k, nullptr, 0.f, o_w, n, LS_EPI_RESIDUAL, residual, out, (cudaStream_t)stream,
                       nullptr, nullptr, nullptr, nullptr, 0);
}

int ls_rmsnorm_gateup_silu(const void* h, int64_t m, int64_t hidden, const void* post_norm_w, float eps,
                           const void* gate_up_w, int64_t intermediate, void* out, ls_stream_t stream) {
  return launch_linear(h, m, hidden, post_norm_w, eps, gate_up_w, 2 * intermediate, LS_EPI_SILU_MUL, nullptr, out,
                       (cudaStream_t)stream, nullptr, nullptr, nullptr, nullptr, 0);
}

int ls_down_residual(const void* act, int64_t m, int64_t intermediate, const void* down_w, int64_t hidden,
                     const void* residual, void* out, ls_stream_t stream) {
  LS_REQUIRE(residual, LS_ERR_INVALID_ARGUMENT, "ls_down_residual: residual is null");
  return launch_linear(act, m, intermediate, nullptr, 0.f, down_w, hidden, LS_EPI_RESIDUAL, residual, out,
                       (cudaStream_t)stream, nullptr, nullptr, nullptr, nullptr, 0);
}

int ls_lmhead_workspace_bytes(int64_t m, int64_t vocab, int64_t* bytes) {
  LS_REQUIRE(bytes && m > 0 && vocab > 0, LS_ERR_INVALID_ARGUMENT, "ls_lmhead_workspace_bytes: bad arguments");
  const int64_t g = lmhead_grid(vocab, m);
  *bytes = 256 + 2 * ((m * g * 4 + 255) / 256) * 256;
  return LS_OK;
}

int ls_lmhead_argmax(const void* h, int64_t m, int64_t hidden, const void* final_norm_w, float eps,
                     const void* lm_head_w, int64_t vocab, int64_t* out_ids, void* workspace,
                     int64_t workspace_bytes, ls_stream_t stream) {
  LS_REQUIRE(out_ids && workspace, LS_ERR_INVALID_ARGUMENT, "ls_lmhead_argmax: null pointer");
  LS_REQUIRE(m >= 1 && m <= 8, LS_ERR_UNSUPPORTED_SHAPE, "ls_lmhead_argmax: m=%lld outside 1..8", (long long)m);
  int64_t need = 0;
  int rc = ls_lmhead_workspace_bytes(m, vocab, &need);
  if (rc) return rc;
  LS_REQUIRE(workspace_bytes >= need, LS_ERR_WORKSPACE, "ls_lmhead_argmax: workspace needs %lld bytes",
             (long long)need);
  const int g = lmhead_grid(vocab, m);
  char* ws = static_cast<char*>(workspace);
  unsigned int* counter = reinterpret_cast<unsigned int*>(ws);
  const int64_t region = ((m * g * 4 + 255) / 256) * 256;
  float* part_val = reinterpret_cast<float*>(ws + 256);
  int* part_idx = reinterpret_cast<int*>(ws + 256 + region);
  return launch_linear(h, m, hidden, final_norm_w, eps, lm_head_w, vocab, 3, nullptr, nullptr,
                       (cudaStream_t)stream, part_val, part_idx, counter, out_ids, g);
}

int ls_gemm_bf16_tcgen05_workspace_bytes(int64_t m, int64_t k, int64_t n, int epilogue, int64_t* bytes) {
  LS_REQUIRE(bytes && m > 0 && m <= 128 && k > 0 && n > 0, LS_ERR_INVALID_ARGUMENT,
             "ls_gemm_bf16_tcgen05_workspace_bytes: bad arguments");
  LS_REQUIRE((epilogue >= LS_EPI_STORE && epilogue <= LS_EPI_SILU_MUL) || epilogue == LS_EPI_STORE_F32 ||
                 epilogue == LS_EPI_SPLIT_F32,
             LS_ERR_INVALID_ARGUMENT, "unknown epilogue %d", epilogue);
  return tc_workspace_bytes(m, k, n, epilogue, bytes);
}

int ls_gemm_bf16_tcgen05_splits(int64_t m, int64_t k, int64_t n, int64_t* splits) {
  LS_REQUIRE(splits && m > 0 && m <= 128 && k > 0 && n > 0, LS_ERR_INVALID_ARGUMENT,
             "ls_gemm_bf16_tcgen05_splits: bad arguments");
  return tc_split_count(m, k, n, splits);
}

int ls_gemm_bf16_tcgen05(const void* x, int64_t m, int64_t k, const void* w, int64_t n, int epilogue,
                         const void* residual, void* out, void* workspace, int64_t workspace_bytes,
                         ls_stream_t stream) {
  LS_REQUIRE((epilogue >= LS_EPI_STORE && epilogue <= LS_EPI_SILU_MUL) || epilogue == LS_EPI_STORE_F32 ||
                 epilogue == LS_EPI_SPLIT_F32,
             LS_ERR_INVALID_ARGUMENT, "unknown epilogue %d", epilogue);
  return launch_gemm_tc(x, m, k, w, n, epilogue, residual, out, workspace, workspace_bytes, (cudaStream_t)stream);
}

int ls_gemm_bf16_tcgen05_big(const void* x, int64_t m, int64_t k, const void* w, int64_t n, int epilogue,
                             const void* residual, void* out, ls_stream_t stream) {
  LS_REQUIRE((epilogue >= LS_EPI_STORE && epilogue <= LS_EPI_SILU_MUL) || epilogue == LS_EPI_STORE_F32,
             LS_ERR_INVALID_ARGUMENT, "unknown epilogue %d", epilogue);
  return launch_gemm_big(x, m, k, w, n, epilogue, residual, out, (cudaStream_t)stream);
}

int ls_gemm_tc_tiled_bytes(int64_t n_rows, int64_t k, int silu, int64_t* bytes) {
  LS_REQUIRE(bytes && n_rows > 0 && k > 0 && (!silu || n_rows % 2 == 0), LS_ERR_INVALID_ARGUMENT,
             "ls_gemm_tc_tiled_bytes: bad arguments");
  *bytes = tc_tiled_bytes(silu ? n_rows / 2 : n_rows, k, silu);
  return LS_OK;
}

int ls_gemm_tc_tile_weight(const void* w, int64_t n_rows, int64_t k, int silu, void* out, ls_stream_t stream) {
  return launch_tc_tile(w, n_rows, k, silu, out, (cudaStream_t)stream);
}

int ls_gemm_bf16_tcgen05_tiled(const void* x, int64_t m, int64_t k, const void* w_tiled, int64_t n, int epilogue,
                               const void* residual, void* out, void* workspace, int64_t workspace_bytes,
                               ls_stream_t stream) {
  LS_REQUIRE(w_tiled, LS_ERR_INVALID_ARGUMENT, "ls_gemm_bf16_tcgen05_tiled: null weights");
  LS_REQUIRE((epilogue >= LS_EPI_STORE && epilogue <= LS_EPI_SILU_MUL) || epilogue == LS_EPI_STORE_F32 ||
                 epilogue == LS_EPI_SPLIT_F32,
             LS_ERR_INVALID_ARGUMENT, "unknown epilogue %d", epilogue);
  return launch_gemm_tc(x, m, k, nullptr, n, epilogue, residual, out, workspace, workspace_bytes,
                        (cudaStream_t)stream, w_tiled);
}

int ls_qk_norm_rope_kvappend(const void* qkv, int64_t batch, int64_t q_len, int64_t num_heads, int64_t num_kv_heads,
                             int64_t head_dim, const void* q_norm_w, const void* k_norm_w, float eps,
                             const void* rope_cos, const void* rope_sin, int64_t rope_len, int64_t rope_offset,
                             const int32_t* cache_pos, int64_t uniform_past, void* k_cache, void* v_cache,
                             int64_t max_seq, void* k_out, void* v_out, void* q_out, ls_stream_t stream) {
  LS_REQUIRE(qkv && q_norm_w && k_norm_w && rope_cos && rope_sin && q_out, LS_ERR_INVALID_ARGUMENT,
             "ls_qk_norm_rope_kvappend: null pointer");
  LS_REQUIRE(head_dim == 128, LS_ERR_UNSUPPORTED_SHAPE, "head_dim=%lld (only 128 is implemented)",
             (long long)head_dim);
  LS_REQUIRE(batch > 0 && q_len > 0 && num_heads > 0 && num_kv_heads > 0 && num_heads % num_kv_heads == 0 &&
                 batch * q_len < (1ll << 31) && (num_heads + num_kv_heads + 3) / 4 <= 65535,
             LS_ERR_INVALID_ARGUMENT, "ls_qk_norm_rope_kvappend: bad sizes");
  LS_REQUIRE((k_cache == nullptr) == (v_cache == nullptr) && (k_out == nullptr) == (v_out == nullptr),
             LS_ERR_INVALID_ARGUMENT, "k/v cache and k/v out come in pairs");
  LS_REQUIRE(rope_len > 0 && rope_offset >= 0, LS_ERR_INVALID_ARGUMENT, "bad rope table");
  LS_REQUIRE(cache_pos || (uniform_past >= rope_offset && uniform_past + q_len <= rope_offset + rope_len),
             LS_ERR_KV_OVERFLOW, "positions outside the rope table");
  LS_REQUIRE(cache_pos || !k_cache || uniform_past + q_len <= max_seq, LS_ERR_KV_OVERFLOW, "cache overflow");
  return launch_qk_norm_rope(qkv, nullptr, 0, batch, q_len, num_heads, num_kv_heads, q_norm_w, k_norm_w, rope_cos, rope_sin,
                             rope_len, rope_offset, cache_pos, uniform_past, k_cache, v_cache, max_seq, k_out, v_out,
                             q_out, eps, (cudaStream_t)stream);
}

int ls_qk_norm_rope_kvappend_splits(const float* qkv_part, int64_t splits, int64_t batch, int64_t q_len,
                                    int64_t num_heads, int64_t num_kv_heads, int64_t head_dim, const void* q_norm_w,
                                    const void* k_norm_w, float eps, const void* rope_cos, const void* rope_sin,
                                    int64_t rope_len, int64_t rope_offset, const int32_t* cache_pos,
                                    int64_t uniform_past, void* k_cache, void* v_cache, int64_t max_seq, void* k_out,
                                    void* v_out, void* q_out, ls_stream_t stream) {
  LS_REQUIRE(qkv_part && splits >= 1 && aligned16(qkv_part) && q_norm_w && k_norm_w && rope_cos && rope_sin && q_out,
             LS_ERR_INVALID_ARGUMENT, "ls_qk_norm_rope_kvappend_splits: null or misaligned pointer");
  LS_REQUIRE(head_dim == 128, LS_ERR_UNSUPPORTED_SHAPE, "head_dim=%lld (only 128 is implemented)",
             (long long)head_dim);
  LS_REQUIRE(batch > 0 && q_len > 0 && num_heads > 0 && num_kv_heads > 0 && num_heads % num_kv_heads == 0 &&
                 batch * q_len < (1ll << 31) && (num_heads + num_kv_heads + 3) / 4 <= 65535,
             LS_ERR_INVALID_ARGUMENT, "ls_qk_norm_rope_kvappend_splits: bad sizes");
  LS_REQUIRE((k_cache == nullptr) == (v_cache == nullptr) && (k_out == nullptr) == (v_out == nullptr),
             LS_ERR_INVALID_ARGUMENT, "k/v cache and k/v out come in pairs");
  LS_REQUIRE(rope_len > 0 && rope_offset >= 0, LS_ERR_INVALID_ARGUMENT, "bad rope table");
  LS_REQUIRE(cache_pos || (uniform_past >= rope_offset && uniform_past + q_len <= rope_offset + rope_len),
             LS_ERR_KV_OVERFLOW, "positions outside the rope table");
  LS_REQUIRE(cache_pos || !k_cache || uniform_past + q_len <= max_seq, LS_ERR_KV_OVERFLOW, "cache overflow");
  return launch_qk_norm_rope(nullptr, qkv_part, splits, batch, q_len, num_heads, num_kv_heads, q_norm_w, k_norm_w,
                             rope_cos, rope_sin, rope_len, rope_offset, cache_pos, uniform_past, k_cache, v_cache,
                             max_seq, k_out, v_out, q_out, eps, (cudaStream_t)stream);
}

static int argmax_chunks(int64_t m, int64_t n) {
  int64_t c = (2 * (int64_t)sm_count() + m - 1) / m;
  const int64_t by_len = (n + 2047) / 2048;
  if (c > by_len) c = by_len;
  if (c < 1) c = 1;
  return (int)c;
}

int ls_argmax_rows_workspace_bytes(int64_t m, int64_t n, int64_t* bytes) {
  LS_REQUIRE(bytes && m > 0 && n > 0, LS_ERR_INVALID_ARGUMENT, "ls_argmax_rows_workspace_bytes: bad arguments");
  const int64_t c = argmax_chunks(m, n);
  *bytes = ((m * 4 + 255) / 256) * 256 + 2 * ((m * c * 4 + 255) / 256) * 256;
  return LS_OK;
}

int ls_argmax_rows(const void* logits, int64_t m, int64_t n, int64_t* out_ids, void* workspace,
                   int64_t workspace_bytes, ls_stream_t stream) {
  LS_REQUIRE(logits && out_ids && workspace, LS_ERR_INVALID_ARGUMENT, "ls_argmax_rows: null pointer");
  LS_REQUIRE(m > 0 && m <= 65535 && n > 0 && n < (1ll << 31), LS_ERR_INVALID_ARGUMENT, "ls_argmax_rows: bad sizes");
  int64_t need = 0;
  int rc = ls_argmax_rows_workspace_bytes(m, n, &need);
  if (rc) return rc;
  LS_REQUIRE(workspace_bytes >= need, LS_ERR_WORKSPACE, "ls_argmax_rows: workspace needs %lld bytes",
             (long long)need);
  const int c = argmax_chunks(m, n);
  char* ws = static_cast<char*>(workspace);
  const int64_t cnt_bytes = ((m * 4 + 255) / 256) * 256, region = ((m * c * 4 + 255) / 256) * 256;
  lsb::argmax_rows_kernel<<<dim3((unsigned)c, (unsigned)m), lsb::kArgmaxThreads, 0, (cudaStream_t)stream>>>(
      static_cast<const __nv_bfloat16*>(logits), (int)n, c, reinterpret_cast<float*>(ws + cnt_bytes),
      reinterpret_cast<int*>(ws + cnt_bytes + region), reinterpret_cast<unsigned int*>(ws), out_ids, 0, 0);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? LS_OK : set_error(LS_ERR_CUDA, "argmax_rows launch: %s", cudaGetErrorString(e));
}

int ls_argmax_rows_keys(const void* logits, int64_t m, int64_t n, int64_t vocab_offset, int64_t* out_keys,
                        void* workspace, int64_t workspace_bytes, ls_stream_t stream) {
  LS_REQUIRE(logits && out_keys && workspace, LS_ERR_INVALID_ARGUMENT, "ls_argmax_rows_keys: null pointer");
  LS_REQUIRE(m > 0 && m <= 65535 && n > 0 && n < (1ll << 31) && vocab_offset >= 0 && vocab_offset + n <= (1ll << 31),
             LS_ERR_INVALID_ARGUMENT, "ls_argmax_rows_keys: bad sizes");
  int64_t need = 0;
  int rc = ls_argmax_rows_workspace_bytes(m, n, &need);
  if (rc) return rc;
  LS_REQUIRE(workspace_bytes >= need, LS_ERR_WORKSPACE, "ls_argmax_rows_keys: workspace needs %lld bytes",
             (long long)need);
  const int c = argmax_chunks(m, n);
  char* ws = static_cast<char*>(workspace);
  const int64_t cnt_bytes = ((m * 4 + 255) / 256) * 256, region = ((m * c * 4 + 255) / 256) * 256;
  lsb::argmax_rows_kernel<<<dim3((unsigned)c, (unsigned)m), lsb::kArgmaxThreads, 0, (cudaStream_t)stream>>>(
      static_cast<const __nv_bfloat16*>(logits), (int)n, c, reinterpret_cast<float*>(ws + cnt_bytes),
      reinterpret_cast<int*>(ws + cnt_bytes + region), reinterpret_cast<unsigned int*>(ws), out_keys, vocab_offset,
      1);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? LS_OK : set_error(LS_ERR_CUDA, "argmax_rows_keys launch: %s", cudaGetErrorString(e));
}

int ls_lmhead_argmax_keys(const void* h, int64_t m, int64_t hidden, const void* final_norm_w, float eps,
                          const void* lm_head_w, int64_t vocab_rows, int64_t vocab_offset, int64_t* out_keys,
                          void* workspace, int64_t workspace_bytes, ls_stream_t stream) {
  LS_REQUIRE(out_keys && workspace, LS_ERR_INVALID_ARGUMENT, "ls_lmhead_argmax_keys: null pointer");
  LS_REQUIRE(m >= 1 && m <= 8, LS_ERR_UNSUPPORTED_SHAPE, "ls_lmhead_argmax_keys: m=%lld outside 1..8", (long long)m);
  LS_REQUIRE(vocab_offset >= 0 && vocab_offset + vocab_rows <= (1ll << 31), LS_ERR_INVALID_ARGUMENT,
             "ls_lmhead_argmax_keys: vocab shard beyond 2^31");
  int64_t need = 0;
  int rc = ls_lmhead_workspace_bytes(m, vocab_rows, &need);
  if (rc) return rc;
  LS_REQUIRE(workspace_bytes >= need, LS_ERR_WORKSPACE, "ls_lmhead_argmax_keys: workspace needs %lld bytes",
             (long long)need);
  const int g = lmhead_grid(vocab_rows, m);
  char* ws = static_cast<char*>(workspace);
  const int64_t region = ((m * g * 4 + 255) / 256) * 256;
  return launch_lmhead_keys(h, m, hidden, final_norm_w, eps, lm_head_w, vocab_rows, vocab_offset, out_keys,
                            (cudaStream_t)stream, reinterpret_cast<float*>(ws + 256),
                            reinterpret_cast<int*>(ws + 256 + region), reinterpret_cast<unsigned int*>(ws), g);
}

int ls_argmax_keys_to_ids(const int64_t* keys, int64_t m, int64_t* out_ids, ls_stream_t stream) {
  LS_REQUIRE(keys && out_ids && m > 0 && m <= 65535, LS_ERR_INVALID_ARGUMENT, "ls_argmax_keys_to_ids: bad arguments");
  lsb::argmax_keys_to_ids_kernel<<<1, 256, 0, (cudaStream_t)stream>>>(keys, m, out_ids);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? LS_OK : set_error(LS_ERR_CUDA, "argmax_keys_to_ids launch: %s", cudaGetErrorString(e));
}



int ls_residual_add_f32(const void* residual, const float* y, int64_t n, void* out, ls_stream_t stream) {
  LS_REQUIRE(residual && y && out && n > 0, LS_ERR_INVALID_ARGUMENT, "ls_residual_add_f32: bad arguments");
  const int threads = 256;
  int64_t blocks = (n + threads - 1) / threads;
  if (blocks > 4 * sm_count()) blocks = 4 * sm_count();
  lsb::residual_add_kernel<<<(unsigned)blocks, threads, 0, (cudaStream_t)stream>>>(
      static_cast<const __nv_bfloat16*>(residual), y, static_cast<__nv_bfloat16*>(out), n);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? LS_OK : set_error(LS_ERR_CUDA, "residual_add launch: %s", cudaGetErrorString(e));
}

int ls_rmsnorm(const void* x, int64_t m, int64_t n, const void* w, float eps, void* out, ls_stream_t stream) {
  LS_REQUIRE(x && w && out, LS_ERR_INVALID_ARGUMENT, "ls_rmsnorm: null pointer");
  LS_REQUIRE(m > 0 && m < (1ll << 31) && n > 0 && n <= (1 << 20), LS_ERR_INVALID_ARGUMENT, "ls_rmsnorm: bad sizes");
  const int vec = (n % 8 == 0) && aligned16(x) && aligned16(w) && aligned16(out) ? 1 : 0;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)m);
  cfg.blockDim = dim3(lsb::norm_threads(n, vec));
  cfg.stream = (cudaStream_t)stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, lsb::rmsnorm_kernel, static_cast<const __nv_bfloat16*>(x), (int)n,
                                     static_cast<const __nv_bfloat16*>(w), eps, static_cast<__nv_bfloat16*>(out), vec);
  return e == cudaSuccess ? LS_OK : set_error(LS_ERR_CUDA, "rmsnorm launch: %s", cudaGetErrorString(e));
}

int ls_residual_rmsnorm_splits(const float* part, int64_t splits, int64_t m, int64_t n, const void* residual,
                               const void* norm_w, float eps, void* out_residual, void* out_norm,
                               ls_stream_t stream) {
  LS_REQUIRE(part && residual && out_residual && (norm_w == nullptr) == (out_norm == nullptr),
             LS_ERR_INVALID_ARGUMENT, "ls_residual_rmsnorm_splits: null pointer");
  LS_REQUIRE(splits >= 1 && m > 0 && m < (1ll << 31) && n > 0 && n <= (1 << 20) && splits * m * n < (1ll << 40),
             LS_ERR_INVALID_ARGUMENT, "ls_residual_rmsnorm_splits: bad sizes");
  LS_REQUIRE(n % 8 == 0 && aligned16(part) && aligned16(residual) && aligned16(out_residual) &&
                 (!norm_w || (aligned16(norm_w) && aligned16(out_norm))),
             LS_ERR_MISALIGNED, "ls_residual_rmsnorm_splits: rows must be multiples of 8 on 16-byte boundaries");
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)m);
  cfg.blockDim = dim3(lsb::norm_threads(n, 1));
  cfg.stream = (cudaStream_t)stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, lsb::residual_norm_splits_kernel, part, (int)splits, (int)m, (int)n,
                                     static_cast<const __nv_bfloat16*>(residual),
                                     static_cast<const __nv_bfloat16*>(norm_w), eps,
                                     static_cast<__nv_bfloat16*>(out_residual), static_cast<__nv_bfloat16*>(out_norm));
  return e == cudaSuccess ? LS_OK : set_error(LS_ERR_CUDA, "residual_norm_splits launch: %s", cudaGetErrorString(e));
}

int ls_silu_mul_splits(const float* part, int64_t splits, int64_t m, int64_t intermediate, void* act,
                       ls_stream_t stream) {
  LS_REQUIRE(part && act, LS_ERR_INVALID_ARGUMENT, "ls_silu_mul_splits: null pointer");
  LS_REQUIRE(splits >= 1 && m > 0 && intermediate > 0 && m * intermediate < (1ll << 40), LS_ERR_INVALID_ARGUMENT,
             "ls_silu_mul_splits: bad sizes");
  LS_REQUIRE(intermediate % 4 == 0 && aligned16(part) && aligned16(act), LS_ERR_MISALIGNED,
             "ls_silu_mul_splits: intermediate must be a multiple of 4, pointers 16-byte aligned");
  const int64_t items = m * intermediate / 4;
  const int threads = 256;
  int64_t blocks = (items + threads - 1) / threads;
  if (blocks > 4 * (int64_t)sm_count()) blocks = 4 * (int64_t)sm_count();
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)blocks);
  cfg.blockDim = dim3(threads);
  cfg.stream = (cudaStream_t)stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, lsb::silu_mul_splits_kernel, part, (int)splits, (int)m, (int)intermediate,
                                     static_cast<__nv_bfloat16*>(act));
  return e == cudaSuccess ? LS_OK : set_error(LS_ERR_CUDA, "silu_mul_splits launch: %s", cudaGetErrorString(e));
}

int ls_sum_splits_f32(const float* part, int64_t splits, int64_t n, float* out, ls_stream_t stream) {
  LS_REQUIRE(part && out && splits >= 1 && n > 0 && n < (1ll << 40), LS_ERR_INVALID_ARGUMENT,
             "ls_sum_splits_f32: bad arguments");
  const int threads = 256;
  int64_t blocks = (n + threads - 1) / threads;
  if (blocks > 4 * (int64_t)sm_count()) blocks = 4 * (int64_t)sm_count();
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)blocks);
  cfg.blockDim = dim3(threads);
  cfg.stream = (cudaStream_t)stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, lsb::sum_splits_kernel, part, (int)splits, n, out);
  return e == cudaSuccess ? LS_OK : set_error(LS_ERR_CUDA, "sum_splits launch: %s", cudaGetErrorString(e));
}

int ls_advance_cursors(int32_t* cache_pos, const int32_t* delta, int64_t batch, int64_t q_len, ls_stream_t stream) {
  LS_REQUIRE(cache_pos && batch > 0, LS_ERR_INVALID_ARGUMENT, "ls_advance_cursors: bad arguments");
  const int threads = 128;
  lsb::advance_cursors_kernel<<<(unsigned)((batch + threads - 1) / threads), threads, 0, (cudaStream_t)stream>>>(
      cache_pos, delta, (int)batch, (int)q_len);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? LS_OK : set_error(LS_ERR_CUDA, "advance_cursors launch: %s", cudaGetErrorString(e));
}

int ls_spec_accept(int64_t* ids, const int64_t* verdict, int64_t batch, int64_t k, int64_t* next_ids,
                   int32_t* accepted, int32_t* cache_pos, int32_t* draft_cache_pos, int64_t* out_tokens,
                   int32_t* out_len, int64_t out_cap, ls_stream_t stream) {
  LS_REQUIRE(ids && verdict && batch > 0 && batch <= (1 << 20) && k >= 1 && k <= 64, LS_ERR_INVALID_ARGUMENT,
             "ls_spec_accept: bad arguments");
  LS_REQUIRE(!(out_tokens || out_len) || (out_tokens && out_len && out_cap > 0 && out_cap < (1 << 30)),
             LS_ERR_INVALID_ARGUMENT, "ls_spec_accept: output log needs out_tokens, out_len and out_cap > 0");
  const int threads = 128;
  lsb::spec_accept_kernel<<<(unsigned)((batch + threads - 1) / threads), threads, 0, (cudaStream_t)stream>>>(
      ids, verdict, (int)batch, (int)k, next_ids, accepted, cache_pos, draft_cache_pos, out_tokens, out_len,
      (int)out_cap);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? LS_OK : set_error(LS_ERR_CUDA, "spec_accept launch: %s", cudaGetErrorString(e));
}

}  // extern "C"
