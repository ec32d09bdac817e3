// Shared device helpers for the leanstack_b200 kernels (sm_100a only).
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>
#include <cstring>

#include "../../include/leanb200.h"

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "leanstack_b200 kernels are written for sm_100a (B200) only"
#endif

namespace lsb {

// ---------------------------------------------------------------------------
// bf16 <-> fp32.  A bf16 is the top half of an fp32, so widening is a shift.
// Narrowing uses the CUDA intrinsic (round to nearest even), the same rounding
// torch applies when an fp32 intermediate is stored as bf16.
// ---------------------------------------------------------------------------
__device__ __forceinline__ float bf16_lo(uint32_t packed) { return __uint_as_float(packed << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t packed) { return __uint_as_float(packed & 0xFFFF0000u); }
__device__ __forceinline__ float bf16_to_f(__nv_bfloat16 v) { return __bfloat162float(v); }
__device__ __forceinline__ __nv_bfloat16 f_to_bf16(float v) { return __float2bfloat16_rn(v); }
// Round an fp32 to the nearest bf16 and return it widened again: models one
// bf16 store of a torch intermediate.
__device__ __forceinline__ float round_bf16(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }

__device__ __forceinline__ void unpack8(const uint4& u, float f[8]) {
  f[0] = bf16_lo(u.x); f[1] = bf16_hi(u.x);
  f[2] = bf16_lo(u.y); f[3] = bf16_hi(u.y);
  f[4] = bf16_lo(u.z); f[5] = bf16_hi(u.z);
  f[6] = bf16_lo(u.w); f[7] = bf16_hi(u.w);
}

__device__ __forceinline__ float dot8(const uint4& w, const uint4& x, float acc) {
  acc = fmaf(bf16_lo(w.x), bf16_lo(x.x), acc);
  acc = fmaf(bf16_hi(w.x), bf16_hi(x.x), acc);
  acc = fmaf(bf16_lo(w.y), bf16_lo(x.y), acc);
  acc = fmaf(bf16_hi(w.y), bf16_hi(x.y), acc);
  acc = fmaf(bf16_lo(w.z), bf16_lo(x.z), acc);
  acc = fmaf(bf16_hi(w.z), bf16_hi(x.z), acc);
  acc = fmaf(bf16_lo(w.w), bf16_lo(x.w), acc);
  acc = fmaf(bf16_hi(w.w), bf16_hi(x.w), acc);
  return acc;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Streaming 16-byte load that does not allocate in L1 (weights are read once).
__device__ __forceinline__ uint4 ldg_stream(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p));
  return r;
}

__device__ __forceinline__ uint4 ldg16(const void* p) { return *reinterpret_cast<const uint4*>(p); }

// Bulk prefetch of [p, p + bytes) into L2 (p and bytes multiples of 16).  Used
// by a kernel launched early under PDL to pull its first weight bytes in while
// the previous kernel finishes: weights never depend on the previous kernel.
__device__ __forceinline__ void prefetch_l2(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// ---------------------------------------------------------------------------
// Programmatic dependent launch.  A kernel launched with the PDL attribute may
// start before its predecessor finishes; it must call grid_dep_wait() before
// reading anything the predecessor wrote.  grid_dep_launch() lets the next
// kernel in the stream begin its own prologue.  Both are no-ops when the
// launch had no PDL attribute.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void grid_dep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void grid_dep_launch() { asm volatile("griddepcontrol.launch_dependents;" :::); }

// Device-side error flag: kernels record the first failure code there (for
// example a KV position beyond the arena) and skip the offending access.  The
// flag is one int per device owned by capi.cu; kernels receive its address.
__device__ __forceinline__ void raise_device_error(int* flag, int code) {
  if (flag) atomicCAS(flag, 0, code);
}

// ---------------------------------------------------------------------------
// Bounded waits.  Every spin in the kernels gives up after the device's wait
// limit (2 s unless ls_set_wait_limit_ns changed it), records LS_ERR_TIMEOUT
// (with the wait site in the bits above the low byte) and reports failure so
// the kernel can drain and return.  The limit sits in the device status block
// right after the error flag, so a kernel reads it through the `err` pointer
// it already receives.
// ---------------------------------------------------------------------------
struct DeviceStatus {
  int error;                      // first LS_ERR_* raised on the device (0: none)
  int pad;
  unsigned long long wait_limit_ns;
};
constexpr unsigned long long kDefaultWaitNs = 2000000000ull;

__device__ __forceinline__ unsigned long long global_timer_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ unsigned long long wait_limit_ns(const int* err) {
  return err ? reinterpret_cast<const volatile DeviceStatus*>(err)->wait_limit_ns : kDefaultWaitNs;
}
// Bounded-wait clock: start() once, then expired() per spin iteration.
struct WaitClock {
  unsigned long long t0, limit;
  __device__ __forceinline__ explicit WaitClock(const int* err) : t0(global_timer_ns()), limit(wait_limit_ns(err)) {}
  __device__ __forceinline__ bool expired() const { return global_timer_ns() - t0 > limit; }
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_fence_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait for the phase with the given parity to complete.  On timeout
// the error code is LS_ERR_TIMEOUT in the low byte and the wait site above it.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* err, int site = 0) {
  if (mbar_try_wait(bar, parity)) return true;
  const WaitClock clk(err);
  while (!mbar_try_wait(bar, parity)) {
    if (clk.expired()) {
      raise_device_error(err, 7 /* LS_ERR_TIMEOUT */ | (site << 8));
      return false;
    }
  }
  return true;
}
// Contiguous global -> shared bulk copy completing on `bar` (16-byte aligned, size % 16 == 0).
__device__ __forceinline__ void bulk_g2s(void* smem_dst, const void* gmem_src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(smem_dst)),
      "l"(gmem_src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ void named_bar_sync(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// q/k RMSNorm of one 128-dim head held by a warp (lane l holds dims 4l..4l+3
// as packed bf16), then the NeoX-half rotary embedding, with the reference's
// bf16 rounding points (src/leanstack/runtime/qwen_explicit.py:733-806):
// n = bf16((x * r) * w), r = rsqrt(mean(x^2) + eps); each RoPE product and the
// sum / difference round to bf16.  w_u: norm weight of the lane's dims; c_u /
// s_u: the cos / sin row at the lane's rotary index (dims mod 64).  Every
// kernel that forms q or k goes through this function, so they agree bit for bit.
__device__ __forceinline__ uint2 head_norm_rope(uint2 raw_u, uint2 w_u, uint2 c_u, uint2 s_u, float eps, int lane) {
  const float raw[4] = {bf16_lo(raw_u.x), bf16_hi(raw_u.x), bf16_lo(raw_u.y), bf16_hi(raw_u.y)};
  float ss = raw[0] * raw[0] + raw[1] * raw[1] + raw[2] * raw[2] + raw[3] * raw[3];
  ss = warp_sum(ss);
  const float r = rsqrtf(ss / 128.f + eps);
  const float wv[4] = {bf16_lo(w_u.x), bf16_hi(w_u.x), bf16_lo(w_u.y), bf16_hi(w_u.y)};
  float n[4], other[4], o[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) n[j] = round_bf16((raw[j] * r) * wv[j]);
#pragma unroll
  for (int j = 0; j < 4; ++j) other[j] = __shfl_xor_sync(0xffffffffu, n[j], 16);
  const bool first_half = lane < 16;
  const float c[4] = {bf16_lo(c_u.x), bf16_hi(c_u.x), bf16_lo(c_u.y), bf16_hi(c_u.y)};
  const float s[4] = {bf16_lo(s_u.x), bf16_hi(s_u.x), bf16_lo(s_u.y), bf16_hi(s_u.y)};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    if (first_half) o[j] = round_bf16(round_bf16(n[j] * c[j]) - round_bf16(other[j] * s[j]));
    else o[j] = round_bf16(round_bf16(n[j] * c[j]) + round_bf16(other[j] * s[j]));
  }
  __nv_bfloat162 lo2 = __floats2bfloat162_rn(o[0], o[1]);
  __nv_bfloat162 hi2 = __floats2bfloat162_rn(o[2], o[3]);
  return make_uint2(*reinterpret_cast<uint32_t*>(&lo2), *reinterpret_cast<uint32_t*>(&hi2));
}



// Orderable 64-bit key of a (logit, vocab id) candidate: a signed max over
// keys picks the largest logit and, among equal logits, the lowest id, so the
// winners of vocab shards on different GPUs combine with one MAX all-reduce.
// -0 is folded into +0 so that the two compare equal, as floats do.
__host__ __device__ __forceinline__ int64_t argmax_key(float v, int64_t id) {
  v += 0.0f;
  uint32_t u;
  memcpy(&u, &v, 4);
  u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
  const uint64_t k = ((uint64_t)u << 32) | (uint64_t)(0xFFFFFFFFu - (uint32_t)id);
  return (int64_t)(k ^ 0x8000000000000000ull);
}
__host__ __device__ __forceinline__ int64_t argmax_key_id(int64_t key) {
  return (int64_t)(0xFFFFFFFFu - (uint32_t)((uint64_t)key & 0xFFFFFFFFull));
}

// ---- fused tensor-parallel all-reduce: exchange region layout ----
struct P2PExchange {
  unsigned char* peer[LS_MAX_TP_RANKS];
  int rank, world, max_ctas, max_rows;
  int width;
  unsigned long long* trace;  // optional: [max_ctas][4] timestamps (main loop done, pushed, flags seen, end)
};
__host__ __device__ __forceinline__ size_t p2p_ctr_offset(int max_ctas) {
  return ((size_t)LS_MAX_TP_RANKS * max_ctas * 4 + 255) / 256 * 256;
}
__host__ __device__ __forceinline__ size_t p2p_recv_offset(int max_ctas) {
  return p2p_ctr_offset(max_ctas) + ((size_t)max_ctas * 4 + 255) / 256 * 256;
}
// Receive area: 2 slots x [LS_MAX_TP_RANKS][max_rows][width] pairs {fp32 bits, call number}.
__host__ __device__ __forceinline__ size_t p2p_region_bytes(int max_ctas, int max_rows, int width) {
  return p2p_recv_offset(max_ctas) + (size_t)2 * LS_MAX_TP_RANKS * max_rows * width * 8;
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
// One 8-byte store / load that peers see whole: the value travels with its call number.
__device__ __forceinline__ void st_pair_sys(uint2* p, uint32_t a, uint32_t b) {
  asm volatile("st.relaxed.sys.global.v2.u32 [%0], {%1, %2};" ::"l"(p), "r"(a), "r"(b) : "memory");
}
__device__ __forceinline__ uint2 ld_pair_sys(const uint2* p) {
  uint2 v;
  asm volatile("ld.relaxed.sys.global.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(p) : "memory");
  return v;
}
}  // namespace lsb

// Host-side helpers shared by the C-ABI translation units.
namespace lsb_host {
int set_error(int code, const char* fmt, ...);
int check_launch(const char* what);
int sm_count();
bool aligned16(const void* p);
int* device_error_ptr();
}  // namespace lsb_host
