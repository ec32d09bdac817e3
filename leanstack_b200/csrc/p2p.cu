// Set-up of the fused tensor-parallel all-reduce: exchange regions in device
// memory, shared between the ranks' processes through CUDA IPC handles (plain
// peer mappings over NVLink; no multicast objects), the C entry point of the
// row-split linear whose epilogue performs the all-reduce (linear_small_m.cu,
// EPI_AR_RESIDUAL), and the standalone one-shot all-reduce + residual of the
// fp32 partials that the tensor-core row-split linears write.
#include "common.cuh"

namespace lsb_host {
int launch_linear_allreduce(const void* x, int64_t m, int64_t k, const void* w, int64_t n, const void* residual,
                            void* out, const lsb::P2PExchange* ex, cudaStream_t stream);
}  // namespace lsb_host

#ifdef LEANB200_PROFILING
namespace lsb {
// Flag ping-pong between two ranks through their exchange regions: rank 0
// writes i into rank 1's flag word and waits for i in its own, rank 1 answers.
// One thread; every wait gives up after kDefaultWaitNs.  times[0] = total ns,
// times[1] = 1 if a wait gave up.
__global__ void p2p_pingpong_kernel(uint32_t* mine, uint32_t* peer, int rank, int iters, unsigned long long* times) {
  const unsigned long long t0 = global_timer_ns();
  int failed = 0;
  for (int i = 1; i <= iters && !failed; ++i) {
    if (rank == 0) st_release_sys(peer, (uint32_t)i);
    const unsigned long long w0 = global_timer_ns();
    while (ld_acquire_sys(mine) < (uint32_t)i) {
      if (global_timer_ns() - w0 > kDefaultWaitNs) { failed = 1; break; }
    }
    if (rank == 1) st_release_sys(peer, (uint32_t)i);
  }
  times[0] = global_timer_ns() - t0;
  times[1] = failed;
}
}  // namespace lsb
#endif  // LEANB200_PROFILING

namespace lsb {

// One-shot all-reduce of a row-split linear's fp32 partials, fused with the
// residual epilogue: out = bf16(residual + bf16(sum over ranks in rank order)).
// Every element travels to every rank together with the call number in one
// 8-byte store; a reader polls its elements until all ranks' call numbers
// match (no flag, fence or barrier between push and sum).  The grid is fixed
// (kArGrid CTAs, each with its own call counter in the region), so every
// CTA's counter equals the number of calls made so far on every rank, and the
// element -> CTA map may change with m without any reader seeing a stale
// element of an older call as current.
constexpr int kArThreads = 256;
constexpr int kArGrid = 128;

// part holds `splits` slabs of M x N (the split partials of the tcgen05
// GEMM's LS_EPI_SPLIT_F32 form, added in slab order before the exchange), or
// one slab.
__global__ void __launch_bounds__(kArThreads) allreduce_residual_kernel(const float* part, int splits,
                                                                       const __nv_bfloat16* residual,
                                                                       __nv_bfloat16* out, int M, int N,
                                                                       P2PExchange ex, int* err) {
  __shared__ uint32_t s_epoch;
  __shared__ int s_abort;
  const int tid = threadIdx.x;
  if (tid == 0) {
    uint32_t* ctr = reinterpret_cast<uint32_t*>(ex.peer[ex.rank] + p2p_ctr_offset(ex.max_ctas)) + blockIdx.x;
    s_epoch = *ctr + 1u;
    *ctr = s_epoch;
    s_abort = 0;
  }
  grid_dep_wait();  // the partials come from the previous kernel
  __syncthreads();
  grid_dep_launch();
  const uint32_t epoch = s_epoch;
  const size_t slot_base = (size_t)(epoch & 1u) * LS_MAX_TP_RANKS * ex.max_rows * ex.width;
  const size_t recv_off = p2p_recv_offset(ex.max_ctas);
  const int total = M * N;
  const int stride = gridDim.x * kArThreads;
  for (int i = blockIdx.x * kArThreads + tid; i < total; i += stride) {
    const int m = i / N, n = i - m * N;
    float v = part[i];
    for (int j = 1; j < splits; ++j) v += part[(size_t)j * total + i];
    const size_t off = slot_base + ((size_t)ex.rank * ex.max_rows + m) * ex.width + n;
    for (int q = 0; q < ex.world; ++q)
      st_pair_sys(reinterpret_cast<uint2*>(ex.peer[q] + recv_off) + off, __float_as_uint(v), epoch);
  }
  const uint2* recv = reinterpret_cast<const uint2*>(ex.peer[ex.rank] + recv_off) + slot_base;
  const WaitClock clk(err);
  for (int i = blockIdx.x * kArThreads + tid; i < total; i += stride) {
    const int m = i / N, n = i - m * N;
    float y = 0.f;
    for (int q = 0; q < ex.world; ++q) {
      const uint2* src = recv + ((size_t)q * ex.max_rows + m) * ex.width + n;
      uint2 v = ld_pair_sys(src);
      while (v.y != epoch) {  // bounded: one limit per CTA, then every thread gives up
        if (*reinterpret_cast<volatile int*>(&s_abort)) break;
        if (clk.expired()) {
          raise_device_error(err, LS_ERR_TIMEOUT | (0x31 << 8));
          s_abort = 1;
          break;
        }
        v = ld_pair_sys(src);
      }
      y += __uint_as_float(v.x);
    }
    out[i] = f_to_bf16(bf16_to_f(residual[i]) + round_bf16(y));
  }
}

}  // namespace lsb

using namespace lsb_host;

namespace {
int to_exchange(const ls_p2p_exchange* ex, int64_t n, const char* who, lsb::P2PExchange* e) {
  if (!ex) return set_error(LS_ERR_INVALID_ARGUMENT, "%s: exchange is null", who);
  if (ex->world < 1 || ex->world > LS_MAX_TP_RANKS || ex->rank < 0 || ex->rank >= ex->world || ex->max_ctas < 1 ||
      ex->max_rows < 1 || ex->width != n)
    return set_error(LS_ERR_INVALID_ARGUMENT, "%s: bad exchange description", who);
  *e = {};
  for (int q = 0; q < ex->world; ++q) {
    if (!ex->peer[q] || !aligned16(ex->peer[q]))
      return set_error(LS_ERR_INVALID_ARGUMENT, "%s: region of rank %d missing", who, q);
    e->peer[q] = static_cast<unsigned char*>(ex->peer[q]);
  }
  e->rank = ex->rank;
  e->world = ex->world;
  e->max_ctas = ex->max_ctas;
  e->max_rows = ex->max_rows;
  e->width = (int)ex->width;
  e->trace = ex->trace;
  return LS_OK;
}
}  // namespace

extern "C" {

#ifdef LEANB200_PROFILING
int ls_p2p_pingpong(void* my_region, void* peer_region, int rank, int iters, unsigned long long* times_dev,
                    ls_stream_t stream) {
  if (!my_region || !peer_region || !times_dev || (rank != 0 && rank != 1) || iters < 1 || iters > (1 << 20))
    return set_error(LS_ERR_INVALID_ARGUMENT, "ls_p2p_pingpong: bad arguments");
  lsb::p2p_pingpong_kernel<<<1, 1, 0, (cudaStream_t)stream>>>(static_cast<uint32_t*>(my_region),
                                                             static_cast<uint32_t*>(peer_region), rank, iters,
                                                             times_dev);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? LS_OK : set_error(LS_ERR_CUDA, "p2p_pingpong launch: %s", cudaGetErrorString(e));
}
#endif  // LEANB200_PROFILING

int ls_p2p_region_bytes(int64_t max_rows, int64_t width, int64_t max_ctas, int64_t* bytes) {
  if (!bytes || max_rows < 1 || max_rows > 128 || width < 1 || width > (1 << 20) || max_ctas < 1 ||
      max_ctas > 4096)
    return set_error(LS_ERR_INVALID_ARGUMENT, "ls_p2p_region_bytes: bad arguments");
  *bytes = (int64_t)lsb::p2p_region_bytes((int)max_ctas, (int)max_rows, (int)width);
  return LS_OK;
}

int ls_p2p_alloc(int64_t bytes, void** region) {
  if (!region || bytes <= 0) return set_error(LS_ERR_INVALID_ARGUMENT, "ls_p2p_alloc: bad arguments");
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, (size_t)bytes);
  if (e == cudaSuccess) e = cudaMemset(p, 0, (size_t)bytes);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e != cudaSuccess) {
    if (p) cudaFree(p);
    return set_error(LS_ERR_CUDA, "ls_p2p_alloc: %s", cudaGetErrorString(e));
  }
  *region = p;
  return LS_OK;
}

int ls_p2p_free(void* region) {
  if (!region) return LS_OK;
  cudaError_t e = cudaFree(region);
  return e == cudaSuccess ? LS_OK : set_error(LS_ERR_CUDA, "ls_p2p_free: %s", cudaGetErrorString(e));
}

int ls_ipc_get_handle(void* region, void* handle64) {
  if (!region || !handle64) return set_error(LS_ERR_INVALID_ARGUMENT, "ls_ipc_get_handle: null pointer");
  static_assert(sizeof(cudaIpcMemHandle_t) == 64, "IPC handle size");
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, region);
  if (e != cudaSuccess) return set_error(LS_ERR_CUDA, "cudaIpcGetMemHandle: %s", cudaGetErrorString(e));
  memcpy(handle64, &h, sizeof(h));
  return LS_OK;
}

int ls_ipc_open(const void* handle64, void** region) {
  if (!handle64 || !region) return set_error(LS_ERR_INVALID_ARGUMENT, "ls_ipc_open: null pointer");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle64, sizeof(h));
  void* p = nullptr;
  cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return set_error(LS_ERR_CUDA, "cudaIpcOpenMemHandle: %s", cudaGetErrorString(e));
  *region = p;
  return LS_OK;
}

int ls_ipc_close(void* region) {
  if (!region) return LS_OK;
  cudaError_t e = cudaIpcCloseMemHandle(region);
  return e == cudaSuccess ? LS_OK : set_error(LS_ERR_CUDA, "cudaIpcCloseMemHandle: %s", cudaGetErrorString(e));
}

int ls_linear_allreduce_residual(const void* x, int64_t m, int64_t k, const void* w, int64_t n, const void* residual,
                                 void* out, const ls_p2p_exchange* ex, ls_stream_t stream) {
  lsb::P2PExchange e;
  int rc = to_exchange(ex, n, "ls_linear_allreduce_residual", &e);
  if (rc) return rc;
  return launch_linear_allreduce(x, m, k, w, n, residual, out, &e, (cudaStream_t)stream);
}

int ls_allreduce_residual_splits(const float* part, int64_t splits, int64_t m, int64_t n, const void* residual,
                                 void* out, const ls_p2p_exchange* ex, ls_stream_t stream) {
  if (!part || !residual || !out || splits < 1 || splits > 64)
    return set_error(LS_ERR_INVALID_ARGUMENT, "ls_allreduce_residual_f32: null pointer or bad split count");
  lsb::P2PExchange e;
  int rc = to_exchange(ex, n, "ls_allreduce_residual_f32", &e);
  if (rc) return rc;
  if (m < 1 || m > e.max_rows || (int64_t)m * n > (1ll << 31) - 1)
    return set_error(LS_ERR_UNSUPPORTED_SHAPE, "ls_allreduce_residual_f32: m=%lld outside 1..%d", (long long)m,
                     e.max_rows);
  if (lsb::kArGrid > e.max_ctas)
    return set_error(LS_ERR_UNSUPPORTED_SHAPE, "ls_allreduce_residual_f32: the exchange holds %d CTA counters, %d needed",
                     e.max_ctas, lsb::kArGrid);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(lsb::kArGrid);
  cfg.blockDim = dim3(lsb::kArThreads);
  cfg.stream = (cudaStream_t)stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t err = cudaLaunchKernelEx(&cfg, lsb::allreduce_residual_kernel, part, (int)splits,
                                       static_cast<const __nv_bfloat16*>(residual), static_cast<__nv_bfloat16*>(out),
                                       (int)m, (int)n, e, device_error_ptr());
  return err == cudaSuccess ? LS_OK
                            : set_error(LS_ERR_CUDA, "allreduce_residual launch: %s", cudaGetErrorString(err));
}

int ls_allreduce_residual_f32(const float* part, int64_t m, int64_t n, const void* residual, void* out,
                              const ls_p2p_exchange* ex, ls_stream_t stream) {
  return ls_allreduce_residual_splits(part, 1, m, n, residual, out, ex, stream);
}

}  // extern "C"
