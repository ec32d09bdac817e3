// Set-up of the fused tensor-parallel all-reduce: exchange regions in device
// memory, shared between the ranks' processes through CUDA IPC handles (plain
// peer mappings over NVLink; no multicast objects), and the C entry point of
// the row-split linear whose epilogue performs the all-reduce
// (linear_small_m.cu, EPI_AR_RESIDUAL).
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

using namespace lsb_host;

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
  if (!bytes || max_rows < 1 || max_rows > 64 || width < 1 || width > (1 << 20) || max_ctas < 1 ||
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
  if (!ex) return set_error(LS_ERR_INVALID_ARGUMENT, "ls_linear_allreduce_residual: exchange is null");
  if (ex->world < 1 || ex->world > LS_MAX_TP_RANKS || ex->rank < 0 || ex->rank >= ex->world || ex->max_ctas < 1 ||
      ex->max_rows < 1 || ex->width != n)
    return set_error(LS_ERR_INVALID_ARGUMENT, "ls_linear_allreduce_residual: bad exchange description");
  lsb::P2PExchange e = {};
  for (int q = 0; q < ex->world; ++q) {
    if (!ex->peer[q] || !aligned16(ex->peer[q]))
      return set_error(LS_ERR_INVALID_ARGUMENT, "ls_linear_allreduce_residual: region of rank %d missing", q);
    e.peer[q] = static_cast<unsigned char*>(ex->peer[q]);
  }
  e.rank = ex->rank;
  e.world = ex->world;
  e.max_ctas = ex->max_ctas;
  e.max_rows = ex->max_rows;
  e.width = (int)ex->width;
  e.trace = ex->trace;
  return launch_linear_allreduce(x, m, k, w, n, residual, out, &e, (cudaStream_t)stream);
}

}  // extern "C"
