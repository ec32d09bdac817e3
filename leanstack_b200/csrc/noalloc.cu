// Greedy head (final RMSNorm + lm_head GEMV + argmax) with library-owned scratch.
//
// ls_lmhead_argmax needs a small caller-provided workspace: one arrival
// counter and, per activation row and CTA, the CTA's best logit and its index.
// ls_lmhead_argmax_noalloc runs the same kernel with that workspace taken from
// a fixed array that lives in this library's device image, so a call allocates
// nothing: no cudaMalloc, no cudaFree, no torch tensor.  It exists for callers
// that cannot allocate device memory on the path that picks the next token: a
// C or FFI host that binds only this library and owns no device allocator, or a
// server that plans every byte of HBM at start-up and forbids any later growth.
//
// Limits and rules of use:
//  * The scratch is kNoAllocScratchBytes (16 KiB) per device.  A call whose
//    workspace would exceed it (m rows x CTAs of the head grid) is rejected with
//    LS_ERR_WORKSPACE before anything is launched.  On a 148-SM B200 every
//    m in 1..8 fits (at most 9,984 bytes).
//  * Every call looks up the scratch array's device address with the device
//    current (a host-side query; it moves no data and allocates nothing), so
//    a context that was torn down and rebuilt is followed.  The first call
//    that sees a new address on a device also zeroes the arrival counter and
//    waits for that on the caller's stream, so it must finish before any other
//    call on that device starts, and it must come before any stream capture.
//  * There is one scratch array per device, shared by every caller of this
//    entry point on that device.  Two calls whose kernels overlap on the GPU
//    (different streams, or different host threads) race on it and may return
//    wrong ids.  Serialise them, e.g. issue them on one stream.
//  * The kernel's last CTA leaves the counter at zero again, so the scratch
//    needs no clearing between calls.
#include <mutex>

#include "common.cuh"

namespace lsb {
// Scratch of ls_lmhead_argmax_noalloc: [0, 256) arrival counter, then the
// per-CTA best values and best indices, each region rounded up to 256 bytes.
constexpr int64_t kNoAllocScratchBytes = 16 * 1024;
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];
}  // namespace lsb

namespace lsb_host {
int launch_linear(const void* x, int64_t m, int64_t k, const void* norm_w, float eps, const void* w, int64_t n,
                  int epi, const void* residual, void* out, cudaStream_t stream, float* part_val, int* part_idx,
                  unsigned int* counter, int64_t* out_ids, int grid_override);
int lmhead_grid(int64_t vocab, int64_t m);

namespace {
constexpr int kMaxDevices = 64;

// Device address of the scratch array on the current device.  The counter is
// cleared (synchronously) the first time an address is seen on a device.
// Returns LS_OK or an error code (message recorded).
int noalloc_scratch(cudaStream_t stream, unsigned char** out) {
  static unsigned char* cleared[kMaxDevices] = {nullptr};
  static std::mutex mu;
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return set_error(LS_ERR_CUDA, "lmhead_argmax_noalloc: cudaGetDevice: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices)
    return set_error(LS_ERR_UNSUPPORTED_SHAPE, "lmhead_argmax_noalloc: device %d beyond %d", dev, kMaxDevices);
  void* ptr = nullptr;
  e = cudaGetSymbolAddress(&ptr, lsb::g_noalloc_scratch);
  if (e != cudaSuccess || !ptr)
    return set_error(LS_ERR_CUDA, "lmhead_argmax_noalloc: cudaGetSymbolAddress: %s", cudaGetErrorString(e));
  std::lock_guard<std::mutex> lock(mu);
  if (cleared[dev] != ptr) {
    // The arrival counter must start at zero.
    e = cudaMemsetAsync(ptr, 0, 256, stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
    if (e != cudaSuccess)
      return set_error(LS_ERR_CUDA, "lmhead_argmax_noalloc: clearing the counter: %s", cudaGetErrorString(e));
    cleared[dev] = static_cast<unsigned char*>(ptr);
  }
  *out = static_cast<unsigned char*>(ptr);
  return LS_OK;
}
}  // namespace
}  // namespace lsb_host

using namespace lsb_host;

extern "C" int ls_lmhead_argmax_noalloc(const void* h, int64_t m, int64_t hidden, const void* final_norm_w,
                                        float eps, const void* lm_head_w, int64_t vocab, int64_t* out_ids,
                                        ls_stream_t stream) {
  if (!h || !lm_head_w || !out_ids) return set_error(LS_ERR_INVALID_ARGUMENT, "ls_lmhead_argmax_noalloc: null pointer");
  if (m < 1 || m > 8)
    return set_error(LS_ERR_UNSUPPORTED_SHAPE, "ls_lmhead_argmax_noalloc: m=%lld outside 1..8", (long long)m);
  if (vocab < 1 || hidden < 1) return set_error(LS_ERR_INVALID_ARGUMENT, "ls_lmhead_argmax_noalloc: bad sizes");
  const int g = lmhead_grid(vocab, m);
  const int64_t region = ((m * g * 4 + 255) / 256) * 256;
  const int64_t need = 256 + 2 * region;
  if (need > lsb::kNoAllocScratchBytes)
    return set_error(LS_ERR_WORKSPACE,
                     "ls_lmhead_argmax_noalloc: m=%lld over %d CTAs needs %lld scratch bytes, more than the fixed %lld",
                     (long long)m, g, (long long)need, (long long)lsb::kNoAllocScratchBytes);
  unsigned char* ws = nullptr;
  int rc = noalloc_scratch((cudaStream_t)stream, &ws);
  if (rc) return rc;
  return launch_linear(h, m, hidden, final_norm_w, eps, lm_head_w, vocab, 3, nullptr, nullptr, (cudaStream_t)stream,
                       reinterpret_cast<float*>(ws + 256), reinterpret_cast<int*>(ws + 256 + region),
                       reinterpret_cast<unsigned int*>(ws), out_ids, g);
}
