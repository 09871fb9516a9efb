// ec_noalloc.cu -- flat search over caller-owned device buffers that allocates
// nothing: the per-chunk candidate lists that ec_flat_search keeps in a
// cudaMalloc'd workspace live here in one file-scope device array instead.
//
// Who needs it: a host whose device memory is carved up in advance (an
// SBCL image that reserves its whole device arena at start-up and hands out
// slices, or a serving loop under a hard per-process memory cap) cannot let
// the library call cudaMalloc mid-request, because the allocation can fail
// once the arena is taken and cudaMalloc / cudaFree may synchronise the whole
// device, stalling every other stream of the request loop.
//
// Limits and sharing:
//   * the scratch holds kScratchBytes (16 MiB) of candidates; a call needs
//     nq x chunks x topk x 8 bytes, chunks = min(256, ceil(n / 8192)), and
//     larger requests are rejected with EC_EINVAL before anything is launched;
//   * there is one array per device, shared by every call on that device:
//     calls whose kernels overlap in time (different streams, or different
//     host threads on one stream without ordering) race on it; calls issued
//     in order on one stream do not;
//   * nothing in the scratch has to start at zero: the scan kernel writes
//     every candidate slot (or its empty marker) before the merge reads it;
//   * the array is placed in device memory when this file's module is
//     loaded on a device: at ec_init for the library's devices, otherwise at
//     the first call with nq > 0 on that device (CUDA loads modules lazily).
//     A host that reserves its device arena up front should therefore call
//     ec_init (or make one search) before it takes the arena;
//   * the array's address is looked up with cudaGetSymbolAddress, with the
//     device current, on the first call in each CUDA context and cached per
//     (device, context); a new context (after cudaDeviceReset, or a caller's
//     own non-primary context) gets a fresh lookup.  Make that first call
//     before any stream capture begins.
#include <cuda.h>

#include <cstdint>
#include <mutex>

#include "ec_ivf.h"
#include "ec_state.h"
#include "embedcuda.h"

namespace ec {
namespace {

constexpr size_t kScratchBytes = size_t(16) << 20;
constexpr int kMaxOrdinals = 64;

static __device__ __align__(256) unsigned char g_search_scratch[kScratchBytes];

std::mutex g_scratch_mu;
struct ScratchSlot {
  void* ctx = nullptr;  // CUcontext the address belongs to
  void* ptr = nullptr;
};
ScratchSlot g_scratch[kMaxOrdinals];

// cuCtxGetCurrent through the runtime's driver entry point (the library
// links no libcuda); nullptr when the driver does not offer it
using CtxGetCurrentFn = CUresult (*)(CUcontext*);
CtxGetCurrentFn ctx_get_current() {
  static CtxGetCurrentFn fn = [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &f, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess) {
      cudaGetLastError();
      return static_cast<CtxGetCurrentFn>(nullptr);
    }
    return reinterpret_cast<CtxGetCurrentFn>(f);
  }();
  return fn;
}

}  // namespace

// address of the current device's scratch array in the current context;
// looked up once per (device, context)
int noalloc_scratch_current(void** out) {
  int dev = -1;
  if (int rc = check_cuda(cudaGetDevice(&dev), "cudaGetDevice")) return rc;
  if (dev < 0 || dev >= kMaxOrdinals) return set_error(EC_EINVAL, "device ordinal %d out of range", dev);
  CUcontext ctx = nullptr;
  if (CtxGetCurrentFn f = ctx_get_current()) f(&ctx);
  std::lock_guard<std::mutex> lk(g_scratch_mu);
  ScratchSlot& s = g_scratch[dev];
  if (!s.ptr || s.ctx != static_cast<void*>(ctx)) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_search_scratch);
    if (e != cudaSuccess || !p) {
      cudaGetLastError();
      return set_error(EC_ECUDA, "scratch address on device %d: %s", dev, cudaGetErrorString(e));
    }
    s.ptr = p;
    s.ctx = ctx;
  }
  *out = s.ptr;
  return EC_OK;
}

namespace {

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace
}  // namespace ec

using namespace ec;

extern "C" int ec_flat_search_noalloc(const float* d_x, int64_t n, int d, const float* d_q, int nq,
                                      int topk, int64_t* d_ids, float* d_scores, void* stream) {
  clear_error();
  if (nq == 0) return EC_OK;
  if (!d_x || !d_q || !d_ids || !d_scores || nq < 0 || n <= 0 || n >= (int64_t(1) << 31))
    return set_error(EC_EINVAL, "bad no-alloc search arguments (device pointers, 0 < n < 2^31, nq >= 0)");
  if (d <= 0 || d % 4 || d > 8192) return set_error(EC_EINVAL, "dimension %d: need d %% 4 == 0, d <= 8192", d);
  if (topk < 1 || topk > 64) return set_error(EC_EINVAL, "topk %d: need 1 <= topk <= 64", topk);
  if (nq > 65535) return set_error(EC_EINVAL, "nq %d: at most 65535 queries per call", nq);
  if (!aligned16(d_x) || !aligned16(d_q)) return set_error(EC_EINVAL, "vectors and queries must be 16-byte aligned");
  // same chunking as ec_flat_search, so the merge sees the same candidate order
  const int64_t nchunks64 = (n + 8191) / 8192;
  const int nchunks = static_cast<int>(nchunks64 < 256 ? nchunks64 : 256);
  const size_t need = static_cast<size_t>(nq) * nchunks * topk * 8;
  if (need > kScratchBytes)
    return set_error(EC_EINVAL,
                     "search needs %zu bytes of candidate scratch, the static scratch holds %zu "
                     "(at most %zu queries per call for n=%lld, topk=%d)",
                     need, kScratchBytes, kScratchBytes / (static_cast<size_t>(nchunks) * topk * 8),
                     static_cast<long long>(n), topk);
  void* scratch = nullptr;
  if (int rc = noalloc_scratch_current(&scratch)) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  auto* cand = static_cast<unsigned long long*>(scratch);
  if (int rc = check_cuda(launch_flat_scan(d_x, n, d, nchunks, d_q, nq, topk, cand, st), "flat scan")) return rc;
  return check_cuda(launch_merge(cand, nq, nchunks, topk, d_ids, d_scores, st), "merge");
}
