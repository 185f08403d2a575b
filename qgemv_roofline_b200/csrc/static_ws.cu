// Workspace compiled into the library, for callers that must not allocate.
//
// The batched SoA GEMV (2..16 columns per launch on the tensor cores) needs a
// workspace for the re-laid activations (and, on tcgen05, per-row-tile
// counters and partial sums).  qgemv_soa_static_ws takes it from this fixed
// array instead of from the caller or from cudaMalloc, so that no call of
// that entry point allocates device memory.
//
// * Size: kStaticWsBytes (2 MiB) per device.  The tcgen05 kernel runs when
//   its workspace fits; otherwise the mma.sync kernel, whose workspace
//   (128 + 2064 * min(ncols, 16) * ceil(K / 512) bytes) fits for K <= 32256
//   with 16 columns.  Larger calls are rejected before anything is launched.
// * Set-up: the first call on a device looks up the array's address on that
//   device (cudaGetSymbolAddress, with that device current) and caches it;
//   later calls reuse it.  Make that first call before any stream capture.
// * Contents: nothing in the array needs to start at zero; every byte the
//   GEMV reads is written by the activation pre-pass of the same call.
// * One array per device: calls that overlap in time on one device (two
//   streams, or two host threads) race on it and corrupt each other's
//   results.  Calls on a single stream are ordered and safe.
#include "qgemv_common.cuh"
#include "qgemv_internal.h"

#include <mutex>

static __device__ __align__(256) unsigned char g_static_ws[qg::kStaticWsBytes];

namespace qg {
namespace {
constexpr int kMaxDevices = 64;
std::mutex g_mu;
void* g_addr[kMaxDevices] = {};
}  // namespace

int static_workspace(void** out, size_t* bytes) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return set_error(ERR_CUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices) return set_error(ERR_UNSUPPORTED, "device %d", dev);
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_addr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_static_ws);
    if (e != cudaSuccess || !p)
      return set_error(ERR_CUDA, "address of the static workspace on device %d: %s", dev,
                       cudaGetErrorString(e));
    g_addr[dev] = p;
  }
  *out = g_addr[dev];
  *bytes = kStaticWsBytes;
  return OK;
}

}  // namespace qg
