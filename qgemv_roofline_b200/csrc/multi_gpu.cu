// One process, several GPUs: a handle that holds a q8_0 / q4_0 matrix
// sharded by rows (rows [g M / P, (g + 1) M / P) on the g-th of its P
// devices), runs every shard's GEMV on its device's stream and, on request,
// all-gathers y so that every device holds all M rows.
//
// Rows are independent, so the GEMVs need no communication; the all-gather
// is one 2-D peer copy per ordered pair of devices (each device pushes its
// rows of every column into every other device's y), over NVLink through
// NVSwitch where the devices can address each other, through the host
// otherwise.  Ordering across devices uses events only:
//   * a device's copies into device k's y wait for everything the caller had
//     queued on k's stream before this call (k may still be reading its y);
//   * k's stream then waits until every other device's rows have landed.
// So the call is asynchronous like the single-GPU entry points, and work the
// caller queues afterwards on device k's stream sees the whole y.
//
// The per-process path for one process per GPU (torch.distributed) is
// ShardedQGemv in shard.py; this handle is for C / C++ hosts that drive
// several GPUs from one thread.  The reference runs on one GPU only.
#include "qgemv_b200.h"
#include "qgemv_common.cuh"
#include "qgemv_internal.h"

namespace qg {
namespace {

struct MgShard {
  void* q = nullptr;  // SoA quant plane, or ggml blocks, of this device's rows
  void* d = nullptr;  // SoA scale plane (null for ggml blocks)
  int64_t r0 = 0, rows = 0;
};

struct MgHandle {
  int n = 0;
  int dev[QGEMV_MAX_RANKS] = {};
  cudaStream_t own[QGEMV_MAX_RANKS] = {};   // the handle's streams (non-blocking)
  cudaEvent_t start[QGEMV_MAX_RANKS] = {};  // a call's start on each device's stream
  cudaEvent_t done[QGEMV_MAX_RANKS] = {};   // a device's rows are in every device's y
  int fmt = 0, layout = -1;                 // layout -1: no matrix yet
  int64_t M = 0, K = 0;
  MgShard sh[QGEMV_MAX_RANKS];
};

// Restores the caller's current device when the entry point returns.
struct DeviceGuard {
  int prev = -1;
  DeviceGuard() {
    if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
  }
  ~DeviceGuard() {
    if (prev >= 0) cudaSetDevice(prev);
  }
};

int fail(cudaError_t e, const char* what, int device) {
  return set_error(ERR_CUDA, "%s on device %d: %s", what, device, cudaGetErrorString(e));
}

void free_shards(MgHandle* h) {
  for (int g = 0; g < h->n; ++g) {
    if (h->sh[g].q || h->sh[g].d) {
      cudaSetDevice(h->dev[g]);
      cudaFree(h->sh[g].q);
      cudaFree(h->sh[g].d);
    }
    h->sh[g] = MgShard{};
  }
  h->layout = -1;
}

void destroy(MgHandle* h) {
  free_shards(h);
  for (int g = 0; g < h->n; ++g) {
    cudaSetDevice(h->dev[g]);
    if (h->own[g]) cudaStreamDestroy(h->own[g]);
    if (h->start[g]) cudaEventDestroy(h->start[g]);
    if (h->done[g]) cudaEventDestroy(h->done[g]);
  }
  delete h;
}

}  // namespace
}  // namespace qg

using namespace qg;

QGEMV_API int qgemv_mg_init(int32_t ndev, const int32_t* devices, void** handle) {
  if (!handle || !devices) return set_error(ERR_NULL, "devices and handle must not be NULL");
  *handle = nullptr;
  if (ndev < 1 || ndev > QGEMV_MAX_RANKS)
    return set_error(ERR_ARG, "ndev=%d outside 1..%d", ndev, QGEMV_MAX_RANKS);
  int count = 0;
  const cudaError_t ce = cudaGetDeviceCount(&count);
  if (ce != cudaSuccess) return set_error(ERR_CUDA, "cudaGetDeviceCount: %s", cudaGetErrorString(ce));
  for (int g = 0; g < ndev; ++g) {
    if (devices[g] < 0 || devices[g] >= count)
      return set_error(ERR_ARG, "device %d does not exist (%d devices)", devices[g], count);
    for (int k = 0; k < g; ++k)
      if (devices[k] == devices[g]) return set_error(ERR_ARG, "device %d listed twice", devices[g]);
  }
  DeviceGuard guard;
  MgHandle* h = new MgHandle();
  h->n = ndev;
  for (int g = 0; g < ndev; ++g) {
    h->dev[g] = devices[g];
    cudaError_t e = cudaSetDevice(devices[g]);
    if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&h->own[g], cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&h->start[g], cudaEventDisableTiming);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&h->done[g], cudaEventDisableTiming);
    if (e != cudaSuccess) {
      const int rc = fail(e, "stream and events", devices[g]);
      destroy(h);
      return rc;
    }
  }
  // peer access between every pair the hardware connects (NVLink / NVSwitch)
  for (int g = 0; g < ndev; ++g) {
    cudaSetDevice(h->dev[g]);
    for (int k = 0; k < ndev; ++k) {
      if (k == g) continue;
      int can = 0;
      cudaError_t e = cudaDeviceCanAccessPeer(&can, h->dev[g], h->dev[k]);
      if (e == cudaSuccess && can) {
        e = cudaDeviceEnablePeerAccess(h->dev[k], 0);
        if (e == cudaErrorPeerAccessAlreadyEnabled) {
          cudaGetLastError();  // already on (another handle, or the caller)
          e = cudaSuccess;
        }
      }
      if (e != cudaSuccess) {
        const int rc = fail(e, "peer access", h->dev[g]);
        destroy(h);
        return rc;
      }
    }
  }
  *handle = h;
  return OK;
}

QGEMV_API int qgemv_mg_shard(void* handle, int format, int layout, const void* q, const void* d,
                             int64_t M, int64_t K) {
  MgHandle* h = static_cast<MgHandle*>(handle);
  if (!h) return set_error(ERR_NULL, "handle must not be NULL");
  if (format != 8 && format != 4)
    return set_error(ERR_ARG, "format must be QGEMV_Q8_0 (8) or QGEMV_Q4_0 (4), got %d", format);
  if (layout != 0 && layout != 1)
    return set_error(ERR_ARG, "layout must be 0 (SoA planes) or 1 (ggml blocks), got %d", layout);
  if (M < 0 || K < 0 || K % QK)
    return set_error(ERR_SHAPE, "M=%lld K=%lld (K must be a multiple of 32)", (long long)M,
                     (long long)K);
  if (M >= ((int64_t)1 << 31) || K >= ((int64_t)1 << 31))
    return set_error(ERR_UNSUPPORTED, "M and K must be below 2^31");
  if (M > 0 && K > 0 && (!q || (layout == 0 && !d)))
    return set_error(ERR_NULL, layout == 0 ? "q and d must not be NULL" : "blocks must not be NULL");
  DeviceGuard guard;
  free_shards(h);
  const int64_t nb = K / QK;
  const int64_t qrow = layout == 1 ? nb * (format == 8 ? Q8_BLOCK : Q4_BLOCK)
                                   : (format == 8 ? K : K / 2);
  const int64_t drow = layout == 1 ? 0 : nb * 2;
  for (int g = 0; g < h->n; ++g) {
    MgShard& s = h->sh[g];
    s.r0 = M * g / h->n;
    s.rows = M * (g + 1) / h->n - s.r0;
    if (s.rows == 0 || K == 0) continue;
    cudaError_t e = cudaSetDevice(h->dev[g]);
    if (e == cudaSuccess) e = cudaMalloc(&s.q, (size_t)(s.rows * qrow));
    if (e == cudaSuccess)
      e = cudaMemcpy(s.q, static_cast<const char*>(q) + s.r0 * qrow, (size_t)(s.rows * qrow),
                     cudaMemcpyDefault);
    if (e == cudaSuccess && drow) e = cudaMalloc(&s.d, (size_t)(s.rows * drow));
    if (e == cudaSuccess && drow)
      e = cudaMemcpy(s.d, static_cast<const char*>(d) + s.r0 * drow, (size_t)(s.rows * drow),
                     cudaMemcpyDefault);
    if (e != cudaSuccess) {
      const int rc = fail(e, "copying the shard", h->dev[g]);
      free_shards(h);
      return rc;
    }
  }
  h->fmt = format;
  h->layout = layout;
  h->M = M;
  h->K = K;
  return OK;
}

QGEMV_API int qgemv_mg_rows(void* handle, int32_t index, int64_t* r0, int64_t* rows) {
  const MgHandle* h = static_cast<const MgHandle*>(handle);
  if (!h || !r0 || !rows) return set_error(ERR_NULL, "handle, r0 and rows must not be NULL");
  if (h->layout < 0) return set_error(ERR_ARG, "no matrix: call qgemv_mg_shard first");
  if (index < 0 || index >= h->n)
    return set_error(ERR_ARG, "index %d outside 0..%d", index, h->n - 1);
  *r0 = h->sh[index].r0;
  *rows = h->sh[index].rows;
  return OK;
}

QGEMV_API int qgemv_mg_gemv(void* handle, const float* const* x, float* const* y, int32_t ncols,
                            int32_t allgather, void* const* streams) {
  MgHandle* h = static_cast<MgHandle*>(handle);
  if (!h) return set_error(ERR_NULL, "handle must not be NULL");
  if (h->layout < 0) return set_error(ERR_ARG, "no matrix: call qgemv_mg_shard first");
  if (ncols < 0) return set_error(ERR_SHAPE, "ncols=%d is negative", ncols);
  if (h->M == 0 || ncols == 0) return OK;
  if (!x || !y) return set_error(ERR_NULL, "x and y must not be NULL");
  for (int g = 0; g < h->n; ++g)
    if (!y[g] || (h->K > 0 && !x[g]))
      return set_error(ERR_NULL, "x[%d] and y[%d] must not be NULL", g, g);
  const bool gather = allgather != 0 && h->n > 1;
  DeviceGuard guard;
  cudaStream_t st[QGEMV_MAX_RANKS];
  for (int g = 0; g < h->n; ++g)
    st[g] = streams && streams[g] ? static_cast<cudaStream_t>(streams[g]) : h->own[g];
  if (gather)
    for (int g = 0; g < h->n; ++g) {
      cudaError_t e = cudaSetDevice(h->dev[g]);
      if (e == cudaSuccess) e = cudaEventRecord(h->start[g], st[g]);
      if (e != cudaSuccess) return fail(e, "recording the call's start", h->dev[g]);
    }
  // every device's rows of every column (x and y as [ncols][K] and [ncols][M])
  for (int g = 0; g < h->n; ++g) {
    const MgShard& s = h->sh[g];
    if (s.rows == 0) continue;
    const cudaError_t e = cudaSetDevice(h->dev[g]);
    if (e != cudaSuccess) return fail(e, "cudaSetDevice", h->dev[g]);
    float* yg = y[g] + s.r0;
    int rc;
    if (h->layout == 0)
      rc = h->fmt == 8 ? qgemv_q8_0_soa(s.q, s.d, x[g], yg, s.rows, h->K, ncols, h->K, h->M, st[g])
                       : qgemv_q4_0_soa(s.q, s.d, x[g], yg, s.rows, h->K, ncols, h->K, h->M, st[g]);
    else
      rc = h->fmt == 8 ? qgemv_q8_0_aos(s.q, x[g], yg, s.rows, h->K, ncols, h->K, h->M, st[g])
                       : qgemv_q4_0_aos(s.q, x[g], yg, s.rows, h->K, ncols, h->K, h->M, st[g]);
    if (rc != OK) return rc;
  }
  if (!gather) return OK;
  // all-gather: device g pushes its rows into every other device's y, after
  // what that device had queued before this call
  const size_t pitch = (size_t)h->M * sizeof(float);
  for (int g = 0; g < h->n; ++g) {
    const MgShard& s = h->sh[g];
    cudaError_t e = cudaSetDevice(h->dev[g]);
    for (int k = 0; k < h->n && e == cudaSuccess; ++k) {
      if (k == g) continue;
      e = cudaStreamWaitEvent(st[g], h->start[k], 0);
      if (e == cudaSuccess && s.rows > 0)
        e = cudaMemcpy2DAsync(y[k] + s.r0, pitch, y[g] + s.r0, pitch,
                              (size_t)s.rows * sizeof(float), (size_t)ncols, cudaMemcpyDefault,
                              st[g]);
    }
    if (e == cudaSuccess) e = cudaEventRecord(h->done[g], st[g]);
    if (e != cudaSuccess) return fail(e, "all-gather copies", h->dev[g]);
  }
  for (int k = 0; k < h->n; ++k) {
    cudaError_t e = cudaSetDevice(h->dev[k]);
    for (int g = 0; g < h->n && e == cudaSuccess; ++g)
      if (g != k) e = cudaStreamWaitEvent(st[k], h->done[g], 0);
    if (e != cudaSuccess) return fail(e, "waiting for the other devices' rows", h->dev[k]);
  }
  return OK;
}

QGEMV_API int qgemv_mg_synchronize(void* handle) {
  MgHandle* h = static_cast<MgHandle*>(handle);
  if (!h) return set_error(ERR_NULL, "handle must not be NULL");
  DeviceGuard guard;
  for (int g = 0; g < h->n; ++g) {
    cudaError_t e = cudaSetDevice(h->dev[g]);
    if (e == cudaSuccess) e = cudaStreamSynchronize(h->own[g]);
    if (e != cudaSuccess) return fail(e, "cudaStreamSynchronize", h->dev[g]);
  }
  return OK;
}

QGEMV_API int qgemv_mg_destroy(void* handle) {
  MgHandle* h = static_cast<MgHandle*>(handle);
  if (!h) return OK;
  DeviceGuard guard;
  for (int g = 0; g < h->n; ++g) {
    cudaSetDevice(h->dev[g]);
    cudaStreamSynchronize(h->own[g]);
  }
  destroy(h);
  return OK;
}
