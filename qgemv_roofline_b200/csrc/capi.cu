// C ABI of libqgemv_b200.so (declared in include/qgemv_b200.h): argument
// validation, error reporting and dispatch to the kernel files.
//
// The reference had no error channel: its harness printed and called exit(1)
// on any CUDA error (src/bench.cu:19-27) and rejected K % 512 != 0
// (src/bench.cu:259).  Here every entry point validates first, returns a
// status code, keeps a per-thread message, and accepts any K % 32 == 0.
#include "qgemv_b200.h"

#include <algorithm>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <map>
#include <set>
#include <utility>
#include <vector>

#include "qgemv_common.cuh"
#include "qgemv_internal.h"

namespace qg {

static thread_local char g_err[512] = "";

int set_error(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return code;
}

int check_launch(const char* what) {
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
  return OK;
}

namespace {
constexpr int kMaxDevices = 64;
std::mutex g_mu;
DeviceInfo g_dev[kMaxDevices];
bool g_dev_ok[kMaxDevices] = {};
std::set<std::pair<const void*, int>> g_smem_set;
struct OccKey {
  const void* f;
  int dev, threads;
  size_t smem;
  bool operator<(const OccKey& o) const {
    return f != o.f ? f < o.f : dev != o.dev ? dev < o.dev
         : threads != o.threads ? threads < o.threads : smem < o.smem;
  }
};
std::map<OccKey, int> g_occ;
}  // namespace

int current_device_info(DeviceInfo& out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return set_error(ERR_CUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices) return set_error(ERR_UNSUPPORTED, "device %d", dev);
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_dev_ok[dev]) {
    DeviceInfo d;
    d.device = dev;
    if ((e = cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, dev)) ||
        (e = cudaDeviceGetAttribute(&d.smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev)) ||
        (e = cudaDeviceGetAttribute(&d.cc_major, cudaDevAttrComputeCapabilityMajor, dev)) ||
        (e = cudaDeviceGetAttribute(&d.cc_minor, cudaDevAttrComputeCapabilityMinor, dev)) ||
        (e = cudaDeviceGetAttribute(&d.l2_bytes, cudaDevAttrL2CacheSize, dev)))
      return set_error(ERR_CUDA, "cudaDeviceGetAttribute: %s", cudaGetErrorString(e));
    if (d.cc_major != 10 || d.cc_minor != 0)
      return set_error(ERR_UNSUPPORTED,
                       "device %d is sm_%d%d; this library is built for sm_100a (B200) only", dev,
                       d.cc_major, d.cc_minor);
    g_dev[dev] = d;
    g_dev_ok[dev] = true;
  }
  out = g_dev[dev];
  return OK;
}

int allow_max_smem(const void* func, const DeviceInfo& dev) {
  std::lock_guard<std::mutex> lk(g_mu);
  auto key = std::make_pair(func, dev.device);
  if (g_smem_set.count(key)) return OK;
  // dynamic + static shared memory must stay within the opt-in maximum
  cudaFuncAttributes fa;
  cudaError_t e = cudaFuncGetAttributes(&fa, func);
  if (e != cudaSuccess)
    return set_error(ERR_CUDA, "cudaFuncGetAttributes: %s", cudaGetErrorString(e));
  e = cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           dev.smem_optin - (int)fa.sharedSizeBytes);
  if (e != cudaSuccess)
    return set_error(ERR_CUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
  g_smem_set.insert(key);
  return OK;
}

int occupancy(const void* func, const DeviceInfo& dev, int threads, size_t smem, int* out) {
  const OccKey key{func, dev.device, threads, smem};
  {
    std::lock_guard<std::mutex> lk(g_mu);
    auto it = g_occ.find(key);
    if (it != g_occ.end()) {
      *out = it->second;
      return OK;
    }
  }
  int occ = 0;
  const cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, func, threads, smem);
  if (e != cudaSuccess || occ < 1)
    return set_error(ERR_CUDA, "occupancy query failed (%s, %d blocks)", cudaGetErrorString(e), occ);
  std::lock_guard<std::mutex> lk(g_mu);
  g_occ[key] = occ;
  *out = occ;
  return OK;
}

namespace {

constexpr int64_t kMaxDim = (int64_t)1 << 31;

bool misaligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) % a) != 0; }

int check_fmt(int format) {
  if (format != 8 && format != 4)
    return set_error(ERR_ARG, "format must be QGEMV_Q8_0 (8) or QGEMV_Q4_0 (4), got %d", format);
  return OK;
}

int check_mk(int64_t M, int64_t K) {
  if (M < 0 || K < 0) return set_error(ERR_SHAPE, "negative shape M=%lld K=%lld", (long long)M, (long long)K);
  if (K % QK) return set_error(ERR_SHAPE, "K=%lld is not a multiple of 32", (long long)K);
  if (M >= kMaxDim || K >= kMaxDim)
    return set_error(ERR_UNSUPPORTED, "M and K must be below 2^31 (M=%lld K=%lld)", (long long)M,
                     (long long)K);
  return OK;
}

// Workspace of a batched SoA call: the tcgen05 kernel's (when it may run) or
// the mma.sync kernel's, whichever is larger (0 when neither runs).
size_t soa_batch_workspace(const GemvCall& probe, bool allow_tc) {
  if (!mma_eligible(probe)) return 0;
  size_t need = mma_workspace_bytes(probe.K, probe.N);
  DeviceInfo dev;
  if (allow_tc && current_device_info(dev) == OK)
    need = std::max(need, tc_soa_workspace_bytes(probe.M, probe.K, probe.N, dev.sms));
  return need;
}

int gemv_entry(int fmt, bool aos, const void* q, const void* d, const float* x, float* y,
               int64_t M, int64_t K, int32_t ncols, int64_t ldx, int64_t ldy, void* stream,
               void* ws = nullptr, size_t ws_bytes = 0, bool caller_ws = false,
               bool allow_tc = true) {
  if (int rc = check_mk(M, K)) return rc;
  if (ncols < 0) return set_error(ERR_SHAPE, "ncols=%d is negative", ncols);
  if (M == 0 || ncols == 0) return OK;
  if (!y || (K > 0 && !x)) return set_error(ERR_NULL, "x and y must not be NULL");
  if (K > 0 && (!q || (!aos && !d)))
    return set_error(ERR_NULL, aos ? "blocks must not be NULL" : "q and d must not be NULL");
  if (ncols > 1 && ldx < K)
    return set_error(ERR_SHAPE, "ldx=%lld < K=%lld", (long long)ldx, (long long)K);
  if (ncols > 1 && ldy < M)
    return set_error(ERR_SHAPE, "ldy=%lld < M=%lld", (long long)ldy, (long long)M);
  if (ncols == 1) {
    ldx = K;
    ldy = M;
  }
  if (K > 0 && misaligned(q, 16))
    return set_error(ERR_ALIGN, aos ? "blocks must be 16-byte aligned" : "q must be 16-byte aligned");
  if (!aos && K > 0 && misaligned(d, 2)) return set_error(ERR_ALIGN, "d must be 2-byte aligned");
  if (misaligned(x, 4) || misaligned(y, 4))
    return set_error(ERR_ALIGN, "x and y must be 4-byte aligned");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (K == 0) return fill_zero_rows(y, M, ncols, ldy, st);
  GemvCall c;
  c.q = q;
  c.d = d;
  c.x = x;
  c.y = y;
  c.M = M;
  c.K = K;
  c.N = ncols;
  c.ldx = ldx;
  c.ldy = ldy;
  c.no_tc = !allow_tc;
  if (!aos) {
    // the tensor-core batch kernels need a workspace: the caller's, or one
    // cached for this stream
    // (two columns on the TMA path need none)
    GemvCall probe = c;
    probe.N = std::min(ncols, 16);
    if (probe.N >= 2 && mma_eligible(probe) && !tma_pair_taken(fmt, false, c)) {
      const size_t need = soa_batch_workspace(probe, allow_tc);
      if (caller_ws) {
        if (!ws || ws_bytes < need)
          return set_error(ERR_ARG, "this call needs a workspace of %zu bytes, got %zu", need,
                           ws_bytes);
        if (misaligned(ws, 16)) return set_error(ERR_ALIGN, "workspace must be 16-byte aligned");
      } else if (int rc = stream_workspace(st, need, &ws)) {
        return rc;
      } else {
        ws_bytes = need;
      }
      c.ws = ws;
      c.ws_bytes = ws_bytes;
    }
  }
  return aos ? gemv_aos(fmt, c, st) : gemv_soa(fmt, c, st);
}

// Per-(device, stream) workspaces of the plain entry points.
std::mutex g_ws_mu;
std::map<std::pair<int, cudaStream_t>, std::pair<void*, size_t>> g_ws;

}  // namespace

int stream_workspace(cudaStream_t st, size_t bytes, void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return set_error(ERR_CUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
  std::lock_guard<std::mutex> lk(g_ws_mu);
  auto& slot = g_ws[std::make_pair(dev, st)];
  if (slot.first && slot.second >= bytes) {
    *out = slot.first;
    return OK;
  }
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  e = cudaStreamIsCapturing(st, &cs);
  if (e != cudaSuccess || cs != cudaStreamCaptureStatusNone)
    return set_error(ERR_UNSUPPORTED,
                     "a batched call on this stream needs a %zu-byte workspace, which cannot be "
                     "allocated during stream capture: make one uncaptured call of this shape "
                     "on the stream first, or pass a workspace (qgemv_soa_ws)",
                     bytes);
  const size_t grow = std::max(bytes, slot.second * 2);
  if (slot.first) {
    // the old buffer may still be read by work queued on this stream
    if ((e = cudaStreamSynchronize(st)) != cudaSuccess || (e = cudaFree(slot.first)) != cudaSuccess)
      return set_error(ERR_CUDA, "releasing the stream workspace: %s", cudaGetErrorString(e));
    slot = std::make_pair(nullptr, (size_t)0);
  }
  void* p = nullptr;
  if ((e = cudaMalloc(&p, grow)) != cudaSuccess)
    return set_error(ERR_CUDA, "allocating a %zu-byte stream workspace: %s", grow,
                     cudaGetErrorString(e));
  slot = std::make_pair(p, grow);
  *out = p;
  return OK;
}

int release_workspaces() {
  std::lock_guard<std::mutex> lk(g_ws_mu);
  int rc = OK;
  for (auto& kv : g_ws) {
    if (!kv.second.first) continue;
    int cur = 0;
    cudaGetDevice(&cur);
    cudaSetDevice(kv.first.first);
    cudaError_t e = cudaDeviceSynchronize();
    if (e == cudaSuccess) e = cudaFree(kv.second.first);
    cudaSetDevice(cur);
    if (e != cudaSuccess && rc == OK)
      rc = set_error(ERR_CUDA, "releasing a stream workspace: %s", cudaGetErrorString(e));
  }
  g_ws.clear();
  return rc;
}

namespace {

}  // namespace
}  // namespace qg

using namespace qg;

extern "C" {

QGEMV_API int qgemv_version(void) { return 100; }

QGEMV_API const char* qgemv_last_error(void) { return g_err; }

QGEMV_API const char* qgemv_status_string(int status) {
  switch (status) {
    case QGEMV_OK: return "QGEMV_OK";
    case QGEMV_ERR_NULL: return "QGEMV_ERR_NULL";
    case QGEMV_ERR_SHAPE: return "QGEMV_ERR_SHAPE";
    case QGEMV_ERR_ALIGN: return "QGEMV_ERR_ALIGN";
    case QGEMV_ERR_CUDA: return "QGEMV_ERR_CUDA";
    case QGEMV_ERR_UNSUPPORTED: return "QGEMV_ERR_UNSUPPORTED";
    case QGEMV_ERR_TIMEOUT: return "QGEMV_ERR_TIMEOUT";
    case QGEMV_ERR_ARG: return "QGEMV_ERR_ARG";
    default: return "QGEMV_ERR_UNKNOWN";
  }
}

QGEMV_API int qgemv_device_info_get(int device, qgemv_device_info* out) {
  if (!out) return set_error(ERR_NULL, "out must not be NULL");
  memset(out, 0, sizeof(*out));
  cudaDeviceProp p;
  cudaError_t e = cudaGetDeviceProperties(&p, device);
  if (e != cudaSuccess)
    return set_error(ERR_CUDA, "cudaGetDeviceProperties(%d): %s", device, cudaGetErrorString(e));
  snprintf(out->name, sizeof(out->name), "%s", p.name);
  out->device = device;
  out->cc_major = p.major;
  out->cc_minor = p.minor;
  out->sms = p.multiProcessorCount;
  out->l2_bytes = p.l2CacheSize;
  cudaDeviceGetAttribute(&out->mem_clock_khz, cudaDevAttrMemoryClockRate, device);
  cudaDeviceGetAttribute(&out->bus_width_bits, cudaDevAttrGlobalMemoryBusWidth, device);
  cudaDeviceGetAttribute(&out->sm_clock_khz, cudaDevAttrClockRate, device);
  cudaDeviceGetAttribute(&out->smem_per_block_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin,
                         device);
  out->datasheet_gbps = 2.0 * out->mem_clock_khz * 1e3 * (out->bus_width_bits / 8.0) / 1e9;
  return OK;
}

QGEMV_API int qgemv_q8_0_soa(const void* q, const void* d, const float* x, float* y, int64_t M,
                             int64_t K, int32_t ncols, int64_t ldx, int64_t ldy, void* stream) {
  return gemv_entry(8, false, q, d, x, y, M, K, ncols, ldx, ldy, stream);
}

QGEMV_API int qgemv_q4_0_soa(const void* q, const void* d, const float* x, float* y, int64_t M,
                             int64_t K, int32_t ncols, int64_t ldx, int64_t ldy, void* stream) {
  return gemv_entry(4, false, q, d, x, y, M, K, ncols, ldx, ldy, stream);
}

QGEMV_API int qgemv_soa_variant_count(void) { return soa_variant_count(); }

QGEMV_API const char* qgemv_soa_variant_name(int variant) { return soa_variant_name(variant); }

QGEMV_API int qgemv_soa_variant(int format, int variant, int32_t grid, const void* q,
                                const void* d, const float* x, float* y, int64_t M, int64_t K,
                                void* stream) {
  if (int rc = check_fmt(format)) return rc;
  if (int rc = check_mk(M, K)) return rc;
  if (grid < 0) return set_error(ERR_ARG, "grid must be >= 0");
  if (M == 0 || K == 0) return set_error(ERR_SHAPE, "variants need M > 0 and K > 0");
  if (!q || !d || !x || !y) return set_error(ERR_NULL, "q, d, x and y must not be NULL");
  if (misaligned(q, 16) || misaligned(d, 2) || misaligned(x, 4) || misaligned(y, 4))
    return set_error(ERR_ALIGN, "q must be 16-byte, d 2-byte, x and y 4-byte aligned");
  GemvCall c;
  c.q = q;
  c.d = d;
  c.x = x;
  c.y = y;
  c.M = M;
  c.K = K;
  c.N = 1;
  c.ldx = K;
  c.ldy = M;
  c.grid_override = grid;
  return gemv_soa_variant(format, variant, c, static_cast<cudaStream_t>(stream));
}

QGEMV_API int qgemv_check_device_error(int clear, void* stream) {
  int v = 0, w = 0, t = 0;
  if (int rc = read_device_error(clear, static_cast<cudaStream_t>(stream), &v)) return rc;
  if (int rc = read_mma_error(clear, static_cast<cudaStream_t>(stream), &w)) return rc;
  if (int rc = read_tc_error(clear, static_cast<cudaStream_t>(stream), &t)) return rc;
  if (!v) v = w;
  if (!v) v = t;
  if (v) return set_error(v, "a kernel reported %s on the device", qgemv_status_string(v));
  return OK;
}

QGEMV_API int qgemv_set_wait_limit(int64_t microseconds) {
  long long cycles = kDefaultSpinLimit;
  if (microseconds > 0) {
    int dev = 0, khz = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&khz, cudaDevAttrClockRate, dev);
    if (e != cudaSuccess) return set_error(ERR_CUDA, "reading the SM clock: %s", cudaGetErrorString(e));
    if (microseconds > (int64_t)1 << 40) return set_error(ERR_ARG, "wait limit too large");
    cycles = (long long)microseconds * (khz > 0 ? khz : 2000000) / 1000;
    if (cycles < 1) cycles = 1;
  }
  if (int rc = set_spin_limit(cycles)) return rc;
  if (int rc = set_mma_spin_limit(cycles)) return rc;
  return set_tc_spin_limit(cycles);
}

QGEMV_API int32_t qgemv_tile_counters_used(int device) { return tile_counters_used(device); }

QGEMV_API int32_t qgemv_tile_counters_capacity(void) { return tile_counters_capacity(); }

QGEMV_API size_t qgemv_soa_workspace_bytes(int format, int64_t M, int64_t K, int32_t ncols) {
  if (check_fmt(format) || check_mk(M, K) || ncols < 2 || M == 0) return 0;
  GemvCall probe;
  probe.M = M;
  probe.K = K;
  probe.N = std::min(ncols, 16);
  // alignment is checked per call; assume aligned planes here
  probe.q = reinterpret_cast<const void*>((uintptr_t)256);
  probe.d = probe.q;
  return soa_batch_workspace(probe, true);
}

QGEMV_API int qgemv_soa_ws(int format, const void* q, const void* d, const float* x, float* y,
                           int64_t M, int64_t K, int32_t ncols, int64_t ldx, int64_t ldy,
                           void* workspace, size_t workspace_bytes, void* stream) {
  if (int rc = check_fmt(format)) return rc;
  return gemv_entry(format, false, q, d, x, y, M, K, ncols, ldx, ldy, stream, workspace,
                    workspace_bytes, true);
}

QGEMV_API int qgemv_release_workspaces(void) { return release_workspaces(); }

QGEMV_API int qgemv_soa_fused(int format, const void* q, const void* d, const float* x, float* y,
                              int64_t M, int64_t K, const qgemv_fuse* fuse, void* stream) {
  if (int rc = check_fmt(format)) return rc;
  if (int rc = check_mk(M, K)) return rc;
  if (!fuse) return set_error(ERR_NULL, "fuse must not be NULL");
  if (fuse->nranks < 1 || fuse->nranks > kMaxRanks || fuse->npeer < 0 ||
      fuse->npeer > kMaxRanks - 1)
    return set_error(ERR_ARG, "nranks must be in [1, %d] and npeer in [0, %d]", kMaxRanks,
                     kMaxRanks - 1);
  if (!fuse->cta_count || !fuse->tok) return set_error(ERR_NULL, "cta_count and tok must be set");
  for (int k = 0; k < fuse->nranks; ++k)
    if (!fuse->sig_out[k]) return set_error(ERR_NULL, "sig_out[%d] is NULL", k);
  for (int k = 0; k < fuse->npeer; ++k)
    if (!fuse->peer_y[k] || misaligned(fuse->peer_y[k], 4))
      return set_error(ERR_ALIGN, "peer_y[%d] must be a 4-byte aligned device pointer", k);
  if (M == 0) return OK;
  if (!q || !d || !x || !y) return set_error(ERR_NULL, "q, d, x and y must not be NULL");
  if (misaligned(q, 16) || misaligned(d, 2) || misaligned(y, 4))
    return set_error(ERR_ALIGN, "q must be 16-byte, d 2-byte and y 4-byte aligned");
  GemvCall c;
  c.q = q;
  c.d = d;
  c.x = x;
  c.y = y;
  c.M = M;
  c.K = K;
  c.N = 1;
  c.ldx = K;
  c.ldy = M;
  if (!tma_eligible(c))
    return set_error(ERR_UNSUPPORTED,
                     "the fused all-gather needs the TMA kernel: K %% 256 == 0, 256 <= K <= 16384, "
                     "x 16-byte aligned");
  for (int k = 0; k < fuse->nranks; ++k) c.f.sig_out[k] = fuse->sig_out[k];
  for (int k = 0; k < fuse->npeer; ++k) c.f.peer_y[k] = fuse->peer_y[k];
  c.f.cta_count = fuse->cta_count;
  c.f.sig_in = fuse->sig_in;
  c.f.tok = fuse->tok;
  c.f.npeer = fuse->npeer;
  c.f.nranks = fuse->nranks;
  return gemv_soa_tma(format, c, static_cast<cudaStream_t>(stream));
}

namespace {
// Single-column GEMV with q8_1 activations (SoA planes or GGUF blocks).
int q81_entry(int format, bool aos, const void* q, const void* d, const float* x, float* y,
              int64_t M, int64_t K, void* stream) {
  if (int rc = check_fmt(format)) return rc;
  if (int rc = check_mk(M, K)) return rc;
  if (M == 0) return OK;
  if (!x || !y || !q || (!aos && !d))
    return set_error(ERR_NULL, aos ? "blocks, x and y must not be NULL"
                                   : "q, d, x and y must not be NULL");
  if (misaligned(q, 16) || (!aos && misaligned(d, 2)) || misaligned(y, 4))
    return set_error(ERR_ALIGN, aos ? "blocks must be 16-byte and y 4-byte aligned"
                                    : "q must be 16-byte, d 2-byte and y 4-byte aligned");
  GemvCall c;
  c.q = q;
  c.d = d;
  c.x = x;
  c.y = y;
  c.M = M;
  c.K = K;
  c.N = 1;
  c.ldx = K;
  c.ldy = M;
  c.act = 1;
  if (!tma_eligible(c))
    return set_error(ERR_UNSUPPORTED,
                     "q8_1 activations run on the TMA kernel only: K %% 256 == 0, "
                     "256 <= K <= 16384, x 16-byte aligned");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int rc = aos ? gemv_aos_tma(format, c, st) : gemv_soa_tma(format, c, st);
  return rc == -1 ? set_error(ERR_UNSUPPORTED, "no q8_1 kernel configuration fits this shape")
                  : rc;
}
}  // namespace

QGEMV_API int qgemv_soa_q8_1(int format, const void* q, const void* d, const float* x, float* y,
                             int64_t M, int64_t K, void* stream) {
  return q81_entry(format, false, q, d, x, y, M, K, stream);
}

QGEMV_API int qgemv_aos_q8_1(int format, const void* blocks, const float* x, float* y,
                             int64_t M, int64_t K, void* stream) {
  return q81_entry(format, true, blocks, nullptr, x, y, M, K, stream);
}

namespace {
int stack_entry(int format, const qgemv_stack_gemv* gemvs, int32_t n,
                const qgemv_stack_ranks* ranks, void** handle) {
  if (int rc = check_fmt(format)) return rc;
  if (!gemvs || !handle) return set_error(ERR_NULL, "gemvs and handle must not be NULL");
  if (n < 1 || n > 65536) return set_error(ERR_ARG, "n=%d out of range [1, 65536]", n);
  StackRanks rk;
  if (ranks) {
    if (ranks->nranks < 1 || ranks->nranks > kMaxRanks || ranks->rank < 0 ||
        ranks->rank >= ranks->nranks)
      return set_error(ERR_ARG, "nranks must be in [1, %d] and rank in [0, nranks)", kMaxRanks);
    if (ranks->nranks > 1 && !ranks->peer_y)
      return set_error(ERR_NULL, "peer_y must not be NULL with more than one rank");
    rk.nranks = ranks->nranks;
    rk.rank = ranks->rank;
  }
  std::vector<StackCall> calls(n);
  for (int j = 0; j < n; ++j) {
    const qgemv_stack_gemv& g = gemvs[j];
    if (int rc = check_mk(g.M, g.K)) return rc;
    if (!g.q || !g.d || !g.y || (j == 0 && !g.x))
      return set_error(ERR_NULL, "stack GEMV %d: NULL pointer", j);
    StackCall c;
    c.q = g.q;
    c.d = g.d;
    c.x = g.x;
    c.y = reinterpret_cast<unsigned long long*>(g.y);
    c.r0 = g.r0;
    c.M = g.M;
    c.M_total = g.M_total;
    c.K = g.K;
    for (int k = 0; k < rk.nranks - 1; ++k)
      c.peer_y[k] = reinterpret_cast<unsigned long long*>(
          ranks->peer_y[(size_t)j * (rk.nranks - 1) + k]);
    calls[j] = c;
  }
  *handle = nullptr;
  return stack_create(format, calls.data(), n, ranks ? &rk : nullptr, handle);
}
}  // namespace

QGEMV_API int qgemv_stack_create(int format, const qgemv_stack_gemv* gemvs, int32_t n,
                                 void** handle) {
  return stack_entry(format, gemvs, n, nullptr, handle);
}

QGEMV_API int qgemv_stack_create_ranks(int format, const qgemv_stack_gemv* gemvs, int32_t n,
                                       const qgemv_stack_ranks* ranks, void** handle) {
  if (!ranks) return set_error(ERR_NULL, "ranks must not be NULL");
  return stack_entry(format, gemvs, n, ranks, handle);
}

QGEMV_API int qgemv_stack_run(void* handle, void* stream) {
  if (!handle) return set_error(ERR_NULL, "handle must not be NULL");
  return stack_run(handle, static_cast<cudaStream_t>(stream));
}

QGEMV_API int qgemv_stack_reset(void* handle, void* stream) {
  if (!handle) return set_error(ERR_NULL, "handle must not be NULL");
  return stack_reset(handle, static_cast<cudaStream_t>(stream));
}

QGEMV_API int qgemv_stack_destroy(void* handle) { return stack_destroy(handle); }

QGEMV_API int qgemv_token_fence(unsigned* const* done, int32_t nranks, const unsigned* done_local,
                                unsigned* tok, void* stream) {
  if (nranks < 1 || nranks > kMaxRanks) return set_error(ERR_ARG, "nranks must be in [1, %d]", kMaxRanks);
  if (!done || !done_local || !tok) return set_error(ERR_NULL, "done, done_local and tok must be set");
  for (int k = 0; k < nranks; ++k)
    if (!done[k]) return set_error(ERR_NULL, "done[%d] is NULL", k);
  return token_fence(const_cast<unsigned* const*>(done), nranks, done_local, tok,
                     static_cast<cudaStream_t>(stream));
}

QGEMV_API int qgemv_soa_static_ws(int format, const void* q, const void* d, const float* x,
                                  float* y, int64_t M, int64_t K, int32_t ncols, int64_t ldx,
                                  int64_t ldy, void* stream) {
  if (int rc = check_fmt(format)) return rc;
  if (int rc = check_mk(M, K)) return rc;
  void* ws = nullptr;
  size_t ws_bytes = 0;
  GemvCall probe;
  probe.q = q;
  probe.d = d;
  probe.M = M;
  probe.K = K;
  probe.N = std::min(std::max(ncols, 0), 16);
  // the tcgen05 kernel where its workspace fits the array (it grows with M,
  // the column count and the SM count), else the mma.sync kernel
  bool allow_tc = false;
  if (M > 0 && probe.N >= 2 && mma_eligible(probe)) {
    allow_tc = soa_batch_workspace(probe, true) <= kStaticWsBytes;
    const size_t need = soa_batch_workspace(probe, allow_tc);
    if (need > kStaticWsBytes)
      return set_error(ERR_UNSUPPORTED,
                       "this call needs %zu bytes of workspace; the static workspace holds %zu "
                       "(K <= 32256 at 16 columns): use qgemv_soa_ws",
                       need, kStaticWsBytes);
    if (int rc = static_workspace(&ws, &ws_bytes)) return rc;
  }
  return gemv_entry(format, false, q, d, x, y, M, K, ncols, ldx, ldy, stream, ws, ws_bytes, true,
                    allow_tc);
}

QGEMV_API size_t qgemv_tiled_bytes(int format, int64_t M, int64_t K) {
  if (check_fmt(format) || check_mk(M, K)) return 0;
  return tiled_bytes(format, M, K);
}

QGEMV_API int qgemv_tile_weights(int format, int layout, const void* q, const void* d, int64_t M,
                                 int64_t K, void* tiled, void* stream) {
  if (int rc = check_fmt(format)) return rc;
  if (int rc = check_mk(M, K)) return rc;
  if (layout != 0 && layout != 1)
    return set_error(ERR_ARG, "layout must be 0 (SoA planes) or 1 (ggml blocks), got %d", layout);
  if (M == 0 || K == 0) return OK;
  if (!q || !tiled || (layout == 0 && !d))
    return set_error(ERR_NULL, "source and destination must not be NULL");
  if (misaligned(tiled, 16)) return set_error(ERR_ALIGN, "tiles must be 16-byte aligned");
  if (layout == 0 && (misaligned(q, 16) || misaligned(d, 2)))
    return set_error(ERR_ALIGN, "q must be 16-byte and d 2-byte aligned");
  return tile_weights(format, layout == 1, q, d, M, K, tiled, static_cast<cudaStream_t>(stream));
}

QGEMV_API size_t qgemv_tiled_workspace_bytes(int64_t K, int32_t ncols) {
  if (K < 0 || K % QK || ncols < 1) return 0;
  return mma_workspace_bytes(K, ncols);
}

QGEMV_API int qgemv_tiled_gemv(int format, const void* tiled, int64_t M, int64_t K,
                               const float* x, float* y, int32_t ncols, int64_t ldx, int64_t ldy,
                               void* workspace, size_t workspace_bytes, void* stream) {
  if (int rc = check_fmt(format)) return rc;
  if (int rc = check_mk(M, K)) return rc;
  if (K > ((int64_t)1 << 20))
    return set_error(ERR_UNSUPPORTED, "K=%lld above 2^20 for batch tiles", (long long)K);
  if (ncols < 0) return set_error(ERR_SHAPE, "ncols=%d is negative", ncols);
  if (M == 0 || ncols == 0) return OK;
  if (!y || (K > 0 && (!x || !tiled))) return set_error(ERR_NULL, "tiles, x and y must not be NULL");
  if (ncols > 1 && ldx < K) return set_error(ERR_SHAPE, "ldx=%lld < K=%lld", (long long)ldx, (long long)K);
  if (ncols > 1 && ldy < M) return set_error(ERR_SHAPE, "ldy=%lld < M=%lld", (long long)ldy, (long long)M);
  if (ncols == 1) {
    ldx = K;
    ldy = M;
  }
  if (K > 0 && misaligned(tiled, 16)) return set_error(ERR_ALIGN, "tiles must be 16-byte aligned");
  if (misaligned(x, 4) || misaligned(y, 4)) return set_error(ERR_ALIGN, "x and y must be 4-byte aligned");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (K == 0) return fill_zero_rows(y, M, ncols, ldy, st);
  const size_t need = mma_workspace_bytes(K, ncols);
  if (workspace) {
    if (workspace_bytes < need)
      return set_error(ERR_ARG, "this call needs a workspace of %zu bytes, got %zu", need,
                       workspace_bytes);
    if (misaligned(workspace, 16)) return set_error(ERR_ALIGN, "workspace must be 16-byte aligned");
  } else if (int rc = stream_workspace(st, need, &workspace)) {
    return rc;
  } else {
    workspace_bytes = need;
  }
  GemvCall c;
  c.q = tiled;
  c.M = M;
  c.K = K;
  c.ldx = ldx;
  c.ldy = ldy;
  c.ws = workspace;
  c.ws_bytes = workspace_bytes;
  for (int n0 = 0; n0 < ncols; n0 += 16) {
    c.N = std::min(16, ncols - n0);
    c.x = x + (int64_t)n0 * ldx;
    c.y = y + (int64_t)n0 * ldy;
    if (int rc = gemv_tiled(format, c, st)) return rc;
  }
  return OK;
}

QGEMV_API size_t qgemv_tc_bytes(int format, int64_t M, int64_t K) {
  if (check_fmt(format) || check_mk(M, K)) return 0;
  return tc_tiles_bytes(format, M, K);
}

QGEMV_API int qgemv_tc_tile(int format, int layout, const void* q, const void* d, int64_t M,
                            int64_t K, void* tiles, void* stream) {
  if (int rc = check_fmt(format)) return rc;
  if (int rc = check_mk(M, K)) return rc;
  if (layout != 0 && layout != 1)
    return set_error(ERR_ARG, "layout must be 0 (SoA planes) or 1 (ggml blocks), got %d", layout);
  if (M == 0 || K == 0) return OK;
  if (!q || !tiles || (layout == 0 && !d))
    return set_error(ERR_NULL, "source and destination must not be NULL");
  if (misaligned(tiles, 16)) return set_error(ERR_ALIGN, "tiles must be 16-byte aligned");
  if (layout == 0 && (misaligned(q, 16) || misaligned(d, 2)))
    return set_error(ERR_ALIGN, "q must be 16-byte and d 2-byte aligned");
  return tile_weights_tc(format, layout == 1, q, d, M, K, tiles, static_cast<cudaStream_t>(stream));
}

QGEMV_API size_t qgemv_tc_workspace_bytes(int64_t M, int64_t K) {
  if (check_mk(M, K)) return 0;
  DeviceInfo dev;
  if (current_device_info(dev)) return 0;
  return tc_workspace_bytes(M, K, dev.sms);
}

QGEMV_API int qgemv_tc_gemv(int format, const void* tiles, int64_t M, int64_t K, const float* x,
                            float* y, int32_t ncols, int64_t ldx, int64_t ldy, void* workspace,
                            size_t workspace_bytes, void* stream) {
  if (int rc = check_fmt(format)) return rc;
  if (int rc = check_mk(M, K)) return rc;
  if (K > ((int64_t)1 << 20))
    return set_error(ERR_UNSUPPORTED, "K=%lld above 2^20 for tc tiles", (long long)K);
  if (ncols < 0) return set_error(ERR_SHAPE, "ncols=%d is negative", ncols);
  if (M == 0 || ncols == 0) return OK;
  if (!y || (K > 0 && (!x || !tiles))) return set_error(ERR_NULL, "tiles, x and y must not be NULL");
  if (ncols > 1 && ldx < K) return set_error(ERR_SHAPE, "ldx=%lld < K=%lld", (long long)ldx, (long long)K);
  if (ncols > 1 && ldy < M) return set_error(ERR_SHAPE, "ldy=%lld < M=%lld", (long long)ldy, (long long)M);
  if (ncols == 1) {
    ldx = K;
    ldy = M;
  }
  if (K > 0 && misaligned(tiles, 16)) return set_error(ERR_ALIGN, "tiles must be 16-byte aligned");
  if (misaligned(x, 4) || misaligned(y, 4)) return set_error(ERR_ALIGN, "x and y must be 4-byte aligned");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (K == 0) return fill_zero_rows(y, M, ncols, ldy, st);
  DeviceInfo dev;
  if (int rc = current_device_info(dev)) return rc;
  const size_t need = tc_workspace_bytes(M, K, dev.sms);
  if (workspace) {
    if (workspace_bytes < need)
      return set_error(ERR_ARG, "this call needs a workspace of %zu bytes, got %zu", need,
                       workspace_bytes);
    if (misaligned(workspace, 16)) return set_error(ERR_ALIGN, "workspace must be 16-byte aligned");
  } else if (int rc = stream_workspace(st, need, &workspace)) {
    return rc;
  } else {
    workspace_bytes = need;
  }
  for (int n0 = 0; n0 < ncols; n0 += 16) {
    const int n = std::min(16, ncols - n0);
    if (int rc = gemv_tc(format, tiles, M, K, x + (int64_t)n0 * ldx, ldx, y + (int64_t)n0 * ldy,
                         ldy, n, workspace, workspace_bytes, st))
      return rc;
  }
  return OK;
}

QGEMV_API size_t qgemv_q8_0_tc_bytes(int64_t M, int64_t K) { return qgemv_tc_bytes(8, M, K); }

QGEMV_API int qgemv_q8_0_tc_tile(int layout, const void* q, const void* d, int64_t M, int64_t K,
                                 void* tiles, void* stream) {
  return qgemv_tc_tile(8, layout, q, d, M, K, tiles, stream);
}

QGEMV_API size_t qgemv_q8_0_tc_workspace_bytes(int64_t M, int64_t K) {
  return qgemv_tc_workspace_bytes(M, K);
}

QGEMV_API int qgemv_q8_0_tc(const void* tiles, int64_t M, int64_t K, const float* x, float* y,
                            int32_t ncols, int64_t ldx, int64_t ldy, void* workspace,
                            size_t workspace_bytes, void* stream) {
  return qgemv_tc_gemv(8, tiles, M, K, x, y, ncols, ldx, ldy, workspace, workspace_bytes, stream);
}

QGEMV_API int qgemv_q8_0_aos(const void* blocks, const float* x, float* y, int64_t M, int64_t K,
                             int32_t ncols, int64_t ldx, int64_t ldy, void* stream) {
  return gemv_entry(8, true, blocks, nullptr, x, y, M, K, ncols, ldx, ldy, stream);
}

QGEMV_API int qgemv_q4_0_aos(const void* blocks, const float* x, float* y, int64_t M, int64_t K,
                             int32_t ncols, int64_t ldx, int64_t ldy, void* stream) {
  return gemv_entry(4, true, blocks, nullptr, x, y, M, K, ncols, ldx, ldy, stream);
}

QGEMV_API int qgemv_quantize_soa(int format, const float* w, int64_t M, int64_t K, int64_t ldw,
                                 void* q, void* d, void* stream) {
  if (int rc = check_fmt(format)) return rc;
  if (int rc = check_mk(M, K)) return rc;
  if (M == 0 || K == 0) return OK;
  if (!w || !q || !d) return set_error(ERR_NULL, "w, q and d must not be NULL");
  if (ldw < K) return set_error(ERR_SHAPE, "ldw=%lld < K=%lld", (long long)ldw, (long long)K);
  if (misaligned(w, 4) || misaligned(d, 2))
    return set_error(ERR_ALIGN, "w must be 4-byte and d 2-byte aligned");
  return quantize(format, w, M, K, ldw, q, d, nullptr, static_cast<cudaStream_t>(stream));
}

QGEMV_API int qgemv_quantize_aos(int format, const float* w, int64_t M, int64_t K, int64_t ldw,
                                 void* blocks, void* stream) {
  if (int rc = check_fmt(format)) return rc;
  if (int rc = check_mk(M, K)) return rc;
  if (M == 0 || K == 0) return OK;
  if (!w || !blocks) return set_error(ERR_NULL, "w and blocks must not be NULL");
  if (ldw < K) return set_error(ERR_SHAPE, "ldw=%lld < K=%lld", (long long)ldw, (long long)K);
  if (misaligned(w, 4)) return set_error(ERR_ALIGN, "w must be 4-byte aligned");
  return quantize(format, w, M, K, ldw, nullptr, nullptr, blocks,
                  static_cast<cudaStream_t>(stream));
}

QGEMV_API int qgemv_dequant_soa(int format, const void* q, const void* d, float* w, int64_t M,
                                int64_t K, void* stream) {
  if (int rc = check_fmt(format)) return rc;
  if (int rc = check_mk(M, K)) return rc;
  if (M == 0 || K == 0) return OK;
  if (!q || !d || !w) return set_error(ERR_NULL, "q, d and w must not be NULL");
  if (misaligned(w, 4) || misaligned(d, 2))
    return set_error(ERR_ALIGN, "w must be 4-byte and d 2-byte aligned");
  return dequant(format, q, d, w, M, K, static_cast<cudaStream_t>(stream));
}

QGEMV_API int qgemv_repack(int format, int to_soa, void* blocks, void* q, void* d, int64_t M,
                           int64_t K, void* stream) {
  if (int rc = check_fmt(format)) return rc;
  if (to_soa != 0 && to_soa != 1) return set_error(ERR_ARG, "to_soa must be 0 or 1");
  if (int rc = check_mk(M, K)) return rc;
  if (M == 0 || K == 0) return OK;
  if (!blocks || !q || !d) return set_error(ERR_NULL, "blocks, q and d must not be NULL");
  if (misaligned(d, 2)) return set_error(ERR_ALIGN, "d must be 2-byte aligned");
  return repack(format, to_soa, blocks, q, d, M, K, static_cast<cudaStream_t>(stream));
}

QGEMV_API int qgemv_roof_stream_read(const void* buf, size_t bytes, uint32_t* sink,
                                     int32_t blocks_per_sm, void* stream) {
  if (!buf || !sink) return set_error(ERR_NULL, "buf and sink must not be NULL");
  if (bytes % 16) return set_error(ERR_SHAPE, "bytes must be a multiple of 16");
  if (misaligned(buf, 16) || misaligned(sink, 4))
    return set_error(ERR_ALIGN, "buf must be 16-byte and sink 4-byte aligned");
  if (blocks_per_sm < 1 || blocks_per_sm > 64)
    return set_error(ERR_ARG, "blocks_per_sm must be in [1, 64]");
  return roof_stream_read(buf, bytes, sink, blocks_per_sm, static_cast<cudaStream_t>(stream));
}

QGEMV_API int qgemv_roof_bulk_read(const void* buf, size_t bytes, uint32_t* sink, int* status,
                                   void* stream) {
  if (!buf || !sink || !status) return set_error(ERR_NULL, "buf, sink and status must not be NULL");
  if (bytes % 16) return set_error(ERR_SHAPE, "bytes must be a multiple of 16");
  if (misaligned(buf, 16) || misaligned(sink, 4) || misaligned(status, 4))
    return set_error(ERR_ALIGN, "buf must be 16-byte aligned; sink and status 4-byte");
  return roof_bulk_read(buf, bytes, sink, status, static_cast<cudaStream_t>(stream));
}

QGEMV_API int qgemv_roof_d2d(void* dst, const void* src, size_t bytes, void* stream) {
  if (!dst || !src) return set_error(ERR_NULL, "dst and src must not be NULL");
  const cudaError_t e =
      cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToDevice, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return set_error(ERR_CUDA, "cudaMemcpyAsync: %s", cudaGetErrorString(e));
  return OK;
}

}  // extern "C"
