// Native timing harness: the reference's time_kernel (src/bench.cu:134-156)
// rebuilt for microsecond-scale calls over rotated weight copies.
//
// The reference bracketed every launch with its own event pair and a
// synchronize, and re-read one weight buffer, so any matrix smaller than L2
// was timed from L2.  Here a run is `warmup` untimed steps and then `steps`
// timed steps issued back to back from C++ (no per-step host round trip),
// and step i of call descriptor j uses weight copy (i % ncopies_j).
//  * Interleaved mode: step i runs every call once, with a CUDA event after
//    each call; a call's device time is the gap between consecutive events
//    (exact, but an event between two launches prevents their overlap).
//  * Grouped mode: call j's launches run back to back as one group with
//    events only between groups, the way a caller streams many GEMVs; each
//    launch may then overlap its start with the previous launch's tail.
#include "qgemv_b200.h"

#include <vector>

#include "qgemv_common.cuh"
#include "qgemv_internal.h"

namespace qg {
namespace {

// layout: 0 SoA, 1 AoS, 2 SoA with q8_1 activations, 3 AoS with q8_1 activations
bool soa_layout(int layout) { return layout == 0 || layout == 2; }

int issue(const qgemv_call_desc& c, int copy, cudaStream_t st) {
  GemvCall g;
  g.q = c.q[copy];
  g.d = soa_layout(c.layout) ? c.d[copy] : nullptr;
  g.x = c.x;
  g.y = c.y;
  g.M = c.M;
  g.K = c.K;
  g.N = c.ncols;
  g.ldx = c.ncols > 1 ? c.ldx : c.K;
  g.ldy = c.ncols > 1 ? c.ldy : c.M;
  if (c.layout >= 2) {  // q8_1 activations: the TMA kernel only
    g.act = 1;
    const int rc = c.layout == 2 ? gemv_soa_tma(c.format, g, st) : gemv_aos_tma(c.format, g, st);
    return rc == -1 ? set_error(ERR_UNSUPPORTED, "q8_1 activations: shape not supported") : rc;
  }
  return c.layout == 0 ? gemv_soa(c.format, g, st) : gemv_aos(c.format, g, st);
}

struct Events {
  std::vector<cudaEvent_t> ev;
  ~Events() {
    for (cudaEvent_t e : ev) cudaEventDestroy(e);
  }
};

}  // namespace
}  // namespace qg

using namespace qg;

extern "C" QGEMV_API int qgemv_time_steps(const qgemv_call_desc* calls, int32_t ncalls,
                                          int32_t warmup, int32_t steps, int32_t grouped,
                                          void* stream, float* ms_out) {
  if (!calls || !ms_out) return set_error(ERR_NULL, "calls and ms_out must not be NULL");
  if (ncalls < 1 || ncalls > 64) return set_error(ERR_ARG, "ncalls must be in [1, 64]");
  if (warmup < 0 || steps < 1) return set_error(ERR_ARG, "need warmup >= 0 and steps >= 1");
  const int64_t nev = (int64_t)steps * ncalls + 1;
  if (nev > (1 << 22)) return set_error(ERR_ARG, "steps * ncalls must stay below 4M");
  for (int j = 0; j < ncalls; ++j) {
    const qgemv_call_desc& c = calls[j];
    if (c.format != 8 && c.format != 4) return set_error(ERR_ARG, "call %d: bad format", j);
    if (c.layout < 0 || c.layout > 3) return set_error(ERR_ARG, "call %d: bad layout", j);
    if (c.layout >= 2 && c.ncols != 1)
      return set_error(ERR_ARG, "call %d: q8_1 activations take one column", j);
    if (c.ncopies < 1 || !c.q || (soa_layout(c.layout) && !c.d))
      return set_error(ERR_NULL, "call %d: needs ncopies >= 1 weight pointers", j);
    if (c.M < 1 || c.K < QK || c.K % QK || c.M >= (1LL << 31) || c.K >= (1LL << 31))
      return set_error(ERR_SHAPE, "call %d: bad shape", j);
    if (c.ncols < 1 || !c.x || !c.y) return set_error(ERR_ARG, "call %d: bad x / y / ncols", j);
    if (c.ncols > 1 && (c.ldx < c.K || c.ldy < c.M))
      return set_error(ERR_SHAPE, "call %d: ldx < K or ldy < M", j);
    for (int k = 0; k < c.ncopies; ++k) {
      if (!c.q[k] || (reinterpret_cast<uintptr_t>(c.q[k]) & 15))
        return set_error(ERR_ALIGN, "call %d copy %d: weights must be 16-byte aligned", j, k);
      if (soa_layout(c.layout) && (!c.d[k] || (reinterpret_cast<uintptr_t>(c.d[k]) & 1)))
        return set_error(ERR_ALIGN, "call %d copy %d: bad scale pointer", j, k);
    }
  }
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  for (int i = 0; i < warmup; ++i)
    for (int j = 0; j < ncalls; ++j)
      if (int rc = issue(calls[j], i % calls[j].ncopies, st)) return rc;

  if (grouped) {
    // Call j's `steps` launches run back to back as one group (copies still
    // rotate); events only at group boundaries, so consecutive launches of a
    // group can overlap their launch and prologue with the previous tail.
    Events E;
    E.ev.resize(ncalls + 1);
    for (int j = 0; j <= ncalls; ++j) {
      const cudaError_t e = cudaEventCreate(&E.ev[j]);
      if (e != cudaSuccess) {
        E.ev.resize(j);
        return set_error(ERR_CUDA, "cudaEventCreate: %s", cudaGetErrorString(e));
      }
    }
    if (cudaStreamSynchronize(st) != cudaSuccess) return check_launch("warm-up");
    cudaEventRecord(E.ev[0], st);
    for (int j = 0; j < ncalls; ++j) {
      for (int i = 0; i < steps; ++i)
        if (int rc = issue(calls[j], i % calls[j].ncopies, st)) return rc;
      cudaEventRecord(E.ev[j + 1], st);
    }
    const cudaError_t e = cudaEventSynchronize(E.ev[ncalls]);
    if (e != cudaSuccess) return set_error(ERR_CUDA, "timed steps: %s", cudaGetErrorString(e));
    cudaEventElapsedTime(&ms_out[0], E.ev[0], E.ev[ncalls]);
    for (int j = 0; j < ncalls; ++j) cudaEventElapsedTime(&ms_out[1 + j], E.ev[j], E.ev[j + 1]);
    return check_launch("qgemv_time_steps");
  }
  Events E;
  E.ev.resize(nev);
  for (int64_t i = 0; i < nev; ++i) {
    const cudaError_t e = cudaEventCreate(&E.ev[i]);
    if (e != cudaSuccess) {
      E.ev.resize(i);
      return set_error(ERR_CUDA, "cudaEventCreate: %s", cudaGetErrorString(e));
    }
  }
  if (cudaStreamSynchronize(st) != cudaSuccess) return check_launch("warm-up");
  cudaEventRecord(E.ev[0], st);
  int64_t k = 1;
  for (int i = 0; i < steps; ++i) {
    for (int j = 0; j < ncalls; ++j) {
      if (int rc = issue(calls[j], i % calls[j].ncopies, st)) return rc;
      cudaEventRecord(E.ev[k++], st);
    }
  }
  const cudaError_t e = cudaEventSynchronize(E.ev[nev - 1]);
  if (e != cudaSuccess) return set_error(ERR_CUDA, "timed steps: %s", cudaGetErrorString(e));
  for (int j = 0; j <= ncalls; ++j) ms_out[j] = 0.0f;
  cudaEventElapsedTime(&ms_out[0], E.ev[0], E.ev[nev - 1]);
  double acc[65] = {0};
  for (int64_t i = 1; i < nev; ++i) {
    float t = 0.0f;
    cudaEventElapsedTime(&t, E.ev[i - 1], E.ev[i]);
    acc[(i - 1) % ncalls] += t;
  }
  for (int j = 0; j < ncalls; ++j) ms_out[1 + j] = (float)acc[j];
  return check_launch("qgemv_time_steps");
}
