// Test infrastructure only: wraps the reference's own host-side quantizers and
// float64 reference matvec (src/bench.cu:32-111 of the reference project) in a
// C ABI, so the oracle can be pinned against the reference's compiled code and
// the reference's CPU matvec can be timed as the CPU baseline.
//
// The reference file is compiled where it lies (the include path is given by
// oracle/Makefile); nothing of it is copied here.  Its `main` is renamed so
// the translation unit links as a shared library, and its kernels are never
// launched.

#define main qgemv_reference_bench_main
#include "bench.cu"
#undef main

#include <thread>

namespace {

template <class Block>
std::vector<Block> rows_to_vec(const void* blocks, size_t r0, size_t r1, int K) {
  const size_t nb = (size_t)K / QK;
  const Block* b = static_cast<const Block*>(blocks) + r0 * nb;
  return std::vector<Block>(b, b + (r1 - r0) * nb);
}

struct Plan {
  int fmt;  // 8 or 4
  int M, K, nthreads;
  std::vector<size_t> r0;                   // first row of each thread
  std::vector<std::vector<block_q8_0>> w8;  // per-thread row slices
  std::vector<std::vector<block_q4_0>> w4;
};

}  // namespace

extern "C" {

int ref_block_bytes(int fmt) {
  return fmt == 8 ? (int)sizeof(block_q8_0) : (int)sizeof(block_q4_0);
}

// w: fp32 [M, K] row-major.  out: M*K/32 ggml blocks.
int ref_quantize_q8_0(const float* w, int M, int K, void* out) {
  if (K % QK) return 1;
  const size_t nb = (size_t)K / QK;
  std::vector<block_q8_0> t;
  for (int r = 0; r < M; ++r) {
    quantize_q8_0(w + (size_t)r * K, K, t);
    memcpy(static_cast<block_q8_0*>(out) + (size_t)r * nb, t.data(), nb * sizeof(block_q8_0));
  }
  return 0;
}

int ref_quantize_q4_0(const float* w, int M, int K, void* out) {
  if (K % QK) return 1;
  const size_t nb = (size_t)K / QK;
  std::vector<block_q4_0> t;
  for (int r = 0; r < M; ++r) {
    quantize_q4_0(w + (size_t)r * K, K, t);
    memcpy(static_cast<block_q4_0*>(out) + (size_t)r * nb, t.data(), nb * sizeof(block_q4_0));
  }
  return 0;
}

// float64 reference matvec over ggml blocks; y: double [M].
int ref_matvec(int fmt, const void* blocks, const float* x, int M, int K, double* y) {
  if (K % QK) return 1;
  std::vector<float> hx(x, x + K);
  std::vector<double> out;
  if (fmt == 8) ref_q8(rows_to_vec<block_q8_0>(blocks, 0, M, K), hx, M, K, out);
  else ref_q4(rows_to_vec<block_q4_0>(blocks, 0, M, K), hx, M, K, out);
  memcpy(y, out.data(), (size_t)M * sizeof(double));
  return 0;
}

// Multi-threaded use of the same routine for the CPU baseline: the rows are
// split into `nthreads` contiguous slices, each owned (as the std::vector the
// reference routine takes) by one thread.  Building the plan copies the
// weights; running it only does the reference's matvec.
void* ref_plan_create(int fmt, const void* blocks, int M, int K, int nthreads) {
  if (K % QK || nthreads < 1 || M < 1) return nullptr;
  Plan* p = new Plan{fmt, M, K, nthreads, {}, {}, {}};
  for (int t = 0; t < nthreads; ++t) {
    const size_t a = (size_t)M * t / nthreads, b = (size_t)M * (t + 1) / nthreads;
    p->r0.push_back(a);
    if (fmt == 8) p->w8.push_back(rows_to_vec<block_q8_0>(blocks, a, b, K));
    else p->w4.push_back(rows_to_vec<block_q4_0>(blocks, a, b, K));
  }
  p->r0.push_back((size_t)M);
  return p;
}

int ref_plan_run(void* plan, const float* x, double* y) {
  Plan* p = static_cast<Plan*>(plan);
  if (!p) return 1;
  std::vector<float> hx(x, x + p->K);
  std::vector<std::thread> th;
  for (int t = 0; t < p->nthreads; ++t) {
    th.emplace_back([p, t, &hx, y] {
      const size_t a = p->r0[t], rows = p->r0[t + 1] - a;
      std::vector<double> out;
      if (p->fmt == 8) ref_q8(p->w8[t], hx, (int)rows, p->K, out);
      else ref_q4(p->w4[t], hx, (int)rows, p->K, out);
      memcpy(y + a, out.data(), rows * sizeof(double));
    });
  }
  for (auto& t : th) t.join();
  return 0;
}

void ref_plan_destroy(void* plan) { delete static_cast<Plan*>(plan); }

}  // extern "C"
