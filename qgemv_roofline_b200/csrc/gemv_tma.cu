// TMA-fed single-column q8_0 / q4_0 SoA GEMV for sm_100a (the hot path).
//
// Same computation as the reference's qgemv_q8_v5_soa_smem /
// qgemv_q4_v5_soa_smem (src/qgemv_kernels.cuh:264-291, 323-352), built
// around the B200 memory engine instead of per-thread loads:
//
//  * One CTA per SM, 17 warps.  Warp 0 is the producer: one lane streams
//    tiles of TR consecutive rows (quant bytes and fp16 scales, each tile
//    two contiguous 1-D bulk copies, cp.async.bulk) into an S-stage
//    shared-memory ring; completion is tracked by per-stage "full" mbarriers
//    (expect_tx) and stages are recycled through "empty" mbarriers.  With one
//    CTA per SM each CTA owns a contiguous row range (one contiguous
//    stream); with two, the CTAs claim tiles of rows at run time from a
//    per-stream counter (TmaArgs::tctr), so faster CTAs take more tiles.
//  * Warps 1..16 consume.  Consumer warp w owns K slice (w % KS) and row
//    group (w / KS); lane l of it owns one 32-weight block of that slice.
//    In the default mode (MODE 1) the lane converts its 32 x values once per
//    kernel into block fixed point, X_j = rint(x_j 2^(22-e)), kept as three
//    byte planes in registers; each block's dot with the integer quants is
//    then exact dp4a arithmetic (q8_0: the raw int8 quants; q4_0: two masks
//    per 8 nibbles and a per-block bias for the -8 offset), folded in int32
//    and scaled into an fp32 accumulator.  MODE 0 (kept for the kernel
//    ladder) unpacks quants to fp32 instead and accumulates with FFMA2.
//    R rows are processed at a time; the R partial dots are reduced across
//    the warp with a transposing butterfly (about R + 4 shuffles for R rows)
//    and stored per (row, slice) in shared memory.
//  * Programmatic dependent launch: the next launch may start once this one
//    has set up; it prefetches only weights before griddepcontrol.wait.
//  * x reaches the CTA as one bulk copy, issued by the producer right after
//    its dependency wait into the last ring stage (still empty then); the
//    consumers convert it from shared memory and release the stage, which
//    then receives its first weight tile.  Per-lane loads of x from L2 (the
//    fallback when a stage cannot hold x) cost ~2 us more per call: every
//    warp of every CTA reads the same bytes at the same moment.
//  * When a stage is released, the producer warp sums the KS slice partials
//    of each row in a fixed order (deterministic) and writes y.
//  * Every mbarrier wait is bounded (~1 s).  On a timeout the CTA raises a
//    shared abort flag so no thread waits further, the producer waits
//    (bounded) for the copies it issued, the kernel returns, and a device
//    error word (read by qgemv_check_device_error) records QGEMV_ERR_TIMEOUT.
//
// Requirements (checked on the host, otherwise the caller uses the
// register-streaming kernel): one column, K % 256 == 0 (so scale rows are
// 16-byte multiples), K <= 16384.
#include "gemv_core.cuh"
#include "qgemv_internal.h"

#include <algorithm>
#include <map>
#include <type_traits>
#include <mutex>
#include <vector>

namespace qg {

__device__ int g_device_error = 0;
// Limit of every bounded wait of the kernels in this file, in clock64 cycles
// (about 1 s by default); qgemv_set_wait_limit changes it per device.
__device__ long long g_spin_limit = 2000000000LL;

// The tile counter of a launch on stream st (device memory, no allocation),
// or null when none is free; defined with the counter pool below.
unsigned* tile_counter(int device, cudaStream_t st);

namespace {

// Consumer warps per CTA: 16 with one CTA per SM, or 8 with two CTAs per SM
// (each with half the shared-memory ring), which lets the next launch's CTA
// start streaming on an SM while this launch's CTA there drains.
constexpr int tma_threads(int cw) { return 32 * (cw + 1); }
// CTAs of `cw` consumer warps per SM: 16 consumer warps per SM in all
constexpr int tma_ctas_per_sm(int cw) { return cw >= 16 ? 1 : 16 / cw; }
constexpr int MAX_STAGES = 8;
constexpr int kPrefetchTiles = 1;  // weight tiles issued before the dependency wait (<= S - 1)
// The current wait limit, read once per wait (only on its slow path).
__device__ __forceinline__ long long spin_limit() { return *(volatile long long*)&g_spin_limit; }

__device__ __forceinline__ uint32_t saddr(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ bool mbar_try(uint32_t bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(done)
      : "r"(bar), "r"(parity)
      : "memory");
  return done != 0;
}

// try_wait with a suspend-time hint: the thread sleeps in hardware until the
// phase completes (or about 0.5 ms pass), instead of spinning on the barrier.
// Suspend-time hint of the mbarrier waits, in ns (0: plain try_wait, which the
// measurements favoured slightly; the hint changed no timing by more than 1 %).
#ifndef QG_MBAR_SUSPEND_NS
#define QG_MBAR_SUSPEND_NS 0u
#endif
__device__ __forceinline__ bool mbar_try_sleep(uint32_t bar, uint32_t parity) {
#if QG_MBAR_SUSPEND_NS == 0
  return mbar_try(bar, parity);
#else
  uint32_t done;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(done)
      : "r"(bar), "r"(parity), "r"(QG_MBAR_SUSPEND_NS)
      : "memory");
  return done != 0;
#endif
}

// Bounded wait; gives up early when another thread raised the abort flag.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag) {
  if (mbar_try_sleep(bar, parity)) return true;
  const long long t0 = clock64(), lim = spin_limit();
  while (!mbar_try_sleep(bar, parity)) {
    if (*abort_flag) return false;
    if (clock64() - t0 > lim) {
      // the error word first, then the CTA's abort flag: whoever sees the
      // flag (and fences) also sees the error word
      atomicExch(&g_device_error, (int)ERR_TIMEOUT);
      __threadfence();
      *abort_flag = 1;
      return false;
    }
  }
  return true;
}

__device__ __forceinline__ void mbar_wait_drain(uint32_t bar, uint32_t parity) {
  const long long t0 = clock64(), lim = spin_limit();
  while (!mbar_try(bar, parity) && clock64() - t0 < lim) {
  }
}

__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes,
                                         uint32_t bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
          "r"(dst),
      "l"(src), "r"(bytes), "r"(bar)
      : "memory");
}

// Loads from a 32-bit shared-window address.  volatile keeps them after the
// mbarrier wait that makes the stage's bytes visible.
__device__ __forceinline__ uint4 lds_v4(uint32_t a) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(a));
  return v;
}
__device__ __forceinline__ unsigned short lds_u16(uint32_t a) {
  unsigned short v;
  asm volatile("ld.shared.u16 %0, [%1];" : "=h"(v) : "r"(a));
  return v;
}

// Sums v[0..R) across the 32 lanes.  Afterwards lane L holds the total of row
// row_of_lane<R>(L); lanes with (L & (32 / R - 1)) == 0 are the owners.
template <int R>
__device__ __forceinline__ float reduce_rows(float (&v)[R], int lane) {
  if (R == 1) return warp_sum(v[0]);
  // Halve the set of rows at each step: lanes with the bit set keep the upper
  // half and receive their partner's copy of it.
#pragma unroll
  for (int h = R / 2, bit = 16; h >= 1; h /= 2, bit /= 2) {
    const bool up = (lane & bit) != 0;
#pragma unroll
    for (int i = 0; i < h; ++i) {
      const float keep = up ? v[i + h] : v[i];
      const float send = up ? v[i] : v[i + h];
      v[i] = keep + __shfl_xor_sync(0xffffffffu, send, bit);
    }
  }
  float s = v[0];
#pragma unroll
  for (int bit = 32 / R / 2; bit >= 1; bit /= 2) s += __shfl_xor_sync(0xffffffffu, s, bit);
  return s;
}

template <int R>
__device__ __forceinline__ int row_of_lane(int lane) {
  // bits 4, 3, ... of the lane (most significant first) select the row
  int r = 0;
#pragma unroll
  for (int h = R / 2, bit = 16; h >= 1; h /= 2, bit /= 2) r += (lane & bit) ? h : 0;
  return r;
}

// --- integer dot products -------------------------------------------------
// a: four quants (signed int8 for q8_0, unsigned bytes for q4_0 nibbles);
// b: four bytes of one plane of the fixed-point activations (planes 0-2 are
// unsigned, plane 3 is signed).
__device__ __forceinline__ int dp4a_su(uint32_t a, uint32_t b, int c) {
  int d;
  asm("dp4a.s32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
__device__ __forceinline__ int dp4a_ss(uint32_t a, uint32_t b, int c) {
  int d;
  asm("dp4a.s32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
__device__ __forceinline__ uint32_t dp4a_uu(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("dp4a.u32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
__device__ __forceinline__ int dp4a_us(uint32_t a, uint32_t b, int c) {
  int d;
  asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

// One 32-element block of x in block fixed point: X_j = rint(x_j * 2^(22-e))
// with |x_j| < 2^e, so |X_j| < 2^22.  X_j = X2 2^16 + X1 2^8 + X0 with X0, X1
// the unsigned low bytes of X_j and X2 its (signed) third byte, so the three
// planes are just bytes 0-2 of the two's-complement X_j.  pl[w][p] packs byte
// p of elements 4w..4w+3.  A block's dot with integer quants q is
// sum_p 2^(8p) * sum_w dp4a(q_w, pl[w][p]): exact in int32 per plane.
// Rounding x_j to the 2^(e-22) grid moves it by at most 2^(e-23) <=
// 2^-22 ||x_block||, so the dot of a row moves by at most
// 2^-22 * sqrt(32) * ||w|| * ||x|| ~ 1.35e-6 ||w|| ||x|| (Cauchy-Schwarz per
// block and across blocks), for any K.
constexpr int NPL = 3;

struct XPlanes {
  uint32_t pl[8][NPL];
  int e;        // block exponent (|x| < 2^e), -149 for an all-zero block
  float bias;   // 128 * sum_j X_j, for the q4_0 offset (see consumer)
  bool finite;
};

__device__ __forceinline__ void make_planes_from(const float (&v)[32], XPlanes& o);

__device__ __forceinline__ void make_planes(const float* __restrict__ xb, XPlanes& o) {
  float v[32];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float4 f = *reinterpret_cast<const float4*>(xb + 4 * i);
    v[4 * i] = f.x; v[4 * i + 1] = f.y; v[4 * i + 2] = f.z; v[4 * i + 3] = f.w;
  }
  make_planes_from(v, o);
}

__device__ __forceinline__ void make_planes_from(const float (&v)[32], XPlanes& o) {
  uint32_t amax = 0u;  // bits of max |x| (ordered like the values for non-NaN)
#pragma unroll
  for (int j = 0; j < 32; ++j) amax = max(amax, __float_as_uint(v[j]) & 0x7FFFFFFFu);
  o.finite = amax < 0x7F800000u;
  int e = -149;
  if (amax >= 0x00800000u) e = (int)(amax >> 23) - 126;  // normal: amax = 0.1m * 2^e
  else if (amax != 0u) frexpf(__uint_as_float(amax), &e);  // subnormal block maximum
  if (!o.finite) e = 0;
  o.e = e;
  int X[32];
  if (e >= -105) {
    // rint(x * 2^(22-e)) without a float-to-int conversion: |x * 2^(22-e)| < 2^22,
    // so x * 2^(22-e) + 1.5 * 2^23 lies in [2^23, 2^24), where the spacing of
    // floats is 1: the FFMA (exact product, one rounding, to nearest even)
    // rounds to the integer, which is the float's bits - 0x4B400000.
    const float sc = __uint_as_float((uint32_t)(149 - e) << 23);  // 2^(22 - e), exact
#pragma unroll
    for (int j = 0; j < 32; ++j)
      X[j] = (int)(__float_as_uint(fmaf(v[j], sc, 12582912.0f)) - 0x4B400000u);
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j) X[j] = __float2int_rn(ldexpf(v[j], 22 - e));
  }
  int sum = 0;  // exact: |sum| < 32 * 2^22
#pragma unroll
  for (int j = 0; j < 32; ++j) sum += X[j];
  o.bias = 128.0f * (float)sum;
  // bytes 0-2 of four consecutive X as three plane words: a 4 x 4 byte
  // transpose (the fourth byte is not needed), 7 PRMTs per 4 elements
#pragma unroll
  for (int w = 0; w < 8; ++w) {
    const uint32_t a = (uint32_t)X[4 * w], b = (uint32_t)X[4 * w + 1];
    const uint32_t c = (uint32_t)X[4 * w + 2], d = (uint32_t)X[4 * w + 3];
    const uint32_t t0 = __byte_perm(a, b, 0x5140);  // a0 b0 a1 b1
    const uint32_t t1 = __byte_perm(c, d, 0x5140);  // c0 d0 c1 d1
    const uint32_t t2 = __byte_perm(a, b, 0x0062);  // a2 b2 .. ..
    const uint32_t t3 = __byte_perm(c, d, 0x0062);  // c2 d2 .. ..
    o.pl[w][0] = __byte_perm(t0, t1, 0x5410);
    o.pl[w][1] = __byte_perm(t0, t1, 0x7632);
    o.pl[w][2] = __byte_perm(t2, t3, 0x5410);
  }
  if (!o.finite) {  // non-finite block: no planes, the scale makes its products NaN
#pragma unroll
    for (int w = 0; w < 8; ++w)
      for (int pl = 0; pl < NPL; ++pl) o.pl[w][pl] = 0u;
    o.bias = 0.0f;
  }
}

// The planes of one x block held in shared memory at 32-bit address xb
// (128 bytes).  A block is exactly 32 banks wide, so in natural order every
// lane of a warp would read the same 4 banks; lane l reads its eight 16-byte
// chunks in the order (i + l) & 7 instead (the 8 lanes of a quarter-warp hit 8
// different bank groups), builds the plane words in that order, and rotates
// them back by l & 7 with three conditional shifts.  The block maximum, the
// rounding and the sum do not depend on the order.
__device__ __forceinline__ void make_planes_smem(uint32_t xb, int lane, XPlanes& o) {
  float v[32];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const uint4 f = lds_v4(xb + (uint32_t)(((i + lane) & 7) << 4));
    v[4 * i] = __uint_as_float(f.x); v[4 * i + 1] = __uint_as_float(f.y);
    v[4 * i + 2] = __uint_as_float(f.z); v[4 * i + 3] = __uint_as_float(f.w);
  }
  make_planes_from(v, o);  // o.pl[i] = plane words of chunk (i + l) & 7
#pragma unroll
  for (int k = 1; k < 8; k <<= 1) {
    const bool b = (lane & k) != 0;
    uint32_t t[8][NPL];
#pragma unroll
    for (int c = 0; c < 8; ++c)
#pragma unroll
      for (int pl = 0; pl < NPL; ++pl) t[c][pl] = b ? o.pl[(c - k) & 7][pl] : o.pl[c][pl];
#pragma unroll
    for (int c = 0; c < 8; ++c)
#pragma unroll
      for (int pl = 0; pl < NPL; ++pl) o.pl[c][pl] = t[c][pl];
  }
}

// The exact integer dot of one 32-weight block with the x planes, folded to
// one float: F = S2 2^16 + (S1 2^8 + S0) (q4_0: 16 x that, minus the bias of
// the -8 offset).  wq: the block's quant words (q8_0: 8 words of int8, word w
// = elements 4w..4w+3; q4_0: 4 words, word t = elements 4t..4t+3 in the low
// nibbles and 16+4t.. in the high nibbles).
// q4_0 quant words split into nibble words: wm[t] = low nibbles of word t
// (elements 4t..4t+3), wm[4 + t] = its high nibbles in place (16 * n of
// elements 16+4t..16+4t+3).
__device__ __forceinline__ void q4_masks(const uint32_t* wq, uint32_t (&wm)[8]) {
#pragma unroll
  for (int t4 = 0; t4 < 4; ++t4) {
    wm[t4] = wq[t4] & 0x0F0F0F0Fu;
    wm[t4 + 4] = wq[t4] & 0xF0F0F0F0u;
  }
}

// block_sums for q4_0 from the nibble words of q4_masks.
__device__ __forceinline__ void block_sums_q4m(const uint32_t (&wm)[8], const XPlanes& xp, int& lo,
                                               int& hi) {
  uint32_t L0 = 0u, L1 = 0u, H0 = 0u, H1 = 0u;
  int L2 = 0, H2 = 0;
#pragma unroll
  for (int t4 = 0; t4 < 4; ++t4) {
    L0 = dp4a_uu(wm[t4], xp.pl[t4][0], L0);
    L1 = dp4a_uu(wm[t4], xp.pl[t4][1], L1);
    L2 = dp4a_us(wm[t4], xp.pl[t4][2], L2);
    H0 = dp4a_uu(wm[t4 + 4], xp.pl[t4 + 4][0], H0);
    H1 = dp4a_uu(wm[t4 + 4], xp.pl[t4 + 4][1], H1);
    H2 = dp4a_us(wm[t4 + 4], xp.pl[t4 + 4][2], H2);
  }
  // 16 * sum n X per plane (all below 2^21 in magnitude); the two low planes
  // fold in int32 (< 2^30), plane 2 stays apart
  const int S0 = (int)((L0 << 4) + H0);
  const int S1 = (int)((L1 << 4) + H1);
  lo = (S1 << 8) + S0;
  hi = (L2 << 4) + H2;
}

template <int FMT>
__device__ __forceinline__ void block_sums(const uint32_t* wq, const XPlanes& xp, int& lo, int& hi) {
  if (FMT == 4) {
    uint32_t wm[8];
    q4_masks(wq, wm);
    block_sums_q4m(wm, xp, lo, hi);
    return;
  }
  int S0 = 0, S1 = 0, S2 = 0;
#pragma unroll
  for (int w = 0; w < 8; ++w) {
    S0 = dp4a_su(wq[w], xp.pl[w][0], S0);
    S1 = dp4a_su(wq[w], xp.pl[w][1], S1);
    S2 = dp4a_ss(wq[w], xp.pl[w][2], S2);
  }
  // the two low planes fold in int32 (< 2^30); plane 2 stays apart
  lo = (S1 << 8) + S0;
  hi = S2;
}

// The block scale 2^t of a lane's x block: t = e - 22 (q4_0: - 4 more), as
// two exact power-of-two factors (each a normal float for every e), or as one
// when d * 2^t is exact for every fp16 d; NaN for a non-finite block.
//
// Fast form (fast: finite block, -100 <= t <= 80): the block's value is
// d * fma(hi, 2^(t+16), fma(lo, 2^t, -bias 2^t)), every factor a normal
// power of two (exact scalings), i.e. the fold and the scale in two FFMAs and
// one FMUL.  Each of its three roundings is at most 2^-24 times a term below
// 21 ||w_block|| ||x_block|| (q4_0; 12 for q8_0), so together under
// 4e-6 ||w|| ||x|| for a row (Cauchy-Schwarz across blocks).
struct XScale {
  float xs1, xs2, xsc;
  float xs16, xnb;  // fast form: 2^(t+16), -bias 2^t
  bool one_factor, fast;
};
template <int FMT>
__device__ __forceinline__ XScale x_scale(const XPlanes& xp) {
  XScale r;
  const int t = xp.e - 22 - (FMT == 4 ? 4 : 0), h = t / 2;
  r.xs1 = xp.finite ? __int_as_float((127 + h) << 23) : __int_as_float(0x7FC00000);
  r.xs2 = __int_as_float((127 + t - h) << 23);
  r.one_factor = t >= -100 && t <= 100;
  r.xsc = r.one_factor ? r.xs1 * r.xs2 : 0.0f;
  r.fast = xp.finite && t >= -100 && t <= 80;
  r.xs16 = r.fast ? __int_as_float((127 + 16 + t) << 23) : 0.0f;
  r.xnb = r.fast && FMT == 4 ? -xp.bias * r.xsc : 0.0f;
  return r;
}

// --- q8_1 activations (opt-in) ---------------------------------------------
// x quantized to int8 per 32-element block, the activation format of ggml's
// q8_1 route: amax = max |x|, id = 127 / amax and dx = amax / 127 (fp32,
// correctly rounded), q_j = rint(fp32(x_j * id)) in [-127, 127].  The block's
// dot with the weights is then one exact int32 dp4a sum times dw * dx; the
// error against the exact dot is that of rounding x to 8 bits per block (up
// to amax / 254 per element), far outside the exact mode's 1e-5 bound.
struct XQ81 {
  uint32_t q[8];  // word w = elements 4w..4w+3 (signed bytes)
  float dx;       // the block scale amax / 127 (0 for an all-zero block, NaN if not finite)
  float dx16;     // dx / 16 (q4_0: the in-place high nibbles count 16 n)
  int bias;       // 128 * sum_j q_j (q4_0: the -8 offset, in the 16 n units)
};

__device__ __forceinline__ void make_q81_from(const float (&v)[32], XQ81& o);

__device__ __forceinline__ void make_q81(const float* __restrict__ xb, XQ81& o) {
  float v[32];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float4 f = *reinterpret_cast<const float4*>(xb + 4 * i);
    v[4 * i] = f.x; v[4 * i + 1] = f.y; v[4 * i + 2] = f.z; v[4 * i + 3] = f.w;
  }
  make_q81_from(v, o);
}

// From shared memory, in the rotated chunk order of make_planes_smem.
__device__ __forceinline__ void make_q81_smem(uint32_t xb, int lane, XQ81& o) {
  float v[32];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const uint4 f = lds_v4(xb + (uint32_t)(((i + lane) & 7) << 4));
    v[4 * i] = __uint_as_float(f.x); v[4 * i + 1] = __uint_as_float(f.y);
    v[4 * i + 2] = __uint_as_float(f.z); v[4 * i + 3] = __uint_as_float(f.w);
  }
  make_q81_from(v, o);  // o.q[i] = quants of chunk (i + l) & 7
#pragma unroll
  for (int k = 1; k < 8; k <<= 1) {
    const bool b = (lane & k) != 0;
    uint32_t t[8];
#pragma unroll
    for (int c = 0; c < 8; ++c) t[c] = b ? o.q[(c - k) & 7] : o.q[c];
#pragma unroll
    for (int c = 0; c < 8; ++c) o.q[c] = t[c];
  }
}

__device__ __forceinline__ void make_q81_from(const float (&v)[32], XQ81& o) {
  uint32_t amax_bits = 0u;
#pragma unroll
  for (int j = 0; j < 32; ++j) amax_bits = max(amax_bits, __float_as_uint(v[j]) & 0x7FFFFFFFu);
  const bool finite = amax_bits < 0x7F800000u;
  const float amax = __uint_as_float(amax_bits);
  const bool live = finite && amax_bits != 0u;
  const float id = live ? __fdiv_rn(127.0f, amax) : 0.0f;
  o.dx = finite ? __fdiv_rn(amax, 127.0f) : __int_as_float(0x7FC00000);
  o.dx16 = o.dx * 0.0625f;
  int q[32], sum = 0;
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    // |x_j * id| <= 127 (+ rounding): adding 1.5 * 2^23 rounds the product to
    // the nearest integer (ties to even), which is the float's bits - 0x4B400000
    const float t = __fadd_rn(__fmul_rn(v[j], id), 12582912.0f);
    q[j] = live ? (int)(__float_as_uint(t) - 0x4B400000u) : 0;
    sum += q[j];
  }
  o.bias = 128 * sum;
#pragma unroll
  for (int w = 0; w < 8; ++w)
    o.q[w] = __byte_perm(__byte_perm((uint32_t)q[4 * w], (uint32_t)q[4 * w + 1], 0x0040),
                         __byte_perm((uint32_t)q[4 * w + 2], (uint32_t)q[4 * w + 3], 0x0040),
                         0x5410);
}

// One block of weights (wq as in block_sums) against q8_1 activations:
// q8_0: dw * dx * sum w q; q4_0: dw * (dx / 16) * (16 sum n q - 128 sum q).
// The integer sum is exact (|.| < 2^20) and so is its conversion.
template <int FMT>
__device__ __forceinline__ float block_q81(const uint32_t* wq, const XQ81& x8, float dw) {
  int S = 0;
  if (FMT == 8) {
#pragma unroll
    for (int w = 0; w < 8; ++w) S = dp4a_ss(wq[w], x8.q[w], S);
    return (float)S * (dw * x8.dx);
  }
  int L = 0, H = 0;
#pragma unroll
  for (int t4 = 0; t4 < 4; ++t4) {
    L = dp4a_us(wq[t4] & 0x0F0F0F0Fu, x8.q[t4], L);
    H = dp4a_us(wq[t4] & 0xF0F0F0F0u, x8.q[t4 + 4], H);
  }
  S = (L << 4) + H - x8.bias;
  return (float)S * (dw * x8.dx16);
}

// The value d * 2^t * F of one block from its plane sums (lo = S1 2^8 + S0,
// hi = S2): the fast form when it holds for every lane of the warp (FAST),
// else the general one.
template <int FMT, bool FAST>
__device__ __forceinline__ float block_value(int lo, int hi, float dv, const XScale& xq,
                                             const XPlanes& xp) {
  if (FAST) return dv * fmaf((float)hi, xq.xs16, fmaf((float)lo, xq.xsc, xq.xnb));
  float Fv = fmaf((float)hi, 65536.0f, (float)lo);
  // q4_0: 16 * sum (n - 8) X = 16 sum n X - 128 sum X; the 1/16 is in the block scale
  if (FMT == 4) Fv -= xp.bias;
  return xq.one_factor ? (dv * xq.xsc) * Fv : ((dv * Fv) * xq.xs1) * xq.xs2;
}

struct TmaArgs {
  const uint8_t* q;
  const unsigned short* d;
  const float* x;
  float* y;
  int M, K, TR, S, KS;
  // 1: x arrives by one bulk copy per CTA into the last ring stage (MODE 1
  // and 2, S >= 3, K * 4 <= stage bytes, no fused all-gather); 0: per-lane
  // loads after the dependency wait
  int xstage;
  // Tile counter of this launch (zero at entry, zero again at exit), or null:
  // null -> each CTA streams its own contiguous row range; else the matrix is
  // cut into global tiles of TR rows, CTA b takes tiles b and b + G (G CTAs)
  // and then claims tiles 2G, 2G + 1, ... with atomicAdd, so CTAs that stream
  // faster take more tiles (a shorter tail of slow CTAs).  The launch's last
  // claim (each CTA makes exactly one failing claim) resets the counter.
  unsigned* tctr;
  FuseArgs f;  // all-gather of y into peer buffers (f.nranks == 0: none)
  // Column strides (elements) of x and y when the kernel runs NC > 1 columns:
  // column n of x starts at x + n * ldx (16-byte aligned), of y at y + n * ldy.
  int64_t ldx, ldy;
};

__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void red_release_sys(unsigned* p, unsigned v) {
  asm volatile("red.release.sys.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Bounded wait until the counter at `c` reaches `target` (mod 2^32).
__device__ __forceinline__ bool wait_count(const unsigned* c, unsigned target,
                                           volatile int* abort_flag) {
  const long long t0 = clock64(), lim = spin_limit();
  while ((int)(ld_acquire_sys(c) - target) < 0) {
    if (abort_flag && *abort_flag) return false;
    if (clock64() - t0 > lim) {
      atomicExch(&g_device_error, (int)ERR_TIMEOUT);
      __threadfence();
      if (abort_flag) *abort_flag = 1;
      return false;
    }
  }
  return true;
}

// MODE 0: quants converted to fp32 with the magic-number trick and FFMA2
//         accumulation (x as fp32).
// MODE 1: x in block fixed point (three byte planes) and exact dp4a integer
//         dot products per 32-weight block, fp32 across blocks.
// MODE 2: x quantized to int8 per block (q8_1 activations, opt-in; changes
//         the numerics) and one dp4a set per block.
// AOS: the weights are ggml blocks [M][K/32] (34 / 18 bytes, d first); a tile
// of rows is then one contiguous range and each lane realigns its block from
// shared memory (MODE 1 only).
// K slices of a row (a power of two): each covers 32 units (MODE 0: 16-byte
// chunks; else 32-weight blocks)
template <int FMT, int MODE>
__host__ __device__ constexpr int slices_of(int K) {
  const int nunits = MODE == 0 ? K / Fmt<FMT>::ELEMS_PER_CHUNK : K / QK;
  int ks = 1;
  while (ks * 32 < nunits) ks *= 2;
  return ks;
}

// KF != 0: the kernel is compiled for K == KF (the row strides of the stage
// become immediate offsets of the shared-memory loads).
// NC: columns of x per launch (1, or 2 in MODE 1).  With two, every lane keeps
// the planes of its x block for both columns and runs each quant word (and,
// for q4_0, its two nibble masks) against both: the weights stream once for
// the pair, and each column's result is bit-identical to a one-column call.
template <int FMT, int MODE, int R, int CONSUMERS, bool AOS = false, int KF = 0, int NC = 1>
__global__ void __launch_bounds__(tma_threads(CONSUMERS), tma_ctas_per_sm(CONSUMERS))
k_gemv_tma(const TmaArgs p) {
  static_assert(NC == 1 || (NC == 2 && MODE == 1), "two columns: exact mode only");
  static_assert(R * NC <= 32, "one reduced value per lane at most");
  using F = Fmt<FMT>;
  constexpr int EPC = F::ELEMS_PER_CHUNK;
  extern __shared__ __align__(128) uint8_t sm[];
  __shared__ __align__(8) unsigned long long full[MAX_STAGES];
  __shared__ __align__(8) unsigned long long empty[MAX_STAGES];
  __shared__ __align__(8) unsigned long long xfull;   // staged x has arrived
  __shared__ __align__(8) unsigned long long xempty;  // every consumer has read it
  __shared__ int abort_flag;
  __shared__ uint32_t x_ready;
  __shared__ int stage_nr[MAX_STAGES];  // rows of the tile in each stage; 0: no more tiles

  const int K = KF ? KF : p.K, TR = p.TR, S = p.S;
  const int KS = KF ? slices_of<FMT, MODE>(KF) : p.KS;
  // bytes per row of the quant plane / of the scale plane (AoS: whole blocks, no plane)
  const int QB = AOS ? (K / QK) * F::BLOCK_BYTES : K / F::ROW_DIV;
  const int DB = AOS ? 0 : K / 16;
  const int STG = TR * (QB + DB);
  float* part = reinterpret_cast<float*>(sm + (size_t)S * STG);  // [S][TR][KS][NC]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int a = (int)((int64_t)p.M * blockIdx.x / gridDim.x);
  const int nrows = (int)((int64_t)p.M * (blockIdx.x + 1) / gridDim.x) - a;
  const int ntiles = (nrows + TR - 1) / TR;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(saddr(&full[s])));
      asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(saddr(&empty[s])),
                   "r"(CONSUMERS));
    }
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(saddr(&xfull)));
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(saddr(&xempty)), "r"(CONSUMERS));
    abort_flag = 0;
    x_ready = 0u;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  // Programmatic dependent launch: the next kernel on the stream may be
  // scheduled now.  It only prefetches weights before its own
  // griddepcontrol.wait, and this kernel never writes weights; x and y are
  // touched only after this kernel's own wait (below), which returns once the
  // previous kernel has completed and its writes are visible.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    int last_issued[MAX_STAGES];
    int fin_r0[MAX_STAGES];  // first row and rows of the tile in each stage
    int fin_nr[MAX_STAGES];
    for (int s = 0; s < MAX_STAGES; ++s) last_issued[s] = -1;
    bool ok = true;
    bool x_issued = false;
    int s = 0;         // stage of step t (t % S)
    uint32_t cyc = 0;  // t / S
    int end_t = -1;    // step of the end marker
    // claimed global tiles (p.tctr): static tiles b, b + G, then tiles 2G + j
    // claimed one atomic each, one step ahead of use
    const int G = gridDim.x, T = (p.M + TR - 1) / TR;
    const unsigned nclaims = (unsigned)(max(0, T - 2 * G) + G);  // each CTA fails once
    bool have_claim = false;
    unsigned claim = 0u;
    if (p.xstage && lane < NC)  // x into L2 while the previous kernel drains (a hint only)
      asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p.x + lane * p.ldx),
                   "r"((uint32_t)K * 4u)
                   : "memory");
    for (int t = 0; ok && (end_t < 0 || t < end_t + S); ++t) {
      // Tile 0 (weights only) is prefetched before the dependency wait, the
      // rest after it.  One tile, not the whole ring: x is loaded right after
      // the wait, and a CTA that starts late (its SM freed at the end of the
      // previous grid) would otherwise queue x behind the prefetched copies.
      // Measured against 2 and S - 1 tiles (x staged): 0.4-0.9 us less per
      // call from 4096 to 49152 rows, 0.4 us more for q8_0 at 98304.
      if (t == kPrefetchTiles) {
        asm volatile("griddepcontrol.wait;" ::: "memory");
        if (p.xstage) {
          // x (which may be the previous kernel's y) as one bulk copy into the
          // last stage, issued before any further weight tile; the stage
          // receives its first tile once every consumer has read x
          if (lane == 0) {
            // column n of x lands at byte n * K * 4 of the stage
            const uint32_t bar = saddr(&xfull);
            asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar),
                         "r"((uint32_t)(K * 4 * NC))
                         : "memory");
#pragma unroll
            for (int n = 0; n < NC; ++n)
              bulk_g2s(saddr(sm + (size_t)(S - 1) * STG + (size_t)n * K * 4), p.x + n * p.ldx,
                       (uint32_t)K * 4u, bar);
          }
          x_issued = true;
        }
      }
      // the tile of step t: first row r0 and rows nr (nr == 0: no more)
      int r0 = 0, nr = 0;
      if (end_t < 0) {
        if (p.tctr == nullptr) {
          r0 = a + t * TR;
          nr = t < ntiles ? min(TR, nrows - t * TR) : 0;
        } else {
          if (lane == 0) {
            int k = t < 2 ? (int)blockIdx.x + t * G : T;
            if (k >= T) {
              // claims start after the dependency wait (t >= 1): the previous
              // launch on this counter has then reset it
              const unsigned tk = have_claim ? claim : atomicAdd(p.tctr, 1u);
              have_claim = false;
              if (tk == nclaims - 1u) atomicExch(p.tctr, 0u);  // the launch's last claim
              k = 2 * G + (int)tk;
            }
            r0 = k * TR;
            nr = k < T ? min(TR, p.M - r0) : 0;
          }
          r0 = __shfl_sync(0xffffffffu, r0, 0);
          nr = __shfl_sync(0xffffffffu, nr, 0);
        }
      }
      if (x_issued && t == S - 1 && nr > 0) {
        ok = __all_sync(0xffffffffu, mbar_wait(saddr(&xempty), 0u, &abort_flag));
        if (!ok) break;
      }
      if (t >= S) {
        // the stage of step t - S (cycle cyc - 1) is released: write its rows of y;
        // every lane waits (acquire), since every lane reads the partials
        ok = __all_sync(0xffffffffu, mbar_wait(saddr(&empty[s]), (cyc - 1u) & 1u, &abort_flag));
        if (!ok) break;
        const int fr0 = fin_r0[s], fnr = fin_nr[s];
        const float* ps = part + (size_t)s * TR * KS * NC;
        for (int i = lane; i < fnr; i += 32) {
#pragma unroll
          for (int n = 0; n < NC; ++n) {
            float v = 0.0f;
            for (int k = 0; k < KS; ++k) v += ps[(i * KS + k) * NC + n];
            p.y[n * p.ldy + fr0 + i] = v;
            if (NC == 1)
              for (int k = 0; k < p.f.npeer; ++k) p.f.peer_y[k][fr0 + i] = v;  // NVLink stores
          }
        }
        __syncwarp();
        fin_nr[s] = 0;
      }
      if (end_t < 0) {
        if (nr > 0) {
          if (lane == 0) {
            const uint32_t qb = (uint32_t)nr * QB, db = (uint32_t)nr * DB;
            const uint32_t bar = saddr(&full[s]);
            uint8_t* st = sm + (size_t)s * STG;
            stage_nr[s] = nr;  // published by the arrive (release)
            asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar),
                         "r"(qb + db)
                         : "memory");
            bulk_g2s(saddr(st), p.q + (int64_t)r0 * QB, qb, bar);
            if (!AOS)
              bulk_g2s(saddr(st + (size_t)TR * QB),
                       reinterpret_cast<const uint8_t*>(p.d) + (int64_t)r0 * DB, db, bar);
            // claim the tile of step t + 1 now, so its latency overlaps the
            // wait for a free stage (after the dependency wait only)
            if (p.tctr != nullptr && t >= 1) {
              claim = atomicAdd(p.tctr, 1u);
              have_claim = true;
            }
          }
          fin_r0[s] = r0;
          fin_nr[s] = nr;
          last_issued[s] = t;
        } else {
          // no more tiles: an empty stage ends the consumers' loop
          if (lane == 0) {
            stage_nr[s] = 0;
            asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(saddr(&full[s]))
                         : "memory");
          }
          fin_nr[s] = 0;
          end_t = t;
        }
      }
      if (++s == S) {
        s = 0;
        ++cyc;
      }
    }
    if (!ok && lane == 0) {
      // aborted: wait (bounded) for every copy still in flight into our smem
      for (int s = 0; s < S; ++s)
        if (last_issued[s] >= 0)
          mbar_wait_drain(saddr(&full[s]), (uint32_t)((last_issued[s] / S) & 1));
      if (x_issued) mbar_wait_drain(saddr(&xfull), 0u);
    }
    if (p.f.nranks > 0) {
      // The CTA that finishes last tells every rank that this rank's slice of
      // y is in its buffer: each CTA orders its stores (system scope) before
      // its count; the last one orders all of them before the signals.  Every
      // CTA counts, aborted or not, so the count stays a multiple of the grid
      // per launch.  A launch that timed out (any CTA of it, or any kernel
      // since the error word was last cleared) sends no signal: the other
      // ranks then time out in their own bounded waits and report it too,
      // instead of reading a slice that was never completely written.
      __threadfence_system();
      __syncwarp();
      if (lane == 0) {
        const unsigned old = atomicAdd(p.f.cta_count, 1u);
        if (old % gridDim.x == gridDim.x - 1) {
          __threadfence_system();
          if (*(volatile int*)&g_device_error == 0)
            for (int k = 0; k < p.f.nranks; ++k) red_release_sys(p.f.sig_out[k], 1u);
        }
      }
    }
    return;
  }

  // -------------------------------------------------------------- consumers
  const int cw = warp - 1;
  const int ks = cw % KS, rg = cw / KS, RG = CONSUMERS / KS;
  const int nch = K / EPC;
  // MODE 0: a lane owns 16-byte chunk c (16 q8_0 / 32 q4_0 weights).
  // MODE 1: a lane owns 32-weight block c (32 bytes q8_0, 16 bytes q4_0).
  const int nunits = MODE == 0 ? nch : K / QK;
  const int c = ks * 32 + lane;
  const bool cval = c < nunits;
  const int cidx = cval ? c : 0;
  // AoS block of this lane: aligned word offset, and whether it starts mid-word
  const int aos_boff = cidx * F::BLOCK_BYTES;
  const int aos_off = aos_boff & ~3;
  const bool aos_odd = (aos_boff & 2) != 0;
  const uint32_t aos_sel = aos_odd ? 0x7654u : 0x5432u;

  float xr[MODE == 0 ? EPC : 1];
  XPlanes xps[NC];    // MODE 1: the planes of the lane's x block, per column
  XPlanes& xp = xps[0];
  XScale xqs[NC] = {};  // MODE 1: the scale 2^t of the lane's x block, per column
  XScale& xq = xqs[0];
  bool fast = false;  // the fast form holds for every lane of the warp (and column)
  XQ81 x8{};          // MODE 2: the lane's x block as int8 quants
  if (MODE == 0) {
    asm volatile("griddepcontrol.wait;" ::: "memory");
#pragma unroll
    for (int e = 0; e < (MODE == 0 ? EPC : 1); ++e) {
      if (FMT == 8) {
        xr[e] = cval ? p.x[cidx * 16 + e] : 0.0f;
      } else {
        // e = 8t + pos: nibble order of cvt_q4_word, divided by 2^shift
        const int t = e >> 3, pp = e & 7;
        const int jj = 4 * t + (pp >> 1) + 16 * (pp & 1);
        xr[e] = cval ? p.x[cidx * 32 + jj] * __int_as_float((127 - q4_shift(pp)) << 23) : 0.0f;
      }
    }
  } else if (p.xstage) {
    // x staged in the last ring stage by the producer (after its dependency
    // wait); every consumer warp releases the stage once it has converted x
    const bool got = __all_sync(0xffffffffu, mbar_wait(saddr(&xfull), 0u, &abort_flag));
    const uint32_t xb = saddr(sm) + (uint32_t)((S - 1) * STG + cidx * 128);
#pragma unroll
    for (int n = 0; n < NC; ++n) {
      if (MODE == 2) {
        if (got && cval) make_q81_smem(xb, lane, x8);  // lanes past K: zero quants, never stored
      } else if (got && cval) {
        make_planes_smem(xb + (uint32_t)(n * K * 4), lane, xps[n]);
      } else {
        for (int w = 0; w < 8; ++w)
          for (int pl = 0; pl < NPL; ++pl) xps[n].pl[w][pl] = 0u;
        xps[n].e = -149;
        xps[n].bias = 0.0f;
        xps[n].finite = true;
      }
    }
    __syncwarp();
    if (lane == 0)
      asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(saddr(&xempty)) : "memory");
    if (MODE == 1) {
      bool f = true;
#pragma unroll
      for (int n = 0; n < NC; ++n) {
        xqs[n] = x_scale<FMT>(xps[n]);
        f = f && xqs[n].fast;
      }
      fast = __all_sync(0xffffffffu, !cval || f);
    }
  } else {
    // Pull the lane's 128 bytes of x into L2 while the previous kernel
    // finishes (a prefetch consumes no data, so it may precede the wait; the
    // previous kernel's own writes to x still land in L2 before the loads).
    if (cval) {
#pragma unroll
      for (int n = 0; n < NC; ++n) {
        asm volatile("prefetch.global.L2 [%0];" ::"l"(p.x + n * p.ldx + cidx * 32));
        asm volatile("prefetch.global.L2 [%0];" ::"l"(p.x + n * p.ldx + cidx * 32 + 31));
      }
    }
    asm volatile("griddepcontrol.wait;" ::: "memory");  // x may be the previous kernel's y
    if (p.f.sig_in) {
      // x is assembled by every rank's previous GEMV: one signal per rank per token
      if (cw == 0 && lane == 0) {
        const unsigned target = (*(volatile const unsigned*)p.f.tok + 1u) * (unsigned)p.f.nranks;
        if (wait_count(p.f.sig_in, target, &abort_flag))
          asm volatile("st.release.cta.shared::cta.u32 [%0], %1;" ::"r"(saddr(&x_ready)), "r"(1u)
                       : "memory");
      }
      const long long t0 = clock64(), lim = 2 * spin_limit();
      for (;;) {
        uint32_t r;
        asm volatile("ld.acquire.cta.shared::cta.u32 %0, [%1];" : "=r"(r) : "r"(saddr(&x_ready))
                     : "memory");
        if (r || abort_flag || clock64() - t0 > lim) break;
      }
    }
#pragma unroll
    for (int n = 0; n < NC; ++n) {
      if (MODE == 2) {
        if (cval) make_q81(p.x + cidx * 32, x8);  // lanes past K: zero quants, never stored
      } else if (cval) {
        make_planes(p.x + n * p.ldx + cidx * 32, xps[n]);
      } else {
        for (int w = 0; w < 8; ++w)
          for (int pl = 0; pl < NPL; ++pl) xps[n].pl[w][pl] = 0u;
        xps[n].e = -149;
        xps[n].bias = 0.0f;
        xps[n].finite = true;
      }
    }
    // X_j = x_j 2^(22-e): the block's dot is its integer dot times 2^(e-22)
    // (q4_0: times 2^-4 more).  With one factor (d * 2^t exact for every fp16
    // d: all but extreme x), (d * 2^t) * F is the same correctly rounded
    // product as (d * F) * 2^t; otherwise two exact factors, so the product
    // only rounds where the true value itself under- or overflows.
    if (MODE == 1) {
      bool f = true;
#pragma unroll
      for (int n = 0; n < NC; ++n) {
        xqs[n] = x_scale<FMT>(xps[n]);
        f = f && xqs[n].fast;
      }
      fast = __all_sync(0xffffffffu, !cval || f);  // lanes past K compute nothing
    }
  }

  int s = 0;         // stage of the next tile
  uint32_t ph = 0u;  // its phase parity
  for (;;) {
    // every lane waits on the barrier, so the bulk-copied bytes are visible to it
    if (!__all_sync(0xffffffffu, mbar_wait(saddr(&full[s]), ph, &abort_flag))) break;
    const int nr = *(volatile int*)&stage_nr[s];  // rows of this stage's tile (0: done)
    if (nr <= 0) break;
    const uint8_t* st = sm + (size_t)s * STG;
    const uint8_t* sd = st + (size_t)TR * QB;
    float* ps = part + (size_t)s * TR * KS * NC;
    for (int r0 = rg * R; r0 < nr; r0 += RG * R) {
      float acc[R * NC];  // acc[r * NC + n]: row r0 + r, column n
#pragma unroll
      for (int i = 0; i < R * NC; ++i) acc[i] = 0.0f;
      if (cval) {
        // Rows r0 + r >= nr of a partial last tile read stale (in-bounds)
        // bytes of the stage; their results are never stored, and rows never
        // mix in the reduction below, so no clamping is needed.
        if (MODE == 0) {
          float dv[R];
          const uint8_t* dbase = sd + (size_t)r0 * DB + (FMT == 8 ? (cidx >> 1) : cidx) * 2;
#pragma unroll
          for (int r = 0; r < R; ++r)
            dv[r] = half_bits_to_float(*reinterpret_cast<const unsigned short*>(dbase + (size_t)r * DB));
          uint4 wv[R];
#pragma unroll
          for (int r = 0; r < R; ++r)
            wv[r] = *reinterpret_cast<const uint4*>(st + (size_t)(r0 + r) * QB + cidx * 16);
          float2 s2[R];
#pragma unroll
          for (int r = 0; r < R; ++r) s2[r] = make_float2(0.0f, 0.0f);
#pragma unroll
          for (int tw = 0; tw < 4; ++tw) {
            if (FMT == 8) {
              const float2 xa = make_float2(xr[(4 * tw) % EPC], xr[(4 * tw + 1) % EPC]);
              const float2 xb = make_float2(xr[(4 * tw + 2) % EPC], xr[(4 * tw + 3) % EPC]);
#pragma unroll
              for (int r = 0; r < R; ++r) {
                float2 ca, cb;
                cvt_q8_word(word_of(wv[r], tw), ca, cb);
                s2[r] = __ffma2_rn(ca, xa, s2[r]);
                s2[r] = __ffma2_rn(cb, xb, s2[r]);
              }
            } else {
#pragma unroll
              for (int r = 0; r < R; ++r) {
                float2 cv[4];
                cvt_q4_word(word_of(wv[r], tw), cv);
#pragma unroll
                for (int i = 0; i < 4; ++i)
                  s2[r] = __ffma2_rn(cv[i], make_float2(xr[(8 * tw + 2 * i) % EPC],
                                                        xr[(8 * tw + 2 * i + 1) % EPC]), s2[r]);
              }
            }
          }
#pragma unroll
          for (int r = 0; r < R; ++r) acc[r] = dv[r] * (s2[r].x + s2[r].y);
        } else {
          // one of two bodies for the whole pass: the fast scale form when it
          // holds for every lane's block (a warp-uniform branch), else the general one
          // SoA: the lane's quants and scale of row r0 + r, as 32-bit shared
          // addresses stepped by the row strides (one add per row each)
          const uint32_t qa0 =
              saddr(sm) + (uint32_t)(s * STG + r0 * QB + cidx * (FMT == 8 ? 32 : 16));
          const uint32_t da0 = saddr(sm) + (uint32_t)(s * STG + TR * QB + r0 * DB + cidx * 2);
          auto rows = [&](auto fast_c) {
            constexpr bool FAST = decltype(fast_c)::value;
            uint32_t qa = qa0, da = da0;
#pragma unroll
          for (int r = 0; r < R; ++r) {
            constexpr int QW = FMT == 8 ? 8 : 4;  // quant words per block
            uint32_t wq[QW];
            float dvr;
            if (AOS) {
              // the lane's block starts at byte cidx * (34|18) of the row
              // (2-byte aligned; rows start on 16-byte boundaries); read the
              // aligned words covering it and realign the quants with PRMT.
              const uint32_t* src =
                  reinterpret_cast<const uint32_t*>(st + (size_t)(r0 + r) * QB + aos_off);
              uint32_t wd[QW + 1];
#pragma unroll
              for (int i = 0; i <= QW; ++i) wd[i] = src[i];
              dvr = half_bits_to_float((unsigned short)(aos_odd ? (wd[0] >> 16) : (wd[0] & 0xFFFFu)));
#pragma unroll
              for (int i = 0; i < QW; ++i) wq[i] = __byte_perm(wd[i], wd[i + 1], aos_sel);
            } else {
              dvr = half_bits_to_float(lds_u16(da));
              da += DB;
              // q8_0: 32 signed quants, word w = elements 4w..4w+3.  q4_0: 16
              // bytes, word t = elements 4t..4t+3 (low nibbles) and
              // 16+4t..16+4t+3 (high nibbles, taken in place as 16 * n)
              const uint4 u0 = lds_v4(qa);
              wq[0] = u0.x; wq[1] = u0.y; wq[2] = u0.z; wq[3] = u0.w;
              if (FMT == 8) {
                const uint4 u1 = lds_v4(qa + 16);
                wq[4 % QW] = u1.x; wq[5 % QW] = u1.y; wq[6 % QW] = u1.z; wq[7 % QW] = u1.w;
              }
              qa += QB;
            }
            if (MODE == 2) {
              acc[r] = block_q81<FMT>(wq, x8, dvr);
            } else if (NC == 1) {
              int lo, hi;
              block_sums<FMT>(wq, xp, lo, hi);
              acc[r] = block_value<FMT, FAST>(lo, hi, dvr, xq, xp);
            } else {
              // the same quant words (q4_0: masked once) against each column's planes
              uint32_t wm[8];
              if (FMT == 4) q4_masks(wq, wm);
#pragma unroll
              for (int n = 0; n < NC; ++n) {
                int lo, hi;
                if (FMT == 4) block_sums_q4m(wm, xps[n], lo, hi);
                else block_sums<FMT>(wq, xps[n], lo, hi);
                acc[r * NC + n] = block_value<FMT, FAST>(lo, hi, dvr, xqs[n], xps[n]);
              }
            }
          }
          };
          if (MODE == 2 || !fast) rows(std::false_type{});
          else rows(std::true_type{});
        }
      }
      const float v = reduce_rows<R * NC>(acc, lane);
      const int rn = row_of_lane<R * NC>(lane);  // r * NC + n
      const int r = rn / NC, n = rn % NC;
      if ((lane & (32 / (R * NC) - 1)) == 0 && r0 + r < nr) ps[((r0 + r) * KS + ks) * NC + n] = v;
    }
    __syncwarp();
    if (lane == 0)
      asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(saddr(&empty[s])) : "memory");
    if (++s == S) {
      s = 0;
      ph ^= 1u;
    }
  }
}

// ------------------------------------------------- persistent decode stack
// One cooperative launch per decode token runs a whole sequence of
// single-column GEMVs (QKV, O, gate+up, down per layer), GEMV j reading GEMV
// j-1's full output, on each of P ranks (one GPU each; P = 1 on one GPU).
// Every rank holds rows of every matrix; one CTA per SM holds a row slice of
// each rank-slice.  Warps of a CTA:
//  * warp 0, producer: streams the weight tiles of GEMV 0, 1, 2, ... through
//    one shared-memory ring without pausing at GEMV boundaries (weights never
//    depend on x), so the next matrices' tiles are in shared memory while the
//    current GEMV waits for its input; when the consumers release a tile it
//    sums the slice partials of each row and stores the row into this rank's
//    output and into every other rank's (peer pointers, NVLink);
//  * warps 1..16, consumers: load x (waiting for it, see below) into shared
//    memory, then run the arithmetic of k_gemv_tma (x in three byte planes,
//    exact dp4a block dots).
// Outputs are 8-byte slots: the row's fp32 bits in the low word and a tag in
// the high word, tag = token * n + j + 1 for GEMV j, written by one 64-bit
// store (single-copy atomic).  A reader of GEMV j's output polls each slot
// until its tag is the expected one, so the slot's value is the one written
// with that tag: no fence, flag or counter is needed between ranks or CTAs
// (the scheme of NCCL's low-latency protocol).  Every CTA has rows in every
// GEMV (the host keeps the grid at most the smallest per-rank row count), so
// a complete input of GEMV j+1 also shows that every CTA of every rank has
// finished reading the inputs of GEMV j and earlier: a buffer is rewritten
// only after every reader is done with it.  The last CTA of the launch to
// finish waits until the last GEMV's output is complete on this rank and
// advances the token count.  All waits are bounded (QGEMV_ERR_TIMEOUT).
struct StackGemv {
  const uint8_t* q;                   // this rank's rows: quant plane
  const unsigned short* d;            // scale plane
  const float* x;                     // GEMV 0: its input floats (other GEMVs: unused)
  unsigned long long* y;              // this GEMV's output slots on this rank (M_total)
  unsigned long long* peer_y[kMaxRanks - 1];  // the same slots on the other ranks
  int r0, M, M_total, K, TR, KS;      // this rank's rows [r0, r0 + M) of M_total
};
struct StackArgs {
  const StackGemv* g;
  int n;
  unsigned* ctr;  // this rank's [token count, CTAs done]
  int npeer;
  int S, SB, PB, XB;  // ring stages, bytes per stage, partial floats per stage, x bytes
};

constexpr int kStackConsumers = 16;
constexpr int kStackXChunk = 4096;  // x elements staged in shared memory at a time
constexpr int kStackThreads = 32 * (kStackConsumers + 1);

__device__ __forceinline__ void st_slot(unsigned long long* p, float v, unsigned tag) {
  const unsigned long long s = ((unsigned long long)tag << 32) | __float_as_uint(v);
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(s) : "memory");
}
__device__ __forceinline__ ulonglong2 ld_slots2(const unsigned long long* p) {
  ulonglong2 v;
  asm volatile("ld.relaxed.sys.global.v2.u64 {%0, %1}, [%2];" : "=l"(v.x), "=l"(v.y) : "l"(p)
               : "memory");
  return v;
}

// Bounded wait until slots [i, i + 2) carry `tag` (no copy).
__device__ __forceinline__ bool wait_tag2(const unsigned long long* src, int i, unsigned tag,
                                          volatile int* abort_flag) {
  long long t0 = -1, lim = 0;
  for (;;) {
    const ulonglong2 v = ld_slots2(src + i);
    if ((unsigned)(v.x >> 32) == tag && (unsigned)(v.y >> 32) == tag) return true;
    if (*abort_flag) return false;
    if (t0 < 0) {
      t0 = clock64();
      lim = spin_limit();
    } else if (clock64() - t0 > lim) {
      atomicExch(&g_device_error, (int)ERR_TIMEOUT);
      __threadfence();
      *abort_flag = 1;
      return false;
    }
  }
}

// One consumer thread's share of x from slots: pairs i = i0, i0 + step, ...
// below K (at most kMaxPairs of them), each stored into xs once its tag is
// `tag`.  Every pass issues all pending loads at once; between passes the
// thread sleeps briefly, so the waiting CTAs do not flood L2 with polls while
// the producers' rows are still on their way.  Bounded.
constexpr int kMaxPairs = 16;  // K <= 16384 with 512 consumer threads
__device__ __forceinline__ bool load_slots(const unsigned long long* src, int i0, int step, int K,
                                           unsigned tag, float* xs, volatile int* abort_flag) {
  uint32_t pending = 0;
#pragma unroll
  for (int v = 0; v < kMaxPairs; ++v)
    if (i0 + v * step < K) pending |= 1u << v;
  long long t0 = -1, lim = 0;
  while (pending) {
#pragma unroll
    for (int v = 0; v < kMaxPairs; ++v) {
      if (pending & (1u << v)) {
        const int i = i0 + v * step;
        const ulonglong2 w = ld_slots2(src + i);
        if ((unsigned)(w.x >> 32) == tag && (unsigned)(w.y >> 32) == tag) {
          xs[i] = __uint_as_float((unsigned)w.x);
          xs[i + 1] = __uint_as_float((unsigned)w.y);
          pending &= ~(1u << v);
        }
      }
    }
    if (!pending) break;
    if (*abort_flag) return false;
    if (t0 < 0) {
      t0 = clock64();
      lim = spin_limit();
    } else if (clock64() - t0 > lim) {
      atomicExch(&g_device_error, (int)ERR_TIMEOUT);
      __threadfence();
      *abort_flag = 1;
      return false;
    }
    __nanosleep(200);
  }
  return true;
}

// R rows of one lane's block from SoA planes in shared memory (quants at
// 32-bit address qa, scale at da, row strides QB / DB): the exact dot of each
// row's block with the lane's x planes, scaled.
template <int FMT, int R, bool FAST>
__device__ __forceinline__ void soa_rows(uint32_t qa, uint32_t da, int QB, int DB,
                                         const XPlanes& xp, const XScale& xq, float (&acc)[R]) {
#pragma unroll
  for (int r = 0; r < R; ++r) {
    constexpr int QW = FMT == 8 ? 8 : 4;
    uint32_t wq[QW];
    const float dvr = half_bits_to_float(lds_u16(da));
    da += DB;
    const uint4 u0 = lds_v4(qa);
    wq[0] = u0.x; wq[1] = u0.y; wq[2] = u0.z; wq[3] = u0.w;
    if (FMT == 8) {
      const uint4 u1 = lds_v4(qa + 16);
      wq[4 % QW] = u1.x; wq[5 % QW] = u1.y; wq[6 % QW] = u1.z; wq[7 % QW] = u1.w;
    }
    qa += QB;
    int lo, hi;
    block_sums<FMT>(wq, xp, lo, hi);
    acc[r] = block_value<FMT, FAST>(lo, hi, dvr, xq, xp);
  }
}

template <int FMT, int R>
__global__ void __launch_bounds__(kStackThreads, 1) k_gemv_stack(const __grid_constant__ StackArgs p) {
  constexpr int CONSUMERS = kStackConsumers;
  using F = Fmt<FMT>;
  extern __shared__ __align__(128) uint8_t sm[];
  __shared__ __align__(8) unsigned long long full[MAX_STAGES];
  __shared__ __align__(8) unsigned long long empty[MAX_STAGES];
  __shared__ __align__(8) unsigned long long xload;  // every consumer warp has stored its part of x
  __shared__ __align__(8) unsigned long long xconv;  // every consumer warp has its planes
  __shared__ int abort_flag;

  const int S = p.S, G = gridDim.x, b = blockIdx.x;
  float* part = reinterpret_cast<float*>(sm + (size_t)S * p.SB);
  float* xs = reinterpret_cast<float*>(sm + (size_t)S * p.SB + (size_t)S * p.PB * 4);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(saddr(&full[s])));
      asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(saddr(&empty[s])),
                   "r"(CONSUMERS));
    }
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(saddr(&xload)), "r"(CONSUMERS));
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(saddr(&xconv)), "r"(CONSUMERS));
    abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  // tag of GEMV j of this token
  const unsigned tok = *(volatile const unsigned*)&p.ctr[0];
  const unsigned tag0 = tok * (unsigned)p.n + 1u;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    // issue cursor (ji, ti) and finalize cursor (jf, tf) over (GEMV, tile).
    // Each cursor keeps its GEMV's parameters in registers, read once (through
    // the read-only path) when the cursor moves to the next GEMV: the
    // descriptors live in global memory, and reloading them for every tile
    // put a global-memory round trip on the producer's per-tile path.
    struct Cur {
      int j, t, a, nrows, ntiles, TR, KS, K, r0;
      const uint8_t* q;
      const uint8_t* d;
      unsigned long long* y;
    };
    auto load_cur = [&](Cur& c, int j) {
      c.j = j;
      c.t = 0;
      if (j >= p.n) return;
      const StackGemv* g = p.g + j;
      const int M = __ldg(&g->M);
      c.TR = __ldg(&g->TR);
      c.KS = __ldg(&g->KS);
      c.K = __ldg(&g->K);
      c.r0 = __ldg(&g->r0);
      c.q = reinterpret_cast<const uint8_t*>(__ldg(reinterpret_cast<const unsigned long long*>(&g->q)));
      c.d = reinterpret_cast<const uint8_t*>(__ldg(reinterpret_cast<const unsigned long long*>(&g->d)));
      c.y = reinterpret_cast<unsigned long long*>(__ldg(reinterpret_cast<const unsigned long long*>(&g->y)));
      c.a = (int)((int64_t)M * b / G);
      c.nrows = (int)((int64_t)M * (b + 1) / G) - c.a;
      c.ntiles = (c.nrows + c.TR - 1) / c.TR;
    };
    Cur ci, cf;
    load_cur(ci, 0);
    load_cur(cf, 0);
    unsigned long long* peer_base[kMaxRanks - 1];  // finalize cursor's peer slots
    const int npeer = p.npeer;
    for (int k = 0; k < npeer; ++k)
      peer_base[k] = reinterpret_cast<unsigned long long*>(
          __ldg(reinterpret_cast<const unsigned long long*>(&p.g[0].peer_y[k])));
    uint32_t u = 0, f = 0;
    int last_issued[MAX_STAGES];
    for (int s = 0; s < MAX_STAGES; ++s) last_issued[s] = -1;
    bool ok = true;
    for (;;) {
      // issue while the ring has room
      while (ci.j < p.n && u - f < (uint32_t)S) {
        if (ci.t >= ci.ntiles) {
          load_cur(ci, ci.j + 1);
          continue;
        }
        if (lane == 0) {
          const int s = (int)(u % (uint32_t)S);
          const int QB = ci.K / F::ROW_DIV, DB = ci.K / 16;
          const int r0 = ci.t * ci.TR, nr = min(ci.TR, ci.nrows - r0);
          const uint32_t bar = saddr(&full[s]);
          uint8_t* st = sm + (size_t)s * p.SB;
          asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar),
                       "r"((uint32_t)nr * (QB + DB))
                       : "memory");
          bulk_g2s(saddr(st), ci.q + (int64_t)(ci.a + r0) * QB, (uint32_t)nr * QB, bar);
          bulk_g2s(saddr(st + (size_t)ci.TR * QB), ci.d + (int64_t)(ci.a + r0) * DB,
                   (uint32_t)nr * DB, bar);
          last_issued[s] = (int)u;
        }
        ++ci.t;
        ++u;
      }
      if (cf.j >= p.n) break;
      if (cf.t < cf.ntiles) {
        // finalize tile f: the consumers are done with it; store its rows
        const int s = (int)(f % (uint32_t)S);
        ok = __all_sync(0xffffffffu, mbar_wait(saddr(&empty[s]), (f / (uint32_t)S) & 1u,
                                               &abort_flag));
        if (!ok) break;
        const int TR = cf.TR, KS = cf.KS;
        const int r0 = cf.t * TR, nr = min(TR, cf.nrows - r0);
        const int row0 = cf.r0 + cf.a + r0;
        const float* ps = part + (size_t)s * p.PB;
        const unsigned tag = tag0 + (unsigned)cf.j;
        for (int i = lane; i < nr; i += 32) {  // partials [KS][TR]: conflict-free
          float v = 0.0f;
          for (int k = 0; k < KS; ++k) v += ps[k * TR + i];
          st_slot(cf.y + row0 + i, v, tag);
          for (int k = 0; k < npeer; ++k) st_slot(peer_base[k] + row0 + i, v, tag);  // NVLink
        }
        __syncwarp();
        ++cf.t;
        ++f;
      }
      if (cf.t >= cf.ntiles) {
        load_cur(cf, cf.j + 1);
        if (cf.j < p.n)
          for (int k = 0; k < npeer; ++k)
            peer_base[k] = reinterpret_cast<unsigned long long*>(
                __ldg(reinterpret_cast<const unsigned long long*>(&p.g[cf.j].peer_y[k])));
      }
    }
    if (!ok) {
      if (lane == 0)
        for (int s = 0; s < S; ++s)
          if (last_issued[s] >= 0)
            mbar_wait_drain(saddr(&full[s]), (uint32_t)((last_issued[s] / S) & 1));
      return;
    }
    // end of the token: the last CTA of this launch waits until the last
    // GEMV's output is complete on this rank, then advances the token count
    unsigned old = 0;
    if (lane == 0) old = atomicAdd(&p.ctr[1], 1u);
    old = __shfl_sync(0xffffffffu, old, 0);
    if (old == (unsigned)G - 1u) {
      const StackGemv& g = p.g[p.n - 1];
      const unsigned tag = tag0 + (unsigned)(p.n - 1);
      bool done = true;
      for (int i = 2 * lane; i < g.M_total && done; i += 64)
        done = wait_tag2(g.y, i, tag, &abort_flag);
      if (__all_sync(0xffffffffu, done) && lane == 0) {
        atomicExch(&p.ctr[1], 0u);
        atomicExch(&p.ctr[0], tok + 1u);
        __threadfence();
      }
    }
    return;
  }

  // -------------------------------------------------------------- consumers
  const int cw = warp - 1, ct = threadIdx.x - 32;  // consumer warp / thread
  uint32_t u = 0, xph = 0;  // tiles consumed; x chunks staged (xload / xconv phases)
  for (int j = 0; j < p.n; ++j) {
    // this GEMV's parameters in registers (the asm statements below clobber
    // memory, so fields read through p.g would be reloaded in every pass)
    const int K = p.g[j].K, TR = p.g[j].TR, KS = p.g[j].KS, Mj = p.g[j].M;
    const float* gx = p.g[j].x;
    const unsigned long long* gsrc = j > 0 ? p.g[j - 1].y : nullptr;
    const int ks = cw % KS, rg = cw / KS, RG = CONSUMERS / KS;
    const int QB = K / F::ROW_DIV, DB = K / 16;
    const int a = (int)((int64_t)Mj * b / G);
    const int nrows = (int)((int64_t)Mj * (b + 1) / G) - a;
    const int ntiles = (nrows + TR - 1) / TR;
    const int c = ks * 32 + lane;
    const bool cval = c < K / QK;
    const int cidx = cval ? c : 0;
    // x of GEMV j into shared memory, kStackXChunk elements at a time (a small
    // staging area leaves room for a deeper weight ring): GEMV 0 reads its
    // input floats; GEMV j > 0 reads GEMV j-1's output slots, each once its
    // tag shows this token's value.  Each lane converts its block when the
    // chunk holding it is staged.  (mbarriers with bounded waits, not named
    // barriers: a warp that gives up must not leave the others waiting
    // without limit.)
    XPlanes xp;
    for (int w = 0; w < 8; ++w)
      for (int pl = 0; pl < NPL; ++pl) xp.pl[w][pl] = 0u;
    xp.e = -149;
    xp.bias = 0.0f;
    xp.finite = true;
    for (int k0 = 0; k0 < K; k0 += kStackXChunk, ++xph) {
      const int kn = min(kStackXChunk, K - k0);
      bool ok = true;
      if (j == 0) {
        for (int i = 4 * ct; i < kn; i += 4 * 32 * CONSUMERS)
          *reinterpret_cast<float4*>(xs + i) = *reinterpret_cast<const float4*>(gx + k0 + i);
      } else {
        ok = load_slots(gsrc + k0, 2 * ct, 2 * 32 * CONSUMERS, kn, tag0 + (unsigned)(j - 1), xs,
                        &abort_flag);
      }
      if (!__all_sync(0xffffffffu, ok)) return;
      if (lane == 0)
        asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(saddr(&xload)) : "memory");
      if (!__all_sync(0xffffffffu, mbar_wait(saddr(&xload), xph & 1u, &abort_flag))) return;
      const int e0 = cidx * QK - k0;  // the lane's block inside this chunk?
      if (cval && e0 >= 0 && e0 < kn) make_planes_smem(saddr(xs) + (uint32_t)(e0 * 4), lane, xp);
      // every consumer has its planes before the next chunk overwrites xs
      __syncwarp();
      if (lane == 0)
        asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(saddr(&xconv)) : "memory");
      if (!__all_sync(0xffffffffu, mbar_wait(saddr(&xconv), xph & 1u, &abort_flag))) return;
    }
    const XScale xq = x_scale<FMT>(xp);
    const bool fast = __all_sync(0xffffffffu, !cval || xq.fast);  // as in k_gemv_tma
    for (int t = 0; t < ntiles; ++t, ++u) {
      const int s = (int)(u % (uint32_t)S);
      if (!__all_sync(0xffffffffu, mbar_wait(saddr(&full[s]), (u / (uint32_t)S) & 1u,
                                             &abort_flag)))
        return;
      const int nr = min(TR, nrows - t * TR);
      const uint32_t sbase = saddr(sm) + (uint32_t)(s * p.SB);
      float* ps = part + (size_t)s * p.PB;
      for (int r0 = rg * R; r0 < nr; r0 += RG * R) {
        float acc[R];
#pragma unroll
        for (int r = 0; r < R; ++r) acc[r] = 0.0f;
        if (cval) {
          // rows beyond nr read stale in-bounds bytes; never stored.  The
          // lane's quants and scale of row r0 + r as 32-bit shared addresses
          // stepped by the row strides, as in k_gemv_tma.
          const uint32_t qa = sbase + (uint32_t)(r0 * QB + cidx * (FMT == 8 ? 32 : 16));
          const uint32_t da = sbase + (uint32_t)(TR * QB + r0 * DB + cidx * 2);
          if (fast) soa_rows<FMT, R, true>(qa, da, QB, DB, xp, xq, acc);
          else soa_rows<FMT, R, false>(qa, da, QB, DB, xp, xq, acc);
        }
        const float v = reduce_rows<R>(acc, lane);
        const int r = row_of_lane<R>(lane);
        if ((lane & (32 / R - 1)) == 0 && r0 + r < nr) ps[ks * TR + r0 + r] = v;
      }
      __syncwarp();
      if (lane == 0)
        asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(saddr(&empty[s])) : "memory");
    }
  }
}

struct TmaPlan {
  int grid, TR, S, KS;
  size_t smem;
};

struct PlanKey {
  const void* f;
  int dev, M, K;
  bool operator<(const PlanKey& o) const {
    return f != o.f ? f < o.f : dev != o.dev ? dev < o.dev : M != o.M ? M < o.M : K < o.K;
  }
};
std::mutex g_plan_mu;
std::map<PlanKey, TmaPlan> g_plans;

// Tile rows, stages and grid for one (kernel, device, M, K); cached, so a
// launch costs one map lookup besides the launch itself.
template <int FMT, int MODE, int R, int CONSUMERS, bool AOS = false, int NC = 1>
int plan_tma(const void* kern, int M, int K, const DeviceInfo& dev, TmaPlan* out) {
  const PlanKey key{kern, dev.device, M, K};
  {
    std::lock_guard<std::mutex> lk(g_plan_mu);
    auto it = g_plans.find(key);
    if (it != g_plans.end()) {
      *out = it->second;
      return OK;
    }
  }
  using F = Fmt<FMT>;
  const int nunits = MODE == 0 ? K / F::ELEMS_PER_CHUNK : K / QK;
  int KS = 1;
  while (KS * 32 < nunits) KS *= 2;
  if (KS > CONSUMERS) return -1;
  const int RG = CONSUMERS / KS;
  const int row_bytes = AOS ? (K / QK) * F::BLOCK_BYTES : K / F::ROW_DIV + K / 16;
  const int unit = RG * R;
  const int ctas_per_sm = tma_ctas_per_sm(CONSUMERS);
  if (int rc = allow_max_smem(kern, dev)) return rc;
  cudaFuncAttributes fa;
  if (cudaFuncGetAttributes(&fa, kern) != cudaSuccess) return check_launch("cudaFuncGetAttributes");
  // shared memory of one CTA when `ctas_per_sm` must fit on an SM (1 KB of
  // each CTA's share is reserved by the hardware)
  const int avail = (ctas_per_sm == 1 ? dev.smem_optin : (228 * 1024) / ctas_per_sm - 1024) -
                    (int)fa.sharedSizeBytes;
  const int tile_target = ctas_per_sm == 1 ? 32 * 1024 : 36 * 1024;
  int TR = unit * std::max(1, tile_target / (unit * row_bytes));
  // per stage: the tile, and the partial sums of its rows per slice and column
  const int part_row = KS * 4 * NC;
  int S = std::min(MAX_STAGES, avail / (TR * row_bytes + TR * part_row));
  while (S < 2 && TR > unit) {  // very long rows: fewer rows per tile
    TR -= unit;
    S = std::min(MAX_STAGES, avail / (TR * row_bytes + TR * part_row));
  }
  if (S < 2) return -1;
  const int xbytes = K * 4 * NC;  // x, every column
  if (MODE != 0 && TR * row_bytes < xbytes) {
    // x is staged in a ring stage: more rows per tile, if three stages still fit
    const int TRx = unit * ((xbytes + unit * row_bytes - 1) / (unit * row_bytes));
    const int Sx = std::min(MAX_STAGES, avail / (TRx * row_bytes + TRx * part_row));
    if (Sx >= 3) {
      TR = TRx;
      S = Sx;
    }
  }
  TmaPlan pl;
  pl.TR = TR;
  pl.S = S;
  pl.KS = KS;
  pl.smem = (size_t)S * (TR * row_bytes + TR * part_row);
  pl.grid = std::max(1, std::min(dev.sms * ctas_per_sm, (M + TR - 1) / TR));
  std::lock_guard<std::mutex> lk(g_plan_mu);
  g_plans[key] = pl;
  *out = pl;
  return OK;
}

template <int FMT, int MODE, int R, int CONSUMERS, bool AOS = false, int KF = 0, int NC = 1>
int launch_tma(const GemvCall& c, const DeviceInfo& dev, cudaStream_t st) {
  if (KF != 0 && c.K != KF) return -1;
  auto kern = k_gemv_tma<FMT, MODE, R, CONSUMERS, AOS, KF, NC>;
  const int K = (int)c.K, M = (int)c.M;
  TmaPlan pl;
  if (int rc = plan_tma<FMT, MODE, R, CONSUMERS, AOS, NC>(reinterpret_cast<const void*>(kern), M,
                                                           K, dev, &pl))
    return rc;
  const int grid = c.grid_override > 0 ? c.grid_override : pl.grid;
  using F = Fmt<FMT>;
  const int64_t stage_bytes =
      (int64_t)pl.TR * (AOS ? (K / QK) * F::BLOCK_BYTES : K / F::ROW_DIV + K / 16);
  // x by one bulk copy per CTA: measured 1.8-2.6 us less per call than
  // per-lane loads of x (every warp of every CTA reading the same 16 KB at
  // the same moment), from 4096 to 98304 rows of K = 4096
  const int xstage =
      MODE != 0 && c.f.nranks == 0 && pl.S >= 3 && (int64_t)K * 4 * NC <= stage_bytes;
  TmaArgs a{static_cast<const uint8_t*>(c.q), static_cast<const unsigned short*>(c.d), c.x, c.y,
            M, K, pl.TR, pl.S, pl.KS, xstage,
            // claimed tiles with two CTAs per SM (measured 2-5 % less per call
            // at 12288-49152 rows, decode stack q4_0 -6 %); with one CTA per SM
            // its lone producer stalls on the claims' latency (q8_0 98304 x 4096
            // 65.3 -> 68.9 us), so those launches keep contiguous ranges.  A grid
            // forced above the tile count (qgemv_soa_variant) is static too: a
            // CTA without a first tile would claim before its dependency wait.
            CONSUMERS < 16 && grid <= (M + pl.TR - 1) / pl.TR ? tile_counter(dev.device, st)
                                                             : nullptr,
            c.f, NC > 1 ? c.ldx : (int64_t)K, NC > 1 ? c.ldy : (int64_t)M};
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(tma_threads(CONSUMERS));
  cfg.dynamicSmemBytes = pl.smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, a);
  if (e != cudaSuccess) return set_error(ERR_CUDA, "k_gemv_tma launch: %s", cudaGetErrorString(e));
  return check_launch("k_gemv_tma");
}

}  // namespace

// ------------------------------------------------------ tile counters
// One counter per stream (by its unique stream id) and one per launch made
// under stream capture (baked into the graph; replays of one executable
// graph are ordered), from a fixed device array: no allocation.  A launch
// claims tiles only after its dependency wait, when the previous launch
// on the same counter has finished and reset it.  Without a free counter
// the launch streams contiguous row ranges (static).
namespace {
constexpr int kTileCounters = 16384;
__device__ unsigned g_tile_ctr[kTileCounters];
struct CounterPool {
  unsigned* base = nullptr;
  std::map<unsigned long long, int> by_stream;
  int next = 0;
};
std::mutex g_ctr_mu;
CounterPool g_ctr_pool[64];
}  // namespace

unsigned* tile_counter(int device, cudaStream_t st) {
  if (device < 0 || device >= 64) return nullptr;
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(st, &cs) != cudaSuccess) {
    cudaGetLastError();  // not sticky; the launch itself reports real errors
    return nullptr;
  }
  unsigned long long id = 0;
  if (cs == cudaStreamCaptureStatusNone && cudaStreamGetId(st, &id) != cudaSuccess) {
    cudaGetLastError();
    return nullptr;
  }
  std::lock_guard<std::mutex> lk(g_ctr_mu);
  CounterPool& pool = g_ctr_pool[device];
  if (!pool.base) {
    if (cs != cudaStreamCaptureStatusNone) return nullptr;  // set up outside capture
    void* b = nullptr;
    if (cudaGetSymbolAddress(&b, g_tile_ctr) != cudaSuccess || !b) {
      cudaGetLastError();
      return nullptr;
    }
    pool.base = static_cast<unsigned*>(b);
  }
  if (cs == cudaStreamCaptureStatusNone) {
    auto it = pool.by_stream.find(id);
    if (it != pool.by_stream.end()) return pool.base + it->second;
    if (pool.next >= kTileCounters) return nullptr;
    pool.by_stream[id] = pool.next;
    return pool.base + pool.next++;
  }
  if (pool.next >= kTileCounters) return nullptr;
  return pool.base + pool.next++;
}

// After a timeout a launch may leave its counter non-zero: zero them all.
int reset_tile_counters(cudaStream_t st) {
  static const unsigned zeros[kTileCounters] = {};
  const cudaError_t e =
      cudaMemcpyToSymbolAsync(g_tile_ctr, zeros, sizeof(zeros), 0, cudaMemcpyHostToDevice, st);
  if (e == cudaSuccess) return OK;
  return set_error(ERR_CUDA, "resetting the tile counters: %s", cudaGetErrorString(e));
}

bool tma_eligible(const GemvCall& c) {
  // bulk copies start on 16-byte boundaries: x, and the scale plane of SoA
  // calls (its rows are K / 16 bytes, a multiple of 16, so the base decides)
  return c.N == 1 && c.K >= 256 && c.K % 256 == 0 && c.K <= 16384 && c.M >= 1 &&
         (reinterpret_cast<uintptr_t>(c.x) & 15) == 0 &&
         (reinterpret_cast<uintptr_t>(c.d) & 15) == 0;
}

// Returns OK, an error status, or -1 when the shape is not handled here.
int gemv_soa_tma(int fmt, const GemvCall& c, cudaStream_t st) {
  if (!tma_eligible(c)) return -1;
  DeviceInfo dev;
  if (int rc = current_device_info(dev)) return rc;
  // Two CTAs of 8 consumer warps per SM overlap one CTA's drain with the
  // next CTA's fill (less idle time per call); one CTA of 16 streams faster
  // once the call is long enough for that to dominate: measured crossovers
  // near 150 MB of q4_0 (64k rows of K = 4096) and 256 MB of q8_0.  q4_0 is
  // issue-bound: 8 rows per pass amortize the per-pass reduction (falls back
  // to 4 rows, then to one CTA of 16, when the tile does not fit).
  int rc = -1;
  const int64_t wbytes = c.M * (c.K / (fmt == 8 ? 1 : 2) + c.K / 16);
  if (c.act == 1) {  // q8_1 activations: one dp4a set per block, the same shapes
    if (fmt == 4) {
      if (wbytes >= ((int64_t)150 << 20)) rc = launch_tma<4, 2, 8, 16>(c, dev, st);
      if (rc == -1) rc = launch_tma<4, 2, 8, 8>(c, dev, st);
      if (rc == -1) rc = launch_tma<4, 2, 4, 16>(c, dev, st);
      return rc;
    }
    if (wbytes < ((int64_t)256 << 20)) rc = launch_tma<8, 2, 4, 8>(c, dev, st);
    if (rc == -1) rc = launch_tma<8, 2, 4, 16>(c, dev, st);
    return rc;
  }
  // K = 4096 (the 7B-class QKV / O / gate+up shape): kernels compiled for it
  if (fmt == 4) {
    const bool big = wbytes >= ((int64_t)150 << 20);
    if (c.K == 4096)
      rc = big ? launch_tma<4, 1, 8, 16, false, 4096>(c, dev, st)
               : launch_tma<4, 1, 8, 8, false, 4096>(c, dev, st);
    if (rc == -1 && big) rc = launch_tma<4, 1, 8, 16>(c, dev, st);
    if (rc == -1) rc = launch_tma<4, 1, 8, 8>(c, dev, st);
    if (rc == -1) rc = launch_tma<4, 1, 4, 8>(c, dev, st);
    if (rc == -1) rc = launch_tma<4, 1, 4, 16>(c, dev, st);
    return rc;
  }
  const bool small = wbytes < ((int64_t)256 << 20);
  if (c.K == 4096)
    rc = small ? launch_tma<8, 1, 4, 8, false, 4096>(c, dev, st)
               : launch_tma<8, 1, 4, 16, false, 4096>(c, dev, st);
  if (rc == -1 && small) rc = launch_tma<8, 1, 4, 8>(c, dev, st);
  if (rc == -1) rc = launch_tma<8, 1, 4, 16>(c, dev, st);
  return rc;
}

bool tma_pair_eligible(const GemvCall& c) {
  // tma_eligible's shape and alignment rules, and column 1 of x 16-byte
  // aligned too (ldx a multiple of 4 floats); exact activations, no fused
  // all-gather
  if (c.N != 2 || c.act != 0 || c.f.nranks != 0 || c.ldx % 4 != 0) return false;
  GemvCall one = c;
  one.N = 1;
  return tma_eligible(one);
}

// Which two-column calls the pair kernel takes.  Its time is set by the
// integer pipe (48 dp4a per 32-weight block-row for the two columns), so it
// pays where the alternative is slower: q4_0 on SoA planes (W [28672, 8192]:
// 39.4 us against 49.7 us on tcgen05) and GGUF blocks (whose other batch
// kernel streams registers: 42.8 / 40.7 us against 221 / 203 us).  q8_0 on
// SoA planes stays on tcgen05 (45.5 us against 49.2 us for the pair kernel).
bool tma_pair_taken(int fmt, bool aos, const GemvCall& c) {
  return (aos || fmt == 4) && tma_pair_eligible(c);
}

// Two columns in one launch (q4_0 planes or GGUF blocks): the weights stream
// once for both.  CTAs per SM and rows per pass were chosen by measurement
// (below).  -1 when the call is not taken (tma_pair_taken).
int gemv_tma_pair(int fmt, bool aos, const GemvCall& c, cudaStream_t st) {
  if (!tma_pair_taken(fmt, aos, c)) return -1;
  DeviceInfo dev;
  if (int rc = current_device_info(dev)) return rc;
  const int64_t wbytes = aos ? c.M * (c.K / 32) * (fmt == 8 ? 34 : 18)
                             : c.M * (c.K / (fmt == 8 ? 1 : 2) + c.K / 16);
  const bool big = wbytes >= ((int64_t)(fmt == 8 ? 256 : 150) << 20);
  int rc = -1;
  if (fmt == 4 && !aos) {
    // q4_0 planes, measured per (rows per pass, CTAs per SM), same bits for
    // all: K >= 8192 one CTA of 16 with 4 rows (28672 x 8192: 39.4 us against
    // 41.5 with two CTAs of 8); long K = 4096 streams one CTA with 8 rows
    // (70000 x 4096: 45.4 us against 50.2 with 4 rows); shorter ones two CTAs
    // with 4 rows (11008 x 4096: 13.1-13.3 us, every variant within 0.8 us)
    if (c.K >= 8192) rc = launch_tma<4, 1, 4, 16, false, 0, 2>(c, dev, st);
    else if (big) rc = launch_tma<4, 1, 8, 16, false, 0, 2>(c, dev, st);
    else rc = launch_tma<4, 1, 4, 8, false, 0, 2>(c, dev, st);
    if (rc == -1) rc = launch_tma<4, 1, 4, 16, false, 0, 2>(c, dev, st);
    return rc;
  }
  // GGUF blocks (the only other calls taken), 4 rows per pass, same bits
  // either way: one CTA of 16 consumers for K >= 8192 or long streams
  // (28672 x 8192: q8_0 42.8 us against 48.5 with two CTAs of 8, q4_0 40.7
  // against 44.7), two CTAs of 8 otherwise (and one when K needs more than 8
  // slices)
  const bool one = c.K >= 8192 || big;
  if (fmt == 8) {
    if (!one) rc = launch_tma<8, 1, 4, 8, true, 0, 2>(c, dev, st);
    if (rc == -1) rc = launch_tma<8, 1, 4, 16, true, 0, 2>(c, dev, st);
    return rc;
  }
  if (!one) rc = launch_tma<4, 1, 4, 8, true, 0, 2>(c, dev, st);
  if (rc == -1) rc = launch_tma<4, 1, 4, 16, true, 0, 2>(c, dev, st);
  return rc;
}

// AoS (GGUF layout) single-column GEMV on the TMA path; -1 when not eligible.
int gemv_aos_tma(int fmt, const GemvCall& c, cudaStream_t st) {
  if (!tma_eligible(c)) return -1;
  DeviceInfo dev;
  if (int rc = current_device_info(dev)) return rc;
  int rc = -1;
  if (c.act == 1) {  // q8_1 activations
    if (fmt == 4) {
      rc = launch_tma<4, 2, 8, 8, true>(c, dev, st);
      if (rc == -1) rc = launch_tma<4, 2, 4, 16, true>(c, dev, st);
      return rc;
    }
    if (c.M * (c.K + c.K / 16) < ((int64_t)256 << 20)) rc = launch_tma<8, 2, 4, 8, true>(c, dev, st);
    if (rc == -1) rc = launch_tma<8, 2, 4, 16, true>(c, dev, st);
    return rc;
  }
  if (fmt == 4) {
    rc = launch_tma<4, 1, 8, 8, true>(c, dev, st);
    if (rc == -1) rc = launch_tma<4, 1, 4, 8, true>(c, dev, st);
    if (rc == -1) rc = launch_tma<4, 1, 4, 16, true>(c, dev, st);
    return rc;
  }
  if (c.M * (c.K + c.K / 16) < ((int64_t)256 << 20)) rc = launch_tma<8, 1, 4, 8, true>(c, dev, st);
  if (rc == -1) rc = launch_tma<8, 1, 4, 16, true>(c, dev, st);
  return rc;
}

int gemv_soa_tma_mode(int fmt, int mode, const GemvCall& c, cudaStream_t st) {
  if (!tma_eligible(c)) return -1;
  DeviceInfo dev;
  if (int rc = current_device_info(dev)) return rc;
  switch (mode) {
    case 0: return fmt == 8 ? launch_tma<8, 0, 2, 16>(c, dev, st) : launch_tma<4, 0, 4, 16>(c, dev, st);
    case 2: return fmt == 8 ? launch_tma<8, 1, 4, 8>(c, dev, st) : launch_tma<4, 1, 4, 8>(c, dev, st);
    case 3: return fmt == 8 ? launch_tma<8, 1, 2, 8>(c, dev, st) : launch_tma<4, 1, 2, 8>(c, dev, st);
    case 4: return fmt == 8 ? launch_tma<8, 1, 8, 8>(c, dev, st) : launch_tma<4, 1, 8, 8>(c, dev, st);
    default: return fmt == 8 ? launch_tma<8, 1, 4, 16>(c, dev, st) : launch_tma<4, 1, 4, 16>(c, dev, st);
  }
}

namespace {
struct FenceArgs {
  unsigned* done[kMaxRanks];
  const unsigned* done_local;
  unsigned* tok;
  int nranks;
};

__global__ void k_token_fence(const FenceArgs f) {
  if (threadIdx.x != 0) return;
  __threadfence_system();
  for (int k = 0; k < f.nranks; ++k) red_release_sys(f.done[k], 1u);
  const unsigned t = *(volatile unsigned*)f.tok;
  wait_count(f.done_local, (t + 1u) * (unsigned)f.nranks, nullptr);
  *(volatile unsigned*)f.tok = t + 1u;
  __threadfence_system();
}
}  // namespace

int token_fence(unsigned* const* done, int nranks, const unsigned* done_local, unsigned* tok,
                cudaStream_t st) {
  FenceArgs f = {};
  for (int k = 0; k < nranks; ++k) f.done[k] = done[k];
  f.done_local = done_local;
  f.tok = tok;
  f.nranks = nranks;
  k_token_fence<<<1, 32, 0, st>>>(f);
  return check_launch("k_token_fence");
}

namespace {
struct StackHandle {
  int fmt, device, n, grid;
  StackArgs args;
  size_t smem;
  StackGemv* dev_g;
  unsigned* ctr;  // [token count, CTAs done]
};
template <int FMT>
constexpr int stack_rows() { return 4; }  // rows per warp pass
auto stack_kernel(int fmt) {
  return fmt == 8 ? k_gemv_stack<8, stack_rows<8>()> : k_gemv_stack<4, stack_rows<4>()>;
}
}  // namespace

int stack_create(int fmt, const StackCall* calls, int n, const StackRanks* ranks, void** out) {
  DeviceInfo dev;
  if (int rc = current_device_info(dev)) return rc;
  if (n < 1) return set_error(ERR_ARG, "a stack needs at least one GEMV");
  const int nranks = ranks ? ranks->nranks : 1;
  if (nranks < 1 || nranks > kMaxRanks)
    return set_error(ERR_ARG, "nranks must be in [1, %d]", kMaxRanks);
  const int R = fmt == 8 ? stack_rows<8>() : stack_rows<4>();
  std::vector<StackGemv> g(n);
  int SB = 0, PB = 0, XB = 0;
  int64_t min_rows = INT64_MAX;
  auto a16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  for (int j = 0; j < n; ++j) {
    const StackCall& c = calls[j];
    if (c.K < 256 || c.K % 256 || c.K > 16384 || c.M < 1)
      return set_error(ERR_UNSUPPORTED,
                       "stack GEMV %d: needs 256 <= K <= 16384, K %% 256 == 0 and rows", j);
    if (c.r0 < 0 || c.r0 + c.M > c.M_total || c.M_total >= ((int64_t)1 << 31))
      return set_error(ERR_SHAPE, "stack GEMV %d: rows [%lld, %lld) outside [0, %lld)", j,
                       (long long)c.r0, (long long)(c.r0 + c.M), (long long)c.M_total);
    if (!a16(c.q) || !a16(c.d) || !a16(c.y) || (j == 0 && !a16(c.x)))
      return set_error(ERR_ALIGN, "stack GEMV %d: q, d, y (and x of GEMV 0) must be 16-byte aligned", j);
    if (j > 0 && calls[j - 1].M_total < c.K)
      return set_error(ERR_SHAPE, "stack GEMV %d: K = %lld exceeds the %lld outputs of GEMV %d", j,
                       (long long)c.K, (long long)calls[j - 1].M_total, j - 1);
    if (c.M_total % 2)
      return set_error(ERR_SHAPE, "stack GEMV %d: M_total must be even", j);
    min_rows = std::min(min_rows, c.M);
    const int QB = (int)(fmt == 8 ? c.K : c.K / 2), DB = (int)(c.K / 16), row = QB + DB;
    const int nunits = (int)(c.K / QK);
    int KS = 1;
    while (KS * 32 < nunits) KS *= 2;
    const int unit = (kStackConsumers / KS) * R;
    const int TR = unit * std::max(1, (32 * 1024) / (unit * row));
    StackGemv s{};
    s.q = static_cast<const uint8_t*>(c.q);
    s.d = static_cast<const unsigned short*>(c.d);
    s.x = c.x;
    s.y = c.y;
    for (int k = 0; k < nranks - 1; ++k) {
      s.peer_y[k] = c.peer_y[k];
      if (!s.peer_y[k] || !a16(s.peer_y[k]))
        return set_error(ERR_ALIGN, "stack GEMV %d: peer_y[%d] must be a 16-byte aligned pointer",
                         j, k);
    }
    s.r0 = (int)c.r0;
    s.M = (int)c.M;
    s.M_total = (int)c.M_total;
    s.K = (int)c.K;
    s.TR = TR;
    s.KS = KS;
    g[j] = s;
    SB = std::max(SB, (TR * row + 15) / 16 * 16);
    PB = std::max(PB, (TR * KS + 3) / 4 * 4);  // keeps the x area 16-byte aligned
    XB = std::max(XB, (int)std::min<int64_t>(c.K, kStackXChunk) * 4);
  }
  const void* kp = reinterpret_cast<const void*>(stack_kernel(fmt));
  if (int rc = allow_max_smem(kp, dev)) return rc;
  cudaFuncAttributes fa;
  if (cudaFuncGetAttributes(&fa, kp) != cudaSuccess) return check_launch("cudaFuncGetAttributes");
  const int avail = dev.smem_optin - (int)fa.sharedSizeBytes - XB;
  const int S = std::min(MAX_STAGES, avail / (SB + 4 * PB));
  if (S < 2) return set_error(ERR_UNSUPPORTED, "stack tiles of %d bytes do not fit twice", SB);
  StackHandle* h = new StackHandle();
  h->fmt = fmt;
  h->device = dev.device;
  h->n = n;
  // every CTA has rows in every GEMV (so a complete input also shows that
  // every CTA has finished with the buffers before it)
  h->grid = (int)std::min<int64_t>(dev.sms, min_rows);
  h->smem = (size_t)S * (SB + 4 * PB) + XB;
  h->ctr = nullptr;
  cudaError_t e = cudaMalloc(&h->dev_g, sizeof(StackGemv) * n);
  if (e == cudaSuccess) e = cudaMalloc(&h->ctr, sizeof(unsigned) * 2);
  if (e == cudaSuccess) e = cudaMemcpy(h->dev_g, g.data(), sizeof(StackGemv) * n, cudaMemcpyHostToDevice);
  if (e == cudaSuccess) e = cudaMemset(h->ctr, 0, sizeof(unsigned) * 2);
  if (e != cudaSuccess) {
    cudaFree(h->dev_g);
    cudaFree(h->ctr);
    delete h;
    return set_error(ERR_CUDA, "stack set-up: %s", cudaGetErrorString(e));
  }
  StackArgs a{};
  a.g = h->dev_g;
  a.n = n;
  a.ctr = h->ctr;
  a.npeer = nranks - 1;
  a.S = S;
  a.SB = SB;
  a.PB = PB;
  a.XB = XB;
  h->args = a;
  *out = h;
  return OK;
}

int stack_run(void* handle, cudaStream_t st) {
  StackHandle* h = static_cast<StackHandle*>(handle);
  int cur = 0;
  cudaGetDevice(&cur);
  if (cur != h->device)
    return set_error(ERR_ARG, "the stack was made on device %d, the current device is %d",
                     h->device, cur);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(h->grid);
  cfg.blockDim = dim3(kStackThreads);
  cfg.dynamicSmemBytes = h->smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;  // every CTA resident: cross-CTA waits
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, stack_kernel(h->fmt), h->args);
  if (e != cudaSuccess) return set_error(ERR_CUDA, "k_gemv_stack launch: %s", cudaGetErrorString(e));
  return check_launch("k_gemv_stack");
}

int stack_reset(void* handle, cudaStream_t st) {
  // token count and CTA count back to zero; the caller zeroes the output
  // slots (stale tags of an aborted token could otherwise match again)
  StackHandle* h = static_cast<StackHandle*>(handle);
  const cudaError_t e = cudaMemsetAsync(h->ctr, 0, sizeof(unsigned) * 2, st);
  if (e != cudaSuccess) return set_error(ERR_CUDA, "stack reset: %s", cudaGetErrorString(e));
  return OK;
}

int stack_destroy(void* handle) {
  StackHandle* h = static_cast<StackHandle*>(handle);
  if (!h) return OK;
  int cur = 0;
  cudaGetDevice(&cur);
  cudaSetDevice(h->device);
  cudaError_t e = cudaDeviceSynchronize();
  cudaFree(h->dev_g);
  cudaFree(h->ctr);
  cudaSetDevice(cur);
  delete h;
  if (e != cudaSuccess) return set_error(ERR_CUDA, "stack release: %s", cudaGetErrorString(e));
  return OK;
}

int set_spin_limit(long long cycles) {
  const cudaError_t e = cudaMemcpyToSymbol(g_spin_limit, &cycles, sizeof(cycles));
  if (e == cudaSuccess) return OK;
  return set_error(ERR_CUDA, "setting the wait limit: %s", cudaGetErrorString(e));
}

int tile_counters_used(int device) {
  if (device < 0 || device >= 64) return -1;
  std::lock_guard<std::mutex> lk(g_ctr_mu);
  return g_ctr_pool[device].next;
}

int tile_counters_capacity() { return kTileCounters; }

int read_device_error(int clear, cudaStream_t st, int* out) {
  int v = 0;
  cudaError_t e = cudaMemcpyFromSymbolAsync(&v, g_device_error, sizeof(int), 0,
                                            cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e != cudaSuccess) return set_error(ERR_CUDA, "reading the device error word: %s", cudaGetErrorString(e));
  if (clear && v) {
    // A launch that timed out may have left its tile counter non-zero; a
    // launch still running on another stream is using its own.  Wait until
    // the device is idle, then zero them all (clearing needs an idle device:
    // no other thread may launch work meanwhile).
    e = cudaDeviceSynchronize();
    if (e != cudaSuccess) return set_error(ERR_CUDA, "waiting for the device: %s", cudaGetErrorString(e));
    const int zero = 0;
    if (int rc = reset_tile_counters(st)) return rc;
    e = cudaMemcpyToSymbolAsync(g_device_error, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) return set_error(ERR_CUDA, "clearing the device error word: %s", cudaGetErrorString(e));
  }
  *out = v;
  return OK;
}

}  // namespace qg
