// Small-batch (2..16 columns) q8_0 / q4_0 SoA GEMV on the tensor cores, sm_100a.
//
// Y[n][r] = sum_k dequant(W)[r][k] X[n][k] for N activation columns, the
// reference's per-row computation (src/qgemv_kernels.cuh:264-291, 323-352)
// applied to N columns at once, so that every weight byte is read from HBM
// once per call instead of once per column.  With 2N flops per weight byte
// the CUDA cores would bound the call from N ~ 4 on; here the products run on
// the tensor cores (mma.sync m16n8k16, f16 operands, fp32 accumulation):
//
//  * x prep (k_xprep, one CTA per column): every column is scaled by an exact
//    power of two 2^s so that max |x'| < 2^15 and split into two fp16 values,
//    x' = hi + lo (hi = fp16(x'), lo = fp16(x' - hi)); hi + lo holds x' to
//    22 significant bits (relative error <= 2^-22 per element, plus an
//    absolute 2^-25 where lo is an fp16 subnormal).  The pairs are written to
//    a workspace already in the order the MMA B fragments need, one K tile of
//    all columns contiguous, so the main kernel fetches a tile with one bulk
//    copy.  Non-finite elements stay non-finite (their columns come out NaN).
//  * Weights: quants become fp16 exactly in registers (q8_0: byte + 0x6480
//    magic and one HADD2; q4_0: nibble + 0x6400 magic and one HADD2/HFMA2),
//    scales d are applied per 32-weight block to the fp32 MMA result:
//    acc += d[r][b] * (W_b . hi_b + W_b . lo_b).  Products of an int8 and an
//    fp16 value are exact; the tensor-core sums of 16 products keep fp32
//    precision (the worst-case total error is below 1e-6 ||w|| ||x|| for any
//    K, against the 1e-5 ||w|| ||x|| contract).
//  * Data movement: one producer warp streams 16-row x 512-k weight tiles
//    with 2-D tensor TMA (cp.async.bulk.tensor, 128-byte swizzle so that the
//    ldmatrix reads of 8 rows hit 8 different bank groups; out-of-range rows
//    and columns of the last tiles arrive as zeros) and their fp16 scales,
//    plus the x tile of the current K range, into a shared-memory ring
//    tracked by mbarriers.  Eight consumer warps each own TW row tiles of the
//    CTA's current chunk and keep their fp32 accumulators in registers across
//    the whole K loop; the x fragments of a K block are loaded once per warp
//    and reused for its TW row tiles.
//  * Programmatic dependent launch: x prep may start while the previous
//    kernel drains (it waits before touching x or the workspace); the main
//    kernel prefetches weight tiles before it waits for x prep.
//  * Every mbarrier wait is bounded (~1 s): on a timeout the CTA raises an
//    abort flag, the producer waits (bounded) for its copies in flight, the
//    kernel returns and a device error word records QGEMV_ERR_TIMEOUT.
#include "qgemv_common.cuh"
#include "qgemv_internal.h"

#include <cuda.h>

#include <algorithm>
#include <cstring>
#include <map>
#include <mutex>
#include <tuple>

namespace qg {

__device__ int g_mma_error = 0;
// Limit of every bounded wait of the kernels in this file, in clock64 cycles
// (about 1 s by default); qgemv_set_wait_limit changes it per device.
__device__ long long g_mma_spin_limit = 2000000000LL;

namespace {

constexpr int CONS = 16;                    // consumer warps per CTA
constexpr int THREADS = 32 * (CONS + 1);
constexpr int TILE = 16;                    // rows per weight tile (MMA M)
constexpr int KC = 512;                     // k elements per weight tile / x tile
constexpr int XS = 4 * KC + 16;             // bytes per column of an x tile (+16: bank spread)
constexpr int HDR = 128;                    // workspace header: 2 floats per column
constexpr int MAXC = 16;                    // columns per launch
constexpr int MAX_STAGES = 48;
constexpr int DST = TILE * (KC / QK) * 2;   // bytes of one tile's scales (512)

// ------------------------------------------------------------ PTX helpers
// The current wait limit, read once per wait (only on its slow path).
__device__ __forceinline__ long long spin_limit() { return *(volatile long long*)&g_mma_spin_limit; }

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

__device__ __forceinline__ bool mbar_test(uint32_t bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(done)
      : "r"(bar), "r"(parity)
      : "memory");
  return done != 0;
}

// Bounded wait; gives up early when another thread raised the abort flag.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag) {
  if (mbar_try(bar, parity)) return true;
  const long long t0 = clock64(), lim = spin_limit();
  while (!mbar_try(bar, parity)) {
    if (*abort_flag) return false;
    if (clock64() - t0 > lim) {
      atomicExch(&g_mma_error, (int)ERR_TIMEOUT);
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

__device__ __forceinline__ void st_release(uint32_t addr, uint32_t v) {
  asm volatile("st.release.cta.shared::cta.u32 [%0], %1;" ::"r"(addr), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire(uint32_t addr) {
  uint32_t v;
  asm volatile("ld.acquire.cta.shared::cta.u32 %0, [%1];" : "=r"(v) : "r"(addr) : "memory");
  return v;
}

// Bounded wait until a ring slot's tag names stage `g` (see the consumers).
__device__ __forceinline__ bool tag_wait(uint32_t addr, uint32_t g, volatile int* abort_flag) {
  if (ld_acquire(addr) == g) return true;
  const long long t0 = clock64(), lim = spin_limit();
  while (ld_acquire(addr) != g) {
    if (*abort_flag) return false;
    if (clock64() - t0 > lim) {
      atomicExch(&g_mma_error, (int)ERR_TIMEOUT);
      __threadfence();
      *abort_flag = 1;
      return false;
    }
  }
  return true;
}

__device__ __forceinline__ void mbar_expect(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes,
                                         uint32_t bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
          "r"(dst),
      "l"(src), "r"(bytes), "r"(bar)
      : "memory");
}

// 2-D tiled tensor copy global -> shared (no multicast).  c0 is the inner
// (contiguous) coordinate in elements; its byte offset is a multiple of 16.
__device__ __forceinline__ void tensor_g2s(uint32_t dst, const CUtensorMap* map, int c0, int c1,
                                           uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(bar)
      : "memory");
}

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

__device__ __forceinline__ uint4 lds128(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(addr));
  return v;
}

__device__ __forceinline__ unsigned short lds16(uint32_t addr) {
  unsigned short v;
  asm volatile("ld.shared.u16 %0, [%1];" : "=h"(v) : "r"(addr));
  return v;
}

// D = A B (C = 0), m16n8k16, f16 x f16 -> f32.
__device__ __forceinline__ void mma16816_zc(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                            uint32_t b1) {
  const float z = 0.0f;
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%10,%10,%10,%10};"
      : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "f"(z));
}

// D = A B + D, m16n8k16, f16 x f16 -> f32.
__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                         uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t lop3_and_xor(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;  // (a & b) ^ c
  asm("lop3.b32 %0, %1, %2, %3, 0x6A;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
__device__ __forceinline__ uint32_t lop3_and_or(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;  // (a & b) | c
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
__device__ __forceinline__ uint32_t hadd2(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("add.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
__device__ __forceinline__ uint32_t hfma2(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

// Quant words -> fp16 pairs, exactly.
// q8_0: word = int8 weights (w0, w1, w2, w3).  Bytes 0 and 2 (or 1 and 3
// after a shift) go into the low mantissa byte of fp16 1024 with their sign
// bit flipped: fp16(1024 + w + 128); adding -1152 leaves w.
__device__ __forceinline__ uint32_t q8_pair02(uint32_t w) {
  return hadd2(lop3_and_xor(w, 0x00FF00FFu, 0x64806480u), 0xE480E480u);
}
__device__ __forceinline__ uint32_t q8_pair13(uint32_t w) { return q8_pair02(w >> 8); }
// q8_0 batch tiles hold u = w + 128 (sign bit flipped): one PRMT puts bytes
// 0 and 2 (1 and 3) under the fp16 exponent byte 0x64, fp16(1024 + u), and
// adding -1152 leaves w -- no shift and no mask.
__device__ __forceinline__ uint32_t q8u_pair02(uint32_t u) {
  return hadd2(__byte_perm(u, 0x64646464u, 0x6240), 0xE480E480u);
}
__device__ __forceinline__ uint32_t q8u_pair13(uint32_t u) {
  return hadd2(__byte_perm(u, 0x64646464u, 0x6341), 0xE480E480u);
}
// q4_0: word = bytes (p0, p1, p2, p3), byte i = n_i | m_i << 4.  Low nibbles
// of bytes 0 and 2: fp16(1024 + n) - 1032 = n - 8.  High nibbles in place:
// fp16(1024 + 16 m) * 1/16 - 72 = m - 8.
__device__ __forceinline__ uint32_t q4_lo02(uint32_t w) {
  return hadd2(lop3_and_or(w, 0x000F000Fu, 0x64006400u), 0xE408E408u);
}
__device__ __forceinline__ uint32_t q4_hi02(uint32_t w) {
  return hfma2(lop3_and_or(w, 0x00F000F0u, 0x64006400u), 0x2C002C00u, 0xD480D480u);
}

// ------------------------------------------------------------------ x prep
// Element order inside one thread-group record (8 elements of a 32-element
// block for MMA thread t): 4t, 4t+2, 4t+1, 4t+3, 16+4t, 18+4t, 17+4t, 19+4t.
// These are the k indices of the fp16 pairs b0, b1 of the two k16 steps,
// matching the quant pairs q*_pair02 / q*_pair13 (low / high half) of the
// word that ldmatrix gives thread t.
__device__ __forceinline__ int rec_elem(int t, int p) {
  const int i = p & 3;
  return (p >> 2) * 16 + 4 * t + ((i & 1) << 1) + (i >> 1);
}

// Splits 2^s into one factor (when representable) or two.
__device__ __forceinline__ void pow2_factors(int s, float& f1, float& f2) {
  if (s >= -126 && s <= 127) {
    f1 = __int_as_float((127 + s) << 23);
    f2 = 1.0f;
  } else {
    const int h = s / 2;
    f1 = __int_as_float((127 + h) << 23);
    f2 = __int_as_float((127 + s - h) << 23);
  }
}

constexpr int XPREP_THREADS = 1024;

__device__ __forceinline__ uint32_t finite_abs_bits(float v) {
  const uint32_t u = __float_as_uint(v) & 0x7FFFFFFFu;
  return u < 0x7F800000u ? u : 0u;
}

__global__ void __launch_bounds__(XPREP_THREADS) k_xprep(const float* __restrict__ x, int64_t ldx,
                                                         int K, int N, uint8_t* __restrict__ ws) {
  // The next kernel (the GEMV) may start prefetching weights now; it reads
  // the workspace only after its own griddepcontrol.wait, i.e. after this
  // grid has completed.  This grid waits for its predecessor (which may have
  // produced x, or may still read the workspace) before touching either.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  __shared__ uint32_t red[32];
  const int n = blockIdx.x;
  const float* xn = x + (int64_t)n * ldx;
  const bool vec = (reinterpret_cast<uintptr_t>(xn) & 15) == 0;  // K % 32 == 0 always
  uint32_t amax = 0u;  // max |x| over finite elements, as bits
  if (vec) {
    const float4* x4 = reinterpret_cast<const float4*>(xn);
    for (int k = threadIdx.x; k < K / 4; k += blockDim.x) {
      const float4 v = x4[k];
      amax = max(max(amax, finite_abs_bits(v.x)), finite_abs_bits(v.y));
      amax = max(max(amax, finite_abs_bits(v.z)), finite_abs_bits(v.w));
    }
  } else {
    for (int k = threadIdx.x; k < K; k += blockDim.x) amax = max(amax, finite_abs_bits(xn[k]));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = max(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = amax;
  __syncthreads();
  if (threadIdx.x < 32) {
    uint32_t v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0u;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = max(v, __shfl_xor_sync(0xffffffffu, v, o));
    if (threadIdx.x == 0) red[0] = v;
  }
  __syncthreads();
  amax = red[0];
  // max |x'| = max |x| 2^s < 2^15 with max |x| = f 2^e, f in [0.5, 1)
  int s = 0;
  if (amax != 0u) {
    int e;
    frexpf(__uint_as_float(amax), &e);
    s = 15 - e;
  }
  float f1, f2, g1, g2;
  pow2_factors(s, f1, f2);
  pow2_factors(-s, g1, g2);
  if (threadIdx.x == 0) {
    float* h = reinterpret_cast<float*>(ws);
    h[2 * n] = g1;
    h[2 * n + 1] = g2;
  }
  const int nkt = (K + KC - 1) / KC;
  const int recs = nkt * (KC / QK) * 4;  // records of 8 elements in this column
  uint8_t* base = ws + HDR + (size_t)n * XS;
  for (int ri = threadIdx.x; ri < recs; ri += blockDim.x) {
    const int kt = ri / ((KC / QK) * 4), rem = ri - kt * ((KC / QK) * 4);
    const int b = rem >> 2, t = rem & 3;
    const int k0 = kt * KC + b * QK;  // a whole 32-element block is inside K or beyond it
    float v[8];
    if (k0 >= K) {
#pragma unroll
      for (int p = 0; p < 8; ++p) v[p] = 0.0f;
    } else if (vec) {
      const float4 a = *reinterpret_cast<const float4*>(xn + k0 + 4 * t);
      const float4 c = *reinterpret_cast<const float4*>(xn + k0 + 16 + 4 * t);
      v[0] = a.x; v[1] = a.z; v[2] = a.y; v[3] = a.w;
      v[4] = c.x; v[5] = c.z; v[6] = c.y; v[7] = c.w;
    } else {
#pragma unroll
      for (int p = 0; p < 8; ++p) v[p] = xn[k0 + rec_elem(t, p)];
    }
    uint32_t hw[4], lw[4];
#pragma unroll
    for (int p = 0; p < 8; p += 2) {
      __half hv[2], lv[2];
#pragma unroll
      for (int q = 0; q < 2; ++q) {
        const float xv = (v[p + q] * f1) * f2;
        hv[q] = __float2half_rn(xv);
        lv[q] = __float2half_rn(xv - __half2float(hv[q]));
      }
      hw[p >> 1] = (uint32_t)__half_as_ushort(hv[0]) | ((uint32_t)__half_as_ushort(hv[1]) << 16);
      lw[p >> 1] = (uint32_t)__half_as_ushort(lv[0]) | ((uint32_t)__half_as_ushort(lv[1]) << 16);
    }
    uint8_t* dst = base + (size_t)kt * N * XS + b * 128 + t * 32;
    *reinterpret_cast<uint4*>(dst) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
    *reinterpret_cast<uint4*>(dst + 16) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
  }
}

// --------------------------------------------------------------- the GEMV
struct MmaArgs {
  CUtensorMap qmap;  // SoA: quants [M][K / ROW_DIV] bytes, box 128 B x 16 rows, 128-byte swizzle
  CUtensorMap dmap;  // SoA: scales [M][K/32] fp16, box (KC/32) x 16 rows
  const uint8_t* tiled;  // batch tiles (see tile layout below), or null for SoA
  const uint8_t* ws;
  float* y;
  int64_t ldy;
  int M, K, N, S;
};

template <int FMT>
struct MmaFmt {
  static constexpr int QROW = FMT == 8 ? KC : KC / 2;  // quant bytes of a tile row
  static constexpr int NBOX = QROW / 128;              // 128-byte boxes per tile
  static constexpr int QST = NBOX * TILE * 128;        // quant bytes per tile
  static constexpr int BLK = QST + DST;                // bytes of one batch tile
  static constexpr int SLOT = (BLK + 1023) / 1024 * 1024;  // ring slot (1024-aligned quants)
};

// Batch-tile layout (qgemv_tiled_bytes / qgemv_tile_weights): for each
// 16-row tile t and 512-column K tile kt, one contiguous block of
// QST + DST bytes at ((kt * T) + t) * (QST + DST), T = ceil(M / 16), so that
// the consecutive tiles of one K tile are consecutive in memory:
//   quants: NBOX boxes of [16 rows][128 bytes]; within a box, 16-byte chunk
//           j of row r is stored at chunk position j ^ (r & 7) (the TMA
//           128-byte swizzle, so that ldmatrix reads are conflict-free);
//           q8_0 bytes hold w + 128 (the int8 with its sign bit flipped);
//   scales: [16 rows][16 blocks] fp16.
// Rows beyond M and columns beyond K hold zero weights.  A few tiles are then one
// bulk copy, which streams at the HBM rate where 16 strided row pieces do not.
// KSPLIT warps share a row tile (each takes KC/32/KSPLIT blocks of every
// stage) and each warp holds TW tiles, so CONS/KSPLIT*TW tiles are in flight
// per CTA: few enough that the ring keeps ~100 KB of weights in flight.
template <int FMT, int NT, int TW, int KSPLIT>
__global__ void __launch_bounds__(THREADS, 1) k_gemv_mma(const __grid_constant__ MmaArgs p) {
  using F = MmaFmt<FMT>;
  extern __shared__ uint8_t sm_raw[];
  __shared__ __align__(8) unsigned long long full[MAX_STAGES];
  __shared__ __align__(8) unsigned long long empty[MAX_STAGES];
  __shared__ __align__(8) unsigned long long xfull[2];
  __shared__ __align__(8) unsigned long long xempty[2];
  __shared__ __align__(8) unsigned long long redfull;
  __shared__ __align__(8) unsigned long long redempty;
  __shared__ uint32_t tag[MAX_STAGES];
  __shared__ int abort_flag;

  const int S = p.S, N = p.N, K = p.K;
  // shared memory: [ring: S slots of (quants, scales), 1024-aligned][x slots 2 x NT*8*XS]
  //                [partial sums: CONS/KSPLIT*(KSPLIT-1) warps x TW*NT*4*32 floats]
  const uint32_t raw = saddr(sm_raw);
  const uint32_t ring = (raw + 1023u) & ~1023u;
  const uint32_t xslot0 = ring + (uint32_t)S * F::SLOT;
  const uint32_t xslot_bytes = (uint32_t)(NT * 8) * XS;
  constexpr int RED_WARP = TW * NT * 4 * 32;  // floats per warp
  float* red = reinterpret_cast<float*>(sm_raw + (xslot0 + 2u * xslot_bytes - raw));

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int T = (p.M + TILE - 1) / TILE;
  const int t0 = (int)((int64_t)T * blockIdx.x / gridDim.x);
  const int ntc = (int)((int64_t)T * (blockIdx.x + 1) / gridDim.x) - t0;  // tiles of this CTA
  const int nkt = (K + KC - 1) / KC;
  constexpr int CH = CONS / KSPLIT * TW;  // tiles per chunk
  const int nch = (ntc + CH - 1) / CH;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(saddr(&full[s])));
      asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(saddr(&empty[s])), "r"(KSPLIT));
      tag[s] = 0xFFFFFFFFu;
    }
    for (int s = 0; s < 2; ++s) {
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(saddr(&xfull[s])));
      asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(saddr(&xempty[s])), "r"(CONS));
    }
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(saddr(&redfull)),
                 "r"(CONS / KSPLIT * (KSPLIT - 1)));
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(saddr(&redempty)),
                 "r"(CONS / KSPLIT));
    abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane != 0) return;
    const uint32_t xbytes = (uint32_t)N * XS;
    const int qrow_bytes = FMT == 8 ? K : K / 2;
    auto issue_stage = [&](uint32_t g, int tile, int kt) {
      const int s = (int)(g % (uint32_t)S);
      const uint32_t bar = saddr(&full[s]);
      const uint32_t slot = ring + (uint32_t)s * F::SLOT;
      // the slot's previous stage has been released: name the new one
      st_release(saddr(&tag[s]), g);
      // boxes wholly beyond the row end (last K tile) are not fetched: the
      // stale bytes there meet x' = 0 and finite quants give exact zeros
      const int nbox = min(F::NBOX, (qrow_bytes - kt * F::QROW) / 128);
      mbar_expect(bar, (uint32_t)nbox * (TILE * 128) + DST);
      for (int bx = 0; bx < nbox; ++bx)
        tensor_g2s(slot + bx * (TILE * 128), &p.qmap, kt * F::QROW + bx * 128, tile * TILE, bar);
      tensor_g2s(slot + F::QST, &p.dmap, kt * (KC / QK), tile * TILE, bar);
    };
    // Weight tiles do not depend on the previous kernel: prefetch the first
    // S of them before waiting for x prep.
    const int first_tc = min(CH, ntc);
    const uint32_t pre = (uint32_t)min(S, first_tc);
    for (uint32_t g = 0; g < pre; ++g) issue_stage(g, t0 + (int)g, 0);
    asm volatile("griddepcontrol.wait;" ::: "memory");
    uint32_t g = 0, xseq = 0;
    int last_x[2] = {-1, -1};
    bool ok = true;
    for (int c = 0; c < nch && ok; ++c) {
      const int tc0 = c * CH, tcn = min(CH, ntc - tc0);
      for (int kt = 0; kt < nkt && ok; ++kt, ++xseq) {
        const int xs = (int)(xseq & 1u);
        if (xseq >= 2 && !mbar_wait(saddr(&xempty[xs]), ((xseq >> 1) - 1) & 1u, &abort_flag)) {
          ok = false;
          break;
        }
        mbar_expect(saddr(&xfull[xs]), xbytes);
        bulk_g2s(xslot0 + (uint32_t)xs * xslot_bytes, p.ws + HDR + (size_t)kt * N * XS, xbytes,
                 saddr(&xfull[xs]));
        last_x[xs] = (int)xseq;
        for (int j = 0; j < tcn; ++j, ++g) {
          if (g < pre) continue;  // prefetched above
          const uint32_t s = g % (uint32_t)S, u = g / (uint32_t)S;
          if (u >= 1 && !mbar_wait(saddr(&empty[s]), (u - 1) & 1u, &abort_flag)) {
            ok = false;
            break;
          }
          issue_stage(g, t0 + tc0 + j, kt);
        }
      }
    }
    if (!ok) {
      // aborted: wait (bounded) for every copy still in flight into our smem
      const uint32_t issued = g > pre ? g : pre;
      for (uint32_t s = 0; s < (uint32_t)S && s < issued; ++s) {
        const uint32_t last = s + ((issued - 1 - s) / (uint32_t)S) * (uint32_t)S;
        mbar_wait_drain(saddr(&full[s]), (last / (uint32_t)S) & 1u);
      }
      for (int xs = 0; xs < 2; ++xs)
        if (last_x[xs] >= 0) mbar_wait_drain(saddr(&xfull[xs]), ((uint32_t)last_x[xs] >> 1) & 1u);
    }
    return;
  }

  // -------------------------------------------------------------- consumers
  // Warp (ts, kh): row tiles ts*TW .. ts*TW+TW-1 of each chunk, K blocks
  // kh*HB .. kh*HB+HB-1 of each stage; the KSPLIT partial sums of a tile meet
  // in shared memory at the end of the chunk (summed in a fixed order).  A warp consumes only some stages
  // of the shared ring, so it has not seen the earlier phases of a slot's
  // barrier; it first waits until the slot's tag names its stage (the
  // producer writes the tag only once the slot's previous stage has been
  // released, hence landed), after which the parity wait is unambiguous.
  const int cw = warp - 1;
  const int ts = cw / KSPLIT, kh = cw % KSPLIT;
  const int gq = lane >> 2, tq = lane & 3;  // MMA group / thread in group
  asm volatile("griddepcontrol.wait;" ::: "memory");  // y and the workspace header
  // ldmatrix row address of this lane within a tile: rows (m & 1) * 8 + rr
  const int lm = lane >> 3, lr = lane & 7;
  const uint32_t a_row_off = (uint32_t)(((lm & 1) * 8 + lr) * 128);
  constexpr int HB = KC / QK / KSPLIT;  // K blocks of a stage per warp

  float acc[TW][NT][4];
  uint32_t g = 0, xseq = 0;
  bool ok = true;
  for (int c = 0; c < nch && ok; ++c) {
    const int tc0 = c * CH, tcn = min(CH, ntc - tc0);
#pragma unroll
    for (int i = 0; i < TW; ++i)
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[i][nt][e] = 0.0f;
    for (int kt = 0; kt < nkt; ++kt, ++xseq, g += (uint32_t)tcn) {
      const int xs = (int)(xseq & 1u);
      bool live[TW];
      uint32_t qst[TW], dst[TW];
      bool good = __all_sync(0xffffffffu,
                             mbar_wait(saddr(&xfull[xs]), (xseq >> 1) & 1u, &abort_flag));
#pragma unroll
      for (int i = 0; i < TW; ++i) {
        const int j = ts * TW + i;
        live[i] = j < tcn;
        const uint32_t gi = g + (uint32_t)j, s = gi % (uint32_t)S;
        qst[i] = ring + s * F::SLOT;
        dst[i] = qst[i] + F::QST;
        if (live[i] && good)
          good = __all_sync(0xffffffffu,
                            tag_wait(saddr(&tag[s]), gi, &abort_flag) &&
                                mbar_wait(saddr(&full[s]), (gi / (uint32_t)S) & 1u, &abort_flag));
      }
      if (!good) {
        ok = false;
        break;
      }
      const uint32_t xb = xslot0 + (uint32_t)xs * xslot_bytes + (uint32_t)gq * XS + tq * 32;
#pragma unroll 1
      for (int bp = kh * (HB / 2); bp < (kh + 1) * (HB / 2); ++bp) {  // pairs of blocks
        // raw quant words of both blocks of the pair: rows g / g+8
        uint32_t aw[TW][2][4];
#pragma unroll
        for (int i = 0; i < TW; ++i) {
          if (!live[i]) continue;
          if (FMT == 8) {
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              const int b = 2 * bp + h;
              const int jj = 2 * (b & 3) + (lm >> 1);
              ldsm_x4(aw[i][h], qst[i] + (uint32_t)(b >> 2) * (TILE * 128) + a_row_off +
                                    (uint32_t)((jj ^ lr) << 4));
            }
          } else {
            const int b = 2 * bp;
            const int jj = (b & 7) + (lm >> 1);
            uint32_t w4[4];
            ldsm_x4(w4, qst[i] + (uint32_t)(b >> 3) * (TILE * 128) + a_row_off +
                            (uint32_t)((jj ^ lr) << 4));
            aw[i][0][0] = w4[0]; aw[i][0][1] = w4[1];
            aw[i][1][0] = w4[2]; aw[i][1][1] = w4[3];
          }
        }
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int b = 2 * bp + h;
          uint4 bh[NT], bl[NT];
#pragma unroll
          for (int nt = 0; nt < NT; ++nt) {
            const uint32_t xa = xb + (uint32_t)(nt * 8) * XS + (uint32_t)b * 128;
            bh[nt] = lds128(xa);
            bl[nt] = lds128(xa + 16);
          }
#pragma unroll
          for (int i = 0; i < TW; ++i) {
            if (!live[i]) continue;
            uint32_t A0[4], A1[4];
            if (FMT == 8) {
              const uint32_t* w = aw[i][h];  // rows g, g+8 x k 4t..4t+3 ; rows g, g+8 x k 16+4t..
              A0[0] = q8_pair02(w[0]); A0[1] = q8_pair02(w[1]);
              A0[2] = q8_pair13(w[0]); A0[3] = q8_pair13(w[1]);
              A1[0] = q8_pair02(w[2]); A1[1] = q8_pair02(w[3]);
              A1[2] = q8_pair13(w[2]); A1[3] = q8_pair13(w[3]);
            } else {
              const uint32_t w0 = aw[i][h][0], w1 = aw[i][h][1];
              const uint32_t v0 = w0 >> 8, v1 = w1 >> 8;
              A0[0] = q4_lo02(w0); A0[1] = q4_lo02(w1);
              A0[2] = q4_lo02(v0); A0[3] = q4_lo02(v1);
              A1[0] = q4_hi02(w0); A1[1] = q4_hi02(w1);
              A1[2] = q4_hi02(v0); A1[3] = q4_hi02(v1);
            }
            const uint32_t da = dst[i] + (uint32_t)gq * ((KC / QK) * 2) + (uint32_t)b * 2;
            const float dg = half_bits_to_float(lds16(da));
            const float dg8 = half_bits_to_float(lds16(da + 8 * (KC / QK) * 2));
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
              // the block's dot: hi and lo parts of both k16 steps in one chain
              float D[4];
              mma16816_zc(D, A0, bh[nt].x, bh[nt].y);
              mma16816(D, A0, bl[nt].x, bl[nt].y);
              mma16816(D, A1, bh[nt].z, bh[nt].w);
              mma16816(D, A1, bl[nt].z, bl[nt].w);
              acc[i][nt][0] = fmaf(dg, D[0], acc[i][nt][0]);
              acc[i][nt][1] = fmaf(dg, D[1], acc[i][nt][1]);
              acc[i][nt][2] = fmaf(dg8, D[2], acc[i][nt][2]);
              acc[i][nt][3] = fmaf(dg8, D[3], acc[i][nt][3]);
            }
          }
        }
      }
      __syncwarp();
      if (lane == 0) {
#pragma unroll
        for (int i = 0; i < TW; ++i) {
          if (!live[i]) continue;
          mbar_arrive(saddr(&empty[(g + (uint32_t)(ts * TW + i)) % (uint32_t)S]));
        }
        mbar_arrive(saddr(&xempty[xs]));
      }
    }
    if (!ok) break;
    // combine the K parts: warps kh >= 1 hand their partial sums to kh = 0
    if (kh >= 1) {
      float* rp = red + ((size_t)ts * (KSPLIT - 1) + (kh - 1)) * RED_WARP + lane;
      if (c >= 1 && !__all_sync(0xffffffffu, mbar_wait(saddr(&redempty), (c - 1) & 1u,
                                                        &abort_flag))) {
        ok = false;
        break;
      }
#pragma unroll
      for (int i = 0; i < TW; ++i)
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
          for (int e = 0; e < 4; ++e) rp[((i * NT + nt) * 4 + e) * 32] = acc[i][nt][e];
      __syncwarp();
      if (lane == 0) mbar_arrive(saddr(&redfull));
      continue;
    }
    if (!__all_sync(0xffffffffu, mbar_wait(saddr(&redfull), c & 1u, &abort_flag))) {
      ok = false;
      break;
    }
#pragma unroll
    for (int k = 0; k < KSPLIT - 1; ++k) {
      const float* rp = red + ((size_t)ts * (KSPLIT - 1) + k) * RED_WARP + lane;
#pragma unroll
      for (int i = 0; i < TW; ++i)
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
          for (int e = 0; e < 4; ++e) acc[i][nt][e] += rp[((i * NT + nt) * 4 + e) * 32];
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(saddr(&redempty));
    // y for this warp's tiles of the chunk
    const float* hdr = reinterpret_cast<const float*>(p.ws);
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int n = nt * 8 + 2 * tq + e;
        if (n >= N) continue;
        const float g1 = hdr[2 * n], g2 = hdr[2 * n + 1];
#pragma unroll
        for (int i = 0; i < TW; ++i) {
          const int j = ts * TW + i;
          if (j >= tcn) continue;
          const int r = (t0 + tc0 + j) * TILE + gq;
          if (r < p.M) p.y[(int64_t)n * p.ldy + r] = (acc[i][nt][e] * g1) * g2;
          if (r + 8 < p.M) p.y[(int64_t)n * p.ldy + r + 8] = (acc[i][nt][e + 2] * g1) * g2;
        }
      }
    }
  }
}

// GEMV over batch tiles.  A stage is TPS consecutive tiles of one K tile
// (about 18 KB: 2 tiles of q8_0, 4 of q4_0), one bulk copy.  Warps 2j and
// 2j+1 own tile j of the current chunk of CN / 2 and take the two K halves of
// each stage; a warp copies its quants and scales from the stage into
// registers (ldmatrix) and releases the slot before it computes, so the ring
// keeps nearly all its stages in flight.  The per-block arithmetic and its
// order are those of k_gemv_mma (two warps per tile), so both give the same
// bits for the same matrix.
template <int FMT, int NT, int CN>
__global__ void __launch_bounds__(32 * (CN + 1), 1) k_gemv_tiles(const __grid_constant__ MmaArgs p) {
  using F = MmaFmt<FMT>;
  constexpr int KSP = 2;                   // warps per tile (K halves)
  constexpr int CT = CN / KSP;             // tiles per chunk
  constexpr int TPS = FMT == 8 ? 2 : 4;    // tiles per stage
  constexpr int SLOT = (TPS * F::BLK + 1023) / 1024 * 1024;
  constexpr int HB = KC / QK / KSP;        // K blocks per warp per stage (8)
  constexpr int AREG = FMT == 8 ? HB : HB / 2;  // ldmatrix.x4 per warp per stage
  constexpr int XSL = 2;                   // x tile slots (prefetched XSL - 1 K steps ahead)
  extern __shared__ uint8_t sm_raw[];
  __shared__ __align__(8) unsigned long long full[MAX_STAGES];
  __shared__ __align__(8) unsigned long long empty[MAX_STAGES];
  __shared__ __align__(8) unsigned long long xfull[XSL];
  __shared__ __align__(8) unsigned long long xempty[XSL];
  __shared__ __align__(8) unsigned long long redfull;
  __shared__ __align__(8) unsigned long long redempty;
  __shared__ uint32_t tag[MAX_STAGES];
  __shared__ int abort_flag;

  const int S = p.S, N = p.N, K = p.K;
  // shared memory: [ring S x SLOT (1024-aligned)][x slots XSL x NT*8*XS][partials CT x NT*4*32 floats]
  const uint32_t raw = saddr(sm_raw);
  const uint32_t ring = (raw + 1023u) & ~1023u;
  const uint32_t xslot0 = ring + (uint32_t)S * SLOT;
  const uint32_t xslot_bytes = (uint32_t)(NT * 8) * XS;
  constexpr int RED_WARP = NT * 4 * 32;
  float* red = reinterpret_cast<float*>(sm_raw + (xslot0 + (uint32_t)XSL * xslot_bytes - raw));

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int T = (p.M + TILE - 1) / TILE;
  const int t0 = (int)((int64_t)T * blockIdx.x / gridDim.x);
  const int ntc = (int)((int64_t)T * (blockIdx.x + 1) / gridDim.x) - t0;
  const int nkt = (K + KC - 1) / KC;
  const int nch = (ntc + CT - 1) / CT;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(saddr(&full[s])));
      asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(saddr(&empty[s])),
                   "r"(KSP * TPS));
      tag[s] = 0xFFFFFFFFu;
    }
    for (int s = 0; s < XSL; ++s) {
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(saddr(&xfull[s])));
      asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(saddr(&xempty[s])), "r"(CN));
    }
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(saddr(&redfull)), "r"(CT));
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(saddr(&redempty)), "r"(CT));
    abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane != 0) return;
    const uint32_t xbytes = (uint32_t)N * XS;
    auto issue_stage = [&](uint32_t g, int tile, int ntile, int kt) {
      const int s = (int)(g % (uint32_t)S);
      const uint32_t bar = saddr(&full[s]);
      st_release(saddr(&tag[s]), g);
      const uint32_t bytes = (uint32_t)ntile * F::BLK;
      mbar_expect(bar, bytes);
      bulk_g2s(ring + (uint32_t)s * SLOT, p.tiled + ((size_t)kt * T + tile) * F::BLK, bytes, bar);
    };
    const int tcn0 = min(CT, ntc), nst0 = (tcn0 + TPS - 1) / TPS;
    const uint32_t pre = (uint32_t)min(S, nst0);
    for (uint32_t g = 0; g < pre; ++g)
      issue_stage(g, t0 + (int)g * TPS, min(TPS, tcn0 - (int)g * TPS), 0);
    asm volatile("griddepcontrol.wait;" ::: "memory");
    // x tiles: sequence q is K tile q % nkt of chunk q / nkt; issued up to
    // XSL - 1 steps ahead of the weight stages, as their slots free up
    const uint32_t nxs = (uint32_t)(nch * nkt);
    uint32_t xnext = 0;
    int last_x[XSL];
    for (int i = 0; i < XSL; ++i) last_x[i] = -1;
    auto issue_x = [&](uint32_t q) {
      const int xs = (int)(q % (uint32_t)XSL);
      mbar_expect(saddr(&xfull[xs]), xbytes);
      bulk_g2s(xslot0 + (uint32_t)xs * xslot_bytes, p.ws + HDR + (size_t)(q % nkt) * N * XS,
               xbytes, saddr(&xfull[xs]));
      last_x[xs] = (int)q;
    };
    auto x_free = [&](uint32_t q) {  // non-blocking: slot of x tile q released?
      return q < (uint32_t)XSL ||
             mbar_test(saddr(&xempty[q % XSL]), ((q / XSL) - 1) & 1u);
    };
    uint32_t g = 0, xseq = 0;
    bool ok = true;
    for (int c = 0; c < nch && ok; ++c) {
      const int tc0 = c * CT, tcn = min(CT, ntc - tc0), nst = (tcn + TPS - 1) / TPS;
      for (int kt = 0; kt < nkt && ok; ++kt, ++xseq) {
        // x tile of this step (blocking), then any later ones whose slots are free
        while (xnext <= xseq) {
          if (xnext >= (uint32_t)XSL &&
              !mbar_wait(saddr(&xempty[xnext % XSL]), ((xnext / XSL) - 1) & 1u, &abort_flag)) {
            ok = false;
            break;
          }
          issue_x(xnext++);
        }
        if (!ok) break;
        while (xnext < nxs && xnext < xseq + XSL && x_free(xnext)) issue_x(xnext++);
        for (int js = 0; js < nst; ++js, ++g) {
          if (g < pre) continue;  // prefetched above
          const uint32_t s = g % (uint32_t)S, u = g / (uint32_t)S;
          if (u >= 1 && !mbar_wait(saddr(&empty[s]), (u - 1) & 1u, &abort_flag)) {
            ok = false;
            break;
          }
          issue_stage(g, t0 + tc0 + js * TPS, min(TPS, tcn - js * TPS), kt);
          if (xnext < nxs && xnext < xseq + XSL && x_free(xnext)) issue_x(xnext++);
        }
      }
    }
    if (!ok) {
      const uint32_t issued = g > pre ? g : pre;
      for (uint32_t s = 0; s < (uint32_t)S && s < issued; ++s) {
        const uint32_t last = s + ((issued - 1 - s) / (uint32_t)S) * (uint32_t)S;
        mbar_wait_drain(saddr(&full[s]), (last / (uint32_t)S) & 1u);
      }
      for (int xs = 0; xs < XSL; ++xs)
        if (last_x[xs] >= 0)
          mbar_wait_drain(saddr(&xfull[xs]), ((uint32_t)last_x[xs] / XSL) & 1u);
    }
    return;
  }

  // -------------------------------------------------------------- consumers
  const int cw = warp - 1;
  const int ts = cw / KSP, kh = cw % KSP;
  const int gq = lane >> 2, tq = lane & 3;
  asm volatile("griddepcontrol.wait;" ::: "memory");  // y and the workspace header
  const int lm = lane >> 3, lr = lane & 7;
  const uint32_t a_row_off = (uint32_t)(((lm & 1) * 8 + lr) * 128);
  const int js = ts / TPS, tin = ts % TPS;  // this warp's stage in a K step, tile in the stage

  float acc[NT][4];
  uint32_t g = 0, xseq = 0;
  bool ok = true;
  for (int c = 0; c < nch && ok; ++c) {
    const int tc0 = c * CT, tcn = min(CT, ntc - tc0), nst = (tcn + TPS - 1) / TPS;
    const bool live = ts < tcn;
    const int tis = min(TPS, tcn - js * TPS);  // tiles in this warp's stage
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[nt][e] = 0.0f;
    for (int kt = 0; kt < nkt; ++kt, ++xseq, g += (uint32_t)nst) {
      const int xs = (int)(xseq % (uint32_t)XSL);
      bool good = __all_sync(0xffffffffu,
                             mbar_wait(saddr(&xfull[xs]), (xseq / XSL) & 1u, &abort_flag));
      uint32_t aw[AREG][4];
      uint32_t dh[2][4];  // scales of rows g and g+8, this warp's 8 blocks (fp16 pairs)
      if (live && good) {
        const uint32_t gi = g + (uint32_t)js, s = gi % (uint32_t)S;
        good = __all_sync(0xffffffffu,
                          tag_wait(saddr(&tag[s]), gi, &abort_flag) &&
                              mbar_wait(saddr(&full[s]), (gi / (uint32_t)S) & 1u, &abort_flag));
        if (good) {
          const uint32_t qb = ring + s * SLOT + (uint32_t)tin * F::BLK;
#pragma unroll
          for (int i = 0; i < AREG; ++i) {
            if (FMT == 8) {
              const int b = kh * HB + i;
              const int jj = 2 * (b & 3) + (lm >> 1);
              ldsm_x4(aw[i], qb + (uint32_t)(b >> 2) * (TILE * 128) + a_row_off +
                                 (uint32_t)((jj ^ lr) << 4));
            } else {
              const int b = kh * HB + 2 * i;
              const int jj = (b & 7) + (lm >> 1);
              ldsm_x4(aw[i], qb + (uint32_t)(b >> 3) * (TILE * 128) + a_row_off +
                                 (uint32_t)((jj ^ lr) << 4));
            }
          }
          const uint32_t db = qb + F::QST + (uint32_t)kh * (HB * 2);
          const uint4 d0 = lds128(db + (uint32_t)gq * ((KC / QK) * 2));
          const uint4 d1 = lds128(db + (uint32_t)(gq + 8) * ((KC / QK) * 2));
          dh[0][0] = d0.x; dh[0][1] = d0.y; dh[0][2] = d0.z; dh[0][3] = d0.w;
          dh[1][0] = d1.x; dh[1][1] = d1.y; dh[1][2] = d1.z; dh[1][3] = d1.w;
          __syncwarp();
          if (lane == 0) {
            // the stage's first warp also answers for the tiles a short stage lacks
            const uint32_t cnt = 1u + ((tin == 0 && kh == 0) ? (uint32_t)(KSP * (TPS - tis)) : 0u);
            asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0], %1;" ::"r"(saddr(&empty[s])),
                         "r"(cnt)
                         : "memory");
          }
        }
      }
      if (!good) {
        ok = false;
        break;
      }
      if (live) {
        const uint32_t xb = xslot0 + (uint32_t)xs * xslot_bytes + (uint32_t)gq * XS + tq * 32;
#pragma unroll
        for (int i = 0; i < HB; ++i) {
          const int b = kh * HB + i;
          uint4 bh[NT], bl[NT];
#pragma unroll
          for (int nt = 0; nt < NT; ++nt) {
            const uint32_t xa = xb + (uint32_t)(nt * 8) * XS + (uint32_t)b * 128;
            bh[nt] = lds128(xa);
            bl[nt] = lds128(xa + 16);
          }
          uint32_t A0[4], A1[4];
          if (FMT == 8) {
            const uint32_t* w = aw[i];  // w + 128 per byte (batch tiles)
            A0[0] = q8u_pair02(w[0]); A0[1] = q8u_pair02(w[1]);
            A0[2] = q8u_pair13(w[0]); A0[3] = q8u_pair13(w[1]);
            A1[0] = q8u_pair02(w[2]); A1[1] = q8u_pair02(w[3]);
            A1[2] = q8u_pair13(w[2]); A1[3] = q8u_pair13(w[3]);
          } else {
            const uint32_t w0 = aw[i >> 1][2 * (i & 1)], w1 = aw[i >> 1][2 * (i & 1) + 1];
            const uint32_t v0 = w0 >> 8, v1 = w1 >> 8;
            A0[0] = q4_lo02(w0); A0[1] = q4_lo02(w1);
            A0[2] = q4_lo02(v0); A0[3] = q4_lo02(v1);
            A1[0] = q4_hi02(w0); A1[1] = q4_hi02(w1);
            A1[2] = q4_hi02(v0); A1[3] = q4_hi02(v1);
          }
          const float dg = half_bits_to_float((unsigned short)(dh[0][i >> 1] >> (16 * (i & 1))));
          const float dg8 = half_bits_to_float((unsigned short)(dh[1][i >> 1] >> (16 * (i & 1))));
#pragma unroll
          for (int nt = 0; nt < NT; ++nt) {
            float D[4];  // the block's dot, as in k_gemv_mma
            mma16816_zc(D, A0, bh[nt].x, bh[nt].y);
            mma16816(D, A0, bl[nt].x, bl[nt].y);
            mma16816(D, A1, bh[nt].z, bh[nt].w);
            mma16816(D, A1, bl[nt].z, bl[nt].w);
            acc[nt][0] = fmaf(dg, D[0], acc[nt][0]);
            acc[nt][1] = fmaf(dg, D[1], acc[nt][1]);
            acc[nt][2] = fmaf(dg8, D[2], acc[nt][2]);
            acc[nt][3] = fmaf(dg8, D[3], acc[nt][3]);
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(saddr(&xempty[xs]));
    }
    if (!ok) break;
    // the K-half warp hands its partial sums to its partner
    float* rp = red + (size_t)ts * RED_WARP + lane;
    if (kh == 1) {
      if (c >= 1 && !__all_sync(0xffffffffu, mbar_wait(saddr(&redempty), (c - 1) & 1u,
                                                        &abort_flag))) {
        ok = false;
        break;
      }
      if (live) {
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
          for (int e = 0; e < 4; ++e) rp[(nt * 4 + e) * 32] = acc[nt][e];
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(saddr(&redfull));
      continue;
    }
    if (!__all_sync(0xffffffffu, mbar_wait(saddr(&redfull), c & 1u, &abort_flag))) {
      ok = false;
      break;
    }
    if (live) {
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[nt][e] += rp[(nt * 4 + e) * 32];
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(saddr(&redempty));
    if (!live) continue;
    const float* hdr = reinterpret_cast<const float*>(p.ws);
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int n = nt * 8 + 2 * tq + e;
        if (n >= N) continue;
        const float g1 = hdr[2 * n], g2 = hdr[2 * n + 1];
        const int r = (t0 + tc0 + ts) * TILE + gq;
        if (r < p.M) p.y[(int64_t)n * p.ldy + r] = (acc[nt][e] * g1) * g2;
        if (r + 8 < p.M) p.y[(int64_t)n * p.ldy + r + 8] = (acc[nt][e + 2] * g1) * g2;
      }
    }
  }
}

// Batch tiles from SoA planes (q: [M][K / ROW_DIV] bytes, d: [M][K/32] fp16)
// or from ggml blocks (AOS: [M][K/32] blocks of 34 / 18 bytes, d first).
// One thread writes one 16-byte chunk of the output.
template <int FMT, bool AOS>
__global__ void __launch_bounds__(256) k_tile(const uint8_t* __restrict__ q,
                                              const unsigned short* __restrict__ d, int64_t M,
                                              int K, uint8_t* __restrict__ out, int64_t nchunks) {
  using F = MmaFmt<FMT>;
  constexpr int BS = FMT == 8 ? 34 : 18;
  const int nb = K / QK;
  const int64_t qrow = FMT == 8 ? K : K / 2;
  for (int64_t c = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; c < nchunks;
       c += (int64_t)gridDim.x * blockDim.x) {
    const int64_t blk = c / (F::BLK / 16);
    const int off = (int)(c - blk * (F::BLK / 16)) * 16;
    const int64_t T = (M + TILE - 1) / TILE;
    const int kt = (int)(blk / T);
    const int64_t tile = blk - (int64_t)kt * T;
    // q8_0 quants are stored as w + 128 (sign bit flipped; padding is w = 0)
    const uint32_t qpad = FMT == 8 ? 0x80808080u : 0u;
    uint32_t w[4] = {0u, 0u, 0u, 0u};
    if (off < F::QST) {
      w[0] = w[1] = w[2] = w[3] = qpad;
      const int bx = off / (TILE * 128), r = (off % (TILE * 128)) / 128, pc = (off % 128) / 16;
      const int j = pc ^ (r & 7);
      const int64_t R = tile * TILE + r;
      const int64_t col = (int64_t)kt * F::QROW + bx * 128 + j * 16;  // quant byte in the row
      if (R < M && col < qrow) {
        if (!AOS) {
          const uint4 v = *reinterpret_cast<const uint4*>(q + R * qrow + col);
          w[0] = v.x ^ qpad; w[1] = v.y ^ qpad; w[2] = v.z ^ qpad; w[3] = v.w ^ qpad;
        } else {
          // q8_0: 16 of a block's 32 quants; q4_0: a block's 16 quant bytes
          const int64_t kb = FMT == 8 ? col / 32 : col / 16;
          const uint8_t* src = q + (R * nb + kb) * BS + 2 + (FMT == 8 ? col % 32 : 0);
#pragma unroll
          for (int i = 0; i < 4; ++i) w[i] = 0u;
#pragma unroll
          for (int i = 0; i < 16; ++i) w[i >> 2] |= (uint32_t)src[i] << (8 * (i & 3));
#pragma unroll
          for (int i = 0; i < 4; ++i) w[i] ^= qpad;
        }
      }
    } else {
      const int o = off - F::QST;
      const int r = o / ((KC / QK) * 2), b0 = (o % ((KC / QK) * 2)) / 2;
      const int64_t R = tile * TILE + r;
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const int kb = kt * (KC / QK) + b0 + e;
        uint32_t h = 0u;
        if (R < M && kb < nb) {
          if (!AOS) {
            h = d[R * nb + kb];
          } else {
            const uint8_t* src = q + (R * nb + kb) * BS;
            h = (uint32_t)src[0] | ((uint32_t)src[1] << 8);
          }
        }
        w[e >> 1] |= h << (16 * (e & 1));
      }
    }
    *reinterpret_cast<uint4*>(out + c * 16) = make_uint4(w[0], w[1], w[2], w[3]);
  }
}

// -------------------------------------------------------------- host side
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

std::mutex g_mu;
EncodeTiledFn g_encode = nullptr;

int get_encode(EncodeTiledFn* out) {
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_encode) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult qres;
    const cudaError_t e =
        cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &qres);
    if (e != cudaSuccess || qres != cudaDriverEntryPointSuccess || !fn)
      return set_error(ERR_CUDA, "cuTensorMapEncodeTiled is not available (%s)",
                       cudaGetErrorString(e));
    g_encode = reinterpret_cast<EncodeTiledFn>(fn);
  }
  *out = g_encode;
  return OK;
}

int encode_maps(int fmt, const void* q, const void* d, int64_t M, int64_t K, MmaArgs& a) {
  EncodeTiledFn enc;
  if (int rc = get_encode(&enc)) return rc;
  const cuuint64_t qrow = (cuuint64_t)(fmt == 8 ? K : K / 2);
  const cuuint64_t qdim[2] = {qrow, (cuuint64_t)M};
  const cuuint64_t qstride[1] = {qrow};
  const cuuint32_t qbox[2] = {128, TILE};
  const cuuint32_t one[2] = {1, 1};
  CUresult r = enc(&a.qmap, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(q), qdim, qstride,
                   qbox, one, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(ERR_CUDA, "tensor map of the quant plane: error %d", (int)r);
  const cuuint64_t ddim[2] = {(cuuint64_t)(K / QK), (cuuint64_t)M};
  const cuuint64_t dstride[1] = {(cuuint64_t)(K / QK) * 2};
  const cuuint32_t dbox[2] = {KC / QK, TILE};
  r = enc(&a.dmap, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, const_cast<void*>(d), ddim, dstride, dbox,
          one, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
          CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(ERR_CUDA, "tensor map of the scale plane: error %d", (int)r);
  return OK;
}

struct MmaPlan {
  int grid, S;
  size_t smem;
};
std::map<std::tuple<const void*, int, int64_t>, MmaPlan> g_plans;

// Consumer warps of the batch-tile kernel: 14 (15 warps with the producer,
// at most 4 per SM sub-partition, so 128 registers a thread) measured faster
// than 16 (17 warps, capped at 96 registers, small spills) at every batch
// width -- N = 16: 82.0 -> 75.9 us (q8_0) at 28672 x 8192 -- and than 12.
constexpr int TILE_CONS = 14;

template <int FMT, int NT, int TW, int KSPLIT, bool TILED>
int launch_mma(const GemvCall& c, const DeviceInfo& dev, cudaStream_t st) {
  using F = MmaFmt<FMT>;
  constexpr int SLOT = TILED ? ((FMT == 8 ? 2 : 4) * F::BLK + 1023) / 1024 * 1024 : F::SLOT;
  constexpr int CN = TILED ? TILE_CONS : CONS;
  constexpr size_t RED = TILED ? (size_t)(CN / 2) * NT * 4 * 32 * sizeof(float)
                               : (size_t)(CONS / KSPLIT) * (KSPLIT - 1) * TW * NT * 4 * 32 *
                                     sizeof(float);
  auto kern = TILED ? k_gemv_tiles<FMT, NT, CN> : k_gemv_mma<FMT, NT, TW, KSPLIT>;
  const void* kp = reinterpret_cast<const void*>(kern);
  MmaPlan pl;
  bool have = false;
  {
    std::lock_guard<std::mutex> lk(g_mu);
    auto it = g_plans.find(std::make_tuple(kp, dev.device, c.M));
    if (it != g_plans.end()) {
      pl = it->second;
      have = true;
    }
  }
  if (!have) {
    if (int rc = allow_max_smem(kp, dev)) return rc;
    cudaFuncAttributes fa;
    if (cudaFuncGetAttributes(&fa, kp) != cudaSuccess) return check_launch("cudaFuncGetAttributes");
    const size_t fixed = 1024 + 2 * (size_t)(NT * 8) * XS + RED;
    const size_t avail = (size_t)dev.smem_optin - fa.sharedSizeBytes;
    if (avail < fixed + 4 * (size_t)SLOT)
      return set_error(ERR_UNSUPPORTED, "shared memory too small for the tensor-core GEMV");
    pl.S = (int)std::min<size_t>(MAX_STAGES, (avail - fixed) / SLOT);
    pl.smem = fixed + (size_t)pl.S * SLOT;
    const int64_t T = (c.M + TILE - 1) / TILE;
    pl.grid = (int)std::max<int64_t>(1, std::min<int64_t>(dev.sms, T));
    std::lock_guard<std::mutex> lk(g_mu);
    g_plans[std::make_tuple(kp, dev.device, c.M)] = pl;
  }
  MmaArgs a;
  memset(&a, 0, sizeof(a));
  if (TILED) {
    a.tiled = static_cast<const uint8_t*>(c.q);
  } else if (int rc = encode_maps(FMT, c.q, c.d, c.M, c.K, a)) {
    return rc;
  }
  a.ws = static_cast<const uint8_t*>(c.ws);
  a.y = c.y;
  a.ldy = c.ldy;
  a.M = (int)c.M;
  a.K = (int)c.K;
  a.N = c.N;
  a.S = pl.S;

  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  // x prep: one CTA per column
  cfg.gridDim = dim3(c.N);
  cfg.blockDim = dim3(XPREP_THREADS);
  cfg.dynamicSmemBytes = 0;
  cudaError_t e = cudaLaunchKernelEx(&cfg, k_xprep, c.x, (int64_t)c.ldx, (int)c.K, c.N,
                                     static_cast<uint8_t*>(c.ws));
  if (e != cudaSuccess) return set_error(ERR_CUDA, "k_xprep launch: %s", cudaGetErrorString(e));
  cfg.gridDim = dim3(c.grid_override > 0 ? c.grid_override : pl.grid);
  cfg.blockDim = dim3(32 * (CN + 1));
  cfg.dynamicSmemBytes = pl.smem;
  e = cudaLaunchKernelEx(&cfg, kern, a);
  if (e != cudaSuccess) return set_error(ERR_CUDA, "k_gemv_mma launch: %s", cudaGetErrorString(e));
  return check_launch("k_gemv_mma");
}

// Two warps per row tile, two tiles per warp (16 tiles in flight per CTA):
// the fastest of the (tiles per warp, warps per tile) splits measured at
// 28672 x 8192 for every batch width.
template <bool TILED>
int dispatch_mma(int fmt, const GemvCall& c, cudaStream_t st) {
  DeviceInfo dev;
  if (int rc = current_device_info(dev)) return rc;
  if (fmt == 8)
    return c.N <= 8 ? launch_mma<8, 1, 2, 2, TILED>(c, dev, st)
                    : launch_mma<8, 2, 2, 2, TILED>(c, dev, st);
  return c.N <= 8 ? launch_mma<4, 1, 2, 2, TILED>(c, dev, st)
                  : launch_mma<4, 2, 2, 2, TILED>(c, dev, st);
}

int check_ws(const GemvCall& c) {
  if (!c.ws || c.ws_bytes < mma_workspace_bytes(c.K, c.N) ||
      (reinterpret_cast<uintptr_t>(c.ws) & 15) != 0)
    return set_error(ERR_ARG, "workspace of %zu bytes (16-byte aligned) needed, got %zu at %p",
                     mma_workspace_bytes(c.K, c.N), c.ws_bytes, c.ws);
  return OK;
}

}  // namespace

int encode_tensor_2d(CUtensorMap* map, bool u16, const void* base, uint64_t inner, uint64_t outer,
                     uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer, bool swizzle128) {
  EncodeTiledFn enc;
  if (int rc = get_encode(&enc)) return rc;
  const cuuint64_t dim[2] = {(cuuint64_t)inner, (cuuint64_t)outer};
  const cuuint64_t stride[1] = {(cuuint64_t)row_bytes};
  const cuuint32_t box[2] = {box_inner, box_outer};
  const cuuint32_t one[2] = {1, 1};
  const CUresult r =
      enc(map, u16 ? CU_TENSOR_MAP_DATA_TYPE_UINT16 : CU_TENSOR_MAP_DATA_TYPE_UINT8, 2,
          const_cast<void*>(base), dim, stride, box, one, CU_TENSOR_MAP_INTERLEAVE_NONE,
          swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(ERR_CUDA, "cuTensorMapEncodeTiled: error %d", (int)r);
  return OK;
}

size_t mma_workspace_bytes(int64_t K, int N) {
  const int64_t nkt = (K + KC - 1) / KC;
  const int cols = std::max(1, std::min(N, MAXC));
  return (size_t)HDR + (size_t)nkt * cols * XS;
}

bool mma_eligible(const GemvCall& c) {
  return c.N >= 2 && c.N <= MAXC && c.K >= 256 && c.K % 256 == 0 && c.K <= (1 << 20) &&
         c.M >= 1 && c.M < ((int64_t)1 << 31) &&
         (reinterpret_cast<uintptr_t>(c.d) & 15) == 0 &&
         (reinterpret_cast<uintptr_t>(c.q) & 15) == 0;
}

// Returns OK, an error status, or -1 when the call is not handled here.
int gemv_soa_mma(int fmt, const GemvCall& c, cudaStream_t st) {
  if (!mma_eligible(c)) return -1;
  if (int rc = check_ws(c)) return rc;
  return dispatch_mma<false>(fmt, c, st);
}

size_t tiled_bytes(int fmt, int64_t M, int64_t K) {
  const int64_t T = (M + TILE - 1) / TILE, nkt = (K + KC - 1) / KC;
  return (size_t)(T * nkt) * (fmt == 8 ? MmaFmt<8>::BLK : MmaFmt<4>::BLK);
}

int tile_weights(int fmt, bool aos, const void* q, const void* d, int64_t M, int64_t K,
                 void* out, cudaStream_t st) {
  const int64_t nchunks = (int64_t)(tiled_bytes(fmt, M, K) / 16);
  if (nchunks == 0) return OK;
  const int grid = (int)std::min<int64_t>((nchunks + 255) / 256, 148 * 16);
  const uint8_t* qb = static_cast<const uint8_t*>(q);
  const unsigned short* db = static_cast<const unsigned short*>(d);
  uint8_t* o = static_cast<uint8_t*>(out);
  if (fmt == 8) {
    if (aos) k_tile<8, true><<<grid, 256, 0, st>>>(qb, db, M, (int)K, o, nchunks);
    else k_tile<8, false><<<grid, 256, 0, st>>>(qb, db, M, (int)K, o, nchunks);
  } else {
    if (aos) k_tile<4, true><<<grid, 256, 0, st>>>(qb, db, M, (int)K, o, nchunks);
    else k_tile<4, false><<<grid, 256, 0, st>>>(qb, db, M, (int)K, o, nchunks);
  }
  return check_launch("k_tile");
}

// GEMV over batch tiles, 1..16 columns per launch.
int gemv_tiled(int fmt, const GemvCall& c, cudaStream_t st) {
  if (int rc = check_ws(c)) return rc;
  return dispatch_mma<true>(fmt, c, st);
}

int set_mma_spin_limit(long long cycles) {
  const cudaError_t e = cudaMemcpyToSymbol(g_mma_spin_limit, &cycles, sizeof(cycles));
  if (e == cudaSuccess) return OK;
  return set_error(ERR_CUDA, "setting the wait limit: %s", cudaGetErrorString(e));
}

int read_mma_error(int clear, cudaStream_t st, int* out) {
  int v = 0;
  cudaError_t e = cudaMemcpyFromSymbolAsync(&v, g_mma_error, sizeof(int), 0,
                                            cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e != cudaSuccess) return set_error(ERR_CUDA, "reading the device error word: %s", cudaGetErrorString(e));
  if (clear && v) {
    const int zero = 0;
    e = cudaMemcpyToSymbolAsync(g_mma_error, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) return set_error(ERR_CUDA, "clearing the device error word: %s", cudaGetErrorString(e));
  }
  *out = v;
  return OK;
}

}  // namespace qg
