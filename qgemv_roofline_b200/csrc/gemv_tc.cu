// Small-batch q8_0 GEMV on the 5th-generation tensor cores (tcgen05, sm_100a).
//
// Y[n][r] = sum_b d[r][b] * sum_j q[r][32b + j] * X[n][32b + j] for up to 16
// columns n per launch, the weights streamed once.  One ggml block is one
// MMA: tcgen05.mma kind::i8 with K = 32 multiplies the block's int8 quants
// (the A operand, read by the tensor core straight from shared memory: no
// conversion instruction) by the block's activations in exact integer form,
// and leaves the integer block dots in tensor memory (TMEM), where the CUDA
// cores scale them once per block:
//
//  * x (prep kernel, many CTAs): each 32-element block of a column is
//    rounded to block fixed point X_j = rint(x_j 2^(22-e)), |x| < 2^e on the
//    block, |X_j| <= 2^22, and split into three signed byte digits
//    X = p0 + 2^8 p1 + 2^16 p2 (p0, p1 in [-128, 127], p2 in [-64, 64]).  The
//    digits are the B operand, row plane * NC + column, so one MMA (M = 128
//    rows, N = 8 to 48, K = 32) computes the three plane sums S_p of every
//    column for 128 rows and one block, exactly (|S_p| < 2^19).  The block
//    scale is 2^(e + sh - 22), where 2^sh normalises the column (max |x 2^sh|
//    in [2^14, 2^15), so no scale leaves the float range); the GEMV derives
//    sh from the prep CTAs' maxima.
//  * epilogue (8 warps; TMEM lane = row): lo = S0 + 2^8 S1 (exact in int32),
//    F = 2^16 S2 + lo in fp32, acc[n] += F * (d * 2^(e+sh-22)); y = acc 2^-sh.
//    The rounding of x to the 2^(e-22) grid moves a row's dot by at most
//    2^-23 sqrt(32) ||w|| ||x|| (Cauchy-Schwarz over each block), the fp32
//    steps by a few ulps of the block terms: well inside 1e-5 ||w|| ||x||.
//    A column holding a NaN or an infinity gives NaN in every row.
//
// Weights are "tc tiles" (qgemv_q8_0_tc_tile, a one-time re-layout): per
// 128 rows x 256 columns one contiguous tile, the quants in the canonical
// 128-byte-swizzled K-major layout the tensor core reads (2 boxes of
// [128 rows][128 bytes]; 16-byte chunk c of row r at chunk position
// c ^ (r % 8) of its 128-byte row; rows in groups of 8 at 1024 bytes), then
// the [128 rows][8 blocks] fp16 scales; rows beyond M and columns beyond K
// hold zero weights.  The tiles of one 128-row tile are consecutive in K.
//
// The (row tile, K tile) units are split evenly over one CTA per SM (a unit
// is 34 KB of weights: the imbalance is at most one unit).  A row tile that
// two or more CTAs share is finished by the epilogue warp that stores the
// last part (a counter per row tile): it adds the CTAs' partial sums in CTA
// order, so results do not depend on timing.
//
// Per CTA (11 warps; 19 for q4_0): warp 0
// streams each unit with bulk copies into two shared-memory rings: the quants
// and the x digits (what the MMAs read) into a ring of 3-6 weight stages,
// freed by the MMAs' commits (and, for q4_0, by the converter warps), and the
// tile's fp16 scales with the x block exponents into an 8-slot scale ring,
// freed by the epilogue; so the weight stream never waits for the epilogue's
// arithmetic.  One thread each of warps 1 and 2 (a tcgen05.mma costs ~80-90
// cycles to issue) issues half of every unit's blocks, 4 (or, at 16 columns,
// 2) blocks into each slot of its own TMEM ring, and commits each slot to an
// mbarrier; the epilogue warps 3..10 (2 groups of four, one warp per TMEM
// lane quarter, group g taking the g-th half of the columns) read
// their part of a whole slot back with one wait (tcgen05.ld), release it and
// accumulate: the TMEM read latency is paid once per slot, not once per
// block.  No barrier joins the epilogue warps: each owns its rows and
// columns, and at the end of a row tile stores y (or, for a row tile shared
// with other CTAs, its part).  For q4_0, the 8 warps after the epilogue's
// widen each unit's nibbles into a 3-slot A ring first.
// Every wait is bounded (the library's wait limit): on timeout the error word
// records QGEMV_ERR_TIMEOUT, the producer stops and waits for its copies, the
// MMA threads stop issuing, the epilogue runs out its loop without waiting,
// and the CTA frees its TMEM before it returns.
#include "qgemv_common.cuh"
#include "qgemv_internal.h"

#include <algorithm>
#include <cstring>

namespace qg {

__device__ int g_tc_error = 0;
__device__ long long g_tc_spin_limit = kDefaultSpinLimit;

namespace {

constexpr int TC_M = 128;                       // rows per tile (MMA M)
constexpr int TC_KT = 256;                      // K per tile
constexpr int TC_BLK = TC_KT / QK;              // blocks per tile (8)
constexpr int TC_ABYTES = TC_M * TC_KT;         // quants of a tile
constexpr int TC_BOX = TC_M * 128;              // one 128-byte-wide box of quants
constexpr int TC_DBYTES = TC_M * TC_BLK * 2;    // fp16 scales of a tile
constexpr int TC_TMEM_COLS = 512;
constexpr int TC_EPI_MAX = 16;                  // epilogue warps, at most (4 column groups)
constexpr int TC_MMAW = 2;                      // MMA-issuing warps (each its own TMEM half)
constexpr int TC_W0E = 1 + TC_MMAW;             // first epilogue warp
constexpr int TC_PMAX = 64;                     // x prep chunks per column, at most
// workspace header: per column and prep chunk, the chunk's max |x| as bits
// (0xFFFFFFFF when the chunk holds a NaN or an infinity)
constexpr int TC_HDR = 16 * TC_PMAX * 4;
constexpr int TC_EMPTY = -100000;               // block exponent of an all-zero block
constexpr int TC_SMEM_MAX = 227 * 1024 - 1024;  // shared memory we use at most (dynamic + scratch)
constexpr int TC_MAXSLOTS = 8;                  // TMEM slots, at most
// units whose weights are copied before the dependency wait (the x digits of
// every unit come after it); the rest of the ring fills after the x copies
// of these, so x does not queue behind a whole ring of weights (28672x8192,
// against prefetching the whole ring: q8_0 8 columns 53.4 -> 52.7 us, q4_0
// 1-2 columns 49.5 -> 49.1 us)
constexpr int TC_PRE = 2;

// What depends on the column count only (the x side, shared with the prep).
template <int NC>
struct TcCfg {
  // MMA N = B rows, of which 3 * NC hold digits (N = 8, 16, 32 or 48)
  static constexpr int NB = NC == 16 ? 48 : NC == 8 ? 32 : NC == 4 ? 16 : 8;
  static constexpr int BBOX = NB * 128;               // one box of x digits
  static constexpr int XB = 2 * BBOX;                 // x digits of a K tile
  static constexpr int XSB = TC_BLK * NC * 4;         // block exponents [block][column] int32
  static constexpr int XT = XB + XSB;                 // x tile bytes (multiple of 16)
  // scale slot: the tile's fp16 scales + x block exponents (read by the epilogue)
  static constexpr int SSLOT = (TC_DBYTES + XSB + 127) / 128 * 128;
  static constexpr int BPS = NC == 16 ? 2 : 4;        // blocks per TMEM slot (one read)
  static constexpr int NSL = TC_BLK / BPS;            // TMEM slots per tile
  static constexpr int SPW = NSL / TC_MMAW;           // of which each MMA warp issues
  static constexpr int REG = TC_TMEM_COLS / TC_MMAW;  // TMEM columns of one MMA warp
  // slots in each MMA warp's own ring
  static constexpr int SLW = REG / (BPS * NB) > TC_MAXSLOTS ? TC_MAXSLOTS : REG / (BPS * NB);
  // kind::i8: s32 accumulators (bits 4-5 = 2), A and B signed (bits 7-9,
  // 10-12 = 1), both K-major (bits 15, 16 = 0), N >> 3 at bit 17, M >> 4 at 24
  static constexpr uint32_t IDESC = (2u << 4) | (1u << 7) | (1u << 10) |
                                    ((uint32_t)(NB >> 3) << 17) | ((uint32_t)(TC_M >> 4) << 24);
};

// q8_0 tiles hold the int8 quants in the MMA's A layout; q4_0 tiles hold the
// nibbles packed as [8 blocks][128 rows][16 bytes], widened to int8 (n - 8)
// in the A layout by 8 converter warps, into a 3-slot A ring.
template <int FMT> __host__ __device__ constexpr int tc_qbytes() { return FMT == 8 ? TC_ABYTES : TC_ABYTES / 2; }
template <int FMT> __host__ __device__ constexpr int tc_tile() { return tc_qbytes<FMT>() + TC_DBYTES; }

template <int FMT, int NC>
struct TcFmt : TcCfg<NC> {
  static constexpr int QB = tc_qbytes<FMT>();         // quant bytes per tile
  static constexpr int TILE = tc_tile<FMT>();         // 34816 (q8_0), 18432 (q4_0)
  static constexpr int CONV = FMT == 8 ? 0 : 8;       // converter warps
  // epilogue: G column groups of 4 warps (one per TMEM lane quarter); 4 groups
  // at 8 and 16 columns measured no faster (28672x8192 q8_0: 56.1 / 75.6 us
  // against 53.9 / 75.6 us with 2), so 2 everywhere
  static constexpr int G = 2;
  static constexpr int EPI = 4 * G;
  static constexpr int SA = FMT == 8 ? 0 : 3;         // A ring slots (q4_0)
  static constexpr int SAD = SA > 0 ? SA : 1;         // SA as a divisor (q8_0 never divides)
  // scale ring slots: q8_0 at 8 and 16 columns 12, where the epilogue's
  // arithmetic makes it the slowest consumer and a deeper ring lets the
  // weights run ahead (28672x8192, 8 columns: 54.8 -> 53.7 us, though it
  // leaves one weight stage fewer; 10 slots and 5 stages: 54.2 us); 8
  // otherwise (q8_0 at 2 columns with 12 slots and 5 weight stages: 44.6 ->
  // 47.2 us; q4_0 at 8 columns: 65.2 -> 66.0 us)
  static constexpr int SS = FMT == 8 && NC >= 8 ? 12 : 8;
  static constexpr int THREADS = 32 * (TC_W0E + EPI + CONV);
  // weight stage: quants + x digits (what the MMAs, or the converters, read)
  static constexpr int WSTAGE = QB + TcCfg<NC>::XB;   // a multiple of 1024
  // left for weight stages: the budget minus alignment slack, the scale and A
  // rings and the epilogue warps' static scratch (8 x 8 NC floats)
  static constexpr int FREE =
      TC_SMEM_MAX - 1024 - SS * TcCfg<NC>::SSLOT - SA * TC_ABYTES - 8 * NC * 4 * 4;
  // weight stages: q4_0 at most 4 (28672x8192, 1-2 columns: 3 / 4 / 5 / 6
  // stages 52.2 / 49.5 / 50.4 / 51.0 us; its 3 A slots, not the weight ring,
  // set the pace: 1 A slot 62 us, 2 slots 51.0 us)
  static constexpr int SWMAX = FMT == 8 ? 8 : 4;
  static constexpr int SW = FREE / WSTAGE > SWMAX ? SWMAX : FREE / WSTAGE;
  static constexpr size_t SMEM =
      (size_t)SW * WSTAGE + (size_t)SA * TC_ABYTES + (size_t)SS * TcCfg<NC>::SSLOT + 1024;
};
static_assert(TcFmt<8, 16>::SMEM + 8 * 16 * 4 * 4 <= TC_SMEM_MAX &&
                  TcFmt<4, 16>::SMEM + 8 * 16 * 4 * 4 <= TC_SMEM_MAX &&
                  TcFmt<8, 2>::SMEM <= TC_SMEM_MAX && TcFmt<4, 2>::SMEM <= TC_SMEM_MAX,
              "ring too large");
static_assert(TcFmt<8, 16>::SW >= 4 && TcFmt<8, 8>::SW >= 4 && TcFmt<4, 16>::SW >= 3 &&
                  TcFmt<8, 2>::SW == 6 && TcFmt<4, 2>::SW == 4,
              "ring depth");
static_assert(TcCfg<16>::SLW == 2 && TcCfg<8>::SLW == 2 && TcCfg<4>::SLW == 4 &&
                  TcCfg<2>::SLW == 8 && TcCfg<16>::SPW >= 1 && TcCfg<2>::SPW >= 1 &&
                  TcCfg<16>::SLW >= TcCfg<16>::SPW && TcCfg<8>::SLW >= TcCfg<8>::SPW,
              "TMEM rings");
static_assert(TC_ABYTES % 1024 == 0 && TcFmt<4, 2>::WSTAGE % 1024 == 0 &&
                  TcFmt<8, 2>::WSTAGE % 1024 == 0,
              "operands stay 1024-byte aligned");

__device__ __forceinline__ long long tc_spin_limit() {
  return *(volatile long long*)&g_tc_spin_limit;
}
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
// Bounded wait; gives up at once when another thread raised the abort flag.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag) {
  if (mbar_try(bar, parity)) return true;
  const long long t0 = clock64(), lim = tc_spin_limit();
  while (!mbar_try(bar, parity)) {
    if (*abort_flag) return false;
    if (clock64() - t0 > lim) {
      atomicExch(&g_tc_error, (int)ERR_TIMEOUT);
      __threadfence();
      *abort_flag = 1;
      return false;
    }
  }
  return true;
}
// Wait for copies and MMAs in flight (they complete on their own) before the
// CTA exits: ignores the abort flag, bounded by the default limit even when
// the configured one is shorter.
__device__ __forceinline__ void mbar_wait_drain(uint32_t bar, uint32_t parity) {
  const long long t0 = clock64(), lim = max(tc_spin_limit(), kDefaultSpinLimit);
  while (!mbar_try(bar, parity) && clock64() - t0 < lim) {
  }
}
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count));
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
          "r"(dst),
      "l"(src), "r"(bytes), "r"(bar)
      : "memory");
}

// Shared-memory matrix descriptor of a K-major operand in the canonical
// 128-byte-swizzled layout: start address >> 4 (bits 0-13), leading byte
// offset 16 >> 4 (bits 16-29; not used by swizzled K-major operands), stride
// byte offset 1024 >> 4 between 8-row groups (bits 32-45), descriptor version
// 1 (bits 46-47), base offset 0 (atoms 1024-byte aligned), layout type 2 =
// SWIZZLE_128B (bits 61-63).  Block b of a box starts 32 * b bytes into the
// atom row: the hardware applies the swizzle to the computed addresses.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t addr) {
  return (uint64_t)((addr >> 4) & 0x3FFFu) | ((uint64_t)1u << 16) | ((uint64_t)(1024u >> 4) << 32) |
         ((uint64_t)1u << 46) | ((uint64_t)2u << 61);
}

// 2-D tiled tensor copy global -> shared (no multicast); c0 is the inner
// coordinate in elements (its byte offset a multiple of 16), c1 the row.
__device__ __forceinline__ void tensor_g2s(uint32_t dst, const CUtensorMap* map, int c0, int c1,
                                           uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(bar)
      : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   bar)
               : "memory");
}

// 32 lanes x NC consecutive 32-bit TMEM columns.
template <int NC>
__device__ __forceinline__ void tmem_ld(uint32_t ta, uint32_t (&v)[NC]) {
  if constexpr (NC == 1) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x1.b32 {%0}, [%1];" : "=r"(v[0]) : "r"(ta));
  } else if constexpr (NC == 2) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x2.b32 {%0, %1}, [%2];"
                 : "=r"(v[0]), "=r"(v[1])
                 : "r"(ta));
  } else if constexpr (NC == 4) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3])
                 : "r"(ta));
  } else if constexpr (NC == 8) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
                 : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]),
                   "=r"(v[6]), "=r"(v[7])
                 : "r"(ta));
  } else {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
        "%11, %12, %13, %14, %15}, [%16];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
          "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]),
          "=r"(v[14]), "=r"(v[15])
        : "r"(ta));
  }
}

struct TcArgs {
  // SoA planes (soa != 0): quants [M][K or K/2] bytes in boxes of 128 bytes x
  // 128 rows, 128-byte swizzle (exactly the MMA's A layout for q8_0); scales
  // [M][K/32] fp16 in boxes of 8 x 128 rows ([row][block], as in a tc tile)
  alignas(64) CUtensorMap qmap;
  alignas(64) CUtensorMap dmap;
  int soa;
  const uint8_t* tiles;  // tc tiles [row tile][K tile] (soa == 0)
  uint8_t* ws;           // header, counters, partial sums, x tiles
  float* y;
  int64_t ldy;
  int M, N, nkt, ntiles;
  int nchunk;                     // x prep chunks per column
  int cnt_off, part_off, xt_off;  // workspace offsets (bytes)
};

// q4_0 nibbles to int8: the 4 bytes of w hold weights j (low nibbles) and
// j + 16 (high nibbles) of 4 consecutive j; n - 8 as a signed byte is the
// nibble with bit 3 flipped (a 4-bit two's complement value), sign-extended:
// m | 0xF0 where bit 3 of m is set, i.e. m + 0x1E * (bit 3 of m).
__device__ __forceinline__ void widen_q4(uint32_t w, uint32_t& lo, uint32_t& hi) {
  const uint32_t ml = (w & 0x0F0F0F0Fu) ^ 0x08080808u;
  const uint32_t mh = ((w >> 4) & 0x0F0F0F0Fu) ^ 0x08080808u;
  lo = ml + (ml & 0x08080808u) * 0x1Eu;  // 0x08 * 0x1E = 0xF0: no carry between bytes
  hi = mh + (mh & 0x08080808u) * 0x1Eu;
}

// The CTA that owns unit u when U units are split over G CTAs as
// [U c / G, U (c + 1) / G).
__device__ __forceinline__ int cta_of(int64_t u, int64_t U, int G) {
  return (int)(((u + 1) * G + U - 1) / U) - 1;
}

// y from the accumulated sum: NaN for a column holding a NaN or an infinity,
// else the sum scaled back by 2^-sh.
__device__ __forceinline__ float finish(float tot, int sh, bool nonfinite) {
  return nonfinite ? __int_as_float(0x7FC00000) : ldexpf(tot, -sh);
}

// 2^k as a float, 0 below the normal range (k <= 15 here).
__device__ __forceinline__ float exp2i(int k) {
  return k >= -126 ? __int_as_float((k + 127) << 23) : 0.0f;
}

template <int FMT, int NC>
__global__ void __launch_bounds__(TcFmt<FMT, NC>::THREADS, 1)
    k_gemv_tc(const __grid_constant__ TcArgs p) {
  using C = TcFmt<FMT, NC>;
  constexpr int SW = C::SW;
  extern __shared__ uint8_t tc_smem_raw[];
  __shared__ __align__(8) unsigned long long full[SW];       // weight stage landed
  __shared__ __align__(8) unsigned long long empty[SW];      // its MMAs (and converters) read it
  __shared__ __align__(8) unsigned long long afull[4];       // q4_0: A slot widened
  __shared__ __align__(8) unsigned long long aempty[4];      // q4_0: its MMAs have read it
  constexpr int SS = C::SS;
  static_assert(SW <= SS, "the first SW units' scales are prefetched into distinct slots");
  __shared__ __align__(8) unsigned long long sfull[SS];   // scale slot landed
  __shared__ __align__(8) unsigned long long sempty[SS];  // the epilogue is done with it
  __shared__ __align__(8) unsigned long long tfull[TC_MMAW][TC_MAXSLOTS];   // MMAs of a slot done
  __shared__ __align__(8) unsigned long long tempty[TC_MMAW][TC_MAXSLOTS];  // the epilogue read it
  __shared__ __align__(8) unsigned long long mma_done;
  __shared__ uint32_t tmem_base;
  __shared__ int abort_flag;
  __shared__ float xscr[C::EPI][8 * NC / C::G];  // per epilogue warp: block scales of a unit

  // 1024-byte-aligned weight ring (the swizzle works on address bits), the A
  // ring (q4_0), then the scale ring
  uint8_t* ring = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(tc_smem_raw) + 1023) & ~(uintptr_t)1023);
  uint8_t* aring = ring + (size_t)SW * C::WSTAGE;
  uint8_t* sring = aring + (size_t)C::SA * TC_ABYTES;
  const uint32_t ring_s = saddr(ring), aring_s = saddr(aring), sring_s = saddr(sring);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t U = (int64_t)p.ntiles * p.nkt;
  const int64_t u0 = U * blockIdx.x / gridDim.x, u1 = U * (blockIdx.x + 1) / gridDim.x;
  const int nunits = (int)(u1 - u0);

  if (threadIdx.x == 0) {
    for (int s = 0; s < SW; ++s) {
      mbar_init(saddr(&full[s]), 1);
      mbar_init(saddr(&empty[s]), TC_MMAW + C::CONV);  // each MMA warp's commit (+ converter warps)
    }
    for (int s = 0; s < C::SA; ++s) {
      mbar_init(saddr(&afull[s]), C::CONV);  // every converter warp
      mbar_init(saddr(&aempty[s]), TC_MMAW);  // each MMA warp's commit
    }
    for (int s = 0; s < SS; ++s) {
      mbar_init(saddr(&sfull[s]), 1);
      mbar_init(saddr(&sempty[s]), C::EPI);  // every epilogue warp
    }
    for (int w = 0; w < TC_MMAW; ++w)
      for (int s = 0; s < C::SLW; ++s) {
        mbar_init(saddr(&tfull[w][s]), 1);
        mbar_init(saddr(&tempty[w][s]), C::EPI);  // every epilogue warp reads every slot
      }
    mbar_init(saddr(&mma_done), TC_MMAW);  // one commit per MMA warp
    abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {  // all of TMEM: one CTA per SM (shared memory)
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     saddr(&tmem_base)),
                 "r"(TC_TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    // unit i: quants -> weight stage i % SW, x digits behind them; the tile's
    // scales and the x block scales -> scale slot i % SS
    if (lane == 0) {
      const uint8_t* xt = p.ws + p.xt_off;
      // weights do not depend on the previous kernel: prefetch TC_PRE units
      // first; the loop below waits on a stage's release only once it has
      // been used (a fresh barrier passes the wait for the phase before it)
      const int pre = min(min(SW, TC_PRE), nunits);
      // unit u's quants and fp16 scales: one tc tile (two bulk copies) or,
      // from SoA planes, 2-D tensor copies of 128 rows (q8_0: two 128-byte
      // boxes; q4_0: one) and one scale box; rows past M read as zeros
      auto load_w = [&](int64_t u, uint32_t wdst, uint32_t sdst, uint32_t fb, uint32_t sb) {
        if (p.soa) {
          const int rt = (int)(u / p.nkt), kt = (int)(u % p.nkt);
          if (FMT == 8) {
            tensor_g2s(wdst, &p.qmap, kt * TC_KT, rt * TC_M, fb);
            tensor_g2s(wdst + TC_BOX, &p.qmap, kt * TC_KT + 128, rt * TC_M, fb);
          } else {
            tensor_g2s(wdst, &p.qmap, kt * (TC_KT / 2), rt * TC_M, fb);
          }
          tensor_g2s(sdst, &p.dmap, kt * TC_BLK, rt * TC_M, sb);
        } else {
          const uint8_t* t = p.tiles + u * C::TILE;
          bulk_g2s(wdst, t, C::QB, fb);
          bulk_g2s(sdst, t + C::QB, TC_DBYTES, sb);
        }
      };
      for (int i = 0; i < pre; ++i) {
        mbar_expect_tx(saddr(&full[i]), (uint32_t)(C::QB + C::XB));
        mbar_expect_tx(saddr(&sfull[i]), (uint32_t)(TC_DBYTES + C::XSB));
        load_w(u0 + i, ring_s + (uint32_t)(i * C::WSTAGE), sring_s + (uint32_t)(i * C::SSLOT),
               saddr(&full[i]), saddr(&sfull[i]));
      }
      asm volatile("griddepcontrol.wait;" ::: "memory");  // x tiles are written by the prep kernel
      for (int i = 0; i < pre; ++i) {
        const uint8_t* x = xt + (int64_t)((u0 + i) % p.nkt) * C::XT;
        bulk_g2s(ring_s + (uint32_t)(i * C::WSTAGE + C::QB), x, C::XB, saddr(&full[i]));
        bulk_g2s(sring_s + (uint32_t)(i * C::SSLOT + TC_DBYTES), x + C::XB, C::XSB, saddr(&sfull[i]));
      }
      int issued = pre;
      for (int i = pre; i < nunits; ++i) {
        const int s = i % SW, j = i % SS;
        if (!mbar_wait(saddr(&empty[s]), (uint32_t)(((i / SW) - 1) & 1), &abort_flag)) break;
        if (i >= SS &&
            !mbar_wait(saddr(&sempty[j]), (uint32_t)(((i / SS) - 1) & 1), &abort_flag))
          break;
        const int64_t u = u0 + i;
        const uint8_t* x = xt + (int64_t)(u % p.nkt) * C::XT;
        mbar_expect_tx(saddr(&full[s]), (uint32_t)(C::QB + C::XB));
        mbar_expect_tx(saddr(&sfull[j]), (uint32_t)(TC_DBYTES + C::XSB));
        load_w(u, ring_s + (uint32_t)(s * C::WSTAGE), sring_s + (uint32_t)(j * C::SSLOT),
               saddr(&full[s]), saddr(&sfull[j]));
        bulk_g2s(ring_s + (uint32_t)(s * C::WSTAGE + C::QB), x, C::XB, saddr(&full[s]));
        bulk_g2s(sring_s + (uint32_t)(j * C::SSLOT + TC_DBYTES), x + C::XB, C::XSB, saddr(&sfull[j]));
        issued = i + 1;
      }
      if (issued < nunits) {  // aborted: wait (bounded) for the copies still in flight
        for (int i = max(0, issued - SW); i < issued; ++i)
          mbar_wait_drain(saddr(&full[i % SW]), (uint32_t)((i / SW) & 1));
        for (int i = max(0, issued - SS); i < issued; ++i)
          mbar_wait_drain(saddr(&sfull[i % SS]), (uint32_t)((i / SS) & 1));
      }
    }
  } else if (warp <= TC_MMAW) {
    // --------------------------------------------------------- MMA issuers
    // one thread per MMA warp; warp w (= mw + 1) issues slots mw * SPW ...
    // (mw + 1) * SPW - 1 of every unit (a tcgen05.mma costs ~80-90 cycles to
    // issue from one thread), into its own ring of SLW TMEM slots in columns
    // mw * REG ...: each ring has one issuer, in order, so a slot's previous
    // use is always issued before the wait for its release
    if (lane == 0) {
      const int mw = warp - 1;
      bool ok = true;
      for (int i = 0; i < nunits && ok; ++i) {
        const int s = i % SW;
        ok = mbar_wait(saddr(&full[s]), (uint32_t)((i / SW) & 1), &abort_flag);
        // q4_0: the widened quants of unit i are in A slot i % SA
        if (ok && FMT == 4)
          ok = mbar_wait(saddr(&afull[i % C::SAD]), (uint32_t)((i / C::SAD) & 1), &abort_flag);
        if (!ok) break;
        tc_fence_after();
        const uint32_t b0 = ring_s + (uint32_t)(s * C::WSTAGE + C::QB);
        const uint32_t a0 = FMT == 8 ? ring_s + (uint32_t)(s * C::WSTAGE)
                                     : aring_s + (uint32_t)((i % C::SAD) * TC_ABYTES);
        // descriptors of block 0; block b adds its byte offset >> 4 (the start
        // address field, bits 0-13, cannot carry: shared addresses < 256 KB)
        const uint64_t da0 = sw128_desc(a0), db0 = sw128_desc(b0);
        // slot sl = mw SPW + r of the tile (blocks sl * BPS ...) into ring
        // slot hl % SLW, hl = SPW i + r
#pragma unroll
        for (int r = 0; r < C::SPW && ok; ++r) {
          const int sl = mw * C::SPW + r;
          const uint32_t hl = (uint32_t)C::SPW * i + r, slot = hl % C::SLW;
          if (hl >= (uint32_t)C::SLW) {
            ok = mbar_wait(saddr(&tempty[mw][slot]), ((hl / C::SLW) - 1) & 1u, &abort_flag);
            if (!ok) break;
            tc_fence_after();
          }
#pragma unroll
          for (int bb = 0; bb < C::BPS; ++bb) {
            // block b: box b / 4, 32-byte K step b % 4 inside its 128-byte rows
            const int b = sl * C::BPS + bb;
            const uint64_t da = da0 + (uint64_t)((((b >> 2) * TC_BOX + (b & 3) * 32)) >> 4);
            const uint64_t db = db0 + (uint64_t)((((b >> 2) * C::BBOX + (b & 3) * 32)) >> 4);
            asm volatile(
                "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
                " tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n}\n" ::"r"(
                    tmem + mw * C::REG + (slot * C::BPS + bb) * C::NB),
                "l"(da), "l"(db), "r"(C::IDESC), "r"(0)
                : "memory");
          }
          tc_commit(saddr(&tfull[mw][slot]));
        }
        if (!ok) break;
        tc_commit(saddr(&empty[s]));  // the stage is free once these MMAs have read it
        if (FMT == 4) tc_commit(saddr(&aempty[i % C::SAD]));  // and so is the A slot
      }
      // every MMA issued completes before the accumulators are freed
      tc_commit(saddr(&mma_done));
      mbar_wait_drain(saddr(&mma_done), 0u);
    }
  } else if (FMT == 4 && warp >= TC_W0E + C::EPI) {
    // ---------------------------------------------------------- converters
    // q4_0: thread (r, h) (one per row of the tile and half of its blocks)
    // widens blocks 4h .. 4h + 3 of row r (16 bytes of nibbles each: weight j
    // low nibble, j + 16 high) into int8 n - 8 at the A layout's swizzled
    // positions, unit after unit into A slot i % SA
    const int ct = threadIdx.x - 32 * (TC_W0E + C::EPI);  // 0..255
    const int r = ct & (TC_M - 1), h = ct >> 7;
    bool ok = true;
    for (int i = 0; i < nunits && ok; ++i) {
      const int s = i % SW;
      ok = mbar_wait(saddr(&full[s]), (uint32_t)((i / SW) & 1), &abort_flag);
      if (ok && i >= C::SA)
        ok = mbar_wait(saddr(&aempty[i % C::SAD]), (uint32_t)(((i / C::SAD) - 1) & 1), &abort_flag);
      if (!ok) break;
      tc_fence_after();  // the A slot was last read by MMAs (async proxy)
      const uint8_t* pk = ring + (size_t)s * C::WSTAGE;
      uint8_t* arow = aring + (size_t)(i % C::SAD) * TC_ABYTES + h * TC_BOX + (r >> 3) * 1024 +
                      (r & 7) * 128;
      uint4 w[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        // block 4h + k of row r: tc tile [block][row][16 bytes]; SoA box
        // [row][128 bytes], 16-byte chunk c at position c ^ (r % 8)
        const int b = 4 * h + k;
        w[k] = *reinterpret_cast<const uint4*>(pk + (p.soa ? r * 128 + ((b ^ (r & 7)) << 4)
                                                            : (b * TC_M + r) * 16));
      }
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        uint4 lo, hi;
        widen_q4(w[k].x, lo.x, hi.x);
        widen_q4(w[k].y, lo.y, hi.y);
        widen_q4(w[k].z, lo.z, hi.z);
        widen_q4(w[k].w, lo.w, hi.w);
        // block 4h + k: box h, 16-byte chunks 2k (weights 0-15) and 2k + 1
        // (weights 16-31) of the row, swizzled
        *reinterpret_cast<uint4*>(arow + (((2 * k) ^ (r & 7)) << 4)) = lo;
        *reinterpret_cast<uint4*>(arow + (((2 * k + 1) ^ (r & 7)) << 4)) = hi;
      }
      // generic-proxy stores, read next by the tensor core (async proxy)
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(saddr(&afull[i % C::SAD]));
        mbar_arrive(saddr(&empty[s]));  // the packed quants are read
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    asm volatile("griddepcontrol.wait;" ::: "memory");  // header and counters
    constexpr int NCH = NC / C::G;  // columns per warp
    const int e = warp - TC_W0E;
    const int quarter = warp & 3;  // TMEM lanes 32 * quarter ... (this warp's rows)
    const int g = e >> 2;          // this warp's columns: g * NCH ... (g + 1) * NCH - 1
    const int row = quarter * 32 + lane;
    // column n's normalisation 2^sh (max |x'| in [2^14, 2^15), exact) from
    // the prep chunks' maxima; nonfinite: the column holds a NaN or an infinity
    int shc[NCH];
    bool nfc[NCH];
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      const uint32_t* cm = reinterpret_cast<const uint32_t*>(p.ws) + (g * NCH + c) * TC_PMAX;
      uint32_t m = 0u;
      bool bad = false;
      for (int k = lane; k < p.nchunk; k += 32) {
        const uint32_t v = cm[k];
        if (v == 0xFFFFFFFFu) bad = true;
        else m = max(m, v);
      }
      for (int o = 16; o; o >>= 1) m = max(m, __shfl_xor_sync(0xffffffffu, m, o));
      int sh = 0;
      if (m != 0u) {
        int ee;
        frexpf(__uint_as_float(m), &ee);  // max = f 2^ee, f in [0.5, 1)
        sh = 15 - ee;
      }
      shc[c] = sh;
      nfc[c] = __any_sync(0xffffffffu, bad);
    }
    // lane l converts the block exponents of (block l / NCH, column l % NCH)
    // (and of block (l + 32) / NCH when 8 NCH > 32) into block scales
    int sh_l = 0;
#pragma unroll
    for (int c = 0; c < NCH; ++c)
      if (c == lane % NCH) sh_l = shc[c];
    unsigned* cnt = reinterpret_cast<unsigned*>(p.ws + p.cnt_off);
    float* part = reinterpret_cast<float*>(p.ws + p.part_off);
    float acc[NCH];
#pragma unroll
    for (int c = 0; c < NCH; ++c) acc[c] = 0.0f;
    for (int i = 0; i < nunits; ++i) {
      const int j = i % SS;
      const int64_t u = u0 + i;
      const int rt = (int)(u / p.nkt), kt = (int)(u % p.nkt);
      // the unit's scales: scale slot j
      mbar_wait(saddr(&sfull[j]), (uint32_t)((i / SS) & 1), &abort_flag);
      const uint8_t* sst = sring + (size_t)j * C::SSLOT;
      const uint4 d8 = *reinterpret_cast<const uint4*>(sst + row * 16);  // 8 fp16
      // block scales 2^(e + sh - 22) of this warp's columns, e = the block's
      // exponent (|x| < 2^e on the block); zero for an all-zero block
      // (converted lane-parallel into this warp's scratch, read back by
      // broadcast)
      const int* ei = reinterpret_cast<const int*>(sst + TC_DBYTES) + g * NCH + lane % NCH;
      float* xs = xscr[e];
      __syncwarp();  // the previous unit's reads of the scratch are done
      if (lane < 8 * NCH) xs[lane] = exp2i(ei[(lane / NCH) * NC] + sh_l - 22);
      if (8 * NCH > 32) xs[lane + 32] = exp2i(ei[((lane + 32) / NCH) * NC] + sh_l - 22);
      __syncwarp();
#pragma unroll
      for (int sl = 0; sl < C::NSL; ++sl) {
        // slot sl of the tile: MMA warp mw's ring slot hl % SLW, hl = SPW i + r
        const int mw = sl / C::SPW, r = sl % C::SPW;
        const uint32_t hl = (uint32_t)C::SPW * i + r, slot = hl % C::SLW;
        mbar_wait(saddr(&tfull[mw][slot]), (hl / C::SLW) & 1u, &abort_flag);
        __syncwarp();
        tc_fence_after();
        const uint32_t ta =
            tmem + ((uint32_t)(quarter * 32) << 16) + mw * C::REG + slot * C::BPS * C::NB + g * NCH;
        uint32_t v[C::BPS][3][NCH];
#pragma unroll
        for (int bb = 0; bb < C::BPS; ++bb)
#pragma unroll
          for (int pl = 0; pl < 3; ++pl)
            tmem_ld<NCH>(ta + (uint32_t)(bb * C::NB + pl * NC), v[bb][pl]);
        asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(saddr(&tempty[mw][slot]));
#pragma unroll
        for (int bb = 0; bb < C::BPS; ++bb) {
          const int b = sl * C::BPS + bb;
          const uint32_t dword = (b >> 1) == 0 ? d8.x : (b >> 1) == 1 ? d8.y : (b >> 1) == 2 ? d8.z : d8.w;
          const uint32_t dh = (b & 1) ? (dword >> 16) : (dword & 0xFFFFu);
          const float dv = __half2float(__ushort_as_half((unsigned short)dh));
#pragma unroll
          for (int c = 0; c < NCH; ++c) {
            const int lo = (int)(v[bb][0][c] + (v[bb][1][c] << 8));  // exact: |lo| < 2^28
            const float f = fmaf((float)(int)v[bb][2][c], 65536.0f, (float)lo);
            acc[c] = fmaf(f, dv * xs[b * NCH + c], acc[c]);
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(saddr(&sempty[j]));
      if (kt != p.nkt - 1 && i != nunits - 1) continue;
      // ---- end of this CTA's part of row tile rt
      const int64_t t0 = (int64_t)rt * p.nkt;
      const int r = rt * TC_M + row;
      if (u0 <= t0 && kt == p.nkt - 1) {  // the whole row tile is this CTA's
#pragma unroll
        for (int c = 0; c < NCH; ++c) {
          const int n = g * NCH + c;
          if (r < p.M && n < p.N) p.y[(int64_t)n * p.ldy + r] = finish(acc[c], shc[c], nfc[c]);
          acc[c] = 0.0f;
        }
        continue;
      }
      // a row tile shared with other CTAs: every warp stores its part (its
      // rows and columns) and counts it in the tile's counter for its warp
      // slot; the warp that stores the last such part adds them, in CTA order
      const int my_side = (u0 / p.nkt == rt) ? 0 : 1;  // the CTA's first or last row tile
#pragma unroll
      for (int c = 0; c < NCH; ++c) {
        part[(((int64_t)blockIdx.x * 2 + my_side) * NC + g * NCH + c) * TC_M + row] = acc[c];
        acc[c] = 0.0f;
      }
      __threadfence();
      __syncwarp();
      const int c0 = cta_of(t0, U, gridDim.x), c1 = cta_of(t0 + p.nkt - 1, U, gridDim.x);
      unsigned last = 0;
      if (lane == 0) last = atomicAdd(&cnt[rt * TC_EPI_MAX + e], 1u) == (unsigned)(c1 - c0);
      if (__shfl_sync(0xffffffffu, last, 0)) {
        __threadfence();
        float tot[NCH];
#pragma unroll
        for (int c = 0; c < NCH; ++c) tot[c] = 0.0f;
        for (int cc = c0; cc <= c1; ++cc) {
          const int side = (U * cc / gridDim.x) / p.nkt == rt ? 0 : 1;
          const float* src = part + (((int64_t)cc * 2 + side) * NC + g * NCH) * TC_M + row;
#pragma unroll
          for (int c = 0; c < NCH; ++c) tot[c] += __ldcg(src + c * TC_M);
        }
#pragma unroll
        for (int c = 0; c < NCH; ++c) {
          const int n = g * NCH + c;
          if (r < p.M && n < p.N) p.y[(int64_t)n * p.ldy + r] = finish(tot[c], shc[c], nfc[c]);
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) {
    __syncwarp();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(TC_TMEM_COLS)
                 : "memory");
  }
}

// ------------------------------------------------------------- x prep
// Grid (chunks, NC): CTA (c, col) handles blocks [c * chunk, (c + 1) * chunk)
// of column col (columns >= N get zeros), one block per warp at a time: the
// block's exponent e (|x| < 2^e on the block), the fixed-point digits of
// rint(x 2^(22 - e)) (written where the B operand reads them; a power-of-two
// normalisation of the column would not change them) and e itself.  The
// CTA's maximum |x| goes to the header, from which the GEMV derives the
// column's normalisation; no pass over the whole column.  CTA (0, 0) also
// clears the counters of the shared row tiles.
constexpr int XT_THREADS = 256;

// Blocks per prep CTA: one per warp while that keeps to TC_PMAX CTAs a column.
int xprep_chunk(int64_t K) {
  const int64_t nblk = (K + TC_KT - 1) / TC_KT * TC_BLK;
  const int64_t per = XT_THREADS / 32;
  const int64_t ctas = std::max<int64_t>(1, std::min<int64_t>(TC_PMAX, (nblk + per - 1) / per));
  return (int)((nblk + ctas - 1) / ctas);
}

template <int NC>
__global__ void __launch_bounds__(XT_THREADS) k_xprep_tc(const float* __restrict__ x, int64_t ldx,
                                                         int K, int N, int chunk, TcArgs p) {
  using C = TcCfg<NC>;
  // the GEMV may launch now and prefetch weights; it reads the workspace only
  // after its griddepcontrol.wait, i.e. after this grid has completed
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  __shared__ uint32_t red[XT_THREADS / 32];
  const int col = blockIdx.y, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const float* xc = x + (int64_t)col * ldx;
  const bool live = col < N;
  if (blockIdx.x == 0 && col == 0) {
    unsigned* cnt = reinterpret_cast<unsigned*>(p.ws + p.cnt_off);
    for (int t = threadIdx.x; t < p.ntiles * TC_EPI_MAX; t += XT_THREADS) cnt[t] = 0u;
  }
  const int nblk = p.nkt * TC_BLK;
  const int b0 = blockIdx.x * chunk, b1 = min(nblk, b0 + chunk);
  uint32_t cmax = 0u;  // max |x| of this warp's blocks, as bits (warp-uniform)
  bool bad = false;    // a NaN or an infinity among them
  for (int gb = b0 + warp; gb < b1; gb += XT_THREADS / 32) {
    const int kt = gb / TC_BLK, b = gb % TC_BLK;
    const int k = gb * QK + lane;
    const float xv = live && k < K ? xc[k] : 0.0f;
    uint32_t a = __float_as_uint(xv) & 0x7FFFFFFFu;
    const bool nonfinite = __any_sync(0xffffffffu, a >= 0x7F800000u);
    bad |= nonfinite;
    const float v = nonfinite ? 0.0f : xv;  // such a column's y is NaN anyway
    a = nonfinite ? 0u : a;
    for (int o = 16; o; o >>= 1) a = max(a, __shfl_xor_sync(0xffffffffu, a, o));
    cmax = max(cmax, a);
    int e = TC_EMPTY;
    if (a != 0u) frexpf(__uint_as_float(a), &e);  // block max = f 2^e, f in [0.5, 1)
    // X = rint(x 2^(22 - e)), |X| <= 2^22 (ldexpf scales exactly here)
    const int X = a == 0u ? 0 : __float2int_rn(ldexpf(v, 22 - e));
    const int p0 = (int)(signed char)(X & 0xFF);
    const int X1 = (X - p0) >> 8;
    const int p1 = (int)(signed char)(X1 & 0xFF);
    const int p2 = (X1 - p1) >> 8;
    uint8_t* xt = p.ws + p.xt_off + (size_t)kt * C::XT;
    const int kb = b * QK + lane;  // element inside the K tile
    const int box = kb >> 7, within = kb & 127, chk = within >> 4;
    const int pv[3] = {p0, p1, p2};
#pragma unroll
    for (int pl = 0; pl < 3; ++pl) {
      const int nrow = pl * NC + col;  // B row
      xt[box * C::BBOX + (nrow >> 3) * 1024 + (nrow & 7) * 128 + ((chk ^ (nrow & 7)) << 4) +
         (within & 15)] = (uint8_t)(signed char)pv[pl];
    }
    if (lane == 0) reinterpret_cast<int*>(xt + C::XB)[b * NC + col] = e;
  }
  if (lane == 0) red[warp] = bad ? 0xFFFFFFFFu : cmax;
  __syncthreads();
  if (threadIdx.x == 0) {
    uint32_t m = 0u;
    for (int w = 0; w < XT_THREADS / 32; ++w)
      m = (m == 0xFFFFFFFFu || red[w] == 0xFFFFFFFFu) ? 0xFFFFFFFFu : max(m, red[w]);
    reinterpret_cast<uint32_t*>(p.ws)[col * TC_PMAX + blockIdx.x] = m;
  }
}

// ------------------------------------------------------------ tc tiles
// One CTA per tile, from SoA planes or ggml blocks: q8_0 quants in 16-byte
// chunks at their swizzled A-layout positions, q4_0 blocks (16 bytes of
// nibbles) packed as [block][row]; then the [row][block] fp16 scales.
// Rows beyond M and blocks beyond K get zero quants and zero scales.
template <int FMT>
__global__ void __launch_bounds__(256) k_tile_tc(const uint8_t* __restrict__ q,
                                                 const unsigned short* __restrict__ d, bool aos,
                                                 int M, int K, int nkt, uint8_t* __restrict__ out) {
  constexpr int BLOCK = FMT == 8 ? Q8_BLOCK : Q4_BLOCK;  // ggml block bytes
  const int kt = blockIdx.x, rt = blockIdx.y;
  uint8_t* t = out + ((int64_t)rt * nkt + kt) * tc_tile<FMT>();
  const int nb = K / QK;
  const int64_t qrow = FMT == 8 ? K : K / 2;  // SoA quant bytes per row
  constexpr int CH = FMT == 8 ? TC_KT / 16 : TC_BLK;  // 16-byte chunks per tile row
  for (int i = threadIdx.x; i < TC_M * CH; i += blockDim.x) {
    // q8_0: consecutive threads read consecutive chunks of a row; q4_0: the
    // same block of consecutive rows (consecutive in the tile)
    const int r = FMT == 8 ? i / CH : i % TC_M, ch = FMT == 8 ? i % CH : i / TC_M;
    const int row = rt * TC_M + r;
    // chunk ch: q8_0 elements kt * 256 + 16 ch ...; q4_0 block kt * 8 + ch
    const int blk = FMT == 8 ? kt * TC_BLK + ch / 2 : kt * TC_BLK + ch;
    const int off = FMT == 8 ? (ch & 1) * 16 : 0;  // byte offset inside the block's quants
    uint4 v = make_uint4(0u, 0u, 0u, 0u);
    if (row < M && blk < nb) {
      if (!aos) {
        v = *reinterpret_cast<const uint4*>(q + (int64_t)row * qrow + (int64_t)blk * (FMT == 8 ? 32 : 16) + off);
      } else {
        const uint8_t* src = q + ((int64_t)row * nb + blk) * BLOCK + 2 + off;
        uint32_t w[4];
        for (int j = 0; j < 4; ++j)
          w[j] = (uint32_t)src[4 * j] | ((uint32_t)src[4 * j + 1] << 8) |
                 ((uint32_t)src[4 * j + 2] << 16) | ((uint32_t)src[4 * j + 3] << 24);
        v = make_uint4(w[0], w[1], w[2], w[3]);
      }
    }
    if (FMT == 8) {
      const int box = ch >> 3, c = ch & 7;
      *reinterpret_cast<uint4*>(t + box * TC_BOX + (r >> 3) * 1024 + (r & 7) * 128 +
                                ((c ^ (r & 7)) << 4)) = v;
    } else {
      *reinterpret_cast<uint4*>(t + (ch * TC_M + r) * 16) = v;
    }
  }
  unsigned short* ts = reinterpret_cast<unsigned short*>(t + tc_qbytes<FMT>());
  for (int i = threadIdx.x; i < TC_M * TC_BLK; i += blockDim.x) {
    const int r = i / TC_BLK, b = i % TC_BLK;
    const int row = rt * TC_M + r, blk = kt * TC_BLK + b;
    unsigned short h = 0;
    if (row < M && blk < nb) {
      if (!aos) {
        h = d[(int64_t)row * nb + blk];
      } else {
        const uint8_t* src = q + ((int64_t)row * nb + blk) * BLOCK;
        h = (unsigned short)(src[0] | (src[1] << 8));
      }
    }
    ts[i] = h;
  }
}

struct WsLayout {
  int cnt_off, part_off, xt_off;
  size_t bytes;
};

template <int NC>
WsLayout ws_layout(int64_t M, int64_t K, int grid) {
  const int64_t nkt = (K + TC_KT - 1) / TC_KT, ntiles = (M + TC_M - 1) / TC_M;
  WsLayout w;
  w.cnt_off = TC_HDR;
  w.part_off = w.cnt_off + (int)((ntiles * TC_EPI_MAX * 4 + 15) / 16 * 16);
  w.xt_off = w.part_off + grid * 2 * NC * TC_M * 4;
  w.bytes = (size_t)w.xt_off + (size_t)nkt * TcCfg<NC>::XT;
  return w;
}

int tc_grid(int64_t M, int64_t K, int sms) {
  const int64_t U = ((K + TC_KT - 1) / TC_KT) * ((M + TC_M - 1) / TC_M);
  return (int)std::max<int64_t>(1, std::min<int64_t>(sms, U));
}

// tiles != nullptr: tc tiles; else SoA planes q, d (K % 256 == 0, 16-byte
// aligned), streamed through 2-D tensor maps.
template <int FMT, int NC>
int launch_tc(const void* tiles, const void* q, const void* d, int64_t M, int64_t K,
              const float* x, int64_t ldx, float* y, int64_t ldy, int N, void* ws,
              size_t ws_bytes, const DeviceInfo& dev, cudaStream_t st) {
  using C = TcFmt<FMT, NC>;
  const int grid = tc_grid(M, K, dev.sms);
  const WsLayout w = ws_layout<NC>(M, K, grid);
  if (ws_bytes < w.bytes)
    return set_error(ERR_ARG, "this call needs a workspace of %zu bytes, got %zu", w.bytes, ws_bytes);
  static bool attr_done[64] = {};
  if (dev.device >= 0 && dev.device < 64 && !attr_done[dev.device]) {
    const cudaError_t e =
        cudaFuncSetAttribute(k_gemv_tc<FMT, NC>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)C::SMEM);
    if (e != cudaSuccess)
      return set_error(ERR_CUDA, "k_gemv_tc shared memory: %s", cudaGetErrorString(e));
    attr_done[dev.device] = true;
  }
  TcArgs a;
  memset(&a, 0, sizeof(a));
  a.soa = tiles == nullptr;
  if (a.soa) {
    const uint64_t qrow = FMT == 8 ? (uint64_t)K : (uint64_t)K / 2;
    if (int rc = encode_tensor_2d(&a.qmap, false, q, qrow, (uint64_t)M, qrow, 128, TC_M, true))
      return rc;
    if (int rc = encode_tensor_2d(&a.dmap, true, d, (uint64_t)(K / QK), (uint64_t)M,
                                  (uint64_t)(K / QK) * 2, TC_BLK, TC_M, false))
      return rc;
  }
  a.tiles = static_cast<const uint8_t*>(tiles);
  a.ws = static_cast<uint8_t*>(ws);
  a.y = y;
  a.ldy = ldy;
  a.M = (int)M;
  a.N = N;
  a.nkt = (int)((K + TC_KT - 1) / TC_KT);
  a.ntiles = (int)((M + TC_M - 1) / TC_M);
  a.cnt_off = w.cnt_off;
  a.part_off = w.part_off;
  a.xt_off = w.xt_off;

  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const int chunk = xprep_chunk(K);
  a.nchunk = (a.nkt * TC_BLK + chunk - 1) / chunk;
  cfg.gridDim = dim3(a.nchunk, NC);
  cfg.blockDim = dim3(XT_THREADS);
  cudaError_t e = cudaLaunchKernelEx(&cfg, k_xprep_tc<NC>, x, ldx, (int)K, N, chunk, a);
  if (e != cudaSuccess) return set_error(ERR_CUDA, "k_xprep_tc launch: %s", cudaGetErrorString(e));
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(C::THREADS);
  cfg.dynamicSmemBytes = C::SMEM;
  e = cudaLaunchKernelEx(&cfg, k_gemv_tc<FMT, NC>, a);
  if (e != cudaSuccess) return set_error(ERR_CUDA, "k_gemv_tc launch: %s", cudaGetErrorString(e));
  return check_launch("k_gemv_tc");
}

}  // namespace

size_t tc_tiles_bytes(int fmt, int64_t M, int64_t K) {
  const int64_t nkt = (K + TC_KT - 1) / TC_KT, ntiles = (M + TC_M - 1) / TC_M;
  return (size_t)(nkt * ntiles) * (fmt == 8 ? tc_tile<8>() : tc_tile<4>());
}

size_t tc_workspace_bytes(int64_t M, int64_t K, int sms) {
  return ws_layout<16>(M, K, tc_grid(M, K, sms)).bytes;
}

int tile_weights_tc(int fmt, bool aos, const void* q, const void* d, int64_t M, int64_t K,
                    void* out, cudaStream_t st) {
  const int nkt = (int)((K + TC_KT - 1) / TC_KT), ntiles = (int)((M + TC_M - 1) / TC_M);
  if (nkt == 0 || ntiles == 0) return OK;
  const uint8_t* qq = static_cast<const uint8_t*>(q);
  const unsigned short* dd = static_cast<const unsigned short*>(d);
  uint8_t* o = static_cast<uint8_t*>(out);
  if (fmt == 8)
    k_tile_tc<8><<<dim3(nkt, ntiles), 256, 0, st>>>(qq, dd, aos, (int)M, (int)K, nkt, o);
  else
    k_tile_tc<4><<<dim3(nkt, ntiles), 256, 0, st>>>(qq, dd, aos, (int)M, (int)K, nkt, o);
  return check_launch("k_tile_tc");
}

template <int FMT>
int gemv_tc_fmt(const void* tiles, const void* q, const void* d, int64_t M, int64_t K,
                const float* x, int64_t ldx, float* y, int64_t ldy, int N, void* ws,
                size_t ws_bytes, const DeviceInfo& dev, cudaStream_t st) {
  if (N <= 2) return launch_tc<FMT, 2>(tiles, q, d, M, K, x, ldx, y, ldy, N, ws, ws_bytes, dev, st);
  if (N <= 4) return launch_tc<FMT, 4>(tiles, q, d, M, K, x, ldx, y, ldy, N, ws, ws_bytes, dev, st);
  if (N <= 8) return launch_tc<FMT, 8>(tiles, q, d, M, K, x, ldx, y, ldy, N, ws, ws_bytes, dev, st);
  return launch_tc<FMT, 16>(tiles, q, d, M, K, x, ldx, y, ldy, N, ws, ws_bytes, dev, st);
}

int gemv_tc(int fmt, const void* tiles, int64_t M, int64_t K, const float* x, int64_t ldx,
            float* y, int64_t ldy, int N, void* ws, size_t ws_bytes, cudaStream_t st) {
  if (M == 0 || N == 0) return OK;
  DeviceInfo dev;
  if (int rc = current_device_info(dev)) return rc;
  if (fmt == 8)
    return gemv_tc_fmt<8>(tiles, nullptr, nullptr, M, K, x, ldx, y, ldy, N, ws, ws_bytes, dev, st);
  return gemv_tc_fmt<4>(tiles, nullptr, nullptr, M, K, x, ldx, y, ldy, N, ws, ws_bytes, dev, st);
}

size_t tc_soa_workspace_bytes(int64_t M, int64_t K, int N, int sms) {
  const int grid = tc_grid(M, K, sms);
  if (N <= 2) return ws_layout<2>(M, K, grid).bytes;
  if (N <= 4) return ws_layout<4>(M, K, grid).bytes;
  if (N <= 8) return ws_layout<8>(M, K, grid).bytes;
  return ws_layout<16>(M, K, grid).bytes;
}

int gemv_soa_tc(int fmt, const GemvCall& c, cudaStream_t st) {
  if (c.no_tc || c.N < 2 || c.N > 16 || c.K < 256 || c.K % 256 || c.K > (1 << 20) || c.M < 1 ||
      (reinterpret_cast<uintptr_t>(c.q) & 15) || (reinterpret_cast<uintptr_t>(c.d) & 15) ||
      !c.ws || (reinterpret_cast<uintptr_t>(c.ws) & 15))
    return -1;
  DeviceInfo dev;
  if (int rc = current_device_info(dev)) return rc;
  if (c.ws_bytes < tc_soa_workspace_bytes(c.M, c.K, c.N, dev.sms)) return -1;
  if (fmt == 8)
    return gemv_tc_fmt<8>(nullptr, c.q, c.d, c.M, c.K, c.x, c.ldx, c.y, c.ldy, c.N, c.ws,
                          c.ws_bytes, dev, st);
  return gemv_tc_fmt<4>(nullptr, c.q, c.d, c.M, c.K, c.x, c.ldx, c.y, c.ldy, c.N, c.ws,
                        c.ws_bytes, dev, st);
}

int set_tc_spin_limit(long long cycles) {
  const cudaError_t e = cudaMemcpyToSymbol(g_tc_spin_limit, &cycles, sizeof(cycles));
  if (e == cudaSuccess) return OK;
  return set_error(ERR_CUDA, "setting the wait limit: %s", cudaGetErrorString(e));
}

int read_tc_error(int clear, cudaStream_t st, int* out) {
  int v = 0;
  cudaError_t e = cudaMemcpyFromSymbolAsync(&v, g_tc_error, sizeof(int), 0, cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e != cudaSuccess)
    return set_error(ERR_CUDA, "reading the device error word: %s", cudaGetErrorString(e));
  if (clear && v) {
    const int zero = 0;
    e = cudaMemcpyToSymbolAsync(g_tc_error, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (e != cudaSuccess)
      return set_error(ERR_CUDA, "clearing the device error word: %s", cudaGetErrorString(e));
  }
  *out = v;
  return OK;
}

}  // namespace qg
