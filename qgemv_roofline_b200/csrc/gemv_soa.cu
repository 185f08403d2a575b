// SoA q8_0 / q4_0 GEMV for sm_100a:  Y[n][r] = sum_k W[r][k] * X[n][k].
//
// Replaces the reference's best kernels, qgemv_q8_v5_soa_smem and
// qgemv_q4_v5_soa_smem (src/qgemv_kernels.cuh:264-291, 323-352), and their
// launches (src/bench.cu:416-419, 433-436), with one persistent design that
// also covers a small batch of N <= 16 activation vectors and any K % 32 == 0.
//
// Design (HBM-read bound: ~1.9 FLOP/B for q8_0, ~3.6 for q4_0):
//  * Persistent grid: (resident CTAs per SM) x (SM count).  Every warp owns a
//    contiguous range of rows, so the work per warp differs by at most one row.
//  * A warp processes R rows at once.  Lane l streams 16-byte chunks
//    l, l+32, ... of each row with 128-bit non-allocating loads, U chunks per
//    row in flight, so R*U*16 bytes per lane are outstanding.
//  * X is staged once per CTA in shared memory (whole K when it fits, else in
//    K tiles with per-row partial sums kept in shared memory).  The x values
//    of one chunk are read once and reused by the R rows.
//  * Quants become floats without the int->float unit (gemv_core.cuh); each
//    product equals q * x exactly, as in the reference.
//  * The block scale d multiplies the per-chunk partial sum (the reference's
//    order); partial dots reduce with warp shuffles.
#include "gemv_core.cuh"
#include "qgemv_internal.h"

#include <algorithm>

namespace qg {
namespace {

constexpr int THREADS = 256;
constexpr int WARPS = THREADS / 32;

template <int FMT, int NC, int R, int U>
__global__ void __launch_bounds__(THREADS)
k_gemv_soa(const uint8_t* __restrict__ q, const unsigned short* __restrict__ d,
           const float* __restrict__ x, int64_t ldx, float* __restrict__ y, int64_t ldy,
           int M, int K, int N, int KT) {
  using F = Fmt<FMT>;
  constexpr int EPC = F::ELEMS_PER_CHUNK;
  extern __shared__ float4 smem_f4[];
  float* xs = reinterpret_cast<float*>(smem_f4);  // [NC][KT]

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t GW = (int64_t)gridDim.x * WARPS;
  int row_begin, row_end, cta_row0, cta_row1, dummy;
  warp_rows(M, (int64_t)blockIdx.x * WARPS + warp, GW, row_begin, row_end);
  warp_rows(M, (int64_t)blockIdx.x * WARPS, GW, cta_row0, dummy);
  warp_rows(M, (int64_t)blockIdx.x * WARPS + WARPS - 1, GW, dummy, cta_row1);
  const int nkt = (K + KT - 1) / KT;
  float* accs = xs + (size_t)NC * KT;  // [cta rows][NC], only when nkt > 1

  const int64_t qrow = K / F::ROW_DIV;  // bytes per quant row
  const int nb = K / QK;                // scales per row

  if (nkt > 1) {
    for (int i = threadIdx.x; i < (cta_row1 - cta_row0) * NC; i += THREADS) accs[i] = 0.0f;
  }

  for (int kt = 0; kt < nkt; ++kt) {
    const int k0 = kt * KT;
    const int kn = min(KT, K - k0);
    __syncthreads();
    stage_x<FMT, NC>(xs, x, ldx, N, k0, kn, KT);
    __syncthreads();

    const int nch = kn / EPC;
    for (int r0 = row_begin; r0 < row_end; r0 += R) {
      float acc[R][NC];
#pragma unroll
      for (int r = 0; r < R; ++r)
#pragma unroll
        for (int n = 0; n < NC; ++n) acc[r][n] = 0.0f;

      const uint8_t* qp[R];
      const unsigned short* dp[R];
      bool rv[R];
#pragma unroll
      for (int r = 0; r < R; ++r) {
        rv[r] = r0 + r < row_end;
        const int rr = rv[r] ? r0 + r : r0;
        qp[r] = q + (int64_t)rr * qrow + k0 / F::ROW_DIV;
        dp[r] = d + (int64_t)rr * nb + k0 / QK;
      }

      for (int c0 = lane; c0 < nch; c0 += 32 * U) {
        uint4 w[U][R];
        float dv[U][R];
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const int c = c0 + 32 * u;
#pragma unroll
          for (int r = 0; r < R; ++r) {
            if (c < nch && rv[r]) {
              w[u][r] = ld_stream_v4(qp[r] + (int64_t)c * 16);
              dv[u][r] = half_bits_to_float(ld_stream_u16(dp[r] + (FMT == 8 ? (c >> 1) : c)));
            } else {
              w[u][r] = make_uint4(0, 0, 0, 0);
              dv[u][r] = 0.0f;
            }
          }
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const int c = c0 + 32 * u;
          if (c >= nch) break;
          float2 s2[R][NC];
#pragma unroll
          for (int r = 0; r < R; ++r)
#pragma unroll
            for (int n = 0; n < NC; ++n) s2[r][n] = make_float2(0.0f, 0.0f);
          dot_chunk<FMT, NC, R>(w[u], xs + c * EPC, KT, s2);
#pragma unroll
          for (int r = 0; r < R; ++r)
#pragma unroll
            for (int n = 0; n < NC; ++n)
              acc[r][n] = fmaf(dv[u][r], s2[r][n].x + s2[r][n].y, acc[r][n]);
        }
      }

#pragma unroll
      for (int r = 0; r < R; ++r) {
#pragma unroll
        for (int n = 0; n < NC; ++n) {
          const float v = warp_sum(acc[r][n]);
          if (lane == 0 && rv[r] && n < N) {
            if (nkt == 1) y[(int64_t)n * ldy + r0 + r] = v;
            else accs[(r0 + r - cta_row0) * NC + n] += v;
          }
        }
      }
    }
  }

  if (nkt > 1) {
    __syncthreads();
    const int rows = cta_row1 - cta_row0;
    for (int i = threadIdx.x; i < rows * NC; i += THREADS) {
      const int rr = i / NC, n = i - rr * NC;
      if (n < N) y[(int64_t)n * ldy + cta_row0 + rr] = accs[i];
    }
  }
}

template <int FMT, int NC, int R, int U>
int launch_soa(const GemvCall& c, const DeviceInfo& dev, cudaStream_t st) {
  auto kern = k_gemv_soa<FMT, NC, R, U>;
  // K tile: whole K when NC*K floats fit the staging budget, else the largest
  // multiple of 32 that does.
  const int64_t budget = (int64_t)kXStageBytes / (4 * NC);
  const int KT = (int)std::min<int64_t>(c.K, budget - budget % QK);
  const int nkt = (int)((c.K + KT - 1) / KT);
  const int max_blocks_rows =
      (int)std::max<int64_t>(1, (c.M + (int64_t)WARPS * R - 1) / (WARPS * R));
  // x tile, plus (with several K tiles) the partial sums of one CTA's rows.
  auto smem_for = [&](int grid) {
    size_t s = (size_t)NC * KT * 4;
    if (nkt > 1) s += ((size_t)((c.M + grid - 1) / grid) + 2) * NC * 4;
    return s;
  };
  if (int rc = allow_max_smem(reinterpret_cast<const void*>(kern), dev)) return rc;
  int occ = 0;
  if (int rc = occupancy(reinterpret_cast<const void*>(kern), dev, THREADS, smem_for(dev.sms), &occ))
    return rc;
  int grid = std::max(std::min(dev.sms * occ, max_blocks_rows), 1);
  if (c.grid_override > 0) grid = c.grid_override;
  const size_t smem = smem_for(grid);  // exact for the grid launched
  if (smem > (size_t)dev.smem_optin)
    return set_error(ERR_UNSUPPORTED,
                     "shared memory for this shape (%zu B) exceeds the device limit", smem);
  kern<<<grid, THREADS, smem, st>>>(static_cast<const uint8_t*>(c.q),
                                    static_cast<const unsigned short*>(c.d), c.x, c.ldx, c.y,
                                    c.ldy, (int)c.M, (int)c.K, c.N, KT);
  return check_launch("k_gemv_soa");
}

// Row blocking per batch width: fewer rows in flight per warp as the number
// of accumulators grows.
template <int FMT>
int dispatch_soa(const GemvCall& c, const DeviceInfo& dev, cudaStream_t st) {
  if (c.N <= 1) {
    const int rc = gemv_soa_tma(FMT, c, st);  // the TMA-fed kernel when the shape allows
    if (rc != -1) return rc;
    return FMT == 8 ? launch_soa<FMT, 1, 4, 1>(c, dev, st) : launch_soa<FMT, 1, 8, 1>(c, dev, st);
  }
  if (c.N <= 2) return launch_soa<FMT, 2, 4, 2>(c, dev, st);
  if (c.N <= 4) return launch_soa<FMT, 4, 2, 2>(c, dev, st);
  if (c.N <= 8) return launch_soa<FMT, 8, 2, 1>(c, dev, st);
  return launch_soa<FMT, 16, 1, 1>(c, dev, st);
}

// Single-column configurations selectable by index (rows per warp R, chunks
// in flight per row U), for the kernel ladder of the benchmark CLI.
struct Variant {
  const char* name;
  int r, u;
};
constexpr Variant kVariants[] = {
    {"soa_r1u4", 1, 4}, {"soa_r2u2", 2, 2}, {"soa_r2u4", 2, 4}, {"soa_r4u1", 4, 1},
    {"soa_r4u2", 4, 2}, {"soa_r4u4", 4, 4}, {"soa_r8u1", 8, 1}, {"soa_r8u2", 8, 2},
    {"soa_tma_dp4a", 0, 0}, {"soa_tma_f32", 0, 0}, {"soa_tma_dp4a_2cta_r4", 0, 0},
    {"soa_tma_dp4a_2cta_r2", 0, 0}, {"soa_tma_dp4a_2cta_r8", 0, 0},
};
constexpr int kNumVariants = sizeof(kVariants) / sizeof(kVariants[0]);

template <int FMT>
int launch_variant(int v, const GemvCall& c, const DeviceInfo& dev, cudaStream_t st) {
  switch (v) {
    case 0: return launch_soa<FMT, 1, 1, 4>(c, dev, st);
    case 1: return launch_soa<FMT, 1, 2, 2>(c, dev, st);
    case 2: return launch_soa<FMT, 1, 2, 4>(c, dev, st);
    case 3: return launch_soa<FMT, 1, 4, 1>(c, dev, st);
    case 4: return launch_soa<FMT, 1, 4, 2>(c, dev, st);
    case 5: return launch_soa<FMT, 1, 4, 4>(c, dev, st);
    case 6: return launch_soa<FMT, 1, 8, 1>(c, dev, st);
    case 7: return launch_soa<FMT, 1, 8, 2>(c, dev, st);
    default: {
      const int mode = v == 8 ? 1 : v == 9 ? 0 : v == 10 ? 2 : v == 11 ? 3 : 4;
      const int rc = gemv_soa_tma_mode(FMT, mode, c, st);
      return rc == -1 ? set_error(ERR_UNSUPPORTED, "shape not handled by the TMA kernel") : rc;
    }
  }
}

}  // namespace

int soa_variant_count() { return kNumVariants; }
const char* soa_variant_name(int v) {
  return (v >= 0 && v < kNumVariants) ? kVariants[v].name : nullptr;
}

int gemv_soa_variant(int fmt, int variant, const GemvCall& c, cudaStream_t st) {
  if (variant < 0 || variant >= kNumVariants)
    return set_error(ERR_ARG, "variant %d out of range [0, %d)", variant, kNumVariants);
  if (c.N != 1) return set_error(ERR_ARG, "variants are single-column kernels");
  DeviceInfo dev;
  if (int rc = current_device_info(dev)) return rc;
  return fmt == 8 ? launch_variant<8>(variant, c, dev, st) : launch_variant<4>(variant, c, dev, st);
}

int gemv_soa(int fmt, const GemvCall& c, cudaStream_t st) {
  DeviceInfo dev;
  int rc = current_device_info(dev);
  if (rc) return rc;
  // More than 16 columns are processed 16 at a time (the weights are re-read).
  GemvCall part = c;
  for (int n0 = 0; n0 < c.N; n0 += 16) {
    part.N = std::min(16, c.N - n0);
    part.x = c.x + (int64_t)n0 * c.ldx;
    part.y = c.y + (int64_t)n0 * c.ldy;
    rc = -1;
    if (part.N == 2) rc = gemv_tma_pair(fmt, false, part, st);  // q4_0: dp4a, weights once
    if (rc == -1 && part.N >= 2 && part.ws) rc = gemv_soa_tc(fmt, part, st);  // tcgen05 batch kernel
    if (rc == -1 && part.N >= 2 && part.ws) rc = gemv_soa_mma(fmt, part, st);  // mma.sync
    if (rc == -1) rc = fmt == 8 ? dispatch_soa<8>(part, dev, st) : dispatch_soa<4>(part, dev, st);
    if (rc) return rc;
  }
  return OK;
}

}  // namespace qg
