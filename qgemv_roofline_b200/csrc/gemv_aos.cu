// AoS (GGUF byte layout) q8_0 / q4_0 GEMV for sm_100a.
//
// Replaces the reference's AoS kernels qgemv_q8_v0/v1/v2 and qgemv_q4_v0/v1/v2
// (src/qgemv_kernels.cuh:39-104, 180-224, 294-320), which read 34- or 18-byte
// blocks with scalar loads.  Here the weights are read exactly as a GGUF
// tensor stores them, with no repack: a 34/18-byte block stride is not
// 16-byte aligned, so a warp first streams the bytes of 32 consecutive blocks
// of each of its R rows with 128-bit loads (from the 16-byte boundary at or
// below the first block) into a per-warp shared-memory slot, then every lane
// takes one whole block from there, realigns its quant words with byte
// permutes and runs the same exact arithmetic as the SoA kernel.
#include "gemv_core.cuh"
#include "qgemv_internal.h"

#include <algorithm>

namespace qg {
namespace {

constexpr int THREADS = 256;
constexpr int WARPS = THREADS / 32;

template <int FMT>
struct Aos {
  static constexpr int BS = Fmt<FMT>::BLOCK_BYTES;
  static constexpr int ROUND_BYTES = 32 * BS;                 // 32 blocks per round
  static constexpr int SLOT = ((ROUND_BYTES + 15) / 16 + 1) * 16;  // + alignment slack
  static constexpr int QWORDS = FMT == 8 ? 8 : 4;             // quant words per block
};

// Loads 16 bytes at global offset `off` (from base), or fewer when the chunk
// runs past `total` (the end of the weight buffer).
__device__ __forceinline__ uint4 load_chunk(const uint8_t* base, int64_t off, int64_t total) {
  if (off + 16 <= total) return ld_stream_v4(base + off);
  uint32_t b[4] = {0, 0, 0, 0};
  for (int i = 0; i < 16 && off + i < total; ++i)
    b[i >> 2] |= (uint32_t)base[off + i] << (8 * (i & 3));
  return make_uint4(b[0], b[1], b[2], b[3]);
}

template <int FMT, int NC, int R>
__global__ void __launch_bounds__(THREADS)
k_gemv_aos(const uint8_t* __restrict__ blocks, const float* __restrict__ x, int64_t ldx,
           float* __restrict__ y, int64_t ldy, int M, int K, int N, int KT) {
  using A = Aos<FMT>;
  extern __shared__ float4 smem_f4[];
  float* xs = reinterpret_cast<float*>(smem_f4);                      // [NC][KT]
  uint8_t* stage = reinterpret_cast<uint8_t*>(xs + (size_t)NC * KT);  // [WARPS][R][SLOT]
  float* accs = reinterpret_cast<float*>(stage + (size_t)WARPS * R * A::SLOT);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t GW = (int64_t)gridDim.x * WARPS;
  int row_begin, row_end, cta_row0, cta_row1, dummy;
  warp_rows(M, (int64_t)blockIdx.x * WARPS + warp, GW, row_begin, row_end);
  warp_rows(M, (int64_t)blockIdx.x * WARPS, GW, cta_row0, dummy);
  warp_rows(M, (int64_t)blockIdx.x * WARPS + WARPS - 1, GW, dummy, cta_row1);
  const int nkt = (K + KT - 1) / KT;
  const int nb = K / QK;
  const int64_t row_bytes = (int64_t)nb * A::BS;
  const int64_t total = (int64_t)M * row_bytes;
  uint8_t* my_stage = stage + (size_t)warp * R * A::SLOT;

  if (nkt > 1) {
    for (int i = threadIdx.x; i < (cta_row1 - cta_row0) * NC; i += THREADS) accs[i] = 0.0f;
  }

  for (int kt = 0; kt < nkt; ++kt) {
    const int k0 = kt * KT;
    const int kn = min(KT, K - k0);
    __syncthreads();
    stage_x<FMT, NC>(xs, x, ldx, N, k0, kn, KT);
    __syncthreads();

    const int tile_blocks = kn / QK;
    for (int r0 = row_begin; r0 < row_end; r0 += R) {
      float acc[R][NC];
#pragma unroll
      for (int r = 0; r < R; ++r)
#pragma unroll
        for (int n = 0; n < NC; ++n) acc[r][n] = 0.0f;

      for (int rb = 0; rb < tile_blocks; rb += 32) {
        const int nblk = min(32, tile_blocks - rb);
        const int b0 = k0 / QK + rb;  // first block of this round in the row
        int delta = 0;
        // Stream the round's bytes of each row into this warp's slots.
#pragma unroll
        for (int r = 0; r < R; ++r) {
          if (r0 + r < row_end) {
            const int64_t start = (int64_t)(r0 + r) * row_bytes + (int64_t)b0 * A::BS;
            const int64_t astart = start & ~(int64_t)15;
            delta = (int)(start - astart);
            const int nchunk = (delta + nblk * A::BS + 15) / 16;
            for (int ch = lane; ch < nchunk; ch += 32) {
              const uint4 v = load_chunk(blocks, astart + 16 * ch, total);
              *reinterpret_cast<uint4*>(my_stage + r * A::SLOT + 16 * ch) = v;
            }
          }
        }
        __syncwarp();
        // All rows of a warp share the alignment offset only if row_bytes is
        // a multiple of 16; recompute it per row.
        if (lane < nblk) {
          uint4 w[2][R];
          float dv[R];
#pragma unroll
          for (int r = 0; r < R; ++r) {
            const int64_t start = (int64_t)(min(r0 + r, row_end - 1)) * row_bytes +
                                  (int64_t)b0 * A::BS;
            const int off = (int)(start & 15) + lane * A::BS;  // even
            const uint32_t* src =
                reinterpret_cast<const uint32_t*>(my_stage + r * A::SLOT + (off & ~3));
            const bool odd = (off & 2) != 0;  // block starts mid-word
            const uint32_t sel = odd ? 0x7654u : 0x5432u;
            uint32_t wd[A::QWORDS + 1];
#pragma unroll
            for (int i = 0; i <= A::QWORDS; ++i) wd[i] = src[i];
            const uint32_t dbits = odd ? (wd[0] >> 16) : (wd[0] & 0xFFFFu);
            uint32_t qw[A::QWORDS];
            if (odd) {
#pragma unroll
              for (int i = 0; i < A::QWORDS; ++i) qw[i] = wd[i + 1];
            } else {
#pragma unroll
              for (int i = 0; i < A::QWORDS; ++i) qw[i] = __byte_perm(wd[i], wd[i + 1], sel);
            }
            const bool live = r0 + r < row_end;
            dv[r] = live ? half_bits_to_float((unsigned short)dbits) : 0.0f;
            w[0][r] = make_uint4(qw[0], qw[1], qw[2], qw[3]);
            if (FMT == 8) w[1][r] = make_uint4(qw[4 % A::QWORDS], qw[5 % A::QWORDS],
                                                qw[6 % A::QWORDS], qw[7 % A::QWORDS]);
          }
          const int xoff = (rb + lane) * QK;  // tile-relative element of this block
          float2 s2[R][NC];
#pragma unroll
          for (int r = 0; r < R; ++r)
#pragma unroll
            for (int n = 0; n < NC; ++n) s2[r][n] = make_float2(0.0f, 0.0f);
          dot_chunk<FMT, NC, R>(w[0], xs + xoff, KT, s2);
          if (FMT == 8) dot_chunk<FMT, NC, R>(w[1], xs + xoff + 16, KT, s2);
#pragma unroll
          for (int r = 0; r < R; ++r)
#pragma unroll
            for (int n = 0; n < NC; ++n)
              acc[r][n] = fmaf(dv[r], s2[r][n].x + s2[r][n].y, acc[r][n]);
        }
        __syncwarp();
        (void)delta;
      }

#pragma unroll
      for (int r = 0; r < R; ++r) {
#pragma unroll
        for (int n = 0; n < NC; ++n) {
          const float v = warp_sum(acc[r][n]);
          if (lane == 0 && r0 + r < row_end && n < N) {
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

template <int FMT, int NC, int R>
int launch_aos(const GemvCall& c, const DeviceInfo& dev, cudaStream_t st) {
  using A = Aos<FMT>;
  auto kern = k_gemv_aos<FMT, NC, R>;
  const int64_t budget = (int64_t)kXStageBytes / (4 * NC);
  const int KT = (int)std::min<int64_t>(c.K, budget - budget % QK);
  const int nkt = (int)((c.K + KT - 1) / KT);
  const int max_blocks_rows =
      (int)std::max<int64_t>(1, (c.M + (int64_t)WARPS * R - 1) / (WARPS * R));
  auto smem_for = [&](int grid) {
    size_t s = (size_t)NC * KT * 4 + (size_t)WARPS * R * A::SLOT;
    if (nkt > 1) s += ((size_t)((c.M + grid - 1) / grid) + 2) * NC * 4;
    return s;
  };
  if (int rc = allow_max_smem(reinterpret_cast<const void*>(kern), dev)) return rc;
  int occ = 0;
  if (int rc = occupancy(reinterpret_cast<const void*>(kern), dev, THREADS, smem_for(dev.sms), &occ))
    return rc;
  int grid = std::max(std::min(dev.sms * occ, max_blocks_rows), 1);
  if (c.grid_override > 0) grid = c.grid_override;
  const size_t smem = smem_for(grid);
  if (smem > (size_t)dev.smem_optin)
    return set_error(ERR_UNSUPPORTED,
                     "shared memory for this shape (%zu B) exceeds the device limit", smem);
  kern<<<grid, THREADS, smem, st>>>(static_cast<const uint8_t*>(c.q), c.x, c.ldx, c.y, c.ldy,
                                    (int)c.M, (int)c.K, c.N, KT);
  return check_launch("k_gemv_aos");
}

template <int FMT>
int dispatch_aos(const GemvCall& c, const DeviceInfo& dev, cudaStream_t st) {
  if (c.N <= 1) {
    const int rc = gemv_aos_tma(FMT, c, st);  // TMA-fed kernel when the shape allows
    if (rc != -1) return rc;
    return launch_aos<FMT, 1, 4>(c, dev, st);
  }
  if (c.N <= 2) return launch_aos<FMT, 2, 4>(c, dev, st);
  if (c.N <= 4) return launch_aos<FMT, 4, 2>(c, dev, st);
  if (c.N <= 8) return launch_aos<FMT, 8, 2>(c, dev, st);
  return launch_aos<FMT, 16, 1>(c, dev, st);
}

}  // namespace

int gemv_aos(int fmt, const GemvCall& c, cudaStream_t st) {
  DeviceInfo dev;
  int rc = current_device_info(dev);
  if (rc) return rc;
  GemvCall part = c;
  for (int n0 = 0; n0 < c.N; n0 += 16) {
    part.N = std::min(16, c.N - n0);
    part.x = c.x + (int64_t)n0 * c.ldx;
    part.y = c.y + (int64_t)n0 * c.ldy;
    rc = part.N == 2 ? gemv_tma_pair(fmt, true, part, st) : -1;
    if (rc == -1) rc = fmt == 8 ? dispatch_aos<8>(part, dev, st) : dispatch_aos<4>(part, dev, st);
    if (rc) return rc;
  }
  return OK;
}

}  // namespace qg
