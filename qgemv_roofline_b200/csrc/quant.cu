// GPU quantizers, dequantizers and AoS<->SoA repack, bit-exact with the
// reference's python/qformats.py (and its C++ twin src/bench.cu:32-69):
//
//   q8_0: amax = max|w|; d = amax / 127 (IEEE fp32 division, round to nearest);
//         id = d > 0 ? 1/d : 0 (correctly rounded reciprocal);
//         q = clamp(rint(fp32(w * id)), -127, 127); d stored as fp16 (RNE).
//   q4_0: mx = signed w at the FIRST index of max|w|; d = mx / -8;
//         id = d != 0 ? 1/d : 0; q = clamp(trunc(fp32(fp32(w * id) + 8.5)), 0, 15)
//         (two separately rounded operations, never fused); byte i of the
//         block = q[i] | q[i+16] << 4.
//
// Every fp32 operation uses an explicitly rounded intrinsic, so the compiler
// cannot contract the multiply and add into one FMA.  One warp quantizes one
// 32-weight block (lane j holds weight j); a warp walks several blocks.
#include "qgemv_common.cuh"
#include "qgemv_internal.h"

#include <algorithm>

namespace qg {
namespace {

constexpr int THREADS = 256;

template <int FMT, bool AOS>
__global__ void __launch_bounds__(THREADS)
k_quantize(const float* __restrict__ w, int64_t ldw, int64_t M, int nb, int8_t* __restrict__ q,
           unsigned short* __restrict__ dq, uint8_t* __restrict__ aos) {
  const int lane = threadIdx.x & 31;
  const int64_t nblocks = M * nb;
  const int64_t gw = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t GW = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t blk = gw; blk < nblocks; blk += GW) {
    const int64_t r = blk / nb;
    const int b = (int)(blk - r * nb);
    const float v = w[r * ldw + (int64_t)b * QK + lane];
    const float a = fabsf(v);
    unsigned short dbits;
    uint32_t qv;  // this lane's quant (int8 as low byte for q8; nibble for q4)
    if (FMT == 8) {
      float amax = a;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
      const float d = __fdiv_rn(amax, 127.0f);
      const float id = d > 0.0f ? __frcp_rn(d) : 0.0f;
      float t = rintf(__fmul_rn(v, id));
      t = fminf(fmaxf(t, -127.0f), 127.0f);
      qv = (uint32_t)(uint8_t)(int8_t)(int)t;
      dbits = __half_as_ushort(__float2half_rn(d));
    } else {
      // first index of the largest magnitude
      float best = a;
      int bidx = lane;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float ob = __shfl_xor_sync(0xffffffffu, best, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bidx, o);
        if (ob > best || (ob == best && oi < bidx)) {
          best = ob;
          bidx = oi;
        }
      }
      const float mx = __shfl_sync(0xffffffffu, v, bidx);
      const float d = __fdiv_rn(mx, -8.0f);
      const float id = d != 0.0f ? __frcp_rn(d) : 0.0f;
      const float t = __fadd_rn(__fmul_rn(v, id), 8.5f);
      int qi = __float2int_rz(t);
      qi = min(max(qi, 0), 15);
      // lanes 0..15 pack (q[j], q[j+16])
      const int hi = __shfl_down_sync(0xffffffffu, qi, 16);
      qv = (uint32_t)(qi | (hi << 4));
      dbits = __half_as_ushort(__float2half_rn(d));
    }
    if (AOS) {
      constexpr int BS = FMT == 8 ? Q8_BLOCK : Q4_BLOCK;
      uint8_t* blkp = aos + blk * BS;
      if (lane == 0) {
        blkp[0] = (uint8_t)(dbits & 0xFF);
        blkp[1] = (uint8_t)(dbits >> 8);
      }
      if (FMT == 8 || lane < 16) blkp[2 + lane] = (uint8_t)qv;
    } else {
      if (lane == 0) dq[blk] = dbits;
      if (FMT == 8) q[r * (int64_t)nb * QK + (int64_t)b * QK + lane] = (int8_t)(uint8_t)qv;
      else if (lane < 16) reinterpret_cast<uint8_t*>(q)[r * (int64_t)nb * 16 + (int64_t)b * 16 + lane] = (uint8_t)qv;
    }
  }
}

// SoA planes -> fp32 weights (qformats.py:43-56).  One thread per weight.
template <int FMT>
__global__ void __launch_bounds__(THREADS)
k_dequant(const uint8_t* __restrict__ q, const unsigned short* __restrict__ dq,
          float* __restrict__ w, int64_t M, int64_t K) {
  const int64_t n = M * K;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / K, k = i - r * K;
    const float d = half_bits_to_float(dq[r * (K / QK) + k / QK]);
    float v;
    if (FMT == 8) {
      v = (float)(int8_t)q[i];
    } else {
      const int j = (int)(k & 31);
      const uint8_t p = q[r * (K / 2) + (k / QK) * 16 + (j & 15)];
      v = (float)((j < 16 ? (p & 0x0F) : (p >> 4))) - 8.0f;
    }
    w[i] = __fmul_rn(v, d);
  }
}

// AoS blocks <-> SoA planes (src/bench.cu:300-314).  One thread per block.
template <int FMT, bool TO_SOA>
__global__ void __launch_bounds__(THREADS)
k_repack(uint8_t* __restrict__ aos, uint8_t* __restrict__ q, unsigned short* __restrict__ dq,
         int64_t nblocks) {
  constexpr int BS = FMT == 8 ? Q8_BLOCK : Q4_BLOCK;
  constexpr int QB = BS - 2;
  for (int64_t b = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; b < nblocks;
       b += (int64_t)gridDim.x * blockDim.x) {
    uint8_t* blk = aos + b * BS;
    uint8_t* qb = q + b * QB;
    if (TO_SOA) {
      dq[b] = (unsigned short)(blk[0] | (blk[1] << 8));
#pragma unroll
      for (int i = 0; i < QB; ++i) qb[i] = blk[2 + i];
    } else {
      const unsigned short dv = dq[b];
      blk[0] = (uint8_t)(dv & 0xFF);
      blk[1] = (uint8_t)(dv >> 8);
#pragma unroll
      for (int i = 0; i < QB; ++i) blk[2 + i] = qb[i];
    }
  }
}

__global__ void k_fill_zero(float* __restrict__ y, int64_t M, int N, int64_t ldy) {
  const int64_t n = M * N;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t c = i / M, r = i - c * M;
    y[c * ldy + r] = 0.0f;
  }
}

int grid_for(int64_t work, int per_thread_items = 1) {
  DeviceInfo dev;
  current_device_info(dev);
  const int64_t want = (work / per_thread_items + THREADS - 1) / THREADS;
  return (int)std::max<int64_t>(1, std::min<int64_t>(want, (int64_t)dev.sms * 8));
}

}  // namespace

int quantize(int fmt, const float* w, int64_t M, int64_t K, int64_t ldw, void* q, void* d,
             void* aos, cudaStream_t st) {
  const int nb = (int)(K / QK);
  const int64_t nblocks = M * nb;
  const int grid = grid_for(nblocks * 32);
  if (aos) {
    if (fmt == 8)
      k_quantize<8, true><<<grid, THREADS, 0, st>>>(w, ldw, M, nb, nullptr, nullptr,
                                                    static_cast<uint8_t*>(aos));
    else
      k_quantize<4, true><<<grid, THREADS, 0, st>>>(w, ldw, M, nb, nullptr, nullptr,
                                                    static_cast<uint8_t*>(aos));
  } else {
    if (fmt == 8)
      k_quantize<8, false><<<grid, THREADS, 0, st>>>(w, ldw, M, nb, static_cast<int8_t*>(q),
                                                     static_cast<unsigned short*>(d), nullptr);
    else
      k_quantize<4, false><<<grid, THREADS, 0, st>>>(w, ldw, M, nb, static_cast<int8_t*>(q),
                                                     static_cast<unsigned short*>(d), nullptr);
  }
  return check_launch("k_quantize");
}

int dequant(int fmt, const void* q, const void* d, float* w, int64_t M, int64_t K,
            cudaStream_t st) {
  const int grid = grid_for(M * K, 4);
  if (fmt == 8)
    k_dequant<8><<<grid, THREADS, 0, st>>>(static_cast<const uint8_t*>(q),
                                           static_cast<const unsigned short*>(d), w, M, K);
  else
    k_dequant<4><<<grid, THREADS, 0, st>>>(static_cast<const uint8_t*>(q),
                                           static_cast<const unsigned short*>(d), w, M, K);
  return check_launch("k_dequant");
}

int repack(int fmt, int to_soa, const void* aos, void* q, void* d, int64_t M, int64_t K,
           cudaStream_t st) {
  const int64_t nblocks = M * (K / QK);
  const int grid = grid_for(nblocks);
  uint8_t* a = static_cast<uint8_t*>(const_cast<void*>(aos));
  uint8_t* qq = static_cast<uint8_t*>(q);
  unsigned short* dd = static_cast<unsigned short*>(d);
  if (fmt == 8) {
    if (to_soa) k_repack<8, true><<<grid, THREADS, 0, st>>>(a, qq, dd, nblocks);
    else k_repack<8, false><<<grid, THREADS, 0, st>>>(a, qq, dd, nblocks);
  } else {
    if (to_soa) k_repack<4, true><<<grid, THREADS, 0, st>>>(a, qq, dd, nblocks);
    else k_repack<4, false><<<grid, THREADS, 0, st>>>(a, qq, dd, nblocks);
  }
  return check_launch("k_repack");
}

int fill_zero_rows(float* y, int64_t M, int N, int64_t ldy, cudaStream_t st) {
  k_fill_zero<<<grid_for(M * N), THREADS, 0, st>>>(y, M, N, ldy);
  return check_launch("k_fill_zero");
}

}  // namespace qg
