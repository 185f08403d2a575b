// Inner arithmetic shared by the SoA and AoS GEMV kernels.
//
// A "chunk" is 16 bytes of quants: 16 q8_0 weights (half a block) or 32 q4_0
// weights (one block).  Quants become floats without the int->float unit: the
// byte or nibble is OR-ed into the mantissa of 2^23 (0x4B000000), and one
// packed f32x2 add subtracts the bias exactly.  Products accumulate with
// packed f32x2 FMAs into two running sums per (row, column).
#pragma once

#include "qgemv_common.cuh"

namespace qg {

constexpr float B23 = 8388608.0f;

// q4_0: the kernel produces the 8 nibbles of a 32-bit word w in the order
// p = 0..7 = (byte0 lo, byte0 hi, byte1 lo, byte1 hi, ..., byte3 hi).  Nibble
// p is weight j = 4t + (p >> 1) + 16 * (p & 1) of the block (t = word index)
// and is extracted at bit offset q4_shift(p), i.e. carries a factor 2^shift.
__host__ __device__ constexpr int q4_shift(int p) {
  return p == 0 ? 0 : p == 1 ? 4 : p == 2 ? 8 : p == 3 ? 12 : p == 4 ? 16 : p == 5 ? 8
       : p == 6 ? 12 : 16;
}

template <int FMT>
struct Fmt;
template <>
struct Fmt<8> {
  static constexpr int ELEMS_PER_CHUNK = 16;
  static constexpr int ROW_DIV = 1;  // quant-row bytes = K / ROW_DIV
  static constexpr int BLOCK_BYTES = Q8_BLOCK;
};
template <>
struct Fmt<4> {
  static constexpr int ELEMS_PER_CHUNK = 32;
  static constexpr int ROW_DIV = 2;
  static constexpr int BLOCK_BYTES = Q4_BLOCK;
};

// Word of 4 int8 quants -> 4 exact floats (two packed pairs).
__device__ __forceinline__ void cvt_q8_word(uint32_t w, float2& a, float2& b) {
  const uint32_t v = w ^ 0x80808080u;  // int8 q -> unsigned q + 128
  a.x = __uint_as_float(__byte_perm(v, MAGIC_2P23, 0x7440));
  a.y = __uint_as_float(__byte_perm(v, MAGIC_2P23, 0x7441));
  b.x = __uint_as_float(__byte_perm(v, MAGIC_2P23, 0x7442));
  b.y = __uint_as_float(__byte_perm(v, MAGIC_2P23, 0x7443));
  const float2 c = make_float2(-(B23 + 128.0f), -(B23 + 128.0f));
  a = __fadd2_rn(a, c);
  b = __fadd2_rn(b, c);
}

// Word of 8 q4_0 nibbles -> 8 exact floats (n - 8) * 2^q4_shift(p).
__device__ __forceinline__ void cvt_q4_word(uint32_t w, float2 (&o)[4]) {
  const uint32_t v2 = w >> 12;
  o[0].x = __uint_as_float((w & 0x0000000Fu) | MAGIC_2P23);
  o[0].y = __uint_as_float((w & 0x000000F0u) | MAGIC_2P23);
  o[1].x = __uint_as_float((w & 0x00000F00u) | MAGIC_2P23);
  o[1].y = __uint_as_float((w & 0x0000F000u) | MAGIC_2P23);
  o[2].x = __uint_as_float((w & 0x000F0000u) | MAGIC_2P23);
  o[2].y = __uint_as_float((v2 & 0x00000F00u) | MAGIC_2P23);
  o[3].x = __uint_as_float((v2 & 0x0000F000u) | MAGIC_2P23);
  o[3].y = __uint_as_float((v2 & 0x000F0000u) | MAGIC_2P23);
  o[0] = __fadd2_rn(o[0], make_float2(-(B23 + 8.0f), -(B23 + 128.0f)));
  o[1] = __fadd2_rn(o[1], make_float2(-(B23 + 2048.0f), -(B23 + 32768.0f)));
  o[2] = __fadd2_rn(o[2], make_float2(-(B23 + 524288.0f), -(B23 + 2048.0f)));
  o[3] = __fadd2_rn(o[3], make_float2(-(B23 + 32768.0f), -(B23 + 524288.0f)));
}

// Where element e of a (32-aligned) K tile goes in the staged x tile, and the
// factor it is multiplied by on the way: natural order for q8_0; for q4_0 the
// nibble production order above, divided by 2^q4_shift(p) (exact).
template <int FMT>
__device__ __forceinline__ void stage_pos(int e, int& pos, float& scale) {
  if (FMT == 8) {
    pos = e;
    scale = 1.0f;
  } else {
    const int blk = e >> 5, j = e & 31;
    const int hi = j >> 4, jj = j & 15, t = jj >> 2, u = jj & 3;
    const int p = 2 * u + hi;
    pos = blk * 32 + 8 * t + p;
    scale = __int_as_float((127 - q4_shift(p)) << 23);  // 2^-shift
  }
}

// Stages columns [0, NC) of X[:, k0:k0+kn] into xs[n * KT + pos]; columns
// n >= N are zero.  Called by all threads of the CTA.
template <int FMT, int NC>
__device__ __forceinline__ void stage_x(float* xs, const float* __restrict__ x, int64_t ldx,
                                        int N, int k0, int kn, int KT) {
  for (int i = threadIdx.x; i < NC * kn; i += blockDim.x) {
    const int n = i / kn, e = i - n * kn;
    int pos;
    float sc;
    stage_pos<FMT>(e, pos, sc);
    xs[n * KT + pos] = n < N ? x[(int64_t)n * ldx + k0 + e] * sc : 0.0f;
  }
}

__device__ __forceinline__ uint32_t word_of(const uint4& v, int t) {
  return t == 0 ? v.x : t == 1 ? v.y : t == 2 ? v.z : v.w;
}

// s2[r][n] += chunk(w[r]) . xc[n]   (xc: staged x of this chunk, column stride KT)
template <int FMT, int NC, int R>
__device__ __forceinline__ void dot_chunk(const uint4 (&w)[R], const float* xc, int KT,
                                          float2 (&s2)[R][NC]) {
#pragma unroll
  for (int t = 0; t < 4; ++t) {
    if (FMT == 8) {
      float2 cv[R][2];
#pragma unroll
      for (int r = 0; r < R; ++r) cvt_q8_word(word_of(w[r], t), cv[r][0], cv[r][1]);
#pragma unroll
      for (int n = 0; n < NC; ++n) {
        const float4 xv = *reinterpret_cast<const float4*>(xc + n * KT + 4 * t);
        const float2 xa = make_float2(xv.x, xv.y), xb = make_float2(xv.z, xv.w);
#pragma unroll
        for (int r = 0; r < R; ++r) {
          s2[r][n] = __ffma2_rn(cv[r][0], xa, s2[r][n]);
          s2[r][n] = __ffma2_rn(cv[r][1], xb, s2[r][n]);
        }
      }
    } else {
      float2 cv[R][4];
#pragma unroll
      for (int r = 0; r < R; ++r) cvt_q4_word(word_of(w[r], t), cv[r]);
#pragma unroll
      for (int n = 0; n < NC; ++n) {
        const float4 xa = *reinterpret_cast<const float4*>(xc + n * KT + 8 * t);
        const float4 xb = *reinterpret_cast<const float4*>(xc + n * KT + 8 * t + 4);
#pragma unroll
        for (int r = 0; r < R; ++r) {
          s2[r][n] = __ffma2_rn(cv[r][0], make_float2(xa.x, xa.y), s2[r][n]);
          s2[r][n] = __ffma2_rn(cv[r][1], make_float2(xa.z, xa.w), s2[r][n]);
          s2[r][n] = __ffma2_rn(cv[r][2], make_float2(xb.x, xb.y), s2[r][n]);
          s2[r][n] = __ffma2_rn(cv[r][3], make_float2(xb.z, xb.w), s2[r][n]);
        }
      }
    }
  }
}

// Per-warp row range [begin, end) for global warp `gw` of `GW`: contiguous,
// sizes differ by at most one row.
__device__ __forceinline__ void warp_rows(int64_t M, int64_t gw, int64_t GW, int& begin,
                                          int& end) {
  begin = (int)(M * gw / GW);
  end = (int)(M * (gw + 1) / GW);
}

}  // namespace qg
