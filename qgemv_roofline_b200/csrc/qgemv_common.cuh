// Shared definitions for the sm_100a q8_0 / q4_0 GEMV library.
//
// Formats (ggml, byte-identical; the reference declares the same two blocks in
// src/qgemv_kernels.cuh:21-26):
//   q8_0 block = fp16 d (little endian) + 32 x int8          = 34 bytes
//   q4_0 block = fp16 d (little endian) + 16 bytes of nibbles = 18 bytes,
//                byte i holds weight i (low nibble) and weight i+16 (high).
// The SoA form keeps the same values in two planes: quants [M][K] int8 (q8_0)
// or [M][K/2] uint8 (q4_0), and scales [M][K/32] fp16.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace qg {

constexpr int QK = 32;
constexpr int Q8_BLOCK = 34;
constexpr int Q4_BLOCK = 18;

// Status codes shared with include/qgemv_b200.h.
enum Status : int {
  OK = 0,
  ERR_NULL = 1,
  ERR_SHAPE = 2,
  ERR_ALIGN = 3,
  ERR_CUDA = 4,
  ERR_UNSUPPORTED = 5,
  ERR_TIMEOUT = 6,
  ERR_ARG = 7,
};

// Records a message for qgemv_last_error() (thread-local) and returns `code`.
int set_error(int code, const char* fmt, ...);
int check_launch(const char* what);  // cudaGetLastError() -> ERR_CUDA + message

// ------------------------------------------------------------- device helpers

// 128-bit streaming load: read-only path, no L1 allocation (each weight byte
// is used once), 256-byte L2 prefetch so a warp's 512-byte row segment turns
// into full DRAM bursts.
__device__ __forceinline__ uint4 ld_stream_v4(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.L2::256B.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

__device__ __forceinline__ uint2 ld_stream_v2(const void* p) {
  uint2 v;
  asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];"
               : "=r"(v.x), "=r"(v.y)
               : "l"(p));
  return v;
}

__device__ __forceinline__ unsigned short ld_stream_u16(const void* p) {
  unsigned short v;
  asm volatile("ld.global.nc.L1::no_allocate.u16 %0, [%1];" : "=h"(v) : "l"(p));
  return v;
}

__device__ __forceinline__ float half_bits_to_float(unsigned short h) {
  return __half2float(__ushort_as_half(h));
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Exact small-integer -> fp32 conversion without the integer-to-float unit.
// An unsigned value u < 2^23 placed in the mantissa of 2^23 (exponent field
// 0x4B) is the float 2^23 + u; subtracting a constant then yields the integer
// exactly.  This is the IEEE-754 identity used e.g. by Kim et al. 2022 ("Who
// Says Elephants Can't Run?") for int4/int8 dequantization.
constexpr uint32_t MAGIC_2P23 = 0x4B000000u;  // bit pattern of 8388608.0f

}  // namespace qg
