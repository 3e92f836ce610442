// int8 weight slices (the reference's ConvRot "i8" GEMM operand, app/gpu/gemm.js:10, 119-130) turned
// into the bf16 operand layout of a tcgen05.mma in shared memory.
//
// The reference dequantises nothing: its GEMM reads each int8 weight as an exact small integer and
// multiplies the dot product by the row's scale in the epilogue (gemm.js:159).  Every integer in
// [-128, 127] is exact in bf16, so the converted slice carries the same values and the tensor core's
// fp32 accumulation of bf16 x int8-as-bf16 products sees what the reference's fp32 loop sees.
//
// Source: a TMA copy of W[n0 .. n0+rows)[k0 .. k0+64) int8 without swizzle (row n at n*64 bytes).
// Destination: the K-major 128-byte-swizzle layout the TMA would have written for a bf16 W slice
// (row n at n*128 bytes, its 16-byte chunk c at position c ^ (n & 7); 1024-byte aligned base).
#pragma once

#include "ptx.cuh"

namespace nsa {

// Four int8 in one word -> four bf16 (two bf16x2 words, element order kept).  Each byte b is biased
// to u = b + 128 and placed in the mantissa of 2^23 (the float 2^23 + u), and 2^23 + 128 is
// subtracted: exact integer arithmetic in fp32, then an exact conversion to bf16.
__device__ __forceinline__ void i8x4_to_bf16(uint32_t w, uint32_t& lo, uint32_t& hi) {
  const uint32_t u = w ^ 0x80808080u;
  const uint64_t bias = f2_pack(-8388736.0f, -8388736.0f);   // -(2^23 + 128)
  const uint64_t v01 = f2_add(f2_pack(__uint_as_float(__byte_perm(u, 0x4B000000u, 0x7440)),
                                      __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7441))), bias);
  const uint64_t v23 = f2_add(f2_pack(__uint_as_float(__byte_perm(u, 0x4B000000u, 0x7442)),
                                      __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7443))), bias);
  float a, b, c, d;
  f2_unpack(v01, a, b);
  f2_unpack(v23, c, d);
  lo = pack_bf16x2(a, b);
  hi = pack_bf16x2(c, d);
}

// Converts one [ROWS][64] int8 slice at src into the bf16 layout at dst with NT threads (thread t of
// the converting group), then makes the writes visible to the tensor core's async proxy.  Each thread
// moves 16-byte pieces: 16 int8 of one row (k 16j .. 16j+15) become that row's chunks 2j and 2j+1.
// A warp reads 512 contiguous bytes per step, and each quarter-warp's eight 16-byte stores land on
// eight distinct chunk positions (two rows of opposite parity), so neither side has bank conflicts.
template <int ROWS, int NT>
__device__ __forceinline__ void convert_i8_slice(const uint8_t* src, uint8_t* dst, int t) {
  static_assert((ROWS * 4) % NT == 0, "whole pieces per thread");
#pragma unroll 4
  for (int it = 0; it < ROWS * 4 / NT; ++it) {
    const int piece = it * NT + t;
    const int n = piece >> 2, j = piece & 3;
    const uint4 w = *reinterpret_cast<const uint4*>(src + n * 64 + j * 16);
    uint4 c0, c1;
    i8x4_to_bf16(w.x, c0.x, c0.y);
    i8x4_to_bf16(w.y, c0.z, c0.w);
    i8x4_to_bf16(w.z, c1.x, c1.y);
    i8x4_to_bf16(w.w, c1.z, c1.w);
    uint8_t* row = dst + n * 128;
    *reinterpret_cast<uint4*>(row + (((2 * j) ^ (n & 7)) << 4)) = c0;
    *reinterpret_cast<uint4*>(row + (((2 * j + 1) ^ (n & 7)) << 4)) = c1;
  }
  fence_proxy_async_smem();
}

}  // namespace nsa
