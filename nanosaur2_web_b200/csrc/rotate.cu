// ConvRot input rotation: ops.rotate (app/gpu/ops.js:38-45) with the hadamard kernel of
// app/gpu/kernels.js:379-407.  Every group of 256 consecutive features of a row is multiplied by the
// normalised regular Hadamard matrix H256 = (H4 x H4 x H4 x H4) / 16, H4 = [[1,1,1,-1],[1,1,-1,1],
// [1,-1,1,1],[-1,1,1,1]] (tools/quant.py:21-30), the rotation the int8 ConvRot weights were built for.
// H4 acts on one base-4 digit of the feature index; the four digits are independent, so the order in
// which they are applied does not change the product.
//
// One group per 16 threads, 16 features per thread.  A thread first holds features 16t .. 16t+15
// (digits 0 and 1 vary inside the thread) and applies H4 to those two digits in registers, then reads
// back features t, 16+t, .., 240+t through shared memory (digits 2 and 3 inside the thread) for the
// other two, and stores those: for each of its 16 values the group's 16 threads write 16 consecutive
// features.  HBM-bound: a row group is read once and written once.
#include "nsa_internal.h"

namespace nsa {

namespace {

constexpr int kRotGroups = 16;                 // groups per 256-thread block
constexpr int kRotStride = 256 + 16;           // floats per group in shared memory (see the reads)

// y = H4 x over four values (a b c e) = x[0..3] of one digit: y0 = a+b+c-e, y1 = a+b-c+e,
// y2 = a-b+c+e, y3 = -a+b+c+e (kernels.js:397-402).
__device__ __forceinline__ void h4(float& a, float& b, float& c, float& e) {
  const float s = a + b, t = c + e, u = a - b, w = c - e;
  const float y0 = s + w, y1 = s - w, y2 = u + t, y3 = t - u;
  a = y0;
  b = y1;
  c = y2;
  e = y3;
}

// Digits 0 (stride 1) and 1 (stride 4) of 16 values held in registers.
__device__ __forceinline__ void h4_two_digits(float (&v)[16]) {
#pragma unroll
  for (int q = 0; q < 4; ++q) h4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
#pragma unroll
  for (int q = 0; q < 4; ++q) h4(v[q], v[q + 4], v[q + 8], v[q + 12]);
}

// 16-byte chunk c of a group, swizzled so that both the contiguous (chunk 4t + j) and the strided
// (feature 16e + t) access patterns spread over the banks.
__device__ __forceinline__ int rot_chunk(int c) { return c ^ ((c >> 3) & 7); }

template <typename TIn, typename TOut>
__global__ void __launch_bounds__(256) rotate_kernel(RotateParams p) {
  __shared__ __align__(16) float s[kRotGroups * kRotStride];
  const int gl = threadIdx.x / 16, t = threadIdx.x % 16;
  const int gpr = p.cols / 256;                                  // groups per row
  const long long g = (long long)blockIdx.x * kRotGroups + gl;   // global group index
  const bool live = g < (long long)p.rows * gpr;
  const long long row = live ? g / gpr : 0;
  const int col0 = live ? (int)(g % gpr) * 256 : 0;
  float* sg = s + gl * kRotStride;
  float v[16];
  if (live) {
    const TIn* src = static_cast<const TIn*>(p.x) + row * p.ldx + col0 + 16 * t;
    if constexpr (sizeof(TIn) == 4) {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float4 f = reinterpret_cast<const float4*>(src)[j];
        v[4 * j] = f.x;
        v[4 * j + 1] = f.y;
        v[4 * j + 2] = f.z;
        v[4 * j + 3] = f.w;
      }
    } else {
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const uint4 w = reinterpret_cast<const uint4*>(src)[j];
        const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          v[8 * j + 2 * q] = __uint_as_float(ws[q] << 16);
          v[8 * j + 2 * q + 1] = __uint_as_float(ws[q] & 0xffff0000u);
        }
      }
    }
    h4_two_digits(v);
#pragma unroll
    for (int j = 0; j < 4; ++j)
      reinterpret_cast<float4*>(sg)[rot_chunk(4 * t + j)] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
  }
  __syncthreads();
  if (!live) return;
#pragma unroll
  for (int e = 0; e < 16; ++e) {
    const int f = 16 * e + t;
    v[e] = sg[rot_chunk(f >> 2) * 4 + (f & 3)];
  }
  h4_two_digits(v);
  TOut* dst = static_cast<TOut*>(p.y) + row * p.ldy + col0 + t;
#pragma unroll
  for (int e = 0; e < 16; ++e) {
    const float y = v[e] * 0.0625f;
    if constexpr (sizeof(TOut) == 4)
      dst[16 * e] = y;
    else
      dst[16 * e] = __float2bfloat16_rn(y);
  }
}

}  // namespace

cudaError_t launch_rotate(const RotateParams& p, cudaStream_t stream) {
  const long long groups = (long long)p.rows * (p.cols / 256);
  if (groups <= 0) return cudaSuccess;
  const long long blocks = (groups + kRotGroups - 1) / kRotGroups;
  if (blocks > 0x7FFFFFFFLL) return cudaErrorInvalidValue;
  const dim3 grid((unsigned)blocks);
  if (!p.in_bf16 && !p.out_bf16) rotate_kernel<float, float><<<grid, 256, 0, stream>>>(p);
  else if (!p.in_bf16) rotate_kernel<float, __nv_bfloat16><<<grid, 256, 0, stream>>>(p);
  else if (!p.out_bf16) rotate_kernel<__nv_bfloat16, float><<<grid, 256, 0, stream>>>(p);
  else rotate_kernel<__nv_bfloat16, __nv_bfloat16><<<grid, 256, 0, stream>>>(p);
  return cudaGetLastError();
}

}  // namespace nsa
