// Row RMSNorm for sm_100a: ops.rmsnorm (app/gpu/ops.js:111-116, kernels.js:62-80)
//   Y[r][c] = X[r][c] * rsqrt(mean_c(X[r][c]^2) + eps) * w[c]
// and the Gemma layer's rmsnorm followed by ops.accumulate (app/models/gemma3.js:74-77, :86-88;
// ops.js:188-192) as one pass: Y[r][c] += X[r][c] * rsqrt(...) * w[c].  The product keeps the
// reference's order, (x * r) * w, so the only difference is the order of the sum of squares.
//
// One warp per row, eight rows per 256-thread block.  Rows of up to 640 fp32 values stay in
// registers (five 16-byte loads per lane, with the weights and, accumulating, Y requested in the same
// round trip); longer rows read the rest a second time (from L1).  The
// kernel is HBM-bound: X is read once, Y written once (and read once when accumulating); bf16 output
// feeds the next GEMM's A operand directly (the QKV projection of the Gemma layer).  The chained form
// (accumulate with a next weight) continues with the next norm of the updated rows, which the Gemma
// layer runs right after each accumulate (the pre-MLP norm, the next layer's input norm): the new Y
// values are still in registers, so Z = rmsnorm(Y) * w2 adds only its own write.
#include <cuda_bf16.h>

#include "nsa_internal.h"

namespace nsa {

namespace {

constexpr int kRmsWarps = 8;
constexpr int kRmsCache = 5;   // float4 per lane held in registers: a 640-wide row (Gemma's hidden size)

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// ss + x^2 + y^2 + z^2 + w^2 in a fixed order of fused multiply-adds (intrinsics: the compiler neither
// contracts nor reorders them), so that every pass over the same values gives the same sum.
__device__ __forceinline__ float sq4_acc(float ss, float4 v) {
  ss = __fmaf_rn(v.x, v.x, ss);
  ss = __fmaf_rn(v.y, v.y, ss);
  ss = __fmaf_rn(v.z, v.z, ss);
  return __fmaf_rn(v.w, v.w, ss);
}

// y = (x * r) * w for four values, then stored (bf16 / fp32) or added to `acc` (the prefetched Y).
template <bool BF16, bool ACC>
__device__ __forceinline__ void emit4(const RmsParams& p, int64_t row, int i, float4 v, float r, float4 w, float4 acc) {
  const float4 y = make_float4(v.x * r * w.x, v.y * r * w.y, v.z * r * w.z, v.w * r * w.w);
  if constexpr (BF16) {
    __nv_bfloat162 lo = __floats2bfloat162_rn(y.x, y.y), hi = __floats2bfloat162_rn(y.z, y.w);
    uint2 u;
    u.x = *reinterpret_cast<uint32_t*>(&lo);
    u.y = *reinterpret_cast<uint32_t*>(&hi);
    reinterpret_cast<uint2*>(static_cast<__nv_bfloat16*>(p.y) + row * p.ldy)[i] = u;
  } else {
    float4* dst = reinterpret_cast<float4*>(static_cast<float*>(p.y) + row * p.ldy) + i;
    if constexpr (ACC)
      *dst = make_float4(acc.x + y.x, acc.y + y.y, acc.z + y.z, acc.w + y.w);
    else
      *dst = y;
  }
}

template <bool BF16, bool ACC>
__device__ __forceinline__ void emit1(const RmsParams& p, int64_t row, int c, float v, float r) {
  const float y = v * r * p.w[c];
  if constexpr (BF16) {
    static_cast<__nv_bfloat16*>(p.y)[row * p.ldy + c] = __float2bfloat16_rn(y);
  } else {
    float* dst = static_cast<float*>(p.y) + row * p.ldy + c;
    if constexpr (ACC)
      *dst += y;
    else
      *dst = y;
  }
}

// z row = y * r2 * w2 for four values (the same product order as emit4), bf16 or fp32.
__device__ __forceinline__ void emit_z4(const RmsParams& p, int64_t row, int i, float4 y, float r2, float4 w) {
  const float4 z = make_float4(y.x * r2 * w.x, y.y * r2 * w.y, y.z * r2 * w.z, y.w * r2 * w.w);
  if (p.z_bf16) {
    __nv_bfloat162 lo = __floats2bfloat162_rn(z.x, z.y), hi = __floats2bfloat162_rn(z.z, z.w);
    uint2 u;
    u.x = *reinterpret_cast<uint32_t*>(&lo);
    u.y = *reinterpret_cast<uint32_t*>(&hi);
    reinterpret_cast<uint2*>(static_cast<__nv_bfloat16*>(p.z) + row * p.ldz)[i] = u;
  } else {
    reinterpret_cast<float4*>(static_cast<float*>(p.z) + row * p.ldz)[i] = z;
  }
}

__device__ __forceinline__ float4 add4(float4 a, float4 b) { return make_float4(a.x + b.x, a.y + b.y, a.z + b.z, a.w + b.w); }
__device__ __forceinline__ float4 norm4(float4 v, float r, float4 w) {
  return make_float4(v.x * r * w.x, v.y * r * w.y, v.z * r * w.z, v.w * r * w.w);
}

// VEC: cols, ldx and ldy multiples of 4 and X, w, Y 16-byte aligned (8-byte for bf16 Y rows).
// CHAIN (VEC, ACC, fp32 Y): then Z = rmsnorm(new Y) * w2, Z's rows 8-byte (bf16) / 16-byte aligned.
template <bool VEC, bool BF16, bool ACC, bool CHAIN>
__global__ void __launch_bounds__(kRmsWarps * 32) rmsnorm_kernel(const RmsParams p) {
  static_assert(!CHAIN || (VEC && ACC && !BF16), "the chained form follows the vector accumulate");
  const int lane = threadIdx.x % 32;
  const int64_t row = (int64_t)blockIdx.x * kRmsWarps + threadIdx.x / 32;
  if (row >= p.rows) return;
  const float* xr = p.x + row * p.ldx;
  float ss = 0.f;
  if constexpr (VEC) {
    // X, the weights and (accumulating) Y of the cached part are all requested before the reduction,
    // so a row costs one memory round trip instead of two
    const float4* x4 = reinterpret_cast<const float4*>(xr);
    const float4* w4 = reinterpret_cast<const float4*>(p.w);
    float4* y4 = ACC ? reinterpret_cast<float4*>(static_cast<float*>(p.y) + row * p.ldy) : nullptr;
    const int nv = p.cols / 4;
    const float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
    float4 v[kRmsCache], wv[kRmsCache], yv[ACC ? kRmsCache : 1];
#pragma unroll
    for (int j = 0; j < kRmsCache; ++j) {
      const int i = lane + 32 * j;
      const bool in = i < nv;
      v[j] = in ? __ldg(x4 + i) : z;
      wv[j] = in ? __ldg(w4 + i) : z;
      if constexpr (ACC) yv[j] = in ? y4[i] : z;
    }
#pragma unroll
    for (int j = 0; j < kRmsCache; ++j) ss = sq4_acc(ss, v[j]);
    for (int i = lane + 32 * kRmsCache; i < nv; i += 32) ss = sq4_acc(ss, __ldg(x4 + i));
    const float r = rsqrtf(warp_sum(ss) / (float)p.cols + p.eps);
    if constexpr (CHAIN) {
      // Y += norm(X), then the next norm over the new Y in the same order of sums as a separate pass
      float ss2 = 0.f;
#pragma unroll
      for (int j = 0; j < kRmsCache; ++j) {
        const int i = lane + 32 * j;
        if (i >= nv) continue;
        yv[j] = add4(yv[j], norm4(v[j], r, wv[j]));
        y4[i] = yv[j];
      }
#pragma unroll
      for (int j = 0; j < kRmsCache; ++j) ss2 = sq4_acc(ss2, lane + 32 * j < nv ? yv[j] : z);
      for (int i = lane + 32 * kRmsCache; i < nv; i += 32) {
        const float4 yn = add4(y4[i], norm4(__ldg(x4 + i), r, __ldg(w4 + i)));
        y4[i] = yn;
        ss2 = sq4_acc(ss2, yn);
      }
      const float r2 = rsqrtf(warp_sum(ss2) / (float)p.cols + p.eps);
      const float4* w24 = reinterpret_cast<const float4*>(p.w2);
#pragma unroll
      for (int j = 0; j < kRmsCache; ++j) {
        const int i = lane + 32 * j;
        if (i < nv) emit_z4(p, row, i, yv[j], r2, __ldg(w24 + i));
      }
      for (int i = lane + 32 * kRmsCache; i < nv; i += 32) emit_z4(p, row, i, y4[i], r2, __ldg(w24 + i));
    } else {
#pragma unroll
      for (int j = 0; j < kRmsCache; ++j) {
        const int i = lane + 32 * j;
        if (i >= nv) continue;
        if constexpr (ACC)
          emit4<BF16, ACC>(p, row, i, v[j], r, wv[j], yv[j]);
        else
          emit4<BF16, ACC>(p, row, i, v[j], r, wv[j], z);
      }
      for (int i = lane + 32 * kRmsCache; i < nv; i += 32) {
        if constexpr (ACC)
          emit4<BF16, ACC>(p, row, i, __ldg(x4 + i), r, __ldg(w4 + i), y4[i]);
        else
          emit4<BF16, ACC>(p, row, i, __ldg(x4 + i), r, __ldg(w4 + i), z);
      }
    }
  } else {
    for (int c = lane; c < p.cols; c += 32) {
      const float t = xr[c];
      ss += t * t;
    }
    const float r = rsqrtf(warp_sum(ss) / (float)p.cols + p.eps);
    for (int c = lane; c < p.cols; c += 32) emit1<BF16, ACC>(p, row, c, xr[c], r);
  }
}

template <bool VEC>
cudaError_t launch_v(const RmsParams& p, cudaStream_t stream) {
  const long long blocks = ((long long)p.rows + kRmsWarps - 1) / kRmsWarps;
  if (blocks > 0x7FFFFFFFLL) return cudaErrorInvalidValue;
  const dim3 grid((unsigned)blocks), block(kRmsWarps * 32);
  if (p.out_bf16)
    rmsnorm_kernel<VEC, true, false, false><<<grid, block, 0, stream>>>(p);
  else if (p.accumulate && VEC && p.w2)
    rmsnorm_kernel<VEC, false, true, VEC><<<grid, block, 0, stream>>>(p);
  else if (p.accumulate)
    rmsnorm_kernel<VEC, false, true, false><<<grid, block, 0, stream>>>(p);
  else
    rmsnorm_kernel<VEC, false, false, false><<<grid, block, 0, stream>>>(p);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_rmsnorm(const RmsParams& p, cudaStream_t stream) {
  if (p.rows <= 0) return cudaSuccess;
  return p.vec ? launch_v<true>(p, stream) : launch_v<false>(p, stream);
}

}  // namespace nsa
