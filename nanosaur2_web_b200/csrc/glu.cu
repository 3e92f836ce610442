// Gated linear unit for sm_100a: ops.glu (app/gpu/ops.js:141-148, kernels.js:346-360)
//   Y[r][j] = act(X[r][j]) * X[r][I + j],  j < I
// over the [gate | up] halves of the gate_up linear's output.  act = SiLU (SwiGLU) or the tanh
// approximation of GELU (Gemma's MLP, app/models/gemma3.js:81; PyTorch's approximate="tanh",
// tools/reference.py:198): 0.5 x (1 + tanh(sqrt(2/pi) (x + 0.044715 x^3))).  X is fp32; Y is fp32
// or bf16 (the down projection's A operand).  HBM-bound: 8 bytes read per output.
#include <cuda_bf16.h>

#include "act.cuh"
#include "nsa_internal.h"

namespace nsa {

namespace {

constexpr int kGluThreads = 256;

// VEC: I, ldx, ldy multiples of 4; X 16-byte aligned, Y 16-byte (fp32) / 8-byte (bf16) aligned.
template <int ACT, bool BF16, bool VEC>
__global__ void __launch_bounds__(kGluThreads) glu_kernel(const GluParams p) {
  const int per_row = VEC ? p.I / 4 : p.I;
  const int64_t n = (int64_t)p.rows * per_row;
  for (int64_t i = (int64_t)blockIdx.x * kGluThreads + threadIdx.x; i < n; i += (int64_t)gridDim.x * kGluThreads) {
    const int64_t r = i / per_row;
    const int j = (int)(i - r * per_row);
    const float* xr = p.x + r * p.ldx;
    if constexpr (VEC) {
      const float4 g = __ldg(reinterpret_cast<const float4*>(xr) + j);
      const float4 u = __ldg(reinterpret_cast<const float4*>(xr + p.I) + j);
      const float4 y = make_float4(glu_act<ACT>(g.x) * u.x, glu_act<ACT>(g.y) * u.y, glu_act<ACT>(g.z) * u.z,
                                   glu_act<ACT>(g.w) * u.w);
      if constexpr (BF16) {
        __nv_bfloat162 lo = __floats2bfloat162_rn(y.x, y.y), hi = __floats2bfloat162_rn(y.z, y.w);
        uint2 o;
        o.x = *reinterpret_cast<uint32_t*>(&lo);
        o.y = *reinterpret_cast<uint32_t*>(&hi);
        reinterpret_cast<uint2*>(static_cast<__nv_bfloat16*>(p.y) + r * p.ldy)[j] = o;
      } else {
        reinterpret_cast<float4*>(static_cast<float*>(p.y) + r * p.ldy)[j] = y;
      }
    } else {
      const float y = glu_act<ACT>(xr[j]) * xr[p.I + j];
      if constexpr (BF16)
        static_cast<__nv_bfloat16*>(p.y)[r * p.ldy + j] = __float2bfloat16_rn(y);
      else
        static_cast<float*>(p.y)[r * p.ldy + j] = y;
    }
  }
}

template <int ACT, bool VEC>
void launch_a(const GluParams& p, dim3 grid, cudaStream_t stream) {
  if (p.out_bf16)
    glu_kernel<ACT, true, VEC><<<grid, kGluThreads, 0, stream>>>(p);
  else
    glu_kernel<ACT, false, VEC><<<grid, kGluThreads, 0, stream>>>(p);
}

// Row permutation of a gate_up weight (or its bias / row scales) for nsa_linear's fused GLU:
// destination row 256 t + j takes gate row 128 t + j for j < 128 and up row I + 128 t + (j - 128)
// otherwise, so that each 256-row tile of the linear holds 128 gate rows and their up rows.
// One 16-byte piece (or one 4-byte word when the rows are not 16-byte multiples) per thread.
template <typename T>
__global__ void __launch_bounds__(kGluThreads) glu_interleave_kernel(const uint8_t* __restrict__ src,
                                                                    uint8_t* __restrict__ dst, int I,
                                                                    int64_t row_bytes) {
  const int64_t per_row = row_bytes / (int64_t)sizeof(T);
  const int64_t n = 2 * (int64_t)I * per_row;
  for (int64_t i = (int64_t)blockIdx.x * kGluThreads + threadIdx.x; i < n; i += (int64_t)gridDim.x * kGluThreads) {
    const int64_t r = i / per_row, c = i - r * per_row;
    const int64_t t = r / 256, j = r % 256;
    const int64_t s = j < 128 ? 128 * t + j : I + 128 * t + (j - 128);
    reinterpret_cast<T*>(dst + r * row_bytes)[c] = reinterpret_cast<const T*>(src + s * row_bytes)[c];
  }
}

}  // namespace

cudaError_t launch_glu_interleave(const void* src, void* dst, int I, int64_t row_bytes, cudaStream_t stream) {
  if (I <= 0) return cudaSuccess;
  const bool vec = row_bytes % 16 == 0 && (reinterpret_cast<uintptr_t>(src) & 15) == 0 &&
                   (reinterpret_cast<uintptr_t>(dst) & 15) == 0;
  const int64_t n = 2 * (int64_t)I * (row_bytes / (vec ? 16 : 4));
  const int64_t want = (n + kGluThreads - 1) / kGluThreads;
  const int64_t cap = (int64_t)device_sm_count() * 8;
  const dim3 grid((unsigned)(want < cap ? want : cap));
  const uint8_t* s = static_cast<const uint8_t*>(src);
  uint8_t* d = static_cast<uint8_t*>(dst);
  if (vec)
    glu_interleave_kernel<uint4><<<grid, kGluThreads, 0, stream>>>(s, d, I, row_bytes);
  else
    glu_interleave_kernel<uint32_t><<<grid, kGluThreads, 0, stream>>>(s, d, I, row_bytes);
  return cudaGetLastError();
}

cudaError_t launch_glu(const GluParams& p, cudaStream_t stream) {
  if (p.rows <= 0) return cudaSuccess;
  const int sms = device_sm_count();
  const int64_t n = (int64_t)p.rows * (p.vec ? p.I / 4 : p.I);
  const int64_t want = (n + kGluThreads - 1) / kGluThreads;
  const dim3 grid((unsigned)(want < (int64_t)sms * 8 ? want : (int64_t)sms * 8));   // grid-stride beyond 8 waves
  if (p.act == 0)
    p.vec ? launch_a<0, true>(p, grid, stream) : launch_a<0, false>(p, grid, stream);
  else
    p.vec ? launch_a<1, true>(p, grid, stream) : launch_a<1, false>(p, grid, stream);
  return cudaGetLastError();
}

}  // namespace nsa
