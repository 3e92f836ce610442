// LoRA side paths packed for nsa_linear's fused delta.
//
// The reference keeps each LoRA as fp32 A [r][K], B [n][r] with a scale (strength * alpha / r) and
// output columns [off, off + n) (app/lora.js:120-150), and ops.linear evaluates
// delta = sum_i scale_i B_i (A_i x) with two GEMMs per entry before adding it in the epilogue
// (app/gpu/ops.js:55-57, 70-86).  Here all entries become two bf16 matrices:
//   A_cat [R][K]: the entries' A rows stacked (rows past the ranks' sum are zero);
//   B_cat [N][R]: row n, columns of entry i = scale_i * B_i[n - off_i] / (alpha * rowScale[n]) for the
//                 entry's output columns, zero elsewhere,
// so that x A_cat^T is one small GEMM and the delta is R more K steps of the main GEMM, whose epilogue
// multiplies by alpha * rowScale[n] (rowScale = 1 for bf16 weights).  A strength change re-packs B_cat.
// Also here: the exact bf16 expansion of int8 weights that the projection's ConvRot form takes.
#include "nsa_internal.h"

namespace nsa {

namespace {

__global__ void lora_pack_a_kernel(const float* __restrict__ A, long long count, __nv_bfloat16* __restrict__ dst) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < count; i += (long long)gridDim.x * blockDim.x)
    dst[i] = __float2bfloat16_rn(A[i]);
}

__global__ void lora_pack_b_kernel(const float* __restrict__ B, int r, int off, int n, int R, int r0, float scale,
                                   float alpha, const float* __restrict__ w_scale, __nv_bfloat16* __restrict__ dst) {
  const long long count = (long long)n * r;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < count; i += (long long)gridDim.x * blockDim.x) {
    const int row = off + (int)(i / r), j = (int)(i % r);
    const float den = alpha * (w_scale ? w_scale[row] : 1.f);
    dst[(long long)row * R + r0 + j] = __float2bfloat16_rn(scale * B[i] / den);
  }
}

__global__ void expand_i8_kernel(const int8_t* __restrict__ w, long long count, __nv_bfloat16* __restrict__ out) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < count; i += (long long)gridDim.x * blockDim.x)
    out[i] = __float2bfloat16_rn((float)w[i]);   // exact: |w| <= 128
}

int blocks_for(long long count) {
  const long long b = (count + 255) / 256;
  const long long cap = (long long)device_sm_count() * 8;
  return (int)(b < 1 ? 1 : b > cap ? cap : b);
}

}  // namespace

cudaError_t launch_expand_i8(const int8_t* w, long long count, __nv_bfloat16* out, cudaStream_t stream) {
  if (count <= 0) return cudaSuccess;
  expand_i8_kernel<<<blocks_for(count), 256, 0, stream>>>(w, count, out);
  return cudaGetLastError();
}

cudaError_t launch_lora_pack(const LoraPackEntry* e, int count, int N, int K, int R, const float* w_scale, float alpha,
                             __nv_bfloat16* a_cat, __nv_bfloat16* b_cat, cudaStream_t stream) {
  cudaError_t err = cudaMemsetAsync(a_cat, 0, (size_t)R * K * 2, stream);
  if (err == cudaSuccess) err = cudaMemsetAsync(b_cat, 0, (size_t)N * R * 2, stream);
  if (err != cudaSuccess) return err;
  int r0 = 0;
  for (int i = 0; i < count; ++i) {
    const long long na = (long long)e[i].r * K, nb = (long long)e[i].n * e[i].r;
    lora_pack_a_kernel<<<blocks_for(na), 256, 0, stream>>>(e[i].A, na, a_cat + (long long)r0 * K);
    lora_pack_b_kernel<<<blocks_for(nb), 256, 0, stream>>>(e[i].B, e[i].r, e[i].off, e[i].n, R, r0, e[i].scale, alpha,
                                                           w_scale, b_cat);
    if ((err = cudaGetLastError()) != cudaSuccess) return err;
    r0 += e[i].r;
  }
  return cudaSuccess;
}

}  // namespace nsa
