// Bandwidth-bound kernels around the attention core:
//   * the prologue that turns packed q|k|v rows into head-major bf16 tiles, applying the per-head
//     RMSNorm and split-half RoPE of the DiT / Gemma q-k norm (app/gpu/kernels.js:311-342 semantics,
//     tools/reference.py:96-104,240-241) on the way, and zero-filling padded / masked rows;
//   * the in-place per-head norm (+RoPE) that mirrors ops.headNorm (app/gpu/ops.js:131-138);
//   * the RoPE table builders of app/models/common.js:15-43.
#include "nsa_internal.h"

namespace nsa {

namespace {

constexpr int kPrologueThreads = 256;
constexpr int kRowBufFloats = 4096;   // one row of up to 4096 head elements per pass

__device__ __forceinline__ float load_elem(const void* base, int64_t idx, int f32) {
  if (f32) return __ldg(reinterpret_cast<const float*>(base) + idx);
  return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(base)[idx]);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// grid: (max(Lq_pad, Lk_pad), B, 3 parts: q / k / v); one CTA handles one row of one part.
__global__ void __launch_bounds__(kPrologueThreads) prologue_kernel(const PrologueParams p) {
  __shared__ float buf[kRowBufFloats];
  __shared__ __align__(16) __nv_bfloat16 obuf[kRowBufFloats];

  const int row = blockIdx.x;
  const int bl = blockIdx.y;          // batch index within the shard
  const int b = p.b_begin + bl;       // global batch index
  const int part = blockIdx.z;
  const int pad = part == 0 ? p.Lq_pad : p.Lk_pad;
  if (row >= pad) return;

  const RowView& view = part == 0 ? p.q : (part == 1 ? p.k : p.v);
  const int H = part == 0 ? p.Hq : p.Hkv;
  const int h_begin = part == 0 ? p.hq_begin : p.hkv_begin;
  const int D = p.D;
  const float* w = part == 0 ? p.q_w : (part == 1 ? p.k_w : nullptr);
  int valid_rows;
  if (part == 0) {
    valid_rows = p.Lq;
  } else {
    valid_rows = p.kv_len ? min(p.kv_len[b], p.Lk) : p.Lk;
  }
  const bool valid = row < valid_rows;
  const bool rope = part < 2 && p.cs != nullptr && row < p.rope_rows;
  __nv_bfloat16* dst = part == 0 ? p.Qs : (part == 1 ? p.Ks : p.Vs);
  const int half = D / 2;
  const int heads_per_pass = kRowBufFloats / D;
  const int nwarps = blockDim.x / 32;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;

  for (int h0 = 0; h0 < H; h0 += heads_per_pass) {
    const int hn = min(heads_per_pass, H - h0);
    const int W = hn * D;
    if (valid) {
      const int64_t src0 = (int64_t)b * view.bstride + (int64_t)row * view.ld + view.off + (int64_t)(h_begin + h0) * D;
      for (int e = threadIdx.x; e < W; e += blockDim.x) buf[e] = load_elem(view.ptr, src0 + e, p.src_f32);
    }
    __syncthreads();
    for (int hh = warp; hh < hn; hh += nwarps) {
      const float* x = buf + hh * D;
      __nv_bfloat16* y = obuf + hh * D;
      if (!valid) {
        for (int i = lane; i < D; i += 32) y[i] = __float2bfloat16(0.f);
        continue;
      }
      float r = 1.f;
      if (w) {
        float ss = 0.f;
        for (int i = lane; i < D; i += 32) ss += x[i] * x[i];
        ss = warp_sum(ss);
        r = rsqrtf(ss / (float)D + p.eps);
      }
      for (int i = lane; i < half; i += 32) {
        float y1 = x[i], y2 = x[i + half];
        if (w) {
          y1 = y1 * r * w[i];
          y2 = y2 * r * w[i + half];
        }
        if (rope) {
          const float c = p.cs[(int64_t)row * half + i];
          const float s = p.cs[p.sin_off + (int64_t)row * half + i];
          const float t1 = y1 * c - y2 * s;
          const float t2 = y2 * c + y1 * s;
          y1 = t1;
          y2 = t2;
        }
        y[i] = __float2bfloat16(y1);
        y[i + half] = __float2bfloat16(y2);
      }
    }
    __syncthreads();
    // 16-byte stores: head hh occupies D contiguous bf16 of row `row` in its [pad][D] slab.
    const int chunks_per_head = D / 8;
    for (int c = threadIdx.x; c < hn * chunks_per_head; c += blockDim.x) {
      const int hh = c / chunks_per_head, sub = c % chunks_per_head;
      const int64_t slab = (int64_t)bl * H + h0 + hh;
      uint4* out = reinterpret_cast<uint4*>(dst + (slab * pad + row) * D + sub * 8);
      *out = *reinterpret_cast<const uint4*>(obuf + hh * D + sub * 8);
    }
    __syncthreads();
  }
}

// ops.headNorm: in place on X[(row_off + l) * ld + col_off + h * D + i]; one warp per (row, head).
template <typename T>
__global__ void head_norm_kernel(T* X, const float* w, int L, int H, int D, int64_t ld, int64_t col_off,
                                 int64_t row_off, const float* cs, int64_t sin_off, float eps) {
  const int gw = (blockIdx.x * blockDim.x + threadIdx.x) / 32;
  const int lane = threadIdx.x % 32;
  if (gw >= L * H) return;
  const int l = gw / H, h = gw % H;
  T* x = X + (row_off + l) * ld + col_off + (int64_t)h * D;
  const int half = D / 2;
  float ss = 0.f;
  for (int i = lane; i < D; i += 32) {
    const float v = static_cast<float>(x[i]);
    ss += v * v;
  }
  ss = warp_sum(ss);
  const float r = rsqrtf(ss / (float)D + eps);
  __syncwarp();
  for (int i = lane; i < half; i += 32) {
    float y1 = static_cast<float>(x[i]) * r * w[i];
    float y2 = static_cast<float>(x[i + half]) * r * w[i + half];
    if (cs) {
      const float c = cs[(int64_t)l * half + i];
      const float s = cs[sin_off + (int64_t)l * half + i];
      const float t1 = y1 * c - y2 * s;
      const float t2 = y2 * c + y1 * s;
      y1 = t1;
      y2 = t2;
    }
    x[i] = static_cast<T>(y1);
    x[i + half] = static_cast<T>(y2);
  }
}

// 1 / theta^(2i/dim) rounded to fp32 the way app/models/common.js:15 does (fp32 exponent, fp32 result).
__device__ __forceinline__ float inv_freq_f32(int i, int dim, double theta) {
  const float e = (float)((2.0 * i) / dim);
  return (float)(1.0 / pow(theta, (double)e));
}

__global__ void rope2d_table_kernel(int h, int w, int D, float* out) {
  const int half = D / 2, quarter = half / 2;
  const int L = h * w;
  const int idx = blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= L * half) return;
  const int l = idx / half, i = idx % half;
  const int y = l / w, x = l % w;
  const double cx = x - (w - 1) / 2.0, cy = y - (h - 1) / 2.0;
  const float f = inv_freq_f32(i % quarter, half, 10000.0);
  const float a = (float)((i < quarter ? cx : cy) * (double)f);
  out[idx] = (float)cos((double)a);
  out[(int64_t)L * half + idx] = (float)sin((double)a);
}

__global__ void rope1d_table_kernel(int L, int D, float theta, float* out) {
  const int half = D / 2;
  const int idx = blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= L * half) return;
  const int l = idx / half, i = idx % half;
  const float f = inv_freq_f32(i, D, (double)theta);
  const float a = (float)((double)l * (double)f);
  out[idx] = (float)cos((double)a);
  out[(int64_t)L * half + idx] = (float)sin((double)a);
}

}  // namespace

cudaError_t launch_prologue(const PrologueParams& p, cudaStream_t stream) {
  const int rows = p.Lq_pad > p.Lk_pad ? p.Lq_pad : p.Lk_pad;
  if (rows <= 0 || p.B <= 0) return cudaSuccess;
  dim3 grid(rows, p.B, 3);
  prologue_kernel<<<grid, kPrologueThreads, 0, stream>>>(p);
  return cudaGetLastError();
}

cudaError_t launch_head_norm(void* X, int f32, const float* w, int L, int H, int D, int64_t ld, int64_t col_off,
                             int64_t row_off, const float* cs, int64_t sin_off, float eps, cudaStream_t stream) {
  const int warps = L * H;
  if (warps <= 0) return cudaSuccess;
  const int threads = 256;
  const int blocks = (warps * 32 + threads - 1) / threads;
  if (f32)
    head_norm_kernel<float><<<blocks, threads, 0, stream>>>(static_cast<float*>(X), w, L, H, D, ld, col_off, row_off,
                                                            cs, sin_off, eps);
  else
    head_norm_kernel<__nv_bfloat16><<<blocks, threads, 0, stream>>>(static_cast<__nv_bfloat16*>(X), w, L, H, D, ld,
                                                                    col_off, row_off, cs, sin_off, eps);
  return cudaGetLastError();
}

cudaError_t launch_rope2d_table(int h, int w, int D, float* out, cudaStream_t stream) {
  const int n = h * w * (D / 2);
  if (n <= 0) return cudaSuccess;
  rope2d_table_kernel<<<(n + 255) / 256, 256, 0, stream>>>(h, w, D, out);
  return cudaGetLastError();
}

cudaError_t launch_rope1d_table(int L, int D, float theta, float* out, cudaStream_t stream) {
  const int n = L * (D / 2);
  if (n <= 0) return cudaSuccess;
  rope1d_table_kernel<<<(n + 255) / 256, 256, 0, stream>>>(L, D, theta, out);
  return cudaGetLastError();
}

}  // namespace nsa
