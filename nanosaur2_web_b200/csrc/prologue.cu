// Bandwidth-bound kernels around the attention core:
//   * the prologue that turns packed q|k|v rows into head-major bf16 tiles, applying the per-head
//     RMSNorm and split-half RoPE of the DiT / Gemma q-k norm (app/gpu/kernels.js:311-342 semantics,
//     tools/reference.py:96-104,240-241) on the way, and zero-filling padded / masked rows;
//   * the in-place per-head norm (+RoPE) that mirrors ops.headNorm (app/gpu/ops.js:131-138);
//   * the RoPE table builders of app/models/common.js:15-43.
#include <algorithm>
#include <numeric>

#include "nsa_internal.h"
#include "ptx.cuh"

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
  if (blockIdx.x == 0 && blockIdx.y == 0 && blockIdx.z == 0)
    for (int i = threadIdx.x; i < p.zero_count; i += blockDim.x) p.zero_ptr[i] = 0;

  const int r_out = blockIdx.x;       // produced row
  const int bl = blockIdx.y;          // batch index within the shard
  const int b = p.b_begin + bl;       // global batch index
  const int part = blockIdx.z + (p.skip_q ? 1 : 0);
  const int pad = p.rows[part];
  if (r_out >= pad) return;
  const int row = p.row0[part] + r_out;   // source row, key / query index and RoPE row

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
  const TileOut& dst = p.out[part];
  if (part == 2 && p.v_tile > 0 && row < valid_rows / p.v_tile * p.v_tile) return;   // read from the input
  const int half = D / 2;
  const int heads_per_pass = kRowBufFloats / D;
  const int nwarps = blockDim.x / 32;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;

  for (int h0 = 0; h0 < H; h0 += heads_per_pass) {
    const int hn = min(heads_per_pass, H - h0);
    const int W = hn * D;
    if (valid) {
      const int64_t src0 = (int64_t)b * view.bstride + (int64_t)(p.src_row0[part] + r_out) * view.ld + view.off +
                           (int64_t)(h_begin + h0) * D;
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
      float* yf = p.out_f32 ? reinterpret_cast<float*>(dst.ptr) + (int64_t)bl * dst.bs + (int64_t)(h0 + hh) * dst.hs +
                                  (int64_t)r_out * dst.rs
                            : nullptr;
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
        if (yf) {   // fp32 tiles (the tf32 path), rounded to tf32: written straight from the lanes, coalesced
          yf[i] = round_tf32(y1);
          yf[i + half] = round_tf32(y2);
        } else {
          y[i] = __float2bfloat16(y1);
          y[i + half] = __float2bfloat16(y2);
        }
      }
    }
    __syncthreads();
    if (p.out_f32) {
      if (!valid) {   // zero rows (padding, masked keys) as fp32
        for (int e = threadIdx.x; e < hn * D; e += blockDim.x) {
          const int hh = e / D, d = e % D;
          reinterpret_cast<float*>(dst.ptr)[(int64_t)bl * dst.bs + (int64_t)(h0 + hh) * dst.hs + (int64_t)r_out * dst.rs + d] = 0.f;
        }
      }
      __syncthreads();
      continue;
    }
    // 16-byte stores: head hh of the produced row occupies D contiguous bf16 at its destination.
    const int chunks_per_head = D / 8;
    for (int c = threadIdx.x; c < hn * chunks_per_head; c += blockDim.x) {
      const int hh = c / chunks_per_head, sub = c % chunks_per_head;
      uint4* out = reinterpret_cast<uint4*>(dst.ptr + (int64_t)bl * dst.bs + (int64_t)(h0 + hh) * dst.hs +
                                            (int64_t)r_out * dst.rs + sub * 8);
      const uint4 val = *reinterpret_cast<const uint4*>(obuf + hh * D + sub * 8);
      *out = val;
      if (part > 0)
        for (int i = 0; i < p.n_peers; ++i) *reinterpret_cast<uint4*>(reinterpret_cast<uint8_t*>(out) + p.peer_off[i]) = val;
    }
    __syncthreads();
  }
  if (part > 0 && p.n_peers > 0) __threadfence_system();   // peer stores visible before any later signal
}

// Vectorised prologue for aligned layouts.  Each head of a row is handled by P consecutive threads;
// thread `sub` owns elements [sub*S, sub*S + S) of both halves of the head (S = D / (2P)), so the
// RoPE pair (i, i + D/2) stays in one thread, every load and store is a 16-byte vector, and the
// RMSNorm sum is a P-lane shuffle reduction.  grid.y = part * B + batch element.
template <int D, int P, typename T>
#ifndef NSA_PROLOGUE_MIN_BLOCKS
#define NSA_PROLOGUE_MIN_BLOCKS 3
#endif
__global__ void __launch_bounds__(256, NSA_PROLOGUE_MIN_BLOCKS) prologue_vec_kernel(const PrologueParams p) {
  constexpr int S = D / (2 * P);
  constexpr int HALF = D / 2;
  constexpr int EPV = 16 / sizeof(T);   // input elements per 16-byte vector
  static_assert(S % 8 == 0 && S % EPV == 0, "vector width");
  if (blockIdx.x == 0 && blockIdx.y == 0)
    for (int i = threadIdx.x; i < p.zero_count; i += blockDim.x) p.zero_ptr[i] = 0;
  const int part = blockIdx.y / p.B + (p.skip_q ? 1 : 0);
  const int bl = blockIdx.y % p.B;
  const int b = p.b_begin + bl;
  const int H = part == 0 ? p.Hq : p.Hkv;
  const int pad = p.rows[part];
  const long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  const int sub = (int)(idx % P);
  const long long rest = idx / P;
  const int hh = (int)(rest % H);
  const long long row_ll = rest / H;
  // Threads past the last row stay until after the shuffle below (all lanes of a warp take part).
  const bool in_range = row_ll < pad;
  const int r_out = in_range ? (int)row_ll : 0;
  const int row = p.row0[part] + r_out;   // source row, key / query index and RoPE row
  const RowView& view = part == 0 ? p.q : (part == 1 ? p.k : p.v);
  const int h_begin = part == 0 ? p.hq_begin : p.hkv_begin;
  const float* w = part == 0 ? p.q_w : (part == 1 ? p.k_w : nullptr);
  const int valid_rows = part == 0 ? p.Lq : (p.kv_len ? min(p.kv_len[b], p.Lk) : p.Lk);
  const bool valid = in_range && row < valid_rows;
  const bool rope = part < 2 && p.cs != nullptr && row < p.rope_rows;
  // V rows of key tiles the attention kernel reads straight from the input: nothing to read or
  // write (V has no norm, so no lane of such a row takes part in a shuffle below)
  if (part == 2 && p.v_tile > 0 && row < valid_rows / p.v_tile * p.v_tile) return;

  float x1[S], x2[S];
#pragma unroll
  for (int i = 0; i < S; ++i) x1[i] = x2[i] = 0.f;
  if (valid) {
    const T* src = reinterpret_cast<const T*>(view.ptr) + (int64_t)b * view.bstride +
                   (int64_t)(p.src_row0[part] + r_out) * view.ld + view.off + (int64_t)(h_begin + hh) * D + sub * S;
#pragma unroll
    for (int v = 0; v < S / EPV; ++v) {
      const uint4 a = __ldg(reinterpret_cast<const uint4*>(src) + v);
      const uint4 c = __ldg(reinterpret_cast<const uint4*>(src + HALF) + v);
      if constexpr (sizeof(T) == 2) {
        const __nv_bfloat162* pa = reinterpret_cast<const __nv_bfloat162*>(&a);
        const __nv_bfloat162* pc = reinterpret_cast<const __nv_bfloat162*>(&c);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 fa = __bfloat1622float2(pa[e]);
          const float2 fc = __bfloat1622float2(pc[e]);
          x1[v * 8 + 2 * e] = fa.x;
          x1[v * 8 + 2 * e + 1] = fa.y;
          x2[v * 8 + 2 * e] = fc.x;
          x2[v * 8 + 2 * e + 1] = fc.y;
        }
      } else {
        const float* fa = reinterpret_cast<const float*>(&a);
        const float* fc = reinterpret_cast<const float*>(&c);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          x1[v * 4 + e] = fa[e];
          x2[v * 4 + e] = fc[e];
        }
      }
    }
  }
  // w is uniform over the block (one part per blockIdx.y), so every lane reaches the shuffle.
  float r = 1.f;
  if (w) {
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < S; ++i) ss += x1[i] * x1[i] + x2[i] * x2[i];
#pragma unroll
    for (int o = 1; o < P; o <<= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    r = rsqrtf(ss / (float)D + p.eps);
  }
  if (!in_range) return;
  if (valid) {
    if (w) {
      const float4* w1 = reinterpret_cast<const float4*>(w + sub * S);
      const float4* w2 = reinterpret_cast<const float4*>(w + HALF + sub * S);
#pragma unroll
      for (int v = 0; v < S / 4; ++v) {
        const float4 a = __ldg(w1 + v), c = __ldg(w2 + v);
        x1[4 * v] *= r * a.x; x1[4 * v + 1] *= r * a.y; x1[4 * v + 2] *= r * a.z; x1[4 * v + 3] *= r * a.w;
        x2[4 * v] *= r * c.x; x2[4 * v + 1] *= r * c.y; x2[4 * v + 2] *= r * c.z; x2[4 * v + 3] *= r * c.w;
      }
    }
    if (rope) {
      const float4* cp = reinterpret_cast<const float4*>(p.cs + (int64_t)row * HALF + sub * S);
      const float4* sp = reinterpret_cast<const float4*>(p.cs + p.sin_off + (int64_t)row * HALF + sub * S);
#pragma unroll
      for (int v = 0; v < S / 4; ++v) {
        const float4 c4 = __ldg(cp + v), s4 = __ldg(sp + v);
        const float cc[4] = {c4.x, c4.y, c4.z, c4.w}, sn[4] = {s4.x, s4.y, s4.z, s4.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float a = x1[4 * v + e], c = x2[4 * v + e];
          x1[4 * v + e] = a * cc[e] - c * sn[e];
          x2[4 * v + e] = c * cc[e] + a * sn[e];
        }
      }
    }
  }
  // From here each thread writes its own chunk.
  const TileOut& to = p.out[part];
  __nv_bfloat16* dst = to.ptr + (int64_t)bl * to.bs + (int64_t)hh * to.hs + (int64_t)r_out * to.rs + sub * S;
#pragma unroll
  for (int v = 0; v < S / 8; ++v) {
    uint4 o1, o2;
    uint32_t* u1 = reinterpret_cast<uint32_t*>(&o1);
    uint32_t* u2 = reinterpret_cast<uint32_t*>(&o2);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      __nv_bfloat162 t1 = __floats2bfloat162_rn(x1[v * 8 + 2 * e], x1[v * 8 + 2 * e + 1]);
      __nv_bfloat162 t2 = __floats2bfloat162_rn(x2[v * 8 + 2 * e], x2[v * 8 + 2 * e + 1]);
      u1[e] = *reinterpret_cast<uint32_t*>(&t1);
      u2[e] = *reinterpret_cast<uint32_t*>(&t2);
    }
    reinterpret_cast<uint4*>(dst)[v] = o1;
    reinterpret_cast<uint4*>(dst + HALF)[v] = o2;
    if (part > 0) {
      // the same k / v rows into the other GPUs' buffers (NVLink stores through their mappings)
      for (int i = 0; i < p.n_peers; ++i) {
        uint8_t* pd = reinterpret_cast<uint8_t*>(dst) + p.peer_off[i];
        reinterpret_cast<uint4*>(pd)[v] = o1;
        reinterpret_cast<uint4*>(pd + HALF * 2)[v] = o2;
      }
    }
  }
  if (part > 0 && p.n_peers > 0) __threadfence_system();   // peer stores visible before any later signal
}

// Lane-per-chunk prologue (bf16 or fp32 input; bf16 tiles, or fp32 tiles rounded to tf32 for the tf32
// path; head dims 64 / 96 / 128).  Eight lanes per head; lane s < D/16
// owns elements [8s, 8s + 8) of both halves of the head, so the RoPE pair (i, i + D/2) stays in one
// lane with one 16-byte load and one 16-byte store per half, and the head's RMSNorm sum is a
// three-step shuffle over its eight lanes (lanes past D/16 contribute zeros).  A thread holds only
// 16 values per row (the norm weights come from shared memory), so the SM runs 32 warps, and the blocks stride over (row, head, lane) items with the next item's two loads issued
// before the current one is normalised, rotated and stored: the kernel is HBM-latency-bound, and this
// keeps about twice as many reads in flight per SM as one (row, head) item per thread.  Any head
// count works (a head's eight lanes are an aligned group of a warp), so every shard of a call takes
// the same kernel and the same summation order.
#ifndef NSA_LANE_MIN_BLOCKS
#define NSA_LANE_MIN_BLOCKS 4
#endif
template <int D, typename T, bool OUT_F32>
__global__ void __launch_bounds__(256, NSA_LANE_MIN_BLOCKS) prologue_lane_kernel(const PrologueParams p) {
  constexpr int NV = sizeof(T) / 2;   // 16-byte input vectors per half (8 bf16 or 2 x 4 fp32)
  constexpr int HALF = D / 2;
  constexpr int P = D / 16;   // lanes of a head that own data
  static_assert(P >= 1 && P <= 8 && D % 16 == 0, "head dim");
  if (blockIdx.x == 0 && blockIdx.y == 0)
    for (int i = threadIdx.x; i < p.zero_count; i += blockDim.x) p.zero_ptr[i] = 0;
  const int part = blockIdx.y / p.B + (p.skip_q ? 1 : 0);
  const int bl = blockIdx.y % p.B;
  const int b = p.b_begin + bl;
  const int H = part == 0 ? p.Hq : p.Hkv;
  const int pad = p.rows[part];
  const RowView& view = part == 0 ? p.q : (part == 1 ? p.k : p.v);
  const int h_begin = part == 0 ? p.hq_begin : p.hkv_begin;
  const float* w = part == 0 ? p.q_w : (part == 1 ? p.k_w : nullptr);
  const int valid_rows = part == 0 ? p.Lq : (p.kv_len ? min(p.kv_len[b], p.Lk) : p.Lk);
  // first produced row: V rows of whole tiles of valid keys come from the input instead
  const int r_begin = (part == 2 && p.v_tile > 0) ? max(0, valid_rows / p.v_tile * p.v_tile - p.row0[2]) : 0;
  // (row, head, lane) items, item = (row * H + head) * 8 + lane; the launcher keeps the count below
  // 2^31 and makes the stride a multiple of 8 * H, so a thread's lane and head never change and its
  // row advances by a constant
  const int nrows = max(pad - r_begin, 0);
  const int count = nrows * H * 8;
  const int stride = gridDim.x * blockDim.x;
  const int di = stride / (8 * H);
  const int it0 = blockIdx.x * blockDim.x + threadIdx.x;
  const int sub = it0 % 8;
  const int hh = (it0 / 8) % H;
  const int i0 = it0 / (8 * H);
  const bool lane_on = sub < P;
  // the part's norm weights, read per row from shared memory (registers are kept for the loads)
  __shared__ __align__(16) float sw[D];
  if (w)
    for (int e = threadIdx.x; e < D; e += blockDim.x) sw[e] = w[e];
  __syncthreads();
  const int ok_rows = min(nrows, valid_rows - p.row0[part] - r_begin);   // rows with data
  // addresses are rebuilt from the kernel parameters at each use (constant-bank operands), which
  // keeps the live registers at what 32 warps per SM allow
  auto load = [&](int i, uint4 (&a)[NV], uint4 (&c)[NV]) {   // produced row r_begin + i (zeros past the data)
    const bool ok = lane_on && i < ok_rows;
    const T* src = reinterpret_cast<const T*>(view.ptr) + (int64_t)b * view.bstride + view.off +
                   (int64_t)(h_begin + hh) * D + sub * 8 + (int64_t)(p.src_row0[part] + r_begin + i) * view.ld;
#pragma unroll
    for (int v = 0; v < NV; ++v) {
      a[v] = ok ? __ldg(reinterpret_cast<const uint4*>(src) + v) : make_uint4(0u, 0u, 0u, 0u);
      c[v] = ok ? __ldg(reinterpret_cast<const uint4*>(src + HALF) + v) : make_uint4(0u, 0u, 0u, 0u);
    }
  };
  const TileOut& to = p.out[part];
#ifndef NSA_LANE_DEPTH
#define NSA_LANE_DEPTH 1
#endif
  constexpr int DEPTH = NSA_LANE_DEPTH;   // items whose loads are in flight beyond the current one
  int i = i0;
  uint4 a[NV], c[NV];
  uint4 pa[DEPTH][NV], pc[DEPTH][NV];
  load(i, a, c);
#pragma unroll
  for (int k = 0; k < DEPTH - 1; ++k) load(i + (k + 1) * di, pa[k], pc[k]);
  // the bound is uniform over the block (its first item), so every lane reaches the shuffles
  for (int first = blockIdx.x * blockDim.x; first < count; first += stride, i += di) {
    load(i + DEPTH * di, pa[DEPTH - 1], pc[DEPTH - 1]);
    const int r_out = r_begin + i;
    const int row = p.row0[part] + r_out;   // key / query index and RoPE row
    const bool in_range = lane_on && i < nrows;
    const bool valid = in_range && row < valid_rows;
    float x1[8], x2[8];
    if constexpr (NV == 1) {
      const uint32_t wa[4] = {a[0].x, a[0].y, a[0].z, a[0].w}, wc[4] = {c[0].x, c[0].y, c[0].z, c[0].w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        x1[2 * e] = __uint_as_float(wa[e] << 16);
        x1[2 * e + 1] = __uint_as_float(wa[e] & 0xffff0000u);
        x2[2 * e] = __uint_as_float(wc[e] << 16);
        x2[2 * e + 1] = __uint_as_float(wc[e] & 0xffff0000u);
      }
    } else {
#pragma unroll
      for (int v = 0; v < 2; ++v) {
        x1[4 * v] = __uint_as_float(a[v].x); x1[4 * v + 1] = __uint_as_float(a[v].y);
        x1[4 * v + 2] = __uint_as_float(a[v].z); x1[4 * v + 3] = __uint_as_float(a[v].w);
        x2[4 * v] = __uint_as_float(c[v].x); x2[4 * v + 1] = __uint_as_float(c[v].y);
        x2[4 * v + 2] = __uint_as_float(c[v].z); x2[4 * v + 3] = __uint_as_float(c[v].w);
      }
    }
    if (w) {   // uniform over the block: every lane reaches the shuffles
      float ss = 0.f;
#pragma unroll
      for (int e = 0; e < 8; ++e) ss += x1[e] * x1[e] + x2[e] * x2[e];
      ss += __shfl_xor_sync(0xffffffffu, ss, 4);
      ss += __shfl_xor_sync(0xffffffffu, ss, 2);
      ss += __shfl_xor_sync(0xffffffffu, ss, 1);
      const float r = rsqrtf(ss / (float)D + p.eps);
      const float4* w1 = reinterpret_cast<const float4*>(sw + (lane_on ? sub * 8 : 0));
      const float4* w2 = reinterpret_cast<const float4*>(sw + HALF + (lane_on ? sub * 8 : 0));
#pragma unroll
      for (int q = 0; q < 2; ++q) {
        const float4 a4 = w1[q], c4 = w2[q];
        const float wa[4] = {a4.x, a4.y, a4.z, a4.w}, wc[4] = {c4.x, c4.y, c4.z, c4.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          x1[4 * q + e] *= r * wa[e];
          x2[4 * q + e] *= r * wc[e];
        }
      }
    }
    if (valid && part < 2 && p.cs != nullptr && row < p.rope_rows) {
      const float4* cp = reinterpret_cast<const float4*>(p.cs + (int64_t)row * HALF + sub * 8);
      const float4* sp = reinterpret_cast<const float4*>(p.cs + p.sin_off + (int64_t)row * HALF + sub * 8);
#pragma unroll
      for (int q = 0; q < 2; ++q) {
        const float4 c4 = __ldg(cp + q), s4 = __ldg(sp + q);
        const float cc[4] = {c4.x, c4.y, c4.z, c4.w}, sn[4] = {s4.x, s4.y, s4.z, s4.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float xa = x1[4 * q + e], xc = x2[4 * q + e];
          x1[4 * q + e] = xa * cc[e] - xc * sn[e];
          x2[4 * q + e] = xc * cc[e] + xa * sn[e];
        }
      }
    }
    if (in_range) {
      const int64_t off = (int64_t)bl * to.bs + (int64_t)hh * to.hs + (int64_t)r_out * to.rs + sub * 8;
      if constexpr (OUT_F32) {   // the tf32 path: fp32 tiles rounded to tf32 (TileOut strides count floats)
        float* dst = reinterpret_cast<float*>(to.ptr) + off;
#pragma unroll
        for (int v = 0; v < 2; ++v) {
          reinterpret_cast<float4*>(dst)[v] = make_float4(round_tf32(x1[4 * v]), round_tf32(x1[4 * v + 1]),
                                                          round_tf32(x1[4 * v + 2]), round_tf32(x1[4 * v + 3]));
          reinterpret_cast<float4*>(dst + HALF)[v] = make_float4(round_tf32(x2[4 * v]), round_tf32(x2[4 * v + 1]),
                                                                 round_tf32(x2[4 * v + 2]), round_tf32(x2[4 * v + 3]));
        }
      } else {
        __nv_bfloat16* dst = to.ptr + off;
        *reinterpret_cast<uint4*>(dst) = make_uint4(pack_bf16x2(x1[0], x1[1]), pack_bf16x2(x1[2], x1[3]),
                                                    pack_bf16x2(x1[4], x1[5]), pack_bf16x2(x1[6], x1[7]));
        *reinterpret_cast<uint4*>(dst + HALF) = make_uint4(pack_bf16x2(x2[0], x2[1]), pack_bf16x2(x2[2], x2[3]),
                                                           pack_bf16x2(x2[4], x2[5]), pack_bf16x2(x2[6], x2[7]));
      }
    }
#pragma unroll
    for (int v = 0; v < NV; ++v) {
      a[v] = pa[0][v];
      c[v] = pc[0][v];
    }
#pragma unroll
    for (int k = 0; k < DEPTH - 1; ++k)
#pragma unroll
      for (int v = 0; v < NV; ++v) {
        pa[k][v] = pa[k + 1][v];
        pc[k][v] = pc[k + 1][v];
      }
  }
}

// Streaming form of the vector prologue (bf16 input, head dim 256): the thread mapping and the
// arithmetic are the vector kernel's, but the blocks of one (part, batch element) stride over its
// (row, head) items, NSA_PROLOGUE_ITEMS per thread, and each thread issues the loads of its next
// item before it normalises, rotates and stores the current one, so its HBM reads stay in flight
// while it computes.  V rows of key tiles the attention kernel reads straight from the input are
// not visited.  At head dim 256 (P = 8, two items of 64 bytes in flight per thread, 16 warps per SM)
// it beats the one-item-per-thread kernel.  The values stay packed two to a register until they are
// used, which is what lets the next item's loads sit beside the current item's arithmetic.
#ifndef NSA_PROLOGUE_ITEMS
#define NSA_PROLOGUE_ITEMS 8   // (row, head) items per thread and part
#endif
constexpr int kStreamThreads = 128;   // 4 resident blocks per SM at <= 128 registers

template <int D, int P>
__global__ void __launch_bounds__(kStreamThreads, 4) prologue_stream_kernel(const PrologueParams p) {
  using T = __nv_bfloat16;
  constexpr int S = D / (2 * P);
  constexpr int HALF = D / 2;
  constexpr int NV = S / 8;   // 16-byte input vectors per half
  static_assert(S % 8 == 0 && kStreamThreads % P == 0, "vector width");
  if (blockIdx.x == 0 && blockIdx.y == 0)
    for (int i = threadIdx.x; i < p.zero_count; i += blockDim.x) p.zero_ptr[i] = 0;
  const int part = blockIdx.y / p.B + (p.skip_q ? 1 : 0);
  const int bl = blockIdx.y % p.B;
  const int b = p.b_begin + bl;
  const int H = part == 0 ? p.Hq : p.Hkv;
  const int pad = p.rows[part];
  const RowView& view = part == 0 ? p.q : (part == 1 ? p.k : p.v);
  const int h_begin = part == 0 ? p.hq_begin : p.hkv_begin;
  const float* w = part == 0 ? p.q_w : (part == 1 ? p.k_w : nullptr);
  const int valid_rows = part == 0 ? p.Lq : (p.kv_len ? min(p.kv_len[b], p.Lk) : p.Lk);
  // first produced row: V rows of whole tiles of valid keys come from the input instead
  const int r_begin = (part == 2 && p.v_tile > 0) ? max(0, valid_rows / p.v_tile * p.v_tile - p.row0[2]) : 0;
  const long long count = (long long)max(pad - r_begin, 0) * H * P;
  const long long stride = (long long)gridDim.x * blockDim.x;
  const int sub = (int)(threadIdx.x % P);   // blockIdx.x * blockDim.x and the stride are multiples of P
  const T* src_b = reinterpret_cast<const T*>(view.ptr) + (int64_t)b * view.bstride + view.off + sub * S;
  const TileOut& to = p.out[part];

  // raw input of one item: NV vectors of each half (zeros past the last item or the valid rows)
  auto load = [&](long long i, uint4 (&a)[NV], uint4 (&c)[NV]) {
    const long long rest = i / P;
    const int hh = (int)(rest % H);
    const int r_out = r_begin + (int)(rest / H);
    const bool valid = i < count && p.row0[part] + r_out < valid_rows;
    const T* src = src_b + (int64_t)(p.src_row0[part] + r_out) * view.ld + (int64_t)(h_begin + hh) * D;
#pragma unroll
    for (int v = 0; v < NV; ++v) {
      a[v] = valid ? __ldg(reinterpret_cast<const uint4*>(src) + v) : make_uint4(0u, 0u, 0u, 0u);
      c[v] = valid ? __ldg(reinterpret_cast<const uint4*>(src + HALF) + v) : make_uint4(0u, 0u, 0u, 0u);
    }
  };

  long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  const long long warp_first = idx - (threadIdx.x % 32);   // loop bound uniform over the warp (shuffles)
  uint4 a[NV], c[NV];
  load(idx, a, c);
  for (long long wf = warp_first; wf < count; wf += stride, idx += stride) {
    uint4 na[NV], nc[NV];
    load(idx + stride, na, nc);
    const bool in_range = idx < count;
    const long long rest = idx / P;
    const int hh = (int)(rest % H);
    const int r_out = r_begin + (int)(rest / H);
    const int row = p.row0[part] + r_out;   // key / query index and RoPE row
    const bool valid = in_range && row < valid_rows;
    const bool rope = part < 2 && p.cs != nullptr && row < p.rope_rows;
    // The values stay packed (two bf16 per register) and are widened where they are used, so that
    // the next item's loads and this item's arithmetic fit beside each other in registers.
    float r = 1.f;
    if (w) {   // w is uniform over the block (one part per blockIdx.y): every lane reaches the shuffle
      uint64_t acc = f2_pack(0.f, 0.f);
#pragma unroll
      for (int v = 0; v < NV; ++v) {
        const uint32_t wa[4] = {a[v].x, a[v].y, a[v].z, a[v].w}, wc[4] = {c[v].x, c[v].y, c[v].z, c[v].w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const uint64_t xa = f2_pack(__uint_as_float(wa[e] << 16), __uint_as_float(wa[e] & 0xffff0000u));
          const uint64_t xc = f2_pack(__uint_as_float(wc[e] << 16), __uint_as_float(wc[e] & 0xffff0000u));
          acc = f2_fma(xa, xa, acc);
          acc = f2_fma(xc, xc, acc);
        }
      }
      float s0, s1;
      f2_unpack(acc, s0, s1);
      float ss = s0 + s1;
#pragma unroll
      for (int o = 1; o < P; o <<= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
      r = rsqrtf(ss / (float)D + p.eps);
    }
    if (in_range) {
      __nv_bfloat16* dst = to.ptr + (int64_t)bl * to.bs + (int64_t)hh * to.hs + (int64_t)r_out * to.rs + sub * S;
      const bool do_w = valid && w != nullptr, do_rope = valid && rope;
#pragma unroll
      for (int v = 0; v < NV; ++v) {
        const uint32_t wa[4] = {a[v].x, a[v].y, a[v].z, a[v].w}, wc[4] = {c[v].x, c[v].y, c[v].z, c[v].w};
        uint32_t o1[4], o2[4];
#pragma unroll
        for (int q = 0; q < 2; ++q) {   // four elements of each half at a time
          float x1[4] = {__uint_as_float(wa[2 * q] << 16), __uint_as_float(wa[2 * q] & 0xffff0000u),
                         __uint_as_float(wa[2 * q + 1] << 16), __uint_as_float(wa[2 * q + 1] & 0xffff0000u)};
          float x2[4] = {__uint_as_float(wc[2 * q] << 16), __uint_as_float(wc[2 * q] & 0xffff0000u),
                         __uint_as_float(wc[2 * q + 1] << 16), __uint_as_float(wc[2 * q + 1] & 0xffff0000u)};
          const int j = sub * S + v * 8 + q * 4;   // element of the first half
          if (do_w) {
            const float4 w1 = __ldg(reinterpret_cast<const float4*>(w + j));
            const float4 w2 = __ldg(reinterpret_cast<const float4*>(w + HALF + j));
            x1[0] *= r * w1.x; x1[1] *= r * w1.y; x1[2] *= r * w1.z; x1[3] *= r * w1.w;
            x2[0] *= r * w2.x; x2[1] *= r * w2.y; x2[2] *= r * w2.z; x2[3] *= r * w2.w;
          }
          if (do_rope) {
            const float4 c4 = __ldg(reinterpret_cast<const float4*>(p.cs + (int64_t)row * HALF + j));
            const float4 s4 = __ldg(reinterpret_cast<const float4*>(p.cs + p.sin_off + (int64_t)row * HALF + j));
            const float cc[4] = {c4.x, c4.y, c4.z, c4.w}, sn[4] = {s4.x, s4.y, s4.z, s4.w};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const float xa = x1[e], xc = x2[e];
              x1[e] = xa * cc[e] - xc * sn[e];
              x2[e] = xc * cc[e] + xa * sn[e];
            }
          }
          o1[2 * q] = pack_bf16x2(x1[0], x1[1]);
          o1[2 * q + 1] = pack_bf16x2(x1[2], x1[3]);
          o2[2 * q] = pack_bf16x2(x2[0], x2[1]);
          o2[2 * q + 1] = pack_bf16x2(x2[2], x2[3]);
        }
        const uint4 u1 = make_uint4(o1[0], o1[1], o1[2], o1[3]), u2 = make_uint4(o2[0], o2[1], o2[2], o2[3]);
        reinterpret_cast<uint4*>(dst)[v] = u1;
        reinterpret_cast<uint4*>(dst + HALF)[v] = u2;
      }
    }
#pragma unroll
    for (int v = 0; v < NV; ++v) {
      a[v] = na[v];
      c[v] = nc[v];
    }
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

namespace {

bool aligned16(const void* ptr, int64_t elem_offset_multiple_bytes) {
  return (reinterpret_cast<uintptr_t>(ptr) & 15) == 0 && (elem_offset_multiple_bytes & 15) == 0;
}

// Every vector access of the fast path is 16-byte aligned iff the bases, strides, offsets and the
// per-thread chunk are (the chunk and head sizes are multiples of 16 bytes by construction).
bool vec_ok(const PrologueParams& p, int elem, int out_elem) {
  const RowView* vs[3] = {&p.q, &p.k, &p.v};
  for (const RowView* v : vs)
    if (!aligned16(v->ptr, v->ld * elem) || ((v->bstride * elem) & 15) || ((v->off * elem) & 15)) return false;
  if (p.cs && (!aligned16(p.cs, p.sin_off * 4))) return false;
  for (int i = p.skip_q ? 1 : 0; i < 3; ++i) {
    const TileOut& o = p.out[i];
    if (!aligned16(o.ptr, o.bs * out_elem) || ((o.hs * out_elem) & 15) || ((o.rs * out_elem) & 15)) return false;
  }
  if ((p.q_w && !aligned16(p.q_w, 0)) || (p.k_w && !aligned16(p.k_w, 0))) return false;
  return true;
}

template <int D, int P>
cudaError_t launch_stream(const PrologueParams& p, cudaStream_t stream) {
  const int rows = (!p.skip_q && p.rows[0] > p.rows[1]) ? p.rows[0] : (p.rows[1] > p.rows[2] ? p.rows[1] : p.rows[2]);
  const int H = (!p.skip_q && p.Hq > p.Hkv) ? p.Hq : p.Hkv;
  const long long threads = ((long long)rows * H * P + NSA_PROLOGUE_ITEMS - 1) / NSA_PROLOGUE_ITEMS;
  const long long groups = (p.skip_q ? 2 : 3) * (long long)p.B;
  // NSA_PROLOGUE_ITEMS items per thread while that fills the SMs; a small call (one or two sequences
  // per GPU) spreads its items over one resident wave instead of running eight in a row per thread
  const long long wave = std::max(1LL, (long long)device_sm_count() * 4 / groups);
  const long long one_each = ((long long)rows * H * P + kStreamThreads - 1) / kStreamThreads;
  const long long blocks = std::max((threads + kStreamThreads - 1) / kStreamThreads, std::min(wave, one_each));
  if (blocks > 0x7FFFFFFFLL || 3LL * p.B > 65535) return cudaErrorInvalidValue;
  prologue_stream_kernel<D, P><<<dim3((unsigned)blocks, (p.skip_q ? 2 : 3) * p.B), kStreamThreads, 0, stream>>>(p);
  return cudaGetLastError();
}

// Lane kernel grid: the blocks of each (part, batch element) stride over its items.
template <int D, typename T>
cudaError_t launch_lane(const PrologueParams& p, cudaStream_t stream) {
  const int rows = (!p.skip_q && p.rows[0] > p.rows[1]) ? p.rows[0] : (p.rows[1] > p.rows[2] ? p.rows[1] : p.rows[2]);
  const int H = (!p.skip_q && p.Hq > p.Hkv) ? p.Hq : p.Hkv;
  const int groups = (p.skip_q ? 2 : 3) * p.B;
  if (3LL * p.B > 65535 || p.Hq < 1 || p.Hkv < 1 || (long long)rows * H * 8 >= (1LL << 31)) return cudaErrorInvalidValue;
  // the stride (blocks * 256 items) must be a multiple of 8 * H for the query and the key heads
  auto need_blocks = [](int h) { return h / std::gcd(h, 32); };
  const long long m = std::lcm(need_blocks(p.skip_q ? p.Hkv : p.Hq), need_blocks(p.Hkv));
#ifndef NSA_LANE_BLOCKS_PER_SM
#define NSA_LANE_BLOCKS_PER_SM 6
#endif
  // six blocks per SM with four resident (measured at config 2: 31.3 us, against 35.4 with one
  // resident wave and 38.0 with eight per SM)
  const long long want = std::max(1LL, (long long)device_sm_count() * NSA_LANE_BLOCKS_PER_SM / groups);
  const long long need = ((long long)rows * H * 8 + 255) / 256;
  const long long bx = (std::max(1LL, std::min(want, need)) + m - 1) / m * m;
  if (bx > 0x7FFFFFFFLL / 256) return cudaErrorInvalidValue;
  if (p.out_f32)
    prologue_lane_kernel<D, T, true><<<dim3((unsigned)bx, groups), 256, 0, stream>>>(p);
  else
    prologue_lane_kernel<D, T, false><<<dim3((unsigned)bx, groups), 256, 0, stream>>>(p);
  return cudaGetLastError();
}

template <int D, int P, typename T>
cudaError_t launch_vec(const PrologueParams& p, cudaStream_t stream) {
  const int rows = (!p.skip_q && p.rows[0] > p.rows[1]) ? p.rows[0] : (p.rows[1] > p.rows[2] ? p.rows[1] : p.rows[2]);
  const int H = (!p.skip_q && p.Hq > p.Hkv) ? p.Hq : p.Hkv;
  const long long threads = (long long)rows * H * P;
  const long long blocks = (threads + 255) / 256;
  if (blocks > 0x7FFFFFFFLL || 3LL * p.B > 65535) return cudaErrorInvalidValue;
  prologue_vec_kernel<D, P, T><<<dim3((unsigned)blocks, (p.skip_q ? 2 : 3) * p.B), 256, 0, stream>>>(p);
  return cudaGetLastError();
}

// threads per head of a row at head dims 96 and 256
#ifndef NSA_PROLOGUE_P96
#define NSA_PROLOGUE_P96 2
#endif
#ifndef NSA_PROLOGUE_P256
#define NSA_PROLOGUE_P256 8
#endif

template <typename T>
cudaError_t launch_vec_t(const PrologueParams& p, cudaStream_t stream) {
  switch (p.D) {
    case 64: return launch_lane<64, T>(p, stream);
    case 96: return launch_lane<96, T>(p, stream);
    case 128: return launch_lane<128, T>(p, stream);
    case 256:
      if constexpr (sizeof(T) == 2) return launch_stream<256, NSA_PROLOGUE_P256>(p, stream);
      return launch_vec<256, NSA_PROLOGUE_P256, T>(p, stream);
    case 512: return launch_vec<512, 16, T>(p, stream);   // the VAE's head dim: 16 lanes per head
    default: return cudaErrorNotSupported;
  }
}

}  // namespace

cudaError_t launch_prologue(const PrologueParams& p, cudaStream_t stream) {
  const int rows = (!p.skip_q && p.rows[0] > p.rows[1]) ? p.rows[0] : (p.rows[1] > p.rows[2] ? p.rows[1] : p.rows[2]);
  if (rows <= 0 || p.B <= 0) return cudaSuccess;
  const int elem = p.src_f32 ? 4 : 2;
  // Rows that also go to other GPUs take the row-per-block kernel: its consecutive threads write
  // each row's head segments contiguously, which NVLink stores need to run at speed.
  // fp32 (tf32-path) tiles come from the lane kernel only (head dims 64 / 96 / 128)
  const bool lane_d = p.D == 64 || p.D == 96 || p.D == 128;
  if (p.n_peers == 0 && (p.out_f32 ? lane_d : (lane_d || p.D == 256 || p.D == 512)) &&
      vec_ok(p, elem, p.out_f32 ? 4 : 2))
    return p.src_f32 ? launch_vec_t<float>(p, stream) : launch_vec_t<__nv_bfloat16>(p, stream);
  dim3 grid(rows, p.B, p.skip_q ? 2 : 3);
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
