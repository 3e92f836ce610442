// Linear layer for sm_100a with the reference's GEMM epilogue: ops.linear (app/gpu/ops.js:50-66)
// over the tiled GEMM of app/gpu/gemm.js, whose epilogue (gemm.js:155-165) is
//   r = alpha * acc (+ bias[n]) (silu), then C = r, C += r, or C += gate[gOff + n] * r (in place).
// The DiT block's output projection is the gated form: x += gate * (a @ W_proj^T + b)
// (app/models/nanosaur2.js:210; tools/reference.py:285).  A and W are bf16 (W in the Linear layout
// [N][K]); C is fp32, the reference's residual stream.
//
// CTA (one per SM, persistent over 128 x 256 output tiles), the QKV projection's structure:
//   warp 0      TMA producer: A [128 rows][64] and W [256 rows][64] slices, 4-stage ring
//   warp 1      TMEM allocator + MMA issuer: 128 x 256 x 16 tcgen05.mma into one of two accumulators
//   warps 2-9   epilogue, two groups of four warps, each group half of the tile's columns; a thread
//               owns one output row: alpha, bias, silu, then the store (16-byte stores) or the
//               residual / gated residual (16-byte fp32 vector reductions into C).  Bias and gate are
//               bulk-copied into shared memory.
#include "nsa_internal.h"
#include "ptx.cuh"

namespace nsa {

namespace {

constexpr int kLinBK = 64;
constexpr int kLinNT = 256;
constexpr int kLinThreads = 320;
constexpr int kLinA = 128 * kLinBK * 2;
constexpr int kLinB = kLinNT * kLinBK * 2;
constexpr int kLinStage = kLinA + kLinB;   // 48 KB
constexpr int kLinStages = 4;
constexpr uint32_t kLinIdesc = idesc_bf16_f32(128, kLinNT, 0, 0);

__device__ __forceinline__ float silu(float x) { return x / (1.f + expf(-x)); }

__global__ void __launch_bounds__(kLinThreads, 1)
    linear_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmW,
                  const LinearParams p) {
  constexpr int S = kLinStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int nvec = p.n_tiles * kLinNT;                               // bias / gate entries staged
  float* sbias = reinterpret_cast<float*>(smem + S * kLinStage);     // [nvec], zeros past N or without a bias
  float* sgate = sbias + nvec;                                       // [nvec], ones without a gate
  uint64_t* full = reinterpret_cast<uint64_t*>(sgate + nvec);
  uint64_t* empty = full + S;
  uint64_t* acc_full = empty + S;
  uint64_t* acc_empty = acc_full + 2;   // 256 epilogue arrivals
  uint64_t* drain = acc_empty + 2;
  uint64_t* pbar = drain + 1;           // bias / gate landed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(pbar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const uint64_t to = p.timeout_ns;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], 256);
    }
    mbar_init(drain, 1);
    mbar_init(pbar, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  // entries the bulk copies do not cover: past N, or no bias / gate at all
  for (int i = threadIdx.x; i < nvec; i += blockDim.x) {
    if (!p.bias || i >= p.N) sbias[i] = 0.f;
    if (!p.gate || i >= p.N) sgate[i] = 1.f;
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int tiles = p.m_tiles * p.n_tiles;
  const int G = gridDim.x;

  if (warp == 0) {
    // ---------------------------------------------------------------- TMA producer
    if (lane == 0) {
      tma_prefetch_desc(&tmA);
      tma_prefetch_desc(&tmW);
      const uint32_t vb = (uint32_t)p.N * 4;
      mbar_arrive_expect_tx(pbar, (p.bias ? vb : 0u) + (p.gate ? vb : 0u));
      if (p.bias) bulk_load(sbias, p.bias, vb, pbar);
      if (p.gate) bulk_load(sgate, p.gate, vb, pbar);
      int step = 0;
      bool ok = true;
      for (int u = blockIdx.x; ok && u < tiles; u += G) {
        const int nt = u % p.n_tiles, m0 = (u / p.n_tiles) * 128;
        for (int ks = 0; ks < p.k_steps; ++ks, ++step) {
          const int s = step % S;
          if (step >= S && !wait_bounded(&empty[s], ((step / S) - 1) & 1, abort_flag, p.err, kErrTimeoutProjection, to)) {
            ok = false;
            break;
          }
          uint8_t* st = smem + s * kLinStage;
          mbar_arrive_expect_tx(&full[s], kLinStage);
          tma_load_2d(st, &tmA, &full[s], ks * kLinBK, m0);
          tma_load_2d(st + kLinA, &tmW, &full[s], ks * kLinBK, nt * kLinNT);
        }
      }
      wait_drain(pbar, 0, to);
      for (int i = step > S ? step - S : 0; i < step; ++i) wait_drain(&full[i % S], (i / S) & 1, to);
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      int step = 0, t = 0;
      bool ok = true;
      for (int u = blockIdx.x; ok && u < tiles; u += G) {
        const int a = t & 1;
        if (t >= 2 && !wait_bounded(&acc_empty[a], ((t >> 1) - 1) & 1, abort_flag, p.err, kErrTimeoutProjection, to)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem + (uint32_t)a * 256u;
        for (int ks = 0; ks < p.k_steps; ++ks, ++step) {
          const int s = step % S;
          if (!wait_bounded(&full[s], (step / S) & 1, abort_flag, p.err, kErrTimeoutProjection, to)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + s * kLinStage), sb = sa + kLinA;
#pragma unroll
          for (int kk = 0; kk < kLinBK / 16; ++kk)
            mma_ss(d_tmem, smem_desc(sa + kk * 32, 16, 1024, 2), smem_desc(sb + kk * 32, 16, 1024, 2), kLinIdesc,
                   (ks > 0 || kk > 0) ? 1u : 0u);
          tc_commit(&empty[s]);
        }
        if (!ok) break;
        tc_commit(&acc_full[a]);
        ++t;
      }
      if (!ok) {
        tc_commit(drain);
        wait_drain(drain, 0, to);
      }
    }
  } else {
    // ---------------------------------------------------------------- epilogue (warps 2-9)
    const int group = (warp - 2) / 4;
    const int quarter = warp % 4;
    const int row_local = quarter * 32 + lane;
    bool params_ready = false;
    int t = 0;
    for (int u = blockIdx.x; u < tiles; u += G) {
      const int nt = u % p.n_tiles, m0 = (u / p.n_tiles) * 128;
      const int a = t & 1;
      bool got = wait_bounded(&acc_full[a], (t >> 1) & 1, abort_flag, p.err, kErrTimeoutProjection, to);
      if (got && !params_ready) {
        got = wait_bounded(pbar, 0, abort_flag, p.err, kErrTimeoutProjection, to);
        params_ready = true;
      }
      if (!__all_sync(0xffffffffu, got)) break;
      tc_fence_after();
      const uint32_t tbase = tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)a * 256u;
      const int r = m0 + row_local;
      float* crow = p.C + (int64_t)r * p.ldc;
#pragma unroll 1
      for (int c64 = group * 128; c64 < group * 128 + 128; c64 += 64) {
        // 64 columns under one wait (warp-wide: every lane, whatever its row)
        uint32_t v64[64];
        tmem_ld64(tbase + (uint32_t)c64, v64);
#pragma unroll
        for (int sub = 0; sub < 4; ++sub) {
          const int c = c64 + sub * 16;
          const int n = nt * kLinNT + c;
          if (r >= p.M || n >= p.N) continue;
          float y[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            float x = p.alpha * __uint_as_float(v64[sub * 16 + i]) + sbias[n + i];
            if (p.act == 1) x = silu(x);
            y[i] = x;
          }
          // The residual forms add into C with vector reductions (each element has one owner, so this
          // is the in-place C += g * r of the reference without a load round trip per chunk).
          if (n + 16 <= p.N) {
            float4* dst = reinterpret_cast<float4*>(crow + n);
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              if (p.resid)
                atomicAdd(dst + q, make_float4(sgate[n + 4 * q] * y[4 * q], sgate[n + 4 * q + 1] * y[4 * q + 1],
                                               sgate[n + 4 * q + 2] * y[4 * q + 2],
                                               sgate[n + 4 * q + 3] * y[4 * q + 3]));
              else
                dst[q] = make_float4(y[4 * q], y[4 * q + 1], y[4 * q + 2], y[4 * q + 3]);
            }
          } else {
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              if (n + i >= p.N) break;
              if (p.resid)
                atomicAdd(crow + n + i, sgate[n + i] * y[i]);
              else
                crow[n + i] = y[i];
            }
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&acc_empty[a]);
      ++t;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace

cudaError_t launch_linear(const LinearParams& p, const CUtensorMap& tmA, const CUtensorMap& tmW, cudaStream_t stream) {
  const int sms = device_sm_count();
  const long long tiles = (long long)p.m_tiles * p.n_tiles;
  if (tiles <= 0) return cudaSuccess;
  if (tiles > 0x7FFFFFFFLL) return cudaErrorInvalidValue;
  const size_t smem = 1024 + (size_t)kLinStages * kLinStage + 2 * (size_t)p.n_tiles * kLinNT * 4 + 256;
  if (smem > 232448) return cudaErrorNotSupported;
  // the limit is raised once per device to the whole 227 KB, so launches of different sizes from
  // several host threads never race on the attribute
  static DeviceOnce once;
  cudaError_t e = once_per_device(once, [] {
    return cudaFuncSetAttribute(linear_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 232448);
  });
  if (e != cudaSuccess) return e;
  const int grid = tiles < sms ? (int)tiles : sms;
  linear_kernel<<<grid, kLinThreads, smem, stream>>>(tmA, tmW, p);
  return cudaGetLastError();
}

}  // namespace nsa
