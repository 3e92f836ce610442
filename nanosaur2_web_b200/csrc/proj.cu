// QKV projection for sm_100a with the attention prologue fused into the GEMM epilogue.
//
// The reference computes the DiT block's q|k|v as `lin(x) = x @ W^T + b` (tools/reference.py:208-210,
// ops.linear in app/gpu/ops.js:50 on the `dit.qkv` weight, app/models/nanosaur2.js:197), the text
// keys / values with a second linear on the text rows (`dit.kv_y`, nanosaur2.js:201), and then runs
// ops.headNorm on q and k (RMSNorm per head + split-half RoPE, nanosaur2.js:199-202).  Here one
// persistent tcgen05 GEMM does the linear and, in its epilogue, the bias, the norm and the RoPE, and
// writes the attention's inputs directly: q' tiles [B][Hq][Lq_pad][D] and packed k'|v' rows
// [B][Lk_pad][2 Hkv D] (the sequence-shard layouts nsa_seq_shard_attention reads).  The qkv matrix
// never reaches HBM.
//
// CTA (one per SM, persistent over output tiles of 128 rows x one group of whole heads):
//   warp 0      TMA producer: X [128 rows][64] and W [heads*D rows][64] slices through a ring
//   warp 1      TMEM allocator + MMA issuer (one thread): 128 x N x 16 tcgen05.mma into one of two
//               accumulators, so the epilogue of a tile overlaps the main loop of the next
//   warps 2-5   epilogue: thread = one output row (its TMEM lane); per head two passes over the
//               accumulator columns: sum of squares, then bias + norm weight + RoPE, bf16 stores
#include "nsa_internal.h"
#include "ptx.cuh"

namespace nsa {

namespace {

constexpr int kProjBK = 64;         // K elements per stage: one 128-byte swizzle row
constexpr int kProjThreads = 192;

template <int D>
struct ProjCfg {
  static constexpr int HPT = D == 96 ? 2 : 256 / D;   // heads per N tile
  static constexpr int NT = HPT * D;                   // 192 at D = 96, 256 otherwise
  static constexpr int A_BYTES = 128 * kProjBK * 2;
  static constexpr int B_BYTES = NT * kProjBK * 2;
  static constexpr int STAGE = A_BYTES + B_BYTES;
  static constexpr int STAGES = (200 * 1024) / STAGE;  // 5 at N = 192, 4 at N = 256
  static constexpr int SMEM = STAGES * STAGE + 1024 + 256;
  static constexpr uint32_t ACC_COLS = 256;            // TMEM columns per accumulator
  static constexpr uint32_t IDESC = idesc_bf16_f32(128, NT, 0, 0);
  static_assert(NT % 16 == 0 && NT <= 256 && STAGE % 1024 == 0 && SMEM <= 232448, "projection tile");
};

__device__ __forceinline__ void store_bf16x16(__nv_bfloat16* dst, const float (&v)[16]) {
  uint4 o[2];
  uint32_t* u = reinterpret_cast<uint32_t*>(o);
#pragma unroll
  for (int e = 0; e < 8; ++e) u[e] = pack_bf16x2(v[2 * e], v[2 * e + 1]);
  reinterpret_cast<uint4*>(dst)[0] = o[0];
  reinterpret_cast<uint4*>(dst)[1] = o[1];
}

template <int D>
__global__ void __launch_bounds__(kProjThreads, 1)
    proj_kernel(const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmW, const ProjParams p) {
  using C = ProjCfg<D>;
  constexpr int S = C::STAGES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S * C::STAGE);
  uint64_t* empty = full + S;
  uint64_t* acc_full = empty + S;    // [2] accumulator ready for the epilogue
  uint64_t* acc_empty = acc_full + 2;   // [2] accumulator read out (128 arrivals)
  uint64_t* drain = acc_empty + 2;      // MMAs of an aborted CTA finished
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
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
      mbar_init(&acc_empty[i], 128);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmX);
    tma_prefetch_desc(&tmW);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  if (blockIdx.x == 0)
    for (int i = threadIdx.x; i < p.zero_count; i += blockDim.x) p.zero_ptr[i] = 0;
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  const int tiles = p.B * p.m_tiles * p.n_tiles;
  const int G = gridDim.x;
  const int nt_q = p.image ? p.Hq / C::HPT : 0;
  const int nt_kv = p.Hkv / C::HPT;
  // tile u -> (local batch element, first row, N tile, part 0/1/2 = q/k/v, first head); false for
  // image k / v tiles wholly past the shard's query rows (those keys belong to other shards)
  auto decode = [&](int u, int& bl, int& m0, int& nt, int& part, int& h0) -> bool {
    nt = u % p.n_tiles;
    const int rest = u / p.n_tiles;
    m0 = (rest % p.m_tiles) * 128;
    bl = rest / p.m_tiles;
    if (nt < nt_q) {
      part = 0;
      h0 = nt * C::HPT;
    } else if (nt < nt_q + nt_kv) {
      part = 1;
      h0 = (nt - nt_q) * C::HPT;
    } else {
      part = 2;
      h0 = (nt - nt_q - nt_kv) * C::HPT;
    }
    return !(p.image && part > 0 && m0 >= p.valid_q);
  };

  if (warp == 0) {
    // ---------------------------------------------------------------- TMA producer
    if (lane == 0) {
      int step = 0;
      bool ok = true;
      for (int u = blockIdx.x; ok && u < tiles; u += G) {
        int bl, m0, nt, part, h0;
        if (!decode(u, bl, m0, nt, part, h0)) continue;
        for (int ks = 0; ks < p.k_steps; ++ks, ++step) {
          const int s = step % S;
          if (step >= S &&
              !wait_bounded(&empty[s], ((step / S) - 1) & 1, abort_flag, p.err, kErrTimeoutProjection, to)) {
            ok = false;
            break;
          }
          uint8_t* st = smem + s * C::STAGE;
          mbar_arrive_expect_tx(&full[s], C::STAGE);
          tma_load_3d(st, &tmX, &full[s], ks * kProjBK, p.x_row0 + m0, bl);
          tma_load_2d(st + C::A_BYTES, &tmW, &full[s], ks * kProjBK, nt * C::NT);
        }
      }
      // loads still landing complete before the CTA may exit
      for (int i = step > S ? step - S : 0; i < step; ++i) wait_drain(&full[i % S], (i / S) & 1, to);
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      int step = 0, t = 0;
      bool ok = true;
      for (int u = blockIdx.x; ok && u < tiles; u += G) {
        int bl, m0, nt, part, h0;
        if (!decode(u, bl, m0, nt, part, h0)) continue;
        const int a = t & 1;
        if (t >= 2 && !wait_bounded(&acc_empty[a], ((t >> 1) - 1) & 1, abort_flag, p.err, kErrTimeoutProjection, to)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem + (uint32_t)a * C::ACC_COLS;
        for (int ks = 0; ks < p.k_steps; ++ks, ++step) {
          const int s = step % S;
          if (!wait_bounded(&full[s], (step / S) & 1, abort_flag, p.err, kErrTimeoutProjection, to)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + s * C::STAGE), sb = sa + C::A_BYTES;
#pragma unroll
          for (int kk = 0; kk < kProjBK / 16; ++kk)
            mma_ss(d_tmem, smem_desc(sa + kk * 32, 16, 1024, 2), smem_desc(sb + kk * 32, 16, 1024, 2), C::IDESC,
                   (ks > 0 || kk > 0) ? 1u : 0u);
          tc_commit(&empty[s]);
        }
        if (!ok) break;
        tc_commit(&acc_full[a]);
        ++t;
      }
      if (!ok) {
        // every MMA already issued finishes before the CTA frees its tensor memory
        tc_commit(drain);
        wait_drain(drain, 0, to);
      }
    }
  } else {
    // ---------------------------------------------------------------- epilogue (warps 2-5)
    const int quarter = warp % 4;   // TMEM lane quarter this warp may access
    const int row_local = quarter * 32 + lane;
    int t = 0;
    for (int u = blockIdx.x; u < tiles; u += G) {
      int bl, m0, nt, part, h0;
      if (!decode(u, bl, m0, nt, part, h0)) continue;
      const int a = t & 1;
      if (!__all_sync(0xffffffffu, wait_bounded(&acc_full[a], (t >> 1) & 1, abort_flag, p.err, kErrTimeoutProjection,
                                                to)))
        break;
      tc_fence_after();
      const uint32_t tbase = tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)a * C::ACC_COLS;
      const int r = m0 + row_local;   // GEMM row
      const int b = p.b_begin + bl;
      const int key = p.key_row0 + r;
      const int kv_valid = p.kv_len ? min(p.kv_len[b], p.Lk) : p.Lk;
      // which rows exist in the destination, and which hold data (the rest are zeros)
      bool write, valid;
      if (part == 0) {
        write = r < p.Lq_pad;
        valid = r < p.valid_q;
      } else if (p.image) {
        write = r < p.valid_q;   // other keys are other shards' (or the text rows)
        valid = write && key < kv_valid;
      } else {
        write = key < p.Lk_pad;
        valid = key < kv_valid;
      }
      const float* w = part == 0 ? p.q_w : (part == 1 ? p.k_w : nullptr);
      const bool rope = p.image && part < 2 && p.cs != nullptr;
      const int rrow = p.rope_row0 + r;
#pragma unroll 1
      for (int hh = 0; hh < C::HPT; ++hh) {
        const int h = h0 + hh;
        const uint32_t col0 = (uint32_t)(hh * D);
        const float* bias = p.bias ? p.bias + nt * C::NT + hh * D : nullptr;
        // pass 1: sum of squares of (acc + bias) over the head (tcgen05.ld is warp-wide: every lane)
        float rn = 1.f;
        if (w) {
          float ss = 0.f;
#pragma unroll 1
          for (int c = 0; c < D; c += 16) {
            uint32_t v[16];
            tmem_ld16(tbase + col0 + (uint32_t)c, v);
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              const float x = __uint_as_float(v[i]) + (bias ? __ldg(bias + c + i) : 0.f);
              ss = fmaf(x, x, ss);
            }
          }
          rn = rsqrtf(ss / (float)D + p.eps);
        }
        __nv_bfloat16* dst;
        if (part == 0)
          dst = p.q_prime + (((int64_t)bl * p.Hq + h) * p.Lq_pad + r) * D;
        else
          dst = p.kv_packed + ((int64_t)bl * p.Lk_pad + key) * p.kv_ld + (part == 2 ? (int64_t)p.Hkv * D : 0) +
                (int64_t)h * D;
        // pass 2: pairs (i, i + D/2): bias, norm weight, RoPE, bf16
#pragma unroll 1
        for (int c = 0; c < D / 2; c += 16) {
          uint32_t v1[16], v2[16];
          tmem_ld16(tbase + col0 + (uint32_t)c, v1);
          tmem_ld16(tbase + col0 + (uint32_t)(c + D / 2), v2);
          float x1[16], x2[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            x1[i] = __uint_as_float(v1[i]) + (bias ? __ldg(bias + c + i) : 0.f);
            x2[i] = __uint_as_float(v2[i]) + (bias ? __ldg(bias + D / 2 + c + i) : 0.f);
          }
          if (w) {
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              x1[i] *= rn * __ldg(w + c + i);
              x2[i] *= rn * __ldg(w + D / 2 + c + i);
            }
          }
          if (rope && valid) {
            const float4* cp = reinterpret_cast<const float4*>(p.cs + (int64_t)rrow * (D / 2) + c);
            const float4* sp = reinterpret_cast<const float4*>(p.cs + p.sin_off + (int64_t)rrow * (D / 2) + c);
#pragma unroll
            for (int q4 = 0; q4 < 4; ++q4) {
              const float4 c4 = __ldg(cp + q4), s4 = __ldg(sp + q4);
              const float cc[4] = {c4.x, c4.y, c4.z, c4.w}, sn[4] = {s4.x, s4.y, s4.z, s4.w};
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const float xa = x1[4 * q4 + e], xc = x2[4 * q4 + e];
                x1[4 * q4 + e] = xa * cc[e] - xc * sn[e];
                x2[4 * q4 + e] = xc * cc[e] + xa * sn[e];
              }
            }
          }
          if (!valid) {
#pragma unroll
            for (int i = 0; i < 16; ++i) x1[i] = x2[i] = 0.f;
          }
          if (write) {
            store_bf16x16(dst + c, x1);
            store_bf16x16(dst + D / 2 + c, x2);
          }
        }
      }
      // the accumulator has been read: the issuer may start the tile after next in it
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

template <int D>
cudaError_t launch_proj_d(const ProjParams& p, const CUtensorMap& tmX, const CUtensorMap& tmW, cudaStream_t stream) {
  using C = ProjCfg<D>;
  static int sms = 0;
  if (!sms) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (sms <= 0) sms = 148;
  }
  const long long tiles = (long long)p.B * p.m_tiles * p.n_tiles;
  if (tiles <= 0) return cudaSuccess;
  if (tiles > 0x7FFFFFFFLL) return cudaErrorInvalidValue;
  cudaError_t e = cudaFuncSetAttribute(proj_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
  if (e != cudaSuccess) return e;
  const int grid = tiles < sms ? (int)tiles : sms;
  proj_kernel<D><<<grid, kProjThreads, C::SMEM, stream>>>(tmX, tmW, p);
  return cudaGetLastError();
}

}  // namespace

int projection_heads_per_tile(int D) {
  switch (D) {
    case 64: return ProjCfg<64>::HPT;
    case 96: return ProjCfg<96>::HPT;
    case 128: return ProjCfg<128>::HPT;
    case 256: return ProjCfg<256>::HPT;
    default: return 0;
  }
}

cudaError_t launch_projection(const ProjParams& p, int D, const CUtensorMap& tmX, const CUtensorMap& tmW,
                              cudaStream_t stream) {
  switch (D) {
    case 64: return launch_proj_d<64>(p, tmX, tmW, stream);
    case 96: return launch_proj_d<96>(p, tmX, tmW, stream);
    case 128: return launch_proj_d<128>(p, tmX, tmW, stream);
    case 256: return launch_proj_d<256>(p, tmX, tmW, stream);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace nsa
