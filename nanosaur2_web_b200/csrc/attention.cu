// Fused multi-head attention forward for sm_100a (B200): tcgen05 MMAs accumulating in tensor memory
// for S = Q K^T and O = P V, K/V tiles staged by TMA, online softmax on the CUDA cores with the key
// bias / padding mask / causal and window masks folded into the score tile.
//
// It replaces the reference's fused WGSL flash kernel (app/gpu/kernels.js:132-305: O = softmax(
// s*QK^T + key bias + key mask) V, keys streamed in blocks with an online max/sum) and its unfused
// GEMM + causal softmax + GEMM fallback for Gemma (app/gpu/ops.js:211-241).
//
// One CTA handles one "block" of NQ query tiles of 128 rows for one (batch, query head):
//   warp 0        TMA producer: K/V tiles through NS-deep rings (and Q tiles when Q lives in
//                 shared memory)
//   warp 1        TMEM allocator + MMA issuer (a single thread issues every tcgen05.mma)
//   warps 2-3     idle (they complete the first warpgroup)
//   warps 4..     one softmax warpgroup per query tile.  A warp may only touch the TMEM lane
//                 quarter (warp id % 4), so lane l of warp w owns query row 32*(w%4) + l of its
//                 tile: it reads its score row with tcgen05.ld, writes bf16 probabilities back
//                 into the same TMEM columns, and finally normalises its output row.
// Head dims 64 and 96 (QTMEM): the producer loads the prologue's Q' tiles into shared memory once,
// and each softmax thread copies its own bf16 query row into tensor memory, so S = Q K^T reads
// only K from shared memory.  Tensor memory (512 columns) for D = 96, BN = 112 keys per tile:
//   S0 [0,112) S1 [112,224) O0 [224,320) O1 [320,416) Q0 [416,464) Q1 [464,512)
// D = 64: S 2 x 128, O 2 x 64, Q 2 x 32.  D = 128: Q in shared memory, S 2 x 128, O 2 x 128.
// D = 256 (NQ = 1): Q in shared memory, S double-buffered [0,128) [128,256), O [256,512).
// P (bf16, two per 32-bit column) overwrites the first BN/2 columns of the S buffer it came from.
// The MMA for the next S into a buffer is issued after the P*V MMA that reads it; tcgen05.mma
// operations issued by one thread execute in order.
#include "attn_tiles.cuh"
#include "nsa_internal.h"
#include "ptx.cuh"

namespace nsa {

namespace {

using namespace tiles;

template <int D>
__global__ void __launch_bounds__(Cfg<D>::THREADS, 1)
    attn_fwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                    const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmVd,
                    const AttnParams p) {
  using C = Cfg<D>;
  constexpr int NQ = C::NQ, NS = C::NS, BN = C::BN;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;
  uint8_t* sK = sQ + NQ * C::Q_TILE_BYTES;
  uint8_t* sV = sK + NS * C::KV_TILE_BYTES;
  float* kb = reinterpret_cast<float*>(sV + NS * C::KV_TILE_BYTES);   // [kKeyBiasMax]
  uint64_t* bars = reinterpret_cast<uint64_t*>(kb + kKeyBiasMax);
  uint64_t* q_full = bars;           // [2]   Q ready for the MMA (QTMEM: rows stored in TMEM)
  uint64_t* q_smem = bars + 2;       //       Q tile(s) landed in shared memory (QTMEM)
  uint64_t* k_full = bars + 3;
  uint64_t* k_empty = k_full + NS;
  uint64_t* v_full = k_empty + NS;
  uint64_t* v_empty = v_full + NS;
  uint64_t* s_full = v_empty + NS;   // [2]   S buffer ready
  uint64_t* p_full = s_full + 2;     // [4]   P half ready: [buffer * 2 + half], buffer = tile (NQ = 2)
                                     //       or S buffer j & 1 (NQ = 1)
  uint64_t* o_full = p_full + 4;     // [2]   O complete (NQ = 1: [0] once per P*V, [1] after the last)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(o_full + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* split_arrival = reinterpret_cast<volatile int*>(tmem_slot + 2);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;

  // ---- work unit: (batch, query head, query block); units of the split tail run as two CTAs,
  // one per half of the unit's key tiles (split_half 0 / 1)
  int unit = (int)blockIdx.x, split_half = -1, split_idx = 0;
  if (p.split_units > 0 && unit >= p.split_first) {
    split_idx = (unit - p.split_first) >> 1;
    split_half = (unit - p.split_first) & 1;
    unit = p.split_first + split_idx;
  }
  const int qb_raw = unit % p.q_blocks;
  const int rest = unit / p.q_blocks;
  const int qb = p.causal ? (p.q_blocks - 1 - qb_raw) : qb_raw;   // long causal blocks first
  const int hl = rest % p.Hq;
  const int bl = rest / p.Hq;
  const int b = p.b_begin + bl;
  const int hkvl = (p.hq_begin + hl) / p.group - p.hkv_begin;
  const int kv_valid = p.kv_len ? min(p.kv_len[b], p.Lk) : p.Lk;
  const int q_row0 = qb * NQ * kTileM;
  const int q_row_end = min(q_row0 + NQ * kTileM, p.Lq);
  int kv_end = kv_valid;
  if (p.causal) kv_end = min(kv_end, q_row_end);
  const int kv_begin = p.window > 0 ? max(0, q_row0 - p.window + 1) : 0;
  int j0 = kv_begin / BN;
  int n = kv_end > kv_begin ? ((kv_end - 1) / BN - j0 + 1) : 0;
  if (split_half >= 0) {
    const int n_first = n / 2;
    if (split_half == 0) {
      n = n_first;
    } else {
      j0 += n_first;
      n -= n_first;
    }
  }
  const int q_tma_row = (bl * p.Hq + hl) * p.Lq_pad + q_row0;
  const int kv_y0 = bl * p.kv_yb + hkvl * p.kv_yh;
  const int k_x = p.k_x0 + hkvl * p.kv_xh, v_x = p.v_x0 + hkvl * p.kv_xh;
  const int vd_x = p.vd_x0 + hkvl * p.vd_xh, vd_y0 = b * p.vd_yb;
  const uint64_t to = p.timeout_ns;

  if (threadIdx.x == 0) {
    mbar_init(&q_full[0], C::QTMEM ? 128 : 1);
    mbar_init(&q_full[1], C::QTMEM ? 128 : 1);
    mbar_init(q_smem, 1);
    for (int s = 0; s < NS; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&k_empty[s], 1);
      mbar_init(&v_full[s], 1);
      mbar_init(&v_empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&o_full[i], 1);
    }
    for (int i = 0; i < 4; ++i) mbar_init(&p_full[i], 128);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
    if (p.v_direct) tma_prefetch_desc(&tmVd);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if constexpr (NQ == 2) {
    if (warp < 4) reg_dealloc<C::REG_CTRL>();
  }
  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0 && n > 0) {
      bool ok = true;
      if constexpr (!C::QTMEM) {
        mbar_arrive_expect_tx(&q_full[0], NQ * C::Q_TILE_BYTES);
        for (int i = 0; i < NQ; ++i)
          for (int c = 0; c < C::NB; ++c)
            tma_load_2d(sQ + i * C::Q_TILE_BYTES + c * C::QBLK_BYTES, &tmQ, &q_full[0], c * C::BLK,
                        q_tma_row + i * kTileM);
      } else {
        // the Q' rows of this block; the softmax threads copy them into tensor memory
        const int hq = p.hq_begin + hl;
        const int qx = p.q_x0 + (hq - p.q_h0) * p.q_xh;
        const int qy = (b - p.q_b0) * p.q_yb + (hq - p.q_h0) * p.q_yh + q_row0;
        mbar_arrive_expect_tx(q_smem, NQ * C::Q_TILE_BYTES);
        for (int i = 0; i < NQ; ++i)
          for (int c = 0; c < C::NB; ++c)
            tma_load_2d(sQ + i * C::Q_TILE_BYTES + c * C::QBLK_BYTES, &tmQ, q_smem, qx + c * C::BLK, qy + i * kTileM);
      }
      auto load_k = [&](int j) -> bool {
        const int s = j % NS;
        if (j >= NS && !wait_bounded(&k_empty[s], ((j / NS) - 1) & 1, abort_flag, p.err, kErrTimeoutLoad, to))
          return false;
        mbar_arrive_expect_tx(&k_full[s], C::KV_TILE_BYTES);
        for (int c = 0; c < C::NB; ++c)
          tma_load_2d(sK + s * C::KV_TILE_BYTES + c * C::KBLK_BYTES, &tmK, &k_full[s], k_x + c * C::BLK,
                      kv_y0 + (j0 + j) * BN);
        return true;
      };
      auto load_v = [&](int j) -> bool {
        const int s = j % NS;
        if (j >= NS && !wait_bounded(&v_empty[s], ((j / NS) - 1) & 1, abort_flag, p.err, kErrTimeoutLoad, to))
          return false;
        mbar_arrive_expect_tx(&v_full[s], C::KV_TILE_BYTES);
        if (p.v_direct && (j0 + j + 1) * BN <= kv_valid) {
          // a tile of valid keys only: straight from the input rows
          for (int c = 0; c < C::NB; ++c)
            tma_load_2d(sV + s * C::KV_TILE_BYTES + c * C::KBLK_BYTES, &tmVd, &v_full[s], vd_x + c * C::BLK,
                        vd_y0 + (j0 + j) * BN);
        } else {
          for (int c = 0; c < C::NB; ++c)
            tma_load_2d(sV + s * C::KV_TILE_BYTES + c * C::KBLK_BYTES, &tmV, &v_full[s], v_x + c * C::BLK,
                        kv_y0 + (j0 + j) * BN);
        }
        return true;
      };
      int k_issued = 0, v_issued = 0;
      ok = load_k(0);
      if (ok) k_issued = 1;
      for (int j = 0; ok && j < n; ++j) {
        if (j + 1 < n) {
          ok = load_k(j + 1);
          if (ok) k_issued = j + 2;
        }
        if (ok) ok = load_v(j);
        if (ok) v_issued = j + 1;
      }
      // On an abort, wait (bounded) for the copies already issued so none lands after exit:
      // the latest issue into each stage completes after the earlier ones.
      if (!ok) {
        wait_drain(C::QTMEM ? q_smem : &q_full[0], 0, 20000000ull);
        for (int j = k_issued - 1; j >= 0 && j >= k_issued - NS; --j) wait_drain(&k_full[j % NS], (j / NS) & 1, 20000000ull);
        for (int j = v_issued - 1; j >= 0 && j >= v_issued - NS; --j) wait_drain(&v_full[j % NS], (j / NS) & 1, 20000000ull);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0 && n > 0) {
      const uint32_t sk = smem_u32(sK), sv = smem_u32(sV);
      // Q source of tile i: TMEM columns (QTMEM) or the shared-memory tile
      auto q_src = [&](int i) -> uint32_t {
        return C::QTMEM ? tmem + C::q_col(i) : smem_u32(sQ) + (uint32_t)(i * C::Q_TILE_BYTES);
      };
      bool ok = true;
      if constexpr (C::QTMEM) {
        ok = wait_bounded(&q_full[0], 0, abort_flag, p.err, kErrTimeoutMma, to) &&
             (NQ == 1 || wait_bounded(&q_full[1], 0, abort_flag, p.err, kErrTimeoutMma, to));
      } else {
        ok = wait_bounded(&q_full[0], 0, abort_flag, p.err, kErrTimeoutMma, to);
      }
      tc_fence_after();
      if constexpr (NQ == 2) {
        if (ok) ok = wait_bounded(&k_full[0], 0, abort_flag, p.err, kErrTimeoutMma, to);
        if (ok) {
          tc_fence_after();
          issue_qk<D>(tmem + C::s_col(0), q_src(0), sk);
          tc_commit(&s_full[0]);
          issue_qk<D>(tmem + C::s_col(1), q_src(1), sk);
          tc_commit(&s_full[1]);
          tc_commit(&k_empty[0]);
        }
        // P*V of tile i for key tile jj, half by half as the softmax hands P over
        auto pv = [&](int i, int jj, int svs) -> bool {
          for (int h = 0; h < 2; ++h) {
            if (!wait_bounded(&p_full[i * 2 + h], jj & 1, abort_flag, p.err, kErrTimeoutMma, to)) return false;
            tc_fence_after();
            issue_pv_half<D>(tmem + C::o_col(i), tmem + C::s_col(i), sv + svs * C::KV_TILE_BYTES, jj > 0, h);
          }
          return true;
        };
        for (int j = 1; ok && j < n; ++j) {
          const int svs = (j - 1) % NS, sks = j % NS;
          ok = wait_bounded(&v_full[svs], ((j - 1) / NS) & 1, abort_flag, p.err, kErrTimeoutMma, to) && pv(0, j - 1, svs);
          if (!ok) break;
          ok = wait_bounded(&k_full[sks], (j / NS) & 1, abort_flag, p.err, kErrTimeoutMma, to);
          if (!ok) break;
          tc_fence_after();
          issue_qk<D>(tmem + C::s_col(0), q_src(0), sk + sks * C::KV_TILE_BYTES);
          tc_commit(&s_full[0]);
          ok = pv(1, j - 1, svs);
          if (!ok) break;
          tc_commit(&v_empty[svs]);
          issue_qk<D>(tmem + C::s_col(1), q_src(1), sk + sks * C::KV_TILE_BYTES);
          tc_commit(&s_full[1]);
          tc_commit(&k_empty[sks]);
        }
        if (ok) {
          const int svs = (n - 1) % NS;
          ok = wait_bounded(&v_full[svs], ((n - 1) / NS) & 1, abort_flag, p.err, kErrTimeoutMma, to);
          for (int i = 0; ok && i < 2; ++i) {
            ok = pv(i, n - 1, svs);
            if (ok) tc_commit(&o_full[i]);
          }
          if (ok) tc_commit(&v_empty[svs]);
        }
      } else {
        // one query tile, S double-buffered: S(0), S(1), then PV(j) followed by S(j+2)
        for (int j = 0; ok && j < 2 && j < n; ++j) {
          ok = wait_bounded(&k_full[j % NS], (j / NS) & 1, abort_flag, p.err, kErrTimeoutMma, to);
          if (!ok) break;
          tc_fence_after();
          issue_qk<D>(tmem + C::s_col(j & 1), q_src(0), sk + (j % NS) * C::KV_TILE_BYTES);
          tc_commit(&s_full[j & 1]);
          tc_commit(&k_empty[j % NS]);
        }
        for (int j = 0; ok && j < n; ++j) {
          const int svs = j % NS;
          ok = wait_bounded(&v_full[svs], (j / NS) & 1, abort_flag, p.err, kErrTimeoutMma, to);
          for (int h = 0; ok && h < 2; ++h) {
            // one barrier pair per S buffer: the softmax may hand over P(j + 1) before this wait
            // for P(j) runs, but never P(j + 2), whose S is issued only after this P*V
            ok = wait_bounded(&p_full[(j & 1) * 2 + h], (j >> 1) & 1, abort_flag, p.err, kErrTimeoutMma, to);
            if (!ok) break;
            tc_fence_after();
            issue_pv_half<D>(tmem + C::o_col(0), tmem + C::s_col(j & 1), sv + svs * C::KV_TILE_BYTES, j > 0, h);
          }
          if (!ok) break;
          tc_commit(&o_full[0]);
          tc_commit(&v_empty[svs]);
          if (j + 2 < n) {
            const int sks = (j + 2) % NS;
            ok = wait_bounded(&k_full[sks], ((j + 2) / NS) & 1, abort_flag, p.err, kErrTimeoutMma, to);
            if (!ok) break;
            tc_fence_after();
            issue_qk<D>(tmem + C::s_col(j & 1), q_src(0), sk + sks * C::KV_TILE_BYTES);
            tc_commit(&s_full[j & 1]);
            tc_commit(&k_empty[sks]);
          }
        }
        if (ok) tc_commit(&o_full[1]);   // every P*V done: the epilogue's barrier
      }
      if (!ok) {
        // let every MMA already issued finish before the CTA tears down its tensor memory
        // (o_full[1] is the last barrier the normal path arrives on, so it is still in phase 0)
        tc_commit(&o_full[1]);
        wait_drain(&o_full[1], 0, 20000000ull);
      }
    }
    __syncwarp();
  } else if (warp >= 4) {
    // ------------------------------------------------------------------ softmax + epilogue
    if constexpr (NQ == 2) reg_alloc<C::REG_SOFTMAX>();
    const int tile = (warp - 4) / 4;
    const int quarter = warp % 4;
    const int row = q_row0 + tile * kTileM + quarter * 32 + lane;
    const int tile_row0 = q_row0 + tile * kTileM;
    const uint32_t lane_base = tmem + ((uint32_t)(quarter * 32) << 16);
    const float sl2 = p.scale_log2;
    const float* bias_b = p.bias ? p.bias + (int64_t)b * p.bias_bstride : nullptr;
    // Key bias + padding mask of the tiles that need one, in log2 units, for keys [kb0, kb0 +
    // kKeyBiasMax): 0 for plain keys, log(w)*log2(e) for biased text keys, -inf past kv_valid.
    // Built once per CTA by the softmax threads (named barrier 1 over them).
    int kb0 = min(kv_valid, bias_b ? p.bias_start : kv_valid);
    kb0 = max(kb0 - kb0 % BN, j0 * BN);
    const int kb_end = (j0 + n) * BN;
    const bool kb_ok = kb_end - kb0 <= kKeyBiasMax;
    if (kb_ok) {
      for (int i = threadIdx.x - 128; i < kb_end - kb0; i += NQ * 128) {
        const int key = kb0 + i;
        float v = 0.f;
        if (bias_b && key >= p.bias_start && key < p.bias_start + p.bias_len) v = bias_b[key - p.bias_start] * kLog2e;
        kb[i] = key < kv_valid ? v : -INFINITY;
      }
    }
    asm volatile("bar.sync 1, %0;" ::"n"(NQ * 128) : "memory");
    bool ok = true;
    if constexpr (C::QTMEM) {
      // this thread's query row into the Q columns of its TMEM lane
      if (n > 0) {
        ok = __all_sync(0xffffffffu, wait_bounded(q_smem, 0, abort_flag, p.err, kErrTimeoutSoftmax, to));
        if (ok) {
          uint32_t qp[D / 2];
          q_row_from_smem<D>(sQ + tile * C::Q_TILE_BYTES, quarter * 32 + lane, qp);
          tmem_st_n<D / 2>(lane_base + C::q_col(tile), qp);
          tc_fence_before();
          mbar_arrive(&q_full[tile]);
        }
      }
    }
    float m_run = -INFINITY, l_run = 0.f;
    for (int j = 0; ok && j < n; ++j) {
      const int sbuf = NQ == 2 ? tile : (j & 1);
      const uint32_t sparity = NQ == 2 ? (uint32_t)(j & 1) : (uint32_t)((j >> 1) & 1);
      ok = __all_sync(0xffffffffu, wait_bounded(&s_full[sbuf], sparity, abort_flag, p.err, kErrTimeoutSoftmax, to));
      if (!ok) break;
      tc_fence_after();
      const int key0 = (j0 + j) * BN;
      const bool t_invalid = key0 + BN > kv_valid;
      const bool t_causal = p.causal && key0 + BN - 1 > tile_row0;
      const bool t_window = p.window > 0 && key0 <= tile_row0 + kTileM - 1 - p.window;
      const bool t_bias = bias_b != nullptr && key0 + BN > p.bias_start && key0 < p.bias_start + p.bias_len;
      const uint32_t s_addr = lane_base + C::s_col(sbuf);
      // Unmasked tiles keep the raw scores and fold the scale into the exponent.  Tiles with a text
      // bias or padding take the bias / -inf from the shared table; tiles on a causal or window
      // edge (or beyond the table) are first rewritten in TMEM, 16 columns at a time, into scaled,
      // biased, masked logits.  Both then use a unit scale.
      float sc = sl2;
      const bool t_table = kb_ok && !t_causal && !t_window && (t_invalid || t_bias);
      if (!t_table && (t_invalid || t_causal || t_window || t_bias)) {
        sc = 1.f;
        const int lo = p.window > 0 ? row - p.window + 1 : 0;            // first visible key
        const int hi = p.causal ? min(kv_valid, row + 1) : kv_valid;     // one past the last
#pragma unroll 1
        for (int cc = 0; cc < BN / 16; ++cc) {
          uint32_t r[16];
          tmem_ld16(s_addr + (uint32_t)(cc * 16), r);
#pragma unroll
          for (int c = 0; c < 16; ++c) {
            const int key = key0 + cc * 16 + c;
            float v = __uint_as_float(r[c]) * sl2;
            if (t_bias && key >= p.bias_start && key < p.bias_start + p.bias_len)
              v += __ldg(bias_b + (key - p.bias_start)) * kLog2e;
            r[c] = __float_as_uint(key >= lo && key < hi ? v : -INFINITY);
          }
          tmem_st16(s_addr + (uint32_t)(cc * 16), r);
        }
      }
      float x[BN];
      {
        uint32_t r[BN];
        tmem_ld_n<BN>(s_addr, r);
#pragma unroll
        for (int c = 0; c < BN; ++c) x[c] = __uint_as_float(r[c]);
      }
      if (t_table) {
        // scaled logits + key bias / -inf from the shared table (broadcast reads)
        sc = 1.f;
        const float4* kt = reinterpret_cast<const float4*>(kb + (key0 - kb0));
        const uint64_t sl2x2 = f2_pack(sl2, sl2);
#pragma unroll
        for (int c = 0; c < BN; c += 4) {
          const float4 kv4 = kt[c / 4];
          f2_unpack(f2_fma(f2_pack(x[c], x[c + 1]), sl2x2, f2_pack(kv4.x, kv4.y)), x[c], x[c + 1]);
          f2_unpack(f2_fma(f2_pack(x[c + 2], x[c + 3]), sl2x2, f2_pack(kv4.z, kv4.w)), x[c + 2], x[c + 3]);
        }
      }
      float mx[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) mx[k] = fmaxf(x[2 * k], x[2 * k + 1]);
#pragma unroll
      for (int c = 8; c < BN; c += 8) {
#pragma unroll
        for (int k = 0; k < 4; ++k) mx[k] = fmax3(mx[k], x[c + 2 * k], x[c + 2 * k + 1]);
      }
      const float tmax = fmax3(mx[0], mx[1], fmaxf(mx[2], mx[3])) * sc;
      const float m_new = fmaxf(m_run, tmax);
      if (j == 0) {
        m_run = m_new;
      } else {
        const bool need = m_new > m_run + kRescaleThreshold;
        if (__any_sync(0xffffffffu, need)) {
          const float alpha = need ? ex2(m_run - m_new) : 1.f;
          if (need) {
            l_run *= alpha;
            m_run = m_new;
          }
          if constexpr (NQ == 1) {
            // O must hold every P*V up to tile j-1 before it is rescaled
            ok = __all_sync(0xffffffffu,
                            wait_bounded(&o_full[0], (uint32_t)((j - 1) & 1), abort_flag, p.err, kErrTimeoutSoftmax, to));
            if (!ok) break;
            tc_fence_after();
          }
          const uint64_t a2 = f2_pack(alpha, alpha);
#pragma unroll 1
          for (int cc = 0; cc < D / 32; ++cc) {
            uint32_t r[32];
            const uint32_t oaddr = lane_base + C::o_col(tile) + (uint32_t)(cc * 32);
            tmem_ld32(oaddr, r);
#pragma unroll
            for (int c = 0; c < 32; c += 2) {
              float lo, hi;
              f2_unpack(f2_mul(f2_pack(__uint_as_float(r[c]), __uint_as_float(r[c + 1])), a2), lo, hi);
              r[c] = __float_as_uint(lo);
              r[c + 1] = __float_as_uint(hi);
            }
            tmem_st32(oaddr, r);
          }
        }
      }
      const float neg_m = m_run == -INFINITY ? 0.f : -m_run;
      const uint64_t sc2 = f2_pack(sc, sc), nm2 = f2_pack(neg_m, neg_m);
      uint64_t ls[4] = {0ull, 0ull, 0ull, 0ull};
      {
        // keys 0..63 -> P columns 0..31
        uint32_t pk[32];
#pragma unroll
        for (int c = 0; c < 32; ++c) {
          float y0, y1;
          f2_unpack(f2_fma(f2_pack(x[2 * c], x[2 * c + 1]), sc2, nm2), y0, y1);
          const float a0 = ex2(y0), a1 = ex2(y1);
          ls[c & 3] = f2_add(ls[c & 3], f2_pack(a0, a1));
          pk[c] = pack_bf16x2(a0, a1);
        }
        tmem_st32(s_addr, pk);
        tc_fence_before();
        mbar_arrive(&p_full[sbuf * 2]);
      }
      {
        // keys 64..BN-1 -> P columns 32..BN/2-1
        uint32_t pk[C::P1_COLS];
#pragma unroll
        for (int c = 0; c < C::P1_COLS; ++c) {
          float y0, y1;
          f2_unpack(f2_fma(f2_pack(x[64 + 2 * c], x[64 + 2 * c + 1]), sc2, nm2), y0, y1);
          const float a0 = ex2(y0), a1 = ex2(y1);
          ls[c & 3] = f2_add(ls[c & 3], f2_pack(a0, a1));
          pk[c] = pack_bf16x2(a0, a1);
        }
        tmem_st_n<C::P1_COLS>(s_addr + 32u, pk);
        tc_fence_before();
        mbar_arrive(&p_full[sbuf * 2 + 1]);
      }
      {
        float s0, s1;
        f2_unpack(f2_add(f2_add(ls[0], ls[1]), f2_add(ls[2], ls[3])), s0, s1);
        l_run += s0 + s1;
      }
    }
    if (ok && n > 0) {
      if constexpr (NQ == 2) {
        ok = wait_bounded(&o_full[tile], 0, abort_flag, p.err, kErrTimeoutSoftmax, to);
      } else {
        // o_full[0] completes once per P*V and may be up to two phases ahead of this thread here,
        // which a parity wait cannot tell apart; the issuer commits o_full[1] once, after the last
        // P*V, for this wait.
        ok = wait_bounded(&o_full[1], 0, abort_flag, p.err, kErrTimeoutSoftmax, to);
      }
      ok = __all_sync(0xffffffffu, ok);
      if (ok) tc_fence_after();
    }
    // Tail split: publish this half's unnormalised O and (m, l); the CTA that finishes second
    // merges both halves (O = (O_a 2^(m_a - m) + O_b 2^(m_b - m)) / (l_a 2^(m_a - m) + l_b 2^(m_b - m))).
    // The go / no-go is CTA-uniform over the softmax threads (bar.red), because the hand-off below
    // uses named barriers that every one of them must reach.
    const bool split_ok = split_half >= 0 && bar_and_pred<1, NQ * 128>(ok);
    if (split_ok) {
      const int urow = tile * kTileM + quarter * 32 + lane;   // row within the unit
      const int64_t mine = ((int64_t)split_idx * 2 + split_half) * (NQ * kTileM) + urow;
      const int64_t other = ((int64_t)split_idx * 2 + (split_half ^ 1)) * (NQ * kTileM) + urow;
#pragma unroll 1
      for (int cc = 0; cc < D / 32; ++cc) {
        uint32_t r[32];
        if (n > 0) {
          tmem_ld32(lane_base + C::o_col(tile) + (uint32_t)(cc * 32), r);
        } else {
#pragma unroll
          for (int c = 0; c < 32; ++c) r[c] = 0u;
        }
        float4* po = reinterpret_cast<float4*>(p.part_o + mine * D + cc * 32);
#pragma unroll
        for (int c = 0; c < 8; ++c)
          po[c] = make_float4(__uint_as_float(r[4 * c]), __uint_as_float(r[4 * c + 1]), __uint_as_float(r[4 * c + 2]),
                              __uint_as_float(r[4 * c + 3]));
      }
      *reinterpret_cast<float2*>(p.part_ml + mine * 2) = make_float2(m_run, l_run);
      __threadfence();
      asm volatile("bar.sync 1, %0;" ::"n"(NQ * 128) : "memory");
      if (threadIdx.x == 128) *split_arrival = atomicAdd(&p.split_count[split_idx], 1);
      asm volatile("bar.sync 1, %0;" ::"n"(NQ * 128) : "memory");
      if (*split_arrival == 1) {
        __threadfence();
        // Merged in a fixed order, the first half's terms first, whichever CTA finished last: the
        // output then does not depend on which half that was.
        const int64_t first = split_half == 0 ? mine : other, second = split_half == 0 ? other : mine;
        const float2 ml0 = __ldcg(reinterpret_cast<const float2*>(p.part_ml + first * 2));
        const float2 ml1 = __ldcg(reinterpret_cast<const float2*>(p.part_ml + second * 2));
        const float m = fmaxf(ml0.x, ml1.x);
        const float w0 = ml0.x == -INFINITY ? 0.f : ex2(ml0.x - m);
        const float w1 = ml1.x == -INFINITY ? 0.f : ex2(ml1.x - m);
        const float l = ml0.y * w0 + ml1.y * w1;
        const float inv = l > 0.f ? 1.f / l : 0.f;
        const float a0 = w0 * inv, a1 = w1 * inv;
        const bool store = row < p.Lq;
        const int64_t obase = (int64_t)b * p.out_bstride + (int64_t)row * p.out_ld + p.out_off +
                              (int64_t)(p.hq_begin + hl) * D;
#pragma unroll 1
        for (int cc = 0; cc < D / 32; ++cc) {
          float v[32];
          const float4* p0 = reinterpret_cast<const float4*>(p.part_o + first * D + cc * 32);
          const float4* p1 = reinterpret_cast<const float4*>(p.part_o + second * D + cc * 32);
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            const float4 x0 = __ldcg(p0 + c), x1 = __ldcg(p1 + c);
            v[4 * c] = x0.x * a0 + x1.x * a1;
            v[4 * c + 1] = x0.y * a0 + x1.y * a1;
            v[4 * c + 2] = x0.z * a0 + x1.z * a1;
            v[4 * c + 3] = x0.w * a0 + x1.w * a1;
          }
          if (store) {
            if (p.out_f32) {
              float4* o = reinterpret_cast<float4*>(reinterpret_cast<float*>(p.out) + obase + cc * 32);
#pragma unroll
              for (int c = 0; c < 8; ++c) o[c] = make_float4(v[4 * c], v[4 * c + 1], v[4 * c + 2], v[4 * c + 3]);
            } else {
              uint4* o = reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(p.out) + obase + cc * 32);
#pragma unroll
              for (int c = 0; c < 4; ++c)
                o[c] = make_uint4(pack_bf16x2(v[8 * c], v[8 * c + 1]), pack_bf16x2(v[8 * c + 2], v[8 * c + 3]),
                                  pack_bf16x2(v[8 * c + 4], v[8 * c + 5]), pack_bf16x2(v[8 * c + 6], v[8 * c + 7]));
            }
          }
        }
        if (threadIdx.x == 128) p.split_count[split_idx] = 0;   // ready for the next launch
      }
    } else if (ok && split_half < 0) {
      const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
      const bool store = row < p.Lq;
      const int64_t obase = (int64_t)b * p.out_bstride + (int64_t)row * p.out_ld + p.out_off +
                            (int64_t)(p.hq_begin + hl) * D;
#pragma unroll 1
      for (int cc = 0; cc < D / 32; ++cc) {
        uint32_t r[32];
        if (n > 0) {
          tmem_ld32(lane_base + C::o_col(tile) + (uint32_t)(cc * 32), r);
        } else {
#pragma unroll
          for (int c = 0; c < 32; ++c) r[c] = 0u;
        }
        if (store) {
          if (p.out_f32) {
            float* o = reinterpret_cast<float*>(p.out) + obase + cc * 32;
#pragma unroll
            for (int c = 0; c < 32; c += 4) {
              float4 v = make_float4(__uint_as_float(r[c]) * inv, __uint_as_float(r[c + 1]) * inv,
                                     __uint_as_float(r[c + 2]) * inv, __uint_as_float(r[c + 3]) * inv);
              *reinterpret_cast<float4*>(o + c) = v;
            }
          } else {
            __nv_bfloat16* o = reinterpret_cast<__nv_bfloat16*>(p.out) + obase + cc * 32;
#pragma unroll
            for (int c = 0; c < 32; c += 8) {
              uint4 v;
              v.x = pack_bf16x2(__uint_as_float(r[c]) * inv, __uint_as_float(r[c + 1]) * inv);
              v.y = pack_bf16x2(__uint_as_float(r[c + 2]) * inv, __uint_as_float(r[c + 3]) * inv);
              v.z = pack_bf16x2(__uint_as_float(r[c + 4]) * inv, __uint_as_float(r[c + 5]) * inv);
              v.w = pack_bf16x2(__uint_as_float(r[c + 6]) * inv, __uint_as_float(r[c + 7]) * inv);
              *reinterpret_cast<uint4*>(o + c) = v;
            }
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
}

template <int D>
cudaError_t setup_d() {
  using C = Cfg<D>;
  cudaError_t e = cudaFuncSetAttribute(attn_fwd_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM_BYTES);
  if (e != cudaSuccess) return e;
  if constexpr (C::NQ == 2) {
    // The setmaxnreg split is only safe if the kernel really launches with REG_LAUNCH registers
    // per thread; anything else could make setmaxnreg.inc wait forever, so refuse to launch.
    cudaFuncAttributes attr;
    e = cudaFuncGetAttributes(&attr, attn_fwd_kernel<D>);
    if (e != cudaSuccess) return e;
    if (attr.numRegs != C::REG_LAUNCH) return cudaErrorInvalidConfiguration;
  }
  return cudaSuccess;
}

template <int D>
cudaError_t launch_d(const AttnParams& p, const CUtensorMap& tmQ, const CUtensorMap& tmK, const CUtensorMap& tmV,
                     const CUtensorMap& tmVd, cudaStream_t stream) {
  using C = Cfg<D>;
  static DeviceOnce once;   // the attribute is set (and the register count checked) once per device
  cudaError_t e = once_per_device(once, &setup_d<D>);
  if (e != cudaSuccess) return e;
  long long blocks = (long long)p.B * p.Hq * p.q_blocks;
  if (p.split_units > 0) {
    // the split tail: split_units units from split_first on, two CTAs each
    if (C::NQ != 2 || p.causal || p.window || p.split_first + p.split_units != blocks) return cudaErrorInvalidValue;
    blocks += p.split_units;
  }
  if (blocks <= 0) return cudaSuccess;
  if (blocks > 0x7FFFFFFFLL) return cudaErrorInvalidValue;
  attn_fwd_kernel<D><<<(unsigned)blocks, C::THREADS, C::SMEM_BYTES, stream>>>(tmQ, tmK, tmV, tmVd, p);
  return cudaGetLastError();
}

}  // namespace

// Head dim 256 runs the persistent kernel of attention_persist.cu unless built with
// NSA_PERSIST_256=0.
#ifndef NSA_PERSIST_256
#define NSA_PERSIST_256 1
#endif

AttnGeometry attention_geometry(int D) {
  switch (D) {
    case 64: return {Cfg<64>::NQ, Cfg<64>::BN, Cfg<64>::BLK, Cfg<64>::QTMEM, Cfg<64>::BN, true};
    case 96: return {Cfg<96>::NQ, Cfg<96>::BN, Cfg<96>::BLK, Cfg<96>::QTMEM, Cfg<96>::BN, true};
    case 128: return {Cfg<128>::NQ, Cfg<128>::BN, Cfg<128>::BLK, Cfg<128>::QTMEM, Cfg<128>::BN, true};
    case 256: return {Cfg<256>::NQ, Cfg<256>::BN, Cfg<256>::BLK, Cfg<256>::QTMEM, Cfg<256>::BN, true};
    case 512: return {1, 128, 64, false, attention_d512_v_box_rows(), false};
    default: return {0, 0, 0, false, 0, false};
  }
}

cudaError_t launch_attention(const AttnParams& p, int D, const CUtensorMap& tmQ, const CUtensorMap& tmK,
                             const CUtensorMap& tmV, const CUtensorMap& tmVd, cudaStream_t stream) {
  switch (D) {
    case 64: return launch_d<64>(p, tmQ, tmK, tmV, tmVd, stream);
    case 96: return launch_d<96>(p, tmQ, tmK, tmV, tmVd, stream);
    case 128: return launch_d<128>(p, tmQ, tmK, tmV, tmVd, stream);
    case 256: return NSA_PERSIST_256 ? launch_attention_persist(p, tmQ, tmK, tmV, tmVd, stream)
                                     : launch_d<256>(p, tmQ, tmK, tmV, tmVd, stream);
    case 512: return launch_attention_d512(p, tmQ, tmK, tmV, stream);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace nsa
