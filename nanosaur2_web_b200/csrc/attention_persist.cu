// Persistent forward attention for head dim 256 (the Gemma3 text encoder's layers, sm_100a).
//
// Same contract and math as attn_fwd_kernel<256> (attention.cu): one 128-row query tile per work
// unit, S double-buffered in tensor memory (S0, S1 and O fill the 512 columns), P written over its
// own S buffer, online softmax with a lazy rescale, causal / window / padding masks and the key-bias
// table.  The difference is the launch: one CTA per SM loops over work units instead of one CTA per
// unit, so TMEM allocation, barrier set-up and the tensor-map prefetch happen once.  The producer
// loads the next unit's Q and first K tiles while the current unit's last P*V run and the softmax
// writes its output.
//
// Work order: unit u = qb_raw * (B * Hq) + (b * Hq + h), with causal query blocks long-first
// (qb = q_blocks - 1 - qb_raw), dealt round-robin (CTA c takes c, c + G, c + 2G, ...), so each CTA
// sees units of falling length, like longest-first list scheduling.
//
// Every role walks the same unit sequence.  Barrier phases are counted across units:
//   * K / V rings: running load indices; S buffers and P halves: the running key-tile index T
//     (buffer T & 1, parity (T >> 1) & 1); o_full[0]: once per P*V (running count);
//   * q_full (Q landed), q_empty (the unit's S MMAs are done with Q), o_full[1] (the unit's last P*V
//     done), o_free (the softmax has read O, so the next unit's first P*V may overwrite it): once
//     per unit with key tiles (units without any are skipped by all roles alike).
// No waiter ever lags two phases: each producer of a phase needs the waiter's earlier progress.
#include "nsa_internal.h"
#include "ptx.cuh"

namespace nsa {

namespace {

constexpr float kLog2eP = 1.4426950408889634f;
constexpr float kRescaleP = 8.0f;   // log2 units: P may reach 2^8 before O is rescaled
constexpr int kKeyBiasP = 1024;     // keys covered by the shared-memory key bias/mask table

// Tile geometry of the persistent one-query-tile kernel: bf16 operands at head dim 256 (Gemma), or
// fp32 operands multiplied as tf32 at head dim 96 (the DiT's fp32 path, tighter than bf16).
template <bool TF32>
struct CfgP {
  static constexpr int D = TF32 ? 96 : 256, BN = 128, NS = 1;
  static constexpr int ESZ = TF32 ? 4 : 2;                   // operand bytes per element
  static constexpr int ROWB = 128;                           // bytes per row of a swizzle block
  static constexpr int BLK = ROWB / ESZ, NB = D / BLK;       // elements per block row, blocks per row
  static constexpr int KMMA = TF32 ? 8 : 16;                 // K of one MMA (32 bytes of a row)
  static constexpr uint32_t SWZ = 2u;                        // 128-byte swizzle
  static constexpr int QBLK_BYTES = kTileM * ROWB;           // [128 rows][BLK]
  static constexpr int KBLK_BYTES = BN * ROWB;
  static constexpr int Q_TILE_BYTES = kTileM * D * ESZ;
  static constexpr int KV_TILE_BYTES = BN * D * ESZ;
  static constexpr int KSTEPS_QK = D / KMMA, KSTEPS_PV = BN / KMMA, PV_HALF0 = 64 / KMMA;
  static constexpr int THREADS = 256;
  static constexpr int NBARS = 4 * NS + 2 + 4 + 2 + 4 + 1;
  static constexpr int SMEM_BYTES = Q_TILE_BYTES + 2 * NS * KV_TILE_BYTES + kKeyBiasP * 4 + NBARS * 8 + 16 + 1024;
  static constexpr uint32_t TMEM_COLS = 512;
  static constexpr uint32_t IDESC_QK = TF32 ? idesc_tf32_f32(128, BN, 0, 0) : idesc_bf16_f32(128, BN, 0, 0);
  static constexpr uint32_t IDESC_PV = TF32 ? idesc_tf32_f32(128, D, 0, 1) : idesc_bf16_f32(128, D, 0, 1);
  static_assert(SMEM_BYTES <= 232448, "shared memory budget");
  static_assert(SMEM_BYTES > 117 * 1024, "one CTA per SM (each allocates all 512 TMEM columns)");
  static_assert(256 + D <= 512, "tensor memory: S0, S1 and O");
  static __device__ __forceinline__ uint32_t s_col(int buf) { return (uint32_t)(buf * BN); }
  static __device__ __forceinline__ uint32_t o_col() { return 256u; }
  static __device__ __forceinline__ uint32_t kmajor_off(int kk, int blk_bytes) {
    constexpr int per_blk = BLK / KMMA;
    return (uint32_t)((kk / per_blk) * blk_bytes + (kk % per_blk) * 32);
  }
};

template <bool TF32>
__device__ __forceinline__ void p_mma_ss(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  if constexpr (TF32) mma_ss_tf32(d, a, b, idesc, acc);
  else mma_ss(d, a, b, idesc, acc);
}
template <bool TF32>
__device__ __forceinline__ void p_mma_ts(uint32_t d, uint32_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  if constexpr (TF32) mma_ts_tf32(d, a, b, idesc, acc);
  else mma_ts(d, a, b, idesc, acc);
}

template <bool TF32>
__device__ __forceinline__ void p_issue_qk(uint32_t d_tmem, uint32_t sq, uint32_t sk) {
  using C = CfgP<TF32>;
#pragma unroll
  for (int kk = 0; kk < C::KSTEPS_QK; ++kk) {
    const uint64_t a = smem_desc(sq + C::kmajor_off(kk, C::QBLK_BYTES), 16, 8 * C::ROWB, C::SWZ);
    const uint64_t b = smem_desc(sk + C::kmajor_off(kk, C::KBLK_BYTES), 16, 8 * C::ROWB, C::SWZ);
    p_mma_ss<TF32>(d_tmem, a, b, C::IDESC_QK, kk > 0 ? 1u : 0u);
  }
}

template <bool TF32>
__device__ __forceinline__ void p_issue_pv_half(uint32_t d_tmem, uint32_t p_tmem, uint32_t sv, bool accumulate,
                                                int half) {
  using C = CfgP<TF32>;
  const int k_begin = half == 0 ? 0 : C::PV_HALF0;
  const int k_end = half == 0 ? C::PV_HALF0 : C::KSTEPS_PV;
#pragma unroll
  for (int kk = k_begin; kk < k_end; ++kk) {
    // V is MN-major: KMMA keys per k-step, head-dim blocks of BLK elements KBLK_BYTES apart; P takes
    // 8 TMEM columns per k-step (16 bf16 keys two to a column, or 8 fp32 keys).  An MN-major tf32
    // operand must use the 128-byte swizzle with 32-byte atoms (layout code 1, 4-row groups 512 bytes
    // apart), which the V map's CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B writes.
    const uint64_t b = smem_desc(sv + (uint32_t)(kk * C::KMMA * C::ROWB), C::KBLK_BYTES, TF32 ? 4 * C::ROWB : 8 * C::ROWB,
                                 TF32 ? 1u : C::SWZ);
    p_mma_ts<TF32>(d_tmem, p_tmem + (uint32_t)(kk * 8), b, C::IDESC_PV, (accumulate || kk > 0) ? 1u : 0u);
  }
}

// One work unit's geometry.
struct Unit {
  int b, bl, hl, hq, hkvl, kv_valid, q_row0, j0, n;
};

__device__ __forceinline__ Unit decode_unit(const AttnParams& p, int u) {
  constexpr int BN = CfgP<false>::BN;
  Unit w;
  const int bh = p.B * p.Hq;
  const int qb_raw = u / bh, rest = u % bh;
  const int qb = p.causal ? (p.q_blocks - 1 - qb_raw) : qb_raw;   // long causal blocks first
  w.hl = rest % p.Hq;
  w.bl = rest / p.Hq;
  w.b = p.b_begin + w.bl;
  w.hq = p.hq_begin + w.hl;
  w.hkvl = w.hq / p.group - p.hkv_begin;
  w.kv_valid = p.kv_len ? min(p.kv_len[w.b], p.Lk) : p.Lk;
  w.q_row0 = qb * kTileM;
  const int q_row_end = min(w.q_row0 + kTileM, p.Lq);
  int kv_end = w.kv_valid;
  if (p.causal) kv_end = min(kv_end, q_row_end);
  const int kv_begin = p.window > 0 ? max(0, w.q_row0 - p.window + 1) : 0;
  w.j0 = kv_begin / BN;
  w.n = kv_end > kv_begin ? ((kv_end - 1) / BN - w.j0 + 1) : 0;
  return w;
}

template <bool TF32>
__global__ void __launch_bounds__(CfgP<TF32>::THREADS, 1)
    attn_persist_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                        const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmVd,
                        const AttnParams p) {
  using C = CfgP<TF32>;
  constexpr int D = C::D, BN = C::BN, NS = C::NS;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;
  uint8_t* sK = sQ + C::Q_TILE_BYTES;
  uint8_t* sV = sK + NS * C::KV_TILE_BYTES;
  float* kb = reinterpret_cast<float*>(sV + NS * C::KV_TILE_BYTES);   // [kKeyBiasP]
  uint64_t* bars = reinterpret_cast<uint64_t*>(kb + kKeyBiasP);
  uint64_t* k_full = bars;               // [NS]
  uint64_t* k_empty = k_full + NS;
  uint64_t* v_full = k_empty + NS;
  uint64_t* v_empty = v_full + NS;
  uint64_t* s_full = v_empty + NS;       // [2] per S buffer
  uint64_t* p_full = s_full + 2;         // [buffer * 2 + half]
  uint64_t* o_full = p_full + 4;         // [0] once per P*V, [1] once per unit (its last P*V)
  uint64_t* q_full = o_full + 2;         // Q of the unit landed
  uint64_t* q_empty = q_full + 1;        // the unit's S MMAs are done with Q
  uint64_t* o_free = q_empty + 1;        // the softmax has read the unit's O (128 arrivals)
  uint64_t* drain = o_free + 1;          // MMA teardown after an abort
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int U = p.B * p.Hq * p.q_blocks;
  const int G = (int)gridDim.x;
  const uint64_t to = p.timeout_ns;

  if (threadIdx.x == 0) {
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
    mbar_init(q_full, 1);
    mbar_init(q_empty, 1);
    mbar_init(o_free, 128);
    mbar_init(drain, 1);
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

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      bool ok = true;
      int gk = 0, gv = 0, ia = 0;   // running K / V loads, active units
      for (int u = blockIdx.x; ok && u < U; u += G) {
        const Unit w = decode_unit(p, u);
        if (w.n == 0) continue;
        const int kv_y0 = w.bl * p.kv_yb + w.hkvl * p.kv_yh;
        const int k_x = p.k_x0 + w.hkvl * p.kv_xh, v_x = p.v_x0 + w.hkvl * p.kv_xh;
        const int vd_x = p.vd_x0 + w.hkvl * p.vd_xh, vd_y0 = w.b * p.vd_yb;
        const int qx = p.q_x0 + (w.hq - p.q_h0) * p.q_xh;
        const int qy = (w.b - p.q_b0) * p.q_yb + (w.hq - p.q_h0) * p.q_yh + w.q_row0;
        if (ia > 0 && !wait_bounded(q_empty, (ia - 1) & 1, abort_flag, p.err, kErrTimeoutLoad, to)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(q_full, C::Q_TILE_BYTES);
        for (int c = 0; c < C::NB; ++c) tma_load_2d(sQ + c * C::QBLK_BYTES, &tmQ, q_full, qx + c * C::BLK, qy);
        auto load_k = [&](int j) -> bool {
          const int s = gk % NS;
          if (gk >= NS && !wait_bounded(&k_empty[s], ((gk / NS) - 1) & 1, abort_flag, p.err, kErrTimeoutLoad, to))
            return false;
          mbar_arrive_expect_tx(&k_full[s], C::KV_TILE_BYTES);
          for (int c = 0; c < C::NB; ++c)
            tma_load_2d(sK + s * C::KV_TILE_BYTES + c * C::KBLK_BYTES, &tmK, &k_full[s], k_x + c * C::BLK,
                        kv_y0 + (w.j0 + j) * BN);
          ++gk;
          return true;
        };
        auto load_v = [&](int j) -> bool {
          const int s = gv % NS;
          if (gv >= NS && !wait_bounded(&v_empty[s], ((gv / NS) - 1) & 1, abort_flag, p.err, kErrTimeoutLoad, to))
            return false;
          mbar_arrive_expect_tx(&v_full[s], C::KV_TILE_BYTES);
          if (p.v_direct && (w.j0 + j + 1) * BN <= w.kv_valid) {
            for (int c = 0; c < C::NB; ++c)
              tma_load_2d(sV + s * C::KV_TILE_BYTES + c * C::KBLK_BYTES, &tmVd, &v_full[s], vd_x + c * C::BLK,
                          vd_y0 + (w.j0 + j) * BN);
          } else {
            for (int c = 0; c < C::NB; ++c)
              tma_load_2d(sV + s * C::KV_TILE_BYTES + c * C::KBLK_BYTES, &tmV, &v_full[s], v_x + c * C::BLK,
                          kv_y0 + (w.j0 + j) * BN);
          }
          ++gv;
          return true;
        };
        // the MMA thread consumes K(0), K(1), then V(j) followed by K(j + 2)
        ok = load_k(0);
        for (int j = 0; ok && j < w.n; ++j) {
          if (j + 1 < w.n) ok = load_k(j + 1);
          if (ok) ok = load_v(j);
        }
        ++ia;
      }
      if (!ok) {
        // bounded wait for the copies already issued, so none lands after the CTA exits
        if (ia > 0 || gk > 0) wait_drain(q_full, ia & 1, 20000000ull);
        if (gk > 0) wait_drain(&k_full[(gk - 1) % NS], ((gk - 1) / NS) & 1, 20000000ull);
        if (gv > 0) wait_drain(&v_full[(gv - 1) % NS], ((gv - 1) / NS) & 1, 20000000ull);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t sq = smem_u32(sQ), sk = smem_u32(sK), sv = smem_u32(sV);
      bool ok = true;
      int gk = 0, gv = 0, ia = 0, T = 0;   // running K / V tiles consumed, active units, key tiles
      auto issue_s = [&](int t_idx, int last) -> bool {   // S(t_idx) into buffer t_idx & 1
        const int s = gk % NS;
        if (!wait_bounded(&k_full[s], (gk / NS) & 1, abort_flag, p.err, kErrTimeoutMma, to)) return false;
        tc_fence_after();
        p_issue_qk<TF32>(tmem + C::s_col(t_idx & 1), sq, sk + (uint32_t)(s * C::KV_TILE_BYTES));
        tc_commit(&s_full[t_idx & 1]);
        tc_commit(&k_empty[s]);
        if (last) tc_commit(q_empty);   // the unit's last S: Q may be replaced
        ++gk;
        return true;
      };
      for (int u = blockIdx.x; ok && u < U; u += G) {
        const Unit w = decode_unit(p, u);
        if (w.n == 0) continue;
        ok = wait_bounded(q_full, ia & 1, abort_flag, p.err, kErrTimeoutMma, to);
        for (int j = 0; ok && j < 2 && j < w.n; ++j) ok = issue_s(T + j, j == w.n - 1);
        for (int j = 0; ok && j < w.n; ++j) {
          const int t = T + j;
          const int s = gv % NS;
          ok = wait_bounded(&v_full[s], (gv / NS) & 1, abort_flag, p.err, kErrTimeoutMma, to);
          // the first P*V overwrites O: the softmax must have read the previous unit's O
          if (ok && j == 0 && ia > 0) ok = wait_bounded(o_free, (ia - 1) & 1, abort_flag, p.err, kErrTimeoutMma, to);
          for (int h = 0; ok && h < 2; ++h) {
            ok = wait_bounded(&p_full[(t & 1) * 2 + h], (t >> 1) & 1, abort_flag, p.err, kErrTimeoutMma, to);
            if (!ok) break;
            tc_fence_after();
            p_issue_pv_half<TF32>(tmem + C::o_col(), tmem + C::s_col(t & 1), sv + (uint32_t)(s * C::KV_TILE_BYTES), j > 0, h);
          }
          if (!ok) break;
          tc_commit(&o_full[0]);
          tc_commit(&v_empty[s]);
          ++gv;
          if (j + 2 < w.n) ok = issue_s(t + 2, j + 2 == w.n - 1);
        }
        if (ok) tc_commit(&o_full[1]);
        T += w.n;
        ++ia;
      }
      if (!ok) {
        // let every MMA already issued finish before the CTA tears down its tensor memory
        tc_commit(drain);
        wait_drain(drain, 0, 20000000ull);
      }
    }
    __syncwarp();
  } else if (warp >= 4) {
    // ------------------------------------------------------------------ softmax + epilogue
    const int quarter = warp % 4;
    const uint32_t lane_base = tmem + ((uint32_t)(quarter * 32) << 16);
    const float sl2 = p.scale_log2;
    bool ok = true;
    int ia = 0, T = 0;
    for (int u = blockIdx.x; ok && u < U; u += G) {
      const Unit w = decode_unit(p, u);
      const int row = w.q_row0 + quarter * 32 + lane;
      const int tile_row0 = w.q_row0;
      const float* bias_b = p.bias ? p.bias + (int64_t)w.b * p.bias_bstride : nullptr;
      // key bias + padding mask table of this unit (the previous unit's loop is done with it)
      asm volatile("bar.sync 1, 128;" ::: "memory");
      int kb0 = min(w.kv_valid, bias_b ? p.bias_start : w.kv_valid);
      kb0 = max(kb0 - kb0 % BN, w.j0 * BN);
      const int kb_end = (w.j0 + w.n) * BN;
      const bool kb_ok = kb_end - kb0 <= kKeyBiasP;
      if (kb_ok) {
        for (int i = threadIdx.x - 128; i < kb_end - kb0; i += 128) {
          const int key = kb0 + i;
          float v = 0.f;
          if (bias_b && key >= p.bias_start && key < p.bias_start + p.bias_len) v = bias_b[key - p.bias_start] * kLog2eP;
          kb[i] = key < w.kv_valid ? v : -INFINITY;
        }
      }
      asm volatile("bar.sync 1, 128;" ::: "memory");
      float m_run = -INFINITY, l_run = 0.f;
      for (int j = 0; ok && j < w.n; ++j) {
        const int t = T + j;
        const int sbuf = t & 1;
        ok = __all_sync(0xffffffffu,
                        wait_bounded(&s_full[sbuf], (uint32_t)((t >> 1) & 1), abort_flag, p.err, kErrTimeoutSoftmax, to));
        if (!ok) break;
        tc_fence_after();
        const int key0 = (w.j0 + j) * BN;
        const bool t_invalid = key0 + BN > w.kv_valid;
        const bool t_causal = p.causal && key0 + BN - 1 > tile_row0;
        const bool t_window = p.window > 0 && key0 <= tile_row0 + kTileM - 1 - p.window;
        const bool t_bias = bias_b != nullptr && key0 + BN > p.bias_start && key0 < p.bias_start + p.bias_len;
        const uint32_t s_addr = lane_base + C::s_col(sbuf);
        float sc = sl2;
        const bool t_table = kb_ok && !t_causal && !t_window && (t_invalid || t_bias);
        if (!t_table && (t_invalid || t_causal || t_window || t_bias)) {
          sc = 1.f;
          const int lo = p.window > 0 ? row - p.window + 1 : 0;              // first visible key
          const int hi = p.causal ? min(w.kv_valid, row + 1) : w.kv_valid;   // one past the last
#pragma unroll 1
          for (int cc = 0; cc < BN / 16; ++cc) {
            uint32_t r[16];
            tmem_ld16(s_addr + (uint32_t)(cc * 16), r);
#pragma unroll
            for (int c = 0; c < 16; ++c) {
              const int key = key0 + cc * 16 + c;
              float v = __uint_as_float(r[c]) * sl2;
              if (t_bias && key >= p.bias_start && key < p.bias_start + p.bias_len)
                v += __ldg(bias_b + (key - p.bias_start)) * kLog2eP;
              r[c] = __float_as_uint(key >= lo && key < hi ? v : -INFINITY);
            }
            tmem_st16(s_addr + (uint32_t)(cc * 16), r);
          }
        }
        float x[BN];
        {
          uint32_t r[BN];
          tmem_ld128(s_addr, r);
#pragma unroll
          for (int c = 0; c < BN; ++c) x[c] = __uint_as_float(r[c]);
        }
        if (t_table) {
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
          const bool need = m_new > m_run + kRescaleP;
          if (__any_sync(0xffffffffu, need)) {
            const float alpha = need ? ex2(m_run - m_new) : 1.f;
            if (need) {
              l_run *= alpha;
              m_run = m_new;
            }
            // O must hold every P*V of the unit up to key tile j - 1 before it is rescaled
            ok = __all_sync(0xffffffffu,
                            wait_bounded(&o_full[0], (uint32_t)((t - 1) & 1), abort_flag, p.err, kErrTimeoutSoftmax, to));
            if (!ok) break;
            tc_fence_after();
            const uint64_t a2 = f2_pack(alpha, alpha);
#pragma unroll 1
            for (int cc = 0; cc < D / 32; ++cc) {
              uint32_t r[32];
              const uint32_t oaddr = lane_base + C::o_col() + (uint32_t)(cc * 32);
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
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          if constexpr (TF32) {
            // keys 64*half .. 64*half+63 -> P columns 64*half .. 64*half+63, fp32 (read as tf32)
            uint32_t pf[64];
#pragma unroll
            for (int c = 0; c < 32; ++c) {
              float y0, y1;
              f2_unpack(f2_fma(f2_pack(x[64 * half + 2 * c], x[64 * half + 2 * c + 1]), sc2, nm2), y0, y1);
              const float a0 = ex2(y0), a1 = ex2(y1);
              ls[c & 3] = f2_add(ls[c & 3], f2_pack(a0, a1));
              pf[2 * c] = __float_as_uint(round_tf32(a0));
              pf[2 * c + 1] = __float_as_uint(round_tf32(a1));
            }
            tmem_st64(s_addr + (uint32_t)(64 * half), pf);
          } else {
            // keys 64*half .. 64*half+63 -> P columns 32*half .. 32*half+31, bf16 pairs
            uint32_t pk[32];
#pragma unroll
            for (int c = 0; c < 32; ++c) {
              float y0, y1;
              f2_unpack(f2_fma(f2_pack(x[64 * half + 2 * c], x[64 * half + 2 * c + 1]), sc2, nm2), y0, y1);
              const float a0 = ex2(y0), a1 = ex2(y1);
              ls[c & 3] = f2_add(ls[c & 3], f2_pack(a0, a1));
              pk[c] = pack_bf16x2(a0, a1);
            }
            tmem_st32(s_addr + (uint32_t)(32 * half), pk);
          }
          tc_fence_before();
          mbar_arrive(&p_full[sbuf * 2 + half]);
        }
        float s0, s1;
        f2_unpack(f2_add(f2_add(ls[0], ls[1]), f2_add(ls[2], ls[3])), s0, s1);
        l_run += s0 + s1;
      }
      if (!ok) break;
      if (w.n > 0) {
        ok = __all_sync(0xffffffffu, wait_bounded(&o_full[1], (uint32_t)(ia & 1), abort_flag, p.err,
                                                  kErrTimeoutSoftmax, to));
        if (!ok) break;
        tc_fence_after();
      }
      const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
      const bool store = row < p.Lq;
      const int64_t obase = (int64_t)w.b * p.out_bstride + (int64_t)row * p.out_ld + p.out_off + (int64_t)w.hq * D;
#pragma unroll 1
      for (int cc = 0; cc < D / 32; ++cc) {
        uint32_t r[32];
        if (w.n > 0) {
          tmem_ld32(lane_base + C::o_col() + (uint32_t)(cc * 32), r);
        } else {
#pragma unroll
          for (int c = 0; c < 32; ++c) r[c] = 0u;
        }
        if (store) {
          if (p.out_f32) {
            float* o = reinterpret_cast<float*>(p.out) + obase + cc * 32;
#pragma unroll
            for (int c = 0; c < 32; c += 4)
              *reinterpret_cast<float4*>(o + c) =
                  make_float4(__uint_as_float(r[c]) * inv, __uint_as_float(r[c + 1]) * inv,
                              __uint_as_float(r[c + 2]) * inv, __uint_as_float(r[c + 3]) * inv);
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
      if (w.n > 0) {
        // O has been read: the next unit's first P*V may overwrite it
        tc_fence_before();
        mbar_arrive(o_free);
        T += w.n;
        ++ia;
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

template <bool TF32>
cudaError_t launch_persist_t(const AttnParams& p, const CUtensorMap& tmQ, const CUtensorMap& tmK,
                             const CUtensorMap& tmV, const CUtensorMap& tmVd, cudaStream_t stream) {
  using C = CfgP<TF32>;
  static DeviceOnce once;
  cudaError_t e = once_per_device(once, [] {
    return cudaFuncSetAttribute(attn_persist_kernel<TF32>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                CfgP<TF32>::SMEM_BYTES);
  });
  if (e != cudaSuccess) return e;
  const int sms = device_sm_count();
  if (p.split_units > 0) return cudaErrorInvalidValue;   // the tail split is for two-tile kernels
  if (TF32 && p.v_direct) return cudaErrorInvalidValue;  // fp32 V tiles come from the prologue
  const long long units = (long long)p.B * p.Hq * p.q_blocks;
  if (units <= 0) return cudaSuccess;
  if (units > 0x7FFFFFFFLL) return cudaErrorInvalidValue;
  const int grid = (int)(units < sms ? units : sms);
  attn_persist_kernel<TF32><<<grid, C::THREADS, C::SMEM_BYTES, stream>>>(tmQ, tmK, tmV, tmVd, p);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_attention_persist(const AttnParams& p, const CUtensorMap& tmQ, const CUtensorMap& tmK,
                                     const CUtensorMap& tmV, const CUtensorMap& tmVd, cudaStream_t stream) {
  return launch_persist_t<false>(p, tmQ, tmK, tmV, tmVd, stream);
}

cudaError_t launch_attention_tf32(const AttnParams& p, const CUtensorMap& tmQ, const CUtensorMap& tmK,
                                  const CUtensorMap& tmV, cudaStream_t stream) {
  return launch_persist_t<true>(p, tmQ, tmK, tmV, tmV, stream);
}

}  // namespace nsa
