// Persistent forward attention with two 128-row query tiles per work unit, head dims 64 and 96 (the
// DiT's joint and image-only attention; sm_100a).
//
// Same contract and math as attn_fwd_kernel<D> (attention.cu): Q in tensor memory, S = Q K^T and
// O += P V as tcgen05 MMAs, the two query tiles' softmax warpgroups alternating on the tensor core,
// P written over its own S columns, online softmax with a lazy rescale, the key-bias / padding /
// causal / window masks.  The difference is the launch: one CTA per SM loops over work items, so
// tensor memory, barriers and tensor maps are set up once per SM instead of once per unit, and an
// item's start overlaps the previous item's end:
//   * the producer loads the next item's Q tiles into shared memory as soon as the softmax threads
//     have copied the current ones into tensor memory, and its K / V rings run on across items;
//   * after its last key tile each softmax warpgroup copies the next item's Q row into tensor
//     memory before it writes the current output, so the next item's first S = Q K^T runs under
//     that epilogue;
//   * warps 2-3 (idle in the per-unit kernel) build each item's key-bias / padding table in shared
//     memory ahead of time, double-buffered by item parity.
//
// Work items: the units (batch, query head, block of 256 query rows), ordered query block fastest
// (u = (b * Hq + h) * q_blocks + qb) without a causal mask and longest first with one
// (u = qb_raw * (B * Hq) + (b * Hq + h), qb = q_blocks - 1 - qb_raw), the last `split_units` of them
// split into two items each (one per half of the unit's key tiles,
// merged by whichever CTA finishes its half second, per query tile).  CTA c takes items c, c + G,
// c + 2G, ...: with the split, a launch whose last round of units would leave SMs idle ends instead
// with every SM on half a unit.
//
// Barrier phases are counted across items (only items with key tiles take part; units without any
// write zeros and are skipped by the producer, the MMA issuer and the table builder alike):
//   * K / V rings: running load indices; s_full[tile], p_full[tile][half]: the running key-tile
//     index t (parity t & 1);
//   * q_smem_full / q_smem_empty (Q tiles in shared memory / copied out), q_full[tile] (Q row in
//     tensor memory), o_full[tile] (the item's last P*V done), o_free[tile] (the softmax has read O),
//     kb_full / kb_empty[item & 1] (key table built / read): once per item.
// No waiter lags two phases: each producer of a phase needs the waiter's earlier progress.
#include "attn_tiles.cuh"
#include "nsa_internal.h"
#include "ptx.cuh"

// Sleep between the table builder's polls of a free table buffer.
#ifndef NSA_P2_BUILDER_SLEEP_NS
#define NSA_P2_BUILDER_SLEEP_NS 2000
#endif

namespace nsa {

namespace {

using namespace tiles;

template <int D>
struct P2Cfg {
  using C = Cfg<D>;
  static_assert(C::NQ == 2 && C::QTMEM, "two query tiles with Q in tensor memory");
  static constexpr int NS = C::NS;
  static constexpr int NBARS = 4 * NS + 2 + 4 + 2 + 2 + 2 + 2 + 2 + 2 + 1;
  static constexpr int KB_FLOATS = 2 * kKeyBiasMax;   // two tables, by item parity
  static constexpr int SMEM_BYTES =
      1024 + 2 * C::Q_TILE_BYTES + 2 * NS * C::KV_TILE_BYTES + KB_FLOATS * 4 + NBARS * 8 + 64;
  static_assert(SMEM_BYTES <= 232448, "shared memory budget");
  static_assert(SMEM_BYTES > 117 * 1024, "one CTA per SM (each allocates all 512 TMEM columns)");
};

// One work item's geometry.
struct Item {
  int half;        // -1: the unit's whole key range; 0 / 1: that half of a split unit
  int split_idx;   // index of the split unit (half >= 0)
  int b, bl, hl, hq, hkvl, kv_valid, q_row0, j0, n;
};

template <int D>
__device__ __forceinline__ Item decode_item(const AttnParams& p, int i) {
  constexpr int BN = Cfg<D>::BN;
  Item w;
  const int whole = p.B * p.Hq * p.q_blocks - p.split_units;   // units that run whole
  int u = i;
  w.half = -1;
  w.split_idx = 0;
  if (i >= whole) {
    w.split_idx = (i - whole) >> 1;
    w.half = (i - whole) & 1;
    u = whole + w.split_idx;
  }
  // Without a causal mask every unit has the same length: consecutive items are the query blocks of
  // one (batch, head), so the CTAs working at the same time share few K / V heads in L2.  With one,
  // blocks are dealt longest first across all heads.
  const int bh = p.B * p.Hq;
  int qb, rest;
  if (p.causal) {
    qb = p.q_blocks - 1 - u / bh;
    rest = u % bh;
  } else {
    qb = u % p.q_blocks;
    rest = u / p.q_blocks;
  }
  w.hl = rest % p.Hq;
  w.bl = rest / p.Hq;
  w.b = p.b_begin + w.bl;
  w.hq = p.hq_begin + w.hl;
  w.hkvl = w.hq / p.group - p.hkv_begin;
  w.kv_valid = p.kv_len ? min(p.kv_len[w.b], p.Lk) : p.Lk;
  w.q_row0 = qb * 2 * kTileM;
  const int q_row_end = min(w.q_row0 + 2 * kTileM, p.Lq);
  int kv_end = w.kv_valid;
  if (p.causal) kv_end = min(kv_end, q_row_end);
  const int kv_begin = p.window > 0 ? max(0, w.q_row0 - p.window + 1) : 0;
  w.j0 = kv_begin / BN;
  w.n = kv_end > kv_begin ? ((kv_end - 1) / BN - w.j0 + 1) : 0;
  if (w.half >= 0) {
    const int n_first = w.n / 2;
    if (w.half == 0) {
      w.n = n_first;
    } else {
      w.j0 += n_first;
      w.n -= n_first;
    }
  }
  return w;
}

// Keys [kb0, kb_end) covered by an item's shared-memory key table; ok = false when they do not fit.
template <int D>
__device__ __forceinline__ void key_table_range(const AttnParams& p, const Item& w, int& kb0, int& kb_end, bool& ok) {
  constexpr int BN = Cfg<D>::BN;
  kb0 = min(w.kv_valid, p.bias ? p.bias_start : w.kv_valid);
  kb0 = max(kb0 - kb0 % BN, w.j0 * BN);
  kb_end = (w.j0 + w.n) * BN;
  ok = kb_end - kb0 <= kKeyBiasMax;
}

// Go / no-go over one query tile's 128 softmax threads (named barriers 2 and 3): every one of them
// reaches it once per item, whatever happened, so the tile's split hand-off below never waits for a
// thread that gave up.
__device__ __forceinline__ bool tile_all(int tile, bool ok) {
  return tile == 0 ? bar_and_pred<2, 128>(ok) : bar_and_pred<3, 128>(ok);
}
__device__ __forceinline__ void tile_sync(int tile) {
  if (tile == 0)
    asm volatile("bar.sync 2, 128;" ::: "memory");
  else
    asm volatile("bar.sync 3, 128;" ::: "memory");
}

template <int D>
__global__ void __launch_bounds__(Cfg<D>::THREADS, 1)
    attn_persist2_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                         const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmVd,
                         const AttnParams p) {
  using C = Cfg<D>;
  constexpr int NS = C::NS, BN = C::BN;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;                                   // [2 tiles][Q tile]
  uint8_t* sK = sQ + 2 * C::Q_TILE_BYTES;
  uint8_t* sV = sK + NS * C::KV_TILE_BYTES;
  float* kb = reinterpret_cast<float*>(sV + NS * C::KV_TILE_BYTES);   // [2][kKeyBiasMax]
  uint64_t* bars = reinterpret_cast<uint64_t*>(kb + P2Cfg<D>::KB_FLOATS);
  uint64_t* k_full = bars;                 // [NS]
  uint64_t* k_empty = k_full + NS;         // [NS]
  uint64_t* v_full = k_empty + NS;         // [NS]
  uint64_t* v_empty = v_full + NS;         // [NS]
  uint64_t* s_full = v_empty + NS;         // [2]  per query tile
  uint64_t* p_full = s_full + 2;           // [4]  [tile * 2 + half]
  uint64_t* o_full = p_full + 4;           // [2]  the item's last P*V of the tile done
  uint64_t* o_free = o_full + 2;           // [2]  the tile's softmax has read O (128 arrivals)
  uint64_t* q_full = o_free + 2;           // [2]  the tile's Q rows are in tensor memory (128)
  uint64_t* q_smem = q_full + 2;           // [0] Q tiles landed in shared memory, [1] copied out (256)
  uint64_t* kb_full = q_smem + 2;          // [2]  key table built (64 arrivals), by item parity
  uint64_t* kb_empty = kb_full + 2;        // [2]  key table read (256 arrivals)
  uint64_t* drain = kb_empty + 2;          // MMA teardown after an abort
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* split_arrival = reinterpret_cast<volatile int*>(tmem_slot + 2);   // [2]

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int I = p.B * p.Hq * p.q_blocks + p.split_units;   // work items
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
      mbar_init(&o_free[i], 128);
      mbar_init(&q_full[i], 128);
      mbar_init(&kb_full[i], 64);
      mbar_init(&kb_empty[i], 256);
    }
    for (int i = 0; i < 4; ++i) mbar_init(&p_full[i], 128);
    mbar_init(&q_smem[0], 1);
    mbar_init(&q_smem[1], 256);
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

  if (warp < 4) reg_dealloc<C::REG_CTRL>();
  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      bool ok = true;
      int gk = 0, gv = 0, ia = 0, gq = 0;   // running K / V / Q loads, items with key tiles
      for (int i = blockIdx.x; ok && i < I; i += G) {
        const Item w = decode_item<D>(p, i);
        if (w.n == 0) continue;
        const int kv_y0 = w.bl * p.kv_yb + w.hkvl * p.kv_yh;
        const int k_x = p.k_x0 + w.hkvl * p.kv_xh, v_x = p.v_x0 + w.hkvl * p.kv_xh;
        const int vd_x = p.vd_x0 + w.hkvl * p.vd_xh, vd_y0 = w.b * p.vd_yb;
        const int qx = p.q_x0 + (w.hq - p.q_h0) * p.q_xh;
        const int qy = (w.b - p.q_b0) * p.q_yb + (w.hq - p.q_h0) * p.q_yh + w.q_row0;
        // the Q tiles of this item, once the softmax threads have copied the previous ones out
        if (ia > 0 && !wait_bounded(&q_smem[1], (ia - 1) & 1, abort_flag, p.err, kErrTimeoutLoad, to)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&q_smem[0], 2 * C::Q_TILE_BYTES);
        for (int t = 0; t < 2; ++t)
          for (int c = 0; c < C::NB; ++c)
            tma_load_2d(sQ + t * C::Q_TILE_BYTES + c * C::QBLK_BYTES, &tmQ, &q_smem[0], qx + c * C::BLK,
                        qy + t * kTileM);
        ++gq;
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
            // a tile of valid keys only: straight from the input rows
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
        // the MMA thread consumes K(0), then V(j - 1) followed by K(j)
        ok = load_k(0);
        for (int j = 0; ok && j < w.n; ++j) {
          if (j + 1 < w.n) ok = load_k(j + 1);
          if (ok) ok = load_v(j);
        }
        ++ia;
      }
      if (!ok) {
        // bounded wait for the copies already issued, so none lands after the CTA exits: the
        // latest issue into each stage completes after the earlier ones
        if (gq > 0) wait_drain(&q_smem[0], (gq - 1) & 1, 20000000ull);
        for (int g = gk - 1; g >= 0 && g >= gk - NS; --g) wait_drain(&k_full[g % NS], (g / NS) & 1, 20000000ull);
        for (int g = gv - 1; g >= 0 && g >= gv - NS; --g) wait_drain(&v_full[g % NS], (g / NS) & 1, 20000000ull);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t sk = smem_u32(sK), sv = smem_u32(sV);
      bool ok = true;
      int gk = 0, gv = 0, ia = 0, T = 0;   // running K / V tiles consumed, items, key tiles
      // P*V of tile `tl` for running key tile t (item-local index jj), half by half as the softmax
      // hands P over
      auto pv = [&](int tl, int t, int jj, int svs) -> bool {
        for (int h = 0; h < 2; ++h) {
          if (!wait_bounded(&p_full[tl * 2 + h], t & 1, abort_flag, p.err, kErrTimeoutMma, to)) return false;
          tc_fence_after();
          issue_pv_half<D>(tmem + C::o_col(tl), tmem + C::s_col(tl), sv + svs * C::KV_TILE_BYTES, jj > 0, h);
        }
        return true;
      };
      for (int i = blockIdx.x; ok && i < I; i += G) {
        const Item w = decode_item<D>(p, i);
        if (w.n == 0) continue;
        const int n = w.n;
        // S(0) of both tiles
        ok = wait_bounded(&q_full[0], ia & 1, abort_flag, p.err, kErrTimeoutMma, to) &&
             wait_bounded(&k_full[gk % NS], (gk / NS) & 1, abort_flag, p.err, kErrTimeoutMma, to);
        if (!ok) break;
        tc_fence_after();
        issue_qk<D>(tmem + C::s_col(0), tmem + C::q_col(0), sk + (gk % NS) * C::KV_TILE_BYTES);
        tc_commit(&s_full[0]);
        ok = wait_bounded(&q_full[1], ia & 1, abort_flag, p.err, kErrTimeoutMma, to);
        if (!ok) break;
        tc_fence_after();
        issue_qk<D>(tmem + C::s_col(1), tmem + C::q_col(1), sk + (gk % NS) * C::KV_TILE_BYTES);
        tc_commit(&s_full[1]);
        tc_commit(&k_empty[gk % NS]);
        ++gk;
        // steady state: PV_0(j-1), S_0(j), PV_1(j-1), S_1(j); the first P*V of each tile overwrites
        // its O, so it waits until the softmax has read the previous item's
        for (int j = 1; j <= n; ++j) {
          const int svs = gv % NS;
          ok = wait_bounded(&v_full[svs], (gv / NS) & 1, abort_flag, p.err, kErrTimeoutMma, to);
          if (ok && j == 1 && ia > 0) ok = wait_bounded(&o_free[0], (ia - 1) & 1, abort_flag, p.err, kErrTimeoutMma, to);
          if (ok) ok = pv(0, T + j - 1, j - 1, svs);
          if (!ok) break;
          if (j == n) tc_commit(&o_full[0]);
          if (j < n) {
            ok = wait_bounded(&k_full[gk % NS], (gk / NS) & 1, abort_flag, p.err, kErrTimeoutMma, to);
            if (!ok) break;
            tc_fence_after();
            issue_qk<D>(tmem + C::s_col(0), tmem + C::q_col(0), sk + (gk % NS) * C::KV_TILE_BYTES);
            tc_commit(&s_full[0]);
          }
          if (j == 1 && ia > 0) ok = wait_bounded(&o_free[1], (ia - 1) & 1, abort_flag, p.err, kErrTimeoutMma, to);
          if (ok) ok = pv(1, T + j - 1, j - 1, svs);
          if (!ok) break;
          if (j == n) tc_commit(&o_full[1]);
          tc_commit(&v_empty[svs]);
          ++gv;
          if (j < n) {
            issue_qk<D>(tmem + C::s_col(1), tmem + C::q_col(1), sk + (gk % NS) * C::KV_TILE_BYTES);
            tc_commit(&s_full[1]);
            tc_commit(&k_empty[gk % NS]);
            ++gk;
          }
        }
        T += n;
        ++ia;
      }
      if (!ok) {
        // let every MMA already issued finish before the CTA tears down its tensor memory
        tc_commit(drain);
        wait_drain(drain, 0, 20000000ull);
      }
    }
    __syncwarp();
  } else if (warp < 4) {
    // ------------------------------------------------------------------ key-table builder (warps 2-3)
    // Per item: 0 for plain keys, log(w) * log2(e) for biased text keys, -inf past kv_valid, for the
    // keys [kb0, kb_end) of the tiles that need a mask, in log2 units.
    const int tid = threadIdx.x - 64;
    int ia = 0;
    for (int i = blockIdx.x; i < I; i += G) {
      const Item w = decode_item<D>(p, i);
      if (w.n == 0) continue;
      const int buf = ia & 1;
      // lane 0 of each warp polls, sleeping between polls (the table is needed an item later)
      bool free_ok = true;
      if (ia >= 2 && lane == 0)
        free_ok = wait_bounded_lazy(&kb_empty[buf], ((ia >> 1) - 1) & 1, abort_flag, p.err, kErrTimeoutLoad, to,
                                    NSA_P2_BUILDER_SLEEP_NS);
      if (!__shfl_sync(0xffffffffu, free_ok, 0)) break;
      int kb0, kb_end;
      bool kb_ok;
      key_table_range<D>(p, w, kb0, kb_end, kb_ok);
      if (kb_ok) {
        const float* bias_b = p.bias ? p.bias + (int64_t)w.b * p.bias_bstride : nullptr;
        float* kt = kb + buf * kKeyBiasMax;
        for (int k = tid; k < kb_end - kb0; k += 64) {
          const int key = kb0 + k;
          float v = 0.f;
          if (bias_b && key >= p.bias_start && key < p.bias_start + p.bias_len) v = bias_b[key - p.bias_start] * kLog2e;
          kt[k] = key < w.kv_valid ? v : -INFINITY;
        }
      }
      mbar_arrive(&kb_full[buf]);
      ++ia;
    }
  } else {
    // ------------------------------------------------------------------ softmax + epilogue
    reg_alloc<C::REG_SOFTMAX>();
    const int tile = (warp - 4) / 4;
    const int quarter = warp % 4;
    const uint32_t lane_base = tmem + ((uint32_t)(quarter * 32) << 16);
    const float sl2 = p.scale_log2;
    // this thread's query row of the item with index `ia` among the CTA's items with key tiles, into
    // the Q columns of its TMEM lane (the tile's S MMAs of the previous item have all completed)
    auto copy_q = [&](int ia_q) -> bool {
      if (!__all_sync(0xffffffffu, wait_bounded(&q_smem[0], ia_q & 1, abort_flag, p.err, kErrTimeoutSoftmax, to)))
        return false;
      uint32_t qp[D / 2];
      q_row_from_smem<D>(sQ + tile * C::Q_TILE_BYTES, quarter * 32 + lane, qp);
      mbar_arrive(&q_smem[1]);   // the row is in registers: the producer may reuse the buffer
      tmem_st_n<D / 2>(lane_base + C::q_col(tile), qp);
      tc_fence_before();
      mbar_arrive(&q_full[tile]);
      return true;
    };
    bool ok = true;
    bool q_ready = false;   // the Q row of the next item with key tiles is already in TMEM
    int ia = 0, T = 0;
    for (int i = blockIdx.x; ok && i < I; i += G) {
      const Item w = decode_item<D>(p, i);
      const int row = w.q_row0 + tile * kTileM + quarter * 32 + lane;
      const int tile_row0 = w.q_row0 + tile * kTileM;
      const float* bias_b = p.bias ? p.bias + (int64_t)w.b * p.bias_bstride : nullptr;
      float m_run = -INFINITY, l_run = 0.f;
      if (w.n > 0) {
        if (!q_ready) ok = copy_q(ia);
        q_ready = false;
        const int buf = ia & 1;
        if (ok) ok = __all_sync(0xffffffffu, wait_bounded(&kb_full[buf], (ia >> 1) & 1, abort_flag, p.err,
                                                          kErrTimeoutSoftmax, to));
        int kb0, kb_end;
        bool kb_ok;
        key_table_range<D>(p, w, kb0, kb_end, kb_ok);
        const float* kbt = kb + buf * kKeyBiasMax;
        for (int j = 0; ok && j < w.n; ++j) {
          const int t = T + j;
          ok = __all_sync(0xffffffffu, wait_bounded(&s_full[tile], (uint32_t)(t & 1), abort_flag, p.err,
                                                    kErrTimeoutSoftmax, to));
          if (!ok) break;
          tc_fence_after();
          const int key0 = (w.j0 + j) * BN;
          const bool t_invalid = key0 + BN > w.kv_valid;
          const bool t_causal = p.causal && key0 + BN - 1 > tile_row0;
          const bool t_window = p.window > 0 && key0 <= tile_row0 + kTileM - 1 - p.window;
          const bool t_bias = bias_b != nullptr && key0 + BN > p.bias_start && key0 < p.bias_start + p.bias_len;
          const uint32_t s_addr = lane_base + C::s_col(tile);
          // Unmasked tiles keep the raw scores and fold the scale into the exponent.  Tiles with a
          // text bias or padding take the bias / -inf from the shared table; tiles on a causal or
          // window edge (or beyond the table) are first rewritten in TMEM, 16 columns at a time,
          // into scaled, biased, masked logits.  Both then use a unit scale.
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
            const float4* kt = reinterpret_cast<const float4*>(kbt + (key0 - kb0));
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
              // S(j) was issued after P*V(j - 1) of this tile, so O holds every earlier P*V here
              const float alpha = need ? ex2(m_run - m_new) : 1.f;
              if (need) {
                l_run *= alpha;
                m_run = m_new;
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
            mbar_arrive(&p_full[tile * 2]);
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
            mbar_arrive(&p_full[tile * 2 + 1]);
          }
          {
            float s0, s1;
            f2_unpack(f2_add(f2_add(ls[0], ls[1]), f2_add(ls[2], ls[3])), s0, s1);
            l_run += s0 + s1;
          }
        }
        // The next item's Q row into TMEM now, before this item's epilogue, so that its first
        // S = Q K^T runs while this output is written.
#ifndef NSA_P2_NO_LOOKAHEAD
        if (ok) {
#else
        if (false) {
#endif
          for (int i2 = i + G; i2 < I; i2 += G) {
            if (decode_item<D>(p, i2).n > 0) {
              ok = copy_q(ia + 1);
              q_ready = true;
              break;
            }
          }
        }
        if (ok) mbar_arrive(&kb_empty[buf]);
        if (ok) ok = __all_sync(0xffffffffu, wait_bounded(&o_full[tile], (uint32_t)(ia & 1), abort_flag, p.err,
                                                          kErrTimeoutSoftmax, to));
        if (ok) tc_fence_after();
      }
      ok = tile_all(tile, ok);
      if (!ok) break;
      if (w.half >= 0) {
        // Split unit: publish this half's unnormalised O and (m, l) per row; the CTA that finishes
        // the tile second merges both halves in a fixed order (first half's terms first), so the
        // output does not depend on which half that was:
        //   O = (O_0 2^(m_0 - m) + O_1 2^(m_1 - m)) / (l_0 2^(m_0 - m) + l_1 2^(m_1 - m))
        const int urow = tile * kTileM + quarter * 32 + lane;   // row within the unit
        const int64_t mine = ((int64_t)w.split_idx * 2 + w.half) * (2 * kTileM) + urow;
        const int64_t first = ((int64_t)w.split_idx * 2) * (2 * kTileM) + urow;
        const int64_t second = first + 2 * kTileM;
#pragma unroll 1
        for (int cc = 0; cc < D / 32; ++cc) {
          uint32_t r[32];
          if (w.n > 0) {
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
        if (w.n > 0) {
          // O has been read: the next item's first P*V of this tile may overwrite it
          tc_fence_before();
          mbar_arrive(&o_free[tile]);
        }
        __threadfence();
        tile_sync(tile);
        if (quarter == 0 && lane == 0) split_arrival[tile] = atomicAdd(&p.split_count[w.split_idx * 2 + tile], 1);
        tile_sync(tile);
        if (split_arrival[tile] == 1) {
          __threadfence();
          const float2 ml0 = __ldcg(reinterpret_cast<const float2*>(p.part_ml + first * 2));
          const float2 ml1 = __ldcg(reinterpret_cast<const float2*>(p.part_ml + second * 2));
          const float m = fmaxf(ml0.x, ml1.x);
          const float w0 = ml0.x == -INFINITY ? 0.f : ex2(ml0.x - m);
          const float w1 = ml1.x == -INFINITY ? 0.f : ex2(ml1.x - m);
          const float l = ml0.y * w0 + ml1.y * w1;
          const float inv = l > 0.f ? 1.f / l : 0.f;
          const float a0 = w0 * inv, a1 = w1 * inv;
          const int64_t obase = (int64_t)w.b * p.out_bstride + (int64_t)row * p.out_ld + p.out_off + (int64_t)w.hq * D;
          if (row < p.Lq) {
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
          if (quarter == 0 && lane == 0) p.split_count[w.split_idx * 2 + tile] = 0;   // ready for the next launch
        }
      } else {
        const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
        const bool store = row < p.Lq;
        const int64_t obase = (int64_t)w.b * p.out_bstride + (int64_t)row * p.out_ld + p.out_off + (int64_t)w.hq * D;
#pragma unroll 1
        for (int cc = 0; cc < D / 32; ++cc) {
          uint32_t r[32];
          if (w.n > 0) {
            tmem_ld32(lane_base + C::o_col(tile) + (uint32_t)(cc * 32), r);
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
          // O has been read: the next item's first P*V of this tile may overwrite it
          tc_fence_before();
          mbar_arrive(&o_free[tile]);
        }
      }
      if (w.n > 0) {
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

template <int D>
cudaError_t setup_p2() {
  using C = Cfg<D>;
  cudaError_t e =
      cudaFuncSetAttribute(attn_persist2_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, P2Cfg<D>::SMEM_BYTES);
  if (e != cudaSuccess) return e;
  // The setmaxnreg split is only safe if the kernel really launches with REG_LAUNCH registers per
  // thread; anything else could make setmaxnreg.inc wait forever, so refuse to launch.
  cudaFuncAttributes attr;
  e = cudaFuncGetAttributes(&attr, attn_persist2_kernel<D>);
  if (e != cudaSuccess) return e;
  if (attr.numRegs != C::REG_LAUNCH) return cudaErrorInvalidConfiguration;
  return cudaSuccess;
}

template <int D>
cudaError_t launch_p2(const AttnParams& p, const CUtensorMap& tmQ, const CUtensorMap& tmK, const CUtensorMap& tmV,
                      const CUtensorMap& tmVd, cudaStream_t stream) {
  using C = Cfg<D>;
  static DeviceOnce once;
  cudaError_t e = once_per_device(once, &setup_p2<D>);
  if (e != cudaSuccess) return e;
  const long long units = (long long)p.B * p.Hq * p.q_blocks;
  if (p.split_units > 0 && (p.causal || p.window || p.split_units > units || p.split_first + p.split_units != units))
    return cudaErrorInvalidValue;
  const long long items = units + p.split_units;
  if (items <= 0) return cudaSuccess;
  if (items > 0x7FFFFFFFLL) return cudaErrorInvalidValue;
  const int sms = device_sm_count();
#ifdef NSA_P2_GRID_ALL
  const int grid = (int)items;
#else
  const int grid = (int)(items < sms ? items : sms);
#endif
  attn_persist2_kernel<D><<<grid, C::THREADS, P2Cfg<D>::SMEM_BYTES, stream>>>(tmQ, tmK, tmV, tmVd, p);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_attention_persist2(const AttnParams& p, int D, const CUtensorMap& tmQ, const CUtensorMap& tmK,
                                      const CUtensorMap& tmV, const CUtensorMap& tmVd, cudaStream_t stream) {
  switch (D) {
    case 64: return launch_p2<64>(p, tmQ, tmK, tmV, tmVd, stream);
    case 96: return launch_p2<96>(p, tmQ, tmK, tmV, tmVd, stream);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace nsa
