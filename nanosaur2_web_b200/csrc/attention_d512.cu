// Forward attention at head dim 512 (the VAE decoder's single-head attention over all latent pixels,
// app/models/vae.js:77-88; tools/reference.py:352-357), sm_100a.
//
// At D = 512 one 128-row query tile's fp32 output alone is 128 x 512 values: all 512 columns of
// tensor memory.  So two CTAs share each query tile, each owning one half of the output columns
// (256), and each computes the whole score tile S = Q K^T itself (the P*V work is split, the
// Q K^T work done twice: 1.5x the algorithmic flops on the tensor cores).  Both CTAs of a pair run
// the identical S MMA sequence, so their running max and sum agree bit for bit and the two halves
// are normalised alike.
//
// Per CTA (256 threads): warp 0 is the TMA producer, warp 1 allocates tensor memory and issues every
// tcgen05.mma, warps 4-7 are the softmax + epilogue (one query row per thread).  Tensor memory:
//   S0 [0,128) S1 [128,256)   score tiles of 128 keys, double-buffered; P (bf16) over their first 64
//   O  [256,512)              this CTA's 256 output columns
// Shared memory: the unit's Q tile resident (8 blocks of [128 rows][64], 128 KB, 128-byte swizzle)
// and one ring of 16 KB stages through which the producer streams, in the order the MMAs consume
// them, each key tile's K as 8 blocks of [128 keys][64] (S = sum over the 8 blocks) and its V half as
// 4 chunks of [32 keys][256] (P*V = sum over the chunks).  Issue order per unit: S(0), S(1), then
// P*V(j) followed by S(j + 2), as in the head-dim-256 kernel.
//
// Persistent: one CTA per SM loops over units u = (query unit) * 2 + column half, query units
// ordered like attention_persist.cu (causal blocks long-first).  Barrier phases are counted across
// units; q_full / q_empty / o_full[1] / o_free once per unit with key tiles.
#include "nsa_internal.h"
#include "ptx.cuh"

namespace nsa {

namespace {

constexpr float kLog2e5 = 1.4426950408889634f;
constexpr float kRescale5 = 8.0f;   // log2 units: P may reach 2^8 before O is rescaled
constexpr int kKeyBias5 = 1024;     // keys covered by the shared-memory key bias/mask table

struct Cfg5 {
  static constexpr int D = 512, DH = 256, BN = 128;
  static constexpr int QBLK = kTileM * 128;            // [128 rows][64] bf16 = 16 KB
  static constexpr int Q_BYTES = 8 * QBLK;             // resident Q tile
  static constexpr int STAGE = 16384;                  // one ring entry
  static constexpr int NSTG = 5;
  static constexpr int VCH_KEYS = 32;                  // keys per V chunk
  static constexpr int VBLK = VCH_KEYS * 128;          // [32 keys][64] bf16 = 4 KB, 4 per chunk
  static constexpr int THREADS = 256;
  static constexpr int NBARS = 2 * NSTG + 2 + 4 + 2 + 4 + 1;
  static constexpr int SMEM_BYTES = 1024 + Q_BYTES + NSTG * STAGE + kKeyBias5 * 4 + NBARS * 8 + 16;
  static constexpr uint32_t IDESC_QK = idesc_bf16_f32(128, BN, 0, 0);
  static constexpr uint32_t IDESC_PV = idesc_bf16_f32(128, DH, 0, 1);
  static_assert(SMEM_BYTES <= 232448, "shared memory budget");
  static __device__ __forceinline__ uint32_t s_col(int buf) { return (uint32_t)(buf * BN); }
  static __device__ __forceinline__ uint32_t o_col() { return 256u; }
};

// One unit's geometry: (batch, query head, 128-row query tile, output column half).
struct Unit5 {
  int b, bl, hl, hq, hkvl, kv_valid, q_row0, j0, n, half;
};

__device__ __forceinline__ Unit5 decode_unit5(const AttnParams& p, int u) {
  constexpr int BN = Cfg5::BN;
  Unit5 w;
  w.half = u & 1;
  const int qu = u >> 1;
  const int bh = p.B * p.Hq;
  const int qb_raw = qu / bh, rest = qu % bh;
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

__global__ void __launch_bounds__(Cfg5::THREADS, 1)
    attn_d512_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                     const __grid_constant__ CUtensorMap tmV, const AttnParams p) {
  using C = Cfg5;
  constexpr int BN = C::BN, NSTG = C::NSTG, DH = C::DH;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;
  uint8_t* ring = sQ + C::Q_BYTES;
  float* kb = reinterpret_cast<float*>(ring + NSTG * C::STAGE);   // [kKeyBias5]
  uint64_t* bars = reinterpret_cast<uint64_t*>(kb + kKeyBias5);
  uint64_t* full = bars;                 // [NSTG] ring entry landed
  uint64_t* empty = full + NSTG;         // [NSTG] ring entry consumed by its MMAs
  uint64_t* s_full = empty + NSTG;       // [2] per S buffer
  uint64_t* p_full = s_full + 2;         // [buffer * 2 + half]
  uint64_t* o_full = p_full + 4;         // [0] once per P*V, [1] once per unit (its last P*V)
  uint64_t* q_full = o_full + 2;         // Q of the unit landed
  uint64_t* q_empty = q_full + 1;        // the unit's S MMAs are done with Q
  uint64_t* o_free = q_empty + 1;        // the softmax has read the unit's O (128 arrivals)
  uint64_t* drain = o_free + 1;          // MMA teardown after an abort
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int U = p.B * p.Hq * p.q_blocks * 2;
  const int G = (int)gridDim.x;
  const uint64_t to = p.timeout_ns;

  if (threadIdx.x == 0) {
    for (int s = 0; s < NSTG; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
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
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
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
      int g = 0, ia = 0, gq = 0;   // running ring entries, units with key tiles, Q loads
      for (int u = blockIdx.x; ok && u < U; u += G) {
        const Unit5 w = decode_unit5(p, u);
        if (w.n == 0) continue;
        const int kv_y0 = w.bl * p.kv_yb + w.hkvl * p.kv_yh;
        const int k_x = p.k_x0 + w.hkvl * p.kv_xh, v_x = p.v_x0 + w.hkvl * p.kv_xh + w.half * DH;
        const int qx = p.q_x0 + (w.hq - p.q_h0) * p.q_xh;
        const int qy = (w.b - p.q_b0) * p.q_yb + (w.hq - p.q_h0) * p.q_yh + w.q_row0;
        if (ia > 0 && !wait_bounded(q_empty, (ia - 1) & 1, abort_flag, p.err, kErrTimeoutLoad, to)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(q_full, C::Q_BYTES);
        for (int c = 0; c < 8; ++c) tma_load_2d(sQ + c * C::QBLK, &tmQ, q_full, qx + c * 64, qy);
        ++gq;
        auto next = [&]() -> uint8_t* {   // the next free ring entry, armed for 16 KB
          const int s = g % NSTG;
          if (g >= NSTG && !wait_bounded(&empty[s], ((g / NSTG) - 1) & 1, abort_flag, p.err, kErrTimeoutLoad, to))
            return nullptr;
          mbar_arrive_expect_tx(&full[s], C::STAGE);
          return ring + s * C::STAGE;
        };
        auto load_k = [&](int j) -> bool {   // the 8 blocks of K tile j, one entry each
          for (int c = 0; c < 8; ++c) {
            uint8_t* dst = next();
            if (!dst) return false;
            tma_load_2d(dst, &tmK, &full[g % NSTG], k_x + c * 64, kv_y0 + (w.j0 + j) * BN);
            ++g;
          }
          return true;
        };
        auto load_v = [&](int j) -> bool {   // this CTA's V half of tile j, 4 chunks of 32 keys
          for (int v = 0; v < BN / C::VCH_KEYS; ++v) {
            uint8_t* dst = next();
            if (!dst) return false;
            for (int blk = 0; blk < DH / 64; ++blk)
              tma_load_2d(dst + blk * C::VBLK, &tmV, &full[g % NSTG], v_x + blk * 64,
                          kv_y0 + (w.j0 + j) * BN + v * C::VCH_KEYS);
            ++g;
          }
          return true;
        };
        // the MMA thread consumes S(0), S(1), then P*V(j) followed by S(j + 2)
        for (int j = 0; ok && j < 2 && j < w.n; ++j) ok = load_k(j);
        for (int j = 0; ok && j < w.n; ++j) {
          ok = load_v(j);
          if (ok && j + 2 < w.n) ok = load_k(j + 2);
        }
        ++ia;
      }
      if (!ok) {
        // bounded wait for the copies already issued, so none lands after the CTA exits
        if (gq > 0) wait_drain(q_full, (gq - 1) & 1, 20000000ull);
        for (int e = g - 1; e >= 0 && e >= g - NSTG; --e) wait_drain(&full[e % NSTG], (e / NSTG) & 1, 20000000ull);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t sq = smem_u32(sQ), sr = smem_u32(ring);
      bool ok = true;
      int g = 0, ia = 0, T = 0;   // running ring entries, units, key tiles
      auto take = [&]() -> int {   // the next ring entry once it has landed, or -1
        const int s = g % NSTG;
        if (!wait_bounded(&full[s], (g / NSTG) & 1, abort_flag, p.err, kErrTimeoutMma, to)) return -1;
        tc_fence_after();
        return s;
      };
      auto issue_s = [&](int t_idx, bool last) -> bool {   // S(t_idx) into buffer t_idx & 1
        const uint32_t d = tmem + C::s_col(t_idx & 1);
        for (int c = 0; c < 8; ++c) {
          const int s = take();
          if (s < 0) return false;
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            const uint64_t a = smem_desc(sq + c * C::QBLK + kk * 32, 16, 1024, 2);
            const uint64_t bd = smem_desc(sr + s * C::STAGE + kk * 32, 16, 1024, 2);
            mma_ss(d, a, bd, C::IDESC_QK, (c > 0 || kk > 0) ? 1u : 0u);
          }
          tc_commit(&empty[s]);
          ++g;
        }
        tc_commit(&s_full[t_idx & 1]);
        if (last) tc_commit(q_empty);   // the unit's last S: Q may be replaced
        return true;
      };
      for (int u = blockIdx.x; ok && u < U; u += G) {
        const Unit5 w = decode_unit5(p, u);
        if (w.n == 0) continue;
        ok = wait_bounded(q_full, ia & 1, abort_flag, p.err, kErrTimeoutMma, to);
        if (ok) tc_fence_after();
        for (int j = 0; ok && j < 2 && j < w.n; ++j) ok = issue_s(T + j, j == w.n - 1);
        for (int j = 0; ok && j < w.n; ++j) {
          const int t = T + j;
          const uint32_t pa = tmem + C::s_col(t & 1);
          // the first P*V overwrites O: the softmax must have read the previous unit's O
          if (j == 0 && ia > 0) ok = wait_bounded(o_free, (ia - 1) & 1, abort_flag, p.err, kErrTimeoutMma, to);
          for (int v = 0; ok && v < BN / C::VCH_KEYS; ++v) {
            if ((v & 1) == 0) {   // chunks 0-1 need P half 0 (keys 0-63), chunks 2-3 half 1
              ok = wait_bounded(&p_full[(t & 1) * 2 + (v >> 1)], (t >> 1) & 1, abort_flag, p.err, kErrTimeoutMma, to);
              if (!ok) break;
              tc_fence_after();
            }
            const int s = take();
            if (s < 0) {
              ok = false;
              break;
            }
#pragma unroll
            for (int kk = 0; kk < C::VCH_KEYS / 16; ++kk) {
              // V is MN-major: 16 keys per k-step, column blocks of 64 elements VBLK bytes apart
              const uint64_t bd = smem_desc(sr + s * C::STAGE + kk * 16 * 128, C::VBLK, 1024, 2);
              mma_ts(tmem + C::o_col(), pa + (uint32_t)(v * 16 + kk * 8), bd, C::IDESC_PV,
                     (j > 0 || v > 0 || kk > 0) ? 1u : 0u);
            }
            tc_commit(&empty[s]);
            ++g;
          }
          if (!ok) break;
          tc_commit(&o_full[0]);
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
      const Unit5 w = decode_unit5(p, u);
      const int row = w.q_row0 + quarter * 32 + lane;
      const int tile_row0 = w.q_row0;
      const float* bias_b = p.bias ? p.bias + (int64_t)w.b * p.bias_bstride : nullptr;
      // key bias + padding mask table of this unit (the previous unit's loop is done with it)
      asm volatile("bar.sync 1, 128;" ::: "memory");
      int kb0 = min(w.kv_valid, bias_b ? p.bias_start : w.kv_valid);
      kb0 = max(kb0 - kb0 % BN, w.j0 * BN);
      const int kb_end = (w.j0 + w.n) * BN;
      const bool kb_ok = kb_end - kb0 <= kKeyBias5;
      if (kb_ok) {
        for (int i = threadIdx.x - 128; i < kb_end - kb0; i += 128) {
          const int key = kb0 + i;
          float v = 0.f;
          if (bias_b && key >= p.bias_start && key < p.bias_start + p.bias_len) v = bias_b[key - p.bias_start] * kLog2e5;
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
                v += __ldg(bias_b + (key - p.bias_start)) * kLog2e5;
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
          const bool need = m_new > m_run + kRescale5;
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
            for (int cc = 0; cc < DH / 32; ++cc) {
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
          // keys 64*half .. 64*half+63 -> P columns 32*half .. 32*half+31
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
      const int64_t obase = (int64_t)w.b * p.out_bstride + (int64_t)row * p.out_ld + p.out_off +
                            (int64_t)w.hq * C::D + w.half * DH;
#pragma unroll 1
      for (int cc = 0; cc < DH / 32; ++cc) {
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
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace

int attention_d512_v_box_rows() { return Cfg5::VCH_KEYS; }

cudaError_t launch_attention_d512(const AttnParams& p, const CUtensorMap& tmQ, const CUtensorMap& tmK,
                                  const CUtensorMap& tmV, cudaStream_t stream) {
  static DeviceOnce once;
  cudaError_t e = once_per_device(once, [] {
    return cudaFuncSetAttribute(attn_d512_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg5::SMEM_BYTES);
  });
  if (e != cudaSuccess) return e;
  if (p.split_units > 0 || p.v_direct) return cudaErrorInvalidValue;
  const long long units = (long long)p.B * p.Hq * p.q_blocks * 2;
  if (units <= 0) return cudaSuccess;
  if (units > 0x7FFFFFFFLL) return cudaErrorInvalidValue;
  const int sms = device_sm_count();
  const int grid = (int)(units < sms ? units : sms);
  attn_d512_kernel<<<grid, Cfg5::THREADS, Cfg5::SMEM_BYTES, stream>>>(tmQ, tmK, tmV, p);
  return cudaGetLastError();
}

}  // namespace nsa
