// Tile geometry and MMA-issue helpers of the per-unit attention kernels (attention.cu): the
// two-query-tile kernels at head dims 64, 96 and 128 and the one-tile kernel at head dim 256.
#pragma once

#include "nsa_internal.h"
#include "ptx.cuh"

namespace nsa {
namespace tiles {

constexpr float kLog2e = 1.4426950408889634f;
constexpr float kRescaleThreshold = 8.0f;   // log2 units: P may reach 2^8 before O is rescaled
constexpr int kKeyBiasMax = 1024;           // keys covered by the shared-memory key bias/mask table

template <int D>
struct Cfg {
  static constexpr bool QTMEM = D <= 96;
  static constexpr int NQ = (D <= 128) ? 2 : 1;
  static constexpr int BN = (D == 96) ? 112 : 128;                   // keys per K/V tile
  static constexpr int NS = (D <= 96) ? 3 : ((D <= 128) ? 2 : 1);    // K and V ring depth
  static constexpr int BLK = (D % 64 == 0) ? 64 : 32;                // elements per swizzle row
  static constexpr int NB = D / BLK;
  static constexpr int ROWB = BLK * 2;                               // bytes per row of one block
  static constexpr uint32_t SWZ = (BLK == 64) ? 2u : 4u;             // 128-byte / 64-byte swizzle
  static constexpr int QBLK_BYTES = kTileM * ROWB;                   // [128 rows][BLK]
  static constexpr int KBLK_BYTES = BN * ROWB;                       // [BN rows][BLK]
  static constexpr int Q_TILE_BYTES = kTileM * D * 2;   // Q tile staged in shared memory
  static constexpr int KV_TILE_BYTES = BN * D * 2;
  static constexpr int KSTEPS_QK = D / 16;
  static constexpr int KSTEPS_PV = BN / 16;
  static constexpr int PV_HALF0 = 4;                                 // k-steps of keys 0..63
  static constexpr int P1_COLS = BN / 2 - 32;                        // P columns of keys 64..BN-1
  static constexpr int THREADS = 128 + NQ * 128;
  // Register split (NQ = 2): the block launches at REG_LAUNCH per thread; the first warpgroup
  // (producer, MMA issuer, two idle warps) drops to REG_CTRL and the two softmax warpgroups rise
  // to REG_SOFTMAX.  128*REG_CTRL + 256*REG_SOFTMAX equals the launch total 384*REG_LAUNCH, so
  // setmaxnreg.inc never waits; the launcher checks the compiled count before every first launch.
  static constexpr int REG_LAUNCH = 168, REG_CTRL = 104, REG_SOFTMAX = 200;
  static_assert(NQ != 2 || 128 * REG_CTRL + 256 * REG_SOFTMAX == THREADS * REG_LAUNCH, "register split");
  static constexpr int SMEM_TILES = NQ * Q_TILE_BYTES + 2 * NS * KV_TILE_BYTES;
  static constexpr int SMEM_KB = kKeyBiasMax * 4;   // key bias/mask table
  // at least 117 KB so that two CTAs never share an SM (each allocates all 512 TMEM columns)
  static constexpr int SMEM_NEED = SMEM_TILES + SMEM_KB + 1024 + 256;
  static constexpr int SMEM_BYTES = SMEM_NEED > 117 * 1024 ? SMEM_NEED : 117 * 1024;
  static constexpr uint32_t TMEM_COLS = 512;
  static constexpr uint32_t IDESC_QK = idesc_bf16_f32(128, BN, 0, 0);
  static constexpr uint32_t IDESC_PV = idesc_bf16_f32(128, D, 0, 1);
  static_assert(SMEM_BYTES <= 232448, "shared memory budget");
  static_assert(BN % 16 == 0 && BN >= 64 && BN <= 128 && KV_TILE_BYTES % 1024 == 0, "key tile");
  static __device__ __forceinline__ uint32_t s_col(int buf) { return (uint32_t)(buf * BN); }
  static __device__ __forceinline__ uint32_t o_col(int tile) {
    return NQ == 2 ? (uint32_t)(2 * BN + tile * (QTMEM ? D : 128)) : 256u;
  }
  static __device__ __forceinline__ uint32_t q_col(int tile) { return (uint32_t)(2 * BN + 2 * D + tile * (D / 2)); }
  // byte offset of MMA k-step kk (16 elements) inside a K-major [rows][D] tile of row blocks
  static __device__ __forceinline__ uint32_t kmajor_off(int kk, int blk_bytes) {
    constexpr int per_blk = BLK / 16;
    return (uint32_t)((kk / per_blk) * blk_bytes + (kk % per_blk) * 32);
  }
};
static_assert(Cfg<96>::QTMEM && 2 * Cfg<96>::BN + 2 * 96 + 96 == 512, "TMEM map, D = 96");
static_assert(2 * Cfg<64>::BN + 2 * 64 + 64 <= 512, "TMEM map, D = 64");

// S = Q K^T for one tile; Q from shared memory (SS) or tensor memory (TS).
template <int D>
__device__ __forceinline__ void issue_qk(uint32_t d_tmem, uint32_t q_src, uint32_t sk) {
  using C = Cfg<D>;
#pragma unroll
  for (int kk = 0; kk < C::KSTEPS_QK; ++kk) {
    const uint64_t b = smem_desc(sk + C::kmajor_off(kk, C::KBLK_BYTES), 16, 8 * C::ROWB, C::SWZ);
    if constexpr (C::QTMEM) {
      mma_ts(d_tmem, q_src + (uint32_t)(kk * 8), b, C::IDESC_QK, kk > 0 ? 1u : 0u);
    } else {
      const uint64_t a = smem_desc(q_src + C::kmajor_off(kk, C::QBLK_BYTES), 16, 8 * C::ROWB, C::SWZ);
      mma_ss(d_tmem, a, b, C::IDESC_QK, kk > 0 ? 1u : 0u);
    }
  }
}

// O (+)= P V over the keys of one P half (keys 0..63, then 64..BN-1): the softmax hands P over in
// two halves so the tensor core starts on the first while the second is still being exponentiated.
template <int D>
__device__ __forceinline__ void issue_pv_half(uint32_t d_tmem, uint32_t p_tmem, uint32_t sv, bool accumulate,
                                              int half) {
  using C = Cfg<D>;
  const int k_begin = half == 0 ? 0 : C::PV_HALF0;
  const int k_end = half == 0 ? C::PV_HALF0 : C::KSTEPS_PV;
#pragma unroll
  for (int kk = k_begin; kk < k_end; ++kk) {
    // V is MN-major: 16 keys per k-step, head-dim blocks of BLK elements KBLK_BYTES apart
    const uint64_t b = smem_desc(sv + (uint32_t)(kk * 16 * C::ROWB), C::KBLK_BYTES, 8 * C::ROWB, C::SWZ);
    mma_ts(d_tmem, p_tmem + (uint32_t)(kk * 8), b, C::IDESC_PV, (accumulate || kk > 0) ? 1u : 0u);
  }
}

// Row r of a staged Q tile (already normalised and rotated by the prologue) as D/2 bf16 pairs, in
// column order, read from the swizzled shared-memory tile.
template <int D>
__device__ __forceinline__ void q_row_from_smem(const uint8_t* tile, int r, uint32_t (&qp)[D / 2]) {
  using C = Cfg<D>;
  constexpr int CHUNKS = C::ROWB / 16;   // 16-byte chunks per row of a swizzle block
#pragma unroll
  for (int blk = 0; blk < C::NB; ++blk) {
#pragma unroll
    for (int c = 0; c < CHUNKS; ++c) {
      // the TMA swizzle XORs the 16-byte chunk index with the row bits above the chunk span
      const int phys = c ^ ((r / (128 / C::ROWB)) % CHUNKS);
      const uint4 a = *reinterpret_cast<const uint4*>(tile + blk * C::QBLK_BYTES + r * C::ROWB + phys * 16);
      const int w0 = (blk * C::BLK + c * 8) / 2;
      qp[w0] = a.x;
      qp[w0 + 1] = a.y;
      qp[w0 + 2] = a.z;
      qp[w0 + 3] = a.w;
    }
  }
}

template <int N>
__device__ __forceinline__ void tmem_ld_n(uint32_t taddr, uint32_t (&r)[N]) {
  if constexpr (N == 112) tmem_ld112(taddr, r);
  else if constexpr (N == 128) tmem_ld128(taddr, r);
  else static_assert(N == 112 || N == 128, "score row width");
}

template <int N>
__device__ __forceinline__ void tmem_st_n(uint32_t taddr, const uint32_t (&r)[N]) {
  if constexpr (N == 24) tmem_st24(taddr, r);
  else if constexpr (N == 32) tmem_st32(taddr, r);
  else if constexpr (N == 48) tmem_st48(taddr, r);
  else static_assert(N == 24 || N == 32 || N == 48, "column count");
}

}  // namespace tiles
}  // namespace nsa
