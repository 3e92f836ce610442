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
//   warps 2-9   epilogue, two groups of four warps (each group covers the 128 TMEM lanes, a thread
//               one output row): group g takes heads g, g+2, ... of the tile (or half of the RoPE
//               pairs when a tile holds one head).  Per head: sum of squares over the accumulator
//               columns, then bias + norm weight + RoPE, bf16 stores.  Bias and norm weights sit in
//               shared memory.  Tensor-memory reads are few and wide (a wait costs about a thousand
//               cycles while the next tile's MMAs run), and each chunk's cos / sin loads are issued
//               before its tensor-memory wait; at head dims 96 and 256 they come through shared
//               memory, one TMA box of the warp's 32 table rows per chunk.
#include "nsa_internal.h"
#include "ptx.cuh"

namespace nsa {

namespace {

constexpr int kProjBK = 64;         // K elements per stage: one 128-byte swizzle row
constexpr int kProjThreads = 320;

template <int D>
struct ProjCfg {
  static constexpr int HPT = D == 96 ? 2 : 256 / D;   // heads per N tile
  static constexpr int NT = HPT * D;                   // 192 at D = 96, 256 otherwise
  static constexpr int A_BYTES = 128 * kProjBK * 2;
  static constexpr int B_BYTES = NT * kProjBK * 2;
  static constexpr int STAGE = A_BYTES + B_BYTES;
  static constexpr uint32_t ACC_COLS = 256;            // TMEM columns per accumulator
  static constexpr uint32_t IDESC = idesc_bf16_f32(128, NT, 0, 0);
  // One head per epilogue group (head dims 96 and 256): the RoPE rows come through shared memory,
  // one TMA box of the warp's 32 table rows per 16-pair chunk (see the epilogue)
  static constexpr bool kTableTma = D == 256 || D == 96;
  static_assert(NT % 16 == 0 && NT <= 256 && STAGE % 1024 == 0, "projection tile");
};

constexpr int kTableWarpBytes = 4096;             // cos [32][16] fp32 + sin [32][16] fp32
constexpr int kTableBytes = 8 * kTableWarpBytes;  // eight epilogue warps (a multiple of 1024)

// 16 consecutive floats of a shared-memory vector (bias, norm weight) in four 16-byte reads; every
// offset used is a multiple of 16 floats.
__device__ __forceinline__ void lds16(const float* src, float (&o)[16]) {
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const float4 v = reinterpret_cast<const float4*>(src)[q];
    o[4 * q] = v.x;
    o[4 * q + 1] = v.y;
    o[4 * q + 2] = v.z;
    o[4 * q + 3] = v.w;
  }
}

// 16 consecutive floats of a global vector (the per-row weight scales of int8 ConvRot weights); all
// lanes of a warp read the same addresses.
__device__ __forceinline__ void ldg16(const float* src, float (&o)[16]) {
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const float4 v = __ldg(reinterpret_cast<const float4*>(src) + q);
    o[4 * q] = v.x;
    o[4 * q + 1] = v.y;
    o[4 * q + 2] = v.z;
    o[4 * q + 3] = v.w;
  }
}

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
    proj_kernel(const __grid_constant__ CUtensorMap tmX0, const __grid_constant__ CUtensorMap tmW0,
                const __grid_constant__ CUtensorMap tmX1, const __grid_constant__ CUtensorMap tmW1,
                const __grid_constant__ CUtensorMap tmCS, const __grid_constant__ CUtensorMap tmT0,
                const __grid_constant__ CUtensorMap tmL0, const __grid_constant__ CUtensorMap tmT1,
                const __grid_constant__ CUtensorMap tmL1, const ProjParams p) {
  using C = ProjCfg<D>;
  const int S = p.stages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int nb0 = p.set[0].n_tiles * C::NT, nb1 = p.n_sets > 1 ? p.set[1].n_tiles * C::NT : 0;
  // head dim 256: per epilogue warp, the cos and sin rows of its 32 output rows for one 16-pair chunk
  // ([32][16] fp32 each, 64-byte swizzle), staged by TMA
  const bool cs_tma = C::kTableTma && p.cs_tma;
  uint8_t* stable = smem + S * C::STAGE;                            // [8 warps][cos 2 KB | sin 2 KB]
  float* sbias0 = reinterpret_cast<float*>(stable + (cs_tma ? kTableBytes : 0));   // [nb0] (zeros without a bias)
  float* sbias1 = sbias0 + nb0;                                    // [nb1]
  float* sqw = sbias1 + nb1;                                       // [D] q norm weight
  float* skw = sqw + D;                                            // [D] k norm weight
  // one head per tile (head dim 256): the two epilogue warps of a TMEM lane quarter each sum the
  // squares of their own half of the row and swap the partial sums here ([tile parity][warp][lane])
  float* xss = skw + D;
  volatile int* xflag = reinterpret_cast<volatile int*>(xss + 2 * 256);   // [warp][lane]: last tile + 1
  uint64_t* full = reinterpret_cast<uint64_t*>(xss + 3 * 256);      // 16-byte aligned (all sizes x 16 B)
  uint64_t* empty = full + S;
  uint64_t* acc_full = empty + S;       // [2] accumulator ready for the epilogue
  uint64_t* acc_empty = acc_full + 2;   // [2] accumulator read out (256 epilogue arrivals)
  uint64_t* drain = acc_empty + 2;      // MMAs of an aborted CTA finished
  uint64_t* pbar = drain + 1;           // bias vectors and norm weights landed
  uint64_t* tbar = pbar + 1;            // [8] one epilogue warp's table chunk landed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tbar + 8);
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
    for (int i = 0; i < 8; ++i) mbar_init(&tbar[i], 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  if (blockIdx.x == 0)
    for (int i = threadIdx.x; i < p.zero_count; i += blockDim.x) p.zero_ptr[i] = 0;
  // a missing bias reads as zeros
  for (int i = threadIdx.x; i < 256; i += blockDim.x) xflag[i] = 0;
  if (!p.set[0].bias)
    for (int i = threadIdx.x; i < nb0; i += blockDim.x) sbias0[i] = 0.f;
  if (nb1 && !p.set[1].bias)
    for (int i = threadIdx.x; i < nb1; i += blockDim.x) sbias1[i] = 0.f;
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  const int tiles0 = p.B * p.set[0].m_tiles * p.set[0].n_tiles;
  const int tiles = tiles0 + (p.n_sets > 1 ? p.B * p.set[1].m_tiles * p.set[1].n_tiles : 0);
  const int G = gridDim.x;
  // tile u -> (row set, local batch element, first row, N tile, part 0/1/2 = q/k/v, first head);
  // false for image k / v tiles wholly past the shard's query rows (other shards' keys)
  auto decode = [&](int u, int& si, int& bl, int& m0, int& nt, int& part, int& h0) -> bool {
    si = u < tiles0 ? 0 : 1;
    if (si) u -= tiles0;
    const ProjSet& q = p.set[si];
    nt = u % q.n_tiles;
    const int rest = u / q.n_tiles;
    m0 = (rest % q.m_tiles) * 128;
    bl = rest / q.m_tiles;
    const int nt_q = q.image ? p.Hq / C::HPT : 0;
    const int nt_kv = p.Hkv / C::HPT;
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
    return !(q.image && part > 0 && m0 >= q.valid_q);
  };

  if (warp == 0) {
    // ---------------------------------------------------------------- TMA producer
    if (lane == 0) {
      tma_prefetch_desc(&tmX0);
      tma_prefetch_desc(&tmW0);
      if (p.n_sets > 1) {
        tma_prefetch_desc(&tmX1);
        tma_prefetch_desc(&tmW1);
      }
      // bias vectors and norm weights: one bulk copy each
      const uint32_t b0 = p.set[0].bias ? (uint32_t)nb0 * 4 : 0u, b1 = (nb1 && p.set[1].bias) ? (uint32_t)nb1 * 4 : 0u;
      mbar_arrive_expect_tx(pbar, b0 + b1 + 2u * D * 4);
      if (b0) bulk_load(sbias0, p.set[0].bias, b0, pbar);
      if (b1) bulk_load(sbias1, p.set[1].bias, b1, pbar);
      bulk_load(sqw, p.q_w, D * 4, pbar);
      bulk_load(skw, p.k_w, D * 4, pbar);
      int step = 0;
      bool ok = true;
      for (int u = blockIdx.x; ok && u < tiles; u += G) {
        int si, bl, m0, nt, part, h0;
        if (!decode(u, si, bl, m0, nt, part, h0)) continue;
        const int steps = p.k_steps + p.set[si].lora_steps;
        for (int ks = 0; ks < steps; ++ks, ++step) {
          const int s = step % S;
          if (step >= S &&
              !wait_bounded(&empty[s], ((step / S) - 1) & 1, abort_flag, p.err, kErrTimeoutProjection, to)) {
            ok = false;
            break;
          }
          uint8_t* st = smem + s * C::STAGE;
          mbar_arrive_expect_tx(&full[s], C::STAGE);
          if (ks < p.k_steps) {
            tma_load_3d(st, si ? &tmX1 : &tmX0, &full[s], ks * kProjBK, p.set[si].x_row0 + m0, bl);
            tma_load_2d(st + C::A_BYTES, si ? &tmW1 : &tmW0, &full[s], ks * kProjBK, nt * C::NT);
          } else {   // LoRA slices: T rows (same row index as x) against B_cat rows
            const int kl = (ks - p.k_steps) * kProjBK;
            tma_load_3d(st, si ? &tmT1 : &tmT0, &full[s], kl, p.set[si].x_row0 + m0, bl);
            tma_load_2d(st + C::A_BYTES, si ? &tmL1 : &tmL0, &full[s], kl, nt * C::NT);
          }
        }
      }
      // copies still landing complete before the CTA may exit
      wait_drain(pbar, 0, to);
      for (int i = step > S ? step - S : 0; i < step; ++i) wait_drain(&full[i % S], (i / S) & 1, to);
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      int step = 0, t = 0;
      bool ok = true;
      for (int u = blockIdx.x; ok && u < tiles; u += G) {
        int si, bl, m0, nt, part, h0;
        if (!decode(u, si, bl, m0, nt, part, h0)) continue;
        const int a = t & 1;
        if (t >= 2 && !wait_bounded(&acc_empty[a], ((t >> 1) - 1) & 1, abort_flag, p.err, kErrTimeoutProjection, to)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem + (uint32_t)a * C::ACC_COLS;
        const int steps = p.k_steps + p.set[si].lora_steps;
        for (int ks = 0; ks < steps; ++ks, ++step) {
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
    // ---------------------------------------------------------------- epilogue (warps 2-9)
    const int ew = warp - 2;
    const int group = ew / 4;
    const int quarter = warp % 4;   // TMEM lane quarter this warp may access
    const int row_local = quarter * 32 + lane;
    // heads of the tile this group handles, and its range of RoPE pairs within a head
    constexpr int HSTEP = C::HPT >= 2 ? 2 : 1;
    const int pair0 = C::HPT >= 2 ? 0 : group * (D / 4);
    const int pair1 = C::HPT >= 2 ? D / 2 : pair0 + D / 4;
    const int hh0 = C::HPT >= 2 ? group : 0;
    bool params_ready = false;
    int t = 0;
    // Head dims 96 and 256: a thread's RoPE row is D/2 cos + D/2 sin values, and 32 lanes of a warp
    // hold 32 rows, so per-thread loads would touch 32 lines per instruction.  Instead lane 0 brings the warp's
    // 32 table rows of one 16-pair chunk into shared memory with two TMA box loads (64-byte swizzle)
    // and every lane reads its row from there without bank conflicts.  One chunk is in flight at a
    // time: the next is issued as soon as the current one has been read.
    uint8_t* tbuf = stable + ew * kTableWarpBytes;
    uint32_t t_issued = 0, t_done = 0;   // table loads of this warp (warp-uniform counts)
    bool aborted = false;
    auto issue_table = [&](int c, int tr0) {   // lane 0 only
      fence_proxy_async_smem();   // the lanes' reads of the previous chunk come before the overwrite
      mbar_arrive_expect_tx(&tbar[ew], kTableWarpBytes);
      tma_load_2d(tbuf, &tmCS, &tbar[ew], c, tr0);
      tma_load_2d(tbuf + kTableWarpBytes / 2, &tmCS, &tbar[ew], c, p.cs_rows + tr0);
    };
    for (int u = blockIdx.x; u < tiles; u += G) {
      int si, bl, m0, nt, part, h0;
      if (!decode(u, si, bl, m0, nt, part, h0)) continue;
      const ProjSet& q = p.set[si];
      const int a = t & 1;
      const int r = m0 + row_local;   // GEMM row
      const int b = p.b_begin + bl;
      const int key = q.key_row0 + r;
      const int kv_valid = p.kv_len ? min(p.kv_len[b], p.Lk) : p.Lk;
      // which rows exist in the destination, and which hold data (the rest are zeros)
      bool write, valid;
      if (part == 0) {
        write = r < p.Lq_pad;
        valid = r < q.valid_q;
      } else if (q.image) {
        write = r < q.valid_q;   // other keys are other shards' (or the text rows)
        valid = write && key < kv_valid;
      } else {
        write = key < p.Lk_pad;
        valid = key < kv_valid;
      }
      const float* wn = part == 0 ? sqw : (part == 1 ? skw : nullptr);
      const bool rope = q.image && part < 2 && p.cs != nullptr && valid;
      const int rrow = q.rope_row0 + r;
      // TMA table path: decided per warp (rows without data are rotated too, then zeroed); the first
      // chunk's rows are in flight during the accumulator wait.  Table rows past the cos block read
      // sin rows or the zero fill, only for rows that hold no data.
      const int tr0 = q.rope_row0 + m0 + quarter * 32;
      const bool rope_w = cs_tma && q.image && part < 2 && p.cs != nullptr && m0 + quarter * 32 < q.valid_q;
      if (rope_w) {
        if (lane == 0) issue_table(pair0, tr0);
        ++t_issued;
      }
      const bool rot = cs_tma ? rope_w : rope;
      bool got = wait_bounded(&acc_full[a], (t >> 1) & 1, abort_flag, p.err, kErrTimeoutProjection, to);
      if (got && !params_ready) {
        got = wait_bounded(pbar, 0, abort_flag, p.err, kErrTimeoutProjection, to);
        params_ready = true;
      }
      if (!__all_sync(0xffffffffu, got)) break;
      tc_fence_after();
      const uint32_t tbase = tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)a * C::ACC_COLS;
      const float* sbias = si ? sbias1 : sbias0;
#pragma unroll 1
      for (int hh = hh0; hh < C::HPT; hh += HSTEP) {
        const int h = h0 + hh;
        const uint32_t col0 = (uint32_t)(hh * D);
        const float* bias = sbias + nt * C::NT + hh * D;
        // int8 ConvRot weights (given as their exact bf16 values): the row scales of this head's columns.
        // Not at head dim 256: that is the Gemma encoder, whose 640-wide linears are never ConvRot
        // weights (the quantiser needs K % 256 == 0, tools/quant.py:43-44), and its epilogue has no
        // registers to spare.
        const float* wsc = (D != 256 && q.w_scale) ? q.w_scale + nt * C::NT + hh * D : nullptr;
        // pass 1: sum of squares of (acc + bias) over the head (tcgen05.ld is warp-wide: every lane),
        // in wide loads: each load's wait is a round trip of the order of a thousand cycles while the
        // MMAs of the next tile write tensor memory
        float rn = 1.f;
        if (wn) {
          constexpr int W1 = D % 64 == 0 ? 64 : 48;
          // one head per tile: this group's columns only (its pairs' two halves), the partner warp's
          // partial sum comes through shared memory; otherwise the whole head
          constexpr bool kSplitSum = C::HPT == 1 && D / 4 == W1;
          float ss = 0.f;
#pragma unroll 1
          for (int c = kSplitSum ? pair0 : 0; c < D; c += kSplitSum ? D / 2 : W1) {
            uint32_t v[W1];
            if constexpr (W1 == 64)
              tmem_ld64(tbase + col0 + (uint32_t)c, v);
            else
              tmem_ld48(tbase + col0 + (uint32_t)c, v);
#pragma unroll
            for (int i0 = 0; i0 < W1; i0 += 16) {
              float bb[16];
              lds16(bias + c + i0, bb);
              if (wsc) {
                float ws[16];
                ldg16(wsc + c + i0, ws);
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                  const float x = fmaf(__uint_as_float(v[i0 + i]), ws[i], bb[i]);
                  ss = fmaf(x, x, ss);
                }
              } else {
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                  const float x = __uint_as_float(v[i0 + i]) + bb[i];
                  ss = fmaf(x, x, ss);
                }
              }
            }
          }
          if constexpr (kSplitSum) {
            // publish, wait (bounded) for the partner warp's partial of the same tile, add in group order
            const int slot = (t & 1) * 256;
            xss[slot + ew * 32 + lane] = ss;
            __threadfence_block();
            xflag[ew * 32 + lane] = t + 1;
            const int pw = ew ^ 4;
            bool seen = xflag[pw * 32 + lane] >= t + 1;
            if (!seen) {
              const uint64_t t0 = globaltimer_ns();
              while (!(seen = xflag[pw * 32 + lane] >= t + 1)) {
                if (*abort_flag) break;
                if (globaltimer_ns() - t0 > to) {
                  *abort_flag = 1;
                  atomicCAS(p.err, 0, kErrTimeoutProjection);
                  break;
                }
              }
            }
            if (!__all_sync(0xffffffffu, seen)) {
              aborted = true;
              break;
            }
            __threadfence_block();
            const float mine = ss, other = xss[slot + pw * 32 + lane];
            ss = group == 0 ? mine + other : other + mine;
          }
          rn = rsqrtf(ss / (float)D + p.eps);
        }
        __nv_bfloat16* dst;
        if (part == 0)
          dst = p.q_prime + (((int64_t)bl * p.Hq + h) * p.Lq_pad + r) * D;
        else
          dst = p.kv_packed + ((int64_t)bl * p.Lk_pad + key) * p.kv_ld + (part == 2 ? (int64_t)p.Hkv * D : 0) +
                (int64_t)h * D;
        // pass 2: pairs (i, i + D/2) of this group: bias, norm weight, RoPE, bf16
#pragma unroll
        for (int c = 0; c < D / 2; c += 16) {
          if (c < pair0 || c >= pair1) continue;
          // the RoPE pairs' cos / sin first: their global loads are then in flight during the TMEM wait
          float cc[16], sn[16];
          if (rope_w) {
            const bool ok = wait_bounded(&tbar[ew], t_done & 1, abort_flag, p.err, kErrTimeoutProjection, to);
            if (!__all_sync(0xffffffffu, ok)) {
              aborted = true;
              break;
            }
            ++t_done;
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              // the 64-byte swizzle XORs the 16-byte chunk index with bits 1-2 of the row
              const int phys = k ^ ((lane >> 1) & 3);
              const float4 c4 = *reinterpret_cast<const float4*>(tbuf + lane * 64 + phys * 16);
              const float4 s4 = *reinterpret_cast<const float4*>(tbuf + kTableWarpBytes / 2 + lane * 64 + phys * 16);
              cc[4 * k] = c4.x; cc[4 * k + 1] = c4.y; cc[4 * k + 2] = c4.z; cc[4 * k + 3] = c4.w;
              sn[4 * k] = s4.x; sn[4 * k + 1] = s4.y; sn[4 * k + 2] = s4.z; sn[4 * k + 3] = s4.w;
            }
            __syncwarp();
            if (c + 16 < pair1) {
              if (lane == 0) issue_table(c + 16, tr0);
              ++t_issued;
            }
          } else if (rope && !cs_tma) {
            const float4* cp = reinterpret_cast<const float4*>(p.cs + (int64_t)rrow * (D / 2) + c);
            const float4* sp = reinterpret_cast<const float4*>(p.cs + p.sin_off + (int64_t)rrow * (D / 2) + c);
#pragma unroll
            for (int q4 = 0; q4 < 4; ++q4) {
              const float4 c4 = __ldg(cp + q4), s4 = __ldg(sp + q4);
              cc[4 * q4] = c4.x; cc[4 * q4 + 1] = c4.y; cc[4 * q4 + 2] = c4.z; cc[4 * q4 + 3] = c4.w;
              sn[4 * q4] = s4.x; sn[4 * q4 + 1] = s4.y; sn[4 * q4 + 2] = s4.z; sn[4 * q4 + 3] = s4.w;
            }
          }
          uint32_t v1[16], v2[16];
          tmem_ld16_pair(tbase + col0 + (uint32_t)c, tbase + col0 + (uint32_t)(c + D / 2), v1, v2);
          float x1[16], x2[16], b1[16], b2[16];
          lds16(bias + c, b1);
          lds16(bias + D / 2 + c, b2);
          if (wsc) {
            float s1[16], s2[16];
            ldg16(wsc + c, s1);
            ldg16(wsc + D / 2 + c, s2);
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              x1[i] = fmaf(__uint_as_float(v1[i]), s1[i], b1[i]);
              x2[i] = fmaf(__uint_as_float(v2[i]), s2[i], b2[i]);
            }
          } else {
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              x1[i] = __uint_as_float(v1[i]) + b1[i];
              x2[i] = __uint_as_float(v2[i]) + b2[i];
            }
          }
          if (wn) {
            lds16(wn + c, b1);
            lds16(wn + D / 2 + c, b2);
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              x1[i] *= rn * b1[i];
              x2[i] *= rn * b2[i];
            }
          }
          if (rot) {
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              const float xa = x1[i], xc = x2[i];
              x1[i] = xa * cc[i] - xc * sn[i];
              x2[i] = xc * cc[i] + xa * sn[i];
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
        if (aborted) break;
      }
      if (aborted) break;
      // the accumulator has been read: the issuer may start the tile after next in it
      tc_fence_before();
      mbar_arrive(&acc_empty[a]);
      ++t;
    }
    // a table load still in flight (the CTA gave up) lands before the CTA's shared memory goes away
    if (t_issued > t_done && lane == 0) wait_drain(&tbar[ew], t_done & 1, to);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

template <int D>
cudaError_t launch_proj_d(ProjParams p, const CUtensorMap* tmX, const CUtensorMap* tmW, const CUtensorMap* tmCS,
                          const CUtensorMap* tmT, const CUtensorMap* tmL, cudaStream_t stream) {
  using C = ProjCfg<D>;
  const int sms = device_sm_count();
  long long tiles = 0;
  size_t bias_bytes = 0;
  for (int s = 0; s < p.n_sets; ++s) {
    tiles += (long long)p.B * p.set[s].m_tiles * p.set[s].n_tiles;
    bias_bytes += (size_t)p.set[s].n_tiles * C::NT * 4;
  }
  if (tiles <= 0) return cudaSuccess;
  if (tiles > 0x7FFFFFFFLL) return cudaErrorInvalidValue;
  // ring depth: as many stages (up to 5) as fit beside the bias vectors, the norm weights, the
  // barriers and the alignment slack
  if (!C::kTableTma || !tmCS) p.cs_tma = 0;
  // the table buffers take shared memory only while a ring of two or more stages still fits
  if (p.cs_tma && (232448 - (long long)(1024 + kTableBytes + bias_bytes + 2 * D * 4 + 3 * 256 * 4 + 256)) / C::STAGE < 2)
    p.cs_tma = 0;
  const size_t fixed = 1024 + (p.cs_tma ? kTableBytes : 0) + bias_bytes + 2 * D * 4 + 3 * 256 * 4 + 256;
  const long long room = 232448 - (long long)fixed;
  int stages = room > 0 ? (int)(room / C::STAGE) : 0;
  if (stages > 5) stages = 5;
  if (stages < 2) return cudaErrorNotSupported;
  p.stages = stages;
  const size_t smem = fixed + (size_t)stages * C::STAGE;
  // the limit is raised once per device to the whole 227 KB, so launches of different sizes from
  // several host threads never race on the attribute
  static DeviceOnce once;
  cudaError_t e = once_per_device(once, [] {
    return cudaFuncSetAttribute(proj_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, 232448);
  });
  if (e != cudaSuccess) return e;
  const int grid = tiles < sms ? (int)tiles : sms;
  const int s1 = p.n_sets > 1 ? 1 : 0;
  // sets without a LoRA pass their x / W maps in the T / B_cat slots (never loaded)
  proj_kernel<D><<<grid, kProjThreads, smem, stream>>>(
      tmX[0], tmW[0], tmX[s1], tmW[s1], p.cs_tma ? *tmCS : tmX[0], p.set[0].lora_steps ? tmT[0] : tmX[0],
      p.set[0].lora_steps ? tmL[0] : tmW[0], p.set[s1].lora_steps ? tmT[s1] : tmX[s1],
      p.set[s1].lora_steps ? tmL[s1] : tmW[s1], p);
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

cudaError_t launch_projection(ProjParams p, int D, const CUtensorMap* tmX, const CUtensorMap* tmW,
                              const CUtensorMap* tmCS, const CUtensorMap* tmT, const CUtensorMap* tmL,
                              cudaStream_t stream) {
  switch (D) {
    case 64: return launch_proj_d<64>(p, tmX, tmW, tmCS, tmT, tmL, stream);
    case 96: return launch_proj_d<96>(p, tmX, tmW, tmCS, tmT, tmL, stream);
    case 128: return launch_proj_d<128>(p, tmX, tmW, tmCS, tmT, tmL, stream);
    case 256: return launch_proj_d<256>(p, tmX, tmW, tmCS, tmT, tmL, stream);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace nsa
