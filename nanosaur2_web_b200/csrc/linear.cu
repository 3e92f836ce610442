// Linear layer for sm_100a with the reference's GEMM epilogue: ops.linear (app/gpu/ops.js:50-66)
// over the tiled GEMM of app/gpu/gemm.js, whose epilogue (gemm.js:155-165) is
//   r = alpha * acc (* rowScale[n] for int8 weights) (+ bias[n]) (+ LoRA delta) (silu), then
//   C = r, C += r, or C += gate[gOff + n] * r (in place).
// The DiT block's output projection is the gated form: x += gate * (a @ W_proj^T + b)
// (app/models/nanosaur2.js:210; tools/reference.py:285).  A is bf16, W bf16 or int8 (the ConvRot
// weights, whose input A the caller has rotated: ops.js:34-38, 54), both in the Linear layout
// [N][K]; C is fp32 (the reference's residual stream) or bf16 for the store form.
//
// CTA (one per SM, persistent over 128 x 256 output tiles), the QKV projection's structure:
//   warp 0      TMA producer: A [128 rows][64] and W [256 rows][64] slices through a ring
//   warp 1      TMEM allocator + MMA issuer: 128 x 256 x 16 tcgen05.mma into one of two accumulators
// With bf16 weights two CTAs on two SMs (a cluster) share each 256 x 256 tile instead: each loads its
// own 128 rows of A and 128 of the tile's 256 W rows, and the even CTA issues M = 256 cta_group::2 MMAs
// that read both CTAs' shared memory and write each CTA's 128 accumulator rows into its own tensor
// memory.  Per SM and K slice the ring then carries 32 KB instead of 48 for the same MMA work, which
// the operand traffic through shared memory (TMA writes plus MMA reads) had bounded at 128 x 256.
//   warps 2-9   epilogue, two groups of four warps, each group half of the tile's columns; a thread
//               owns one output row of 32 (fp32) or 64 (bf16) columns at a time: alpha, row scale,
//               bias, silu, gate, then the row goes into the warp's 128-byte-swizzled staging rows and
//               one lane hands the [32 rows][128 bytes] box to the TMA: a tiled store, or for the
//               residual forms an fp32 add-reduce into C performed in L2 (the reference's in-place
//               C += gate * r).  Rows and columns past M / N are clipped by the tensor map.
//   warps 10-13 (int8 weights only) converters: each int8 W slice lands beside the stage's bf16 slot
//               and is rewritten there as the bf16 operand (wconv.cuh) before the MMA reads it.
//
// LoRA side paths (ops.js:55-57, 70-86: delta = sum_i scale_i B_i (A_i x), added before the
// activation) run as extra K steps of the same accumulation: after the K/64 slices of A and W come
// the slices of T = x A_cat^T [M][R] (one small GEMM before this one) against B_cat [N][R], whose rows
// hold scale_i B_i / (alpha * rowScale[n]) (nsa_lora_pack), so that the epilogue's alpha * rowScale
// multiplies the delta back to scale_i B_i (A_i x).
#include "nsa_internal.h"
#include "act.cuh"
#include "ptx.cuh"
#include "wconv.cuh"

namespace nsa {

namespace {

constexpr int kLinBK = 64;
constexpr int kLinNT = 256;
constexpr int kLinA = 128 * kLinBK * 2;
constexpr int kLinB = kLinNT * kLinBK * 2;
constexpr int kLinB8 = kLinNT * kLinBK;   // int8 W slice
constexpr uint32_t kLinIdesc = idesc_bf16_f32(128, kLinNT, 0, 0);
constexpr uint32_t kLinIdescPair = idesc_bf16_f32(256, kLinNT, 0, 0);
constexpr uint32_t kLinIdescPairHalf = idesc_bf16_f32(256, kLinNT / 2, 0, 0);
// a last column tile with at most 128 columns inside N (te.o and the MLP's down projection at N = 640)
// multiplies only its first 128 W rows: half the MMA time of that tile
constexpr uint32_t kLinIdescHalf = idesc_bf16_f32(128, kLinNT / 2, 0, 0);

// A stage holds ATOMS K slices of 64 (one 128-byte swizzle row each) of A and of this CTA's W rows,
// atom j of A at j * A_ATOM and of W at A_BYTES + j * B_ATOM.  CTA pairs take 128-wide K steps: eight
// MMAs per barrier wait and commit of the issuing thread, whose per-step overhead (wait, commit,
// bookkeeping) otherwise leaves the tensor pipe idle between steps; single CTAs keep 64-wide steps,
// which leave room for a four-stage ring.
template <bool I8, bool PAIR>
struct LinCfg {
  static_assert(!(I8 && PAIR), "int8 weights run on single CTAs");
  static constexpr int THREADS = I8 ? 448 : 320;
  static constexpr int ATOMS = PAIR ? 2 : 1;
  static constexpr int BK = 64 * ATOMS;
  static constexpr int BROWS = PAIR ? kLinNT / 2 : kLinNT;   // W rows per CTA
  static constexpr int A_ATOM = 128 * 128, B_ATOM = BROWS * 128;
  static constexpr int A_BYTES = ATOMS * A_ATOM, B_BYTES = ATOMS * B_ATOM;
  // 48 KB single, 64 KB per CTA of a pair, 64 KB for int8 (the bf16 W slot plus the int8 landing slot)
  static constexpr int STAGE = A_BYTES + B_BYTES + (I8 ? kLinB8 : 0);
  static constexpr int STAGES = I8 ? 3 : (PAIR ? 3 : 4);
  static_assert(STAGE % 1024 == 0, "stage alignment");
  static_assert(!I8 || (A_BYTES == kLinA && B_BYTES == kLinB), "int8 stage layout");
};
constexpr int kLinStaging = 8 * 4096;   // one [32 rows][128 bytes] staging box per epilogue warp

__device__ __forceinline__ float silu(float x) { return x / (1.f + expf(-x)); }

template <bool I8, bool PAIR>
__global__ void __launch_bounds__(LinCfg<I8, PAIR>::THREADS, 1)
    linear_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmW,
                  const __grid_constant__ CUtensorMap tmT, const __grid_constant__ CUtensorMap tmL,
                  const __grid_constant__ CUtensorMap tmC, const LinearParams p) {
  using Cfg = LinCfg<I8, PAIR>;
  constexpr int S = Cfg::STAGES;
  constexpr int STAGE = Cfg::STAGE;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* staging = smem + S * STAGE;                               // [8 warps][32 rows][128 bytes]
  uint64_t* full = reinterpret_cast<uint64_t*>(staging + kLinStaging);
  uint64_t* empty = full + S;
  uint64_t* conv = empty + S;           // int8: the stage's bf16 W slot is written (4 converter warps)
  uint64_t* acc_full = conv + S;
  uint64_t* acc_empty = acc_full + 2;   // 256 epilogue arrivals (a pair: one per epilogue warp of both CTAs)
  uint64_t* drain = acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const uint64_t to = p.timeout_ns;
  // K steps per tile: the main ones over A and W, then the LoRA ones over T and B_cat
  const int ksteps = (p.k_steps + Cfg::ATOMS - 1) / Cfg::ATOMS;
  const int steps = ksteps + (p.lora_steps + Cfg::ATOMS - 1) / Cfg::ATOMS;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
      mbar_init(&conv[s], 4);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], PAIR ? 16 : 256);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    if constexpr (PAIR) {
      tmem_alloc_pair(tmem_slot, 512);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(tmem_slot, 512);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  if constexpr (PAIR)
    cluster_sync();   // both CTAs' barriers exist before either signals the other's
  else
    __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // work units: 128-row tiles, or 256-row tiles of a CTA pair (this CTA: rows rank * 128 .. + 127)
  const uint32_t rank = PAIR ? cluster_ctarank() : 0u;
  constexpr int MU = PAIR ? 256 : 128;
  const int tiles = (PAIR ? (p.m_tiles + 1) / 2 : p.m_tiles) * p.n_tiles;
  const int G = PAIR ? (int)gridDim.x / 2 : (int)gridDim.x;
  const int u0 = PAIR ? (int)blockIdx.x / 2 : (int)blockIdx.x;
  // a pair's last column tile with at most 128 columns inside N: N = 128 MMAs whose B rows come 64
  // from each CTA (W rows n0 .. n0+63 and n0+64 .. n0+127)
  auto half_tile = [&](int nt) { return p.N - nt * kLinNT <= kLinNT / 2; };

  if (warp == 0) {
    // ---------------------------------------------------------------- TMA producer
    if (lane == 0) {
      tma_prefetch_desc(&tmA);
      tma_prefetch_desc(&tmW);
      tma_prefetch_desc(&tmC);
      if (p.lora_steps) {
        tma_prefetch_desc(&tmT);
        tma_prefetch_desc(&tmL);
      }
      int step = 0;
      bool ok = true;
      for (int u = u0; ok && u < tiles; u += G) {
        const int nt = u % p.n_tiles, m0 = (u / p.n_tiles) * MU + (int)rank * 128;
        for (int ks = 0; ks < steps; ++ks, ++step) {
          const int s = step % S;
          if (step >= S && !wait_bounded(&empty[s], ((step / S) - 1) & 1, abort_flag, p.err, kErrTimeoutProjection, to)) {
            ok = false;
            break;
          }
          uint8_t* st = smem + s * STAGE;
          if constexpr (!I8) {
            // atoms of A (or T) and of this CTA's W (or B_cat) rows; a pair's boxes all complete on the
            // rank-0 CTA's barrier, which expects both CTAs' bytes
            const bool main = ks < ksteps;
            const CUtensorMap* ma = main ? &tmA : &tmT;
            const CUtensorMap* mw = main ? &tmW : &tmL;
            const int kx = (main ? ks : ks - ksteps) * Cfg::BK;
            const int brow = nt * kLinNT + (PAIR ? (int)rank * (half_tile(nt) ? kLinNT / 4 : kLinNT / 2) : 0);
            if constexpr (PAIR) {
              const uint32_t fbar = mapa_shared(&full[s], 0);
              if (rank == 0) mbar_arrive_expect_tx(&full[s], 2 * STAGE);
#pragma unroll
              for (int j = 0; j < Cfg::ATOMS; ++j) {
                tma_load_2d_pair(st + j * Cfg::A_ATOM, ma, fbar, kx + 64 * j, m0);
                tma_load_2d_pair(st + Cfg::A_BYTES + j * Cfg::B_ATOM, mw, fbar, kx + 64 * j, brow);
              }
            } else {
              mbar_arrive_expect_tx(&full[s], STAGE);
#pragma unroll
              for (int j = 0; j < Cfg::ATOMS; ++j) {
                tma_load_2d(st + j * Cfg::A_ATOM, ma, &full[s], kx + 64 * j, m0);
                tma_load_2d(st + Cfg::A_BYTES + j * Cfg::B_ATOM, mw, &full[s], kx + 64 * j, brow);
              }
            }
          } else if (ks < ksteps) {
            mbar_arrive_expect_tx(&full[s], kLinA + (I8 ? kLinB8 : kLinB));
            tma_load_2d(st, &tmA, &full[s], ks * kLinBK, m0);
            tma_load_2d(st + kLinA + (I8 ? kLinB : 0), &tmW, &full[s], ks * kLinBK, nt * kLinNT);
          } else {   // int8 weights' LoRA slices: T rows against B_cat rows, straight into the bf16 slots
            mbar_arrive_expect_tx(&full[s], kLinA + kLinB);
            tma_load_2d(st, &tmT, &full[s], (ks - ksteps) * kLinBK, m0);
            tma_load_2d(st + kLinA, &tmL, &full[s], (ks - ksteps) * kLinBK, nt * kLinNT);
          }
        }
      }
      // boxes still in flight (a CTA that gave up) land before shared memory goes away; a pair's
      // complete on the rank-0 CTA's barriers, which track both CTAs' boxes
      if (rank == 0)
        for (int i = step > S ? step - S : 0; i < step; ++i) wait_drain(&full[i % S], (i / S) & 1, to);
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer (rank 0 of a pair)
    if (lane == 0 && rank == 0) {
      int step = 0, t = 0;
      bool ok = true;
      // a pair's commits arrive on the barrier of the same offset in each CTA
      auto commit = [&](uint64_t* bar) {
        if constexpr (PAIR) {
          tc_commit_pair(mapa_shared(bar, 0));
          tc_commit_pair(mapa_shared(bar, 1));
        } else {
          tc_commit(bar);
        }
      };
      for (int u = u0; ok && u < tiles; u += G) {
        const int a = t & 1;
        if (t >= 2 && !wait_bounded(&acc_empty[a], ((t >> 1) - 1) & 1, abort_flag, p.err, kErrTimeoutProjection, to)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem + (uint32_t)a * 256u;
        const bool half = half_tile(u % p.n_tiles);
        const uint32_t idesc = PAIR ? (half ? kLinIdescPairHalf : kLinIdescPair) : (half ? kLinIdescHalf : kLinIdesc);
        // the stage's barrier was peeked at (non-blocking) before the previous step's MMAs; only a
        // stage that was not ready then costs a blocking wait here
        bool ready = false;
        for (int ks = 0; ks < steps; ++ks, ++step) {
          const int s = step % S;
          uint64_t* fb = I8 ? &conv[s] : &full[s];
          if (!ready && !wait_bounded(fb, (step / S) & 1, abort_flag, p.err, kErrTimeoutProjection, to)) {
            ok = false;
            break;
          }
          if (ks + 1 < steps) {
            const int s1 = (step + 1) % S;
            ready = mbar_test_wait(I8 ? &conv[s1] : &full[s1], ((step + 1) / S) & 1);
          }
          const uint32_t sa = smem_u32(smem + s * STAGE);
          const uint64_t da0 = smem_desc(sa, 16, 1024, 2), db0 = smem_desc(sa + Cfg::A_BYTES, 16, 1024, 2);
#pragma unroll
          for (int kk = 0; kk < Cfg::BK / 16; ++kk) {
            // descriptor start addresses in 16-byte units: atom kk / 4, 32 bytes per K step of 16 inside it
            const uint64_t da = da0 + (uint64_t)(((kk >> 2) * Cfg::A_ATOM + (kk & 3) * 32) >> 4);
            const uint64_t db = db0 + (uint64_t)(((kk >> 2) * Cfg::B_ATOM + (kk & 3) * 32) >> 4);
            if constexpr (PAIR)
              mma_ss_pair(d_tmem, da, db, idesc, (ks > 0 || kk > 0) ? 1u : 0u);
            else
              mma_ss(d_tmem, da, db, idesc, (ks > 0 || kk > 0) ? 1u : 0u);
          }
          commit(&empty[s]);
        }
        if (!ok) break;
        commit(&acc_full[a]);
        ++t;
      }
      if (!ok) {
        if constexpr (PAIR)
          tc_commit_pair(mapa_shared(drain, 0));
        else
          tc_commit(drain);
        wait_drain(drain, 0, to);
      }
    }
  } else if (warp < 10) {
    // ---------------------------------------------------------------- epilogue (warps 2-9)
    const int group = (warp - 2) / 4;
    const int quarter = warp % 4;
    uint8_t* stg = staging + (warp - 2) * 4096;
    const bool f32_out = p.C16 == nullptr;
    int t = 0;
    // the accumulator has been read: this warp's share of the release (a pair: one arrival per warp on
    // the rank-0 CTA's barrier, after every lane's loads)
    auto release_acc = [&](int a) {
      tc_fence_before();
      if constexpr (PAIR) {
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(mapa_shared(&acc_empty[a], 0));
      } else {
        mbar_arrive(&acc_empty[a]);
      }
    };
    for (int u = u0; u < tiles; u += G) {
      const int nt = u % p.n_tiles, m0 = (u / p.n_tiles) * MU + (int)rank * 128;
      const int a = t & 1;
      const bool got = wait_bounded(&acc_full[a], (t >> 1) & 1, abort_flag, p.err, kErrTimeoutProjection, to);
      if (!__all_sync(0xffffffffu, got)) break;
      tc_fence_after();
      const uint32_t tbase = tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)a * 256u;
      const int row0 = m0 + quarter * 32;   // this warp's 32 rows (TMEM lanes)
      if (p.glu) {
        // Fused GLU (ops.glu after the gate_up linear, gemma3.js:80-81): with the weight rows
        // interleaved per tile (nsa_glu_interleave), accumulator column c < 128 is the gate and 128 + c
        // the up projection of output feature 128 * nt + c.  Group g writes features 64g .. 64g + 63:
        // y = act(gate) * up in fp32, then one 64-column bf16 box, or two 32-column fp32 boxes.
        const int f0 = nt * 128 + group * 64;   // first output column of this warp's box(es)
        const int n_out = p.N / 2;
        if (f0 < n_out && row0 < p.M) {
#pragma unroll 1
          for (int h = 0; h < 2; ++h) {
            const int cg = group * 64 + h * 32;   // gate column in the tile; up at 128 + cg
            uint32_t gv[32], uv[32];
            tmem_ld32(tbase + (uint32_t)cg, gv);
            tmem_ld32(tbase + 128u + (uint32_t)cg, uv);
            if (f32_out || h == 0) {   // the staging rows are free once the previous box has been read
              if (lane == 0) bulk_wait_read_all();
              __syncwarp();
            }
            uint8_t* row = stg + lane * 128;
#pragma unroll
            for (int q = 0; q < 8; ++q) {   // four features at a time
              const int ng = nt * kLinNT + cg + 4 * q;   // interleaved weight rows of the gate / up values
              const float4 bg = p.bias ? __ldg(reinterpret_cast<const float4*>(p.bias + ng)) : make_float4(0.f, 0.f, 0.f, 0.f);
              const float4 bu = p.bias ? __ldg(reinterpret_cast<const float4*>(p.bias + ng + 128)) : make_float4(0.f, 0.f, 0.f, 0.f);
              float4 mg = make_float4(p.alpha, p.alpha, p.alpha, p.alpha), mu = mg;
              if (I8 || p.w_scale) {
                const float4 rg = __ldg(reinterpret_cast<const float4*>(p.w_scale + ng));
                const float4 ru = __ldg(reinterpret_cast<const float4*>(p.w_scale + ng + 128));
                mg = make_float4(mg.x * rg.x, mg.y * rg.y, mg.z * rg.z, mg.w * rg.w);
                mu = make_float4(mu.x * ru.x, mu.y * ru.y, mu.z * ru.z, mu.w * ru.w);
              }
              const float bgv[4] = {bg.x, bg.y, bg.z, bg.w}, buv[4] = {bu.x, bu.y, bu.z, bu.w};
              const float mgv[4] = {mg.x, mg.y, mg.z, mg.w}, muv[4] = {mu.x, mu.y, mu.z, mu.w};
              float y[4];
#pragma unroll
              for (int i = 0; i < 4; ++i) {
                const float g = mgv[i] * __uint_as_float(gv[4 * q + i]) + bgv[i];
                const float up = muv[i] * __uint_as_float(uv[4 * q + i]) + buv[i];
                y[i] = (p.glu == 1 ? glu_act<0>(g) : glu_act<1>(g)) * up;
              }
              if (f32_out) {
                *reinterpret_cast<uint4*>(row + ((q ^ (lane & 7)) << 4)) =
                    make_uint4(__float_as_uint(y[0]), __float_as_uint(y[1]), __float_as_uint(y[2]), __float_as_uint(y[3]));
              } else {   // bf16: features 4q .. 4q+3 of this half are half a 16-byte chunk
                const int c = h * 4 + q / 2;
                uint2* dst = reinterpret_cast<uint2*>(row + ((c ^ (lane & 7)) << 4) + (q & 1) * 8);
                *dst = make_uint2(pack_bf16x2(y[0], y[1]), pack_bf16x2(y[2], y[3]));
              }
            }
            if (f32_out || h == 1) {
              fence_proxy_async_smem();
              __syncwarp();
              if (lane == 0) {
                tma_store_2d(&tmC, stg, f32_out ? f0 + h * 32 : f0, row0);
                bulk_commit_group();
              }
            }
          }
        }
        release_acc(a);
        ++t;
        continue;
      }
#pragma unroll 1
      for (int c64 = group * 128; c64 < group * 128 + 128; c64 += 64) {
        const int n64 = nt * kLinNT + c64;
        if (n64 >= p.N) break;   // warp-uniform: nothing of this chunk is inside C
        uint32_t v[64];
        tmem_ld64(tbase + (uint32_t)c64, v);
#pragma unroll
        for (int h = 0; h < 2; ++h) {   // fp32: two boxes of 32 columns; bf16: one box of 64
          if (!f32_out && h == 1) break;
          const int n0 = n64 + h * 32;
          if (n0 >= p.N || row0 >= p.M) continue;
          // the previous box of this warp must have left the staging rows
          if (lane == 0) bulk_wait_read_all();
          __syncwarp();
          uint8_t* row = stg + lane * 128;
#pragma unroll
          for (int c = 0; c < 8; ++c) {   // 16-byte chunk c of the row, at position c ^ (row & 7)
            float y[8];
#pragma unroll
            for (int g4 = 0; g4 < 2; ++g4) {   // columns in fours: bias, row scale, gate (zero / one past N)
              if (f32_out && g4 == 1) break;
              const int j0 = f32_out ? 4 * c : 8 * c + 4 * g4;   // first column of the four within the box
              const int n = n0 + j0;
              const bool in = n < p.N;
              const float4 bb = in && p.bias ? __ldg(reinterpret_cast<const float4*>(p.bias + n)) : make_float4(0.f, 0.f, 0.f, 0.f);
              float4 mm = make_float4(p.alpha, p.alpha, p.alpha, p.alpha);
              if ((I8 || p.w_scale) && in) {
                const float4 rs = __ldg(reinterpret_cast<const float4*>(p.w_scale + n));
                mm = make_float4(mm.x * rs.x, mm.y * rs.y, mm.z * rs.z, mm.w * rs.w);
              }
              const float4 gg = in && p.gate ? __ldg(reinterpret_cast<const float4*>(p.gate + n)) : make_float4(1.f, 1.f, 1.f, 1.f);
              const float bv[4] = {bb.x, bb.y, bb.z, bb.w}, mv[4] = {mm.x, mm.y, mm.z, mm.w}, gv[4] = {gg.x, gg.y, gg.z, gg.w};
#pragma unroll
              for (int i = 0; i < 4; ++i) {
                // both candidate indices are compile-time constants (no local-memory copy of v)
                const uint32_t acc = f32_out ? v[h * 32 + 4 * c + i] : v[(8 * c + 4 * g4 + i) & 63];
                float x = mv[i] * __uint_as_float(acc) + bv[i];
                if (p.act == 1) x = silu(x);
                y[4 * g4 + i] = p.resid ? gv[i] * x : x;
              }
            }
            const uint4 w = f32_out ? make_uint4(__float_as_uint(y[0]), __float_as_uint(y[1]), __float_as_uint(y[2]),
                                                 __float_as_uint(y[3]))
                                    : make_uint4(pack_bf16x2(y[0], y[1]), pack_bf16x2(y[2], y[3]), pack_bf16x2(y[4], y[5]),
                                                 pack_bf16x2(y[6], y[7]));
            *reinterpret_cast<uint4*>(row + ((c ^ (lane & 7)) << 4)) = w;
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            if (p.resid)
              tma_reduce_add_2d(&tmC, stg, n0, row0);
            else
              tma_store_2d(&tmC, stg, n0, row0);
            bulk_commit_group();
          }
        }
      }
      release_acc(a);
      ++t;
    }
    if (lane == 0) bulk_wait_all();
  } else if (I8) {
    // ---------------------------------------------------------------- int8 converters (warps 10-13)
    const int ct = threadIdx.x - 320;
    int step = 0;
    bool ok = true;
    for (int u = u0; ok && u < tiles; u += G) {
      for (int ks = 0; ks < steps; ++ks, ++step) {
        const int s = step % S;
        ok = __all_sync(0xffffffffu,
                        wait_bounded(&full[s], (step / S) & 1, abort_flag, p.err, kErrTimeoutProjection, to));
        if (!ok) break;
        uint8_t* st = smem + s * STAGE;
        if (ks < ksteps) convert_i8_slice<kLinNT, 128>(st + kLinA + kLinB, st + kLinA, ct);
        __syncwarp();
        if (lane == 0) mbar_arrive(&conv[s]);
      }
    }
  }
  tc_fence_before();
  if constexpr (PAIR)
    cluster_sync();   // neither CTA leaves while the other may still touch its shared or tensor memory
  else
    __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    if constexpr (PAIR)
      tmem_dealloc_pair(tmem, 512);
    else
      tmem_dealloc(tmem, 512);
  }
}

template <bool I8, bool PAIR>
constexpr size_t linear_smem() {
  return 1024 + (size_t)LinCfg<I8, PAIR>::STAGES * LinCfg<I8, PAIR>::STAGE + kLinStaging + 256;
}
static_assert(linear_smem<false, false>() <= 232448 && linear_smem<true, false>() <= 232448 &&
                  linear_smem<false, true>() <= 232448,
              "shared memory");

template <bool I8, bool PAIR>
cudaError_t launch_linear_t(const LinearParams& p, const CUtensorMap& tmA, const CUtensorMap& tmW,
                            const CUtensorMap& tmT, const CUtensorMap& tmL, const CUtensorMap& tmC,
                            cudaStream_t stream) {
  const int sms = device_sm_count();
  const long long tiles = (long long)(PAIR ? (p.m_tiles + 1) / 2 : p.m_tiles) * p.n_tiles;
  if (tiles <= 0) return cudaSuccess;
  if (tiles > 0x7FFFFFFFLL) return cudaErrorInvalidValue;
  constexpr size_t smem = linear_smem<I8, PAIR>();
  // the limit is raised once per device to the whole 227 KB, so launches of different sizes from
  // several host threads never race on the attribute; a pair kernel also records how many of its
  // two-CTA clusters fit on the device at once (the persistent grid must not exceed it)
  static DeviceOnce once;
  static int max_clusters[128];
  cudaError_t e = once_per_device(once, [] {
    cudaError_t r = cudaFuncSetAttribute(linear_kernel<I8, PAIR>, cudaFuncAttributeMaxDynamicSharedMemorySize, 232448);
    if (r != cudaSuccess || !PAIR) return r;
    int dev = 0;
    if ((r = cudaGetDevice(&dev)) != cudaSuccess) return r;
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.gridDim = dim3(2 * (unsigned)device_sm_count());
    cfg.blockDim = dim3(LinCfg<I8, PAIR>::THREADS);
    cfg.dynamicSmemBytes = linear_smem<I8, PAIR>();
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    r = cudaOccupancyMaxActiveClusters(&n, linear_kernel<I8, PAIR>, &cfg);
    if (r == cudaSuccess && n < 1) r = cudaErrorNotSupported;
    if (r == cudaSuccess) max_clusters[dev & 127] = n;
    return r;
  });
  if (e != cudaSuccess) return e;
  if constexpr (PAIR) {
    int dev = 0;
    if ((e = cudaGetDevice(&dev)) != cudaSuccess) return e;
    const int mc = max_clusters[dev & 127];
    const int clusters = tiles < mc ? (int)tiles : mc;
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.gridDim = dim3(2 * (unsigned)clusters);
    cfg.blockDim = dim3(LinCfg<I8, PAIR>::THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, linear_kernel<I8, PAIR>, tmA, tmW, tmT, tmL, tmC, p);
  } else {
    const int grid = tiles < sms ? (int)tiles : sms;
    linear_kernel<I8, PAIR><<<grid, LinCfg<I8, PAIR>::THREADS, smem, stream>>>(tmA, tmW, tmT, tmL, tmC, p);
    return cudaGetLastError();
  }
}

}  // namespace

cudaError_t launch_linear(const LinearParams& p, const CUtensorMap& tmA, const CUtensorMap& tmW, const CUtensorMap& tmT,
                          const CUtensorMap& tmL, const CUtensorMap& tmC, cudaStream_t stream) {
  if (p.w_i8) return launch_linear_t<true, false>(p, tmA, tmW, tmT, tmL, tmC, stream);
  return p.pair ? launch_linear_t<false, true>(p, tmA, tmW, tmT, tmL, tmC, stream)
                : launch_linear_t<false, false>(p, tmA, tmW, tmT, tmL, tmC, stream);
}

}  // namespace nsa
