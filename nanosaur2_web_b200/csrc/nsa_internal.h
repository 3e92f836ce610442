// Private interface between the C ABI (api.cu) and the kernels (prologue.cu, attention.cu).
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

namespace nsa {

constexpr int kTileM = 128;  // query rows per tensor-core tile (one TMEM lane per row)
constexpr int kTileN = 128;  // keys per K/V tile

// One strided input matrix: element (b, row, col) lives at ptr[b*bstride + row*ld + off + col];
// each batch element holds `rows` rows.
struct RowView {
  const void* ptr;
  int64_t ld;
  int64_t bstride;
  int64_t off;
  int64_t rows;
};

constexpr int kMaxPeers = 8;   // GPUs of one box a sequence-sharded prologue writes to

// Destination of prepared bf16 rows: element (local batch bl, local head h, produced row r, d) at
// ptr[bl*bs + h*hs + r*rs + d].  Head-major tiles: hs = pad*D, rs = D; packed K|V rows: hs = D.
struct TileOut {
  __nv_bfloat16* ptr;
  int64_t bs, hs, rs;
};

// Prologue: raw rows -> bf16 tiles (rows padded with zeros), with the optional per-head RMSNorm and
// split-half RoPE of the query/key rows.  Part 0 = q, 1 = k, 2 = v.  Produced row r of part i is
// logical row row0[i] + r (its key / query index and RoPE table row), read from source row
// src_row0[i] + r.
struct PrologueParams {
  RowView q, k, v;
  int src_f32;          // 1: fp32 input, 0: bf16 input
  int B;                // batch elements handled (shard)
  int b_begin;          // first batch element of the shard
  int Lq, Lk;           // query rows, key rows per batch element
  int Hq, Hkv, D;       // heads in the shard
  int hq_begin, hkv_begin;
  const float* q_w;     // [D] or null (no norm)
  const float* k_w;     // [D] or null
  const float* cs;      // RoPE table: cos [rope_rows][D/2] then sin at sin_off; null = no RoPE
  int64_t sin_off;
  int rope_rows;        // rows [0, rope_rows) of q and k get RoPE
  float eps;
  const int* kv_len;    // [B_total] valid keys per batch element (null: Lk)
  TileOut out[3];
  int rows[3];          // rows produced per part (padded counts)
  int row0[3];          // logical row (query / key index, RoPE row) of produced row 0, per part
  int src_row0[3];      // row of the source buffer holding produced row 0, per part
  int skip_q;           // 1: no Q tiles (the attention kernel prepares Q itself)
  int* zero_ptr;        // zero_count ints cleared by the first block (the attention's split counters)
  int zero_count;
  // > 0: the attention kernel reads V straight from the input for key tiles of v_tile rows that
  // hold only valid keys; the prologue then writes V rows only from the first tile that does not
  // (the last partial tile and the padding, zero-filled).
  int v_tile;
  // k and v rows also go to n_peers further copies of their buffer: the destination plus
  // peer_off[i] bytes (another GPU's buffer mapped into this process; sequence shards).
  int n_peers;
  int64_t peer_off[kMaxPeers];
  // 1: the tiles are fp32 (the tf32 path; TileOut::ptr then points at floats and its strides count
  // floats); 0: bf16
  int out_f32;
};

struct AttnParams {
  int B, Hq, Hkv, group;   // shard sizes (B, Hq, Hkv) and query heads per kv head
  int b_begin, hq_begin;   // shard origin (output and per-batch inputs are indexed globally)
  int hkv_begin;           // first kv head held in the K/V tiles
  int Lq, Lq_pad, Lk, Lk_pad;
  // K / V tile (x, y) of local kv head h and key k: x = k_x0 (v_x0) + h*kv_xh + c*blk,
  // y = bl*kv_yb + h*kv_yh + k  (head-major tiles: x0 = xh = 0, yb = Hkv*Lk_pad, yh = Lk_pad)
  int k_x0, v_x0, kv_xh, kv_yb, kv_yh;
  const int* kv_len;       // [B_total] or null
  const float* bias;       // natural-log additive key bias for keys >= bias_start, or null
  int bias_start, bias_len;
  int64_t bias_bstride;
  float scale_log2;        // softmax scale * log2(e)
  int causal, window;
  void* out;
  int out_f32;
  int64_t out_ld, out_bstride, out_off;
  int q_blocks;            // query blocks (NQ tiles each) per (b, head)
  int* err;
  unsigned long long timeout_ns;
  // Query tile of the prologue's Q' tiles: box (x, y) with x = q_x0 + (head - q_h0)*q_xh + c*blk and
  // y = (b - q_b0)*q_yb + (head - q_h0)*q_yh + row.
  int q_x0, q_xh, q_yb, q_yh;
  int q_b0, q_h0;
  // Tail split (two query tiles per CTA, no causal mask or window): the work units from
  // split_first on (the last, partial wave) run as two CTAs each, one per half of the key tiles.
  // Each writes its unnormalised O and (m, l) per row to part_o / part_ml; whichever finishes
  // second (split_count) merges the halves and writes the output.  split_units = 0: no split.
  int split_first, split_units;
  float* part_o;         // [split_units][2][2 * 128][D]
  float* part_ml;        // [split_units][2][2 * 128][2]
  int* split_count;      // [split_units][2] (one per query tile), zero at launch (the prologue clears it)
  // V straight from the input (tmVd) for key tiles that hold only valid keys: box (x, y) with
  // x = vd_x0 + h*vd_xh + c*blk (h = local kv head), y = b*vd_yb + key (b = global batch index);
  // other tiles come from the prologue's V tiles (tmV).
  int v_direct, vd_x0, vd_xh, vd_yb;
};

// Work units at or above this count in the last wave are not split (bounds the partial-result
// scratch: half the SMs of a B200).
constexpr int kSplitUnitsMax = 74;

// Tile geometry of the attention kernel for a head dim.
struct AttnGeometry {
  int NQ;       // query tiles of 128 rows per CTA
  int BN;       // keys per K/V tile (TMA box rows)
  int blk;      // swizzle block width in elements (TMA box columns)
  bool qtmem;   // Q copied into tensor memory by the softmax threads (S = Q K^T reads it from there)
  int v_rows;   // rows of the V tiles' TMA box (BN, or the 32-key chunks of head dim 512)
  bool v_direct_ok;   // the kernel can read V straight from the input rows
};
AttnGeometry attention_geometry(int D);   // NQ = 0: unsupported head dim
// head dim 512 (attention_d512.cu): two CTAs per 128-row query tile, one per half of the output
// columns; no V-from-input path and no tail split
cudaError_t launch_attention_d512(const AttnParams& p, const CUtensorMap& tmQ, const CUtensorMap& tmK,
                                  const CUtensorMap& tmV, cudaStream_t stream);
int attention_d512_v_box_rows();
// persistent head-dim-256 kernel (attention_persist.cu): one CTA per SM looping over work units
cudaError_t launch_attention_persist(const AttnParams& p, const CUtensorMap& tmQ, const CUtensorMap& tmK,
                                     const CUtensorMap& tmV, const CUtensorMap& tmVd, cudaStream_t stream);
// the same persistent kernel at head dim 96 on fp32 Q' / K' / V' tiles with tf32 MMAs (the fp32 path
// whose tolerance is tighter than bf16); maps are fp32 boxes of [rows][32] with the 128-byte swizzle,
// the V map with 32-byte swizzle atoms (an MN-major tf32 operand needs that layout)
cudaError_t launch_attention_tf32(const AttnParams& p, const CUtensorMap& tmQ, const CUtensorMap& tmK,
                                  const CUtensorMap& tmV, cudaStream_t stream);

cudaError_t launch_prologue(const PrologueParams& p, cudaStream_t stream);

// QKV projection GEMM with the prologue in its epilogue (proj.cu): rows of X [.][K] times W^T
// ([N][K], q heads then k then v, or k then v for the text rows), + bias, then per head the q/k
// RMSNorm and split-half RoPE, written straight into the sequence-shard layouts: q' tiles
// [B][Hq][Lq_pad][D] and packed k'|v' rows [B][Lk_pad][2 Hkv D].  One launch covers up to two row
// sets (the image rows, then the text rows).  GEMM row r of set s and batch element bl is input row
// x_row0 + r of that set's X, query row r (image rows) and key row key_row0 + r.
struct ProjSet {
  int image;               // 1: q|k|v of the image rows; 0: k|v of the text rows
  int m_tiles, n_tiles;    // 128-row tiles per batch element, head-group tiles over N
  int rows;                // GEMM rows per batch element (Lq_pad or Lk_pad - L)
  int valid_q;             // image: query rows of the shard (rows past it are zeros in q')
  int key_row0;            // key index of GEMM row 0 (image: q_begin, text: L)
  int x_row0;              // input row of GEMM row 0
  int rope_row0;           // RoPE table row of GEMM row 0 (image: q_begin)
  const float* bias;       // [n_tiles * heads-per-tile * D] or null
  const float* w_scale;    // per-row weight scales (int8 ConvRot weights given as bf16) or null
  int lora_steps;          // 64-wide LoRA K slices after the K/64 of x and W (tmT / tmL of the set)
};
struct ProjParams {
  int B, b_begin;          // batch elements of the call and the first one's global index
  int k_steps;             // 64-element slices of K
  int Hq, Hkv;             // heads (whole model: sequence shards take whole heads)
  int Lk, Lq_pad, Lk_pad;  // keys; padded rows of q' and kv_packed
  int64_t kv_ld;           // elements per kv_packed row
  int n_sets;              // 1 or 2
  ProjSet set[2];
  int stages;              // depth of the shared-memory ring (chosen to fit beside the bias vectors)
  const float* q_w;        // [D] q RMSNorm weight
  const float* k_w;        // [D] k RMSNorm weight
  const float* cs;         // RoPE table (image rows): cos [rows][D/2], sin at sin_off; null = none
  int64_t sin_off;
  int cs_tma;              // head dim 256: the table is also mapped as tmCS ([2 cs_rows][128] fp32,
  int cs_rows;             //   box [32 rows][16], 64-byte swizzle) and staged per epilogue warp by TMA
  float eps;
  const int* kv_len;       // [B_total] valid keys, or null (Lk)
  __nv_bfloat16* q_prime;
  __nv_bfloat16* kv_packed;
  int* zero_ptr;           // zero_count ints cleared by CTA 0 (the attention's split counters)
  int zero_count;
  int* err;
  unsigned long long timeout_ns;
};
// D in {64, 96, 128, 256}; cudaErrorInvalidValue otherwise, cudaErrorNotSupported when the bias
// vectors leave no room for a 2-stage ring.  tmX[s]: 3-D map [B][rows][K] over set s's input, box
// [1][128][64], 128-byte swizzle; tmW[s]: 2-D map [N][K], box [heads-per-tile * D][64].
// tmT[s] / tmL[s]: set s's LoRA operands (3-D map [B][x rows][R] over T, box [1][128][64]; 2-D map
// [N][R] over B_cat, box [N tile][64]), read only when set[s].lora_steps > 0.
cudaError_t launch_projection(ProjParams p, int D, const CUtensorMap* tmX, const CUtensorMap* tmW,
                              const CUtensorMap* tmCS, const CUtensorMap* tmT, const CUtensorMap* tmL,
                              cudaStream_t stream);
int projection_heads_per_tile(int D);   // 0: unsupported head dim

// Linear layer with the reference's GEMM epilogue (linear.cu): C = epilogue(alpha * A W^T) over M x N
// with A [M][K] bf16 (tmA: 2-D map, box [128][64], 128-byte swizzle) and W [N][K] bf16 (tmW: box
// [256][64], 128-byte swizzle) or int8 (w_i8: box [256][64] without swizzle, converted in shared memory;
// w_scale[n] multiplies row n's dot product); r = alpha*acc (*w_scale[n]) (+ bias[n]) (silu if act == 1),
// then C[m][n] = r or, with resid, C[m][n] += gate[n] * r (gate null: 1); with C16 set, the bf16 store
// form C16[m][n] = r instead (bias, gate and w_scale 16-byte aligned).  lora_steps more K slices follow the K/64 of A and W: T (tmT, [M][R] bf16,
// box [128][64]) against B_cat (tmL, [N][R] bf16, box [256][64]).  C / C16 have row pitch ldc (already
// offset by cOff).
struct LinearParams {
  int M, N, k_steps, m_tiles, n_tiles;
  int lora_steps;
  float alpha;
  const float* bias;   // [N] or null (16-byte aligned, N a multiple of 4)
  const float* gate;   // [N] (offset by gOff) or null
  int resid;
  int act;             // 0 none, 1 silu
  int w_i8;            // W is int8 with per-row scales w_scale[N]
  int pair;            // bf16 W only: CTA pairs on 256 x 256 tiles (tmW / tmL boxes of 128 rows instead of 256)
  int glu;             // 1 SiLU / 2 GELU-tanh GLU of the [128 gate | 128 up] column halves of each tile
                       // (weight rows interleaved per tile): C has N / 2 columns
  const float* w_scale;   // per-row scales [N]: required with w_i8, optional for bf16 W (an expanded int8 W)
  float* C;
  __nv_bfloat16* C16;  // bf16 output instead of C (store form only)
  int64_t ldc;
  int* err;
  unsigned long long timeout_ns;
};
// tmC: 2-D map over C ([M][N] at C + cOff, row pitch ldc; fp32 box [32 rows][32], bf16 box [32 rows][64],
// 128-byte swizzle): the epilogue's tiled stores and fp32 add-reductions.
cudaError_t launch_linear(const LinearParams& p, const CUtensorMap& tmA, const CUtensorMap& tmW, const CUtensorMap& tmT,
                          const CUtensorMap& tmL, const CUtensorMap& tmC, cudaStream_t stream);

// ConvRot input rotation (rotate.cu): Y[r][g*256 + i] = sum_j H256[i][j] X[r][g*256 + j] / 16 for every
// group g of 256 columns (cols a multiple of 256; X rows 16-byte aligned).
struct RotateParams {
  int rows, cols;
  int64_t ldx, ldy;
  const void* x;    // fp32, or bf16 when in_bf16
  void* y;          // fp32, or bf16 when out_bf16
  int in_bf16, out_bf16;
};
cudaError_t launch_rotate(const RotateParams& p, cudaStream_t stream);

// LoRA packing (lora.cu): A_cat [R][K] and B_cat [N][R] bf16 from fp32 entries (device pointers).
struct LoraPackEntry {
  const float* A;   // [r][K]
  const float* B;   // [n][r]
  int r, off, n;
  float scale;
};
cudaError_t launch_expand_i8(const int8_t* w, long long count, __nv_bfloat16* out, cudaStream_t stream);
cudaError_t launch_lora_pack(const LoraPackEntry* e, int count, int N, int K, int R, const float* w_scale, float alpha,
                             __nv_bfloat16* a_cat, __nv_bfloat16* b_cat, cudaStream_t stream);

// Row RMSNorm (rmsnorm.cu): Y[r][c] (=|+=) X[r][c] * rsqrt(mean(X[r]^2) + eps) * w[c].
struct RmsParams {
  int rows, cols;
  int64_t ldx, ldy;
  const float* x;
  const float* w;
  void* y;          // fp32, or bf16 when out_bf16
  int out_bf16;
  int accumulate;   // fp32 Y only
  int vec;          // cols, ldx, ldy multiples of 4; x, w, y 16-byte aligned
  float eps;
  const float* w2;  // accumulate only: Z = rmsnorm(Y after the add) * w2 (vec path), or null
  void* z;          // fp32, or bf16 when z_bf16
  int64_t ldz;
  int z_bf16;
};
cudaError_t launch_rmsnorm(const RmsParams& p, cudaStream_t stream);

// Gated linear unit (glu.cu): Y[r][j] = act(X[r][j]) * X[r][I + j].
struct GluParams {
  int rows, I;
  int64_t ldx, ldy;
  const float* x;
  void* y;          // fp32, or bf16 when out_bf16
  int out_bf16;
  int act;          // 0 SiLU, 1 GELU (tanh approximation)
  int vec;          // I, ldx, ldy multiples of 4; x 16-byte, y 16 (fp32) / 8 (bf16) byte aligned
};
cudaError_t launch_glu(const GluParams& p, cudaStream_t stream);
// Gate/up row interleave per 128-row tile for the linear's fused GLU (glu.cu); row_bytes a multiple of 4.
cudaError_t launch_glu_interleave(const void* src, void* dst, int I, int64_t row_bytes, cudaStream_t stream);

// Returns cudaErrorInvalidValue for unsupported head dims.
cudaError_t launch_attention(const AttnParams& p, int D, const CUtensorMap& tmQ, const CUtensorMap& tmK,
                             const CUtensorMap& tmV, const CUtensorMap& tmVd, cudaStream_t stream);

cudaError_t launch_head_norm(void* X, int f32, const float* w, int L, int H, int D, int64_t ld, int64_t col_off,
                             int64_t row_off, const float* cs, int64_t sin_off, float eps, cudaStream_t stream);
cudaError_t launch_rope2d_table(int h, int w, int D, float* out, cudaStream_t stream);
cudaError_t launch_rope1d_table(int L, int D, float theta, float* out, cudaStream_t stream);

int* device_error_word();   // address of the library's device error word on the current device
// SM count of the current device (cached per device; safe to call from several host threads).
int device_sm_count();
// First-launch set-up of a kernel on the current device (shared-memory attribute, register check):
// `setup` runs at most once per device and per `state`, under a lock, so host threads that launch
// concurrently never race on it; a failed set-up is retried at the next launch.
struct DeviceOnce {
  bool done[128] = {};
};
cudaError_t once_per_device(DeviceOnce& state, cudaError_t (*setup)());
void record_error(const std::string& msg);   // sets the calling thread's nsa_last_error() message

}  // namespace nsa
