/*
 * nsattn.h - C ABI of the B200 (sm_100a) Nanosaur2 attention library (libnsattn.so).
 *
 * Drop-in for the attention hot path of the Nanosaur2 web app: the operator surface the models call
 * (`ops.attention`, `ops.headNorm` in app/gpu/ops.js) plus the fused call sequence of one DiT block
 * / one Gemma3 layer, over caller-owned device buffers and a caller stream.
 *
 * Conventions
 *  - All pointers are device pointers except descriptors (host structs, read during the call).
 *  - Work is stream-ordered on `stream` (a cudaStream_t; NULL = legacy default stream).  Calls only
 *    enqueue kernels; like the reference's command recording (app/gpu/device.js:170-216) nothing
 *    blocks unless stated.
 *  - Every entry point returns an nsa_status and never aborts the process; no C++ exception crosses
 *    the ABI.  nsa_last_error() gives the message of the last failing call on the calling thread.
 *  - Buffers and workspaces are owned by the caller; the library never calls a device allocator
 *    (nsa_fused_attention_noalloc uses a fixed scratch array compiled into the library instead).
 *  - Strides and offsets are in elements.  Matrices are row-major packed rows as in the reference:
 *    element (b, row, col) of a view is at ptr[b*bstride + row*ld + off + col].
 */
#ifndef NSATTN_H
#define NSATTN_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define NSA_ABI_VERSION 4

typedef enum nsa_status {
  NSA_OK = 0,
  NSA_ERR_INVALID_ARGUMENT = 1, /* bad pointer / shape / stride: the reference throws (ops.js:210,216) */
  NSA_ERR_UNSUPPORTED = 2,      /* a shape no kernel covers, e.g. head dim (kernels.js:133) */
  NSA_ERR_WORKSPACE = 3,        /* workspace missing or smaller than *_workspace_size() */
  NSA_ERR_CUDA = 4,             /* CUDA runtime / driver error while enqueueing */
  NSA_ERR_DEVICE = 5            /* a kernel reported a device-side error (a bounded wait expired);
                                   surfaces at nsa_check_device, like device.js:224-231 */
} nsa_status;

typedef enum nsa_dtype { NSA_F32 = 0, NSA_BF16 = 1 } nsa_dtype;

/* Tensor-core precision of the attention products (the descriptors' `compute` field).
 *   NSA_COMPUTE_BF16: q/k/v (fp32 or bf16) are rounded to bf16, fp32 accumulation (the default).
 *   NSA_COMPUTE_TF32: fp32 inputs stay fp32 through the prologue and are multiplied at tf32 precision
 *     (10-bit mantissa against bf16's 7), fp32 accumulation: the closer match to the reference's fp32
 *     math (kernels.js:132-305, tools/reference.py:230-237) at half the bf16 tensor rate.  Head dim
 *     96 with fp32 inputs only (the DiT's fp32 path); other shapes return NSA_ERR_UNSUPPORTED. */
typedef enum nsa_compute { NSA_COMPUTE_BF16 = 0, NSA_COMPUTE_TF32 = 1 } nsa_compute;

/* Library version string, e.g. "nsattn 0.1.0 sm_100a". */
const char* nsa_version(void);
/* Message of the last failing call on the calling thread ("" if none). */
const char* nsa_last_error(void);
const char* nsa_status_string(nsa_status status);

/* ------------------------------------------------------------------------------------------------
 * ops.attention (app/gpu/ops.js:194-242): multi-head attention over packed rows.
 *   q: [Lq, ldq] with head h at column qOff + h*D; k, v: [Lk, ldk] / [Lk, ldv] with kv head
 *   h/group at kOff / vOff + (h/group)*D; output [Lq, ldo] with head h at oOff + h*D.
 *   bias: optional additive score bias per key, bias[key - biasStart] for keys biasStart ..
 *   biasStart+biasLen-1 (kernels.js:199-207); -inf drops a key.  causal keeps keys j <= i
 *   (kernels.js:44).  Extensions over the reference: a batch dimension with per-batch valid key
 *   counts (`kv_len`, keys >= kv_len[b] are masked like kernels.js:269-271), a sliding window, and a
 *   batch x head shard (b_begin/b_count, h_begin/h_count; 0 counts mean "all").
 * q/k/v may be fp32 (the reference's dtype) or bf16; the tensor cores compute in bf16 with fp32
 * accumulation.  The output is fp32 or bf16.
 * ------------------------------------------------------------------------------------------------ */
typedef struct nsa_attention_desc {
  int32_t Lq, Lk, H, D;
  int64_t ldq, ldk, ldv;
  int64_t qOff, kOff, vOff;
  int32_t group;      /* query heads per kv head (ops.js `group`, 1 for the DiT, 4 for Gemma) */
  int32_t causal;     /* ops.js `causal` */
  int32_t window;     /* 0 = none; else key j is visible to query i iff i - window < j */
  int32_t biasStart;  /* ops.js `biasStart` */
  int32_t biasLen;    /* number of bias entries per batch element (0 = no bias) */
  int32_t B;          /* batch elements (>= 1) */
  int64_t q_bstride, k_bstride, v_bstride, bias_bstride, o_bstride;
  int64_t ldo, oOff;  /* reference: ldo = H*D, oOff = 0 */
  int32_t in_dtype;   /* nsa_dtype of q, k, v */
  int32_t out_dtype;  /* nsa_dtype of out */
  float scale;        /* 0 = 1/sqrt(D) (ops.js:206,214) */
  int32_t b_begin, b_count, h_begin, h_count;
  int32_t compute;    /* nsa_compute (0: bf16 tensor cores) */
} nsa_attention_desc;

size_t nsa_attention_workspace_size(const nsa_attention_desc* desc);
/* Replaces ops.attention (app/gpu/ops.js:199). */
nsa_status nsa_attention(const nsa_attention_desc* desc, const void* q, const void* k, const void* v,
                         const float* bias, const int32_t* kv_len, void* out, void* workspace,
                         size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------------------------------------
 * ops.headNorm (app/gpu/ops.js:131-138, kernels.js:311-342): in place, per-head RMSNorm
 * y = x * rsqrt(mean(x^2) + eps) * weight over L rows x H heads of D values at
 * X[(rowOff + l)*ld + colOff + h*D], then, when cs is given, split-half RoPE of pair (i, i + D/2)
 * with cos cs[l*D/2 + i] and sin cs[sinOff + l*D/2 + i].  X is fp32 or bf16.
 * ------------------------------------------------------------------------------------------------ */
nsa_status nsa_head_norm(void* X, int32_t dtype, const float* weight, int32_t L, int32_t H, int32_t D,
                         int64_t ld, int64_t colOff, int64_t rowOff, const float* cs, int64_t sinOff,
                         float eps, void* stream);

/* ------------------------------------------------------------------------------------------------
 * Fused attention step of one DiT block / one Gemma3 layer over the packed qkv buffer, replacing
 * the call sequence headNorm(q, cs) + headNorm(k, cs) [+ headNorm(text k)] + attention(bias,
 * biasStart) of app/models/nanosaur2.js:196-208 and app/models/gemma3.js:63-70
 * (tools/reference.py:272-286 and :186-194).
 *   qkv: [B][Lk rows][ld]; rows [0, Lq) hold q|k|v (queries; their q and k get the q/k norm and,
 *   when cs is given, RoPE with table row = row index); rows [Lq, Lk) hold extra keys (the DiT's
 *   text k|v rows: k norm only, no RoPE; q columns unused).  kv_len[b] (optional) = valid keys of
 *   element b; rows beyond it are ignored (text padding).  bias (optional): [B][biasLen] natural-log
 *   key bias for keys biasStart.. (the DiT passes biasStart = Lq and log prompt weights,
 *   app/models/nanosaur2.js:113,207).  q_norm_w / k_norm_w: [D] fp32 (Gemma's stored w - 1 already
 *   lifted by +1, gemma3.js:22).  Output: out[b*o_bstride + row*ldo + oOff + h*D + d], rows < Lq.
 * ------------------------------------------------------------------------------------------------ */
typedef struct nsa_fused_desc {
  int32_t B;
  int32_t Lq;         /* query rows = RoPE rows */
  int32_t Lk;         /* key rows (>= Lq) */
  int32_t Hq, Hkv, D; /* DiT 16/16/96, Gemma 4/1/256 */
  int64_t ld, bstride;
  int64_t qOff, kOff, vOff;
  int32_t in_dtype, out_dtype;
  float eps;          /* 1e-6 in both models */
  int64_t sinOff;     /* offset of the sin block in cs (tables from nsa_rope*_table: Lq*D/2) */
  int32_t causal, window;
  int32_t biasStart, biasLen;
  int64_t bias_bstride;
  int64_t ldo, o_bstride, oOff;
  float scale;        /* 0 = 1/sqrt(D) */
  int32_t b_begin, b_count, h_begin, h_count;
  int32_t compute;    /* nsa_compute (0: bf16 tensor cores) */
} nsa_fused_desc;

size_t nsa_fused_attention_workspace_size(const nsa_fused_desc* desc);
nsa_status nsa_fused_attention(const nsa_fused_desc* desc, const void* qkv, const float* q_norm_w,
                               const float* k_norm_w, const float* cs, const int32_t* kv_len,
                               const float* bias, void* out, void* workspace, size_t workspace_bytes,
                               void* stream);

/* ------------------------------------------------------------------------------------------------
 * nsa_fused_attention_noalloc: no counterpart in the reference (its WebGPU path always allocates
 * through its buffer pool).  The same fused step as nsa_fused_attention for callers that cannot
 * allocate device memory (a host runtime whose allocator is closed to plugins, or a process that
 * must not call cudaMalloc while it shares the GPU): instead of a caller workspace it uses a scratch
 * array of NSA_NOALLOC_SCRATCH_BYTES built into the library, which every GPU that loads it holds
 * until exit.  The caller passes only inputs and outputs; nothing on this path calls an allocator.
 *  - Shapes whose nsa_fused_attention_workspace_size() exceeds NSA_NOALLOC_SCRATCH_BYTES are
 *    rejected with NSA_ERR_WORKSPACE and a message (e.g. one config-2 DiT batch element or a
 *    16 x 1024-token Gemma layer fit; the batch-2 DiT call does not).
 *  - Every call looks up the scratch address on the current device (cudaGetSymbolAddress).  The
 *    first call on a device also loads the module that holds the array there, which is when the
 *    driver reserves its 64 MiB (an implicit device allocation that can synchronise the device);
 *    with CUDA_MODULE_LOADING=EAGER that happens when the library is loaded instead.  Make the first
 *    call at start-up, before any stream capture.
 *  - All calls share the scratch and it keeps the previous call's contents.  What must start at
 *    zero (the counters of the tail split) is cleared by each call's own prologue.  Calls that
 *    overlap on the GPU (other streams or threads on the same device) race on it: order them, e.g.
 *    on one stream.
 * ------------------------------------------------------------------------------------------------ */
#define NSA_NOALLOC_SCRATCH_BYTES (64u << 20)
nsa_status nsa_fused_attention_noalloc(const nsa_fused_desc* desc, const void* qkv, const float* q_norm_w,
                                       const float* k_norm_w, const float* cs, const int32_t* kv_len,
                                       const float* bias, void* out, void* stream);

/* ------------------------------------------------------------------------------------------------
 * Sequence-sharded DiT joint attention (the 16384-token high-resolution case).  No counterpart in
 * the reference, which runs on one device: this is the nsa_fused_attention call of the DiT block
 * (app/models/nanosaur2.js:196-208) split by query rows over the GPUs of one box.  Rank r owns
 * image rows [q_begin, q_begin + q_count); every rank holds all text rows.
 *   1. nsa_seq_shard_prologue normalises and rotates the rank's query rows into q_prime, and
 *      writes the k'|v' rows of its image rows and of all text rows into kv_packed, each at its
 *      global key row.
 *   2. The caller gathers rows [0, Lq) of kv_packed across ranks: per batch element they are one
 *      contiguous block with q_count rows per rank (one in-place ncclAllGather per element).
 *   3. nsa_seq_shard_attention runs the rank's queries over all keys of kv_packed.
 * Layouts: kv_packed [b_count][kv_rows][2*Hkv*D] bf16, k' heads at columns [0, Hkv*D) and v' heads
 * at [Hkv*D, 2*Hkv*D); q_prime [b_count][Hq][q_pad][D] bf16 (q_pad = q_count rounded up to the
 * query tile).  Both hold the elements [b_begin, b_begin + b_count) of the descriptor, so a caller
 * that overlaps the gather of element b with the attention of element b-1 calls each step with
 * b_count = 1 and pointers advanced by one element.
 * The descriptor is that of nsa_fused_attention (Lq = image rows, Lk = image + text rows,
 * kv_len[b] = valid keys of element b), with whole heads (h_begin 0, h_count 0 or Hq); a causal
 * mask or window only with the full-sequence shard {0, Lq, ., .} (one GPU, e.g. a Gemma layer
 * through nsa_seq_shard_projection).  out receives the rank's rows: out[b*o_bstride + i*ldo + oOff + h*D + d] for
 * local row i = global row q_begin + i.
 * ------------------------------------------------------------------------------------------------ */
typedef struct nsa_seq_shard {
  int32_t q_begin;         /* first image row (query and key) this rank owns */
  int32_t q_count;         /* number of image rows this rank owns */
  int32_t qkv_image_row0;  /* row of qkv holding image row q_begin (q_begin for a full-length qkv,
                              0 for a local [own image rows | text rows] buffer) */
  int32_t qkv_text_row0;   /* row of qkv holding key row Lq, the first text row (Lq, or q_count) */
} nsa_seq_shard;

/* Byte sizes of q_prime and kv_packed for the descriptor's b_count elements, and the rows of one
 * element of kv_packed (its stride is kv_rows * 2*Hkv*D elements). */
nsa_status nsa_seq_shard_buffer_sizes(const nsa_fused_desc* desc, const nsa_seq_shard* shard,
                                      size_t* q_prime_bytes, size_t* kv_packed_bytes, int32_t* kv_rows);
nsa_status nsa_seq_shard_prologue(const nsa_fused_desc* desc, const nsa_seq_shard* shard, const void* qkv,
                                  const float* q_norm_w, const float* k_norm_w, const float* cs,
                                  const int32_t* kv_len, void* q_prime, void* kv_packed, void* stream);
/* CUDA IPC for the peer buffers: nsa_ipc_export writes NSA_IPC_HANDLE_BYTES describing the
 * device allocation holding device_ptr (a cudaIpcMemHandle_t and the offset into it); another
 * process passes them to nsa_ipc_import, which maps the allocation on its current device (peer
 * access enabled) and returns the same address in its space; nsa_ipc_close unmaps it. */
#define NSA_IPC_HANDLE_BYTES 72
nsa_status nsa_ipc_export(const void* device_ptr, void* handle_out);
nsa_status nsa_ipc_import(const void* handle, void** device_ptr_out);
nsa_status nsa_ipc_close(void* device_ptr);
/* One stream-ordered copy (cudaMemcpyAsync, cudaMemcpyDefault): with a peer mapping from
 * nsa_ipc_import as dst, the copy engines move the rank's k'|v' rows over NVLink without SMs. */
nsa_status nsa_memcpy_async(void* dst, const void* src, size_t bytes, void* stream);

/* Step 1 fused with step 2 over peer memory: also stores the image rows' k'|v' into each of
 * kv_peers[0 .. n_peers) (n_peers <= 8): the other GPUs' kv_packed buffers for the same batch
 * elements, mapped into this process (CUDA IPC), at the same offsets as in kv_packed.  The stores
 * cross NVLink directly from the prologue's registers.  Before any GPU's attention reads
 * kv_packed, every GPU's prologue must have completed (a barrier on the stream, e.g. a one-element
 * all-reduce); before a prologue overwrites a peer's kv_packed, that peer's previous attention
 * must have completed. */
nsa_status nsa_seq_shard_prologue_peers(const nsa_fused_desc* desc, const nsa_seq_shard* shard, const void* qkv,
                                        const float* q_norm_w, const float* k_norm_w, const float* cs,
                                        const int32_t* kv_len, void* q_prime, void* kv_packed,
                                        void* const* kv_peers, int32_t n_peers, void* stream);
nsa_status nsa_seq_shard_attention(const nsa_fused_desc* desc, const nsa_seq_shard* shard,
                                   const void* q_prime, const void* kv_packed, const int32_t* kv_len,
                                   const float* bias, void* out, void* stream);

/* ------------------------------------------------------------------------------------------------
 * nsa_seq_shard_projection: step 1 computed from the block input instead of from qkv.  The
 * reference builds qkv with ops.linear (app/gpu/ops.js:50; tools/reference.py:208-210, 272, 282):
 * q|k|v = x @ W_qkv^T + b_qkv over the image rows (`dit.qkv`, app/models/nanosaur2.js:197) and
 * k|v = x_text @ W_kv^T + b_kv over the text rows (`dit.kv_y`, nanosaur2.js:201), then runs
 * ops.headNorm on q and k (nanosaur2.js:199-202).  Here one tcgen05 GEMM per row set computes the
 * linear, and its epilogue adds the bias, applies the per-head RMSNorm and the RoPE, and writes
 * q_prime and kv_packed exactly as nsa_seq_shard_prologue does (same layouts and zero padding; on
 * one GPU use the full-sequence shard {0, Lq, 0, 0}).  The qkv matrix is never materialised.
 * Inputs bf16 (desc->in_dtype NSA_BF16); weights bf16 in the PyTorch Linear layout [out][K] with
 * rows q heads, then k heads, then v heads (w_kv: k heads, then v heads); biases fp32 or NULL.
 * K a multiple of 8, all pointers and row pitches 16-byte aligned.  Head dims 64, 96, 128, 256 with
 * Hq and Hkv multiples of the heads one output tile holds (2 at D = 96 and 128, 4 at 64, 1 at 256).
 * ------------------------------------------------------------------------------------------------ */
typedef struct nsa_proj_desc {
  int32_t K;                  /* input features (model width) */
  const void* x;              /* image rows: element (b, row, k) at x[b*x_bstride + row*ldx + k] */
  int64_t ldx, x_bstride;
  int32_t x_rows;             /* rows of one element of x; image row q_begin is row qkv_image_row0 */
  const void* w_qkv;          /* [(Hq + 2*Hkv)*D][K] */
  const float* b_qkv;         /* [(Hq + 2*Hkv)*D] or NULL */
  const void* x_text;         /* text rows (keys Lq .. Lk-1) at x_text[b*text_bstride + t*ld_text + k],
                                 text row 0 at row qkv_text_row0; NULL when Lk == Lq */
  int64_t ld_text, text_bstride;
  int32_t text_rows;          /* rows of one element of x_text */
  const void* w_kv;           /* [2*Hkv*D][K] */
  const float* b_kv;          /* [2*Hkv*D] or NULL */
  /* int8 ConvRot weights (tools/quant.py:48-57): w_qkv / w_kv hold the int8 values as exact bf16
   * (nsa_expand_i8, once at load) and these the per-row scales, multiplied before the bias (the
   * reference's "i8" GEMM epilogue, app/gpu/gemm.js:159); x / x_text must be the rotated inputs
   * (nsa_rotate).  NULL: plain bf16 weights.  Head dims 64, 96 and 128. */
  const float* w_qkv_scale;
  const float* w_kv_scale;
  /* LoRA side paths (app/gpu/ops.js:55-57, 70-86) of each weight, packed by nsa_lora_pack with the
   * same scales and alpha 1: rank R a multiple of 64 (0: none).  The call first writes T = x A^T into
   * lora_t (bf16: [b_count][x_rows][R_qkv], then [b_count][text_rows][R_kv]) and then accumulates
   * T B^T with the weight's product. */
  int32_t lora_rank_qkv;
  const void* lora_a_qkv;     /* bf16 [R_qkv][K] */
  const void* lora_b_qkv;     /* bf16 [(Hq + 2*Hkv)*D][R_qkv] */
  int32_t lora_rank_kv;
  const void* lora_a_kv;      /* bf16 [R_kv][K] */
  const void* lora_b_kv;      /* bf16 [2*Hkv*D][R_kv] */
  void* lora_t;
} nsa_proj_desc;
nsa_status nsa_seq_shard_projection(const nsa_fused_desc* desc, const nsa_seq_shard* shard,
                                    const nsa_proj_desc* proj, const float* q_norm_w, const float* k_norm_w,
                                    const float* cs, const int32_t* kv_len, void* q_prime, void* kv_packed,
                                    void* stream);

/* ------------------------------------------------------------------------------------------------
 * nsa_linear: ops.linear(gpu, x, W, {bias, resid, gate, gOff, act, ldc, cOff}) (app/gpu/ops.js:50-66)
 * with the epilogue of the reference's tiled GEMM (app/gpu/gemm.js:155-165):
 *   r = alpha * sum_k A[m][k] W[n][k] (* w_scale[n]) (+ bias[n]) (+ LoRA delta[m][n]) (silu when act = 1),
 *   then C[m*ldc + cOff + n] = r, or with resid: C[...] += r, or with resid and a gate:
 *   C[...] += gate[gOff + n] * r.
 * The DiT block's output projection is the gated form (app/models/nanosaur2.js:210). A is bf16
 * [M][lda], W in the Linear layout [N][K], C fp32 (the reference's residual stream) or, with
 * out_dtype NSA_BF16, bf16 (store form only: the next GEMM's operand), bias and gate fp32.
 * K, lda multiples of 8; N, ldc, cOff and gOff multiples of 4; pointers 16-byte aligned.
 * Weight formats (the reference's GEMM B formats "bf16" and "i8", gemm.js:9-10):
 *   NSA_W_BF16  W bf16 [N][K]; a non-NULL w_scale[N] multiplies row n's dot product as for NSA_W_I8
 *               (an int8 ConvRot weight expanded once by nsa_expand_i8: the same values, so the same
 *               results as NSA_W_I8, at the bf16 MMA rate for twice the weight bytes).
 *   NSA_W_I8    W int8 [N][K] of the ConvRot-quantised model (tools/quant.py:48-57) with the per-row
 *               fp32 scale w_scale[N] (gemm.js:159); K a multiple of 16.  A must be the rotated input
 *               (nsa_rotate, ops.rotate: ops.js:34-45, 54), as the reference passes `xr`.
 * LoRA side paths (ops.js:55-57, 70-86; app/lora.js:143-150): lora_rank R > 0 adds
 *   delta = sum_i scale_i * B_i (A_i x) over the entries packed by nsa_lora_pack into lora_a [R][K] and
 *   lora_b [N][R] (bf16).  The call first writes T = A @ lora_a^T into the caller's scratch lora_t
 *   (bf16 [M][R]), then accumulates T @ lora_b^T in the same tensor-memory accumulator as A @ W^T.
 * Fused GLU (glu = 1 SiLU, 2 GELU-tanh): the gate_up linear followed by ops.glu (app/models/gemma3.js:
 *   80-81; ops.js:141-148) in one call.  W (and bias, w_scale) must be in the tiled order that
 *   nsa_glu_interleave writes from the [gate; up] layout; then
 *   C[m*ldc + cOff + j] = act(r_gate[m][j]) * r_up[m][j] for j < N / 2, with r as above before the act.
 *   N a multiple of 256; no resid, gate, act or LoRA (NSA_ERR_INVALID_ARGUMENT otherwise).
 * ------------------------------------------------------------------------------------------------ */
typedef enum nsa_weight_format { NSA_W_BF16 = 0, NSA_W_I8 = 1 } nsa_weight_format;
/* Tile schedule (the result is the same bits either way):
 *   NSA_LINEAR_SINGLE  one CTA per 128 x 256 tile, 64-wide K steps;
 *   NSA_LINEAR_PAIR    two CTAs (a cluster on two SMs) per 256 x 256 tile, each loading its 128 rows of A
 *                      and half the tile's W rows, 128-wide K steps; bf16 weights and M > 128 only;
 *   NSA_LINEAR_AUTO    pairs for bf16 weights when K + lora_rank >= 2048 and M x N >= 2^26 (on B200 pairs
 *                      measured 10% ahead at 16384 x 4096 x 4096 and level or behind on the DiT and Gemma
 *                      linears), unless NSA_LINEAR_PAIR=0. */
typedef enum nsa_linear_schedule { NSA_LINEAR_AUTO = 0, NSA_LINEAR_SINGLE = 1, NSA_LINEAR_PAIR = 2 } nsa_linear_schedule;
typedef struct nsa_linear_desc {
  int32_t M, N, K;
  int64_t lda;      /* A row pitch in elements */
  int64_t ldc;      /* C row pitch in elements (0: N) */
  int64_t cOff;     /* first column of C written (opts.cOff) */
  int64_t gOff;     /* offset into gate (opts.gOff) */
  float alpha;      /* 0 means 1 */
  int32_t resid;    /* 1: accumulate into C (opts.resid) */
  int32_t act;      /* 0: none, 1: silu (opts.act) */
  int32_t out_dtype;        /* NSA_F32 (C is float*) or NSA_BF16 (C is bf16, no resid) */
  int32_t w_format;         /* NSA_W_BF16 or NSA_W_I8 */
  const float* w_scale;     /* [N] per-row scales: required for NSA_W_I8, optional for NSA_W_BF16 */
  int32_t lora_rank;        /* R, a multiple of 64 (nsa_lora_rank); 0: no LoRA */
  const void* lora_a;       /* bf16 [R][K] */
  const void* lora_b;       /* bf16 [N][R] */
  void* lora_t;             /* bf16 [M][R] scratch written by the call */
  int32_t glu;              /* 0: none; 1 SiLU / 2 GELU-tanh GLU of the interleaved gate|up output (C: N / 2 columns) */
  int32_t schedule;         /* NSA_LINEAR_AUTO (0), NSA_LINEAR_SINGLE or NSA_LINEAR_PAIR (bf16 W only) */
} nsa_linear_desc;
nsa_status nsa_linear(const nsa_linear_desc* desc, const void* A, const void* W, const float* bias,
                      const float* gate, void* C, void* stream);

/* nsa_rotate: ops.rotate(gpu, x) (app/gpu/ops.js:38-45, the hadamard kernel of kernels.js:379-407):
 * every group of 256 consecutive columns of a row is multiplied by the normalised regular Hadamard
 * matrix H256 = (H4 (x) H4 (x) H4 (x) H4) / 16 (tools/quant.py:21-30).  X and Y fp32 or bf16 (a bf16 Y
 * is nsa_linear's A for int8 weights); cols a multiple of 256; row pitches multiples of 8 elements;
 * pointers 16-byte aligned; X and Y must not overlap. */
typedef struct nsa_rotate_desc {
  int32_t rows, cols;
  int64_t ldx;         /* X row pitch in elements (0: cols) */
  int64_t ldy;         /* Y row pitch in elements (0: cols) */
  int32_t in_dtype;    /* NSA_F32 or NSA_BF16 */
  int32_t out_dtype;   /* NSA_F32 or NSA_BF16 */
} nsa_rotate_desc;
nsa_status nsa_rotate(const nsa_rotate_desc* desc, const void* X, void* Y, void* stream);

/* LoRA entries of one linear (app/lora.js:143-150): A [r][K] and B [n][r] fp32 device matrices (for
 * int8 weights A's rows already rotated, as the reference's loader does, app/lora.js:126), the output
 * columns [off, off + n) of the linear (the slice of a stacked q|k|v weight) and the scale
 * strength * alpha / r.  nsa_lora_rank returns R = the ranks' sum rounded up to 64 (0 for none);
 * nsa_lora_pack writes lora_a [R][K] and lora_b [N][R] for nsa_linear: lora_b's rows are divided by
 * alpha * w_scale[n] (w_scale NULL for bf16 weights), which the linear's epilogue multiplies back.  A
 * strength change (or another alpha) is a re-pack; the entries array is host memory. */
typedef struct nsa_lora_entry {
  const float* A;
  const float* B;
  int32_t r, off, n;
  float scale;
} nsa_lora_entry;
int32_t nsa_lora_rank(const nsa_lora_entry* entries, int32_t count);
/* int8 weights -> their exact bf16 values (every integer in [-128, 127] is a bf16), for the
 * projection's ConvRot form: count elements, out 16-byte aligned. */
nsa_status nsa_expand_i8(const int8_t* W, int64_t count, void* out_bf16, void* stream);
nsa_status nsa_lora_pack(const nsa_lora_entry* entries, int32_t count, int32_t N, int32_t K, const float* w_scale,
                         float alpha, void* lora_a, void* lora_b, void* stream);

/* ------------------------------------------------------------------------------------------------
 * nsa_rmsnorm: ops.rmsnorm(gpu, x, weight, cols, eps, out) (app/gpu/ops.js:111-116, kernels.js:62-80)
 *   Y[r*ldy + c] = X[r*ldx + c] * rsqrt(mean_c(X[r][c]^2) + eps) * weight[c]
 * over `rows` rows of `cols` fp32 values.  out_dtype NSA_BF16 writes the next GEMM's bf16 operand
 * (the Gemma layer's input norm before te.qkv, app/models/gemma3.js:62-63).  accumulate = 1 (fp32 Y
 * only) fuses the ops.accumulate that follows (ops.js:188-192; gemma3.js:74-77, the post-attention
 * norm added into the residual stream): Y[...] += X * r * weight.  X and Y must not overlap.
 * ------------------------------------------------------------------------------------------------ */
typedef struct nsa_rmsnorm_desc {
  int32_t rows, cols;
  int64_t ldx;         /* X row pitch in elements (0: cols) */
  int64_t ldy;         /* Y row pitch in elements (0: cols) */
  int32_t out_dtype;   /* NSA_F32 or NSA_BF16 */
  int32_t accumulate;  /* 1: Y += norm(X) (NSA_F32 only) */
  float eps;           /* >= 0; the reference's default is 1e-6 */
  /* With accumulate = 1, optionally the next norm of the same rows in the same pass: the Gemma layer's
   * pre-MLP norm after the post-attention accumulate, and the next layer's input norm after the
   * post-MLP one (gemma3.js:77-79, 88 then 62): Z = rmsnorm(Y after the add) * next_weight, with the
   * same eps.  Y's new values stay in registers, so Z costs its own write only. */
  const float* next_weight;   /* [cols] or NULL (no Z) */
  void* Z;                    /* [rows][ldz] */
  int64_t ldz;                /* Z row pitch in elements (0: cols) */
  int32_t z_dtype;            /* NSA_F32 or NSA_BF16 */
} nsa_rmsnorm_desc;
nsa_status nsa_rmsnorm(const nsa_rmsnorm_desc* desc, const float* X, const float* weight, void* Y, void* stream);

/* ------------------------------------------------------------------------------------------------
 * nsa_glu: ops.glu(gpu, x, act) (app/gpu/ops.js:141-148, kernels.js:346-360) over the [gate | up]
 * halves of a gate_up linear's output:  Y[r*ldy + j] = act(X[r*ldx + j]) * X[r*ldx + I + j], j < I.
 * act 0 = SiLU (SwiGLU), 1 = GELU with the tanh approximation (Gemma's MLP, app/models/gemma3.js:81).
 * X fp32; Y fp32 or bf16 (the down projection's operand).  X and Y must not overlap.
 * ------------------------------------------------------------------------------------------------ */
typedef struct nsa_glu_desc {
  int32_t rows, I;
  int64_t ldx;         /* X row pitch in elements (0: 2*I) */
  int64_t ldy;         /* Y row pitch in elements (0: I) */
  int32_t act;         /* 0 SiLU, 1 GELU (tanh) */
  int32_t out_dtype;   /* NSA_F32 or NSA_BF16 */
} nsa_glu_desc;
nsa_status nsa_glu(const nsa_glu_desc* desc, const float* X, void* Y, void* stream);
/* nsa_glu_interleave: the row order nsa_linear's fused GLU reads.  src holds 2I rows of row_bytes
 * bytes, the gate rows [0, I) above the up rows [I, 2I) (a gate_up weight, bias or w_scale); dst row
 * 256 t + j is gate row 128 t + j for j < 128 and up row I + 128 t + (j - 128) otherwise.  I a
 * multiple of 128; row_bytes a multiple of 4; src and dst 4-byte aligned and not overlapping.  A
 * one-time weight preparation, like the reference's load-time conversions. */
nsa_status nsa_glu_interleave(const void* src, void* dst, int32_t I, int64_t row_bytes, void* stream);

/* ------------------------------------------------------------------------------------------------
 * RoPE tables in the reference layout: cos block [L][D/2] then sin block [L][D/2] (sinOff = L*D/2).
 *   nsa_rope2d_table: app/models/common.js:28-43 (tools/reference.py:220-227): L = h*w tokens,
 *     the first D/4 pairs rotate by the centred column, the next D/4 by the centred row, theta 1e4.
 *   nsa_rope1d_table: app/models/common.js:18-24 (tools/reference.py:169-172).
 * out: device fp32 buffer of L*D floats.
 * ------------------------------------------------------------------------------------------------ */
nsa_status nsa_rope2d_table(int32_t h, int32_t w, int32_t D, float* out, void* stream);
nsa_status nsa_rope1d_table(int32_t L, int32_t D, float theta, float* out, void* stream);

/* ------------------------------------------------------------------------------------------------
 * Device-side failure surfacing (app/gpu/device.js:224-231 turns async validation errors into a
 * throw at the next read/sync).  Synchronises `stream`, reads and clears the device error word of
 * the current device: NSA_ERR_DEVICE if any kernel gave up a bounded wait since the last check.
 * ------------------------------------------------------------------------------------------------ */
nsa_status nsa_check_device(void* stream);

/* Self-test of the failure path: launches one CTA that waits on a barrier nothing arrives on, with
 * a limit of `timeout_us`; the wait expires, the kernel records the error and returns.  A following
 * nsa_check_device reports NSA_ERR_DEVICE and the context stays usable. */
nsa_status nsa_selftest_wait_timeout(int32_t timeout_us, void* stream);

/* ------------------------------------------------------------------------------------------------
 * Profiler (app/gpu/device.js:61-80,185-196,235-288: per-dispatch timestamps aggregated per kernel
 * name with a flop count).  When enabled, each library launch is bracketed by CUDA events on its
 * stream.  nsa_profiler_read synchronises the recorded events and returns one entry per kernel name.
 * ------------------------------------------------------------------------------------------------ */
typedef struct nsa_kernel_stat {
  char name[32];
  int64_t launches;
  double total_ms;
  double flops;   /* algorithmic flops (4*B*H*valid pairs*D for attention, ops.js:207) */
  double bytes;   /* algorithmic HBM bytes (prologue: bytes read + written) */
} nsa_kernel_stat;

void nsa_profiler_enable(int32_t on);
void nsa_profiler_reset(void);
int32_t nsa_profiler_read(nsa_kernel_stat* out, int32_t max_entries);

#ifdef __cplusplus
}
#endif

#endif /* NSATTN_H */
