/* Node.js N-API addon over libnsattn.so: the binding the reference's engine would load in place of
 * the WGSL dispatches behind its JS operators (app/gpu/ops.js).  Each export takes one options object
 * carrying the same fields as the JS operator it replaces, plus the device handles (CUDA device
 * pointers and the stream, as BigInt values) of the buffers the JS side owns:
 *
 *   attention(opts)        ops.attention(gpu, {q,k,v,Lq,Lk,H,D,ldq,ldk,ldv,qOff,kOff,vOff,group,
 *                          causal,bias,biasStart,out}) (ops.js:194-242) -> nsa_attention
 *   attentionWorkspaceBytes(opts)                                        -> nsa_attention_workspace_size
 *   headNorm(opts)         ops.headNorm(gpu, X, weight, {L,H,D,ld,colOff,rowOff,cs,eps})
 *                          (ops.js:131-138)                               -> nsa_head_norm
 *   fusedAttention(opts)   the DiT block's / Gemma layer's headNorm + attention sequence
 *                          (nanosaur2.js:196-208, gemma3.js:63-70)        -> nsa_fused_attention
 *   fusedWorkspaceBytes(opts)                                            -> nsa_fused_attention_workspace_size
 *   linear(opts)           ops.linear(gpu, x, W, {bias,resid,gate,gOff,act,ldc,cOff}) (ops.js:50-66),
 *                          with int8 ConvRot weights (wI8, wScale) and packed LoRAs (loraRank, loraA,
 *                          loraB, loraT), the fused GLU of a gate_up linear (glu: 1 silu, 2 gelu_tanh) and
 *                          the tile schedule (schedule: 0 auto, 1 single CTAs, 2 CTA pairs)
 *   rotate(opts)           ops.rotate(gpu, x) (ops.js:38-45)                -> nsa_rotate
 *   loraPack(opts)         the LoRA side paths of one weight (app/lora.js:143-150), entries
 *                          [{A, B, r, off, n, scale}]; returns the packed rank R -> nsa_lora_pack
 *   expandI8(opts)         int8 weights -> exact bf16 values (the projection's ConvRot form)
 *                                                                        -> nsa_expand_i8
 *   rmsnorm(opts)          ops.rmsnorm(gpu, x, weight, cols, eps, out) (ops.js:111-116), with the chained
 *                          next norm of an accumulate (nextWeight, nextOut, ldz, nextOutBf16)
 *   glu(opts)              ops.glu(gpu, x, act) (ops.js:141-148)
 *   gluInterleave(opts)    a gate_up weight / bias / scale in the fused GLU's row order
 *                          {src, dst, I, rowBytes}                        -> nsa_glu_interleave
 *   rope2dTable(opts) / ropeTable(opts)   common.js:28-43 / 18-24 into a device buffer
 *   checkDevice(opts)      the async error surfacing at read/sync (device.js:224-231)
 *
 * A failing call throws, as the JS operators throw on bad shapes (ops.js:210,216; kernels.js:133):
 * the error's code is nsa_status_string(status) and its message nsa_last_error().  Build with
 * node-gyp (binding.gyp next to this file), linking libnsattn.so.
 */
#include <node_api.h>
#include <stdbool.h>
#include <stdint.h>
#include <string.h>

#include "nsattn.h"

/* ----------------------------------------------------------------------------- option readers */

static bool has(napi_env env, napi_value obj, const char* key) {
  bool h = false;
  napi_has_named_property(env, obj, key, &h);
  return h;
}

/* A numeric option (JS number or BigInt); `dflt` when absent or undefined. */
static int64_t num(napi_env env, napi_value obj, const char* key, int64_t dflt) {
  if (!has(env, obj, key)) return dflt;
  napi_value v;
  napi_valuetype t;
  napi_get_named_property(env, obj, key, &v);
  napi_typeof(env, v, &t);
  if (t == napi_bigint) {
    int64_t x = 0;
    bool lossless = false;
    napi_get_value_bigint_int64(env, v, &x, &lossless);
    return x;
  }
  if (t == napi_boolean) {
    bool b = false;
    napi_get_value_bool(env, v, &b);
    return b ? 1 : 0;
  }
  if (t != napi_number) return dflt;
  double d = 0;
  napi_get_value_double(env, v, &d);
  return (int64_t)d;
}

static float fnum(napi_env env, napi_value obj, const char* key, float dflt) {
  if (!has(env, obj, key)) return dflt;
  napi_value v;
  napi_valuetype t;
  napi_get_named_property(env, obj, key, &v);
  napi_typeof(env, v, &t);
  if (t != napi_number) return dflt;
  double d = 0;
  napi_get_value_double(env, v, &d);
  return (float)d;
}

/* A device handle (BigInt pointer); NULL when absent, null or undefined. */
static void* ptr(napi_env env, napi_value obj, const char* key) {
  if (!has(env, obj, key)) return NULL;
  napi_value v;
  napi_valuetype t;
  napi_get_named_property(env, obj, key, &v);
  napi_typeof(env, v, &t);
  if (t != napi_bigint) return NULL;
  uint64_t x = 0;
  bool lossless = false;
  napi_get_value_bigint_uint64(env, v, &x, &lossless);
  return (void*)(uintptr_t)x;
}

static napi_value opts_arg(napi_env env, napi_callback_info info) {
  size_t argc = 1;
  napi_value opts = NULL;
  napi_get_cb_info(env, info, &argc, &opts, NULL, NULL);
  if (argc < 1) {
    napi_throw_type_error(env, NULL, "expected one options object");
    return NULL;
  }
  return opts;
}

/* Throws for a failing status (the JS operators throw synchronously); returns undefined. */
static napi_value done(napi_env env, nsa_status st) {
  if (st != NSA_OK) napi_throw_error(env, nsa_status_string(st), nsa_last_error());
  napi_value u;
  napi_get_undefined(env, &u);
  return u;
}

static napi_value size_value(napi_env env, size_t bytes) {
  napi_value v;
  napi_create_bigint_uint64(env, (uint64_t)bytes, &v);
  return v;
}

static int32_t dtype(napi_env env, napi_value o, const char* key) {
  return num(env, o, key, 0) ? NSA_BF16 : NSA_F32;   /* opts.<key>Bf16: true for bf16 buffers */
}

/* ----------------------------------------------------------------------------- ops.attention */

static void attention_desc(napi_env env, napi_value o, nsa_attention_desc* d) {
  memset(d, 0, sizeof *d);
  d->Lq = (int32_t)num(env, o, "Lq", 0);
  d->Lk = (int32_t)num(env, o, "Lk", 0);
  d->H = (int32_t)num(env, o, "H", 0);
  d->D = (int32_t)num(env, o, "D", 0);
  d->ldq = num(env, o, "ldq", (int64_t)d->H * d->D);
  d->ldk = num(env, o, "ldk", 0);
  d->ldv = num(env, o, "ldv", 0);
  d->qOff = num(env, o, "qOff", 0);
  d->kOff = num(env, o, "kOff", 0);
  d->vOff = num(env, o, "vOff", 0);
  d->group = (int32_t)num(env, o, "group", 1);
  d->causal = (int32_t)num(env, o, "causal", 0);
  d->window = (int32_t)num(env, o, "window", 0);
  d->biasStart = (int32_t)num(env, o, "biasStart", 0);
  d->biasLen = has(env, o, "bias") ? (int32_t)num(env, o, "biasLen", (int64_t)d->Lk - d->biasStart) : 0;
  d->B = (int32_t)num(env, o, "B", 1);
  d->q_bstride = num(env, o, "qBstride", 0);
  d->k_bstride = num(env, o, "kBstride", 0);
  d->v_bstride = num(env, o, "vBstride", 0);
  d->bias_bstride = num(env, o, "biasBstride", 0);
  d->o_bstride = num(env, o, "oBstride", 0);
  d->ldo = num(env, o, "ldo", (int64_t)d->H * d->D);
  d->oOff = num(env, o, "oOff", 0);
  d->in_dtype = dtype(env, o, "inBf16");
  d->out_dtype = dtype(env, o, "outBf16");
  d->scale = fnum(env, o, "scale", 0.f);
}

static napi_value Attention(napi_env env, napi_callback_info info) {
  napi_value o = opts_arg(env, info);
  if (!o) return NULL;
  nsa_attention_desc d;
  attention_desc(env, o, &d);
  return done(env, nsa_attention(&d, ptr(env, o, "q"), ptr(env, o, "k"), ptr(env, o, "v"), ptr(env, o, "bias"),
                                 ptr(env, o, "kvLen"), ptr(env, o, "out"), ptr(env, o, "workspace"),
                                 (size_t)num(env, o, "workspaceBytes", 0), ptr(env, o, "stream")));
}

static napi_value AttentionWorkspaceBytes(napi_env env, napi_callback_info info) {
  napi_value o = opts_arg(env, info);
  if (!o) return NULL;
  nsa_attention_desc d;
  attention_desc(env, o, &d);
  return size_value(env, nsa_attention_workspace_size(&d));
}

/* ----------------------------------------------------------------------------- ops.headNorm */

static napi_value HeadNorm(napi_env env, napi_callback_info info) {
  napi_value o = opts_arg(env, info);
  if (!o) return NULL;
  const int32_t L = (int32_t)num(env, o, "L", 0), H = (int32_t)num(env, o, "H", 0), D = (int32_t)num(env, o, "D", 0);
  return done(env, nsa_head_norm(ptr(env, o, "X"), dtype(env, o, "bf16"), ptr(env, o, "weight"), L, H, D,
                                 num(env, o, "ld", (int64_t)H * D), num(env, o, "colOff", 0), num(env, o, "rowOff", 0),
                                 ptr(env, o, "cs"), num(env, o, "sinOff", (int64_t)L * D / 2),
                                 fnum(env, o, "eps", 1e-6f), ptr(env, o, "stream")));
}

/* ----------------------------------------------------------------------------- fused call sites */

static void fused_desc(napi_env env, napi_value o, nsa_fused_desc* d) {
  memset(d, 0, sizeof *d);
  d->B = (int32_t)num(env, o, "B", 1);
  d->Lq = (int32_t)num(env, o, "Lq", 0);
  d->Lk = (int32_t)num(env, o, "Lk", d->Lq);
  d->Hq = (int32_t)num(env, o, "Hq", 16);
  d->Hkv = (int32_t)num(env, o, "Hkv", d->Hq);
  d->D = (int32_t)num(env, o, "D", 96);
  d->ld = num(env, o, "ld", 0);
  d->bstride = num(env, o, "bstride", d->ld * d->Lk);
  d->qOff = num(env, o, "qOff", 0);
  d->kOff = num(env, o, "kOff", (int64_t)d->Hq * d->D);
  d->vOff = num(env, o, "vOff", (int64_t)(d->Hq + d->Hkv) * d->D);
  d->in_dtype = dtype(env, o, "inBf16");
  d->out_dtype = dtype(env, o, "outBf16");
  d->eps = fnum(env, o, "eps", 1e-6f);
  d->sinOff = num(env, o, "sinOff", (int64_t)d->Lq * d->D / 2);
  d->causal = (int32_t)num(env, o, "causal", 0);
  d->window = (int32_t)num(env, o, "window", 0);
  d->biasStart = (int32_t)num(env, o, "biasStart", d->Lq);
  d->biasLen = has(env, o, "bias") ? (int32_t)num(env, o, "biasLen", (int64_t)d->Lk - d->biasStart) : 0;
  d->bias_bstride = num(env, o, "biasBstride", d->biasLen);
  d->ldo = num(env, o, "ldo", (int64_t)d->Hq * d->D);
  d->o_bstride = num(env, o, "oBstride", d->ldo * d->Lq);
  d->oOff = num(env, o, "oOff", 0);
  d->scale = fnum(env, o, "scale", 0.f);
}

static napi_value FusedAttention(napi_env env, napi_callback_info info) {
  napi_value o = opts_arg(env, info);
  if (!o) return NULL;
  nsa_fused_desc d;
  fused_desc(env, o, &d);
  return done(env, nsa_fused_attention(&d, ptr(env, o, "qkv"), ptr(env, o, "qNorm"), ptr(env, o, "kNorm"),
                                       ptr(env, o, "cs"), ptr(env, o, "kvLen"), ptr(env, o, "bias"), ptr(env, o, "out"),
                                       ptr(env, o, "workspace"), (size_t)num(env, o, "workspaceBytes", 0),
                                       ptr(env, o, "stream")));
}

static napi_value FusedWorkspaceBytes(napi_env env, napi_callback_info info) {
  napi_value o = opts_arg(env, info);
  if (!o) return NULL;
  nsa_fused_desc d;
  fused_desc(env, o, &d);
  return size_value(env, nsa_fused_attention_workspace_size(&d));
}

/* ----------------------------------------------------------------------------- GEMM and row ops */

static napi_value Linear(napi_env env, napi_callback_info info) {
  napi_value o = opts_arg(env, info);
  if (!o) return NULL;
  nsa_linear_desc d;
  memset(&d, 0, sizeof d);
  d.M = (int32_t)num(env, o, "M", 0);
  d.N = (int32_t)num(env, o, "N", 0);
  d.K = (int32_t)num(env, o, "K", 0);
  d.lda = num(env, o, "lda", d.K);
  d.ldc = num(env, o, "ldc", 0);
  d.cOff = num(env, o, "cOff", 0);
  d.gOff = num(env, o, "gOff", 0);
  d.alpha = fnum(env, o, "alpha", 1.f);
  d.resid = (int32_t)num(env, o, "resid", 0);
  d.act = (int32_t)num(env, o, "act", 0);
  d.out_dtype = dtype(env, o, "outBf16");
  d.w_format = num(env, o, "wI8", 0) ? NSA_W_I8 : NSA_W_BF16;
  d.w_scale = (const float*)ptr(env, o, "wScale");
  d.lora_rank = (int32_t)num(env, o, "loraRank", 0);
  d.lora_a = ptr(env, o, "loraA");
  d.lora_b = ptr(env, o, "loraB");
  d.lora_t = ptr(env, o, "loraT");
  d.glu = (int32_t)num(env, o, "glu", 0);
  d.schedule = (int32_t)num(env, o, "schedule", NSA_LINEAR_AUTO);
  return done(env, nsa_linear(&d, ptr(env, o, "x"), ptr(env, o, "W"), ptr(env, o, "bias"), ptr(env, o, "gate"),
                              ptr(env, o, "out"), ptr(env, o, "stream")));
}

static napi_value Rmsnorm(napi_env env, napi_callback_info info) {
  napi_value o = opts_arg(env, info);
  if (!o) return NULL;
  nsa_rmsnorm_desc d;
  memset(&d, 0, sizeof d);
  d.rows = (int32_t)num(env, o, "rows", 0);
  d.cols = (int32_t)num(env, o, "cols", 0);
  d.ldx = num(env, o, "ldx", 0);
  d.ldy = num(env, o, "ldy", 0);
  d.out_dtype = dtype(env, o, "outBf16");
  d.accumulate = (int32_t)num(env, o, "accumulate", 0);
  d.eps = fnum(env, o, "eps", 1e-6f);
  d.next_weight = (const float*)ptr(env, o, "nextWeight");
  d.Z = ptr(env, o, "nextOut");
  d.ldz = num(env, o, "ldz", 0);
  d.z_dtype = dtype(env, o, "nextOutBf16");
  return done(env, nsa_rmsnorm(&d, ptr(env, o, "x"), ptr(env, o, "weight"), ptr(env, o, "out"), ptr(env, o, "stream")));
}

static napi_value Glu(napi_env env, napi_callback_info info) {
  napi_value o = opts_arg(env, info);
  if (!o) return NULL;
  nsa_glu_desc d;
  memset(&d, 0, sizeof d);
  d.rows = (int32_t)num(env, o, "rows", 0);
  d.I = (int32_t)num(env, o, "I", 0);
  d.ldx = num(env, o, "ldx", 0);
  d.ldy = num(env, o, "ldy", 0);
  d.act = (int32_t)num(env, o, "act", 0);
  d.out_dtype = dtype(env, o, "outBf16");
  return done(env, nsa_glu(&d, ptr(env, o, "x"), ptr(env, o, "out"), ptr(env, o, "stream")));
}

static napi_value GluInterleave(napi_env env, napi_callback_info info) {
  napi_value o = opts_arg(env, info);
  if (!o) return NULL;
  return done(env, nsa_glu_interleave(ptr(env, o, "src"), ptr(env, o, "dst"), (int32_t)num(env, o, "I", 0),
                                      num(env, o, "rowBytes", 0), ptr(env, o, "stream")));
}

static napi_value Rotate(napi_env env, napi_callback_info info) {
  napi_value o = opts_arg(env, info);
  if (!o) return NULL;
  nsa_rotate_desc d;
  memset(&d, 0, sizeof d);
  d.rows = (int32_t)num(env, o, "rows", 0);
  d.cols = (int32_t)num(env, o, "cols", 0);
  d.ldx = num(env, o, "ldx", 0);
  d.ldy = num(env, o, "ldy", 0);
  d.in_dtype = dtype(env, o, "inBf16");
  d.out_dtype = dtype(env, o, "outBf16");
  return done(env, nsa_rotate(&d, ptr(env, o, "x"), ptr(env, o, "out"), ptr(env, o, "stream")));
}

static napi_value ExpandI8(napi_env env, napi_callback_info info) {
  napi_value o = opts_arg(env, info);
  if (!o) return NULL;
  return done(env, nsa_expand_i8((const int8_t*)ptr(env, o, "W"), num(env, o, "count", 0), ptr(env, o, "out"),
                                 ptr(env, o, "stream")));
}

#define NSA_ADDON_MAX_LORAS 64

static napi_value LoraPack(napi_env env, napi_callback_info info) {
  napi_value o = opts_arg(env, info);
  if (!o) return NULL;
  nsa_lora_entry e[NSA_ADDON_MAX_LORAS];
  uint32_t count = 0;
  if (has(env, o, "entries")) {
    napi_value arr;
    napi_get_named_property(env, o, "entries", &arr);
    napi_get_array_length(env, arr, &count);
  }
  if (count > NSA_ADDON_MAX_LORAS) {
    napi_throw_error(env, "NSA_ERR_INVALID_ARGUMENT", "too many LoRA entries for one weight");
    return NULL;
  }
  napi_value arr;
  if (count) napi_get_named_property(env, o, "entries", &arr);
  for (uint32_t i = 0; i < count; ++i) {
    napi_value it;
    napi_get_element(env, arr, i, &it);
    e[i].A = (const float*)ptr(env, it, "A");
    e[i].B = (const float*)ptr(env, it, "B");
    e[i].r = (int32_t)num(env, it, "r", 0);
    e[i].off = (int32_t)num(env, it, "off", 0);
    e[i].n = (int32_t)num(env, it, "n", 0);
    e[i].scale = fnum(env, it, "scale", 1.f);
  }
  nsa_status st = nsa_lora_pack(e, (int32_t)count, (int32_t)num(env, o, "N", 0), (int32_t)num(env, o, "K", 0),
                                (const float*)ptr(env, o, "wScale"), fnum(env, o, "alpha", 1.f), ptr(env, o, "loraA"),
                                ptr(env, o, "loraB"), ptr(env, o, "stream"));
  if (st != NSA_OK) return done(env, st);   /* throws */
  napi_value r;
  napi_create_int32(env, nsa_lora_rank(e, (int32_t)count), &r);
  return r;
}

/* ----------------------------------------------------------------------------- tables, errors */

static napi_value Rope2dTable(napi_env env, napi_callback_info info) {
  napi_value o = opts_arg(env, info);
  if (!o) return NULL;
  return done(env, nsa_rope2d_table((int32_t)num(env, o, "h", 0), (int32_t)num(env, o, "w", 0),
                                    (int32_t)num(env, o, "D", 96), ptr(env, o, "out"), ptr(env, o, "stream")));
}

static napi_value RopeTable(napi_env env, napi_callback_info info) {
  napi_value o = opts_arg(env, info);
  if (!o) return NULL;
  return done(env, nsa_rope1d_table((int32_t)num(env, o, "L", 0), (int32_t)num(env, o, "D", 256),
                                    fnum(env, o, "theta", 10000.f), ptr(env, o, "out"), ptr(env, o, "stream")));
}

static napi_value CheckDevice(napi_env env, napi_callback_info info) {
  napi_value o = opts_arg(env, info);
  if (!o) return NULL;
  return done(env, nsa_check_device(ptr(env, o, "stream")));
}

static void export_fn(napi_env env, napi_value exports, const char* name, napi_callback cb) {
  napi_value fn;
  napi_create_function(env, name, NAPI_AUTO_LENGTH, cb, NULL, &fn);
  napi_set_named_property(env, exports, name, fn);
}

static napi_value Init(napi_env env, napi_value exports) {
  export_fn(env, exports, "attention", Attention);
  export_fn(env, exports, "attentionWorkspaceBytes", AttentionWorkspaceBytes);
  export_fn(env, exports, "headNorm", HeadNorm);
  export_fn(env, exports, "fusedAttention", FusedAttention);
  export_fn(env, exports, "fusedWorkspaceBytes", FusedWorkspaceBytes);
  export_fn(env, exports, "linear", Linear);
  export_fn(env, exports, "rmsnorm", Rmsnorm);
  export_fn(env, exports, "glu", Glu);
  export_fn(env, exports, "gluInterleave", GluInterleave);
  export_fn(env, exports, "rotate", Rotate);
  export_fn(env, exports, "loraPack", LoraPack);
  export_fn(env, exports, "expandI8", ExpandI8);
  export_fn(env, exports, "rope2dTable", Rope2dTable);
  export_fn(env, exports, "ropeTable", RopeTable);
  export_fn(env, exports, "checkDevice", CheckDevice);
  napi_value v;
  napi_create_string_utf8(env, nsa_version(), NAPI_AUTO_LENGTH, &v);
  napi_set_named_property(env, exports, "version", v);
  return exports;
}

NAPI_MODULE(NODE_GYP_MODULE_NAME, Init)
