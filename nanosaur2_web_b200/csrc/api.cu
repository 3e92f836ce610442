// C ABI of libnsattn.so (declared in include/nsattn.h): argument validation, workspace planning,
// TMA descriptor encoding, the per-kernel profiler and the device error word.
#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "nsa_internal.h"
#include "nsattn.h"
#include "ptx.cuh"

namespace {

thread_local std::string g_last_error;

nsa_status fail(nsa_status s, const std::string& msg) {
  g_last_error = msg;
  return s;
}

nsa_status cuda_fail(cudaError_t e, const char* what) {
  return fail(NSA_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

// The library's device error word.  Kernels record the first device-side error here; the host
// reads and clears it in nsa_check_device.  Every device that loads the library has its own copy.
__device__ int g_device_error_word;

constexpr unsigned long long kDefaultTimeoutNs = 2000000000ull;   // 2 s per bounded wait

unsigned long long wait_timeout_ns() {
  static unsigned long long v = [] {
    const char* s = std::getenv("NSA_WAIT_TIMEOUT_MS");
    if (s && *s) {
      const double ms = std::atof(s);
      if (ms > 0) return (unsigned long long)(ms * 1e6);
    }
    return kDefaultTimeoutNs;
  }();
  return v;
}

// ------------------------------------------------------------------------------------ profiler

// Valid (query, key) pairs of an attention launch whose per-batch key counts (kv_len) live on the
// device: the profiler copies them into pinned host memory on the launch's stream, before the start
// event, and counts the pairs when the records are read (after the stop event has completed).
struct PairCount {
  int Bs = 0, Lq = 0, Lk = 0, causal = 0, window = 0, D = 0, Hqs = 0;
  int32_t* kv_host = nullptr;   // [Bs] pinned, or null: every element has Lk keys
};

struct ProfRecord {
  std::string name;
  double flops, bytes;
  cudaEvent_t start, stop;
  PairCount pairs;   // Bs > 0: flops are counted from the copied kv_len at read time
};

std::mutex g_prof_mu;
bool g_prof_on = false;
std::vector<ProfRecord> g_prof_records;
std::vector<cudaEvent_t> g_event_pool;
std::vector<int32_t*> g_pinned_pool;   // pinned kv_len copies, kBatchSlots ints each
constexpr int kBatchSlots = 4096;

cudaEvent_t take_event() {
  if (!g_event_pool.empty()) {
    cudaEvent_t e = g_event_pool.back();
    g_event_pool.pop_back();
    return e;
  }
  cudaEvent_t e = nullptr;
  cudaEventCreate(&e);
  return e;
}

// Valid (query, key) pairs of one batch element with n valid keys: query i sees keys
// [max(0, i - window + 1), min(n, i + 1)) when causal, [.., n) otherwise (the kernels' masks).
double valid_pairs(int Lq, int n, int causal, int window) {
  if (!causal && window <= 0) return (double)Lq * n;
  double pairs = 0;
  for (int i = 0; i < Lq; ++i) {
    const int hi = causal ? std::min(n, i + 1) : n;
    const int lo = window > 0 ? std::max(0, i - window + 1) : 0;
    if (hi > lo) pairs += hi - lo;
  }
  return pairs;
}

double pair_flops(const PairCount& c) {
  double f = 0;
  for (int b = 0; b < c.Bs; ++b) {
    const int n = c.kv_host ? std::min(std::max(c.kv_host[b], 0), c.Lk) : c.Lk;
    f += 4.0 * c.Hqs * valid_pairs(c.Lq, n, c.causal, c.window) * c.D;
  }
  return f;
}

template <class Launch>
cudaError_t profiled(const char* name, double flops, double bytes, cudaStream_t stream, Launch&& launch,
                     PairCount pairs = PairCount{}, const int32_t* kv_len_dev = nullptr) {
  bool on;
  {
    std::lock_guard<std::mutex> lk(g_prof_mu);
    on = g_prof_on;
  }
  if (!on) return launch();
  cudaEvent_t a, b;
  {
    std::lock_guard<std::mutex> lk(g_prof_mu);
    a = take_event();
    b = take_event();
    if (pairs.Bs > 0 && kv_len_dev) {
      if (pairs.Bs > kBatchSlots) {
        pairs.Bs = 0;   // too many elements to copy: keep the host-side count
      } else {
        if (g_pinned_pool.empty()) {
          int32_t* h = nullptr;
          if (cudaMallocHost(&h, kBatchSlots * sizeof(int32_t)) == cudaSuccess) g_pinned_pool.push_back(h);
        }
        if (!g_pinned_pool.empty()) {
          pairs.kv_host = g_pinned_pool.back();
          g_pinned_pool.pop_back();
          cudaMemcpyAsync(pairs.kv_host, kv_len_dev, pairs.Bs * sizeof(int32_t), cudaMemcpyDeviceToHost, stream);
        } else {
          pairs.Bs = 0;
        }
      }
    }
  }
  cudaEventRecord(a, stream);
  const cudaError_t e = launch();
  cudaEventRecord(b, stream);
  std::lock_guard<std::mutex> lk(g_prof_mu);
  g_prof_records.push_back({name, flops, bytes, a, b, pairs});
  return e;
}

// ------------------------------------------------------------------------------------ TMA maps

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// Map over a bf16 matrix [rows][width] with a row pitch of `ld` elements; boxes of
// [box_rows rows][blk elements] with the swizzle the tcgen05 descriptors expect.
bool encode_rows(CUtensorMap* map, const void* base, int64_t width, int64_t ld, int64_t rows, int blk, int box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  const cuuint64_t dims[2] = {(cuuint64_t)width, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)ld * 2};
  const cuuint32_t box[2] = {(cuuint32_t)blk, (cuuint32_t)box_rows};
  const cuuint32_t estr[2] = {1, 1};
  const CUtensorMapSwizzle sw = blk == 64 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B;
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Map over a head-major tile buffer [rows][D] of bf16 (esize 2) or fp32 (esize 4) elements; boxes of
// [box_rows rows][blk elements], swizzled by the box row's width (128 or 64 bytes) as the tcgen05
// descriptors expect.
// atom32: the 128-byte swizzle with 32-byte atoms (MN-major tf32 operands of tcgen05.mma).
bool encode_tiles(CUtensorMap* map, void* base, int D, int64_t rows, int blk, int box_rows, int esize = 2,
                  bool atom32 = false) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  const cuuint64_t dims[2] = {(cuuint64_t)D, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)D * esize};
  const cuuint32_t box[2] = {(cuuint32_t)blk, (cuuint32_t)box_rows};
  const cuuint32_t estr[2] = {1, 1};
  const CUtensorMapSwizzle sw = atom32                 ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B
                                : blk * esize == 128 ? CU_TENSOR_MAP_SWIZZLE_128B
                                                     : CU_TENSOR_MAP_SWIZZLE_64B;
  const CUtensorMapDataType dt = esize == 4 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  return fn(map, dt, 2, base, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// ------------------------------------------------------------------------------------ planning

size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }
int64_t round_up(int64_t x, int64_t a) { return (x + a - 1) / a * a; }

struct Plan {
  int B, Lq, Lk, Hq, group, D;       // full problem
  int b0, Bs, hq0, Hqs, hkv0, Hkvs;  // shard
  int NQ, BN, blk, Lq_pad, Lk_pad;
  int v_rows;         // V tiles' TMA box rows
  bool v_direct_ok;   // the head dim's kernel can read V from the input rows
  bool tf32;          // fp32 tiles and tf32 MMAs (NSA_COMPUTE_TF32)
  int esize;          // bytes per tile element (2 bf16, 4 fp32)
  bool qtmem;
  int split_cap;   // work units whose key range may be split over two CTAs (0: never)
  size_t q_bytes, k_bytes, v_bytes, split_bytes, total;
};

// Scratch of the tail split (nsa::AttnParams::part_o / part_ml / split_count) for `units` units.
size_t split_scratch_bytes(int units, int NQ, int D) {
  if (units <= 0) return 0;
  const size_t rows = (size_t)units * 2 * NQ * nsa::kTileM;
  return align_up(rows * D * 4, 256) + align_up(rows * 2 * 4, 256) + align_up((size_t)units * 2 * 4, 256);
}

struct SplitScratch {
  float* part_o;
  float* part_ml;
  int* count;
};

SplitScratch split_scratch(uint8_t* base, int units, int NQ, int D) {
  const size_t rows = (size_t)units * 2 * NQ * nsa::kTileM;
  SplitScratch s;
  s.part_o = reinterpret_cast<float*>(base);
  s.part_ml = reinterpret_cast<float*>(base + align_up(rows * D * 4, 256));
  s.count = reinterpret_cast<int*>(base + align_up(rows * D * 4, 256) + align_up(rows * 2 * 4, 256));
  return s;
}

unsigned env_flag(const char* name, unsigned dflt) {
  const char* v = std::getenv(name);
  return (v && *v) ? (unsigned)std::atoi(v) : dflt;
}

// Units of the last, partial wave that run as two half-key-range CTAs each, or 0.  The split pays
// when at most half the SMs would otherwise be busy in that wave: the wave then takes half as
// long.  NSA_SPLIT_TAIL=0 turns it off.
int split_units_for(const Plan& pl, int causal, int window) {
  static const unsigned enabled = env_flag("NSA_SPLIT_TAIL", 1);
  if (!enabled || pl.split_cap <= 0 || causal || window || pl.Lk < 2 * pl.BN) return 0;
  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
      sms <= 0)
    return 0;
  const long long units = (long long)pl.Bs * pl.Hqs * (pl.Lq_pad / (pl.NQ * nsa::kTileM));
  const int rem = (int)(units % sms);
  return (rem > 0 && 2 * rem <= sms && rem <= pl.split_cap) ? rem : 0;
}

struct CommonArgs {
  int B, Lq, Lk, H, group, D, causal, window, in_dtype, out_dtype;
  int b_begin, b_count, h_begin, h_count;
  int compute;   // nsa_compute
};

nsa_status make_plan(const CommonArgs& a, Plan* pl) {
  if (a.B < 1 || a.Lq < 1 || a.Lk < 1 || a.H < 1 || a.D < 1)
    return fail(NSA_ERR_INVALID_ARGUMENT, "B, Lq, Lk, H and D must be >= 1");
  if (a.group < 1 || a.H % a.group != 0)
    return fail(NSA_ERR_INVALID_ARGUMENT, "group must divide the number of query heads");
  if (a.compute != NSA_COMPUTE_BF16 && a.compute != NSA_COMPUTE_TF32)
    return fail(NSA_ERR_INVALID_ARGUMENT, "compute must be NSA_COMPUTE_BF16 or NSA_COMPUTE_TF32");
  const bool tf32 = a.compute == NSA_COMPUTE_TF32;
  if (tf32 && (a.D != 96 || a.in_dtype != NSA_F32))
    return fail(NSA_ERR_UNSUPPORTED, "tf32 compute covers head dim 96 with fp32 inputs");
  // the tf32 kernel: one 128-row query tile per unit, 128-key tiles, fp32 boxes of 32 elements
  const nsa::AttnGeometry geo = tf32 ? nsa::AttnGeometry{1, 128, 32, false, 128, false} : nsa::attention_geometry(a.D);
  const int NQ = geo.NQ;
  if (NQ == 0)
    return fail(NSA_ERR_UNSUPPORTED,
                "attention: unsupported head dim " + std::to_string(a.D) + " (64, 96, 128, 256, 512)");
  if (a.in_dtype != NSA_F32 && a.in_dtype != NSA_BF16) return fail(NSA_ERR_INVALID_ARGUMENT, "bad input dtype");
  if (a.out_dtype != NSA_F32 && a.out_dtype != NSA_BF16) return fail(NSA_ERR_INVALID_ARGUMENT, "bad output dtype");
  if (a.window < 0) return fail(NSA_ERR_INVALID_ARGUMENT, "window must be >= 0");
  if (a.causal && a.Lq > a.Lk) return fail(NSA_ERR_INVALID_ARGUMENT, "causal attention needs Lq <= Lk");
  if (a.b_begin < 0 || a.b_begin >= a.B || a.b_count < 0 || a.b_begin + a.b_count > a.B)
    return fail(NSA_ERR_INVALID_ARGUMENT, "batch shard out of range");
  if (a.h_begin < 0 || a.h_begin >= a.H || a.h_count < 0 || a.h_begin + a.h_count > a.H)
    return fail(NSA_ERR_INVALID_ARGUMENT, "head shard out of range");
  Plan p{};
  p.B = a.B; p.Lq = a.Lq; p.Lk = a.Lk; p.Hq = a.H; p.group = a.group; p.D = a.D;
  p.b0 = a.b_begin; p.Bs = a.b_count ? a.b_count : a.B - a.b_begin;
  p.hq0 = a.h_begin; p.Hqs = a.h_count ? a.h_count : a.H - a.h_begin;
  p.hkv0 = p.hq0 / a.group;
  p.Hkvs = (p.hq0 + p.Hqs - 1) / a.group - p.hkv0 + 1;
  p.NQ = NQ;
  p.BN = geo.BN;
  p.blk = geo.blk;
  p.qtmem = geo.qtmem;
  p.v_rows = geo.v_rows;
  p.v_direct_ok = geo.v_direct_ok;
  p.tf32 = tf32;
  p.esize = tf32 ? 4 : 2;
  p.Lq_pad = (int)round_up(a.Lq, (int64_t)NQ * nsa::kTileM);
  p.Lk_pad = (int)round_up(a.Lk, geo.BN);
  const int64_t q_rows = (int64_t)p.Bs * p.Hqs * p.Lq_pad;
  const int64_t kv_rows = (int64_t)p.Bs * p.Hkvs * p.Lk_pad;
  if (q_rows >= (int64_t)1 << 31 || kv_rows >= (int64_t)1 << 31 || (int64_t)p.Bs * p.Hqs * (p.Lq_pad / (NQ * 128)) >= (int64_t)1 << 31)
    return fail(NSA_ERR_UNSUPPORTED, "problem too large for one launch");
  p.q_bytes = align_up((size_t)q_rows * a.D * p.esize, 1024);
  p.k_bytes = align_up((size_t)kv_rows * a.D * p.esize, 1024);
  p.v_bytes = p.k_bytes;
  const long long units = (long long)p.Bs * p.Hqs * (p.Lq_pad / (NQ * nsa::kTileM));
  p.split_cap = (NQ == 2 && !a.causal && !a.window) ? (int)std::min<long long>(units, nsa::kSplitUnitsMax) : 0;
  p.split_bytes = split_scratch_bytes(p.split_cap, NQ, a.D);
  p.total = p.q_bytes + p.k_bytes + p.v_bytes + p.split_bytes + 1024;
  *pl = p;
  return NSA_OK;
}

nsa_status check_out(const void* out, int out_dtype, int64_t ldo, int64_t oOff, int64_t o_bstride) {
  if (!out) return fail(NSA_ERR_INVALID_ARGUMENT, "out is NULL");
  const int64_t v = out_dtype == NSA_F32 ? 4 : 8;   // 16-byte vector stores of each row segment
  if ((reinterpret_cast<uintptr_t>(out) & 15) || ldo % v || oOff % v || o_bstride % v)
    return fail(NSA_ERR_INVALID_ARGUMENT, "out, ldo, oOff and o_bstride must keep rows 16-byte aligned");
  return NSA_OK;
}

// Attention parameters shared by every entry point; the caller sets the Q / K / V tile coordinates.
nsa::AttnParams attn_params(const Plan& pl, const CommonArgs& a, const float* bias, int bias_start, int bias_len,
                            int64_t bias_bstride, const int32_t* kv_len, float scale, void* out, int64_t ldo,
                            int64_t o_bstride, int64_t oOff, int* err) {
  nsa::AttnParams ap{};
  ap.B = pl.Bs;
  ap.Hq = pl.Hqs;
  ap.Hkv = pl.Hkvs;
  ap.group = pl.group;
  ap.b_begin = pl.b0;
  ap.hq_begin = pl.hq0;
  ap.hkv_begin = pl.hkv0;
  ap.Lq = pl.Lq;
  ap.Lq_pad = pl.Lq_pad;
  ap.Lk = pl.Lk;
  ap.Lk_pad = pl.Lk_pad;
  ap.kv_len = kv_len;
  ap.bias = bias_len > 0 ? bias : nullptr;
  ap.bias_start = bias_start;
  ap.bias_len = bias_len;
  ap.bias_bstride = bias_bstride;
  const float s = scale > 0.f ? scale : 1.0f / std::sqrt((float)pl.D);
  ap.scale_log2 = s * 1.4426950408889634f;
  ap.causal = a.causal;
  ap.window = a.window;
  ap.out = out;
  ap.out_f32 = a.out_dtype == NSA_F32;
  ap.out_ld = ldo;
  ap.out_bstride = o_bstride;
  ap.out_off = oOff;
  ap.q_blocks = pl.Lq_pad / (pl.NQ * nsa::kTileM);
  ap.err = err;
  ap.timeout_ns = wait_timeout_ns();
  return ap;
}

void set_split(nsa::AttnParams* ap, const Plan& pl, const CommonArgs& a, const SplitScratch& s) {
  const int r = split_units_for(pl, a.causal, a.window);
  if (r <= 0) return;
  ap->split_units = r;
  ap->split_first = pl.Bs * pl.Hqs * (pl.Lq_pad / (pl.NQ * nsa::kTileM)) - r;
  ap->part_o = s.part_o;
  ap->part_ml = s.part_ml;
  ap->split_count = s.count;
}

// Algorithmic flops of one attention launch: 4 * B * H * valid pairs * D (app/gpu/ops.js:207), the
// causal and window masks counted here; per-batch key counts on the device (kv_len) are counted by
// the profiler from a copy (attn_pairs).
double attn_flops(const Plan& pl, const CommonArgs& a) {
  return 4.0 * pl.Bs * pl.Hqs * valid_pairs(pl.Lq, pl.Lk, a.causal, a.window) * pl.D;
}

PairCount attn_pairs(const Plan& pl, const CommonArgs& a) {
  PairCount c;
  c.Bs = pl.Bs;
  c.Lq = pl.Lq;
  c.Lk = pl.Lk;
  c.causal = a.causal;
  c.window = a.window;
  c.D = pl.D;
  c.Hqs = pl.Hqs;
  return c;
}

// Prologue + attention launches shared by nsa_attention and nsa_fused_attention.
nsa_status run(const Plan& pl, nsa::PrologueParams pp, const CommonArgs& a, const float* bias, int bias_start,
               int bias_len, int64_t bias_bstride, const int32_t* kv_len, float scale, void* out, int64_t ldo,
               int64_t o_bstride, int64_t oOff, void* ws, size_t ws_bytes, cudaStream_t stream) {
  if (!ws || ws_bytes < pl.total)
    return fail(NSA_ERR_WORKSPACE, "workspace of " + std::to_string(pl.total) + " bytes required, got " +
                                       std::to_string(ws_bytes));
  uint8_t* base = reinterpret_cast<uint8_t*>(align_up(reinterpret_cast<uintptr_t>(ws), 1024));
  auto* Qs = reinterpret_cast<__nv_bfloat16*>(base);
  auto* Ks = reinterpret_cast<__nv_bfloat16*>(base + pl.q_bytes);
  auto* Vs = reinterpret_cast<__nv_bfloat16*>(base + pl.q_bytes + pl.k_bytes);

  int* err = nsa::device_error_word();
  if (!err) return fail(NSA_ERR_CUDA, "cannot resolve the device error word on this device");

  pp.src_f32 = a.in_dtype == NSA_F32;
  pp.out_f32 = pl.tf32 ? 1 : 0;
  pp.B = pl.Bs;
  pp.b_begin = pl.b0;
  pp.Lq = pl.Lq;
  pp.Lk = pl.Lk;
  pp.Hq = pl.Hqs;
  pp.Hkv = pl.Hkvs;
  pp.D = pl.D;
  pp.hq_begin = pl.hq0;
  pp.hkv_begin = pl.hkv0;
  pp.kv_len = kv_len;
  pp.out[0] = {Qs, (int64_t)pl.Hqs * pl.Lq_pad * pl.D, (int64_t)pl.Lq_pad * pl.D, pl.D};
  pp.out[1] = {Ks, (int64_t)pl.Hkvs * pl.Lk_pad * pl.D, (int64_t)pl.Lk_pad * pl.D, pl.D};
  pp.out[2] = {Vs, (int64_t)pl.Hkvs * pl.Lk_pad * pl.D, (int64_t)pl.Lk_pad * pl.D, pl.D};
  pp.rows[0] = pl.Lq_pad;
  pp.rows[1] = pp.rows[2] = pl.Lk_pad;
  for (int i = 0; i < 3; ++i) pp.row0[i] = pp.src_row0[i] = 0;
  const SplitScratch split = split_scratch(base + pl.q_bytes + pl.k_bytes + pl.v_bytes, pl.split_cap, pl.NQ, pl.D);
  pp.zero_ptr = pl.split_cap > 0 ? split.count : nullptr;   // the attention's split counters start at zero
  pp.zero_count = 2 * pl.split_cap;   // two counters (query tiles) per split unit
  auto al16 = [](const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15) == 0; };
  pp.skip_q = 0;
  // V needs no normalisation: for bf16 rows that a tiled map can cover (16-byte aligned rows and
  // head offsets, whole rows per batch element) the attention kernel reads V tiles of valid keys
  // straight from the input, and the prologue writes only the last partial tile and the padding.
  static const unsigned v_direct_enabled = env_flag("NSA_V_DIRECT", 1);   // NSA_V_DIRECT=0 turns it off
  const bool v_direct = v_direct_enabled && pl.v_direct_ok && a.in_dtype == NSA_BF16 && al16(pp.v.ptr) &&
                        pp.v.ld % 8 == 0 && pp.v.off % 8 == 0 &&
                        (pl.B == 1 || (pp.v.bstride > 0 && pp.v.bstride % pp.v.ld == 0)) &&
                        pp.v.off + (int64_t)(pl.hkv0 + pl.Hkvs) * pl.D <= pp.v.ld;
  pp.v_tile = v_direct ? pl.BN : 0;
  const double in_elem = a.in_dtype == NSA_F32 ? 4.0 : 2.0;
  // algorithmic bytes: q and k rows, and the v rows the prologue writes (all, or about one tile)
  const double v_rows = v_direct ? (double)pl.BN : (double)pl.Lk;
  const double pro_bytes = (double)pl.Bs * ((double)pl.Lq * pl.Hqs + (pl.Lk + v_rows) * pl.Hkvs) * pl.D *
                           (in_elem + 2.0);
  cudaError_t e = profiled("prologue", 0.0, pro_bytes, stream, [&] { return nsa::launch_prologue(pp, stream); });
  if (e != cudaSuccess) return cuda_fail(e, "prologue launch");

  CUtensorMap tq, tk, tv;
  const bool maps_ok = encode_tiles(&tq, Qs, pl.D, (int64_t)pl.Bs * pl.Hqs * pl.Lq_pad, pl.blk, nsa::kTileM, pl.esize);
  if (!maps_ok || !encode_tiles(&tk, Ks, pl.D, (int64_t)pl.Bs * pl.Hkvs * pl.Lk_pad, pl.blk, pl.BN, pl.esize) ||
      !encode_tiles(&tv, Vs, pl.D, (int64_t)pl.Bs * pl.Hkvs * pl.Lk_pad, pl.blk, pl.v_rows, pl.esize, pl.tf32))
    return fail(NSA_ERR_CUDA, "cuTensorMapEncodeTiled failed (driver entry point unavailable?)");
  CUtensorMap tvd = tv;
  if (v_direct) {
    // the input rows of every batch element: [B * rows per element][ld]
    const int64_t total_rows = pl.B == 1 ? pp.v.rows : (int64_t)(pl.B - 1) * (pp.v.bstride / pp.v.ld) + pp.v.rows;
    if (!encode_rows(&tvd, pp.v.ptr, pp.v.ld, pp.v.ld, total_rows, pl.blk, pl.BN))
      return fail(NSA_ERR_CUDA, "cuTensorMapEncodeTiled failed (driver entry point unavailable?)");
  }

  nsa::AttnParams ap = attn_params(pl, a, bias, bias_start, bias_len, bias_bstride, kv_len, scale, out, ldo,
                                   o_bstride, oOff, err);
  ap.k_x0 = ap.v_x0 = ap.kv_xh = 0;
  ap.kv_yb = pl.Hkvs * pl.Lk_pad;
  ap.kv_yh = pl.Lk_pad;
  set_split(&ap, pl, a, split);
  if (v_direct) {
    ap.v_direct = 1;
    ap.vd_x0 = (int)(pp.v.off + (int64_t)pl.hkv0 * pl.D);
    ap.vd_xh = pl.D;
    ap.vd_yb = pl.B == 1 ? 0 : (int)(pp.v.bstride / pp.v.ld);
  }
  // the prologue's head-major Q tiles, already normalised and rotated
  ap.q_x0 = 0;
  ap.q_xh = 0;
  ap.q_yb = pl.Hqs * pl.Lq_pad;
  ap.q_yh = pl.Lq_pad;
  ap.q_b0 = pl.b0;
  ap.q_h0 = pl.hq0;
  const double flops = attn_flops(pl, a);
  e = profiled(pl.tf32 ? "attention_tf32" : "attention", flops, 0.0, stream,
               [&] {
                 return pl.tf32 ? nsa::launch_attention_tf32(ap, tq, tk, tv, stream)
                                : nsa::launch_attention(ap, pl.D, tq, tk, tv, tvd, stream);
               },
               attn_pairs(pl, a), kv_len ? kv_len + pl.b0 : nullptr);
  if (e != cudaSuccess) return cuda_fail(e, "attention launch");
  return NSA_OK;
}

__global__ void selftest_wait_kernel(int* err, unsigned long long timeout_ns) {
  __shared__ uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    nsa::mbar_init(&bar, 1);
    abort_flag = 0;
    nsa::fence_mbar_init();
  }
  __syncthreads();
  // nothing ever arrives on `bar`: the bounded wait must expire and record the error
  if (threadIdx.x == 0) nsa::wait_bounded(&bar, 0, &abort_flag, err, 0x1E5, timeout_ns);
  __syncthreads();
}

CommonArgs common_from(const nsa_attention_desc* d) {
  return CommonArgs{d->B, d->Lq, d->Lk, d->H, d->group, d->D, d->causal, d->window, d->in_dtype, d->out_dtype,
                    d->b_begin, d->b_count, d->h_begin, d->h_count, d->compute};
}

CommonArgs common_from(const nsa_fused_desc* d) {
  const int group = d->Hkv > 0 ? d->Hq / d->Hkv : 0;
  return CommonArgs{d->B, d->Lq, d->Lk, d->Hq, group, d->D, d->causal, d->window, d->in_dtype, d->out_dtype,
                    d->b_begin, d->b_count, d->h_begin, d->h_count, d->compute};
}

// ------------------------------------------------------------------------------------ sequence shards

// One rank's part of a sequence-sharded fused call: the plan of its q_count query rows over all Lk
// keys, and the layout of its q_prime / kv_packed buffers.
struct SeqPlan {
  Plan pl;             // Lq = q_count, Lq_pad = q_pad; Lk / Lk_pad of the whole key sequence
  CommonArgs a;        // the descriptor with Lq = q_count
  int L;               // image rows (the descriptor's Lq)
  int q_begin, q_count, img_row0, text_row0;
  int64_t kv_ld;       // elements per kv_packed row: 2 * Hkv * D
  size_t q_tiles_bytes;  // the q' tiles at the start of q_prime; the tail-split scratch follows
  size_t q_bytes, kv_bytes;
};

nsa_status make_seq_plan(const nsa_fused_desc* d, const nsa_seq_shard* s, SeqPlan* sp) {
  if (!d || !s) return fail(NSA_ERR_INVALID_ARGUMENT, "desc and shard must not be NULL");
  if (d->Hkv < 1 || d->Hq % d->Hkv) return fail(NSA_ERR_INVALID_ARGUMENT, "Hkv must divide Hq");
  if (d->Lk < d->Lq) return fail(NSA_ERR_INVALID_ARGUMENT, "Lk must be >= Lq (query rows are also key rows)");
  // Causal masks and windows compare query and key indices; they are exact when the shard holds every
  // query row (q_begin 0, q_count Lq: one GPU), where local and global query indices coincide.
  if ((d->causal || d->window) && !(s->q_begin == 0 && s->q_count == d->Lq))
    return fail(NSA_ERR_UNSUPPORTED, "a causal mask or a window needs a shard that holds every query row");
  if (d->h_begin != 0 || (d->h_count != 0 && d->h_count != d->Hq))
    return fail(NSA_ERR_UNSUPPORTED, "sequence sharding takes whole heads (h_begin 0, h_count 0 or Hq)");
  if (s->q_begin < 0 || s->q_count < 1 || (int64_t)s->q_begin + s->q_count > d->Lq)
    return fail(NSA_ERR_INVALID_ARGUMENT, "shard rows [q_begin, q_begin + q_count) must lie in [0, Lq)");
  if (s->qkv_image_row0 < 0 || s->qkv_text_row0 < 0)
    return fail(NSA_ERR_INVALID_ARGUMENT, "qkv_image_row0 and qkv_text_row0 must be >= 0");
  if (d->D == 512)
    return fail(NSA_ERR_UNSUPPORTED, "head dim 512 runs through nsa_attention / nsa_fused_attention, not sequence shards");
  if (d->compute != NSA_COMPUTE_BF16)
    return fail(NSA_ERR_UNSUPPORTED, "sequence shards compute in bf16 (compute = NSA_COMPUTE_BF16)");
  SeqPlan p{};
  p.a = common_from(d);
  p.a.Lq = s->q_count;
  nsa_status st = make_plan(p.a, &p.pl);
  if (st != NSA_OK) return st;
  p.L = d->Lq;
  p.q_begin = s->q_begin;
  p.q_count = s->q_count;
  p.img_row0 = s->qkv_image_row0;
  p.text_row0 = s->qkv_text_row0;
  p.kv_ld = 2LL * d->Hkv * d->D;
  if ((int64_t)p.pl.Bs * p.pl.Lk_pad >= (int64_t)1 << 31)
    return fail(NSA_ERR_UNSUPPORTED, "problem too large for one launch");
  p.q_tiles_bytes = align_up((size_t)p.pl.Bs * p.pl.Hqs * p.pl.Lq_pad * p.pl.D * 2, 1024);
  p.q_bytes = p.q_tiles_bytes + p.pl.split_bytes;
  p.kv_bytes = (size_t)p.pl.Bs * p.pl.Lk_pad * p.kv_ld * 2;
  *sp = p;
  return NSA_OK;
}

bool aligned16(const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15) == 0; }

// ------------------------------------------------------------------------------------ CUDA IPC

using GetAddressRangeFn = CUresult (*)(CUdeviceptr*, size_t*, CUdeviceptr);

GetAddressRangeFn address_range_fn() {
  static GetAddressRangeFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<GetAddressRangeFn>(p);
  });
  return fn;
}

std::mutex g_ipc_mu;
std::vector<std::pair<void*, void*>> g_ipc_open;   // (pointer handed out, mapping base)

}  // namespace

namespace nsa {

void record_error(const std::string& msg) { g_last_error = msg; }

// Resolved at every call rather than cached: after a cudaDeviceReset (or anything else that reloads
// the module) a cached address would be stale, and the lookup is cheap.
int* device_error_word() {
  void* p = nullptr;
  if (cudaGetSymbolAddress(&p, g_device_error_word) != cudaSuccess) return nullptr;
  return static_cast<int*>(p);
}

int device_sm_count() {
  static std::mutex mu;
  static int cache[128] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 128) return 148;
  std::lock_guard<std::mutex> lk(mu);
  if (cache[dev] <= 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) return 148;
    cache[dev] = n;
  }
  return cache[dev];
}

cudaError_t once_per_device(DeviceOnce& state, cudaError_t (*setup)()) {
  static std::mutex mu;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 128) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lk(mu);
  if (state.done[dev]) return cudaSuccess;
  e = setup();
  if (e == cudaSuccess) state.done[dev] = true;
  return e;
}

}  // namespace nsa

extern "C" {

const char* nsa_version(void) { return "nsattn 0.1.0 sm_100a"; }

const char* nsa_last_error(void) { return g_last_error.c_str(); }

const char* nsa_status_string(nsa_status s) {
  switch (s) {
    case NSA_OK: return "ok";
    case NSA_ERR_INVALID_ARGUMENT: return "invalid argument";
    case NSA_ERR_UNSUPPORTED: return "unsupported";
    case NSA_ERR_WORKSPACE: return "workspace too small";
    case NSA_ERR_CUDA: return "cuda error";
    case NSA_ERR_DEVICE: return "device-side error";
  }
  return "unknown status";
}

size_t nsa_attention_workspace_size(const nsa_attention_desc* desc) {
  if (!desc) return 0;
  Plan pl;
  if (make_plan(common_from(desc), &pl) != NSA_OK) return 0;
  return pl.total;
}

nsa_status nsa_attention(const nsa_attention_desc* d, const void* q, const void* k, const void* v, const float* bias,
                         const int32_t* kv_len, void* out, void* workspace, size_t workspace_bytes, void* stream) {
  if (!d) return fail(NSA_ERR_INVALID_ARGUMENT, "desc is NULL");
  if (!q || !k || !v) return fail(NSA_ERR_INVALID_ARGUMENT, "q, k and v must be device pointers");
  const CommonArgs a = common_from(d);
  Plan pl;
  nsa_status st = make_plan(a, &pl);
  if (st != NSA_OK) return st;
  if ((st = check_out(out, d->out_dtype, d->ldo, d->oOff, d->o_bstride)) != NSA_OK) return st;
  if (d->biasLen < 0) return fail(NSA_ERR_INVALID_ARGUMENT, "biasLen must be >= 0");
  if (d->biasLen > 0 && !bias) return fail(NSA_ERR_INVALID_ARGUMENT, "biasLen > 0 needs a bias pointer");
  nsa::PrologueParams pp{};
  pp.q = {q, d->ldq, d->q_bstride, d->qOff, d->Lq};
  pp.k = {k, d->ldk, d->k_bstride, d->kOff, d->Lk};
  pp.v = {v, d->ldv, d->v_bstride, d->vOff, d->Lk};
  pp.q_w = nullptr;
  pp.k_w = nullptr;
  pp.cs = nullptr;
  pp.rope_rows = 0;
  pp.eps = 0.f;
  return run(pl, pp, a, bias, d->biasStart, bias ? d->biasLen : 0, d->bias_bstride, kv_len, d->scale, out, d->ldo,
             d->o_bstride, d->oOff, workspace, workspace_bytes, static_cast<cudaStream_t>(stream));
}

size_t nsa_fused_attention_workspace_size(const nsa_fused_desc* desc) {
  if (!desc) return 0;
  Plan pl;
  if (make_plan(common_from(desc), &pl) != NSA_OK) return 0;
  return pl.total;
}

nsa_status nsa_fused_attention(const nsa_fused_desc* d, const void* qkv, const float* q_norm_w, const float* k_norm_w,
                               const float* cs, const int32_t* kv_len, const float* bias, void* out, void* workspace,
                               size_t workspace_bytes, void* stream) {
  if (!d) return fail(NSA_ERR_INVALID_ARGUMENT, "desc is NULL");
  if (!qkv) return fail(NSA_ERR_INVALID_ARGUMENT, "qkv is NULL");
  if (!q_norm_w || !k_norm_w) return fail(NSA_ERR_INVALID_ARGUMENT, "q/k norm weights are required");
  if (d->Hkv < 1 || d->Hq % d->Hkv) return fail(NSA_ERR_INVALID_ARGUMENT, "Hkv must divide Hq");
  if (d->Lk < d->Lq) return fail(NSA_ERR_INVALID_ARGUMENT, "Lk must be >= Lq (query rows are also key rows)");
  const CommonArgs a = common_from(d);
  Plan pl;
  nsa_status st = make_plan(a, &pl);
  if (st != NSA_OK) return st;
  if ((st = check_out(out, d->out_dtype, d->ldo, d->oOff, d->o_bstride)) != NSA_OK) return st;
  if (d->biasLen < 0) return fail(NSA_ERR_INVALID_ARGUMENT, "biasLen must be >= 0");
  if (d->biasLen > 0 && !bias) return fail(NSA_ERR_INVALID_ARGUMENT, "biasLen > 0 needs a bias pointer");
  if (cs && d->D % 2) return fail(NSA_ERR_INVALID_ARGUMENT, "RoPE needs an even head dim");
  nsa::PrologueParams pp{};
  pp.q = {qkv, d->ld, d->bstride, d->qOff, d->Lk};
  pp.k = {qkv, d->ld, d->bstride, d->kOff, d->Lk};
  pp.v = {qkv, d->ld, d->bstride, d->vOff, d->Lk};
  pp.q_w = q_norm_w;
  pp.k_w = k_norm_w;
  pp.cs = cs;
  pp.sin_off = d->sinOff;
  pp.rope_rows = cs ? d->Lq : 0;
  pp.eps = d->eps;
  return run(pl, pp, a, bias, d->biasStart, bias ? d->biasLen : 0, d->bias_bstride, kv_len, d->scale, out, d->ldo,
             d->o_bstride, d->oOff, workspace, workspace_bytes, static_cast<cudaStream_t>(stream));
}

nsa_status nsa_head_norm(void* X, int32_t dtype, const float* weight, int32_t L, int32_t H, int32_t D, int64_t ld,
                         int64_t colOff, int64_t rowOff, const float* cs, int64_t sinOff, float eps, void* stream) {
  if (!X || !weight) return fail(NSA_ERR_INVALID_ARGUMENT, "X and weight must be device pointers");
  if (dtype != NSA_F32 && dtype != NSA_BF16) return fail(NSA_ERR_INVALID_ARGUMENT, "bad dtype");
  if (L < 0 || H < 1 || D < 2 || D % 2) return fail(NSA_ERR_INVALID_ARGUMENT, "need L >= 0, H >= 1, even D");
  const double bytes = 2.0 * L * H * D * (dtype == NSA_F32 ? 4.0 : 2.0);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e = profiled(cs ? "head_norm_rope" : "head_norm", 0.0, bytes, s, [&] {
    return nsa::launch_head_norm(X, dtype == NSA_F32, weight, L, H, D, ld, colOff, rowOff, cs, sinOff, eps, s);
  });
  if (e != cudaSuccess) return cuda_fail(e, "head_norm launch");
  return NSA_OK;
}

nsa_status nsa_rope2d_table(int32_t h, int32_t w, int32_t D, float* out, void* stream) {
  if (!out) return fail(NSA_ERR_INVALID_ARGUMENT, "out is NULL");
  if (h < 1 || w < 1 || D < 4 || D % 4) return fail(NSA_ERR_INVALID_ARGUMENT, "need h, w >= 1 and D % 4 == 0");
  cudaError_t e = nsa::launch_rope2d_table(h, w, D, out, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "rope2d table launch");
  return NSA_OK;
}

nsa_status nsa_rope1d_table(int32_t L, int32_t D, float theta, float* out, void* stream) {
  if (!out) return fail(NSA_ERR_INVALID_ARGUMENT, "out is NULL");
  if (L < 1 || D < 2 || D % 2 || !(theta > 0.f)) return fail(NSA_ERR_INVALID_ARGUMENT, "need L >= 1, even D, theta > 0");
  cudaError_t e = nsa::launch_rope1d_table(L, D, theta, out, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "rope1d table launch");
  return NSA_OK;
}

nsa_status nsa_check_device(void* stream) {
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int* w = nsa::device_error_word();
  if (!w) return fail(NSA_ERR_CUDA, "cannot resolve the device error word on this device");
  int host = 0;
  cudaError_t e = cudaMemcpyAsync(&host, w, sizeof(int), cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaMemsetAsync(w, 0, sizeof(int), s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return cuda_fail(e, "device check");
  if (host != 0) {
    char buf[96];
    std::snprintf(buf, sizeof buf, "device-side error 0x%x (a bounded wait expired)", host);
    return fail(NSA_ERR_DEVICE, buf);
  }
  return NSA_OK;
}

nsa_status nsa_selftest_wait_timeout(int32_t timeout_us, void* stream) {
  if (timeout_us < 1 || timeout_us > 10000000) return fail(NSA_ERR_INVALID_ARGUMENT, "timeout_us in [1, 1e7]");
  int* w = nsa::device_error_word();
  if (!w) return fail(NSA_ERR_CUDA, "cannot resolve the device error word on this device");
  selftest_wait_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(w, (unsigned long long)timeout_us * 1000ull);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "self-test launch");
  return NSA_OK;
}

void nsa_profiler_enable(int32_t on) {
  std::lock_guard<std::mutex> lk(g_prof_mu);
  g_prof_on = on != 0;
}

void nsa_profiler_reset(void) {
  std::lock_guard<std::mutex> lk(g_prof_mu);
  for (auto& r : g_prof_records) {
    cudaEventSynchronize(r.stop);
    g_event_pool.push_back(r.start);
    g_event_pool.push_back(r.stop);
    if (r.pairs.kv_host) g_pinned_pool.push_back(r.pairs.kv_host);
  }
  g_prof_records.clear();
}

int32_t nsa_profiler_read(nsa_kernel_stat* out, int32_t max_entries) {
  std::lock_guard<std::mutex> lk(g_prof_mu);
  std::vector<nsa_kernel_stat> stats;
  for (auto& r : g_prof_records) {
    cudaEventSynchronize(r.stop);
    float ms = 0.f;
    cudaEventElapsedTime(&ms, r.start, r.stop);
    nsa_kernel_stat* st = nullptr;
    for (auto& s : stats)
      if (r.name == s.name) st = &s;
    if (!st) {
      stats.push_back(nsa_kernel_stat{});
      st = &stats.back();
      std::snprintf(st->name, sizeof st->name, "%s", r.name.c_str());
    }
    st->launches += 1;
    st->total_ms += ms;
    st->flops += r.pairs.kv_host ? pair_flops(r.pairs) : r.flops;
    st->bytes += r.bytes;
  }
  const int32_t n = (int32_t)stats.size();
  for (int32_t i = 0; out && i < n && i < max_entries; ++i) out[i] = stats[i];
  return n;
}

nsa_status nsa_ipc_export(const void* device_ptr, void* handle_out) {
  if (!device_ptr || !handle_out) return fail(NSA_ERR_INVALID_ARGUMENT, "device_ptr and handle_out are required");
  GetAddressRangeFn range = address_range_fn();
  if (!range) return fail(NSA_ERR_CUDA, "cuMemGetAddressRange unavailable");
  CUdeviceptr base = 0;
  size_t size = 0;
  if (range(&base, &size, reinterpret_cast<CUdeviceptr>(device_ptr)) != CUDA_SUCCESS)
    return fail(NSA_ERR_INVALID_ARGUMENT, "device_ptr is not in a device allocation");
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base));
  if (e != cudaSuccess) return cuda_fail(e, "cudaIpcGetMemHandle");
  const uint64_t off = reinterpret_cast<uintptr_t>(device_ptr) - static_cast<uintptr_t>(base);
  std::memcpy(handle_out, &h, sizeof h);
  std::memcpy(static_cast<uint8_t*>(handle_out) + sizeof h, &off, sizeof off);
  return NSA_OK;
}

nsa_status nsa_ipc_import(const void* handle, void** device_ptr_out) {
  if (!handle || !device_ptr_out) return fail(NSA_ERR_INVALID_ARGUMENT, "handle and device_ptr_out are required");
  cudaIpcMemHandle_t h;
  uint64_t off = 0;
  std::memcpy(&h, handle, sizeof h);
  std::memcpy(&off, static_cast<const uint8_t*>(handle) + sizeof h, sizeof off);
  void* base = nullptr;
  cudaError_t e = cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return cuda_fail(e, "cudaIpcOpenMemHandle");
  void* ptr = static_cast<uint8_t*>(base) + off;
  {
    std::lock_guard<std::mutex> lk(g_ipc_mu);
    g_ipc_open.emplace_back(ptr, base);
  }
  *device_ptr_out = ptr;
  return NSA_OK;
}

nsa_status nsa_ipc_close(void* device_ptr) {
  void* base = nullptr;
  {
    std::lock_guard<std::mutex> lk(g_ipc_mu);
    for (size_t i = 0; i < g_ipc_open.size(); ++i)
      if (g_ipc_open[i].first == device_ptr) {
        base = g_ipc_open[i].second;
        g_ipc_open.erase(g_ipc_open.begin() + (long)i);
        break;
      }
  }
  if (!base) return fail(NSA_ERR_INVALID_ARGUMENT, "not a pointer returned by nsa_ipc_import");
  cudaError_t e = cudaIpcCloseMemHandle(base);
  if (e != cudaSuccess) return cuda_fail(e, "cudaIpcCloseMemHandle");
  return NSA_OK;
}

nsa_status nsa_memcpy_async(void* dst, const void* src, size_t bytes, void* stream) {
  if (!dst || !src) return fail(NSA_ERR_INVALID_ARGUMENT, "dst and src are required");
  cudaError_t e = cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDefault, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "cudaMemcpyAsync");
  return NSA_OK;
}

nsa_status nsa_seq_shard_buffer_sizes(const nsa_fused_desc* desc, const nsa_seq_shard* shard, size_t* q_prime_bytes,
                                      size_t* kv_packed_bytes, int32_t* kv_rows) {
  SeqPlan sp;
  nsa_status st = make_seq_plan(desc, shard, &sp);
  if (st != NSA_OK) return st;
  if (q_prime_bytes) *q_prime_bytes = sp.q_bytes;
  if (kv_packed_bytes) *kv_packed_bytes = sp.kv_bytes;
  if (kv_rows) *kv_rows = sp.pl.Lk_pad;
  return NSA_OK;
}

nsa_status nsa_seq_shard_prologue(const nsa_fused_desc* d, const nsa_seq_shard* s, const void* qkv,
                                  const float* q_norm_w, const float* k_norm_w, const float* cs, const int32_t* kv_len,
                                  void* q_prime, void* kv_packed, void* stream) {
  return nsa_seq_shard_prologue_peers(d, s, qkv, q_norm_w, k_norm_w, cs, kv_len, q_prime, kv_packed, nullptr, 0,
                                      stream);
}

nsa_status nsa_seq_shard_prologue_peers(const nsa_fused_desc* d, const nsa_seq_shard* s, const void* qkv,
                                        const float* q_norm_w, const float* k_norm_w, const float* cs,
                                        const int32_t* kv_len, void* q_prime, void* kv_packed,
                                        void* const* kv_peers, int32_t n_peers, void* stream) {
  if (n_peers < 0 || n_peers > nsa::kMaxPeers || (n_peers > 0 && !kv_peers))
    return fail(NSA_ERR_INVALID_ARGUMENT, "n_peers must be in [0, 8] with a kv_peers array");
  for (int i = 0; i < n_peers; ++i)
    if (!kv_peers[i] || (reinterpret_cast<uintptr_t>(kv_peers[i]) & 15))
      return fail(NSA_ERR_INVALID_ARGUMENT, "kv_peers must be 16-byte aligned device pointers");
  SeqPlan sp;
  nsa_status st = make_seq_plan(d, s, &sp);
  if (st != NSA_OK) return st;
  if (!qkv) return fail(NSA_ERR_INVALID_ARGUMENT, "qkv is NULL");
  if (!q_norm_w || !k_norm_w) return fail(NSA_ERR_INVALID_ARGUMENT, "q/k norm weights are required");
  if (!q_prime || !kv_packed || !aligned16(q_prime) || !aligned16(kv_packed))
    return fail(NSA_ERR_INVALID_ARGUMENT, "q_prime and kv_packed must be 16-byte aligned device pointers");
  if (cs && d->D % 2) return fail(NSA_ERR_INVALID_ARGUMENT, "RoPE needs an even head dim");
  const Plan& pl = sp.pl;
  nsa::PrologueParams pp{};
  pp.q = {qkv, d->ld, d->bstride, d->qOff, d->Lk};
  pp.k = {qkv, d->ld, d->bstride, d->kOff, d->Lk};
  pp.v = {qkv, d->ld, d->bstride, d->vOff, d->Lk};
  pp.q_w = q_norm_w;
  pp.k_w = k_norm_w;
  pp.cs = cs;
  pp.sin_off = d->sinOff;
  pp.rope_rows = cs ? sp.L : 0;
  pp.eps = d->eps;
  pp.src_f32 = d->in_dtype == NSA_F32;
  pp.B = pl.Bs;
  pp.b_begin = pl.b0;
  pp.Lq = sp.q_begin + sp.q_count;   // query rows past the shard are zero padding
  pp.Lk = pl.Lk;
  pp.Hq = pl.Hqs;
  pp.Hkv = pl.Hkvs;
  pp.D = pl.D;
  pp.hq_begin = 0;
  pp.hkv_begin = 0;
  pp.kv_len = kv_len;
  auto* Q = static_cast<__nv_bfloat16*>(q_prime);
  auto* KV = static_cast<__nv_bfloat16*>(kv_packed);
  const int64_t kv_elem = (int64_t)pl.Lk_pad * sp.kv_ld;   // one batch element of kv_packed
  const int64_t v_col = (int64_t)pl.Hkvs * pl.D;
  // the shard's own image rows: q' tiles, and k'|v' at their global key rows
  pp.out[0] = {Q, (int64_t)pl.Hqs * pl.Lq_pad * pl.D, (int64_t)pl.Lq_pad * pl.D, pl.D};
  pp.out[1] = {KV + sp.q_begin * sp.kv_ld, kv_elem, pl.D, sp.kv_ld};
  pp.out[2] = {KV + sp.q_begin * sp.kv_ld + v_col, kv_elem, pl.D, sp.kv_ld};
  pp.rows[0] = pl.Lq_pad;
  pp.rows[1] = pp.rows[2] = sp.q_count;
  for (int i = 0; i < 3; ++i) {
    pp.row0[i] = sp.q_begin;
    pp.src_row0[i] = sp.img_row0;
  }
  // the image rows' k'|v' also go to the other GPUs' kv_packed (same offsets, through their mappings)
  pp.n_peers = n_peers;
  for (int i = 0; i < n_peers; ++i)
    pp.peer_off[i] = reinterpret_cast<const uint8_t*>(kv_peers[i]) - reinterpret_cast<const uint8_t*>(kv_packed);
  pp.skip_q = 0;
  const SplitScratch split =
      split_scratch(static_cast<uint8_t*>(q_prime) + sp.q_tiles_bytes, pl.split_cap, pl.NQ, pl.D);
  pp.zero_ptr = pl.split_cap > 0 ? split.count : nullptr;   // the attention's split counters start at zero
  pp.zero_count = 2 * pl.split_cap;   // two counters (query tiles) per split unit
  const double in_elem = d->in_dtype == NSA_F32 ? 4.0 : 2.0;
  const cudaStream_t strm = static_cast<cudaStream_t>(stream);
  double bytes = (double)pl.Bs * sp.q_count * (pl.Hqs + 2.0 * pl.Hkvs) * pl.D * (in_elem + 2.0);
  cudaError_t e = profiled("prologue", 0.0, bytes, strm, [&] { return nsa::launch_prologue(pp, strm); });
  if (e != cudaSuccess) return cuda_fail(e, "prologue launch");
  // the text rows (and the zero padding up to kv_rows), which every rank computes for itself
  if (pl.Lk_pad > sp.L) {
    pp.skip_q = 1;
    pp.n_peers = 0;   // every GPU computes the text rows itself
    pp.zero_ptr = nullptr;
    pp.zero_count = 0;
    pp.out[1].ptr = KV + (int64_t)sp.L * sp.kv_ld;
    pp.out[2].ptr = KV + (int64_t)sp.L * sp.kv_ld + v_col;
    pp.rows[1] = pp.rows[2] = pl.Lk_pad - sp.L;
    pp.row0[1] = pp.row0[2] = sp.L;
    pp.src_row0[1] = pp.src_row0[2] = sp.text_row0;
    bytes = (double)pl.Bs * (pl.Lk - sp.L) * 2.0 * pl.Hkvs * pl.D * (in_elem + 2.0);
    e = profiled("prologue", 0.0, bytes, strm, [&] { return nsa::launch_prologue(pp, strm); });
    if (e != cudaSuccess) return cuda_fail(e, "prologue launch");
  }
  return NSA_OK;
}

namespace {

// 128-byte-swizzled bf16 map over `rank` dims (dims[0] contiguous) for the projection's operands.
bool encode_sw128(CUtensorMap* map, const void* base, int rank, const cuuint64_t* dims, const cuuint64_t* strides,
                  const cuuint32_t* box) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  const cuuint32_t estr[3] = {1, 1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, (cuuint32_t)rank, const_cast<void*>(base), dims, strides, box,
            estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// 2-D tiled map over a row-major matrix [rows][width] (row pitch `ld` elements of `esz` bytes), boxes
// of [box_rows][box_cols].
bool encode_2d(CUtensorMap* m, const void* base, CUtensorMapDataType dt, int esz, int64_t width, int64_t rows,
               int64_t ld, uint32_t box_rows, CUtensorMapSwizzle sw, uint32_t box_cols = 64) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  const cuuint64_t dims[2] = {(cuuint64_t)width, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)(ld * esz)};
  const cuuint32_t box[2] = {box_cols, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  return fn(m, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// CTA pairs for the bf16 linear: on unless NSA_LINEAR_PAIR=0 (read once).
bool linear_pairs_enabled() {
  static const unsigned on = env_flag("NSA_LINEAR_PAIR", 1);
  return on != 0;
}

// The LoRA factor T = A @ lora_a^T (bf16 [rows][R], row pitch R) with the linear kernel's store form:
// the first of the two GEMMs the reference runs per side path (app/gpu/ops.js:80).
cudaError_t run_lora_factor(const void* A, int64_t lda, int rows, int K, const void* lora_a, int R, void* T, int* err,
                            cudaStream_t strm) {
  CUtensorMap ta, la, tc;
  if (!encode_2d(&ta, A, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, K, rows, lda, 128, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !encode_2d(&la, lora_a, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, K, R, K, 256, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !encode_2d(&tc, T, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, R, rows, R, 32, CU_TENSOR_MAP_SWIZZLE_128B, 64))
    return cudaErrorInvalidValue;
  nsa::LinearParams pt{};
  pt.M = rows;
  pt.N = R;
  pt.k_steps = (K + 63) / 64;
  pt.m_tiles = (rows + 127) / 128;
  pt.n_tiles = (R + 255) / 256;
  pt.alpha = 1.f;
  pt.C16 = static_cast<__nv_bfloat16*>(T);
  pt.ldc = R;
  pt.err = err;
  pt.timeout_ns = wait_timeout_ns();
  return profiled("linear_lora_t", 2.0 * rows * (double)R * K, 0.0, strm,
                  [&] { return nsa::launch_linear(pt, ta, la, ta, la, tc, strm); });
}

// X map [elements][rows][K] (box [1][128][64]) and W map [N][K] (box [N tile][64]) of one GEMM.
bool proj_maps(CUtensorMap* tx, CUtensorMap* tw, const void* x, int64_t ld, int64_t bstride, int rows, int b_count,
               const void* w, int K, int N, int n_tile) {
  const cuuint64_t xd[3] = {(cuuint64_t)K, (cuuint64_t)rows, (cuuint64_t)b_count};
  const cuuint64_t xs[2] = {(cuuint64_t)ld * 2, (cuuint64_t)(bstride > 0 ? bstride : (int64_t)rows * ld) * 2};
  const cuuint32_t xb[3] = {64, 128, 1};
  const cuuint64_t wd[2] = {(cuuint64_t)K, (cuuint64_t)N};
  const cuuint64_t ws[1] = {(cuuint64_t)K * 2};
  const cuuint32_t wb[2] = {64, (cuuint32_t)n_tile};
  return encode_sw128(tx, x, 3, xd, xs, xb) && encode_sw128(tw, w, 2, wd, ws, wb);
}

}  // namespace

nsa_status nsa_seq_shard_projection(const nsa_fused_desc* d, const nsa_seq_shard* s, const nsa_proj_desc* proj,
                                    const float* q_norm_w, const float* k_norm_w, const float* cs,
                                    const int32_t* kv_len, void* q_prime, void* kv_packed, void* stream) {
  SeqPlan sp;
  nsa_status st = make_seq_plan(d, s, &sp);
  if (st != NSA_OK) return st;
  if (!proj) return fail(NSA_ERR_INVALID_ARGUMENT, "proj is NULL");
  if (d->in_dtype != NSA_BF16) return fail(NSA_ERR_UNSUPPORTED, "the projection takes bf16 inputs and weights");
  if (!q_norm_w || !k_norm_w) return fail(NSA_ERR_INVALID_ARGUMENT, "q/k norm weights are required");
  const int D = d->D;
  const int hpt = nsa::projection_heads_per_tile(D);
  if (!hpt) return fail(NSA_ERR_UNSUPPORTED, "the projection supports head dims 64, 96, 128 and 256");
  if (d->Hq % hpt || d->Hkv % hpt)
    return fail(NSA_ERR_UNSUPPORTED, "Hq and Hkv must be multiples of " + std::to_string(hpt) +
                                         " (the heads of one projection tile)");
  const Plan& pl = sp.pl;
  const int K = proj->K;
  auto a16 = [](const void* ptr) { return ptr == nullptr || (reinterpret_cast<uintptr_t>(ptr) & 15) == 0; };
  if (K < 1 || K % 8) return fail(NSA_ERR_INVALID_ARGUMENT, "K must be a positive multiple of 8");
  if (!proj->x || !proj->w_qkv || proj->x_rows < 1 || proj->ldx < K || proj->ldx % 8 || proj->x_bstride % 8 ||
      proj->x_bstride < 0 || (pl.Bs > 1 && proj->x_bstride == 0))
    return fail(NSA_ERR_INVALID_ARGUMENT, "x needs ldx >= K, ldx and x_bstride multiples of 8, and x_rows >= 1");
  if ((int64_t)sp.img_row0 + sp.q_count > proj->x_rows)
    return fail(NSA_ERR_INVALID_ARGUMENT, "the shard's image rows exceed x_rows");
  if (!a16(proj->x) || !a16(proj->w_qkv) || !a16(proj->b_qkv) || !a16(q_norm_w) || !a16(k_norm_w) || !a16(cs) ||
      !a16(q_prime) || !a16(kv_packed) || !q_prime || !kv_packed)
    return fail(NSA_ERR_INVALID_ARGUMENT, "pointers must be 16-byte aligned (q_prime and kv_packed non-NULL)");
  if (cs && d->sinOff % 4) return fail(NSA_ERR_INVALID_ARGUMENT, "sinOff must be a multiple of 4");
  const bool text = pl.Lk > sp.L;
  if (text && (!proj->x_text || !proj->w_kv || proj->text_rows < 1 || proj->ld_text < K || proj->ld_text % 8 ||
               proj->text_bstride % 8 || proj->text_bstride < 0 || (pl.Bs > 1 && proj->text_bstride == 0) ||
               !a16(proj->x_text) || !a16(proj->w_kv) || !a16(proj->b_kv)))
    return fail(NSA_ERR_INVALID_ARGUMENT,
                "text keys (Lk > Lq) need x_text and w_kv (16-byte aligned, ld_text >= K, multiples of 8)");
  if (text && (int64_t)sp.text_row0 + (pl.Lk - sp.L) > proj->text_rows)
    return fail(NSA_ERR_INVALID_ARGUMENT, "the text rows exceed text_rows");
  if ((proj->w_qkv_scale || proj->w_kv_scale) && D == 256)
    return fail(NSA_ERR_UNSUPPORTED, "ConvRot weight scales at head dims 64, 96 and 128 (the Gemma encoder's "
                                     "640-wide linears are never int8)");
  if (!a16(proj->w_qkv_scale) || !a16(proj->w_kv_scale))
    return fail(NSA_ERR_INVALID_ARGUMENT, "weight scales must be 16-byte aligned");
  const int Rq = proj->lora_rank_qkv, Rk = text ? proj->lora_rank_kv : 0;
  if (Rq < 0 || Rq % 64 || Rk < 0 || Rk % 64)
    return fail(NSA_ERR_INVALID_ARGUMENT, "LoRA ranks must be multiples of 64 (0: none)");
  if ((Rq && (!proj->lora_a_qkv || !proj->lora_b_qkv)) || (Rk && (!proj->lora_a_kv || !proj->lora_b_kv)) ||
      ((Rq || Rk) && !proj->lora_t) || !a16(proj->lora_a_qkv) || !a16(proj->lora_b_qkv) || !a16(proj->lora_a_kv) ||
      !a16(proj->lora_b_kv) || !a16(proj->lora_t))
    return fail(NSA_ERR_INVALID_ARGUMENT, "a LoRA needs 16-byte aligned lora_a, lora_b and the lora_t scratch");
  int* err = nsa::device_error_word();
  if (!err) return fail(NSA_ERR_CUDA, "cannot resolve the device error word on this device");
  const cudaStream_t strm = static_cast<cudaStream_t>(stream);
  auto* Q = static_cast<__nv_bfloat16*>(q_prime);
  auto* KV = static_cast<__nv_bfloat16*>(kv_packed);
  const SplitScratch split =
      split_scratch(static_cast<uint8_t*>(q_prime) + sp.q_tiles_bytes, pl.split_cap, pl.NQ, pl.D);

  nsa::ProjParams pp{};
  pp.B = pl.Bs;
  pp.b_begin = pl.b0;
  pp.k_steps = (K + 63) / 64;
  pp.Hq = d->Hq;
  pp.Hkv = d->Hkv;
  pp.Lk = pl.Lk;
  pp.Lq_pad = pl.Lq_pad;
  pp.Lk_pad = pl.Lk_pad;
  pp.kv_ld = sp.kv_ld;
  pp.q_w = q_norm_w;
  pp.k_w = k_norm_w;
  pp.cs = cs;
  pp.sin_off = d->sinOff;
  pp.eps = d->eps;
  pp.kv_len = kv_len;
  pp.q_prime = Q;
  pp.kv_packed = KV;
  pp.zero_ptr = pl.split_cap > 0 ? split.count : nullptr;   // the attention's split counters start at zero
  pp.zero_count = 2 * pl.split_cap;   // two counters (query tiles) per split unit
  pp.err = err;
  pp.timeout_ns = wait_timeout_ns();

  // LoRA factors T = x A^T per set and batch element, into lora_t ([b_count][x_rows][R_qkv], then
  // [b_count][text_rows][R_kv]), and the maps the kernel's extra K slices read
  CUtensorMap tt[2], tl[2];
  auto* T0 = static_cast<__nv_bfloat16*>(proj->lora_t);
  auto* T1 = T0 ? T0 + (int64_t)pl.Bs * proj->x_rows * Rq : nullptr;
  auto lora_maps = [&](int si, const void* x, int64_t ld, int64_t bstride, int rows, const void* a, const void* bcat,
                       int R, __nv_bfloat16* T, int N) -> nsa_status {
    for (int bl = 0; bl < pl.Bs; ++bl) {
      cudaError_t e = run_lora_factor(static_cast<const __nv_bfloat16*>(x) + (int64_t)(pl.b0 + bl) * bstride, ld, rows,
                                      K, a, R, T + (int64_t)bl * rows * R, err, strm);
      if (e != cudaSuccess) return cuda_fail(e, "LoRA factor launch");
    }
    const cuuint64_t td[3] = {(cuuint64_t)R, (cuuint64_t)rows, (cuuint64_t)pl.Bs};
    const cuuint64_t ts[2] = {(cuuint64_t)R * 2, (cuuint64_t)rows * R * 2};
    const cuuint32_t tb[3] = {64, 128, 1};
    const cuuint64_t ld2[2] = {(cuuint64_t)R, (cuuint64_t)N};
    const cuuint64_t ls[1] = {(cuuint64_t)R * 2};
    const cuuint32_t lb[2] = {64, (cuuint32_t)(hpt * D)};
    if (!encode_sw128(&tt[si], T, 3, td, ts, tb) || !encode_sw128(&tl[si], bcat, 2, ld2, ls, lb))
      return fail(NSA_ERR_CUDA, "cuTensorMapEncodeTiled failed for the LoRA operands");
    return NSA_OK;
  };
  if (Rq) {
    nsa_status ls = lora_maps(0, proj->x, proj->ldx, proj->x_bstride, proj->x_rows, proj->lora_a_qkv,
                              proj->lora_b_qkv, Rq, T0, (d->Hq + 2 * d->Hkv) * D);
    if (ls != NSA_OK) return ls;
  }
  if (Rk) {
    nsa_status ls = lora_maps(1, proj->x_text, proj->ld_text, proj->text_bstride, proj->text_rows, proj->lora_a_kv,
                              proj->lora_b_kv, Rk, T1, 2 * d->Hkv * D);
    if (ls != NSA_OK) return ls;
  }

  // set 0, the image rows: q|k|v of the shard's own rows, q' rows past them zero
  CUtensorMap tx[2], tw[2];
  const auto* x0 = static_cast<const __nv_bfloat16*>(proj->x) + (int64_t)pl.b0 * proj->x_bstride;
  if (!proj_maps(&tx[0], &tw[0], x0, proj->ldx, proj->x_bstride, proj->x_rows, pl.Bs, proj->w_qkv, K,
                 (d->Hq + 2 * d->Hkv) * D, hpt * D))
    return fail(NSA_ERR_CUDA, "cuTensorMapEncodeTiled failed for the projection operands");
  nsa::ProjSet& img = pp.set[0];
  img.image = 1;
  img.rows = pl.Lq_pad;
  img.m_tiles = pl.Lq_pad / 128;
  img.n_tiles = (d->Hq + 2 * d->Hkv) / hpt;
  img.valid_q = sp.q_count;
  img.key_row0 = sp.q_begin;
  img.x_row0 = sp.img_row0;
  img.rope_row0 = sp.q_begin;
  img.bias = proj->b_qkv;
  img.w_scale = proj->w_qkv_scale;
  img.lora_steps = Rq / 64;
  pp.n_sets = 1;
  double flops = 2.0 * pl.Bs * sp.q_count * (double)(d->Hq + 2 * d->Hkv) * D * (K + Rq);
  // set 1, the text rows (every rank computes them) and the zero padding up to kv_rows
  if (text) {
    const auto* t0 = static_cast<const __nv_bfloat16*>(proj->x_text) + (int64_t)pl.b0 * proj->text_bstride;
    if (!proj_maps(&tx[1], &tw[1], t0, proj->ld_text, proj->text_bstride, proj->text_rows, pl.Bs, proj->w_kv, K,
                   2 * d->Hkv * D, hpt * D))
      return fail(NSA_ERR_CUDA, "cuTensorMapEncodeTiled failed for the projection operands");
    nsa::ProjSet& txt = pp.set[1];
    txt.image = 0;
    txt.rows = pl.Lk_pad - sp.L;
    txt.m_tiles = (txt.rows + 127) / 128;
    txt.n_tiles = 2 * d->Hkv / hpt;
    txt.valid_q = 0;
    txt.key_row0 = sp.L;
    txt.x_row0 = sp.text_row0;
    txt.rope_row0 = 0;
    txt.bias = proj->b_kv;
    txt.w_scale = proj->w_kv_scale;
    txt.lora_steps = Rk / 64;
    pp.n_sets = 2;
    flops += 2.0 * pl.Bs * (pl.Lk - sp.L) * (double)(2 * d->Hkv) * D * (K + Rk);
  }
  // head dims 96 and 256: the RoPE table as a [2 * rows][D/2] fp32 map (cos block, then sin block),
  // boxes of [32 rows][16 values] with the 64-byte swizzle, for the epilogue's per-warp staging
  CUtensorMap tcs;
  const CUtensorMap* tcs_ptr = nullptr;
  if ((D == 256 || D == 96) && cs && d->sinOff > 0 && d->sinOff % (D / 2) == 0) {
    EncodeTiledFn fn = encode_fn();
    const cuuint64_t cd[2] = {(cuuint64_t)(D / 2), (cuuint64_t)(2 * (d->sinOff / (D / 2)))};
    const cuuint64_t cst[1] = {(cuuint64_t)(D / 2) * 4};
    const cuuint32_t cb[2] = {16, 32};
    const cuuint32_t ce[2] = {1, 1};
    if (fn && fn(&tcs, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(cs), cd, cst, cb, ce,
                 CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                 CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS) {
      tcs_ptr = &tcs;
      pp.cs_tma = 1;
      pp.cs_rows = (int)(d->sinOff / (D / 2));
    }
  }
  cudaError_t e = profiled("projection", flops, 0.0, strm,
                           [&] { return nsa::launch_projection(pp, D, tx, tw, tcs_ptr, tt, tl, strm); });
  if (e == cudaErrorNotSupported)
    return fail(NSA_ERR_UNSUPPORTED, "the projection's bias vectors do not fit in shared memory");
  if (e != cudaSuccess) return cuda_fail(e, "projection launch");
  if (!text && pl.Lk_pad > sp.L) {
    for (int bl = 0; bl < pl.Bs; ++bl) {
      e = cudaMemsetAsync(KV + ((int64_t)bl * pl.Lk_pad + sp.L) * sp.kv_ld, 0, (size_t)(pl.Lk_pad - sp.L) * sp.kv_ld * 2,
                          strm);
      if (e != cudaSuccess) return cuda_fail(e, "kv padding");
    }
  }
  return NSA_OK;
}

nsa_status nsa_linear(const nsa_linear_desc* d, const void* A, const void* W, const float* bias, const float* gate,
                      void* C, void* stream) {
  if (!d) return fail(NSA_ERR_INVALID_ARGUMENT, "desc is NULL");
  if (!A || !W || !C) return fail(NSA_ERR_INVALID_ARGUMENT, "A, W and C must be device pointers");
  if (d->M < 1 || d->N < 1 || d->K < 1) return fail(NSA_ERR_INVALID_ARGUMENT, "M, N and K must be >= 1");
  if (d->glu < 0 || d->glu > 2) return fail(NSA_ERR_INVALID_ARGUMENT, "glu is 0 (none), 1 (silu) or 2 (gelu_tanh)");
  const int64_t n_out = d->glu ? d->N / 2 : d->N;   // the fused GLU writes half the columns
  const int64_t ldc = d->ldc ? d->ldc : n_out;
  if (d->K % 8 || d->lda < d->K || d->lda % 8)
    return fail(NSA_ERR_INVALID_ARGUMENT, "K and lda must be multiples of 8 with lda >= K");
  if (d->glu && (d->N % 256 || d->resid || gate || d->act || d->lora_rank))
    return fail(NSA_ERR_INVALID_ARGUMENT, "the fused GLU needs N a multiple of 256 and no resid, gate, act or LoRA");
  if (d->N % 4 || ldc % 4 || d->cOff % 4 || d->gOff % 4 || d->cOff < 0 || d->gOff < 0 || ldc < d->cOff + n_out)
    return fail(NSA_ERR_INVALID_ARGUMENT, "N, ldc, cOff and gOff must be multiples of 4, with ldc >= cOff + N");
  if (d->out_dtype != NSA_F32 && d->out_dtype != NSA_BF16) return fail(NSA_ERR_INVALID_ARGUMENT, "bad out_dtype");
  if (d->w_format != NSA_W_BF16 && d->w_format != NSA_W_I8)
    return fail(NSA_ERR_INVALID_ARGUMENT, "w_format is NSA_W_BF16 or NSA_W_I8");
  const bool i8 = d->w_format == NSA_W_I8;
  auto a16 = [](const void* ptr) { return ptr == nullptr || (reinterpret_cast<uintptr_t>(ptr) & 15) == 0; };
  if (!a16(A) || !a16(W) || !a16(C) || !a16(bias) || !a16(gate) || !a16(d->w_scale) || !a16(d->lora_a) ||
      !a16(d->lora_b) || !a16(d->lora_t))
    return fail(NSA_ERR_INVALID_ARGUMENT, "pointers must be 16-byte aligned");
  if (gate && !d->resid) return fail(NSA_ERR_INVALID_ARGUMENT, "a gate needs resid (C += gate * r)");
  if (d->out_dtype == NSA_BF16 && d->resid)
    return fail(NSA_ERR_INVALID_ARGUMENT, "the bf16 output is the store form (no resid)");
  if (d->act != 0 && d->act != 1) return fail(NSA_ERR_INVALID_ARGUMENT, "act is 0 (none) or 1 (silu)");
  if (i8 && !d->w_scale) return fail(NSA_ERR_INVALID_ARGUMENT, "int8 weights need w_scale[N]");
  if (i8 && d->K % 16) return fail(NSA_ERR_INVALID_ARGUMENT, "int8 weights need K a multiple of 16");
  const int R = d->lora_rank;
  if (R < 0 || R % 64) return fail(NSA_ERR_INVALID_ARGUMENT, "lora_rank must be a multiple of 64 (0: no LoRA)");
  if (R && (!d->lora_a || !d->lora_b || !d->lora_t))
    return fail(NSA_ERR_INVALID_ARGUMENT, "a LoRA needs lora_a, lora_b and the lora_t scratch");
  if (d->out_dtype == NSA_BF16 && (ldc % 8 || d->cOff % 8))
    return fail(NSA_ERR_INVALID_ARGUMENT, "a bf16 C needs ldc and cOff multiples of 8 (16-byte rows)");
  if (d->schedule < NSA_LINEAR_AUTO || d->schedule > NSA_LINEAR_PAIR)
    return fail(NSA_ERR_INVALID_ARGUMENT, "schedule is NSA_LINEAR_AUTO, NSA_LINEAR_SINGLE or NSA_LINEAR_PAIR");
  if (d->schedule == NSA_LINEAR_PAIR && (i8 || d->M <= 128))
    return fail(NSA_ERR_INVALID_ARGUMENT, "CTA pairs need bf16 weights and M > 128");
  int* err = nsa::device_error_word();
  if (!err) return fail(NSA_ERR_CUDA, "cannot resolve the device error word on this device");
  const cudaStream_t strm = static_cast<cudaStream_t>(stream);
  const float alpha = d->alpha != 0.f ? d->alpha : 1.f;
  // A [M][K] bf16 and W [N][K] (bf16 swizzled for the MMA, or int8 plain rows for the converters)
  auto map2d = [](CUtensorMap* m, const void* base, CUtensorMapDataType dt, int esz, int64_t width, int64_t rows,
                  int64_t ld, uint32_t box_rows, CUtensorMapSwizzle sw, uint32_t box_cols = 64) {
    return encode_2d(m, base, dt, esz, width, rows, ld, box_rows, sw, box_cols);
  };
  const auto BF = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  const auto SW = CU_TENSOR_MAP_SWIZZLE_128B;
  auto base_params = [&](int M, int N, int K) {
    nsa::LinearParams p{};
    p.M = M;
    p.N = N;
    p.k_steps = (K + 63) / 64;
    p.m_tiles = (M + 127) / 128;
    p.n_tiles = (N + 255) / 256;
    p.alpha = 1.f;
    p.err = err;
    p.timeout_ns = wait_timeout_ns();
    return p;
  };
  CUtensorMap ta, tw, tt, tl, tc;
  if (R) {
    // T = A @ lora_a^T, bf16 [M][R]: the LoRA's first factor, one small GEMM before the main one
    cudaError_t e = run_lora_factor(A, d->lda, d->M, d->K, d->lora_a, R, d->lora_t, err, strm);
    if (e != cudaSuccess) return cuda_fail(e, "LoRA factor launch");
  }
  // CTA pairs (256 x 256 tiles, each CTA loading 128 of a tile's W rows, 128-wide K steps) lead only on
  // large GEMMs (16384 x 4096 x 4096: 1491 vs 1344 TFLOP/s); on the DiT and Gemma linears (K 640-2048,
  // 2-14 tiles per SM) single CTAs with their deeper 64-wide ring are level or ahead
  const bool pair = d->schedule == NSA_LINEAR_PAIR ||
                    (d->schedule == NSA_LINEAR_AUTO && !i8 && d->K + R >= 2048 &&
                     (int64_t)d->M * d->N >= (int64_t(1) << 26) && linear_pairs_enabled());
  const uint32_t wbox = pair ? 128 : 256;
  bool ok = map2d(&ta, A, BF, 2, d->K, d->M, d->lda, 128, SW) &&
            (i8 ? map2d(&tw, W, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, d->K, d->N, d->K, 256, CU_TENSOR_MAP_SWIZZLE_NONE)
                : map2d(&tw, W, BF, 2, d->K, d->N, d->K, wbox, SW));
  if (ok && R) ok = map2d(&tt, d->lora_t, BF, 2, R, d->M, R, 128, SW) && map2d(&tl, d->lora_b, BF, 2, R, d->N, R, wbox, SW);
  const bool c16 = d->out_dtype == NSA_BF16;
  if (ok)
    ok = c16 ? map2d(&tc, static_cast<__nv_bfloat16*>(C) + d->cOff, BF, 2, n_out, d->M, ldc, 32, SW, 64)
             : map2d(&tc, static_cast<float*>(C) + d->cOff, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, n_out, d->M, ldc, 32, SW, 32);
  if (!ok) return fail(NSA_ERR_CUDA, "cuTensorMapEncodeTiled failed for the linear operands");
  nsa::LinearParams p = base_params(d->M, d->N, d->K);
  p.lora_steps = R / 64;
  p.alpha = alpha;
  p.bias = bias;
  p.gate = gate ? gate + d->gOff : nullptr;
  p.resid = d->resid ? 1 : 0;
  p.act = d->act;
  p.w_i8 = i8 ? 1 : 0;
  p.w_scale = d->w_scale;
  p.glu = d->glu;
  p.pair = pair ? 1 : 0;
  if (d->out_dtype == NSA_BF16)
    p.C16 = static_cast<__nv_bfloat16*>(C) + d->cOff;
  else
    p.C = static_cast<float*>(C) + d->cOff;
  p.ldc = ldc;
  const double flops = 2.0 * d->M * (double)d->N * (d->K + R);
  cudaError_t e = profiled(i8 ? "linear_i8" : "linear", flops, 0.0, strm,
                           [&] { return nsa::launch_linear(p, ta, tw, R ? tt : ta, R ? tl : tw, tc, strm); });
  if (e != cudaSuccess) return cuda_fail(e, "linear launch");
  return NSA_OK;
}

nsa_status nsa_rotate(const nsa_rotate_desc* d, const void* X, void* Y, void* stream) {
  if (!d) return fail(NSA_ERR_INVALID_ARGUMENT, "desc is NULL");
  if (d->rows < 0 || d->cols < 256 || d->cols % 256)
    return fail(NSA_ERR_INVALID_ARGUMENT, "need rows >= 0 and cols a positive multiple of 256");
  const int64_t ldx = d->ldx ? d->ldx : d->cols, ldy = d->ldy ? d->ldy : d->cols;
  if (ldx < d->cols || ldy < d->cols || ldx % 8 || ldy % 8)
    return fail(NSA_ERR_INVALID_ARGUMENT, "ldx and ldy must be multiples of 8 and >= cols");
  if ((d->in_dtype != NSA_F32 && d->in_dtype != NSA_BF16) || (d->out_dtype != NSA_F32 && d->out_dtype != NSA_BF16))
    return fail(NSA_ERR_INVALID_ARGUMENT, "bad in_dtype / out_dtype");
  if (d->rows == 0) return NSA_OK;
  if (!X || !Y || !aligned16(X) || !aligned16(Y))
    return fail(NSA_ERR_INVALID_ARGUMENT, "X and Y must be 16-byte aligned device pointers");
  const int ei = d->in_dtype == NSA_F32 ? 4 : 2, eo = d->out_dtype == NSA_F32 ? 4 : 2;
  const uintptr_t x0 = reinterpret_cast<uintptr_t>(X), y0 = reinterpret_cast<uintptr_t>(Y);
  const uintptr_t x1 = x0 + (uintptr_t)(((int64_t)(d->rows - 1) * ldx + d->cols) * ei);
  const uintptr_t y1 = y0 + (uintptr_t)(((int64_t)(d->rows - 1) * ldy + d->cols) * eo);
  if (x0 < y1 && y0 < x1) return fail(NSA_ERR_INVALID_ARGUMENT, "X and Y must not overlap");
  nsa::RotateParams p{};
  p.rows = d->rows;
  p.cols = d->cols;
  p.ldx = ldx;
  p.ldy = ldy;
  p.x = X;
  p.y = Y;
  p.in_bf16 = d->in_dtype == NSA_BF16;
  p.out_bf16 = d->out_dtype == NSA_BF16;
  const cudaStream_t strm = static_cast<cudaStream_t>(stream);
  cudaError_t e = profiled("rotate", 0.0, (double)d->rows * d->cols * (ei + eo), strm,
                           [&] { return nsa::launch_rotate(p, strm); });
  if (e != cudaSuccess) return cuda_fail(e, "rotate launch");
  return NSA_OK;
}

nsa_status nsa_expand_i8(const int8_t* W, int64_t count, void* out_bf16, void* stream) {
  if (count < 0) return fail(NSA_ERR_INVALID_ARGUMENT, "count must be >= 0");
  if (count == 0) return NSA_OK;
  if (!W || !out_bf16 || !aligned16(out_bf16)) return fail(NSA_ERR_INVALID_ARGUMENT, "W and a 16-byte aligned out");
  cudaError_t e = nsa::launch_expand_i8(W, count, static_cast<__nv_bfloat16*>(out_bf16), static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "expand_i8 launch");
  return NSA_OK;
}

int32_t nsa_lora_rank(const nsa_lora_entry* entries, int32_t count) {
  if (!entries || count <= 0) return 0;
  int64_t r = 0;
  for (int i = 0; i < count; ++i) r += entries[i].r > 0 ? entries[i].r : 0;
  r = (r + 63) / 64 * 64;
  return r > 0x7FFFFFFF ? -1 : (int32_t)r;
}

nsa_status nsa_lora_pack(const nsa_lora_entry* entries, int32_t count, int32_t N, int32_t K, const float* w_scale,
                         float alpha, void* lora_a, void* lora_b, void* stream) {
  if (count < 0 || (count > 0 && !entries)) return fail(NSA_ERR_INVALID_ARGUMENT, "entries is NULL");
  if (N < 1 || K < 1) return fail(NSA_ERR_INVALID_ARGUMENT, "N and K must be >= 1");
  if (!(alpha != 0.f)) alpha = 1.f;
  std::vector<nsa::LoraPackEntry> pe;
  for (int i = 0; i < count; ++i) {
    const nsa_lora_entry& e = entries[i];
    if (e.r < 1 || e.n < 1 || e.off < 0 || (int64_t)e.off + e.n > N || !e.A || !e.B)
      return fail(NSA_ERR_INVALID_ARGUMENT, "LoRA entry " + std::to_string(i) +
                                                ": need r >= 1, 0 <= off, off + n <= N and device A, B");
    pe.push_back({e.A, e.B, e.r, e.off, e.n, e.scale});
  }
  const int32_t R = nsa_lora_rank(entries, count);
  if (R <= 0) return count == 0 ? NSA_OK : fail(NSA_ERR_INVALID_ARGUMENT, "LoRA ranks overflow");
  if (!lora_a || !lora_b) return fail(NSA_ERR_INVALID_ARGUMENT, "lora_a and lora_b must be device pointers");
  const cudaStream_t strm = static_cast<cudaStream_t>(stream);
  cudaError_t e = nsa::launch_lora_pack(pe.data(), count, N, K, R, w_scale, alpha,
                                        static_cast<__nv_bfloat16*>(lora_a), static_cast<__nv_bfloat16*>(lora_b), strm);
  if (e != cudaSuccess) return cuda_fail(e, "LoRA pack");
  return NSA_OK;
}

nsa_status nsa_rmsnorm(const nsa_rmsnorm_desc* d, const float* X, const float* weight, void* Y, void* stream) {
  if (!d) return fail(NSA_ERR_INVALID_ARGUMENT, "desc is NULL");
  if (d->rows < 0 || d->cols < 1) return fail(NSA_ERR_INVALID_ARGUMENT, "need rows >= 0 and cols >= 1");
  const int64_t ldx = d->ldx ? d->ldx : d->cols, ldy = d->ldy ? d->ldy : d->cols;
  if (ldx < d->cols || ldy < d->cols) return fail(NSA_ERR_INVALID_ARGUMENT, "ldx and ldy must be >= cols");
  if (d->out_dtype != NSA_F32 && d->out_dtype != NSA_BF16) return fail(NSA_ERR_INVALID_ARGUMENT, "bad out_dtype");
  if (d->accumulate && d->out_dtype != NSA_F32) return fail(NSA_ERR_INVALID_ARGUMENT, "accumulate needs an fp32 Y");
  if (!(d->eps >= 0.f)) return fail(NSA_ERR_INVALID_ARGUMENT, "eps must be >= 0");
  if (d->rows == 0) return NSA_OK;   // nothing to normalise (empty tensors may carry NULL pointers)
  if (!X || !weight || !Y) return fail(NSA_ERR_INVALID_ARGUMENT, "X, weight and Y must be device pointers");
  const int esz = d->out_dtype == NSA_F32 ? 4 : 2;
  // X and Y must not overlap (a row's values are read before and while its outputs are written)
  const uintptr_t x0 = reinterpret_cast<uintptr_t>(X), y0 = reinterpret_cast<uintptr_t>(Y);
  const uintptr_t x1 = x0 + (uintptr_t)(((int64_t)(d->rows - 1) * ldx + d->cols) * 4);
  const uintptr_t y1 = y0 + (uintptr_t)(((int64_t)(d->rows - 1) * ldy + d->cols) * esz);
  if (x0 < y1 && y0 < x1) return fail(NSA_ERR_INVALID_ARGUMENT, "X and Y must not overlap");
  nsa::RmsParams p{};
  p.rows = d->rows;
  p.cols = d->cols;
  p.ldx = ldx;
  p.ldy = ldy;
  p.x = X;
  p.w = weight;
  p.y = Y;
  p.out_bf16 = d->out_dtype == NSA_BF16;
  p.accumulate = d->accumulate ? 1 : 0;
  p.eps = d->eps;
  p.vec = d->cols % 4 == 0 && ldx % 4 == 0 && ldy % 4 == 0 && (x0 & 15) == 0 &&
          (reinterpret_cast<uintptr_t>(weight) & 15) == 0 && (y0 & (uintptr_t)(4 * esz - 1)) == 0;
  double bytes = (double)d->rows * d->cols * (4.0 + esz * (d->accumulate ? 2.0 : 1.0));
  if (d->next_weight) {
    // the chained next norm: Z = rmsnorm(Y after the add) * next_weight
    if (!d->accumulate) return fail(NSA_ERR_INVALID_ARGUMENT, "next_weight needs accumulate = 1");
    if (!d->Z) return fail(NSA_ERR_INVALID_ARGUMENT, "next_weight needs Z");
    if (d->z_dtype != NSA_F32 && d->z_dtype != NSA_BF16) return fail(NSA_ERR_INVALID_ARGUMENT, "bad z_dtype");
    const int64_t ldz = d->ldz ? d->ldz : d->cols;
    const int zsz = d->z_dtype == NSA_F32 ? 4 : 2;
    const uintptr_t z0 = reinterpret_cast<uintptr_t>(d->Z);
    if (ldz < d->cols || ldz % 4 || !p.vec || (z0 & (uintptr_t)(4 * zsz - 1)) ||
        (reinterpret_cast<uintptr_t>(d->next_weight) & 15))
      return fail(NSA_ERR_INVALID_ARGUMENT,
                  "the chained norm needs cols, ldx, ldy, ldz multiples of 4 and 16-byte aligned X, Y, weights and Z rows");
    const uintptr_t z1 = z0 + (uintptr_t)(((int64_t)(d->rows - 1) * ldz + d->cols) * zsz);
    if ((z0 < y1 && y0 < z1) || (z0 < x1 && x0 < z1)) return fail(NSA_ERR_INVALID_ARGUMENT, "Z must not overlap X or Y");
    p.w2 = d->next_weight;
    p.z = d->Z;
    p.ldz = ldz;
    p.z_bf16 = d->z_dtype == NSA_BF16 ? 1 : 0;
    bytes += (double)d->rows * d->cols * zsz;
  }
  const cudaStream_t strm = static_cast<cudaStream_t>(stream);
  cudaError_t e = profiled("rmsnorm", 0.0, bytes, strm, [&] { return nsa::launch_rmsnorm(p, strm); });
  if (e != cudaSuccess) return cuda_fail(e, "rmsnorm launch");
  return NSA_OK;
}

nsa_status nsa_glu_interleave(const void* src, void* dst, int32_t I, int64_t row_bytes, void* stream) {
  if (!src || !dst) return fail(NSA_ERR_INVALID_ARGUMENT, "src and dst must be device pointers");
  if (I < 128 || I % 128) return fail(NSA_ERR_INVALID_ARGUMENT, "I must be a positive multiple of 128");
  if (row_bytes < 4 || row_bytes % 4) return fail(NSA_ERR_INVALID_ARGUMENT, "row_bytes must be a positive multiple of 4");
  if ((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(dst)) & 3)
    return fail(NSA_ERR_INVALID_ARGUMENT, "src and dst must be 4-byte aligned");
  const uintptr_t bytes = (uintptr_t)(2 * (int64_t)I * row_bytes);
  const uintptr_t s0 = reinterpret_cast<uintptr_t>(src), d0 = reinterpret_cast<uintptr_t>(dst);
  if (s0 < d0 + bytes && d0 < s0 + bytes) return fail(NSA_ERR_INVALID_ARGUMENT, "src and dst must not overlap");
  const cudaStream_t strm = static_cast<cudaStream_t>(stream);
  cudaError_t e = nsa::launch_glu_interleave(src, dst, I, row_bytes, strm);
  if (e != cudaSuccess) return cuda_fail(e, "glu interleave launch");
  return NSA_OK;
}

nsa_status nsa_glu(const nsa_glu_desc* d, const float* X, void* Y, void* stream) {
  if (!d) return fail(NSA_ERR_INVALID_ARGUMENT, "desc is NULL");
  if (d->rows < 0 || d->I < 1) return fail(NSA_ERR_INVALID_ARGUMENT, "need rows >= 0 and I >= 1");
  const int64_t ldx = d->ldx ? d->ldx : 2 * (int64_t)d->I, ldy = d->ldy ? d->ldy : d->I;
  if (ldx < 2 * (int64_t)d->I || ldy < d->I) return fail(NSA_ERR_INVALID_ARGUMENT, "need ldx >= 2*I and ldy >= I");
  if (d->act != 0 && d->act != 1) return fail(NSA_ERR_INVALID_ARGUMENT, "act is 0 (silu) or 1 (gelu_tanh)");
  if (d->out_dtype != NSA_F32 && d->out_dtype != NSA_BF16) return fail(NSA_ERR_INVALID_ARGUMENT, "bad out_dtype");
  if (d->rows == 0) return NSA_OK;
  if (!X || !Y) return fail(NSA_ERR_INVALID_ARGUMENT, "X and Y must be device pointers");
  const int esz = d->out_dtype == NSA_F32 ? 4 : 2;
  const uintptr_t x0 = reinterpret_cast<uintptr_t>(X), y0 = reinterpret_cast<uintptr_t>(Y);
  const uintptr_t x1 = x0 + (uintptr_t)(((int64_t)(d->rows - 1) * ldx + 2 * (int64_t)d->I) * 4);
  const uintptr_t y1 = y0 + (uintptr_t)(((int64_t)(d->rows - 1) * ldy + d->I) * esz);
  if (x0 < y1 && y0 < x1) return fail(NSA_ERR_INVALID_ARGUMENT, "X and Y must not overlap");
  nsa::GluParams p{};
  p.rows = d->rows;
  p.I = d->I;
  p.ldx = ldx;
  p.ldy = ldy;
  p.x = X;
  p.y = Y;
  p.out_bf16 = d->out_dtype == NSA_BF16;
  p.act = d->act;
  p.vec = d->I % 4 == 0 && ldx % 4 == 0 && ldy % 4 == 0 && (x0 & 15) == 0 && (y0 & (uintptr_t)(4 * esz - 1)) == 0;
  const double bytes = (double)d->rows * d->I * (8.0 + esz);
  const cudaStream_t strm = static_cast<cudaStream_t>(stream);
  cudaError_t e = profiled("glu", 0.0, bytes, strm, [&] { return nsa::launch_glu(p, strm); });
  if (e != cudaSuccess) return cuda_fail(e, "glu launch");
  return NSA_OK;
}

nsa_status nsa_seq_shard_attention(const nsa_fused_desc* d, const nsa_seq_shard* s, const void* q_prime,
                                   const void* kv_packed, const int32_t* kv_len, const float* bias, void* out,
                                   void* stream) {
  SeqPlan sp;
  nsa_status st = make_seq_plan(d, s, &sp);
  if (st != NSA_OK) return st;
  if (!q_prime || !kv_packed || !aligned16(q_prime) || !aligned16(kv_packed))
    return fail(NSA_ERR_INVALID_ARGUMENT, "q_prime and kv_packed must be 16-byte aligned device pointers");
  if ((st = check_out(out, d->out_dtype, d->ldo, d->oOff, d->o_bstride)) != NSA_OK) return st;
  if (d->biasLen < 0) return fail(NSA_ERR_INVALID_ARGUMENT, "biasLen must be >= 0");
  if (d->biasLen > 0 && !bias) return fail(NSA_ERR_INVALID_ARGUMENT, "biasLen > 0 needs a bias pointer");
  int* err = nsa::device_error_word();
  if (!err) return fail(NSA_ERR_CUDA, "cannot resolve the device error word on this device");
  const Plan& pl = sp.pl;
  CUtensorMap tq, tkv;
  if (!encode_tiles(&tq, const_cast<void*>(q_prime), pl.D, (int64_t)pl.Bs * pl.Hqs * pl.Lq_pad, pl.blk, nsa::kTileM) ||
      !encode_rows(&tkv, kv_packed, sp.kv_ld, sp.kv_ld, (int64_t)pl.Bs * pl.Lk_pad, pl.blk, pl.BN))
    return fail(NSA_ERR_CUDA, "cuTensorMapEncodeTiled failed (driver entry point unavailable?)");
  nsa::AttnParams ap = attn_params(pl, sp.a, bias, d->biasStart, bias ? d->biasLen : 0, d->bias_bstride, kv_len,
                                   d->scale, out, d->ldo, d->o_bstride, d->oOff, err);
  // k' head h at columns [h*D, h*D + D) of the packed rows, v' head h at [(Hkv + h)*D, ...)
  ap.k_x0 = 0;
  ap.v_x0 = pl.Hkvs * pl.D;
  ap.kv_xh = pl.D;
  ap.kv_yb = pl.Lk_pad;
  ap.kv_yh = 0;
  ap.q_x0 = 0;
  ap.q_xh = 0;
  ap.q_yb = pl.Hqs * pl.Lq_pad;
  ap.q_yh = pl.Lq_pad;
  ap.q_b0 = pl.b0;
  ap.q_h0 = 0;
  set_split(&ap, pl, sp.a,
            split_scratch(static_cast<uint8_t*>(const_cast<void*>(q_prime)) + sp.q_tiles_bytes, pl.split_cap, pl.NQ,
                          pl.D));
  const cudaStream_t strm = static_cast<cudaStream_t>(stream);
  cudaError_t e = profiled("attention", attn_flops(pl, sp.a), 0.0, strm,
                           [&] { return nsa::launch_attention(ap, pl.D, tq, tkv, tkv, tkv, strm); },
                           attn_pairs(pl, sp.a), kv_len ? kv_len + pl.b0 : nullptr);
  if (e != cudaSuccess) return cuda_fail(e, "attention launch");
  return NSA_OK;
}

}  // extern "C"
