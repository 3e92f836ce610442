// nsa_fused_attention_noalloc: the fused DiT / Gemma attention step for callers that cannot
// allocate device memory.
//
// Some hosts of this library cannot hand it a workspace: an embedding runtime whose allocator is
// closed to plugins, a caller that must not call cudaMalloc while the GPU is shared with a latency-
// critical process (a device allocation can synchronise the device), or a binding layer that only
// passes the tensors it already owns.  nsa_fused_attention needs caller-provided scratch for the
// head-major bf16 Q/K/V tiles its prologue writes; this entry point instead uses a fixed scratch
// array compiled into the library, so the caller passes only inputs and outputs and nothing on this
// path calls cudaMalloc, cudaFree or any allocating routine.
//
// The array is kNoAllocScratchBytes (64 MiB) of device memory.  Every GPU that loads this part of
// the library holds it until the process exits.  It is reserved when the module is loaded on a
// device: with CUDA's default lazy loading that is this entry point's first call on that device (a
// device allocation the driver makes, which can synchronise the device), with
// CUDA_MODULE_LOADING=EAGER it is when the library is loaded.  A caller that must avoid that
// allocation on its hot path makes one call at start-up, before any stream capture.  All calls on a device share it, and it keeps what
// the previous call left: the prologue rewrites every byte the attention kernel later reads (zero
// rows included), so nothing has to be cleared between calls.  Two calls whose work overlaps on the
// GPU (different streams, or different host threads on the same device) race on the array; callers
// must order them, e.g. by issuing them on one stream.
#include <string>

#include "nsa_internal.h"
#include "nsattn.h"

namespace {

constexpr size_t kNoAllocScratchBytes = NSA_NOALLOC_SCRATCH_BYTES;

// The scratch lives here, in this file.  In host code `g_noalloc_scratch` is only a host-side stand-in
// for the device array, not a device address: the address a kernel may use is looked up per device
// with cudaGetSymbolAddress below.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

// Device address of the array on the current device, looked up with that device current.  It is
// resolved at every call instead of cached: after a cudaDeviceReset, or anything else that unloads
// and reloads the module, a cached address would point at freed memory, and the lookup is cheap.
// The first lookup on a device loads this file's module there (CUDA loads modules lazily by
// default), which is when the array is reserved.
void* scratch_address(nsa_status* st) {
  void* p = nullptr;
  const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
  if (e != cudaSuccess || p == nullptr) {
    *st = NSA_ERR_CUDA;
    return nullptr;
  }
  *st = NSA_OK;
  return p;
}

}  // namespace

extern "C" nsa_status nsa_fused_attention_noalloc(const nsa_fused_desc* desc, const void* qkv, const float* q_norm_w,
                                                  const float* k_norm_w, const float* cs, const int32_t* kv_len,
                                                  const float* bias, void* out, void* stream) {
  if (!desc) {
    nsa::record_error("nsa_fused_attention_noalloc: desc is NULL");
    return NSA_ERR_INVALID_ARGUMENT;
  }
  const size_t need = nsa_fused_attention_workspace_size(desc);
  if (need == 0) {
    // invalid or unsupported shape: let the regular entry point report the reason
    return nsa_fused_attention(desc, qkv, q_norm_w, k_norm_w, cs, kv_len, bias, out, nullptr, 0, stream);
  }
  if (need > kNoAllocScratchBytes) {
    nsa::record_error("nsa_fused_attention_noalloc: this shape needs " + std::to_string(need) +
                      " bytes of scratch, above the built-in " + std::to_string(kNoAllocScratchBytes) +
                      " bytes; split the batch or use nsa_fused_attention with a workspace");
    return NSA_ERR_WORKSPACE;
  }
  nsa_status st;
  void* scratch = scratch_address(&st);
  if (!scratch) {
    nsa::record_error("nsa_fused_attention_noalloc: cannot look up the scratch array on this device");
    return st;
  }
  return nsa_fused_attention(desc, qkv, q_norm_w, k_norm_w, cs, kv_len, bias, out, scratch, kNoAllocScratchBytes,
                             stream);
}
