// fg_paged_decode_attn_noalloc: paged decode attention that allocates nothing
// and takes no workspace from the caller.
//
// Who needs it. fg_paged_decode_attn splits long contexts over several CTAs
// and parks their fp32 partial results in caller-provided scratch. Some
// callers cannot provide it: a host runtime that owns every byte of device
// memory through its own pool and refuses cudaMalloc once it is serving, or
// a thin FFI binding (cgo, JNI, a C plugin) that has no device allocator at
// hand. cudaMalloc / cudaFree may also synchronise the device, which such a
// decode loop must not do. For them this entry point keeps the scratch in a
// file-scope device array of kNoAllocScratchBytes (8 MiB): every GPU that
// loads the library holds that much until the process exits.
//
// Contract.
//  - The first call on a device resolves the array's device address
//    (cudaGetSymbolAddress, with that device current) and caches it with
//    the CUDA context it belongs to; make that first call before any stream
//    capture. A call under a different context (after cudaDeviceReset, or a
//    driver-API context of its own) resolves the address again.
//  - Calls whose split partials would not fit in 8 MiB (see
//    fg_attn_workspace_bytes) are rejected with FG_ERR_ARG before any work.
//  - All calls on a device share the one array and it keeps the previous
//    call's contents. Nothing in it needs to start at zero: every split
//    slot a call reads is written by that same call first. Calls that
//    overlap on the GPU (different streams, no ordering) race on it.
//  - Results are those of fg_paged_decode_attn with the same arguments.
#pragma once
#include <cudaTypedefs.h>

#include <mutex>

#include "attention.cuh"

namespace fg {
namespace attn {

constexpr size_t kNoAllocScratchBytes = size_t(8) << 20;
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

constexpr int kNoAllocMaxDevices = 64;
static void* g_noalloc_addr[kNoAllocMaxDevices] = {nullptr};
static CUcontext g_noalloc_ctx[kNoAllocMaxDevices] = {nullptr};
static std::mutex g_noalloc_mu;

// The calling thread's current CUDA context (driver entry point, no -lcuda).
static int current_context(CUcontext* ctx) {
  static PFN_cuCtxGetCurrent_v4000 get = nullptr;
  if (!get) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &fn, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess) {
      set_last_error("fg_paged_decode_attn_noalloc: cuCtxGetCurrent unavailable");
      return FG_ERR_CUDA;
    }
    get = reinterpret_cast<PFN_cuCtxGetCurrent_v4000>(fn);
  }
  if (get(ctx) != CUDA_SUCCESS) {
    set_last_error("fg_paged_decode_attn_noalloc: cuCtxGetCurrent failed");
    return FG_ERR_CUDA;
  }
  return FG_OK;
}

// Device address of g_noalloc_scratch on the current device. The host-side
// symbol is only a stand-in for the device array and must never be handed to
// a kernel; the address comes from cudaGetSymbolAddress, cached per device
// together with the context it was resolved in.
static int noalloc_scratch(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    set_last_error("fg_paged_decode_attn_noalloc: cudaGetDevice: %s", cudaGetErrorString(e));
    return FG_ERR_CUDA;
  }
  if (dev < 0 || dev >= kNoAllocMaxDevices) {
    set_last_error("fg_paged_decode_attn_noalloc: device ordinal %d is beyond the %d this entry point "
                   "keeps addresses for", dev, kNoAllocMaxDevices);
    return FG_ERR_ARG;
  }
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  CUcontext ctx = nullptr;
  if (g_noalloc_addr[dev] != nullptr) {
    const int rc = current_context(&ctx);
    if (rc) return rc;
  }
  if (g_noalloc_addr[dev] == nullptr || ctx != g_noalloc_ctx[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr) {
      set_last_error("fg_paged_decode_attn_noalloc: cudaGetSymbolAddress: %s",
                     cudaGetErrorString(e));
      return FG_ERR_CUDA;
    }
    const int rc = current_context(&ctx);  // the runtime made the device's context current
    if (rc) return rc;
    g_noalloc_addr[dev] = p;
    g_noalloc_ctx[dev] = ctx;
  }
  *out = g_noalloc_addr[dev];
  return FG_OK;
}

}  // namespace attn
}  // namespace fg

extern "C" {

int fg_paged_decode_attn_noalloc(const fg_bf16* q, const fg_bf16* k_cache, const fg_bf16* v_cache,
                                 const int32_t* block_table, const int32_t* seq_lens,
                                 const float* sinks, fg_bf16* out, int B, int nq, int nkv, int hd,
                                 int block_size, int num_blocks, int max_blocks, int max_seq_len,
                                 int window, float scale, fg_stream_t stream) {
  const size_t need = fg_attn_workspace_bytes(B, nq, nkv, hd, max_seq_len, window);
  FG_REQUIRE(need <= fg::attn::kNoAllocScratchBytes,
             "fg_paged_decode_attn_noalloc: %d sequences x %d heads up to %d tokens need %zu bytes "
             "of split scratch, above the built-in %zu; call fg_paged_decode_attn with a workspace",
             B, nq, max_seq_len, need, fg::attn::kNoAllocScratchBytes);
  void* scratch = nullptr;
  if (need > 0) {
    const int rc = fg::attn::noalloc_scratch(&scratch);
    if (rc) return rc;
  }
  return fg_paged_decode_attn(q, k_cache, v_cache, block_table, seq_lens, sinks, out, scratch,
                              need > 0 ? fg::attn::kNoAllocScratchBytes : 0, B, nq, nkv, hd,
                              block_size, num_blocks, max_blocks, max_seq_len, window, scale,
                              stream);
}

}  // extern "C"
