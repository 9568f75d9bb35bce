// Shared device/host helpers for the fgb200 kernels (sm_100a only).
//
// Everything that waits on the device waits with a bound: mbarrier waits and
// flag spins give up after a %globaltimer deadline, record a status word in
// g_fg_device_status and let the kernel leave through its normal exit path.
// No error path traps, asserts or exits the grid.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/fgb200.h"

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "fgb200 kernels are written for sm_100a only"
#endif

namespace fg {

// ---------------------------------------------------------------------------
// device status word (per device, per loaded library)
// ---------------------------------------------------------------------------
// Bit layout: low 8 bits = DeviceCode of the first failure, bits 8..31 =
// the site that failed. Reset and read by fg_device_status(). The library is
// built as one translation unit (fgb200.cu includes every component), so the
// word is defined here once.
__device__ unsigned int g_fg_device_status = 0;

enum DeviceCode : unsigned int {
  DEV_OK = 0,
  DEV_MBAR_TIMEOUT = 1,    // an mbarrier wait ran past its deadline
  DEV_FLAG_TIMEOUT = 2,    // a peer flag wait ran past its deadline
  DEV_BAD_INDEX = 3,       // a block-table / slot / token index was out of range
  DEV_SCALE_RANGE = 4,     // an MXFP4 block scale lies outside its row's exact window
};

__device__ __forceinline__ void record_device_error(unsigned int code, unsigned int site) {
  atomicCAS(&g_fg_device_status, 0u, (site << 8) | (code & 0xffu));
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

// Wait bound for intra-CTA pipeline barriers. A healthy wait completes in
// microseconds; the bound only guards against a programming error.
constexpr uint64_t kMbarTimeoutNs = 2000000000ull;  // 2 s

// ---------------------------------------------------------------------------
// flags written by another GPU (system scope)
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// spin (bounded) until *p reaches seq (wrap-safe); false on timeout, after
// recording a peer flag timeout at `site` in the device status word
__device__ __forceinline__ bool wait_at_least(const uint32_t* p, uint32_t seq, uint64_t timeout_ns,
                                              unsigned int site) {
  if ((int32_t)(ld_acquire_sys(p) - seq) >= 0) return true;
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t it = 1;; ++it) {
    if ((int32_t)(ld_acquire_sys(p) - seq) >= 0) return true;
    if ((it & 63u) == 0) {
      if (globaltimer_ns() - t0 > timeout_ns) {
        record_device_error(DEV_FLAG_TIMEOUT, site);
        return false;
      }
      __nanosleep(256);
    }
  }
}

// ---------------------------------------------------------------------------
// bf16 helpers
// ---------------------------------------------------------------------------
__device__ __forceinline__ float bf2f(__nv_bfloat16 v) { return __bfloat162float(v); }
__device__ __forceinline__ __nv_bfloat16 f2bf(float v) { return __float2bfloat16_rn(v); }
// round-trip through bf16: the value a bf16 tensor op would have produced
__device__ __forceinline__ float rbf(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}
__device__ __forceinline__ float2 unpack_bf16x2(uint32_t v) {
  __nv_bfloat162 b = *reinterpret_cast<__nv_bfloat162*>(&v);
  return __bfloat1622float2(b);
}

// ---------------------------------------------------------------------------
// shared-memory address helpers
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------------------
// mbarrier (all waits bounded)
// ---------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
// Returns false (and records the site) when the deadline passes.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, unsigned int site) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t it = 1;; ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((it & 255u) == 0 && globaltimer_ns() - t0 > kMbarTimeoutNs) {
      record_device_error(DEV_MBAR_TIMEOUT, site);
      return false;
    }
  }
}

// ---------------------------------------------------------------------------
// TMA (tensor copies, plain: one CTA, own shared memory)
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tma_load_2d_hint(uint32_t dst, const CUtensorMap* map, uint32_t bar,
                                                 int32_t x, int32_t y, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%3, %4}], [%2], %5;" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(x), "r"(y), "l"(policy)
      : "memory");
}
__device__ __forceinline__ void prefetch_tensormap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}
__device__ __forceinline__ uint64_t l2_policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ uint64_t l2_policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// ---------------------------------------------------------------------------
// bulk (non-tensor) copy global -> own shared memory, completion on an mbarrier
// ---------------------------------------------------------------------------
__device__ __forceinline__ void bulk_load(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar,
                                          uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1], %2, [%3], %4;" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(bar), "l"(policy)
      : "memory");
}

// ---------------------------------------------------------------------------
// programmatic dependent launch: a kernel launched with programmatic stream
// serialisation may start while its predecessor drains; everything that
// reads the predecessor's results (or writes what it reads) must come after
// griddep_wait(). Both are no-ops for a normal launch.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ---------------------------------------------------------------------------
// warp helpers
// ---------------------------------------------------------------------------
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

}  // namespace fg

// ---------------------------------------------------------------------------
// host-side helpers shared by the .cu files
// ---------------------------------------------------------------------------
namespace fg {
void set_last_error(const char* fmt, ...);
int check_launch(const char* what);
// cuTensorMapEncodeTiled through the runtime's driver entry point (no -lcuda)
int make_tmap_2d_bf16(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer,
                      uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer,
                      CUtensorMapSwizzle swizzle);
int num_sms();
bool pdl_enabled();

// Launch with programmatic stream serialisation (PDL) unless disabled by
// FGB200_PDL=0; the kernel must call griddep_wait() before dependent work.
template <typename... KArgs, typename... Args>
int launch_k(const char* what, void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem,
             cudaStream_t st, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
  if (e != cudaSuccess) {
    set_last_error("%s: launch failed: %s", what, cudaGetErrorString(e));
    (void)cudaGetLastError();
    return FG_ERR_CUDA;
  }
  return check_launch(what);
}
// Launch as a thread-block cluster of `cluster` CTAs (plus PDL as launch_k).
template <typename... KArgs, typename... Args>
int launch_kc(const char* what, void (*kern)(KArgs...), dim3 grid, dim3 cluster, dim3 block,
              size_t smem, cudaStream_t st, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  int na = 0;
  if (cluster.x * cluster.y * cluster.z > 1) {
    attr[na].id = cudaLaunchAttributeClusterDimension;
    attr[na].val.clusterDim.x = cluster.x;
    attr[na].val.clusterDim.y = cluster.y;
    attr[na].val.clusterDim.z = cluster.z;
    ++na;
  }
  if (pdl_enabled()) {
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
  if (e != cudaSuccess) {
    set_last_error("%s: launch failed: %s", what, cudaGetErrorString(e));
    (void)cudaGetLastError();
    return FG_ERR_CUDA;
  }
  return check_launch(what);
}
}  // namespace fg

#define FG_REQUIRE(cond, ...)              \
  do {                                     \
    if (!(cond)) {                         \
      fg::set_last_error(__VA_ARGS__);     \
      return FG_ERR_ARG;                   \
    }                                      \
  } while (0)
