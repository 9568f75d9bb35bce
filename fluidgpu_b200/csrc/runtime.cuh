// Host-side plumbing shared by every entry point: error text, the device
// status word, tensor-map encoding and SM count.
#include <cudaTypedefs.h>

#include <atomic>
#include <cstdarg>
#include <cstdlib>
#include <cstdio>
#include <mutex>

#pragma once
#include "common.cuh"

namespace fg {

static thread_local char t_last_error[512] = "";

void set_last_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(t_last_error, sizeof(t_last_error), fmt, ap);
  va_end(ap);
}

static std::atomic<unsigned long long> g_launches{0};

int check_launch(const char* what) {
  g_launches.fetch_add(1, std::memory_order_relaxed);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_last_error("%s: %s", what, cudaGetErrorString(e));
    return FG_ERR_CUDA;
  }
  return FG_OK;
}

static PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
static std::once_flag g_encode_once;

static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  std::call_once(g_encode_once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess) {
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    }
  });
  return g_encode;
}

int make_tmap_2d_bf16(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer,
                      uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer,
                      CUtensorMapSwizzle swizzle) {
  auto fn = encode_fn();
  if (!fn) {
    set_last_error("cuTensorMapEncodeTiled unavailable from the driver");
    return FG_ERR_CUDA;
  }
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0 || (row_stride_bytes & 15) != 0) {
    set_last_error("tensor map: base %p / row stride %llu not 16-byte aligned", base,
                   (unsigned long long)row_stride_bytes);
    return FG_ERR_ARG;
  }
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_stride_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides,
                  box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_last_error("cuTensorMapEncodeTiled failed (%d): dims %llu x %llu box %u x %u", (int)r,
                   (unsigned long long)inner, (unsigned long long)outer, box_inner, box_outer);
    return FG_ERR_CUDA;
  }
  return FG_OK;
}

bool pdl_enabled() {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("FGB200_PDL");
    v = (e && e[0] == '0') ? 0 : 1;
  }
  return v == 1;
}

int num_sms() {
  static int cached[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) dev = 0;
  if (!cached[dev]) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    cached[dev] = n > 0 ? n : 148;
  }
  return cached[dev];
}

}  // namespace fg

extern "C" {

const char* fg_last_error(void) { return fg::t_last_error; }

int fg_version(void) { return 1; }

unsigned long long fg_launch_count(void) { return fg::g_launches.load(std::memory_order_relaxed); }

int fg_device_status(unsigned int* status, int reset, fg_stream_t stream) {
  FG_REQUIRE(status != nullptr, "fg_device_status: null status pointer");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  unsigned int v = 0;
  cudaError_t e = cudaMemcpyFromSymbolAsync(&v, fg::g_fg_device_status, sizeof(v), 0,
                                            cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e == cudaSuccess && reset && v != 0) {
    const unsigned int zero = 0;
    e = cudaMemcpyToSymbolAsync(fg::g_fg_device_status, &zero, sizeof(zero), 0,
                                cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  }
  if (e != cudaSuccess) {
    fg::set_last_error("fg_device_status: %s", cudaGetErrorString(e));
    return FG_ERR_CUDA;
  }
  *status = v;
  return FG_OK;
}

}  // extern "C"
