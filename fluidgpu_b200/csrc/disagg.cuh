// Consumer side of the disaggregated step's hand-offs: the first kernel that
// reads what another GPU stored (fg_gemm_bf16_packed_routed) waits for its
// flag itself, so no separate wait kernel sits between the hand-off and the
// work it feeds.
//
// Flags carry values, not toggles. Both sides compute the value of a
// message from their own per-step epoch counter (advanced once per step by
// fg_counter_add, after every wait of the step): value = epoch * seq_mul +
// seq_add, e.g. step * layers + layer + 1. A waiting CTA spins until the flag
// reaches its value (wrap-safe compare), so every CTA of the grid, however
// late it starts, waits for the same message and nothing needs resetting.
// Waits are bounded: on expiry the device status records a peer flag
// timeout (site 0x5xx) and the kernel finishes on whatever it reads.
//
// The data another GPU wrote is read through L2 (ld.global.cg): it is
// coherent there, and an SM's L1 may still hold the previous message's lines.
//
// Programmatic dependent launch: these kernels let their dependents launch
// only after the wait (griddepcontrol.launch_dependents follows it). A
// dependent launched earlier would sit in its own bounded pipeline waits
// for as long as the other GPU takes.
#pragma once
#include "common.cuh"
#include "elementwise.cuh"

namespace fg {
namespace disagg {

constexpr int kMaxFlags = 8;

struct WaitSpec {
  const uint32_t* flags[kMaxFlags];
  int n_flags;
  int rows_per_flag;  // row r waits flags[r / rows_per_flag]; 0: every row waits all flags
  const uint32_t* epoch;
  uint32_t seq_mul, seq_add;
  uint64_t timeout_ns;
};

__device__ __forceinline__ void wait_row(const WaitSpec& w, int row, unsigned int site) {
  if (threadIdx.x == 0 && w.n_flags > 0) {
    const uint32_t target = *w.epoch * w.seq_mul + w.seq_add;
    if (w.rows_per_flag > 0) {
      wait_at_least(w.flags[row / w.rows_per_flag], target, w.timeout_ns, site);
    } else {
      for (int i = 0; i < w.n_flags; ++i) wait_at_least(w.flags[i], target, w.timeout_ns, site + 1);
    }
  }
  __syncthreads();
}

// Rows gathered from other GPUs' buffers: row r is row r % rows_per_src of
// src[r / rows_per_src] (a peer's memory, read over NVLink), copied to
// copy[r] on this GPU as it is read.
struct GatherSpec {
  const uint4* src[kMaxFlags];
  int rows_per_src;
  uint4* copy;
};

// out[r] = RMSNorm(x[r]) once row r's flag has arrived (fg_rmsnorm semantics);
// GATHER: x[r] is read from gs.src (and kept in gs.copy) instead of x
template <int THREADS, bool GATHER>
__global__ void __launch_bounds__(THREADS) rmsnorm_wait_kernel(const uint4* __restrict__ x,
                                                               const uint4* __restrict__ w,
                                                               uint4* __restrict__ out, int H, float eps,
                                                               int mode, const WaitSpec ws, const GatherSpec gs) {
  griddep_wait();
  __shared__ float red[THREADS / 32];
  wait_row(ws, blockIdx.x, 0x501);
  griddep_launch_dependents();
  const int H8 = H >> 3;
  const uint4* xr = GATHER ? gs.src[blockIdx.x / gs.rows_per_src] + (int64_t)(blockIdx.x % gs.rows_per_src) * H8
                           : x + (int64_t)blockIdx.x * H8;
  uint4* orow = out + (int64_t)blockIdx.x * H8;
  constexpr int kMaxVec = 4;
  uint4 xv[kMaxVec];
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < kMaxVec; ++j) {
    const int i = threadIdx.x + j * THREADS;
    if (i < H8) xv[j] = __ldcg(xr + i);  // all of the row's loads in flight at once
  }
#pragma unroll
  for (int j = 0; j < kMaxVec; ++j) {
    const int i = threadIdx.x + j * THREADS;
    if (i < H8) {
      if (GATHER) gs.copy[(int64_t)blockIdx.x * H8 + i] = xv[j];
      const uint32_t* p = reinterpret_cast<const uint32_t*>(&xv[j]);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float2 f = unpack_bf16x2(p[q]);
        ss += f.x * f.x + f.y * f.y;
      }
    }
  }
  const float rstd = rsqrtf(block_sum<THREADS>(ss, red) / (float)H + eps);
#pragma unroll
  for (int j = 0; j < kMaxVec; ++j) {
    const int i = threadIdx.x + j * THREADS;
    if (i < H8) {
      const uint4 wv = w[i];
      const uint32_t* p = reinterpret_cast<const uint32_t*>(&xv[j]);
      const uint32_t* pw = reinterpret_cast<const uint32_t*>(&wv);
      uint4 o;
      uint32_t* po = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float2 f = unpack_bf16x2(p[q]);
        const float2 g = unpack_bf16x2(pw[q]);
        po[q] = mode == FG_NORM_LLAMA ? pack_bf16x2(g.x * rbf(f.x * rstd), g.y * rbf(f.y * rstd))
                                      : pack_bf16x2(g.x * (f.x * rstd), g.y * (f.y * rstd));
      }
      orow[i] = o;
    }
  }
}

// Once every shard's flag has arrived: h[r] = bf16(p[0][r] + ... + p[S-1][r])
// (fp32 sums in shard order, fg_sum_partials) and x[r] = RMSNorm(h[r]).
template <int THREADS>
__global__ void __launch_bounds__(THREADS) sum_rmsnorm_wait_kernel(const float4* __restrict__ parts, int S,
                                                                   long long plane4, uint4* __restrict__ h_out,
                                                                   const uint4* __restrict__ w,
                                                                   uint4* __restrict__ x_out, int H, float eps,
                                                                   int mode, const WaitSpec ws) {
  griddep_wait();
  __shared__ float red[THREADS / 32];
  wait_row(ws, blockIdx.x, 0x503);
  griddep_launch_dependents();
  const int H8 = H >> 3;
  const long long row4 = (long long)blockIdx.x * (H >> 2);
  constexpr int kMaxVec = 4;
  uint4 hv[kMaxVec];
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < kMaxVec; ++j) {
    const int i = threadIdx.x + j * THREADS;  // 8 values: two float4 of each plane
    if (i < H8) {
      float4 a = __ldcg(parts + row4 + 2 * i), b = __ldcg(parts + row4 + 2 * i + 1);
      for (int s = 1; s < S; ++s) {
        const float4 c = __ldcg(parts + s * plane4 + row4 + 2 * i);
        const float4 d = __ldcg(parts + s * plane4 + row4 + 2 * i + 1);
        a.x += c.x; a.y += c.y; a.z += c.z; a.w += c.w;
        b.x += d.x; b.y += d.y; b.z += d.z; b.w += d.w;
      }
      hv[j] = make_uint4(pack_bf16x2(a.x, a.y), pack_bf16x2(a.z, a.w), pack_bf16x2(b.x, b.y),
                         pack_bf16x2(b.z, b.w));
      h_out[(int64_t)blockIdx.x * H8 + i] = hv[j];
      const uint32_t* p = reinterpret_cast<const uint32_t*>(&hv[j]);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float2 f = unpack_bf16x2(p[q]);
        ss += f.x * f.x + f.y * f.y;
      }
    }
  }
  const float rstd = rsqrtf(block_sum<THREADS>(ss, red) / (float)H + eps);
#pragma unroll
  for (int j = 0; j < kMaxVec; ++j) {
    const int i = threadIdx.x + j * THREADS;
    if (i < H8) {
      const uint4 wv = w[i];
      const uint32_t* p = reinterpret_cast<const uint32_t*>(&hv[j]);
      const uint32_t* pw = reinterpret_cast<const uint32_t*>(&wv);
      uint4 o;
      uint32_t* po = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float2 f = unpack_bf16x2(p[q]);
        const float2 g = unpack_bf16x2(pw[q]);
        po[q] = mode == FG_NORM_LLAMA ? pack_bf16x2(g.x * rbf(f.x * rstd), g.y * rbf(f.y * rstd))
                                      : pack_bf16x2(g.x * (f.x * rstd), g.y * (f.y * rstd));
      }
      x_out[(int64_t)blockIdx.x * H8 + i] = o;
    }
  }
}

__global__ void counter_add_kernel(uint32_t* counter, uint32_t delta) {
  griddep_wait();
  griddep_launch_dependents();
  if (threadIdx.x == 0) *counter += delta;
}

inline int make_wait(WaitSpec& ws, uint32_t* const* flags, int n_flags, int rows_per_flag, const uint32_t* epoch,
                     uint32_t seq_mul, uint32_t seq_add, int timeout_ms, const char* what) {
  memset(&ws, 0, sizeof(ws));
  FG_REQUIRE(n_flags >= 0 && n_flags <= kMaxFlags, "%s: n_flags=%d (0..%d)", what, n_flags, kMaxFlags);
  FG_REQUIRE(n_flags == 0 || (flags && epoch), "%s: waiting needs flags and an epoch", what);
  for (int i = 0; i < n_flags; ++i) {
    FG_REQUIRE(flags[i] != nullptr, "%s: flags[%d] is null", what, i);
    ws.flags[i] = flags[i];
  }
  ws.n_flags = n_flags;
  ws.rows_per_flag = rows_per_flag;
  ws.epoch = epoch;
  ws.seq_mul = seq_mul;
  ws.seq_add = seq_add;
  ws.timeout_ns = (uint64_t)(timeout_ms > 0 ? timeout_ms : 2000) * 1000000ull;
  return FG_OK;
}

}  // namespace disagg
}  // namespace fg

extern "C" {

int fg_rmsnorm_wait(const fg_bf16* x, const fg_bf16* weight, fg_bf16* out, int T, int H, float eps,
                    int weight_mode, uint32_t* const* flags, int n_flags, int rows_per_flag,
                    const uint32_t* epoch, uint32_t seq_mul, uint32_t seq_add, int timeout_ms,
                    fg_stream_t stream) {
  FG_REQUIRE(x && weight && out, "fg_rmsnorm_wait: null pointer");
  FG_REQUIRE(T >= 0 && H > 0 && H % 8 == 0 && H <= 8192, "fg_rmsnorm_wait: H=%d (multiple of 8, <= 8192)", H);
  FG_REQUIRE(weight_mode == FG_NORM_LLAMA || weight_mode == FG_NORM_FP32MUL, "fg_rmsnorm_wait: bad weight_mode");
  FG_REQUIRE((((uintptr_t)x | (uintptr_t)weight | (uintptr_t)out) & 15) == 0,
             "fg_rmsnorm_wait: pointers must be 16-byte aligned");
  FG_REQUIRE(n_flags == 0 || (rows_per_flag > 0 && (long long)rows_per_flag * n_flags >= T),
             "fg_rmsnorm_wait: %d flags of %d rows do not cover %d rows", n_flags, rows_per_flag, T);
  fg::disagg::WaitSpec ws;
  const int rc = fg::disagg::make_wait(ws, flags, n_flags, rows_per_flag, epoch, seq_mul, seq_add, timeout_ms,
                                       "fg_rmsnorm_wait");
  if (rc) return rc;
  if (T == 0) return FG_OK;
  fg::disagg::GatherSpec gs;
  memset(&gs, 0, sizeof(gs));
  return fg::launch_k("fg_rmsnorm_wait", fg::disagg::rmsnorm_wait_kernel<256, false>, dim3(T), dim3(256), 0,
                      (cudaStream_t)stream, reinterpret_cast<const uint4*>(x),
                      reinterpret_cast<const uint4*>(weight), reinterpret_cast<uint4*>(out), H, eps,
                      weight_mode, ws, gs);
}

int fg_rmsnorm_gather_wait(const fg_bf16* const* srcs, int n_src, int rows_per_src, fg_bf16* gathered,
                           const fg_bf16* weight, fg_bf16* out, int T, int H, float eps, int weight_mode,
                           uint32_t* const* flags, int n_flags, int rows_per_flag, const uint32_t* epoch,
                           uint32_t seq_mul, uint32_t seq_add, int timeout_ms, fg_stream_t stream) {
  FG_REQUIRE(srcs && gathered && weight && out, "fg_rmsnorm_gather_wait: null pointer");
  FG_REQUIRE(n_src >= 1 && n_src <= fg::disagg::kMaxFlags && rows_per_src > 0 &&
                 (long long)n_src * rows_per_src >= T,
             "fg_rmsnorm_gather_wait: %d sources of %d rows (1..%d sources) do not cover %d rows", n_src,
             rows_per_src, fg::disagg::kMaxFlags, T);
  FG_REQUIRE(T >= 0 && H > 0 && H % 8 == 0 && H <= 8192, "fg_rmsnorm_gather_wait: H=%d (multiple of 8, <= 8192)",
             H);
  FG_REQUIRE(weight_mode == FG_NORM_LLAMA || weight_mode == FG_NORM_FP32MUL,
             "fg_rmsnorm_gather_wait: bad weight_mode");
  FG_REQUIRE((((uintptr_t)gathered | (uintptr_t)weight | (uintptr_t)out) & 15) == 0,
             "fg_rmsnorm_gather_wait: pointers must be 16-byte aligned");
  FG_REQUIRE(n_flags == 0 || (rows_per_flag > 0 && (long long)rows_per_flag * n_flags >= T),
             "fg_rmsnorm_gather_wait: %d flags of %d rows do not cover %d rows", n_flags, rows_per_flag, T);
  fg::disagg::GatherSpec gs;
  memset(&gs, 0, sizeof(gs));
  for (int i = 0; i < n_src; ++i) {
    FG_REQUIRE(srcs[i] != nullptr && ((uintptr_t)srcs[i] & 15) == 0,
               "fg_rmsnorm_gather_wait: srcs[%d] is null or not 16-byte aligned", i);
    gs.src[i] = reinterpret_cast<const uint4*>(srcs[i]);
  }
  gs.rows_per_src = rows_per_src;
  gs.copy = reinterpret_cast<uint4*>(gathered);
  fg::disagg::WaitSpec ws;
  const int rc = fg::disagg::make_wait(ws, flags, n_flags, rows_per_flag, epoch, seq_mul, seq_add, timeout_ms,
                                       "fg_rmsnorm_gather_wait");
  if (rc) return rc;
  if (T == 0) return FG_OK;
  return fg::launch_k("fg_rmsnorm_gather_wait", fg::disagg::rmsnorm_wait_kernel<256, true>, dim3(T), dim3(256),
                      0, (cudaStream_t)stream, static_cast<const uint4*>(nullptr),
                      reinterpret_cast<const uint4*>(weight), reinterpret_cast<uint4*>(out), H, eps,
                      weight_mode, ws, gs);
}

int fg_sum_rmsnorm_wait(const float* partials, int S, fg_bf16* h_out, const fg_bf16* weight, fg_bf16* x_out,
                        int T, int H, float eps, int weight_mode, uint32_t* const* flags, int n_flags,
                        const uint32_t* epoch, uint32_t seq_mul, uint32_t seq_add, int timeout_ms,
                        fg_stream_t stream) {
  FG_REQUIRE(partials && h_out && weight && x_out, "fg_sum_rmsnorm_wait: null pointer");
  FG_REQUIRE(S >= 1 && T >= 0 && H > 0 && H % 8 == 0 && H <= 8192,
             "fg_sum_rmsnorm_wait: S=%d H=%d (multiple of 8, <= 8192)", S, H);
  FG_REQUIRE(weight_mode == FG_NORM_LLAMA || weight_mode == FG_NORM_FP32MUL, "fg_sum_rmsnorm_wait: bad weight_mode");
  FG_REQUIRE((((uintptr_t)partials | (uintptr_t)h_out | (uintptr_t)weight | (uintptr_t)x_out) & 15) == 0,
             "fg_sum_rmsnorm_wait: pointers must be 16-byte aligned");
  fg::disagg::WaitSpec ws;
  const int rc = fg::disagg::make_wait(ws, flags, n_flags, 0, epoch, seq_mul, seq_add, timeout_ms,
                                       "fg_sum_rmsnorm_wait");
  if (rc) return rc;
  if (T == 0) return FG_OK;
  return fg::launch_k("fg_sum_rmsnorm_wait", fg::disagg::sum_rmsnorm_wait_kernel<256>, dim3(T), dim3(256), 0,
                      (cudaStream_t)stream, reinterpret_cast<const float4*>(partials), S,
                      (long long)T * H / 4, reinterpret_cast<uint4*>(h_out), reinterpret_cast<const uint4*>(weight),
                      reinterpret_cast<uint4*>(x_out), H, eps, weight_mode, ws);
}

int fg_preload(void) {
  // the module holding this library's kernels (found through one of them),
  // then every function in it loaded (driver entry points, no -lcuda)
  using GetModule = CUresult (*)(CUmodule*, CUfunction);
  using Count = CUresult (*)(unsigned int*, CUmodule);
  using Enumerate = CUresult (*)(CUfunction*, unsigned int, CUmodule);
  using Load = CUresult (*)(CUfunction);
  void *p_mod = nullptr, *p_count = nullptr, *p_enum = nullptr, *p_load = nullptr;
  cudaDriverEntryPointQueryResult q1, q2, q3, q4;
  if (cudaGetDriverEntryPoint("cuFuncGetModule", &p_mod, cudaEnableDefault, &q1) != cudaSuccess ||
      cudaGetDriverEntryPoint("cuModuleGetFunctionCount", &p_count, cudaEnableDefault, &q2) != cudaSuccess ||
      cudaGetDriverEntryPoint("cuModuleEnumerateFunctions", &p_enum, cudaEnableDefault, &q3) != cudaSuccess ||
      cudaGetDriverEntryPoint("cuFuncLoad", &p_load, cudaEnableDefault, &q4) != cudaSuccess ||
      q1 != cudaDriverEntryPointSuccess || q2 != cudaDriverEntryPointSuccess || q3 != cudaDriverEntryPointSuccess ||
      q4 != cudaDriverEntryPointSuccess) {
    fg::set_last_error("fg_preload: driver entry points for module enumeration unavailable");
    return FG_ERR_CUDA;
  }
  cudaFunction_t any = nullptr;
  cudaError_t e = cudaGetFuncBySymbol(&any, reinterpret_cast<const void*>(fg::disagg::counter_add_kernel));
  if (e != cudaSuccess) {
    fg::set_last_error("fg_preload: cudaGetFuncBySymbol: %s", cudaGetErrorString(e));
    return FG_ERR_CUDA;
  }
  CUmodule mod = nullptr;
  unsigned int n = 0;
  if (reinterpret_cast<GetModule>(p_mod)(&mod, reinterpret_cast<CUfunction>(any)) != CUDA_SUCCESS ||
      reinterpret_cast<Count>(p_count)(&n, mod) != CUDA_SUCCESS) {
    fg::set_last_error("fg_preload: cannot enumerate the library's kernels");
    return FG_ERR_CUDA;
  }
  CUfunction* fns = static_cast<CUfunction*>(malloc(sizeof(CUfunction) * (n ? n : 1)));
  if (!fns) {
    fg::set_last_error("fg_preload: out of host memory");
    return FG_ERR_CUDA;
  }
  int rc = FG_OK;
  if (reinterpret_cast<Enumerate>(p_enum)(fns, n, mod) != CUDA_SUCCESS) {
    fg::set_last_error("fg_preload: cuModuleEnumerateFunctions failed");
    rc = FG_ERR_CUDA;
  }
  for (unsigned int i = 0; rc == FG_OK && i < n; ++i) {
    if (reinterpret_cast<Load>(p_load)(fns[i]) != CUDA_SUCCESS) {
      fg::set_last_error("fg_preload: cuFuncLoad failed for kernel %u of %u", i, n);
      rc = FG_ERR_CUDA;
    }
  }
  free(fns);
  // the GEMM plans' resident-cluster counts too (best effort: without them
  // the plans count CTA slots instead)
  int (*active)[9] = nullptr;
  if (rc == FG_OK) (void)fg::gemm::active_clusters_table(active);
  return rc;
}

int fg_counter_add(uint32_t* counter, uint32_t delta, fg_stream_t stream) {
  FG_REQUIRE(counter, "fg_counter_add: null pointer");
  return fg::launch_k("fg_counter_add", fg::disagg::counter_add_kernel, dim3(1), dim3(32), 0,
                      (cudaStream_t)stream, counter, delta);
}

}  // extern "C"
