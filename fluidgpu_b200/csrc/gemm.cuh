// Dense bf16 GEMM for the decode step on 5th-generation tensor cores.
//
// Decode GEMMs are "skinny": T (tokens in the batch, 1..256) is far smaller
// than the output width N (4096..128256). The kernel therefore computes the
// transposed product D^T = W * X^T ("swap AB"): the weight tile is the MMA's
// M=128 operand and the tokens are its N dimension (16..256), so a single
// tcgen05.mma.cta_group::1.kind::f16 (M=128, N=BN, K=16) covers a whole
// 128-feature x BN-token tile and no tensor-core lane is wasted on padding.
//
// Pipeline per CTA (128 threads, one tile, one K slice):
//   warp 0 lane 0 : TMA producer. Streams W[128 x 64] and X[BN x 64] bf16
//                   tiles (128-byte swizzle) into a STAGES-deep ring.
//   warp 1 lane 0 : MMA issuer. 4 x tcgen05.mma per stage into a TMEM fp32
//                   accumulator (128 lanes x BN columns); tcgen05.commit
//                   frees the stage.
//   all 4 warps   : epilogue. tcgen05.ld (32x32b) brings row r = feature,
//                   columns = tokens into registers; bias / residual /
//                   SwiGLU are applied and bf16 stored token-major.
// Split-K: CTAs of one tile that own different K slices write fp32 partials
// into the caller's workspace; the last CTA to finish (atomic ticket) sums
// them, applies the epilogue and rearms the ticket.
//
// The weights are read exactly once per call (L2 evict_first hint); X is
// tiny and re-read by every tile (evict_last hint).
#pragma once
#include "common.cuh"

namespace fg {
namespace gemm {

constexpr int BM = 128;  // output features per tile (MMA M)
// Split-K tickets sit at the start of every workspace, so calls of any shape
// that share a workspace see the same (zero) tickets; partial sums follow.
constexpr int kMaxTickets = 16384;
constexpr size_t kTicketBytes = kMaxTickets * sizeof(unsigned int);
constexpr int BK = 64;   // K elements per stage = one 128-byte swizzle row
constexpr int kThreads = 128;

struct Params {
  __nv_bfloat16* out;
  const __nv_bfloat16* residual;
  const __nv_bfloat16* bias;
  float* partial;          // [tiles][splits][BN][BM]
  unsigned int* tickets;   // [tiles]
  int T, N, K;
  int ldo;                 // row stride of out (elements)
  int epilogue;
  int splits;
  int kb_per_split;
  int num_kb;
  int n_tiles;
};

template <int BN, int STAGES>
struct Layout {
  static constexpr int A_BYTES = BM * BK * 2;
  static constexpr int B_BYTES = BN * BK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int BAR_OFFSET = STAGES * STAGE_BYTES;
  static constexpr int TOTAL = BAR_OFFSET + (2 * STAGES + 1) * 8 + 16 + 16;
  static constexpr int DYN_SMEM = TOTAL + 1024;  // slack for 1024-byte alignment
  static constexpr uint32_t TMEM_COLS = BN < 32 ? 32 : BN;
  static_assert(A_BYTES % 1024 == 0 && B_BYTES % 1024 == 0, "tiles must keep 1024B alignment");
};

// UMMA shared-memory descriptor, K-major operand, 128-byte swizzle:
// 8-row x 128-byte swizzle atoms stacked every 1024 bytes (SBO = 1024).
__device__ __forceinline__ uint64_t sw128_kmajor_desc(uint32_t saddr) {
  return (uint64_t)((saddr & 0x3FFFFu) >> 4) | (1ull << 16) | (64ull << 32) | (1ull << 46) |
         (2ull << 61);
}

// Instruction descriptor for kind::f16: bf16 A/B, fp32 D, both K-major.
__host__ __device__ constexpr uint32_t idesc_bf16(int m, int n) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) |
         ((uint32_t)(m >> 4) << 24);
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_mma(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc,
                                       uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void tc_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   bar)
               : "memory");
}
__device__ __forceinline__ void tc_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,"
      "%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ float silu(float x) { return x / (1.f + __expf(-x)); }

// Apply the epilogue to 16 consecutive token columns of one accumulator row.
// row = TMEM lane (0..127) inside the tile; xch = SwiGLU exchange buffer
// [BN][64] fp32 in shared memory.
template <int BN>
__device__ __forceinline__ void epilogue_chunk(const Params& p, int n_tile, int t_tile, int row,
                                               int j0, const float (&v)[16], float* xch,
                                               bool up_half) {
  const int t_base = t_tile * BN + j0;
  if (p.epilogue == FG_EPI_SWIGLU) {
    // rows [0,64): gate of feature n_tile*64 + row; rows [64,128): up of the same
    if (up_half) {
      const int nrow = n_tile * BM + row;
      const float b = (p.bias && nrow < p.N) ? bf2f(p.bias[nrow]) : 0.f;
#pragma unroll
      for (int i = 0; i < 16; ++i) xch[(j0 + i) * 64 + (row - 64)] = rbf(v[i] + b);
    }
    return;
  }
  const int n = n_tile * BM + row;
  if (n >= p.N) return;
  const float b = p.bias ? bf2f(p.bias[n]) : 0.f;
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const int t = t_base + i;
    if (t < p.T) {
      float y = v[i] + b;
      if (p.epilogue == FG_EPI_RESIDUAL) y = bf2f(p.residual[(int64_t)t * p.ldo + n]) + rbf(y);
      p.out[(int64_t)t * p.ldo + n] = f2bf(y);
    }
  }
}

template <int BN>
__device__ __forceinline__ void swiglu_finish(const Params& p, int n_tile, int t_tile, int row,
                                              int j0, const float (&v)[16], const float* xch) {
  // called by the gate half (row < 64) after the up half filled xch
  const int f = n_tile * 64 + row;  // feature index in [0, N/2)
  const int nrow = n_tile * BM + row;
  if (nrow >= p.N) return;
  const float b = p.bias ? bf2f(p.bias[nrow]) : 0.f;
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const int t = t_tile * BN + j0 + i;
    if (t < p.T) {
      const float g = rbf(v[i] + b);
      const float u = xch[(j0 + i) * 64 + row];
      p.out[(int64_t)t * p.ldo + f] = f2bf(rbf(silu(g)) * u);
    }
  }
}

template <int BN, int STAGES>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_bf16_kernel(const __grid_constant__ CUtensorMap tm_w,
                     const __grid_constant__ CUtensorMap tm_x, const Params p) {
  using L = Layout<BN, STAGES>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int n_tile = blockIdx.x;
  const int t_tile = blockIdx.y;
  const int split = blockIdx.z;
  const int kb0 = split * p.kb_per_split;
  const int kb1 = min(kb0 + p.kb_per_split, p.num_kb);
  const int nk = kb1 - kb0;

  const uint32_t sbase = smem_u32(smem);
  const uint32_t bar_full = sbase + L::BAR_OFFSET;              // STAGES x 8 bytes
  const uint32_t bar_empty = bar_full + STAGES * 8;             // STAGES x 8 bytes
  const uint32_t bar_accum = bar_empty + STAGES * 8;            // 8 bytes
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::BAR_OFFSET + (2 * STAGES + 1) * 8);
  int* counters = reinterpret_cast<int*>(tmem_slot + 2);  // [0]=issued [1]=consumed [2]=last

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(bar_full + 8 * s, 1);
      mbar_init(bar_empty + 8 * s, 1);
    }
    mbar_init(bar_accum, 1);
    counters[0] = 0;
    counters[1] = 0;
    fence_mbar_init();
    prefetch_tensormap(&tm_w);
    prefetch_tensormap(&tm_x);
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(L::TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0 && lane == 0) {
    // ---------------- TMA producer ----------------
    const uint64_t pol_w = l2_policy_evict_first();
    const uint64_t pol_x = l2_policy_evict_last();
    int issued = 0;
    for (int i = 0; i < nk; ++i) {
      const int s = i % STAGES;
      const uint32_t ph = (uint32_t)(i / STAGES) & 1u;
      if (!mbar_wait(bar_empty + 8 * s, ph ^ 1u, 0x101)) break;
      mbar_arrive_expect_tx(bar_full + 8 * s, L::STAGE_BYTES);
      const uint32_t a_dst = sbase + s * L::STAGE_BYTES;
      const int kx = (kb0 + i) * BK;
      tma_load_2d_hint(a_dst, &tm_w, bar_full + 8 * s, kx, n_tile * BM, pol_w);
      tma_load_2d_hint(a_dst + L::A_BYTES, &tm_x, bar_full + 8 * s, kx, t_tile * BN, pol_x);
      ++issued;
    }
    counters[0] = issued;
  } else if (warp == 1 && lane == 0) {
    // ---------------- MMA issuer ----------------
    constexpr uint32_t idesc = idesc_bf16(BM, BN);
    int consumed = 0;
    for (int i = 0; i < nk; ++i) {
      const int s = i % STAGES;
      const uint32_t ph = (uint32_t)(i / STAGES) & 1u;
      if (!mbar_wait(bar_full + 8 * s, ph, 0x102)) break;
      tc_fence_after();
      const uint32_t a_addr = sbase + s * L::STAGE_BYTES;
      const uint64_t adesc = sw128_kmajor_desc(a_addr);
      const uint64_t bdesc = sw128_kmajor_desc(a_addr + L::A_BYTES);
#pragma unroll
      for (int kk = 0; kk < BK / 16; ++kk) {
        // +32 bytes along K inside the 128-byte swizzle row = +2 in the 16-byte address field
        tc_mma(tmem, adesc + 2 * kk, bdesc + 2 * kk, idesc, (i > 0 || kk > 0) ? 1u : 0u);
      }
      tc_commit(bar_empty + 8 * s);
      ++consumed;
    }
    counters[1] = consumed;
    tc_commit(bar_accum);  // arrives once every MMA issued above has completed
  }
  __syncwarp();

  // ---------------- epilogue ----------------
  const bool acc_ok = mbar_wait(bar_accum, 0, 0x103);
  tc_fence_after();
  const int row = warp * 32 + lane;  // accumulator row = TMEM lane
  const uint32_t taddr = tmem + ((uint32_t)(warp * 32) << 16);
  float* xch = reinterpret_cast<float*>(smem);  // stage ring is idle once the accumulator is final
  const bool swiglu = p.epilogue == FG_EPI_SWIGLU;
  const int tile_id = t_tile * p.n_tiles + n_tile;

  if (p.splits == 1) {
#pragma unroll 1
    for (int j0 = 0; j0 < BN; j0 += 16) {
      float v[16];
      tc_ld16(taddr + j0, v);
      if (!acc_ok) {
#pragma unroll
        for (int i = 0; i < 16; ++i) v[i] = 0.f;
      }
      epilogue_chunk<BN>(p, n_tile, t_tile, row, j0, v, xch, row >= 64);
    }
    if (swiglu) {
      __syncthreads();
      if (row < 64) {
#pragma unroll 1
        for (int j0 = 0; j0 < BN; j0 += 16) {
          float v[16];
          tc_ld16(taddr + j0, v);
          swiglu_finish<BN>(p, n_tile, t_tile, row, j0, v, xch);
        }
      } else {
        // keep the warp converged for the .sync.aligned loads of warps 0-1
      }
    }
  } else {
    // write this slice's partial sums: [BN][BM] so a warp stores 128 contiguous bytes per column
    float* part = p.partial + ((int64_t)tile_id * p.splits + split) * (BN * BM);
#pragma unroll 1
    for (int j0 = 0; j0 < BN; j0 += 16) {
      float v[16];
      tc_ld16(taddr + j0, v);
#pragma unroll
      for (int i = 0; i < 16; ++i) __stcg(part + (j0 + i) * BM + row, acc_ok ? v[i] : 0.f);
    }
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
      const unsigned int prev = atomicAdd(p.tickets + tile_id, 1u);
      counters[2] = (prev == (unsigned int)(p.splits - 1)) ? 1 : 0;
    }
    __syncthreads();
    if (counters[2]) {
      __threadfence();
      const float* base = p.partial + (int64_t)tile_id * p.splits * (BN * BM);
#pragma unroll 1
      for (int j0 = 0; j0 < BN; j0 += 16) {
        float v[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) v[i] = 0.f;
        for (int s = 0; s < p.splits; ++s) {
#pragma unroll
          for (int i = 0; i < 16; ++i) v[i] += __ldcg(base + (int64_t)s * BN * BM + (j0 + i) * BM + row);
        }
        epilogue_chunk<BN>(p, n_tile, t_tile, row, j0, v, xch, row >= 64);
      }
      if (swiglu) {
        __syncthreads();
        if (row < 64) {
#pragma unroll 1
          for (int j0 = 0; j0 < BN; j0 += 16) {
            float v[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) v[i] = 0.f;
            for (int s = 0; s < p.splits; ++s) {
#pragma unroll
              for (int i = 0; i < 16; ++i)
                v[i] += __ldcg(base + (int64_t)s * BN * BM + (j0 + i) * BM + row);
            }
            swiglu_finish<BN>(p, n_tile, t_tile, row, j0, v, xch);
          }
        }
      }
      if (threadIdx.x == 0) p.tickets[tile_id] = 0u;  // rearm for the next call
    }
  }

  // ---------------- teardown ----------------
  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0) {
    // after a failed wait: let TMA copies that were issued but never consumed land
    for (int i = counters[1]; i < counters[0]; ++i) {
      mbar_wait(bar_full + 8 * (i % STAGES), (uint32_t)(i / STAGES) & 1u, 0x104);
    }
  }
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(L::TMEM_COLS)
                 : "memory");
  }
}

inline int pick_bn(int T) {
  if (T <= 16) return 16;
  if (T <= 32) return 32;
  if (T <= 64) return 64;
  if (T <= 128) return 128;
  return 256;
}

inline int pick_splits(int T, int N, int K) {
  const int bn = pick_bn(T);
  const int tiles = ((N + BM - 1) / BM) * ((T + bn - 1) / bn);
  const int num_kb = (K + BK - 1) / BK;
  const int sms = num_sms();
  if (tiles >= sms) return 1;
  int s = sms / tiles;                 // one wave of at most one CTA per SM
  s = s < num_kb / 4 ? s : num_kb / 4; // at least 4 stages of K per slice
  if (s < 1) s = 1;
  // even slices: no empty CTA
  const int per = (num_kb + s - 1) / s;
  return (num_kb + per - 1) / per;
}

template <int BN, int STAGES>
int launch(const Params& p, const CUtensorMap& tw, const CUtensorMap& tx, cudaStream_t st) {
  using L = Layout<BN, STAGES>;
  auto kern = gemm_bf16_kernel<BN, STAGES>;
  static bool attr_done[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!attr_done[dev & 63]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::DYN_SMEM);
    if (e != cudaSuccess) {
      set_last_error("fg_gemm_bf16: cudaFuncSetAttribute: %s", cudaGetErrorString(e));
      return FG_ERR_CUDA;
    }
    attr_done[dev & 63] = true;
  }
  dim3 grid(p.n_tiles, (p.T + BN - 1) / BN, p.splits);
  kern<<<grid, kThreads, L::DYN_SMEM, st>>>(tw, tx, p);
  return check_launch("fg_gemm_bf16");
}

}  // namespace gemm
}  // namespace fg

extern "C" {

int fg_gemm_pick_splits(int T, int N, int K) {
  if (T <= 0 || N <= 0 || K <= 0) return 1;
  return fg::gemm::pick_splits(T, N, K);
}

size_t fg_gemm_workspace_bytes(int T, int N, int K, int splits) {
  if (T <= 0 || N <= 0 || K <= 0) return 0;
  if (splits <= 0) splits = fg::gemm::pick_splits(T, N, K);
  if (splits <= 1) return 0;
  const int bn = fg::gemm::pick_bn(T);
  const size_t tiles = (size_t)((N + fg::gemm::BM - 1) / fg::gemm::BM) * ((T + bn - 1) / bn);
  // ticket block, then the partial sums
  return fg::gemm::kTicketBytes + tiles * splits * bn * fg::gemm::BM * sizeof(float);
}

int fg_gemm_bf16(const fg_bf16* x, const fg_bf16* w, fg_bf16* out, const fg_bf16* residual,
                 const fg_bf16* bias, int T, int N, int K, int epilogue, int splits,
                 void* workspace, size_t workspace_bytes, fg_stream_t stream) {
  using namespace fg::gemm;
  FG_REQUIRE(x && w && out, "fg_gemm_bf16: null pointer");
  FG_REQUIRE(T >= 0 && N > 0 && K > 0 && K % 8 == 0, "fg_gemm_bf16: bad sizes T=%d N=%d K=%d", T,
             N, K);
  FG_REQUIRE(epilogue == FG_EPI_STORE || epilogue == FG_EPI_RESIDUAL || epilogue == FG_EPI_SWIGLU,
             "fg_gemm_bf16: bad epilogue %d", epilogue);
  FG_REQUIRE(epilogue != FG_EPI_RESIDUAL || residual != nullptr,
             "fg_gemm_bf16: residual epilogue needs a residual");
  FG_REQUIRE(epilogue != FG_EPI_SWIGLU || N % BM == 0,
             "fg_gemm_bf16: SwiGLU needs N (=2*I) to be a multiple of 128, got %d", N);
  FG_REQUIRE((((uintptr_t)x | (uintptr_t)w) & 15) == 0, "fg_gemm_bf16: x/w must be 16-byte aligned");
  if (T == 0) return FG_OK;
  const int num_kb = (K + BK - 1) / BK;
  if (splits <= 0) splits = pick_splits(T, N, K);
  if (splits > num_kb) splits = num_kb;
  const int per = (num_kb + splits - 1) / splits;
  splits = (num_kb + per - 1) / per;  // no empty K slice
  const int bn = pick_bn(T);
  Params p;
  p.out = reinterpret_cast<__nv_bfloat16*>(out);
  p.residual = reinterpret_cast<const __nv_bfloat16*>(residual);
  p.bias = reinterpret_cast<const __nv_bfloat16*>(bias);
  p.T = T;
  p.N = N;
  p.K = K;
  p.ldo = epilogue == FG_EPI_SWIGLU ? N / 2 : N;
  p.epilogue = epilogue;
  p.splits = splits;
  p.kb_per_split = per;
  p.num_kb = num_kb;
  p.n_tiles = (N + BM - 1) / BM;
  p.partial = nullptr;
  p.tickets = nullptr;
  if (splits > 1) {
    const size_t need = fg_gemm_workspace_bytes(T, N, K, splits);
    FG_REQUIRE(workspace != nullptr && workspace_bytes >= need,
               "fg_gemm_bf16: split-K needs %zu workspace bytes, got %zu", need, workspace_bytes);
    FG_REQUIRE(((uintptr_t)workspace & 255) == 0, "fg_gemm_bf16: workspace must be 256-byte aligned");
    const size_t tiles = (size_t)p.n_tiles * ((T + bn - 1) / bn);
    FG_REQUIRE(tiles <= (size_t)kMaxTickets, "fg_gemm_bf16: %zu tiles exceed the %d split-K tickets",
               tiles, kMaxTickets);
    p.tickets = reinterpret_cast<unsigned int*>(workspace);
    p.partial = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(workspace) + kTicketBytes);
  }
  CUtensorMap tw, tx;
  int rc = fg::make_tmap_2d_bf16(&tw, w, (uint64_t)K, (uint64_t)N, (uint64_t)K * 2, BK, BM,
                                 CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  rc = fg::make_tmap_2d_bf16(&tx, x, (uint64_t)K, (uint64_t)T, (uint64_t)K * 2, BK, bn,
                             CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  switch (bn) {
    case 16: return launch<16, 8>(p, tw, tx, st);
    case 32: return launch<32, 8>(p, tw, tx, st);
    case 64: return launch<64, 6>(p, tw, tx, st);
    case 128: return launch<128, 5>(p, tw, tx, st);
    default: return launch<256, 4>(p, tw, tx, st);
  }
}

}  // extern "C"
