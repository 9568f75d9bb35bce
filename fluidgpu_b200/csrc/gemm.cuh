// Dense bf16 GEMM for the decode step on 5th-generation tensor cores.
//
// Decode GEMMs are "skinny": T (tokens in the batch, 1..256) is far smaller
// than the output width N (4096..128256), so the time is the weight stream
// from HBM. The kernel computes the transposed product D^T = W * X^T ("swap
// AB"): a 128-row weight tile is the M=128 operand of
// tcgen05.mma.cta_group::1.kind::f16 and the tokens are its N dimension
// (BN = 16..256), fp32 accumulation in TMEM.
//
// Weight streaming. Weights are static, so they are packed once
// (fg_pack_weight_bf16) into contiguous 16 KB tiles [N/128][K/64][128x64] that
// already hold the 128-byte-swizzled K-major image the UMMA descriptor reads:
// one 1-D bulk copy (cp.async.bulk) moves a whole tile, a long contiguous
// stream per CTA. Row-major weights are also accepted (2-D TMA boxes).
//
// Work distribution, by the number of 128 x BN output tiles:
//  - tiles >= half the resident CTA slots (gate_up, lm_head): one CTA per
//    tile; with packed weights this streams at 90-99% of the HBM peak.
//  - fewer tiles (qkv, o_proj, down): a thread-block cluster of S <= 8 CTAs
//    per tile, CTA r owning K slice r; S is the largest that keeps all the
//    tiles' clusters resident in one wave (for one CTA per SM the device's
//    own count of resident clusters per size, cudaOccupancyMaxActiveClusters). The fp32 partial tiles are reduced
//    through distributed shared memory: every CTA parks its accumulator in
//    its own shared memory, and after a cluster barrier CTA r sums rows
//    [r*128/S, (r+1)*128/S) across the S CTAs and runs the epilogue for them.
//    No global partials, no second kernel. S = 1 is a plain CTA per tile.
//  - on request (splits < 0): persistent stream-K. The work is U = tiles x
//    (K/64) units; G CTAs take contiguous unit ranges of equal length. A CTA
//    whose range covers a whole tile runs its epilogue directly; CTAs sharing
//    a tile write fp32 partials to the workspace and the last to arrive
//    (atomic ticket) sums them and runs the epilogue.
//
// Warp roles (192 threads):
//   warp 0 lane 0 : producer. Weight tiles (bulk copy, L2 evict_first) for the
//                   first ring stages are issued BEFORE griddepcontrol.wait, so
//                   under programmatic dependent launch the stream starts
//                   while the previous kernel drains; activation tiles (2-D
//                   TMA, L2 evict_last) follow the wait.
//   warp 1 lane 0 : MMA issuer, 4 x (128 x BN x 16) MMAs per 64-wide K step,
//                   tcgen05.commit frees ring stages; two TMEM accumulators
//                   alternate between segments.
//   warps 2-5     : epilogue. tcgen05.ld (32x32b) of their TMEM lane quarter;
//                   bias / residual / SwiGLU; bf16 stores, token-major.
#pragma once
#include <mutex>
#include <cooperative_groups.h>

#include "common.cuh"

namespace fg {
namespace gemm {

constexpr int BM = 128;             // output features per tile (MMA M)
constexpr int BK = 64;              // K elements per unit = one 128-byte swizzle row
constexpr int kTileBytes = BM * BK * 2;
constexpr int kThreads = 192;
// split tickets sit at the start of every workspace so calls of any shape
// that share one see the same (zero) tickets; partial sums follow
constexpr int kMaxTickets = 16384;
constexpr size_t kTicketBytes = kMaxTickets * sizeof(unsigned int);

constexpr int kMaxRoutes = 8;  // peer destinations / flags of a routed GEMM

struct Params {
  __nv_bfloat16* out;
  const __nv_bfloat16* residual;
  const __nv_bfloat16* bias;
  const uint8_t* w_packed;   // packed weights (PACKED kernels)
  float* partial;            // [tiles][max_contrib][BN][BM]
  unsigned int* tickets;     // [tiles]
  int T, N, K;
  int ldo;                   // row stride of out (elements)
  int epilogue;
  int n_tiles, t_tiles, nkb;
  long long units;           // tiles * nkb
  int grid;                  // G (stream-K) / tiles (cluster kernel)
  int max_contrib;
  int split;                 // S: CTAs per tile along K (cluster kernel)
  // routed output (fg_gemm_bf16_packed_routed): row t of the result goes to
  // dst[t / dst_rows] at row t % dst_rows (FG_ROUTE_SPLIT) or to every dst[d]
  // at row dst_row0 + t (FG_ROUTE_BROADCAST); route 0 writes `out`
  int route, n_dst, dst_rows, dst_row0;
  void* dst[kMaxRoutes];
  // completion signal: after every CTA's stores, the last CTA (ticket)
  // release-stores epoch[0] * seq_mul + seq_add into each sig[i] (system scope)
  int n_sig, total_ctas;
  uint32_t* sig[kMaxRoutes];
  const uint32_t* epoch;
  uint32_t seq_mul, seq_add;
  unsigned int* sig_ticket;
};

// Store value v of output row t (a token), column n, where the Params route it.
template <typename T>
__device__ __forceinline__ void store_out(const Params& p, int t, int n, T v) {
  if (p.route == 0) {
    reinterpret_cast<T*>(p.out)[(int64_t)t * p.ldo + n] = v;
  } else if (p.route == FG_ROUTE_SPLIT) {
    const int d = t / p.dst_rows;
    reinterpret_cast<T*>(p.dst[d])[(int64_t)(t - d * p.dst_rows) * p.ldo + n] = v;
  } else {
    for (int d = 0; d < p.n_dst; ++d)
      reinterpret_cast<T*>(p.dst[d])[(int64_t)(p.dst_row0 + t) * p.ldo + n] = v;
  }
}

// After a CTA's last store: publish the result once every CTA of the grid
// has stored (see Params). Executed by all threads of the CTA.
__device__ __forceinline__ void signal_done(const Params& p) {
  if (p.n_sig == 0) return;
  __threadfence_system();  // this thread's (peer) stores before the ticket
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned int prev = atomicAdd(p.sig_ticket, 1u);
    if (prev == (unsigned int)(p.total_ctas - 1)) {
      __threadfence_system();
      const uint32_t v = *p.epoch * p.seq_mul + p.seq_add;
      for (int i = 0; i < p.n_sig; ++i) st_release_sys(p.sig[i], v);
      *p.sig_ticket = 0u;  // rearmed: the next grid's CTAs count after griddep_wait
    }
  }
}

template <int BN, int STAGES>
struct Layout {
  static constexpr int A_BYTES = kTileBytes;
  static constexpr int B_BYTES = BN * BK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int XCH_OFFSET = STAGES * STAGE_BYTES;       // SwiGLU exchange, bf16 [BN][64]
  static constexpr int XCH_BYTES = BN * 64 * 2;
  static constexpr int BAR_OFFSET = XCH_OFFSET + XCH_BYTES;     // full[S] empty[S] accf[2] acce[2]
  static constexpr int MISC_OFFSET = BAR_OFFSET + (2 * STAGES + 4) * 8;
  static constexpr int TOTAL = MISC_OFFSET + 64;
  static constexpr int DYN_SMEM = TOTAL + 1024;                 // slack for 1024-byte alignment
  static constexpr uint32_t TMEM_COLS = 2 * BN < 32 ? 32 : 2 * BN;
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

// named barrier over the four epilogue warps
__device__ __forceinline__ void epi_sync() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

__device__ __forceinline__ long long unit_begin(long long U, int G, int c) {
  return (U * (long long)c) / G;
}
// the CTA whose unit range holds unit u
__device__ __forceinline__ int cta_of_unit(long long U, int G, long long u) {
  int c = (int)((u * G) / U);
  while (c + 1 < G && unit_begin(U, G, c + 1) <= u) ++c;
  while (c > 0 && unit_begin(U, G, c) > u) --c;
  return c;
}

// Tile t covers weight rows n_tile * 128.. and tokens t_tile * BN..; token
// tiles vary fastest, so the CTAs resident at one time share few weight
// tiles and a large-T GEMM (prefill) reads each weight tile from HBM once,
// its other token tiles hitting L2. With one token tile (decode) t = n_tile.
__device__ __forceinline__ int tile_n(const Params& p, int tile) { return tile / p.t_tiles; }
__device__ __forceinline__ int tile_t(const Params& p, int tile) { return tile - (tile / p.t_tiles) * p.t_tiles; }

// Epilogue of one 128 x BN tile from a value source load16(j0, v[16]) giving
// columns j0..j0+15 of accumulator row `row` (= 32*q + lane).
template <int BN, class Load>
__device__ __forceinline__ void apply_epilogue(const Params& p, int n_tile, int t_tile, int q, int lane,
                                               __nv_bfloat16* xch, Load&& load16) {
  const int row = q * 32 + lane;
  if (p.epilogue == FG_EPI_SWIGLU) {
    // rows [0,64) hold gate features n_tile*64 + row, rows [64,128) the matching up
    if (q >= 2) {
      const int nrow = n_tile * BM + row;
      const float b = p.bias ? bf2f(p.bias[nrow]) : 0.f;
#pragma unroll 1
      for (int j0 = 0; j0 < BN; j0 += 16) {
        float v[16];
        load16(j0, v);
#pragma unroll
        for (int i = 0; i < 16; ++i) xch[(j0 + i) * 64 + (row - 64)] = f2bf(v[i] + b);
      }
    }
    epi_sync();
    if (q < 2) {
      const int nrow = n_tile * BM + row;
      const float b = p.bias ? bf2f(p.bias[nrow]) : 0.f;
      const int f = n_tile * 64 + row;
#pragma unroll 1
      for (int j0 = 0; j0 < BN; j0 += 16) {
        float v[16];
        load16(j0, v);
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const int t = t_tile * BN + j0 + i;
          if (t < p.T) {
            const float g = rbf(v[i] + b);
            const float u = bf2f(xch[(j0 + i) * 64 + row]);
            p.out[(int64_t)t * p.ldo + f] = f2bf(rbf(silu(g)) * u);
          }
        }
      }
    }
    epi_sync();  // xch is free again
    return;
  }
  const int n = n_tile * BM + row;
  const bool in = n < p.N;
  const float b = (p.bias && in) ? bf2f(p.bias[n]) : 0.f;
#pragma unroll 1
  for (int j0 = 0; j0 < BN; j0 += 16) {
    float v[16];
    load16(j0, v);  // every lane loads (TMEM loads are warp-collective)
    if (!in) continue;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const int t = t_tile * BN + j0 + i;
      if (t < p.T) {
        float y = v[i] + b;
        if (p.epilogue == FG_EPI_F32) {
          if (p.residual) y += bf2f(p.residual[(int64_t)t * p.ldo + n]);
          store_out<float>(p, t, n, y);
          continue;
        }
        if (p.epilogue == FG_EPI_RESIDUAL) y = bf2f(p.residual[(int64_t)t * p.ldo + n]) + rbf(y);
        store_out<__nv_bfloat16>(p, t, n, f2bf(y));
      }
    }
  }
}

template <int BN, int STAGES, bool PACKED>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_bf16_kernel(const __grid_constant__ CUtensorMap tm_w,
                     const __grid_constant__ CUtensorMap tm_x, const Params p) {
  using L = Layout<BN, STAGES>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const long long U = p.units;
  const int G = p.grid;
  const long long u0 = unit_begin(U, G, blockIdx.x);
  const long long u1 = unit_begin(U, G, blockIdx.x + 1);

  const uint32_t sbase = smem_u32(smem);
  const uint32_t bar_full = sbase + L::BAR_OFFSET;
  const uint32_t bar_empty = bar_full + STAGES * 8;
  const uint32_t bar_accf = bar_empty + STAGES * 8;  // 2 barriers
  const uint32_t bar_acce = bar_accf + 16;           // 2 barriers
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::MISC_OFFSET);
  int* misc = reinterpret_cast<int*>(smem + L::MISC_OFFSET + 16);  // [0] issued [1] consumed [2] last
  __nv_bfloat16* xch = reinterpret_cast<__nv_bfloat16*>(smem + L::XCH_OFFSET);

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(bar_full + 8 * s, 1);
      mbar_init(bar_empty + 8 * s, 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(bar_accf + 8 * b, 1);
      mbar_init(bar_acce + 8 * b, 4);  // one arrival per epilogue warp
    }
    misc[0] = 0;
    misc[1] = 0;
    fence_mbar_init();
    if (!PACKED) prefetch_tensormap(&tm_w);
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
  if (threadIdx.x == 0) griddep_launch_dependents();

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- producer ----------------
      const uint64_t pol_w = l2_policy_evict_first();
      const uint64_t pol_x = l2_policy_evict_last();
      const long long n = u1 - u0;
      const int pre = (int)(n < STAGES ? n : STAGES);
      auto load_w = [&](long long u, int s) {
        const int tile = (int)(u / p.nkb);
        const int kb = (int)(u - (long long)tile * p.nkb);
        const int n_tile = tile_n(p, tile);
        const uint32_t dst = sbase + s * L::STAGE_BYTES;
        if (PACKED) {
          const uint8_t* src = p.w_packed + ((size_t)n_tile * p.nkb + kb) * kTileBytes;
          bulk_load(dst, src, kTileBytes, bar_full + 8 * s, pol_w);
        } else {
          tma_load_2d_hint(dst, &tm_w, bar_full + 8 * s, kb * BK, n_tile * BM, pol_w);
        }
      };
      auto load_x = [&](long long u, int s) {
        const int tile = (int)(u / p.nkb);
        const int kb = (int)(u - (long long)tile * p.nkb);
        const int t_tile = tile_t(p, tile);
        tma_load_2d_hint(sbase + s * L::STAGE_BYTES + L::A_BYTES, &tm_x, bar_full + 8 * s, kb * BK,
                         t_tile * BN, pol_x);
      };
      // the weights do not depend on earlier kernels: start streaming them now
      for (int i = 0; i < pre; ++i) {
        mbar_arrive_expect_tx(bar_full + 8 * i, L::STAGE_BYTES);
        load_w(u0 + i, i);
      }
      griddep_wait();
      for (int i = 0; i < pre; ++i) load_x(u0 + i, i);
      int issued = pre;
      for (long long i = pre; i < n; ++i) {
        const int s = (int)(i % STAGES);
        const uint32_t ph = (uint32_t)(i / STAGES) & 1u;
        if (!mbar_wait(bar_empty + 8 * s, ph ^ 1u, 0x101)) break;
        mbar_arrive_expect_tx(bar_full + 8 * s, L::STAGE_BYTES);
        load_w(u0 + i, s);
        load_x(u0 + i, s);
        ++issued;
      }
      misc[0] = issued;
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer ----------------
      constexpr uint32_t idesc = idesc_bf16(BM, BN);
      long long i = 0;
      int seg = 0;
      bool ok = true;
      for (long long u = u0; u < u1 && ok; ++seg) {
        const int tile = (int)(u / p.nkb);
        const int kb0 = (int)(u - (long long)tile * p.nkb);
        const long long left = u1 - u;
        const int nseg = (int)((p.nkb - kb0) < left ? (p.nkb - kb0) : left);
        const int buf = seg & 1;
        if (!mbar_wait(bar_acce + 8 * buf, (uint32_t)((seg >> 1) & 1) ^ 1u, 0x102)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem + buf * BN;
        for (int j = 0; j < nseg; ++j, ++i) {
          const int s = (int)(i % STAGES);
          const uint32_t ph = (uint32_t)(i / STAGES) & 1u;
          if (!mbar_wait(bar_full + 8 * s, ph, 0x103)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = sbase + s * L::STAGE_BYTES;
          const uint64_t adesc = sw128_kmajor_desc(a_addr);
          const uint64_t bdesc = sw128_kmajor_desc(a_addr + L::A_BYTES);
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            // +32 bytes along K inside the 128-byte swizzle row = +2 in the address field
            tc_mma(d, adesc + 2 * kk, bdesc + 2 * kk, idesc, (j > 0 || kk > 0) ? 1u : 0u);
          }
          tc_commit(bar_empty + 8 * s);
          misc[1] = (int)(i + 1);
        }
        tc_commit(bar_accf + 8 * buf);  // arrives when this segment's MMAs are done
        u += nseg;
      }
    }
  } else {
    // ---------------- epilogue (warps 2..5) ----------------
    griddep_wait();
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    const int row = q * 32 + lane;
    int seg = 0;
    for (long long u = u0; u < u1; ++seg) {
      const int tile = (int)(u / p.nkb);
      const int kb0 = (int)(u - (long long)tile * p.nkb);
      const long long left = u1 - u;
      const int nseg = (int)((p.nkb - kb0) < left ? (p.nkb - kb0) : left);
      const bool whole = (kb0 == 0) && (nseg == p.nkb);
      const int buf = seg & 1;
      const bool acc_ok = mbar_wait(bar_accf + 8 * buf, (uint32_t)(seg >> 1) & 1u, 0x104);
      tc_fence_after();
      const uint32_t taddr = tmem + buf * BN + ((uint32_t)(q * 32) << 16);
      auto from_tmem = [&](int j0, float (&v)[16]) {
        tc_ld16(taddr + j0, v);
        if (!acc_ok) {
#pragma unroll
          for (int i = 0; i < 16; ++i) v[i] = 0.f;
        }
      };
      if (whole) {
        apply_epilogue<BN>(p, tile_n(p, tile), tile_t(p, tile), q, lane, xch, from_tmem);
      } else {
        const long long first = (long long)tile * p.nkb;
        const int c_first = cta_of_unit(U, G, first);
        const int c_last = cta_of_unit(U, G, first + p.nkb - 1);
        // partial layout [BN/4][BM][4]: a warp stores / loads 512 contiguous bytes per float4
        float4* slot = reinterpret_cast<float4*>(
            p.partial + ((size_t)tile * p.max_contrib + (blockIdx.x - c_first)) * (BN * BM));
#pragma unroll 1
        for (int j0 = 0; j0 < BN; j0 += 16) {
          float v[16];
          from_tmem(j0, v);
#pragma unroll
          for (int i = 0; i < 4; ++i)
            __stcg(slot + ((j0 >> 2) + i) * BM + row, make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]));
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(bar_acce + 8 * buf);  // accumulator read: MMA may reuse it
        __threadfence();
        epi_sync();
        if (threadIdx.x == 64) {
          const unsigned int prev = atomicAdd(p.tickets + tile, 1u);
          misc[2] = (prev == (unsigned int)(c_last - c_first)) ? 1 : 0;
        }
        epi_sync();
        if (misc[2]) {
          __threadfence();
          const int count = c_last - c_first + 1;
          const float4* base = reinterpret_cast<const float4*>(
              p.partial + (size_t)tile * p.max_contrib * (BN * BM));
          auto from_partials = [&](int j0, float (&v)[16]) {
#pragma unroll
            for (int i = 0; i < 16; ++i) v[i] = 0.f;
            // four contributors' loads in flight per round trip
            for (int c = 0; c < count; c += 4) {
              float4 r[4][4];
#pragma unroll
              for (int cc = 0; cc < 4; ++cc) {
#pragma unroll
                for (int i = 0; i < 4; ++i)
                  r[cc][i] = (c + cc < count)
                                 ? __ldcg(base + (size_t)(c + cc) * (BN * BM / 4) + ((j0 >> 2) + i) * BM + row)
                                 : make_float4(0.f, 0.f, 0.f, 0.f);
              }
#pragma unroll
              for (int cc = 0; cc < 4; ++cc) {
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                  v[4 * i] += r[cc][i].x;
                  v[4 * i + 1] += r[cc][i].y;
                  v[4 * i + 2] += r[cc][i].z;
                  v[4 * i + 3] += r[cc][i].w;
                }
              }
            }
          };
          apply_epilogue<BN>(p, tile_n(p, tile), tile_t(p, tile), q, lane, xch, from_partials);
          if (threadIdx.x == 64) p.tickets[tile] = 0u;  // rearm for the next call
        }
        u += nseg;
        continue;
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar_acce + 8 * buf);
      u += nseg;
    }
  }

  // ---------------- teardown ----------------
  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0) {
    // after a failed wait: let bulk / TMA copies that were issued but never
    // consumed land before the CTA's shared memory is released
    for (int i = misc[1]; i < misc[0]; ++i)
      mbar_wait(bar_full + 8 * (i % STAGES), (uint32_t)(i / STAGES) & 1u, 0x105);
  }
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(L::TMEM_COLS)
                 : "memory");
  }
}

// ---------------------------------------------------------------------------
// cluster split-K kernel: grid (tiles, S), cluster (1, S, 1)
// ---------------------------------------------------------------------------
template <int BN, int STAGES, bool PACKED>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_cluster_kernel(const __grid_constant__ CUtensorMap tm_w,
                        const __grid_constant__ CUtensorMap tm_x, const Params p) {
  using L = Layout<BN, STAGES>;
  static_assert(BN * BM * 4 <= STAGES * L::STAGE_BYTES, "ring too small for the partial tile");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int tile = blockIdx.x;
  const int S = p.split;
  const int r = blockIdx.y;  // rank inside the cluster (cluster dims (1, S, 1))
  const int kb0 = (p.nkb * r) / S;
  const int kb1 = (p.nkb * (r + 1)) / S;
  const int n = kb1 - kb0;
  const int n_tile = tile_n(p, tile);
  const int t_tile = tile_t(p, tile);

  const uint32_t sbase = smem_u32(smem);
  const uint32_t bar_full = sbase + L::BAR_OFFSET;
  const uint32_t bar_empty = bar_full + STAGES * 8;
  const uint32_t bar_accf = bar_empty + STAGES * 8;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::MISC_OFFSET);
  int* misc = reinterpret_cast<int*>(smem + L::MISC_OFFSET + 16);  // [0] issued [1] consumed
  __nv_bfloat16* xch = reinterpret_cast<__nv_bfloat16*>(smem + L::XCH_OFFSET);
  float4* red = reinterpret_cast<float4*>(smem);  // [BN/4][BM] float4, reuses the ring

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(bar_full + 8 * s, 1);
      mbar_init(bar_empty + 8 * s, 1);
    }
    mbar_init(bar_accf, 1);
    misc[0] = 0;
    misc[1] = 0;
    fence_mbar_init();
    if (!PACKED) prefetch_tensormap(&tm_w);
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
  if (threadIdx.x == 0) griddep_launch_dependents();

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- producer ----------------
      const uint64_t pol_w = l2_policy_evict_first();
      const uint64_t pol_x = l2_policy_evict_last();
      auto load_w = [&](int kb, int s) {
        const uint32_t dst = sbase + s * L::STAGE_BYTES;
        if (PACKED) {
          bulk_load(dst, p.w_packed + ((size_t)n_tile * p.nkb + kb) * kTileBytes, kTileBytes,
                    bar_full + 8 * s, pol_w);
        } else {
          tma_load_2d_hint(dst, &tm_w, bar_full + 8 * s, kb * BK, n_tile * BM, pol_w);
        }
      };
      auto load_x = [&](int kb, int s) {
        tma_load_2d_hint(sbase + s * L::STAGE_BYTES + L::A_BYTES, &tm_x, bar_full + 8 * s, kb * BK,
                         t_tile * BN, pol_x);
      };
      const int pre = n < STAGES ? n : STAGES;
      for (int i = 0; i < pre; ++i) {  // weights first: independent of earlier kernels
        mbar_arrive_expect_tx(bar_full + 8 * i, L::STAGE_BYTES);
        load_w(kb0 + i, i);
      }
      griddep_wait();
      for (int i = 0; i < pre; ++i) load_x(kb0 + i, i);
      int issued = pre;
      for (int i = pre; i < n; ++i) {
        const int s = i % STAGES;
        const uint32_t ph = (uint32_t)(i / STAGES) & 1u;
        if (!mbar_wait(bar_empty + 8 * s, ph ^ 1u, 0x111)) break;
        mbar_arrive_expect_tx(bar_full + 8 * s, L::STAGE_BYTES);
        load_w(kb0 + i, s);
        load_x(kb0 + i, s);
        ++issued;
      }
      misc[0] = issued;
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer ----------------
      constexpr uint32_t idesc = idesc_bf16(BM, BN);
      for (int i = 0; i < n; ++i) {
        const int s = i % STAGES;
        const uint32_t ph = (uint32_t)(i / STAGES) & 1u;
        if (!mbar_wait(bar_full + 8 * s, ph, 0x112)) break;
        tc_fence_after();
        const uint32_t a_addr = sbase + s * L::STAGE_BYTES;
        const uint64_t adesc = sw128_kmajor_desc(a_addr);
        const uint64_t bdesc = sw128_kmajor_desc(a_addr + L::A_BYTES);
#pragma unroll
        for (int kk = 0; kk < BK / 16; ++kk)
          tc_mma(tmem, adesc + 2 * kk, bdesc + 2 * kk, idesc, (i > 0 || kk > 0) ? 1u : 0u);
        tc_commit(bar_empty + 8 * s);
        misc[1] = i + 1;
      }
      tc_commit(bar_accf);
    }
  } else {
    // ---------------- accumulator readers (warps 2..5) ----------------
    griddep_wait();
    const int q = warp & 3;
    const int row = q * 32 + lane;
    const bool acc_ok = mbar_wait(bar_accf, 0, 0x113);
    tc_fence_after();
    const uint32_t taddr = tmem + ((uint32_t)(q * 32) << 16);
    auto from_tmem = [&](int j0, float (&v)[16]) {
      tc_ld16(taddr + j0, v);
      if (!acc_ok) {
#pragma unroll
        for (int i = 0; i < 16; ++i) v[i] = 0.f;
      }
    };
    if (S == 1) {
      apply_epilogue<BN>(p, n_tile, t_tile, q, lane, xch, from_tmem);
    } else {
      // park the partial tile in this CTA's shared memory (the ring is idle:
      // every stage was consumed before the accumulator completed)
#pragma unroll 1
      for (int j0 = 0; j0 < BN; j0 += 16) {
        float v[16];
        from_tmem(j0, v);
#pragma unroll
        for (int i = 0; i < 4; ++i)
          red[((j0 >> 2) + i) * BM + row] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
      }
    }
  }

  // ---------------- drain + TMEM release ----------------
  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int i = misc[1]; i < misc[0]; ++i)
      mbar_wait(bar_full + 8 * (i % STAGES), (uint32_t)(i / STAGES) & 1u, 0x114);
  }
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(L::TMEM_COLS)
                 : "memory");
  }
  if (S == 1) {
    signal_done(p);
    return;
  }

  // ---------------- cluster reduction through distributed shared memory ----------------
  namespace cgx = cooperative_groups;
  cgx::cluster_group cluster = cgx::this_cluster();
  cluster.sync();  // every CTA's partial tile is in its shared memory
  const float4* peer[8];
#pragma unroll
  for (int c = 0; c < 8; ++c) peer[c] = c < S ? cluster.map_shared_rank(red, c) : red;
  const int tid = threadIdx.x;
  if (p.epilogue == FG_EPI_SWIGLU) {
    // features [f0, f1) of this tile: gate row f, up row f + 64
    const int f0 = (64 * r) / S, f1 = (64 * (r + 1)) / S, nf = f1 - f0;
    for (int e = tid; e < nf * (BN / 4); e += kThreads) {
      const int f = f0 + e % nf;
      const int j4 = e / nf;
      float4 g = make_float4(0.f, 0.f, 0.f, 0.f), u = g;
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        if (c < S) {
          const float4 a = peer[c][j4 * BM + f];
          const float4 b = peer[c][j4 * BM + f + 64];
          g.x += a.x; g.y += a.y; g.z += a.z; g.w += a.w;
          u.x += b.x; u.y += b.y; u.z += b.z; u.w += b.w;
        }
      }
      const float bg = p.bias ? bf2f(p.bias[n_tile * BM + f]) : 0.f;
      const float bu = p.bias ? bf2f(p.bias[n_tile * BM + f + 64]) : 0.f;
      const float gv[4] = {g.x, g.y, g.z, g.w}, uv[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int t = t_tile * BN + j4 * 4 + i;
        if (t < p.T) {
          const float gg = rbf(gv[i] + bg);
          const float uu = rbf(uv[i] + bu);
          p.out[(int64_t)t * p.ldo + n_tile * 64 + f] = f2bf(rbf(silu(gg)) * uu);
        }
      }
    }
  } else {
    const int r0 = (BM * r) / S, r1 = (BM * (r + 1)) / S, nr = r1 - r0;
    for (int e = tid; e < nr * (BN / 4); e += kThreads) {
      const int rr = r0 + e % nr;
      const int j4 = e / nr;
      const int nn = n_tile * BM + rr;
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        if (c < S) {
          const float4 a = peer[c][j4 * BM + rr];
          v.x += a.x; v.y += a.y; v.z += a.z; v.w += a.w;
        }
      }
      if (nn >= p.N) continue;
      const float b = p.bias ? bf2f(p.bias[nn]) : 0.f;
      const float vv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int t = t_tile * BN + j4 * 4 + i;
        if (t < p.T) {
          float y = vv[i] + b;
          if (p.epilogue == FG_EPI_F32) {
            if (p.residual) y += bf2f(p.residual[(int64_t)t * p.ldo + nn]);
            store_out<float>(p, t, nn, y);
            continue;
          }
          if (p.epilogue == FG_EPI_RESIDUAL) y = bf2f(p.residual[(int64_t)t * p.ldo + nn]) + rbf(y);
          store_out<__nv_bfloat16>(p, t, nn, f2bf(y));
        }
      }
    }
  }
  cluster.sync();  // peers may still read this CTA's partial tile
  signal_done(p);
}

// ---------------------------------------------------------------------------
// weight packing: [N,K] row-major -> [ceil(N/128)][ceil(K/64)][128 x 64] tiles,
// each the 128-byte-swizzled K-major image (16-byte chunk c of row r stored
// at chunk c ^ (r % 8)); padding rows / columns are zero.
// ---------------------------------------------------------------------------
__global__ void pack_weight_kernel(const uint4* __restrict__ w, uint4* __restrict__ packed, int N,
                                   int K, int nkb, long long chunks) {
  griddep_wait();
  const long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= chunks) return;
  const long long tile = idx >> 10;  // 1024 chunks of 16 B per tile
  const int within = (int)(idx & 1023);
  const int r = within >> 3;
  const int c = (within & 7) ^ (r & 7);
  const int nt = (int)(tile / nkb);
  const int kb = (int)(tile - (long long)nt * nkb);
  const int n = nt * BM + r;
  const int k = kb * BK + c * 8;
  uint4 v = make_uint4(0, 0, 0, 0);
  if (n < N && k < K) v = w[((long long)n * K + k) >> 3];
  packed[idx] = v;
}

inline int pick_bn(int T) {
  if (T <= 16) return 16;
  if (T <= 32) return 32;
  if (T <= 64) return 64;
  if (T <= 128) return 128;
  return 256;
}

constexpr int kMinSliceSteps = 4;  // fewest K steps (64 columns each) a split slice gets

struct Plan {
  int bn, n_tiles, t_tiles, nkb, grid, max_contrib, split;
  bool streamk;
  long long units;
};

inline int ctas_per_sm(int bn) { return bn >= 256 ? 1 : 2; }

// Clusters of s CTAs (1 x s x 1) of the cluster kernel for BN tokens that the
// current device keeps resident at once (cudaOccupancyMaxActiveClusters: it
// counts shared memory, TMEM-free occupancy and how clusters pack into the
// GPCs, which a CTA count alone does not); -1 if it cannot be asked.
template <int BN, int STAGES>
int query_active_clusters(int s) {
  using L = Layout<BN, STAGES>;
  auto kern = gemm_cluster_kernel<BN, STAGES, true>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::DYN_SMEM) != cudaSuccess) {
    (void)cudaGetLastError();
    return -1;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(1, s, 1);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = L::DYN_SMEM;
  cudaLaunchAttribute attr;
  attr.id = cudaLaunchAttributeClusterDimension;
  attr.val.clusterDim.x = 1;
  attr.val.clusterDim.y = s;
  attr.val.clusterDim.z = 1;
  cfg.attrs = &attr;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess) {
    (void)cudaGetLastError();
    return -1;
  }
  return n;
}

// Resident clusters for every (BN, split) of the decode plans on the current
// device, asked once per device; false without a device (the plan then falls
// back to counting CTAs).
inline bool active_clusters_table(int (*&table)[9]) {
  static std::mutex mu;
  static int cache[64][5][9];
  static bool done[64] = {false};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    (void)cudaGetLastError();
    return false;
  }
  std::lock_guard<std::mutex> lock(mu);
  if (!done[dev & 63]) {
    for (int sp = 1; sp <= 8; ++sp) {
      cache[dev & 63][0][sp] = query_active_clusters<16, 6>(sp);
      cache[dev & 63][1][sp] = query_active_clusters<32, 5>(sp);
      cache[dev & 63][2][sp] = query_active_clusters<64, 4>(sp);
      cache[dev & 63][3][sp] = query_active_clusters<128, 3>(sp);
      cache[dev & 63][4][sp] = query_active_clusters<256, 4>(sp);
      for (int b = 0; b < 5; ++b)
        if (cache[dev & 63][b][sp] < 1) return false;  // not known: ask again next time
    }
    done[dev & 63] = true;
  }
  table = cache[dev & 63];
  return true;
}

inline int bn_index(int bn) { return bn <= 16 ? 0 : bn <= 32 ? 1 : bn <= 64 ? 2 : bn <= 128 ? 3 : 4; }

// splits == 0: automatic (cluster kernel); > 0: cluster kernel with that many
// K slices per tile (capped at 8 and at K/64); < 0: persistent stream-K over
// -splits CTAs (the only mode that needs a workspace).
inline Plan make_plan(int T, int N, int K, int splits) {
  Plan pl;
  pl.bn = pick_bn(T);
  pl.n_tiles = (N + BM - 1) / BM;
  pl.t_tiles = (T + pl.bn - 1) / pl.bn;
  pl.nkb = (K + BK - 1) / BK;
  const long long tiles = (long long)pl.n_tiles * pl.t_tiles;
  pl.units = tiles * pl.nkb;
  const long long slots = (long long)num_sms() * ctas_per_sm(pl.bn);
  pl.streamk = false;
  pl.split = 1;
  pl.max_contrib = 1;
  if (splits == 0 && pl.t_tiles >= 2 && tiles >= slots) {
    // many tokens (prefill): a persistent grid walking whole tiles, so each
    // CTA's epilogue overlaps its next tile's MMAs (two accumulators) and the
    // per-tile prologue is paid once per CTA; the grid divides the tiles
    // exactly, so no tile is split and no workspace is needed. Below two
    // waves of tiles the grid must still cover most SMs.
    const long long g_min = tiles >= 2 * slots ? slots / 2 : (slots * 4) / 5;
    for (long long g = slots; g >= g_min; --g) {
      if (tiles % g == 0) {
        splits = (int)-g;
        break;
      }
    }
  }
  if (splits < 0) {
    pl.streamk = true;
    pl.grid = (int)(-splits < pl.units ? -splits : pl.units);
  } else if (splits > 0) {
    pl.split = splits;
  } else {
    // as many K slices per tile (at least kMinSliceSteps K steps each) as
    // keep every tile's cluster resident in one wave: more CTAs stream the
    // weights at once, and a second wave of clusters costs more than the
    // slices save (measured on B200 over every split of the decode shapes of
    // Llama-3-8B and gpt-oss-20b, T = 32-256). One CTA per SM (BN >= 128):
    // the device's own count of resident clusters per size. Two per SM: about
    // 82% of the CTA slots, where clusters still packed into the GPCs in one
    // wave (5 x 48 = 240 CTAs did, 6 x 48 = 288 did not).
    const int max_split = pl.nkb / kMinSliceSteps < 8 ? pl.nkb / kMinSliceSteps : 8;
    int (*table)[9] = nullptr;
    if (pl.bn >= 128 && active_clusters_table(table)) {
      const int* active = table[bn_index(pl.bn)];
      for (int sp = 1; sp <= max_split; ++sp)
        if (tiles <= active[sp]) pl.split = sp;
    } else {
      const long long fit = (slots * 41) / (50 * tiles);
      pl.split = (int)(fit < max_split ? fit : max_split);
    }
  }
  if (!pl.streamk) {
    if (pl.split > 8) pl.split = 8;
    if (pl.split > pl.nkb) pl.split = pl.nkb;
    if (pl.split < 1) pl.split = 1;
    pl.grid = (int)tiles;
  } else {
    if (pl.grid < 1) pl.grid = 1;
    const long long per = pl.units / pl.grid;  // shortest unit range of a CTA
    pl.max_contrib = (int)((pl.nkb + per - 1) / per + 1);
    if (pl.max_contrib > pl.grid) pl.max_contrib = pl.grid;
  }
  return pl;
}

inline size_t workspace_bytes(const Plan& pl) {
  if (!pl.streamk) return 0;
  const long long tiles = (long long)pl.n_tiles * pl.t_tiles;
  const bool any_split = pl.grid > tiles || (pl.units % pl.grid) != 0 || (pl.units / pl.grid) % pl.nkb != 0;
  if (!any_split) return 0;  // every CTA owns whole tiles
  return kTicketBytes + (size_t)tiles * pl.max_contrib * pl.bn * BM * sizeof(float);
}

template <int BN, int STAGES, bool PACKED>
int launch(const Params& p, const CUtensorMap& tw, const CUtensorMap& tx, cudaStream_t st,
           bool streamk) {
  using L = Layout<BN, STAGES>;
  auto ksk = gemm_bf16_kernel<BN, STAGES, PACKED>;
  auto kcl = gemm_cluster_kernel<BN, STAGES, PACKED>;
  static bool attr_done[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!attr_done[dev & 63]) {
    cudaError_t e = cudaFuncSetAttribute(ksk, cudaFuncAttributeMaxDynamicSharedMemorySize, L::DYN_SMEM);
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(kcl, cudaFuncAttributeMaxDynamicSharedMemorySize, L::DYN_SMEM);
    if (e != cudaSuccess) {
      set_last_error("fg_gemm_bf16: cudaFuncSetAttribute: %s", cudaGetErrorString(e));
      return FG_ERR_CUDA;
    }
    attr_done[dev & 63] = true;
  }
  if (streamk)
    return launch_k("fg_gemm_bf16", ksk, dim3(p.grid), dim3(kThreads), L::DYN_SMEM, st, tw, tx, p);
  return launch_kc("fg_gemm_bf16", kcl, dim3(p.grid, p.split), dim3(1, p.split, 1), dim3(kThreads),
                   L::DYN_SMEM, st, tw, tx, p);
}

// Routing and completion signal of fg_gemm_bf16_packed_routed (none for the
// plain entry points).
struct Route {
  int route = 0, n_dst = 0, dst_rows = 0, dst_row0 = 0;
  void* const* dst = nullptr;
  int n_sig = 0;
  uint32_t* const* sig = nullptr;
  const uint32_t* epoch = nullptr;
  uint32_t seq_mul = 0, seq_add = 0;
  uint32_t* ticket = nullptr;
};

template <bool PACKED>
int run(const fg_bf16* x, const void* w, fg_bf16* out, const fg_bf16* residual, const fg_bf16* bias,
        int T, int N, int K, int epilogue, int splits, void* workspace, size_t workspace_bytes_,
        cudaStream_t st, const Route& rt = Route()) {
  const Plan pl = make_plan(T, N, K, splits);
  Params p;
  memset(&p, 0, sizeof(p));
  p.out = reinterpret_cast<__nv_bfloat16*>(out);
  p.residual = reinterpret_cast<const __nv_bfloat16*>(residual);
  p.bias = reinterpret_cast<const __nv_bfloat16*>(bias);
  p.w_packed = PACKED ? reinterpret_cast<const uint8_t*>(w) : nullptr;
  p.T = T;
  p.N = N;
  p.K = K;
  p.ldo = epilogue == FG_EPI_SWIGLU ? N / 2 : N;
  p.epilogue = epilogue;
  p.n_tiles = pl.n_tiles;
  p.t_tiles = pl.t_tiles;
  p.nkb = pl.nkb;
  p.units = pl.units;
  p.grid = pl.grid;
  p.max_contrib = pl.max_contrib;
  p.split = pl.split;
  p.partial = nullptr;
  p.tickets = nullptr;
  p.route = rt.route;
  p.n_dst = rt.n_dst;
  p.dst_rows = rt.dst_rows;
  p.dst_row0 = rt.dst_row0;
  for (int i = 0; i < rt.n_dst; ++i) p.dst[i] = rt.dst[i];
  p.n_sig = rt.n_sig;
  for (int i = 0; i < rt.n_sig; ++i) p.sig[i] = rt.sig[i];
  p.epoch = rt.epoch;
  p.seq_mul = rt.seq_mul;
  p.seq_add = rt.seq_add;
  p.sig_ticket = rt.ticket;
  p.total_ctas = pl.grid * pl.split;
  if (rt.route != 0 || rt.n_sig != 0) {
    FG_REQUIRE(!pl.streamk, "fg_gemm_bf16_packed_routed: T=%d N=%d K=%d plans the persistent kernel; "
               "routed output and signals need a decode-size plan", T, N, K);
  }
  const size_t need = workspace_bytes(pl);
  if (need) {
    const long long tiles = (long long)pl.n_tiles * pl.t_tiles;
    FG_REQUIRE(tiles <= kMaxTickets, "fg_gemm_bf16: %lld tiles exceed the %d split tickets", tiles,
               kMaxTickets);
    FG_REQUIRE(workspace != nullptr && workspace_bytes_ >= need,
               "fg_gemm_bf16: needs %zu workspace bytes, got %zu", need, workspace_bytes_);
    FG_REQUIRE(((uintptr_t)workspace & 255) == 0, "fg_gemm_bf16: workspace must be 256-byte aligned");
    p.tickets = reinterpret_cast<unsigned int*>(workspace);
    p.partial = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(workspace) + kTicketBytes);
  }
  CUtensorMap tw, tx;
  memset(&tw, 0, sizeof(tw));
  int rc;
  if (!PACKED) {
    rc = make_tmap_2d_bf16(&tw, w, (uint64_t)K, (uint64_t)N, (uint64_t)K * 2, BK, BM,
                           CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
  }
  rc = make_tmap_2d_bf16(&tx, x, (uint64_t)K, (uint64_t)T, (uint64_t)K * 2, BK, pl.bn,
                         CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  switch (pl.bn) {
    case 16: return launch<16, 6, PACKED>(p, tw, tx, st, pl.streamk);
    case 32: return launch<32, 5, PACKED>(p, tw, tx, st, pl.streamk);
    case 64: return launch<64, 4, PACKED>(p, tw, tx, st, pl.streamk);
    case 128: return launch<128, 3, PACKED>(p, tw, tx, st, pl.streamk);
    default: return launch<256, 4, PACKED>(p, tw, tx, st, pl.streamk);
  }
}

}  // namespace gemm
}  // namespace fg

extern "C" {

int fg_gemm_grid(int T, int N, int K, int splits) {
  if (T <= 0 || N <= 0 || K <= 0) return 0;
  return fg::gemm::make_plan(T, N, K, splits).grid;
}

int fg_gemm_split(int T, int N, int K, int splits) {
  if (T <= 0 || N <= 0 || K <= 0) return 0;
  const fg::gemm::Plan pl = fg::gemm::make_plan(T, N, K, splits);
  return pl.streamk ? 1 : pl.split;
}

size_t fg_gemm_workspace_bytes(int T, int N, int K, int splits) {
  if (T <= 0 || N <= 0 || K <= 0) return 0;
  return fg::gemm::workspace_bytes(fg::gemm::make_plan(T, N, K, splits));
}

size_t fg_packed_weight_bytes(int N, int K) {
  if (N <= 0 || K <= 0) return 0;
  return (size_t)((N + fg::gemm::BM - 1) / fg::gemm::BM) * ((K + fg::gemm::BK - 1) / fg::gemm::BK) *
         fg::gemm::kTileBytes;
}

int fg_pack_weight_bf16(const fg_bf16* w, void* packed, int N, int K, fg_stream_t stream) {
  FG_REQUIRE(w && packed, "fg_pack_weight_bf16: null pointer");
  FG_REQUIRE(N > 0 && K > 0 && K % 8 == 0, "fg_pack_weight_bf16: bad sizes N=%d K=%d", N, K);
  FG_REQUIRE((((uintptr_t)w | (uintptr_t)packed) & 15) == 0,
             "fg_pack_weight_bf16: pointers must be 16-byte aligned");
  const int nkb = (K + fg::gemm::BK - 1) / fg::gemm::BK;
  const long long chunks = (long long)fg_packed_weight_bytes(N, K) / 16;
  int (*active)[9] = nullptr;  // ask the device for the GEMM plans now, before any stream capture
  (void)fg::gemm::active_clusters_table(active);
  const int threads = 256;
  return fg::launch_k("fg_pack_weight_bf16", fg::gemm::pack_weight_kernel,
                      dim3((unsigned)((chunks + threads - 1) / threads)), dim3(threads), 0,
                      (cudaStream_t)stream, reinterpret_cast<const uint4*>(w),
                      reinterpret_cast<uint4*>(packed), N, K, nkb, chunks);
}

static int gemm_checks(const fg_bf16* x, const void* w, fg_bf16* out, const fg_bf16* residual,
                       int T, int N, int K, int epilogue) {
  using namespace fg::gemm;
  FG_REQUIRE(x && w && out, "fg_gemm_bf16: null pointer");
  FG_REQUIRE(T >= 0 && N > 0 && K > 0 && K % 8 == 0, "fg_gemm_bf16: bad sizes T=%d N=%d K=%d", T,
             N, K);
  FG_REQUIRE(epilogue == FG_EPI_STORE || epilogue == FG_EPI_RESIDUAL || epilogue == FG_EPI_SWIGLU ||
                 epilogue == FG_EPI_F32,
             "fg_gemm_bf16: bad epilogue %d", epilogue);
  FG_REQUIRE(epilogue != FG_EPI_RESIDUAL || residual != nullptr,
             "fg_gemm_bf16: residual epilogue needs a residual");
  FG_REQUIRE(epilogue != FG_EPI_SWIGLU || N % BM == 0,
             "fg_gemm_bf16: SwiGLU needs N (=2*I) to be a multiple of 128, got %d", N);
  FG_REQUIRE((((uintptr_t)x | (uintptr_t)w) & 15) == 0, "fg_gemm_bf16: x/w must be 16-byte aligned");
  return FG_OK;
}

int fg_gemm_bf16(const fg_bf16* x, const fg_bf16* w, fg_bf16* out, const fg_bf16* residual,
                 const fg_bf16* bias, int T, int N, int K, int epilogue, int splits,
                 void* workspace, size_t workspace_bytes, fg_stream_t stream) {
  int rc = gemm_checks(x, w, out, residual, T, N, K, epilogue);
  if (rc || T == 0) return rc;
  return fg::gemm::run<false>(x, w, out, residual, bias, T, N, K, epilogue, splits, workspace,
                              workspace_bytes, (cudaStream_t)stream);
}

int fg_gemm_bf16_packed(const fg_bf16* x, const void* w_packed, fg_bf16* out,
                        const fg_bf16* residual, const fg_bf16* bias, int T, int N, int K,
                        int epilogue, int splits, void* workspace, size_t workspace_bytes,
                        fg_stream_t stream) {
  int rc = gemm_checks(x, w_packed, out, residual, T, N, K, epilogue);
  if (rc || T == 0) return rc;
  return fg::gemm::run<true>(x, w_packed, out, residual, bias, T, N, K, epilogue, splits,
                             workspace, workspace_bytes, (cudaStream_t)stream);
}

int fg_gemm_bf16_packed_routed(const fg_bf16* x, const void* w_packed, const fg_bf16* residual,
                               const fg_bf16* bias, int T, int N, int K, int epilogue, int route,
                               void* const* dst, int n_dst, int dst_rows, int dst_row0,
                               uint32_t* const* sig_flags, int n_sig, const uint32_t* epoch,
                               uint32_t seq_mul, uint32_t seq_add, uint32_t* ticket,
                               fg_stream_t stream) {
  using fg::gemm::kMaxRoutes;
  FG_REQUIRE(route == FG_ROUTE_SPLIT || route == FG_ROUTE_BROADCAST,
             "fg_gemm_bf16_packed_routed: route must be FG_ROUTE_SPLIT or FG_ROUTE_BROADCAST");
  FG_REQUIRE(epilogue == FG_EPI_STORE || epilogue == FG_EPI_RESIDUAL || epilogue == FG_EPI_F32,
             "fg_gemm_bf16_packed_routed: epilogue %d cannot be routed (STORE, RESIDUAL or F32)", epilogue);
  FG_REQUIRE(dst && n_dst >= 1 && n_dst <= kMaxRoutes, "fg_gemm_bf16_packed_routed: n_dst=%d (1..%d)",
             n_dst, kMaxRoutes);
  for (int i = 0; i < n_dst; ++i) FG_REQUIRE(dst[i] != nullptr, "fg_gemm_bf16_packed_routed: dst[%d] is null", i);
  FG_REQUIRE(route != FG_ROUTE_SPLIT || (dst_rows > 0 && (long long)dst_rows * n_dst >= T),
             "fg_gemm_bf16_packed_routed: %d destinations of %d rows cannot take %d rows", n_dst, dst_rows, T);
  FG_REQUIRE(route != FG_ROUTE_BROADCAST || dst_row0 >= 0, "fg_gemm_bf16_packed_routed: dst_row0 < 0");
  FG_REQUIRE(n_sig >= 0 && n_sig <= kMaxRoutes, "fg_gemm_bf16_packed_routed: n_sig=%d (0..%d)", n_sig,
             kMaxRoutes);
  FG_REQUIRE(n_sig == 0 || (sig_flags && epoch && ticket),
             "fg_gemm_bf16_packed_routed: signalling needs flags, an epoch and a ticket");
  for (int i = 0; i < n_sig; ++i)
    FG_REQUIRE(sig_flags[i] != nullptr, "fg_gemm_bf16_packed_routed: sig_flags[%d] is null", i);
  FG_REQUIRE(residual != nullptr || epilogue != FG_EPI_RESIDUAL,
             "fg_gemm_bf16_packed_routed: FG_EPI_RESIDUAL needs a residual");
  fg::gemm::Route rt;
  rt.route = route;
  rt.n_dst = n_dst;
  rt.dst = dst;
  rt.dst_rows = dst_rows;
  rt.dst_row0 = dst_row0;
  rt.n_sig = n_sig;
  rt.sig = sig_flags;
  rt.epoch = epoch;
  rt.seq_mul = seq_mul;
  rt.seq_add = seq_add;
  rt.ticket = ticket;
  return fg::gemm::run<true>(x, w_packed, nullptr, residual, bias, T, N, K, epilogue, 0, nullptr, 0,
                             (cudaStream_t)stream, rt);
}

}  // extern "C"
