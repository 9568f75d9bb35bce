// Paged GQA decode attention (one query token per sequence), HBM-bound.
//
// KV layout in HBM, per layer: k_cache / v_cache [num_blocks][nkv][16][hd]
// bf16, so one page of one KV head (16 tokens x hd) is a contiguous
// 2 KB (hd=64) or 4 KB (hd=128) run. The block table maps
// (sequence, page) -> physical block, like vLLM's paged cache.
//
// CTA = (split, kv head g, sequence b); 5 warps:
//   warp 4 (lane 0): producer. TMA-loads each page's K and V tiles
//                    (box 64 dims x 16 tokens, 128-byte swizzle, plain
//                    non-cluster copies) into a STAGES-deep shared ring,
//                    completion tracked by mbarrier transaction counts.
//   warps 0-3      : consumers, page i handled by warp i % 4. Per page:
//                    S[16 x 16] = Q K^T with the G = nq/nkv query heads of the
//                    group as the MMA rows (m16n8k16 bf16, fp32 accumulate,
//                    operands fetched from the swizzled ring by ldmatrix),
//                    online softmax in exp2 domain with quad warp shuffles,
//                    O[16 x hd] += P V (V fetched with ldmatrix.trans).
// The four warps' (m, l, O) are merged in shared memory. With one split per
// sequence the CTA writes the normalised output (sinks applied); otherwise it
// writes fp32 partials that fg_attn_combine merges.
//
// Window: only tokens kv >= L - window take part (transformers' sliding mask
// keeps kv > q - window with q = L - 1); pages outside are never loaded.
// Sinks (gpt-oss): exp(sink_h) joins head h's softmax denominator only.
#pragma once
#include "common.cuh"

namespace fg {
namespace attn {

constexpr int kBlock = 16;     // tokens per page
constexpr int kConsumers = 4;  // consumer warps
constexpr int kThreads = (kConsumers + 1) * 32;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kNegBig = -1.0e30f;
constexpr int kMinSlice = 8;   // fewest pages a split slice is given
constexpr int kMaxSplits = 128;  // most slices plan_splits gives one (sequence, kv head)
constexpr int kCombineThreads = 512;  // a multiple of every supported head dim
constexpr int kSerialSplits = 8;      // up to this many, the combine walks splits in order

struct Params {
  const __nv_bfloat16* q;   // [B][nq][hd]
  const int32_t* block_table;
  const int32_t* seq_lens;
  const float* sinks;       // [nq] or null
  __nv_bfloat16* out;       // [B][nq*hd]
  float* part_o;            // [B][nq][splits][hd]
  float* part_ml;           // [B][nq][splits][2]
  int B, nq, nkv, G;
  int max_blocks, num_blocks;
  int splits;               // slices per (sequence, kv head)
  int window;
  float scale_log2;         // softmax scale * log2(e)
};

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void mma_bf16(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                         uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// address of 16-byte chunk `chunk` (0 .. HD/8-1) of token row `tok` inside a
// page tile made of HD/64 boxes of [16 rows][128 bytes], 128-byte swizzle
__device__ __forceinline__ uint32_t tile_addr(uint32_t base, int tok, int chunk) {
  const int box = chunk >> 3, c = chunk & 7;
  return base + box * 2048 + tok * 128 + ((c ^ (tok & 7)) << 4);
}

template <int HD, int STAGES>
struct Layout {
  static constexpr int BOXES = HD / 64;
  static constexpr int TILE_BYTES = BOXES * 2048;     // one page of K (or V)
  static constexpr int STAGE_BYTES = 2 * TILE_BYTES;  // K + V
  static constexpr int BAR_OFFSET = STAGES * STAGE_BYTES;
  static constexpr int TOTAL = BAR_OFFSET + 2 * STAGES * 8;
  static constexpr int DYN_SMEM = TOTAL + 1024;
  // merge scratch (reuses the ring): O [4][16][HD] + m,l [4][16]
  static_assert(kConsumers * 16 * HD * 4 + kConsumers * 16 * 2 * 4 <= BAR_OFFSET,
                "ring too small for the merge scratch");
};

template <int HD, int STAGES>
// four resident CTAs per SM at hd 64 (96 registers): a 2 KB page per K or V
// tile leaves a CTA with half the bytes per page step of hd 128, so more CTAs
// keep the same bytes in flight; hd 128 fits three (128 registers)
__global__ void __launch_bounds__(kThreads, HD == 64 ? 4 : 3) paged_attn_kernel(
    const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_v,
    const Params p) {
  using L = Layout<HD, STAGES>;
  constexpr int KT = HD / 16;  // k-steps for Q K^T and dim pairs for P V
  constexpr int ND = HD / 8;   // n-tiles of O
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int split = blockIdx.x, g = blockIdx.y, b = blockIdx.z;
  const int G = p.G;
  griddep_wait();  // q, the new token's KV and seq_lens come from earlier kernels
  if (threadIdx.x == 0) griddep_launch_dependents();

  const int Lq = p.seq_lens[b];
  const int lo = p.window > 0 ? max(0, Lq - p.window) : 0;
  const int pbeg = lo / kBlock, pend = (Lq + kBlock - 1) / kBlock;
  // this sequence's pages split evenly over its active slices (>= kMinSlice
  // pages each), from its actual length: a plan made for a longer bucket
  // still gives every CTA of the sequence the same share
  const int P = max(pend - pbeg, 0);
  const int active = min(p.splits, max(1, (P + kMinSlice - 1) / kMinSlice));
  const int my0 = split < active ? pbeg + (int)((int64_t)split * P / active) : pend;
  const int my1 = split < active ? pbeg + (int)((int64_t)(split + 1) * P / active) : pend;
  const int npages = my1 - my0;

  if (npages <= 0) {
    if (p.splits > 1) {
      // empty slice: an all-masked partial for the combine step
      if (threadIdx.x < G) {
        const int64_t hi = ((int64_t)b * p.nq + g * G + threadIdx.x) * p.splits + split;
        p.part_ml[2 * hi] = kNegBig;
        p.part_ml[2 * hi + 1] = 0.f;
      }
    } else {
      // nothing to attend (seq_len 0): zero output
      for (int e = threadIdx.x; e < G * HD; e += blockDim.x)
        p.out[((int64_t)b * p.nq + g * G) * HD + e] = f2bf(0.f);
    }
    return;
  }

  const uint32_t sbase = smem_u32(smem);
  const uint32_t bar_full = sbase + L::BAR_OFFSET;
  const uint32_t bar_empty = bar_full + STAGES * 8;
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(bar_full + 8 * s, 1);
      mbar_init(bar_empty + 8 * s, 1);
    }
    fence_mbar_init();
    prefetch_tensormap(&tm_k);
    prefetch_tensormap(&tm_v);
  }
  __syncthreads();

  if (warp == kConsumers) {
    // ---------------- producer ----------------
    if (lane == 0) {
      const int32_t* bt = p.block_table + (int64_t)b * p.max_blocks;
      const uint64_t pol = l2_policy_evict_first();
      int issued = 0;
      for (int i = 0; i < npages; ++i) {
        const int s = i % STAGES;
        const uint32_t ph = (uint32_t)(i / STAGES) & 1u;
        if (!mbar_wait(bar_empty + 8 * s, ph ^ 1u, 0x201)) break;
        const int page = my0 + i;
        int blk = page < p.max_blocks ? bt[page] : -1;
        if (blk < 0 || blk >= p.num_blocks) {
          record_device_error(DEV_BAD_INDEX, 0x202);
          blk = 0;  // keep the pipeline whole; the result is flagged invalid
        }
        const int row = (blk * p.nkv + g) * kBlock;
        const uint32_t st = sbase + s * L::STAGE_BYTES;
        mbar_arrive_expect_tx(bar_full + 8 * s, L::STAGE_BYTES);
#pragma unroll
        for (int bx = 0; bx < L::BOXES; ++bx) {
          tma_load_2d_hint(st + bx * 2048, &tm_k, bar_full + 8 * s, bx * 64, row, pol);
          tma_load_2d_hint(st + L::TILE_BYTES + bx * 2048, &tm_v, bar_full + 8 * s, bx * 64, row,
                           pol);
        }
        ++issued;
      }
      if (issued < npages) {
        // a consumer gave up: let every copy already issued land before the
        // CTA (and its shared memory) goes away
        for (int s = 0; s < STAGES && s < issued; ++s) {
          const int last = s + ((issued - 1 - s) / STAGES) * STAGES;
          mbar_wait(bar_full + 8 * s, (uint32_t)(last / STAGES) & 1u, 0x204);
        }
      }
    }
  } else {
    // ---------------- consumers ----------------
    // Q fragments (A operand, rows = heads of this group, zero beyond G)
    uint32_t qf[KT][4];
    {
      const int r0 = lane >> 2, r1 = r0 + 8;
      const int c = (lane & 3) * 2;
      const uint32_t* q0 = reinterpret_cast<const uint32_t*>(
          p.q + ((int64_t)b * p.nq + g * G + r0) * HD);
      const uint32_t* q1 = reinterpret_cast<const uint32_t*>(
          p.q + ((int64_t)b * p.nq + g * G + r1) * HD);
#pragma unroll
      for (int kt = 0; kt < KT; ++kt) {
        qf[kt][0] = r0 < G ? q0[(kt * 16 + c) >> 1] : 0u;
        qf[kt][1] = r1 < G ? q1[(kt * 16 + c) >> 1] : 0u;
        qf[kt][2] = r0 < G ? q0[(kt * 16 + 8 + c) >> 1] : 0u;
        qf[kt][3] = r1 < G ? q1[(kt * 16 + 8 + c) >> 1] : 0u;
      }
    }
    float o[ND][4];
#pragma unroll
    for (int i = 0; i < ND; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
    float m0 = kNegBig, m1 = kNegBig, l0 = 0.f, l1 = 0.f;

    // per-lane ldmatrix row/chunk selectors
    const int k_tok = ((lane >> 4) << 3) + (lane & 7);  // Q K^T: tokens 0-7 | 8-15
    const int k_sub = (lane >> 3) & 1;                  // low / high 8 dims of the k-step
    const int v_tok = (((lane >> 3) & 1) << 3) + (lane & 7);
    const int v_sub = lane >> 4;

    for (int i = warp; i < npages; i += kConsumers) {
      const int s = i % STAGES;
      const uint32_t ph = (uint32_t)(i / STAGES) & 1u;
      // warp-uniform decision: ldmatrix / mma below need the whole warp
      if (!__all_sync(0xffffffffu, mbar_wait(bar_full + 8 * s, ph, 0x203))) break;
      const uint32_t kbase = sbase + s * L::STAGE_BYTES;
      const uint32_t vbase = kbase + L::TILE_BYTES;
      float sc[2][4];
#pragma unroll
      for (int n = 0; n < 2; ++n) sc[n][0] = sc[n][1] = sc[n][2] = sc[n][3] = 0.f;
#pragma unroll
      for (int kt = 0; kt < KT; ++kt) {
        uint32_t kb[4];
        ldsm_x4(kb, tile_addr(kbase, k_tok, kt * 2 + k_sub));
        mma_bf16(sc[0], qf[kt], kb[0], kb[1]);
        mma_bf16(sc[1], qf[kt], kb[2], kb[3]);
      }
      // scale, mask, online softmax (rows r0 = lane/4 and r1 = lane/4 + 8)
      const int tok0 = (my0 + i) * kBlock + (lane & 3) * 2;
      float mx0 = kNegBig, mx1 = kNegBig;
#pragma unroll
      for (int n = 0; n < 2; ++n) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int t = tok0 + n * 8 + (e & 1);
          const bool valid = t >= lo && t < Lq;
          sc[n][e] = valid ? sc[n][e] * p.scale_log2 : kNegBig;
        }
        mx0 = fmaxf(mx0, fmaxf(sc[n][0], sc[n][1]));
        mx1 = fmaxf(mx1, fmaxf(sc[n][2], sc[n][3]));
      }
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
      const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
      const float a0 = exp2f(m0 - mn0), a1 = exp2f(m1 - mn1);
      m0 = mn0;
      m1 = mn1;
      float ps[2][4];
#pragma unroll
      for (int n = 0; n < 2; ++n) {
        ps[n][0] = exp2f(sc[n][0] - mn0);
        ps[n][1] = exp2f(sc[n][1] - mn0);
        ps[n][2] = exp2f(sc[n][2] - mn1);
        ps[n][3] = exp2f(sc[n][3] - mn1);
      }
      l0 = l0 * a0 + ps[0][0] + ps[0][1] + ps[1][0] + ps[1][1];
      l1 = l1 * a1 + ps[0][2] + ps[0][3] + ps[1][2] + ps[1][3];
#pragma unroll
      for (int nd = 0; nd < ND; ++nd) {
        o[nd][0] *= a0;
        o[nd][1] *= a0;
        o[nd][2] *= a1;
        o[nd][3] *= a1;
      }
      uint32_t pa[4];
      pa[0] = pack_bf16x2(ps[0][0], ps[0][1]);
      pa[1] = pack_bf16x2(ps[0][2], ps[0][3]);
      pa[2] = pack_bf16x2(ps[1][0], ps[1][1]);
      pa[3] = pack_bf16x2(ps[1][2], ps[1][3]);
#pragma unroll
      for (int c2 = 0; c2 < KT; ++c2) {
        uint32_t vb[4];
        ldsm_x4_t(vb, tile_addr(vbase, v_tok, c2 * 2 + v_sub));
        mma_bf16(o[2 * c2], pa, vb[0], vb[1]);
        mma_bf16(o[2 * c2 + 1], pa, vb[2], vb[3]);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(bar_empty + 8 * s);
    }
    // row sums: reduce the quad
    l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
    l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
    l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
    l1 += __shfl_xor_sync(0xffffffffu, l1, 2);

    // ---------------- merge the 4 consumer warps ----------------
    asm volatile("bar.sync 1, %0;" ::"n"(kConsumers * 32) : "memory");  // ring is idle now
    float* so = reinterpret_cast<float*>(smem);              // [4][16][HD]
    float* sml = so + kConsumers * 16 * HD;                  // [4][16][2]
    {
      const int r0 = lane >> 2, r1 = r0 + 8, c = (lane & 3) * 2;
      float* ow = so + warp * 16 * HD;
#pragma unroll
      for (int nd = 0; nd < ND; ++nd) {
        if (r0 < G) {
          ow[r0 * HD + nd * 8 + c] = o[nd][0];
          ow[r0 * HD + nd * 8 + c + 1] = o[nd][1];
        }
        if (r1 < G) {
          ow[r1 * HD + nd * 8 + c] = o[nd][2];
          ow[r1 * HD + nd * 8 + c + 1] = o[nd][3];
        }
      }
      if ((lane & 3) == 0) {
        sml[(warp * 16 + r0) * 2] = m0;
        sml[(warp * 16 + r0) * 2 + 1] = l0;
        sml[(warp * 16 + r1) * 2] = m1;
        sml[(warp * 16 + r1) * 2 + 1] = l1;
      }
    }
    asm volatile("bar.sync 1, %0;" ::"n"(kConsumers * 32) : "memory");
    for (int e = threadIdx.x; e < G * HD; e += kConsumers * 32) {
      const int h = e / HD, d = e - h * HD;
      float M = kNegBig;
#pragma unroll
      for (int w = 0; w < kConsumers; ++w) M = fmaxf(M, sml[(w * 16 + h) * 2]);
      float lsum = 0.f, osum = 0.f;
#pragma unroll
      for (int w = 0; w < kConsumers; ++w) {
        const float f = exp2f(sml[(w * 16 + h) * 2] - M);
        lsum += sml[(w * 16 + h) * 2 + 1] * f;
        osum += so[(w * 16 + h) * HD + d] * f;
      }
      const int hg = g * G + h;
      if (p.splits == 1) {
        const float sink = p.sinks ? exp2f(p.sinks[hg] * kLog2e - M) : 0.f;
        p.out[((int64_t)b * p.nq + hg) * HD + d] = f2bf(osum / (lsum + sink));
      } else {
        const int64_t hi = ((int64_t)b * p.nq + hg) * p.splits + split;
        p.part_o[hi * HD + d] = osum;
        if (d == 0) {
          p.part_ml[2 * hi] = M;
          p.part_ml[2 * hi + 1] = lsum;
        }
      }
    }
  }
}

// block-wide max (kMax) or sum of one float per thread; every thread gets the
// same value, combined in one fixed order
template <bool kMax>
__device__ __forceinline__ float block_reduce(float v, float* red) {
#pragma unroll
  for (int o = 16; o; o >>= 1) {
    const float w = __shfl_xor_sync(0xffffffffu, v, o);
    v = kMax ? fmaxf(v, w) : v + w;
  }
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float r = red[0];
  for (int i = 1; i < (int)(blockDim.x >> 5); ++i) r = kMax ? fmaxf(r, red[i]) : r + red[i];
  __syncthreads();  // red is reused by the next call
  return r;
}

// merge split partials: grid (nq, B), block a multiple of hd that covers every
// split (at most kCombineThreads). Up to kSerialSplits splits, one group of hd
// threads each walks the splits in order. Beyond that, thread s reads split s's
// running max and denominator (two block reductions give the global max and
// the rescaled denominator) and the weighted partial outputs are summed by
// blockDim / hd groups of hd threads over interleaved splits, so no thread
// walks all splits one dependent load at a time; the groups are added in index
// order (the result does not depend on timing)
__global__ void __launch_bounds__(kCombineThreads) attn_combine_kernel(const Params p, int hd) {
  __shared__ float s_f[kMaxSplits];
  __shared__ float s_red[kCombineThreads / 32];
  __shared__ float s_o[kCombineThreads];
  griddep_wait();
  griddep_launch_dependents();
  const int h = blockIdx.x, b = blockIdx.y, t = threadIdx.x;
  const int S = p.splits;
  const int64_t base = ((int64_t)b * p.nq + h) * S;
  const float* ml = p.part_ml + 2 * base;
  if (S <= kSerialSplits) {
    float M = kNegBig;
    for (int s = 0; s < S; ++s) M = fmaxf(M, ml[2 * s]);
    float lsum = p.sinks ? exp2f(p.sinks[h] * kLog2e - M) : 0.f;
    float osum = 0.f;
    for (int s = 0; s < S; ++s) {
      const float m = ml[2 * s];
      if (m <= kNegBig) continue;  // empty slice
      const float f = exp2f(m - M);
      lsum += ml[2 * s + 1] * f;
      osum += p.part_o[(base + s) * hd + t] * f;
    }
    p.out[((int64_t)b * p.nq + h) * hd + t] = f2bf(lsum > 0.f ? osum / lsum : 0.f);
    return;
  }
  const float m = t < S ? ml[2 * t] : kNegBig;
  const float l = t < S ? ml[2 * t + 1] : 0.f;
  const float M = block_reduce<true>(m, s_red);
  const float f = m <= kNegBig ? 0.f : exp2f(m - M);  // empty slices carry nothing
  float lsum = block_reduce<false>(l * f, s_red);
  if (p.sinks) lsum += exp2f(p.sinks[h] * kLog2e - M);
  if (t < S) s_f[t] = f;
  __syncthreads();
  const int d = t % hd, grp = t / hd, ngrp = (int)blockDim.x / hd;
  float o = 0.f;
#pragma unroll 4
  for (int s = grp; s < S; s += ngrp) {
    const float fs = s_f[s];
    if (fs != 0.f) o += p.part_o[(base + s) * hd + d] * fs;
  }
  s_o[t] = o;
  __syncthreads();
  if (grp == 0) {
    float acc = 0.f;
    for (int g2 = 0; g2 < ngrp; ++g2) acc += s_o[g2 * hd + d];
    p.out[((int64_t)b * p.nq + h) * hd + d] = f2bf(lsum > 0.f ? acc / lsum : 0.f);
  }
}

// resident CTAs per SM of the attention kernel for head dim `hd` (sets the
// kernel's dynamic shared-memory limit on first use per device)
template <int HD, int STAGES>
int ensure_attr_and_occupancy() {
  using L = Layout<HD, STAGES>;
  static int occ[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (occ[dev & 63] == 0) {
    auto kern = paged_attn_kernel<HD, STAGES>;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::DYN_SMEM) !=
        cudaSuccess)
      return -1;
    int n = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kern, kThreads, L::DYN_SMEM) != cudaSuccess ||
        n < 1)
      return -1;
    occ[dev & 63] = n;
  }
  return occ[dev & 63];
}

inline int occupancy(int hd) {
  return hd == 128 ? ensure_attr_and_occupancy<128, 8>() : ensure_attr_and_occupancy<64, 8>();
}

// Split plan: slices per (sequence, kv head) for a batch whose longest
// sequence has max_seq_len tokens (window bounds the span). Each candidate
// slice count S is priced with a model of this kernel on B200, fitted to a
// sweep of batch 16-128 x context 2048-8192 (32 q / 8 kv heads, hd 128;
// within 8% of every measured time):
//   - the B*nkv*S CTAs run in waves of (resident CTAs per SM x SMs);
//   - a CTA streams its K/V pages at most kCtaRate (its own copy and math
//     pipeline), all resident CTAs together at most kReadRate (HBM, reads);
//   - each wave adds kWaveCost (a CTA's prologue, pipeline fill, partials);
//   - S > 1 adds the merge kernel: kMergeCost plus its partials' traffic.
// Few slices leave SMs idle or the last wave long; many slices pay the
// per-CTA cost and the merge. The cheapest S wins (the fewer on a tie).
// The kernel then splits each sequence's actual pages evenly over its slices.
constexpr double kCtaRate = 24.2e3;   // bytes per microsecond, one CTA
constexpr double kReadRate = 7.44e6;  // bytes per microsecond, all CTAs
constexpr double kWaveCost = 3.4;     // microseconds per wave
constexpr double kMergeCost = 5.8;    // microseconds, the merge kernel

inline double plan_cost_us(double pairs, double bytes_per_pair, int s, double slots, int hd) {
  const double n = pairs * s;
  const double w = bytes_per_pair / s;  // bytes per CTA
  const double full = floor(n / slots), rem = n - full * slots;
  double t = full * (w / fmin(kCtaRate, kReadRate / slots) + kWaveCost);
  if (rem > 0) t += w / fmin(kCtaRate, kReadRate / rem) + kWaveCost;
  // partial O and (m, l) per (query head, slice), written then read; four
  // query heads per kv head assumed for the partials' size
  if (s > 1) t += kMergeCost + pairs * 4.0 * s * (hd * 4.0 + 8.0) * 2.0 / kReadRate;
  return t;
}

inline int plan_splits(int B, int nkv, int hd, int max_seq_len, int window) {
  int span = max_seq_len;
  if (window > 0 && window + kBlock < span) span = window + kBlock;
  const int pages = (span + kBlock - 1) / kBlock;
  if (pages <= 0 || B <= 0 || nkv <= 0) return 1;
  const int occ = occupancy(hd);
  const double slots = (double)(occ > 0 ? occ : 2) * num_sms();
  const double pairs = (double)B * nkv;
  const double bytes_per_pair = (double)pages * kBlock * hd * 2.0 /* K and V */ * 2.0 /* bf16 */;
  int max_s = pages / kMinSlice;
  if (max_s > kMaxSplits) max_s = kMaxSplits;
  if (max_s < 1) max_s = 1;
  int best_s = 1;
  double best = plan_cost_us(pairs, bytes_per_pair, 1, slots, hd);
  for (int s = 2; s <= max_s; ++s) {
    const double t = plan_cost_us(pairs, bytes_per_pair, s, slots, hd);
    if (t < best * (1.0 - 1e-9)) {
      best = t;
      best_s = s;
    }
  }
  return best_s;
}

template <int HD, int STAGES>
int launch(const Params& p, const CUtensorMap& tk, const CUtensorMap& tv, cudaStream_t st) {
  using L = Layout<HD, STAGES>;
  auto kern = paged_attn_kernel<HD, STAGES>;
  if (ensure_attr_and_occupancy<HD, STAGES>() < 1) {
    set_last_error("fg_paged_decode_attn: cannot set the kernel's shared-memory limit");
    return FG_ERR_CUDA;
  }
  int rc = launch_k("fg_paged_decode_attn", kern, dim3(p.splits, p.nkv, p.B), dim3(kThreads),
                    L::DYN_SMEM, st, tk, tv, p);
  if (rc || p.splits == 1) return rc;
  // one group of HD threads for a few splits; beyond that about eight splits
  // per group, at least one thread per split, at most kCombineThreads threads
  static_assert(kCombineThreads % HD == 0 && kMaxSplits <= kCombineThreads, "combine block shape");
  static_assert(kSerialSplits <= HD, "the serial form has one group");
  const int ngrp = p.splits <= kSerialSplits
                       ? 1
                       : min(kCombineThreads / HD, max((p.splits + HD - 1) / HD, (p.splits + 7) / 8));
  return launch_k("fg_paged_decode_attn(combine)", attn_combine_kernel, dim3(p.nq, p.B),
                  dim3(HD * ngrp), 0, st, p, HD);
}

// ---------------------------------------------------------------------------
// Prefill (many query positions per sequence), causal, from the paged cache.
//
// Queries: q [B*S][nq][hd] for S consecutive positions per sequence starting
// at p0[b] (tokens of one sequence contiguous); their K/V are already in the
// pages (fg_rope_kv_append_tokens), together with any context cached before
// p0[b]. CTA = (block of 64/G positions, kv head g, sequence b); its 64 MMA
// rows are (position j, head g*G + h) pairs, 16 per consumer warp. The
// producer streams the pages the block can see (causal, window) through the
// same TMA ring as decode; every consumer warp reads every page (its own
// rows), so a page's K/V feed all G heads and all the block's positions.
// Row r attends key k iff k <= pos(r) and (window == 0 or k > pos(r) - window);
// sinks join each head's denominator. Output o [B*S][nq][hd] bf16.
struct PrefillParams {
  const __nv_bfloat16* q;
  const int32_t* block_table;
  const int32_t* p0;        // [B] position of each sequence's first query
  const float* sinks;       // [nq] or null
  __nv_bfloat16* out;
  int B, S, nq, nkv, G, QP; // QP = 64 / G positions per CTA
  int max_blocks, num_blocks;
  int window;
  float scale_log2;
};

template <int HD, int STAGES>
__global__ void __launch_bounds__(kThreads) prefill_attn_kernel(
    const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_v,
    const PrefillParams p) {
  using L = Layout<HD, STAGES>;
  constexpr int KT = HD / 16;
  constexpr int ND = HD / 8;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qb = blockIdx.x, g = blockIdx.y, b = blockIdx.z;
  const int G = p.G, QP = p.QP;
  griddep_wait();  // q and the pages come from earlier kernels
  if (threadIdx.x == 0) griddep_launch_dependents();

  const int base = p.p0[b];
  const int j0 = qb * QP;                       // first position offset of the block
  const int jn = min(QP, p.S - j0);             // positions in this block
  if (jn <= 0) return;
  const int qlo = base + j0, qhi = base + j0 + jn - 1;  // query positions
  const int klo = p.window > 0 ? max(0, qlo - p.window + 1) : 0;
  const int pbeg = klo / kBlock, pend = qhi / kBlock + 1;
  const int npages = pend - pbeg;

  const uint32_t sbase = smem_u32(smem);
  const uint32_t bar_full = sbase + L::BAR_OFFSET;
  const uint32_t bar_empty = bar_full + STAGES * 8;
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(bar_full + 8 * s, 1);
      mbar_init(bar_empty + 8 * s, kConsumers);  // every consumer warp reads every page
    }
    fence_mbar_init();
    prefetch_tensormap(&tm_k);
    prefetch_tensormap(&tm_v);
  }
  __syncthreads();

  if (warp == kConsumers) {
    if (lane == 0) {
      const int32_t* bt = p.block_table + (int64_t)b * p.max_blocks;
      const uint64_t pol = l2_policy_evict_last();  // pages are re-read by the other query blocks
      int issued = 0;
      for (int i = 0; i < npages; ++i) {
        const int s = i % STAGES;
        if (!mbar_wait(bar_empty + 8 * s, ((uint32_t)(i / STAGES) & 1u) ^ 1u, 0x211)) break;
        const int page = pbeg + i;
        int blk = page < p.max_blocks ? bt[page] : -1;
        if (blk < 0 || blk >= p.num_blocks) {
          record_device_error(DEV_BAD_INDEX, 0x212);
          blk = 0;
        }
        const int row = (blk * p.nkv + g) * kBlock;
        const uint32_t st = sbase + s * L::STAGE_BYTES;
        mbar_arrive_expect_tx(bar_full + 8 * s, L::STAGE_BYTES);
#pragma unroll
        for (int bx = 0; bx < L::BOXES; ++bx) {
          tma_load_2d_hint(st + bx * 2048, &tm_k, bar_full + 8 * s, bx * 64, row, pol);
          tma_load_2d_hint(st + L::TILE_BYTES + bx * 2048, &tm_v, bar_full + 8 * s, bx * 64, row, pol);
        }
        ++issued;
      }
      if (issued < npages) {
        for (int s = 0; s < STAGES && s < issued; ++s) {
          const int last = s + ((issued - 1 - s) / STAGES) * STAGES;
          mbar_wait(bar_full + 8 * s, (uint32_t)(last / STAGES) & 1u, 0x214);
        }
      }
    }
    return;
  }

  // ---------------- consumers: warp w owns rows 16w .. 16w+15 ----------------
  const int r0 = warp * 16 + (lane >> 2), r1 = r0 + 8;
  const int jr0 = r0 / G, jr1 = r1 / G;           // position offsets within the block
  const int hr0 = g * G + r0 % G, hr1 = g * G + r1 % G;
  const bool ok0 = jr0 < jn, ok1 = jr1 < jn;
  const int pos0 = qlo + jr0, pos1 = qlo + jr1;
  uint32_t qf[KT][4];
  {
    const int c = (lane & 3) * 2;
    const uint32_t* q0 = reinterpret_cast<const uint32_t*>(
        p.q + (((int64_t)b * p.S + j0 + jr0) * p.nq + hr0) * HD);
    const uint32_t* q1 = reinterpret_cast<const uint32_t*>(
        p.q + (((int64_t)b * p.S + j0 + jr1) * p.nq + hr1) * HD);
#pragma unroll
    for (int kt = 0; kt < KT; ++kt) {
      qf[kt][0] = ok0 ? q0[(kt * 16 + c) >> 1] : 0u;
      qf[kt][1] = ok1 ? q1[(kt * 16 + c) >> 1] : 0u;
      qf[kt][2] = ok0 ? q0[(kt * 16 + 8 + c) >> 1] : 0u;
      qf[kt][3] = ok1 ? q1[(kt * 16 + 8 + c) >> 1] : 0u;
    }
  }
  float o[ND][4];
#pragma unroll
  for (int i = 0; i < ND; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m0 = kNegBig, m1 = kNegBig, l0 = 0.f, l1 = 0.f;
  const int k_tok = ((lane >> 4) << 3) + (lane & 7);
  const int k_sub = (lane >> 3) & 1;
  const int v_tok = (((lane >> 3) & 1) << 3) + (lane & 7);
  const int v_sub = lane >> 4;
  const int lo0 = p.window > 0 ? pos0 - p.window + 1 : 0, lo1 = p.window > 0 ? pos1 - p.window + 1 : 0;

  for (int i = 0; i < npages; ++i) {
    const int s = i % STAGES;
    if (!__all_sync(0xffffffffu, mbar_wait(bar_full + 8 * s, (uint32_t)(i / STAGES) & 1u, 0x213))) break;
    const uint32_t kbase = sbase + s * L::STAGE_BYTES;
    const uint32_t vbase = kbase + L::TILE_BYTES;
    float sc[2][4];
#pragma unroll
    for (int n = 0; n < 2; ++n) sc[n][0] = sc[n][1] = sc[n][2] = sc[n][3] = 0.f;
#pragma unroll
    for (int kt = 0; kt < KT; ++kt) {
      uint32_t kb[4];
      ldsm_x4(kb, tile_addr(kbase, k_tok, kt * 2 + k_sub));
      mma_bf16(sc[0], qf[kt], kb[0], kb[1]);
      mma_bf16(sc[1], qf[kt], kb[2], kb[3]);
    }
    const int tok0 = (pbeg + i) * kBlock + (lane & 3) * 2;
    float mx0 = kNegBig, mx1 = kNegBig;
#pragma unroll
    for (int n = 0; n < 2; ++n) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int t = tok0 + n * 8 + (e & 1);
        const bool valid = e < 2 ? (ok0 && t <= pos0 && t >= lo0) : (ok1 && t <= pos1 && t >= lo1);
        sc[n][e] = valid ? sc[n][e] * p.scale_log2 : kNegBig;
      }
      mx0 = fmaxf(mx0, fmaxf(sc[n][0], sc[n][1]));
      mx1 = fmaxf(mx1, fmaxf(sc[n][2], sc[n][3]));
    }
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
    const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
    const float a0 = exp2f(m0 - mn0), a1 = exp2f(m1 - mn1);
    m0 = mn0;
    m1 = mn1;
    // masked keys contribute nothing, also while a row has no valid key yet
    // (a sliding window starts later for the block's later positions)
    float ps[2][4];
#pragma unroll
    for (int n = 0; n < 2; ++n) {
      ps[n][0] = sc[n][0] > 0.5f * kNegBig ? exp2f(sc[n][0] - mn0) : 0.f;
      ps[n][1] = sc[n][1] > 0.5f * kNegBig ? exp2f(sc[n][1] - mn0) : 0.f;
      ps[n][2] = sc[n][2] > 0.5f * kNegBig ? exp2f(sc[n][2] - mn1) : 0.f;
      ps[n][3] = sc[n][3] > 0.5f * kNegBig ? exp2f(sc[n][3] - mn1) : 0.f;
    }
    l0 = l0 * a0 + ps[0][0] + ps[0][1] + ps[1][0] + ps[1][1];
    l1 = l1 * a1 + ps[0][2] + ps[0][3] + ps[1][2] + ps[1][3];
#pragma unroll
    for (int nd = 0; nd < ND; ++nd) {
      o[nd][0] *= a0;
      o[nd][1] *= a0;
      o[nd][2] *= a1;
      o[nd][3] *= a1;
    }
    uint32_t pa[4];
    pa[0] = pack_bf16x2(ps[0][0], ps[0][1]);
    pa[1] = pack_bf16x2(ps[0][2], ps[0][3]);
    pa[2] = pack_bf16x2(ps[1][0], ps[1][1]);
    pa[3] = pack_bf16x2(ps[1][2], ps[1][3]);
#pragma unroll
    for (int c2 = 0; c2 < KT; ++c2) {
      uint32_t vb[4];
      ldsm_x4_t(vb, tile_addr(vbase, v_tok, c2 * 2 + v_sub));
      mma_bf16(o[2 * c2], pa, vb[0], vb[1]);
      mma_bf16(o[2 * c2 + 1], pa, vb[2], vb[3]);
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(bar_empty + 8 * s);
  }
  l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
  l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
  const float s0 = p.sinks ? exp2f(p.sinks[hr0] * kLog2e - m0) : 0.f;
  const float s1 = p.sinks ? exp2f(p.sinks[hr1] * kLog2e - m1) : 0.f;
  const float inv0 = 1.f / (l0 + s0), inv1 = 1.f / (l1 + s1);
  const int c = (lane & 3) * 2;
  __nv_bfloat16* out0 = p.out + (((int64_t)b * p.S + j0 + jr0) * p.nq + hr0) * HD;
  __nv_bfloat16* out1 = p.out + (((int64_t)b * p.S + j0 + jr1) * p.nq + hr1) * HD;
#pragma unroll
  for (int nd = 0; nd < ND; ++nd) {
    if (ok0) *reinterpret_cast<uint32_t*>(out0 + nd * 8 + c) = pack_bf16x2(o[nd][0] * inv0, o[nd][1] * inv0);
    if (ok1) *reinterpret_cast<uint32_t*>(out1 + nd * 8 + c) = pack_bf16x2(o[nd][2] * inv1, o[nd][3] * inv1);
  }
}

template <int HD, int STAGES>
int launch_prefill(const PrefillParams& p, const CUtensorMap& tk, const CUtensorMap& tv, cudaStream_t st) {
  using L = Layout<HD, STAGES>;
  auto kern = prefill_attn_kernel<HD, STAGES>;
  static bool attr_done[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!attr_done[dev & 63]) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::DYN_SMEM) != cudaSuccess) {
      set_last_error("fg_prefill_attn: cannot set the kernel's shared-memory limit");
      return FG_ERR_CUDA;
    }
    attr_done[dev & 63] = true;
  }
  return launch_k("fg_prefill_attn", kern, dim3((p.S + p.QP - 1) / p.QP, p.nkv, p.B), dim3(kThreads),
                  L::DYN_SMEM, st, tk, tv, p);
}

}  // namespace attn
}  // namespace fg

extern "C" {

int fg_attn_splits(int B, int nkv, int hd, int max_seq_len, int window) {
  if (B <= 0 || nkv <= 0 || (hd != 64 && hd != 128) || max_seq_len <= 0) return 0;
  return fg::attn::plan_splits(B, nkv, hd, max_seq_len, window);
}

size_t fg_attn_workspace_bytes(int B, int nq, int nkv, int hd, int max_seq_len, int window) {
  if (B <= 0 || nq <= 0 || nkv <= 0 || (hd != 64 && hd != 128) || max_seq_len <= 0) return 0;
  const int splits = fg::attn::plan_splits(B, nkv, hd, max_seq_len, window);
  if (splits <= 1) return 0;
  const size_t rows = (size_t)B * nq * splits;
  return ((rows * hd * sizeof(float) + 255) & ~size_t(255)) + rows * 2 * sizeof(float);
}

int fg_paged_decode_attn(const fg_bf16* q, const fg_bf16* k_cache, const fg_bf16* v_cache,
                         const int32_t* block_table, const int32_t* seq_lens, const float* sinks,
                         fg_bf16* out, void* workspace, size_t workspace_bytes, int B, int nq,
                         int nkv, int hd, int block_size, int num_blocks, int max_blocks,
                         int max_seq_len, int window, float scale, fg_stream_t stream) {
  using namespace fg::attn;
  FG_REQUIRE(q && k_cache && v_cache && block_table && seq_lens && out,
             "fg_paged_decode_attn: null pointer");
  FG_REQUIRE(hd == 64 || hd == 128, "fg_paged_decode_attn: hd must be 64 or 128, got %d", hd);
  FG_REQUIRE(block_size == kBlock, "fg_paged_decode_attn: block_size must be 16, got %d", block_size);
  FG_REQUIRE(nkv > 0 && nq % nkv == 0 && nq / nkv <= 16,
             "fg_paged_decode_attn: nq/nkv must be an integer <= 16 (nq=%d nkv=%d)", nq, nkv);
  FG_REQUIRE(B >= 0 && num_blocks > 0 && max_blocks > 0 && max_seq_len > 0 && window >= 0,
             "fg_paged_decode_attn: bad sizes");
  FG_REQUIRE(max_seq_len <= max_blocks * kBlock,
             "fg_paged_decode_attn: max_seq_len %d exceeds the block table (%d blocks)",
             max_seq_len, max_blocks);
  FG_REQUIRE((((uintptr_t)q | (uintptr_t)k_cache | (uintptr_t)v_cache) & 15) == 0,
             "fg_paged_decode_attn: q/k/v must be 16-byte aligned");
  if (B == 0) return FG_OK;
  Params p;
  p.q = reinterpret_cast<const __nv_bfloat16*>(q);
  p.block_table = block_table;
  p.seq_lens = seq_lens;
  p.sinks = sinks;
  p.out = reinterpret_cast<__nv_bfloat16*>(out);
  p.B = B;
  p.nq = nq;
  p.nkv = nkv;
  p.G = nq / nkv;
  p.max_blocks = max_blocks;
  p.num_blocks = num_blocks;
  p.window = window;
  p.scale_log2 = scale * kLog2e;
  p.splits = plan_splits(B, nkv, hd, max_seq_len, window);
  p.part_o = nullptr;
  p.part_ml = nullptr;
  if (p.splits > 1) {
    const size_t rows = (size_t)B * nq * p.splits;
    const size_t o_bytes = (rows * hd * sizeof(float) + 255) & ~size_t(255);
    const size_t need = o_bytes + rows * 2 * sizeof(float);
    FG_REQUIRE(workspace != nullptr && workspace_bytes >= need,
               "fg_paged_decode_attn: needs %zu workspace bytes, got %zu", need, workspace_bytes);
    p.part_o = reinterpret_cast<float*>(workspace);
    p.part_ml = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(workspace) + o_bytes);
  }
  const uint64_t rows = (uint64_t)num_blocks * nkv * kBlock;
  CUtensorMap tk, tv;
  int rc = fg::make_tmap_2d_bf16(&tk, k_cache, hd, rows, (uint64_t)hd * 2, 64, kBlock,
                                 CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  rc = fg::make_tmap_2d_bf16(&tv, v_cache, hd, rows, (uint64_t)hd * 2, 64, kBlock,
                             CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (hd == 128) return launch<128, 8>(p, tk, tv, st);
  return launch<64, 8>(p, tk, tv, st);
}

int fg_prefill_attn(const fg_bf16* q, const fg_bf16* k_cache, const fg_bf16* v_cache,
                    const int32_t* block_table, const int32_t* first_pos, const float* sinks, fg_bf16* out,
                    int B, int S, int nq, int nkv, int hd, int block_size, int num_blocks, int max_blocks,
                    int window, float scale, fg_stream_t stream) {
  using namespace fg::attn;
  FG_REQUIRE(q && k_cache && v_cache && block_table && first_pos && out, "fg_prefill_attn: null pointer");
  FG_REQUIRE(hd == 64 || hd == 128, "fg_prefill_attn: hd must be 64 or 128, got %d", hd);
  FG_REQUIRE(block_size == kBlock, "fg_prefill_attn: block_size must be 16, got %d", block_size);
  FG_REQUIRE(nkv > 0 && nq % nkv == 0 && nq / nkv <= 16 && 64 % (nq / nkv) == 0,
             "fg_prefill_attn: nq/nkv must divide 64 (nq=%d nkv=%d)", nq, nkv);
  FG_REQUIRE(B >= 0 && S >= 0 && num_blocks > 0 && max_blocks > 0 && window >= 0, "fg_prefill_attn: bad sizes");
  FG_REQUIRE((((uintptr_t)q | (uintptr_t)k_cache | (uintptr_t)v_cache | (uintptr_t)out) & 15) == 0,
             "fg_prefill_attn: q/k/v/out must be 16-byte aligned");
  if (B == 0 || S == 0) return FG_OK;
  PrefillParams p;
  p.q = reinterpret_cast<const __nv_bfloat16*>(q);
  p.block_table = block_table;
  p.p0 = first_pos;
  p.sinks = sinks;
  p.out = reinterpret_cast<__nv_bfloat16*>(out);
  p.B = B;
  p.S = S;
  p.nq = nq;
  p.nkv = nkv;
  p.G = nq / nkv;
  p.QP = 64 / p.G;
  p.max_blocks = max_blocks;
  p.num_blocks = num_blocks;
  p.window = window;
  p.scale_log2 = scale * kLog2e;
  const uint64_t rows = (uint64_t)num_blocks * nkv * kBlock;
  CUtensorMap tk, tv;
  int rc = fg::make_tmap_2d_bf16(&tk, k_cache, hd, rows, (uint64_t)hd * 2, 64, kBlock, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  rc = fg::make_tmap_2d_bf16(&tv, v_cache, hd, rows, (uint64_t)hd * 2, 64, kBlock, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (hd == 128) return launch_prefill<128, 8>(p, tk, tv, st);
  return launch_prefill<64, 8>(p, tk, tv, st);
}

}  // extern "C"
