// gpt-oss MoE feed-forward for the decode step: router top-k, token permute,
// MXFP4 expert GEMMs on tcgen05, weighted un-permute.
//
// Reference semantics (transformers' GptOssMLP, which the reference runner
// calls at runner.py:432-457 and the vLLM expert paths restate at
// vllm_integration.py:452-485, 527-551):
//   logits = x W_r^T + b_r              (bf16)
//   top-k over the logits (ties: lower expert id), scores = softmax(top-k)
//   per expert e: gu = x W1_e + b1_e (bf16), gate = gu[::2], up = gu[1::2]
//                 act = (clamp(up,-7,7) + 1) * clamp(gate,max=7) * sigmoid(1.702 * gate)
//                 y = act W2_e + b2_e (bf16)
//   out[t] += y * score (bf16, experts in ascending order), then + residual.
// Expert weights are MXFP4 (OCP microscaling: e2m1 values, one e8m0 scale per
// 32 elements along K), dequantised to bf16 exactly as transformers'
// convert_moe_packed_tensors does; the dequantisation happens in shared
// memory, so HBM moves 4.25 bits per weight and only for routed experts.
//
// Packed MXFP4 weight layout (fg_pack_mxfp4): per expert, per 128-row tile,
// per 64-wide K step, a 4352-byte record: 128 rows x 32 bytes of e2m1 pairs
// (low nibble = even k) followed by 128 rows x 2 e8m0 scales. For the fused
// SwiGLU-OAI epilogue the gate/up rows are interleaved in blocks of 64 as in
// the dense path (the caller orders rows before packing).
#pragma once
#include "gemm.cuh"

namespace fg {
namespace moe {

using gemm::BK;
using gemm::BM;

constexpr int kValBytes = BM * BK / 2;           // 4096
constexpr int kScaleBytes = BM * (BK / 32);      // 256
constexpr int kRecBytes = kValBytes + kScaleBytes;  // 4352
constexpr int kMaxE = 64;

// ---------------------------------------------------------------------------
// router: logits, top-k (value desc, index asc), softmax over the selected
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) router_topk_kernel(
    const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ w,
    const __nv_bfloat16* __restrict__ bias, int H, int E, int k, __nv_bfloat16* __restrict__ out_w,
    int32_t* __restrict__ out_idx, __nv_bfloat16* __restrict__ out_logits) {
  griddep_wait();
  griddep_launch_dependents();
  __shared__ float logit[kMaxE];
  const int t = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint4* xr = reinterpret_cast<const uint4*>(x + (int64_t)t * H);
  const int H8 = H >> 3;
  for (int e = warp; e < E; e += 8) {
    const uint4* wr = reinterpret_cast<const uint4*>(w + (int64_t)e * H);
    float acc = 0.f;
    for (int i = lane; i < H8; i += 32) {
      const uint4 a = xr[i], b = wr[i];
      const uint32_t* pa = reinterpret_cast<const uint32_t*>(&a);
      const uint32_t* pb = reinterpret_cast<const uint32_t*>(&b);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float2 fa = unpack_bf16x2(pa[q]), fb = unpack_bf16x2(pb[q]);
        acc += fa.x * fb.x + fa.y * fb.y;
      }
    }
    acc = warp_sum(acc);
    if (lane == 0) {
      const float v = rbf(acc + (bias ? bf2f(bias[e]) : 0.f));  // bf16 logits, as the linear
      logit[e] = v;
      if (out_logits) out_logits[(int64_t)t * E + e] = f2bf(v);
    }
  }
  __syncthreads();
  if (warp == 0) {
    // each lane holds up to two experts
    float v0 = lane < E ? logit[lane] : -INFINITY;
    float v1 = lane + 32 < E ? logit[lane + 32] : -INFINITY;
    float sel_v[8];
    int sel_i[8];
    for (int j = 0; j < k; ++j) {
      float bv = v0;
      int bi = lane;
      if (v1 > bv) {
        bv = v1;
        bi = lane + 32;
      }
      if (bi >= E) bi = 0x7fffffff;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ov > bv || (ov == bv && oi < bi)) {
          bv = ov;
          bi = oi;
        }
      }
      sel_v[j] = bv;
      sel_i[j] = bi;
      if (bi == lane) v0 = -INFINITY;
      if (bi == lane + 32) v1 = -INFINITY;
    }
    if (lane == 0) {
      float m = sel_v[0], s = 0.f, p[8];
      for (int j = 0; j < k; ++j) {
        p[j] = __expf(sel_v[j] - m);
        s += p[j];
      }
      for (int j = 0; j < k; ++j) {
        out_idx[(int64_t)t * k + j] = sel_i[j];
        out_w[(int64_t)t * k + j] = f2bf(p[j] / s);
      }
    }
  }
}

// ---------------------------------------------------------------------------
// permute: deterministic counting sort of (token, slot) pairs by expert
// ---------------------------------------------------------------------------
// One CTA of 32 warps. Pair p = t*k + j goes to row offsets[e] + rank, rank =
// number of earlier pairs (in p order) routed to the same expert.
__global__ void __launch_bounds__(1024) permute_kernel(
    const int32_t* __restrict__ idx, int n, int E, int BN, int max_items,
    int32_t* __restrict__ offsets, int32_t* __restrict__ perm_pair, int32_t* __restrict__ inv,
    int32_t* __restrict__ items, int32_t* __restrict__ item_count) {
  griddep_wait();
  griddep_launch_dependents();
  __shared__ int cnt[32][kMaxE];
  __shared__ int base[kMaxE + 1];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int chunk = (n + 31) / 32;
  const int p0 = warp * chunk, p1 = min(n, p0 + chunk);
  for (int e = lane; e < E; e += 32) cnt[warp][e] = 0;
  __syncwarp();
  for (int p = p0 + lane; p < p1; p += 32) {
    int e = idx[p];
    if (e < 0 || e >= E) {
      record_device_error(DEV_BAD_INDEX, 0x301);
      e = 0;
    }
    atomicAdd(&cnt[warp][e], 1);
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int run = 0;
    for (int e = 0; e < E; ++e) {
      base[e] = run;
      for (int w = 0; w < 32; ++w) {
        const int c = cnt[w][e];
        cnt[w][e] = run;  // start of warp w's pairs for expert e
        run += c;
      }
    }
    base[E] = run;
    int ni = 0;
    for (int e = 0; e < E; ++e) {
      const int ne = base[e + 1] - base[e];
      for (int tt = 0; tt * BN < ne && ni < max_items; ++tt, ++ni) {
        items[2 * ni] = e;
        items[2 * ni + 1] = tt;
      }
    }
    *item_count = ni;
  }
  __syncthreads();
  for (int e = threadIdx.x; e <= E; e += blockDim.x) offsets[e] = base[e];
  // ranks: the warp walks its chunk 32 pairs at a time, in order
  const unsigned lt = (1u << lane) - 1u;
  for (int p = p0; p < p1; p += 32) {
    const int q = p + lane;
    int e = q < p1 ? idx[q] : -1;
    if (q < p1 && (e < 0 || e >= E)) e = 0;
    const unsigned same = __match_any_sync(0xffffffffu, e);
    const int r = __popc(same & lt);
    int pos = 0;
    if (q < p1) pos = cnt[warp][e] + r;
    __syncwarp();
    // the highest lane of each group advances that expert's counter
    if (q < p1 && (same >> lane) == 1u) cnt[warp][e] += r + 1;
    __syncwarp();
    if (q < p1) {
      perm_pair[pos] = q;
      inv[q] = pos;
    }
  }
}

// rows of x in permuted order: out[i] = x[perm_pair[i] / k]
__global__ void gather_rows_kernel(const uint4* __restrict__ x, const int32_t* __restrict__ perm_pair,
                                   int k, int H8, uint4* __restrict__ out) {
  griddep_wait();
  griddep_launch_dependents();
  const int i = blockIdx.x;
  const int t = perm_pair[i] / k;
  const uint4* src = x + (int64_t)t * H8;
  uint4* dst = out + (int64_t)i * H8;
  for (int c = threadIdx.x; c < H8; c += blockDim.x) dst[c] = src[c];
}

// out[t] = residual[t] + sum over the k experts (ascending id) of y[inv] * w
__global__ void unpermute_kernel(const __nv_bfloat16* __restrict__ y, const int32_t* __restrict__ inv,
                                 const int32_t* __restrict__ idx,
                                 const __nv_bfloat16* __restrict__ wts,
                                 const __nv_bfloat16* __restrict__ residual,
                                 __nv_bfloat16* __restrict__ out, int k, int H) {
  griddep_wait();
  griddep_launch_dependents();
  const int t = blockIdx.x;
  int order[8];
  for (int j = 0; j < k; ++j) order[j] = j;
  // insertion sort of the k slots by expert id (k <= 8)
  for (int a = 1; a < k; ++a) {
    const int v = order[a];
    int b = a - 1;
    while (b >= 0 && idx[(int64_t)t * k + order[b]] > idx[(int64_t)t * k + v]) {
      order[b + 1] = order[b];
      --b;
    }
    order[b + 1] = v;
  }
  for (int h = threadIdx.x; h < H; h += blockDim.x) {
    float acc = 0.f;
    for (int a = 0; a < k; ++a) {
      const int j = order[a];
      const int row = inv[(int64_t)t * k + j];
      const float wv = bf2f(wts[(int64_t)t * k + j]);
      acc = rbf(acc + rbf(bf2f(y[(int64_t)row * H + h]) * wv));
    }
    out[(int64_t)t * H + h] = f2bf(residual ? bf2f(residual[(int64_t)t * H + h]) + acc : acc);
  }
}

// ---------------------------------------------------------------------------
// MXFP4 packing: values [E][N][K/2] u8 + scales [E][N][K/32] u8 -> records
// ---------------------------------------------------------------------------
__global__ void pack_mxfp4_kernel(const uint8_t* __restrict__ vals, const uint8_t* __restrict__ scales,
                                  uint8_t* __restrict__ packed, int N, int K, int n_tiles, int nkb,
                                  long long records) {
  griddep_wait();
  const long long rec = blockIdx.x;
  if (rec >= records) return;
  const int kb = (int)(rec % nkb);
  const int nt = (int)((rec / nkb) % n_tiles);
  const long long e = rec / ((long long)nkb * n_tiles);
  uint8_t* dst = packed + rec * kRecBytes;
  for (int i = threadIdx.x; i < kRecBytes; i += blockDim.x) {
    uint8_t v = 0;
    if (i < kValBytes) {
      const int r = i >> 5, byte = i & 31;
      const int n = nt * BM + r, kk = kb * BK + byte * 2;
      if (n < N && kk < K) v = vals[(e * N + n) * (K / 2) + (kk >> 1)];
    } else {
      const int j = i - kValBytes;
      const int r = j >> 1, blk = j & 1;
      const int n = nt * BM + r, kk = kb * BK + blk * 32;
      v = 127;  // scale 1.0 for padding (its values are zero)
      if (n < N && kk < K) v = scales[(e * N + n) * (K / 32) + (kk >> 5)];
    }
    dst[i] = v;
  }
}

// ---------------------------------------------------------------------------
// MXFP4 x bf16 grouped GEMM (swap-AB, tcgen05 kind::f16 after an exact
// in-shared-memory dequantisation of the weight tile)
// ---------------------------------------------------------------------------
struct GemmParams {
  const uint8_t* w;           // packed records [E][n_tiles][nkb]
  const __nv_bfloat16* bias;  // [E][N] (packed row order) or null
  const int32_t* offsets;     // [E+1] rows of each expert in x / out
  const int32_t* items;       // [max_items][2] = (expert, token tile)
  const int32_t* item_count;
  __nv_bfloat16* out;         // [rows][ldo]
  int N, K, n_tiles, nkb, ldo, epilogue;
};

constexpr int kConvWarps = 8;
constexpr int kMoeThreads = (2 + kConvWarps) * 32;  // producer, MMA, converters

template <int BN, int STAGES>
struct MLayout {
  static constexpr int A_BYTES = BM * BK * 2;   // dequantised bf16 tile
  static constexpr int X_BYTES = BN * BK * 2;
  static constexpr int RAW_BYTES = 5120;         // >= kRecBytes, keeps 1 KB alignment
  static constexpr int STAGE_BYTES = A_BYTES + X_BYTES + RAW_BYTES;
  static constexpr int LUT_OFFSET = STAGES * STAGE_BYTES;   // 256 x bf16x2
  static constexpr int XCH_OFFSET = LUT_OFFSET + 1024;      // bf16 [BN][64]
  static constexpr int BAR_OFFSET = XCH_OFFSET + BN * 64 * 2;
  static constexpr int MISC_OFFSET = BAR_OFFSET + (3 * STAGES + 1) * 8;
  static constexpr int TOTAL = MISC_OFFSET + 32;
  static constexpr int DYN_SMEM = TOTAL + 1024;
  static constexpr uint32_t TMEM_COLS = BN < 32 ? 32 : BN;
  static_assert(RAW_BYTES >= kRecBytes && STAGE_BYTES % 1024 == 0, "stage layout");
};

// bf16 bits of the 16 e2m1 codes (sign, 2-bit exponent, 1-bit mantissa)
__device__ __forceinline__ uint32_t e2m1_bf16_bits(uint32_t c) {
  const uint32_t mag = c & 7u;
  uint32_t bits;
  if (mag == 0) bits = 0;
  else if (mag == 1) bits = 0x3F00u;  // 0.5
  else bits = ((mag >> 1) + 126u) << 7 | ((mag & 1u) << 6);  // 2^(e-1) * (1 + m/2)
  return bits | ((c & 8u) << 12);
}

__device__ __forceinline__ float swiglu_oai(float g, float u) {
  // transformers' GptOssExperts._apply_gate in bf16 arithmetic: each tensor op rounds
  g = fminf(g, 7.f);
  u = fminf(fmaxf(u, -7.f), 7.f);
  const float ga = rbf(g * 1.702f);
  const float sg = rbf(1.f / (1.f + __expf(-ga)));
  const float glu = rbf(g * sg);
  return rbf(rbf(u + 1.f) * glu);
}

template <int BN, int STAGES>
__global__ void __launch_bounds__(kMoeThreads, 1)
    moe_gemm_kernel(const __grid_constant__ CUtensorMap tm_x, const GemmParams p) {
  using L = MLayout<BN, STAGES>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  griddep_wait();  // routing results come from the permute kernel
  if (threadIdx.x == 0) griddep_launch_dependents();
  const int item = blockIdx.y;
  if (item >= *p.item_count) return;
  const int e = p.items[2 * item];
  const int t_tile = p.items[2 * item + 1];
  const int row0 = p.offsets[e] + t_tile * BN;
  const int row_end = p.offsets[e + 1];
  const int n_tile = blockIdx.x;
  const int nkb = p.nkb;

  const uint32_t sbase = smem_u32(smem);
  const uint32_t bar_full = sbase + L::BAR_OFFSET;  // TMA landed (raw + x)
  const uint32_t bar_conv = bar_full + STAGES * 8;  // converters done
  const uint32_t bar_empty = bar_conv + STAGES * 8; // MMA done with the stage
  const uint32_t bar_accf = bar_empty + STAGES * 8;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::MISC_OFFSET);
  int* misc = reinterpret_cast<int*>(smem + L::MISC_OFFSET + 16);
  uint32_t* lut = reinterpret_cast<uint32_t*>(smem + L::LUT_OFFSET);
  __nv_bfloat16* xch = reinterpret_cast<__nv_bfloat16*>(smem + L::XCH_OFFSET);

  // byte -> two bf16 (low nibble first) lookup table
  for (int i = threadIdx.x; i < 256; i += blockDim.x)
    lut[i] = e2m1_bf16_bits(i & 15u) | (e2m1_bf16_bits(i >> 4) << 16);
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(bar_full + 8 * s, 1);
      mbar_init(bar_conv + 8 * s, kConvWarps);
      mbar_init(bar_empty + 8 * s, 1);
    }
    mbar_init(bar_accf, 1);
    misc[0] = 0;
    misc[1] = 0;
    fence_mbar_init();
    prefetch_tensormap(&tm_x);
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(L::TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  gemm::tc_fence_before();
  __syncthreads();
  gemm::tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- producer ----------------
      const uint64_t pol_w = l2_policy_evict_first();
      const uint64_t pol_x = l2_policy_evict_last();
      const uint8_t* wrec = p.w + ((size_t)e * p.n_tiles + n_tile) * nkb * kRecBytes;
      int issued = 0;
      for (int i = 0; i < nkb; ++i) {
        const int s = i % STAGES;
        const uint32_t ph = (uint32_t)(i / STAGES) & 1u;
        if (!mbar_wait(bar_empty + 8 * s, ph ^ 1u, 0x311)) break;
        const uint32_t st = sbase + s * L::STAGE_BYTES;
        mbar_arrive_expect_tx(bar_full + 8 * s, kRecBytes + L::X_BYTES);
        bulk_load(st + L::A_BYTES + L::X_BYTES, wrec + (size_t)i * kRecBytes, kRecBytes,
                  bar_full + 8 * s, pol_w);
        tma_load_2d_hint(st + L::A_BYTES, &tm_x, bar_full + 8 * s, i * BK, row0, pol_x);
        ++issued;
      }
      misc[0] = issued;
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer ----------------
      constexpr uint32_t idesc = gemm::idesc_bf16(BM, BN);
      for (int i = 0; i < nkb; ++i) {
        const int s = i % STAGES;
        const uint32_t ph = (uint32_t)(i / STAGES) & 1u;
        if (!mbar_wait(bar_conv + 8 * s, ph, 0x312)) break;
        gemm::tc_fence_after();
        const uint32_t st = sbase + s * L::STAGE_BYTES;
        const uint64_t adesc = gemm::sw128_kmajor_desc(st);
        const uint64_t bdesc = gemm::sw128_kmajor_desc(st + L::A_BYTES);
#pragma unroll
        for (int kk = 0; kk < BK / 16; ++kk)
          gemm::tc_mma(tmem, adesc + 2 * kk, bdesc + 2 * kk, idesc, (i > 0 || kk > 0) ? 1u : 0u);
        gemm::tc_commit(bar_empty + 8 * s);
        misc[1] = i + 1;
      }
      gemm::tc_commit(bar_accf);
    }
  } else {
    // ---------------- converters: e2m1 + e8m0 -> bf16, 128-byte-swizzled K-major ----------------
    const int ct = threadIdx.x - 64;  // 0 .. 255
    for (int i = 0; i < nkb; ++i) {
      const int s = i % STAGES;
      const uint32_t ph = (uint32_t)(i / STAGES) & 1u;
      const bool ok = mbar_wait(bar_full + 8 * s, ph, 0x313);
      uint8_t* st = smem + s * L::STAGE_BYTES;
      const uint8_t* raw = st + L::A_BYTES + L::X_BYTES;
      if (ok) {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int q = ct + j * 256;  // 16-byte output chunk: row r, chunk c (8 values)
          const int r = q >> 3, c = q & 7;
          const uint32_t v4 = *reinterpret_cast<const uint32_t*>(raw + r * 32 + c * 4);
          const uint32_t sc = raw[kValBytes + r * 2 + (c >> 2)];
          // 2^(sc-127) as bf16x2 (exact power of two; e8m0 0 and 255 are not produced here)
          const uint32_t sb = (sc & 0xFFu) << 7;
          uint32_t sbits = sb | (sb << 16);
          const __nv_bfloat162 s2 = *reinterpret_cast<const __nv_bfloat162*>(&sbits);
          uint4 o;
          uint32_t* po = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
          for (int b = 0; b < 4; ++b) {
            const uint32_t pair = lut[(v4 >> (8 * b)) & 0xFFu];
            __nv_bfloat162 v2 = *reinterpret_cast<const __nv_bfloat162*>(&pair);
            v2 = __hmul2(v2, s2);
            po[b] = *reinterpret_cast<uint32_t*>(&v2);
          }
          *reinterpret_cast<uint4*>(st + r * 128 + ((c ^ (r & 7)) << 4)) = o;
        }
      }
      fence_proxy_async_smem();  // generic-proxy writes -> tensor-core reads
      __syncwarp();
      if (lane == 0) mbar_arrive(bar_conv + 8 * s);
    }
    // ---------------- epilogue: warps 2..5 read the four TMEM lane quarters ----------------
    if (warp < 6) {
      const int q = warp & 3;
      const int row = q * 32 + lane;
      const bool acc_ok = mbar_wait(bar_accf, 0, 0x314);
      gemm::tc_fence_after();
      const uint32_t taddr = tmem + ((uint32_t)(q * 32) << 16);
      const __nv_bfloat16* bias = p.bias ? p.bias + (size_t)e * p.N : nullptr;
      if (p.epilogue == FG_EPI_SWIGLU_OAI) {
        if (q >= 2) {
          const int nrow = n_tile * BM + row;
          const float b = (bias && nrow < p.N) ? bf2f(bias[nrow]) : 0.f;
#pragma unroll 1
          for (int j0 = 0; j0 < BN; j0 += 16) {
            float v[16];
            gemm::tc_ld16(taddr + j0, v);
#pragma unroll
            for (int ii = 0; ii < 16; ++ii) xch[(j0 + ii) * 64 + (row - 64)] = f2bf(acc_ok ? v[ii] + b : 0.f);
          }
        }
        asm volatile("bar.sync 1, 128;" ::: "memory");
        if (q < 2) {
          const int nrow = n_tile * BM + row;
          const float b = (bias && nrow < p.N) ? bf2f(bias[nrow]) : 0.f;
          const int f = n_tile * 64 + row;
#pragma unroll 1
          for (int j0 = 0; j0 < BN; j0 += 16) {
            float v[16];
            gemm::tc_ld16(taddr + j0, v);
#pragma unroll
            for (int ii = 0; ii < 16; ++ii) {
              const int rr = row0 + j0 + ii;
              if (rr < row_end && nrow < p.N) {
                const float g = rbf((acc_ok ? v[ii] : 0.f) + b);
                const float u = bf2f(xch[(j0 + ii) * 64 + row]);
                p.out[(int64_t)rr * p.ldo + f] = f2bf(swiglu_oai(g, u));
              }
            }
          }
        }
      } else {
        const int nrow = n_tile * BM + row;
        const float b = (bias && nrow < p.N) ? bf2f(bias[nrow]) : 0.f;
#pragma unroll 1
        for (int j0 = 0; j0 < BN; j0 += 16) {
          float v[16];
          gemm::tc_ld16(taddr + j0, v);
          if (nrow >= p.N) continue;
#pragma unroll
          for (int ii = 0; ii < 16; ++ii) {
            const int rr = row0 + j0 + ii;
            if (rr < row_end) p.out[(int64_t)rr * p.ldo + nrow] = f2bf((acc_ok ? v[ii] : 0.f) + b);
          }
        }
      }
    }
  }

  gemm::tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int i = misc[1]; i < misc[0]; ++i)
      mbar_wait(bar_full + 8 * (i % STAGES), (uint32_t)(i / STAGES) & 1u, 0x315);
  }
  __syncthreads();
  if (warp == 0) {
    gemm::tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(L::TMEM_COLS)
                 : "memory");
  }
}

}  // namespace moe
}  // namespace fg

extern "C" {

int fg_moe_router_topk(const fg_bf16* x, const fg_bf16* w, const fg_bf16* bias, int T, int H, int E,
                       int k, fg_bf16* weights, int32_t* indices, fg_bf16* logits,
                       fg_stream_t stream) {
  FG_REQUIRE(x && w && weights && indices, "fg_moe_router_topk: null pointer");
  FG_REQUIRE(T >= 0 && H > 0 && H % 8 == 0 && E > 0 && E <= fg::moe::kMaxE && k > 0 && k <= 8 &&
                 k <= E,
             "fg_moe_router_topk: bad sizes T=%d H=%d E=%d k=%d", T, H, E, k);
  FG_REQUIRE((((uintptr_t)x | (uintptr_t)w) & 15) == 0, "fg_moe_router_topk: x/w must be 16-byte aligned");
  if (T == 0) return FG_OK;
  return fg::launch_k("fg_moe_router_topk", fg::moe::router_topk_kernel, dim3(T), dim3(256), 0,
                      (cudaStream_t)stream, reinterpret_cast<const __nv_bfloat16*>(x),
                      reinterpret_cast<const __nv_bfloat16*>(w),
                      reinterpret_cast<const __nv_bfloat16*>(bias), H, E, k,
                      reinterpret_cast<__nv_bfloat16*>(weights), indices,
                      reinterpret_cast<__nv_bfloat16*>(logits));
}

int fg_moe_max_items(int T, int k, int E, int BN) {
  if (T <= 0 || k <= 0 || E <= 0 || BN <= 0) return 0;
  return E + (T * k + BN - 1) / BN;
}

int fg_moe_tile_tokens(int T, int k, int E) {
  const int avg = (T * k + E - 1) / (E > 0 ? E : 1);
  return avg <= 16 ? 16 : (avg <= 32 ? 32 : 64);
}

int fg_moe_permute(const int32_t* indices, int T, int k, int E, int BN, int32_t* offsets,
                   int32_t* perm_pair, int32_t* inv, int32_t* items, int32_t* item_count,
                   fg_stream_t stream) {
  FG_REQUIRE(indices && offsets && perm_pair && inv && items && item_count,
             "fg_moe_permute: null pointer");
  FG_REQUIRE(T >= 0 && k > 0 && E > 0 && E <= fg::moe::kMaxE && (BN == 16 || BN == 32 || BN == 64),
             "fg_moe_permute: bad sizes");
  return fg::launch_k("fg_moe_permute", fg::moe::permute_kernel, dim3(1), dim3(1024), 0,
                      (cudaStream_t)stream, indices, T * k, E, BN, fg_moe_max_items(T, k, E, BN),
                      offsets, perm_pair, inv, items, item_count);
}

int fg_moe_gather(const fg_bf16* x, const int32_t* perm_pair, int T, int k, int H, fg_bf16* out,
                  fg_stream_t stream) {
  FG_REQUIRE(x && perm_pair && out, "fg_moe_gather: null pointer");
  FG_REQUIRE(T >= 0 && k > 0 && H % 8 == 0, "fg_moe_gather: bad sizes");
  if (T == 0) return FG_OK;
  return fg::launch_k("fg_moe_gather", fg::moe::gather_rows_kernel, dim3(T * k), dim3(128), 0,
                      (cudaStream_t)stream, reinterpret_cast<const uint4*>(x), perm_pair, k, H / 8,
                      reinterpret_cast<uint4*>(out));
}

int fg_moe_unpermute(const fg_bf16* y, const int32_t* inv, const int32_t* indices,
                     const fg_bf16* weights, const fg_bf16* residual, fg_bf16* out, int T, int k,
                     int H, fg_stream_t stream) {
  FG_REQUIRE(y && inv && indices && weights && out, "fg_moe_unpermute: null pointer");
  FG_REQUIRE(T >= 0 && k > 0 && k <= 8 && H > 0, "fg_moe_unpermute: bad sizes");
  if (T == 0) return FG_OK;
  return fg::launch_k("fg_moe_unpermute", fg::moe::unpermute_kernel, dim3(T), dim3(256), 0,
                      (cudaStream_t)stream, reinterpret_cast<const __nv_bfloat16*>(y), inv, indices,
                      reinterpret_cast<const __nv_bfloat16*>(weights),
                      reinterpret_cast<const __nv_bfloat16*>(residual),
                      reinterpret_cast<__nv_bfloat16*>(out), k, H);
}

size_t fg_mxfp4_packed_bytes(int E, int N, int K) {
  if (E <= 0 || N <= 0 || K <= 0) return 0;
  return (size_t)E * ((N + 127) / 128) * ((K + 63) / 64) * fg::moe::kRecBytes;
}

int fg_pack_mxfp4(const uint8_t* values, const uint8_t* scales, void* packed, int E, int N, int K,
                  fg_stream_t stream) {
  FG_REQUIRE(values && scales && packed, "fg_pack_mxfp4: null pointer");
  FG_REQUIRE(E > 0 && N > 0 && K > 0 && K % 32 == 0, "fg_pack_mxfp4: K=%d must be a multiple of 32", K);
  const int n_tiles = (N + 127) / 128, nkb = (K + 63) / 64;
  const long long records = (long long)E * n_tiles * nkb;
  return fg::launch_k("fg_pack_mxfp4", fg::moe::pack_mxfp4_kernel, dim3((unsigned)records), dim3(256),
                      0, (cudaStream_t)stream, values, scales, reinterpret_cast<uint8_t*>(packed), N, K,
                      n_tiles, nkb, records);
}

int fg_moe_gemm_mxfp4(const fg_bf16* x, const void* w_packed, const fg_bf16* bias,
                      const int32_t* offsets, const int32_t* items, const int32_t* item_count,
                      int max_items, fg_bf16* out, int rows, int N, int K, int BN, int epilogue,
                      fg_stream_t stream) {
  using namespace fg::moe;
  FG_REQUIRE(x && w_packed && offsets && items && item_count && out, "fg_moe_gemm_mxfp4: null pointer");
  FG_REQUIRE(rows >= 0 && N > 0 && K > 0 && K % 64 == 0, "fg_moe_gemm_mxfp4: bad sizes N=%d K=%d", N, K);
  FG_REQUIRE(epilogue == FG_EPI_STORE || epilogue == FG_EPI_SWIGLU_OAI,
             "fg_moe_gemm_mxfp4: epilogue must be FG_EPI_STORE or FG_EPI_SWIGLU_OAI");
  FG_REQUIRE(epilogue != FG_EPI_SWIGLU_OAI || N % 128 == 0,
             "fg_moe_gemm_mxfp4: SwiGLU needs N (=2*I) a multiple of 128");
  FG_REQUIRE(BN == 16 || BN == 32 || BN == 64, "fg_moe_gemm_mxfp4: BN must be 16, 32 or 64");
  FG_REQUIRE((((uintptr_t)x | (uintptr_t)w_packed) & 15) == 0, "fg_moe_gemm_mxfp4: alignment");
  if (rows == 0 || max_items == 0) return FG_OK;
  GemmParams p;
  p.w = reinterpret_cast<const uint8_t*>(w_packed);
  p.bias = reinterpret_cast<const __nv_bfloat16*>(bias);
  p.offsets = offsets;
  p.items = items;
  p.item_count = item_count;
  p.out = reinterpret_cast<__nv_bfloat16*>(out);
  p.N = N;
  p.K = K;
  p.n_tiles = (N + 127) / 128;
  p.nkb = K / 64;
  p.ldo = epilogue == FG_EPI_SWIGLU_OAI ? N / 2 : N;
  p.epilogue = epilogue;
  CUtensorMap tx;
  int rc = fg::make_tmap_2d_bf16(&tx, x, (uint64_t)K, (uint64_t)rows, (uint64_t)K * 2, 64, BN,
                                 CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  cudaStream_t st = (cudaStream_t)stream;
  auto go = [&](auto kern, int smem) -> int {
    static bool done[3][64] = {{false}};
    int dev = 0;
    cudaGetDevice(&dev);
    const int slot = BN == 16 ? 0 : (BN == 32 ? 1 : 2);
    if (!done[slot][dev & 63]) {
      cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
      if (e != cudaSuccess) {
        fg::set_last_error("fg_moe_gemm_mxfp4: cudaFuncSetAttribute: %s", cudaGetErrorString(e));
        return FG_ERR_CUDA;
      }
      done[slot][dev & 63] = true;
    }
    return fg::launch_k("fg_moe_gemm_mxfp4", kern, dim3(p.n_tiles, max_items), dim3(kMoeThreads), smem,
                        st, tx, p);
  };
  if (BN == 16) return go(moe_gemm_kernel<16, 4>, MLayout<16, 4>::DYN_SMEM);
  if (BN == 32) return go(moe_gemm_kernel<32, 4>, MLayout<32, 4>::DYN_SMEM);
  return go(moe_gemm_kernel<64, 4>, MLayout<64, 4>::DYN_SMEM);
}

}  // extern "C"
