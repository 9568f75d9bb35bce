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
// 32 elements along K). The products equal those of transformers' exact bf16
// dequantisation (convert_moe_packed_tensors); the values are decoded on the
// SM into tensor memory, so HBM moves 4.25 bits per weight and only for
// routed experts.
//
// Packed MXFP4 weight layout (fg_pack_mxfp4): per expert, per 128-row tile,
// per 64-wide K step, a 4352-byte record (layout at pack_mxfp4_kernel). For
// the fused SwiGLU-OAI epilogue the gate/up rows are interleaved in blocks of
// 64 as in the dense path (the caller orders rows before packing).
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
// router: logits rounded once from their exact value, top-k, softmax
// ---------------------------------------------------------------------------
// logit[t,e] is the bf16 nearest (ties to even) to the exact real number
// x[t] . w[e] + b[e]. Every bf16 x bf16 product is exact (16 significant
// bits), so the only rounding the reference's bf16 linear performs that is
// implementation-defined is its accumulation; summing the products exactly
// and rounding once gives the one result every faithful bf16 linear
// approximates, independent of reduction order. The CPU oracle computes the
// same number (an exactly rounded sum, then one bf16 rounding), so router
// indices can be compared with zero tolerance.
//
// Exact sums, two ways (both end in the same digit array and rounding):
//  * fast path, when every nonzero element of x and w[e] is a finite normal
//    bf16 and their exponents span at most kFastSpan binades: each product is
//    taken exactly in fp32 (a bf16 x bf16 product of normal operands whose
//    exponents keep it in fp32's normal range), placed at a fixed binary point
//    (the smallest product exponent of the row pair) into a 128-bit integer
//    per lane; lanes are summed with shuffles. No product can fall outside the
//    window, so nothing is lost.
//  * full-range path otherwise (subnormals, wide exponent spread): a Kulisch
//    accumulator, 18 digits of 32 bits (weights 2^-266 .. 2^310) covering
//    every bf16 x bf16 product, kept in shared memory per warp; lanes add
//    their products with 64-bit shared atomics (digit sums carry lazily).
// Non-finite inputs give a NaN logit.
namespace exact {

constexpr int kDigits = 18;     // 32-bit digits of the full-range accumulator
constexpr int kOrigin = 266;    // bit 0 of digit 0 weighs 2^-266 (the smallest product LSB)
constexpr int kFastSpan = 86;   // max (max - min) of summed biased exponents on the fast path

// bf16 bits -> exact (mantissa m >= 0, LSB exponent e): |v| = m * 2^e
__device__ __forceinline__ void decompose(uint32_t b, int& m, int& e) {
  const int field = (b >> 7) & 0xff;
  m = (int)(b & 0x7f) | (field ? 0x80 : 0);
  e = (field ? field : 1) - 134;
}

// per-row exponent statistics of bf16 words (two elements per u32):
// fmax: largest biased exponent field (0x7f80 = non-finite present),
// fmin: smallest field among nonzero elements (0 = a subnormal present)
struct ExpStats {
  uint32_t fmax = 0, fmin = 0x7f807f80u;
  __device__ __forceinline__ void add(uint32_t w) {
    const uint32_t f = w & 0x7f807f80u;
    const uint32_t zero = __vcmpeq2(w & 0x7fff7fffu, 0u);  // 0xffff in zero halves
    fmax = __vmaxu2(fmax, f);
    fmin = __vminu2(fmin, f | (zero & 0x7f807f80u));
  }
  __device__ __forceinline__ void add4(const uint4& v) {
    add(v.x); add(v.y); add(v.z); add(v.w);
  }
  // reduce over the warp; returns fields as plain integers
  __device__ __forceinline__ void reduce(int& hi, int& lo) const {
    uint32_t a = max(fmax >> 23, (fmax >> 7) & 0xffu);
    uint32_t b = min(fmin >> 23, (fmin >> 7) & 0xffu);
    hi = (int)__reduce_max_sync(0xffffffffu, a);
    lo = (int)__reduce_min_sync(0xffffffffu, b);
  }
};

// Round sign * sum_i D[i] 2^(32 i - kOrigin) (D normalised, 32-bit digits)
// to the nearest bf16, ties to even. Returns the bf16 bits.
__device__ uint16_t round_digits_bf16(const uint32_t* D, bool neg) {
  int top = -1;
  for (int i = kDigits - 1; i >= 0; --i)
    if (D[i]) {
      top = 32 * i + 31 - __clz(D[i]);
      break;
    }
  if (top < 0) return 0;  // exact zero: +0
  // bit position (frame) of the last kept bit: 8 significant bits, or the
  // bf16 subnormal quantum 2^-133
  int q = max(top - 7, kOrigin - 133);
  auto bit = [&](int p) -> uint32_t { return (D[p >> 5] >> (p & 31)) & 1u; };
  uint32_t kept = 0;
  for (int p = top; p >= q; --p) kept = (kept << 1) | bit(p);
  const uint32_t rbit = bit(q - 1);
  bool sticky = false;
  const int sp = q - 1;  // bits strictly below sp
  for (int i = 0; i < (sp >> 5); ++i) sticky |= D[i] != 0u;
  if (sp & 31) sticky |= (D[sp >> 5] & ((1u << (sp & 31)) - 1u)) != 0u;
  if (rbit && (sticky || (kept & 1u))) ++kept;
  if (kept == 256u) {
    kept = 128u;
    ++q;
  }
  uint32_t bits;
  if (kept < 128u) {
    bits = kept;  // subnormal (q is the subnormal quantum's position)
  } else {
    const int biased = q - kOrigin + 134;
    bits = biased >= 255 ? 0x7f80u : (((uint32_t)biased << 7) | (kept & 0x7fu));
  }
  return (uint16_t)(bits | (neg ? 0x8000u : 0u));
}

// Normalise lazily-carried int64 digit sums into 32-bit digits + sign and
// round (one thread).
__device__ uint16_t finish_digits(const long long* acc) {
  uint32_t D[kDigits];
  long long c = 0;
  for (int i = 0; i < kDigits; ++i) {
    const long long v = acc[i] + c;
    D[i] = (uint32_t)v;
    c = v >> 32;  // arithmetic: floor division
  }
  const bool neg = c < 0;
  if (neg) {  // two's complement negate
    uint32_t carry = 1;
    for (int i = 0; i < kDigits; ++i) {
      const uint64_t v = (uint64_t)(~D[i]) + carry;
      D[i] = (uint32_t)v;
      carry = (uint32_t)(v >> 32);
    }
  }
  return round_digits_bf16(D, neg);
}

// add the signed value v * 2^(pos - kOrigin), |v| < 2^32, to the
// lazily-carried digits as two pieces of magnitude < 2^32 (one thread)
__device__ __forceinline__ void add_at(long long* acc, long long v, int pos) {
  const long long t = v * (1ll << (pos & 31));  // |t| < 2^63
  acc[pos >> 5] += t & 0xffffffffll;
  acc[(pos >> 5) + 1] += t >> 32;  // arithmetic: t = hi * 2^32 + lo
}

// Exact dot product x . w (+ bias) of n8 groups of 8 bf16 over one warp;
// `acc` is this warp's kDigits shared-memory digits (lane 0 returns the
// bf16 bits of the rounded result). (xhi, xlo): the x row's exponent stats.
__device__ uint16_t warp_exact_dot(const uint4* __restrict__ xr, const uint4* __restrict__ wr, int n8,
                                   const __nv_bfloat16* bias, int xhi, int xlo, long long* acc, int lane) {
  ExpStats ws;
  for (int i = lane; i < n8; i += 32) ws.add4(wr[i]);
  int whi, wlo;
  ws.reduce(whi, wlo);
  const uint32_t bbits = bias ? (uint32_t)__bfloat16_as_ushort(*bias) : 0u;
  const bool nonfinite = xhi == 255 || whi == 255 || ((bbits >> 7) & 0xff) == 0xff;
  if (nonfinite) return 0x7fc0;  // NaN
  for (int i = lane; i < kDigits; i += 32) acc[i] = 0;
  __syncwarp();
  const bool any = xhi > 0 && whi > 0;  // both rows have a nonzero element
  const bool fast = any && xlo > 0 && wlo > 0 && (xhi + whi) - (xlo + wlo) <= kFastSpan &&
                    xlo + wlo >= 128 && xhi + whi <= 380;
  if (fast) {
    // fp32 product exponents lie in [xlo + wlo - 127, xhi + whi - 126]; the
    // binary point sits at the smallest: fp32 product bits (e, m24) land at
    // shift s = e - e0 in [0, kFastSpan + 1]; |sum| < 2^(24 + 87 + 14) < 2^127.
    const int e0 = xlo + wlo - 127;
    unsigned __int128 sum = 0;
    for (int i = lane; i < n8; i += 32) {
      const uint4 a = xr[i], b = wr[i];
      const uint32_t* pa = reinterpret_cast<const uint32_t*>(&a);
      const uint32_t* pb = reinterpret_cast<const uint32_t*>(&b);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float2 fa = unpack_bf16x2(pa[q]), fb = unpack_bf16x2(pb[q]);
        const float p2[2] = {__fmul_rn(fa.x, fb.x), __fmul_rn(fa.y, fb.y)};
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const uint32_t pbits = __float_as_uint(p2[h]);
          const int e = (int)((pbits >> 23) & 0xffu);
          if (e == 0) continue;  // a zero operand (nonzero products are normal here)
          const uint64_t m = (pbits & 0x7fffffu) | 0x800000u;
          const unsigned __int128 v = (unsigned __int128)m << (e - e0);
          sum = (pbits >> 31) ? sum - v : sum + v;
        }
      }
    }
    uint64_t lo = (uint64_t)sum, hi = (uint64_t)(sum >> 64);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const uint64_t olo = __shfl_xor_sync(0xffffffffu, lo, o);
      const uint64_t ohi = __shfl_xor_sync(0xffffffffu, hi, o);
      const uint64_t nlo = lo + olo;
      hi = hi + ohi + (nlo < lo ? 1u : 0u);
      lo = nlo;
    }
    if (lane == 0) {
      // sum * 2^(e0 - 150): fp32 significand LSB weight is 2^(e - 150);
      // the two's complement words go in at their positions, the top one signed
      const int pos = e0 - 150 + kOrigin;  // frame position of the sum's bit 0
      add_at(acc, (long long)(uint32_t)lo, pos);
      add_at(acc, (long long)(uint32_t)(lo >> 32), pos + 32);
      add_at(acc, (long long)(uint32_t)hi, pos + 64);
      add_at(acc, (long long)(int32_t)(hi >> 32), pos + 96);
    }
  } else if (any) {
    for (int i = lane; i < n8; i += 32) {
      const uint4 a = xr[i], b = wr[i];
      const uint32_t* pa = reinterpret_cast<const uint32_t*>(&a);
      const uint32_t* pb = reinterpret_cast<const uint32_t*>(&b);
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const uint32_t xa = (pa[q >> 1] >> (16 * (q & 1))) & 0xffffu;
        const uint32_t wb = (pb[q >> 1] >> (16 * (q & 1))) & 0xffffu;
        int mx, ex, mw, ew;
        decompose(xa, mx, ex);
        decompose(wb, mw, ew);
        const long long p = (long long)(mx * mw);
        if (p == 0) continue;
        const int pos = ex + ew + kOrigin;
        const long long v = p << (pos & 31);  // p > 0, < 2^47
        atomicAdd(reinterpret_cast<unsigned long long*>(acc + (pos >> 5)),
                  (unsigned long long)(((xa ^ wb) & 0x8000u) ? -v : v));
      }
    }
  }
  __syncwarp();
  if (lane != 0) return 0;
  if (bias) {
    int mb, eb;
    decompose(bbits, mb, eb);
    if (mb) add_at(acc, (bbits & 0x8000u) ? -(long long)mb : (long long)mb, eb + kOrigin);
  }
  return finish_digits(acc);
}

// bf16 nearest (ties to even) to a finite double
__device__ __forceinline__ uint16_t dbl_to_bf16(double v) {
  const uint64_t b = __double_as_longlong(v);
  const uint16_t sign = (uint16_t)((b >> 48) & 0x8000u);
  const int ef = (int)((b >> 52) & 0x7ff);
  if (ef == 0x7ff) return (uint16_t)(sign | 0x7fc0u);
  if (ef == 0) return sign;  // fp64 subnormals are far below bf16's range
  const uint64_t m = (b & 0xfffffffffffffull) | (1ull << 52);  // value = m * 2^(ef - 1075)
  // last kept bit: 8 significant bits, or the bf16 subnormal quantum 2^-133
  const int lsb_exp = max(ef - 1023 - 7, -133);
  const int drop = lsb_exp - (ef - 1075);  // >= 45
  if (drop >= 64) return sign;             // below half the smallest subnormal
  uint64_t kept = m >> drop;
  const uint64_t rem = m & ((1ull << drop) - 1), half = 1ull << (drop - 1);
  if (rem > half || (rem == half && (kept & 1))) ++kept;
  int e = lsb_exp;
  if (kept == 256) {
    kept = 128;
    ++e;
  }
  if (kept < 128) return (uint16_t)(sign | kept);
  const int biased = e + 7 + 127;
  if (biased >= 255) return (uint16_t)(sign | 0x7f80u);
  return (uint16_t)(sign | ((uint32_t)biased << 7) | (kept & 0x7f));
}

// The same logit through an fp64 sum with a rigorous error bound, when that
// settles it. A product of two bf16 values is exact in fp64 (8-bit
// significands; every bf16 value, subnormals included, is an fp64 normal),
// and any summation order of n exact terms in fp64 lands within
// gamma_(n-1) * sum|p_i| of the exact sum (u = 2^-53, gamma_k = k u/(1 - k u);
// all terms are multiples of 2^-266, far above fp64's subnormals, so the
// standard model holds). E = (n 2^-52) * (fp64 sum of |p_i|) is at least that
// bound with margin for the rounding of |p_i|'s own sum, and lo / hi = s -/+ 2E
// computed in fp64 still enclose the exact sum. Rounding to nearest even is
// monotone, so if lo and hi round to the same finite nonzero bf16, every real
// between them does too and that is the exact logit. Otherwise (a rounding
// midpoint within the bound, a result that rounds to zero or overflows, a
// non-finite input) returns false and warp_exact_dot decides. Every lane
// returns the same answer (lane 0's sums are broadcast).
__device__ bool warp_filtered_dot(const uint4* __restrict__ xr, const uint4* __restrict__ wr, int n8,
                                  const __nv_bfloat16* bias, int lane, uint16_t& out) {
  double s = 0.0, a = 0.0;
  for (int i = lane; i < n8; i += 32) {
    const uint4 xa = xr[i], wb = wr[i];
    const uint32_t* pa = reinterpret_cast<const uint32_t*>(&xa);
    const uint32_t* pb = reinterpret_cast<const uint32_t*>(&wb);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float2 fa = unpack_bf16x2(pa[q]), fb = unpack_bf16x2(pb[q]);
      const double p0 = __dmul_rn((double)fa.x, (double)fb.x);
      const double p1 = __dmul_rn((double)fa.y, (double)fb.y);
      s = __dadd_rn(__dadd_rn(s, p0), p1);
      a = __dadd_rn(__dadd_rn(a, fabs(p0)), fabs(p1));
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    s = __dadd_rn(s, __shfl_xor_sync(0xffffffffu, s, o));
    a = __dadd_rn(a, __shfl_xor_sync(0xffffffffu, a, o));
  }
  s = __shfl_sync(0xffffffffu, s, 0);
  a = __shfl_sync(0xffffffffu, a, 0);
  if (bias) {
    const double b = (double)__bfloat162float(*bias);
    s = __dadd_rn(s, b);
    a = __dadd_rn(a, fabs(b));
  }
  if (!isfinite(s) || !isfinite(a)) return false;
  const double n = 8.0 * n8 + 1.0;  // terms, the bias included
  const double e2 = 2.0 * __dmul_rn(a, n * 0x1p-52);
  const uint16_t r_lo = dbl_to_bf16(__dsub_rn(s, e2));
  const uint16_t r_hi = dbl_to_bf16(__dadd_rn(s, e2));
  if (r_lo != r_hi || (r_lo & 0x7fffu) == 0 || (r_lo & 0x7f80u) == 0x7f80u) return false;
  out = r_lo;
  return true;
}

}  // namespace exact

// Top-k of the E <= 64 logits a warp holds (lane e has experts e and e+32),
// by value with the lower expert id first on ties, then the softmax over the
// k selected: p_j = exp(v_j - v_0) in fp64, s = p_0 + ... + p_{k-1} in order,
// weight_j = bf16(p_j / s) rounded once. Lane 0 writes the k pairs.
__device__ __forceinline__ void warp_topk_softmax(float v0, float v1, int lane, int E, int k,
                                                  __nv_bfloat16* __restrict__ out_w,
                                                  int32_t* __restrict__ out_idx) {
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
    double p[8], s = 0.0;
    for (int j = 0; j < k; ++j) {
      p[j] = exp((double)sel_v[j] - (double)sel_v[0]);
      s += p[j];
    }
    for (int j = 0; j < k; ++j) {
      out_idx[j] = sel_i[j];
      out_w[j] = __ushort_as_bfloat16(exact::dbl_to_bf16(p[j] / s));
    }
  }
}

// One CTA of 32 warps per token: the x row's exponent statistics first (all
// warps), then warp w computes the exactly rounded logits of experts w, w+32
// (an fp64 sum with an error bound where that settles the rounding, the
// exact accumulation otherwise), and warp 0 selects the top-k.
__global__ void __launch_bounds__(1024) router_topk_kernel(
    const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ w,
    const __nv_bfloat16* __restrict__ bias, int H, int E, int k, __nv_bfloat16* __restrict__ out_w,
    int32_t* __restrict__ out_idx, __nv_bfloat16* __restrict__ out_logits) {
  griddep_wait();
  griddep_launch_dependents();
  __shared__ float logit[kMaxE];
  __shared__ long long digits[32][exact::kDigits];
  __shared__ int s_hi[32], s_lo[32];
  const int t = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint4* xr = reinterpret_cast<const uint4*>(x + (int64_t)t * H);
  const int H8 = H >> 3;
  {
    exact::ExpStats xs;
    for (int i = threadIdx.x; i < H8; i += blockDim.x) xs.add4(xr[i]);
    int hi, lo;
    xs.reduce(hi, lo);
    if (lane == 0) {
      s_hi[warp] = hi;
      s_lo[warp] = lo;
    }
  }
  __syncthreads();
  int xhi = 0, xlo = 255;
  for (int i = 0; i < 32; ++i) {
    xhi = max(xhi, s_hi[i]);
    xlo = min(xlo, s_lo[i]);
  }
  for (int e = warp; e < E; e += 32) {
    const uint4* wr = reinterpret_cast<const uint4*>(w + (int64_t)e * H);
    uint16_t b;
    if (!exact::warp_filtered_dot(xr, wr, H8, bias ? bias + e : nullptr, lane, b))
      b = exact::warp_exact_dot(xr, wr, H8, bias ? bias + e : nullptr, xhi, xlo, digits[warp], lane);
    if (lane == 0) {
      logit[e] = bf2f(__ushort_as_bfloat16(b));
      if (out_logits) out_logits[(int64_t)t * E + e] = __ushort_as_bfloat16(b);
    }
  }
  __syncthreads();
  if (warp == 0)
    warp_topk_softmax(lane < E ? logit[lane] : -INFINITY, lane + 32 < E ? logit[lane + 32] : -INFINITY,
                      lane, E, k, out_w + (int64_t)t * k, out_idx + (int64_t)t * k);
}

// Top-k and softmax of router logits that are already computed (the vLLM
// MoE runner receives them from the gate linear): one warp per token.
__global__ void __launch_bounds__(256) topk_softmax_kernel(const __nv_bfloat16* __restrict__ logits, int T,
                                                           int E, int k, __nv_bfloat16* __restrict__ out_w,
                                                           int32_t* __restrict__ out_idx) {
  griddep_wait();
  griddep_launch_dependents();
  const int lane = threadIdx.x & 31;
  const int t = blockIdx.x * 8 + (threadIdx.x >> 5);
  if (t >= T) return;
  const __nv_bfloat16* row = logits + (int64_t)t * E;
  warp_topk_softmax(lane < E ? bf2f(row[lane]) : -INFINITY, lane + 32 < E ? bf2f(row[lane + 32]) : -INFINITY,
                    lane, E, k, out_w + (int64_t)t * k, out_idx + (int64_t)t * k);
}

// ---------------------------------------------------------------------------
// permute: deterministic counting sort of (token, slot) pairs by expert
// ---------------------------------------------------------------------------
// One CTA of 32 warps. Pair p = t*k + j goes to row offsets[e] + rank, rank =
// number of earlier pairs (in p order) routed to the same expert.
__global__ void __launch_bounds__(1024) permute_kernel(
    const int32_t* __restrict__ idx, int n, int E, int BN, int e_lo, int e_hi, int max_items,
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
  __shared__ int tot[kMaxE], tile0[kMaxE + 1];
  __syncthreads();
  if (threadIdx.x < E) {
    int c = 0;
    for (int w = 0; w < 32; ++w) c += cnt[w][threadIdx.x];
    tot[threadIdx.x] = c;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    // expert row offsets and the first work item of each expert
    int run = 0, ti = 0;
    for (int e = 0; e < E; ++e) {
      base[e] = run;
      tile0[e] = ti;
      run += tot[e];
      if (e >= e_lo && e < e_hi) ti += (tot[e] + BN - 1) / BN;  // work items of this shard's experts
    }
    base[E] = run;
    tile0[E] = ti;
    *item_count = min(ti, max_items);
  }
  __syncthreads();
  if (threadIdx.x < E) {
    const int e = threadIdx.x;
    int run = base[e];
    for (int w = 0; w < 32; ++w) {
      const int c = cnt[w][e];
      cnt[w][e] = run;  // start of warp w's pairs for expert e
      run += c;
    }
    for (int i = tile0[e]; i < tile0[e + 1] && i < max_items; ++i) {
      items[2 * i] = e;
      items[2 * i + 1] = i - tile0[e];
    }
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

// bf16x2 -> f16x2 (exact in the f16 normal range)
__device__ __forceinline__ uint32_t bf16x2_to_f16x2(uint32_t w) {
  uint32_t r;
  asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(__uint_as_float(w & 0xFFFF0000u)),
      "f"(__uint_as_float(w << 16)));
  return r;
}

// rows of x in permuted order, as f16: out[i] = x[perm_pair[i] / k]
__global__ void gather_rows_kernel(const uint4* __restrict__ x, const int32_t* __restrict__ perm_pair,
                                   int k, int H8, uint4* __restrict__ out) {
  griddep_wait();
  griddep_launch_dependents();
  const int i = blockIdx.x;
  const int t = perm_pair[i] / k;
  const uint4* src = x + (int64_t)t * H8;
  uint4* dst = out + (int64_t)i * H8;
  for (int c = threadIdx.x; c < H8; c += blockDim.x) {
    const uint4 v = src[c];
    dst[c] = make_uint4(bf16x2_to_f16x2(v.x), bf16x2_to_f16x2(v.y), bf16x2_to_f16x2(v.z),
                        bf16x2_to_f16x2(v.w));
  }
}

// out[t] = residual[t] + sum over the k experts (ascending id) of y[inv] * w,
// each product and partial sum rounded to bf16 as transformers' index_add_
// accumulation does; 8 features per thread step (H % 8 == 0)
// With an expert range [e_lo, e_hi) only those slots count (an expert-parallel
// shard's part) and out_f32 writes the bf16-rounded sum as fp32 for
// fg_sum_partials.
__global__ void __launch_bounds__(128) unpermute_kernel(const __nv_bfloat16* __restrict__ y,
                                                        const int32_t* __restrict__ inv,
                                                        const int32_t* __restrict__ idx,
                                                        const __nv_bfloat16* __restrict__ wts,
                                                        const __nv_bfloat16* __restrict__ residual,
                                                        void* __restrict__ out_, int k, int H, int e_lo,
                                                        int e_hi, int out_f32) {
  griddep_wait();
  griddep_launch_dependents();
  __shared__ int s_row[8];
  __shared__ float s_w[8];
  __shared__ int s_k;
  const int t = blockIdx.x;
  if (threadIdx.x == 0) {
    int order[8], kk = 0;
    for (int j = 0; j < k; ++j) {
      const int e = idx[(int64_t)t * k + j];
      if (e >= e_lo && e < e_hi) order[kk++] = j;
    }
    // insertion sort of the counted slots by expert id (k <= 8), stable
    for (int a = 1; a < kk; ++a) {
      const int v = order[a];
      int b = a - 1;
      while (b >= 0 && idx[(int64_t)t * k + order[b]] > idx[(int64_t)t * k + v]) {
        order[b + 1] = order[b];
        --b;
      }
      order[b + 1] = v;
    }
    for (int a = 0; a < kk; ++a) {
      s_row[a] = inv[(int64_t)t * k + order[a]];
      s_w[a] = bf2f(wts[(int64_t)t * k + order[a]]);
    }
    s_k = kk;
  }
  __syncthreads();
  k = s_k;
  const int H8 = H >> 3;
  for (int c = threadIdx.x; c < H8; c += blockDim.x) {
    float acc[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] = 0.f;
    for (int a = 0; a < k; ++a) {
      const uint4 v = reinterpret_cast<const uint4*>(y + (int64_t)s_row[a] * H)[c];
      const uint32_t* pv = reinterpret_cast<const uint32_t*>(&v);
      const float wv = s_w[a];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 f = unpack_bf16x2(pv[i]);
        acc[2 * i] = rbf(acc[2 * i] + rbf(f.x * wv));
        acc[2 * i + 1] = rbf(acc[2 * i + 1] + rbf(f.y * wv));
      }
    }
    if (out_f32) {
      float4* o4 = reinterpret_cast<float4*>(reinterpret_cast<float*>(out_) + (int64_t)t * H) + 2 * c;
      o4[0] = make_float4(acc[0], acc[1], acc[2], acc[3]);
      o4[1] = make_float4(acc[4], acc[5], acc[6], acc[7]);
      continue;
    }
    uint4 o;
    uint32_t* po = reinterpret_cast<uint32_t*>(&o);
    if (residual) {
      const uint4 r = reinterpret_cast<const uint4*>(residual + (int64_t)t * H)[c];
      const uint32_t* pr = reinterpret_cast<const uint32_t*>(&r);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 f = unpack_bf16x2(pr[i]);
        po[i] = pack_bf16x2(f.x + acc[2 * i], f.y + acc[2 * i + 1]);
      }
    } else {
#pragma unroll
      for (int i = 0; i < 4; ++i) po[i] = pack_bf16x2(acc[2 * i], acc[2 * i + 1]);
    }
    reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(out_) + (int64_t)t * H)[c] = o;
  }
}

// ---------------------------------------------------------------------------
// MXFP4 packing: values [E][N][K/2] u8 + scales [E][N][K/32] u8 -> records
// ---------------------------------------------------------------------------
// Record (one expert, one 128-row tile, one 64-wide K step), 4352 bytes:
//   [0, 2048)     K elements 0..31:  row r's 16 bytes of e2m1 pairs at r*16
//   [2048, 4096)  K elements 32..63: row r at 2048 + r*16   (low nibble = even k)
//   [4096, 4352)  row r's two block codes at 4096 + 2r: c = s - s_ref(row) + 24
// The nkb records of one (expert, row tile) are followed by that tile's
// s_ref int32 [128] (tile stride = nkb * 4352 + 512 bytes), s_ref(row) =
// (largest exponent among the row's nonzero blocks) - 13. A block then dequantises
// exactly in f16 as e2m1 * 2^(c-24) (c in [1, 37]: magnitudes 2^-24 .. 49152,
// all multiples of the f16 subnormal step) and the epilogue multiplies the
// fp32 accumulator by 2^(s_ref-127): the products are the bf16-dequantised
// weights' products scaled by one power of two per row, so the result is
// that of the exact bf16 dequantisation. A nonzero block more than 36
// binades below its row's largest cannot be held exactly; packing records
// DEV_SCALE_RANGE for it (real checkpoints stay far inside the window).
constexpr int kRowRefBias = 13;
constexpr int kSrefBytes = BM * 4;

__host__ __device__ inline size_t tile_stride(int nkb) { return (size_t)nkb * kRecBytes + kSrefBytes; }

__global__ void mxfp4_rowref_kernel(const uint8_t* __restrict__ vals, const uint8_t* __restrict__ scales,
                                    uint8_t* __restrict__ packed, int E, int N, int K, int n_pad) {
  griddep_wait();
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (long long)E * n_pad) return;
  const long long e = i / n_pad;
  const int n = (int)(i % n_pad);
  int smax = -1;
  if (n < N) {
    const uint8_t* v = vals + (e * N + n) * (K / 2);
    const uint8_t* s = scales + (e * N + n) * (K / 32);
    for (int b = 0; b < K / 32; ++b) {
      const uint4 q = *reinterpret_cast<const uint4*>(v + b * 16);
      // nonzero if any nibble has a nonzero magnitude (sign-only codes are zeros)
      const bool nz = ((q.x | q.y | q.z | q.w) & 0x77777777u) != 0u;
      if (nz && (int)s[b] > smax) smax = s[b];
    }
  }
  const int nkb = K / BK;
  int32_t* sref = reinterpret_cast<int32_t*>(packed + ((size_t)e * (n_pad / BM) + n / BM) * tile_stride(nkb) +
                                             (size_t)nkb * kRecBytes);
  sref[n % BM] = (smax < 0 ? 127 : smax) - kRowRefBias;
}

__global__ void pack_mxfp4_kernel(const uint8_t* __restrict__ vals, const uint8_t* __restrict__ scales,
                                  uint8_t* __restrict__ packed, int N, int K, int n_tiles, int nkb,
                                  long long records) {
  griddep_wait();
  const long long rec = blockIdx.x;
  if (rec >= records) return;
  const int kb = (int)(rec % nkb);
  const int nt = (int)((rec / nkb) % n_tiles);
  const long long e = rec / ((long long)nkb * n_tiles);
  uint8_t* tile = packed + ((size_t)e * n_tiles + nt) * tile_stride(nkb);
  uint8_t* dst = tile + (size_t)kb * kRecBytes;
  const int32_t* sref = reinterpret_cast<const int32_t*>(tile + (size_t)nkb * kRecBytes);
  for (int i = threadIdx.x; i < kRecBytes; i += blockDim.x) {
    uint8_t v = 0;
    if (i < kValBytes) {
      const int h = i >> 11, r = (i & 2047) >> 4, j = i & 15;
      const int n = nt * BM + r, kk = kb * BK + (h * 16 + j) * 2;
      if (n < N && kk < K) v = vals[(e * N + n) * (K / 2) + (kk >> 1)];
    } else {
      const int q = i - kValBytes;
      const int r = q >> 1, blk = q & 1;
      const int n = nt * BM + r, kk = kb * BK + blk * 32;
      v = 24;  // multiplier 1 for padding (its values are zero)
      if (n < N && kk < K) {
        int c = (int)scales[(e * N + n) * (K / 32) + (kk >> 5)] - sref[r] + 24;
        if (c < 1) {
          const uint4 w = *reinterpret_cast<const uint4*>(vals + (e * N + n) * (K / 2) + (kk >> 1));
          if (((w.x | w.y | w.z | w.w) & 0x77777777u) != 0u) record_device_error(DEV_SCALE_RANGE, 0x320);
          c = 0;
        }
        v = (uint8_t)c;
      }
    }
    dst[i] = v;
  }
}

// ---------------------------------------------------------------------------
// MXFP4 x activation grouped GEMM (swap-AB). Weights are decoded (e2m1 ->
// f16 by the hardware conversion, times the block scale) straight into
// tensor memory and used as the A operand of tcgen05.mma kind::f16 (A from
// TMEM, B = the f16 activation tile from shared memory). Only the 4.25-bit
// records and the activation tiles cross shared memory, so the kernel
// streams HBM instead of saturating shared-memory bandwidth with expanded
// tiles.
//
// At decode sizes a 128 x 16 MMA covers only 1088 bytes of MXFP4, so the
// serial per-step paths bound it, not bandwidth: one MMA-issuing thread's
// (barrier wait, MMAs, commit, issue slots shared with the converters on
// its sub-partition) costs more than the tensor pipe's ~52 cycles per MMA,
// and one converter warpgroup's (record read, tcgen05.st, arrive) more than
// a step's share of HBM time. So the kernel is built for two resident CTAs
// per SM (two issuing threads, half the tensor memory and shared memory
// each), each issuing thread takes one barrier wait and one commit per step,
// and each CTA has two converter warpgroups on alternate steps.
//
// Persistent: two CTAs per SM walk the work units (permute item x 128-row
// tile) u = blockIdx.x + j * gridDim.x; a unit's K runs in steps of two
// 64-wide records. 16 warps:
//   warp 0       weight producer: one bulk copy per step into a ring
//   warp 2       activation producer: the step's 2-D TMA tiles into an
//                activation ring of its own, deeper than the A stages
//                (XS > AST; measured faster than sharing their indices)
//   warp 1       TMEM owner and MMA issuer (8 x K16 per step into one of
//                two accumulators, so the epilogue overlaps the next unit);
//                one commit per step frees the A stage, and the converters
//                hold a_full until the activation tile has landed
//   warps 4-11   converters, two warpgroups taking alternate steps (one
//                group's serial read -> store -> arrive chain per step was
//                the bound with one): a thread per weight row decodes its
//                128 values of the step into a TMEM A stage (tcgen05.st); the thread
//                that sees an A stage freed also frees that step's
//                activation stage (x_empty), so the MMA thread still takes
//                one wait and one commit per step
//   warps 12-15  epilogue: accumulator x 2^(s_ref-127) + bias, SwiGLU-OAI
//                (gate rows 0-63 of a tile, up rows 64-127; f16 out) or
//                store (bf16 out)
// ---------------------------------------------------------------------------
struct GemmParams {
  const uint8_t* w;           // packed tiles [E][n_tiles] of nkb records + s_ref[128]
  const __nv_bfloat16* bias;  // [E][N] (packed row order) or null
  const int32_t* offsets;     // [E+1] rows of each expert in x / out
  const int32_t* items;       // [max_items][2] = (expert, token tile)
  const int32_t* item_count;
  void* out;                  // [rows][ldo]: f16 after SwiGLU-OAI, else bf16
  int N, K, n_tiles, nkb, ldo, epilogue;
  int e_base;                 // expert id of the first packed expert (expert-parallel shards)
};

constexpr int kConvWarp0 = 4;
constexpr int kConvGroups = 2;  // converter warpgroups, taking alternate steps
constexpr int kEpiWarp0 = kConvWarp0 + 4 * kConvGroups;
constexpr int kMoeWarps = kEpiWarp0 + 4;
constexpr int kMoeThreads = kMoeWarps * 32;
constexpr int kMoeCtasPerSm = 2;

template <int BN>
struct MLayout {
  static constexpr int KS = 2;                                      // records per step
  static constexpr int AST = BN <= 32 ? 3 : 2;                     // TMEM A stages of KS * 32 columns
  static constexpr int DCOL0 = AST * KS * 32;                      // two accumulators of BN columns follow
  // weight ring (steps) and activation ring (steps, deeper than the A stages;
  // shared memory for two CTAs per SM bounds the pair)
  static constexpr int WS = BN == 16 ? 8 : 6;
  static constexpr int XS = BN == 64 ? 3 : 6;
  static constexpr int X_TILE = BN * BK * 2;                       // [BN][64] f16, 128B swizzle
  static constexpr int X_STAGE = KS * X_TILE;
  static constexpr int W_STAGE = KS * kRecBytes;
  static constexpr int W_OFFSET = XS * X_STAGE;
  static constexpr int XCH_OFFSET = W_OFFSET + WS * W_STAGE;       // bf16 [BN][64]
  static constexpr int BAR_OFFSET = (XCH_OFFSET + BN * 64 * 2 + 7) / 8 * 8;
  // w_full[WS] w_empty[WS] x_full[XS] x_empty[XS] a_full[A] a_empty[A] acc_full[2] acc_empty[2] mma_done
  static constexpr int MISC_OFFSET = BAR_OFFSET + (2 * WS + 2 * XS + 2 * AST + 5) * 8;
  static constexpr int TOTAL = MISC_OFFSET + 16;
  static constexpr int DYN_SMEM = TOTAL + 1024;  // + slack for the 1024-byte alignment
  static constexpr uint32_t TMEM_COLS = 256;     // half of the SM's: two CTAs per SM
  static_assert(X_TILE % 1024 == 0 && kRecBytes % 16 == 0, "stage alignment");
  static_assert(XS >= AST, "a step's activation stage is released after its A stage");
  static_assert(DCOL0 + 2 * BN <= (int)TMEM_COLS, "tensor memory budget");
  static_assert(kMoeCtasPerSm * (DYN_SMEM + 1024) <= 233472, "shared memory budget (two CTAs per SM)");
};

// instruction descriptor for kind::f16 with f16 A/B, fp32 D, K-major
__host__ __device__ constexpr uint32_t idesc_f16(int m, int n) {
  return (1u << 4) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

__device__ __forceinline__ void tc_mma_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(tmem_d),
      "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void tc_st32(uint32_t taddr, const uint32_t (&a)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,"
      "%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(a[4]), "r"(a[5]), "r"(a[6]), "r"(a[7]),
      "r"(a[8]), "r"(a[9]), "r"(a[10]), "r"(a[11]), "r"(a[12]), "r"(a[13]), "r"(a[14]), "r"(a[15]),
      "r"(a[16]), "r"(a[17]), "r"(a[18]), "r"(a[19]), "r"(a[20]), "r"(a[21]), "r"(a[22]), "r"(a[23]),
      "r"(a[24]), "r"(a[25]), "r"(a[26]), "r"(a[27]), "r"(a[28]), "r"(a[29]), "r"(a[30]), "r"(a[31])
      : "memory");
}

// eight e2m1 values (one 32-bit word, low nibble first) -> four f16x2 words
__device__ __forceinline__ void e2m1x8_to_f16x2(uint32_t v, uint32_t* o) {
  asm("{\n\t.reg .b8 b0, b1, b2, b3;\n\t"
      "mov.b32 {b0, b1, b2, b3}, %4;\n\t"
      "cvt.rn.f16x2.e2m1x2 %0, b0;\n\t"
      "cvt.rn.f16x2.e2m1x2 %1, b1;\n\t"
      "cvt.rn.f16x2.e2m1x2 %2, b2;\n\t"
      "cvt.rn.f16x2.e2m1x2 %3, b3;\n\t}"
      : "=r"(o[0]), "=r"(o[1]), "=r"(o[2]), "=r"(o[3])
      : "r"(v));
}

// f16 bits of 2^(c-24), c in [0, 37], in both halves
__device__ __forceinline__ uint32_t pow2_f16x2(uint32_t c) {
  const uint32_t h = c >= 10u ? (c - 9u) << 10 : 1u << c;
  return h | (h << 16);
}

__device__ __forceinline__ uint32_t hmul2_bits(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
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

// (expert, first row, end row, row tile) of work unit u
struct Unit {
  int e, row0, row_end, nt;
};
__device__ __forceinline__ Unit unit_of(const GemmParams& p, int u, int BN) {
  const int item = u / p.n_tiles;
  Unit w;
  w.nt = u - item * p.n_tiles;
  const int e = p.items[2 * item];  // global expert id: rows of x / out
  w.row0 = p.offsets[e] + p.items[2 * item + 1] * BN;
  w.row_end = p.offsets[e + 1];
  w.e = e - p.e_base;               // index into this shard's packed weights and biases
  return w;
}

template <int BN>
__global__ void __launch_bounds__(kMoeThreads, kMoeCtasPerSm)
    moe_gemm_kernel(const __grid_constant__ CUtensorMap tm_x, const GemmParams p) {
  using L = MLayout<BN>;
  constexpr int WS = L::WS, XS = L::XS, kKS = L::KS, kAStages = L::AST, kDCol0 = L::DCOL0;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t sbase = smem_u32(smem);
  const uint32_t w_full = sbase + L::BAR_OFFSET;
  const uint32_t w_empty = w_full + WS * 8;
  const uint32_t x_full = w_empty + WS * 8;
  const uint32_t x_empty = x_full + XS * 8;
  const uint32_t a_full = x_empty + XS * 8;
  const uint32_t a_empty = a_full + kAStages * 8;
  const uint32_t acc_full = a_empty + kAStages * 8;
  const uint32_t acc_empty = acc_full + 2 * 8;
  const uint32_t mma_done = acc_empty + 2 * 8;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::MISC_OFFSET);
  int* issued = reinterpret_cast<int*>(smem + L::MISC_OFFSET + 4);  // [0] weights, [1] activations
  __nv_bfloat16* xch = reinterpret_cast<__nv_bfloat16*>(smem + L::XCH_OFFSET);

  if (threadIdx.x == 0) {
    for (int s = 0; s < WS; ++s) {
      mbar_init(w_full + 8 * s, 1);
      mbar_init(w_empty + 8 * s, 4);  // the converter warps of the step's warpgroup
    }
    for (int s = 0; s < XS; ++s) {
      mbar_init(x_full + 8 * s, 1);
      mbar_init(x_empty + 8 * s, 1);  // one converter thread relays the MMA commit
    }
    for (int s = 0; s < kAStages; ++s) {
      mbar_init(a_full + 8 * s, 4);
      mbar_init(a_empty + 8 * s, 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(acc_full + 8 * b, 1);
      mbar_init(acc_empty + 8 * b, 4);
    }
    mbar_init(mma_done, 1);
    issued[0] = issued[1] = 0;
    fence_mbar_init();
    prefetch_tensormap(&tm_x);
  }
  // routing results come from the permute kernel; the tensor memory is
  // allocated only after the previous kernel has finished with the SM's
  griddep_wait();
  if (warp == 1) {
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
  if (threadIdx.x == 0) griddep_launch_dependents();

  const int U = *p.item_count * p.n_tiles;
  const int G = gridDim.x;
  const int my_units = (int)blockIdx.x < U ? (U - 1 - (int)blockIdx.x) / G + 1 : 0;
  const int nkb = p.nkb;
  const int nsteps = (nkb + kKS - 1) / kKS;  // steps per unit
  const int NS = my_units * nsteps;            // steps this CTA runs
  auto step_count = [&](int t) { return min(kKS, nkb - t * kKS); };  // records in step t of a unit

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- weight producer ----------------
      const uint64_t pol_w = l2_policy_evict_first();
      int g = 0;
      bool ok = true;
      for (int j = 0; j < my_units && ok; ++j) {
        const Unit w = unit_of(p, blockIdx.x + j * G, BN);
        const uint8_t* wrec = p.w + ((size_t)w.e * p.n_tiles + w.nt) * tile_stride(nkb);
        for (int t = 0; t < nsteps; ++t, ++g) {
          const int s = g % WS;
          if (!mbar_wait(w_empty + 8 * s, ((uint32_t)(g / WS) & 1u) ^ 1u, 0x321)) {
            ok = false;
            break;
          }
          const uint32_t bytes = (uint32_t)step_count(t) * kRecBytes;
          mbar_arrive_expect_tx(w_full + 8 * s, bytes);
          bulk_load(sbase + L::W_OFFSET + s * L::W_STAGE, wrec + (size_t)t * L::W_STAGE, bytes,
                    w_full + 8 * s, pol_w);
        }
      }
      issued[0] = g;
    }
  } else if (warp == 2) {
    if (lane == 0) {
      // ---------------- activation producer ----------------
      const uint64_t pol_x = l2_policy_evict_last();
      int g = 0;
      bool ok = true;
      for (int j = 0; j < my_units && ok; ++j) {
        const Unit w = unit_of(p, blockIdx.x + j * G, BN);
        for (int t = 0; t < nsteps; ++t, ++g) {
          const int s = g % XS;
          // stage s is free once the MMAs of step g - XS have completed
          if (!mbar_wait(x_empty + 8 * s, ((uint32_t)(g / XS) & 1u) ^ 1u, 0x322)) {
            ok = false;
            break;
          }
          const int cnt = step_count(t);
          mbar_arrive_expect_tx(x_full + 8 * s, (uint32_t)(cnt * L::X_TILE));
          for (int kk = 0; kk < cnt; ++kk)
            tma_load_2d_hint(sbase + s * L::X_STAGE + kk * L::X_TILE, &tm_x, x_full + 8 * s,
                             (t * kKS + kk) * BK, w.row0, pol_x);
        }
      }
      issued[1] = g;
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer ----------------
      constexpr uint32_t idesc = idesc_f16(BM, BN);
      int g = 0;
      bool ok = true;
      for (int j = 0; j < my_units && ok; ++j) {
        const int buf = j & 1;
        if (!mbar_wait(acc_empty + 8 * buf, ((uint32_t)(j >> 1) & 1u) ^ 1u, 0x323)) break;
        gemm::tc_fence_after();
        const uint32_t d = tmem + kDCol0 + buf * BN;
        for (int t = 0; t < nsteps; ++t, ++g) {
          const int sa = g % kAStages, sx = g % XS;
          // a_full also covers the step's activation tile: a converter saw
          // x_full before arriving (one wait per step on this thread); the
          // commit below frees the A stage, and through a converter the
          // activation stage
          if (!mbar_wait(a_full + 8 * sa, (uint32_t)(g / kAStages) & 1u, 0x324)) {
            ok = false;
            break;
          }
          gemm::tc_fence_after();
          const int cnt = step_count(t);
          for (int kk = 0; kk < cnt; ++kk) {
            const uint64_t bdesc = gemm::sw128_kmajor_desc(sbase + sx * L::X_STAGE + kk * L::X_TILE);
            const uint32_t a = tmem + sa * (kKS * 32) + kk * 32;
#pragma unroll
            for (int k16 = 0; k16 < BK / 16; ++k16)
              tc_mma_ts(d, a + k16 * 8, bdesc + 2 * k16, idesc, (t > 0 || kk > 0 || k16 > 0) ? 1u : 0u);
          }
          gemm::tc_commit(a_empty + 8 * sa);
        }
        if (ok) gemm::tc_commit(acc_full + 8 * buf);
      }
      // every MMA of this thread has completed before the CTA moves on
      gemm::tc_commit(mma_done);
      mbar_wait(mma_done, 0, 0x326);
    }
  } else if (warp >= kConvWarp0 && warp < kEpiWarp0) {
    // ---------------- converters ----------------
    // each warpgroup takes every kConvGroups-th step, so that many steps'
    // shared-memory reads and TMEM stores are in flight at once
    const int q = warp & 3;
    const int row = q * 32 + lane;  // weight row of this thread, also its TMEM lane
    for (int g = (warp - kConvWarp0) >> 2; g < NS; g += kConvGroups) {
      const int s = g % WS, sa = g % kAStages;
      if (!mbar_wait(w_full + 8 * s, (uint32_t)(g / WS) & 1u, 0x327)) break;
      if (!mbar_wait(a_empty + 8 * sa, ((uint32_t)(g / kAStages) & 1u) ^ 1u, 0x328)) break;
      gemm::tc_fence_after();
      // that wait saw the MMAs of step g - AST complete: their activation
      // stage may be refilled
      if (q == 0 && lane == 0 && g >= kAStages) mbar_arrive(x_empty + 8 * ((g - kAStages) % XS));
      const int cnt = step_count(g % nsteps);
      for (int kk = 0; kk < cnt; ++kk) {
        // weight row `row` of record kk: 64 e2m1 values -> 32 f16x2 columns
        const uint8_t* rec = smem + L::W_OFFSET + s * L::W_STAGE + kk * kRecBytes;
        const uint4 v0 = *reinterpret_cast<const uint4*>(rec + row * 16);
        const uint4 v1 = *reinterpret_cast<const uint4*>(rec + 2048 + row * 16);
        const uint32_t codes = *reinterpret_cast<const uint16_t*>(rec + kValBytes + 2 * row);
        const uint32_t m0 = pow2_f16x2(codes & 0xFFu), m1 = pow2_f16x2(codes >> 8);
        uint32_t a[32];
        e2m1x8_to_f16x2(v0.x, a + 0);
        e2m1x8_to_f16x2(v0.y, a + 4);
        e2m1x8_to_f16x2(v0.z, a + 8);
        e2m1x8_to_f16x2(v0.w, a + 12);
        e2m1x8_to_f16x2(v1.x, a + 16);
        e2m1x8_to_f16x2(v1.y, a + 20);
        e2m1x8_to_f16x2(v1.z, a + 24);
        e2m1x8_to_f16x2(v1.w, a + 28);
#pragma unroll
        for (int c = 0; c < 16; ++c) a[c] = hmul2_bits(a[c], m0);
#pragma unroll
        for (int c = 16; c < 32; ++c) a[c] = hmul2_bits(a[c], m1);
        tc_st32(tmem + ((uint32_t)(q * 32) << 16) + sa * (kKS * 32) + kk * 32, a);
      }
      asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
      gemm::tc_fence_before();
      // the step's activation tile must have landed before a_full releases the MMA
      if (q == 0) {
        int ok = 1;
        if (lane == 0) ok = mbar_wait(x_full + 8 * (g % XS), (uint32_t)(g / XS) & 1u, 0x325) ? 1 : 0;
        if (!__shfl_sync(0xffffffffu, ok, 0)) break;
      }
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(a_full + 8 * sa);
        mbar_arrive(w_empty + 8 * s);
      }
    }
  } else if (warp >= kEpiWarp0) {
    // ---------------- epilogue ----------------
    const int q = warp & 3;
    const int row = q * 32 + lane;
    // every epilogue warp runs all units (the named barriers below stay
    // matched); after a failed wait the rest are written as zeros unwaited
    bool failed = false;
    for (int j = 0; j < my_units; ++j) {
      const int buf = j & 1;
      const bool acc_ok = !failed && mbar_wait(acc_full + 8 * buf, (uint32_t)(j >> 1) & 1u, 0x329);
      failed = !acc_ok;
      gemm::tc_fence_after();
      const Unit w = unit_of(p, blockIdx.x + j * G, BN);
      const int nrow = w.nt * BM + row;
      const int32_t* sref = reinterpret_cast<const int32_t*>(
          p.w + ((size_t)w.e * p.n_tiles + w.nt) * tile_stride(p.nkb) + (size_t)p.nkb * kRecBytes);
      const float rs = ldexpf(1.f, sref[row] - 127);
      const float b = (p.bias && nrow < p.N) ? bf2f(p.bias[(size_t)w.e * p.N + nrow]) : 0.f;
      const uint32_t taddr = tmem + ((uint32_t)(q * 32) << 16) + kDCol0 + buf * BN;
      if (p.epilogue == FG_EPI_SWIGLU_OAI) {
        if (q >= 2) {
#pragma unroll 1
          for (int j0 = 0; j0 < BN; j0 += 16) {
            float v[16];
            gemm::tc_ld16(taddr + j0, v);
#pragma unroll
            for (int ii = 0; ii < 16; ++ii)
              xch[(j0 + ii) * 64 + (row - 64)] = f2bf(acc_ok ? v[ii] * rs + b : 0.f);
          }
        }
        asm volatile("bar.sync 1, 128;" ::: "memory");
        if (q < 2) {
          const int f = w.nt * 64 + row;
#pragma unroll 1
          for (int j0 = 0; j0 < BN; j0 += 16) {
            float v[16];
            gemm::tc_ld16(taddr + j0, v);
#pragma unroll
            for (int ii = 0; ii < 16; ++ii) {
              const int rr = w.row0 + j0 + ii;
              if (rr < w.row_end && nrow < p.N) {
                const float g = rbf((acc_ok ? v[ii] : 0.f) * rs + b);
                const float u = bf2f(xch[(j0 + ii) * 64 + row]);
                reinterpret_cast<__half*>(p.out)[(int64_t)rr * p.ldo + f] = __float2half_rn(swiglu_oai(g, u));
              }
            }
          }
        }
        gemm::tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(acc_empty + 8 * buf);
        asm volatile("bar.sync 1, 128;" ::: "memory");  // xch is free for the next unit
      } else {
#pragma unroll 1
        for (int j0 = 0; j0 < BN; j0 += 16) {
          float v[16];
          gemm::tc_ld16(taddr + j0, v);
          if (nrow >= p.N) continue;
#pragma unroll
          for (int ii = 0; ii < 16; ++ii) {
            const int rr = w.row0 + j0 + ii;
            if (rr < w.row_end)
              reinterpret_cast<__nv_bfloat16*>(p.out)[(int64_t)rr * p.ldo + nrow] =
                  f2bf((acc_ok ? v[ii] : 0.f) * rs + b);
          }
        }
        gemm::tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(acc_empty + 8 * buf);
      }
    }
  }

  gemm::tc_fence_before();
  __syncthreads();
  // no copy may land after the CTA exits: wait for each ring's last issued steps
  if (threadIdx.x == 0) {
    const int n = issued[0];
    for (int g = n - WS < 0 ? 0 : n - WS; g < n; ++g)
      mbar_wait(w_full + 8 * (g % WS), (uint32_t)(g / WS) & 1u, 0x32a);
  } else if (threadIdx.x == 64) {
    const int n = issued[1];
    for (int g = n - XS < 0 ? 0 : n - XS; g < n; ++g)
      mbar_wait(x_full + 8 * (g % XS), (uint32_t)(g / XS) & 1u, 0x32b);
  }
  __syncthreads();
  if (warp == 1) {
    gemm::tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(L::TMEM_COLS)
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
  FG_REQUIRE(T >= 0 && H > 0 && H % 8 == 0 && H <= 16384 && E > 0 && E <= fg::moe::kMaxE && k > 0 &&
                 k <= 8 && k <= E,
             "fg_moe_router_topk: bad sizes T=%d H=%d E=%d k=%d (H %% 8 == 0, H <= 16384, E <= 64, k <= 8)",
             T, H, E, k);
  FG_REQUIRE((((uintptr_t)x | (uintptr_t)w) & 15) == 0, "fg_moe_router_topk: x/w must be 16-byte aligned");
  if (T == 0) return FG_OK;
  return fg::launch_k("fg_moe_router_topk", fg::moe::router_topk_kernel, dim3(T), dim3(1024), 0,
                      (cudaStream_t)stream, reinterpret_cast<const __nv_bfloat16*>(x),
                      reinterpret_cast<const __nv_bfloat16*>(w),
                      reinterpret_cast<const __nv_bfloat16*>(bias), H, E, k,
                      reinterpret_cast<__nv_bfloat16*>(weights), indices,
                      reinterpret_cast<__nv_bfloat16*>(logits));
}

int fg_moe_topk_softmax(const fg_bf16* logits, int T, int E, int k, fg_bf16* weights, int32_t* indices,
                        fg_stream_t stream) {
  FG_REQUIRE(logits && weights && indices, "fg_moe_topk_softmax: null pointer");
  FG_REQUIRE(T >= 0 && E > 0 && E <= fg::moe::kMaxE && k > 0 && k <= 8 && k <= E,
             "fg_moe_topk_softmax: bad sizes (E <= 64, k <= 8)");
  if (T == 0) return FG_OK;
  return fg::launch_k("fg_moe_topk_softmax", fg::moe::topk_softmax_kernel, dim3((T + 7) / 8), dim3(256), 0,
                      (cudaStream_t)stream, reinterpret_cast<const __nv_bfloat16*>(logits), T, E, k,
                      reinterpret_cast<__nv_bfloat16*>(weights), indices);
}

int fg_moe_max_items(int T, int k, int E, int BN) {
  if (T <= 0 || k <= 0 || E <= 0 || BN <= 0) return 0;
  return E + (T * k + BN - 1) / BN;
}

int fg_moe_tile_tokens(int T, int k, int E) {
  // room for twice the mean rows per expert, so most experts stream their
  // weights once (one token tile)
  const int avg = (T * k + E - 1) / (E > 0 ? E : 1);
  return avg <= 8 ? 16 : (avg <= 16 ? 32 : 64);
}

int fg_moe_permute(const int32_t* indices, int T, int k, int E, int BN, int e_lo, int e_hi,
                   int32_t* offsets, int32_t* perm_pair, int32_t* inv, int32_t* items,
                   int32_t* item_count, fg_stream_t stream) {
  FG_REQUIRE(indices && offsets && perm_pair && inv && items && item_count,
             "fg_moe_permute: null pointer");
  FG_REQUIRE(T >= 0 && k > 0 && E > 0 && E <= fg::moe::kMaxE && (BN == 16 || BN == 32 || BN == 64),
             "fg_moe_permute: bad sizes");
  FG_REQUIRE(0 <= e_lo && e_lo < e_hi && e_hi <= E, "fg_moe_permute: bad expert range [%d, %d)", e_lo, e_hi);
  return fg::launch_k("fg_moe_permute", fg::moe::permute_kernel, dim3(1), dim3(1024), 0,
                      (cudaStream_t)stream, indices, T * k, E, BN, e_lo, e_hi, fg_moe_max_items(T, k, E, BN),
                      offsets, perm_pair, inv, items, item_count);
}

int fg_moe_gather(const fg_bf16* x, const int32_t* perm_pair, int T, int k, int H, fg_f16* out,
                  fg_stream_t stream) {
  FG_REQUIRE(x && perm_pair && out, "fg_moe_gather: null pointer");
  FG_REQUIRE(T >= 0 && k > 0 && H % 8 == 0, "fg_moe_gather: bad sizes");
  if (T == 0) return FG_OK;
  return fg::launch_k("fg_moe_gather", fg::moe::gather_rows_kernel, dim3(T * k), dim3(128), 0,
                      (cudaStream_t)stream, reinterpret_cast<const uint4*>(x), perm_pair, k, H / 8,
                      reinterpret_cast<uint4*>(out));
}

int fg_moe_unpermute(const fg_bf16* y, const int32_t* inv, const int32_t* indices,
                     const fg_bf16* weights, const fg_bf16* residual, void* out, int T, int k,
                     int H, int e_lo, int e_hi, int out_f32, fg_stream_t stream) {
  FG_REQUIRE(y && inv && indices && weights && out, "fg_moe_unpermute: null pointer");
  FG_REQUIRE(T >= 0 && k > 0 && k <= 8 && H > 0 && H % 8 == 0, "fg_moe_unpermute: bad sizes (H %% 8 == 0)");
  FG_REQUIRE(e_lo >= 0 && e_lo < e_hi, "fg_moe_unpermute: bad expert range [%d, %d)", e_lo, e_hi);
  FG_REQUIRE(!out_f32 || residual == nullptr, "fg_moe_unpermute: an fp32 partial takes no residual");
  FG_REQUIRE((((uintptr_t)y | (uintptr_t)out | (uintptr_t)residual) & 15) == 0,
             "fg_moe_unpermute: y/residual/out must be 16-byte aligned");
  if (T == 0) return FG_OK;
  return fg::launch_k("fg_moe_unpermute", fg::moe::unpermute_kernel, dim3(T), dim3(128), 0,
                      (cudaStream_t)stream, reinterpret_cast<const __nv_bfloat16*>(y), inv, indices,
                      reinterpret_cast<const __nv_bfloat16*>(weights),
                      reinterpret_cast<const __nv_bfloat16*>(residual), out, k, H, e_lo, e_hi, out_f32);
}

size_t fg_mxfp4_packed_bytes(int E, int N, int K) {
  if (E <= 0 || N <= 0 || K <= 0 || K % 64) return 0;
  return (size_t)E * ((N + 127) / 128) * fg::moe::tile_stride(K / 64);
}

int fg_pack_mxfp4(const uint8_t* values, const uint8_t* scales, void* packed, int E, int N, int K,
                  fg_stream_t stream) {
  FG_REQUIRE(values && scales && packed, "fg_pack_mxfp4: null pointer");
  FG_REQUIRE(E > 0 && N > 0 && K > 0 && K % 64 == 0, "fg_pack_mxfp4: K=%d must be a multiple of 64", K);
  FG_REQUIRE((((uintptr_t)values | (uintptr_t)packed) & 15) == 0, "fg_pack_mxfp4: values/packed alignment");
  const int n_tiles = (N + 127) / 128, nkb = K / 64, n_pad = n_tiles * 128;
  const long long records = (long long)E * n_tiles * nkb;
  uint8_t* out = reinterpret_cast<uint8_t*>(packed);
  const long long rows = (long long)E * n_pad;
  int rc = fg::launch_k("fg_pack_mxfp4(rows)", fg::moe::mxfp4_rowref_kernel, dim3((unsigned)((rows + 255) / 256)),
                        dim3(256), 0, (cudaStream_t)stream, values, scales, out, E, N, K, n_pad);
  if (rc) return rc;
  return fg::launch_k("fg_pack_mxfp4", fg::moe::pack_mxfp4_kernel, dim3((unsigned)records), dim3(256), 0,
                      (cudaStream_t)stream, values, scales, out, N, K, n_tiles, nkb, records);
}

int fg_moe_gemm_mxfp4(const fg_f16* x, const void* w_packed, const fg_bf16* bias,
                      const int32_t* offsets, const int32_t* items, const int32_t* item_count,
                      int max_items, void* out, int rows, int N, int K, int BN, int epilogue, int e_base,
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
  p.out = out;
  p.N = N;
  p.K = K;
  p.n_tiles = (N + 127) / 128;
  p.nkb = K / 64;
  p.ldo = epilogue == FG_EPI_SWIGLU_OAI ? N / 2 : N;
  p.epilogue = epilogue;
  p.e_base = e_base;
  CUtensorMap tx;
  int rc = fg::make_tmap_2d_bf16(&tx, x, (uint64_t)K, (uint64_t)rows, (uint64_t)K * 2, 64, BN,
                                 CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  cudaStream_t st = (cudaStream_t)stream;
  const int grid = std::min(kMoeCtasPerSm * fg::num_sms(), max_items * p.n_tiles);
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
    return fg::launch_k("fg_moe_gemm_mxfp4", kern, dim3(grid), dim3(kMoeThreads), smem, st, tx, p);
  };
  if (BN == 16) return go(moe_gemm_kernel<16>, MLayout<16>::DYN_SMEM);
  if (BN == 32) return go(moe_gemm_kernel<32>, MLayout<32>::DYN_SMEM);
  return go(moe_gemm_kernel<64>, MLayout<64>::DYN_SMEM);
}

}  // extern "C"
