// Small bandwidth-bound kernels of the decode step: embedding gather,
// RMSNorm, RoPE + paged KV append, greedy argmax and position advance.
//
// Each one moves a few hundred KB per decode step; they are written for
// 16-byte vector accesses and one CTA per token row.
#pragma once
#include "common.cuh"

namespace fg {

// ---------------------------------------------------------------------------
// embedding gather (runner.py:128-134 embed stage)
// ---------------------------------------------------------------------------
__global__ void embed_kernel(const int64_t* __restrict__ ids, const uint4* __restrict__ table,
                             uint4* __restrict__ out, int H8, int vocab) {
  griddep_wait();
  griddep_launch_dependents();
  const int t = blockIdx.x;
  const int64_t id = ids[t];
  const bool ok = id >= 0 && id < vocab;
  if (!ok && threadIdx.x == 0) record_device_error(DEV_BAD_INDEX, 1);
  const uint4* src = table + (ok ? id : 0) * (int64_t)H8;
  uint4* dst = out + (int64_t)t * H8;
  for (int i = threadIdx.x; i < H8; i += blockDim.x) dst[i] = ok ? src[i] : make_uint4(0, 0, 0, 0);
}

// ---------------------------------------------------------------------------
// RMSNorm: one CTA per row, fp32 statistics
// ---------------------------------------------------------------------------
template <int THREADS>
__device__ __forceinline__ float block_sum(float v, float* red) {
  v = warp_sum(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  if (l == 0) red[w] = v;
  __syncthreads();
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < THREADS / 32; ++i) s += red[i];
  return s;
}

template <int THREADS>
__global__ void __launch_bounds__(THREADS) rmsnorm_kernel(const uint4* __restrict__ x,
                                                          const uint4* __restrict__ w,
                                                          uint4* __restrict__ out, int H,
                                                          float eps, int mode) {
  griddep_wait();
  griddep_launch_dependents();
  __shared__ float red[THREADS / 32];
  const int H8 = H >> 3;
  const uint4* xr = x + (int64_t)blockIdx.x * H8;
  uint4* orow = out + (int64_t)blockIdx.x * H8;
  // rows up to 8192 wide stay in registers (4 x 8 values per thread)
  constexpr int kMaxVec = 4;
  uint4 xv[kMaxVec];
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < kMaxVec; ++j) {
    const int i = threadIdx.x + j * THREADS;
    if (i < H8) {
      xv[j] = xr[i];
      const uint32_t* p = reinterpret_cast<const uint32_t*>(&xv[j]);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        float2 f = unpack_bf16x2(p[q]);
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
        if (mode == FG_NORM_LLAMA) {
          po[q] = pack_bf16x2(g.x * rbf(f.x * rstd), g.y * rbf(f.y * rstd));
        } else {
          po[q] = pack_bf16x2(g.x * (f.x * rstd), g.y * (f.y * rstd));
        }
      }
      orow[i] = o;
    }
  }
}

// ---------------------------------------------------------------------------
// RoPE (rotate-half) + paged KV append, one decode token per sequence
// ---------------------------------------------------------------------------
// grid (B, nq + 2*nkv), block hd/2: thread i rotates the pair (i, i + hd/2).
// token b of qkv belongs to sequence seq_ids[b] (seq_ids null: sequence b,
// one token per sequence as in decode) at position positions[b]
__global__ void rope_kv_append_kernel(const __nv_bfloat16* __restrict__ qkv,
                                      const int32_t* __restrict__ seq_ids,
                                      const int32_t* __restrict__ positions,
                                      const float* __restrict__ inv_freq, float attn_scaling,
                                      const int32_t* __restrict__ block_table, int max_blocks,
                                      int num_blocks, __nv_bfloat16* __restrict__ q_out,
                                      __nv_bfloat16* __restrict__ k_cache,
                                      __nv_bfloat16* __restrict__ v_cache, int nq, int nkv, int hd,
                                      int block_size) {
  griddep_wait();
  griddep_launch_dependents();
  const int b = blockIdx.x;
  const int head = blockIdx.y;
  const int i = threadIdx.x;
  const int half = hd >> 1;
  const int width = (nq + 2 * nkv) * hd;
  const int pos = positions[b];
  const __nv_bfloat16* src = qkv + (int64_t)b * width + (int64_t)head * hd;

  float x1 = bf2f(src[i]);
  float x2 = bf2f(src[i + half]);
  float o1 = x1, o2 = x2;
  if (head < nq + nkv) {
    // cos/sin in fp32, scaled, then rounded to the activation dtype (bf16)
    const float ang = (float)pos * inv_freq[i];
    const float c = rbf(cosf(ang) * attn_scaling);
    const float s = rbf(sinf(ang) * attn_scaling);
    o1 = rbf(rbf(x1 * c) - rbf(x2 * s));
    o2 = rbf(rbf(x2 * c) + rbf(x1 * s));
  }
  if (head < nq) {
    __nv_bfloat16* dst = q_out + ((int64_t)b * nq + head) * hd;
    dst[i] = f2bf(o1);
    dst[i + half] = f2bf(o2);
    return;
  }
  const int seq = seq_ids ? seq_ids[b] : b;
  const int page = pos / block_size;
  int blk = (pos >= 0 && page < max_blocks) ? block_table[(int64_t)seq * max_blocks + page] : -1;
  if (blk < 0 || blk >= num_blocks) {
    if (i == 0) record_device_error(DEV_BAD_INDEX, 2);
    return;
  }
  const bool is_k = head < nq + nkv;
  const int g = is_k ? head - nq : head - nq - nkv;
  __nv_bfloat16* cache = is_k ? k_cache : v_cache;
  __nv_bfloat16* dst =
      cache + (((int64_t)blk * nkv + g) * block_size + (pos % block_size)) * (int64_t)hd;
  dst[i] = f2bf(o1);
  dst[i + half] = f2bf(o2);
}

// ---------------------------------------------------------------------------
// greedy argmax over a bf16 logits row (lowest index wins ties)
// ---------------------------------------------------------------------------
__device__ __forceinline__ void argmax_merge(float& v, int& i, float ov, int oi) {
  if (ov > v || (ov == v && oi < i)) {
    v = ov;
    i = oi;
  }
}

template <int THREADS>
__global__ void __launch_bounds__(THREADS) argmax_kernel(const __nv_bfloat16* __restrict__ logits,
                                                         int64_t* __restrict__ out, int V) {
  griddep_wait();
  griddep_launch_dependents();
  __shared__ float sv[THREADS / 32];
  __shared__ int si[THREADS / 32];
  const __nv_bfloat16* row = logits + (int64_t)blockIdx.x * V;
  float best = -INFINITY;
  int besti = 0x7fffffff;
  const bool vec = ((reinterpret_cast<uintptr_t>(row) & 15) == 0);
  if (vec) {
    const int V8 = V >> 3;
    const uint4* r8 = reinterpret_cast<const uint4*>(row);
    for (int j = threadIdx.x; j < V8; j += THREADS) {
      const uint4 u = r8[j];
      const uint32_t* p = reinterpret_cast<const uint32_t*>(&u);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float2 f = unpack_bf16x2(p[q]);
        argmax_merge(best, besti, f.x, j * 8 + 2 * q);
        argmax_merge(best, besti, f.y, j * 8 + 2 * q + 1);
      }
    }
    for (int j = (V8 << 3) + threadIdx.x; j < V; j += THREADS) argmax_merge(best, besti, bf2f(row[j]), j);
  } else {
    for (int j = threadIdx.x; j < V; j += THREADS) argmax_merge(best, besti, bf2f(row[j]), j);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, best, o);
    const int oi = __shfl_xor_sync(0xffffffffu, besti, o);
    argmax_merge(best, besti, ov, oi);
  }
  const int w = threadIdx.x >> 5;
  if ((threadIdx.x & 31) == 0) {
    sv[w] = best;
    si[w] = besti;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int k = 1; k < THREADS / 32; ++k) argmax_merge(best, besti, sv[k], si[k]);
    out[blockIdx.x] = besti;
  }
}

// ---------------------------------------------------------------------------
// plain paged KV append (already-rotated keys): T tokens, token t belongs to
// sequence seq[t] at position pos[t]. grid (T, 2*nkv), block hd/8 (16 B each)
// ---------------------------------------------------------------------------
__global__ void kv_append_kernel(const uint4* __restrict__ k, const uint4* __restrict__ v,
                                 const int32_t* __restrict__ seq, const int32_t* __restrict__ pos,
                                 const int32_t* __restrict__ block_table, int max_blocks,
                                 int num_blocks, uint4* __restrict__ k_cache,
                                 uint4* __restrict__ v_cache, int nkv, int hd8, int block_size) {
  griddep_wait();
  griddep_launch_dependents();
  const int t = blockIdx.x;
  const int head = blockIdx.y;
  const bool is_k = head < nkv;
  const int g = is_k ? head : head - nkv;
  const int b = seq[t];
  const int p = pos[t];
  const int page = p / block_size;
  const int blk = (b >= 0 && p >= 0 && page < max_blocks) ? block_table[(int64_t)b * max_blocks + page] : -1;
  if (blk < 0 || blk >= num_blocks) {
    if (threadIdx.x == 0) record_device_error(DEV_BAD_INDEX, 3);
    return;
  }
  const uint4* src = (is_k ? k : v) + ((int64_t)t * nkv + g) * hd8;
  uint4* dst = (is_k ? k_cache : v_cache) +
               (((int64_t)blk * nkv + g) * block_size + p % block_size) * hd8;
  for (int i = threadIdx.x; i < hd8; i += blockDim.x) dst[i] = src[i];
}

// out = bf16(a + b), 8 elements per thread
// out[i] = bf16(p[0][i] + p[1][i] + ... + p[S-1][i]), fp32 sums in shard order
__global__ void sum_partials_kernel(const float4* __restrict__ parts, int S, long long n4,
                                    uint2* __restrict__ out) {
  griddep_wait();
  griddep_launch_dependents();
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n4) return;
  float4 a = parts[i];
  for (int s = 1; s < S; ++s) {
    const float4 b = parts[(long long)s * n4 + i];
    a.x += b.x;
    a.y += b.y;
    a.z += b.z;
    a.w += b.w;
  }
  out[i] = make_uint2(pack_bf16x2(a.x, a.y), pack_bf16x2(a.z, a.w));
}

__global__ void add_kernel(const uint4* __restrict__ a, const uint4* __restrict__ b,
                           uint4* __restrict__ out, long long n8) {
  griddep_wait();
  griddep_launch_dependents();
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n8) return;
  const uint4 x = a[i], y = b[i];
  const uint32_t* px = reinterpret_cast<const uint32_t*>(&x);
  const uint32_t* py = reinterpret_cast<const uint32_t*>(&y);
  uint4 o;
  uint32_t* po = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const float2 fx = unpack_bf16x2(px[q]), fy = unpack_bf16x2(py[q]);
    po[q] = pack_bf16x2(fx.x + fy.x, fx.y + fy.y);
  }
  out[i] = o;
}

__global__ void advance_kernel(int32_t* positions, int32_t* seq_lens, int B) {
  griddep_wait();
  griddep_launch_dependents();
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b < B) {
    if (positions) positions[b] += 1;
    if (seq_lens) seq_lens[b] += 1;
  }
}

}  // namespace fg

extern "C" {

int fg_embed(const int64_t* ids, const fg_bf16* table, fg_bf16* out, int T, int H, int vocab,
             fg_stream_t stream) {
  FG_REQUIRE(ids && table && out, "fg_embed: null pointer");
  FG_REQUIRE(T >= 0 && H > 0 && vocab > 0 && H % 8 == 0, "fg_embed: bad sizes T=%d H=%d", T, H);
  FG_REQUIRE(((uintptr_t)table & 15) == 0 && ((uintptr_t)out & 15) == 0,
             "fg_embed: table/out must be 16-byte aligned");
  if (T == 0) return FG_OK;
  return fg::launch_k("fg_embed", fg::embed_kernel, dim3(T), dim3(128), 0, (cudaStream_t)stream,
                      ids, reinterpret_cast<const uint4*>(table), reinterpret_cast<uint4*>(out),
                      H / 8, vocab);
}

int fg_rmsnorm(const fg_bf16* x, const fg_bf16* weight, fg_bf16* out, int T, int H, float eps,
               int weight_mode, fg_stream_t stream) {
  FG_REQUIRE(x && weight && out, "fg_rmsnorm: null pointer");
  FG_REQUIRE(T >= 0 && H > 0 && H % 8 == 0 && H <= 8 * 256 * 4,
             "fg_rmsnorm: H=%d must be a multiple of 8 and <= 8192", H);
  FG_REQUIRE(weight_mode == FG_NORM_LLAMA || weight_mode == FG_NORM_FP32MUL,
             "fg_rmsnorm: bad weight_mode %d", weight_mode);
  FG_REQUIRE((((uintptr_t)x | (uintptr_t)weight | (uintptr_t)out) & 15) == 0,
             "fg_rmsnorm: pointers must be 16-byte aligned");
  if (T == 0) return FG_OK;
  return fg::launch_k("fg_rmsnorm", fg::rmsnorm_kernel<256>, dim3(T), dim3(256), 0,
                      (cudaStream_t)stream, reinterpret_cast<const uint4*>(x),
                      reinterpret_cast<const uint4*>(weight), reinterpret_cast<uint4*>(out), H, eps,
                      weight_mode);
}

static int rope_kv_append_launch(const fg_bf16* qkv, const int32_t* seq_ids, const int32_t* positions,
                                 const float* inv_freq, float attention_scaling, const int32_t* block_table,
                                 int max_blocks, int num_blocks, fg_bf16* q_out, fg_bf16* k_cache,
                                 fg_bf16* v_cache, int T, int nq, int nkv, int hd, int block_size,
                                 fg_stream_t stream) {
  FG_REQUIRE(qkv && positions && inv_freq && block_table && q_out && k_cache && v_cache,
             "fg_rope_kv_append: null pointer");
  FG_REQUIRE(T >= 0 && nq > 0 && nkv > 0 && nq % nkv == 0, "fg_rope_kv_append: bad heads");
  FG_REQUIRE(hd % 2 == 0 && hd <= 256 && block_size > 0 && max_blocks > 0 && num_blocks > 0,
             "fg_rope_kv_append: bad hd=%d / block_size=%d", hd, block_size);
  if (T == 0) return FG_OK;
  return fg::launch_k("fg_rope_kv_append", fg::rope_kv_append_kernel, dim3(T, nq + 2 * nkv),
                      dim3(hd / 2), 0, (cudaStream_t)stream,
                      reinterpret_cast<const __nv_bfloat16*>(qkv), seq_ids, positions, inv_freq,
                      attention_scaling, block_table, max_blocks, num_blocks,
                      reinterpret_cast<__nv_bfloat16*>(q_out),
                      reinterpret_cast<__nv_bfloat16*>(k_cache),
                      reinterpret_cast<__nv_bfloat16*>(v_cache), nq, nkv, hd, block_size);
}

int fg_rope_kv_append(const fg_bf16* qkv, const int32_t* positions, const float* inv_freq,
                      float attention_scaling, const int32_t* block_table, int max_blocks,
                      int num_blocks, fg_bf16* q_out, fg_bf16* k_cache, fg_bf16* v_cache, int B,
                      int nq, int nkv, int hd, int block_size, fg_stream_t stream) {
  return rope_kv_append_launch(qkv, nullptr, positions, inv_freq, attention_scaling, block_table, max_blocks,
                               num_blocks, q_out, k_cache, v_cache, B, nq, nkv, hd, block_size, stream);
}

int fg_rope_kv_append_tokens(const fg_bf16* qkv, const int32_t* seq_ids, const int32_t* positions,
                             const float* inv_freq, float attention_scaling, const int32_t* block_table,
                             int max_blocks, int num_blocks, fg_bf16* q_out, fg_bf16* k_cache,
                             fg_bf16* v_cache, int T, int nq, int nkv, int hd, int block_size,
                             fg_stream_t stream) {
  FG_REQUIRE(seq_ids, "fg_rope_kv_append_tokens: null seq_ids");
  return rope_kv_append_launch(qkv, seq_ids, positions, inv_freq, attention_scaling, block_table, max_blocks,
                               num_blocks, q_out, k_cache, v_cache, T, nq, nkv, hd, block_size, stream);
}

int fg_kv_append(const fg_bf16* k, const fg_bf16* v, const int32_t* seq_ids,
                 const int32_t* positions, const int32_t* block_table, int max_blocks,
                 int num_blocks, fg_bf16* k_cache, fg_bf16* v_cache, int T, int nkv, int hd,
                 int block_size, fg_stream_t stream) {
  FG_REQUIRE(k && v && seq_ids && positions && block_table && k_cache && v_cache,
             "fg_kv_append: null pointer");
  FG_REQUIRE(T >= 0 && nkv > 0 && hd > 0 && hd % 8 == 0 && block_size > 0 && max_blocks > 0 &&
                 num_blocks > 0,
             "fg_kv_append: bad sizes");
  FG_REQUIRE((((uintptr_t)k | (uintptr_t)v | (uintptr_t)k_cache | (uintptr_t)v_cache) & 15) == 0,
             "fg_kv_append: pointers must be 16-byte aligned");
  if (T == 0) return FG_OK;
  return fg::launch_k("fg_kv_append", fg::kv_append_kernel, dim3(T, 2 * nkv),
                      dim3(hd / 8 < 32 ? 32 : hd / 8), 0, (cudaStream_t)stream,
                      reinterpret_cast<const uint4*>(k), reinterpret_cast<const uint4*>(v), seq_ids,
                      positions, block_table, max_blocks, num_blocks,
                      reinterpret_cast<uint4*>(k_cache), reinterpret_cast<uint4*>(v_cache), nkv,
                      hd / 8, block_size);
}

int fg_argmax(const fg_bf16* logits, int64_t* out, int T, int V, fg_stream_t stream) {
  FG_REQUIRE(logits && out, "fg_argmax: null pointer");
  FG_REQUIRE(T >= 0 && V > 0, "fg_argmax: bad sizes");
  if (T == 0) return FG_OK;
  return fg::launch_k("fg_argmax", fg::argmax_kernel<1024>, dim3(T), dim3(1024), 0,
                      (cudaStream_t)stream, reinterpret_cast<const __nv_bfloat16*>(logits), out, V);
}

int fg_add_bf16(const fg_bf16* a, const fg_bf16* b, fg_bf16* out, long long n, fg_stream_t stream) {
  FG_REQUIRE(a && b && out, "fg_add_bf16: null pointer");
  FG_REQUIRE(n >= 0 && n % 8 == 0, "fg_add_bf16: n=%lld must be a multiple of 8", n);
  FG_REQUIRE((((uintptr_t)a | (uintptr_t)b | (uintptr_t)out) & 15) == 0,
             "fg_add_bf16: pointers must be 16-byte aligned");
  if (n == 0) return FG_OK;
  const long long n8 = n / 8;
  return fg::launch_k("fg_add_bf16", fg::add_kernel, dim3((unsigned)((n8 + 255) / 256)), dim3(256), 0,
                      (cudaStream_t)stream, reinterpret_cast<const uint4*>(a),
                      reinterpret_cast<const uint4*>(b), reinterpret_cast<uint4*>(out), n8);
}

int fg_sum_partials(const float* partials, int S, long long n, fg_bf16* out, fg_stream_t stream) {
  FG_REQUIRE(partials && out, "fg_sum_partials: null pointer");
  FG_REQUIRE(S >= 1 && n >= 0 && n % 4 == 0, "fg_sum_partials: S=%d n=%lld (n %% 4 == 0)", S, n);
  FG_REQUIRE((((uintptr_t)partials) & 15) == 0 && (((uintptr_t)out) & 7) == 0,
             "fg_sum_partials: alignment");
  if (n == 0) return FG_OK;
  const long long n4 = n / 4;
  return fg::launch_k("fg_sum_partials", fg::sum_partials_kernel, dim3((unsigned)((n4 + 255) / 256)),
                      dim3(256), 0, (cudaStream_t)stream, reinterpret_cast<const float4*>(partials), S, n4,
                      reinterpret_cast<uint2*>(out));
}

int fg_advance(int32_t* positions, int32_t* seq_lens, int B, fg_stream_t stream) {
  FG_REQUIRE(B >= 0, "fg_advance: bad B");
  if (B == 0 || (!positions && !seq_lens)) return FG_OK;
  return fg::launch_k("fg_advance", fg::advance_kernel, dim3((B + 255) / 256), dim3(256), 0,
                      (cudaStream_t)stream, positions, seq_lens, B);
}

}  // extern "C"
