/*
 * fgb200.h - C ABI of the B200 (sm_100a) decode-step kernels.
 *
 * This is the boundary a host binding (ctypes, cgo, JNI, a C++ runtime)
 * links against. Signatures hold plain pointers, sizes and a CUDA stream:
 * no torch or C++ types. Every entry point:
 *   - returns FG_OK (0) or an FG_ERR_* code; fg_last_error() gives the text;
 *   - only enqueues work on `stream` (asynchronous, no implicit sync);
 *   - never allocates device memory: scratch space ("workspace") is passed in
 *     by the caller, sized by the matching *_workspace_bytes() query.
 * Device buffers hold bf16 as raw 16-bit patterns (fg_bf16).
 *
 * Reference interfaces replaced (paths inside the FluidGPU project):
 *   fluidgpu_runtime/fluidgpu_torch/runner.py        CausalLMRunner (decode step)
 *   fluidgpu_runtime/fluidgpu_torch/kv_cache.py      LayerKVCache.update
 *   fluidgpu_runtime/fluidgpu_torch/comm.py          ProcessGroupComm.send/recv
 *   cpp_runtime/include/comm_backend.cu              pcie/rdma handlers, polling kernels
 */
#ifndef FGB200_H_
#define FGB200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef uint16_t fg_bf16;          /* bfloat16 bit pattern */
typedef uint16_t fg_f16;           /* IEEE binary16 bit pattern */
typedef struct CUstream_st* fg_stream_t; /* == cudaStream_t */

/* status codes (ProcessGroupComm raises AssertionError / RuntimeError in the
 * reference; a host binding maps these codes onto those exceptions) */
#define FG_OK 0
#define FG_ERR_ARG 1     /* bad argument: shape, alignment, null pointer */
#define FG_ERR_CUDA 2    /* CUDA runtime error while enqueueing */
#define FG_ERR_TIMEOUT 3 /* a bounded device wait gave up */
#define FG_ERR_PEER 4    /* peer buffer not mapped / peer access unavailable */

/* GEMM epilogues (fg_gemm_bf16) */
#define FG_EPI_STORE 0     /* out[t,n] = bf16(acc (+ bias)) */
#define FG_EPI_RESIDUAL 1  /* out[t,n] = bf16(residual[t,n] + bf16(acc (+ bias))) */
#define FG_EPI_SWIGLU 2    /* out[t,j] = bf16(silu(g) * u), g/u rows interleaved per 64 */
#define FG_EPI_SWIGLU_OAI 3 /* gpt-oss: (clamp(u,-7,7)+1) * g' * sigmoid(1.702 g'), g' = min(g,7) */
#define FG_EPI_F32 4       /* out[t,n] = acc (+ bias) (+ residual[t,n] if given), fp32 out: a
                            * tensor-parallel partial sum, added up by fg_sum_partials */

/* routes of fg_gemm_bf16_packed_routed */
#define FG_ROUTE_SPLIT 1     /* row t -> dst[t / dst_rows], row t % dst_rows */
#define FG_ROUTE_BROADCAST 2 /* row t -> every dst[d], row dst_row0 + t */

/* RMSNorm weight application (fg_rmsnorm) */
#define FG_NORM_LLAMA 0    /* w * bf16(x * rstd)    (LlamaRMSNorm)  */
#define FG_NORM_FP32MUL 1  /* bf16(w * (x * rstd))  (GptOssRMSNorm) */

/* ---- diagnostics ------------------------------------------------------- */

/* Text of the last host-side error on the calling thread. */
const char* fg_last_error(void);
/* ABI version; bumped on any signature change. */
int fg_version(void);
/* Number of kernels this library has launched in this process (all devices,
 * all threads): lets a caller count the device work of a region. */
unsigned long long fg_launch_count(void);
/* Copy the device status word of the current device into *status (0 = no
 * device-side failure since the last reset) and optionally reset it. The low
 * 8 bits hold the failure kind (1 pipeline wait timeout, 2 peer flag timeout,
 * 3 index out of range), the rest the failing site. Synchronises `stream`. */
int fg_device_status(unsigned int* status, int reset, fg_stream_t stream);

/* ---- decode-step kernels ------------------------------------------------ */

/* Embedding gather: out[t,:] = table[ids[t],:].
 * Replaces executor.run_stage("embed", embed_tokens) in
 * fluidgpu_torch/runner.py:128-134. Out-of-range ids write zeros and set the
 * device status (index out of range). */
int fg_embed(const int64_t* ids, const fg_bf16* table, fg_bf16* out, int T, int H, int vocab,
             fg_stream_t stream);

/* RMSNorm over rows of x[T,H]: layer.input_layernorm / post_attention_layernorm
 * / model.norm as called at fluidgpu_torch/runner.py:183, :350 and :168.
 * weight_mode is FG_NORM_LLAMA or FG_NORM_FP32MUL. */
int fg_rmsnorm(const fg_bf16* x, const fg_bf16* weight, fg_bf16* out, int T, int H, float eps,
               int weight_mode, fg_stream_t stream);

/* Dense bf16 GEMM on tcgen05 tensor cores, fp32 accumulation in TMEM:
 *   acc[t,n] = sum_k x[t,k] * w[n,k]      x:[T,K] row-major, w:[N,K] row-major
 * with the epilogue `epilogue` (FG_EPI_*). For FG_EPI_SWIGLU, w holds the
 * gate and up projections interleaved in blocks of 64 rows (gate rows
 * j..j+63, then up rows j..j+63) and out is [T, N/2].
 * Replaces the nn.Linear calls q/k/v/o_proj, gate/up/down_proj and lm_head
 * at fluidgpu_torch/runner.py:273-276, :347, :420, :430, :168.
 * K must be a multiple of 8 (16-byte rows); x, w 16-byte aligned.
 * The work (output tiles x 64-wide K steps) is spread evenly over a
 * persistent grid (stream-K); splits = 0 sizes that grid to the SMs,
 * splits > 0 cuts every tile into about `splits` K slices instead. Tiles
 * shared by several CTAs are reduced through `workspace`
 * (fg_gemm_workspace_bytes bytes, 256-byte aligned; 0 means none needed).
 * The first 64 KiB of the workspace hold reduction tickets: zero them once
 * before the first call; every call leaves them zero again, so one workspace
 * serves calls of any shape in stream order. Calls that overlap on the GPU
 * must not share a workspace. */
int fg_gemm_bf16(const fg_bf16* x, const fg_bf16* w, fg_bf16* out, const fg_bf16* residual,
                 const fg_bf16* bias, int T, int N, int K, int epilogue, int splits,
                 void* workspace, size_t workspace_bytes, fg_stream_t stream);
/* Same GEMM with the weight in the packed tile layout of fg_pack_weight_bf16:
 * each CTA then streams whole 16 KB tiles with 1-D bulk copies. */
int fg_gemm_bf16_packed(const fg_bf16* x, const void* w_packed, fg_bf16* out,
                        const fg_bf16* residual, const fg_bf16* bias, int T, int N, int K,
                        int epilogue, int splits, void* workspace, size_t workspace_bytes,
                        fg_stream_t stream);
/* fg_gemm_bf16_packed whose result goes straight to other ranks' buffers
 * and announces itself there: the hand-off of the disaggregated step made by
 * the producing kernel, in place of the reference's NCCL send at the task
 * boundary (fluidgpu_torch/executor.py:104-123, comm.py:24-46).
 *   route FG_ROUTE_SPLIT     : result row t (a token) -> dst[t / dst_rows] at
 *                              row t % dst_rows (rows of several ranks' batches
 *                              back to their ranks)
 *   route FG_ROUTE_BROADCAST : row t -> every dst[d] at row dst_row0 + t (one
 *                              rank's rows to each shard of a sharded group)
 * dst holds n_dst <= 8 row-major buffers of row stride N (fp32 for
 * FG_EPI_F32, else bf16), usually peer memory mapped through CUDA IPC. When
 * every CTA has stored, the last one (counted on `ticket`, a zeroed u32 of
 * this GPU that the call leaves zero again; one per call site) release-stores
 * epoch[0] * seq_mul + seq_add into each of the n_sig <= 8 u32 flags
 * (system scope), which fg_rmsnorm_wait / fg_sum_rmsnorm_wait on the
 * receiving GPU wait for. Epilogues STORE, RESIDUAL (residual local, [T,N])
 * and F32; decode-size T only (the cluster kernel's plans). The pointer
 * arrays are read at the call (copied into the launch). No counterpart in
 * the reference. */
int fg_gemm_bf16_packed_routed(const fg_bf16* x, const void* w_packed, const fg_bf16* residual,
                               const fg_bf16* bias, int T, int N, int K, int epilogue, int route,
                               void* const* dst, int n_dst, int dst_rows, int dst_row0,
                               uint32_t* const* sig_flags, int n_sig, const uint32_t* epoch,
                               uint32_t seq_mul, uint32_t seq_add, uint32_t* ticket,
                               fg_stream_t stream);
/* Pack a row-major weight w:[N,K] into [ceil(N/128)][ceil(K/64)] tiles of
 * 128 x 64 bf16 (16 KB), each stored as the 128-byte-swizzled K-major image
 * the tensor cores read (16-byte chunk c of row r at chunk c ^ (r % 8));
 * padding is zero. `packed` holds fg_packed_weight_bytes(N, K) bytes. */
int fg_pack_weight_bf16(const fg_bf16* w, void* packed, int N, int K, fg_stream_t stream);
size_t fg_packed_weight_bytes(int N, int K);
/* Launch shape fg_gemm_bf16 plans for (T, N, K, splits): fg_gemm_grid is the
 * number of CTAs of a persistent (many-token) plan, or of output tiles of a
 * decode plan, each tile then run by fg_gemm_split CTAs along K (a thread-
 * block cluster reducing through distributed shared memory); a persistent
 * plan's split is 1. */
int fg_gemm_grid(int T, int N, int K, int splits);
int fg_gemm_split(int T, int N, int K, int splits);
/* Workspace bytes fg_gemm_bf16 needs for (T, N, K, splits). 0 if none. */
size_t fg_gemm_workspace_bytes(int T, int N, int K, int splits);

/* RoPE + paged KV append for one decode token per sequence.
 * qkv:[B, (nq+2*nkv)*hd] (q heads, then k heads, then v heads; bf16)
 * positions:[B] int32 = index of the new token in its sequence
 * cos/sin are computed from inv_freq:[hd/2] fp32 and attention_scaling,
 * rounded to bf16 as the HF rotary embedding does; rotation uses the
 * rotate-half convention (apply_rotary_pos_emb).
 * Writes q_out:[B, nq, hd] and the roped k / raw v of token b into
 * k_cache/v_cache:[num_blocks, nkv, block_size, hd] at block
 * block_table[b*max_blocks + pos/block_size], offset pos%block_size.
 * Replaces q/k/v split + apply_rotary_pos_emb + LayerKVCache.update
 * (fluidgpu_torch/runner.py:268-293, kv_cache.py:73-113). */
int fg_rope_kv_append(const fg_bf16* qkv, const int32_t* positions, const float* inv_freq,
                      float attention_scaling, const int32_t* block_table, int max_blocks,
                      int num_blocks, fg_bf16* q_out, fg_bf16* k_cache, fg_bf16* v_cache, int B,
                      int nq, int nkv, int hd, int block_size, fg_stream_t stream);
/* fg_rope_kv_append for T tokens of any sequences: token t (row t of qkv and
 * q_out) belongs to sequence seq_ids[t] at position positions[t] (a prefill
 * chunk: S consecutive positions per sequence). */
int fg_rope_kv_append_tokens(const fg_bf16* qkv, const int32_t* seq_ids, const int32_t* positions,
                             const float* inv_freq, float attention_scaling, const int32_t* block_table,
                             int max_blocks, int num_blocks, fg_bf16* q_out, fg_bf16* k_cache,
                             fg_bf16* v_cache, int T, int nq, int nkv, int hd, int block_size,
                             fg_stream_t stream);

/* Paged KV append of already-rotated keys: token t (k,v:[T, nkv, hd]) of
 * sequence seq_ids[t] at position positions[t] goes to its page slot. The
 * LayerKVCache.update surface (fluidgpu_torch/kv_cache.py:73-113) on the
 * paged layout; used where RoPE ran elsewhere (prefill, foreign callers). */
int fg_kv_append(const fg_bf16* k, const fg_bf16* v, const int32_t* seq_ids,
                 const int32_t* positions, const int32_t* block_table, int max_blocks,
                 int num_blocks, fg_bf16* k_cache, fg_bf16* v_cache, int T, int nkv, int hd,
                 int block_size, fg_stream_t stream);

/* Paged GQA decode attention, one query token per sequence.
 * q:[B, nq, hd]; k_cache/v_cache:[num_blocks, nkv, block_size, hd];
 * block_table:[B, max_blocks] int32; seq_lens:[B] int32 (tokens to attend,
 * including the new one). window > 0 keeps only the last `window` tokens
 * (transformers' sliding-window mask: kv > q - window). sinks:[nq] fp32 or
 * NULL adds exp(sink) to each head's softmax denominator (gpt-oss s_aux).
 * out:[B, nq*hd] bf16. Split-K over pages; partials live in `workspace`
 * (fg_attn_workspace_bytes). Requires hd in {64,128}, block_size == 16.
 * Replaces eager_attention_forward / SDPA over LayerKVCache
 * (fluidgpu_torch/runner.py:299-335, masks :713-823, sinks :914-920). */
int fg_paged_decode_attn(const fg_bf16* q, const fg_bf16* k_cache, const fg_bf16* v_cache,
                         const int32_t* block_table, const int32_t* seq_lens, const float* sinks,
                         fg_bf16* out, void* workspace, size_t workspace_bytes, int B, int nq,
                         int nkv, int hd, int block_size, int num_blocks, int max_blocks,
                         int max_seq_len, int window, float scale, fg_stream_t stream);
/* Slices per (sequence, kv head) fg_paged_decode_attn plans for a batch of
 * B sequences of at most max_seq_len tokens (window as in
 * fg_paged_decode_attn): chosen so the B*nkv*slices CTAs fill whole waves of
 * the GPU. Each sequence's actual pages are split evenly over its slices.
 * 0 on bad sizes. */
int fg_attn_splits(int B, int nkv, int hd, int max_seq_len, int window);
/* Workspace bytes fg_paged_decode_attn needs for these sizes (0 if none). */
size_t fg_attn_workspace_bytes(int B, int nq, int nkv, int hd, int max_seq_len, int window);

/* Causal prefill attention over the paged cache: q [B*S][nq][hd] holds S
 * consecutive query positions per sequence starting at first_pos[b] (their
 * K/V already appended, earlier context cached before them); query at
 * position p attends keys k <= p (and k > p - window when window > 0), sinks
 * as in fg_paged_decode_attn. out [B*S][nq][hd] bf16. nq/nkv must divide 64.
 * Replaces the reference's prefill attention over the whole prompt
 * (runner.py:66-116 with the masks of :713-823). */
int fg_prefill_attn(const fg_bf16* q, const fg_bf16* k_cache, const fg_bf16* v_cache,
                    const int32_t* block_table, const int32_t* first_pos, const float* sinks, fg_bf16* out,
                    int B, int S, int nq, int nkv, int hd, int block_size, int num_blocks, int max_blocks,
                    int window, float scale, fg_stream_t stream);

/* Paged decode attention for callers that cannot allocate device memory (a
 * runtime that owns all device memory through its own pool and refuses
 * cudaMalloc while serving, or an FFI binding without a device allocator).
 * No counterpart in the reference: it exists for such hosts. Same arguments
 * and results as fg_paged_decode_attn, minus the workspace: the split
 * scratch is a built-in 8 MiB device array that every GPU loading this
 * library holds until exit. The first call on a device resolves that
 * array's address (make it before any stream capture); calls needing more
 * than 8 MiB (fg_attn_workspace_bytes) fail with FG_ERR_ARG; calls share
 * the array, so calls that overlap on the GPU race. Allocates nothing. */
int fg_paged_decode_attn_noalloc(const fg_bf16* q, const fg_bf16* k_cache, const fg_bf16* v_cache,
                                 const int32_t* block_table, const int32_t* seq_lens,
                                 const float* sinks, fg_bf16* out, int B, int nq, int nkv, int hd,
                                 int block_size, int num_blocks, int max_blocks, int max_seq_len,
                                 int window, float scale, fg_stream_t stream);

/* Greedy token: out[t] = argmax_v logits[t, v] (lowest index on ties), the
 * argmax the reference engine takes after norm_lm_head (engine.py:295-300,
 * :337-343). */
int fg_argmax(const fg_bf16* logits, int64_t* out, int T, int V, fg_stream_t stream);

/* ---- gpt-oss MoE feed-forward (runner.py:432-457 moe_router / moe_experts /
 * moe_combine; GptOssMLP semantics; vllm_integration.py:452-485) -------- */

/* Router: logits[t,e] = bf16(x[t] . w[e] + bias[e]) (w:[E,H]), top-k by value
 * (ties: lower expert id), weights = bf16(softmax over the k selected logits).
 * weights,indices:[T,k]; logits:[T,E] or NULL. E <= 64, k <= 8. */
int fg_moe_router_topk(const fg_bf16* x, const fg_bf16* w, const fg_bf16* bias, int T, int H, int E,
                       int k, fg_bf16* weights, int32_t* indices, fg_bf16* logits,
                       fg_stream_t stream);
/* Top-k + softmax of given router logits [T,E] (the vLLM MoE runner's input,
 * vllm_integration.py:452-464: topk over the logits, softmax over the
 * selected): ties to the lower expert id, weights = bf16(softmax in fp32).
 * weights,indices:[T,k]. E <= 64, k <= 8. */
int fg_moe_topk_softmax(const fg_bf16* logits, int T, int E, int k, fg_bf16* weights, int32_t* indices,
                        fg_stream_t stream);
/* Token tile (16/32/64) the expert GEMMs use for T tokens, and the bound on
 * (expert, token tile) work items fg_moe_permute emits. */
int fg_moe_tile_tokens(int T, int k, int E);
int fg_moe_max_items(int T, int k, int E, int BN);
/* Deterministic counting sort of the T*k (token, slot) pairs by expert:
 * offsets:[E+1] rows of each expert; perm_pair:[T*k] pair id (t*k+j) of each
 * permuted row (pairs of one expert stay in (t, j) order); inv:[T*k] row of
 * each pair; items:[fg_moe_max_items][2] (expert, token tile), item_count:[1]. */
int fg_moe_permute(const int32_t* indices, int T, int k, int E, int BN, int e_lo, int e_hi,
                   int32_t* offsets, int32_t* perm_pair, int32_t* inv, int32_t* items,
                   int32_t* item_count, fg_stream_t stream);
/* out[i,:] = x[perm_pair[i] / k, :] for the T*k permuted rows, as f16 (the
 * operand type of fg_moe_gemm_mxfp4; every bf16 value with |x| >= 2^-17 is
 * exact in f16, smaller ones round to the f16 subnormal step 2^-24). */
int fg_moe_gather(const fg_bf16* x, const int32_t* perm_pair, int T, int k, int H, fg_f16* out,
                  fg_stream_t stream);
/* Pack MXFP4 expert weights: values:[E][N][K/2] (e2m1 pairs, low nibble =
 * even k), scales:[E][N][K/32] (e8m0) -> records of 128 rows x 64 K
 * (4096 B values + 256 B scales), fg_mxfp4_packed_bytes(E,N,K) bytes. */
int fg_pack_mxfp4(const uint8_t* values, const uint8_t* scales, void* packed, int E, int N, int K,
                  fg_stream_t stream);
size_t fg_mxfp4_packed_bytes(int E, int N, int K);
/* Grouped expert GEMM on tcgen05: for every work item (expert e, token tile),
 * acc = x[rows of e] . W_e^T with W_e packed MXFP4 [N,K] (fg_pack_mxfp4) and
 * x f16 rows [rows,K]. The weights are decoded on the SM into tensor memory
 * (e2m1 -> f16, times the block scale relative to a per-row reference
 * exponent, exact) and multiplied with fp32 accumulation; the accumulator is
 * rescaled by the row's reference power of two, so the result is that of the
 * exact bf16 dequantisation transformers performs. Epilogue FG_EPI_STORE
 * (+ bias[e]) -> out: bf16 [rows,N]; FG_EPI_SWIGLU_OAI (+ bias, gate/up rows
 * interleaved per 64, SwiGLU-OAI rounded to bf16 per op) -> out: f16
 * [rows,N/2] (the bf16 values, the next call's operand). Only experts that
 * received tokens read their weights. w_packed holds experts e_base, e_base+1,
 * ... (an expert-parallel shard's slice; 0 for all experts). */
int fg_moe_gemm_mxfp4(const fg_f16* x, const void* w_packed, const fg_bf16* bias,
                      const int32_t* offsets, const int32_t* items, const int32_t* item_count,
                      int max_items, void* out, int rows, int N, int K, int BN, int epilogue, int e_base,
                      fg_stream_t stream);
/* out[t] = residual[t] + sum over the k slots in ascending expert id of
 * bf16(y[inv[t*k+j]] * weights[t,j]), each addition rounded to bf16 (the
 * index_add_ order of GptOssExperts.forward); residual may be NULL.
 * Only slots whose expert lies in [e_lo, e_hi) count (an expert-parallel
 * shard's part; 0, E for all); out_f32 != 0 writes that sum as fp32 (no
 * residual) for fg_sum_partials, else bf16. H % 8 == 0; 16-byte aligned. */
int fg_moe_unpermute(const fg_bf16* y, const int32_t* inv, const int32_t* indices,
                     const fg_bf16* weights, const fg_bf16* residual, void* out, int T, int k,
                     int H, int e_lo, int e_hi, int out_f32, fg_stream_t stream);

/* out = bf16(a + b) over n bf16 elements (n % 8 == 0): the residual add of
 * the moe_combine group (runner.py:454-457) when it runs apart from the
 * experts group (otherwise fg_moe_unpermute fuses it). */
int fg_add_bf16(const fg_bf16* a, const fg_bf16* b, fg_bf16* out, long long n, fg_stream_t stream);

/* out[i] = bf16(partials[0][i] + ... + partials[S-1][i]), fp32 sums in shard
 * order: the consumer side of a sharded feed-forward group (tensor-parallel
 * FFN partials, the first carrying the residual; expert-parallel MoE
 * partials), the reduce-by-consumer that replaces an all-reduce. partials
 * [S][n] fp32, n % 4 == 0. No counterpart in the reference, which runs each
 * FFN group on one rank (its vLLM path sums two expert halves with a torch
 * add, vllm_integration.py:1085-1093). */
int fg_sum_partials(const float* partials, int S, long long n, fg_bf16* out, fg_stream_t stream);

/* ---- NVLink hand-off between ranks (replaces the NCCL send/recv of
 * ProcessGroupComm.send_tensor / recv_tensor, comm.py:24-46, at the task
 * boundaries of executor.py:104-123; design ancestor: the IPC-buffer + flag
 * and RDMA-write + flag handlers of cpp_runtime comm_backend.cu:92-381,
 * :1078-1187) ------------------------------------------------------------ */

/* Bytes of one rank's mailbox: data [world][nslot][slot_bytes], sequence
 * flags, acks, device-side counters. Zero it before first use. */
size_t fg_mailbox_bytes(int world, int nslot, size_t slot_bytes);
/* CUDA IPC export of the allocation holding `ptr`: 64-byte handle + offset of
 * ptr inside it (comm_backend.cu:118-152 exchanges the same handles). */
int fg_ipc_export(const void* ptr, void* handle_out, size_t* offset_out);
/* Map a peer allocation (peer access enabled lazily): *ptr_out = base + offset. */
int fg_ipc_import(const void* handle, size_t offset, void** ptr_out);
int fg_ipc_close(void* base_plus_offset, size_t offset);
/* Store nbytes of src (16-byte aligned, nbytes % 16 == 0, <= slot_bytes)
 * into rank dst's mailbox slot for messages from `me`, then release the
 * slot's sequence flag. Waits (bounded, timeout_ms) until dst drained the
 * slot's previous message. Graph-capturable: sequence numbers live on the
 * device. */
int fg_handoff_put(const void* src, size_t nbytes, void* my_mailbox, void* peer_mailbox, int world,
                   int me, int dst, int nslot, size_t slot_bytes, int timeout_ms, fg_stream_t stream);
/* Wait (bounded, timeout_ms; on expiry the device status records a peer flag
 * timeout) for the next message from src, copy it to out, ack the slot. */
int fg_handoff_recv(void* out, size_t nbytes, void* my_mailbox, void* peer_mailbox, int world,
                    int me, int src, int nslot, size_t slot_bytes, int timeout_ms, fg_stream_t stream);

/* Direct (zero-copy) hand-off on a mailbox made with nslot = 1. The sender
 * stores its tensor straight into its slot in the receiver's mailbox (the
 * address fg_mailbox_slot gives for the peer's mailbox, src = sender) from
 * its own producing kernel, then fg_handoff_signal publishes it (sequence
 * number, system-scope release); the receiver's fg_handoff_wait spins
 * (bounded by timeout_ms, device status 2 on expiry) until it arrives, and
 * the receiver's kernels then read the slot in place. No acks: valid only
 * where the sender's next message on the channel depends on data the
 * receiver produced after its last read of the slot (strict alternation of
 * the main path between two ranks). No counterpart in the reference (its
 * send/recv copy through NCCL buffers). */
void* fg_mailbox_slot(void* mailbox, int world, int nslot, size_t slot_bytes, int src, int slot);
int fg_handoff_signal(void* my_mailbox, void* peer_mailbox, int world, int me, int dst, size_t slot_bytes,
                      fg_stream_t stream);
int fg_handoff_wait(void* my_mailbox, int world, int me, int src, size_t slot_bytes, int timeout_ms,
                    fg_stream_t stream);

/* ---- consumers of routed hand-offs (fg_gemm_bf16_packed_routed) -------
 * The first kernel that reads rows another GPU stored waits for their flags
 * itself (no separate wait kernel). A flag carries a value: the consumer
 * waits until it reaches epoch[0] * seq_mul + seq_add (wrap-safe), computed
 * from its own per-step epoch counter exactly as the producer computed the
 * value it stored, so every CTA waits for the same message whenever it
 * starts. Waits give up after timeout_ms (device status 2, site 0x5xx).
 * flags: n_flags <= 8 u32 pointers in this GPU's memory (read at the call).
 * No counterpart in the reference (its receive is an NCCL recv into a
 * buffer, executor.py:104-123). */
/* fg_rmsnorm after row r's flag (flags[r / rows_per_flag]) has arrived. */
int fg_rmsnorm_wait(const fg_bf16* x, const fg_bf16* weight, fg_bf16* out, int T, int H, float eps,
                    int weight_mode, uint32_t* const* flags, int n_flags, int rows_per_flag,
                    const uint32_t* epoch, uint32_t seq_mul, uint32_t seq_add, int timeout_ms,
                    fg_stream_t stream);
/* fg_rmsnorm_wait over rows that live on other GPUs: row r is row
 * r % rows_per_src of srcs[r / rows_per_src] (peer buffers, read over NVLink
 * once the row's flag has arrived), written to gathered[r] on this GPU as it
 * is read, and out[r] = RMSNorm(row r). The FFN side of the disaggregated
 * step in its pull form: the attention GPUs' O-proj stores stay in their own
 * memory, and the FFN GPU moves the rows (replaces the reference's recv of
 * the hidden state at the attention -> FFN boundary, executor.py:104-123). */
int fg_rmsnorm_gather_wait(const fg_bf16* const* srcs, int n_src, int rows_per_src, fg_bf16* gathered,
                           const fg_bf16* weight, fg_bf16* out, int T, int H, float eps, int weight_mode,
                           uint32_t* const* flags, int n_flags, int rows_per_flag, const uint32_t* epoch,
                           uint32_t seq_mul, uint32_t seq_add, int timeout_ms, fg_stream_t stream);
/* After all n_flags flags: h_out[r] = bf16(partials[0][r] + ... +
 * partials[S-1][r]) (fp32 sums in shard order, as fg_sum_partials; partials
 * [S][T][H] fp32) and x_out[r] = fg_rmsnorm(h_out[r]): the reduce-by-consumer
 * of a tensor-parallel FFN fused with the next layer's input norm. */
int fg_sum_rmsnorm_wait(const float* partials, int S, fg_bf16* h_out, const fg_bf16* weight, fg_bf16* x_out,
                        int T, int H, float eps, int weight_mode, uint32_t* const* flags, int n_flags,
                        const uint32_t* epoch, uint32_t seq_mul, uint32_t seq_add, int timeout_ms,
                        fg_stream_t stream);
/* *counter += delta on the device (the per-step epoch of the hand-offs). */
int fg_counter_add(uint32_t* counter, uint32_t delta, fg_stream_t stream);
/* Load every kernel of this library into the current device's context now.
 * Under CUDA's lazy loading a kernel's first launch loads its code, and the
 * load waits for the device's work in flight; when that work is a kernel
 * waiting for another GPU whose progress needs a launch this host has not
 * made yet, the two GPUs stall each other. Ranks that wait on one another
 * (the disaggregated step, P2PComm) call this once per device before their
 * first step. It also asks the device how many GEMM clusters of each size it
 * keeps resident (the decode GEMM plans use it; fg_pack_weight_bf16 asks too). */
int fg_preload(void);

/* positions[b] += 1 and seq_lens[b] += 1 after a decode step
 * (LayerKVCache.advance, kv_cache.py:140-144). Either pointer may be NULL. */
int fg_advance(int32_t* positions, int32_t* seq_lens, int B, fg_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* FGB200_H_ */
