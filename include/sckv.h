/*
 * sckv.h — C ABI of the B200 paged KV-cache library (libsckv.so).
 *
 * Plain pointers, sizes and int status codes; no framework types. Every
 * device-side call is asynchronous and ordered on the `stream` argument
 * (a cudaStream_t passed as void*, NULL = legacy default stream). A pool
 * handle is not thread-safe: callers serialise calls on one handle (the
 * Python façade holds an RLock, as the reference arena does).
 *
 * Device layout of a pool (one allocation, element type = kv dtype):
 *     data  [num_layers][max_pages][2 (K,V)][num_kv_heads][page_tokens][head_dim]
 *     int8 scales  [num_layers][max_pages][2][num_kv_heads][page_tokens]   fp16
 *     fp8  scales  [num_layers][max_pages][2][num_kv_heads]                fp32
 * A page id therefore names the same 16-token slot in every layer, which is
 * the reference's page: one id covers [L,1,H,16,D] of K and of V
 * (native/native_engine.py:250-257).
 *
 * Status codes mirror the reference C ABI (native/synapcore_native.mm:45-49).
 */
#ifndef SCKV_H
#define SCKV_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define SCKV_API __attribute__((visibility("default")))
#else
#define SCKV_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes (native/synapcore_native.mm:45-49 for 0, -1, -3, -4) ---- */
#define SCKV_OK                 0
#define SCKV_ERR_INVALID_ARG   -1
#define SCKV_ERR_BOUNDS        -3   /* page id / block index / length out of range */
#define SCKV_ERR_ALIGNMENT     -4
#define SCKV_ERR_CUDA          -5   /* a CUDA runtime call failed */
#define SCKV_ERR_POOL_EXHAUSTED -6  /* allocation needs more pages than exist */
#define SCKV_ERR_TIMEOUT       -7   /* a bounded in-kernel wait gave up */
#define SCKV_ERR_UNSUPPORTED   -8   /* dtype / head_dim combination not built */
#define SCKV_ERR_SCRATCH_LIMIT -9   /* needs more than the fixed no-allocation scratch */

/* ---- element types ---- */
#define SCKV_DTYPE_F16       0
#define SCKV_DTYPE_BF16      1
#define SCKV_DTYPE_INT8      2   /* reference int8 mode: per-(token,head) fp16 scale */
#define SCKV_DTYPE_FP8_E4M3  3   /* per-(layer,page,K|V,head) fp32 scale = max|x|/448 */
#define SCKV_DTYPE_F32       4   /* query / output / source type only */

typedef struct sckv_pool sckv_pool;
typedef struct sckv_exchange sckv_exchange;

/* ========================================================================== */
/* Pool lifetime                                                               */
/* ========================================================================== */

/* Byte sizes of the three device regions a pool needs.
 * alloc_bytes covers the on-device allocator (free ring, LRU clocks,
 * refcounts, control words, status word). */
SCKV_API int sckv_pool_required_bytes(int num_layers, int num_kv_heads, int head_dim,
                             int page_tokens, int64_t max_pages, int kv_dtype,
                             size_t* data_bytes, size_t* scale_bytes,
                             size_t* alloc_bytes);

/* Allocate and zero a pool on `device` (cudaMalloc). Replaces the pool
 * allocation of PagedKVArena.__init__ (native/native_engine.py:232-295).
 * page_tokens must be 16 (PagedKVArena.PAGE_TOKENS, native_engine.py:230). */
SCKV_API int sckv_pool_create(int num_layers, int num_kv_heads, int head_dim,
                     int page_tokens, int64_t max_pages, int kv_dtype,
                     int device, sckv_pool** out);

/* Same, over caller-owned device memory of the sizes returned by
 * sckv_pool_required_bytes (the library neither zeroes nor frees it except
 * through sckv_alloc_reset, which initialises the allocator region). */
SCKV_API int sckv_pool_wrap(int num_layers, int num_kv_heads, int head_dim,
                   int page_tokens, int64_t max_pages, int kv_dtype,
                   int device, void* data, void* scales, void* alloc_state,
                   sckv_pool** out);

/* Release a pool (frees memory only if sckv_pool_create allocated it).
 * Replaces PagedKVArena.clear's pool drop (native/native_engine.py:421-432). */
SCKV_API void sckv_pool_destroy(sckv_pool* pool);

/* Device pointers of the pool regions (for zero-copy host views). */
SCKV_API int sckv_pool_pointers(const sckv_pool* pool, void** data, void** scales,
                       void** alloc_state);

/* ========================================================================== */
/* Kernel 1 — scatter-append through the block table                          */
/* ========================================================================== */

/* Append new K/V tokens of `n_seqs` sequences into their pages.
 * Replaces the per-request concatenate-append of
 * ModularAttentionEngine.forward_numpy (models/adapters.py:1194-1207).
 *
 * k_new, v_new : [n_layers][n_tokens][num_kv_heads][head_dim] of src_dtype
 *                (F16 / BF16 / F32); tokens of sequence b occupy rows
 *                cu_tokens[b] .. cu_tokens[b+1]-1, in position order.
 * cu_tokens    : int32 [n_seqs+1] device, cu_tokens[0] = 0.
 * start_pos    : int32 [n_seqs] device, position of the first new token.
 * block_table  : int32 [n_seqs][bt_stride] device; entry j = page id of
 *                positions 16j..16j+15 (only the first max_blocks are used).
 * Writes pool layers layer0 .. layer0+n_layers-1. Pools of type INT8
 * quantise per (token, head) exactly as quantize_kv_int8_numpy
 * (native/native_engine.py:207-216); FP8 pools keep a per-page-head scale
 * max|x|/448 that grows as tokens arrive (older codes of that page-head
 * are re-encoded under the grown scale). */
SCKV_API int sckv_append(sckv_pool* pool, int layer0, int n_layers,
                const void* k_new, const void* v_new, int src_dtype,
                int n_seqs, int n_tokens, const int32_t* cu_tokens,
                const int32_t* start_pos, const int32_t* block_table,
                int64_t bt_stride, int max_blocks, void* stream);

/* Write whole pages: k_src/v_src are [n_pages][num_layers][num_kv_heads][16][head_dim]
 * of src_dtype — the reference page layout [L,1,H,16,D] without its unit
 * axis. Replaces the copy / quantise body of PagedKVArena.write_page_fp16
 * (native/native_engine.py:339-359). */
SCKV_API int sckv_write_pages(sckv_pool* pool, const int32_t* page_ids, int n_pages,
                     const void* k_src, const void* v_src, int src_dtype,
                     void* stream);

/* Write int8 codes + fp16 scales: kq/vq [n][L][H][16][D] int8,
 * ks/vs [n][L][H][16] fp16. INT8 pools store them as given; F16 pools store
 * the dequantised fp16(q * f32(scale)). Replaces
 * PagedKVArena.write_page_quantized (native/native_engine.py:361-386). */
SCKV_API int sckv_write_pages_quantized(sckv_pool* pool, const int32_t* page_ids,
                               int n_pages, const int8_t* kq, const void* ks,
                               const int8_t* vq, const void* vs, void* stream);

/* ========================================================================== */
/* Kernel 2 — paged gather / compaction and copy-on-write page copy           */
/* ========================================================================== */

/* Gather pages, in list order, into contiguous
 * out_k/out_v [n_layers][num_kv_heads][n_tokens][head_dim] of out_dtype
 * (F16 / BF16 / F32), token t taken from page page_ids[t/16] slot t%16;
 * n_tokens <= 16*n_pages. INT8 / FP8 pools are dequantised
 * (dequantize_kv_int8_numpy, native/native_engine.py:219-221).
 * Replaces PagedKVArena.gather_contiguous_kv_numpy and read_page_fp16
 * (native/native_engine.py:388-419). */
SCKV_API int sckv_gather(sckv_pool* pool, int layer0, int n_layers,
                const int32_t* page_ids, int n_pages, int n_tokens,
                void* out_k, void* out_v, int out_dtype, void* stream);

/* Copy pages src_ids[i] -> dst_ids[i] in every layer, K, V and scales.
 * The device half of a copy-on-write fork: replaces the eager per-layer
 * copy of a matched prefix in ContinuousBatchScheduler._prefill_request_numpy
 * (engine/scheduler.py:150-152). */
SCKV_API int sckv_copy_pages(sckv_pool* pool, const int32_t* src_ids,
                    const int32_t* dst_ids, int n_pages, void* stream);

/* ========================================================================== */
/* Kernels 3+4 — paged decode attention (split-K), fused FP8 dequant          */
/* ========================================================================== */

/* Bytes of scratch sckv_decode_attn needs for these sizes (split partials);
 * 0 when the chosen split is 1 (an unsplit launch writes its output
 * directly) or on bad arguments. */
SCKV_API size_t sckv_decode_workspace_bytes(const sckv_pool* pool, int n_seqs,
                                   int num_q_heads, int max_blocks,
                                   int chunk_pages);

/* One query token per sequence: out[b][hq] = softmax(scale * q[b][hq] . K^T) V
 * over the first ctx_lens[b] tokens of sequence b in layer `layer`, with
 * q head hq reading kv head hq / (num_q_heads / num_kv_heads).
 * Replaces the SDPA of ModularAttentionEngine.forward_numpy
 * (models/adapters.py:1209-1229; GQA repeat at :1211-1215, scale at :1121).
 *
 * q   : [n_seqs][num_q_heads][head_dim] of q_dtype (F16 / BF16 / F32)
 * out : [n_seqs][num_q_heads][head_dim] of out_dtype (F16 / BF16 / F32)
 * block_table : int32 [n_seqs][bt_stride]; bt_stride 0 makes every sequence
 *               read row 0 (prefill: query token t of one sequence is a
 *               "sequence" of length start+t+1 over the same pages).
 * chunk_pages : pages per split (split-K unit); <= 0 picks one. A fixed
 *               value makes each sequence's result independent of the batch.
 * workspace   : device scratch of sckv_decode_workspace_bytes bytes (may be
 *               NULL when that is 0), 16-byte aligned.
 * Pool dtypes F16, BF16 (bf16 queries for the tensor-core kernel),
 * FP8_E4M3 (per-page-head scale) and INT8 (per-token fp16 scales);
 * num_q_heads / num_kv_heads <= 16. Kernel choice: tensor cores (mma.sync,
 * TMA page boxes) for FP8 / INT8 pools and for G = num_q_heads /
 * num_kv_heads >= 2; CUDA cores for 16-bit MHA pools.
 * SCKV_DECODE_KERNEL=simt|mma overrides (the CUDA-core kernel takes INT8
 * only with G in {1, 2, 4, 8}). Accumulation is fp32. */
SCKV_API int sckv_decode_attn(sckv_pool* pool, int layer, const void* q, int q_dtype,
                     int num_q_heads, const int32_t* block_table,
                     int64_t bt_stride, int max_blocks, const int32_t* ctx_lens,
                     int n_seqs, float scale, void* out, int out_dtype,
                     void* workspace, size_t workspace_bytes, int chunk_pages,
                     void* stream);

/* One decode token per sequence with its K/V append in the same launch:
 * the result equals sckv_append of row b of k_new / v_new
 * ([n_seqs][num_kv_heads][head_dim] of src_dtype F16 / BF16 / F32, 16-byte
 * aligned) at position ctx_lens[b] - 1 of sequence b (layer `layer`),
 * followed by sckv_decode_attn over ctx_lens[b] tokens — the KV-cache concat
 * and SDPA of one decode step of ModularAttentionEngine.forward_numpy
 * (models/adapters.py:1194-1229). The warp that reads the page holding
 * position ctx_lens[b] - 1 stores the new row into the pool and into its
 * staged copy of the page, so no separate append kernel runs. The page a
 * sequence appends into must be read by no other sequence of the call (the
 * arena's copy-on-write keeps a page that is still being filled private;
 * another reader would race with the store). Every other argument as
 * sckv_decode_attn. F16 / BF16 pools only (SCKV_ERR_UNSUPPORTED
 * otherwise: one-byte pools quantise a row against its page or token scale,
 * use sckv_append then sckv_decode_attn). A sequence whose ctx_lens[b] is
 * out of range or whose page id is invalid is reported as by
 * sckv_decode_attn and its row is not stored. */
SCKV_API int sckv_decode_attn_append(sckv_pool* pool, int layer, const void* q,
                     int q_dtype, int num_q_heads, const void* k_new,
                     const void* v_new, int src_dtype,
                     const int32_t* block_table, int64_t bt_stride,
                     int max_blocks, const int32_t* ctx_lens, int n_seqs,
                     float scale, void* out, int out_dtype, void* workspace,
                     size_t workspace_bytes, int chunk_pages, void* stream);

/* Causal prefill attention: for each of n_seqs sequences, the query tokens
 * cu_q[b] .. cu_q[b+1]-1 sit at positions start_pos[b] + i and attend to
 * every token of that sequence at positions <= their own (the new tokens'
 * K/V must already be appended). Replaces the prompt pass of
 * ModularAttentionEngine.forward_numpy with its causal mask
 * (models/adapters.py:1209-1229, mask at :1218-1224).
 * q/out : [n_tokens][num_q_heads][head_dim]; cu_q int32 [n_seqs+1];
 * start_pos int32 [n_seqs]; block_table [n_seqs][bt_stride] (device).
 * All pool types: tcgen05.mma with S and O accumulators in tensor memory
 * (persistent CTAs claiming work from a per-launch counter); FP8 and int8
 * pages are decoded (times their scales) into f16 tiles in shared memory
 * first. fp32 accumulation. BF16 pools need bf16 queries; num_q_heads /
 * num_kv_heads must be a power of two <= 16; otherwise SCKV_ERR_UNSUPPORTED.
 * SCKV_PREFILL_KERNEL=mma selects the older mma.m16n8k16 kernel (F16, BF16,
 * FP8 with even num_kv_heads). */
SCKV_API int sckv_prefill_attn(sckv_pool* pool, int layer, const void* q,
                      int q_dtype, int num_q_heads, int n_seqs, int n_tokens,
                      const int32_t* cu_q, const int32_t* start_pos,
                      const int32_t* block_table, int64_t bt_stride,
                      int max_blocks, float scale, void* out, int out_dtype,
                      void* stream);

/* Fused attention input for new tokens: optional RMSNorm of
 * q and k, rotary position embedding of both at positions start_pos[b] + i,
 * then the K/V append of sckv_append for one layer; the rotated q lands in
 * q_out. Replaces the QK-norm, RoPE and KV-cache concat of
 * ModularAttentionEngine.forward_numpy (models/adapters.py:1171-1207, with
 * rmsnorm_f32 :1129-1132 and apply_rope_f32 :1134-1146), in fp32 and the
 * reference's operation order.
 * q_in/q_out : [n_tokens][num_q_heads][head_dim]; k_in/v_in [n_tokens][Hkv][D].
 * q_norm_len / k_norm_len: 0 (no norm), head_dim (per-head fp16 weights) or
 * heads x head_dim (one norm over the whole projection).
 * inv_freq: device fp32 [head_dim / 2], 1 / theta^(2i / head_dim) as the
 * reference computes it; positions are divided by rope_scaling.
 * Pools f16 / bf16, and int8 (each K / V row stored as the arena stores its
 * fp16 pages: the fp16 value quantised per row, native/native_engine.py:
 * 207-216); FP8 pools: SCKV_ERR_UNSUPPORTED (their page scales span 16
 * tokens: sckv_append). head_dim 128, at most 256 heads. */
SCKV_API int sckv_append_rope(sckv_pool* pool, int layer, const void* q_in,
                     void* q_out, int num_q_heads, int q_dtype,
                     int q_out_dtype, const void* k_in, const void* v_in,
                     int src_dtype, const void* q_norm_w, int q_norm_len,
                     const void* k_norm_w, int k_norm_len, float eps,
                     const float* inv_freq, float rope_scaling, int n_seqs,
                     int n_tokens, const int32_t* cu_tokens,
                     const int32_t* start_pos, const int32_t* block_table,
                     int64_t bt_stride, int max_blocks, void* stream);

/* Projections + per-head QK-norm + RoPE + K/V append of one layer in one
 * tcgen05 kernel (head_dim 128). f16 / bf16 pools take the rows directly;
 * an int8 pool gets each new K / V row quantised as the arena quantises its
 * fp16 pages (native/native_engine.py:207-216); an FP8 pool gets the rows
 * staged in fp16 in the workspace and stored by the FP8 append (page
 * scales grow with the tokens a page holds), one more launch. Replaces q/k/v = x @ W^T
 * (models/adapters.py:1167-1169, fp16 weights), the per-head RMSNorm
 * (:1171-1185), RoPE (:1191-1192) and the KV-cache concat (:1194-1207) of
 * ModularAttentionEngine.forward_numpy: k and v of token i of sequence b
 * land in slot start_pos[b] + i of the sequence's pages of `layer`, the
 * rotated q in q_out [n_tokens][num_q_heads][128].
 * x : [n_tokens][hidden] in x_dtype (F16 or BF16, the weights' type);
 *     x_lo (optional, same shape) is added to x in the products — an fp32
 *     input split by sckv_split_hi_lo keeps fp32 accuracy this way.
 * w_q [num_q_heads*128][hidden], w_k / w_v [Hkv*128][hidden] row-major.
 * q_norm_len / k_norm_len: 0 or 128 (per-head fp16 weights); whole-width
 * norms return SCKV_ERR_UNSUPPORTED (use the projections + sckv_append_rope).
 * workspace: >= sckv_qkv_workspace_bytes(...) bytes: the per-token cos / sin
 * table, plus fp32 partial sums and per-token (position, page) entries when
 * few token tiles make the kernel split the hidden dim across CTAs (a
 * second, finishing launch then applies the norm, rotation and stores).
 * The launches use programmatic dependent launch: each may start its set-up
 * while the kernel before it in the stream finishes, and reads nothing
 * before that kernel has completed.
 * hidden % 8 == 0; x, x_lo, weights, q_out and workspace 16-byte aligned. */
SCKV_API int sckv_qkv_append(sckv_pool* pool, int layer, const void* x,
                     const void* x_lo, int x_dtype, int n_tokens, int hidden,
                     const void* w_q, const void* w_k, const void* w_v,
                     int num_q_heads, const void* q_norm_w, int q_norm_len,
                     const void* k_norm_w, int k_norm_len, float eps,
                     const float* inv_freq, float rope_scaling, int n_seqs,
                     const int32_t* cu_tokens, const int32_t* start_pos,
                     const int32_t* block_table, int64_t bt_stride,
                     int max_blocks, void* q_out, int q_out_dtype,
                     void* workspace, size_t workspace_bytes, void* stream);

/* Workspace sckv_qkv_append needs for this call shape (0 on bad arguments). */
SCKV_API size_t sckv_qkv_workspace_bytes(const sckv_pool* pool, int n_tokens,
                     int num_q_heads, int hidden);

/* fp32 x -> hi = round(x), lo = round(x - hi) in F16 or BF16 (n elements):
 * the two-part input of sckv_qkv_append for fp32 activations. */
SCKV_API int sckv_split_hi_lo(const float* x, int64_t n, void* hi, void* lo,
                     int dtype, void* stream);

/* Output projection after attention: out = x @ w_o^T, the last step of
 * ModularAttentionEngine.forward_numpy (models/adapters.py:1231, attn_out
 * fp32 times the fp16 o_proj weights, fp32 result). The plain mode of the
 * sckv_qkv_append kernel (tcgen05, fp32 accumulation).
 * x : [n_tokens][in_features] in x_dtype (F16 or BF16, the weights' type);
 *     x_lo (optional) as in sckv_qkv_append: an fp32 attention output split
 *     by sckv_split_hi_lo keeps fp32 accuracy.
 * w_o [out_features][in_features] row-major; out [n_tokens][out_features]
 * in out_dtype (F32, F16 or BF16).
 * out_features % 128 == 0 and in_features % 8 == 0, else
 * SCKV_ERR_UNSUPPORTED. workspace: >= sckv_o_proj_workspace_bytes(...)
 * (fp32 partial sums when few token tiles make the kernel split
 * in_features across CTAs; 0 bytes otherwise, and workspace may be NULL).
 * x, x_lo, w_o, out and workspace 16-byte aligned. Failures inside the
 * kernel are recorded in the pool's status word (kernel id 14). */
SCKV_API int sckv_o_proj(sckv_pool* pool, const void* x, const void* x_lo,
                     int x_dtype, int n_tokens, int in_features,
                     const void* w_o, int out_features, void* out,
                     int out_dtype, void* workspace, size_t workspace_bytes,
                     void* stream);

/* Workspace sckv_o_proj needs for this call shape (0 on bad arguments). */
SCKV_API size_t sckv_o_proj_workspace_bytes(const sckv_pool* pool,
                     int n_tokens, int in_features, int out_features);

/* ========================================================================== */
/* KV-head-sharded output exchange (no reference counterpart: the reference  */
/* has no multi-process code; this is the optional layout of a multi-GPU box) */
/* ========================================================================== */
/* In the KV-head-sharded layout rank r of `world` holds every sequence but
 * only kv heads [r*Hkv/world, (r+1)*Hkv/world) and the q heads that read them.
 * The exchange object owns, in this GPU's memory, a full-head output buffer
 * of out_bytes and a flag word per source rank; every rank maps every other
 * rank's buffer and flags through CUDA IPC (one process per GPU, one box).
 * Peer memory is reached by ordinary stores and flag loads/stores only.
 *
 * Set-up: sckv_exchange_create on each rank, sckv_exchange_ipc_handles
 * (128 bytes: buffer handle, flags handle), exchange those bytes between the
 * ranks (e.g. an all-gather of the process group), sckv_exchange_open_peer
 * for every other rank. world <= 8. */
SCKV_API int sckv_exchange_create(int device, int world, int rank, size_t out_bytes,
                         sckv_exchange** out);
SCKV_API void* sckv_exchange_buffer(const sckv_exchange* ex);
SCKV_API int sckv_exchange_ipc_handles(const sckv_exchange* ex, uint8_t* out_handles);
SCKV_API int sckv_exchange_open_peer(sckv_exchange* ex, int peer, const uint8_t* handles);
SCKV_API void sckv_exchange_destroy(sckv_exchange* ex);

/* sckv_decode_attn for this rank's heads (q [n_seqs][num_q_heads][128] holds
 * q heads rank*num_q_heads .. +num_q_heads-1, the pool this rank's kv heads),
 * whose epilogue stores output element (b, h, d) at element
 * out_offset + (b * num_q_heads_total + rank * num_q_heads + h) * 128 + d of
 * EVERY rank's exchange buffer (out_dtype F32 / F16 / BF16; num_q_heads_total
 * = world * num_q_heads), then, once those stores are complete, sets this
 * rank's flag to the call's epoch on every rank. epoch: non-zero, increasing
 * per call, the same on every rank for the same layer and step; or 0 to
 * take the next value of this rank's device-side epoch counter (last
 * signalled + 1), which keeps the call capturable in a CUDA graph. k_new /
 * v_new (both NULL or both set; F16 / BF16 pools): the new token's rows of
 * this rank's kv heads, appended in the same launch as by
 * sckv_decode_attn_append. Replaces the decode + NCCL all-gather pair of the
 * layout. All ranks' buffers must be open. */
SCKV_API int sckv_decode_attn_exchange(sckv_pool* pool, sckv_exchange* ex, int layer,
                             const void* q, int q_dtype, int num_q_heads,
                             const void* k_new, const void* v_new, int src_dtype,
                             const int32_t* block_table, int64_t bt_stride,
                             int max_blocks, const int32_t* ctx_lens, int n_seqs,
                             float scale, int out_dtype, int64_t out_offset,
                             int num_q_heads_total, uint32_t epoch,
                             void* workspace, size_t workspace_bytes,
                             int chunk_pages, void* stream);

/* Stream-ordered wait until every rank's flag here reached `epoch` (then the
 * full-head output of that call is in this rank's buffer for every kernel
 * launched after it on `stream`); epoch 0 waits for the last epoch this rank
 * signalled (read on the device when the wait runs). Bounded: after
 * limit_us (0 = 2 s) the kernel records SCKV_ERR_TIMEOUT (detail = the late
 * rank) in the exchange's status word and returns. */
SCKV_API int sckv_exchange_wait(sckv_exchange* ex, uint32_t epoch, unsigned limit_us, void* stream);

/* The exchange's status word (code, detail, kernel, count); clear != 0 resets it. */
SCKV_API int sckv_exchange_status(const sckv_exchange* ex, int32_t out[4], int clear, void* stream);

/* Fixed per-GPU scratch behind sckv_decode_attn_noalloc (4 MiB). */
#define SCKV_NOALLOC_SCRATCH_BYTES (4u << 20)

/* sckv_decode_attn for callers that cannot allocate device memory; this entry
 * point has no counterpart in the reference. The split-K partials go to a
 * fixed SCKV_NOALLOC_SCRATCH_BYTES device array inside the library (one per
 * GPU, held until exit) instead of a caller workspace; nothing is allocated
 * per call. chunk_pages <= 0 picks a split that fits; a request whose
 * partials cannot fit (n_seqs * num_q_heads * splits * 520 bytes when
 * splits > 1; an unsplit request needs none) returns SCKV_ERR_SCRATCH_LIMIT
 * before launching anything, after the same argument checks as
 * sckv_decode_attn. The first call on a device (and the first after a device
 * reset, which moves the array) resolves the array's device address, so make
 * it before any stream capture. All calls share the array: calls that
 * overlap on the GPU race. Leaves the caller's current device unchanged. */
SCKV_API int sckv_decode_attn_noalloc(sckv_pool* pool, int layer, const void* q,
                             int q_dtype, int num_q_heads,
                             const int32_t* block_table, int64_t bt_stride,
                             int max_blocks, const int32_t* ctx_lens,
                             int n_seqs, float scale, void* out, int out_dtype,
                             int chunk_pages, void* stream);

/* ========================================================================== */
/* Kernel 5 — on-device free list allocator and LRU eviction                  */
/* ========================================================================== */
/* The allocator restates PagedKVArena's bookkeeping on the device
 * (native/native_engine.py:289-337): a FIFO free ring initialised to
 * 0..max_pages-1, a step clock, a last-used clock per page, and LRU victim
 * choice (smallest last-used) when the ring is empty. Pages with a nonzero
 * pin count are never victims. */

/* Reset: ring = 0..P-1, clock = 0, all pages free, counters 0. */
SCKV_API int sckv_alloc_reset(sckv_pool* pool, void* stream);

/* Allocate n pages in order, as n successive _allocate_page_slot_unlocked
 * calls for new keys (native/native_engine.py:318-337): each takes the ring
 * head, else evicts the least recently used unpinned allocated page; the
 * clock advances by one per page and the page's last-used becomes the clock.
 * out_ids[i] = page id; out_victims[i] = evicted page id or -1 (may be NULL).
 * If pin != 0 the pages start with pin count 1. Fails with
 * SCKV_ERR_POOL_EXHAUSTED (status word) if fewer than n pages can be had. */
SCKV_API int sckv_alloc_pages(sckv_pool* pool, int n, int pin, int32_t* out_ids,
                     int32_t* out_victims, void* stream);

/* Return pages to the ring tail (FIFO), as PagedKVArena.evict_prefix_hash
 * (native/native_engine.py:307-316). Unallocated ids are skipped. */
SCKV_API int sckv_free_pages(sckv_pool* pool, const int32_t* ids, int n, void* stream);

/* Touch pages in order, as n successive lookup_page_id calls
 * (native/native_engine.py:297-305): clock += 1 each; a valid id's last-used
 * becomes the clock; an id of -1 is a miss (clock only). */
SCKV_API int sckv_touch_pages(sckv_pool* pool, const int32_t* ids, int n, void* stream);

/* Add `delta` to the pin counts of pages (copy-on-write sharing). */
SCKV_API int sckv_pin_pages(sckv_pool* pool, const int32_t* ids, int n, int delta,
                   void* stream);

/* Drop one pin from each page (a sequence letting go of its pages). A page
 * whose pin count reaches zero returns to the ring tail in list order, or,
 * with keep_cached != 0, stays allocated as an LRU eviction candidate (a
 * cached prefix page). Ids in one call must be distinct. The device side of
 * freeing a request's KV (the reference drops its per-request arrays,
 * engine/scheduler.py:369-371). */
SCKV_API int sckv_release_pages(sckv_pool* pool, const int32_t* ids, int n,
                       int keep_cached, void* stream);

/* Evict the n least recently used unpinned allocated pages to the ring
 * tail, oldest first; out_ids (may be NULL) receives them, -1 padded. */
SCKV_API int sckv_evict_lru(sckv_pool* pool, int n, int32_t* out_ids, void* stream);

/* Occupancy-bounded eviction: evict unpinned allocated pages in LRU order
 * until at most max_allocated pages are allocated (or no unpinned page is
 * left), the allocated count being read on the device, so a serving loop
 * needs no host accounting or device read for it (and the call can sit in a
 * captured graph). out_count (device int32, may be NULL) receives how many
 * were evicted. Each eviction counts as in sckv_evict_lru. No reference
 * counterpart: the reference evicts only when an allocation finds the free
 * list empty (native/native_engine.py:324-331), which sckv_alloc_pages does;
 * this is the "evict at X % full" policy of a continuous-batching server. */
SCKV_API int sckv_evict_to_watermark(sckv_pool* pool, int64_t max_allocated,
                             int32_t* out_count, void* stream);

/* Decode-step page reservation, fully on device: for b in 0..n_seqs-1 in
 * order, if ctx_lens[b] % 16 == 0 a page is allocated (as sckv_alloc_pages,
 * pinned) into block_table[b][ctx_lens[b]/16]; then ctx_lens[b] += 1. */
SCKV_API int sckv_reserve_decode(sckv_pool* pool, int32_t* block_table,
                        int64_t bt_stride, int max_blocks, int32_t* ctx_lens,
                        int n_seqs, void* stream);

/* Read allocator counters (synchronises `stream`):
 * out[0] ring head, out[1] ring tail (free = tail-head), out[2] step clock,
 * out[3] evictions, out[4] allocated pages. */
SCKV_API int sckv_alloc_state(const sckv_pool* pool, int64_t out[5], void* stream);

/* ========================================================================== */
/* Status word                                                                 */
/* ========================================================================== */
/* Kernels never trap; they record the first error in a device status word:
 * out[0] code (SCKV_ERR_*), out[1] detail (offending index / value),
 * out[2] kernel id, out[3] count of errors. Synchronises `stream`. */
SCKV_API int sckv_get_status(const sckv_pool* pool, int32_t out[4], void* stream);
SCKV_API int sckv_clear_status(sckv_pool* pool, void* stream);

/* Failure-path self test: one kernel waits (bounded, limit_us <= 2 s) on a
 * barrier nothing completes, gives up and records SCKV_ERR_TIMEOUT (detail
 * -1) in the status word, exactly as a stalled pipeline kernel would; the
 * context stays usable. No counterpart in the reference. */
SCKV_API int sckv_selftest_wait_timeout(sckv_pool* pool, unsigned limit_us, void* stream);

/* ========================================================================== */
/* KV prefix hash table (host, C++)                                            */
/* ========================================================================== */
/* Open-addressed 1024-slot table of 80-byte slots, laid out exactly as the
 * reference's NativeKVPrefixSlot {u8 prefix_hash[32]; u8 parent_hash[32];
 * u32 occupied; u32 token_end; f64 created_at} (native/synapcore_native.mm:
 * 93-100), operating on caller memory `table` (1024*80 bytes; e.g. the KV
 * region of an index file mapping). Home slot = u32le(hash[0:4]) & 1023,
 * 64 linear probes. */

/* Replaces synapcore_native_kv_lookup (native/synapcore_native.mm:716-734):
 * 1 if present (out_token_end set when non-NULL), else 0. */
SCKV_API int sckv_kv_lookup(const uint8_t* table, const uint8_t* prefix_hash32,
                   uint32_t* out_token_end);

/* Replaces synapcore_native_kv_insert (native/synapcore_native.mm:736-780):
 * 1 = stored in an empty or equal slot; 2 = overwrote the probe window's
 * oldest created_at slot, whose hash goes to out_evicted_hash32 (if not
 * NULL) and *evictions is incremented (if not NULL); 3 = the window was full
 * but no slot had created_at < +inf (all NaN or +inf): the home slot was
 * overwritten and counted as an eviction, its hash still goes to
 * out_evicted_hash32, but the reference's Python bridge reports no evicted
 * hash for this case (native/native_engine.py:1747-1752) while its C++
 * returns 2 — treat 3 as 2 to follow the C++; SCKV_ERR_INVALID_ARG on NULL
 * table/hash. */
SCKV_API int sckv_kv_insert(uint8_t* table, const uint8_t* prefix_hash32,
                   const uint8_t* parent_hash32, uint32_t token_end,
                   double timestamp, uint8_t* out_evicted_hash32,
                   uint64_t* evictions);

/* ========================================================================== */
/* Misc                                                                        */
/* ========================================================================== */
SCKV_API const char* sckv_version(void);
/* Where the calling thread's last SCKV_ERR_CUDA came from
 * ("file:line call: CUDA error name"); "" if none. No reference counterpart
 * (the reference's native calls report only status codes). */
SCKV_API const char* sckv_last_error(void);
/* Kernels this library has launched in this process, all devices (for
 * launch accounting around a timed region). No reference counterpart. */
SCKV_API unsigned long long sckv_launch_count(void);
SCKV_API const char* sckv_status_string(int code);

#ifdef __cplusplus
}
#endif
#endif /* SCKV_H */
