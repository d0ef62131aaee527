// Definitions shared by the decode-attention translation units.
#pragma once

#include "sckv_internal.cuh"

namespace sckv_detail {

constexpr int kConsumerWarps = 4;
constexpr int kThreads = (kConsumerWarps + 1) * 32;
constexpr int kHD = 128;  // head_dim handled by this kernel
constexpr int kMaxExchangeRanks = 8;  // ranks of one box in the KV-head-sharded exchange

struct DecodeParams {
  const uint8_t* pool;
  const float* fp8_scales;  // the pool's scale region: FP8 float per page-head, or int8 fp16 per token
  const void* q;
  void* out;
  float* part_acc;  // [n_seqs][Hq][max_splits][HD]
  float* part_ml;   // [n_seqs][Hq][max_splits][2]
  const int32_t* block_table;
  const int32_t* ctx_lens;
  int32_t* status;
  int64_t bt_stride;
  int64_t max_pages;
  int max_blocks;
  int n_seqs;
  int hq;
  int hkv;
  int layer;
  int chunk_pages;
  int max_splits;
  int q_dtype;
  int out_dtype;
  float scale_log2;
  // KV-head-sharded exchange (n_peer > 0): the output of (sequence b, local
  // q head h) goes to element out_off + (b * out_hq_total + out_head0 + h) *
  // HD of every rank's full-head buffer peer_out[r] (plain stores over
  // NVLink; peer_out[rank] is the local buffer) instead of `out`
  void* peer_out[kMaxExchangeRanks];
  int n_peer;
  int out_hq_total;
  int out_head0;
  int64_t out_off;
  // fused append (16-bit pools; k_new null: none): row (b, h) of k_new /
  // v_new [n_seqs][Hkv][HD] of new_dtype is sequence b's token at position
  // ctx_lens[b] - 1; the warp that consumes that page stores it into the
  // pool page and into its staged copy before the page's scores
  const void* k_new;
  const void* v_new;
  int new_dtype;
};

// 8 consecutive values of a new K / V row as the pool's 16-bit type, rounded
// as sckv_append stores them (same type: copied; else through fp32, RN).
__device__ __forceinline__ uint4 new_row8(const void* src, int64_t idx, int src_dtype, int pool_dtype) {
  if (src_dtype == pool_dtype) return *reinterpret_cast<const uint4*>(reinterpret_cast<const uint16_t*>(src) + idx);
  float v[8];
  if (src_dtype == SCKV_DTYPE_F32) {
    const float4 a = *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(src) + idx);
    const float4 c = *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(src) + idx + 4);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = c.x; v[5] = c.y; v[6] = c.z; v[7] = c.w;
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = sckv_load_as_float(src, idx + i, src_dtype);
  }
  uint32_t w[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    if (pool_dtype == SCKV_DTYPE_F16) {
      __half2 h2 = __floats2half2_rn(v[2 * i], v[2 * i + 1]);
      w[i] = *reinterpret_cast<uint32_t*>(&h2);
    } else {
      __nv_bfloat162 b2 = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
      w[i] = *reinterpret_cast<uint32_t*>(&b2);
    }
  }
  return make_uint4(w[0], w[1], w[2], w[3]);
}

// Orders this thread's generic-proxy shared-memory stores before later
// async-proxy (bulk copy / TMA) writes to the same bytes.
__device__ __forceinline__ void fence_proxy_async_shared() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Page id and in-page row of sequence b's new token when the fused append
// applies to local page j (the page holding position ctx - 1), else -1. A
// context out of range (reported by clamp_ctx) or an invalid page id
// (reported by the producer) stores nothing.
__device__ __forceinline__ int32_t fused_append_page(const DecodeParams& p, int b, int ctx, int j, int* row) {
  if (p.k_new == nullptr || ctx < 1 || j != (ctx - 1) / SCKV_PAGE_TOKENS) return -1;
  if (__ldg(p.ctx_lens + b) != ctx) return -1;
  const int32_t page = __ldg(p.block_table + (int64_t)b * p.bt_stride + j);
  if (page < 0 || page >= p.max_pages) return -1;
  *row = (ctx - 1) % SCKV_PAGE_TOKENS;
  return page;
}

// One output element of (sequence b, q head hq, dim d).
__device__ __forceinline__ void store_out(const DecodeParams& p, int b, int hq, int d, float v) {
  if (p.n_peer == 0) {
    sckv_store_from_float(p.out, ((int64_t)b * p.hq + hq) * kHD + d, p.out_dtype, v);
    return;
  }
  const int64_t idx = p.out_off + ((int64_t)b * p.out_hq_total + p.out_head0 + hq) * kHD + d;
  for (int r = 0; r < p.n_peer; ++r) sckv_store_from_float(p.peer_out[r], idx, p.out_dtype, v);
}

__device__ __forceinline__ int clamp_ctx(const DecodeParams& p, int b, bool report) {
  int ctx = __ldg(p.ctx_lens + b);
  const int cap = p.max_blocks * SCKV_PAGE_TOKENS;
  if (ctx < 0 || ctx > cap) {
    if (report) sckv_report(p.status, SCKV_ERR_BOUNDS, ctx, KID_DECODE);
    ctx = ctx < 0 ? 0 : cap;
  }
  return ctx;
}

// Tensor-core decode for grouped-query heads (sckv_decode_mma.cu). Returns
// SCKV_ERR_UNSUPPORTED when the combination is not built there, so the
// caller can use the CUDA-core kernel instead.
int launch_decode_mma(const sckv_pool* pool, int G, const DecodeParams& prm, cudaStream_t stream);

// Causal prefill on tcgen05 / tensor memory (sckv_prefill_tc.cu) for f16 and
// bf16 pools; SCKV_ERR_UNSUPPORTED for anything else.
int launch_prefill_tc(const sckv_pool* pool, int layer, const void* q, int q_dtype, int num_q_heads, int n_seqs,
                      int n_tokens, const int32_t* cu_q, const int32_t* start_pos, const int32_t* block_table,
                      int64_t bt_stride, int max_blocks, float scale, void* out, int out_dtype, int lg_g,
                      cudaStream_t stream);

// Merge of split partials (shared by both decode kernels).
int launch_combine(const DecodeParams& prm, cudaStream_t stream);

}  // namespace sckv_detail
