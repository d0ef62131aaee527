// Definitions shared by the decode-attention translation units.
#pragma once

#include "sckv_internal.cuh"

namespace sckv_detail {

constexpr int kConsumerWarps = 4;
constexpr int kThreads = (kConsumerWarps + 1) * 32;
constexpr int kHD = 128;  // head_dim handled by this kernel

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
};

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
