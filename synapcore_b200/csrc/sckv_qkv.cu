// Fused attention input on the 5th-generation tensor cores: the q / k / v
// projections, the optional per-head QK-norm, RoPE and the K/V page append of
// one layer in one kernel.
//
// Replaces, for one layer of ModularAttentionEngine.forward_numpy
// (models/adapters.py:1148-1207): q/k/v = x @ W^T with fp16 weights
// (:1167-1169), the per-head RMSNorm of q and k (:1171-1185, rmsnorm_f32
// :1129-1132), RoPE at positions start + i (:1191-1192, apply_rope_f32
// :1134-1146) and the KV-cache concat of fp16(k), fp16(v) (:1194-1207). The
// rotated q goes to q_out for the attention kernels.
//
// One CTA computes a 128-token x 128-dim tile: one head of q, k or v
// (grid.x = q heads, then k heads, then v heads; grid.y = token tiles), so
// every thread of the epilogue owns one token's whole head vector in one
// tensor-memory lane and the norm and the (i, i + 64) rotation pairs stay
// inside the thread.
//   warp 0     TMA: per 64-wide step of the hidden dim, the x tile (and its
//              low part, for fp32 inputs split into hi + lo) and the weight
//              tile (128 rows of W), 128-byte swizzle, into a 4-stage ring.
//   warp 1     allocates 128 TMEM columns and issues
//              acc (128 x 128 fp32) += x . W^T   4 x tcgen05.mma (K = 16) per step
//              (8 with the low part); tcgen05.commit frees the stage.
//   warps 2-5  epilogue: tcgen05.ld of the thread's row, per-head RMSNorm,
//              RoPE with a per-token cos / sin table (computed once per call
//              by rope_table_kernel, the same operations as
//              sckv_append_rope), rounding to the output / pool type and
//              the stores (q_out row, or the K / V row of the token's page).
// The epilogue follows the reference's fp32 operation order with IEEE
// operations; the projection sums in fp32 in the tensor core's order.
//
// The same kernel in its plain mode is the output projection after
// attention, attn_out @ W_o^T with fp16 weights (models/adapters.py:1231):
// 128-column output tiles take the place of the heads, and the epilogue
// stores the fp32 sums (or their 16-bit rounding) with no norm, rotation or
// page append.
#include <cuda.h>
#include <math.h>

#include <algorithm>

#include "sckv_internal.cuh"
#include "sckv_mma_common.cuh"
#include "sckv_tcgen05.cuh"

using namespace sckv_mma;
using namespace sckv_tc;

namespace {

constexpr int kQkvBM = 128;                      // tokens per tile (UMMA M)
constexpr int kHead = 128;                       // head_dim: output dims of one head
constexpr int kQkvBK = 64;                       // hidden elements per step: 128-byte rows
constexpr int kQkvTile = kQkvBM * kQkvBK * 2;    // one 128-row operand tile: 16 KiB
constexpr int kQkvThreads = 192;
constexpr int kRopePairs = 64;                   // head_dim / 2

// kHeads heads of one kind per CTA: UMMA N = 128 kHeads (256 halves the
// shared-memory reads of x per flop; used when the grid still fills the GPU).
template <bool kSplit, int kHeads>
struct QkvCfg {
  static constexpr int kBN = kHead * kHeads;
  static constexpr int kStages = (kSplit && kHeads == 2) ? 3 : 4;
  static constexpr int kStageBytes = (2 + kHeads - 1 + (kSplit ? 1 : 0)) * kQkvTile;  // x, W (, x_lo)
  static constexpr int kOffW = kQkvTile;
  static constexpr int kOffLo = kQkvTile * (1 + kHeads);
  static constexpr int kBarOff = kStages * kStageBytes;
  static constexpr int kBytes = 1024 + kBarOff + (2 * kStages + 5) * 8 + 16;
  static constexpr uint32_t kTmemCols = 2 * kBN;  // double-buffered accumulator
};

struct QkvParams {
  void* q_out;
  void* pool_data;
  __half* pool_scales;     // int8 pools: fp16 per-token scales [L][P][K|V][H][16]
  __half* k_stage;         // FP8 pools: the new K / V rows [n_tok][Hkv][128] fp16, appended afterwards
  __half* v_stage;
  int32_t* status;
  const __half* q_norm_w;  // [128] or null
  const __half* k_norm_w;  // [128] or null
  const float2* rope_cs;   // [n_tok][64] (cos, sin); split: written by the projection kernel itself
  const float* inv_freq;   // [64]
  float rope_scaling;
  float* partial;          // split-K: fp32 sums per (tile, split), layout of split_part_index, else null
  const int32_t* cu;
  const int32_t* start_pos;
  const int32_t* bt;
  int64_t bt_stride;
  int64_t max_pages;
  int max_blocks;
  int n_seqs;
  int n_tok;
  int hidden;
  int hq;
  int hkv;
  int layer;
  int q_out_dtype;
  int pool_dtype;
  int k_steps_per_split;  // hidden steps of 64 per split
  int n_groups;           // head groups (of kHeads heads) over q, k and v
  int group_block;        // head groups per block of the tile order (see qkv_tile)
  int m_tiles;            // token tiles of 128
  int n_tiles;            // n_groups * m_tiles * splits
  int hd_total;           // (hq + 2 hkv) * 128 output columns
  int k_splits;           // splits of the hidden dim (1: none)
  int2* tok_meta;         // split: per token (position, page of its K/V slot or -1), written by the projection
  int plain;              // plain projection (o_proj): no norm, rotation or append
  float eps;
};

// Destination page row of token t (k / v): the slab (layer, page) of its
// block, or -1 (out-of-range position or page, reported once per token by
// the caller's choice of `report`).
__device__ __forceinline__ int64_t slab_at(const QkvParams& p, int b, int pos, bool report) {
  const int blk = pos / SCKV_PAGE_TOKENS;
  if (pos < 0 || blk >= p.max_blocks) {
    if (report) sckv_report(p.status, SCKV_ERR_BOUNDS, pos < 0 ? pos : blk, KID_QKV);
    return -1;
  }
  const int32_t page = __ldg(p.bt + (int64_t)b * p.bt_stride + blk);
  if (page < 0 || page >= p.max_pages) {
    if (report) sckv_report(p.status, SCKV_ERR_BOUNDS, page, KID_QKV);
    return -1;
  }
  return (int64_t)p.layer * p.max_pages + page;
}

__device__ __forceinline__ int64_t token_slab(const QkvParams& p, int t, int* pos_out, bool report) {
  const int b = sckv_find_seq(p.cu, p.n_seqs, t);
  const int pos = __ldg(p.start_pos + b) + (t - __ldg(p.cu + b));
  *pos_out = pos;
  return slab_at(p, b, pos, report);
}

// cos / sin of every (token, frequency) pair: position start_pos[b] + i
// divided by rope_scaling, times inv_freq[j], as sckv_append_rope computes
// them (apply_rope_f32, models/adapters.py:1134-1146).
__global__ void rope_table_kernel(const float* inv_freq, float rope_scaling, int n_seqs, int n_tok,
                                  const int32_t* cu, const int32_t* start_pos, float2* cs) {
  pdl_wait();
  pdl_trigger();
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (int64_t)n_tok * kRopePairs) return;
  const int t = (int)(idx / kRopePairs), j = (int)(idx % kRopePairs);
  const int b = sckv_find_seq(cu, n_seqs, t);
  const int pos = __ldg(start_pos + b) + (t - __ldg(cu + b));
  const float fpos = __fdiv_rn((float)pos, rope_scaling);
  const float ang = __fmul_rn(fpos, __ldg(inv_freq + j));
  float s, c;
  sincosf(ang, &s, &c);
  cs[idx] = make_float2(c, s);
}

// fp32 x -> hi = round(x), lo = round(x - hi) in the MMA's 16-bit type, so
// hi . W + lo . W carries x to ~2^-22 relative (W is exact in that type).
__global__ void split_hi_lo_kernel(const float* x, int64_t n, uint16_t* hi, uint16_t* lo, int bf16) {
  pdl_wait();
  pdl_trigger();
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const float v = x[i];
    if (bf16) {
      const __nv_bfloat16 h = __float2bfloat16_rn(v);
      const __nv_bfloat16 l = __float2bfloat16_rn(v - __bfloat162float(h));
      hi[i] = __bfloat16_as_ushort(h);
      lo[i] = __bfloat16_as_ushort(l);
    } else {
      const __half h = __float2half_rn(v);
      const __half l = __float2half_rn(v - __half2float(h));
      hi[i] = __half_as_ushort(h);
      lo[i] = __half_as_ushort(l);
    }
  }
}

// 32 fp32 values -> 32 elements of `dtype` at dst + idx (idx % 8 == 0, 16-byte aligned).
__device__ __forceinline__ void store32(void* dst, int64_t idx, int dtype, const float (&y)[32]) {
  if (dtype == SCKV_DTYPE_F32) {
    float4* d = reinterpret_cast<float4*>(reinterpret_cast<float*>(dst) + idx);
#pragma unroll
    for (int i = 0; i < 8; ++i) d[i] = make_float4(y[4 * i], y[4 * i + 1], y[4 * i + 2], y[4 * i + 3]);
  } else {
    const bool bf = dtype == SCKV_DTYPE_BF16;
    uint4* d = reinterpret_cast<uint4*>(reinterpret_cast<uint16_t*>(dst) + idx);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      uint32_t w[4];
#pragma unroll
      for (int k = 0; k < 4; ++k)
        w[k] = bf ? pack2<true>(y[8 * i + 2 * k], y[8 * i + 2 * k + 1])
                  : pack2<false>(y[8 * i + 2 * k], y[8 * i + 2 * k + 1]);
      d[i] = make_uint4(w[0], w[1], w[2], w[3]);
    }
  }
}

// int8 pools: a K or V row is stored as the arena quantises its fp16 pages
// (quantize_kv_int8_numpy, native/native_engine.py:207-215): the fp16 value
// x, s = max(max|x| / 127, 1e-7) in fp32, codes rint(x / s) clipped to
// +-127, s kept as fp16. IEEE division, as the append kernel does.
__device__ __forceinline__ float f16_round(float x) { return __half2float(__float2half_rn(x)); }
__device__ __forceinline__ float int8_row_scale(float amax) { return fmaxf(amax / 127.0f, 1e-7f); }
__device__ __forceinline__ uint32_t int8_code4(float a, float b, float c, float d, float s) {
  const float v[4] = {a, b, c, d};
  uint32_t w = 0;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float r = fminf(fmaxf(rintf(f16_round(v[i]) / s), -127.0f), 127.0f);
    w |= (uint32_t)(uint8_t)(int8_t)r << (8 * i);
  }
  return w;
}
__device__ __forceinline__ int64_t int8_scale_index(const QkvParams& p, int64_t slab, int kv, int head, int pos) {
  return ((slab * 2 + kv) * p.hkv + head) * SCKV_PAGE_TOKENS + pos % SCKV_PAGE_TOKENS;
}

// Split-K partial sums: per (head tile g = head + heads x token tile, split
// z) a 128-row x 128-column fp32 tile stored as [16 column octets][128
// rows][8]: the epilogue thread of row r writes its octets as 32-byte runs
// that sit side by side across the warp, and the finishing warp of a row
// reads each octet as two lanes' float4s, one full sector. Index of the
// first float of (g, z, octet, row).
__device__ __forceinline__ int64_t split_part_index(int64_t g, int ks, int z, int octet, int row) {
  return (((g * ks + z) * 16 + octet) * 128 + row) * 8;
}

// Split over the hidden dim: while its MMAs run, the projection kernel's
// epilogue warps look up every token's sequence, position and K/V page and
// its cos / sin row (the operations of rope_table_kernel), so the finishing
// kernel's loads are all independent. e = epilogue thread (0..127). A
// token whose slot is out of range is reported here, once.
__device__ __forceinline__ void token_meta(const QkvParams& p, int e) {
  float2* cs = const_cast<float2*>(p.rope_cs);
  for (int t = blockIdx.x * 128 + e; t < p.n_tok; t += gridDim.x * 128) {
    const int b = sckv_find_seq(p.cu, p.n_seqs, t);
    const int pos = __ldg(p.start_pos + b) + (t - __ldg(p.cu + b));
    const int64_t slab = slab_at(p, b, pos, true);
    p.tok_meta[t] = make_int2(pos, slab < 0 ? -1 : (int)(slab - (int64_t)p.layer * p.max_pages));
    const float fpos = __fdiv_rn((float)pos, p.rope_scaling);
    float4* d = reinterpret_cast<float4*>(cs + (int64_t)t * kRopePairs);
#pragma unroll 4
    for (int j = 0; j < kRopePairs; j += 2) {
      float s0, c0, s1, c1;
      sincosf(__fmul_rn(fpos, __ldg(p.inv_freq + j)), &s0, &c0);
      sincosf(__fmul_rn(fpos, __ldg(p.inv_freq + j + 1)), &s1, &c1);
      d[j >> 1] = make_float4(c0, s0, c1, s1);
    }
  }
}

// Split-K finish: one warp per (token, output head) adds the splits' fp32
// sums in split order, then applies the per-head RMSNorm, the rotation and
// the stores of the fused epilogue (plain mode: the stores only). Lane l
// holds dims 4l .. 4l + 3, so the rotation partner (d + 64) of lane l < 16
// is lane l + 16. Every load (partial sums, the token's position and page,
// its cos / sin) is independent of the others; 40 registers keep the grid
// of a 128-token decode batch in one wave.
__global__ void __launch_bounds__(256, 6) qkv_finish_kernel(const QkvParams p, int k_splits) {
  pdl_wait();
  pdl_trigger();
  const int lane = threadIdx.x & 31;
  const int64_t wid = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  const int n_heads = p.hq + 2 * p.hkv;
  if (wid >= (int64_t)p.n_tok * n_heads) return;
  const int t = (int)(wid / n_heads), hidx = (int)(wid % n_heads);
  const int kind = hidx < p.hq ? 0 : (hidx < p.hq + p.hkv ? 1 : 2);
  const int head = kind == 0 ? hidx : (kind == 1 ? hidx - p.hq : hidx - p.hq - p.hkv);
  const int64_t g = (int64_t)(t / kQkvBM) * n_heads + hidx;
  const float4* src = reinterpret_cast<const float4*>(p.partial + split_part_index(g, k_splits, 0, lane >> 1,
                                                                                    t % kQkvBM)) + (lane & 1);
  constexpr int64_t kSplitStride = 16 * 128 * 8 / 4;  // float4s between one split's tile and the next
  float4 v[4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
    if (i < k_splits) v[i] = __ldcg(src + i * kSplitStride);
  int2 meta = make_int2(0, 0);  // (position, page)
  float4 cs0 = make_float4(1.f, 0.f, 1.f, 0.f), cs1 = cs0;
  if (!p.plain) {
    meta = __ldg(p.tok_meta + t);
    if (kind < 2) {
      // (cos, sin) of dims 4l .. 4l + 3 (mod 64)
      const float4* c4 = reinterpret_cast<const float4*>(p.rope_cs + (int64_t)t * kRopePairs + ((4 * lane) & 63));
      cs0 = __ldg(c4);
      cs1 = __ldg(c4 + 1);
    }
  }
  float x[4] = {0.f, 0.f, 0.f, 0.f};
  for (int z0 = 0; z0 < k_splits; z0 += 4) {
    if (z0 > 0) {
#pragma unroll
      for (int i = 0; i < 4; ++i)
        if (z0 + i < k_splits) v[i] = __ldcg(src + (z0 + i) * kSplitStride);
    }
#pragma unroll
    for (int i = 0; i < 4; ++i)
      if (z0 + i < k_splits) {
        x[0] = __fadd_rn(x[0], v[i].x);
        x[1] = __fadd_rn(x[1], v[i].y);
        x[2] = __fadd_rn(x[2], v[i].z);
        x[3] = __fadd_rn(x[3], v[i].w);
      }
  }
  const __half* nw = kind == 0 ? p.q_norm_w : (kind == 1 ? p.k_norm_w : nullptr);
  if (nw != nullptr) {
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < 4; ++i) ss = __fmaf_rn(x[i], x[i], ss);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss = __fadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, o));
    const float inv = __fdiv_rn(1.f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)kHead), p.eps)));
#pragma unroll
    for (int i = 0; i < 4; ++i) x[i] = __fmul_rn(__fmul_rn(x[i], inv), __half2float(__ldg(nw + 4 * lane + i)));
  }
  float y[4] = {x[0], x[1], x[2], x[3]};
  if (kind < 2 && !p.plain) {
    const bool first = lane < 16;  // dims 4l.. in the first half; the partner lane holds d + 64
    const float cn[4] = {cs0.x, cs0.z, cs1.x, cs1.z}, sn[4] = {cs0.y, cs0.w, cs1.y, cs1.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float other = __shfl_xor_sync(0xffffffffu, x[i], 16);
      y[i] = first ? __fsub_rn(__fmul_rn(x[i], cn[i]), __fmul_rn(other, sn[i]))
                   : __fadd_rn(__fmul_rn(x[i], cn[i]), __fmul_rn(other, sn[i]));
    }
  }
  int64_t dst;
  void* out;
  int out_dtype;
  if (kind == 0) {
    dst = ((int64_t)t * p.hq + head) * kHead;
    out = p.q_out;
    out_dtype = p.q_out_dtype;
  } else if (p.k_stage != nullptr) {
    dst = ((int64_t)t * p.hkv + head) * kHead;
    out = kind == 1 ? p.k_stage : p.v_stage;
    out_dtype = SCKV_DTYPE_F16;
  } else {
    if (meta.y < 0) return;  // reported by token_meta
    const int64_t slab = (int64_t)p.layer * p.max_pages + meta.y;
    dst = (((slab * 2 + (kind - 1)) * p.hkv + head) * SCKV_PAGE_TOKENS + meta.x % SCKV_PAGE_TOKENS) * kHead;
    out = p.pool_data;
    out_dtype = p.pool_dtype;
  }
  dst += 4 * lane;
  if (out_dtype == SCKV_DTYPE_INT8) {
    // the row's scale: max over the warp's 128 fp16 values
    float m = fmaxf(fmaxf(fabsf(f16_round(y[0])), fabsf(f16_round(y[1]))),
                    fmaxf(fabsf(f16_round(y[2])), fabsf(f16_round(y[3]))));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    const float s8 = int8_row_scale(m);
    *reinterpret_cast<uint32_t*>(reinterpret_cast<uint8_t*>(out) + dst) = int8_code4(y[0], y[1], y[2], y[3], s8);
    if (lane == 0)
      p.pool_scales[int8_scale_index(p, (int64_t)p.layer * p.max_pages + meta.y, kind - 1, head, meta.x)] =
          __float2half_rn(s8);
  } else if (out_dtype == SCKV_DTYPE_F32) {
    *reinterpret_cast<float4*>(reinterpret_cast<float*>(out) + dst) = make_float4(y[0], y[1], y[2], y[3]);
  } else if (out_dtype == SCKV_DTYPE_BF16) {
    *reinterpret_cast<uint2*>(reinterpret_cast<uint16_t*>(out) + dst) =
        make_uint2(pack2<true>(y[0], y[1]), pack2<true>(y[2], y[3]));
  } else {
    *reinterpret_cast<uint2*>(reinterpret_cast<uint16_t*>(out) + dst) =
        make_uint2(pack2<false>(y[0], y[1]), pack2<false>(y[2], y[3]));
  }
}

// Geometry of work tile t. Head groups come in blocks of group_block:
// tiles run head group within the block fastest, then token tile, then
// block, then hidden split. CTAs working at the same time share each x tile
// (read by the block's groups together), and consecutive waves walk the
// token tiles of one block, whose weights (group_block x kHeads x 128 rows)
// stay in L2 until the next block starts; x is read once per block.
struct QkvTile {
  int kind, head0, kind_heads, m0, z, s0, nk;
};

template <int kHeads>
__device__ __forceinline__ QkvTile qkv_tile(const QkvParams& p, int t) {
  QkvTile q;
  const int gq = (p.hq + kHeads - 1) / kHeads, gk = (p.hkv + kHeads - 1) / kHeads;
  const int per_split = p.n_groups * p.m_tiles;
  q.z = t / per_split;
  const int r = t - q.z * per_split;
  const int blk = r / (p.group_block * p.m_tiles);
  const int r2 = r - blk * p.group_block * p.m_tiles;
  const int g0 = blk * p.group_block;
  const int gsz = min(p.group_block, p.n_groups - g0);  // the last block may be smaller
  const int m = r2 / gsz;
  const int gx = g0 + (r2 - m * gsz);
  q.m0 = m * kQkvBM;
  q.kind = gx < gq ? 0 : (gx < gq + gk ? 1 : 2);  // q, k, v
  q.head0 = (gx - (q.kind == 0 ? 0 : (q.kind == 1 ? gq : gq + gk))) * kHeads;
  q.kind_heads = q.kind == 0 ? p.hq : p.hkv;
  const int nk_all = (p.hidden + kQkvBK - 1) / kQkvBK;
  q.s0 = q.z * p.k_steps_per_split;
  q.nk = min(nk_all - q.s0, p.k_steps_per_split);
  return q;
}

// Persistent: one CTA per SM walks tiles blockIdx.x, + gridDim.x, ...; the
// accumulator is double-buffered in tensor memory (2 x 128 kHeads columns),
// so the MMAs of a CTA's next tile run while its epilogue drains the last.
template <bool kBF16, bool kSplit, int kHeads>
__global__ void __launch_bounds__(kQkvThreads, 1)
    qkv_append_kernel(const QkvParams p, const __grid_constant__ CUtensorMap xmap,
                      const __grid_constant__ CUtensorMap xlomap, const __grid_constant__ CUtensorMap wqmap,
                      const __grid_constant__ CUtensorMap wkmap, const __grid_constant__ CUtensorMap wvmap) {
  using SM = QkvCfg<kSplit, kHeads>;
  constexpr int kQkvStages = SM::kStages;
  extern __shared__ __align__(16) uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(base + SM::kBarOff);  // [S] stage landed (TMA)
  uint64_t* empty = full + kQkvStages;                               // [S] stage read by its MMAs (commit)
  uint64_t* acc_full = empty + kQkvStages;                           // [2] a tile's MMAs finished (commit)
  uint64_t* acc_empty = acc_full + 2;                                // [2] its epilogue read it (128 threads)
  uint64_t* mma_done = acc_empty + 2;                                // every MMA issued finished (drain)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kQkvStages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], 128);
    }
    mbar_init(mma_done, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, SM::kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // the set-up above may overlap the previous kernel; the inputs may not
  pdl_wait();
  pdl_trigger();

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&xmap)) : "memory");
      uint32_t gcount = 0;  // stages issued by this CTA
      bool aborted = false;
      for (int t = blockIdx.x; t < p.n_tiles && !aborted; t += gridDim.x) {
        const QkvTile tl = qkv_tile<kHeads>(p, t);
        const CUtensorMap* wmap = tl.kind == 0 ? &wqmap : (tl.kind == 1 ? &wkmap : &wvmap);
        const int row0 = tl.head0 * kHead;  // rows past the last head read as zeros
        for (int s = 0; s < tl.nk; ++s) {
          const uint32_t st = gcount % kQkvStages;
          if (gcount >= kQkvStages) {
            if (*abort_flag ||
                !mbar_wait_bounded(&empty[st], ((gcount / kQkvStages) - 1) & 1, SCKV_WAIT_LIMIT_NS)) {
              if (!*abort_flag) sckv_report(p.status, SCKV_ERR_TIMEOUT, blockIdx.x, KID_QKV);
              *abort_flag = 1;
              aborted = true;
              break;
            }
          }
          const uint32_t stage = smem_u32(base + st * SM::kStageBytes);
          mbar_arrive_expect_tx(&full[st], SM::kStageBytes);
          const int kx = (tl.s0 + s) * kQkvBK;
          tma_load_2d(stage, &xmap, kx, tl.m0, &full[st]);
          tma_load_2d(stage + SM::kOffW, wmap, kx, row0, &full[st]);
          if (kSplit) tma_load_2d(stage + SM::kOffLo, &xlomap, kx, tl.m0, &full[st]);
          ++gcount;
        }
      }
      // copies still in flight land before the CTA may exit
      for (uint32_t k = gcount > kQkvStages ? gcount - kQkvStages : 0; k < gcount; ++k)
        mbar_wait_bounded(&full[k % kQkvStages], (k / kQkvStages) & 1, SCKV_WAIT_LIMIT_NS);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    constexpr uint32_t kIdesc = instr_desc_f16(kBF16, SM::kBN, false);
    const uint64_t stage_desc0 = smem_desc_sw128(smem_u32(base), 16, 1024);  // stage 0's x tile
    bool ok = true;
    uint32_t gcount = 0;  // stages consumed
    int lt = 0;           // tiles of this CTA
    for (int t = blockIdx.x; t < p.n_tiles && ok; t += gridDim.x, ++lt) {
      const QkvTile tl = qkv_tile<kHeads>(p, t);
      const int buf = lt & 1;
      // the buffer's previous tile (lt - 2) has been read by the epilogue
      if (lt >= 2 && (*abort_flag || !warp_wait(&acc_empty[buf], ((lt >> 1) - 1) & 1))) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t acc = tmem + (uint32_t)(buf * SM::kBN);
      for (int s = 0; s < tl.nk; ++s) {
        const uint32_t st = gcount % kQkvStages;
        if (*abort_flag || !warp_wait(&full[st], (gcount / kQkvStages) & 1)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (lane == 0) {
          // A = x rows (tokens), B = W rows (output dims), both K-major:
          // 128-byte rows, 8-row groups 1024 bytes apart; K = 16 is 32 bytes
          const uint64_t adesc = desc_advance(stage_desc0, st * (uint32_t)SM::kStageBytes);
          const uint64_t bdesc = desc_advance(adesc, (uint32_t)SM::kOffW);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            const uint64_t bk = desc_advance(bdesc, (uint32_t)(kk * 32));
            umma_ss(acc, desc_advance(adesc, (uint32_t)(kk * 32)), bk, kIdesc, (s > 0 || kk > 0) ? 1u : 0u);
            if (kSplit) umma_ss(acc, desc_advance(adesc, (uint32_t)(SM::kOffLo + kk * 32)), bk, kIdesc, 1u);
          }
          umma_commit(&empty[st]);
        }
        __syncwarp();
        ++gcount;
      }
      if (!ok) break;
      if (lane == 0) umma_commit(&acc_full[buf]);
      __syncwarp();
    }
    if (!ok) {
      if (lane == 0 && !*abort_flag) sckv_report(p.status, SCKV_ERR_TIMEOUT, blockIdx.x, KID_QKV);
      if (lane == 0) *abort_flag = 1;
    }
    // every MMA issued above has finished before the tensor memory is freed
    if (lane == 0) umma_commit(mma_done);
    __syncwarp();
    warp_wait(mma_done, 0);
  } else {
    // ------------------------------------------------------------ epilogue
    const int quad = warp & 3;  // TMEM lanes 32 quad .. 32 quad + 31
    int lt = 0;
    for (int t = blockIdx.x; t < p.n_tiles; t += gridDim.x, ++lt) {
      const QkvTile tl = qkv_tile<kHeads>(p, t);
      const int buf = lt & 1;
      const int tok = tl.m0 + quad * 32 + lane;
      // split: per-token lookups for the finishing kernel, while the MMAs run
      if (p.partial != nullptr && lt == 0 && !p.plain) token_meta(p, threadIdx.x - 64);
      const bool ready = warp_wait(&acc_full[buf], (lt >> 1) & 1);
      tc_fence_after();
      // warp-uniform: the tensor-memory loads below are warp-wide
      const int aborted = __shfl_sync(0xffffffffu, *abort_flag, 0);
      if (!ready || aborted) break;
      const uint32_t acc = tmem + (uint32_t)(buf * SM::kBN) + ((uint32_t)(quad * 32) << 16);
      if (p.partial != nullptr) {
        // split-K: raw fp32 sums of this split (rows past the last token
        // too); qkv_finish_kernel adds the splits and applies the norm,
        // rotation and stores
        const int n_heads = p.hq + 2 * p.hkv;
        const int hidx = (tl.kind == 0 ? 0 : (tl.kind == 1 ? p.hq : p.hq + p.hkv)) + tl.head0;
        const int64_t g = (int64_t)(tl.m0 / kQkvBM) * n_heads + hidx;
        const int row = quad * 32 + lane;
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          uint32_t r[32];
          tmem_ld32(acc + c * 32, r);
          tc_wait_ld();
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            float4* d4 = reinterpret_cast<float4*>(p.partial + split_part_index(g, p.k_splits, tl.z, c * 4 + q, row));
            d4[0] = make_float4(__uint_as_float(r[8 * q]), __uint_as_float(r[8 * q + 1]),
                                __uint_as_float(r[8 * q + 2]), __uint_as_float(r[8 * q + 3]));
            d4[1] = make_float4(__uint_as_float(r[8 * q + 4]), __uint_as_float(r[8 * q + 5]),
                                __uint_as_float(r[8 * q + 6]), __uint_as_float(r[8 * q + 7]));
          }
        }
      } else {
        const __half* nw = tl.kind == 0 ? p.q_norm_w : (tl.kind == 1 ? p.k_norm_w : nullptr);
        const bool live = tok < p.n_tok;
        // the token's page slab (k and v tiles); q rows go to q_out; FP8
        // pools stage the k / v rows for the FP8 append
        const bool stage = tl.kind > 0 && p.k_stage != nullptr;  // tile-uniform
        int pos = 0;
        const int64_t slot_row = (live && tl.kind > 0 && !stage) ? token_slab(p, tok, &pos, tl.head0 == 0) : -1;
#pragma unroll 1
        for (int hh = 0; hh < kHeads; ++hh) {
          const int head = tl.head0 + hh;
          if (head >= tl.kind_heads) break;  // warp-uniform
          const uint32_t trow = acc + (uint32_t)(hh * kHead);
          // every lane reads the tensor memory (the loads are warp-wide); rows
          // past the last token are computed and dropped
          float inv = 1.f;
          if (nw != nullptr) {
            float ss = 0.f;
#pragma unroll
            for (int c = 0; c < 4; ++c) {
              uint32_t r[32];
              tmem_ld32(trow + c * 32, r);
              tc_wait_ld();
#pragma unroll
              for (int i = 0; i < 32; ++i) {
                const float x = __uint_as_float(r[i]);
                ss = __fmaf_rn(x, x, ss);
              }
            }
            inv = __fdiv_rn(1.f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)kHead), p.eps)));
          }
          int64_t dst = -1;
          void* out = p.q_out;
          int out_dtype = p.q_out_dtype;
          if (live && tl.kind == 0) {
            dst = ((int64_t)tok * p.hq + head) * kHead;
          } else if (live && stage) {
            dst = ((int64_t)tok * p.hkv + head) * kHead;
            out = tl.kind == 1 ? p.k_stage : p.v_stage;
            out_dtype = SCKV_DTYPE_F16;
          } else if (slot_row >= 0) {
            // data layout [L][P][K|V][H][16][D]
            dst = (((slot_row * 2 + (tl.kind - 1)) * p.hkv + head) * SCKV_PAGE_TOKENS + pos % SCKV_PAGE_TOKENS) *
                  kHead;
            out = p.pool_data;
            out_dtype = p.pool_dtype;
          }
          // int8 pools: a first pass finds the row's largest fp16 magnitude,
          // the second stores the codes (tile-uniform, so the tensor-memory
          // loads stay warp-wide)
          const bool q8 = tl.kind > 0 && p.pool_dtype == SCKV_DTYPE_INT8;
          float amax = 0.f, s8 = 1.f;
#pragma unroll 1
          for (int pass = q8 ? 0 : 1; pass < 2; ++pass) {
#pragma unroll 1
          for (int hf = 0; hf < 2; ++hf) {
            // dims d = 32 hf + i and their rotation partners d + 64
            uint32_t r1[32], r2[32];
            tmem_ld32(trow + hf * 32, r1);
            tmem_ld32(trow + 64 + hf * 32, r2);
            tc_wait_ld();
            if (dst < 0) continue;
            float y1[32], y2[32];
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              const int d = hf * 32 + i;
              float x1 = __uint_as_float(r1[i]), x2 = __uint_as_float(r2[i]);
              if (nw != nullptr) {
                x1 = __fmul_rn(__fmul_rn(x1, inv), __half2float(__ldg(nw + d)));
                x2 = __fmul_rn(__fmul_rn(x2, inv), __half2float(__ldg(nw + d + kRopePairs)));
              }
              if (tl.kind < 2 && !p.plain) {
                const float2 cs = __ldg(p.rope_cs + (int64_t)tok * kRopePairs + d);
                y1[i] = __fsub_rn(__fmul_rn(x1, cs.x), __fmul_rn(x2, cs.y));
                y2[i] = __fadd_rn(__fmul_rn(x2, cs.x), __fmul_rn(x1, cs.y));
              } else {
                y1[i] = x1;
                y2[i] = x2;
              }
            }
            if (!q8) {
              store32(out, dst + hf * 32, out_dtype, y1);
              store32(out, dst + 64 + hf * 32, out_dtype, y2);
            } else if (pass == 0) {
#pragma unroll
              for (int i = 0; i < 32; ++i)
                amax = fmaxf(amax, fmaxf(fabsf(f16_round(y1[i])), fabsf(f16_round(y2[i]))));
            } else {
              uint8_t* o8 = reinterpret_cast<uint8_t*>(out);
#pragma unroll
              for (int half = 0; half < 2; ++half) {
                const float* y = half ? y2 : y1;
                uint4* d4 = reinterpret_cast<uint4*>(o8 + dst + half * 64 + hf * 32);
#pragma unroll
                for (int v = 0; v < 2; ++v)
                  d4[v] = make_uint4(int8_code4(y[16 * v], y[16 * v + 1], y[16 * v + 2], y[16 * v + 3], s8),
                                     int8_code4(y[16 * v + 4], y[16 * v + 5], y[16 * v + 6], y[16 * v + 7], s8),
                                     int8_code4(y[16 * v + 8], y[16 * v + 9], y[16 * v + 10], y[16 * v + 11], s8),
                                     int8_code4(y[16 * v + 12], y[16 * v + 13], y[16 * v + 14], y[16 * v + 15], s8));
              }
            }
          }
          if (q8 && pass == 0) {
            s8 = int8_row_scale(amax);
            if (dst >= 0)
              p.pool_scales[int8_scale_index(p, slot_row, tl.kind - 1, head, pos)] = __float2half_rn(s8);
          }
          }
        }
      }
      // the accumulator buffer may take the tile after next
      tc_fence_before();
      mbar_arrive(&acc_empty[buf]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, SM::kTmemCols);
  }
}

// 2-D map over a row-major [rows][hidden] 16-bit matrix, boxes of 64 x box_rows.
int encode_rows(CUtensorMap* map, const void* ptr, int rows, int hidden, bool bf16, int box_rows) {
  PFN_cuTensorMapEncodeTiled_v12000 encode = tensor_map_encoder();
  if (encode == nullptr) return SCKV_ERR_CUDA;
  const cuuint64_t dims[2] = {(cuuint64_t)hidden, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)hidden * 2};
  const cuuint32_t box[2] = {(cuuint32_t)kQkvBK, (cuuint32_t)box_rows};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = encode(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
                            const_cast<void*>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                            CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? SCKV_OK : sckv_record_error(__FILE__, __LINE__, "cuTensorMapEncodeTiled", "failed");
}

template <bool kBF16, bool kSplit, int kHeads>
int launch_qkv(const QkvParams& prm_in, const CUtensorMap (&maps)[5], int n_groups, int m_tiles, int num_sms,
               cudaStream_t stream, int k_splits = 1) {
  auto kern = qkv_append_kernel<kBF16, kSplit, kHeads>;
  constexpr int smem = QkvCfg<kSplit, kHeads>::kBytes;
  static_assert(smem <= 227 * 1024, "shared memory");
  QkvParams prm = prm_in;
  prm.n_groups = n_groups;
  prm.m_tiles = m_tiles;
  // weights of one block of head groups: at most ~40 MB of L2, blocks of
  // equal size
  const int64_t w_group_bytes = (int64_t)QkvCfg<kSplit, kHeads>::kBN * prm.hidden * 2;
  const int64_t n_blocks = std::max<int64_t>(1, (n_groups * w_group_bytes + (40LL << 20) - 1) / (40LL << 20));
  prm.group_block = (int)((n_groups + n_blocks - 1) / n_blocks);
  const int64_t n_tiles = (int64_t)n_groups * m_tiles * k_splits;
  if (n_tiles > INT32_MAX) return SCKV_ERR_UNSUPPORTED;
  prm.n_tiles = (int)n_tiles;
  SCKV_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
  // persistent: one CTA per SM (the shared memory allows no second)
  const int grid = (int)(n_tiles < num_sms ? n_tiles : num_sms);
  SCKV_CUDA_CHECK(sckv_launch_pdl(kern, dim3(grid), dim3(kQkvThreads), smem, stream, prm, maps[0], maps[1],
                                  maps[2], maps[3], maps[4]));
  SCKV_LAUNCH_CHECK();
  return SCKV_OK;
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

// Hidden steps per split: the whole hidden dim when the token tiles x heads
// already give every other SM a CTA, else split so about one CTA per SM
// streams a slice of the weights (at least 4 steps of 64 per split).
int qkv_steps_per_split(int64_t n_tokens, int64_t n_heads, int hidden, int num_sms) {
  const int nk = (hidden + kQkvBK - 1) / kQkvBK;
  const int64_t ctas = ((n_tokens + kQkvBM - 1) / kQkvBM) * n_heads;
  if (ctas * 2 > num_sms || nk < 8) return nk;
  // about one tile per SM (two per SM measured slower: the finishing pass
  // then reads twice the partial sums)
  int64_t ks = num_sms / ctas;
  ks = ks < 2 ? 2 : (ks > 8 ? 8 : ks);
  if (ks > nk / 4) ks = nk / 4;
  return (int)((nk + ks - 1) / ks);
}

// Split-K partial sums: a 128 x 128 fp32 tile per (output tile, token tile, split).
size_t split_part_bytes(int64_t n_tokens, int64_t n_tiles_out, int64_t ks) {
  if (ks <= 1) return 0;
  return (size_t)ks * n_tiles_out * ((n_tokens + kQkvBM - 1) / kQkvBM) * kQkvBM * kHead * sizeof(float);
}

// Workspace of one sckv_qkv_append call, in order: the cos / sin table;
// split over the hidden dim, the partial sums and the per-token lookups;
// for FP8 pools, the new K and V rows in fp16 (the FP8 append takes them
// from there). Offsets are 256-byte aligned.
struct QkvWs {
  size_t part, meta, kstage, vstage, total;
};

inline size_t align256(size_t b) { return (b + 255) & ~size_t(255); }

QkvWs qkv_workspace(int64_t n_tokens, int64_t hkv, int64_t n_heads, int hidden, int num_sms, bool stage_kv) {
  const int per = qkv_steps_per_split(n_tokens, n_heads, hidden, num_sms);
  const int nk = (hidden + kQkvBK - 1) / kQkvBK;
  const int64_t ks = (nk + per - 1) / per;
  QkvWs w;
  w.part = align256((size_t)n_tokens * kRopePairs * sizeof(float2));
  w.meta = align256(w.part + split_part_bytes(n_tokens, n_heads, ks));
  w.kstage = align256(w.meta + (ks > 1 ? (size_t)n_tokens * sizeof(int2) : 0));
  const size_t rows = stage_kv ? (size_t)n_tokens * hkv * kHead * sizeof(__half) : 0;
  w.vstage = align256(w.kstage + rows);
  w.total = w.vstage + rows;
  return w;
}

size_t oproj_workspace_bytes(int64_t n_tokens, int in_features, int out_features, int num_sms) {
  const int64_t n_out = out_features / kHead;
  if (n_out <= 0) return 0;
  const int per = qkv_steps_per_split(n_tokens, n_out, in_features, num_sms);
  const int nk = (in_features + kQkvBK - 1) / kQkvBK;
  return split_part_bytes(n_tokens, n_out, (nk + per - 1) / per);
}

// The projection launch (and, split over the hidden dim, the finishing
// pass) for the fused q / k / v kernel and the plain output projection.
int launch_projection(const QkvParams& prm, const CUtensorMap (&maps)[5], bool bf16, bool has_lo, int k_splits,
                      int heads, int n_groups, int mt, int sms, cudaStream_t s) {
  if (k_splits > 1) {
    const int rc = has_lo ? (bf16 ? launch_qkv<true, true, 1>(prm, maps, n_groups, mt, sms, s, k_splits)
                                  : launch_qkv<false, true, 1>(prm, maps, n_groups, mt, sms, s, k_splits))
                          : (bf16 ? launch_qkv<true, false, 1>(prm, maps, n_groups, mt, sms, s, k_splits)
                                  : launch_qkv<false, false, 1>(prm, maps, n_groups, mt, sms, s, k_splits));
    if (rc != SCKV_OK) return rc;
    const int64_t warps = (int64_t)prm.n_tok * (prm.hq + 2 * prm.hkv);
    SCKV_CUDA_CHECK(sckv_launch_pdl(qkv_finish_kernel, dim3((unsigned)((warps + 7) / 8)), dim3(256), 0, s, prm,
                                    k_splits));
    SCKV_LAUNCH_CHECK();
    return SCKV_OK;
  }
  if (heads == 2) {
    if (bf16)
      return has_lo ? launch_qkv<true, true, 2>(prm, maps, n_groups, mt, sms, s)
                    : launch_qkv<true, false, 2>(prm, maps, n_groups, mt, sms, s);
    return has_lo ? launch_qkv<false, true, 2>(prm, maps, n_groups, mt, sms, s)
                  : launch_qkv<false, false, 2>(prm, maps, n_groups, mt, sms, s);
  }
  if (bf16)
    return has_lo ? launch_qkv<true, true, 1>(prm, maps, n_groups, mt, sms, s)
                  : launch_qkv<true, false, 1>(prm, maps, n_groups, mt, sms, s);
  return has_lo ? launch_qkv<false, true, 1>(prm, maps, n_groups, mt, sms, s)
                : launch_qkv<false, false, 1>(prm, maps, n_groups, mt, sms, s);
}

}  // namespace

extern "C" size_t sckv_qkv_workspace_bytes(const sckv_pool* pool, int n_tokens, int num_q_heads, int hidden) {
  if (pool == nullptr || n_tokens < 0 || num_q_heads <= 0 || hidden <= 0) return 0;
  return qkv_workspace(n_tokens, pool->num_kv_heads, (int64_t)num_q_heads + 2LL * pool->num_kv_heads, hidden,
                       pool->num_sms, pool->kv_dtype == SCKV_DTYPE_FP8_E4M3)
      .total;
}

extern "C" int sckv_split_hi_lo(const float* x, int64_t n, void* hi, void* lo, int dtype, void* stream) {
  if (n < 0 || (n > 0 && (!x || !hi || !lo))) return SCKV_ERR_INVALID_ARG;
  if (dtype != SCKV_DTYPE_F16 && dtype != SCKV_DTYPE_BF16) return SCKV_ERR_INVALID_ARG;
  if (n == 0) return SCKV_OK;
  const int64_t blocks = (n + 255) / 256;
  SCKV_CUDA_CHECK(sckv_launch_pdl(split_hi_lo_kernel, dim3((unsigned)(blocks < 4096 ? blocks : 4096)), dim3(256), 0,
                                  as_stream(stream), x, n, reinterpret_cast<uint16_t*>(hi),
                                  reinterpret_cast<uint16_t*>(lo), (int)(dtype == SCKV_DTYPE_BF16)));
  SCKV_LAUNCH_CHECK();
  return SCKV_OK;
}

extern "C" int sckv_qkv_append(sckv_pool* pool, int layer, const void* x, const void* x_lo, int x_dtype,
                               int n_tokens, int hidden, const void* w_q, const void* w_k, const void* w_v,
                               int num_q_heads, const void* q_norm_w, int q_norm_len, const void* k_norm_w,
                               int k_norm_len, float eps, const float* inv_freq, float rope_scaling, int n_seqs,
                               const int32_t* cu_tokens, const int32_t* start_pos, const int32_t* block_table,
                               int64_t bt_stride, int max_blocks, void* q_out, int q_out_dtype, void* workspace,
                               size_t workspace_bytes, void* stream) {
  if (pool == nullptr || layer < 0 || layer >= pool->num_layers) return SCKV_ERR_INVALID_ARG;
  if (n_tokens < 0 || n_seqs < 0 || num_q_heads <= 0 || hidden <= 0) return SCKV_ERR_INVALID_ARG;
  if (x_dtype != SCKV_DTYPE_F16 && x_dtype != SCKV_DTYPE_BF16) return SCKV_ERR_INVALID_ARG;
  if (q_out_dtype != SCKV_DTYPE_F32 && q_out_dtype != SCKV_DTYPE_F16 && q_out_dtype != SCKV_DTYPE_BF16)
    return SCKV_ERR_INVALID_ARG;
  // 16-bit pools; int8 pools (each K / V row quantised as the arena does);
  // FP8 pools through a second launch (their page scales span 16 tokens)
  if (pool->kv_dtype != SCKV_DTYPE_F16 && pool->kv_dtype != SCKV_DTYPE_BF16 && pool->kv_dtype != SCKV_DTYPE_INT8 &&
      pool->kv_dtype != SCKV_DTYPE_FP8_E4M3)
    return SCKV_ERR_UNSUPPORTED;
  if (pool->head_dim != kHead) return SCKV_ERR_UNSUPPORTED;
  // norms over the whole projection need every head of a token: the
  // unfused path (projection, then sckv_append_rope) covers them
  if ((q_norm_len != 0 && q_norm_len != kHead) || (k_norm_len != 0 && k_norm_len != kHead))
    return SCKV_ERR_UNSUPPORTED;
  if ((q_norm_len != 0 && q_norm_w == nullptr) || (k_norm_len != 0 && k_norm_w == nullptr))
    return SCKV_ERR_INVALID_ARG;
  if (hidden % 8 != 0) return SCKV_ERR_UNSUPPORTED;  // 16-byte row pitch for the tensor maps
  if (n_tokens == 0 || n_seqs == 0) return SCKV_OK;
  if (!x || !w_q || !w_k || !w_v || !inv_freq || !cu_tokens || !start_pos || !block_table || !q_out ||
      !workspace || max_blocks <= 0 || bt_stride < max_blocks || !(rope_scaling != 0.f))
    return SCKV_ERR_INVALID_ARG;
  const bool stage_kv = pool->kv_dtype == SCKV_DTYPE_FP8_E4M3;
  const QkvWs ws = qkv_workspace(n_tokens, pool->num_kv_heads, (int64_t)num_q_heads + 2LL * pool->num_kv_heads,
                                 hidden, pool->num_sms, stage_kv);
  if (workspace_bytes < ws.total) return SCKV_ERR_INVALID_ARG;
  if (!aligned16(x) || (x_lo && !aligned16(x_lo)) || !aligned16(w_q) || !aligned16(w_k) || !aligned16(w_v) ||
      !aligned16(q_out) || !aligned16(workspace))
    return SCKV_ERR_ALIGNMENT;
  const int hkv = pool->num_kv_heads;
  const int64_t n_heads = (int64_t)num_q_heads + 2LL * hkv;
  const int64_t m_tiles = ((int64_t)n_tokens + kQkvBM - 1) / kQkvBM;
  if (n_heads > INT32_MAX || m_tiles > 65535) return SCKV_ERR_UNSUPPORTED;
  if ((int64_t)num_q_heads * kHead > INT32_MAX || (int64_t)hkv * kHead > INT32_MAX) return SCKV_ERR_UNSUPPORTED;

  // two heads per CTA (N = 256) once that still gives every SM a tile;
  // split over the hidden dim when even one head per CTA leaves SMs idle
  const int64_t groups2 = (num_q_heads + 1) / 2 + 2 * ((hkv + 1) / 2);
  const int per_split = qkv_steps_per_split(n_tokens, n_heads, hidden, pool->num_sms);
  const int nk = (hidden + kQkvBK - 1) / kQkvBK;
  const int k_splits = (nk + per_split - 1) / per_split;
  const int heads = (k_splits == 1 && groups2 * m_tiles >= pool->num_sms) ? 2 : 1;
  const int n_groups = heads == 2 ? (int)groups2 : (int)n_heads;

  const bool bf16 = x_dtype == SCKV_DTYPE_BF16;
  CUtensorMap maps[5];
  int rc = encode_rows(&maps[0], x, n_tokens, hidden, bf16, kQkvBM);
  if (rc == SCKV_OK) rc = encode_rows(&maps[1], x_lo ? x_lo : x, n_tokens, hidden, bf16, kQkvBM);
  if (rc == SCKV_OK) rc = encode_rows(&maps[2], w_q, num_q_heads * kHead, hidden, bf16, heads * kHead);
  if (rc == SCKV_OK) rc = encode_rows(&maps[3], w_k, hkv * kHead, hidden, bf16, heads * kHead);
  if (rc == SCKV_OK) rc = encode_rows(&maps[4], w_v, hkv * kHead, hidden, bf16, heads * kHead);
  if (rc != SCKV_OK) return rc;

  cudaStream_t s = as_stream(stream);
  SCKV_DEVICE_GUARD(pool->device);
  float2* cs = reinterpret_cast<float2*>(workspace);
  if (k_splits == 1) {
    // the fused epilogue reads a per-token cos / sin table (split over the
    // hidden dim, the projection kernel fills it while its MMAs run)
    const int64_t n_cs = (int64_t)n_tokens * kRopePairs;
    SCKV_CUDA_CHECK(sckv_launch_pdl(rope_table_kernel, dim3((unsigned)((n_cs + 255) / 256)), dim3(256), 0, s,
                                    inv_freq, rope_scaling, n_seqs, n_tokens, cu_tokens, start_pos, cs));
    SCKV_LAUNCH_CHECK();
  }

  QkvParams prm{};
  prm.q_out = q_out;
  prm.pool_data = pool->data;
  prm.pool_scales = reinterpret_cast<__half*>(pool->scales);
  prm.status = pool->status;
  prm.q_norm_w = q_norm_len ? reinterpret_cast<const __half*>(q_norm_w) : nullptr;
  prm.k_norm_w = k_norm_len ? reinterpret_cast<const __half*>(k_norm_w) : nullptr;
  prm.rope_cs = cs;
  prm.inv_freq = inv_freq;
  prm.rope_scaling = rope_scaling;
  prm.cu = cu_tokens;
  prm.start_pos = start_pos;
  prm.bt = block_table;
  prm.bt_stride = bt_stride;
  prm.max_pages = pool->max_pages;
  prm.max_blocks = max_blocks;
  prm.n_seqs = n_seqs;
  prm.n_tok = n_tokens;
  prm.hidden = hidden;
  prm.hq = num_q_heads;
  prm.hkv = hkv;
  prm.layer = layer;
  prm.q_out_dtype = q_out_dtype;
  prm.pool_dtype = pool->kv_dtype;
  prm.eps = eps;
  prm.k_steps_per_split = per_split;
  prm.hd_total = (int)(n_heads * kHead);
  prm.k_splits = k_splits;
  char* wsb = reinterpret_cast<char*>(workspace);
  if (k_splits > 1) {
    prm.partial = reinterpret_cast<float*>(wsb + ws.part);
    prm.tok_meta = reinterpret_cast<int2*>(wsb + ws.meta);
  }
  if (stage_kv) {
    prm.k_stage = reinterpret_cast<__half*>(wsb + ws.kstage);
    prm.v_stage = reinterpret_cast<__half*>(wsb + ws.vstage);
  }
  rc = launch_projection(prm, maps, bf16, x_lo != nullptr, k_splits, heads, n_groups, (int)m_tiles,
                         pool->num_sms, s);
  if (rc != SCKV_OK || !stage_kv) return rc;
  // FP8 pools: the page-head scales grow with the tokens a page holds, so
  // the rows go through the FP8 append (scale growth, re-encoding)
  return sckv_append(pool, layer, 1, prm.k_stage, prm.v_stage, SCKV_DTYPE_F16, n_seqs, n_tokens, cu_tokens,
                     start_pos, block_table, bt_stride, max_blocks, stream);
}

extern "C" size_t sckv_o_proj_workspace_bytes(const sckv_pool* pool, int n_tokens, int in_features,
                                              int out_features) {
  if (pool == nullptr || n_tokens < 0 || in_features <= 0 || out_features <= 0) return 0;
  return oproj_workspace_bytes(n_tokens, in_features, out_features, pool->num_sms);
}

extern "C" int sckv_o_proj(sckv_pool* pool, const void* x, const void* x_lo, int x_dtype, int n_tokens,
                           int in_features, const void* w_o, int out_features, void* out, int out_dtype,
                           void* workspace, size_t workspace_bytes, void* stream) {
  if (pool == nullptr || n_tokens < 0 || in_features <= 0 || out_features <= 0) return SCKV_ERR_INVALID_ARG;
  if (x_dtype != SCKV_DTYPE_F16 && x_dtype != SCKV_DTYPE_BF16) return SCKV_ERR_INVALID_ARG;
  if (out_dtype != SCKV_DTYPE_F32 && out_dtype != SCKV_DTYPE_F16 && out_dtype != SCKV_DTYPE_BF16)
    return SCKV_ERR_INVALID_ARG;
  // 128-column output tiles are stored whole; 16-byte row pitch for the tensor maps
  if (out_features % kHead != 0 || in_features % 8 != 0) return SCKV_ERR_UNSUPPORTED;
  if (n_tokens == 0) return SCKV_OK;
  if (!x || !w_o || !out) return SCKV_ERR_INVALID_ARG;
  const size_t need = oproj_workspace_bytes(n_tokens, in_features, out_features, pool->num_sms);
  if (need > 0 && (workspace == nullptr || workspace_bytes < need)) return SCKV_ERR_INVALID_ARG;
  if (!aligned16(x) || (x_lo && !aligned16(x_lo)) || !aligned16(w_o) || !aligned16(out) ||
      (need > 0 && !aligned16(workspace)))
    return SCKV_ERR_ALIGNMENT;
  const int64_t m_tiles = ((int64_t)n_tokens + kQkvBM - 1) / kQkvBM;
  if (m_tiles > 65535) return SCKV_ERR_UNSUPPORTED;
  const int n_out = out_features / kHead;  // 128-column output tiles ("heads" of the fused kernel)

  const int64_t groups2 = (n_out + 1) / 2;
  const int per_split = qkv_steps_per_split(n_tokens, n_out, in_features, pool->num_sms);
  const int nk = (in_features + kQkvBK - 1) / kQkvBK;
  const int k_splits = (nk + per_split - 1) / per_split;
  const int heads = (k_splits == 1 && groups2 * m_tiles >= pool->num_sms) ? 2 : 1;
  const int n_groups = heads == 2 ? (int)groups2 : n_out;

  const bool bf16 = x_dtype == SCKV_DTYPE_BF16;
  CUtensorMap maps[5];
  int rc = encode_rows(&maps[0], x, n_tokens, in_features, bf16, kQkvBM);
  if (rc == SCKV_OK) rc = encode_rows(&maps[1], x_lo ? x_lo : x, n_tokens, in_features, bf16, kQkvBM);
  if (rc == SCKV_OK) rc = encode_rows(&maps[2], w_o, out_features, in_features, bf16, heads * kHead);
  if (rc != SCKV_OK) return rc;
  maps[3] = maps[2];  // no k / v tiles in a plain projection
  maps[4] = maps[2];
  SCKV_DEVICE_GUARD(pool->device);

  QkvParams prm{};
  prm.q_out = out;
  prm.status = pool->status;
  prm.n_tok = n_tokens;
  prm.hidden = in_features;
  prm.hq = n_out;
  prm.hkv = 0;
  prm.q_out_dtype = out_dtype;
  prm.pool_dtype = pool->kv_dtype;
  prm.plain = 1;
  prm.rope_scaling = 1.f;
  prm.k_steps_per_split = per_split;
  prm.hd_total = out_features;
  prm.k_splits = k_splits;
  prm.partial = k_splits > 1 ? reinterpret_cast<float*>(workspace) : nullptr;
  return launch_projection(prm, maps, bf16, x_lo != nullptr, k_splits, heads, n_groups, (int)m_tiles,
                           pool->num_sms, as_stream(stream));
}
