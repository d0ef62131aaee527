// Kernel 1 (scatter-append, whole-page writes) and kernel 2 (gather, CoW copy).
//
// All of these are HBM-bound byte movers: each thread moves 16-byte vectors,
// grids are sized in multiples of the SM count, and int8 / fp8 pools quantise
// in registers on the way in and dequantise on the way out.
#include "sckv_internal.cuh"

namespace {

struct Geo {
  int L, H, D;
  int64_t P;
  int dtype;
  void* data;
  void* scales;
  int32_t* status;
};

Geo geo_of(const sckv_pool* p) {
  Geo g;
  g.L = p->num_layers;
  g.H = p->num_kv_heads;
  g.D = p->head_dim;
  g.P = p->max_pages;
  g.dtype = p->kv_dtype;
  g.data = p->data;
  g.scales = p->scales;
  g.status = p->status;
  return g;
}

// Element offset of row (layer, page, kv, head, slot) in the pool.
__device__ __forceinline__ int64_t row_off(const Geo& g, int64_t layer, int64_t page, int kv, int h,
                                           int slot) {
  return ((((layer * g.P + page) * 2 + kv) * g.H + h) * SCKV_PAGE_TOKENS + slot) * (int64_t)g.D;
}

// fp8 scale index of (layer, page, kv, head).
__device__ __forceinline__ int64_t fp8_scale_idx(const Geo& g, int64_t layer, int64_t page, int kv,
                                                 int h) {
  return ((layer * g.P + page) * 2 + kv) * g.H + h;
}

// int8 scale index of (layer, page, kv, head, slot).
__device__ __forceinline__ int64_t int8_scale_idx(const Geo& g, int64_t layer, int64_t page, int kv,
                                                  int h, int slot) {
  return (((layer * g.P + page) * 2 + kv) * g.H + h) * SCKV_PAGE_TOKENS + slot;
}

// Load 8 consecutive source values as float.
__device__ __forceinline__ void load8(const void* src, int64_t idx, int dtype, float v[8]) {
  if (dtype == SCKV_DTYPE_F32) {
    const float4* p = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(src) + idx);
    float4 a = p[0], b = p[1];
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  } else {
    uint4 raw = *reinterpret_cast<const uint4*>(reinterpret_cast<const uint16_t*>(src) + idx);
    const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      if (dtype == SCKV_DTYPE_F16) {
        __half2 h2 = *reinterpret_cast<const __half2*>(&w[i]);
        float2 f = __half22float2(h2);
        v[2 * i] = f.x; v[2 * i + 1] = f.y;
      } else {
        __nv_bfloat162 b2 = *reinterpret_cast<const __nv_bfloat162*>(&w[i]);
        float2 f = __bfloat1622float2(b2);
        v[2 * i] = f.x; v[2 * i + 1] = f.y;
      }
    }
  }
}

// Store 8 floats as 16-bit dtype (16 bytes).
__device__ __forceinline__ void store8_16(void* dst, int64_t idx, int dtype, const float v[8]) {
  uint32_t w[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    if (dtype == SCKV_DTYPE_F16) {
      __half2 h2 = __floats2half2_rn(v[2 * i], v[2 * i + 1]);
      w[i] = *reinterpret_cast<uint32_t*>(&h2);
    } else {
      __nv_bfloat162 b2 = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
      w[i] = *reinterpret_cast<uint32_t*>(&b2);
    }
  }
  *reinterpret_cast<uint4*>(reinterpret_cast<uint16_t*>(dst) + idx) = make_uint4(w[0], w[1], w[2], w[3]);
}

// Find sequence b with cu[b] <= t < cu[b+1] (cu non-decreasing, cu[0] = 0).

// Resolve the destination page of (seq b, position pos); -1 on error (reported).
__device__ __forceinline__ int64_t resolve_page(const Geo& g, const int32_t* bt, int64_t stride,
                                                int max_blocks, int b, int pos, int kid) {
  if (pos < 0) { sckv_report(g.status, SCKV_ERR_BOUNDS, pos, kid); return -1; }
  int blk = pos / SCKV_PAGE_TOKENS;
  if (blk >= max_blocks) { sckv_report(g.status, SCKV_ERR_BOUNDS, blk, kid); return -1; }
  int32_t page = __ldg(bt + (int64_t)b * stride + blk);
  if (page < 0 || page >= g.P) { sckv_report(g.status, SCKV_ERR_BOUNDS, page, kid); return -1; }
  return page;
}

// ---------------------------------------------------------------------------
// Append, 16-bit pools: one block per new token. Thread 0 resolves the
// token's sequence, position and page once; the block then copies the
// token's rows of every layer, K and V and head in 16-byte chunks (the H
// rows of one (layer, K|V) are contiguous in the source, 16-token-strided
// in the page).
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) append16_kernel(Geo g, int layer0, int n_layers, const void* k_new,
                                                       const void* v_new, int src_dtype, int n_seqs, int n_tokens,
                                                       const int32_t* cu, const int32_t* start_pos, const int32_t* bt,
                                                       int64_t stride, int max_blocks) {
  __shared__ int64_t s_page;
  __shared__ int s_slot;
  const int t = blockIdx.x;
  if (threadIdx.x == 0) {
    const int b = sckv_find_seq(cu, n_seqs, t);
    const int pos = __ldg(start_pos + b) + (t - __ldg(cu + b));
    s_page = resolve_page(g, bt, stride, max_blocks, b, pos, KID_APPEND);
    s_slot = pos % SCKV_PAGE_TOKENS;
  }
  __syncthreads();
  const int64_t page = s_page;
  if (page < 0) return;
  const int slot = s_slot;
  const int cpr = g.D / 8;           // 16-byte chunks per row
  const int per_pair = g.H * cpr;    // chunks of one (layer, K|V): H rows
  const int total = n_layers * 2 * per_pair;
  for (int i = threadIdx.x; i < total; i += blockDim.x) {
    const int pair = i / per_pair, j = i - pair * per_pair;
    const int l = pair >> 1, kv = pair & 1;
    const int h = j / cpr, c = j - h * cpr;
    const void* src = kv ? v_new : k_new;
    const int64_t sidx = (((int64_t)l * n_tokens + t) * g.H) * g.D + (int64_t)j * 8;
    const int64_t didx = row_off(g, layer0 + l, page, kv, h, slot) + c * 8;
    if (src_dtype == g.dtype) {
      *reinterpret_cast<uint4*>(reinterpret_cast<uint16_t*>(g.data) + didx) =
          *reinterpret_cast<const uint4*>(reinterpret_cast<const uint16_t*>(src) + sidx);
    } else {
      float v[8];
      load8(src, sidx, src_dtype, v);
      store8_16(g.data, didx, g.dtype, v);
    }
  }
}

// ---------------------------------------------------------------------------
// int8 quantisation of one row of D values held by a warp (lane holds D/32).
// quantize_kv_int8_numpy (native/native_engine.py:207-216):
//   s = max(max|x| / 127, 1e-7) in fp32; q = clip(rint(x / s), -127, 127);
//   stored scale = fp16(s).
// ---------------------------------------------------------------------------
template <int VPL>
__device__ __forceinline__ void quant_row_int8(const float x[VPL], int8_t q[VPL], __half* s_out) {
  float m = 0.f;
#pragma unroll
  for (int i = 0; i < VPL; ++i) m = fmaxf(m, fabsf(x[i]));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  const float s = fmaxf(m / 127.0f, 1e-7f);
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    float r = rintf(x[i] / s);
    r = fminf(fmaxf(r, -127.0f), 127.0f);
    q[i] = static_cast<int8_t>(r);
  }
  *s_out = __float2half_rn(s);
}

// Append into an int8 pool: one warp per (layer, token, kv, head) row. D <= 256.
__global__ void append_int8_kernel(Geo g, int layer0, int n_layers, const void* k_new,
                                   const void* v_new, int src_dtype, int n_seqs, int n_tokens,
                                   const int32_t* cu, const int32_t* start_pos, const int32_t* bt,
                                   int64_t stride, int max_blocks) {
  const int lane = threadIdx.x & 31;
  const int64_t rows = (int64_t)n_layers * n_tokens * 2 * g.H;
  const int64_t warp0 = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  const int vpl = g.D / 32;  // values per lane (D % 32 == 0 required)
  for (int64_t r0 = warp0; r0 < rows; r0 += nwarps) {
    int64_t r = r0;
    int h = (int)(r % g.H); r /= g.H;
    int kv = (int)(r % 2); r /= 2;
    int t = (int)(r % n_tokens);
    int l = (int)(r / n_tokens);
    int b = sckv_find_seq(cu, n_seqs, t);
    int pos = __ldg(start_pos + b) + (t - __ldg(cu + b));
    int64_t page = resolve_page(g, bt, stride, max_blocks, b, pos, KID_APPEND);
    if (page < 0) continue;
    const void* src = kv ? v_new : k_new;
    int64_t sidx = (((int64_t)l * n_tokens + t) * g.H + h) * g.D;
    float x[8];
    int8_t q[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) x[i] = (i < vpl) ? sckv_load_as_float(src, sidx + lane * vpl + i, src_dtype) : 0.f;
    __half s;
    quant_row_int8<8>(x, q, &s);
    int slot = pos % SCKV_PAGE_TOKENS;
    int8_t* dst = reinterpret_cast<int8_t*>(g.data) + row_off(g, layer0 + l, page, kv, h, slot);
#pragma unroll
    for (int i = 0; i < 8; ++i)
      if (i < vpl) dst[lane * vpl + i] = q[i];
    if (lane == 0)
      reinterpret_cast<__half*>(g.scales)[int8_scale_idx(g, layer0 + l, page, kv, h, slot)] = s;
  }
}

// ---------------------------------------------------------------------------
// fp8 page-head update: one warp owns (layer, page, kv, head) and folds in
// `n_new` new rows starting at slot `slot0` (slots < slot0 hold earlier tokens).
//   s_new = max(s_old, max|x_new| / 448)   (s_old = 0 for a fresh page, slot0 == 0)
//   if s_new > s_old and slot0 > 0: old codes c -> enc(dec(c) * s_old / s_new)
//   new codes = enc(x / s_new); s_new == 0 -> codes 0.
// enc = e4m3 round-to-nearest-even with saturation; dec exact.
// ---------------------------------------------------------------------------
__device__ void fp8_page_head_update(const Geo& g, int64_t layer, int64_t page, int kv, int h,
                                     int slot0, int n_new, const void* src, int64_t src_row0,
                                     int64_t src_row_stride, int src_dtype) {
  const int lane = threadIdx.x & 31;
  float* scales = reinterpret_cast<float*>(g.scales);
  const int64_t sidx = fp8_scale_idx(g, layer, page, kv, h);
  const float s_old = (slot0 == 0) ? 0.f : scales[sidx];
  float m = 0.f;
  for (int r = 0; r < n_new; ++r)
    for (int d = lane; d < g.D; d += 32)
      m = fmaxf(m, fabsf(sckv_load_as_float(src, src_row0 + r * src_row_stride + d, src_dtype)));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  const float s_new = fmaxf(s_old, m / 448.0f);
  uint8_t* base = reinterpret_cast<uint8_t*>(g.data) + row_off(g, layer, page, kv, h, 0);
  if (s_new > s_old && slot0 > 0) {
    for (int i = lane; i < slot0 * g.D; i += 32) {
      float x = sckv_fp8_to_float(base[i]) * s_old;
      base[i] = sckv_float_to_fp8(x / s_new);
    }
  }
  for (int r = 0; r < n_new; ++r)
    for (int d = lane; d < g.D; d += 32) {
      float x = sckv_load_as_float(src, src_row0 + r * src_row_stride + d, src_dtype);
      base[(slot0 + r) * g.D + d] = (s_new > 0.f) ? sckv_float_to_fp8(x / s_new) : (uint8_t)0;
    }
  __syncwarp();
  if (lane == 0) scales[sidx] = s_new;
}

// Append into an fp8 pool: one warp per (layer, seq, kv, head), walking the
// pages the sequence's new tokens touch in order.
__global__ void append_fp8_kernel(Geo g, int layer0, int n_layers, const void* k_new,
                                  const void* v_new, int src_dtype, int n_seqs, int n_tokens,
                                  const int32_t* cu, const int32_t* start_pos, const int32_t* bt,
                                  int64_t stride, int max_blocks) {
  const int64_t units = (int64_t)n_layers * n_seqs * 2 * g.H;
  const int64_t warp0 = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t u = warp0; u < units; u += nwarps) {
    int64_t r = u;
    int h = (int)(r % g.H); r /= g.H;
    int kv = (int)(r % 2); r /= 2;
    int b = (int)(r % n_seqs);
    int l = (int)(r / n_seqs);
    const int t0 = __ldg(cu + b), t1 = __ldg(cu + b + 1);
    const int p0 = __ldg(start_pos + b);
    const void* src = kv ? v_new : k_new;
    int t = t0;
    while (t < t1) {
      const int pos = p0 + (t - t0);
      const int slot0 = pos % SCKV_PAGE_TOKENS;
      const int n_new = min(t1 - t, SCKV_PAGE_TOKENS - slot0);
      int64_t page = resolve_page(g, bt, stride, max_blocks, b, pos, KID_APPEND);
      if (page >= 0) {
        int64_t src_row0 = (((int64_t)l * n_tokens + t) * g.H + h) * g.D;
        fp8_page_head_update(g, layer0 + l, page, kv, h, slot0, n_new, src, src_row0,
                             (int64_t)g.H * g.D, src_dtype);
      }
      t += n_new;
    }
  }
}

// ---------------------------------------------------------------------------
// Whole-page writes. Source [n][L][H][16][D] (reference page without unit axis).
// ---------------------------------------------------------------------------
__global__ void write_pages16_kernel(Geo g, const int32_t* ids, int n, const void* k_src,
                                     const void* v_src, int src_dtype) {
  const int cpr = g.D / 8;
  const int64_t per_page = (int64_t)g.L * g.H * SCKV_PAGE_TOKENS * cpr;  // chunks per page per K|V
  const int64_t total = (int64_t)n * 2 * per_page;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    int64_t r = i;
    int c = (int)(r % cpr); r /= cpr;
    int slot = (int)(r % SCKV_PAGE_TOKENS); r /= SCKV_PAGE_TOKENS;
    int h = (int)(r % g.H); r /= g.H;
    int l = (int)(r % g.L); r /= g.L;
    int kv = (int)(r % 2);
    int pi = (int)(r / 2);
    int32_t page = __ldg(ids + pi);
    if (page < 0 || page >= g.P) { sckv_report(g.status, SCKV_ERR_BOUNDS, page, KID_WRITE_PAGES); continue; }
    const void* src = kv ? v_src : k_src;
    int64_t sidx = ((((int64_t)pi * g.L + l) * g.H + h) * SCKV_PAGE_TOKENS + slot) * g.D + c * 8;
    int64_t didx = row_off(g, l, page, kv, h, slot) + c * 8;
    if (src_dtype == g.dtype) {
      *reinterpret_cast<uint4*>(reinterpret_cast<uint16_t*>(g.data) + didx) =
          *reinterpret_cast<const uint4*>(reinterpret_cast<const uint16_t*>(src) + sidx);
    } else {
      float v[8];
      load8(src, sidx, src_dtype, v);
      store8_16(g.data, didx, g.dtype, v);
    }
  }
}

// int8 pool page writes: warp per (page, kv, layer, head, slot) row.
__global__ void write_pages_int8_kernel(Geo g, const int32_t* ids, int n, const void* k_src,
                                        const void* v_src, int src_dtype) {
  const int lane = threadIdx.x & 31;
  const int64_t rows = (int64_t)n * 2 * g.L * g.H * SCKV_PAGE_TOKENS;
  const int64_t warp0 = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  const int vpl = g.D / 32;
  for (int64_t r0 = warp0; r0 < rows; r0 += nwarps) {
    int64_t r = r0;
    int slot = (int)(r % SCKV_PAGE_TOKENS); r /= SCKV_PAGE_TOKENS;
    int h = (int)(r % g.H); r /= g.H;
    int l = (int)(r % g.L); r /= g.L;
    int kv = (int)(r % 2);
    int pi = (int)(r / 2);
    int32_t page = __ldg(ids + pi);
    if (page < 0 || page >= g.P) {
      if (lane == 0) sckv_report(g.status, SCKV_ERR_BOUNDS, page, KID_WRITE_PAGES);
      continue;
    }
    const void* src = kv ? v_src : k_src;
    int64_t sidx = ((((int64_t)pi * g.L + l) * g.H + h) * SCKV_PAGE_TOKENS + slot) * g.D;
    float x[8];
    int8_t q[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) x[i] = (i < vpl) ? sckv_load_as_float(src, sidx + lane * vpl + i, src_dtype) : 0.f;
    __half s;
    quant_row_int8<8>(x, q, &s);
    int8_t* dst = reinterpret_cast<int8_t*>(g.data) + row_off(g, l, page, kv, h, slot);
#pragma unroll
    for (int i = 0; i < 8; ++i)
      if (i < vpl) dst[lane * vpl + i] = q[i];
    if (lane == 0) reinterpret_cast<__half*>(g.scales)[int8_scale_idx(g, l, page, kv, h, slot)] = s;
  }
}

// fp8 pool page writes: warp per (page, kv, layer, head) page-head.
__global__ void write_pages_fp8_kernel(Geo g, const int32_t* ids, int n, const void* k_src,
                                       const void* v_src, int src_dtype) {
  const int64_t units = (int64_t)n * 2 * g.L * g.H;
  const int64_t warp0 = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t u = warp0; u < units; u += nwarps) {
    int64_t r = u;
    int h = (int)(r % g.H); r /= g.H;
    int l = (int)(r % g.L); r /= g.L;
    int kv = (int)(r % 2);
    int pi = (int)(r / 2);
    int32_t page = __ldg(ids + pi);
    if (page < 0 || page >= g.P) {
      if ((threadIdx.x & 31) == 0) sckv_report(g.status, SCKV_ERR_BOUNDS, page, KID_WRITE_PAGES);
      continue;
    }
    const void* src = kv ? v_src : k_src;
    int64_t src_row0 = (((int64_t)pi * g.L + l) * g.H + h) * SCKV_PAGE_TOKENS * g.D;
    fp8_page_head_update(g, l, page, kv, h, 0, SCKV_PAGE_TOKENS, src, src_row0, g.D, src_dtype);
  }
}

// int8 codes + fp16 scales -> int8 pool (copy) or fp16/bf16 pool (dequantise).
// Thread per element-row chunk of 16 values.
__global__ void write_pages_quantized_kernel(Geo g, const int32_t* ids, int n, const int8_t* kq,
                                             const __half* ks, const int8_t* vq, const __half* vs) {
  const int cpr = g.D / 16;
  const int64_t total = (int64_t)n * 2 * g.L * g.H * SCKV_PAGE_TOKENS * cpr;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    int64_t r = i;
    int c = (int)(r % cpr); r /= cpr;
    int slot = (int)(r % SCKV_PAGE_TOKENS); r /= SCKV_PAGE_TOKENS;
    int h = (int)(r % g.H); r /= g.H;
    int l = (int)(r % g.L); r /= g.L;
    int kv = (int)(r % 2);
    int pi = (int)(r / 2);
    int32_t page = __ldg(ids + pi);
    if (page < 0 || page >= g.P) { sckv_report(g.status, SCKV_ERR_BOUNDS, page, KID_WRITE_PAGES); continue; }
    const int8_t* qsrc = kv ? vq : kq;
    const __half* ssrc = kv ? vs : ks;
    int64_t srow = (((int64_t)pi * g.L + l) * g.H + h) * SCKV_PAGE_TOKENS + slot;
    int4 codes = *reinterpret_cast<const int4*>(qsrc + srow * g.D + c * 16);
    __half s = ssrc[srow];
    int64_t drow_elems = row_off(g, l, page, kv, h, slot);
    if (g.dtype == SCKV_DTYPE_INT8) {
      *reinterpret_cast<int4*>(reinterpret_cast<int8_t*>(g.data) + drow_elems + c * 16) = codes;
      if (c == 0) reinterpret_cast<__half*>(g.scales)[int8_scale_idx(g, l, page, kv, h, slot)] = s;
    } else {
      const int8_t* cb = reinterpret_cast<const int8_t*>(&codes);
      const float sf = __half2float(s);
      float v[8];
#pragma unroll
      for (int half = 0; half < 2; ++half) {
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          // dequantize_kv_int8_numpy (native/native_engine.py:219-221):
          // fp16(f32(q) * f32(scale)); kept at fp16 precision even for a bf16 pool.
          v[j] = __half2float(__float2half_rn(static_cast<float>(cb[half * 8 + j]) * sf));
        }
        store8_16(g.data, drow_elems + c * 16 + half * 8, g.dtype, v);
      }
    }
  }
}

// ---------------------------------------------------------------------------
// Gather: out[l][h][t][D] = pool[layer0+l][ids[t/16]][kv][h][t%16][:] (dequantised).
// Thread per 8-element chunk.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) gather_kernel(Geo g, int layer0, int n_layers, const int32_t* ids,
                                                     int n_pages, int n_tokens, void* out_k, void* out_v,
                                                     int out_dtype) {
  // one block per (page of the list, layer): the page's slab of that layer
  // ([K|V][H][16][D], contiguous) goes to rows 16 i .. 16 i + 15 of every
  // (K|V, head) plane of the output
  const int i = blockIdx.x / n_layers;
  const int l = blockIdx.x - i * n_layers;
  const int32_t page = __ldg(ids + i);
  if (page < 0 || page >= g.P) {
    if (threadIdx.x == 0) sckv_report(g.status, SCKV_ERR_BOUNDS, page, KID_GATHER);
    return;
  }
  const int cpr = g.D / 8;
  const int per_head = SCKV_PAGE_TOKENS * cpr;  // chunks of one (K|V, head): 16 rows
  const int total = 2 * g.H * per_head;
  const int64_t slab = row_off(g, layer0 + l, page, 0, 0, 0);
  for (int j = threadIdx.x; j < total; j += blockDim.x) {
    const int kh = j / per_head, r = j - kh * per_head;
    const int kv = kh / g.H, h = kh - kv * g.H;
    const int slot = r / cpr, c = r - slot * cpr;
    const int t = i * SCKV_PAGE_TOKENS + slot;
    if (t >= n_tokens) continue;
    const int64_t sidx = slab + (int64_t)j * 8;
    const int64_t didx = (((int64_t)l * g.H + h) * n_tokens + t) * g.D + c * 8;
    void* out = kv ? out_v : out_k;
    if ((g.dtype == SCKV_DTYPE_F16 || g.dtype == SCKV_DTYPE_BF16) && out_dtype == g.dtype) {
      *reinterpret_cast<uint4*>(reinterpret_cast<uint16_t*>(out) + didx) =
          *reinterpret_cast<const uint4*>(reinterpret_cast<const uint16_t*>(g.data) + sidx);
      continue;
    }
    float v[8];
    if (g.dtype == SCKV_DTYPE_F16 || g.dtype == SCKV_DTYPE_BF16) {
      load8(g.data, sidx, g.dtype, v);
    } else if (g.dtype == SCKV_DTYPE_INT8) {
      const float sf = __half2float(reinterpret_cast<const __half*>(g.scales)[int8_scale_idx(g, layer0 + l, page, kv, h, slot)]);
      uint2 raw = *reinterpret_cast<const uint2*>(reinterpret_cast<const int8_t*>(g.data) + sidx);
      const int8_t* cb = reinterpret_cast<const int8_t*>(&raw);
#pragma unroll
      for (int q = 0; q < 8; ++q) v[q] = __half2float(__float2half_rn(static_cast<float>(cb[q]) * sf));
    } else {  // fp8
      const float sf = reinterpret_cast<const float*>(g.scales)[fp8_scale_idx(g, layer0 + l, page, kv, h)];
      uint2 raw = *reinterpret_cast<const uint2*>(reinterpret_cast<const uint8_t*>(g.data) + sidx);
      const uint8_t* cb = reinterpret_cast<const uint8_t*>(&raw);
#pragma unroll
      for (int q = 0; q < 8; ++q) v[q] = sckv_fp8_to_float(cb[q]) * sf;
    }
    if (out_dtype == SCKV_DTYPE_F32) {
      float4* o = reinterpret_cast<float4*>(reinterpret_cast<float*>(out) + didx);
      o[0] = make_float4(v[0], v[1], v[2], v[3]);
      o[1] = make_float4(v[4], v[5], v[6], v[7]);
    } else {
      store8_16(out, didx, out_dtype, v);
    }
  }
}

// ---------------------------------------------------------------------------
// Copy-on-write page copy: every layer's slab (and scales) src -> dst.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) copy_pages_kernel(Geo g, const int32_t* src_ids, const int32_t* dst_ids,
                                                         int n) {
  // one block per (page pair, layer): the layer's contiguous slab, then its scales
  const int pi = blockIdx.x / g.L;
  const int l = blockIdx.x - pi * g.L;
  const int32_t s = __ldg(src_ids + pi), d = __ldg(dst_ids + pi);
  if (s < 0 || s >= g.P || d < 0 || d >= g.P) {
    if (threadIdx.x == 0) sckv_report(g.status, SCKV_ERR_BOUNDS, (s < 0 || s >= g.P) ? s : d, KID_COPY);
    return;
  }
  const int64_t slab_bytes = 2LL * g.H * SCKV_PAGE_TOKENS * g.D * (g.dtype <= SCKV_DTYPE_BF16 ? 2 : 1);
  const int vec_per_slab = (int)(slab_bytes / 16);
  const uint4* src = reinterpret_cast<const uint4*>(reinterpret_cast<const char*>(g.data) + ((int64_t)l * g.P + s) * slab_bytes);
  uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<char*>(g.data) + ((int64_t)l * g.P + d) * slab_bytes);
  for (int v = threadIdx.x; v < vec_per_slab; v += blockDim.x) dst[v] = src[v];
  if (g.scales != nullptr) {
    if (g.dtype == SCKV_DTYPE_INT8) {
      const int per = 2 * g.H * SCKV_PAGE_TOKENS;
      const __half* ss = reinterpret_cast<const __half*>(g.scales) + ((int64_t)l * g.P + s) * per;
      __half* ds = reinterpret_cast<__half*>(g.scales) + ((int64_t)l * g.P + d) * per;
      for (int k = threadIdx.x; k < per; k += blockDim.x) ds[k] = ss[k];
    } else {
      const int per = 2 * g.H;
      const float* ss = reinterpret_cast<const float*>(g.scales) + ((int64_t)l * g.P + s) * per;
      float* ds = reinterpret_cast<float*>(g.scales) + ((int64_t)l * g.P + d) * per;
      for (int k = threadIdx.x; k < per; k += blockDim.x) ds[k] = ss[k];
    }
  }
}

int grid_for(const sckv_pool* p, int64_t work_items, int threads) {
  int64_t blocks = (work_items + threads - 1) / threads;
  int64_t cap = (int64_t)p->num_sms * 8;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  return (int)blocks;
}

bool is_src_dtype(int d) { return d == SCKV_DTYPE_F16 || d == SCKV_DTYPE_BF16 || d == SCKV_DTYPE_F32; }

// ---------------------------------------------------------------------------
// Fused attention input for new tokens: optional RMSNorm of q and k, rotary
// position embedding of both, then the K/V append (16-bit pools). Restates
// models/adapters.py:1171-1207 in the reference's operation order, in fp32:
//   rmsnorm_f32 (:1129-1132): x * (1 / sqrt(mean(x^2) + eps)) * w, over one
//     head (weights of head_dim) or the whole projection (H x head_dim);
//   apply_rope_f32 (:1134-1146): angle_i = (pos / scaling) * inv_freq[i],
//     out = [x1 cos - x2 sin, x2 cos + x1 sin] on the two halves;
//   k, v -> pool type (round to nearest even) into the token's page slot.
// The rotated q goes to q_out for the attention call. One CTA (8 warps) per
// token; a warp handles one head row of 128 values, 4 per lane: dims l and
// l + 32 of the first half and their partners in the second half, so the
// rotation needs no lane exchange.
constexpr int kRopeWarps = 8;
constexpr int kRopeMaxHeads = 256;

__device__ __forceinline__ float rope_warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// int8 pools: one warp's K or V row (4 values per lane at `dims`) stored as
// the arena stores its fp16 pages: the fp16 value, quantised per row as
// quantize_kv_int8_numpy does (native/native_engine.py:207-216).
__device__ __forceinline__ void store_row_int8(const Geo& g, int layer, int64_t page, int kv, int h, int pos,
                                               const int (&dims)[4], const float (&y)[4]) {
  float x[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) x[i] = __half2float(__float2half_rn(y[i]));
  int8_t q[4];
  __half s;
  quant_row_int8<4>(x, q, &s);
  const int64_t off = row_off(g, layer, page, kv, h, pos % SCKV_PAGE_TOKENS);
  int8_t* d = reinterpret_cast<int8_t*>(g.data);
#pragma unroll
  for (int i = 0; i < 4; ++i) d[off + dims[i]] = q[i];
  if ((threadIdx.x & 31) == 0)
    reinterpret_cast<__half*>(g.scales)[int8_scale_idx(g, layer, page, kv, h, pos % SCKV_PAGE_TOKENS)] = s;
}

__global__ void __launch_bounds__(kRopeWarps * 32) append_rope_kernel(
    Geo g, int layer, const void* q_in, void* q_out, int hq, int q_dtype, int q_out_dtype, const void* k_in,
    const void* v_in, int src_dtype, const __half* q_w, int q_norm_len, const __half* k_w, int k_norm_len,
    float eps, const float* inv_freq, float rope_scaling, int n_seqs, int n_tokens, const int32_t* cu,
    const int32_t* start_pos, const int32_t* bt, int64_t stride, int max_blocks) {
  __shared__ float ss[2 * kRopeMaxHeads];  // sum of squares per q head, then per k head
  const int t = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int D = g.D, half = D / 2;  // D == 128
  const int hk = g.H;
  const int b = sckv_find_seq(cu, n_seqs, t);
  const int pos = __ldg(start_pos + b) + (t - __ldg(cu + b));
  const int64_t page = resolve_page(g, bt, stride, max_blocks, b, pos, KID_APPEND);
  const int dims[4] = {lane, lane + 32, half + lane, half + lane + 32};
  // pass 1: sums of squares of every q and k head row
  for (int r = warp; r < hq + hk; r += kRopeWarps) {
    const bool isq = r < hq;
    const int64_t base = isq ? ((int64_t)t * hq + r) * D : ((int64_t)t * hk + (r - hq)) * D;
    float a = 0.f;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float x = sckv_load_as_float(isq ? q_in : k_in, base + dims[i], isq ? q_dtype : src_dtype);
      a = fmaf(x, x, a);
    }
    a = rope_warp_sum(a);
    if (lane == 0) ss[isq ? r : kRopeMaxHeads + (r - hq)] = a;
  }
  __syncthreads();
  float q_full = 0.f, k_full = 0.f;
  if (q_norm_len == hq * D && q_norm_len != D)
    for (int h = 0; h < hq; ++h) q_full += ss[h];
  if (k_norm_len == hk * D && k_norm_len != D)
    for (int h = 0; h < hk; ++h) k_full += ss[kRopeMaxHeads + h];
  const float fpos = __fdiv_rn((float)pos, rope_scaling);
  float cs[2], sn[2];
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const float ang = __fmul_rn(fpos, __ldg(inv_freq + dims[i]));
    sincosf(ang, &sn[i], &cs[i]);
  }
  // pass 2: normalise, rotate, store
  for (int r = warp; r < hq + hk; r += kRopeWarps) {
    const bool isq = r < hq;
    const int h = isq ? r : r - hq;
    const int64_t base = isq ? ((int64_t)t * hq + h) * D : ((int64_t)t * hk + h) * D;
    const int nlen = isq ? q_norm_len : k_norm_len;
    const __half* w = isq ? q_w : k_w;
    float x[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) x[i] = sckv_load_as_float(isq ? q_in : k_in, base + dims[i], isq ? q_dtype : src_dtype);
    if (nlen != 0) {
      const bool per_head = nlen == D;
      const float sum = per_head ? ss[isq ? h : kRopeMaxHeads + h] : (isq ? q_full : k_full);
      const float var = __fdiv_rn(sum, (float)nlen);
      const float inv = __fdiv_rn(1.f, __fsqrt_rn(__fadd_rn(var, eps)));
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int wi = per_head ? dims[i] : h * D + dims[i];
        x[i] = __fmul_rn(__fmul_rn(x[i], inv), __half2float(w[wi]));
      }
    }
    float y[4];
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      y[i] = __fsub_rn(__fmul_rn(x[i], cs[i]), __fmul_rn(x[i + 2], sn[i]));
      y[i + 2] = __fadd_rn(__fmul_rn(x[i + 2], cs[i]), __fmul_rn(x[i], sn[i]));
    }
    if (isq) {
#pragma unroll
      for (int i = 0; i < 4; ++i) sckv_store_from_float(q_out, base + dims[i], q_out_dtype, y[i]);
    } else if (page >= 0) {
      if (g.dtype == SCKV_DTYPE_INT8) {
        store_row_int8(g, layer, page, 0, h, pos, dims, y);
      } else {
        const int64_t off = row_off(g, layer, page, 0, h, pos % SCKV_PAGE_TOKENS);
#pragma unroll
        for (int i = 0; i < 4; ++i) sckv_store_from_float(g.data, off + dims[i], g.dtype, y[i]);
      }
    }
  }
  // v: copied into the page as is
  if (page >= 0) {
    for (int r = warp; r < hk; r += kRopeWarps) {
      const int64_t base = ((int64_t)t * hk + r) * D;
      if (g.dtype == SCKV_DTYPE_INT8) {
        float y[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) y[i] = sckv_load_as_float(v_in, base + dims[i], src_dtype);
        store_row_int8(g, layer, page, 1, r, pos, dims, y);
        continue;
      }
      const int64_t off = row_off(g, layer, page, 1, r, pos % SCKV_PAGE_TOKENS);
#pragma unroll
      for (int i = 0; i < 4; ++i)
        sckv_store_from_float(g.data, off + dims[i], g.dtype, sckv_load_as_float(v_in, base + dims[i], src_dtype));
    }
  }
}

}  // namespace

extern "C" int sckv_append(sckv_pool* p, int layer0, int n_layers, const void* k_new, const void* v_new,
                           int src_dtype, int n_seqs, int n_tokens, const int32_t* cu_tokens,
                           const int32_t* start_pos, const int32_t* block_table, int64_t bt_stride,
                           int max_blocks, void* stream) {
  if (p == nullptr || !is_src_dtype(src_dtype)) return SCKV_ERR_INVALID_ARG;
  if (layer0 < 0 || n_layers <= 0 || layer0 + n_layers > p->num_layers) return SCKV_ERR_INVALID_ARG;
  if (n_seqs < 0 || n_tokens < 0) return SCKV_ERR_INVALID_ARG;
  if (n_seqs == 0 || n_tokens == 0) return SCKV_OK;
  if (!k_new || !v_new || !cu_tokens || !start_pos || !block_table || bt_stride < max_blocks || max_blocks <= 0)
    return SCKV_ERR_INVALID_ARG;
  if ((reinterpret_cast<uintptr_t>(k_new) | reinterpret_cast<uintptr_t>(v_new)) & 15) return SCKV_ERR_ALIGNMENT;
  Geo g = geo_of(p);
  cudaStream_t s = as_stream(stream);
  SCKV_DEVICE_GUARD(p->device);
  if (p->kv_dtype == SCKV_DTYPE_F16 || p->kv_dtype == SCKV_DTYPE_BF16) {
    // one block per new token
    append16_kernel<<<n_tokens, 256, 0, s>>>(g, layer0, n_layers, k_new, v_new, src_dtype, n_seqs,
                                                           n_tokens, cu_tokens, start_pos, block_table, bt_stride,
                                                           max_blocks);
  } else if (p->kv_dtype == SCKV_DTYPE_INT8) {
    if (p->head_dim % 32 != 0) return SCKV_ERR_UNSUPPORTED;
    int64_t work = (int64_t)n_layers * n_tokens * 2 * p->num_kv_heads * 32;
    append_int8_kernel<<<grid_for(p, work, 256), 256, 0, s>>>(g, layer0, n_layers, k_new, v_new, src_dtype, n_seqs,
                                                              n_tokens, cu_tokens, start_pos, block_table, bt_stride,
                                                              max_blocks);
  } else {
    int64_t work = (int64_t)n_layers * n_seqs * 2 * p->num_kv_heads * 32;
    append_fp8_kernel<<<grid_for(p, work, 256), 256, 0, s>>>(g, layer0, n_layers, k_new, v_new, src_dtype, n_seqs,
                                                             n_tokens, cu_tokens, start_pos, block_table, bt_stride,
                                                             max_blocks);
  }
  SCKV_LAUNCH_CHECK();
  return SCKV_OK;
}

extern "C" int sckv_write_pages(sckv_pool* p, const int32_t* ids, int n, const void* k_src, const void* v_src,
                                int src_dtype, void* stream) {
  if (p == nullptr || !is_src_dtype(src_dtype) || n < 0) return SCKV_ERR_INVALID_ARG;
  if (n == 0) return SCKV_OK;
  if (!ids || !k_src || !v_src) return SCKV_ERR_INVALID_ARG;
  if ((reinterpret_cast<uintptr_t>(k_src) | reinterpret_cast<uintptr_t>(v_src)) & 15) return SCKV_ERR_ALIGNMENT;
  Geo g = geo_of(p);
  cudaStream_t s = as_stream(stream);
  SCKV_DEVICE_GUARD(p->device);
  if (p->kv_dtype == SCKV_DTYPE_F16 || p->kv_dtype == SCKV_DTYPE_BF16) {
    int64_t work = (int64_t)n * 2 * p->num_layers * p->num_kv_heads * SCKV_PAGE_TOKENS * (p->head_dim / 8);
    write_pages16_kernel<<<grid_for(p, work, 256), 256, 0, s>>>(g, ids, n, k_src, v_src, src_dtype);
  } else if (p->kv_dtype == SCKV_DTYPE_INT8) {
    if (p->head_dim % 32 != 0) return SCKV_ERR_UNSUPPORTED;
    int64_t work = (int64_t)n * 2 * p->num_layers * p->num_kv_heads * SCKV_PAGE_TOKENS * 32;
    write_pages_int8_kernel<<<grid_for(p, work, 256), 256, 0, s>>>(g, ids, n, k_src, v_src, src_dtype);
  } else {
    int64_t work = (int64_t)n * 2 * p->num_layers * p->num_kv_heads * 32;
    write_pages_fp8_kernel<<<grid_for(p, work, 256), 256, 0, s>>>(g, ids, n, k_src, v_src, src_dtype);
  }
  SCKV_LAUNCH_CHECK();
  return SCKV_OK;
}

extern "C" int sckv_write_pages_quantized(sckv_pool* p, const int32_t* ids, int n, const int8_t* kq, const void* ks,
                                          const int8_t* vq, const void* vs, void* stream) {
  if (p == nullptr || n < 0) return SCKV_ERR_INVALID_ARG;
  if (n == 0) return SCKV_OK;
  if (!ids || !kq || !ks || !vq || !vs) return SCKV_ERR_INVALID_ARG;
  if (p->kv_dtype != SCKV_DTYPE_INT8 && p->kv_dtype != SCKV_DTYPE_F16 && p->kv_dtype != SCKV_DTYPE_BF16)
    return SCKV_ERR_UNSUPPORTED;
  if ((reinterpret_cast<uintptr_t>(kq) | reinterpret_cast<uintptr_t>(vq)) & 15) return SCKV_ERR_ALIGNMENT;
  Geo g = geo_of(p);
  SCKV_DEVICE_GUARD(p->device);
  int64_t work = (int64_t)n * 2 * p->num_layers * p->num_kv_heads * SCKV_PAGE_TOKENS * (p->head_dim / 16);
  write_pages_quantized_kernel<<<grid_for(p, work, 256), 256, 0, as_stream(stream)>>>(
      g, ids, n, kq, reinterpret_cast<const __half*>(ks), vq, reinterpret_cast<const __half*>(vs));
  SCKV_LAUNCH_CHECK();
  return SCKV_OK;
}

extern "C" int sckv_gather(sckv_pool* p, int layer0, int n_layers, const int32_t* ids, int n_pages, int n_tokens,
                           void* out_k, void* out_v, int out_dtype, void* stream) {
  if (p == nullptr || !is_src_dtype(out_dtype)) return SCKV_ERR_INVALID_ARG;
  if (layer0 < 0 || n_layers <= 0 || layer0 + n_layers > p->num_layers) return SCKV_ERR_INVALID_ARG;
  if (n_pages < 0 || n_tokens < 0 || n_tokens > n_pages * SCKV_PAGE_TOKENS) return SCKV_ERR_INVALID_ARG;
  if (n_tokens == 0) return SCKV_OK;
  if (!ids || !out_k || !out_v) return SCKV_ERR_INVALID_ARG;
  if ((reinterpret_cast<uintptr_t>(out_k) | reinterpret_cast<uintptr_t>(out_v)) & 15) return SCKV_ERR_ALIGNMENT;
  Geo g = geo_of(p);
  SCKV_DEVICE_GUARD(p->device);
  // one block per (listed page holding gathered tokens, layer)
  const int64_t blocks = (int64_t)((n_tokens + SCKV_PAGE_TOKENS - 1) / SCKV_PAGE_TOKENS) * n_layers;
  if (blocks > INT32_MAX) return SCKV_ERR_INVALID_ARG;
  gather_kernel<<<(unsigned)blocks, 256, 0, as_stream(stream)>>>(g, layer0, n_layers, ids, n_pages, n_tokens, out_k,
                                                                 out_v, out_dtype);
  SCKV_LAUNCH_CHECK();
  return SCKV_OK;
}

extern "C" int sckv_copy_pages(sckv_pool* p, const int32_t* src_ids, const int32_t* dst_ids, int n, void* stream) {
  if (p == nullptr || n < 0) return SCKV_ERR_INVALID_ARG;
  if (n == 0) return SCKV_OK;
  if (!src_ids || !dst_ids) return SCKV_ERR_INVALID_ARG;
  Geo g = geo_of(p);
  SCKV_DEVICE_GUARD(p->device);
  // one block per (page pair, layer)
  const int64_t blocks = (int64_t)n * p->num_layers;
  if (blocks > INT32_MAX) return SCKV_ERR_INVALID_ARG;
  copy_pages_kernel<<<(unsigned)blocks, 256, 0, as_stream(stream)>>>(g, src_ids, dst_ids, n);
  SCKV_LAUNCH_CHECK();
  return SCKV_OK;
}

extern "C" int sckv_append_rope(sckv_pool* p, int layer, const void* q_in, void* q_out, int num_q_heads,
                                int q_dtype, int q_out_dtype, const void* k_in, const void* v_in, int src_dtype,
                                const void* q_norm_w, int q_norm_len, const void* k_norm_w, int k_norm_len,
                                float eps, const float* inv_freq, float rope_scaling, int n_seqs, int n_tokens,
                                const int32_t* cu_tokens, const int32_t* start_pos, const int32_t* block_table,
                                int64_t bt_stride, int max_blocks, void* stream) {
  if (p == nullptr || layer < 0 || layer >= p->num_layers || n_seqs < 0 || n_tokens < 0 || num_q_heads <= 0)
    return SCKV_ERR_INVALID_ARG;
  // 16-bit and int8 pools (rows quantised as the arena does); FP8 page
  // scales span 16 tokens and go through sckv_append
  if (p->kv_dtype != SCKV_DTYPE_F16 && p->kv_dtype != SCKV_DTYPE_BF16 && p->kv_dtype != SCKV_DTYPE_INT8)
    return SCKV_ERR_UNSUPPORTED;
  if (p->head_dim != 128 || num_q_heads > kRopeMaxHeads || p->num_kv_heads > kRopeMaxHeads)
    return SCKV_ERR_UNSUPPORTED;
  if (!is_src_dtype(src_dtype) || !is_src_dtype(q_dtype) || !is_src_dtype(q_out_dtype)) return SCKV_ERR_INVALID_ARG;
  const int D = p->head_dim;
  if (q_norm_len != 0 && q_norm_len != D && q_norm_len != num_q_heads * D) return SCKV_ERR_INVALID_ARG;
  if (k_norm_len != 0 && k_norm_len != D && k_norm_len != p->num_kv_heads * D) return SCKV_ERR_INVALID_ARG;
  if ((q_norm_len && !q_norm_w) || (k_norm_len && !k_norm_w)) return SCKV_ERR_INVALID_ARG;
  if (!(rope_scaling > 0.f) || !(eps >= 0.f)) return SCKV_ERR_INVALID_ARG;
  if (n_seqs == 0 || n_tokens == 0) return SCKV_OK;
  if (!q_in || !q_out || !k_in || !v_in || !inv_freq || !cu_tokens || !start_pos || !block_table ||
      bt_stride < max_blocks || max_blocks <= 0)
    return SCKV_ERR_INVALID_ARG;
  Geo g = geo_of(p);
  SCKV_DEVICE_GUARD(p->device);
  append_rope_kernel<<<n_tokens, kRopeWarps * 32, 0, as_stream(stream)>>>(
      g, layer, q_in, q_out, num_q_heads, q_dtype, q_out_dtype, k_in, v_in, src_dtype,
      reinterpret_cast<const __half*>(q_norm_w), q_norm_len, reinterpret_cast<const __half*>(k_norm_w), k_norm_len,
      eps, inv_freq, rope_scaling, n_seqs, n_tokens, cu_tokens, start_pos, block_table, bt_stride, max_blocks);
  SCKV_LAUNCH_CHECK();
  return SCKV_OK;
}
