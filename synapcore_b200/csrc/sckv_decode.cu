// Kernels 3 + 4: paged decode attention with split-K over pages and fused
// FP8-e4m3 per-page-scale dequantisation.
//
// Math (models/adapters.py:1209-1229 restated per query token):
//   s_t = scale * q . k_t ; p = softmax(s) ; o = sum_t p_t v_t
// with q head hq reading kv head hq / G (GQA repeat, adapters.py:1211-1215).
//
// Structure (one CTA = 4 consumer warps + 1 producer warp):
//  * Work items are (split, seq, kv_head): `chunk_pages` consecutive pages of
//    one sequence's block table for one kv head and all G query heads that
//    read it. CTAs take items round-robin (persistent grid).
//  * The producer lane streams page-heads (K 16xD and V 16xD, each one
//    contiguous run in the pool) into an S-stage shared-memory ring with
//    cp.async.bulk; a full/empty mbarrier pair per stage orders the ring.
//  * Consumer warp w takes pages w, w+4, ... of the item. Lane (half, c)
//    holds head dims 8c..8c+7 of tokens half, half+2, ..., half+14; q.k
//    partials are reduce-scattered across the 16 lanes of a half (8
//    shuffles per query row), online softmax uses a warp-uniform running
//    max, and probabilities are broadcast back with 8 shuffles.
//  * At item end the 4 warps merge (m, l, acc) through shared memory; an
//    unsplit sequence writes its output, a split one writes an unnormalised
//    partial that `combine_kernel` merges.
//  * Every mbarrier wait is bounded (SCKV_WAIT_LIMIT_NS); on expiry the CTA
//    records SCKV_ERR_TIMEOUT, stops issuing, drains copies in flight and
//    returns. Invalid page ids are recorded (SCKV_ERR_BOUNDS) and page 0 is
//    read in their place so the ring stays consistent.
#include <cuda.h>
#include <math.h>
#include <stdlib.h>
#include <string.h>

#include <mutex>

#include "sckv_decode_common.cuh"

using namespace sckv_detail;

namespace {

template <int KVDT>
struct KV;
template <>
struct KV<SCKV_DTYPE_F16> {
  static constexpr int kBytes = 2;
  __device__ static __forceinline__ void load8(const uint8_t* p, float f[8]) {
    uint4 r = *reinterpret_cast<const uint4*>(p);
    const uint32_t w[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float2 v = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
      f[2 * i] = v.x; f[2 * i + 1] = v.y;
    }
  }
};
template <>
struct KV<SCKV_DTYPE_BF16> {
  static constexpr int kBytes = 2;
  __device__ static __forceinline__ void load8(const uint8_t* p, float f[8]) {
    uint4 r = *reinterpret_cast<const uint4*>(p);
    const uint32_t w[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float2 v = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w[i]));
      f[2 * i] = v.x; f[2 * i + 1] = v.y;
    }
  }
};
template <>
struct KV<SCKV_DTYPE_FP8_E4M3> {
  static constexpr int kBytes = 1;
  __device__ static __forceinline__ void load8(const uint8_t* p, float f[8]) {
    uint2 r = *reinterpret_cast<const uint2*>(p);
    const uint32_t w[2] = {r.x, r.y};
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      __half2_raw lo = __nv_cvt_fp8x2_to_halfraw2(static_cast<__nv_fp8x2_storage_t>(w[i] & 0xffffu), __NV_E4M3);
      __half2_raw hi = __nv_cvt_fp8x2_to_halfraw2(static_cast<__nv_fp8x2_storage_t>(w[i] >> 16), __NV_E4M3);
      float2 a = __half22float2(__half2(lo));
      float2 b = __half22float2(__half2(hi));
      f[4 * i] = a.x; f[4 * i + 1] = a.y; f[4 * i + 2] = b.x; f[4 * i + 3] = b.y;
    }
  }
};

// int8 codes of the arena's quant mode; the per-token fp16 scales are applied
// to the score (K) and the probability (V), not to each element.
template <>
struct KV<SCKV_DTYPE_INT8> {
  static constexpr int kBytes = 1;
  __device__ static __forceinline__ void load8(const uint8_t* p, float f[8]) {
    uint2 r = *reinterpret_cast<const uint2*>(p);
    const uint32_t w[2] = {r.x, r.y};
#pragma unroll
    for (int i = 0; i < 2; ++i)
#pragma unroll
      for (int b = 0; b < 4; ++b) f[4 * i + b] = (float)(int8_t)((w[i] >> (8 * b)) & 0xffu);
  }
};

// Reduce-scatter 8 partial sums over the 16 lanes of a half-warp: afterwards
// lane c holds the full sum of element c >> 1.
__device__ __forceinline__ float reduce_scatter8(const float v[8], int c) {
  float a[4];
  const bool u3 = c & 8;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    float send = u3 ? v[j] : v[j + 4];
    float keep = u3 ? v[j + 4] : v[j];
    a[j] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
  }
  float b2[2];
  const bool u2 = c & 4;
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    float send = u2 ? a[j] : a[j + 2];
    float keep = u2 ? a[j + 2] : a[j];
    b2[j] = keep + __shfl_xor_sync(0xffffffffu, send, 4);
  }
  const bool u1 = c & 2;
  float send = u1 ? b2[0] : b2[1];
  float r = (u1 ? b2[1] : b2[0]) + __shfl_xor_sync(0xffffffffu, send, 2);
  r += __shfl_xor_sync(0xffffffffu, r, 1);
  return r;
}

template <int G, int KVDT, int S>
struct Smem {
  // page i -> warp i % kConsumerWarps and ring slot i % S: S a multiple of the
  // warp count keeps every use of a slot with one warp (see the phase-parity
  // wait in the consumer loop)
  static_assert(S % kConsumerWarps == 0, "ring depth must be a multiple of the consumer warps");
  static constexpr int kPH = SCKV_PAGE_TOKENS * kHD * KV<KVDT>::kBytes;  // bytes of one page-head
  // int8 stages also carry the page-head's 16 K and 16 V token scales (fp16)
  static constexpr int kTokScaleBytes = (KVDT == SCKV_DTYPE_INT8) ? SCKV_PAGE_TOKENS * 2 : 0;
  static constexpr int kStageBytes = 2 * kPH + 2 * kTokScaleBytes;
  static constexpr int kRingBytes = S * kStageBytes;
  static constexpr int kRedFloats = kConsumerWarps * G * (kHD + 2);
  static constexpr int kBytes = kRingBytes + 2 * S * 8 + kRedFloats * 4 + 16;
};

template <int G, int KVDT, int S>
__global__ void __launch_bounds__(kThreads, (G <= 2 ? 3 : (G == 4 ? 2 : 1)))
    decode_kernel(const DecodeParams p) {
  using SM = Smem<G, KVDT, S>;
  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t* ring = smem;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + SM::kRingBytes);
  uint64_t* empty = full + S;
  float* red = reinterpret_cast<float*>(empty + S);  // [warp][g][HD] then m,l
  volatile int* abort_flag = reinterpret_cast<volatile int*>(red + SM::kRedFloats);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int i = 0; i < S; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();

  const int per_split = p.n_seqs * p.hkv;
  const int n_items = per_split * p.max_splits;
  const int64_t layer_base = (int64_t)p.layer * p.max_pages;
  const int64_t slab_bytes = (int64_t)2 * p.hkv * SM::kPH;

  if (warp == kConsumerWarps) {
    // ------------------------------------------------------------ producer
    if (lane != 0) return;
    uint32_t gcount = 0;
    bool aborted = false;
    for (int item = blockIdx.x; item < n_items && !aborted; item += gridDim.x) {
      const int split = item / per_split;
      const int rem = item - split * per_split;
      const int b = rem / p.hkv;
      const int h = rem - b * p.hkv;
      const int ctx = clamp_ctx(p, b, split == 0 && h == 0);
      const int npages = (ctx + SCKV_PAGE_TOKENS - 1) / SCKV_PAGE_TOKENS;
      const int j0 = split * p.chunk_pages;
      if (j0 >= npages) continue;
      const int j1 = min(npages, j0 + p.chunk_pages);
      const int32_t* bt_row = p.block_table + (int64_t)b * p.bt_stride;
      for (int j = j0; j < j1; ++j) {
        const uint32_t st = gcount % S;
        if (gcount >= S) {
          if (!mbar_wait_bounded(&empty[st], ((gcount / S) - 1) & 1, SCKV_WAIT_LIMIT_NS) || *abort_flag) {
            if (!*abort_flag) sckv_report(p.status, SCKV_ERR_TIMEOUT, item, KID_DECODE);
            *abort_flag = 1;
            aborted = true;
            break;
          }
        }
        int32_t page = __ldg(bt_row + j);
        if (page < 0 || page >= p.max_pages) {
          sckv_report(p.status, SCKV_ERR_BOUNDS, page, KID_DECODE);
          page = 0;
        }
        const uint8_t* src = p.pool + (layer_base + page) * slab_bytes + (int64_t)h * SM::kPH;
        uint8_t* dst = ring + st * SM::kStageBytes;
        mbar_arrive_expect_tx(&full[st], SM::kStageBytes);
        bulk_g2s(dst, src, SM::kPH, &full[st]);
        bulk_g2s(dst + SM::kPH, src + (int64_t)p.hkv * SM::kPH, SM::kPH, &full[st]);
        if (KVDT == SCKV_DTYPE_INT8) {
          // scales [layer][page][K|V][head][16 tokens] fp16: 32 bytes per page-head
          const uint8_t* ssrc = reinterpret_cast<const uint8_t*>(p.fp8_scales) +
                                ((layer_base + page) * 2 * p.hkv + h) * SM::kTokScaleBytes;
          bulk_g2s(dst + 2 * SM::kPH, ssrc, SM::kTokScaleBytes, &full[st]);
          bulk_g2s(dst + 2 * SM::kPH + SM::kTokScaleBytes, ssrc + (int64_t)p.hkv * SM::kTokScaleBytes,
                   SM::kTokScaleBytes, &full[st]);
        }
        ++gcount;
      }
    }
    // Drain: the last min(gcount, S) issued stages must have landed before exit.
    const uint32_t first = gcount > S ? gcount - S : 0;
    for (uint32_t k = first; k < gcount; ++k) mbar_wait_bounded(&full[k % S], (k / S) & 1, SCKV_WAIT_LIMIT_NS);
    return;
  }

  // -------------------------------------------------------------- consumers
  const int hf = lane >> 4;   // token parity
  const int c = lane & 15;    // dim group: dims 8c..8c+7
  const int tok_mine = hf + 2 * (c >> 1);  // token whose score this lane holds after reduce-scatter
  uint32_t gbase = 0;
  bool aborted = false;
  for (int item = blockIdx.x; item < n_items; item += gridDim.x) {
    const int split = item / per_split;
    const int rem = item - split * per_split;
    const int b = rem / p.hkv;
    const int h = rem - b * p.hkv;
    const int ctx = clamp_ctx(p, b, false);
    const int npages = (ctx + SCKV_PAGE_TOKENS - 1) / SCKV_PAGE_TOKENS;
    const int j0 = split * p.chunk_pages;
    if (j0 >= npages) continue;
    const int j1 = min(npages, j0 + p.chunk_pages);
    const int n = j1 - j0;
    const int nsplits = (npages + p.chunk_pages - 1) / p.chunk_pages;

    float q[G][8], acc[G][8], m[G], l[G];
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const int64_t qoff = ((int64_t)b * p.hq + (int64_t)h * G + g) * kHD + c * 8;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        q[g][j] = sckv_load_as_float(p.q, qoff + j, p.q_dtype) * p.scale_log2;
        acc[g][j] = 0.f;
      }
      m[g] = -INFINITY;
      l[g] = 0.f;
    }
    const int32_t* bt_row = p.block_table + (int64_t)b * p.bt_stride;

    for (int i = warp; i < n; i += kConsumerWarps) {
      const uint32_t gi = gbase + i;
      const uint32_t st = gi % S;
      float kscale = 1.f, vscale = 1.f;
      if (KVDT == SCKV_DTYPE_FP8_E4M3) {
        int32_t page = __ldg(bt_row + j0 + i);
        if (page < 0 || page >= p.max_pages) page = 0;
        const int64_t si = ((layer_base + page) * 2) * p.hkv + h;
        kscale = __ldg(p.fp8_scales + si);
        vscale = __ldg(p.fp8_scales + si + p.hkv);
      }
      if (!aborted) {
        if (*abort_flag || !mbar_wait_bounded(&full[st], (gi / S) & 1, SCKV_WAIT_LIMIT_NS)) {
          if (lane == 0 && !*abort_flag) sckv_report(p.status, SCKV_ERR_TIMEOUT, item, KID_DECODE);
          if (lane == 0) *abort_flag = 1;
          aborted = true;
        }
      }
      bool fused = false;  // this warp stored the sequence's new token into the staged page
      if (!aborted) {
        uint8_t* sK = ring + st * SM::kStageBytes;
        const uint8_t* sV = sK + SM::kPH;
        const int nv = min(SCKV_PAGE_TOKENS, ctx - (j0 + i) * SCKV_PAGE_TOKENS);
        if constexpr (KVDT == SCKV_DTYPE_F16 || KVDT == SCKV_DTYPE_BF16) {
          int row = 0;
          const int32_t page = fused_append_page(p, b, ctx, j0 + i, &row);
          if (page >= 0) {
            // fused append: lanes 0-15 the K row, 16-31 the V row, dims 8c..8c+7
            const uint4 v = new_row8(hf ? p.v_new : p.k_new, ((int64_t)b * p.hkv + h) * kHD + c * 8, p.new_dtype, KVDT);
            const int off = row * kHD * 2 + c * 16;  // in the page-head
            *reinterpret_cast<uint4*>(sK + hf * SM::kPH + off) = v;
            uint8_t* pool = const_cast<uint8_t*>(p.pool);
            *reinterpret_cast<uint4*>(pool + (layer_base + page) * slab_bytes + ((int64_t)hf * p.hkv + h) * SM::kPH +
                                      off) = v;
            fused = true;
            __syncwarp();
          }
        }
        if (KVDT == SCKV_DTYPE_INT8) {
          // this lane's score and probability belong to token tok_mine
          const __half* ts = reinterpret_cast<const __half*>(sK + 2 * SM::kPH);
          kscale = __half2float(ts[tok_mine]);
          vscale = __half2float(ts[SCKV_PAGE_TOKENS + tok_mine]);
        }

        float part[G][8];
#pragma unroll
        for (int t = 0; t < 8; ++t) {
          float kf[8];
          KV<KVDT>::load8(sK + ((hf + 2 * t) * kHD + c * 8) * KV<KVDT>::kBytes, kf);
#pragma unroll
          for (int g = 0; g < G; ++g) {
            float d = 0.f;
#pragma unroll
            for (int j = 0; j < 8; ++j) d = fmaf(q[g][j], kf[j], d);
            part[g][t] = d;
          }
        }
        float pv[G], alpha[G];
#pragma unroll
        for (int g = 0; g < G; ++g) {
          float sc = reduce_scatter8(part[g], c) * kscale;
          if (tok_mine >= nv) sc = -INFINITY;
          float mp = sc;
          mp = fmaxf(mp, __shfl_xor_sync(0xffffffffu, mp, 2));
          mp = fmaxf(mp, __shfl_xor_sync(0xffffffffu, mp, 4));
          mp = fmaxf(mp, __shfl_xor_sync(0xffffffffu, mp, 8));
          mp = fmaxf(mp, __shfl_xor_sync(0xffffffffu, mp, 16));
          const float m_new = fmaxf(m[g], mp);
          float pr;
          if (m_new == -INFINITY) {
            alpha[g] = 1.f;
            pr = 0.f;
          } else {
            alpha[g] = exp2f(m[g] - m_new);
            pr = exp2f(sc - m_new);
          }
          m[g] = m_new;
          l[g] = l[g] * alpha[g] + ((c & 1) ? 0.f : pr);
          pv[g] = pr * vscale;
        }
#pragma unroll
        for (int g = 0; g < G; ++g)
#pragma unroll
          for (int j = 0; j < 8; ++j) acc[g][j] *= alpha[g];
#pragma unroll
        for (int t = 0; t < 8; ++t) {
          const int tok = hf + 2 * t;
          float vf[8];
          KV<KVDT>::load8(sV + (tok * kHD + c * 8) * KV<KVDT>::kBytes, vf);
          if (nv < SCKV_PAGE_TOKENS && tok >= nv) {
#pragma unroll
            for (int j = 0; j < 8; ++j) vf[j] = 0.f;
          }
#pragma unroll
          for (int g = 0; g < G; ++g) {
            const float pt = __shfl_sync(0xffffffffu, pv[g], (hf << 4) | (2 * t));
#pragma unroll
            for (int j = 0; j < 8; ++j) acc[g][j] = fmaf(pt, vf[j], acc[g][j]);
          }
        }
      }
      // the slot's next bulk copy (async proxy) comes after this warp's stores
      if (fused) fence_proxy_async_shared();
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[st]);
    }
    gbase += n;

    // ---- merge the two token halves, then the four warps.
#pragma unroll
    for (int g = 0; g < G; ++g) {
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[g][j] += __shfl_xor_sync(0xffffffffu, acc[g][j], 16);
      float ls = l[g];
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) ls += __shfl_xor_sync(0xffffffffu, ls, o);
      l[g] = ls;
    }
    float* red_acc = red;                                         // [warp][g][HD]
    float* red_ml = red + kConsumerWarps * G * kHD;               // [warp][g][2]
    if (hf == 0) {
#pragma unroll
      for (int g = 0; g < G; ++g)
#pragma unroll
        for (int j = 0; j < 8; ++j) red_acc[(warp * G + g) * kHD + c * 8 + j] = acc[g][j];
    }
    if (lane == 0) {
#pragma unroll
      for (int g = 0; g < G; ++g) {
        red_ml[(warp * G + g) * 2] = m[g];
        red_ml[(warp * G + g) * 2 + 1] = l[g];
      }
    }
    named_bar_sync(1, kConsumerWarps * 32);
    const int d = threadIdx.x;  // 0..127 = head dim
#pragma unroll
    for (int g = 0; g < G; ++g) {
      float M = -INFINITY;
#pragma unroll
      for (int w = 0; w < kConsumerWarps; ++w) M = fmaxf(M, red_ml[(w * G + g) * 2]);
      float L = 0.f, O = 0.f;
      if (M != -INFINITY) {
#pragma unroll
        for (int w = 0; w < kConsumerWarps; ++w) {
          const float mw = red_ml[(w * G + g) * 2];
          if (mw == -INFINITY) continue;
          const float e = exp2f(mw - M);
          L = fmaf(red_ml[(w * G + g) * 2 + 1], e, L);
          O = fmaf(red_acc[(w * G + g) * kHD + d], e, O);
        }
      }
      const int hq = h * G + g;
      if (nsplits == 1) {
        const float o = (L > 0.f) ? O / L : 0.f;
        store_out(p, b, hq, d, o);
      } else {
        const int64_t slot = ((int64_t)b * p.hq + hq) * p.max_splits + split;
        p.part_acc[slot * kHD + d] = O;
        if (d == 0) {
          p.part_ml[slot * 2] = M;
          p.part_ml[slot * 2 + 1] = L;
        }
      }
    }
    named_bar_sync(1, kConsumerWarps * 32);
  }
}

// Merge split partials: one CTA of HD threads per (seq, q head).
__global__ void combine_kernel(const DecodeParams p) {
  const int b = blockIdx.x / p.hq;
  const int hq = blockIdx.x - b * p.hq;
  const int d = threadIdx.x;
  int ctx = __ldg(p.ctx_lens + b);
  const int cap = p.max_blocks * SCKV_PAGE_TOKENS;
  ctx = ctx < 0 ? 0 : (ctx > cap ? cap : ctx);
  const int npages = (ctx + SCKV_PAGE_TOKENS - 1) / SCKV_PAGE_TOKENS;
  const int ns = (npages + p.chunk_pages - 1) / p.chunk_pages;
  if (ns == 0) {
    store_out(p, b, hq, d, 0.f);
    return;
  }
  if (ns == 1) return;
  const int64_t base = ((int64_t)b * p.hq + hq) * p.max_splits;
  float M = -INFINITY;
  for (int s = 0; s < ns; ++s) M = fmaxf(M, p.part_ml[(base + s) * 2]);
  float L = 0.f, O = 0.f;
  if (M != -INFINITY) {
    for (int s = 0; s < ns; ++s) {
      const float ms = p.part_ml[(base + s) * 2];
      if (ms == -INFINITY) continue;
      const float e = exp2f(ms - M);
      L = fmaf(p.part_ml[(base + s) * 2 + 1], e, L);
      O = fmaf(p.part_acc[(base + s) * kHD + d], e, O);
    }
  }
  store_out(p, b, hq, d, L > 0.f ? O / L : 0.f);
}

}  // namespace

namespace sckv_detail {

// Merges split partials and writes zeros for empty sequences; runs after
// either decode kernel.
int launch_combine(const DecodeParams& prm, cudaStream_t stream) {
  combine_kernel<<<prm.n_seqs * prm.hq, kHD, 0, stream>>>(prm);
  SCKV_LAUNCH_CHECK();
  return SCKV_OK;
}

}  // namespace sckv_detail

namespace {

template <int G, int KVDT, int S>
int launch_decode(const sckv_pool* pool, const DecodeParams& prm, cudaStream_t stream) {
  using SM = Smem<G, KVDT, S>;
  auto kern = decode_kernel<G, KVDT, S>;
  static bool configured[64] = {};
  const int dev = pool->device;
  if (dev < 64 && !configured[dev]) {
    SCKV_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, SM::kBytes));
    configured[dev] = true;
  }
  int occ = 0;
  SCKV_CUDA_CHECK(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, kThreads, SM::kBytes));
  if (occ < 1) occ = 1;
  const int n_items = prm.n_seqs * prm.hkv * prm.max_splits;
  int grid = pool->num_sms * occ;
  if (grid > n_items) grid = n_items;
  if (grid < 1) grid = 1;
  kern<<<grid, kThreads, SM::kBytes, stream>>>(prm);
  SCKV_LAUNCH_CHECK();
  return launch_combine(prm, stream);
}

template <int KVDT, int S>
int dispatch_g(const sckv_pool* pool, int G, const DecodeParams& prm, cudaStream_t s) {
  switch (G) {
    case 1: return launch_decode<1, KVDT, S>(pool, prm, s);
    case 2: return launch_decode<2, KVDT, S>(pool, prm, s);
    case 4: return launch_decode<4, KVDT, S>(pool, prm, s);
    case 8: return launch_decode<8, KVDT, S>(pool, prm, s);
    default: return SCKV_ERR_UNSUPPORTED;
  }
}

// Grouped-query heads share each K/V page among G query rows: those go to
// the tensor-core kernel. A bf16 pool multiplies in bf16, so it needs bf16
// queries to keep q exact. SCKV_DECODE_KERNEL=simt|mma overrides (for
// measuring one kernel against the other).
bool use_tensor_core_path(const sckv_pool* pool, int G, int q_dtype) {
  static int forced = -2;
  if (forced == -2) {
    const char* e = getenv("SCKV_DECODE_KERNEL");
    forced = (e == nullptr) ? -1 : (strcmp(e, "mma") == 0 ? 1 : (strcmp(e, "simt") == 0 ? 0 : -1));
  }
  if (pool->kv_dtype == SCKV_DTYPE_BF16 && q_dtype != SCKV_DTYPE_BF16) return false;
  if (G > 16) return false;
  if (forced >= 0) return forced == 1;
  // one-byte pages: decoding the codes costs the same per page whatever G
  // is, and the tensor-core kernel does it with fewer instructions than the
  // CUDA-core one, so it takes MHA pools too
  if (pool->kv_dtype == SCKV_DTYPE_INT8 || pool->kv_dtype == SCKV_DTYPE_FP8_E4M3) return true;
  return G >= 2;
}

int pick_chunk(const sckv_pool* pool, int n_seqs, int max_blocks) {
  // Aim for >= 16 items per CTA slot so round-robin tails stay small,
  // with at least 16 pages (256 tokens) per item.
  const int slots = pool->num_sms * 3;
  const int64_t units = (int64_t)n_seqs * pool->num_kv_heads;
  int64_t splits = (16LL * slots + units - 1) / units;
  if (splits < 1) splits = 1;
  int chunk = (int)((max_blocks + splits - 1) / splits);
  if (chunk < 16) chunk = 16;
  if (chunk > max_blocks) chunk = max_blocks;
  return chunk;
}

}  // namespace

extern "C" size_t sckv_decode_workspace_bytes(const sckv_pool* pool, int n_seqs, int num_q_heads, int max_blocks,
                                              int chunk_pages) {
  if (pool == nullptr || n_seqs <= 0 || num_q_heads <= 0 || max_blocks <= 0) return 0;
  if (chunk_pages <= 0) chunk_pages = pick_chunk(pool, n_seqs, max_blocks);
  const int64_t splits = (max_blocks + chunk_pages - 1) / chunk_pages;
  // an unsplit launch writes its output directly and never touches partials
  if (splits <= 1) return 0;
  const int64_t slots = (int64_t)n_seqs * num_q_heads * splits;
  return (size_t)(slots * (kHD + 2) * sizeof(float));
}

namespace {

// Argument checks shared by both decode entry points, run before anything
// else so a bad call reports INVALID_ARG / UNSUPPORTED whatever its size.
int validate_decode_args(const sckv_pool* pool, int layer, const void* q, int q_dtype, int num_q_heads,
                         const int32_t* block_table, int64_t bt_stride, int max_blocks, const int32_t* ctx_lens,
                         int n_seqs, const void* out, int out_dtype) {
  if (pool == nullptr) return SCKV_ERR_INVALID_ARG;
  if (pool->head_dim != kHD) return SCKV_ERR_UNSUPPORTED;
  if (layer < 0 || layer >= pool->num_layers) return SCKV_ERR_INVALID_ARG;
  if (n_seqs <= 0 || num_q_heads <= 0 || max_blocks <= 0 || (bt_stride != 0 && bt_stride < max_blocks))
    return SCKV_ERR_INVALID_ARG;
  if (num_q_heads % pool->num_kv_heads != 0) return SCKV_ERR_INVALID_ARG;
  if (!q || !out || !block_table || !ctx_lens) return SCKV_ERR_INVALID_ARG;
  if (q_dtype != SCKV_DTYPE_F16 && q_dtype != SCKV_DTYPE_BF16 && q_dtype != SCKV_DTYPE_F32) return SCKV_ERR_INVALID_ARG;
  if (out_dtype != SCKV_DTYPE_F16 && out_dtype != SCKV_DTYPE_BF16 && out_dtype != SCKV_DTYPE_F32)
    return SCKV_ERR_INVALID_ARG;
  if (pool->device < 0) return SCKV_ERR_INVALID_ARG;
  return SCKV_OK;
}

}  // namespace

namespace {

// Where an exchange decode writes: element offset of the layer's slice in
// every rank's full-head buffer, the full head count, this rank's first head.
struct ExchangeTarget {
  const sckv_exchange* ex;
  int64_t out_off;
  int hq_total;
  int head0;
};

// New K / V rows a decode call stores before attending (sckv_decode_attn_append).
struct FusedAppend {
  const void* k;
  const void* v;
  int dtype;
};

int decode_attn_impl(sckv_pool* pool, int layer, const void* q, int q_dtype, int num_q_heads,
                     const int32_t* block_table, int64_t bt_stride, int max_blocks, const int32_t* ctx_lens,
                     int n_seqs, float scale, void* out, int out_dtype, void* workspace, size_t workspace_bytes,
                     int chunk_pages, void* stream, const ExchangeTarget* xt, const FusedAppend* fa = nullptr);

}  // namespace

extern "C" int sckv_decode_attn(sckv_pool* pool, int layer, const void* q, int q_dtype, int num_q_heads,
                                const int32_t* block_table, int64_t bt_stride, int max_blocks,
                                const int32_t* ctx_lens, int n_seqs, float scale, void* out, int out_dtype,
                                void* workspace, size_t workspace_bytes, int chunk_pages, void* stream) {
  return decode_attn_impl(pool, layer, q, q_dtype, num_q_heads, block_table, bt_stride, max_blocks, ctx_lens, n_seqs,
                          scale, out, out_dtype, workspace, workspace_bytes, chunk_pages, stream, nullptr);
}

extern "C" int sckv_decode_attn_append(sckv_pool* pool, int layer, const void* q, int q_dtype, int num_q_heads,
                                       const void* k_new, const void* v_new, int src_dtype,
                                       const int32_t* block_table, int64_t bt_stride, int max_blocks,
                                       const int32_t* ctx_lens, int n_seqs, float scale, void* out, int out_dtype,
                                       void* workspace, size_t workspace_bytes, int chunk_pages, void* stream) {
  if (pool == nullptr) return SCKV_ERR_INVALID_ARG;
  if (pool->kv_dtype != SCKV_DTYPE_F16 && pool->kv_dtype != SCKV_DTYPE_BF16) return SCKV_ERR_UNSUPPORTED;
  if (k_new == nullptr || v_new == nullptr) return SCKV_ERR_INVALID_ARG;
  if (src_dtype != SCKV_DTYPE_F16 && src_dtype != SCKV_DTYPE_BF16 && src_dtype != SCKV_DTYPE_F32)
    return SCKV_ERR_INVALID_ARG;
  if ((reinterpret_cast<uintptr_t>(k_new) | reinterpret_cast<uintptr_t>(v_new)) & 15) return SCKV_ERR_ALIGNMENT;
  const FusedAppend fa{k_new, v_new, src_dtype};
  return decode_attn_impl(pool, layer, q, q_dtype, num_q_heads, block_table, bt_stride, max_blocks, ctx_lens, n_seqs,
                          scale, out, out_dtype, workspace, workspace_bytes, chunk_pages, stream, nullptr, &fa);
}

extern "C" int sckv_decode_attn_exchange(sckv_pool* pool, sckv_exchange* ex, int layer, const void* q, int q_dtype,
                                         int num_q_heads, const void* k_new, const void* v_new, int src_dtype,
                                         const int32_t* block_table, int64_t bt_stride, int max_blocks,
                                         const int32_t* ctx_lens, int n_seqs, float scale, int out_dtype,
                                         int64_t out_offset, int num_q_heads_total, uint32_t epoch, void* workspace,
                                         size_t workspace_bytes, int chunk_pages, void* stream) {
  if (pool == nullptr || ex == nullptr || ex->device != pool->device) return SCKV_ERR_INVALID_ARG;
  for (int r = 0; r < ex->world; ++r)
    if (!ex->opened[r]) return SCKV_ERR_INVALID_ARG;  // every peer's buffers must be mapped
  const int head0 = ex->rank * num_q_heads;
  if (num_q_heads <= 0 || num_q_heads_total != ex->world * num_q_heads || out_offset < 0)
    return SCKV_ERR_INVALID_ARG;
  if ((k_new == nullptr) != (v_new == nullptr)) return SCKV_ERR_INVALID_ARG;
  if (k_new != nullptr) {
    if (pool->kv_dtype != SCKV_DTYPE_F16 && pool->kv_dtype != SCKV_DTYPE_BF16) return SCKV_ERR_UNSUPPORTED;
    if (src_dtype != SCKV_DTYPE_F16 && src_dtype != SCKV_DTYPE_BF16 && src_dtype != SCKV_DTYPE_F32)
      return SCKV_ERR_INVALID_ARG;
    if ((reinterpret_cast<uintptr_t>(k_new) | reinterpret_cast<uintptr_t>(v_new)) & 15) return SCKV_ERR_ALIGNMENT;
  }
  const size_t esz = out_dtype == SCKV_DTYPE_F32 ? 4 : 2;
  const int64_t end = out_offset + (int64_t)n_seqs * num_q_heads_total * kHD;
  if (n_seqs <= 0 || (size_t)end * esz > ex->out_bytes) return SCKV_ERR_INVALID_ARG;
  if (((out_offset * (int64_t)esz) & 15) != 0) return SCKV_ERR_ALIGNMENT;
  const ExchangeTarget xt{ex, out_offset, num_q_heads_total, head0};
  const FusedAppend fa{k_new, v_new, src_dtype};
  int rc = decode_attn_impl(pool, layer, q, q_dtype, num_q_heads, block_table, bt_stride, max_blocks, ctx_lens,
                            n_seqs, scale, ex->out, out_dtype, workspace, workspace_bytes, chunk_pages, stream, &xt,
                            k_new != nullptr ? &fa : nullptr);
  if (rc != SCKV_OK) return rc;
  SCKV_DEVICE_GUARD(pool->device);
  return launch_exchange_signal(ex, epoch, as_stream(stream));
}

namespace {

int decode_attn_impl(sckv_pool* pool, int layer, const void* q, int q_dtype, int num_q_heads,
                     const int32_t* block_table, int64_t bt_stride, int max_blocks, const int32_t* ctx_lens,
                     int n_seqs, float scale, void* out, int out_dtype, void* workspace, size_t workspace_bytes,
                     int chunk_pages, void* stream, const ExchangeTarget* xt, const FusedAppend* fa) {
  const int vrc = validate_decode_args(pool, layer, q, q_dtype, num_q_heads, block_table, bt_stride, max_blocks,
                                      ctx_lens, n_seqs, out, out_dtype);
  if (vrc != SCKV_OK) return vrc;
  if (chunk_pages <= 0) chunk_pages = pick_chunk(pool, n_seqs, max_blocks);
  const size_t need = sckv_decode_workspace_bytes(pool, n_seqs, num_q_heads, max_blocks, chunk_pages);
  if (need > 0 && (workspace == nullptr || workspace_bytes < need)) return SCKV_ERR_INVALID_ARG;
  if (reinterpret_cast<uintptr_t>(workspace) & 15) return SCKV_ERR_ALIGNMENT;

  DecodeParams prm{};
  prm.pool = reinterpret_cast<const uint8_t*>(pool->data);
  prm.fp8_scales = reinterpret_cast<const float*>(pool->scales);
  prm.q = q;
  prm.out = out;
  prm.max_splits = (max_blocks + chunk_pages - 1) / chunk_pages;
  const int64_t slots = (int64_t)n_seqs * num_q_heads * prm.max_splits;
  prm.part_acc = reinterpret_cast<float*>(workspace);
  prm.part_ml = prm.part_acc + slots * kHD;
  prm.block_table = block_table;
  prm.ctx_lens = ctx_lens;
  prm.status = pool->status;
  prm.bt_stride = bt_stride;
  prm.max_pages = pool->max_pages;
  prm.max_blocks = max_blocks;
  prm.n_seqs = n_seqs;
  prm.hq = num_q_heads;
  prm.hkv = pool->num_kv_heads;
  prm.layer = layer;
  prm.chunk_pages = chunk_pages;
  prm.q_dtype = q_dtype;
  prm.out_dtype = out_dtype;
  prm.scale_log2 = scale * 1.4426950408889634f;
  if (xt != nullptr) {
    prm.n_peer = xt->ex->world;
    for (int r = 0; r < xt->ex->world; ++r) prm.peer_out[r] = xt->ex->peer_out[r];
    prm.out_hq_total = xt->hq_total;
    prm.out_head0 = xt->head0;
    prm.out_off = xt->out_off;
  }
  if (fa != nullptr) {
    prm.k_new = fa->k;
    prm.v_new = fa->v;
    prm.new_dtype = fa->dtype;
  }
  const int G = num_q_heads / pool->num_kv_heads;
  cudaStream_t s = as_stream(stream);
  SCKV_DEVICE_GUARD(pool->device);
  if (use_tensor_core_path(pool, G, q_dtype)) {
    const int rc = launch_decode_mma(pool, G, prm, s);
    if (rc != SCKV_ERR_UNSUPPORTED) return rc;
  }
  switch (pool->kv_dtype) {
    case SCKV_DTYPE_F16: return dispatch_g<SCKV_DTYPE_F16, 8>(pool, G, prm, s);
    case SCKV_DTYPE_BF16: return dispatch_g<SCKV_DTYPE_BF16, 8>(pool, G, prm, s);
    case SCKV_DTYPE_FP8_E4M3: return dispatch_g<SCKV_DTYPE_FP8_E4M3, 16>(pool, G, prm, s);
    case SCKV_DTYPE_INT8: return dispatch_g<SCKV_DTYPE_INT8, 16>(pool, G, prm, s);
    default: return SCKV_ERR_UNSUPPORTED;
  }
}

}  // namespace

// ---------------------------------------------------------------------------
// Decode attention for callers that cannot allocate device memory.
//
// Some hosts of this library have no way to obtain scratch memory for a call:
// a serving process whose device memory is owned up front by another
// allocator (the page pool plus a fixed arena take nearly all of HBM, and a
// stray cudaMalloc would fail or stall every stream on the device), or a
// language binding that exposes only the pool handle and its own buffers.
// For them the split-K partials live in a fixed file-scope device array of
// SCKV_NOALLOC_SCRATCH_BYTES per GPU, reserved when the library's module is
// loaded on that GPU and held until the process exits.
//
// The array's name is only a host-side stand-in for the device symbol, so the
// host resolves its device address (with that device current) through
// cudaGetSymbolAddress and passes the address down; device code could name
// the array directly. The first call on a device performs that set-up, so
// make it before capturing any stream into a CUDA graph. A device reset, or
// any other teardown and re-creation of the device's primary context, loads
// the module again and moves the array; the next call sees the new context's
// id and resolves the address again (so, after a reset, again make one call
// before any capture).
//
// Every call reuses the same array and it keeps the last call's contents.
// Nothing in it needs to start at zero: each split partial a call reads is
// written earlier in the same call. Calls whose work overlaps on the GPU (two
// streams, or two host threads) race on the array; serialise them. The
// host-side set-up itself is safe to enter from several threads at once.
// ---------------------------------------------------------------------------
namespace {

constexpr size_t kNoAllocScratchBytes = SCKV_NOALLOC_SCRATCH_BYTES;
static_assert(kNoAllocScratchBytes % 256 == 0, "scratch size must keep 256-byte alignment");

static __device__ __align__(256) float g_noalloc_scratch[kNoAllocScratchBytes / sizeof(float)];

// Per device: the array's device address and the id of the context it was
// resolved in.
struct NoAllocScratchSlot {
  std::mutex mu;
  void* addr = nullptr;
  unsigned long long ctx_id = 0;
};
NoAllocScratchSlot g_noalloc_slots[64];

using CtxGetCurrentFn = CUresult (*)(CUcontext*);
using CtxGetIdFn = CUresult (*)(CUcontext, unsigned long long*);

// Unique id of the calling thread's current context; 0 when the driver cannot
// say (the address is then resolved on every call).
unsigned long long current_context_id() {
  static CtxGetCurrentFn get_current = nullptr;
  static CtxGetIdFn get_id = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_current = reinterpret_cast<CtxGetCurrentFn>(fn);
    fn = nullptr;
    if (cudaGetDriverEntryPoint("cuCtxGetId", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_id = reinterpret_cast<CtxGetIdFn>(fn);
  });
  if (get_current == nullptr || get_id == nullptr) return 0;
  CUcontext ctx = nullptr;
  if (get_current(&ctx) != CUDA_SUCCESS || ctx == nullptr) return 0;
  unsigned long long id = 0;
  if (get_id(ctx, &id) != CUDA_SUCCESS) return 0;
  return id;
}

}  // namespace

extern "C" int sckv_decode_attn_noalloc(sckv_pool* pool, int layer, const void* q, int q_dtype, int num_q_heads,
                                        const int32_t* block_table, int64_t bt_stride, int max_blocks,
                                        const int32_t* ctx_lens, int n_seqs, float scale, void* out, int out_dtype,
                                        int chunk_pages, void* stream) {
  const int vrc = validate_decode_args(pool, layer, q, q_dtype, num_q_heads, block_table, bt_stride, max_blocks,
                                      ctx_lens, n_seqs, out, out_dtype);
  if (vrc != SCKV_OK) return vrc;
  const int dev = pool->device;
  if (dev >= 64) return SCKV_ERR_INVALID_ARG;
  int chunk = chunk_pages;
  if (chunk <= 0) {
    // Default split, widened until the partials fit the fixed buffer (an
    // unsplit launch needs none).
    chunk = pick_chunk(pool, n_seqs, max_blocks);
    while (chunk < max_blocks &&
           sckv_decode_workspace_bytes(pool, n_seqs, num_q_heads, max_blocks, chunk) > kNoAllocScratchBytes)
      chunk = chunk * 2 < max_blocks ? chunk * 2 : max_blocks;
  }
  if (sckv_decode_workspace_bytes(pool, n_seqs, num_q_heads, max_blocks, chunk) > kNoAllocScratchBytes)
    return SCKV_ERR_SCRATCH_LIMIT;
  SCKV_DEVICE_GUARD(dev);
  void* scratch = nullptr;
  {
    NoAllocScratchSlot& slot = g_noalloc_slots[dev];
    std::lock_guard<std::mutex> lock(slot.mu);
    const unsigned long long id = current_context_id();
    if (slot.addr == nullptr || id == 0 || id != slot.ctx_id) {
      void* addr = nullptr;
      SCKV_CUDA_CHECK(cudaGetSymbolAddress(&addr, g_noalloc_scratch));
      slot.addr = addr;
      slot.ctx_id = id;
    }
    scratch = slot.addr;
  }
  return sckv_decode_attn(pool, layer, q, q_dtype, num_q_heads, block_table, bt_stride, max_blocks, ctx_lens, n_seqs,
                          scale, out, out_dtype, scratch, kNoAllocScratchBytes, chunk, stream);
}
