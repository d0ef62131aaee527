// Tensor-core paged decode attention for grouped-query heads.
//
// Same math, work items, pipeline and split-K partials as decode_kernel in
// sckv_decode.cu (softmax(scale q K^T) V, models/adapters.py:1209-1229), but
// the G query rows that share a kv head (GQA repeat, adapters.py:1211-1215)
// are multiplied against each 16-token page on the tensor cores:
//
//   S^T[16 tok x 8 q] = K[16 tok x 128] . Q^T[128 x 8 q]     8 x mma.m16n8k16
//   O^T[128 x 8 q]   += V^T[128 x 16 tok] . P^T[16 tok x 8 q] 8 x mma.m16n8k16
//
// with fp32 accumulation. Pages are staged by TMA tensor copies
// (cp.async.bulk.tensor.3d, 128-byte swizzle) so the 8-row fragment loads hit
// distinct banks. 16-bit pages feed ldmatrix / ldmatrix.trans directly. FP8
// pages are decoded in registers (cvt e4m3x2 -> f16x2, exact) under a fixed
// permutation of head dims and tokens that lets each lane read contiguous
// bytes; the permutation is applied to q and undone on output, so results are
// the plain dot products. S^T's accumulator fragment becomes P^T's operand
// fragment through movmatrix.trans. q rows G..7 of the tile are zero.
//
// Precision: f16 operands for f16 and FP8 pools (q converted to f16, exact
// for bf16 queries in range; P in f16); bf16 operands for bf16 pools (needs
// bf16 queries; P split into bf16 hi + lo parts so its rounding stays below
// 2^-16). Scores are scaled in fp32 after the MMA.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <math.h>

#include "sckv_decode_common.cuh"
#include "sckv_mma_common.cuh"

using namespace sckv_detail;
using namespace sckv_mma;

namespace {

// One stage = one page of HG kv heads: for each 128-byte column block of the
// head dim (1 for FP8, 2 for 16-bit), a TMA box [K|V][HG heads][16 tok][128 B]
// (128-byte swizzle); FP8 adds the page's 2*H fp32 scales.
template <int KVDT, int NQT, int HG, int S>
struct MmaSmem {
  static constexpr int kBoxes = MmaKV<KVDT>::kEB;    // column blocks of 128 bytes
  static constexpr int kBoxStride = 2 * HG * kBoxBytes;  // bytes of one column block (K and V, HG heads)
  static constexpr int kStageBytes = kBoxes * kBoxStride;
  static constexpr int kRingBytes = S * kStageBytes;
  static constexpr int kG = 8 * NQT;                 // q rows per tile
  static constexpr int kRedFloats = kConsumerWarps * kG * (kHD + 2);
  static constexpr int kScaleSlot = 64;              // FP8: floats per stage (2*H <= 64)
  static constexpr int kTokScaleSlot = 2 * HG * SCKV_PAGE_TOKENS;  // int8: halfs per stage (K, V of HG heads)
  static constexpr int kScaleBytes = (KVDT == SCKV_DTYPE_FP8_E4M3) ? S * kScaleSlot * 4
                                     : (KVDT == SCKV_DTYPE_INT8) ? S * kTokScaleSlot * 2 : 0;
  static constexpr int kBytes = 1024 + kRingBytes + kScaleBytes + 2 * S * 8 + kRedFloats * 4 + 16;
};

// Resident CTAs per SM the launch bounds promise: three when the ring and
// reduction area fit three CTAs' shared memory, else two.
template <int KVDT, int NQT, int HG, int S>
constexpr int mma_min_blocks() {
  return MmaSmem<KVDT, NQT, HG, S>::kBytes <= 74 * 1024 ? 3 : 2;
}

template <int KVDT, int NQT, int HG, int S>
__global__ void __launch_bounds__(kThreads, (mma_min_blocks<KVDT, NQT, HG, S>()))
    decode_mma_kernel(const DecodeParams p, const __grid_constant__ CUtensorMap tmap) {
  using SM = MmaSmem<KVDT, NQT, HG, S>;
  constexpr bool kBF16 = (KVDT == SCKV_DTYPE_BF16);
  constexpr bool kFP8 = (KVDT == SCKV_DTYPE_FP8_E4M3);
  constexpr bool kINT8 = (KVDT == SCKV_DTYPE_INT8);
  constexpr bool kB8 = kFP8 || kINT8;  // one-byte codes, decoded in registers
  constexpr int kG = SM::kG;
  constexpr int kWPH = kConsumerWarps / HG;  // consumer warps per head
  // Pages go to the kWPH warps of a head in turn (page i -> warp i % kWPH) and
  // page i lands in ring slot i % S. With S a multiple of kWPH every use of a
  // slot belongs to the same warps, so a warp waiting for a slot has consumed
  // the slot's previous use and the phase-parity wait cannot be satisfied by
  // an older phase of the same parity.
  static_assert(S % kWPH == 0, "ring depth must be a multiple of the warps per head");
  extern __shared__ __align__(16) uint8_t smem_raw[];
  // swizzled TMA destinations need 1024-byte alignment
  uint8_t* ring = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float* sscale = reinterpret_cast<float*>(ring + SM::kRingBytes);  // FP8 [S][kScaleSlot]: K scales of all heads, then V
  // int8 [S][K|V][HG][16]: per-token fp16 scales of this group's heads
  const __half* stok = reinterpret_cast<const __half*>(ring + SM::kRingBytes);
  uint64_t* full = reinterpret_cast<uint64_t*>(ring + SM::kRingBytes + SM::kScaleBytes);
  uint64_t* empty = full + S;
  float* red = reinterpret_cast<float*>(empty + S);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(red + SM::kRedFloats);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int i = 0; i < S; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], HG);  // one consumer warp per head reads each stage
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();

  const int G = p.hq / p.hkv;
  const int n_groups = p.hkv / HG;
  const int per_split = p.n_seqs * n_groups;
  const int n_items = per_split * p.max_splits;
  const int64_t layer_base = (int64_t)p.layer * p.max_pages;

  if (warp == kConsumerWarps) {
    // ------------------------------------------------------------ producer
    if (lane != 0) return;
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmap)) : "memory");
    uint32_t gcount = 0;
    bool aborted = false;
    const uint32_t tx = SM::kStageBytes + (kFP8 ? 8 * p.hkv : 0) + (kINT8 ? SM::kTokScaleSlot * 2 : 0);
    for (int item = blockIdx.x; item < n_items && !aborted; item += gridDim.x) {
      const int split = item / per_split;
      const int rem = item - split * per_split;
      const int b = rem / n_groups;
      const int h0 = (rem - b * n_groups) * HG;
      const int ctx = clamp_ctx(p, b, split == 0 && h0 == 0);
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
        if (((j - j0) & 7) == 0 && j + 16 < j1)
          asm volatile("prefetch.global.L2 [%0];" ::"l"(bt_row + j + 16));
        int32_t page = __ldg(bt_row + j);
        if (page < 0 || page >= p.max_pages) {
          sckv_report(p.status, SCKV_ERR_BOUNDS, page, KID_DECODE);
          page = 0;
        }
        const int slab = (int)(layer_base + page);
        const uint32_t dst = smem_u32(ring + st * SM::kStageBytes);
        mbar_arrive_expect_tx(&full[st], tx);
        if (kFP8)  // K and V scales of every head of this (layer, page): 8*H contiguous bytes
          bulk_g2s(sscale + st * SM::kScaleSlot, p.fp8_scales + (int64_t)slab * 2 * p.hkv, 8 * p.hkv, &full[st]);
        if (kINT8) {
          // scales [layer][page][K|V][head][16 tokens] fp16: the group's HG heads are 32 * HG
          // contiguous bytes for K and again for V
          const uint8_t* sb = reinterpret_cast<const uint8_t*>(p.fp8_scales);
          uint8_t* sd = ring + SM::kRingBytes + st * SM::kTokScaleSlot * 2;
          bulk_g2s(sd, sb + ((int64_t)slab * 2 * p.hkv + h0) * 32, HG * 32, &full[st]);
          bulk_g2s(sd + HG * 32, sb + (((int64_t)slab * 2 + 1) * p.hkv + h0) * 32, HG * 32, &full[st]);
        }
#pragma unroll
        for (int bx = 0; bx < SM::kBoxes; ++bx)
          tma_load_5d(dst + bx * SM::kBoxStride, &tmap, bx * (128 / MmaKV<KVDT>::kEB), 0, h0, 0, slab, &full[st]);
        ++gcount;
      }
    }
    const uint32_t first = gcount > S ? gcount - S : 0;
    for (uint32_t k = first; k < gcount; ++k) mbar_wait_bounded(&full[k % S], (k / S) & 1, SCKV_WAIT_LIMIT_NS);
    return;
  }

  // -------------------------------------------------------------- consumers
  const int g = lane >> 2;  // fragment row group
  const int t = lane & 3;   // thread in group
  const int hg = warp / kWPH;   // head of the group this warp works on
  const int sub = warp % kWPH;  // its share of the pages
  uint32_t gbase = 0;
  bool aborted = false;
  for (int item = blockIdx.x; item < n_items; item += gridDim.x) {
    const int split = item / per_split;
    const int rem = item - split * per_split;
    const int b = rem / n_groups;
    const int h0 = (rem - b * n_groups) * HG;
    const int h = h0 + hg;
    const int ctx = clamp_ctx(p, b, false);
    const int npages = (ctx + SCKV_PAGE_TOKENS - 1) / SCKV_PAGE_TOKENS;
    const int j0 = split * p.chunk_pages;
    if (j0 >= npages) continue;
    const int j1 = min(npages, j0 + p.chunk_pages);
    const int n = j1 - j0;
    const int nsplits = (npages + p.chunk_pages - 1) / p.chunk_pages;

    // q^T fragments (B operand of S^T = K Q^T): rows 8nq+g of this kv head's q block.
    uint32_t qf[NQT][8][2];
#pragma unroll
    for (int nq = 0; nq < NQT; ++nq) {
      const int qr = 8 * nq + g;
      const int64_t qoff = ((int64_t)b * p.hq + (int64_t)h * G + qr) * kHD;
#pragma unroll
      for (int s = 0; s < 8; ++s) {
        const int d0 = kB8 ? 16 * s + 4 * t : 16 * s + 2 * t;
        const int d1 = kB8 ? d0 + 2 : d0 + 8;
        float v0 = 0.f, v1 = 0.f, v2 = 0.f, v3 = 0.f;
        if (qr < G) {
          v0 = sckv_load_as_float(p.q, qoff + d0, p.q_dtype);
          v1 = sckv_load_as_float(p.q, qoff + d0 + 1, p.q_dtype);
          v2 = sckv_load_as_float(p.q, qoff + d1, p.q_dtype);
          v3 = sckv_load_as_float(p.q, qoff + d1 + 1, p.q_dtype);
        }
        qf[nq][s][0] = pack2<kBF16>(v0, v1);
        qf[nq][s][1] = pack2<kBF16>(v2, v3);
      }
    }
    // int8: K codes enter the score MMAs offset by +1152 (cvt_b8x4_biased),
    // so a score row carries 1152 * sum_d q[d] extra, removed per page below
    // (one page's 128-dim dot product: no precision issue). V codes stay
    // exact: an offset there would grow with the context inside the
    // tensor-core accumulator.
    float qcorr[NQT][2];
#pragma unroll
    for (int nq = 0; nq < NQT; ++nq) {
      qcorr[nq][0] = qcorr[nq][1] = 0.f;
      if (kINT8) {
        float part = 0.f;  // this lane's 32 dims of q row 8 nq + g, as the MMA sees them (f16)
#pragma unroll
        for (int s = 0; s < 8; ++s) {
#pragma unroll
          for (int r2 = 0; r2 < 2; ++r2) {
            const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&qf[nq][s][r2]));
            part += f.x + f.y;
          }
        }
        part += __shfl_xor_sync(0xffffffffu, part, 1);
        part += __shfl_xor_sync(0xffffffffu, part, 2);
        // score columns of this lane are q rows 2t and 2t + 1 (held by lanes 4 (2t + c))
#pragma unroll
        for (int c = 0; c < 2; ++c) qcorr[nq][c] = 1152.f * __shfl_sync(0xffffffffu, part, 4 * (2 * t + c));
      }
    }
    float acc[NQT][8][4];
    float m[NQT][2], l[NQT][2];
#pragma unroll
    for (int nq = 0; nq < NQT; ++nq) {
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int c = 0; c < 4; ++c) acc[nq][i][c] = 0.f;
      m[nq][0] = m[nq][1] = -INFINITY;
      l[nq][0] = l[nq][1] = 0.f;
    }
    float vref = 0.f;      // FP8: reference V scale of this warp's accumulator
    float inv_vref = 0.f;  // 1 / vref (0 while vref is 0)

    for (int i = sub; i < n; i += kWPH) {
      const uint32_t gi = gbase + i;
      const uint32_t st = gi % S;
      float kscale = 1.f, vscale = 1.f;
      if (!aborted) {
        if (*abort_flag || !mbar_wait_bounded(&full[st], (gi / S) & 1, SCKV_WAIT_LIMIT_NS)) {
          if (lane == 0 && !*abort_flag) sckv_report(p.status, SCKV_ERR_TIMEOUT, item, KID_DECODE);
          if (lane == 0) *abort_flag = 1;
          aborted = true;
        }
      }
      bool fused = false;  // this warp stored its head's new token into the staged page
      if (!aborted) {
        const uint32_t stage = smem_u32(ring + st * SM::kStageBytes);
        const uint32_t sK = stage + hg * kBoxBytes;         // K of head hg, column block 0
        const uint32_t sV = stage + (HG + hg) * kBoxBytes;  // V of head hg, column block 0
        const int nv = min(SCKV_PAGE_TOKENS, ctx - (j0 + i) * SCKV_PAGE_TOKENS);
        if constexpr (!kB8) {
          int row = 0;
          const int32_t page = fused_append_page(p, b, ctx, j0 + i, &row);
          if (page >= 0) {
            // fused append: lane = (K|V, 64-dim column block, 16-byte chunk);
            // the staged row sits in the 128-byte swizzle (chunk ^ row % 8)
            const int kvh = lane >> 4, bx = (lane >> 3) & 1, ch = lane & 7;
            const int dim0 = bx * 64 + ch * 8;
            const uint4 v = new_row8(kvh ? p.v_new : p.k_new, ((int64_t)b * p.hkv + h) * kHD + dim0, p.new_dtype, KVDT);
            *reinterpret_cast<uint4*>(ring + st * SM::kStageBytes + bx * SM::kBoxStride + (kvh * HG + hg) * kBoxBytes +
                                      row * 128 + ((ch ^ (row & 7)) << 4)) = v;
            constexpr int64_t kPH = SCKV_PAGE_TOKENS * kHD * 2;  // bytes of one 16-bit page-head
            uint8_t* pool = const_cast<uint8_t*>(p.pool);
            *reinterpret_cast<uint4*>(pool + ((layer_base + page) * 2 * p.hkv + (int64_t)kvh * p.hkv + h) * kPH +
                                      row * kHD * 2 + dim0 * 2) = v;
            fused = true;
            __syncwarp();
          }
        }
        float ksA = 1.f, ksB = 1.f, vsA = 1.f, vsB = 1.f;  // int8: scales of tokens g, g + 8
        if (kFP8) {
          kscale = sscale[st * SM::kScaleSlot + h];
          vscale = sscale[st * SM::kScaleSlot + p.hkv + h];
        }
        if (kINT8) {
          const __half* ts = stok + st * SM::kTokScaleSlot;
          ksA = __half2float(ts[hg * SCKV_PAGE_TOKENS + g]);
          ksB = __half2float(ts[hg * SCKV_PAGE_TOKENS + g + 8]);
          vsA = __half2float(ts[(HG + hg) * SCKV_PAGE_TOKENS + g]);
          vsB = __half2float(ts[(HG + hg) * SCKV_PAGE_TOKENS + g + 8]);
        }

        // ---------------- S^T = K . Q^T (two accumulators to halve the MMA chain)
        float sc[NQT][4], sc2[NQT][4];
#pragma unroll
        for (int nq = 0; nq < NQT; ++nq)
#pragma unroll
          for (int c = 0; c < 4; ++c) sc[nq][c] = sc2[nq][c] = 0.f;
        {
          const int row = (lane & 7) + ((lane >> 3) & 1) * 8;
          if (kB8) {
#pragma unroll
            for (int c2 = 0; c2 < 4; ++c2) {
              const int chunk = 2 * c2 + (lane >> 4);
              uint32_t w0, w1, w2, w3;
              ldsm_x4(sK + row * 128 + ((chunk ^ (row & 7)) << 4), w0, w1, w2, w3);
              uint32_t a[4];
              cvt_b8x4_biased<KVDT>(w0, a[0], a[2]);
              cvt_b8x4_biased<KVDT>(w1, a[1], a[3]);
#pragma unroll
              for (int nq = 0; nq < NQT; ++nq) mma16816<false>(sc[nq], a, qf[nq][2 * c2][0], qf[nq][2 * c2][1]);
              cvt_b8x4_biased<KVDT>(w2, a[0], a[2]);
              cvt_b8x4_biased<KVDT>(w3, a[1], a[3]);
#pragma unroll
              for (int nq = 0; nq < NQT; ++nq)
                mma16816<false>(sc2[nq], a, qf[nq][2 * c2 + 1][0], qf[nq][2 * c2 + 1][1]);
            }
          } else {
#pragma unroll
            for (int s = 0; s < 8; ++s) {
              const int cb = 2 * (s & 3) + (lane >> 4);
              uint32_t a[4];
              ldsm_x4(sK + (s >> 2) * SM::kBoxStride + row * 128 + ((cb ^ (row & 7)) << 4), a[0], a[1], a[2], a[3]);
#pragma unroll
              for (int nq = 0; nq < NQT; ++nq) {
                if (s & 1) mma16816<kBF16>(sc2[nq], a, qf[nq][s][0], qf[nq][s][1]);
                else mma16816<kBF16>(sc[nq], a, qf[nq][s][0], qf[nq][s][1]);
              }
            }
          }
        }

        // ---------------- online softmax, stale running max: the reference max
        // moves only when a score exceeds it by more than 2^8, so p <= 256 and
        // the accumulator rescale is rare. Every lane tests its own scores
        // against the (column-uniform) reference; the column max over the 8
        // lanes of a q column is reduced only when some score crossed it.
        // int8: the per-token K scale multiplies its score row (tokens g, g + 8)
        const float sscaleA = p.scale_log2 * kscale * ksA;
        const float sscaleB = p.scale_log2 * kscale * ksB;
        float sv[NQT][4];
        bool grow = false;
#pragma unroll
        for (int nq = 0; nq < NQT; ++nq) {
#pragma unroll
          for (int c = 0; c < 2; ++c) {
            const float sA = (g < nv) ? (sc[nq][c] + sc2[nq][c] - qcorr[nq][c]) * sscaleA : -INFINITY;
            const float sB = (g + 8 < nv) ? (sc[nq][2 + c] + sc2[nq][2 + c] - qcorr[nq][c]) * sscaleB : -INFINITY;
            sv[nq][c] = sA;
            sv[nq][2 + c] = sB;
            grow |= (fmaxf(sA, sB) > m[nq][c] + 8.f);
          }
        }
        if (__any_sync(0xffffffffu, grow)) {
#pragma unroll
          for (int nq = 0; nq < NQT; ++nq) {
#pragma unroll
            for (int c = 0; c < 2; ++c) {
              float mx = fmaxf(sv[nq][c], sv[nq][2 + c]);
              mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
              mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
              mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
              const float mn = fmaxf(m[nq][c], mx);
              const float alpha = (mn == -INFINITY) ? 1.f : exp2f(m[nq][c] - mn);
              m[nq][c] = mn;
              l[nq][c] *= alpha;
#pragma unroll
              for (int mi = 0; mi < 8; ++mi) {
                acc[nq][mi][c] *= alpha;
                acc[nq][mi][2 + c] *= alpha;
              }
            }
          }
        }
        // FP8 V scale: folded into P relative to a per-item reference scale so
        // P stays in the normal f16 range; the accumulator is in units of vref.
        float pscale = 1.f;
        if (kFP8) {
          if (vref == 0.f) {
            vref = vscale;
            inv_vref = (vscale > 0.f) ? 1.f / vscale : 0.f;
          }
          pscale = vscale * inv_vref;
          if (pscale > 64.f) {
            const float rb = vref / vscale;
#pragma unroll
            for (int nq = 0; nq < NQT; ++nq)
#pragma unroll
              for (int mi = 0; mi < 8; ++mi)
#pragma unroll
                for (int c = 0; c < 4; ++c) acc[nq][mi][c] *= rb;
            vref = vscale;
            inv_vref = 1.f / vscale;
            pscale = 1.f;
          }
        }
        // P multipliers of rows g and g + 8: FP8 the page's V-scale ratio;
        // int8 each token's V scale over the item's reference (token 0 of
        // the first page), moved to the page's largest live scale when a
        // ratio passes 64 so P stays in f16 range; 0 for masked rows
        float pscaleA = pscale, pscaleB = pscale;
        if (kINT8) {
          const __half* tv = stok + st * SM::kTokScaleSlot + (HG + hg) * SCKV_PAGE_TOKENS;
          if (vref == 0.f) {
            const float v0 = __half2float(tv[0]);
            vref = (v0 > 0.f) ? v0 : 1.f;
            inv_vref = 1.f / vref;
          }
          pscaleA = (g < nv) ? vsA * inv_vref : 0.f;
          pscaleB = (g + 8 < nv) ? vsB * inv_vref : 0.f;
          if (__any_sync(0xffffffffu, pscaleA > 64.f || pscaleB > 64.f)) {
            float vmax = 0.f;
            for (int i = 0; i < nv; ++i) vmax = fmaxf(vmax, __half2float(tv[i]));
            const float rb = vref / vmax;
#pragma unroll
            for (int nq = 0; nq < NQT; ++nq)
#pragma unroll
              for (int mi = 0; mi < 8; ++mi)
#pragma unroll
                for (int c = 0; c < 4; ++c) acc[nq][mi][c] *= rb;
            vref = vmax;
            inv_vref = 1.f / vmax;
            pscaleA = (g < nv) ? vsA * inv_vref : 0.f;
            pscaleB = (g + 8 < nv) ? vsB * inv_vref : 0.f;
          }
        }
        uint32_t pb[NQT][2][2];  // P^T B fragments: [nq][hi/lo part][reg]
#pragma unroll
        for (int nq = 0; nq < NQT; ++nq) {
          float pa[2], pbv[2];
#pragma unroll
          for (int c = 0; c < 2; ++c) {
            const float mref = m[nq][c];
            pa[c] = (mref == -INFINITY) ? 0.f : ex2_approx(sv[nq][c] - mref);
            pbv[c] = (mref == -INFINITY) ? 0.f : ex2_approx(sv[nq][2 + c] - mref);
            l[nq][c] += pa[c] + pbv[c];
            if (kB8) {
              pa[c] *= pscaleA;
              pbv[c] *= pscaleB;
            }
          }
          pb[nq][0][0] = movm_t(pack2<kBF16>(pa[0], pa[1]));
          pb[nq][0][1] = movm_t(pack2<kBF16>(pbv[0], pbv[1]));
          if (kBF16) {
            pb[nq][1][0] = movm_t(pack2<true>(pa[0] - round16<true>(pa[0]), pa[1] - round16<true>(pa[1])));
            pb[nq][1][1] = movm_t(pack2<true>(pbv[0] - round16<true>(pbv[0]), pbv[1] - round16<true>(pbv[1])));
          }
        }

        // ---------------- O^T += V^T . P^T
        {
          const int jm = lane >> 3;
          if (kB8) {
            // ldmatrix.trans over b16 units: a lane gets tokens 2t,2t+1 x dims 2g,2g+1
            // of a 16-byte chunk; A row g <-> dim 2g, row g+8 <-> dim 2g+1.
            const int vtok = (lane & 7) + 8 * (jm & 1);
#pragma unroll
            for (int c2 = 0; c2 < 4; ++c2) {
              const int chunk = 2 * c2 + (jm >> 1);
              uint32_t r0, r1, r2, r3;
              ldsm_x4_t(sV + vtok * 128 + ((chunk ^ (vtok & 7)) << 4), r0, r1, r2, r3);
              uint32_t a[4];
              cvt_b8x4<KVDT>(__byte_perm(r0, 0, 0x3120), a[0], a[1]);
              cvt_b8x4<KVDT>(__byte_perm(r1, 0, 0x3120), a[2], a[3]);
              if (nv < SCKV_PAGE_TOKENS) {
                a[0] = mask_pair(a[0], 2 * t, 2 * t + 1, nv);
                a[1] = mask_pair(a[1], 2 * t, 2 * t + 1, nv);
                a[2] = mask_pair(a[2], 2 * t + 8, 2 * t + 9, nv);
                a[3] = mask_pair(a[3], 2 * t + 8, 2 * t + 9, nv);
              }
#pragma unroll
              for (int nq = 0; nq < NQT; ++nq) mma16816<false>(acc[nq][2 * c2], a, pb[nq][0][0], pb[nq][0][1]);
              cvt_b8x4<KVDT>(__byte_perm(r2, 0, 0x3120), a[0], a[1]);
              cvt_b8x4<KVDT>(__byte_perm(r3, 0, 0x3120), a[2], a[3]);
              if (nv < SCKV_PAGE_TOKENS) {
                a[0] = mask_pair(a[0], 2 * t, 2 * t + 1, nv);
                a[1] = mask_pair(a[1], 2 * t, 2 * t + 1, nv);
                a[2] = mask_pair(a[2], 2 * t + 8, 2 * t + 9, nv);
                a[3] = mask_pair(a[3], 2 * t + 8, 2 * t + 9, nv);
              }
#pragma unroll
              for (int nq = 0; nq < NQT; ++nq)
                mma16816<false>(acc[nq][2 * c2 + 1], a, pb[nq][0][0], pb[nq][0][1]);
            }
          } else {
            const int tok = (lane & 7) + 8 * (jm >> 1);
#pragma unroll
            for (int mi = 0; mi < 8; ++mi) {
              const int cb = 2 * (mi & 3) + (jm & 1);
              uint32_t a[4];
              ldsm_x4_t(sV + (mi >> 2) * SM::kBoxStride + tok * 128 + ((cb ^ (tok & 7)) << 4), a[0], a[1], a[2], a[3]);
              if (nv < SCKV_PAGE_TOKENS) {
                a[0] = mask_pair(a[0], 2 * t, 2 * t + 1, nv);
                a[1] = mask_pair(a[1], 2 * t, 2 * t + 1, nv);
                a[2] = mask_pair(a[2], 2 * t + 8, 2 * t + 9, nv);
                a[3] = mask_pair(a[3], 2 * t + 8, 2 * t + 9, nv);
              }
#pragma unroll
              for (int nq = 0; nq < NQT; ++nq) {
                mma16816<kBF16>(acc[nq][mi], a, pb[nq][0][0], pb[nq][0][1]);
                if (kBF16) mma16816<true>(acc[nq][mi], a, pb[nq][1][0], pb[nq][1][1]);
              }
            }
          }
        }
      }
      // the slot's next TMA copy (async proxy) comes after this warp's stores
      if (fused) fence_proxy_async_shared();
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[st]);
    }
    gbase += n;

    // ---- reduce l over the 8 row groups, then merge the warps of each head
    float* red_acc = red;                             // [warp][q][HD]
    float* red_ml = red + kConsumerWarps * kG * kHD;  // [warp][q][2]
#pragma unroll
    for (int nq = 0; nq < NQT; ++nq) {
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        float ls = l[nq][c];
        ls += __shfl_xor_sync(0xffffffffu, ls, 4);
        ls += __shfl_xor_sync(0xffffffffu, ls, 8);
        ls += __shfl_xor_sync(0xffffffffu, ls, 16);
        const int q = 8 * nq + 2 * t + c;
        if (g == 0 && q < G) {
          red_ml[(warp * kG + q) * 2] = m[nq][c];
          red_ml[(warp * kG + q) * 2 + 1] = ls;
        }
      }
#pragma unroll
      for (int mi = 0; mi < 8; ++mi) {
        // FP8: A row g <-> dim 16mi+2g, row g+8 <-> dim 16mi+2g+1
        const int dA = kB8 ? 16 * mi + 2 * g : 16 * mi + g;
        const int dB = kB8 ? dA + 1 : dA + 8;
        const float vs = kB8 ? vref : 1.f;
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          const int q = 8 * nq + 2 * t + c;
          if (q < G) {
            red_acc[(warp * kG + q) * kHD + dA] = acc[nq][mi][c] * vs;
            red_acc[(warp * kG + q) * kHD + dB] = acc[nq][mi][2 + c] * vs;
          }
        }
      }
    }
    named_bar_sync(1, kConsumerWarps * 32);
    const int d = threadIdx.x;  // head dim
    for (int hh = 0; hh < HG; ++hh) {
      for (int q = 0; q < G; ++q) {
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < kWPH; ++w) M = fmaxf(M, red_ml[((hh * kWPH + w) * kG + q) * 2]);
        float L = 0.f, O = 0.f;
        if (M != -INFINITY) {
#pragma unroll
          for (int w = 0; w < kWPH; ++w) {
            const int ww = hh * kWPH + w;
            const float mw = red_ml[(ww * kG + q) * 2];
            if (mw == -INFINITY) continue;
            const float e = exp2f(mw - M);
            L = fmaf(red_ml[(ww * kG + q) * 2 + 1], e, L);
            O = fmaf(red_acc[(ww * kG + q) * kHD + d], e, O);
          }
        }
        const int hq = (h0 + hh) * G + q;
        if (nsplits == 1) {
          store_out(p, b, hq, d, (L > 0.f) ? O / L : 0.f);
        } else {
          const int64_t slot = ((int64_t)b * p.hq + hq) * p.max_splits + split;
          p.part_acc[slot * kHD + d] = O;
          if (d == 0) {
            p.part_ml[slot * 2] = M;
            p.part_ml[slot * 2 + 1] = L;
          }
        }
      }
    }
    named_bar_sync(1, kConsumerWarps * 32);
  }
}

template <int KVDT, int NQT, int HG, int S>
int launch_mma(const sckv_pool* pool, const DecodeParams& prm, cudaStream_t stream) {
  using SM = MmaSmem<KVDT, NQT, HG, S>;
  auto kern = decode_mma_kernel<KVDT, NQT, HG, S>;
  static bool configured[64] = {};
  const int dev = pool->device;
  if (dev < 0 || dev >= 64) return SCKV_ERR_INVALID_ARG;
  sckv_pool* mp = const_cast<sckv_pool*>(pool);  // the map is a cache inside the handle
  const int rc = ensure_tmap(pool, HG, mp->tmap_kv, &mp->tmap_ready);
  if (rc != SCKV_OK) return rc;
  if (!configured[dev]) {
    SCKV_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, SM::kBytes));
    configured[dev] = true;
  }
  int occ = 0;
  SCKV_CUDA_CHECK(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, kThreads, SM::kBytes));
  if (occ < 1) occ = 1;
  const int n_items = prm.n_seqs * (prm.hkv / HG) * prm.max_splits;
  int grid = pool->num_sms * occ;
  if (grid > n_items) grid = n_items;
  if (grid < 1) grid = 1;
  const CUtensorMap* map = reinterpret_cast<const CUtensorMap*>(pool->tmap_kv);
  kern<<<grid, kThreads, SM::kBytes, stream>>>(prm, *map);
  SCKV_LAUNCH_CHECK();
  return launch_combine(prm, stream);
}

template <int KVDT, int HG, int S>
int launch_mma_nq(const sckv_pool* pool, int G, const DecodeParams& prm, cudaStream_t stream) {
  return G > 8 ? launch_mma<KVDT, 2, HG, S>(pool, prm, stream) : launch_mma<KVDT, 1, HG, S>(pool, prm, stream);
}

}  // namespace

namespace sckv_detail {

int launch_decode_mma(const sckv_pool* pool, int G, const DecodeParams& prm, cudaStream_t stream) {
  if (pool->head_dim != kHD || G < 1 || G > 16) return SCKV_ERR_UNSUPPORTED;
  if ((int64_t)pool->num_layers * pool->max_pages > INT32_MAX) return SCKV_ERR_UNSUPPORTED;
  const int H = pool->num_kv_heads;
  // Stages hold one page of HG kv heads (16 KiB for HG=4 FP8 / HG=2 16-bit);
  // ring depths are multiples of the warps per head (4 / HG).
  switch (pool->kv_dtype) {
    case SCKV_DTYPE_F16:
      return (H % 2 == 0) ? launch_mma_nq<SCKV_DTYPE_F16, 2, 4>(pool, G, prm, stream)
                          : launch_mma_nq<SCKV_DTYPE_F16, 1, 8>(pool, G, prm, stream);
    case SCKV_DTYPE_BF16:
      return (H % 2 == 0) ? launch_mma_nq<SCKV_DTYPE_BF16, 2, 4>(pool, G, prm, stream)
                          : launch_mma_nq<SCKV_DTYPE_BF16, 1, 8>(pool, G, prm, stream);
    case SCKV_DTYPE_FP8_E4M3:
      // the page's 2*H scales travel as one bulk copy: needs H even (and <= 32)
      if (H > 32 || H % 2 != 0) return SCKV_ERR_UNSUPPORTED;
      // 4 heads per stage: three CTAs of 3 stages per SM keep as many bytes in
      // flight as two of 5 and hide the MMA / convert latencies better
      // (Qwen3 FP8: 0.791 -> 0.746 ms per layer launch)
      return (H % 4 == 0) ? launch_mma_nq<SCKV_DTYPE_FP8_E4M3, 4, 3>(pool, G, prm, stream)
                          : launch_mma_nq<SCKV_DTYPE_FP8_E4M3, 2, 10>(pool, G, prm, stream);
    case SCKV_DTYPE_INT8:
      // per-token scales of the group's heads travel as two bulk copies
      if (pool->scales == nullptr) return SCKV_ERR_UNSUPPORTED;
      return (H % 4 == 0) ? launch_mma_nq<SCKV_DTYPE_INT8, 4, 3>(pool, G, prm, stream)
                          : (H % 2 == 0) ? launch_mma_nq<SCKV_DTYPE_INT8, 2, 10>(pool, G, prm, stream)
                                         : launch_mma_nq<SCKV_DTYPE_INT8, 1, 16>(pool, G, prm, stream);
    default:
      return SCKV_ERR_UNSUPPORTED;
  }
}

}  // namespace sckv_detail
