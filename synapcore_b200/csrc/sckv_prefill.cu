// Paged causal prefill attention on the tensor cores.
//
// For each sequence, T new query tokens at positions start..start+T-1 attend
// to every cached token at positions <= their own (models/adapters.py:
// 1209-1229 with the causal mask of :1218-1224 and pos_offset = start). The
// new tokens' K/V are already in the pages (appended first).
//
// Tiling (flash-attention style, one CTA = 4 compute warps + 1 TMA warp):
// a work item is (sequence, tile of 64/G query tokens, kv head); its 64
// query rows are (token, q head) pairs of the G heads that read the kv head,
// 16 rows per warp. Pages stream through an S-stage ring (TMA tensor copies,
// 128-byte swizzle, one kv head per box) and every warp multiplies its rows
// against every page it can see:
//   S[16 x 16 keys] = Q . K^T   (16 x mma.m16n8k16)
//   O[16 x 128]    += P . V     (16 x mma.m16n8k16)
// with fp32 accumulation; P reuses S's accumulator fragment as the A operand.
// The running max is stale (moves only by more than 2^8) as in the decode
// kernel. FP8 pages decode in registers; their V scale is folded into P
// relative to a per-item reference scale.
#include <math.h>
#include <stdlib.h>
#include <string.h>

#include "sckv_decode_common.cuh"
#include "sckv_mma_common.cuh"

using namespace sckv_detail;
using namespace sckv_mma;

namespace {

constexpr int kRows = 64;  // query rows per item (16 per compute warp)

struct PrefillParams {
  const uint8_t* pool;
  const float* fp8_scales;
  const void* q;    // [n_tokens][hq][128]
  void* out;        // [n_tokens][hq][128]
  const int32_t* cu_q;       // [n_seqs + 1]
  const int32_t* start_pos;  // [n_seqs]
  const int32_t* block_table;
  int32_t* status;
  int64_t bt_stride;
  int64_t max_pages;
  int max_blocks;
  int n_seqs;
  int n_tokens;
  int hq;
  int hkv;
  int lg_g;  // log2(G)
  int layer;
  int q_dtype;
  int out_dtype;
  float scale_log2;
};

template <int KVDT, int S>
struct PrefillSmem {
  static constexpr int kBoxes = MmaKV<KVDT>::kEB;
  static constexpr int kBoxStride = 2 * kBoxBytes;  // one kv head: K and V
  static constexpr int kStageBytes = kBoxes * kBoxStride;
  static constexpr int kRingBytes = S * kStageBytes;
  static constexpr int kScaleSlot = 64;
  static constexpr int kScaleBytes = (KVDT == SCKV_DTYPE_FP8_E4M3) ? S * kScaleSlot * 4 : 0;
  static constexpr int kFixedBytes = 1024 + kRingBytes + kScaleBytes + 2 * S * 8 + 16;
};

// Tokens of sequence s, clamped to what its block table can hold.
__device__ __forceinline__ int seq_tokens(const PrefillParams& p, int s, int* start_out, bool report) {
  int t0 = __ldg(p.cu_q + s), t1 = __ldg(p.cu_q + s + 1);
  int st = __ldg(p.start_pos + s);
  int T = t1 - t0;
  const int cap = p.max_blocks * SCKV_PAGE_TOKENS;
  if (T < 0 || st < 0 || t0 < 0 || t1 > p.n_tokens || st + T > cap) {
    if (report) sckv_report(p.status, SCKV_ERR_BOUNDS, s, KID_DECODE);
    T = 0;
    st = 0;
  }
  *start_out = st;
  return T;
}

template <int KVDT, int S>
__global__ void __launch_bounds__(kThreads, 1)
    prefill_kernel(const PrefillParams p, const __grid_constant__ CUtensorMap tmap) {
  using SM = PrefillSmem<KVDT, S>;
  constexpr bool kBF16 = (KVDT == SCKV_DTYPE_BF16);
  constexpr bool kFP8 = (KVDT == SCKV_DTYPE_FP8_E4M3);
  extern __shared__ __align__(16) uint8_t smem_raw[];
  uint8_t* ring = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float* sscale = reinterpret_cast<float*>(ring + SM::kRingBytes);
  uint64_t* full = reinterpret_cast<uint64_t*>(ring + SM::kRingBytes + SM::kScaleBytes);
  uint64_t* empty = full + S;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(empty + S);
  int* tile_cum = const_cast<int*>(reinterpret_cast<volatile int*>(abort_flag + 4));  // [n_seqs + 1]

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int G = 1 << p.lg_g;
  const int BQ = kRows >> p.lg_g;  // query tokens per item
  if (threadIdx.x == 0) {
    for (int i = 0; i < S; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], kConsumerWarps);
    }
    *abort_flag = 0;
    fence_mbar_init();
    int acc = 0;
    tile_cum[0] = 0;
    for (int s = 0; s < p.n_seqs; ++s) {
      int st;
      const int T = seq_tokens(p, s, &st, blockIdx.x == 0);
      acc += (T + BQ - 1) / BQ;
      tile_cum[s + 1] = acc;
    }
  }
  __syncthreads();
  const int total_tiles = tile_cum[p.n_seqs];
  const int n_items = total_tiles * p.hkv;
  const int64_t layer_base = (int64_t)p.layer * p.max_pages;

  // item -> (sequence, tile, kv head); tiles visited from the last (most keys) down
  auto decode_item = [&](int item, int& seq, int& tile, int& h) {
    h = item % p.hkv;
    const int gt = total_tiles - 1 - item / p.hkv;
    int lo = 0, hi = p.n_seqs - 1;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (tile_cum[mid] <= gt) lo = mid; else hi = mid - 1;
    }
    seq = lo;
    tile = gt - tile_cum[lo];
  };

  if (warp == kConsumerWarps) {
    // ------------------------------------------------------------ producer
    if (lane != 0) return;
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmap)) : "memory");
    uint32_t gcount = 0;
    bool aborted = false;
    const uint32_t tx = SM::kStageBytes + (kFP8 ? 8 * p.hkv : 0);
    for (int item = blockIdx.x; item < n_items && !aborted; item += gridDim.x) {
      int seq, tile, h;
      decode_item(item, seq, tile, h);
      int s0;
      const int T = seq_tokens(p, seq, &s0, false);
      const int tok_last = min(T, (tile + 1) * BQ) - 1;
      const int jlast = (s0 + tok_last) / SCKV_PAGE_TOKENS;
      const int32_t* bt_row = p.block_table + (int64_t)seq * p.bt_stride;
      for (int j = 0; j <= jlast; ++j) {
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
        const int slab = (int)(layer_base + page);
        const uint32_t dst = smem_u32(ring + st * SM::kStageBytes);
        mbar_arrive_expect_tx(&full[st], tx);
        if (kFP8)
          bulk_g2s(sscale + st * SM::kScaleSlot, p.fp8_scales + (int64_t)slab * 2 * p.hkv, 8 * p.hkv, &full[st]);
#pragma unroll
        for (int bx = 0; bx < SM::kBoxes; ++bx)
          tma_load_5d(dst + bx * SM::kBoxStride, &tmap, bx * (128 / MmaKV<KVDT>::kEB), 0, h, 0, slab, &full[st]);
        ++gcount;
      }
    }
    const uint32_t first = gcount > S ? gcount - S : 0;
    for (uint32_t k = first; k < gcount; ++k) mbar_wait_bounded(&full[k % S], (k / S) & 1, SCKV_WAIT_LIMIT_NS);
    return;
  }

  // -------------------------------------------------------------- consumers
  const int g = lane >> 2;
  const int t = lane & 3;
  const int r0 = warp * 16 + g;  // this lane's two query rows: r0 and r0 + 8
  uint32_t gbase = 0;
  bool aborted = false;
  for (int item = blockIdx.x; item < n_items; item += gridDim.x) {
    int seq, tile, h;
    decode_item(item, seq, tile, h);
    int s0;
    const int T = seq_tokens(p, seq, &s0, false);
    const int ctx_total = s0 + T;
    const int tok0 = tile * BQ;
    const int tok_last = min(T, tok0 + BQ) - 1;
    const int jlast = (s0 + tok_last) / SCKV_PAGE_TOKENS;
    const int q_base = __ldg(p.cu_q + seq);
    // rows -> (token, q head)
    int rtok[2], rhead[2];
    bool rvalid[2];
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const int r = r0 + 8 * u;
      rtok[u] = tok0 + (r >> p.lg_g);
      rhead[u] = h * G + (r & (G - 1));
      rvalid[u] = rtok[u] < T;
    }
    // the warp's last visible key: the largest token among its rows
    const int warp_tok_hi = min(T - 1, tok0 + ((warp * 16 + 15) >> p.lg_g));
    const int warp_key_hi = s0 + warp_tok_hi;
    const bool warp_active = tok0 + ((warp * 16) >> p.lg_g) < T;  // a warp past the tile's end only drains the ring

    // Q fragments (A operand): rows r0, r0+8; k-step s covers dims 16s.. (FP8: permuted)
    uint32_t qa[8][4];
#pragma unroll
    for (int s = 0; s < 8; ++s) {
      const int d0 = kFP8 ? 16 * s + 4 * t : 16 * s + 2 * t;
      const int d1 = kFP8 ? d0 + 2 : d0 + 8;
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        float v0 = 0.f, v1 = 0.f, v2 = 0.f, v3 = 0.f;
        if (rvalid[u]) {
          const int64_t qoff = ((int64_t)(q_base + rtok[u]) * p.hq + rhead[u]) * kHD;
          v0 = sckv_load_as_float(p.q, qoff + d0, p.q_dtype);
          v1 = sckv_load_as_float(p.q, qoff + d0 + 1, p.q_dtype);
          v2 = sckv_load_as_float(p.q, qoff + d1, p.q_dtype);
          v3 = sckv_load_as_float(p.q, qoff + d1 + 1, p.q_dtype);
        }
        qa[s][u] = pack2<kBF16>(v0, v1);      // a0a1 (u=0) / a2a3 (u=1)
        qa[s][2 + u] = pack2<kBF16>(v2, v3);  // a4a5 / a6a7
      }
    }
    float acc[16][4];
#pragma unroll
    for (int i = 0; i < 16; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
    float m[2] = {-INFINITY, -INFINITY}, l[2] = {0.f, 0.f};
    float vref = 0.f;

    for (int j = 0; j <= jlast; ++j) {
      const uint32_t gi = gbase + j;
      const uint32_t st = gi % S;
      if (!aborted) {
        if (*abort_flag || !mbar_wait_bounded(&full[st], (gi / S) & 1, SCKV_WAIT_LIMIT_NS)) {
          if (lane == 0 && !*abort_flag) sckv_report(p.status, SCKV_ERR_TIMEOUT, item, KID_DECODE);
          if (lane == 0) *abort_flag = 1;
          aborted = true;
        }
      }
      if (!aborted && warp_active && j * SCKV_PAGE_TOKENS <= warp_key_hi) {
        const uint32_t stage = smem_u32(ring + st * SM::kStageBytes);
        const uint32_t sK = stage;
        const uint32_t sV = stage + kBoxBytes;
        float kscale = 1.f, vscale = 1.f;
        if (kFP8) {
          kscale = sscale[st * SM::kScaleSlot + h];
          vscale = sscale[st * SM::kScaleSlot + p.hkv + h];
        }
        // ---------------- S = Q K^T (two n-tiles of 8 keys)
        float sc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
        const int mat = lane >> 3;
        const int key = (lane & 7) + 8 * (kFP8 ? (mat & 1) : (mat >> 1));
        if (kFP8) {
#pragma unroll
          for (int c2 = 0; c2 < 4; ++c2) {
            const int chunk = 2 * c2 + (mat >> 1);
            uint32_t w0, w1, w2, w3;
            ldsm_x4(sK + key * 128 + ((chunk ^ (key & 7)) << 4), w0, w1, w2, w3);
            uint32_t b00, b01, b10, b11;
            cvt_fp8x4(w0, b00, b01);
            cvt_fp8x4(w1, b10, b11);
            mma16816<false>(sc[0], qa[2 * c2], b00, b01);
            mma16816<false>(sc[1], qa[2 * c2], b10, b11);
            cvt_fp8x4(w2, b00, b01);
            cvt_fp8x4(w3, b10, b11);
            mma16816<false>(sc[0], qa[2 * c2 + 1], b00, b01);
            mma16816<false>(sc[1], qa[2 * c2 + 1], b10, b11);
          }
        } else {
#pragma unroll
          for (int s = 0; s < 8; ++s) {
            const int chunk = 2 * s + (mat & 1);
            uint32_t r0_, r1_, r2_, r3_;
            ldsm_x4(sK + (chunk >> 3) * SM::kBoxStride + key * 128 + (((chunk & 7) ^ (key & 7)) << 4), r0_, r1_,
                    r2_, r3_);
            mma16816<kBF16>(sc[0], qa[s], r0_, r1_);
            mma16816<kBF16>(sc[1], qa[s], r2_, r3_);
          }
        }
        // ---------------- causal mask, stale running max
        const float sscale = p.scale_log2 * kscale;
        float sv[2][4];  // [n-tile][c]: c0,c1 row r0 keys (2t, 2t+1); c2,c3 row r0+8
        float pm[2];
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          const int lim = rvalid[u] ? s0 + rtok[u] : -1;  // last visible key position
          float mx = -INFINITY;
#pragma unroll
          for (int nt = 0; nt < 2; ++nt)
#pragma unroll
            for (int c = 0; c < 2; ++c) {
              const int kpos = j * SCKV_PAGE_TOKENS + nt * 8 + 2 * t + c;
              const float v = (kpos <= lim) ? sc[nt][2 * u + c] * sscale : -INFINITY;
              sv[nt][2 * u + c] = v;
              mx = fmaxf(mx, v);
            }
          mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
          mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
          pm[u] = mx;
        }
        const bool grow = (pm[0] > m[0] + 8.f) || (pm[1] > m[1] + 8.f);
        if (__any_sync(0xffffffffu, grow)) {
#pragma unroll
          for (int u = 0; u < 2; ++u) {
            const float mn = fmaxf(m[u], pm[u]);
            const float alpha = (mn == -INFINITY) ? 1.f : exp2f(m[u] - mn);
            m[u] = mn;
            l[u] *= alpha;
#pragma unroll
            for (int nt = 0; nt < 16; ++nt) {
              acc[nt][2 * u] *= alpha;
              acc[nt][2 * u + 1] *= alpha;
            }
          }
        }
        float pscale = 1.f;
        if (kFP8) {
          if (vref == 0.f) vref = vscale;
          pscale = (vref > 0.f) ? vscale / vref : 0.f;
          if (pscale > 64.f) {
            const float rb = vref / vscale;
#pragma unroll
            for (int nt = 0; nt < 16; ++nt)
#pragma unroll
              for (int c = 0; c < 4; ++c) acc[nt][c] *= rb;
            vref = vscale;
            pscale = 1.f;
          }
        }
        float pv[2][4];
#pragma unroll
        for (int nt = 0; nt < 2; ++nt)
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            const float mref = m[c >> 1];
            const float pr = (mref == -INFINITY) ? 0.f : exp2f(sv[nt][c] - mref);
            l[c >> 1] += pr;
            pv[nt][c] = kFP8 ? pr * pscale : pr;
          }
        // P as the A operand: rows r0 / r0+8, keys 2t.. (n-tile 0) and 8+2t.. (n-tile 1)
        uint32_t pa[4] = {pack2<kBF16>(pv[0][0], pv[0][1]), pack2<kBF16>(pv[0][2], pv[0][3]),
                          pack2<kBF16>(pv[1][0], pv[1][1]), pack2<kBF16>(pv[1][2], pv[1][3])};
        uint32_t pl[4] = {0u, 0u, 0u, 0u};
        if (kBF16) {
          pl[0] = pack2<true>(pv[0][0] - round16<true>(pv[0][0]), pv[0][1] - round16<true>(pv[0][1]));
          pl[1] = pack2<true>(pv[0][2] - round16<true>(pv[0][2]), pv[0][3] - round16<true>(pv[0][3]));
          pl[2] = pack2<true>(pv[1][0] - round16<true>(pv[1][0]), pv[1][1] - round16<true>(pv[1][1]));
          pl[3] = pack2<true>(pv[1][2] - round16<true>(pv[1][2]), pv[1][3] - round16<true>(pv[1][3]));
        }
        // ---------------- O += P V
        const int nv = min(SCKV_PAGE_TOKENS, ctx_total - j * SCKV_PAGE_TOKENS);
        const int vkey = (lane & 7) + 8 * (mat & 1);
        if (kFP8) {
#pragma unroll
          for (int c2 = 0; c2 < 4; ++c2) {
            const int chunk = 2 * c2 + (mat >> 1);
            uint32_t w0, w1, w2, w3;
            ldsm_x4_t(sV + vkey * 128 + ((chunk ^ (vkey & 7)) << 4), w0, w1, w2, w3);
            // w0: keys 0-7 / w1: keys 8-15 of chunk 2c2; w2, w3: chunk 2c2+1
            const uint32_t ws[4] = {w0, w1, w2, w3};
#pragma unroll
            for (int cc = 0; cc < 2; ++cc) {
              uint32_t lo0, hi0, lo1, hi1;
              cvt_fp8x4(__byte_perm(ws[2 * cc], 0, 0x3120), lo0, hi0);
              cvt_fp8x4(__byte_perm(ws[2 * cc + 1], 0, 0x3120), lo1, hi1);
              if (nv < SCKV_PAGE_TOKENS) {
                lo0 = mask_pair(lo0, 2 * t, 2 * t + 1, nv);
                hi0 = mask_pair(hi0, 2 * t, 2 * t + 1, nv);
                lo1 = mask_pair(lo1, 2 * t + 8, 2 * t + 9, nv);
                hi1 = mask_pair(hi1, 2 * t + 8, 2 * t + 9, nv);
              }
              const int nt = 2 * (2 * c2 + cc);  // n-tiles (chunk, even dims) and (chunk, odd dims)
              mma16816<false>(acc[nt], pa, lo0, lo1);
              mma16816<false>(acc[nt + 1], pa, hi0, hi1);
            }
          }
        } else {
#pragma unroll
          for (int c2 = 0; c2 < 8; ++c2) {
            const int chunk = 2 * c2 + (mat >> 1);
            uint32_t b0a, b1a, b0b, b1b;
            ldsm_x4_t(sV + (chunk >> 3) * SM::kBoxStride + vkey * 128 + (((chunk & 7) ^ (vkey & 7)) << 4), b0a,
                      b1a, b0b, b1b);
            if (nv < SCKV_PAGE_TOKENS) {
              b0a = mask_pair(b0a, 2 * t, 2 * t + 1, nv);
              b1a = mask_pair(b1a, 2 * t + 8, 2 * t + 9, nv);
              b0b = mask_pair(b0b, 2 * t, 2 * t + 1, nv);
              b1b = mask_pair(b1b, 2 * t + 8, 2 * t + 9, nv);
            }
            mma16816<kBF16>(acc[2 * c2], pa, b0a, b1a);
            mma16816<kBF16>(acc[2 * c2 + 1], pa, b0b, b1b);
            if (kBF16) {
              mma16816<true>(acc[2 * c2], pl, b0a, b1a);
              mma16816<true>(acc[2 * c2 + 1], pl, b0b, b1b);
            }
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[st]);
    }
    gbase += jlast + 1;

    // ---- normalise and write the two rows of this lane
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      float ls = l[u];
      ls += __shfl_xor_sync(0xffffffffu, ls, 1);
      ls += __shfl_xor_sync(0xffffffffu, ls, 2);
      const float inv = (ls > 0.f) ? (kFP8 ? vref : 1.f) / ls : 0.f;
      if (!rvalid[u]) continue;
      const int64_t obase = ((int64_t)(q_base + rtok[u]) * p.hq + rhead[u]) * kHD;
#pragma unroll
      for (int nt = 0; nt < 16; ++nt) {
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          // column 2t+c of n-tile nt -> head dim
          const int col = 2 * t + c;
          const int dim = kFP8 ? 16 * (nt >> 1) + 2 * col + (nt & 1) : 8 * nt + col;
          sckv_store_from_float(p.out, obase + dim, p.out_dtype, acc[nt][2 * u + c] * inv);
        }
      }
    }
  }
}

template <int KVDT, int S>
int launch_prefill(const sckv_pool* pool, const PrefillParams& prm, int max_tiles, cudaStream_t stream) {
  using SM = PrefillSmem<KVDT, S>;
  auto kern = prefill_kernel<KVDT, S>;
  const int dev = pool->device;
  if (dev < 0 || dev >= 64) return SCKV_ERR_INVALID_ARG;
  sckv_pool* mp = const_cast<sckv_pool*>(pool);  // the map is a cache inside the handle
  int rc = ensure_tmap(pool, 1, mp->tmap_kv1, &mp->tmap1_ready);
  if (rc != SCKV_OK) return rc;
  const int smem = SM::kFixedBytes + 4 * (prm.n_seqs + 2);
  if (smem > 227 * 1024) return SCKV_ERR_INVALID_ARG;
  SCKV_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
  int occ = 0;
  SCKV_CUDA_CHECK(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, kThreads, smem));
  if (occ < 1) occ = 1;
  const int64_t items = (int64_t)max_tiles * prm.hkv;
  int64_t grid = (int64_t)pool->num_sms * occ;
  if (grid > items) grid = items;
  if (grid < 1) grid = 1;
  kern<<<(int)grid, kThreads, smem, stream>>>(prm, *reinterpret_cast<const CUtensorMap*>(pool->tmap_kv1));
  SCKV_LAUNCH_CHECK();
  return SCKV_OK;
}

}  // namespace

extern "C" int sckv_prefill_attn(sckv_pool* pool, int layer, const void* q, int q_dtype, int num_q_heads, int n_seqs,
                                 int n_tokens, const int32_t* cu_q, const int32_t* start_pos,
                                 const int32_t* block_table, int64_t bt_stride, int max_blocks, float scale, void* out,
                                 int out_dtype, void* stream) {
  if (pool == nullptr) return SCKV_ERR_INVALID_ARG;
  if (pool->head_dim != kHD) return SCKV_ERR_UNSUPPORTED;
  if (layer < 0 || layer >= pool->num_layers) return SCKV_ERR_INVALID_ARG;
  if (n_seqs <= 0 || n_tokens < 0 || num_q_heads <= 0 || max_blocks <= 0 || bt_stride < max_blocks)
    return SCKV_ERR_INVALID_ARG;
  if (n_seqs > 16384) return SCKV_ERR_INVALID_ARG;
  if (n_tokens == 0) return SCKV_OK;
  if (!q || !out || !cu_q || !start_pos || !block_table) return SCKV_ERR_INVALID_ARG;
  if (num_q_heads % pool->num_kv_heads != 0) return SCKV_ERR_INVALID_ARG;
  const int G = num_q_heads / pool->num_kv_heads;
  if (G > 16 || (G & (G - 1)) != 0) return SCKV_ERR_UNSUPPORTED;
  if (q_dtype != SCKV_DTYPE_F16 && q_dtype != SCKV_DTYPE_BF16 && q_dtype != SCKV_DTYPE_F32) return SCKV_ERR_INVALID_ARG;
  if (out_dtype != SCKV_DTYPE_F16 && out_dtype != SCKV_DTYPE_BF16 && out_dtype != SCKV_DTYPE_F32)
    return SCKV_ERR_INVALID_ARG;
  if (pool->kv_dtype == SCKV_DTYPE_BF16 && q_dtype != SCKV_DTYPE_BF16) return SCKV_ERR_UNSUPPORTED;
  if ((int64_t)pool->num_layers * pool->max_pages > INT32_MAX) return SCKV_ERR_UNSUPPORTED;
  int lg = 0;
  while ((1 << lg) < G) ++lg;
  PrefillParams prm{};
  prm.pool = reinterpret_cast<const uint8_t*>(pool->data);
  prm.fp8_scales = reinterpret_cast<const float*>(pool->scales);
  prm.q = q;
  prm.out = out;
  prm.cu_q = cu_q;
  prm.start_pos = start_pos;
  prm.block_table = block_table;
  prm.status = pool->status;
  prm.bt_stride = bt_stride;
  prm.max_pages = pool->max_pages;
  prm.max_blocks = max_blocks;
  prm.n_seqs = n_seqs;
  prm.n_tokens = n_tokens;
  prm.hq = num_q_heads;
  prm.hkv = pool->num_kv_heads;
  prm.lg_g = lg;
  prm.layer = layer;
  prm.q_dtype = q_dtype;
  prm.out_dtype = out_dtype;
  prm.scale_log2 = scale * 1.4426950408889634f;
  // every pool type: the tensor-memory kernel (sckv_prefill_tc.cu) unless
  // SCKV_PREFILL_KERNEL=mma asks for this one (f16 / bf16 / FP8)
  const char* env = getenv("SCKV_PREFILL_KERNEL");
  const bool forced = env != nullptr && strcmp(env, "mma") == 0;
  SCKV_DEVICE_GUARD(pool->device);
  if (!forced) {
    const int rc = launch_prefill_tc(pool, layer, q, q_dtype, num_q_heads, n_seqs, n_tokens, cu_q, start_pos,
                                     block_table, bt_stride, max_blocks, scale, out, out_dtype, lg,
                                     as_stream(stream));
    if (rc != SCKV_ERR_UNSUPPORTED) return rc;
  }
  if (pool->kv_dtype == SCKV_DTYPE_INT8) return SCKV_ERR_UNSUPPORTED;
  if (pool->kv_dtype == SCKV_DTYPE_FP8_E4M3 && (pool->num_kv_heads % 2 != 0 || pool->num_kv_heads > 32))
    return SCKV_ERR_UNSUPPORTED;
  const int BQ = kRows >> lg;
  const int max_tiles = (n_tokens + BQ - 1) / BQ + n_seqs;  // upper bound on sum of ceil(T_s / BQ)
  cudaStream_t s = as_stream(stream);
  switch (pool->kv_dtype) {
    case SCKV_DTYPE_F16: return launch_prefill<SCKV_DTYPE_F16, 6>(pool, prm, max_tiles, s);
    case SCKV_DTYPE_BF16: return launch_prefill<SCKV_DTYPE_BF16, 6>(pool, prm, max_tiles, s);
    case SCKV_DTYPE_FP8_E4M3: return launch_prefill<SCKV_DTYPE_FP8_E4M3, 10>(pool, prm, max_tiles, s);
    default: return SCKV_ERR_UNSUPPORTED;
  }
}
