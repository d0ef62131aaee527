// Paged causal prefill attention on the 5th-generation tensor cores
// (tcgen05.mma, accumulators in tensor memory).
//
// Same contract as prefill_kernel in sckv_prefill.cu (models/adapters.py:
// 1209-1229, causal mask :1218-1224, query t of a sequence at position
// start + t sees keys 0..start + t), for every pool type (one-byte pages
// are decoded into f16 tiles by the producer warps).
//
// Work item = (sequence, two tiles of 128 query rows, kv head). The rows
// are (token, q head) pairs of the G heads that read the kv head, so a tile
// holds 128 / G tokens; both tiles share every K/V tile loaded. One
// persistent CTA per SM (512 TMEM columns) claims items from a work counter;
// 16 warps (a warp runs on SM sub-partition warp % 4):
//   warps 0, 3  claim items (warp 0), load the item's Q (one TMA box per
//              64-dim half and tile for 16-bit q; f32 q is written by the
//              softmax threads) and stream K: 4 pages (64 keys) per tile,
//              one 2 KiB box per (page, 64-dim half), 128-byte swizzle, into
//              a ring laid out as the UMMA K-major canonical tile
//              (consecutive pages are consecutive rows); each warp copies
//              two pages of a tile (one TMA issue holds its warp ~0.1 us).
//              One-byte pools stage the codes by TMA and decode them with
//              all lanes.
//   warps 2, 12 stream V the same way into their own ring.
//   warp 1     allocates the tensor memory; its lane 0 alone issues the
//              MMAs and commits and does its own bounded waits:
//                S[w][b] (128 x 64 fp32) = Q[w] . K^T   8 x tcgen05.mma (K = 16)
//                O[w]    (128 x 128 fp32) += P[w][b] . V  4 x tcgen05.mma (A from TMEM)
//              for both Q tiles w, S double-buffered; K(j) is released when
//              both S(j) finished, V(j) after both PV(j). Completion is
//              signalled with tcgen05.commit on mbarriers. Its issue rate
//              paces the kernel, so its sub-partition (1) holds no producer
//              and no Q conversion.
//   warps 4-7, 8-11  softmax of Q tile 0, 1: thread i owns query row i (TMEM
//              lane i): loads its 64 scores with tcgen05.ld, masks (only tiles
//              the causal limit cuts), keeps a stale running max (moves only
//              by more than 2^8, rescaling O in TMEM when it does), writes
//              P = 2^(s*scale - m) as f16 / bf16 back over S (tcgen05.st;
//              3-input max and packed fp32 FMA / add), one barrier arrival
//              per warp, and at the end of the item normalises its O row and
//              stores it.
//   warps 14, 15  convert Q in place when it arrives in the other 16-bit
//              type than the MMAs'.
// bf16 pools split P into bf16 hi + lo parts (two PV products) so P's
// rounding stays below 2^-16 relative; f16 pools use P in f16.
// Slots past the sequence's last token (they may hold anything) are zeroed
// in the V tile before the PV product; their scores are masked.
#include <cuda.h>
#include <math.h>

#include "sckv_internal.cuh"
#include "sckv_mma_common.cuh"
#include "sckv_tcgen05.cuh"

using namespace sckv_mma;
using namespace sckv_tc;

namespace {

constexpr int kHDim = 128;
constexpr int kRowsTc = 128;                  // query rows per Q tile (UMMA M)
constexpr int kQTiles = 2;                    // Q tiles per item, sharing every K/V tile
constexpr int kKeysTc = 64;                   // keys per K/V tile (4 pages)
constexpr int kPagesTc = kKeysTc / SCKV_PAGE_TOKENS;
constexpr int kThreadsTc = 512;  // 16 warps, roles below
constexpr int kSoftmaxThreads = 128;  // per softmax warpgroup (one per Q tile)
constexpr uint32_t kTmemCols = 512;
// TMEM columns: S[w][b] at 64 (2 w + b), O[w] at 256 + 128 w
constexpr uint32_t kColS = 0;
constexpr uint32_t kColO = 256;

// warps: 0 claims items, loads Q and half of each K tile; 3 the other half
// of K; 2 and 12 the two halves of V; 1 issues the MMAs; 4-7 and 8-11 are
// the softmax warpgroups of Q tiles 0 and 1; 14 and 15 convert Q in place
// when it arrives by TMA in the other 16-bit type (else idle). Warp 13 stays
// idle: it would share SM sub-partition 1 (warp % 4) with the MMA-issuing
// thread, whose issue rate paces the kernel.
constexpr int kWarpK0 = 0, kWarpMma = 1, kWarpV0 = 2, kWarpK1 = 3, kWarpV1 = 12;

constexpr int kQHalf = kRowsTc * 128;         // one 64-dim half of a Q tile: 16 KiB
constexpr int kQTileBytes = 2 * kQHalf;
constexpr int kTileHalf = kKeysTc * 128;      // one 64-dim half of a K or V tile: 8 KiB
constexpr int kSlotBytes = 2 * kTileHalf;     // a K (or V) tile: lo and hi halves
// Shared-memory layout per pool type. One-byte pools (FP8, int8) stage each
// page's codes by TMA and have the producer warps decode them into the f16
// K / V rings (3 slots, to make room for the staging).
template <int KVDT>
struct TcCfg {
  static constexpr bool kB8 = KVDT == SCKV_DTYPE_FP8_E4M3 || KVDT == SCKV_DTYPE_INT8;
  static constexpr bool kBF16 = KVDT == SCKV_DTYPE_BF16;  // MMA type; f16 otherwise
  static constexpr int kStages = kB8 ? 3 : 4;
  static constexpr int kPageBox = SCKV_PAGE_TOKENS * 128;          // one page's codes: 16 rows x 128 B
  static constexpr int kStageSlot = 2 * kPageBox;                  // a producer warp's two pages of a tile
  static constexpr int kOffK = kQTiles * kQTileBytes;              // K ring [kStages]
  static constexpr int kOffV = kOffK + kStages * kSlotBytes;       // V ring [kStages]
  static constexpr int kOffStage = kOffV + kStages * kSlotBytes;   // [4 producer warps][2][kStageSlot]
  static constexpr int kOffBar = kOffStage + (kB8 ? 4 * 2 * kStageSlot : 0);
  static constexpr int kNumBars = 4 * kStages + 4 + 4 + 4 + 2 + 3 + 4 + (kB8 ? 8 : 0) + 1;
  static constexpr int kOffItemRing = kOffBar + kNumBars * 8;      // int[4]
  static constexpr int kOffTmemSlot = kOffItemRing + 16;
  static constexpr int kOffAbort = kOffTmemSlot + 4;
  static constexpr int kOffPartial = kOffTmemSlot + 16;
  static constexpr int kOffTileCum = kOffPartial + kThreadsTc * 4;
  static constexpr int kFixedSmem = 1024 + kOffTileCum;            // + 4 * (n_seqs + 1)
};

struct TcParams {
  const void* q;
  void* out;
  const int32_t* cu_q;
  const int32_t* start_pos;
  const int32_t* block_table;
  int32_t* status;
  int64_t bt_stride;
  int64_t max_pages;
  int max_blocks;
  int n_seqs;
  int n_tokens;
  int hq;
  int hkv;
  int lg_g;
  int layer;
  int q_dtype;
  int out_dtype;
  // how Q reaches shared memory: 0 the softmax threads load and convert it;
  // 1 TMA, q has the MMA's type; 2 TMA of the other 16-bit type, then warps
  // 14 and 15 convert the tile in place (bf16 <-> f16, rounded as load_q8 does)
  int q_tma;
  const void* kv_scales;  // one-byte pools: FP8 fp32 [L][P][K|V][H], int8 fp16 [L][P][K|V][H][16]
  unsigned long long* next_item;  // work counter, zero at launch
  float scale_log2;
};

// Tokens of sequence s (0 and a reported bounds error if its offsets or
// start are out of range).
__device__ __forceinline__ int tc_seq_tokens(const TcParams& p, int s, int* start_out, bool report) {
  const int t0 = __ldg(p.cu_q + s), t1 = __ldg(p.cu_q + s + 1);
  int st = __ldg(p.start_pos + s);
  int T = t1 - t0;
  const int cap = p.max_blocks * SCKV_PAGE_TOKENS;
  if (T < 0 || st < 0 || t0 < 0 || t1 > p.n_tokens || st + T > cap) {
    if (report) sckv_report(p.status, SCKV_ERR_BOUNDS, s, KID_PREFILL);
    T = 0;
    st = 0;
  }
  *start_out = st;
  return T;
}

// 8 query values (dims d..d+7 of one row) as packed f16 / bf16 pairs.
template <bool kBF16>
__device__ __forceinline__ uint4 load_q8(const void* q, int64_t idx, int dtype) {
  if (dtype == (kBF16 ? SCKV_DTYPE_BF16 : SCKV_DTYPE_F16))
    return *reinterpret_cast<const uint4*>(reinterpret_cast<const uint16_t*>(q) + idx);
  float v[8];
  if (dtype == SCKV_DTYPE_F32) {
    const float4 a = *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(q) + idx);
    const float4 b = *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(q) + idx + 4);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  } else {
    // the other 16-bit type: one 16-byte load, converted in registers (the
    // values are exact in fp32, so the MMA type sees them rounded once)
    const uint4 raw = *reinterpret_cast<const uint4*>(reinterpret_cast<const uint16_t*>(q) + idx);
    const uint32_t w4[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      if (dtype == SCKV_DTYPE_BF16) {
        v[2 * i] = __uint_as_float(w4[i] << 16);
        v[2 * i + 1] = __uint_as_float(w4[i] & 0xFFFF0000u);
      } else {
        const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w4[i]));
        v[2 * i] = f.x;
        v[2 * i + 1] = f.y;
      }
    }
  }
  uint4 r;
  r.x = pack2<kBF16>(v[0], v[1]);
  r.y = pack2<kBF16>(v[2], v[3]);
  r.z = pack2<kBF16>(v[4], v[5]);
  r.w = pack2<kBF16>(v[6], v[7]);
  return r;
}

// sm_100 arithmetic the softmax threads use to save issue slots: a 3-input
// max, and packed pairs of fp32 values (two independent round-to-nearest
// fp32 operations per instruction, the same results as two scalar ones).
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}
__device__ __forceinline__ uint64_t f32x2(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void f32x2_split(uint64_t v, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ uint64_t fma_f32x2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t add_f32x2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t mul_f32x2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
// a packed pair times a packed factor, rounded to a 16-bit pair
template <bool kBF16>
__device__ __forceinline__ uint32_t mul_pack2(float x, float y, uint64_t f2) {
  float a, b;
  f32x2_split(mul_f32x2(f32x2(x, y), f2), a, b);
  return pack2<kBF16>(a, b);
}

// One work item's geometry, derived identically by every role. An item is
// (sequence, pair of 128-row Q tiles, kv head); Q tile w holds tokens
// tok0 + w BQ .. tok0 + (w + 1) BQ - 1.
struct TcItem {
  int seq, h, s0, T, tok0, n_k, jlast, vlim, q_base;
  int n_w[kQTiles];  // K tiles Q tile w needs (0: the tile holds no token)
};

__device__ __forceinline__ TcItem tc_item(const TcParams& p, const int* tile_cum, int total_tiles, int item, int BQ) {
  TcItem it;
  it.h = item % p.hkv;
  const int gt = total_tiles - 1 - item / p.hkv;  // heavy tiles (last of a sequence) first
  int lo = 0, hi = p.n_seqs - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (tile_cum[mid] <= gt) lo = mid; else hi = mid - 1;
  }
  it.seq = lo;
  const int pair = gt - tile_cum[lo];
  it.T = tc_seq_tokens(p, it.seq, &it.s0, false);
  it.tok0 = pair * kQTiles * BQ;
  int key_last = 0;
#pragma unroll
  for (int w = 0; w < kQTiles; ++w) {
    const int t_lo = it.tok0 + w * BQ;
    if (t_lo < it.T) {
      key_last = it.s0 + min(it.T, t_lo + BQ) - 1;  // last key a row of this tile sees
      it.n_w[w] = key_last / kKeysTc + 1;
    } else {
      it.n_w[w] = 0;
    }
  }
  it.n_k = it.n_w[0] > it.n_w[1] ? it.n_w[0] : it.n_w[1];
  it.jlast = key_last / SCKV_PAGE_TOKENS;  // last page of the item (the last live tile's)
  it.vlim = min(it.s0 + it.T, (it.jlast + 1) * SCKV_PAGE_TOKENS);  // V rows at or past this key get zeroed
  it.q_base = __ldg(p.cu_q + it.seq);
  return it;
}

// 3-D tiled TMA load; coordinates (dim, head, token).
__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap* map, int x, int y, int z,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
      "[%5];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
      : "memory");
}

// Persistent, one CTA per SM: each CTA claims items from the launch's work
// counter (one of the pool's, taken round-robin per launch and zeroed just
// before it, so launches on other streams use other counters), heaviest-first
// within each sequence, until they run out. K/V tiles of all its items are
// numbered by one running counter (ring slot g % 4), and each softmax
// warpgroup numbers its own S tiles by another (S / P buffer g & 1), which
// fixes every barrier's phase.
template <int KVDT>
__global__ void __launch_bounds__(kThreadsTc, 1)
    prefill_tc_kernel(const TcParams p, const __grid_constant__ CUtensorMap tmap,
                      const __grid_constant__ CUtensorMap qmap) {
  using C = TcCfg<KVDT>;
  constexpr bool kBF16 = C::kBF16;
  constexpr int kStagesTc = C::kStages;
  constexpr int kOffK = C::kOffK, kOffV = C::kOffV, kOffBar = C::kOffBar, kNumBars = C::kNumBars;
  constexpr int kOffItemRing = C::kOffItemRing, kOffTmemSlot = C::kOffTmemSlot, kOffAbort = C::kOffAbort;
  constexpr int kOffPartial = C::kOffPartial, kOffTileCum = C::kOffTileCum;
  extern __shared__ __align__(16) uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(base + kOffBar);
  uint64_t* k_full = bars;                      // [S] K tile landed (two producer warps' TMA)
  uint64_t* k_empty = bars + kStagesTc;         // [S] every S product of the K tile finished (commit)
  uint64_t* v_full = bars + 2 * kStagesTc;      // [S] V tile landed
  uint64_t* v_empty = bars + 3 * kStagesTc;     // [S] every PV product of the V tile finished (commit)
  uint64_t* s_full = bars + 4 * kStagesTc;      // [w][2] S of warpgroup w's tile in TMEM (commit)
  uint64_t* p_full = s_full + 4;                // [w][2] P of warpgroup w's tile in TMEM (one arrival per warp)
  // [w][2] PV of warpgroup w's tile g finished (commit to pv_done[w][g & 1]).
  // A softmax thread waits for PV(g) only after S(g) (epilogue) or S(g + 1)
  // (O rescale) landed; that commit covers every MMA issued before it,
  // PV(g - 2) included, and PV(g + 2) cannot start before this thread writes
  // P(g + 2). So the barrier is at PV(g)'s phase or one past it and the
  // parity wait is unambiguous however rarely the thread waits on it.
  uint64_t* pv_done = p_full + 4;
  uint64_t* o_empty = pv_done + 4;              // [w] warpgroup w's O was read out (one arrival per warp)
  uint64_t* q_full = o_empty + 2;               // Q of the item in shared memory (TMA, or 256 softmax threads)
  uint64_t* q_empty = q_full + 1;               // every S of the item finished (commit): Q may be replaced
  uint64_t* mma_done = q_full + 2;              // every issued MMA finished (drain)
  // [4] item k's index is in item_ring[k & 3] (warp 0). The producers run at
  // most two items ahead of the softmax warps (Q of item k + 1 waits for all
  // S of item k, and S of item k past its second tile waits for the softmax
  // of item k), so a slot is never rewritten while unread.
  uint64_t* item_full = q_full + 3;
  // one-byte pools: [producer warp role 2 kv + part][2] staged page codes landed (TMA)
  uint64_t* stage_full = item_full + 4;
  // Q converted in place (q_tma 2; 64 threads of warps 14, 15): the MMAs wait for this instead of q_full
  uint64_t* q_conv = stage_full + (C::kB8 ? 8 : 0);
  volatile int* item_ring = reinterpret_cast<volatile int*>(base + kOffItemRing);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(base + kOffTmemSlot);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(base + kOffAbort);
  int* partial = reinterpret_cast<int*>(base + kOffPartial);
  int* tile_cum = reinterpret_cast<int*>(base + kOffTileCum);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int G = 1 << p.lg_g;
  const int BQ = kRowsTc >> p.lg_g;  // tokens per Q tile
  const int BQ2 = kQTiles * BQ;      // tokens per item

  // ---- Q-tile pairs per sequence, prefix-summed by the whole CTA
  {
    const int per = (p.n_seqs + kThreadsTc - 1) / kThreadsTc;
    const int s0 = threadIdx.x * per, s1 = min(p.n_seqs, s0 + per);
    int local = 0;
    for (int s = s0; s < s1; ++s) {
      int st;
      const int T = tc_seq_tokens(p, s, &st, blockIdx.x == 0);
      local += (T + BQ2 - 1) / BQ2;
    }
    partial[threadIdx.x] = local;
    if (threadIdx.x == 0) {
      for (int i = 0; i < kNumBars; ++i) {
        uint64_t* bar = &bars[i];
        uint32_t count = 1;
        if (bar >= k_full && bar < k_full + kStagesTc) count = 2;   // two K producer warps
        if (bar >= v_full && bar < v_full + kStagesTc) count = 2;   // two V producer warps
        if (bar >= p_full && bar < p_full + 4) count = kSoftmaxThreads / 32;   // one arrival per warp
        if (bar >= o_empty && bar < o_empty + 2) count = kSoftmaxThreads / 32;
        if (bar == q_full && !p.q_tma) count = kQTiles * kSoftmaxThreads;
        if (bar == q_conv) count = 2 * 32;
        mbar_init(bar, count);
      }
      *abort_flag = 0;
      fence_mbar_init();
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      int acc = 0;
      for (int i = 0; i < kThreadsTc; ++i) {
        const int v = partial[i];
        partial[i] = acc;
        acc += v;
      }
      tile_cum[0] = 0;
    }
    __syncthreads();
    int run = partial[threadIdx.x];
    for (int s = s0; s < s1; ++s) {
      int st;
      const int T = tc_seq_tokens(p, s, &st, false);
      run += (T + BQ2 - 1) / BQ2;
      tile_cum[s + 1] = run;
    }
    __syncthreads();
  }
  const int total_tiles = tile_cum[p.n_seqs];
  const int n_items = total_tiles * p.hkv;

  if (warp == kWarpMma) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (C::kB8 && (warp == kWarpK0 || warp == kWarpK1 || warp == kWarpV0 || warp == kWarpV1)) {
    // ------------------------------------------------------ producers, one-byte pools
    // Each warp stages its two pages of a tile by TMA (two tiles ahead) and
    // decodes them, all lanes, into the f16 ring in the UMMA K-major layout:
    // lane (r, hf) turns token row r's dims 64 hf .. 64 hf + 63 into f16
    // times the scale (FP8: the page-head's fp32 scale, applied in fp32;
    // int8: the token's fp16 scale, one exact f16 product as the reference's
    // dequantisation rounds it). The ring slot is full once both warps of a
    // tile (K or V) arrived.
    const int kv = (warp == kWarpV0 || warp == kWarpV1) ? 1 : 0;
    const int part = (warp == kWarpK1 || warp == kWarpV1) ? 1 : 0;  // pages 2 part, 2 part + 1
    const int role = 2 * kv + part;
    const bool leader = warp == kWarpK0;
    if (lane == 0) asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmap)) : "memory");
    if (lane == 0 && leader && p.q_tma)
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&qmap)) : "memory");
    const int64_t layer_base = (int64_t)p.layer * p.max_pages;
    uint64_t* fulls = kv ? v_full : k_full;
    uint64_t* empties = kv ? v_empty : k_empty;
    uint64_t* sfull = stage_full + 2 * role;
    uint8_t* stg = base + C::kOffStage + role * 2 * C::kStageSlot;
    const int r = lane >> 1, hf = lane & 1;
    // This lane's scales (int8: the token's fp16 value) of the tile decoded
    // next (scl_dec) and of the tile staged last (scl_new). Kept in named
    // registers, not an array indexed by the staging slot (that would live in
    // local memory, and storing a scale there waits for its global load).
    // A tile's scales are loaded after its copies are issued and moved into
    // scl_dec one tile later, so no copy issue waits on a scale load.
    float scl_dec0 = 0.f, scl_dec1 = 0.f, scl_new0 = 0.f, scl_new1 = 0.f;
    int g = 0;        // tiles of this warp's ring so far
    uint32_t sg = 0;  // staged tiles issued
    uint32_t sc = 0;  // staged tiles decoded
    int q_issued = 0;  // items whose Q the leader loaded by TMA
    bool aborted = false;
    for (int k = 0;; ++k) {
      int item;
      if (leader) {
        int claimed = 0;
        if (lane == 0) {
          // an index >= n_items tells every role to stop
          claimed = aborted ? n_items : (int)min((unsigned long long)n_items, atomicAdd(p.next_item, 1ULL));
          item_ring[k & 3] = claimed;
          mbar_arrive(&item_full[k & 3]);
        }
        item = __shfl_sync(0xffffffffu, claimed, 0);
      } else {
        const int ab = __shfl_sync(0xffffffffu, *abort_flag, 0);
        if (aborted || ab || !warp_wait(&item_full[k & 3], (k >> 2) & 1)) {
          aborted = true;
          break;
        }
        item = item_ring[k & 3];
      }
      if (item >= n_items) break;
      const TcItem it = tc_item(p, tile_cum, total_tiles, item, BQ);
      if (leader && p.q_tma) {
        // Q of the item by TMA once every S product of the previous item
        // (the only reader of the Q tiles) has finished
        int okq = 1;
        if (lane == 0) {
          if (k > 0 && (*abort_flag || !mbar_wait_bounded(q_empty, (k - 1) & 1, SCKV_WAIT_LIMIT_NS))) {
            okq = 0;
          } else {
            const int live = it.n_w[1] > 0 ? 2 : 1;
            mbar_arrive_expect_tx(q_full, (uint32_t)live * 2u * kQHalf);
            for (int w = 0; w < live; ++w) {
              const int tok = it.q_base + it.tok0 + w * BQ;
              tma_load_3d(smem_u32(base + w * kQTileBytes), &qmap, 0, it.h * G, tok, q_full);
              tma_load_3d(smem_u32(base + w * kQTileBytes + kQHalf), &qmap, 64, it.h * G, tok, q_full);
            }
            ++q_issued;
          }
        }
        if (!__shfl_sync(0xffffffffu, okq, 0)) {
          aborted = true;
          continue;  // publishes the stop marker next
        }
      }
      const int32_t* bt_row = p.block_table + (int64_t)it.seq * p.bt_stride;
      // this warp's page ids of a local tile (0 past the item's last page)
      auto fetch_ids = [&](int j, int32_t& a, int32_t& b) {
        const int first = j * kPagesTc + 2 * part;
        a = first <= it.jlast ? __ldg(bt_row + first) : 0;
        b = first + 1 <= it.jlast ? __ldg(bt_row + first + 1) : 0;
      };
      auto scale_of = [&](int32_t page) -> float {
        const int64_t sidx = ((layer_base + page) * 2 + kv) * p.hkv + it.h;
        if (KVDT == SCKV_DTYPE_INT8)
          return __half2float(__ldg(reinterpret_cast<const __half*>(p.kv_scales) + sidx * 16 + r));
        return __ldg(reinterpret_cast<const float*>(p.kv_scales) + sidx);
      };
      int32_t nid0 = 0, nid1 = 0;  // page ids of the next tile to stage (fetched one tile ahead)
      fetch_ids(0, nid0, nid1);
      auto issue = [&](int j) {
        const int first = j * kPagesTc + 2 * part;
        const int np = max(0, min(2, it.jlast + 1 - first));
        const uint32_t sl = sg & 1;
        int32_t pg0 = nid0, pg1 = nid1;
        if (j + 1 < it.n_k) fetch_ids(j + 1, nid0, nid1);
        if (np > 0 && (pg0 < 0 || pg0 >= p.max_pages)) {
          if (lane == 0) sckv_report(p.status, SCKV_ERR_BOUNDS, pg0, KID_PREFILL);
          pg0 = 0;
        }
        if (np > 1 && (pg1 < 0 || pg1 >= p.max_pages)) {
          if (lane == 0) sckv_report(p.status, SCKV_ERR_BOUNDS, pg1, KID_PREFILL);
          pg1 = 0;
        }
        if (lane == 0) {
          mbar_arrive_expect_tx(&sfull[sl], (uint32_t)np * C::kPageBox);
          if (np > 0)
            tma_load_5d(smem_u32(stg + sl * C::kStageSlot), &tmap, 0, 0, it.h, kv, (int)(layer_base + pg0),
                        &sfull[sl]);
          if (np > 1)
            tma_load_5d(smem_u32(stg + sl * C::kStageSlot + C::kPageBox), &tmap, 0, 0, it.h, kv,
                        (int)(layer_base + pg1), &sfull[sl]);
        }
        scl_dec0 = scl_new0;
        scl_dec1 = scl_new1;
        scl_new0 = np > 0 ? scale_of(pg0) : 0.f;
        scl_new1 = np > 1 ? scale_of(pg1) : 0.f;
        ++sg;
      };
      if (it.n_k > 0) issue(0);
      if (it.n_k > 1) issue(1);
      if (it.n_k == 1) {
        scl_dec0 = scl_new0;
        scl_dec1 = scl_new1;
      }
      for (int j = 0; j < it.n_k; ++j) {
        const int gt = g + j;
        const int st = gt % kStagesTc;
        if (gt >= kStagesTc && !warp_wait(&empties[st], ((gt / kStagesTc) - 1) & 1)) {
          aborted = true;
          break;
        }
        const uint32_t sl = sc & 1;
        if (!warp_wait(&sfull[sl], (sc >> 1) & 1)) {
          aborted = true;
          break;
        }
        const int first = j * kPagesTc + 2 * part;
        const int np = max(0, min(2, it.jlast + 1 - first));
        uint8_t* slot = base + (kv ? kOffV : kOffK) + st * kSlotBytes;
#pragma unroll
        for (int i = 0; i < 2; ++i) {
          if (i >= np) break;
          const uint8_t* src = stg + sl * C::kStageSlot + i * C::kPageBox + r * 128;
          uint8_t* dst = slot + hf * kTileHalf + (2 * part + i) * 2048 + r * 128;
          const float sv = i == 0 ? scl_dec0 : scl_dec1;
          const __half2 s2 = __float2half2_rn(sv);  // int8: the stored fp16 scale, exact
          const uint64_t sv2 = f32x2(sv, sv);        // FP8: the fp32 scale, one packed multiply per pair
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            // 16 codes: dims 64 hf + 16 c .. + 15 (128-byte swizzle: chunk ^ row)
            const uint4 w = *reinterpret_cast<const uint4*>(src + (((4 * hf + c) ^ (r & 7)) << 4));
            const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
            uint32_t o[8];
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              uint32_t lo, hi;
              cvt_b8x4<KVDT>(ws[q], lo, hi);
              if (KVDT == SCKV_DTYPE_INT8) {
                const __half2 a = __hmul2(*reinterpret_cast<const __half2*>(&lo), s2);
                const __half2 b = __hmul2(*reinterpret_cast<const __half2*>(&hi), s2);
                lo = *reinterpret_cast<const uint32_t*>(&a);
                hi = *reinterpret_cast<const uint32_t*>(&b);
              } else {
                const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&lo));
                const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&hi));
                lo = mul_pack2<false>(a.x, a.y, sv2);
                hi = mul_pack2<false>(b.x, b.y, sv2);
              }
              o[2 * q] = lo;
              o[2 * q + 1] = hi;
            }
            *reinterpret_cast<uint4*>(dst + (((2 * c) ^ (r & 7)) << 4)) = make_uint4(o[0], o[1], o[2], o[3]);
            *reinterpret_cast<uint4*>(dst + (((2 * c + 1) ^ (r & 7)) << 4)) = make_uint4(o[4], o[5], o[6], o[7]);
          }
        }
        // the decoded tile is read by the tensor cores (async proxy)
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&fulls[st]);
        ++sc;
        if (j + 2 < it.n_k) {
          issue(j + 2);
        } else {
          scl_dec0 = scl_new0;
          scl_dec1 = scl_new1;
        }
      }
      if (aborted && !leader) break;
      g += it.n_k;
    }
    if (aborted && lane == 0) {
      if (!*abort_flag) sckv_report(p.status, SCKV_ERR_TIMEOUT, blockIdx.x, KID_PREFILL);
      *abort_flag = 1;
    }
    // staged copies (and Q copies) still in flight land before the CTA retires
    if (lane == 0)
      for (uint32_t t = sc; t < sg; ++t) mbar_wait_bounded(&sfull[t & 1], (t >> 1) & 1, SCKV_WAIT_LIMIT_NS);
    if (lane == 0 && q_issued > 0) mbar_wait_bounded(q_full, (q_issued - 1) & 1, SCKV_WAIT_LIMIT_NS);
  } else if (warp == kWarpK0 || warp == kWarpK1 || warp == kWarpV0 || warp == kWarpV1) {
    // ------------------------------------------------------------ producers
    // one TMA issue holds its warp ~0.1 us, so K and V each get two warps,
    // each copying two of a tile's four pages
    if (lane == 0) {
      const int kv = (warp == kWarpV0 || warp == kWarpV1) ? 1 : 0;
      const int part = (warp == kWarpK1 || warp == kWarpV1) ? 1 : 0;  // pages 2 part, 2 part + 1
      const bool leader = warp == kWarpK0;
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmap)) : "memory");
      if (leader && p.q_tma)
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&qmap)) : "memory");
      const int64_t layer_base = (int64_t)p.layer * p.max_pages;
      uint64_t* fulls = kv ? v_full : k_full;
      uint64_t* empties = kv ? v_empty : k_empty;
      int g = 0, q_issued = 0;
      bool aborted = false;
      for (int k = 0;; ++k) {
        int item;
        if (leader) {
          // claim the next item; an index >= n_items tells every role to stop
          item = aborted ? n_items : (int)min((unsigned long long)n_items, atomicAdd(p.next_item, 1ULL));
          item_ring[k & 3] = item;
          mbar_arrive(&item_full[k & 3]);
        } else {
          if (aborted || *abort_flag || !mbar_wait_bounded(&item_full[k & 3], (k >> 2) & 1, SCKV_WAIT_LIMIT_NS)) {
            aborted = true;
            break;
          }
          item = item_ring[k & 3];
        }
        if (item >= n_items) break;
        const TcItem it = tc_item(p, tile_cum, total_tiles, item, BQ);
        if (leader && p.q_tma) {
          if (k > 0 && (*abort_flag || !mbar_wait_bounded(q_empty, (k - 1) & 1, SCKV_WAIT_LIMIT_NS))) {
            aborted = true;
            continue;  // publishes the stop marker next
          }
          const int live = it.n_w[1] > 0 ? 2 : 1;
          mbar_arrive_expect_tx(q_full, (uint32_t)live * 2u * kQHalf);
          for (int w = 0; w < live; ++w) {
            const int tok = it.q_base + it.tok0 + w * BQ;
            tma_load_3d(smem_u32(base + w * kQTileBytes), &qmap, 0, it.h * G, tok, q_full);
            tma_load_3d(smem_u32(base + w * kQTileBytes + kQHalf), &qmap, 64, it.h * G, tok, q_full);
          }
          ++q_issued;
        }
        const int32_t* bt_row = p.block_table + (int64_t)it.seq * p.bt_stride;
        // this warp's two page ids of local tile j, fetched one tile ahead
        // so their load latency overlaps the copies being issued
        auto fetch_ids = [&](int j, int (&ids)[2]) {
#pragma unroll
          for (int i = 0; i < 2; ++i) {
            const int blk = j * kPagesTc + 2 * part + i;
            ids[i] = blk <= it.jlast ? __ldg(bt_row + blk) : 0;
          }
        };
        int ids_next[2], ids_cur[2];
        fetch_ids(0, ids_next);
        for (int j = 0; j < it.n_k; ++j) {
          ids_cur[0] = ids_next[0];
          ids_cur[1] = ids_next[1];
          if (j + 1 < it.n_k) fetch_ids(j + 1, ids_next);
          const int gt = g + j;
          const int st = gt % kStagesTc;
          if (gt >= kStagesTc &&
              (*abort_flag ||
               !mbar_wait_bounded(&empties[st], ((gt / kStagesTc) - 1) & 1, SCKV_WAIT_LIMIT_NS))) {
            aborted = true;
            break;
          }
          // pages of the tile this warp copies (the last tile may have fewer)
          const int first = j * kPagesTc + 2 * part;
          const int np = max(0, min(2, it.jlast + 1 - first));
          const uint32_t slot = smem_u32(base + (kv ? kOffV : kOffK) + st * kSlotBytes);
          mbar_arrive_expect_tx(&fulls[st], (uint32_t)np * 2u * 2048u);
          for (int i = 0; i < np; ++i) {
            int32_t page = ids_cur[i];
            if (page < 0 || page >= p.max_pages) {
              sckv_report(p.status, SCKV_ERR_BOUNDS, page, KID_PREFILL);
              page = 0;
            }
            const int slab = (int)(layer_base + page);
            const int pg = 2 * part + i;
            tma_load_5d(slot + pg * 2048, &tmap, 0, 0, it.h, kv, slab, &fulls[st]);
            tma_load_5d(slot + kTileHalf + pg * 2048, &tmap, 64, 0, it.h, kv, slab, &fulls[st]);
          }
        }
        if (aborted && !leader) break;
        g += it.n_k;
      }
      if (aborted) {
        if (!*abort_flag) sckv_report(p.status, SCKV_ERR_TIMEOUT, blockIdx.x, KID_PREFILL);
        *abort_flag = 1;
      }
      // nothing of ours may still be landing when the CTA retires
      for (int t = g > kStagesTc ? g - kStagesTc : 0; t < g; ++t)
        mbar_wait_bounded(&fulls[t % kStagesTc], (t / kStagesTc) & 1, SCKV_WAIT_LIMIT_NS);
      if (q_issued > 0) mbar_wait_bounded(q_full, (q_issued - 1) & 1, SCKV_WAIT_LIMIT_NS);
    }
  } else if (warp == kWarpMma && lane == 0) {
    // ------------------------------------------------------------ MMA issuer
    // One thread issues every MMA and commit and does its own bounded waits:
    // warp-wide waits and the reconvergence around single-lane issues cost
    // more than the issues themselves (lanes 1-31 go straight to the final
    // barrier and join the tensor-memory release there).
    auto wait1 = [&](uint64_t* bar, uint32_t parity) -> bool {
      return mbar_wait_bounded(bar, parity, SCKV_WAIT_LIMIT_NS);
    };
    constexpr uint32_t kIdescS = instr_desc_f16(kBF16, kKeysTc, false);
    constexpr uint32_t kIdescPV = instr_desc_f16(kBF16, kHDim, true);
    // descriptors of the first Q tile, K slot and V slot; every operand of
    // an MMA is one of them advanced by a byte offset
    const uint64_t q_desc0 = smem_desc_sw128(smem_u32(base), 16, 1024);
    const uint64_t k_desc0 = smem_desc_sw128(smem_u32(base + kOffK), 16, 1024);
    const uint64_t v_desc0 = smem_desc_sw128(smem_u32(base + kOffV), kTileHalf, 1024);
    bool ok = true;
    int gk = 0;                     // K/V tiles issued
    int gs[kQTiles] = {0, 0};       // S tiles issued per warpgroup
    int items_w[kQTiles] = {0, 0};  // items with a live Q tile w so far
    // PV of local K/V tile i (global gi): O[w] (+)= P[w] . V for each live Q tile
    auto issue_pv = [&](const TcItem& it, int gi, int i, const int (&gw0)[kQTiles]) -> bool {
      const int st = gi % kStagesTc;
      if (!wait1(&v_full[st], (gi / kStagesTc) & 1)) return false;
      tc_fence_after();
      uint8_t* vslot = base + kOffV + st * kSlotBytes;
      const int key0 = i * kKeysTc;
      if (key0 + kKeysTc > it.vlim) {
        // zero the V rows of keys >= vlim (both 64-dim halves): their slots
        // were never written or hold an older tile
        const int r0 = max(0, it.vlim - key0);
        const int n16 = (kKeysTc - r0) * 8;  // 16-byte chunks per half
        for (int c = 0; c < 2 * n16; ++c) {
          const int half = c / n16, rc = c - half * n16;
          *reinterpret_cast<uint4*>(vslot + half * kTileHalf + (r0 + (rc >> 3)) * 128 + (rc & 7) * 16) =
              make_uint4(0u, 0u, 0u, 0u);
        }
        fence_proxy_async_smem();
      }
      const uint64_t v_desc = desc_advance(v_desc0, (uint32_t)(st * kSlotBytes));
      bool live[kQTiles];
      int bw[kQTiles];
#pragma unroll
      for (int w = 0; w < kQTiles; ++w) {
        live[w] = i < it.n_w[w];
        const int gw = gw0[w] + i;
        bw[w] = gw & 1;
        if (!live[w]) continue;
        if (!wait1(&p_full[w * 2 + bw[w]], (gw >> 1) & 1)) return false;
        if (i == 0 && items_w[w] > 0) {
          // O[w] still holds this warpgroup's previous item until its
          // epilogue has read it
          if (!wait1(&o_empty[w], (items_w[w] - 1) & 1)) return false;
        }
      }
      tc_fence_after();
      {
        // the two Q tiles' accumulation chains interleave, so each MMA's
        // dependency on the previous one into the same O overlaps the other's
#pragma unroll
        for (int pg = 0; pg < kPagesTc; ++pg) {
          // B = V rows of page pg: N = 128 dims in two 64-dim halves (LBO),
          // K = 16 keys in two groups of 8 rows (SBO)
          const uint64_t bdesc = desc_advance(v_desc, (uint32_t)(pg * 2048));
#pragma unroll
          for (int w = 0; w < kQTiles; ++w) {
            if (!live[w]) continue;
            const uint32_t s_col = tmem + kColS + (uint32_t)((2 * w + bw[w]) * kKeysTc);
            const uint32_t o_col = tmem + kColO + (uint32_t)(w * kHDim);
            umma_ts(o_col, s_col + (uint32_t)(pg * 8), bdesc, kIdescPV, (i > 0 || pg > 0) ? 1u : 0u);
            if (kBF16) umma_ts(o_col, s_col + (uint32_t)(pg * 8 + 32), bdesc, kIdescPV, 1u);
          }
        }
#pragma unroll
        for (int w = 0; w < kQTiles; ++w)
          if (live[w]) umma_commit(&pv_done[w * 2 + bw[w]]);
      }
      umma_commit(&v_empty[st]);
      return true;
    };
    for (int k = 0; ok; ++k) {
      if (*abort_flag || !wait1(&item_full[k & 3], (k >> 2) & 1)) {
        ok = false;
        break;
      }
      const int item = item_ring[k & 3];
      if (item >= n_items) break;
      const TcItem it = tc_item(p, tile_cum, total_tiles, item, BQ);
      if (*abort_flag || !wait1(p.q_tma == 2 ? q_conv : q_full, k & 1)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const int gw0[kQTiles] = {gs[0], gs[1]};
      for (int j = 0; j < it.n_k; ++j) {
        const int gj = gk + j;
        const int st = gj % kStagesTc;
        if (*abort_flag || !wait1(&k_full[st], (gj / kStagesTc) & 1)) {
          ok = false;
          break;
        }
        tc_fence_after();
        {
          const uint64_t k_desc = desc_advance(k_desc0, (uint32_t)(st * kSlotBytes));
          // the two Q tiles' 8-step chains interleave: an N = 64 product is
          // short, so back-to-back MMAs into one accumulator would each wait
          // for the previous one
#pragma unroll
          for (int ks = 0; ks < 8; ++ks) {
            const int half = ks >> 2, kk = ks & 3;
            const uint64_t bdesc = desc_advance(k_desc, (uint32_t)(half * kTileHalf + kk * 32));
#pragma unroll
            for (int w = 0; w < kQTiles; ++w) {
              if (j >= it.n_w[w]) continue;
              const int b = (gw0[w] + j) & 1;
              const uint64_t adesc = desc_advance(q_desc0, (uint32_t)(w * kQTileBytes + half * kQHalf + kk * 32));
              umma_ss(tmem + kColS + (uint32_t)((2 * w + b) * kKeysTc), adesc, bdesc, kIdescS, ks > 0 ? 1u : 0u);
            }
          }
#pragma unroll
          for (int w = 0; w < kQTiles; ++w)
            if (j < it.n_w[w]) umma_commit(&s_full[w * 2 + ((gw0[w] + j) & 1)]);
          umma_commit(&k_empty[st]);
          if (j == it.n_k - 1) umma_commit(q_empty);  // Q no longer read once these S are done
        }
        if (j >= 1 && !issue_pv(it, gj - 1, j - 1, gw0)) {
          ok = false;
          break;
        }
      }
      if (!ok || !issue_pv(it, gk + it.n_k - 1, it.n_k - 1, gw0)) {
        ok = false;
        break;
      }
      gk += it.n_k;
#pragma unroll
      for (int w = 0; w < kQTiles; ++w) {
        gs[w] += it.n_w[w];
        if (it.n_w[w] > 0) ++items_w[w];
      }
    }
    if (!ok) {
      if (!*abort_flag) sckv_report(p.status, SCKV_ERR_TIMEOUT, blockIdx.x, KID_PREFILL);
      *abort_flag = 1;
    }
    // drain: every MMA issued above has finished before TMEM is released
    umma_commit(mma_done);
    wait1(mma_done, 0);
  } else if (warp >= 4 && warp < 12) {
    // ------------------------------------------------------------ softmax
    const int w = (warp - 4) >> 2;       // Q tile of this warpgroup
    const int quad = warp & 3;           // TMEM lanes 32 quad .. 32 quad + 31
    const int row = quad * 32 + lane;    // query row = TMEM lane
    const uint32_t t_row = tmem + ((uint32_t)(quad * 32) << 16);
    const uint32_t col_s = kColS + (uint32_t)(2 * w * kKeysTc);
    const uint32_t col_o = kColO + (uint32_t)(w * kHDim);
    uint64_t* my_s_full = s_full + 2 * w;
    uint64_t* my_p_full = p_full + 2 * w;
    uint64_t* my_pv_done = pv_done + 2 * w;
    uint8_t* q_tile = base + w * kQTileBytes;
    bool ok = true;
    int g = 0;
    for (int k = 0; ok; ++k) {
      if (*abort_flag || !warp_wait(&item_full[k & 3], (k >> 2) & 1)) {
        ok = false;
        break;
      }
      const int item = item_ring[k & 3];
      if (item >= n_items) break;
      const TcItem it = tc_item(p, tile_cum, total_tiles, item, BQ);
      const int rtok = it.tok0 + w * BQ + (row >> p.lg_g);
      const int rhead = it.h * G + (row & (G - 1));
      const bool valid = rtok < it.T;
      const int lim = valid ? it.s0 + rtok : -1;  // last key this row sees
      const int tile_lim = it.s0 + it.tok0 + w * BQ;  // keys up to here are seen by every row of the tile
      if (!p.q_tma) {
        // Q row -> shared memory, 128-byte swizzled K-major (the layout a TMA
        // copy with SWIZZLE_128B produces). This warpgroup's previous S
        // products are all finished: it waited for every one of them.
        const int64_t qoff = ((int64_t)(it.q_base + rtok) * p.hq + rhead) * kHDim;
#pragma unroll
        for (int c = 0; c < 16; ++c) {
          const int half = c >> 3, ch = c & 7;
          const uint4 v = valid ? load_q8<kBF16>(p.q, qoff + c * 8, p.q_dtype) : make_uint4(0u, 0u, 0u, 0u);
          *reinterpret_cast<uint4*>(q_tile + half * kQHalf + row * 128 + ((ch ^ (row & 7)) << 4)) = v;
        }
        fence_proxy_async_smem();
        mbar_arrive(q_full);
      }
      const int n = it.n_w[w];
      if (n == 0) continue;  // no token of this item falls in this Q tile
      float m = -INFINITY, l = 0.f;
      for (int j = 0; j < n; ++j) {
        const int gj = g + j;
        const int b = gj & 1;
        if (*abort_flag || !warp_wait(&my_s_full[b], (gj >> 1) & 1)) {
          ok = false;
          break;
        }
        tc_fence_after();
        float sv[kKeysTc];
        {
          uint32_t r0[32], r1[32];
          tmem_ld32(t_row + col_s + b * kKeysTc, r0);
          tmem_ld32(t_row + col_s + b * kKeysTc + 32, r1);
          tc_wait_ld();
#pragma unroll
          for (int c = 0; c < 32; ++c) {
            sv[c] = __uint_as_float(r0[c]);
            sv[32 + c] = __uint_as_float(r1[c]);
          }
        }
        // row max of the raw scores (the scale is positive); tiles every row
        // of the Q tile sees in full skip the causal mask
        const int key0 = j * kKeysTc;
        if (key0 + kKeysTc - 1 > tile_lim) {
#pragma unroll
          for (int c = 0; c < kKeysTc; ++c) sv[c] = (key0 + c <= lim) ? sv[c] : -INFINITY;
        }
        // (one max loop for both cases: the kernel's roles share one
        // instruction cache, so duplicated unrolled code costs)
        float pm = -INFINITY;
#pragma unroll
        for (int c = 0; c < kKeysTc; c += 2) pm = fmax3(pm, sv[c], sv[c + 1]);
        pm *= p.scale_log2;
        // stale running max (log2 units): move it only when a tile's max
        // exceeds it by more than 8
        float alpha = 1.f;
        bool rescale = false;
        if (pm > m + 8.f) {
          if (m != -INFINITY) {
            alpha = ex2_approx(m - pm);
            rescale = true;
          }
          m = pm;
          l *= alpha;
        }
        if (__any_sync(0xffffffffu, rescale) && j > 0) {
          // O holds PV of tiles 0..j-1 of this Q tile: wait for the last, then
          // scale this warp's rows
          if (!warp_wait(&my_pv_done[(gj - 1) & 1], ((gj - 1) >> 1) & 1)) {
            ok = false;
            break;
          }
          tc_fence_after();
#pragma unroll 1
          for (int cc = 0; cc < 4; ++cc) {
            uint32_t r[32];
            tmem_ld32(t_row + col_o + cc * 32, r);
            tc_wait_ld();
#pragma unroll
            for (int c = 0; c < 32; ++c) r[c] = __float_as_uint(__uint_as_float(r[c]) * alpha);
            tmem_st32(t_row + col_o + cc * 32, r);
          }
          tc_wait_st();
        }
        // P = 2^(s - m), packed two keys per column over S's first columns
        {
          uint32_t ph[32], plo[32];
          // a row that sees no key yet (m = -inf) has every score -inf: 2^-inf = 0
          const float mm = (m == -INFINITY) ? 0.f : m;
          // per key pair: one packed FMA, two exponentials, one packed add
          // into the (even, odd) sums
          const uint64_t scale2 = f32x2(p.scale_log2, p.scale_log2), negm2 = f32x2(-mm, -mm);
          const uint64_t minus1 = f32x2(-1.f, -1.f);
          uint64_t ls2 = f32x2(0.f, 0.f);
#pragma unroll
          for (int c = 0; c < 32; ++c) {
            float x0, x1;
            f32x2_split(fma_f32x2(f32x2(sv[2 * c], sv[2 * c + 1]), scale2, negm2), x0, x1);
            const float p0 = ex2_approx(x0);
            const float p1 = ex2_approx(x1);
            ls2 = add_f32x2(ls2, f32x2(p0, p1));
            ph[c] = pack2<kBF16>(p0, p1);
            if (kBF16) {
              // lo = p - bf16(p), exact: the hi pair widened back from ph by
              // bit operations, then one packed fma(hi, -1, p)
              const uint64_t hi2 = f32x2(__uint_as_float(ph[c] << 16), __uint_as_float(ph[c] & 0xFFFF0000u));
              float l0, l1;
              f32x2_split(fma_f32x2(hi2, minus1, f32x2(p0, p1)), l0, l1);
              plo[c] = pack2<true>(l0, l1);
            }
          }
          float ls0, ls1;
          f32x2_split(ls2, ls0, ls1);
          tmem_st32(t_row + col_s + b * kKeysTc, ph);
          if (kBF16) tmem_st32(t_row + col_s + b * kKeysTc + 32, plo);
          l += ls0 + ls1;
          tc_wait_st();
        }
        // every thread's P stores completed (wait::st) and are ordered before
        // the warp's sync; one arrival per warp releases them to the MMA thread
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&my_p_full[b]);
      }
      if (!ok) break;
      // ---- epilogue: O / l for this thread's row, once the tile's last PV finished
      const int glast = g + n - 1;
      if (!warp_wait(&my_pv_done[glast & 1], (glast >> 1) & 1)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const float inv = (l > 0.f) ? 1.f / l : 0.f;
      const uint64_t inv2 = f32x2(inv, inv);
      const int64_t obase = ((int64_t)(it.q_base + rtok) * p.hq + rhead) * kHDim;
#pragma unroll 1
      for (int cc = 0; cc < 4; ++cc) {
        uint32_t r[32];
        tmem_ld32(t_row + col_o + cc * 32, r);
        tc_wait_ld();
        if (valid) {
          if (p.out_dtype == SCKV_DTYPE_F32) {
            float* o = reinterpret_cast<float*>(p.out) + obase + cc * 32;
#pragma unroll
            for (int c = 0; c < 32; c += 4)
              *reinterpret_cast<float4*>(o + c) =
                  make_float4(__uint_as_float(r[c]) * inv, __uint_as_float(r[c + 1]) * inv,
                              __uint_as_float(r[c + 2]) * inv, __uint_as_float(r[c + 3]) * inv);
          } else {
            const bool obf = p.out_dtype == SCKV_DTYPE_BF16;
            uint16_t* o = reinterpret_cast<uint16_t*>(p.out) + obase + cc * 32;
#pragma unroll
            for (int c = 0; c < 32; c += 8) {
              uint4 wv;
              uint32_t* wp = &wv.x;
#pragma unroll
              for (int kk = 0; kk < 4; ++kk) {
                const float a = __uint_as_float(r[c + 2 * kk]), bb = __uint_as_float(r[c + 2 * kk + 1]);
                wp[kk] = obf ? mul_pack2<true>(a, bb, inv2) : mul_pack2<false>(a, bb, inv2);
              }
              *reinterpret_cast<uint4*>(o + c) = wv;
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&o_empty[w]);  // O[w] may be overwritten by the next item's PV
      g += n;
    }
    if (!ok) {
      if (lane == 0 && !*abort_flag) sckv_report(p.status, SCKV_ERR_TIMEOUT, blockIdx.x, KID_PREFILL);
      if (lane == 0) *abort_flag = 1;
    }
  } else if (warp >= 14 && p.q_tma == 2) {
    // ------------------------------------------------------------ Q conversion
    // Q arrived by TMA in the other 16-bit type: convert both Q tiles in
    // place, 16-byte chunk by chunk (the 128-byte swizzle only permutes
    // chunks), while the softmax warps finish the previous item. A tile
    // with no token of the item holds stale values that no MMA reads.
    const int ct = threadIdx.x - 14 * 32;  // 0..63
    bool ok = true;
    for (int k = 0; ok; ++k) {
      if (*abort_flag || !warp_wait(&item_full[k & 3], (k >> 2) & 1)) {
        ok = false;
        break;
      }
      if (item_ring[k & 3] >= n_items) break;
      if (*abort_flag || !warp_wait(q_full, k & 1)) {
        ok = false;
        break;
      }
      for (int c = ct; c < kQTiles * kQTileBytes / 16; c += 2 * 32) {
        uint4* chunk = reinterpret_cast<uint4*>(base + c * 16);
        const uint4 raw = *chunk;
        const uint32_t w4[4] = {raw.x, raw.y, raw.z, raw.w};
        uint32_t o4[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          float lo, hi;
          if (kBF16) {  // f16 q, bf16 MMA (sckv_prefill_attn takes bf16 q for bf16 pools today)
            const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w4[i]));
            lo = f.x;
            hi = f.y;
          } else {  // bf16 q, f16 MMA
            lo = __uint_as_float(w4[i] << 16);
            hi = __uint_as_float(w4[i] & 0xFFFF0000u);
          }
          o4[i] = pack2<kBF16>(lo, hi);
        }
        *chunk = make_uint4(o4[0], o4[1], o4[2], o4[3]);
      }
      // the converted tiles are read by the tensor cores (async proxy)
      fence_proxy_async_smem();
      mbar_arrive(q_conv);
    }
    if (!ok) {
      if (lane == 0 && !*abort_flag) sckv_report(p.status, SCKV_ERR_TIMEOUT, blockIdx.x, KID_PREFILL);
      if (lane == 0) *abort_flag = 1;
    }
  }
  // the MMA warp's lane 0 rejoins lanes 1-31 (which skipped the issuer loop)
  // so the block barrier and the tensor-memory release run converged
  if (warp == kWarpMma) __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (warp == kWarpMma) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
  }
}

template <int KVDT>
int launch_tc(const sckv_pool* pool, const TcParams& prm, int max_items, const CUtensorMap& qmap,
              cudaStream_t stream) {
  auto kern = prefill_tc_kernel<KVDT>;
  sckv_pool* mp = const_cast<sckv_pool*>(pool);  // the map is a cache inside the handle
  int rc = ensure_tmap(pool, 1, mp->tmap_kv2, &mp->tmap2_ready, 1);
  if (rc != SCKV_OK) return rc;
  const int smem = TcCfg<KVDT>::kFixedSmem + 4 * (prm.n_seqs + 1);
  if (smem > 227 * 1024) return SCKV_ERR_UNSUPPORTED;
  SCKV_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
  SCKV_CUDA_CHECK(cudaMemsetAsync(prm.next_item, 0, sizeof(unsigned long long), stream));
  // one CTA per SM: 512 TMEM columns are the whole of an SM's tensor memory
  int grid = pool->num_sms;
  if (grid > max_items) grid = max_items;
  const CUtensorMap* kv_map = reinterpret_cast<const CUtensorMap*>(pool->tmap_kv2);
  kern<<<grid, kThreadsTc, smem, stream>>>(prm, *kv_map, prm.q_tma ? qmap : *kv_map);
  SCKV_LAUNCH_CHECK();
  return SCKV_OK;
}

}  // namespace

namespace sckv_detail {

// Tensor-memory prefill for every pool type. Returns SCKV_ERR_UNSUPPORTED
// for combinations it does not build (the caller then tries prefill_kernel).
int launch_prefill_tc(const sckv_pool* pool, int layer, const void* q, int q_dtype, int num_q_heads, int n_seqs,
                      int n_tokens, const int32_t* cu_q, const int32_t* start_pos, const int32_t* block_table,
                      int64_t bt_stride, int max_blocks, float scale, void* out, int out_dtype, int lg_g,
                      cudaStream_t stream) {
  if (pool->head_dim != kHDim || n_seqs > 16384 || !(scale > 0.f)) return SCKV_ERR_UNSUPPORTED;
  const bool byte_pool = pool->kv_dtype == SCKV_DTYPE_FP8_E4M3 || pool->kv_dtype == SCKV_DTYPE_INT8;
  if (byte_pool && pool->scales == nullptr) return SCKV_ERR_UNSUPPORTED;
  if (!byte_pool && pool->kv_dtype != SCKV_DTYPE_F16 && pool->kv_dtype != SCKV_DTYPE_BF16) return SCKV_ERR_UNSUPPORTED;
  // 16-byte vector loads of q and stores of out
  if ((reinterpret_cast<uintptr_t>(q) & 15) || (reinterpret_cast<uintptr_t>(out) & 15)) return SCKV_ERR_UNSUPPORTED;
  TcParams prm{};
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
  prm.lg_g = lg_g;
  prm.layer = layer;
  prm.q_dtype = q_dtype;
  prm.out_dtype = out_dtype;
  prm.scale_log2 = scale * 1.4426950408889634f;
  prm.next_item = sckv_take_work_counter(pool);
  prm.kv_scales = pool->scales;
  const int BQ = kRowsTc >> lg_g;
  const int BQ2 = kQTiles * BQ;
  const int64_t max_tiles = (int64_t)(n_tokens + BQ2 - 1) / BQ2 + n_seqs;  // >= sum of ceil(T_s / BQ2)
  const int64_t max_items = max_tiles * pool->num_kv_heads;
  if (max_items > INT32_MAX) return SCKV_ERR_UNSUPPORTED;
  // 16-bit q arrives by TMA (converted in place by warps 14, 15 when it is
  // not the MMA's type): a 3-D view (dim, head, token) whose boxes of 64
  // dims x G heads x 128/G tokens are exactly an item's 128 rows, in row order
  CUtensorMap qmap;
  prm.q_tma = 0;
  // the MMA's element type: bf16 for bf16 pools, f16 otherwise (one-byte
  // pages are decoded into f16)
  const int mma_dtype = pool->kv_dtype == SCKV_DTYPE_BF16 ? SCKV_DTYPE_BF16 : SCKV_DTYPE_F16;
  if (q_dtype == SCKV_DTYPE_F16 || q_dtype == SCKV_DTYPE_BF16) {
    PFN_cuTensorMapEncodeTiled_v12000 encode = tensor_map_encoder();
    if (encode != nullptr) {
      const cuuint64_t dims[3] = {(cuuint64_t)kHDim, (cuuint64_t)num_q_heads, (cuuint64_t)n_tokens};
      const cuuint64_t strides[2] = {(cuuint64_t)kHDim * 2, (cuuint64_t)num_q_heads * kHDim * 2};
      const cuuint32_t box[3] = {64, (cuuint32_t)(1 << lg_g), (cuuint32_t)BQ};
      const cuuint32_t estr[3] = {1, 1, 1};
      if (encode(&qmap, CU_TENSOR_MAP_DATA_TYPE_UINT16, 3, const_cast<void*>(q), dims, strides, box, estr,
                 CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                 CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS)
        prm.q_tma = q_dtype == mma_dtype ? 1 : 2;
    }
  }
  switch (pool->kv_dtype) {
    case SCKV_DTYPE_BF16: return launch_tc<SCKV_DTYPE_BF16>(pool, prm, (int)max_items, qmap, stream);
    case SCKV_DTYPE_F16: return launch_tc<SCKV_DTYPE_F16>(pool, prm, (int)max_items, qmap, stream);
    case SCKV_DTYPE_FP8_E4M3: return launch_tc<SCKV_DTYPE_FP8_E4M3>(pool, prm, (int)max_items, qmap, stream);
    case SCKV_DTYPE_INT8: return launch_tc<SCKV_DTYPE_INT8>(pool, prm, (int)max_items, qmap, stream);
    default: return SCKV_ERR_UNSUPPORTED;
  }
}

}  // namespace sckv_detail
