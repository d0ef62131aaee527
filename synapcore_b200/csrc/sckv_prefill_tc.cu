// Paged causal prefill attention on the 5th-generation tensor cores
// (tcgen05.mma, accumulators in tensor memory).
//
// Same contract as prefill_kernel in sckv_prefill.cu (models/adapters.py:
// 1209-1229, causal mask :1218-1224, query t of a sequence at position
// start + t sees keys 0..start + t), for f16 and bf16 pools.
//
// Work item = (sequence, tile of 128 query rows, kv head). The rows are
// (token, q head) pairs of the G heads that read the kv head, so a tile holds
// 128 / G tokens. Persistent CTAs (two per SM) claim items from a counter;
// 7 warps per CTA:
//   warp 0     claims items, loads the item's Q (one TMA box per 64-dim half
//              when q has the pool's type, else the softmax warps write it)
//              and streams K: 4 pages (64 keys) per tile, one 2 KiB box per
//              (page, 64-dim half), 128-byte swizzle, into a 2-slot ring laid
//              out as the UMMA K-major canonical tile (consecutive pages are
//              consecutive rows).
//   warp 6     streams V the same way into its own 2-slot ring (one TMA issue
//              holds its warp ~0.1 us, so K and V get a warp each).
//   warp 1     allocates 256 tensor-memory columns and issues the MMAs:
//                S[b] (128 x 64 fp32)  = Q . K^T        8 x tcgen05.mma (K = 16)
//                O    (128 x 128 fp32) += P[b] . V      4 x tcgen05.mma (A from TMEM)
//              S double-buffered, so S(j+1) runs while the softmax works on
//              S(j); K(j) is released when S(j) finishes, V(j) after PV(j).
//              Completion is signalled with tcgen05.commit on mbarriers.
//   warps 2-5  softmax: thread i owns query row i (TMEM lane i): loads its 64
//              scores with tcgen05.ld, masks (only tiles the causal limit cuts),
//              keeps a stale running max (moves only by more than 2^8,
//              rescaling O in TMEM when it does), writes P = 2^(s*scale - m)
//              as f16 / bf16 back over S (tcgen05.st), and at the end of the
//              item normalises its O row and stores it.
// bf16 pools split P into bf16 hi + lo parts (two PV products) so P's
// rounding stays below 2^-16 relative; f16 pools use P in f16.
// Slots past the sequence's last token (they may hold anything) are zeroed
// in the V tile before the PV product; their scores are masked.
#include <cuda.h>
#include <math.h>

#include "sckv_internal.cuh"
#include "sckv_mma_common.cuh"

using namespace sckv_mma;

namespace {

constexpr int kHDim = 128;
constexpr int kRowsTc = 128;                  // query rows per item (UMMA M)
constexpr int kKeysTc = 64;                   // keys per tile (4 pages)
constexpr int kPagesTc = kKeysTc / SCKV_PAGE_TOKENS;
constexpr int kStagesTc = 2;
constexpr int kThreadsTc = 224;  // warp 0 K / Q copies, 1 MMA, 2-5 softmax, 6 V copies
constexpr int kSoftmaxThreads = 128;
constexpr uint32_t kTmemCols = 256;
constexpr uint32_t kColS = 0;                 // S[b] at columns 64 b
constexpr uint32_t kColO = 128;

constexpr int kQHalf = kRowsTc * 128;         // one 64-dim half of Q: 16 KiB
constexpr int kTileHalf = kKeysTc * 128;      // one 64-dim half of a K or V tile: 8 KiB
constexpr int kSlotBytes = 2 * kTileHalf;     // a K (or V) tile: lo and hi halves
constexpr int kOffK = 2 * kQHalf;             // K ring [kStagesTc]
constexpr int kOffV = kOffK + kStagesTc * kSlotBytes;  // V ring [kStagesTc]
constexpr int kOffBar = kOffV + kStagesTc * kSlotBytes;
constexpr int kNumBars = 22;
constexpr int kOffItemRing = kOffBar + kNumBars * 8;  // int[4]
constexpr int kOffTmemSlot = kOffItemRing + 16;
constexpr int kOffAbort = kOffTmemSlot + 4;
constexpr int kOffPartial = kOffTmemSlot + 16;
constexpr int kOffTileCum = kOffPartial + kThreadsTc * 4;
constexpr int kFixedSmem = 1024 + kOffTileCum;  // + 4 * (n_seqs + 1)


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
  int q_tma;  // q arrives by TMA (its type is the MMA's)
  unsigned long long* next_item;  // work counter, zero at launch
  float scale_log2;
};

// ------------------------------------------------------------------ tcgen05
// Shared-memory matrix descriptor, 128-byte swizzle (sm100 layout: start,
// leading and stride byte offsets in 16-byte units, version 1, swizzle code 2).
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t saddr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
  uint64_t d = (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

// Instruction descriptor of kind::f16 with fp32 accumulation, M = 128.
__host__ __device__ constexpr uint32_t instr_desc_f16(bool bf16, int n, bool b_mn_major) {
  return (1u << 4) | ((bf16 ? 1u : 0u) << 7) | ((bf16 ? 1u : 0u) << 10) | ((b_mn_major ? 1u : 0u) << 16) |
         ((uint32_t)(n >> 3) << 17) | ((uint32_t)(kRowsTc >> 4) << 24);
}

__device__ __forceinline__ void umma_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                        uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}\n" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(0), "r"(0), "r"(0), "r"(0));
}

__device__ __forceinline__ void umma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                        uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, {%5, %6, %7, %8}, p;\n\t}\n" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(0), "r"(0), "r"(0), "r"(0));
}

__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tc_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// 32 consecutive fp32 columns of this thread's TMEM lane.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]),
      "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]),
      "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}

// 2^x by the hardware approximation (flushes denormals; 2^-inf = 0).
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Every lane of the warp waits; the result is the same on all lanes.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity) {
  const bool ok = mbar_wait_bounded(bar, parity, SCKV_WAIT_LIMIT_NS);
  return __all_sync(0xffffffffu, ok);
}

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
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = sckv_load_as_float(q, idx + i, dtype);
  }
  uint4 r;
  r.x = pack2<kBF16>(v[0], v[1]);
  r.y = pack2<kBF16>(v[2], v[3]);
  r.z = pack2<kBF16>(v[4], v[5]);
  r.w = pack2<kBF16>(v[6], v[7]);
  return r;
}

// One work item's geometry, derived identically by every role.
struct TcItem {
  int seq, h, s0, T, tok0, key_last, jlast, n_tiles, ctx_total, vlim, q_base;
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
  const int tile = gt - tile_cum[lo];
  it.T = tc_seq_tokens(p, it.seq, &it.s0, false);
  it.tok0 = tile * BQ;
  const int tok_last = min(it.T, it.tok0 + BQ) - 1;
  it.key_last = it.s0 + tok_last;                      // last key any row of the item sees
  it.jlast = it.key_last / SCKV_PAGE_TOKENS;            // last page
  it.n_tiles = it.key_last / kKeysTc + 1;
  it.ctx_total = it.s0 + it.T;
  it.vlim = min(it.ctx_total, (it.jlast + 1) * SCKV_PAGE_TOKENS);  // V rows at or past this key get zeroed
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

// Persistent: each CTA claims items from a counter in the pool's control
// words (heaviest-first order within each sequence) until they run out.
// Tiles of all its items are numbered by one running counter g, which fixes
// every barrier's phase (stage g % 2, S / P buffer g & 1). Calls on one pool
// must not overlap on the GPU (they share the counter).
template <bool kBF16>
__global__ void __launch_bounds__(kThreadsTc, 2)
    prefill_tc_kernel(const TcParams p, const __grid_constant__ CUtensorMap tmap,
                      const __grid_constant__ CUtensorMap qmap) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(base + kOffBar);
  // K and V have rings of their own: K(g) is released as soon as S(g) is
  // done, so K(g + 2) streams in while the softmax still works on tile g.
  uint64_t* k_full = bars + 14;    // [2] K tile landed (TMA)
  uint64_t* k_empty = bars + 16;   // [2] S finished with the K slot (commit)
  uint64_t* v_full = bars + 18;    // [2] V tile landed (TMA)
  uint64_t* v_empty = bars + 20;   // [2] PV finished with the V slot (commit)
  uint64_t* s_full = bars + 0;     // [2] S(g) in TMEM (commit)
  uint64_t* p_full = bars + 2;     // [2] P(g) in TMEM (128 softmax threads)
  // [2] PV(g) finished (commit to pv_done[g & 1]). A softmax thread waits for
  // PV(g) only after S(g) landed (or, for a rescale, S(g + 1)), and that
  // commit covers every MMA issued before it, PV(g - 2) included; PV(g + 2)
  // cannot start before this thread writes P(g + 2). So the barrier is at
  // PV(g)'s phase or one past it and the parity wait is unambiguous however
  // rarely the thread waits on it.
  uint64_t* pv_done = bars + 4;
  uint64_t* q_full = bars + 6;    // Q of the item in shared memory (TMA, or 128 softmax threads)
  uint64_t* q_empty = bars + 7;   // every S of the item finished (commit): Q may be replaced
  uint64_t* o_empty = bars + 8;   // the item's O was read out (128 softmax threads)
  uint64_t* mma_done = bars + 9;  // every issued MMA finished (drain)
  // [4] item k's index is in item_ring[k & 3] (producer). The producer runs
  // at most two items ahead of the softmax warps (its Q load for item k + 1
  // waits for all S of item k, and S of item k past its second tile waits
  // for the softmax of item k), so a slot is never rewritten while unread.
  uint64_t* item_full = bars + 10;
  volatile int* item_ring = reinterpret_cast<volatile int*>(base + kOffItemRing);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(base + kOffTmemSlot);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(base + kOffAbort);
  int* partial = reinterpret_cast<int*>(base + kOffPartial);
  int* tile_cum = reinterpret_cast<int*>(base + kOffTileCum);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int G = 1 << p.lg_g;
  const int BQ = kRowsTc >> p.lg_g;  // tokens per item

  // ---- tiles per sequence, prefix-summed by the whole CTA
  {
    const int per = (p.n_seqs + kThreadsTc - 1) / kThreadsTc;
    const int s0 = threadIdx.x * per, s1 = min(p.n_seqs, s0 + per);
    int local = 0;
    for (int s = s0; s < s1; ++s) {
      int st;
      const int T = tc_seq_tokens(p, s, &st, blockIdx.x == 0);
      local += (T + BQ - 1) / BQ;
    }
    partial[threadIdx.x] = local;
    if (threadIdx.x == 0) {
      for (int i = 0; i < kNumBars; ++i) {
        uint64_t* bar = &bars[i];
        const bool by_softmax = bar == &p_full[0] || bar == &p_full[1] || bar == o_empty ||
                                (bar == q_full && !p.q_tma);
        mbar_init(bar, by_softmax ? kSoftmaxThreads : 1);
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
      run += (T + BQ - 1) / BQ;
      tile_cum[s + 1] = run;
    }
    __syncthreads();
  }
  const int total_tiles = tile_cum[p.n_seqs];
  const int n_items = total_tiles * p.hkv;

  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0 || warp == 6) {
    // ------------------------------------------------------------ producers
    // warp 0 claims items and streams Q and the K ring, warp 6 streams the
    // V ring: two issuing warps, because one TMA issue holds its warp ~0.1 us
    if (lane == 0) {
      const int kv = warp == 6 ? 1 : 0;
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmap)) : "memory");
      if (kv == 0 && p.q_tma)
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&qmap)) : "memory");
      const int64_t layer_base = (int64_t)p.layer * p.max_pages;
      int g = 0, q_issued = 0, issued = 0;
      bool aborted = false;
      for (int k = 0;; ++k) {
        int item;
        if (kv == 0) {
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
        if (kv == 0 && p.q_tma) {
          if (k > 0 &&
              (*abort_flag || !mbar_wait_bounded(q_empty, (k - 1) & 1, SCKV_WAIT_LIMIT_NS))) {
            aborted = true;
            continue;  // publishes the stop marker next
          }
          mbar_arrive_expect_tx(q_full, 2u * kQHalf);
          tma_load_3d(smem_u32(base), &qmap, 0, it.h * G, it.q_base + it.tok0, q_full);
          tma_load_3d(smem_u32(base + kQHalf), &qmap, 64, it.h * G, it.q_base + it.tok0, q_full);
          ++q_issued;
        }
        const int32_t* bt_row = p.block_table + (int64_t)it.seq * p.bt_stride;
        // page ids of local tile j, fetched one tile ahead so their load
        // latency overlaps the copies being issued (a TMA issue orders
        // everything before it)
        auto fetch_ids = [&](int j, int (&ids)[kPagesTc]) {
#pragma unroll
          for (int pg = 0; pg < kPagesTc; ++pg) {
            const int blk = j * kPagesTc + pg;
            ids[pg] = blk <= it.jlast ? __ldg(bt_row + blk) : 0;
          }
        };
        int ids_next[kPagesTc], ids_cur[kPagesTc];
        fetch_ids(0, ids_next);
        for (int j = 0; j < it.n_tiles; ++j) {
#pragma unroll
          for (int pg = 0; pg < kPagesTc; ++pg) ids_cur[pg] = ids_next[pg];
          if (j + 1 < it.n_tiles) fetch_ids(j + 1, ids_next);
          // K(g) waits only for S(g - 2) to finish, V(g) for PV(g - 2)
          const int gt = g + j;
          const int st = gt % kStagesTc;
          uint64_t* full = kv ? &v_full[st] : &k_full[st];
          uint64_t* empty = kv ? &v_empty[st] : &k_empty[st];
          if (gt >= kStagesTc &&
              (*abort_flag || !mbar_wait_bounded(empty, ((gt / kStagesTc) - 1) & 1, SCKV_WAIT_LIMIT_NS))) {
            aborted = true;
            break;
          }
          const int np = min(kPagesTc, it.jlast + 1 - j * kPagesTc);
          const uint32_t slot = smem_u32(base + (kv ? kOffV : kOffK) + st * kSlotBytes);
          mbar_arrive_expect_tx(full, (uint32_t)np * 2u * 2048u);
          for (int pg = 0; pg < np; ++pg) {
            int32_t page = ids_cur[pg];
            if (page < 0 || page >= p.max_pages) {
              sckv_report(p.status, SCKV_ERR_BOUNDS, page, KID_PREFILL);
              page = 0;
            }
            const int slab = (int)(layer_base + page);
            tma_load_5d(slot + pg * 2048, &tmap, 0, 0, it.h, kv, slab, full);
            tma_load_5d(slot + kTileHalf + pg * 2048, &tmap, 64, 0, it.h, kv, slab, full);
          }
          ++issued;
        }
        g += it.n_tiles;
        if (kv == 1 && aborted) break;
      }
      if (aborted) {
        if (!*abort_flag) sckv_report(p.status, SCKV_ERR_TIMEOUT, blockIdx.x, KID_PREFILL);
        *abort_flag = 1;
      }
      // nothing of ours may still be landing when the CTA retires
      uint64_t* fulls = kv ? v_full : k_full;
      for (int t = issued > kStagesTc ? issued - kStagesTc : 0; t < issued; ++t)
        mbar_wait_bounded(&fulls[t % kStagesTc], (t / kStagesTc) & 1, SCKV_WAIT_LIMIT_NS);
      if (q_issued > 0) mbar_wait_bounded(q_full, (q_issued - 1) & 1, SCKV_WAIT_LIMIT_NS);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    constexpr uint32_t kIdescS = instr_desc_f16(kBF16, kKeysTc, false);
    constexpr uint32_t kIdescPV = instr_desc_f16(kBF16, kHDim, true);
    const uint32_t q_smem = smem_u32(base);
    bool ok = true;
    int g = 0, k = 0;
    // PV of global tile gi = local tile li of item k: O (+)= P . V
    auto issue_pv = [&](const TcItem& it, int gi, int li) -> bool {
      const int b = gi & 1;
      const int st = gi % kStagesTc;
      if (!warp_wait(&p_full[b], (gi >> 1) & 1)) return false;
      tc_fence_after();
      if (li == 0 && k > 0) {
        // O still holds the previous item until its epilogue has read it
        if (!warp_wait(o_empty, (k - 1) & 1)) return false;
        tc_fence_after();
      }
      if (!warp_wait(&v_full[st], (gi / kStagesTc) & 1)) return false;
      tc_fence_after();
      uint8_t* vslot = base + kOffV + st * kSlotBytes;
      const int key0 = li * kKeysTc;
      if (key0 + kKeysTc > it.vlim) {
        // zero the V rows of keys >= vlim (both 64-dim halves): their slots
        // were never written or hold an older tile
        const int r0 = max(0, it.vlim - key0);
        const int n16 = (kKeysTc - r0) * 8;  // 16-byte chunks per half
        for (int c = lane; c < 2 * n16; c += 32) {
          const int half = c / n16, rc = c - half * n16;
          *reinterpret_cast<uint4*>(vslot + half * kTileHalf + (r0 + (rc >> 3)) * 128 + (rc & 7) * 16) =
              make_uint4(0u, 0u, 0u, 0u);
        }
        fence_proxy_async_smem();
        __syncwarp();
      }
      if (lane == 0) {
        const uint32_t v_smem = smem_u32(vslot);
#pragma unroll
        for (int pg = 0; pg < kPagesTc; ++pg) {
          // B = V rows of page pg: N = 128 dims in two 64-dim halves (LBO),
          // K = 16 keys in two groups of 8 rows (SBO)
          const uint64_t bdesc = smem_desc_sw128(v_smem + pg * 2048, kTileHalf, 1024);
          const uint32_t a_col = tmem + kColS + (uint32_t)(b * kKeysTc) + (uint32_t)(pg * 8);
          umma_ts(tmem + kColO, a_col, bdesc, kIdescPV, (li > 0 || pg > 0) ? 1u : 0u);
          if (kBF16) umma_ts(tmem + kColO, a_col + 32, bdesc, kIdescPV, 1u);
        }
        umma_commit(&v_empty[st]);
        umma_commit(&pv_done[b]);
      }
      __syncwarp();
      return true;
    };
    for (; ok; ++k) {
      if (*abort_flag || !warp_wait(&item_full[k & 3], (k >> 2) & 1)) {
        ok = false;
        break;
      }
      const int item = item_ring[k & 3];
      if (item >= n_items) break;
      const TcItem it = tc_item(p, tile_cum, total_tiles, item, BQ);
      if (*abort_flag || !warp_wait(q_full, k & 1)) {
        ok = false;
        break;
      }
      tc_fence_after();
      for (int j = 0; j < it.n_tiles; ++j) {
        const int gj = g + j;
        const int st = gj % kStagesTc;
        const int b = gj & 1;
        if (*abort_flag || !warp_wait(&k_full[st], (gj / kStagesTc) & 1)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (lane == 0) {
          const uint32_t k_smem = smem_u32(base + kOffK + st * kSlotBytes);
#pragma unroll
          for (int ks = 0; ks < 8; ++ks) {
            const int half = ks >> 2, kk = ks & 3;
            const uint64_t adesc = smem_desc_sw128(q_smem + half * kQHalf + kk * 32, 16, 1024);
            const uint64_t bdesc = smem_desc_sw128(k_smem + half * kTileHalf + kk * 32, 16, 1024);
            umma_ss(tmem + kColS + (uint32_t)(b * kKeysTc), adesc, bdesc, kIdescS, ks > 0 ? 1u : 0u);
          }
          umma_commit(&k_empty[st]);
          umma_commit(&s_full[b]);
          if (j == it.n_tiles - 1) umma_commit(q_empty);  // Q no longer read once these S are done
        }
        __syncwarp();
        if (j >= 1 && !issue_pv(it, gj - 1, j - 1)) {
          ok = false;
          break;
        }
      }
      if (!ok || !issue_pv(it, g + it.n_tiles - 1, it.n_tiles - 1)) {
        ok = false;
        break;
      }
      g += it.n_tiles;
    }
    if (!ok) {
      if (lane == 0 && !*abort_flag) sckv_report(p.status, SCKV_ERR_TIMEOUT, blockIdx.x, KID_PREFILL);
      if (lane == 0) *abort_flag = 1;
    }
    // drain: every MMA issued above has finished before TMEM is released
    if (lane == 0) umma_commit(mma_done);
    __syncwarp();
    warp_wait(mma_done, 0);
  } else {
    // ------------------------------------------------------------ softmax
    const int quad = warp & 3;            // TMEM lanes 32 quad .. 32 quad + 31
    const int row = quad * 32 + lane;     // query row = TMEM lane
    const uint32_t t_row = tmem + ((uint32_t)(quad * 32) << 16);
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
      const int rtok = it.tok0 + (row >> p.lg_g);
      const int rhead = it.h * G + (row & (G - 1));
      const bool valid = rtok < it.T;
      const int lim = valid ? it.s0 + rtok : -1;  // last key this row sees
      if (!p.q_tma) {
        // Q row -> shared memory, 128-byte swizzled K-major (the layout a TMA
        // copy with SWIZZLE_128B produces). The previous item's S products
        // are all finished: this thread waited for every one of them.
        const int64_t qoff = ((int64_t)(it.q_base + rtok) * p.hq + rhead) * kHDim;
#pragma unroll
        for (int c = 0; c < 16; ++c) {
          const int half = c >> 3, ch = c & 7;
          const uint4 v = valid ? load_q8<kBF16>(p.q, qoff + c * 8, p.q_dtype) : make_uint4(0u, 0u, 0u, 0u);
          *reinterpret_cast<uint4*>(base + half * kQHalf + row * 128 + ((ch ^ (row & 7)) << 4)) = v;
        }
        fence_proxy_async_smem();
        mbar_arrive(q_full);
      }
      float m = -INFINITY, l = 0.f;
      for (int j = 0; j < it.n_tiles; ++j) {
        const int gj = g + j;
        const int b = gj & 1;
        if (*abort_flag || !warp_wait(&s_full[b], (gj >> 1) & 1)) {
          ok = false;
          break;
        }
        tc_fence_after();
        float sv[kKeysTc];
        {
          uint32_t r0[32], r1[32];
          tmem_ld32(t_row + kColS + b * kKeysTc, r0);
          tmem_ld32(t_row + kColS + b * kKeysTc + 32, r1);
          tc_wait_ld();
#pragma unroll
          for (int c = 0; c < 32; ++c) {
            sv[c] = __uint_as_float(r0[c]);
            sv[32 + c] = __uint_as_float(r1[c]);
          }
        }
        // row max of the raw scores (the scale is positive); tiles every row
        // of the item sees in full skip the causal mask
        const int key0 = j * kKeysTc;
        float pm = -INFINITY;
        if (key0 + kKeysTc - 1 <= it.s0 + it.tok0) {
#pragma unroll
          for (int c = 0; c < kKeysTc; ++c) pm = fmaxf(pm, sv[c]);
        } else {
#pragma unroll
          for (int c = 0; c < kKeysTc; ++c) {
            const float v = (key0 + c <= lim) ? sv[c] : -INFINITY;
            sv[c] = v;
            pm = fmaxf(pm, v);
          }
        }
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
          // O holds PV of tiles 0..j-1 of this item: wait for the last, then
          // scale this warp's rows
          if (!warp_wait(&pv_done[(gj - 1) & 1], ((gj - 1) >> 1) & 1)) {
            ok = false;
            break;
          }
          tc_fence_after();
#pragma unroll 1
          for (int cc = 0; cc < 4; ++cc) {
            uint32_t r[32];
            tmem_ld32(t_row + kColO + cc * 32, r);
            tc_wait_ld();
#pragma unroll
            for (int c = 0; c < 32; ++c) r[c] = __float_as_uint(__uint_as_float(r[c]) * alpha);
            tmem_st32(t_row + kColO + cc * 32, r);
          }
          tc_wait_st();
        }
        // P = 2^(s - m), packed two keys per column over S's first columns
        {
          uint32_t ph[32], plo[32];
          // a row that sees no key yet (m = -inf) has every score -inf: 2^-inf = 0
          const float mm = (m == -INFINITY) ? 0.f : m;
          float ls0 = 0.f, ls1 = 0.f;
#pragma unroll
          for (int c = 0; c < 32; ++c) {
            const float p0 = ex2_approx(fmaf(sv[2 * c], p.scale_log2, -mm));
            const float p1 = ex2_approx(fmaf(sv[2 * c + 1], p.scale_log2, -mm));
            ls0 += p0;
            ls1 += p1;
            ph[c] = pack2<kBF16>(p0, p1);
            if (kBF16) plo[c] = pack2<true>(p0 - round16<true>(p0), p1 - round16<true>(p1));
          }
          tmem_st32(t_row + kColS + b * kKeysTc, ph);
          if (kBF16) tmem_st32(t_row + kColS + b * kKeysTc + 32, plo);
          l += ls0 + ls1;
          tc_wait_st();
        }
        tc_fence_before();
        mbar_arrive(&p_full[b]);
      }
      if (!ok) break;
      // ---- epilogue: O / l for this thread's row, once the item's last PV finished
      const int glast = g + it.n_tiles - 1;
      if (!warp_wait(&pv_done[glast & 1], (glast >> 1) & 1)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const float inv = (l > 0.f) ? 1.f / l : 0.f;
      const int64_t obase = ((int64_t)(it.q_base + rtok) * p.hq + rhead) * kHDim;
#pragma unroll 1
      for (int cc = 0; cc < 4; ++cc) {
        uint32_t r[32];
        tmem_ld32(t_row + kColO + cc * 32, r);
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
              uint4 w;
              uint32_t* wp = &w.x;
#pragma unroll
              for (int kk = 0; kk < 4; ++kk) {
                const float a = __uint_as_float(r[c + 2 * kk]) * inv, bb = __uint_as_float(r[c + 2 * kk + 1]) * inv;
                wp[kk] = obf ? pack2<true>(a, bb) : pack2<false>(a, bb);
              }
              *reinterpret_cast<uint4*>(o + c) = w;
            }
          }
        }
      }
      tc_fence_before();
      mbar_arrive(o_empty);  // O may be overwritten by the next item's PV
      g += it.n_tiles;
    }
    if (!ok) {
      if (lane == 0 && !*abort_flag) sckv_report(p.status, SCKV_ERR_TIMEOUT, blockIdx.x, KID_PREFILL);
      if (lane == 0) *abort_flag = 1;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
  }
}

template <bool kBF16>
int launch_tc(const sckv_pool* pool, const TcParams& prm, int max_items, const CUtensorMap& qmap,
              cudaStream_t stream) {
  auto kern = prefill_tc_kernel<kBF16>;
  sckv_pool* mp = const_cast<sckv_pool*>(pool);  // the map is a cache inside the handle
  int rc = ensure_tmap(pool, 1, mp->tmap_kv2, &mp->tmap2_ready, 1);
  if (rc != SCKV_OK) return rc;
  const int smem = kFixedSmem + 4 * (prm.n_seqs + 1);
  SCKV_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
  SCKV_CUDA_CHECK(cudaMemsetAsync(prm.next_item, 0, sizeof(unsigned long long), stream));
  int occ = 0;
  SCKV_CUDA_CHECK(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, kThreadsTc, smem));
  if (occ < 1) occ = 1;
  if (occ > 2) occ = 2;  // two CTAs x 256 TMEM columns fill an SM's tensor memory
  int grid = pool->num_sms * occ;
  if (grid > max_items) grid = max_items;
  const CUtensorMap* kv_map = reinterpret_cast<const CUtensorMap*>(pool->tmap_kv2);
  kern<<<grid, kThreadsTc, smem, stream>>>(prm, *kv_map, prm.q_tma ? qmap : *kv_map);
  SCKV_LAUNCH_CHECK();
  return SCKV_OK;
}

}  // namespace

namespace sckv_detail {

// Tensor-memory prefill for f16 / bf16 pools. Returns SCKV_ERR_UNSUPPORTED
// for combinations it does not build (the caller then uses prefill_kernel).
int launch_prefill_tc(const sckv_pool* pool, int layer, const void* q, int q_dtype, int num_q_heads, int n_seqs,
                      int n_tokens, const int32_t* cu_q, const int32_t* start_pos, const int32_t* block_table,
                      int64_t bt_stride, int max_blocks, float scale, void* out, int out_dtype, int lg_g,
                      cudaStream_t stream) {
  if (pool->kv_dtype != SCKV_DTYPE_F16 && pool->kv_dtype != SCKV_DTYPE_BF16) return SCKV_ERR_UNSUPPORTED;
  if (pool->head_dim != kHDim || n_seqs > 16384 || !(scale > 0.f)) return SCKV_ERR_UNSUPPORTED;
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
  prm.next_item = reinterpret_cast<unsigned long long*>(pool->ctl + CTL_PREFILL_NEXT);
  const int BQ = kRowsTc >> lg_g;
  const int64_t max_tiles = (int64_t)(n_tokens + BQ - 1) / BQ + n_seqs;  // >= sum of ceil(T_s / BQ)
  const int64_t max_items = max_tiles * pool->num_kv_heads;
  if (max_items > INT32_MAX) return SCKV_ERR_UNSUPPORTED;
  // q in the MMA's element type arrives by TMA: a 3-D view (dim, head,
  // token) whose boxes of 64 dims x G heads x 128/G tokens are exactly an
  // item's 128 rows, in row order
  CUtensorMap qmap;
  prm.q_tma = 0;
  if (q_dtype == pool->kv_dtype) {
    PFN_cuTensorMapEncodeTiled_v12000 encode = tensor_map_encoder();
    if (encode != nullptr) {
      const cuuint64_t dims[3] = {(cuuint64_t)kHDim, (cuuint64_t)num_q_heads, (cuuint64_t)n_tokens};
      const cuuint64_t strides[2] = {(cuuint64_t)kHDim * 2, (cuuint64_t)num_q_heads * kHDim * 2};
      const cuuint32_t box[3] = {64, (cuuint32_t)(1 << lg_g), (cuuint32_t)BQ};
      const cuuint32_t estr[3] = {1, 1, 1};
      if (encode(&qmap, CU_TENSOR_MAP_DATA_TYPE_UINT16, 3, const_cast<void*>(q), dims, strides, box, estr,
                 CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                 CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS)
        prm.q_tma = 1;
    }
  }
  return pool->kv_dtype == SCKV_DTYPE_BF16 ? launch_tc<true>(pool, prm, (int)max_items, qmap, stream)
                                           : launch_tc<false>(pool, prm, (int)max_items, qmap, stream);
}

}  // namespace sckv_detail
