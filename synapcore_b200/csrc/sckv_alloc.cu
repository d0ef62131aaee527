// Kernel 5: on-device page allocator with FIFO free ring and LRU eviction.
//
// Restates PagedKVArena's bookkeeping (native/native_engine.py:289-337):
//   * free_pages = deque(range(max_pages)), popleft() on allocation,
//     append() on eviction of a key            -> ring[head..tail) (FIFO)
//   * step_clock += 1 per allocation / lookup  -> ctl[CTL_CLOCK]
//   * page_last_used[key] = step_clock         -> last_used[page]
//   * victim = min(page_table, key=last_used)  -> smallest last_used among
//     allocated, unpinned pages (clock values are unique, so no ties).
// A batch of n allocations equals n sequential _allocate_page_slot_unlocked
// calls for new keys: first the ring head, then victims in increasing
// last_used order, clocks clock+1 .. clock+n in request order.
//
// All kernels are single-CTA (1024 threads): the work is a few passes over
// the per-page arrays plus an in-shared-memory sort of the chosen victims.
#include "sckv_internal.cuh"

namespace {

constexpr int kT = 1024;          // threads of the allocator CTA
constexpr int kSortCap = 4096;    // victims selected per round

struct AllocView {
  int64_t* ctl;
  int32_t* ring;
  int64_t* last_used;
  int32_t* pin;
  int32_t* state;
  int32_t* status;
  int64_t P;
};

AllocView view_of(const sckv_pool* p) {
  AllocView a;
  a.ctl = p->ctl;
  a.ring = p->ring;
  a.last_used = p->last_used;
  a.pin = p->pin;
  a.state = p->state;
  a.status = p->status;
  a.P = p->max_pages;
  return a;
}

struct SelectSmem {
  unsigned long long keys[kSortCap];
  int32_t vals[kSortCap];
  unsigned int hist[256];
  unsigned long long red_u64[kT / 32];
  int red_i32[kT / 32];
  int count;
  unsigned long long bcast;
  int bcast_i;
};

__device__ __forceinline__ bool is_candidate(const AllocView& a, int64_t i) {
  return a.state[i] == PAGE_ALLOCATED && a.pin[i] == 0;
}

// Block-wide sum / max helpers (all kT threads must call).
__device__ int block_sum_int(int v, SelectSmem& s) {
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int w = threadIdx.x >> 5;
  if ((threadIdx.x & 31) == 0) s.red_i32[w] = v;
  __syncthreads();
  if (threadIdx.x == 0) {
    int t = 0;
    for (int i = 0; i < kT / 32; ++i) t += s.red_i32[i];
    s.bcast_i = t;
  }
  __syncthreads();
  int r = s.bcast_i;
  __syncthreads();
  return r;
}

__device__ unsigned long long block_max_u64(unsigned long long v, SelectSmem& s) {
  for (int o = 16; o > 0; o >>= 1) {
    unsigned long long u = __shfl_xor_sync(0xffffffffu, v, o);
    v = u > v ? u : v;
  }
  const int w = threadIdx.x >> 5;
  if ((threadIdx.x & 31) == 0) s.red_u64[w] = v;
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned long long t = 0;
    for (int i = 0; i < kT / 32; ++i) t = s.red_u64[i] > t ? s.red_u64[i] : t;
    s.bcast = t;
  }
  __syncthreads();
  unsigned long long r = s.bcast;
  __syncthreads();
  return r;
}

// Exclusive prefix sum of one int per thread (block-wide), returns the
// exclusive prefix and writes the total to *total.
__device__ int block_exclusive_scan(int v, int* total, SelectSmem& s) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  int x = v;
  for (int o = 1; o < 32; o <<= 1) {
    int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) s.red_i32[w] = x;
  __syncthreads();
  if (w == 0) {
    int t = (lane < kT / 32) ? s.red_i32[lane] : 0;
    for (int o = 1; o < 32; o <<= 1) {
      int y = __shfl_up_sync(0xffffffffu, t, o);
      if (lane >= o) t += y;
    }
    if (lane < kT / 32) s.red_i32[lane] = t;  // inclusive per-warp totals
  }
  __syncthreads();
  const int warp_prefix = (w == 0) ? 0 : s.red_i32[w - 1];
  const int tot = s.red_i32[kT / 32 - 1];
  __syncthreads();
  *total = tot;
  return warp_prefix + x - v;
}

// Bitonic sort of s.keys/vals[0..n2) ascending by key (n2 power of two <= kSortCap).
__device__ void bitonic_sort(SelectSmem& s, int n2) {
  for (int k = 2; k <= n2; k <<= 1) {
    for (int j = k >> 1; j > 0; j >>= 1) {
      for (int i = threadIdx.x; i < n2; i += kT) {
        const int ixj = i ^ j;
        if (ixj > i) {
          const bool up = ((i & k) == 0);
          unsigned long long ki = s.keys[i], kj = s.keys[ixj];
          if ((ki > kj) == up) {
            s.keys[i] = kj; s.keys[ixj] = ki;
            int32_t t = s.vals[i]; s.vals[i] = s.vals[ixj]; s.vals[ixj] = t;
          }
        }
      }
      __syncthreads();
    }
  }
}

// Select the `want` (<= kSortCap) smallest last_used keys among candidates
// with key > lo (strictly), ascending in s.keys/vals[0..found). Keys are unique.
__device__ int select_smallest(const AllocView& a, unsigned long long lo, int want, SelectSmem& s) {
  // Pass 1: candidate count above lo, and max key.
  int cnt = 0;
  unsigned long long mx = 0;
  for (int64_t i = threadIdx.x; i < a.P; i += kT) {
    if (is_candidate(a, i)) {
      unsigned long long k = (unsigned long long)a.last_used[i];
      if (k > lo) { ++cnt; mx = k > mx ? k : mx; }
    }
  }
  const int total = block_sum_int(cnt, s);
  mx = block_max_u64(mx, s);
  if (total == 0 || want <= 0) return 0;
  unsigned long long thresh = mx;  // collect keys in (lo, thresh]
  if (total > want) {
    // Radix select of the want-th smallest key, 8 bits at a time from the top byte of mx.
    int top = 0;
    while (top < 7 && (mx >> (8 * (top + 1))) != 0) ++top;
    unsigned long long prefix = 0;
    int k = want;
    for (int byte = top; byte >= 0; --byte) {
      const int shift = 8 * byte;
      const unsigned long long himask = (byte == 7) ? 0ULL : ~((1ULL << (shift + 8)) - 1ULL);
      for (int i = threadIdx.x; i < 256; i += kT) s.hist[i] = 0;
      __syncthreads();
      for (int64_t i = threadIdx.x; i < a.P; i += kT) {
        if (!is_candidate(a, i)) continue;
        unsigned long long key = (unsigned long long)a.last_used[i];
        if (key <= lo || ((key ^ prefix) & himask) != 0) continue;
        atomicAdd(&s.hist[(key >> shift) & 255ULL], 1u);
      }
      __syncthreads();
      if (threadIdx.x == 0) {
        int cum = 0, d = 0;
        for (d = 0; d < 256; ++d) {
          if (cum + (int)s.hist[d] >= k) break;
          cum += s.hist[d];
        }
        s.bcast = prefix | ((unsigned long long)d << shift);
        s.bcast_i = k - cum;
      }
      __syncthreads();
      prefix = s.bcast;
      k = s.bcast_i;
      __syncthreads();
    }
    thresh = prefix;
  }
  // Collect keys in (lo, thresh].
  if (threadIdx.x == 0) s.count = 0;
  __syncthreads();
  for (int64_t i = threadIdx.x; i < a.P; i += kT) {
    if (!is_candidate(a, i)) continue;
    unsigned long long key = (unsigned long long)a.last_used[i];
    if (key > lo && key <= thresh) {
      int slot = atomicAdd(&s.count, 1);
      if (slot < kSortCap) { s.keys[slot] = key; s.vals[slot] = (int32_t)i; }
    }
  }
  __syncthreads();
  int found = s.count < kSortCap ? s.count : kSortCap;
  int n2 = 1;
  while (n2 < found) n2 <<= 1;
  for (int i = found + threadIdx.x; i < n2; i += kT) { s.keys[i] = ~0ULL; s.vals[i] = -1; }
  __syncthreads();
  bitonic_sort(s, n2);
  return found < want ? found : want;
}

// Core allocation of n pages. emit(k, page, victim) is called by some thread
// for each k in 0..n-1. Returns false (and reports) when the pool cannot
// provide n pages. Pages get last_used = clock0 + 1 + k and pin = pin0.
template <typename Emit>
__device__ bool alloc_core(const AllocView& a, int n, int pin0, SelectSmem& s, Emit emit, int kid) {
  const int64_t head = a.ctl[CTL_HEAD];
  const int64_t tail = a.ctl[CTL_TAIL];
  const int64_t clock0 = a.ctl[CTL_CLOCK];
  const int64_t avail = tail - head;
  const int f = (int)(n < avail ? n : avail);
  const int e = n - f;
  if (e > 0) {
    // Victims must pre-exist this batch: count allocated unpinned pages.
    int cnt = 0;
    for (int64_t i = threadIdx.x; i < a.P; i += kT) cnt += is_candidate(a, i) ? 1 : 0;
    const int total = block_sum_int(cnt, s);
    if (total < e) {
      if (threadIdx.x == 0) sckv_report(a.status, SCKV_ERR_POOL_EXHAUSTED, n, kid);
      return false;
    }
  }
  for (int k = threadIdx.x; k < f; k += kT) {
    const int32_t id = a.ring[(head + k) % a.P];
    a.state[id] = PAGE_ALLOCATED;
    a.last_used[id] = clock0 + 1 + k;
    a.pin[id] = pin0;
    emit(k, id, -1);
  }
  __syncthreads();
  // Victims: e smallest last_used among pages allocated before this batch.
  unsigned long long lo = 0;
  int done = 0;
  bool first_round = true;
  while (done < e) {
    const int want = (e - done) < kSortCap ? (e - done) : kSortCap;
    // Keys of this batch's fresh pages are > clock0; restrict to <= clock0 by
    // selecting among pages whose key <= clock0 (they are the only ones smaller).
    const int got = select_smallest(a, first_round ? 0ULL : lo, want, s);
    first_round = false;
    if (got < want) {  // cannot happen after the count check, but stay safe
      if (threadIdx.x == 0) sckv_report(a.status, SCKV_ERR_POOL_EXHAUSTED, n, kid);
      return false;
    }
    lo = s.keys[got - 1];
    __syncthreads();
    for (int k = threadIdx.x; k < got; k += kT) {
      const int32_t id = s.vals[k];
      const int kk = f + done + k;
      a.last_used[id] = clock0 + 1 + kk;
      a.pin[id] = pin0;
      emit(kk, id, id);
    }
    __syncthreads();
    done += got;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    a.ctl[CTL_HEAD] = head + f;
    a.ctl[CTL_CLOCK] = clock0 + n;
    a.ctl[CTL_EVICTIONS] += e;
    a.ctl[CTL_ALLOCATED] += f;
  }
  __syncthreads();
  return true;
}

__global__ void reset_kernel(AllocView a) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < a.P; i += (int64_t)gridDim.x * blockDim.x) {
    a.ring[i] = (int32_t)i;
    a.last_used[i] = 0;
    a.pin[i] = 0;
    a.state[i] = PAGE_FREE;
  }
  if (blockIdx.x == 0 && threadIdx.x < CTL_WORDS) a.ctl[threadIdx.x] = (threadIdx.x == CTL_TAIL) ? a.P : 0;
  if (blockIdx.x == 0 && threadIdx.x < 4) a.status[threadIdx.x] = 0;
}

__global__ void __launch_bounds__(kT) alloc_kernel(AllocView a, int n, int pin0, int32_t* out_ids,
                                                   int32_t* out_victims) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  SelectSmem& s = *reinterpret_cast<SelectSmem*>(smem_raw);
  bool ok = alloc_core(a, n, pin0, s,
                       [&](int k, int32_t id, int32_t victim) {
                         out_ids[k] = id;
                         if (out_victims) out_victims[k] = victim;
                       },
                       KID_ALLOC);
  if (!ok) {
    for (int k = threadIdx.x; k < n; k += kT) {
      out_ids[k] = -1;
      if (out_victims) out_victims[k] = -1;
    }
  }
}

// Sort (id, index) pairs of one chunk to find first occurrences of each id.
__global__ void __launch_bounds__(kT) free_kernel(AllocView a, const int32_t* ids, int n) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  SelectSmem& s = *reinterpret_cast<SelectSmem*>(smem_raw);
  __shared__ int keep_flag[kT];
  for (int base = 0; base < n; base += kT) {
    const int m = (n - base) < kT ? (n - base) : kT;
    const int i = threadIdx.x;
    int32_t id = -1;
    if (i < m) id = ids[base + i];
    const bool valid = (i < m) && id >= 0 && id < a.P;
    if (i < m && !(id >= 0 && id < a.P) && id != -1) sckv_report(a.status, SCKV_ERR_BOUNDS, id, KID_FREE);
    // keys: valid -> (id << 32 | i), invalid -> max
    s.keys[i] = valid ? (((unsigned long long)(uint32_t)id << 32) | (unsigned)i) : ~0ULL;
    s.vals[i] = i;
    __syncthreads();
    bitonic_sort(s, kT);
    // first occurrence: sorted position j whose id differs from j-1
    {
      const int j = threadIdx.x;
      const unsigned long long kj = s.keys[j];
      bool first = kj != ~0ULL;
      if (first && j > 0) first = (s.keys[j - 1] >> 32) != (kj >> 32);
      const int orig = (int)(kj & 0xffffffffULL);
      if (kj != ~0ULL) keep_flag[orig] = first ? 1 : 0;
    }
    if (!valid && i < kT) keep_flag[i] = 0;
    __syncthreads();
    int keep = 0;
    if (valid && keep_flag[i]) keep = (a.state[id] == PAGE_ALLOCATED) ? 1 : 0;
    int total = 0;
    const int pos = block_exclusive_scan(keep, &total, s);
    const int64_t tail = a.ctl[CTL_TAIL];
    if (keep) {
      a.ring[(tail + pos) % a.P] = id;
      a.state[id] = PAGE_FREE;
      a.pin[id] = 0;
      a.last_used[id] = 0;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      a.ctl[CTL_TAIL] = tail + total;
      a.ctl[CTL_EVICTIONS] += total;
      a.ctl[CTL_ALLOCATED] -= total;
    }
    __syncthreads();
  }
}

// Drop one pin from each listed page, in list order; a page whose pin count
// reaches zero goes to the ring tail (FIFO) — or, with keep_cached, stays
// allocated as an LRU eviction candidate. Ids in one call must be distinct.
__global__ void __launch_bounds__(kT) release_kernel(AllocView a, const int32_t* ids, int n, int keep_cached) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  SelectSmem& s = *reinterpret_cast<SelectSmem*>(smem_raw);
  for (int base = 0; base < n; base += kT) {
    const int i = base + threadIdx.x;
    int freed = 0;
    int32_t id = -1;
    if (i < n) {
      id = ids[i];
      if (id >= 0 && id < a.P && a.state[id] == PAGE_ALLOCATED) {
        const int old = atomicSub(&a.pin[id], 1);
        if (old <= 0) {
          atomicAdd(&a.pin[id], 1);
          sckv_report(a.status, SCKV_ERR_INVALID_ARG, id, KID_PIN);
        } else if (old == 1 && !keep_cached) {
          freed = 1;
        }
      } else if (id != -1) {
        sckv_report(a.status, SCKV_ERR_BOUNDS, id, KID_PIN);
      }
    }
    int total = 0;
    const int pos = block_exclusive_scan(freed, &total, s);
    const int64_t tail = a.ctl[CTL_TAIL];
    if (freed) {
      a.ring[(tail + pos) % a.P] = id;
      a.state[id] = PAGE_FREE;
      a.last_used[id] = 0;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      a.ctl[CTL_TAIL] = tail + total;
      a.ctl[CTL_ALLOCATED] -= total;
    }
    __syncthreads();
  }
}

__global__ void touch_kernel(AllocView a, const int32_t* ids, int n) {
  const int64_t clock0 = a.ctl[CTL_CLOCK];
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    const int32_t id = ids[i];
    if (id < 0) continue;
    if (id >= a.P) { sckv_report(a.status, SCKV_ERR_BOUNDS, id, KID_TOUCH); continue; }
    if (a.state[id] != PAGE_ALLOCATED) continue;
    atomicMax(reinterpret_cast<unsigned long long*>(&a.last_used[id]), (unsigned long long)(clock0 + 1 + i));
  }
}

__global__ void touch_finish_kernel(AllocView a, int n) { a.ctl[CTL_CLOCK] += n; }

__global__ void pin_kernel(AllocView a, const int32_t* ids, int n, int delta) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    const int32_t id = ids[i];
    if (id < 0 || id >= a.P) { sckv_report(a.status, SCKV_ERR_BOUNDS, id, KID_PIN); continue; }
    const int old = atomicAdd(&a.pin[id], delta);
    if (old + delta < 0) {
      atomicAdd(&a.pin[id], -delta);
      sckv_report(a.status, SCKV_ERR_INVALID_ARG, id, KID_PIN);
    }
  }
}

// LRU eviction of n pages, or (watermark >= 0) of as many as bring the
// allocated count down to the watermark, read on the device.
__global__ void __launch_bounds__(kT) evict_kernel(AllocView a, int n, int64_t watermark, int32_t* out_ids,
                                                   int32_t* out_count) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  SelectSmem& s = *reinterpret_cast<SelectSmem*>(smem_raw);
  if (watermark >= 0) {
    const int64_t over = a.ctl[CTL_ALLOCATED] - watermark;
    n = over > 0 ? (int)(over < a.P ? over : a.P) : 0;
  }
  int done = 0;
  unsigned long long lo = 0;
  while (done < n) {
    const int want = (n - done) < kSortCap ? (n - done) : kSortCap;
    const int got = select_smallest(a, lo, want, s);
    if (got == 0) break;
    const int64_t tail = a.ctl[CTL_TAIL];
    __syncthreads();
    for (int k = threadIdx.x; k < got; k += kT) {
      const int32_t id = s.vals[k];
      a.ring[(tail + k) % a.P] = id;
      a.state[id] = PAGE_FREE;
      a.last_used[id] = 0;
      if (out_ids) out_ids[done + k] = id;
    }
    lo = s.keys[got - 1];
    __syncthreads();
    if (threadIdx.x == 0) {
      a.ctl[CTL_TAIL] = tail + got;
      a.ctl[CTL_EVICTIONS] += got;
      a.ctl[CTL_ALLOCATED] -= got;
    }
    __syncthreads();
    done += got;
    if (got < want) break;
  }
  if (out_ids)
    for (int k = done + threadIdx.x; k < n; k += kT) out_ids[k] = -1;
  if (out_count && threadIdx.x == 0) *out_count = done;
}

// Decode-step reservation: sequences whose next token starts a page get one,
// in sequence order (the k-th such sequence receives the k-th allocation).
__global__ void __launch_bounds__(kT) reserve_kernel(AllocView a, int32_t* bt, int64_t stride, int max_blocks,
                                                     int32_t* ctx_lens, int n_seqs) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  SelectSmem& s = *reinterpret_cast<SelectSmem*>(smem_raw);
  __shared__ int32_t page_of_rank[kT];
  // Validate lengths and check capacity first, so a failing call changes nothing.
  int need_local = 0, bad_local = 0;
  for (int b = threadIdx.x; b < n_seqs; b += kT) {
    const int ctx = ctx_lens[b];
    if (ctx < 0 || ctx >= max_blocks * SCKV_PAGE_TOKENS) {
      sckv_report(a.status, SCKV_ERR_BOUNDS, b, KID_RESERVE);
      ++bad_local;
    } else if (ctx % SCKV_PAGE_TOKENS == 0) {
      ++need_local;
    }
  }
  const int n_need = block_sum_int(need_local, s);
  const int n_bad = block_sum_int(bad_local, s);
  if (n_bad > 0) return;
  int cand_local = 0;
  for (int64_t i = threadIdx.x; i < a.P; i += kT) cand_local += is_candidate(a, i) ? 1 : 0;
  const int n_cand = block_sum_int(cand_local, s);
  const int64_t avail = a.ctl[CTL_TAIL] - a.ctl[CTL_HEAD];
  __syncthreads();
  if ((int64_t)n_need > avail + n_cand) {
    if (threadIdx.x == 0) sckv_report(a.status, SCKV_ERR_POOL_EXHAUSTED, n_need, KID_RESERVE);
    return;
  }
  for (int base = 0; base < n_seqs; base += kT) {
    const int b = base + threadIdx.x;
    int needs = 0;
    if (b < n_seqs) needs = (ctx_lens[b] % SCKV_PAGE_TOKENS == 0) ? 1 : 0;
    int total = 0;
    const int r = block_exclusive_scan(needs, &total, s);
    if (total > 0) {
      if (!alloc_core(a, total, 1, s, [&](int k, int32_t id, int32_t) { page_of_rank[k] = id; }, KID_RESERVE))
        return;
      if (needs) {
        const int ctx = ctx_lens[b];
        bt[(int64_t)b * stride + ctx / SCKV_PAGE_TOKENS] = page_of_rank[r];
      }
    }
    __syncthreads();
  }
  for (int b = threadIdx.x; b < n_seqs; b += kT) ctx_lens[b] = ctx_lens[b] + 1;
}

constexpr size_t kSelectSmemBytes = sizeof(SelectSmem);

int configure(const void* fn) {
  SCKV_CUDA_CHECK(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSelectSmemBytes));
  return SCKV_OK;
}

int ensure_configured(int device) {
  static bool done[64] = {};
  if (device < 0 || device >= 64) return SCKV_ERR_INVALID_ARG;
  if (done[device]) return SCKV_OK;
  int rc = configure(reinterpret_cast<const void*>(alloc_kernel));
  if (rc == SCKV_OK) rc = configure(reinterpret_cast<const void*>(free_kernel));
  if (rc == SCKV_OK) rc = configure(reinterpret_cast<const void*>(evict_kernel));
  if (rc == SCKV_OK) rc = configure(reinterpret_cast<const void*>(reserve_kernel));
  if (rc == SCKV_OK) rc = configure(reinterpret_cast<const void*>(release_kernel));
  if (rc == SCKV_OK) done[device] = true;
  return rc;
}

}  // namespace

extern "C" int sckv_alloc_reset(sckv_pool* p, void* stream) {
  if (p == nullptr) return SCKV_ERR_INVALID_ARG;
  SCKV_DEVICE_GUARD(p->device);
  int rc = ensure_configured(p->device);
  if (rc != SCKV_OK) return rc;
  int64_t blocks = (p->max_pages + 255) / 256;
  if (blocks > (int64_t)p->num_sms * 8) blocks = (int64_t)p->num_sms * 8;
  if (blocks < 1) blocks = 1;
  reset_kernel<<<(int)blocks, 256, 0, as_stream(stream)>>>(view_of(p));
  SCKV_LAUNCH_CHECK();
  return SCKV_OK;
}

extern "C" int sckv_alloc_pages(sckv_pool* p, int n, int pin, int32_t* out_ids, int32_t* out_victims, void* stream) {
  if (p == nullptr || n < 0 || (n > 0 && out_ids == nullptr)) return SCKV_ERR_INVALID_ARG;
  if (n == 0) return SCKV_OK;
  SCKV_DEVICE_GUARD(p->device);
  int rc = ensure_configured(p->device);
  if (rc != SCKV_OK) return rc;
  alloc_kernel<<<1, kT, kSelectSmemBytes, as_stream(stream)>>>(view_of(p), n, pin ? 1 : 0, out_ids, out_victims);
  SCKV_LAUNCH_CHECK();
  return SCKV_OK;
}

extern "C" int sckv_free_pages(sckv_pool* p, const int32_t* ids, int n, void* stream) {
  if (p == nullptr || n < 0 || (n > 0 && ids == nullptr)) return SCKV_ERR_INVALID_ARG;
  if (n == 0) return SCKV_OK;
  SCKV_DEVICE_GUARD(p->device);
  int rc = ensure_configured(p->device);
  if (rc != SCKV_OK) return rc;
  free_kernel<<<1, kT, kSelectSmemBytes, as_stream(stream)>>>(view_of(p), ids, n);
  SCKV_LAUNCH_CHECK();
  return SCKV_OK;
}

extern "C" int sckv_touch_pages(sckv_pool* p, const int32_t* ids, int n, void* stream) {
  if (p == nullptr || n < 0 || (n > 0 && ids == nullptr)) return SCKV_ERR_INVALID_ARG;
  if (n == 0) return SCKV_OK;
  SCKV_DEVICE_GUARD(p->device);
  cudaStream_t s = as_stream(stream);
  int blocks = (n + 255) / 256;
  if (blocks > p->num_sms * 4) blocks = p->num_sms * 4;
  touch_kernel<<<blocks, 256, 0, s>>>(view_of(p), ids, n);
  SCKV_LAUNCH_CHECK();
  touch_finish_kernel<<<1, 1, 0, s>>>(view_of(p), n);
  SCKV_LAUNCH_CHECK();
  return SCKV_OK;
}

extern "C" int sckv_pin_pages(sckv_pool* p, const int32_t* ids, int n, int delta, void* stream) {
  if (p == nullptr || n < 0 || (n > 0 && ids == nullptr)) return SCKV_ERR_INVALID_ARG;
  if (n == 0 || delta == 0) return SCKV_OK;
  SCKV_DEVICE_GUARD(p->device);
  int blocks = (n + 255) / 256;
  if (blocks > p->num_sms * 4) blocks = p->num_sms * 4;
  pin_kernel<<<blocks, 256, 0, as_stream(stream)>>>(view_of(p), ids, n, delta);
  SCKV_LAUNCH_CHECK();
  return SCKV_OK;
}

extern "C" int sckv_release_pages(sckv_pool* p, const int32_t* ids, int n, int keep_cached, void* stream) {
  if (p == nullptr || n < 0 || (n > 0 && ids == nullptr)) return SCKV_ERR_INVALID_ARG;
  if (n == 0) return SCKV_OK;
  SCKV_DEVICE_GUARD(p->device);
  int rc = ensure_configured(p->device);
  if (rc != SCKV_OK) return rc;
  release_kernel<<<1, kT, kSelectSmemBytes, as_stream(stream)>>>(view_of(p), ids, n, keep_cached ? 1 : 0);
  SCKV_LAUNCH_CHECK();
  return SCKV_OK;
}

extern "C" int sckv_evict_lru(sckv_pool* p, int n, int32_t* out_ids, void* stream) {
  if (p == nullptr || n < 0) return SCKV_ERR_INVALID_ARG;
  if (n == 0) return SCKV_OK;
  SCKV_DEVICE_GUARD(p->device);
  int rc = ensure_configured(p->device);
  if (rc != SCKV_OK) return rc;
  evict_kernel<<<1, kT, kSelectSmemBytes, as_stream(stream)>>>(view_of(p), n, -1, out_ids, nullptr);
  SCKV_LAUNCH_CHECK();
  return SCKV_OK;
}

extern "C" int sckv_evict_to_watermark(sckv_pool* p, int64_t max_allocated, int32_t* out_count, void* stream) {
  if (p == nullptr || max_allocated < 0) return SCKV_ERR_INVALID_ARG;
  SCKV_DEVICE_GUARD(p->device);
  int rc = ensure_configured(p->device);
  if (rc != SCKV_OK) return rc;
  evict_kernel<<<1, kT, kSelectSmemBytes, as_stream(stream)>>>(view_of(p), 0, max_allocated, nullptr, out_count);
  SCKV_LAUNCH_CHECK();
  return SCKV_OK;
}

extern "C" int sckv_reserve_decode(sckv_pool* p, int32_t* bt, int64_t stride, int max_blocks, int32_t* ctx_lens,
                                   int n_seqs, void* stream) {
  if (p == nullptr || n_seqs < 0 || max_blocks <= 0 || stride < max_blocks) return SCKV_ERR_INVALID_ARG;
  if (n_seqs == 0) return SCKV_OK;
  if (bt == nullptr || ctx_lens == nullptr) return SCKV_ERR_INVALID_ARG;
  SCKV_DEVICE_GUARD(p->device);
  int rc = ensure_configured(p->device);
  if (rc != SCKV_OK) return rc;
  reserve_kernel<<<1, kT, kSelectSmemBytes, as_stream(stream)>>>(view_of(p), bt, stride, max_blocks, ctx_lens,
                                                                 n_seqs);
  SCKV_LAUNCH_CHECK();
  return SCKV_OK;
}

extern "C" int sckv_alloc_state(const sckv_pool* p, int64_t out[5], void* stream) {
  if (p == nullptr || out == nullptr) return SCKV_ERR_INVALID_ARG;
  SCKV_DEVICE_GUARD(p->device);
  cudaStream_t s = as_stream(stream);
  SCKV_CUDA_CHECK(cudaMemcpyAsync(out, p->ctl, 5 * sizeof(int64_t), cudaMemcpyDeviceToHost, s));
  SCKV_CUDA_CHECK(cudaStreamSynchronize(s));
  return SCKV_OK;
}
