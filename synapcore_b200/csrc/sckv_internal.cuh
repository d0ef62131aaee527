// Internal definitions shared by the libsckv CUDA translation units.
#pragma once

#include <cuda_runtime.h>
#include <stdio.h>
#include <atomic>
#include <utility>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <cuda_fp8.h>
#include <stdint.h>

#include "sckv.h"

#define SCKV_PAGE_TOKENS 16

// Kernel ids recorded in status word slot 2.
enum SckvKernelId : int32_t {
  KID_APPEND = 1,
  KID_WRITE_PAGES = 2,
  KID_GATHER = 3,
  KID_COPY = 4,
  KID_DECODE = 5,
  KID_COMBINE = 6,
  KID_ALLOC = 7,
  KID_FREE = 8,
  KID_TOUCH = 9,
  KID_PIN = 10,
  KID_EVICT = 11,
  KID_RESERVE = 12,
  KID_PREFILL = 13,
  KID_QKV = 14,
  KID_SELFTEST = 15,
  KID_EXCHANGE = 16,
};

// Allocator control words (int64, device).
enum SckvCtl : int {
  CTL_HEAD = 0,       // ring head (monotonic)
  CTL_TAIL = 1,       // ring tail (monotonic); free = tail - head
  CTL_CLOCK = 2,      // step clock
  CTL_EVICTIONS = 3,  // evictions (LRU victims + explicit frees)
  CTL_ALLOCATED = 4,  // pages currently allocated
  CTL_WORDS = 8,
};

// Page states.
enum SckvPageState : int32_t { PAGE_FREE = 0, PAGE_ALLOCATED = 1 };

// Work counters for persistent kernels that claim items dynamically: each
// launch takes the next one round-robin (zeroed on its stream just before
// the launch), so launches on different streams do not share a counter
// unless more than SCKV_WORK_COUNTERS of them are in flight at once.
#define SCKV_WORK_COUNTERS 64

// Layout of the allocator region (alloc_state), each part 256-byte aligned:
//   int64 ctl[CTL_WORDS]
//   int32 status[4]
//   uint64 work[SCKV_WORK_COUNTERS]
//   int32 ring[P]
//   int64 last_used[P]
//   int32 pin[P]
//   int32 state[P]
struct sckv_pool {
  int num_layers;
  int num_kv_heads;
  int head_dim;
  int page_tokens;
  int64_t max_pages;
  int kv_dtype;
  int device;
  int owns_memory;
  void* data;
  void* scales;
  void* alloc_state;
  int64_t* ctl;
  int32_t* status;
  unsigned long long* work_counters;
  mutable unsigned int next_work_counter;  // host-side round-robin index (atomic)
  int32_t* ring;
  int64_t* last_used;
  int32_t* pin;
  int32_t* state;
  size_t data_bytes;
  size_t scale_bytes;
  size_t alloc_bytes;
  int num_sms;
  // TMA tensor map over the page data (a CUtensorMap, encoded on first use
  // by the tensor-core decode kernel).
  alignas(64) unsigned char tmap_kv[128];
  int tmap_ready;  // box shape code the map was encoded for (0 = not yet)
  // A second map with one-head boxes (prefill attention).
  alignas(64) unsigned char tmap_kv1[128];
  int tmap1_ready;
  // A third map with one-head, K-or-V boxes (tensor-memory prefill).
  alignas(64) unsigned char tmap_kv2[128];
  int tmap2_ready;
};

// KV-head-sharded output exchange between the ranks of one box (one process
// per GPU): a full-head output buffer and an epoch flag per source rank in
// this GPU's memory, plus the CUDA IPC mappings of every peer's buffer and
// flags (peer_out[rank] / peer_flags[rank] are the local ones).
struct sckv_exchange {
  int device;
  int world;
  int rank;
  void* out;
  size_t out_bytes;
  uint32_t* flags;   // [world]: the last epoch each rank signalled here
  int32_t* status;   // [4]: code, detail, kernel, count (as a pool's status word)
  uint32_t* counter; // the last epoch this rank signalled (device; epoch 0 calls continue from it)
  void* peer_out[8];
  uint32_t* peer_flags[8];
  int opened[8];
};

namespace sckv_detail {
// Stream-ordered after a rank's exchange decode: flags[rank] = epoch on every
// rank (release, system scope), once the decode's peer stores are complete.
int launch_exchange_signal(const sckv_exchange* ex, uint32_t epoch, cudaStream_t stream);
}  // namespace sckv_detail

// Next work counter of the pool for one launch (thread-safe on the host).
static inline unsigned long long* sckv_take_work_counter(const sckv_pool* p) {
  const unsigned int i = __atomic_fetch_add(&p->next_work_counter, 1u, __ATOMIC_RELAXED);
  return p->work_counters + (i % SCKV_WORK_COUNTERS);
}

static inline int sckv_elem_bytes(int dtype) {
  switch (dtype) {
    case SCKV_DTYPE_F16:
    case SCKV_DTYPE_BF16: return 2;
    case SCKV_DTYPE_INT8:
    case SCKV_DTYPE_FP8_E4M3: return 1;
    case SCKV_DTYPE_F32: return 4;
    default: return 0;
  }
}

// Elements of one (layer, page) slab: 2 * H * T * D.
static inline int64_t sckv_slab_elems(const sckv_pool* p) {
  return 2LL * p->num_kv_heads * p->page_tokens * p->head_dim;
}

// ---------------------------------------------------------------------------
// Status word: first error wins (code, detail, kernel), count accumulates.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void sckv_report(int32_t* status, int32_t code,
                                            int32_t detail, int32_t kernel) {
  if (status == nullptr) return;
  if (atomicCAS(&status[0], 0, code) == 0) {
    status[1] = detail;
    status[2] = kernel;
  }
  atomicAdd(&status[3], 1);
}

// Sequence of token t: the last b with cu[b] <= t (cu: n_seqs + 1 offsets).
__device__ __forceinline__ int sckv_find_seq(const int32_t* cu, int n_seqs, int t) {
  int lo = 0, hi = n_seqs - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (__ldg(cu + mid) <= t) lo = mid; else hi = mid - 1;
  }
  return lo;
}

// ---------------------------------------------------------------------------
// Value conversion helpers.
// ---------------------------------------------------------------------------
__device__ __forceinline__ float sckv_load_as_float(const void* base, int64_t idx, int dtype) {
  switch (dtype) {
    case SCKV_DTYPE_F16: return __half2float(reinterpret_cast<const __half*>(base)[idx]);
    case SCKV_DTYPE_BF16: return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(base)[idx]);
    default: return reinterpret_cast<const float*>(base)[idx];
  }
}

__device__ __forceinline__ void sckv_store_from_float(void* base, int64_t idx, int dtype, float v) {
  switch (dtype) {
    case SCKV_DTYPE_F16: reinterpret_cast<__half*>(base)[idx] = __float2half_rn(v); break;
    case SCKV_DTYPE_BF16: reinterpret_cast<__nv_bfloat16*>(base)[idx] = __float2bfloat16_rn(v); break;
    default: reinterpret_cast<float*>(base)[idx] = v; break;
  }
}

// e4m3 byte -> float (hardware conversion through f16; exact).
__device__ __forceinline__ float sckv_fp8_to_float(uint8_t b) {
  __half_raw hr = __nv_cvt_fp8_to_halfraw(static_cast<__nv_fp8_storage_t>(b), __NV_E4M3);
  return __half2float(__half(hr));
}

// float -> e4m3 byte, round to nearest even, saturating to +-448.
__device__ __forceinline__ uint8_t sckv_float_to_fp8(float x) {
  return static_cast<uint8_t>(__nv_cvt_float_to_fp8(x, __NV_SATFINITE, __NV_E4M3));
}

// ---------------------------------------------------------------------------
// PTX wrappers: shared-memory mbarriers and bulk (TMA, non-tensor) copies.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Bounded wait on an mbarrier phase. Returns false after `limit_ns` of
// waiting (the caller records SCKV_ERR_TIMEOUT and winds down).
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity,
                                                  uint64_t limit_ns) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (globaltimer_ns() - t0 > limit_ns) return false;
  }
}

// Global -> shared bulk copy completing on an mbarrier (bytes % 16 == 0,
// both addresses 16-byte aligned).
__device__ __forceinline__ void bulk_g2s(void* dst_smem, const void* src_gmem, uint32_t bytes,
                                         uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst_smem)),
      "l"(src_gmem), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void named_bar_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// Error helpers for host code. A failing CUDA call leaves a description
// ("file:line what: error name") in a per-thread buffer that
// sckv_last_error() returns, so SCKV_ERR_CUDA can be traced to its call.
inline char* sckv_error_buffer() {
  static thread_local char buf[256] = {0};
  return buf;
}

inline int sckv_record_error(const char* file, int line, const char* what, const char* err) {
  const char* base = file;
  for (const char* c = file; *c; ++c)
    if (*c == '/') base = c + 1;
  // bounded fields: the message fits the 256-byte buffer
  snprintf(sckv_error_buffer(), 256, "%.64s:%d %.96s: %.64s", base, line, what, err);
  return SCKV_ERR_CUDA;
}

#define SCKV_CUDA_CHECK(expr)                                                            \
  do {                                                                                   \
    cudaError_t _e = (expr);                                                             \
    if (_e != cudaSuccess) return sckv_record_error(__FILE__, __LINE__, #expr, cudaGetErrorName(_e)); \
  } while (0)

// Makes a pool's device current for the rest of the enclosing scope and puts
// the calling thread's previous device back on exit, so no entry point leaves
// the caller on another GPU.
class SckvDeviceGuard {
 public:
  SckvDeviceGuard() = default;
  SckvDeviceGuard(const SckvDeviceGuard&) = delete;
  SckvDeviceGuard& operator=(const SckvDeviceGuard&) = delete;
  cudaError_t enter(int dev) {
    cudaError_t e = cudaGetDevice(&prev_);
    if (e != cudaSuccess) return e;
    if (prev_ == dev) return cudaSuccess;
    e = cudaSetDevice(dev);
    if (e == cudaSuccess) switched_ = true;
    return e;
  }
  ~SckvDeviceGuard() {
    if (switched_) cudaSetDevice(prev_);
  }

 private:
  int prev_ = 0;
  bool switched_ = false;
};

#define SCKV_DEVICE_GUARD(dev)           \
  SckvDeviceGuard _sckv_device_guard;    \
  SCKV_CUDA_CHECK(_sckv_device_guard.enter(dev))

// Kernels launched by this library in this process (every launch site is
// followed by exactly one SCKV_LAUNCH_CHECK, which counts it).
inline std::atomic<unsigned long long>& sckv_launch_counter() {
  static std::atomic<unsigned long long> n{0};
  return n;
}

// Programmatic dependent launch. A kernel launched with sckv_launch_pdl may
// start while the kernel before it in the stream is still running (once
// that one has called pdl_trigger or finished); it must call pdl_wait before
// it reads anything an earlier kernel wrote, which waits for the earlier
// kernel to complete and its memory to be visible. Kernels call pdl_trigger
// after their own pdl_wait, so a dependent never starts before the kernel
// two places back has completed.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

template <typename... KArgs, typename... Args>
inline cudaError_t sckv_launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem,
                                   cudaStream_t stream, Args&&... args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

#define SCKV_LAUNCH_CHECK()                                                              \
  do {                                                                                   \
    sckv_launch_counter().fetch_add(1, std::memory_order_relaxed);                       \
    cudaError_t _e = cudaGetLastError();                                                 \
    if (_e != cudaSuccess) return sckv_record_error(__FILE__, __LINE__, "kernel launch", cudaGetErrorName(_e)); \
  } while (0)

static inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

// Wait limit for in-kernel barrier waits: 2 seconds.
#define SCKV_WAIT_LIMIT_NS 2000000000ULL
