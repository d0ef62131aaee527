// Pool lifetime, device pointers and the status word.
#include <new>

#include "sckv_internal.cuh"

namespace {

constexpr size_t kAlign = 256;

inline size_t align_up(size_t x) { return (x + kAlign - 1) / kAlign * kAlign; }

struct AllocLayout {
  size_t ctl, status, work, ring, last_used, pin, state, total;
};

AllocLayout alloc_layout(int64_t P) {
  AllocLayout a{};
  size_t off = 0;
  a.ctl = off;       off = align_up(off + CTL_WORDS * sizeof(int64_t));
  a.status = off;    off = align_up(off + 4 * sizeof(int32_t));
  a.work = off;      off = align_up(off + SCKV_WORK_COUNTERS * sizeof(unsigned long long));
  a.ring = off;      off = align_up(off + static_cast<size_t>(P) * sizeof(int32_t));
  a.last_used = off; off = align_up(off + static_cast<size_t>(P) * sizeof(int64_t));
  a.pin = off;       off = align_up(off + static_cast<size_t>(P) * sizeof(int32_t));
  a.state = off;     off = align_up(off + static_cast<size_t>(P) * sizeof(int32_t));
  a.total = off;
  return a;
}

int validate_geometry(int L, int H, int D, int T, int64_t P, int dtype) {
  if (L <= 0 || H <= 0 || D <= 0 || P <= 0) return SCKV_ERR_INVALID_ARG;
  if (T != SCKV_PAGE_TOKENS) return SCKV_ERR_INVALID_ARG;
  if (D % 16 != 0 || D > 256) return SCKV_ERR_INVALID_ARG;
  if (P > INT32_MAX - 1) return SCKV_ERR_INVALID_ARG;
  if (dtype != SCKV_DTYPE_F16 && dtype != SCKV_DTYPE_BF16 && dtype != SCKV_DTYPE_INT8 &&
      dtype != SCKV_DTYPE_FP8_E4M3)
    return SCKV_ERR_INVALID_ARG;
  return SCKV_OK;
}

}  // namespace

extern "C" int sckv_alloc_reset(sckv_pool* pool, void* stream);

extern "C" int sckv_pool_required_bytes(int L, int H, int D, int T, int64_t P, int dtype,
                                        size_t* data_bytes, size_t* scale_bytes,
                                        size_t* alloc_bytes) {
  int rc = validate_geometry(L, H, D, T, P, dtype);
  if (rc != SCKV_OK) return rc;
  const size_t slab = 2ULL * H * T * D;
  const size_t data = static_cast<size_t>(L) * static_cast<size_t>(P) * slab * sckv_elem_bytes(dtype);
  size_t scales = 0;
  if (dtype == SCKV_DTYPE_INT8) scales = static_cast<size_t>(L) * P * 2ULL * H * T * sizeof(__half);
  // fp8 scales are staged with 16-byte bulk copies of aligned 4-float blocks:
  // pad so the last block stays inside the region.
  if (dtype == SCKV_DTYPE_FP8_E4M3) scales = (static_cast<size_t>(L) * P * 2ULL * H * sizeof(float) + 63) / 64 * 64;
  if (data_bytes) *data_bytes = data;
  if (scale_bytes) *scale_bytes = scales;
  if (alloc_bytes) *alloc_bytes = alloc_layout(P).total;
  return SCKV_OK;
}

static int pool_init_common(sckv_pool* p, int L, int H, int D, int T, int64_t P, int dtype,
                            int device) {
  p->num_layers = L;
  p->num_kv_heads = H;
  p->head_dim = D;
  p->page_tokens = T;
  p->max_pages = P;
  p->kv_dtype = dtype;
  p->device = device;
  sckv_pool_required_bytes(L, H, D, T, P, dtype, &p->data_bytes, &p->scale_bytes, &p->alloc_bytes);
  AllocLayout a = alloc_layout(P);
  char* base = static_cast<char*>(p->alloc_state);
  p->ctl = reinterpret_cast<int64_t*>(base + a.ctl);
  p->status = reinterpret_cast<int32_t*>(base + a.status);
  p->work_counters = reinterpret_cast<unsigned long long*>(base + a.work);
  p->ring = reinterpret_cast<int32_t*>(base + a.ring);
  p->last_used = reinterpret_cast<int64_t*>(base + a.last_used);
  p->pin = reinterpret_cast<int32_t*>(base + a.pin);
  p->state = reinterpret_cast<int32_t*>(base + a.state);
  int sms = 0;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device) != cudaSuccess) return SCKV_ERR_CUDA;
  p->num_sms = sms;
  return SCKV_OK;
}

extern "C" int sckv_pool_create(int L, int H, int D, int T, int64_t P, int dtype, int device,
                                sckv_pool** out) {
  if (out == nullptr) return SCKV_ERR_INVALID_ARG;
  *out = nullptr;
  int rc = validate_geometry(L, H, D, T, P, dtype);
  if (rc != SCKV_OK) return rc;
  SCKV_DEVICE_GUARD(device);
  size_t data_b = 0, scale_b = 0, alloc_b = 0;
  sckv_pool_required_bytes(L, H, D, T, P, dtype, &data_b, &scale_b, &alloc_b);
  sckv_pool* p = new (std::nothrow) sckv_pool{};
  if (p == nullptr) return SCKV_ERR_INVALID_ARG;
  p->owns_memory = 1;
  if (cudaMalloc(&p->data, data_b) != cudaSuccess) { delete p; return SCKV_ERR_CUDA; }
  if (scale_b && cudaMalloc(&p->scales, scale_b) != cudaSuccess) {
    cudaFree(p->data); delete p; return SCKV_ERR_CUDA;
  }
  if (cudaMalloc(&p->alloc_state, alloc_b) != cudaSuccess) {
    cudaFree(p->data); if (p->scales) cudaFree(p->scales); delete p; return SCKV_ERR_CUDA;
  }
  rc = pool_init_common(p, L, H, D, T, P, dtype, device);
  if (rc == SCKV_OK && cudaMemset(p->data, 0, data_b) != cudaSuccess) rc = SCKV_ERR_CUDA;
  if (rc == SCKV_OK && scale_b && cudaMemset(p->scales, 0, scale_b) != cudaSuccess) rc = SCKV_ERR_CUDA;
  if (rc == SCKV_OK) rc = sckv_alloc_reset(p, nullptr);
  if (rc == SCKV_OK && cudaDeviceSynchronize() != cudaSuccess) rc = SCKV_ERR_CUDA;
  if (rc != SCKV_OK) { sckv_pool_destroy(p); return rc; }
  *out = p;
  return SCKV_OK;
}

extern "C" int sckv_pool_wrap(int L, int H, int D, int T, int64_t P, int dtype, int device, void* data,
                              void* scales, void* alloc_state, sckv_pool** out) {
  if (out == nullptr) return SCKV_ERR_INVALID_ARG;
  *out = nullptr;
  int rc = validate_geometry(L, H, D, T, P, dtype);
  if (rc != SCKV_OK) return rc;
  if (data == nullptr || alloc_state == nullptr) return SCKV_ERR_INVALID_ARG;
  if ((dtype == SCKV_DTYPE_INT8 || dtype == SCKV_DTYPE_FP8_E4M3) && scales == nullptr) return SCKV_ERR_INVALID_ARG;
  if ((reinterpret_cast<uintptr_t>(data) & 15) || (reinterpret_cast<uintptr_t>(alloc_state) & 15) ||
      (scales && (reinterpret_cast<uintptr_t>(scales) & 15)))
    return SCKV_ERR_ALIGNMENT;
  sckv_pool* p = new (std::nothrow) sckv_pool{};
  if (p == nullptr) return SCKV_ERR_INVALID_ARG;
  p->owns_memory = 0;
  p->data = data;
  p->scales = (dtype == SCKV_DTYPE_INT8 || dtype == SCKV_DTYPE_FP8_E4M3) ? scales : nullptr;
  p->alloc_state = alloc_state;
  rc = pool_init_common(p, L, H, D, T, P, dtype, device);
  if (rc != SCKV_OK) { delete p; return rc; }
  *out = p;
  return SCKV_OK;
}

extern "C" void sckv_pool_destroy(sckv_pool* p) {
  if (p == nullptr) return;
  if (p->owns_memory) {
    SckvDeviceGuard guard;
    guard.enter(p->device);
    if (p->data) cudaFree(p->data);
    if (p->scales) cudaFree(p->scales);
    if (p->alloc_state) cudaFree(p->alloc_state);
  }
  delete p;
}

extern "C" int sckv_pool_pointers(const sckv_pool* p, void** data, void** scales, void** alloc_state) {
  if (p == nullptr) return SCKV_ERR_INVALID_ARG;
  if (data) *data = p->data;
  if (scales) *scales = p->scales;
  if (alloc_state) *alloc_state = p->alloc_state;
  return SCKV_OK;
}

extern "C" int sckv_get_status(const sckv_pool* p, int32_t out[4], void* stream) {
  if (p == nullptr || out == nullptr) return SCKV_ERR_INVALID_ARG;
  cudaStream_t s = as_stream(stream);
  SCKV_CUDA_CHECK(cudaMemcpyAsync(out, p->status, 4 * sizeof(int32_t), cudaMemcpyDeviceToHost, s));
  SCKV_CUDA_CHECK(cudaStreamSynchronize(s));
  return SCKV_OK;
}

extern "C" int sckv_clear_status(sckv_pool* p, void* stream) {
  if (p == nullptr) return SCKV_ERR_INVALID_ARG;
  SCKV_CUDA_CHECK(cudaMemsetAsync(p->status, 0, 4 * sizeof(int32_t), as_stream(stream)));
  return SCKV_OK;
}

namespace {

// Waits on an mbarrier nothing ever arrives on, with the bounded wait every
// pipeline kernel uses: it gives up after limit_ns and records
// SCKV_ERR_TIMEOUT (detail -1) in the pool's status word, as a stalled
// pipeline would.
__global__ void selftest_wait_kernel(int32_t* status, uint64_t limit_ns) {
  __shared__ uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0 && !mbar_wait_bounded(&bar, 0, limit_ns))
    sckv_report(status, SCKV_ERR_TIMEOUT, -1, KID_SELFTEST);
}

}  // namespace

extern "C" int sckv_selftest_wait_timeout(sckv_pool* p, unsigned limit_us, void* stream) {
  if (p == nullptr || limit_us == 0 || limit_us > 2000000u) return SCKV_ERR_INVALID_ARG;
  SCKV_DEVICE_GUARD(p->device);
  selftest_wait_kernel<<<1, 32, 0, as_stream(stream)>>>(p->status, (uint64_t)limit_us * 1000ull);
  SCKV_LAUNCH_CHECK();
  return SCKV_OK;
}

extern "C" const char* sckv_version(void) { return "sckv 0.1.0 sm_100a"; }

extern "C" const char* sckv_last_error(void) { return sckv_error_buffer(); }

extern "C" unsigned long long sckv_launch_count(void) {
  return sckv_launch_counter().load(std::memory_order_relaxed);
}

extern "C" const char* sckv_status_string(int code) {
  switch (code) {
    case SCKV_OK: return "ok";
    case SCKV_ERR_INVALID_ARG: return "invalid argument";
    case SCKV_ERR_BOUNDS: return "index out of bounds";
    case SCKV_ERR_ALIGNMENT: return "misaligned pointer";
    case SCKV_ERR_CUDA: return "CUDA runtime error";
    case SCKV_ERR_POOL_EXHAUSTED: return "page pool exhausted";
    case SCKV_ERR_TIMEOUT: return "in-kernel wait timed out";
    case SCKV_ERR_UNSUPPORTED: return "unsupported dtype or shape";
    case SCKV_ERR_SCRATCH_LIMIT: return "request exceeds the fixed no-allocation scratch";
    default: return "unknown status";
  }
}
