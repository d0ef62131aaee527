// KV-head-sharded output exchange over NVLink (one process per GPU of a box).
//
// In the KV-head-sharded layout every rank holds all sequences but only
// kv heads [r*Hkv/n, (r+1)*Hkv/n) and the q heads that read them; after each
// layer every rank needs the full [B, Hq, D] attention output. Instead of a
// separate all-gather, sckv_decode_attn_exchange (sckv_decode.cu) makes the
// decode epilogue store each output element into every rank's full-head
// buffer directly (plain stores through CUDA IPC mappings, so the bytes cross
// NVLink while the attention of other items is still running), and this file
// supplies the rest:
//   * the exchange object: a full-head output buffer and a flag word per
//     source rank in this GPU's memory, exported as CUDA IPC handles and
//     mapped by every peer;
//   * exchange_signal_kernel: stream-ordered after a rank's decode (whose
//     kernels have then completed), a system-scope fence and a release store
//     of the call's epoch into flags[rank] on every rank;
//   * exchange_wait_kernel: an acquire spin on the local flags until every
//     rank's epoch reached the awaited one, bounded in time; on expiry it
//     records SCKV_ERR_TIMEOUT (detail = the rank that is late) in the
//     exchange's status word and returns, so the context stays usable.
// Epochs are either passed by the caller or, with epoch 0, taken from a
// device counter of this rank's signals (next = last + 1; the wait then
// awaits the last one signalled), so a step of several layers can be
// captured once in a CUDA graph and replayed.
// No TMA or multicast touches peer memory; only ordinary stores and the flag
// loads / stores do.
#include <cstring>
#include <new>

#include "sckv_internal.cuh"

namespace {

constexpr int kMaxRanks = 8;
constexpr size_t kCtlBytes = 256;  // flags [8] u32 at 0, status [4] i32 at 128, epoch counter u32 at 192

struct SignalArgs {
  uint32_t* flags[kMaxRanks];
  uint32_t* counter;
  int world;
  int rank;
  uint32_t epoch;  // 0: the counter's next
};

__global__ void exchange_signal_kernel(SignalArgs a) {
  const int r = threadIdx.x;
  const uint32_t e = a.epoch != 0 ? a.epoch : *a.counter + 1u;
  __syncthreads();  // every thread has read the counter before it moves
  if (r == 0) *a.counter = e;
  if (r >= a.world) return;
  // the decode launches before this kernel in the stream have completed;
  // their stores to every rank's buffer become visible system-wide before
  // the flag does
  __threadfence_system();
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(a.flags[r] + a.rank), "r"(e) : "memory");
}

__global__ void exchange_wait_kernel(const uint32_t* flags, int world, uint32_t epoch_arg, const uint32_t* counter,
                                     int32_t* status, unsigned long long limit_ns) {
  const int r = threadIdx.x;
  // epoch 0: the last epoch this rank signalled (none yet: nothing to wait for)
  const uint32_t epoch = epoch_arg != 0 ? epoch_arg : *counter;
  if (r < world && epoch != 0) {
    const uint64_t t0 = globaltimer_ns();
    for (;;) {
      uint32_t v;
      asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(flags + r) : "memory");
      if ((int32_t)(v - epoch) >= 0) break;
      if (globaltimer_ns() - t0 > limit_ns) {
        sckv_report(status, SCKV_ERR_TIMEOUT, r, KID_EXCHANGE);
        break;
      }
      __nanosleep(100);
    }
  }
  __threadfence();
}

bool valid_ex(const sckv_exchange* ex) { return ex != nullptr && ex->world >= 1 && ex->world <= kMaxRanks; }

}  // namespace

namespace sckv_detail {

int launch_exchange_signal(const sckv_exchange* ex, uint32_t epoch, cudaStream_t stream) {
  SignalArgs a{};
  for (int r = 0; r < ex->world; ++r) a.flags[r] = ex->peer_flags[r];
  a.counter = ex->counter;
  a.world = ex->world;
  a.rank = ex->rank;
  a.epoch = epoch;
  exchange_signal_kernel<<<1, 32, 0, stream>>>(a);
  SCKV_LAUNCH_CHECK();
  return SCKV_OK;
}

}  // namespace sckv_detail

extern "C" int sckv_exchange_create(int device, int world, int rank, size_t out_bytes, sckv_exchange** out) {
  if (out == nullptr) return SCKV_ERR_INVALID_ARG;
  *out = nullptr;
  if (device < 0 || world < 1 || world > kMaxRanks || rank < 0 || rank >= world || out_bytes == 0)
    return SCKV_ERR_INVALID_ARG;
  SCKV_DEVICE_GUARD(device);
  sckv_exchange* ex = new (std::nothrow) sckv_exchange{};
  if (ex == nullptr) return SCKV_ERR_INVALID_ARG;
  ex->device = device;
  ex->world = world;
  ex->rank = rank;
  ex->out_bytes = (out_bytes + 255) & ~size_t(255);
  void* ctl = nullptr;
  if (cudaMalloc(&ex->out, ex->out_bytes) != cudaSuccess || cudaMalloc(&ctl, kCtlBytes) != cudaSuccess ||
      cudaMemset(ctl, 0, kCtlBytes) != cudaSuccess || cudaMemset(ex->out, 0, ex->out_bytes) != cudaSuccess ||
      cudaDeviceSynchronize() != cudaSuccess) {
    if (ex->out) cudaFree(ex->out);
    if (ctl) cudaFree(ctl);
    delete ex;
    return sckv_record_error(__FILE__, __LINE__, "exchange buffers", "allocation failed");
  }
  ex->flags = reinterpret_cast<uint32_t*>(ctl);
  ex->status = reinterpret_cast<int32_t*>(reinterpret_cast<uint8_t*>(ctl) + 128);
  ex->counter = reinterpret_cast<uint32_t*>(reinterpret_cast<uint8_t*>(ctl) + 192);
  ex->peer_out[rank] = ex->out;
  ex->peer_flags[rank] = ex->flags;
  ex->opened[rank] = 1;
  *out = ex;
  return SCKV_OK;
}

extern "C" void* sckv_exchange_buffer(const sckv_exchange* ex) { return valid_ex(ex) ? ex->out : nullptr; }

extern "C" int sckv_exchange_ipc_handles(const sckv_exchange* ex, uint8_t* out_handles) {
  if (!valid_ex(ex) || out_handles == nullptr) return SCKV_ERR_INVALID_ARG;
  SCKV_DEVICE_GUARD(ex->device);
  cudaIpcMemHandle_t h;
  SCKV_CUDA_CHECK(cudaIpcGetMemHandle(&h, ex->out));
  memcpy(out_handles, &h, sizeof(h));
  SCKV_CUDA_CHECK(cudaIpcGetMemHandle(&h, ex->flags));
  memcpy(out_handles + sizeof(h), &h, sizeof(h));
  return SCKV_OK;
}

extern "C" int sckv_exchange_open_peer(sckv_exchange* ex, int peer, const uint8_t* handles) {
  if (!valid_ex(ex) || handles == nullptr || peer < 0 || peer >= ex->world) return SCKV_ERR_INVALID_ARG;
  if (peer == ex->rank || ex->opened[peer]) return SCKV_OK;
  SCKV_DEVICE_GUARD(ex->device);
  cudaIpcMemHandle_t h;
  void* p_out = nullptr;
  void* p_ctl = nullptr;
  memcpy(&h, handles, sizeof(h));
  SCKV_CUDA_CHECK(cudaIpcOpenMemHandle(&p_out, h, cudaIpcMemLazyEnablePeerAccess));
  memcpy(&h, handles + sizeof(h), sizeof(h));
  const cudaError_t e = cudaIpcOpenMemHandle(&p_ctl, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) {
    cudaIpcCloseMemHandle(p_out);
    return sckv_record_error(__FILE__, __LINE__, "cudaIpcOpenMemHandle(flags)", cudaGetErrorName(e));
  }
  ex->peer_out[peer] = p_out;
  ex->peer_flags[peer] = reinterpret_cast<uint32_t*>(p_ctl);
  ex->opened[peer] = 1;
  return SCKV_OK;
}

extern "C" int sckv_exchange_wait(sckv_exchange* ex, uint32_t epoch, unsigned limit_us, void* stream) {
  if (!valid_ex(ex)) return SCKV_ERR_INVALID_ARG;
  const unsigned long long limit_ns =
      (limit_us == 0 || limit_us > 2000000u) ? SCKV_WAIT_LIMIT_NS : (unsigned long long)limit_us * 1000ull;
  SCKV_DEVICE_GUARD(ex->device);
  exchange_wait_kernel<<<1, 32, 0, as_stream(stream)>>>(ex->flags, ex->world, epoch, ex->counter, ex->status,
                                                         limit_ns);
  SCKV_LAUNCH_CHECK();
  return SCKV_OK;
}

extern "C" int sckv_exchange_status(const sckv_exchange* ex, int32_t out[4], int clear, void* stream) {
  if (!valid_ex(ex) || out == nullptr) return SCKV_ERR_INVALID_ARG;
  SCKV_DEVICE_GUARD(ex->device);
  cudaStream_t s = as_stream(stream);
  SCKV_CUDA_CHECK(cudaMemcpyAsync(out, ex->status, 4 * sizeof(int32_t), cudaMemcpyDeviceToHost, s));
  SCKV_CUDA_CHECK(cudaStreamSynchronize(s));
  if (clear) SCKV_CUDA_CHECK(cudaMemsetAsync(ex->status, 0, 4 * sizeof(int32_t), s));
  return SCKV_OK;
}

extern "C" void sckv_exchange_destroy(sckv_exchange* ex) {
  if (!valid_ex(ex)) return;
  SckvDeviceGuard guard;
  guard.enter(ex->device);
  cudaDeviceSynchronize();
  for (int r = 0; r < ex->world; ++r) {
    if (r == ex->rank || !ex->opened[r]) continue;
    cudaIpcCloseMemHandle(ex->peer_out[r]);
    cudaIpcCloseMemHandle(ex->peer_flags[r]);
  }
  cudaFree(ex->out);
  cudaFree(ex->flags);
  delete ex;
}
