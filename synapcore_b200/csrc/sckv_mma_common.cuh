// Tensor-core and TMA building blocks shared by the decode and prefill kernels.
#pragma once

#include <cuda.h>
#include <cudaTypedefs.h>

#include "sckv_internal.cuh"

namespace sckv_mma {

constexpr int kBoxBytes = 16 * 128;  // one TMA box: 16 rows x 128 bytes (swizzled)

template <int KVDT>
struct MmaKV;
template <>
struct MmaKV<SCKV_DTYPE_F16> {
  static constexpr int kEB = 2;
};
template <>
struct MmaKV<SCKV_DTYPE_BF16> {
  static constexpr int kEB = 2;
};
template <>
struct MmaKV<SCKV_DTYPE_FP8_E4M3> {
  static constexpr int kEB = 1;
};
template <>
struct MmaKV<SCKV_DTYPE_INT8> {
  static constexpr int kEB = 1;
};

// Byte address of (row, byte) inside a 128-byte-swizzled 16 x 128 B box.
__device__ __forceinline__ uint32_t swz(uint32_t box, int row, int byte) {
  return box + row * 128 + ((((byte >> 4) ^ (row & 7))) << 4) + (byte & 15);
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ uint32_t lds32(uint32_t addr) {
  uint32_t v;
  asm volatile("ld.shared.b32 %0, [%1];" : "=r"(v) : "r"(addr));
  return v;
}

__device__ __forceinline__ uint32_t movm_t(uint32_t a) {
  uint32_t d;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(d) : "r"(a));
  return d;
}

template <bool BF16>
__device__ __forceinline__ void mma16816(float c[4], const uint32_t a[4], uint32_t b0, uint32_t b1) {
  if (BF16) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  } else {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
}

__device__ __forceinline__ uint32_t fp8x2_to_f16x2(uint32_t two_bytes) {
  __half2_raw h = __nv_cvt_fp8x2_to_halfraw2(static_cast<__nv_fp8x2_storage_t>(two_bytes & 0xffffu), __NV_E4M3);
  return *reinterpret_cast<uint32_t*>(&h);
}

// Four e4m3 bytes -> two f16x2: bytes (0,1) -> lo, bytes (2,3) -> hi (exact).
__device__ __forceinline__ void cvt_fp8x4(uint32_t x, uint32_t& lo, uint32_t& hi) {
  asm("{\n\t.reg .b16 l16, h16;\n\tmov.b32 {l16, h16}, %2;\n\t"
      "cvt.rn.f16x2.e4m3x2 %0, l16;\n\tcvt.rn.f16x2.e4m3x2 %1, h16;\n\t}"
      : "=r"(lo), "=r"(hi)
      : "r"(x));
}

// 2^x by the hardware approximation (flushes denormals; 2^-inf = 0).
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Four int8 codes -> two f16x2 (exact), same byte order as cvt_fp8x4. Each
// byte, offset by 128, becomes the low byte of the f16 1024 + u (exponent
// field 25, so the 10 mantissa bits count units); subtracting 1152 leaves the
// code. (The bias-and-subtract construction of small integers in floating
// point, applied to f16.)
__device__ __forceinline__ void cvt_s8x4(uint32_t x, uint32_t& lo, uint32_t& hi) {
  const uint32_t u = x ^ 0x80808080u;
  const uint32_t l = __byte_perm(u, 0x64646464u, 0x4140);
  const uint32_t h = __byte_perm(u, 0x64646464u, 0x4342);
  const __half2 bias = __halves2half2(__ushort_as_half(0x6480), __ushort_as_half(0x6480));  // 1152
  const __half2 lv = __hsub2(*reinterpret_cast<const __half2*>(&l), bias);
  const __half2 hv = __hsub2(*reinterpret_cast<const __half2*>(&h), bias);
  lo = *reinterpret_cast<const uint32_t*>(&lv);
  hi = *reinterpret_cast<const uint32_t*>(&hv);
}

// One-byte codes -> two f16x2 in the byte order of cvt_fp8x4.
template <int KVDT>
__device__ __forceinline__ void cvt_b8x4(uint32_t x, uint32_t& lo, uint32_t& hi) {
  if (KVDT == SCKV_DTYPE_INT8) cvt_s8x4(x, lo, hi);
  else cvt_fp8x4(x, lo, hi);
}

// As cvt_b8x4, but int8 codes come out offset by +1152 (the f16 1024 + u
// before the subtraction): for callers that remove the offset from whole
// dot products instead of from every code.
template <int KVDT>
__device__ __forceinline__ void cvt_b8x4_biased(uint32_t x, uint32_t& lo, uint32_t& hi) {
  if (KVDT == SCKV_DTYPE_INT8) {
    const uint32_t u = x ^ 0x80808080u;
    lo = __byte_perm(u, 0x64646464u, 0x4140);
    hi = __byte_perm(u, 0x64646464u, 0x4342);
  } else {
    cvt_fp8x4(x, lo, hi);
  }
}

template <bool BF16>
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  if (BF16) {
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
  }
  __half2 v = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

template <bool BF16>
__device__ __forceinline__ float round16(float x) {
  return BF16 ? __bfloat162float(__float2bfloat16_rn(x)) : __half2float(__float2half_rn(x));
}

// Keep the f16/bf16 halves of `r` whose tokens are < nv.
__device__ __forceinline__ uint32_t mask_pair(uint32_t r, int tok_lo, int tok_hi, int nv) {
  const uint32_t m = (tok_lo < nv ? 0x0000ffffu : 0u) | (tok_hi < nv ? 0xffff0000u : 0u);
  return r & m;
}

// 5-D tiled TMA load; coordinates (dim, token, head, K|V, slab).
__device__ __forceinline__ void tma_load_5d(uint32_t dst, const CUtensorMap* map, int x, int tok, int head, int kv,
                                            int slab, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.5d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5, "
      "%6}], [%7];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(tok), "r"(head), "r"(kv), "r"(slab), "r"(smem_u32(bar))
      : "memory");
}

// Rank-5 TMA map over the page data: dims {head dim, token, head, K|V,
// layer x page}, boxes of {128 bytes of the head dim, 16 tokens, HG heads,
// KVB of K|V, 1 page}, 128-byte swizzle. `slot` caches it in the pool handle;
// `ready` records HG * 4 + KVB once encoded.
// The driver's tensor-map encoder, looked up once (nullptr if unavailable).
inline PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 encode = nullptr;
  if (encode == nullptr) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess && fn != nullptr)
      encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  }
  return encode;
}

inline int ensure_tmap(const sckv_pool* pool, int HG, unsigned char* slot, int* ready, int KVB = 2) {
  if (*ready == HG * 4 + KVB) return SCKV_OK;
  PFN_cuTensorMapEncodeTiled_v12000 encode = tensor_map_encoder();
  if (encode == nullptr)
    return sckv_record_error(__FILE__, __LINE__, "cudaGetDriverEntryPoint", "cuTensorMapEncodeTiled not found");
  const cuuint64_t eb = (cuuint64_t)sckv_elem_bytes(pool->kv_dtype);
  const cuuint64_t D = (cuuint64_t)pool->head_dim, H = (cuuint64_t)pool->num_kv_heads;
  const cuuint64_t dims[5] = {D, (cuuint64_t)SCKV_PAGE_TOKENS, H, 2,
                              (cuuint64_t)pool->num_layers * (cuuint64_t)pool->max_pages};
  const cuuint64_t strides[4] = {D * eb, SCKV_PAGE_TOKENS * D * eb, H * SCKV_PAGE_TOKENS * D * eb,
                                 2 * H * SCKV_PAGE_TOKENS * D * eb};
  const cuuint32_t box[5] = {(cuuint32_t)(128 / eb), (cuuint32_t)SCKV_PAGE_TOKENS, (cuuint32_t)HG, (cuuint32_t)KVB,
                             1};
  const cuuint32_t estr[5] = {1, 1, 1, 1, 1};
  const CUtensorMapDataType dt = (eb == 2) ? CU_TENSOR_MAP_DATA_TYPE_UINT16 : CU_TENSOR_MAP_DATA_TYPE_UINT8;
  CUresult r = encode(reinterpret_cast<CUtensorMap*>(slot), dt, 5, pool->data, dims, strides, box, estr,
                      CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                      CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    char what[64];
    snprintf(what, sizeof what, "CUresult %d", (int)r);
    return sckv_record_error(__FILE__, __LINE__, "cuTensorMapEncodeTiled", what);
  }
  *ready = HG * 4 + KVB;
  return SCKV_OK;
}

}  // namespace sckv_mma
