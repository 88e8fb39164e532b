// common.cuh -- shared device helpers for the sm_100a paged-Q8 attention path.
//
// Q8_0 block format (identical to the reference's block_q8_0,
// kernel/ggml_shim.cuh:90-94): 34 bytes per 32 elements -- bytes 0..1 hold the
// fp16 scale d (little-endian), bytes 2..33 the int8 quants.  A row of D
// elements is D/32 consecutive blocks (136 bytes at D = 128).
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <cuda_fp8.h>
#include <stdint.h>

namespace g9 {

constexpr int QK = 32;          // elements per Q8_0 block
constexpr int QBLOCK = 34;      // bytes per Q8_0 block

enum DType : int { DT_F16 = 0, DT_BF16 = 1, DT_F32 = 2, DT_FP8 = 3 /* e4m3, outputs only */ };

__host__ __device__ inline int q8_row_bytes(int D) { return (D / QK) * QBLOCK; }

// Error word written by device code when a bounded wait gives up or an
// argument fails an in-kernel check.  Read/reset through the C ABI
// (gfx906_fa_get_device_error).  Bit 0: mbarrier wait timed out; bit 1:
// block-table entry out of range; bit 2: tensor-memory allocation failed.
// Each translation unit has its own copy (no relocatable device code); the
// C ABI ORs them together (see G9_ERROR_ACCESSORS).
static __device__ unsigned int g_device_error;

enum DeviceError : unsigned int {
  ERR_WAIT_TIMEOUT = 1u,
  ERR_BAD_PAGE = 2u,
  ERR_TMEM = 4u,
};

__device__ __forceinline__ void raise_error(unsigned int bits) { atomicOr(&g_device_error, bits); }

// ---------------------------------------------------------------------------
// element loads (fp16 / bf16 / fp32 -> fp32)
// ---------------------------------------------------------------------------
__device__ __forceinline__ float load_one(const void* p, int64_t i, int dt) {
  if (dt == DT_F16) return __half2float(reinterpret_cast<const __half*>(p)[i]);
  if (dt == DT_BF16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
  return reinterpret_cast<const float*>(p)[i];
}

// four consecutive elements starting at element i (i multiple of 4, base
// aligned to 4 elements).
__device__ __forceinline__ void load_four(const void* p, int64_t i, int dt, float v[4]) {
  if (dt == DT_F32) {
    float4 f = *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(p) + i);
    v[0] = f.x; v[1] = f.y; v[2] = f.z; v[3] = f.w;
    return;
  }
  uint2 u = *reinterpret_cast<const uint2*>(reinterpret_cast<const uint16_t*>(p) + i);
  if (dt == DT_F16) {
    float2 a = __half22float2(*reinterpret_cast<__half2*>(&u.x));
    float2 b = __half22float2(*reinterpret_cast<__half2*>(&u.y));
    v[0] = a.x; v[1] = a.y; v[2] = b.x; v[3] = b.y;
  } else {
    v[0] = __uint_as_float(u.x << 16);
    v[1] = __uint_as_float(u.x & 0xffff0000u);
    v[2] = __uint_as_float(u.y << 16);
    v[3] = __uint_as_float(u.y & 0xffff0000u);
  }
}

// ---------------------------------------------------------------------------
// mbarrier + bulk-async copy (TMA engine) wrappers
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;"
               ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait: polls until the phase completes or about two seconds of
// wall time (%globaltimer) have passed; on timeout it records
// ERR_WAIT_TIMEOUT and returns false, and callers skip the remaining work of
// the CTA.  Nothing in a correct run comes near the limit.
constexpr uint64_t kWaitLimitNs = 2000000000ull;

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ bool mbar_wait_limit(uint64_t* bar, uint32_t parity, uint64_t limit_ns) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_ns();
  for (uint32_t i = 1;; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 255) == 0 && global_ns() - t0 > limit_ns) break;
  }
  raise_error(ERR_WAIT_TIMEOUT);
  return false;
}

__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
  return mbar_wait_limit(bar, parity, kWaitLimitNs);
}

// 1-D bulk copy global -> this CTA's shared memory, completion signalled as
// transaction bytes on `bar`.  src, dst 16-byte aligned, bytes % 16 == 0.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
      ::"r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// Ampere-style asynchronous copy global -> shared of 16 or 8 bytes, and the
// arrive-on-completion that ties a thread's outstanding copies to an mbarrier.
__device__ __forceinline__ void cp_async(void* dst, const void* src, int bytes) {
  if (bytes == 16)
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
  else
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}

__device__ __forceinline__ void cp_async_arrive_noinc(uint64_t* bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ int lane_id() { return threadIdx.x & 31; }
__device__ __forceinline__ int warp_id() { return threadIdx.x >> 5; }

}  // namespace g9

// Host accessors for this translation unit's error word.
#define G9_ERROR_ACCESSORS(tag)                                                        \
  namespace g9 {                                                                       \
  cudaError_t err_get_##tag(unsigned int* out) {                                       \
    return cudaMemcpyFromSymbol(out, g_device_error, sizeof(unsigned int));            \
  }                                                                                    \
  cudaError_t err_clear_##tag() {                                                      \
    unsigned int z = 0;                                                                \
    return cudaMemcpyToSymbol(g_device_error, &z, sizeof(unsigned int));               \
  }                                                                                    \
  }
