// attn_common.cuh -- helpers shared by the attention kernels.
#pragma once

#include "common.cuh"
#include "gfx906_fa_b200.h"

namespace g9 {

constexpr float kLog2e = 1.4426950408889634f;

// Query / output element access through the G9AttnBatch strides.
__device__ __forceinline__ int64_t q_offset(const G9AttnBatch& p, int b, int t, int hq) {
  const int qs = p.q_start ? p.q_start[b] : 0;
  return (int64_t)b * p.q_seq_stride + (int64_t)(qs + t) * p.q_tok_stride + (int64_t)hq * p.q_head_stride;
}
__device__ __forceinline__ int64_t o_offset(const G9AttnBatch& p, int b, int t, int hq) {
  const int qs = p.q_start ? p.q_start[b] : 0;
  return (int64_t)b * p.o_seq_stride + (int64_t)(qs + t) * p.o_tok_stride + (int64_t)hq * p.o_head_stride;
}
__device__ __forceinline__ int seq_nq(const G9AttnBatch& p, int b) { return p.n_q ? p.n_q[b] : p.seq_q; }

// Number of keys any query of sequence b can see (exclusive end).
__device__ __forceinline__ int seq_kv_end(const G9AttnBatch& p, int b, int nq) {
  int end = p.kv_len[b];
  if (p.q_abs) {
    const int64_t lim = (int64_t)p.q_abs[b] + nq;      // last token sees keys <= q_abs + nq - 1
    if (lim < end) end = lim < 0 ? 0 : (int)lim;
  }
  return end;
}

__device__ __forceinline__ void store_out2(void* out, int dt, int64_t off, float a, float b) {
  if (dt == DT_F32) {
    *reinterpret_cast<float2*>(reinterpret_cast<float*>(out) + off) = make_float2(a, b);
  } else if (dt == DT_F16) {
    *reinterpret_cast<__half2*>(reinterpret_cast<__half*>(out) + off) = __floats2half2_rn(a, b);
  } else {
    *reinterpret_cast<__nv_bfloat162*>(reinterpret_cast<__nv_bfloat16*>(out) + off) =
        __floats2bfloat162_rn(a, b);
  }
}

// ---------------------------------------------------------------------------
// warp-level tensor-core MMA (m16n8k16, 16-bit inputs, fp32 accumulators)
// ---------------------------------------------------------------------------
// Register-only: not volatile, so the compiler may schedule shared-memory
// loads for later fragments ahead of it.
__device__ __forceinline__ void mma_f16_16816(float c[4], const uint32_t a[4], const uint32_t b[2]) {
  asm(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}

__device__ __forceinline__ void mma_bf16_16816(float c[4], const uint32_t a[4], const uint32_t b[2]) {
  asm(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}

// Four 8x8 b16 matrices; thread l gets, of each matrix, the 4 bytes at
// columns 2*(l%4), 2*(l%4)+1 of row l/4.  Lanes 8m..8m+7 supply the row
// addresses of matrix m (16-byte aligned rows).
__device__ __forceinline__ void ldmatrix_x4(uint32_t r[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

__device__ __forceinline__ uint2 lds_u64(uint32_t addr) {
  uint2 v;
  asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(addr));
  return v;
}

__device__ __forceinline__ void ldmatrix_x4_trans(uint32_t r[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

__device__ __forceinline__ uint32_t pack_half2(float lo, float hi) {
  __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

__device__ __forceinline__ uint32_t pack_bf162(float lo, float hi) {
  __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

// Two int8 values (low 16 bits of `pair`) -> exact fp16x2.  fp16 with exponent
// 2^10 has unit spacing, so 0x6400 | u is exactly 1024 + u for u in 0..255;
// flipping the sign bit maps int8 b to u = b + 128, and subtracting 1152
// recovers b exactly.
__device__ __forceinline__ uint32_t i8x2_to_h2(uint32_t pair) {
  const uint32_t t = __byte_perm(pair ^ 0x8080u, 0x64646464u, 0x5140);
  __half2 h = *reinterpret_cast<const __half2*>(&t);
  const __half2 bias = __halves2half2(__ushort_as_half(0x6480), __ushort_as_half(0x6480));  // 1152
  h = __hsub2(h, bias);
  return *reinterpret_cast<uint32_t*>(&h);
}

__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ uint16_t lds_u16(uint32_t addr) {
  uint16_t v;
  asm volatile("ld.shared.u16 %0, [%1];" : "=h"(v) : "r"(addr));
  return v;
}

__device__ __forceinline__ float half_bits_to_float(uint16_t h) { return __half2float(__ushort_as_half(h)); }

}  // namespace g9
