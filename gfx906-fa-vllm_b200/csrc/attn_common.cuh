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
__device__ __forceinline__ int seq_nq(const G9AttnBatch& p, int b) {
  if (p.n_q) return p.n_q[b];
  if (p.flags & G9_F_CU_SEQLENS) return p.q_start[b + 1] - p.q_start[b];
  return p.seq_q;
}
// a causal rule is in force (per-sequence q_abs given, or the chunk ends at the last key)
__device__ __forceinline__ bool has_causal(const G9AttnBatch& p) {
  return p.q_abs != nullptr || (p.flags & G9_F_CAUSAL_END);
}

// Keys of sequence b: kv_len[b] clamped to what the block table can address
// and to the host bound max_kv the launch was planned with, so a kv_len
// beyond either never reads past the sequence's block-table row or a
// workspace sized from max_kv.
__device__ __forceinline__ int seq_len_kv(const G9AttnBatch& p, int b) {
  int64_t L = p.kv_len[b];
  const int64_t cap = (int64_t)p.max_blocks * p.block_size;
  if (L > cap) L = cap;
  if (L > p.max_kv) L = p.max_kv;
  return L < 0 ? 0 : (int)L;
}

// Position of query token 0 of sequence b (token t sits at qpos0 + t): q_abs,
// or the chunk ending at the last key.  L = seq_len_kv(p, b).
__device__ __forceinline__ int64_t seq_qpos0(const G9AttnBatch& p, int b, int nq, int L) {
  return p.q_abs ? (int64_t)p.q_abs[b] : (int64_t)L - nq;
}
// causal offset of sequence b (0 when has_causal is false)
__device__ __forceinline__ int seq_qabs(const G9AttnBatch& p, int b, int nq, int L) {
  return p.q_abs ? p.q_abs[b] : ((p.flags & G9_F_CAUSAL_END) ? L - nq : 0);
}

// Number of keys any query of sequence b can see (exclusive end).
__device__ __forceinline__ int seq_kv_end(const G9AttnBatch& p, int b, int nq) {
  int end = seq_len_kv(p, b);
  if (has_causal(p)) {
    const int64_t lim = (int64_t)seq_qabs(p, b, nq, end) + nq;   // last token sees keys <= q_abs + nq - 1
    if (lim < end) end = lim < 0 ? 0 : (int)lim;
  }
  return end;
}

// First key any query of sequence b can see: 0, or with a sliding window
// the first key inside token 0's window (key k is visible to position qp iff
// qp - k < window).
__device__ __forceinline__ int seq_kv_begin(const G9AttnBatch& p, int b, int nq) {
  if (p.window <= 0) return 0;
  const int64_t lo = seq_qpos0(p, b, nq, seq_len_kv(p, b)) - p.window + 1;
  return lo < 0 ? 0 : (lo > 0x7fffffff ? 0x7fffffff : (int)lo);
}

// Lower visibility limit of query token t (keys k >= the value are inside its
// window); INT_MIN without a window.
__device__ __forceinline__ int window_lo(const G9AttnBatch& p, int64_t qpos0, int t) {
  if (p.window <= 0) return -0x7fffffff - 1;
  const int64_t lo = qpos0 + t - p.window + 1;
  return lo < -0x7fffffff ? -0x7fffffff : (lo > 0x7fffffff ? 0x7fffffff : (int)lo);
}

// A block-table entry that must not be dereferenced.
__device__ __forceinline__ bool page_bad(const G9AttnBatch& p, int phys) {
  return phys < 0 || (p.num_blocks > 0 && phys >= p.num_blocks);
}

// Soft-capped score in log2 units: cap * tanh(raw * scale / cap) * log2(e),
// with in = scale / cap and out = cap * log2(e) precomputed on the host.
__device__ __forceinline__ float softcap_log2(float raw, float in, float out) { return out * tanhf(raw * in); }

// Sink of query head hq in log2 units (0 weight when there is none).
__device__ __forceinline__ float sink_log2(const G9AttnBatch& p, int hq) {
  return p.sinks ? p.sinks[hq] * 1.4426950408889634f : -INFINITY;
}

// Factor folded into a final output row's normalisation: 1 / *out_scale for
// fp8 outputs (vLLM's static per-tensor output scale), else 1.
__device__ __forceinline__ float out_quant_factor(const G9AttnBatch& p) {
  return p.out_dtype == DT_FP8 ? 1.f / *p.out_scale : 1.f;
}

__device__ __forceinline__ uint8_t to_fp8(float x) {
  return (uint8_t)__nv_cvt_float_to_fp8(x, __NV_SATFINITE, __NV_E4M3);
}

__device__ __forceinline__ void store_out2(void* out, int dt, int64_t off, float a, float b) {
  if (dt == DT_FP8) {
    *reinterpret_cast<__nv_fp8x2_storage_t*>(reinterpret_cast<uint8_t*>(out) + off) =
        __nv_cvt_float2_to_fp8x2(make_float2(a, b), __NV_SATFINITE, __NV_E4M3);
  } else if (dt == DT_F32) {
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
