// q8_store.cu -- Q8_0 KV-store kernel for sm_100a.
//
// One warp per (token, kv-head) row.  Each lane loads 4 consecutive elements
// with one 8-byte (16-bit types) or 16-byte (fp32) vector load, so a 32-
// element Q8_0 block is spread over 8 lanes and its absmax needs three
// butterfly shuffles.  The quantised row is assembled in shared memory and
// written with the widest store the destination alignment allows (8 bytes
// for the 136-byte rows of D = 128).
//
// Numerics follow the reference kernel exactly
// (extension/gfx906_fa_quant.cu:51-84): fp32 absmax, d = amax / 127.0f
// (IEEE division), id = d > 0 ? 1/d : 0 (IEEE reciprocal), q = rint(v * id)
// (round half to even) clamped to [-128, 127], scale stored as fp16(d) with
// round-to-nearest-even.  This translation unit is built without
// --use_fast_math, so `/` is the correctly rounded division.
//
// The same kernel serves three callers:
//   * dense quantisation (quantize_q8_0, gfx906_fa_quant.cu:100-129),
//   * the paged K store by slot_mapping (reshape_and_cache_q8,
//     gfx906_fa_quant.cu:150-200),
//   * the fused K+V store that replaces vLLM's Triton reshape_and_cache
//     (backend.py:416-425): V is either copied as 16-bit rows or quantised
//     to Q8_0 with the same rules as K.
#include "common.cuh"
#include "gfx906_fa_b200.h"

namespace g9 {

struct StoreArgs {
  const void* key;              // [T, Hkv, D], element strides below
  const void* value;            // may be null (v_mode == 0)
  const int64_t* slot_mapping;  // [T]; null -> slot = token index
  uint8_t* k_cache;
  uint8_t* v_cache;
  int64_t key_tok, key_head;    // elements
  int64_t val_tok, val_head;    // elements
  int64_t kc_blk, kc_tok, kc_head;  // bytes
  int64_t vc_blk, vc_tok, vc_head;  // bytes
  int key_dt, val_dt;
  int v_mode;                   // 0: no V, 1: copy 16-bit rows, 2: Q8_0 rows, 3: Q8_0 page-transposed
  int T, Hkv, D, bs;
  int k_store_w;                // widest aligned store for K rows (2, 4 or 8 bytes)
  int v_store_w;                // same for V rows
  int vec_ok_k, vec_ok_v;       // 1 when 4-element vector loads are aligned
  int hkv_log2, bs_log2;        // fast path: log2 of Hkv and block size (powers of two)
  int k_tok16;                  // fast16 path: a token's 8 Q8_0 K rows are 1088 contiguous, 16-byte aligned bytes
  // fused RoPE (rope_store_kernel only)
  void* query;                  // [T, Hq, D], rotated in place (may be null)
  int q_dt, Hq;
  int64_t q_tok, q_head;        // elements
  const int64_t* positions;     // [T]
  const void* cos_sin;          // [max_pos, rot]: cos of pair j at j, sin at rot/2 + j
  int cs_dt, rot, neox;
};

constexpr int kWarps = 8;
constexpr int kMaxD = 512;
constexpr int kStage = ((kMaxD / QK) * QBLOCK + 7) & ~7;   // 544 bytes per warp

// Quantise the 4 elements v of this lane (elements e0 .. e0+3 of a row; a
// 32-element block spans 8 lanes) into their Q8_0 block in `stage`.  Every
// lane of the warp must call it (the block absmax is a shuffle reduction);
// inactive lanes pass zeros.
__device__ __forceinline__ void quant4_to_stage(const float v[4], int e0, bool active, uint8_t* stage) {
  float amax = fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3])));
  amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
  amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
  amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 4));
  const float d = amax / 127.0f;
  const float id = d > 0.0f ? __frcp_rn(d) : 0.0f;
  if (active) {
    const int blk = e0 / QK;                 // block index within the row
    const int j = (e0 % QK) / 4;             // lane slot within the block (0..7)
    uint8_t* out = stage + blk * QBLOCK;
    uint32_t packed = 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      int qi = __float2int_rn(v[i] * id);
      qi = max(-128, min(127, qi));
      packed |= (uint32_t)(qi & 0xff) << (8 * i);
    }
    // byte offset 2 + 4j is 2-aligned: two 16-bit stores
    uint16_t* o16 = reinterpret_cast<uint16_t*>(out + 2 + 4 * j);
    o16[0] = (uint16_t)(packed & 0xffffu);
    o16[1] = (uint16_t)(packed >> 16);
    if (j == 0) {
      __half dh = __float2half_rn(d);
      *reinterpret_cast<uint16_t*>(out) = __half_as_ushort(dh);
    }
  }
}

// Quantise one row of D elements held as 4 elements per lane per 128-element
// chunk and leave the Q8_0 bytes in `stage`.
__device__ __forceinline__ void quant_row_to_stage(const void* src, int64_t base, int dt, int D,
                                                   bool vec_ok, uint8_t* stage) {
  const int lane = lane_id();
  for (int c0 = 0; c0 < D; c0 += 128) {
    const int e0 = c0 + 4 * lane;             // first element this lane owns
    const bool active = e0 < D;
    float v[4] = {0.f, 0.f, 0.f, 0.f};
    if (active) {
      if (vec_ok) {
        load_four(src, base + e0, dt, v);
      } else {
#pragma unroll
        for (int i = 0; i < 4; ++i) v[i] = load_one(src, base + e0 + i, dt);
      }
    }
    quant4_to_stage(v, e0, active, stage);
  }
  __syncwarp();
}

__device__ __forceinline__ void stage_to_global(const uint8_t* stage, uint8_t* dst, int bytes, int w) {
  const int lane = lane_id();
  if (w == 8) {
    for (int i = lane; i < bytes / 8; i += 32)
      reinterpret_cast<uint64_t*>(dst)[i] = reinterpret_cast<const uint64_t*>(stage)[i];
  } else if (w == 4) {
    for (int i = lane; i < bytes / 4; i += 32)
      reinterpret_cast<uint32_t*>(dst)[i] = reinterpret_cast<const uint32_t*>(stage)[i];
  } else {
    for (int i = lane; i < bytes / 2; i += 32)
      reinterpret_cast<uint16_t*>(dst)[i] = reinterpret_cast<const uint16_t*>(stage)[i];
  }
  __syncwarp();
}

// V row of (token t, head h) into slot (blk, off) per v_mode: Q8_0 token row
// (2), page-transposed Q8_0 record (3), or a 16-bit copy (1).  `stage` is
// the warp's shared-memory row buffer.
__device__ __forceinline__ void store_v_row(const StoreArgs& a, int t, int h, int64_t blk, int64_t off,
                                            uint8_t* stage) {
  const int rb = q8_row_bytes(a.D);
  if (a.v_mode == 2) {
    quant_row_to_stage(a.value, (int64_t)t * a.val_tok + (int64_t)h * a.val_head, a.val_dt, a.D,
                       a.vec_ok_v, stage);
    stage_to_global(stage, a.v_cache + blk * a.vc_blk + off * a.vc_tok + h * a.vc_head, rb,
                    a.v_store_w);
  } else if (a.v_mode == 3) {
    // page-transposed record of (page, head): fp16 scales [D/32][bs], then
    // int8 values [D][bs]
    quant_row_to_stage(a.value, (int64_t)t * a.val_tok + (int64_t)h * a.val_head, a.val_dt, a.D,
                       a.vec_ok_v, stage);
    uint8_t* rec = a.v_cache + blk * a.vc_blk + h * a.vc_head;
    const int nb = a.D / QK;
    const int lane = lane_id();
    for (int j = lane; j < nb; j += 32)
      *reinterpret_cast<uint16_t*>(rec + 2 * ((int64_t)j * a.bs + off)) =
          *reinterpret_cast<const uint16_t*>(stage + j * QBLOCK);
    uint8_t* qv = rec + 2 * nb * a.bs + off;
    for (int i = lane; i < a.D; i += 32) qv[(int64_t)i * a.bs] = stage[(i / QK) * QBLOCK + 2 + (i % QK)];
    __syncwarp();
  } else if (a.v_mode == 1) {
    const uint16_t* src = reinterpret_cast<const uint16_t*>(a.value) +
                          (int64_t)t * a.val_tok + (int64_t)h * a.val_head;
    uint8_t* dst = a.v_cache + blk * a.vc_blk + off * a.vc_tok + h * a.vc_head;
    const int lane = lane_id();
    if (a.v_store_w == 8 && a.vec_ok_v) {
      for (int i = lane; i < a.D / 4; i += 32)
        reinterpret_cast<uint2*>(dst)[i] = reinterpret_cast<const uint2*>(src)[i];
    } else {
      for (int i = lane; i < a.D; i += 32)
        reinterpret_cast<uint16_t*>(dst)[i] = src[i];
    }
  }
}

__global__ void __launch_bounds__(kWarps * 32) q8_store_kernel(StoreArgs a) {
  __shared__ __align__(16) uint8_t stage_all[kWarps][kStage];
  uint8_t* stage = stage_all[warp_id()];
  const int rb = q8_row_bytes(a.D);
  const int64_t rows = (int64_t)a.T * a.Hkv;
  for (int64_t row = (int64_t)blockIdx.x * kWarps + warp_id(); row < rows;
       row += (int64_t)gridDim.x * kWarps) {
    const int t = (int)(row / a.Hkv);
    const int h = (int)(row % a.Hkv);
    const int64_t slot = a.slot_mapping ? a.slot_mapping[t] : (int64_t)t;
    if (slot < 0) continue;                              // padded token
    const int64_t blk = slot / a.bs, off = slot % a.bs;
    // ---- K: quantise -------------------------------------------------------
    quant_row_to_stage(a.key, (int64_t)t * a.key_tok + (int64_t)h * a.key_head, a.key_dt, a.D,
                       a.vec_ok_k, stage);
    stage_to_global(stage, a.k_cache + blk * a.kc_blk + off * a.kc_tok + h * a.kc_head, rb,
                    a.k_store_w);
    // ---- V -----------------------------------------------------------------
    store_v_row(a, t, h, blk, off, stage);
  }
}

// Fast path for head_dim 128, 16-bit K / V, aligned rows, V copied or
// absent: each warp takes 4 rows per iteration and issues all their K and V
// loads first (the general kernel above walks one row at a time, so every
// row waited a full DRAM latency and little was in flight).  Lane l holds
// elements 4l..4l+3 of a row, i.e. slot l%8 of 32-element block l/8; the
// quantisation arithmetic is the general kernel's.  V rows go from
// registers straight to the cache; the Q8_0 K rows are assembled in shared
// memory so that they leave as aligned 8-byte stores.
constexpr int kFastRows = 4;
constexpr int kFastRowBytes = (128 / QK) * QBLOCK;       // 136

__global__ void __launch_bounds__(kWarps * 32) q8_store_fast_kernel(StoreArgs a) {
  __shared__ __align__(16) uint8_t stage_all[kWarps][kFastRows * kFastRowBytes];
  uint8_t* stage = stage_all[warp_id()];
  const int lane = lane_id();
  const int64_t rows = (int64_t)a.T * a.Hkv;
  const bool bf_k = a.key_dt == DT_BF16, bf_v = a.val_dt == DT_BF16;
  (void)bf_v;
  for (int64_t r0 = ((int64_t)blockIdx.x * kWarps + warp_id()) * kFastRows; r0 < rows;
       r0 += (int64_t)gridDim.x * kWarps * kFastRows) {
    uint2 kraw[kFastRows], vraw[kFastRows];
    int64_t kdst[kFastRows], vdst[kFastRows];   // byte offsets in the caches, -1: skip the row
#pragma unroll
    for (int i = 0; i < kFastRows; ++i) {
      const uint32_t row = (uint32_t)(r0 + i);
      const bool valid = r0 + i < rows;
      const uint32_t t = row >> a.hkv_log2, h = row & ((1u << a.hkv_log2) - 1);
      const int64_t s = valid ? (a.slot_mapping ? a.slot_mapping[t] : (int64_t)t) : -1;
      if (s >= 0) {
        const uint64_t s64 = (uint64_t)s;
        const uint32_t blk = (uint32_t)(s64 >> a.bs_log2);
        const uint32_t off = (uint32_t)s64 & ((1u << a.bs_log2) - 1);
        // cache strides < 2^31 (checked by the launcher), the in-page part
        // below one page stride: one 32x32->64 multiply per address
        kdst[i] = (int64_t)((uint64_t)blk * (uint32_t)a.kc_blk + (off * (uint32_t)a.kc_tok + h * (uint32_t)a.kc_head));
        vdst[i] = (int64_t)((uint64_t)blk * (uint32_t)a.vc_blk + (off * (uint32_t)a.vc_tok + h * (uint32_t)a.vc_head));
      } else {
        kdst[i] = vdst[i] = -1;
      }
      // contiguous [T, Hkv, 128] rows (checked by the launcher)
      kraw[i] = valid ? *reinterpret_cast<const uint2*>(reinterpret_cast<const uint16_t*>(a.key) + (size_t)row * 128 + 4 * lane)
                      : make_uint2(0u, 0u);
      vraw[i] = (valid && a.v_mode == G9_V_COPY16)
                    ? *reinterpret_cast<const uint2*>(reinterpret_cast<const uint16_t*>(a.value) + (size_t)row * 128 + 4 * lane)
                    : make_uint2(0u, 0u);
    }
#pragma unroll
    for (int i = 0; i < kFastRows; ++i) {
      float v[4];
      if (bf_k) {
        v[0] = __uint_as_float(kraw[i].x << 16); v[1] = __uint_as_float(kraw[i].x & 0xffff0000u);
        v[2] = __uint_as_float(kraw[i].y << 16); v[3] = __uint_as_float(kraw[i].y & 0xffff0000u);
      } else {
        const float2 x0 = __half22float2(*reinterpret_cast<const __half2*>(&kraw[i].x));
        const float2 x1 = __half22float2(*reinterpret_cast<const __half2*>(&kraw[i].y));
        v[0] = x0.x; v[1] = x0.y; v[2] = x1.x; v[3] = x1.y;
      }
      float amax = fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3])));
      amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
      amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
      amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 4));
      // amax / 127 correctly rounded without the IEEE division routine:
      // y = amax * fl(1/127), then one residual-correction step of the
      // reciprocal product (Markstein's method: r = amax - y*127 exactly by
      // FMA, y' = y + r*fl(1/127)).  Exact for every finite fp16 and bf16
      // value, which are all the values amax can take here (16-bit inputs);
      // tests/test_store_gpu.py::test_fast_store_every_16bit_absmax checks
      // all of them on the GPU against the oracle's IEEE division.
      constexpr float kInv127 = 1.0f / 127.0f;
      const float y127 = __fmul_rn(amax, kInv127);
      const float dq = fmaf(fmaf(-y127, 127.0f, amax), kInv127, y127);
      const float id = dq > 0.0f ? __frcp_rn(dq) : 0.0f;
      // rint(v*id) clamped to [-128, 127] without the (quarter-rate)
      // float->int conversion: the product is rounded to fp32 as in the
      // reference, then adding 1.5*2^23 rounds it to an integer with ties to
      // even (exactly rintf for |x| < 2^22) and leaves it in the low mantissa
      // bits; the clamp is applied to the sum, and the int8 is its low byte.
      // Identical to the general kernel for finite inputs.  When the block's
      // scale underflows so far that 1/d is infinite, a zero element gives
      // 0 * inf = NaN: it becomes 0, as the general kernel's float -> int
      // conversion (and the reference's) makes it; +-inf products clamp.
      constexpr float kMagic = 12582912.0f;
      uint32_t rb[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        float r = __fadd_rn(__fmul_rn(v[e], id), kMagic);
        r = r == r ? r : kMagic;
        r = fminf(fmaxf(r, kMagic - 128.0f), kMagic + 127.0f);
        rb[e] = __float_as_uint(r);
      }
      const uint32_t packed = __byte_perm(__byte_perm(rb[0], rb[1], 0x0040), __byte_perm(rb[2], rb[3], 0x0040), 0x5410);
      uint8_t* out = stage + i * kFastRowBytes + (lane >> 3) * QBLOCK;
      uint16_t* o16 = reinterpret_cast<uint16_t*>(out + 2 + 4 * (lane & 7));
      o16[0] = (uint16_t)(packed & 0xffffu);
      o16[1] = (uint16_t)(packed >> 16);
      if ((lane & 7) == 0) *reinterpret_cast<uint16_t*>(out) = __half_as_ushort(__float2half_rn(dq));
      if (a.v_mode == G9_V_COPY16 && vdst[i] >= 0)
        *reinterpret_cast<uint2*>(a.v_cache + vdst[i] + 8 * lane) = vraw[i];
    }
    __syncwarp();
    // each Q8_0 K row (17 x 8 bytes) leaves from lanes 0..16
#pragma unroll
    for (int i = 0; i < kFastRows; ++i)
      if (lane < kFastRowBytes / 8 && kdst[i] >= 0)
        reinterpret_cast<uint64_t*>(a.k_cache + kdst[i])[lane] =
            reinterpret_cast<const uint64_t*>(stage + i * kFastRowBytes)[lane];
    __syncwarp();
  }
}

// The same store with 16-byte accesses (16-byte aligned K / V rows and V
// cache): half a warp per row, lane l of the half holding elements 8l ..
// 8l+7, so a 32-element block is 4 lanes (two shuffles for its absmax) and
// a warp keeps 8 rows of loads in flight.  Quantisation arithmetic is the
// one above, element for element.
constexpr int kRows16 = 8;

__global__ void __launch_bounds__(kWarps * 32) q8_store_fast16_kernel(StoreArgs a) {
  __shared__ __align__(16) uint8_t stage_all[kWarps][kRows16 * kFastRowBytes];
  __shared__ int64_t kdst_all[kWarps][kRows16];
  uint8_t* stage = stage_all[warp_id()];
  int64_t* kdst_s = kdst_all[warp_id()];
  const int lane = lane_id();
  const int half = lane >> 4, hl = lane & 15;
  const int64_t rows = (int64_t)a.T * a.Hkv;
  const bool bf_k = a.key_dt == DT_BF16;
  for (int64_t r0 = ((int64_t)blockIdx.x * kWarps + warp_id()) * kRows16; r0 < rows;
       r0 += (int64_t)gridDim.x * kWarps * kRows16) {
    uint4 kraw[kRows16 / 2], vraw[kRows16 / 2];
    int64_t slot[kRows16 / 2];          // destinations are derived from the slot where they are used
#pragma unroll
    for (int k = 0; k < kRows16 / 2; ++k) {
      const int64_t row64 = r0 + 2 * k + half;
      const bool valid = row64 < rows;
      const uint32_t row = (uint32_t)row64;
      const uint32_t t = row >> a.hkv_log2;
      slot[k] = valid ? (a.slot_mapping ? a.slot_mapping[t] : (int64_t)t) : -1;
      kraw[k] = valid ? reinterpret_cast<const uint4*>(a.key)[(size_t)row * 16 + hl] : make_uint4(0u, 0u, 0u, 0u);
      vraw[k] = (valid && a.v_mode == G9_V_COPY16) ? reinterpret_cast<const uint4*>(a.value)[(size_t)row * 16 + hl]
                                                   : make_uint4(0u, 0u, 0u, 0u);
    }
#pragma unroll
    for (int k = 0; k < kRows16 / 2; ++k) {
      const uint32_t w[4] = {kraw[k].x, kraw[k].y, kraw[k].z, kraw[k].w};
      float v[8];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        if (bf_k) {
          v[2 * e] = __uint_as_float(w[e] << 16); v[2 * e + 1] = __uint_as_float(w[e] & 0xffff0000u);
        } else {
          const float2 x = __half22float2(*reinterpret_cast<const __half2*>(&w[e]));
          v[2 * e] = x.x; v[2 * e + 1] = x.y;
        }
      }
      float amax = fabsf(v[0]);                       // NaN only if every element is NaN, as above
#pragma unroll
      for (int e = 1; e < 8; ++e) amax = fmaxf(amax, fabsf(v[e]));
      amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
      amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
      constexpr float kInv127 = 1.0f / 127.0f;
      const float y127 = __fmul_rn(amax, kInv127);
      const float dq = fmaf(fmaf(-y127, 127.0f, amax), kInv127, y127);
      const float id = dq > 0.0f ? __frcp_rn(dq) : 0.0f;
      constexpr float kMagic = 12582912.0f;
      uint32_t rb[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        float r = __fadd_rn(__fmul_rn(v[e], id), kMagic);
        r = r == r ? r : kMagic;
        r = fminf(fmaxf(r, kMagic - 128.0f), kMagic + 127.0f);
        rb[e] = __float_as_uint(r);
      }
      const uint32_t p0 = __byte_perm(__byte_perm(rb[0], rb[1], 0x0040), __byte_perm(rb[2], rb[3], 0x0040), 0x5410);
      const uint32_t p1 = __byte_perm(__byte_perm(rb[4], rb[5], 0x0040), __byte_perm(rb[6], rb[7], 0x0040), 0x5410);
      const int r = 2 * k + half;
      uint8_t* out = stage + r * kFastRowBytes + (hl >> 2) * QBLOCK;
      uint16_t* o16 = reinterpret_cast<uint16_t*>(out + 2 + 8 * (hl & 3));
      o16[0] = (uint16_t)(p0 & 0xffffu);
      o16[1] = (uint16_t)(p0 >> 16);
      o16[2] = (uint16_t)(p1 & 0xffffu);
      o16[3] = (uint16_t)(p1 >> 16);
      if ((hl & 3) == 0) *reinterpret_cast<uint16_t*>(out) = __half_as_ushort(__float2half_rn(dq));
      if (slot[k] >= 0) {
        const uint32_t h = (uint32_t)(r0 + r) & ((1u << a.hkv_log2) - 1);
        const uint64_t s64 = (uint64_t)slot[k];
        const uint32_t blk = (uint32_t)(s64 >> a.bs_log2);
        const uint32_t off = (uint32_t)s64 & ((1u << a.bs_log2) - 1);
        if (hl == 0)
          kdst_s[r] = (int64_t)((uint64_t)blk * (uint32_t)a.kc_blk + (off * (uint32_t)a.kc_tok + h * (uint32_t)a.kc_head));
        if (a.v_mode == G9_V_COPY16)
          *reinterpret_cast<uint4*>(a.v_cache + (int64_t)((uint64_t)blk * (uint32_t)a.vc_blk +
                                                          (off * (uint32_t)a.vc_tok + h * (uint32_t)a.vc_head)) +
                                    16 * hl) = vraw[k];
      } else if (hl == 0) {
        kdst_s[r] = -1;
      }
    }
    __syncwarp();
    if (a.k_tok16) {
      // eight kv heads: the warp's 8 rows are one token's heads, adjacent in
      // the cache (1088 bytes, 16-byte aligned): 68 16-byte stores
      const int64_t kd = kdst_s[0];
      if (kd >= 0) {
#pragma unroll
        for (int it = lane; it < kRows16 * kFastRowBytes / 16; it += 32)
          reinterpret_cast<uint4*>(a.k_cache + kd)[it] = reinterpret_cast<const uint4*>(stage)[it];
      }
      __syncwarp();
      continue;
    }
    // the 8 Q8_0 K rows (17 x 8 bytes each) leave as 136 aligned 8-byte stores
#pragma unroll
    for (int it = lane; it < kRows16 * (kFastRowBytes / 8); it += 32) {
      const int r = it / (kFastRowBytes / 8), wd = it - r * (kFastRowBytes / 8);
      const int64_t kd = kdst_s[r];
      if (kd >= 0)
        reinterpret_cast<uint64_t*>(a.k_cache + kd)[wd] = reinterpret_cast<const uint64_t*>(stage + r * kFastRowBytes)[wd];
    }
    __syncwarp();
  }
}

// ---------------------------------------------------------------------------
// Fused RoPE + KV store (head_dim 128).  The rows of K (T x Hkv) and of Q
// (T x Hq) are one grid-stride list: a K row is rotated, rounded once to
// its element type and written back in place (the rotated key the unfused
// rotary op would leave), then quantised to Q8_0 into the cache by slot with
// its V row stored per v_mode; a Q row is rotated and written back.  Lane l
// holds elements 4l .. 4l+3.  Rotation, in fp32 with separately rounded
// products (no FMA contraction), for pair (x, y) with angle cos c / sin s:
//   x' = x*c - y*s,  y' = y*c + x*s
// NeoX style pairs element i with i + rot/2 (partner lane l ^ rot/8);
// GPT-J style pairs 2j with 2j+1 (inside a lane).  Elements >= rot are not
// rotated.  cos/sin of pair j at position p: cos_sin[p*rot + j] and
// cos_sin[p*rot + rot/2 + j] (vLLM's cos_sin_cache).
// ---------------------------------------------------------------------------
__device__ __forceinline__ float round_to(float x, int dt) {
  if (dt == DT_F16) return __half2float(__float2half_rn(x));
  if (dt == DT_BF16) return __bfloat162float(__float2bfloat16_rn(x));
  return x;
}

__device__ __forceinline__ void store_four(void* p, int64_t i, int dt, const float v[4]) {
  if (dt == DT_F32) {
    *reinterpret_cast<float4*>(reinterpret_cast<float*>(p) + i) = make_float4(v[0], v[1], v[2], v[3]);
  } else if (dt == DT_F16) {
    __half2 a = __floats2half2_rn(v[0], v[1]), b = __floats2half2_rn(v[2], v[3]);
    *reinterpret_cast<uint2*>(reinterpret_cast<uint16_t*>(p) + i) =
        make_uint2(*reinterpret_cast<uint32_t*>(&a), *reinterpret_cast<uint32_t*>(&b));
  } else {
    __nv_bfloat162 a = __floats2bfloat162_rn(v[0], v[1]), b = __floats2bfloat162_rn(v[2], v[3]);
    *reinterpret_cast<uint2*>(reinterpret_cast<uint16_t*>(p) + i) =
        make_uint2(*reinterpret_cast<uint32_t*>(&a), *reinterpret_cast<uint32_t*>(&b));
  }
}

__device__ __forceinline__ void rope4(const StoreArgs& a, int64_t pos, int lane, float v[4]) {
  const int rot = a.rot, half = rot >> 1;
  const int64_t cb = pos * rot;
  const int e0 = 4 * lane;
  if (a.neox) {
    float p[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) p[k] = __shfl_xor_sync(0xffffffffu, v[k], half >> 2);
    if (e0 < rot) {
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int i = e0 + k;
        const int j = i < half ? i : i - half;
        const float c = load_one(a.cos_sin, cb + j, a.cs_dt), s = load_one(a.cos_sin, cb + half + j, a.cs_dt);
        v[k] = i < half ? __fsub_rn(__fmul_rn(v[k], c), __fmul_rn(p[k], s))
                        : __fadd_rn(__fmul_rn(v[k], c), __fmul_rn(p[k], s));
      }
    }
  } else if (e0 < rot) {
#pragma unroll
    for (int k = 0; k < 4; k += 2) {
      const int j = (e0 + k) >> 1;
      const float c = load_one(a.cos_sin, cb + j, a.cs_dt), s = load_one(a.cos_sin, cb + half + j, a.cs_dt);
      const float x = v[k], y = v[k + 1];
      v[k] = __fsub_rn(__fmul_rn(x, c), __fmul_rn(y, s));
      v[k + 1] = __fadd_rn(__fmul_rn(y, c), __fmul_rn(x, s));
    }
  }
}

__global__ void __launch_bounds__(kWarps * 32) rope_store_kernel(StoreArgs a) {
  __shared__ __align__(16) uint8_t stage_all[kWarps][kFastRowBytes];
  uint8_t* stage = stage_all[warp_id()];
  const int lane = lane_id();
  const int64_t rows_k = (int64_t)a.T * a.Hkv;
  const int64_t rows = rows_k + (a.query ? (int64_t)a.T * a.Hq : 0);
  for (int64_t row = (int64_t)blockIdx.x * kWarps + warp_id(); row < rows; row += (int64_t)gridDim.x * kWarps) {
    const bool isk = row < rows_k;
    const int64_t r = isk ? row : row - rows_k;
    const int H = isk ? a.Hkv : a.Hq;
    const int t = (int)(r / H), h = (int)(r % H);
    void* src = isk ? const_cast<void*>(a.key) : a.query;
    const int dt = isk ? a.key_dt : a.q_dt;
    const int64_t base = isk ? (int64_t)t * a.key_tok + (int64_t)h * a.key_head
                             : (int64_t)t * a.q_tok + (int64_t)h * a.q_head;
    float v[4];
    load_four(src, base + 4 * lane, dt, v);
    rope4(a, a.positions[t], lane, v);
#pragma unroll
    for (int k = 0; k < 4; ++k) v[k] = round_to(v[k], dt);
    store_four(src, base + 4 * lane, dt, v);
    if (!isk) continue;
    const int64_t slot = a.slot_mapping[t];
    // the whole warp takes the branch together (slot is per row)
    if (slot < 0) continue;
    const int64_t blk = slot / a.bs, off = slot % a.bs;
    quant4_to_stage(v, 4 * lane, true, stage);
    __syncwarp();
    stage_to_global(stage, a.k_cache + blk * a.kc_blk + off * a.kc_tok + h * a.kc_head, kFastRowBytes,
                    a.k_store_w);
    store_v_row(a, t, h, blk, off, stage);
  }
}

static int store_width(const void* base, int64_t a, int64_t b, int64_t c, int row_bytes) {
  uintptr_t m = (uintptr_t)base | (uintptr_t)a | (uintptr_t)b | (uintptr_t)c | (uintptr_t)row_bytes;
  if ((m & 7) == 0) return 8;
  if ((m & 3) == 0) return 4;
  return 2;
}

static bool vec_aligned(const void* base, int dt, int64_t s0, int64_t s1) {
  const int esz = dt == DT_F32 ? 4 : 2;
  const uintptr_t align = dt == DT_F32 ? 16 : 8;
  return ((uintptr_t)base % align) == 0 && (s0 % 4) == 0 && (s1 % 4) == 0 && esz > 0;
}

static int grid_for_rows(int64_t rows) {
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  int64_t want = (rows + kWarps - 1) / kWarps;
  int64_t cap = (int64_t)sms * 16;               // grid-stride beyond 16 CTAs per SM
  return (int)(want < cap ? (want > 0 ? want : 1) : cap);
}

cudaError_t launch_store(const StoreArgs& a, cudaStream_t stream) {
  const int64_t rows = (int64_t)a.T * a.Hkv;
  if (rows == 0) return cudaSuccess;
  auto pow2 = [](int64_t x) { return x > 0 && (x & (x - 1)) == 0; };
  auto small = [](int64_t x) { return x >= 0 && x < 0x7fffffff; };
  const bool fast = a.D == 128 && rows < 0x7fffffff && a.key_dt != DT_F32 && a.vec_ok_k && a.k_store_w == 8 &&
                    pow2(a.Hkv) && pow2(a.bs) && a.key_tok == (int64_t)a.Hkv * 128 && a.key_head == 128 &&
                    small(a.kc_blk) && small(a.kc_tok) && small(a.kc_head) &&
                    (a.v_mode == G9_V_NONE ||
                     (a.v_mode == G9_V_COPY16 && a.val_dt != DT_F32 && a.vec_ok_v && a.v_store_w == 8 &&
                      a.val_tok == (int64_t)a.Hkv * 128 && a.val_head == 128 && small(a.vc_blk) &&
                      small(a.vc_tok) && small(a.vc_head)));
  if (fast) {
    StoreArgs f = a;
    f.hkv_log2 = __builtin_ctzll((unsigned long long)a.Hkv);
    f.bs_log2 = __builtin_ctzll((unsigned long long)a.bs);
    // 16-byte rows: K (and a copied V) 16-byte aligned, V cache rows too
    const bool w16 = ((uintptr_t)a.key % 16) == 0 &&
                     (a.v_mode == G9_V_NONE ||
                      (((uintptr_t)a.value % 16) == 0 &&
                       (((uintptr_t)a.v_cache | (uintptr_t)a.vc_blk | (uintptr_t)a.vc_tok | (uintptr_t)a.vc_head) % 16) == 0));
    f.k_tok16 = a.Hkv == kRows16 && a.kc_head == kFastRowBytes &&
                (((uintptr_t)a.k_cache | (uintptr_t)a.kc_blk | (uintptr_t)a.kc_tok) % 16) == 0;
    if (w16)
      q8_store_fast16_kernel<<<grid_for_rows((rows + kRows16 - 1) / kRows16), kWarps * 32, 0, stream>>>(f);
    else
      q8_store_fast_kernel<<<grid_for_rows((rows + kFastRows - 1) / kFastRows), kWarps * 32, 0, stream>>>(f);
  } else {
    q8_store_kernel<<<grid_for_rows(rows), kWarps * 32, 0, stream>>>(a);
  }
  return cudaGetLastError();
}

}  // namespace g9

G9_ERROR_ACCESSORS(store)

using namespace g9;

extern "C" cudaError_t launch_quantize_q8_0_dense(const void* x, uint8_t* y, int N, int D,
                                                  cudaStream_t stream) {
  return gfx906_fa_quantize_q8_0(x, G9_DT_F16, y, (int64_t)N, D, stream);
}

extern "C" cudaError_t gfx906_fa_quantize_q8_0(const void* x, int x_dtype, uint8_t* y, int64_t N,
                                               int D, cudaStream_t stream) {
  if (D % QK != 0 || D <= 0 || D > kMaxD || N < 0 || x_dtype < 0 || x_dtype > 2) return cudaErrorInvalidValue;
  if (N == 0) return cudaSuccess;
  if (N > INT32_MAX) return cudaErrorInvalidValue;
  StoreArgs a{};
  const int rb = q8_row_bytes(D);
  a.key = x; a.key_dt = x_dtype; a.key_tok = D; a.key_head = 0;
  a.k_cache = y; a.kc_blk = rb; a.kc_tok = 0; a.kc_head = 0;
  a.T = (int)N; a.Hkv = 1; a.D = D; a.bs = 1;
  a.k_store_w = store_width(y, rb, 0, 0, rb);
  a.vec_ok_k = vec_aligned(x, x_dtype, D, 0);
  return launch_store(a, stream);
}

extern "C" cudaError_t launch_reshape_and_cache_q8(
    const void* key, const int64_t* slot_mapping, uint8_t* k_cache_q8, int num_tokens,
    int num_kv_heads, int head_size, int block_size, int64_t key_token_stride,
    int64_t key_head_stride, int64_t cache_block_stride, int64_t cache_token_stride,
    int64_t cache_head_stride, cudaStream_t stream) {
  return gfx906_fa_store_kv(key, G9_DT_F16, key_token_stride, key_head_stride, nullptr, G9_DT_F16, 0, 0,
                            slot_mapping, k_cache_q8, cache_block_stride, cache_token_stride,
                            cache_head_stride, nullptr, 0, 0, 0, G9_V_NONE, num_tokens, num_kv_heads,
                            head_size, block_size, stream);
}

extern "C" cudaError_t gfx906_fa_store_kv(
    const void* key, int key_dtype, int64_t key_token_stride, int64_t key_head_stride,
    const void* value, int value_dtype, int64_t value_token_stride, int64_t value_head_stride,
    const int64_t* slot_mapping, uint8_t* k_cache, int64_t k_block_stride, int64_t k_token_stride,
    int64_t k_head_stride, uint8_t* v_cache, int64_t v_block_stride, int64_t v_token_stride,
    int64_t v_head_stride, int v_mode, int num_tokens, int num_kv_heads, int head_size,
    int block_size, cudaStream_t stream) {
  if (head_size % QK != 0 || head_size <= 0 || head_size > kMaxD) return cudaErrorInvalidValue;
  if (num_tokens < 0 || num_kv_heads <= 0 || block_size <= 0) return cudaErrorInvalidValue;
  if (key_dtype < 0 || key_dtype > 2) return cudaErrorInvalidValue;
  if (v_mode < 0 || v_mode > 3) return cudaErrorInvalidValue;
  if (v_mode == G9_V_Q8T && (((uintptr_t)v_cache | (uintptr_t)v_block_stride | (uintptr_t)v_head_stride) & 1))
    return cudaErrorInvalidValue;                   // fp16 scales are written with 2-byte stores
  if (v_mode == G9_V_COPY16 && value_dtype == G9_DT_F32) return cudaErrorInvalidValue;
  if (v_mode != G9_V_NONE && (value == nullptr || v_cache == nullptr)) return cudaErrorInvalidValue;
  if (num_tokens == 0) return cudaSuccess;
  StoreArgs a{};
  const int rb = q8_row_bytes(head_size);
  a.key = key; a.key_dt = key_dtype; a.key_tok = key_token_stride; a.key_head = key_head_stride;
  a.value = value; a.val_dt = value_dtype; a.val_tok = value_token_stride; a.val_head = value_head_stride;
  a.slot_mapping = slot_mapping;
  a.k_cache = k_cache; a.kc_blk = k_block_stride; a.kc_tok = k_token_stride; a.kc_head = k_head_stride;
  a.v_cache = v_cache; a.vc_blk = v_block_stride; a.vc_tok = v_token_stride; a.vc_head = v_head_stride;
  a.v_mode = v_mode;
  a.T = num_tokens; a.Hkv = num_kv_heads; a.D = head_size; a.bs = block_size;
  a.k_store_w = store_width(k_cache, k_block_stride, k_token_stride, k_head_stride, rb);
  a.vec_ok_k = vec_aligned(key, key_dtype, key_token_stride, key_head_stride);
  if (v_mode == G9_V_Q8 || v_mode == G9_V_Q8T) {
    a.v_store_w = store_width(v_cache, v_block_stride, v_token_stride, v_head_stride, rb);
    a.vec_ok_v = vec_aligned(value, value_dtype, value_token_stride, value_head_stride);
  } else if (v_mode == G9_V_COPY16) {
    a.v_store_w = store_width(v_cache, v_block_stride, v_token_stride, v_head_stride, 2 * head_size);
    a.vec_ok_v = vec_aligned(value, value_dtype, value_token_stride, value_head_stride);
  }
  return launch_store(a, stream);
}

extern "C" cudaError_t gfx906_fa_rope_store_kv(
    void* query, int query_dtype, int64_t query_token_stride, int64_t query_head_stride, int num_heads_q,
    void* key, int key_dtype, int64_t key_token_stride, int64_t key_head_stride, const void* value,
    int value_dtype, int64_t value_token_stride, int64_t value_head_stride, const int64_t* positions,
    const void* cos_sin_cache, int cos_sin_dtype, int rot_dim, int is_neox, const int64_t* slot_mapping,
    uint8_t* k_cache, int64_t k_block_stride, int64_t k_token_stride, int64_t k_head_stride, uint8_t* v_cache,
    int64_t v_block_stride, int64_t v_token_stride, int64_t v_head_stride, int v_mode, int num_tokens,
    int num_kv_heads, int head_size, int block_size, cudaStream_t stream) {
  if (head_size != 128 || num_tokens < 0 || num_kv_heads <= 0 || block_size <= 0) return cudaErrorInvalidValue;
  if (!(rot_dim == 32 || rot_dim == 64 || rot_dim == 128)) return cudaErrorInvalidValue;
  if (key_dtype < 0 || key_dtype > 2 || cos_sin_dtype < 0 || cos_sin_dtype > 2 || v_mode < 0 || v_mode > 3)
    return cudaErrorInvalidValue;
  if (query && (num_heads_q <= 0 || query_dtype < 0 || query_dtype > 2)) return cudaErrorInvalidValue;
  if (!key || !positions || !cos_sin_cache || !slot_mapping || !k_cache) return cudaErrorInvalidValue;
  if (v_mode != G9_V_NONE && (value == nullptr || v_cache == nullptr)) return cudaErrorInvalidValue;
  if (v_mode == G9_V_COPY16 && value_dtype == G9_DT_F32) return cudaErrorInvalidValue;
  if (v_mode == G9_V_Q8T && (((uintptr_t)v_cache | (uintptr_t)v_block_stride | (uintptr_t)v_head_stride) & 1))
    return cudaErrorInvalidValue;
  // rows are read and written as 4-element vectors
  if (!vec_aligned(key, key_dtype, key_token_stride, key_head_stride) ||
      (query && !vec_aligned(query, query_dtype, query_token_stride, query_head_stride)))
    return cudaErrorInvalidValue;
  if (num_tokens == 0) return cudaSuccess;
  StoreArgs a{};
  const int rb = q8_row_bytes(head_size);
  a.key = key; a.key_dt = key_dtype; a.key_tok = key_token_stride; a.key_head = key_head_stride;
  a.value = value; a.val_dt = value_dtype; a.val_tok = value_token_stride; a.val_head = value_head_stride;
  a.slot_mapping = slot_mapping;
  a.k_cache = k_cache; a.kc_blk = k_block_stride; a.kc_tok = k_token_stride; a.kc_head = k_head_stride;
  a.v_cache = v_cache; a.vc_blk = v_block_stride; a.vc_tok = v_token_stride; a.vc_head = v_head_stride;
  a.v_mode = v_mode;
  a.T = num_tokens; a.Hkv = num_kv_heads; a.D = head_size; a.bs = block_size;
  a.k_store_w = store_width(k_cache, k_block_stride, k_token_stride, k_head_stride, rb);
  if (v_mode == G9_V_Q8 || v_mode == G9_V_Q8T) {
    a.v_store_w = store_width(v_cache, v_block_stride, v_token_stride, v_head_stride, rb);
    a.vec_ok_v = vec_aligned(value, value_dtype, value_token_stride, value_head_stride);
  } else if (v_mode == G9_V_COPY16) {
    a.v_store_w = store_width(v_cache, v_block_stride, v_token_stride, v_head_stride, 2 * head_size);
    a.vec_ok_v = vec_aligned(value, value_dtype, value_token_stride, value_head_stride);
  }
  a.query = query; a.q_dt = query_dtype; a.q_tok = query_token_stride; a.q_head = query_head_stride;
  a.Hq = num_heads_q;
  a.positions = positions; a.cos_sin = cos_sin_cache; a.cs_dt = cos_sin_dtype; a.rot = rot_dim;
  a.neox = is_neox ? 1 : 0;
  const int64_t rows = (int64_t)num_tokens * (num_kv_heads + (query ? num_heads_q : 0));
  rope_store_kernel<<<grid_for_rows(rows), kWarps * 32, 0, stream>>>(a);
  return cudaGetLastError();
}
