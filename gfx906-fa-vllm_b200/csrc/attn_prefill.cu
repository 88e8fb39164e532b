// attn_prefill.cu -- prefill / chunked-prefill attention on 5th-generation
// tensor cores (tcgen05 + tensor memory), fed by TMA.
//
// Replaces the reference's flat tile kernel for long query chunks
// (kernel/fattn-q8.cuh:835-1087 behind gfx906_fa_launch,
// extension/gfx906_fa_launcher.cu:53-209, and the gather + forward pair of
// extension/gfx906_fa_paged.py:333-445).
//
// Two kernels per call:
//
//  1. pack (CUDA cores, HBM-bound): the Q8_0 pages a prefill sequence can
//     see are dequantised ONCE per call into fp16 staging tiles -- K as
//     [key][d] rows, V transposed as [d][key] 128x128 tiles -- and Q is
//     converted to fp16 with the GQA group packed into rows (row = t*G + g).
//     Dequantisation is one rounding: q8 * d computed in fp32, rounded to
//     fp16.  Doing it once per call instead of once per (query tile, kv
//     tile) pair keeps the conversion work out of the tensor-core loop,
//     where it would compete with the softmax for issue slots.
//
//  2. attention (tcgen05): one CTA per two 128-row query tiles (256 packed
//     rows) of one kv head, so every K/V tile loaded by TMA (128-byte
//     swizzled) feeds two tiles of MMAs.  warp 0 drives TMA, warp 1 allocates
//     tensor memory and issues tcgen05.mma from one thread, and two softmax
//     warpgroups (one per query tile) run one thread per query row (row i =
//     TMEM lane i).  Tensor memory: S0 S1 (128 fp32 columns each; P_i is
//     written as packed fp16 over S_i), O0 O1 (128 columns each).  The MMA
//     order PV0(j) S0(j+1) PV1(j) S1(j+1) keeps the tensor core on one tile
//     while the other tile's softmax runs.  Exponentials run on MUFU
//     (ex2.approx), packed arithmetic (f32x2) keeps the softmax's issue
//     slots few.  The running max is
//     rescaled lazily (only when it grows by more than 2^8), so O is rarely
//     touched by the softmax warps.
//
// Masking is the reference's: keys k >= kv_len ignored; causal rule
// k <= q_abs[b] + t (fattn-q8.cuh:646-654); optional fp16 additive mask.
// Rows without a visible key produce zeros.  All mbarrier waits are bounded.
#include <algorithm>
#include <cstring>

#include <cuda.h>

#include "attn_common.cuh"

namespace g9 {

namespace pf {
constexpr int D = 128;
constexpr int BM = 128;          // query rows per tile (two tiles per CTA)
constexpr int BN = 128;          // keys per tile
constexpr int KST = 3;           // K smem stages
constexpr int VST = 2;           // V smem stages
constexpr int TILE_BYTES = BM * D * 2;   // 32 KB (Q and K tiles)
static_assert(D == BN, "V^T tiles share the K tiles' row coordinates");
constexpr int MAXS = 128;        // prefill sequences per launch
// warp 0: TMA, warp 1: MMA, warps 4-7 / 8-11: softmax of query tile 0 / 1.
// setmaxnreg split: launch 384 threads x 168 = 64512 = 128*REG_CTRL + 256*REG_SOFTMAX
constexpr int NTHREADS = 384;
constexpr int REG_CTRL = 72;
constexpr int REG_SOFTMAX = 216;
static_assert(128 * REG_CTRL + 256 * REG_SOFTMAX <= NTHREADS * 168, "register split exceeds the launch budget");
constexpr float kRescaleThreshold = 8.0f;  // log2 units
}  // namespace pf

struct PrefillParams {
  CUtensorMap tm_q;
  CUtensorMap tm_k;
  CUtensorMap tm_v;
  G9AttnBatch p;
  int G, Hkv;
  int nseq;
  int min_rows;                  // sequences with n_q * G <= min_rows are left to the decode kernel
  int RT, KT;                    // row / key tiles per head (all sequences)
  int seq_b[pf::MAXS];
  int rtile_off[pf::MAXS + 1];
  int ktile_off[pf::MAXS + 1];
  float scale_log2;
  float cap_in, cap_out;         // soft-cap: scale / softcap and softcap * log2(e) (softcap > 0)
  int out_vec;                   // output base and strides are 16-byte multiples: staged row stores
  int v_direct;                  // page-transposed Q8_0 V, 16-token multiple pages, 16-byte aligned records
  __half* qp;                    // [Hkv][RT*128][128]
  __half* kp;                    // [Hkv][KT*128][128]
  __half* vt;                    // [Hkv][KT][128 d][128 keys]: V^T tiles
};

__device__ __forceinline__ int find_seq(const int* off, int n, int x) {
  int lo = 0, hi = n;            // largest i with off[i] <= x
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (off[mid] <= x) lo = mid; else hi = mid;
  }
  return lo;
}

// ===========================================================================
// pack kernels
// ===========================================================================

// K / V tile (head h, key tile kt): 128 keys of one sequence.
__global__ void __launch_bounds__(256) pack_kv_kernel(const __grid_constant__ PrefillParams pp) {
  using namespace pf;
  __shared__ __align__(16) __half vs[BN][D + 8];      // V tile, padded rows
  const G9AttnBatch& p = pp.p;
  const int kt = blockIdx.x;
  const int h = blockIdx.y;
  const int i = find_seq(pp.ktile_off, pp.nseq, kt);
  const int j = kt - pp.ktile_off[i];
  const int b = pp.seq_b[i];
  const int nq = seq_nq(p, b);
  if (nq * pp.G <= pp.min_rows) return;                // handled by the decode kernel
  const int L = min(seq_len_kv(p, b), (pp.ktile_off[i + 1] - pp.ktile_off[i]) * BN);
  if ((j + 1) * BN <= seq_kv_begin(p, b, nq)) return;  // before every row's window: never read
  __half* kdst = pp.kp + ((int64_t)h * pp.KT + kt) * BN * D;
  __half* vdst = pp.vt + ((int64_t)h * pp.KT + kt) * (int64_t)D * BN;
  // Page-transposed Q8_0 V is already [dim][token] inside a page: with pages
  // of a multiple of 16 tokens and 16-byte aligned records, row d of the V^T
  // tile is built from 16-byte loads of 16 tokens (one page each) without a
  // shared-memory transpose.
  const bool v_direct = pp.v_direct != 0;
  for (int it = threadIdx.x; it < BN * 8; it += blockDim.x) {
    const int key_l = it >> 3;
    const int c = it & 7;                 // 16-element chunk
    const int key = j * BN + key_l;
    __align__(16) __half kv[16];
    __align__(16) __half vv[16];
    const int phys = key < L ? p.block_table[(int64_t)b * p.max_blocks + key / p.block_size] : -1;
    const bool bad = key < L && page_bad(p, phys);
    if (bad && c == 0) raise_error(ERR_BAD_PAGE);      // its keys are packed as zero vectors
    if (key < L && !bad) {
      const int64_t off_t = (int64_t)(key % p.block_size);
      const uint8_t* krow = p.k_cache + (int64_t)phys * p.k_page_stride + off_t * p.k_tok_stride +
                            (int64_t)h * p.k_head_stride;
      const uint8_t* kb = krow + (c >> 1) * QBLOCK;
      const float dk = __half2float(__ushort_as_half(*reinterpret_cast<const uint16_t*>(kb)));
      const uint16_t* kq = reinterpret_cast<const uint16_t*>(kb + 2 + (c & 1) * 16);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const uint16_t w = kq[e];
        kv[2 * e] = __float2half_rn((float)(int8_t)(w & 0xff) * dk);
        kv[2 * e + 1] = __float2half_rn((float)(int8_t)(w >> 8) * dk);
      }
      const uint8_t* vrow = p.v_cache + (int64_t)phys * p.v_page_stride + off_t * p.v_tok_stride +
                            (int64_t)h * p.v_head_stride;
      if (v_direct) {
        // V written below
      } else if (p.v_fmt == G9_VFMT_Q8T) {
        // page-transposed record: scale (block j, token t) at 2*(j*bs + t),
        // int8 (dim, token t) at 2*(D/32)*bs + dim*bs + t
        const uint8_t* rec = p.v_cache + (int64_t)phys * p.v_page_stride + (int64_t)h * p.v_head_stride;
        const int bsz = p.block_size;
        const float dv = __half2float(__ushort_as_half(
            *reinterpret_cast<const uint16_t*>(rec + 2 * ((int64_t)(c >> 1) * bsz + off_t))));
        const int8_t* vq = reinterpret_cast<const int8_t*>(rec + 2 * (D / QK) * bsz + off_t) + (int64_t)(c * 16) * bsz;
#pragma unroll
        for (int e = 0; e < 16; ++e) vv[e] = __float2half_rn((float)vq[(int64_t)e * bsz] * dv);
      } else if (p.v_fmt == G9_VFMT_Q8) {
        const uint8_t* vb = vrow + (c >> 1) * QBLOCK;
        const float dv = __half2float(__ushort_as_half(*reinterpret_cast<const uint16_t*>(vb)));
        const uint16_t* vq = reinterpret_cast<const uint16_t*>(vb + 2 + (c & 1) * 16);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const uint16_t w = vq[e];
          vv[2 * e] = __float2half_rn((float)(int8_t)(w & 0xff) * dv);
          vv[2 * e + 1] = __float2half_rn((float)(int8_t)(w >> 8) * dv);
        }
      } else if (p.v_fmt == G9_VFMT_F16) {
        const uint32_t* v32 = reinterpret_cast<const uint32_t*>(vrow + c * 32);
#pragma unroll
        for (int e = 0; e < 8; ++e) reinterpret_cast<uint32_t*>(vv)[e] = v32[e];
      } else {   // bf16 V -> fp16 (the MMA uses fp16 for P and V)
        const __nv_bfloat16* vb16 = reinterpret_cast<const __nv_bfloat16*>(vrow + c * 32);
#pragma unroll
        for (int e = 0; e < 16; ++e) vv[e] = __float2half_rn(__bfloat162float(vb16[e]));
      }
    } else {
#pragma unroll
      for (int e = 0; e < 16; ++e) kv[e] = vv[e] = __float2half_rn(0.f);
    }
    uint4* kd = reinterpret_cast<uint4*>(kdst + (int64_t)key_l * D + c * 16);
    kd[0] = reinterpret_cast<uint4*>(kv)[0];
    kd[1] = reinterpret_cast<uint4*>(kv)[1];
    if (!v_direct) {
      uint4* vsd = reinterpret_cast<uint4*>(&vs[key_l][c * 16]);
      vsd[0] = reinterpret_cast<uint4*>(vv)[0];
      vsd[1] = reinterpret_cast<uint4*>(vv)[1];
    }
  }
  if (v_direct) {
    // item = (dim d, 16-key group g); a warp covers 32 consecutive dims of one
    // group: 32 contiguous 16-byte loads when the page holds 16 tokens
    const int bsz = p.block_size;
    for (int it = threadIdx.x; it < D * (BN / 16); it += blockDim.x) {
      const int d = it % D;
      const int g = it / D;
      const int key = j * BN + g * 16;
      __align__(16) __half o16[16];
      const int phys = key < L ? p.block_table[(int64_t)b * p.max_blocks + key / bsz] : -1;
      if (key < L && !page_bad(p, phys)) {
        const int off_t = key % bsz;
        const uint8_t* rec = p.v_cache + (int64_t)phys * p.v_page_stride + (int64_t)h * p.v_head_stride;
        const uint4 q = *reinterpret_cast<const uint4*>(rec + 2 * (D / QK) * bsz + (int64_t)d * bsz + off_t);
        const uint4* sc = reinterpret_cast<const uint4*>(rec + 2 * ((int64_t)(d / QK) * bsz + off_t));
        __align__(16) __half dv[16];
        reinterpret_cast<uint4*>(dv)[0] = sc[0];
        reinterpret_cast<uint4*>(dv)[1] = sc[1];
        const int8_t* qb = reinterpret_cast<const int8_t*>(&q);
        const int nvalid = min(16, L - key);
#pragma unroll
        for (int e = 0; e < 16; ++e)
          o16[e] = e < nvalid ? __float2half_rn((float)qb[e] * __half2float(dv[e])) : __float2half_rn(0.f);
      } else {
#pragma unroll
        for (int e = 0; e < 16; ++e) o16[e] = __float2half_rn(0.f);
      }
      uint4* dst = reinterpret_cast<uint4*>(vdst + (int64_t)d * BN + g * 16);
      dst[0] = reinterpret_cast<uint4*>(o16)[0];
      dst[1] = reinterpret_cast<uint4*>(o16)[1];
    }
    return;
  }
  __syncthreads();
  // transposed write: V^T tile [d][key], 8 keys (16 bytes) per item
  for (int it = threadIdx.x; it < D * (BN / 8); it += blockDim.x) {
    const int d = it / (BN / 8);
    const int k8 = (it % (BN / 8)) * 8;
    __align__(16) __half t8[8];
#pragma unroll
    for (int e = 0; e < 8; ++e)
      t8[e] = vs[k8 + e][d];
    *reinterpret_cast<uint4*>(vdst + (int64_t)d * BN + k8) = *reinterpret_cast<uint4*>(t8);
  }
}

// Q tile (head h, row tile rt): rows r = t*G + g -> fp16.
__global__ void __launch_bounds__(256) pack_q_kernel(const __grid_constant__ PrefillParams pp) {
  using namespace pf;
  const G9AttnBatch& p = pp.p;
  const int rt = blockIdx.x;
  const int h = blockIdx.y;
  const int i = find_seq(pp.rtile_off, pp.nseq, rt);
  const int m = rt - pp.rtile_off[i];
  const int b = pp.seq_b[i];
  const int nq = seq_nq(p, b);
  if (nq * pp.G <= pp.min_rows) return;
  __half* dst = pp.qp + ((int64_t)h * pp.RT + rt) * BM * D;
  for (int it = threadIdx.x; it < BM * (D / 8); it += blockDim.x) {
    const int r = it / (D / 8);
    const int c8 = (it % (D / 8)) * 8;
    const int rg = m * BM + r;
    const int t = rg / pp.G;
    __align__(16) __half v[8];
    if (t < nq) {
      const int hq = h * pp.G + (rg - t * pp.G);
      const int64_t base = q_offset(p, b, t, hq) + c8;
#pragma unroll
      for (int e = 0; e < 8; ++e) v[e] = __float2half_rn(load_one(p.q, base + e, p.q_dtype));
    } else {
#pragma unroll
      for (int e = 0; e < 8; ++e) v[e] = __float2half_rn(0.f);
    }
    *reinterpret_cast<uint4*>(dst + (int64_t)r * D + c8) = *reinterpret_cast<uint4*>(v);
  }
}

// ===========================================================================
// tcgen05 / TMA / TMEM wrappers
// ===========================================================================
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* tm, int c0, int c1, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
      ::"r"(smem_u32(dst)), "l"(tm), "r"(c0), "r"(c1), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
               ::"r"(smem_u32(bar)) : "memory");
}

// D[tmem] (+)= A[smem desc] * B[smem desc]^T
__device__ __forceinline__ void tc_mma_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                          uint32_t accum) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
      ::"r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accum)
      : "memory");
}

// D[tmem] (+)= A[tmem] * B[smem desc]^T
__device__ __forceinline__ void tc_mma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                          uint32_t accum) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}"
      ::"r"(d_tmem), "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accum)
      : "memory");
}

// 32 consecutive 32-bit columns of this warp's 32 lanes
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};"
      ::"r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
        "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]),
        "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]),
        "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}

__device__ __forceinline__ uint32_t tmem_ld1(uint32_t taddr) {
  uint32_t r;
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x1.b32 {%0}, [%1];" : "=r"(r) : "r"(taddr));
  return r;
}

__device__ __forceinline__ void tmem_st1(uint32_t taddr, uint32_t r) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x1.b32 [%0], {%1};" ::"r"(taddr), "r"(r) : "memory");
}

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Shared-memory matrix descriptor: K-major, 128-byte swizzle, 8-row groups
// 1024 bytes apart (the layout TMA writes for a box of 64 fp16 x rows).
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFF);            // start address
  d |= (uint64_t)1 << 16;                            // leading byte offset (unused for SW128 K-major)
  d |= (uint64_t)(1024 >> 4) << 32;                  // stride byte offset
  d |= (uint64_t)1 << 46;                            // descriptor version (sm_100)
  d |= (uint64_t)2 << 61;                            // SWIZZLE_128B
  return d;
}

// Instruction descriptor, kind::f16: fp16 A/B, fp32 D, both K-major.
constexpr uint32_t kIdesc = (1u << 4)                       // D format f32
                            | (0u << 7) | (0u << 10)        // A, B f16
                            | ((uint32_t)(pf::BN >> 3) << 17)   // N
                            | ((uint32_t)(pf::BM >> 4) << 24);  // M

// ===========================================================================
// attention kernel
// ===========================================================================
// Packed fp32 pairs (Blackwell f32x2 arithmetic: one instruction, two lanes).
__device__ __forceinline__ uint64_t f2pack(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void f2unpack(uint64_t v, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ uint64_t f2fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}
__device__ __forceinline__ uint64_t f2add(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

// MASK: general softmax input (additive mask and/or non-positive scale);
// otherwise the max is taken on the raw scores and the scale is folded into
// one FMA per score.
//
// CTA = two 128-row query tiles of one kv head sharing every K/V tile.
// warp 0: TMA producer; warp 1: TMEM owner and MMA issuer (warps 0-3 give
// registers to the softmax warpgroups through setmaxnreg); warps 4-7:
// softmax of tile 0, warps 8-11: softmax of tile 1 (thread = row = TMEM
// lane; warp w reaches TMEM lanes 32*(w % 4) .. +31).  Tensor memory: S0 S1 (P_i written as packed
// fp16 over the first 64 columns of S_i), O0 O1.  MMA order per key tile j:
//   PV0(j)  S0(j+1)  PV1(j)  S1(j+1)
// so the tensor core works on one tile while the other tile's softmax runs.
// Tile i's S(j+1) is issued after its PV(j), which (MMAs of one thread run in
// issue order) both protects P_i(j) and means that when the softmax sees
// S_i(j+1) complete, O_i holds every PV before it and may be rescaled.
template <bool MASK>
__global__ void __launch_bounds__(pf::NTHREADS, 1) prefill_kernel(const __grid_constant__ PrefillParams pp) {
  using namespace pf;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // 1024-byte alignment for the swizzled tiles
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  uint8_t* sQ = smem;                        // 2 tiles
  uint8_t* sK = smem + 2 * TILE_BYTES;
  uint8_t* sV = sK + KST * TILE_BYTES;
  __shared__ __align__(8) uint64_t bar_q;
  __shared__ __align__(8) uint64_t bar_kfull[KST], bar_kempty[KST];
  __shared__ __align__(8) uint64_t bar_vfull[VST], bar_vempty[VST];
  __shared__ __align__(8) uint64_t bar_s[2];     // S_i tile ready (MMA -> softmax i)
  __shared__ __align__(8) uint64_t bar_p[2];     // P_i tile ready (softmax i -> MMA)
  __shared__ __align__(8) uint64_t bar_ph[2];    // first half of P_i (keys 0..63) ready
  __shared__ __align__(8) uint64_t bar_o[2];     // last PV_i finished
  __shared__ uint32_t tmem_base_sh;
  __shared__ int abort_flag;

  const G9AttnBatch& p = pp.p;
  const int warp = warp_id();
  const int lane = lane_id();

  // ---- work item: heavy (late) row-tile pairs first ---------------------------
  const int idx = blockIdx.x;
  const int h = idx % pp.Hkv;
  const int grt = pp.RT - 2 - 2 * (idx / pp.Hkv);          // first global row tile of the pair
  const int si = find_seq(pp.rtile_off, pp.nseq, grt);
  const int m = grt - pp.rtile_off[si];
  const int b = pp.seq_b[si];
  const int nq = seq_nq(p, b);
  const int R = nq * pp.G;
  // keys of the sequence, clamped also to the staging tiles its kv bound sized
  const int kv_len = min(seq_len_kv(p, b), (pp.ktile_off[si + 1] - pp.ktile_off[si]) * BN);
  const int qabs = seq_qabs(p, b, nq, kv_len);
  const bool causal = has_causal(p);
  const int row0 = m * BM;
  if (row0 >= R || R <= pp.min_rows) return;              // padding pair / decode-sized sequence
  const bool has1 = row0 + BM < R;                         // second tile holds rows
  const int t_hi = min(nq - 1, (row0 + 2 * BM - 1) / pp.G);
  int key_end = kv_len;                                    // keys any row of the pair sees
  if (causal) key_end = min(key_end, max(0, qabs + t_hi + 1));
  const int64_t qpos0 = seq_qpos0(p, b, nq, kv_len);
  // sliding window: key tiles before the first row's window are skipped
  const int j0 = min(max(window_lo(p, qpos0, row0 / pp.G), 0) / BN, (key_end + BN - 1) / BN);
  const int nkv = (key_end + BN - 1) / BN - j0;           // key tiles j0 .. j0 + nkv - 1
  const int q_row_g = (h * pp.RT + grt) * BM;
  const int k_row_g = (h * pp.KT + pp.ktile_off[si] + j0) * BN;

  if (threadIdx.x == 0) {
    mbar_init(&bar_q, 1);
    for (int i = 0; i < KST; ++i) { mbar_init(&bar_kfull[i], 1); mbar_init(&bar_kempty[i], 1); }
    for (int i = 0; i < VST; ++i) { mbar_init(&bar_vfull[i], 1); mbar_init(&bar_vempty[i], 1); }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bar_s[i], 1); mbar_init(&bar_p[i], 128); mbar_init(&bar_ph[i], 128); mbar_init(&bar_o[i], 1);
    }
    abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    // 512 tensor-memory columns: S0 (0..127), S1 (128..255), O0 (256..383), O1 (384..511)
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;"
                 ::"r"(smem_u32(&tmem_base_sh)));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base_sh;

  if (warp < 4) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(REG_CTRL));
    if (nkv > 0 && warp == 0 && lane == 0) {
      // ======================= TMA producer ==================================
      mbar_arrive_expect_tx(&bar_q, 2 * TILE_BYTES);
      for (int i = 0; i < 2; ++i) {
        tma_load_2d(sQ + i * TILE_BYTES, &pp.tm_q, 0, q_row_g + i * BM, &bar_q);
        tma_load_2d(sQ + i * TILE_BYTES + TILE_BYTES / 2, &pp.tm_q, 64, q_row_g + i * BM, &bar_q);
      }
      for (int j = 0; j < nkv; ++j) {
        const int ks = j % KST;
        if (j >= KST && !mbar_wait(&bar_kempty[ks], ((j / KST) - 1) & 1)) { abort_flag = 1; break; }
        uint8_t* kd = sK + ks * TILE_BYTES;
        mbar_arrive_expect_tx(&bar_kfull[ks], TILE_BYTES);
        tma_load_2d(kd, &pp.tm_k, 0, k_row_g + j * BN, &bar_kfull[ks]);   // key tile j0 + j
        tma_load_2d(kd + TILE_BYTES / 2, &pp.tm_k, 64, k_row_g + j * BN, &bar_kfull[ks]);
        const int vs = j % VST;
        if (j >= VST && !mbar_wait(&bar_vempty[vs], ((j / VST) - 1) & 1)) { abort_flag = 1; break; }
        uint8_t* vd = sV + vs * TILE_BYTES;
        mbar_arrive_expect_tx(&bar_vfull[vs], TILE_BYTES);
        tma_load_2d(vd, &pp.tm_v, 0, k_row_g + j * BN, &bar_vfull[vs]);
        tma_load_2d(vd + TILE_BYTES / 2, &pp.tm_v, 64, k_row_g + j * BN, &bar_vfull[vs]);
      }
    } else if (nkv > 0 && warp == 1 && lane == 0) {
      // ======================= MMA issuer ====================================
      const uint32_t q_s = smem_u32(sQ);
      auto issue_s = [&](int i, int j) {
        const uint32_t k_s = smem_u32(sK + (j % KST) * TILE_BYTES);
        const uint32_t qi = q_s + i * TILE_BYTES;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk >> 2) * (TILE_BYTES / 2) + (kk & 3) * 32;
          tc_mma_ss(tmem + i * 128, sw128_desc(qi + off), sw128_desc(k_s + off), kIdesc, kk > 0);
        }
        tc_commit(&bar_s[i]);
      };
      // half h of O_i += P_i V: keys 64h .. 64h+63 (P columns 32h .. 32h+31)
      auto issue_pv = [&](int i, int j, int h) {
        const uint32_t v_s = smem_u32(sV + (j % VST) * TILE_BYTES);
#pragma unroll
        for (int k4 = 0; k4 < BN / 32; ++k4) {
          const int kk = h * (BN / 32) + k4;
          const uint32_t off = (kk >> 2) * (TILE_BYTES / 2) + (kk & 3) * 32;
          tc_mma_ts(tmem + 256 + i * 128, tmem + i * 128 + kk * 8, sw128_desc(v_s + off), kIdesc,
                    (j > 0 || kk > 0) ? 1u : 0u);
        }
      };
      bool ok = mbar_wait(&bar_q, 0) && mbar_wait(&bar_kfull[0], 0);
      if (ok) {
        tc_fence_after();
        issue_s(0, 0);
        if (has1) issue_s(1, 0);
        tc_commit(&bar_kempty[0]);
      }
      for (int j = 0; ok && j < nkv; ++j) {
        const bool more = j + 1 < nkv;
        if (!mbar_wait(&bar_vfull[j % VST], (j / VST) & 1)) { ok = false; break; }
        if (more && !mbar_wait(&bar_kfull[(j + 1) % KST], ((j + 1) / KST) & 1)) { ok = false; break; }
        // P_i V starts on the first half of P_i while the softmax still
        // computes the second half
        if (!mbar_wait(&bar_ph[0], j & 1)) { ok = false; break; }
        tc_fence_after();
        issue_pv(0, j, 0);
        if (!mbar_wait(&bar_p[0], j & 1)) { ok = false; break; }
        tc_fence_after();
        issue_pv(0, j, 1);
        if (more) issue_s(0, j + 1);
        if (has1) {
          if (!mbar_wait(&bar_ph[1], j & 1)) { ok = false; break; }
          tc_fence_after();
          issue_pv(1, j, 0);
          if (!mbar_wait(&bar_p[1], j & 1)) { ok = false; break; }
          tc_fence_after();
          issue_pv(1, j, 1);
          if (more) issue_s(1, j + 1);
        }
        tc_commit(&bar_vempty[j % VST]);
        if (more) tc_commit(&bar_kempty[(j + 1) % KST]);
      }
      if (ok) { tc_commit(&bar_o[0]); tc_commit(&bar_o[1]); }
      if (!ok) abort_flag = 1;
    }
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(REG_SOFTMAX));
    const int wi = (warp - 4) >> 2;                        // query tile of this warpgroup
    const int r = (warp & 3) * 32 + lane;                  // TMEM lane == row
    const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
    const uint32_t tS = tmem + wi * 128;
    const uint32_t tO = tmem + 256 + wi * 128;
    const int rg = row0 + wi * BM + r;
    const int t = rg / pp.G;
    const bool row_valid = rg < R;
    int row_end = kv_len;                                  // keys this row sees
    if (causal) row_end = min(row_end, max(0, qabs + t + 1));
    if (!row_valid) row_end = 0;
    const int row_lo = window_lo(p, qpos0, t);             // and its window's first key
    // keys every row of this tile sees
    int key_full = kv_len;
    if (causal) key_full = min(key_full, max(0, qabs + (row0 + wi * BM) / pp.G + 1));
    const bool active = nkv > 0 && (wi == 0 || has1);
    float m_run = -INFINITY, l_run = 0.f;                  // log2 units, scale applied
    bool alive = true;
    for (int j = 0; active && j < nkv && alive; ++j) {
      if (!mbar_wait(&bar_s[wi], j & 1)) alive = false;
      if (!__all_sync(0xffffffffu, alive)) { alive = false; break; }
      tc_fence_after();
      uint32_t s[4][32];
#pragma unroll
      for (int c = 0; c < 4; ++c) tmem_ld32(tS + lane_off + c * 32, s[c]);
      tmem_wait_ld();
      const int k0 = (j0 + j) * BN;
      const bool need_mask = MASK || (k0 + BN > key_full) || !row_valid;
      if (need_mask) {
#pragma unroll
        for (int c = 0; c < 4; ++c)
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            float x = __uint_as_float(s[c][e]);
            const int k = k0 + c * 32 + e;
            if constexpr (MASK) {
              // general scores: soft-cap, additive mask, sliding window
              x = p.softcap > 0.f ? softcap_log2(x, pp.cap_in, pp.cap_out) : x * pp.scale_log2;
              if (p.mask && row_valid && k < kv_len)
                x += kLog2e * __half2float(reinterpret_cast<const __half*>(p.mask)[
                    (int64_t)b * p.mask_seq_stride + (int64_t)t * p.mask_tok_stride + k]);
              if (k < row_lo) x = -INFINITY;
            }
            if (k >= row_end) x = -INFINITY;
            s[c][e] = __float_as_uint(x);
          }
      }
      float mc[4];
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        mc[c] = __uint_as_float(s[c][0]);
#pragma unroll
        for (int e = 1; e < 31; e += 2) mc[c] = fmax3(mc[c], __uint_as_float(s[c][e]), __uint_as_float(s[c][e + 1]));
        mc[c] = fmaxf(mc[c], __uint_as_float(s[c][31]));
      }
      float mx = fmaxf(fmaxf(mc[0], mc[1]), fmaxf(mc[2], mc[3]));
      if constexpr (!MASK) mx *= pp.scale_log2;   // scale > 0: max commutes with the scale
      // lazy rescale: keep the old max unless the new one exceeds it by
      // more than 2^8.  tcgen05.ld/st are warp-collective, so the O rescale
      // is decided by a warp vote; rows that do not need it scale by 1.
      float alpha = 1.f;
      bool rescale_o = false;
      if (mx != -INFINITY && (m_run == -INFINITY || mx > m_run + kRescaleThreshold)) {
        if (m_run != -INFINITY) {
          alpha = fast_exp2(m_run - mx);
          l_run *= alpha;
          rescale_o = j > 0;
        }
        m_run = mx;
      }
      if (__any_sync(0xffffffffu, rescale_o)) {
        // S_i(j) complete => every earlier PV_i complete: rescale O_i in place
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint32_t o[32];
          tmem_ld32(tO + lane_off + c * 32, o);
          tmem_wait_ld();
#pragma unroll
          for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * alpha);
          tmem_st32(tO + lane_off + c * 32, o);
        }
      }
      // P = 2^(x - m), all on MUFU (ex2.approx).  Moving a share to a
      // polynomial on the FMA pipe measured slower on the current kernel
      // (32K prefill: 1/4 of the pairs 1065-1090, 1/8 1131-1146, none
      // 1147-1172 TFLOP/s): the softmax warps are bound by issue slots, and
      // the polynomial costs about six per score against one MUFU issue.
      const float mu = m_run == -INFINITY ? 0.f : m_run;
      const float sc = MASK ? 1.f : pp.scale_log2;
      const uint64_t sc2 = f2pack(sc, sc);
      const uint64_t nmu2 = f2pack(-mu, -mu);
      uint64_t ls2[2] = {0ull, 0ull};                     // row-sum pairs (0.0f bit pattern is 0)
#pragma unroll
      for (int c = 0; c < 8; ++c) {                        // 16 keys -> 8 packed columns
        uint32_t pk[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const uint64_t x2 = f2fma(f2pack(__uint_as_float(s[c >> 1][(c & 1) * 16 + 2 * e]),
                                           __uint_as_float(s[c >> 1][(c & 1) * 16 + 2 * e + 1])), sc2, nmu2);
          float x0, x1;
          f2unpack(x2, x0, x1);
          const uint64_t p2 = f2pack(fast_exp2(x0), fast_exp2(x1));
          ls2[e & 1] = f2add(ls2[e & 1], p2);
          float p0, p1;
          f2unpack(p2, p0, p1);
          pk[e] = pack_half2(p0, p1);
        }
        asm volatile(
            "tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};"
            ::"r"(tS + lane_off + c * 8), "r"(pk[0]), "r"(pk[1]), "r"(pk[2]), "r"(pk[3]), "r"(pk[4]),
              "r"(pk[5]), "r"(pk[6]), "r"(pk[7])
            : "memory");
        if (c == 3) {
          // keys 0..63 of P (and any rescale of O above) are in tensor memory:
          // the first half of P V may start
          tmem_wait_st();
          tc_fence_before();
          mbar_arrive(&bar_ph[wi]);
        }
      }
      {
        float a0, a1, b0, b1;
        f2unpack(ls2[0], a0, a1);
        f2unpack(ls2[1], b0, b1);
        l_run += (a0 + a1) + (b0 + b1);
      }
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&bar_p[wi]);
    }
    // ---- epilogue: O / l -> out ---------------------------------------------------
    if (active) {
      if (alive && mbar_wait(&bar_o[wi], 0)) {
        tc_fence_after();
        const int g = rg - t * pp.G;
        if (p.sinks && l_run > 0.f) l_run += fast_exp2(sink_log2(p, h * pp.G + g) - m_run);
        const float inv = (l_run > 0.f ? 1.f / l_run : 0.f) * out_quant_factor(p);
        if (pp.out_vec) {
          // Rows are staged in the (now idle) K/V stages, then written as
          // contiguous 16-byte pieces of each row: a thread-per-row store
          // touches 32 sectors per warp instruction.  Every MMA has finished
          // (bar_o follows the last one), so no tensor-core read of the K/V
          // stages is outstanding.  Row pitch = row bytes + 16: the 16-byte
          // stores of 8 consecutive rows hit distinct banks.
          const int es = p.out_dtype == DT_F32 ? 4 : p.out_dtype == DT_FP8 ? 1 : 2;
          const int rb = D * es;
          const int pitch = rb + 16;
          uint8_t* stage = sK + (warp - 4) * 32 * (D * 4 + 16);
          uint8_t* myrow = stage + lane * pitch;
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            uint32_t o[32];
            tmem_ld32(tO + lane_off + c * 32, o);
            tmem_wait_ld();
            uint32_t w[16];
            if (p.out_dtype == DT_F32) {
#pragma unroll
              for (int q4 = 0; q4 < 8; ++q4) {
                const float4 v = make_float4(__uint_as_float(o[4 * q4]) * inv, __uint_as_float(o[4 * q4 + 1]) * inv,
                                             __uint_as_float(o[4 * q4 + 2]) * inv, __uint_as_float(o[4 * q4 + 3]) * inv);
                *reinterpret_cast<float4*>(myrow + c * 128 + q4 * 16) = v;
              }
            } else if (p.out_dtype == DT_FP8) {
#pragma unroll
              for (int e = 0; e < 32; e += 4) {
                const __nv_fp8x2_storage_t lo = __nv_cvt_float2_to_fp8x2(
                    make_float2(__uint_as_float(o[e]) * inv, __uint_as_float(o[e + 1]) * inv), __NV_SATFINITE, __NV_E4M3);
                const __nv_fp8x2_storage_t hi = __nv_cvt_float2_to_fp8x2(
                    make_float2(__uint_as_float(o[e + 2]) * inv, __uint_as_float(o[e + 3]) * inv), __NV_SATFINITE, __NV_E4M3);
                w[e / 4] = (uint32_t)lo | ((uint32_t)hi << 16);
              }
              *reinterpret_cast<uint4*>(myrow + c * 32) = make_uint4(w[0], w[1], w[2], w[3]);
              *reinterpret_cast<uint4*>(myrow + c * 32 + 16) = make_uint4(w[4], w[5], w[6], w[7]);
            } else {
#pragma unroll
              for (int e = 0; e < 32; e += 2)
                w[e / 2] = p.out_dtype == DT_F16
                               ? pack_half2(__uint_as_float(o[e]) * inv, __uint_as_float(o[e + 1]) * inv)
                               : pack_bf162(__uint_as_float(o[e]) * inv, __uint_as_float(o[e + 1]) * inv);
#pragma unroll
              for (int q4 = 0; q4 < 4; ++q4)
                *reinterpret_cast<uint4*>(myrow + c * 64 + q4 * 16) =
                    make_uint4(w[4 * q4], w[4 * q4 + 1], w[4 * q4 + 2], w[4 * q4 + 3]);
            }
          }
          __syncwarp();
          const int cpr = rb / 16;                        // 16-byte pieces per row
          const int rpi = 32 / cpr;                       // rows per warp instruction
          const int wrow0 = row0 + wi * BM + (warp & 3) * 32;
          for (int rr = lane / cpr; rr < 32; rr += rpi) {
            const int rgw = wrow0 + rr;
            if (rgw >= R) break;
            const int tw = rgw / pp.G;
            const int64_t obw = o_offset(p, b, tw, h * pp.G + (rgw - tw * pp.G)) * es;
            const int pc = lane % cpr;
            *reinterpret_cast<uint4*>(reinterpret_cast<uint8_t*>(p.out) + obw + pc * 16) =
                *reinterpret_cast<const uint4*>(stage + rr * pitch + pc * 16);
          }
        } else {
          const int64_t ob = row_valid ? o_offset(p, b, t, h * pp.G + g) : 0;
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            uint32_t o[32];
            tmem_ld32(tO + lane_off + c * 32, o);
            tmem_wait_ld();
            if (row_valid) {
#pragma unroll
              for (int e = 0; e < 32; e += 2)
                store_out2(p.out, p.out_dtype, ob + c * 32 + e, __uint_as_float(o[e]) * inv,
                           __uint_as_float(o[e + 1]) * inv);
            }
          }
        }
      } else {
        abort_flag = 1;
      }
    } else if (nkv == 0 && row_valid) {
      // no visible key for any row of this pair: zeros
      const int64_t ob = o_offset(p, b, t, h * pp.G + (rg - t * pp.G));
      for (int e = 0; e < D; e += 2) store_out2(p.out, p.out_dtype, ob + e, 0.f, 0.f);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0 && abort_flag) raise_error(ERR_WAIT_TIMEOUT);
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;" ::"r"(tmem));
  }
}

// ===========================================================================
// host side
// ===========================================================================
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn get_encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(f);
  }
  return fn;
}

// 2-D fp16 tensor [rows][128], box 64 x box_rows, 128-byte swizzle
static bool make_tmap(CUtensorMap* tm, const void* base, int64_t rows, int box_rows) {
  EncodeTiledFn enc = get_encode_fn();
  if (!enc) return false;
  cuuint64_t dims[2] = {(cuuint64_t)pf::D, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)pf::D * 2};
  cuuint32_t box[2] = {64, (cuuint32_t)box_rows};
  cuuint32_t es[2] = {1, 1};
  return enc(tm, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box, es,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

struct PrefillPlan {
  int RT = 0, KT = 0;
  size_t q_bytes = 0, k_bytes = 0, v_bytes = 0, total = 0;
};

// n_q caps and kv caps are host-side upper bounds
static PrefillPlan plan_prefill(const G9AttnBatch& p, int nseq, const int* nq_cap, const int* kv_cap) {
  PrefillPlan pl;
  const int G = p.num_heads_q / p.num_heads_kv;
  for (int i = 0; i < nseq; ++i) {
    pl.RT += 2 * (int)(((int64_t)nq_cap[i] * G + 2 * pf::BM - 1) / (2 * pf::BM));   // whole tile pairs
    pl.KT += (kv_cap[i] + pf::BN - 1) / pf::BN;
  }
  const size_t tile = (size_t)pf::TILE_BYTES;
  pl.q_bytes = (size_t)p.num_heads_kv * pl.RT * tile;
  pl.k_bytes = (size_t)p.num_heads_kv * pl.KT * tile;
  pl.v_bytes = pl.k_bytes;
  pl.total = pl.q_bytes + pl.k_bytes + pl.v_bytes + 1024;
  return pl;
}

// Sequences run in groups of at most MAXS whose fp16 staging fits kGroupBudget
// (a single sequence above it forms a group alone); groups run one after the
// other on the same workspace.  So a batch of many long padded sequences (the
// reference API's [B, Hq, Sq_pad, D] layout) needs the staging of its largest
// group, not of the whole batch.  Returns the end of the group starting at base.
constexpr size_t kGroupBudget = (size_t)1 << 30;
static int group_end(const G9AttnBatch& p, int nseq, const int* nq_cap, const int* kv_cap, int base) {
  const int G = p.num_heads_q / p.num_heads_kv;
  const size_t tile = (size_t)pf::TILE_BYTES * p.num_heads_kv;
  size_t bytes = 1024;                                  // plan_prefill's total, grown one sequence at a time
  int end = base;
  while (end < nseq && end - base < pf::MAXS) {
    const size_t rt = 2 * (size_t)(((int64_t)nq_cap[end] * G + 2 * pf::BM - 1) / (2 * pf::BM));
    const size_t kt = (size_t)((kv_cap[end] + pf::BN - 1) / pf::BN);
    const size_t add = (rt + 2 * kt) * tile;
    if (end > base && bytes + add > kGroupBudget) break;
    bytes += add;
    ++end;
  }
  return end;
}

static cudaError_t check_prefill_batch(const G9AttnBatch& p) {
  if (p.head_dim != pf::D) return cudaErrorInvalidValue;
  if (p.num_heads_kv <= 0 || p.num_heads_q <= 0 || p.num_heads_q % p.num_heads_kv) return cudaErrorInvalidValue;
  if (p.block_size <= 0 || p.q_dtype < 0 || p.q_dtype > 2 || p.out_dtype < 0 || p.out_dtype > 3) return cudaErrorInvalidValue;
  if (p.out_dtype == G9_DT_FP8E4M3 && !p.out_scale) return cudaErrorInvalidValue;
  if (p.v_fmt < 0 || p.v_fmt > 3) return cudaErrorInvalidValue;
  // K rows and Q8_0 V rows are read with 2-byte loads, 16-bit V rows with 4-byte loads
  if (((uintptr_t)p.k_cache | (uintptr_t)p.k_page_stride | (uintptr_t)p.k_tok_stride | (uintptr_t)p.k_head_stride) & 1)
    return cudaErrorInvalidValue;
  const uintptr_t va = (p.v_fmt == G9_VFMT_Q8 || p.v_fmt == G9_VFMT_Q8T) ? 1 : 3;
  if (((uintptr_t)p.v_cache | (uintptr_t)p.v_page_stride | (uintptr_t)p.v_tok_stride | (uintptr_t)p.v_head_stride) & va)
    return cudaErrorInvalidValue;
  return cudaSuccess;
}

cudaError_t run_prefill(const G9AttnBatch& p, int nseq, const int* seq_ids, const int* nq_cap,
                        const int* kv_cap, int min_rows, void* ws, size_t ws_bytes, cudaStream_t stream) {
  using namespace pf;
  cudaError_t e = check_prefill_batch(p);
  if (e != cudaSuccess) return e;
  for (int next = 0; next < nseq;) {
    const int base = next;
    const int n = group_end(p, nseq, nq_cap, kv_cap, base) - base;
    next = base + n;
    PrefillPlan pl = plan_prefill(p, n, nq_cap + base, kv_cap + base);
    if (pl.RT == 0) continue;
    if (!ws || ws_bytes < pl.total) return cudaErrorInvalidValue;
    PrefillParams pp;
    memset(&pp, 0, sizeof(pp));
    pp.p = p;
    pp.G = p.num_heads_q / p.num_heads_kv;
    pp.Hkv = p.num_heads_kv;
    pp.nseq = n;
    pp.min_rows = min_rows;
    pp.scale_log2 = p.scale * kLog2e;
    {
      const int64_t es = p.out_dtype == DT_F32 ? 4 : p.out_dtype == DT_FP8 ? 1 : 2;
      pp.out_vec = (reinterpret_cast<uintptr_t>(p.out) % 16 == 0) && (p.o_seq_stride * es) % 16 == 0 &&
                   (p.o_tok_stride * es) % 16 == 0 && (p.o_head_stride * es) % 16 == 0;
      pp.v_direct = p.v_fmt == G9_VFMT_Q8T && p.block_size % 16 == 0 &&
                    reinterpret_cast<uintptr_t>(p.v_cache) % 16 == 0 && p.v_page_stride % 16 == 0 &&
                    p.v_head_stride % 16 == 0;
    }
    if (p.softcap > 0.f) {
      pp.cap_in = p.scale / p.softcap;
      pp.cap_out = p.softcap * kLog2e;
    }
    int ro = 0, ko = 0;
    for (int i = 0; i < n; ++i) {
      pp.seq_b[i] = seq_ids[base + i];
      pp.rtile_off[i] = ro;
      pp.ktile_off[i] = ko;
      ro += 2 * (int)(((int64_t)nq_cap[base + i] * pp.G + 2 * BM - 1) / (2 * BM));
      ko += (kv_cap[base + i] + BN - 1) / BN;
    }
    pp.rtile_off[n] = ro;
    pp.ktile_off[n] = ko;
    pp.RT = ro;
    pp.KT = ko;
    uint8_t* w = reinterpret_cast<uint8_t*>(((uintptr_t)ws + 1023) & ~(uintptr_t)1023);
    pp.qp = reinterpret_cast<__half*>(w);
    pp.kp = reinterpret_cast<__half*>(w + pl.q_bytes);
    pp.vt = reinterpret_cast<__half*>(w + pl.q_bytes + pl.k_bytes);
    if (!make_tmap(&pp.tm_q, pp.qp, (int64_t)pp.Hkv * pp.RT * BM, BM) ||
        !make_tmap(&pp.tm_k, pp.kp, (int64_t)pp.Hkv * std::max(pp.KT, 1) * BN, BN) ||
        !make_tmap(&pp.tm_v, pp.vt, (int64_t)pp.Hkv * std::max(pp.KT, 1) * D, BN))
      return cudaErrorInvalidValue;
    if (pp.KT > 0) {
      pack_kv_kernel<<<dim3(pp.KT, pp.Hkv), 256, 0, stream>>>(pp);
      if ((e = cudaGetLastError()) != cudaSuccess) return e;
    }
    pack_q_kernel<<<dim3(pp.RT, pp.Hkv), 256, 0, stream>>>(pp);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    const size_t smem = (size_t)(2 + KST + VST) * TILE_BYTES + 1024;
    // general score path: mask, non-positive scale, soft-cap or sliding window
    const bool general = p.mask || !(p.scale > 0.f) || p.softcap > 0.f || p.window > 0;
    auto kern = general ? prefill_kernel<true> : prefill_kernel<false>;
    if ((e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem)) != cudaSuccess)
      return e;
    kern<<<pp.Hkv * (pp.RT / 2), NTHREADS, smem, stream>>>(pp);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
  }
  return cudaSuccess;
}

size_t prefill_ws_bytes(const G9AttnBatch& p, int nseq, const int* nq_cap, const int* kv_cap) {
  size_t best = 0;
  for (int base = 0; base < nseq;) {
    const int n = group_end(p, nseq, nq_cap, kv_cap, base) - base;
    best = std::max(best, plan_prefill(p, n, nq_cap + base, kv_cap + base).total);
    base += n;
  }
  return best;
}

}  // namespace g9

G9_ERROR_ACCESSORS(prefill)

using namespace g9;

extern "C" size_t gfx906_fa_prefill_workspace_size(const G9AttnBatch* batch, int num_prefill_seqs,
                                                   const int* nq_cap, const int* kv_cap) {
  if (!batch || num_prefill_seqs < 0 || (num_prefill_seqs > 0 && (!nq_cap || !kv_cap))) return 0;
  if (batch->num_heads_kv <= 0 || batch->num_heads_q <= 0) return 0;
  return prefill_ws_bytes(*batch, num_prefill_seqs, nq_cap, kv_cap);
}

extern "C" cudaError_t gfx906_fa_prefill_tc(const G9AttnBatch* batch, int num_prefill_seqs, const int* seq_ids,
                                            const int* nq_cap, const int* kv_cap, void* workspace,
                                            size_t workspace_bytes, cudaStream_t stream) {
  if (!batch || num_prefill_seqs < 0) return cudaErrorInvalidValue;
  if (num_prefill_seqs == 0) return cudaSuccess;
  if (!seq_ids || !nq_cap || !kv_cap) return cudaErrorInvalidValue;
  for (int i = 0; i < num_prefill_seqs; ++i)
    if (seq_ids[i] < 0 || seq_ids[i] >= batch->num_seqs || nq_cap[i] < 0 || kv_cap[i] < 0)
      return cudaErrorInvalidValue;
  return run_prefill(*batch, num_prefill_seqs, seq_ids, nq_cap, kv_cap, 0, workspace, workspace_bytes, stream);
}
