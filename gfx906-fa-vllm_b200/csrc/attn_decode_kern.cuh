#pragma once
// attn_decode_kern.cuh -- split-K flash decoding straight from the paged Q8_0 cache:
// the kernels and their launcher template.  attn_decode.cu plans a batch and
// dispatches; the attn_decode_v*.cu files instantiate the launcher per V
// format and score path (separate translation units compile in parallel).
//
//
// Replaces the reference's direct-paged tile kernel
// (kernel/fattn-q8-paged.cuh:381-641, launched by gfx906_fa_launch_paged,
// extension/gfx906_fa_launcher.cu:222-352) for short query chunks.  Design:
//
//  * Persistent CTAs (one per SM): warpgroups 0-1 compute (8 warps),
//    warpgroup 2 produces (warp 8 issues copies, warps 9-11 only hand their
//    registers to the compute warps through setmaxnreg).  The work list is
//    (KV chunk, kv-head group, sequence); CTAs walk it round-robin and the
//    producer keeps prefetching across item boundaries, so HBM stays busy
//    while a chunk's epilogue runs.
//  * The producer streams whole pages with bulk-async copies (TMA engine)
//    into a 3-slot shared-memory ring, one mbarrier per slot for "full" and
//    one for "empty".  Rows of one token (all heads of the group) are copied
//    contiguously and padded to an odd multiple of 16 bytes, which makes the
//    tensor-core operand loads bank-conflict free.
//  * GQA packing: one warp owns one kv head and computes all G query heads x
//    n_q query tokens of it (rows r = t*G + g, up to 32) against each page:
//    S = Q.K^T with mma.sync m16n8k16 (Q in fp16, K int8 converted exactly to
//    fp16, the per-block fp16 scale applied in fp32 after each 32-wide block),
//    online softmax in base 2, O += P.V with P in fp16 (bf16 for bf16 V) and
//    V as stored (or Q8_0 dequantised to fp16 in registers).  So the only
//    roundings beyond fp32 are Q and P to 16 bits and, for Q8_0 V, the
//    dequantised V to fp16.
//  * With fewer than 8 kv heads per CTA, the warps of one head split the
//    pages of a stage; each keeps its own softmax state.
//  * A chunk's result is final when the sequence has one chunk and its head
//    one warp; otherwise each warp's normalised partial O and its (max, sum)
//    go to the workspace and a combine kernel merges them (log-sum-exp
//    weights).
//
// Masking follows the reference: keys at k >= kv_len are ignored, with
// q_abs the causal rule is k <= q_abs[b] + t (fattn-q8.cuh:646-654), and an
// optional fp16 additive mask is added to the scaled score.  Rows without any
// visible key produce zeros.  Every mbarrier wait is bounded (common.cuh).
#include <algorithm>
#include <cstdlib>
#include <mutex>

#include "attn_common.cuh"

namespace g9 {

namespace dec {
constexpr int D = 128;
constexpr int PAGE = 16;
constexpr int NWC = 8;                      // compute warps (warpgroups 0, 1)
constexpr int NTHREADS = 384;               // + warpgroup 2: warp 8 produces, 9-11 exit
constexpr int MAXST = 4;                    // max pipeline slots (3 or 4 chosen per launch)
constexpr int MAXP = 16;                    // max pages per stage
constexpr int MAXG = 16;                    // max page-slot groups (compute warps / HG)
// Optional geometry of the transposed consumer at one kv head per CTA
// (GFX906_FA_DECODE_TRW=16): 16 compute warps + a producer warpgroup (640
// threads launched at 96 registers: 16*32*104 + 4*32*64 = 640*96).  The
// default is the 8-warp geometry above with two pages per warp.
constexpr int NWC_TR = 16;
constexpr int NTHREADS_TR = 640;
constexpr int REG_COMPUTE_TR = 104;
constexpr int REG_PRODUCER_TR = 64;
constexpr int kMaxRanksTR = 4095;           // (sequence, head group) pairs: prefix sums in shared memory
// 16-bit V tokens per copy group of the transposed kernel, measured over
// 2, 4, 8 (16): at 1-2 heads per CTA 8 is fastest, at 4-8 heads 4
constexpr int kVgtSmallHG = 8;
constexpr int kVgtLargeHG = 4;
constexpr int QROW = 272;                   // smem bytes per Q row (256 + pad, conflict-free ldmatrix)
// setmaxnreg split: launch 384 threads x 168 = 64512 = 256*224 + 128*56 (the producer's
// per-group stream state needs 56 to stay out of local memory)
constexpr int REG_COMPUTE = 224;
constexpr int REG_PRODUCER = 56;
constexpr float kRescaleLog2 = 8.0f;        // lazy-max threshold (log2 units): P <= 2^8
}  // namespace dec

struct DecodeParams {
  G9AttnBatch p;
  int G;                  // query heads per kv head
  int HG;                 // kv heads per CTA
  int HGN;                // head groups (num_heads_kv / HG)
  int NG;                 // page-slot groups per CTA (NWC / HG), each with its own item stream
  int P;                  // pages per stage (= NG * PPW)
  int ppw;                // pages per compute warp per stage
  int CP;                 // pages per chunk (multiple of ppw)
  int S_max;              // chunks per sequence (upper bound)
  int n_items;
  int R_pad;              // 16 * MT
  int rb_k, rb_v;         // bytes of one K / V row
  int vrec;               // page-transposed Q8_0 V: bytes of one (page, head) record
  int vrec_contig;        // 1: the records of a CTA's kv heads are adjacent (one copy per page)
  int kgs, vgs;           // smem bytes per K group (4 tokens) / V group (vgt tokens), padded to odd x 16
  int vgt;                // 16-bit V: tokens per shared-memory group
  int contig;             // 1: rows of consecutive tokens are adjacent (one copy per group)
  int kwhole;             // 1: a page's K rows are one copy into an unpadded shared-memory page
  int cps_log2;           // log2 of the producer's copy slots per page (2..32 slots)
  int joint;              // 1: a page's K rows and V records are adjacent in HBM and in shared memory (one copy)
  int kps, vbase, vps;    // shared memory: K of page slot j at kps*j, V at vbase + vps*j (stage-relative)
  int kpage, vpage;       // smem bytes per page
  int stage_bytes;
  int q_off;              // smem offset of the Q tiles (MT == 2)
  int max_rows;           // sequences with n_q * G above this are left to the prefill kernel
  int nst;                // pipeline slots of this launch
  int nt;                 // transposed consumer: n-tiles of 8 query rows
  int tr;                 // 0, or compute warps of the transposed consumer (<= 8 rows, page-transposed Q8_0 V)
  // Balanced split (the transposed kernels): units = pages of each rank
  // (sequence b, head group z; rank = b*HGN + z) in rank order; stream s of
  // the nstreams = grid*NG item streams owns units [s*T/N, (s+1)*T/N),
  // N = min(nstreams, T).  A stream's piece of one rank is a segment; its
  // partial result goes to slot s + rank.
  int nranks, nstreams;
  int qtr_off;            // smem offset of the transposed consumer's Q tiles (three n-tiles)
  int cpre_off;           // smem offset of the rank prefix sums (nranks + 1 ints)
  int* cpre_g;            // the same prefix sums, written by CTA 0 for the combine
  uint32_t tr_tab;        // transposed consumer: key order per quad (see decode_consumer_tr)
  float scale_log2;
  float cap_in, cap_out;  // soft-cap: scale / softcap and softcap * log2(e) (softcap > 0)
  unsigned int* counter;  // work-queue counter (zeroed before the launch)
  float* opart;           // [B][Hkv][S_max][R_pad][D]
  float2* ml;             // [B][Hkv][S_max][R_pad]
};

// Per stage and page-slot group (the HG warps g*HG .. g*HG+HG-1 that share
// one item): the group's item (-1: no work in this stage), its first page,
// valid pages, whether the item ends here; per page slot: copy issued.
struct StageMeta {
  int item[dec::MAXG], page0[dec::MAXG], npages[dec::MAXG], last[dec::MAXG];
  int ok[dec::MAXP];
  int done;                               // terminator: every group's stream has ended
};

__device__ __forceinline__ void decode_item(const DecodeParams& d, int item, int& b, int& z, int& s) {
  const int per = d.p.num_seqs * d.HGN;
  s = item / per;
  const int rem = item - s * per;
  b = rem / d.HGN;
  z = rem - b * d.HGN;
}

// Pages of sequence b any of its query rows can see: [ps, npg).  ps > 0 only
// with a sliding window (pages wholly before token 0's window are skipped).
__device__ __forceinline__ void seq_pages(const G9AttnBatch& p, int b, int nq, int& ps, int& npg) {
  npg = (seq_kv_end(p, b, nq) + dec::PAGE - 1) / dec::PAGE;
  ps = min(seq_kv_begin(p, b, nq) / dec::PAGE, npg);
}

// chunks of sequence b for the queue-driven kernels
__device__ __forceinline__ int seq_nsplit(const DecodeParams& d, int b, int nq) {
  int ps, npg;
  seq_pages(d.p, b, nq, ps, npg);
  return npg == ps ? 1 : (npg - ps + d.CP - 1) / d.CP;
}

// page range [pb, pe) of an item; returns false for items with nothing to do.
// An item with pe == pb (sequence without visible keys) is still emitted for
// chunk 0 so that zeros get written.
__device__ __forceinline__ bool item_pages(const DecodeParams& d, int b, int s, int& pb, int& pe,
                                           int& nsplit) {
  const int nq = seq_nq(d.p, b);
  int ps, npg;
  seq_pages(d.p, b, nq, ps, npg);
  nsplit = npg == ps ? 1 : (npg - ps + d.CP - 1) / d.CP;
  if (nq <= 0 || nq * d.G > d.max_rows || s >= nsplit) return false;
  pb = ps + s * d.CP;
  pe = min(npg, pb + d.CP);
  return true;
}


// ---------------------------------------------------------------------------
// Transposed consumer (at most 8 query rows per kv head, page-transposed
// Q8_0 V).  The query rows are the N = 8 side of m16n8k16 instead of padding
// a 16-row M tile:
//   S^T = K . Q^T   (A = 16 keys x 16 dims of K, B = 16 dims x 8 rows of Q)
//   O^T += V^T . P^T (A = 16 dims x 16 keys of V, B = 16 keys x 8 rows of P)
// so a page takes 8 + 8 MMAs instead of 16 + 16, a thread holds 4 scores per
// page instead of 8, and O^T is 32 registers.
//
// Exact int8 -> fp16 without a subtraction: (0x64 << 8) | (b ^ 0x80) is
// 1152 + b.  The K side starts each block's accumulator at -1152 * (sum of
// the block's Q dims), which cancels the offset exactly in the algebra (the
// same fp16 Q values enter both).  The V side runs one extra MMA per block
// whose A operand is a row of ones: it accumulates sum_k (P s_v)[k] with the
// same fp16 B fragment the value MMAs use, and the epilogue subtracts 1152
// times it.  V's per-(key, block) scale is applied to P (two half2 products
// per block) instead of to V.
//
// Key order: accumulator row (m-slot) s of S^T is key sigma(s); after the
// in-register transpose (movmatrix) the same slot is k-slot s of the P.V
// product, whose V^T fragment comes straight from ldmatrix rows of 16 keys:
// thread j gets keys 4j .. 4j+3, and k-slots (2j, 2j+1) take two of them
// ("lo"), (2j+8, 2j+9) the other two ("hi").  Which two go low is chosen per
// quad on the host so that the K rows a warp reads in one instruction fall
// in different shared-memory banks for the launch's K layout (tr_tab: per
// quad q, bits 8q.. hold lo0, lo1, hi0, hi1 as 2-bit positions).
// ---------------------------------------------------------------------------
// Units of a rank: its visible pages [ps, real), or one masked unit when its
// rows see no key (so that its zero output is written); 0 for sequences this
// kernel skips.  `real` returns the end of the pages that exist, `ps` the
// first page (unit u of the rank is page ps + u).
__device__ __forceinline__ int rank_units(const DecodeParams& d, int rank, int& real, int& ps) {
  const int b = rank / d.HGN;
  const int nq = seq_nq(d.p, b);
  real = 0;
  ps = 0;
  if (nq <= 0 || nq * d.G > d.max_rows) return 0;
  seq_pages(d.p, b, nq, ps, real);
  return max(real - ps, 1);
}
__device__ __forceinline__ int64_t bal_bound(int s, int64_t T, int N) { return (int64_t)s * T / N; }
// stream owning unit u (0 <= u < T, N <= T so no stream is empty)
__device__ __forceinline__ int bal_sid(int64_t u, int64_t T, int N) {
  int s = (int)(u * N / T);
  if (s + 1 < N && bal_bound(s + 1, T, N) <= u) ++s;
  return s;
}

__device__ __forceinline__ uint32_t movmatrix_trans(uint32_t a) {
  uint32_t r;
  asm("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(r) : "r"(a));
  return r;
}

// two int8 (low 16 bits of x, zero-extended) -> fp16x2 of 1152 + b
__device__ __forceinline__ uint32_t i8x2_to_h2_biased(uint32_t x) {
  return __byte_perm(x ^ 0x8080u, 0x64646464u, 0x5140);
}

// d = a.b + c with the accumulator rows (c0, c1, c0, c1)
__device__ __forceinline__ void mma_f16_16816_c(float d[4], const uint32_t a[4], const uint32_t b[2], float c0,
                                                float c1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%10,%11,%10,%11};"
      : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]), "f"(c0), "f"(c1));
}

__device__ __forceinline__ uint32_t hmul2_u32(uint32_t a, uint32_t b) {
  __half2 r = __hmul2(*reinterpret_cast<const __half2*>(&a), *reinterpret_cast<const __half2*>(&b));
  return *reinterpret_cast<uint32_t*>(&r);
}

constexpr float kRescaleLog2T = 6.0f;     // P <= 2^6: P * s_v stays finite in fp16 for any fp16 V

template <int VT, bool MASK, int NST, int PPW, int NW, int NT>
__device__ __forceinline__ void decode_consumer_tr(const DecodeParams& d, uint8_t* smem, uint64_t* full_bar,
                                                   uint64_t* empty_bar, StageMeta* meta, int warp, int lane) {
  using namespace dec;
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(NW == NWC_TR ? REG_COMPUTE_TR : REG_COMPUTE));
  const G9AttnBatch& p = d.p;
  const int hl = warp % d.HG;       // local kv head
  const int sub = warp / d.HG;      // page-slot group
  const int j4 = lane & 3;
  const int rq = lane >> 2;
  // this lane's two K rows (m-slots rq and rq + 8) and its V byte selectors
  const uint32_t tq = (d.tr_tab >> (8 * (rq >> 1))) & 0xffu;
  const int tA = 4 * (rq >> 1) + (int)((tq >> (2 * (rq & 1))) & 3u);
  const int tB = 4 * (rq >> 1) + (int)((tq >> (4 + 2 * (rq & 1))) & 3u);
  const uint32_t tj = (d.tr_tab >> (8 * j4)) & 0xffu;
  const uint32_t l0 = tj & 3u, l1 = (tj >> 2) & 3u, h0 = (tj >> 4) & 3u, h1 = (tj >> 6) & 3u;
  const uint32_t sel_lo = l0 | 0x40u | (l1 << 8) | 0x4000u;
  const uint32_t sel_hi = h0 | 0x40u | (h1 << 8) | 0x4000u;
  const uint32_t ssel_lo = (2 * l0) | ((2 * l0 + 1) << 4) | ((2 * l1) << 8) | ((2 * l1 + 1) << 12);
  const uint32_t ssel_hi = (2 * h0) | ((2 * h0 + 1) << 4) | ((2 * h1) << 8) | ((2 * h1 + 1) << 12);
  const int hgb_k = d.HG * d.rb_k;
  const uint32_t kofA = (uint32_t)((tA >> 2) * d.kgs + (tA & 3) * hgb_k + hl * d.rb_k);
  const uint32_t kofB = (uint32_t)((tB >> 2) * d.kgs + (tB & 3) * hgb_k + hl * d.rb_k);
  // 16-bit V rows: this lane's ldmatrix.trans row address (matrix mi = lane/8:
  // keys of k-slots 8*(mi/2) + lane%8, dims 8*(mi%2) .. +7 of an m-tile)
  uint32_t vkoff = 0;
  if constexpr (VT <= 1) {
    const int mi = lane >> 3, ri = lane & 7;
    const int q = ri >> 1, e = ri & 1;
    const uint32_t tqv = (d.tr_tab >> (8 * q)) & 0xffu;
    const int key = 4 * q + (int)((tqv >> ((mi >> 1) ? 4 + 2 * e : 2 * e)) & 3u);
    vkoff = (uint32_t)((key / d.vgt) * d.vgs + (key % d.vgt) * d.HG * d.rb_v + hl * d.rb_v + (mi & 1) * 16);
  }

  // n-tile nt holds query rows 8*nt .. 8*nt+7; this thread's accumulator
  // columns are rows 8*nt + 2*j4 + c, c = 0, 1
  // With three n-tiles the Q^T fragments live in this warp's shared-memory
  // Q tile (fp16 rows, QROW bytes apart) and are loaded per block with
  // ldmatrix; with fewer they stay in registers.
  constexpr bool QSM = NT >= 3;
  float o[NT][8][4];       // O^T: m-tile mt = dims 16mt .. 16mt+15
  float corr[NT][4];       // row `blk` of this tile: sum over keys of (P s_v) for block blk
  uint32_t qb[QSM ? 1 : NT][8][2];   // Q^T B fragments per 16-dim k-step (registers)
  float kc[QSM ? 1 : NT][4][2];   // -1152 * sum of block blk's Q dims, per column row (registers)
  float mrow[NT][2], lrow[NT][2];
  // item state kept live: rows, and per column row the exclusive end of its
  // visible keys (-1 for a padding row); the rest is decoded from the item
  // again at the epilogue
  int cur_item = -1, cR = 0;
  int klim[NT][2];
  int klo[MASK ? NT : 1][2];   // sliding window: first visible key per column row

  const uint32_t smem_base = smem_u32(smem);
  auto ld16 = [&](uint32_t a) { return (uint32_t)*reinterpret_cast<const uint16_t*>(smem + (a - smem_base)); };
  auto ld64 = [&](uint32_t a) { return *reinterpret_cast<const uint2*>(smem + (a - smem_base)); };
  // per warp: the Q tile, then the K-offset constants [nt][blk][row] (fp32)
  const uint32_t qs_base = smem_base + d.qtr_off + warp * (NT * 8 * QROW + 512);
  const uint32_t qk_base = qs_base + NT * 8 * QROW;
  // B fragments of k-steps 2*blk and 2*blk + 1 for n-tile nt: {b0, b1} each
  auto q_frags = [&](int nt, int blk, uint32_t q4[4]) {
    if constexpr (QSM) {
      const int mi = lane >> 3, ri = lane & 7;
      ldmatrix_x4(q4, qs_base + (8 * nt + ri) * QROW + ((2 * blk + (mi >> 1)) * 16 + (mi & 1) * 8) * 2);
    } else {
      q4[0] = qb[nt][2 * blk][0]; q4[1] = qb[nt][2 * blk][1];
      q4[2] = qb[nt][2 * blk + 1][0]; q4[3] = qb[nt][2 * blk + 1][1];
    }
  };

  auto start_item = [&](int b, int h) {
    if constexpr (QSM) __syncwarp();
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
      for (int mt = 0; mt < 8; ++mt)
#pragma unroll
        for (int c = 0; c < 4; ++c) o[nt][mt][c] = 0.f;
#pragma unroll
      for (int c = 0; c < 4; ++c) corr[nt][c] = 0.f;
      mrow[nt][0] = mrow[nt][1] = -INFINITY;
      lrow[nt][0] = lrow[nt][1] = 0.f;
    }
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      // Q row 8nt + rq: dims 16ks + 2*j4 (+1) and 16ks + 2*j4 + 8 (+9); all loads first
      const int rr = 8 * nt + rq;
      const bool v = rr < cR;
      const int t = v ? rr / d.G : 0;
      const int64_t base = v ? q_offset(p, b, t, h * d.G + (rr - t * d.G)) : 0;
      float qf[16][2];
      if (p.q_dtype == DT_F32) {
        const float* q = reinterpret_cast<const float*>(p.q);
        float2 x[16];
#pragma unroll
        for (int i = 0; i < 16; ++i)
          x[i] = v ? *reinterpret_cast<const float2*>(q + base + (i >> 1) * 16 + (i & 1) * 8 + 2 * j4)
                   : make_float2(0.f, 0.f);
#pragma unroll
        for (int i = 0; i < 16; ++i) { qf[i][0] = x[i].x; qf[i][1] = x[i].y; }
      } else {
        const uint16_t* q = reinterpret_cast<const uint16_t*>(p.q);
        uint32_t x[16];
#pragma unroll
        for (int i = 0; i < 16; ++i)
          x[i] = v ? *reinterpret_cast<const uint32_t*>(q + base + (i >> 1) * 16 + (i & 1) * 8 + 2 * j4) : 0u;
        const bool bf = p.q_dtype == DT_BF16;
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          if (bf) {
            qf[i][0] = __uint_as_float(x[i] << 16);
            qf[i][1] = __uint_as_float(x[i] & 0xffff0000u);
          } else {
            const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&x[i]));
            qf[i][0] = f.x;
            qf[i][1] = f.y;
          }
        }
      }
      float qs[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const uint32_t hq = pack_half2(qf[i][0], qf[i][1]);
        if constexpr (QSM)
          asm volatile("st.shared.u32 [%0], %1;" ::"r"(qs_base + rr * QROW + ((i >> 1) * 16 + (i & 1) * 8 + 2 * j4) * 2),
                       "r"(hq));
        else
          qb[nt][i >> 1][i & 1] = hq;
        const float2 r = __half22float2(*reinterpret_cast<const __half2*>(&hq));   // the values the MMA sees
        qs[i >> 2] += r.x + r.y;
      }
#pragma unroll
      for (int blk = 0; blk < 4; ++blk) {
        float s = qs[blk];
        s += __shfl_xor_sync(0xffffffffu, s, 1);
        s += __shfl_xor_sync(0xffffffffu, s, 2);       // row rr's block sum, on all 4 lanes of the quad
        if constexpr (QSM) {
          if (j4 == 0) asm volatile("st.shared.f32 [%0], %1;" ::"r"(qk_base + ((nt * 4 + blk) * 8 + rq) * 4), "f"(-1152.f * s));
        } else {
          kc[nt][blk][0] = -1152.f * __shfl_sync(0xffffffffu, s, 8 * j4);
          kc[nt][blk][1] = -1152.f * __shfl_sync(0xffffffffu, s, 8 * j4 + 4);
        }
      }
    }
    if constexpr (QSM) __syncwarp();
  };

  // balanced split: this warp's stream and the rank prefix sums
  const int* cpre = reinterpret_cast<const int*>(smem + d.cpre_off);
  const int sid = blockIdx.x * d.NG + sub;
  const int64_t T = cpre[d.nranks];
  const int NS = (int)(T < d.nstreams ? T : (int64_t)d.nstreams);

  auto epilogue = [&]() {
    const int rank = cur_item - sid;
    const int cb = rank / d.HGN, cz = rank - cb * d.HGN;
    // the stream holds the whole rank: final output, else a partial
    const bool whole = cpre[rank] >= bal_bound(sid, T, NS) && cpre[rank + 1] <= bal_bound(sid + 1, T, NS);
    const int h = cz * d.HG + hl;
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        float v = lrow[nt][c];
        v += __shfl_xor_sync(0xffffffffu, v, 4);
        v += __shfl_xor_sync(0xffffffffu, v, 8);
        v += __shfl_xor_sync(0xffffffffu, v, 16);
        lrow[nt][c] = v;
      }
      float cv[4][2];
#pragma unroll
      for (int blk = 0; blk < 4; ++blk) {
        cv[blk][0] = 1152.f * __shfl_sync(0xffffffffu, corr[nt][0], 4 * blk + j4);
        cv[blk][1] = 1152.f * __shfl_sync(0xffffffffu, corr[nt][1], 4 * blk + j4);
      }
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        const int r = 8 * nt + 2 * j4 + c;
        if (r >= cR) continue;
        const float l = lrow[nt][c];
        float inv = l > 0.f ? 1.f / l : 0.f;
        if (whole) {
          const int t = r / d.G;
          const int hq = h * d.G + (r - t * d.G);
          // a sink adds its weight to the denominator once, where the row is final
          if (p.sinks && l > 0.f) inv = 1.f / (l + fast_exp2(sink_log2(p, hq) - mrow[nt][c]));
          inv *= out_quant_factor(p);
          const int64_t ob = o_offset(p, cb, t, hq);
#pragma unroll
          for (int mt = 0; mt < 8; ++mt)
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) {
              const float x = (o[nt][mt][2 * hh + c] - cv[mt >> 1][c]) * inv;
              const int64_t off = ob + mt * 16 + hh * 8 + rq;
              if (p.out_dtype == DT_FP8) reinterpret_cast<uint8_t*>(p.out)[off] = to_fp8(x);
              else if (p.out_dtype == DT_F32) reinterpret_cast<float*>(p.out)[off] = x;
              else if (p.out_dtype == DT_F16) reinterpret_cast<__half*>(p.out)[off] = __float2half_rn(x);
              else reinterpret_cast<__nv_bfloat16*>(p.out)[off] = __float2bfloat16_rn(x);
            }
        } else {
          const int64_t row = ((int64_t)cur_item * d.HG + hl) * d.R_pad + r;
          float* op = d.opart + row * D;
#pragma unroll
          for (int mt = 0; mt < 8; ++mt)
#pragma unroll
            for (int hh = 0; hh < 2; ++hh)
              op[mt * 16 + hh * 8 + rq] = (o[nt][mt][2 * hh + c] - cv[mt >> 1][c]) * inv;
          if (rq == 0) d.ml[row] = make_float2(mrow[nt][c], l);
        }
      }
    }
  };

  auto begin_item = [&](int item) {
      cur_item = item;
      const int rank = item - sid;
      const int cb = rank / d.HGN, cz = rank - cb * d.HGN;
      const int cnq = seq_nq(p, cb);
      cR = cnq * d.G;
      const int ckv = seq_len_kv(p, cb);
      const int cqabs = seq_qabs(p, cb, cnq, ckv);
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          const int r = 8 * nt + 2 * j4 + c;
          int lim = ckv;
          if (has_causal(p)) lim = min(lim, cqabs + r / d.G + 1);
          klim[nt][c] = r < cR ? lim : -1;
          if constexpr (MASK) klo[nt][c] = window_lo(p, seq_qpos0(p, cb, cnq, ckv), r / d.G);
        }
      start_item(cb, cz * d.HG + hl);
  };

  // The stream's first item is known from the prefix sums alone (the
  // producer's first claim computes the same), so its Q loads go out now and
  // overlap the first page copies instead of following them.
  if (sid < NS) {
    const int64_t u = bal_bound(sid, T, NS);
    int lo = 0, hi = d.nranks;                  // last rank with cpre <= u, then past empty ranks
    while (hi - lo > 1) {
      const int mid = (lo + hi) >> 1;
      if (cpre[mid] <= u) lo = mid; else hi = mid;
    }
    while (cpre[lo + 1] <= u) ++lo;
    begin_item(sid + lo);
  }

  for (int it = 0;; ++it) {
    const int slot = it % NST;
    if (!mbar_wait(&full_bar[slot], (it / NST) & 1)) break;
    if (meta[slot].done) break;
    const int item = meta[slot].item[sub];
    const int page0 = meta[slot].page0[sub];
    const int npages = meta[slot].npages[sub];
    const bool last = meta[slot].last[sub] != 0;
    if (item >= 0 && item != cur_item) begin_item(item);
    bool pok[PPW];
    int first_ok = -1;
#pragma unroll
    for (int pp = PPW - 1; pp >= 0; --pp) {
      pok[pp] = item >= 0 && pp < npages && meta[slot].ok[sub * PPW + pp];
      if (pok[pp]) first_ok = pp;
    }
    if (first_ok >= 0) {
      int psrc[PPW];
#pragma unroll
      for (int pp = 0; pp < PPW; ++pp) psrc[pp] = sub * PPW + (pok[pp] ? pp : first_ok);
      const uint32_t stage_base = smem_base + slot * d.stage_bytes;
      // ---------------- S^T = K Q^T (K fragments shared by the n-tiles) --------
      float sacc[PPW][NT][4];
#pragma unroll
      for (int pp = 0; pp < PPW; ++pp) {
        const uint32_t kb = stage_base + psrc[pp] * d.kps;
        const uint32_t rA = kb + kofA, rB = kb + kofB;
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
          for (int c = 0; c < 4; ++c) sacc[pp][nt][c] = 0.f;
#pragma unroll
        for (int blk = 0; blk < 4; ++blk) {
          const uint32_t cA = rA + blk * QBLOCK + 2 + 2 * j4, cB = rB + blk * QBLOCK + 2 + 2 * j4;
          uint32_t a0[4], a1[4];
          a0[0] = i8x2_to_h2_biased(ld16(cA));
          a0[1] = i8x2_to_h2_biased(ld16(cB));
          a0[2] = i8x2_to_h2_biased(ld16(cA + 8));
          a0[3] = i8x2_to_h2_biased(ld16(cB + 8));
          a1[0] = i8x2_to_h2_biased(ld16(cA + 16));
          a1[1] = i8x2_to_h2_biased(ld16(cB + 16));
          a1[2] = i8x2_to_h2_biased(ld16(cA + 24));
          a1[3] = i8x2_to_h2_biased(ld16(cB + 24));
          const float dA = half_bits_to_float((uint16_t)ld16(rA + blk * QBLOCK));
          const float dB = half_bits_to_float((uint16_t)ld16(rB + blk * QBLOCK));
#pragma unroll
          for (int nt = 0; nt < NT; ++nt) {
            uint32_t q4[4];
            q_frags(nt, blk, q4);
            float acc[4];
            float k0, k1;
            if constexpr (QSM) {
              const float2 kk = *reinterpret_cast<const float2*>(smem + (qk_base - smem_base) + ((nt * 4 + blk) * 8 + 2 * j4) * 4);
              k0 = kk.x; k1 = kk.y;
            } else {
              k0 = kc[nt][blk][0]; k1 = kc[nt][blk][1];
            }
            mma_f16_16816_c(acc, a0, q4, k0, k1);
            mma_f16_16816(acc, a1, q4 + 2);
            sacc[pp][nt][0] = fmaf(acc[0], dA, sacc[pp][nt][0]);
            sacc[pp][nt][1] = fmaf(acc[1], dA, sacc[pp][nt][1]);
            sacc[pp][nt][2] = fmaf(acc[2], dB, sacc[pp][nt][2]);
            sacc[pp][nt][3] = fmaf(acc[3], dB, sacc[pp][nt][3]);
          }
        }
      }
      // ---------------- mask + online softmax (base 2, lazy max) --------------
      float tmx[NT][2];
      bool grow = false;
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          const int kv_lim = klim[nt][c];
          tmx[nt][c] = -INFINITY;
#pragma unroll
          for (int pp = 0; pp < PPW; ++pp) {
            const int k0 = (page0 + pp) * PAGE;
            const bool page_full = !MASK && pok[pp] && k0 + PAGE <= kv_lim;
#pragma unroll
            for (int hb = 0; hb < 2; ++hb) {
              float x = sacc[pp][nt][2 * hb + c] * d.scale_log2;
              if (!page_full) {
                const int k = k0 + (hb ? tB : tA);
                bool vis = pok[pp] && k < kv_lim;
                if constexpr (MASK) {
                  // general scores: soft-cap, additive mask, sliding window
                  if (p.softcap > 0.f) x = softcap_log2(sacc[pp][nt][2 * hb + c], d.cap_in, d.cap_out);
                  if (p.mask && vis) {
                    const int cb = (cur_item - sid) / d.HGN;
                    const int t = (8 * nt + 2 * j4 + c) / d.G;
                    x += kLog2e * __half2float(reinterpret_cast<const __half*>(p.mask)[
                        (int64_t)cb * p.mask_seq_stride + (int64_t)t * p.mask_tok_stride + k]);
                  }
                  vis = vis && k >= klo[nt][c];
                }
                x = vis ? x : -INFINITY;
              }
              sacc[pp][nt][2 * hb + c] = x;
              tmx[nt][c] = fmaxf(tmx[nt][c], x);
            }
          }
          grow |= tmx[nt][c] > mrow[nt][c] + kRescaleLog2T;
        }
      if (__any_sync(0xffffffffu, grow)) {
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          float alpha[2];
#pragma unroll
          for (int c = 0; c < 2; ++c) {
            float mx = tmx[nt][c];
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
            alpha[c] = 1.f;
            if (mx > mrow[nt][c] + kRescaleLog2T) {        // uniform over the lanes of this row
              alpha[c] = fast_exp2(mrow[nt][c] - mx);
              mrow[nt][c] = mx;
              lrow[nt][c] *= alpha[c];
            }
          }
#pragma unroll
          for (int mt = 0; mt < 8; ++mt) {
            o[nt][mt][0] *= alpha[0]; o[nt][mt][2] *= alpha[0];
            o[nt][mt][1] *= alpha[1]; o[nt][mt][3] *= alpha[1];
          }
          corr[nt][0] *= alpha[0]; corr[nt][2] *= alpha[0];
          corr[nt][1] *= alpha[1]; corr[nt][3] *= alpha[1];
        }
      }
      uint32_t pb[PPW][NT][2];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          const float mu = mrow[nt][c] == -INFINITY ? 0.f : mrow[nt][c];
          float ls = 0.f;
#pragma unroll
          for (int pp = 0; pp < PPW; ++pp)
#pragma unroll
            for (int hb = 0; hb < 2; ++hb) {
              const float pv = fast_exp2(sacc[pp][nt][2 * hb + c] - mu);
              sacc[pp][nt][2 * hb + c] = pv;
              ls += pv;
            }
          lrow[nt][c] += ls;
        }
#pragma unroll
        for (int pp = 0; pp < PPW; ++pp) {
          if constexpr (VT == 1) {
            pb[pp][nt][0] = movmatrix_trans(pack_bf162(sacc[pp][nt][0], sacc[pp][nt][1]));
            pb[pp][nt][1] = movmatrix_trans(pack_bf162(sacc[pp][nt][2], sacc[pp][nt][3]));
          } else {
            pb[pp][nt][0] = movmatrix_trans(pack_half2(sacc[pp][nt][0], sacc[pp][nt][1]));
            pb[pp][nt][1] = movmatrix_trans(pack_half2(sacc[pp][nt][2], sacc[pp][nt][3]));
          }
        }
      }
      // ---------------- O^T += V^T P^T (V fragments shared by the n-tiles) -----
      if constexpr (VT <= 1) {
        // 16-bit V rows: one ldmatrix.trans per 16-dim m-tile, no conversion
#pragma unroll
        for (int pp = 0; pp < PPW; ++pp) {
          const uint32_t vrow = stage_base + d.vbase + psrc[pp] * d.vps + vkoff;
#pragma unroll
          for (int mt = 0; mt < 8; ++mt) {
            uint32_t av[4];
            ldmatrix_x4_trans(av, vrow + mt * 32);
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
              if constexpr (VT == 1) mma_bf16_16816(o[nt][mt], av, pb[pp][nt]);
              else mma_f16_16816(o[nt][mt], av, pb[pp][nt]);
            }
          }
        }
      } else {
      const uint32_t ones = 0x3c003c00u;
#pragma unroll
      for (int pp = 0; pp < PPW; ++pp) {
        const uint32_t vrec = stage_base + d.vbase + psrc[pp] * d.vps + hl * d.vrec;
#pragma unroll
        for (int blk = 0; blk < 4; ++blk) {
          uint32_t r4[4];
          ldmatrix_x4(r4, vrec + 2 * 4 * PAGE + (blk * 32 + lane) * PAGE);
          const uint2 sc = ld64(vrec + blk * 2 * PAGE + 8 * j4);
          const uint32_t s_lo = __byte_perm(sc.x, sc.y, ssel_lo), s_hi = __byte_perm(sc.x, sc.y, ssel_hi);
          uint32_t w[4];
#pragma unroll
          for (int m = 0; m < 4; ++m) w[m] = r4[m] ^ 0x80808080u;
          const uint32_t av0[4] = {__byte_perm(w[0], 0x64646464u, sel_lo), __byte_perm(w[1], 0x64646464u, sel_lo),
                                   __byte_perm(w[0], 0x64646464u, sel_hi), __byte_perm(w[1], 0x64646464u, sel_hi)};
          const uint32_t av1[4] = {__byte_perm(w[2], 0x64646464u, sel_lo), __byte_perm(w[3], 0x64646464u, sel_lo),
                                   __byte_perm(w[2], 0x64646464u, sel_hi), __byte_perm(w[3], 0x64646464u, sel_hi)};
          const uint32_t a1s = rq == blk ? ones : 0u;
          const uint32_t aones[4] = {a1s, 0u, a1s, 0u};
#pragma unroll
          for (int nt = 0; nt < NT; ++nt) {
            const uint32_t bq[2] = {hmul2_u32(pb[pp][nt][0], s_lo), hmul2_u32(pb[pp][nt][1], s_hi)};
            mma_f16_16816(o[nt][2 * blk], av0, bq);
            mma_f16_16816(o[nt][2 * blk + 1], av1, bq);
            mma_f16_16816(corr[nt], aones, bq);
          }
        }
      }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty_bar[slot]);
    if (item >= 0 && last) epilogue();
  }
}

// MT: 16-row m-tiles (1 or 2).  VT: V format (0 fp16, 1 bf16, 2 Q8_0 rows,
// 3 Q8_0 page-transposed records).
// NST: shared-memory pipeline slots.  PPW: pages per compute warp per stage.
// TRW: 0, or the compute warps (8 or 16) of the transposed consumer (MT 1 or
// 2, VT 3 only) with NT n-tiles of 8 query rows.
template <int MT, int VT, bool MASK, int NST, int PPW, int TRW = 0, int NT = 1>
__global__ void __launch_bounds__(TRW == dec::NWC_TR ? dec::NTHREADS_TR : dec::NTHREADS, 1)
    decode_kernel(const DecodeParams d) {
  constexpr bool TR = TRW != 0;
  using namespace dec;
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ __align__(8) uint64_t full_bar[NST];
  __shared__ __align__(8) uint64_t empty_bar[NST];
  __shared__ StageMeta meta[NST];

  const int warp = warp_id();
  const int lane = lane_id();
  const G9AttnBatch& p = d.p;
  constexpr int NWC = TR ? TRW : dec::NWC;   // compute warps; warp NWC produces

  if (threadIdx.x == 0) {
    for (int i = 0; i < NST; ++i) {
      mbar_init(&full_bar[i], 1);
      mbar_init(&empty_bar[i], NWC);
    }
    fence_barrier_init();
  }
  // Launched with programmatic stream serialisation: everything above may
  // overlap the previous kernel's tail; nothing it wrote is read before this
  // wait.  The dependent combine grid may be scheduled from here on (it waits
  // for this grid's completion itself).
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;");
  if constexpr (TR) {
    // rank prefix sums (balanced split): every thread loads the lengths of
    // some ranks (one parallel pass over the sequences), then warp 0 scans
    int* cpre = reinterpret_cast<int*>(smem + d.cpre_off);
    const int n = d.nranks;
    for (int r = threadIdx.x; r < n; r += blockDim.x) {
      int real, ps;
      cpre[r] = rank_units(d, r, real, ps);
    }
    __syncthreads();
    if (warp == 0) {
      const int per = (n + 31) / 32;
      const int r0 = min(n, lane * per), r1 = min(n, r0 + per);
      int sum = 0;
      for (int r = r0; r < r1; ++r) sum += cpre[r];
      int incl = sum;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int v = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += v;
      }
      int run = incl - sum;
      for (int r = r0; r < r1; ++r) {
        const int u = cpre[r];
        cpre[r] = run;
        if (blockIdx.x == 0) d.cpre_g[r] = run;
        run += u;
      }
      if (lane == 31) {
        cpre[n] = incl;
        if (blockIdx.x == 0) d.cpre_g[n] = incl;
      }
    }
  }
  __syncthreads();

  // =========================================================================
  // producer warpgroup (warp 8 issues copies, 9-11 only give up registers).
  // Each bulk copy moves the row groups of two consecutive tokens (all HG
  // heads) into a slot padded to an odd multiple of 16 bytes: half as many
  // copy requests as one per token, and with the key order below still
  // conflict-free for the tensor-core operand loads.
  // =========================================================================
  if (warp >= NWC) {
    if constexpr (TRW == NWC_TR) asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(REG_PRODUCER_TR));
    else asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(REG_PRODUCER));
    if (warp != NWC) return;
    int it = 0;
    bool alive = true;
    const int hgb_k = d.HG * d.rb_k, hgb_v = d.HG * d.rb_v;
    const uint32_t kbytes_page = (uint32_t)(PAGE * hgb_k);
    const uint32_t vbytes_page = (uint32_t)(PAGE * hgb_v);
    // copy slots per page, a power of two >= the copies a page needs, so a
    // loop iteration of the warp issues the copies of 32 / slots pages
    const int cps_log2 = d.cps_log2, kCopies = 1 << cps_log2;
    // Lane g < NG holds group g's stream: its item and the next page to copy.
    // Items are claimed dynamically, so streams that drew short chunks take
    // more; a claim skips items without work (chunks past a sequence's end).
    // Each stage's plan (and its block-table lookups, and a group's next
    // claim) is made one stage ahead, so those latencies overlap the previous
    // stage's empty-slot wait and copies.
    // balanced split (transposed kernels): lane g's stream, next unit, end
    const int* cpre = reinterpret_cast<const int*>(smem + d.cpre_off);
    int bal_u = 0, bal_hi = 0, bal_rank = 0;
    const int bal_sid0 = blockIdx.x * d.NG + lane;
    if constexpr (TR) {
      const int64_t T = cpre[d.nranks];
      const int NS = (int)(T < d.nstreams ? T : (int64_t)d.nstreams);
      if (lane < d.NG && bal_sid0 < NS) {
        bal_u = (int)bal_bound(bal_sid0, T, NS);
        bal_hi = (int)bal_bound(bal_sid0 + 1, T, NS);
        int lo = 0, hi = d.nranks;                 // last rank with cpre <= bal_u
        while (hi - lo > 1) {
          const int mid = (lo + hi) >> 1;
          if (cpre[mid] <= bal_u) lo = mid; else hi = mid;
        }
        bal_rank = lo;
      }
    }
    int g_real = 0;                                // pages of the current item that exist
    auto claim = [&](int& item_, int& b_, int& h0_, int& pb_, int& pe_, int& real_) -> bool {
      if constexpr (TR) {
        if (bal_u >= bal_hi) return false;
        while (cpre[bal_rank + 1] <= bal_u) ++bal_rank;   // ranks without units
        const int c0 = cpre[bal_rank];
        int ps;
        rank_units(d, bal_rank, real_, ps);
        item_ = bal_sid0 + bal_rank;
        b_ = bal_rank / d.HGN;
        h0_ = (bal_rank - b_ * d.HGN) * d.HG;
        pb_ = ps + bal_u - c0;
        pe_ = ps + min(bal_hi, cpre[bal_rank + 1]) - c0;
        bal_u = c0 + (pe_ - ps);
        return true;
      } else {
      for (;;) {
        const int item = (int)atomicAdd(d.counter, 1u);
        if (item >= d.n_items) return false;
        int b, z, s, pb, pe, nsplit;
        decode_item(d, item, b, z, s);
        if (!item_pages(d, b, s, pb, pe, nsplit)) continue;
        item_ = item; b_ = b; h0_ = z * d.HG; pb_ = pb; pe_ = pe; real_ = pe;
        return true;
      }
      }
    };
    const int gl = min(lane / PPW, MAXG - 1), pp = lane % PPW;   // page slot l = gl*PPW + pp
    // block-table entry of this lane's page slot under a plan held by the group lanes
    auto lookup = [&](bool act, int b_, int pg_, int pe_, int real_, bool& valid) -> int {
      const unsigned amask = __ballot_sync(0xffffffffu, act);
      const int s_b = __shfl_sync(0xffffffffu, b_, gl);
      const int s_pg = __shfl_sync(0xffffffffu, pg_, gl);
      const int s_pe = __shfl_sync(0xffffffffu, min(pe_, real_), gl);
      valid = lane < d.P && ((amask >> gl) & 1) && s_pg + pp < s_pe;
      return valid ? p.block_table[(int64_t)s_b * p.max_blocks + s_pg + pp] : -1;
    };
    if (!TR && d.NG == 1) {
      constexpr int kCopies1 = 2 * PAGE;     // copy slots per page (12 used with adjacent rows, 32 without)
    // one group (HG = 8 heads per CTA): a single item stream, block-table
    // entries read one stage ahead.  Measured 18% faster than the general
    // per-group loop below for fp16 V (page-sized stages), equal for Q8_0 V.
    while (alive) {
      int item = 0;
      if (lane == 0) item = (int)atomicAdd(d.counter, 1u);
      item = __shfl_sync(0xffffffffu, item, 0);
      if (item >= d.n_items) break;
      int b, z, s, pb, pe, nsplit;
      decode_item(d, item, b, z, s);
      if (!item_pages(d, b, s, pb, pe, nsplit)) continue;
      const int h0 = z * d.HG;
      // block-table entries are read one stage ahead, so their latency hides
      // behind the previous stage's copies and the empty-slot wait
      int phys_next = -1;
      if (lane < min(d.P, pe - pb)) phys_next = p.block_table[(int64_t)b * p.max_blocks + pb + lane];
      for (int pg = pb;; pg += d.P) {
        const int slot = it % NST;
        const int phys = phys_next;
        const int npg = max(0, min(d.P, pe - pg));
        phys_next = -1;
        if (lane < min(d.P, pe - pg - d.P)) phys_next = p.block_table[(int64_t)b * p.max_blocks + pg + d.P + lane];
        if (it >= NST && !mbar_wait(&empty_bar[slot], ((it / NST) - 1) & 1)) { alive = false; break; }
        const bool bad = page_bad(p, phys);
        const bool ok = lane < npg && !bad;
        if (lane < npg && bad) raise_error(ERR_BAD_PAGE);
        if (lane < MAXP) meta[slot].ok[lane] = ok ? 1 : 0;
        const unsigned okmask = __ballot_sync(0xffffffffu, ok);
        const bool last = pg + d.P >= pe;
        if (lane == 0) {
          meta[slot].item[0] = item; meta[slot].done = 0;
          meta[slot].page0[0] = pg;
          meta[slot].npages[0] = npg;
          meta[slot].last[0] = last ? 1 : 0;
        }
        __syncwarp();
        if (lane == 0) mbar_arrive_expect_tx(&full_bar[slot], __popc(okmask) * (kbytes_page + vbytes_page));
        __syncwarp();
        uint8_t* kdst0 = smem + slot * d.stage_bytes;
        uint8_t* vdst0 = kdst0 + d.vbase;
        // uniform trip count for the whole warp (the shuffle needs every lane)
        for (int c0 = 0; c0 < d.P * kCopies1; c0 += 32) {
          const int c = c0 + lane;
          const int j = min(c / kCopies1, MAXP - 1);
          const int r = c - j * kCopies1;
          const int phys_j = __shfl_sync(0xffffffffu, phys, j);
          if (c >= d.P * kCopies1 || j >= npg || !((okmask >> j) & 1)) continue;
          // K: 4 groups of 4 tokens, V: 8 groups of 2 tokens (slots 0-3 / 4-11
          // as whole-group copies, or 0-15 / 16-31 token by token)
          const int nkc = d.contig ? 4 : 16;
          const bool isk = r < nkc;
          const int q = isk ? r : r - nkc;
          if constexpr (VT == 3) {
            if (!isk) {
              // one copy of the adjacent records of all HG heads, or one per head
              if (q >= (d.vrec_contig ? 1 : d.HG)) continue;
              bulk_g2s(vdst0 + j * d.vpage + q * d.vrec,
                       p.v_cache + (int64_t)phys_j * p.v_page_stride + (int64_t)(h0 + q) * p.v_head_stride,
                       d.vrec_contig ? d.HG * d.vrec : d.vrec, &full_bar[slot]);
              continue;
            }
          }
          if (!isk && q >= (d.contig ? 8 : 16)) continue;
          const int hgb = isk ? hgb_k : hgb_v;
          const int gt = isk ? 4 : 2;             // tokens per group
          const uint8_t* src = (isk ? p.k_cache : p.v_cache) +
                               (int64_t)phys_j * (isk ? p.k_page_stride : p.v_page_stride) +
                               (int64_t)h0 * (isk ? p.k_head_stride : p.v_head_stride);
          const int64_t ts = isk ? p.k_tok_stride : p.v_tok_stride;
          uint8_t* base = isk ? kdst0 + j * d.kpage : vdst0 + j * d.vpage;
          const int gs = isk ? d.kgs : d.vgs;
          if (d.contig) {
            bulk_g2s(base + q * gs, src + (int64_t)(gt * q) * ts, gt * hgb, &full_bar[slot]);
          } else {                                // token rows of a group are not adjacent in HBM
            bulk_g2s(base + (q / gt) * gs + (q % gt) * hgb, src + (int64_t)q * ts, hgb, &full_bar[slot]);
          }
        }
        ++it;
        if (last) break;
      }
    }
    } else {
    int g_item = -1, g_b = 0, g_h0 = 0, g_pg = 0, g_pe = 0;
    bool g_active = false, g_exhausted = lane >= d.NG;
    if (!g_exhausted) {
      g_active = claim(g_item, g_b, g_h0, g_pg, g_pe, g_real);
      g_exhausted = !g_active;
    }
    bool pvalid;
    int phys = lookup(g_active, g_b, g_pg, g_pe, g_real, pvalid);
    while (alive) {
      const unsigned active = __ballot_sync(0xffffffffu, g_active);
      if (active == 0) break;
      // plan of the next stage: the same item's next pages, or a new claim
      int n_item = g_item, n_b = g_b, n_h0 = g_h0, n_pg = g_pg + PPW, n_pe = g_pe, n_real = g_real;
      bool n_active = g_active && n_pg < n_pe;
      if (!n_active && !g_exhausted) {
        n_active = claim(n_item, n_b, n_h0, n_pg, n_pe, n_real);
        g_exhausted = !n_active;
      }
      bool n_pvalid;
      const int n_phys = lookup(n_active, n_b, n_pg, n_pe, n_real, n_pvalid);
      const int slot = it % NST;
      if (it >= NST && !mbar_wait(&empty_bar[slot], ((it / NST) - 1) & 1)) { alive = false; break; }
      const bool bad = page_bad(p, phys);
      const bool ok = pvalid && !bad;
      if (pvalid && bad) raise_error(ERR_BAD_PAGE);
      if (lane < MAXP) meta[slot].ok[lane] = ok ? 1 : 0;
      if (lane < MAXG) {
        meta[slot].item[lane] = g_active ? g_item : -1;
        meta[slot].page0[lane] = g_pg;
        meta[slot].npages[lane] = g_active ? max(0, min(PPW, g_pe - g_pg)) : 0;
        meta[slot].last[lane] = (g_active && g_pg + PPW >= g_pe) ? 1 : 0;
      }
      if (lane == 0) meta[slot].done = 0;
      const unsigned okmask = __ballot_sync(0xffffffffu, ok);
      __syncwarp();
      if (lane == 0) mbar_arrive_expect_tx(&full_bar[slot], __popc(okmask) * (kbytes_page + vbytes_page));
      __syncwarp();
      uint8_t* kdst0 = smem + slot * d.stage_bytes;
      uint8_t* vdst0 = kdst0 + d.vbase;
      // uniform trip count for the whole warp (the shuffles need every lane)
      for (int c0 = 0; c0 < d.P * kCopies; c0 += 32) {
        const int c = c0 + lane;
        const int j = min(c >> cps_log2, MAXP - 1);
        const int r = c - j * kCopies;
        const int phys_j = __shfl_sync(0xffffffffu, phys, j);
        const int h0 = __shfl_sync(0xffffffffu, g_h0, min(j / PPW, MAXG - 1));
        if (c >= d.P * kCopies || !((okmask >> j) & 1)) continue;
        // K: 4 groups of 4 tokens, V: 8 groups of 2 tokens (slots 0-3 / 4-11
        // as whole-group copies, or 0-15 / 16-31 token by token)
        if (d.joint) {
          // the page's K rows and V records, adjacent in HBM, in one copy
          if (r == 0)
            bulk_g2s(kdst0 + j * d.kps, p.k_cache + (int64_t)phys_j * p.k_page_stride,
                     kbytes_page + vbytes_page, &full_bar[slot]);
          continue;
        }
        const int nkc = d.kwhole ? 1 : (d.contig ? 4 : 16);
        const bool isk = r < nkc;
        const int q = isk ? r : r - nkc;
        if constexpr (VT == 3) {
          if (!isk) {
            // one copy of the adjacent records of all HG heads, or one per head
            if (q >= (d.vrec_contig ? 1 : d.HG)) continue;
            bulk_g2s(vdst0 + j * d.vps + q * d.vrec,
                     p.v_cache + (int64_t)phys_j * p.v_page_stride + (int64_t)(h0 + q) * p.v_head_stride,
                     d.vrec_contig ? d.HG * d.vrec : d.vrec, &full_bar[slot]);
            continue;
          }
        }
        if (!isk && q >= (d.contig ? PAGE / d.vgt : 16)) continue;
        const int hgb = isk ? hgb_k : hgb_v;
        const int gt = isk ? (d.kwhole ? PAGE : 4) : d.vgt;   // tokens per copy
        const uint8_t* src = (isk ? p.k_cache : p.v_cache) +
                             (int64_t)phys_j * (isk ? p.k_page_stride : p.v_page_stride) +
                             (int64_t)h0 * (isk ? p.k_head_stride : p.v_head_stride);
        const int64_t ts = isk ? p.k_tok_stride : p.v_tok_stride;
        uint8_t* base = isk ? kdst0 + j * d.kps : vdst0 + j * d.vps;
        const int gs = isk ? d.kgs : d.vgs;
        if (d.contig) {
          bulk_g2s(base + q * gs, src + (int64_t)(gt * q) * ts, gt * hgb, &full_bar[slot]);
        } else {                                // token rows of a group are not adjacent in HBM
          bulk_g2s(base + (q / gt) * gs + (q % gt) * hgb, src + (int64_t)q * ts, hgb, &full_bar[slot]);
        }
      }
      ++it;
      g_item = n_item; g_b = n_b; g_h0 = n_h0; g_pg = n_pg; g_pe = n_pe; g_real = n_real; g_active = n_active;
      phys = n_phys;
      pvalid = n_pvalid;
    }
    }
    // terminator stage
    if (alive) {
      const int slot = it % NST;
      if (it < NST || mbar_wait(&empty_bar[slot], ((it / NST) - 1) & 1)) {
        if (lane == 0) {
          meta[slot].done = 1;
          mbar_arrive(&full_bar[slot]);
        }
      }
    }
    return;
  }

  // =========================================================================
  // compute warps
  // =========================================================================
  if constexpr (TR) {
    static_assert(VT != 2, "transposed consumer: 16-bit V rows or page-transposed Q8_0 V");
    decode_consumer_tr<VT, MASK, NST, PPW, NWC, NT>(d, smem, full_bar, empty_bar, meta, warp, lane);
  } else {
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(REG_COMPUTE));
  const int hl = warp % d.HG;       // local kv head
  const int sub = warp / d.HG;      // page-slot group: its own stream of items
  const int j4 = lane & 3;          // quad lane
  const int rq = lane >> 2;         // row within an 8-row group

  constexpr bool QS = MT == 2;      // Q tile in shared memory instead of registers
  uint32_t qa[QS ? 1 : MT][8][4];   // Q fragments (fp16), MT == 1 only
  float o[MT][16][4];
  float mrow[MT][2], lrow[MT][2];
  int cur_item = -1, cb = 0, cz = 0, cs = 0, cnq = 0, cR = 0, ckv = 0, cqabs = 0, cnsplit = 1;

  auto reset_state = [&]() {
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) {
#pragma unroll
      for (int nt = 0; nt < 16; ++nt)
#pragma unroll
        for (int c = 0; c < 4; ++c) o[mt][nt][c] = 0.f;
      mrow[mt][0] = mrow[mt][1] = -INFINITY;
      lrow[mt][0] = lrow[mt][1] = 0.f;
    }
  };

  const uint32_t smem_base = smem_u32(smem);
  // shared-memory loads as plain C++ loads through the __shared__ array (the
  // compiler folds constant offsets and schedules them; the "memory" clobber
  // of the mbarrier waits keeps them after the data has landed)
  auto ld16 = [&](uint32_t a) { return *reinterpret_cast<const uint16_t*>(smem + (a - smem_base)); };
  auto ld8 = [&](uint32_t a) { return (uint32_t)*reinterpret_cast<const uint8_t*>(smem + (a - smem_base)); };
  auto ld64 = [&](uint32_t a) { return *reinterpret_cast<const uint2*>(smem + (a - smem_base)); };
  const uint32_t qs_base = smem_base + d.q_off + warp * (MT * 16 * QROW);   // this warp's Q tile

  auto load_q = [&](int b, int h) {
    if constexpr (QS) {
      // each warp owns its tile (the groups switch items independently)
      __syncwarp();
      {
        for (int i = lane; i < MT * 16 * 64; i += 32) {   // 64 element pairs per row
          const int r = i >> 6, c = (i & 63) * 2;
          float x0 = 0.f, x1 = 0.f;
          if (r < cR) {
            const int t = r / d.G;
            const int64_t base = q_offset(p, b, t, h * d.G + (r - t * d.G));
            x0 = load_one(p.q, base + c, p.q_dtype);
            x1 = load_one(p.q, base + c + 1, p.q_dtype);
          }
          const uint32_t v = pack_half2(x0, x1);
          asm volatile("st.shared.u32 [%0], %1;" ::"r"(qs_base + r * QROW + c * 2), "r"(v));
        }
      }
      __syncwarp();
    } else {
      // all loads of both rows are issued before any conversion, so the
      // item switch costs one memory latency instead of one per element
      const int rA = rq, rB = rq + 8;
      const bool vA = rA < cR, vB = rB < cR;
      const int tA = vA ? rA / d.G : 0, tB = vB ? rB / d.G : 0;
      const int64_t baseA = vA ? q_offset(p, b, tA, h * d.G + (rA - tA * d.G)) : 0;
      const int64_t baseB = vB ? q_offset(p, b, tB, h * d.G + (rB - tB * d.G)) : 0;
      if (p.q_dtype == DT_F32) {
        float2 xa[16], xb[16];
        const float* qf = reinterpret_cast<const float*>(p.q);
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const int dd = (i >> 1) * 16 + (i & 1) * 8 + 2 * j4;
          xa[i] = vA ? *reinterpret_cast<const float2*>(qf + baseA + dd) : make_float2(0.f, 0.f);
          xb[i] = vB ? *reinterpret_cast<const float2*>(qf + baseB + dd) : make_float2(0.f, 0.f);
        }
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          // a0: (row, k lo)  a1: (row+8, k lo)  a2: (row, k hi)  a3: (row+8, k hi)
          qa[0][i >> 1][(i & 1) * 2 + 0] = pack_half2(xa[i].x, xa[i].y);
          qa[0][i >> 1][(i & 1) * 2 + 1] = pack_half2(xb[i].x, xb[i].y);
        }
      } else {
        uint32_t xa[16], xb[16];
        const uint16_t* qh = reinterpret_cast<const uint16_t*>(p.q);
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const int dd = (i >> 1) * 16 + (i & 1) * 8 + 2 * j4;
          xa[i] = vA ? *reinterpret_cast<const uint32_t*>(qh + baseA + dd) : 0u;
          xb[i] = vB ? *reinterpret_cast<const uint32_t*>(qh + baseB + dd) : 0u;
        }
        const bool bf = p.q_dtype == DT_BF16;
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          uint32_t a = xa[i], c = xb[i];
          if (bf) {
            a = pack_half2(__uint_as_float(a << 16), __uint_as_float(a & 0xffff0000u));
            c = pack_half2(__uint_as_float(c << 16), __uint_as_float(c & 0xffff0000u));
          }
          qa[0][i >> 1][(i & 1) * 2 + 0] = a;
          qa[0][i >> 1][(i & 1) * 2 + 1] = c;
        }
      }
    }
  };

  // A fragment of Q for (m-tile mt, k-step ks)
  auto q_frag = [&](int mt, int ks, uint32_t a[4]) {
    if constexpr (QS) {
      // matrices: (rows 0-7 | 8-15) x (k 0-7 | 8-15) -> a0..a3
      const int mi = lane >> 3, ri = lane & 7;
      const uint32_t addr = qs_base + (mt * 16 + (mi & 1) * 8 + ri) * QROW + ks * 32 + (mi >> 1) * 16;
      asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                   : "=r"(a[0]), "=r"(a[1]), "=r"(a[2]), "=r"(a[3])
                   : "r"(addr));
    } else {
#pragma unroll
      for (int i = 0; i < 4; ++i) a[i] = qa[0][ks][i];
    }
  };


  auto epilogue = [&]() {
    // quad-reduce the running sums
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        float v = lrow[mt][hh];
        v += __shfl_xor_sync(0xffffffffu, v, 1);
        v += __shfl_xor_sync(0xffffffffu, v, 2);
        lrow[mt][hh] = v;
      }
    const int h = cz * d.HG + hl;
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) {
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        const int r = mt * 16 + rq + hh * 8;
        if (r >= cR) continue;
        const float l = lrow[mt][hh];
        float inv = l > 0.f ? 1.f / l : 0.f;
        if (cnsplit == 1) {
          const int t = r / d.G;
          const int hq = h * d.G + (r - t * d.G);
          if (p.sinks && l > 0.f) inv = 1.f / (l + fast_exp2(sink_log2(p, hq) - mrow[mt][hh]));
          inv *= out_quant_factor(p);
          const int64_t ob = o_offset(p, cb, t, hq);
#pragma unroll
          for (int nt = 0; nt < 16; ++nt)
            store_out2(p.out, p.out_dtype, ob + nt * 8 + 2 * j4, o[mt][nt][hh * 2] * inv,
                       o[mt][nt][hh * 2 + 1] * inv);
        } else {
          const int64_t row = (((int64_t)cb * p.num_heads_kv + h) * d.S_max + cs) * d.R_pad + r;
          float* op = d.opart + row * D;
#pragma unroll
          for (int nt = 0; nt < 16; ++nt)
            *reinterpret_cast<float2*>(op + nt * 8 + 2 * j4) =
                make_float2(o[mt][nt][hh * 2] * inv, o[mt][nt][hh * 2 + 1] * inv);
          if (j4 == 0) d.ml[row] = make_float2(mrow[mt][hh], l);
        }
      }
    }
  };

  for (int it = 0;; ++it) {
    const int slot = it % NST;
    if (!mbar_wait(&full_bar[slot], (it / NST) & 1)) break;
    if (meta[slot].done) break;
    const int item = meta[slot].item[sub];        // -1: this warp's group has no work in the stage
    const int page0 = meta[slot].page0[sub];
    const int npages = meta[slot].npages[sub];
    const bool last = meta[slot].last[sub] != 0;
    if (item >= 0 && item != cur_item) {
      cur_item = item;
      decode_item(d, item, cb, cz, cs);
      cnq = seq_nq(p, cb);
      cR = cnq * d.G;
      ckv = seq_len_kv(p, cb);
      cqabs = seq_qabs(p, cb, cnq, ckv);
      int pb, pe;
      item_pages(d, cb, cs, pb, pe, cnsplit);
      reset_state();
      load_q(cb, cz * d.HG + hl);
    }
    // This warp's page slots sub*PPW .. +PPW-1 of the stage.  The pages are
    // processed together, branch-free, so their loads, conversions and MMAs
    // interleave.  A slot without a valid page reads the data of a valid one
    // (finite values) and has all its scores masked to -inf.
    bool pok[PPW];
    int first_ok = -1;
#pragma unroll
    for (int pp = PPW - 1; pp >= 0; --pp) {
      const int s = sub * PPW + pp;
      pok[pp] = item >= 0 && pp < npages && meta[slot].ok[s];
      if (pok[pp]) first_ok = pp;
    }
    if (first_ok >= 0) {
      int psrc[PPW];
#pragma unroll
      for (int pp = 0; pp < PPW; ++pp) psrc[pp] = sub * PPW + (pok[pp] ? pp : first_ok);
      // Key order: accumulator column n of n-tile nt (k-slot nt*8 + n of the
      // P.V product) is physical key 4*(n/2) + e, e = {0,3} for nt = 0 and
      // {1,2} for nt = 1 (by n & 1).  An n-tile then takes one key of each
      // V pair group and, per 4-token K group, two keys whose rows sit in
      // different bank halves -- the 8 rows it reads are conflict-free for
      // both the K fragments and the ldmatrix V fragments.
      const int hgb_k = d.HG * d.rb_k, hgb_v = d.HG * d.rb_v;
      auto kaddr = [&](int key) { return (uint32_t)((key >> 2) * d.kgs + (key & 3) * hgb_k); };
      auto vaddr = [&](int key) { return (uint32_t)((key >> 1) * d.vgs + (key & 1) * hgb_v); };
      auto slot_key = [](int nt, int n) { return 4 * (n >> 1) + (nt == 0 ? 3 * (n & 1) : 1 + (n & 1)); };
      const uint32_t stage_base = smem_base + slot * d.stage_bytes;
      // ---------------- S = Q K^T --------------------------------------------
      float sacc[PPW][MT][2][4];
#pragma unroll
      for (int pp = 0; pp < PPW; ++pp)
#pragma unroll
        for (int mt = 0; mt < MT; ++mt)
#pragma unroll
          for (int nt = 0; nt < 2; ++nt)
#pragma unroll
            for (int c = 0; c < 4; ++c) sacc[pp][mt][nt][c] = 0.f;
#pragma unroll
      for (int pp = 0; pp < PPW; ++pp) {
      const uint32_t kb = stage_base + psrc[pp] * d.kps + hl * d.rb_k;
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
        const uint32_t krow = kb + kaddr(slot_key(nt, rq));              // B operand row (key)
        const uint32_t kcol0 = kb + kaddr(slot_key(nt, 2 * j4));         // accumulator column keys
        const uint32_t kcol1 = kb + kaddr(slot_key(nt, 2 * j4 + 1));
#pragma unroll
        for (int blk = 0; blk < 4; ++blk) {
          const uint32_t qb = krow + blk * QBLOCK + 2 + 2 * j4;
          uint32_t b0[2], b1[2];
          b0[0] = i8x2_to_h2(ld16(qb));
          b0[1] = i8x2_to_h2(ld16(qb + 8));
          b1[0] = i8x2_to_h2(ld16(qb + 16));
          b1[1] = i8x2_to_h2(ld16(qb + 24));
          const float dk0 = half_bits_to_float(ld16(kcol0 + blk * QBLOCK));
          const float dk1 = half_bits_to_float(ld16(kcol1 + blk * QBLOCK));
#pragma unroll
          for (int mt = 0; mt < MT; ++mt) {
            float acc[4] = {0.f, 0.f, 0.f, 0.f};
            uint32_t a0[4], a1[4];
            q_frag(mt, 2 * blk, a0);
            q_frag(mt, 2 * blk + 1, a1);
            mma_f16_16816(acc, a0, b0);
            mma_f16_16816(acc, a1, b1);
            sacc[pp][mt][nt][0] = fmaf(acc[0], dk0, sacc[pp][mt][nt][0]);
            sacc[pp][mt][nt][1] = fmaf(acc[1], dk1, sacc[pp][mt][nt][1]);
            sacc[pp][mt][nt][2] = fmaf(acc[2], dk0, sacc[pp][mt][nt][2]);
            sacc[pp][mt][nt][3] = fmaf(acc[3], dk1, sacc[pp][mt][nt][3]);
          }
        }
      }
      }
      // ---------------- mask + online softmax (base 2) ------------------------
      // Lazy running max: a row keeps its reference max m until one of its
      // scores exceeds m by more than 2^8; only then (rare after the first
      // pages) is the row max reduced over the quad and O / l rescaled.  So
      // P <= 2^8, and the usual page needs no shuffles and no rescale.
      uint32_t pa[PPW][MT][4];
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) {
        float tmx[2] = {-INFINITY, -INFINITY};
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          const int r = mt * 16 + rq + hh * 8;
          const int t = r / d.G;
          int kv_lim = ckv;                                      // exclusive
          if (has_causal(p)) kv_lim = min(kv_lim, cqabs + t + 1);
          if (r >= cR) kv_lim = -1;
          const int kv_lo = MASK ? window_lo(p, seq_qpos0(p, cb, cnq, ckv), t) : 0;
#pragma unroll
          for (int pp = 0; pp < PPW; ++pp) {
            const int k0 = (page0 + pp) * PAGE;
            // pages every row sees completely need no per-element mask
            const bool page_full = !MASK && pok[pp] && k0 + PAGE <= ckv && (!has_causal(p) || k0 + PAGE <= cqabs + 1);
#pragma unroll
            for (int nt = 0; nt < 2; ++nt)
#pragma unroll
              for (int c = 0; c < 2; ++c) {
                float x = sacc[pp][mt][nt][hh * 2 + c] * d.scale_log2;
                if (!page_full) {
                  const int k = k0 + 4 * j4 + (nt == 0 ? 3 * c : 1 + c);   // physical key of column 2*j4 + c
                  bool vis = pok[pp] && k < kv_lim;
                  if constexpr (MASK) {
                    // general scores: soft-cap, additive mask, sliding window
                    if (p.softcap > 0.f) x = softcap_log2(sacc[pp][mt][nt][hh * 2 + c], d.cap_in, d.cap_out);
                    if (p.mask && vis)
                      x += kLog2e * __half2float(reinterpret_cast<const __half*>(p.mask)[
                          (int64_t)cb * p.mask_seq_stride + (int64_t)t * p.mask_tok_stride + k]);
                    vis = vis && k >= kv_lo;
                  }
                  x = vis ? x : -INFINITY;
                }
                sacc[pp][mt][nt][hh * 2 + c] = x;
                tmx[hh] = fmaxf(tmx[hh], x);
              }
          }
        }
        const bool grow = tmx[0] > mrow[mt][0] + kRescaleLog2 || tmx[1] > mrow[mt][1] + kRescaleLog2;
        if (__any_sync(0xffffffffu, grow)) {
          float alpha2[2];
#pragma unroll
          for (int hh = 0; hh < 2; ++hh) {
            float mx = tmx[hh];
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
            alpha2[hh] = 1.f;
            if (mx > mrow[mt][hh] + kRescaleLog2) {              // uniform over the quad
              alpha2[hh] = fast_exp2(mrow[mt][hh] - mx);          // 0 for the first visible key
              mrow[mt][hh] = mx;
              lrow[mt][hh] *= alpha2[hh];
            }
          }
#pragma unroll
          for (int nt = 0; nt < 16; ++nt) {
            o[mt][nt][0] *= alpha2[0];
            o[mt][nt][1] *= alpha2[0];
            o[mt][nt][2] *= alpha2[1];
            o[mt][nt][3] *= alpha2[1];
          }
        }
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          const float mu = mrow[mt][hh] == -INFINITY ? 0.f : mrow[mt][hh];
          float ls = 0.f;
#pragma unroll
          for (int pp = 0; pp < PPW; ++pp)
#pragma unroll
            for (int nt = 0; nt < 2; ++nt)
#pragma unroll
              for (int c = 0; c < 2; ++c) {
                const float pv = fast_exp2(sacc[pp][mt][nt][hh * 2 + c] - mu);
                sacc[pp][mt][nt][hh * 2 + c] = pv;
                ls += pv;
              }
          lrow[mt][hh] += ls;
        }
#pragma unroll
        for (int pp = 0; pp < PPW; ++pp) {
          if constexpr (VT == 1) {
            pa[pp][mt][0] = pack_bf162(sacc[pp][mt][0][0], sacc[pp][mt][0][1]);
            pa[pp][mt][1] = pack_bf162(sacc[pp][mt][0][2], sacc[pp][mt][0][3]);
            pa[pp][mt][2] = pack_bf162(sacc[pp][mt][1][0], sacc[pp][mt][1][1]);
            pa[pp][mt][3] = pack_bf162(sacc[pp][mt][1][2], sacc[pp][mt][1][3]);
          } else {
            pa[pp][mt][0] = pack_half2(sacc[pp][mt][0][0], sacc[pp][mt][0][1]);
            pa[pp][mt][1] = pack_half2(sacc[pp][mt][0][2], sacc[pp][mt][0][3]);
            pa[pp][mt][2] = pack_half2(sacc[pp][mt][1][0], sacc[pp][mt][1][1]);
            pa[pp][mt][3] = pack_half2(sacc[pp][mt][1][2], sacc[pp][mt][1][3]);
          }
        }
      }
      // ---------------- O += P V ------------------------------------------------
#pragma unroll
      for (int pp = 0; pp < PPW; ++pp) {
      const uint32_t vb = stage_base + d.vbase + psrc[pp] * d.vps + hl * d.rb_v;
      if constexpr (VT < 2) {
        // ldmatrix.trans: thread i addresses matrix i/8 row i%8; matrices
        // (keys 0-7 | 8-15) x (d block nt | nt+1)
        const int mi = lane >> 3, ri = lane & 7;
        const uint32_t vrow = vb + vaddr(slot_key(mi & 1, ri)) + (mi >> 1) * 16;
#pragma unroll
        for (int ntp = 0; ntp < 8; ++ntp) {
          uint32_t r4[4];
          ldmatrix_x4_trans(r4, vrow + ntp * 32);
          const uint32_t bA[2] = {r4[0], r4[1]};
          const uint32_t bB[2] = {r4[2], r4[3]};
#pragma unroll
          for (int mt = 0; mt < MT; ++mt) {
            if constexpr (VT == 1) {
              mma_bf16_16816(o[mt][2 * ntp], pa[pp][mt], bA);
              mma_bf16_16816(o[mt][2 * ntp + 1], pa[pp][mt], bB);
            } else {
              mma_f16_16816(o[mt][2 * ntp], pa[pp][mt], bA);
              mma_f16_16816(o[mt][2 * ntp + 1], pa[pp][mt], bB);
            }
          }
        }
      } else if constexpr (VT == 3) {
        // Page-transposed Q8_0 V: dim rows of 16 keys.  ldmatrix hands each
        // thread the 4 bytes of keys 4*j4 .. 4*j4+3 of dim nt*8 + rq; the
        // B fragment wants k-slots (2*j4, 2*j4+1) = keys (4*j4, 4*j4+3) and
        // (2*j4+8, 2*j4+9) = keys (4*j4+1, 4*j4+2) (the key order above), so
        // a byte permute builds each pair.  int8 -> fp16 is exact
        // ((0x6400 | (b ^ 0x80)) - 1152); the scale is applied in fp16.
        const uint32_t vrec = stage_base + d.vbase + psrc[pp] * d.vps + hl * d.vrec;
        const __half2 bias = __halves2half2(__ushort_as_half(0x6480), __ushort_as_half(0x6480));  // 1152
#pragma unroll
        for (int blk = 0; blk < 4; ++blk) {
          uint32_t r4[4];
          ldmatrix_x4(r4, vrec + 2 * 4 * PAGE + (blk * 32 + lane) * PAGE);
          const uint2 sc = ld64(vrec + blk * 2 * PAGE + 8 * j4);
          const uint32_t s03u = __byte_perm(sc.x, sc.y, 0x7610);
          const uint32_t s12u = __byte_perm(sc.x, sc.y, 0x5432);
          const __half2 s03 = *reinterpret_cast<const __half2*>(&s03u);
          const __half2 s12 = *reinterpret_cast<const __half2*>(&s12u);
#pragma unroll
          for (int m = 0; m < 4; ++m) {
            const uint32_t w = r4[m] ^ 0x80808080u;
            uint32_t t0 = __byte_perm(w, 0x64646464u, 0x4340);
            uint32_t t1 = __byte_perm(w, 0x64646464u, 0x4241);
            const __half2 x0 = __hmul2(__hsub2(*reinterpret_cast<__half2*>(&t0), bias), s03);
            const __half2 x1 = __hmul2(__hsub2(*reinterpret_cast<__half2*>(&t1), bias), s12);
            const uint32_t bq[2] = {*reinterpret_cast<const uint32_t*>(&x0), *reinterpret_cast<const uint32_t*>(&x1)};
#pragma unroll
            for (int mt = 0; mt < MT; ++mt) mma_f16_16816(o[mt][blk * 4 + m], pa[pp][mt], bq);
          }
        }
      } else {
        // V rows are Q8_0: B fragment element (key k, dim n) = q8[k][n] * d[k][n/32]
        // k-slots 2j, 2j+1, 2j+8, 2j+9
        const uint32_t r0 = vb + vaddr(slot_key(0, 2 * j4));
        const uint32_t r1 = vb + vaddr(slot_key(0, 2 * j4 + 1));
        const uint32_t r8 = vb + vaddr(slot_key(1, 2 * j4));
        const uint32_t r9 = vb + vaddr(slot_key(1, 2 * j4 + 1));
#pragma unroll
        for (int blk = 0; blk < 4; ++blk) {
          const uint32_t so = blk * QBLOCK;
          const __half2 s01 = __halves2half2(__ushort_as_half(ld16(r0 + so)), __ushort_as_half(ld16(r1 + so)));
          const __half2 s89 = __halves2half2(__ushort_as_half(ld16(r8 + so)), __ushort_as_half(ld16(r9 + so)));
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const int nt = blk * 4 + q;
            const uint32_t off = so + 2 + q * 8 + rq;          // dim n = nt*8 + rq
            const uint32_t v0 = ld8(r0 + off), v1 = ld8(r1 + off), v8 = ld8(r8 + off), v9 = ld8(r9 + off);
            uint32_t h01 = i8x2_to_h2(v0 | (v1 << 8));
            uint32_t h89 = i8x2_to_h2(v8 | (v9 << 8));
            __half2 x01 = __hmul2(*reinterpret_cast<__half2*>(&h01), s01);
            __half2 x89 = __hmul2(*reinterpret_cast<__half2*>(&h89), s89);
            const uint32_t bq[2] = {*reinterpret_cast<uint32_t*>(&x01), *reinterpret_cast<uint32_t*>(&x89)};
#pragma unroll
            for (int mt = 0; mt < MT; ++mt) mma_f16_16816(o[mt][nt], pa[pp][mt], bq);
          }
        }
      }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty_bar[slot]);
    if (item >= 0 && last) epilogue();
  }
  }
}

// ---------------------------------------------------------------------------
// combine: merge the partial results (per chunk and per warp of a head) of
// sequences with more than one
// ---------------------------------------------------------------------------
// One CTA per (kv head, sequence); each query row (R <= 32) gets W = 32 / R
// warps (at most 4), which split the row's partials.  A warp reduces its
// partials' maxima, then, 32 partials at a time, lane j computes the weight
// l_s * 2^(m_s - M) of partial base + j and every lane accumulates 4 of the
// 128 output dims (weights broadcast by shuffle, 16-byte loads).  The W
// warps of a row then combine their maxima, sums and numerators through
// shared memory.
constexpr int kCombineMaxParts = 1024;
constexpr int kCombineMaxW = 4;
static __global__ void __launch_bounds__(1024) decode_combine_kernel(const DecodeParams d) {
  __shared__ float cm[32];                    // per warp (rows x W <= 32): max
  __shared__ float cl[32];                    // den (relative to that max)
  __shared__ float4 cn[32][32];               // numerators, 4 dims per lane
  const G9AttnBatch& p = d.p;
  const int b = blockIdx.y;
  const int h = blockIdx.x;
  // launched as a programmatic dependent of the decode kernel: wait for its
  // partial results to be complete and visible
  asm volatile("griddepcontrol.wait;" ::: "memory");
  // the sequence's query count and (balanced split) its rank's unit range
  // are independent loads: issue them together
  const int rank = b * d.HGN + h / d.HG;
  int64_t T = 0;
  int u0 = 0, u1 = 0;
  if (d.tr) {
    T = d.cpre_g[d.nranks];
    u0 = d.cpre_g[rank];
    u1 = d.cpre_g[rank + 1];
  }
  const int nq = seq_nq(p, b);
  if (nq <= 0 || nq * d.G > d.max_rows) return;
  int nsplit, first;            // partials of this (sequence, head): first slot, count
  int64_t pstride;              // rows between consecutive partials
  if (d.tr) {
    // balanced split: the streams holding units of this rank
    const int NS = (int)(T < d.nstreams ? T : (int64_t)d.nstreams);
    if (u1 <= u0) return;
    const int f = bal_sid(u0, T, NS), l = bal_sid(u1 - 1, T, NS);
    nsplit = l - f + 1;
    first = (f + rank) * d.HG + h % d.HG;
    pstride = (int64_t)d.HG * d.R_pad;
  } else {
    nsplit = seq_nsplit(d, b, nq);                    // partials (chunks) of this sequence
    first = (b * p.num_heads_kv + h) * d.S_max;
    pstride = d.R_pad;
  }
  if (nsplit <= 1) return;
  const int R = nq * d.G;
  // rows per CTA: all of them, or one per CTA (gridDim.z = rows) when there
  // are few (kv head, sequence) pairs and each row has many partials
  const int rpc = gridDim.z > 1 ? 1 : d.max_rows;
  const int W = blockDim.x / (32 * rpc);                // warps per row (uniform)
  const int warp = threadIdx.x >> 5;
  const int r = blockIdx.z * rpc + warp / W, wi = warp - (warp / W) * W;
  const int lane = threadIdx.x & 31;
  const bool active = r < R;
  // partial range of this warp: [s0, s1)
  const int per = (nsplit + W - 1) / W;
  const int s0 = min(nsplit, wi * per), s1 = min(nsplit, s0 + per);
  const int64_t row0 = (int64_t)first * d.R_pad + (active ? r : 0);
  const float* op = d.opart + row0 * dec::D + 4 * lane;
  float M = -INFINITY;
  float den = 0.f;
  float4 num = make_float4(0.f, 0.f, 0.f, 0.f);
  constexpr int kFew = 8;
  if (s1 - s0 <= kFew) {
    // the usual case: this warp's partials' (max, sum) and output rows are
    // loaded together, one memory round trip
    float2 ml = make_float2(-INFINITY, 0.f);
    if (active && s0 + lane < s1) ml = d.ml[row0 + (int64_t)(s0 + lane) * pstride];
    float4 v[kFew];
#pragma unroll
    for (int j = 0; j < kFew; ++j)
      v[j] = (active && s0 + j < s1) ? *reinterpret_cast<const float4*>(op + (int64_t)(s0 + j) * pstride * dec::D)
                                     : make_float4(0.f, 0.f, 0.f, 0.f);
    M = ml.x;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
    const float mu = M == -INFINITY ? 0.f : M;
    const float w = ml.x == -INFINITY ? 0.f : ml.y * fast_exp2(ml.x - mu);
    den = w;
#pragma unroll
    for (int j = 0; j < kFew; ++j) {
      const float wj = __shfl_sync(0xffffffffu, w, j);
      num.x = fmaf(wj, v[j].x, num.x); num.y = fmaf(wj, v[j].y, num.y);
      num.z = fmaf(wj, v[j].z, num.z); num.w = fmaf(wj, v[j].w, num.w);
    }
  } else {
  if (active)
    for (int s = s0 + lane; s < s1; s += 32) M = fmaxf(M, d.ml[row0 + (int64_t)s * pstride].x);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
  const float mu = M == -INFINITY ? 0.f : M;
  for (int base = s0; active && base < s1; base += 32) {
    float w = 0.f;
    if (base + lane < s1) {
      const float2 ml = d.ml[row0 + (int64_t)(base + lane) * pstride];
      w = ml.y * fast_exp2(ml.x - mu);
    }
    den += w;
    const int n = min(32, s1 - base);              // warp-uniform
#pragma unroll 4
    for (int j = 0; j < n; ++j) {
      const float wj = __shfl_sync(0xffffffffu, w, j);
      const float4 v = *reinterpret_cast<const float4*>(op + (int64_t)(base + j) * pstride * dec::D);
      num.x = fmaf(wj, v.x, num.x); num.y = fmaf(wj, v.y, num.y);
      num.z = fmaf(wj, v.z, num.z); num.w = fmaf(wj, v.w, num.w);
    }
  }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) den += __shfl_xor_sync(0xffffffffu, den, o);
  if (active) {
    if (lane == 0) { cm[warp] = M; cl[warp] = den; }
    cn[warp][lane] = num;
  }
  __syncthreads();
  if (!active || wi != 0) return;
  float Mt = -INFINITY;
  for (int k = 0; k < W; ++k) Mt = fmaxf(Mt, cm[warp + k]);
  const float mt = Mt == -INFINITY ? 0.f : Mt;
  float dsum = 0.f;
  float4 nsum = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int k = 0; k < W; ++k) {
    const float mk = cm[warp + k];
    const float a = mk == -INFINITY ? 0.f : fast_exp2(mk - mt);
    dsum += a * cl[warp + k];
    const float4 v = cn[warp + k][lane];
    nsum.x = fmaf(a, v.x, nsum.x); nsum.y = fmaf(a, v.y, nsum.y);
    nsum.z = fmaf(a, v.z, nsum.z); nsum.w = fmaf(a, v.w, nsum.w);
  }
  const int t = r / d.G;
  const int hq = h * d.G + (r - t * d.G);
  if (p.sinks && dsum > 0.f) dsum += fast_exp2(sink_log2(p, hq) - mt);
  const float inv = (dsum > 0.f ? 1.f / dsum : 0.f) * out_quant_factor(p);
  const int64_t off = o_offset(p, b, t, hq) + 4 * lane;
  store_out2(p.out, p.out_dtype, off, nsum.x * inv, nsum.y * inv);
  store_out2(p.out, p.out_dtype, off + 2, nsum.z * inv, nsum.w * inv);
}

// ---------------------------------------------------------------------------

// ---------------------------------------------------------------------------
// launcher (host side), instantiated in the attn_decode_v*.cu files
// ---------------------------------------------------------------------------
// Launch with programmatic stream serialisation: the kernel may start while
// the previous kernel in the stream finishes; it runs griddepcontrol.wait
// before touching anything that kernel wrote.
template <typename... Args>
static cudaError_t launch_pdl(void (*kern)(Args...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                              const DecodeParams& d) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, d);
}

static inline int num_sms() {
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  return sms;
}

template <int MT, int VT, bool MASK>
cudaError_t launch_decode_t(const DecodeParams& d, cudaStream_t stream) {
  // one Q tile per compute warp (MT == 2)
  const size_t smem = (size_t)d.q_off + (MT == 2 && !d.tr ? (size_t)dec::NWC * MT * 16 * dec::QROW : 0) +
                      (d.tr ? (size_t)((((d.nranks + 1) * 4 + 15) & ~15) + (d.nt >= 3 ? dec::NWC * (24 * dec::QROW + 512) : 0))
                            : 0);
  auto kern = d.nst == 4 ? decode_kernel<MT, VT, MASK, 4, 1> : decode_kernel<MT, VT, MASK, 3, 1>;
  if constexpr (MT == 1) {
    if (d.ppw == 2) kern = decode_kernel<MT, VT, MASK, 3, 2>;
    if constexpr (VT == 3) {
      if (d.tr == dec::NWC_TR) {
        kern = d.nst == 4 ? decode_kernel<1, 3, MASK, 4, 1, dec::NWC_TR> : decode_kernel<1, 3, MASK, 3, 1, dec::NWC_TR>;
      } else if (d.tr && d.nt == 1) {
        kern = d.nst == 4 ? decode_kernel<1, 3, MASK, 4, 1, dec::NWC> : decode_kernel<1, 3, MASK, 3, 1, dec::NWC>;
        if (d.ppw == 2) kern = decode_kernel<1, 3, MASK, 3, 2, dec::NWC>;
      } else if (d.tr) {
        kern = d.nst == 4 ? decode_kernel<1, 3, MASK, 4, 1, dec::NWC, 2> : decode_kernel<1, 3, MASK, 3, 1, dec::NWC, 2>;
        if (d.ppw == 2) kern = decode_kernel<1, 3, MASK, 3, 2, dec::NWC, 2>;
      }
    }
  } else if constexpr (VT != 2) {
    if (d.tr) {
      if (d.nt == 3 && d.ppw == 2)
        kern = decode_kernel<2, VT, MASK, 2, 2, dec::NWC, 3>;
      else if (d.nt == 3)
        kern = d.nst == 4 ? decode_kernel<2, VT, MASK, 4, 1, dec::NWC, 3> : decode_kernel<2, VT, MASK, 3, 1, dec::NWC, 3>;
      else
        kern = d.nst == 4 ? decode_kernel<2, VT, MASK, 4, 1, dec::NWC, 2> : decode_kernel<2, VT, MASK, 3, 1, dec::NWC, 2>;
    }
  }
  if constexpr (MT == 1 && VT <= 1) {
    if (d.tr) {
      if (d.nt == 1 && d.ppw == 2)
        kern = d.nst == 3 ? decode_kernel<1, VT, MASK, 3, 2, dec::NWC, 1> : decode_kernel<1, VT, MASK, 2, 2, dec::NWC, 1>;
      else if (d.nt == 1)
        kern = d.nst == 4 ? decode_kernel<1, VT, MASK, 4, 1, dec::NWC, 1> : decode_kernel<1, VT, MASK, 3, 1, dec::NWC, 1>;
      else
        kern = d.nst == 4 ? decode_kernel<1, VT, MASK, 4, 1, dec::NWC, 2> : decode_kernel<1, VT, MASK, 3, 1, dec::NWC, 2>;
    }
  }
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  const int grid = d.tr ? d.nstreams / d.NG : std::max(1, std::min(d.n_items, num_sms()));
  e = launch_pdl(kern, dim3(grid), dim3(d.tr == dec::NWC_TR ? dec::NTHREADS_TR : dec::NTHREADS), smem, stream, d);
  if (e != cudaSuccess) return e;
  if (d.tr || d.S_max > 1) {   // balanced split: any rank may span streams
    // same shared-memory carve-out as the decode kernel, so the SMs need no
    // L1 / shared reconfiguration between the two launches
    static const cudaError_t carve = cudaFuncSetAttribute(
        decode_combine_kernel, cudaFuncAttributePreferredSharedMemoryCarveout, (int)cudaSharedmemCarveoutMaxShared);
    (void)carve;
    if ((int64_t)d.p.num_heads_kv * d.p.num_seqs < 2 * num_sms()) {
      // few (head, sequence) pairs: one CTA per query row, 8 warps each
      // warps per row: about four partials each (the balanced split gives a
      // rank about nstreams / nranks + 1 of them), 2 .. 32, so that the grid
      // stays about one wave of CTAs
      const int est = d.tr ? d.nstreams / std::max(1, d.nranks) + 2 : d.S_max;
      int rw = 2;
      while (rw < 32 && 4 * rw < est) rw *= 2;
      e = launch_pdl(decode_combine_kernel, dim3(d.p.num_heads_kv, d.p.num_seqs, d.max_rows), dim3(32 * rw),
                     0, stream, d);
    } else {
      // warps per row: enough that each takes at most 8 partials (one round
      // trip of loads), no more, so that the grid stays one wave of CTAs
      const int est = d.tr ? d.nstreams / std::max(1, d.nranks) + 2 : d.S_max;
      const int cw = std::max(1, std::min({kCombineMaxW, 32 / d.max_rows, (est + 7) / 8}));
      e = launch_pdl(decode_combine_kernel, dim3(d.p.num_heads_kv, d.p.num_seqs), dim3(32 * d.max_rows * cw), 0,
                     stream, d);
    }
  }
  return e;
}

}  // namespace g9
