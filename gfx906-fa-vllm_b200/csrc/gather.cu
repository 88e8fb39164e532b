// gather.cu -- block_table page gather (paged Q8 K + 16-bit V -> contiguous
// BHSD) for sm_100a.
//
// One CTA per (sequence, page).  When the cache pages are dense
// ([bs][Hkv][row] with 16-byte aligned page starts, the layout of the
// reference's k_cache_q8 / value_cache tensors) one elected thread issues two
// bulk-async copies (TMA engine) that bring the whole K page and V page of all
// kv heads into shared memory, completion tracked by one mbarrier; the CTA
// then writes each head's run of rows to its BHSD destination with coalesced
// vector stores.  Otherwise rows are read with plain vector loads.
//
// Output semantics are the reference's gather_paged_kv_q8_kernel_v2
// (extension/gfx906_fa_gather.cu:190-357):
//   * V rows at token >= seq_len are written as zeros (the whole padded
//     range up to Sk);
//   * K rows at token >= seq_len are NOT written (callers mask them by
//     KV_max);
//   * a page whose block_table entry is < 0, or that lies beyond
//     max_blocks_per_seq, counts as fully out of range.
#include "common.cuh"
#include "gfx906_fa_b200.h"

namespace g9 {

struct GatherArgs {
  const uint8_t* kc;            // K cache bytes
  const uint8_t* vc;            // V cache bytes (16-bit elements)
  const int32_t* bt;
  const int32_t* sl;
  uint8_t* ko;
  uint8_t* vo;
  int64_t kc_blk, kc_tok, kc_head;   // bytes
  int64_t vc_blk, vc_tok, vc_head;   // bytes
  int B, Hkv, Sk, D, rb, bs, max_blocks;
  int num_blocks;                // > 0: entries >= num_blocks are out of range (and flagged)
  int kw;                        // K store width (2, 4 or 8 bytes)
};

constexpr int kGatherThreads = 256;

template <int W>
__device__ __forceinline__ void copy_w(uint8_t* dst, const uint8_t* src) {
  if constexpr (W == 16) *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(src);
  else if constexpr (W == 8) *reinterpret_cast<uint2*>(dst) = *reinterpret_cast<const uint2*>(src);
  else if constexpr (W == 4) *reinterpret_cast<uint32_t*>(dst) = *reinterpret_cast<const uint32_t*>(src);
  else *reinterpret_cast<uint16_t*>(dst) = *reinterpret_cast<const uint16_t*>(src);
}

// Write the valid K rows [0, nvalid) of every head of this page.  `row_src`
// gives the source address of (token-in-page t, head h).
template <int W, typename SrcFn>
__device__ __forceinline__ void write_k_rows(const GatherArgs& a, int b, int tok0, int nvalid,
                                             SrcFn row_src) {
  const int per_row = a.rb / W;
  const int per_head = nvalid * per_row;
  const int total = a.Hkv * per_head;
  for (int i = threadIdx.x; i < total; i += blockDim.x) {
    const int h = i / per_head;
    const int r = i - h * per_head;
    const int t = r / per_row;
    const int c = r - t * per_row;
    uint8_t* dst = a.ko + (((int64_t)b * a.Hkv + h) * a.Sk + tok0 + t) * a.rb + c * W;
    copy_w<W>(dst, row_src(t, h) + c * W);
  }
}

// kFixed: 16-token pages, D = 128 (136-byte K rows, 256-byte V rows) and
// 8-byte K stores: the write loops index with compile-time divisors.
template <bool kBulk, bool kFixed = false>
__global__ void __launch_bounds__(kGatherThreads) gather_kernel(GatherArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ __align__(8) uint64_t bar;
  __shared__ int s_phys, s_len;
  const int page = blockIdx.x;
  const int b = blockIdx.y;
  const int tok0 = page * a.bs;
  if (tok0 >= a.Sk) return;
  if (threadIdx.x == 0) {
    s_len = a.sl[b];
    int ph = page < a.max_blocks ? a.bt[(int64_t)b * a.max_blocks + page] : -1;
    if (a.num_blocks > 0 && ph >= a.num_blocks) {
      if (tok0 < s_len) raise_error(ERR_BAD_PAGE);
      ph = -1;
    }
    s_phys = ph;
  }
  __syncthreads();
  const int L = s_len;
  const int phys = s_phys;
  const int ntok = min(a.bs, a.Sk - tok0);                 // rows of this page inside Sk
  const bool oob = tok0 >= L || phys < 0;
  const int nvalid = oob ? 0 : min(ntok, L - tok0);
  const int vrow = 2 * a.D;

  const uint8_t* kpage = a.kc + (int64_t)(phys < 0 ? 0 : phys) * a.kc_blk;
  const uint8_t* vpage = a.vc + (int64_t)(phys < 0 ? 0 : phys) * a.vc_blk;
  const uint8_t* ksrc = kpage;
  const uint8_t* vsrc = vpage;
  int64_t k_tok = a.kc_tok, k_head = a.kc_head, v_tok = a.vc_tok, v_head = a.vc_head;

  if constexpr (kBulk) {
    if (nvalid > 0) {
      const uint32_t kbytes = (uint32_t)(a.bs * a.Hkv * a.rb);
      const uint32_t vbytes = (uint32_t)(a.bs * a.Hkv * vrow);
      if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        fence_barrier_init();
        mbar_arrive_expect_tx(&bar, kbytes + vbytes);
        bulk_g2s(smem, kpage, kbytes, &bar);
        bulk_g2s(smem + kbytes, vpage, vbytes, &bar);
      }
      __syncthreads();
      if (!mbar_wait(&bar, 0)) return;
      ksrc = smem;
      vsrc = smem + kbytes;
      k_tok = (int64_t)a.Hkv * a.rb; k_head = a.rb;
      v_tok = (int64_t)a.Hkv * vrow; v_head = vrow;
    }
  }

  if constexpr (kFixed) {
    // V: 16 tokens x 16 chunks of 16 bytes per head; K: 16 rows x 17 words of 8 bytes per head
    for (int i = threadIdx.x; i < a.Hkv * 256; i += blockDim.x) {
      const int h = i >> 8, t = (i >> 4) & 15, c = i & 15;
      if (t >= ntok) continue;
      uint4 val = make_uint4(0u, 0u, 0u, 0u);
      if (t < nvalid) val = *reinterpret_cast<const uint4*>(vsrc + t * v_tok + h * v_head + c * 16);
      *reinterpret_cast<uint4*>(a.vo + (((int64_t)b * a.Hkv + h) * a.Sk + tok0 + t) * 256 + c * 16) = val;
    }
    for (int i = threadIdx.x; i < a.Hkv * 272; i += blockDim.x) {
      const int h = i / 272, r = i - h * 272;
      const int t = r / 17, c = r - t * 17;
      if (t >= nvalid) continue;
      *reinterpret_cast<uint2*>(a.ko + (((int64_t)b * a.Hkv + h) * a.Sk + tok0 + t) * 136 + c * 8) =
          *reinterpret_cast<const uint2*>(ksrc + t * k_tok + h * k_head + c * 8);
    }
    return;
  }
  // ---- V: copy valid rows, zero the rest of the page up to Sk -------------
  {
    const int chunks = vrow / 16;                  // 16-byte chunks per row
    const int total = a.Hkv * ntok * chunks;
    for (int i = threadIdx.x; i < total; i += blockDim.x) {
      const int h = i / (ntok * chunks);
      const int r = i - h * (ntok * chunks);
      const int t = r / chunks;
      const int c = r - t * chunks;
      uint4 val = make_uint4(0u, 0u, 0u, 0u);
      if (t < nvalid) val = *reinterpret_cast<const uint4*>(vsrc + t * v_tok + h * v_head + c * 16);
      uint8_t* dst = a.vo + (((int64_t)b * a.Hkv + h) * a.Sk + tok0 + t) * vrow + c * 16;
      *reinterpret_cast<uint4*>(dst) = val;
    }
  }
  // ---- K: valid rows only --------------------------------------------------
  if (nvalid > 0) {
    auto src = [&](int t, int h) { return ksrc + t * k_tok + h * k_head; };
    if (a.kw == 8) write_k_rows<8>(a, b, tok0, nvalid, src);
    else if (a.kw == 4) write_k_rows<4>(a, b, tok0, nvalid, src);
    else write_k_rows<2>(a, b, tok0, nvalid, src);
  }
}

}  // namespace g9

G9_ERROR_ACCESSORS(gather)

using namespace g9;

extern "C" cudaError_t gfx906_fa_gather_paged_kv_q8_checked(
    const uint8_t* key_cache_q8, const void* value_cache, const int32_t* block_table,
    const int32_t* seq_lens, uint8_t* k_out, void* v_out, int num_seqs, int num_kv_heads, int Sk,
    int D, int bytes_per_row, int block_size, int max_blocks_per_seq, int num_blocks, int64_t cache_block_stride,
    int64_t cache_token_stride, int64_t cache_head_stride_q8, int64_t v_cache_block_stride,
    int64_t v_cache_token_stride, int64_t v_cache_head_stride, cudaStream_t stream) {
  if (num_seqs == 0 || num_kv_heads == 0 || Sk == 0) return cudaSuccess;
  if (D % QK != 0 || D <= 0 || bytes_per_row != q8_row_bytes(D) || block_size <= 0 || Sk < 0 ||
      num_seqs < 0 || num_kv_heads < 0 || max_blocks_per_seq < 0)
    return cudaErrorInvalidValue;
  if (num_seqs > 65535) return cudaErrorInvalidValue;
  GatherArgs a{};
  a.kc = key_cache_q8;
  a.vc = reinterpret_cast<const uint8_t*>(value_cache);
  a.bt = block_table; a.sl = seq_lens;
  a.ko = k_out; a.vo = reinterpret_cast<uint8_t*>(v_out);
  a.kc_blk = cache_block_stride; a.kc_tok = cache_token_stride; a.kc_head = cache_head_stride_q8;
  a.vc_blk = v_cache_block_stride * 2; a.vc_tok = v_cache_token_stride * 2; a.vc_head = v_cache_head_stride * 2;
  a.B = num_seqs; a.Hkv = num_kv_heads; a.Sk = Sk; a.D = D; a.rb = bytes_per_row;
  a.bs = block_size; a.max_blocks = max_blocks_per_seq;
  a.num_blocks = num_blocks;
  // K row stores: widest width that keeps every destination row aligned
  const uintptr_t km = (uintptr_t)k_out | (uintptr_t)bytes_per_row | (uintptr_t)key_cache_q8 |
                       (uintptr_t)cache_block_stride | (uintptr_t)cache_token_stride |
                       (uintptr_t)cache_head_stride_q8;
  a.kw = (km & 7) == 0 ? 8 : ((km & 3) == 0 ? 4 : 2);
  // V rows are 2D bytes (multiple of 64): 16-byte stores need 16-byte aligned
  // buffers and row strides
  if (((uintptr_t)v_out | (uintptr_t)value_cache | (uintptr_t)a.vc_tok | (uintptr_t)a.vc_head |
       (uintptr_t)a.vc_blk) & 15)
    return cudaErrorInvalidValue;
  const int64_t kbytes = (int64_t)block_size * num_kv_heads * bytes_per_row;
  const int64_t vbytes = (int64_t)block_size * num_kv_heads * 2 * D;
  const bool dense = cache_token_stride == (int64_t)num_kv_heads * bytes_per_row &&
                     cache_head_stride_q8 == bytes_per_row &&
                     a.vc_tok == (int64_t)num_kv_heads * 2 * D && a.vc_head == 2 * D;
  const bool bulk = dense && (kbytes % 16 == 0) && (vbytes % 16 == 0) &&
                    (cache_block_stride % 16 == 0) && (a.vc_blk % 16 == 0) &&
                    ((uintptr_t)key_cache_q8 % 16 == 0) && kbytes + vbytes <= 200 * 1024;
  dim3 grid((Sk + block_size - 1) / block_size, num_seqs);
  if (bulk) {
    const size_t smem = (size_t)(kbytes + vbytes);
    const bool fixed = block_size == 16 && D == 128 && a.kw == 8;
    auto kern = fixed ? gather_kernel<true, true> : gather_kernel<true, false>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    kern<<<grid, kGatherThreads, smem, stream>>>(a);
  } else {
    gather_kernel<false><<<grid, kGatherThreads, 0, stream>>>(a);
  }
  return cudaGetLastError();
}

extern "C" cudaError_t launch_gather_paged_kv_q8(
    const uint8_t* key_cache_q8, const void* value_cache, const int32_t* block_table,
    const int32_t* seq_lens, uint8_t* k_out, void* v_out, int num_seqs, int num_kv_heads, int Sk,
    int D, int bytes_per_row, int block_size, int max_blocks_per_seq, int64_t cache_block_stride,
    int64_t cache_token_stride, int64_t cache_head_stride_q8, int64_t v_cache_block_stride,
    int64_t v_cache_token_stride, int64_t v_cache_head_stride, cudaStream_t stream) {
  return gfx906_fa_gather_paged_kv_q8_checked(key_cache_q8, value_cache, block_table, seq_lens, k_out, v_out,
                                              num_seqs, num_kv_heads, Sk, D, bytes_per_row, block_size,
                                              max_blocks_per_seq, 0, cache_block_stride, cache_token_stride,
                                              cache_head_stride_q8, v_cache_block_stride, v_cache_token_stride,
                                              v_cache_head_stride, stream);
}
