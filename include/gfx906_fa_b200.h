/*
 * gfx906_fa_b200.h -- C ABI of the sm_100a paged-Q8 attention library
 * (libgfx906fa_b200.so).
 *
 * Plain pointers, sizes and CUDA streams only.  Every entry point is
 * asynchronous on `stream`, allocates nothing unless its comment says so, and
 * returns cudaSuccess or the error of the failed launch / argument check
 * (cudaErrorInvalidValue for rejected arguments).
 *
 * The first group keeps the names and argument lists of the reference's
 * extern "C" launchers (nick413-bit/gfx906-fa-vllm, HIP), with hipError_t /
 * hipStream_t replaced by their CUDA equivalents and __half pointers passed
 * as const void*.  The second group is new: dtype-generic stores, the
 * split-K decode / tensor-core prefill attention with caller-provided
 * workspace, and the device error word.
 */
#ifndef GFX906_FA_B200_H_
#define GFX906_FA_B200_H_

#include <stddef.h>
#include <stdint.h>
#include <cuda_runtime_api.h>

#ifdef __cplusplus
extern "C" {
#endif

/* element types of Q / K / V / O buffers */
#define G9_DT_F16 0
#define G9_DT_BF16 1
#define G9_DT_F32 2
#define G9_DT_FP8E4M3 3   /* attention output only: out = sat_e4m3(o / *out_scale), vLLM's static
                             per-tensor fp8 output quantisation */

/* V handling of gfx906_fa_store_kv */
#define G9_V_NONE 0   /* K only */
#define G9_V_COPY16 1 /* V copied as 16-bit rows (fp16 / bf16) */
#define G9_V_Q8 2     /* V quantised to Q8_0 like K, token rows */
#define G9_V_Q8T 3    /* V quantised to Q8_0, page-transposed records (G9_VFMT_Q8T) */

/* ======================================================================= */
/* Reference launchers (same names and argument meaning)                    */
/* ======================================================================= */

/* Dense Q8_0 quantisation of N rows of D fp16 values into N rows of
 * D/32*34 bytes.  Replaces launch_quantize_q8_0_dense
 * (extension/gfx906_fa_quant.cu:206-212). */
cudaError_t launch_quantize_q8_0_dense(const void* x, uint8_t* y, int N, int D,
                                       cudaStream_t stream);

/* Quantise fp16 K tokens [num_tokens, Hkv, D] (element strides) and scatter
 * them into the paged Q8 cache by slot_mapping (byte strides); slot < 0 skips
 * the token.  Replaces launch_reshape_and_cache_q8
 * (extension/gfx906_fa_quant.cu:225-239). */
cudaError_t launch_reshape_and_cache_q8(const void* key, const int64_t* slot_mapping,
                                        uint8_t* k_cache_q8, int num_tokens, int num_kv_heads,
                                        int head_size, int block_size, int64_t key_token_stride,
                                        int64_t key_head_stride, int64_t cache_block_stride,
                                        int64_t cache_token_stride, int64_t cache_head_stride,
                                        cudaStream_t stream);

/* Paged K_q8 [NB, bs, Hkv, bytes_per_row] + fp16 V [NB, bs, Hkv, D] ->
 * contiguous k_out [B, Hkv, Sk, bytes_per_row], v_out [B, Hkv, Sk, D].
 * V rows at token >= seq_lens[b] are zeroed, K rows there are not written;
 * a page with block_table entry < 0 counts as out of range.  Strides are in
 * bytes for the K cache and in elements for V.  Replaces
 * launch_gather_paged_kv_q8 (extension/gfx906_fa_gather.cu:362-383). */
cudaError_t launch_gather_paged_kv_q8(const uint8_t* key_cache_q8, const void* value_cache,
                                      const int32_t* block_table, const int32_t* seq_lens,
                                      uint8_t* k_out, void* v_out, int num_seqs, int num_kv_heads,
                                      int Sk, int D, int bytes_per_row, int block_size,
                                      int max_blocks_per_seq, int64_t cache_block_stride,
                                      int64_t cache_token_stride, int64_t cache_head_stride_q8,
                                      int64_t v_cache_block_stride, int64_t v_cache_token_stride,
                                      int64_t v_cache_head_stride, cudaStream_t stream);

/* ======================================================================= */
/* New entry points                                                         */
/* ======================================================================= */

/* launch_gather_paged_kv_q8 with the cache's page count: block-table entries
 * >= num_blocks are treated like negative ones (the page counts as out of
 * range) and set bit 1 of the device error word, so a corrupt table cannot
 * send a copy outside the cache allocation.  num_blocks <= 0 checks nothing
 * (the reference launcher's behaviour). */
cudaError_t gfx906_fa_gather_paged_kv_q8_checked(
    const uint8_t* key_cache_q8, const void* value_cache, const int32_t* block_table, const int32_t* seq_lens,
    uint8_t* k_out, void* v_out, int num_seqs, int num_kv_heads, int Sk, int D, int bytes_per_row, int block_size,
    int max_blocks_per_seq, int num_blocks, int64_t cache_block_stride, int64_t cache_token_stride,
    int64_t cache_head_stride_q8, int64_t v_cache_block_stride, int64_t v_cache_token_stride,
    int64_t v_cache_head_stride, cudaStream_t stream);

/* Dense Q8_0 quantisation of N rows of D elements of type x_dtype
 * (G9_DT_*) -- the dtype-generic form of launch_quantize_q8_0_dense. */
cudaError_t gfx906_fa_quantize_q8_0(const void* x, int x_dtype, uint8_t* y, int64_t N, int D,
                                    cudaStream_t stream);

/* Fused KV store: K [T, Hkv, D] quantised to Q8_0 into k_cache and, per
 * v_mode, V [T, Hkv, D] copied (G9_V_COPY16) or quantised (G9_V_Q8 token
 * rows, G9_V_Q8T page-transposed records; v_token_stride is ignored for the
 * latter) into v_cache, both addressed by slot_mapping (slot < 0 skips the
 * token).
 * Element strides for key/value, byte strides for the caches.  Replaces the
 * pair vLLM triton_reshape_and_cache_flash + reshape_and_cache_q8 called by
 * Gfx906FAImpl.do_kv_cache_update (extension/gfx906_fa_backend.py:405-442). */
cudaError_t gfx906_fa_store_kv(const void* key, int key_dtype, int64_t key_token_stride,
                               int64_t key_head_stride, const void* value, int value_dtype,
                               int64_t value_token_stride, int64_t value_head_stride,
                               const int64_t* slot_mapping, uint8_t* k_cache, int64_t k_block_stride,
                               int64_t k_token_stride, int64_t k_head_stride, uint8_t* v_cache,
                               int64_t v_block_stride, int64_t v_token_stride,
                               int64_t v_head_stride, int v_mode, int num_tokens, int num_kv_heads,
                               int head_size, int block_size, cudaStream_t stream);

/* Fused RoPE + KV store, the kernel behind vLLM's RoPE / KV-cache fusion
 * hook (AttentionImpl.do_rope_and_kv_cache_update; the reference backend
 * has none: extension/gfx906_fa_backend.py:444-445).  K [T, Hkv, 128] and,
 * when query is not NULL, Q [T, Hq, 128] are rotated in place by the
 * position's angles (positions int64 [T]; cos_sin_cache [max_pos, rot_dim]
 * with cos of pair j at column j and sin at rot_dim/2 + j; NeoX style pairs
 * (i, i + rot_dim/2), GPT-J style (2j, 2j+1); rot_dim 32, 64 or 128),
 * computed in fp32 and rounded once to the tensor's type; the rotated K is
 * then quantised to Q8_0 into k_cache and V stored per v_mode, both by
 * slot_mapping (slot < 0: rotated in place, not stored).  Strides as for
 * gfx906_fa_store_kv. */
cudaError_t gfx906_fa_rope_store_kv(
    void* query, int query_dtype, int64_t query_token_stride, int64_t query_head_stride, int num_heads_q,
    void* key, int key_dtype, int64_t key_token_stride, int64_t key_head_stride, const void* value,
    int value_dtype, int64_t value_token_stride, int64_t value_head_stride, const int64_t* positions,
    const void* cos_sin_cache, int cos_sin_dtype, int rot_dim, int is_neox, const int64_t* slot_mapping,
    uint8_t* k_cache, int64_t k_block_stride, int64_t k_token_stride, int64_t k_head_stride, uint8_t* v_cache,
    int64_t v_block_stride, int64_t v_token_stride, int64_t v_head_stride, int v_mode, int num_tokens,
    int num_kv_heads, int head_size, int block_size, cudaStream_t stream);

/* ----------------------------------------------------------------------- */
/* Attention over a batch of sequences                                       */
/* ----------------------------------------------------------------------- */

/* V cache formats */
#define G9_VFMT_F16 0
#define G9_VFMT_BF16 1
#define G9_VFMT_Q8 2
/* Q8_0 V, page-transposed: the Q8_0 blocks of V (the same int8 values and
 * fp16 scales as G9_VFMT_Q8) are stored per (page, kv head) as one record of
 * block_size*(head_dim/32)*34 bytes at page*v_page_stride + h*v_head_stride:
 *   bytes [0, 2*(head_dim/32)*block_size): fp16 scale of block j of token t
 *                                           at 2*(j*block_size + t)
 *   then head_dim rows of block_size int8: value of dim d of token t at
 *        2*(head_dim/32)*block_size + d*block_size + t
 * so that the tensor cores read the keys of one dim as consecutive bytes.
 * v_tok_stride is ignored.  No reference counterpart (the reference keeps V
 * in fp16). */
#define G9_VFMT_Q8T 3

/* One attention call.  All pointers are device pointers.
 *
 * Query row (sequence b, token t < n_q[b], query head hq) is read at
 *   q + b*q_seq_stride + (q_start[b] + t)*q_tok_stride + hq*q_head_stride
 * (elements of q_dtype) and its output written at the same position of
 * `out` with the o_* strides (elements of out_dtype).  q_start == NULL means
 * 0, n_q == NULL means seq_q for every sequence; seq_q is also the maximum
 * of n_q.
 *
 * Key / value row (sequence b, key k < kv_len[b], kv head h) lives in page
 * block_table[b*max_blocks + k/block_size] at
 *   page*page_stride + (k%block_size)*tok_stride + h*head_stride   (bytes).
 * K rows are Q8_0 (head_dim/32*34 bytes); V rows are fp16 / bf16 or Q8_0
 * (v_fmt), or Q8_0 page-transposed records (G9_VFMT_Q8T, above).  max_kv is a host-side upper bound of kv_len.
 *
 * Visibility: key k is visible to query token t iff k < kv_len[b] and, when
 * q_abs != NULL, k <= q_abs[b] + t (the reference's inline causal rule,
 * kernel/fattn-q8.cuh:646-654).  `mask` (optional, fp16, additive) adds
 * mask[b*mask_seq_stride + t*mask_tok_stride + k] to the scaled score
 * (kernel/fattn-q8.cuh:628-631).  Query heads map to kv heads by
 * hq / (num_heads_q / num_heads_kv).  A query row with no visible key is
 * written as zeros.
 *
 * Query positions: token t of sequence b sits at qp = q_abs[b] + t, or at
 * kv_len[b] - n_q[b] + t without q_abs (the last query token is the last
 * key).  The sliding window keeps keys qp - window < k <= (causal limit);
 * the reference kernel's logit soft-cap (kernel/fattn-q8.cuh:638-640) maps
 * the scaled score s to softcap * tanh(s / softcap) before the mask is added;
 * a sink adds exp(sink[hq]) (relative to the row's max) to the softmax
 * denominator of every row of query head hq, as vLLM's attention-sink models
 * define it.  kv_len[b] is clamped to max_blocks * block_size and to max_kv.
 * A block-table entry that is negative, or >= num_blocks when num_blocks > 0,
 * is never dereferenced: it sets bit 1 of the device error word and its keys
 * are dropped (decode) or read as zero vectors (prefill). */
typedef struct G9AttnBatch {
  const void* q;
  int q_dtype;
  int64_t q_seq_stride, q_tok_stride, q_head_stride;
  const int32_t* q_start;
  const int32_t* n_q;
  int seq_q;
  void* out;
  int out_dtype;
  int64_t o_seq_stride, o_tok_stride, o_head_stride;
  const uint8_t* k_cache;
  int64_t k_page_stride, k_tok_stride, k_head_stride;
  const uint8_t* v_cache;
  int64_t v_page_stride, v_tok_stride, v_head_stride;
  int v_fmt;
  const int32_t* block_table;
  int max_blocks;
  int block_size;
  const int32_t* kv_len;
  int max_kv;
  const int32_t* q_abs;
  const void* mask;
  int64_t mask_seq_stride, mask_tok_stride;
  int num_seqs, num_heads_q, num_heads_kv, head_dim;
  float scale;
  /* Fields below are optional; a zero-initialised value turns each off. */
  int num_blocks;       /* pages in the cache: entries >= num_blocks (and < 0) are bad pages (0: not checked) */
  float softcap;        /* > 0: scaled score s -> softcap * tanh(s / softcap), before the mask */
  int window;           /* > 0: sliding window, key k visible to query position qp only if qp - k < window */
  const float* sinks;   /* [num_heads_q] fp32 logits (scaled-score units) added to each row's softmax
                           denominator only, or NULL */
  int flags;            /* G9_F_* below */
  const float* out_scale; /* out_dtype G9_DT_FP8E4M3: device fp32 scalar; each output element is
                             o / *out_scale rounded to e4m3 (nearest even), saturated to +-448 */
} G9AttnBatch;

/* G9AttnBatch.flags */
#define G9_F_CU_SEQLENS 1  /* n_q == NULL: q_start holds num_seqs + 1 offsets (vLLM's query_start_loc) and
                              n_q[b] = q_start[b + 1] - q_start[b] */
#define G9_F_CAUSAL_END 2  /* q_abs == NULL: causal with q_abs[b] = kv_len[b] - n_q[b] (the query chunk
                              ends at the last key, vLLM's chunked-prefill convention) */

/* Split-K flash decoding straight from the paged Q8 cache (no gather):
 * persistent CTAs walk (KV chunk, kv-head group, sequence) items, stream
 * whole pages into shared memory with bulk-async copies and compute all query
 * heads of a GQA group (and all query tokens) together on tensor cores; a
 * second kernel merges per-chunk partial results.  Handles the sequences
 * whose GQA-packed query rows n_q * (Hq/Hkv) fit in min(32, seq_q*Hq/Hkv);
 * others are skipped.  Requirements: head_dim 128, block_size 16,
 * num_heads_kv in {1, 2, 4} or a multiple of 8, pages laid out
 * [block_size][Hkv][row] (dense rows), 16-byte aligned pages.
 * gfx906_fa_decode_workspace_size returns 0 when the batch is not supported.
 * workspace: device scratch of at least that many bytes (16-byte aligned);
 * its contents need no initialisation. */
size_t gfx906_fa_decode_workspace_size(const G9AttnBatch* batch);
cudaError_t gfx906_fa_decode_splitk(const G9AttnBatch* batch, void* workspace, size_t workspace_bytes,
                                    cudaStream_t stream);

/* Allocation-free form of gfx906_fa_decode_splitk, for callers that cannot
 * allocate device memory when they call (code inside an allocator's own
 * hooks, runtimes that own the whole device heap, plugin hosts with a fixed
 * budget).  No counterpart in the reference.  The split-K partial results go
 * to a 32 MiB array that the library holds in static device memory on every
 * GPU that loads it, until the process exits; batches whose decode workspace
 * (gfx906_fa_decode_workspace_size) exceeds 32 MiB are rejected with
 * cudaErrorInvalidValue.  The first call on each device looks up the array's
 * device address (cudaGetSymbolAddress) with that device current; make that
 * first call before any stream capture.  All calls share the one array and
 * it keeps whatever the last call left; the one part that must start at zero
 * (a work counter) is cleared by each call on its stream.
 * Calls that overlap on the GPU (different streams, or different host
 * threads, on one device) race on it and must be serialised by the caller.
 * Allocates nothing: no cudaMalloc / cudaFree. */
cudaError_t gfx906_fa_decode_splitk_noalloc(const G9AttnBatch* batch, cudaStream_t stream);

/* Tensor-core prefill: for each listed sequence (seq_ids[i], up to nq_cap[i]
 * query tokens, up to kv_cap[i] visible keys -- host-side upper bounds) the
 * visible Q8 pages are dequantised once into fp16 staging tiles in the
 * workspace, then one CTA per 128 GQA-packed query rows of a kv head runs
 * S = Q K^T and O += P V on tcgen05 tensor cores with the accumulators in
 * tensor memory, fed by TMA.  Requirements: head_dim 128, K rows readable
 * with 2-byte loads, 16-bit V rows with 4-byte loads.  This entry computes
 * every listed sequence (gfx906_fa_attention leaves the short ones to the
 * decode kernel).  workspace: at least gfx906_fa_prefill_workspace_size()
 * bytes; no initialisation needed. */
size_t gfx906_fa_prefill_workspace_size(const G9AttnBatch* batch, int num_prefill_seqs, const int* nq_cap,
                                        const int* kv_cap);
cudaError_t gfx906_fa_prefill_tc(const G9AttnBatch* batch, int num_prefill_seqs, const int* seq_ids,
                                 const int* nq_cap, const int* kv_cap, void* workspace, size_t workspace_bytes,
                                 cudaStream_t stream);

/* Whole-batch attention: sequences whose GQA-packed query rows
 * (n_q * Hq/Hkv) fit in 32 run on the split-K decode kernel, longer query
 * chunks on the tensor-core prefill kernel; both read the same paged Q8
 * cache.  nq_host / kv_host (host arrays of num_seqs ints, optional) give
 * exact per-sequence query counts and upper bounds of the KV lengths -- with
 * them the routing is decided on the host and the workspace is sized
 * exactly; without them seq_q / max_kv bound every sequence and each kernel
 * picks its sequences on the device.  The same nq_host / kv_host must be
 * passed to the size query and to the call.  Replaces the path choice of
 * forward_paged (extension/gfx906_fa_paged.py:60-70,255-376). */
size_t gfx906_fa_attention_workspace_size(const G9AttnBatch* batch, const int* nq_host, const int* kv_host);
cudaError_t gfx906_fa_attention(const G9AttnBatch* batch, const int* nq_host, const int* kv_host, void* workspace,
                                size_t workspace_bytes, cudaStream_t stream);

/* Reference flat attention: Q fp32 [B, Hq, Sq, D], K_q8 [B, Hkv, Skv,
 * D/32*34], V fp16 [B, Hkv, Skv, D] -> O fp32 [B, Sq, Hq, D] (BSHD, as the
 * reference kernel writes it).  KV_max: int32 [B, grid_x] as expanded by the
 * reference's C++ (one value per sequence, repeated per query tile) or NULL;
 * MASK_f16: additive fp16 [B, Sq, mask_seq_kv_padded] or NULL;
 * Q_ABS_OFFSET_d: int32 [B] inline-causal offsets or NULL (exclusive with
 * the mask).  O_meta is accepted and not written (the reference only writes
 * it with KV splitting, which it never enables).  head_dim must be 128.
 * Allocates its workspace with cudaMallocAsync on `stream` and frees it the
 * same way.  Replaces gfx906_fa_launch (extension/gfx906_fa_launcher.cu:53-75). */
cudaError_t gfx906_fa_launch(const float* Q_fp32, const void* K_q8, const void* V_f16, float* O_fp32, void* O_meta,
                             const int* KV_max_d, const void* MASK_f16, int32_t mask_seq_kv_padded,
                             const int32_t* Q_ABS_OFFSET_d, int batch, int heads_q, int heads_kv, int seq_q,
                             int seq_kv, int head_dim, float scale, cudaStream_t stream);

/* Reference direct-paged attention: Q fp32 [B, Hq, Sq, D] against K_paged
 * [NB, 16, Hkv, D/32*34] / fp16 V_paged [NB, 16, Hkv, D] (byte strides)
 * through block_table -> O fp32 [B, Sq, Hq, D] (BSHD).  kv_max_d: int32
 * [B, grid_x] expanded per-sequence lengths (gfx906_fa.cpp:604).  Same
 * workspace behaviour as gfx906_fa_launch.  Replaces gfx906_fa_launch_paged
 * (extension/gfx906_fa_launcher.cu:222-249). */
cudaError_t gfx906_fa_launch_paged(const float* Q_fp32, const void* K_paged, const void* V_paged,
                                   const int32_t* block_table, const int32_t* kv_max_d, float* O_fp32, void* O_meta,
                                   const void* MASK_f16, int32_t mask_seq_kv_padded, const int32_t* Q_ABS_OFFSET_d,
                                   int batch, int heads_q, int heads_kv, int seq_q, int max_seq_kv, int head_dim,
                                   int block_size, int max_blocks_per_seq, int64_t k_block_stride,
                                   int64_t k_token_stride, int64_t k_head_stride, int64_t v_block_stride,
                                   int64_t v_token_stride, int64_t v_head_stride, float scale, cudaStream_t stream);

/* Device error word (bit 0: a bounded wait timed out, bit 1: a block-table
 * entry was out of range, bit 2: tensor-memory allocation failed).
 * gfx906_fa_get_device_error synchronises the current device and reads it;
 * gfx906_fa_clear_device_error resets it to zero. */
cudaError_t gfx906_fa_get_device_error(unsigned int* out);
cudaError_t gfx906_fa_clear_device_error(void);

/* Self-test of the bounded waits every kernel uses: launches one thread that
 * waits on an mbarrier nothing arrives at, with a limit of limit_ns
 * (<= 100 ms).  The wait gives up, sets bit 0 of the device error word and
 * writes 1 to *done (device int; 2 would mean the wait completed).  The
 * context stays usable.  No reference counterpart (failure-detection test
 * hook). */
cudaError_t gfx906_fa_selftest_wait_timeout(uint64_t limit_ns, int* done, cudaStream_t stream);

/* Library version string (static storage). */
const char* gfx906_fa_version(void);

#ifdef __cplusplus
}
#endif

#endif /* GFX906_FA_B200_H_ */
