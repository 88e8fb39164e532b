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

/* V handling of gfx906_fa_store_kv */
#define G9_V_NONE 0   /* K only */
#define G9_V_COPY16 1 /* V copied as 16-bit rows (fp16 / bf16) */
#define G9_V_Q8 2     /* V quantised to Q8_0 like K */

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

/* Dense Q8_0 quantisation of N rows of D elements of type x_dtype
 * (G9_DT_*) -- the dtype-generic form of launch_quantize_q8_0_dense. */
cudaError_t gfx906_fa_quantize_q8_0(const void* x, int x_dtype, uint8_t* y, int64_t N, int D,
                                    cudaStream_t stream);

/* Fused KV store: K [T, Hkv, D] quantised to Q8_0 into k_cache and, per
 * v_mode, V [T, Hkv, D] copied (G9_V_COPY16) or quantised (G9_V_Q8) into
 * v_cache, both addressed by slot_mapping (slot < 0 skips the token).
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

/* Device error word (bit 0: a bounded wait timed out, bit 1: a block-table
 * entry was out of range, bit 2: tensor-memory allocation failed).
 * gfx906_fa_get_device_error synchronises the current device and reads it;
 * gfx906_fa_clear_device_error resets it to zero. */
cudaError_t gfx906_fa_get_device_error(unsigned int* out);
cudaError_t gfx906_fa_clear_device_error(void);

/* Library version string (static storage). */
const char* gfx906_fa_version(void);

#ifdef __cplusplus
}
#endif

#endif /* GFX906_FA_B200_H_ */
