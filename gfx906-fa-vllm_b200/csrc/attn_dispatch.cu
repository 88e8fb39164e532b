// attn_dispatch.cu -- routes one attention batch to the decode (split-K,
// mma.sync) and prefill (tcgen05) kernels, and implements the reference's two
// attention launchers on top of that.
//
// Routing rule, evaluated per sequence on the device by both kernels: a
// sequence whose GQA-packed query rows (n_q * Hq/Hkv) fit in the decode row
// cap (decode_row_cap: 24 for the transposed decode consumer, else 32) goes to
// the decode kernel, which streams its Q8 pages once; longer query chunks go to
// the tensor-core prefill kernel.  Host-side n_q / kv_len bounds, when the
// caller has them (vLLM's metadata builder does), size the prefill workspace
// exactly; otherwise seq_q / max_kv bound every sequence.
#include <algorithm>
#include <vector>

#include "attn_common.cuh"

namespace g9 {
cudaError_t run_prefill(const G9AttnBatch& p, int nseq, const int* seq_ids, const int* nq_cap,
                        const int* kv_cap, int min_rows, void* ws, size_t ws_bytes, cudaStream_t stream);
size_t prefill_ws_bytes(const G9AttnBatch& p, int nseq, const int* nq_cap, const int* kv_cap);
int decode_row_cap(const G9AttnBatch& p);
}  // namespace g9

using namespace g9;

namespace {

struct Route {
  bool decode = false;
  std::vector<int> ids, nq, kv;
};

// allow_decode: the decode kernel is usable for this batch (dense 16-token
// pages, head_dim 128); otherwise every sequence goes to the prefill kernel.
Route route(const G9AttnBatch& b, const int* nq_host, const int* kv_host, bool allow_decode) {
  Route r;
  const int G = b.num_heads_q / std::max(1, b.num_heads_kv);
  const int cap = decode_row_cap(b);
  for (int i = 0; i < b.num_seqs; ++i) {
    const int nq = nq_host ? nq_host[i] : b.seq_q;
    const int kv = kv_host ? kv_host[i] : b.max_kv;
    if (nq <= 0) continue;
    // nq is exact with host n_q, an upper bound (seq_q) without
    const bool surely_small = (int64_t)nq * G <= cap;
    const bool maybe_small = nq_host ? surely_small : true;
    if (allow_decode && maybe_small) r.decode = true;
    if (allow_decode && surely_small) continue;
    r.ids.push_back(i);               // may be (or is) prefill-sized
    r.nq.push_back(nq);
    r.kv.push_back(kv);
  }
  return r;
}

size_t align_up(size_t x) { return (x + 1023) & ~(size_t)1023; }

bool decode_usable(const G9AttnBatch& b) { return gfx906_fa_decode_workspace_size(&b) > 0; }

size_t ws_size_impl(const G9AttnBatch& b, const int* nq_host, const int* kv_host, bool allow_decode) {
  Route r = route(b, nq_host, kv_host, allow_decode && decode_usable(b));
  const size_t dec = r.decode ? gfx906_fa_decode_workspace_size(&b) : 0;
  const size_t pre = r.ids.empty() ? 0 : prefill_ws_bytes(b, (int)r.ids.size(), r.nq.data(), r.kv.data());
  return align_up(dec) + align_up(pre) + 1024;
}

cudaError_t attention_impl(const G9AttnBatch& b, const int* nq_host, const int* kv_host, void* workspace,
                           size_t workspace_bytes, cudaStream_t stream, bool allow_decode) {
  if (b.num_seqs == 0 || b.seq_q == 0) return cudaSuccess;
  if (b.num_heads_kv <= 0 || b.num_heads_q <= 0 || b.num_heads_q % b.num_heads_kv) return cudaErrorInvalidValue;
  Route r = route(b, nq_host, kv_host, allow_decode && decode_usable(b));
  const size_t dec = r.decode ? gfx906_fa_decode_workspace_size(&b) : 0;
  const size_t pre = r.ids.empty() ? 0 : prefill_ws_bytes(b, (int)r.ids.size(), r.nq.data(), r.kv.data());
  const size_t need = align_up(dec) + align_up(pre) + 1024;
  if (!workspace || workspace_bytes < need) return cudaErrorInvalidValue;
  uint8_t* w = reinterpret_cast<uint8_t*>(((uintptr_t)workspace + 1023) & ~(uintptr_t)1023);
  cudaError_t e = cudaSuccess;
  if (!r.ids.empty()) {
    e = run_prefill(b, (int)r.ids.size(), r.ids.data(), r.nq.data(), r.kv.data(), r.decode ? decode_row_cap(b) : 0,
                    w + align_up(dec), align_up(pre), stream);
    if (e != cudaSuccess) return e;
  }
  if (r.decode) e = gfx906_fa_decode_splitk(&b, w, align_up(dec), stream);
  return e;
}

}  // namespace

extern "C" size_t gfx906_fa_attention_workspace_size(const G9AttnBatch* batch, const int* nq_host,
                                                     const int* kv_host) {
  return batch ? ws_size_impl(*batch, nq_host, kv_host, true) : 0;
}

extern "C" cudaError_t gfx906_fa_attention(const G9AttnBatch* batch, const int* nq_host, const int* kv_host,
                                           void* workspace, size_t workspace_bytes, cudaStream_t stream) {
  if (!batch) return cudaErrorInvalidValue;
  return attention_impl(*batch, nq_host, kv_host, workspace, workspace_bytes, stream, true);
}

// ---------------------------------------------------------------------------
// reference launchers
// ---------------------------------------------------------------------------
namespace {

// KV_max arrives expanded to [B, grid_x] (gfx906_fa.cpp:191-212); the value
// is the same for every tile, take tile 0.  No KV_max means `fill`.
__global__ void kv_len_from_expanded(const int* kv_max, int grid_x, int fill, int B, int* out) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b < B) out[b] = kv_max ? kv_max[(int64_t)b * grid_x] : fill;
}

__global__ void identity_table(int B, int* out) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b < B) out[b] = b;
}

// query tiles per sequence of the reference launcher (launcher.cu:201-206)
int ref_grid_x(int seq_q) {
  const int nc = seq_q > 32 ? 64 : seq_q > 16 ? 32 : seq_q > 8 ? 16 : seq_q > 4 ? 8 : seq_q > 2 ? 4 : 2;
  return (seq_q + nc - 1) / nc;
}

// Runs `b` with scratch from the stream-ordered allocator (the reference
// launchers have no workspace argument).  flat: contiguous [B, Hkv, Skv]
// tensors, described as one page per sequence through an identity table.
cudaError_t run_with_pool(G9AttnBatch& b, const int* kv_max_expanded, int grid_x, int kv_fill, bool flat,
                          cudaStream_t stream) {
  const int B = b.num_seqs;
  // When some sequence needs the prefill kernel (every sequence has seq_q
  // query rows here), its staging is sized per sequence from the actual
  // context lengths: KV_max is read to the host (one synchronisation of
  // `stream`) instead of bounding every sequence by the longest.
  std::vector<int> nq_host, kv_host;
  const int G = b.num_heads_q / b.num_heads_kv;
  if (flat || (int64_t)b.seq_q * G > decode_row_cap(b)) {
    nq_host.assign(B, b.seq_q);
    kv_host.assign(B, kv_fill);
    if (kv_max_expanded) {
      cudaError_t e = cudaMemcpy2DAsync(kv_host.data(), sizeof(int), kv_max_expanded, (size_t)grid_x * sizeof(int),
                                        sizeof(int), B, cudaMemcpyDeviceToHost, stream);
      if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
      if (e != cudaSuccess) return e;
      for (int& k : kv_host) k = std::max(0, std::min(k, b.max_kv));
    }
  }
  const int* nqh = nq_host.empty() ? nullptr : nq_host.data();
  const int* kvh = kv_host.empty() ? nullptr : kv_host.data();
  const size_t ws = ws_size_impl(b, nqh, kvh, !flat);
  const size_t ints = align_up((size_t)2 * B * sizeof(int));
  void* mem = nullptr;
  cudaError_t e = cudaMallocAsync(&mem, ws + ints, stream);
  if (e != cudaSuccess) return e;
  int* kvl = reinterpret_cast<int*>(mem);
  int* bt = kvl + B;
  kv_len_from_expanded<<<(B + 127) / 128, 128, 0, stream>>>(kv_max_expanded, grid_x, kv_fill, B, kvl);
  if (flat) identity_table<<<(B + 127) / 128, 128, 0, stream>>>(B, bt);
  e = cudaGetLastError();
  if (e == cudaSuccess) {
    b.kv_len = kvl;
    if (flat) b.block_table = bt;
    e = attention_impl(b, nqh, kvh, reinterpret_cast<uint8_t*>(mem) + ints, ws, stream, !flat);
  }
  cudaError_t f = cudaFreeAsync(mem, stream);
  return e != cudaSuccess ? e : f;
}

}  // namespace

extern "C" cudaError_t gfx906_fa_launch(const float* Q_fp32, const void* K_q8, const void* V_f16, float* O_fp32,
                                        void* O_meta, const int* KV_max_d, const void* MASK_f16,
                                        int32_t mask_seq_kv_padded, const int32_t* Q_ABS_OFFSET_d, int batch,
                                        int heads_q, int heads_kv, int seq_q, int seq_kv, int head_dim,
                                        float scale, cudaStream_t stream) {
  (void)O_meta;   // only written by the reference when KV splitting is on, which it never is
  if (head_dim != 128 || heads_kv <= 0 || heads_q % heads_kv) return cudaErrorInvalidValue;
  if (batch < 0 || seq_q < 0 || seq_kv < 0) return cudaErrorInvalidValue;
  if (MASK_f16 && Q_ABS_OFFSET_d) return cudaErrorInvalidValue;
  if (batch == 0 || seq_q == 0) return cudaSuccess;
  const int rb = q8_row_bytes(head_dim);
  G9AttnBatch b{};
  b.q = Q_fp32;
  b.q_dtype = G9_DT_F32;
  b.q_seq_stride = (int64_t)heads_q * seq_q * head_dim;
  b.q_tok_stride = head_dim;
  b.q_head_stride = (int64_t)seq_q * head_dim;
  b.seq_q = seq_q;
  b.out = O_fp32;                                   // BSHD, as the reference kernel writes it
  b.out_dtype = G9_DT_F32;
  b.o_seq_stride = (int64_t)seq_q * heads_q * head_dim;
  b.o_tok_stride = (int64_t)heads_q * head_dim;
  b.o_head_stride = head_dim;
  // contiguous [B, Hkv, Skv, row]: one page of seq_kv tokens per sequence
  b.k_cache = reinterpret_cast<const uint8_t*>(K_q8);
  b.k_page_stride = (int64_t)heads_kv * seq_kv * rb;
  b.k_tok_stride = rb;
  b.k_head_stride = (int64_t)seq_kv * rb;
  b.v_cache = reinterpret_cast<const uint8_t*>(V_f16);
  b.v_page_stride = (int64_t)heads_kv * seq_kv * head_dim * 2;
  b.v_tok_stride = head_dim * 2;
  b.v_head_stride = (int64_t)seq_kv * head_dim * 2;
  b.v_fmt = G9_VFMT_F16;
  b.max_blocks = 1;
  b.block_size = std::max(seq_kv, 1);
  b.max_kv = seq_kv;
  b.q_abs = Q_ABS_OFFSET_d;
  b.mask = MASK_f16;
  b.mask_seq_stride = (int64_t)seq_q * mask_seq_kv_padded;
  b.mask_tok_stride = mask_seq_kv_padded;
  b.num_seqs = batch;
  b.num_heads_q = heads_q;
  b.num_heads_kv = heads_kv;
  b.head_dim = head_dim;
  b.scale = scale;
  // the flat layout is not made of 16-token pages: every sequence takes the
  // prefill path, whose pack kernel reads any row layout
  return run_with_pool(b, KV_max_d, ref_grid_x(seq_q), seq_kv, true, stream);
}

extern "C" cudaError_t gfx906_fa_launch_paged(const float* Q_fp32, const void* K_paged, const void* V_paged,
                                              const int32_t* block_table, const int32_t* kv_max_d, float* O_fp32,
                                              void* O_meta, const void* MASK_f16, int32_t mask_seq_kv_padded,
                                              const int32_t* Q_ABS_OFFSET_d, int batch, int heads_q,
                                              int heads_kv, int seq_q, int max_seq_kv, int head_dim,
                                              int block_size, int max_blocks_per_seq, int64_t k_block_stride,
                                              int64_t k_token_stride, int64_t k_head_stride,
                                              int64_t v_block_stride, int64_t v_token_stride,
                                              int64_t v_head_stride, float scale, cudaStream_t stream) {
  (void)O_meta;
  if (head_dim != 128 || heads_kv <= 0 || heads_q % heads_kv || block_size != 16) return cudaErrorInvalidValue;
  if (batch < 0 || seq_q < 0) return cudaErrorInvalidValue;
  if (MASK_f16 && Q_ABS_OFFSET_d) return cudaErrorInvalidValue;
  if (batch == 0 || seq_q == 0) return cudaSuccess;
  G9AttnBatch b{};
  b.q = Q_fp32;
  b.q_dtype = G9_DT_F32;
  b.q_seq_stride = (int64_t)heads_q * seq_q * head_dim;
  b.q_tok_stride = head_dim;
  b.q_head_stride = (int64_t)seq_q * head_dim;
  b.seq_q = seq_q;
  b.out = O_fp32;
  b.out_dtype = G9_DT_F32;
  b.o_seq_stride = (int64_t)seq_q * heads_q * head_dim;
  b.o_tok_stride = (int64_t)heads_q * head_dim;
  b.o_head_stride = head_dim;
  b.k_cache = reinterpret_cast<const uint8_t*>(K_paged);
  b.k_page_stride = k_block_stride;
  b.k_tok_stride = k_token_stride;
  b.k_head_stride = k_head_stride;
  b.v_cache = reinterpret_cast<const uint8_t*>(V_paged);
  b.v_page_stride = v_block_stride;
  b.v_tok_stride = v_token_stride;
  b.v_head_stride = v_head_stride;
  b.v_fmt = G9_VFMT_F16;
  b.block_table = block_table;
  b.max_blocks = max_blocks_per_seq;
  b.block_size = block_size;
  b.max_kv = std::max(max_seq_kv, max_blocks_per_seq * block_size);
  b.q_abs = Q_ABS_OFFSET_d;
  b.mask = MASK_f16;
  b.mask_seq_stride = (int64_t)seq_q * mask_seq_kv_padded;
  b.mask_tok_stride = mask_seq_kv_padded;
  b.num_seqs = batch;
  b.num_heads_q = heads_q;
  b.num_heads_kv = heads_kv;
  b.head_dim = head_dim;
  b.scale = scale;
  return run_with_pool(b, kv_max_d, ref_grid_x(seq_q), b.max_kv, false, stream);
}
