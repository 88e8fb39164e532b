// torch_ops.cpp -- the `gfx906_fa` torch extension module.
//
// Same module name, function names, keyword arguments, output allocation and
// error behaviour as the reference's pybind module
// (extension/gfx906_fa.cpp:660-690): TORCH_CHECK on every argument (raising
// RuntimeError), outputs allocated with torch::empty on the input's device,
// every launch asynchronous on the current CUDA stream.  The work itself is
// done by the C ABI in libgfx906fa_b200.so (include/gfx906_fa_b200.h); this
// file only validates, allocates and forwards pointers.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "gfx906_fa_b200.h"

namespace {

#define CHECK_CUDA(x) TORCH_CHECK((x).device().is_cuda(), #x " must be a CUDA tensor")
#define CHECK_CONTIG(x) TORCH_CHECK((x).is_contiguous(), #x " must be contiguous")

int dtype_code(const torch::Tensor& t, const char* name) {
  switch (t.scalar_type()) {
    case torch::kFloat16: return G9_DT_F16;
    case torch::kBFloat16: return G9_DT_BF16;
    case torch::kFloat32: return G9_DT_F32;
    default: TORCH_CHECK(false, name, " must be fp16, bf16 or fp32, got ", t.scalar_type());
  }
  return -1;
}

void check_status(cudaError_t e, const char* what) {
  TORCH_CHECK(e == cudaSuccess, what, " failed: ", cudaGetErrorString(e));
}

cudaStream_t cur_stream() { return at::cuda::getCurrentCUDAStream().stream(); }

// ---------------------------------------------------------------------------
// quantize_q8_0 (extension/gfx906_fa.cpp:273-309)
// ---------------------------------------------------------------------------
torch::Tensor quantize_q8_0(torch::Tensor k_fp16) {
  CHECK_CUDA(k_fp16);
  CHECK_CONTIG(k_fp16);
  TORCH_CHECK(k_fp16.dim() >= 1, "k_fp16 must have at least 1 dim");
  const int dt = dtype_code(k_fp16, "k_fp16");
  const int64_t D = k_fp16.size(-1);
  TORCH_CHECK(D % 32 == 0 && D > 0 && D <= 512, "last dim must be a multiple of 32 (<= 512)");
  const int64_t N = D ? k_fp16.numel() / D : 0;
  std::vector<int64_t> shape(k_fp16.sizes().begin(), k_fp16.sizes().end());
  shape.back() = (D / 32) * 34;
  auto out = torch::empty(shape, k_fp16.options().dtype(torch::kUInt8));
  c10::cuda::CUDAGuard g(k_fp16.device());
  check_status(gfx906_fa_quantize_q8_0(k_fp16.data_ptr(), dt, out.data_ptr<uint8_t>(), N, (int)D,
                                       cur_stream()),
               "launch_quantize_q8_0_dense");
  return out;
}

// ---------------------------------------------------------------------------
// reshape_and_cache_q8 (extension/gfx906_fa.cpp:322-374)
// ---------------------------------------------------------------------------
void reshape_and_cache_q8(torch::Tensor key, torch::Tensor slot_mapping, torch::Tensor k_cache_q8) {
  CHECK_CUDA(key);
  CHECK_CUDA(slot_mapping);
  CHECK_CUDA(k_cache_q8);
  const int kdt = dtype_code(key, "key");
  TORCH_CHECK(slot_mapping.dtype() == torch::kInt64, "slot_mapping must be int64");
  TORCH_CHECK(k_cache_q8.dtype() == torch::kUInt8, "k_cache_q8 must be uint8");
  TORCH_CHECK(key.dim() == 3, "key must be [num_tokens, Hkv, D]");
  TORCH_CHECK(k_cache_q8.dim() == 4, "k_cache_q8 must be [B, bs, Hkv, bytes]");
  TORCH_CHECK(key.stride(2) == 1, "key last dim must be contiguous");
  CHECK_CONTIG(slot_mapping);
  CHECK_CONTIG(k_cache_q8);
  const int T = key.size(0), Hkv = key.size(1), D = key.size(2);
  TORCH_CHECK(D % 32 == 0, "head_size must be multiple of 32");
  const int rb = (D / 32) * 34;
  const int bs = k_cache_q8.size(1);
  TORCH_CHECK(k_cache_q8.size(2) == Hkv, "k_cache_q8 Hkv mismatch: got ", k_cache_q8.size(2),
              " vs key Hkv=", Hkv);
  TORCH_CHECK(k_cache_q8.size(3) == rb, "k_cache_q8 last dim mismatch: got ", k_cache_q8.size(3),
              " expected ", rb);
  TORCH_CHECK(slot_mapping.size(0) == T, "slot_mapping length mismatch");
  c10::cuda::CUDAGuard g(key.device());
  check_status(gfx906_fa_store_kv(key.data_ptr(), kdt, key.stride(0), key.stride(1), nullptr, G9_DT_F16, 0, 0,
                                  slot_mapping.data_ptr<int64_t>(), k_cache_q8.data_ptr<uint8_t>(),
                                  (int64_t)bs * Hkv * rb, (int64_t)Hkv * rb, rb, nullptr, 0, 0, 0,
                                  G9_V_NONE, T, Hkv, D, bs, cur_stream()),
               "launch_reshape_and_cache_q8");
}

// ---------------------------------------------------------------------------
// gather_paged_kv_q8 (extension/gfx906_fa.cpp:393-498)
// ---------------------------------------------------------------------------
std::vector<torch::Tensor> gather_paged_kv_q8(torch::Tensor key_cache_q8, torch::Tensor value_cache,
                                              torch::Tensor block_table, torch::Tensor seq_lens,
                                              int64_t Sk, c10::optional<torch::Tensor> k_out_opt,
                                              c10::optional<torch::Tensor> v_out_opt) {
  CHECK_CUDA(key_cache_q8);
  CHECK_CUDA(value_cache);
  CHECK_CUDA(block_table);
  CHECK_CUDA(seq_lens);
  TORCH_CHECK(key_cache_q8.dtype() == torch::kUInt8, "key_cache_q8 must be uint8");
  TORCH_CHECK(value_cache.dtype() == torch::kFloat16 || value_cache.dtype() == torch::kBFloat16,
              "value_cache must be fp16 (or bf16)");
  TORCH_CHECK(seq_lens.dtype() == torch::kInt32, "seq_lens must be int32");
  TORCH_CHECK(key_cache_q8.dim() == 4, "key_cache_q8 must be 4D");
  TORCH_CHECK(value_cache.dim() == 4, "value_cache must be 4D");
  CHECK_CONTIG(key_cache_q8);
  CHECK_CONTIG(value_cache);
  const int NB = key_cache_q8.size(0), bs = key_cache_q8.size(1), Hkv = key_cache_q8.size(2);
  const int rb = key_cache_q8.size(3), D = value_cache.size(3);
  TORCH_CHECK(value_cache.size(0) == NB, "value_cache blocks mismatch");
  TORCH_CHECK(value_cache.size(1) == bs, "value_cache block_size mismatch");
  TORCH_CHECK(value_cache.size(2) == Hkv, "value_cache Hkv mismatch");
  TORCH_CHECK(D % 32 == 0, "D must be multiple of 32");
  TORCH_CHECK(rb == (D / 32) * 34, "bytes_per_row must equal (D/32)*34, got ", rb,
              " vs expected ", (D / 32) * 34);
  TORCH_CHECK(block_table.dtype() == torch::kInt32, "block_table must be int32 (caller should .to(torch.int32))");
  TORCH_CHECK(block_table.is_contiguous(), "block_table must be contiguous");
  TORCH_CHECK(seq_lens.is_contiguous(), "seq_lens must be contiguous");
  TORCH_CHECK(block_table.dim() == 2, "block_table must be [num_seqs, max_blocks]");
  const int B = block_table.size(0), MB = block_table.size(1);
  TORCH_CHECK(seq_lens.size(0) == B, "seq_lens vs block_table batch mismatch");
  TORCH_CHECK(Sk > 0 && (Sk % 32) == 0, "Sk must be positive multiple of 32, got ", Sk);
  auto use_or_alloc = [&](const c10::optional<torch::Tensor>& buf, at::TensorOptions opts,
                          int64_t last) -> torch::Tensor {
    if (buf.has_value()) {
      const auto& t = buf.value();
      if (t.dim() == 4 && t.size(0) == B && t.size(1) == Hkv && t.size(2) == Sk && t.size(3) == last &&
          t.dtype() == opts.dtype() && t.device() == opts.device() && t.is_contiguous())
        return t;
    }
    return torch::empty({(int64_t)B, (int64_t)Hkv, Sk, last}, opts);
  };
  auto k_out = use_or_alloc(k_out_opt, key_cache_q8.options(), rb);
  auto v_out = use_or_alloc(v_out_opt, value_cache.options(), D);
  c10::cuda::CUDAGuard g(key_cache_q8.device());
  check_status(gfx906_fa_gather_paged_kv_q8_checked(key_cache_q8.data_ptr<uint8_t>(), value_cache.data_ptr(),
                                         block_table.data_ptr<int32_t>(), seq_lens.data_ptr<int32_t>(),
                                         k_out.data_ptr<uint8_t>(), v_out.data_ptr(), B, Hkv, (int)Sk, D,
                                         rb, bs, MB, NB, (int64_t)bs * Hkv * rb, (int64_t)Hkv * rb, rb,
                                         (int64_t)bs * Hkv * D, (int64_t)Hkv * D, D, cur_stream()),
               "launch_gather_paged_kv_q8");
  return {k_out, v_out};
}

// ---------------------------------------------------------------------------
// store_kv: fused K (Q8_0) + V store by slot_mapping (new)
// ---------------------------------------------------------------------------
void store_kv(torch::Tensor key, torch::Tensor value, torch::Tensor slot_mapping, torch::Tensor k_cache,
              torch::Tensor v_cache, int64_t v_mode) {
  CHECK_CUDA(key);
  CHECK_CUDA(slot_mapping);
  CHECK_CUDA(k_cache);
  const int kdt = dtype_code(key, "key");
  TORCH_CHECK(key.dim() == 3 && key.stride(2) == 1, "key must be [T, Hkv, D] with contiguous D");
  TORCH_CHECK(slot_mapping.dtype() == torch::kInt64 && slot_mapping.dim() == 1, "slot_mapping must be int64 [T]");
  CHECK_CONTIG(slot_mapping);
  TORCH_CHECK(v_mode >= 0 && v_mode <= 3,
              "v_mode must be 0 (none), 1 (copy), 2 (q8_0 rows) or 3 (q8_0 page-transposed)");
  const int T = key.size(0), Hkv = key.size(1), D = key.size(2);
  TORCH_CHECK(slot_mapping.size(0) == T, "slot_mapping length mismatch");
  // k_cache / v_cache: 4-D [NB, bs, Hkv, row] views (any dtype) with byte strides
  TORCH_CHECK(k_cache.dim() == 4 && k_cache.size(2) == Hkv, "k_cache must be [NB, bs, Hkv, row]");
  const int bs = k_cache.size(1);
  const int64_t ke = k_cache.element_size();
  const void* vptr = nullptr;
  int vdt = G9_DT_F16;
  int64_t vts = 0, vhs = 0, vb0 = 0, vb1 = 0, vb2 = 0;
  uint8_t* vc = nullptr;
  if (v_mode != 0) {
    CHECK_CUDA(value);
    CHECK_CUDA(v_cache);
    vdt = dtype_code(value, "value");
    TORCH_CHECK(value.dim() == 3 && value.size(0) == T && value.size(1) == Hkv && value.size(2) == D &&
                    value.stride(2) == 1,
                "value must be [T, Hkv, D] with contiguous D");
    vptr = value.data_ptr();
    vts = value.stride(0);
    vhs = value.stride(1);
    const int64_t ve = v_cache.element_size();
    if (v_mode == G9_V_Q8T) {
      TORCH_CHECK(v_cache.dim() == 3 && v_cache.size(1) == Hkv && v_cache.dtype() == torch::kUInt8 &&
                      v_cache.size(2) == (int64_t)bs * (D / 32) * 34 && v_cache.stride(2) == 1,
                  "v_cache must be uint8 [NB, Hkv, block_size*(D/32)*34] page-transposed records");
      vb0 = v_cache.stride(0);
      vb2 = v_cache.stride(1);
    } else {
      TORCH_CHECK(v_cache.dim() == 4 && v_cache.size(1) == bs && v_cache.size(2) == Hkv,
                  "v_cache must be [NB, bs, Hkv, row]");
      vb0 = v_cache.stride(0) * ve;
      vb1 = v_cache.stride(1) * ve;
      vb2 = v_cache.stride(2) * ve;
    }
    vc = reinterpret_cast<uint8_t*>(v_cache.data_ptr());
  }
  c10::cuda::CUDAGuard g(key.device());
  check_status(gfx906_fa_store_kv(key.data_ptr(), kdt, key.stride(0), key.stride(1), vptr, vdt, vts, vhs,
                                  slot_mapping.data_ptr<int64_t>(), reinterpret_cast<uint8_t*>(k_cache.data_ptr()),
                                  k_cache.stride(0) * ke, k_cache.stride(1) * ke, k_cache.stride(2) * ke, vc, vb0,
                                  vb1, vb2, (int)v_mode, T, Hkv, D, bs, cur_stream()),
               "gfx906_fa_store_kv");
}

// ---------------------------------------------------------------------------
// rope_store_kv: fused RoPE (query and key rotated in place) + KV store (new)
// ---------------------------------------------------------------------------
void rope_store_kv(c10::optional<torch::Tensor> query, torch::Tensor key, torch::Tensor value,
                   torch::Tensor positions, torch::Tensor cos_sin_cache, bool is_neox, torch::Tensor slot_mapping,
                   torch::Tensor k_cache, torch::Tensor v_cache, int64_t v_mode) {
  CHECK_CUDA(key);
  CHECK_CUDA(positions);
  CHECK_CUDA(cos_sin_cache);
  CHECK_CUDA(slot_mapping);
  CHECK_CUDA(k_cache);
  const int kdt = dtype_code(key, "key");
  TORCH_CHECK(key.dim() == 3 && key.stride(2) == 1, "key must be [T, Hkv, D] with contiguous D");
  const int T = key.size(0), Hkv = key.size(1), D = key.size(2);
  TORCH_CHECK(D == 128, "head_size must be 128");
  TORCH_CHECK(positions.dtype() == torch::kInt64 && positions.dim() == 1 && positions.size(0) >= T &&
                  positions.is_contiguous(), "positions must be contiguous int64 [>= T]");
  TORCH_CHECK(slot_mapping.dtype() == torch::kInt64 && slot_mapping.dim() == 1 && slot_mapping.size(0) == T &&
                  slot_mapping.is_contiguous(), "slot_mapping must be contiguous int64 [T]");
  TORCH_CHECK(cos_sin_cache.dim() == 2 && cos_sin_cache.is_contiguous(), "cos_sin_cache must be [max_pos, rot_dim]");
  const int csdt = dtype_code(cos_sin_cache, "cos_sin_cache");
  const int rot = cos_sin_cache.size(1);
  TORCH_CHECK(rot == 32 || rot == 64 || rot == 128, "rot_dim must be 32, 64 or 128, got ", rot);
  TORCH_CHECK(v_mode >= 0 && v_mode <= 3, "v_mode must be 0..3");
  void* qptr = nullptr;
  int qdt = G9_DT_F16, Hq = 0;
  int64_t qts = 0, qhs = 0;
  if (query.has_value()) {
    auto q = query.value();
    CHECK_CUDA(q);
    TORCH_CHECK(q.dim() == 3 && q.size(0) >= T && q.size(2) == D && q.stride(2) == 1,
                "query must be [>= T, Hq, D] with contiguous D");
    qdt = dtype_code(q, "query");
    qptr = q.data_ptr();
    Hq = q.size(1);
    qts = q.stride(0);
    qhs = q.stride(1);
  }
  TORCH_CHECK(k_cache.dim() == 4 && k_cache.size(2) == Hkv, "k_cache must be [NB, bs, Hkv, row]");
  const int bs = k_cache.size(1);
  const int64_t ke = k_cache.element_size();
  const void* vptr = nullptr;
  int vdt = G9_DT_F16;
  int64_t vts = 0, vhs = 0, vb0 = 0, vb1 = 0, vb2 = 0;
  uint8_t* vc = nullptr;
  if (v_mode != 0) {
    CHECK_CUDA(value);
    CHECK_CUDA(v_cache);
    vdt = dtype_code(value, "value");
    TORCH_CHECK(value.dim() == 3 && value.size(0) == T && value.size(1) == Hkv && value.size(2) == D &&
                    value.stride(2) == 1, "value must be [T, Hkv, D] with contiguous D");
    vptr = value.data_ptr();
    vts = value.stride(0);
    vhs = value.stride(1);
    if (v_mode == G9_V_Q8T) {
      TORCH_CHECK(v_cache.dim() == 3 && v_cache.size(1) == Hkv && v_cache.dtype() == torch::kUInt8,
                  "v_cache must be uint8 [NB, Hkv, record]");
      vb0 = v_cache.stride(0);
      vb2 = v_cache.stride(1);
    } else {
      TORCH_CHECK(v_cache.dim() == 4 && v_cache.size(1) == bs && v_cache.size(2) == Hkv,
                  "v_cache must be [NB, bs, Hkv, row]");
      const int64_t ve = v_cache.element_size();
      vb0 = v_cache.stride(0) * ve;
      vb1 = v_cache.stride(1) * ve;
      vb2 = v_cache.stride(2) * ve;
    }
    vc = reinterpret_cast<uint8_t*>(v_cache.data_ptr());
  }
  c10::cuda::CUDAGuard g(key.device());
  check_status(gfx906_fa_rope_store_kv(qptr, qdt, qts, qhs, Hq, key.data_ptr(), kdt, key.stride(0), key.stride(1),
                                       vptr, vdt, vts, vhs, positions.data_ptr<int64_t>(), cos_sin_cache.data_ptr(),
                                       csdt, rot, is_neox ? 1 : 0, slot_mapping.data_ptr<int64_t>(),
                                       reinterpret_cast<uint8_t*>(k_cache.data_ptr()), k_cache.stride(0) * ke,
                                       k_cache.stride(1) * ke, k_cache.stride(2) * ke, vc, vb0, vb1, vb2,
                                       (int)v_mode, T, Hkv, D, bs, cur_stream()),
               "gfx906_fa_rope_store_kv");
}

// ---------------------------------------------------------------------------
// attention
// ---------------------------------------------------------------------------
G9AttnBatch batch_base(const torch::Tensor& key_cache_q8, const torch::Tensor& value_cache, int v_fmt,
                       const torch::Tensor& block_table, const torch::Tensor& kv_len) {
  G9AttnBatch b{};
  const int64_t ke = key_cache_q8.element_size();
  const int64_t ve = value_cache.element_size();
  b.k_cache = reinterpret_cast<const uint8_t*>(key_cache_q8.data_ptr());
  b.k_page_stride = key_cache_q8.stride(0) * ke;
  b.k_tok_stride = key_cache_q8.stride(1) * ke;
  b.k_head_stride = key_cache_q8.stride(2) * ke;
  b.v_cache = reinterpret_cast<const uint8_t*>(value_cache.data_ptr());
  if (v_fmt == G9_VFMT_Q8T) {           // [NB, Hkv, record] uint8
    b.v_page_stride = value_cache.stride(0);
    b.v_tok_stride = 0;
    b.v_head_stride = value_cache.stride(1);
  } else {
    b.v_page_stride = value_cache.stride(0) * ve;
    b.v_tok_stride = value_cache.stride(1) * ve;
    b.v_head_stride = value_cache.stride(2) * ve;
  }
  b.v_fmt = v_fmt;
  b.block_table = block_table.data_ptr<int32_t>();
  b.max_blocks = block_table.size(1);
  b.block_size = key_cache_q8.size(1);
  b.kv_len = kv_len.data_ptr<int32_t>();
  b.num_seqs = block_table.size(0);
  b.num_heads_kv = key_cache_q8.size(2);
  b.num_blocks = key_cache_q8.size(0);      // entries past the cache are flagged, never read
  return b;
}

// Optional score features (not in the reference ops): logit soft-cap,
// sliding window, per-query-head sinks.  `sinks_c` keeps a contiguous fp32
// copy alive for the launch.
void set_features(G9AttnBatch& b, int64_t Hq, double softcap, int64_t window, c10::optional<torch::Tensor>& sinks,
                  torch::Tensor& sinks_c, const torch::Tensor& like) {
  TORCH_CHECK(softcap >= 0.0, "softcap must be >= 0 (0 disables it)");
  TORCH_CHECK(window >= 0, "sliding_window must be >= 0 (0 disables it)");
  b.softcap = (float)softcap;
  b.window = (int)window;
  if (sinks.has_value()) {
    auto s = sinks.value();
    CHECK_CUDA(s);
    TORCH_CHECK(s.dim() == 1 && s.size(0) == Hq, "sinks must be [num_heads_q]");
    TORCH_CHECK(s.device() == like.device(), "sinks must be on the query's device");
    sinks_c = s.to(torch::kFloat32).contiguous();
    b.sinks = sinks_c.data_ptr<float>();
  }
}

// 4-D caches hold token rows; a 3-D uint8 [NB, Hkv, record] cache holds
// page-transposed Q8_0 records (G9_VFMT_Q8T).
int infer_v_fmt(const torch::Tensor& value_cache, int64_t D) {
  if (value_cache.dim() == 3) {
    TORCH_CHECK(value_cache.dtype() == torch::kUInt8, "a 3-D value_cache must be uint8 page-transposed Q8_0");
    return G9_VFMT_Q8T;
  }
  if (value_cache.dtype() == torch::kUInt8) {
    TORCH_CHECK(value_cache.size(3) == (D / 32) * 34, "Q8_0 value_cache last dim must be (D/32)*34");
    return G9_VFMT_Q8;
  }
  TORCH_CHECK(value_cache.size(3) == D, "value_cache D mismatch q D");
  if (value_cache.dtype() == torch::kFloat16) return G9_VFMT_F16;
  TORCH_CHECK(value_cache.dtype() == torch::kBFloat16, "value_cache must be fp16, bf16 or uint8 (Q8_0)");
  return G9_VFMT_BF16;
}

void check_paged(const torch::Tensor& key_cache_q8, const torch::Tensor& value_cache,
                 const torch::Tensor& block_table, const torch::Tensor& seq_lens, int64_t D, int64_t B) {
  CHECK_CUDA(key_cache_q8);
  CHECK_CUDA(value_cache);
  CHECK_CUDA(block_table);
  CHECK_CUDA(seq_lens);
  TORCH_CHECK(key_cache_q8.dtype() == torch::kUInt8, "key_cache_q8 must be uint8");
  TORCH_CHECK(block_table.dtype() == torch::kInt32, "block_table must be int32");
  TORCH_CHECK(seq_lens.dtype() == torch::kInt32, "seq_lens must be int32");
  TORCH_CHECK(key_cache_q8.dim() == 4, "key_cache_q8 must be [num_blocks, block_size, Hkv, bytes_per_row]");
  TORCH_CHECK(D == 128, "head_dim must be 128");
  TORCH_CHECK(key_cache_q8.size(3) == (D / 32) * 34, "bytes_per_row must equal (D/32)*34");
  TORCH_CHECK(value_cache.size(0) == key_cache_q8.size(0), "value_cache blocks mismatch");
  if (value_cache.dim() == 3) {
    TORCH_CHECK(value_cache.size(1) == key_cache_q8.size(2), "value_cache Hkv mismatch");
    TORCH_CHECK(value_cache.size(2) == key_cache_q8.size(1) * key_cache_q8.size(3) && value_cache.stride(2) == 1,
                "page-transposed value_cache must be [num_blocks, Hkv, block_size*(D/32)*34]");
  } else {
    TORCH_CHECK(value_cache.dim() == 4, "value_cache must be [num_blocks, block_size, Hkv, D]");
    TORCH_CHECK(value_cache.size(1) == key_cache_q8.size(1), "value_cache block_size mismatch");
    TORCH_CHECK(value_cache.size(2) == key_cache_q8.size(2), "value_cache Hkv mismatch");
    TORCH_CHECK(value_cache.stride(3) == 1, "cache rows must be contiguous");
  }
  TORCH_CHECK(key_cache_q8.stride(3) == 1, "cache rows must be contiguous");
  TORCH_CHECK(block_table.dim() == 2 && block_table.size(0) == B, "block_table[0] must equal batch");
  TORCH_CHECK(seq_lens.dim() == 1 && seq_lens.size(0) == B, "seq_lens must be [batch]");
  TORCH_CHECK(block_table.is_contiguous() && seq_lens.is_contiguous(), "block_table / seq_lens must be contiguous");
}

// Runs one batch through gfx906_fa_attention (decode and/or tensor-core
// prefill), workspace from the caching allocator.
void run_attention(G9AttnBatch& b, const torch::Tensor& like, const int* nq_host = nullptr,
                   const int* kv_host = nullptr) {
  const size_t ws = gfx906_fa_attention_workspace_size(&b, nq_host, kv_host);
  TORCH_CHECK(ws > 0, "attention: unsupported shape");
  auto wsbuf = torch::empty({(int64_t)ws}, like.options().dtype(torch::kUInt8));
  check_status(gfx906_fa_attention(&b, nq_host, kv_host, wsbuf.data_ptr(), ws, cur_stream()),
               "gfx906_fa_attention");
}

void set_mask_qabs(G9AttnBatch& b, int64_t B, int64_t Sq, int64_t min_cols, c10::optional<torch::Tensor>& mask,
                   c10::optional<torch::Tensor>& q_abs_offset, torch::Tensor& mask_c, torch::Tensor& qo_c) {
  TORCH_CHECK(!(mask.has_value() && q_abs_offset.has_value()),
              "q_abs_offset and mask are mutually exclusive (inline causal replaces mask)");
  if (mask.has_value()) {
    auto m = mask.value();
    CHECK_CUDA(m);
    TORCH_CHECK(m.dtype() == torch::kFloat16, "mask must be fp16");
    TORCH_CHECK(m.dim() == 3 && m.size(0) == B && m.size(1) == Sq, "mask must be [B, Sq, Skv_pad]");
    TORCH_CHECK(m.size(2) >= min_cols, "mask.size(2) must cover every key (", min_cols, ")");
    mask_c = m.contiguous();
    b.mask = mask_c.data_ptr();
    b.mask_seq_stride = mask_c.size(1) * mask_c.size(2);
    b.mask_tok_stride = mask_c.size(2);
  }
  if (q_abs_offset.has_value()) {
    auto qo = q_abs_offset.value();
    CHECK_CUDA(qo);
    TORCH_CHECK(qo.dtype() == torch::kInt32 && qo.dim() == 1 && qo.size(0) == B, "q_abs_offset must be int32 [B]");
    qo_c = qo.contiguous();
    b.q_abs = qo_c.data_ptr<int32_t>();
  }
}

// forward (extension/gfx906_fa.cpp:120-265): q [B, Hq, Sq, D], k_q8
// [B, Hkv, Skv, D/32*34], v [B, Hkv, Skv, D] -> fp32 [B, Hq, Sq, D].
// kv_max int32 [B], mask fp16 [B, Sq, >=Skv], q_abs_offset int32 [B].
torch::Tensor forward(torch::Tensor q, torch::Tensor k_q8, torch::Tensor v, double scale,
                      c10::optional<torch::Tensor> kv_max, c10::optional<torch::Tensor> mask,
                      c10::optional<torch::Tensor> q_abs_offset, double softcap, int64_t sliding_window,
                      c10::optional<torch::Tensor> sinks) {
  CHECK_CUDA(q);
  CHECK_CUDA(k_q8);
  CHECK_CUDA(v);
  CHECK_CONTIG(q);
  CHECK_CONTIG(k_q8);
  CHECK_CONTIG(v);
  const int qdt = dtype_code(q, "q");
  TORCH_CHECK(k_q8.dtype() == torch::kUInt8, "k_q8 must be uint8 (block_q8_0 bytes)");
  TORCH_CHECK(q.dim() == 4, "q must be 4D [B, Hq, Sq, D]");
  TORCH_CHECK(v.dim() == 4, "v_fp16 must be 4D [B, Hkv, Skv, D]");
  const int64_t B = q.size(0), Hq = q.size(1), Sq = q.size(2), D = q.size(3);
  const int64_t Hkv = v.size(1), Skv = v.size(2);
  TORCH_CHECK(v.size(0) == B, "v batch mismatch");
  TORCH_CHECK(D % 32 == 0, "head_dim must be multiple of 32");
  TORCH_CHECK(D == 128, "head_dim must be 128");
  TORCH_CHECK(k_q8.dim() == 4 && k_q8.size(0) == B && k_q8.size(1) == Hkv && k_q8.size(2) == Skv,
              "k_q8 first 3 dims must match [B, Hkv, Skv]");
  TORCH_CHECK(k_q8.size(3) == (D / 32) * 34, "k_q8 last dim = (D/32)*34 bytes");
  TORCH_CHECK(Hq % Hkv == 0, "heads_q must be divisible by heads_kv");
  const int vfmt = infer_v_fmt(v, D);
  auto out = torch::empty({B, Hq, Sq, D}, q.options().dtype(torch::kFloat32));
  if (B == 0 || Sq == 0) return out;
  c10::cuda::CUDAGuard g(q.device());
  const int64_t rb = (D / 32) * 34, vrow = v.size(3) * v.element_size();
  auto ids = torch::arange(B, q.options().dtype(torch::kInt32)).view({B, 1});
  torch::Tensor kvl;
  if (kv_max.has_value()) {
    auto kvm = kv_max.value();
    CHECK_CUDA(kvm);
    TORCH_CHECK(kvm.dtype() == torch::kInt32, "kv_max must be int32");
    TORCH_CHECK(kvm.dim() == 1 && kvm.size(0) == B, "kv_max must be 1D [B]");
    kvl = kvm.clamp(0, Skv).to(torch::kInt32).contiguous();
  } else {
    kvl = torch::full({B}, Skv, q.options().dtype(torch::kInt32));
  }
  G9AttnBatch b{};
  b.q = q.data_ptr();
  b.q_dtype = qdt;
  b.q_seq_stride = Hq * Sq * D;
  b.q_tok_stride = D;
  b.q_head_stride = Sq * D;
  b.seq_q = Sq;
  b.out = out.data_ptr();
  b.out_dtype = G9_DT_F32;
  b.o_seq_stride = Hq * Sq * D;
  b.o_tok_stride = D;
  b.o_head_stride = Sq * D;
  b.k_cache = k_q8.data_ptr<uint8_t>();
  b.k_page_stride = Hkv * Skv * rb;
  b.k_tok_stride = rb;
  b.k_head_stride = Skv * rb;
  b.v_cache = reinterpret_cast<const uint8_t*>(v.data_ptr());
  b.v_page_stride = Hkv * Skv * vrow;
  b.v_tok_stride = vrow;
  b.v_head_stride = Skv * vrow;
  b.v_fmt = vfmt;
  b.block_table = ids.data_ptr<int32_t>();
  b.max_blocks = 1;
  b.block_size = std::max<int64_t>(Skv, 1);
  b.kv_len = kvl.data_ptr<int32_t>();
  b.max_kv = Skv;
  b.num_seqs = B;
  b.num_heads_q = Hq;
  b.num_heads_kv = Hkv;
  b.head_dim = D;
  b.scale = (float)scale;
  torch::Tensor mask_c, qo_c, sinks_c;
  set_mask_qabs(b, B, Sq, Skv, mask, q_abs_offset, mask_c, qo_c);
  set_features(b, Hq, softcap, sliding_window, sinks, sinks_c, q);
  // contiguous [B, Hkv, Skv, row] tensors are not 16-token pages: the batch
  // goes to the tensor-core path, whose pack step reads any row layout
  run_attention(b, q);
  return out;
}

// forward_paged_direct (extension/gfx906_fa.cpp:516-658): q [B, Hq, Sq, D]
// (fp32 as in the reference; fp16 / bf16 also accepted) -> fp32 [B, Hq, Sq, D].
torch::Tensor forward_paged_direct(torch::Tensor q, torch::Tensor key_cache_q8, torch::Tensor value_cache,
                                   torch::Tensor block_table, torch::Tensor seq_lens, double scale,
                                   c10::optional<torch::Tensor> mask, c10::optional<torch::Tensor> q_abs_offset,
                                   double softcap, int64_t sliding_window, c10::optional<torch::Tensor> sinks) {
  CHECK_CUDA(q);
  CHECK_CONTIG(q);
  TORCH_CHECK(q.dim() == 4, "q must be 4D [B, Hq, Sq, D]");
  const int qdt = dtype_code(q, "q");
  const int64_t B = q.size(0), Hq = q.size(1), Sq = q.size(2), D = q.size(3);
  check_paged(key_cache_q8, value_cache, block_table, seq_lens, D, B);
  const int vfmt = infer_v_fmt(value_cache, D);
  TORCH_CHECK(key_cache_q8.size(1) == 16, "Only block_size=16 supported, got ", key_cache_q8.size(1));
  TORCH_CHECK(Hq % key_cache_q8.size(2) == 0, "heads_q must be divisible by heads_kv");
  auto out = torch::empty({B, Hq, Sq, D}, q.options().dtype(torch::kFloat32));
  if (B == 0 || Sq == 0) return out;
  c10::cuda::CUDAGuard g(q.device());
  G9AttnBatch b = batch_base(key_cache_q8, value_cache, vfmt, block_table, seq_lens);
  b.q = q.data_ptr();
  b.q_dtype = qdt;
  b.q_seq_stride = Hq * Sq * D;
  b.q_tok_stride = D;
  b.q_head_stride = Sq * D;
  b.seq_q = Sq;
  b.out = out.data_ptr();
  b.out_dtype = G9_DT_F32;
  b.o_seq_stride = Hq * Sq * D;
  b.o_tok_stride = D;
  b.o_head_stride = Sq * D;
  b.max_kv = b.max_blocks * b.block_size;
  b.num_heads_q = Hq;
  b.head_dim = D;
  b.scale = (float)scale;
  torch::Tensor mask_c, qo_c, sinks_c;
  set_mask_qabs(b, B, Sq, b.max_kv, mask, q_abs_offset, mask_c, qo_c);
  set_features(b, Hq, softcap, sliding_window, sinks, sinks_c, q);
  // Sequences of Sq*G rows above the decode kernel's cap take the prefill
  // kernel, whose staging grows with each sequence's visible keys: size it
  // from the actual lengths (one host read of seq_lens) rather than bounding
  // every sequence by max_blocks * block_size.
  if (Sq * (Hq / key_cache_q8.size(2)) > 24) {
    auto sl_host = seq_lens.to(torch::kCPU);
    std::vector<int> nqh(B, (int)Sq), kvh(B);
    for (int64_t i = 0; i < B; ++i)
      kvh[i] = std::max(0, std::min<int>(sl_host.data_ptr<int32_t>()[i], b.max_kv));
    run_attention(b, q, nqh.data(), kvh.data());
  } else {
    run_attention(b, q);
  }
  return out;
}

// paged_attention: vLLM-layout entry.  query [T, Hq, D] (fp16/bf16/fp32),
// caches as [NB, bs, Hkv, row] views (any strides with contiguous rows),
// query_start_loc int32 [B+1], seq_lens int32 [B].  Causal with
// q_abs = seq_len - n_q (vLLM's chunked-prefill convention).  Writes `out`
// [T, Hq, D] (allocated in the query dtype when not given).  Optional host
// lists give exact query lengths / context-length bounds for routing.
torch::Tensor paged_attention(torch::Tensor query, torch::Tensor key_cache_q8, torch::Tensor value_cache,
                              torch::Tensor block_table, torch::Tensor seq_lens, torch::Tensor query_start_loc,
                              int64_t max_query_len, int64_t max_seq_len, double scale,
                              c10::optional<torch::Tensor> out_opt,
                              c10::optional<std::vector<int64_t>> query_lens_host,
                              c10::optional<std::vector<int64_t>> seq_lens_host, double softcap,
                              int64_t sliding_window, c10::optional<torch::Tensor> sinks,
                              c10::optional<torch::Tensor> output_scale) {
  CHECK_CUDA(query);
  CHECK_CUDA(query_start_loc);
  TORCH_CHECK(query.dim() == 3 && query.stride(2) == 1, "query must be [T, Hq, D] with contiguous D");
  const int qdt = dtype_code(query, "query");
  const int64_t T = query.size(0), Hq = query.size(1), D = query.size(2);
  const int64_t B = block_table.size(0);
  check_paged(key_cache_q8, value_cache, block_table, seq_lens, D, B);
  TORCH_CHECK(query_start_loc.dtype() == torch::kInt32 && query_start_loc.dim() == 1 &&
                  query_start_loc.size(0) == B + 1 && query_start_loc.is_contiguous(),
              "query_start_loc must be int32 [B+1]");
  TORCH_CHECK(Hq % key_cache_q8.size(2) == 0, "heads_q must be divisible by heads_kv");
  const int vfmt = infer_v_fmt(value_cache, D);
  torch::Tensor out;
  if (out_opt.has_value()) {
    out = out_opt.value();
    CHECK_CUDA(out);
    TORCH_CHECK(out.dim() == 3 && out.size(0) >= T && out.size(1) == Hq && out.size(2) == D && out.stride(2) == 1,
                "out must be [>=T, Hq, D] with contiguous D");
    TORCH_CHECK(out.device() == query.device(), "out must be on the query's device");
  } else {
    out = torch::empty({T, Hq, D}, query.options());
  }
  if (B == 0 || T == 0) return out;
  c10::cuda::CUDAGuard g(query.device());
  G9AttnBatch b = batch_base(key_cache_q8, value_cache, vfmt, block_table, seq_lens);
  b.q = query.data_ptr();
  b.q_dtype = qdt;
  b.q_tok_stride = query.stride(0);
  b.q_head_stride = query.stride(1);
  // n_q and the causal offsets (q_abs = seq_len - n_q) are derived in the
  // kernels from query_start_loc and seq_lens: no extra launches
  b.q_start = query_start_loc.data_ptr<int32_t>();
  b.flags = G9_F_CU_SEQLENS | G9_F_CAUSAL_END;
  b.seq_q = (int)max_query_len;
  b.out = out.data_ptr();
  torch::Tensor oscale_c;
  if (out.scalar_type() == torch::kFloat8_e4m3fn) {
    // vLLM's static per-tensor fp8 output quantisation: out = e4m3(o / scale)
    TORCH_CHECK(output_scale.has_value(), "an fp8 (e4m3) out needs output_scale");
    oscale_c = output_scale.value().to(torch::kFloat32).reshape({-1}).contiguous();
    TORCH_CHECK(oscale_c.numel() == 1 && oscale_c.device() == query.device(),
                "output_scale must be one fp32 value on the query's device");
    b.out_dtype = G9_DT_FP8E4M3;
    b.out_scale = oscale_c.data_ptr<float>();
  } else {
    TORCH_CHECK(!output_scale.has_value(), "output_scale applies to an fp8 (e4m3) out only");
    b.out_dtype = dtype_code(out, "out");
  }
  b.o_tok_stride = out.stride(0);
  b.o_head_stride = out.stride(1);
  b.max_kv = (int)max_seq_len;
  b.num_heads_q = Hq;
  b.head_dim = D;
  b.scale = (float)scale;
  std::vector<int> nqh, kvh;
  if (query_lens_host.has_value()) {
    TORCH_CHECK((int64_t)query_lens_host->size() == B, "query_lens_host must have num_seqs entries");
    for (auto x : *query_lens_host) nqh.push_back((int)x);
  }
  if (seq_lens_host.has_value()) {
    TORCH_CHECK((int64_t)seq_lens_host->size() == B, "seq_lens_host must have num_seqs entries");
    for (auto x : *seq_lens_host) kvh.push_back((int)x);
  }
  torch::Tensor sinks_c;
  set_features(b, Hq, softcap, sliding_window, sinks, sinks_c, query);
  run_attention(b, query, nqh.empty() ? nullptr : nqh.data(), kvh.empty() ? nullptr : kvh.data());
  return out;
}

unsigned int device_error(bool clear) {
  unsigned int v = 0;
  check_status(gfx906_fa_get_device_error(&v), "gfx906_fa_get_device_error");
  if (clear) check_status(gfx906_fa_clear_device_error(), "gfx906_fa_clear_device_error");
  return v;
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "gfx906_fa on sm_100a: paged Q8_0 KV store, page gather and flash attention";
  m.def("quantize_q8_0", &quantize_q8_0,
        "Quantize a tensor (last dim D) to block_q8_0 uint8 [..., D/32*34] on the device",
        py::arg("k_fp16"));
  m.def("reshape_and_cache_q8", &reshape_and_cache_q8,
        "Quantize new K tokens and scatter them into the paged Q8 cache by slot_mapping (in place)",
        py::arg("key"), py::arg("slot_mapping"), py::arg("k_cache_q8"));
  m.def("gather_paged_kv_q8", &gather_paged_kv_q8,
        "Paged K_q8 + paged V -> contiguous BHSD; returns [k_out, v_out]. V tail zeroed per seq_lens; "
        "K tail left unwritten. k_out/v_out reused when their shape matches exactly.",
        py::arg("key_cache_q8"), py::arg("value_cache"), py::arg("block_table"), py::arg("seq_lens"),
        py::arg("Sk"), py::arg("k_out") = c10::nullopt, py::arg("v_out") = c10::nullopt);
  m.def("store_kv", &store_kv,
        "Fused KV store by slot_mapping: K -> Q8_0, V copied (v_mode=1) or quantized (v_mode=2)",
        py::arg("key"), py::arg("value"), py::arg("slot_mapping"), py::arg("k_cache"), py::arg("v_cache"),
        py::arg("v_mode") = 1);
  m.def("rope_store_kv", &rope_store_kv,
        "Fused RoPE + KV store: query / key rotated in place (fp32, rounded once), K -> Q8_0, V per v_mode, "
        "by slot_mapping",
        py::arg("query"), py::arg("key"), py::arg("value"), py::arg("positions"), py::arg("cos_sin_cache"),
        py::arg("is_neox"), py::arg("slot_mapping"), py::arg("k_cache"), py::arg("v_cache"), py::arg("v_mode") = 1);
  m.def("forward", &forward, "FA forward (Q fp32/fp16/bf16, K q8_0, V fp16): fp32 [B, Hq, Sq, D]",
        py::arg("q"), py::arg("k_q8"), py::arg("v_fp16"), py::arg("scale"), py::arg("kv_max") = c10::nullopt,
        py::arg("mask") = c10::nullopt, py::arg("q_abs_offset") = c10::nullopt, py::arg("softcap") = 0.0,
        py::arg("sliding_window") = 0, py::arg("sinks") = c10::nullopt);
  m.def("forward_paged_direct", &forward_paged_direct,
        "Direct-paged flash attention (no gather): q [B, Hq, Sq, D] -> fp32 [B, Hq, Sq, D]",
        py::arg("q"), py::arg("key_cache_q8"), py::arg("value_cache"), py::arg("block_table"),
        py::arg("seq_lens"), py::arg("scale"), py::arg("mask") = c10::nullopt,
        py::arg("q_abs_offset") = c10::nullopt, py::arg("softcap") = 0.0, py::arg("sliding_window") = 0,
        py::arg("sinks") = c10::nullopt);
  m.def("paged_attention", &paged_attention,
        "Varlen causal paged attention in vLLM layout: query [T, Hq, D] -> out [T, Hq, D]",
        py::arg("query"), py::arg("key_cache_q8"), py::arg("value_cache"), py::arg("block_table"),
        py::arg("seq_lens"), py::arg("query_start_loc"), py::arg("max_query_len"), py::arg("max_seq_len"),
        py::arg("scale"), py::arg("out") = c10::nullopt, py::arg("query_lens_host") = c10::nullopt,
        py::arg("seq_lens_host") = c10::nullopt, py::arg("softcap") = 0.0, py::arg("sliding_window") = 0,
        py::arg("sinks") = c10::nullopt, py::arg("output_scale") = c10::nullopt);
  m.def("device_error", &device_error, "Read (and optionally clear) the library's device error word",
        py::arg("clear") = false);
}
