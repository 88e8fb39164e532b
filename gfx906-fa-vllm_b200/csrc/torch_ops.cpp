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
  check_status(launch_gather_paged_kv_q8(key_cache_q8.data_ptr<uint8_t>(), value_cache.data_ptr(),
                                         block_table.data_ptr<int32_t>(), seq_lens.data_ptr<int32_t>(),
                                         k_out.data_ptr<uint8_t>(), v_out.data_ptr(), B, Hkv, (int)Sk, D,
                                         rb, bs, MB, (int64_t)bs * Hkv * rb, (int64_t)Hkv * rb, rb,
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
  TORCH_CHECK(v_mode >= 0 && v_mode <= 2, "v_mode must be 0 (none), 1 (copy) or 2 (q8_0)");
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
    TORCH_CHECK(v_cache.dim() == 4 && v_cache.size(1) == bs && v_cache.size(2) == Hkv,
                "v_cache must be [NB, bs, Hkv, row]");
    vptr = value.data_ptr();
    vts = value.stride(0);
    vhs = value.stride(1);
    const int64_t ve = v_cache.element_size();
    vb0 = v_cache.stride(0) * ve;
    vb1 = v_cache.stride(1) * ve;
    vb2 = v_cache.stride(2) * ve;
    vc = reinterpret_cast<uint8_t*>(v_cache.data_ptr());
  }
  c10::cuda::CUDAGuard g(key.device());
  check_status(gfx906_fa_store_kv(key.data_ptr(), kdt, key.stride(0), key.stride(1), vptr, vdt, vts, vhs,
                                  slot_mapping.data_ptr<int64_t>(), reinterpret_cast<uint8_t*>(k_cache.data_ptr()),
                                  k_cache.stride(0) * ke, k_cache.stride(1) * ke, k_cache.stride(2) * ke, vc, vb0,
                                  vb1, vb2, (int)v_mode, T, Hkv, D, bs, cur_stream()),
               "gfx906_fa_store_kv");
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
  m.def("device_error", &device_error, "Read (and optionally clear) the library's device error word",
        py::arg("clear") = false);
}
