"""vLLM plugin surface, checked without a GPU (reference: tests/test_backend.py
test_registration / test_kv_cache_shape_compat, extension/setup.py:55-60)."""
import os

import pytest

from _util import ROOT

PKG = os.path.join(ROOT, "gfx906-fa-vllm_b200")


def _backend():
    pytest.importorskip("vllm")
    if not os.path.exists(os.path.join(PKG, "gfx906_fa.so")):
        pytest.skip("extension not built")
    import gfx906_fa_backend
    return gfx906_fa_backend


def test_registration():
    be = _backend()
    from vllm.v1.attention.backends.registry import AttentionBackendEnum
    assert AttentionBackendEnum.CUSTOM.get_class() is be.Gfx906FABackend
    assert be.Gfx906FABackend.get_name() == "CUSTOM"


def test_kv_cache_shape_matches_triton():
    be = _backend()
    from vllm.v1.attention.backends.triton_attn import TritonAttentionBackend
    for args in [(128, 16, 8, 128, "auto"), (7, 32, 1, 128, "auto")]:
        assert be.Gfx906FABackend.get_kv_cache_shape(*args) == TritonAttentionBackend.get_kv_cache_shape(*args)
    with pytest.raises(ValueError):
        be.Gfx906FABackend.get_kv_cache_shape(8, 24, 8, 128)


def test_backend_flags():
    be = _backend()
    B = be.Gfx906FABackend
    assert B.accept_output_buffer is True
    assert B.forward_includes_kv_cache_update is False
    assert B.supports_block_size(16) and B.supports_block_size(32) and not B.supports_block_size(8)
    assert B.supports_head_size(128) and not B.supports_head_size(64)


def test_impl_rejects_unsupported_features():
    be = _backend()
    kw = dict(num_heads=8, head_size=128, scale=0.1, num_kv_heads=2, alibi_slopes=None,
              sliding_window=None, kv_cache_dtype="auto")
    be.Gfx906FAImpl(**kw)
    for bad in (dict(alibi_slopes=[1.0] * 8), dict(head_size=64)):
        with pytest.raises(NotImplementedError):
            be.Gfx906FAImpl(**{**kw, **bad})
    # malformed feature arguments are rejected, not ignored
    import torch
    for bad in (dict(sliding_window=-4), dict(sinks=torch.zeros(3))):
        with pytest.raises(ValueError):
            be.Gfx906FAImpl(**{**kw, **bad})


def test_impl_accepts_window_softcap_sinks():
    """Sliding window, logit soft-cap and sinks are computed by the kernels
    (the reference backend rejected them, extension/gfx906_fa_backend.py:249-254)."""
    be = _backend()
    import torch
    impl = be.Gfx906FAImpl(num_heads=8, head_size=128, scale=0.1, num_kv_heads=2, alibi_slopes=None,
                           sliding_window=4096, kv_cache_dtype="auto", logits_soft_cap=30.0,
                           sinks=torch.zeros(8, dtype=torch.bfloat16))
    assert impl.sliding_window == 4096 and impl.logits_soft_cap == 30.0
    assert impl._sinks_f32().dtype == torch.float32
    assert be.Gfx906FABackend.supports_sink()


def test_kv_cache_views_layout():
    """Q8_0 K rows are packed densely at the start of each page's K half."""
    be = _backend()
    import torch
    kv = torch.zeros((3, 2, 16, 8, 128), dtype=torch.float16)
    k_q8, v = be.kv_cache_views(kv)
    assert tuple(k_q8.shape) == (3, 16, 8, 136) and k_q8.dtype == torch.uint8
    assert k_q8.stride() == (2 * 16 * 8 * 256, 8 * 136, 136, 1)
    k_q8[1, 0, 0, 0] = 7
    assert kv.view(torch.uint8).view(3, 2, -1)[1, 0, 0] == 7
    assert v.data_ptr() == kv[:, 1].data_ptr()
    k2, v2 = be.kv_cache_views(kv, "q8_0")
    # page-transposed Q8_0 V: one record of 16*136 bytes per (page, kv head),
    # right after the page's K rows (K and V of a page are one byte range)
    assert v2.dtype == torch.uint8 and tuple(v2.shape) == (3, 8, 16 * 136)
    assert v2.stride() == (2 * 16 * 8 * 256, 16 * 136, 1)
    assert v2.data_ptr() == k2.data_ptr() + 16 * 8 * 136
    v2[2, 1, 0] = 9
    assert kv.view(torch.uint8).view(3, -1)[2, 16 * 8 * 136 + 16 * 136] == 9


def test_entry_point_declared():
    src = open(os.path.join(PKG, "setup.py")).read()
    assert "vllm.general_plugins" in src and "gfx906_fa = gfx906_fa_backend:register" in src


def test_graph_support_and_fused_output_quant_flags():
    """Pure decode steps may be captured in CUDA graphs; static per-tensor
    fp8 output quantisation is fused (the reference declared neither)."""
    be = _backend()
    from vllm.v1.attention.backend import AttentionCGSupport
    from vllm.model_executor.layers.quantization.utils.quant_utils import kFp8StaticTensorSym
    assert be.Gfx906FAMetadataBuilder._cudagraph_support == AttentionCGSupport.UNIFORM_SINGLE_TOKEN_DECODE
    impl = be.Gfx906FAImpl(num_heads=8, head_size=128, scale=0.1, num_kv_heads=2, alibi_slopes=None,
                           sliding_window=None, kv_cache_dtype="auto")
    assert impl.fused_output_quant_supported(kFp8StaticTensorSym)
    assert impl.fused_rope_kvcache_supported()
    impl._legacy = True
    assert not impl.fused_output_quant_supported(kFp8StaticTensorSym)
    assert not impl.fused_rope_kvcache_supported()
