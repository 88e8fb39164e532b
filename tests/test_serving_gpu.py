"""Serving-side features of the vLLM backend path on the GPU: fp8 (e4m3)
output quantisation fused into the attention epilogues (vLLM's static
per-tensor output scale; the reference refuses output quantisation,
extension/gfx906_fa_backend.py:293-294) and CUDA-graph capture of pure
decode steps (the reference builder declares no graph support,
extension/gfx906_fa_backend.py:72-109), both against the fp32 oracle."""
import numpy as np
import pytest
import torch

from _paged import ATOL, RTOL, PagedCase, assert_close
from _util import to_np

pytestmark = pytest.mark.gpu
dev = "cuda"


def _gfx():
    import gfx906_fa
    return gfx906_fa


def _cu(nq):
    return torch.tensor(np.concatenate([[0], np.cumsum(nq)]), dtype=torch.int32)


def _e4m3_step(x):
    """Spacing of e4m3 values at |x| (3 mantissa bits; subnormal step 2^-9)."""
    ax = np.maximum(np.abs(x), 2.0 ** -6)
    return 2.0 ** (np.floor(np.log2(ax)) - 3)


@pytest.mark.parametrize("v_fmt", ["q8t", "f16"])
def test_fp8_output_quantisation(v_fmt):
    """Decode (split-K and whole rows), verify rows and a prefill chunk write
    e4m3(o / scale); each element is within the attention tolerance plus one
    e4m3 step of the oracle's value divided by the scale."""
    g = _gfx()
    lens, nq = [3000, 700, 900, 40], [1, 4, 300, 1]
    case = PagedCase(lens, 8, v_fmt=v_fmt, seed=71)
    gq = torch.Generator().manual_seed(72)
    q = torch.randn((sum(nq), 48, 128), generator=gq).to(torch.bfloat16)
    s = 0.01
    out = torch.full((sum(nq), 48, 128), 0, dtype=torch.float8_e4m3fn, device=dev)
    g.paged_attention(q.to(dev), case.k_cache, case.v_cache, case.block_table.to(dev),
                      torch.from_numpy(case.seq_lens).to(dev), _cu(nq).to(dev), max(nq), max(lens), case.scale,
                      out=out, output_scale=torch.tensor([s], device=dev), query_lens_host=nq, seq_lens_host=lens)
    got = out.float().cpu().numpy()
    ref = case.oracle_varlen(to_np(q), "bf16", nq)
    err = np.abs(got * s - ref)
    bound = ATOL + RTOL * np.abs(ref) + s * _e4m3_step(ref / s)
    assert (err <= bound).all(), f"{int((err > bound).sum())} fp8 outputs out of bound, max err {err.max():.3e}"
    # saturation: a scale that pushes |o| / scale past 448 clamps instead of overflowing
    g.paged_attention(q.to(dev), case.k_cache, case.v_cache, case.block_table.to(dev),
                      torch.from_numpy(case.seq_lens).to(dev), _cu(nq).to(dev), max(nq), max(lens), case.scale,
                      out=out, output_scale=torch.tensor([1e-4], device=dev), query_lens_host=nq, seq_lens_host=lens)
    o = out.float().cpu().numpy()
    assert np.isfinite(o).all() and np.abs(o).max() <= 448.0


def test_fp8_output_needs_scale():
    g = _gfx()
    case = PagedCase([100], 8, seed=73)
    q = torch.randn((1, 48, 128), device=dev, dtype=torch.bfloat16)
    out = torch.empty((1, 48, 128), dtype=torch.float8_e4m3fn, device=dev)
    with pytest.raises(RuntimeError):
        g.paged_attention(q, case.k_cache, case.v_cache, case.block_table.to(dev),
                          torch.from_numpy(case.seq_lens).to(dev), _cu([1]).to(dev), 1, 100, case.scale, out=out)


@pytest.mark.parametrize("v_fmt", ["q8_0", "fp16"])
def test_impl_decode_in_cuda_graph(v_fmt):
    """Capture Gfx906FAImpl.forward for a 16-sequence decode batch with the
    metadata the builder makes for capture, then replay it after rewriting
    the lengths (longer and shorter than at capture) and the query in the
    persistent buffers, as vLLM does between steps."""
    pytest.importorskip("vllm")
    import oracle as O
    import gfx906_fa_backend as be
    from test_paged_gpu import _FakeLayer, _Hist
    B, Hq, Hkv, D, BS = 16, 48, 8, 128, 16
    full = [int(x) for x in np.random.default_rng(5).integers(100, 6000, size=B)]
    h = _Hist(full, Hkv, seed=74, dtype=torch.bfloat16)
    impl = be.Gfx906FAImpl(num_heads=Hq, head_size=D, scale=1.0 / np.sqrt(D), num_kv_heads=Hkv, alibi_slopes=None,
                           sliding_window=None, kv_cache_dtype="auto")
    impl._v_fmt = v_fmt
    layer = _FakeLayer()
    kv_cache = torch.zeros((h.NB, 2, BS, Hkv, D), dtype=torch.bfloat16, device=dev)
    impl.do_kv_cache_update(layer, h.key.to(dev), h.val.to(dev), kv_cache, h.slots.to(dev))
    # persistent input buffers
    q_buf = torch.zeros((B, Hq, D), dtype=torch.bfloat16, device=dev)
    sl_buf = torch.tensor([L - 50 for L in full], dtype=torch.int32, device=dev)
    bt_buf = h.bt.to(dev)
    qsl = torch.arange(B + 1, dtype=torch.int32, device=dev)
    out = torch.zeros((B, Hq * D), dtype=torch.bfloat16, device=dev)
    meta = be.Gfx906FAMetadata(num_actual_tokens=B, max_query_len=1,
                               max_seq_len=int(bt_buf.shape[1]) * BS,      # what build_for_cudagraph_capture sets
                               query_start_loc=qsl, seq_lens=sl_buf, block_table=bt_buf,
                               slot_mapping=torch.zeros(B, dtype=torch.int64, device=dev),
                               query_lens_host=[1] * B, seq_lens_host=[L - 50 for L in full])
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for _ in range(2):
            impl.forward(layer, q_buf, None, None, kv_cache, meta, output=out)
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        impl.forward(layer, q_buf, None, None, kv_cache, meta, output=out)
    kc, vc = h.oracle_caches(v_q8=(v_fmt == "q8_0"))
    for step, delta in enumerate([0, -700, -3]):
        lens = [max(1, L + delta) for L in full]
        gq = torch.Generator().manual_seed(80 + step)
        q = torch.randn((B, Hq, D), generator=gq).to(torch.bfloat16)
        q_buf.copy_(q.to(dev))
        sl_buf.copy_(torch.tensor(lens, dtype=torch.int32, device=dev))
        graph.replay()
        torch.cuda.synchronize()
        la = np.asarray(lens, np.int32)
        ref = O.attention_paged(to_np(q), "bf16", np.arange(B, dtype=np.int32), np.ones(B, np.int32), kc, vc,
                                h.bt.numpy(), la, 1.0 / np.sqrt(D), Hkv, q_abs=la - 1,
                                v_fmt="q8" if v_fmt == "q8_0" else "bf16")
        assert_close(to_np(out.float()).reshape(B, Hq, D), ref, what=f"graph replay {step} ({v_fmt})")


def test_impl_fused_fp8_output():
    """Gfx906FAImpl.forward with vLLM's fused static fp8 output quantisation:
    the output buffer is e4m3 [T, Hq*D] and output_scale a device scalar."""
    pytest.importorskip("vllm")
    import gfx906_fa_backend as be
    from test_paged_gpu import LENS, NQ, _FakeLayer, _Hist, _impl_step
    h = _Hist(LENS, 8, seed=75, dtype=torch.bfloat16)
    q, _ = _impl_step(be, h, NQ, "q8_0", False, torch.bfloat16)             # the query of one engine step
    impl = be.Gfx906FAImpl(num_heads=48, head_size=128, scale=1.0 / np.sqrt(128), num_kv_heads=8, alibi_slopes=None,
                           sliding_window=None, kv_cache_dtype="auto")
    impl._v_fmt = "q8_0"
    kv_cache = torch.zeros((h.NB, 2, 16, 8, 128), dtype=torch.bfloat16, device=dev)
    impl.do_kv_cache_update(None, h.key.to(dev), h.val.to(dev), kv_cache, h.slots.to(dev))
    T = sum(NQ)
    meta = be.Gfx906FAMetadata(num_actual_tokens=T, max_query_len=max(NQ), max_seq_len=max(LENS),
                               query_start_loc=_cu(NQ).to(dev),
                               seq_lens=torch.tensor(LENS, dtype=torch.int32, device=dev), block_table=h.bt.to(dev),
                               slot_mapping=torch.zeros(T, dtype=torch.int64, device=dev),
                               query_lens_host=list(NQ), seq_lens_host=list(LENS))
    s = 0.02
    out = torch.zeros((T, 48 * 128), dtype=torch.float8_e4m3fn, device=dev)
    impl.forward(_FakeLayer(), q.to(dev), None, None, kv_cache, meta, output=out,
                 output_scale=torch.tensor(s, dtype=torch.float32, device=dev))
    got = out.float().cpu().numpy().reshape(T, 48, 128)
    ref = h.oracle(q, NQ, v_q8=True)
    err = np.abs(got * s - ref)
    bound = ATOL + RTOL * np.abs(ref) + s * _e4m3_step(ref / s)
    assert (err <= bound).all(), f"{int((err > bound).sum())} fp8 outputs out of bound"
