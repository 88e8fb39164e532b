"""Tensor-core (tcgen05) prefill / chunked-prefill attention against the
fp32 dequant + softmax oracle (|d| <= 2e-3 + 1e-2 |ref|).

Mirrors the reference's tests/test_inline_causal.py (prefill chunks with
q_abs_offset against fp32 causal attention), tests/test_paged.py (prefill,
mixed batches, GQA 48/8) and tests/test_sweep.py (flat forward over Sq and
Skv)."""
import numpy as np
import pytest
import torch

import oracle as O
from _paged import PagedCase, assert_close
from _util import to_np

pytestmark = pytest.mark.gpu
dev = "cuda"


def _gfx():
    import gfx906_fa
    return gfx906_fa


def _q(shape, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    return torch.randn(shape, generator=g).to(dtype)


def _cu(nq):
    return torch.tensor(np.concatenate([[0], np.cumsum(nq)]), dtype=torch.int32)


@pytest.mark.parametrize("Hq,Hkv,lens,nq", [
    (8, 2, [512, 384], [256, 128]),          # tests/test_inline_causal.py shapes
    (48, 8, [700], [700]),                   # full causal prefill, GQA 6
    (8, 8, [1000, 130], [1000, 130]),
    (6, 1, [2048], [333]),                   # TP=8 slice, chunk at an offset
    (64, 8, [300, 5000], [40, 200]),
])
def test_varlen_causal_prefill(Hq, Hkv, lens, nq):
    case = PagedCase(lens, Hkv, seed=Hq + len(lens))
    q = _q((sum(nq), Hq, 128), torch.float16, seed=7)
    out = _gfx().paged_attention(q.to(dev), case.k_cache, case.v_cache, case.block_table.to(dev),
                                 torch.from_numpy(case.seq_lens).to(dev), _cu(nq).to(dev), max(nq), max(lens),
                                 case.scale, query_lens_host=nq, seq_lens_host=lens)
    assert_close(to_np(out.float()), case.oracle_varlen(to_np(q), None, nq), what=f"prefill {Hq}/{Hkv}")


def test_varlen_without_host_lengths():
    """No host lengths: every sequence may be either kind; both kernels run
    and each picks its own sequences on the device."""
    lens, nq = [900, 64, 3000], [300, 1, 4]
    case = PagedCase(lens, 8, seed=5)
    q = _q((sum(nq), 48, 128), torch.bfloat16, seed=1)
    out = _gfx().paged_attention(q.to(dev), case.k_cache, case.v_cache, case.block_table.to(dev),
                                 torch.from_numpy(case.seq_lens).to(dev), _cu(nq).to(dev), max(nq), max(lens),
                                 case.scale)
    # bf16 output: its rounding (<= 2^-9 relative) is inside the relative term
    assert_close(to_np(out.float()), case.oracle_varlen(to_np(q), "bf16", nq), what="mixed")


@pytest.mark.parametrize("v_fmt", ["q8", "q8t", "bf16"])
def test_prefill_v_formats(v_fmt):
    lens, nq = [640], [640]
    case = PagedCase(lens, 8, v_fmt=v_fmt, seed=2)
    q = _q((640, 48, 128), torch.float16, seed=2)
    out = _gfx().paged_attention(q.to(dev), case.k_cache, case.v_cache, case.block_table.to(dev),
                                 torch.from_numpy(case.seq_lens).to(dev), _cu(nq).to(dev), 640, 640, case.scale,
                                 query_lens_host=nq, seq_lens_host=lens)
    assert_close(to_np(out.float()), case.oracle_varlen(to_np(q), None, nq), what=v_fmt)


@pytest.mark.parametrize("bs", [16, 32, 24])
def test_prefill_q8t_page_sizes(bs):
    """Page-transposed Q8_0 V staged for the tensor cores: pages of 16 and 32
    tokens take the direct 16-token loads, 24-token pages the general path;
    the ragged lengths end inside a 16-token group and inside a key tile."""
    lens, nq = [1001, 333], [300, 333]
    case = PagedCase(lens, 8, bs=bs, v_fmt="q8t", seed=3)
    q = _q((sum(nq), 48, 128), torch.bfloat16, seed=4)
    out = _gfx().paged_attention(q.to(dev), case.k_cache, case.v_cache, case.block_table.to(dev),
                                 torch.from_numpy(case.seq_lens).to(dev), _cu(nq).to(dev), max(nq), max(lens),
                                 case.scale, query_lens_host=nq, seq_lens_host=lens)
    assert_close(to_np(out.float()), case.oracle_varlen(to_np(q), "bf16", nq), what=f"q8t bs={bs}")
    assert _gfx().device_error(True) == 0


@pytest.mark.parametrize("Sq,Skv", [(1, 64), (7, 300), (64, 64), (200, 512), (512, 1024)])
def test_flat_forward_sweep(Sq, Skv):
    """gfx906_fa.forward on contiguous [B, Hkv, Skv] K_q8 / V (the gather
    path's layout), GQA 4, batch 2, kv_max per sequence, no causal rule
    (tests/test_sweep.py)."""
    g = _gfx()
    B, Hq, Hkv, D = 2, 8, 2, 128
    k = _q((B, Hkv, Skv, D), torch.float16, seed=Skv)
    v = _q((B, Hkv, Skv, D), torch.float16, seed=Skv + 1)
    q = _q((B, Hq, Sq, D), torch.float32, seed=Sq)
    k_q8 = g.quantize_q8_0(k.to(dev))
    kv_max = torch.tensor([Skv, max(1, Skv - 17)], dtype=torch.int32)
    out = g.forward(q.to(dev), k_q8, v.to(dev), 1.0 / np.sqrt(D), kv_max=kv_max.to(dev))
    ref = O.attention_bhsd(to_np(q), None, to_np(k_q8), to_np(v), 1.0 / np.sqrt(D), kv_max=to_np(kv_max))
    assert_close(to_np(out), ref, what=f"flat {Sq}x{Skv}")


def test_flat_forward_inline_causal():
    g = _gfx()
    B, Hq, Hkv, D, Sq, Skv = 2, 8, 2, 128, 256, 512
    k = _q((B, Hkv, Skv, D), torch.float16, seed=1)
    v = _q((B, Hkv, Skv, D), torch.float16, seed=2)
    q = _q((B, Hq, Sq, D), torch.float32, seed=3)
    k_q8 = g.quantize_q8_0(k.to(dev))
    qa = torch.tensor([Skv - Sq, 100], dtype=torch.int32)
    out = g.forward(q.to(dev), k_q8, v.to(dev), 1.0 / np.sqrt(D), q_abs_offset=qa.to(dev))
    ref = O.attention_bhsd(to_np(q), None, to_np(k_q8), to_np(v), 1.0 / np.sqrt(D), q_abs=to_np(qa))
    assert_close(to_np(out), ref, what="flat causal")


def test_direct_paged_long_chunk_goes_to_tensor_cores():
    """forward_paged_direct with Sq*G > 32 rows: same op, tensor-core path."""
    lens = [600, 1500]
    case = PagedCase(lens, 8, seed=8)
    Sq = 64
    q = _q((2, 48, Sq, 128), torch.float32, seed=8)
    qa = (case.seq_lens - Sq).astype(np.int32)
    out = _gfx().forward_paged_direct(q.to(dev), case.k_cache, case.v_cache, case.block_table.to(dev),
                                      torch.from_numpy(case.seq_lens).to(dev), case.scale,
                                      q_abs_offset=torch.from_numpy(qa).to(dev))
    assert_close(to_np(out), case.oracle_bhsd(to_np(q), None, q_abs=qa), what="direct long")


def test_no_device_error_flagged():
    assert _gfx().device_error(True) == 0
