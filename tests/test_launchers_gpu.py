"""The reference-named attention launchers through the C ABI, with the
reference's argument meaning (extension/gfx906_fa_launcher.cu:53-75,
222-249, called as extension/gfx906_fa.cpp:191-246,590-653 does): fp32 Q
[B, Hq, Sq, D], KV_max expanded to [B, grid_x], fp32 output in BSHD
[B, Sq, Hq, D], inline-causal offsets or an additive fp16 mask; checked
against the fp32 oracle (|d| <= 2e-3 + 1e-2 |ref|)."""
import ctypes

import numpy as np
import pytest
import torch

import oracle as O
from _paged import PagedCase, assert_close
from _util import capi, to_np

pytestmark = pytest.mark.gpu
dev = "cuda"
D = 128


def _grid_x(seq_q):
    """query tiles per sequence of the reference launcher (gfx906_fa.cpp:596-604)"""
    nc = 64 if seq_q > 32 else 32 if seq_q > 16 else 16 if seq_q > 8 else 8 if seq_q > 4 else 4 if seq_q > 2 else 2
    return (seq_q + nc - 1) // nc


def _expand(kv_max, seq_q):
    return kv_max.view(-1, 1).expand(-1, _grid_x(seq_q)).contiguous()


def _p(t):
    return ctypes.c_void_p(0 if t is None else t.data_ptr())


def _lib():
    lib = capi()
    i32, i64, f32, vp = ctypes.c_int, ctypes.c_int64, ctypes.c_float, ctypes.c_void_p
    lib.gfx906_fa_launch.argtypes = [vp, vp, vp, vp, vp, vp, vp, i32, vp, i32, i32, i32, i32, i32, i32, f32, vp]
    lib.gfx906_fa_launch_paged.argtypes = [vp, vp, vp, vp, vp, vp, vp, vp, i32, vp, i32, i32, i32, i32, i32, i32,
                                           i32, i32, i64, i64, i64, i64, i64, i64, f32, vp]
    return lib


def _q(shape, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    return torch.randn(shape, generator=g).to(dtype)


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


@pytest.mark.parametrize("mode", ["plain", "causal", "mask"])
@pytest.mark.parametrize("Sq,Skv", [(1, 300), (7, 500), (200, 640)])
def test_gfx906_fa_launch(mode, Sq, Skv):
    import gfx906_fa
    B, Hq, Hkv = 2, 8, 2
    k = _q((B, Hkv, Skv, D), torch.float16, 1)
    v = _q((B, Hkv, Skv, D), torch.float16, 2)
    q = _q((B, Hq, Sq, D), torch.float32, 3).to(dev)
    k_q8 = gfx906_fa.quantize_q8_0(k.to(dev))
    vd = v.to(dev)
    kv_max = torch.tensor([Skv, max(1, Skv - 37)], dtype=torch.int32)
    qa = mask = None
    pad = 0
    if mode == "causal":
        qa = torch.tensor([Skv - Sq, max(0, Skv // 3 - Sq)], dtype=torch.int32)
    elif mode == "mask":
        pad = ((Skv + 63) // 64) * 64
        g = torch.Generator().manual_seed(4)
        mask = (torch.randn((B, Sq, pad), generator=g) * 2).half()
        mask[:, :, ::7] = float("-inf")
    o = torch.full((B, Sq, Hq, D), float("nan"), dtype=torch.float32, device=dev)
    meta = torch.empty((B, Sq, Hq, 2), dtype=torch.float32, device=dev)
    kvx = _expand(kv_max, Sq).to(dev)
    qad = None if qa is None else qa.to(dev)
    md = None if mask is None else mask.to(dev)
    e = _lib().gfx906_fa_launch(_p(q), _p(k_q8), _p(vd), _p(o), _p(meta), _p(kvx), _p(md), pad, _p(qad), B, Hq, Hkv,
                                Sq, Skv, D, 1.0 / np.sqrt(D), _stream())
    assert e == 0
    torch.cuda.synchronize()
    ref = O.attention_bhsd(to_np(q), None, to_np(k_q8), to_np(v), 1.0 / np.sqrt(D), kv_max=to_np(kv_max),
                           q_abs=None if qa is None else to_np(qa), mask=None if mask is None else to_np(mask))
    assert_close(to_np(o), ref.transpose(0, 2, 1, 3), what=f"gfx906_fa_launch {mode} {Sq}x{Skv}")


@pytest.mark.parametrize("mode", ["plain", "causal", "mask"])
@pytest.mark.parametrize("Sq", [1, 4, 100])
def test_gfx906_fa_launch_paged(mode, Sq):
    B, Hq, Hkv = 3, 48, 8
    lens = [900, 130, 2000]
    case = PagedCase(lens, Hkv, seed=5)             # fp16 V pages, the reference's V format
    q = _q((B, Hq, Sq, D), torch.float32, 6).to(dev)
    sl = torch.from_numpy(case.seq_lens)
    qa = mask = None
    pad = 0
    if mode == "causal":
        qa = (sl - Sq).to(torch.int32)
    elif mode == "mask":
        pad = case.max_blocks * 16
        g = torch.Generator().manual_seed(7)
        mask = (torch.randn((B, Sq, pad), generator=g) * 2).half()
        mask[:, :, 3::11] = float("-inf")
    o = torch.full((B, Sq, Hq, D), float("nan"), dtype=torch.float32, device=dev)
    meta = torch.empty((B, Sq, Hq, 2), dtype=torch.float32, device=dev)
    kvx = _expand(sl, Sq).to(dev)
    bt = case.block_table.to(dev)
    rb = 136
    e = _lib().gfx906_fa_launch_paged(
        _p(q), _p(case.k_cache), _p(case.v_cache), _p(bt), _p(kvx), _p(o), _p(meta),
        _p(None if mask is None else mask.to(dev)) if mask is not None else ctypes.c_void_p(0), pad,
        _p(None if qa is None else qa.to(dev)) if qa is not None else ctypes.c_void_p(0),
        B, Hq, Hkv, Sq, case.max_blocks * 16, D, 16, case.max_blocks,
        16 * Hkv * rb, Hkv * rb, rb, 16 * Hkv * D * 2, Hkv * D * 2, D * 2, 1.0 / np.sqrt(D), _stream())
    assert e == 0
    torch.cuda.synchronize()
    ref = case.oracle_bhsd(to_np(q), None, q_abs=None if qa is None else to_np(qa),
                           mask=None if mask is None else to_np(mask))
    assert_close(to_np(o), ref.transpose(0, 2, 1, 3), what=f"gfx906_fa_launch_paged {mode} Sq={Sq}")


def test_launchers_reject_bad_arguments():
    lib = _lib()
    s = _stream()
    # head_dim 64
    assert lib.gfx906_fa_launch(None, None, None, None, None, None, None, 0, None, 1, 8, 2, 1, 16, 64, 0.1, s) == 1
    # block_size 32
    assert lib.gfx906_fa_launch_paged(None, None, None, None, None, None, None, None, 0, None, 1, 8, 2, 1, 32, 128,
                                      32, 1, 0, 0, 0, 0, 0, 0, 0.1, s) == 1
    # empty batch is a no-op
    assert lib.gfx906_fa_launch(None, None, None, None, None, None, None, 0, None, 0, 8, 2, 1, 16, 128, 0.1, s) == 0
