"""Page gather on the GPU, bit-exact against the oracle and the reference's
golden vectors (tests/test_gather.py of the reference: V exact including the
zero tail, K exact on valid rows, seq_len 0 / 30 / Sk)."""
import os

import numpy as np
import pytest
import torch

import oracle as O
from _util import to_np

pytestmark = pytest.mark.gpu
dev = "cuda"
GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _gfx():
    import gfx906_fa
    return gfx906_fa


def _check(kc, vc, bt, sl, Sk, k_fill=0):
    k_out = torch.full((bt.shape[0], kc.shape[2], Sk, kc.shape[3]), k_fill, dtype=torch.uint8, device=dev)
    v_out = torch.empty((bt.shape[0], kc.shape[2], Sk, vc.shape[3]), dtype=vc.dtype, device=dev)
    ko, vo = _gfx().gather_paged_kv_q8(kc.to(dev), vc.to(dev), bt.to(dev), sl.to(dev), Sk, k_out=k_out, v_out=v_out)
    assert ko.data_ptr() == k_out.data_ptr() and vo.data_ptr() == v_out.data_ptr()   # reused buffers
    rk = np.full(tuple(k_out.shape), k_fill, np.uint8)
    rk, rv = O.gather(to_np(kc), to_np(vc), to_np(bt), to_np(sl), Sk, k_out=rk)
    assert np.array_equal(to_np(vo), rv)
    assert np.array_equal(to_np(ko), rk)          # includes untouched K tail rows


@pytest.mark.parametrize("case", ["basic", "old_path"])
def test_gather_golden(case):
    g = np.load(os.path.join(GOLD, "gather_golden.npz"))
    p = f"gather_{case}_"
    sl = g[p + "seq_lens"]
    Sk = int(g[p + "Sk"])
    ko, vo = _gfx().gather_paged_kv_q8(torch.from_numpy(g[p + "k_cache"]).to(dev),
                                       torch.from_numpy(g[p + "v_cache"]).to(dev),
                                       torch.from_numpy(g[p + "block_table"]).to(dev),
                                       torch.from_numpy(sl).to(dev), Sk)
    assert np.array_equal(to_np(vo), g[p + "v_ref"])
    ko = to_np(ko)
    for s, L in enumerate(sl):
        assert np.array_equal(ko[s, :, :L], g[p + "k_ref"][s, :, :L])


def test_gather_random_stress_and_edges():
    gen = torch.Generator().manual_seed(42)
    NB, bs, Hkv, D, B, MB, Sk = 64, 16, 4, 128, 8, 8, 128
    kc = torch.randint(0, 256, (NB, bs, Hkv, D // 32 * 34), generator=gen, dtype=torch.uint8)
    vc = torch.randn((NB, bs, Hkv, D), generator=gen).half()
    bt = torch.randint(0, NB, (B, MB), generator=gen, dtype=torch.int32)
    bt[2, 3] = -1                          # a hole in the table
    sl = torch.tensor([0, 1, 63, 64, 17, 128, 100, 30], dtype=torch.int32)
    _check(kc, vc, bt, sl, Sk, k_fill=0xAB)


def test_gather_sk_beyond_table_and_d64():
    gen = torch.Generator().manual_seed(7)
    NB, bs, Hkv, D, B, MB, Sk = 16, 16, 2, 64, 3, 2, 64      # Sk > MB*bs: pages past the table
    kc = torch.randint(0, 256, (NB, bs, Hkv, D // 32 * 34), generator=gen, dtype=torch.uint8)
    vc = torch.randn((NB, bs, Hkv, D), generator=gen).half()
    bt = torch.randint(0, NB, (B, MB), generator=gen, dtype=torch.int32)
    sl = torch.tensor([32, 20, 0], dtype=torch.int32)
    _check(kc, vc, bt, sl, Sk, k_fill=0x11)


def test_gather_config2_full_size():
    """16 sequences x 4096 tokens, Hkv 8, 70 000-page pool,
    block tables are seeded random page permutations."""
    gen = torch.Generator().manual_seed(2)
    NB, bs, Hkv, D, B, L = 70000, 16, 8, 128, 16, 4096
    MB = L // bs
    kc = torch.randint(0, 256, (NB, bs, Hkv, D // 32 * 34), generator=gen, dtype=torch.uint8)
    vc = torch.randint(-30000, 30000, (NB, bs, Hkv, D), generator=gen, dtype=torch.int16).view(torch.float16)
    bt = torch.randperm(NB, generator=gen)[:B * MB].to(torch.int32).view(B, MB)
    sl = torch.full((B,), L, dtype=torch.int32)
    ko, vo = _gfx().gather_paged_kv_q8(kc.to(dev), vc.to(dev), bt.to(dev), sl.to(dev), L)
    # size-independent check: every gathered row equals its source page row
    idx = bt.long()                                               # [B, MB]
    k_ref = kc[idx].reshape(B, L, Hkv, -1).permute(0, 2, 1, 3)
    v_ref = vc[idx].reshape(B, L, Hkv, D).permute(0, 2, 1, 3)
    assert torch.equal(ko.cpu(), k_ref)
    assert torch.equal(vo.cpu().view(torch.int16), v_ref.contiguous().view(torch.int16))
