"""Failure detection without a GPU fault: bad block-table entries, context
lengths beyond the block table, and a bounded wait that runs out.

A block-table entry that is negative (or >= the cache's page count) is never
dereferenced: it sets bit 1 of the device error word; the decode kernel drops
that page's keys, the prefill pack step reads them as zero vectors, the
gather treats the page as out of range (the reference's rule for negative
entries, extension/gfx906_fa_gather.cu:190-357).  A bounded mbarrier wait
that gives up sets bit 0 and lets the kernel return.  Nothing here faults,
traps or hangs the GPU: every wait is bounded and every bad address is
skipped before it is formed."""
import ctypes

import numpy as np
import pytest
import torch

import oracle as O
from _paged import PagedCase, assert_close
from _util import capi, to_np

pytestmark = pytest.mark.gpu
dev = "cuda"
ERR_WAIT, ERR_PAGE = 1, 2


def _gfx():
    import gfx906_fa
    return gfx906_fa


def _q(shape, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    return torch.randn(shape, generator=g).to(dtype)


def _cu(nq):
    return torch.tensor(np.concatenate([[0], np.cumsum(nq)]), dtype=torch.int32)


@pytest.mark.parametrize("v_fmt", ["q8t", "f16", "q8"])
@pytest.mark.parametrize("bad", ["negative", "past_cache"])
def test_decode_bad_page_is_dropped_and_flagged(v_fmt, bad):
    g = _gfx()
    g.device_error(True)
    lens, nq = [3000, 700, 1200], [1, 1, 4]
    case = PagedCase(lens, 8, v_fmt=v_fmt, seed=61)
    bt = case.block_table.clone()
    bt[0, 10] = -1 if bad == "negative" else case.NB + 5
    bt[2, 3] = -1 if bad == "negative" else case.NB
    q = _q((sum(nq), 48, 128), torch.bfloat16, seed=62)
    out = g.paged_attention(q.to(dev), case.k_cache, case.v_cache, bt.to(dev),
                            torch.from_numpy(case.seq_lens).to(dev), _cu(nq).to(dev), 4, 3000, case.scale,
                            query_lens_host=nq, seq_lens_host=lens)
    assert g.device_error(True) & ERR_PAGE
    case.block_table = bt
    ref = case.oracle_varlen(to_np(q), "bf16", nq, num_blocks=case.NB)
    assert_close(to_np(out.float()), ref, what=f"decode with a {bad} page")
    assert g.device_error(True) == 0                 # the word clears


def test_prefill_bad_page_is_flagged_and_earlier_rows_exact():
    """Prefill chunk of 700 tokens at offset 1300 with page 120 (keys
    1920..1935) bad: rows that cannot see it match the oracle; the word
    carries bit 1."""
    g = _gfx()
    g.device_error(True)
    lens, nq = [2000], [700]
    case = PagedCase(lens, 8, v_fmt="q8t", seed=63)
    bt = case.block_table.clone()
    bt[0, 120] = -1
    q = _q((700, 48, 128), torch.float16, seed=64)
    out = g.paged_attention(q.to(dev), case.k_cache, case.v_cache, bt.to(dev),
                            torch.from_numpy(case.seq_lens).to(dev), _cu(nq).to(dev), 700, 2000, case.scale,
                            query_lens_host=nq, seq_lens_host=lens)
    assert g.device_error(True) & ERR_PAGE
    o = to_np(out.float())
    assert np.isfinite(o).all()
    ref = case.oracle_varlen(to_np(q), None, nq)
    t_ok = 1920 - 1300                                # tokens t < 620 see keys <= 1300 + t < 1920
    assert_close(o[:t_ok], ref[:t_ok], what="prefill rows before the bad page")


def test_gather_page_past_cache_counts_as_out_of_range():
    g = _gfx()
    g.device_error(True)
    lens = [300, 170]
    case = PagedCase(lens, 8, seed=65)
    bt = case.block_table.clone()
    bt[0, 5] = case.NB + 100
    Sk = 320
    k_out = torch.zeros((2, 8, Sk, 136), dtype=torch.uint8, device=dev)
    ko, vo = g.gather_paged_kv_q8(case.k_cache, case.v_cache, bt.to(dev), torch.from_numpy(case.seq_lens).to(dev),
                                  Sk, k_out=k_out)
    assert g.device_error(True) & ERR_PAGE
    bt_ref = bt.numpy().copy()
    bt_ref[0, 5] = -1
    kr, vr = O.gather(case.k_np, case.v_np, bt_ref, case.seq_lens, Sk)
    assert np.array_equal(to_np(ko), kr)
    assert np.array_equal(to_np(vo).view(np.uint16), vr.view(np.uint16))


def test_context_longer_than_block_table_is_clamped():
    """kv_len beyond max_blocks * block_size reads no block-table entry
    past the sequence's row: the extra keys do not exist."""
    g = _gfx()
    g.device_error(True)
    lens = [1600, 500]                                 # 100 pages: the block table's width
    case = PagedCase(lens, 8, v_fmt="q8t", seed=66)
    sl = case.seq_lens.copy()
    sl[0] = 1600 + 300
    q = _q((2, 48, 1, 128), torch.float32, seed=67)
    out = g.forward_paged_direct(q.to(dev), case.k_cache, case.v_cache, case.block_table.to(dev),
                                 torch.from_numpy(sl).to(dev), case.scale)
    assert_close(to_np(out), case.oracle_bhsd(to_np(q), None), what="clamped context")
    assert g.device_error(True) == 0


def test_bounded_wait_gives_up_and_context_survives():
    """A wait nothing will complete, limited to 2 ms: the kernel returns,
    bit 0 is set, the word clears, and the next attention call works."""
    g = _gfx()
    g.device_error(True)
    lib = capi()
    lib.gfx906_fa_selftest_wait_timeout.argtypes = [ctypes.c_uint64, ctypes.c_void_p, ctypes.c_void_p]
    done = torch.zeros(1, dtype=torch.int32, device=dev)
    e = lib.gfx906_fa_selftest_wait_timeout(2_000_000, ctypes.c_void_p(done.data_ptr()),
                                            ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert e == 0
    torch.cuda.synchronize()
    assert int(done.item()) == 1
    assert g.device_error(True) == ERR_WAIT
    assert g.device_error(True) == 0
    # limits beyond 100 ms are refused on the host
    assert lib.gfx906_fa_selftest_wait_timeout(10 ** 9, ctypes.c_void_p(done.data_ptr()), None) == 1
    lens = [700, 40]
    case = PagedCase(lens, 8, seed=68)
    q = _q((2, 48, 1, 128), torch.float32, seed=69)
    out = g.forward_paged_direct(q.to(dev), case.k_cache, case.v_cache, case.block_table.to(dev),
                                 torch.from_numpy(case.seq_lens).to(dev), case.scale)
    assert_close(to_np(out), case.oracle_bhsd(to_np(q), None), what="after the timeout")
