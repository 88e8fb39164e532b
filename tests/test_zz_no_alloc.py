"""The allocation-free decode entry point (gfx906_fa_decode_splitk_noalloc).

It exists for callers that cannot allocate device memory at call time, such
as code running inside an allocator's own hooks or hosts that give a plugin a
fixed memory budget: instead of a caller-provided workspace it uses a 32 MiB
array the library keeps in static device memory.  This test calls it through
the C ABI twice in a row (different queries, so the second call runs on the
first call's leftover scratch contents) and compares each result with the
regular workspace entry point, gfx906_fa_decode_splitk, within the attention
tolerance used by every other GPU test.  The file name sorts last, so a run
that stops at the first failure has run everything else before it.
"""
import ctypes

import numpy as np
import pytest
import torch

from _paged import PagedCase, assert_close
from _util import G9AttnBatch, capi, to_np

pytestmark = pytest.mark.gpu
dev = "cuda"


def _batch(case, q, out, bt, sl):
    B, Hq, D = q.shape
    b = G9AttnBatch()
    b.q, b.q_dtype = q.data_ptr(), 1                       # bf16
    b.q_seq_stride, b.q_tok_stride, b.q_head_stride = Hq * D, 0, D
    b.seq_q = 1
    b.out, b.out_dtype = out.data_ptr(), 2                 # fp32
    b.o_seq_stride, b.o_tok_stride, b.o_head_stride = Hq * D, 0, D
    b.k_cache = case.k_cache.data_ptr()
    b.k_page_stride, b.k_tok_stride, b.k_head_stride = 16 * case.Hkv * 136, case.Hkv * 136, 136
    b.v_cache = case.v_cache.data_ptr()
    b.v_page_stride, b.v_tok_stride, b.v_head_stride = 16 * case.Hkv * 256, case.Hkv * 256, 256
    b.v_fmt = 0
    b.block_table, b.max_blocks, b.block_size = bt.data_ptr(), bt.shape[1], 16
    b.kv_len, b.max_kv = sl.data_ptr(), int(case.seq_lens.max())
    b.num_seqs, b.num_heads_q, b.num_heads_kv, b.head_dim = B, Hq, case.Hkv, D
    b.scale = case.scale
    return b


def test_noalloc_decode_matches_workspace_entry_two_calls():
    lib = capi()
    lib.gfx906_fa_decode_workspace_size.restype = ctypes.c_size_t
    lib.gfx906_fa_decode_workspace_size.argtypes = [ctypes.POINTER(G9AttnBatch)]
    lib.gfx906_fa_decode_splitk.argtypes = [ctypes.POINTER(G9AttnBatch), ctypes.c_void_p, ctypes.c_size_t,
                                            ctypes.c_void_p]
    lib.gfx906_fa_decode_splitk_noalloc.argtypes = [ctypes.POINTER(G9AttnBatch), ctypes.c_void_p]
    lens = [4100, 77, 1, 2500, 900]                    # several KV chunks per sequence
    case = PagedCase(lens, 8, seed=77)
    bt = case.block_table.to(dev)
    sl = torch.from_numpy(case.seq_lens).to(dev)
    stream = torch.cuda.current_stream().cuda_stream
    for call in range(2):
        g = torch.Generator().manual_seed(100 + call)
        q = torch.randn((len(lens), 48, 128), generator=g).to(torch.bfloat16).to(dev)
        out_ref = torch.zeros((len(lens), 48, 128), dtype=torch.float32, device=dev)
        out_na = torch.full_like(out_ref, float("nan"))
        b_ref = _batch(case, q, out_ref, bt, sl)
        ws = lib.gfx906_fa_decode_workspace_size(ctypes.byref(b_ref))
        assert ws > 0
        wsbuf = torch.empty(ws, dtype=torch.uint8, device=dev)
        assert lib.gfx906_fa_decode_splitk(ctypes.byref(b_ref), wsbuf.data_ptr(), ws, stream) == 0
        b_na = _batch(case, q, out_na, bt, sl)
        assert lib.gfx906_fa_decode_splitk_noalloc(ctypes.byref(b_na), stream) == 0
        torch.cuda.synchronize()
        assert_close(to_np(out_na), to_np(out_ref), what=f"no-alloc call {call}")
        # and against the fp32 oracle
        ref = case.oracle_bhsd(to_np(q.float()).reshape(len(lens), 48, 1, 128), None)
        assert_close(to_np(out_na).reshape(len(lens), 48, 1, 128), ref, what=f"no-alloc vs oracle {call}")


def test_noalloc_rejects_batches_beyond_the_scratch():
    """A batch whose partial results need more than 32 MiB is refused."""
    lib = capi()
    lib.gfx906_fa_decode_workspace_size.restype = ctypes.c_size_t
    lib.gfx906_fa_decode_workspace_size.argtypes = [ctypes.POINTER(G9AttnBatch)]
    lib.gfx906_fa_decode_splitk_noalloc.argtypes = [ctypes.POINTER(G9AttnBatch), ctypes.c_void_p]
    case = PagedCase([64], 8, seed=1)
    q = torch.zeros((512, 48, 128), dtype=torch.bfloat16, device=dev)
    out = torch.zeros((512, 48, 128), dtype=torch.float32, device=dev)
    bt = torch.zeros((512, 2048), dtype=torch.int32, device=dev)
    sl = torch.zeros(512, dtype=torch.int32, device=dev)
    b = _batch(case, q, out, bt, sl)
    b.max_kv = 32768
    assert lib.gfx906_fa_decode_workspace_size(ctypes.byref(b)) > (32 << 20)
    assert lib.gfx906_fa_decode_splitk_noalloc(ctypes.byref(b), torch.cuda.current_stream().cuda_stream) == 1
