"""Parity at the benchmark sizes: the configurations bench.py times, checked
against the fp32 oracle (|d| <= 2e-3 + 1e-2 |ref|).

Long contexts make the full oracle expensive, so the chunked-prefill cases
check a spread of query tokens (first, last, every 128-row tile edge of the
GQA-packed layout, the rest seeded-random) over every query head; decode
batches are checked in full.  Mirrors the reference's chunked-prefill test
(tests/test_inline_causal.py:105-165: chunks with q_abs_offset against fp32
causal attention) at the BASELINE sizes."""
import numpy as np
import pytest
import torch

from _paged import PagedCase, assert_close
from _util import to_np

pytestmark = pytest.mark.gpu
dev = "cuda"
G = 6          # GQA 48/8


def _gfx():
    import gfx906_fa
    return gfx906_fa


def _q(shape, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    return torch.randn(shape, generator=g).to(dtype)


def _cu(nq):
    return torch.tensor(np.concatenate([[0], np.cumsum(nq)]), dtype=torch.int32)


def _pick_tokens(n, count, seed):
    """Token indices of an n-token chunk: both ends, the tokens whose
    packed rows (t*G + g) straddle 128-row tile edges, and random others."""
    edges = {0, n - 1}
    for r in range(0, n * G, 128):
        edges.update({r // G, max(0, (r - 1) // G)})
    edges = sorted(t for t in edges if 0 <= t < n)
    rng = np.random.default_rng(seed)
    sel = list(rng.choice(edges, size=min(len(edges), count // 2), replace=False))
    rest = np.setdiff1d(np.arange(n), sel)
    sel += list(rng.choice(rest, size=count - len(sel), replace=False))
    return np.array(sorted(set(int(t) for t in sel) | {0, n - 1}), dtype=np.int64)


def _run(case, q, nq, lens):
    return _gfx().paged_attention(q.to(dev), case.k_cache, case.v_cache, case.block_table.to(dev),
                                  torch.from_numpy(case.seq_lens).to(dev), _cu(nq).to(dev), max(nq), max(lens),
                                  case.scale, query_lens_host=nq, seq_lens_host=lens)


@pytest.mark.parametrize("v_fmt", ["q8t", "f16"])
def test_config4_chunk_at_24k(v_fmt):
    """one 8192-query chunk at offset 24576 against
    32768 keys (the last chunk of the 32K prefill bench.py times): 256 key
    tiles per row tile, the lazy-rescale path and TMA row coordinates past
    2^16 in the staging tiles."""
    L, C = 32768, 8192
    case = PagedCase([L], 8, v_fmt=v_fmt, seed=41)
    q = _q((C, 48, 128), torch.bfloat16, seed=42)
    out = _run(case, q, [C], [L])
    toks = _pick_tokens(C, 64, seed=3)
    ref = case.oracle_rows(to_np(q)[toks], "bf16", np.zeros(len(toks), np.int64), (L - C) + toks)
    assert_close(to_np(out.float())[toks], ref, what=f"config 4 chunk ({v_fmt} V)")


def test_config4_first_chunk():
    """The first 8192-token chunk (offset 0): causal diagonal tiles only."""
    C = 8192
    case = PagedCase([C], 8, v_fmt="q8t", seed=43)
    q = _q((C, 48, 128), torch.bfloat16, seed=44)
    out = _run(case, q, [C], [C])
    toks = _pick_tokens(C, 48, seed=4)
    ref = case.oracle_rows(to_np(q)[toks], "bf16", np.zeros(len(toks), np.int64), toks)
    assert_close(to_np(out.float())[toks], ref, what="config 4 first chunk")


def test_config5_mixed_batch():
    """BASELINE config 5 shape: speculative-verify sequences (4 query tokens,
    causal within the 4) with contexts of 64K+ beside the two 4096-token
    prefill chunks at offsets 0 and 24K, in one paged_attention call (decode
    and tensor-core kernels on the same cache)."""
    verify = [65536, 70001, 66000, 81234]
    lens = verify + [4096, 24576 + 4096]
    nq = [4] * len(verify) + [4096, 4096]
    case = PagedCase(lens, 8, v_fmt="q8t", seed=51)
    q = _q((sum(nq), 48, 128), torch.bfloat16, seed=52)
    out = to_np(_run(case, q, nq, lens).float())
    qn = to_np(q)
    starts = np.concatenate([[0], np.cumsum(nq)[:-1]])
    # every verify row, and 40 tokens of each prefill chunk
    rows, seqs, qabs = [], [], []
    for b, (L, n) in enumerate(zip(lens, nq)):
        toks = np.arange(n) if n == 4 else _pick_tokens(n, 40, seed=b)
        rows += list(starts[b] + toks)
        seqs += [b] * len(toks)
        qabs += list(L - n + toks)
    rows = np.array(rows)
    ref = case.oracle_rows(qn[rows], "bf16", seqs, qabs)
    assert_close(out[rows], ref, what="config 5 mixed batch")


def test_config3_full_batch():
    """BASELINE config 3 in full: 64 decode sequences, contexts U[1K, 32K],
    every sequence and head checked (the balanced split puts stream
    boundaries at different pages in every sequence)."""
    rng = np.random.default_rng(3)
    lens = [int(x) for x in rng.integers(1024, 32769, size=64)]
    case = PagedCase(lens, 8, v_fmt="q8t", seed=31)
    q = _q((64, 48, 128), torch.bfloat16, seed=32)
    out = _gfx().forward_paged_direct(q.view(64, 48, 1, 128).to(dev), case.k_cache, case.v_cache,
                                      case.block_table.to(dev), torch.from_numpy(case.seq_lens).to(dev), case.scale)
    ref = case.oracle_bhsd(to_np(q).reshape(64, 48, 1, 128), "bf16")
    assert_close(to_np(out), ref, what="config 3 full batch")


def test_config1_golden_prefill_and_decode():
    """BASELINE config 1 on the GPU against the reference pipeline's own
    output (tests/golden/config1_golden.npz, made by running the reference's
    CPU functions): 512-token causal prefill, then the decode token."""
    import os
    z = np.load(os.path.join(os.path.dirname(__file__), "golden", "config1_golden.npz"))
    q, bt = z["cfg1_q"], z["cfg1_block_table"]
    kq, vq = z["cfg1_k_q8_ref"], z["cfg1_v_q8_ref"]
    sc = float(z["cfg1_scale"])
    NB, bs, Hkv, L = 40, 16, 2, 513
    kc = np.zeros((NB, bs, Hkv, 136), np.uint8)
    vc = np.zeros_like(kc)
    for t in range(L):
        kc[bt[0, t // bs], t % bs] = kq[t]
        vc[bt[0, t // bs], t % bs] = vq[t]
    g = _gfx()
    kcd, vcd = torch.from_numpy(kc).to(dev), torch.from_numpy(vc).to(dev)
    btd = torch.from_numpy(bt).to(dev)
    o = g.paged_attention(torch.from_numpy(q[:512]).to(dev), kcd, vcd, btd,
                          torch.tensor([512], dtype=torch.int32, device=dev),
                          torch.tensor([0, 512], dtype=torch.int32, device=dev), 512, 512, sc,
                          out=torch.empty((512, 8, 128), dtype=torch.float32, device=dev),
                          query_lens_host=[512], seq_lens_host=[512])
    assert_close(to_np(o)[::8], z["cfg1_prefill_out"], what="config 1 prefill vs reference")
    o = g.paged_attention(torch.from_numpy(q[512:513]).to(dev), kcd, vcd, btd,
                          torch.tensor([513], dtype=torch.int32, device=dev),
                          torch.tensor([0, 1], dtype=torch.int32, device=dev), 1, 513, sc,
                          out=torch.empty((1, 8, 128), dtype=torch.float32, device=dev))
    assert_close(to_np(o), z["cfg1_decode_out"], what="config 1 decode vs reference")
    assert g.device_error(True) == 0


def test_prefill_sequences_in_staging_groups():
    """Three long-context prefill chunks whose fp16 staging together exceeds
    the 1 GiB group budget run as two groups, one after the other, on one
    workspace; every chunk is checked."""
    lens, nq = [100000, 90000, 80000], [1024, 1024, 1024]
    case = PagedCase(lens, 8, v_fmt="q8t", seed=61)
    q = _q((sum(nq), 48, 128), torch.bfloat16, seed=62)
    out = to_np(_run(case, q, nq, lens).float())
    qn = to_np(q)
    rows, seqs, qabs = [], [], []
    for b, (L, n) in enumerate(zip(lens, nq)):
        toks = _pick_tokens(n, 12, seed=b)
        rows += list(b * 1024 + toks)
        seqs += [b] * len(toks)
        qabs += list(L - n + toks)
    rows = np.array(rows)
    assert_close(out[rows], case.oracle_rows(qn[rows], "bf16", seqs, qabs), what="staging groups")
