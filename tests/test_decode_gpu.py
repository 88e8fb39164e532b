"""Split-K decode attention straight from the paged Q8 cache, against the
fp32 dequant + softmax oracle (tolerance |d| <= 2e-3 + 1e-2 |ref|).

Cases follow the reference's own attention tests: batched decode with GQA
48/8 and mixed context lengths (tests/test_decode_batch.py), the per-rank
TP=8 slice Hq/Hkv = 6/1 (tests/test_fa_mixed_batch.py), inline-causal
chunks via q_abs_offset (tests/test_inline_causal.py), plus the edges the
reference leaves undefined (empty sequences, holes in lengths)."""
import os

import numpy as np
import pytest
import torch

import oracle as O
from _paged import PagedCase, assert_close
from _util import to_np

pytestmark = pytest.mark.gpu
dev = "cuda"
GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _gfx():
    import gfx906_fa
    return gfx906_fa


def _q(shape, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    return torch.randn(shape, generator=g).to(dtype)


def _qnp(q):
    return (to_np(q), "bf16") if q.dtype == torch.bfloat16 else (to_np(q), None)


def _direct(case, q, **kw):
    return _gfx().forward_paged_direct(q.to(dev), case.k_cache, case.v_cache, case.block_table.to(dev),
                                       torch.from_numpy(case.seq_lens).to(dev), case.scale, **kw)


@pytest.mark.parametrize("Hq,Hkv", [(48, 8), (8, 4), (6, 1), (8, 2), (16, 4), (64, 8), (32, 32)])
def test_direct_decode_gqa(Hq, Hkv):
    lens = [1, 17, 300, 1024, 2500, 16, 33, 4100]
    case = PagedCase(lens, Hkv, seed=Hq * 10 + Hkv)
    q = _q((len(lens), Hq, 1, 128), torch.float32, seed=1)
    out = _direct(case, q)
    assert_close(to_np(out), case.oracle_bhsd(to_np(q), None), what=f"decode {Hq}/{Hkv}")


@pytest.mark.parametrize("v_fmt", ["f16", "bf16", "q8", "q8t"])
@pytest.mark.parametrize("qdt", [torch.float32, torch.float16, torch.bfloat16])
def test_direct_decode_formats(v_fmt, qdt):
    lens = [5000, 77, 1, 2049]
    case = PagedCase(lens, 8, v_fmt=v_fmt, seed=3)
    q = _q((4, 48, 1, 128), qdt, seed=2)
    out = _direct(case, q)
    qn, tag = _qnp(q)
    assert_close(to_np(out), case.oracle_bhsd(qn, tag), what=f"{v_fmt}/{qdt}")


@pytest.mark.parametrize("Hq,Hkv", [(48, 8), (8, 4), (6, 1), (16, 2), (16, 16), (32, 32)])
@pytest.mark.parametrize("Sq", [1, 2, 3, 4, 5])
def test_direct_decode_q8t(Hq, Hkv, Sq):
    """Page-transposed Q8_0 V across kv-head group sizes (1, 2, 4, 8 heads per
    CTA and several CTAs per sequence) and 1..32 query rows per kv head: one,
    two and three 8-row n-tiles of the transposed consumer (padding rows
    included); above 24 rows per kv head the sequences go to the prefill
    kernel."""
    lens = [4100, 1, 77, 2500, 16, 900]
    case = PagedCase(lens, Hkv, v_fmt="q8t", seed=Hq + Hkv + Sq)
    q = _q((len(lens), Hq, Sq, 128), torch.bfloat16, seed=Sq)
    qa = (case.seq_lens - Sq).astype(np.int32)
    kw = {"q_abs_offset": torch.from_numpy(qa).to(dev)} if Sq > 1 else {}
    out = _direct(case, q, **kw)
    qn, tag = _qnp(q)
    assert_close(to_np(out), case.oracle_bhsd(qn, tag, q_abs=qa if Sq > 1 else None),
                 what=f"q8t {Hq}/{Hkv} Sq={Sq}")


@pytest.mark.parametrize("Sq", [2, 4, 5])
def test_direct_causal_spec_decode(Sq):
    """Sq query tokens per sequence, causal inside the chunk
    (q_abs_offset = seq_len - Sq); 6*Sq rows per kv head -> two m-tiles."""
    lens = [4096, 700, 16, 9000]
    case = PagedCase(lens, 8, seed=Sq)
    q = _q((4, 48, Sq, 128), torch.float32, seed=Sq)
    qa = (case.seq_lens - Sq).astype(np.int32)
    out = _direct(case, q, q_abs_offset=torch.from_numpy(qa).to(dev))
    assert_close(to_np(out), case.oracle_bhsd(to_np(q), None, q_abs=qa), what=f"Sq={Sq}")


def test_direct_additive_mask():
    lens = [300, 129]
    case = PagedCase(lens, 2, seed=9)
    Sq = 2
    q = _q((2, 8, Sq, 128), torch.float32, seed=9)
    g = torch.Generator().manual_seed(5)
    skv = case.max_blocks * 16
    mask = torch.where(torch.rand((2, Sq, skv), generator=g) < 0.3, -65504.0, 0.0).half()
    mask[:, :, 7] = 0.5
    out = _direct(case, q, mask=mask.to(dev))
    assert_close(to_np(out), case.oracle_bhsd(to_np(q), None, mask=to_np(mask)), what="mask")


@pytest.mark.parametrize("Hq,Hkv,Sq", [(16, 2, 2), (6, 1, 1), (48, 8, 3)])
def test_direct_additive_mask_q8t(Hq, Hkv, Sq):
    """Additive mask with page-transposed Q8_0 V (transposed consumer, one to
    three n-tiles)."""
    lens = [300, 129, 2000]
    case = PagedCase(lens, Hkv, v_fmt="q8t", seed=Hq + Sq)
    q = _q((3, Hq, Sq, 128), torch.bfloat16, seed=Sq)
    g = torch.Generator().manual_seed(7)
    skv = case.max_blocks * 16
    mask = torch.where(torch.rand((3, Sq, skv), generator=g) < 0.3, -65504.0, 0.0).half()
    mask[:, :, 7] = 0.5
    out = _direct(case, q, mask=mask.to(dev))
    qn, tag = _qnp(q)
    assert_close(to_np(out), case.oracle_bhsd(qn, tag, mask=to_np(mask)), what=f"mask q8t {Hq}/{Hkv}/{Sq}")


def test_empty_and_short_sequences():
    lens = [0, 1, 15, 16, 17]
    case = PagedCase(lens, 4, seed=11)
    q = _q((5, 8, 1, 128), torch.float32, seed=4)
    o = to_np(_direct(case, q))
    assert (o[0] == 0).all()
    assert_close(o, case.oracle_bhsd(to_np(q), None), what="short")


def test_config1_decode_token_matches_reference_golden():
    """BASELINE config 1 decode token (L = 513, Hq/Hkv 8/2, K and V Q8_0)
    against the reference pipeline's output stored in the golden fixture."""
    c = np.load(os.path.join(GOLD, "config1_golden.npz"))
    bt = c["cfg1_block_table"]
    NB, bs, Hkv, L = 40, 16, 2, 513
    kc = np.zeros((NB, bs, Hkv, 136), np.uint8)
    vc = np.zeros_like(kc)
    for t in range(L):
        kc[bt[0, t // bs], t % bs] = c["cfg1_k_q8_ref"][t]
        vc[bt[0, t // bs], t % bs] = c["cfg1_v_q8_ref"][t]
    q = torch.from_numpy(c["cfg1_q"][512:513]).float().permute(1, 0, 2).unsqueeze(0)   # [1, 8, 1, 128]
    out = _gfx().forward_paged_direct(q.contiguous().to(dev), torch.from_numpy(kc).to(dev),
                                      torch.from_numpy(vc).to(dev), torch.from_numpy(bt).to(dev),
                                      torch.tensor([L], dtype=torch.int32, device=dev), float(c["cfg1_scale"]))
    ref = c["cfg1_decode_out"].transpose(1, 0, 2)[None]                                 # [1, 8, 1, 128]
    assert_close(to_np(out), ref, what="config1 decode")


def test_paged_attention_varlen_inplace_cache():
    """vLLM layout: one [NB, 2, bs, Hkv, D] fp16 allocation; the Q8_0 K rows
    live densely at the start of each page's K half, V stays fp16."""
    g = _gfx()
    Hq, Hkv, D, bs = 48, 8, 128, 16
    lens = [3000, 1, 40, 777]
    nq = [1, 1, 4, 3]
    case = PagedCase(lens, Hkv, seed=21)
    NB = case.NB
    kv = torch.zeros((NB, 2, bs, Hkv, D), dtype=torch.float16, device=dev)
    kvb = kv.view(torch.uint8).view(NB, 2, bs * Hkv * 2 * D)
    rb = case.rb
    k_view = kvb[:, 0, :bs * Hkv * rb].view(NB, bs, Hkv, rb)
    k_view.copy_(case.k_cache)
    kv[:, 1].copy_(case.v_cache)
    T = sum(nq)
    q = _q((T, Hq, D), torch.bfloat16, seed=8)
    cu = torch.tensor(np.concatenate([[0], np.cumsum(nq)]), dtype=torch.int32)
    out = g.paged_attention(q.to(dev), k_view, kv[:, 1], case.block_table.to(dev),
                            torch.from_numpy(case.seq_lens).to(dev), cu.to(dev), max(nq), max(lens),
                            case.scale)
    assert out.dtype == torch.bfloat16
    ref = case.oracle_varlen(to_np(q), "bf16", nq)
    # bf16 output: its rounding (<= 2^-9 relative) is inside the relative term
    assert_close(to_np(out.float()), ref, what="varlen")


def test_config3_decode_full_size_subset_checked():
    """64 sequences, L ~ U[1K, 32K], GQA 48/8, bf16 Q.
    The whole batch runs on the GPU; 6 sequences are checked against the
    oracle (the kernel treats every sequence identically)."""
    rng = np.random.default_rng(3)
    lens = rng.integers(1024, 32769, size=64).tolist()
    case = PagedCase(lens, 8, seed=33)
    q = _q((64, 48, 1, 128), torch.bfloat16, seed=3)
    out = to_np(_direct(case, q))
    pick = [0, 7, int(np.argmax(lens)), int(np.argmin(lens)), 40, 63]
    ref = case.oracle_bhsd(to_np(q)[pick], "bf16", pick=pick)
    assert_close(out[pick], ref, what="config3 subset")


def test_no_device_error_flagged():
    assert _gfx().device_error(True) == 0


@pytest.mark.parametrize("hkv", [1, 2, 8])
def test_decode_backend_cache_layout(hkv):
    """Decode over the backend's own cache: one vLLM allocation [NB, 2, bs,
    Hkv, D] with Q8_0 K rows and page-transposed Q8_0 V records adjacent at
    each page's start (one copy per page when a CTA holds all kv heads)."""
    import gfx906_fa_paged as P
    lens = [3000, 17, 1, 777]
    B, bs, D = len(lens), 16, 128
    npg = [(L + bs - 1) // bs for L in lens]
    NB = sum(npg) + 5
    g = torch.Generator().manual_seed(hkv)
    perm = torch.randperm(NB, generator=g).to(torch.int32)
    bt = torch.full((B, max(npg)), -1, dtype=torch.int32)
    c = 0
    for b, n in enumerate(npg):
        bt[b, :n] = perm[c:c + n]
        c += n
    kv = torch.zeros((NB, 2, bs, hkv, D), dtype=torch.float16, device=dev)
    k8, v8 = P.kv_cache_views(kv, "q8_0")
    T = sum(lens)
    key = torch.randn((T, hkv, D), generator=g).half()
    val = torch.randn((T, hkv, D), generator=g).half()
    seq_of = np.repeat(np.arange(B), lens)
    starts = np.concatenate([[0], np.cumsum(lens)[:-1]])
    tpos = np.arange(T) - starts[seq_of]
    slots = torch.from_numpy(bt.numpy()[seq_of, tpos // bs].astype(np.int64) * bs + tpos % bs)
    _gfx().store_kv(key.to(dev), val.to(dev), slots.to(dev), k8, v8, 3)
    q = _q((B, 6 * hkv, 1, D), torch.bfloat16, seed=hkv)
    sl = torch.tensor(lens, dtype=torch.int32)
    out = _gfx().forward_paged_direct(q.to(dev), k8, v8, bt.to(dev), sl.to(dev), 1.0 / np.sqrt(D))
    rb = D // 32 * 34
    ref = O.attention_paged(*_qnp(q)[:1], _qnp(q)[1], np.zeros(B, np.int32), np.ones(B, np.int32),
                            np.ascontiguousarray(to_np(k8)), np.ascontiguousarray(to_np(v8)), bt.numpy(),
                            sl.numpy(), 1.0 / np.sqrt(D), hkv, v_fmt="q8t",
                            v_strides=(hkv * bs * rb, 0, bs * rb), q_strides=(6 * hkv * D, D, D),
                            out_shape=(B, 6 * hkv, 1, D), o_strides=(6 * hkv * D, D, D))
    assert_close(to_np(out), ref, what=f"backend layout hkv={hkv}")
