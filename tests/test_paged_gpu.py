"""`forward_paged` (all three branches) and the vLLM backend's
`Gfx906FAImpl.do_kv_cache_update` -> `forward`, end to end on the GPU against
the fp32 oracle.

Mirrors the reference's tests/test_backend.py:115-163 (a fake layer, a
hand-built Gfx906FAMetadata, do_kv_cache_update then forward, compared with
an fp32 reference), tests/test_paged.py and
tests/test_direct_paged_bitexact.py (direct path against the gather path)."""
import numpy as np
import pytest
import torch

import oracle as O
from _paged import ATOL, RTOL, assert_close
from _util import to_np

pytestmark = pytest.mark.gpu
dev = "cuda"
D, BS = 128, 16


def _paged_mod():
    import gfx906_fa_paged
    return gfx906_fa_paged


class _Hist:
    """Seeded K/V history of B sequences in a shuffled page pool, with
    oracle-side Q8_0 caches built from the same fp16 values."""

    def __init__(self, lens, Hkv, seed, dtype=torch.float16, extra_pages=5):
        g = torch.Generator().manual_seed(seed)
        self.lens = list(lens)
        self.B, self.Hkv = len(lens), Hkv
        npg = [(L + BS - 1) // BS for L in lens]
        self.NB = sum(npg) + extra_pages
        self.max_blocks = max(npg)
        perm = torch.randperm(self.NB, generator=g).to(torch.int32)
        bt = torch.zeros((self.B, self.max_blocks), dtype=torch.int32)
        c = 0
        for b, n in enumerate(npg):
            bt[b, :n] = perm[c:c + n]
            c += n
        self.bt = bt
        T = sum(lens)
        self.key = torch.randn((T, Hkv, D), generator=g).to(dtype)
        self.val = torch.randn((T, Hkv, D), generator=g).to(dtype)
        seq_of = np.repeat(np.arange(self.B), lens)
        starts = np.concatenate([[0], np.cumsum(lens)[:-1]])
        tpos = np.arange(T) - starts[seq_of]
        self.slots = torch.from_numpy(bt.numpy()[seq_of, tpos // BS].astype(np.int64) * BS + tpos % BS)
        self.seq_of, self.tpos = seq_of, tpos
        self.dtype = dtype

    def oracle_caches(self, v_q8):
        """K as Q8_0 rows (oracle quantiser), V as 16-bit rows or Q8_0 rows."""
        kd = "bf16" if self.dtype == torch.bfloat16 else None
        kc = np.zeros((self.NB, BS, self.Hkv, 136), np.uint8)
        O.reshape_and_cache(to_np(self.key), self.slots.numpy(), kc, dtype=kd)
        if v_q8:
            vc = np.zeros_like(kc)
            O.reshape_and_cache(to_np(self.val), self.slots.numpy(), vc, dtype=kd)
        else:
            vc = np.zeros((self.NB, BS, self.Hkv, D), np.uint16)
            O.store_v16(to_np(self.val).view(np.uint16), self.slots.numpy(), vc)
        return kc, vc

    def oracle(self, q, nq, v_q8, **feat):
        kc, vc = self.oracle_caches(v_q8)
        nq = np.asarray(nq, np.int32)
        qs = np.concatenate([[0], np.cumsum(nq)[:-1]]).astype(np.int32)
        lens = np.asarray(self.lens, np.int32)
        qd = "bf16" if q.dtype == torch.bfloat16 else None
        vfmt = "q8" if v_q8 else ("bf16" if self.dtype == torch.bfloat16 else "f16")
        return O.attention_paged(to_np(q), qd, qs, nq, kc, vc, self.bt.numpy(), lens, 1.0 / np.sqrt(D), self.Hkv,
                                 q_abs=lens - nq, v_fmt=vfmt, **feat)


def _cu(nq):
    return torch.tensor(np.concatenate([[0], np.cumsum(nq)]), dtype=torch.int32)


def _q(T, Hq, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    return torch.randn((T, Hq, D), generator=g).to(dtype)


LENS, NQ = [700, 37, 1500, 300, 2100], [1, 1, 5, 300, 64]


def _fp16_caches(h):
    """The reference's cache tensors: 16-bit K / V pages and a Q8_0 K cache."""
    import gfx906_fa
    k16 = torch.zeros((h.NB, BS, h.Hkv, D), dtype=h.dtype, device=dev)
    v16 = torch.zeros_like(k16)
    s = h.slots.to(dev)
    k16.view(-1, h.Hkv, D)[s] = h.key.to(dev)
    v16.view(-1, h.Hkv, D)[s] = h.val.to(dev)
    kq8 = torch.zeros((h.NB, BS, h.Hkv, 136), dtype=torch.uint8, device=dev)
    gfx906_fa.reshape_and_cache_q8(h.key.to(dev), s, kq8)
    return k16, v16, kq8


def _forward_paged(h, q, k16, v16, kq8, **kw):
    fp = _paged_mod()
    return fp.forward_paged(q.to(dev), k16, v16, h.bt.to(dev), torch.tensor(h.lens, dtype=torch.int32, device=dev),
                            _cu(NQ).to(dev), max(NQ), max(h.lens), **kw)


def test_forward_paged_direct_branch():
    h = _Hist(LENS, 8, seed=1)
    k16, v16, kq8 = _fp16_caches(h)
    q = _q(sum(NQ), 48, torch.float16, seed=2)
    out = _forward_paged(h, q, k16, v16, kq8, key_cache_q8=kq8)
    assert out.shape == (sum(NQ), 48 * D) and out.dtype == torch.float32      # the reference's return value
    assert_close(to_np(out).reshape(-1, 48, D), h.oracle(q, NQ, v_q8=False), what="forward_paged direct")


def test_forward_paged_gather_branch_matches_direct(monkeypatch):
    """GFX906_FA_DIRECT_PAGED=0: gather_paged_kv_q8 + Q scatter into
    [B, Hq, max_q, D] + flat forward + unscatter.  Against the oracle, and
    against the direct branch: rows served by the same tensor-core kernel in
    both branches (the prefill chunks) agree within abs 1e-4 / rel 1e-3 as
    the reference's tests/test_direct_paged_bitexact.py:153-154 requires;
    decode rows use the split-K kernel in the direct branch and the tensor-
    core kernel (K dequantised to fp16) in the gather branch, so they are
    held to the oracle tolerance."""
    fp = _paged_mod()
    h = _Hist(LENS, 8, seed=3)
    k16, v16, kq8 = _fp16_caches(h)
    q = _q(sum(NQ), 48, torch.float16, seed=4)
    direct = to_np(_forward_paged(h, q, k16, v16, kq8, key_cache_q8=kq8)).reshape(-1, 48, D)
    for fused in (True, False):
        monkeypatch.setattr(fp, "_DIRECT_PAGED_MODE", "0")
        monkeypatch.setattr(fp, "_FUSED", fused)
        gat = to_np(_forward_paged(h, q, k16, v16, kq8, key_cache_q8=kq8)).reshape(-1, 48, D)
        assert_close(gat, h.oracle(q, NQ, v_q8=False), what=f"forward_paged gather (fused={fused})")
        pre = np.concatenate([np.arange(s, s + n) for s, n in zip(np.cumsum([0] + NQ[:-1]), NQ) if n * 6 > 24])
        assert_close(gat[pre], direct[pre], atol=1e-4, rtol=1e-3, what="gather vs direct (prefill rows)")
        assert_close(gat, direct, what="gather vs direct")


def test_forward_paged_legacy_branch():
    """key_cache_q8=None: gather the 16-bit pages, quantise K on the fly,
    flat forward (the reference's legacy path)."""
    h = _Hist(LENS, 8, seed=5)
    k16, v16, kq8 = _fp16_caches(h)
    q = _q(sum(NQ), 48, torch.float16, seed=6)
    out = to_np(_forward_paged(h, q, k16, v16, kq8, key_cache_q8=None)).reshape(-1, 48, D)
    assert_close(out, h.oracle(q, NQ, v_q8=False), what="forward_paged legacy")


def test_forward_paged_writes_out_in_model_dtype():
    h = _Hist(LENS, 8, seed=7, dtype=torch.bfloat16)
    k16, v16, kq8 = _fp16_caches(h)
    q = _q(sum(NQ), 48, torch.bfloat16, seed=8)
    out = torch.full((sum(NQ), 48, D), float("nan"), dtype=torch.bfloat16, device=dev)
    r = _forward_paged(h, q, k16, v16, kq8, key_cache_q8=kq8, out=out)
    assert r is out
    assert_close(to_np(out.float()), h.oracle(q, NQ, v_q8=False), what="forward_paged out= bf16")


# ---------------------------------------------------------------------------
# vLLM backend Impl
# ---------------------------------------------------------------------------
def _backend():
    pytest.importorskip("vllm")
    import gfx906_fa_backend
    return gfx906_fa_backend


class _FakeLayer(torch.nn.Module):
    """The attributes do_kv_cache_update reads (reference test_backend.py:53-62)."""

    def __init__(self):
        super().__init__()
        self._k_scale = torch.tensor(1.0, device=dev)
        self._v_scale = torch.tensor(1.0, device=dev)
        self._q_scale_float = 1.0


def _impl_step(be, h, nq, v_fmt, legacy, dtype, feat=None, host_lists=True):
    """History of every sequence except its last nq tokens written in one
    do_kv_cache_update call, then one engine step: the new tokens' K/V
    written, then forward over the mixed batch."""
    Hq, Hkv = 48, h.Hkv
    feat = feat or {}
    sinks = feat.get("sinks")
    impl = be.Gfx906FAImpl(num_heads=Hq, head_size=D, scale=1.0 / np.sqrt(D), num_kv_heads=Hkv, alibi_slopes=None,
                           sliding_window=feat.get("window"), kv_cache_dtype="auto",
                           logits_soft_cap=feat.get("softcap"), sinks=None if sinks is None else sinks.to(dev))
    impl._v_fmt = v_fmt
    impl._legacy = legacy
    layer = _FakeLayer()
    kv_cache = torch.zeros((h.NB, 2, BS, Hkv, D), dtype=dtype, device=dev)
    is_new = np.zeros(len(h.slots), bool)
    starts = np.concatenate([[0], np.cumsum(h.lens)[:-1]])
    for b, (L, n) in enumerate(zip(h.lens, nq)):
        is_new[starts[b] + L - n:starts[b] + L] = True
    old, new = np.nonzero(~is_new)[0], np.nonzero(is_new)[0]
    key, val = h.key.to(dev), h.val.to(dev)
    slots = h.slots.to(dev)
    impl.do_kv_cache_update(layer, key[old], val[old], kv_cache, slots[old])
    impl.do_kv_cache_update(layer, key[new], val[new], kv_cache, slots[new])
    T = sum(nq)
    q = _q(T, Hq, dtype, seed=9)
    meta = be.Gfx906FAMetadata(
        num_actual_tokens=T, max_query_len=max(nq), max_seq_len=max(h.lens),
        query_start_loc=_cu(nq).to(dev), seq_lens=torch.tensor(h.lens, dtype=torch.int32, device=dev),
        block_table=h.bt.to(dev), slot_mapping=slots[new],
        query_lens_host=list(nq) if host_lists else None, seq_lens_host=list(h.lens) if host_lists else None)
    output = torch.full((T + 3, Hq * D), float("nan"), dtype=dtype, device=dev)   # vLLM pads the buffer
    res = impl.forward(layer, q.to(dev), key[new], val[new], kv_cache, meta, output=output)
    assert res is output
    return q, output[:T].view(T, Hq, D)


@pytest.mark.parametrize("v_fmt,legacy,dtype", [
    ("fp16", False, torch.float16),
    ("fp16", False, torch.bfloat16),
    ("q8_0", False, torch.bfloat16),
    ("fp16", True, torch.float16),
])
def test_impl_kv_update_then_forward(v_fmt, legacy, dtype):
    be = _backend()
    h = _Hist(LENS, 8, seed=10, dtype=dtype)
    q, out = _impl_step(be, h, NQ, v_fmt, legacy, dtype)
    ref = h.oracle(q, NQ, v_q8=(v_fmt == "q8_0"))
    # model-dtype output: its rounding (<= 2^-9 relative) is inside the relative term
    assert_close(to_np(out.float()), ref, what=f"Impl {v_fmt} legacy={legacy} {dtype}")


def test_impl_without_host_lists():
    be = _backend()
    h = _Hist(LENS, 8, seed=11, dtype=torch.bfloat16)
    q, out = _impl_step(be, h, NQ, "q8_0", False, torch.bfloat16, host_lists=False)
    assert_close(to_np(out.float()), h.oracle(q, NQ, v_q8=True), what="Impl without host lists")


def test_impl_window_softcap_sinks():
    be = _backend()
    h = _Hist(LENS, 8, seed=12, dtype=torch.bfloat16)
    sinks = torch.randn((48,), generator=torch.Generator().manual_seed(3)).to(torch.bfloat16)
    feat = dict(window=400, softcap=20.0, sinks=sinks)
    q, out = _impl_step(be, h, NQ, "q8_0", False, torch.bfloat16, feat=feat)
    ref = h.oracle(q, NQ, v_q8=True, window=400, softcap=20.0, sinks=sinks.float().numpy())
    assert_close(to_np(out.float()), ref, what="Impl window+softcap+sinks")


def test_impl_profiling_run_fills_zeros():
    be = _backend()
    impl = be.Gfx906FAImpl(num_heads=8, head_size=D, scale=0.1, num_kv_heads=2, alibi_slopes=None,
                           sliding_window=None, kv_cache_dtype="auto")
    out = torch.ones((4, 8 * D), dtype=torch.float16, device=dev)
    impl.forward(_FakeLayer(), out, None, None, None, None, output=out)
    assert torch.count_nonzero(out) == 0
