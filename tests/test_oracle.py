"""Pins the CPU oracle against the reference's own golden vectors.

The fixtures in tests/golden/ were produced by tests/golden/make_golden.py from
the reference's CPU-runnable Python (nick413-bit/gfx906-fa-vllm):
ref_quantize_q8_0_cpu (tests/test_quant.py:29-52), _ref_gather
(tests/test_gather.py:15-38), _gather_kv_q8 (extension/gfx906_fa_paged.py:148-194),
dequantize_q8_0 (tests/test_q8_roundtrip.py:21-36) and sdpa_ref
(tests/test_inline_causal.py:76-102).
"""
import os

import numpy as np
import pytest

import oracle as O

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _load(name):
    return np.load(os.path.join(GOLD, name))


@pytest.mark.parametrize("case", ["randn", "outliers", "edges", "subnormal", "rank3_d64"])
def test_quant_matches_reference_cpu(case):
    """The oracle restates the device kernel in fp32; the reference's CPU
    function computes d and 1/d in double, so the reference's own tolerance
    applies: at most 1 LSB, under 1 % of bytes (tests/test_quant.py:66-73)."""
    g = _load("quant_golden.npz")
    x, y = g[f"quant_{case}_x"], g[f"quant_{case}_y"]
    o = O.quantize_q8_0(x)
    assert o.shape == y.shape
    d = np.abs(o.astype(np.int32) - y.astype(np.int32))
    assert d.max() <= 1
    assert (d > 0).mean() < 0.01


def test_quant_block_rules():
    """Kernel rules of gfx906_fa_quant.cu:51-84 on hand-made blocks."""
    x = np.zeros((3, 32), np.float32)
    x[1, :] = np.linspace(-2, 2, 32)
    x[2, 0] = 127.0                # amax 127 -> d = 1, id = 1
    x[2, 1] = 2.5                  # rintf(2.5) = 2 (half to even)
    x[2, 2] = -3.5                 # rintf(-3.5) = -4
    y = O.quantize_q8_0(x)
    assert (y[0] == 0).all()                                     # zero block: d = 0, q = 0
    assert y[1, 2 + 31].view(np.int8) == 127 and y[1, 2].view(np.int8) == -127
    assert y[2, 2:5].view(np.int8).tolist() == [127, 2, -4]
    d = y[2, :2].copy().view(np.float16)[0]
    assert d == np.float16(1.0)


@pytest.mark.parametrize("case", ["basic", "old_path"])
def test_gather_matches_reference(case):
    g = _load("gather_golden.npz")
    p = f"gather_{case}_"
    sl = g[p + "seq_lens"]
    ko, vo = O.gather(g[p + "k_cache"], g[p + "v_cache"], g[p + "block_table"], sl, int(g[p + "Sk"]))
    assert np.array_equal(vo, g[p + "v_ref"])                    # V exact incl. zero tail
    for s, L in enumerate(sl):
        assert np.array_equal(ko[s, :, :L], g[p + "k_ref"][s, :, :L])   # K exact on valid rows
    ms = int(sl.max())
    assert np.array_equal(vo[:, :, :ms], g[p + "v_old"])


def test_dequant_roundtrip():
    """store -> gather -> dequant equals dense quant -> dequant
    (tests/test_q8_roundtrip.py:39-132, tolerance 1e-6 there; exact here)."""
    rng = np.random.default_rng(0)
    T, Hkv, D, bs, NB = 128, 8, 128, 16, 64
    key = (rng.standard_normal((T, Hkv, D)) * 0.5).astype(np.float16)
    cache = np.zeros((NB, bs, Hkv, O.row_bytes(D)), np.uint8)
    bt = np.arange(T // bs, dtype=np.int32).reshape(1, -1)
    slots = (bt[0, np.arange(T) // bs].astype(np.int64) * bs + np.arange(T) % bs)
    O.reshape_and_cache(key, slots, cache)
    vc = np.zeros((NB, bs, Hkv, D), np.float16)
    k_out, _ = O.gather(cache, vc, bt, np.array([T], np.int32), T)
    rec = O.dequantize_q8_0(k_out, D)[0].transpose(1, 0, 2)
    ref = O.dequantize_q8_0(O.quantize_q8_0(key.reshape(-1, D)), D).reshape(T, Hkv, D)
    assert np.array_equal(rec, ref)


def _cfg1_cache():
    c = _load("config1_golden.npz")
    bt = c["cfg1_block_table"]
    kq, vq = c["cfg1_k_q8_ref"], c["cfg1_v_q8_ref"]
    NB, bs, Hkv, L = 40, 16, 2, 513
    kc = np.zeros((NB, bs, Hkv, 136), np.uint8)
    vc = np.zeros_like(kc)
    for t in range(L):
        kc[bt[0, t // bs], t % bs] = kq[t]
        vc[bt[0, t // bs], t % bs] = vq[t]
    return c, kc, vc, bt


def test_config1_attention_matches_reference():
    """Config 1 pipeline of the reference (quant -> paged -> _gather_kv_q8 ->
    dequantize_q8_0 -> causal sdpa_ref) against the oracle's paged attention."""
    c, kc, vc, bt = _cfg1_cache()
    q, sc = c["cfg1_q"], float(c["cfg1_scale"])
    o = O.attention_paged(q[:512].copy(), None, np.array([0]), np.array([512]), kc, vc, bt,
                          np.array([512]), sc, 2, q_abs=np.array([0]), v_q8=True)
    assert np.abs(o[::8] - c["cfg1_prefill_out"]).max() < 1e-5
    o = O.attention_paged(q[512:513].copy(), None, np.array([0]), np.array([1]), kc, vc, bt,
                          np.array([513]), sc, 2, q_abs=np.array([512]), v_q8=True)
    assert np.abs(o - c["cfg1_decode_out"]).max() < 1e-5


def test_f16_conversion_matches_numpy():
    rng = np.random.default_rng(1)
    v = np.concatenate([rng.standard_normal(4000) * s for s in (1e-7, 1e-5, 1e-3, 1, 1e3, 6e4)])
    v = np.concatenate([v, [0.0, -0.0, 65504.0, 65519.9, 65520.0, 1e9, -1e9, 5.96e-8, 2.98e-8, 2.99e-8]])
    v = v.astype(np.float32)
    with np.errstate(over="ignore"):
        ref = v.astype(np.float16).view(np.uint16)
    got = np.array([O.lib().q8o_f32_to_f16(float(x)) for x in v], dtype=np.uint16)
    assert np.array_equal(got, ref)


def _np_attention(q, k, v, scale, kv_len, q_abs=None):
    """Direct numpy fp64 attention on dense [Hq, Sq, D] / [Hkv, Skv, D]."""
    Hq, Sq, D = q.shape
    Hkv = k.shape[0]
    G = Hq // Hkv
    out = np.zeros((Hq, Sq, D))
    for hq in range(Hq):
        for t in range(Sq):
            lim = kv_len if q_abs is None else min(kv_len, q_abs + t + 1)
            if lim <= 0:
                continue
            s = k[hq // G, :lim] @ q[hq, t].astype(np.float64) * scale
            p = np.exp(s - s.max())
            out[hq, t] = p @ v[hq // G, :lim] / p.sum()
    return out


@pytest.mark.parametrize("v_kind", ["f16", "bf16", "q8"])
def test_attention_bhsd_matches_direct_numpy(v_kind):
    """The flat-layout oracle (one page of Skv tokens per sequence) against a
    plain numpy computation on dequantised tensors."""
    rng = np.random.default_rng(4)
    B, Hq, Hkv, Sq, Skv, D = 2, 4, 2, 3, 40, 128
    q = rng.standard_normal((B, Hq, Sq, D)).astype(np.float32)
    k16 = rng.standard_normal((B, Hkv, Skv, D)).astype(np.float16)
    kq = O.quantize_q8_0(k16)
    v32 = rng.standard_normal((B, Hkv, Skv, D)).astype(np.float32)
    if v_kind == "q8":
        v_arr = O.quantize_q8_0(v32.astype(np.float16))
        v_deq = O.dequantize_q8_0(v_arr, D)
    elif v_kind == "bf16":
        v_arr = (v32.view(np.uint32) >> 16).astype(np.uint16)          # truncation to bf16 bits
        v_deq = (v_arr.astype(np.uint32) << 16).view(np.float32)
    else:
        v_arr = v32.astype(np.float16)
        v_deq = v_arr.astype(np.float32)
    kv_max = np.array([Skv, 17], np.int32)
    qa = np.array([Skv - Sq, 5], np.int32)
    o = O.attention_bhsd(q, None, kq, v_arr, 0.125, kv_max=kv_max, q_abs=qa, v_q8=v_kind == "q8")
    kd = O.dequantize_q8_0(kq, D)
    for b in range(B):
        ref = _np_attention(q[b], kd[b], v_deq[b], 0.125, int(kv_max[b]), int(qa[b]))
        assert np.abs(o[b] - ref).max() < 1e-5


def test_q8t_layout_matches_q8_rows():
    """The page-transposed Q8_0 V records (store_v_q8t) hold exactly the
    blocks of the Q8_0 row store: attention over either layout is identical,
    and every record byte maps back to its row byte."""
    rng = np.random.default_rng(5)
    Hkv, D, bs, NB = 2, 128, 16, 9
    lens = np.array([40, 75], np.int32)
    T = int(lens.sum())
    val = rng.standard_normal((T, Hkv, D)).astype(np.float16)
    key = rng.standard_normal((T, Hkv, D)).astype(np.float16)
    perm = rng.permutation(NB).astype(np.int32)
    bt = np.full((2, 5), -1, np.int32)
    bt[0, :3], bt[1, :5] = perm[:3], perm[3:8]
    slots = np.concatenate([bt[0, np.arange(40) // bs] * bs + np.arange(40) % bs,
                            bt[1, np.arange(75) // bs] * bs + np.arange(75) % bs]).astype(np.int64)
    rb = O.row_bytes(D)
    k_cache = np.zeros((NB, bs, Hkv, rb), np.uint8)
    O.reshape_and_cache(key, slots, k_cache)
    v_rows = np.zeros((NB, bs, Hkv, rb), np.uint8)
    O.reshape_and_cache(val, slots, v_rows)
    v_rec = np.zeros((NB, Hkv, bs * rb), np.uint8)
    O.store_v_q8t(val, slots, v_rec, bs)
    nb = D // 32
    for page in range(NB):
        for h in range(Hkv):
            for t in range(bs):
                row = v_rows[page, t, h].reshape(nb, 34)
                rec = v_rec[page, h]
                for j in range(nb):
                    assert rec[2 * (j * bs + t)] == row[j, 0] and rec[2 * (j * bs + t) + 1] == row[j, 1]
                    got = rec[2 * nb * bs + (j * 32) * bs + t:2 * nb * bs + (j * 32 + 32) * bs + t:bs]
                    assert np.array_equal(got, row[j, 2:])
    q = rng.standard_normal((T, 8, D)).astype(np.float16)
    q_start = np.array([0, 40], np.int32)
    args = (q, None, q_start, lens, k_cache)
    kw = dict(q_abs=np.zeros(2, np.int32))
    a = O.attention_paged(*args, v_rows, bt, lens, 0.088, Hkv, v_fmt="q8", **kw)
    b = O.attention_paged(*args, v_rec, bt, lens, 0.088, Hkv, v_fmt="q8t",
                          v_strides=(Hkv * bs * rb, 0, bs * rb), **kw)
    assert np.array_equal(a, b)


def test_torch_path_matches_c_oracle():
    """The torch restatement of the reference's CPU pipeline (gather,
    dequantize_q8_0, repeat_interleave, SDPA with the causal keep-mask) and
    the C oracle agree on a mixed decode / prefill batch."""
    import torch
    import torch_path as TP
    rng = np.random.default_rng(5)
    Hq, Hkv, D, bs = 12, 2, 128, 16
    lens, nq = [200, 37, 64], [1, 1, 20]
    NB = sum((L + bs - 1) // bs for L in lens) + 3
    perm = rng.permutation(NB).astype(np.int32)
    MB = max((L + bs - 1) // bs for L in lens)
    bt = np.zeros((len(lens), MB), np.int32)
    c = 0
    for b, L in enumerate(lens):
        n = (L + bs - 1) // bs
        bt[b, :n] = perm[c:c + n]
        c += n
    kc = O.quantize_q8_0(rng.standard_normal((NB, bs, Hkv, D)).astype(np.float16))
    vc = rng.standard_normal((NB, bs, Hkv, D)).astype(np.float16)
    q = rng.standard_normal((sum(nq), Hq, D)).astype(np.float16)
    scale = 1 / np.sqrt(D)
    nqa = np.array(nq, np.int32)
    ref = O.attention_paged(q, None, np.concatenate([[0], np.cumsum(nq)[:-1]]).astype(np.int32), nqa, kc, vc, bt,
                            np.array(lens, np.int32), scale, Hkv, q_abs=np.array(lens, np.int32) - nqa)
    out = TP.attention_varlen(torch.from_numpy(q), torch.from_numpy(kc), torch.from_numpy(vc), torch.from_numpy(bt),
                              lens, nq, scale)
    assert np.abs(out.numpy() - ref).max() < 1e-4
