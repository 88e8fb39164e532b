"""Generate the golden fixtures under tests/golden/ from the reference's OWN
CPU-runnable Python (nick413-bit/gfx906-fa-vllm).

Run once in a container that has the reference checked out (path given by
--reference, default $GFX906_REFERENCE); the GPU box never needs it.  The
reference's compiled extension `gfx906_fa` is HIP-only, so a stub module
stands in for it: none of the functions used below call into it.

Reference functions used (imported from the reference tree, not copied):
  * ref_quantize_q8_0_cpu   tests/test_quant.py:29-52
  * dequantize_q8_0         tests/test_q8_roundtrip.py:21-36
  * _ref_gather             tests/test_gather.py:15-38
  * _gather_kv_q8           extension/gfx906_fa_paged.py:148-194
  * _gather_kv              extension/gfx906_fa_paged.py:83-145
  * sdpa_ref                tests/test_inline_causal.py:76-102

Inputs are generated on the CPU from fixed seeds with torch.Generator and are
stored in the fixtures (small shapes only), so the tests never regenerate
them.
"""
from __future__ import annotations

import argparse
import importlib
import os
import sys
import types

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def _import_reference(ref: str):
    stub = types.ModuleType("gfx906_fa")
    sys.modules["gfx906_fa"] = stub
    sys.path.insert(0, os.path.join(ref, "extension"))
    sys.path.insert(0, os.path.join(ref, "tests"))
    paged = importlib.import_module("gfx906_fa_paged")
    tq = importlib.import_module("test_quant")
    trt = importlib.import_module("test_q8_roundtrip")
    tg = importlib.import_module("test_gather")
    tg.dev = torch.device("cpu")          # its module-level device is "cuda"
    tic = importlib.import_module("test_inline_causal")
    return paged, tq, trt, tg, tic


def _randn_f16(g, shape, scale=1.0):
    return (torch.randn(shape, generator=g, dtype=torch.float32) * scale).to(torch.float16)


def make_quant(tq, out):
    """Dense Q8_0 quantisation: reference CPU function on assorted inputs."""
    g = torch.Generator().manual_seed(1234)
    cases = {}
    x = _randn_f16(g, (64, 128))
    cases["randn"] = x
    y = _randn_f16(g, (32, 128))
    o = torch.rand((32, 128), generator=g) < 0.01            # 1 % outliers x8 (config 2)
    y = torch.where(o, y * 8, y)
    cases["outliers"] = y
    z = torch.zeros((4, 128), dtype=torch.float16)
    z[1, 5] = 1.0                                             # single non-zero per block
    z[2, :32] = torch.arange(32, dtype=torch.float16) - 16    # integer ramp (ties)
    z[3] = torch.tensor(65504.0, dtype=torch.float16)         # fp16 max
    cases["edges"] = z
    s = (torch.randn((8, 64), generator=g) * 1e-6).to(torch.float16)   # subnormal fp16
    cases["subnormal"] = s
    w = _randn_f16(g, (3, 5, 64), 0.5)                         # rank-3, D=64
    cases["rank3_d64"] = w
    for name, v in cases.items():
        out[f"quant_{name}_x"] = v.numpy()
        out[f"quant_{name}_y"] = tq.ref_quantize_q8_0_cpu(v).numpy()


def make_gather(paged, tg, out):
    """Fused-gather semantics: the reference's torch gathers on seeded inputs
    (the shapes of tests/test_gather.py:test_gather_basic / _matches_old_path)."""
    for name, (NB, bs, Hkv, D, B, MB, Sk, seq_lens, seed) in {
        "basic": (8, 16, 2, 64, 3, 4, 64, [0, 30, 64], 0),
        "old_path": (32, 16, 2, 128, 4, 4, 64, [10, 32, 48, 5], 123),
    }.items():
        g = torch.Generator().manual_seed(seed)
        rb = (D // 32) * 34
        kc = torch.randint(0, 256, (NB, bs, Hkv, rb), generator=g, dtype=torch.uint8)
        vc = _randn_f16(g, (NB, bs, Hkv, D))
        bt = torch.randint(0, NB, (B, MB), generator=g, dtype=torch.int32)
        sl = torch.tensor(seq_lens, dtype=torch.int32)
        k_ref, v_ref = tg._ref_gather(kc, vc, bt, sl, Sk)
        max_sk = int(max(seq_lens))
        k_old, v_old = paged._gather_kv_q8(kc, vc, bt, sl, max_sk)
        p = f"gather_{name}_"
        out[p + "k_cache"] = kc.numpy()
        out[p + "v_cache"] = vc.numpy()
        out[p + "block_table"] = bt.numpy()
        out[p + "seq_lens"] = sl.numpy()
        out[p + "Sk"] = np.array(Sk)
        out[p + "k_ref"] = k_ref.numpy()
        out[p + "v_ref"] = v_ref.numpy()
        out[p + "k_old"] = k_old.numpy()
        out[p + "v_old"] = v_old.numpy()


def make_config1(paged, tq, trt, tic, out):
    """1 sequence, Hq/Hkv = 8/2, D = 128, block_size 16,
    512-token causal prefill plus one decode token (L = 513).  K and V are
    quantised to Q8_0 with the reference CPU quantiser, paged through a seeded
    random block_table, gathered with _gather_kv_q8, dequantised with
    dequantize_q8_0 and run through sdpa_ref (fp32, causal)."""
    g = torch.Generator().manual_seed(2024)
    Hq, Hkv, D, bs, L = 8, 2, 128, 16, 513
    n_pages = (L + bs - 1) // bs                    # 33
    NB = 40
    q = _randn_f16(g, (L, Hq, D))
    k = _randn_f16(g, (L, Hkv, D))
    v = _randn_f16(g, (L, Hkv, D))
    perm = torch.randperm(NB, generator=g)[:n_pages].to(torch.int32)
    bt = perm.view(1, n_pages)
    rb = (D // 32) * 34
    k_q8 = tq.ref_quantize_q8_0_cpu(k)              # [L, Hkv, rb]
    v_q8 = tq.ref_quantize_q8_0_cpu(v)
    kc = torch.zeros((NB, bs, Hkv, rb), dtype=torch.uint8)
    vc = torch.zeros((NB, bs, Hkv, rb), dtype=torch.uint8)
    for t in range(L):
        kc[bt[0, t // bs], t % bs] = k_q8[t]
        vc[bt[0, t // bs], t % bs] = v_q8[t]
    scale = 1.0 / (D ** 0.5)
    outs = {}
    for tag, (Lk, n_q) in {"prefill": (512, 512), "decode": (513, 1)}.items():
        sl = torch.tensor([Lk], dtype=torch.int32)
        kg, vg = paged._gather_kv_q8(kc, vc, bt, sl, Lk)     # [1, Hkv, Lk, rb]
        kd = trt.dequantize_q8_0(kg, D)[0].permute(1, 0, 2)  # [Lk, Hkv, D]
        vd = trt.dequantize_q8_0(vg, D)[0].permute(1, 0, 2)
        qs = q[Lk - n_q:Lk].float()
        # sdpa_ref takes fp16 K/V but only calls .float() on them; hand it the
        # fp32 dequantised tensors directly (no extra rounding).
        outs[tag] = tic.sdpa_ref(qs, kd, vd, Hq, Hkv, scale, n_q)   # [n_q, Hq, D]
    out["cfg1_q"] = q.numpy()
    out["cfg1_k"] = k.numpy()
    out["cfg1_v"] = v.numpy()
    out["cfg1_block_table"] = bt.numpy()
    out["cfg1_k_q8_ref"] = k_q8.numpy()
    out["cfg1_v_q8_ref"] = v_q8.numpy()
    out["cfg1_prefill_out"] = outs["prefill"][::8].numpy()      # every 8th query token
    out["cfg1_decode_out"] = outs["decode"].numpy()
    out["cfg1_scale"] = np.array(scale, dtype=np.float64)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("GFX906_REFERENCE"),
                    help="checkout of the reference project (or set $GFX906_REFERENCE)")
    args = ap.parse_args()
    if not args.reference:
        ap.error("--reference (or $GFX906_REFERENCE) is required")
    torch.set_num_threads(4)
    paged, tq, trt, tg, tic = _import_reference(args.reference)
    quant, gath, cfg1 = {}, {}, {}
    make_quant(tq, quant)
    make_gather(paged, tg, gath)
    make_config1(paged, tq, trt, tic, cfg1)
    np.savez_compressed(os.path.join(HERE, "quant_golden.npz"), **quant)
    np.savez_compressed(os.path.join(HERE, "gather_golden.npz"), **gath)
    np.savez_compressed(os.path.join(HERE, "config1_golden.npz"), **cfg1)
    for f in ("quant_golden.npz", "gather_golden.npz", "config1_golden.npz"):
        print(f, os.path.getsize(os.path.join(HERE, f)))


if __name__ == "__main__":
    main()
