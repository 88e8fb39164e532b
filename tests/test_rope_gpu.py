"""Fused RoPE + KV store (gfx906_fa.rope_store_kv and the backend's
do_rope_and_kv_cache_update) against the oracle: query and key rotated in
fp32 and rounded once (bit-exact), the rotated key quantised to Q8_0 in the
cache (bit-exact, the quantiser pinned to the reference's), V stored per
v_mode.  The reference backend has no RoPE fusion
(extension/gfx906_fa_backend.py:444-445)."""
import numpy as np
import pytest
import torch

import oracle as O
from _util import to_np

pytestmark = pytest.mark.gpu
dev = "cuda"
D, BS = 128, 16


def _cos_sin(max_pos, rot, base=10000.0):
    """vLLM's RotaryEmbedding cache: [max_pos, rot] = cat(cos, sin)."""
    inv = 1.0 / (base ** (torch.arange(0, rot, 2, dtype=torch.float32) / rot))
    f = torch.outer(torch.arange(max_pos, dtype=torch.float32), inv)
    return torch.cat([f.cos(), f.sin()], dim=-1)


def _case(T, Hq, Hkv, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn((T, Hq, D), generator=g).to(dtype)
    k = torch.randn((T, Hkv, D), generator=g).to(dtype)
    v = torch.randn((T, Hkv, D), generator=g).to(dtype)
    pos = torch.randint(0, 4000, (T,), generator=g, dtype=torch.int64)
    NB = (T + BS - 1) // BS + 3
    slots = torch.randperm(NB * BS, generator=g)[:T].to(torch.int64)
    slots[::7] = -1                                   # padded tokens: rotated, not stored
    return q, k, v, pos, slots, NB


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("neox", [True, False])
@pytest.mark.parametrize("rot", [128, 64])
@pytest.mark.parametrize("cs_dtype", [torch.float32, torch.bfloat16])
def test_rope_store_bitexact(dtype, neox, rot, cs_dtype):
    import gfx906_fa
    T, Hq, Hkv = 77, 48, 8
    q, k, v, pos, slots, NB = _case(T, Hq, Hkv, dtype, seed=rot + int(neox))
    cs = _cos_sin(4096, rot).to(cs_dtype)
    qd, kd, vd = q.to(dev), k.to(dev), v.to(dev)
    kc = torch.zeros((NB, BS, Hkv, 136), dtype=torch.uint8, device=dev)
    vc = torch.zeros((NB, BS, Hkv, D), dtype=dtype, device=dev)
    gfx906_fa.rope_store_kv(qd, kd, vd, pos.to(dev), cs.to(dev), neox, slots.to(dev), kc, vc, 1)
    tag = "bf16" if dtype == torch.bfloat16 else None
    csf = cs.float().numpy()
    q_ref = O.rope(to_np(q), tag, pos.numpy(), csf, neox)
    k_ref = O.rope(to_np(k), tag, pos.numpy(), csf, neox)
    assert np.array_equal(to_np(qd), q_ref), "query rotation"
    assert np.array_equal(to_np(kd), k_ref), "key rotation"
    kc_ref = np.zeros((NB, BS, Hkv, 136), np.uint8)
    O.reshape_and_cache(k_ref, slots.numpy(), kc_ref, dtype=tag)
    assert np.array_equal(to_np(kc), kc_ref), "Q8_0 K of the rotated key"
    vc_ref = np.zeros((NB, BS, Hkv, D), np.uint16)
    O.store_v16(to_np(v).view(np.uint16), slots.numpy(), vc_ref)
    assert np.array_equal(to_np(vc).view(np.uint16), vc_ref), "V rows"


def test_rope_store_page_transposed_v_and_no_query():
    import gfx906_fa
    T, Hkv = 50, 8
    _, k, v, pos, slots, NB = _case(T, 8, Hkv, torch.bfloat16, seed=3)
    cs = _cos_sin(4096, 128)
    kd = k.to(dev)
    kc = torch.zeros((NB, BS, Hkv, 136), dtype=torch.uint8, device=dev)
    vc = torch.zeros((NB, Hkv, BS * 136), dtype=torch.uint8, device=dev)
    gfx906_fa.rope_store_kv(None, kd, v.to(dev), pos.to(dev), cs.to(dev), True, slots.to(dev), kc, vc, 3)
    k_ref = O.rope(to_np(k), "bf16", pos.numpy(), cs.numpy(), True)
    assert np.array_equal(to_np(kd), k_ref)
    vc_ref = np.zeros((NB, Hkv, BS * 136), np.uint8)
    O.store_v_q8t(to_np(v), slots.numpy(), vc_ref, BS, dtype="bf16")
    assert np.array_equal(to_np(vc), vc_ref)


@pytest.mark.parametrize("v_fmt", ["fp16", "q8_0"])
def test_backend_fused_rope_hook_matches_unfused(v_fmt):
    """Gfx906FAImpl.do_rope_and_kv_cache_update (vLLM's fused RoPE + KV
    cache hook) leaves the same query, key and cache bytes as rotating with
    the oracle and then calling do_kv_cache_update."""
    pytest.importorskip("vllm")
    import gfx906_fa_backend as be
    T, Hq, Hkv = 40, 48, 8
    q, k, v, pos, slots, NB = _case(T, Hq, Hkv, torch.bfloat16, seed=9)
    cs = _cos_sin(4096, 128).to(torch.bfloat16)
    impl = be.Gfx906FAImpl(num_heads=Hq, head_size=D, scale=0.088, num_kv_heads=Hkv, alibi_slopes=None,
                           sliding_window=None, kv_cache_dtype="auto")
    impl._v_fmt = v_fmt
    assert impl.fused_rope_kvcache_supported()
    kv_a = torch.zeros((NB, 2, BS, Hkv, D), dtype=torch.bfloat16, device=dev)
    kv_b = torch.zeros_like(kv_a)
    qa, ka = q.reshape(T, Hq * D).to(dev), k.reshape(T, Hkv * D).to(dev)     # vLLM passes 2-D views
    impl.do_rope_and_kv_cache_update(None, qa, ka, v.reshape(T, Hkv * D).to(dev), pos.to(dev), cs.to(dev), True,
                                     kv_a, slots.to(dev))
    q_ref = O.rope(to_np(q), "bf16", pos.numpy(), cs.float().numpy(), True)
    k_ref = O.rope(to_np(k), "bf16", pos.numpy(), cs.float().numpy(), True)
    assert np.array_equal(to_np(qa).reshape(T, Hq, D), q_ref)
    assert np.array_equal(to_np(ka).reshape(T, Hkv, D), k_ref)
    k_rot = torch.from_numpy(k_ref.view(np.int16)).view(torch.bfloat16).to(dev)
    impl.do_kv_cache_update(None, k_rot, v.to(dev), kv_b, slots.to(dev))
    assert torch.equal(kv_a.view(torch.uint8), kv_b.view(torch.uint8))
