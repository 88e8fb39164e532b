"""The reference's own torch CPU path for paged-Q8 attention, restated.

TEST INFRASTRUCTURE ONLY: used by bench.py's reference arm / cpu_baseline
leg and by tests/, never by the shipped package.

The reference checks its kernels against a pure-torch pipeline that runs on
the CPU as well: page gather by fancy indexing
(extension/gfx906_fa_paged.py:148-194, `_gather_kv_q8`), Q8_0 dequantisation
(tests/test_q8_roundtrip.py:21-36, `dequantize_q8_0`: int8 times the fp16
block scale in fp32), GQA by repeat_interleave and
torch.nn.functional.scaled_dot_product_attention with an explicit causal
keep-mask k <= (Sk - Sq) + i (tests/test_paged.py:120-149).  This module
performs those steps in the same order with torch on the host, so that the
CPU baseline is the reference's algorithm and torch's own SDPA kernel, timed
on the host's cores.  The reference files are not read at run time.
"""
from __future__ import annotations

import torch

QK, BLOCK_BYTES = 32, 34


def gather_kv_q8(key_cache_q8: torch.Tensor, value_cache: torch.Tensor, block_table: torch.Tensor,
                 seq_lens: torch.Tensor, max_seqlen_k: int):
    """Paged [NB, bs, Hkv, row] caches -> [B, Hkv, Sk, row] (V rows past
    seq_lens zeroed), by fancy indexing over the block table."""
    NB, bs, Hkv, _ = key_cache_q8.shape
    B = block_table.shape[0]
    nb = (max_seqlen_k + bs - 1) // bs
    bt = block_table[:, :nb].to(torch.long)
    k = key_cache_q8[bt].view(B, -1, Hkv, key_cache_q8.shape[-1])[:, :max_seqlen_k]
    v = value_cache[bt].view(B, -1, Hkv, value_cache.shape[-1])[:, :max_seqlen_k]
    pos = torch.arange(max_seqlen_k, dtype=seq_lens.dtype)
    keep = (pos.unsqueeze(0) < seq_lens.unsqueeze(1)).view(B, max_seqlen_k, 1, 1)
    v = v * keep.to(v.dtype)
    return k.permute(0, 2, 1, 3).contiguous(), v.permute(0, 2, 1, 3).contiguous()


def dequantize_q8_0(q8: torch.Tensor, D: int) -> torch.Tensor:
    """uint8 [..., D/32*34] -> fp32 [..., D]: int8 value times fp16 scale."""
    prefix = q8.shape[:-1]
    blk = q8.reshape(-1, D // QK, BLOCK_BYTES)
    scale = blk[:, :, :2].contiguous().view(torch.float16).float()[..., 0:1]
    q = blk[:, :, 2:].view(torch.int8).float()
    return (q * scale).reshape(*prefix, D)


def attention_varlen(query: torch.Tensor, key_cache_q8: torch.Tensor, value_cache: torch.Tensor,
                     block_table: torch.Tensor, seq_lens, q_lens, scale: float, v_q8: bool = False) -> torch.Tensor:
    """query [T, Hq, D] (vLLM layout, sequences back to back) -> fp32
    [T, Hq, D]; causal with the query chunk ending at the last key."""
    T, Hq, D = query.shape
    Hkv = key_cache_q8.shape[2]
    out = torch.empty((T, Hq, D), dtype=torch.float32)
    t0 = 0
    for s, (Lk, n) in enumerate(zip(seq_lens, q_lens)):
        Lk, n = int(Lk), int(n)
        k8, v = gather_kv_q8(key_cache_q8, value_cache, block_table[s:s + 1],
                             torch.tensor([Lk], dtype=torch.int32), Lk)
        k = dequantize_q8_0(k8, D)
        v = dequantize_q8_0(v, D) if v_q8 else v.float()
        if Hq > Hkv:
            k = k.repeat_interleave(Hq // Hkv, dim=1)
            v = v.repeat_interleave(Hq // Hkv, dim=1)
        q = query[t0:t0 + n].permute(1, 0, 2).unsqueeze(0).float()
        mask = None
        if n > 1:
            mask = torch.arange(Lk).unsqueeze(0) <= (torch.arange(n).unsqueeze(1) + (Lk - n))
        o = torch.nn.functional.scaled_dot_product_attention(q, k, v, attn_mask=mask, scale=scale)
        out[t0:t0 + n] = o[0].permute(1, 0, 2)
        t0 += n
    return out
