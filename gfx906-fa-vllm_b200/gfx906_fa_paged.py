"""Paged-KV wrapper around the `gfx906_fa` operators (sm_100a build).

Keeps the reference's module API (extension/gfx906_fa_paged.py of
nick413-bit/gfx906-fa-vllm): `forward_paged(...)` with the same arguments and
the same return value ([num_tokens, Hq*D] fp32), the `_gather_kv` /
`_gather_kv_q8` helpers and the GFX906_FA_* environment knobs.  Behind it:

  * key_cache_q8 given (the quantise-at-store design):
      - direct path (default): `gfx906_fa.paged_attention` reads the paged
        Q8 cache in place -- the split-K decode kernel for short query chunks
        and the tensor-core prefill kernel for long ones, decided per
        sequence with no host loop and no padding of the batch to max_q;
      - gather path (GFX906_FA_DIRECT_PAGED=0): `gather_paged_kv_q8` into
        contiguous BHSD buffers, then the flat `gfx906_fa.forward`, as the
        reference's fused path does (gfx906_fa_paged.py:333-445).
  * key_cache_q8 None (legacy): gather 16-bit K/V, quantise K every call with
    `quantize_q8_0`, flat forward (gfx906_fa_paged.py:370-376).

Every path runs on the GPU; a missing `gfx906_fa` extension raises at import.
"""
from __future__ import annotations

import math
import os as _os
import time as _time
from typing import Optional, Tuple

import torch

import gfx906_fa

_DBG = _os.environ.get("GFX906_FA_FWD_DEBUG", "0") == "1"
_FUSED = _os.environ.get("GFX906_FA_FUSED", "1") != "0"
# "auto" and "1": direct paged attention; "0": gather + flat forward.  The
# reference's auto heuristic (B >= MIN_BATCH and max_q <= MAX_SQ) chose
# between two gfx906 kernels with different costs; here the direct path
# covers every batch shape, so the knobs are accepted and only "0" changes
# the path.
_DIRECT_PAGED_MODE = _os.environ.get("GFX906_FA_DIRECT_PAGED", "auto").lower()
_DIRECT_PAGED_MIN_BATCH = int(_os.environ.get("GFX906_FA_DIRECT_PAGED_MIN_BATCH", "2"))
_DIRECT_PAGED_MAX_SQ = int(_os.environ.get("GFX906_FA_DIRECT_PAGED_MAX_SQ", "16"))


def q8_row_bytes(head_size: int) -> int:
    return (head_size // 32) * 34


def kv_cache_views(kv_cache: torch.Tensor, v_fmt: str = "fp16"):
    """Views of one vLLM KV allocation [NB, 2, bs, Hkv, D] (16-bit), the
    backend's cache layout:

    k_q8: uint8 [NB, bs, Hkv, D/32*34] -- dense Q8_0 rows at the start of
          each page;
    v:    the V half [NB, bs, Hkv, D] (fp16 mode), or (q8_0) uint8
          [NB, Hkv, bs*D/32*34] page-transposed Q8_0 records (per kv head the
          fp16 block scales [D/32][bs], then the int8 values [D][bs]) placed
          right after the K rows, so that a page's K and V are one contiguous
          byte range (2*bs*Hkv*D/32*34 bytes, which fits the page's
          2*bs*Hkv*D*2 bytes) and the decode kernel can fetch both with one
          copy.
    """
    NB, two, bs, Hkv, D = kv_cache.shape
    rb = q8_row_bytes(D)
    raw = kv_cache.view(torch.uint8).view(NB, -1)
    k_q8 = raw[:, :bs * Hkv * rb].view(NB, bs, Hkv, rb)
    if v_fmt == "q8_0":
        v = raw[:, bs * Hkv * rb:2 * bs * Hkv * rb].view(NB, Hkv, bs * rb)
    else:
        v = kv_cache[:, 1]
    return k_q8, v


def _should_use_direct_paged(num_seqs: int, max_seqlen_q: int) -> bool:
    """Path choice (reference: gfx906_fa_paged.py:60-70).  Only an explicit
    GFX906_FA_DIRECT_PAGED=0 selects the gather path."""
    return _DIRECT_PAGED_MODE != "0"


def _fwdlog(msg: str) -> None:
    if not _DBG:
        return
    try:
        _os.makedirs("/tmp/gfx906_fa_debug", exist_ok=True)
        with open(f"/tmp/gfx906_fa_debug/fwd-{_os.getpid()}.log", "a") as f:
            f.write(f"[{_time.time():.3f}] {msg}\n")
    except Exception:
        pass


def _gather_kv(key_cache: torch.Tensor, value_cache: torch.Tensor, block_table: torch.Tensor,
               seq_lens: torch.Tensor, max_seqlen_k: int) -> Tuple[torch.Tensor, torch.Tensor]:
    """16-bit paged K/V -> [B, Hkv, max_seqlen_k, D] with positions past
    seq_lens zeroed (reference: gfx906_fa_paged.py:83-145).  Torch indexing
    on the cache's device; used by the legacy path only."""
    num_blocks, block_size, Hkv, D = key_cache.shape
    B = block_table.shape[0]
    nb = (max_seqlen_k + block_size - 1) // block_size
    bt = block_table[:, :nb].to(torch.long)
    k = key_cache[bt].reshape(B, -1, Hkv, D)[:, :max_seqlen_k]
    v = value_cache[bt].reshape(B, -1, Hkv, D)[:, :max_seqlen_k]
    pos = torch.arange(max_seqlen_k, device=seq_lens.device, dtype=seq_lens.dtype)
    keep = (pos.unsqueeze(0) < seq_lens.unsqueeze(1)).view(B, max_seqlen_k, 1, 1).to(k.dtype)
    return (k * keep).permute(0, 2, 1, 3).contiguous(), (v * keep).permute(0, 2, 1, 3).contiguous()


def _gather_kv_q8(key_cache_q8: torch.Tensor, value_cache: torch.Tensor, block_table: torch.Tensor,
                  seq_lens: torch.Tensor, max_seqlen_k: int) -> Tuple[torch.Tensor, torch.Tensor]:
    """Paged K_q8 + V -> contiguous [B, Hkv, max_seqlen_k, ...] with the
    reference's semantics (gfx906_fa_paged.py:148-194): V past seq_lens is
    zero, K there is unspecified.  Runs the bulk-async gather kernel."""
    sk_pad = ((max_seqlen_k + 31) // 32) * 32
    k, v = gfx906_fa.gather_paged_kv_q8(key_cache_q8, value_cache, block_table.to(torch.int32).contiguous(),
                                        seq_lens.to(torch.int32).contiguous(), sk_pad)
    return k[:, :, :max_seqlen_k], v[:, :, :max_seqlen_k]


def forward_paged(
    query: torch.Tensor,            # [num_tokens, Hq, D]
    key_cache: torch.Tensor,        # [num_blocks, block_size, Hkv, D]  16-bit (legacy path only)
    value_cache: torch.Tensor,      # [num_blocks, block_size, Hkv, D]  16-bit (or Q8_0 bytes), or
                                    # [num_blocks, Hkv, block_size*(D/32)*34] page-transposed Q8_0
    block_table: torch.Tensor,      # [num_seqs, max_blocks]            int32
    seq_lens: torch.Tensor,         # [num_seqs]                        int32
    cu_seqlens_q: torch.Tensor,     # [num_seqs+1]                      int32
    max_seqlen_q: int,
    max_seqlen_k: int,
    scale: Optional[float] = None,
    key_cache_q8: Optional[torch.Tensor] = None,   # [num_blocks, bs, Hkv, (D/32)*34] uint8
    q_pad_buf: Optional[torch.Tensor] = None,
    mask_buf: Optional[torch.Tensor] = None,
    k_gather_buf: Optional[torch.Tensor] = None,
    v_gather_buf: Optional[torch.Tensor] = None,
    out: Optional[torch.Tensor] = None,
    query_lens_host: Optional[list] = None,
    seq_lens_host: Optional[list] = None,
    softcap: float = 0.0,
    sliding_window: int = 0,
    sinks: Optional[torch.Tensor] = None,
    output_scale: Optional[torch.Tensor] = None,
) -> torch.Tensor:
    """vLLM-layout paged attention (reference: gfx906_fa_paged.py:197-465).

    Returns [num_tokens, Hq*D] fp32 like the reference, unless `out`
    ([num_tokens, Hq, D] in any float dtype) is given, in which case the
    result is written there directly and `out` is returned.  Causal with
    q_abs = seq_len - n_q when max_seqlen_q > 1 (gfx906_fa_paged.py:289-295);
    decode rows see their whole context.  q_pad_buf / mask_buf are accepted
    for signature compatibility and unused (no padding is needed).

    Beyond the reference: `softcap` (> 0: score -> softcap * tanh(score /
    softcap)), `sliding_window` (> 0: a query at position qp sees keys k with
    qp - k < sliding_window) and `sinks` ([Hq] logits added to each softmax
    denominator), on every path; `output_scale` with an fp8 (e4m3) `out`:
    vLLM's static per-tensor output quantisation, out = e4m3(o / scale)
    (direct path)."""
    num_tokens, Hq, D = query.shape
    num_seqs = block_table.shape[0]
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    bt = block_table if block_table.dtype == torch.int32 else block_table.to(torch.int32)
    sl = seq_lens if seq_lens.dtype == torch.int32 else seq_lens.to(torch.int32)
    bt, sl = bt.contiguous(), sl.contiguous()
    cu = cu_seqlens_q if cu_seqlens_q.dtype == torch.int32 else cu_seqlens_q.to(torch.int32)
    cu = cu.contiguous()

    # page-transposed Q8_0 V is only read by the direct kernels
    v_q8t = value_cache is not None and value_cache.dim() == 3
    if key_cache_q8 is not None and (v_q8t or _should_use_direct_paged(num_seqs, max_seqlen_q)):
        if _DBG:
            _fwdlog(f"forward_paged DIRECT: T={num_tokens} Hq={Hq} B={num_seqs} "
                    f"max_q={max_seqlen_q} max_k={max_seqlen_k}")
        o = out if out is not None else torch.empty((num_tokens, Hq, D), dtype=torch.float32,
                                                    device=query.device)
        gfx906_fa.paged_attention(query, key_cache_q8, value_cache, bt, sl, cu, int(max_seqlen_q),
                                  int(max_seqlen_k), float(scale), out=o, query_lens_host=query_lens_host,
                                  seq_lens_host=seq_lens_host, softcap=float(softcap),
                                  sliding_window=int(sliding_window), sinks=sinks, output_scale=output_scale)
        return o if out is not None else o.view(num_tokens, Hq * D)

    # ---- gather + flat forward (reference fused / legacy paths) -------------
    if output_scale is not None:
        raise NotImplementedError("fp8 output quantisation is implemented on the direct paged path only")
    Sk_pad = ((max_seqlen_k + 31) // 32) * 32
    if key_cache_q8 is not None:
        if _FUSED:
            rb = (D // 32) * 34
            kbuf = k_gather_buf if (k_gather_buf is not None and tuple(k_gather_buf.shape) ==
                                    (num_seqs, key_cache_q8.shape[2], Sk_pad, rb)) else None
            vbuf = v_gather_buf if (v_gather_buf is not None and tuple(v_gather_buf.shape) ==
                                    (num_seqs, value_cache.shape[2], Sk_pad, value_cache.shape[3])) else None
            K_q8, V = gfx906_fa.gather_paged_kv_q8(key_cache_q8, value_cache, bt, sl, Sk_pad,
                                                   k_out=kbuf, v_out=vbuf)
        else:
            K_q8, V = _gather_kv_q8(key_cache_q8, value_cache, bt, sl, max_seqlen_k)
            K_q8, V = K_q8.contiguous(), V.contiguous()
    else:
        K, V = _gather_kv(key_cache, value_cache, bt, sl, max_seqlen_k)
        K_q8 = gfx906_fa.quantize_q8_0(K)
    # pack Q into [B, Hq, max_q, D] with one scatter (no host loop)
    n_q = (cu[1:num_seqs + 1] - cu[:num_seqs]).to(torch.long)
    tok = torch.arange(num_tokens, device=query.device)
    seq_of_tok = torch.repeat_interleave(torch.arange(num_seqs, device=query.device), n_q,
                                         output_size=num_tokens)
    pos_in_seq = tok - cu[:num_seqs].to(torch.long)[seq_of_tok]
    q_padded = torch.zeros((num_seqs, Hq, max_seqlen_q, D), dtype=query.dtype, device=query.device)
    q_padded[seq_of_tok, :, pos_in_seq] = query
    q_abs = (sl.to(torch.long) - n_q).to(torch.int32) if max_seqlen_q > 1 else None
    o_pad = gfx906_fa.forward(q_padded, K_q8, V, float(scale), kv_max=sl, q_abs_offset=q_abs,
                              softcap=float(softcap), sliding_window=int(sliding_window), sinks=sinks)
    o_flat = o_pad[seq_of_tok, :, pos_in_seq]                     # [T, Hq, D] fp32
    if out is not None:
        out.copy_(o_flat)
        return out
    return o_flat.reshape(num_tokens, Hq * D)
