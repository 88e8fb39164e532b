"""Builders for seeded paged-KV test cases (CPU generation, GPU copies)."""
import numpy as np
import torch

import oracle as O
from _util import to_np

ATOL, RTOL = 2e-3, 1e-2          # |out - ref| <= ATOL + RTOL * |ref| (fp32 dequant reference)


class PagedCase:
    """Random paged Q8_0 cache for B sequences: K quantised by the device
    store kernel (bit-exact with the oracle), V fp16 / bf16 / Q8_0 token rows
    ("q8") / Q8_0 page-transposed records ("q8t", [NB, Hkv, bs*D/32*34])."""

    def __init__(self, seq_lens, Hkv, D=128, bs=16, v_fmt="f16", seed=0, extra_pages=7,
                 device="cuda", kv_scale=1.0):
        import gfx906_fa
        g = torch.Generator().manual_seed(seed)
        self.B, self.Hkv, self.D, self.bs = len(seq_lens), Hkv, D, bs
        self.seq_lens = np.asarray(seq_lens, np.int32)
        npg = [(int(L) + bs - 1) // bs for L in seq_lens]
        self.max_blocks = max(1, max(npg))
        NB = sum(npg) + extra_pages
        self.NB = NB
        perm = torch.randperm(NB, generator=g).to(torch.int32)
        bt = torch.full((self.B, self.max_blocks), -1, dtype=torch.int32)
        c = 0
        for b, n in enumerate(npg):
            bt[b, :n] = perm[c:c + n]
            c += n
        self.block_table = bt
        rb = D // 32 * 34
        self.rb = rb
        T = int(sum(seq_lens))
        key = (torch.randn((max(T, 1), Hkv, D), generator=g) * kv_scale).half()
        vdt = torch.bfloat16 if v_fmt == "bf16" else torch.float16
        val = (torch.randn((max(T, 1), Hkv, D), generator=g) * kv_scale).to(vdt)
        # slot of token t of sequence b, vectorised
        if T:
            seq_of = np.repeat(np.arange(self.B), self.seq_lens)
            starts = np.concatenate([[0], np.cumsum(self.seq_lens)[:-1]])
            tpos = np.arange(T) - starts[seq_of]
            slots = bt.numpy()[seq_of, tpos // bs].astype(np.int64) * bs + tpos % bs
            slots = torch.from_numpy(slots)
        else:
            slots = torch.tensor([-1], dtype=torch.int64)
        self.k_cache = torch.zeros((NB, bs, Hkv, rb), dtype=torch.uint8, device=device)
        if v_fmt == "q8":
            self.v_cache = torch.zeros((NB, bs, Hkv, rb), dtype=torch.uint8, device=device)
            mode = 2
        elif v_fmt == "q8t":
            self.v_cache = torch.zeros((NB, Hkv, bs * rb), dtype=torch.uint8, device=device)
            mode = 3
        else:
            self.v_cache = torch.zeros((NB, bs, Hkv, D), dtype=vdt, device=device)
            mode = 1
        gfx906_fa.store_kv(key.to(device), val.to(device), slots.to(device), self.k_cache, self.v_cache, mode)
        self.v_fmt = v_fmt
        self.k_np = to_np(self.k_cache)
        self.v_np = to_np(self.v_cache)
        torch.cuda.synchronize()

    @property
    def scale(self):
        return 1.0 / float(np.sqrt(self.D))

    def _v_strides(self):
        if self.v_fmt == "q8t":
            return (self.Hkv * self.bs * self.rb, 0, self.bs * self.rb)
        vb = self.rb if self.v_fmt == "q8" else 2 * self.D
        return (self.bs * self.Hkv * vb, self.Hkv * vb, vb)

    def oracle_varlen(self, q, q_dtype, n_q, causal=True, q_abs=None, mask=None, pick=None, **feat):
        """q [T, Hq, D] numpy (fp16 / fp32 / bf16-as-uint16).  `feat`:
        softcap / window / sinks / num_blocks of oracle.attention_paged."""
        n_q = np.asarray(n_q, np.int32)
        q_start = np.concatenate([[0], np.cumsum(n_q)[:-1]]).astype(np.int32)
        if causal and q_abs is None:
            q_abs = self.seq_lens - n_q
        return O.attention_paged(q, q_dtype, q_start, n_q, self.k_np, self.v_np,
                                 self.block_table.numpy(), self.seq_lens, self.scale, self.Hkv,
                                 q_abs=q_abs if causal else None, mask=mask, v_fmt=self.v_fmt,
                                 v_strides=self._v_strides(), **feat)

    def oracle_rows(self, q_rows, q_dtype, seq, q_abs_rows, **feat):
        """Selected query tokens only: q_rows [n, Hq, D] are single tokens of
        sequences seq[i] at causal positions q_abs_rows[i] (the token sees
        keys <= q_abs_rows[i]).  Each becomes a one-token pseudo-sequence
        over its sequence's block-table row, so long contexts stay cheap."""
        seq = np.asarray(seq, np.int64)
        n = len(seq)
        bt = self.block_table.numpy()[seq]
        return O.attention_paged(np.ascontiguousarray(q_rows), q_dtype, np.arange(n, dtype=np.int32),
                                 np.ones(n, np.int32), self.k_np, self.v_np, bt, self.seq_lens[seq], self.scale,
                                 self.Hkv, q_abs=np.asarray(q_abs_rows, np.int32), v_fmt=self.v_fmt,
                                 v_strides=self._v_strides(), **feat)

    def oracle_bhsd(self, q, q_dtype, q_abs=None, mask=None, pick=None, **feat):
        """q [B', Hq, Sq, D] padded layout (forward_paged_direct); `pick`
        selects which sequences q belongs to (default: all)."""
        B, Hq, Sq, D = q.shape
        bt = self.block_table.numpy() if pick is None else self.block_table.numpy()[pick]
        sl = self.seq_lens if pick is None else self.seq_lens[pick]
        return O.attention_paged(q, q_dtype, np.zeros(B, np.int32), np.full(B, Sq, np.int32),
                                 self.k_np, self.v_np, bt, sl, self.scale, self.Hkv, q_abs=q_abs, mask=mask,
                                 v_fmt=self.v_fmt, q_strides=(Hq * Sq * D, D, Sq * D),
                                 out_shape=(B, Hq, Sq, D), o_strides=(Hq * Sq * D, D, Sq * D),
                                 v_strides=self._v_strides(), **feat)


def assert_close(out, ref, atol=ATOL, rtol=RTOL, what=""):
    out = np.asarray(out, np.float32)
    ref = np.asarray(ref, np.float32)
    assert out.shape == ref.shape, (out.shape, ref.shape)
    assert np.isfinite(out).all(), f"{what}: non-finite output"
    err = np.abs(out - ref)
    bound = atol + rtol * np.abs(ref)
    bad = err > bound
    rel_rms = float(np.sqrt((err ** 2).mean() / max((ref ** 2).mean(), 1e-30)))
    assert not bad.any(), (f"{what}: {int(bad.sum())} of {bad.size} elements out of tolerance; "
                           f"max err {err.max():.3e}, rel rms {rel_rms:.3e}")
    return rel_rms
