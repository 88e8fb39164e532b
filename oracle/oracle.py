"""numpy/ctypes front end of the CPU oracle (oracle/q8_oracle.c).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and
bench.py's CPU-baseline legs, never by the shipped package.  Every function
restates a step of the reference (nick413-bit/gfx906-fa-vllm); the C source
header maps each one to the reference file:line it follows.

Arrays are numpy; 16-bit floats travel as numpy float16 (fp16) or as uint16
tagged with dtype="bf16".
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
SRC = os.path.join(HERE, "q8_oracle.c")
LIB = os.path.join(HERE, "libq8oracle.so")

DT_F16, DT_BF16, DT_F32 = 0, 1, 2
QK = 32
BLOCK_BYTES = 34


def row_bytes(D: int) -> int:
    return (D // QK) * BLOCK_BYTES


def build(force: bool = False) -> str:
    """Compile the oracle with gcc (IEEE float, no fast-math, OpenMP)."""
    if force or not os.path.exists(LIB) or os.path.getmtime(LIB) < os.path.getmtime(SRC):
        tmp = LIB + f".tmp{os.getpid()}"
        subprocess.check_call(["gcc", "-O2", "-fopenmp", "-fPIC", "-shared", "-Wall",
                               "-o", tmp, SRC, "-lm"])
        os.replace(tmp, LIB)
    return LIB


_lib = None


def lib():
    global _lib
    if _lib is None:
        _lib = ctypes.CDLL(build())
        _lib.q8o_f32_to_f16.restype = ctypes.c_uint16
        _lib.q8o_f32_to_f16.argtypes = [ctypes.c_float]
        _lib.q8o_f16_to_f32.restype = ctypes.c_float
        _lib.q8o_f16_to_f32.argtypes = [ctypes.c_uint16]
    return _lib


def _p(a):
    return ctypes.c_void_p(a.ctypes.data) if a is not None else ctypes.c_void_p(0)


def _i64(x):
    return ctypes.c_int64(int(x))


def _dtype_code(x: np.ndarray, dtype: str | None) -> int:
    if dtype == "bf16":
        assert x.dtype == np.uint16
        return DT_BF16
    if x.dtype == np.float16:
        return DT_F16
    if x.dtype == np.float32:
        return DT_F32
    raise TypeError(f"unsupported element type {x.dtype} / {dtype}")


# --------------------------------------------------------------------------
# Q8_0 quantisation (gfx906_fa_quant.cu:45-129)
# --------------------------------------------------------------------------
def quantize_q8_0(x: np.ndarray, dtype: str | None = None) -> np.ndarray:
    """[..., D] -> uint8 [..., D/32*34]; bit-exact restatement of the kernel."""
    x = np.ascontiguousarray(x)
    D = x.shape[-1]
    assert D % QK == 0
    N = x.size // D
    out = np.empty(x.shape[:-1] + (row_bytes(D),), dtype=np.uint8)
    lib().q8o_quantize_dense(_p(x), ctypes.c_int(_dtype_code(x, dtype)), _p(out),
                             _i64(N), ctypes.c_int(D))
    return out


def reshape_and_cache(key: np.ndarray, slot_mapping: np.ndarray, k_cache: np.ndarray,
                      dtype: str | None = None) -> None:
    """In-place store of quantised K rows into k_cache [NB, bs, Hkv, D/32*34]
    by slot (gfx906_fa_quant.cu:150-200).  key [T, Hkv, D] contiguous."""
    key = np.ascontiguousarray(key)
    slot_mapping = np.ascontiguousarray(slot_mapping, dtype=np.int64)
    assert k_cache.flags.c_contiguous and k_cache.dtype == np.uint8
    T, Hkv, D = key.shape
    NB, bs, Hkv2, rb = k_cache.shape
    assert Hkv2 == Hkv and rb == row_bytes(D)
    lib().q8o_reshape_and_cache(_p(key), ctypes.c_int(_dtype_code(key, dtype)), _p(slot_mapping),
                                _p(k_cache), ctypes.c_int(T), ctypes.c_int(Hkv), ctypes.c_int(D),
                                ctypes.c_int(bs), _i64(Hkv * D), _i64(D), _i64(bs * Hkv * rb),
                                _i64(Hkv * rb), _i64(rb))


def store_v_q8t(value: np.ndarray, slot_mapping: np.ndarray, v_cache: np.ndarray, bs: int,
                dtype: str | None = None) -> None:
    """In-place store of V into page-transposed Q8_0 records v_cache
    [NB, Hkv, bs*D/32*34] (this build's V layout; no reference counterpart).
    The Q8_0 blocks are those of quantize_q8_0(value) -- scale of block j of
    token t at bytes 2*(j*bs + t), int8 of dim d at 2*(D/32)*bs + d*bs + t."""
    T, Hkv, D = value.shape
    nb = D // QK
    rows = quantize_q8_0(value, dtype).reshape(T, Hkv, nb, BLOCK_BYTES)
    for t in range(T):
        s = int(slot_mapping[t])
        if s < 0:
            continue
        page, off = divmod(s, bs)
        for h in range(Hkv):
            rec = v_cache[page, h]
            for j in range(nb):
                rec[2 * (j * bs + off):2 * (j * bs + off) + 2] = rows[t, h, j, :2]
                rec[2 * nb * bs + (j * QK) * bs + off:2 * nb * bs + (j * QK + QK) * bs + off:bs] = rows[t, h, j, 2:]


def store_v16(value: np.ndarray, slot_mapping: np.ndarray, v_cache: np.ndarray) -> None:
    """In-place fp16/bf16 copy of V rows by slot (vLLM's reshape_and_cache for V)."""
    value = np.ascontiguousarray(value)
    T, Hkv, D = value.shape
    NB, bs, _, _ = v_cache.shape
    lib().q8o_store_v16(_p(value.view(np.uint16)), _p(np.ascontiguousarray(slot_mapping, np.int64)),
                        _p(v_cache.view(np.uint16)), ctypes.c_int(T), ctypes.c_int(Hkv),
                        ctypes.c_int(D), ctypes.c_int(bs), _i64(Hkv * D), _i64(D),
                        _i64(bs * Hkv * D), _i64(Hkv * D), _i64(D))


# --------------------------------------------------------------------------
# Gather (gfx906_fa_gather.cu:190-357)
# --------------------------------------------------------------------------
def gather(k_cache: np.ndarray, v_cache: np.ndarray, block_table: np.ndarray,
           seq_lens: np.ndarray, Sk: int, k_out: np.ndarray | None = None,
           v_out: np.ndarray | None = None):
    """Paged -> contiguous BHSD.  V rows past seq_len are zeroed; K rows there
    keep whatever k_out held (zeros when k_out is not given)."""
    NB, bs, Hkv, rb = k_cache.shape
    D = v_cache.shape[-1]
    B, max_blocks = block_table.shape
    bt = np.ascontiguousarray(block_table, dtype=np.int32)
    sl = np.ascontiguousarray(seq_lens, dtype=np.int32)
    if k_out is None:
        k_out = np.zeros((B, Hkv, Sk, rb), dtype=np.uint8)
    if v_out is None:
        v_out = np.zeros((B, Hkv, Sk, D), dtype=v_cache.dtype)
    lib().q8o_gather(_p(np.ascontiguousarray(k_cache)), _p(np.ascontiguousarray(v_cache).view(np.uint16)),
                     _p(bt), _p(sl), _p(k_out), _p(v_out.view(np.uint16)), ctypes.c_int(B),
                     ctypes.c_int(Hkv), ctypes.c_int(Sk), ctypes.c_int(D), ctypes.c_int(rb),
                     ctypes.c_int(bs), ctypes.c_int(max_blocks))
    return k_out, v_out


# --------------------------------------------------------------------------
# Dequantisation (tests/test_q8_roundtrip.py:21-36)
# --------------------------------------------------------------------------
def dequantize_q8_0(q8: np.ndarray, D: int) -> np.ndarray:
    """uint8 [..., D/32*34] -> float32 [..., D]: int8 value times fp16 scale."""
    nb = D // QK
    blk = np.ascontiguousarray(q8).reshape(-1, nb, BLOCK_BYTES)
    d = blk[:, :, :2].copy().view(np.float16).astype(np.float32)       # [N, nb, 1]
    qs = blk[:, :, 2:].view(np.int8).astype(np.float32)                 # [N, nb, 32]
    return (qs * d).reshape(q8.shape[:-1] + (D,))


# --------------------------------------------------------------------------
# Attention reference
# --------------------------------------------------------------------------
def attention_paged(q: np.ndarray, q_dtype: str | None, q_start: np.ndarray, n_q: np.ndarray,
                    k_cache: np.ndarray, v_cache: np.ndarray, block_table: np.ndarray,
                    kv_len: np.ndarray, scale: float, Hkv: int, q_abs: np.ndarray | None = None,
                    mask: np.ndarray | None = None, v_q8: bool = False,
                    q_strides: tuple[int, int, int] | None = None,
                    out_shape: tuple | None = None,
                    o_strides: tuple[int, int, int] | None = None,
                    k_strides: tuple[int, int, int] | None = None,
                    v_strides: tuple[int, int, int] | None = None,
                    nthreads: int = 0, bs: int | None = None, v_fmt: str | None = None,
                    softcap: float = 0.0, window: int = 0, sinks: np.ndarray | None = None,
                    num_blocks: int = 0) -> np.ndarray:
    """fp32 dequant + softmax reference (double accumulation).

    Default layouts are vLLM's: q [T, Hq, D] with token rows q_start[b] + t;
    k_cache [NB, bs, Hkv, D/32*34] u8; v_cache [NB, bs, Hkv, D] fp16 (or q8
    bytes when v_q8).  Strides (seq, tok, head) are in elements for q/out and
    (page, tok, head) in bytes for the caches.  bs: tokens per page (default
    k_cache.shape[1]); v_fmt: "f16" (default), "bf16", "q8" (= v_q8) or "q8t"
    (page-transposed Q8_0 records, v_cache [NB, Hkv, bs*D/32*34], v_strides
    (page, unused, head)).
    softcap > 0: score s -> softcap * tanh(s / softcap) before the mask;
    window > 0: key k visible to query position qp only if qp - k < window
    (qp = q_abs + t, or kv_len - n_q + t without q_abs); sinks [Hq] fp32:
    exp(sink) joins each row's softmax denominator; num_blocks > 0: keys on
    pages whose entry is < 0 or >= num_blocks are dropped.
    """
    vcode = {"f16": 0, "bf16": 1, "q8": 2, "q8t": 3}[v_fmt or ("q8" if v_q8 else "f16")]
    v_q8 = vcode == 2
    q = np.ascontiguousarray(q)
    D = q.shape[-1]
    Hq = q.shape[1]                    # [T, Hq, D] or [B, Hq, Sq, D]
    B = int(len(n_q))
    if q_strides is None:
        q_strides = (0, Hq * D, D)
    if out_shape is None:
        out_shape = q.shape
        o_strides = q_strides
    out = np.zeros(out_shape, dtype=np.float32)
    NB = k_cache.shape[0]
    if bs is None:
        bs = k_cache.shape[1]
    rb = row_bytes(D)
    if k_strides is None:
        k_strides = (bs * Hkv * rb, Hkv * rb, rb)
    if v_strides is None:
        vb = rb if v_q8 else 2 * D
        v_strides = (bs * Hkv * vb, Hkv * vb, vb)
    bt = np.ascontiguousarray(block_table, dtype=np.int32)
    max_blocks = bt.shape[1]
    qs = np.ascontiguousarray(q_start, dtype=np.int32)
    nq = np.ascontiguousarray(n_q, dtype=np.int32)
    kl = np.ascontiguousarray(kv_len, dtype=np.int32)
    qa = None if q_abs is None else np.ascontiguousarray(q_abs, dtype=np.int32)
    m_seq = m_tok = 0
    mk = None
    if mask is not None:
        mk = np.ascontiguousarray(mask).view(np.uint16)
        m_seq, m_tok = mk.shape[1] * mk.shape[2], mk.shape[2]
    sk = None if sinks is None else np.ascontiguousarray(sinks, dtype=np.float32)
    lib().q8o_attention_ex(
        _p(q.view(np.uint16) if q.dtype != np.float32 else q), ctypes.c_int(_dtype_code(q, q_dtype)),
        _i64(q_strides[0]), _i64(q_strides[1]), _i64(q_strides[2]), _p(qs), _p(nq),
        _p(out), _i64(o_strides[0]), _i64(o_strides[1]), _i64(o_strides[2]),
        _p(np.ascontiguousarray(k_cache)), _p(np.ascontiguousarray(v_cache).view(np.uint8)),
        ctypes.c_int(vcode), _i64(k_strides[0]), _i64(k_strides[1]), _i64(k_strides[2]),
        _i64(v_strides[0]), _i64(v_strides[1]), _i64(v_strides[2]), _p(bt), ctypes.c_int(max_blocks),
        ctypes.c_int(bs), _p(kl), _p(qa), _p(mk), _i64(m_seq), _i64(m_tok), ctypes.c_int(B),
        ctypes.c_int(Hq), ctypes.c_int(Hkv), ctypes.c_int(D), ctypes.c_float(scale),
        ctypes.c_int(nthreads), ctypes.c_float(softcap), ctypes.c_int(int(window)), _p(sk),
        ctypes.c_int(int(num_blocks)))
    return out


def attention_bhsd(q: np.ndarray, q_dtype: str | None, k_q8: np.ndarray, v: np.ndarray,
                   scale: float, kv_max: np.ndarray | None = None,
                   q_abs: np.ndarray | None = None, mask: np.ndarray | None = None,
                   v_q8: bool = False, nthreads: int = 0) -> np.ndarray:
    """Reference for the flat `forward` op: q [B, Hq, Sq, D], k_q8 [B, Hkv, Skv,
    D/32*34], v [B, Hkv, Skv, D] -> fp32 [B, Hq, Sq, D].  Every padded query
    row is computed, as the reference kernel does (fattn-q8.cuh:1041-1068)."""
    B, Hq, Sq, D = q.shape
    _, Hkv, Skv, _ = v.shape
    # contiguous per-(b,h) K rows == one page of Skv tokens per sequence with
    # head stride Skv*row
    rb = row_bytes(D)
    vb = rb if v_q8 else 2 * D
    bt = np.arange(B, dtype=np.int32).reshape(B, 1)
    kl = np.full(B, Skv, np.int32) if kv_max is None else np.asarray(kv_max, np.int32)
    return attention_paged(
        q, q_dtype, np.zeros(B, np.int32), np.full(B, Sq, np.int32),
        k_q8, v, bt, kl, scale, Hkv, q_abs=q_abs, mask=mask, v_q8=v_q8,
        q_strides=(Hq * Sq * D, D, Sq * D), out_shape=(B, Hq, Sq, D),
        o_strides=(Hq * Sq * D, D, Sq * D),
        k_strides=(Hkv * Skv * rb, rb, Skv * rb), v_strides=(Hkv * Skv * vb, vb, Skv * vb),
        nthreads=nthreads, bs=max(Skv, 1), v_fmt="q8" if v_q8 else ("bf16" if v.dtype == np.uint16 else "f16"))


# --------------------------------------------------------------------------
# Fused RoPE + store (no reference counterpart: the reference backend has no
# RoPE fusion, extension/gfx906_fa_backend.py:444-445).  Rotation as vLLM's
# rotary embedding defines it, computed in fp32 with each product and sum
# rounded separately, then rounded once to the tensor's element type.
# --------------------------------------------------------------------------
def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """fp32 -> bf16 bit patterns (uint16), round to nearest even (finite inputs)."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    return u.astype(np.uint16)


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.ascontiguousarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def rope(x: np.ndarray, dtype: str | None, positions: np.ndarray, cos_sin: np.ndarray, neox: bool) -> np.ndarray:
    """x [T, H, D] (fp16, fp32, or bf16 as uint16 with dtype="bf16");
    cos_sin [max_pos, rot] float32 (cos of pair j at j, sin at rot/2 + j).
    Returns the rotated tensor in x's storage type."""
    xf = bf16_bits_to_f32(x) if dtype == "bf16" else x.astype(np.float32)
    xf = xf.copy()
    rot = cos_sin.shape[1]
    half = rot // 2
    cs = cos_sin[np.asarray(positions, np.int64)].astype(np.float32)      # [T, rot]
    c = cs[:, None, :half]
    s = cs[:, None, half:]
    if neox:
        a, b = xf[..., :half].copy(), xf[..., half:rot].copy()
        xf[..., :half] = (a * c) - (b * s)
        xf[..., half:rot] = (b * c) + (a * s)
    else:
        a, b = xf[..., 0:rot:2].copy(), xf[..., 1:rot:2].copy()
        xf[..., 0:rot:2] = (a * c) - (b * s)
        xf[..., 1:rot:2] = (b * c) + (a * s)
    if dtype == "bf16":
        return f32_to_bf16_bits(xf)
    return xf.astype(x.dtype)
