"""Helpers shared by the tests (no test functions here)."""
import ctypes
import os
import re

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "gfx906-fa-vllm_b200")
LIB = os.path.join(PKG, "libgfx906fa_b200.so")
HEADER = os.path.join(ROOT, "include", "gfx906_fa_b200.h")


def header_functions(path=HEADER):
    """Names of the functions declared in a C header (simple declarations)."""
    src = open(path).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return re.findall(r"^\s*(?:const\s+)?[A-Za-z_][A-Za-z0-9_]*\s*\*?\s*([A-Za-z_][A-Za-z0-9_]*)\s*\(",
                      src, flags=re.M)


class G9AttnBatch(ctypes.Structure):
    """ctypes mirror of G9AttnBatch (include/gfx906_fa_b200.h), field for field."""
    _fields_ = [
        ("q", ctypes.c_void_p), ("q_dtype", ctypes.c_int),
        ("q_seq_stride", ctypes.c_int64), ("q_tok_stride", ctypes.c_int64), ("q_head_stride", ctypes.c_int64),
        ("q_start", ctypes.c_void_p), ("n_q", ctypes.c_void_p), ("seq_q", ctypes.c_int),
        ("out", ctypes.c_void_p), ("out_dtype", ctypes.c_int),
        ("o_seq_stride", ctypes.c_int64), ("o_tok_stride", ctypes.c_int64), ("o_head_stride", ctypes.c_int64),
        ("k_cache", ctypes.c_void_p),
        ("k_page_stride", ctypes.c_int64), ("k_tok_stride", ctypes.c_int64), ("k_head_stride", ctypes.c_int64),
        ("v_cache", ctypes.c_void_p),
        ("v_page_stride", ctypes.c_int64), ("v_tok_stride", ctypes.c_int64), ("v_head_stride", ctypes.c_int64),
        ("v_fmt", ctypes.c_int), ("block_table", ctypes.c_void_p), ("max_blocks", ctypes.c_int),
        ("block_size", ctypes.c_int), ("kv_len", ctypes.c_void_p), ("max_kv", ctypes.c_int),
        ("q_abs", ctypes.c_void_p), ("mask", ctypes.c_void_p),
        ("mask_seq_stride", ctypes.c_int64), ("mask_tok_stride", ctypes.c_int64),
        ("num_seqs", ctypes.c_int), ("num_heads_q", ctypes.c_int), ("num_heads_kv", ctypes.c_int),
        ("head_dim", ctypes.c_int), ("scale", ctypes.c_float),
        ("num_blocks", ctypes.c_int), ("softcap", ctypes.c_float), ("window", ctypes.c_int),
        ("sinks", ctypes.c_void_p), ("flags", ctypes.c_int), ("out_scale", ctypes.c_void_p),
    ]


def capi():
    return ctypes.CDLL(LIB)


def to_np(t):
    """torch tensor (any device) -> numpy, 16-bit floats kept bit-exact."""
    import torch
    t = t.detach().cpu()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16)
    return t.numpy()
