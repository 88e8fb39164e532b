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


def capi():
    return ctypes.CDLL(LIB)


def to_np(t):
    """torch tensor (any device) -> numpy, 16-bit floats kept bit-exact."""
    import torch
    t = t.detach().cpu()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16)
    return t.numpy()
