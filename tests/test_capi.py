"""The C-ABI library loads without a GPU and exports every symbol that
include/*.h declares; the torch extension exposes the reference's op names."""
import ctypes
import glob
import os

import pytest

from _util import LIB, ROOT, capi, header_functions


def _built():
    return os.path.exists(LIB)


@pytest.mark.skipif(not _built(), reason="library not built")
def test_every_declared_symbol_is_exported():
    lib = capi()
    headers = glob.glob(os.path.join(ROOT, "include", "*.h"))
    assert headers
    names = [n for h in headers for n in header_functions(h)]
    assert "launch_gather_paged_kv_q8" in names and "launch_reshape_and_cache_q8" in names
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing


@pytest.mark.skipif(not _built(), reason="library not built")
def test_version_string():
    lib = capi()
    lib.gfx906_fa_version.restype = ctypes.c_char_p
    assert b"sm_100a" in lib.gfx906_fa_version()


@pytest.mark.skipif(not _built(), reason="library not built")
def test_reference_launchers_reject_bad_arguments_without_launching():
    """Argument checks run on the host before any launch, so they work (and
    return cudaErrorInvalidValue = 1) even with no GPU present."""
    lib = capi()
    # D not a multiple of 32
    assert lib.launch_quantize_q8_0_dense(None, None, 4, 48, None) == 1
    # head_size not a multiple of 32
    assert lib.launch_reshape_and_cache_q8(None, None, None, 1, 1, 40, 16, ctypes.c_int64(40),
                                           ctypes.c_int64(40), ctypes.c_int64(0), ctypes.c_int64(0),
                                           ctypes.c_int64(0), None) == 1
    # empty work is a successful no-op (reference: quant.cu:241, gather.cu:384)
    assert lib.launch_quantize_q8_0_dense(None, None, 0, 128, None) == 0


def test_extension_exposes_reference_ops():
    import importlib
    pytest.importorskip("torch")
    if not os.path.exists(os.path.join(ROOT, "gfx906-fa-vllm_b200", "gfx906_fa.so")):
        pytest.skip("extension not built")
    m = importlib.import_module("gfx906_fa")
    for name in ("quantize_q8_0", "reshape_and_cache_q8", "gather_paged_kv_q8"):
        assert hasattr(m, name)
