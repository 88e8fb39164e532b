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


@pytest.mark.parametrize("hkv", [1, 2, 4, 8, 16])
@pytest.mark.parametrize("v_fmt", [0, 3])
def test_decode_plans_dense_pages_for_every_head_count(hkv, v_fmt):
    """Host-side planning only (no launch): a dense paged decode batch must be
    accepted by the split-K decode kernel for every kv-head count a tensor-
    parallel rank can hold (a rejection would silently route decode to the
    128-row tensor-core prefill kernel).  v_fmt 0: fp16 V rows; 3: page-
    transposed Q8_0 V records."""
    from _util import G9AttnBatch
    lib = capi()
    lib.gfx906_fa_decode_workspace_size.restype = ctypes.c_size_t
    lib.gfx906_fa_decode_workspace_size.argtypes = [ctypes.POINTER(G9AttnBatch)]
    D, bs, rb, B = 128, 16, 136, 4
    b = G9AttnBatch()
    b.q, b.q_dtype = 1 << 20, 1
    b.q_seq_stride, b.q_tok_stride, b.q_head_stride = 6 * hkv * D, 0, D
    b.seq_q = 1
    b.out, b.out_dtype = 2 << 20, 1
    b.o_seq_stride, b.o_tok_stride, b.o_head_stride = 6 * hkv * D, 0, D
    b.k_cache = 3 << 20
    b.k_page_stride, b.k_tok_stride, b.k_head_stride = 2 * bs * hkv * 2 * D, hkv * rb, rb
    b.v_cache = 4 << 20
    if v_fmt == 3:
        b.v_page_stride, b.v_tok_stride, b.v_head_stride = 2 * bs * hkv * 2 * D, 0, bs * rb
    else:
        b.v_page_stride, b.v_tok_stride, b.v_head_stride = 2 * bs * hkv * 2 * D, hkv * 2 * D, 2 * D
    b.v_fmt = v_fmt
    b.block_table, b.max_blocks, b.block_size = 5 << 20, 2048, bs
    b.kv_len, b.max_kv = 6 << 20, 32768
    b.num_seqs, b.num_heads_q, b.num_heads_kv, b.head_dim = B, 6 * hkv, hkv, D
    b.scale = 0.088
    assert lib.gfx906_fa_decode_workspace_size(ctypes.byref(b)) > 0


def test_ctypes_batch_matches_c_layout(tmp_path):
    """The tests' ctypes G9AttnBatch has the C struct's size and field
    offsets (compiled with gcc against include/gfx906_fa_b200.h)."""
    import shutil
    import subprocess
    from _util import G9AttnBatch
    if not shutil.which("gcc") or not os.path.exists("/usr/local/cuda/include/cuda_runtime_api.h"):
        pytest.skip("gcc / CUDA headers not available")
    names = [f[0] for f in G9AttnBatch._fields_]
    src = tmp_path / "layout.c"
    src.write_text('#include <stdio.h>\n#include <stddef.h>\n#include "gfx906_fa_b200.h"\nint main(void) {\n'
                   '  printf("%zu\\n", sizeof(G9AttnBatch));\n' +
                   "".join(f'  printf("%zu\\n", offsetof(G9AttnBatch, {n}));\n' for n in names) + "  return 0;\n}\n")
    exe = tmp_path / "layout"
    subprocess.check_call(["gcc", "-I", os.path.join(ROOT, "include"), "-I", "/usr/local/cuda/include",
                           str(src), "-o", str(exe)])
    vals = [int(x) for x in subprocess.check_output([str(exe)]).split()]
    assert vals[0] == ctypes.sizeof(G9AttnBatch)
    assert vals[1:] == [getattr(G9AttnBatch, n).offset for n in names]


@pytest.mark.skipif(not _built(), reason="library not built")
def test_prefill_staging_is_bounded_for_padded_batches():
    """Host-side sizing only (no launch): a config-5-shaped batch in the
    reference API's padded layout (every sequence has Sq_pad = 4096 query
    rows) runs its tensor-core sequences in groups whose fp16 staging fits
    1 GiB, so its workspace stays near the largest group instead of the sum
    over all 34 sequences (about 9.4 GB); with exact host query lengths the
    verify rows go to the decode kernel and only the two chunks are staged."""
    from _util import G9AttnBatch
    lib = capi()
    lib.gfx906_fa_attention_workspace_size.restype = ctypes.c_size_t
    lib.gfx906_fa_attention_workspace_size.argtypes = [ctypes.POINTER(G9AttnBatch), ctypes.c_void_p,
                                                       ctypes.c_void_p]
    rng = __import__("numpy").random.default_rng(5)
    kv = [int(x) for x in rng.integers(16384, 100001, size=32)] + [4096, 24576 + 4096]
    B, hkv, D, bs, rb = len(kv), 8, 128, 16, 136
    b = G9AttnBatch()
    b.q, b.q_dtype = 1 << 20, 2
    b.q_seq_stride, b.q_tok_stride, b.q_head_stride = 48 * 4096 * D, D, 4096 * D
    b.seq_q = 4096
    b.out, b.out_dtype = 2 << 20, 2
    b.o_seq_stride, b.o_tok_stride, b.o_head_stride = 48 * 4096 * D, D, 4096 * D
    b.k_cache = 3 << 20
    b.k_page_stride, b.k_tok_stride, b.k_head_stride = bs * hkv * rb, hkv * rb, rb
    b.v_cache = 4 << 20
    b.v_page_stride, b.v_tok_stride, b.v_head_stride = bs * hkv * 2 * D, hkv * 2 * D, 2 * D
    b.block_table, b.max_blocks, b.block_size = 5 << 20, 6300, bs
    b.kv_len, b.max_kv = 6 << 20, 6300 * bs
    b.num_seqs, b.num_heads_q, b.num_heads_kv, b.head_dim = B, 48, hkv, D
    b.scale = 0.088
    padded = (ctypes.c_int * B)(*([4096] * B))
    kvh = (ctypes.c_int * B)(*kv)
    ws_padded = lib.gfx906_fa_attention_workspace_size(ctypes.byref(b), padded, kvh)
    exact = (ctypes.c_int * B)(*([4] * 32 + [4096, 4096]))
    ws_exact = lib.gfx906_fa_attention_workspace_size(ctypes.byref(b), exact, kvh)
    assert 0 < ws_exact < ws_padded <= (1 << 30) + (64 << 20), (ws_exact, ws_padded)
