"""CPU: the C-ABI library loads and exports every function that the headers
in include/ declare, and the Python binding covers all of them. No kernel
runs here."""
import ctypes
import os
import re

import pytest

from conftest import ROOT

HEADERS = [os.path.join(ROOT, "include", h)
           for h in ("eakv.h", "eakv_cuda.h", "eakv_ggml.h", "eakv_llama.h", "eakv_nccl.h")]


def declared_functions():
    names = []
    for h in HEADERS:
        text = open(h).read()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        for m in re.finditer(r"\b(eakv_[a-z0-9_]+)\s*\(", text):
            names.append(m.group(1))
    return sorted(set(names))


def test_headers_declare_reference_api():
    names = declared_functions()
    # reference include/eakv.h:25-83, one for one
    ref = ["eakv_cache_create", "eakv_cache_free", "eakv_cache_load_raw", "eakv_cache_append",
           "eakv_cache_advance", "eakv_cache_clear", "eakv_checkpoint", "eakv_restore",
           "eakv_attention_scores", "eakv_attention_output", "eakv_cache_save",
           "eakv_cache_load", "eakv_cache_seq_len", "eakv_cache_n_layers", "eakv_cache_n_heads",
           "eakv_cache_head_dim", "eakv_cache_max_seq_len", "eakv_cache_compression_ratio"]
    # reference include/eakv_ggml.h:36-52
    ref += ["eakv_quantize_row", "eakv_dequantize_row", "eakv_vec_dot_q4_f32"]
    # reference include/eakv_llama.h:26-41
    ref += ["eakv_from_llama_state", "eakv_from_llama_state_append"]
    for r in ref:
        assert r in names


def test_library_exports_every_declared_symbol():
    import eakv_b200
    L = ctypes.CDLL(eakv_b200.LIB_PATH)
    missing = [n for n in declared_functions() if not hasattr(L, n)]
    assert not missing, missing


def test_binding_covers_every_declared_symbol():
    import eakv_b200
    assert set(declared_functions()) <= set(eakv_b200.SIGNATURES)


def test_library_is_sm100a_only():
    """The shared library embeds code for sm_100a and was built for it."""
    from eakv_b200 import build as B
    assert B.ARCH == ["-gencode", "arch=compute_100a,code=sm_100a"]


def test_error_codes_match_reference():
    import eakv_b200 as E
    text = open(HEADERS[0]).read()
    for name, val in (("EAKV_OK", 0), ("EAKV_ERR_IO", -1), ("EAKV_ERR_FORMAT", -2),
                      ("EAKV_ERR_ALLOC", -3), ("EAKV_ERR_INVALID", -4)):
        assert re.search(rf"#define {name}\s+{val}\b", text)
        assert getattr(E, name) == val


def test_create_rejects_bad_params_without_device():
    """Argument checks of src/cache.c:13-16 happen before any CUDA call."""
    import eakv_b200 as E
    L = E.lib()
    assert not L.eakv_cache_create(0, 8, 128, 64)
    assert not L.eakv_cache_create(2, 0, 128, 64)
    assert not L.eakv_cache_create(2, 8, 128, 0)
    assert not L.eakv_cache_create(2, 3, 100, 64)     # 300 % 64 != 0
    assert L.eakv_last_error() == E.EAKV_ERR_INVALID
    L.eakv_cache_free(None)                            # NULL is a no-op
    assert L.eakv_cache_seq_len(None) == 0
    assert L.eakv_cache_compression_ratio(None) == 0.0
    assert L.eakv_checkpoint(None) == 0
    assert L.eakv_restore(None, 0) == E.EAKV_ERR_INVALID


def test_nccl_is_resolved_at_run_time():
    """The multi-GPU calls (include/eakv_nccl.h) find NCCL at run time, with
    no link dependency: the library reports the loaded NCCL's version and
    makes unique ids (128 bytes, a new one per call) without a GPU."""
    import eakv_b200 as E
    assert E.nccl_version() >= 21000
    a, b = E.nccl_unique_id(), E.nccl_unique_id()
    assert len(a) == E.NCCL_ID_BYTES == 128 and a != b
    import subprocess
    out = subprocess.run(["ldd", E.LIB_PATH], capture_output=True, text=True).stdout
    assert "nccl" not in out
