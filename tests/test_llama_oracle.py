"""CPU: the restated llama.cpp state import (oracle.llama_import: f16 ->
f32, [pos][head][dim] -> [head][pos][dim], append, advance; reference
src/llama_bridge.c:19-288) against the golden .eakv files made by the
reference's own bridge, and, when oracle/_ref is built, the reference bridge
itself on malformed buffers (the error codes the device import must give).
The half -> float decode that lets the bridge compile here
(oracle/ggml_stub/ggml.h) is checked on every half value."""
import ctypes
import os

import numpy as np
import pytest

from conftest import golden
from gpu_util import assert_blocks_equal, parse_eakv, ref_blocks
from oracle import oracle as O

NAMES = ["rows", "vtrans", "append_vtrans"]


def states(g, name):
    L, H, hd, cells, vt, first = [int(x) for x in g[f"{name}_shape"]]
    full = g[f"{name}_state"].tobytes()
    part = g[f"{name}_first"].tobytes() if first < cells else full
    return (L, H, hd, cells, vt, first), full, part


def kv_from_state(state, L, H, hd, cells, vt):
    """Inverse of oracle.llama_state for cells with one sequence id."""
    embd = H * hd
    off = 8 + cells * 12 + 8
    k = np.empty((L, cells, embd), np.float16)
    v = np.empty((L, cells, embd), np.float16)
    for l in range(L):
        off += 12
        k[l] = np.frombuffer(state, np.float16, cells * embd, off).reshape(cells, embd)
        off += cells * embd * 2
    for l in range(L):
        off += 12
        a = np.frombuffer(state, np.float16, cells * embd, off)
        v[l] = a.reshape(embd, cells).T if vt else a.reshape(cells, embd)
        off += cells * embd * 2
    return k, v


@pytest.mark.parametrize("name", NAMES)
def test_restated_import_matches_golden(name):
    g = golden("llama.npz")
    (L, H, hd, cells, vt, first), full, _ = states(g, name)
    k, v = kv_from_state(full, L, H, hd, cells, vt)
    rc = O.llama_import(k[:, :first], v[:, :first], H, hd, cells)
    if first < cells:
        O.llama_import(k, v, H, hd, cells, cache=rc, start_pos=first)
    assert_blocks_equal(ref_blocks(rc), parse_eakv(g[f"{name}_file"].tobytes())[1])


def test_fp16_stub_is_exact():
    O.build()
    L = ctypes.CDLL(O.FP16_STUB_SO)
    h = np.arange(65536, dtype=np.uint16)
    f = np.zeros(65536, np.float32)
    L.fp16_stub_convert(ctypes.c_void_p(h.ctypes.data), ctypes.c_void_p(f.ctypes.data), 65536)
    assert np.array_equal(f.view(np.uint32), h.view(np.float16).astype(np.float32).view(np.uint32))


def ref_import_rc(state, L, H, hd, max_seq):
    R = ctypes.CDLL(O.REF_LLAMA_SO)
    R.eakv_from_llama_state.argtypes = [ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int,
                                        ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                        ctypes.POINTER(ctypes.c_void_p)]
    R.eakv_cache_free.argtypes = [ctypes.c_void_p]
    buf = np.frombuffer(state, np.uint8)
    c = ctypes.c_void_p()
    rc = R.eakv_from_llama_state(buf.ctypes.data, buf.size, L, H, hd, max_seq, ctypes.byref(c))
    if rc == 0:
        R.eakv_cache_free(c)
    return rc


# (description, state transform, L, H, hd, max_seq, expected reference code)
def error_cases():
    rng = np.random.default_rng(1)
    k = rng.standard_normal((2, 10, 128)).astype(np.float16)
    st = O.llama_state(k, k, 0)
    empty = O.llama_state(k[:, :0], k[:, :0], 0)
    return [
        ("ok", st, 2, 2, 64, 16, 0),
        ("short", st[:7], 2, 2, 64, 16, -4),
        ("layers differ", st, 3, 2, 64, 16, -2),
        ("cells > max", st, 2, 2, 64, 8, -2),
        ("truncated V", st[:-1], 2, 2, 64, 16, -2),
        ("truncated cells", st[:100], 2, 2, 64, 16, -2),
        ("no layers", st, 0, 2, 64, 16, -4),
        ("no cells", empty, 2, 2, 64, 16, -2),
    ]


@pytest.mark.skipif(not os.path.exists(O.REF_LLAMA_SO), reason="oracle/_ref not built")
def test_reference_bridge_error_codes():
    for what, st, L, H, hd, mx, code in error_cases():
        assert ref_import_rc(st, L, H, hd, mx) == code, what
