"""GPU: llama.cpp state import (eakv_b200/csrc/llama.cu) against the golden
.eakv files the reference's src/llama_bridge.c made of the same states (bit
for bit), the restated bridge on larger random states, and the reference's
error codes on malformed buffers."""
import numpy as np
import pytest

import eakv_b200 as E
from conftest import golden
from gpu_util import assert_blocks_equal, device_blocks, ref_blocks, saved_bytes
from oracle import oracle as O
from test_llama_oracle import NAMES, error_cases, states

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("name", NAMES)
def test_import_matches_reference_file(gpu, name):
    g = golden("llama.npz")
    (L, H, hd, cells, vt, first), full, part = states(g, name)
    c = E.Cache.from_llama_state(part, L, H, hd, cells)
    try:
        if first < cells:
            assert c.append_llama_state(full, L, H, hd, first) == 0
        assert c.seq_len == cells
        assert saved_bytes(c) == g[f"{name}_file"].tobytes()
    finally:
        c.free()


@pytest.mark.parametrize("vt", [0, 1])
def test_import_random_states(gpu, vt):
    rng = np.random.default_rng(40 + vt)
    L, H, hd, cells, max_seq = 3, 4, 128, 333, 400
    k = (rng.standard_normal((L, cells, H * hd)) * 4).astype(np.float16)
    v = rng.standard_normal((L, cells, H * hd)).astype(np.float16)
    ids = [list(range(t % 3 + 1)) for t in range(cells)]          # 1-3 sequence ids per cell
    first = 100
    st_first = O.llama_state(k[:, :first], v[:, :first], vt, seq_ids=ids[:first])
    st_full = O.llama_state(k, v, vt, seq_ids=ids)
    rc = O.llama_import(k[:, :first], v[:, :first], H, hd, max_seq)
    O.llama_import(k, v, H, hd, max_seq, cache=rc, start_pos=first)
    c = E.Cache.from_llama_state(st_first, L, H, hd, max_seq)
    try:
        assert c.seq_len == first
        assert c.append_llama_state(st_full, L, H, hd, first) == 0
        assert c.seq_len == cells
        assert c.append_llama_state(st_full, L, H, hd, cells) == 0     # nothing new
        assert_blocks_equal(device_blocks(c), ref_blocks(rc))
    finally:
        c.free()


def test_import_error_codes(gpu):
    for what, st, L, H, hd, mx, code in error_cases():
        if code == 0:
            E.Cache.from_llama_state(st, L, H, hd, mx).free()
            continue
        with pytest.raises(E.EakvError) as ei:
            E.Cache.from_llama_state(st, L, H, hd, mx)
        assert ei.value.rc == code, what


def test_append_checks(gpu):
    rng = np.random.default_rng(2)
    k = rng.standard_normal((1, 20, 64)).astype(np.float16)
    st = O.llama_state(k, k, 0)
    c = E.Cache.from_llama_state(O.llama_state(k[:, :10], k[:, :10], 0), 1, 1, 64, 32)
    try:
        assert c.append_llama_state(st, 1, 1, 64, 5) == -4        # start_pos != seq_len
        assert c.append_llama_state(st, 1, 2, 32, 10) == -4       # shape differs from the cache
        assert c.append_llama_state(st, 1, 1, 64, 10) == 0
        assert c.seq_len == 20
    finally:
        c.free()
