"""GPU: .eakv save/load round trips and interchange with the reference's
files, plus the reference's own C test programs linked against
libeakv_b200.so (oracle/_ref/b200test_*, when they were built)."""
import glob
import os
import subprocess
import tempfile

import numpy as np
import pytest

import eakv_b200 as E
from conftest import ROOT, golden
from gpu_util import bits, kv_data, saved_bytes

pytestmark = pytest.mark.gpu


def test_roundtrip_keeps_everything(gpu):
    """tests/test_io_c.c:6-44: metadata kept, scores equal."""
    L, H, hd, S = 2, 4, 128, 32
    rng = np.random.default_rng(0)
    data = kv_data(rng, L, H, S, hd)
    with E.Cache(L, H, hd, S) as c, tempfile.TemporaryDirectory() as td:
        assert c.load_raw(data, S) == 0
        p = os.path.join(td, "rt.eakv")
        assert c.save(p) == 0
        d = E.Cache.load(p)
        assert (d.seq_len, d.n_layers, d.n_kv_heads, d.head_dim, d.max_seq_len) == (S, L, H, hd, S)
        q = np.ones(H * hd, np.float32)
        for l in range(L):
            assert np.array_equal(bits(c.scores(q, l, H, H)), bits(d.scores(q, l, H, H)))
        assert saved_bytes(d) == saved_bytes(c)
        d.free()


def test_partial_cache_saves_dense(gpu):
    """seq_len < max_seq_len: the file holds each head's first seq_len
    positions (dense), and loads back to the same attention."""
    L, H, hd, S, maxS = 1, 3, 64, 20, 50
    rng = np.random.default_rng(1)
    data = kv_data(rng, L, H, S, hd)
    with E.Cache(L, H, hd, maxS) as c, E.Cache(L, H, hd, S) as tight, \
            tempfile.TemporaryDirectory() as td:
        assert c.load_raw(data, S) == 0
        assert tight.load_raw(data, S) == 0
        assert saved_bytes(c) == saved_bytes(tight)
        p = os.path.join(td, "p.eakv")
        assert c.save(p) == 0
        d = E.Cache.load(p)
        q = rng.standard_normal(H * hd).astype(np.float32)
        assert np.array_equal(bits(c.scores(q, 0, H, H)), bits(d.scores(q, 0, H, H)))
        d.free()


def test_load_reference_written_file(gpu):
    """A file written by the reference's io.c loads and reproduces the
    reference's attention scores."""
    g = golden("quantize.npz")
    with tempfile.TemporaryDirectory() as td:
        p = os.path.join(td, "ref.eakv")
        open(p, "wb").write(g["eakv_file"].tobytes())
        c = E.Cache.load(p)
        assert saved_bytes(c) == g["eakv_file"].tobytes()
        c.free()


def test_load_errors(gpu):
    """tests/test_io_c.c:46-65 codes."""
    L = E.lib()
    import ctypes
    out = ctypes.c_void_p()
    assert L.eakv_cache_load(b"/tmp/does_not_exist_eakv_b200.eakv", ctypes.byref(out)) == E.EAKV_ERR_IO
    with tempfile.TemporaryDirectory() as td:
        p = os.path.join(td, "bad.eakv")
        open(p, "wb").write(b"NOPE" + bytes(508))
        assert L.eakv_cache_load(p.encode(), ctypes.byref(out)) == E.EAKV_ERR_FORMAT
        open(p, "wb").write(b"EAKV")
        assert L.eakv_cache_load(p.encode(), ctypes.byref(out)) == E.EAKV_ERR_FORMAT
        # truncated payload
        with E.Cache(1, 2, 64, 8) as c:
            c.load_raw(np.ones((1, 2, 2, 8, 64), np.float32), 8)
            raw = saved_bytes(c)
        open(p, "wb").write(raw[:-200])
        assert L.eakv_cache_load(p.encode(), ctypes.byref(out)) == E.EAKV_ERR_FORMAT


B200TESTS = sorted(glob.glob(os.path.join(ROOT, "oracle", "_ref", "b200test_*")))


@pytest.mark.skipif(not B200TESTS, reason="reference C tests were not built against the library")
@pytest.mark.parametrize("exe", B200TESTS, ids=[os.path.basename(p) for p in B200TESTS])
def test_reference_ctests_on_b200(gpu, exe):
    """The reference's own test programs, compiled unmodified against
    include/eakv.h and linked with libeakv_b200.so, pass on the device."""
    r = subprocess.run([exe], capture_output=True, text=True, timeout=300, cwd=tempfile.gettempdir())
    assert r.returncode == 0, r.stdout + r.stderr
    assert "FAIL" not in r.stdout
