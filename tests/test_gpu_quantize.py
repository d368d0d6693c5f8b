"""GPU parity of the quantize / append kernel and the .eakv writer:
packed nibbles, scales and biases bit-exact against the reference."""
import numpy as np
import pytest

import eakv_b200 as E
from conftest import golden
from gpu_util import (assert_blocks_equal, device_blocks, kv_data, ref_blocks, saved_bytes)
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def test_reference_file_byte_identical(gpu):
    """The golden edge-case groups (NaN, +-0, inf, denormals, range 0, ...)
    quantized on the device and saved give the reference's .eakv file."""
    g = golden("quantize.npz")
    x = g["x"]
    _, _, H, S, hd = x.shape
    with E.Cache(1, H, hd, S) as c:
        assert c.load_raw(x, S) == 0
        raw = saved_bytes(c)
    assert raw == g["eakv_file"].tobytes()


@pytest.mark.parametrize("L,H,hd,S,maxS", [(1, 4, 64, 37, 64), (2, 8, 128, 130, 200),
                                           (3, 2, 128, 1, 1), (1, 1, 64, 64, 64),
                                           (1, 3, 256, 65, 70)])
def test_load_raw_bit_exact(gpu, L, H, hd, S, maxS):
    rng = np.random.default_rng(L * 1000 + S)
    data = kv_data(rng, L, H, S, hd)
    data.reshape(-1)[::97] *= 1e-3
    data.reshape(-1)[::1013] = 0.0
    rc = O.RefCache(L, H, hd, maxS)
    rc.load_raw(data, S)
    with E.Cache(L, H, hd, maxS) as c:
        assert c.load_raw(data, S) == 0
        assert c.seq_len == S
        assert_blocks_equal(device_blocks(c), ref_blocks(rc))


def test_quantize_many_random_groups(gpu):
    """~1M groups across magnitudes, ties and zeros."""
    rng = np.random.default_rng(7)
    H, S, hd = 16, 4096, 64
    x = rng.standard_normal((1, 2, H, S, hd)).astype(np.float32)
    x *= np.exp(rng.uniform(-20, 20, (1, 2, H, S, 1))).astype(np.float32)
    x[..., ::3, :] = np.round(x[..., ::3, :])
    x[..., ::11, 5] = -0.0
    rc = O.RefCache(1, H, hd, S)
    rc.load_raw(x, S)
    with E.Cache(1, H, hd, S) as c:
        assert c.load_raw(x, S) == 0
        assert_blocks_equal(device_blocks(c), ref_blocks(rc))


@pytest.mark.parametrize("hd,step", [(64, 1), (128, 1), (128, 8), (64, 5)])
def test_append_matches_bulk(gpu, hd, step):
    """tests/test_append.c:40-159: appending token by token (or in batches)
    then advancing equals one bulk load_raw, bit for bit."""
    L, H, S = 2, 4, 29
    rng = np.random.default_rng(hd + step)
    data = kv_data(rng, L, H, S, hd)
    with E.Cache(L, H, hd, S) as bulk, E.Cache(L, H, hd, S) as inc:
        assert bulk.load_raw(data, S) == 0
        for t in range(0, S, step):
            n = min(step, S - t)
            for l in range(L):
                for kv in range(2):
                    sl = np.ascontiguousarray(data[l, kv, :, t:t + n, :])
                    assert inc.append(sl, l, kv, n) == 0
            assert inc.advance(n) == 0
        assert inc.seq_len == S
        assert saved_bytes(bulk) == saved_bytes(inc)


def test_append_step_device(gpu):
    """One-launch append of every layer and K/V from device memory equals
    per-(layer, kv) host appends."""
    import torch
    L, H, hd, S, n = 3, 2, 128, 50, 3
    rng = np.random.default_rng(3)
    base = kv_data(rng, L, H, S, hd)
    step = rng.standard_normal((L, 2, H, n, hd)).astype(np.float32)
    with E.Cache(L, H, hd, S + n) as a, E.Cache(L, H, hd, S + n) as b:
        assert a.load_raw(base, S) == 0
        assert b.load_raw(base, S) == 0
        for l in range(L):
            for kv in range(2):
                assert a.append(np.ascontiguousarray(step[l, kv]), l, kv, n) == 0
        a.advance(n)
        d = torch.from_numpy(step).to(gpu)
        assert b.append_step_device(d, n) == 0
        b.synchronize()
        b.advance(n)
        assert saved_bytes(a) == saved_bytes(b)


def test_append_rejections(gpu):
    """tests/test_append.c:179-210 error codes."""
    with E.Cache(2, 4, 64, 8) as c:
        tok = np.zeros(4 * 64, np.float32)
        assert c.load_raw(np.zeros((2, 2, 4, 8, 64), np.float32), 8) == 0
        assert c.advance(1) == E.EAKV_ERR_INVALID
        assert c.append(tok, 0, 0, 1) == E.EAKV_ERR_INVALID
        c.clear()
        assert c.append(tok, 5, 0, 1) == E.EAKV_ERR_INVALID
        assert c.append(tok, 0, 2, 1) == E.EAKV_ERR_INVALID
        assert c.append(tok, 0, 0, 0) == E.EAKV_ERR_INVALID
        assert E.lib().eakv_cache_append(None, E._ptr(tok), 0, 0, 1) == E.EAKV_ERR_INVALID
        assert E.lib().eakv_cache_append(c.h, None, 0, 0, 1) == E.EAKV_ERR_INVALID
        assert c.load_raw(np.zeros(1, np.float32), 64) == E.EAKV_ERR_INVALID


def test_checkpoint_restore(gpu):
    """tests/test_checkpoint.c: O(1) rollback, bounds, append after restore."""
    with E.Cache(2, 2, 64, 256) as c:
        assert c.checkpoint() == 0
        assert c.load_raw(np.zeros((2, 2, 2, 16, 64), np.float32), 16) == 0
        assert c.checkpoint() == 16
        assert c.restore(8) == 0 and c.seq_len == 8
        assert c.restore(16) == E.EAKV_ERR_INVALID and c.seq_len == 8
        assert c.restore(-1) == E.EAKV_ERR_INVALID
        z = np.zeros(2 * 4 * 64, np.float32)
        for l in range(2):
            assert c.append(z, l, 0, 4) == 0
            assert c.append(z, l, 1, 4) == 0
        assert c.advance(4) == 0 and c.seq_len == 12
        assert c.compression_ratio() == pytest.approx(40 / 256)
        c.clear()
        assert c.seq_len == 0 and c.compression_ratio() == 0.0
