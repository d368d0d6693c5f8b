"""GPU: device validate (reference kernels/validate.ea:14-71 as src/cli.c:
39-98 runs it) and dequantize (kernels/dequantize_avx512.ea:10-89) of a
resident cache against the restated kernels on the same blocks: codes
equal, values bit for bit."""
import os
import tempfile

import numpy as np
import pytest

import eakv_b200 as E
from gpu_util import bits, kv_data, parse_eakv, saved_bytes
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def oracle_codes(raw):
    """q4_validate over every (layer, K/V) block of a .eakv file."""
    _, blocks = parse_eakv(raw)
    L = O.olib()
    out = []
    for w, s, b in blocks:
        s = np.ascontiguousarray(s)
        b = np.ascontiguousarray(b)
        out.append(L.q4_validate(O.ptr(s), O.ptr(b), O.ptr(s), O.ptr(b), s.size))
    return np.array(out, np.int32)


def corrupt(raw, layer, kv, group, field, value):
    """A copy of a .eakv file with the scale (field 0) or bias (field 1) of
    one group of one block replaced."""
    (nl, nh, hd, sl), _ = parse_eakv(raw)
    offs = np.frombuffer(raw[512:512 + 16 * nl], np.uint64)
    ng = nh * hd * sl // 64
    o = int(offs[layer * 2 + kv]) + ng * 32 + field * ng * 4 + group * 4
    b = bytearray(raw)
    b[o:o + 4] = np.array([value], np.float32).tobytes()
    return bytes(b)


def load_bytes(raw):
    with tempfile.TemporaryDirectory() as td:
        p = os.path.join(td, "c.eakv")
        open(p, "wb").write(raw)
        return E.Cache.load(p)


def test_validate_clean_and_nan_bias(gpu):
    L, H, hd, S = 2, 2, 128, 70
    rng = np.random.default_rng(3)
    data = kv_data(rng, L, H, S, hd)
    with E.Cache(L, H, hd, S) as c:
        assert c.load_raw(data, S) == 0
        assert (c.validate() == 0).all()
    data[1, 1, 1, 40, 0] = np.nan      # NaN at element 0 of a group: its bias is NaN
    with E.Cache(L, H, hd, S) as c:
        assert c.load_raw(data, S) == 0
        got = c.validate()
        assert np.array_equal(got, oracle_codes(saved_bytes(c)))
        assert got[3] == 2 and (np.delete(got, 3) == 0).all()


def test_validate_corrupted_files(gpu):
    """NaN and negative scales cannot come out of the quantizer; they come
    from a damaged file. The first failing group in the reference's order
    decides, scale NaN before bias NaN before negative scale."""
    L, H, hd, S = 2, 3, 64, 64
    rng = np.random.default_rng(4)
    with E.Cache(L, H, hd, S) as c:
        assert c.load_raw(kv_data(rng, L, H, S, hd), S) == 0
        raw = saved_bytes(c)
    cases = [
        [(0, 0, 5, 0, np.nan)],                                   # NaN scale
        [(0, 1, 7, 1, -np.nan)],                                  # negative-sign NaN bias
        [(1, 0, 100, 0, -2.0)],                                   # negative scale
        [(1, 1, 50, 0, -1.0), (1, 1, 20, 1, np.nan)],             # earlier group wins
        [(0, 0, 9, 0, -0.0)],                                     # -0.0 is not below zero
        [(1, 0, 33, 0, np.float32(-np.inf))],
    ]
    for edits in cases:
        r = raw
        for layer, kv, grp, field, val in edits:
            r = corrupt(r, layer, kv, grp, field, val)
        d = load_bytes(r)
        try:
            assert np.array_equal(d.validate(), oracle_codes(r)), edits
        finally:
            d.free()


@pytest.mark.parametrize("hd", [64, 128])
def test_dequantize_ranges(gpu, hd):
    import torch
    L, H, S, maxS = 2, 3, 200, 256
    rng = np.random.default_rng(hd)
    data = kv_data(rng, L, H, S, hd)
    with E.Cache(L, H, hd, maxS) as c:
        assert c.load_raw(data, S) == 0
        rc = O.RefCache(L, H, hd, maxS)
        rc.load_raw(data, S)
        for layer, kv, a, b in [(0, 0, 0, S), (1, 1, 63, 129), (0, 1, 199, 200), (1, 0, 5, 5)]:
            got = c.dequantize(layer, kv, a, b)
            lkv = layer * 2 + kv
            for h in range(H):
                g0 = h * rc.gph + a * rc.gpd
                g1 = h * rc.gph + b * rc.gpd
                ref = O.dequantize(rc.w[lkv, g0:g1], rc.s[lkv, g0:g1], rc.b[lkv, g0:g1])
                assert np.array_equal(bits(got[h].reshape(-1)), bits(ref)), (layer, kv, a, b, h)
        d_out = torch.full((H, 10, hd), -1.0, device=gpu)
        c.dequantize_device(1, 0, 30, 40, d_out)
        torch.cuda.synchronize()
        assert np.array_equal(bits(d_out.cpu().numpy()), bits(c.dequantize(1, 0, 30, 40)))
        for bad in [(2, 0, 0, 1), (0, 2, 0, 1), (0, 0, 10, 5), (0, 0, 0, S + 1), (0, 0, -1, 3)]:
            with pytest.raises(E.EakvError):
                c.dequantize(*bad)
