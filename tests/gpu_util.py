"""Helpers shared by the GPU parity tests (no test functions here)."""
import os
import tempfile

import numpy as np

from oracle import oracle as O


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


def kv_data(rng, L, H, S, hd, outlier=True):
    """K = N(0,1) x per-(layer, head, channel) log-uniform [0.5, 8]; V = N(0,1)."""
    d = np.empty((L, 2, H, S, hd), np.float32)
    if outlier:
        scale = np.exp(rng.uniform(np.log(0.5), np.log(8.0), (L, H, 1, hd))).astype(np.float32)
    else:
        scale = np.float32(1.0)
    d[:, 0] = rng.standard_normal((L, H, S, hd)).astype(np.float32) * scale
    d[:, 1] = rng.standard_normal((L, H, S, hd)).astype(np.float32)
    return d


def parse_eakv(raw):
    hdr = raw[:512]
    nl = int(np.frombuffer(hdr[14:18], np.uint32)[0])
    nh = int(np.frombuffer(hdr[18:22], np.uint32)[0])
    hd = int(np.frombuffer(hdr[22:26], np.uint32)[0])
    sl = int(np.frombuffer(hdr[26:30], np.uint32)[0])
    offs = np.frombuffer(raw[512:512 + 16 * nl], np.uint64)
    ng = nh * hd * sl // 64
    blocks = []
    for o in offs:
        o = int(o)
        w = np.frombuffer(raw[o:o + ng * 32], np.uint8).reshape(ng, 32)
        s = np.frombuffer(raw[o + ng * 32:o + ng * 36], np.float32)
        b = np.frombuffer(raw[o + ng * 36:o + ng * 40], np.float32)
        blocks.append((w, s, b))
    return (nl, nh, hd, sl), blocks


def saved_bytes(cache):
    with tempfile.TemporaryDirectory() as td:
        p = os.path.join(td, "c.eakv")
        rc = cache.save(p)
        assert rc == 0, rc
        return open(p, "rb").read()


def device_blocks(cache):
    """Dense (w, s, b) per (layer, kv) of a device cache, read back through
    the library's own save path."""
    return parse_eakv(saved_bytes(cache))[1]


def ref_blocks(rc):
    """Dense (w, s, b) per (layer, kv) of an oracle RefCache."""
    out = []
    n = rc.seq_len * rc.gpd
    for lkv in range(rc.nl * 2):
        ws, ss, bs = [], [], []
        for h in range(rc.nh):
            g0 = h * rc.gph
            ws.append(rc.w[lkv, g0:g0 + n])
            ss.append(rc.s[lkv, g0:g0 + n])
            bs.append(rc.b[lkv, g0:g0 + n])
        out.append((np.concatenate(ws), np.concatenate(ss), np.concatenate(bs)))
    return out


def assert_blocks_equal(a, b):
    assert len(a) == len(b)
    for i, ((w1, s1, b1), (w2, s2, b2)) in enumerate(zip(a, b)):
        assert np.array_equal(w1, w2), f"nibbles differ in block {i}"
        assert np.array_equal(bits(s1), bits(s2)), f"scales differ in block {i}"
        assert np.array_equal(bits(b1), bits(b2)), f"biases differ in block {i}"


def assert_close(got, ref, atol=1e-4, rtol=1e-4, what=""):
    """|got - ref| <= atol + rtol*|ref| elementwise (the parity tolerance of
    scores and outputs)."""
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    err = np.abs(got - ref)
    lim = atol + rtol * np.abs(ref)
    bad = ~(err <= lim)
    if bad.any():
        i = int(np.argmax(np.where(bad, err - lim, -np.inf)))
        raise AssertionError(f"{what}: {bad.sum()} of {bad.size} outside tolerance; worst at {i}: "
                             f"got {got.flat[i]!r} ref {ref.flat[i]!r} err {err.flat[i]:.3e}")
    return float(err.max()) if err.size else 0.0


# decode kernel selection for E.force_path: the automatic choice, the
# CUDA-core kernel, the mma.sync tensor-core kernel, the tcgen05 kernel
PATH_CODE = {"auto": 0, "simt": 1, "mma": 2, "umma": 3}
