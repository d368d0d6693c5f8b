"""CPU: the oracle is pinned to the reference before it is trusted.

* The restated kernels reproduce every committed golden fixture bit for bit
  (fixtures come from the reference's own host code, tests/golden/make_golden.py).
* The reference's scalar quantizer src/ggml_type.c agrees with the restated
  Ea quantizer on packed nibbles and biases of every group and on scales of
  every group with range > 0 (when it was built, oracle/_ref/ggml_scalar.so).
* The reference's own C test programs pass when linked with the restated
  kernels (when built, oracle/_ref/reftest_*).
* Known-answer case of tests/test_ggml_type.c:121-151 (ramp 0..63).
"""
import ctypes
import glob
import os
import subprocess

import numpy as np
import pytest

from conftest import golden
from oracle import oracle as O


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


def test_quantize_golden():
    g = golden("quantize.npz")
    x = g["x"].reshape(-1, 64)
    w, s, b = O.quantize(x)
    assert np.array_equal(w, g["w"])
    assert np.array_equal(bits(s), bits(g["s"]))
    assert np.array_equal(bits(b), bits(g["b"]))


def test_quantize_edge_semantics():
    g = golden("quantize.npz")
    x = g["x"].reshape(-1, 64)
    w, s, b = O.quantize(x)
    # range 0 -> scale 1, all nibbles 0 (quantize_simd.ea:32-38)
    assert s[1] == 1.0 and not w[1].any() and b[1] == 3.0
    # first zero wins for min (+0 then -0 / -0 then +0)
    assert bits(b[3:4])[0] == 0x00000000 and bits(b[4:5])[0] == 0x80000000
    # NaN in element 0 sticks in the bias, scale falls back to 1
    assert np.isnan(b[6]) and s[6] == 1.0 and not w[6].any()


def test_known_answer_ramp():
    """tests/test_ggml_type.c:121-151: src = 0..63 -> monotone, ends near 0 and 63."""
    x = np.arange(64, dtype=np.float32)
    w, s, b = O.quantize(x)
    d = O.dequantize(w, s, b)
    assert np.all(np.diff(d) >= 0)
    assert d[0] < 1.0 and d[63] > 60.0
    assert np.max(np.abs(d - x)) <= s[0] / 2 + 1e-5


@pytest.mark.parametrize("name", ["mha128", "gqa64_8to2", "gqa128_4to1", "mha64"])
def test_attention_golden(name):
    g = golden(f"attn_{name}.npz")
    L, nq, nkv, hd, S, maxS = [int(v) for v in g["shape"]]
    rc = O.RefCache(L, nkv, hd, maxS)
    rc.load_raw(g["data"], S)
    for l in range(L):
        assert np.array_equal(bits(rc.scores(g["q"][l], l, nq, nkv)), bits(g["scores"][l]))
        assert np.array_equal(bits(rc.output(g["weights"][l], l, nq, nkv)), bits(g["output"][l]))
        assert np.array_equal(bits(rc.fused(g["q"][l], l, nq, nkv)), bits(g["fused"][l]))


def test_fused_equals_composition():
    """Two-pass fused attention == scores -> softmax -> V-sum within 1e-5."""
    g = golden("attn_gqa128_4to1.npz")
    L, nq, nkv, hd, S, maxS = [int(v) for v in g["shape"]]
    rc = O.RefCache(L, nkv, hd, maxS)
    rc.load_raw(g["data"], S)
    comp = rc.output(O.softmax_rows(rc.scores(g["q"][0], 0, nq, nkv), nq, S), 0, nq, nkv)
    np.testing.assert_allclose(rc.fused(g["q"][0], 0, nq, nkv), comp, atol=1e-5, rtol=1e-5)


def test_restated_mha_fused_matches_generalised():
    """q4_fused_attention_multi_f32 (fused_attention.ea:190) == the GQA/hd64
    generalisation at n_q == n_kv, hd 128."""
    g = golden("attn_mha128.npz")
    L, nq, nkv, hd, S, maxS = [int(v) for v in g["shape"]]
    rc = O.RefCache(L, nkv, hd, maxS)
    rc.load_raw(g["data"], S)
    kw, ks, kb = rc._blk(0, 0)
    vw, vs, vb = rc._blk(0, 1)
    q = np.ascontiguousarray(g["q"][0])
    out = np.zeros(nq * hd, np.float32)
    P = O.ptr
    O.olib().q4_fused_attention_multi_f32(P(q), P(kw), P(ks), P(kb), P(vw), P(vs), P(vb), P(out),
                                          S, nq, rc.gph)
    assert np.array_equal(bits(out), bits(g["fused"][0]))


def test_append_equals_bulk_oracle():
    """tests/test_append.c:40-119 invariant on the oracle cache: token-by-token
    append == bulk load_raw, bit for bit."""
    rng = np.random.default_rng(5)
    L, H, hd, S = 2, 2, 64, 20
    data = rng.standard_normal((L, 2, H, S, hd)).astype(np.float32)
    bulk = O.RefCache(L, H, hd, S)
    bulk.load_raw(data, S)
    inc = O.RefCache(L, H, hd, S)
    for t in range(S):
        for l in range(L):
            for kv in range(2):
                inc.append(data[l, kv, :, t:t + 1, :], l, kv, 1)
        inc.advance(1)
    assert np.array_equal(bulk.w, inc.w)
    assert np.array_equal(bits(bulk.s), bits(inc.s)) and np.array_equal(bits(bulk.b), bits(inc.b))


@pytest.mark.skipif(not os.path.exists(O.GGML_SCALAR_SO), reason="oracle/_ref not built")
def test_ggml_scalar_witness_random():
    rng = np.random.default_rng(1)
    n = 4096
    x = (rng.standard_normal((n, 64)) * np.exp(rng.uniform(-8, 8, (n, 1)))).astype(np.float32)
    x[::5] = np.round(x[::5] * 2) / 2
    w, s, b = O.quantize(x)
    G = ctypes.CDLL(O.GGML_SCALAR_SO)
    blk = np.zeros(n * 40, np.uint8)
    G.eakv_quantize_row(ctypes.c_void_p(x.ctypes.data), ctypes.c_void_p(blk.ctypes.data),
                        ctypes.c_int64(n * 64))
    blk = blk.reshape(n, 40)
    d = blk[:, 32:36].copy().view(np.float32)[:, 0]
    m = blk[:, 36:40].copy().view(np.float32)[:, 0]
    assert np.array_equal(blk[:, :32], w)
    assert np.array_equal(bits(m), bits(b))
    live = d > 0
    assert np.array_equal(bits(d[live]), bits(s[live]))


REFTESTS = sorted(glob.glob(os.path.join(os.path.dirname(O.REF_SO), "reftest_*")))


@pytest.mark.skipif(not REFTESTS, reason="oracle/_ref not built")
@pytest.mark.parametrize("exe", REFTESTS, ids=[os.path.basename(p) for p in REFTESTS])
def test_reference_ctests_on_oracle(exe):
    r = subprocess.run([exe], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stdout + r.stderr


@pytest.mark.parametrize("hd", [64, 128])
def test_single_head_kernels_match_multi_head_rows(hd):
    """Row a10: the reference's single-head kernels with a group offset
    (kernels/fused_k_score.ea:9-153, fused_v_sum.ea:7-77 and their _64 forms)
    restated, against the pinned multi-head restatements: head h of a
    multi-head block through the single-head form is row h of the multi-head
    result, bit for bit."""
    rng = np.random.default_rng(hd)
    L, H, S, maxS = 1, 3, 77, 90
    data = rng.standard_normal((L, 2, H, S, hd)).astype(np.float32)
    rc = O.RefCache(L, H, hd, maxS)
    rc.load_raw(data, S)
    q = rng.standard_normal(H * hd).astype(np.float32)
    multi = rc.scores(q, 0, H, H).reshape(H, S)
    w = rng.random(H * S).astype(np.float32)
    vmulti = rc.output(w, 0, H, H).reshape(H, hd)
    for h in range(H):
        assert np.array_equal(bits(rc.scores_single(q[h * hd:(h + 1) * hd], 0, h)),
                              bits(multi[h]))
        assert np.array_equal(bits(rc.output_single(w[h * S:(h + 1) * S], 0, h)),
                              bits(vmulti[h]))
