"""Generates the golden fixtures in tests/golden/ (committed; rerun only to
refresh them). Needs the reference checkout, because every fixture comes
from the reference's own host code:

    make -C oracle ref            # builds oracle/_ref/ from the reference sources
    python tests/golden/make_golden.py

The reference ships no golden vectors (its tests only check invariants), so
the fixtures are produced by oracle/_ref/libeakv_ref.so: the reference's
unmodified src/cache.c, src/attention.c and src/io.c linked with the C
restatement of its Ea kernels. Quantization is additionally pinned by the
reference's compilable scalar quantizer src/ggml_type.c:21-90
(oracle/_ref/ggml_scalar.so): both must agree bit for bit on every group
whose range is > 0 (at range == 0 ggml_type.c stores scale 0 where the Ea
kernel stores 1, a known inconsistency inside the reference).

Outputs:
  quantize.npz   edge-case groups, the reference's .eakv file of them (eakv_file), and
                 the packed nibbles / scales / biases read back from it
  attn_<name>.npz  seeded K/V/queries, reference scores, softmax weights,
                 reference V-sum output and two-pass fused attention output
  ggml.npz       q4_1_eakv ggml blocks, dequantized values and vec_dot results of
                 the reference's src/ggml_type.c built with AVX-512
                 (oracle/_ref/ggml_avx512.so)
  llama.npz      llama.cpp sequence states (f16 rows / transposed V, a two-step
                 append) and the .eakv files the reference's src/llama_bridge.c
                 makes of them (oracle/_ref/libeakv_ref_llama.so)
"""
import ctypes
import os
import sys
import tempfile

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)
from oracle import oracle as O  # noqa: E402

OUT = os.path.dirname(os.path.abspath(__file__))

# (name, n_layers, n_q_heads, n_kv_heads, head_dim, seq_len, max_seq_len, seed)
ATTN_CONFIGS = [
    ("mha128", 2, 2, 2, 128, 40, 48, 11),
    ("gqa64_8to2", 1, 8, 2, 64, 100, 128, 12),
    ("gqa128_4to1", 1, 8, 2, 128, 70, 70, 13),
    ("mha64", 1, 4, 4, 64, 32, 32, 14),
]


def kv_data(rng, L, H, S, hd):
    """K = N(0,1) x per-(layer, head, channel) scale log-uniform in [0.5, 8];
    V = N(0,1). Layout [layer][kv][head][pos][dim]."""
    d = np.empty((L, 2, H, S, hd), np.float32)
    scale = np.exp(rng.uniform(np.log(0.5), np.log(8.0), (L, H, 1, hd))).astype(np.float32)
    d[:, 0] = rng.standard_normal((L, H, S, hd)).astype(np.float32) * scale
    d[:, 1] = rng.standard_normal((L, H, S, hd)).astype(np.float32)
    return d


def edge_groups(rng):
    g = []
    g.append(np.arange(64, dtype=np.float32))                        # tests/test_ggml_type.c:121
    g.append(np.full(64, 3.0, np.float32))                           # range 0
    g.append(np.zeros(64, np.float32))
    z = np.abs(rng.standard_normal(64)).astype(np.float32) + 1
    z[3], z[9] = 0.0, -0.0                                           # first zero +0
    g.append(z.copy())
    z[3], z[9] = -0.0, 0.0                                           # first zero -0
    g.append(z.copy())
    n = -np.abs(rng.standard_normal(64)).astype(np.float32) - 1
    n[7], n[20] = -0.0, 0.0                                          # max is a zero
    g.append(n)
    x = rng.standard_normal(64).astype(np.float32)
    x[0] = np.nan                                                    # NaN in element 0 sticks
    g.append(x)
    x = rng.standard_normal(64).astype(np.float32)
    x[17] = np.nan                                                   # later NaN skipped
    x[40] = np.nan
    g.append(x)
    x = rng.standard_normal(64).astype(np.float32)
    x[5] = np.inf
    g.append(x)
    x = rng.standard_normal(64).astype(np.float32)
    x[60] = -np.inf
    g.append(x)
    g.append((rng.standard_normal(64) * 1e-42).astype(np.float32))   # denormals
    x = (rng.standard_normal(64) * 1e37).astype(np.float32)
    x[0], x[1] = 3e38, -3e38                                         # range overflows to inf
    g.append(x)
    # values landing exactly on q + 0.5 boundaries
    g.append((np.arange(64) % 16 + 0.5).astype(np.float32) * np.float32(0.25))
    g.append(np.linspace(-1, 1, 64).astype(np.float32))
    for sc in (1e-30, 1e-5, 1.0, 1e5, 1e30):
        for _ in range(4):
            g.append((rng.standard_normal(64) * sc).astype(np.float32))
    while len(g) % 8:
        g.append(rng.standard_normal(64).astype(np.float32))
    return np.stack(g)


def parse_eakv(raw):
    """(header fields, [(w, s, b) per layer*2]) of a .eakv file."""
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


def ref_save(R, c):
    with tempfile.TemporaryDirectory() as td:
        p = os.path.join(td, "x.eakv")
        assert R.eakv_cache_save(c, p.encode()) == 0
        return open(p, "rb").read()


def make_quantize(rng, R):
    groups = edge_groups(rng)                     # [n, 64]
    n = groups.shape[0]
    H = 2
    S = n // (2 * H)
    x = groups.reshape(1, 2, H, S, 64)
    c = R.eakv_cache_create(1, H, 64, S)
    assert R.eakv_cache_load_raw(c, x.ctypes.data, S) == 0
    raw = ref_save(R, c)
    R.eakv_cache_free(c)
    (_, _, _, _), blocks = parse_eakv(raw)
    w = np.concatenate([b[0] for b in blocks])
    s = np.concatenate([b[1] for b in blocks])
    b = np.concatenate([b[2] for b in blocks])
    # restated kernel == reference host + restated kernel
    w2, s2, b2 = O.quantize(groups)
    assert np.array_equal(w, w2) and np.array_equal(s.view(np.uint32), s2.view(np.uint32))
    assert np.array_equal(b.view(np.uint32), b2.view(np.uint32))
    # witness: the reference's own scalar quantizer (ggml_type.c)
    G = ctypes.CDLL(O.GGML_SCALAR_SO)
    blk = np.zeros(n * 40, np.uint8)
    G.eakv_quantize_row(ctypes.c_void_p(groups.ctypes.data), ctypes.c_void_p(blk.ctypes.data),
                        ctypes.c_int64(n * 64))
    blk = blk.reshape(n, 40)
    gd = blk[:, 32:36].copy().view(np.float32)[:, 0]
    gm = blk[:, 36:40].copy().view(np.float32)[:, 0]
    live = gd > 0                                 # range > 0 groups (NaN range excluded)
    assert np.array_equal(blk[:, :32], w), "nibbles differ from ggml_type.c"
    assert np.array_equal(gm.view(np.uint32), b.view(np.uint32)), "bias differs from ggml_type.c"
    assert np.array_equal(gd[live].view(np.uint32), s[live].view(np.uint32))
    np.savez_compressed(os.path.join(OUT, "quantize.npz"), x=x, eakv_file=np.frombuffer(raw, np.uint8),
                        w=w, s=s, b=b)
    print(f"quantize.npz: {n} groups, file {len(raw)} B, witness agreed on {live.sum()} groups")


def make_attention(R):
    for name, L, nq, nkv, hd, S, maxS, seed in ATTN_CONFIGS:
        rng = np.random.default_rng(seed)
        data = kv_data(rng, L, nkv, S, hd)
        q = rng.standard_normal((L, nq, hd)).astype(np.float32)
        c = R.eakv_cache_create(L, nkv, hd, maxS)
        assert R.eakv_cache_load_raw(c, data.ctypes.data, S) == 0
        rc = O.RefCache(L, nkv, hd, maxS)
        rc.load_raw(data, S)
        scores = np.zeros((L, nq * S), np.float32)
        weights = np.zeros((L, nq * S), np.float32)
        output = np.zeros((L, nq * hd), np.float32)
        fused = np.zeros((L, nq * hd), np.float32)
        for l in range(L):
            ql = np.ascontiguousarray(q[l])
            R.eakv_attention_scores(c, ql.ctypes.data, l, nq, nkv, scores[l].ctypes.data)
            assert np.array_equal(scores[l].view(np.uint32), rc.scores(ql, l, nq, nkv).view(np.uint32))
            weights[l] = O.softmax_rows(scores[l], nq, S)
            wl = np.ascontiguousarray(weights[l])
            R.eakv_attention_output(c, wl.ctypes.data, l, nq, nkv, output[l].ctypes.data)
            assert np.array_equal(output[l].view(np.uint32), rc.output(wl, l, nq, nkv).view(np.uint32))
            fused[l] = rc.fused(ql, l, nq, nkv)
        R.eakv_cache_free(c)
        np.savez_compressed(os.path.join(OUT, f"attn_{name}.npz"), data=data, q=q, scores=scores,
                            weights=weights, output=output, fused=fused,
                            shape=np.array([L, nq, nkv, hd, S, maxS], np.int32))
        print(f"attn_{name}.npz: L={L} nq={nq} nkv={nkv} hd={hd} S={S} max={maxS}")


def make_ggml(rng):
    """q4_1_eakv ggml type (src/ggml_type.c) from the reference's AVX-512
    build (oracle/_ref/ggml_avx512.so); the restatement must agree."""
    G = ctypes.CDLL(O.GGML_AVX512_SO)
    e = edge_groups(rng)
    specials = rng.choice(np.array([0.0, -0.0, 1.0, -1.0, np.nan, np.inf, -np.inf, 1e-40, -1e-40,
                                    3e38, -3e38], np.float32), (64, 64))
    rnd = (rng.standard_normal((256, 64)) * np.exp(rng.uniform(-30, 30, (256, 1)))).astype(np.float32)
    x = np.concatenate([e, specials, rnd]).astype(np.float32)
    blocks = O.ggml_quantize(x, G)
    assert np.array_equal(blocks, O.ggml_quantize(x)), "restated from_float differs"
    deq = O.ggml_dequantize(blocks, G)
    assert np.array_equal(deq.view(np.uint32), O.ggml_dequantize(blocks).view(np.uint32))
    # vec_dot: 6 rows of 4 blocks (256 elements) against random queries
    vx = blocks[-24:].reshape(6, 4 * 40)
    vy = rng.standard_normal((6, 256)).astype(np.float32)
    dot = O.ggml_vec_dot(vx, vy, G)
    assert np.array_equal(dot.view(np.uint32), O.ggml_vec_dot(vx, vy).view(np.uint32))
    np.savez_compressed(os.path.join(OUT, "ggml.npz"), x=x, blocks=blocks, deq=deq, vx=vx, vy=vy,
                        dot=dot)
    print(f"ggml.npz: {x.shape[0]} blocks, vec_dot {vx.shape[0]} rows")


# (name, n_layers, n_kv_heads, head_dim, cells, v_trans, first import cells)
LLAMA_CONFIGS = [
    ("rows", 2, 2, 64, 70, 0, 70),
    ("vtrans", 1, 2, 128, 65, 1, 65),
    ("append_vtrans", 1, 2, 64, 100, 1, 40),   # 40 cells, then cells 40..99 appended
]


def make_llama(rng):
    """llama.cpp state import (src/llama_bridge.c) by the reference's own
    bridge (oracle/_ref/libeakv_ref_llama.so); files saved with the
    reference's eakv_cache_save (cells == max_seq_len, so they are dense)."""
    R = ctypes.CDLL(O.REF_LLAMA_SO)
    R.eakv_from_llama_state.argtypes = [ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int,
                                        ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                        ctypes.POINTER(ctypes.c_void_p)]
    R.eakv_from_llama_state_append.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t,
                                               ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                               ctypes.c_int]
    R.eakv_cache_save.argtypes = [ctypes.c_void_p, ctypes.c_char_p]
    R.eakv_cache_free.argtypes = [ctypes.c_void_p]
    out = {}
    for name, L, H, hd, cells, vt, first in LLAMA_CONFIGS:
        embd = H * hd
        k = (rng.standard_normal((L, cells, embd)) * 3).astype(np.float16)
        v = rng.standard_normal((L, cells, embd)).astype(np.float16)
        k[0, 0, :4] = [np.inf, -np.inf, 0.0, -0.0]
        v[0, 1, 5] = np.nan
        full = O.llama_state(k, v, vt)
        part = O.llama_state(k[:, :first], v[:, :first], vt)
        buf = np.frombuffer(part, np.uint8)
        c = ctypes.c_void_p()
        assert R.eakv_from_llama_state(buf.ctypes.data, buf.size, L, H, hd, cells,
                                       ctypes.byref(c)) == 0
        if first < cells:
            fb = np.frombuffer(full, np.uint8)
            assert R.eakv_from_llama_state_append(c, fb.ctypes.data, fb.size, L, H, hd, first) == 0
        with tempfile.TemporaryDirectory() as td:
            p = os.path.join(td, "x.eakv")
            assert R.eakv_cache_save(c, p.encode()) == 0
            raw = open(p, "rb").read()
        R.eakv_cache_free(c)
        # the restated bridge gives the same blocks
        rc = O.llama_import(k[:, :first], v[:, :first], H, hd, cells)
        if first < cells:
            O.llama_import(k, v, H, hd, cells, cache=rc, start_pos=first)
        _, blocks = parse_eakv(raw)
        n = rc.seq_len * rc.gpd
        for lkv, (w, s_, b) in enumerate(blocks):
            for h in range(H):
                sl = slice(h * n, (h + 1) * n)
                g0 = h * rc.gph
                assert np.array_equal(w[sl], rc.w[lkv, g0:g0 + n])
                assert np.array_equal(s_[sl].view(np.uint32), rc.s[lkv, g0:g0 + n].view(np.uint32))
                assert np.array_equal(b[sl].view(np.uint32), rc.b[lkv, g0:g0 + n].view(np.uint32))
        out[f"{name}_state"] = np.frombuffer(full, np.uint8)
        if first < cells:
            out[f"{name}_first"] = np.frombuffer(part, np.uint8)
        out[f"{name}_file"] = np.frombuffer(raw, np.uint8)
        out[f"{name}_shape"] = np.array([L, H, hd, cells, vt, first], np.int32)
        print(f"llama {name}: L={L} H={H} hd={hd} cells={cells} v_trans={vt} first={first}")
    np.savez_compressed(os.path.join(OUT, "llama.npz"), **out)


def main():
    R = O.rlib()
    rng = np.random.default_rng(2026)
    make_quantize(rng, R)
    make_attention(R)
    make_ggml(np.random.default_rng(2027))
    make_llama(np.random.default_rng(2028))


if __name__ == "__main__":
    main()
