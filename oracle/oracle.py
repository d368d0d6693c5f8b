"""Parity checker: Python side of the CPU oracle. TEST INFRASTRUCTURE ONLY.

Imported by tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg,
never by the product (eakv_b200/). It drives two CPU builds:

* _build/liboracle.so - oracle_kernels.c, the C restatement of the
  reference's Ea kernels (always buildable: `make -C oracle`);
* _ref/libeakv_ref.so - the reference's own host sources (src/cache.c,
  src/attention.c, src/io.c, compiled unmodified where they lie) linked with
  that restatement (`make -C oracle ref`; needs the reference checkout, so
  it is built in the development container and travels prebuilt).

`RefCache` restates the reference host's cache layout and dispatch
(src/cache.c:11-151, src/attention.c:3-63) in numpy on top of
liboracle.so, so parity tests do not depend on _ref being present.
"""
import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))

def _avx512():
    try:
        flags = open("/proc/cpuinfo").read()
        return all(f in flags for f in ("avx512f", "avx512bw", "avx512dq", "avx512vl"))
    except OSError:
        return False


AVX512 = _avx512()
_SFX = "_v4" if AVX512 else ""
ORACLE_SO = os.path.join(HERE, "_build", f"liboracle{_SFX}.so")
REF_SO = os.path.join(HERE, "_ref", f"libeakv_ref{_SFX}.so")
GGML_SCALAR_SO = os.path.join(HERE, "_ref", "ggml_scalar.so")
GGML_AVX512_SO = os.path.join(HERE, "_ref", "ggml_avx512.so")

_P = ctypes.c_void_p
_I = ctypes.c_int32


def build():
    """Compile liboracle.so if it is missing or stale."""
    src = os.path.join(HERE, "oracle_kernels.c")
    if not os.path.exists(ORACLE_SO) or os.path.getmtime(ORACLE_SO) < os.path.getmtime(src):
        subprocess.run(["make", "-s", "-C", HERE], check=True)
    return ORACLE_SO


_olib = None


def olib():
    global _olib
    if _olib is None:
        build()
        L = ctypes.CDLL(ORACLE_SO)
        L.q4_quantize_split_f32.argtypes = [_P, _P, _P, _P, _I]
        L.q4_dequantize_avx512_f32.argtypes = [_P, _P, _P, _P, _I]
        for n in ("q4_fused_k_score_multi_f32", "q4_fused_k_score_multi_64_f32",
                  "q4_fused_v_sum_multi_f32", "q4_fused_v_sum_multi_64_f32"):
            getattr(L, n).argtypes = [_P, _P, _P, _P, _P, _I, _I, _I]
        for n in ("q4_k_score_gqa_f32", "q4_k_score_gqa_64_f32", "q4_v_sum_gqa_f32",
                  "q4_v_sum_gqa_64_f32"):
            getattr(L, n).argtypes = [_P, _P, _P, _P, _P, _I, _I, _I, _I]
        for n in ("q4_fused_k_score_f32", "q4_fused_k_score_64_f32", "q4_fused_v_sum_f32",
                  "q4_fused_v_sum_64_f32"):
            getattr(L, n).argtypes = [_P, _P, _P, _P, _P, _I, _I]
        L.q4_fused_attention_multi_f32.argtypes = [_P] * 8 + [_I, _I, _I]
        L.oracle_fused_attention.argtypes = [_P] * 8 + [_I, _I, _I, _I, _I]
        L.q4_validate.argtypes = [_P, _P, _P, _P, _I]
        L.q4_validate.restype = _I
        L.oracle_ggml_quantize_row.argtypes = [_P, _P, ctypes.c_int64]
        L.oracle_ggml_dequantize_row.argtypes = [_P, _P, ctypes.c_int64]
        L.oracle_ggml_vec_dot.argtypes = [ctypes.c_int, _P, ctypes.c_size_t, _P, ctypes.c_size_t,
                                          _P, ctypes.c_size_t, ctypes.c_int]
        _olib = L
    return _olib


def ptr(a):
    return a.ctypes.data


def quantize(x):
    """q4_quantize_split_f32 + the host's i32 -> u8 narrowing
    (src/cache.c:85-92). x: f32[n_groups*64] -> (u8[n,32], f32[n], f32[n])."""
    x = np.ascontiguousarray(x, np.float32).reshape(-1)
    n = x.size // 64
    w = np.zeros(n * 32, np.int32)
    s = np.zeros(n, np.float32)
    b = np.zeros(n, np.float32)
    olib().q4_quantize_split_f32(ptr(x), ptr(w), ptr(s), ptr(b), n)
    return w.astype(np.uint8).reshape(n, 32), s, b


def dequantize(w, s, b):
    w = np.ascontiguousarray(w, np.uint8).reshape(-1)
    n = w.size // 32
    out = np.zeros(n * 64, np.float32)
    olib().q4_dequantize_avx512_f32(ptr(w), ptr(np.ascontiguousarray(s, np.float32)),
                                    ptr(np.ascontiguousarray(b, np.float32)), ptr(out), n)
    return out


def _ggml_fns(lib):
    if lib is None:
        L = olib()
        return (L.oracle_ggml_quantize_row, L.oracle_ggml_dequantize_row, L.oracle_ggml_vec_dot)
    for n in ("eakv_quantize_row", "eakv_dequantize_row"):
        getattr(lib, n).argtypes = [_P, _P, ctypes.c_int64]
    lib.eakv_vec_dot_q4_f32.argtypes = [ctypes.c_int, _P, ctypes.c_size_t, _P, ctypes.c_size_t,
                                        _P, ctypes.c_size_t, ctypes.c_int]
    return lib.eakv_quantize_row, lib.eakv_dequantize_row, lib.eakv_vec_dot_q4_f32


def ggml_quantize(x, lib=None):
    """ggml q4_1_eakv from_float (src/ggml_type.c:21-93, AVX-512 build):
    f32[n*64] -> u8[n][40] blocks {qs[32], d, m}. `lib`: a CDLL exporting
    the reference names (the compiled reference, or the CUDA library);
    None: the restatement."""
    x = np.ascontiguousarray(x, np.float32).reshape(-1)
    n = x.size // 64
    out = np.zeros(n * 40, np.uint8)
    _ggml_fns(lib)[0](ptr(x), ptr(out), n * 64)
    return out.reshape(n, 40)


def ggml_dequantize(blocks, lib=None):
    blocks = np.ascontiguousarray(blocks, np.uint8).reshape(-1)
    n = blocks.size // 40
    out = np.zeros(n * 64, np.float32)
    _ggml_fns(lib)[1](ptr(blocks), ptr(out), n * 64)
    return out


def ggml_vec_dot(blocks, y, lib=None):
    """Row r of `blocks` (u8[nrc][nb*40]) dotted with row r of y
    (f32[nrc][nb*64]) -> f32[nrc] (ggml_type.c:138-242, nrc rows)."""
    blocks = np.ascontiguousarray(blocks, np.uint8)
    y = np.ascontiguousarray(y, np.float32)
    nrc, n = y.shape
    s = np.zeros(nrc, np.float32)
    _ggml_fns(lib)[2](n, ptr(s), 4, ptr(blocks), blocks.shape[1], ptr(y), n * 4, nrc)
    return s


class RefCache:
    """The reference host's cache (src/cache.c:11-51): per (layer, kv) a
    block of max_groups groups, head stride gph = max_seq_len*head_dim/64."""

    def __init__(self, n_layers, n_kv_heads, head_dim, max_seq_len):
        self.nl, self.nh, self.hd, self.max_seq = n_layers, n_kv_heads, head_dim, max_seq_len
        self.gpd = head_dim // 64
        self.gph = max_seq_len * self.gpd
        self.seq_len = 0
        mg = self.nh * self.gph
        self.w = np.zeros((n_layers * 2, mg, 32), np.uint8)
        self.s = np.zeros((n_layers * 2, mg), np.float32)
        self.b = np.zeros((n_layers * 2, mg), np.float32)

    def _put(self, lkv, h, g0, x):
        w, s, b = quantize(x)
        n = s.size
        base = h * self.gph + g0
        self.w[lkv, base:base + n] = w
        self.s[lkv, base:base + n] = s
        self.b[lkv, base:base + n] = b

    def load_raw(self, data, seq_len):
        """src/cache.c:60-100; data f32[L][2][H][seq_len][hd]."""
        data = np.asarray(data, np.float32).reshape(self.nl * 2, self.nh, seq_len * self.hd)
        for lkv in range(self.nl * 2):
            for h in range(self.nh):
                self._put(lkv, h, 0, data[lkv, h, :seq_len * self.gpd * 64])
        self.seq_len = seq_len

    def append(self, data, layer, kv, n_tok):
        """src/cache.c:102-151; data f32[H][n_tok][hd]; does not advance."""
        data = np.asarray(data, np.float32).reshape(self.nh, n_tok * self.hd)
        for h in range(self.nh):
            self._put(layer * 2 + kv, h, self.seq_len * self.gpd, data[h, :n_tok * self.gpd * 64])

    def advance(self, n):
        self.seq_len += n

    def _blk(self, layer, kv):
        i = layer * 2 + kv
        return (np.ascontiguousarray(self.w[i]), np.ascontiguousarray(self.s[i]),
                np.ascontiguousarray(self.b[i]))

    def scores(self, q, layer, n_q, n_kv):
        """src/attention.c:3-32 dispatch."""
        q = np.ascontiguousarray(q, np.float32)
        out = np.zeros(n_q * self.seq_len, np.float32)
        w, s, b = self._blk(layer, 0)
        L = olib()
        if self.hd == 64:
            if n_q == n_kv:
                L.q4_fused_k_score_multi_64_f32(ptr(q), ptr(w), ptr(s), ptr(b), ptr(out),
                                                self.seq_len, n_q, self.gph)
            else:
                L.q4_k_score_gqa_64_f32(ptr(q), ptr(w), ptr(s), ptr(b), ptr(out), self.seq_len,
                                        n_q, n_kv, self.gph)
        else:
            if n_q == n_kv:
                L.q4_fused_k_score_multi_f32(ptr(q), ptr(w), ptr(s), ptr(b), ptr(out),
                                             self.seq_len, n_q, self.gph)
            else:
                L.q4_k_score_gqa_f32(ptr(q), ptr(w), ptr(s), ptr(b), ptr(out), self.seq_len,
                                     n_q, n_kv, self.gph)
        return out

    def output(self, wts, layer, n_q, n_kv):
        """src/attention.c:34-63 dispatch."""
        wts = np.ascontiguousarray(wts, np.float32)
        out = np.zeros(n_q * self.hd, np.float32)
        w, s, b = self._blk(layer, 1)
        L = olib()
        if self.hd == 64:
            if n_q == n_kv:
                L.q4_fused_v_sum_multi_64_f32(ptr(wts), ptr(w), ptr(s), ptr(b), ptr(out),
                                              self.seq_len, n_q, self.gph)
            else:
                L.q4_v_sum_gqa_64_f32(ptr(wts), ptr(w), ptr(s), ptr(b), ptr(out), self.seq_len,
                                      n_q, n_kv, self.gph)
        else:
            if n_q == n_kv:
                L.q4_fused_v_sum_multi_f32(ptr(wts), ptr(w), ptr(s), ptr(b), ptr(out),
                                           self.seq_len, n_q, self.gph)
            else:
                L.q4_v_sum_gqa_f32(ptr(wts), ptr(w), ptr(s), ptr(b), ptr(out), self.seq_len,
                                   n_q, n_kv, self.gph)
        return out

    def fused(self, q, layer, n_q, n_kv, seq_range=None):
        """Two-pass fused softmax attention (kernels/fused_attention.ea:190-373
        generalised to GQA / head_dim 64). seq_range=(lo, hi) restricts the
        attended positions."""
        q = np.ascontiguousarray(q, np.float32)
        out = np.zeros(n_q * self.hd, np.float32)
        lo, hi = (0, self.seq_len) if seq_range is None else seq_range
        kw, ks, kb = self._blk(layer, 0)
        vw, vs, vb = self._blk(layer, 1)
        if lo:
            # shift every head's view by lo positions (heads stay gph apart)
            g = lo * self.gpd
            kw, ks, kb = (np.ascontiguousarray(kw[g:]), np.ascontiguousarray(ks[g:]),
                          np.ascontiguousarray(kb[g:]))
            vw, vs, vb = (np.ascontiguousarray(vw[g:]), np.ascontiguousarray(vs[g:]),
                          np.ascontiguousarray(vb[g:]))
        olib().oracle_fused_attention(ptr(q), ptr(kw), ptr(ks), ptr(kb), ptr(vw), ptr(vs),
                                      ptr(vb), ptr(out), hi - lo, n_q, n_kv, self.gph, self.hd)
        return out

    def scores_single(self, q, layer, head):
        """Scores of one query vector against KV head `head` through the
        reference's single-head kernel with a group offset
        (kernels/fused_k_score.ea:9-153, fused_k_score_64.ea:5-94)."""
        q = np.ascontiguousarray(q, np.float32)
        out = np.zeros(self.seq_len, np.float32)
        w, s, b = self._blk(layer, 0)
        fn = olib().q4_fused_k_score_64_f32 if self.hd == 64 else olib().q4_fused_k_score_f32
        fn(ptr(q), ptr(w), ptr(s), ptr(b), ptr(out), self.seq_len, head * self.gph)
        return out

    def output_single(self, wts, layer, head):
        """V sum of one weight row over KV head `head` through the reference's
        single-head kernel (kernels/fused_v_sum.ea:7-77, fused_v_sum_64.ea:5-50)."""
        wts = np.ascontiguousarray(wts, np.float32)
        out = np.zeros(self.hd, np.float32)
        w, s, b = self._blk(layer, 1)
        fn = olib().q4_fused_v_sum_64_f32 if self.hd == 64 else olib().q4_fused_v_sum_f32
        fn(ptr(wts), ptr(w), ptr(s), ptr(b), ptr(out), self.seq_len, head * self.gph)
        return out

    def dequant_head(self, layer, kv, h):
        """f32[seq_len][hd] of one head (kernels/dequantize_avx512.ea)."""
        g0 = h * self.gph
        n = self.seq_len * self.gpd
        return dequantize(self.w[layer * 2 + kv, g0:g0 + n], self.s[layer * 2 + kv, g0:g0 + n],
                          self.b[layer * 2 + kv, g0:g0 + n]).reshape(self.seq_len, self.hd)


def softmax_rows(scores, n_q, seq_len):
    """Caller-side softmax between the two calls (HOWTO.md section 3 of the
    reference): per row, max from -1e6 as in fused_attention.ea:38, exp,
    normalize."""
    s = np.asarray(scores, np.float32).reshape(n_q, seq_len).astype(np.float64)
    m = np.maximum(s.max(axis=1, keepdims=True), -1e6)
    e = np.exp(s - m)
    return (e / e.sum(axis=1, keepdims=True)).astype(np.float32).reshape(-1)


# ---- reference host library (optional, prebuilt from reference sources) ----

_rlib = None


def ref_available():
    return os.path.exists(REF_SO)


def rlib():
    """libeakv_ref.so: reference host C + restated kernels."""
    global _rlib
    if _rlib is None:
        if not ref_available():
            raise FileNotFoundError(REF_SO)
        L = ctypes.CDLL(REF_SO)
        L.eakv_cache_create.restype = _P
        L.eakv_cache_create.argtypes = [_I, _I, _I, _I]
        L.eakv_cache_free.argtypes = [_P]
        L.eakv_cache_load_raw.argtypes = [_P, _P, _I]
        L.eakv_cache_append.argtypes = [_P, _P, _I, _I, _I]
        L.eakv_cache_advance.argtypes = [_P, _I]
        L.eakv_attention_scores.argtypes = [_P, _P, _I, _I, _I, _P]
        L.eakv_attention_output.argtypes = [_P, _P, _I, _I, _I, _P]
        L.eakv_cache_save.argtypes = [_P, ctypes.c_char_p]
        L.eakv_cache_load.argtypes = [ctypes.c_char_p, ctypes.POINTER(_P)]
        L.eakv_cache_seq_len.argtypes = [_P]
        _rlib = L
    return _rlib


# ---------------------------------------------------------------------------
# llama.cpp sequence state (reference src/llama_bridge.c:19-288)

REF_LLAMA_SO = os.path.join(HERE, "_ref", "libeakv_ref_llama.so")
FP16_STUB_SO = os.path.join(HERE, "_build", "fp16_stub.so")


def llama_state(k, v, v_trans, seq_ids=None, k_type=1, v_size_el=2):
    """Bytes of a llama.cpp sequence state in the layout the reference
    bridge parses: k, v f16 [n_layers][cells][n_embd]; v_trans stores each
    V layer as columns [n_embd][cells]."""
    k = np.ascontiguousarray(k, np.float16)
    v = np.ascontiguousarray(v, np.float16)
    L, cells, embd = k.shape
    out = [np.array([1, cells], np.uint32).tobytes()]
    for t in range(cells):
        ids = [0] if seq_ids is None else seq_ids[t]
        out.append(np.array([t], np.int32).tobytes())
        out.append(np.array([len(ids)], np.uint32).tobytes())
        out.append(np.array(ids, np.int32).tobytes())
    out.append(np.array([1 if v_trans else 0, L], np.uint32).tobytes())
    for l in range(L):
        out.append(np.array([k_type], np.int32).tobytes())
        out.append(np.array([embd * 2], np.uint64).tobytes())
        out.append(k[l].tobytes())
    for l in range(L):
        out.append(np.array([k_type], np.int32).tobytes())
        if v_trans:
            out.append(np.array([v_size_el, embd], np.uint32).tobytes())
            out.append(np.ascontiguousarray(v[l].T).tobytes())
        else:
            out.append(np.array([embd * 2], np.uint64).tobytes())
            out.append(v[l].tobytes())
    return b"".join(out)


def llama_import(k, v, n_kv_heads, head_dim, max_seq_len, cache=None, start_pos=0):
    """The bridge's arithmetic restated: f16 -> f32, [pos][head][dim] ->
    [head][pos][dim], eakv_cache_append per (layer, K/V), then advance
    (llama_bridge.c:74-160 / :215-283). Returns the RefCache."""
    k = np.asarray(k, np.float16)
    v = np.asarray(v, np.float16)
    L, cells, embd = k.shape
    if cache is None:
        cache = RefCache(L, n_kv_heads, head_dim, max_seq_len)
    new = cells - start_pos
    for kv, src in ((0, k), (1, v)):
        for l in range(L):
            x = src[l, start_pos:].astype(np.float32).reshape(new, n_kv_heads, head_dim)
            cache.append(np.ascontiguousarray(x.transpose(1, 0, 2)), l, kv, new)
    cache.advance(new)
    return cache
