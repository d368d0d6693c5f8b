"""CPU: the restated q4_1_eakv ggml type (oracle/oracle_kernels.c, the
reference's src/ggml_type.c:21-242 AVX-512 build) against the golden
fixture made by the compiled reference, and, when oracle/_ref is built,
against the compiled reference itself on fresh random and special inputs."""
import ctypes
import os

import numpy as np
import pytest

from conftest import golden
from oracle import oracle as O


def bits(a):
    return np.ascontiguousarray(a).view(np.uint32)


def test_restated_ggml_type_matches_golden():
    g = golden("ggml.npz")
    assert np.array_equal(O.ggml_quantize(g["x"]), g["blocks"])
    assert np.array_equal(bits(O.ggml_dequantize(g["blocks"])), bits(g["deq"]))
    assert np.array_equal(bits(O.ggml_vec_dot(g["vx"], g["vy"])), bits(g["dot"]))


def test_golden_covers_the_special_cases():
    g = golden("ggml.npz")
    x = g["x"]
    d = g["blocks"][:, 32:36].copy().view(np.float32)[:, 0]
    assert np.isnan(x).any() and np.isinf(x).any()
    assert (d == 0).any()                      # constant blocks store d = 0
    assert np.isnan(d).any() or np.isinf(d).any()


@pytest.mark.skipif(not os.path.exists(O.GGML_AVX512_SO), reason="oracle/_ref not built")
def test_restated_ggml_type_matches_compiled_reference():
    G = ctypes.CDLL(O.GGML_AVX512_SO)
    rng = np.random.default_rng(42)
    x = (rng.standard_normal((3000, 64)) * np.exp(rng.uniform(-40, 40, (3000, 1)))).astype(np.float32)
    x[:300] = rng.choice(np.array([0.0, -0.0, 2.0, -2.0, np.nan, np.inf, -np.inf, 1e-41],
                                  np.float32), (300, 64))
    x[300:600] = np.round(x[300:600])
    b = O.ggml_quantize(x)
    assert np.array_equal(b, O.ggml_quantize(x, G))
    assert np.array_equal(bits(O.ggml_dequantize(b)), bits(O.ggml_dequantize(b, G)))
    vx = b[:2000].reshape(250, 8 * 40)
    vy = rng.standard_normal((250, 512)).astype(np.float32)
    assert np.array_equal(bits(O.ggml_vec_dot(vx, vy)), bits(O.ggml_vec_dot(vx, vy, G)))
