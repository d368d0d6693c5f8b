"""GPU: the q4_1_eakv ggml type kernels (eakv_b200/csrc/ggml.cu) against
the restated reference (src/ggml_type.c:21-242, AVX-512 build), bit for
bit (NaN payloads aside, see same_f32): blocks, dequantized values and dot
products, through the device entry points and through the reference's
host-pointer names."""
import numpy as np
import pytest

import eakv_b200 as E
from conftest import golden
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def bits(a):
    return np.ascontiguousarray(a).view(np.uint32)


def same_f32(a, b):
    """Bit-equal, except that any NaN matches any NaN: the payload of a NaN
    that arithmetic makes (range = inf - inf, range / 15, fma with a NaN)
    is the hardware's own (x86 keeps an operand's payload or makes
    0xFFC00000, the GPU makes 0x7FFFFFFF), and neither format defines it."""
    a = np.ascontiguousarray(a, np.float32)
    b = np.ascontiguousarray(b, np.float32)
    return bool(np.all((bits(a) == bits(b)) | (np.isnan(a) & np.isnan(b))))


def same_blocks(a, b):
    """q4_1_eakv blocks: nibble bytes exactly, d and m by same_f32."""
    a = np.ascontiguousarray(a, np.uint8).reshape(-1, 40)
    b = np.ascontiguousarray(b, np.uint8).reshape(-1, 40)
    return (np.array_equal(a[:, :32], b[:, :32]) and
            same_f32(a[:, 32:].copy().view(np.float32), b[:, 32:].copy().view(np.float32)))


def test_host_entry_points_match_golden(gpu):
    g = golden("ggml.npz")
    L = E.lib()
    assert same_blocks(O.ggml_quantize(g["x"], L), g["blocks"])
    assert same_f32(O.ggml_dequantize(g["blocks"], L), g["deq"])
    assert same_f32(O.ggml_vec_dot(g["vx"], g["vy"], L), g["dot"])


@pytest.mark.parametrize("n_blocks", [1, 7, 4096, 100003])
def test_device_quantize_dequantize(gpu, n_blocks):
    import torch
    rng = np.random.default_rng(n_blocks)
    x = (rng.standard_normal((n_blocks, 64)) *
         np.exp(rng.uniform(-20, 20, (n_blocks, 1)))).astype(np.float32)
    k = min(n_blocks, 64)
    x[:k // 2] = rng.choice(np.array([0.0, -0.0, 1.0, np.nan, np.inf, -np.inf, 1e-41],
                                     np.float32), (k // 2, 64))
    ref = O.ggml_quantize(x)
    dx = torch.from_numpy(x).to(gpu)
    db = torch.zeros(n_blocks * 40, dtype=torch.uint8, device=gpu)
    E.ggml_quantize_row_device(dx, db, n_blocks * 64)
    torch.cuda.synchronize()
    assert same_blocks(db.cpu().numpy(), ref)
    out = torch.empty(n_blocks * 64, dtype=torch.float32, device=gpu)
    E.ggml_dequantize_row_device(db, out, n_blocks * 64)
    torch.cuda.synchronize()
    assert same_f32(out.cpu().numpy(), O.ggml_dequantize(ref))


def test_partial_block_is_ignored(gpu):
    """k = 64 nb + r quantizes nb blocks and writes nothing after them."""
    import torch
    rng = np.random.default_rng(3)
    x = rng.standard_normal(3 * 64 + 17).astype(np.float32)
    db = torch.full((4 * 40,), 0xAB, dtype=torch.uint8, device=gpu)
    E.ggml_quantize_row_device(torch.from_numpy(x).to(gpu), db, x.size)
    torch.cuda.synchronize()
    got = db.cpu().numpy()
    assert np.array_equal(got[:120].reshape(3, 40), O.ggml_quantize(x[:192]))
    assert (got[120:] == 0xAB).all()


@pytest.mark.parametrize("nrc,nb", [(1, 2), (2, 2), (333, 2), (40, 64), (5000, 1)])
def test_device_vec_dot(gpu, nrc, nb):
    import torch
    rng = np.random.default_rng(nrc * 7 + nb)
    x = (rng.standard_normal((nrc * nb, 64)) * 3).astype(np.float32)
    vx = O.ggml_quantize(x).reshape(nrc, nb * 40)
    vy = rng.standard_normal((nrc, nb * 64)).astype(np.float32)
    ref = O.ggml_vec_dot(vx, vy)
    s = torch.zeros(nrc, dtype=torch.float32, device=gpu)
    E.ggml_vec_dot_device(nb * 64, s, 4, torch.from_numpy(vx).to(gpu), nb * 40,
                          torch.from_numpy(vy).to(gpu), nb * 256, nrc)
    torch.cuda.synchronize()
    assert np.array_equal(bits(s.cpu().numpy()), bits(ref))


def test_device_vec_dot_strided_rows(gpu):
    """Rows at byte strides wider than a row, outputs at a stride."""
    import torch
    rng = np.random.default_rng(9)
    nrc, nb = 17, 3
    x = rng.standard_normal((nrc * nb, 64)).astype(np.float32)
    dense = O.ggml_quantize(x).reshape(nrc, nb * 40)
    vx = np.zeros((nrc, nb * 40 + 24), np.uint8)
    vx[:, :nb * 40] = dense
    vy = np.zeros((nrc, nb * 64 + 5), np.float32)
    vy[:, :nb * 64] = rng.standard_normal((nrc, nb * 64))
    ref = O.ggml_vec_dot(dense, np.ascontiguousarray(vy[:, :nb * 64]))
    s = torch.full((nrc * 3,), -1.0, dtype=torch.float32, device=gpu)
    E.ggml_vec_dot_device(nb * 64, s, 12, torch.from_numpy(vx).to(gpu), vx.shape[1],
                          torch.from_numpy(vy).to(gpu), vy.shape[1] * 4, nrc)
    torch.cuda.synchronize()
    got = s.cpu().numpy().reshape(nrc, 3)
    assert np.array_equal(bits(got[:, 0]), bits(ref))
    assert (got[:, 1:] == -1.0).all()


def test_invalid_arguments(gpu):
    with pytest.raises(E.EakvError):
        E.ggml_quantize_row_device(None, None, 64)
