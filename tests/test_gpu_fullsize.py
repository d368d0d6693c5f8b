"""GPU, full size: one sequence of the cfg4 shape (Llama-3-8B GQA 4:1, 32
layers x 8 KV heads x 32768 positions x head_dim 128, 1.34 GB of Q4), where
the oracle cannot run the whole step in seconds. Checked through properties
that do not depend on size:

* sampled rows against a float64 softmax-attention over the cache's own
  dequantized K and V (the quantizer is bit-exact to the reference, tested
  elsewhere), at the 1e-4 bar;
* the same rows with splits of 256 pages, the longest the planner makes;
* V linearity: a cache holding 2V gives exactly twice the output, bit for
  bit (doubling V doubles every scale and bias exactly and leaves the
  nibbles alone; the kernel's power-of-two operand scaling absorbs it);
* quantize round trip: every dequantized element within half a quantum
  (scale / 2, plus rounding) of its input."""
import numpy as np
import pytest

import eakv_b200 as E
from conftest import HAS_GPU
from gpu_util import assert_close, bits

pytestmark = pytest.mark.gpu

L, NQ, H, HD, S = 32, 32, 8, 128, 32768


@pytest.fixture(scope="module")
def full():
    if not HAS_GPU:
        pytest.skip("no CUDA device")
    import torch
    torch.cuda.set_device(0)
    gpu = torch.device("cuda:0")
    g = torch.Generator(device=gpu)
    g.manual_seed(2024)
    ch = torch.exp(torch.empty(L, H, 1, HD, device=gpu).uniform_(np.log(0.5), np.log(8.0),
                                                                  generator=g))
    a = E.Cache(L, H, HD, S)
    b = E.Cache(L, H, HD, S)
    vs = {}
    for l in range(L):
        k = torch.randn(H, S, HD, device=gpu, generator=g) * ch[l]
        v = torch.randn(H, S, HD, device=gpu, generator=g)
        v2 = v * 2.0
        # the caches quantize on their own streams: the inputs must be
        # complete before, and alive until, those kernels have run
        torch.cuda.synchronize()
        for c, vv in ((a, v), (b, v2)):
            assert c.append_device(k, l, 0, S) == 0
            assert c.append_device(vv, l, 1, S) == 0
        a.synchronize()
        b.synchronize()
        if l in (0, 31):
            vs[l] = (k.cpu().numpy(), v.cpu().numpy())
    for c in (a, b):
        assert c.advance(S) == 0
    q = torch.randn(1, L, NQ, HD, device=gpu, generator=g)
    torch.cuda.synchronize()
    yield a, b, q, vs
    a.free()
    b.free()


def decode(cache, q):
    import torch
    out = torch.empty_like(q)
    s = torch.cuda.Stream()
    E.decode_attention([cache], q, NQ, out, stream=s.cuda_stream)
    s.synchronize()
    return out.cpu().numpy()


def check_rows(a, q, out):
    qn = q.cpu().numpy()[0]
    G = NQ // H
    for l, h in [(0, 0), (7, 5), (31, 7)]:
        k = a.dequantize(l, 0, 0, S)[h].astype(np.float64)     # [S][HD]
        v = a.dequantize(l, 1, 0, S)[h].astype(np.float64)
        for j in range(G):
            qh = qn[l, h * G + j].astype(np.float64)
            sc = k @ qh / np.sqrt(HD)
            p = np.exp(sc - sc.max())
            ref = (p @ v) / p.sum()
            assert_close(out[l, h * G + j], ref, what=f"layer {l} head {h * G + j}")
    assert E.device_status(0) == 0


def test_sampled_rows_against_float64(full):
    a, _, q, _ = full
    check_rows(a, q, decode(a, q)[0])


def test_longest_splits_against_float64(full):
    """Splits of 256 pages, the longest the planner makes (the tensor core's
    f32 accumulators drift past the bar over one 512-page row)."""
    a, _, q, _ = full
    E.force_splits(S // 64 // 256)
    try:
        out = decode(a, q)[0]
    finally:
        E.force_splits(0)
    check_rows(a, q, out)


def test_v_linearity_is_exact(full):
    a, b, q, _ = full
    assert np.array_equal(bits(decode(b, q) / 2.0), bits(decode(a, q)))


def test_quantize_round_trip(full):
    a, _, _, vs = full
    for l, (k, v) in vs.items():
        for kv, x in ((0, k), (1, v)):
            d = a.dequantize(l, kv, 0, S)                      # [H][S][HD]
            xr = x.reshape(H, S, HD // 64, 64)
            span = xr.max(axis=-1, keepdims=True) - xr.min(axis=-1, keepdims=True)
            err = np.abs(d.reshape(xr.shape) - xr)
            # half a quantum (range / 30) plus the f32 rounding of the arithmetic
            assert (err <= span / 30 * (1 + 1e-5) + 1e-6 * np.abs(xr)).all(), (l, kv)
