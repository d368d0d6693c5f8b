"""GPU, at size: one sequence of each remaining BASELINE shape, decoded whole
(every layer, every head, all positions) through the C ABI, with three
sampled layers checked row by row.

* cfg5: Llama-3-70B GQA 8:1, 80 layers x 64 Q / 8 KV heads x 131072
  positions x head_dim 128 (13.4 GB of Q4): the 8-head tensor-core kernel.
* cfg3: Llama-2-7B MHA, 32 layers x 32 / 32 heads x 8192 positions x 128.
* cfg2: TinyLlama GQA 8:1, 22 layers x 32 Q / 4 KV heads x 2048 x 64.

The K/V of every layer are generated on the device; those of the sampled
layers are also copied to the host and loaded into a one-layer oracle cache (the reference's layout and quantizer, bit-exact with
the device's), whose two-pass fused attention (kernels/fused_attention.ea:
190-373) is the parity reference for every query head of the layer. A
float64 attention over the oracle's dequantized K and V measures the
device's own precision. Each check runs with the planner's splits, with the
longest splits the planner allows (256 pages), and on the CUDA-core kernel.

The worst error is recorded as a fraction of the 1e-4 abs + 1e-4 rel bar;
with EAKV_PARITY_REPORT=<file> set, one JSON line per check is appended
there."""
import json
import os

import numpy as np
import pytest

import eakv_b200 as E
from conftest import HAS_GPU
from oracle import oracle as O

pytestmark = pytest.mark.gpu

SHAPES = {
    "cfg5": dict(L=80, NQ=64, H=8, HD=128, S=131072, layers=(0, 41, 79)),
    "cfg3": dict(L=32, NQ=32, H=32, HD=128, S=8192, layers=(0, 17, 31)),
    "cfg2": dict(L=22, NQ=32, H=4, HD=64, S=2048, layers=(0, 11, 21)),
}
MAX_SPLIT_PAGES = 256


def tol_frac(got, ref, atol=1e-4, rtol=1e-4):
    """Largest |got - ref| / (atol + rtol |ref|): 1.0 is the parity bar."""
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    return float(np.max(np.abs(got - ref) / (atol + rtol * np.abs(ref))))


def report(**kw):
    path = os.environ.get("EAKV_PARITY_REPORT")
    if path:
        with open(path, "a") as f:
            f.write(json.dumps(kw) + "\n")


@pytest.fixture(scope="module", params=sorted(SHAPES))
def shape(request):
    if not HAS_GPU:
        pytest.skip("no CUDA device")
    import torch
    name = request.param
    p = SHAPES[name]
    L, NQ, H, HD, S = p["L"], p["NQ"], p["H"], p["HD"], p["S"]
    torch.cuda.set_device(0)
    gpu = torch.device("cuda:0")
    rng = np.random.default_rng(31 + L)
    g = torch.Generator(device=gpu)
    g.manual_seed(77 + L)
    c = E.Cache(L, H, HD, S)
    refs = {}
    for l in range(L):
        # K = N(0,1) x per-channel log-uniform [0.5, 8], V = N(0,1)
        ch = torch.exp(torch.empty(H, 1, HD, device=gpu).uniform_(np.log(0.5), np.log(8.0),
                                                                   generator=g))
        k = torch.randn(H, S, HD, device=gpu, generator=g) * ch
        v = torch.randn(H, S, HD, device=gpu, generator=g)
        torch.cuda.synchronize()   # the cache quantizes on its own stream
        assert c.append_device(k, l, 0, S) == 0
        assert c.append_device(v, l, 1, S) == 0
        c.synchronize()
        if l in p["layers"]:
            r = O.RefCache(1, H, HD, S)
            r.load_raw(torch.stack([k, v]).cpu().numpy()[None], S)
            refs[l] = r
    assert c.advance(S) == 0
    qn = rng.standard_normal((1, L, NQ, HD), dtype=np.float32)
    q = torch.from_numpy(qn).to(gpu)
    yield name, p, c, refs, qn, q
    c.free()


def decode(cache, q, NQ):
    import torch
    out = torch.full_like(q, float("nan"))
    s = torch.cuda.Stream()
    E.decode_attention([cache], q, NQ, out, stream=s.cuda_stream)
    s.synchronize()
    return out.cpu().numpy()[0]


_exact = {}


def exact_and_oracle(name, p, refs, qn):
    """Per sampled layer: the float64 attention over the quantized K/V and the
    oracle's two-pass f32 result (computed once per shape)."""
    if name not in _exact:
        NQ, H, HD = p["NQ"], p["H"], p["HD"]
        G = NQ // H
        res = {}
        for l, r in refs.items():
            want = r.fused(qn[0, l], 0, NQ, H).reshape(NQ, HD)
            ex = np.empty((NQ, HD))
            for h in range(H):
                k = r.dequant_head(0, 0, h).astype(np.float64)
                v = r.dequant_head(0, 1, h).astype(np.float64)
                qh = qn[0, l, h * G:(h + 1) * G].astype(np.float64)      # [G][HD]
                sc = k @ qh.T / np.sqrt(HD)                              # [S][G]
                pr = np.exp(sc - sc.max(axis=0))
                ex[h * G:(h + 1) * G] = (pr.T @ v) / pr.sum(axis=0)[:, None]
            res[l] = (ex, want)
        _exact.clear()
        _exact[name] = res
    return _exact[name]


def check(name, mode, p, refs, qn, out):
    """The device result against the float64 attention (its precision, held
    to the bar) and against the oracle. The oracle runs the reference's f32
    two-pass algorithm, whose sequential sums drop the smallest weights once
    the running sum is large: at 131072 positions that costs it up to ~1e-3
    relative, more than the bar. So the device must match the oracle within
    the bar, or else be closer to the exact result than the oracle is."""
    worst_o = worst_f = oracle_f = 0.0
    for l, (ex, want) in exact_and_oracle(name, p, refs, qn).items():
        worst_o = max(worst_o, tol_frac(out[l], want))
        worst_f = max(worst_f, tol_frac(out[l], ex))
        oracle_f = max(oracle_f, tol_frac(want, ex))
    report(shape=name, mode=mode, frac_vs_oracle=worst_o, frac_vs_float64=worst_f,
           oracle_frac_vs_float64=oracle_f)
    assert worst_f <= 1.0, f"{name} {mode}: {worst_f:.3f} of the bar against float64"
    assert worst_o <= 1.0 or worst_f < oracle_f, (
        f"{name} {mode}: {worst_o:.3f} of the bar against the oracle, whose own error is "
        f"{oracle_f:.3f} of it (device: {worst_f:.3f})")
    assert E.device_status(0) == 0


def test_planner_splits(shape):
    name, p, c, refs, qn, q = shape
    check(name, f"planner ({E.decode_splits([c], p['NQ'])} splits)", p, refs, qn,
          decode(c, q, p["NQ"]))


def test_longest_splits(shape):
    """Splits of 256 pages (the precision cap of the tensor-core kernel's
    f32 accumulators), or one split when the row is shorter."""
    name, p, c, refs, qn, q = shape
    n = max(1, p["S"] // 64 // MAX_SPLIT_PAGES)
    E.force_splits(n)
    try:
        out = decode(c, q, p["NQ"])
    finally:
        E.force_splits(0)
    check(name, f"longest ({n} splits)", p, refs, qn, out)


def test_cuda_core_kernel(shape):
    """The independent CUDA-core formulation of the same decode."""
    name, p, c, refs, qn, q = shape
    E.force_path(1)
    try:
        out = decode(c, q, p["NQ"])
    finally:
        E.force_path(0)
    check(name, "cuda-core kernel, planner splits", p, refs, qn, out)


@pytest.mark.parametrize("longest", [False, True], ids=["planner", "longest"])
def test_tcgen05_kernel(shape, longest):
    """The tcgen05 formulation (exact s32 accumulation of the V side in
    tensor memory, 32-bit fixed-point P'); head_dim 128 shapes only (others
    keep the automatic choice and are covered above)."""
    name, p, c, refs, qn, q = shape
    if p["HD"] != 128:
        pytest.skip("the tcgen05 kernel serves head_dim 128")
    n = max(1, p["S"] // 64 // MAX_SPLIT_PAGES) if longest else 0
    E.force_path(3)
    E.force_splits(n)
    try:
        out = decode(c, q, p["NQ"])
    finally:
        E.force_path(0)
        E.force_splits(0)
    check(name, f"tcgen05 kernel, {'longest' if longest else 'planner'} splits", p, refs, qn, out)
