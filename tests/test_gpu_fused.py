"""GPU parity of the fused flash-decoding path against the oracle's
two-pass fused attention (reference kernels/fused_attention.ea:190-373,
generalised to GQA and head_dim 64): |err| <= 1e-4 + 1e-4*|ref|."""
import numpy as np
import pytest

import eakv_b200 as E
from conftest import golden
from gpu_util import PATH_CODE, assert_close, kv_data
from oracle import oracle as O

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _reset_splits():
    E.force_splits(0)
    E.force_path(0)
    yield
    E.force_splits(0)
    E.force_path(0)


# "auto" is the library's own choice; "simt" forces the CUDA-core kernel,
# "mma" the mma.sync tensor-core kernel and "umma" the tcgen05 kernel (shapes
# a forced kernel does not serve fall back to the automatic choice)
PATHS = ["auto", "simt", "mma", "umma"]
# the two tensor-core formulations, for the edge cases below (the tcgen05 one
# serves head_dim 128; its cases use that head_dim)
TC_PATHS = ["auto", "umma"]


@pytest.mark.parametrize("path", TC_PATHS)
@pytest.mark.parametrize("name", ["mha128", "gqa64_8to2", "gqa128_4to1", "mha64"])
def test_golden_fused(gpu, name, path):
    E.force_path(PATH_CODE[path])
    g = golden(f"attn_{name}.npz")
    L, nq, nkv, hd, S, maxS = [int(v) for v in g["shape"]]
    with E.Cache(L, nkv, hd, maxS) as c:
        assert c.load_raw(g["data"], S) == 0
        for l in range(L):
            assert_close(c.fused(g["q"][l], l, nq, nkv), g["fused"][l], what=name)


CASES = [
    # L, nq, nkv, hd, S, maxS
    (1, 8, 8, 128, 1, 16),
    (1, 8, 8, 128, 2048, 2048),     # config 1 shape
    (2, 32, 4, 64, 1000, 1024),     # GQA 8:1, head_dim 64
    (1, 32, 8, 128, 3000, 3100),    # GQA 4:1
    (1, 64, 8, 128, 700, 700),      # GQA 8:1, head_dim 128
    (1, 4, 2, 64, 130, 200),        # GQA 2:1
    (1, 12, 4, 128, 333, 400),      # ratio 3 (odd group)
    (1, 7, 1, 64, 95, 100),         # ratio 7
    (1, 16, 1, 128, 257, 300),      # ratio 16 (two passes)
]


@pytest.mark.parametrize("path", PATHS)
@pytest.mark.parametrize("L,nq,nkv,hd,S,maxS", CASES)
def test_fused_random(gpu, L, nq, nkv, hd, S, maxS, path):
    E.force_path(PATH_CODE[path])
    rng = np.random.default_rng(S * 7 + nq)
    data = kv_data(rng, L, nkv, S, hd)
    rc = O.RefCache(L, nkv, hd, maxS)
    rc.load_raw(data, S)
    with E.Cache(L, nkv, hd, maxS) as c:
        assert c.load_raw(data, S) == 0
        for l in range(L):
            q = rng.standard_normal(nq * hd).astype(np.float32)
            assert_close(c.fused(q, l, nq, nkv), rc.fused(q, l, nq, nkv), what=f"layer {l}")


@pytest.mark.parametrize("path", PATHS)
@pytest.mark.parametrize("splits", [1, 2, 3, 7, 64])
def test_forced_splits(gpu, splits, path):
    """Split + exact LSE combine gives the same result as one pass."""
    E.force_path(PATH_CODE[path])
    L, nq, nkv, hd, S = 1, 16, 4, 128, 1111
    rng = np.random.default_rng(splits)
    data = kv_data(rng, L, nkv, S, hd)
    rc = O.RefCache(L, nkv, hd, S)
    rc.load_raw(data, S)
    q = rng.standard_normal(nq * hd).astype(np.float32)
    with E.Cache(L, nkv, hd, S) as c:
        assert c.load_raw(data, S) == 0
        E.force_splits(splits)
        assert_close(c.fused(q, 0, nq, nkv), rc.fused(q, 0, nq, nkv), what=f"{splits} splits")


@pytest.mark.parametrize("path", PATHS)
def test_large_scores_softmax_stability(gpu, path):
    """Queries scaled x30: scores in the hundreds, softmax near one-hot."""
    E.force_path(PATH_CODE[path])
    L, nq, nkv, hd, S = 1, 8, 2, 128, 500
    rng = np.random.default_rng(77)
    data = kv_data(rng, L, nkv, S, hd)
    rc = O.RefCache(L, nkv, hd, S)
    rc.load_raw(data, S)
    q = (rng.standard_normal(nq * hd) * 30).astype(np.float32)
    with E.Cache(L, nkv, hd, S) as c:
        assert c.load_raw(data, S) == 0
        assert_close(c.fused(q, 0, nq, nkv), rc.fused(q, 0, nq, nkv), what="sharp softmax")


@pytest.mark.parametrize("path,hd", [("auto", 64), ("umma", 128)])
def test_decode_batch_ragged(gpu, path, hd):
    """Batched decode over caches of different lengths and every layer."""
    import torch
    E.force_path(PATH_CODE[path])
    B, L, nq, nkv, maxS = 5, 3, 16, 4, 600
    lens = [1, 64, 65, 333, 600]
    rng = np.random.default_rng(21)
    caches, refs = [], []
    for b in range(B):
        data = kv_data(rng, L, nkv, lens[b], hd)
        c = E.Cache(L, nkv, hd, maxS)
        assert c.load_raw(data, lens[b]) == 0
        rc = O.RefCache(L, nkv, hd, maxS)
        rc.load_raw(data, lens[b])
        caches.append(c)
        refs.append(rc)
    q = rng.standard_normal((B, L, nq, hd)).astype(np.float32)
    dq = torch.from_numpy(q).to(gpu)
    do = torch.full((B, L, nq, hd), float("nan"), device=gpu)
    E.decode_attention(caches, dq, nq, do)
    caches[0].synchronize()
    out = do.cpu().numpy()
    for b in range(B):
        for l in range(L):
            assert_close(out[b, l].reshape(-1), refs[b].fused(q[b, l], l, nq, nkv),
                         what=f"cache {b} layer {l}")
    # host-buffer variant
    out2 = np.zeros_like(q)
    E.decode_attention_host(caches, q, nq, out2)
    np.testing.assert_array_equal(out2, out)
    for c in caches:
        c.free()


@pytest.mark.parametrize("shape", ["by_cache", "by_layer"])
@pytest.mark.parametrize("pinned", [False, True])
def test_decode_host_pipelined(gpu, shape, pinned):
    """At 256 KiB of queries and more, the host-buffer decode runs in chunks
    (caches, or the layers of a single cache) whose copies overlap the
    other chunks' decodes; every chunk keeps the whole batch's split plan,
    so the outputs equal the device-buffer form's bit for bit."""
    import torch
    if shape == "by_cache":
        lens, L, nq, nkv, hd, maxS = [1, 64, 100, 333, 257, 129], 6, 64, 8, 128, 400
    else:
        lens, L, nq, nkv, hd, maxS = [130], 33, 64, 8, 128, 130
    B = len(lens)
    assert B * L * nq * hd * 4 >= 1 << 20   # the size at which chunking starts
    rng = np.random.default_rng(77)
    caches, refs = [], []
    for b in range(B):
        data = kv_data(rng, L, nkv, lens[b], hd)
        c = E.Cache(L, nkv, hd, maxS)
        assert c.load_raw(data, lens[b]) == 0
        rc = O.RefCache(L, nkv, hd, maxS)
        rc.load_raw(data, lens[b])
        caches.append(c)
        refs.append(rc)
    q = rng.standard_normal((B, L, nq, hd)).astype(np.float32)
    do = torch.full((B, L, nq, hd), float("nan"), device=gpu)
    E.decode_attention(caches, torch.from_numpy(q).to(gpu), nq, do)
    caches[0].synchronize()
    out = do.cpu().numpy()
    if pinned:
        qh = torch.from_numpy(q).pin_memory()
        oh = torch.full((B, L, nq, hd), float("nan")).pin_memory()
        E.decode_attention_host(caches, qh, nq, oh)
        out2 = oh.numpy()
    else:
        out2 = np.full_like(q, np.nan)
        E.decode_attention_host(caches, q, nq, out2)
    np.testing.assert_array_equal(out2, out)
    for b in range(B):
        for l in (0, L // 2, L - 1):
            assert_close(out2[b, l].reshape(-1), refs[b].fused(q[b, l], l, nq, nkv),
                         what=f"cache {b} layer {l}")
    for c in caches:
        c.free()


@pytest.mark.parametrize("path", TC_PATHS)
def test_partial_ranges_and_lse_combine(gpu, path):
    """Sequence split across (simulated) ranks: partial outputs + LSE over
    disjoint position ranges, merged by eakv_lse_combine == full attention."""
    import torch
    E.force_path(PATH_CODE[path])
    L, nq, nkv, hd, S = 2, 8, 2, 128, 1000
    rng = np.random.default_rng(33)
    data = kv_data(rng, L, nkv, S, hd)
    rc = O.RefCache(L, nkv, hd, S)
    rc.load_raw(data, S)
    q = rng.standard_normal((1, L, nq, hd)).astype(np.float32)
    bounds = [0, 100, 100, 101, 640, 1000]   # includes an empty range
    P = len(bounds) - 1
    with E.Cache(L, nkv, hd, S) as c:
        assert c.load_raw(data, S) == 0
        dq = torch.from_numpy(q).to(gpu)
        parts = torch.empty((P, L * nq, hd), device=gpu)
        lse = torch.empty((P, L * nq), device=gpu)
        for p in range(P):
            E.decode_attention_partial([c], dq, nq, bounds[p], bounds[p + 1], parts[p], lse[p])
        c.synchronize()
        for p in range(P):
            if bounds[p] == bounds[p + 1]:
                assert torch.isneginf(lse[p]).all()   # empty range: no weight in the merge
                continue
            for l in range(L):
                ref = rc.fused(q[0, l], l, nq, nkv, seq_range=(bounds[p], bounds[p + 1]))
                assert_close(parts[p, l * nq:(l + 1) * nq].cpu().numpy().reshape(-1), ref,
                             what=f"part {p} layer {l}")
        out = torch.empty((L * nq, hd), device=gpu)
        lse_out = torch.empty(L * nq, device=gpu)
        E.lse_combine(P, L * nq, hd, parts, lse, out, lse_out)
        torch.cuda.synchronize()
        for l in range(L):
            assert_close(out[l * nq:(l + 1) * nq].cpu().numpy().reshape(-1),
                         rc.fused(q[0, l], l, nq, nkv), what=f"combined layer {l}")
        # empty range: lse = -inf, merging it changes nothing
        E.decode_attention_partial([c], dq, nq, 1000, 1000, parts[0], lse[0])
        c.synchronize()
        assert torch.isneginf(lse[0]).all()


@pytest.mark.parametrize("path", TC_PATHS)
def test_fused_empty_cache_is_nan(gpu, path):
    """seq_len 0: the reference's fused kernel divides 0 by a zero sum."""
    E.force_path(PATH_CODE[path])
    with E.Cache(1, 2, 128, 64) as c:
        out = c.fused(np.ones(4 * 128, np.float32), 0, 4, 2)
        assert np.isnan(out).all()


@pytest.mark.parametrize("path,hd", [("auto", 64), ("umma", 128)])
def test_restore_limits_attention(gpu, path, hd):
    """After restore(n), attention sees exactly the first n positions."""
    E.force_path(PATH_CODE[path])
    L, nq, nkv, S = 1, 4, 4, 300
    rng = np.random.default_rng(8)
    data = kv_data(rng, L, nkv, S, hd)
    rc = O.RefCache(L, nkv, hd, S)
    rc.load_raw(data, S)
    rc.seq_len = 190
    with E.Cache(L, nkv, hd, S) as c:
        assert c.load_raw(data, S) == 0
        assert c.restore(190) == 0
        q = rng.standard_normal(nq * hd).astype(np.float32)
        assert_close(c.fused(q, 0, nq, nkv), rc.fused(q, 0, nq, nkv), what="restored")


def test_device_status_clean(gpu):
    assert E.device_status(0, reset=False) == 0


@pytest.mark.parametrize("path", TC_PATHS)
@pytest.mark.parametrize("vscale", [1e-30, 1e-3, 1.0, 1e4, 1e30])
def test_extreme_value_scales(gpu, vscale, path):
    """V values over 60 orders of magnitude and a K/V range that grows
    along the sequence: the tensor-core paths rescale their P' operands
    (f16 limbs, or the tcgen05 kernel's fixed point) by the V-scale exponent."""
    E.force_path(PATH_CODE[path])
    L, nq, nkv, hd, S = 1, 16, 4, 128, 640
    rng = np.random.default_rng(int(np.log10(vscale)) + 100)
    data = kv_data(rng, L, nkv, S, hd)
    data[0, 1] *= np.float32(vscale)
    data[0, 1, :, S // 2:] *= np.float32(64.0)      # scales jump mid-sequence
    rc = O.RefCache(L, nkv, hd, S)
    rc.load_raw(data, S)
    q = rng.standard_normal(nq * hd).astype(np.float32)
    with E.Cache(L, nkv, hd, S) as c:
        assert c.load_raw(data, S) == 0
        ref = rc.fused(q, 0, nq, nkv)
        got = c.fused(q, 0, nq, nkv)
        assert_close(got / vscale, ref / vscale, what=f"V scale {vscale}")


@pytest.mark.parametrize("path,hd", [("auto", 64), ("umma", 128)])
@pytest.mark.parametrize("qscale", [1e-6, 1e-2, 1e3])
def test_query_magnitudes(gpu, qscale, path, hd):
    E.force_path(PATH_CODE[path])
    L, nq, nkv, S = 1, 32, 4, 300
    rng = np.random.default_rng(5)
    data = kv_data(rng, L, nkv, S, hd)
    rc = O.RefCache(L, nkv, hd, S)
    rc.load_raw(data, S)
    q = (rng.standard_normal(nq * hd) * qscale).astype(np.float32)
    with E.Cache(L, nkv, hd, S) as c:
        assert c.load_raw(data, S) == 0
        assert_close(c.fused(q, 0, nq, nkv), rc.fused(q, 0, nq, nkv), what=f"q x{qscale}")


@pytest.mark.parametrize("path", PATHS)
@pytest.mark.parametrize("L,nq,nkv,hd,lens,splits", [
    (2, 32, 8, 128, [3000, 1, 640, 2999], 0),   # planner's splits, ragged batch
    (3, 64, 8, 128, [1300, 700], 5),             # 8 heads per CTA
    (2, 32, 4, 64, [2048], 7),                   # head_dim 64, 8:1
    (1, 8, 8, 128, [2048, 100], 3),              # MHA (one live head of four)
    (1, 12, 4, 128, [999], 4),                   # ratio 3
])
def test_split_merge_in_kernel_equals_separate_pass(gpu, path, L, nq, nkv, hd, lens, splits):
    """The last CTA of a row group merges the group's splits inside the decode
    launch; a second kernel doing the same merge after the decode gives the
    same bits. Three calls in a row: every call returns the split counters to
    zero, so each call merges exactly once per row group."""
    import torch
    E.force_path(PATH_CODE[path])
    rng = np.random.default_rng(sum(lens) + nq)
    maxS = max(lens)
    caches = []
    for n in lens:
        c = E.Cache(L, nkv, hd, maxS)
        assert c.load_raw(kv_data(rng, L, nkv, n, hd), n) == 0
        caches.append(c)
    E.force_splits(splits)
    try:
        assert E.decode_splits(caches, nq) > 1
        assert E.decode_launches(caches, nq) == 1
        for call in range(3):
            q = torch.from_numpy(
                rng.standard_normal((len(lens), L, nq, hd)).astype(np.float32)).to(gpu)
            one = torch.full_like(q, float("nan"))
            two = torch.full_like(q, float("nan"))
            E.decode_attention(caches, q, nq, one)
            E.separate_merge(True)
            try:
                E.decode_attention(caches, q, nq, two)
            finally:
                E.separate_merge(False)
            caches[0].synchronize()
            assert torch.equal(one.view(torch.int32), two.view(torch.int32)), f"call {call}"
            assert not torch.isnan(one).any()
    finally:
        E.force_splits(0)
    assert E.device_status(0) == 0
    for c in caches:
        c.free()
