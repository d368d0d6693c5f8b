"""GPU parity of the two-call attention API (eakv_attention_scores /
eakv_attention_output) against the reference's results.

Scores are computed in the reference's exact operation order and must be
bit-identical; the V-sum is bit-identical while the sequence fits one chunk
(<= 512 positions) and within |err| <= 1e-4 + 1e-4*|ref| beyond.
"""
import numpy as np
import pytest

import eakv_b200 as E
from conftest import golden
from gpu_util import assert_close, bits, kv_data
from oracle import oracle as O

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("name", ["mha128", "gqa64_8to2", "gqa128_4to1", "mha64"])
def test_golden_two_call(gpu, name):
    g = golden(f"attn_{name}.npz")
    L, nq, nkv, hd, S, maxS = [int(v) for v in g["shape"]]
    with E.Cache(L, nkv, hd, maxS) as c:
        assert c.load_raw(g["data"], S) == 0
        for l in range(L):
            s = c.scores(g["q"][l], l, nq, nkv)
            assert np.array_equal(bits(s), bits(g["scores"][l])), "scores not bit-exact"
            o = c.output(g["weights"][l], l, nq, nkv)
            assert np.array_equal(bits(o), bits(g["output"][l])), "V-sum not bit-exact"


CASES = [
    # L, nq, nkv, hd, S, maxS
    (1, 8, 8, 128, 1, 16),
    (1, 8, 8, 128, 63, 64),
    (2, 4, 4, 64, 65, 100),
    (1, 32, 4, 64, 777, 1024),      # TinyLlama ratio 8:1
    (1, 32, 8, 128, 1500, 1600),    # Llama-3 ratio 4:1
    (1, 16, 16, 128, 2048, 2048),   # README bench shape family
    (1, 12, 4, 128, 300, 333),      # ratio 3
    (1, 64, 8, 128, 600, 640),      # ratio 8, head_dim 128
]


@pytest.mark.parametrize("L,nq,nkv,hd,S,maxS", CASES)
def test_random_two_call(gpu, L, nq, nkv, hd, S, maxS):
    rng = np.random.default_rng(S + nq)
    data = kv_data(rng, L, nkv, S, hd)
    rc = O.RefCache(L, nkv, hd, maxS)
    rc.load_raw(data, S)
    with E.Cache(L, nkv, hd, maxS) as c:
        assert c.load_raw(data, S) == 0
        for l in range(L):
            q = rng.standard_normal(nq * hd).astype(np.float32)
            s_ref = rc.scores(q, l, nq, nkv)
            s = c.scores(q, l, nq, nkv)
            assert np.array_equal(bits(s), bits(s_ref)), "scores not bit-exact"
            w = O.softmax_rows(s_ref, nq, S)
            o_ref = rc.output(w, l, nq, nkv)
            o = c.output(w, l, nq, nkv)
            if S <= 512:
                assert np.array_equal(bits(o), bits(o_ref)), "V-sum not bit-exact"
            else:
                assert_close(o, o_ref, what="V-sum")


def test_subset_kv_heads_and_uniform_weights(gpu):
    """n_kv below the cache's head count attends the first n_kv heads, as
    the reference's kernels do; uniform weights as in its bench."""
    L, H, hd, S = 1, 8, 128, 256
    rng = np.random.default_rng(9)
    data = kv_data(rng, L, H, S, hd)
    rc = O.RefCache(L, H, hd, S)
    rc.load_raw(data, S)
    with E.Cache(L, H, hd, S) as c:
        assert c.load_raw(data, S) == 0
        q = rng.standard_normal(4 * hd).astype(np.float32)
        assert np.array_equal(bits(c.scores(q, 0, 4, 4)), bits(rc.scores(q, 0, 4, 4)))
        w = np.full(4 * S, 1.0 / S, np.float32)
        assert np.array_equal(bits(c.output(w, 0, 4, 4)), bits(rc.output(w, 0, 4, 4)))


@pytest.mark.parametrize("S", [513, 1000, 4097])
@pytest.mark.parametrize("H,nq,nkv", [(8, 8, 8), (8, 32, 8), (8, 4, 4)])
def test_chunked_v_sum(gpu, S, H, nq, nkv):
    """Beyond 512 positions the V-sum runs in blocks of 1..8 pages chosen
    from the call's size (more, shorter blocks for short sequences), and the
    last block of each head group adds the blocks' sums in order: within the
    tolerance of the reference's single chain, also when n_kv is below the
    cache's head count. The blocks meet at counters in the cache's workspace,
    which the fused decode uses too: a decode between two V-sums leaves the
    second one bit-identical to the first."""
    chunked_case(S, H, nq, nkv)


@pytest.mark.parametrize("S", [20000, 32768, 36000])
def test_chunked_v_sum_many_blocks(gpu, S):
    """Long sequences (8-page blocks): 40 and 64 blocks per sequence are
    merged by the last block inside the launch, 71 by a second kernel."""
    chunked_case(S, 8, 32, 8)


@pytest.mark.parametrize("S", [300, 1000, 20000, 36000])
def test_v_sum_device_buffers_at_any_float_offset(gpu, S):
    """The device V-sum takes the caller's weight and output buffers at any
    4-byte offset (here one float past a 256-byte boundary): one block
    writing the output itself (300 positions), the blocks' sums merged inside
    the launch (16 and 40 blocks) or by a second kernel (71); it equals the
    host-buffer call bit for bit."""
    import torch
    L, H, nq, nkv, hd = 1, 8, 32, 8, 128
    rng = np.random.default_rng(S + 5)
    data = kv_data(rng, L, H, S, hd)
    with E.Cache(L, H, hd, S) as c:
        assert c.load_raw(data, S) == 0
        w = rng.random(nq * S, dtype=np.float32) / S
        want = c.output(w, 0, nq, nkv)
        wbuf = torch.zeros(nq * S + 1, device=gpu)
        wbuf[1:] = torch.from_numpy(w).to(gpu)
        obuf = torch.full((nq * hd + 1,), float("nan"), device=gpu)
        torch.cuda.synchronize()   # the cache runs on its own stream
        c.output_device(wbuf[1:], 0, nq, nkv, obuf[1:])
        c.synchronize()
        assert np.array_equal(bits(obuf[1:].cpu().numpy()), bits(want))
    assert E.device_status(0) == 0


def chunked_case(S, H, nq, nkv):
    L, hd = 1, 128
    rng = np.random.default_rng(S * 3 + nq)
    data = kv_data(rng, L, H, S, hd)
    rc = O.RefCache(L, H, hd, S)
    rc.load_raw(data, S)
    with E.Cache(L, H, hd, S) as c:
        assert c.load_raw(data, S) == 0
        q = rng.standard_normal(nq * hd).astype(np.float32)
        w = O.softmax_rows(rc.scores(q, 0, nq, nkv), nq, S)
        o1 = c.output(w, 0, nq, nkv)
        assert_close(o1, rc.output(w, 0, nq, nkv), what=f"V-sum S={S}")
        if nkv == H:
            c.fused(q, 0, nq, nkv)
        o2 = c.output(w, 0, nq, nkv)
        assert np.array_equal(bits(o1), bits(o2)), "repeated V-sum differs"
    assert E.device_status(0) == 0


def test_device_entry_points(gpu):
    import torch
    L, nq, nkv, hd, S = 1, 16, 4, 128, 200
    rng = np.random.default_rng(4)
    data = kv_data(rng, L, nkv, S, hd)
    rc = O.RefCache(L, nkv, hd, S)
    rc.load_raw(data, S)
    with E.Cache(L, nkv, hd, S) as c:
        d = torch.from_numpy(data).to(gpu)
        assert c.load_raw_device(d, S) == 0
        q = rng.standard_normal(nq * hd).astype(np.float32)
        dq = torch.from_numpy(q).to(gpu)
        ds = torch.empty(nq * S, device=gpu)
        assert E.lib().eakv_attention_scores_device(c.h, dq.data_ptr(), 0, nq, nkv,
                                                    ds.data_ptr()) == 0
        c.synchronize()
        s_ref = rc.scores(q, 0, nq, nkv)
        assert np.array_equal(bits(ds.cpu().numpy()), bits(s_ref))
        w = O.softmax_rows(s_ref, nq, S)
        dw = torch.from_numpy(w).to(gpu)
        do = torch.empty(nq * hd, device=gpu)
        assert E.lib().eakv_attention_output_device(c.h, dw.data_ptr(), 0, nq, nkv,
                                                    do.data_ptr()) == 0
        c.synchronize()
        assert np.array_equal(bits(do.cpu().numpy()), bits(rc.output(w, 0, nq, nkv)))


def test_rejected_calls_fill_nan(gpu):
    """The reference runs out of bounds on these; here they are refused with
    NaN output and an error code (its attention calls return void)."""
    with E.Cache(1, 4, 128, 32) as c:
        assert c.load_raw(np.ones((1, 2, 4, 32, 128), np.float32), 32) == 0
        q = np.ones(6 * 128, np.float32)
        s = c.scores(q, 0, 6, 4)              # 6 % 4 != 0
        assert np.isnan(s).all()
        assert E.last_error()[0] == E.EAKV_ERR_INVALID
        s = c.scores(np.ones(8 * 128, np.float32), 1, 8, 8)   # layer / heads out of range
        assert np.isnan(s).all()
        s = c.scores(np.ones(4 * 128, np.float32), 0, 4, 4)   # valid again
        assert np.isfinite(s).all() and E.last_error()[0] == E.EAKV_OK


def test_empty_cache(gpu):
    """seq_len 0: scores write nothing, the V-sum writes zeros (the
    reference stores its zero-initialised accumulators)."""
    with E.Cache(1, 2, 64, 16) as c:
        out = c.output(np.zeros(0, np.float32), 0, 2, 2)
        assert np.array_equal(out, np.zeros(2 * 64, np.float32))
        assert c.scores(np.ones(2 * 64, np.float32), 0, 2, 2).size == 0


def test_unsupported_head_dim_rejected(gpu):
    with E.Cache(1, 2, 256, 16) as c:
        assert c.load_raw(np.ones((1, 2, 2, 16, 256), np.float32), 16) == 0
        s = c.scores(np.ones(2 * 256, np.float32), 0, 2, 2)
        assert np.isnan(s).all() and E.last_error()[0] == E.EAKV_ERR_INVALID


@pytest.mark.parametrize("hd,S,maxS", [(128, 301, 320), (64, 511, 512), (128, 64, 64)])
def test_single_head_cache_against_single_head_kernels(gpu, hd, S, maxS):
    """Row a10: a one-head cache (n_q = n_kv = 1) through the library's
    two-call API and its fused decode, against the reference's single-head
    kernels restated in the oracle (kernels/fused_k_score.ea:9-153,
    fused_v_sum.ea:7-77 and the _64 forms): scores and V sum bit for bit
    (one chunk), the fused path within 1e-4."""
    rng = np.random.default_rng(hd + S)
    L = 2
    data = kv_data(rng, L, 1, S, hd)
    rc = O.RefCache(L, 1, hd, maxS)
    rc.load_raw(data, S)
    with E.Cache(L, 1, hd, maxS) as c:
        assert c.load_raw(data, S) == 0
        for l in range(L):
            q = rng.standard_normal(hd).astype(np.float32)
            s_ref = rc.scores_single(q, l, 0)
            assert np.array_equal(bits(c.scores(q, l, 1, 1)), bits(s_ref)), "scores"
            w = O.softmax_rows(s_ref, 1, S)
            assert np.array_equal(bits(c.output(w, l, 1, 1)), bits(rc.output_single(w, l, 0))), \
                "V sum"
            assert_close(c.fused(q, l, 1, 1), rc.fused(q, l, 1, 1), what=f"fused layer {l}")
