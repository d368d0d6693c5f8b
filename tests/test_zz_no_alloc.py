"""GPU: eakv_decode_attention_noalloc, the batched decode for callers that
cannot allocate device memory (a framework's caching allocator owns the GPU,
or a decode loop must not block on cudaMalloc/cudaFree). Its split workspace
(records and counters) lives in fixed arrays in the library instead of in
cache scratch.

Named so pytest collects it last: if it fails, a run that stops at the first
failure has already run every other test. Passes alone in a fresh process
and after the other tests (the shared arrays keep the last call's records,
and no result may depend on them).
"""
import numpy as np
import pytest

import eakv_b200 as E
from gpu_util import assert_close, bits, kv_data
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def _caches(rng, B, L, nkv, hd, S, gpu):
    """Caches filled from device buffers, so none of them has scratch yet:
    any device allocation by a later call would show in device_bytes."""
    import torch
    cs, datas = [], []
    for _ in range(B):
        c = E.Cache(L, nkv, hd, S)
        data = kv_data(rng, L, nkv, S, hd)
        d = torch.from_numpy(data).to(gpu)
        assert c.load_raw_device(d, S) == 0
        c.synchronize()
        cs.append(c)
        datas.append(data)
    return cs, datas


@pytest.mark.parametrize("nq,nkv,hd", [(8, 8, 128), (32, 4, 64), (32, 8, 128)])
def test_noalloc_matches_decode_twice(gpu, nq, nkv, hd):
    """Two calls in a row through the C ABI, on caches that no allocating call
    has touched: each equals the allocating entry point bit for bit (same
    kernels, same split plan) and, on the first call, the oracle within the
    1e-4 parity bar. Short batches of long rows make the planner split rows,
    so the fixed arrays are used."""
    import torch
    E.force_splits(0)
    rng = np.random.default_rng(nq + hd)
    B, L, S = 2, 2, 1500
    caches, datas = _caches(rng, B, L, nkv, hd, S, gpu)
    assert E.decode_splits(caches, nq) > 1, "expected a split plan (the workspace in use)"
    held = [c.device_bytes for c in caches]
    qs, gots = [], []
    for call in range(2):
        q = torch.from_numpy(rng.standard_normal((B, L, nq, hd)).astype(np.float32)).to(gpu)
        got = torch.full_like(q, float("nan"))
        rc = E.decode_attention_noalloc(caches, q, nq, got)
        assert rc == E.EAKV_OK, E.last_error()
        torch.cuda.synchronize()
        # nothing grew: the caches' scratch is still unallocated
        assert [c.device_bytes for c in caches] == held, f"call {call}"
        qs.append(q)
        gots.append(got.cpu().numpy())
    ref = O.RefCache(L, nkv, hd, S)
    ref.load_raw(datas[0], S)
    qn = qs[0].cpu().numpy()
    for l in range(L):
        assert_close(gots[0][0, l].reshape(-1), ref.fused(qn[0, l], l, nq, nkv),
                     what=f"oracle, layer {l}")
    # the allocating entry point, after both calls: the same bits
    for call, (q, got_n) in enumerate(zip(qs, gots)):
        want = torch.empty_like(q)
        E.decode_attention(caches, q, nq, want)
        caches[0].synchronize()
        assert np.array_equal(bits(got_n), bits(want.cpu().numpy())), f"call {call}"
    assert E.device_status(0) == 0
    for c in caches:
        c.free()


def test_noalloc_leaves_device_memory_alone(gpu):
    """After the first call on the device (which may load the library's
    module), further calls change neither the free device memory nor the
    caches' holdings."""
    import torch
    rng = np.random.default_rng(5)
    L, nq, nkv, hd, S = 2, 32, 8, 128, 3000
    caches, _ = _caches(rng, 2, L, nkv, hd, S, gpu)
    assert E.decode_splits(caches, nq) > 1
    q = torch.from_numpy(rng.standard_normal((2, L, nq, hd)).astype(np.float32)).to(gpu)
    out = torch.empty_like(q)
    assert E.decode_attention_noalloc(caches, q, nq, out) == E.EAKV_OK, E.last_error()
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    held = [c.device_bytes for c in caches]
    for _ in range(3):
        assert E.decode_attention_noalloc(caches, q, nq, out) == E.EAKV_OK, E.last_error()
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    assert free1 >= free0, (free0, free1)
    assert [c.device_bytes for c in caches] == held
    for c in caches:
        c.free()


def test_noalloc_rejects_oversize_workspace(gpu):
    """A plan whose split records exceed the fixed array is refused up front."""
    import torch
    rng = np.random.default_rng(1)
    L, nq, nkv, hd, S = 8, 32, 8, 128, 4096
    caches, _ = _caches(rng, 1, L, nkv, hd, S, gpu)
    q = torch.zeros((1, L, nq, hd), device=gpu)
    out = torch.zeros_like(q)
    E.force_splits(64)      # 256 rows x 64 splits x 130 floats > 4 MiB
    try:
        rc = E.decode_attention_noalloc(caches, q, nq, out)
        assert rc == E.EAKV_ERR_INVALID
        assert "exceeds" in E.last_error()[1]
    finally:
        E.force_splits(0)
    for c in caches:
        c.free()
