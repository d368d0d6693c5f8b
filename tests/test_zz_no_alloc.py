"""GPU: eakv_decode_attention_noalloc, the batched decode for callers that
cannot allocate device memory (a framework's caching allocator owns the GPU,
or a decode loop must not block on cudaMalloc/cudaFree). Its split-merge
workspace is a fixed 4 MiB array in the library instead of cache scratch.

Named so pytest collects it last: if it fails, a run that stops at the first
failure has already run every other test. Passes alone in a fresh process
and after the other tests (the shared array keeps the last call's contents,
and no result may depend on them).
"""
import numpy as np
import pytest

import eakv_b200 as E
from gpu_util import assert_close, kv_data

pytestmark = pytest.mark.gpu


def _caches(rng, B, L, nkv, hd, S):
    cs = []
    for _ in range(B):
        c = E.Cache(L, nkv, hd, S)
        assert c.load_raw(kv_data(rng, L, nkv, S, hd), S) == 0
        cs.append(c)
    return cs


@pytest.mark.parametrize("nq,nkv,hd", [(8, 8, 128), (32, 4, 64), (32, 8, 128)])
def test_noalloc_matches_decode_twice(gpu, nq, nkv, hd):
    """Two calls in a row through the C ABI, each equal to the allocating
    entry point within the parity tolerance. Short batches of long rows
    make the planner split rows, so the fixed workspace is used."""
    import torch
    E.force_splits(0)
    rng = np.random.default_rng(nq + hd)
    B, L, S = 2, 2, 1500
    caches = _caches(rng, B, L, nkv, hd, S)
    for call in range(2):
        q = torch.from_numpy(rng.standard_normal((B, L, nq, hd)).astype(np.float32)).to(gpu)
        ref = torch.empty_like(q)
        got = torch.full_like(q, float("nan"))
        E.decode_attention(caches, q, nq, ref)
        rc = E.decode_attention_noalloc(caches, q, nq, got)
        assert rc == E.EAKV_OK, E.last_error()
        caches[0].synchronize()
        assert E.decode_launches(caches, nq) == 2, "expected a split (workspace) plan"
        assert_close(got.cpu().numpy(), ref.cpu().numpy(), what=f"call {call}")
    for c in caches:
        c.free()


def test_noalloc_rejects_oversize_workspace(gpu):
    """A plan whose workspace exceeds the fixed array is refused up front."""
    import torch
    rng = np.random.default_rng(1)
    L, nq, nkv, hd, S = 8, 32, 8, 128, 4096
    caches = _caches(rng, 1, L, nkv, hd, S)
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
