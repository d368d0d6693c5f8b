"""Failure detection on the GPU without a fault: every pipeline wait of the
decode kernels is bounded. A test hook stops one page of every work item
from ever being requested, so the wait for it runs out (nothing else ever
completes that barrier). The kernel must record the timeout in the device
status word, wait for the copies it did request, and return; the context
stays usable and the next call is correct again."""
import numpy as np
import pytest

import eakv_b200 as E
from gpu_util import PATH_CODE, assert_close, kv_data
from oracle import oracle as O

pytestmark = pytest.mark.gpu

STATUS_WAIT_TIMEOUT = 1
BUDGET = 4096   # polls per wait: a few milliseconds


@pytest.fixture(autouse=True)
def _reset_hooks():
    E.test_stall(-1, 0)
    E.force_splits(0)
    E.force_path(0)
    yield
    E.test_stall(-1, 0)
    E.force_splits(0)
    E.force_path(0)


@pytest.mark.parametrize("path", ["auto", "simt", "mma", "umma"])
@pytest.mark.parametrize("splits,page", [(0, 0), (1, 5), (3, 1)])
def test_wait_timeout_sets_status(gpu, path, splits, page):
    E.force_path(PATH_CODE[path])
    E.force_splits(splits)
    L, nq, nkv, hd, S = 1, 16, 4, 128, 1000     # 16 pages per head
    rng = np.random.default_rng(7 + page)
    data = kv_data(rng, L, nkv, S, hd)
    rc = O.RefCache(L, nkv, hd, S)
    rc.load_raw(data, S)
    q = rng.standard_normal(nq * hd).astype(np.float32)
    with E.Cache(L, nkv, hd, S) as c:
        assert c.load_raw(data, S) == 0
        E.device_status(0, reset=True)
        assert E.device_status(0) == 0

        E.test_stall(page, BUDGET)
        c.fused(q, 0, nq, nkv)          # the launch itself succeeds
        st = E.device_status(0, reset=True)
        assert st & STATUS_WAIT_TIMEOUT, f"status {st}"
        assert E.device_status(0) == 0  # reset took

        # same context, hooks off: correct results and a clean status
        E.test_stall(-1, 0)
        assert_close(c.fused(q, 0, nq, nkv), rc.fused(q, 0, nq, nkv), what="after timeout")
        assert E.device_status(0) == 0


def test_budget_alone_does_not_time_out(gpu):
    """A small budget by itself is enough for pages that do arrive."""
    L, nq, nkv, hd, S = 2, 32, 8, 128, 3000
    rng = np.random.default_rng(11)
    data = kv_data(rng, L, nkv, S, hd)
    rc = O.RefCache(L, nkv, hd, S)
    rc.load_raw(data, S)
    with E.Cache(L, nkv, hd, S) as c:
        assert c.load_raw(data, S) == 0
        E.device_status(0, reset=True)
        E.test_stall(-1, 1 << 16)
        for l in range(L):
            q = rng.standard_normal(nq * hd).astype(np.float32)
            assert_close(c.fused(q, l, nq, nkv), rc.fused(q, l, nq, nkv), what=f"layer {l}")
        assert E.device_status(0) == 0
