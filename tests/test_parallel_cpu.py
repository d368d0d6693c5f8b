"""CPU (gloo, world_size 2 and 3): the host-side logic of the sequence-split
decode - page-aligned sharding of positions across ranks, all-gather of the
per-rank (normalized output, natural-log LSE) and the exact merge - against
the single-process oracle. Each rank computes its partial with the oracle
restricted to its position range; no GPU is involved."""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

from eakv_b200.parallel import merge_partials_np, seq_shard


def test_seq_shard_partitions():
    for S in (1, 63, 64, 65, 1000, 32768, 131072):
        for world in (1, 2, 3, 4, 8):
            cuts = [seq_shard(S, world, r) for r in range(world)]
            assert cuts[0][0] == 0 and cuts[-1][1] == S
            for (b0, e0), (b1, e1) in zip(cuts, cuts[1:]):
                assert e0 == b1
            for b, e in cuts[:-1]:
                assert b % 64 == 0 and e % 64 == 0 or e == S
    with pytest.raises(ValueError):
        seq_shard(10, 2, 2)


def _partial_oracle(rc, q, layer, nq, nkv, lo, hi):
    """(normalized output, natural LSE) over positions [lo, hi) with the
    oracle: LSE from the oracle's own scores, output from its fused kernel."""
    from oracle import oracle as O
    if hi <= lo:
        return np.full(nq * rc.hd, np.nan, np.float32), np.full(nq, -np.inf, np.float32)
    out = rc.fused(q, layer, nq, nkv, seq_range=(lo, hi))
    s = rc.scores(q, layer, nq, nkv).reshape(nq, rc.seq_len)[:, lo:hi].astype(np.float64)
    m = s.max(axis=1)
    lse = m + np.log(np.exp(s - m[:, None]).sum(axis=1))
    return out, lse.astype(np.float32)


def _worker(rank, world, port, S, result_q):
    import torch
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from oracle import oracle as O
        rng = np.random.default_rng(0)              # same data on every rank
        L, nq, nkv, hd = 2, 8, 2, 64
        data = rng.standard_normal((L, 2, nkv, S, hd)).astype(np.float32)
        q = rng.standard_normal((L, nq, hd)).astype(np.float32)
        rc = O.RefCache(L, nkv, hd, S)
        rc.load_raw(data, S)
        lo, hi = seq_shard(S, world, rank)
        outs, lses = [], []
        for l in range(L):
            o, s = _partial_oracle(rc, q[l], l, nq, nkv, lo, hi)
            outs.append(o.reshape(nq, hd))
            lses.append(s)
        part = torch.from_numpy(np.concatenate(outs))            # [L*nq][hd]
        lse = torch.from_numpy(np.concatenate(lses))             # [L*nq]
        parts = [torch.empty_like(part) for _ in range(world)]
        lsel = [torch.empty_like(lse) for _ in range(world)]
        dist.all_gather(parts, part)
        dist.all_gather(lsel, lse)
        merged, _ = merge_partials_np(np.stack([p.numpy() for p in parts]),
                                      np.stack([x.numpy() for x in lsel]))
        full = np.concatenate([rc.fused(q[l], l, nq, nkv).reshape(nq, hd) for l in range(L)])
        err = np.abs(merged - full)
        ok = bool(np.all(err <= 1e-4 + 1e-4 * np.abs(full)))
        result_q.put((rank, ok, float(err.max())))
    finally:
        dist.destroy_process_group()


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


@pytest.mark.parametrize("world,S", [(2, 1000), (3, 200), (2, 70)])
def test_sequence_split_gloo(world, S):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, S, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, ok, err in results:
        assert ok, f"rank {rank}: max err {err}"


def test_merge_handles_empty_parts():
    outs = np.zeros((3, 2, 4), np.float32)
    outs[0] = 1.0
    outs[2] = 3.0
    lses = np.array([[0.0, 1.0], [-np.inf, -np.inf], [0.0, -np.inf]], np.float32)
    out, lse = merge_partials_np(outs, lses)
    np.testing.assert_allclose(out[0], 2.0, rtol=1e-6)        # equal weights of 1 and 3
    np.testing.assert_allclose(out[1], 1.0, rtol=1e-6)        # only part 0 counts
    np.testing.assert_allclose(lse, [np.log(2.0), 1.0], rtol=1e-6)


def test_shard_layout():
    from eakv_b200.parallel import shard_layout
    assert shard_layout(1, 8) == (1, 1)
    assert shard_layout(2, 8) == (2, 1)
    assert shard_layout(8, 8) == (8, 1)
    assert shard_layout(16, 8) == (8, 2)      # beyond one KV head per rank: split sequences
    assert shard_layout(6, 4) == (2, 3)
    assert shard_layout(4, 8, seq_shards=2) == (2, 2)
    assert shard_layout(8, 8, seq_shards=8) == (1, 8)
    with pytest.raises(ValueError):
        shard_layout(4, 8, seq_shards=3)
    with pytest.raises(ValueError):
        shard_layout(8, 2, seq_shards=2)      # 4 head shards of 2 KV heads


def _worker_2d(rank, world, port, seq_shards, S, result_q):
    """KV-head shards x sequence split: each rank holds the KV heads of its
    head shard (with their query heads) over its slice of the positions;
    ranks of one head shard all-gather and merge over their own group."""
    import torch
    import torch.distributed as dist
    from eakv_b200.parallel import shard_layout
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from oracle import oracle as O
        L, nq, nkv, hd = 1, 8, 4, 64
        hs, ss = shard_layout(world, nkv, seq_shards)
        h_i, s_i = rank // ss, rank % ss
        groups = [dist.new_group(ranks=[h * ss + k for k in range(ss)]) for h in range(hs)]
        rng = np.random.default_rng(1)
        data = rng.standard_normal((L, 2, nkv, S, hd)).astype(np.float32)
        q = rng.standard_normal((L, nq, hd)).astype(np.float32)
        kh, qh = nkv // hs, nq // hs
        mine = np.ascontiguousarray(data[:, :, h_i * kh:(h_i + 1) * kh])
        qm = np.ascontiguousarray(q[:, h_i * qh:(h_i + 1) * qh])
        rc = O.RefCache(L, kh, hd, S)
        rc.load_raw(mine, S)
        lo, hi = seq_shard(S, ss, s_i)
        o, s = _partial_oracle(rc, qm[0], 0, qh, kh, lo, hi)
        part = torch.from_numpy(o.reshape(qh, hd))
        lse = torch.from_numpy(s)
        parts = [torch.empty_like(part) for _ in range(ss)]
        lsel = [torch.empty_like(lse) for _ in range(ss)]
        dist.all_gather(parts, part, group=groups[h_i])
        dist.all_gather(lsel, lse, group=groups[h_i])
        merged, _ = merge_partials_np(np.stack([p.numpy() for p in parts]),
                                      np.stack([x.numpy() for x in lsel]))
        full_rc = O.RefCache(L, nkv, hd, S)
        full_rc.load_raw(data, S)
        full = full_rc.fused(q[0], 0, nq, nkv).reshape(nq, hd)[h_i * qh:(h_i + 1) * qh]
        err = np.abs(merged - full)
        ok = bool(np.all(err <= 1e-4 + 1e-4 * np.abs(full)))
        result_q.put((rank, ok, float(err.max())))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,seq_shards,S", [(4, 2, 300), (2, 1, 130)])
def test_head_shards_times_sequence_split_gloo(world, seq_shards, S):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker_2d, args=(r, world, port, seq_shards, S, q))
             for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, ok, err in results:
        assert ok, f"rank {rank}: max err {err}"


def _worker_lost(rank, world, port, result_q):
    """Rank 1 leaves between steps (after one merged step); rank 0's next
    gather must end with an error, not hang."""
    import datetime
    import torch
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=10))
    part = torch.full((4, 8), float(rank))
    parts = [torch.empty_like(part) for _ in range(world)]
    dist.all_gather(parts, part)                   # one good step
    if rank == 1:
        result_q.put((rank, "left"))
        result_q.close()
        result_q.join_thread()                     # the message is out before the exit
        os._exit(0)                                # no further collective, no clean shutdown
    try:
        dist.all_gather(parts, part)
        result_q.put((rank, "no error"))
    except Exception as e:                         # noqa: BLE001 - any error ends the wait
        result_q.put((rank, f"raised {type(e).__name__}"))


def test_lost_rank_ends_the_next_gather_with_an_error():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker_lost, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert results[1] == "left"
    assert results[0].startswith("raised"), results[0]
