"""GPU, 2 and 4 ranks: the library's sequence-split decode over NCCL
(eakv_decode_attention_split, include/eakv_nccl.h), one process per GPU.

Every rank holds its page-aligned slice of the positions of every sequence
in its own caches; the library decodes the slice, all-gathers the (output,
LSE) records over its own NCCL communicator and merges them. Each rank's
result is checked against the oracle's two-pass attention over the whole
sequence (1e-4 abs + 1e-4 rel), and all ranks must hold the same bits. With
4 GPUs the KV heads are also split in two head shards, each a sequence-split
group of 2. Skipped when fewer GPUs than ranks are visible. torch.distributed
(gloo) only carries the NCCL id; NVLS is off in the children."""
import os
import socket

import numpy as np
import pytest

from conftest import HAS_GPU

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, hs, lens, L, result_q):
    import datetime
    import torch
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    dec = None
    caches = []
    try:
        import eakv_b200 as E
        from eakv_b200.parallel import SeqSplitDecoder, seq_shard
        from gpu_util import assert_close, kv_data
        from oracle import oracle as O
        torch.cuda.set_device(rank)
        E.set_device(rank)
        dev = torch.device("cuda", rank)
        nq, nkv, hd = 16, 4, 128
        ss = world // hs
        h_i, s_i = rank // ss, rank % ss
        groups = [dist.new_group(ranks=[h * ss + k for k in range(ss)]) for h in range(hs)]
        rng = np.random.default_rng(11)              # the same data on every rank
        datas = [kv_data(rng, L, nkv, n, hd) for n in lens]
        q = rng.standard_normal((len(lens), L, nq, hd)).astype(np.float32)
        kh, qh = nkv // hs, nq // hs
        cuts = [seq_shard(n, ss, s_i) for n in lens]
        cap = max(1, max(hi - lo for lo, hi in cuts))   # one cache shape per batch
        for b, (lo, hi) in enumerate(cuts):
            c = E.Cache(L, kh, hd, cap)
            if hi > lo:
                mine = np.ascontiguousarray(datas[b][:, :, h_i * kh:(h_i + 1) * kh, lo:hi])
                assert c.load_raw(mine, hi - lo) == 0
            caches.append(c)
        dec = SeqSplitDecoder(caches, qh, hd, group=groups[h_i], device=rank)
        dq = torch.from_numpy(np.ascontiguousarray(q[:, :, h_i * qh:(h_i + 1) * qh])).to(dev)
        stream = torch.cuda.Stream(dev)
        outs = []
        for _ in range(2):                           # two steps in a row
            do = torch.full_like(dq, float("nan"))
            # every rank is ready before any enters the NCCL collective: a rank
            # that failed earlier ends this host barrier with an error instead
            # of leaving its peers waiting in the collective on the GPU
            dist.barrier()
            dec.step(dq, do, stream=stream)
            stream.synchronize()
            outs.append(do.cpu().numpy())
        assert np.array_equal(outs[0].view(np.uint32), outs[1].view(np.uint32))
        # the host-buffer form (chunked from 256 KiB of queries on) gives the same bits
        hq = np.ascontiguousarray(q[:, :, h_i * qh:(h_i + 1) * qh])
        ho = np.full_like(hq, np.nan)
        dist.barrier()
        dec.step_host(hq, ho, stream=stream)
        assert np.array_equal(ho.view(np.uint32), outs[0].view(np.uint32)), "host form differs"
        for b, n in enumerate(lens):
            rc = O.RefCache(L, nkv, hd, n)
            rc.load_raw(datas[b], n)
            for l in range(L):
                full = rc.fused(q[b, l], l, nq, nkv).reshape(nq, hd)
                assert_close(outs[0][b, l], full[h_i * qh:(h_i + 1) * qh],
                             what=f"rank {rank} sequence {b} layer {l}")
        assert E.device_status(rank) == 0
        result_q.put((rank, "ok", outs[0].tobytes()))
    except Exception as e:                           # noqa: BLE001 - reported to the parent
        result_q.put((rank, f"{type(e).__name__}: {e}", b""))
    finally:
        if dec is not None:
            dec.close()
        for c in caches:
            c.free()
        dist.destroy_process_group()


def _run(world, hs, lens, L=2):
    import torch
    import torch.multiprocessing as mp
    if not HAS_GPU or torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, hs, lens, L, q))
             for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    for _ in procs:
        r, msg, out = q.get(timeout=600)
        results[r] = (msg, out)
    for p in procs:
        p.join(timeout=120)
    for r, (msg, _) in sorted(results.items()):
        assert msg == "ok", f"rank {r}: {msg}"
    ss = world // hs
    for r in range(world):   # the ranks of a group hold the same bits
        assert results[r][1] == results[(r // ss) * ss][1], f"rank {r} differs from its group"


@pytest.mark.parametrize("lens,L", [([1000, 333], 2), ([50, 2048], 2), ([300] * 6, 22)])
def test_sequence_split_two_gpus(lens, L):
    """[50, 2048]: the second rank's slice of the first sequence is empty.
    Six caches of 22 layers: 1.1 MB of queries, so the host-buffer form runs
    in chunks, one all-gather each."""
    _run(2, 1, lens, L)


def test_head_shards_times_sequence_split_four_gpus():
    _run(4, 2, [1500, 700])


def _worker_lost(rank, world, port, result_q):
    """Rank 1 leaves after one good step (no destroy, no further collective).
    Rank 0 learns it at the host barrier before its next step (gloo, 10 s),
    never enters the collective, and ends its communicator with
    eakv_nccl_comm_abort."""
    import datetime
    import torch
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=10))
    import eakv_b200 as E
    from eakv_b200.parallel import SeqSplitDecoder
    from gpu_util import kv_data
    torch.cuda.set_device(rank)
    E.set_device(rank)
    rng = np.random.default_rng(3)
    L, nq, nkv, hd, S = 1, 8, 2, 128, 256
    c = E.Cache(L, nkv, hd, S)
    assert c.load_raw(kv_data(rng, L, nkv, S, hd), S) == 0
    dec = SeqSplitDecoder([c], nq, hd, device=rank)
    dq = torch.from_numpy(rng.standard_normal((1, L, nq, hd)).astype(np.float32)).to(rank)
    do = torch.empty_like(dq)
    stream = torch.cuda.Stream(rank)
    dist.barrier()
    dec.step(dq, do, stream=stream)               # one good step
    stream.synchronize()
    if rank == 1:
        result_q.put((rank, "left"))
        result_q.close()
        result_q.join_thread()
        os._exit(0)                                # gone between steps
    try:
        dist.barrier()                             # the host learns of it here
        result_q.put((rank, "no error"))
    except Exception as e:                         # noqa: BLE001 - any error ends the wait
        dec.comm.abort()                           # no collective of it is in flight
        result_q.put((rank, f"raised {type(e).__name__}, aborted"))
    c.free()


def test_lost_rank_between_steps_two_gpus():
    import torch
    import torch.multiprocessing as mp
    if not HAS_GPU or torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker_lost, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert results[1] == "left"
    assert results[0].startswith("raised") and results[0].endswith("aborted"), results[0]


def test_c_host_split_two_gpus(tmp_path):
    """The library's multi-GPU split from a plain C host (tests/c/split_c_host.c):
    no Python in the ranks, the NCCL id passed through a file, host buffers
    only; each rank checks the merged result against a single-GPU decode of
    the whole sequences within 1e-4."""
    import shutil
    import subprocess
    import sys
    import torch
    if not HAS_GPU or torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    cc = shutil.which("gcc") or shutil.which("cc")
    if not cc:
        pytest.skip("no C compiler")
    import eakv_b200 as E
    from conftest import ROOT
    libdir = os.path.dirname(E.LIB_PATH)
    exe = str(tmp_path / "split_c_host")
    subprocess.run([cc, "-O2", "-Wall", "-I", os.path.join(ROOT, "include"),
                    os.path.join(ROOT, "tests", "c", "split_c_host.c"), "-L", libdir,
                    "-leakv_b200", f"-Wl,-rpath,{libdir}", "-lm", "-o", exe], check=True)
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    idf = str(tmp_path / "nccl.id")
    procs = [subprocess.Popen([exe, str(r), "2", idf], stdout=subprocess.PIPE,
                              stderr=subprocess.PIPE, text=True, env=env) for r in range(2)]
    outs = []
    for p in procs:
        try:
            o, e = p.communicate(timeout=300)
        except subprocess.TimeoutExpired:
            for pp in procs:
                pp.kill()
            raise
        outs.append((p.returncode, o, e))
    for r, (rc, o, e) in enumerate(outs):
        sys.stderr.write(e)
        # NCCL may print its version banner on stdout first
        last = o.strip().splitlines()[-1] if o.strip() else ""
        assert rc == 0 and last.startswith("ok"), f"rank {r}: rc {rc} {o!r} {e!r}"
