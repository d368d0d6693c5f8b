#!/usr/bin/env python
"""Benchmark of the eakv hot path on B200: Q4 decode attention.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config 4] [--impl b200|reference]

Metric: "Q4 decode-attention KV tokens/s per GPU; achieved
HBM GB/s vs B200 peak". One KV token is one cached position of one sequence
across all layers and KV heads, K and V read once: layers*kv_heads*2*
(head_dim/64)*40 bytes. A step is one fused decode-attention pass of every
sequence over every layer (softmax(QK^T/sqrt d)V on the Q4 cache).

Default workload (N=1): config 4 of BASELINE.json, the shape the north-star
target is quoted on - Llama-3-8B GQA 4:1, 32 layers, 32 Q / 8 KV heads,
head_dim 128, 32768 cached positions, 16 sequences (21.5 GB of Q4 cache,
far above the 126 MB L2, so no flush is needed). Under torchrun (N > 1) the
same 16 sequences are spread over the N GPUs (strong scaling): N/2 KV-head
shards, each split in two by sequence, so every step's NCCL all-gather of
the (output, LSE) records and their merge are inside the timed region;
--dp instead gives every rank its own 16 sequences (weak scaling, no
data-path collective). Rank 0 prints one JSON line with the whole-job
throughput and the max-over-ranks step time.

--impl reference times the reference's CPU implementation of the same step
(reference host C src/cache.c + src/attention.c, compiled from its sources,
with the C restatement of its Ea kernels) on the host's cores, one sequence
per thread, on a bounded sample of the workload.
"""
import argparse
import json
import os
import platform
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "Q4 decode-attention KV tokens/s per GPU; achieved HBM GB/s vs B200 peak"
UNIT = "KV tokens/s"
# decode kernel selection (eakv_test_force_path codes)
PATH_CODES = {"auto": 0, "simt": 1, "mma": 2, "umma": 3}

CONFIGS = {
    1: dict(workload="cfg1 README MHA 8/8 heads d128 S2048 B1", L=1, nq=8, nkv=8, hd=128,
            S=2048, B=1),
    2: dict(workload="cfg2 TinyLlama-1.1B GQA 8:1 d64 S2048 B1", L=22, nq=32, nkv=4, hd=64,
            S=2048, B=1),
    # each step first quantize-appends one new token of every layer and K/V
    # (restore to S-1, append, advance) and then attends all S positions
    3: dict(workload="cfg3 Llama-2-7B MHA d128 S8192 B1 + 1-token append per step", L=32,
            nq=32, nkv=32, hd=128, S=8192, B=1, append=True),
    # multi-GPU: KV-head shards x a two-way sequence split (strong scaling)
    4: dict(workload="cfg4 Llama-3-8B GQA 4:1 d128 S32768 B16", L=32, nq=32, nkv=8, hd=128,
            S=32768, B=16, shard=True, seq_shards=2),
    # multi-GPU: the KV heads (with their query heads) are sharded over the
    # GPUs; beyond one KV head per GPU (or with --seq-shards) every rank of a
    # head shard holds a page-aligned slice of every sequence, and the
    # partial (output, LSE) of those ranks are all-gathered over NCCL and merged
    5: dict(workload="cfg5 Llama-3-70B GQA 8:1 d128 S131072 B4 (KV-head shards x sequence "
            "split)", L=80, nq=64, nkv=8, hd=128, S=131072, B=4, shard=True),
}

FALLBACK_HBM_GBS = 6650.0


def bytes_per_token(c):
    return c["L"] * c["nkv"] * 2 * (c["hd"] // 64) * 40


def measured_peak():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def ncu_traffic(kernel_key):
    """DRAM bytes per algorithmic byte of a kernel, from the committed ncu
    summary (a capture whose traffic scales with the pages read)."""
    p = os.path.join(ROOT, "profiles", "traffic.json")
    try:
        with open(p) as f:
            return json.load(f).get(kernel_key)
    except Exception:
        return None


class ClockSampler:
    """nvidia-smi clocks/throttle sampling while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device):
        self.device = device
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100", "-i", str(self.device)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
            t0 = time.time()
            while not self.lines and time.time() - t0 < 5:
                time.sleep(0.02)
        except Exception:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def mark(self):
        return len(self.lines)

    def stop(self, since=0):
        if not self.proc:
            return None
        time.sleep(0.15)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        rows = [l.split(", ") for l in self.lines[since:] if l.count(",") >= 8]
        if not rows:
            rows = [l.split(", ") for l in self.lines if l.count(",") >= 8]
        if not rows:
            return None
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        pw = [float(r[3]) for r in rows if r[3].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].strip() == "Active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons,
                "power_w": statistics.median(pw) if pw else None, "samples": len(rows)}


# ---------------------------------------------------------------------------
# CPU reference (the reference's own host code + restated kernels)

def cpu_reference(cfg, threads, seconds, seed=0):
    """KV tokens/s of the reference's two-call path (scores, host softmax,
    V-sum) run by `threads` host threads, each on its own one-layer cache of
    the workload's shape. Returns (tokens_per_s, sample description, kind)."""
    from oracle import oracle as O
    hd, nq, nkv, S, L = cfg["hd"], cfg["nq"], cfg["nkv"], cfg["S"], cfg["L"]
    rng = np.random.default_rng(seed)
    data = rng.standard_normal((1, 2, nkv, S, hd)).astype(np.float32)
    data[0, 0] *= np.exp(rng.uniform(np.log(0.5), np.log(8.0), (nkv, 1, hd))).astype(np.float32)
    q = rng.standard_normal(nq * hd).astype(np.float32)
    use_ref = O.ref_available()
    caches = []
    if use_ref:
        R = O.rlib()
        for _ in range(threads):
            c = R.eakv_cache_create(1, nkv, hd, S)
            assert R.eakv_cache_load_raw(c, data.ctypes.data, S) == 0
            caches.append(c)

        def unit(c, scores, out):
            R.eakv_attention_scores(c, q.ctypes.data, 0, nq, nkv, scores.ctypes.data)
            w = softmax_f32(scores, nq, S)
            R.eakv_attention_output(c, w.ctypes.data, 0, nq, nkv, out.ctypes.data)
        kind = "reference"
    else:
        for _ in range(threads):
            rc = O.RefCache(1, nkv, hd, S)
            rc.load_raw(data, S)
            caches.append(rc)

        def unit(c, scores, out):
            s = c.scores(q, 0, nq, nkv)
            c.output(softmax_f32(s, nq, S), 0, nq, nkv)
        kind = "port"

    done = [0] * threads
    stop = threading.Event()

    def worker(i):
        scores = np.zeros(nq * S, np.float32)
        out = np.zeros(nq * hd, np.float32)
        while not stop.is_set():
            unit(caches[i], scores, out)
            done[i] += 1

    ths = [threading.Thread(target=worker, args=(i,)) for i in range(threads)]
    t0 = time.perf_counter()
    for t in ths:
        t.start()
    time.sleep(seconds)
    stop.set()
    for t in ths:
        t.join()
    dt = time.perf_counter() - t0
    units = sum(done)
    if use_ref:
        for c in caches:
            O.rlib().eakv_cache_free(c)
    # L layer-units of one sequence yield S KV tokens
    tps = units * S / L / dt
    sample = (f"{units} (sequence, layer) units of {nkv} KV heads x {S} positions "
              f"(scores + host softmax + V-sum, {threads} thread(s), {dt:.1f} s), "
              f"scaled by 1/{L} layers per KV token")
    return tps, sample, kind


def cpu_model():
    """The host CPU's model name (first /proc/cpuinfo entry), for the record."""
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return platform.processor() or "unknown"


def cpu_reference_pinned(cfg, seconds):
    """cpu_reference on one thread pinned to one core of this process's set
    (the affinity is restored afterwards)."""
    try:
        old = os.sched_getaffinity(0)
        os.sched_setaffinity(0, {min(old)})
    except (AttributeError, OSError):
        old = None
    try:
        return cpu_reference(cfg, 1, seconds)
    finally:
        if old is not None:
            os.sched_setaffinity(0, old)


def softmax_f32(scores, nq, S):
    s = scores.reshape(nq, S)
    m = np.maximum(s.max(axis=1, keepdims=True), np.float32(-1e6))
    e = np.exp(s - m)
    e /= e.sum(axis=1, keepdims=True)
    return np.ascontiguousarray(e.reshape(-1), np.float32)


def host_threads():
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


# ---------------------------------------------------------------------------

def dist_setup(n_gpus):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    return world, rank, local


def run_reference(args, cfg, world, rank):
    if rank != 0:
        return
    threads = host_threads()
    per_step = []
    # each step is a bounded sample (about args.cpu_seconds of CPU work on
    # every thread); the sample count is capped so the run stays short
    cpu_reference(cfg, threads, 1.0)   # warm-up
    for _ in range(max(1, min(args.steps, 3))):
        tps, sample, kind = cpu_reference(cfg, threads, args.cpu_seconds)
        per_step.append(tps)
    value = statistics.median(per_step)
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": cfg["B"] * cfg["S"] / value * 1e3,
        "higher_is_better": True, "scaling": "strong" if cfg.get("shard") else "weak",
        "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded N(0,1) K/V, per-channel log-uniform[0.5,8] K scale)",
        "config": config_json(cfg, world), "impl": "reference",
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": kind,
                         "cpu": cpu_model(),
                         "sample": sample},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def layout(cfg, world, seq_shards=0):
    """(head shards, sequence shards) of a sharded config on `world` ranks;
    seq_shards 0 takes the config's own choice."""
    if not cfg.get("shard") or world == 1:
        return 1, 1
    from eakv_b200.parallel import shard_layout
    ss = seq_shards or cfg.get("seq_shards", 0)
    if ss and world % ss:
        ss = 0
    return shard_layout(world, cfg["nkv"], ss)


def config_json(cfg, world, seq_shards=0):
    hs, ss = layout(cfg, world, seq_shards)
    sharded = bool(cfg.get("shard"))
    if sharded and world > 1:
        par = (f"kv-head shards x{hs}, sequence split x{ss}"
               + (" (NCCL all-gather of (output, LSE) records + exact merge, in the library)"
                  if ss > 1 else " (no data-path collective)"))
    elif sharded:
        par = "single GPU"
    else:
        par = f"dp{world} (independent sequences per GPU)"
    return {"workload": cfg["workload"], "layers": cfg["L"], "q_heads": cfg["nq"],
            "kv_heads": cfg["nkv"], "head_dim": cfg["hd"], "seq_len": cfg["S"],
            "sequences": cfg["B"], "global_batch": cfg["B"] * (1 if sharded else world),
            "parallelism": par,
            "bytes_per_kv_token": bytes_per_token(cfg),
            "l2": ("L2 flushed before every timed step (512 MB device write, outside the "
                   "timed events)" if needs_flush(cfg) else
                   "inputs larger than L2 (Q4 cache >> 126 MB), no flush")}


L2_BYTES = 126 << 20


def needs_flush(cfg):
    """Caches that fit a few times into L2 would be read from L2 on the next
    step; those configs flush it between timed steps."""
    return cfg["B"] * cfg["S"] * bytes_per_token(cfg) < 4 * L2_BYTES


def build_caches(E, torch, cfg, device, seed, S=None):
    """B caches filled with seeded synthetic K/V through the device append
    path: a pool of 4 K and 4 V slices [kv_heads][S][head_dim] is
    quantized into every (cache, layer) in rotation. S overrides the
    positions per cache (a rank's slice under the sequence split)."""
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    H, hd, L, B = cfg["nkv"], cfg["hd"], cfg["L"], cfg["B"]
    S = cfg["S"] if S is None else S
    P = 4
    kpool, vpool = [], []
    for _ in range(P):
        ch = torch.exp(torch.empty(H, 1, hd, device=device).uniform_(np.log(0.5), np.log(8.0),
                                                                     generator=g))
        kpool.append((torch.randn(H, S, hd, device=device, generator=g) * ch).contiguous())
        vpool.append(torch.randn(H, S, hd, device=device, generator=g).contiguous())
    torch.cuda.synchronize()
    caches = []
    for b in range(B):
        c = E.Cache(L, H, hd, S)
        for l in range(L):
            assert c.append_device(kpool[(b + l) % P], l, 0, S) == 0
            assert c.append_device(vpool[(b + 3 * l + 1) % P], l, 1, S) == 0
        c.synchronize()
        assert c.advance(S) == 0
        caches.append(c)
    del kpool, vpool
    torch.cuda.empty_cache()
    return caches


def run_b200(args, cfg, world, rank, local):
    import torch
    import eakv_b200 as E
    torch.cuda.set_device(local)
    E.set_device(local)
    E.force_path(PATH_CODES[args.path])
    if args.splits:
        E.force_splits(args.splits)
    if args.separate_merge:
        E.separate_merge(True)
    dev = torch.device("cuda", local)
    # this rank's share: its KV heads (with their query heads) and, under a
    # sequence split, its slice of every sequence
    hs, ss = layout(cfg, world, args.seq_shards)
    lcfg = dict(cfg, nkv=cfg["nkv"] // hs, nq=cfg["nq"] // hs)
    split = ss > 1
    sub = None
    if split:
        import torch.distributed as dist
        from eakv_b200.parallel import seq_shard
        # one process group per head shard (every rank creates every group);
        # it only carries the NCCL id of the library's communicator
        for h in range(hs):
            g_ = dist.new_group(ranks=[h * ss + k for k in range(ss)])
            if h == rank // ss:
                sub = g_
        lo, hi = seq_shard(cfg["S"], ss, rank % ss)
        caches = build_caches(E, torch, lcfg, dev, seed=1234 + rank, S=hi - lo)
    else:
        caches = build_caches(E, torch, lcfg, dev, seed=1234 + rank)
    B, L, nq, hd = lcfg["B"], lcfg["L"], lcfg["nq"], lcfg["hd"]
    # a stream of our own: the legacy default stream has handle 0, which the
    # library reads as "the cache's stream"; events must sit on the stream
    # the kernels run on
    stream = torch.cuda.Stream(dev)
    torch.cuda.set_stream(stream)
    sh = stream.cuda_stream
    # the ranks of one head shard attend with the same queries
    gq = torch.Generator(device=dev)
    gq.manual_seed(4321 + rank // ss)
    qs = [torch.randn(B, L, nq, hd, device=dev, generator=gq) for _ in range(4)]
    out = torch.empty(B, L, nq, hd, device=dev)
    launches_per_step = E.decode_launches(caches, nq)
    decoder = None
    if split:
        from eakv_b200.parallel import SeqSplitDecoder
        decoder = SeqSplitDecoder(caches, nq, hd, group=sub, device=local)
        # the library decodes two halves of the caches, each followed by its
        # merge kernel after the all-gather (one of each for a single cache)
        launches_per_step = 2 * (launches_per_step + 1) if len(caches) > 1 \
            else launches_per_step + 1

    appending = bool(cfg.get("append"))
    if appending:
        S_full = caches[0].seq_len
        new_kv = torch.randn(L, 2, lcfg["nkv"], 1, hd, device=dev)
        for c in caches:
            c.set_stream(sh)
        launches_per_step += 1   # the append of every layer and K/V (one launch)

    def step(q_in, o, mid=None):
        if appending:
            for c in caches:
                c.restore(S_full - 1)
                c.append_step_device(new_kv, 1)
                c.advance(1)
            if mid is not None:
                mid.record(stream)   # decode launch time = this event -> step end
        if split:
            decoder.step(q_in, o, stream=sh)
        else:
            E.decode_attention(caches, q_in, nq, o, stream=sh)

    def barrier():
        if world > 1:
            import torch.distributed as dist
            dist.barrier()

    def max_over_ranks(x):
        if world > 1:
            import torch.distributed as dist
            t = torch.tensor([x], device=dev, dtype=torch.float64)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            return float(t.item())
        return x

    for i in range(args.warmup):
        step(qs[i % 4], out)
    torch.cuda.synchronize()
    barrier()

    # Latency-bound steps (the small configs) replay CUDA graphs of the same
    # library calls: one graph of the per-step append (positions are the same
    # every step: each step restores the cache to S_full - 1 first) and one
    # decode graph per query buffer. The cache's host-side length is kept in
    # step with restore/advance outside the graphs.
    use_graph = (args.graph == "on" or (args.graph == "auto" and needs_flush(cfg))) and not split
    if use_graph:
        g_dec, g_app = [], None
        if appending:
            for c in caches:
                c.restore(S_full - 1)
            g_app = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g_app, stream=stream, capture_error_mode="thread_local"):
                for c in caches:
                    c.append_step_device(new_kv, 1)
            for c in caches:
                c.advance(1)
        for k in range(4):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=stream, capture_error_mode="thread_local"):
                E.decode_attention(caches, qs[k], nq, out, stream=sh)
            g_dec.append(g)

        def step(q_in, o, mid=None):   # noqa: F811 (graph replay of the step above)
            if appending:
                for c in caches:
                    c.restore(S_full - 1)
                g_app.replay()
                for c in caches:
                    c.advance(1)
                if mid is not None:
                    mid.record(stream)
            g_dec[next(k for k in range(4) if qs[k] is q_in)].replay()

        for i in range(args.warmup):
            step(qs[i % 4], out)
        torch.cuda.synchronize()
        barrier()
    clocks = ClockSampler(local)
    clocks.start()
    mark = clocks.mark()
    torch.cuda.synchronize()
    barrier()
    flush = torch.empty(512 << 20, dtype=torch.uint8, device=dev) if needs_flush(cfg) else None
    evs = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps + 1)]
    mids = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)] if appending \
        else [None] * args.steps
    if flush is None:
        evs[0].record(stream)
        for i in range(args.steps):
            step(qs[i % 4], out, mids[i])
            evs[i + 1].record(stream)
        begins = evs[:-1]
    else:
        # each step timed on its own, after an L2 flush outside its events
        begins = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
        for i in range(args.steps):
            flush.fill_(i & 0xFF)
            begins[i].record(stream)
            step(qs[i % 4], out, mids[i])
            evs[i + 1].record(stream)
    torch.cuda.synchronize()
    barrier()
    clk = clocks.stop(mark)
    steps_ms = [begins[i].elapsed_time(evs[i + 1]) for i in range(args.steps)]
    if appending:
        per = [mids[i].elapsed_time(evs[i + 1]) for i in range(args.steps)]
    else:
        per = steps_ms
    ms_step = max_over_ranks(sum(steps_ms) / args.steps)
    avg_launch_ms = max_over_ranks(sum(per) / len(per))
    status = E.device_status(local)

    # end to end: host (pinned) queries in, host output back, every step
    qh_t = torch.randn(B, L, nq, hd, pin_memory=True)
    oh_t = torch.empty(B, L, nq, hd, pin_memory=True)
    qh, oh = qh_t.numpy(), oh_t.numpy()
    qd = torch.empty(B, L, nq, hd, device=dev)

    if appending:
        kv_host = torch.randn(L, 2, lcfg["nkv"], 1, hd, pin_memory=True)

    def step_host():
        if appending:
            # the new token arrives from the host like the query does
            new_kv.copy_(kv_host, non_blocking=True)
            for c in caches:
                c.restore(S_full - 1)
                c.append_step_device(new_kv, 1)
                c.advance(1)
        if split:
            decoder.step_host(qh, oh, stream=sh)
        else:
            E.decode_attention_host(caches, qh, nq, oh, stream=sh)

    for _ in range(2):
        step_host()
    torch.cuda.synchronize()
    barrier()
    if flush is None:
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(args.steps):
            step_host()
        e1.record(stream)
        torch.cuda.synchronize()
        e2e_total = e0.elapsed_time(e1)
    else:
        e2e_total = 0.0
        for i in range(args.steps):
            flush.fill_(i & 0xFF)
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            step_host()
            e1.record(stream)
            torch.cuda.synchronize()
            e2e_total += e0.elapsed_time(e1)
    e2e_ms = max_over_ranks(e2e_total / args.steps)
    assert np.isfinite(oh).all()

    # whole job: every rank's sequences, or (sharded) each sequence once
    tokens_step = B * cfg["S"] * (1 if cfg.get("shard") else world)
    value = tokens_step / (ms_step / 1e3)
    bpt = bytes_per_token(lcfg)
    # one decode launch per rank covers all of the rank's positions
    alg_bytes_launch = B * (caches[0].seq_len) * bpt
    peak, peak_kind = measured_peak()
    achieved = alg_bytes_launch / (avg_launch_ms / 1e3) / 1e9
    G = nq // lcfg["nkv"]
    if args.path != "simt" and hd in (64, 128):
        gh = max(d for d in range(1, min(G, 8) + 1) if G % d == 0)   # query heads per CTA
        if args.path == "umma" and hd == 128:
            kname = f"decode_umma_kernel<{8 if gh > 4 else 4}>"
        else:
            kname = f"decode_mma_kernel<{hd},{8 if gh > 4 else 4}>"
    else:
        gc = 8 if G % 8 == 0 else 4 if G % 4 == 0 else 2 if G % 2 == 0 else 1
        kname = f"decode_simt_kernel<{hd},{gc}>"
    traffic_ratio = ncu_traffic(kname)
    result = None
    if rank == 0:
        cpu = None
        if world == 1 and not args.no_cpu:
            tps, sample, kind = cpu_reference_pinned(cfg, args.cpu_seconds)
            cpu = {"value": tps, "unit": UNIT, "cores": 1, "kind": kind, "sample": sample,
                   "cpu": cpu_model(), "pinned": True}
        result = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step,
            "higher_is_better": True, "scaling": "strong" if cfg.get("shard") else "weak",
            "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded torch.randn K/V on device, per-channel log-uniform[0.5,8] "
                    "K scale, 4-slice pool rotated over caches/layers)",
            "config": config_json(cfg, world, args.seq_shards),
            "step_launch": ("CUDA graph replay of the library calls" if use_graph
                            else "direct library calls"),
            "e2e": {"value": tokens_step / (e2e_ms / 1e3), "unit": UNIT,
                    "h2d_bytes_per_step": int(qh.nbytes) + (int(kv_host.numel()) * 4
                                                            if appending else 0),
                    "d2h_bytes_per_step": int(oh.nbytes),
                    "api": ("eakv_decode_attention_split_host" if split
                            else "eakv_decode_attention_host")},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "peak_source": f"{peak_kind} hbm_gbs",
                         "traffic": (traffic_ratio * alg_bytes_launch) if traffic_ratio
                         else None,
                         "kernel": kname,
                         "algorithmic_bytes_per_launch": alg_bytes_launch},
            "cpu_baseline": cpu,
            "gpu_launches": launches_per_step * args.steps,
            "clocks": clk,
            "device_status": status,
        }
        print(json.dumps(result), flush=True)
    if decoder is not None:
        torch.cuda.synchronize()
        barrier()
        decoder.close()
    for c in caches:
        c.free()
    return result


def run_ggml(args, world, rank, local):
    """The q4_1_eakv ggml block type (llama.cpp integration): from_float,
    to_float and vec_dot on device buffers, one JSON line each, with the
    reference's AVX-512 code (or its restatement) timed on one host thread
    on a bounded sample. HBM-bound; 1 GiB of f32 per pass (> L2)."""
    import ctypes
    import torch
    import eakv_b200 as E
    from oracle import oracle as O
    if rank != 0:
        return
    torch.cuda.set_device(local)
    E.set_device(local)
    dev = torch.device("cuda", local)
    stream = torch.cuda.Stream(dev)
    torch.cuda.set_stream(stream)
    sh = stream.cuda_stream
    nb = 1 << 22                                   # 4.2 M blocks: 1 GiB of f32, 168 MB of blocks
    k = nb * 64
    x = torch.randn(k, device=dev)
    blocks = torch.empty(nb * 40, dtype=torch.uint8, device=dev)
    out = torch.empty(k, device=dev)
    row = 128                                      # vec_dot: rows of one head_dim
    nrc = k // row
    y = torch.randn(k, device=dev)
    s = torch.empty(nrc, device=dev)
    ops = {
        "from_float": (lambda: E.ggml_quantize_row_device(x, blocks, k, sh), nb * (256 + 40)),
        "to_float": (lambda: E.ggml_dequantize_row_device(blocks, out, k, sh), nb * (40 + 256)),
        "vec_dot": (lambda: E.ggml_vec_dot_device(row, s, 4, blocks, row // 64 * 40, y, row * 4,
                                                   nrc, sh), nb * (40 + 256) + nrc * 4),
    }
    peak, peak_kind = measured_peak()
    have_ref = os.path.exists(O.GGML_AVX512_SO)
    H = ctypes.CDLL(O.GGML_AVX512_SO) if have_ref else None
    hx = np.random.default_rng(0).standard_normal(1 << 20).astype(np.float32)   # 16384 blocks
    hb = O.ggml_quantize(hx, H)
    hy = np.random.default_rng(1).standard_normal(hx.size).astype(np.float32)
    host = {
        "from_float": lambda: O.ggml_quantize(hx, H),
        "to_float": lambda: O.ggml_dequantize(hb, H),
        "vec_dot": lambda: O.ggml_vec_dot(hb.reshape(-1, 80), hy.reshape(-1, 128), H),
    }
    for name, (fn, nbytes) in ops.items():
        for _ in range(args.warmup):
            fn()
        torch.cuda.synchronize()
        evs = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps + 1)]
        evs[0].record(stream)
        for i in range(args.steps):
            fn()
            evs[i + 1].record(stream)
        torch.cuda.synchronize()
        ms = evs[0].elapsed_time(evs[-1]) / args.steps
        gbs = nbytes / (ms / 1e3) / 1e9
        t0, reps = time.time(), 0
        while time.time() - t0 < args.cpu_seconds / 3:
            host[name]()
            reps += 1
        cpu_gbs = reps * (hx.size // 64) * (nbytes / nb) / (time.time() - t0) / 1e9
        print(json.dumps({
            "metric": f"q4_1_eakv ggml {name} GB/s (HBM bytes moved)", "value": gbs,
            "unit": "GB/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic (torch.randn)",
            "config": {"workload": f"ggml {name}: {nb} blocks of 64 (1 GiB f32)"
                                   + (f", rows of {row}" if name == "vec_dot" else ""),
                       "l2": "inputs larger than L2, no flush"},
            "roofline": {"bound": "hbm", "achieved": gbs, "peak": peak, "unit": "GB/s",
                         "frac": gbs / peak, "peak_source": f"{peak_kind} hbm_gbs",
                         "traffic": None, "algorithmic_bytes_per_launch": nbytes},
            "cpu_baseline": {"value": cpu_gbs, "unit": "GB/s", "cores": 1,
                             "kind": "reference" if have_ref else "port",
                             "sample": f"{hx.size // 64} blocks, {reps} passes"},
            "gpu_launches": args.steps,
        }), flush=True)


def _line(name, value, unit, ms, args, workload, nbytes=None, cpu=None, launches=None):
    peak, peak_kind = measured_peak()
    roof = None
    if nbytes is not None:
        gbs = nbytes / (ms / 1e3) / 1e9
        roof = {"bound": "hbm", "achieved": gbs, "peak": peak, "unit": "GB/s",
                "frac": gbs / peak, "peak_source": f"{peak_kind} hbm_gbs", "traffic": None,
                "algorithmic_bytes_per_launch": nbytes}
    print(json.dumps({
        "metric": name, "value": value, "unit": unit, "n_gpus": 1, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded)",
        "config": {"workload": workload, "l2": "inputs larger than L2, no flush"},
        "roofline": roof, "cpu_baseline": cpu, "gpu_launches": launches,
    }), flush=True)


def _time(fn, args, stream):
    import torch
    for _ in range(args.warmup):
        fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        fn()
    e1.record(stream)
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / args.steps


TWOCALL_SHAPES = [
    # the reference benchmark's shapes (benchmarks/bench_libeakv.c:160-164: MHA,
    # 8 heads, head_dim 128), then one layer of a cfg4 sequence (GQA 4:1)
    ("reference bench 7B-like 1L 8H d128 S2048", 1, 8, 8, 128, 2048),
    ("reference bench 7B-like 1L 8H d128 S8192", 1, 8, 8, 128, 8192),
    ("reference bench 7B-like 32L 8H d128 S2048", 32, 8, 8, 128, 2048),
    ("cfg4 one layer of one sequence: 32 Q / 8 KV heads d128 S32768", 1, 32, 8, 128, 32768),
]


def run_twocall(args, world, rank, local):
    """The reference's own API calls on the device cache, each on the
    shapes the reference benchmark times (benchmarks/bench_libeakv.c:131-151,
    :186-191, :222-223) and on one cfg4 layer: the two-call attention
    (eakv_attention_scores / eakv_attention_output) on device buffers, timed
    with CUDA events after an L2 flush, with their HBM roofline; the same
    calls with host buffers (the reference's contract, PCIe and the host
    synchronization included, wall clock); load_raw from host f32; save and
    load of the .eakv file. The reference's host code with the restated
    kernels (oracle/_ref) runs the same calls on one host thread beside it.
    Weights for the V sum are the softmax of the scores."""
    import ctypes
    import tempfile
    import torch
    import eakv_b200 as E
    from oracle import oracle as O
    if rank != 0:
        return
    torch.cuda.set_device(local)
    E.set_device(local)
    dev = torch.device("cuda", local)
    stream = torch.cuda.Stream(dev)
    torch.cuda.set_stream(stream)
    flush = torch.empty(512 << 20, dtype=torch.uint8, device=dev)
    peak, peak_kind = measured_peak()
    R = O.rlib() if O.ref_available() else None
    rng = np.random.default_rng(0)

    def line(metric, value, unit, ms, workload, nbytes=None, cpu=None, launches=None):
        roof = None
        if nbytes is not None:
            gbs = nbytes / (ms / 1e3) / 1e9
            roof = {"bound": "hbm", "achieved": gbs, "peak": peak, "unit": "GB/s",
                    "frac": gbs / peak, "peak_source": f"{peak_kind} hbm_gbs", "traffic": None,
                    "algorithmic_bytes_per_launch": nbytes}
        print(json.dumps({
            "metric": metric, "value": value, "unit": unit, "n_gpus": 1, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded)",
            "config": {"workload": workload, "l2": "L2 flushed before every timed call"},
            "roofline": roof, "cpu_baseline": cpu, "gpu_launches": launches}), flush=True)

    def dev_time(fn):
        for _ in range(args.warmup):
            fn()
        ts = []
        for i in range(args.steps):
            flush.fill_(i & 0xFF)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            fn()
            e1.record(stream)
            ts.append((e0, e1))
        torch.cuda.synchronize()
        return sorted(a.elapsed_time(b) for a, b in ts)[len(ts) // 2]

    def wall(fn, reps):
        fn()
        t0 = time.perf_counter()
        for _ in range(reps):
            fn()
        return (time.perf_counter() - t0) / reps * 1e3

    shapes = TWOCALL_SHAPES if args.shape < 0 else [TWOCALL_SHAPES[args.shape]]
    for name, L, nq, nkv, hd, S in shapes:
        data = rng.standard_normal((L, 2, nkv, S, hd), dtype=np.float32)
        c = E.Cache(L, nkv, hd, S)
        c.set_stream(stream.cuda_stream)
        ms_load = wall(lambda: c.load_raw(data, S), max(2, min(args.steps, 5)))
        q = rng.standard_normal(nq * hd, dtype=np.float32)
        dq = torch.from_numpy(q).to(dev)
        dsc = torch.empty(nq * S, device=dev)
        dout = torch.empty(nq * hd, device=dev)
        q4 = nkv * S * (hd // 64) * 40                     # Q4 bytes of one (layer, K/V)
        ms_s = dev_time(lambda: c.scores_device(dq, 0, nq, nkv, dsc))
        w = torch.softmax(dsc.view(nq, S), dim=1).reshape(-1).contiguous()
        ms_o = dev_time(lambda: c.output_device(w, 0, nq, nkv, dout))
        torch.cuda.synchronize()
        wh = w.cpu().numpy()
        ms_sh = wall(lambda: c.scores(q, 0, nq, nkv), max(3, args.steps))
        ms_oh = wall(lambda: c.output(wh, 0, nq, nkv), max(3, args.steps))
        with tempfile.TemporaryDirectory() as td:
            path = os.path.join(td, "c.eakv")
            ms_save = wall(lambda: c.save(path), 3)
            fsize = os.path.getsize(path)
            ms_fload = wall(lambda: E.Cache.load(path).free(), 3)
            cpu = {}
            if R is not None and not args.no_cpu:
                rc_ = R.eakv_cache_create(L, nkv, hd, S)
                sc = np.zeros(nq * S, np.float32)
                out = np.zeros(nq * hd, np.float32)
                reps = max(1, min(20, int(2e8 // (nq * S * hd))))
                cpu["load_raw"] = wall(lambda: R.eakv_cache_load_raw(rc_, data.ctypes.data, S), 2)
                cpu["scores"] = wall(lambda: R.eakv_attention_scores(
                    rc_, q.ctypes.data, 0, nq, nkv, sc.ctypes.data), reps)
                cpu["output"] = wall(lambda: R.eakv_attention_output(
                    rc_, wh.ctypes.data, 0, nq, nkv, out.ctypes.data), reps)
                rpath = os.path.join(td, "r.eakv").encode()
                cpu["save"] = wall(lambda: R.eakv_cache_save(rc_, rpath), 2)

                def rload():
                    h = ctypes.c_void_p()
                    R.eakv_cache_load(rpath, ctypes.byref(h))
                    R.eakv_cache_free(h)
                cpu["load"] = wall(rload, 2)
                R.eakv_cache_free(rc_)

        def cb(op, value, unit):
            if op not in cpu:
                return None
            return {"value": value(cpu[op]), "unit": unit, "cores": 1, "kind": "reference",
                    "sample": f"the same call on the reference's host code, {op}"}

        sc_bytes = q4 + nq * S * 4 + nq * hd * 4
        out_bytes = q4 + nq * S * 4 + nq * hd * 4
        wl = f"{name} ({L} layer(s) cached, layer 0 attended)"
        line("attention_scores device: KV positions/s", nkv * S / (ms_s / 1e3), "KV head-positions/s",
             ms_s, wl, nbytes=sc_bytes, launches=1,
             cpu=cb("scores", lambda t: nkv * S / (t / 1e3), "KV head-positions/s"))
        line("attention_output device: KV positions/s", nkv * S / (ms_o / 1e3), "KV head-positions/s",
             ms_o, wl, nbytes=out_bytes, launches=None,
             cpu=cb("output", lambda t: nkv * S / (t / 1e3), "KV head-positions/s"))
        line("attention_scores host API (copies + sync, wall clock): KV positions/s",
             nkv * S / (ms_sh / 1e3), "KV head-positions/s", ms_sh, wl,
             cpu=cb("scores", lambda t: nkv * S / (t / 1e3), "KV head-positions/s"))
        line("attention_output host API (copies + sync, wall clock): KV positions/s",
             nkv * S / (ms_oh / 1e3), "KV head-positions/s", ms_oh, wl,
             cpu=cb("output", lambda t: nkv * S / (t / 1e3), "KV head-positions/s"))
        line("load_raw from host f32 (PCIe + quantize, wall clock) GB/s of f32", data.nbytes /
             (ms_load / 1e3) / 1e9, "GB/s", ms_load, wl,
             cpu=cb("load_raw", lambda t: data.nbytes / (t / 1e3) / 1e9, "GB/s"))
        line("save .eakv GB/s of file (wall clock)", fsize / (ms_save / 1e3) / 1e9, "GB/s",
             ms_save, wl, cpu=cb("save", lambda t: fsize / (t / 1e3) / 1e9, "GB/s"))
        line("load .eakv GB/s of file (wall clock)", fsize / (ms_fload / 1e3) / 1e9, "GB/s",
             ms_fload, wl, cpu=cb("load", lambda t: fsize / (t / 1e3) / 1e9, "GB/s"))
        c.free()


def run_inspect(args, world, rank, local):
    """Device validate and dequantize of a resident cache on one cfg4
    sequence (32 layers x 8 KV heads x 32768 positions, 1.34 GB of pages)."""
    import torch
    import eakv_b200 as E
    if rank != 0:
        return
    torch.cuda.set_device(local)
    E.set_device(local)
    dev = torch.device("cuda", local)
    cfg = dict(CONFIGS[4], B=1)
    (c,) = build_caches(E, torch, cfg, dev, seed=7)
    stream = torch.cuda.Stream(dev)
    torch.cuda.set_stream(stream)
    c.set_stream(stream.cuda_stream)
    L, H, hd, S = cfg["L"], cfg["nkv"], cfg["hd"], cfg["S"]
    groups = L * 2 * H * S * hd // 64
    ms = _time(lambda: c.validate(), args, stream)
    _line("device validate GB/s (scale/bias bytes read)", groups * 8 / (ms / 1e3) / 1e9, "GB/s", ms,
          args, f"validate: cfg4 sequence, {groups} groups, codes copied back each call",
          nbytes=groups * 8, launches=args.steps)
    out = torch.empty(H, S, hd, device=dev)
    ms = _time(lambda: c.dequantize_device(5, 1, 0, S, out, stream.cuda_stream), args, stream)
    nb = H * S * hd // 64 * 40 + H * S * hd * 4
    _line("dequantize GB/s (Q4 read + f32 written)", nb / (ms / 1e3) / 1e9, "GB/s", ms, args,
          f"dequantize one (layer, V) block: {H} heads x {S} positions x {hd}", nbytes=nb,
          launches=args.steps)
    c.free()


def run_llama(args, world, rank, local):
    """llama.cpp state import: host state buffer in,
    device cache out, PCIe inside the timed region (the API's own
    contract); the reference bridge on the host cores beside it."""
    import ctypes
    import torch
    import eakv_b200 as E
    from oracle import oracle as O
    if rank != 0:
        return
    torch.cuda.set_device(local)
    E.set_device(local)
    L, H, hd, cells = 32, 8, 128, 4096
    rng = np.random.default_rng(0)
    k = rng.standard_normal((L, cells, H * hd), dtype=np.float32).astype(np.float16)
    state = O.llama_state(k, k, 1)
    buf = np.frombuffer(state, np.uint8)
    for _ in range(max(1, args.warmup // 2)):
        E.Cache.from_llama_state(state, L, H, hd, cells).free()
    t0 = time.time()
    reps = max(1, min(args.steps, 5))
    for _ in range(reps):
        E.Cache.from_llama_state(state, L, H, hd, cells).free()
    ms = (time.time() - t0) / reps * 1e3
    cpu = None
    if os.path.exists(O.REF_LLAMA_SO):
        R = ctypes.CDLL(O.REF_LLAMA_SO)
        R.eakv_from_llama_state.argtypes = [ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int,
                                            ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                            ctypes.POINTER(ctypes.c_void_p)]
        R.eakv_cache_free.argtypes = [ctypes.c_void_p]
        t0, n = time.time(), 0
        while time.time() - t0 < args.cpu_seconds / 2 or n == 0:
            cc = ctypes.c_void_p()
            assert R.eakv_from_llama_state(buf.ctypes.data, buf.size, L, H, hd, cells,
                                           ctypes.byref(cc)) == 0
            R.eakv_cache_free(cc)
            n += 1
        cpu_s = (time.time() - t0) / n
        cpu = {"value": buf.size / cpu_s / 1e9, "unit": "GB/s of state", "cores": 1,
               "kind": "reference", "sample": f"{n} whole imports"}
    _line("llama.cpp state import GB/s of state (host buffer -> device cache, wall clock)",
          buf.size / (ms / 1e3) / 1e9, "GB/s of state", ms, args,
          f"llama state: {L} layers x {H} KV heads x {hd} x {cells} cells, f16, v_trans=1 "
          f"({buf.size / 1e9:.2f} GB)", cpu=cpu, launches=None)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--config", type=int, default=4, choices=sorted(CONFIGS))
    ap.add_argument("--op", default="decode",
                    choices=["decode", "twocall", "ggml", "inspect", "llama"],
                    help="time another part instead: the reference's two-call attention API "
                         "and its load_raw / save / load, the q4_1_eakv ggml type kernels, "
                         "device validate + dequantize, or the llama.cpp state import")
    ap.add_argument("--shape", type=int, default=-1,
                    help="--op twocall: only this entry of its shape list (0-3; 3 is one cfg4 layer)")
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--cpu-seconds", type=float, default=8.0)
    ap.add_argument("--batch", type=int, default=0,
                    help="override sequences per GPU (smaller cases for profiling)")
    ap.add_argument("--seq", type=int, default=0, help="override cached positions")
    ap.add_argument("--force-simt", action="store_true",
                    help="same as --path simt")
    ap.add_argument("--path", default="auto", choices=list(PATH_CODES),
                    help="decode kernel: automatic choice, the CUDA-core kernel, the mma.sync "
                         "tensor-core kernel or the tcgen05 kernel")
    ap.add_argument("--seq-shards", type=int, default=0,
                    help="sharded configs: ranks per sequence split (0: the config's "
                         "choice - cfg4 two, cfg5 as many KV-head shards as divide the "
                         "ranks and the rest split the sequence)")
    ap.add_argument("--dp", action="store_true",
                    help="cfg4 under torchrun: every rank decodes its own 16 sequences "
                         "(weak scaling, no data-path collective) instead of sharding them")
    ap.add_argument("--graph", default="auto", choices=["auto", "on", "off"],
                    help="replay the device step from CUDA graphs (auto: for the small, "
                         "launch-latency-bound configs that flush L2 between steps)")
    ap.add_argument("--separate-merge", action="store_true",
                    help="merge sequence splits in a second kernel after the decode instead of "
                         "in the decode kernel (for side-by-side measurement)")
    ap.add_argument("--splits", type=int, default=0,
                    help="force this many sequence splits per row (0: planner's choice)")
    args = ap.parse_args()
    if args.force_simt:
        args.path = "simt"
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    cfg = dict(CONFIGS[args.config])
    if args.dp:
        cfg["shard"] = False
    if args.batch:
        cfg["B"] = args.batch
        cfg["workload"] += f" (batch overridden to {args.batch})"
    if args.seq:
        cfg["S"] = args.seq
        cfg["workload"] += f" (seq_len overridden to {args.seq})"
    world, rank, local = dist_setup(args.gpus)
    try:
        if args.op == "twocall":
            run_twocall(args, world, rank, local)
        elif args.op == "ggml":
            run_ggml(args, world, rank, local)
        elif args.op == "inspect":
            run_inspect(args, world, rank, local)
        elif args.op == "llama":
            run_llama(args, world, rank, local)
        elif args.impl == "reference":
            run_reference(args, cfg, world, rank)
        else:
            run_b200(args, cfg, world, rank, local)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
