"""Multi-GPU plumbing for the decode path: one process per GPU.

Two ways to spread the work:

* Independent sequences (the default): each rank owns whole sequences and
  decodes them with `eakv_decode_attention`; no data-path collective.
* Sequence split, for a context larger than one GPU's share: rank r holds
  positions [begin_r, end_r) of every sequence in its own local caches,
  computes that range's normalized output and natural-log LSE with
  `eakv_decode_attention_partial`, the ranks all-gather (output, LSE), and
  `eakv_lse_combine` merges them exactly:

      out = sum_r exp(lse_r - L) out_r,   L = log sum_r exp(lse_r).

Softmax attention over a set of positions does not depend on their order,
so a rank's slice can sit at local positions 0.. of its caches.

torch.distributed is the plumbing (NCCL on GPUs, gloo on CPU for the
tests); the kernels are the library's.
"""
import math

import numpy as np

from . import decode_attention_partial, lse_combine

PAGE = 64


def seq_shard(seq_len, world, rank, align=PAGE):
    """[begin, end) of positions rank `rank` of `world` holds: contiguous,
    page-aligned cuts of [0, seq_len) in rank order (the last rank takes the
    remainder). Empty ranges are allowed for tiny sequences."""
    if world <= 0 or not (0 <= rank < world):
        raise ValueError("bad world/rank")
    per = -(-seq_len // world)                 # ceil
    per = -(-per // align) * align             # page-aligned share
    begin = min(seq_len, rank * per)
    end = min(seq_len, begin + per) if rank < world - 1 else seq_len
    return begin, max(begin, end)


def shard_layout(world, n_kv_heads, seq_shards=0):
    """(head_shards, seq_shards) with head_shards * seq_shards == world.

    KV heads are independent (each GPU decodes its heads for every
    sequence, no exchange), so by default as many head shards as divide
    both `world` and `n_kv_heads` are used and the remaining factor splits
    the sequence. `seq_shards` > 0 fixes the split instead; it must divide
    `world`, and `world // seq_shards` must divide `n_kv_heads`.
    Rank r belongs to head shard r // seq_shards and sequence slice
    r % seq_shards."""
    if world <= 0 or n_kv_heads <= 0:
        raise ValueError("bad world/heads")
    if seq_shards <= 0:
        hs = math.gcd(world, n_kv_heads)
        return hs, world // hs
    if world % seq_shards or n_kv_heads % (world // seq_shards):
        raise ValueError(f"{seq_shards} sequence shards do not fit {world} ranks and "
                         f"{n_kv_heads} KV heads")
    return world // seq_shards, seq_shards


def merge_partials_np(outs, lses):
    """Reference merge on the host: outs [P][rows][d], lses [P][rows] ->
    (out [rows][d], lse [rows]). Used by the CPU tests of the split logic."""
    outs = np.asarray(outs, np.float64)
    lses = np.asarray(lses, np.float64)
    M = np.max(lses, axis=0)
    finite = np.isfinite(M)
    Ms = np.where(finite, M, 0.0)
    w = np.where(np.isfinite(lses), np.exp(lses - Ms[None]), 0.0)      # [P][rows]
    L = w.sum(axis=0)
    # an empty part carries lse = -inf (weight 0) and a NaN output: skip it
    outs = np.where((w > 0)[:, :, None], outs, 0.0)
    out = np.einsum("pr,prd->rd", w, outs) / np.where(L > 0, L, np.nan)[:, None]
    lse = np.where(L > 0, Ms + np.log(np.where(L > 0, L, 1.0)), -np.inf)
    return out.astype(np.float32), lse.astype(np.float32)


class SeqSplitDecoder:
    """Sequence-split decode over a torch.distributed process group.

    caches: this rank's local caches (its slice of every sequence).
    Every rank calls `step` with the same queries; every rank receives the
    merged output. Collectives are issued in the same order on all ranks.
    """

    def __init__(self, caches, n_q_heads, head_dim, group=None):
        import torch
        import torch.distributed as dist
        self.dist = dist
        self.torch = torch
        self.caches = caches
        self.n_q = n_q_heads
        self.hd = head_dim
        self.group = group
        self.world = dist.get_world_size(group)
        self.rows = len(caches) * caches[0].n_layers * n_q_heads

    def step(self, d_q, d_out, stream=None):
        """One decode step. `stream` is a torch.cuda.Stream (a private one is
        made if None): the partial kernel, the all-gathers and the merge are
        all ordered on it, so nothing here synchronizes the host."""
        torch, dist = self.torch, self.dist
        dev = d_q.device
        if stream is None:
            if getattr(self, "_stream", None) is None:
                self._stream = torch.cuda.Stream(dev)
            stream = self._stream
        with torch.cuda.stream(stream):
            h = stream.cuda_stream
            part = torch.empty(self.rows, self.hd, device=dev, dtype=torch.float32)
            lse = torch.empty(self.rows, device=dev, dtype=torch.float32)
            decode_attention_partial(self.caches, d_q, self.n_q, 0, -1, part, lse, stream=h)
            parts = torch.empty(self.world, self.rows, self.hd, device=dev, dtype=torch.float32)
            lses = torch.empty(self.world, self.rows, device=dev, dtype=torch.float32)
            dist.all_gather_into_tensor(parts, part, group=self.group)
            dist.all_gather_into_tensor(lses, lse, group=self.group)
            lse_combine(self.world, self.rows, self.hd, parts, lses, d_out, None, stream=h)
        return d_out
