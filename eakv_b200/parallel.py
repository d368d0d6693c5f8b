"""Multi-GPU plumbing for the decode path: one process per GPU.

Two ways to spread the work:

* KV-head shards: each rank holds some KV heads (with their query heads)
  of every sequence and layer and decodes them with `eakv_decode_attention`;
  heads are independent, so there is no data-path collective.
* Sequence split, for a context larger than one GPU's share: rank r holds
  positions [begin_r, end_r) of every sequence in its own local caches, and
  `eakv_decode_attention_split` (include/eakv_nccl.h) computes that range's
  record (normalized output, natural-log LSE), all-gathers the records of
  the group over the library's own NCCL communicator and merges them
  exactly, all on one CUDA stream:

      out = sum_r exp(lse_r - L) out_r,   L = log sum_r exp(lse_r).

Softmax attention over a set of positions does not depend on their order,
so a rank's slice can sit at local positions 0.. of its caches.

torch.distributed is only the launcher's plumbing here (it carries the NCCL
unique id to the ranks of a group); the data path is the library's.
"""
import math

import numpy as np

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
    """Sequence-split decode over one group of ranks, through the library.

    caches: this rank's local caches (its slice of every sequence). The
    group's first rank makes an NCCL unique id, torch.distributed carries it
    to the others, and every rank joins the library's communicator on
    `device` (collective: every rank of the group constructs its decoder at
    the same point). Every rank calls `step` with the same queries, in the
    same order; every rank receives the merged output.
    """

    def __init__(self, caches, n_q_heads, head_dim, group=None, device=None):
        import torch.distributed as dist
        from . import NcclComm, nccl_unique_id
        self.caches = caches
        self.n_q = n_q_heads
        self.hd = head_dim
        self.world = dist.get_world_size(group)
        rank = dist.get_rank(group)
        leader = dist.get_global_rank(group, 0) if group is not None else 0
        box = [nccl_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(box, src=leader, group=group)
        dev = caches[0].device if device is None else device
        self.comm = NcclComm(self.world, box[0], rank, dev)

    def step(self, d_q, d_out, stream=None):
        """One decode step: `stream` is a CUDA stream handle (int) or a
        torch.cuda.Stream; the partial decode, the all-gather and the merge
        are all queued on it, and nothing synchronizes the host."""
        from . import decode_attention_split
        h = getattr(stream, "cuda_stream", stream)
        decode_attention_split(self.caches, d_q, self.n_q, d_out, self.comm, stream=h)
        return d_out

    def step_host(self, queries, output, stream=None):
        """One step with host buffers (numpy or pinned torch CPU tensors):
        copies overlapped with the library's chunked split steps."""
        from . import decode_attention_split_host
        h = getattr(stream, "cuda_stream", stream)
        decode_attention_split_host(self.caches, queries, self.n_q, output, self.comm, stream=h)
        return output

    def close(self):
        self.comm.destroy()
