"""Sequence sharding across processes (one per GPU).

The encoder needs no exchange step: each rank holds a full model replica and
embeds a contiguous shard of the packed sequences.  shard_bounds() is the
token-balanced split le_embed_ids uses across devices inside one process
(work of a sequence of length L: 226,492,416 L + 36,864 L^2 FLOP); the only
collective is the optional gather of the embeddings to one rank.
"""
from __future__ import annotations

import numpy as np

GEMM_FLOP_PER_TOKEN = 226492416.0
ATTN_FLOP_PER_L2 = 36864.0


def seq_work(lengths) -> np.ndarray:
    L = np.asarray(lengths, np.float64)
    return GEMM_FLOP_PER_TOKEN * L + ATTN_FLOP_PER_L2 * L * L


def shard_bounds(offsets, n: int) -> list[int]:
    """Cut points c[0]=0 <= ... <= c[n]=nseq of contiguous, work-balanced
    shards: shard i is sequences [c[i], c[i+1])."""
    offsets = np.asarray(offsets)
    nseq = offsets.size - 1
    w = seq_work(np.diff(offsets))
    total = float(w.sum())
    cut = [0] + [nseq] * n
    acc, k = 0.0, 1
    for s in range(nseq):
        if k >= n:
            break
        acc += float(w[s])
        while k < n and acc >= total * k / n:
            cut[k] = s + 1
            k += 1
    return cut


def local_shard(ids, offsets, rank: int, world: int):
    """(ids, offsets, first, last) of this rank's shard, offsets rebased."""
    offsets = np.asarray(offsets, np.int32)
    c = shard_bounds(offsets, world)
    a, b = c[rank], c[rank + 1]
    sub_offs = (offsets[a:b + 1] - offsets[a]).astype(np.int32)
    return np.asarray(ids[offsets[a]:offsets[b]], np.int32), sub_offs, a, b


def embed_sharded(embed_fn, ids, offsets, dim: int, group=None, dst: int = 0):
    """Embed this rank's shard with embed_fn(ids, offsets) -> [n][dim] and
    gather all shards on rank `dst` (None elsewhere).  The gather pads each
    shard to the largest one (torch.distributed.gather needs equal shapes)."""
    import torch
    import torch.distributed as dist
    rank, world = dist.get_rank(group), dist.get_world_size(group)
    sub_ids, sub_offs, a, b = local_shard(ids, offsets, rank, world)
    out = embed_fn(sub_ids, sub_offs) if b > a else np.zeros((0, dim), np.float32)
    cut = shard_bounds(offsets, world)
    rows = max(cut[i + 1] - cut[i] for i in range(world))
    backend = dist.get_backend(group)
    dev = torch.device("cuda", torch.cuda.current_device()) if backend == "nccl" else torch.device("cpu")
    buf = torch.zeros(rows, dim, dtype=torch.float32, device=dev)
    if b > a:
        buf[:b - a] = torch.from_numpy(np.ascontiguousarray(out, np.float32)).to(dev)
    gl = [torch.zeros_like(buf) for _ in range(world)] if rank == dst else None
    dist.gather(buf, gl, dst=dst, group=group)
    if rank != dst:
        return None
    return np.concatenate([gl[i][:cut[i + 1] - cut[i]].cpu().numpy() for i in range(world)], axis=0)
