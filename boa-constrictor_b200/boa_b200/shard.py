"""Multi-GPU sharding of one BOA2 file (one process per GPU).

Chunks are independent, so rank r of W takes the contiguous range
``[n*r//W, n*(r+1)//W)`` (all chunks but the last have the same length, so
equal counts are equal bytes).  The only exchange is one all-reduce over
disjoint per-chunk slots, which gathers every chunk's compressed byte length
and first byte; each rank then knows every payload offset (an exclusive
prefix sum) and writes its own payload bytes at its offset in the shared
output file.  Rank 0 writes the header first and the index last.  Decompress
needs no exchange at all: chunk i's bytes start at i * chunk_len, so each rank
writes its decoded chunks straight into the shared output file.  No data-path
collective; the process group carries only the length all-reduce and
barriers.
"""
from __future__ import annotations

import numpy as np
import torch


def shard_range(n_chunks: int, world: int, rank: int):
    return (n_chunks * rank) // world, (n_chunks * (rank + 1)) // world


def collective_device(dist):
    return torch.device("cuda", torch.cuda.current_device()) if dist.get_backend() == "nccl" else torch.device("cpu")


def gather_lengths(dist, n_chunks: int, lo: int, hi: int, sizes_bytes_local, firsts_local):
    """All ranks get the full (sizes_bytes[n], first_bytes[n]) vectors."""
    t = torch.zeros((2, n_chunks), dtype=torch.int64)
    t[0, lo:hi] = torch.as_tensor(np.asarray(sizes_bytes_local, dtype=np.int64))
    t[1, lo:hi] = torch.as_tensor(np.asarray(firsts_local, dtype=np.int64))
    if dist is not None:
        t = t.to(collective_device(dist))
        dist.all_reduce(t)      # disjoint slots: the sum is a gather
        t = t.cpu()
    return t[0].numpy(), t[1].numpy()


def write_sharded(path, header: bytes, index_fn, sizes_bytes, lo: int, payload: bytes, dist, rank: int):
    """Write header (rank 0), this rank's payload at its offset, then the index
    (rank 0).  index_fn(offsets) returns the index bytes."""
    offsets = np.zeros(len(sizes_bytes), dtype=np.int64)
    if len(sizes_bytes) > 1:
        offsets[1:] = np.cumsum(sizes_bytes)[:-1]
    if rank == 0:
        with open(path, "wb") as f:
            f.write(header)
    if dist is not None:
        dist.barrier()
    if payload:
        with open(path, "r+b") as f:
            f.seek(len(header) + int(offsets[lo]))
            f.write(payload)
    if dist is not None:
        dist.barrier()
    if rank == 0:
        with open(path, "r+b") as f:
            f.seek(len(header) + int(np.sum(sizes_bytes)))
            f.write(index_fn(offsets))
            f.truncate()
    if dist is not None:
        dist.barrier()
    return offsets


def write_decoded(path, total_len: int, chunk_len: int, lo: int, payload: bytes, dist, rank: int) -> None:
    """Rank 0 creates `path` with total_len bytes; every rank then writes its
    decoded chunks (which start with chunk `lo`) at byte offset
    lo * chunk_len.  Returns once every rank has written."""
    if rank == 0:
        with open(path, "wb") as f:
            f.truncate(total_len)
    if dist is not None:
        dist.barrier()
    if payload:
        with open(path, "r+b") as f:
            f.seek(lo * chunk_len)
            f.write(payload)
    if dist is not None:
        dist.barrier()
