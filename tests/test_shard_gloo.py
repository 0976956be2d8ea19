"""Multi-rank sharding of one BOA2 file, on CPU gloo ranks (world size 2).

The device codec is replaced by a deterministic stand-in that turns a chunk
into fake u32 words; what is tested is the host logic of boa_b200.shard: the
contiguous per-rank ranges, the all-reduce that gathers per-chunk lengths and
first bytes, and every rank writing its payload at the right offset, so the
file equals the single-process one and parses with the reference-compatible
reader.
"""
import os
import socket

import numpy as np
import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

from boa_b200 import container as C
from boa_b200.shard import gather_lengths, shard_range, write_decoded, write_sharded


def _fake_words(chunk: np.ndarray) -> np.ndarray:
    # length depends on content, so offsets differ per chunk
    n = 1 + int(chunk.sum()) % 7
    return (np.arange(n, dtype=np.uint32) * 2654435761 + np.uint32(chunk[0])).astype(np.uint32)


def _write(path, data: bytes, n_chunks: int, world: int, rank: int, dist_mod):
    chunk_len, n, last = C.chunking(len(data), 0, n_chunks)
    lens = [chunk_len] * (n - 1) + [last]
    lo, hi = shard_range(n, world, rank)
    buf = np.frombuffer(data, np.uint8)
    sizes, firsts, payload = [], [], b""
    for i in range(lo, hi):
        ch = buf[i * chunk_len:i * chunk_len + lens[i]]
        w = _fake_words(ch)
        sizes.append(4 * len(w)); firsts.append(int(ch[0])); payload += w.astype("<u4").tobytes()
    sizes_all, firsts_all = gather_lengths(dist_mod, n, lo, hi, sizes, firsts)
    hdr = C.header_bytes(C.make_flags(16), len(data), chunk_len, n, last, b"\x00" * 16)
    write_sharded(path, hdr, lambda offs: C.index_bytes(firsts_all.tolist(), offs.tolist(), sizes_all.tolist()),
                  sizes_all, lo, payload, dist_mod, rank)


def _worker(rank, world, port, path, data, n_chunks):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        _write(path, data, n_chunks, world, rank, dist)
    finally:
        dist.destroy_process_group()


def _free_port():
    s = socket.socket(); s.bind(("127.0.0.1", 0)); p = s.getsockname()[1]; s.close(); return p


@pytest.mark.parametrize("n_chunks", [5, 16, 33])
def test_two_rank_file_equals_single_rank(tmp_path, n_chunks):
    rng = np.random.default_rng(n_chunks)
    data = rng.integers(0, 256, 4000 + n_chunks).astype(np.uint8).tobytes()
    single = tmp_path / "one.boa"
    _write(str(single), data, n_chunks, 1, 0, None)
    multi = tmp_path / "two.boa"
    mp.start_processes(_worker, args=(2, _free_port(), str(multi), data, n_chunks), nprocs=2, join=True,
                       start_method="spawn")
    a, b = single.read_bytes(), multi.read_bytes()
    assert a == b
    p = C.parse(b)
    assert p.n_chunks == n_chunks and sum(p.full_lens) == len(data)


def test_shard_ranges_cover_all_chunks():
    for n in (1, 2, 7, 1000, 8192):
        for w in (1, 2, 3, 4, 8):
            got = [shard_range(n, w, r) for r in range(w)]
            assert got[0][0] == 0 and got[-1][1] == n
            assert all(got[i][1] == got[i + 1][0] for i in range(w - 1))


def _decode_worker(rank, world, port, path, data, n_chunks):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        chunk_len, n, last = C.chunking(len(data), 0, n_chunks)
        lo, hi = shard_range(n, world, rank)
        mine = data[lo * chunk_len:min(hi * chunk_len, len(data))]     # this rank's "decoded" chunks
        write_decoded(path, len(data), chunk_len, lo, mine, dist, rank)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("n_chunks,world", [(5, 2), (33, 2), (7, 3)])
def test_ranks_assemble_decoded_file_without_a_data_collective(tmp_path, n_chunks, world):
    """Multi-rank decompress: each rank writes its own decoded chunks at
    chunk_index * chunk_len of one shared file; only barriers are exchanged."""
    rng = np.random.default_rng(100 + n_chunks)
    data = rng.integers(0, 256, 3000 + n_chunks).astype(np.uint8).tobytes()
    out = tmp_path / "dec.bin"
    mp.start_processes(_decode_worker, args=(world, _free_port(), str(out), data, n_chunks), nprocs=world,
                       join=True, start_method="spawn")
    assert out.read_bytes() == data
