"""Drop-in for the reference ``boa.py``: ``BOA(device, filepath, model)`` returns
a ``BoaFile`` with ``compress(data_path, seq_size=0, chunks_count=0,
progress=True)``, ``decompress(progress=True) -> bytes``, ``read_from_disk()``
and ``get_metadata()`` (boa.py:7-313), writing and reading the same ``BOA2``
container (boa.py:47-157).

Differences by design:
  * every wave of chunks goes through the fused sm_100a codec kernel
    (codec.encode_device / decode_device) instead of a per-byte Python loop;
  * ``flags`` records the quantiser (bit 0), the table precision (bits 8-15)
    and the model's operand kind (bits 16-23, checked on decompress);
  * when ``torch.distributed`` is initialised with more than one rank, the
    chunks are split into contiguous, byte-balanced ranges, one per rank (one
    GPU per rank); each rank codes its range, the per-chunk word counts and
    first bytes are all-gathered (the only collective), and every rank writes
    its own payload bytes at the offsets that the gathered counts imply.
    ``decompress`` splits the index the same way; each rank writes its decoded
    chunks at their offsets in a shared output file (no collective moves
    data) and every rank returns the whole file read back from it.
"""
from __future__ import annotations

import os
from pathlib import Path

import numpy as np
import torch

import codec as _codec
from boa_b200 import container as C
from boa_b200.shard import gather_lengths, shard_range, write_decoded, write_sharded


def _dist():
    import torch.distributed as dist
    if dist.is_available() and dist.is_initialized() and dist.get_world_size() > 1:
        return dist
    return None


def BOA(device, filepath: str, model):
    IS_CUDA = str(device).startswith("cuda") and torch.cuda.is_available()
    if not IS_CUDA:
        raise RuntimeError("boa_b200 runs on CUDA devices only; BOA(device='cpu', ...) has no implementation here")
    dev = torch.device(device)
    if dev.index is None:
        dev = torch.device("cuda", torch.cuda.current_device())

    class BoaFile:
        MAGIC = C.MAGIC
        IDX = C.IDX
        VERSION = C.VERSION

        def __init__(self, filepath: str, model):
            self.filepath = Path(filepath)
            self.model = model
            self.compressed_data = []
            self.first_bytes = []
            self.lengths = []
            self.metadata = {}
            self.precision = _codec.PRECISION

        def _model_fingerprint(self) -> bytes:
            return C.model_fingerprint(self.model)

        def _gpu_streams(self, n):
            try:
                s = int(os.getenv("BOA_GPU_STREAMS", "5000"))
            except Exception:
                s = 5000
            return max(1, min(int(s), int(n)))

        def _read_file(self):
            data = Path(self.filepath).read_bytes()
            p = C.parse(data)
            self._flags = p.flags
            payload = memoryview(data)[p.payload_start:p.index_start]
            self.compressed_data = [bytes(payload[p.offsets[i]:p.offsets[i] + p.lengths[i]])
                                    for i in range(p.n_chunks)]
            self.first_bytes = p.first_bytes
            self.lengths = p.full_lens
            self.metadata = {"chunk_len": int(p.chunk_len), "n_chunks": int(p.n_chunks),
                             "last_chunk_len": int(p.last_chunk_len), "uncompressed_len": int(p.uncompressed_len)}

        def read_from_disk(self):
            self._read_file()
            print("File loaded successfully")

        def get_metadata(self):
            return dict(self.metadata)

        # Waves are pipelined: while the kernel codes wave k, the host packs
        # wave k + 1 into pinned memory and writes out wave k - 1.  A wave's
        # results are read (and the model's device-side errors checked) only
        # when it is the one wave in flight, so each error is attributed to
        # its wave before that wave is written.
        def _pack_wave(self, mm, lens, chunk_len, b0, b1):
            """Chunks [b0, b1) of the input in pinned host memory (CPU work)."""
            nb = b1 - b0
            maxL = max(lens[b0:b1])
            host = torch.zeros((nb, maxL), dtype=torch.uint8, pin_memory=True)
            hv = host.numpy()
            for j, i in enumerate(range(b0, b1)):
                s = i * chunk_len
                hv[j, :lens[i]] = mm[s:s + lens[i]]
            return host, lens[b0:b1]

        def _enqueue_encode(self, packed):
            """H2D, encode kernel and D2H of one packed wave, all asynchronous."""
            host, wl = packed
            X = host.to(dev, non_blocking=True)
            L_d = torch.tensor(wl, dtype=torch.int32).pin_memory().to(dev, non_blocking=True)
            words, sizes = _codec.encode_device(self.model, X, L_d, precision=self.precision)
            w_h = torch.empty(words.shape, dtype=words.dtype, pin_memory=True)
            s_h = torch.empty(sizes.shape, dtype=sizes.dtype, pin_memory=True)
            w_h.copy_(words, non_blocking=True)
            s_h.copy_(sizes, non_blocking=True)
            return host, w_h, s_h

        def _finish_encode(self, pending):
            """Wait for the wave in flight: (first bytes, per-chunk u32 LE payloads)."""
            host, w_h, s_h = pending
            self.model._native_handle(dev).check()
            sz = s_h.numpy().astype(np.int64)
            wh = w_h.numpy().view(np.uint32)
            return host.numpy()[:, 0].astype(np.int64), [wh[j, :sz[j]].astype("<u4").tobytes()
                                                         for j in range(len(sz))]

        def _encode_waves(self, mm, lens, chunk_len, b_first, b_end, stream_n):
            """Yield (first bytes, payloads) of the waves of chunks [b_first, b_end), in order."""
            pending = None
            for b0 in range(b_first, b_end, stream_n):
                packed = self._pack_wave(mm, lens, chunk_len, b0, min(b0 + stream_n, b_end))
                done = self._finish_encode(pending) if pending is not None else None
                pending = self._enqueue_encode(packed)
                if done is not None:
                    yield done
            if pending is not None:
                yield self._finish_encode(pending)

        # ------------------------------------------------------------------
        def compress(self, data_path: str, seq_size: int = 0, chunks_count: int = 0, progress: bool = True,
                     resume: bool = False):
            """boa.py:159-268.  One process: every wave's payload is appended to
            the file as soon as it is coded (StreamingWriter); with resume=True a
            run that stopped between waves continues after the last complete
            wave.  Several ranks: each codes its contiguous chunk range and
            writes its payload at the gathered offsets."""
            p = Path(data_path)
            total = p.stat().st_size
            if total <= 0:
                raise ValueError("Input file is empty")
            chunk_len, n_chunks, last = C.chunking(total, seq_size, chunks_count)
            self.metadata = {"chunk_len": chunk_len, "n_chunks": n_chunks, "uncompressed_len": int(total),
                             "last_chunk_len": int(last if last else chunk_len)}
            lens = [chunk_len] * (n_chunks - 1) + [last]
            for i, ln in enumerate(lens):    # codec.py:28
                assert ln >= 1, f"Chunk {i} must have length >= 1"
            dist = _dist()
            world, rank = (dist.get_world_size(), dist.get_rank()) if dist else (1, 0)
            lo, hi = shard_range(n_chunks, world, rank)
            mm = np.memmap(p, dtype=np.uint8, mode="r")
            stream_n = self._gpu_streams(max(hi - lo, 1))
            hdr = C.header_bytes(C.make_flags(self.precision, getattr(self.model, "weight_format", None)), total,
                                 chunk_len, n_chunks, last,
                                 self._model_fingerprint())
            if dist is None:
                w = C.StreamingWriter(self.filepath, hdr, n_chunks, resume=resume)
                try:
                    for firsts, payload in self._encode_waves(mm, lens, chunk_len, w.chunks_done, n_chunks,
                                                              stream_n):
                        w.append(firsts, payload)
                    w.finish()
                finally:
                    w.close()
                self.compressed_data = []
                self.first_bytes = list(w.firsts)
                self.lengths = lens
                if progress:
                    print(f"Compression complete: {n_chunks} chunks, chunk_len={chunk_len}, last={last}")
                return
            sizes_local = np.zeros(hi - lo, dtype=np.int64)
            firsts_local = np.zeros(hi - lo, dtype=np.int64)
            payloads = []
            b0 = lo
            for firsts, payload in self._encode_waves(mm, lens, chunk_len, lo, hi, stream_n):
                b1 = b0 + len(payload)
                firsts_local[b0 - lo:b1 - lo] = firsts
                sizes_local[b0 - lo:b1 - lo] = [len(x) for x in payload]
                payloads.append(b"".join(payload))
                b0 = b1
            sizes_bytes, firsts = gather_lengths(dist, n_chunks, lo, hi, sizes_local, firsts_local)
            write_sharded(self.filepath, hdr, lambda offs: C.index_bytes(firsts.tolist(), offs.tolist(),
                                                                         sizes_bytes.tolist()),
                          sizes_bytes, lo, b"".join(payloads), dist, rank)
            self.compressed_data = []
            self.first_bytes = [int(b) for b in firsts]
            self.lengths = lens
            if progress and rank == 0:
                print(f"Compression complete: {n_chunks} chunks, chunk_len={chunk_len}, last={last}")

        def _pack_words(self, lens, precision, b0, b1):
            """The words, sizes, lengths and first bytes of chunks [b0, b1) in pinned memory."""
            wl = lens[b0:b1]
            comp = [np.frombuffer(c, dtype="<u4") for c in self.compressed_data[b0:b1]]
            pitch = max(_codec.pitch_words_for(max(wl), precision), max(len(c) for c in comp))
            words = torch.zeros((b1 - b0, pitch), dtype=torch.int32, pin_memory=True)
            wv = words.numpy().view(np.uint32)
            for j, c in enumerate(comp):
                wv[j, :len(c)] = c
            meta = torch.tensor([[len(c) for c in comp], list(wl), [int(b) & 0xFF for b in self.first_bytes[b0:b1]]],
                                dtype=torch.int32).pin_memory()
            return words, meta, wl

        def _enqueue_decode(self, packed, precision):
            words, meta, wl = packed
            w_d = words.to(dev, non_blocking=True)
            m_d = meta.to(dev, non_blocking=True)
            out = _codec.decode_device(self.model, w_d, m_d[0], m_d[1], m_d[2].to(torch.uint8), max_len=max(wl),
                                       precision=precision)
            o_h = torch.empty(out.shape, dtype=torch.uint8, pin_memory=True)
            o_h.copy_(out, non_blocking=True)
            return words, meta, o_h, wl

        def _finish_decode(self, pending):
            words, meta, o_h, wl = pending
            self.model._native_handle(dev).check()
            ov = o_h.numpy()
            return b"".join(ov[j, :wl[j]].tobytes() for j in range(len(wl)))

        # ------------------------------------------------------------------
        def decompress(self, progress: bool = True, out_path: str | None = None) -> bytes:
            """boa.py:274-308.  With several ranks, the decoded file is assembled
            in `out_path` (default: this file's path + '.decoded'), each rank
            writing its own chunks there; every rank returns the whole file."""
            self._read_file()
            bq, precision = C.flags_precision(self._flags)
            wf = C.flags_weight_format(self._flags)
            mine = getattr(self.model, "weight_format", None)
            if wf is not None and mine is not None and wf != mine:
                raise ValueError(f"this file was coded with {wf} projections; the model computes {mine}, whose "
                                 f"probabilities differ: construct it with weight_format={wf!r}")
            if not bq:
                raise ValueError("this file was coded with the reference float quantiser (flags bit 0 clear); "
                                 "its probabilities come from other kernels and cannot be reproduced bit for bit")
            n = len(self.compressed_data)
            lens = self.lengths
            dist = _dist()
            world, rank = (dist.get_world_size(), dist.get_rank()) if dist else (1, 0)
            lo, hi = shard_range(n, world, rank)
            stream_n = self._gpu_streams(max(hi - lo, 1))
            parts = []
            pending = None
            for b0 in range(lo, hi, stream_n):
                packed = self._pack_words(lens, precision, b0, min(b0 + stream_n, hi))
                done = self._finish_decode(pending) if pending is not None else None
                pending = self._enqueue_decode(packed, precision)
                if done is not None:
                    parts.append(done)
            if pending is not None:
                parts.append(self._finish_decode(pending))
            mine = b"".join(parts)
            if not dist:
                return mine
            target = Path(out_path) if out_path else Path(str(self.filepath) + ".decoded")
            write_decoded(target, int(self.metadata["uncompressed_len"]), int(self.metadata["chunk_len"]), lo, mine,
                          dist, rank)
            return target.read_bytes()

    return BoaFile(filepath, model)
