"""The chunked ``BOA2`` container (boa.py:17-31, 47-157, 185-194, 252-262).

Layout, all little-endian::

    'BOA2' | u32 version=1 | u32 flags | u64 uncompressed_len | u32 chunk_len |
    u32 n_chunks | u32 last_chunk_len | u8 fp_len | fp (blake2s-16 of the model
    class name) | payload = concat(per-chunk u32 words) |
    index = 'IDX1' + n x u8 first_bytes + n x uvarint(offset deltas) +
            n x uvarint(byte lengths) | u32 crc32(index)

``flags`` is ignored by the reference reader (boa.py:121).  This build sets
bit 0 for streams coded with its integer quantiser, stores the table
precision in bits 8-15 and the model's operand kind in bits 16-23; files with bit 0 clear were coded with the
reference's float quantiser at precision 24.
"""
from __future__ import annotations

import hashlib
import math
import struct
import zlib
from dataclasses import dataclass, field

MAGIC = b"BOA2"
IDX = b"IDX1"
VERSION = 1
FLAG_BQ = 0x1
HEADER_FIXED = 4 + 4 + 4 + 8 + 4 + 4 + 4 + 1


# bits 16-23 of flags: the model's projection operand kind (0: not recorded).
# Streams decode only under the kind that coded them.
WEIGHT_FORMAT_CODES = {"tf32": 1, "bf16": 2, "fp16": 3, "tf32x3": 4, "f16x2": 5}


def make_flags(precision: int, weight_format: str | None = None) -> int:
    f = FLAG_BQ | ((int(precision) & 0xFF) << 8)
    if weight_format is not None:
        f |= WEIGHT_FORMAT_CODES[weight_format] << 16
    return f


def flags_weight_format(flags: int) -> str | None:
    """The operand kind recorded in flags, or None for files that do not record one."""
    code = (flags >> 16) & 0xFF
    for k, v in WEIGHT_FORMAT_CODES.items():
        if v == code:
            return k
    return None


def flags_precision(flags: int) -> tuple[bool, int]:
    """(uses the integer quantiser, table precision)."""
    if flags & FLAG_BQ:
        p = (flags >> 8) & 0xFF
        return True, (p if p else 16)
    return False, 24


def uvarint_encode(x: int) -> bytes:
    out = bytearray()
    while True:
        b = x & 0x7F
        x >>= 7
        out.append(b | (0x80 if x else 0))
        if not x:
            return bytes(out)


def uvarint_decode(buf, pos: int):
    x = 0
    s = 0
    while True:
        if pos >= len(buf):
            raise ValueError("Truncated index (uvarint runs past the end)")
        b = buf[pos]
        pos += 1
        x |= (b & 0x7F) << s
        if not (b & 0x80):
            return x, pos
        s += 7


def model_fingerprint(model) -> bytes:
    """blake2s-16 of the model's class name (boa.py:85-87)."""
    name = getattr(model, "__class__", type(model)).__name__
    return hashlib.blake2s(name.encode(), digest_size=16).digest()


def chunking(total_size: int, seq_size: int = 0, chunks_count: int = 0):
    """(chunk_len, n_chunks, last_chunk_len) exactly as boa.py:167-176."""
    if seq_size and chunks_count:
        chunk_len = int(seq_size); n_chunks = math.ceil(total_size / chunk_len)
    elif seq_size:
        chunk_len = int(seq_size); n_chunks = math.ceil(total_size / chunk_len)
    elif chunks_count:
        n_chunks = max(int(chunks_count), 1); chunk_len = math.ceil(total_size / n_chunks)
    else:
        raise ValueError("Provide either 'seq_size' or 'chunks_count'.")
    last = int(total_size - (n_chunks - 1) * chunk_len) if n_chunks > 1 else int(total_size)
    return int(chunk_len), int(n_chunks), int(last)


def header_bytes(flags: int, total_size: int, chunk_len: int, n_chunks: int, last_chunk_len: int,
                 fp: bytes) -> bytes:
    return (MAGIC + struct.pack("<I", VERSION) + struct.pack("<I", flags) + struct.pack("<Q", total_size)
            + struct.pack("<I", chunk_len) + struct.pack("<I", n_chunks) + struct.pack("<I", last_chunk_len)
            + struct.pack("<B", len(fp)) + fp)


def index_bytes(first_bytes, offsets, lengths) -> bytes:
    idx = bytearray(IDX)
    idx += bytes(int(b) & 0xFF for b in first_bytes)
    prev = 0
    for o in offsets:
        idx += uvarint_encode(int(o) - prev)
        prev = int(o)
    for ln in lengths:
        idx += uvarint_encode(int(ln))
    crc = zlib.crc32(idx) & 0xFFFFFFFF
    return bytes(idx) + struct.pack("<I", crc)


@dataclass
class Parsed:
    flags: int
    uncompressed_len: int
    chunk_len: int
    n_chunks: int
    last_chunk_len: int
    fingerprint: bytes
    payload_start: int
    index_start: int
    first_bytes: list = field(default_factory=list)
    offsets: list = field(default_factory=list)
    lengths: list = field(default_factory=list)

    @property
    def full_lens(self):
        n = self.n_chunks
        return [int(self.chunk_len)] * (n - 1) + [int(self.last_chunk_len)] if n else []


def parse(data: bytes) -> Parsed:
    """Parse and validate a BOA2 file (boa.py:114-157), with bounds checks the
    reference leaves to Python's slicing."""
    mm = memoryview(data)
    if len(data) < HEADER_FIXED + 4 or bytes(mm[0:4]) != MAGIC:
        raise ValueError("Bad file magic")
    p = 4
    version, = struct.unpack_from("<I", mm, p); p += 4
    if version != VERSION:
        raise ValueError(f"Unsupported version {version}")
    flags, = struct.unpack_from("<I", mm, p); p += 4
    ulen, = struct.unpack_from("<Q", mm, p); p += 8
    chunk_len, = struct.unpack_from("<I", mm, p); p += 4
    n, = struct.unpack_from("<I", mm, p); p += 4
    last_chunk_len, = struct.unpack_from("<I", mm, p); p += 4
    hlen = mm[p]; p += 1
    fp = bytes(mm[p:p + hlen]); p += hlen
    crc = struct.unpack_from("<I", mm, len(mm) - 4)[0]
    idx_pos = data.rfind(IDX)
    if idx_pos < 0 or idx_pos < p:
        raise ValueError("Index not found")
    if (zlib.crc32(data[idx_pos:len(data) - 4]) & 0xFFFFFFFF) != crc:
        raise ValueError("Bad index CRC")
    q = idx_pos + len(IDX)
    if q + n > len(data) - 4:
        raise ValueError("Truncated index")
    first_bytes = list(mm[q:q + n]); q += n
    offsets = [0] * n
    prev = 0
    for i in range(n):
        d, q = uvarint_decode(mm, q)
        prev += d
        offsets[i] = prev
    lengths = [0] * n
    for i in range(n):
        lengths[i], q = uvarint_decode(mm, q)
    payload_len = idx_pos - p
    for i in range(n):
        if offsets[i] + lengths[i] > payload_len:
            raise ValueError(f"Chunk {i} runs past the payload")
        if lengths[i] % 4:
            raise ValueError(f"Chunk {i} length is not a whole number of u32 words")
    return Parsed(flags, ulen, chunk_len, n, last_chunk_len, fp, p, idx_pos, first_bytes, offsets, lengths)


# ---------------------------------------------------------------------------
# Streaming / resumable writer
# ---------------------------------------------------------------------------
PROVISIONAL = b"IDXP"


def provisional_index(first_bytes, lengths) -> bytes:
    """'IDXP' | u32 k | k x u8 first_bytes | k x uvarint(byte lengths) | u32 crc32.
    Offsets are the running sum of the lengths (payload written in order)."""
    idx = bytearray(PROVISIONAL) + struct.pack("<I", len(lengths))
    idx += bytes(int(b) & 0xFF for b in first_bytes)
    for ln in lengths:
        idx += uvarint_encode(int(ln))
    return bytes(idx) + struct.pack("<I", zlib.crc32(idx) & 0xFFFFFFFF)


def parse_provisional(data: bytes, payload_start: int):
    """(first_bytes, lengths) recorded by the last complete provisional index."""
    pos = data.rfind(PROVISIONAL)
    if pos < payload_start or pos + 12 > len(data):
        raise ValueError("no provisional index: nothing to resume")
    k, = struct.unpack_from("<I", data, pos + 4)
    q = pos + 8
    if q + k > len(data):
        raise ValueError("truncated provisional index")
    firsts = list(data[q:q + k])
    q += k
    lengths = []
    mm = memoryview(data)
    for _ in range(k):
        ln, q = uvarint_decode(mm, q)
        lengths.append(ln)
    if q + 4 > len(data):
        raise ValueError("truncated provisional index")
    crc, = struct.unpack_from("<I", data, q)
    if (zlib.crc32(data[pos:q]) & 0xFFFFFFFF) != crc:
        raise ValueError("bad provisional index CRC")
    if payload_start + sum(lengths) != pos:
        raise ValueError("provisional index does not follow its payload")
    return firsts, lengths


class StreamingWriter:
    """Write a BOA2 file wave by wave (boa.py:195-262 streams the payload the
    same way).  After every wave the payload is followed by a provisional
    index that records the chunks written so far, so a run that stops between
    waves can resume after the last complete one (``resume=True``); finish()
    replaces it with the final 'IDX1' index, which is all a reader sees."""

    def __init__(self, path, header: bytes, n_chunks: int, resume: bool = False):
        import os
        self.path = str(path)
        self.n_chunks = int(n_chunks)
        self.payload_start = len(header)
        self.firsts: list[int] = []
        self.lengths: list[int] = []
        if resume and os.path.exists(self.path):
            with open(self.path, "rb") as f:
                data = f.read()
            if data[:len(header)] != header:
                raise ValueError("cannot resume: the file header differs (another input, chunking or model)")
            self.firsts, self.lengths = parse_provisional(data, self.payload_start)
            if len(self.lengths) > self.n_chunks:
                raise ValueError("cannot resume: the file records more chunks than the input has")
            self.f = open(self.path, "r+b")
        else:
            self.f = open(self.path, "wb")
            self.f.write(header)
            self._write_tail(provisional_index([], []))

    @property
    def chunks_done(self) -> int:
        return len(self.lengths)

    def _end(self) -> int:
        return self.payload_start + sum(self.lengths)

    def _write_tail(self, tail: bytes):
        self.f.seek(self._end())
        self.f.write(tail)
        self.f.truncate()
        self.f.flush()

    def append(self, first_bytes, payloads) -> None:
        """Add the next chunks: their first bytes and u32 word payloads (bytes)."""
        if self.chunks_done + len(payloads) > self.n_chunks:
            raise ValueError("more chunks than the header declares")
        self.f.seek(self._end())
        for b in payloads:
            self.f.write(b)
        self.firsts.extend(int(x) & 0xFF for x in first_bytes)
        self.lengths.extend(len(b) for b in payloads)
        self._write_tail(provisional_index(self.firsts, self.lengths))

    def finish(self) -> None:
        if self.chunks_done != self.n_chunks:
            raise ValueError(f"finish after {self.chunks_done} of {self.n_chunks} chunks")
        offsets, off = [], 0
        for ln in self.lengths:
            offsets.append(off)
            off += ln
        self._write_tail(index_bytes(self.firsts, offsets, self.lengths))
        self.f.close()

    def close(self) -> None:
        if not self.f.closed:
            self.f.close()
