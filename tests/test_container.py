"""BOA2 container: byte-exact with the reference writer, parsed identically by
the reference reader (fixtures from tests/golden/make_golden.py), plus the
reader's failure modes (boa.py:117-133)."""
import json
import os
import struct

import numpy as np
import pytest

from boa_b200 import container as C

G = os.path.join(os.path.dirname(__file__), "golden")


class BoaBytePredictor:
    pass


def _case():
    meta = json.load(open(os.path.join(G, "ref_container.json")))
    return meta, meta["inputs"]


def _ours(inp, flags):
    comp = [np.asarray(w, dtype=np.uint32) for w in inp["words"]]
    sizes = [4 * len(c) for c in comp]
    offs = [int(x) for x in np.concatenate([[0], np.cumsum(sizes)[:-1]])]
    return (C.header_bytes(flags, inp["uncompressed_len"], inp["chunk_len"], len(comp), inp["last_chunk_len"],
                           C.model_fingerprint(BoaBytePredictor()))
            + b"".join(c.astype("<u4").tobytes() for c in comp) + C.index_bytes(inp["first_bytes"], offs, sizes))


def test_writer_matches_reference_bytes():
    meta, inp = _case()
    ref = open(os.path.join(G, "ref_container.boa"), "rb").read()
    assert _ours(inp, 0) == ref


def test_reader_matches_reference_parse():
    meta, inp = _case()
    for blob, key in ((open(os.path.join(G, "ref_container.boa"), "rb").read(), "reference_parse_of_reference_file"),
                      (_ours(inp, C.make_flags(16)), "reference_parse_of_our_file")):
        p = C.parse(blob)
        exp = meta[key]
        assert p.first_bytes == exp["first_bytes"]
        assert p.full_lens == exp["lengths"]
        assert {"chunk_len": p.chunk_len, "n_chunks": p.n_chunks, "last_chunk_len": p.last_chunk_len,
                "uncompressed_len": p.uncompressed_len} == exp["metadata"]
        payload = blob[p.payload_start:p.index_start]
        got = [payload[o:o + ln].hex() for o, ln in zip(p.offsets, p.lengths)]
        assert got == exp["payload_hex"]


def test_flags_roundtrip():
    assert C.flags_precision(C.make_flags(16)) == (True, 16)
    assert C.flags_precision(0) == (False, 24)
    for wf in C.WEIGHT_FORMAT_CODES:
        f = C.make_flags(16, wf)
        assert C.flags_weight_format(f) == wf and C.flags_precision(f) == (True, 16)
    assert C.flags_weight_format(C.make_flags(16)) is None


def test_uvarint():
    for x in (0, 1, 127, 128, 300, 2**32 - 1, 2**40 + 5):
        enc = C.uvarint_encode(x)
        assert C.uvarint_decode(enc, 0) == (x, len(enc))


@pytest.mark.parametrize("total,seq,cnt", [(1000, 0, 16), (1 << 20, 0, 16), (67108864, 0, 1000),
                                           (67108864, 0, 8192), (999, 100, 0), (1000, 100, 5)])
def test_chunking_matches_reference_rule(total, seq, cnt):
    chunk_len, n, last = C.chunking(total, seq, cnt)
    assert (n - 1) * chunk_len + last == total
    assert 1 <= last <= chunk_len


def test_more_chunks_than_bytes_leaves_empty_chunks():
    # boa.py:167-176 computes a non-positive last chunk here; the reference codec
    # then rejects the empty chunks (codec.py:28) and so does this build
    chunk_len, n, last = C.chunking(1, 0, 16)
    assert (chunk_len, n) == (1, 16) and last < 1


def test_reader_rejects_corruption():
    meta, inp = _case()
    good = _ours(inp, C.make_flags(16))
    with pytest.raises(ValueError, match="magic"):
        C.parse(b"XXXX" + good[4:])
    with pytest.raises(ValueError, match="version"):
        C.parse(good[:4] + struct.pack("<I", 2) + good[8:])
    bad = bytearray(good); bad[-6] ^= 0x55
    with pytest.raises(ValueError, match="CRC"):
        C.parse(bytes(bad))
    with pytest.raises(ValueError):
        C.parse(good[:len(good) // 2])
    with pytest.raises(ValueError, match="Index not found"):
        C.parse(good.replace(C.IDX, b"XXXX"))
