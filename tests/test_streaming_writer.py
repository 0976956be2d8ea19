"""Streaming / resumable BOA2 writer: a file written wave by wave, with a stop
between waves and a resume, equals the file written in one go and parses with
the reference-compatible reader; an incomplete file is not a valid container."""
import numpy as np
import pytest

from boa_b200 import container as C


def _case(n, seed=0):
    rng = np.random.default_rng(seed)
    words = [rng.integers(0, 2**32, size=int(k), dtype=np.uint64).astype("<u4").tobytes()
             for k in rng.integers(0, 9, n)]
    firsts = [int(x) for x in rng.integers(0, 256, n)]
    return words, firsts


def _header(n):
    return C.header_bytes(C.make_flags(16), 1000 * n - 10, 1000, n, 990, b"\x01" * 16)


def _one_shot(path, n, words, firsts):
    sizes = [len(w) for w in words]
    offs = [int(x) for x in np.concatenate([[0], np.cumsum(sizes)[:-1]])] if n else []
    with open(path, "wb") as f:
        f.write(_header(n))
        f.write(b"".join(words))
        f.write(C.index_bytes(firsts, offs, sizes))


@pytest.mark.parametrize("n,wave", [(10, 3), (7, 7), (33, 5)])
def test_resumed_file_equals_one_shot(tmp_path, n, wave):
    words, firsts = _case(n, n)
    ref = tmp_path / "ref.boa"
    _one_shot(ref, n, words, firsts)
    out = tmp_path / "out.boa"
    w = C.StreamingWriter(out, _header(n), n)
    stop = min(n, 2 * wave)
    for b in range(0, stop, wave):
        w.append(firsts[b:b + wave], words[b:b + wave])
    w.close()                                     # the run stops between waves
    with pytest.raises(ValueError):
        C.parse(out.read_bytes())                 # not a valid container yet
    w = C.StreamingWriter(out, _header(n), n, resume=True)
    assert w.chunks_done == stop
    for b in range(w.chunks_done, n, wave):
        w.append(firsts[b:b + wave], words[b:b + wave])
    w.finish()
    assert out.read_bytes() == ref.read_bytes()
    p = C.parse(out.read_bytes())
    assert p.first_bytes == firsts and p.lengths == [len(x) for x in words]


def test_resume_rejects_another_header(tmp_path):
    words, firsts = _case(6)
    out = tmp_path / "o.boa"
    w = C.StreamingWriter(out, _header(6), 6)
    w.append(firsts[:3], words[:3])
    w.close()
    with pytest.raises(ValueError):
        C.StreamingWriter(out, _header(7), 7, resume=True)


def test_resume_without_file_starts_fresh(tmp_path):
    words, firsts = _case(4)
    out = tmp_path / "new.boa"
    w = C.StreamingWriter(out, _header(4), 4, resume=True)
    assert w.chunks_done == 0
    w.append(firsts, words)
    w.finish()
    assert C.parse(out.read_bytes()).n_chunks == 4
