"""Vocabulary-subset remap (main.py:221-239, 462-478, 508-516): host mapping
on CPU, and a full BoaFile round trip with a vocab-37 model on the GPU."""
import numpy as np
import pytest
import torch

from boa_b200.vocab import remap, unmap, vocab_subset


def _data(seed, n, values):
    rng = np.random.default_rng(seed)
    return rng.choice(np.asarray(values, np.uint8), n).tobytes()


def test_remap_round_trip_and_order():
    values = [3, 7, 9, 200, 255, 0]
    train = _data(0, 5000, values)
    v, lookup, inverse, unique = vocab_subset(train)
    assert v == len(values)
    assert list(unique) == sorted(values)
    assert lookup[0] == 0 and lookup[255] == v - 1          # indices follow byte order
    data = _data(1, 777, values)
    idx = remap(data, lookup, unique)
    assert max(idx) < v
    assert unmap(idx, inverse) == data


def test_unseen_byte_is_rejected():
    v, lookup, inverse, unique = vocab_subset(_data(2, 100, [1, 2, 3]))
    with pytest.raises(ValueError):
        remap(bytes([1, 2, 4]), lookup, unique)


@pytest.mark.gpu
def test_boafile_round_trip_with_vocab_subset(tmp_path):
    from boa import BOA
    from model import seeded_model
    values = list(range(40, 77))                              # 37 byte values
    train = _data(3, 10000, values)
    v, lookup, inverse, unique = vocab_subset(train)
    data = _data(4, 30000, values)
    src = tmp_path / "remapped.bin"
    src.write_bytes(remap(data, lookup, unique))
    m = seeded_model(64, 2, vocab_size=v)
    out = tmp_path / "x.boa"
    BOA("cuda", str(out), m).compress(str(src), chunks_count=7, progress=False)
    got = BOA("cuda", str(out), m).decompress(progress=False)
    assert unmap(got, inverse) == data
    # bytes outside the model's vocabulary are an error, not a silent corruption
    import codec
    from boa_b200._native import BoaError
    bad = [torch.from_numpy(np.frombuffer(data[:50], np.uint8).copy()[None, :])]
    with pytest.raises(BoaError):
        codec.compress_GPU(m, bad)
