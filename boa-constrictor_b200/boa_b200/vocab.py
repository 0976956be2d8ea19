"""Vocabulary-subset remapping (main.py:221-239, 462-478, 508-516).

A model trained on data that uses only some byte values has vocab_size equal
to the number of distinct bytes.  Bytes map to indices 0 .. vocab_size - 1 in
increasing byte order before compression (the codec then codes indices with a
vocab_size-way table) and map back after decompression."""
from __future__ import annotations

import numpy as np


def vocab_subset(train_bytes):
    """(vocab_size, lookup[256] byte -> index, inverse[256] index -> byte, unique bytes)."""
    arr = np.frombuffer(bytes(train_bytes), dtype=np.uint8)
    unique = np.unique(arr)
    lookup = np.zeros(256, dtype=np.uint8)
    lookup[unique] = np.arange(len(unique), dtype=np.uint8)
    inverse = np.zeros(256, dtype=np.uint8)
    inverse[:len(unique)] = unique
    return int(len(unique)), lookup, inverse, unique


def remap(data, lookup, unique) -> bytes:
    """Bytes -> indices.  Raises ValueError for a byte value the training data
    did not contain (the reference prints an error and skips compression)."""
    arr = np.frombuffer(bytes(data), dtype=np.uint8)
    seen = np.zeros(256, dtype=bool)
    seen[unique] = True
    if not seen[arr].all():
        raise ValueError("compression input contains bytes not seen in the training data")
    return lookup[arr].tobytes()


def unmap(data, inverse) -> bytes:
    """Indices -> bytes."""
    return inverse[np.frombuffer(bytes(data), dtype=np.uint8)].tobytes()
