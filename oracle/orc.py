"""ctypes wrapper around ``oracle/liborc.so`` (the C restatement of the coder).

TEST INFRASTRUCTURE ONLY.  Mirrors the reference coder semantics of
``gpu_range_coder.py:57-210`` (see ``oracle/rc_oracle.c`` for line cites).
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liborc.so")
_lib = None

MODE_REF = 0   # fp32 probabilities, reference float quantiser (build_cdf_fast)
MODE_BQ = 1    # fp32 logits, integer quantiser of this build


def build() -> str:
    src = os.path.join(_HERE, "rc_oracle.c")
    if (not os.path.exists(_LIB_PATH)) or os.path.getmtime(_LIB_PATH) < os.path.getmtime(src):
        subprocess.check_call(["make", "-s", "-C", _HERE, "liborc.so"])
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        build()
        L = ctypes.CDLL(_LIB_PATH)
        P = ctypes.c_void_p
        i = ctypes.c_int
        L.orc_cdf_ref.argtypes = [P, i, i, P]
        L.orc_cdf_bq.argtypes = [P, i, i, P]
        L.orc_freq_bq.argtypes = [P, i, i, P]
        L.orc_exp_det.argtypes = [ctypes.c_float]
        L.orc_exp_det.restype = ctypes.c_float
        L.orc_encode_batch.argtypes = [i, i, i, i, i, P, P, P, P, i, P]
        L.orc_decode_batch.argtypes = [i, i, i, i, i, P, P, i, P, P, P]
        L.orc_encode_cdfs.argtypes = [i, i, i, i, P, P, P, P, i, P]
        _lib = L
    return _lib


def _p(a: np.ndarray):
    return a.ctypes.data_as(ctypes.c_void_p)


def cdf_ref(probs: np.ndarray, precision: int = 24) -> np.ndarray:
    probs = np.ascontiguousarray(probs, dtype=np.float32)
    K = probs.shape[-1]
    out = np.empty(K + 1, dtype=np.uint32)
    lib().orc_cdf_ref(_p(probs), K, precision, _p(out))
    return out


def cdf_bq(logits: np.ndarray, precision: int = 16) -> np.ndarray:
    logits = np.ascontiguousarray(logits, dtype=np.float32)
    K = logits.shape[-1]
    out = np.empty(K + 1, dtype=np.uint32)
    rc = lib().orc_cdf_bq(_p(logits), K, precision, _p(out))
    if rc:
        raise ValueError(f"orc_cdf_bq rc={rc}")
    return out


def cdf_rows(rows: np.ndarray, mode: int, precision: int) -> np.ndarray:
    """Quantise every row of an [..., K] array into [..., K+1] CDFs."""
    rows = np.ascontiguousarray(rows, dtype=np.float32)
    K = rows.shape[-1]
    flat = rows.reshape(-1, K)
    out = np.empty((flat.shape[0], K + 1), dtype=np.uint32)
    f = cdf_ref if mode == MODE_REF else cdf_bq
    for r in range(flat.shape[0]):
        out[r] = f(flat[r], precision)
    return out.reshape(rows.shape[:-1] + (K + 1,))


def exp_det(x: float) -> float:
    return float(lib().orc_exp_det(ctypes.c_float(x)))


def encode(rows: np.ndarray, syms: np.ndarray, counts, precision: int, mode: int,
           pitch: int):
    """rows [N,T,K] f32, syms [N,T] i32 -> (words [N,pitch] u32, sizes [N] i32, status)."""
    rows = np.ascontiguousarray(rows, dtype=np.float32)
    syms = np.ascontiguousarray(syms, dtype=np.int32)
    N, T, K = rows.shape
    counts = np.ascontiguousarray(np.asarray(counts, dtype=np.int32))
    out = np.zeros((N, pitch), dtype=np.uint32)
    sizes = np.zeros(N, dtype=np.int32)
    st = lib().orc_encode_batch(N, T, K, precision, mode, _p(rows), _p(syms), _p(counts),
                                _p(out), pitch, _p(sizes))
    return out, sizes, st


def decode(rows: np.ndarray, words: np.ndarray, sizes, counts, precision: int, mode: int):
    rows = np.ascontiguousarray(rows, dtype=np.float32)
    N, T, K = rows.shape
    words = np.ascontiguousarray(words, dtype=np.uint32)
    sizes = np.ascontiguousarray(np.asarray(sizes, dtype=np.int32))
    counts = np.ascontiguousarray(np.asarray(counts, dtype=np.int32))
    out = np.full((N, T), -1, dtype=np.int32)
    st = lib().orc_decode_batch(N, T, K, precision, mode, _p(rows), _p(words), words.shape[1],
                                _p(sizes), _p(counts), _p(out))
    if st:
        raise ValueError(f"orc_decode_batch rc={st}")
    return out


def encode_cdfs(cdfs: np.ndarray, syms: np.ndarray, counts, precision: int, pitch: int):
    cdfs = np.ascontiguousarray(cdfs, dtype=np.uint32)
    syms = np.ascontiguousarray(syms, dtype=np.int32)
    N, T, K1 = cdfs.shape
    counts = np.ascontiguousarray(np.asarray(counts, dtype=np.int32))
    out = np.zeros((N, pitch), dtype=np.uint32)
    sizes = np.zeros(N, dtype=np.int32)
    st = lib().orc_encode_cdfs(N, T, K1 - 1, precision, _p(cdfs), _p(syms), _p(counts),
                               _p(out), pitch, _p(sizes))
    return out, sizes, st
