"""CPU restatement of the reference's CPU codec loops (TEST / BASELINE ONLY).

Restates compress_CPU / decompress_CPU (codec.py:154-323): for t = 1..L-1 the
fp32 model steps all streams (model.py:124-131), probabilities are softmax of
the logits (codec.py:213,300) and each stream codes one symbol.  The
reference codes with the third-party ``constriction`` coder, which is absent
here; this restatement codes with the C oracle of the reference's own GPU
coder (quantiser + range coder of gpu_range_coder.py:57-210) at PRECISION 24,
or with this build's integer quantiser at PRECISION 16 (``mode="bq"``).
It is the CPU baseline and the end-to-end CPU check, never the product.
"""
from __future__ import annotations

import ctypes

import numpy as np
import torch

from oracle import model_oracle as mo
from oracle import orc


def _setup():
    L = orc.lib()
    P, i = ctypes.c_void_p, ctypes.c_int
    L.orc_enc_state_size.restype = ctypes.c_size_t
    L.orc_dec_state_size.restype = ctypes.c_size_t
    L.orc_enc_init_n.argtypes = [P, i]
    L.orc_encode_step.argtypes = [i, i, i, i, P, P, P, P, P, i]
    L.orc_encode_finish_n.argtypes = [i, P, P, i, P]
    L.orc_dec_init_n.argtypes = [P, i, P, i, P]
    L.orc_decode_step.argtypes = [i, i, i, i, P, P, P, P, i, P, P]
    return L


def _p(a):
    return a.ctypes.data_as(ctypes.c_void_p)


def compress(sd, chunks: list, mode: str = "ref", precision: int | None = None):
    """chunks: list of 1-D uint8 arrays -> (list of u32 arrays, first_bytes, lens)."""
    L = _setup()
    cfg = mo.config_from_state_dict(sd)
    m = orc.MODE_REF if mode == "ref" else orc.MODE_BQ
    P = precision or (24 if mode == "ref" else 16)
    N = len(chunks)
    lens = np.array([len(c) for c in chunks], np.int64)
    maxL = int(lens.max())
    X = np.zeros((N, maxL), np.int64)
    for i, c in enumerate(chunks):
        X[i, :len(c)] = c
    pitch = max(64, 2 * maxL)
    out = np.zeros((N, pitch), np.uint32)
    st = np.zeros(N * L.orc_enc_state_size(), np.uint8)
    L.orc_enc_init_n(_p(st), N)
    state = mo.init_state(cfg, N)
    prev = torch.from_numpy(X[:, 0].copy())
    for t in range(1, maxL):
        active = (lens > t).astype(np.uint8)
        logits, state = mo.step(sd, cfg, prev, state)
        rows = (torch.softmax(logits, -1) if m == orc.MODE_REF else logits).float().numpy()
        syms = X[:, t].astype(np.int32)
        L.orc_encode_step(N, cfg.vocab, P, m, _p(np.ascontiguousarray(rows)), _p(syms), _p(active), _p(st),
                          _p(out), pitch)
        prev = torch.where(torch.from_numpy(active.astype(bool)), torch.from_numpy(X[:, t]), prev)
    sizes = np.zeros(N, np.int32)
    rc = L.orc_encode_finish_n(N, _p(st), _p(out), pitch, _p(sizes))
    if rc:
        raise RuntimeError(f"oracle encoder status {rc}")
    return [out[i, :sizes[i]].copy() for i in range(N)], [int(x) for x in X[:, 0]], [int(x) for x in lens]


def decompress(sd, comp: list, lens: list, first_bytes: list, mode: str = "ref", precision: int | None = None):
    L = _setup()
    cfg = mo.config_from_state_dict(sd)
    m = orc.MODE_REF if mode == "ref" else orc.MODE_BQ
    P = precision or (24 if mode == "ref" else 16)
    N = len(comp)
    lens = np.asarray(lens, np.int64)
    maxL = int(lens.max())
    pitch = max(1, max(len(c) for c in comp))
    words = np.zeros((N, pitch), np.uint32)
    sizes = np.zeros(N, np.int32)
    for i, c in enumerate(comp):
        words[i, :len(c)] = c
        sizes[i] = len(c)
    d = np.zeros(N * L.orc_dec_state_size(), np.uint8)
    L.orc_dec_init_n(_p(d), N, _p(words), pitch, _p(sizes))
    out = np.zeros((N, maxL), np.uint8)
    out[:, 0] = first_bytes
    state = mo.init_state(cfg, N)
    prev = torch.tensor(first_bytes, dtype=torch.int64)
    sym = np.zeros(N, np.int32)
    for t in range(1, maxL):
        active = (lens > t).astype(np.uint8)
        logits, state = mo.step(sd, cfg, prev, state)
        rows = (torch.softmax(logits, -1) if m == orc.MODE_REF else logits).float().numpy()
        rc = L.orc_decode_step(N, cfg.vocab, P, m, _p(np.ascontiguousarray(rows)), _p(active), _p(d), _p(words),
                               pitch, _p(sizes), _p(sym))
        if rc:
            raise RuntimeError(f"oracle decoder status {rc}")
        a = active.astype(bool)
        out[a, t] = sym[a]
        prev = torch.where(torch.from_numpy(a), torch.from_numpy(sym.astype(np.int64)), prev)
    return [out[i, :lens[i]].copy() for i in range(N)]
