"""Seeded synthetic inputs standing in for the reference's datasets.

The reference experiments compress CMS/ATLAS/HepMC/CAMEL/CFD files that are
not available here; these generators produce data with the shapes, sizes and
value distributions the benchmark configurations specify.  All draws use
numpy's PCG64 (``np.random.default_rng``) in the order written below, so the
bytes are a pure function of the seed and size.

config 1  ``markov``   order-1 Markov bytes, transition rows ~ Dirichlet(0.05),
                       first byte uniform (seed 1, 1 MiB)
config 2/3 ``hep``     event records: i32 LE id (from 0), u16 n ~ Poisson(40),
                       n x (f32 pt ~ LogNormal(1,1), f32 eta ~ N(0, 2),
                       f32 phi ~ U(-pi, pi), i16 pdgId from {+-11, +-13, 22,
                       +-211, 2112} w.p. 0.1/0.1/0.3/0.4/0.1, sign uniform for
                       the charged ones), truncated to the size (seed 2, 64 MiB)
config 4  ``mixed``    hep records (seed 3) for size - 128 MiB, then a float64
                       256^3 field: sum of 8 random sinusoids + N(0, 1e-3),
                       row-major (field rng seeded with (3, 1))
"""
from __future__ import annotations

import math

import numpy as np

MiB = 1 << 20

_PARTICLE = np.dtype([("pt", "<f4"), ("eta", "<f4"), ("phi", "<f4"), ("pdg", "<i2")])   # 14 bytes
_EVENT = np.dtype([("id", "<i4"), ("n", "<u2")])                                            # 6 bytes


def markov(size: int = MiB, seed: int = 1, alpha: float = 0.05) -> bytes:
    rng = np.random.default_rng(seed)
    P = rng.dirichlet(np.full(256, alpha), size=256)
    cum = np.cumsum(P, axis=1)
    cum[:, -1] = 1.0
    x0 = int(rng.integers(0, 256))
    u = rng.random(size - 1)
    out = np.empty(size, dtype=np.uint8)
    out[0] = x0
    # vectorised over 256 "current byte" classes would need the previous byte;
    # walk the chain in blocks with a per-row searchsorted
    cur = x0
    rows = [cum[i] for i in range(256)]
    ss = np.searchsorted
    for t in range(1, size):
        cur = int(ss(rows[cur], u[t - 1], side="right"))
        if cur > 255:
            cur = 255
        out[t] = cur
    return out.tobytes()


def hep_records(size: int, seed: int = 2) -> bytes:
    rng = np.random.default_rng(seed)
    mean_event = _EVENT.itemsize + 40 * _PARTICLE.itemsize
    n_events = int(size / mean_event * 1.05) + 64
    n = rng.poisson(40, size=n_events).astype(np.int64)
    P = int(n.sum())
    pt = rng.lognormal(1.0, 1.0, P).astype(np.float32)
    eta = rng.normal(0.0, 2.0, P).astype(np.float32)
    phi = rng.uniform(-math.pi, math.pi, P).astype(np.float32)
    kinds = rng.choice(5, size=P, p=[0.1, 0.1, 0.3, 0.4, 0.1])
    sign = np.where(rng.integers(0, 2, P) == 0, 1, -1)
    base = np.array([11, 13, 22, 211, 2112], dtype=np.int64)[kinds]
    charged = np.isin(kinds, [0, 1, 3])
    pdg = np.where(charged, base * sign, base).astype(np.int16)
    ev = np.empty(n_events, dtype=_EVENT)
    ev["id"] = np.arange(n_events, dtype=np.int64).astype(np.int32)
    ev["n"] = n.astype(np.uint16)
    evb = ev.view(np.uint8).reshape(n_events, _EVENT.itemsize)
    parts = np.empty(P, dtype=_PARTICLE)
    parts["pt"], parts["eta"], parts["phi"], parts["pdg"] = pt, eta, phi, pdg
    pb = parts.view(np.uint8)
    bounds = np.zeros(n_events + 1, dtype=np.int64)
    bounds[1:] = np.cumsum(n) * _PARTICLE.itemsize
    pieces = []
    for e in range(n_events):        # header, then that event's particles
        pieces.append(evb[e])
        pieces.append(pb[bounds[e]:bounds[e + 1]])
    buf = np.concatenate(pieces)
    if buf.size < size:
        raise RuntimeError("hep_records: event budget too small")
    return buf[:size].tobytes()


def cfd_field(n: int = 256, seed=(3, 1)) -> bytes:
    rng = np.random.default_rng(seed)
    amp = rng.uniform(0.5, 1.5, 8)
    kv = rng.integers(1, 9, size=(8, 3))
    ph = rng.uniform(0.0, 2 * math.pi, 8)
    g = np.arange(n, dtype=np.float64) * (2 * math.pi / n)
    f = np.zeros((n, n, n), dtype=np.float64)
    for i in range(8):
        # separable phase: k.x = kx*x + ky*y + kz*z
        a = kv[i, 0] * g[:, None, None] + kv[i, 1] * g[None, :, None] + kv[i, 2] * g[None, None, :]
        f += amp[i] * np.sin(a + ph[i])
    f += rng.normal(0.0, 1e-3, f.shape)
    return f.astype("<f8").tobytes()


def mixed(size: int = 1 << 30, seed: int = 3) -> bytes:
    field = cfd_field(256, (seed, 1))
    return hep_records(size - len(field), seed) + field


def config_data(config: int, size: int | None = None) -> bytes:
    if config == 1:
        return markov(size or MiB, 1)
    if config in (2, 3):
        return hep_records(size or 64 * MiB, 2)
    if config == 4:
        return mixed(size or (1 << 30), 3)
    raise ValueError(f"no synthetic data for config {config}")
