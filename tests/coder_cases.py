"""Seeded coder test cases shared by the CPU and GPU coder tests."""
import numpy as np

from oracle import orc


def make_case(seed: int, N: int, T: int, K: int, mode: int, precision: int, sigma: float = 3.0,
              skew: bool = False):
    """rows [N,T,K] f32 (probs for MODE_REF, logits for MODE_BQ), syms [N,T] drawn
    from each row's own quantised table, ragged counts [N] (incl. 0 and T)."""
    rng = np.random.default_rng(seed)
    logits = rng.normal(0.0, sigma, (N, T, K)).astype(np.float32)
    if skew:
        # near-deterministic rows: one dominant entry, the rest tiny, forcing
        # both long no-renorm runs and freq-1 symbols (long pending-carry runs)
        dom = rng.integers(0, K, (N, T))
        logits = rng.normal(-30.0, 1.0, (N, T, K)).astype(np.float32)
        np.put_along_axis(logits, dom[..., None], 30.0, axis=-1)
    if mode == orc.MODE_REF:
        p = np.exp(logits.astype(np.float64) - logits.max(-1, keepdims=True))
        rows = (p / p.sum(-1, keepdims=True)).astype(np.float32)
    else:
        rows = logits
    cdfs = orc.cdf_rows(rows, mode, precision)
    u = rng.integers(0, 1 << precision, (N, T))
    syms = np.empty((N, T), dtype=np.int32)
    for i in range(N):
        for t in range(T):
            syms[i, t] = np.searchsorted(cdfs[i, t], u[i, t], side="right") - 1
    if skew:
        # force some freq-1 (least probable) symbols into the stream
        flip = rng.random((N, T)) < 0.2
        syms = np.where(flip, rng.integers(0, K, (N, T)), syms).astype(np.int32)
    counts = rng.integers(0, T + 1, N).astype(np.int32)
    counts[0] = T
    if N > 1:
        counts[1] = 0
    return rows, syms, counts
