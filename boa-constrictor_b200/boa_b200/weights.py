"""Weight layout helpers.

``flatten_state_dict`` writes the fp32 vector in exactly the order of the
reference exporter ``portability_solved_cpp/convert_boa_weights.py:16-135``:
embedding; per block ln1.{w,b}, mamba.in_proj.weight, in_proj.bias (zeros when
absent), conv1d.weight, conv1d.bias, x_proj.weight, dt_proj.{weight,bias},
A_log, D, out_proj.weight, out_proj.bias (zeros when absent), ln2.{w,b},
ff.0.{w,b}, ff.2.{w,b}; then head.0.{w,b}, head.2.{w,b}.  ``boa_model_create``
consumes this vector, and ``write_bin`` / ``read_bin`` produce / parse the same
``.bin`` files the reference exporter writes.
"""
from __future__ import annotations

import math

import numpy as np


def _np(t):
    import torch
    if isinstance(t, torch.Tensor):
        return t.detach().to("cpu", torch.float32).contiguous().numpy().ravel()
    return np.asarray(t, dtype=np.float32).ravel()


def n_layers_of(sd) -> int:
    n = 0
    while f"blocks.{n}.ln1.weight" in sd:
        n += 1
    return n


def flatten_state_dict(sd) -> np.ndarray:
    parts = [_np(sd["embedding.weight"])]
    for i in range(n_layers_of(sd)):
        p = f"blocks.{i}."
        m = p + "mamba."
        parts += [_np(sd[p + "ln1.weight"]), _np(sd[p + "ln1.bias"])]
        w_in = sd[m + "in_proj.weight"]
        parts.append(_np(w_in))
        parts.append(_np(sd[m + "in_proj.bias"]) if m + "in_proj.bias" in sd
                     else np.zeros(w_in.shape[0], np.float32))
        parts.append(_np(sd[m + "conv1d.weight"]))
        if m + "conv1d.bias" in sd:
            parts.append(_np(sd[m + "conv1d.bias"]))
        parts += [_np(sd[m + "x_proj.weight"]), _np(sd[m + "dt_proj.weight"]), _np(sd[m + "dt_proj.bias"]),
                  _np(sd[m + "A_log"]), _np(sd[m + "D"])]
        w_out = sd[m + "out_proj.weight"]
        parts.append(_np(w_out))
        parts.append(_np(sd[m + "out_proj.bias"]) if m + "out_proj.bias" in sd
                     else np.zeros(w_out.shape[0], np.float32))
        parts += [_np(sd[p + "ln2.weight"]), _np(sd[p + "ln2.bias"]),
                  _np(sd[p + "ff.0.weight"]), _np(sd[p + "ff.0.bias"]),
                  _np(sd[p + "ff.2.weight"]), _np(sd[p + "ff.2.bias"])]
    parts += [_np(sd["head.0.weight"]), _np(sd["head.0.bias"]),
              _np(sd["head.2.weight"]), _np(sd["head.2.bias"])]
    return np.ascontiguousarray(np.concatenate(parts).astype(np.float32))


def flat_size(d_model: int, n_layers: int, vocab: int = 256) -> int:
    d, E, R, F = d_model, 2 * d_model, math.ceil(d_model / 16), 4 * d_model
    per = (2 * d + 2 * E * d + 2 * E + 4 * E + E + (R + 32) * E + E * R + E + 16 * E + E
           + d * E + d + 2 * d + F * d + F + d * F + d)
    return vocab * d + n_layers * per + d * d + d + vocab * d + vocab


def write_bin(sd, path: str) -> None:
    """Same bytes as convert_boa_weights.py:22-133 (fp32, no header)."""
    flatten_state_dict(sd).tofile(path)


def read_bin(path: str) -> np.ndarray:
    return np.fromfile(path, dtype=np.float32)
