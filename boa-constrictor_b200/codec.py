"""Drop-in for the reference ``codec.py`` (codec.py:11-151).

``compress_GPU`` / ``decompress_GPU`` keep the reference signatures and
return types, but the per-byte loop (model step -> softmax -> coder step, one
launch each plus host syncs per byte in the reference, codec.py:56-79 and
125-143) runs as one persistent sm_100a kernel per wave of chunks
(``boa_codec_encode`` / ``boa_codec_decode`` in libboa_b200.so).  Tables are
built by this build's integer quantiser at ``PRECISION`` (16 by default), so the
streams are not interchangeable with the reference's float-quantised ones; the
container records which was used (see boa_b200.container).

``compress_CPU`` / ``decompress_CPU`` exist only to fail loudly: this build has
no CPU execution path.

The ``encode_device`` / ``decode_device`` helpers take and return device
tensors (no host copies) for callers that keep data resident in HBM.
"""
from __future__ import annotations

import ctypes

import numpy as np
import torch

from boa_b200 import _native as _n

IS_CUDA = torch.cuda.is_available()
PRECISION = 16


def pitch_words_for(max_len: int, precision: int = PRECISION) -> int:
    """Words per stream that always suffice: every coded byte costs at most
    `precision` bits, plus the flush (2 words) and a pending carry run."""
    return max(8, (max(max_len - 1, 0) * precision + 31) // 32 + 6)


def _ws(model, dev, n):
    nm = model._native_handle(dev)
    return nm, torch.empty(nm.workspace_bytes(n), dtype=torch.uint8, device=dev)


@torch.inference_mode()
def encode_device(model, X: torch.Tensor, lens: torch.Tensor, precision: int = PRECISION,
                  pitch_words: int | None = None, workspace: torch.Tensor | None = None):
    """X [N, maxL] uint8 (device), lens [N] int32 (device) ->
    (words [N, pitch] int32 view of u32, sizes [N] int32), all on the device."""
    dev = X.device
    N, maxL = X.shape
    if pitch_words is None:
        pitch_words = pitch_words_for(maxL, precision)
    nm = model._native_handle(dev)
    if workspace is None:
        workspace = torch.empty(nm.workspace_bytes(N), dtype=torch.uint8, device=dev)
    words = torch.empty((N, pitch_words), dtype=torch.int32, device=dev)
    sizes = torch.empty((N,), dtype=torch.int32, device=dev)
    X = X.contiguous()
    lens = lens.to(torch.int32).contiguous()
    with torch.cuda.device(dev):
        _n.call("boa_codec_encode", nm.h, N, ctypes.c_void_p(X.data_ptr()), ctypes.c_int64(X.stride(0)),
                ctypes.c_void_p(lens.data_ptr()), ctypes.c_void_p(words.data_ptr()), int(pitch_words),
                ctypes.c_void_p(sizes.data_ptr()), int(precision), ctypes.c_void_p(workspace.data_ptr()),
                ctypes.c_size_t(workspace.numel()), ctypes.c_void_p(_n.stream_ptr(dev)))
    return words, sizes


@torch.inference_mode()
def decode_device(model, words: torch.Tensor, sizes: torch.Tensor, lens: torch.Tensor, first: torch.Tensor,
                  max_len: int | None = None, precision: int = PRECISION, workspace: torch.Tensor | None = None):
    """words [N, pitch] (device, u32 as int32), sizes [N] int32, lens [N] int32,
    first [N] uint8 -> out [N, maxL] uint8 on the device."""
    dev = words.device
    N, pitch = words.shape
    if max_len is None:
        max_len = int(lens.max().item())
    nm = model._native_handle(dev)
    if workspace is None:
        workspace = torch.empty(nm.workspace_bytes(N), dtype=torch.uint8, device=dev)
    out = torch.empty((N, max_len), dtype=torch.uint8, device=dev)
    words = words.contiguous()
    with torch.cuda.device(dev):
        _n.call("boa_codec_decode", nm.h, N, ctypes.c_void_p(words.data_ptr()), int(pitch),
                ctypes.c_void_p(sizes.to(torch.int32).contiguous().data_ptr()),
                ctypes.c_void_p(lens.to(torch.int32).contiguous().data_ptr()),
                ctypes.c_void_p(first.to(torch.uint8).contiguous().data_ptr()),
                ctypes.c_void_p(out.data_ptr()), ctypes.c_int64(out.stride(0)), int(precision),
                ctypes.c_void_p(workspace.data_ptr()), ctypes.c_size_t(workspace.numel()),
                ctypes.c_void_p(_n.stream_ptr(dev)))
    return out


def _device(device):
    d = torch.device(device)
    if d.type != "cuda":
        raise RuntimeError("boa_b200 codec runs on CUDA only")
    if d.index is None:
        d = torch.device("cuda", torch.cuda.current_device())
    return d


@torch.inference_mode()
def compress_GPU(model, x_list: list, device="cuda", progress=True, num_workers: int = 8,
                 precision: int = PRECISION):
    """x_list: N tensors [1, L_i] of bytes -> (list[np.uint32 array], first_bytes, lengths)
    (codec.py:11-86)."""
    dev = _device(device)
    N = len(x_list)
    assert N >= 1, "Need at least one chunk."
    Ls = []
    for i, x in enumerate(x_list):
        assert x.ndim == 2 and x.shape[0] == 1, f"Chunk {i} must be [1, L_i]"
        assert x.shape[1] >= 1, f"Chunk {i} must have length >= 1"
        Ls.append(int(x.shape[1]))
    maxL = max(Ls)
    host = torch.zeros((N, maxL), dtype=torch.uint8, pin_memory=True)
    for i, x in enumerate(x_list):
        host[i, :Ls[i]] = x[0].to(torch.uint8)
    first_bytes = host[:, 0].tolist()
    X = host.to(dev, non_blocking=True)
    lens = torch.tensor(Ls, dtype=torch.int32).to(dev, non_blocking=True)
    words, sizes = encode_device(model, X, lens, precision=precision)
    sizes_h = sizes.cpu().numpy()
    words_h = words.cpu().numpy().view(np.uint32)
    out = [words_h[i, :int(sizes_h[i])].copy() for i in range(N)]
    return out, first_bytes, Ls


@torch.inference_mode()
def decompress_GPU(model, compressed_list, full_lens: list, first_bytes: list, device="cuda", progress=True,
                   num_workers: int = 8, precision: int = PRECISION):
    """-> list of N uint8 arrays shaped (1, L_i) (codec.py:89-151)."""
    dev = _device(device)
    N = len(compressed_list)
    assert N >= 1 and len(full_lens) == N and len(first_bytes) == N
    assert all(L >= 1 for L in full_lens)
    maxL = max(full_lens)
    comp = [np.asarray(c).view(np.uint32) if np.asarray(c).dtype != np.uint32 else np.asarray(c)
            for c in compressed_list]
    pitch = max(pitch_words_for(maxL, precision), max(c.shape[0] for c in comp))
    host = np.zeros((N, pitch), dtype=np.uint32)
    sizes = np.zeros(N, dtype=np.int32)
    for i, c in enumerate(comp):
        host[i, :c.shape[0]] = c
        sizes[i] = c.shape[0]
    words = torch.from_numpy(host.view(np.int32)).pin_memory().to(dev, non_blocking=True)
    sizes_d = torch.from_numpy(sizes).to(dev)
    lens_d = torch.tensor(list(full_lens), dtype=torch.int32).to(dev)
    first_d = torch.tensor([int(b) & 0xFF for b in first_bytes], dtype=torch.uint8).to(dev)
    out = decode_device(model, words, sizes_d, lens_d, first_d, max_len=maxL, precision=precision)
    out_h = out.cpu().numpy()
    return [out_h[i, :full_lens[i]].reshape(1, -1).copy() for i in range(N)]


def compress_CPU(*args, **kwargs):
    raise RuntimeError("boa_b200 has no CPU codec path; run on a CUDA device (sm_100a)")


def decompress_CPU(*args, **kwargs):
    raise RuntimeError("boa_b200 has no CPU codec path; run on a CUDA device (sm_100a)")
