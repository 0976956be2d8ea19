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


INT32_MAX = (1 << 31) - 1


@torch.inference_mode()
def encode_device(model, X: torch.Tensor, lens: torch.Tensor, precision: int = PRECISION,
                  pitch_words: int | None = None, workspace: torch.Tensor | None = None,
                  pos_begin: int = 1, pos_end: int | None = None):
    """X [N, maxL] uint8 (device), lens [N] int32 (device) ->
    (words [N, pitch] int32 view of u32, sizes [N] int32), all on the device.

    Codes positions [pos_begin, pos_end) of every chunk (default: all of
    them).  A range that does not start at 1 continues from the recurrent
    state that the previous range left in `workspace` (pass the same one); each
    range is its own bitstream.  Only enqueues work on the current stream:
    device-side errors surface through ``model.native(dev).check()``."""
    dev = X.device
    N, maxL = X.shape
    stop = INT32_MAX if pos_end is None else int(pos_end)
    if pos_begin < 1 or stop <= pos_begin:
        raise ValueError("need 1 <= pos_begin < pos_end")
    if pitch_words is None:
        pitch_words = pitch_words_for(max(min(stop, maxL) - pos_begin, 0) + 1, precision)
    nm = model._native_handle(dev)
    if workspace is None:
        workspace = torch.empty(nm.workspace_bytes(N), dtype=torch.uint8, device=dev)
    words = torch.empty((N, pitch_words), dtype=torch.int32, device=dev)
    sizes = torch.empty((N,), dtype=torch.int32, device=dev)
    X = X.contiguous()
    lens = lens.to(torch.int32).contiguous()
    with torch.cuda.device(dev):
        # byte rows start at position pos_begin - 1 (the byte before the range)
        _n.call("boa_codec_encode_range", nm.h, N, ctypes.c_void_p(X.data_ptr() + (pos_begin - 1)),
                ctypes.c_int64(X.stride(0)), ctypes.c_void_p(lens.data_ptr()), int(pos_begin), int(stop),
                ctypes.c_void_p(words.data_ptr()), int(pitch_words), ctypes.c_void_p(sizes.data_ptr()),
                int(precision), ctypes.c_void_p(workspace.data_ptr()), ctypes.c_size_t(workspace.numel()),
                ctypes.c_void_p(_n.stream_ptr(dev)))
    return words, sizes


@torch.inference_mode()
def decode_device(model, words: torch.Tensor, sizes: torch.Tensor, lens: torch.Tensor, first: torch.Tensor,
                  max_len: int | None = None, precision: int = PRECISION, workspace: torch.Tensor | None = None,
                  pos_begin: int = 1, pos_end: int | None = None, out: torch.Tensor | None = None):
    """words [N, pitch] (device, u32 as int32), sizes [N] int32, lens [N] int32,
    first [N] uint8 -> out [N, maxL] uint8 on the device.

    With a range [pos_begin, pos_end) only those positions are decoded into
    `out` (pass the tensor the earlier ranges filled, and the same workspace);
    the byte before the range is read from ``out[:, pos_begin - 1]``.  Only
    enqueues work on the current stream."""
    dev = words.device
    N, pitch = words.shape
    stop = INT32_MAX if pos_end is None else int(pos_end)
    if pos_begin < 1 or stop <= pos_begin:
        raise ValueError("need 1 <= pos_begin < pos_end")
    nm = model._native_handle(dev)
    if workspace is None:
        workspace = torch.empty(nm.workspace_bytes(N), dtype=torch.uint8, device=dev)
    if out is None:
        if max_len is None:
            max_len = int(lens.max().item())
        out = torch.empty((N, max_len), dtype=torch.uint8, device=dev)
    if pos_begin == 1:
        prev = first.to(torch.uint8).contiguous()
    else:
        if pos_begin - 1 >= out.shape[1]:
            raise ValueError("pos_begin lies beyond the output rows")
        prev = out[:, pos_begin - 1].contiguous()
    words = words.contiguous()
    with torch.cuda.device(dev):
        _n.call("boa_codec_decode_range", nm.h, N, ctypes.c_void_p(words.data_ptr()), int(pitch),
                ctypes.c_void_p(sizes.to(torch.int32).contiguous().data_ptr()),
                ctypes.c_void_p(lens.to(torch.int32).contiguous().data_ptr()), int(pos_begin), int(stop),
                ctypes.c_void_p(prev.data_ptr()), ctypes.c_void_p(out.data_ptr() + (pos_begin - 1)),
                ctypes.c_int64(out.stride(0)), int(precision), ctypes.c_void_p(workspace.data_ptr()),
                ctypes.c_size_t(workspace.numel()), ctypes.c_void_p(_n.stream_ptr(dev)))
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
    model._native_handle(dev).check()
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
    model._native_handle(dev).check()
    return [out_h[i, :full_lens[i]].reshape(1, -1).copy() for i in range(N)]


def compress_CPU(*args, **kwargs):
    raise RuntimeError("boa_b200 has no CPU codec path; run on a CUDA device (sm_100a)")


def decompress_CPU(*args, **kwargs):
    raise RuntimeError("boa_b200 has no CPU codec path; run on a CUDA device (sm_100a)")


class RangeCodec:
    """Codes a fixed batch of chunks in consecutive position ranges, from host
    buffers to host buffers, carrying each side's recurrent model state on the
    device between calls (``boa_codec_encode_range`` /
    ``boa_codec_decode_range``).  For chunks too long to code in one launch
    (each call is a bounded piece of work) and for streaming producers and
    consumers.  No reference counterpart: the reference loops code a chunk
    from its first byte to its last (codec.py:56-79,125-143).

    ``encode(seg, a, b)`` takes ``seg`` [N, b - a + 1] uint8 (positions
    [a - 1, b) of every chunk, zero padded past a chunk's end; pinned host
    memory copies asynchronously) and returns (words [N, pitch] uint32,
    sizes [N] int32) as numpy arrays; ``decode(words, sizes, a, b)`` returns
    positions [a, b) of every chunk as [N, b - a] uint8.  Ranges must be
    coded in order on each side; every range is its own bitstream."""

    def __init__(self, model, lens, first_bytes, device="cuda", precision: int = PRECISION):
        self.dev = _device(device)
        self.model = model
        self.precision = precision
        self.lens_h = np.asarray(lens, dtype=np.int32)
        self.N = len(self.lens_h)
        self.nm = model._native_handle(self.dev)
        self.lens = torch.from_numpy(self.lens_h).to(self.dev)
        self.first = torch.tensor([int(b) & 0xFF for b in first_bytes], dtype=torch.uint8).to(self.dev)
        nb = self.nm.workspace_bytes(self.N)
        self.ws_enc = torch.empty(nb, dtype=torch.uint8, device=self.dev)
        self.ws_dec = torch.empty(nb, dtype=torch.uint8, device=self.dev)
        self.prev_dec = self.first.clone()

    @torch.inference_mode()
    def encode(self, seg, pos_begin: int, pos_end: int):
        seg_t = torch.as_tensor(seg)
        X = seg_t.to(self.dev, non_blocking=True)
        words, sizes = _encode_range_rows(self, X, pos_begin, pos_end)
        w_h = words.cpu().numpy().view(np.uint32)
        s_h = sizes.cpu().numpy()
        self.nm.check()
        return w_h, s_h

    @torch.inference_mode()
    def decode(self, words, sizes, pos_begin: int, pos_end: int):
        w = torch.from_numpy(np.ascontiguousarray(words).view(np.int32)).to(self.dev, non_blocking=True)
        s = torch.from_numpy(np.ascontiguousarray(sizes, dtype=np.int32)).to(self.dev, non_blocking=True)
        out = torch.zeros((self.N, pos_end - pos_begin + 1), dtype=torch.uint8, device=self.dev)
        prev = self.first if pos_begin == 1 else self.prev_dec
        with torch.cuda.device(self.dev):
            _n.call("boa_codec_decode_range", self.nm.h, self.N, ctypes.c_void_p(w.data_ptr()), int(w.shape[1]),
                    ctypes.c_void_p(s.data_ptr()), ctypes.c_void_p(self.lens.data_ptr()), int(pos_begin),
                    int(pos_end), ctypes.c_void_p(prev.data_ptr()), ctypes.c_void_p(out.data_ptr()),
                    ctypes.c_int64(out.stride(0)), int(self.precision), ctypes.c_void_p(self.ws_dec.data_ptr()),
                    ctypes.c_size_t(self.ws_dec.numel()), ctypes.c_void_p(_n.stream_ptr(self.dev)))
        # the byte before the next range: the last position of this one each chunk reached
        last = torch.clamp(torch.minimum(self.lens, torch.tensor(pos_end, device=self.dev)) - pos_begin, min=0)
        self.prev_dec = torch.where(self.lens > pos_begin - 1, out.gather(1, last.long()[:, None])[:, 0], prev)
        out_h = out[:, 1:].cpu().numpy()
        self.nm.check()
        return out_h


def _encode_range_rows(rc: "RangeCodec", X: torch.Tensor, pos_begin: int, pos_end: int):
    """Encode positions [pos_begin, pos_end) from rows that start at position
    pos_begin - 1 (X [N, pos_end - pos_begin + 1] on the device)."""
    N = rc.N
    pitch = pitch_words_for(pos_end - pos_begin + 1, rc.precision)
    words = torch.empty((N, pitch), dtype=torch.int32, device=rc.dev)
    sizes = torch.empty((N,), dtype=torch.int32, device=rc.dev)
    X = X.contiguous()
    with torch.cuda.device(rc.dev):
        _n.call("boa_codec_encode_range", rc.nm.h, N, ctypes.c_void_p(X.data_ptr()), ctypes.c_int64(X.stride(0)),
                ctypes.c_void_p(rc.lens.data_ptr()), int(pos_begin), int(pos_end),
                ctypes.c_void_p(words.data_ptr()), int(pitch), ctypes.c_void_p(sizes.data_ptr()),
                int(rc.precision), ctypes.c_void_p(rc.ws_enc.data_ptr()), ctypes.c_size_t(rc.ws_enc.numel()),
                ctypes.c_void_p(_n.stream_ptr(rc.dev)))
    return words, sizes
