"""Drop-in for the reference ``gpu_range_coder`` module (gpu_range_coder.py).

``gpu.queue.RangeCoderBatch`` keeps the reference's constructor and method
names (gpu_range_coder.py:488-550) but runs on libboa_b200.so (sm_100a,
prebuilt in-tree, no build at import time).  Defaults reproduce the reference
bitstream exactly: PRECISION 24 and the reference float quantiser
(build_cdf_fast, gpu_range_coder.py:57-79) applied to fp32 probabilities.
Optional keyword ``quantiser="bq"`` selects this build's integer quantiser,
which takes fp32 logits instead and is the one the fused codec uses.

Work is issued on torch's current CUDA stream; methods that return host data
synchronise that stream only.
"""
from __future__ import annotations

import ctypes

import numpy as np

from boa_b200 import _native as _n

__all__ = ["stream", "gpu"]

PRECISION = 24


def _dev_index(t) -> int:
    return t.device.index if t.device.index is not None else 0


class _BatchCore:
    """Owns one native boa_rc_batch handle."""

    def __init__(self, N: int, K: int, pitch_words: int, precision: int, quantiser: int, device: int):
        _n.require_cuda()
        h = ctypes.c_void_p()
        _n.call("boa_rc_create", ctypes.byref(h), int(N), int(K), int(pitch_words), int(precision),
                int(quantiser), int(device))
        self.h = h
        self.N, self.K, self.pitch, self.precision, self.quantiser = N, K, pitch_words, precision, quantiser
        self.device = device

    def close(self):
        if getattr(self, "h", None) is not None and self.h.value:
            _n.load().boa_rc_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class gpu:
    class queue:
        class RangeCoderBatch:
            """Batched GPU range coder, one stream per chunk (gpu_range_coder.py:488-550)."""

            def __init__(self, N: int, K: int, maxL: int, pitch_bytes: int | None = None, *,
                         precision: int = PRECISION, quantiser: str = "ref", device: int | None = None):
                import torch
                if pitch_bytes is None:
                    pitch_bytes = max(256, maxL * 8)
                self.N, self.K, self.maxL = int(N), int(K), int(maxL)
                pitch_words = (int(pitch_bytes) + 3) // 4
                q = {"ref": _n.BOA_QUANT_REF, "bq": _n.BOA_QUANT_BQ}[quantiser]
                if device is None:
                    _n.require_cuda()
                    device = torch.cuda.current_device()
                self._core = _BatchCore(self.N, self.K, pitch_words, int(precision), q, int(device))
                self.pitch_words = pitch_words

            # -- host <-> device --------------------------------------------------
            def load_compressed_list(self, compressed_list):
                if len(compressed_list) != self.N:
                    raise RuntimeError("compressed_list length must equal N")
                buf = np.zeros((self.N, self.pitch_words), dtype=np.uint32)
                sizes = np.zeros(self.N, dtype=np.int32)
                for i, c in enumerate(compressed_list):
                    a = np.asarray(c)
                    if a.ndim != 1 or a.dtype.itemsize != 4 or a.dtype.kind != "u":
                        raise RuntimeError("Each compressed item must be uint32[?]")
                    if a.shape[0] > self.pitch_words:
                        raise RuntimeError("Compressed stream exceeds pitch; increase pitch")
                    buf[i, :a.shape[0]] = a
                    sizes[i] = a.shape[0]
                _n.call("boa_rc_load", self._core.h, buf.ctypes.data_as(ctypes.c_void_p),
                        sizes.ctypes.data_as(ctypes.c_void_p), ctypes.c_void_p(_n.stream_ptr()))

            def set_sizes_list(self, sizes_list):
                if len(sizes_list) != self.N:
                    raise RuntimeError("sizes_list length must equal N")
                s = np.ascontiguousarray(np.asarray(sizes_list, dtype=np.int32))
                _n.call("boa_rc_set_sizes", self._core.h, s.ctypes.data_as(ctypes.c_void_p),
                        ctypes.c_void_p(_n.stream_ptr()))

            def get_sizes_list(self):
                s = np.zeros(self.N, dtype=np.int32)
                _n.call("boa_rc_get_sizes", self._core.h, s.ctypes.data_as(ctypes.c_void_p),
                        ctypes.c_void_p(_n.stream_ptr()))
                return [int(x) for x in s]

            def get_compressed_list(self):
                sizes = np.zeros(self.N, dtype=np.int32)
                _n.call("boa_rc_get_sizes", self._core.h, sizes.ctypes.data_as(ctypes.c_void_p),
                        ctypes.c_void_p(_n.stream_ptr()))
                buf = np.zeros((self.N, self.pitch_words), dtype=np.uint32)
                _n.call("boa_rc_get_words", self._core.h, buf.ctypes.data_as(ctypes.c_void_p),
                        ctypes.c_void_p(_n.stream_ptr()))
                return [buf[i, :max(0, int(sizes[i]))].copy() for i in range(self.N)]

            # -- coding -----------------------------------------------------------
            def _mask_ptr(self, mask):
                import torch
                if mask is None:
                    return None, 0
                assert mask.is_cuda and mask.shape == (self.N,)
                if mask.dtype != torch.uint8:
                    mask = mask.to(torch.uint8)
                mask = mask.contiguous()
                return mask, int(mask.data_ptr())

            def encode_step(self, symbols_gpu, probs_gpu, mask=None):
                import torch
                assert symbols_gpu.is_cuda and probs_gpu.is_cuda
                assert symbols_gpu.numel() == self.N and tuple(probs_gpu.shape) == (self.N, self.K)
                symbols_gpu = symbols_gpu.to(torch.int32).contiguous()
                probs_gpu = probs_gpu.to(torch.float32).contiguous()
                mask, mp = self._mask_ptr(mask)
                _n.call("boa_rc_encode_step", self._core.h, ctypes.c_void_p(symbols_gpu.data_ptr()),
                        ctypes.c_void_p(probs_gpu.data_ptr()), ctypes.c_void_p(mp),
                        ctypes.c_void_p(_n.stream_ptr()))

            def finalize(self):
                _n.call("boa_rc_finalize", self._core.h, ctypes.c_void_p(_n.stream_ptr()))

            def init_decoder(self):
                _n.call("boa_rc_init_decoder", self._core.h, ctypes.c_void_p(_n.stream_ptr()))

            def decode_step(self, probs_gpu, out_symbols_gpu, mask=None):
                import torch
                assert probs_gpu.is_cuda and out_symbols_gpu.is_cuda
                assert tuple(probs_gpu.shape) == (self.N, self.K) and out_symbols_gpu.numel() == self.N
                assert out_symbols_gpu.dtype == torch.int32 and out_symbols_gpu.is_contiguous()
                probs_gpu = probs_gpu.to(torch.float32).contiguous()
                mask, mp = self._mask_ptr(mask)
                _n.call("boa_rc_decode_step", self._core.h, ctypes.c_void_p(probs_gpu.data_ptr()),
                        ctypes.c_void_p(out_symbols_gpu.data_ptr()), ctypes.c_void_p(mp),
                        ctypes.c_void_p(_n.stream_ptr()))


class _ModelStub:
    def __init__(self, kind: str, **kwargs):
        self.kind = kind
        self.kwargs = kwargs


class stream:
    """constriction-shaped single-stream coder (gpu_range_coder.py:390-481).

    In the reference these classes are stubs whose compiled backends do not
    exist; here they work, on the GPU, with the reference quantiser at
    PRECISION 24 (one stream per object).
    """

    class model:
        class Categorical(_ModelStub):
            def __init__(self, perfect: bool = False):
                super().__init__("categorical", perfect=perfect)

    class queue:
        class RangeEncoder:
            def __init__(self):
                self._symbols: list[int] = []
                self._probs: list[np.ndarray] = []

            def clear(self):
                self._symbols, self._probs = [], []

            def encode(self, symbols, model, probs):
                if not isinstance(model, _ModelStub) or model.kind != "categorical":
                    raise TypeError("Only Categorical model is supported")
                symbols = np.atleast_1d(np.asarray(symbols, dtype=np.int32))
                probs = np.asarray(probs, dtype=np.float32)
                if symbols.ndim != 1:
                    raise ValueError("symbols must be rank-1")
                if probs.ndim != 2 or probs.shape[0] != symbols.shape[0]:
                    raise ValueError("probs must be rank-2 with probs.shape[0] == len(symbols)")
                self._symbols.extend(int(s) for s in symbols)
                self._probs.extend(np.array(r) for r in probs)

            def get_compressed(self):
                import torch
                if not self._symbols:
                    return np.zeros(0, dtype=np.uint32)
                K = self._probs[0].shape[0]
                T = len(self._symbols)
                b = gpu.queue.RangeCoderBatch(1, K, T)
                syms = torch.tensor(self._symbols, dtype=torch.int32, device="cuda")
                probs = torch.from_numpy(np.stack(self._probs)).to("cuda")
                for t in range(T):
                    b.encode_step(syms[t:t + 1], probs[t:t + 1])
                b.finalize()
                return b.get_compressed_list()[0]

        class RangeDecoder:
            def __init__(self, compressed):
                self._words = np.asarray(compressed, dtype=np.uint32).ravel()
                self._batch = None

            def decode(self, model, probs_or_amt, *rest):
                import torch
                if not isinstance(model, _ModelStub) or model.kind != "categorical":
                    raise TypeError("Only Categorical model is supported")
                probs = np.asarray(probs_or_amt, dtype=np.float32)
                if probs.ndim != 2:
                    raise ValueError("probs must be rank-2")
                K = probs.shape[1]
                if self._batch is None:
                    self._batch = gpu.queue.RangeCoderBatch(1, K, max(1, self._words.shape[0]))
                    self._batch.load_compressed_list([self._words])
                    self._batch.init_decoder()
                out = torch.empty(1, dtype=torch.int32, device="cuda")
                res = []
                for r in range(probs.shape[0]):
                    p = torch.from_numpy(probs[r:r + 1]).to("cuda")
                    self._batch.decode_step(p, out)
                    res.append(int(out.item()))
                return np.asarray(res, dtype=np.int32)
