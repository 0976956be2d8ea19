"""The allocation-free encode entry point (boa_rc_encode_noalloc) against the
allocating one (boa_rc_create + boa_rc_encode_step + boa_rc_finalize), through
the C-ABI, on two calls in a row.

It is for callers that cannot allocate device memory while they code: a
plugin host or framework that owns the device memory pool and forbids
allocation after start-up, or a real-time service that must not stall on
cudaMalloc.  Its coder state lives in a static per-device array shared by
every call; each call synchronises its stream to report errors.  This file
runs last so that a failure here leaves every other test already run; it
also passes alone in a fresh process.
"""
import ctypes

import numpy as np
import pytest
import torch

from boa_b200 import _native as _n

pytestmark = pytest.mark.gpu


def _case(seed, N, T, K=256):
    rng = np.random.default_rng(seed)
    logits = rng.normal(0.0, 3.0, (T, N, K)).astype(np.float32)
    syms = rng.integers(0, K, (T, N)).astype(np.int32)
    mask = (rng.random((T, N)) < 0.9).astype(np.uint8)
    mask[:, 0] = 1
    return logits, syms, mask


def _allocating(logits, syms, mask, precision, pitch):
    """The existing entry points: a RangeCoderBatch with its own device state."""
    import gpu_range_coder as gr
    T, N, K = logits.shape
    b = gr.gpu.queue.RangeCoderBatch(N, K, T, pitch_bytes=4 * pitch, precision=precision, quantiser="bq")
    L = torch.from_numpy(logits).cuda(); S = torch.from_numpy(syms).cuda(); M = torch.from_numpy(mask).cuda()
    for t in range(T):
        b.encode_step(S[t].contiguous(), L[t].contiguous(), mask=M[t].contiguous())
    b.finalize()
    return b.get_compressed_list()


def _noalloc(logits, syms, mask, precision, pitch):
    T, N, K = logits.shape
    L = torch.from_numpy(logits).cuda(); S = torch.from_numpy(syms).cuda(); M = torch.from_numpy(mask).cuda()
    words = torch.zeros((N, pitch), dtype=torch.int32, device="cuda")
    sizes = torch.zeros(N, dtype=torch.int32, device="cuda")
    torch.cuda.synchronize()
    _n.call("boa_rc_encode_noalloc", N, K, T, precision, ctypes.c_void_p(L.data_ptr()),
            ctypes.c_void_p(S.data_ptr()), ctypes.c_void_p(M.data_ptr()), ctypes.c_void_p(words.data_ptr()),
            pitch, ctypes.c_void_p(sizes.data_ptr()), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    w = words.cpu().numpy().view(np.uint32)
    s = sizes.cpu().numpy()
    return [w[i, :s[i]].copy() for i in range(N)]


def test_noalloc_matches_allocating_entry_point_twice():
    # two calls in a row: the second must not see state left by the first
    for seed, N, T in ((1, 300, 40), (2, 97, 57)):
        logits, syms, mask = _case(seed, N, T)
        pitch = (T * 16 + 31) // 32 + 6
        a = _allocating(logits, syms, mask, 16, pitch)
        b = _noalloc(logits, syms, mask, 16, pitch)
        assert len(a) == len(b) == N
        for i in range(N):
            assert np.array_equal(a[i], b[i]), (seed, i)


def test_noalloc_rejects_too_many_streams():
    with pytest.raises(_n.BoaError):
        _n.call("boa_rc_encode_noalloc", (1 << 16) + 1, 256, 0, 16, None, None, None,
                ctypes.c_void_p(16), 8, ctypes.c_void_p(16), None)
