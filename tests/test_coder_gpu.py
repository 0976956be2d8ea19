"""GPU range coder vs the CPU oracle, bit for bit, through the C-ABI."""
import numpy as np
import pytest
import torch

from oracle import orc
from coder_cases import make_case

pytestmark = pytest.mark.gpu


def _gpu_encode(rows, syms, counts, precision, quant, pitch):
    import gpu_range_coder as gr
    N, T, K = rows.shape
    b = gr.gpu.queue.RangeCoderBatch(N, K, T, pitch_bytes=4 * pitch, precision=precision, quantiser=quant)
    R = torch.from_numpy(rows).cuda()
    S = torch.from_numpy(syms).cuda()
    C = torch.from_numpy(counts).cuda()
    for t in range(T):
        b.encode_step(S[:, t].contiguous(), R[:, t].contiguous(), mask=(C > t))
    b.finalize()
    return b.get_compressed_list()


def _gpu_decode(rows, comp, counts, precision, quant, pitch):
    import gpu_range_coder as gr
    N, T, K = rows.shape
    b = gr.gpu.queue.RangeCoderBatch(N, K, T, pitch_bytes=4 * pitch, precision=precision, quantiser=quant)
    b.load_compressed_list(comp)
    b.init_decoder()
    R = torch.from_numpy(rows).cuda()
    C = torch.from_numpy(counts).cuda()
    out = torch.full((N, T), -1, dtype=torch.int32, device="cuda")
    o = torch.empty(N, dtype=torch.int32, device="cuda")
    for t in range(T):
        m = C > t
        b.decode_step(R[:, t].contiguous(), o, mask=m)
        out[:, t] = torch.where(m, o, out[:, t])
    return out.cpu().numpy()


CASES = [("ref", orc.MODE_REF, 24), ("bq", orc.MODE_BQ, 16), ("bq", orc.MODE_BQ, 24), ("ref", orc.MODE_REF, 16)]


@pytest.mark.parametrize("quant,mode,precision", CASES)
@pytest.mark.parametrize("skew", [False, True])
@pytest.mark.parametrize("K", [256, 200])
def test_encode_decode_bit_exact(quant, mode, precision, skew, K):
    N, T = 37, 96
    rows, syms, counts = make_case(100 + precision + K, N, T, K, mode, precision, skew=skew)
    pitch = 2 * T + 8
    ow, osz, st = orc.encode(rows, syms, counts, precision, mode, pitch)
    assert st == 0
    comp = _gpu_encode(rows, syms, counts, precision, quant, pitch)
    for i in range(N):
        assert len(comp[i]) == osz[i], i
        assert np.array_equal(comp[i], ow[i, :osz[i]]), i
    dec = _gpu_decode(rows, [ow[i, :osz[i]] for i in range(N)], counts, precision, quant, pitch)
    for i in range(N):
        assert np.array_equal(dec[i, :counts[i]], syms[i, :counts[i]]), i


def test_overflow_is_reported():
    import gpu_range_coder as gr
    from boa_b200._native import BoaError
    rows, syms, counts = make_case(9, 4, 64, 256, orc.MODE_BQ, 16)
    b = gr.gpu.queue.RangeCoderBatch(4, 256, 64, pitch_bytes=16, quantiser="bq", precision=16)
    R = torch.from_numpy(rows).cuda(); S = torch.from_numpy(syms).cuda()
    for t in range(64):
        b.encode_step(S[:, t].contiguous(), R[:, t].contiguous())
    b.finalize()
    with pytest.raises(BoaError):
        b.get_compressed_list()


def test_many_streams_bq():
    """A wave-sized batch (5000 streams, BOA_GPU_STREAMS default, boa.py:207)."""
    N, T = 5000, 8
    rows, syms, counts = make_case(77, N, T, 256, orc.MODE_BQ, 16)
    ow, osz, st = orc.encode(rows, syms, counts, 16, orc.MODE_BQ, 2 * T + 8)
    comp = _gpu_encode(rows, syms, counts, 16, "bq", 2 * T + 8)
    assert all(np.array_equal(comp[i], ow[i, :osz[i]]) for i in range(N))


@pytest.mark.parametrize("K,period", [(256, 0), (256, 24), (200, 7)])
def test_multi_step_entry_points_match_single_steps(K, period):
    """boa_rc_encode_steps / decode_steps (one launch for many steps, slots
    reused every `period` steps) write the words the oracle writes for the
    same step sequence, and decode it back."""
    import ctypes
    from boa_b200 import _native as _n
    N, T = 45, 80
    P = period if period > 0 else T
    rows, syms, _ = make_case(7 + K + period, N, P, K, orc.MODE_BQ, 16)
    rng = np.random.default_rng(period + 1)
    mask = (rng.random((P, N)) > 0.2).astype(np.uint8)
    slot = np.array([t % P for t in range(T)])
    # the equivalent step sequence for the oracle: masked steps are skipped
    full_rows = rows[:, slot]                        # [N, T, K]
    full_syms = syms[:, slot]
    keep = mask[slot].T.astype(bool)                 # [N, T]
    counts = keep.sum(1).astype(np.int32)
    o_rows = np.zeros_like(full_rows)
    o_syms = np.zeros_like(full_syms)
    for i in range(N):
        o_rows[i, :counts[i]] = full_rows[i, keep[i]]
        o_syms[i, :counts[i]] = full_syms[i, keep[i]]
    pitch = T // 2 + 16
    ow, osz, st = orc.encode(o_rows, o_syms, counts, 16, orc.MODE_BQ, pitch)
    assert st == 0
    R = torch.from_numpy(np.ascontiguousarray(rows.transpose(1, 0, 2))).cuda()     # [P, N, K]
    S = torch.from_numpy(np.ascontiguousarray(syms.T)).cuda()                      # [P, N]
    M = torch.from_numpy(mask).cuda()
    h = ctypes.c_void_p()
    _n.call("boa_rc_create", ctypes.byref(h), N, K, pitch, 16, _n.BOA_QUANT_BQ, 0)
    try:
        sp = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
        _n.call("boa_rc_encode_steps", h, T, period, ctypes.c_void_p(S.data_ptr()), N,
                ctypes.c_void_p(R.data_ptr()), N * K, ctypes.c_void_p(M.data_ptr()), N, sp)
        _n.call("boa_rc_finalize", h, sp)
        words = np.zeros((N, pitch), np.uint32)
        sizes = np.zeros(N, np.int32)
        _n.call("boa_rc_get_sizes", h, sizes.ctypes.data_as(ctypes.c_void_p), sp)
        _n.call("boa_rc_get_words", h, words.ctypes.data_as(ctypes.c_void_p), sp)
        assert np.array_equal(sizes, osz)
        for i in range(N):
            assert np.array_equal(words[i, :sizes[i]], ow[i, :osz[i]]), i
        _n.call("boa_rc_init_decoder", h, sp)
        out = torch.full((T, N), -1, dtype=torch.int32, device="cuda")
        # decode with the same slot layout, one output row per step
        Rf = torch.from_numpy(np.ascontiguousarray(full_rows.transpose(1, 0, 2))).cuda()   # [T, N, K]
        Mf = torch.from_numpy(np.ascontiguousarray(mask[slot])).cuda()                    # [T, N]
        _n.call("boa_rc_decode_steps", h, T, 0, ctypes.c_void_p(Rf.data_ptr()), N * K,
                ctypes.c_void_p(out.data_ptr()), N, ctypes.c_void_p(Mf.data_ptr()), N, sp)
        got = out.cpu().numpy().T                                                          # [N, T]
        for i in range(N):
            assert np.array_equal(got[i, keep[i]], full_syms[i, keep[i]]), i
    finally:
        _n.load().boa_rc_destroy(h)


@pytest.mark.parametrize("precision", [16, 24])
def test_gpu_coder_on_golden_quantiser_rows(precision):
    """The GPU coder, fed the committed golden logit rows (including NaN and
    +inf rows, which fall back to the uniform table), writes the bitstream the
    oracle writes from the committed tables."""
    import os
    z = np.load(os.path.join(os.path.dirname(__file__), "golden", "bq_tables.npz"))
    base = z["rows"]                                           # [5, 256]
    N, T = base.shape[0], 64
    rows = np.repeat(base[:, None, :], T, axis=1)              # [N, T, 256]
    syms = ((np.arange(T)[None, :] * 7 + np.arange(N)[:, None] * 31) % 256).astype(np.int32)
    counts = np.full(N, T, np.int32)
    pitch = (T * precision + 31) // 32 + 8
    ow, osz, st = orc.encode(rows, syms, counts, precision, orc.MODE_BQ, pitch)
    assert st == 0
    comp = _gpu_encode(rows, syms, counts, precision, "bq", pitch)
    for i in range(N):
        assert np.array_equal(comp[i], ow[i, :osz[i]]), i
