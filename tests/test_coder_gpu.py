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
