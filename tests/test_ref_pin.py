"""Pin the CPU oracle to the reference's own CUDA coder.

``oracle/_ref`` holds the reference extension compiled unmodified from
gpu_range_coder.py:26-325 by ``oracle/build_ref.py``.  On a GPU box, feed it
seeded probabilities and compare its bitstreams and decoded symbols with the
oracle at PRECISION 24 (the reference's constant, gpu_range_coder.py:40).
"""
import numpy as np
import pytest
import torch

from oracle import orc, build_ref
from coder_cases import make_case

pytestmark = pytest.mark.gpu


def _ref_module():
    mod = build_ref.load()
    if mod is None:
        pytest.skip("oracle/_ref not built (reference tree absent when building)")
    return mod


@pytest.mark.parametrize("skew", [False, True])
def test_oracle_matches_reference_kernel(skew):
    mod = _ref_module()
    N, T, K = 29, 80, 256
    rows, syms, counts = make_case(500 + int(skew), N, T, K, orc.MODE_REF, 24, skew=skew)
    pitch = max(256, T * 8) // 4
    b = mod.RangeCoderBatch(N, K, pitch)
    R = torch.from_numpy(rows).cuda(); S = torch.from_numpy(syms).cuda()
    C = torch.from_numpy(counts).cuda()
    for t in range(T):
        r = R[:, t].contiguous(); s = S[:, t].contiguous(); m = (C > t).to(torch.uint8)
        b.encode_step_from_device(s.data_ptr(), r.data_ptr(), m.data_ptr())
    b.finalize()
    ref_comp = b.get_compressed_host()
    ow, osz, st = orc.encode(rows, syms, counts, 24, orc.MODE_REF, pitch)
    for i in range(N):
        assert np.array_equal(np.asarray(ref_comp[i]), ow[i, :osz[i]]), i
    # decode with the reference kernel
    d = mod.RangeCoderBatch(N, K, pitch)
    d.load_compressed_from_host([np.asarray(c, dtype=np.uint32) for c in ref_comp])
    d.init_decoder_from_current_bytes()
    out = torch.empty(N, dtype=torch.int32, device="cuda")
    dec = np.full((N, T), -1, np.int32)
    for t in range(T):
        r = R[:, t].contiguous(); m = (C > t).to(torch.uint8)
        d.decode_step_to_device(r.data_ptr(), out.data_ptr(), m.data_ptr())
        torch.cuda.synchronize()
        o = out.cpu().numpy()
        mm = counts > t
        dec[mm, t] = o[mm]
    for i in range(N):
        assert np.array_equal(dec[i, :counts[i]], syms[i, :counts[i]])
