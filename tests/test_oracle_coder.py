"""CPU checks of the oracle coder and quantisers (no GPU)."""
import numpy as np
import pytest

from oracle import orc
from coder_cases import make_case


@pytest.mark.parametrize("mode,precision", [(orc.MODE_REF, 24), (orc.MODE_BQ, 16),
                                            (orc.MODE_BQ, 24), (orc.MODE_REF, 16)])
@pytest.mark.parametrize("skew", [False, True])
def test_roundtrip(mode, precision, skew):
    rows, syms, counts = make_case(11 + precision + 3 * mode, 6, 200, 256, mode, precision, skew=skew)
    words, sizes, st = orc.encode(rows, syms, counts, precision, mode, pitch=2 * 200 + 8)
    assert st == 0
    assert sizes[1] == 0  # a stream with no symbols writes nothing (gpu_range_coder.py:148)
    dec = orc.decode(rows, words, sizes, counts, precision, mode)
    for i in range(rows.shape[0]):
        assert np.array_equal(dec[i, :counts[i]], syms[i, :counts[i]])


def test_bq_table_invariants():
    rng = np.random.default_rng(5)
    for sigma in (0.0, 0.1, 3.0, 30.0):
        for K in (1, 2, 7, 200, 256, 1000):
            x = rng.normal(0, sigma, K).astype(np.float32)
            for P in (16, 24):
                if 2 * K > (1 << P):
                    continue
                c = orc.cdf_bq(x, P).astype(np.int64)
                f = np.diff(c)
                assert c[0] == 0 and c[-1] == (1 << P)
                assert f.min() >= 1
    # non-finite rows -> uniform table
    x = np.zeros(256, np.float32); x[3] = np.nan
    f = np.diff(orc.cdf_bq(x, 16).astype(np.int64))
    assert f.min() == f.max() == 256


def test_bq_monotone_in_logit():
    rng = np.random.default_rng(6)
    x = rng.normal(0, 3, 256).astype(np.float32)
    f = np.diff(orc.cdf_bq(x, 16).astype(np.int64))
    am = int(np.argmax(x))
    order = np.argsort(x, kind="stable")
    ff = f.copy(); ff[am] = f.max()  # remainder goes to the argmax only
    assert np.all(np.diff(ff[order]) >= 0)


def test_ref_cdf_degenerate_rows():
    z = np.zeros(256, np.float32)
    c = orc.cdf_ref(z, 24).astype(np.int64)
    assert c[1] == 65536 and c[-1] == 1 << 24
    c = orc.cdf_ref(np.full(256, np.nan, np.float32), 24).astype(np.int64)
    assert np.all(np.diff(c) == 65536)


def test_exp_det_accuracy():
    xs = np.linspace(-31.9, 0, 4001).astype(np.float32)
    e = np.array([orc.exp_det(float(v)) for v in xs])
    ref = np.exp(xs.astype(np.float64))
    assert np.max(np.abs(e - ref) / ref) < 3e-6
    assert orc.exp_det(0.0) == 1.0
    assert orc.exp_det(-40.0) == 0.0


def test_compressed_size_near_entropy():
    rows, syms, counts = make_case(3, 4, 2000, 256, orc.MODE_BQ, 16)
    counts[:] = 2000
    cdfs = orc.cdf_rows(rows, orc.MODE_BQ, 16).astype(np.int64)
    words, sizes, st = orc.encode(rows, syms, counts, 16, orc.MODE_BQ, pitch=4100)
    assert st == 0
    for i in range(4):
        ideal = -np.sum(np.log2((np.take_along_axis(cdfs[i], syms[i][:, None] + 1, 1)[:, 0]
                                 - np.take_along_axis(cdfs[i], syms[i][:, None], 1)[:, 0]) / 65536.0))
        assert sizes[i] * 32 <= ideal + 96
