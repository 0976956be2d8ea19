"""Failure detection without a GPU fault: every device-side wait is bounded;
when one runs out the kernel returns, the host reports BOA_ERR_TIMEOUT, and
the CUDA context keeps working."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_bounded_wait_times_out_and_context_survives():
    import codec
    from boa_b200 import _native as _n
    from model import seeded_model
    with pytest.raises(_n.BoaError) as ei:
        _n.call("boa_diag_timeout", 200_000_000, 0)        # about 0.1 s of SM cycles
    assert ei.value.code == _n.BOA_ERR_TIMEOUT
    # the context is still usable: a normal round trip right after
    m = seeded_model(64, 2)
    rng = np.random.default_rng(5)
    xs = [torch.from_numpy(rng.integers(0, 256, (1, n)).astype(np.uint8)) for n in (7, 40)]
    comp, first, Ls = codec.compress_GPU(m, xs)
    outs = codec.decompress_GPU(m, comp, Ls, first)
    assert all(np.array_equal(x.numpy(), o) for x, o in zip(xs, outs))


def test_diag_timeout_rejects_bad_budget():
    from boa_b200 import _native as _n
    with pytest.raises(_n.BoaError) as ei:
        _n.call("boa_diag_timeout", 10, 0)
    assert ei.value.code == _n.BOA_ERR_ARG
