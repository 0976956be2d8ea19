"""CPU pins: seeded init, oracle model restatement, synthetic generators,
weight layout (no GPU)."""
import hashlib
import json
import os

import numpy as np
import torch

G = os.path.join(os.path.dirname(__file__), "golden")


def test_seeded_init_is_stable():
    from model import seeded_model
    exp = json.load(open(os.path.join(G, "seeded_init.json")))
    sd = seeded_model(exp["d_model"], exp["num_layers"], seed=exp["seed"]).state_dict()
    assert sorted(sd) == exp["keys"]
    h = hashlib.sha256()
    for k in sorted(sd):
        h.update(k.encode())
        h.update(sd[k].detach().float().contiguous().numpy().tobytes())
    assert h.hexdigest() == exp["sha256"]


def test_state_dict_keys_match_reference_exporter():
    """Every key convert_boa_weights.py:16-135 reads exists, with mamba_ssm shapes."""
    from model import seeded_model
    sd = seeded_model(64, 2).state_dict()
    d, E, R = 64, 128, 4
    assert sd["embedding.weight"].shape == (256, d)
    for i in range(2):
        p = f"blocks.{i}.mamba."
        assert sd[p + "in_proj.weight"].shape == (2 * E, d)
        assert sd[p + "conv1d.weight"].shape == (E, 1, 4) and sd[p + "conv1d.bias"].shape == (E,)
        assert sd[p + "x_proj.weight"].shape == (R + 32, E)
        assert sd[p + "dt_proj.weight"].shape == (E, R) and sd[p + "dt_proj.bias"].shape == (E,)
        assert torch.allclose(sd[p + "A_log"].exp(), torch.arange(1, 17.).repeat(E, 1))
        assert torch.all(sd[p + "D"] == 1)
        assert sd[p + "out_proj.weight"].shape == (d, E)
        assert p + "in_proj.bias" not in sd and p + "out_proj.bias" not in sd
        dt = torch.nn.functional.softplus(sd[p + "dt_proj.bias"])
        assert dt.min() >= 1e-4 * 0.999 and dt.max() <= 0.1 * 1.001
    for k in ("head.0.weight", "head.0.bias", "head.2.weight", "head.2.bias"):
        assert k in sd


def test_flat_weights_order_and_size(tmp_path):
    from model import seeded_model
    from boa_b200.weights import flatten_state_dict, flat_size, write_bin, read_bin
    sd = seeded_model(64, 2).state_dict()
    flat = flatten_state_dict(sd)
    assert flat.size == flat_size(64, 2)
    assert np.array_equal(flat[:256 * 64], sd["embedding.weight"].numpy().ravel())
    off = 256 * 64 + 64 + 64
    assert np.array_equal(flat[off:off + 256 * 64], sd["blocks.0.mamba.in_proj.weight"].numpy().ravel())
    assert np.all(flat[off + 256 * 64: off + 256 * 64 + 256] == 0)   # in_proj.bias slot
    assert np.array_equal(flat[-256:], sd["head.2.bias"].numpy())
    p = tmp_path / "w.bin"
    write_bin(sd, str(p))
    assert np.array_equal(read_bin(str(p)), flat)


def test_oracle_matches_committed_logits():
    from model import seeded_model
    from oracle import model_oracle as mo
    z = np.load(os.path.join(G, "oracle_c1_logits.npz"))
    sd = {k: v.float() for k, v in seeded_model(64, 2).state_dict().items()}
    lg = mo.forward(sd, mo.config_from_state_dict(sd), torch.from_numpy(z["tokens"]), dtype=torch.float64)
    assert np.abs(lg.numpy() - z["logits"]).max() < 1e-5


def test_oracle_step_equals_fp32_fp64():
    from model import seeded_model
    from oracle import model_oracle as mo
    sd = {k: v.float() for k, v in seeded_model(64, 2).state_dict().items()}
    cfg = mo.config_from_state_dict(sd)
    toks = torch.randint(0, 256, (3, 10), generator=torch.Generator().manual_seed(1))
    a = mo.forward(sd, cfg, toks, dtype=torch.float32)
    b = mo.forward(sd, cfg, toks, dtype=torch.float64)
    assert (torch.softmax(a, -1) - torch.softmax(b.float(), -1)).abs().max() < 1e-5


def test_synthetic_digests():
    from boa_b200 import synthetic
    exp = json.load(open(os.path.join(G, "synthetic.json")))
    d1 = synthetic.config_data(1)
    assert len(d1) == exp["config1_len"]
    assert hashlib.sha256(d1).hexdigest() == exp["config1_sha256"]
    d2 = synthetic.hep_records(1 << 20, 2)
    assert hashlib.sha256(d2).hexdigest() == exp["hep_1MiB_seed2_sha256"]


def test_hep_record_structure():
    from boa_b200 import synthetic
    import struct
    d = synthetic.hep_records(200_000, 2)
    pos, ev = 0, 0
    while pos + 6 <= len(d):
        eid, n = struct.unpack_from("<iH", d, pos)
        assert eid == ev
        pos += 6
        for _ in range(n):
            if pos + 14 > len(d):
                break
            pt, eta, phi, pdg = struct.unpack_from("<fffh", d, pos)
            assert pt > 0 and -3.2 < phi < 3.2 and abs(pdg) in (11, 13, 22, 211, 2112)
            pos += 14
        ev += 1
    assert ev > 300


def test_bq_quantiser_matches_golden_tables():
    """The C oracle's integer quantiser reproduces the committed tables
    (wide / narrow / near-deterministic / NaN / +inf rows, K = 256 and 37,
    totals 2^16 and 2^24)."""
    from oracle import orc
    z = np.load(os.path.join(G, "bq_tables.npz"))
    for P in (16, 24):
        for r in range(z["rows"].shape[0]):
            assert np.array_equal(orc.cdf_bq(z["rows"][r], P), z[f"cdf{P}"][r]), (P, r)
        assert np.array_equal(orc.cdf_bq(z["row37"], P), z[f"cdf37_{P}"]), P
    c = z["cdf16"]
    assert np.all(c[:, -1] == 1 << 16) and np.all(np.diff(c.astype(np.int64), axis=1) >= 1)
