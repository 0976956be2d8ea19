"""boa_b200.weights.write_bin writes byte for byte the .bin that the
reference's own exporter (portability_solved_cpp/convert_boa_weights.py:16-135)
writes for the same state_dict.  The reference's digests for the seeded models
at the configuration shapes are in tests/golden/ref_weights.json, made by
tests/golden/make_golden.py from the reference tree; this test needs neither
the reference nor a GPU."""
import hashlib
import json
import os

import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
PINS = json.load(open(os.path.join(HERE, "golden", "ref_weights.json")))


@pytest.mark.parametrize("key", sorted(PINS))
def test_write_bin_equals_reference_exporter(key, tmp_path):
    from model import seeded_model
    from boa_b200.weights import write_bin, read_bin, flatten_state_dict
    pin = PINS[key]
    sd = seeded_model(pin["d_model"], pin["num_layers"], seed=pin["seed"]).state_dict()
    path = tmp_path / "w.bin"
    write_bin(sd, str(path))
    raw = path.read_bytes()
    assert len(raw) == pin["bytes"]
    assert hashlib.sha256(raw).hexdigest() == pin["sha256"]
    # and the vector boa_model_create consumes is that file's content
    assert read_bin(str(path)).tobytes() == flatten_state_dict(sd).tobytes()
