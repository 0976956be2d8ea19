"""Host-side arithmetic of bench.py (CPU): the algorithmic bytes and FLOPs the
rooflines divide by, the traffic records they read, the peaks, and the
chunking of the configuration inputs."""
import importlib.util
import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def bench():
    spec = importlib.util.spec_from_file_location("bench_under_test", os.path.join(ROOT, "bench.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_algorithmic_units(bench):
    # recurrent state read + written per coded byte: 2 * L * E * (16 + 3) * 4
    assert bench.state_bytes_per_coded_byte(256, 8) == 622592
    assert bench.state_bytes_per_coded_byte(64, 2) == 38912
    # projection multiply-adds per coded byte at d256/L8 (15.47 MFLOP)
    assert bench.gemm_macs_per_byte(256, 8) == 7733248


def test_traffic_records_match_shape_kind_launch_and_block(bench):
    recs = json.load(open(os.path.join(ROOT, "profiles", "traffic.json")))
    for rec in recs.values():
        m = rec["model"]
        got = bench.traffic_per_coded_byte(m["d_model"], m["num_layers"], rec["weights"], rec["launch"],
                                           rec.get("time_block", 1))
        assert got is not None
        # a record is found for its own key; ncu bytes are within 2x of the algorithmic bytes
        assert 0.5 < rec["dram_bytes_per_coded_byte"] / rec["algorithmic_bytes_per_coded_byte"] < 2.0
    # the 8-position encode record is distinct from the 4-position one
    t4 = bench.traffic_per_coded_byte(256, 8, "f16x2", "encode", 4)
    t8 = bench.traffic_per_coded_byte(256, 8, "f16x2", "encode", 8)
    assert t4 and t8 and t8 < t4
    assert bench.traffic_per_coded_byte(256, 8, "f16x2", "encode", 2) is None
    assert bench.traffic_per_coded_byte(512, 16, "bf16", "decode") is None


def test_peaks(bench):
    hbm, src = bench.measured_peak()
    assert hbm > 1000 and src
    bf16, _ = bench.measured_tensor_peak("f16x2")
    tf32, note = bench.measured_tensor_peak("tf32x3")
    assert tf32 == pytest.approx(bf16 / 2) and "halved" in note


def test_config_chunking(bench):
    """1000 chunks as configuration 2 cuts its input (here a 1 MiB sample),
    the last one shorter, rebuilt byte for byte from the chunk array."""
    import numpy as np
    data = bytes(np.random.default_rng(3).integers(0, 256, 64 * bench.MiB // 64, dtype=np.uint8))
    arr, lens = bench.chunk_array(data, 1000)
    assert arr.shape[0] == len(lens) and sum(lens) == len(data)
    assert b"".join(arr[i, :n].tobytes() for i, n in enumerate(lens)) == data
    assert bench.CONFIGS[2]["fmt"] == "f16x2" and bench.CONFIGS[4]["fmt"] == "bf16"


def test_cli_help():
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--help"], capture_output=True, text=True,
                       timeout=120)
    assert r.returncode == 0 and "--weights" in r.stdout and "f16x2" in r.stdout
