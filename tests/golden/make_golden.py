"""Regenerate the committed CPU golden fixtures in tests/golden/.

Run in a container that has the reference tree (--reference points at it):
    python tests/golden/make_golden.py [--reference /path/to/reference]

Fixtures:
  ref_container.boa / ref_container.json
      A BOA2 file written by the reference's own BoaFile._write_file
      (boa.py:89-112, imported from the reference tree) for fixed fake
      payloads, plus what the reference's _read_file (boa.py:114-157) parses
      from it and from a file written by this build's container module with
      the quantiser flag set (the reference reader ignores flags).
  seeded_init.json
      sha256 of the fp32 state_dict of model.seeded_model(64, 2) (seed 0) and a
      few sample values: pins this build's seeded Mamba-standard init.
  oracle_c1_logits.npz
      oracle logits (computed in fp64, stored fp32) of that model for 3 streams x 24 seeded tokens.
  synthetic.json
      sha256 of the config-1 input and of the first 1 MiB of the config-2 input.
  ref_weights.json
      sha256 and size of the .bin that the reference's own weight exporter
      (portability_solved_cpp/convert_boa_weights.py:16-135, imported from the
      reference tree) writes for the seeded models at the configuration
      shapes (d_model 64 / 2 layers, 256 / 8): pins boa_b200.weights.write_bin.
  bq_tables.npz
      seeded logit rows (wide, narrow, near-deterministic, NaN, +inf, K = 256
      and K = 37) and their BQ integer-quantiser CDFs at totals 2^16 and 2^24
      from the C oracle: pins this build's quantiser definition.
"""
from __future__ import annotations

import argparse
import hashlib
import importlib.util
import json
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "boa-constrictor_b200"))
sys.path.insert(0, ROOT)


def bq_rows():
    rng = np.random.default_rng(77)
    rows = [rng.normal(0, 3, 256), rng.normal(0, 0.1, 256), rng.normal(-30, 1, 256)]
    rows[2][5] = 30.0                                  # one dominant entry: many frequency-1 symbols
    nan_row = rng.normal(0, 1, 256)
    nan_row[17] = np.nan                               # degenerate: uniform table
    inf_row = rng.normal(0, 1, 256)
    inf_row[3] = np.inf
    rows += [nan_row, inf_row]
    return np.asarray(rows, np.float32), rng.normal(0, 2, 37).astype(np.float32)


def write_bq_tables():
    from oracle import orc
    rows, row37 = bq_rows()
    out = {"rows": rows, "row37": row37}
    for P in (16, 24):
        out[f"cdf{P}"] = np.stack([orc.cdf_bq(r, P) for r in rows])
        out[f"cdf37_{P}"] = orc.cdf_bq(row37, P)
    np.savez_compressed(os.path.join(HERE, "bq_tables.npz"), **out)


def container_case():
    rng = np.random.default_rng(123)
    comp = [rng.integers(0, 2**32, size=k, dtype=np.uint64).astype(np.uint32) for k in (3, 0, 7, 130, 1)]
    first = [7, 0, 255, 128, 33]
    ulen, chunk_len, last = 5 * 1000 - 400, 1000, 600
    return comp, first, ulen, chunk_len, last


def load_reference_boa(reference: str):
    sys.path.insert(0, reference)          # reference boa.py imports its own codec lazily
    spec = importlib.util.spec_from_file_location("reference_boa", os.path.join(reference, "boa.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


WEIGHT_PIN_SHAPES = [(64, 2), (256, 8)]


def write_ref_weights(reference: str):
    """Run the reference exporter on the seeded state_dicts; record digests."""
    import tempfile
    from model import seeded_model
    spec = importlib.util.spec_from_file_location(
        "reference_convert", os.path.join(reference, "portability_solved_cpp", "convert_boa_weights.py"))
    conv = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(conv)
    out = {}
    with tempfile.TemporaryDirectory() as tmp:
        for d, L in WEIGHT_PIN_SHAPES:
            pt, bn = os.path.join(tmp, "m.pt"), os.path.join(tmp, "m.bin")
            torch.save(seeded_model(d, L).state_dict(), pt)
            conv.convert(pt, bn)
            raw = open(bn, "rb").read()
            out[f"d{d}_L{L}"] = {"d_model": d, "num_layers": L, "seed": 0, "bytes": len(raw),
                                 "sha256": hashlib.sha256(raw).hexdigest()}
    with open(os.path.join(HERE, "ref_weights.json"), "w") as f:
        json.dump(out, f, indent=1)


class BoaBytePredictor(torch.nn.Module):
    """Stand-in whose class name gives the reference fingerprint."""


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=None,
                    help="reference checkout (default: $BOA_REFERENCE_ROOT or a sibling 'reference' directory)")
    ap.add_argument("--only-bq", action="store_true", help="write bq_tables.npz only (no reference tree needed)")
    ap.add_argument("--only-weights", action="store_true", help="write ref_weights.json only")
    a = ap.parse_args()
    if a.only_bq:
        write_bq_tables()
        return
    from boa_b200 import container as C
    from model import seeded_model
    from boa_b200 import synthetic
    from oracle import model_oracle as mo

    # --- container written by the reference ---
    from oracle.build_ref import reference_root
    root = a.reference or reference_root()
    if not root:
        raise SystemExit("make_golden: no reference checkout (pass --reference or set BOA_REFERENCE_ROOT)")
    write_ref_weights(root)
    if a.only_weights:
        return
    ref = load_reference_boa(root)
    comp, first, ulen, chunk_len, last = container_case()
    path = os.path.join(HERE, "ref_container.boa")
    bf = ref.BOA("cpu", path, BoaBytePredictor())
    bf._write_file([c.astype("<u4").tobytes() for c in comp], first, ulen, chunk_len, last)
    bf2 = ref.BOA("cpu", path, BoaBytePredictor())
    bf2._read_file()
    ours_path = os.path.join(HERE, "_ours_tmp.boa")
    payload = b"".join(c.astype("<u4").tobytes() for c in comp)
    sizes = [4 * len(c) for c in comp]
    offs = [int(x) for x in np.concatenate([[0], np.cumsum(sizes)[:-1]])]
    with open(ours_path, "wb") as f:
        f.write(C.header_bytes(C.make_flags(16), ulen, chunk_len, len(comp), last,
                               C.model_fingerprint(BoaBytePredictor())))
        f.write(payload)
        f.write(C.index_bytes(first, offs, sizes))
    bf3 = ref.BOA("cpu", ours_path, BoaBytePredictor())
    bf3._read_file()
    os.remove(ours_path)
    meta = {
        "inputs": {"words": [c.tolist() for c in comp], "first_bytes": first, "uncompressed_len": ulen,
                   "chunk_len": chunk_len, "last_chunk_len": last},
        "reference_parse_of_reference_file": {"first_bytes": [int(x) for x in bf2.first_bytes],
                                              "lengths": bf2.lengths, "metadata": bf2.metadata,
                                              "payload_hex": [c.hex() for c in bf2.compressed_data]},
        "reference_parse_of_our_file": {"first_bytes": [int(x) for x in bf3.first_bytes],
                                        "lengths": bf3.lengths, "metadata": bf3.metadata,
                                        "payload_hex": [c.hex() for c in bf3.compressed_data]},
    }
    with open(os.path.join(HERE, "ref_container.json"), "w") as f:
        json.dump(meta, f, indent=1)

    # --- seeded init fingerprint ---
    m = seeded_model(64, 2)
    sd = m.state_dict()
    h = hashlib.sha256()
    for k in sorted(sd):
        h.update(k.encode())
        h.update(sd[k].detach().float().contiguous().numpy().tobytes())
    samples = {k: [float(x) for x in sd[k].flatten()[:3]] for k in sorted(sd)}
    with open(os.path.join(HERE, "seeded_init.json"), "w") as f:
        json.dump({"d_model": 64, "num_layers": 2, "seed": 0, "sha256": h.hexdigest(),
                   "keys": sorted(sd), "first_values": samples}, f, indent=1)

    # --- oracle logits ---
    sdf = {k: v.detach().float() for k, v in sd.items()}
    cfg = mo.config_from_state_dict(sdf)
    toks = np.random.default_rng(9).integers(0, 256, (3, 24)).astype(np.int64)
    lg = mo.forward(sdf, cfg, torch.from_numpy(toks), dtype=torch.float64).numpy()
    np.savez_compressed(os.path.join(HERE, "oracle_c1_logits.npz"), tokens=toks, logits=lg.astype(np.float32))

    # --- synthetic data digests ---
    d1 = synthetic.config_data(1)
    d2 = synthetic.hep_records(1 << 20, 2)
    with open(os.path.join(HERE, "synthetic.json"), "w") as f:
        json.dump({"config1_sha256": hashlib.sha256(d1).hexdigest(), "config1_len": len(d1),
                   "hep_1MiB_seed2_sha256": hashlib.sha256(d2).hexdigest()}, f, indent=1)
    write_bq_tables()
    print("golden fixtures written to", HERE)


if __name__ == "__main__":
    main()
