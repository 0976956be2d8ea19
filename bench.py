#!/usr/bin/env python
"""Benchmark of the BoaConstrictor compress/decompress hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config 2] [--impl ours|reference]
                    [--segment S] [--scaling weak|strong] [--weights f16x2|tf32x3|tf32|fp16|bf16]

Default workload: configuration 2 of the benchmark spec -- 64 MiB of seeded
HEP-like event records, chunks_count = 1000 (67,109 B per chunk), the
BoaConstrictor d_model 256 / 8 layers model with seeded random init, and
projections in the fp32-equivalent 2xFP16 operand kind (every fp32 weight and
activation carried as an fp16 hi and a 2^11-scaled fp16 residual, 22
significant bits, products accumulated in fp32; the reference model is fp32
nn.Linear, and at this shape the kernel's probabilities are within 1.5e-8 of
an fp64 evaluation, the reference's fp32 arithmetic within 6e-9).  --weights
tf32x3 runs the 3xTF32 split instead.  Recurrent state, element-wise math and
accumulation are fp32.

A step is one pass of the hot path over one batch: compress, then
decompress, positions [a, a + S) of every chunk of the input (S = --segment,
4096 by default), with each side's recurrent model state carried on the
device from the previous step (boa_codec_encode_range / decode_range; each
segment is its own bitstream).  Consecutive steps walk through the chunks and
start over at position 1 after the last, so the timed steps code the
configuration's own input, a bounded launch at a time.  The first warm-up
steps are checked for a lossless round trip, and so is every timed step.

With N ranks (torchrun, one GPU each) --scaling weak (default) gives every
rank its own copy of the workload (an N x 64 MiB job); --scaling strong splits
the configuration's chunks into N contiguous shares.  No collective touches
the data path: the device times are max-reduced once, after the timed region.

``value`` is the whole-job round-trip throughput with inputs resident in HBM:
bytes of all ranks / max over ranks of (compress + decompress) device time,
in MiB/s (2^20 B/s, the unit of the reference's C++ port, boa.cpp:39).
``e2e`` is the same through the public host API (codec.RangeCodec: pinned
host bytes in, host words out, host words in, host bytes out, every step).

``--impl reference`` times the reference algorithm's CPU restatement
(oracle/codec_oracle.py: fp32 model + softmax + the reference coder at
PRECISION 24) on this host's cores over a bounded sample of the workload.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "boa-constrictor_b200"))

MiB = 1 << 20

CONFIGS = {
    1: dict(name="config1 markov 1 MiB, chunks_count=16, d_model=64, num_layers=2", d=64, L=2, chunks=16,
            data=("markov", 1 << 20), fmt="f16x2"),
    2: dict(name="config2 hep-records 64 MiB, chunks_count=1000, d_model=256, num_layers=8", d=256, L=8,
            chunks=1000, data=("hep", 64 * MiB), fmt="f16x2"),
    3: dict(name="config3 hep-records 64 MiB, chunks_count=8192, d_model=256, num_layers=8", d=256, L=8,
            chunks=8192, data=("hep", 64 * MiB), fmt="f16x2"),
    4: dict(name="config4 records + CFD field 1 GiB, chunks_count=65536, d_model=512, num_layers=16, bf16",
            d=512, L=16, chunks=65536, data=("mixed", 1 << 30), fmt="bf16"),
    5: dict(name="config5 range coder only, 16384 streams x 65536 symbols, logits N(0, 3^2), BQ 2^16",
            streams=16384, symbols=65536, slab=64),
}


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--config", type=int, default=2, choices=sorted(CONFIGS))
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--weights", default=None, choices=["tf32x3", "f16x2", "tf32", "fp16", "bf16"])
    ap.add_argument("--segment", type=int, default=4096, help="positions of every chunk coded per step")
    ap.add_argument("--scaling", default="weak", choices=["weak", "strong"])
    ap.add_argument("--size", type=int, default=None, help="override input bytes (testing)")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    return ap.parse_args()


def make_data(cfg, size=None):
    from boa_b200 import synthetic
    kind, n = cfg["data"]
    n = size or n
    if kind == "markov":
        return synthetic.markov(n, 1)
    if kind == "mixed":
        if n >= (1 << 30):
            return synthetic.mixed(n, 3)
        # a scaled-down config 4: the same records-then-field layout, 7/8 records
        field = synthetic.cfd_field(256, (3, 1))[:n // 8]
        return synthetic.hep_records(n - len(field), 3) + field
    return synthetic.hep_records(n, 2)


def chunk_array(data: bytes, n_chunks: int):
    import numpy as np
    from boa_b200 import container as C
    chunk_len, n, last = C.chunking(len(data), 0, n_chunks)
    lens = [chunk_len] * (n - 1) + [last]
    arr = np.zeros((n, chunk_len), dtype=np.uint8)
    buf = np.frombuffer(data, dtype=np.uint8)
    full = (n - 1) * chunk_len
    arr[:n - 1] = buf[:full].reshape(n - 1, chunk_len)
    arr[n - 1, :last] = buf[full:]
    return arr, lens


def state_bytes_per_coded_byte(d, L):
    """Algorithmic HBM bytes per coded byte: read + write of the recurrent
    state, SSM (L * E * 16 fp32) and conv window (L * E * 3 fp32)."""
    E = 2 * d
    return 2 * L * E * (16 + 3) * 4


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled while the timed region runs."""

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.path = None

    def __enter__(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.index), f"--query-gpu={q}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *a):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        rows = []
        try:
            for line in open(self.path):
                parts = [p.strip() for p in line.split(",")]
                if len(parts) >= 9:
                    rows.append(parts)
            os.remove(self.path)
        except Exception:
            pass
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        reasons = set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            for nm, v in zip(names, r[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(nm)
        loaded = [s for s in sm if s > 300] or sm
        return {"sm_mhz": statistics.median(loaded) if loaded else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": sorted(reasons), "samples": len(rows)}


def measured_peak():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        j = json.load(open(p))
        return float(j["hbm_gbs"]), "measured (MEASURED_PEAKS.json hbm_gbs)"
    except Exception:
        return 6650.0, "fallback 6.65 TB/s"


def measured_tensor_peak(fmt):
    """Dense tensor peak for the operand kind: the measured cuBLAS bf16 burst
    figure (MEASURED_PEAKS.json), halved for tf32 operands."""
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        bf16 = float(json.load(open(p))["bf16_tflops"])
        src = "measured bf16 (MEASURED_PEAKS.json bf16_tflops)"
    except Exception:
        bf16, src = 1590.0, "fallback 1.59 PFLOP/s bf16"
    if fmt in ("tf32", "tf32x3"):
        return bf16 / 2, src + ", halved for tf32 operands"
    return bf16, src


def traffic_per_coded_byte(d, L, fmt, launch, time_block=1):
    """ncu DRAM bytes per coded byte of the decode or encode launch, for the
    model shape, operand kind and positions per kernel step the capture was
    taken on (None otherwise)."""
    p = os.path.join(ROOT, "profiles", "traffic.json")
    try:
        for rec in json.load(open(p)).values():
            if (rec.get("model") == {"d_model": d, "num_layers": L} and rec.get("weights") == fmt
                    and rec.get("launch") == launch and rec.get("time_block", 1) == time_block):
                return float(rec["dram_bytes_per_coded_byte"])
    except Exception:
        pass
    return None


# ---------------------------------------------------------------------------
def gemm_macs_per_byte(d, L, V=256):
    """Projection multiply-adds per coded byte (in_proj, x_proj, dt_proj,
    out_proj, ff.0, ff.2 per layer; head.0, head.2)."""
    E, R = 2 * d, (d + 15) // 16
    return L * (d * 2 * E + E * (R + 32) + R * E + E * d + 8 * d * d) + d * d + V * d


def cpu_baseline(cfg, arr, lens, seconds_target=20.0):
    """The reference algorithm's CPU restatement on a bounded sample (the
    first L_s bytes of the first n_s chunks).  Returns the baseline record and
    the sample, so the GPU path can code the very same bytes."""
    import numpy as np
    import torch
    from model import seeded_model
    from oracle import codec_oracle as co
    torch.set_num_threads(os.cpu_count() or 1)
    sd = {k: v.float() for k, v in seeded_model(cfg["d"], cfg["L"]).state_dict().items()}
    n_s = min(32, arr.shape[0])
    L_s = 64
    # calibrate the sample length so the run takes about seconds_target
    chunks = [arr[i, :L_s] for i in range(n_s)]
    t0 = time.perf_counter()
    co.compress(sd, chunks)
    dt = time.perf_counter() - t0
    L_s = int(max(64, min(min(lens[:n_s]), L_s * (seconds_target / 2) / max(dt, 1e-3))))
    chunks = [arr[i, :L_s].copy() for i in range(n_s)]
    t0 = time.perf_counter()
    comp, first, ls = co.compress(sd, chunks)
    t1 = time.perf_counter()
    out = co.decompress(sd, comp, ls, first)
    t2 = time.perf_counter()
    assert all(np.array_equal(a, b) for a, b in zip(out, chunks))
    nbytes = n_s * L_s
    rec = {"value": nbytes / MiB / (t2 - t0), "unit": "MiB/s", "cores": torch.get_num_threads(), "kind": "port",
           "sample": f"{n_s} chunks x first {L_s} bytes of the workload's chunks, compress + decompress",
           "compress_MiBps": nbytes / MiB / (t1 - t0), "decompress_MiBps": nbytes / MiB / (t2 - t1),
           "bits_per_byte": 32.0 * sum(len(c) for c in comp) / nbytes}
    return rec, chunks, 32 * sum(len(c) for c in comp)


def run_reference(args, cfg, rank):
    if rank != 0:
        return
    import numpy as np
    import torch
    from model import seeded_model
    from oracle import codec_oracle as co
    torch.set_num_threads(os.cpu_count() or 1)
    data = make_data(cfg, args.size)
    arr, lens = chunk_array(data, cfg["chunks"])
    sd = {k: v.float() for k, v in seeded_model(cfg["d"], cfg["L"]).state_dict().items()}
    n_s, L_s = min(16, arr.shape[0]), 96
    chunks = [arr[i, :L_s] for i in range(n_s)]
    for _ in range(args.warmup):
        comp, first, ls = co.compress(sd, chunks)
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        comp, first, ls = co.compress(sd, chunks)
        out = co.decompress(sd, comp, ls, first)
        times.append(time.perf_counter() - t0)
        assert all(np.array_equal(a, b) for a, b in zip(out, chunks))
    nbytes = n_s * L_s
    t = sum(times)
    v = args.steps * nbytes / MiB / t
    line = {"impl": "reference", "metric": "compress+decompress round-trip throughput", "value": v,
            "unit": "MiB/s", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": 1000 * t / args.steps, "higher_is_better": True, "scaling": args.scaling,
            "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": cfg["name"], "sample": f"{n_s} chunks x {L_s} bytes per step"},
            "cpu_baseline": {"value": v, "unit": "MiB/s", "cores": torch.get_num_threads(), "kind": "port",
                             "sample": f"{n_s} chunks x first {L_s} bytes of the workload's chunks per step"},
            "e2e": {"value": v, "unit": "MiB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


DTYPES = {"tf32x3": "f32 (3xTF32: tf32 hi + lo operand halves, fp32 accumulation)",
          "f16x2": "f32 (2xFP16: fp16 hi + 2^11-scaled fp16 residual, 22-bit operands, fp32 accumulation)",
          "tf32": "tf32 products / f32", "fp16": "fp16 products / f32", "bf16": "bf16 products / f32"}


# ---------------------------------------------------------------------------
def run_ours(args, cfg, rank, world, local_rank, dist):
    import numpy as np
    import torch
    import codec
    from model import seeded_model
    from boa_b200.shard import shard_range

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    fmt = args.weights or cfg["fmt"]
    data = make_data(cfg, args.size)
    arr, lens = chunk_array(data, cfg["chunks"])
    n_all = arr.shape[0]
    if args.scaling == "strong" and world > 1:
        lo, hi = shard_range(n_all, world, rank)
        arr, lens = arr[lo:hi], lens[lo:hi]
    n, maxL = arr.shape
    total_bytes = int(sum(lens))
    model = seeded_model(cfg["d"], cfg["L"], weight_format=fmt)
    nm = model.native(dev)
    X = torch.from_numpy(arr).to(dev)
    Ld = torch.tensor(lens, dtype=torch.int32, device=dev)
    lens_np = np.asarray(lens, np.int64)
    first = X[:, 0].contiguous()
    out = torch.zeros((n, maxL), dtype=torch.uint8, device=dev)
    # Waves: each direction keeps its recurrent state for the chunks of one
    # wave; waves hold as many chunks as two states fit in 60 % of the free
    # device memory (all of them, except for configuration 4)
    free_b, _ = torch.cuda.mem_get_info(dev)
    per_chunk = nm.workspace_bytes(32) / 32
    wave = int(min(n, max(32, (0.6 * free_b / (2 * per_chunk)) // 32 * 32)))
    waves = [(w0, min(w0 + wave, n)) for w0 in range(0, n, wave)]
    ws_e = torch.empty(nm.workspace_bytes(wave), dtype=torch.uint8, device=dev)
    ws_d = torch.empty_like(ws_e)
    stream = torch.cuda.current_stream(dev)
    S = max(1, args.segment)
    segs = [(a, min(a + S, maxL)) for a in range(1, max(maxL, 2), S)]
    nseg = len(segs)
    n_units = nseg * len(waves)            # one pass: every segment of every wave

    def unit(k):
        """Step k's (wave, segment): the segments of a wave in order, then the next wave."""
        k %= n_units
        return waves[k // nseg], segs[k % nseg]

    def seg_bytes(k):
        """Input bytes a step accounts for: its coded positions, plus the raw
        first byte of every chunk for a wave's first segment."""
        (w0, w1), (a, b) = unit(k)
        coded = int(np.clip(np.minimum(lens_np[w0:w1], b) - a, 0, None).sum())
        return coded + ((w1 - w0) if a == 1 else 0)

    def step(k):
        (w0, w1), (a, b) = unit(k)
        words, sizes = codec.encode_device(model, X[w0:w1], Ld[w0:w1], workspace=ws_e, pos_begin=a, pos_end=b)
        e_mid = torch.cuda.Event(enable_timing=True)
        e_mid.record(stream)
        codec.decode_device(model, words, sizes, Ld[w0:w1], first[w0:w1], workspace=ws_d, pos_begin=a, pos_end=b,
                            out=out[w0:w1])
        return sizes, e_mid

    def verify(steps_done):
        """Decoded bytes equal the input wherever the steps so far decoded."""
        for k in range(min(steps_done, n_units)):
            (w0, w1), (a, b) = unit(k)
            o, x = out[w0:w1, a:b], X[w0:w1, a:b]
            mask = torch.arange(a, b, device=dev)[None, :] < Ld[w0:w1, None]
            if not torch.equal(o[mask], x[mask]):
                raise RuntimeError("round trip mismatch")

    def barrier():
        if dist is not None:
            dist.barrier()

    # warm-up: the first W segments of a separate pass, checked
    for w in range(max(args.warmup, 1)):
        step(w)
    nm.check()
    verify(max(args.warmup, 1))

    # timed device-resident region
    out.zero_()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    mids, sizes_l = [], []
    barrier()
    torch.cuda.synchronize(dev)
    with ClockSampler(local_rank) as clk:
        for k in range(args.steps):
            ev[k][0].record(stream)
            sz, e_mid = step(k)
            ev[k][1].record(stream)
            mids.append(e_mid)
            sizes_l.append(sz)
        torch.cuda.synchronize(dev)
    barrier()
    nm.check()
    verify(args.steps)
    t_c = sum(ev[k][0].elapsed_time(mids[k]) for k in range(args.steps)) / 1000.0
    t_d = sum(mids[k].elapsed_time(ev[k][1]) for k in range(args.steps)) / 1000.0
    step_bytes = [seg_bytes(k) for k in range(args.steps)]
    bytes_timed = sum(step_bytes)
    coded_timed = sum(b - ((unit(k)[0][1] - unit(k)[0][0]) if unit(k)[1][0] == 1 else 0)
                      for k, b in enumerate(step_bytes))
    words_timed = sum(int(sz.to(torch.int64).sum().item()) for sz in sizes_l)
    tt = torch.tensor([t_c + t_d, t_c, t_d], dtype=torch.float64, device=dev)
    if dist is not None:
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
    t_tot, t_c, t_d = (float(x) for x in tt.cpu())
    # every rank codes the same amount (weak) or its share (strong): sum over ranks
    bt = torch.tensor([bytes_timed], dtype=torch.float64, device=dev)
    if dist is not None:
        dist.all_reduce(bt)
    job_bytes = float(bt.item())
    value = job_bytes / MiB / t_tot

    # end-to-end through the public host API, from pinned host segments
    e2e = None
    if not args.no_e2e:
        del ws_e, ws_d
        torch.cuda.empty_cache()
        n_host = min(args.steps, n_units)
        host_segs = []
        for k in range(n_host):
            (w0, w1), (a, b) = unit(k)
            hseg = torch.zeros((w1 - w0, b - a + 1), dtype=torch.uint8).pin_memory()
            hseg.numpy()[:] = arr[w0:w1, a - 1:b]
            host_segs.append(hseg)
        h2d = d2h = 0
        outs = []
        rcod, rwave = None, None
        barrier()
        torch.cuda.synchronize(dev)
        t0 = time.perf_counter()
        for k in range(args.steps):
            (w0, w1), (a, b) = unit(k)
            if rwave != (w0, w1):                     # a new wave: a coder for its chunks
                rcod = None
                rcod, rwave = codec.RangeCodec(model, lens[w0:w1], arr[w0:w1, 0], device=dev), (w0, w1)
            hseg = host_segs[k % n_units]
            w_h, s_h = rcod.encode(hseg, a, b)
            o_h = rcod.decode(w_h, s_h, a, b)
            h2d += hseg.numel() + w_h.nbytes + s_h.nbytes
            d2h += w_h.nbytes + s_h.nbytes + o_h.nbytes
            if k < n_units:
                outs.append(o_h)
        torch.cuda.synchronize(dev)
        te = torch.tensor([time.perf_counter() - t0], dtype=torch.float64, device=dev)
        if dist is not None:
            dist.all_reduce(te, op=dist.ReduceOp.MAX)
        for k, o_h in enumerate(outs):
            (w0, w1), (a, b) = unit(k)
            ref = arr[w0:w1, a:b].copy()
            ref[np.arange(b - a)[None, :] >= (lens_np[w0:w1] - a)[:, None]] = 0
            if not np.array_equal(o_h, ref):
                raise RuntimeError("e2e round trip mismatch")
        e2e = {"value": job_bytes / MiB / float(te.item()), "unit": "MiB/s",
               "h2d_bytes_per_step": h2d // args.steps, "d2h_bytes_per_step": d2h // args.steps,
               "api": "codec.RangeCodec.encode / decode (pinned host segments in, host words and bytes out)"}
        barrier()

    if rank != 0:
        return
    sb = state_bytes_per_coded_byte(cfg["d"], cfg["L"])
    peak, peak_src = measured_peak()
    tpb = traffic_per_coded_byte(cfg["d"], cfg["L"], fmt, "decode")
    # dominant kernel: the decode launch (one position per kernel step)
    alg_d = sb * coded_timed + bytes_timed + 4 * words_timed
    ach_d = alg_d / t_d / 1e9
    roof = {"bound": "hbm", "kernel": "k_boa_step decode launch (fused model+quantiser+coder, one position per step)",
            "achieved": ach_d, "peak": peak, "unit": "GB/s", "frac": ach_d / peak, "peak_source": peak_src,
            "traffic": (tpb * coded_timed / args.steps if tpb else None),
            "algorithmic_bytes_per_launch": alg_d / args.steps,
            "per_unit": f"{sb} B recurrent-state read+write per coded byte"}
    # encode launch: time blocks of tb positions read and write the state once
    # per block; tb is what the library chose for a wave's segment launch
    (w0, w1), (a0, a1) = unit(0)
    tb = nm.time_block(w1 - w0, a1 - a0)
    alg_c = sb * coded_timed // tb + bytes_timed + 4 * words_timed
    ach_c = alg_c / t_c / 1e9
    tpb_c = traffic_per_coded_byte(cfg["d"], cfg["L"], fmt, "encode", tb)
    roof_c = {"bound": "hbm", "kernel": f"k_boa_step encode launch (time blocks of {tb} positions)",
              "achieved": ach_c, "peak": peak, "unit": "GB/s", "frac": ach_c / peak,
              "traffic": (tpb_c * coded_timed / args.steps if tpb_c else None),
              "algorithmic_bytes_per_launch": alg_c / args.steps,
              "per_unit": f"{sb // tb} B recurrent-state read+write per coded byte"}
    # tensor pipe: the model's projection FLOPs, and what the split kind issues
    macs = gemm_macs_per_byte(cfg["d"], cfg["L"])
    products = {"tf32x3": 4, "f16x2": 4}.get(fmt, 1)   # tensor products issued per multiply
    tf_peak, tf_src = measured_tensor_peak(fmt)
    fl_d = 2.0 * macs * coded_timed * products / t_d / 1e12
    roof_t = {"bound": "tensor", "kernel": "k_boa_step decode launch, projections",
              "achieved": fl_d, "peak": tf_peak, "unit": "TFLOP/s", "frac": fl_d / tf_peak, "peak_source": tf_src,
              "per_unit": f"{2 * macs} model FLOP per coded byte x {products} tensor products per multiply "
                          f"({fmt})"}
    cpu, size_ref = None, None
    if world == 1 and not args.no_cpu_baseline:
        cpu, sample, ref_bits = cpu_baseline(cfg, arr, lens)
        xs = [torch.from_numpy(c).reshape(1, -1) for c in sample]
        comp, _, _ = codec.compress_GPU(model, xs, device=dev)
        gpu_bits = 32 * sum(len(c) for c in comp)
        size_ref = {"ratio": gpu_bits / ref_bits, "bits_gpu": gpu_bits, "bits_reference_path": ref_bits,
                    "sample": cpu["sample"].replace(", compress + decompress", ""),
                    "reference_path": "fp32 model, softmax, build_cdf_fast at PRECISION 24, reference range coder "
                                      "(oracle/codec_oracle.py)",
                    "gpu_path": f"{fmt} kernel, integer quantiser at PRECISION 16, whole-chunk streams"}
    passes = args.steps / n_units
    line = {
        "metric": "compress+decompress round-trip throughput", "value": value, "unit": "MiB/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1000.0 * t_tot / args.steps, "higher_is_better": True, "scaling": args.scaling,
        "vs_baseline": None, "dtype": DTYPES[fmt],
        "data": "synthetic (seeded HEP-like records, random-init seeded weights)",
        "config": {"workload": cfg["name"], "chunks_per_gpu": n, "chunk_len": maxL, "bytes_per_gpu": total_bytes,
                   "step": f"positions [a, a + {S}) of every chunk of a wave of {wave} chunks, recurrent state "
                           f"carried between steps; {n_units} steps make one pass over the input "
                           f"({passes:.2f} passes timed)",
                   "weights": fmt, "precision": codec.PRECISION,
                   "parallelism": f"chunk shards x{world} ({args.scaling})",
                   "l2": "inputs larger than L2: recurrent state %d MB per side" %
                         (sb * min(wave, n) // 2 // 1000000)},
        "compress_MiBps": job_bytes / MiB / t_c,
        "decompress_MiBps": job_bytes / MiB / t_d,
        "compress_MBps_1e6": job_bytes / 1e6 / t_c,
        "decompress_MBps_1e6": job_bytes / 1e6 / t_d,
        "bits_per_byte": 32.0 * words_timed / bytes_timed,
        "size_vs_reference": size_ref,
        "roofline": roof, "roofline_encode": roof_c, "roofline_tensor": roof_t, "cpu_baseline": cpu, "e2e": e2e,
        "clocks": clk.summary(), "gpu_launches": 2 * args.steps,
    }
    print(json.dumps(line), flush=True)

# ---------------------------------------------------------------------------
def _coder_slab(n_streams, n_steps, seed, device):
    """Logits ~ N(0, 3^2) and symbols drawn from their softmax, [steps, streams]."""
    import torch
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    logits = torch.randn((n_steps, n_streams, 256), generator=g, device=device) * 3.0
    sym = torch.empty((n_steps, n_streams), dtype=torch.int32, device=device)
    for i in range(n_steps):
        sym[i] = torch.multinomial(torch.softmax(logits[i], -1), 1, generator=g).view(-1).to(torch.int32)
    return logits, sym


def coder_cpu_baseline(seconds_target=15.0):
    """The CPU coder oracle (BQ quantiser, 2^16) on a bounded sample of config 5,
    on every host thread: the streams are split into one contiguous share per
    thread (the C coder releases the GIL, and streams are independent)."""
    import concurrent.futures as cf
    import numpy as np
    import torch
    from oracle import orc
    n_thr = min(64, max(1, os.cpu_count() or 1))   # at most 64 shares (<= 270 MB of logits)
    per, t = 16, 256                     # streams per thread, symbols per stream
    n = per * n_thr
    logits, sym = _coder_slab(n, t, 4, torch.device("cpu"))
    rows = logits.permute(1, 0, 2).contiguous().numpy()
    syms = sym.t().contiguous().numpy()
    pitch = (t * 16 + 31) // 32 + 8
    shares = [(np.ascontiguousarray(rows[k * per:(k + 1) * per]), np.ascontiguousarray(syms[k * per:(k + 1) * per]))
              for k in range(n_thr)]
    counts = np.full(per, t, np.int32)
    deadline = time.perf_counter() + seconds_target / 3

    def work(share):
        r, sy = share
        reps, ok = 0, True
        while True:
            w, sz, st = orc.encode(r, sy, counts, 16, orc.MODE_BQ, pitch)
            out = orc.decode(r, w, sz, counts, 16, orc.MODE_BQ)
            ok = ok and st == 0 and np.array_equal(out, sy)
            reps += 1
            if time.perf_counter() > deadline:
                return reps, ok

    t0 = time.perf_counter()
    with cf.ThreadPoolExecutor(max_workers=n_thr) as ex:
        res = list(ex.map(work, shares))
    dt = time.perf_counter() - t0
    assert all(ok for _, ok in res)
    done = sum(r for r, _ in res) * per * t
    return {"value": done / MiB / dt, "unit": "MiB/s", "cores": n_thr, "kind": "port",
            "sample": f"{n_thr} threads x {per} streams x {t} symbols, encode + decode, repeated until "
                      f"{seconds_target / 3:.0f} s"}


def run_coder(args, cfg, rank, world, local_rank, dist):
    """Config 5: the range coder alone.  Each stream codes one symbol per step
    from 256 fp32 logits (in-kernel BQ quantiser, total 2^16).  A slab of
    `slab` steps of logits and symbols is generated on the device (untimed) and
    cycled through by the multi-step entry points boa_rc_encode_steps /
    boa_rc_decode_steps (one launch per direction, coder state in registers)."""
    import ctypes
    import numpy as np
    import torch
    import codec
    from boa_b200 import _native as _n
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    N = cfg["streams"]
    S = cfg["slab"]
    T = max(S, ((args.size or cfg["symbols"]) // S) * S)
    t0 = time.perf_counter()
    logits, sym = _coder_slab(N, S, 4 + 1000 * rank, dev)
    torch.cuda.synchronize(dev)
    t_gen = time.perf_counter() - t0
    pitch = codec.pitch_words_for(T + 1, 16)
    lib = _n.load()

    def one_round_trip(timed):
        h = ctypes.c_void_p()
        _n.call("boa_rc_create", ctypes.byref(h), N, 256, pitch, 16, _n.BOA_QUANT_BQ, local_rank)
        try:
            out = torch.full((S, N), -1, dtype=torch.int32, device=dev)
            stream = torch.cuda.current_stream(dev)
            sp = ctypes.c_void_p(stream.cuda_stream)
            e0, e1, e2 = (torch.cuda.Event(enable_timing=True) for _ in range(3))
            if dist is not None:
                dist.barrier()
            torch.cuda.synchronize(dev)
            e0.record(stream)
            _n.call("boa_rc_encode_steps", h, T, S, ctypes.c_void_p(sym.data_ptr()), N,
                    ctypes.c_void_p(logits.data_ptr()), N * 256, None, 0, sp)
            _n.call("boa_rc_finalize", h, sp)
            e1.record(stream)
            _n.call("boa_rc_init_decoder", h, sp)
            _n.call("boa_rc_decode_steps", h, T, S, ctypes.c_void_p(logits.data_ptr()), N * 256,
                    ctypes.c_void_p(out.data_ptr()), N, None, 0, sp)
            e2.record(stream)
            torch.cuda.synchronize(dev)
            sizes = np.zeros(N, np.int32)
            _n.call("boa_rc_get_sizes", h, sizes.ctypes.data_as(ctypes.c_void_p), sp)
            # the decoder ends on the last slab pass: any earlier error would derail it
            if not torch.equal(out, sym):
                raise RuntimeError("coder round trip mismatch")
            return e0.elapsed_time(e1) / 1000.0, e1.elapsed_time(e2) / 1000.0, int(sizes.astype(np.int64).sum())
        finally:
            lib.boa_rc_destroy(h)

    for _ in range(max(args.warmup, 1)):
        one_round_trip(False)
    te = td = 0.0
    words = 0
    with ClockSampler(local_rank) as clk:
        for _ in range(args.steps):
            a_, b_, words = one_round_trip(True)
            te += a_
            td += b_
    tt = torch.tensor([te + td, te, td], dtype=torch.float64, device=dev)
    if dist is not None:
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
    t_tot, te, td = (float(x) for x in tt.cpu())
    if rank != 0:
        return
    syms_total = N * T
    peak, peak_src = measured_peak()
    code_bytes = 4.0 * words / syms_total
    per_sym = 256 * 4 + code_bytes                     # logits row + the words read back
    ach = per_sym * N * T / (td / args.steps) / 1e9
    roof = {"bound": "hbm", "kernel": "k_rc_decode_bq_steps (all decode steps, one warp per stream)",
            "achieved": ach, "peak": peak, "unit": "GB/s", "frac": ach / peak, "peak_source": peak_src,
            "traffic": None, "algorithmic_bytes_per_launch": per_sym * N * T,
            "per_unit": "1024 B fp32 logits + code bytes per decoded symbol (coder state stays in registers)"}
    line = {
        "metric": "range-coder encode+decode round-trip throughput", "value": world * args.steps * syms_total / MiB / t_tot,
        "unit": "MiB/s (1 symbol = 1 byte)", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1000.0 * t_tot / args.steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32 logits, u32 coder", "data": "synthetic (seeded N(0, 3^2) logits, symbols "
        "drawn from their softmax)",
        "config": {"workload": cfg["name"], "streams_per_gpu": N, "symbols_per_stream": T, "slab_steps": S,
                   "slab_generation_s": t_gen, "l2": "inputs larger than L2: logits slab %d MB" % (S * N * 1024 // 1000000)},
        "encode_Msym_per_s": world * args.steps * syms_total / 1e6 / te,
        "decode_Msym_per_s": world * args.steps * syms_total / 1e6 / td,
        "bits_per_symbol": 32.0 * words / syms_total,
        "roofline": roof, "cpu_baseline": (coder_cpu_baseline() if world == 1 and not args.no_cpu_baseline else None),
        "e2e": None, "clocks": clk.summary(), "gpu_launches": args.steps * 4,
    }
    print(json.dumps(line), flush=True)


def main():
    args = parse()
    cfg = CONFIGS[args.config]
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        if args.config == 5:
            if rank == 0:
                cb = coder_cpu_baseline()
                print(json.dumps({"impl": "reference", "metric": "range-coder encode+decode round-trip throughput",
                                  "value": cb["value"], "unit": "MiB/s (1 symbol = 1 byte)", "n_gpus": world,
                                  "steps": args.steps, "warmup": args.warmup, "higher_is_better": True,
                                  "scaling": "weak", "vs_baseline": None, "dtype": "f32 logits, u32 coder",
                                  "data": "synthetic", "config": {"workload": cfg["name"], "sample": cb["sample"]},
                                  "cpu_baseline": cb, "e2e": {"value": cb["value"], "unit": "MiB/s",
                                                              "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}),
                      flush=True)
            return
        run_reference(args, cfg, rank)
        return
    dist = None
    if world > 1:
        import datetime
        import torch
        import torch.distributed as tdist
        torch.cuda.set_device(local_rank)
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        tdist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600))
        dist = tdist
    try:
        if args.config == 5:
            run_coder(args, cfg, rank, world, local_rank, dist)
        else:
            run_ours(args, cfg, rank, world, local_rank, dist)
    finally:
        if dist is not None:
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
