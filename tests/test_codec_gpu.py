"""Fused codec kernel on the GPU: lossless round trips (ragged and edge-case
chunks, reordered batches, BoaFile container), tables bit-exact with the CPU
quantiser, compressed size against the oracle's ideal code length."""
import os

import numpy as np
import pytest
import torch

from oracle import orc
from oracle import model_oracle as mo

pytestmark = pytest.mark.gpu


def _model(d=64, L=2, fmt="tf32x3"):
    from model import seeded_model
    return seeded_model(d, L, weight_format=fmt)


def _chunks(seed, lens, alphabet=256):
    rng = np.random.default_rng(seed)
    return [torch.from_numpy(rng.integers(0, alphabet, (1, n)).astype(np.uint8)) for n in lens]


@pytest.mark.parametrize("fmt", ["tf32x3", "f16x2", "tf32", "fp16"])
def test_roundtrip_ragged(fmt):
    import codec
    m = _model(fmt=fmt)
    lens = [1, 2, 3, 17, 100, 333, 64, 1, 250] * 3
    xs = _chunks(1, lens)
    comp, first, Ls = codec.compress_GPU(m, xs)
    assert Ls == lens and first == [int(x[0, 0]) for x in xs]
    assert len(comp[0]) == 0           # a one-byte chunk codes nothing (boa stores byte 0 raw)
    outs = codec.decompress_GPU(m, comp, Ls, first)
    for x, o in zip(xs, outs):
        assert np.array_equal(x.numpy(), o)


def test_decode_in_another_batch_order():
    """Probabilities do not depend on which chunks share a CTA: decode a
    permuted subset of what was encoded together."""
    import codec
    m = _model()
    lens = [40 + 7 * i for i in range(37)]
    xs = _chunks(2, lens)
    comp, first, Ls = codec.compress_GPU(m, xs)
    idx = list(range(36, -1, -2)) + [5]
    outs = codec.decompress_GPU(m, [comp[i] for i in idx], [Ls[i] for i in idx], [first[i] for i in idx])
    for j, i in enumerate(idx):
        assert np.array_equal(xs[i].numpy(), outs[j])


def test_stream_matches_cpu_coder_on_gpu_logits():
    """The in-kernel quantiser + coder equal the CPU oracle coder run on the
    kernel's own logits (tables bit-exact, bitstream bit-exact)."""
    import codec
    m = _model()
    lens = [30, 55, 9]
    xs = _chunks(3, lens)
    comp, first, Ls = codec.compress_GPU(m, xs)
    maxL = max(lens)
    toks = np.zeros((3, maxL), np.int64)
    for i, x in enumerate(xs):
        toks[i, :lens[i]] = x.numpy()[0]
    lg = m(torch.from_numpy(toks).cuda()).cpu().numpy()        # logits for next byte
    rows = lg[:, :-1]                                           # predict byte t from prefix < t
    syms = toks[:, 1:].astype(np.int32)
    counts = np.array([n - 1 for n in lens], np.int32)
    w, s, st = orc.encode(rows, syms, counts, 16, orc.MODE_BQ, pitch=64)
    assert st == 0
    for i in range(3):
        assert np.array_equal(comp[i], w[i, :s[i]]), i


def test_boafile_roundtrip_config1(tmp_path):
    from boa import BOA
    from boa_b200 import synthetic
    data = synthetic.config_data(1)[:96 * 1024]
    src = tmp_path / "in.bin"; src.write_bytes(data)
    m = _model()
    bf = BOA("cuda", str(tmp_path / "out.boa"), m)
    bf.compress(str(src), chunks_count=16, progress=False)
    out = BOA("cuda", str(tmp_path / "out.boa"), m).decompress(progress=False)
    assert out == data
    meta = bf.get_metadata()
    assert meta["n_chunks"] == 16 and meta["uncompressed_len"] == len(data)


def test_boafile_input_errors(tmp_path):
    """boa.py:164 and codec.py:24-28: an empty input is a ValueError, a split
    that leaves a chunk shorter than one byte an AssertionError; a file that is
    not BOA2 is a ValueError on read."""
    from boa import BOA
    m = _model()
    empty = tmp_path / "empty.bin"; empty.write_bytes(b"")
    with pytest.raises(ValueError, match="empty"):
        BOA("cuda", str(tmp_path / "e.boa"), m).compress(str(empty), progress=False)
    one = tmp_path / "one.bin"; one.write_bytes(b"x")
    with pytest.raises(AssertionError):
        BOA("cuda", str(tmp_path / "o.boa"), m).compress(str(one), chunks_count=16, progress=False)
    junk = tmp_path / "junk.boa"; junk.write_bytes(b"NOPE" + bytes(64))
    with pytest.raises(ValueError):
        BOA("cuda", str(junk), m).decompress(progress=False)


def test_compressed_size_vs_oracle_ideal():
    """Code length within 0.5% of the oracle's ideal -sum log2 p (fp64 model,
    exact softmax) over the coded bytes, plus the 2-3 flush words per chunk."""
    import codec
    from boa_b200 import synthetic
    m = _model()
    data = np.frombuffer(synthetic.config_data(1)[:8 * 2048], dtype=np.uint8).reshape(8, 2048)
    xs = [torch.from_numpy(r.copy()).reshape(1, -1) for r in data]
    comp, first, Ls = codec.compress_GPU(m, xs)
    bits = sum(32 * len(c) for c in comp)
    sd = {k: v.float() for k, v in m.state_dict().items()}
    lg = mo.forward(sd, mo.config_from_state_dict(sd), torch.from_numpy(data.astype(np.int64)), dtype=torch.float64)
    lp = torch.log_softmax(lg[:, :-1], -1).gather(-1, torch.from_numpy(data[:, 1:].astype(np.int64))[..., None])
    ideal = float(-lp.sum() / np.log(2))
    assert bits <= ideal * 1.005 + 8 * 96, (bits, ideal)


def test_pitch_overflow_is_an_error():
    import codec
    from boa_b200._native import BoaError
    m = _model()
    x = torch.randint(0, 256, (4, 500), dtype=torch.uint8).cuda()
    lens = torch.full((4,), 500, dtype=torch.int32).cuda()
    with pytest.raises(BoaError) as ei:
        codec.encode_device(m, x, lens, pitch_words=8)
        m.native(x.device).check()               # device-side errors surface at the status call
    assert ei.value.code == 3                    # BOA_ERR_OVERFLOW
    m.native(x.device).check()                   # and are cleared once reported


def test_roundtrip_d256_split_and_single():
    """d_model 256 with 16-bit weights: a small batch runs as 2-CTA clusters,
    a large one as single CTAs; streams from either decode in the other."""
    import codec
    m = _model(256, 2, "fp16")
    lens = [60 + (i * 7) % 50 for i in range(40)]
    xs = _chunks(5, lens)
    comp, first, Ls = codec.compress_GPU(m, xs)                 # 40 chunks -> clusters
    outs = codec.decompress_GPU(m, comp, Ls, first)
    assert all(np.array_equal(x.numpy(), o) for x, o in zip(xs, outs))
    # the same chunks inside a large batch (single-CTA decomposition)
    pad = _chunks(6, [60] * 2400)
    comp2, first2, Ls2 = codec.compress_GPU(m, xs + pad)
    assert all(np.array_equal(a, b) for a, b in zip(comp, comp2[:40]))


@pytest.mark.parametrize("d,fmt", [(64, "tf32"), (256, "fp16"), (64, "tf32x3"), (256, "tf32x3"), (64, "f16x2"),
                                   (256, "f16x2")])
def test_time_blocked_encode_matches_one_position_steps(d, fmt):
    """Encode in time blocks of 4 and of 8 positions, and with the block the
    launch chooses (the default), writes the same words as encode one
    position per kernel step, for lengths that end at every offset inside a
    block; decode (always one position per step) reads them back."""
    import codec
    m = _model(d, 2, fmt)
    nm = m.native(torch.device("cuda", 0))
    lens = [1, 2, 3, 4, 5, 6, 7, 8, 9, 15, 16, 17, 63, 64, 65, 130] * 3
    xs = _chunks(9, lens)
    nm.set_time_block(1)
    comp1, first1, Ls1 = codec.compress_GPU(m, xs)
    for tb in (4, 8, 0):
        nm.set_time_block(tb)
        comp, first, Ls = codec.compress_GPU(m, xs)
        assert first1 == first and Ls1 == Ls
        assert all(np.array_equal(a, b) for a, b in zip(comp1, comp)), tb
    outs = codec.decompress_GPU(m, comp, Ls, first)
    assert all(np.array_equal(x.numpy(), o) for x, o in zip(xs, outs))


def test_time_block_choice():
    """The launch's choice between blocks of 4 and 8: 8 when it fills the
    waves of CTAs better (1000 chunks of 2xFP16 at d_model 256: 1000 CTAs of
    one chunk in 7 waves instead of 500 in 4), 4 where blocks of 8 do not fit
    the model's chunk runs; a fixed setting wins."""
    m = _model(256, 2, "f16x2")
    nm = m.native(torch.device("cuda", 0))
    assert nm.time_block(1000, 4096) == 8
    assert nm.time_block(1000, 3) == 1
    assert nm.time_block(16, 128) == 8                             # one wave either way: fewer steps
    for tb in (1, 4, 8):
        nm.set_time_block(tb)
        assert nm.time_block(1000, 4096) == tb
    nm.set_time_block(0)
    small = _model(64, 2, "tf32x3").native(torch.device("cuda", 0))
    assert small.time_block(1000, 4096) == 4                      # chunk runs of 4 columns


def test_boafile_resume_after_interrupted_compress(tmp_path, monkeypatch):
    """BoaFile.compress appends each wave as it is coded; a run that stops
    after two waves resumes with resume=True and ends with the same file as an
    uninterrupted run."""
    from boa import BOA
    from boa_b200 import synthetic
    monkeypatch.setenv("BOA_GPU_STREAMS", "5")
    data = synthetic.config_data(1)[:24000]
    src = tmp_path / "in.bin"
    src.write_bytes(data)
    m = _model()
    one = tmp_path / "one.boa"
    BOA("cuda", str(one), m).compress(str(src), chunks_count=23, progress=False)
    two = tmp_path / "two.boa"
    bf = BOA("cuda", str(two), m)
    calls = {"n": 0}
    real = bf._pack_wave

    def flaky(*a, **k):
        calls["n"] += 1
        if calls["n"] > 3:
            raise KeyboardInterrupt("simulated stop")
        return real(*a, **k)
    bf._pack_wave = flaky
    with pytest.raises(KeyboardInterrupt):
        bf.compress(str(src), chunks_count=23, progress=False)
    BOA("cuda", str(two), m).compress(str(src), chunks_count=23, progress=False, resume=True)
    assert two.read_bytes() == one.read_bytes()
    assert BOA("cuda", str(two), m).decompress(progress=False) == data


def test_roundtrip_d512_bf16():
    """Config-4 model shape (d_model 512, bf16 operands), fewer layers: encode
    in time blocks, decode one position per step, lossless."""
    import codec
    m = _model(512, 2, "bf16")
    lens = [1, 9, 70, 131, 40] * 3
    xs = _chunks(13, lens)
    comp, first, Ls = codec.compress_GPU(m, xs)
    outs = codec.decompress_GPU(m, comp, Ls, first)
    assert all(np.array_equal(x.numpy(), o) for x, o in zip(xs, outs))


@pytest.mark.parametrize("d,L,fmt", [(64, 2, "tf32x3"), (256, 2, "tf32x3"), (256, 2, "fp16"), (256, 2, "f16x2")])
def test_position_ranges_continue_the_model_state(d, L, fmt):
    """Coding [1, a), [a, b), [b, end) as three launches that carry the
    recurrent state in one workspace uses exactly the probabilities of one
    whole-chunk launch: each range's words equal the CPU oracle coder run on
    the whole-sequence logits of that range's positions, and decoding the
    ranges in the same order restores every chunk.  Boundaries fall inside
    and at the edges of 4-position time blocks, and past some chunks' ends."""
    import codec
    m = _model(d, L, fmt)
    dev = torch.device("cuda", 0)
    lens = [1, 5, 37, 70, 71, 96, 129, 130, 200] * 4
    xs = _chunks(21, lens)
    N, maxL = len(lens), max(lens)
    host = np.zeros((N, maxL), np.uint8)
    for i, x in enumerate(xs):
        host[i, :lens[i]] = x.numpy()[0]
    X = torch.from_numpy(host).to(dev)
    Ld = torch.tensor(lens, dtype=torch.int32, device=dev)
    lg = m(X.long()).cpu().numpy()                        # whole-sequence logits (next-byte)
    nm = m.native(dev)
    ws_e = torch.empty(nm.workspace_bytes(N), dtype=torch.uint8, device=dev)
    ws_d = torch.empty_like(ws_e)
    bounds = [1, 38, 71, 131, maxL + 5]
    out = torch.zeros((N, maxL), dtype=torch.uint8, device=dev)
    first = X[:, 0].contiguous()
    for a, b in zip(bounds[:-1], bounds[1:]):
        words, sizes = codec.encode_device(m, X, Ld, workspace=ws_e, pos_begin=a, pos_end=b)
        codec.decode_device(m, words, sizes, Ld, first, workspace=ws_d, pos_begin=a, pos_end=b, out=out)
        nm.check()
        # the oracle coder on the whole-sequence logits of positions [a, min(b, len))
        span = b - a
        rows = np.zeros((N, span, 256), np.float32)
        syms = np.zeros((N, span), np.int32)
        counts = np.zeros(N, np.int32)
        for i, n in enumerate(lens):
            k = max(0, min(b, n) - a)
            counts[i] = k
            if k:
                rows[i, :k] = lg[i, a - 1:a - 1 + k]
                syms[i, :k] = host[i, a:a + k]
        w, s, st = orc.encode(rows, syms, counts, 16, orc.MODE_BQ, pitch=words.shape[1])
        assert st == 0
        wh, sh = words.cpu().numpy().view(np.uint32), sizes.cpu().numpy()
        for i in range(N):
            if counts[i]:
                assert sh[i] == s[i] and np.array_equal(wh[i, :sh[i]], w[i, :s[i]]), (a, b, i)
    assert torch.equal(out.cpu(), torch.from_numpy(host))


def test_range_codec_host_round_trip():
    """codec.RangeCodec (the public host-buffer form of the position ranges,
    what the bench's end-to-end leg calls): segments of host bytes in, words
    out, words in, bytes out; every segment decodes to its input, and the
    words equal those of encode_device over the same ranges."""
    import codec
    m = _model(64, 2)
    dev = torch.device("cuda", 0)
    lens = [1, 3, 50, 99, 100, 101, 257] * 3
    xs = _chunks(31, lens)
    N, maxL = len(lens), max(lens)
    host = np.zeros((N, maxL), np.uint8)
    for i, x in enumerate(xs):
        host[i, :lens[i]] = x.numpy()[0]
    rc = codec.RangeCodec(m, lens, host[:, 0], device=dev)
    X = torch.from_numpy(host).to(dev)
    Ld = torch.tensor(lens, dtype=torch.int32, device=dev)
    ws = torch.empty(m.native(dev).workspace_bytes(N), dtype=torch.uint8, device=dev)
    S = 64
    for a in range(1, maxL, S):
        b = min(a + S, maxL)
        seg = torch.from_numpy(np.ascontiguousarray(host[:, a - 1:b])).pin_memory()
        w, s = rc.encode(seg, a, b)
        out = rc.decode(w, s, a, b)
        ref = host[:, a:b].copy()
        ref[np.arange(b - a)[None, :] >= (np.asarray(lens) - a)[:, None]] = 0
        assert np.array_equal(out, ref), a
        wd, sd = codec.encode_device(m, X, Ld, workspace=ws, pos_begin=a, pos_end=b)
        wd, sd = wd.cpu().numpy().view(np.uint32), sd.cpu().numpy()
        for i in range(N):
            if min(lens[i], b) > a:
                assert s[i] == sd[i] and np.array_equal(w[i, :s[i]], wd[i, :sd[i]]), (a, i)


def test_decompress_refuses_another_operand_kind(tmp_path):
    """The file records the operand kind that coded it (flags bits 16-23);
    decompressing with a model of another kind, whose probabilities differ,
    is a ValueError instead of garbage."""
    from boa import BOA
    from boa_b200 import container as C
    from boa_b200 import synthetic
    data = synthetic.config_data(1)[:8192]
    src = tmp_path / "in.bin"
    src.write_bytes(data)
    out = tmp_path / "o.boa"
    BOA("cuda", str(out), _model(64, 2, "f16x2")).compress(str(src), chunks_count=4, progress=False)
    assert C.flags_weight_format(C.parse(out.read_bytes()).flags) == "f16x2"
    assert BOA("cuda", str(out), _model(64, 2, "f16x2")).decompress(progress=False) == data
    with pytest.raises(ValueError, match="f16x2"):
        BOA("cuda", str(out), _model(64, 2, "tf32x3")).decompress(progress=False)
