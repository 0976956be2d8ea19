"""Two GPUs: a stream encoded on one GPU decodes on another (the kernels are
device-invariant, so a file written anywhere reads anywhere), and a BOA2 file
written by two NCCL ranks, one GPU each, is byte-identical to the one-GPU
file and decodes on both ranks."""
import datetime
import os
import socket

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
need2 = pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                           reason="needs two GPUs")


def _chunks(seed, lens):
    rng = np.random.default_rng(seed)
    return [torch.from_numpy(rng.integers(0, 256, (1, n)).astype(np.uint8)) for n in lens]


@need2
@pytest.mark.parametrize("d,L,fmt", [(64, 2, "tf32x3"), (256, 8, "tf32x3"), (256, 8, "f16x2"), (64, 2, "f16x2"),
                                     (256, 2, "fp16")])
def test_encode_on_gpu0_decode_on_last_gpu(d, L, fmt):
    """Configuration 3's cross-GPU round trip: encode on GPU 0, decode on the
    box's last GPU (GPU 7 on an 8-GPU box), and re-encode there to the same
    words."""
    import codec
    from model import seeded_model
    last = f"cuda:{torch.cuda.device_count() - 1}"
    m = seeded_model(d, L, weight_format=fmt)
    xs = _chunks(21, [1, 5, 64, 200, 333] * 4)
    comp, first, Ls = codec.compress_GPU(m, xs, device="cuda:0")
    outs = codec.decompress_GPU(m, comp, Ls, first, device=last)
    assert all(np.array_equal(x.numpy(), o) for x, o in zip(xs, outs))
    comp1, _, _ = codec.compress_GPU(m, xs, device=last)
    assert all(np.array_equal(a, b) for a, b in zip(comp, comp1))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank_worker(rank, world, port, data_path, out_path):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    try:
        from boa import BOA
        from model import seeded_model
        m = seeded_model(64, 2)
        BOA("cuda", out_path, m).compress(data_path, chunks_count=24, progress=False)
        dist.barrier()
        got = BOA("cuda", out_path, m).decompress(progress=False)
        with open(data_path, "rb") as f:
            assert got == f.read()
        dist.barrier()
    finally:
        dist.destroy_process_group()


@need2
def test_two_rank_nccl_file_equals_one_gpu_file(tmp_path):
    import torch.multiprocessing as mp
    from boa import BOA
    from boa_b200 import synthetic
    from model import seeded_model
    data = synthetic.config_data(1)[:40000]
    src = tmp_path / "in.bin"
    src.write_bytes(data)
    one = tmp_path / "one.boa"
    torch.cuda.set_device(0)
    BOA("cuda", str(one), seeded_model(64, 2)).compress(str(src), chunks_count=24, progress=False)
    two = tmp_path / "two.boa"
    mp.start_processes(_rank_worker, args=(2, _free_port(), str(src), str(two)), nprocs=2, join=True,
                       start_method="spawn")
    assert one.read_bytes() == two.read_bytes()
