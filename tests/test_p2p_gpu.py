"""One-shot all-reduce over NVLink / NVSwitch peer memory (larql_cuda_p2p_*), the reduction of the
tensor-parallel decode.  Needs two GPUs of one node (skipped otherwise): two processes exchange their CUDA IPC
handles over a gloo group, then sum vectors of several lengths in place; every rank must hold exactly the f32
sum taken in rank order, also through a captured CUDA graph replayed with new data."""
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")
L = pytest.importorskip("larql_cuda")


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _ref(vals):
    s = np.zeros(vals.shape[1], np.float32)
    for r in range(vals.shape[0]):
        s = (s + vals[r]).astype(np.float32)
    return s


def _worker(rank, world, port, out_dir):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    be = L.CudaBackend(rank)
    try:
        h = be.p2p_init(rank, world, 4096)
        hs = [None] * world
        dist.all_gather_object(hs, h)
        be.p2p_connect(hs)
        rng = np.random.default_rng(7)  # the same draws on every rank
        for n in (4096, 1000, 4096, 3, 4096, 2048):
            vals = rng.standard_normal((world, n)).astype(np.float32)
            buf = torch.from_numpy(vals[rank].copy()).cuda()
            be.p2p_allreduce_dev(buf, n)
            be.sync()
            assert np.array_equal(buf.cpu().numpy().view(np.uint32), _ref(vals).view(np.uint32)), n
        # captured and replayed
        stream = torch.cuda.Stream()
        buf = torch.zeros(4096, dtype=torch.float32, device="cuda")
        be.p2p_allreduce_dev(buf, 4096, stream=stream.cuda_stream)  # warm-up call outside the capture
        stream.synchronize()
        be.sync()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            be.p2p_allreduce_dev(buf, 4096, stream=stream.cuda_stream)
        for _ in range(3):
            vals = rng.standard_normal((world, 4096)).astype(np.float32)
            buf.copy_(torch.from_numpy(vals[rank]))
            torch.cuda.synchronize()
            dist.barrier()
            with torch.cuda.stream(stream):
                g.replay()
            stream.synchronize()
            be.sync()
            assert np.array_equal(buf.cpu().numpy().view(np.uint32), _ref(vals).view(np.uint32))
        del g
        dist.barrier()
        open(os.path.join(out_dir, f"ok{rank}"), "w").close()
    finally:
        be.close()
        dist.destroy_process_group()


def test_p2p_allreduce_two_gpus(tmp_path):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp
    mp.spawn(_worker, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True)
    assert all((tmp_path / f"ok{r}").exists() for r in range(2))
