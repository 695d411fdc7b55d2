"""Copy-engine gather to the root rank (RootWindow) on two GPUs, two processes.

Each rank writes two blocks of its own data into rank 0's buffer with
cudaMemcpyAsync through CUDA IPC; rank 0 checks every byte against what the
ranks hold.  Skipped on a box with fewer than two GPUs.
"""

import os
import socket

import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, results):
    import sys

    import torch.distributed as dist

    here = os.path.dirname(os.path.abspath(__file__))
    sys.path.insert(0, os.path.join(here, "..", "custom-ml-library_b200"))
    from tensorsmith_b200.distributed import RootWindow

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    import datetime

    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        n = 3 * 1024 + 8  # elements per block (bf16), not a multiple of 1 KB
        window = RootWindow((2 * world * n,), torch.bfloat16, dev)
        assert window.ok
        stream = torch.cuda.Stream(device=dev)
        blocks = []
        for blk in range(2):
            src = torch.arange(n, device=dev, dtype=torch.float32).mul_(0.5).add_(1000 * rank + 100 * blk)
            src = src.to(torch.bfloat16)
            blocks.append(src)
            stream.wait_stream(torch.cuda.current_stream())
            window.put(src, 2 * ((blk * world + rank) * n), stream)
        torch.cuda.current_stream().wait_stream(stream)
        window.done(dev)
        expected = [None] * world
        dist.all_gather_object(expected, [b.cpu() for b in blocks])
        ok = True
        if rank == 0:
            got = window.buffer.cpu().view(2, world, n)
            for r in range(world):
                for blk in range(2):
                    ok &= torch.equal(got[blk, r], expected[r][blk])
        window.close()
        results.put((rank, ok))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_root_window_copy_engine_gather():
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    results = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, results)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=180)
    for p in procs:
        if p.is_alive():
            p.kill()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    got = dict(results.get(timeout=5) for _ in procs)
    assert got == {0: True, 1: True}
