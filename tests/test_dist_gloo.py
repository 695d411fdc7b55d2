"""Host-side logic of batch x head sharding, exercised with world_size-2 gloo
ranks on CPU (no GPU): shard bounds cover every pair exactly once and the
gather to rank 0 reassembles the full tensor in pair order."""

import multiprocessing as mp
import os
import socket

import pytest
import torch

from tensorsmith_b200.distributed import ShardPlan, gather_to_root, shard_view


def test_plan_partitions_pairs():
    for world in (1, 2, 3, 4, 8):
        covered = []
        for r in range(world):
            plan = ShardPlan(32, 32, world, r)
            covered.extend(range(plan.start, plan.stop))
        assert covered == list(range(1024))
    assert ShardPlan(32, 32, 8, 3).size == 128
    assert ShardPlan(3, 1, 2, 1).pair_ids() == [(1, 0), (2, 0)]
    with pytest.raises(ValueError):
        ShardPlan(2, 2, 2, 2)


def test_shard_view_of_btdh_layout():
    b, t, h, d = 2, 5, 4, 3
    base = torch.arange(b * t * h * d, dtype=torch.float32).reshape(b, t, h, d)
    x = base.permute(0, 2, 1, 3)
    plan = ShardPlan(b, h, 2, 1)
    view = shard_view(x, plan)
    assert view.shape == (1, 4, t, d) and view.data_ptr() == x[1].data_ptr()
    torch.testing.assert_close(view[0], x[1])
    contiguous = x.contiguous()
    odd = shard_view(contiguous, ShardPlan(b, h, 4, 1))
    assert odd.shape == (1, 2, t, d)
    torch.testing.assert_close(odd[0], contiguous[0, 2:4])
    with pytest.raises(ValueError):
        shard_view(x, ShardPlan(b, h, 4, 1))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, queue):
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=__import__("datetime").timedelta(seconds=20))
    try:
        b, h, t, d = 2, 4, 3, 2
        full = torch.arange(b * h * t * d, dtype=torch.float32).reshape(b, h, t, d)
        plan = ShardPlan(b, h, world, rank)
        local = shard_view(full, plan) * 1.0
        out = gather_to_root(local, plan)
        # block by block, asynchronously, into per-rank strided places of one buffer
        blocks = torch.zeros(world, plan.size, t, d) if rank == 0 else None
        works = []
        for c0 in range(0, plan.size, 2):
            targets = [blocks[r : r + 1, c0 : c0 + 2] for r in range(world)] if rank == 0 else None
            works.append(gather_to_root(local[:, c0 : c0 + 2], plan, out=targets, async_op=True))
        for work in works:
            work.wait()
        # asynchronously into one contiguous full buffer
        whole = torch.zeros(world * plan.size, t, d).reshape(world, plan.size, t, d) if rank == 0 else None
        work = gather_to_root(local, plan, out=whole, async_op=True)
        work.wait()
        # an asynchronous call on the root without `out` would lose its result
        refused = True
        if rank == 0:
            try:
                gather_to_root(local, plan, async_op=True)
                refused = False
            except ValueError:
                pass
        dist.barrier()
        if rank == 0:
            queue.put(("ok", torch.equal(out.reshape(b, h, t, d), full)
                       and torch.equal(blocks.reshape(b, h, t, d), full)
                       and torch.equal(whole.reshape(b, h, t, d), full) and refused))
        else:
            queue.put(("ok", out is None))
    except Exception as error:  # pragma: no cover - reported to the parent
        queue.put(("error", repr(error)))
    finally:
        dist.destroy_process_group()


def test_gather_to_root_world2():
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, queue)) for r in range(2)]
    for p in procs:
        p.start()
    results = [queue.get(timeout=60) for _ in procs]
    for p in procs:
        p.join(timeout=30)
    assert all(kind == "ok" and flag for kind, flag in results), results


def test_gather_to_root_single_rank():
    plan = ShardPlan(2, 2, 1, 0)
    local = torch.arange(2 * 2 * 3 * 4, dtype=torch.float32).reshape(2, 2, 3, 4)
    assert gather_to_root(local, plan) is local
    out = torch.empty_like(local)
    assert gather_to_root(local, plan, out=out) is out and torch.equal(out, local)
    out2 = torch.empty_like(local)
    assert gather_to_root(local, plan, out=out2, async_op=True) is None and torch.equal(out2, local)
    with pytest.raises(ValueError):
        gather_to_root(local, plan, async_op=True)


def _window_worker(rank, world, port, queue):
    import torch.distributed as dist

    from tensorsmith_b200.distributed import RootWindow

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=__import__("datetime").timedelta(seconds=20))
    try:
        # Host memory cannot be exported over CUDA IPC: every rank must learn
        # that the window is unusable (and keep its NCCL path), none may hang.
        window = RootWindow((64,), torch.float32, torch.device("cpu"))
        mapped = window.ok
        has_buffer = window.buffer is not None
        refused = False
        try:
            window.put(torch.zeros(4), 0, None)
        except RuntimeError:
            refused = True
        window.close()
        queue.put(("ok", (not mapped) and has_buffer == (rank == 0) and refused))
    except Exception as error:  # pragma: no cover - reported to the parent
        queue.put(("error", repr(error)))
    finally:
        dist.destroy_process_group()


def test_root_window_falls_back_together_world2():
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_window_worker, args=(r, 2, port, queue)) for r in range(2)]
    for p in procs:
        p.start()
    results = [queue.get(timeout=60) for _ in procs]
    for p in procs:
        p.join(timeout=30)
    assert all(kind == "ok" and flag for kind, flag in results), results
