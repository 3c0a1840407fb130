"""Host logic of the expert-parallel path on CPU (gloo, world size 2): the
expert partition and the in-rank-order exchange of the 64-byte window
handles that smoe_cuda_ep_attach expects. No GPU needed."""
import os
import socket

import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

import smoe_cuda as S


def test_partition_covers_every_expert_once():
    for E, world in [(128, 1), (128, 2), (128, 4), (128, 8)]:
        seen = []
        for r in range(world):
            base, per = S.ep_partition(E, world, r)
            assert per == E // world and base == r * per
            seen += list(range(base, base + per))
        assert seen == list(range(E))
    with pytest.raises(ValueError):
        S.ep_partition(128, 3, 0)
    with pytest.raises(ValueError):
        S.ep_partition(128, 2, 2)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, q):
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    mine = bytes([rank + 1]) * 64            # stands in for a cudaIpcMemHandle blob
    handles = S.ep_exchange_handles(mine, world)
    arr = (S.EpHandle * world)()             # what Context.ep_attach builds
    for r, b in enumerate(handles):
        import ctypes
        ctypes.memmove(arr[r].bytes, b, 64)
    q.put((rank, [bytes(arr[r].bytes) for r in range(world)], S.ep_partition(128, world, rank)))
    dist.barrier()
    dist.destroy_process_group()


def test_handle_exchange_in_rank_order():
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, handles, (base, per) in got:
        assert handles == [bytes([r + 1]) * 64 for r in range(world)]
        assert (base, per) == (rank * 64, 64)


def _rank_absent(rank, world, port, q):
    """Rank 1 joins the process group but never takes part in the handle
    exchange (it exits); rank 0 must get SmoeCudaError within its timeout."""
    import datetime
    import time
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=20))
    if rank == 1:
        time.sleep(8)                        # never exchanges, then leaves
        q.put((rank, "left"))
        return
    t0 = time.monotonic()
    try:
        S.ep_exchange_handles(bytes(64), world, timeout_s=3.0)
        q.put((rank, "no error"))
    except S.SmoeCudaError as e:
        q.put((rank, f"error after {time.monotonic() - t0:.1f} s: {e}"))


def test_handle_exchange_with_an_absent_rank_times_out():
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank_absent, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert got[1] == "left"
    assert got[0].startswith("error after"), got[0]
    assert float(got[0].split()[2]) < 15.0
