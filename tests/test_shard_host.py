"""Host side of bank sharding, on CPU: the bank split and the handle exchange
over torch.distributed (gloo, world size 2, 127.0.0.1)."""
import os
import socket

import pytest
import torch.multiprocessing as mp


def test_shard_banks(pkg):
    assert pkg.shard_banks(0, 1) == [0, 1, 2, 3]
    assert [pkg.shard_banks(r, 2) for r in range(2)] == [[0, 1], [2, 3]]
    assert [pkg.shard_banks(r, 4) for r in range(4)] == [[0], [1], [2], [3]]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _gather_worker(rank, world, port, q):
    import importlib
    import sys
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    import torch.distributed as dist
    pkg = importlib.import_module("4pe_u250_b200")
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=__import__("datetime").timedelta(seconds=60))
    try:
        handle = bytes([rank]) * pkg.SHARD_HANDLE_BYTES
        q.put((rank, pkg.gather_handles(handle)))
    finally:
        dist.destroy_process_group()


def test_gather_handles_rank_order():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_gather_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank in range(2):
        assert got[rank] == [bytes([0]) * 64, bytes([1]) * 64]
