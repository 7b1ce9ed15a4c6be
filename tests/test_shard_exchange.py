"""The partial exchange of bank sharding, on CPU with gloo ranks: each rank
computes the bank partials of the banks it holds (the oracle's per-bank
chains, emulator:216-264), the ranks all-gather them, and every rank
combines the four in bank order as (p0 + p1) + (p2 + p3)
(int4_linear_controller.cpp:1384-1439).  The result must be bitwise the
single-process GEMV, for groups of 2 and 4 ranks."""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

SEED, LAYER = 31, 0


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _case():
    import importlib
    synth = importlib.import_module("4pe_u250_b200.synth")
    F = importlib.import_module("4pe_u250_b200.formats")
    banks = synth.empty_banks()
    synth.fill_matrix(banks, LAYER, F.MODE_GATE, SEED)
    x = synth.normal(4096, 0.0, 1.0, SEED, synth.STREAM_INPUT)
    return banks, x, F.MODE_GATE


def _worker(rank, world, port, q):
    import datetime
    import importlib
    import sys
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    import torch
    import torch.distributed as dist
    from oracle import Oracle
    pkg = importlib.import_module("4pe_u250_b200")
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120))
    try:
        banks, x, mode = _case()
        orc = Oracle()
        qa, ea = orc.quantize_g32(x)
        _, part = orc.gemv(banks, LAYER, mode, qa, ea)  # every bank's partial; keep only the ones held
        mine = torch.from_numpy(np.ascontiguousarray(part[pkg.shard_banks(rank, world)]))
        got = [torch.empty_like(mine) for _ in range(world)]
        dist.all_gather(got, mine)
        y = pkg.combine_bank_partials(torch.cat(got).numpy())
        q.put((rank, y.view(np.uint32).tobytes()))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_sharded_partials_combine_bit_exact(world, oracle):
    banks, x, mode = _case()
    qa, ea = oracle.quantize_g32(x)
    y, part = oracle.gemv(banks, LAYER, mode, qa, ea)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for r in range(world):
        assert got[r] == y.view(np.uint32).tobytes(), r
    # The order matters: a different pairing of the same partials rounds differently somewhere.
    other = ((part[0] + part[2]) + (part[1] + part[3])).astype(np.float32)
    assert not np.array_equal(other.view(np.uint32), y.view(np.uint32))
