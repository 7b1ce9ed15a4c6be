"""Bank-sharded decode on 2 and 4 GPUs (one process per GPU, peers mapped over
NVLink): every rank's logits and final residual must equal a single-GPU
context's, bit for bit.  Skipped on boxes with fewer GPUs."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

LAYERS, SEED, TOKENS = 2, 11, 6


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _inputs():
    rng = np.random.default_rng(SEED)
    return rng.normal(0.0, 0.02, size=(TOKENS, 4096)).astype(np.float32)


def _shard_worker(rank, world, port, q):
    import datetime
    import importlib
    import sys
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    import torch.distributed as dist
    pkg = importlib.import_module("4pe_u250_b200")
    synth = importlib.import_module("4pe_u250_b200.synth")
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120))
    try:
        ctx = pkg.Context(device=rank, num_layers=LAYERS, kv_capacity=64, rank=rank, world=world)
        ctx.load_banks(synth.model_banks(LAYERS, SEED))  # loads only the banks this rank holds
        ctx.load_rope()
        ctx.attach_peers()
        x = _inputs()
        outs = []
        for pos in range(TOKENS):
            dist.barrier()
            logits, res = ctx.decode_token(pos, x[pos], want_residual=True)
            outs.append((logits.view(np.uint32).copy(), res.view(np.uint32).copy()))
        dist.barrier()
        q.put((rank, outs))
        ctx.close()
    finally:
        dist.destroy_process_group()


def _single_gpu_reference(pkg, synth):
    ctx = pkg.Context(device=0, num_layers=LAYERS, kv_capacity=64)
    ctx.load_banks(synth.model_banks(LAYERS, SEED))
    ctx.load_rope()
    x = _inputs()
    ref = []
    for pos in range(TOKENS):
        logits, res = ctx.decode_token(pos, x[pos], want_residual=True)
        ref.append((logits.view(np.uint32).copy(), res.view(np.uint32).copy()))
    ctx.close()
    return ref


@pytest.mark.parametrize("world", [2, 4])
def test_sharded_decode_matches_single_gpu(pkg, synth, world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    ref = _single_gpu_reference(pkg, synth)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_shard_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=600) for _ in procs)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for rank in range(world):
        for pos in range(TOKENS):
            assert np.array_equal(got[rank][pos][0], ref[pos][0]), (rank, pos)
            assert np.array_equal(got[rank][pos][1], ref[pos][1]), (rank, pos)
