"""i4d_linear_bank_noalloc: the linear stage with its scratch in a static
device array, called through the C ABI on caller-owned device buffers.

Its partials must equal those of i4d_linear_bank (tolerance: bit-exact) on
two calls in a row, and streams larger than the static scratch must be
rejected with I4D_ERR_SIZE.  The file is named to be collected last, so it
also runs after every other GPU test in the same process.
"""
import numpy as np
import pytest

import kat_vectors as K

pytestmark = pytest.mark.gpu

SUPERBLOCK = 4224 * 64
MAX_SUPERBLOCKS = 22


@pytest.fixture(scope="module")
def nctx(pkg):
    return pkg.Context(num_layers=1, kv_capacity=16)


def _random_case(seed, lit, out_tiles):
    rng = np.random.default_rng(seed)
    sb = rng.integers(0, 256, size=out_tiles * lit // 16 * SUPERBLOCK, dtype=np.uint8)
    q = rng.integers(-8191, 8192, size=lit * 256).astype(np.int16)
    e = rng.integers(120, 141, size=lit * 8).astype(np.uint8)
    return sb, q, e


def _noalloc(ctx, sb, lit, out_tiles, q, e, hls_zero_start):
    import torch
    dev = torch.device("cuda", 0)
    sb_d = torch.from_numpy(sb).to(dev)
    q_d = torch.from_numpy(q).to(dev)
    e_d = torch.from_numpy(e).to(dev)
    outs = []
    for _ in range(2):
        out_d = torch.full((out_tiles * 128,), float("nan"), dtype=torch.float32, device=dev)
        torch.cuda.synchronize()
        ctx.linear_bank_noalloc(sb_d.data_ptr(), sb.nbytes, lit, out_tiles, q_d.data_ptr(), e_d.data_ptr(),
                                out_d.data_ptr(), hls_zero_start=hls_zero_start)
        outs.append(out_d.cpu().numpy())
    return outs


def _bits(a):
    return np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)


@pytest.mark.parametrize("mode,out_tiles,pattern", K.LINEAR_CASES)
def test_noalloc_matches_linear_bank_kat(nctx, mode, out_tiles, pattern):
    model, lit, q, e, expected = K.linear_case(mode, out_tiles, pattern)
    sb = np.ascontiguousarray(model).reshape(-1)
    for hls in (True, False):
        ref = nctx.linear_bank(sb, lit, out_tiles, q, e, hls_zero_start=hls)
        first, second = _noalloc(nctx, sb, lit, out_tiles, q, e, hls)
        assert _bits(first).tolist() == _bits(ref).tolist()
        assert _bits(second).tolist() == _bits(ref).tolist()
        if hls:  # the testbench's expected partials assume the HLS chain start
            assert _bits(first).tolist() == _bits(expected).tolist()


@pytest.mark.parametrize("lit,out_tiles", [(4, 32), (4, 88), (11, 32)])
def test_noalloc_matches_linear_bank_decoder_slices(nctx, lit, out_tiles):
    # O-sized (8 superblocks), GATE/UP-sized and DOWN-sized (22: the limit).
    sb, q, e = _random_case(1000 + lit * out_tiles, lit, out_tiles)
    ref = nctx.linear_bank(sb, lit, out_tiles, q, e, hls_zero_start=False)
    first, second = _noalloc(nctx, sb, lit, out_tiles, q, e, False)
    assert _bits(first).tolist() == _bits(ref).tolist()
    assert _bits(second).tolist() == _bits(ref).tolist()


def test_noalloc_allocates_no_device_memory(nctx):
    # The entry point's defining property: after a first call (which looks up
    # the static array's address), further calls leave the device's free
    # memory exactly where it was.  Every buffer is made before the baseline.
    import torch
    lit, out_tiles = 11, 32
    sb, q, e = _random_case(77, lit, out_tiles)
    dev = torch.device("cuda", 0)
    sb_d, q_d, e_d = (torch.from_numpy(a).to(dev) for a in (sb, q, e))
    out_d = torch.zeros(out_tiles * 128, dtype=torch.float32, device=dev)
    args = (sb_d.data_ptr(), sb.nbytes, lit, out_tiles, q_d.data_ptr(), e_d.data_ptr(), out_d.data_ptr())
    torch.cuda.synchronize()
    nctx.linear_bank_noalloc(*args)
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info(0)
    for _ in range(5):
        nctx.linear_bank_noalloc(*args)
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info(0)
    assert free1 == free0, (free0, free1)


@pytest.mark.parametrize("lit,out_tiles", [(4, 92), (4, 252)])
def test_noalloc_rejects_streams_beyond_the_scratch(pkg, nctx, lit, out_tiles):
    import torch
    n = out_tiles * lit // 16 * SUPERBLOCK
    assert n > MAX_SUPERBLOCKS * SUPERBLOCK
    dev = torch.device("cuda", 0)
    sb_d = torch.zeros(n, dtype=torch.uint8, device=dev)
    q_d = torch.zeros(lit * 256, dtype=torch.int16, device=dev)
    e_d = torch.zeros(lit * 8, dtype=torch.uint8, device=dev)
    out_d = torch.zeros(out_tiles * 128, dtype=torch.float32, device=dev)
    with pytest.raises(pkg.I4DError) as info:
        nctx.linear_bank_noalloc(sb_d.data_ptr(), n, lit, out_tiles, q_d.data_ptr(), e_d.data_ptr(),
                                 out_d.data_ptr())
    assert info.value.status == pkg.ERR_SIZE
    assert "static scratch" in str(info.value)
