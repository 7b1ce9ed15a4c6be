"""The bank-image producer on the device (i4d_pack_autoround_matrix,
i4d_pack_fp32_head) against the reference packer: SHA-256 of every bank's
superblocks equal to tests/golden/pack_golden.json (made by running
scripts/autoround_pack_llama2_u250.py on the same seeded inputs); and bank
images loaded from device memory decode exactly as from host memory."""
import hashlib
import json
import os
import sys

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "golden"))
import gen_pack_golden as G  # noqa: E402  (seeded inputs only)

GOLDEN = json.load(open(os.path.join(HERE, "golden", "pack_golden.json")))


@pytest.fixture(scope="module")
def images(F):
    import torch
    imgs = [torch.zeros(F.BANK_BYTES, dtype=torch.uint8, device="cuda") for _ in range(4)]
    yield imgs
    del imgs
    torch.cuda.empty_cache()


@pytest.mark.parametrize("case", GOLDEN["cases"], ids=[c["name"] for c in GOLDEN["cases"]])
def test_gpu_pack_matches_reference(pkg, F, images, case):
    import torch
    mode = case["mode"]
    inp = G.pack_inputs(mode, case["seed"])
    ptrs = [t.data_ptr() for t in images]
    layer = 3
    with pkg.Context(num_layers=1, kv_capacity=8) as ctx:
        if mode == 7:
            head = torch.from_numpy(inp).cuda()
            ctx.pack_fp32_head(head.data_ptr(), ptrs)
            off = F.matrix_word_offset(0, mode) * 64
        else:
            nib = torch.from_numpy(inp[0]).cuda()
            sc = torch.from_numpy(inp[1]).cuda()
            ctx.pack_autoround_matrix(layer, mode, nib.data_ptr(), sc.data_ptr(), ptrs)
            off = F.matrix_word_offset(layer, mode) * 64
    n = F.mode_data_words(mode) * 64
    got = [hashlib.sha256(t[off:off + n].cpu().numpy().tobytes()).hexdigest() for t in images]
    assert got == case["bank_sha256"]


def test_load_bank_from_device_memory(pkg, synth, rope_lut):
    import torch
    banks = synth.model_banks(1, 7)
    x = np.random.default_rng(0).normal(0, 0.02, 4096).astype(np.float32)
    with pkg.Context(num_layers=1, kv_capacity=8) as h, pkg.Context(num_layers=1, kv_capacity=8) as d:
        h.load_banks(banks)
        dev = [torch.from_numpy(b).cuda() for b in banks]
        for p in range(4):
            d.load_bank_device(p, dev[p].data_ptr())
        for c in (h, d):
            c.load_rope(rope_lut)
        a = h.decode_token(0, x)
        b = d.decode_token(0, x)
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
