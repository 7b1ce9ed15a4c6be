"""The AR4 stream driver (4pe_u250_b200/packer.py, mirroring
scripts/autoround_pack_llama2_u250.py main()): a 1-layer AutoRound export
written from known arrays packs into the same device images as the per-matrix
entry points (pinned to the reference packer in test_gpu_pack.py) given the
same arrays, with the norm words in place and the embeddings returned."""
import struct

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

PROJ = [(0, 4096, 4096), (1, 4096, 4096), (2, 4096, 4096), (3, 4096, 4096),
        (4, 11008, 4096), (5, 11008, 4096), (6, 4096, 11008)]


def test_pack_autoround_file(pkg, F, tmp_path):
    import torch
    packer = __import__("4pe_u250_b200.packer", fromlist=["pack_autoround_file"])
    rng = np.random.default_rng(21)
    emb = rng.standard_normal((32000, 4096), dtype=np.float32)
    norms = [rng.random(4096, dtype=np.float32) for _ in range(3)]
    mats = {m: (rng.integers(0, 256, (r, c // 2), dtype=np.uint8),
                (rng.random((r, c // 128), dtype=np.float32) * np.float32(0.05)).astype(np.float32))
            for m, r, c in PROJ}
    head = (rng.standard_normal((32000, 4096), dtype=np.float32) * np.float32(0.02)).astype(np.float32)
    path = tmp_path / "autoround_w4g128.bin"
    with open(path, "wb") as f:
        hdr = struct.pack("<4sIIIIIIII", b"AR4\0", 1, 4096, 11008, 1, 32, 32, 32000, 128)
        f.write(hdr + bytes(256 - len(hdr)))
        f.write(emb.tobytes())
        for m, _, _ in PROJ:
            if m == 0:
                f.write(norms[0].tobytes())
            if m == 4:
                f.write(norms[1].tobytes())
            f.write(mats[m][0].tobytes())
            f.write(mats[m][1].tobytes())
        f.write(norms[2].tobytes())
        f.write(head.tobytes())
    with pkg.Context(num_layers=1, kv_capacity=8) as ctx:
        images, emb_out, h = packer.pack_autoround_file(ctx, str(path))
        assert h["layers"] == 1 and np.array_equal(emb_out, emb)
        want = [torch.zeros(F.BANK_BYTES, dtype=torch.uint8, device="cuda") for _ in range(4)]
        ptrs = [t.data_ptr() for t in want]
        for m, _, _ in PROJ:
            nib, sc = (torch.from_numpy(a).cuda() for a in mats[m])
            ctx.pack_autoround_matrix(0, m, nib.data_ptr(), sc.data_ptr(), ptrs)
        hd = torch.from_numpy(head).cuda()
        ctx.pack_fp32_head(hd.data_ptr(), ptrs)
        for p in range(4):
            for which, layer in ((0, 0), (1, 0), (2, 0)):
                off = F.norm_word_offset(layer, which) * F.WORD_BYTES
                want[p][off:off + 4096] = torch.from_numpy(norms[which][p * 1024:(p + 1) * 1024].view(np.uint8)).cuda()
            assert torch.equal(images[p], want[p]), p
