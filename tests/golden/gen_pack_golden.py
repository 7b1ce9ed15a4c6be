"""Generates tests/golden/pack_golden.json: SHA-256 digests of the bank
superblocks the REFERENCE packer (scripts/autoround_pack_llama2_u250.py)
writes for seeded AutoRound inputs.  Run in a container that has the
reference tree (I4D_REF_ROOT; the packer is imported from its scripts/); the digests travel, the
reference does not.

Inputs (reproduced by tests from the seeds, see pack_inputs below):
  AutoRound matrix: raw offset-binary nibbles uint8[M][K/2] and FP32 group-128
  scales [M][K/128] (about 1 % of them exact Q1.15 half-ulp ties, a few
  beyond the Q1.15 range); unpacked as read_ar_matrix does
  (autoround_pack_llama2_u250.py:413-424, nested in main(), restated here
  in four lines), Q/K rows permuted by the reference's permute_qk_rows,
  padded, and packed per bank by its pack_matrix_to_super_blocks.
  FP32 LM head [32000][4096]: packed by the reference's
  pack_logits_into_banks (its max-abs RTN path).
"""
import hashlib
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))

CASES = [  # (name, mode, seed)
    ("q", 0, 101), ("k", 1, 102), ("v", 2, 103), ("gate", 4, 104), ("down", 6, 105), ("head", 7, 106),
]


def valid_shape(mode):
    return {0: (4096, 4096), 1: (4096, 4096), 2: (4096, 4096), 3: (4096, 4096), 4: (11008, 4096),
            5: (11008, 4096), 6: (4096, 11008), 7: (32000, 4096)}[mode]


def pack_inputs(mode, seed):
    """Seeded inputs of one case: (raw nibbles, FP32 scales) or the FP32 head."""
    rng = np.random.default_rng(seed)
    M, K = valid_shape(mode)
    if mode == 7:
        head = (rng.standard_normal((M, K), dtype=np.float32) * np.float32(0.02)).astype(np.float32)
        head[5, :128] = 0.0  # an all-zero group (the 1e-8 floor)
        return head
    raw = rng.integers(0, 256, (M, K // 2), dtype=np.uint8)
    sc = (rng.random((M, K // 128), dtype=np.float32) * np.float32(0.05) + np.float32(1e-4)).astype(np.float32)
    ties = rng.random(sc.shape) < 0.01
    sc[ties] = ((rng.integers(0, 2000, int(ties.sum())) + 0.5) / 32768.0).astype(np.float32)
    sc.flat[rng.integers(0, sc.size, 8)] = np.float32(1.5)   # saturate at +32767
    sc.flat[rng.integers(0, sc.size, 8)] = np.float32(-1.2)  # saturate at -32768
    return raw, sc


def main():
    # Needs the reference tree: I4D_REF_ROOT names it.
    sys.path.insert(0, os.path.join(os.environ["I4D_REF_ROOT"], "scripts"))
    import autoround_pack_llama2_u250 as ref

    out = {"source": "scripts/autoround_pack_llama2_u250.py (pack_matrix_to_super_blocks, permute_qk_rows, "
                     "pack_logits_into_banks)", "cases": []}
    for name, mode, seed in CASES:
        (_, padded_out, _, padded_in, out_tiles, lit, _, _, _) = ref.matrix_shape_info(mode)
        digests = []
        if mode == 7:
            head = pack_inputs(mode, seed)
            start = (ref.DATA_BASE_WORD + ref.get_data_offset(0, ref.MODE_LOGITS)) * ref.WORD_BYTES

            class Capture:
                def __init__(self):
                    self.data = None

                def __setitem__(self, sl, val):
                    assert sl.start == start
                    self.data = np.array(val, dtype=np.uint8)

            banks = [Capture() for _ in range(4)]
            ref.pack_logits_into_banks(banks, head_raw=head)
            digests = [hashlib.sha256(b.data.tobytes()).hexdigest() for b in banks]
        else:
            raw, sc = pack_inputs(mode, seed)
            M, K = valid_shape(mode)
            # read_ar_matrix (autoround_pack_llama2_u250.py:413-424)
            w = np.empty((M, K), dtype=np.int8)
            w[:, 0::2] = (raw & 0x0F).astype(np.int8) - 8
            w[:, 1::2] = (raw >> 4).astype(np.int8) - 8
            s = np.clip(np.round(sc * 32768.0), -32768, 32767).astype(np.int16)
            if mode in (ref.MODE_Q, ref.MODE_K):
                w = ref.permute_qk_rows(w)
                s = ref.permute_qk_rows(s)
            if (padded_out, padded_in) != (M, K):
                w_pad = np.zeros((padded_out, padded_in), dtype=np.int8)
                w_pad[:M, :K] = w
                s_pad = np.zeros((padded_out, padded_in // 128), dtype=np.int16)
                s_pad[:M, :K // 128] = s
                w, s = w_pad, s_pad
            for p in range(4):
                b = ref.pack_matrix_to_super_blocks(p, w, s, out_tiles, lit, padded_out, padded_in)
                digests.append(hashlib.sha256(b.tobytes()).hexdigest())
        out["cases"].append({"name": name, "mode": mode, "seed": seed, "bank_sha256": digests})
        print(name, digests[0][:16], flush=True)
    with open(os.path.join(HERE, "pack_golden.json"), "w") as f:
        json.dump(out, f, indent=1)


if __name__ == "__main__":
    main()
