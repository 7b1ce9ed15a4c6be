"""The oracle's restatement of the AutoRound packer (oracle.pack_autoround_banks)
against the reference packer's own output: SHA-256 of every bank's
superblocks equal to tests/golden/pack_golden.json, which
tests/golden/gen_pack_golden.py made by running
scripts/autoround_pack_llama2_u250.py on the same seeded inputs."""
import hashlib
import json
import os
import sys

import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "golden"))
import gen_pack_golden as G  # noqa: E402  (seeded inputs only; no reference import)

GOLDEN = json.load(open(os.path.join(HERE, "golden", "pack_golden.json")))


@pytest.mark.parametrize("case", GOLDEN["cases"], ids=[c["name"] for c in GOLDEN["cases"]])
def test_pack_restatement_matches_reference(case):
    import oracle
    inp = G.pack_inputs(case["mode"], case["seed"])
    if case["mode"] == 7:
        banks = oracle.pack_autoround_banks(7, head=inp)
    else:
        banks = oracle.pack_autoround_banks(case["mode"], raw=inp[0], scales=inp[1])
    assert [hashlib.sha256(b.tobytes()).hexdigest() for b in banks] == case["bank_sha256"]
