"""Regenerates tests/golden/packer_golden.json (digests of the C packer on a
seeded matrix).  The digests were cross-checked against the reference's own
pack_matrix_to_super_blocks (test_c_packer_matches_reference_python_packer)
in a container where the reference tree was mounted."""
import hashlib
import importlib
import json
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
sys.path.insert(0, os.path.dirname(HERE))

from test_synth_packer import _small_case  # noqa: E402

synth = importlib.import_module("4pe_u250_b200.synth")
w, s, M, K = _small_case()
out = {"pack_arrays": {str(b): hashlib.sha256(synth.pack_arrays(w, s, b, M // 128, K // 1024).tobytes()).hexdigest()
                       for b in range(4)}}
json.dump(out, open(os.path.join(HERE, "packer_golden.json"), "w"), indent=1)
print(out)
