"""The persistent token kernel past its first attention window: 300 decode
steps (positions 0..299: one full 256-token window, then a second) bit-equal,
logits and residuals at every position, to the staged per-operation path,
whose attention step is pinned bit-exact to the oracle up to position 4095
(test_gpu_ops.py)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

LAYERS, SEED, STEPS = 2, 13, 300


def test_token_kernel_multi_window_matches_staged(pkg, synth, rope_lut):
    banks = synth.model_banks(LAYERS, SEED)
    x = np.random.default_rng(SEED).normal(0.0, 0.02, (STEPS, 4096)).astype(np.float32)
    with pkg.Context(num_layers=LAYERS, kv_capacity=512) as t, \
            pkg.Context(num_layers=LAYERS, kv_capacity=512, flags=pkg.FLAG_STAGED) as s:
        for c in (t, s):
            c.load_banks(banks)
            c.load_rope(rope_lut)
        for pos in range(STEPS):
            lt, rt = t.decode_token(pos, x[pos], want_residual=True)
            ls, rs = s.decode_token(pos, x[pos], want_residual=True)
            assert np.array_equal(lt.view(np.uint32), ls.view(np.uint32)), pos
            assert np.array_equal(rt.view(np.uint32), rs.view(np.uint32)), pos
