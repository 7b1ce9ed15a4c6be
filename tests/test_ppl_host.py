"""Host logic of Context.perplexity (no GPU): chunk boundaries, the break on
a chunk shorter than 2 tokens and the in-order double sum of the emulator's
loop (calculate_perplexity, emulator:1852-1944), with a stand-in for the
device call i4d_eval_nll."""
import math

import numpy as np
import pytest


class _FakeCtx:
    kv_capacity = 0

    def __init__(self):
        self.calls = []

    def eval_nll(self, ids):
        ids = np.asarray(ids)
        self.calls.append(ids.copy())
        return (ids[1:].astype(np.float64) * 0.001) + 1.0 / (1.0 + ids[:-1])


def _reference_loop(ids, chunk):
    total, count = 0.0, 0
    for start in range(0, (len(ids) + chunk - 1) // chunk * chunk, chunk):
        end = min(len(ids), start + chunk)
        if end - start < 2:
            break
        for pos in range(end - start - 1):
            total += float(ids[start + pos + 1]) * 0.001 + 1.0 / (1.0 + float(ids[start + pos]))
            count += 1
    return total / count, math.exp(total / count), count


@pytest.mark.parametrize("n,chunk", [(2, 4096), (45, 20), (41, 20), (40, 20), (100, 7)])
def test_perplexity_chunk_loop(pkg, n, chunk):
    ids = np.random.default_rng(n).integers(3, 32000, n).astype(np.int32)
    ctx = _FakeCtx()
    loss, ppl, count = pkg.Context.perplexity(ctx, ids, chunk=chunk)
    want = _reference_loop(ids, chunk)
    assert count == want[2]
    assert loss == pytest.approx(want[0], rel=1e-15) and ppl == pytest.approx(want[1], rel=1e-15)
    assert all(len(c) >= 2 and len(c) <= chunk for c in ctx.calls)


def test_perplexity_default_chunk_and_short_input(pkg):
    ctx = _FakeCtx()
    ids = np.arange(3, 5003, dtype=np.int32)
    pkg.Context.perplexity(ctx, ids)
    assert [len(c) for c in ctx.calls] == [4096, 904]  # MAX_SEQ_LEN chunks when the capacity is unset
    with pytest.raises(ValueError):
        pkg.Context.perplexity(_FakeCtx(), np.array([7], np.int32))
