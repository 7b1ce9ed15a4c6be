"""The attention item's windowed state chain, restated on the CPU.

The token kernel's attention item (csrc/i4d_attn_item.cuh) does not run the
reference's token-order state recurrence (emulator:656-685) token by token.
It takes 256-token windows; 16 worker warps of 16 tokens each sum their part
of every run of non-event tokens (pre: before the warp's first event, post:
after its last, the runs between two of its events whole), a run spanning
warps is completed by walking back over the partial sums, and warp 0 applies
the runs as sums and the events one by one -- but only when the state's
magnitude plus the window's sum of |value| fits in int32 and the window has
at most kMaxEv events; otherwise it runs the recurrence token by token.

This file checks that transformation on its own, against the recurrence
(restated from the oracle's attention_head, which is pinned to the compiled
reference emulator), on coefficient and value sequences built to hit every
branch: sparse and dense events, events on warp and window boundaries,
ragged window ends, and values that saturate the int32 state; and that the
coefficient phase, which carries the running maximum from window to window,
gives the reference's coefficients and events.  The GPU parity tests
(tests/test_gpu_ops.py) check the kernel itself against the oracle.
"""
import numpy as np
import pytest

from oracle import Oracle

M30 = (1 << 30) - 1
WIN, WARPS, TPW, MAX_EV = 256, 16, 16, 96
I32_MAX, I32_MIN = (1 << 31) - 1, -(1 << 31)


def rhe(v, sh):
    """Round-half-even arithmetic right shift (emulator:507-517)."""
    return (v + (1 << (sh - 1)) - 1 + ((v >> sh) & 1)) >> sh


def wrap32(v):
    return ((v + (1 << 31)) & 0xFFFFFFFF) - (1 << 31)


def mulq17(a, c):
    return wrap32(rhe(np.asarray(a, np.int64) * np.int64(c), 17))


def sat32(v):
    return np.clip(v, I32_MIN, I32_MAX)


def reference_chain(coef, event, vals):
    """emulator:656-685 as the oracle states it: per token, rescale then add v
    at a new maximum (token 0 starts the state), else add mulq17(v, c);
    saturating at every step.  vals: [tokens][dims] int64 (v8 << shift)."""
    st = np.zeros(vals.shape[1], np.int64)
    z = 0
    for t in range(len(coef)):
        c = int(coef[t])
        if t == 0:
            st = vals[0].copy()
            z = 1 << 17
        elif event[t]:
            st = sat32(mulq17(st, c) + vals[t])
            z = ((int(rhe(z * c, 17)) & M30) + (1 << 17)) & M30
        else:
            st = sat32(st + mulq17(vals[t], c))
            z = (z + c) & M30
    return st, z


def window_chain(coef, event, vals):
    """The item's windowed form (csrc/i4d_attn_item.cuh), window by window."""
    n = len(coef)
    dims = vals.shape[1]
    st = np.zeros(dims, np.int64)
    z = 1 << 17
    for k in range((n + WIN - 1) // WIN):
        t0, cnt = k * WIN, min(WIN, n - k * WIN)
        c = [int(x) for x in coef[t0:t0 + cnt]]
        ev = [bool(x) for x in event[t0:t0 + cnt]]
        # the value of each token: v at an event, else mulq17(v, c)
        x = np.stack([vals[t0 + i] if ev[i] else mulq17(vals[t0 + i], c[i]) for i in range(cnt)])
        nev = sum(ev)
        # run pass: per warp pre / post parts, interior runs, magnitude sums
        pre = np.zeros((WARPS, dims), np.int64)
        post = np.zeros((WARPS, dims), np.int64)
        zpre, zpost = [0] * WARPS, [0] * WARPS
        mag = np.zeros((WARPS, dims), np.int64)
        rs, zs, evv, ec = {}, {}, {}, {}
        mask = []
        for w in range(WARPS):
            lo, hi = w * TPW, min((w + 1) * TPW, cnt)
            before = sum(ev[:lo])
            mine = [i for i in range(lo, max(lo, hi)) if ev[i]]
            mask.append(bool(mine))
            if lo < cnt:
                mag[w] = np.minimum(np.abs(x[lo:hi]).clip(max=I32_MAX).sum(axis=0), 1 << 31)
            r, acc, zacc = before, np.zeros(dims, np.int64), 0
            for i in range(lo, max(lo, hi)):
                if ev[i]:
                    if r == before:
                        pre[w], zpre[w] = acc, zacc
                    else:
                        rs[r], zs[r] = acc, zacc
                    evv[r], ec[r] = x[i], c[i]
                    r, acc, zacc = r + 1, np.zeros(dims, np.int64), 0
                else:
                    acc, zacc = acc + x[i], zacc + c[i]
            if not mine:
                pre[w], zpre[w] = acc, zacc
            else:
                post[w], zpost[w] = acc, zacc
        # walk-back: the run closed by each warp's first event, and the final run
        def walk(w, own_post):
            if own_post:
                return post[w].copy(), zpost[w]
            tot, zt = pre[w].copy(), zpre[w]
            opened = max([u for u in range(w) if mask[u]], default=-1)
            if opened >= 0:
                tot, zt = tot + post[opened], zt + zpost[opened]
            for u in range(opened + 1, w):
                tot, zt = tot + pre[u], zt + zpre[u]
            return tot, zt
        for w in range(WARPS):
            if mask[w]:
                rs[sum(ev[:w * TPW])], zs[sum(ev[:w * TPW])] = walk(w, False)
        rs[nev], zs[nev] = walk(WARPS - 1, mask[WARPS - 1])
        # apply
        fits = (np.abs(st) + mag.sum(axis=0)) <= I32_MAX
        if nev <= MAX_EV and fits.all():
            st = st + rs[0]
            z = (z + zs[0]) & M30
            for e in range(nev):
                if k == 0 and e == 0:
                    st, z = evv[0].copy(), 1 << 17
                else:
                    st = mulq17(st, ec[e]) + evv[e]
                    z = ((int(rhe(z * ec[e], 17)) & M30) + (1 << 17)) & M30
                st = st + rs[e + 1]
                z = (z + zs[e + 1]) & M30
            assert (np.abs(st) <= I32_MAX).all()
        else:
            for i in range(cnt):
                if ev[i]:
                    if t0 + i == 0:
                        st, z = vals[0].copy(), 1 << 17
                    else:
                        st = sat32(mulq17(st, c[i]) + vals[t0 + i])
                        z = ((int(rhe(z * c[i], 17)) & M30) + (1 << 17)) & M30
                else:
                    st = sat32(st + mulq17(vals[t0 + i], c[i]))
                    z = (z + c[i]) & M30
    return st, z


def coefficients(scores, orc):
    """Softmax coefficients and events from the running maximum
    (emulator:656-672), with the oracle's fixed-point exp."""
    coef, event = [1 << 17], [True]
    m = int(scores[0])
    for s in scores[1:]:
        s = int(s)
        if s <= m:
            coef.append(orc.L.i4o_exp_negative_q17(max(s - m, I32_MIN)))
            event.append(False)
        else:
            coef.append(orc.L.i4o_exp_negative_q17(max(m - s, I32_MIN)))
            event.append(True)
            m = s
    return np.array(coef, np.int64), np.array(event)


def values(rng, n, shift_of_t, dims=32):
    v8 = rng.integers(-127, 128, size=(n, dims))
    sh = np.array([shift_of_t(t) for t in range(n)], np.int64)
    return wrap32(v8.astype(np.int64) << sh[:, None])


CASES = {
    # noisy scores with a slow upward drift: sparse events, mostly one run per warp
    "sparse": (700, lambda rng, n: np.cumsum(rng.integers(-40, 44, n)), lambda t: 13),
    # a new maximum on most tokens: windows past kMaxEv events go token by token
    "dense": (530, lambda rng, n: np.arange(n) * 50 + rng.integers(0, 40, n), lambda t: 13),
    # one event every 16 tokens, on the first token of each warp's range
    "warp_edges": (520, lambda rng, n: np.where(np.arange(n) % 16 == 0, np.arange(n) * 100, -10**6), lambda t: 12),
    # events on the last token of each warp's range and at window boundaries
    "warp_ends": (515, lambda rng, n: np.where(np.arange(n) % 16 == 15, np.arange(n) * 100,
                                               np.where(np.arange(n) % 256 == 0, np.arange(n) * 100, -10**6)),
                  lambda t: 12),
    # values near the int32 limit from token 300 on: the second window saturates
    "saturating": (420, lambda rng, n: rng.integers(-200, 200, n), lambda t: 24 if t >= 300 else 6),
    # short context inside one window, ragged end
    "short": (83, lambda rng, n: np.cumsum(rng.integers(-60, 80, n)), lambda t: 14),
}


@pytest.mark.parametrize("name", sorted(CASES))
def test_window_chain_equals_token_recurrence(name):
    n, scores_of, shift_of = CASES[name]
    rng = np.random.default_rng(sum(map(ord, name)))
    orc = Oracle()
    coef, event = coefficients(scores_of(rng, n), orc)
    vals = values(rng, n, shift_of)
    want = reference_chain(coef, event, vals)
    got = window_chain(coef, event, vals)
    assert np.array_equal(got[0], want[0]) and got[1] == want[1]


def test_cases_reach_both_paths():
    """The cases above take the summed path with events in some windows and
    the token-by-token path in others (too many events, or saturation)."""
    orc = Oracle()
    paths = set()
    for name, (n, scores_of, shift_of) in CASES.items():
        rng = np.random.default_rng(sum(map(ord, name)))
        coef, event = coefficients(scores_of(rng, n), orc)
        vals = values(rng, n, shift_of)
        st = np.zeros(32, np.int64)
        for k in range((n + WIN - 1) // WIN):
            t0, cnt = k * WIN, min(WIN, n - k * WIN)
            ev = event[t0:t0 + cnt]
            x = np.stack([vals[t0 + i] if ev[i] else mulq17(vals[t0 + i], int(coef[t0 + i])) for i in range(cnt)])
            summed = ev.sum() <= MAX_EV and ((np.abs(st) + np.abs(x).sum(axis=0)) <= I32_MAX).all()
            paths.add(("summed" if summed else "sequential", bool(ev.sum() > 0)))
            st, _ = reference_chain(coef[:t0 + cnt], event[:t0 + cnt], vals[:t0 + cnt])
    assert ("summed", True) in paths and ("sequential", True) in paths


def window_coefficients(scores, orc):
    """The item's coefficient phase (one warp per 32-token word of a
    window): the running maximum before a token is the largest of the carry
    into the window, the window's earlier words and the prefix of its own
    word; the last word's warp hands max(carry, its prefix) on as the next
    window's carry."""
    n = len(scores)
    coef, event = np.zeros(n, np.int64), np.zeros(n, bool)
    carry = I32_MIN
    for k in range((n + WIN - 1) // WIN):
        t0, cnt = k * WIN, min(WIN, n - k * WIN)
        sc = [int(s) for s in scores[t0:t0 + cnt]]
        nxt = carry
        for w in range((cnt + 31) // 32):
            word = sc[w * 32:(w + 1) * 32]
            c_in = max([carry] + sc[:w * 32])
            pm = I32_MIN
            for i, s in enumerate(word):
                prev = max(c_in, pm)
                t = t0 + w * 32 + i
                ev = t == 0 or s > prev
                if t == 0:
                    c = 1 << 17
                elif not ev:
                    c = orc.L.i4o_exp_negative_q17(max(s - prev, I32_MIN))
                else:
                    c = orc.L.i4o_exp_negative_q17(max(prev - s, I32_MIN))
                coef[t], event[t] = c, ev
                pm = max(pm, s)
            if (w + 1) * 32 >= cnt:
                nxt = max(c_in, pm)
        carry = nxt
    return coef, event


@pytest.mark.parametrize("name", sorted(CASES))
def test_window_coefficients_carry_the_running_maximum(name):
    n, scores_of, _ = CASES[name]
    rng = np.random.default_rng(sum(map(ord, name)))
    orc = Oracle()
    scores = scores_of(rng, n)
    want = coefficients(scores, orc)
    got = window_coefficients(scores, orc)
    assert np.array_equal(got[0], want[0]) and np.array_equal(got[1], want[1])
