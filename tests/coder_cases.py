"""Crafted coder-interval sequences for the encoder tests (host-side helper, no GPU).

The reference encoder (rust/src/arith_coder.rs:80-119) renormalises one bit at a
time; the GPU encoder does it in closed form (all agreeing top bits at once, then
all straddle steps at once).  Real text rarely reaches three of its branches:
 * low == high after the interval update (32 agreeing bits leave at once);
 * a run of 31 straddle (E3) steps in one symbol;
 * a pending run longer than 32 bits when the next agreeing bit leaves.
``crafted_sequences`` builds interval sequences that reach each of them, found by
stepping a model of the reference encoder's state; ``branch_counts`` reports how
often a sequence reaches them, so a test can check its own coverage.
"""
from __future__ import annotations

import numpy as np

HALF, QUARTER, MASK = 1 << 31, 1 << 30, (1 << 32) - 1


def step(state, lo, hi, total):
    """One encode_symbol of the reference (arith_coder.rs:80-119) on (low, high,
    pending); returns the new state and (agreeing bits, straddle steps, pending + agreeing)."""
    low, high, pending = state
    r = high - low + 1
    high = low + (hi * r) // total - 1
    low = low + (lo * r) // total
    k1 = j = 0
    tot = 0
    while True:
        if ((low ^ high) & HALF) == 0:
            if k1 == 0:
                tot = pending + 1
            k1 += 1
            pending = 0
            low = (low << 1) & MASK
            high = ((high << 1) & MASK) | 1
        elif low & ~high & QUARTER:
            j += 1
            pending += 1
            low = ((low << 1) ^ HALF) & MASK
            high = (((high ^ HALF) << 1) | HALF | 1) & MASK
        else:
            break
    return (low, high, pending), (k1, j, tot + max(k1 - 1, 0) if k1 else 0)


def _solve(state, target_low, target_high, total):
    """(lo, hi) with lo < hi <= total whose update moves state to exactly
    (target_low, target_high) before renormalisation, or None."""
    low, high, _ = state
    r = high - low + 1
    a, b = target_low - low, target_high - low + 1
    if a < 0 or b <= a or b > r:
        return None
    lo = -(-a * total // r)                  # smallest lo with lo * r // total >= a
    hi = -(-b * total // r)
    if lo * r // total != a or hi * r // total != b or not (lo < hi <= total):
        return None
    return lo, hi


def crafted_sequences(total: int, seed: int = 0, n_seq: int = 24, length: int = 400):
    """Interval sequences (lists of (lo, hi)) that reach the rare branches."""
    rng = np.random.default_rng(seed)
    seqs = []
    for si in range(n_seq):
        st = (0, MASK, 0)
        seq = []
        mode = si % 4
        while len(seq) < length:
            pick = None
            want = rng.integers(0, 5) if mode == 3 else mode
            if want == 0:     # the interval collapses to one value: 32 agreeing bits
                for _ in range(64):
                    lo = int(rng.integers(0, total - 1))
                    r = st[1] - st[0] + 1
                    if ((lo + 1) * r) // total - (lo * r) // total == 1:
                        pick = (lo, lo + 1)
                        break
            elif want == 1:   # exactly 0x7FFFFFFF / 0x80000000: 31 straddle steps
                pick = _solve(st, HALF - 1, HALF, total)
            elif want == 2:   # narrow intervals across the half: pending bits pile up
                mid = st[0] + (st[1] - st[0]) // 2
                w = int(rng.integers(0, 8))
                pick = _solve(st, max(st[0], mid - w), min(st[1], mid + 1 + w), total)
            if pick is None:  # an ordinary symbol of random width moves the state on
                width = int(np.exp(rng.uniform(0, np.log(total))))
                lo = int(rng.integers(0, total - width + 1))
                pick = (lo, lo + max(1, width))
            seq.append(pick)
            st, _ = step(st, pick[0], pick[1], total)
        seqs.append(seq)
    return seqs


def random_sequences(total: int, seed: int = 1, n_seq: int = 40, length: int = 600):
    """Intervals of log-uniform width anywhere in [0, total]."""
    rng = np.random.default_rng(seed)
    out = []
    for _ in range(n_seq):
        w = np.exp(rng.uniform(0, np.log(total), length)).astype(np.int64).clip(1, total)
        lo = (rng.uniform(0, 1, length) * (total - w + 1)).astype(np.int64)
        out.append(list(zip(lo.tolist(), (lo + w).tolist())))
    return out


def branch_counts(seqs, total: int) -> dict:
    """How often the sequences reach each rare branch of the closed-form encoder."""
    c = {"all_32_agree": 0, "straddle_31": 0, "pending_over_32": 0, "pending_over_64": 0, "symbols": 0}
    for seq in seqs:
        st = (0, MASK, 0)
        for lo, hi in seq:
            st, (k1, j, tot) = step(st, lo, hi, total)
            c["symbols"] += 1
            c["all_32_agree"] += k1 >= 32
            c["straddle_31"] += j >= 31
            c["pending_over_32"] += tot > 32
            c["pending_over_64"] += tot > 64
    return c
