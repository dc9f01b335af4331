"""Numerics of the split attention of the paged cache, on the CPU.

The paged decoder kernel (hb_decoder.cuh, ``attention_paged``) splits one
head's positions [0, n) into S ranges of ``ceil(n / S)`` rounded up to 32
positions (trailing ranges may be empty); each range keeps its own max m_s,
sum of exp(score - m_s) and unnormalised P.V in FP32, and the last split
to finish rescales them by exp(m_s - M) to the common max M.  This
restates that arithmetic in float32 NumPy and bounds its error against a
float64 softmax for the split counts the kernel uses (up to 10 at batch 1
for the Qwen shape) and beyond, down to one position per split.  The GPU
kernel itself is compared with the oracle in tests/test_long_context.py.
"""

import numpy as np
import pytest
from ml_dtypes import bfloat16


def split_ranges(n, s):
    chunk = -(-n // s)
    chunk = (chunk + 31) & ~31
    out = []
    for i in range(s):
        lo = min(n, i * chunk)
        out.append((lo, min(n, lo + chunk)))
    return out


def split_attention(q, keys, values, s):
    """float32 split-and-combine attention of one head: q [64], keys /
    values [n, 64] (BF16 values held in float32)."""
    f = np.float32
    parts = []
    for lo, hi in split_ranges(keys.shape[0], s):
        if lo == hi:
            parts.append((f(-np.inf), f(0.0), np.zeros(64, np.float32)))
            continue
        scores = (keys[lo:hi] @ q).astype(np.float32) * f(0.125)
        m = scores.max()
        e = np.exp(scores - m).astype(np.float32)
        parts.append((m, e.sum(dtype=np.float32), (e[:, None] * values[lo:hi]).sum(axis=0, dtype=np.float32)))
    big = max(p[0] for p in parts)
    den, num = f(0.0), np.zeros(64, np.float32)
    for m, total, pv in parts:
        w = np.exp(f(m - big)).astype(np.float32)
        den = f(den + w * total)
        num = (num + w * pv).astype(np.float32)
    return num / den


def reference(q, keys, values):
    scores = keys.astype(np.float64) @ q.astype(np.float64) * 0.125
    w = np.exp(scores - scores.max())
    return (w / w.sum()) @ values.astype(np.float64)


def test_split_ranges_cover_every_position_once():
    for n in list(range(1, 300)) + [1000, 2049, 4096]:
        for s in (1, 2, 3, 7, 10, 37, 74, 148):
            covered = np.zeros(n, np.int32)
            for lo, hi in split_ranges(n, s):
                assert 0 <= lo <= hi <= n
                covered[lo:hi] += 1
            assert (covered == 1).all(), (n, s)


@pytest.mark.parametrize("n", [1, 65, 300, 1025, 4033])
@pytest.mark.parametrize("s", [1, 2, 3, 10, 74])
def test_split_combine_matches_float64_softmax(n, s):
    rng = np.random.default_rng(n * 131 + s)
    q = (rng.standard_normal(64) * 2.0).astype(np.float32)
    keys = rng.standard_normal((n, 64)).astype(bfloat16).astype(np.float32)
    values = rng.standard_normal((n, 64)).astype(bfloat16).astype(np.float32)
    got = split_attention(q, keys, values, s)
    want = reference(q, keys, values)
    # far below one BF16 unit (2^-8 relative) of the published outputs
    assert np.abs(got - want).max() <= 2e-5 * max(1.0, np.abs(want).max())
