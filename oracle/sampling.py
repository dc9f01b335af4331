"""CPU oracle for token sampling -- TEST INFRASTRUCTURE ONLY.

Only ``tests/`` may import this module, as the checker of the on-device
sampler (``hb_sample`` / ``hb_sampler_select`` in ``libhawkb200.so``).  The
product path never calls it.

A NumPy restatement of the reference's ``Sampler.select``
(npu_llm/runtime/sampling.py:416-445) and the steps it calls: penalties
(``apply_penalties``, :327-363), logit bias (``apply_logit_bias``, :366-380),
temperature, top-k (``filter_top_k``, :383-389), top-p (``filter_top_p``,
:392-406), the guarded softmax (``_softmax``, :409-421) and the multinomial
draw of ``numpy.random.Generator.choice(n, p=...)``: cumulative sum,
normalised by its last element, then ``searchsorted(u, side="right")`` of one
``Generator.random()`` draw ``u``.  ``select_with_uniform`` takes that ``u``
explicitly, so the request's own generator can stay on the host while the
selection runs elsewhere; ``tests/golden/make_sampling_golden.py`` pins it to
the reference ``Sampler`` with seeded generators.

``pairwise_sum`` restates NumPy's summation order for contiguous float32 and
float64 arrays (blocks of at most 128 elements summed with eight
accumulators, halves split at multiples of eight); the device sampler follows
the same tree so its softmax denominators match ``ndarray.sum`` bit for bit.
"""

from dataclasses import dataclass, field

import numpy as np


@dataclass(frozen=True)
class Params:
    """The fields of the reference ``SamplingParams`` the selection reads."""

    temperature: float = 0.0
    top_p: float = 1.0
    top_k: int = 0
    repetition_penalty: float = 1.0
    presence_penalty: float = 0.0
    frequency_penalty: float = 0.0
    logit_bias: dict = field(default_factory=dict)

    def reorder_free(self):
        return (self.repetition_penalty == 1.0 and self.presence_penalty == 0.0
                and self.frequency_penalty == 0.0 and (self.temperature == 0.0 or self.top_k == 1))

    def greedy_for(self, vocab):
        """Parameters that cannot change the argmax (sampling.py:243-255)."""
        return self.reorder_free() and not any(0 <= t < vocab for t in self.logit_bias)


def history_counts(history, vocab):
    """Unique in-vocabulary history tokens (ascending) and their counts."""
    if not len(history):
        return np.zeros(0, np.int64), np.zeros(0, np.float32)
    tokens, counts = np.unique(np.asarray(history, np.int64), return_counts=True)
    keep = (tokens >= 0) & (tokens < vocab)
    return tokens[keep], counts[keep].astype(np.float32)


def apply_penalties(scores, history, p):
    if not len(history):
        return scores
    if p.repetition_penalty == 1.0 and p.presence_penalty == 0.0 and p.frequency_penalty == 0.0:
        return scores
    tokens, counts = history_counts(history, scores.shape[0])
    if not tokens.shape[0]:
        return scores
    chosen = scores[tokens]
    if p.repetition_penalty != 1.0:
        chosen = np.where(chosen > 0, chosen / p.repetition_penalty, chosen * p.repetition_penalty)
    chosen = chosen - p.frequency_penalty * counts
    chosen = chosen - p.presence_penalty
    scores[tokens] = chosen
    return scores


def apply_bias(scores, bias):
    for token, value in bias.items():
        if 0 <= int(token) < scores.shape[0]:
            scores[int(token)] += value
    return scores


def top_k_mask(scores, k):
    if k <= 0 or k >= scores.shape[0]:
        return scores
    threshold = np.partition(scores, -k)[-k]
    scores[scores < threshold] = -np.inf
    return scores


def guarded_softmax(scores):
    finite = scores[np.isfinite(scores)]
    peak = finite.max() if finite.size else 0.0
    shifted = np.exp(scores - peak, where=np.isfinite(scores), out=np.zeros_like(scores))
    total = shifted.sum()
    if not np.isfinite(total) or total <= 0:
        out = np.zeros_like(scores)
        out[int(np.argmax(scores))] = 1.0
        return out
    return shifted / total


def top_p_mask(scores, top_p):
    if top_p >= 1.0:
        return scores
    order = np.argsort(scores)[::-1]
    probs = guarded_softmax(scores[order])
    cumulative = np.cumsum(probs)
    keep = cumulative - probs < top_p
    keep[0] = True
    scores[order[~keep]] = -np.inf
    return scores


def final_distribution(scores):
    """The float64 vector handed to ``Generator.choice`` (sampling.py:440-444)."""
    probs = guarded_softmax(scores).astype(np.float64)
    probs /= probs.sum()
    return probs


def draw(probs, u):
    """``Generator.choice(len(probs), p=probs)`` given its one uniform draw ``u``."""
    cdf = probs.cumsum()
    cdf /= cdf[-1]
    return int(cdf.searchsorted(u, side="right"))


def select_with_uniform(logits, history, params, u):
    """Token chosen by ``Sampler(params).select(logits, history)`` when the
    request generator's next ``random()`` is ``u`` (``u`` is unused on the
    greedy and temperature-0 paths, which draw nothing)."""
    scores = np.asarray(logits, dtype=np.float32)
    if params.greedy_for(scores.shape[0]):
        return int(np.argmax(scores))
    scores = apply_penalties(scores.copy(), history, params)
    scores = apply_bias(scores, params.logit_bias)
    if params.temperature == 0.0:
        return int(np.argmax(scores))
    scores = scores / params.temperature
    scores = top_k_mask(scores, params.top_k)
    scores = top_p_mask(scores, params.top_p)
    return draw(final_distribution(scores), u)


def draws_uniform(params, vocab):
    """Whether one selection consumes a ``random()`` draw."""
    return not params.greedy_for(vocab) and params.temperature != 0.0


# -- logprobs ---------------------------------------------------------------------
def log_softmax(logits):
    """float64 log-probabilities (npu_llm/runtime/stopping.py:101-109): the
    finite maximum subtracted, non-finite scores at -inf, minus the log of
    the pairwise float64 sum of exp."""
    scores = np.asarray(logits, dtype=np.float64)
    finite = np.isfinite(scores)
    if not finite.any():
        raise ValueError("logits contain no finite value")
    shifted = np.where(finite, scores - scores[finite].max(), -np.inf)
    return shifted - np.log(np.exp(shifted).sum())


def top_logprobs(values, count):
    """The ``count`` largest log-probabilities, largest first, as the
    decoder's logprobs entry orders them (argpartition + argsort)."""
    count = min(count, values.shape[0])
    if count <= 0:
        return np.zeros(0, np.int64)
    best = np.argpartition(values, -count)[-count:]
    return best[np.argsort(values[best])[::-1]]


# -- NumPy's summation order -------------------------------------------------
def pairwise_sum(values):
    """``values.sum()`` for a contiguous 1-D float32 / float64 array, in
    NumPy's order: n < 8 summed left to right from zero; 8 <= n <= 128 in
    eight strided accumulators combined as ((r0+r1)+(r2+r3))+((r4+r5)+(r6+r7))
    plus the tail left to right; larger n split at half rounded down to a
    multiple of eight, each half summed the same way."""
    a = np.ascontiguousarray(values)
    dtype = a.dtype.type

    def rec(lo, n):
        if n < 8:
            res = dtype(0)
            for i in range(n):
                res = dtype(res + a[lo + i])
            return res
        if n <= 128:
            r = [a[lo + j] for j in range(8)]
            i = 8
            while i < n - n % 8:
                for j in range(8):
                    r[j] = dtype(r[j] + a[lo + i + j])
                i += 8
            res = dtype(dtype(dtype(r[0] + r[1]) + dtype(r[2] + r[3])) + dtype(dtype(r[4] + r[5]) + dtype(r[6] + r[7])))
            while i < n:
                res = dtype(res + a[lo + i])
                i += 1
            return res
        n2 = n // 2
        n2 -= n2 % 8
        return dtype(rec(lo, n2) + rec(lo + n2, n - n2))

    return rec(0, a.shape[0])
