#!/usr/bin/env python3
"""Generate the golden vectors that pin the sampling oracle to the reference.

Run in a container that has the reference checkout (read-only) at
``--reference`` (default: the ``REFERENCE_ROOT`` environment variable).  It
imports the reference's ``runtime/sampling.py`` (pure NumPy), runs
``Sampler(params).select`` twice per case with a seeded generator, and writes
``sampling.npz`` next to this script: the two tokens the reference chose per
case, and the reference ``log_softmax`` (runtime/stopping.py) of the first
logits at the first token and its five largest entries.  The cases themselves (logits, history, bias) are rebuilt from seeds by
``cases()`` and ``build()`` below, which do not touch the reference.  Nothing
at test time reads the reference; ``tests/test_sampling.py`` replays the
cases through ``oracle.sampling.select_with_uniform`` with the seed's
``random()`` draws, and on a GPU through the device sampler.
"""

import argparse
import importlib.util
import os
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent

# (temperature, top_p, top_k, repetition, presence, frequency, bias?, history?)
PARAMS = [
    (0.0, 1.0, 0, 1.0, 0.0, 0.0, False, False),   # greedy
    (0.7, 1.0, 0, 1.0, 0.0, 0.0, False, False),
    (1.0, 1.0, 0, 1.0, 0.0, 0.0, False, False),
    (1.5, 1.0, 0, 1.0, 0.0, 0.0, False, False),
    (1.0, 1.0, 1, 1.0, 0.0, 0.0, False, False),   # top-1: greedy
    (0.8, 1.0, 5, 1.0, 0.0, 0.0, False, False),
    (1.0, 1.0, 50, 1.0, 0.0, 0.0, False, False),
    (1.2, 1.0, 700, 1.0, 0.0, 0.0, False, False),
    (1.0, 0.5, 0, 1.0, 0.0, 0.0, False, False),
    (0.9, 0.9, 0, 1.0, 0.0, 0.0, False, False),
    (1.0, 0.99, 0, 1.0, 0.0, 0.0, False, False),
    (0.7, 0.9, 40, 1.0, 0.0, 0.0, False, False),
    (1.0, 0.3, 200, 1.0, 0.0, 0.0, False, False),
    (1.0, 1.0, 0, 1.3, 0.0, 0.0, False, True),    # repetition penalty
    (0.8, 1.0, 0, 1.0, 0.5, 0.3, False, True),    # presence + frequency
    (0.9, 0.95, 20, 1.1, -0.4, 0.2, True, True),  # everything
    (1.0, 1.0, 0, 1.0, 0.0, 0.0, True, False),    # bias only
    (0.0, 1.0, 0, 1.2, 0.0, 0.5, False, True),    # penalties, temperature 0: argmax
    (0.0, 1.0, 0, 1.0, 0.0, 0.0, True, False),    # bias, temperature 0: argmax
    (2.0, 0.8, 0, 1.0, 0.0, 0.0, False, False),
]
SCALES = (0.05, 1.0, 4.0)    # flat (random-init-like), moderate, peaked logits
VOCABS = (1024, 4096)


def load_reference(root, name="sampling"):
    spec = importlib.util.spec_from_file_location(f"reference_{name}", Path(root) / f"npu_llm/runtime/{name}.py")
    module = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(module)
    return module


LOGPROB_TOP = 5


def cases():
    """Deterministic case specs: (vocab, scale, params tuple, case seed)."""
    out = []
    seed = 1000
    for vocab in VOCABS:
        for scale in SCALES:
            for pi, spec in enumerate(PARAMS):
                if vocab == 4096 and pi % 3:
                    continue  # the larger vocabulary on a subset
                out.append((vocab, scale, spec, seed))
                seed += 1
    return out


def build(vocab, scale, spec, seed):
    rng = np.random.default_rng(seed)
    logits = [(rng.standard_normal(vocab) * scale).astype(np.float32) for _ in range(2)]
    history = rng.integers(0, vocab, 12).tolist() + rng.integers(0, 4, 4).tolist() + [vocab + 5] if spec[7] else []
    bias = {}
    if spec[6]:
        for token in rng.integers(0, vocab, 6).tolist():
            bias[int(token)] = float(np.round(rng.uniform(-5, 5), 3))
        bias[vocab + 3] = 50.0  # outside the vocabulary: ignored
    return logits, history, bias


def main():
    parser = argparse.ArgumentParser()
    parser.add_argument("--reference", default=os.environ.get("REFERENCE_ROOT"))
    args = parser.parse_args()
    if not args.reference:
        raise SystemExit("pass --reference or set REFERENCE_ROOT")
    ref = load_reference(args.reference)
    stopping = load_reference(args.reference, "stopping")
    rows = []
    lp_token, lp_top_ids, lp_top_vals = [], [], []
    for vocab, scale, spec, seed in cases():
        logits, history, bias = build(vocab, scale, spec, seed)
        t, top_p, top_k, rep, pres, freq, _, _ = spec
        params = ref.SamplingParams(temperature=t, top_p=top_p, top_k=top_k, repetition_penalty=rep,
                                    presence_penalty=pres, frequency_penalty=freq, logit_bias=bias,
                                    seed=seed)
        sampler = ref.Sampler(params, vocab_size=vocab)
        rows.append([sampler.select(logits[0], history), sampler.select(logits[1], history)])
        # the reference log_softmax of the first logits: the chosen token and the top entries
        values = stopping.log_softmax(logits[0])
        best = np.argpartition(values, -LOGPROB_TOP)[-LOGPROB_TOP:]
        best = best[np.argsort(values[best])[::-1]]
        lp_token.append(values[rows[-1][0]])
        lp_top_ids.append(best)
        lp_top_vals.append(values[best])
    np.savez_compressed(HERE / "sampling.npz", tokens=np.asarray(rows, np.int64),
                        logprob_token=np.asarray(lp_token, np.float64),
                        logprob_top_ids=np.asarray(lp_top_ids, np.int64),
                        logprob_top_values=np.asarray(lp_top_vals, np.float64))
    print(f"wrote {len(rows)} cases to {HERE / 'sampling.npz'}")


if __name__ == "__main__":
    main()
