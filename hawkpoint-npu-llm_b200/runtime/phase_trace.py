"""Per-phase device timing of one decode launch.

The decoder kernel stamps %globaltimer at fixed points of every phase in
every CTA when tracing is on (``B200DecoderEngine.profile(trace=True)``,
``hb_profile(engine, 2)``): phase start, inputs ready, prologue (norm or
attention) done, outputs stored.  This prints, per phase kind, the median
over layers of: the wait for the previous phase's words, the prologue, the
GEMV with its epilogue, and the whole phase (the latest CTA of each).  It is
the timing view the reference's ``HAWKPOINT_PROFILE`` phase totals give
for the NPU path (npu_llm/runtime/generate.py:94-101), resolved per phase.

    python hawkpoint-npu-llm_b200/runtime/phase_trace.py --model qwen2.5-0.5b \\
        --context 4096 --depths 256 4032

Synthetic seeded weights; the prompt is prefilled, three steps warm up,
and the fourth decode step is traced.
"""

import argparse
import sys
from pathlib import Path

import numpy as np

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))

from runtime import synthetic  # noqa: E402
from runtime.b200_engine import B200DecoderEngine  # noqa: E402

KINDS = ((0, "qkv"), (1, "attn"), (2, "mlp_in"), (3, "mlp_out"))


def trace_step(engine, ids, depth, warm=3):
    """Stamps [G, 4L+2, 8] (ns) of the decode launch at position depth+warm."""
    tok, _ = engine.prefill(ids[:depth], slot=0)
    for i in range(warm):
        tok = engine.step_argmax(tok, depth + i, slot=0)
    engine.profile(True, trace=True)
    engine.step_argmax(tok, depth + warm, slot=0)
    stamps = engine.phase_trace().astype(np.int64)
    engine.profile(False)
    return stamps


def summarize(stamps, layers):
    """{kind: (wait, prologue, gemv+epilogue, phase)} in microseconds, and
    the launch span from the first CTA's start to the head's last output."""
    out = {}
    for kind, name in KINDS:
        ks = [4 * layer + kind for layer in range(layers)]
        start = np.array([stamps[:, k, 0].min() for k in ks])
        ready = np.array([stamps[:, k, 1].max() for k in ks])
        prologue = np.array([stamps[:, k, 6].max() for k in ks])
        done = np.array([stamps[:, k, 3].max() for k in ks])
        out[name] = tuple(float(np.median(v)) / 1e3 for v in (ready - start, prologue - ready, done - prologue,
                                                              done - start))
    span = float(stamps[:, 4 * layers, 3].max() - stamps[:, 0, 0].min()) / 1e3
    return out, span


def critical_path(stamps, layers):
    """Per phase kind, medians over layers 1.. (us) measured from the moment
    the previous phase's last CTA stored its outputs: its inputs gathered by
    the median and by the last CTA, then the median CTA's norm (or, for
    attn, the barrier after the gather), GEMV and epilogue, and the critical
    span to this phase's last store."""
    out = {}
    for kind, name in KINDS:
        vals = []
        for layer in range(1, layers):
            k = 4 * layer + kind
            pub = stamps[:, k - 1, 3].max()
            g, n6, c2, s3 = (stamps[:, k, i] for i in (1, 6, 2, 3))
            vals.append((np.median(g - pub), g.max() - pub, np.median(n6 - g), np.median(c2 - n6),
                         np.median(s3 - c2), s3.max() - pub))
        out[name] = tuple(float(v) / 1e3 for v in np.median(np.array(vals, dtype=np.float64), axis=0))
    k = 4 * layers
    pub = stamps[:, k - 1, 3].max()
    out["head"] = (float(np.median(stamps[:, k, 1] - pub)) / 1e3, float(stamps[:, k, 1].max() - pub) / 1e3,
                   float(np.median(stamps[:, k, 6] - stamps[:, k, 1])) / 1e3,
                   float(np.median(stamps[:, k, 2] - stamps[:, k, 6])) / 1e3,
                   float(np.median(stamps[:, k, 3] - stamps[:, k, 2])) / 1e3,
                   float(stamps[:, k, 3].max() - pub) / 1e3)
    return out


def main():
    parser = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    parser.add_argument("--model", default="qwen2.5-0.5b", choices=sorted(synthetic.SHAPES))
    parser.add_argument("--weights", default="bf16", choices=["bf16", "w8"])
    parser.add_argument("--context", type=int, default=4096)
    parser.add_argument("--depths", type=int, nargs="+", default=[256, 4032])
    parser.add_argument("--device", type=int, default=0)
    parser.add_argument("--critical-path", action="store_true",
                        help="also print each phase's chain from the previous phase's last store")
    args = parser.parse_args()
    model = synthetic.build(args.model, seed=0).materialize()
    engine = B200DecoderEngine(model, weights=args.weights, device=args.device, max_batch=8, context=args.context)
    try:
        ids = synthetic.prompt_ids(model.shape.vocab, max(args.depths), seed=3)
        for depth in args.depths:
            rows, span = summarize(trace_step(engine, ids, depth), model.shape.layers)
            print(f"{args.model} {args.weights} context {args.context}, decode at position {depth + 3}: "
                  f"launch span {span:.1f} us")
            for name, (wait, prologue, gemv, phase) in rows.items():
                print(f"  {name:8s} wait {wait:6.2f}  prologue {prologue:6.2f}  gemv+epilogue {gemv:6.2f}  "
                      f"phase {phase:6.2f} us (median over layers)")
            if args.critical_path:
                stamps = trace_step(engine, ids, depth)
                print("  critical path from the previous phase's last store (us; median over layers 1..):")
                print("  phase     inputs(median CTA)  inputs(last CTA)  norm/sync  gemv  epilogue  last store")
                for name, v in critical_path(stamps, model.shape.layers).items():
                    print(f"  {name:8s} " + "  ".join(f"{x:8.2f}" for x in v))
    finally:
        engine.close()


if __name__ == "__main__":
    main()
