"""Host side of the per-phase trace summary (runtime/phase_trace.py): the
medians it reports from a synthetic stamp array."""

import numpy as np

from runtime.phase_trace import summarize


def test_summary_takes_the_latest_cta_and_the_median_over_layers():
    layers, ctas = 3, 4
    stamps = np.zeros((ctas, 4 * layers + 2, 8), np.int64)
    t = 0
    for k in range(4 * layers + 1):
        for c in range(ctas):
            # phase k: start t (+c), inputs ready +1000 ns (+10 c), prologue
            # done +3000, outputs stored +7000 (the last CTA 100 ns later)
            stamps[c, k, 0] = t + c
            stamps[c, k, 1] = t + 1000 + 10 * c
            stamps[c, k, 6] = t + 3000
            stamps[c, k, 3] = t + 7000 + (100 if c == ctas - 1 else 0)
        t += 10000
    rows, span = summarize(stamps, layers)
    for name in ("qkv", "attn", "mlp_in", "mlp_out"):
        wait, prologue, gemv, phase = rows[name]
        assert abs(wait - 1.030) < 1e-9
        assert abs(prologue - (3000 - 1030) / 1e3) < 1e-9
        assert abs(gemv - 4.1) < 1e-9
        assert abs(phase - 7.1) < 1e-9
    assert abs(span - (4 * layers * 10000 + 7100) / 1e3) < 1e-9
