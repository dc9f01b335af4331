"""Symmetric per-output-row int8 quantisation of a projection matrix.

Restates the reference quantiser (npu_llm/tools/convert_smollm2.py:81-86) with
the same FP32 arithmetic so the int8 bytes and the scales are bit-identical:

* ``scale[r] = max(max_k |w[r, k]| / 127, float32 tiny)`` computed in float32;
* ``q[r, k] = clip(rint(w[r, k] / scale[r]), -127, 127)`` with float32 division
  and round-half-to-even.

The reference stores the scale as float32 (4 bytes per row), so this build
does too.
"""

import numpy as np


_TINY = np.finfo(np.float32).tiny


def quantize_per_output_channel(weight):
    w = np.asarray(weight, dtype=np.float32)
    if w.ndim != 2:
        raise ValueError("quantisation expects a [rows, K] matrix")
    peak = np.abs(w).max(axis=1)
    scale = np.maximum(peak / np.float32(127.0), np.float32(_TINY)).astype(np.float32)
    ratio = w / scale[:, None]
    q = np.clip(np.rint(ratio), np.float32(-127.0), np.float32(127.0))
    return q.astype(np.int8), scale
