"""The tcgen05 tensor-core GEMM (hb_tc_gemm) against a float64 reference.

y[n][r] = sum_k W[r][k] X[n][k] with BF16 W and X (N(0, 1)) in the packed
row-group layout; FP32 accumulation over K products of magnitude ~1 keeps the
error far below 1e-3 * sqrt(K), the tolerance used here.  Shapes cover the
Qwen2.5-0.5B projections at prefill / multi-stream batch sizes, split-K, a
partial last 128-row tile, N = 1 and N = 256.
"""

import ctypes

import numpy as np
import pytest
from ml_dtypes import bfloat16

from runtime import hb_lib, layout

pytestmark = pytest.mark.gpu

SHAPES = [
    (1152, 896, 32),    # qkv, 32-position prefill
    (896, 4864, 64),    # down, 64 streams (split-K)
    (9728, 896, 16),    # gate_up
    (960, 576, 40),     # SmolLM2 qkv: partial last tile, n not a multiple of 16
    (256, 256, 1),
    (896, 896, 256),
]


def run_gemm(w, x):
    import torch

    lib = hb_lib.load()
    rows, k = w.shape
    n = x.shape[0]
    n8 = -(-n // 8) * 8
    xp = np.zeros((n8, k), bfloat16)
    xp[:n] = x
    dev = torch.device("cuda", 0)
    wd = torch.from_numpy(layout.pack_matrix_bytes(w)).to(dev)
    xd = torch.from_numpy(layout.pack_matrix_bytes(xp)).to(dev)
    y = torch.empty((n, rows), dtype=torch.float32, device=dev)
    nscr = lib.hb_tc_gemm_scratch_bytes(rows, k, n)
    scr = torch.zeros(nscr, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev).cuda_stream
    hb_lib.check(lib.hb_tc_gemm(wd.data_ptr(), rows, k, xd.data_ptr(), n,
                                ctypes.cast(y.data_ptr(), ctypes.POINTER(ctypes.c_float)),
                                scr.data_ptr(), nscr, ctypes.c_void_p(stream)))
    hb_lib.check(lib.hb_tc_gemm_status(scr.data_ptr(), ctypes.c_void_p(stream)))
    return y.cpu().numpy(), (wd, xd, y, scr)


@pytest.mark.parametrize("rows,k,n", SHAPES)
def test_tc_gemm_matches_float64(rows, k, n):
    rng = np.random.default_rng(rows + k + n)
    w = rng.standard_normal((rows, k), dtype=np.float32).astype(bfloat16)
    x = rng.standard_normal((n, k), dtype=np.float32).astype(bfloat16)
    y, _ = run_gemm(w, x)
    ref = x.astype(np.float64) @ w.astype(np.float64).T
    err = np.abs(y - ref).max()
    assert err <= 1e-3 * np.sqrt(k), f"max |error| {err:.3e}"


def test_tc_gemm_is_deterministic():
    """Split-K partials are summed in slice order across the tile's
    cluster, whichever slice finishes first: repeated calls give identical
    bits."""
    rng = np.random.default_rng(5)
    w = rng.standard_normal((896, 4864), dtype=np.float32).astype(bfloat16)
    x = rng.standard_normal((48, 4864), dtype=np.float32).astype(bfloat16)
    a, _ = run_gemm(w, x)
    b, _ = run_gemm(w, x)
    assert np.array_equal(a, b)


def test_tc_gemm_rejects_bad_shapes():
    lib = hb_lib.load()
    buf = ctypes.c_void_p(16)
    with pytest.raises(ValueError):
        hb_lib.check(lib.hb_tc_gemm(buf, 896, 100, buf, 8, ctypes.cast(buf, ctypes.POINTER(ctypes.c_float)),
                                    buf, 1 << 20, None))
    with pytest.raises(ValueError):
        hb_lib.check(lib.hb_tc_gemm(buf, 896, 896, buf, 300, ctypes.cast(buf, ctypes.POINTER(ctypes.c_float)),
                                    buf, 1 << 20, None))
