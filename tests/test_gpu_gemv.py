"""Standalone weight-streaming GEMV (the matrix_vector shapes of the GEMV microbenchmark) against a PyTorch FP32
reference of the same op: ``bf16(W_f32 @ x_f32)`` (the BF16 projection of
npu_llm/runtime/cpu_backend.py:64-69) and the W8 form
``bf16((q_f32 @ x_f32) * scale)`` (npu_llm/kernels/decoder_layer_bf16.cc:64-80).

Tolerance: the FP32 sum is order-dependent (the BF16 kernels accumulate on
the tensor cores), so the BF16 output may differ from the reference's
rounding by one BF16 unit in the last place (plus 1e-5 of sum(|w x|) where
the sum cancels to nearly zero); FP32 outputs must agree to 1e-5 of
sum(|w x|).  The fused argmax must equal the first
maximum of the kernel's own FP32 outputs, and the reference argmax whenever
the reference top-2 margin exceeds 1e-3.
"""

import ctypes

import numpy as np
import pytest
from ml_dtypes import bfloat16

from runtime import hb_lib, layout
from runtime.quantize import quantize_per_output_channel

pytestmark = pytest.mark.gpu

SHAPES = [(896, 896), (4864, 896), (896, 4864), (576, 1536), (151936, 896)]


def _torch():
    import torch

    return torch


def run_gemv(w_packed, scales, fmt, rows, k, x_bf16, flags):
    torch = _torch()
    lib = hb_lib.load()
    dev = torch.device("cuda:0")
    w = torch.from_numpy(np.ascontiguousarray(w_packed)).to(dev)
    s = torch.from_numpy(np.ascontiguousarray(scales)).to(dev) if scales is not None else None
    batch = x_bf16.shape[0]
    x = torch.from_numpy(np.ascontiguousarray(x_bf16).view(np.int16)).to(dev)
    out_mode = flags & 3
    if out_mode == hb_lib.HB_GEMV_OUT_BF16:
        y = torch.zeros((batch, rows), dtype=torch.int16, device=dev)
    else:
        y = torch.zeros((batch, rows), dtype=torch.float32, device=dev)
    am = torch.full((batch,), -1, dtype=torch.int32, device=dev)
    nscratch = lib.hb_gemv_scratch_bytes(rows, batch)
    scratch = torch.zeros(nscratch, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream().cuda_stream
    rc = lib.hb_gemv(
        w.data_ptr(), s.data_ptr() if s is not None else None, layout.FORMATS[fmt], rows, k,
        x.data_ptr(), batch, y.data_ptr(), flags, am.data_ptr(), scratch.data_ptr(), nscratch,
        ctypes.c_void_p(stream))
    hb_lib.check(rc)
    torch.cuda.synchronize()
    if out_mode == hb_lib.HB_GEMV_OUT_BF16:
        out = y.cpu().numpy().view(np.uint16).view(bfloat16).astype(np.float32)
    else:
        out = y.cpu().numpy()
    return out, am.cpu().numpy()


def reference(w_f32, x_f32, scales=None):
    torch = _torch()
    wt = torch.from_numpy(w_f32).cuda()
    xt = torch.from_numpy(x_f32).cuda()
    ref = (xt @ wt.T)
    if scales is not None:
        ref = ref * torch.from_numpy(scales).cuda()
    mag = (xt.abs() @ wt.abs().T)
    if scales is not None:
        mag = mag * torch.from_numpy(np.abs(scales)).cuda()
    return ref.cpu().numpy(), mag.cpu().numpy()


def bf16_ulp(v):
    a = np.abs(v).astype(np.float32)
    e = np.floor(np.log2(np.maximum(a, 1e-30)))
    return np.exp2(e - 7)


@pytest.mark.parametrize("fmt", ["bf16", "w8"])
@pytest.mark.parametrize("batch", [1, 8])
@pytest.mark.parametrize("rows,k", SHAPES)
def test_gemv_matches_torch_fp32(rows, k, batch, fmt):
    rng = np.random.default_rng([rows, k, batch])
    w = rng.standard_normal((rows, k), dtype=np.float32).astype(bfloat16)
    x = rng.standard_normal((batch, k), dtype=np.float32).astype(bfloat16)
    if fmt == "w8":
        q, scales = quantize_per_output_channel(w)
        packed = layout.pack_matrix_bytes(q)
        w_f32 = q.astype(np.float32)
    else:
        scales = None
        packed = layout.pack_matrix_bytes(w)
        w_f32 = w.astype(np.float32)
    x_f32 = x.astype(np.float32)
    ref, mag = reference(w_f32, x_f32, scales)

    out_bf16, _ = run_gemv(packed, scales, fmt, rows, k, x, hb_lib.HB_GEMV_OUT_BF16)
    ref_bf16 = ref.astype(bfloat16).astype(np.float32)
    # one BF16 unit of the larger of the two (the FP32 sums may straddle a
    # rounding midpoint or a power of two in different summation orders),
    # plus the FP32 accumulation error bound for results that cancel to ~0
    diff = np.abs(out_bf16 - ref_bf16)
    ulp = bf16_ulp(np.maximum(np.abs(out_bf16), np.abs(ref_bf16)))
    bad = diff > ulp * 1.01 + 1e-5 * mag + 1e-30
    assert not bad.any(), (
        f"{bad.sum()} BF16 outputs off by more than one unit; first at "
        f"{np.argwhere(bad)[0]}: got {out_bf16[bad][0]}, ref {ref[bad][0]}")
    assert np.mean(diff > 0) < 0.01

    out_f32, am = run_gemv(packed, scales, fmt, rows, k, x,
                           hb_lib.HB_GEMV_OUT_F32 | hb_lib.HB_GEMV_ARGMAX)
    assert np.all(np.abs(out_f32 - ref) <= 1e-5 * mag + 1e-6)
    for b in range(batch):
        assert am[b] == int(np.argmax(out_f32[b]))
        top2 = np.sort(ref[b])[-2:]
        if top2[1] - top2[0] > 1e-3:
            assert am[b] == int(np.argmax(ref[b]))


def test_gemv_argmax_first_index_on_ties():
    rows, k = 1024, 64
    w = np.zeros((rows, k), np.float32)
    w[[5, 77, 900], 0] = 1.0
    x = np.zeros((1, k), np.float32)
    x[0, 0] = 2.0
    packed = layout.pack_matrix_bytes(w.astype(bfloat16))
    _, am = run_gemv(packed, None, "bf16", rows, k, x.astype(bfloat16),
                     hb_lib.HB_GEMV_OUT_NONE | hb_lib.HB_GEMV_ARGMAX)
    assert am[0] == 5


@pytest.mark.parametrize("rows,k", [(1024, 64), (896, 4864)])
def test_gemv_argmax_ranks_nan_first_like_numpy(rows, k):
    """np.argmax order (npu_llm/runtime/generate.py:713): a NaN output ranks
    above every number and the first NaN wins, so the fused argmax always
    names a row of the matrix, even when every output is NaN."""
    x = np.zeros((1, k), np.float32)
    x[0, 0] = 2.0
    for nan_rows, expect in (([500, 77, rows - 3], 77), (list(range(rows)), 0)):
        w = np.zeros((rows, k), np.float32)
        w[3, 0] = 100.0
        w[nan_rows, 0] = np.nan
        packed = layout.pack_matrix_bytes(w.astype(bfloat16))
        out, am = run_gemv(packed, None, "bf16", rows, k, x.astype(bfloat16),
                           hb_lib.HB_GEMV_OUT_F32 | hb_lib.HB_GEMV_ARGMAX)
        assert np.isnan(out[0, nan_rows]).all()
        assert am[0] == expect == int(np.argmax(out[0]))


def test_gemv_rejects_bad_shapes():
    lib = hb_lib.load()
    rc = lib.hb_gemv(None, None, 0, 12, 16, None, 1, None, 0, None, None, 0, None)
    assert rc == hb_lib.HB_ERR_INVALID_ARG
    with pytest.raises(ValueError):
        hb_lib.check(rc)
