"""hb_gemv_noalloc: the GEMV entry point for callers that cannot allocate
device memory (its scratch is a fixed array inside the library).

Called through the C ABI on the same inputs as hb_gemv (which takes a scratch
buffer from the caller), twice in a row, and compared with it: the two run the
same kernel, so outputs and argmax must agree within the GEMV tests' tolerance
(they are in fact expected to be identical).  The second call checks that the
state a call leaves in the shared array does not leak into the next one.
The outputs are also checked against an FP32 reference of the same product,
for BF16 and W8 weights, with FP32 / argmax-only outputs, and for calls of
different grid sizes queued back to back on one stream (they reuse the same
partial slots), and a launch whose device wait runs out (test hook) reports
-1 in-band.  This file is named to be collected last.
"""

import ctypes

import numpy as np
import pytest
from ml_dtypes import bfloat16

from runtime import hb_lib, layout

pytestmark = pytest.mark.gpu


def _case(rows, k, batch, seed):
    import torch

    rng = np.random.default_rng([rows, k, batch, seed])
    w = rng.standard_normal((rows, k), dtype=np.float32).astype(bfloat16)
    x = rng.standard_normal((batch, k), dtype=np.float32).astype(bfloat16)
    dev = torch.device("cuda:0")
    wd = torch.from_numpy(layout.pack_matrix_bytes(w)).to(dev)
    xd = torch.from_numpy(np.ascontiguousarray(x).view(np.int16)).to(dev)
    return wd, xd


def _outputs(rows, batch):
    import torch

    dev = torch.device("cuda:0")
    return (torch.zeros((batch, rows), dtype=torch.float32, device=dev),
            torch.full((batch,), -1, dtype=torch.int32, device=dev))


@pytest.mark.parametrize("rows,k,batch", [(151936, 896, 1), (4864, 896, 8), (896, 4864, 1)])
def test_noalloc_matches_gemv_twice(rows, k, batch):
    import torch

    lib = hb_lib.load()
    flags = hb_lib.HB_GEMV_OUT_F32 | hb_lib.HB_GEMV_ARGMAX
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    wd, xd = _case(rows, k, batch, seed=1)
    y_ref, am_ref = _outputs(rows, batch)
    nscratch = lib.hb_gemv_scratch_bytes(rows, batch)
    scratch = torch.zeros(nscratch, dtype=torch.uint8, device="cuda:0")
    hb_lib.check(lib.hb_gemv(wd.data_ptr(), None, 0, rows, k, xd.data_ptr(), batch, y_ref.data_ptr(), flags,
                             am_ref.data_ptr(), scratch.data_ptr(), nscratch, stream))
    for _ in range(2):
        y, am = _outputs(rows, batch)
        hb_lib.check(lib.hb_gemv_noalloc(wd.data_ptr(), None, 0, rows, k, xd.data_ptr(), batch, y.data_ptr(),
                                         flags, am.data_ptr(), stream))
        torch.cuda.synchronize()
        ref = y_ref.cpu().numpy()
        got = y.cpu().numpy()
        assert np.all(np.abs(got - ref) <= 1e-5 * np.abs(ref) + 1e-6)
        assert np.array_equal(am.cpu().numpy(), am_ref.cpu().numpy())
        assert np.array_equal(am.cpu().numpy(), got.argmax(axis=1).astype(np.int32))


def test_noalloc_rejects_oversized_requests():
    lib = hb_lib.load()
    rc = lib.hb_gemv_noalloc(ctypes.c_void_p(256), None, 0, 896, 896, ctypes.c_void_p(256), 9, None,
                             hb_lib.HB_GEMV_OUT_NONE | hb_lib.HB_GEMV_ARGMAX, ctypes.c_void_p(256), None)
    assert rc == hb_lib.HB_ERR_UNSUPPORTED
    assert b"scratch" in lib.hb_library_error()


def _fp32_reference(w, x, scales=None):
    ref = x.astype(np.float32) @ w.astype(np.float32).T
    return ref * scales[None, :] if scales is not None else ref


def test_noalloc_w8_and_argmax_only_against_fp32():
    """W8 weights (int8 + FP32 row scales) with FP32 output, and the same
    product with argmax only (HB_GEMV_OUT_NONE): both against FP32 numpy."""
    import torch
    from runtime.quantize import quantize_per_output_channel

    lib = hb_lib.load()
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    rows, k, batch = 4864, 896, 3
    rng = np.random.default_rng(11)
    wf = rng.standard_normal((rows, k), dtype=np.float32) * 0.02
    q, scales = quantize_per_output_channel(wf)
    x = rng.standard_normal((batch, k), dtype=np.float32).astype(bfloat16)
    dev = torch.device("cuda:0")
    wd = torch.from_numpy(layout.pack_matrix_bytes(np.ascontiguousarray(q))).to(dev)
    sd = torch.from_numpy(np.ascontiguousarray(scales, np.float32)).to(dev)
    xd = torch.from_numpy(np.ascontiguousarray(x).view(np.int16)).to(dev)
    ref = _fp32_reference(q, x, scales)
    y, am = _outputs(rows, batch)
    fp = ctypes.cast(sd.data_ptr(), ctypes.POINTER(ctypes.c_float))
    hb_lib.check(lib.hb_gemv_noalloc(wd.data_ptr(), fp, hb_lib.HB_WEIGHTS_W8, rows, k, xd.data_ptr(), batch,
                                     y.data_ptr(), hb_lib.HB_GEMV_OUT_F32 | hb_lib.HB_GEMV_ARGMAX, am.data_ptr(),
                                     stream))
    torch.cuda.synchronize()
    got = y.cpu().numpy()
    assert np.all(np.abs(got - ref) <= 1e-4 * np.abs(ref) + 1e-5), np.abs(got - ref).max()
    assert np.array_equal(am.cpu().numpy(), got.argmax(axis=1).astype(np.int32))
    _, am2 = _outputs(rows, batch)
    hb_lib.check(lib.hb_gemv_noalloc(wd.data_ptr(), fp, hb_lib.HB_WEIGHTS_W8, rows, k, xd.data_ptr(), batch, None,
                                     hb_lib.HB_GEMV_OUT_NONE | hb_lib.HB_GEMV_ARGMAX, am2.data_ptr(), stream))
    torch.cuda.synchronize()
    assert np.array_equal(am2.cpu().numpy(), am.cpu().numpy())


def test_noalloc_back_to_back_grid_sizes_on_one_stream():
    """A 151,936-row call (one CTA per SM) and an 896-row call (112 CTAs)
    queued on one stream without a synchronisation between them: each
    equals hb_gemv on its own scratch and the FP32 reference."""
    import torch

    lib = hb_lib.load()
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    flags = hb_lib.HB_GEMV_OUT_F32 | hb_lib.HB_GEMV_ARGMAX
    cases = []
    for rows, k, batch in ((151936, 896, 2), (896, 896, 2)):
        rng = np.random.default_rng([rows, 3])
        w = rng.standard_normal((rows, k), dtype=np.float32).astype(bfloat16)
        x = rng.standard_normal((batch, k), dtype=np.float32).astype(bfloat16)
        dev = torch.device("cuda:0")
        wd = torch.from_numpy(layout.pack_matrix_bytes(w)).to(dev)
        xd = torch.from_numpy(np.ascontiguousarray(x).view(np.int16)).to(dev)
        y, am = _outputs(rows, batch)
        cases.append((rows, k, batch, w, x, wd, xd, y, am))
    for rows, k, batch, w, x, wd, xd, y, am in cases:
        hb_lib.check(lib.hb_gemv_noalloc(wd.data_ptr(), None, 0, rows, k, xd.data_ptr(), batch, y.data_ptr(), flags,
                                         am.data_ptr(), stream))
    torch.cuda.synchronize()
    for rows, k, batch, w, x, wd, xd, y, am in cases:
        ref = _fp32_reference(w, x)
        got = y.cpu().numpy()
        assert np.all(np.abs(got - ref) <= 1e-4 * np.abs(ref) + 1e-4 * np.sqrt(k)), (rows, np.abs(got - ref).max())
        y2, am2 = _outputs(rows, batch)
        nscratch = lib.hb_gemv_scratch_bytes(rows, batch)
        scratch = torch.zeros(nscratch, dtype=torch.uint8, device="cuda:0")
        hb_lib.check(lib.hb_gemv(wd.data_ptr(), None, 0, rows, k, xd.data_ptr(), batch, y2.data_ptr(), flags,
                                 am2.data_ptr(), scratch.data_ptr(), nscratch, stream))
        torch.cuda.synchronize()
        assert np.array_equal(y2.cpu().numpy(), got)
        assert np.array_equal(am2.cpu().numpy(), am.cpu().numpy())


def test_noalloc_reports_a_device_wait_that_gave_up():
    """The first CTA of the next launch waits on a flag nothing sets
    (hb_test_gemv_stall_next, a 1 ms limit): the launch aborts and every
    batch row's argmax reads -1, the in-band timeout report of the
    allocation-free entry point; the next call is correct again.  No GPU
    fault is involved."""
    import torch

    lib = hb_lib.load()
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    rows, k, batch = 151936, 896, 2
    wd, xd = _case(rows, k, batch, 21)
    _, am = _outputs(rows, batch)
    am.fill_(7)
    hb_lib.check(lib.hb_test_gemv_stall_next(1_000_000))
    hb_lib.check(lib.hb_gemv_noalloc(wd.data_ptr(), None, hb_lib.HB_WEIGHTS_BF16, rows, k, xd.data_ptr(), batch, None,
                                     hb_lib.HB_GEMV_OUT_NONE | hb_lib.HB_GEMV_ARGMAX, am.data_ptr(), stream))
    torch.cuda.synchronize()
    assert am.cpu().numpy().tolist() == [-1] * batch
    _, again = _outputs(rows, batch)
    hb_lib.check(lib.hb_gemv_noalloc(wd.data_ptr(), None, hb_lib.HB_WEIGHTS_BF16, rows, k, xd.data_ptr(), batch, None,
                                     hb_lib.HB_GEMV_OUT_NONE | hb_lib.HB_GEMV_ARGMAX, again.data_ptr(), stream))
    torch.cuda.synchronize()
    assert all(0 <= t < rows for t in again.cpu().numpy().tolist())
