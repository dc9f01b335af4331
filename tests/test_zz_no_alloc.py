"""hb_gemv_noalloc: the GEMV entry point for callers that cannot allocate
device memory (its scratch is a fixed array inside the library).

Called through the C ABI on the same inputs as hb_gemv (which takes a scratch
buffer from the caller), twice in a row, and compared with it: the two run the
same kernel, so outputs and argmax must agree within the GEMV tests' tolerance
(they are in fact expected to be identical).  The second call checks that the
state a call leaves in the shared array does not leak into the next one.
This file is named to be collected last.
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
