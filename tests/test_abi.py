"""libhawkb200.so loads without a GPU, exports every entry point that
include/hawkb200.h declares, and rejects bad arguments before touching CUDA."""

import ctypes
import re

import pytest

from conftest import REPO


def header_functions():
    text = (REPO / "include" / "hawkb200.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"^\s*(?:const\s+)?[\w\s\*]+?\b(hb_\w+)\s*\(", text, flags=re.M)))


@pytest.fixture(scope="module")
def lib():
    import importlib.util
    spec = importlib.util.spec_from_file_location("build_lib", REPO / "hawkpoint-npu-llm_b200" / "build_lib.py")
    build_lib = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(build_lib)
    build_lib.build(quiet=True)
    from runtime import hb_lib
    return hb_lib.load()


def test_every_declared_symbol_is_exported(lib):
    names = header_functions()
    assert len(names) >= 18
    from runtime import hb_lib
    for name in names:
        assert hasattr(lib, name), name
        assert name in hb_lib.SIGNATURES, f"{name} has no ctypes signature"


def test_bad_descriptors_are_rejected_without_a_device(lib):
    from runtime import hb_lib
    handle = ctypes.c_void_p()
    assert lib.hb_create(None, 0, ctypes.byref(handle)) == hb_lib.HB_ERR_INVALID_ARG
    desc = hb_lib.HbModelDesc()
    desc.abi_version = 999
    assert lib.hb_create(ctypes.byref(desc), 0, ctypes.byref(handle)) == hb_lib.HB_ERR_INVALID_ARG
    assert b"abi_version" in lib.hb_library_error()
    desc.abi_version = hb_lib.ABI_VERSION
    desc.head_dim = 32
    assert lib.hb_create(ctypes.byref(desc), 0, ctypes.byref(handle)) == hb_lib.HB_ERR_UNSUPPORTED
    assert lib.hb_destroy(None) == hb_lib.HB_OK


def test_layout_offsets_outside_the_blob_are_rejected(lib):
    import numpy as np
    from runtime import hb_lib, layout, synthetic
    shape = synthetic.TINY_QWEN
    lay = layout.plan(shape)
    table = lay.layer_table()
    table[0].w_down = lay.total  # past the end
    cos = np.zeros((64, 32), np.float32)
    desc = hb_lib.HbModelDesc(
        abi_version=hb_lib.ABI_VERSION, family=1, hidden=shape.hidden, intermediate=shape.intermediate,
        q_heads=shape.q_heads, kv_heads=shape.kv_heads, head_dim=64, layers=shape.layers, vocab=shape.vocab,
        context=64, has_qkv_bias=1, weight_format=0, max_slots=1, max_batch=1, rms_eps=1e-6,
        blob_bytes=lay.total, gamma_final=lay.gamma_final, w_lm=lay.w_lm, s_lm=0, embedding=lay.embedding)
    desc.layer_offsets = table
    desc.rope_cos = cos.ctypes.data_as(ctypes.POINTER(ctypes.c_float))
    desc.rope_sin = cos.ctypes.data_as(ctypes.POINTER(ctypes.c_float))
    handle = ctypes.c_void_p()
    assert lib.hb_create(ctypes.byref(desc), 0, ctypes.byref(handle)) == hb_lib.HB_ERR_INVALID_ARG
    assert b"outside the blob" in lib.hb_library_error()


def test_gemv_rejects_bad_shapes_on_the_host(lib):
    from runtime import hb_lib
    assert lib.hb_gemv(None, None, 0, 12, 16, None, 1, None, 0, None, None, 0, None) == hb_lib.HB_ERR_INVALID_ARG
    # K must be a multiple of 32 (the tensor-core step covers 32 columns)
    fake = ctypes.c_void_p(256)
    assert lib.hb_gemv(fake, None, 0, 16, 48, fake, 1, fake, 0, None, fake, 1 << 20, None) == hb_lib.HB_ERR_INVALID_ARG
    assert lib.hb_gemv_scratch_bytes(896, 1) >= 32


def test_missing_library_fails_loudly(monkeypatch, tmp_path):
    from runtime import hb_lib
    monkeypatch.setattr(hb_lib, "_lib", None)
    monkeypatch.setattr(hb_lib, "LIB_PATH", tmp_path / "nope.so")
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        hb_lib.load()


def test_context_rules_are_checked_on_the_host(lib):
    """Contexts above 64 positions must be whole 64-position pages, at most
    4096; the check runs before any device is touched."""
    import numpy as np
    from runtime import hb_lib, layout, synthetic
    from runtime.b200_engine import B200DecoderEngine
    shape = synthetic.TINY_QWEN
    lay = layout.plan(shape)
    table = lay.layer_table()
    for context in (100, 8192, 4160):
        cos = np.zeros((context, 32), np.float32)
        desc = hb_lib.HbModelDesc(
            abi_version=hb_lib.ABI_VERSION, family=1, hidden=shape.hidden, intermediate=shape.intermediate,
            q_heads=shape.q_heads, kv_heads=shape.kv_heads, head_dim=64, layers=shape.layers, vocab=shape.vocab,
            context=context, has_qkv_bias=1, weight_format=0, max_slots=1, max_batch=1, rms_eps=1e-6,
            blob_bytes=lay.total, gamma_final=lay.gamma_final, w_lm=lay.w_lm, s_lm=0, embedding=lay.embedding)
        desc.layer_offsets = table
        desc.rope_cos = cos.ctypes.data_as(ctypes.POINTER(ctypes.c_float))
        desc.rope_sin = cos.ctypes.data_as(ctypes.POINTER(ctypes.c_float))
        handle = ctypes.c_void_p()
        assert lib.hb_create(ctypes.byref(desc), 0, ctypes.byref(handle)) == hb_lib.HB_ERR_UNSUPPORTED
        assert b"multiple of 64" in lib.hb_library_error()
    model = synthetic.build("tiny-qwen", seed=1)
    for context in (100, 32, 8192):
        with pytest.raises(ValueError, match="multiple of 64"):
            B200DecoderEngine(model, context=context)
