"""ctypes binding of libhawkb200.so (declarations in include/hawkb200.h).

Loading fails loudly when the library is missing: there is no CPU fallback.
"""

import ctypes
import os
from pathlib import Path

from runtime.layout import HbLayerOffsets

PKG = Path(__file__).resolve().parents[1]
LIB_PATH = Path(os.environ.get("HAWKB200_LIB", PKG / "lib" / "libhawkb200.so"))

HB_OK = 0
HB_ERR_INVALID_ARG = -1
HB_ERR_CUDA = -2
HB_ERR_DEVICE_TIMEOUT = -3
HB_ERR_UNSUPPORTED = -4
HB_ERR_STATE = -5

HB_WEIGHTS_BF16 = 0
HB_WEIGHTS_W8 = 1

HB_STEP_ARGMAX = 1
HB_STEP_LOGITS = 2
HB_STEP_DEVICE_LOGITS = 4
HB_DUMP_HIDDEN = 0
HB_DUMP_KV = 1
HB_DUMP_TRACE = 2

HB_GEMV_OUT_BF16 = 0
HB_GEMV_OUT_F32 = 1
HB_GEMV_OUT_NONE = 2
HB_GEMV_ARGMAX = 4

ABI_VERSION = 1


class HbModelDesc(ctypes.Structure):
    _fields_ = [
        ("abi_version", ctypes.c_int32),
        ("family", ctypes.c_int32),
        ("hidden", ctypes.c_int32),
        ("intermediate", ctypes.c_int32),
        ("q_heads", ctypes.c_int32),
        ("kv_heads", ctypes.c_int32),
        ("head_dim", ctypes.c_int32),
        ("layers", ctypes.c_int32),
        ("vocab", ctypes.c_int32),
        ("context", ctypes.c_int32),
        ("has_qkv_bias", ctypes.c_int32),
        ("weight_format", ctypes.c_int32),
        ("max_slots", ctypes.c_int32),
        ("max_batch", ctypes.c_int32),
        ("rms_eps", ctypes.c_float),
        ("reserved0", ctypes.c_int32),
        ("blob_bytes", ctypes.c_uint64),
        ("gamma_final", ctypes.c_uint64),
        ("w_lm", ctypes.c_uint64),
        ("s_lm", ctypes.c_uint64),
        ("embedding", ctypes.c_uint64),
        ("layer_offsets", ctypes.POINTER(HbLayerOffsets)),
        ("rope_cos", ctypes.POINTER(ctypes.c_float)),
        ("rope_sin", ctypes.POINTER(ctypes.c_float)),
    ]


class HbSampling(ctypes.Structure):
    """hb_sampling: one token selection's parameters (include/hawkb200.h)."""

    _fields_ = [
        ("temperature", ctypes.c_float),
        ("top_p", ctypes.c_float),
        ("repetition_penalty", ctypes.c_float),
        ("presence_penalty", ctypes.c_float),
        ("frequency_penalty", ctypes.c_float),
        ("top_k", ctypes.c_int32),
        ("n_history", ctypes.c_int32),
        ("history_tokens", ctypes.POINTER(ctypes.c_int32)),
        ("history_counts", ctypes.POINTER(ctypes.c_float)),
        ("n_bias", ctypes.c_int32),
        ("bias_tokens", ctypes.POINTER(ctypes.c_int32)),
        ("bias_values", ctypes.POINTER(ctypes.c_float)),
        ("uniform", ctypes.c_double),
    ]


class HbError(RuntimeError):
    def __init__(self, code, message):
        super().__init__(f"libhawkb200 error {code}: {message}")
        self.code = code


class HbTimeout(HbError):
    """A bounded device wait gave up; the engine is still usable."""


_P = ctypes.c_void_p
_I = ctypes.c_int
_I32P = ctypes.POINTER(ctypes.c_int32)
_FP = ctypes.POINTER(ctypes.c_float)

# name -> (restype, argtypes); every symbol include/hawkb200.h declares
SIGNATURES = {
    "hb_create": (_I, [ctypes.POINTER(HbModelDesc), _I, ctypes.POINTER(_P)]),
    "hb_load_weights": (_I, [_P, _P, ctypes.c_size_t, _I]),
    "hb_destroy": (_I, [_P]),
    "hb_step": (_I, [_P, _I, _I, _I, _I, _FP, _I32P]),
    "hb_prefill": (_I, [_P, _I, _I32P, _I, _I, _FP, _I32P]),
    "hb_generate": (_I, [_P, _I, _I32P, _I, _I, _I, _I32P]),
    "hb_step_batch": (_I, [_P, _I, _I32P, _I32P, _I32P, _I, _FP, _I32P]),
    "hb_reset": (_I, [_P, _I]),
    "hb_copy_prefix": (_I, [_P, _I, _I, _I]),
    "hb_last_error": (ctypes.c_char_p, [_P]),
    "hb_debug_dump": (_I, [_P, _I, _P, ctypes.c_size_t]),
    "hb_profile": (_I, [_P, _I]),
    "hb_profile_read": (_I, [_P, _FP, _FP, _I, ctypes.POINTER(_I)]),
    "hb_set_stream": (_I, [_P, _P]),
    "hb_test_stall_next": (_I, [_P, ctypes.c_uint64]),
    "hb_test_gemv_stall_next": (_I, [ctypes.c_uint64]),
    "hb_gemv_scratch_bytes": (ctypes.c_size_t, [_I, _I]),
    "hb_gemv": (_I, [_P, _P, _I, _I, _I, _P, _I, _P, _I, _P, _P, ctypes.c_size_t, _P]),
    "hb_gemv_noalloc": (_I, [_P, _P, _I, _I, _I, _P, _I, _P, _I, _P, _P]),
    "hb_sampler_create": (_I, [_I, _I, ctypes.POINTER(_P)]),
    "hb_sampler_select": (_I, [_P, _P, _I, ctypes.POINTER(HbSampling), _I32P]),
    "hb_sampler_destroy": (_I, [_P]),
    "hb_sample": (_I, [_P, _I, ctypes.POINTER(HbSampling), _I32P]),
    "hb_sample_batch": (_I, [_P, _I, _I32P, ctypes.POINTER(HbSampling), _I32P]),
    "hb_read_logits": (_I, [_P, _I, _FP]),
    "hb_sampler_logprobs": (_I, [_P, _P, _I, _I, _I, ctypes.POINTER(ctypes.c_double), _I32P,
                                 ctypes.POINTER(ctypes.c_double)]),
    "hb_logprobs": (_I, [_P, _I, _I, _I, ctypes.POINTER(ctypes.c_double), _I32P, ctypes.POINTER(ctypes.c_double)]),
    "hb_tc_gemm_scratch_bytes": (ctypes.c_size_t, [_I, _I, _I]),
    "hb_tc_gemm": (_I, [_P, _I, _I, _P, _I, _FP, _P, ctypes.c_size_t, _P]),
    "hb_tc_gemm_status": (_I, [_P, _P]),
    "hb_step_rows": (_I, [_P, _I, _I32P, _I32P, _I32P, _I, _I32P, _I32P, _FP]),
    "hb_prefill_tc": (_I, [_P, _I, _I32P, _I, _I, _FP, _I32P]),
    "hb_library_error": (ctypes.c_char_p, []),
    "hb_device_sm_count": (_I, [_I]),
}

_lib = None


def load():
    """Load libhawkb200.so once and declare every entry point."""
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        raise RuntimeError(
            f"{LIB_PATH} is missing: build it with "
            "`python hawkpoint-npu-llm_b200/build_lib.py` (there is no CPU fallback)"
        )
    lib = ctypes.CDLL(str(LIB_PATH))
    for name, (restype, argtypes) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = restype
        fn.argtypes = argtypes
    _lib = lib
    return lib


def check(rc, engine=None):
    """Raise the Python exception matching a libhawkb200 return code."""
    if rc == HB_OK:
        return
    lib = load()
    message = (lib.hb_last_error(engine) if engine else lib.hb_library_error()) or b""
    message = message.decode(errors="replace")
    if rc == HB_ERR_INVALID_ARG:
        raise ValueError(message)
    if rc == HB_ERR_DEVICE_TIMEOUT:
        raise HbTimeout(rc, message)
    raise HbError(rc, message)
