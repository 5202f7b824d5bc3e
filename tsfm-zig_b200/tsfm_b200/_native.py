"""ctypes binding of the C ABI in include/tsfm_b200.h.

The shared library is built in-tree (``make -C tsfm-zig_b200``) next to this file. There is no
fallback: importing the package without the library raises, so nothing can silently run a CPU
path in its place.
"""
import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libtsfm_b200.so")

TSFM_OK = 0
STATUS_NAMES = {
    0: "OK", 1: "INVALID_ARGUMENT", 2: "INVALID_CONFIG", 3: "MISSING_TENSOR", 4: "SHAPE_MISMATCH",
    5: "UNSUPPORTED_DTYPE", 6: "CUDA", 7: "OUT_OF_MEMORY", 8: "DEVICE_TIMEOUT", 9: "EMPTY_INPUT",
    10: "HORIZON_TOO_LONG", 11: "UNSUPPORTED", 12: "DEGENERATE_INPUT", 13: "ASYMMETRIC_QUANTILES",
    14: "COVARIATES_UNSUPPORTED", 15: "NO_DEVICE", 16: "BUFFER_TOO_SMALL", 17: "IO",
    18: "RAGGED_INPUT", 19: "RAGGED_BLOCKS",
}
class TsfmError(RuntimeError):
    """A non-zero tsfm_status, with the library's message."""

    def __init__(self, code, message):
        self.code = code
        self.name = STATUS_NAMES.get(code, str(code))
        super().__init__(f"{self.name}: {message}")


# The structures and enumerations live in tsfm_spec.abi (pure Python, shared with the oracle).
from tsfm_spec.abi import (COMPUTE, DTYPE, FAMILY, LAYER_KIND, Config, Covariates,  # noqa: E402,F401
                           Tensor, TimestralOptions)

# Every function the header declares: name -> (restype, argtypes).
_P = ctypes.c_void_p
_I32 = ctypes.c_int32
_I64 = ctypes.c_int64
_SZ = ctypes.c_size_t
_F = ctypes.c_float
SIGNATURES = {
    "tsfm_last_error": (ctypes.c_char_p, []),
    "tsfm_status_string": (ctypes.c_char_p, [_I32]),
    "tsfm_device_count": (_I32, [ctypes.POINTER(_I32)]),
    "tsfm_version": (ctypes.c_char_p, []),
    "tsfm_model_create": (_I32, [ctypes.POINTER(Config), ctypes.POINTER(Tensor), _SZ, _I32,
                                 ctypes.POINTER(_I32), _I32, ctypes.POINTER(_P)]),
    "tsfm_model_destroy": (None, [_P]),
    "tsfm_model_weight_bytes": (_I32, [_P, ctypes.POINTER(ctypes.c_uint64)]),
    "tsfm_forecast_chronos2": (_I32, [_P, _P, _SZ, _SZ, _SZ, _P]),
    "tsfm_forecast_bolt": (_I32, [_P, _P, _SZ, _SZ, _SZ, _P]),
    "tsfm_forecast_timestral": (_I32, [_P, _P, _P, _SZ, _SZ, _SZ, _SZ, ctypes.POINTER(Covariates),
                                       ctypes.POINTER(TimestralOptions), _P]),
    "tsfm_timestral_default_options": (None, [ctypes.POINTER(TimestralOptions)]),
    "tsfm_forecast_chronos2_device": (_I32, [_P, _P, _SZ, _SZ, _SZ, _P, _P]),
    "tsfm_forecast_bolt_device": (_I32, [_P, _P, _SZ, _SZ, _SZ, _P, _P]),
    "tsfm_profile_enable": (_I32, [_P, _I32]),
    "tsfm_profile_reset": (_I32, [_P]),
    "tsfm_profile_read": (_I32, [_P, ctypes.c_char_p, ctypes.POINTER(ctypes.c_uint64),
                                 ctypes.POINTER(ctypes.c_double), ctypes.POINTER(ctypes.c_double)]),
    "tsfm_last_launch_count": (_I32, [_P, ctypes.POINTER(ctypes.c_uint64)]),
    "tsfm_weight_register": (_P, [_P, _SZ]),
    "tsfm_weight_release": (None, [_P]),
    "tsfm_sgemm_nt": (ctypes.c_int, [ctypes.c_int, ctypes.c_int, ctypes.c_int, _F, _P, ctypes.c_int, _P,
                                     ctypes.c_int, _P, ctypes.c_int, _P]),
    "tsfm_sgemm_nn": (ctypes.c_int, [ctypes.c_int, ctypes.c_int, ctypes.c_int, _P, ctypes.c_int, _P,
                                     ctypes.c_int, _P, ctypes.c_int, _P]),
    "tsfm_sgemm_nt_noalloc": (_I32, [ctypes.c_int, ctypes.c_int, ctypes.c_int, _F, _P, ctypes.c_int, _P,
                                     ctypes.c_int, _P, ctypes.c_int, _P]),
    "tsfm_kernel_linear": (_I32, [_P, _I32, _P, _I32, _P, _P, _I32, _I32, _I64, _I64, _I64, _I64, _I64,
                                  _I64, _P]),
    "tsfm_kernel_linear_corrected": (_I32, [_P, _P, _P, _P, _P, _I32, _I32, _I64, _I64, _I64, _I32, _P]),
    "tsfm_kernel_split_f16c": (_I32, [_P, _I64, _I64, _P, _P, _P]),
    "tsfm_kernel_weight_f16c": (_I32, [_P, _I64, _I64, _P, _P, ctypes.POINTER(_F), _P]),
    "tsfm_kernel_linear_f16c": (_I32, [_P, _P, _P, _P, _F, _P, _P, _P, _I32, _I32, _I64, _I64, _I64, _I32, _P]),
    "tsfm_relative_bucket": (_I32, [_I64, _I32, _I32]),
    "tsfm_test_bounded_wait": (_I32, [_I64, _P]),
    "tsfm_kernel_patch": (_I32, [_I32, _P, _I64, _I64, _I64, _I32, _F, _I32, _I32, _P, _P, _P, _P, _P]),
    "tsfm_kernel_timestral_block_inputs": (_I32, [_P, _P, _I64, _I64, _P, _P, _I64, _I32, _I32, _P, _I32,
                                                  ctypes.c_double, _I32, _I32, _P, _P, _P, _P, _P, _P]),
    "tsfm_kernel_attention": (_I32, [_P, _P, _P, _I64, _P, _I64, _P, _P, _I32, _I32, _I32, _F, _I32, _I32, _P]),
    "tsfm_kernel_attention_ex": (_I32, [_P, _P, _P, _I64, _P, _I64, _P, _I64, _P, _I64, _P, _I64, _P, _P, _I32, _I32,
                                        _I32, _F, _I32, _I32, _I32, _I32, _I32, _P]),
    "tsfm_kernel_rmsnorm": (_I32, [_P, _P, _P, _I32, _I64, _I64, _F, _P]),
    "tsfm_kernel_rmsnorm_ex": (_I32, [_P, _P, _P, _I32, _P, _I64, _I64, _I64, _F, _P]),
    "tsfm_kernel_target_encode": (_I32, [_P, _P, _I64, _I64, _I64, _P, _I64, _I64, _I32, _P, _P]),
    "tsfm_csv_format": (_I32, [_P, _SZ, _SZ, _SZ, _P, _SZ, _I32, _P, _SZ, ctypes.POINTER(_SZ)]),
    "tsfm_csv_write": (_I32, [_P, _SZ, _SZ, _SZ, _P, _SZ, _I32, _I32, ctypes.POINTER(_SZ)]),
    "tsfm_csv_format_device": (_I32, [_P, _SZ, _SZ, _SZ, _P, _SZ, _P, _SZ, ctypes.POINTER(_SZ), _P]),
    "tsfm_parse_blocks": (_I32, [_P, _SZ, _I32, _P, _SZ, ctypes.POINTER(_SZ), ctypes.POINTER(_SZ),
                                 ctypes.POINTER(_SZ)]),
    "tsfm_parse_blocks_device": (_I32, [_P, _SZ, _P, _P, _SZ, ctypes.POINTER(_SZ), ctypes.POINTER(_SZ),
                                        ctypes.POINTER(_SZ), _P]),
    "tsfm_csv_profile_enable": (_I32, [_I32, _I32]),
    "tsfm_csv_profile_read": (_I32, [_I32, ctypes.c_char_p, ctypes.POINTER(ctypes.c_uint64),
                                     ctypes.POINTER(ctypes.c_double)]),
}


def _load():
    if not os.path.exists(LIB_PATH):
        raise ImportError(
            f"tsfm_b200: {LIB_PATH} is missing; build it with `make -C tsfm-zig_b200` "
            "(there is no CPU fallback)")
    lib = ctypes.CDLL(LIB_PATH)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


lib = _load()


def last_error():
    return lib.tsfm_last_error().decode()


def check(status):
    if status != TSFM_OK:
        raise TsfmError(status, last_error())
    return status


def device_count():
    n = ctypes.c_int32(0)
    st = lib.tsfm_device_count(ctypes.byref(n))
    return n.value if st == TSFM_OK else 0
