"""ORACLE binding — test infrastructure only (see oracle.h).

ctypes over oracle/liboracle.so, the CPU restatement of the reference forecast path. Only the
tests, __graft_entry__.smoke() and bench.py's CPU-baseline / reference legs may import this, and
only as the checker or the timed CPU baseline.
"""
import ctypes
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")


def _load():
    if not os.path.exists(LIB_PATH):
        raise ImportError(f"{LIB_PATH} missing: run `make -C oracle`")
    lib = ctypes.CDLL(LIB_PATH)
    P, SZ, I32, F = ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int32, ctypes.c_float
    sig = {
        "oracle_set_threads": (I32, [I32]),
        "oracle_get_threads": (I32, []),
        "oracle_set_operand_emulation": (I32, [I32]),
        "oracle_set_operand_emulation_class": (I32, [I32, I32]),
        "oracle_set_operand_emulation_tf32": (I32, [I32]),
        "oracle_last_error": (ctypes.c_char_p, []),
        "oracle_model_create": (I32, [P, P, SZ, ctypes.POINTER(P)]),
        "oracle_model_destroy": (None, [P]),
        "oracle_forecast_chronos2": (I32, [P, P, SZ, SZ, SZ, P]),
        "oracle_forecast_bolt": (I32, [P, P, SZ, SZ, SZ, P]),
        "oracle_forecast_timestral": (I32, [P, P, P, SZ, SZ, SZ, SZ, P, P, P]),
        "oracle_relative_bucket": (I32, [ctypes.c_int64, ctypes.c_uint32, ctypes.c_uint32]),
        "oracle_quantile_linear": (F, [P, SZ, F]),
        "oracle_self_attend": (I32, [I32, P, P, P, P, SZ, SZ, SZ, SZ, SZ, SZ, F, P, P]),
        "oracle_mask_pick": (I32, [I32, I32, I32]),
        "oracle_parse_blocks": (I32, [ctypes.c_char_p, P, SZ, ctypes.POINTER(SZ), ctypes.POINTER(SZ),
                                      ctypes.POINTER(SZ)]),
        "oracle_linear": (I32, [P, P, P, P, SZ, SZ, SZ]),
        "oracle_rmsnorm": (I32, [P, P, P, SZ, SZ, F]),
        "oracle_chronos2_patch": (I32, [P, SZ, SZ, SZ, SZ, F, I32, P, P, P, P]),
        "oracle_bolt_patch": (I32, [P, SZ, SZ, SZ, SZ, I32, P, P, P, P]),
        "oracle_timestral_block_inputs": (I32, [P, P, SZ, SZ, SZ, SZ, P, I32, ctypes.c_double, I32, I32, P, P, P, P,
                                                P]),
        "oracle_target_encode": (I32, [P, P, SZ, SZ, SZ, P, SZ, SZ, I32, P]),
        "oracle_f32_digits_batch": (None, [P, SZ, P, P]),
        "oracle_f32_digits_search_batch": (None, [P, SZ, P, P]),
        "oracle_f32_text": (SZ, [F, ctypes.c_char_p]),
        "oracle_f64_text": (SZ, [ctypes.c_double, ctypes.c_char_p]),
        "oracle_csv_format": (SZ, [P, SZ, SZ, SZ, P, SZ, P, SZ]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(lib, name)
        fn.restype, fn.argtypes = res, args
    return lib


lib = _load()


def _ptr(a):
    return None if a is None else a.ctypes.data


def check(st):
    if st != 0:
        raise RuntimeError(f"oracle status {st}: {lib.oracle_last_error().decode()}")


class OracleModel:
    """A checkpoint loaded into the CPU restatement. `parsed` is a tsfm_spec.config.ParsedConfig."""

    def __init__(self, parsed, tensors, table_fn):
        table, keep = table_fn(tensors)
        h = ctypes.c_void_p()
        check(lib.oracle_model_create(ctypes.addressof(parsed.struct), ctypes.addressof(table), len(tensors),
                                      ctypes.byref(h)))
        del keep
        self.h = h
        self.parsed = parsed
        self.q = parsed.struct.num_quantiles

    def __del__(self):
        if getattr(self, "h", None):
            lib.oracle_model_destroy(self.h)
            self.h = None

    def forecast_chronos2(self, x, horizon):
        x = np.ascontiguousarray(x, np.float32)
        out = np.empty((x.shape[0], horizon, self.q), np.float32)
        check(lib.oracle_forecast_chronos2(self.h, _ptr(x), x.shape[0], x.shape[1], horizon, _ptr(out)))
        return out

    def forecast_bolt(self, x, horizon):
        x = np.ascontiguousarray(x, np.float32)
        out = np.empty((x.shape[0], horizon, self.q), np.float32)
        check(lib.oracle_forecast_bolt(self.h, _ptr(x), x.shape[0], x.shape[1], horizon, _ptr(out)))
        return out

    def forecast_timestral(self, inputs, observed, horizon, cov=None, opts=None):
        x = np.ascontiguousarray(inputs, np.float32)
        o = np.ascontiguousarray(observed, np.uint8)
        b, v, t = x.shape
        out = np.empty((b, v, horizon, self.q), np.float32)
        check(lib.oracle_forecast_timestral(self.h, _ptr(x), _ptr(o), b, v, t, horizon,
                                            None if cov is None else ctypes.addressof(cov),
                                            None if opts is None else ctypes.addressof(opts), _ptr(out)))
        return out


def set_threads(n):
    lib.oracle_set_threads(int(n))


def get_threads():
    return lib.oracle_get_threads()


# CSV output (oracle_csv.cpp).
def f32_digits(x, search=False):
    """(digits, exponent) arrays of the shortest round-trip decimal of each float32 magnitude:
    Ryu, or (search=True) the printf / strtof digit-count search."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    e = np.empty(x.size, dtype=np.int32)
    if search:
        d = np.empty(x.size, dtype=np.uint64)
        lib.oracle_f32_digits_search_batch(x.ctypes.data, x.size, d.ctypes.data, e.ctypes.data)
    else:
        d = np.empty(x.size, dtype=np.uint32)
        lib.oracle_f32_digits_batch(x.ctypes.data, x.size, d.ctypes.data, e.ctypes.data)
    return d.astype(np.uint64), e


def f32_text(x):
    buf = ctypes.create_string_buffer(64)
    n = lib.oracle_f32_text(float(np.float32(x)), buf)
    return buf.raw[:n].decode()


def f64_text(x):
    buf = ctypes.create_string_buffer(64)
    n = lib.oracle_f64_text(float(x), buf)
    return buf.raw[:n].decode()


def csv_format(values, levels):
    """writeCsv text (bytes) of a (series, variates, horizon, levels) forecast."""
    v = np.ascontiguousarray(values, dtype=np.float32)
    if v.ndim == 3:
        v = v[:, None]
    lv = np.ascontiguousarray(levels, dtype=np.float64)
    s, nv, h, q = v.shape
    n = lib.oracle_csv_format(v.ctypes.data, s, nv, h, lv.ctypes.data, q, None, 0)
    out = np.empty(max(n, 1), dtype=np.uint8)
    lib.oracle_csv_format(v.ctypes.data, s, nv, h, lv.ctypes.data, q, out.ctypes.data, out.size)
    return out[:n].tobytes()
