"""CSV output of a forecast, rendered on the GPU: the tsfm-zig CLI's writeCsv (src/main.zig:181-198).

`values` is the forecast (series, variates, horizon, levels) float32, as every forecaster returns
it (Chronos-2 / Bolt results are (series, horizon, levels): variates = 1); `levels` are the
quantile levels (float64). The text: "series,variate,step,q<level>..." then one line per
(series, variate, step) with step counted from 1, numbers printed as Zig's "{d}".
"""
import ctypes

import numpy as np

from ._native import TsfmError, check, lib

_SZ = ctypes.c_size_t


def _shape(values):
    v = np.ascontiguousarray(values, dtype=np.float32)
    if v.ndim == 3:
        v = v[:, None]
    if v.ndim != 4:
        raise ValueError("values must be (series, horizon, levels) or (series, variates, horizon, levels)")
    return v


def format_csv(values, levels, device=0):
    """The CSV text (bytes) of a forecast held in host memory."""
    v = _shape(values)
    lv = np.ascontiguousarray(levels, dtype=np.float64)
    if lv.shape != (v.shape[3],):
        raise ValueError("one level per quantile column")
    s, nv, h, q = v.shape
    need = _SZ(0)
    st = lib.tsfm_csv_format(v.ctypes.data, s, nv, h, lv.ctypes.data, q, device, None, 0, ctypes.byref(need))
    if st not in (0, 16):
        check(st)
    out = np.empty(max(need.value, 1), dtype=np.uint8)
    n = _SZ(0)
    check(lib.tsfm_csv_format(v.ctypes.data, s, nv, h, lv.ctypes.data, q, device, out.ctypes.data, out.size,
                              ctypes.byref(n)))
    return out[:n.value].tobytes()


def write_csv(values, levels, fd, device=0):
    """Writes the CSV text to an open file descriptor; returns the byte count."""
    v = _shape(values)
    lv = np.ascontiguousarray(levels, dtype=np.float64)
    if lv.shape != (v.shape[3],):
        raise ValueError("one level per quantile column")
    s, nv, h, q = v.shape
    n = _SZ(0)
    check(lib.tsfm_csv_write(v.ctypes.data, s, nv, h, lv.ctypes.data, q, device, fd, ctypes.byref(n)))
    return n.value


def format_csv_device(values_ptr, series, variates, horizon, levels, out_ptr, capacity, stream=0):
    """Device-resident variant: values and out are device pointers of the current device; returns
    the text's byte count (raises TsfmError BUFFER_TOO_SMALL, with the needed size in the message,
    when capacity is short)."""
    lv = np.ascontiguousarray(levels, dtype=np.float64)
    n = _SZ(0)
    st = lib.tsfm_csv_format_device(values_ptr, series, variates, horizon, lv.ctypes.data, lv.size, out_ptr,
                                    capacity, ctypes.byref(n), stream)
    if st == 16:
        raise TsfmError(st, f"needs {n.value} bytes")
    check(st)
    return n.value


def profile(enable=True, device=0):
    """Start (and reset) or stop per-kernel timing of the CSV kernels on a device."""
    check(lib.tsfm_csv_profile_enable(device, 1 if enable else 0))


def profile_read(kernel, device=0):
    """{"launches", "ms"} of one CSV kernel ("describe", "scan" or "text") since profiling started."""
    n, ms = ctypes.c_uint64(0), ctypes.c_double(0)
    check(lib.tsfm_csv_profile_read(device, kernel.encode(), ctypes.byref(n), ctypes.byref(ms)))
    return {"launches": n.value, "ms": ms.value}
