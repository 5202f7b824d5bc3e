"""Series CSV input, split and parsed on the GPU: the tsfm-zig reader's parseBlocks
(core/series.zig:21-68). Blank-line-separated blocks of equal-length rows; '#' lines skipped;
comma- or space-separated values; empty or unparsable tokens are NaN."""
import ctypes

import numpy as np

from ._native import check, lib

_SZ = ctypes.c_size_t


def parse_blocks(text, device=0):
    """(blocks, rows, len) float64 array of a series file's text (bytes or str)."""
    if isinstance(text, str):
        text = text.encode()
    buf = np.frombuffer(text, dtype=np.uint8) if text else np.zeros(1, np.uint8)
    b, r, n = _SZ(0), _SZ(0), _SZ(0)
    check(lib.tsfm_parse_blocks(buf.ctypes.data, len(text), device, None, 0, ctypes.byref(b), ctypes.byref(r),
                                ctypes.byref(n)))
    out = np.empty((b.value, r.value, n.value), np.float64)
    check(lib.tsfm_parse_blocks(buf.ctypes.data, len(text), device, out.ctypes.data, out.size, ctypes.byref(b),
                                ctypes.byref(r), ctypes.byref(n)))
    return out


def parse_blocks_device(text_ptr, length, values_ptr=None, values_f32_ptr=None, capacity=0, stream=0):
    """Device-resident variant: text and outputs are device pointers of the current device.
    Returns (blocks, rows, len); with no output pointer only the shape is computed."""
    b, r, n = _SZ(0), _SZ(0), _SZ(0)
    check(lib.tsfm_parse_blocks_device(text_ptr, length, values_ptr, values_f32_ptr, capacity, ctypes.byref(b),
                                       ctypes.byref(r), ctypes.byref(n), stream))
    return b.value, r.value, n.value
