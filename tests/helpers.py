"""Shared test helpers (paths, device probe, tolerance scale)."""
import os

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def has_gpu():
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


def instance_scale(x):
    """Population std of the observed values per series (the instance-norm scale of
    chronos2/forecaster.zig:100-119), 0 -> 1e-5, all-missing -> 1: the sigma of the tolerance."""
    out = []
    for row in np.asarray(x, np.float64):
        obs = row[~np.isnan(row)]
        if obs.size == 0:
            out.append(1.0)
            continue
        s = float(np.sqrt(np.mean((obs - obs.mean()) ** 2)))
        out.append(s if s > 0 else 1e-5)
    return np.array(out)


def e4m3_bits(x):
    """E4M3 encodings (uint8) of float32 values, round to nearest even and saturating at +-448
    (the `cvt.rn.satfinite.e4m3x2.f32` conversion): the FP8 companions of corrected products are
    compared with these bit for bit."""
    x = np.asarray(x, np.float32)
    a = np.abs(x).astype(np.float64)
    sign = np.where(np.signbit(x), 0x80, 0).astype(np.uint8)
    out = np.zeros(x.shape, np.uint8)
    sub = a < 2.0 ** -6
    q = np.rint(a[sub] / 2.0 ** -9).astype(np.int64)  # 0..8; 8 encodes 2^-6 (exponent field 1)
    out[sub] = q.astype(np.uint8)
    norm = ~sub & np.isfinite(a)
    an = np.minimum(a[norm], 448.0)
    e = np.floor(np.log2(an)).astype(np.int64)
    m = np.rint(an / np.exp2(e - 3)).astype(np.int64) - 8
    carry = m == 8
    e = np.where(carry, e + 1, e)
    m = np.where(carry, 0, m)
    code = ((e + 7) << 3) | m
    out[norm] = np.minimum(code, 0x7E).astype(np.uint8)
    out[~np.isfinite(a)] = np.where(np.isnan(a[~np.isfinite(a)]), 0x7F, 0x7E).astype(np.uint8)
    return out | sign
