"""Checkpoint tensor tables and covariate arrays in the C ABI's layout (tsfm_tensor,
tsfm_covariates of include/tsfm_b200.h). Loads no native library."""
import numpy as np

from .abi import DTYPE, Covariates, Tensor

_NP_DTYPE = {np.dtype(np.float32): "F32", np.dtype(np.float16): "F16", np.dtype(np.uint16): "BF16"}


def tensor_table(tensors):
    """(ctypes array of tsfm_tensor, keep-alive list) over a name -> numpy array mapping.
    uint16 arrays are read as raw bfloat16 bits."""
    keep = []
    arr = (Tensor * len(tensors))()
    for i, name in enumerate(sorted(tensors)):
        a = np.ascontiguousarray(tensors[name])
        if a.dtype not in _NP_DTYPE:
            raise TypeError(f"tensor {name}: unsupported dtype {a.dtype}")
        nb = name.encode()
        keep += [a, nb]
        arr[i].name = nb
        arr[i].data = a.ctypes.data
        arr[i].dtype = DTYPE[_NP_DTYPE[a.dtype]]
        arr[i].numel = a.size
    return arr, keep


def covariates(past=None, known=None, cat_past=None, cat_known=None):
    """(tsfm_covariates, keep-alive list) over (series, channels, len) arrays
    (timestral/forecaster.zig:37-46): `past` and `cat_past` cover the context (len = t), `known`
    and `cat_known` the context plus the horizon (len = t + horizon); NaN marks a missing value.
    Numeric channels are float32, categorical codes float64."""
    c, keep = Covariates(), []
    for name, arr, dt in (("past", past, np.float32), ("known", known, np.float32),
                          ("cat_past", cat_past, np.float64), ("cat_known", cat_known, np.float64)):
        if arr is None:
            continue
        a = np.ascontiguousarray(arr, dtype=dt)
        if a.ndim != 3:
            raise ValueError(f"{name} covariates must be (series, channels, len)")
        keep.append(a)
        setattr(c, name, a.ctypes.data)
        setattr(c, "n_" + name, a.shape[1])
    return c, keep
