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
