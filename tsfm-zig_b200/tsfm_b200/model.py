"""Model: a loaded checkpoint on one or more GPUs, driven through the C ABI.

Mirrors the reference's per-family entry points: `forecast_chronos2` is
chronos2/forecaster.zig:14-22, `forecast_bolt` chronos_bolt/forecaster.zig:22,
`forecast_timestral` timestral/forecaster.zig:57-69. Inputs and outputs are numpy arrays in host
memory (pinned or pageable); the *_device variants take raw device pointers.
"""
import ctypes

import numpy as np

from tsfm_spec import config as config_mod
from tsfm_spec.table import covariates, tensor_table  # noqa: F401

from ._native import COMPUTE, TimestralOptions, check, lib


def timestral_options(**kw):
    """tsfm_timestral_options with the reference defaults (timestral/forecaster.zig:21-32),
    overridden by keyword."""
    o = TimestralOptions()
    lib.tsfm_timestral_default_options(ctypes.byref(o))
    for k, v in kw.items():
        if not hasattr(o, k):
            raise TypeError(f"unknown Timestral option {k}")
        setattr(o, k, int(v) if isinstance(v, bool) else v)
    return o


class Model:
    def __init__(self, cfg, tensors, devices=(0,), compute="f16"):
        self.parsed = config_mod.parse(cfg)
        self.family = self.parsed.family
        self.cfg = cfg
        table, keep = tensor_table(tensors)
        devs = (ctypes.c_int32 * len(devices))(*devices)
        h = ctypes.c_void_p()
        check(lib.tsfm_model_create(ctypes.byref(self.parsed.struct), table, len(tensors), COMPUTE[compute], devs,
                                    len(devices), ctypes.byref(h)))
        del keep
        self._h = h
        self.devices = tuple(devices)

    @property
    def handle(self):
        return self._h

    @property
    def num_quantiles(self):
        return self.parsed.struct.num_quantiles

    @property
    def quantiles(self):
        return self.parsed.quantiles

    def close(self):
        if self._h:
            lib.tsfm_model_destroy(self._h)
            self._h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def weight_bytes(self):
        v = ctypes.c_uint64()
        check(lib.tsfm_model_weight_bytes(self._h, ctypes.byref(v)))
        return v.value

    # -- Chronos-2 / Chronos-Bolt ---------------------------------------------------------------
    def _univariate(self, fn, inputs, horizon, out=None):
        x = np.ascontiguousarray(inputs, dtype=np.float32)
        if x.ndim != 2:
            raise ValueError("inputs must be (series, steps)")
        b, t = x.shape
        if out is None:
            out = np.empty((b, horizon, self.num_quantiles), np.float32)
        check(fn(self._h, x.ctypes.data, b, t, horizon, out.ctypes.data))
        return out

    def forecast_chronos2(self, inputs, horizon, out=None):
        return self._univariate(lib.tsfm_forecast_chronos2, inputs, horizon, out)

    def forecast_bolt(self, inputs, horizon, out=None):
        return self._univariate(lib.tsfm_forecast_bolt, inputs, horizon, out)

    def forecast_chronos2_device(self, in_ptr, b, t, horizon, out_ptr, stream=0):
        check(lib.tsfm_forecast_chronos2_device(self._h, in_ptr, b, t, horizon, out_ptr, stream or None))

    def forecast_bolt_device(self, in_ptr, b, t, horizon, out_ptr, stream=0):
        check(lib.tsfm_forecast_bolt_device(self._h, in_ptr, b, t, horizon, out_ptr, stream or None))

    # -- Timestral ------------------------------------------------------------------------------
    def forecast_timestral(self, inputs, horizon, observed=None, cov=None, opts=None, out=None):
        """(series, variates, horizon, Q) quantiles after (series, variates, t) `inputs`.
        `observed` defaults to the finite entries of `inputs` (unobserved steps are passed as 0,
        as the reference expects). `cov` is a `covariates(...)` pair or None; `opts` a
        `timestral_options(...)` struct or None for the defaults."""
        x = np.ascontiguousarray(inputs, dtype=np.float32)
        if x.ndim != 3:
            raise ValueError("inputs must be (series, variates, steps)")
        if observed is None:
            observed = np.isfinite(x)
        obs = observed.view(np.uint8) if (isinstance(observed, np.ndarray) and observed.dtype == np.bool_
                                          and observed.flags.c_contiguous) else np.ascontiguousarray(observed, np.uint8)
        # The library reads inputs only where observed, so unobserved steps need no zero fill.
        b, v, t = x.shape
        if out is None:
            out = np.empty((b, v, horizon, self.num_quantiles), np.float32)
        cstruct = None if cov is None else ctypes.byref(cov[0] if isinstance(cov, tuple) else cov)
        ostruct = None if opts is None else ctypes.byref(opts)
        check(lib.tsfm_forecast_timestral(self._h, x.ctypes.data, obs.ctypes.data, b, v, t, horizon, cstruct, ostruct,
                                          out.ctypes.data))
        return out

    # -- profiling ------------------------------------------------------------------------------
    def profile(self, enable=True):
        check(lib.tsfm_profile_enable(self._h, int(enable)))

    def profile_reset(self):
        check(lib.tsfm_profile_reset(self._h))

    def profile_read(self, cls):
        n, ms, work = ctypes.c_uint64(), ctypes.c_double(), ctypes.c_double()
        check(lib.tsfm_profile_read(self._h, cls.encode(), ctypes.byref(n), ctypes.byref(ms), ctypes.byref(work)))
        return {"launches": n.value, "ms": ms.value, "work": work.value}

    def last_launch_count(self):
        n = ctypes.c_uint64()
        check(lib.tsfm_last_launch_count(self._h, ctypes.byref(n)))
        return n.value
