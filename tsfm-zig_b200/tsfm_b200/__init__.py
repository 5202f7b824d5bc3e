"""tsfm_b200: B200-native forecast backend for tsfm-zig checkpoints (Chronos-2, Chronos-Bolt,
Timestral). The compute lives in libtsfm_b200.so (sm_100a CUDA + C++ behind a C ABI); this
package is its Python binding."""
from tsfm_spec import config, synthetic

from . import csv, series
from ._native import (LIB_PATH, STATUS_NAMES, TsfmError, check, device_count, last_error, lib)
from .model import Model, covariates, tensor_table, timestral_options

__all__ = ["Model", "TsfmError", "config", "csv", "series", "synthetic", "lib", "check", "last_error", "device_count",
           "tensor_table", "covariates", "timestral_options", "LIB_PATH", "STATUS_NAMES"]
