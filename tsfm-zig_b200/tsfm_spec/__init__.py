"""tsfm_spec: the formats the backend and its CPU oracle share, in pure Python (no native library).

config.json parsing and family detection (config), the checkpoint tensor table and covariate
arrays in the C ABI's layout (table), the ctypes structures of include/tsfm_b200.h (abi), and
the seeded synthetic checkpoints and series the tests and the bench use (synthetic)."""
from . import abi, config, synthetic, table

__all__ = ["abi", "config", "synthetic", "table"]
