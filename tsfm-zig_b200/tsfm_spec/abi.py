"""The C ABI's data types (include/tsfm_b200.h) as ctypes structures, and its enumerations.

Pure description: importing this module loads no native library, so the config parser, the
checkpoint table and the synthetic inputs can feed the CPU oracle without the CUDA backend."""
import ctypes

FAMILY = {"chronos2": 1, "chronos_bolt": 2, "timestral": 3}
DTYPE = {"F32": 0, "F16": 1, "BF16": 2}
COMPUTE = {"bf16": 0, "tf32": 1, "f16": 2, "f16c": 3}
LAYER_KIND = {"time": 0, "variate": 1, "time_variate": 2, "variate_time": 3}


class Tensor(ctypes.Structure):
    _fields_ = [("name", ctypes.c_char_p), ("data", ctypes.c_void_p), ("dtype", ctypes.c_int32),
                ("numel", ctypes.c_uint64)]


class Config(ctypes.Structure):
    _fields_ = [
        ("family", ctypes.c_int32), ("d_model", ctypes.c_int32), ("d_ff", ctypes.c_int32),
        ("num_heads", ctypes.c_int32), ("d_kv", ctypes.c_int32), ("num_layers", ctypes.c_int32),
        ("num_decoder_layers", ctypes.c_int32), ("patch_size", ctypes.c_int32),
        ("context_length", ctypes.c_int32), ("max_output_patches", ctypes.c_int32),
        ("prediction_length", ctypes.c_int32), ("num_quantiles", ctypes.c_int32),
        ("quantiles", ctypes.POINTER(ctypes.c_double)), ("layer_norm_epsilon", ctypes.c_double),
        ("rope_theta", ctypes.c_double), ("time_encoding_scale", ctypes.c_double),
        ("use_arcsinh", ctypes.c_int32), ("use_reg_token", ctypes.c_int32),
        ("relative_attention_num_buckets", ctypes.c_int32),
        ("relative_attention_max_distance", ctypes.c_int32),
        ("decoder_start_token_id", ctypes.c_int32), ("reg_token_id", ctypes.c_int32),
        ("block_size", ctypes.c_int32), ("n_layer_kinds", ctypes.c_int32),
        ("layer_kinds", ctypes.POINTER(ctypes.c_int32)), ("rope_partial_factor", ctypes.c_double),
        ("minimum_scale", ctypes.c_double), ("quantile_width_factor", ctypes.c_double),
        ("covariate_enabled", ctypes.c_int32), ("attend_missing_patches", ctypes.c_int32),
        ("time_attn_gate", ctypes.c_int32), ("variate_attn_gate", ctypes.c_int32),
    ]


class Covariates(ctypes.Structure):
    _fields_ = [("past", ctypes.c_void_p), ("n_past", ctypes.c_size_t),
                ("known", ctypes.c_void_p), ("n_known", ctypes.c_size_t),
                ("cat_past", ctypes.c_void_p), ("n_cat_past", ctypes.c_size_t),
                ("cat_known", ctypes.c_void_p), ("n_cat_known", ctypes.c_size_t)]


class TimestralOptions(ctypes.Structure):
    _fields_ = [("max_context", ctypes.c_size_t), ("per_shot_horizon_patches", ctypes.c_size_t),
                ("quantile_real_cap_k", ctypes.c_float), ("extreme_value_threshold", ctypes.c_float),
                ("symmetric_averaging", ctypes.c_int32), ("clip_nonnegative", ctypes.c_int32)]


def default_timestral_options():
    """tsfm_timestral_options with the reference defaults (timestral/forecaster.zig:21-32; the
    same values tsfm_timestral_default_options writes)."""
    o = TimestralOptions()
    o.max_context = 0
    o.per_shot_horizon_patches = 32
    o.quantile_real_cap_k = 1e4
    o.extreme_value_threshold = 1e30
    o.symmetric_averaging = 1
    o.clip_nonnegative = 1
    return o
