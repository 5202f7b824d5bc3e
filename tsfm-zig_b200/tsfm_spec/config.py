"""config.json -> tsfm_config, mirroring the reference's family detection and validation.

Family detection follows core/family.zig (Registry order of src/families.zig:9: Timestral,
Chronos-2, Chronos-Bolt; the first family that claims a config wins, and a config nobody claims
is an error, not a guess). The checks each family's `validate()` makes on fields that the C
struct does not carry (activation name, patch stride) are made here; the library re-checks the
rest.
"""
import ctypes

from .abi import FAMILY, LAYER_KIND, Config

REGISTRY_ORDER = ("timestral", "chronos2", "chronos_bolt")
FAMILY_NAMES = {"timestral": "Timestral", "chronos2": "Chronos-2", "chronos_bolt": "Chronos-Bolt"}


class UnsupportedArchitecture(ValueError):
    pass


class InvalidConfig(ValueError):
    pass


def has_architecture(cfg, arch):
    """core/family.zig:113-123: `architectures` must be an array containing `arch`; malformed
    configs simply do not match."""
    if not isinstance(cfg, dict):
        return False
    a = cfg.get("architectures")
    if not isinstance(a, list):
        return False
    return any(isinstance(x, str) and x == arch for x in a)


def is_timestral(cfg):
    """timestral/config.zig:113-119: recognised by its own required keys."""
    return isinstance(cfg, dict) and all(k in cfg for k in ("block_schedule", "quantile_knots", "patch_size"))


MATCHERS = {
    "timestral": is_timestral,
    "chronos2": lambda c: has_architecture(c, "Chronos2Model"),
    "chronos_bolt": lambda c: has_architecture(c, "ChronosBoltModelForForecasting"),
}


def detect(cfg):
    """Registry.detect: the family name that claims the config, or None."""
    for fam in REGISTRY_ORDER:
        if MATCHERS[fam](cfg):
            return fam
    return None


class ParsedConfig:
    """A tsfm_config struct plus the arrays it points into."""

    def __init__(self, family, struct, keep, raw):
        self.family = family
        self.struct = struct
        self._keep = keep
        self.raw = raw

    @property
    def quantiles(self):
        return [self.struct.quantiles[i] for i in range(self.struct.num_quantiles)]


def _dbl_array(xs):
    arr = (ctypes.c_double * len(xs))(*[float(x) for x in xs])
    return arr


def parse(cfg):
    fam = detect(cfg)
    if fam is None:
        raise UnsupportedArchitecture("config.json is not a known family (supported: Timestral, Chronos-2, Chronos-Bolt)")
    s = Config()
    s.family = FAMILY[fam]
    keep = []
    if fam == "chronos2":
        ch = cfg["chronos_config"]
        if cfg.get("dense_act_fn", "relu") != "relu":
            raise InvalidConfig("UnsupportedActivation")
        if ch["input_patch_size"] != ch["output_patch_size"] or ch["input_patch_stride"] != ch["input_patch_size"]:
            raise InvalidConfig("InvalidConfig: patch size / stride")
        q = _dbl_array(ch["quantiles"])
        keep.append(q)
        s.d_model, s.d_ff, s.num_heads = cfg["d_model"], cfg["d_ff"], cfg["num_heads"]
        s.d_kv, s.num_layers = cfg["d_kv"], cfg["num_layers"]
        s.patch_size, s.context_length = ch["input_patch_size"], ch["context_length"]
        s.max_output_patches = ch["max_output_patches"]
        s.num_quantiles, s.quantiles = len(ch["quantiles"]), q
        s.layer_norm_epsilon = cfg.get("layer_norm_epsilon", 1e-6)
        s.rope_theta = cfg.get("rope_theta", 10000.0)
        s.time_encoding_scale = ch["time_encoding_scale"]
        s.use_arcsinh = int(ch.get("use_arcsinh", True))
        s.use_reg_token = int(ch.get("use_reg_token", True))
    elif fam == "chronos_bolt":
        ch = cfg["chronos_config"]
        if cfg.get("dense_act_fn", "relu") != "relu":
            raise InvalidConfig("UnsupportedActivation")
        if ch["input_patch_stride"] != ch["input_patch_size"]:
            raise InvalidConfig("UnsupportedPatchStride")
        q = _dbl_array(ch["quantiles"])
        keep.append(q)
        s.d_model, s.d_ff, s.num_heads = cfg["d_model"], cfg["d_ff"], cfg["num_heads"]
        s.d_kv, s.num_layers = cfg["d_kv"], cfg["num_layers"]
        s.num_decoder_layers = cfg["num_decoder_layers"]
        s.patch_size, s.context_length = ch["input_patch_size"], ch["context_length"]
        s.prediction_length = ch["prediction_length"]
        s.num_quantiles, s.quantiles = len(ch["quantiles"]), q
        s.layer_norm_epsilon = cfg.get("layer_norm_epsilon", 1e-6)
        s.use_reg_token = int(ch.get("use_reg_token", False))
        s.relative_attention_num_buckets = cfg.get("relative_attention_num_buckets", 32)
        s.relative_attention_max_distance = cfg.get("relative_attention_max_distance", 128)
        s.decoder_start_token_id = cfg.get("decoder_start_token_id", 0)
        s.reg_token_id = cfg.get("reg_token_id", 1)
    else:
        q = _dbl_array(cfg["quantile_knots"])
        kinds = (ctypes.c_int32 * len(cfg["block_schedule"]))()
        for i, k in enumerate(cfg["block_schedule"]):
            if k not in LAYER_KIND:
                raise InvalidConfig("UnknownLayerKind")
            kinds[i] = LAYER_KIND[k]
        keep += [q, kinds]
        s.d_model, s.num_heads = cfg["d_model"], cfg["num_heads"]
        s.d_ff = cfg["mlp_hidden_dim"]
        s.d_kv = cfg["d_model"] // cfg["num_heads"]
        s.num_layers = len(cfg["block_schedule"])
        s.n_layer_kinds, s.layer_kinds = len(cfg["block_schedule"]), kinds
        s.patch_size, s.context_length = cfg["patch_size"], cfg["context_length"]
        s.block_size = cfg["block_size"]
        s.num_quantiles, s.quantiles = len(cfg["quantile_knots"]), q
        s.layer_norm_epsilon = cfg.get("norm_eps", 1e-6)
        s.rope_theta = cfg.get("rope_theta", 10000.0)
        s.rope_partial_factor = cfg.get("rope_partial_factor", 0.5)
        s.minimum_scale = cfg.get("minimum_scale", 1e-6)
        s.quantile_width_factor = cfg.get("quantile_width_factor", 2.0)
        s.use_arcsinh = int(cfg.get("use_asinh", True))
        s.covariate_enabled = int(cfg.get("covariate_enabled", True))
        s.attend_missing_patches = int(cfg.get("attend_missing_patches", True))
        s.time_attn_gate = int(cfg.get("time_attn_gate", "sdpa_sigmoid") == "sdpa_sigmoid")
        s.variate_attn_gate = int(cfg.get("variate_attn_gate", "sdpa_sigmoid") == "sdpa_sigmoid")
        # timestral/config.zig:74-85
        if cfg["d_model"] % cfg["num_heads"]:
            raise InvalidConfig("InvalidConfig: d_model % num_heads")
        rd = int(float(cfg["d_model"] // cfg["num_heads"]) * s.rope_partial_factor)
        if rd == 0 or rd % 2:
            raise InvalidConfig("InvalidConfig: rope dim")
        if cfg.get("stabilize_with_global", False):
            raise InvalidConfig("InvalidConfig: stabilize_with_global")
        if cfg.get("attn_bias", False) or cfg.get("mlp_bias", False):
            raise InvalidConfig("UnsupportedBias")
        kn = list(cfg["quantile_knots"])
        if any(not (a < b) for a, b in zip(kn, kn[1:])) or 0.5 not in kn:
            raise InvalidConfig("InvalidConfig: quantile knots")
    return ParsedConfig(fam, s, keep, cfg)
