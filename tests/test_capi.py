"""The C-ABI surface without compute: the library loads, exports every function the header
declares, reports errors as codes + messages, and checks configs and checkpoint tables before it
touches a device. Family detection mirrors core/family.zig's tests. CPU only."""
import ctypes
import os
import re

import numpy as np
import pytest

import tsfm_b200 as tb
from tsfm_b200 import config as cm
from tsfm_b200 import synthetic as syn
from tsfm_b200._native import SIGNATURES

from helpers import ROOT, has_gpu


def header_functions():
    text = open(os.path.join(ROOT, "include", "tsfm_b200.h")).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(tsfm_\w+)\s*\(", text)))


def test_library_exports_every_declared_function():
    names = header_functions()
    assert len(names) >= 20
    for n in names:
        assert hasattr(tb.lib, n), n
    assert sorted(SIGNATURES) == names


def test_library_is_the_in_tree_build():
    assert os.path.dirname(tb.LIB_PATH).startswith(os.path.join(ROOT, "tsfm-zig_b200"))
    assert tb.lib.tsfm_version().decode().startswith("tsfm-b200")


def test_status_strings():
    for code in tb.STATUS_NAMES:
        assert tb.lib.tsfm_status_string(code)
    assert tb.lib.tsfm_status_string(999) == b"unknown status"


def test_registry_detects_each_family():
    assert cm.detect(syn.chronos2_config(num_layers=1)) == "chronos2"
    assert cm.detect(syn.bolt_config(num_layers=1)) == "chronos_bolt"
    assert cm.detect(syn.timestral_config(num_layers=1)) == "timestral"
    # No silent fallback: a config nobody claims is an error (core/family.zig:150-155).
    assert cm.detect({}) is None
    with pytest.raises(cm.UnsupportedArchitecture):
        cm.parse({"architectures": ["Other"]})


def test_has_architecture_tolerates_malformed_configs():
    # core/family.zig:168-176
    assert cm.has_architecture({"architectures": ["X", "Y"]}, "Y")
    assert not cm.has_architecture({"architectures": ["X"]}, "Y")
    assert not cm.has_architecture({}, "Y")
    assert not cm.has_architecture({"architectures": "Y"}, "Y")
    assert not cm.has_architecture([], "Y")
    assert not cm.has_architecture({"architectures": [1, None]}, "Y")


def tiny_c2():
    return syn.chronos2_config(d_model=128, d_ff=256, num_heads=2, num_layers=1, context_length=256,
                               max_output_patches=4)


def create(cfg, tensors, compute="bf16"):
    parsed = cm.parse(cfg)
    table, keep = tb.tensor_table(tensors)
    h = ctypes.c_void_p()
    devs = (ctypes.c_int32 * 1)(0)
    st = tb.lib.tsfm_model_create(ctypes.byref(parsed.struct), table, len(tensors), tb._native.COMPUTE[compute],
                                  devs, 1, ctypes.byref(h))
    if st == 0:
        tb.lib.tsfm_model_destroy(h)
    return st, tb.last_error()


def test_invalid_config_is_rejected_before_any_device():
    cfg = tiny_c2()
    cfg["d_kv"] = 32  # d_model != num_heads * d_kv
    st, msg = create(cfg, {})
    assert tb.STATUS_NAMES[st] == "INVALID_CONFIG" and "InvalidConfig" in msg
    cfg = tiny_c2()
    cfg["chronos_config"]["use_reg_token"] = False
    assert tb.STATUS_NAMES[create(cfg, {})[0]] == "INVALID_CONFIG"


def test_checkpoint_table_errors_mirror_weights_get():
    # core/safetensors.zig:59-79: missing tensor, element count, dtype.
    cfg = tiny_c2()
    w = syn.random_checkpoint(cfg)
    bad = dict(w)
    del bad["encoder.block.0.layer.2.mlp.wo.weight"]
    st, msg = create(cfg, bad)
    assert tb.STATUS_NAMES[st] == "MISSING_TENSOR" and "mlp.wo.weight" in msg
    bad = dict(w)
    bad["shared.weight"] = np.zeros((3, 128), np.float32)
    st, msg = create(cfg, bad)
    assert tb.STATUS_NAMES[st] == "SHAPE_MISMATCH" and "shared.weight" in msg
    with pytest.raises(TypeError):
        tb.tensor_table({"x": np.zeros(3, np.float64)})


def test_unsupported_compute_type():
    st, msg = create(tiny_c2(), syn.random_checkpoint(tiny_c2()), compute="tf32")
    assert tb.STATUS_NAMES[st] == "UNSUPPORTED"


@pytest.mark.skipif(has_gpu(), reason="checks the no-device path")
def test_no_device_is_an_error_not_a_fallback():
    st, msg = create(tiny_c2(), syn.random_checkpoint(tiny_c2()))
    assert tb.STATUS_NAMES[st] == "NO_DEVICE"
    n = ctypes.c_int32(-1)
    assert tb.STATUS_NAMES[tb.lib.tsfm_device_count(ctypes.byref(n))] == "NO_DEVICE" and n.value == 0


def test_forecast_argument_checks_need_no_device():
    # null model / wrong family are reported, never crash
    assert tb.STATUS_NAMES[tb.lib.tsfm_forecast_chronos2(None, None, 1, 1, 1, None)] == "INVALID_ARGUMENT"
    opts = tb._native.TimestralOptions()
    tb.lib.tsfm_timestral_default_options(ctypes.byref(opts))
    assert opts.per_shot_horizon_patches == 32 and opts.symmetric_averaging == 1
    assert abs(opts.quantile_real_cap_k - 1e4) < 1e-3


def test_synthetic_series_statistics():
    x = syn.seeded_series(8, 2048, seed=1)
    frac = np.isnan(x).mean()
    assert 0.03 < frac < 0.07
    assert np.array_equal(np.isnan(x), np.isnan(syn.seeded_series(8, 2048, seed=1)))


def test_product_relative_bucket_matches_reference_table(kat):
    # The library's own relativeBucket (host code that builds the Bolt encoder's bias table) against
    # the reference's 281 expected bucket ids (chronos_bolt/model.zig test block, via kat.json), bit
    # for bit, and against transformers' T5 over a wider range of offsets.
    k = kat["relative_bucket"]
    got = [tb.lib.tsfm_relative_bucket(k["rel_start"] + i, k["num_buckets"], k["max_distance"])
           for i in range(len(k["expected"]))]
    assert got == k["expected"]
    t5 = pytest.importorskip("transformers.models.t5.modeling_t5")
    torch = pytest.importorskip("torch")
    rel = torch.arange(-700, 701)
    want = t5.T5Attention._relative_position_bucket(rel, bidirectional=True, num_buckets=32, max_distance=128)
    assert [tb.lib.tsfm_relative_bucket(int(r), 32, 128) for r in rel] == want.tolist()


def test_truncated_tensor_table_is_refused_before_any_device_work():
    # A checkpoint table cut short (the last tensors missing, as a truncated safetensors header
    # would leave it) fails with MISSING_TENSOR naming the first absent tensor, on the CPU.
    cfg = syn.chronos2_config(d_model=128, d_ff=256, num_heads=2, num_layers=2, context_length=512,
                              max_output_patches=8)
    w = syn.random_checkpoint(cfg, seed=3)
    names = sorted(w)
    kept = {k: w[k] for k in names[: len(names) // 2]}
    parsed = cm.parse(cfg)
    table, keep = tb.tensor_table(kept)
    h = ctypes.c_void_p()
    st = tb.lib.tsfm_model_create(ctypes.byref(parsed.struct), table, len(kept), 2, None, 0, ctypes.byref(h))
    assert tb.STATUS_NAMES[st] == "MISSING_TENSOR"
    assert "missing tensor" in tb.last_error()
    assert not h.value
