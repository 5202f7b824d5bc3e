"""Chronos-2 forecasts on the GPU against the oracle (the CPU restatement of
chronos2/forecaster.zig + chronos2/model.zig) on the same random-init checkpoints and seeded
series. Tolerance (BF16 operands, FP32 accumulation): max |dq| <= 1e-2 * sigma per series, sigma =
the population std of the observed context (the instance-norm scale)."""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

import tsfm_b200 as tb  # noqa: E402
from oracle import binding as ob  # noqa: E402
from tsfm_b200 import synthetic as syn  # noqa: E402

from helpers import instance_scale  # noqa: E402

pytestmark = pytest.mark.gpu
TOL_BF16 = 1e-2


def tiny_cfg(**kw):
    base = dict(d_model=128, d_ff=256, num_heads=2, num_layers=2, context_length=512, max_output_patches=8)
    base.update(kw)
    return syn.chronos2_config(**base)


@pytest.fixture(scope="module")
def tiny():
    cfg = tiny_cfg()
    w = syn.random_checkpoint(cfg, seed=3, norm_jitter=0.1)
    gpu = tb.Model(cfg, w)
    ora = ob.OracleModel(gpu.parsed, w, tb.tensor_table)
    return cfg, w, gpu, ora


def rel_err(got, want, x):
    sig = instance_scale(x)
    return float(np.max(np.abs(got - want) / sig[:, None, None]))


def edge_inputs(t, seed=5):
    x = syn.seeded_series(8, t, seed=seed)
    x[1, :] = np.nan                # all missing: loc 0, scale 1
    x[2, :] = 3.25                  # constant: scale 0 -> 1e-5
    x[3, : t // 2] = np.nan         # long leading gap
    x[4, 16:48] = np.nan            # whole missing patches
    x[5, -1] = np.nan
    return x


@pytest.mark.parametrize("t,horizon", [(500, 100), (512, 128), (700, 1), (16, 64), (33, 17)])
def test_tiny_matches_oracle(tiny, t, horizon):
    _, _, gpu, ora = tiny
    x = edge_inputs(t)
    got = gpu.forecast_chronos2(x, horizon)
    want = ora.forecast_chronos2(x, horizon)
    assert got.shape == want.shape == (8, horizon, 21)
    assert np.isfinite(got).all()
    assert rel_err(got, want, x[:, -512:]) <= TOL_BF16


def test_replicas_are_bit_identical(tiny):
    # Series are sharded across replicas (one host thread each); the result must not depend on
    # the shard count. Two replicas on one device exercise the same sharding code path.
    cfg, w, gpu, _ = tiny
    two = tb.Model(cfg, w, devices=(0, 0))
    x = syn.seeded_series(13, 400, seed=11)
    a = gpu.forecast_chronos2(x, 77)
    b = two.forecast_chronos2(x, 77)
    assert np.array_equal(a, b)


def test_device_entry_point_matches_host_path(tiny):
    _, _, gpu, _ = tiny
    x = syn.seeded_series(5, 300, seed=2)
    host = gpu.forecast_chronos2(x, 64)
    xd = torch.from_numpy(x).cuda()
    out = torch.empty((5, 64, 21), device="cuda")
    gpu.forecast_chronos2_device(xd.data_ptr(), 5, 300, 64, out.data_ptr(), torch.cuda.current_stream().cuda_stream)
    assert np.array_equal(out.cpu().numpy(), host)


def test_argument_errors(tiny):
    _, _, gpu, _ = tiny
    with pytest.raises(tb.TsfmError, match="HORIZON_TOO_LONG"):
        gpu.forecast_chronos2(np.zeros((1, 32), np.float32), 8 * 16 + 1)
    with pytest.raises(tb.TsfmError, match="EMPTY_INPUT"):
        gpu.forecast_chronos2(np.zeros((0, 32), np.float32), 8)


def test_full_shape_chronos2_matches_oracle():
    # BASELINE configs[2] shape: 768-d, 12 layers, ctx 8192, H 1024 (2 series; the oracle needs
    # ~130 GFLOP per series).
    cfg = syn.chronos2_config()
    w = syn.random_checkpoint(cfg, seed=20261201)
    gpu = tb.Model(cfg, w)
    ora = ob.OracleModel(gpu.parsed, w, tb.tensor_table)
    x = syn.seeded_series(2, 8192, seed=100)
    got = gpu.forecast_chronos2(x, 1024)
    want = ora.forecast_chronos2(x, 1024)
    assert np.isfinite(got).all()
    assert rel_err(got, want, x) <= TOL_BF16
