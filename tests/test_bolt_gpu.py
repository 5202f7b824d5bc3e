"""Chronos-Bolt forecasts on the GPU against the oracle (the CPU restatement of
chronos_bolt/forecaster.zig + chronos_bolt/model.zig), including the long-horizon loop that
feeds every quantile path back and reduces the q^2 samples per step (chronos_bolt/forecaster.zig:45-78).

Tolerance: max |dq| <= 1e-2 * sigma per series (sigma = the population std of the observed
context, the instance-norm scale; Bolt has no sinh, so the bound applies as is), plus 4 float32
ulps of max(|q|, |loc|) for the float32 storage of q = v * sigma + loc."""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

import tsfm_b200 as tb  # noqa: E402
from oracle import binding as ob  # noqa: E402
from tsfm_b200 import synthetic as syn  # noqa: E402

from helpers import instance_scale  # noqa: E402

pytestmark = pytest.mark.gpu
TOL = 1e-2
EPS32 = float(np.finfo(np.float32).eps)


def rel_err(got, want, x):
    sig = instance_scale(x)[:, None, None]
    loc = np.array([np.nanmean(r) if np.isfinite(r).any() else 0.0 for r in x])[:, None, None]
    floor = 4 * EPS32 * np.maximum(np.abs(want), np.abs(loc))
    return float(np.max(np.maximum(np.abs(got - want) - floor, 0.0) / sig))


def tiny_cfg(**kw):
    base = dict(d_model=128, d_ff=256, num_heads=2, num_layers=2, num_decoder_layers=1, context_length=256,
                prediction_length=16)
    base.update(kw)
    return syn.bolt_config(**base)


def models(cfg, seed=4):
    w = syn.random_checkpoint(cfg, seed=seed, norm_jitter=0.1)
    gpu = tb.Model(cfg, w)
    return gpu, ob.OracleModel(gpu.parsed, w, tb.tensor_table)


@pytest.fixture(scope="module")
def tiny():
    return models(tiny_cfg())


def edge_inputs(t, seed=6):
    x = syn.seeded_series(7, t, seed=seed)
    x[1, :] = np.nan          # all missing
    x[2, :] = -1.5            # constant
    x[3, : t // 2] = np.nan   # leading gap
    x[4, 16:48] = np.nan      # missing patches
    return x


@pytest.mark.parametrize("t,horizon", [(250, 16), (256, 10), (300, 48), (40, 33), (17, 16)])
def test_tiny_matches_oracle(tiny, t, horizon):
    gpu, ora = tiny
    x = edge_inputs(t)
    got = gpu.forecast_bolt(x, horizon)
    want = ora.forecast_bolt(x, horizon)
    assert got.shape == want.shape == (7, horizon, 9)
    assert np.isfinite(got).all()
    assert rel_err(got, want, x[:, -256:]) <= TOL


def test_without_reg_token_and_no_valid_key():
    # use_reg_token = false: an all-missing series has no valid key at all, and the reference's
    # additive -floatMax mask then averages every key uniformly.
    # The reference validates token ids against the vocabulary, which shrinks to the start token
    # alone without [REG] (chronos_bolt/config.zig:43-58).
    cfg = tiny_cfg(use_reg_token=False)
    cfg["reg_token_id"] = 0
    gpu, ora = models(cfg)
    x = edge_inputs(200)
    got = gpu.forecast_bolt(x, 40)
    want = ora.forecast_bolt(x, 40)
    assert np.isfinite(got).all()
    assert rel_err(got, want, x) <= TOL


def test_replicas_are_bit_identical(tiny):
    gpu, _ = tiny
    cfg = tiny_cfg()
    w = syn.random_checkpoint(cfg, seed=4, norm_jitter=0.1)
    two = tb.Model(cfg, w, devices=(0, 0))
    x = syn.seeded_series(9, 200, seed=3)
    assert np.array_equal(gpu.forecast_bolt(x, 40), two.forecast_bolt(x, 40))


def test_graph_replays_match_plain_runs(tiny):
    # The third call with the same shapes and buffers replays a captured CUDA graph; it must read
    # the new inputs and give exactly what a plain run gives (the host path and the device path).
    gpu, _ = tiny
    cfg = tiny_cfg()
    w = syn.random_checkpoint(cfg, seed=4, norm_jitter=0.1)
    xs = [syn.seeded_series(6, 230, seed=40 + i) for i in range(4)]
    plain = [tb.Model(cfg, w).forecast_bolt(x, 40) for x in xs]
    for x, want in zip(xs, plain):
        assert np.array_equal(gpu.forecast_bolt(x, 40), want)
    xd = torch.empty((6, 230), device="cuda")
    out = torch.empty((6, 40, 9), device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    for x, want in zip(xs, plain):
        xd.copy_(torch.from_numpy(x))
        gpu.forecast_bolt_device(xd.data_ptr(), 6, 230, 40, out.data_ptr(), s)
        assert np.array_equal(out.cpu().numpy(), want)


def test_bolt_small_shape_matches_oracle():
    # BASELINE configs[0] shape: Bolt-small (512-d, 6 layers, ctx 2048, 9 quantiles, P = 64);
    # horizon 192 runs the first block plus two quantile-path blocks.
    gpu, ora = models(syn.bolt_config(), seed=20261201)
    x = syn.seeded_series(6, 2048, seed=50)
    got = gpu.forecast_bolt(x, 192)
    want = ora.forecast_bolt(x, 192)
    assert np.isfinite(got).all()
    err = rel_err(got, want, x)
    print(f"Bolt-small configs[0]: max |dq|/sigma = {err:.3e}")
    assert err <= TOL


@pytest.mark.parametrize("dtype", [np.float32, "bf16"])
def test_bolt_base_shape_matches_oracle(dtype):
    # BASELINE configs[1] shape: Bolt-base (768-d, 12 layers, 12 heads, d_ff 3072, ctx 2048,
    # 9 quantiles, P = 64) at horizon 256 = 4 passes, every quantile path fed back
    # (chronos_bolt/forecaster.zig:45-78), from an F32 and from a BF16 checkpoint (converted on
    # the device like the reference converts at load, core/safetensors.zig:81-92).
    cfg = syn.bolt_config(d_model=768, d_ff=3072, num_heads=12, num_layers=12)
    w = syn.random_checkpoint(cfg, seed=20261201, dtype=dtype)
    gpu = tb.Model(cfg, w)
    ora = ob.OracleModel(gpu.parsed, w, tb.tensor_table)
    x = syn.seeded_series(3, 2048, seed=2000)
    got = gpu.forecast_bolt(x, 256)
    want = ora.forecast_bolt(x, 256)
    assert got.shape == (3, 256, 9)
    assert np.isfinite(got).all()
    err = rel_err(got, want, x)
    print(f"Bolt-base configs[1] ({dtype if isinstance(dtype, str) else 'f32'} checkpoint): max |dq|/sigma = {err:.3e}")
    assert err <= TOL
