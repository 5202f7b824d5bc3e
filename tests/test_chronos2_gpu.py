"""Chronos-2 forecasts on the GPU against the oracle (the CPU restatement of
chronos2/forecaster.zig + chronos2/model.zig) on the same random-init checkpoints and seeded
series.

Tolerance: max |dq| <= 1e-2 * sigma per series (the BF16-class bound), sigma = the population
std of the observed context (the instance-norm scale), plus 4 float32 ulps of the larger of |q|
and |loc|: the reference itself stores q = sinh(v) * sigma + loc in float32, so two correct
implementations can differ by that much (it matters only for near-constant series, where sigma
falls to 1e-5). The tiny configs run FP16 operands with FP32 accumulation; the full BASELINE
shape meets the bound in the corrected mode (FP16 + FP8 correction products, TSFM_COMPUTE_F16C),
which is tested there and on the tiny configs too. BF16 operands are checked against a looser
bound, since their 8-bit significand cannot meet 1e-2 * sigma once sinh amplifies the head's
output."""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

import tsfm_b200 as tb  # noqa: E402
from oracle import binding as ob  # noqa: E402
from tsfm_b200 import synthetic as syn  # noqa: E402

from helpers import instance_scale  # noqa: E402

pytestmark = pytest.mark.gpu
TOL = 1e-2       # F16 operands (BF16-class tolerance of the spec)
TOL_BF16_RANGE = 0.2  # BF16 operands: a sanity bound, not a parity claim
EPS32 = float(np.finfo(np.float32).eps)


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
    """max |dq| / sigma after discounting 4 float32 ulps of max(|q|, |loc|)."""
    sig = instance_scale(x)[:, None, None]
    loc = np.array([np.nanmean(r) if np.isfinite(r).any() else 0.0 for r in x])[:, None, None]
    floor = 4 * EPS32 * np.maximum(np.abs(want), np.abs(loc))
    excess = np.maximum(np.abs(got - want) - floor, 0.0)
    return float(np.max(excess / sig))


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
    assert rel_err(got, want, x[:, -512:]) <= TOL


@pytest.mark.parametrize("b,t,compute", [(8, 500, "f16"), (130, 512, "f16"), (130, 512, "bf16")])
def test_fused_norm_path_matches_oracle(b, t, compute):
    # d_model a multiple of 256: the time-attention RMSNorm of layers 1.. runs inside the previous
    # layer's wo GEMM (16-bit copy of x * s_r * gamma plus per-tile sums of squares) and the QKV
    # GEMM that reads it (rows scaled by rs / s_r). 130 series x 41 tokens (5,330 rows) takes the
    # CTA-pair tiles, 8 series the single-CTA ones; norm weights are jittered so that a wrong
    # gamma shows.
    cfg = tiny_cfg(d_model=256, d_ff=512, num_heads=4, num_layers=3)
    w = syn.random_checkpoint(cfg, seed=21, norm_jitter=0.1)
    gpu = tb.Model(cfg, w, compute=compute)
    ora = ob.OracleModel(gpu.parsed, w, tb.tensor_table)
    x = syn.seeded_series(b, t, seed=31)
    x[1, :] = np.nan
    x[2, 40:120] = np.nan
    got = gpu.forecast_chronos2(x, 100)
    want = ora.forecast_chronos2(x, 100)
    assert np.isfinite(got).all()
    assert rel_err(got, want, x) <= (TOL if compute == "f16" else TOL_BF16_RANGE)


def test_bf16_operands_run_and_stay_close(tiny):
    cfg, w, _, ora = tiny
    bf = tb.Model(cfg, w, compute="bf16")
    x = syn.seeded_series(6, 500, seed=9)
    assert rel_err(bf.forecast_chronos2(x, 100), ora.forecast_chronos2(x, 100), x) <= TOL_BF16_RANGE


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


@pytest.mark.parametrize("b,t", [(130, 200), (2100, 8192), (8200, 8192)])
def test_chunked_host_path_matches_device_path(tiny, b, t):
    # The host entry point splits a batch into 1, 2 or 4 chunks by its copy volume (under 64 MB, up
    # to 256 MB, more), with the copies on a second stream; every series must come out exactly as
    # from one device-resident forecast (pageable and pinned buffers).
    _, _, gpu, _ = tiny
    x = syn.seeded_series(b, t, seed=11)
    xd = torch.from_numpy(x).cuda()
    out = torch.empty((b, 48, 21), device="cuda")
    gpu.forecast_chronos2_device(xd.data_ptr(), b, t, 48, out.data_ptr(), torch.cuda.current_stream().cuda_stream)
    want = out.cpu().numpy()
    assert np.array_equal(gpu.forecast_chronos2(x, 48), want)
    xp = torch.from_numpy(x).pin_memory().numpy()
    op = torch.empty((b, 48, 21)).pin_memory().numpy()
    gpu.forecast_chronos2(xp, 48, out=op)
    assert np.array_equal(op, want)


def test_graph_replays_match_plain_runs(tiny):
    # The third call with the same shapes and buffers replays a captured CUDA graph; it must read
    # the new inputs and give exactly what a plain run gives (the host path and the device path).
    cfg, w, gpu, _ = tiny
    xs = [syn.seeded_series(5, 333, seed=50 + i) for i in range(4)]
    plain = [tb.Model(cfg, w).forecast_chronos2(x, 48) for x in xs]
    for x, want in zip(xs, plain):
        assert np.array_equal(gpu.forecast_chronos2(x, 48), want)
    xd = torch.empty((5, 333), device="cuda")
    out = torch.empty((5, 48, 21), device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    for x, want in zip(xs, plain):
        xd.copy_(torch.from_numpy(x))
        gpu.forecast_chronos2_device(xd.data_ptr(), 5, 333, 48, out.data_ptr(), s)
        assert np.array_equal(out.cpu().numpy(), want)


def test_argument_errors(tiny):
    _, _, gpu, _ = tiny
    with pytest.raises(tb.TsfmError, match="HORIZON_TOO_LONG"):
        gpu.forecast_chronos2(np.zeros((1, 32), np.float32), 8 * 16 + 1)
    with pytest.raises(tb.TsfmError, match="EMPTY_INPUT"):
        gpu.forecast_chronos2(np.zeros((0, 32), np.float32), 8)


@pytest.mark.parametrize("t,horizon", [(500, 100), (33, 17)])
def test_tiny_corrected_matches_oracle(tiny, t, horizon):
    # TSFM_COMPUTE_F16C on the edge inputs (all missing, constant, long gaps, t not a multiple of
    # the patch): the corrected products write and read the FP8 companions of every GEMM input.
    cfg, w, _, ora = tiny
    gpu = tb.Model(cfg, w, compute="f16c")
    x = edge_inputs(t)
    got = gpu.forecast_chronos2(x, horizon)
    want = ora.forecast_chronos2(x, horizon)
    assert np.isfinite(got).all()
    assert rel_err(got, want, x[:, -512:]) <= TOL


@pytest.mark.parametrize("b", [8, 130])
def test_fused_norm_corrected_matches_oracle(b):
    # The corrected products through the fused-norm GEMMs (the wo epilogue writes the next layer's
    # FP16 input and its FP8 companion), single-CTA (8 series) and CTA-pair (130 series) tiles.
    cfg = tiny_cfg(d_model=256, d_ff=512, num_heads=4, num_layers=3)
    w = syn.random_checkpoint(cfg, seed=21, norm_jitter=0.1)
    gpu = tb.Model(cfg, w, compute="f16c")
    ora = ob.OracleModel(gpu.parsed, w, tb.tensor_table)
    x = syn.seeded_series(b, 512, seed=31)
    x[1, :] = np.nan
    x[2, 40:120] = np.nan
    got = gpu.forecast_chronos2(x, 100)
    want = ora.forecast_chronos2(x, 100)
    assert np.isfinite(got).all()
    assert rel_err(got, want, x) <= TOL


def full_shape(compute, b, seed=100):
    cfg = syn.chronos2_config()
    w = syn.random_checkpoint(cfg, seed=20261201)
    gpu = tb.Model(cfg, w, compute=compute)
    ora = ob.OracleModel(gpu.parsed, w, tb.tensor_table)
    x = syn.seeded_series(b, 8192, seed=seed)
    got = gpu.forecast_chronos2(x, 1024)
    want = ora.forecast_chronos2(x, 1024)
    assert np.isfinite(got).all()
    return got, want, x


def test_full_shape_chronos2_matches_oracle():
    # BASELINE configs[2] shape (768-d, 12 layers, ctx 8192, H 1024) on 8 series in the corrected
    # mode (TSFM_COMPUTE_F16C), against the plain bound max |dq| <= 1e-2 * sigma on every quantile,
    # the tails included. (oracle/precision_study.py predicts 2.7e-3 for this scheme.)
    got, want, x = full_shape("f16c", 8)
    err = np.abs(got - want) / instance_scale(x)[:, None, None]
    print(f"full shape, corrected: max |dq|/sigma = {err.max():.3e}, p99 = {np.quantile(err, 0.99):.3e}")
    assert np.max(err) <= TOL
    assert np.quantile(err, 0.99) <= 1e-3


def test_full_shape_plain_f16_characterised():
    # Single-pass FP16 operands at the same shape: not a parity claim (the tails exceed 1e-2 *
    # sigma: q = sinh(v) * sigma + loc multiplies the error of v by cosh(v)); a sanity bound and
    # the bulk of the distribution only.
    got, want, x = full_shape("f16", 2)
    err = np.abs(got - want) / instance_scale(x)[:, None, None]
    print(f"full shape, plain FP16: max |dq|/sigma = {err.max():.3e}, p99 = {np.quantile(err, 0.99):.3e}")
    assert np.max(err) <= 5e-2
    assert np.quantile(err, 0.99) <= 5e-3
