"""Failure detection without a GPU fault (the reference has no device code, so these cover this
backend's own failure paths).

- A bounded device wait that runs out: the warp-specialised kernels wait on mbarriers with a wall-
  clock limit; here the same wait runs on a barrier that nothing arrives on with a 2 ms limit. The
  kernel returns, the host reports TSFM_ERR_DEVICE_TIMEOUT, and the context stays usable (a
  forecast afterwards matches one made before).
- One replica's worker failing while the others join: with TSFM_FAIL_REPLICA=1 the second
  replica's forecast worker fails on the host before touching its device; the call returns the
  error, the first worker's thread is joined, and the model forecasts normally afterwards."""
import os

import numpy as np
import pytest

torch = pytest.importorskip("torch")

import tsfm_b200 as tb  # noqa: E402
from tsfm_b200 import synthetic as syn  # noqa: E402

pytestmark = pytest.mark.gpu


def tiny_c2():
    cfg = syn.chronos2_config(d_model=128, d_ff=256, num_heads=2, num_layers=2, context_length=512,
                              max_output_patches=8)
    return cfg, syn.random_checkpoint(cfg, seed=3)


def test_bounded_wait_expires_and_the_context_survives():
    cfg, w = tiny_c2()
    m = tb.Model(cfg, w)
    x = syn.seeded_series(4, 300, seed=1)
    before = m.forecast_chronos2(x, 48)
    st = tb.lib.tsfm_test_bounded_wait(2_000_000, torch.cuda.current_stream().cuda_stream)
    assert tb.STATUS_NAMES[st] == "DEVICE_TIMEOUT"
    assert "gave up" in tb.last_error()
    assert tb.lib.tsfm_test_bounded_wait(500, None) != 0  # limits outside [1 us, 2 s] are refused
    after = m.forecast_chronos2(x, 48)
    assert np.array_equal(before, after)


@pytest.mark.parametrize("family", ["chronos2", "timestral"])
def test_one_replica_worker_fails_others_join(family, monkeypatch):
    if family == "chronos2":
        cfg, w = tiny_c2()
        two = tb.Model(cfg, w, devices=(0, 0))
        x = syn.seeded_series(6, 300, seed=2)
        run = lambda: two.forecast_chronos2(x, 48)  # noqa: E731
    else:
        cfg = syn.timestral_config(d_model=128, num_heads=2, mlp_hidden_dim=256, num_layers=2, patch=16,
                                   context_length=512, block_size=8)
        w = syn.random_checkpoint(cfg, seed=5)
        two = tb.Model(cfg, w, devices=(0, 0))
        x = syn.seeded_series(6, 300, seed=4).reshape(6, 1, 300)
        o = np.isfinite(x)
        run = lambda: two.forecast_timestral(np.where(o, x, 0).astype(np.float32), 32,  # noqa: E731
                                             observed=o.astype(np.uint8))
    want = run()
    monkeypatch.setenv("TSFM_FAIL_REPLICA", "1")
    with pytest.raises(tb.TsfmError) as e:
        run()
    assert e.value.name == "INVALID_ARGUMENT" and "injected failure" in str(e.value)
    monkeypatch.delenv("TSFM_FAIL_REPLICA")
    assert np.array_equal(run(), want)
