"""Bit-exact parity of the forecasters' indexing work on the GPU, through the C ABI, against the
oracle on the same inputs: patch geometry (left padding, truncation to the context), the validity
of every patch as a key, the REG slot, the instance-norm statistics and the patch features of
Chronos-2 (chronos2/forecaster.zig:94-143) and Chronos-Bolt (chronos_bolt/forecaster.zig:150-197),
and Timestral's window statistics, key validity, first observed patch per group and features
(timestral/model.zig:253-362).

Bit for bit: key validity, first observed patch, the mask columns, the time column, loc and scale
(f64 sums rounded once to f32, sqrt correctly rounded on both sides), and every feature value that
involves no asinh. Values through asinh (the device's asinhf against the host C library's) are
compared within 2 float32 ulps."""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

import tsfm_b200 as tb  # noqa: E402
from oracle import binding as ob  # noqa: E402
from tsfm_b200 import synthetic as syn  # noqa: E402

pytestmark = pytest.mark.gpu
CHRONOS2, BOLT = 1, 2


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


def ulps(a, b):
    """|a - b| in float32 ulps (sign-aware integer distance); NaN against NaN counts as equal, NaN
    against a number as far apart."""
    a = np.ascontiguousarray(a, np.float32)
    b = np.ascontiguousarray(b, np.float32)
    ia = bits(a).astype(np.int64)
    ib = bits(b).astype(np.int64)
    ia = np.where(ia >= 0x80000000, 0x80000000 - ia, ia)
    ib = np.where(ib >= 0x80000000, 0x80000000 - ib, ib)
    d = np.abs(ia - ib)
    na, nb = np.isnan(a), np.isnan(b)
    return np.where(na & nb, 0, np.where(na | nb, 1 << 31, d))


def edge_series(b, t, seed):
    x = syn.seeded_series(b, t, seed=seed)
    x[1, :] = np.nan                      # all missing: loc 0, scale 1, no valid patch
    x[2, :] = 3.25                        # constant: scale 0 -> 1e-5
    x[3, : t // 2] = np.nan               # long leading gap
    if t > 64:
        x[4, 16:48] = np.nan              # whole missing patches
    x[5, -1] = np.nan
    x[6, ::3] = np.nan                    # every third step missing
    return x


def gpu_patch(family, x, context, ps, tscale=1.0, arcsinh=1, use_reg=1):
    b, t_in = x.shape
    t = min(t_in, context)
    n_ctx = (t + (ps - t % ps) % ps) // ps
    seq = n_ctx + (1 if family == BOLT and use_reg else 0)
    width = (3 if family == CHRONOS2 else 2) * ps
    xd = torch.from_numpy(np.ascontiguousarray(x, np.float32)).cuda()
    loc = torch.empty(b, device="cuda")
    scale = torch.empty(b, device="cuda")
    feats = torch.full((b, n_ctx, width), float("nan"), device="cuda")
    kv = torch.full((b, seq), 7, dtype=torch.uint8, device="cuda")
    tb.check(tb.lib.tsfm_kernel_patch(family, xd.data_ptr(), b, t_in, context, ps, tscale, arcsinh, use_reg,
                                      loc.data_ptr(), scale.data_ptr(), feats.data_ptr(), kv.data_ptr(),
                                      torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    return loc.cpu().numpy(), scale.cpu().numpy(), feats.cpu().numpy(), kv.cpu().numpy()


def oracle_patch(family, x, context, ps, tscale=1.0, arcsinh=1, use_reg=1):
    x = np.ascontiguousarray(x, np.float32)
    b, t_in = x.shape
    t = min(t_in, context)
    n_ctx = (t + (ps - t % ps) % ps) // ps
    seq = n_ctx + (1 if family == BOLT and use_reg else 0)
    width = (3 if family == CHRONOS2 else 2) * ps
    loc, scale = np.empty(b, np.float32), np.empty(b, np.float32)
    feats = np.empty((b, n_ctx, width), np.float32)
    kv = np.empty((b, seq), np.uint8)
    if family == CHRONOS2:
        ob.check(ob.lib.oracle_chronos2_patch(x.ctypes.data, b, t_in, context, ps, tscale, arcsinh, loc.ctypes.data,
                                              scale.ctypes.data, feats.ctypes.data, kv.ctypes.data))
    else:
        ob.check(ob.lib.oracle_bolt_patch(x.ctypes.data, b, t_in, context, ps, use_reg, loc.ctypes.data,
                                          scale.ctypes.data, feats.ctypes.data, kv.ctypes.data))
    return loc, scale, feats, kv


@pytest.mark.parametrize("t_in,context", [(500, 512), (512, 512), (700, 512), (33, 512), (16, 512), (8192, 8192),
                                          (3000, 2048)])
def test_chronos2_patch_indexing_bit_exact(t_in, context):
    ps = 16
    x = edge_series(8, t_in, seed=t_in)
    got = gpu_patch(CHRONOS2, x, context, ps, tscale=float(context))
    want = oracle_patch(CHRONOS2, x, context, ps, tscale=float(context))
    for g, w in zip(got[:2], want[:2]):  # loc, scale
        assert np.array_equal(bits(g), bits(w))
    assert np.array_equal(got[3], want[3])  # key validity
    gf, wf = got[2], want[2]
    assert np.array_equal(bits(gf[..., :ps]), bits(wf[..., :ps]))            # time encoding
    assert np.array_equal(bits(gf[..., 2 * ps:]), bits(wf[..., 2 * ps:]))    # observed mask (padding = 0)
    assert ulps(gf[..., ps:2 * ps], wf[..., ps:2 * ps]).max() <= 2           # asinh((x - loc) / scale)


@pytest.mark.parametrize("t_in,context,use_reg", [(2048, 2048, 1), (2100, 2048, 1), (300, 2048, 0), (31, 512, 1),
                                                  (129, 512, 0)])
def test_bolt_patch_indexing_bit_exact(t_in, context, use_reg):
    ps = 16
    x = edge_series(8, t_in, seed=t_in + 1)
    got = gpu_patch(BOLT, x, context, ps, arcsinh=0, use_reg=use_reg)
    want = oracle_patch(BOLT, x, context, ps, arcsinh=0, use_reg=use_reg)
    for g, w in zip(got[:3], want[:3]):  # loc, scale, features (no asinh in Bolt)
        assert np.array_equal(bits(g), bits(w))
    assert np.array_equal(got[3], want[3])  # key validity incl. the REG slot


@pytest.mark.parametrize("cov,attend_missing", [(False, 1), (False, 0), (True, 1)])
def test_timestral_block_inputs_bit_exact(cov, attend_missing):
    # 5 groups of rows [target, target, past, known] (covariates) or [target, target] (none), t
    # context steps then (with covariates) hl known-future steps; leading gaps, whole missing
    # patches, an unobserved group, a binary known row, and NaN values marked observed (their
    # statistics follow Zig's NaN-skipping @max).
    rng = np.random.default_rng(11 + int(cov) + 2 * attend_missing)
    ps, groups, t, hl = 32, 5, 256, 64
    roles = np.array([0, 0, 1, 2] if cov else [0, 0], np.int8)
    vall = len(roles)
    rows = groups * vall
    x = syn.seeded_series(rows, t + hl, seed=77).astype(np.float32)
    obs = rng.random((rows, t + hl)) > 0.1
    obs[0, :100] = False                      # leading gap
    obs[1, 64:160] = False                    # whole missing patches
    obs[vall: 2 * vall, :] = False            # group 1 never observed
    if cov:
        x[3] = (rng.random(t + hl) > 0.5).astype(np.float32)  # a binary known row
        obs[3] = True
        x[7, :] = 2.5                          # a constant known row
    x = np.where(obs, x, 0.0).astype(np.float32)
    w = t + hl if cov else t
    full, full_obs = np.ascontiguousarray(x[:, :w]), np.ascontiguousarray(obs[:, :w].astype(np.uint8))
    n = w // ps
    want_loc, want_sc = np.empty((rows, n), np.float32), np.empty((rows, n), np.float32)
    want_f = np.empty((rows, n, 2 * ps), np.float32)
    want_kv, want_fo = np.empty((rows, n), np.uint8), np.empty(groups, np.int32)
    ob.check(ob.lib.oracle_timestral_block_inputs(full.ctypes.data, full_obs.ctypes.data, rows, w, ps, vall,
                                                  roles.ctypes.data, int(cov), 1e-6, 1, attend_missing,
                                                  want_loc.ctypes.data, want_sc.ctypes.data, want_f.ctypes.data,
                                                  want_kv.ctypes.data, want_fo.ctypes.data))
    dev = torch.device("cuda")
    ctx = torch.from_numpy(np.ascontiguousarray(x[:, :t])).to(dev)
    cobs = torch.from_numpy(np.ascontiguousarray(obs[:, :t].astype(np.uint8))).to(dev)
    kf = torch.from_numpy(np.ascontiguousarray(x[:, t:])).to(dev)
    kfm = torch.from_numpy(np.ascontiguousarray(obs[:, t:].astype(np.uint8))).to(dev)
    rd = torch.from_numpy(roles).to(dev)
    loc = torch.empty((rows, n), device=dev)
    sc = torch.empty((rows, n), device=dev)
    feats = torch.full((rows, n, 2 * ps), float("nan"), device=dev)
    kv = torch.full((rows, n), 7, dtype=torch.uint8, device=dev)
    fo = torch.empty(groups, dtype=torch.int32, device=dev)
    tb.check(tb.lib.tsfm_kernel_timestral_block_inputs(
        ctx.data_ptr(), cobs.data_ptr(), rows, t, kf.data_ptr() if cov else None, kfm.data_ptr() if cov else None,
        hl if cov else 0, ps, vall, rd.data_ptr(), int(cov), 1e-6, 1, attend_missing, loc.data_ptr(), sc.data_ptr(),
        feats.data_ptr(), kv.data_ptr(), fo.data_ptr(), torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    assert np.array_equal(bits(loc.cpu().numpy()), bits(want_loc))
    assert np.array_equal(bits(sc.cpu().numpy()), bits(want_sc))
    assert np.array_equal(kv.cpu().numpy(), want_kv)
    first = fo.cpu().numpy()
    assert np.array_equal(np.where(first >= n, 0, first), want_fo)  # no observed patch: >= n, read as 0
    gf = feats.cpu().numpy()
    assert np.array_equal(bits(gf[..., ps:]), bits(want_f[..., ps:]))  # missing flags
    assert ulps(gf[..., :ps], want_f[..., :ps]).max() <= 2             # asinh((x - loc) / scale)
