"""The oracle against the reference's own known-answer tests (tests/golden/kat.json, extracted
from the reference's test blocks by tests/golden/make_golden.py) and against float64 restatements.
CPU only."""
import ctypes

import numpy as np
import pytest

from oracle import binding as ob


def test_relative_bucket_matches_reference_table(kat):
    # chronos_bolt/model.zig:383-391 (ids from transformers' T5 for rel = -140..140)
    k = kat["relative_bucket"]
    got = [ob.lib.oracle_relative_bucket(k["rel_start"] + i, k["num_buckets"], k["max_distance"])
           for i in range(len(k["expected"]))]
    assert got == k["expected"]


def test_relative_bucket_matches_transformers_wider_range():
    t5 = pytest.importorskip("transformers.models.t5.modeling_t5")
    import torch
    rel = torch.arange(-700, 701)
    want = t5.T5Attention._relative_position_bucket(rel, bidirectional=True, num_buckets=32, max_distance=128)
    got = [ob.lib.oracle_relative_bucket(int(r), 32, 128) for r in rel]
    assert got == want.tolist()


def test_quantile_linear_cases(kat):
    # chronos_bolt/forecaster.zig:222-228
    k = kat["quantile_linear"]
    v = np.array(k["sorted"], np.float32)
    for case in k["cases"]:
        got = ob.lib.oracle_quantile_linear(v.ctypes.data, v.size, case["level"])
        if case["tol"]:
            assert abs(got - case["expected"]) <= case["tol"]
        else:
            assert got == case["expected"]


def test_quantile_linear_matches_torch_quantile():
    import torch
    rng = np.random.default_rng(3)
    for n in (2, 5, 81):
        v = np.sort(rng.standard_normal(n).astype(np.float32))
        for level in (0.0, 0.01, 0.1, 0.375, 0.5, 0.9, 0.99, 1.0):
            got = ob.lib.oracle_quantile_linear(v.ctypes.data, n, level)
            want = torch.quantile(torch.from_numpy(v), level).item()
            assert abs(got - want) <= 1e-6 * max(1.0, abs(want))


def parse(text):
    vals = np.zeros(4096, np.float64)
    b, r, l = ctypes.c_size_t(), ctypes.c_size_t(), ctypes.c_size_t()
    st = ob.lib.oracle_parse_blocks(text.encode(), vals.ctypes.data, vals.size, ctypes.byref(b), ctypes.byref(r),
                                    ctypes.byref(l))
    return st, vals[: b.value * r.value * l.value], (b.value, r.value, l.value)


def test_parse_blocks_reference_cases(kat):
    # core/series.zig:95-112
    k = kat["parse_blocks"]
    st, vals, (b, r, l) = parse(k["ok"]["text"])
    assert st == 0
    assert (b, r, l) == (k["ok"]["shape"]["blocks"], k["ok"]["shape"]["rows"], k["ok"]["shape"]["len"])
    for i, v in k["ok"]["values"].items():
        assert vals[int(i)] == v
    for i in k["ok"]["nan_indices"]:
        assert np.isnan(vals[i])
    codes = {"RaggedInput": 1, "RaggedBlocks": 2, "EmptyInput": 3}
    for case in k["errors"]:
        assert parse(case["text"])[0] == codes[case["error"]], case


def test_mask_pick_table(kat):
    # core/attn.zig:191-197
    order = kat["mask_order"]
    for case in kat["mask_pick"]["cases"]:
        got = ob.lib.oracle_mask_pick(case["causal"], case["all_keys_valid"], case["additive"])
        assert order[got] == case["variant"]


def allowed(mask, kv, i, j):
    return {"full": True, "keys_additive": bool(kv[j]), "causal": j <= i,
            "causal_keys": j == i or (bool(kv[j]) and j <= i), "full_keys": j == i or bool(kv[j])}[mask]


def test_every_mask_matches_float64_reference(kat):
    # core/attn.zig:156-189: n = 11, hd = 8, fused-qkv-like stride 3*hd + 2, key i % 3 != 1 valid,
    # scale 0.35, with and without a bias, tolerance 1e-4.
    n, hd = 11, 8
    ld = 3 * hd + 2
    rng = np.random.default_rng(0x7A11)
    qkv = (rng.random(n * ld, dtype=np.float32) * 2 - 1).astype(np.float32)
    kv = np.array([i % 3 != 1 for i in range(n)], np.uint8)
    bias = (rng.random(n * n, dtype=np.float32) * 4 - 2).astype(np.float32)
    q, k, v = qkv[0:], qkv[hd:], qkv[2 * hd:]
    for mi, mask in enumerate(kat["mask_order"]):
        for b in (None, bias):
            got = np.zeros(n * hd, np.float32)
            st = ob.lib.oracle_self_attend(mi, q.ctypes.data, k.ctypes.data, v.ctypes.data, got.ctypes.data,
                                           ld, ld, ld, hd, n, hd, 0.35, kv.ctypes.data,
                                           None if b is None else b.ctypes.data)
            assert st == 0
            want = np.zeros((n, hd))
            for i in range(n):
                s = np.array([np.dot(qkv[i * ld:i * ld + hd].astype(np.float64),
                                     qkv[j * ld + hd:j * ld + 2 * hd].astype(np.float64)) * 0.35
                              + (0.0 if b is None else float(b[i * n + j])) for j in range(n)])
                ok = np.array([allowed(mask, kv, i, j) for j in range(n)])
                e = np.where(ok, np.exp(s - s[ok].max()), 0.0)
                p = e / e.sum()
                for j in range(n):
                    want[i] += p[j] * qkv[j * ld + 2 * hd:j * ld + 3 * hd]
            np.testing.assert_allclose(got.reshape(n, hd), want, atol=1e-4, err_msg=mask)


def test_linear_and_rmsnorm_match_float64():
    rng = np.random.default_rng(5)
    rows, out, inn = 37, 29, 23
    x = rng.standard_normal((rows, inn)).astype(np.float32)
    w = rng.standard_normal((out, inn)).astype(np.float32)
    b = rng.standard_normal(out).astype(np.float32)
    y = np.zeros((rows, out), np.float32)
    assert ob.lib.oracle_linear(x.ctypes.data, w.ctypes.data, b.ctypes.data, y.ctypes.data, rows, out, inn) == 0
    np.testing.assert_allclose(y, x.astype(np.float64) @ w.T.astype(np.float64) + b, atol=1e-4)
    scale = (1 + 0.1 * rng.standard_normal(inn)).astype(np.float32)
    o = np.zeros_like(x)
    assert ob.lib.oracle_rmsnorm(x.ctypes.data, scale.ctypes.data, o.ctypes.data, rows, inn, 1e-6) == 0
    xd = x.astype(np.float64)
    want = xd / np.sqrt((xd ** 2).mean(1, keepdims=True) + 1e-6) * scale
    np.testing.assert_allclose(o, want, rtol=1e-5, atol=1e-6)


def test_oracle_threads_do_not_change_results():
    # The reference guarantees --threads 1 and the default are bit-identical (README.md:282).
    rng = np.random.default_rng(9)
    x = rng.standard_normal((300, 200)).astype(np.float32)
    w = rng.standard_normal((150, 200)).astype(np.float32)
    ys = []
    orig = ob.get_threads()
    for nt in (1, 4):
        ob.set_threads(nt)
        y = np.zeros((300, 150), np.float32)
        ob.lib.oracle_linear(x.ctypes.data, w.ctypes.data, None, y.ctypes.data, 300, 150, 200)
        ys.append(y)
    ob.set_threads(orig)
    assert np.array_equal(ys[0], ys[1])


def test_e4m3_encoder_known_values():
    # The test-side E4M3 encoder used for the FP8 companions: exact values, subnormals, rounding
    # to nearest even at a tie, saturation.
    from helpers import e4m3_bits
    vals = np.array([0.0, 2.0 ** -9, 2.0 ** -6, 1.0, 1.125, 1.0625, 1.1875, 448.0, 500.0, -1.5, 2.0 ** -10,
                     3 * 2.0 ** -10, 240.0, 0.0146484375], np.float32)
    want = [0x00, 0x01, 0x08, 0x38, 0x39, 0x38, 0x3A, 0x7E, 0x7E, 0xBC, 0x00, 0x02, 0x77, 0x08]
    assert e4m3_bits(vals).tolist() == want
