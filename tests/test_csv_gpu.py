"""GPU CSV output (tsfm_csv_format / tsfm_csv_write / tsfm_csv_format_device) against the oracle's
writeCsv restatement (src/main.zig:181-198): byte-identical text for forecasts of every shape the
layout has (one line, many levels, more than 32 levels per line, no series), for special values
(nan, +-inf, +-0, subnormals, the extremes) and for random bit patterns over the whole f32 range;
the buffer-size protocol; a file-descriptor sink; and a full-size run checked by digest."""
import ctypes
import hashlib
import os
import tempfile

import numpy as np
import pytest

from oracle import binding as ob

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def csvmod():
    import torch
    assert torch.cuda.is_available()
    from tsfm_b200 import csv
    return csv


def forecast_values(shape, seed, kind="normal"):
    rng = np.random.default_rng(seed)
    n = int(np.prod(shape))
    if kind == "bits":
        bits = rng.integers(0, 2 ** 32, size=n, dtype=np.uint64).astype(np.uint32)
        return bits.view(np.float32).reshape(shape)
    x = rng.standard_normal(n) * 10.0 ** rng.integers(-6, 7, n)
    return x.astype(np.float32).reshape(shape)


def levels_for(q):
    return np.round(np.linspace(0.01, 0.99, q), 4) if q > 1 else np.array([0.5] * q)


@pytest.mark.parametrize("shape", [(1, 1, 1, 1), (3, 2, 17, 9), (5, 1, 64, 21), (2, 3, 5, 40), (7, 1, 33, 32),
                                   (1, 1, 100, 65), (0, 1, 16, 9), (4, 4, 1, 3), (2, 1, 9, 200), (1, 1, 3, 1000),
                                   (1, 1, 40, 0)])
def test_format_matches_oracle(csvmod, shape):
    v = forecast_values(shape, seed=sum(shape))
    lv = levels_for(shape[3])
    assert csvmod.format_csv(v, lv) == ob.csv_format(v, lv)


def test_special_values(csvmod):
    specials = np.array([0.0, -0.0, np.inf, -np.inf, np.nan, -np.nan, 1e-45, -1e-45, 1.17549435e-38,
                         3.4028235e38, -3.4028235e38, 1.0, 100.0, 1e-7, 0.1, 16777216.0, 2.0 ** 100, 2.0 ** -126,
                         123456.789, -0.000123], dtype=np.float32)
    v = np.tile(specials, 3).reshape(3, 1, 4, 5)
    lv = [0.1, 0.25, 0.5, 0.75, 0.9]
    assert csvmod.format_csv(v, lv) == ob.csv_format(v, lv)


def test_random_bit_patterns_over_the_whole_range(csvmod):
    v = forecast_values((64, 1, 1024, 32), seed=3, kind="bits")
    lv = levels_for(32)
    assert csvmod.format_csv(v, lv) == ob.csv_format(v, lv)


def test_every_exponent_and_neighbours(csvmod):
    vals = []
    for e in range(-149, 128):
        p = np.float32(np.ldexp(1.0, e))
        vals += [p, np.nextafter(p, np.float32(0)), np.nextafter(p, np.float32(np.inf)), -p]
    v = np.array(vals, np.float32)
    v = v[: v.size // 4 * 4].reshape(-1, 1, 1, 4)
    lv = [0.1, 0.5, 0.9, 0.99]
    assert csvmod.format_csv(v, lv) == ob.csv_format(v, lv)


def test_buffer_too_small_reports_the_needed_size(csvmod):
    import tsfm_b200 as tb
    v = forecast_values((2, 1, 8, 3), seed=1)
    lv = np.array([0.1, 0.5, 0.9])
    want = ob.csv_format(v, lv)
    n = ctypes.c_size_t(0)
    st = tb.lib.tsfm_csv_format(v.ctypes.data, 2, 1, 8, lv.ctypes.data, 3, 0, None, 0, ctypes.byref(n))
    assert st == 16 and n.value == len(want)
    buf = np.zeros(len(want) - 1, np.uint8)
    st = tb.lib.tsfm_csv_format(v.ctypes.data, 2, 1, 8, lv.ctypes.data, 3, 0, buf.ctypes.data, buf.size,
                                ctypes.byref(n))
    assert st == 16 and n.value == len(want)
    buf = np.zeros(len(want), np.uint8)
    st = tb.lib.tsfm_csv_format(v.ctypes.data, 2, 1, 8, lv.ctypes.data, 3, 0, buf.ctypes.data, buf.size,
                                ctypes.byref(n))
    assert st == 0 and buf.tobytes() == want


def test_write_to_a_file_descriptor(csvmod):
    v = forecast_values((9, 2, 40, 21), seed=4)
    lv = levels_for(21)
    with tempfile.TemporaryFile() as f:
        n = csvmod.write_csv(v, lv, f.fileno())
        f.seek(0)
        got = f.read()
    want = ob.csv_format(v, lv)
    assert n == len(want) and got == want


def test_device_resident_variant(csvmod):
    import torch
    v = forecast_values((6, 1, 50, 9), seed=8)
    lv = levels_for(9)
    want = ob.csv_format(v, lv)
    dv = torch.from_numpy(v).cuda()
    out = torch.empty(len(want) + 64, dtype=torch.uint8, device="cuda")
    n = csvmod.format_csv_device(dv.data_ptr(), 6, 1, 50, lv, out.data_ptr(), out.numel())
    assert n == len(want)
    assert out[:n].cpu().numpy().tobytes() == want
    with pytest.raises(Exception, match="BUFFER_TOO_SMALL"):
        csvmod.format_csv_device(dv.data_ptr(), 6, 1, 50, lv, out.data_ptr(), len(want) - 1)


def test_chunked_full_size_digest(csvmod):
    # 2048 series x 1024 steps x 21 levels (44 M values, six 32 MiB chunks): the digest of the
    # GPU text equals the oracle's.
    v = forecast_values((2048, 1, 1024, 21), seed=12)
    lv = levels_for(21)
    got = csvmod.format_csv(v, lv)
    want = ob.csv_format(v, lv)
    assert len(got) == len(want)
    assert hashlib.sha256(got).digest() == hashlib.sha256(want).digest()


def test_csv_reads_back_bit_exactly_full_size(csvmod):
    # Property at the bench's full size (8192 series x 1024 steps x 21 levels): the GPU reader
    # (core/series.zig parseBlocks, f64 then f32 as the reference's toF32) turns the GPU writer's
    # text back into exactly the forecast's f32 values; the prefix columns are the line indices.
    import torch
    from tsfm_b200 import series
    rng = np.random.default_rng(99)
    v = (rng.standard_normal((8192, 1, 1024, 21)) * 10.0 ** rng.integers(-4, 5, (8192, 1, 1, 1))).astype(np.float32)
    lv = levels_for(21)
    dv = torch.from_numpy(v).cuda()
    import tsfm_b200 as tb
    need = ctypes.c_size_t(0)
    tb.lib.tsfm_csv_format_device(dv.data_ptr(), 8192, 1, 1024, lv.ctypes.data, 21, None, 0, ctypes.byref(need),
                                  None)
    text = torch.empty(need.value, dtype=torch.uint8, device="cuda")
    n = csvmod.format_csv_device(dv.data_ptr(), 8192, 1, 1024, lv, text.data_ptr(), text.numel())
    shape = series.parse_blocks_device(text.data_ptr(), n)
    assert shape == (1, 8192 * 1024 + 1, 24)
    back = torch.empty(shape[1] * shape[2], dtype=torch.float32, device="cuda")
    series.parse_blocks_device(text.data_ptr(), n, None, back.data_ptr(), back.numel())
    torch.cuda.synchronize()
    back = back.view(shape[1], shape[2])
    assert torch.isnan(back[0]).all()  # the header's tokens are not numbers
    assert torch.equal(back[1:, 3:].contiguous().view(torch.int32), dv.view(-1, 21).view(torch.int32))
    idx = torch.arange(8192 * 1024, device="cuda")
    assert torch.equal(back[1:, 0], (idx // 1024).float())
    assert torch.equal(back[1:, 2], (idx % 1024 + 1).float())
