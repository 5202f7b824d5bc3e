"""CSV output without a GPU: the oracle's restatement of writeCsv (src/main.zig:181-198) and of
Zig's "{d}" number rendering, pinned against (1) a digit-count search with glibc's correctly
rounded printf / strtof, (2) numpy's Dragon4 positional formatting (an independent shortest
round-trip implementation), (3) the header sample in the reference's README (README.md:33) and
the CLI usage text (src/main.zig:46). Plus the argument checks of the C ABI that need no device."""
import ctypes

import numpy as np
import pytest

import tsfm_b200 as tb
from oracle import binding as ob


def special_floats():
    """Powers of two over the whole exponent range with their neighbours, subnormals, the
    extremes, integers, and decimal-looking values."""
    out = []
    for e in range(-149, 128):
        p = np.float32(np.ldexp(1.0, e))
        out += [p, np.nextafter(p, np.float32(0)), np.nextafter(p, np.float32(np.inf))]
    out += list(np.arange(1, 70001, dtype=np.float32))
    out += list((np.arange(1, 20001, dtype=np.float64) / 1000.0).astype(np.float32))
    out += list((np.arange(1, 5001, dtype=np.float64) * 1e-7).astype(np.float32))
    out += [np.float32(x) for x in (1e-45, 1.4e-45, 1.17549435e-38, 3.4028235e38, 16777216, 16777217,
                                    33554436, 9.999999e-5, 0.3, 2.0 / 3.0, 1e10, 1e-10, 123456.789)]
    x = np.array(out, dtype=np.float32)
    x = x[np.isfinite(x) & (x > 0)]
    return x


def random_bits(n, seed):
    rng = np.random.default_rng(seed)
    bits = rng.integers(1, 0x7F800000, size=n, dtype=np.uint32)
    return bits.view(np.float32)


def test_ryu_digits_match_the_digit_search():
    x = np.concatenate([special_floats(), random_bits(1_000_000, 5)])
    d, e = ob.f32_digits(x)
    ds, es = ob.f32_digits(x, search=True)
    bad = np.flatnonzero((d != ds) | (e != es))
    assert bad.size == 0, [(float(x[i]), int(d[i]), int(e[i]), int(ds[i]), int(es[i])) for i in bad[:5]]


def numpy_text(v):
    return np.format_float_positional(np.float32(v), unique=True, trim="-")


def test_value_text_matches_numpy_dragon4():
    rng = np.random.default_rng(9)
    x = np.concatenate([special_floats()[::7], random_bits(60_000, 6), -random_bits(20_000, 7),
                        rng.standard_normal(60_000).astype(np.float32) * 10.0 ** rng.integers(-8, 9, 60_000)])
    x = x.astype(np.float32)
    bad = [(float(v), ob.f32_text(v), numpy_text(v)) for v in x if ob.f32_text(v) != numpy_text(v)]
    assert not bad, bad[:5]


def test_special_values_print_as_zig_does():
    assert ob.f32_text(np.float32(0.0)) == "0"
    assert ob.f32_text(np.float32(-0.0)) == "-0"
    assert ob.f32_text(np.float32(np.inf)) == "inf"
    assert ob.f32_text(np.float32(-np.inf)) == "-inf"
    assert ob.f32_text(np.float32(np.nan)) == "nan"
    assert ob.f32_text(-np.float32(np.nan)) == "nan"
    assert ob.f32_text(np.float32(100.0)) == "100"
    assert ob.f32_text(np.float32(1e-7)) == "0.0000001"
    assert ob.f32_text(np.float32(3.4028235e38)) == "340282350000000000000000000000000000000"
    assert ob.f32_text(np.float32(1.4e-45)) == "0." + "0" * 44 + "1"


def test_levels_match_float64_shortest_text():
    levels = [0.01, 0.05, 0.1, 0.2, 0.25, 0.3, 0.4, 0.5, 0.6, 0.7, 0.75, 0.8, 0.9, 0.95, 0.99, 0.025, 0.975,
              1e-20, 1e21, 0.1 + 0.2, 1.0 / 3.0]
    for lv in levels:
        assert ob.f64_text(lv) == np.format_float_positional(np.float64(lv), unique=True, trim="-"), lv


def test_header_matches_the_readme_sample():
    # README.md:33 shows "series,variate,step,q0.01,q0.05,...,q0.99" for the 21-level sets.
    levels = [0.01, 0.05] + [round(0.1 * i, 1) for i in range(1, 10)] + [0.95, 0.99]
    text = ob.csv_format(np.zeros((0, 1, 1, len(levels)), np.float32), levels).decode()
    assert text.startswith("series,variate,step,q0.01,q0.05,q0.1,")
    assert text.endswith(",q0.95,q0.99\n")
    assert text.count("\n") == 1


def python_write_csv(values, levels):
    """writeCsv restated in Python (src/main.zig:181-198) with numpy's shortest formatting."""
    s_, v_, h_, q_ = values.shape
    lines = ["series,variate,step" + "".join(",q" + np.format_float_positional(np.float64(l), unique=True,
                                                                                  trim="-") for l in levels)]
    for s in range(s_):
        for v in range(v_):
            for t in range(h_):
                lines.append(f"{s},{v},{t + 1}" + "".join("," + numpy_text(x) for x in values[s, v, t]))
    return ("\n".join(lines) + "\n").encode()


@pytest.mark.parametrize("shape", [(2, 3, 5, 4), (1, 1, 1, 1), (3, 1, 12, 9), (1, 2, 3, 40)])
def test_csv_layout_matches_a_python_restatement(shape):
    rng = np.random.default_rng(sum(shape))
    values = (rng.standard_normal(shape) * 100).astype(np.float32)
    levels = np.linspace(0.05, 0.95, shape[3])
    assert ob.csv_format(values, levels) == python_write_csv(values, levels)


def test_capi_csv_argument_checks_need_no_device():
    n = ctypes.c_size_t(0)
    lv = np.array([0.5])
    # A null length pointer and a null values pointer with work to do are argument errors.
    assert tb.lib.tsfm_csv_format(None, 1, 1, 1, lv.ctypes.data, 1, 0, None, 0, None) == 1
    assert tb.lib.tsfm_csv_format(None, 1, 1, 1, lv.ctypes.data, 1, 0, None, 0, ctypes.byref(n)) == 1
    assert tb.lib.tsfm_csv_write(None, 1, 1, 1, lv.ctypes.data, 1, 0, -1, ctypes.byref(n)) == 1
    # More levels than the kernels' line buffers hold.
    many = np.full(1001, 0.5)
    vals = np.zeros(1001, np.float32)
    assert tb.lib.tsfm_csv_format(vals.ctypes.data, 1, 1, 1, many.ctypes.data, 1001, 0, None, 0,
                                  ctypes.byref(n)) == 11
