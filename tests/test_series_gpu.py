"""GPU series reader (tsfm_parse_blocks / tsfm_parse_blocks_device) against the reference's own
parseBlocks test cases (core/series.zig:95-112, golden fixture) and against the oracle's
restatement (glibc strtod for the numbers) on generated files: comma and whitespace separated
lines, comments, runs of blank lines, CRLF endings, empty and unparsable tokens, numbers in
every notation (shortest, %.17g, fixed, exponent, hexadecimal, halfway cases, 100-digit
strings), the error cases in the reference's order, and a long-line file of 8 M values."""
import ctypes

import numpy as np
import pytest

from oracle import binding as ob

pytestmark = pytest.mark.gpu

ORACLE_CODES = {0: 0, 1: 18, 2: 19, 3: 9}


@pytest.fixture(scope="module")
def series():
    import torch
    assert torch.cuda.is_available()
    from tsfm_b200 import series
    return series


def oracle_parse(text):
    data = text.encode() if isinstance(text, str) else text
    cap = max(16, data.count(b",") + data.count(b" ") + data.count(b"\t") + data.count(b"\n") + 16)
    vals = np.zeros(cap, np.float64)
    b, r, l = ctypes.c_size_t(), ctypes.c_size_t(), ctypes.c_size_t()
    st = ob.lib.oracle_parse_blocks(data, vals.ctypes.data, vals.size, ctypes.byref(b), ctypes.byref(r),
                                    ctypes.byref(l))
    return ORACLE_CODES[st], vals[: b.value * r.value * l.value].reshape(b.value, r.value, l.value)


def gpu_parse(text):
    import tsfm_b200 as tb
    data = text.encode() if isinstance(text, str) else text
    buf = np.frombuffer(data, np.uint8) if data else np.zeros(1, np.uint8)
    b, r, l = ctypes.c_size_t(), ctypes.c_size_t(), ctypes.c_size_t()
    st = tb.lib.tsfm_parse_blocks(buf.ctypes.data, len(data), 0, None, 0, ctypes.byref(b), ctypes.byref(r),
                                  ctypes.byref(l))
    if st != 0:
        return st, None
    out = np.empty((b.value, r.value, l.value), np.float64)
    st = tb.lib.tsfm_parse_blocks(buf.ctypes.data, len(data), 0, out.ctypes.data, out.size, ctypes.byref(b),
                                  ctypes.byref(r), ctypes.byref(l))
    return st, out


def same(a, b):
    assert a.shape == b.shape
    na, nb = np.isnan(a), np.isnan(b)
    assert (na == nb).all()
    assert (a[~na].view(np.uint64) == b[~nb].view(np.uint64)).all()


def test_reference_cases(series, kat):
    k = kat["parse_blocks"]
    st, vals = gpu_parse(k["ok"]["text"])
    assert st == 0
    assert vals.shape == (k["ok"]["shape"]["blocks"], k["ok"]["shape"]["rows"], k["ok"]["shape"]["len"])
    flat = vals.ravel()
    for i, v in k["ok"]["values"].items():
        assert flat[int(i)] == v
    for i in k["ok"]["nan_indices"]:
        assert np.isnan(flat[i])
    codes = {"RaggedInput": 18, "RaggedBlocks": 19, "EmptyInput": 9}
    for case in k["errors"]:
        assert gpu_parse(case["text"])[0] == codes[case["error"]], case


def number_texts(rng, n):
    out = []
    for _ in range(n):
        d = rng.standard_normal() * 10.0 ** rng.integers(-30, 30)
        k = rng.integers(0, 9)
        if k == 0:
            out.append(repr(float(d)))
        elif k == 1:
            out.append("%.17g" % d)
        elif k == 2:
            out.append("%.*f" % (int(rng.integers(0, 12)), d / 10.0 ** rng.integers(0, 20)))
        elif k == 3:
            out.append("%.*e" % (int(rng.integers(0, 25)), d))
        elif k == 4:
            out.append(float(d).hex())
        elif k == 5:
            out.append(repr(float(np.float32(d))))
        elif k == 6:
            out.append(rng.choice(["nan", "NaN", "-inf", "Infinity", "", "abc", "1e", ".", "+.5", "5.", "-0",
                                   "1e400", "1e-400", "4.9e-324", "2.4703282292062328e-324", "0x1p-1074"]))
        elif k == 7:
            digits = "".join(str(x) for x in rng.integers(0, 10, int(rng.integers(20, 120))))
            out.append(digits[0] + "." + digits[1:] + "e" + str(int(rng.integers(-330, 310))))
        else:
            # exact halfway point between two adjacent doubles, printed with all its digits
            a = abs(d) if d != 0 else 1.0
            lo, hi = a, np.nextafter(a, np.inf)
            from decimal import Decimal, getcontext
            getcontext().prec = 800
            mid = (Decimal(lo) + Decimal(hi)) / 2
            out.append(format(mid, "f") if abs(mid.adjusted()) < 40 else format(mid, "e"))
    return out


def make_file(rng, blocks, rows, length, sep=",", crlf=False, extras=True):
    nums = number_texts(rng, blocks * rows * length)
    lines, k = [], 0
    if extras:
        lines.append("# generated series")
    for b in range(blocks):
        for r in range(rows):
            toks = nums[k:k + length]
            k += length
            if sep == ",":
                toks = [(" " * int(rng.integers(0, 2))) + t + (" " * int(rng.integers(0, 2))) for t in toks]
                line = ",".join(toks)
            else:
                toks = [t if t else "nan" for t in toks]
                line = "".join(t + rng.choice([" ", "  ", "\t", " \t "]) for t in toks).rstrip()
            if extras and rng.random() < 0.2:
                line = "  " + line + " \t"
            lines.append(line)
            if extras and rng.random() < 0.1:
                lines.append("# comment inside a block")
        lines += [""] * int(rng.integers(1, 3))
    eol = "\r\n" if crlf else "\n"
    return eol.join(lines) + (eol if rng.random() < 0.5 else "")


@pytest.mark.parametrize("seed,shape,sep,crlf", [(1, (3, 2, 7), ",", False), (2, (1, 5, 40), ",", True),
                                                 (3, (4, 1, 33), " ", False), (4, (2, 3, 1), " ", True),
                                                 (5, (6, 4, 65), ",", False), (6, (1, 1, 1), ",", False)])
def test_generated_files_match_oracle(series, seed, shape, sep, crlf):
    rng = np.random.default_rng(seed)
    text = make_file(rng, *shape, sep=sep, crlf=crlf)
    st, want = oracle_parse(text)
    got_st, got = gpu_parse(text)
    assert got_st == st == 0
    assert got.shape == shape
    same(got, want)


def test_numbers_bit_exact_against_strtod(series):
    rng = np.random.default_rng(11)
    toks = number_texts(rng, 60000)
    text = "\n".join(",".join(toks[i:i + 100]) for i in range(0, 60000, 100)) + "\n"
    st, want = oracle_parse(text)
    got_st, got = gpu_parse(text)
    assert st == got_st == 0
    same(got, want)


@pytest.mark.parametrize("text", ["1,2\n3\n", "1 2\n\n3 4\n5 6\n", "1,2\n3,4\n\n5,6\n", "# only\n\n", "", "\n\n",
                                  "1,2\n\n3,4\n5,6\n\n7\n", "1\n2\n\n3\n\n4\n5\n"])
def test_errors_in_the_reference_order(series, text):
    st, _ = oracle_parse(text)
    assert gpu_parse(text)[0] == st


def test_device_variant_f32(series):
    import torch
    rng = np.random.default_rng(21)
    text = make_file(rng, 2, 3, 50).encode()
    st, want = oracle_parse(text)
    dt = torch.from_numpy(np.frombuffer(text, np.uint8).copy()).cuda()
    shape = series.parse_blocks_device(dt.data_ptr(), len(text))
    assert shape == want.shape
    o64 = torch.empty(want.size, dtype=torch.float64, device="cuda")
    o32 = torch.empty(want.size, dtype=torch.float32, device="cuda")
    series.parse_blocks_device(dt.data_ptr(), len(text), o64.data_ptr(), o32.data_ptr(), want.size)
    torch.cuda.synchronize()
    same(o64.cpu().numpy().reshape(want.shape), want)
    with np.errstate(over="ignore"):
        f = want.astype(np.float32)
    g = o32.cpu().numpy().reshape(want.shape)
    assert ((np.isnan(f) & np.isnan(g)) | (f.view(np.uint32) == g.view(np.uint32))).all()


@pytest.mark.parametrize("offset", [1, 3, 7, 13])
def test_device_variant_unaligned_text(series, offset):
    # The text starts at an odd address: edge chunks are read byte by byte.
    import torch
    rng = np.random.default_rng(30 + offset)
    text = make_file(rng, 2, 2, 300, sep=" " if offset % 2 else ",").encode()
    st, want = oracle_parse(text)
    buf = torch.zeros(len(text) + 32, dtype=torch.uint8, device="cuda")
    buf[offset:offset + len(text)] = torch.from_numpy(np.frombuffer(text, np.uint8).copy()).cuda()
    ptr = buf.data_ptr() + offset
    assert series.parse_blocks_device(ptr, len(text)) == want.shape
    o64 = torch.empty(want.size, dtype=torch.float64, device="cuda")
    series.parse_blocks_device(ptr, len(text), o64.data_ptr(), None, want.size)
    torch.cuda.synchronize()
    same(o64.cpu().numpy().reshape(want.shape), want)


def test_long_lines_full_size(series):
    # 1024 series x 8192 values, one series per line (the CLI's input layout at context 8192).
    rng = np.random.default_rng(5)
    x = (rng.standard_normal((1024, 8192)) * 100).astype(np.float32)
    x[rng.random(x.shape) < 0.05] = np.nan
    lines = [",".join("" if np.isnan(v) else repr(float(v)) for v in row) for row in x]
    text = ("\n".join(lines) + "\n").encode()
    st, want = oracle_parse(text)
    got = series.parse_blocks(text)
    assert st == 0 and got.shape == (1, 1024, 8192)
    same(got, want)
