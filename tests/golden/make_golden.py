"""Extract the reference's own known-answer vectors into tests/golden/kat.json.

Run in a checkout that has the reference tree beside the repository (../reference), or set
$TSFM_REFERENCE to its path; the tests read only the JSON this writes, so the reference is not needed at
test time. Every vector is read from the reference's test blocks, not retyped:

  - chronos_bolt/model.zig    test "relativeBucket matches transformers for -140..140"
      (the `expected` bucket ids for rel = -140..140, num_buckets 32, max_distance 128)
  - chronos_bolt/forecaster.zig test "quantileLinear interpolates like torch.quantile"
      (the sample array and each (level, expected) pair)
  - core/series.zig           tests "parseBlocks reads ..." and "parseBlocks rejects ..."
      (the input texts, the expected shape / values and the expected error names)
  - core/attn.zig             test "Mask.pick maps causality and key validity ..."
      (each (causal, all_keys_valid, additive) -> variant row)
"""
import json
import os
import re
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
REF = os.environ.get("TSFM_REFERENCE", os.path.join(os.path.dirname(ROOT), "reference"))


def read(rel):
    with open(os.path.join(REF, rel)) as f:
        return f.read()


def test_block(src, name):
    start = src.index('test "' + name)
    depth, i = 0, src.index("{", start)
    for j in range(i, len(src)):
        if src[j] == "{":
            depth += 1
        elif src[j] == "}":
            depth -= 1
            if depth == 0:
                return src[start : j + 1]
    raise ValueError(name)


def zig_string(lit):
    return bytes(lit, "utf-8").decode("unicode_escape")


def main():
    out = {}

    src = read("src/chronos_bolt/model.zig")
    blk = test_block(src, "relativeBucket matches transformers")
    arr = re.search(r"const expected = \[_\]u8\{([^}]*)\}", blk).group(1)
    rng = re.search(r"@intCast\(i\)\) - (\d+)", blk).group(1)
    call = re.search(r"relativeBucket\(rel, (\d+), (\d+)\)", blk)
    out["relative_bucket"] = {
        "rel_start": -int(rng),
        "num_buckets": int(call.group(1)),
        "max_distance": int(call.group(2)),
        "expected": [int(x) for x in arr.replace("\n", " ").split(",") if x.strip()],
        "source": "src/chronos_bolt/model.zig:383-391",
    }

    src = read("src/chronos_bolt/forecaster.zig")
    blk = test_block(src, "quantileLinear interpolates like torch.quantile")
    arr = re.search(r"const v = \[_\]f32\{([^}]*)\}", blk).group(1)
    cases = []
    for m in re.finditer(r"expect(?:Equal|ApproxEqAbs)\(@as\(f32, ([0-9.]+)\), quantileLinear\(&v, ([0-9.]+)\)(?:, ([0-9.e-]+))?\)", blk):
        cases.append({"level": float(m.group(2)), "expected": float(m.group(1)), "tol": float(m.group(3) or 0.0)})
    out["quantile_linear"] = {
        "sorted": [float(x) for x in arr.split(",")],
        "cases": cases,
        "source": "src/chronos_bolt/forecaster.zig:222-228",
    }

    src = read("src/core/series.zig")
    blk = test_block(src, "parseBlocks reads blank-line-separated blocks")
    text = zig_string(re.search(r'parseBlocks\(a, "((?:[^"\\]|\\.)*)"\)', blk).group(1))
    shape = {k: int(v) for v, k in re.findall(r"expectEqual\(@as\(usize, (\d+)\), b\.(\w+)\)", blk)}
    values = {int(i): float(v) for v, i in re.findall(r"expectEqual\(@as\(f64, ([0-9.]+)\), b\.data\[(\d+)\]\)", blk)}
    nans = [int(i) for i in re.findall(r"isNan\(b\.data\[(\d+)\]\)", blk)]
    errors = []
    blk2 = test_block(src, "parseBlocks rejects ragged and empty input")
    for err, lit in re.findall(r'expectError\(error\.(\w+), parseBlocks\(a, "((?:[^"\\]|\\.)*)"\)\)', blk2):
        errors.append({"text": zig_string(lit), "error": err})
    out["parse_blocks"] = {
        "ok": {"text": text, "shape": shape, "values": values, "nan_indices": nans},
        "errors": errors,
        "source": "src/core/series.zig:95-112",
    }

    src = read("src/core/attn.zig")
    blk = test_block(src, "Mask.pick maps causality")
    rows = []
    for variant, a, b, c in re.findall(r"expectEqual\(Mask\.(\w+), Mask\.pick\((\w+), (\w+), (\w+)\)\)", blk):
        rows.append({"causal": a == "true", "all_keys_valid": b == "true", "additive": c == "true", "variant": variant})
    out["mask_pick"] = {"cases": rows, "source": "src/core/attn.zig:191-197"}
    enum = re.search(r"pub const Mask = enum \{(.*?)pub fn pick", src, re.S).group(1)
    out["mask_order"] = re.findall(r"^\s*(\w+),", enum, re.M)

    dst = os.path.join(os.path.dirname(os.path.abspath(__file__)), "kat.json")
    with open(dst, "w") as f:
        json.dump(out, f, indent=1, sort_keys=True)
    print("wrote", dst, {k: (len(v["expected"]) if k == "relative_bucket" else "") for k, v in out.items() if isinstance(v, dict)})


if __name__ == "__main__":
    sys.exit(main())
