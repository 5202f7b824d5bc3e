"""ORACLE precision study — test infrastructure only; nothing in the product imports it.

Runs the CPU restatement of the Chronos-2 forward at BASELINE's configs[2] shape (768-d, 12
layers, 12 heads, d_ff 3072, context 8192, horizon 1024, 21 quantiles; random-init N(0, 0.02)
weights, seed 20261201) on seeded series, once with the reference's FP32 arithmetic and once per
operand-rounding run (oracle/oracle_emul.cpp), and prints per run the forecast error
max |dq| / sigma (sigma = the population std of the observed context, the instance-norm scale)
and its 99th percentile.

Each scheme rounds the operands of the encoder's products (and q, k, v and the attention
probabilities) the way a device product with those operands would; the FP32-accurate quantile
head and the TF32 patch-feature products are modelled as on the device. The study shows which
operand precision meets the 1e-2 * sigma bound before any kernel is written for it.

    python oracle/precision_study.py --series 8 --runs "1;2;6"

A run is a scheme number, optionally followed by per-class overrides: "6:2=2,6=2" applies scheme
6 to every 16-bit product except the attention output (class 2) and the MLP's wo (class 6),
which take scheme 2 (classes: 1 q/k/v, 2 attention output, 3 group v, 4 group o, 5 MLP wi,
6 MLP wo, 7 patch-embedding output). A trailing "t" ("2t") also rounds the TF32-operand
products of the patch features to TF32, as a single-pass TF32 product on the device does.
"""
import argparse
import os
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "tsfm-zig_b200"))

from oracle import binding as ob  # noqa: E402
from tsfm_spec import config as spec_config  # noqa: E402
from tsfm_spec import synthetic as syn  # noqa: E402
from tsfm_spec.table import tensor_table  # noqa: E402

SCHEMES = {
    1: "FP16 operands",
    2: "FP16 + FP8 corrections (x_hi w_lo + x_lo w_hi in e4m3)",
    3: "FP16, three products (x_hi w_hi + x_lo w_hi + x_hi w_lo)",
    4: "FP16, weight split only (x_hi w_hi + x_hi w_lo)",
    5: "BF16 operands",
    6: "FP16 + FP8 weight correction only",
    7: "FP16 + FP8 input correction only",
}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--series", type=int, default=4)
    ap.add_argument("--seed", type=int, default=100)
    ap.add_argument("--runs", default="1;2;3;4;6;7")
    ap.add_argument("--context", type=int, default=8192)
    ap.add_argument("--horizon", type=int, default=1024)
    a = ap.parse_args()
    cfg = syn.chronos2_config(context_length=a.context)
    w = syn.random_checkpoint(cfg, seed=20261201)
    model = ob.OracleModel(spec_config.parse(cfg), w, tensor_table)
    x = syn.seeded_series(a.series, a.context, seed=a.seed)
    sig = np.array([np.nanstd(r) for r in x])[:, None, None]
    t0 = time.time()
    ob.check(ob.lib.oracle_set_operand_emulation(0))
    ref = model.forecast_chronos2(x, a.horizon)
    print(f"FP32 reference: {a.series} series in {time.time() - t0:.1f} s", flush=True)
    for run in [r.strip() for r in a.runs.split(";") if r.strip()]:
        base, _, over = run.partition(":")
        tf32 = base.endswith("t")
        sc = int(base.rstrip("t"))
        ob.check(ob.lib.oracle_set_operand_emulation(sc))
        ob.check(ob.lib.oracle_set_operand_emulation_tf32(int(tf32)))
        for item in [o for o in over.split(",") if o]:
            cls, _, sch = item.partition("=")
            ob.check(ob.lib.oracle_set_operand_emulation_class(int(cls), int(sch)))
        t0 = time.time()
        got = model.forecast_chronos2(x, a.horizon)
        ob.check(ob.lib.oracle_set_operand_emulation(0))
        err = np.abs(got - ref) / sig
        per = err.reshape(a.series, -1).max(axis=1)
        label = SCHEMES[sc] + ("; TF32 patch products" if tf32 else "") + (f"; overrides {over}" if over else "")
        print(f"run {run} ({label}): max |dq|/sigma = {err.max():.3e}, p99 = "
              f"{np.quantile(err, 0.99):.3e}, per series max = "
              f"[{', '.join(f'{v:.2e}' for v in per)}] ({time.time() - t0:.1f} s)", flush=True)


if __name__ == "__main__":
    main()
