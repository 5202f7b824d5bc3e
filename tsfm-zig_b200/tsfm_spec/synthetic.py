"""Seeded synthetic checkpoints and series (no hub access, no datasets).

Checkpoints: every matrix and bias ~ N(0, 0.02); norm scales = 1 (or 1 + N(0, norm_jitter) when
asked, which makes the tests sensitive to a dropped scale); `shared`, `forecast_query` and the
relative-position table ~ N(0, 0.02). Tensor names and shapes are those the reference's
`Model.load` functions read (chronos2/model.zig:77-125, chronos_bolt/model.zig:101-172,
timestral/model.zig:136-200).

Series i: rng = default_rng(seed + i); sigma ~ LogNormal(0, 1); period ~ U(7, 168);
phase ~ U(0, 2 pi); x_t = sigma sin(2 pi t / period + phase) + random walk of N(0, 0.05 sigma)
steps + N(0, 0.1 sigma) noise; a fraction `nan_frac` of values set to NaN.
"""
import json
import os
import struct

import numpy as np

# Chronos-2's 21 levels: 0.01, 0.05, 0.10, 0.15, ..., 0.90, 0.95, 0.99.
CHRONOS2_QUANTILES = [0.01] + [round(0.05 * i, 2) for i in range(1, 20)] + [0.99]
NINE_QUANTILES = [0.1, 0.2, 0.3, 0.4, 0.5, 0.6, 0.7, 0.8, 0.9]


def chronos2_config(d_model=768, d_ff=3072, num_heads=12, num_layers=12, context_length=8192,
                    patch=16, max_output_patches=64, quantiles=None, time_encoding_scale=None):
    q = list(quantiles or CHRONOS2_QUANTILES)
    return {
        "architectures": ["Chronos2Model"],
        "d_model": d_model, "d_ff": d_ff, "num_heads": num_heads, "d_kv": d_model // num_heads,
        "num_layers": num_layers, "layer_norm_epsilon": 1e-6, "rope_theta": 10000.0,
        "dense_act_fn": "relu",
        "chronos_config": {
            "context_length": context_length, "input_patch_size": patch, "input_patch_stride": patch,
            "output_patch_size": patch, "max_output_patches": max_output_patches, "quantiles": q,
            "time_encoding_scale": float(time_encoding_scale or context_length),
            "use_arcsinh": True, "use_reg_token": True,
        },
    }


def bolt_config(d_model=512, d_ff=2048, num_heads=8, num_layers=6, num_decoder_layers=1,
                context_length=2048, patch=16, prediction_length=64, quantiles=None, use_reg_token=True):
    return {
        "architectures": ["ChronosBoltModelForForecasting"],
        "d_model": d_model, "d_ff": d_ff, "num_heads": num_heads, "d_kv": d_model // num_heads,
        "num_layers": num_layers, "num_decoder_layers": num_decoder_layers, "layer_norm_epsilon": 1e-6,
        "dense_act_fn": "relu", "relative_attention_num_buckets": 32,
        "relative_attention_max_distance": 128, "decoder_start_token_id": 0, "reg_token_id": 1,
        "chronos_config": {
            "context_length": context_length, "input_patch_size": patch, "input_patch_stride": patch,
            "prediction_length": prediction_length, "quantiles": list(quantiles or NINE_QUANTILES),
            "use_reg_token": use_reg_token,
        },
    }


def timestral_config(d_model=1024, num_heads=16, mlp_hidden_dim=4096, num_layers=16, patch=32,
                     context_length=4096, block_size=32, schedule="time_variate", quantiles=None):
    sched = schedule if isinstance(schedule, list) else [schedule] * num_layers
    return {
        "patch_size": patch, "d_model": d_model, "num_heads": num_heads, "mlp_hidden_dim": mlp_hidden_dim,
        "block_schedule": sched, "quantile_knots": list(quantiles or NINE_QUANTILES),
        "block_size": block_size, "context_length": context_length, "rope_theta": 10000.0,
        "rope_partial_factor": 0.5, "norm_eps": 1e-6, "attn_bias": False, "mlp_bias": False,
        "time_attn_gate": "sdpa_sigmoid", "variate_attn_gate": "sdpa_sigmoid", "minimum_scale": 1e-6,
        "use_asinh": True, "stabilize_with_global": False, "covariate_enabled": True,
        "split_context_horizon_attn": True, "attend_missing_patches": True, "quantile_width_factor": 2.0,
    }


def tensor_shapes(cfg):
    """Name -> shape of every tensor the family's Model.load reads (norm scales flagged)."""
    shapes = {}
    norms = set()
    if "block_schedule" in cfg:
        d, ps, hid, q = cfg["d_model"], cfg["patch_size"], cfg["mlp_hidden_dim"], len(cfg["quantile_knots"])
        for n, (o, i) in {"hidden_layer": (4 * d, 2 * ps), "output_layer": (d, 4 * d), "residual_layer": (d, 2 * ps)}.items():
            shapes[f"representation.patch_proj.{n}.weight"] = (o, i)
            shapes[f"representation.patch_proj.{n}.bias"] = (o,)
        shapes["representation.forecast_query"] = (d,)
        for n, (o, i) in {"hidden_layer": (4 * d, d), "output_layer": (ps * q, 4 * d), "residual_layer": (ps * q, d)}.items():
            shapes[f"head.projection.{n}.weight"] = (o, i)
        shapes["transformer.out_norm.scale"] = (d,)
        norms.add("transformer.out_norm.scale")
        for li, kind in enumerate(cfg["block_schedule"]):
            n_attn = 1 if kind in ("time", "variate") else 2
            for ai in range(n_attn):
                is_time = (kind in ("time", "time_variate") and ai == 0) or (kind == "variate_time" and ai == 1)
                p = f"transformer.layers.{li}."
                shapes[p + f"attn_norms.{ai}.scale"] = (d,)
                norms.add(p + f"attn_norms.{ai}.scale")
                shapes[p + f"attns.{ai}.wQKV.weight"] = (3 * d, d)
                shapes[p + f"attns.{ai}.wO.weight"] = (d, d)
                gate = cfg.get("time_attn_gate" if is_time else "variate_attn_gate", "sdpa_sigmoid")
                if gate == "sdpa_sigmoid":
                    shapes[p + f"attns.{ai}._gate.weight"] = (d, d)
            shapes[f"transformer.layers.{li}.mlp_norm.scale"] = (d,)
            norms.add(f"transformer.layers.{li}.mlp_norm.scale")
            shapes[f"transformer.layers.{li}.mlp.w12.weight"] = (2 * hid, d)
            shapes[f"transformer.layers.{li}.mlp.w3.weight"] = (d, hid)
        return shapes, norms
    arch = cfg["architectures"][0]
    d, ff, ch = cfg["d_model"], cfg["d_ff"], cfg["chronos_config"]
    ps = ch["input_patch_size"]
    q = len(ch["quantiles"])
    if arch == "Chronos2Model":
        emb = {"hidden_layer": (ff, 3 * ps), "output_layer": (d, ff), "residual_layer": (d, 3 * ps)}
        head = {"hidden_layer": (ff, d), "output_layer": (q * ps, ff), "residual_layer": (q * ps, d)}
        for pre, blk in (("input_patch_embedding", emb), ("output_patch_embedding", head)):
            for n, (o, i) in blk.items():
                shapes[f"{pre}.{n}.weight"] = (o, i)
                shapes[f"{pre}.{n}.bias"] = (o,)
        shapes["encoder.final_layer_norm.weight"] = (d,)
        norms.add("encoder.final_layer_norm.weight")
        shapes["shared.weight"] = (2, d)
        for li in range(cfg["num_layers"]):
            for which in (0, 1):
                p = f"encoder.block.{li}.layer.{which}."
                shapes[p + "layer_norm.weight"] = (d,)
                norms.add(p + "layer_norm.weight")
                for m in "qkvo":
                    shapes[p + f"self_attention.{m}.weight"] = (d, d)
            p = f"encoder.block.{li}.layer.2."
            shapes[p + "layer_norm.weight"] = (d,)
            norms.add(p + "layer_norm.weight")
            shapes[p + "mlp.wi.weight"] = (ff, d)
            shapes[p + "mlp.wo.weight"] = (d, ff)
        return shapes, norms
    # Chronos-Bolt
    inner = cfg["num_heads"] * cfg["d_kv"]
    out_dim = q * ch["prediction_length"]
    emb = {"hidden_layer": (ff, 2 * ps), "output_layer": (d, ff), "residual_layer": (d, 2 * ps)}
    head = {"hidden_layer": (ff, d), "output_layer": (out_dim, ff), "residual_layer": (out_dim, d)}
    for pre, blk in (("input_patch_embedding", emb), ("output_patch_embedding", head)):
        for n, (o, i) in blk.items():
            shapes[f"{pre}.{n}.weight"] = (o, i)
            shapes[f"{pre}.{n}.bias"] = (o,)
    shapes["shared.weight"] = (2 if ch.get("use_reg_token", False) else 1, d)
    shapes["encoder.block.0.layer.0.SelfAttention.relative_attention_bias.weight"] = (
        cfg.get("relative_attention_num_buckets", 32), cfg["num_heads"])
    for n in ("encoder.final_layer_norm.weight", "decoder.final_layer_norm.weight"):
        shapes[n] = (d,)
        norms.add(n)
    for i in range(cfg["num_layers"]):
        p = f"encoder.block.{i}."
        for n in (p + "layer.0.layer_norm.weight", p + "layer.1.layer_norm.weight"):
            shapes[n] = (d,)
            norms.add(n)
        for m in "qkv":
            shapes[p + f"layer.0.SelfAttention.{m}.weight"] = (inner, d)
        shapes[p + "layer.0.SelfAttention.o.weight"] = (d, inner)
        shapes[p + "layer.1.DenseReluDense.wi.weight"] = (ff, d)
        shapes[p + "layer.1.DenseReluDense.wo.weight"] = (d, ff)
    for i in range(cfg["num_decoder_layers"]):
        p = f"decoder.block.{i}."
        for n in (p + "layer.0.layer_norm.weight", p + "layer.1.layer_norm.weight", p + "layer.2.layer_norm.weight"):
            shapes[n] = (d,)
            norms.add(n)
        shapes[p + "layer.0.SelfAttention.v.weight"] = (inner, d)
        shapes[p + "layer.0.SelfAttention.o.weight"] = (d, inner)
        for m in "qkv":
            shapes[p + f"layer.1.EncDecAttention.{m}.weight"] = (inner, d)
        shapes[p + "layer.1.EncDecAttention.o.weight"] = (d, inner)
        shapes[p + "layer.2.DenseReluDense.wi.weight"] = (ff, d)
        shapes[p + "layer.2.DenseReluDense.wo.weight"] = (d, ff)
    return shapes, norms


def random_checkpoint(cfg, seed=20261201, std=0.02, norm_jitter=0.0, dtype=np.float32):
    """Name -> array of a random-init checkpoint for `cfg` (generated in sorted-name order).
    dtype: np.float32, np.float16, or "bf16" (raw bfloat16 bits as uint16, round to nearest even),
    the safetensors storage types the reference loads (core/safetensors.zig:81-92)."""
    shapes, norms = tensor_shapes(cfg)
    rng = np.random.default_rng(seed)
    out = {}
    for name in sorted(shapes):
        shp = shapes[name]
        if name in norms:
            a = np.ones(shp, np.float32)
            if norm_jitter:
                a += rng.standard_normal(shp, dtype=np.float32) * np.float32(norm_jitter)
        else:
            a = rng.standard_normal(shp, dtype=np.float32) * np.float32(std)
        if isinstance(dtype, str) and dtype == "bf16":
            out[name] = to_bf16_bits(a)
        else:
            out[name] = a.astype(dtype) if dtype != np.float32 else a
    return out


def seeded_series(b, t, seed=7, nan_frac=0.05):
    """(b, t) float32 series per the generator described in the module docstring."""
    out = np.empty((b, t), np.float32)
    tt = np.arange(t, dtype=np.float64)
    for i in range(b):
        rng = np.random.default_rng(seed + i)
        sigma = rng.lognormal(0.0, 1.0)
        period = rng.uniform(7.0, 168.0)
        phase = rng.uniform(0.0, 2.0 * np.pi)
        x = sigma * np.sin(2.0 * np.pi * tt / period + phase)
        x += np.cumsum(rng.normal(0.0, 0.05 * sigma, t))
        x += rng.normal(0.0, 0.1 * sigma, t)
        if nan_frac > 0:
            x[rng.random(t) < nan_frac] = np.nan
        out[i] = x.astype(np.float32)
    return out


def ar1_covariates(b, c, t, seed=11, phi=0.9):
    """(b, c, t) AR(1) covariates with N(0, 1) innovations."""
    rng = np.random.default_rng(seed)
    out = np.empty((b, c, t), np.float32)
    e = rng.standard_normal((b, c, t))
    x = np.zeros((b, c))
    for i in range(t):
        x = phi * x + e[:, :, i]
        out[:, :, i] = x
    return out


def write_checkpoint(directory, cfg, tensors):
    """Write config.json and model.safetensors (F32/F16/BF16 as given) into `directory`."""
    os.makedirs(directory, exist_ok=True)
    with open(os.path.join(directory, "config.json"), "w") as f:
        json.dump(cfg, f)
    header, blobs, off = {}, [], 0
    for name in sorted(tensors):
        a = np.ascontiguousarray(tensors[name])
        if a.dtype == np.float32:
            dt = "F32"
        elif a.dtype == np.float16:
            dt = "F16"
        elif a.dtype == np.uint16:
            dt = "BF16"  # raw bfloat16 bits
        else:
            raise ValueError(a.dtype)
        raw = a.tobytes()
        header[name] = {"dtype": dt, "shape": list(a.shape), "data_offsets": [off, off + len(raw)]}
        blobs.append(raw)
        off += len(raw)
    hb = json.dumps(header).encode()
    hb += b" " * ((8 - len(hb) % 8) % 8)
    with open(os.path.join(directory, "model.safetensors"), "wb") as f:
        f.write(struct.pack("<Q", len(hb)))
        f.write(hb)
        for r in blobs:
            f.write(r)


def to_bf16_bits(a):
    """float32 array -> uint16 bfloat16 bits (round to nearest even)."""
    u = np.ascontiguousarray(a, np.float32).view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    return u.astype(np.uint16)
