// Chronos-2 on the device: the encoder-only patched transformer of chronos2/model.zig and the
// forecaster of chronos2/forecaster.zig, as one stream of kernels per chunk of series.
//
// Per layer (chronos2/model.zig:189-203):
//   rmsnorm(x) -> xn;  [q|k|v] = xn Wqkv^T with rotate-half RoPE fused in the epilogue;
//   flash attention (scale 1, T5 key mask);  x += o Wo^T (accumulate epilogue);
//   rmsnorm(x) -> xn;  v = xn Wv^T;  x += v Wo^T  (singleton-group attention, model.zig:265-269);
//   rmsnorm(x) -> xn;  h = relu(xn Wi^T);  x += h Wo^T.
// The residual stream x stays FP32 in HBM; GEMM operands are FP16 (or BF16) with FP32
// accumulation; in the corrected mode (TSFM_COMPUTE_F16C) every 16-bit GEMM input is written with
// its FP8 companion and every product adds the FP8 correction terms (kernels.h).
// The patch embedding writes straight into each series' sequence rows (row-remapped epilogue);
// the REG token and the future-patch embeddings, identical for every series, are computed once
// at load and broadcast. The head runs only on the future-patch rows.
#include <cmath>
#include <cstdlib>
#include <cstring>

#include "model.h"
#include "ops.h"

#include <algorithm>

namespace tsfm {


Status c2_validate(const tsfm_config &c) {
    // chronos2/config.zig:44-55
    if (c.num_heads <= 0 || c.d_model != c.num_heads * c.d_kv) return Status::fail(TSFM_ERR_INVALID_CONFIG, "InvalidConfig: d_model != num_heads * d_kv");
    if (c.d_ff <= 0 || c.num_layers <= 0) return Status::fail(TSFM_ERR_INVALID_CONFIG, "InvalidConfig: d_ff / num_layers");
    if (c.patch_size <= 0) return Status::fail(TSFM_ERR_INVALID_CONFIG, "InvalidConfig: patch size");
    if (c.context_length <= 0 || c.max_output_patches <= 0) return Status::fail(TSFM_ERR_INVALID_CONFIG, "InvalidConfig: context_length / max_output_patches");
    if (c.num_quantiles <= 0 || !c.quantiles) return Status::fail(TSFM_ERR_INVALID_CONFIG, "InvalidConfig: quantiles");
    if (!c.use_reg_token) return Status::fail(TSFM_ERR_INVALID_CONFIG, "UnsupportedConfig: use_reg_token = false");
    if (!(c.time_encoding_scale > 0) || !(c.layer_norm_epsilon > 0)) return Status::fail(TSFM_ERR_INVALID_CONFIG, "InvalidConfig: time_encoding_scale / eps");
    // Kernel constraints of this backend.
    if (c.d_kv != 64) return Status::fail(TSFM_ERR_UNSUPPORTED, "Chronos-2: head width must be 64");
    if (c.d_model % 64 || c.d_ff % 8) return Status::fail(TSFM_ERR_UNSUPPORTED, "Chronos-2: d_model % 64 and d_ff % 8 must be 0");
    if ((3 * c.patch_size) % 4 || (c.num_quantiles * c.patch_size) % 4)
        return Status::fail(TSFM_ERR_UNSUPPORTED, "Chronos-2: patch feature rows must be 16-byte multiples");
    return Status::ok();
}

Status c2_check_tensors(const tsfm_config &c, const TensorTable &t) {
    const int64_t d = c.d_model, ps = c.patch_size, hid = c.d_ff, q = c.num_quantiles;
    struct Blk {
        const char *prefix;
        int64_t in, out;
    };
    for (const Blk &b : {Blk{"input_patch_embedding", 3 * ps, d}, Blk{"output_patch_embedding", d, q * ps}}) {
        const std::string p = b.prefix;
        TSFM_TRY(t.check(p + ".hidden_layer.weight", hid * b.in));
        TSFM_TRY(t.check(p + ".hidden_layer.bias", hid));
        TSFM_TRY(t.check(p + ".output_layer.weight", b.out * hid));
        TSFM_TRY(t.check(p + ".output_layer.bias", b.out));
        TSFM_TRY(t.check(p + ".residual_layer.weight", b.out * b.in));
        TSFM_TRY(t.check(p + ".residual_layer.bias", b.out));
    }
    TSFM_TRY(t.check("encoder.final_layer_norm.weight", d));
    TSFM_TRY(t.check("shared.weight", 2 * d));
    for (int li = 0; li < c.num_layers; ++li) {
        for (int which = 0; which < 2; ++which) {
            const std::string p = strf("encoder.block.%d.layer.%d.", li, which);
            TSFM_TRY(t.check(p + "layer_norm.weight", d));
            for (const char *nm : {"q", "k", "v", "o"}) TSFM_TRY(t.check(p + "self_attention." + nm + ".weight", d * d));
        }
        TSFM_TRY(t.check(strf("encoder.block.%d.layer.2.layer_norm.weight", li), d));
        TSFM_TRY(t.check(strf("encoder.block.%d.layer.2.mlp.wi.weight", li), hid * d));
        TSFM_TRY(t.check(strf("encoder.block.%d.layer.2.mlp.wo.weight", li), d * hid));
    }
    return Status::ok();
}

Status c2_load(Replica &r, const tsfm_config &c, const TensorTable &t, int act, C2Dev &w) {
    const int64_t d = c.d_model, ps = c.patch_size, hid = c.d_ff, q = c.num_quantiles;
    // act: the 16-bit weights' upload type; E_F16C = FP16 weights with FP8 correction companions
    // (FP16 activations, each GEMM input written with its companion).
    w.corr = act == E_F16C;
    w.act = w.corr ? E_F16 : act;
    // The patch features enter a TF32 product (K = 3 * patch); every other product takes 16-bit
    // operands of type `act`.
    TSFM_TRY(load_resblock(r, t, "input_patch_embedding", 3 * ps, hid, d, true, E_F32, act, w.in_embed));
    {
        const std::string p = "output_patch_embedding";
        std::vector<float> m;
        TSFM_TRY(t.get(p + ".hidden_layer.weight", hid * d, m));
        TSFM_TRY(upload_lin3(r, m, hid, d, w.head_hidden));
        TSFM_TRY(t.get(p + ".hidden_layer.bias", hid, m));
        TSFM_TRY(upload_bias(r, m, w.head_hidden.hi));
        TSFM_TRY(t.get(p + ".output_layer.weight", q * ps * hid, m));
        TSFM_TRY(upload_lin3(r, m, q * ps, hid, w.head_output));
        TSFM_TRY(t.get(p + ".output_layer.bias", q * ps, m));
        TSFM_TRY(upload_bias(r, m, w.head_output.hi));
        TSFM_TRY(t.get(p + ".residual_layer.weight", q * ps * d, m));
        TSFM_TRY(upload_lin3(r, m, q * ps, d, w.head_residual));
        TSFM_TRY(t.get(p + ".residual_layer.bias", q * ps, m));
        TSFM_TRY(upload_bias(r, m, w.head_residual.hi));
    }
    std::vector<float> v;
    TSFM_TRY(t.get("encoder.final_layer_norm.weight", d, v));
    TSFM_TRY(upload_f32(r, v, &w.final_norm));
    TSFM_TRY(t.get("shared.weight", 2 * d, v));
    std::vector<float> reg(v.begin() + d, v.begin() + 2 * d);
    TSFM_TRY(upload_f32(r, reg, &w.reg));
    for (int li = 0; li < c.num_layers; ++li) {
        C2Dev::Layer L;
        for (int which = 0; which < 2; ++which) {
            const std::string p = strf("encoder.block.%d.layer.%d.", li, which);
            TSFM_TRY(t.get(p + "layer_norm.weight", d, v));
            TSFM_TRY(upload_f32(r, v, which == 0 ? &L.time_norm : &L.group_norm));
            const tsfm_tensor *tq, *tk, *tv, *to;
            TSFM_TRY(t.raw(p + "self_attention.q.weight", d * d, &tq));
            TSFM_TRY(t.raw(p + "self_attention.k.weight", d * d, &tk));
            TSFM_TRY(t.raw(p + "self_attention.v.weight", d * d, &tv));
            TSFM_TRY(t.raw(p + "self_attention.o.weight", d * d, &to));
            if (which == 0) {
                TSFM_TRY(upload_lin_raw(r, {tq, tk, tv}, nullptr, 3 * d, d, act, L.qkv));
                TSFM_TRY(upload_lin_raw(r, {to}, nullptr, d, d, act, L.o));
            } else {
                // Singleton groups: only v and o take part (chronos2/model.zig:265-269); q and k are
                // still required to exist, as the reference loads them. o(v(x)) = x (W_o W_v)^T:
                // one GEMM with the product formed in float64 and rounded once.
                TSFM_TRY(upload_fold_raw(r, to, tv, d, d, d, act, L.gvo));
            }
        }
        TSFM_TRY(t.get(strf("encoder.block.%d.layer.2.layer_norm.weight", li), d, v));
        TSFM_TRY(upload_f32(r, v, &L.mlp_norm));
        const tsfm_tensor *twi, *two;
        TSFM_TRY(t.raw(strf("encoder.block.%d.layer.2.mlp.wi.weight", li), hid * d, &twi));
        TSFM_TRY(t.raw(strf("encoder.block.%d.layer.2.mlp.wo.weight", li), d * hid, &two));
        TSFM_TRY(upload_lin_raw(r, {twi}, nullptr, hid, d, act, L.wi));
        TSFM_TRY(upload_lin_raw(r, {two}, nullptr, d, hid, act, L.wo));
        w.layers.push_back(L);
    }
    // RoPE tables for every position a sequence can have (chronos2/model.zig:107-113, 178-187).
    const int64_t hd = c.d_kv, half = hd / 2;
    const int64_t max_ctx_patches = (c.context_length + ps - 1) / ps;
    w.max_seq = max_ctx_patches + 1 + c.max_output_patches;
    std::vector<float> inv(half), cs(w.max_seq * half), sn(w.max_seq * half);
    const float base = (float)c.rope_theta;
    for (int64_t i = 0; i < half; ++i) inv[i] = 1.0f / std::pow(base, (float)(2 * i) / (float)hd);
    for (int64_t tok = 0; tok < w.max_seq; ++tok)
        for (int64_t i = 0; i < half; ++i) {
            const float ang = inv[i] * (float)tok;
            cs[tok * half + i] = std::cos(ang);
            sn[tok * half + i] = std::sin(ang);
        }
    TSFM_TRY(upload_f32(r, cs, &w.rope_cos));
    TSFM_TRY(upload_f32(r, sn, &w.rope_sin));

    // Future patches carry only their time encoding (chronos2/forecaster.zig:146-154), the same for
    // every series: embed them once for the longest horizon.
    const int64_t nf = c.max_output_patches;
    std::vector<float> ff(nf * 3 * ps, 0.0f);
    for (int64_t p = 0; p < nf; ++p)
        for (int64_t i = 0; i < ps; ++i) {
            const float tv = (float)(p * ps + i) / (float)c.time_encoding_scale;
            uint32_t u;
            std::memcpy(&u, &tv, 4);
            if ((u & 0x7f800000u) != 0x7f800000u) u = (u + 0x1000u) & ~0x1fffu;  // TF32 operand
            float tr;
            std::memcpy(&tr, &u, 4);
            ff[p * 3 * ps + i] = tr;
        }
    float *d_ff = nullptr;
    TSFM_TRY(upload_f32(r, ff, &d_ff));
    TSFM_TRY(upload_f32(r, std::vector<float>(nf * d, 0.0f), &w.fut_emb));
    DevBuf tmp, tmp8;
    TSFM_TRY(tmp.alloc(nf * hid * 2));  // 16-bit hidden activations
    LinearCall hx, ox;                   // their FP8 companion (corrected products)
    if (w.corr) {
        TSFM_TRY(tmp8.alloc(nf * hid * 2));
        hx.y8 = tmp8.p;
        ox.x8 = tmp8.p;
        hx.ldy8 = ox.ldx8 = 2 * hid;
    }
    cudaStream_t s = r.stream;
    TSFM_TRY(op_linear(r, s, w.in_embed.hidden, d_ff, nf, 3 * ps, tmp.p, hid, out_mode_for(w.act), 1, &hx));
    TSFM_TRY(op_linear(r, s, w.in_embed.residual, d_ff, nf, 3 * ps, w.fut_emb, d, OUT_F32, 0));
    TSFM_TRY(op_linear(r, s, w.in_embed.output, tmp.p, nf, hid, w.fut_emb, d, OUT_F32_ACC, 0, &ox));
    TSFM_CUDA(cudaStreamSynchronize(s), "Chronos-2 future embeddings");
    TSFM_TRY(check_device_error(r));
    return Status::ok();
}

static void c2_geometry(const tsfm_config &c, int64_t t_in, int64_t horizon, int64_t &t, int64_t &start, int64_t &pad,
                        int64_t &n_ctx, int64_t &n_out, int64_t &seq) {
    const int64_t ps = c.patch_size;
    t = std::min<int64_t>(t_in, c.context_length);
    start = t_in - t;
    pad = (ps - t % ps) % ps;
    n_ctx = (t + pad) / ps;
    n_out = (horizon + ps - 1) / ps;
    seq = n_ctx + 1 + n_out;
}

// The time-attention RMSNorm of encoder layers 1.. runs inside the GEMMs around it
// (LinearCall::norm_*) when d_model is a multiple of 256 and the operands are 16-bit;
// TSFM_FUSED_NORM=0 keeps the separate norm kernel.
static bool c2_fused_norm(const tsfm_config &c) {
    static const bool on = [] {
        const char *v = std::getenv("TSFM_FUSED_NORM");
        return !(v && v[0] == '0');
    }();
    return on && c.d_model % 256 == 0;
}

static size_t c2_workspace(const tsfm_config &c, bool corr, int64_t nb, int64_t t_in, int64_t horizon) {
    int64_t t, start, pad, n_ctx, n_out, seq;
    c2_geometry(c, t_in, horizon, t, start, pad, n_ctx, n_out, seq);
    const int64_t d = c.d_model, ff = c.d_ff, ps = c.patch_size, q = c.num_quantiles, rows = nb * seq;
    size_t b = 0;
    b += Arena::span(nb * 4) * 2;
    b += Arena::span(nb * n_ctx * 3 * ps * 4);
    b += Arena::span(nb * seq);
    b += Arena::span(rows * d * 4);
    b += Arena::span(rows * d * 2);
    b += Arena::span(rows * 3 * d * 2);
    b += Arena::span(rows * d * 2);
    b += Arena::span(rows * ff * 2);
    b += Arena::span(nb * n_out * q * ps * 4);
    b += Arena::span(nb * n_out * d * 4) * 2;   // head input, hi / lo
    b += Arena::span(nb * n_out * ff * 4) * 2;  // head hidden, hi / lo
    if (c2_fused_norm(c)) {
        b += Arena::span(rows * 4);              // row factors
        b += Arena::span(rows * (d / 256) * 4);  // row sums of squares per column tile
    }
    if (corr) {  // FP8 companions of xn, ao and h
        b += Arena::span(rows * 2 * d) * 2;
        b += Arena::span(rows * 2 * ff);
    }
    return b;
}

static Status c2_forward(Replica &r, const tsfm_config &c, const C2Dev &w, const float *d_in, int64_t b,
                         int64_t t_in, int64_t horizon, float *d_out, cudaStream_t s) {
    int64_t t, start, pad, n_ctx, n_out, seq;
    c2_geometry(c, t_in, horizon, t, start, pad, n_ctx, n_out, seq);
    const int64_t d = c.d_model, ff = c.d_ff, ps = c.patch_size, q = c.num_quantiles, nh = c.num_heads;
    const float eps = (float)c.layer_norm_epsilon;
    const int64_t rows = b * seq;
    if (seq > w.max_seq) return Status::fail(TSFM_ERR_INVALID_ARGUMENT, "Chronos-2: sequence longer than the RoPE table");

    Arena &ws = r.ws;
    ws.reset();
    float *loc = ws.take<float>(b), *scl = ws.take<float>(b);
    float *feats = ws.take<float>(b * n_ctx * 3 * ps);
    uint8_t *kv = ws.take<uint8_t>(b * seq);
    float *x = ws.take<float>(rows * d);
    // 16-bit activations (element type w.act)
    uint16_t *xn = ws.take<uint16_t>(rows * d);
    uint16_t *qkv = ws.take<uint16_t>(rows * 3 * d);
    uint16_t *ao = ws.take<uint16_t>(rows * d);
    uint16_t *h = ws.take<uint16_t>(rows * ff);
    const int A16 = out_mode_for(w.act);
    float *raw = ws.take<float>(b * n_out * q * ps);
    float *hid_hi = ws.take<float>(b * n_out * d), *hid_lo = ws.take<float>(b * n_out * d);
    float *hh_hi = ws.take<float>(b * n_out * ff), *hh_lo = ws.take<float>(b * n_out * ff);
    const bool fused = c2_fused_norm(c) && (w.act == E_F16 || w.act == E_BF16);
    const int np = (int)(d / 256);
    float *nS = fused ? ws.take<float>(rows) : nullptr;       // row factors of the MLP norm
    float *nP = fused ? ws.take<float>(rows * np) : nullptr;  // row sums of squares per column tile
    // Corrected products: FP8 companions of the GEMM inputs xn, ao and h.
    uint8_t *xn8 = w.corr ? ws.take<uint8_t>(rows * 2 * d) : nullptr;
    uint8_t *ao8 = w.corr ? ws.take<uint8_t>(rows * 2 * d) : nullptr;
    uint8_t *h8 = w.corr ? ws.take<uint8_t>(rows * 2 * ff) : nullptr;
    auto in8 = [](LinearCall &lc, uint8_t *x8, int64_t cols) {  // the product's input companion
        lc.x8 = x8;
        lc.ldx8 = 2 * cols;
    };
    if (ws.used > ws.buf.bytes) return Status::fail(TSFM_ERR_OUT_OF_MEMORY, "Chronos-2: workspace too small");

    // 1. instance norm + patch features (TF32-rounded FP32) + key validity.
    {
        PatchCall pc;
        pc.inputs = d_in;
        pc.stride = t_in;
        pc.start = start;
        pc.t = t;
        pc.b = b;
        pc.ps = (int)ps;
        pc.pad = (int)pad;
        pc.n_ctx = (int)n_ctx;
        pc.feat_kind = 0;
        pc.tscale = (float)c.time_encoding_scale;
        pc.arcsinh = c.use_arcsinh;
        pc.feat_mode = OUT_TF32;
        pc.feats = feats;
        pc.loc = loc;
        pc.scale = scl;
        pc.key_valid = kv;
        pc.seq = seq;
        pc.extra_valid = (int)(1 + n_out);
        LaunchScope ls(r, s, K_PATCH, (double)b * t * 4 + (double)b * n_ctx * 3 * ps * 4);
        TSFM_TRY(launch_patch(pc, s));
    }
    // 2. patch embedding ResBlock straight into the sequence rows: x = res(f) + out(relu(hid(f))).
    {
        const int64_t m = b * n_ctx;
        LinearCall hx;
        hx.y8 = h8;
        hx.ldy8 = 2 * ff;
        TSFM_TRY(op_linear(r, s, w.in_embed.hidden, feats, m, 3 * ps, h, ff, A16, 1, &hx));
        LinearCall remap;
        remap.rm_g = n_ctx;
        remap.rm_G = seq;
        remap.rm_off = 0;
        TSFM_TRY(op_linear(r, s, w.in_embed.residual, feats, m, 3 * ps, x, d, OUT_F32, 0, &remap));
        in8(remap, h8, ff);
        TSFM_TRY(op_linear(r, s, w.in_embed.output, h, m, ff, x, d, OUT_F32_ACC, 0, &remap));
        LaunchScope ls(r, s, K_OTHER, (double)b * (1 + n_out) * d * 8);
        TSFM_TRY(launch_broadcast_rows(x, b, seq, n_ctx, w.reg, 1, d, s));
        TSFM_TRY(launch_broadcast_rows(x, b, seq, n_ctx + 1, w.fut_emb, n_out, d, s));
    }
    // 3. encoder layers.
    if (fused) {
        // The time-attention RMSNorm of layers 1.. is fused into the GEMMs around it: the previous
        // layer's wo GEMM (K = d_ff, whose long main loop hides the extra epilogue work) also
        // writes x * s_r * gamma in 16 bits to xn, s_r = the MLP norm's row factor, and the row's
        // sums of squares per 256-column tile; the QKV GEMM multiplies its rows by rs / s_r. The
        // other two norms stay separate: fused into the K = d_model residual GEMMs, the epilogue's
        // residual reads outlast their main loop (measured slower than the separate norm kernel).
        for (size_t li = 0; li < w.layers.size(); ++li) {
            const C2Dev::Layer &L = w.layers[li];
            LinearCall qc;
            qc.rope_cos = w.rope_cos;
            qc.rope_sin = w.rope_sin;
            qc.rope_cols = (int)(2 * d);
            qc.rope_p1 = 0;
            qc.rope_p2 = seq;
            in8(qc, xn8, d);
            if (li == 0) {
                TSFM_TRY(op_rmsnorm(r, s, x, L.time_norm, xn, A16, rows, d, eps, 0, 0, 0, nullptr, xn8));
            } else {
                qc.norm_in = nP;
                qc.norm_parts = np;
                qc.norm_dim = d;
                qc.norm_eps = eps;
                qc.norm_s_in = nS;
            }
            TSFM_TRY(op_linear(r, s, L.qkv, xn, rows, d, qkv, 3 * d, A16, 0, &qc));
            {
                AttentionCall ac;
                ac.err = static_cast<int *>(r.err.p);
                ac.q = qkv;
                ac.k = qkv + d;
                ac.v = qkv + 2 * d;
                ac.dtype = w.act;
                ac.ld_qkv = 3 * d;
                ac.o = ao;
                ac.ld_o = d;
                ac.key_valid = kv;
                ac.kv_stride = seq;
                ac.groups = (int)b;
                ac.heads = (int)nh;
                ac.n = (int)seq;
                ac.scale = 1.0f;
                ac.mask_mode = 0;
                ac.o8 = ao8;
                ac.ld_o8 = 2 * d;
                LaunchScope ls(r, s, K_ATTN, 4.0 * (double)b * nh * seq * seq * 64);
                TSFM_TRY(launch_attention(ac, s));
            }
            LinearCall oc, gc, ic, wc;
            in8(oc, ao8, d);
            in8(gc, xn8, d);
            in8(ic, xn8, d);
            in8(wc, h8, ff);
            ic.y8 = h8;
            ic.ldy8 = 2 * ff;
            TSFM_TRY(op_linear(r, s, L.o, ao, rows, d, x, d, OUT_F32_ACC, 0, &oc));
            TSFM_TRY(op_rmsnorm(r, s, x, L.group_norm, xn, A16, rows, d, eps, 0, 0, 0, nullptr, xn8));
            TSFM_TRY(op_linear(r, s, L.gvo, xn, rows, d, x, d, OUT_F32_ACC, 0, &gc));
            const bool last = li + 1 == w.layers.size();
            TSFM_TRY(op_rmsnorm(r, s, x, L.mlp_norm, xn, A16, rows, d, eps, 0, 0, 0, last ? nullptr : nS, xn8));
            TSFM_TRY(op_linear(r, s, L.wi, xn, rows, d, h, ff, A16, 1, &ic));
            if (!last) {
                wc.norm_out = nP;
                wc.norm_x16 = xn;
                wc.ld_x16 = d;
                wc.norm_gamma = w.layers[li + 1].time_norm;
                wc.norm_s_in = nS;
                wc.norm_x8 = xn8;
                wc.ld_nx8 = 2 * d;
            }
            TSFM_TRY(op_linear(r, s, L.wo, h, rows, ff, x, d, OUT_F32_ACC, 0, &wc));
        }
    }
    if (!fused)
    for (const C2Dev::Layer &L : w.layers) {
        TSFM_TRY(op_rmsnorm(r, s, x, L.time_norm, xn, A16, rows, d, eps, 0, 0, 0, nullptr, xn8));
        LinearCall rope;
        in8(rope, xn8, d);
        rope.rope_cos = w.rope_cos;
        rope.rope_sin = w.rope_sin;
        rope.rope_cols = (int)(2 * d);
        rope.rope_p1 = 0;
        rope.rope_p2 = seq;
        TSFM_TRY(op_linear(r, s, L.qkv, xn, rows, d, qkv, 3 * d, A16, 0, &rope));
        {
            AttentionCall ac;
            ac.err = static_cast<int *>(r.err.p);
            ac.q = qkv;
            ac.k = qkv + d;
            ac.v = qkv + 2 * d;
            ac.dtype = w.act;
            ac.ld_qkv = 3 * d;
            ac.o = ao;
            ac.ld_o = d;
            ac.key_valid = kv;
            ac.kv_stride = seq;
            ac.groups = (int)b;
            ac.heads = (int)nh;
            ac.n = (int)seq;
            ac.scale = 1.0f;
            ac.mask_mode = 0;
            ac.o8 = ao8;
            ac.ld_o8 = 2 * d;
            LaunchScope ls(r, s, K_ATTN, 4.0 * (double)b * nh * seq * seq * 64);
            TSFM_TRY(launch_attention(ac, s));
        }
        LinearCall oc, gc, ic, wc;
        in8(oc, ao8, d);
        in8(gc, xn8, d);
        in8(ic, xn8, d);
        in8(wc, h8, ff);
        ic.y8 = h8;
        ic.ldy8 = 2 * ff;
        TSFM_TRY(op_linear(r, s, L.o, ao, rows, d, x, d, OUT_F32_ACC, 0, &oc));
        TSFM_TRY(op_rmsnorm(r, s, x, L.group_norm, xn, A16, rows, d, eps, 0, 0, 0, nullptr, xn8));
        TSFM_TRY(op_linear(r, s, L.gvo, xn, rows, d, x, d, OUT_F32_ACC, 0, &gc));
        TSFM_TRY(op_rmsnorm(r, s, x, L.mlp_norm, xn, A16, rows, d, eps, 0, 0, 0, nullptr, xn8));
        TSFM_TRY(op_linear(r, s, L.wi, xn, rows, d, h, ff, A16, 1, &ic));
        TSFM_TRY(op_linear(r, s, L.wo, h, rows, ff, x, d, OUT_F32_ACC, 0, &wc));
    }
    // 4. final norm on the future-patch rows only, then the quantile head.
    const int64_t m = b * n_out;
    TSFM_TRY(op_rmsnorm(r, s, x, w.final_norm, hid_hi, OUT_F32, m, d, eps, n_out, seq, n_ctx + 1));
    // FP32-accurate head: out(relu(hidden(x))) + residual(x) with split-TF32 products.
    TSFM_TRY(op_split(r, s, hid_hi, hid_lo, m, d, d));
    TSFM_TRY(op_linear3(r, s, w.head_hidden, hid_hi, hid_lo, m, d, hh_hi, ff, false, 1));
    TSFM_TRY(op_split(r, s, hh_hi, hh_lo, m, ff, ff));
    TSFM_TRY(op_linear3(r, s, w.head_residual, hid_hi, hid_lo, m, d, raw, q * ps, false, 0));
    TSFM_TRY(op_linear3(r, s, w.head_output, hh_hi, hh_lo, m, ff, raw, q * ps, true, 0));
    {
        HeadPostCall hc;
        hc.raw = raw;
        hc.loc = loc;
        hc.scale = scl;
        hc.out = d_out;
        hc.b = b;
        hc.horizon = horizon;
        hc.q = (int)q;
        hc.ps = (int)ps;
        hc.n_out = (int)n_out;
        hc.arcsinh = c.use_arcsinh;
        hc.layout = 0;
        LaunchScope ls(r, s, K_HEAD, (double)b * horizon * q * 8);
        TSFM_TRY(launch_head_post(hc, s));
    }
    return Status::ok();
}

// Chunks of series sized so the workspace stays within the budget (the reference bounds its
// scratch the same way: chronos2/forecaster.zig:42-57).
Status c2_forecast(Replica &r, const tsfm_config &c, const C2Dev &w, const float *d_in, int64_t b, int64_t t_in,
                   int64_t horizon, float *d_out, cudaStream_t s) {
    const size_t per = c2_workspace(c, w.corr, 1, t_in, horizon);
    int64_t chunk = std::max<int64_t>(1, std::min<int64_t>(b, (int64_t)(workspace_budget(r) / std::max<size_t>(per, 1))));
    const int64_t nchunks = (b + chunk - 1) / chunk;
    chunk = (b + nchunks - 1) / nchunks;
    TSFM_TRY(r.ws.reserve(c2_workspace(c, w.corr, chunk, t_in, horizon)));
    const int64_t q = c.num_quantiles;
    for (int64_t s0 = 0; s0 < b; s0 += chunk) {
        const int64_t n = std::min(chunk, b - s0);
        TSFM_TRY(c2_forward(r, c, w, d_in + s0 * t_in, n, t_in, horizon, d_out + s0 * horizon * q, s));
    }
    return Status::ok();
}

}  // namespace tsfm
