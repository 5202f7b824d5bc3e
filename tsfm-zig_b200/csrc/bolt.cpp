// Chronos-Bolt on the device: the T5 encoder over patch embeddings, the one-token decoder with
// cross-attention, the quantile head (chronos_bolt/model.zig) and the forecaster with its
// long-horizon quantile-path loop (chronos_bolt/forecaster.zig).
//
// Per encoder layer (chronos_bolt/model.zig:222-237): rmsnorm -> [q|k|v] GEMM -> flash attention
// with the shared relative-position bias added in-tile (T5: no 1/sqrt(d) scale, additive key mask)
// -> x += o GEMM -> rmsnorm -> relu FFN -> x += wo GEMM. The decoder keeps one token per series:
// self-attention over one key is o(v(norm x)); cross-attention reads K and V projected from the
// encoder output in one GEMM over all encoder rows; FFN; final norm; FP32-accurate head.
// Horizons beyond one block run every quantile path as its own context row and reduce the q^2
// samples per step to q empirical quantiles on the device (chronos_bolt/forecaster.zig:45-78).
#include <algorithm>
#include <cstring>

#include "model.h"
#include "ops.h"

namespace tsfm {

// relativeBucket (chronos_bolt/model.zig:74-85): T5 bidirectional bucket with the float32 log.
int64_t relative_bucket(int64_t rel, uint32_t num_buckets, uint32_t max_distance) {
    const uint32_t half = num_buckets / 2;
    const uint32_t base = rel > 0 ? half : 0;
    const uint32_t rp = (uint32_t)(rel < 0 ? -rel : rel);
    const uint32_t max_exact = half / 2;
    if (rp < max_exact) return base + rp;
    const float ratio = (float)rp / (float)max_exact;
    const float denom = (float)std::log((double)max_distance / (double)max_exact);
    const float large_f = std::log(ratio) / denom * (float)(half - max_exact);
    const uint32_t large = max_exact + (uint32_t)large_f;
    return base + std::min(large, half - 1);
}

namespace {

int64_t inner_dim(const tsfm_config &c) { return (int64_t)c.num_heads * c.d_kv; }
int64_t vocab(const tsfm_config &c) { return c.use_reg_token ? 2 : 1; }

struct Geo {
    int64_t pad, n_patch, seq;
};
Geo geometry(const tsfm_config &c, int64_t len) {
    const int64_t ps = c.patch_size;
    Geo g;
    g.pad = (ps - len % ps) % ps;
    g.n_patch = (len + g.pad) / ps;
    g.seq = g.n_patch + (c.use_reg_token ? 1 : 0);
    return g;
}

size_t block_workspace(const tsfm_config &c, int64_t nb, int64_t len) {
    const Geo g = geometry(c, len);
    const int64_t d = c.d_model, ff = c.d_ff, in = inner_dim(c), ps = c.patch_size;
    const int64_t q = c.num_quantiles, P = c.prediction_length, rows = nb * g.seq;
    size_t b = 0;
    b += Arena::span(nb * 4) * 2;                        // loc, scale
    b += Arena::span(nb * g.n_patch * 2 * ps * 4);       // features
    b += Arena::span(nb * g.seq);                        // key validity
    b += Arena::span(rows * d * 4);                      // x
    b += Arena::span(rows * d * 2);                      // xn / encoder output (16-bit)
    b += Arena::span(rows * 3 * in * 2);                 // qkv / cross k,v
    b += Arena::span(rows * in * 2);                     // attention output
    b += Arena::span(rows * std::max(ff, d) * 2);        // FFN hidden
    b += Arena::span(nb * d * 4);                        // decoder x
    b += Arena::span(nb * d * 2);                        // decoder xn
    b += Arena::span(nb * in * 2) * 2;                   // decoder q, attention out
    b += Arena::span(nb * d * 4) * 2;                    // head input hi / lo
    b += Arena::span(nb * ff * 4) * 2;                   // head hidden hi / lo
    b += Arena::span(nb * q * P * 4);                    // raw head output
    return b;
}

// One encoder/decoder pass for n rows of context (row s at ctx + s * stride + offset, length len):
// out (n, q, P) in data units (chronos_bolt/forecaster.zig:129-220).
Status predict_chunk(Replica &r, const tsfm_config &c, const BoltDev &w, const float *ctx, int64_t stride,
                     int64_t offset, int64_t len, int64_t n, float *out, cudaStream_t s) {
    const Geo g = geometry(c, len);
    const int64_t d = c.d_model, ff = c.d_ff, in = inner_dim(c), ps = c.patch_size, nh = c.num_heads;
    const int64_t q = c.num_quantiles, P = c.prediction_length;
    const int64_t rows = n * g.seq;
    const float eps = (float)c.layer_norm_epsilon;
    if (g.seq > w.max_seq) return Status::fail(TSFM_ERR_INVALID_ARGUMENT, "Chronos-Bolt: context longer than the model's");
    Arena &ws = r.ws;
    ws.reset();
    float *loc = ws.take<float>(n), *scl = ws.take<float>(n);
    float *feats = ws.take<float>(n * g.n_patch * 2 * ps);
    uint8_t *kv = ws.take<uint8_t>(n * g.seq);
    float *x = ws.take<float>(rows * d);
    uint16_t *xn = ws.take<uint16_t>(rows * d);
    uint16_t *qkv = ws.take<uint16_t>(rows * 3 * in);
    uint16_t *ao = ws.take<uint16_t>(rows * in);
    uint16_t *hbuf = ws.take<uint16_t>(rows * std::max(ff, d));
    float *xd = ws.take<float>(n * d);
    uint16_t *xdn = ws.take<uint16_t>(n * d);
    uint16_t *qd = ws.take<uint16_t>(n * in), *ad = ws.take<uint16_t>(n * in);
    float *hid_hi = ws.take<float>(n * d), *hid_lo = ws.take<float>(n * d);
    float *hh_hi = ws.take<float>(n * ff), *hh_lo = ws.take<float>(n * ff);
    float *raw = ws.take<float>(n * q * P);
    if (ws.used > ws.buf.bytes) return Status::fail(TSFM_ERR_OUT_OF_MEMORY, "Chronos-Bolt: workspace too small");
    const int A16 = out_mode_for(w.act);

    {
        PatchCall pc;
        pc.inputs = ctx;
        pc.stride = stride;
        pc.start = offset;
        pc.t = len;
        pc.b = n;
        pc.ps = (int)ps;
        pc.pad = (int)g.pad;
        pc.n_ctx = (int)g.n_patch;
        pc.feat_kind = 1;
        pc.arcsinh = 0;
        pc.feat_mode = OUT_TF32;
        pc.feats = feats;
        pc.loc = loc;
        pc.scale = scl;
        pc.key_valid = kv;
        pc.seq = g.seq;
        pc.extra_valid = c.use_reg_token ? 1 : 0;
        LaunchScope ls(r, s, K_PATCH, (double)n * len * 4 + (double)n * g.n_patch * 2 * ps * 4);
        TSFM_TRY(launch_patch(pc, s));
    }
    {
        const int64_t m = n * g.n_patch;
        TSFM_TRY(op_linear(r, s, w.in_embed.hidden, feats, m, 2 * ps, hbuf, ff, A16, 1));
        LinearCall remap;
        remap.rm_g = g.n_patch;
        remap.rm_G = g.seq;
        TSFM_TRY(op_linear(r, s, w.in_embed.residual, feats, m, 2 * ps, x, d, OUT_F32, 0, &remap));
        TSFM_TRY(op_linear(r, s, w.in_embed.output, hbuf, m, ff, x, d, OUT_F32_ACC, 0, &remap));
        if (c.use_reg_token) {
            LaunchScope ls(r, s, K_OTHER, (double)n * d * 8);
            TSFM_TRY(launch_broadcast_rows(x, n, g.seq, g.n_patch, w.reg, 1, d, s));
        }
    }
    for (const BoltDev::Enc &L : w.enc) {
        TSFM_TRY(op_rmsnorm(r, s, x, L.attn_norm, xn, A16, rows, d, eps));
        TSFM_TRY(op_linear(r, s, L.qkv, xn, rows, d, qkv, 3 * in, A16, 0));
        {
            AttentionCall ac;
            ac.err = static_cast<int *>(r.err.p);
            ac.q = qkv;
            ac.k = qkv + in;
            ac.v = qkv + 2 * in;
            ac.dtype = w.act;
            ac.ld_qkv = 3 * in;
            ac.o = ao;
            ac.ld_o = in;
            ac.key_valid = kv;
            ac.kv_stride = g.seq;
            ac.rel_bias = w.rel;
            ac.rel_stride = 2 * w.max_seq - 1;
            ac.rel_center = w.max_seq - 1;
            ac.groups = (int)n;
            ac.heads = (int)nh;
            ac.n = (int)g.seq;
            ac.scale = 1.0f;
            ac.mask_mode = 0;
            LaunchScope ls(r, s, K_ATTN, 4.0 * (double)n * nh * g.seq * g.seq * 64);
            TSFM_TRY(launch_attention(ac, s));
        }
        TSFM_TRY(op_linear(r, s, L.o, ao, rows, in, x, d, OUT_F32_ACC, 0));
        TSFM_TRY(op_rmsnorm(r, s, x, L.ffn_norm, xn, A16, rows, d, eps));
        TSFM_TRY(op_linear(r, s, L.wi, xn, rows, d, hbuf, ff, A16, 1));
        TSFM_TRY(op_linear(r, s, L.wo, hbuf, rows, ff, x, d, OUT_F32_ACC, 0));
    }
    // Encoder output (the final norm) in 16-bit: it only feeds the cross K/V projection.
    TSFM_TRY(op_rmsnorm(r, s, x, w.enc_final, xn, A16, rows, d, eps));

    // Decoder: one token per series, starting from shared[decoder_start_token_id].
    {
        LaunchScope ls(r, s, K_OTHER, (double)n * d * 8);
        TSFM_TRY(launch_broadcast_rows(xd, n, 1, 0, w.start, 1, d, s));
    }
    for (const BoltDev::Dec &L : w.dec) {
        TSFM_TRY(op_rmsnorm(r, s, xd, L.self_norm, xdn, A16, n, d, eps));
        TSFM_TRY(op_linear(r, s, L.self_v, xdn, n, d, ad, in, A16, 0));
        TSFM_TRY(op_linear(r, s, L.self_o, ad, n, in, xd, d, OUT_F32_ACC, 0));
        TSFM_TRY(op_rmsnorm(r, s, xd, L.cross_norm, xdn, A16, n, d, eps));
        TSFM_TRY(op_linear(r, s, L.cross_q, xdn, n, d, qd, in, A16, 0));
        TSFM_TRY(op_linear(r, s, L.cross_kv, xn, rows, d, qkv, 2 * in, A16, 0));
        {
            CrossAttnCall cc;
            cc.q = qd;
            cc.k = qkv;
            cc.v = qkv + in;
            cc.dtype = w.act;
            cc.ld_q = in;
            cc.ld_kv = 2 * in;
            cc.ld_o = in;
            cc.o = ad;
            cc.key_valid = kv;
            cc.b = n;
            cc.heads = (int)nh;
            cc.seq = (int)g.seq;
            LaunchScope ls(r, s, K_ATTN, 4.0 * (double)n * nh * g.seq * 64);
            TSFM_TRY(launch_cross_attention(cc, s));
        }
        TSFM_TRY(op_linear(r, s, L.cross_o, ad, n, in, xd, d, OUT_F32_ACC, 0));
        TSFM_TRY(op_rmsnorm(r, s, xd, L.ffn_norm, xdn, A16, n, d, eps));
        TSFM_TRY(op_linear(r, s, L.wi, xdn, n, d, hbuf, ff, A16, 1));
        TSFM_TRY(op_linear(r, s, L.wo, hbuf, n, ff, xd, d, OUT_F32_ACC, 0));
    }
    // Final decoder norm, FP32-accurate head, inverse instance norm.
    TSFM_TRY(op_rmsnorm(r, s, xd, w.dec_final, hid_hi, OUT_F32, n, d, eps));
    TSFM_TRY(op_split(r, s, hid_hi, hid_lo, n, d, d));
    TSFM_TRY(op_linear3(r, s, w.head_hidden, hid_hi, hid_lo, n, d, hh_hi, ff, false, 1));
    TSFM_TRY(op_split(r, s, hh_hi, hh_lo, n, ff, ff));
    TSFM_TRY(op_linear3(r, s, w.head_residual, hid_hi, hid_lo, n, d, raw, q * P, false, 0));
    TSFM_TRY(op_linear3(r, s, w.head_output, hh_hi, hh_lo, n, ff, raw, q * P, true, 0));
    HeadPostCall hc;
    hc.raw = raw;
    hc.loc = loc;
    hc.scale = scl;
    hc.out = out;
    hc.b = n;
    hc.q = (int)q;
    hc.ps = (int)P;
    hc.arcsinh = 0;
    hc.layout = 1;
    LaunchScope ls(r, s, K_HEAD, (double)n * q * P * 8);
    return launch_head_post(hc, s);
}

// predictBlock (chronos_bolt/forecaster.zig:116-127): chunks sized by the workspace budget.
Status predict_block(Replica &r, const tsfm_config &c, const BoltDev &w, const float *ctx, int64_t stride,
                     int64_t offset, int64_t len, int64_t n, float *out, cudaStream_t s) {
    const size_t per = block_workspace(c, 1, len);
    int64_t chunk = std::max<int64_t>(1, std::min<int64_t>(n, (int64_t)(workspace_budget(r) / std::max<size_t>(per, 1))));
    const int64_t nchunks = (n + chunk - 1) / chunk;
    chunk = (n + nchunks - 1) / nchunks;
    TSFM_TRY(r.ws.reserve(block_workspace(c, chunk, len)));
    const int64_t qP = (int64_t)c.num_quantiles * c.prediction_length;
    for (int64_t s0 = 0; s0 < n; s0 += chunk) {
        const int64_t m = std::min(chunk, n - s0);
        TSFM_TRY(predict_chunk(r, c, w, ctx + s0 * stride, stride, offset, len, m, out + s0 * qP, s));
    }
    return Status::ok();
}

Status load_lin(Replica &r, const TensorTable &t, const std::string &name, int64_t out, int64_t in, int act, DLin &dst) {
    const tsfm_tensor *w;
    TSFM_TRY(t.raw(name, out * in, &w));
    return upload_lin_raw(r, {w}, nullptr, out, in, act, dst);
}

Status load_concat(Replica &r, const TensorTable &t, const std::vector<std::string> &names, int64_t out_each, int64_t in,
                   int act, DLin &dst) {
    std::vector<const tsfm_tensor *> parts;
    for (const auto &nm : names) {
        const tsfm_tensor *w;
        TSFM_TRY(t.raw(nm, out_each * in, &w));
        parts.push_back(w);
    }
    return upload_lin_raw(r, parts, nullptr, out_each * (int64_t)names.size(), in, act, dst);
}

Status load_norm(Replica &r, const TensorTable &t, const std::string &name, int64_t d, float **dst) {
    std::vector<float> v;
    TSFM_TRY(t.get(name, d, v));
    return upload_f32(r, v, dst);
}

}  // namespace

Status bolt_validate(const tsfm_config &c) {
    // chronos_bolt/config.zig:48-59
    if (c.d_model <= 0 || c.d_ff <= 0 || c.num_heads <= 0 || c.d_kv <= 0) return Status::fail(TSFM_ERR_INVALID_CONFIG, "InvalidConfig: dimensions");
    if (c.num_layers <= 0 || c.num_decoder_layers <= 0) return Status::fail(TSFM_ERR_INVALID_CONFIG, "InvalidConfig: layers");
    if (c.patch_size <= 0 || c.prediction_length <= 0 || c.context_length <= 0) return Status::fail(TSFM_ERR_INVALID_CONFIG, "InvalidConfig: patch / prediction / context");
    if (c.num_quantiles <= 0 || !c.quantiles) return Status::fail(TSFM_ERR_INVALID_CONFIG, "InvalidConfig: quantiles");
    if (c.relative_attention_num_buckets < 4 || c.relative_attention_num_buckets % 2) return Status::fail(TSFM_ERR_INVALID_CONFIG, "InvalidConfig: buckets");
    if (c.reg_token_id < 0 || c.reg_token_id >= vocab(c) || c.decoder_start_token_id < 0 || c.decoder_start_token_id >= vocab(c))
        return Status::fail(TSFM_ERR_INVALID_CONFIG, "InvalidConfig: token ids");
    // Kernel constraints of this backend.
    if (c.d_kv != 64) return Status::fail(TSFM_ERR_UNSUPPORTED, "Chronos-Bolt: head width must be 64");
    if (c.d_model % 8 || c.d_ff % 8) return Status::fail(TSFM_ERR_UNSUPPORTED, "Chronos-Bolt: d_model % 8 and d_ff % 8 must be 0");
    if ((2 * c.patch_size) % 4 || ((int64_t)c.num_quantiles * c.prediction_length) % 4)
        return Status::fail(TSFM_ERR_UNSUPPORTED, "Chronos-Bolt: feature / head rows must be 16-byte multiples");
    if (c.num_quantiles * c.num_quantiles > 256) return Status::fail(TSFM_ERR_UNSUPPORTED, "Chronos-Bolt: at most 16 quantiles");
    return Status::ok();
}

Status bolt_check_tensors(const tsfm_config &c, const TensorTable &t) {
    const int64_t d = c.d_model, ff = c.d_ff, in = inner_dim(c), ps = c.patch_size;
    const int64_t out_dim = (int64_t)c.num_quantiles * c.prediction_length;
    TSFM_TRY(check_resblock(t, "input_patch_embedding", 2 * ps, ff, d, true));
    TSFM_TRY(check_resblock(t, "output_patch_embedding", d, ff, out_dim, true));
    TSFM_TRY(t.check("shared.weight", vocab(c) * d));
    TSFM_TRY(t.check("encoder.block.0.layer.0.SelfAttention.relative_attention_bias.weight",
                     (int64_t)c.relative_attention_num_buckets * c.num_heads));
    TSFM_TRY(t.check("encoder.final_layer_norm.weight", d));
    TSFM_TRY(t.check("decoder.final_layer_norm.weight", d));
    for (int i = 0; i < c.num_layers; ++i) {
        const std::string p = strf("encoder.block.%d.", i);
        TSFM_TRY(t.check(p + "layer.0.layer_norm.weight", d));
        for (const char *m : {"q", "k", "v"}) TSFM_TRY(t.check(p + "layer.0.SelfAttention." + m + ".weight", in * d));
        TSFM_TRY(t.check(p + "layer.0.SelfAttention.o.weight", d * in));
        TSFM_TRY(t.check(p + "layer.1.layer_norm.weight", d));
        TSFM_TRY(t.check(p + "layer.1.DenseReluDense.wi.weight", ff * d));
        TSFM_TRY(t.check(p + "layer.1.DenseReluDense.wo.weight", d * ff));
    }
    for (int i = 0; i < c.num_decoder_layers; ++i) {
        const std::string p = strf("decoder.block.%d.", i);
        for (const char *nm : {"layer.0.layer_norm.weight", "layer.1.layer_norm.weight", "layer.2.layer_norm.weight"})
            TSFM_TRY(t.check(p + nm, d));
        TSFM_TRY(t.check(p + "layer.0.SelfAttention.v.weight", in * d));
        TSFM_TRY(t.check(p + "layer.0.SelfAttention.o.weight", d * in));
        for (const char *m : {"q", "k", "v"}) TSFM_TRY(t.check(p + "layer.1.EncDecAttention." + m + ".weight", in * d));
        TSFM_TRY(t.check(p + "layer.1.EncDecAttention.o.weight", d * in));
        TSFM_TRY(t.check(p + "layer.2.DenseReluDense.wi.weight", ff * d));
        TSFM_TRY(t.check(p + "layer.2.DenseReluDense.wo.weight", d * ff));
    }
    return Status::ok();
}

Status bolt_load(Replica &r, const tsfm_config &c, const TensorTable &t, int act, BoltDev &w) {
    const int64_t d = c.d_model, ff = c.d_ff, in = inner_dim(c), ps = c.patch_size, nh = c.num_heads;
    const int64_t out_dim = (int64_t)c.num_quantiles * c.prediction_length;
    w.act = act;
    TSFM_TRY(load_resblock(r, t, "input_patch_embedding", 2 * ps, ff, d, true, E_F32, act, w.in_embed));
    {
        const std::string p = "output_patch_embedding";
        std::vector<float> m;
        TSFM_TRY(t.get(p + ".hidden_layer.weight", ff * d, m));
        TSFM_TRY(upload_lin3(r, m, ff, d, w.head_hidden));
        TSFM_TRY(t.get(p + ".hidden_layer.bias", ff, m));
        TSFM_TRY(upload_bias(r, m, w.head_hidden.hi));
        TSFM_TRY(t.get(p + ".output_layer.weight", out_dim * ff, m));
        TSFM_TRY(upload_lin3(r, m, out_dim, ff, w.head_output));
        TSFM_TRY(t.get(p + ".output_layer.bias", out_dim, m));
        TSFM_TRY(upload_bias(r, m, w.head_output.hi));
        TSFM_TRY(t.get(p + ".residual_layer.weight", out_dim * d, m));
        TSFM_TRY(upload_lin3(r, m, out_dim, d, w.head_residual));
        TSFM_TRY(t.get(p + ".residual_layer.bias", out_dim, m));
        TSFM_TRY(upload_bias(r, m, w.head_residual.hi));
    }
    std::vector<float> shared;
    TSFM_TRY(t.get("shared.weight", vocab(c) * d, shared));
    TSFM_TRY(upload_f32(r, std::vector<float>(shared.begin() + (int64_t)c.decoder_start_token_id * d,
                                              shared.begin() + (int64_t)(c.decoder_start_token_id + 1) * d),
                        &w.start));
    if (c.use_reg_token)
        TSFM_TRY(upload_f32(r, std::vector<float>(shared.begin() + (int64_t)c.reg_token_id * d,
                                                  shared.begin() + (int64_t)(c.reg_token_id + 1) * d),
                            &w.reg));
    TSFM_TRY(load_norm(r, t, "encoder.final_layer_norm.weight", d, &w.enc_final));
    TSFM_TRY(load_norm(r, t, "decoder.final_layer_norm.weight", d, &w.dec_final));
    for (int i = 0; i < c.num_layers; ++i) {
        const std::string p = strf("encoder.block.%d.", i);
        BoltDev::Enc L;
        TSFM_TRY(load_norm(r, t, p + "layer.0.layer_norm.weight", d, &L.attn_norm));
        TSFM_TRY(load_concat(r, t, {p + "layer.0.SelfAttention.q.weight", p + "layer.0.SelfAttention.k.weight",
                                    p + "layer.0.SelfAttention.v.weight"}, in, d, act, L.qkv));
        TSFM_TRY(load_lin(r, t, p + "layer.0.SelfAttention.o.weight", d, in, act, L.o));
        TSFM_TRY(load_norm(r, t, p + "layer.1.layer_norm.weight", d, &L.ffn_norm));
        TSFM_TRY(load_lin(r, t, p + "layer.1.DenseReluDense.wi.weight", ff, d, act, L.wi));
        TSFM_TRY(load_lin(r, t, p + "layer.1.DenseReluDense.wo.weight", d, ff, act, L.wo));
        w.enc.push_back(L);
    }
    for (int i = 0; i < c.num_decoder_layers; ++i) {
        const std::string p = strf("decoder.block.%d.", i);
        BoltDev::Dec L;
        TSFM_TRY(load_norm(r, t, p + "layer.0.layer_norm.weight", d, &L.self_norm));
        TSFM_TRY(load_lin(r, t, p + "layer.0.SelfAttention.v.weight", in, d, act, L.self_v));
        TSFM_TRY(load_lin(r, t, p + "layer.0.SelfAttention.o.weight", d, in, act, L.self_o));
        TSFM_TRY(load_norm(r, t, p + "layer.1.layer_norm.weight", d, &L.cross_norm));
        TSFM_TRY(load_lin(r, t, p + "layer.1.EncDecAttention.q.weight", in, d, act, L.cross_q));
        TSFM_TRY(load_concat(r, t, {p + "layer.1.EncDecAttention.k.weight", p + "layer.1.EncDecAttention.v.weight"},
                             in, d, act, L.cross_kv));
        TSFM_TRY(load_lin(r, t, p + "layer.1.EncDecAttention.o.weight", d, in, act, L.cross_o));
        TSFM_TRY(load_norm(r, t, p + "layer.2.layer_norm.weight", d, &L.ffn_norm));
        TSFM_TRY(load_lin(r, t, p + "layer.2.DenseReluDense.wi.weight", ff, d, act, L.wi));
        TSFM_TRY(load_lin(r, t, p + "layer.2.DenseReluDense.wo.weight", d, ff, act, L.wo));
        w.dec.push_back(L);
    }
    // Relative-position bias by key - query offset for every length up to the context
    // (positionBias, chronos_bolt/model.zig:195-205): rel[h][off + max_seq - 1].
    std::vector<float> table;
    TSFM_TRY(t.get("encoder.block.0.layer.0.SelfAttention.relative_attention_bias.weight",
                   (int64_t)c.relative_attention_num_buckets * nh, table));
    w.max_seq = (c.context_length + c.patch_size - 1) / c.patch_size + (c.use_reg_token ? 1 : 0);
    const int64_t width = 2 * w.max_seq - 1;
    std::vector<float> rel(nh * width);
    for (int64_t off = -(w.max_seq - 1); off <= w.max_seq - 1; ++off) {
        const int64_t bucket = relative_bucket(off, (uint32_t)c.relative_attention_num_buckets,
                                               (uint32_t)c.relative_attention_max_distance);
        for (int64_t h = 0; h < nh; ++h) rel[h * width + off + w.max_seq - 1] = table[bucket * nh + h];
    }
    TSFM_TRY(upload_f32(r, rel, &w.rel));
    std::vector<float> lv(c.num_quantiles);
    for (int i = 0; i < c.num_quantiles; ++i) lv[i] = (float)c.quantiles[i];
    TSFM_TRY(upload_f32(r, lv, &w.levels));
    return Status::ok();
}

// forecaster.forecast (chronos_bolt/forecaster.zig:22-80).
Status bolt_forecast(Replica &r, const tsfm_config &c, const BoltDev &w, const float *d_in, int64_t b, int64_t t_in,
                     int64_t horizon, float *d_out, cudaStream_t s) {
    const int64_t q = c.num_quantiles, P = c.prediction_length, max_ctx = c.context_length;
    const int64_t len0 = std::min(t_in, max_ctx);
    const int64_t bq = b * q;
    // Forecaster buffers: pred (b*q rows of P), raw (b*q*q rows of P), two context buffers.
    const int64_t max_len = std::min(len0 + (horizon + P - 1) / P * P, max_ctx);
    const bool long_h = horizon > P;
    size_t fc_bytes = Arena::span(bq * P * 4);
    if (long_h) fc_bytes += Arena::span(bq * q * P * 4) + 2 * Arena::span(bq * max_len * 4);
    TSFM_TRY(r.fc.reserve(fc_bytes));
    Arena &fc = r.fc;
    fc.reset();
    float *pred = fc.take<float>(bq * P);
    float *raw = long_h ? fc.take<float>(bq * q * P) : nullptr;
    float *cur = long_h ? fc.take<float>(bq * max_len) : nullptr;
    float *next = long_h ? fc.take<float>(bq * max_len) : nullptr;

    TSFM_TRY(predict_block(r, c, w, d_in, t_in, t_in - len0, len0, b, pred, s));
    {
        LaunchScope ls(r, s, K_OTHER, (double)b * q * P * 8);
        TSFM_TRY(launch_bolt_store(pred, d_out, b, (int)q, (int)P, horizon, 0, s));
    }
    int64_t done = std::min(P, horizon);
    if (done >= horizon) return Status::ok();
    int64_t len = len0;
    {
        LaunchScope ls(r, s, K_OTHER, (double)bq * len * 8);
        TSFM_TRY(launch_bolt_replicate(d_in, t_in, t_in - len0, len0, (int)q, cur, b, s));
    }
    while (done < horizon) {
        const int64_t new_len = std::min(len + P, max_ctx), skip = len + P - new_len;
        {
            LaunchScope ls(r, s, K_OTHER, (double)bq * new_len * 8);
            TSFM_TRY(launch_bolt_extend(cur, len, pred, (int)P, next, new_len, skip, bq, s));
        }
        std::swap(cur, next);
        len = new_len;
        TSFM_TRY(predict_block(r, c, w, cur, len, 0, len, bq, raw, s));
        {
            LaunchScope ls(r, s, K_OTHER, (double)bq * q * P * 4);
            TSFM_TRY(launch_bolt_quantiles(raw, w.levels, pred, b, (int)q, (int)P, s));
        }
        {
            LaunchScope ls(r, s, K_OTHER, (double)b * q * P * 8);
            TSFM_TRY(launch_bolt_store(pred, d_out, b, (int)q, (int)P, horizon, done, s));
        }
        done += P;
    }
    return Status::ok();
}

}  // namespace tsfm
