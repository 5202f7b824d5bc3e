// Timestral on the device: the decoder-only time/variate transformer of timestral/model.zig and
// the block-autoregressive forecaster of timestral/forecaster.zig.
//
// Host side (C++; timestral/forecaster.zig:57-141): options and argument checks, the uploads of the
// raw arrays. Device side, once per forecast: categorical target encoding and the covariate
// channels, the input rows of the forward and mirrored passes (forward fill, left padding to a
// patch multiple; both passes of the symmetric average batched as one run over twice the series);
// then per block: statistics + features, patch embedding, the transformer over
// [Enc ; Dec] tokens (fused QKV|gate GEMM with partial RoPE in its epilogue, flash attention with
// the encoder causal_keys / decoder-chain masks, 11x11 variate attention, gated output, SwiGLU
// MLP), the FP32-accurate head with the monotone quantile construction, the refine frame, the
// feedback of medians / known futures / blanks; then the quantile cap, the NaN check, the
// symmetric average and the non-negative clip.
#include <algorithm>
#include <climits>
#include <cstdlib>
#include <cmath>
#include <cstring>

#include "model.h"
#include "ops.h"
#include "timestral_kernels.h"

namespace tsfm {

namespace {

int64_t hd_of(const tsfm_config &c) { return c.d_model / c.num_heads; }
int64_t rope_dim(const tsfm_config &c) { return (int64_t)((double)hd_of(c) * c.rope_partial_factor); }

// The (attention, is_time) list of a layer kind (timestral/config.zig:94-100).
int layer_axes(int kind, bool *is_time) {
    switch (kind) {
        case TSFM_LAYER_TIME: is_time[0] = true; return 1;
        case TSFM_LAYER_VARIATE: is_time[0] = false; return 1;
        case TSFM_LAYER_TIME_VARIATE: is_time[0] = true; is_time[1] = false; return 2;
        default: is_time[0] = false; is_time[1] = true; return 2;
    }
}

// Config.supportsKnownCovariates (timestral/config.zig:49-72).
bool supports_known(const tsfm_config &c) {
    if (!c.covariate_enabled) return false;
    std::vector<bool> ops;
    for (int i = 0; i < c.n_layer_kinds; ++i) {
        bool it[2];
        const int na = layer_axes(c.layer_kinds[i], it);
        for (int a = 0; a < na; ++a) ops.push_back(it[a]);
    }
    for (size_t i = 0; i < ops.size(); ++i) {
        if (!ops[i]) continue;
        bool any_time = false, any_var = false;
        for (size_t j = i + 1; j < ops.size(); ++j) {
            any_time = any_time || ops[j];
            any_var = any_var || !ops[j];
        }
        if (any_time && any_var) return true;
    }
    return false;
}

int median_index(const tsfm_config &c) {
    for (int i = 0; i < c.num_quantiles; ++i)
        if (c.quantiles[i] == 0.5) return i;
    return 0;
}

// ---------------------------------------------------------------------------------------------
// Device forward

struct Block {
    int64_t groups, vall, v, t, h, ps;
    bool cov;
};

// The first RMSNorm of layers 1.. runs inside the GEMMs around it (LinearCall::norm_*): the
// previous layer's w3 GEMM (K = the MLP width, whose long main loop hides the extra epilogue
// work) also writes x * s_r * gamma in 16 bits, s_r = the MLP norm's row factor, and the row's
// sums of squares per 256-column tile; the layer's first q/k/v(/gate) GEMM multiplies its rows by
// rs / s_r. Needs d_model a multiple of 256 and 16-bit operands; TSFM_FUSED_NORM=0 turns it off.
static bool ts_fused_norm(const tsfm_config &c, int act) {
    static const bool on = [] {
        const char *v = std::getenv("TSFM_FUSED_NORM");
        return !(v && v[0] == '0');
    }();
    return on && c.d_model % 256 == 0 && (act == E_F16 || act == E_BF16);
}

size_t block_workspace(const tsfm_config &c, const TsDev &w, const Block &k) {
    const int64_t d = c.d_model, hid = c.d_ff, q = c.num_quantiles, ps = k.ps;
    const int64_t R = k.groups * k.vall, hl = k.h * ps, wlen = k.cov ? k.t + hl : k.t, n = wlen / ps;
    const int64_t sl = n + k.h, rows = R * sl, nt = k.groups * k.v;
    const int64_t cols = w.max_qkv_cols;
    size_t b = 0;
    b += Arena::span(R * n * 4) * 2 + Arena::span(R * 4) * 2 + Arena::span(R) * 2 + Arena::span(R * n);
    b += Arena::span(k.groups * 4) + Arena::span(R * n * 2 * ps * 4);
    b += Arena::span(k.groups * sl * 32 * 4) * 2;
    b += Arena::span(rows * d * 4) + Arena::span(rows * d * 2) + Arena::span(rows * cols * 2) + Arena::span(rows * d * 2);
    b += Arena::span(rows * std::max<int64_t>(2 * hid, 4 * d) * 2) + Arena::span(rows * hid * 2);
    b += Arena::span(nt * k.h * 8) + Arena::span(nt * 8);
    b += Arena::span(nt * k.h * d * 4) * 2 + Arena::span(nt * k.h * 4 * d * 4) * 2 + Arena::span(nt * hl * q * 4) * 2;
    if (ts_fused_norm(c, w.act)) b += Arena::span(rows * 4) + Arena::span(rows * (d / 256) * 4);
    if (w.corr)  // FP8 companions of xn, the attention output (and its FP32 form), a and the patch hidden
        b += Arena::span(rows * 2 * d) * 2 + Arena::span(rows * d * 4) + Arena::span(rows * 2 * hid) +
             Arena::span(R * n * 2 * 4 * d);
    return b;
}

// Model.predictBlock (timestral/model.zig:220-432) for `groups` series at context length t:
// writes qs (groups * v, h * ps, q).
Status predict_block(Replica &r, const tsfm_config &c, const TsDev &w, const Block &k, const float *ctx,
                     const uint8_t *obs, const float *kf, const uint8_t *kfm, int64_t kf_ld, float *qs, cudaStream_t s) {
    const int64_t d = c.d_model, hid = c.d_ff, q = c.num_quantiles, ps = k.ps, nh = c.num_heads;
    const int64_t R = k.groups * k.vall, hl = k.h * ps, wlen = k.cov ? k.t + hl : k.t, n = wlen / ps;
    const int64_t ne = n, sl = ne + k.h, rows = R * sl, l = k.t / ps, nt = k.groups * k.v;
    const float eps = (float)c.layer_norm_epsilon;
    const int A16 = out_mode_for(w.act);
    Arena &ws = r.ws;
    ws.reset();
    float *loc = ws.take<float>(R * n), *scl = ws.take<float>(R * n);
    float *kloc = ws.take<float>(R), *kscl = ws.take<float>(R);
    uint8_t *binary = ws.take<uint8_t>(R), *bidir = ws.take<uint8_t>(R);
    uint8_t *kv = ws.take<uint8_t>(R * n);
    int *first_obs = ws.take<int>(k.groups);
    float *feats = ws.take<float>(R * n * 2 * ps);
    float *cs = ws.take<float>(k.groups * sl * 32), *sn = ws.take<float>(k.groups * sl * 32);
    float *x = ws.take<float>(rows * d);
    uint16_t *xn = ws.take<uint16_t>(rows * d);
    uint16_t *qkvg = ws.take<uint16_t>(rows * w.max_qkv_cols);
    uint16_t *o16 = ws.take<uint16_t>(rows * d);
    uint16_t *h16 = ws.take<uint16_t>(rows * std::max<int64_t>(2 * hid, 4 * d));
    uint16_t *a16 = ws.take<uint16_t>(rows * hid);
    int64_t *head_rows = ws.take<int64_t>(nt * k.h);
    int64_t *target_row = ws.take<int64_t>(nt);
    float *hid_hi = ws.take<float>(nt * k.h * d), *hid_lo = ws.take<float>(nt * k.h * d);
    float *hh_hi = ws.take<float>(nt * k.h * 4 * d), *hh_lo = ws.take<float>(nt * k.h * 4 * d);
    float *raw = ws.take<float>(nt * hl * q);
    const bool fused = ts_fused_norm(c, w.act);
    const int np = (int)(d / 256);
    float *nS = fused ? ws.take<float>(rows) : nullptr;       // row factors of the MLP norm
    float *nP = fused ? ws.take<float>(rows * np) : nullptr;  // row sums of squares per column tile
    // Corrected products: FP8 companions of the GEMM inputs, and the attention output in FP32 (its
    // FP16 value and companion are formed after the output gate).
    uint8_t *xn8 = w.corr ? ws.take<uint8_t>(rows * 2 * d) : nullptr;
    uint8_t *o8 = w.corr ? ws.take<uint8_t>(rows * 2 * d) : nullptr;
    float *o32 = w.corr ? ws.take<float>(rows * d) : nullptr;
    uint8_t *a8 = w.corr ? ws.take<uint8_t>(rows * 2 * hid) : nullptr;
    uint8_t *h8 = w.corr ? ws.take<uint8_t>(R * n * 2 * 4 * d) : nullptr;
    if (ws.used > ws.buf.bytes) return Status::fail(TSFM_ERR_OUT_OF_MEMORY, "Timestral: workspace too small");

    // 1. statistics, features, key validity, first observed patch.
    TSFM_CUDA(cudaMemsetAsync(first_obs, 0x7f, k.groups * sizeof(int), s), "timestral: first_obs");
    {
        TsStatsCall sc;
        sc.ctx = ctx;
        sc.obs = obs;
        sc.t = k.t;
        sc.kf = kf;
        sc.kfm = kfm;
        sc.kf_ld = kf_ld;
        sc.hl = hl;
        sc.cov = k.cov;
        sc.rows = R;
        sc.ps = (int)ps;
        sc.vall = (int)k.vall;
        sc.roles = w.roles;
        sc.min_scale = c.minimum_scale;
        sc.use_asinh = c.use_arcsinh;
        sc.attend_missing = c.attend_missing_patches;
        sc.loc = loc;
        sc.scale = scl;
        sc.kloc = kloc;
        sc.kscale = kscl;
        sc.binary = binary;
        sc.key_valid = kv;
        sc.first_obs = first_obs;
        LaunchScope ls(r, s, K_PATCH, (double)R * wlen * 5 * 2);
        TSFM_TRY(launch_ts_stats(sc, feats, s));
    }
    // 2. patch embedding into the encoder rows; forecast queries into the decoder rows.
    {
        const int64_t m = R * n;
        LinearCall hx;
        hx.y8 = h8;
        hx.ldy8 = 8 * d;
        TSFM_TRY(op_linear(r, s, w.patch_proj.hidden, feats, m, 2 * ps, h16, 4 * d, A16, 2, &hx));
        LinearCall remap;
        remap.rm_g = n;
        remap.rm_G = sl;
        TSFM_TRY(op_linear(r, s, w.patch_proj.residual, feats, m, 2 * ps, x, d, OUT_F32, 0, &remap));
        remap.x8 = h8;
        remap.ldx8 = 8 * d;
        TSFM_TRY(op_linear(r, s, w.patch_proj.output, h16, m, 4 * d, x, d, OUT_F32_ACC, 0, &remap));
        LaunchScope ls(r, s, K_OTHER, (double)R * k.h * d * 8);
        TSFM_TRY(launch_broadcast_rows(x, R, sl, ne, w.fq_rep, k.h, d, s));
    }
    // 3. RoPE tables relative to each group's first observed patch; per-row attention flags;
    //    head row indices.
    {
        LaunchScope ls(r, s, K_OTHER, (double)k.groups * sl * 32 * 8);
        TSFM_TRY(launch_ts_rope(first_obs, k.groups, sl, ne, l, w.inv_freq, 32, cs, sn, s));
    }
    {
        LaunchScope ls(r, s, K_OTHER, (double)R + (double)nt * (k.h + 1) * 8);
        TSFM_TRY(launch_ts_rows(w.roles, R, (int)k.vall, (int)k.v, sl, ne, (int)k.h, k.cov, bidir, head_rows,
                                target_row, s));
    }
    // 4. transformer (runTransformer, timestral/model.zig:434-482).
    for (size_t li = 0; li < w.layers.size(); ++li) {
        const TsDev::Layer &L = w.layers[li];
        for (int ai = 0; ai < L.n_attn; ++ai) {
            const TsDev::Attn &a = L.attns[ai];
            const int64_t cols = a.qkvg.out;
            const bool pre = fused && li > 0 && ai == 0;  // xn holds the previous w3's fused norm input
            if (!pre) TSFM_TRY(op_rmsnorm(r, s, x, a.norm, xn, A16, rows, d, eps, 0, 0, 0, nullptr, xn8));
            LinearCall rope;
            rope.x8 = xn8;
            rope.ldx8 = 2 * d;
            if (pre) {
                rope.norm_in = nP;
                rope.norm_parts = np;
                rope.norm_dim = d;
                rope.norm_eps = eps;
                rope.norm_s_in = nS;
            }
            if (a.is_time) {
                rope.rope_cos = cs;
                rope.rope_sin = sn;
                rope.rope_cols = (int)(2 * d);
                rope.rope_p1 = sl * k.vall;
                rope.rope_p2 = sl;
            }
            TSFM_TRY(op_linear(r, s, a.qkvg, xn, rows, d, qkvg, cols, A16, 0, &rope));
            if (a.is_time) {
                AttentionCall ac;
                ac.err = static_cast<int *>(r.err.p);
                ac.q = qkvg;
                ac.k = qkvg + d;
                ac.v = qkvg + 2 * d;
                ac.dtype = w.act;
                ac.ld_qkv = cols;
                ac.o = o16;
                ac.ld_o = d;
                ac.key_valid = kv;
                ac.kv_stride = ne;
                ac.groups = (int)R;
                ac.heads = (int)nh;
                ac.n = (int)sl;
                ac.scale = 1.0f / std::sqrt((float)hd_of(c));
                ac.mask_mode = 1;
                ac.ne = (int)ne;
                ac.l = (int)l;
                ac.group_bidir = bidir;
                ac.o32 = o32;  // corrected products: FP32 output, gated below
                ac.ld_o32 = d;
                LaunchScope ls(r, s, K_ATTN, 2.0 * (double)R * nh * sl * sl * 64);
                TSFM_TRY(launch_attention(ac, s));
            } else {
                TsVariateCall vc;
                vc.qkv = qkvg;
                vc.ld = cols;
                vc.d = d;
                vc.o = o16;
                vc.ldo = d;
                vc.dtype = w.act;
                vc.groups = k.groups;
                vc.sl = sl;
                vc.ne = ne;
                vc.vall = (int)k.vall;
                vc.heads = (int)nh;
                vc.key_valid = kv;
                vc.roles = w.roles;
                vc.cov = k.cov;
                vc.scale = 1.0f / std::sqrt((float)hd_of(c));
                if (w.corr) {  // FP32 output, gated below
                    vc.o32 = o32;
                    vc.ld_o32 = d;
                } else if (a.gate) {  // applied as the output is written
                    vc.gate = qkvg + 3 * d;
                    vc.ldg = cols;
                }
                LaunchScope ls(r, s, K_ATTN, 4.0 * (double)k.groups * sl * nh * k.vall * k.vall * 64);
                TSFM_TRY(launch_ts_variate(vc, s));
            }
            if (w.corr) {
                LaunchScope ls(r, s, K_OTHER, (double)rows * d * 10);
                TSFM_TRY(launch_ts_gate_x8(o32, d, a.gate ? qkvg + 3 * d : nullptr, cols, rows, d, o16, d, o8, 2 * d, s));
            } else if (a.gate && a.is_time) {
                LaunchScope ls(r, s, K_OTHER, (double)rows * d * 6);
                TSFM_TRY(launch_ts_gate(o16, d, qkvg + 3 * d, cols, rows, d, w.act, s));
            }
            LinearCall oc;
            oc.x8 = o8;
            oc.ldx8 = 2 * d;
            TSFM_TRY(op_linear(r, s, a.o, o16, rows, d, x, d, OUT_F32_ACC, 0, &oc));
        }
        const bool next = fused && li + 1 < w.layers.size();
        TSFM_TRY(op_rmsnorm(r, s, x, L.mlp_norm, xn, A16, rows, d, eps, 0, 0, 0, next ? nS : nullptr, xn8));
        if (L.glu) {
            LinearCall gc;
            gc.x8 = xn8;
            gc.ldx8 = 2 * d;
            gc.y8 = a8;
            gc.ldy8 = 2 * hid;
            TSFM_TRY(op_linear(r, s, L.w12, xn, rows, d, a16, hid, A16, ACT_GLU, &gc));
        } else {
            TSFM_TRY(op_linear(r, s, L.w12, xn, rows, d, h16, 2 * hid, A16, 0));
            LaunchScope ls(r, s, K_OTHER, (double)rows * hid * 6);
            TSFM_TRY(launch_ts_swiglu(h16, a16, rows, hid, w.act, s));
        }
        LinearCall wc;
        wc.x8 = a8;
        wc.ldx8 = 2 * hid;
        if (next) {
            wc.norm_out = nP;
            wc.norm_x16 = xn;
            wc.ld_x16 = d;
            wc.norm_gamma = w.layers[li + 1].attns[0].norm;
            wc.norm_s_in = nS;
            wc.norm_x8 = xn8;
            wc.ld_nx8 = 2 * d;
        }
        TSFM_TRY(op_linear(r, s, L.w3, a16, rows, hid, x, d, OUT_F32_ACC, 0, &wc));
    }
    // 5. out_norm on the target rows' decoder tokens, FP32-accurate head, monotone quantiles.
    const int64_t mh = nt * k.h;
    {
        RmsNormCall rc;
        rc.x = x;
        rc.scale = w.out_norm;
        rc.out = hid_hi;
        rc.out_mode = OUT_F32;
        rc.rows = mh;
        rc.dim = d;
        rc.eps = eps;
        rc.rows_idx = head_rows;
        LaunchScope ls(r, s, K_NORM, (double)mh * d * 8);
        TSFM_TRY(launch_rmsnorm(rc, s));
    }
    TSFM_TRY(op_split(r, s, hid_hi, hid_lo, mh, d, d));
    TSFM_TRY(op_linear3(r, s, w.head_hidden, hid_hi, hid_lo, mh, d, hh_hi, 4 * d, false, 2));
    TSFM_TRY(op_split(r, s, hh_hi, hh_lo, mh, 4 * d, 4 * d));
    TSFM_TRY(op_linear3(r, s, w.head_residual, hid_hi, hid_lo, mh, d, raw, ps * q, false, 0));
    TSFM_TRY(op_linear3(r, s, w.head_output, hh_hi, hh_lo, mh, 4 * d, raw, ps * q, true, 0));
    TsHeadCall hc;
    hc.raw = raw;
    hc.out = qs;
    hc.loc = loc;
    hc.scale = scl;
    hc.target_row = target_row;
    hc.nt = nt;
    hc.hl = hl;
    hc.n = n;
    hc.l = l;
    hc.q = (int)q;
    hc.m = median_index(c);
    hc.widths = w.widths;
    hc.wf = (float)c.quantile_width_factor;
    hc.use_asinh = c.use_arcsinh;
    LaunchScope ls(r, s, K_HEAD, (double)nt * hl * q * 8);
    return launch_ts_head(hc, s);
}

Status load_norm(Replica &r, const TensorTable &t, const std::string &name, int64_t d, float **dst) {
    std::vector<float> v;
    TSFM_TRY(t.get(name, d, v));
    return upload_f32(r, v, dst);
}

}  // namespace

Status ts_validate(const tsfm_config &c) {
    // timestral/config.zig:74-85
    if (c.num_heads <= 0 || c.d_model % c.num_heads) return Status::fail(TSFM_ERR_INVALID_CONFIG, "InvalidConfig: d_model % num_heads");
    const int64_t rd = rope_dim(c);
    if (rd == 0 || rd % 2) return Status::fail(TSFM_ERR_INVALID_CONFIG, "InvalidConfig: rope dim");
    if (c.n_layer_kinds <= 0 || !c.layer_kinds) return Status::fail(TSFM_ERR_INVALID_CONFIG, "InvalidConfig: block_schedule");
    for (int i = 0; i < c.n_layer_kinds; ++i)
        if (c.layer_kinds[i] < 0 || c.layer_kinds[i] > 3) return Status::fail(TSFM_ERR_INVALID_CONFIG, "UnknownLayerKind");
    if (c.num_quantiles <= 0 || !c.quantiles) return Status::fail(TSFM_ERR_INVALID_CONFIG, "InvalidConfig: quantile knots");
    bool median = false;
    for (int i = 0; i < c.num_quantiles; ++i) {
        median = median || c.quantiles[i] == 0.5;
        if (i > 0 && !(c.quantiles[i - 1] < c.quantiles[i])) return Status::fail(TSFM_ERR_INVALID_CONFIG, "InvalidConfig: quantile knots");
    }
    if (!median) return Status::fail(TSFM_ERR_INVALID_CONFIG, "InvalidConfig: no 0.5 knot");
    if (c.patch_size <= 0 || c.block_size <= 0 || c.context_length <= 0 || c.d_ff <= 0)
        return Status::fail(TSFM_ERR_INVALID_CONFIG, "InvalidConfig: sizes");
    // Kernel constraints of this backend.
    if (hd_of(c) != 64) return Status::fail(TSFM_ERR_UNSUPPORTED, "Timestral: head width must be 64");
    if (c.d_model % 64 || c.d_ff % 8 || (2 * c.patch_size) % 4 || ((int64_t)c.patch_size * c.num_quantiles) % 4)
        return Status::fail(TSFM_ERR_UNSUPPORTED, "Timestral: dimensions must keep 16-byte rows");
    if (c.num_quantiles > 32) return Status::fail(TSFM_ERR_UNSUPPORTED, "Timestral: at most 32 quantiles");
    return Status::ok();
}

Status ts_check_tensors(const tsfm_config &c, const TensorTable &t) {
    const int64_t d = c.d_model, ps = c.patch_size, hid = c.d_ff, q = c.num_quantiles;
    TSFM_TRY(check_resblock(t, "representation.patch_proj", 2 * ps, 4 * d, d, true));
    TSFM_TRY(t.check("representation.forecast_query", d));
    TSFM_TRY(check_resblock(t, "head.projection", d, 4 * d, ps * q, false));
    TSFM_TRY(t.check("transformer.out_norm.scale", d));
    for (int li = 0; li < c.n_layer_kinds; ++li) {
        bool it[2];
        const int na = layer_axes(c.layer_kinds[li], it);
        for (int ai = 0; ai < na; ++ai) {
            TSFM_TRY(t.check(strf("transformer.layers.%d.attn_norms.%d.scale", li, ai), d));
            TSFM_TRY(t.check(strf("transformer.layers.%d.attns.%d.wQKV.weight", li, ai), 3 * d * d));
            TSFM_TRY(t.check(strf("transformer.layers.%d.attns.%d.wO.weight", li, ai), d * d));
            if (it[ai] ? c.time_attn_gate : c.variate_attn_gate)
                TSFM_TRY(t.check(strf("transformer.layers.%d.attns.%d._gate.weight", li, ai), d * d));
        }
        TSFM_TRY(t.check(strf("transformer.layers.%d.mlp_norm.scale", li), d));
        TSFM_TRY(t.check(strf("transformer.layers.%d.mlp.w12.weight", li), 2 * hid * d));
        TSFM_TRY(t.check(strf("transformer.layers.%d.mlp.w3.weight", li), d * hid));
    }
    return Status::ok();
}

Status ts_load(Replica &r, const tsfm_config &c, const TensorTable &t, int act, TsDev &w) {
    const int64_t d = c.d_model, ps = c.patch_size, hid = c.d_ff, q = c.num_quantiles, nh = c.num_heads, hd = hd_of(c);
    // act: the 16-bit weights' upload type; E_F16C = FP16 weights with FP8 correction companions.
    w.corr = act == E_F16C;
    w.act = w.corr ? E_F16 : act;
    TSFM_TRY(load_resblock(r, t, "representation.patch_proj", 2 * ps, 4 * d, d, true, E_F32, act, w.patch_proj));
    std::vector<float> v;
    TSFM_TRY(t.get("representation.forecast_query", d, v));
    std::vector<float> rep;
    for (int i = 0; i < c.block_size; ++i) rep.insert(rep.end(), v.begin(), v.end());
    TSFM_TRY(upload_f32(r, rep, &w.fq_rep));
    TSFM_TRY(t.get("head.projection.hidden_layer.weight", 4 * d * d, v));
    TSFM_TRY(upload_lin3(r, v, 4 * d, d, w.head_hidden));
    TSFM_TRY(t.get("head.projection.output_layer.weight", ps * q * 4 * d, v));
    TSFM_TRY(upload_lin3(r, v, ps * q, 4 * d, w.head_output));
    TSFM_TRY(t.get("head.projection.residual_layer.weight", ps * q * d, v));
    TSFM_TRY(upload_lin3(r, v, ps * q, d, w.head_residual));
    TSFM_TRY(load_norm(r, t, "transformer.out_norm.scale", d, &w.out_norm));
    w.max_qkv_cols = 3 * d;
    for (int li = 0; li < c.n_layer_kinds; ++li) {
        TsDev::Layer L;
        bool it[2];
        L.n_attn = layer_axes(c.layer_kinds[li], it);
        for (int ai = 0; ai < L.n_attn; ++ai) {
            TsDev::Attn &a = L.attns[ai];
            a.is_time = it[ai];
            a.gate = (it[ai] ? c.time_attn_gate : c.variate_attn_gate) != 0;
            TSFM_TRY(load_norm(r, t, strf("transformer.layers.%d.attn_norms.%d.scale", li, ai), d, &a.norm));
            std::vector<const tsfm_tensor *> parts(1);
            TSFM_TRY(t.raw(strf("transformer.layers.%d.attns.%d.wQKV.weight", li, ai), 3 * d * d, &parts[0]));
            // permuteQkv (timestral/model.zig:72-85): rows (qkv, head_dim, heads) -> (qkv, head, head_dim).
            std::vector<int32_t> map((size_t)(3 * d));
            for (int64_t sel = 0; sel < 3; ++sel)
                for (int64_t h = 0; h < nh; ++h)
                    for (int64_t dd = 0; dd < hd; ++dd)
                        map[(size_t)((sel * nh + h) * hd + dd)] = (int32_t)(sel * d + dd * nh + h);
            if (a.gate) {
                // One GEMM yields [q | k | v | gate].
                parts.resize(2);
                TSFM_TRY(t.raw(strf("transformer.layers.%d.attns.%d._gate.weight", li, ai), d * d, &parts[1]));
                for (int64_t i = 0; i < d; ++i) map.push_back((int32_t)(3 * d + i));
            }
            const int64_t cols = (int64_t)map.size();
            w.max_qkv_cols = std::max(w.max_qkv_cols, cols);
            TSFM_TRY(upload_lin_raw(r, parts, &map, cols, d, act, a.qkvg));
            const tsfm_tensor *to;
            TSFM_TRY(t.raw(strf("transformer.layers.%d.attns.%d.wO.weight", li, ai), d * d, &to));
            TSFM_TRY(upload_lin_raw(r, {to}, nullptr, d, d, act, a.o));
        }
        TSFM_TRY(load_norm(r, t, strf("transformer.layers.%d.mlp_norm.scale", li), d, &L.mlp_norm));
        const tsfm_tensor *t12, *t3;
        TSFM_TRY(t.raw(strf("transformer.layers.%d.mlp.w12.weight", li), 2 * hid * d, &t12));
        TSFM_TRY(t.raw(strf("transformer.layers.%d.mlp.w3.weight", li), d * hid, &t3));
        if (hid % 128 == 0) {
            // [gate | up] per 128-unit block, so one GEMM tile holds matching gate and up columns
            // and its epilogue writes gate * silu(up) (MlpAct.run, timestral/model.zig:159-165).
            std::vector<int32_t> map((size_t)(2 * hid));
            for (int64_t blk = 0; blk < hid / 128; ++blk)
                for (int64_t i = 0; i < 128; ++i) {
                    map[(size_t)(blk * 256 + i)] = (int32_t)(blk * 128 + i);
                    map[(size_t)(blk * 256 + 128 + i)] = (int32_t)(hid + blk * 128 + i);
                }
            TSFM_TRY(upload_lin_raw(r, {t12}, &map, 2 * hid, d, act, L.w12));
            L.glu = true;
        } else {
            if (w.corr)
                return Status::fail(TSFM_ERR_UNSUPPORTED, "TSFM_COMPUTE_F16C: Timestral needs mlp_hidden_dim % 128 == 0");
            TSFM_TRY(upload_lin_raw(r, {t12}, nullptr, 2 * hid, d, act, L.w12));
        }
        TSFM_TRY(upload_lin_raw(r, {t3}, nullptr, d, hid, act, L.w3));
        w.layers.push_back(L);
    }
    // inv_freq with zeros past rope_dim / 2 (identity rotation) (timestral/model.zig:180-188).
    const int64_t rd = rope_dim(c);
    std::vector<float> inv(hd / 2, 0.0f);
    const float base = (float)c.rope_theta;
    for (int64_t i = 0; i < rd / 2; ++i) inv[i] = 1.0f / std::pow(base, (float)(2 * i) / (float)rd);
    TSFM_TRY(upload_f32(r, inv, &w.inv_freq));
    // Quantile widths of the monotone head (timestral/model.zig:510-514).
    const int m = median_index(c);
    std::vector<float> widths(q, 0.0f);
    for (int i = m + 1; i < q; ++i) widths[i] = (float)(c.quantiles[i] - c.quantiles[i - 1]);
    for (int i = 0; i < m; ++i) widths[i] = (float)(c.quantiles[i + 1] - c.quantiles[i]);
    TSFM_TRY(upload_f32(r, widths, &w.widths));
    return Status::ok();
}

// forecaster.forecast (timestral/forecaster.zig:57-180) for b series on one replica; all arrays
// are host memory, `out` is (b, v, horizon, q).
Status ts_forecast(Replica &r, const tsfm_config &c, TsDev &w, const float *inputs, const uint8_t *observed, size_t b,
                   size_t v, size_t t0, size_t horizon, const tsfm_covariates *covp, const tsfm_timestral_options &opts,
                   float *out) {
    const int64_t q = c.num_quantiles, ps = c.patch_size;
    tsfm_timestral_options o = opts;
    if (o.max_context == 0) o.max_context = (size_t)c.context_length;
    o.per_shot_horizon_patches = std::min<size_t>(std::max<size_t>(o.per_shot_horizon_patches, 1), (size_t)c.block_size);
    tsfm_covariates cov{};
    if (covp) cov = *covp;
    const bool any_cov = cov.past || cov.known || cov.cat_past || cov.cat_known;
    if (any_cov && !c.covariate_enabled) return Status::fail(TSFM_ERR_COVARIATES_UNSUPPORTED, "CovariatesUnsupported");
    if ((cov.known || cov.cat_known) && !supports_known(c))
        return Status::fail(TSFM_ERR_COVARIATES_UNSUPPORTED, "KnownCovariatesUnsupported");

    // Covariate channels of a series: numeric past / known first, then the categorical ones (target-
    // encoded on the device against a univariate target, else rounded; forecaster.zig:92-103).
    const bool have_target = (cov.cat_past || cov.cat_known) && v == 1;
    const size_t np = cov.past ? cov.n_past : 0, nk = cov.known ? cov.n_known : 0;
    const size_t ncp = cov.cat_past ? cov.n_cat_past : 0, nck = cov.cat_known ? cov.n_cat_known : 0;
    const size_t n_past = np + ncp, n_known = nk + nck;
    if (n_past == 0 && n_known == 0 && any_cov) return Status::fail(TSFM_ERR_INVALID_ARGUMENT, "InvalidInput");
    if (o.symmetric_averaging)
        for (int64_t i = 0; i < q; ++i)
            if (std::fabs(c.quantiles[i] + c.quantiles[q - 1 - i] - 1.0) > 1e-9)
                return Status::fail(TSFM_ERR_ASYMMETRIC_QUANTILES, "AsymmetricQuantiles");

    // forecastRaw input preparation for the forward pass and, batched after it, the mirrored pass.
    const size_t vall = v + n_past + n_known;
    const size_t keep = std::min(t0, o.max_context);
    const size_t t = (keep + ps - 1) / ps * ps;
    const size_t hpad = (horizon + ps - 1) / ps * ps;
    const int passes = o.symmetric_averaging ? 2 : 1;
    const int64_t groups = (int64_t)b * passes, R = groups * (int64_t)vall;
    // Roles of one series' rows: targets, past-only, known-future.
    std::vector<int8_t> roles(vall);
    for (size_t i = 0; i < vall; ++i) roles[i] = i < v ? 0 : (i < v + n_past ? 1 : 2);
    const bool covw = vall > v;
    const int64_t nt = groups * (int64_t)v;
    const int med = median_index(c);

    // Device buffers that live across blocks.
    const int64_t max_t = std::max<int64_t>((int64_t)t, (int64_t)std::max<size_t>(ps, o.max_context / ps * ps)) + hpad;
    size_t fc_bytes = Arena::span(R * t * 4) + Arena::span(R * t) + 2 * Arena::span(R * max_t * 4) +
                      2 * Arena::span(R * max_t) + Arena::span(R * hpad * 4) + Arena::span(R * hpad) +
                      Arena::span(nt * horizon * q * 4) * 2 + Arena::span(nt * o.per_shot_horizon_patches * ps * q * 4) +
                      Arena::span(b * v) + Arena::span(vall) + Arena::span(16) + Arena::span(b * v * t0 * 4) +
                      Arena::span(b * v * t0) + Arena::span(b * n_past * t0 * 4) +
                      Arena::span(b * n_known * (t0 + horizon) * 4) + Arena::span(b * ncp * t0 * 8) +
                      Arena::span(b * nck * (t0 + horizon) * 8) + (have_target ? Arena::span(b * t0 * 8) : 0);
    TSFM_TRY(r.fc.reserve(fc_bytes));
    Arena &fc = r.fc;
    fc.reset();
    float *d_rows0 = fc.take<float>(R * t);
    uint8_t *d_mask0 = fc.take<uint8_t>(R * t);
    float *ctx_a = fc.take<float>(R * max_t), *ctx_b = fc.take<float>(R * max_t);
    uint8_t *msk_a = fc.take<uint8_t>(R * max_t), *msk_b = fc.take<uint8_t>(R * max_t);
    float *d_kf = fc.take<float>(R * hpad);
    uint8_t *d_kfm = fc.take<uint8_t>(R * hpad);
    float *d_raw = fc.take<float>(nt * horizon * q);
    float *d_out = fc.take<float>(nt * horizon * q);
    float *d_qs = fc.take<float>(nt * (int64_t)o.per_shot_horizon_patches * ps * q);
    uint8_t *d_clip = fc.take<uint8_t>(b * v);
    int8_t *d_roles = fc.take<int8_t>(vall);
    int *d_nan = fc.take<int>(4);
    float *d_in = fc.take<float>(b * v * t0);
    uint8_t *d_obs = fc.take<uint8_t>(b * v * t0);
    float *d_past = fc.take<float>(b * n_past * t0);
    float *d_known = fc.take<float>(b * n_known * (t0 + horizon));
    double *d_cat_past = fc.take<double>(b * ncp * t0);
    double *d_cat_known = fc.take<double>(b * nck * (t0 + horizon));
    double *d_target = have_target ? fc.take<double>(b * t0) : nullptr;
    if (fc.used > fc.buf.bytes) return Status::fail(TSFM_ERR_OUT_OF_MEMORY, "Timestral: forecaster buffers too small");
    cudaStream_t s = r.stream;
    // The raw arrays go up once; the rows (both passes), masks, known futures and clip flags are
    // built on the device.
    TSFM_CUDA(cudaMemcpyAsync(d_in, inputs, b * v * t0 * 4, cudaMemcpyHostToDevice, s), "timestral: inputs");
    TSFM_CUDA(cudaMemcpyAsync(d_obs, observed, b * v * t0, cudaMemcpyHostToDevice, s), "timestral: observed");
    const size_t kl = t0 + horizon;
    if (np)
        TSFM_CUDA(cudaMemcpy2DAsync(d_past, n_past * t0 * 4, cov.past, np * t0 * 4, np * t0 * 4, b,
                                    cudaMemcpyHostToDevice, s),
                  "timestral: past covariates");
    if (nk)
        TSFM_CUDA(cudaMemcpy2DAsync(d_known, n_known * kl * 4, cov.known, nk * kl * 4, nk * kl * 4, b,
                                    cudaMemcpyHostToDevice, s),
                  "timestral: known covariates");
    if (ncp)
        TSFM_CUDA(cudaMemcpyAsync(d_cat_past, cov.cat_past, b * ncp * t0 * 8, cudaMemcpyHostToDevice, s),
                  "timestral: categorical past covariates");
    if (nck)
        TSFM_CUDA(cudaMemcpyAsync(d_cat_known, cov.cat_known, b * nck * kl * 8, cudaMemcpyHostToDevice, s),
                  "timestral: categorical known covariates");
    if (ncp || nck) {
        LaunchScope ls(r, s, K_PATCH, (double)b * (ncp + nck) * t0 * kl);
        if (have_target) TSFM_TRY(launch_ts_target(d_in, d_obs, (int64_t)b, (int64_t)t0, (int64_t)o.max_context, d_target, s));
        TSFM_TRY(launch_ts_cat_encode(d_cat_past, (int64_t)b, (int64_t)ncp, (int64_t)t0, (int64_t)t0, d_target, d_past,
                                      (int64_t)n_past, (int64_t)np, s));
        TSFM_TRY(launch_ts_cat_encode(d_cat_known, (int64_t)b, (int64_t)nck, (int64_t)kl, (int64_t)t0, d_target,
                                      d_known, (int64_t)n_known, (int64_t)nk, s));
    }
    TSFM_CUDA(cudaMemcpyAsync(d_roles, roles.data(), vall, cudaMemcpyHostToDevice, s), "timestral: roles");
    {
        TsPrepareCall pc;
        pc.inputs = d_in;
        pc.observed = d_obs;
        pc.past = n_past ? d_past : nullptr;
        pc.known = n_known ? d_known : nullptr;
        pc.b = (int64_t)b;
        pc.v = (int64_t)v;
        pc.n_past = (int64_t)n_past;
        pc.n_known = (int64_t)n_known;
        pc.t0 = (int64_t)t0;
        pc.horizon = (int64_t)horizon;
        pc.keep = (int64_t)keep;
        pc.t = (int64_t)t;
        pc.hpad = (int64_t)hpad;
        pc.passes = passes;
        pc.rows = d_rows0;
        pc.rows2 = ctx_a;
        pc.mask = d_mask0;
        pc.mask2 = msk_a;
        pc.kf = d_kf;
        pc.kfm = d_kfm;
        pc.clip = o.clip_nonnegative ? d_clip : nullptr;
        LaunchScope ls(r, s, K_PATCH, (double)R * t * 10);
        TSFM_TRY(launch_ts_prepare(pc, s));
    }
    TSFM_CUDA(cudaMemsetAsync(d_nan, 0, 16, s), "timestral: nan flag");
    w.roles = d_roles;

    // blockDecode (timestral/forecaster.zig:423-563), groups chunked by the workspace budget.
    int64_t tcur = (int64_t)t;
    float *ctx = ctx_a, *nctx = ctx_b;
    uint8_t *cm = msk_a, *nm = msk_b;
    int64_t remaining = (int64_t)(horizon + ps - 1) / ps, done = 0;
    const bool known_any = n_known > 0;
    while (remaining > 0) {
        const int64_t block = std::min<int64_t>((int64_t)o.per_shot_horizon_patches, remaining), blen = block * ps;
        Block k{groups, (int64_t)vall, (int64_t)v, tcur, block, ps, covw};
        const size_t per_group = block_workspace(c, w, Block{1, (int64_t)vall, (int64_t)v, tcur, block, ps, covw});
        int64_t chunk = std::max<int64_t>(1, std::min<int64_t>(groups, (int64_t)(workspace_budget(r) / std::max<size_t>(per_group, 1))));
        const int64_t nchunks = (groups + chunk - 1) / chunk;
        chunk = (groups + nchunks - 1) / nchunks;
        Block kc = k;
        kc.groups = chunk;
        TSFM_TRY(r.ws.reserve(block_workspace(c, w, kc)));
        for (int64_t g0 = 0; g0 < groups; g0 += chunk) {
            Block kk = k;
            kk.groups = std::min(chunk, groups - g0);
            const int64_t r0 = g0 * (int64_t)vall;
            TSFM_TRY(predict_block(r, c, w, kk, ctx + r0 * tcur, cm + r0 * tcur, known_any ? d_kf + r0 * hpad + done : nullptr,
                                   known_any ? d_kfm + r0 * hpad + done : nullptr, (int64_t)hpad,
                                   d_qs + g0 * (int64_t)v * blen * q, s));
        }
        if (block > 1) {
            TsRefineCall rc;
            rc.qs = d_qs;
            rc.ctx = ctx;
            rc.mask = cm;
            rc.t = tcur;
            rc.groups = groups;
            rc.vall = (int)vall;
            rc.v = (int)v;
            rc.ps = (int)ps;
            rc.h = (int)block;
            rc.q = (int)q;
            rc.med = med;
            rc.min_scale = c.minimum_scale;
            LaunchScope ls(r, s, K_HEAD, (double)nt * tcur * 8);
            TSFM_TRY(launch_ts_refine(rc, s));
        }
        {
            LaunchScope ls(r, s, K_OTHER, (double)nt * blen * q * 8);
            TSFM_TRY(launch_ts_store(d_qs, d_raw, nt, blen, (int)q, (int64_t)horizon, done, s));
        }
        remaining -= block;
        done += blen;
        if (remaining == 0) break;
        const int64_t nt_len = tcur + blen;
        const int64_t keep_t = nt_len > (int64_t)o.max_context
                                   ? std::max<int64_t>(ps, (int64_t)o.max_context / ps * ps)
                                   : nt_len;
        if (keep_t > max_t) return Status::fail(TSFM_ERR_INVALID_ARGUMENT, "Timestral: context buffer too small");
        TsFeedbackCall fb;
        fb.ctx = ctx;
        fb.mask = cm;
        fb.t = tcur;
        fb.rows = R;
        fb.keep_t = keep_t;
        fb.blen = blen;
        fb.qs = d_qs;
        fb.q = (int)q;
        fb.med = med;
        fb.vall = (int)vall;
        fb.v = (int)v;
        fb.roles = d_roles;
        fb.kf = d_kf;
        fb.kfm = d_kfm;
        fb.hpad = (int64_t)hpad;
        fb.done = done - blen;
        fb.extreme = o.extreme_value_threshold;
        fb.nctx = nctx;
        fb.nmask = nm;
        {
            LaunchScope ls(r, s, K_OTHER, (double)R * keep_t * 10);
            TSFM_TRY(launch_ts_feedback(fb, s));
        }
        std::swap(ctx, nctx);
        std::swap(cm, nm);
        tcur = keep_t;
    }
    // Quantile cap + NaN check (forecaster.zig:396-419), then the symmetric average and clip.
    {
        TsCapCall cc;
        cc.out = d_raw;
        cc.rows_ctx = d_rows0;
        cc.mask = d_mask0;
        cc.t = (int64_t)t;
        cc.groups = groups;
        cc.horizon = (int64_t)horizon;
        cc.vall = (int)vall;
        cc.v = (int)v;
        cc.q = (int)q;
        cc.cap_k = o.quantile_real_cap_k;
        cc.min_scale = c.minimum_scale;
        cc.nan_flag = d_nan;
        LaunchScope ls(r, s, K_OTHER, (double)nt * (t * 5 + horizon * q * 8));
        TSFM_TRY(launch_ts_cap(cc, s));
    }
    {
        const int64_t rows_out = (int64_t)(b * v);
        LaunchScope ls(r, s, K_OTHER, (double)rows_out * horizon * q * 12);
        TSFM_TRY(launch_ts_finish(d_raw, passes == 2 ? d_raw + rows_out * horizon * q : nullptr,
                                  o.clip_nonnegative ? d_clip : nullptr, d_out, rows_out, (int64_t)horizon, (int)q, s));
    }
    int nan_flag = 0;
    TSFM_CUDA(cudaMemcpyAsync(&nan_flag, d_nan, 4, cudaMemcpyDeviceToHost, s), "timestral: nan flag");
    TSFM_CUDA(cudaMemcpyAsync(out, d_out, b * v * horizon * q * 4, cudaMemcpyDeviceToHost, s), "timestral: results");
    TSFM_CUDA(cudaStreamSynchronize(s), "timestral");
    if (nan_flag) return Status::fail(TSFM_ERR_DEGENERATE_INPUT, "DegenerateInput: a forecast is NaN");
    return Status::ok();
}

}  // namespace tsfm
