// ORACLE — test infrastructure only (see oracle.h): a CPU restatement of tsfm-zig's forecast path,
// each function citing the reference file:line it follows. Compiled with -ffp-contract=off so FP32
// expressions round in the order they are written, as Zig's strict float mode does.
#include "oracle.h"

#include <omp.h>

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <limits>
#include <map>
#include <memory>
#include <string>
#include <thread>
#include <vector>

namespace oracle {
void matmul_nt_packed(const float *x, const float *wt, float *y, size_t rows, size_t out, size_t in,
                      float alpha);
void emul_matmul(float *y, const float *x, size_t rows, const float *w, size_t out, size_t in, int scheme,
                 bool tf32, bool tf32_round);
float emul_store16(float v, int scheme);
}

namespace {

thread_local std::string g_err;
const float kFloatMax = std::numeric_limits<float>::max();
const float kInf = std::numeric_limits<float>::infinity();

struct Fail {
    int32_t code;
};

// Precision study (oracle_set_operand_emulation, oracle_emul.cpp): when g_emul is non-zero, the
// Chronos-2 forward rounds the operands of its products the way the device's reduced-precision
// tensor-core products consume them. g_emul_scope is set around each product by the caller:
// 0 = not emulated (FP32, e.g. the FP32-accurate head), 1 = TF32 device operands, 2 = 16-bit
// device operands. g_emul_class names the product (0 unnamed, 1 q/k/v, 2 attention output o,
// 3 group v, 4 group o, 5 MLP wi, 6 MLP wo, 7 patch-embedding output); g_emul_by_class[c] >= 0
// overrides the scheme for that class. Off (0) by default: the restatement's own arithmetic is
// the reference's FP32.
int g_emul = 0;
int g_emul_scope = 0;
int g_emul_class = 0;
int g_emul_by_class[8] = {-1, -1, -1, -1, -1, -1, -1, -1};
bool g_emul_tf32_round = false;  // round TF32-operand products in every scheme
struct EmulScope {
    int saved, saved_class;
    explicit EmulScope(int s, int cls = -1) : saved(g_emul_scope), saved_class(g_emul_class) {
        g_emul_scope = s;
        if (cls >= 0) g_emul_class = cls;
    }
    ~EmulScope() {
        g_emul_scope = saved;
        g_emul_class = saved_class;
    }
};
int emul_scheme() {
    const int o = g_emul_by_class[g_emul_class & 7];
    return o >= 0 ? o : g_emul;
}
[[noreturn]] void fail(int32_t code, const std::string &msg) {
    g_err = msg;
    throw Fail{code};
}

// ---------------------------------------------------------------------------------------------
// core/nn.zig
//
// Zig's @max / @min on floats return the other operand when one is NaN; they are restated as
// std::fmax / std::fmin (std::max / std::min would propagate a NaN in the first position), and
// std.math.clamp(v, lo, hi) = @max(lo, @min(v, hi)) as std::fmax(lo, std::fmin(v, hi)).

// A weight matrix [out, in] (host f32) with its transposed copy for the blocked product.
struct Weight {
    std::vector<float> data;
    std::vector<float> wt;
    size_t out = 0, in = 0;
    void init(std::vector<float> d, size_t o, size_t i) {
        data = std::move(d);
        out = o;
        in = i;
        wt.assign(o * i, 0.0f);
        for (size_t r = 0; r < o; ++r)
            for (size_t c = 0; c < i; ++c) wt[c * o + r] = data[r * i + c];
    }
};

// nn.linear (core/nn.zig:270-293): y = x w^T, then bias added per row (linearCols :252-258).
void linear(float *y, const float *x, size_t rows, const Weight &w, const float *bias) {
    if (g_emul != 0 && g_emul_scope != 0 && emul_scheme() != 0)
        oracle::emul_matmul(y, x, rows, w.data.data(), w.out, w.in, emul_scheme(), g_emul_scope == 1,
                            g_emul_tf32_round);
    else
        oracle::matmul_nt_packed(x, w.wt.data(), y, rows, w.out, w.in, 1.0f);
    if (bias)
        for (size_t r = 0; r < rows; ++r)
            for (size_t j = 0; j < w.out; ++j) y[r * w.out + j] += bias[j];
}

// gemmNT for attention scores: C[m, n] = alpha * A[m, k] B[n, k]^T with strides (nn.zig:49-60).
void gemm_nt(float *c, size_t ldc, const float *a, size_t lda, const float *b, size_t ldb, size_t m,
             size_t n, size_t k, float alpha) {
    for (size_t i = 0; i < m; ++i)
        for (size_t j = 0; j < n; ++j) {
            float s = 0.0f;
            for (size_t p = 0; p < k; ++p) s += a[i * lda + p] * b[j * ldb + p];
            c[i * ldc + j] = alpha * s;
        }
}

// gemmNN: C[m, n] = A[m, k] B[k, n] (nn.zig:165-239): rows accumulate over p in order; zero
// coefficients are skipped as the builtin kernel does.
void gemm_nn(float *c, size_t ldc, const float *a, size_t lda, const float *b, size_t ldb, size_t m,
             size_t n, size_t k) {
    for (size_t i = 0; i < m; ++i) {
        float *cr = c + i * ldc;
        for (size_t j = 0; j < n; ++j) cr[j] = 0.0f;
        for (size_t p = 0; p < k; ++p) {
            const float av = a[i * lda + p];
            if (av == 0.0f) continue;
            const float *br = b + p * ldb;
            for (size_t j = 0; j < n; ++j) cr[j] += av * br[j];
        }
    }
}

// expVec (nn.zig:344-359): Cephes expf range reduction + degree-6 polynomial.
float exp_vec(float x_in) {
    float x = std::fmin(std::fmax(x_in, -87.33654f), 88.72284f);
    float fx = std::round(x * 1.44269504088896341f);
    float r = x - fx * 0.693359375f;
    r = r - fx * -2.12194440e-4f;
    float y = 1.9875691500e-4f;
    y = y * r + 1.3981999507e-3f;
    y = y * r + 8.3334519073e-3f;
    y = y * r + 4.1665795894e-2f;
    y = y * r + 1.6666665459e-1f;
    y = y * r + 5.0000001201e-1f;
    y = y * r * r + r + 1.0f;
    const int32_t n = (int32_t)fx;
    uint32_t bits = (uint32_t)(n + 127) << 23;
    float pow2;
    std::memcpy(&pow2, &bits, 4);
    return y * pow2;
}

// nn.softmax (nn.zig:470-505): max-subtract, -inf gets exactly 0, normalise by 1/sum.
void softmax(float *row, size_t n) {
    float mx = -kInf;
    for (size_t i = 0; i < n; ++i) mx = std::fmax(mx, row[i]);
    float sum = 0.0f;
    for (size_t i = 0; i < n; ++i) {
        const float e = row[i] == -kInf ? 0.0f : exp_vec(row[i] - mx);
        row[i] = e;
        sum += e;
    }
    const float inv = 1.0f / sum;
    for (size_t i = 0; i < n; ++i) row[i] *= inv;
}

// nn.rmsNorm (nn.zig:374-396).
void rms_norm(float *out, const float *x, size_t rows, size_t dim, const float *scale, float eps) {
#pragma omp parallel for schedule(static) if (rows >= 256)
    for (long r = 0; r < (long)rows; ++r) {
        const float *xr = x + r * dim;
        float ss = 0.0f;
        for (size_t i = 0; i < dim; ++i) ss += xr[i] * xr[i];
        const float inv = 1.0f / std::sqrt(ss / (float)dim + eps);
        float *o = out + r * dim;
        for (size_t i = 0; i < dim; ++i) o[i] = xr[i] * inv * scale[i];
    }
}

inline float silu_vec(float v) { return v / (1.0f + exp_vec(-v)); }  // siluInPlace (nn.zig:399)
inline float softplus(float x) { return x > 20.0f ? x : std::log1p(std::exp(x)); }  // nn.zig:516

void relu(float *x, size_t n) {
    for (size_t i = 0; i < n; ++i) x[i] = std::fmax(x[i], 0.0f);
}
void add_in_place(float *dst, const float *src, size_t n) {
    for (size_t i = 0; i < n; ++i) dst[i] += src[i];
}

// nn.ropeHalf (nn.zig:448-467).
void rope_half(float *x, const float *cs, const float *sn, size_t half) {
    for (size_t i = 0; i < half; ++i) {
        const float x1 = x[i], x2 = x[half + i];
        x[i] = x1 * cs[i] - x2 * sn[i];
        x[half + i] = x2 * cs[i] + x1 * sn[i];
    }
}

// nn.clampNonfinite (nn.zig:522-563).
void clamp_nonfinite(float *v, size_t n) {
    float hi = -kInf, lo = kInf;
    bool any_inf = false;
    for (size_t i = 0; i < n; ++i) {
        const float x = v[i];
        if (std::isfinite(x)) {
            hi = std::fmax(hi, x);
            lo = std::fmin(lo, x);
        } else if (std::isinf(x)) {
            any_inf = true;
        }
    }
    if (!any_inf) return;
    for (size_t i = 0; i < n; ++i) {
        if (v[i] == kInf) v[i] = hi;
        if (v[i] == -kInf) v[i] = lo;
        if (std::isinf(v[i])) v[i] = 0.0f;
    }
}

// ---------------------------------------------------------------------------------------------
// core/attn.zig

enum Mask { M_FULL = 0, M_KEYS_ADDITIVE = 1, M_CAUSAL = 2, M_CAUSAL_KEYS = 3, M_FULL_KEYS = 4 };

// Mask.pick (attn.zig:24-28).
Mask mask_pick(bool causal, bool all_keys_valid, bool additive) {
    if (all_keys_valid) return causal ? M_CAUSAL : M_FULL;
    if (causal) return M_CAUSAL_KEYS;
    return additive ? M_KEYS_ADDITIVE : M_FULL_KEYS;
}

// maskedSoftmax (attn.zig:35-67).
void masked_softmax(Mask mask, float *scores, size_t n, const uint8_t *key_valid) {
    switch (mask) {
        case M_FULL:
            for (size_t i = 0; i < n; ++i) softmax(scores + i * n, n);
            break;
        case M_KEYS_ADDITIVE:
            for (size_t i = 0; i < n; ++i) {
                float *row = scores + i * n;
                for (size_t j = 0; j < n; ++j)
                    if (!key_valid[j]) row[j] += -kFloatMax;
                softmax(row, n);
            }
            break;
        case M_CAUSAL:
            for (size_t i = 0; i < n; ++i) {
                softmax(scores + i * n, i + 1);
                for (size_t j = i + 1; j < n; ++j) scores[i * n + j] = 0.0f;
            }
            break;
        case M_CAUSAL_KEYS:
        case M_FULL_KEYS:
            for (size_t i = 0; i < n; ++i) {
                float *row = scores + i * n;
                for (size_t j = 0; j < n; ++j) {
                    const bool allowed = j == i || (key_valid[j] && (mask == M_FULL_KEYS || j <= i));
                    if (!allowed) row[j] = -kInf;
                }
                softmax(row, n);
            }
            break;
    }
}

// selfAttend (attn.zig:72-96): scores = scale q k^T (+bias), masked softmax, o = P v.
void self_attend(Mask mask, float *scores, const float *q, const float *k, const float *v, float *o,
                 size_t ldq, size_t ldk, size_t ldv, size_t ldo, size_t n, size_t hd, float scale,
                 const uint8_t *key_valid, const float *bias) {
    gemm_nt(scores, n, q, ldq, k, ldk, n, n, hd, scale);
    if (bias) add_in_place(scores, bias, n * n);
    masked_softmax(mask, scores, n, key_valid);
    if (g_emul != 0 && g_emul_scope == 2)
        for (size_t i = 0; i < n * n; ++i) scores[i] = oracle::emul_store16(scores[i], g_emul);
    gemm_nn(o, ldo, scores, n, v, ldv, n, hd, n);
}

// core/resblock.zig:64-79: output(act(hidden(x))) + residual(x).
struct ResBlock {
    Weight hidden, output, residual;
    std::vector<float> hb, ob, rb;
    bool bias = true;
    bool silu = false;
    // Emulation scopes of the three products (precision study only): input side and output.
    int emul_in = 0, emul_out = 0;
    void forward(float *y, const float *x, size_t rows) const {
        std::vector<float> h(rows * hidden.out);
        {
            EmulScope sc(emul_in);
            linear(h.data(), x, rows, hidden, bias ? hb.data() : nullptr);
        }
        if (silu)
            for (auto &e : h) e = silu_vec(e);
        else
            relu(h.data(), h.size());
        {
            EmulScope sc(emul_out, 7);
            linear(y, h.data(), rows, output, bias ? ob.data() : nullptr);
        }
        std::vector<float> r(rows * output.out);
        {
            EmulScope sc(emul_in);
            linear(r.data(), x, rows, residual, bias ? rb.data() : nullptr);
        }
        add_in_place(y, r.data(), rows * output.out);
    }
};

// ---------------------------------------------------------------------------------------------
// Weight table lookup: core/safetensors.zig:59-97 semantics (missing -> MissingTensor, element
// count -> ShapeMismatch, F16/BF16 converted to F32).

float half_to_float(uint16_t h) {
    const uint32_t sign = (uint32_t)(h & 0x8000) << 16;
    uint32_t exp = (h >> 10) & 0x1f, mant = h & 0x3ff;
    uint32_t bits;
    if (exp == 0) {
        if (mant == 0) {
            bits = sign;
        } else {  // subnormal
            int e = -1;
            do {
                ++e;
                mant <<= 1;
            } while ((mant & 0x400) == 0);
            mant &= 0x3ff;
            bits = sign | ((uint32_t)(127 - 15 - e) << 23) | (mant << 13);
        }
    } else if (exp == 31) {
        bits = sign | 0x7f800000u | (mant << 13);
    } else {
        bits = sign | ((exp + 112) << 23) | (mant << 13);
    }
    float f;
    std::memcpy(&f, &bits, 4);
    return f;
}

struct Table {
    std::map<std::string, const tsfm_tensor *> by_name;
    Table(const tsfm_tensor *t, size_t n) {
        for (size_t i = 0; i < n; ++i) by_name[t[i].name] = &t[i];
    }
    std::vector<float> get(const std::string &name, size_t numel) const {
        auto it = by_name.find(name);
        if (it == by_name.end()) fail(TSFM_ERR_MISSING_TENSOR, "missing tensor: " + name);
        const tsfm_tensor *t = it->second;
        if (t->dtype != TSFM_DTYPE_F32 && t->dtype != TSFM_DTYPE_F16 && t->dtype != TSFM_DTYPE_BF16)
            fail(TSFM_ERR_UNSUPPORTED_DTYPE, "tensor " + name + " has unsupported dtype");
        if (t->numel != numel)
            fail(TSFM_ERR_SHAPE_MISMATCH, "tensor " + name + ": expected " + std::to_string(numel) +
                                              " elements, file has " + std::to_string(t->numel));
        std::vector<float> out(numel);
        if (t->dtype == TSFM_DTYPE_F32) {
            std::memcpy(out.data(), t->data, numel * 4);
        } else {
            const uint16_t *s = (const uint16_t *)t->data;
            for (size_t i = 0; i < numel; ++i) {
                if (t->dtype == TSFM_DTYPE_BF16) {
                    uint32_t bits = (uint32_t)s[i] << 16;
                    std::memcpy(&out[i], &bits, 4);
                } else {
                    out[i] = half_to_float(s[i]);
                }
            }
        }
        return out;
    }
    Weight weight(const std::string &name, size_t out, size_t in) const {
        Weight w;
        w.init(get(name, out * in), out, in);
        return w;
    }
    ResBlock resblock(const std::string &prefix, size_t in, size_t hid, size_t out, bool bias,
                      bool silu) const {
        ResBlock b;
        b.bias = bias;
        b.silu = silu;
        b.hidden = weight(prefix + ".hidden_layer.weight", hid, in);
        b.output = weight(prefix + ".output_layer.weight", out, hid);
        b.residual = weight(prefix + ".residual_layer.weight", out, in);
        if (bias) {
            b.hb = get(prefix + ".hidden_layer.bias", hid);
            b.ob = get(prefix + ".output_layer.bias", out);
            b.rb = get(prefix + ".residual_layer.bias", out);
        }
        return b;
    }
};

std::string fmt(const char *f, int a) {
    char buf[256];
    snprintf(buf, sizeof buf, f, a);
    return buf;
}
std::string fmt2(const char *f, int a, int b) {
    char buf[256];
    snprintf(buf, sizeof buf, f, a, b);
    return buf;
}

// ---------------------------------------------------------------------------------------------
// Chronos-2 (chronos2/model.zig, chronos2/forecaster.zig)

struct C2Attn {
    std::vector<float> norm;
    Weight q, k, v, o;
};
struct C2Layer {
    C2Attn time, group;
    std::vector<float> mlp_norm;
    Weight wi, wo;
};

// runChunk's masked instance norm and context-patch features (chronos2/forecaster.zig:94-143)
// for nb series (row li at inputs + li * stride + start, t steps, left-padded by pad): loc, scale
// (f64 sums, population std, 0 -> 1e-5, all missing -> 0 / 1), features [time, value, mask] per
// patch and each patch's validity (any observed step).
void c2_patch_features(const float *inputs, size_t stride, size_t start, size_t t, size_t pad, size_t n_ctx,
                       size_t ps, float tscale, bool arcsinh, size_t nb, float *loc, float *scale, float *feats,
                       uint8_t *ctx_valid) {
    for (size_t li = 0; li < nb; ++li) {
        const float *row = inputs + li * stride + start;
        double count = 0, sum = 0;
        for (size_t i = 0; i < t; ++i)
            if (!std::isnan(row[i])) {
                count += 1;
                sum += row[i];
            }
        float lo = 0.0f, sc = 1.0f;
        if (count > 0) {
            lo = (float)(sum / count);
            double ss = 0;
            for (size_t i = 0; i < t; ++i)
                if (!std::isnan(row[i])) {
                    const float dv = row[i] - lo;
                    ss += (double)dv * (double)dv;
                }
            sc = (float)std::sqrt(ss / count);
            if (sc == 0.0f) sc = 1e-5f;
        }
        loc[li] = lo;
        scale[li] = sc;
        for (size_t p = 0; p < n_ctx; ++p) {
            bool any = false;
            const size_t base = (li * n_ctx + p) * 3 * ps;
            for (size_t i = 0; i < ps; ++i) {
                const size_t j = p * ps + i;
                const long src = (long)j - (long)pad;
                bool obs = false;
                float val = 0.0f;
                if (src >= 0 && src < (long)t) {
                    const float xv = row[src];
                    if (!std::isnan(xv)) {
                        obs = true;
                        val = (xv - lo) / sc;
                        if (arcsinh) val = std::asinh(val);
                    }
                }
                feats[base + i] = ((float)j - (float)(n_ctx * ps)) / tscale;
                feats[base + ps + i] = val;
                feats[base + 2 * ps + i] = obs ? 1.0f : 0.0f;
                any = any || obs;
            }
            ctx_valid[li * n_ctx + p] = any;
        }
    }
}

struct Chronos2 {
    tsfm_config c{};
    std::vector<double> quantiles;
    ResBlock input_embed, output_embed;
    std::vector<C2Layer> layers;
    std::vector<float> final_norm, reg, inv_freq;

    // Model.load (chronos2/model.zig:77-125).
    void load(const Table &w) {
        const size_t d = c.d_model, ps = c.patch_size, hid = c.d_ff, q = c.num_quantiles;
        input_embed = w.resblock("input_patch_embedding", 3 * ps, hid, d, true, false);
        input_embed.emul_in = 1;   // device: TF32 patch features
        input_embed.emul_out = 2;  // device: 16-bit hidden activations
        output_embed = w.resblock("output_patch_embedding", d, hid, q * ps, true, false);
        final_norm = w.get("encoder.final_layer_norm.weight", d);
        std::vector<float> shared = w.get("shared.weight", 2 * d);
        reg.assign(shared.begin() + d, shared.begin() + 2 * d);
        for (int li = 0; li < c.num_layers; ++li) {
            C2Layer L;
            for (int which = 0; which < 2; ++which) {
                const std::string p = fmt2("encoder.block.%d.layer.%d.", li, which);
                C2Attn a;
                a.norm = w.get(p + "layer_norm.weight", d);
                a.q = w.weight(p + "self_attention.q.weight", d, d);
                a.k = w.weight(p + "self_attention.k.weight", d, d);
                a.v = w.weight(p + "self_attention.v.weight", d, d);
                a.o = w.weight(p + "self_attention.o.weight", d, d);
                (which == 0 ? L.time : L.group) = std::move(a);
            }
            L.mlp_norm = w.get(fmt("encoder.block.%d.layer.2.layer_norm.weight", li), d);
            L.wi = w.weight(fmt("encoder.block.%d.layer.2.mlp.wi.weight", li), hid, d);
            L.wo = w.weight(fmt("encoder.block.%d.layer.2.mlp.wo.weight", li), d, hid);
            layers.push_back(std::move(L));
        }
        const size_t hd = c.d_kv;
        inv_freq.resize(hd / 2);
        const float base = (float)c.rope_theta;
        for (size_t i = 0; i < hd / 2; ++i)
            inv_freq[i] = 1.0f / std::pow(base, (float)(2 * i) / (float)hd);
    }

    // Model.encode (chronos2/model.zig:144-206) with timeAttention :208-262 and
    // groupAttention :265-269; TimeJob.attend :283-308.
    void encode(float *x, const uint8_t *key_valid, size_t b, size_t n_ctx, size_t n_out) const {
        const size_t d = c.d_model, hid = c.d_ff, nh = c.num_heads, hd = c.d_kv, half = hd / 2;
        const size_t seq = n_ctx + 1 + n_out, rows = b * seq;
        const float eps = (float)c.layer_norm_epsilon;
        std::vector<float> xn(rows * d), delta(rows * d), mlp_h(rows * hid), qb(rows * d),
            kb(rows * d), vb(rows * d), ab(rows * d);
        bool all_valid = true;
        for (size_t i = 0; i < b * seq; ++i) all_valid = all_valid && key_valid[i];
        std::vector<float> cos_t(seq * half), sin_t(seq * half);
        for (size_t tok = 0; tok < seq; ++tok)
            for (size_t i = 0; i < half; ++i) {
                const float ang = inv_freq[i] * (float)tok;
                cos_t[tok * half + i] = std::cos(ang);
                sin_t[tok * half + i] = std::sin(ang);
            }
        const Mask mask = mask_pick(false, all_valid, true);
        EmulScope enc_scope(2, 0);  // every encoder product takes 16-bit device operands
        for (const C2Layer &L : layers) {
            rms_norm(xn.data(), x, rows, d, L.time.norm.data(), eps);
            g_emul_class = 1;
            linear(qb.data(), xn.data(), rows, L.time.q, nullptr);
            linear(kb.data(), xn.data(), rows, L.time.k, nullptr);
            linear(vb.data(), xn.data(), rows, L.time.v, nullptr);
            for (size_t r = 0; r < rows; ++r) {
                const size_t tok = r % seq;
                for (size_t h = 0; h < nh; ++h) {
                    rope_half(&qb[r * d + h * hd], &cos_t[tok * half], &sin_t[tok * half], half);
                    rope_half(&kb[r * d + h * hd], &cos_t[tok * half], &sin_t[tok * half], half);
                }
            }
            if (g_emul != 0)  // q, k, v stored in 16 bits on the device
                for (size_t i = 0; i < rows * d; ++i) {
                    qb[i] = oracle::emul_store16(qb[i], g_emul);
                    kb[i] = oracle::emul_store16(kb[i], g_emul);
                    vb[i] = oracle::emul_store16(vb[i], g_emul);
                }
#pragma omp parallel
            {
                std::vector<float> scores(seq * seq);
#pragma omp for schedule(static)
                for (long item = 0; item < (long)(b * nh); ++item) {
                    const size_t r = item / nh, h = item % nh, off = r * seq * d + h * hd;
                    self_attend(mask, scores.data(), &qb[off], &kb[off], &vb[off], &ab[off], d, d, d,
                                d, seq, hd, 1.0f, key_valid + r * seq, nullptr);
                }
            }
            g_emul_class = 2;
            linear(delta.data(), ab.data(), rows, L.time.o, nullptr);
            add_in_place(x, delta.data(), rows * d);

            rms_norm(xn.data(), x, rows, d, L.group.norm.data(), eps);
            g_emul_class = 3;
            linear(vb.data(), xn.data(), rows, L.group.v, nullptr);
            g_emul_class = 4;
            linear(delta.data(), vb.data(), rows, L.group.o, nullptr);
            add_in_place(x, delta.data(), rows * d);

            rms_norm(xn.data(), x, rows, d, L.mlp_norm.data(), eps);
            g_emul_class = 5;
            linear(mlp_h.data(), xn.data(), rows, L.wi, nullptr);
            relu(mlp_h.data(), mlp_h.size());
            g_emul_class = 6;
            linear(delta.data(), mlp_h.data(), rows, L.wo, nullptr);
            add_in_place(x, delta.data(), rows * d);
        }
        rms_norm(x, x, rows, d, final_norm.data(), eps);
    }

    // forecaster.forecast (chronos2/forecaster.zig:14-50) and runChunk :59-204.
    void forecast(const float *inputs, size_t b, size_t t_in, size_t horizon, float *out) const {
        const size_t ps = c.patch_size;
        if (b == 0 || t_in == 0) fail(TSFM_ERR_EMPTY_INPUT, "EmptyInput");
        if (horizon == 0 || horizon > (size_t)c.max_output_patches * ps)
            fail(TSFM_ERR_HORIZON_TOO_LONG, "HorizonTooLong");
        const size_t t = std::min(t_in, (size_t)c.context_length), start = t_in - t;
        const size_t pad = (ps - t % ps) % ps, n_ctx = (t + pad) / ps, n_out = (horizon + ps - 1) / ps;
        const size_t seq = n_ctx + 1 + n_out;
        const size_t budget = 16u * 1024 * 1024, per = std::max<size_t>(1, seq * c.d_model * 24);
        const size_t chunk = std::min(b, std::max<size_t>(1, budget / per));
        for (size_t s0 = 0; s0 < b; s0 += chunk)
            run_chunk(out, inputs, s0, std::min(b, s0 + chunk), t_in, start, t, pad, n_ctx, n_out,
                      horizon);
    }

    void run_chunk(float *out, const float *inputs, size_t s0, size_t s1, size_t stride, size_t start,
                   size_t t, size_t pad, size_t n_ctx, size_t n_out, size_t horizon) const {
        const size_t d = c.d_model, ps = c.patch_size, q = c.num_quantiles;
        const size_t seq = n_ctx + 1 + n_out, nb = s1 - s0;
        const float tscale = (float)c.time_encoding_scale;
        const bool arcsinh = c.use_arcsinh != 0;
        std::vector<float> loc(nb), scale(nb), feats(nb * n_ctx * 3 * ps), fut(nb * n_out * 3 * ps);
        std::vector<uint8_t> ctx_valid(nb * n_ctx);
        c2_patch_features(inputs + s0 * stride, stride, start, t, pad, n_ctx, ps, tscale, arcsinh, nb, loc.data(),
                          scale.data(), feats.data(), ctx_valid.data());
        for (size_t li = 0; li < nb; ++li) {
            for (size_t p = 0; p < n_out; ++p) {
                const size_t base = (li * n_out + p) * 3 * ps;
                for (size_t i = 0; i < ps; ++i) {
                    fut[base + i] = (float)(p * ps + i) / tscale;
                    fut[base + ps + i] = 0.0f;
                    fut[base + 2 * ps + i] = 0.0f;
                }
            }
        }
        std::vector<float> emb(nb * n_ctx * d), fut_emb(nb * n_out * d);
        input_embed.forward(emb.data(), feats.data(), nb * n_ctx);
        input_embed.forward(fut_emb.data(), fut.data(), nb * n_out);
        std::vector<float> x(nb * seq * d);
        std::vector<uint8_t> kv(nb * seq);
        for (size_t li = 0; li < nb; ++li) {
            float *xb = &x[li * seq * d];
            std::memcpy(xb, &emb[li * n_ctx * d], n_ctx * d * 4);
            std::memcpy(xb + n_ctx * d, reg.data(), d * 4);
            std::memcpy(xb + (n_ctx + 1) * d, &fut_emb[li * n_out * d], n_out * d * 4);
            std::memcpy(&kv[li * seq], &ctx_valid[li * n_ctx], n_ctx);
            kv[li * seq + n_ctx] = 1;
            for (size_t p = 0; p < n_out; ++p) kv[li * seq + n_ctx + 1 + p] = 1;
        }
        encode(x.data(), kv.data(), nb, n_ctx, n_out);
        std::vector<float> hidden(nb * n_out * d), raw(nb * n_out * q * ps);
        for (size_t li = 0; li < nb; ++li)
            std::memcpy(&hidden[li * n_out * d], &x[(li * seq + n_ctx + 1) * d], n_out * d * 4);
        output_embed.forward(raw.data(), hidden.data(), nb * n_out);
        for (size_t li = 0; li < nb; ++li) {
            const size_t s = s0 + li;
            for (size_t p = 0; p < n_out; ++p)
                for (size_t i = 0; i < ps; ++i) {
                    const size_t step = p * ps + i;
                    if (step >= horizon) continue;
                    for (size_t qi = 0; qi < q; ++qi) {
                        float v = raw[(li * n_out + p) * q * ps + qi * ps + i];
                        if (arcsinh) v = std::sinh(v);
                        v = v * scale[li] + loc[li];
                        out[(s * horizon + step) * q + qi] = v;
                    }
                }
        }
    }
};

// ---------------------------------------------------------------------------------------------
// Chronos-Bolt (chronos_bolt/model.zig, chronos_bolt/forecaster.zig)

// relativeBucket (chronos_bolt/model.zig:74-85): T5 bidirectional bucket with the float32 log.
size_t relative_bucket(int64_t rel, uint32_t num_buckets, uint32_t max_distance) {
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

// quantileLinear (chronos_bolt/forecaster.zig:83-93), ATen's two-sided lerp.
float quantile_linear(const float *sorted, size_t n, float level) {
    const float rank = level * (float)(n - 1);
    const float lo_f = std::floor(rank);
    const size_t lo = (size_t)lo_f;
    const size_t hi = std::min((size_t)std::ceil(rank), n - 1);
    const float w = rank - lo_f;
    const float a = sorted[lo], bb = sorted[hi];
    return w < 0.5f ? a + w * (bb - a) : bb - (bb - a) * (1.0f - w);
}

struct BoltEnc {
    std::vector<float> attn_norm, ffn_norm;
    Weight q, k, v, o, wi, wo;
};
struct BoltDec {
    std::vector<float> self_norm, cross_norm, ffn_norm;
    Weight self_v, self_o, cross_q, cross_k, cross_v, cross_o, wi, wo;
};

// runChunk's instance norm and patch features (chronos_bolt/forecaster.zig:150-197) for nb rows
// (row li at ctx + li * stride + offset, len steps, left-padded by pad): loc, scale, features
// [value, mask] per patch, each patch's validity in kv (row stride seq), and the REG token's
// validity after the patches when use_reg.
void bolt_patch_features(const float *ctx, size_t stride, size_t offset, size_t len, size_t pad, size_t n_patch,
                         size_t ps, size_t seq, bool use_reg, size_t nb, float *loc, float *scale, float *feats,
                         uint8_t *kv) {
    for (size_t li = 0; li < nb; ++li) {
        const float *row = ctx + li * stride + offset;
        double count = 0, sum = 0;
        for (size_t i = 0; i < len; ++i)
            if (!std::isnan(row[i])) {
                count += 1;
                sum += row[i];
            }
        float lo = 0.0f, sc = 1.0f;
        if (count > 0) {
            lo = (float)(sum / count);
            double ss = 0;
            for (size_t i = 0; i < len; ++i)
                if (!std::isnan(row[i])) {
                    const float dv = row[i] - lo;
                    ss += (double)dv * (double)dv;
                }
            sc = (float)std::sqrt(ss / count);
            if (sc == 0.0f) sc = 1e-5f;
        }
        loc[li] = lo;
        scale[li] = sc;
        for (size_t p = 0; p < n_patch; ++p) {
            bool any = false;
            const size_t base = (li * n_patch + p) * 2 * ps;
            for (size_t i = 0; i < ps; ++i) {
                const long src = (long)(p * ps + i) - (long)pad;
                bool obs = false;
                float val = 0.0f;
                if (src >= 0) {
                    const float xv = row[src];
                    if (!std::isnan(xv)) {
                        obs = true;
                        val = (xv - lo) / sc;
                    }
                }
                feats[base + i] = val;
                feats[base + ps + i] = obs ? 1.0f : 0.0f;
                any = any || obs;
            }
            kv[li * seq + p] = any;
        }
        if (use_reg) kv[li * seq + n_patch] = 1;
    }
}

struct Bolt {
    tsfm_config c{};
    std::vector<double> quantiles;
    ResBlock input_embed, output_embed;
    std::vector<float> shared, rel_bias, enc_final, dec_final;
    std::vector<BoltEnc> enc;
    std::vector<BoltDec> dec;

    size_t inner() const { return (size_t)c.num_heads * c.d_kv; }
    size_t vocab() const { return c.use_reg_token ? 2 : 1; }

    // Model.load (chronos_bolt/model.zig:101-172).
    void load(const Table &w) {
        const size_t d = c.d_model, ff = c.d_ff, in = inner(), ps = c.patch_size;
        const size_t out_dim = (size_t)c.num_quantiles * c.prediction_length;
        input_embed = w.resblock("input_patch_embedding", 2 * ps, ff, d, true, false);
        output_embed = w.resblock("output_patch_embedding", d, ff, out_dim, true, false);
        shared = w.get("shared.weight", vocab() * d);
        rel_bias = w.get("encoder.block.0.layer.0.SelfAttention.relative_attention_bias.weight",
                         (size_t)c.relative_attention_num_buckets * c.num_heads);
        enc_final = w.get("encoder.final_layer_norm.weight", d);
        dec_final = w.get("decoder.final_layer_norm.weight", d);
        for (int i = 0; i < c.num_layers; ++i) {
            BoltEnc L;
            L.attn_norm = w.get(fmt("encoder.block.%d.layer.0.layer_norm.weight", i), d);
            L.q = w.weight(fmt("encoder.block.%d.layer.0.SelfAttention.q.weight", i), in, d);
            L.k = w.weight(fmt("encoder.block.%d.layer.0.SelfAttention.k.weight", i), in, d);
            L.v = w.weight(fmt("encoder.block.%d.layer.0.SelfAttention.v.weight", i), in, d);
            L.o = w.weight(fmt("encoder.block.%d.layer.0.SelfAttention.o.weight", i), d, in);
            L.ffn_norm = w.get(fmt("encoder.block.%d.layer.1.layer_norm.weight", i), d);
            L.wi = w.weight(fmt("encoder.block.%d.layer.1.DenseReluDense.wi.weight", i), ff, d);
            L.wo = w.weight(fmt("encoder.block.%d.layer.1.DenseReluDense.wo.weight", i), d, ff);
            enc.push_back(std::move(L));
        }
        for (int i = 0; i < c.num_decoder_layers; ++i) {
            BoltDec L;
            L.self_norm = w.get(fmt("decoder.block.%d.layer.0.layer_norm.weight", i), d);
            L.self_v = w.weight(fmt("decoder.block.%d.layer.0.SelfAttention.v.weight", i), in, d);
            L.self_o = w.weight(fmt("decoder.block.%d.layer.0.SelfAttention.o.weight", i), d, in);
            L.cross_norm = w.get(fmt("decoder.block.%d.layer.1.layer_norm.weight", i), d);
            L.cross_q = w.weight(fmt("decoder.block.%d.layer.1.EncDecAttention.q.weight", i), in, d);
            L.cross_k = w.weight(fmt("decoder.block.%d.layer.1.EncDecAttention.k.weight", i), in, d);
            L.cross_v = w.weight(fmt("decoder.block.%d.layer.1.EncDecAttention.v.weight", i), in, d);
            L.cross_o = w.weight(fmt("decoder.block.%d.layer.1.EncDecAttention.o.weight", i), d, in);
            L.ffn_norm = w.get(fmt("decoder.block.%d.layer.2.layer_norm.weight", i), d);
            L.wi = w.weight(fmt("decoder.block.%d.layer.2.DenseReluDense.wi.weight", i), ff, d);
            L.wo = w.weight(fmt("decoder.block.%d.layer.2.DenseReluDense.wo.weight", i), d, ff);
            dec.push_back(std::move(L));
        }
    }

    // Model.encode (chronos_bolt/model.zig:210-254), positionBias :195-205, SelfJob :335-357.
    void encode(float *x, const uint8_t *key_valid, size_t nb, size_t seq) const {
        const size_t d = c.d_model, ff = c.d_ff, in = inner(), nh = c.num_heads, hd = c.d_kv;
        const size_t rows = nb * seq;
        const float eps = (float)c.layer_norm_epsilon;
        std::vector<float> xn(rows * d), delta(rows * d), mlp_h(rows * ff), qb(rows * in),
            kb(rows * in), vb(rows * in), ab(rows * in), bias(nh * seq * seq);
        for (size_t i = 0; i < seq; ++i)
            for (size_t j = 0; j < seq; ++j) {
                const size_t bucket = relative_bucket((int64_t)j - (int64_t)i,
                                                      c.relative_attention_num_buckets,
                                                      c.relative_attention_max_distance);
                for (size_t h = 0; h < nh; ++h) bias[h * seq * seq + i * seq + j] = rel_bias[bucket * nh + h];
            }
        bool all_valid = true;
        for (size_t i = 0; i < rows; ++i) all_valid = all_valid && key_valid[i];
        const Mask mask = mask_pick(false, all_valid, true);
        for (const BoltEnc &L : enc) {
            rms_norm(xn.data(), x, rows, d, L.attn_norm.data(), eps);
            linear(qb.data(), xn.data(), rows, L.q, nullptr);
            linear(kb.data(), xn.data(), rows, L.k, nullptr);
            linear(vb.data(), xn.data(), rows, L.v, nullptr);
#pragma omp parallel
            {
                std::vector<float> scores(seq * seq);
#pragma omp for schedule(static)
                for (long item = 0; item < (long)(nb * nh); ++item) {
                    const size_t r = item / nh, h = item % nh, off = r * seq * in + h * hd;
                    self_attend(mask, scores.data(), &qb[off], &kb[off], &vb[off], &ab[off], in, in, in,
                                in, seq, hd, 1.0f, key_valid + r * seq, &bias[h * seq * seq]);
                }
            }
            linear(delta.data(), ab.data(), rows, L.o, nullptr);
            add_in_place(x, delta.data(), rows * d);
            rms_norm(xn.data(), x, rows, d, L.ffn_norm.data(), eps);
            linear(mlp_h.data(), xn.data(), rows, L.wi, nullptr);
            relu(mlp_h.data(), mlp_h.size());
            linear(delta.data(), mlp_h.data(), rows, L.wo, nullptr);
            add_in_place(x, delta.data(), rows * d);
        }
        rms_norm(x, x, rows, d, enc_final.data(), eps);
    }

    // Model.decode (chronos_bolt/model.zig:258-308), CrossJob :360-381.
    void decode(float *out, const float *encx, const uint8_t *key_valid, size_t nb, size_t seq) const {
        const size_t d = c.d_model, ff = c.d_ff, in = inner(), nh = c.num_heads, hd = c.d_kv;
        const float eps = (float)c.layer_norm_epsilon;
        std::vector<float> x(nb * d), xn(nb * d), delta(nb * d), mlp_h(nb * ff), qd(nb * in),
            vd(nb * in), ad(nb * in), kb(nb * seq * in), vb(nb * seq * in);
        const float *start = &shared[(size_t)c.decoder_start_token_id * d];
        for (size_t r = 0; r < nb; ++r) std::memcpy(&x[r * d], start, d * 4);
        for (const BoltDec &L : dec) {
            rms_norm(xn.data(), x.data(), nb, d, L.self_norm.data(), eps);
            linear(vd.data(), xn.data(), nb, L.self_v, nullptr);
            linear(delta.data(), vd.data(), nb, L.self_o, nullptr);
            add_in_place(x.data(), delta.data(), nb * d);

            rms_norm(xn.data(), x.data(), nb, d, L.cross_norm.data(), eps);
            linear(qd.data(), xn.data(), nb, L.cross_q, nullptr);
            linear(kb.data(), encx, nb * seq, L.cross_k, nullptr);
            linear(vb.data(), encx, nb * seq, L.cross_v, nullptr);
#pragma omp parallel
            {
                std::vector<float> scores(seq);
#pragma omp for schedule(static)
                for (long item = 0; item < (long)(nb * nh); ++item) {
                    const size_t r = item / nh, h = item % nh;
                    const float *qh = &qd[r * in + h * hd];
                    for (size_t j = 0; j < seq; ++j) {
                        const float *kh = &kb[(r * seq + j) * in + h * hd];
                        float s = 0.0f;
                        for (size_t cc = 0; cc < hd; ++cc) s += qh[cc] * kh[cc];
                        scores[j] = s;
                        if (!key_valid[r * seq + j]) scores[j] += -kFloatMax;
                    }
                    softmax(scores.data(), seq);
                    float *oh = &ad[r * in + h * hd];
                    for (size_t cc = 0; cc < hd; ++cc) oh[cc] = 0.0f;
                    for (size_t j = 0; j < seq; ++j) {
                        const float *vh = &vb[(r * seq + j) * in + h * hd];
                        for (size_t cc = 0; cc < hd; ++cc) oh[cc] += scores[j] * vh[cc];
                    }
                }
            }
            linear(delta.data(), ad.data(), nb, L.cross_o, nullptr);
            add_in_place(x.data(), delta.data(), nb * d);

            rms_norm(xn.data(), x.data(), nb, d, L.ffn_norm.data(), eps);
            linear(mlp_h.data(), xn.data(), nb, L.wi, nullptr);
            relu(mlp_h.data(), mlp_h.size());
            linear(delta.data(), mlp_h.data(), nb, L.wo, nullptr);
            add_in_place(x.data(), delta.data(), nb * d);
        }
        rms_norm(out, x.data(), nb, d, dec_final.data(), eps);
    }

    // forecaster.runChunk (chronos_bolt/forecaster.zig:129-220).
    void run_chunk(float *out, const float *ctx, size_t stride, size_t offset, size_t len, size_t s0,
                   size_t s1) const {
        const size_t d = c.d_model, ps = c.patch_size, q = c.num_quantiles, P = c.prediction_length;
        const bool use_reg = c.use_reg_token != 0;
        const size_t pad = (ps - len % ps) % ps, n_patch = (len + pad) / ps;
        const size_t seq = n_patch + (use_reg ? 1 : 0), nb = s1 - s0;
        std::vector<float> loc(nb), scale(nb), feats(nb * n_patch * 2 * ps);
        std::vector<uint8_t> kv(nb * seq);
        bolt_patch_features(ctx + s0 * stride, stride, offset, len, pad, n_patch, ps, seq, use_reg, nb, loc.data(),
                            scale.data(), feats.data(), kv.data());
        std::vector<float> emb(nb * n_patch * d);
        input_embed.forward(emb.data(), feats.data(), nb * n_patch);
        std::vector<float> x(nb * seq * d);
        for (size_t li = 0; li < nb; ++li) {
            std::memcpy(&x[li * seq * d], &emb[li * n_patch * d], n_patch * d * 4);
            if (use_reg)
                std::memcpy(&x[(li * seq + n_patch) * d], &shared[(size_t)c.reg_token_id * d], d * 4);
        }
        encode(x.data(), kv.data(), nb, seq);
        std::vector<float> hidden(nb * d), raw(nb * q * P);
        decode(hidden.data(), x.data(), kv.data(), nb, seq);
        output_embed.forward(raw.data(), hidden.data(), nb);
        for (size_t li = 0; li < nb; ++li)
            for (size_t i = 0; i < q * P; ++i)
                out[(s0 + li) * q * P + i] = raw[li * q * P + i] * scale[li] + loc[li];
    }

    // predictBlock (chronos_bolt/forecaster.zig:116-127), chunkSize :107-111.
    void predict_block(float *out, const float *ctx, size_t stride, size_t offset, size_t len,
                       size_t n) const {
        const size_t ps = c.patch_size;
        const size_t n_patch = (len + ps - 1) / ps, seq = n_patch + (c.use_reg_token ? 1 : 0);
        const size_t budget = 16u * 1024 * 1024;
        const size_t per = std::max<size_t>(1, seq * ((size_t)c.d_model * 12 + c.d_ff));
        const size_t chunk = std::min(n, std::max<size_t>(1, budget / per));
        for (size_t s0 = 0; s0 < n; s0 += chunk)
            run_chunk(out, ctx, stride, offset, len, s0, std::min(n, s0 + chunk));
    }

    static void store_block(float *out, const float *pred, size_t b, size_t q, size_t P,
                            size_t horizon, size_t block_start) {
        for (size_t s = 0; s < b; ++s)
            for (size_t p = 0; p < P; ++p) {
                const size_t step = block_start + p;
                if (step >= horizon) break;
                for (size_t qi = 0; qi < q; ++qi)
                    out[(s * horizon + step) * q + qi] = pred[(s * q + qi) * P + p];
            }
    }

    // forecaster.forecast (chronos_bolt/forecaster.zig:22-80).
    void forecast(const float *inputs, size_t b, size_t t_in, size_t horizon, float *out) const {
        const size_t q = c.num_quantiles, P = c.prediction_length, max_ctx = c.context_length;
        if (b == 0 || t_in == 0 || horizon == 0) fail(TSFM_ERR_EMPTY_INPUT, "EmptyInput");
        const size_t len0 = std::min(t_in, max_ctx);
        std::vector<float> pred(b * q * P);
        predict_block(pred.data(), inputs, t_in, t_in - len0, len0, b);
        store_block(out, pred.data(), b, q, P, horizon, 0);
        size_t done = std::min(P, horizon);
        if (done >= horizon) return;
        size_t len = len0;
        std::vector<float> cur(b * q * len);
        for (size_t s = 0; s < b; ++s)
            for (size_t qi = 0; qi < q; ++qi)
                std::memcpy(&cur[(s * q + qi) * len], inputs + s * t_in + t_in - len0, len0 * 4);
        std::vector<float> levels(q), samples(q * q), raw(b * q * q * P);
        for (size_t i = 0; i < q; ++i) levels[i] = (float)quantiles[i];
        while (done < horizon) {
            const size_t new_len = std::min(len + P, max_ctx), skip = len + P - new_len;
            std::vector<float> next(b * q * new_len);
            for (size_t row = 0; row < b * q; ++row)
                for (size_t i = 0; i < new_len; ++i) {
                    const size_t j = skip + i;
                    next[row * new_len + i] = j < len ? cur[row * len + j] : pred[row * P + (j - len)];
                }
            cur.swap(next);
            len = new_len;
            predict_block(raw.data(), cur.data(), len, 0, len, b * q);
            for (size_t s = 0; s < b; ++s)
                for (size_t p = 0; p < P; ++p) {
                    for (size_t k = 0; k < q * q; ++k) samples[k] = raw[(s * q * q + k) * P + p];
                    std::sort(samples.begin(), samples.end());
                    for (size_t qi = 0; qi < q; ++qi)
                        pred[(s * q + qi) * P + p] = quantile_linear(samples.data(), q * q, levels[qi]);
                }
            store_block(out, pred.data(), b, q, P, horizon, done);
            done += P;
        }
    }
};

// ---------------------------------------------------------------------------------------------
// Timestral (timestral/model.zig, timestral/forecaster.zig)

enum Role { R_TARGET = 0, R_PAST = 1, R_KNOWN = 2 };

struct TAttn {
    bool is_time = false;
    std::vector<float> norm;
    Weight qkv, out, gate;
    bool has_gate = false;
};
struct TLayer {
    TAttn attns[2];
    int n_attn = 0;
    std::vector<float> mlp_norm;
    Weight w12, w3;
};

struct Welford {
    double w, mean, m2;
};
Welford welford_combine(Welford a, Welford b) {  // timestral/forecaster.zig:567-577
    const double w = a.w + b.w;
    if (w == 0) return {0, 0, 0};
    const double w_safe = std::fmax(w, std::numeric_limits<double>::min());
    const double delta = b.mean - a.mean;
    return {w, a.mean + delta * b.w / w_safe, a.m2 + b.m2 + delta * delta * a.w * b.w / w_safe};
}

// patchStats / StatsJob (timestral/model.zig:213-216, 712-750): causal per-patch loc and scale of
// each row, f64 running sums over the observed steps, rounded to f32.
void ts_patch_stats(float *loc, float *scale, const float *data, const uint8_t *observed, size_t rows, size_t t,
                size_t ps, double min_scale) {
    const size_t n = t / ps;
    for (size_t r = 0; r < rows; ++r) {
        double cum_w = 0, cum_x = 0, m2 = 0, prev_mean = 0;
        for (size_t p = 0; p < n; ++p) {
            for (size_t k = 0; k < ps; ++k) {
                const size_t i = p * ps + k;
                const double w = observed[r * t + i] ? 1.0 : 0.0;
                const double x = data[r * t + i];
                cum_w += w;
                cum_x += w * x;
                const double den = std::fmax(cum_w, 1.0);
                const double mean = cum_x / den;
                m2 += (x - prev_mean) * (x - mean) * w;
                prev_mean = mean;
            }
            const double den = std::fmax(cum_w, 1.0);
            const double variance = m2 / std::fmax(den - 1.0, 1.0);
            loc[r * n + p] = (float)prev_mean;
            scale[r * n + p] = (float)std::fmax(std::sqrt(variance), min_scale);
        }
    }
}

// predictBlock's window statistics and patch features (timestral/model.zig:253-327) over rows of
// w steps (full / full_obs): causal per-patch loc and scale, known rows (role 2, with covariates)
// normalised by their whole-row mean and std (binary rows unscaled and without asinh), features
// [asinh((x - loc) / scale), missing] per step (emb_in rows of 2 * ps per patch).
void ts_block_features(float *loc, float *scale, float *emb_in, const float *full, const uint8_t *full_obs,
                       size_t rows, size_t w, size_t ps, size_t vall, const std::vector<Role> &roles, bool cov,
                       double min_scale, bool use_arcsinh) {
    const size_t n = w / ps;
    ts_patch_stats(loc, scale, full, full_obs, rows, w, ps, min_scale);
    const float eps32 = std::numeric_limits<float>::epsilon();
    for (size_t r = 0; r < rows; ++r) {
        const bool known = cov && roles[r % vall] == R_KNOWN;
        float kloc = 0.0f, kscale = 1.0f;
        bool binary = false;
        if (known) {
            float cnt = 0.0f, sum = 0.0f;
            bool zero_one = true, any = false;
            for (size_t i = 0; i < w; ++i)
                if (full_obs[r * w + i]) {
                    const float xv = full[r * w + i];
                    cnt += 1.0f;
                    sum += xv;
                    zero_one = zero_one && (xv == 0.0f || xv == 1.0f);
                    any = true;
                }
            kloc = sum / std::fmax(cnt, 1.0f);
            float ss = 0.0f;
            for (size_t i = 0; i < w; ++i)
                if (full_obs[r * w + i]) {
                    const float dv = full[r * w + i] - kloc;
                    ss += dv * dv;
                }
            kscale = std::fmax(std::sqrt(ss / std::fmax(cnt, 1.0f)), (float)min_scale);
            binary = zero_one && any;
            if (binary) {
                kloc = 0.0f;
                kscale = 1.0f;
            }
        }
        for (size_t p = 0; p < n; ++p) {
            const float lo = known ? kloc : loc[r * n + p];
            const float sc = std::fmax(known ? kscale : scale[r * n + p], eps32);
            float *dst = &emb_in[(r * n + p) * 2 * ps];
            for (size_t i = 0; i < ps; ++i) {
                const bool o = full_obs[r * w + p * ps + i];
                float v = 0.0f;
                if (o) {
                    v = (full[r * w + p * ps + i] - lo) / sc;
                    if (use_arcsinh && !(known && binary)) v = std::asinh(v);
                }
                dst[i] = v;
                dst[ps + i] = o ? 0.0f : 1.0f;
            }
        }
    }
}

// predictBlock's key validity and first observed patch per group (timestral/model.zig:344-362):
// a patch is a valid key when any step is observed (or, with attend_missing, once the row has
// started); first_obs[g] = the group's first observed patch (0 when none).
void ts_key_valid(uint8_t *key_valid, size_t *first_obs, const uint8_t *full_obs, size_t rows, size_t w, size_t ps,
                  size_t vall, size_t groups, bool attend_missing) {
    const size_t ne = w / ps;
    for (size_t g = 0; g < groups; ++g) first_obs[g] = ne;
    for (size_t r = 0; r < rows; ++r) {
        const size_t grp = r / vall;
        bool started = false;
        for (size_t p = 0; p < ne; ++p) {
            bool o = false;
            for (size_t i = 0; i < ps; ++i) o = o || full_obs[r * w + p * ps + i];
            if (o) first_obs[grp] = std::min(first_obs[grp], p);
            started = started || o;
            key_valid[r * ne + p] = attend_missing ? (o || started) : o;
        }
    }
    for (size_t g = 0; g < groups; ++g)
        if (first_obs[g] == ne) first_obs[g] = 0;
}

struct Timestral {
    tsfm_config c{};
    std::vector<double> knots;
    std::vector<int32_t> kinds;
    ResBlock patch_proj, head;
    std::vector<float> forecast_query, out_norm, inv_freq;
    std::vector<TLayer> layers;

    size_t hd() const { return (size_t)c.d_model / c.num_heads; }
    size_t rope_dim() const { return (size_t)((double)hd() * c.rope_partial_factor); }
    size_t median_index() const {
        for (size_t i = 0; i < knots.size(); ++i)
            if (knots[i] == 0.5) return i;
        return 0;
    }
    // Config.supportsKnownCovariates (timestral/config.zig:49-72).
    bool supports_known() const {
        if (!c.covariate_enabled) return false;
        std::vector<bool> ops;
        for (int32_t k : kinds) {
            if (k == TSFM_LAYER_TIME) ops.push_back(true);
            else if (k == TSFM_LAYER_VARIATE) ops.push_back(false);
            else if (k == TSFM_LAYER_TIME_VARIATE) { ops.push_back(true); ops.push_back(false); }
            else { ops.push_back(false); ops.push_back(true); }
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

    // permuteQkv (timestral/model.zig:72-85): (qkv, head_dim, heads) -> (qkv, head, head_dim).
    static std::vector<float> permute_qkv(const std::vector<float> &src, size_t d, size_t nh,
                                          size_t hd) {
        std::vector<float> dst(3 * d * d);
        for (size_t sel = 0; sel < 3; ++sel)
            for (size_t h = 0; h < nh; ++h)
                for (size_t dd = 0; dd < hd; ++dd) {
                    const size_t src_row = sel * d + dd * nh + h, dst_row = (sel * nh + h) * hd + dd;
                    std::memcpy(&dst[dst_row * d], &src[src_row * d], d * 4);
                }
        return dst;
    }

    // Model.load (timestral/model.zig:136-200).
    void load(const Table &w) {
        const size_t d = c.d_model, ps = c.patch_size, hid = c.d_ff, nh = c.num_heads;
        patch_proj = w.resblock("representation.patch_proj", 2 * ps, 4 * d, d, true, true);
        forecast_query = w.get("representation.forecast_query", d);
        head = w.resblock("head.projection", d, 4 * d, ps * knots.size(), false, true);
        out_norm = w.get("transformer.out_norm.scale", d);
        for (size_t li = 0; li < kinds.size(); ++li) {
            TLayer L;
            const int32_t k = kinds[li];
            bool is_time[2];
            L.n_attn = (k == TSFM_LAYER_TIME || k == TSFM_LAYER_VARIATE) ? 1 : 2;
            is_time[0] = (k == TSFM_LAYER_TIME || k == TSFM_LAYER_TIME_VARIATE);
            is_time[1] = (k == TSFM_LAYER_VARIATE_TIME);
            for (int ai = 0; ai < L.n_attn; ++ai) {
                TAttn &a = L.attns[ai];
                a.is_time = is_time[ai];
                a.norm = w.get(fmt2("transformer.layers.%d.attn_norms.%d.scale", (int)li, ai), d);
                std::vector<float> raw =
                    w.get(fmt2("transformer.layers.%d.attns.%d.wQKV.weight", (int)li, ai), 3 * d * d);
                a.qkv.init(permute_qkv(raw, d, nh, hd()), 3 * d, d);
                a.out = w.weight(fmt2("transformer.layers.%d.attns.%d.wO.weight", (int)li, ai), d, d);
                a.has_gate = a.is_time ? c.time_attn_gate != 0 : c.variate_attn_gate != 0;
                if (a.has_gate)
                    a.gate = w.weight(fmt2("transformer.layers.%d.attns.%d._gate.weight", (int)li, ai), d, d);
            }
            L.mlp_norm = w.get(fmt("transformer.layers.%d.mlp_norm.scale", (int)li), d);
            L.w12 = w.weight(fmt("transformer.layers.%d.mlp.w12.weight", (int)li), 2 * hid, d);
            L.w3 = w.weight(fmt("transformer.layers.%d.mlp.w3.weight", (int)li), d, hid);
            layers.push_back(std::move(L));
        }
        inv_freq.assign(hd() / 2, 0.0f);
        const float base = (float)c.rope_theta;
        for (size_t i = 0; i < rope_dim() / 2; ++i)
            inv_freq[i] = 1.0f / std::pow(base, (float)(2 * i) / (float)rope_dim());
    }

    // patchStats / StatsJob (timestral/model.zig:213-216, 712-750).
    void patch_stats(float *loc, float *scale, const float *data, const uint8_t *observed,
                     size_t rows, size_t t) const {
        ts_patch_stats(loc, scale, data, observed, rows, t, c.patch_size, c.minimum_scale);
    }

    struct Geo {
        size_t rows, groups, vall, ne, l, h;
        const std::vector<Role> *roles;
        bool cov;
        const std::vector<uint8_t> *key_valid;
        bool keys_all_valid;
        const std::vector<size_t> *first_obs;
        size_t sl() const { return ne + h; }
        Role role(size_t r) const { return (*roles)[r % vall]; }
    };

    // timeAttention + TimeJob.rope/attend (timestral/model.zig:487-519, 558-635).
    void time_attention(float *out, const float *xn, const TAttn &a, const Geo &g,
                        const std::vector<float> &cos_t, const std::vector<float> &sin_t) const {
        const size_t d = c.d_model, nh = c.num_heads, hdim = hd(), half = hdim / 2;
        const size_t rows = g.rows, sl = g.sl(), ne = g.ne, l = g.l, h = g.h;
        std::vector<float> qkv(rows * sl * 3 * d), oa(rows * sl * d), gate;
        linear(qkv.data(), xn, rows * sl, a.qkv, nullptr);
        if (a.has_gate) {
            gate.resize(rows * sl * d);
            linear(gate.data(), xn, rows * sl, a.gate, nullptr);
        }
        for (size_t idx = 0; idx < rows * sl; ++idx) {
            const size_t r = idx / sl, tok = idx % sl, grp = r / g.vall;
            const float *cs = &cos_t[(grp * sl + tok) * half], *sn = &sin_t[(grp * sl + tok) * half];
            for (size_t hh = 0; hh < nh; ++hh) {
                rope_half(&qkv[idx * 3 * d + hh * hdim], cs, sn, half);
                rope_half(&qkv[idx * 3 * d + d + hh * hdim], cs, sn, half);
            }
        }
        const float sm_scale = 1.0f / std::sqrt((float)hdim);
#pragma omp parallel
        {
            std::vector<float> scores(std::max(ne * ne, h * sl));
#pragma omp for schedule(static)
            for (long item = 0; item < (long)(rows * nh); ++item) {
                const size_t r = item / nh, hh = item % nh, off = hh * hdim;
                const bool bidir = g.cov && g.role(r) == R_KNOWN;
                const size_t base = r * sl * 3 * d;
                const float *q = &qkv[base + off], *k = &qkv[base + d + off], *v = &qkv[base + 2 * d + off];
                float *o = &oa[r * sl * d + off];
                const uint8_t *kv = &(*g.key_valid)[r * ne];
                const Mask mask = mask_pick(!bidir, g.keys_all_valid, false);
                self_attend(mask, scores.data(), q, k, v, o, 3 * d, 3 * d, 3 * d, d, ne, hdim, sm_scale,
                            kv, nullptr);
                gemm_nt(scores.data(), sl, &qkv[base + ne * 3 * d + off], 3 * d, k, 3 * d, h, sl, hdim,
                        sm_scale);
                for (size_t j = 0; j < h; ++j) {
                    float *row = &scores[j * sl];
                    if (g.keys_all_valid) {
                        for (size_t kk = l; kk < ne; ++kk) row[kk] = -kInf;
                        const size_t end = ne + j + 1;
                        softmax(row, end);
                        for (size_t kk = end; kk < sl; ++kk) row[kk] = 0.0f;
                    } else {
                        for (size_t kk = 0; kk < ne; ++kk)
                            if (kk >= l || !kv[kk]) row[kk] = -kInf;
                        for (size_t kk = ne + j + 1; kk < sl; ++kk) row[kk] = -kInf;
                        softmax(row, sl);
                    }
                }
                gemm_nn(o + ne * d, d, scores.data(), sl, v, 3 * d, h, hdim, sl);
            }
        }
        if (a.has_gate)
            for (size_t i = 0; i < oa.size(); ++i) oa[i] = oa[i] / (1.0f + exp_vec(-gate[i]));
        linear(out, oa.data(), rows * sl, a.out, nullptr);
    }

    // variateAttention + VariateJob (timestral/model.zig:525-544, 648-709).
    void variate_attention(float *out, const float *xn, const TAttn &a, const Geo &g) const {
        const size_t d = c.d_model, nh = c.num_heads, hdim = hd();
        const size_t rows = g.rows, sl = g.sl(), ne = g.ne, vall = g.vall;
        std::vector<float> qkv(rows * sl * 3 * d), o(rows * sl * d), gate;
        linear(qkv.data(), xn, rows * sl, a.qkv, nullptr);
        if (a.has_gate) {
            gate.resize(rows * sl * d);
            linear(gate.data(), xn, rows * sl, a.gate, nullptr);
        }
        const float sm_scale = 1.0f / std::sqrt((float)hdim);
#pragma omp parallel
        {
            std::vector<float> sc(vall);
            std::vector<uint8_t> allowed(vall * vall);
#pragma omp for schedule(static)
            for (long item = 0; item < (long)(g.groups * sl); ++item) {
                const size_t grp = item / sl, tok = item % sl, r0 = grp * vall;
                for (size_t iq = 0; iq < vall; ++iq)
                    for (size_t ik = 0; ik < vall; ++ik) {
                        bool ok = ik == iq;
                        if (!ok) {
                            const bool valid = tok >= ne || (*g.key_valid)[(r0 + ik) * ne + tok];
                            bool forbidden = false;
                            if (g.cov) {
                                const Role rq = (*g.roles)[iq], rk = (*g.roles)[ik];
                                forbidden = (rq != R_TARGET && rk == R_TARGET) || (rq == R_KNOWN && rk != R_KNOWN);
                            }
                            ok = valid && !forbidden;
                        }
                        allowed[iq * vall + ik] = ok;
                    }
                for (size_t hh = 0; hh < nh; ++hh) {
                    const size_t qoff = hh * hdim;
                    for (size_t iq = 0; iq < vall; ++iq) {
                        const float *qs = &qkv[(r0 + iq) * sl * 3 * d + tok * 3 * d + qoff];
                        for (size_t ik = 0; ik < vall; ++ik) {
                            if (!allowed[iq * vall + ik]) {
                                sc[ik] = -kInf;
                                continue;
                            }
                            const float *ks = &qkv[(r0 + ik) * sl * 3 * d + tok * 3 * d + d + qoff];
                            float s = 0.0f;
                            for (size_t cc = 0; cc < hdim; ++cc) s += qs[cc] * ks[cc];
                            sc[ik] = s * sm_scale;
                        }
                        softmax(sc.data(), vall);
                        float *dst = &o[(r0 + iq) * sl * d + tok * d + qoff];
                        for (size_t cc = 0; cc < hdim; ++cc) dst[cc] = 0.0f;
                        for (size_t ik = 0; ik < vall; ++ik) {
                            const float wgt = sc[ik];
                            if (wgt == 0.0f) continue;
                            const float *vs = &qkv[(r0 + ik) * sl * 3 * d + tok * 3 * d + 2 * d + qoff];
                            for (size_t cc = 0; cc < hdim; ++cc) dst[cc] += wgt * vs[cc];
                        }
                    }
                }
            }
        }
        if (a.has_gate)
            for (size_t i = 0; i < o.size(); ++i) o[i] = o[i] / (1.0f + exp_vec(-gate[i]));
        linear(out, o.data(), rows * sl, a.out, nullptr);
    }

    // runTransformer (timestral/model.zig:434-482).
    void run_transformer(float *x, const Geo &g) const {
        const size_t d = c.d_model, sl = g.sl(), rows = g.rows, hid = c.d_ff;
        const float eps = (float)c.layer_norm_epsilon;
        std::vector<float> xn(rows * sl * d), delta(rows * sl * d), mlp_h(rows * sl * 2 * hid),
            mlp_a(rows * sl * hid);
        const size_t half = hd() / 2;
        std::vector<float> cos_t(g.groups * sl * half), sin_t(g.groups * sl * half);
        for (size_t grp = 0; grp < g.groups; ++grp)
            for (size_t tok = 0; tok < sl; ++tok) {
                const int64_t time = tok < g.ne ? (int64_t)tok : (int64_t)(g.l + tok - g.ne);
                const float pos = (float)(time - (int64_t)(*g.first_obs)[grp]);
                for (size_t i = 0; i < half; ++i) {
                    const float ang = inv_freq[i] * pos;
                    cos_t[(grp * sl + tok) * half + i] = std::cos(ang);
                    sin_t[(grp * sl + tok) * half + i] = std::sin(ang);
                }
            }
        for (const TLayer &L : layers) {
            for (int ai = 0; ai < L.n_attn; ++ai) {
                const TAttn &a = L.attns[ai];
                rms_norm(xn.data(), x, rows * sl, d, a.norm.data(), eps);
                if (a.is_time)
                    time_attention(delta.data(), xn.data(), a, g, cos_t, sin_t);
                else
                    variate_attention(delta.data(), xn.data(), a, g);
                add_in_place(x, delta.data(), rows * sl * d);
            }
            rms_norm(xn.data(), x, rows * sl, d, L.mlp_norm.data(), eps);
            linear(mlp_h.data(), xn.data(), rows * sl, L.w12, nullptr);
            for (size_t i = 0; i < rows * sl; ++i)  // MlpAct.run: gate * silu(up) (model.zig:159-165)
                for (size_t j = 0; j < hid; ++j) {
                    const float gt = mlp_h[i * 2 * hid + j], up = mlp_h[i * 2 * hid + hid + j];
                    mlp_a[i * hid + j] = gt * (up / (1.0f + exp_vec(-up)));
                }
            linear(delta.data(), mlp_a.data(), rows * sl, L.w3, nullptr);
            add_in_place(x, delta.data(), rows * sl * d);
        }
    }

    // Model.predictBlock (timestral/model.zig:220-432).
    void predict_block(float *out, const float *ctx, const uint8_t *obs, size_t t, size_t groups,
                       const std::vector<Role> &roles, size_t h, const float *known_future,
                       const uint8_t *known_future_obs) const {
        const size_t ps = c.patch_size, d = c.d_model, q = knots.size();
        const size_t vall = roles.size(), rows = groups * vall, l = t / ps, hl = h * ps;
        bool cov = false;
        size_t n_tgt = 0;
        for (Role r : roles) {
            cov = cov || r != R_TARGET;
            if (r == R_TARGET) ++n_tgt;
        }
        if (!cov && known_future) fail(TSFM_ERR_INVALID_ARGUMENT, "InvalidInput");
        if (cov && (h < 1 || h > (size_t)c.block_size)) fail(TSFM_ERR_INVALID_ARGUMENT, "BlockTooLong");
        const size_t w = cov ? t + hl : t, n = w / ps;
        std::vector<float> fbuf;
        std::vector<uint8_t> fobuf;
        const float *full = ctx;
        const uint8_t *full_obs = obs;
        if (cov) {
            fbuf.assign(rows * w, 0.0f);
            fobuf.assign(rows * w, 0);
            for (size_t r = 0; r < rows; ++r) {
                std::memcpy(&fbuf[r * w], ctx + r * t, t * 4);
                std::memcpy(&fobuf[r * w], obs + r * t, t);
                if (known_future) {
                    std::memcpy(&fbuf[r * w + t], known_future + r * hl, hl * 4);
                    std::memcpy(&fobuf[r * w + t], known_future_obs + r * hl, hl);
                }
            }
            full = fbuf.data();
            full_obs = fobuf.data();
        }
        std::vector<float> loc(rows * n), scale(rows * n);
        std::vector<float> emb_in(rows * n * 2 * ps);
        ts_block_features(loc.data(), scale.data(), emb_in.data(), full, full_obs, rows, w, ps, vall, roles, cov,
                          c.minimum_scale, c.use_arcsinh != 0);
        const size_t ne = n, sl = ne + h;
        std::vector<float> x(rows * sl * d), enc(rows * ne * d);
        patch_proj.forward(enc.data(), emb_in.data(), rows * ne);
        for (size_t r = 0; r < rows; ++r) {
            std::memcpy(&x[r * sl * d], &enc[r * ne * d], ne * d * 4);
            for (size_t j = 0; j < h; ++j) std::memcpy(&x[(r * sl + ne + j) * d], forecast_query.data(), d * 4);
        }
        std::vector<uint8_t> key_valid(rows * ne);
        std::vector<size_t> first_obs(groups, ne);
        ts_key_valid(key_valid.data(), first_obs.data(), full_obs, rows, w, c.patch_size, vall, groups,
                     c.attend_missing_patches != 0);
        bool all_valid = true;
        for (uint8_t v : key_valid) all_valid = all_valid && v;
        Geo g{rows, groups, vall, ne, l, h, &roles, cov, &key_valid, all_valid, &first_obs};
        run_transformer(x.data(), g);

        const size_t n_rows_out = groups * n_tgt;
        std::vector<float> dec(n_rows_out * h * d), raw(n_rows_out * hl * q);
        size_t oi = 0;
        for (size_t r = 0; r < rows; ++r) {
            if (roles[r % vall] != R_TARGET) continue;
            rms_norm(&dec[oi * h * d], &x[(r * sl + ne) * d], h, d, out_norm.data(), (float)c.layer_norm_epsilon);
            ++oi;
        }
        head.forward(raw.data(), dec.data(), n_rows_out * h);
        const size_t m = median_index();
        std::vector<float> widths(q, 0.0f);
        for (size_t i = m + 1; i < q; ++i) widths[i] = (float)(knots[i] - knots[i - 1]);
        for (size_t i = 0; i < m; ++i) widths[i] = (float)(knots[i + 1] - knots[i]);
        const float wf = (float)c.quantile_width_factor;
        oi = 0;
        for (size_t r = 0; r < rows; ++r) {
            if (roles[r % vall] != R_TARGET) continue;
            const float lo = loc[r * n + l - 1], sc = scale[r * n + l - 1];
            for (size_t s = 0; s < hl; ++s) {
                const float *rv = &raw[(oi * hl + s) * q];
                float *ov = &out[(oi * hl + s) * q];
                const float med = rv[m];
                float acc = 0.0f;
                for (size_t i = m + 1; i < q; ++i) {
                    acc += wf * widths[i] * softplus(rv[i]);
                    ov[i] = std::fmax(-kFloatMax, std::fmin(med + acc, kFloatMax));  // std.math.clamp
                }
                acc = 0.0f;
                for (size_t i = m; i > 0;) {
                    --i;
                    acc += wf * widths[i] * softplus(rv[i]);
                    ov[i] = std::fmax(-kFloatMax, std::fmin(med - acc, kFloatMax));
                }
                ov[m] = med;
                for (size_t i = 0; i < q; ++i) {
                    const float y = c.use_arcsinh ? std::sinh(ov[i]) : ov[i];
                    ov[i] = y * sc + lo;
                }
                clamp_nonfinite(ov, q);
            }
            ++oi;
        }
    }

    // refineBlock (timestral/forecaster.zig:582-662).
    void refine_block(float *qs, const float *ctx, const uint8_t *mask, size_t groups, size_t vall,
                      size_t v, size_t t, size_t h) const {
        const size_t ps = c.patch_size, q = knots.size(), med = median_index(), l = t / ps;
        std::vector<float> loc(l), scale(l), loc_j(h), scale_j(h);
        const double clip = std::sqrt((double)kFloatMax) / 1e3;
        std::vector<double> sinh_med(h * ps), folded(ps);
        for (size_t g = 0; g < groups; ++g)
            for (size_t i = 0; i < v; ++i) {
                const size_t r = g * vall + i;
                const float *row_ctx = ctx + r * t;
                const uint8_t *row_mask = mask + r * t;
                patch_stats(loc.data(), scale.data(), row_ctx, row_mask, 1, t);
                const float loc0 = loc[l - 1], scale0 = scale[l - 1];
                float *block = qs + (g * v + i) * h * ps * q;
                for (size_t s = 0; s < h * ps; ++s)
                    sinh_med[s] = ((double)block[s * q + med] - (double)loc0) / (double)scale0;
                Welford state{0, 0, 0};
                for (size_t p = 0; p < l; ++p) {
                    double cnt = 0, sum = 0;
                    for (size_t k = 0; k < ps; ++k)
                        if (row_mask[p * ps + k]) {
                            cnt += 1;
                            sum += row_ctx[p * ps + k];
                        }
                    Welford pm{cnt, 0, 0};
                    if (cnt > 0) {
                        pm.mean = sum / std::fmax(cnt, 1.0);
                        for (size_t k = 0; k < ps; ++k)
                            if (row_mask[p * ps + k]) {
                                const double dv = (double)row_ctx[p * ps + k] - pm.mean;
                                pm.m2 += dv * dv;
                            }
                    }
                    state = welford_combine(state, pm);
                }
                const double offset = state.mean;
                for (size_t j = 0; j < h; ++j) {
                    const double variance = std::fmax(state.m2 / std::fmax(state.w - 1.0, 1.0), 0.0);
                    const double sc = std::fmax(std::sqrt(variance), c.minimum_scale);
                    loc_j[j] = (float)state.mean;
                    scale_j[j] = (float)sc;
                    double bsum = 0;
                    for (size_t k = 0; k < ps; ++k) {
                        folded[k] = std::fmax(-clip, std::fmin(sinh_med[j * ps + k] * sc + state.mean - offset, clip)) + offset;
                        bsum += folded[k];
                    }
                    const double bmean = bsum / (double)ps;
                    double bm2 = 0;
                    for (size_t k = 0; k < ps; ++k) bm2 += (folded[k] - bmean) * (folded[k] - bmean);
                    state = welford_combine(state, {(double)ps, bmean, bm2});
                }
                loc_j[0] = loc0;
                scale_j[0] = scale0;
                for (size_t s = 0; s < h * ps; ++s) {
                    float *rowq = block + s * q;
                    const float lj = loc_j[s / ps], sj = scale_j[s / ps];
                    for (size_t k = 0; k < q; ++k) rowq[k] = (rowq[k] - loc0) / scale0 * sj + lj;
                    clamp_nonfinite(rowq, q);
                }
            }
    }

    // blockDecode (timestral/forecaster.zig:423-563).
    void block_decode(float *out, const std::vector<float> &rows_in, const std::vector<uint8_t> &mask_in,
                      const float *kf, const uint8_t *kfm, size_t hpad, size_t groups,
                      const std::vector<Role> &roles, size_t t_in, size_t horizon,
                      const tsfm_timestral_options &o) const {
        const size_t ps = c.patch_size, q = knots.size(), med = median_index(), vall = roles.size();
        const size_t nrows = groups * vall;
        size_t v = 0;
        for (Role r : roles)
            if (r == R_TARGET) ++v;
        const size_t nt = groups * v;
        size_t t = t_in;
        std::vector<float> ctx = rows_in;
        std::vector<uint8_t> cmask = mask_in;
        size_t remaining = (horizon + ps - 1) / ps, done = 0;
        while (remaining > 0) {
            const size_t block = std::min(o.per_shot_horizon_patches, remaining), blen = block * ps;
            std::vector<float> qs(nt * blen * q);
            std::vector<float> kfb;
            std::vector<uint8_t> kfmb;
            if (kf) {
                kfb.resize(nrows * blen);
                kfmb.resize(nrows * blen);
                for (size_t r = 0; r < nrows; ++r) {
                    std::memcpy(&kfb[r * blen], kf + r * hpad + done, blen * 4);
                    std::memcpy(&kfmb[r * blen], kfm + r * hpad + done, blen);
                }
            }
            predict_block(qs.data(), ctx.data(), cmask.data(), t, groups, roles, block,
                          kf ? kfb.data() : nullptr, kf ? kfmb.data() : nullptr);
            if (block > 1) refine_block(qs.data(), ctx.data(), cmask.data(), groups, vall, v, t, block);
            for (size_t r = 0; r < nt; ++r)
                for (size_t s = 0; s < blen; ++s) {
                    if (done + s >= horizon) break;
                    std::memcpy(&out[(r * horizon + done + s) * q], &qs[(r * blen + s) * q], q * 4);
                }
            remaining -= block;
            done += blen;
            if (remaining == 0) break;
            const size_t nt_len = t + blen;
            const size_t keep_t = nt_len > o.max_context ? std::max(ps, o.max_context / ps * ps) : nt_len;
            std::vector<float> nctx(nrows * keep_t);
            std::vector<uint8_t> nmask(nrows * keep_t);
            for (size_t g = 0; g < groups; ++g) {
                size_t ti = 0;
                for (size_t i = 0; i < vall; ++i) {
                    const size_t r = g * vall + i, trow = g * v + ti;
                    const size_t start = nt_len - keep_t;
                    const size_t ncopy = start < t ? t - start : 0;
                    if (ncopy > 0) {
                        std::memcpy(&nctx[r * keep_t], &ctx[r * t + start], ncopy * 4);
                        std::memcpy(&nmask[r * keep_t], &cmask[r * t + start], ncopy);
                    }
                    const size_t s0 = start < t ? 0 : start - t;
                    for (size_t s = s0; s < s0 + (keep_t - ncopy); ++s) {
                        const size_t j = s - s0 + ncopy;
                        switch (roles[i]) {
                            case R_TARGET: {
                                float m = qs[(trow * blen + s) * q + med];
                                if (!std::isfinite(m) || std::fabs(m) >= o.extreme_value_threshold) m = 0.0f;
                                nctx[r * keep_t + j] = m;
                                nmask[r * keep_t + j] = 1;
                                break;
                            }
                            case R_KNOWN:
                                nctx[r * keep_t + j] = kfb[r * blen + s];
                                nmask[r * keep_t + j] = kfmb[r * blen + s];
                                break;
                            case R_PAST:
                                nctx[r * keep_t + j] = 0.0f;
                                nmask[r * keep_t + j] = 0;
                                break;
                        }
                    }
                    if (roles[i] == R_TARGET) ++ti;
                }
            }
            ctx.swap(nctx);
            cmask.swap(nmask);
            t = keep_t;
        }
    }

    struct Rows {
        const float *past = nullptr;
        size_t n_past = 0;
        const float *known = nullptr;
        size_t n_known = 0;
    };

    // forecastRaw (timestral/forecaster.zig:303-421).
    std::vector<float> forecast_raw(const float *inputs, const uint8_t *observed, size_t b, size_t v,
                                    size_t t0, size_t horizon, const Rows &cov,
                                    const tsfm_timestral_options &o) const {
        const size_t ps = c.patch_size, q = knots.size();
        const size_t vall = v + cov.n_past + cov.n_known, nrows = b * vall;
        std::vector<Role> roles(vall);
        for (size_t i = 0; i < vall; ++i) roles[i] = i < v ? R_TARGET : (i < v + cov.n_past ? R_PAST : R_KNOWN);
        const size_t keep = std::min(t0, o.max_context);
        const size_t t = (keep + ps - 1) / ps * ps;
        std::vector<float> rows(nrows * t, 0.0f);
        std::vector<uint8_t> mask(nrows * t, 0);
        const size_t hpad = (horizon + ps - 1) / ps * ps;
        std::vector<float> kf(nrows * hpad, 0.0f);
        std::vector<uint8_t> kfm(nrows * hpad, 0);
        for (size_t s = 0; s < b; ++s)
            for (size_t i = 0; i < vall; ++i) {
                const size_t r = s * vall + i;
                float last = 0.0f;
                bool seen = false;
                for (size_t j = 0; j < t0; ++j) {
                    float val;
                    bool ob;
                    if (roles[i] == R_TARGET) {
                        const size_t idx = (s * v + i) * t0 + j;
                        if (observed[idx]) {
                            last = inputs[idx];
                            seen = true;
                        }
                        val = seen ? last : 0.0f;
                        ob = observed[idx] != 0;
                    } else if (roles[i] == R_PAST) {
                        const float xv = cov.past[(s * cov.n_past + (i - v)) * t0 + j];
                        ob = !std::isnan(xv);
                        val = ob ? xv : 0.0f;
                    } else {
                        const float xv = cov.known[(s * cov.n_known + (i - v - cov.n_past)) * (t0 + horizon) + j];
                        ob = !std::isnan(xv);
                        val = ob ? xv : 0.0f;
                    }
                    if (j >= t0 - keep) {
                        const size_t dst = r * t + (t - keep) + (j - (t0 - keep));
                        rows[dst] = val;
                        mask[dst] = ob;
                    }
                }
                if (roles[i] == R_KNOWN)
                    for (size_t j = 0; j < horizon; ++j) {
                        const float xv = cov.known[(s * cov.n_known + (i - v - cov.n_past)) * (t0 + horizon) + t0 + j];
                        kfm[r * hpad + j] = !std::isnan(xv);
                        kf[r * hpad + j] = kfm[r * hpad + j] ? xv : 0.0f;
                    }
            }
        const size_t ntg = b * v;
        std::vector<float> out(ntg * horizon * q);
        const bool known_any = cov.n_known > 0;
        block_decode(out.data(), rows, mask, known_any ? kf.data() : nullptr,
                     known_any ? kfm.data() : nullptr, hpad, b, roles, t, horizon, o);
        if (o.quantile_real_cap_k > 0) {
            const size_t n = t / ps;
            std::vector<float> loc(n), scale(n);
            for (size_t s = 0; s < b; ++s)
                for (size_t i = 0; i < v; ++i) {
                    const size_t r = s * vall + i;
                    patch_stats(loc.data(), scale.data(), &rows[r * t], &mask[r * t], 1, t);
                    float mx = -kInf, mn = kInf;
                    for (size_t j = 0; j < t; ++j)
                        if (mask[r * t + j]) {
                            mx = std::fmax(mx, rows[r * t + j]);
                            mn = std::fmin(mn, rows[r * t + j]);
                        }
                    if (std::isinf(mx)) mx = 0.0f;
                    if (std::isinf(mn)) mn = 0.0f;
                    const float a = scale[n - 1] * o.quantile_real_cap_k;
                    float *dst = &out[(s * v + i) * horizon * q];
                    for (size_t k = 0; k < horizon * q; ++k)
                        dst[k] = std::fmax(mn - a, std::fmin(dst[k], mx + a));  // std.math.clamp
                }
        }
        for (float xv : out)
            if (std::isnan(xv)) fail(TSFM_ERR_DEGENERATE_INPUT, "DegenerateInput");
        return out;
    }

    // targetEncode / slotOf (timestral/forecaster.zig:243-301).
    static long slot_of(const std::vector<double> &cats, double code) {
        if (std::isnan(code)) return -1;
        auto it = std::lower_bound(cats.begin(), cats.end(), code);
        if (it != cats.end() && *it == code) return it - cats.begin();
        return -1;
    }
    static void target_encode(const double *target, const double *past, size_t t, const double *future,
                              size_t nf, float *out_past, float *out_future) {
        const double smooth = 1.0;
        double item_count = 0, item_sum = 0;
        for (size_t i = 0; i < t; ++i)
            if (std::isfinite(target[i])) {
                item_count += 1;
                item_sum += target[i];
            }
        const double item_mean = item_count > 0 ? item_sum / item_count : 0.0;
        std::vector<double> cats;
        for (size_t i = 0; i < t; ++i)
            if (std::isfinite(past[i])) cats.push_back(past[i]);
        std::sort(cats.begin(), cats.end());
        cats.erase(std::unique(cats.begin(), cats.end()), cats.end());
        const size_t nc = cats.size();
        std::vector<double> sums(nc + 1, 0.0), counts(nc + 1, 0.0);
        for (size_t i = 0; i < t; ++i) {
            if (!std::isfinite(target[i])) continue;
            const long s = slot_of(cats, past[i]);
            const size_t slot = s < 0 ? nc : (size_t)s;
            sums[slot] += target[i];
            counts[slot] += 1;
        }
        for (size_t i = 0; i < t; ++i) {
            const long s = slot_of(cats, past[i]);
            const size_t slot = s < 0 ? nc : (size_t)s;
            out_past[i] = (float)((smooth * item_mean + sums[slot]) / (smooth + counts[slot]));
        }
        if (future)
            for (size_t i = 0; i < nf; ++i) {
                const double cv = future[i];
                double val;
                if (std::isnan(cv)) {
                    val = (smooth * item_mean + sums[nc]) / (smooth + counts[nc]);
                } else {
                    const long s = slot_of(cats, cv);
                    val = s >= 0 ? (smooth * item_mean + sums[s]) / (smooth + counts[s]) : item_mean;
                }
                out_future[i] = (float)val;
            }
    }

    // forecaster.forecast (timestral/forecaster.zig:57-141) and finish :163-180.
    void forecast(const float *inputs, const uint8_t *observed, size_t b, size_t v, size_t t,
                  size_t horizon, const tsfm_covariates *covp, const tsfm_timestral_options &opts,
                  float *result) const {
        const size_t q = knots.size();
        tsfm_timestral_options o = opts;
        if (o.max_context == 0) o.max_context = c.context_length;
        o.per_shot_horizon_patches = std::min(o.per_shot_horizon_patches, (size_t)c.block_size);
        tsfm_covariates cov{};
        if (covp) cov = *covp;
        const bool any_cov = cov.past || cov.known || cov.cat_past || cov.cat_known;
        if (horizon == 0 || b == 0 || v == 0 || t == 0) fail(TSFM_ERR_EMPTY_INPUT, "EmptyInput");
        if (any_cov && !c.covariate_enabled) fail(TSFM_ERR_COVARIATES_UNSUPPORTED, "CovariatesUnsupported");
        if ((cov.known || cov.cat_known) && !supports_known())
            fail(TSFM_ERR_COVARIATES_UNSUPPORTED, "KnownCovariatesUnsupported");
        // encodingTarget (forecaster.zig:201-216) for a univariate target.
        std::vector<double> target;
        const bool have_target = (cov.cat_past || cov.cat_known) && v == 1;
        if (have_target) {
            target.resize(b * t);
            for (size_t s = 0; s < b; ++s) {
                bool started = false;
                float last = 0.0f;
                for (size_t i = 0; i < t; ++i) {
                    if (observed[s * t + i]) {
                        started = true;
                        last = inputs[s * t + i];
                    }
                    const bool in_window = t <= o.max_context || i >= t - o.max_context;
                    target[s * t + i] = started && in_window ? (double)last : std::nan("");
                }
            }
        }
        // encodeCategorical (forecaster.zig:220-238).
        auto encode_cat = [&](const double *codes, size_t nc, size_t len) {
            std::vector<float> outv(b * nc * len);
            for (size_t s = 0; s < b; ++s)
                for (size_t j = 0; j < nc; ++j) {
                    const double *row = codes + (s * nc + j) * len;
                    float *dst = &outv[(s * nc + j) * len];
                    if (!have_target) {
                        for (size_t i = 0; i < len; ++i) dst[i] = (float)row[i];
                        continue;
                    }
                    target_encode(&target[s * t], row, t, len > t ? row + t : nullptr, len - t, dst,
                                  len > t ? dst + t : nullptr);
                    for (size_t i = 0; i < t; ++i)
                        if (std::isnan(target[s * t + i]) && std::isnan(row[i])) dst[i] = std::nanf("");
                }
            return outv;
        };
        std::vector<float> enc_past, enc_known;
        if (cov.cat_past) enc_past = encode_cat(cov.cat_past, cov.n_cat_past, t);
        if (cov.cat_known) enc_known = encode_cat(cov.cat_known, cov.n_cat_known, t + horizon);
        // catChannels (forecaster.zig:189-197).
        auto cat_channels = [&](const float *a, size_t ca, const std::vector<float> &bb, size_t cb, size_t len) {
            std::vector<float> outv;
            if (ca + cb == 0) return outv;
            outv.resize(b * (ca + cb) * len);
            for (size_t i = 0; i < b; ++i) {
                if (a) std::memcpy(&outv[i * (ca + cb) * len], a + i * ca * len, ca * len * 4);
                if (!bb.empty()) std::memcpy(&outv[(i * (ca + cb) + ca) * len], &bb[i * cb * len], cb * len * 4);
            }
            return outv;
        };
        const size_t ncp = cov.cat_past ? cov.n_cat_past : 0, nck = cov.cat_known ? cov.n_cat_known : 0;
        const size_t np = cov.past ? cov.n_past : 0, nk = cov.known ? cov.n_known : 0;
        std::vector<float> past_rows = cat_channels(cov.past, np, enc_past, ncp, t);
        std::vector<float> known_rows = cat_channels(cov.known, nk, enc_known, nck, t + horizon);
        Rows rows;
        rows.n_past = np + ncp;
        rows.n_known = nk + nck;
        rows.past = past_rows.empty() ? nullptr : past_rows.data();
        rows.known = known_rows.empty() ? nullptr : known_rows.data();
        if (rows.n_past == 0 && rows.n_known == 0 && any_cov) fail(TSFM_ERR_INVALID_ARGUMENT, "InvalidInput");

        std::vector<float> res;
        if (o.symmetric_averaging) {
            for (size_t i = 0; i < q; ++i)
                if (std::fabs(knots[i] + knots[q - 1 - i] - 1.0) > 1e-9)
                    fail(TSFM_ERR_ASYMMETRIC_QUANTILES, "AsymmetricQuantiles");
            std::vector<float> neg(b * v * t), npast(past_rows.size()), nknown(known_rows.size());
            for (size_t i = 0; i < neg.size(); ++i) neg[i] = -inputs[i];
            for (size_t i = 0; i < npast.size(); ++i) npast[i] = -past_rows[i];
            for (size_t i = 0; i < nknown.size(); ++i) nknown[i] = -known_rows[i];
            Rows mrows = rows;
            mrows.past = npast.empty() ? nullptr : npast.data();
            mrows.known = nknown.empty() ? nullptr : nknown.data();
            res = forecast_raw(inputs, observed, b, v, t, horizon, rows, o);
            std::vector<float> mir = forecast_raw(neg.data(), observed, b, v, t, horizon, mrows, o);
            for (size_t i = 0; i < b * v * horizon; ++i) {
                float *a = &res[i * q];
                const float *m = &mir[i * q];
                for (size_t j = 0; j < q; ++j) a[j] = 0.5f * (a[j] + -m[q - 1 - j]);
            }
        } else {
            res = forecast_raw(inputs, observed, b, v, t, horizon, rows, o);
        }
        if (o.clip_nonnegative)
            for (size_t r = 0; r < b * v; ++r) {
                bool any = false, all_nonneg = true;
                for (size_t i = 0; i < t; ++i)
                    if (observed[r * t + i] && std::isfinite(inputs[r * t + i])) {
                        any = true;
                        all_nonneg = all_nonneg && inputs[r * t + i] >= 0;
                    }
                if (any && all_nonneg)
                    for (size_t k = 0; k < horizon * q; ++k)
                        res[r * horizon * q + k] = std::fmax(res[r * horizon * q + k], 0.0f);
            }
        std::memcpy(result, res.data(), res.size() * 4);
    }
};

}  // namespace

struct oracle_model {
    int32_t family = 0;
    std::unique_ptr<Chronos2> c2;
    std::unique_ptr<Bolt> bolt;
    std::unique_ptr<Timestral> ts;
};

template <class F>
static int32_t guarded(F &&f) {
    try {
        g_err.clear();
        f();
        return TSFM_OK;
    } catch (const Fail &e) {
        return e.code;
    } catch (const std::bad_alloc &) {
        g_err = "out of memory";
        return TSFM_ERR_OUT_OF_MEMORY;
    } catch (const std::exception &e) {
        g_err = e.what();
        return TSFM_ERR_INVALID_ARGUMENT;
    }
}

extern "C" {

int32_t oracle_set_threads(int32_t n) {
    if (n > 0) omp_set_num_threads(n);
    return TSFM_OK;
}
int32_t oracle_get_threads(void) { return omp_get_max_threads(); }
int32_t oracle_set_operand_emulation(int32_t scheme) {
    if (scheme < 0 || scheme > 7) return TSFM_ERR_INVALID_ARGUMENT;
    g_emul = scheme;
    for (int &c : g_emul_by_class) c = -1;
    g_emul_tf32_round = false;
    return TSFM_OK;
}
int32_t oracle_set_operand_emulation_tf32(int32_t round) {
    g_emul_tf32_round = round != 0;
    return TSFM_OK;
}
int32_t oracle_set_operand_emulation_class(int32_t cls, int32_t scheme) {
    if (cls < 1 || cls > 7 || scheme < -1 || scheme > 7) return TSFM_ERR_INVALID_ARGUMENT;
    g_emul_by_class[cls] = scheme;
    return TSFM_OK;
}
const char *oracle_last_error(void) { return g_err.c_str(); }

int32_t oracle_model_create(const tsfm_config *cfg, const tsfm_tensor *tensors, size_t n_tensors,
                            oracle_model **out) {
    return guarded([&] {
        if (!cfg || !out || (!tensors && n_tensors)) fail(TSFM_ERR_INVALID_ARGUMENT, "null argument");
        Table tab(tensors, n_tensors);
        auto m = std::make_unique<oracle_model>();
        m->family = cfg->family;
        std::vector<double> qs(cfg->quantiles, cfg->quantiles + cfg->num_quantiles);
        if (cfg->family == TSFM_CHRONOS2) {
            m->c2 = std::make_unique<Chronos2>();
            m->c2->c = *cfg;
            m->c2->quantiles = qs;
            m->c2->load(tab);
        } else if (cfg->family == TSFM_CHRONOS_BOLT) {
            m->bolt = std::make_unique<Bolt>();
            m->bolt->c = *cfg;
            m->bolt->quantiles = qs;
            m->bolt->load(tab);
        } else if (cfg->family == TSFM_TIMESTRAL) {
            m->ts = std::make_unique<Timestral>();
            m->ts->c = *cfg;
            m->ts->knots = qs;
            m->ts->kinds.assign(cfg->layer_kinds, cfg->layer_kinds + cfg->n_layer_kinds);
            m->ts->load(tab);
        } else {
            fail(TSFM_ERR_INVALID_CONFIG, "unknown family");
        }
        *out = m.release();
    });
}

void oracle_model_destroy(oracle_model *m) { delete m; }

int32_t oracle_forecast_chronos2(oracle_model *m, const float *inputs, size_t b, size_t t,
                                 size_t horizon, float *out) {
    return guarded([&] {
        if (!m || !m->c2) fail(TSFM_ERR_INVALID_ARGUMENT, "not a Chronos-2 model");
        m->c2->forecast(inputs, b, t, horizon, out);
    });
}

int32_t oracle_forecast_bolt(oracle_model *m, const float *inputs, size_t b, size_t t,
                             size_t horizon, float *out) {
    return guarded([&] {
        if (!m || !m->bolt) fail(TSFM_ERR_INVALID_ARGUMENT, "not a Chronos-Bolt model");
        m->bolt->forecast(inputs, b, t, horizon, out);
    });
}

int32_t oracle_forecast_timestral(oracle_model *m, const float *inputs, const uint8_t *observed,
                                  size_t b, size_t v, size_t t, size_t horizon,
                                  const tsfm_covariates *cov, const tsfm_timestral_options *opts,
                                  float *out) {
    return guarded([&] {
        if (!m || !m->ts) fail(TSFM_ERR_INVALID_ARGUMENT, "not a Timestral model");
        tsfm_timestral_options o;
        if (opts) {
            o = *opts;
        } else {
            o.max_context = 0;
            o.per_shot_horizon_patches = 32;
            o.quantile_real_cap_k = 1e4f;
            o.extreme_value_threshold = 1e30f;
            o.symmetric_averaging = 1;
            o.clip_nonnegative = 1;
        }
        if (o.per_shot_horizon_patches == 0) o.per_shot_horizon_patches = 1;
        m->ts->forecast(inputs, observed, b, v, t, horizon, cov, o, out);
    });
}

int32_t oracle_relative_bucket(int64_t rel, uint32_t num_buckets, uint32_t max_distance) {
    return (int32_t)relative_bucket(rel, num_buckets, max_distance);
}

float oracle_quantile_linear(const float *sorted, size_t n, float level) {
    return quantile_linear(sorted, n, level);
}

int32_t oracle_self_attend(int32_t mask, const float *q, const float *k, const float *v, float *o,
                           size_t ldq, size_t ldk, size_t ldv, size_t ldo, size_t n, size_t hd,
                           float scale, const uint8_t *key_valid, const float *bias) {
    return guarded([&] {
        std::vector<float> scores(n * n);
        self_attend((Mask)mask, scores.data(), q, k, v, o, ldq, ldk, ldv, ldo, n, hd, scale, key_valid,
                    bias);
    });
}

int32_t oracle_mask_pick(int32_t causal, int32_t all_keys_valid, int32_t additive) {
    return (int32_t)mask_pick(causal != 0, all_keys_valid != 0, additive != 0);
}

// encodingTarget + encodeCategorical (timestral/forecaster.zig:201-238) for one kind of
// categorical covariate: codes (b, nc, len), len = t (past) or t + horizon (known); out f32 of the
// same shape. With have_target == 0 the codes are only rounded.
int32_t oracle_target_encode(const float *inputs, const uint8_t *observed, size_t b, size_t t, size_t max_context,
                             const double *codes, size_t nc, size_t len, int32_t have_target, float *out) {
    std::vector<double> target(b * t);
    for (size_t s = 0; s < b; ++s) {
        bool started = false;
        float last = 0.0f;
        for (size_t i = 0; i < t; ++i) {
            if (observed[s * t + i]) {
                started = true;
                last = inputs[s * t + i];
            }
            const bool in_window = t <= max_context || i >= t - max_context;
            target[s * t + i] = started && in_window ? (double)last : std::nan("");
        }
    }
    for (size_t s = 0; s < b; ++s)
        for (size_t j = 0; j < nc; ++j) {
            const double *row = codes + (s * nc + j) * len;
            float *dst = out + (s * nc + j) * len;
            if (!have_target) {
                for (size_t i = 0; i < len; ++i) dst[i] = (float)row[i];
                continue;
            }
            Timestral::target_encode(&target[s * t], row, t, len > t ? row + t : nullptr, len - t, dst,
                                     len > t ? dst + t : nullptr);
            for (size_t i = 0; i < t; ++i)
                if (std::isnan(target[s * t + i]) && std::isnan(row[i])) dst[i] = std::nanf("");
        }
    return 0;
}

// series.parseBlocks (core/series.zig:21-68).
int32_t oracle_parse_blocks(const char *text, double *values, size_t cap, size_t *blocks_out,
                            size_t *rows_out, size_t *len_out) {
    std::vector<double> vals;
    size_t blocks = 0, rows_in_block = 0, rows = 0, len = 0;
    bool have_len = false;
    auto trim = [](const std::string &s, const char *ws) {
        const size_t a = s.find_first_not_of(ws);
        if (a == std::string::npos) return std::string();
        const size_t bpos = s.find_last_not_of(ws);
        return s.substr(a, bpos - a + 1);
    };
    auto parse_value = [&](const std::string &tok) {
        const std::string s = trim(tok, " \t\r");
        if (s.empty()) return std::nan("");
        char *end = nullptr;
        const double v = std::strtod(s.c_str(), &end);
        if (end != s.c_str() + s.size()) return std::nan("");
        return v;
    };
    std::string all(text);
    size_t pos = 0;
    while (true) {
        const size_t nl = all.find('\n', pos);
        const std::string raw = all.substr(pos, nl == std::string::npos ? std::string::npos : nl - pos);
        const std::string line = trim(raw, " \t\r");
        if (!line.empty() && line[0] == '#') {
        } else if (line.empty()) {
            if (rows_in_block > 0) {
                if (blocks == 0) rows = rows_in_block;
                else if (rows_in_block != rows) return 2;
                ++blocks;
                rows_in_block = 0;
            }
        } else {
            const size_t before = vals.size();
            if (line.find(',') != std::string::npos) {
                size_t p = 0;
                while (true) {
                    const size_t cpos = line.find(',', p);
                    vals.push_back(parse_value(line.substr(p, cpos == std::string::npos ? std::string::npos : cpos - p)));
                    if (cpos == std::string::npos) break;
                    p = cpos + 1;
                }
            } else {
                size_t p = 0;
                while (p < line.size()) {
                    while (p < line.size() && (line[p] == ' ' || line[p] == '\t')) ++p;
                    if (p >= line.size()) break;
                    size_t e = p;
                    while (e < line.size() && line[e] != ' ' && line[e] != '\t') ++e;
                    vals.push_back(parse_value(line.substr(p, e - p)));
                    p = e;
                }
            }
            const size_t n = vals.size() - before;
            if (!have_len) {
                len = n;
                have_len = true;
            } else if (n != len) {
                return 1;
            }
            ++rows_in_block;
        }
        if (nl == std::string::npos) break;
        pos = nl + 1;
    }
    if (rows_in_block > 0) {
        if (blocks == 0) rows = rows_in_block;
        else if (rows_in_block != rows) return 2;
        ++blocks;
    }
    if (blocks == 0 || len == 0) return 3;
    if (vals.size() > cap) return 4;
    std::memcpy(values, vals.data(), vals.size() * sizeof(double));
    *blocks_out = blocks;
    *rows_out = rows;
    *len_out = len;
    return 0;
}

int32_t oracle_linear(const float *x, const float *w, const float *bias, float *y, size_t rows,
                      size_t out, size_t in) {
    return guarded([&] {
        Weight wt;
        wt.init(std::vector<float>(w, w + out * in), out, in);
        linear(y, x, rows, wt, bias);
    });
}

int32_t oracle_chronos2_patch(const float *inputs, size_t b, size_t t_in, size_t context_length, size_t ps,
                              float tscale, int32_t arcsinh, float *loc, float *scale, float *feats,
                              uint8_t *key_valid) {
    return guarded([&] {
        const size_t t = std::min(t_in, context_length), pad = (ps - t % ps) % ps, n_ctx = (t + pad) / ps;
        c2_patch_features(inputs, t_in, t_in - t, t, pad, n_ctx, ps, tscale, arcsinh != 0, b, loc, scale, feats,
                          key_valid);
    });
}

int32_t oracle_bolt_patch(const float *inputs, size_t b, size_t t_in, size_t context_length, size_t ps,
                          int32_t use_reg, float *loc, float *scale, float *feats, uint8_t *key_valid) {
    return guarded([&] {
        const size_t len = std::min(t_in, context_length), pad = (ps - len % ps) % ps, n_patch = (len + pad) / ps;
        bolt_patch_features(inputs, t_in, t_in - len, len, pad, n_patch, ps, n_patch + (use_reg ? 1 : 0),
                            use_reg != 0, b, loc, scale, feats, key_valid);
    });
}

int32_t oracle_timestral_block_inputs(const float *full, const uint8_t *full_obs, size_t rows, size_t w, size_t ps,
                                      size_t vall, const int8_t *roles, int32_t cov, double min_scale,
                                      int32_t use_asinh, int32_t attend_missing, float *loc, float *scale,
                                      float *feats, uint8_t *key_valid, int32_t *first_obs) {
    return guarded([&] {
        if (ps == 0 || vall == 0 || rows % vall || w % ps) fail(TSFM_ERR_INVALID_ARGUMENT, "block geometry");
        std::vector<Role> rv(vall);
        for (size_t i = 0; i < vall; ++i) rv[i] = (Role)roles[i];
        ts_block_features(loc, scale, feats, full, full_obs, rows, w, ps, vall, rv, cov != 0, min_scale,
                          use_asinh != 0);
        std::vector<size_t> fo(rows / vall);
        ts_key_valid(key_valid, fo.data(), full_obs, rows, w, ps, vall, rows / vall, attend_missing != 0);
        for (size_t g = 0; g < fo.size(); ++g) first_obs[g] = (int32_t)fo[g];
    });
}

int32_t oracle_rmsnorm(const float *x, const float *scale, float *out, size_t rows, size_t dim,
                       float eps) {
    return guarded([&] { rms_norm(out, x, rows, dim, scale, eps); });
}

}  // extern "C"
