// ORACLE — test infrastructure only (see oracle.h). Operand-rounding emulation for the precision
// study (oracle_set_operand_emulation): the same FP32 products as the restatement, computed from
// operands rounded the way a reduced-precision tensor-core product consumes them. Scheme 0 (the
// default) is never routed here; the reference's FP32 arithmetic is untouched.
//
// Schemes for products whose device operands are 16-bit (x [rows, in], w [out, in], y = x w^T):
//   1  FP16 operands                               y = f16(x) f16(w)
//   2  FP16 + FP8 corrections                      y = x_hi w_hi + e4m3(x_hi) e4m3(w_lo) + e4m3(x_lo) e4m3(w_hi)
//   3  FP16, three products (split x and w)         y = x_hi w_hi + f16(x_lo) w_hi + x_hi f16(w_lo)
//   4  FP16, weight split only                      y = x_hi w_hi + x_hi f16(w_lo)
//   5  BF16 operands                               y = bf16(x) bf16(w)
//   6  FP16 + FP8 weight correction only            y = x_hi w_hi + e4m3(x_hi) e4m3(w_lo)
//   7  FP16 + FP8 input correction only             y = x_hi w_hi + e4m3(x_lo) e4m3(w_hi)
// with x_hi = f16(x), x_lo = x - x_hi, w_hi = f16(w), w_lo = w - w_hi (both differences exact in
// FP32). The FP8 operands carry power-of-two scales: e4m3(x_hi 2^-5), e4m3(x_lo 2^7),
// e4m3(w_lo 2^sb), e4m3(w_hi 2^(sb-12)), sb = min(floor(log2(448 / max|w_lo|)),
// floor(log2(448 / max|w|)) + 12), so every correction product carries the scale 2^(sb-5) and the
// FP16 product's weight w_hi 2^(sb-5) stays within FP16's range (at most 448 * 128 = 57344).
// Products with TF32 device operands round both operands to TF32 (round to nearest, ties away) in
// schemes 1 and 5, and in the other schemes when `tf32_round` is set (FP32 otherwise).
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <vector>

namespace oracle {

void matmul_nt_packed(const float *x, const float *wt, float *y, size_t rows, size_t out, size_t in,
                      float alpha);

float round_f16(float x) { return (float)(_Float16)x; }

float round_bf16(float x) {
    uint32_t u;
    std::memcpy(&u, &x, 4);
    if ((u & 0x7f800000u) != 0x7f800000u) u = (u + 0x7fffu + ((u >> 16) & 1u)) & 0xffff0000u;
    float r;
    std::memcpy(&r, &u, 4);
    return r;
}

float round_tf32(float x) {
    uint32_t u;
    std::memcpy(&u, &x, 4);
    if ((u & 0x7f800000u) != 0x7f800000u) u = (u + 0x1000u) & ~0x1fffu;
    float r;
    std::memcpy(&r, &u, 4);
    return r;
}

// Round to a binary format with `mbits` stored mantissa bits and smallest normal exponent `emin`
// (subnormals below), nearest-even, saturating at +-maxv (the satfinite conversion).
static float round_small(float x, int mbits, int emin, float maxv) {
    if (x == 0.0f || !std::isfinite(x)) return x;
    const float a = std::fabs(x);
    int e;
    std::frexp(a, &e);
    const int ex = std::max(e - 1, emin);
    const float ulp = std::ldexp(1.0f, ex - mbits);
    float r = std::nearbyint(a / ulp) * ulp;
    if (r > maxv) r = maxv;
    return std::copysign(r, x);
}

float round_e4m3(float x) { return round_small(x, 3, -6, 448.0f); }

static int floor_log2(double v) { return (int)std::floor(std::log2(v)); }

// y[rows, out] = x w^T under `scheme`; `tf32` marks a product with TF32 device operands.
void emul_matmul(float *y, const float *x, size_t rows, const float *w, size_t out, size_t in, int scheme,
                 bool tf32, bool tf32_round) {
    const size_t nx = rows * in, nw = out * in;
    std::vector<float> wt(nw), xa(nx), wa(nw);
    auto transpose_into = [&](const std::vector<float> &src, std::vector<float> &dst) {
        for (size_t r = 0; r < out; ++r)
            for (size_t c = 0; c < in; ++c) dst[c * out + r] = src[r * in + c];
    };
    if (tf32) {
        const bool round = scheme == 1 || scheme == 5 || tf32_round;
        for (size_t i = 0; i < nw; ++i) wa[i] = round ? round_tf32(w[i]) : w[i];
        for (size_t i = 0; i < nx; ++i) xa[i] = round ? round_tf32(x[i]) : x[i];
        transpose_into(wa, wt);
        matmul_nt_packed(xa.data(), wt.data(), y, rows, out, in, 1.0f);
        return;
    }
    if (scheme == 1 || scheme == 5) {
        auto rnd = scheme == 1 ? round_f16 : round_bf16;
        for (size_t i = 0; i < nw; ++i) wa[i] = rnd(w[i]);
        for (size_t i = 0; i < nx; ++i) xa[i] = rnd(x[i]);
        transpose_into(wa, wt);
        matmul_nt_packed(xa.data(), wt.data(), y, rows, out, in, 1.0f);
        return;
    }
    // Split schemes: the FP16 main product first.
    std::vector<float> w_lo(nw), x_lo(nx);
    float m = 0.0f, m_lo = 0.0f;
    for (size_t i = 0; i < nw; ++i) {
        wa[i] = round_f16(w[i]);
        w_lo[i] = w[i] - wa[i];
        m = std::max(m, std::fabs(wa[i]));
        m_lo = std::max(m_lo, std::fabs(w_lo[i]));
    }
    for (size_t i = 0; i < nx; ++i) {
        xa[i] = round_f16(x[i]);
        x_lo[i] = x[i] - xa[i];
    }
    transpose_into(wa, wt);
    matmul_nt_packed(xa.data(), wt.data(), y, rows, out, in, 1.0f);
    std::vector<float> part(rows * out), xc(nx), wc(nw);
    auto add_part = [&]() {
        for (size_t i = 0; i < rows * out; ++i) y[i] += part[i];
    };
    const bool corr_w = scheme == 2 || scheme == 3 || scheme == 4 || scheme == 6;
    const bool corr_x = scheme == 2 || scheme == 3 || scheme == 7;
    const bool fp8 = scheme == 2 || scheme == 6 || scheme == 7;
    int sb = 0;
    if (fp8) {
        sb = m > 0.0f ? floor_log2(448.0 / m) + 12 : 0;
        if (m_lo > 0.0f) sb = std::min(sb, floor_log2(448.0 / m_lo));
    }
    if (corr_w) {  // x_hi w_lo
        if (fp8) {
            const float sw = std::ldexp(1.0f, sb), sx = std::ldexp(1.0f, -5);
            for (size_t i = 0; i < nw; ++i) wc[i] = round_e4m3(w_lo[i] * sw) / sw;
            for (size_t i = 0; i < nx; ++i) xc[i] = round_e4m3(xa[i] * sx) / sx;
        } else {
            for (size_t i = 0; i < nw; ++i) wc[i] = round_f16(w_lo[i]);
            xc = xa;
        }
        transpose_into(wc, wt);
        matmul_nt_packed(xc.data(), wt.data(), part.data(), rows, out, in, 1.0f);
        add_part();
    }
    if (corr_x) {  // x_lo w_hi
        if (fp8) {
            const float sw = std::ldexp(1.0f, sb - 12), sx = std::ldexp(1.0f, 7);
            for (size_t i = 0; i < nw; ++i) wc[i] = round_e4m3(wa[i] * sw) / sw;
            for (size_t i = 0; i < nx; ++i) xc[i] = round_e4m3(x_lo[i] * sx) / sx;
        } else {
            wc = wa;
            for (size_t i = 0; i < nx; ++i) xc[i] = round_f16(x_lo[i]);
        }
        transpose_into(wc, wt);
        matmul_nt_packed(xc.data(), wt.data(), part.data(), rows, out, in, 1.0f);
        add_part();
    }
}

// The 16-bit storage of attention operands (q, k, v after RoPE; probabilities) under `scheme`.
float emul_store16(float v, int scheme) { return scheme == 5 ? round_bf16(v) : round_f16(v); }

}  // namespace oracle
