// ORACLE — test infrastructure only (see oracle.h). The FP32 matrix product of the CPU
// restatement: y[r, j] = sum_k x[r, k] * w[j, k], each output element reduced sequentially over k
// with fused multiply-adds (the reference's builtin kernel uses @mulAdd, core/nn.zig:95), by exactly
// one thread, so the result does not depend on the thread count (core/nn.zig:285-288).
//
// This file is compiled with -ffp-contract=fast; the rest of the oracle uses strict FP32 order.
#include <cstddef>
#include <cstring>
#include <omp.h>

namespace oracle {

typedef float v8 __attribute__((vector_size(32), aligned(4)));

static inline v8 load8(const float *p) {
    v8 v;
    std::memcpy(&v, p, sizeof(v));
    return v;
}
static inline void store8(float *p, v8 v) { std::memcpy(p, &v, sizeof(v)); }

// wt is w transposed: wt[k * out + j] = w[j * in + k].
static void tile_4x16(const float *x, size_t in, const float *wt, size_t out, float *y, size_t r,
                      size_t c, float alpha) {
    v8 acc[4][2];
    for (int i = 0; i < 4; ++i) acc[i][0] = acc[i][1] = (v8){0, 0, 0, 0, 0, 0, 0, 0};
    const float *x0 = x + (r + 0) * in, *x1 = x + (r + 1) * in, *x2 = x + (r + 2) * in,
                *x3 = x + (r + 3) * in;
    for (size_t k = 0; k < in; ++k) {
        const v8 b0 = load8(wt + k * out + c), b1 = load8(wt + k * out + c + 8);
        const float a0 = x0[k], a1 = x1[k], a2 = x2[k], a3 = x3[k];
        acc[0][0] += a0 * b0; acc[0][1] += a0 * b1;
        acc[1][0] += a1 * b0; acc[1][1] += a1 * b1;
        acc[2][0] += a2 * b0; acc[2][1] += a2 * b1;
        acc[3][0] += a3 * b0; acc[3][1] += a3 * b1;
    }
    for (int i = 0; i < 4; ++i) {
        store8(y + (r + i) * out + c, acc[i][0] * alpha);
        store8(y + (r + i) * out + c + 8, acc[i][1] * alpha);
    }
}

static void tile_1x16(const float *x, size_t in, const float *wt, size_t out, float *y, size_t r,
                      size_t c, float alpha) {
    v8 a0 = (v8){0, 0, 0, 0, 0, 0, 0, 0}, a1 = a0;
    const float *xr = x + r * in;
    for (size_t k = 0; k < in; ++k) {
        const float a = xr[k];
        a0 += a * load8(wt + k * out + c);
        a1 += a * load8(wt + k * out + c + 8);
    }
    store8(y + r * out + c, a0 * alpha);
    store8(y + r * out + c + 8, a1 * alpha);
}

static void scalar_cell(const float *x, size_t in, const float *wt, size_t out, float *y, size_t r,
                        size_t c, float alpha) {
    float s = 0.0f;
    const float *xr = x + r * in;
    for (size_t k = 0; k < in; ++k) s += xr[k] * wt[k * out + c];
    y[r * out + c] = alpha * s;
}

// y[rows, out] = alpha * x[rows, in] @ w^T, with wt = w^T ([in, out]).
void matmul_nt_packed(const float *x, const float *wt, float *y, size_t rows, size_t out, size_t in,
                      float alpha) {
    const size_t RB = 16, CB = 64;
    const size_t nrb = (rows + RB - 1) / RB, ncb = (out + CB - 1) / CB;
    const long total = (long)(nrb * ncb);
#pragma omp parallel for schedule(static) if (rows * out * in >= (1u << 18))
    for (long t = 0; t < total; ++t) {
        const size_t rb = (size_t)t / ncb, cb = (size_t)t % ncb;
        const size_t r0 = rb * RB, r1 = r0 + RB < rows ? r0 + RB : rows;
        const size_t c0 = cb * CB, c1 = c0 + CB < out ? c0 + CB : out;
        size_t c = c0;
        for (; c + 16 <= c1; c += 16) {
            size_t r = r0;
            for (; r + 4 <= r1; r += 4) tile_4x16(x, in, wt, out, y, r, c, alpha);
            for (; r < r1; ++r) tile_1x16(x, in, wt, out, y, r, c, alpha);
        }
        for (; c < c1; ++c)
            for (size_t r = r0; r < r1; ++r) scalar_cell(x, in, wt, out, y, r, c, alpha);
    }
}

}  // namespace oracle
