#include "ops.h"

namespace tsfm {

Status load_resblock(Replica &r, const TensorTable &t, const std::string &prefix, int64_t in, int64_t hid,
                     int64_t out, bool bias, int in_dtype, int hidden_dtype, DResBlock &dst) {
    std::vector<float> w;
    TSFM_TRY(t.get(prefix + ".hidden_layer.weight", hid * in, w));
    TSFM_TRY(upload_lin(r, w, hid, in, in_dtype, dst.hidden));
    TSFM_TRY(t.get(prefix + ".output_layer.weight", out * hid, w));
    TSFM_TRY(upload_lin(r, w, out, hid, hidden_dtype, dst.output));
    TSFM_TRY(t.get(prefix + ".residual_layer.weight", out * in, w));
    TSFM_TRY(upload_lin(r, w, out, in, in_dtype, dst.residual));
    if (bias) {
        TSFM_TRY(t.get(prefix + ".hidden_layer.bias", hid, w));
        TSFM_TRY(upload_bias(r, w, dst.hidden));
        TSFM_TRY(t.get(prefix + ".output_layer.bias", out, w));
        TSFM_TRY(upload_bias(r, w, dst.output));
        TSFM_TRY(t.get(prefix + ".residual_layer.bias", out, w));
        TSFM_TRY(upload_bias(r, w, dst.residual));
    }
    return Status::ok();
}

Status op_linear(Replica &r, cudaStream_t s, const DLin &L, const void *x, int64_t M, int64_t ldx, void *y, int64_t ldy,
              int out_mode, int act, const LinearCall *extra) {
    LinearCall c;
    if (extra) c = *extra;
    c.x = x;
    c.w = L.w;
    c.dtype = L.dtype;
    c.M = M;
    c.N = L.out;
    c.K = L.in;
    c.ldx = ldx;
    c.ldw = L.in;
    c.y = y;
    c.ldy = ldy;
    c.out_mode = out_mode;
    c.bias = L.b;
    c.act = act;
    c.err = static_cast<int *>(r.err.p);
    // A corrected weight needs its activation's FP8 companion; a plain weight ignores one.
    if (L.w8) {
        if (!c.x8) return Status::fail(TSFM_ERR_INVALID_ARGUMENT, "linear: a corrected weight needs the input's FP8 companion");
        c.w8 = L.w8;
        c.ldw8 = 2 * L.in;
        c.acc_scale = L.acc_scale;
    } else {
        c.x8 = nullptr;
    }
    LaunchScope ls(r, s, K_GEMM, 2.0 * (double)M * (double)L.out * (double)L.in);
    return launch_linear(c, s);
}

Status op_rmsnorm(Replica &r, cudaStream_t s, const float *x, const float *scale, void *out, int out_mode, int64_t rows,
               int64_t dim, float eps, int64_t g, int64_t G, int64_t off, float *inv_out, void *out8) {
    RmsNormCall c;
    c.inv_out = inv_out;
    c.out8 = out8;
    c.ld8 = 2 * dim;
    c.x = x;
    c.scale = scale;
    c.out = out;
    c.out_mode = out_mode;
    c.rows = rows;
    c.dim = dim;
    c.eps = eps;
    c.g = g;
    c.G = G;
    c.off = off;
    LaunchScope ls(r, s, K_NORM, (double)rows * dim * (4.0 + (out_mode == OUT_F16 || out_mode == OUT_BF16 ? 2.0 : 4.0) +
                                                       (out8 ? 2.0 : 0.0)));
    return launch_rmsnorm(c, s);
}


Status check_resblock(const TensorTable &t, const std::string &p, int64_t in, int64_t hid, int64_t out, bool bias) {
    TSFM_TRY(t.check(p + ".hidden_layer.weight", hid * in));
    TSFM_TRY(t.check(p + ".output_layer.weight", out * hid));
    TSFM_TRY(t.check(p + ".residual_layer.weight", out * in));
    if (bias) {
        TSFM_TRY(t.check(p + ".hidden_layer.bias", hid));
        TSFM_TRY(t.check(p + ".output_layer.bias", out));
        TSFM_TRY(t.check(p + ".residual_layer.bias", out));
    }
    return Status::ok();
}

Status op_linear3(Replica &r, cudaStream_t s, const DLin3 &L, const float *x_hi, const float *x_lo, int64_t M,
                  int64_t ldx, float *y, int64_t ldy, bool accumulate, int act) {
    DLin hi_nobias = L.hi;
    hi_nobias.b = nullptr;
    TSFM_TRY(op_linear(r, s, hi_nobias, x_lo, M, ldx, y, ldy, accumulate ? OUT_F32_ACC : OUT_F32, 0));
    TSFM_TRY(op_linear(r, s, L.lo, x_hi, M, ldx, y, ldy, OUT_F32_ACC, 0));
    return op_linear(r, s, L.hi, x_hi, M, ldx, y, ldy, OUT_F32_ACC, act);
}

Status op_split(Replica &r, cudaStream_t s, float *x, float *x_lo, int64_t rows, int64_t cols, int64_t ld) {
    LaunchScope ls(r, s, K_OTHER, (double)rows * cols * 12.0);
    return launch_split_tf32(x, rows, cols, ld, 1.0f, x, x_lo, ld, s);
}

size_t workspace_budget(Replica &r) {
    size_t free_b = 0, total_b = 0;
    if (cudaMemGetInfo(&free_b, &total_b) != cudaSuccess) return r.ws.buf.bytes;
    return (size_t)(0.6 * (double)(free_b + r.ws.buf.bytes));
}

}  // namespace tsfm
