// The reference's CUDA GEMM seam (platform/cuda/gemm.c:232-330) on this backend's tensor-core
// kernel: same four entry points, same host-pointer, row-major, padded-stride semantics, 0 on
// success. Each product is computed as three TF32 products of split operands
// (a = a_hi + a_lo, b = b_hi + b_lo; a b ~= a_hi b_hi + a_hi b_lo + a_lo b_hi) accumulated in
// FP32, which keeps FP32 SGEMM accuracy. Only the n columns of each output row are written, so
// the padding of a strided output survives (the reference's gpu_test.zig:18-23 sentinel check).
#include <cstring>
#include <memory>
#include <vector>

#include "runtime.h"

using namespace tsfm;

namespace {

struct SeamCtx {
    int device = -1;
    cudaStream_t stream = nullptr;
    DevBuf raw_a, raw_b, raw_bt, ahi, alo, bhi, blo, c;
    DevBuf err;
    PinnedBuf err_host;  // the error word's copy, read after the one synchronisation per call
    ~SeamCtx() {
        if (stream) cudaStreamDestroy(stream);
    }
};

thread_local std::unique_ptr<SeamCtx> g_ctx;

struct RegWeight {
    DevBuf data;
    size_t len = 0;
};

Status ctx(SeamCtx **out) {
    int dev = 0;
    TSFM_CUDA(cudaGetDevice(&dev), "cudaGetDevice");
    if (!g_ctx || g_ctx->device != dev) {
        g_ctx.reset(new SeamCtx());
        g_ctx->device = dev;
        TSFM_CUDA(cudaStreamCreateWithFlags(&g_ctx->stream, cudaStreamNonBlocking), "cudaStreamCreate");
        TSFM_TRY(g_ctx->err.alloc(16));
        TSFM_CUDA(cudaMemset(g_ctx->err.p, 0, 16), "clear error word");
        TSFM_TRY(g_ctx->err_host.ensure(16));
    }
    *out = g_ctx.get();
    return Status::ok();
}

Status grow(DevBuf &b, size_t n) { return n <= b.bytes ? Status::ok() : b.alloc(n); }

// Where B comes from: host rows [n, k] (NT), host rows [k, n] (NN), or the same on the device (a
// registered weight, read in place).
enum BSource { B_HOST_NK, B_HOST_KN, B_DEV_NK, B_DEV_KN };

// C[m, n] = alpha * A[m, k] B^T with B as [n, k] (or B as [k, n] for the NN forms, transposed on
// the device): A and C host rows (lda, ldc), B per `src` with row stride ldb.
Status sgemm_impl(int m, int n, int k, float alpha, const float *A, int lda, const float *B, int ldb, float *C, int ldc,
                  BSource src) {
    if (m <= 0 || n <= 0 || k <= 0) return Status::fail(TSFM_ERR_INVALID_ARGUMENT, "sgemm: empty product");
    const bool nk = src == B_HOST_NK || src == B_DEV_NK;
    if (!A || !B || !C || lda < k || ldb < (nk ? k : n) || ldc < n)
        return Status::fail(TSFM_ERR_INVALID_ARGUMENT, "sgemm: bad operands");
    SeamCtx *x = nullptr;
    TSFM_TRY(ctx(&x));
    const int64_t kp = (k + 3) / 4 * 4, np = (n + 3) / 4 * 4;
    TSFM_TRY(grow(x->raw_a, (size_t)m * k * 4));
    TSFM_TRY(grow(x->ahi, (size_t)m * kp * 4));
    TSFM_TRY(grow(x->alo, (size_t)m * kp * 4));
    TSFM_TRY(grow(x->bhi, (size_t)n * kp * 4));
    TSFM_TRY(grow(x->blo, (size_t)n * kp * 4));
    TSFM_TRY(grow(x->c, (size_t)m * np * 4));
    cudaStream_t s = x->stream;
    TSFM_CUDA(cudaMemcpy2DAsync(x->raw_a.p, (size_t)k * 4, A, (size_t)lda * 4, (size_t)k * 4, m, cudaMemcpyHostToDevice, s),
              "sgemm: copy A");
    // B as [n, k] rows at b_nk with stride ld_nk: in place (registered NT), copied (host NT), or
    // transposed on the device (NN).
    const float *b_nk = B;
    int64_t ld_nk = ldb;
    if (src == B_HOST_NK) {
        TSFM_TRY(grow(x->raw_b, (size_t)n * k * 4));
        TSFM_CUDA(cudaMemcpy2DAsync(x->raw_b.p, (size_t)k * 4, B, (size_t)ldb * 4, (size_t)k * 4, n,
                                    cudaMemcpyHostToDevice, s),
                  "sgemm: copy B");
        b_nk = static_cast<const float *>(x->raw_b.p);
        ld_nk = k;
    } else if (src != B_DEV_NK) {
        const float *b_kn = B;
        int64_t ld_kn = ldb;
        if (src == B_HOST_KN) {
            TSFM_TRY(grow(x->raw_bt, (size_t)k * n * 4));
            TSFM_CUDA(cudaMemcpy2DAsync(x->raw_bt.p, (size_t)n * 4, B, (size_t)ldb * 4, (size_t)n * 4, k,
                                        cudaMemcpyHostToDevice, s),
                      "sgemm: copy B");
            b_kn = static_cast<const float *>(x->raw_bt.p);
            ld_kn = n;
        }
        TSFM_TRY(grow(x->raw_b, (size_t)n * k * 4));
        TSFM_TRY(launch_transpose_f32(b_kn, k, n, ld_kn, static_cast<float *>(x->raw_b.p), k, s));
        b_nk = static_cast<const float *>(x->raw_b.p);
        ld_nk = k;
    }
    float *ahi = static_cast<float *>(x->ahi.p), *alo = static_cast<float *>(x->alo.p);
    float *bhi = static_cast<float *>(x->bhi.p), *blo = static_cast<float *>(x->blo.p);
    TSFM_TRY(launch_split_tf32(static_cast<const float *>(x->raw_a.p), m, k, k, alpha, ahi, alo, kp, s));
    TSFM_TRY(launch_split_tf32(b_nk, n, k, ld_nk, 1.0f, bhi, blo, kp, s));
    LinearCall lc;
    lc.dtype = E_F32;
    lc.M = m;
    lc.N = n;
    lc.K = kp;
    lc.ldx = kp;
    lc.ldw = kp;
    lc.y = x->c.p;
    lc.ldy = np;
    lc.err = static_cast<int *>(x->err.p);
    lc.x = alo;
    lc.w = bhi;
    lc.out_mode = OUT_F32;
    TSFM_TRY(launch_linear(lc, s));
    lc.x = ahi;
    lc.w = blo;
    lc.out_mode = OUT_F32_ACC;
    TSFM_TRY(launch_linear(lc, s));
    lc.x = ahi;
    lc.w = bhi;
    TSFM_TRY(launch_linear(lc, s));
    TSFM_CUDA(cudaMemcpy2DAsync(C, (size_t)ldc * 4, x->c.p, (size_t)np * 4, (size_t)n * 4, m, cudaMemcpyDeviceToHost, s),
              "sgemm: copy C");
    int *code = static_cast<int *>(x->err_host.p);
    TSFM_CUDA(cudaMemcpyAsync(code, x->err.p, 4, cudaMemcpyDeviceToHost, s), "sgemm: error word");
    TSFM_CUDA(cudaStreamSynchronize(s), "sgemm");
    if (*code) {
        const int site = *code;
        cudaMemset(x->err.p, 0, 4);
        *code = 0;
        return Status::fail(TSFM_ERR_DEVICE_TIMEOUT, strf("sgemm: a kernel wait gave up (site 0x%04x)", site));
    }
    return Status::ok();
}

// The seam keeps gemm.c's int return (0 = success); the message goes to tsfm_last_error().
int seam_status(const Status &st) { return set_last_error(st); }

}  // namespace

extern "C" {

void *tsfm_weight_register(const float *data, size_t len) {
    if (!data || len == 0) return nullptr;
    try {
        std::unique_ptr<RegWeight> w(new RegWeight());
        if (!w->data.alloc(len * 4)) return nullptr;
        if (cudaMemcpy(w->data.p, data, len * 4, cudaMemcpyHostToDevice) != cudaSuccess) return nullptr;
        w->len = len;
        return w.release();
    } catch (...) {
        return nullptr;
    }
}

void tsfm_weight_release(void *handle) { delete static_cast<RegWeight *>(handle); }

int tsfm_sgemm_nt(int m, int n, int k, float alpha, const float *A, int lda, const float *B, int ldb, float *C, int ldc,
                  void *b_buf) {
    try {
        if (b_buf) {
            RegWeight *w = static_cast<RegWeight *>(b_buf);
            if (n <= 0 || k <= 0 || (size_t)(n - 1) * ldb + k > w->len)
                return seam_status(Status::fail(TSFM_ERR_INVALID_ARGUMENT, "sgemm: registered weight too small"));
            return seam_status(sgemm_impl(m, n, k, alpha, A, lda, static_cast<const float *>(w->data.p), ldb, C, ldc,
                                          B_DEV_NK));
        }
        return seam_status(sgemm_impl(m, n, k, alpha, A, lda, B, ldb, C, ldc, B_HOST_NK));
    } catch (...) {
        return seam_status(Status::fail(TSFM_ERR_OUT_OF_MEMORY, "sgemm: host allocation failed"));
    }
}

int tsfm_sgemm_nn(int m, int n, int k, const float *A, int lda, const float *B, int ldb, float *C, int ldc, void *b_buf) {
    try {
        // B is [k, n] row-major: transposed to [n, k] on the device for the NT product (a registered
        // weight is read where it lives; it never returns to the host).
        if (b_buf) {
            RegWeight *w = static_cast<RegWeight *>(b_buf);
            if (n <= 0 || k <= 0 || (size_t)(k - 1) * ldb + n > w->len)
                return seam_status(Status::fail(TSFM_ERR_INVALID_ARGUMENT, "sgemm: registered weight too small"));
            return seam_status(sgemm_impl(m, n, k, 1.0f, A, lda, static_cast<const float *>(w->data.p), ldb, C, ldc,
                                          B_DEV_KN));
        }
        return seam_status(sgemm_impl(m, n, k, 1.0f, A, lda, B, ldb, C, ldc, B_HOST_KN));
    } catch (...) {
        return seam_status(Status::fail(TSFM_ERR_OUT_OF_MEMORY, "sgemm: host allocation failed"));
    }
}

}  // extern "C"
