// The reference's CUDA GEMM seam (platform/cuda/gemm.c:232-330) on this backend's tensor-core
// kernel: same four entry points, same host-pointer, row-major, padded-stride semantics, 0 on
// success. Each product is computed as three TF32 products of split operands
// (a = a_hi + a_lo, b = b_hi + b_lo; a b ~= a_hi b_hi + a_hi b_lo + a_lo b_hi) accumulated in
// FP32, which keeps FP32 SGEMM accuracy. Only the n columns of each output row are written, so
// the padding of a strided output survives (the reference's gpu_test.zig:18-23 sentinel check).
#include <cstring>
#include <vector>

#include "runtime.h"

using namespace tsfm;

namespace {

struct SeamCtx {
    int device = -1;
    cudaStream_t stream = nullptr;
    DevBuf raw_a, raw_b, ahi, alo, bhi, blo, c;
    DevBuf err;
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
    }
    *out = g_ctx.get();
    return Status::ok();
}

Status grow(DevBuf &b, size_t n) { return n <= b.bytes ? Status::ok() : b.alloc(n); }

// C[m, n] = alpha * A[m, k] B[n, k]^T; `b_rows` is B as [n, k] (ldb), on the device when
// b_is_device.
Status sgemm_nt_impl(int m, int n, int k, float alpha, const float *A, int lda, const float *B, int ldb, float *C,
                     int ldc, bool b_is_device) {
    if (m <= 0 || n <= 0 || k <= 0) return Status::fail(TSFM_ERR_INVALID_ARGUMENT, "sgemm: empty product");
    if (!A || !B || !C || lda < k || ldb < k || ldc < n) return Status::fail(TSFM_ERR_INVALID_ARGUMENT, "sgemm: bad operands");
    SeamCtx *x = nullptr;
    TSFM_TRY(ctx(&x));
    const int64_t kp = (k + 3) / 4 * 4, np = (n + 3) / 4 * 4;
    TSFM_TRY(grow(x->raw_a, (size_t)m * k * 4));
    TSFM_TRY(grow(x->raw_b, (size_t)n * k * 4));
    TSFM_TRY(grow(x->ahi, (size_t)m * kp * 4));
    TSFM_TRY(grow(x->alo, (size_t)m * kp * 4));
    TSFM_TRY(grow(x->bhi, (size_t)n * kp * 4));
    TSFM_TRY(grow(x->blo, (size_t)n * kp * 4));
    TSFM_TRY(grow(x->c, (size_t)m * np * 4));
    cudaStream_t s = x->stream;
    TSFM_CUDA(cudaMemcpy2DAsync(x->raw_a.p, (size_t)k * 4, A, (size_t)lda * 4, (size_t)k * 4, m, cudaMemcpyHostToDevice, s),
              "sgemm: copy A");
    TSFM_CUDA(cudaMemcpy2DAsync(x->raw_b.p, (size_t)k * 4, B, (size_t)ldb * 4, (size_t)k * 4, n,
                                b_is_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice, s),
              "sgemm: copy B");
    float *ahi = static_cast<float *>(x->ahi.p), *alo = static_cast<float *>(x->alo.p);
    float *bhi = static_cast<float *>(x->bhi.p), *blo = static_cast<float *>(x->blo.p);
    TSFM_TRY(launch_split_tf32(static_cast<const float *>(x->raw_a.p), m, k, k, alpha, ahi, alo, kp, s));
    TSFM_TRY(launch_split_tf32(static_cast<const float *>(x->raw_b.p), n, k, k, 1.0f, bhi, blo, kp, s));
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
    TSFM_CUDA(cudaStreamSynchronize(s), "sgemm");
    int code = 0;
    TSFM_CUDA(cudaMemcpy(&code, x->err.p, 4, cudaMemcpyDeviceToHost), "sgemm: error word");
    if (code) {
        cudaMemset(x->err.p, 0, 4);
        return Status::fail(TSFM_ERR_DEVICE_TIMEOUT, strf("sgemm: a kernel wait gave up (site 0x%04x)", code));
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
            if ((size_t)(n - 1) * ldb + k > w->len) return seam_status(Status::fail(TSFM_ERR_INVALID_ARGUMENT, "sgemm: registered weight too small"));
            return seam_status(sgemm_nt_impl(m, n, k, alpha, A, lda, static_cast<const float *>(w->data.p), ldb, C, ldc, true));
        }
        return seam_status(sgemm_nt_impl(m, n, k, alpha, A, lda, B, ldb, C, ldc, false));
    } catch (...) {
        return seam_status(Status::fail(TSFM_ERR_OUT_OF_MEMORY, "sgemm: host allocation failed"));
    }
}

int tsfm_sgemm_nn(int m, int n, int k, const float *A, int lda, const float *B, int ldb, float *C, int ldc, void *b_buf) {
    try {
        if (m <= 0 || n <= 0 || k <= 0 || !A || !C || ldb < n)
            return seam_status(Status::fail(TSFM_ERR_INVALID_ARGUMENT, "sgemm: bad operands"));
        // B is [k, n] row-major: transpose to [n, k] for the NT product.
        std::vector<float> host_b;
        const float *src = B;
        if (b_buf) {
            RegWeight *w = static_cast<RegWeight *>(b_buf);
            if ((size_t)(k - 1) * ldb + n > w->len) return seam_status(Status::fail(TSFM_ERR_INVALID_ARGUMENT, "sgemm: registered weight too small"));
            host_b.resize((size_t)(k - 1) * ldb + n);
            if (cudaMemcpy(host_b.data(), w->data.p, host_b.size() * 4, cudaMemcpyDeviceToHost) != cudaSuccess)
                return seam_status(Status::fail(TSFM_ERR_CUDA, "sgemm: read registered weight"));
            src = host_b.data();
        }
        if (!src) return seam_status(Status::fail(TSFM_ERR_INVALID_ARGUMENT, "sgemm: null B"));
        std::vector<float> bt((size_t)n * k);
        for (int p = 0; p < k; ++p)
            for (int j = 0; j < n; ++j) bt[(size_t)j * k + p] = src[(size_t)p * ldb + j];
        return seam_status(sgemm_nt_impl(m, n, k, 1.0f, A, lda, bt.data(), k, C, ldc, false));
    } catch (...) {
        return seam_status(Status::fail(TSFM_ERR_OUT_OF_MEMORY, "sgemm: host allocation failed"));
    }
}

}  // extern "C"
