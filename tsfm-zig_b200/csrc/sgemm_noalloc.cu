// tsfm_sgemm_nt_noalloc: the FP32-accurate (split-TF32) product of the GEMM seam for callers that
// cannot allocate device memory. Some hosts of this library must not call cudaMalloc once they
// are running: cudaMalloc and cudaFree synchronise the whole device (stalling every other stream a
// latency-bound serving loop keeps busy), allocation-free real-time loops forbid them after
// start-up, and processes that hand all device memory to their own pool leave nothing for a
// library to take. This entry point allocates nothing: its scratch (the hi/lo TF32 splits of A and
// B, and the device error word) lives in the file-scope array below, a fixed 16 MiB that every GPU
// which loads the library holds until the process exits.
//
// Limits and sharing: the array holds the error word (256 bytes) and four split operands, A's hi and
// lo parts of m * round_up(k, 4) floats and B's of n * round_up(k, 4), each sub-buffer rounded up
// to 64 floats (256 bytes). So a product fits when
//   round_up(m * round_up(k, 4), 64) + round_up(n * round_up(k, 4), 64) <= 2^21 - 64 floats
// (for k a multiple of 64: m + n <= 32767); larger products are rejected with
// TSFM_ERR_INVALID_ARGUMENT before anything runs. Every call shares the one array and its contents
// persist from the previous call, so the error word is cleared on entry; calls that overlap on the
// GPU (other host threads, or other streams) race on the array.
//
// Set-up: the first call on each device looks up the array's device address with
// cudaGetSymbolAddress (with that device current) and caches it; that lookup may load this
// library's device code onto the device, so make the first call before any stream capture.
#include <mutex>

#include "runtime.h"

using namespace tsfm;

namespace {

constexpr size_t kScratchBytes = size_t(16) << 20;          // 16 MiB
constexpr size_t kHeaderBytes = 256;                          // device error word + padding
// Floats for one hi and one lo part of each operand, sub-buffers in 64-float steps: 2^21 - 64.
constexpr int64_t kMaxPartFloats = (int64_t)((kScratchBytes - kHeaderBytes) / sizeof(float) / 2) / 64 * 64;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kScratchBytes];

std::mutex g_mu;
void *g_addr[64] = {nullptr};

// Device address of the scratch array on the current device (looked up once per device).
Status scratch_address(void **out) {
    int dev = 0;
    TSFM_CUDA(cudaGetDevice(&dev), "cudaGetDevice");
    if (dev < 0 || dev >= 64) return Status::fail(TSFM_ERR_NO_DEVICE, "device ordinal out of range");
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g_addr[dev]) {
        void *p = nullptr;
        TSFM_CUDA(cudaGetSymbolAddress(&p, g_noalloc_scratch), "cudaGetSymbolAddress(scratch)");
        g_addr[dev] = p;
    }
    *out = g_addr[dev];
    return Status::ok();
}

Status run(int m, int n, int k, float alpha, const float *A, int lda, const float *B, int ldb, float *C, int ldc,
           cudaStream_t s) {
    if (m <= 0 || n <= 0 || k <= 0) return Status::fail(TSFM_ERR_INVALID_ARGUMENT, "sgemm_noalloc: empty product");
    if (!A || !B || !C || lda < k || ldb < k || ldc < n)
        return Status::fail(TSFM_ERR_INVALID_ARGUMENT, "sgemm_noalloc: bad operands");
    const int64_t kp = (k + 3) / 4 * 4;  // TF32 rows padded to 16-byte strides for the tensor map
    const int64_t need_m = (int64_t)m * kp, need_n = (int64_t)n * kp;
    const auto span = [](int64_t floats) { return (floats + 63) / 64 * 64; };  // 256-byte sub-buffers
    if (span(need_m) + span(need_n) > kMaxPartFloats)
        return Status::fail(TSFM_ERR_INVALID_ARGUMENT,
                            strf("sgemm_noalloc: round_up(m*round_up(k,4),64) + round_up(n*round_up(k,4),64) = %lld "
                                 "exceeds the scratch limit of %lld floats",
                                 (long long)(span(need_m) + span(need_n)), (long long)kMaxPartFloats));
    void *base = nullptr;
    TSFM_TRY(scratch_address(&base));
    int *err = static_cast<int *>(base);
    float *split = reinterpret_cast<float *>(static_cast<char *>(base) + kHeaderBytes);
    float *ahi = split, *alo = ahi + span(need_m), *bhi = alo + span(need_m), *blo = bhi + span(need_n);
    TSFM_CUDA(cudaMemsetAsync(err, 0, sizeof(int), s), "sgemm_noalloc: clear error word");
    TSFM_TRY(launch_split_tf32(A, m, k, lda, alpha, ahi, alo, kp, s));
    TSFM_TRY(launch_split_tf32(B, n, k, ldb, 1.0f, bhi, blo, kp, s));
    LinearCall lc;
    lc.dtype = E_F32;
    lc.M = m;
    lc.N = n;
    lc.K = kp;
    lc.ldx = kp;
    lc.ldw = kp;
    lc.y = C;
    lc.ldy = ldc;
    lc.err = err;
    lc.x = alo;  // smallest terms first
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
    int code = 0;
    TSFM_CUDA(cudaMemcpyAsync(&code, err, sizeof(int), cudaMemcpyDeviceToHost, s), "sgemm_noalloc: read error word");
    TSFM_CUDA(cudaStreamSynchronize(s), "sgemm_noalloc");
    if (code) return Status::fail(TSFM_ERR_DEVICE_TIMEOUT, strf("sgemm_noalloc: a kernel wait gave up (site 0x%04x)", code));
    return Status::ok();
}

}  // namespace

extern "C" {

int32_t tsfm_sgemm_nt_noalloc(int m, int n, int k, float alpha, const float *A, int lda, const float *B, int ldb,
                              float *C, int ldc, void *stream) {
    try {
        return set_last_error(run(m, n, k, alpha, A, lda, B, ldb, C, ldc, static_cast<cudaStream_t>(stream)));
    } catch (...) {
        return set_last_error(Status::fail(TSFM_ERR_INVALID_ARGUMENT, "sgemm_noalloc: unexpected exception"));
    }
}

}  // extern "C"
