// Weight upload on the device: checkpoint tensors go up as stored (F32, F16 or BF16) and are
// converted, concatenated, row-permuted and folded by kernels, so loading costs one copy of the
// file bytes per device instead of host-side conversion loops (the device counterpart of the
// reference's F16/BF16 -> F32 loader, core/safetensors.zig:81-92).
#include "kernels.h"

#include <cuda_bf16.h>
#include <cuda_fp16.h>

namespace tsfm {

namespace {

__device__ __forceinline__ float load_src(const void *src, int dt, int64_t i) {
    if (dt == E_F32) return static_cast<const float *>(src)[i];
    if (dt == E_F16) return __half2float(static_cast<const __half *>(src)[i]);
    return __uint_as_float((uint32_t) static_cast<const uint16_t *>(src)[i] << 16);
}

// dst row r, column c = src row (map ? map[r] : r), column c, in the destination format:
// E_F16 (round to nearest even), E_BF16 (round to nearest even), E_F32 (TF32 operand: round to
// nearest, ties away, on the 13 dropped bits; non-finite values kept).
__global__ void convert_rows_kernel(const void *src, int src_dt, const int32_t *map, void *dst, int dst_dt, int64_t rows,
                                    int64_t cols) {
    const int64_t total = rows * cols;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = i / cols, c = i - r * cols;
        const int64_t sr = map ? (int64_t)map[r] : r;
        const float v = load_src(src, src_dt, sr * cols + c);
        if (dst_dt == E_F16) {
            static_cast<__half *>(dst)[i] = __float2half_rn(v);
        } else if (dst_dt == E_BF16) {
            static_cast<__nv_bfloat16 *>(dst)[i] = __float2bfloat16_rn(v);
        } else {
            uint32_t u = __float_as_uint(v);
            if ((u & 0x7f800000u) != 0x7f800000u) u = (u + 0x1000u) & ~0x1fffu;
            static_cast<float *>(dst)[i] = __uint_as_float(u);
        }
    }
}

// c = a (m x k) times b (k x n) in float64, rounded to float once, then to the destination
// format. The sum runs as two interleaved partial sums (even and odd k) added at the end, each
// term a separately rounded product, as the host reference of this product does.
__global__ void fold_f64_kernel(const void *a, int a_dt, const void *b, int b_dt, void *dst, int dst_dt, int64_t m,
                                int64_t k, int64_t n) {
    const int64_t i = blockIdx.y, j = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= m || j >= n) return;
    double s0 = 0.0, s1 = 0.0;
    int64_t x = 0;
    for (; x + 1 < k; x += 2) {
        s0 = __dadd_rn(s0, __dmul_rn((double)load_src(a, a_dt, i * k + x), (double)load_src(b, b_dt, x * n + j)));
        s1 = __dadd_rn(s1, __dmul_rn((double)load_src(a, a_dt, i * k + x + 1), (double)load_src(b, b_dt, (x + 1) * n + j)));
    }
    if (x < k) s0 = __dadd_rn(s0, __dmul_rn((double)load_src(a, a_dt, i * k + x), (double)load_src(b, b_dt, x * n + j)));
    const float v = (float)__dadd_rn(s0, s1);
    const int64_t o = i * n + j;
    if (dst_dt == E_F16)
        static_cast<__half *>(dst)[o] = __float2half_rn(v);
    else if (dst_dt == E_BF16)
        static_cast<__nv_bfloat16 *>(dst)[o] = __float2bfloat16_rn(v);
    else
        static_cast<float *>(dst)[o] = v;
}

}  // namespace

Status launch_convert_rows(const void *src, int src_dt, const int32_t *map, void *dst, int dst_dt, int64_t rows,
                           int64_t cols, cudaStream_t s) {
    if (rows <= 0 || cols <= 0) return Status::ok();
    const int64_t total = rows * cols;
    const int grid = (int)std::min<int64_t>((total + 255) / 256, (int64_t)num_sms() * 32);
    convert_rows_kernel<<<grid, 256, 0, s>>>(src, src_dt, map, dst, dst_dt, rows, cols);
    TSFM_CUDA(cudaGetLastError(), "weight conversion: launch");
    return Status::ok();
}

Status launch_fold_f64(const void *a, int a_dt, const void *b, int b_dt, void *dst, int dst_dt, int64_t m, int64_t k,
                       int64_t n, cudaStream_t s) {
    if (m <= 0 || n <= 0 || m > 65535) return Status::fail(TSFM_ERR_INVALID_ARGUMENT, "weight fold: bad shape");
    const dim3 grid((unsigned)((n + 127) / 128), (unsigned)m);
    fold_f64_kernel<<<grid, 128, 0, s>>>(a, a_dt, b, b_dt, dst, dst_dt, m, k, n);
    TSFM_CUDA(cudaGetLastError(), "weight fold: launch");
    return Status::ok();
}

}  // namespace tsfm
