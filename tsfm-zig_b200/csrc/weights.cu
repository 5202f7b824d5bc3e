// Weight upload on the device: checkpoint tensors go up as stored (F32, F16 or BF16) and are
// converted, concatenated, row-permuted and folded by kernels, so loading costs one copy of the
// file bytes per device instead of host-side conversion loops (the device counterpart of the
// reference's F16/BF16 -> F32 loader, core/safetensors.zig:81-92).
#include "kernels.h"
#include "ptx.cuh"

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <cmath>
#include <cstring>

namespace tsfm {

namespace {

__device__ __forceinline__ float load_src(const void *src, int dt, int64_t i) {
    if (dt == E_F32) return static_cast<const float *>(src)[i];
    if (dt == E_F16) return __half2float(static_cast<const __half *>(src)[i]);
    return __uint_as_float((uint32_t) static_cast<const uint16_t *>(src)[i] << 16);
}

// dst row r, column c = src row (map ? map[r] : r), column c, in the destination format:
// E_F16 (round to nearest even), E_BF16 (round to nearest even), E_F32 (TF32 operand: round to
// nearest, ties away, on the 13 dropped bits; non-finite values kept), E_F32X (exact).
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
        } else if (dst_dt == E_F32X) {
            static_cast<float *>(dst)[i] = v;
        } else {
            uint32_t u = __float_as_uint(v);
            if ((u & 0x7f800000u) != 0x7f800000u) u = (u + 0x1000u) & ~0x1fffu;
            static_cast<float *>(dst)[i] = __uint_as_float(u);
        }
    }
}

// Range of a weight for its corrected form: mx[0] = max |f16(w)|, mx[1] = max |w - f16(w)| (as
// float bits; non-negative floats order like their bits).
__global__ void corr_range_kernel(const float *w, int64_t n, unsigned *mx) {
    float m = 0.0f, ml = 0.0f;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const float x = w[i];
        const float h = __half2float(__float2half_rn(x));
        m = fmaxf(m, fabsf(h));
        ml = fmaxf(ml, fabsf(x - h));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        ml = fmaxf(ml, __shfl_xor_sync(0xffffffffu, ml, o));
    }
    if ((threadIdx.x & 31) == 0) {
        atomicMax(&mx[0], __float_as_uint(m));
        atomicMax(&mx[1], __float_as_uint(ml));
    }
}

__device__ __forceinline__ uint8_t e4m3_byte(float v) { return (uint8_t)(e4m3x2(v, 0.0f) & 0xffu); }

// w16 = f16(w) * s_hi (exact: a power of two that keeps every value within FP16's normal range),
// w8[r, c] = e4m3((w - f16(w)) * s_lo8), w8[r, cols + c] = e4m3(f16(w) * s_hi8).
__global__ void corr_split_kernel(const float *w, int64_t rows, int64_t cols, float s_hi, float s_lo8, float s_hi8,
                                  __half *w16, uint8_t *w8) {
    const int64_t total = rows * cols;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = i / cols, c = i - r * cols;
        const float x = w[i];
        const float h = __half2float(__float2half_rn(x));
        w16[i] = __float2half_rn(h * s_hi);
        w8[r * 2 * cols + c] = e4m3_byte((x - h) * s_lo8);
        w8[r * 2 * cols + cols + c] = e4m3_byte(h * s_hi8);
    }
}

__global__ void split_x8_kernel(const float *x, int64_t rows, int64_t cols, int64_t ldx, __half *x16, int64_t ld16,
                                uint8_t *x8, int64_t ld8) {
    const int64_t total = rows * cols;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = i / cols, c = i - r * cols;
        const float v = x[r * ldx + c];
        const __half h = __float2half_rn(v);
        const float hf = __half2float(h);
        x16[r * ld16 + c] = h;
        x8[r * ld8 + c] = e4m3_byte(hf * kX8HiScale);
        x8[r * ld8 + cols + c] = e4m3_byte((v - hf) * kX8LoScale);
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

// dst[c, r] = src[r, c]; a 32 x 32 tile per block of 32 x 8 threads, staged in shared memory
// (one padding column, so the transposed reads hit 32 different banks).
__global__ void transpose_f32_kernel(const float *src, int64_t rows, int64_t cols, int64_t ld_src, float *dst,
                                     int64_t ld_dst) {
    __shared__ float tile[32][33];
    const int64_t r0 = (int64_t)blockIdx.y * 32, c0 = (int64_t)blockIdx.x * 32;
    for (int i = threadIdx.y; i < 32; i += 8) {
        const int64_t r = r0 + i, c = c0 + threadIdx.x;
        if (r < rows && c < cols) tile[i][threadIdx.x] = src[r * ld_src + c];
    }
    __syncthreads();
    for (int i = threadIdx.y; i < 32; i += 8) {
        const int64_t c = c0 + i, r = r0 + threadIdx.x;
        if (r < rows && c < cols) dst[c * ld_dst + r] = tile[threadIdx.x][i];
    }
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

Status build_corrected_weight(const float *w, int64_t rows, int64_t cols, void *w16, void *w8, int *s_out,
                              cudaStream_t s) {
    if (rows <= 0 || cols <= 0) return Status::fail(TSFM_ERR_INVALID_ARGUMENT, "corrected weight: empty");
    unsigned *mx = nullptr;
    TSFM_CUDA(cudaMallocAsync(reinterpret_cast<void **>(&mx), 2 * sizeof(unsigned), s), "corrected weight: range buffer");
    unsigned h[2] = {0, 0};
    cudaError_t e = cudaMemsetAsync(mx, 0, 2 * sizeof(unsigned), s);
    const int64_t total = rows * cols;
    const int grid = (int)std::min<int64_t>((total + 255) / 256, (int64_t)num_sms() * 32);
    if (e == cudaSuccess) {
        corr_range_kernel<<<grid, 256, 0, s>>>(w, total, mx);
        e = cudaGetLastError();
    }
    if (e == cudaSuccess) e = cudaMemcpyAsync(h, mx, sizeof(h), cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    cudaFreeAsync(mx, s);
    if (e != cudaSuccess) return Status::cuda(e, "corrected weight: range");
    float m, ml;
    std::memcpy(&m, &h[0], 4);
    std::memcpy(&ml, &h[1], 4);
    // sb: the largest power of two that keeps w_lo * 2^sb and f16(w) * 2^(sb - 12) within E4M3's
    // 448; then f16(w) * 2^(sb - 5) stays at or below 448 * 2^7 = 57344 < 65504.
    int sb = 0;
    if (m > 0.0f && std::isfinite(m)) {
        sb = std::ilogb(448.0 / (double)m) + 12;
        if (ml > 0.0f && std::isfinite(ml)) sb = std::min(sb, std::ilogb(448.0 / (double)ml));
    }
    const int sh = sb - 5;
    corr_split_kernel<<<grid, 256, 0, s>>>(w, rows, cols, std::ldexp(1.0f, sh), std::ldexp(1.0f, sb),
                                           std::ldexp(1.0f, sb - 12), static_cast<__half *>(w16),
                                           static_cast<uint8_t *>(w8));
    TSFM_CUDA(cudaGetLastError(), "corrected weight: split");
    *s_out = sh;
    return Status::ok();
}

Status launch_transpose_f32(const float *src, int64_t rows, int64_t cols, int64_t ld_src, float *dst, int64_t ld_dst,
                            cudaStream_t s) {
    if (rows <= 0 || cols <= 0) return Status::ok();
    const int64_t ty = (rows + 31) / 32, tx = (cols + 31) / 32;
    if (ty > 65535) return Status::fail(TSFM_ERR_INVALID_ARGUMENT, "transpose: too many rows");
    transpose_f32_kernel<<<dim3((unsigned)tx, (unsigned)ty), dim3(32, 8), 0, s>>>(src, rows, cols, ld_src, dst, ld_dst);
    TSFM_CUDA(cudaGetLastError(), "transpose: launch");
    return Status::ok();
}

Status launch_split_x8(const float *x, int64_t rows, int64_t cols, int64_t ldx, void *x16, int64_t ld16, void *x8,
                       int64_t ld8, cudaStream_t s) {
    if (rows <= 0 || cols <= 0) return Status::ok();
    const int64_t total = rows * cols;
    const int grid = (int)std::min<int64_t>((total + 255) / 256, (int64_t)num_sms() * 32);
    split_x8_kernel<<<grid, 256, 0, s>>>(x, rows, cols, ldx, static_cast<__half *>(x16), ld16,
                                         static_cast<uint8_t *>(x8), ld8);
    TSFM_CUDA(cudaGetLastError(), "split x8: launch");
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
