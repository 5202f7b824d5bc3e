// Memory-bound kernels specific to Chronos-Bolt: the one-token decoder's cross-attention and the
// long-horizon quantile-path loop (context extension, q^2-sample quantiles, block store).
#include "kernels.h"
#include "ptx.cuh"

#include <cuda_fp16.h>

namespace tsfm {

namespace {

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// One CTA per series, one warp per head (blockDim = 32 * heads_per_block), scores in shared
// memory. Each lane owns head dims (2 lane, 2 lane + 1).
template <bool F16>
__device__ __forceinline__ float2 ld2(const void *base, int64_t idx) {
    if constexpr (F16) {
        const __half2 v = *reinterpret_cast<const __half2 *>(static_cast<const __half *>(base) + idx);
        return __half22float2(v);
    } else {
        const __nv_bfloat162 v = *reinterpret_cast<const __nv_bfloat162 *>(static_cast<const __nv_bfloat16 *>(base) + idx);
        return make_float2(__low2float(v), __high2float(v));
    }
}

template <bool F16>
__global__ void cross_attn_kernel(CrossAttnCall c) {
    extern __shared__ float sc[];  // [warps][seq]
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int h = blockIdx.y * (blockDim.x >> 5) + warp;
    const int64_t s = blockIdx.x;
    if (h >= c.heads) return;
    float *row = sc + warp * c.seq;
    const float2 qv = ld2<F16>(c.q, s * c.ld_q + h * 64 + 2 * lane);
    const float q0 = qv.x, q1 = qv.y;
    const uint8_t *kv = c.key_valid + s * c.seq;
    bool any = false;
    for (int j = 0; j < c.seq; ++j) any = any || kv[j];
    float mx = -INFINITY;
    for (int j = 0; j < c.seq; ++j) {
        const float2 kk = ld2<F16>(c.k, (s * c.seq + j) * c.ld_kv + h * 64 + 2 * lane);
        float d = warp_sum(q0 * kk.x + q1 * kk.y);
        // -floatMax addition: invalid keys drop out unless no key is valid, where every score
        // rounds to the same value (uniform average).
        if (!any) d = 0.0f;
        else if (!kv[j]) d = -INFINITY;
        if (lane == 0) row[j] = d;
        mx = fmaxf(mx, d);
    }
    __syncwarp();
    float sum = 0.0f;
    for (int j = lane; j < c.seq; j += 32) {
        const float e = row[j] == -INFINITY ? 0.0f : expf(row[j] - mx);
        row[j] = e;
        sum += e;
    }
    sum = warp_sum(sum);
    __syncwarp();
    const float inv = 1.0f / sum;
    float o0 = 0.0f, o1 = 0.0f;
    for (int j = 0; j < c.seq; ++j) {
        const float p = row[j];
        if (p == 0.0f) continue;
        const float2 vv = ld2<F16>(c.v, (s * c.seq + j) * c.ld_kv + h * 64 + 2 * lane);
        o0 += p * vv.x;
        o1 += p * vv.y;
    }
    const int64_t oi = s * c.ld_o + h * 64 + 2 * lane;
    if constexpr (F16)
        *reinterpret_cast<__half2 *>(static_cast<__half *>(c.o) + oi) = __floats2half2_rn(o0 * inv, o1 * inv);
    else
        *reinterpret_cast<__nv_bfloat162 *>(static_cast<__nv_bfloat16 *>(c.o) + oi) = __floats2bfloat162_rn(o0 * inv, o1 * inv);
}

__global__ void bolt_store_kernel(const float *pred, float *out, int64_t b, int q, int P, int64_t horizon, int64_t start) {
    const int64_t n = b * (int64_t)P * q;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const int qi = (int)(i % q);
        const int p = (int)((i / q) % P);
        const int64_t s = i / ((int64_t)q * P);
        const int64_t step = start + p;
        if (step < horizon) out[(s * horizon + step) * q + qi] = pred[(s * q + qi) * P + p];
    }
}

__global__ void bolt_extend_kernel(const float *cur, int64_t len, const float *pred, int P, float *next, int64_t new_len,
                                   int64_t skip, int64_t rows) {
    const int64_t n = rows * new_len;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t row = i / new_len, col = i % new_len, j = skip + col;
        next[i] = j < len ? cur[row * len + j] : pred[row * P + (j - len)];
    }
}

// One thread per (series, step); q*q <= 1024 samples sorted by insertion into a local buffer.
__global__ void bolt_quantiles_kernel(const float *raw, const float *levels, float *pred, int64_t b, int q, int P) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= b * P) return;
    const int64_t s = i / P;
    const int p = (int)(i % P);
    const int n = q * q;
    float buf[256];
    for (int k = 0; k < n; ++k) {
        const float x = raw[(s * n + k) * (int64_t)P + p];
        int j = k - 1;
        while (j >= 0 && buf[j] > x) {
            buf[j + 1] = buf[j];
            --j;
        }
        buf[j + 1] = x;
    }
    for (int qi = 0; qi < q; ++qi) {
        // quantileLinear (chronos_bolt/forecaster.zig:83-93)
        const float rank = levels[qi] * (float)(n - 1);
        const float lo_f = floorf(rank);
        const int lo = (int)lo_f;
        const int hi = min((int)ceilf(rank), n - 1);
        const float w = rank - lo_f;
        const float a = buf[lo], bb = buf[hi];
        pred[(s * q + qi) * (int64_t)P + p] = w < 0.5f ? a + w * (bb - a) : bb - (bb - a) * (1.0f - w);
    }
}

__global__ void bolt_replicate_kernel(const float *src, int64_t stride, int64_t offset, int64_t len, int rep, float *dst,
                                      int64_t rows) {
    const int64_t n = rows * rep * len;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t col = i % len, r = i / (len * rep);
        dst[i] = src[r * stride + offset + col];
    }
}

int grid_for(int64_t total, int block) {
    const int64_t g = (total + block - 1) / block;
    const int64_t cap = (int64_t)num_sms() * 16;
    return (int)std::max<int64_t>(1, std::min<int64_t>(g, cap));
}

}  // namespace

Status launch_cross_attention(const CrossAttnCall &c, cudaStream_t stream) {
    if (c.b <= 0 || c.heads <= 0 || c.seq <= 0) return Status::fail(TSFM_ERR_INVALID_ARGUMENT, "cross attention: empty");
    const int per = std::min(c.heads, 8);
    const size_t smem = (size_t)per * c.seq * sizeof(float);
    if (smem > 48 * 1024) return Status::fail(TSFM_ERR_UNSUPPORTED, "cross attention: sequence too long");
    dim3 grid((unsigned)c.b, (unsigned)((c.heads + per - 1) / per));
    if (c.dtype == E_F16)
        cross_attn_kernel<true><<<grid, 32 * per, smem, stream>>>(c);
    else
        cross_attn_kernel<false><<<grid, 32 * per, smem, stream>>>(c);
    TSFM_CUDA(cudaGetLastError(), "cross attention: launch");
    return Status::ok();
}

Status launch_bolt_store(const float *pred, float *out, int64_t b, int q, int P, int64_t horizon, int64_t start,
                         cudaStream_t stream) {
    const int64_t n = b * (int64_t)P * q;
    if (n <= 0) return Status::ok();
    bolt_store_kernel<<<grid_for(n, 256), 256, 0, stream>>>(pred, out, b, q, P, horizon, start);
    TSFM_CUDA(cudaGetLastError(), "bolt store: launch");
    return Status::ok();
}

Status launch_bolt_extend(const float *cur, int64_t len, const float *pred, int P, float *next, int64_t new_len,
                          int64_t skip, int64_t rows, cudaStream_t stream) {
    const int64_t n = rows * new_len;
    if (n <= 0) return Status::ok();
    bolt_extend_kernel<<<grid_for(n, 256), 256, 0, stream>>>(cur, len, pred, P, next, new_len, skip, rows);
    TSFM_CUDA(cudaGetLastError(), "bolt extend: launch");
    return Status::ok();
}

Status launch_bolt_replicate(const float *src, int64_t stride, int64_t offset, int64_t len, int rep, float *dst,
                             int64_t rows, cudaStream_t stream) {
    const int64_t n = rows * rep * len;
    if (n <= 0) return Status::ok();
    bolt_replicate_kernel<<<grid_for(n, 256), 256, 0, stream>>>(src, stride, offset, len, rep, dst, rows);
    TSFM_CUDA(cudaGetLastError(), "bolt replicate: launch");
    return Status::ok();
}

Status launch_bolt_quantiles(const float *raw, const float *levels, float *pred, int64_t b, int q, int P,
                             cudaStream_t stream) {
    if (q * q > 256) return Status::fail(TSFM_ERR_UNSUPPORTED, "Chronos-Bolt: more than 16 quantiles in the long-horizon loop");
    const int64_t n = b * P;
    if (n <= 0) return Status::ok();
    bolt_quantiles_kernel<<<(unsigned)((n + 127) / 128), 128, 0, stream>>>(raw, levels, pred, b, q, P);
    TSFM_CUDA(cudaGetLastError(), "bolt quantiles: launch");
    return Status::ok();
}

}  // namespace tsfm
