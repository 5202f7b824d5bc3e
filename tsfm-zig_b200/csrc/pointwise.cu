// Memory-bound kernels of the forecast path: RMSNorm, instance normalisation + patch features,
// sequence assembly of the shared embeddings, head post-processing and weight conversion.
// All are coalesced and vectorised where the layout allows; none has a reduction whose order
// depends on the launch shape.
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

__device__ __forceinline__ void put(void *out, int mode, int64_t idx, float v) {
    if (mode == OUT_BF16)
        reinterpret_cast<__nv_bfloat16 *>(out)[idx] = __float2bfloat16_rn(v);
    else if (mode == OUT_F16)
        reinterpret_cast<__half *>(out)[idx] = __float2half_rn(v);
    else
        reinterpret_cast<float *>(out)[idx] = mode == OUT_TF32 ? to_tf32(v) : v;
}

// nn.rmsNorm (core/nn.zig:374-396): one warp per row.
__global__ void rmsnorm_kernel(RmsNormCall c) {
    const int64_t r = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (r >= c.rows) return;
    const int64_t in_row = c.rows_idx ? c.rows_idx[r] : c.g > 0 ? (r / c.g) * c.G + r % c.g + c.off : r;
    const float *x = c.x + in_row * c.dim;
    const bool vec = (c.dim % 4) == 0;
    float ss = 0.0f;
    if (vec) {
        for (int64_t i = lane * 4; i < c.dim; i += 128) {
            const float4 v = *reinterpret_cast<const float4 *>(x + i);
            ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
        }
    } else {
        for (int64_t i = lane; i < c.dim; i += 32) ss += x[i] * x[i];
    }
    ss = warp_sum(ss);
    const float inv = 1.0f / sqrtf(ss / (float)c.dim + c.eps);
    if (c.inv_out && lane == 0) c.inv_out[r] = inv;
    const int64_t ob = r * c.dim;
    if (vec) {
        for (int64_t i = lane * 4; i < c.dim; i += 128) {
            const float4 v = *reinterpret_cast<const float4 *>(x + i);
            const float4 s = __ldg(reinterpret_cast<const float4 *>(c.scale + i));
            const float o0 = v.x * inv * s.x, o1 = v.y * inv * s.y, o2 = v.z * inv * s.z, o3 = v.w * inv * s.w;
            if (c.out_mode == OUT_BF16) {
                __nv_bfloat162 a = __floats2bfloat162_rn(o0, o1), b = __floats2bfloat162_rn(o2, o3);
                uint2 pk;
                pk.x = *reinterpret_cast<uint32_t *>(&a);
                pk.y = *reinterpret_cast<uint32_t *>(&b);
                *reinterpret_cast<uint2 *>(reinterpret_cast<__nv_bfloat16 *>(c.out) + ob + i) = pk;
            } else if (c.out_mode == OUT_F16) {
                __half2 a = __floats2half2_rn(o0, o1), b = __floats2half2_rn(o2, o3);
                uint2 pk;
                pk.x = *reinterpret_cast<uint32_t *>(&a);
                pk.y = *reinterpret_cast<uint32_t *>(&b);
                *reinterpret_cast<uint2 *>(reinterpret_cast<__half *>(c.out) + ob + i) = pk;
                if (c.out8) {
                    const float2 fa = __half22float2(a), fb = __half22float2(b);
                    uint8_t *row8 = static_cast<uint8_t *>(c.out8) + r * c.ld8;
                    *reinterpret_cast<uint32_t *>(row8 + i) =
                        e4m3x2(fa.x * kX8HiScale, fa.y * kX8HiScale) |
                        (e4m3x2(fb.x * kX8HiScale, fb.y * kX8HiScale) << 16);
                    *reinterpret_cast<uint32_t *>(row8 + c.dim + i) =
                        e4m3x2((o0 - fa.x) * kX8LoScale, (o1 - fa.y) * kX8LoScale) |
                        (e4m3x2((o2 - fb.x) * kX8LoScale, (o3 - fb.y) * kX8LoScale) << 16);
                }
            } else {
                float4 w = c.out_mode == OUT_TF32 ? make_float4(to_tf32(o0), to_tf32(o1), to_tf32(o2), to_tf32(o3))
                                           : make_float4(o0, o1, o2, o3);
                *reinterpret_cast<float4 *>(reinterpret_cast<float *>(c.out) + ob + i) = w;
            }
        }
    } else {
        for (int64_t i = lane; i < c.dim; i += 32) put(c.out, c.out_mode, ob + i, x[i] * inv * c.scale[i]);
    }
}

// rmsnorm_kernel for rows of NC * 256 values (NC <= 4: Chronos-2 / Bolt / Timestral widths): the
// warp reads its row once, each lane holding 8 consecutive values per 256-value chunk in registers
// (256-bit loads), and writes 16-byte (16-bit output), 8-byte (FP8 companion) or 32-byte (FP32)
// runs. Same per-element arithmetic as rmsnorm_kernel; the row's sum of squares is accumulated in
// another order, so the factor can differ from that kernel's in the last bit.
template <int NC>
__global__ void __launch_bounds__(256) rmsnorm_v8_kernel(RmsNormCall c) {
    const int64_t r = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (r >= c.rows) return;
    const int64_t in_row = c.rows_idx ? c.rows_idx[r] : c.g > 0 ? (r / c.g) * c.G + r % c.g + c.off : r;
    const float *x = c.x + in_row * c.dim;
    float v[NC][8];
#pragma unroll
    for (int k = 0; k < NC; ++k) ld_global_v8(x + 256 * k + 8 * lane, v[k]);
    float ss = 0.0f;
#pragma unroll
    for (int k = 0; k < NC; ++k)
#pragma unroll
        for (int j = 0; j < 8; ++j) ss = fmaf(v[k][j], v[k][j], ss);
    ss = warp_sum(ss);
    const float inv = 1.0f / sqrtf(ss / (float)c.dim + c.eps);
    if (c.inv_out && lane == 0) c.inv_out[r] = inv;
    const int64_t ob = r * c.dim;
#pragma unroll
    for (int k = 0; k < NC; ++k) {
        const int64_t i = 256 * k + 8 * lane;
        float s[8], o[8];
        ld_global_v8(c.scale + i, s);
#pragma unroll
        for (int j = 0; j < 8; ++j) o[j] = v[k][j] * inv * s[j];
        if (c.out_mode == OUT_BF16 || c.out_mode == OUT_F16) {
            uint32_t pk[4];
            float2 f[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                if (c.out_mode == OUT_BF16) {
                    __nv_bfloat162 a = __floats2bfloat162_rn(o[2 * e], o[2 * e + 1]);
                    pk[e] = *reinterpret_cast<uint32_t *>(&a);
                } else {
                    __half2 a = __floats2half2_rn(o[2 * e], o[2 * e + 1]);
                    pk[e] = *reinterpret_cast<uint32_t *>(&a);
                    f[e] = __half22float2(a);
                }
            }
            *reinterpret_cast<uint4 *>(static_cast<uint16_t *>(c.out) + ob + i) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
            if (c.out_mode == OUT_F16 && c.out8) {
                uint8_t *row8 = static_cast<uint8_t *>(c.out8) + r * c.ld8;
                uint32_t hi[2], lo[2];
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const float2 fa = f[2 * h], fb = f[2 * h + 1];
                    const float *oo = o + 4 * h;
                    hi[h] = e4m3x2(fa.x * kX8HiScale, fa.y * kX8HiScale) |
                            (e4m3x2(fb.x * kX8HiScale, fb.y * kX8HiScale) << 16);
                    lo[h] = e4m3x2((oo[0] - fa.x) * kX8LoScale, (oo[1] - fa.y) * kX8LoScale) |
                            (e4m3x2((oo[2] - fb.x) * kX8LoScale, (oo[3] - fb.y) * kX8LoScale) << 16);
                }
                *reinterpret_cast<uint2 *>(row8 + i) = make_uint2(hi[0], hi[1]);
                *reinterpret_cast<uint2 *>(row8 + c.dim + i) = make_uint2(lo[0], lo[1]);
            }
        } else {
            if (c.out_mode == OUT_TF32) {
#pragma unroll
                for (int j = 0; j < 8; ++j) o[j] = to_tf32(o[j]);
            }
            st_global_v8(static_cast<float *>(c.out) + ob + i, __float_as_uint(o[0]), __float_as_uint(o[1]),
                         __float_as_uint(o[2]), __float_as_uint(o[3]), __float_as_uint(o[4]), __float_as_uint(o[5]),
                         __float_as_uint(o[6]), __float_as_uint(o[7]));
        }
    }
}

__device__ __forceinline__ double block_sum_d(double v, double *red) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    __syncthreads();
    if (lane == 0) red[w] = v;
    __syncthreads();
    double t = 0.0;
    if (threadIdx.x < 32) {
        t = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.0;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
        if (threadIdx.x == 0) red[32] = t;
    }
    __syncthreads();
    return red[32];
}

// Instance norm over observed values (f64 sums, population std, 0 -> 1e-5, all missing -> loc 0,
// scale 1), then per-step patch features; one CTA per series.
// Chronos-2: chronos2/forecaster.zig:94-143; Chronos-Bolt: chronos_bolt/forecaster.zig:150-197.
__global__ void patch_kernel(PatchCall c) {
    __shared__ double red[33];
    const int64_t s = blockIdx.x;
    const float *row = c.inputs + s * c.stride + c.start;
    double cnt = 0.0, sum = 0.0;
    for (int64_t i = threadIdx.x; i < c.t; i += blockDim.x) {
        const float v = row[i];
        if (!isnan(v)) {
            cnt += 1.0;
            sum += (double)v;
        }
    }
    cnt = block_sum_d(cnt, red);
    sum = block_sum_d(sum, red);
    float lo = 0.0f, sc = 1.0f;
    if (cnt > 0.0) {
        lo = (float)(sum / cnt);
        double ss = 0.0;
        for (int64_t i = threadIdx.x; i < c.t; i += blockDim.x) {
            const float v = row[i];
            if (!isnan(v)) {
                const float dv = v - lo;
                ss += (double)dv * (double)dv;
            }
        }
        ss = block_sum_d(ss, red);
        sc = (float)sqrt(ss / cnt);
        if (sc == 0.0f) sc = 1e-5f;
    }
    if (threadIdx.x == 0) {
        c.loc[s] = lo;
        c.scale[s] = sc;
    }
    const int ps = c.ps;
    const int width = c.feat_kind == 0 ? 3 * ps : 2 * ps;
    const int64_t nsteps = (int64_t)c.n_ctx * ps;
    const float tbase = (float)((int64_t)c.n_ctx * ps);
    for (int64_t idx = threadIdx.x; idx < nsteps; idx += blockDim.x) {
        const int64_t p = idx / ps;
        const int i = (int)(idx % ps);
        const int64_t src = idx - c.pad;
        bool obs = false;
        float val = 0.0f;
        if (src >= 0 && src < c.t) {
            const float xv = row[src];
            if (!isnan(xv)) {
                obs = true;
                val = (xv - lo) / sc;
                if (c.arcsinh) val = asinhf(val);
            }
        }
        const int64_t fb = (s * c.n_ctx + p) * width;
        if (c.feat_kind == 0) {
            put(c.feats, c.feat_mode, fb + i, ((float)idx - tbase) / c.tscale);
            put(c.feats, c.feat_mode, fb + ps + i, val);
            put(c.feats, c.feat_mode, fb + 2 * ps + i, obs ? 1.0f : 0.0f);
        } else {
            put(c.feats, c.feat_mode, fb + i, val);
            put(c.feats, c.feat_mode, fb + ps + i, obs ? 1.0f : 0.0f);
        }
    }
    for (int64_t p = threadIdx.x; p < c.n_ctx; p += blockDim.x) {
        bool any = false;
        for (int i = 0; i < ps; ++i) {
            const int64_t src = p * ps + i - c.pad;
            if (src >= 0 && src < c.t && !isnan(row[src])) any = true;
        }
        c.key_valid[s * c.seq + p] = any;
    }
    for (int e = threadIdx.x; e < c.extra_valid; e += blockDim.x) c.key_valid[s * c.seq + c.n_ctx + e] = 1;
}

__global__ void broadcast_rows_kernel(float *x, int64_t b, int64_t seq, int64_t row0, const float *src,
                                      int64_t n_rows, int64_t d4) {
    const int64_t total = b * n_rows * d4;
    for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total; idx += (int64_t)gridDim.x * blockDim.x) {
        const int64_t c4 = idx % d4, r = (idx / d4) % n_rows, s = idx / (d4 * n_rows);
        reinterpret_cast<float4 *>(x + (s * seq + row0 + r) * d4 * 4)[c4] = __ldg(reinterpret_cast<const float4 *>(src + r * d4 * 4) + c4);
    }
}

// chronos2/forecaster.zig:186-203 (layout 0) and chronos_bolt/forecaster.zig:209-219 (layout 1).
__global__ void head_post_kernel(HeadPostCall c) {
    const int64_t total = c.layout == 0 ? c.b * c.horizon * c.q : c.b * (int64_t)c.q * c.ps;
    for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total; idx += (int64_t)gridDim.x * blockDim.x) {
        if (c.layout == 0) {
            const int qi = (int)(idx % c.q);
            const int64_t step = (idx / c.q) % c.horizon, s = idx / (c.q * c.horizon);
            const int64_t p = step / c.ps;
            const int i = (int)(step % c.ps);
            float v = c.raw[(s * c.n_out + p) * (int64_t)c.q * c.ps + (int64_t)qi * c.ps + i];
            if (c.arcsinh) v = sinhf(v);
            c.out[idx] = v * c.scale[s] + c.loc[s];
        } else {
            const int64_t s = idx / ((int64_t)c.q * c.ps);
            c.out[idx] = c.raw[idx] * c.scale[s] + c.loc[s];
        }
    }
}

__global__ void convert_kernel(const float *src, void *dst, int64_t n, int mode) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        put(dst, mode, i, src[i]);
}

__global__ void split_tf32_kernel(const float *src, int64_t rows, int64_t cols, int64_t ld_src, float alpha, float *hi,
                                  float *lo, int64_t ld_dst) {
    const int64_t total = rows * ld_dst;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = i / ld_dst, c = i % ld_dst;
        float h = 0.0f, l = 0.0f;
        if (c < cols) {
            const float v = alpha * src[r * ld_src + c];
            h = to_tf32(v);
            l = to_tf32(v - h);
        }
        hi[i] = h;
        lo[i] = l;
    }
}

int grid_for(int64_t total, int block) {
    const int64_t g = (total + block - 1) / block;
    const int64_t cap = (int64_t)num_sms() * 16;
    return (int)std::max<int64_t>(1, std::min<int64_t>(g, cap));
}

}  // namespace

// The bounded mbarrier wait of the warp-specialised kernels, on a barrier that nothing arrives on:
// the wait gives up after `limit_ns`, records its site in *err and the kernel returns.
__global__ void bounded_wait_kernel(int *err, unsigned long long limit_ns) {
    __shared__ uint64_t bar;
    __shared__ int abort_flag;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        abort_flag = 0;
        fence_barrier_init();
    }
    __syncthreads();
    if (threadIdx.x == 0) (void)mbar_wait(&bar, 0, &abort_flag, err, ERR_SITE_WAIT_TEST, limit_ns);
}

Status launch_bounded_wait(int *err, unsigned long long limit_ns, cudaStream_t stream) {
    bounded_wait_kernel<<<1, 32, 0, stream>>>(err, limit_ns);
    TSFM_CUDA(cudaGetLastError(), "bounded wait: launch");
    return Status::ok();
}

Status launch_rmsnorm(const RmsNormCall &c, cudaStream_t stream) {
    if (c.rows <= 0 || c.dim <= 0) return Status::fail(TSFM_ERR_INVALID_ARGUMENT, "rmsnorm: empty");
    if ((c.dim % 4) == 0 && ((reinterpret_cast<uintptr_t>(c.x) | reinterpret_cast<uintptr_t>(c.scale) |
                              reinterpret_cast<uintptr_t>(c.out)) & 15))
        return Status::fail(TSFM_ERR_INVALID_ARGUMENT, "rmsnorm: buffers must be 16-byte aligned");
    if (c.out8 && (c.out_mode != OUT_F16 || c.dim % 4 || c.ld8 % 4 || c.ld8 < 2 * c.dim ||
                   (reinterpret_cast<uintptr_t>(c.out8) & 3)))
        return Status::fail(TSFM_ERR_INVALID_ARGUMENT, "rmsnorm: an FP8 companion needs an FP16 output, dim % 4 == 0");
    const int64_t blocks = (c.rows + 7) / 8;
    const auto al = [](const void *p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0; };
    const bool f32_out = c.out_mode != OUT_BF16 && c.out_mode != OUT_F16;
    const bool v8 = c.dim % 256 == 0 && c.dim <= 1024 && al(c.x, 32) && al(c.scale, 32) &&
                    al(c.out, f32_out ? 32 : 16) && (!c.out8 || (al(c.out8, 8) && c.ld8 % 8 == 0));
    if (v8) {
        switch (c.dim / 256) {
        case 1: rmsnorm_v8_kernel<1><<<(unsigned)blocks, 256, 0, stream>>>(c); break;
        case 2: rmsnorm_v8_kernel<2><<<(unsigned)blocks, 256, 0, stream>>>(c); break;
        case 3: rmsnorm_v8_kernel<3><<<(unsigned)blocks, 256, 0, stream>>>(c); break;
        default: rmsnorm_v8_kernel<4><<<(unsigned)blocks, 256, 0, stream>>>(c); break;
        }
        TSFM_CUDA(cudaGetLastError(), "rmsnorm: launch");
        return Status::ok();
    }
    rmsnorm_kernel<<<(unsigned)blocks, 256, 0, stream>>>(c);
    TSFM_CUDA(cudaGetLastError(), "rmsnorm: launch");
    return Status::ok();
}

Status launch_patch(const PatchCall &c, cudaStream_t stream) {
    if (c.b <= 0 || c.t <= 0 || c.n_ctx <= 0) return Status::fail(TSFM_ERR_INVALID_ARGUMENT, "patch: empty");
    patch_kernel<<<(unsigned)c.b, 256, 0, stream>>>(c);
    TSFM_CUDA(cudaGetLastError(), "patch: launch");
    return Status::ok();
}

Status launch_broadcast_rows(float *x, int64_t b, int64_t seq, int64_t row0, const float *src, int64_t n_rows,
                             int64_t d, cudaStream_t stream) {
    if (b <= 0 || n_rows <= 0) return Status::ok();
    if (d % 4) return Status::fail(TSFM_ERR_INVALID_ARGUMENT, "broadcast: d % 4 != 0");
    const int64_t total = b * n_rows * (d / 4);
    broadcast_rows_kernel<<<grid_for(total, 256), 256, 0, stream>>>(x, b, seq, row0, src, n_rows, d / 4);
    TSFM_CUDA(cudaGetLastError(), "broadcast: launch");
    return Status::ok();
}

Status launch_head_post(const HeadPostCall &c, cudaStream_t stream) {
    const int64_t total = c.layout == 0 ? c.b * c.horizon * c.q : c.b * (int64_t)c.q * c.ps;
    if (total <= 0) return Status::ok();
    head_post_kernel<<<grid_for(total, 256), 256, 0, stream>>>(c);
    TSFM_CUDA(cudaGetLastError(), "head: launch");
    return Status::ok();
}

Status launch_split_tf32(const float *src, int64_t rows, int64_t cols, int64_t ld_src, float alpha, float *hi,
                         float *lo, int64_t ld_dst, cudaStream_t stream) {
    if (rows <= 0 || ld_dst <= 0) return Status::ok();
    split_tf32_kernel<<<grid_for(rows * ld_dst, 256), 256, 0, stream>>>(src, rows, cols, ld_src, alpha, hi, lo, ld_dst);
    TSFM_CUDA(cudaGetLastError(), "split: launch");
    return Status::ok();
}

Status launch_convert(const float *src, void *dst, int64_t n, int mode, cudaStream_t stream) {
    if (n <= 0) return Status::ok();
    convert_kernel<<<grid_for(n, 256), 256, 0, stream>>>(src, dst, n, mode);
    TSFM_CUDA(cudaGetLastError(), "convert: launch");
    return Status::ok();
}

}  // namespace tsfm
