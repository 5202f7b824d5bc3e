// Device helpers for the FP8 companions of FP16 activations (corrected products, kernels.h).
#pragma once

#include <cuda_fp16.h>

#include "kernels.h"
#include "ptx.cuh"

namespace tsfm {

// The companion bytes of 32 consecutive values x_j = v_j * mul of one row of an FP16 activation:
// hi byte j = e4m3(f16(x_j) * kX8HiScale), lo byte j = e4m3((x_j - f16(x_j)) * kX8LoScale), four
// bytes per word (value 4q + i in byte i of word q). x_j is rounded exactly as the FP16 output of
// the same value is.
__device__ __forceinline__ void pack_x8_32(const float *v, uint32_t (&hi)[8], uint32_t (&lo)[8], float mul = 1.0f) {
#pragma unroll
    for (int q = 0; q < 8; ++q) {
        float h[4], l[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const float x = v[4 * q + j] * mul;
            const float xh = __half2float(__float2half_rn(x));
            h[j] = xh * kX8HiScale;
            l[j] = (x - xh) * kX8LoScale;
        }
        hi[q] = e4m3x2(h[0], h[1]) | (e4m3x2(h[2], h[3]) << 16);
        lo[q] = e4m3x2(l[0], l[1]) | (e4m3x2(l[2], l[3]) << 16);
    }
}

// pack_x8_32 for values whose FP16 roundings are already packed: x[j] (FP32) and h[e] = the FP16
// pair (x[2e], x[2e + 1]), low half first. The high parts scale the FP16 pair by 1/32 in FP16 and
// convert it directly: exact for results in FP16's normal range, and below it (|f16(x)| < 2^-9)
// both routes give E4M3 zero, so the bytes equal pack_x8_32's.
__device__ __forceinline__ void pack_x8_f16x2_32(const float *x, const uint32_t *h, uint32_t (&hi)[8],
                                                 uint32_t (&lo)[8]) {
    const __half2 k = __float2half2_rn(kX8HiScale);
#pragma unroll
    for (int q = 0; q < 8; ++q) {
        const uint32_t a = h[2 * q], b = h[2 * q + 1];
        const __half2 sa = __hmul2(*reinterpret_cast<const __half2 *>(&a), k);
        const __half2 sb = __hmul2(*reinterpret_cast<const __half2 *>(&b), k);
        hi[q] = e4m3x2_f16x2(*reinterpret_cast<const uint32_t *>(&sa)) |
                (e4m3x2_f16x2(*reinterpret_cast<const uint32_t *>(&sb)) << 16);
        const float2 fa = __half22float2(*reinterpret_cast<const __half2 *>(&a));
        const float2 fb = __half22float2(*reinterpret_cast<const __half2 *>(&b));
        lo[q] = e4m3x2((x[4 * q] - fa.x) * kX8LoScale, (x[4 * q + 1] - fa.y) * kX8LoScale) |
                (e4m3x2((x[4 * q + 2] - fb.x) * kX8LoScale, (x[4 * q + 3] - fb.y) * kX8LoScale) << 16);
    }
}

// The companion of 32 values of one row written to global memory: row8[col0 + j] = hi byte j,
// row8[half + col0 + j] = lo byte j, with 16-byte stores (row8 + col0 and row8 + half + col0
// 16-byte aligned).
__device__ __forceinline__ void store_x8_32(uint8_t *row8, int64_t half, int64_t col0, const float *v,
                                            float mul = 1.0f) {
    uint32_t hi[8], lo[8];
    pack_x8_32(v, hi, lo, mul);
    uint4 *ph = reinterpret_cast<uint4 *>(row8 + col0);
    uint4 *pl = reinterpret_cast<uint4 *>(row8 + half + col0);
    ph[0] = make_uint4(hi[0], hi[1], hi[2], hi[3]);
    ph[1] = make_uint4(hi[4], hi[5], hi[6], hi[7]);
    pl[0] = make_uint4(lo[0], lo[1], lo[2], lo[3]);
    pl[1] = make_uint4(lo[4], lo[5], lo[6], lo[7]);
}

// Staging box of a warp's companion of 64 columns for two TMA stores: 32 rows (one per lane) of
// 64 hi bytes at `box`, the lo bytes 2048 bytes further, both in the 64-byte swizzle of a tensor
// map with 64-byte boxes (16-byte chunk c of row r at chunk c ^ ((r / 2) % 4)). `part` selects
// columns [32 part, 32 part + 32) of the 64.
__device__ __forceinline__ void stage_x8_32(uint8_t *box, int lane, int part, const uint32_t (&hi)[8],
                                            const uint32_t (&lo)[8]) {
    const int sw = (lane >> 1) & 3;
    uint8_t *rh = box + lane * 64, *rl = box + 2048 + lane * 64;
    *reinterpret_cast<uint4 *>(rh + (((2 * part) ^ sw) << 4)) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
    *reinterpret_cast<uint4 *>(rh + (((2 * part + 1) ^ sw) << 4)) = make_uint4(hi[4], hi[5], hi[6], hi[7]);
    *reinterpret_cast<uint4 *>(rl + (((2 * part) ^ sw) << 4)) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
    *reinterpret_cast<uint4 *>(rl + (((2 * part + 1) ^ sw) << 4)) = make_uint4(lo[4], lo[5], lo[6], lo[7]);
}

}  // namespace tsfm
