// Device helpers for the FP8 companions of FP16 activations (corrected products, kernels.h).
#pragma once

#include <cuda_fp16.h>

#include "kernels.h"
#include "ptx.cuh"

namespace tsfm {

// The FP8 companion of 32 consecutive values x_j = v_j * mul of one row of an FP16 activation:
// row8[col0 + j] = e4m3(f16(x_j) * kX8HiScale), row8[half + col0 + j] = e4m3((x_j - f16(x_j)) *
// kX8LoScale), written with 16-byte stores (row8 + col0 and row8 + half + col0 16-byte aligned).
// x_j is rounded exactly as the FP16 output of the same value is.
__device__ __forceinline__ void store_x8_32(uint8_t *row8, int64_t half, int64_t col0, const float *v,
                                            float mul = 1.0f) {
    uint32_t hi[8], lo[8];
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
    uint4 *ph = reinterpret_cast<uint4 *>(row8 + col0);
    uint4 *pl = reinterpret_cast<uint4 *>(row8 + half + col0);
    ph[0] = make_uint4(hi[0], hi[1], hi[2], hi[3]);
    ph[1] = make_uint4(hi[4], hi[5], hi[6], hi[7]);
    pl[0] = make_uint4(lo[0], lo[1], lo[2], lo[3]);
    pl[1] = make_uint4(lo[4], lo[5], lo[6], lo[7]);
}

}  // namespace tsfm
