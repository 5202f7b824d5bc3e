// Launch wrappers shared by the family forwards: every kernel launch goes through one of these,
// which records it (class, algorithmic work) on the replica's profiler.
#pragma once

#include "model.h"

namespace tsfm {

Status load_resblock(Replica &r, const TensorTable &t, const std::string &prefix, int64_t in, int64_t hid,
                     int64_t out, bool bias, int in_dtype, int hidden_dtype, DResBlock &dst);
Status check_resblock(const TensorTable &t, const std::string &prefix, int64_t in, int64_t hid, int64_t out, bool bias);

// y (out_mode: 0 bf16, 1 f32, 2 f32 +=) = act(x[M, L.in] L.w^T + L.b); `extra` carries row remap / RoPE,
// and for a corrected weight (L.w8 set) the input's FP8 companion (x8, ldx8) and optionally the
// output's (y8, ldy8).
Status op_linear(Replica &r, cudaStream_t s, const DLin &L, const void *x, int64_t M, int64_t ldx, void *y,
                 int64_t ldy, int out_mode, int act, const LinearCall *extra = nullptr);
// y (+)= act(x W^T + b) to FP32 accuracy: three TF32 products of split operands (x = x_hi + x_lo
// from launch_split_tf32, W from upload_lin3), smallest terms first; act applies to the final sum.
Status op_linear3(Replica &r, cudaStream_t s, const DLin3 &L, const float *x_hi, const float *x_lo, int64_t M,
                  int64_t ldx, float *y, int64_t ldy, bool accumulate, int act);
// Splits x [rows, cols] (row stride ld) in place into x_hi (written over x) and x_lo.
Status op_split(Replica &r, cudaStream_t s, float *x, float *x_lo, int64_t rows, int64_t cols, int64_t ld);
// out8: the FP8 companion of an FP16 output (row stride 2 * dim bytes), or null.
Status op_rmsnorm(Replica &r, cudaStream_t s, const float *x, const float *scale, void *out, int out_mode,
                  int64_t rows, int64_t dim, float eps, int64_t g = 0, int64_t G = 0, int64_t off = 0,
                  float *inv_out = nullptr, void *out8 = nullptr);

}  // namespace tsfm
