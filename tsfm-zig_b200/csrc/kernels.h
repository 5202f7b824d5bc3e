// Internal API between the host runtime (C++) and the CUDA kernels. No torch types anywhere.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

#include "../../include/tsfm_b200.h"

namespace tsfm {

// Element types of tensor-core operands and 16-bit activations. E_F16C is a weight-upload request
// only: an FP16 weight with its FP8 correction companion (DLin::w8), for corrected products.
// E_U8 names byte tensors (the FP8 companions) in tensor maps.
// E_F32X is exact FP32 (no TF32 rounding), a conversion target of the weight kernels.
enum ElemType { E_BF16 = 0, E_F16 = 1, E_F32 = 2, E_F16C = 3, E_U8 = 4, E_F32X = 5 };

// Corrected products (FP16 operands plus FP8 correction terms; TSFM_COMPUTE_F16C).
// A 16-bit activation x [M, K] of a corrected product has an FP8 companion x8 [M, 2K] (bytes):
//   x8[r, c]     = e4m3(x_hi[r, c] * kX8HiScale),      x_hi = f16(x)
//   x8[r, K + c] = e4m3((x - x_hi)[r, c] * kX8LoScale)
// and a weight W [N, K] is stored as W16 = f16(W) * 2^s with the companion
//   w8[n, c]     = e4m3(w_lo[n, c] * 2^sb),            w_lo = W - f16(W)
//   w8[n, K + c] = e4m3(f16(W)[n, c] * 2^(sb - 12)),   s = sb - 5,
// so x8 . w8 over 2K columns = 2^s (x_hi w_lo + x_lo f16(W)) and the accumulator holds
// 2^s (x_hi f16(W) + x_hi w_lo + x_lo f16(W)) ~= 2^s x W; the epilogue multiplies by 2^-s.
constexpr float kX8HiScale = 1.0f / 32.0f;
constexpr float kX8LoScale = 128.0f;
// Output modes of the kernels that write activations.
enum OutMode { OUT_BF16 = 0, OUT_F32 = 1, OUT_F32_ACC = 2, OUT_TF32 = 3, OUT_F16 = 4 };
inline int out_mode_for(int elem) { return elem == E_F16 ? OUT_F16 : elem == E_BF16 ? OUT_BF16 : OUT_TF32; }

struct Status {
    int code = 0;
    std::string msg;
    static Status ok() { return Status{}; }
    static Status fail(int c, std::string m) {
        Status s;
        s.code = c;
        s.msg = std::move(m);
        return s;
    }
    static Status cuda(cudaError_t e, const std::string &where) {
        return fail(e == cudaErrorMemoryAllocation ? TSFM_ERR_OUT_OF_MEMORY : TSFM_ERR_CUDA,
                    where + ": " + cudaGetErrorString(e));
    }
    explicit operator bool() const { return code == 0; }
};

#define TSFM_TRY(expr)                  \
    do {                                \
        ::tsfm::Status _s = (expr);     \
        if (!_s) return _s;             \
    } while (0)

#define TSFM_CUDA(expr, where)                                   \
    do {                                                         \
        cudaError_t _e = (expr);                                 \
        if (_e != cudaSuccess) return ::tsfm::Status::cuda(_e, where); \
    } while (0)

// y = epilogue(x[M, K] · w[N, K]^T). x and w share one element type: BF16 or FP16 (kind::f16) or
// FP32 read as TF32 (kind::tf32).
enum : int { ACT_GLU = 3 };

struct LinearCall {
    const void *x = nullptr;
    const void *w = nullptr;
    int dtype = E_BF16;
    int64_t M = 0, N = 0, K = 0, ldx = 0, ldw = 0;
    void *y = nullptr;
    int64_t ldy = 0;
    int out_mode = OUT_BF16;  // OutMode; OUT_F32_ACC: y += result
    const float *bias = nullptr;
    // 0 none, 1 relu, 2 silu, ACT_GLU: gated pairs. With ACT_GLU the weight's rows come in 256-row
    // blocks [g (128) | u (128)] and y has N / 2 columns: y[:, 128 t + c] = g[c] * silu(u[c]) for
    // block t (mulSilu, core/nn.zig:302-563; N a multiple of 256, 16-bit y, no bias or remap).
    int act = 0;
    // output row remap: y row = (r / rm_g) * rm_G + r % rm_g + rm_off when rm_g > 0
    int64_t rm_g = 0, rm_G = 0, rm_off = 0;
    // rotate-half RoPE on columns [0, rope_cols), 64-wide heads; tables [positions, 32]
    const float *rope_cos = nullptr, *rope_sin = nullptr;
    int rope_cols = 0;
    int64_t rope_p1 = 0, rope_p2 = 1;  // position index = (r / p1) * p2 + r % p2 (p1 == 0: r % p2)
    int *err = nullptr;                // device error word
    // Fused RMSNorm (rmsNorm, core/nn.zig:367-396) across a residual GEMM and the GEMM that reads
    // its normalised rows, without a pass of its own over the FP32 residual stream.
    // Reader side (norm_in set): the product's row r is multiplied by rs / norm_s_in[r] (1 when
    // norm_s_in is null) before bias, activation and RoPE, where
    // rs = 1 / sqrt(sum_p norm_in[p * M + r] / norm_dim + norm_eps); rs goes to norm_s_out[r].
    const float *norm_in = nullptr;
    int norm_parts = 0;
    int64_t norm_dim = 0;
    float norm_eps = 1e-6f;
    const float *norm_s_in = nullptr;
    float *norm_s_out = nullptr;
    // Residual side (norm_out set; out_mode OUT_F32_ACC, 16-bit operands, N % 256 == 0, no
    // activation, remap or RoPE): y += result as usual, and also
    //   norm_x16[r, c] = y[r, c] * s_r * norm_gamma[c] in the operand type, with s_r = rs of the
    //   reader side when norm_in is set, else norm_s_in[r];
    //   norm_out[(c / 256) * M + r] = sum over the 256 columns of column tile c / 256 of y[r, c]^2.
    // Any positive s_r keeps the 16-bit copy in range; the next GEMM's reader side undoes it.
    float *norm_out = nullptr;
    void *norm_x16 = nullptr;
    int64_t ld_x16 = 0;
    const float *norm_gamma = nullptr;
    // Corrected product (x8 set; dtype E_F16, K % 8 == 0): the FP8 companions of x and w (layouts
    // above, row strides in bytes) add the correction terms, and the result is multiplied by
    // acc_scale = 2^-s before the epilogue. Runs the FP8 stages first, then the FP16 ones.
    const void *x8 = nullptr;
    int64_t ldx8 = 0;
    const void *w8 = nullptr;
    int64_t ldw8 = 0;
    float acc_scale = 1.0f;
    // Correction columns: 2K (0 = default) adds both terms; K adds only the weight term
    // x_hi (W - f16(W)) (the first half of both companions), half the FP8 work.
    int64_t x8_cols = 0;
    // FP8 companion of a 16-bit output (y8 set; the output's column count a multiple of 64):
    // y8 row r = [e4m3(f16(y) * kX8HiScale) | e4m3((y - f16(y)) * kX8LoScale)], each part as
    // wide as y, row stride ldy8 bytes. With norm_out, norm_x8 is the companion of norm_x16.
    void *y8 = nullptr;
    int64_t ldy8 = 0;
    void *norm_x8 = nullptr;
    int64_t ld_nx8 = 0;
};
Status launch_linear(const LinearCall &c, cudaStream_t stream);

// Flash attention over groups of n tokens, head width 64, 16-bit q/k/v/o (dtype E_BF16 / E_F16).
struct AttentionCall {
    const void *q = nullptr, *k = nullptr, *v = nullptr;
    int dtype = E_BF16;
    int64_t ld_qkv = 0;
    void *o = nullptr;
    int64_t ld_o = 0;
    const uint8_t *key_valid = nullptr;  // (groups, kv_len) or null
    int64_t kv_stride = 0;               // stride of key_valid between groups (default n)
    const float *rel_bias = nullptr;     // per head, indexed by key - query offset, or null
    int64_t rel_stride = 0;              // floats per head (0: 2n - 1)
    int64_t rel_center = -1;             // index of offset 0 (-1: n - 1)
    int groups = 0, heads = 0, n = 0;
    float scale = 1.0f;
    // 0: T5 additive (keys_additive / full); 1: causal over valid keys, diagonal open;
    // 2: bidirectional over valid keys, diagonal open. For modes 1-2, queries i >= ne are
    // decoder queries reading keys [0, l) that are valid plus [ne, i].
    int mask_mode = 0;
    int ne = 0, l = 0;
    const uint8_t *group_bidir = nullptr;  // per group: 1 = bidirectional encoder rows (mode 1 only)
    int *err = nullptr;                    // device error word for the bounded waits of the tcgen05 path
    int force_path = 0;                    // 0: automatic, 1: tcgen05 path only (error if unsupported), 2: mma.sync path,
                                           // 3: the tcgen05 kernel with two softmax threads per row
    // FP8 companion of the FP16 output (kernels.h layout, width heads * 64; tcgen05 path only: a
    // call the tcgen05 path does not take fails rather than leave it unwritten).
    void *o8 = nullptr;
    int64_t ld_o8 = 0;
    // FP32 output instead of o (row stride ld_o32, 16-byte aligned rows on the tcgen05 path): for a
    // corrected product whose input is formed after the attention (an output gate).
    float *o32 = nullptr;
    int64_t ld_o32 = 0;
};
Status launch_attention(const AttentionCall &c, cudaStream_t stream);
// The tcgen05 path (attention_tc.cu): true when it handles this call's mask and shapes.
bool attention_tc_supported(const AttentionCall &c);
Status launch_attention_tc(const AttentionCall &c, cudaStream_t stream);

// 2-D TMA descriptor with the 128-byte swizzle over a row-major [outer, inner] matrix of 16-bit or
// 32-bit elements with row stride `ld` elements; box = [box_outer, box_inner]. `map` points to a
// CUtensorMap (128 bytes).
Status make_tmap_2d(void *map, const void *base, int dtype, int64_t inner, int64_t outer, int64_t ld,
                    uint32_t box_inner, uint32_t box_outer);
// Weight conversion on the device (weights.cu). dst row r = src row (map ? map[r] : r), converted
// from src_dt (E_F32 / E_F16 / E_BF16) to dst_dt (E_F16, E_BF16, or E_F32 = TF32-rounded).
Status launch_convert_rows(const void *src, int src_dt, const int32_t *map, void *dst, int dst_dt, int64_t rows,
                           int64_t cols, cudaStream_t s);
// dst = a (m x k) b (k x n) in float64, rounded to float, then to dst_dt (E_F16, E_BF16, or E_F32 /
// E_F32X: the float itself).
Status launch_fold_f64(const void *a, int a_dt, const void *b, int b_dt, void *dst, int dst_dt, int64_t m, int64_t k,
                       int64_t n, cudaStream_t s);

// Corrected-product weight (kernels.h layouts above) from an exact FP32 weight w [rows, cols] on
// the device: w16 = f16(w) * 2^s, w8 [rows, 2 cols] its FP8 companion; returns s (the epilogue
// multiplies by 2^-s). Reads back the weight's range (a stream synchronisation).
Status build_corrected_weight(const float *w, int64_t rows, int64_t cols, void *w16, void *w8, int *s_out,
                              cudaStream_t s);
// dst[c, r] = src[r, c] for a [rows, cols] FP32 matrix (row strides ld_src, ld_dst), 32 x 32 tiles
// through shared memory.
Status launch_transpose_f32(const float *src, int64_t rows, int64_t cols, int64_t ld_src, float *dst, int64_t ld_dst,
                            cudaStream_t s);
// An FP16 activation and its FP8 companion from FP32 values: x16 = f16(x), x8 row r =
// [e4m3(x16 * kX8HiScale) | e4m3((x - x16) * kX8LoScale)] (row strides in elements / bytes).
Status launch_split_x8(const float *x, int64_t rows, int64_t cols, int64_t ldx, void *x16, int64_t ld16, void *x8,
                       int64_t ld8, cudaStream_t s);

// cudaFuncSetAttribute(MaxDynamicSharedMemorySize) per (device, kernel) only when `bytes` exceeds
// what was set before: the attribute stays set in the context (a ceiling for every later launch),
// and setting it on every launch costs host time.
Status ensure_smem_attr(const void *func, int bytes);

// 3-D tensor map over `groups` blocks of `rows` rows (each `width` elements, row stride `ld`,
// blocks back to back), box (box_inner, box_rows, 1), 128-byte swizzle: a box that runs past the
// last row of its block is clipped there.
Status make_tmap_grouped_rows(void *map, const void *base, int dtype, int64_t width, int64_t rows, int64_t groups,
                              int64_t ld, uint32_t box_inner, uint32_t box_rows);

// RMSNorm: out[r] = x[in_row(r)] * (1 / sqrt(mean(x^2) + eps)) * scale.
// in_row(r) = (r / g) * G + r % g + off when g > 0. out_mode: OUT_BF16, OUT_F32, OUT_TF32, OUT_F16.
struct RmsNormCall {
    const float *x = nullptr;
    const float *scale = nullptr;
    void *out = nullptr;
    int out_mode = 0;
    int64_t rows = 0, dim = 0;
    float eps = 1e-6f;
    int64_t g = 0, G = 0, off = 0;
    const int64_t *rows_idx = nullptr;  // when set: in_row(r) = rows_idx[r]
    float *inv_out = nullptr;           // when set: the row's factor 1 / sqrt(mean(x^2) + eps)
    // FP8 companion of an FP16 output (kernels.h layout; dim % 4 == 0): row r at out8 + r * ld8
    // bytes, the low part `dim` bytes after the high part.
    void *out8 = nullptr;
    int64_t ld8 = 0;
};
Status launch_rmsnorm(const RmsNormCall &c, cudaStream_t stream);

// Chronos-2 / Chronos-Bolt instance normalisation and patch features (chronos2/forecaster.zig:94-154,
// chronos_bolt/forecaster.zig:150-197), one CTA per series.
struct PatchCall {
    const float *inputs = nullptr;  // row s at inputs + s * stride + start, length t
    int64_t stride = 0, start = 0, t = 0;
    int64_t b = 0;
    int ps = 16, pad = 0, n_ctx = 0;
    int feat_kind = 0;      // 0 Chronos-2 [time, value, mask], 1 Chronos-Bolt [value, mask]
    float tscale = 1.0f;
    int arcsinh = 1;
    int feat_mode = OUT_TF32;  // features: OUT_BF16, OUT_F32, OUT_TF32 or OUT_F16
    void *feats = nullptr;  // (b * n_ctx, feat_width)
    float *loc = nullptr, *scale = nullptr;  // (b)
    uint8_t *key_valid = nullptr;            // (b, seq): [0, n_ctx) written, then `extra_valid` ones
    int64_t seq = 0;
    int extra_valid = 0;
};
Status launch_patch(const PatchCall &c, cudaStream_t stream);

// Copies `n_rows` rows of `src` (d floats) into every series' sequence at rows
// s * seq + row0 .. + n_rows (the shared REG and future-patch embeddings).
Status launch_broadcast_rows(float *x, int64_t b, int64_t seq, int64_t row0, const float *src,
                             int64_t n_rows, int64_t d, cudaStream_t stream);

// Chronos-2 head post-processing (chronos2/forecaster.zig:186-203): out[(s*H + step)*Q + qi] =
// sinh(raw[(s*n_out + p)*Q*ps + qi*ps + i]) * scale[s] + loc[s] for step = p*ps + i < H.
struct HeadPostCall {
    const float *raw = nullptr;
    const float *loc = nullptr, *scale = nullptr;
    float *out = nullptr;
    int64_t b = 0, horizon = 0;
    int q = 0, ps = 0, n_out = 0;
    int arcsinh = 1;
    int layout = 0;  // 0 Chronos-2 (patch, q, ps) rows; 1 Chronos-Bolt (q, P) rows -> (b, q, P) store
};
Status launch_head_post(const HeadPostCall &c, cudaStream_t stream);

// A kernel whose only work is one bounded mbarrier wait on a barrier that nothing arrives on (the
// failure-detection test): it records its site in *err after `limit_ns` and returns.
Status launch_bounded_wait(int *err, unsigned long long limit_ns, cudaStream_t stream);

// FP32 -> OutMode conversion of a device buffer.
Status launch_convert(const float *src, void *dst, int64_t n, int mode, cudaStream_t stream);

int num_sms();

}  // namespace tsfm

namespace tsfm {
// 3xTF32 operand split for FP32-accurate products: hi = tf32(alpha * x), lo = tf32(alpha * x - hi)
// for a [rows, cols] matrix with row stride ld_src; outputs have row stride ld_dst, padding columns
// [cols, ld_dst) are zeroed.
Status launch_split_tf32(const float *src, int64_t rows, int64_t cols, int64_t ld_src, float alpha, float *hi,
                         float *lo, int64_t ld_dst, cudaStream_t stream);
}  // namespace tsfm

namespace tsfm {
// One-query cross-attention (chronos_bolt/model.zig:360-381): per (series, head) softmax over the
// series' `seq` keys of q · k_j with the T5 additive -floatMax mask (a series with no valid key
// averages uniformly), o = sum_j p_j v_j. q: [b, ld_q] (head h at h*64), k/v rows s*seq + j with
// row stride ld_kv, o: [b, ld_o]; all 16-bit of `dtype`; head width 64.
struct CrossAttnCall {
    const void *q = nullptr, *k = nullptr, *v = nullptr;
    int dtype = E_BF16;
    int64_t ld_q = 0, ld_kv = 0, ld_o = 0;
    void *o = nullptr;
    const uint8_t *key_valid = nullptr;  // (b, seq)
    int64_t b = 0;
    int heads = 0, seq = 0;
};
Status launch_cross_attention(const CrossAttnCall &c, cudaStream_t stream);

// storeBlock (chronos_bolt/forecaster.zig:97-105): out[(s*H + start + p)*q + qi] =
// pred[(s*q + qi)*P + p] for start + p < H.
Status launch_bolt_store(const float *pred, float *out, int64_t b, int q, int P, int64_t horizon, int64_t start,
                         cudaStream_t stream);

// Context rows of the next Bolt block (chronos_bolt/forecaster.zig:56-64): next[row, i] =
// (skip + i < len ? cur[row, skip + i] : pred[row, skip + i - len]) for rows of `rows` with
// new_len columns; cur is [rows, len], pred [rows, P].
Status launch_bolt_extend(const float *cur, int64_t len, const float *pred, int P, float *next, int64_t new_len,
                          int64_t skip, int64_t rows, cudaStream_t stream);

// Empirical quantiles of the q*q path samples per (series, step) (chronos_bolt/forecaster.zig:66-75):
// samples k = raw[(s*q*q + k)*P + p], sorted ascending, quantile_linear at each level ->
// pred[(s*q + qi)*P + p].
Status launch_bolt_quantiles(const float *raw, const float *levels, float *pred, int64_t b, int q, int P,
                             cudaStream_t stream);
}  // namespace tsfm

namespace tsfm {
// dst[(r*rep + k) * len + i] = src[r * stride + offset + i]: every series' context copied once per
// quantile path (chronos_bolt/forecaster.zig:47-48).
Status launch_bolt_replicate(const float *src, int64_t stride, int64_t offset, int64_t len, int rep, float *dst,
                             int64_t rows, cudaStream_t stream);
}  // namespace tsfm
