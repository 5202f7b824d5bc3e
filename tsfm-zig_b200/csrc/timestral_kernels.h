// Launch interface of the Timestral-specific kernels (timestral_kernels.cu).
#pragma once

#include "kernels.h"

namespace tsfm {

// Window (context, then known futures or blanks when cov), per-row causal statistics, known-row
// whole statistics, key validity, first observed patch per group, and patch features.
struct TsStatsCall {
    const float *ctx = nullptr;
    const uint8_t *obs = nullptr;
    int64_t t = 0;                 // context steps (multiple of ps)
    const float *kf = nullptr;     // known futures of this block (rows, hl) at row stride kf_ld, or null (blanks)
    const uint8_t *kfm = nullptr;
    int64_t kf_ld = 0;
    int64_t hl = 0;                // horizon steps of this block (h * ps)
    int cov = 0;                   // covariate window: t + hl steps
    int64_t rows = 0;
    int ps = 0, vall = 0;
    const int8_t *roles = nullptr;  // per row of a group: 0 target, 1 past, 2 known
    double min_scale = 1e-6;
    int use_asinh = 1, attend_missing = 1;
    float *loc = nullptr, *scale = nullptr;     // (rows, n)
    float *kloc = nullptr, *kscale = nullptr;   // (rows)
    uint8_t *binary = nullptr;                  // (rows)
    uint8_t *key_valid = nullptr;               // (rows, n)
    int *first_obs = nullptr;                   // (groups), initialised to INT_MAX
    int raw_feats = 0;                          // features as computed (else TF32-rounded operands)
};
Status launch_ts_stats(const TsStatsCall &c, float *feats, cudaStream_t s);

Status launch_ts_rope(const int *first_obs, int64_t groups, int64_t sl, int64_t ne, int64_t l, const float *inv_freq,
                      int half, float *cs, float *sn, cudaStream_t s);
// forecastRaw's input rows (forecaster.zig:319-388) built on the device from the raw arrays:
// per (pass, series, row) the last `keep` steps left-padded to t, targets forward-filled from their
// last observed step (0 before the first), covariates with NaN as unobserved (0), the known
// futures; the second pass (symmetric averaging) negates every value. Optionally the non-negative
// clip flag per (series, target) (forecaster.zig:163-180).
struct TsPrepareCall {
    const float *inputs = nullptr;     // (b, v, t0)
    const uint8_t *observed = nullptr; // (b, v, t0)
    const float *past = nullptr;       // (b, n_past, t0) or null
    const float *known = nullptr;      // (b, n_known, t0 + horizon) or null
    int64_t b = 0, v = 0, n_past = 0, n_known = 0, t0 = 0, horizon = 0, keep = 0, t = 0, hpad = 0;
    int passes = 1;
    float *rows = nullptr, *rows2 = nullptr;    // (passes * b * vall, t); rows2: optional copy
    uint8_t *mask = nullptr, *mask2 = nullptr;  // same shape
    float *kf = nullptr;                        // (passes * b * vall, hpad)
    uint8_t *kfm = nullptr;
    uint8_t *clip = nullptr;                    // (b * v) or null
};
Status launch_ts_prepare(const TsPrepareCall &c, cudaStream_t s);

// Categorical covariates (forecaster.zig:92-103, 201-301). With a univariate target, each code row
// is target-encoded: target = the series' forward-filled observed value inside the --max-context
// window (NaN elsewhere); a context step maps to (mean + sum) / (1 + count) over the earlier and
// later context steps with the same code and a finite target (sums in step order, f64); codes that
// are not finite share one slot; a future step with a code never seen in the context gets the
// mean. Without a target the codes are only rounded to f32. `out` rows are (b, chan_total, len)
// and the encoded channels start at chan0.
Status launch_ts_target(const float *inputs, const uint8_t *observed, int64_t b, int64_t t0, int64_t max_context,
                        double *target, cudaStream_t s);
Status launch_ts_cat_encode(const double *codes, int64_t b, int64_t ncat, int64_t len, int64_t t0, const double *target,
                            float *out, int64_t chan_total, int64_t chan0, cudaStream_t s);

// Row flags and head / target row indices of one block; target rows are the first v of every
// group of vall rows (role 0).
Status launch_ts_rows(const int8_t *roles, int64_t rows, int vall, int v, int64_t sl, int64_t ne, int h, bool cov,
                      uint8_t *bidir, int64_t *head_rows, int64_t *target_row, cudaStream_t s);
Status launch_ts_gate(void *o, int64_t ldo, const void *g, int64_t ldg, int64_t rows, int64_t d, int dtype, cudaStream_t s);
// o16 = f16(v) and its FP8 companion (kernels.h layout) from v = o32 * sigmoid(g) (nn.mulSigmoid,
// in FP32), or v = o32 when g is null: the input of a corrected output projection. d % 8 == 0,
// 16-byte aligned rows.
Status launch_ts_gate_x8(const float *o32, int64_t ld32, const void *g, int64_t ldg, int64_t rows, int64_t d, void *o16,
                         int64_t ldo, void *o8, int64_t ld8, cudaStream_t s);
Status launch_ts_swiglu(const void *h, void *a, int64_t rows, int64_t hid, int dtype, cudaStream_t s);

struct TsVariateCall {
    const void *qkv = nullptr;  // [rows * sl, ld]: q at h*64, k at d + h*64, v at 2d + h*64
    int64_t ld = 0, d = 0;
    void *o = nullptr;
    int64_t ldo = 0;
    int dtype = E_F16;
    int64_t groups = 0, sl = 0, ne = 0;
    int vall = 0, heads = 0;
    const uint8_t *key_valid = nullptr;  // (rows, ne)
    const int8_t *roles = nullptr;
    int cov = 0;
    float scale = 0.125f;
    // Optional output gate (nn.mulSigmoid): o *= sigmoid(gate[row, :]), gate rows at stride ldg.
    const void *gate = nullptr;
    int64_t ldg = 0;
    // FP32 output instead of o, ungated (row stride ld_o32; the tensor-core path only): for a
    // corrected product, whose FP16 input and FP8 companion launch_ts_gate_x8 then forms.
    float *o32 = nullptr;
    int64_t ld_o32 = 0;
};
// With c.gate set the output comes back gated.
Status launch_ts_variate(const TsVariateCall &c, cudaStream_t s);

struct TsHeadCall {
    const float *raw = nullptr;  // (nt * hl, q) head outputs
    float *out = nullptr;        // (nt * hl, q)
    const float *loc = nullptr, *scale = nullptr;  // (rows, n)
    const int64_t *target_row = nullptr;           // nt -> row
    int64_t nt = 0, hl = 0, n = 0, l = 0;
    int q = 0, m = 0;
    const float *widths = nullptr;
    float wf = 2.0f;
    int use_asinh = 1;
};
Status launch_ts_head(const TsHeadCall &c, cudaStream_t s);

struct TsRefineCall {
    float *qs = nullptr;  // (groups * v, h * ps, q), modified in place
    const float *ctx = nullptr;
    const uint8_t *mask = nullptr;
    int64_t t = 0, groups = 0;
    int vall = 0, v = 0, ps = 0, h = 0, q = 0, med = 0;
    double min_scale = 1e-6;
};
Status launch_ts_refine(const TsRefineCall &c, cudaStream_t s);

Status launch_ts_store(const float *qs, float *out, int64_t nt, int64_t blen, int q, int64_t horizon, int64_t done,
                       cudaStream_t s);

struct TsFeedbackCall {
    const float *ctx = nullptr;
    const uint8_t *mask = nullptr;
    int64_t t = 0, rows = 0, keep_t = 0, blen = 0;
    const float *qs = nullptr;  // (groups * v, blen, q)
    int q = 0, med = 0, vall = 0, v = 0;
    const int8_t *roles = nullptr;
    const float *kf = nullptr;  // (rows, hpad) known futures of the whole horizon
    const uint8_t *kfm = nullptr;
    int64_t hpad = 0, done = 0;
    float extreme = 1e30f;
    float *nctx = nullptr;
    uint8_t *nmask = nullptr;
};
Status launch_ts_feedback(const TsFeedbackCall &c, cudaStream_t s);

struct TsCapCall {
    float *out = nullptr;  // (groups * v, horizon, q)
    const float *rows_ctx = nullptr;
    const uint8_t *mask = nullptr;
    int64_t t = 0, groups = 0, horizon = 0;
    int vall = 0, v = 0, q = 0;
    float cap_k = 1e4f;
    double min_scale = 1e-6;
    int *nan_flag = nullptr;
};
Status launch_ts_cap(const TsCapCall &c, cudaStream_t s);

Status launch_ts_finish(const float *fwd, const float *mir, const uint8_t *clip_row, float *out, int64_t rows,
                        int64_t horizon, int q, cudaStream_t s);

}  // namespace tsfm
