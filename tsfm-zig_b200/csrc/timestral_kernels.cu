// Kernels specific to Timestral (timestral/model.zig, timestral/forecaster.zig): per-row causal
// statistics and patch features, per-group RoPE tables, the attention gate and SwiGLU
// activations, the 11x11 variate attention, the monotone quantile head, the refine frame, the
// block feedback, the quantile cap and the symmetric average. Rows of one series are
// contiguous and ordered targets, past-only covariates, known-future covariates.
#include <cfloat>
#include <climits>
#include <type_traits>

#include "kernels.h"
#include "ptx.cuh"
#include "timestral_kernels.h"

#include <cuda_fp16.h>

namespace tsfm {

namespace {

__device__ __forceinline__ float load16(const void *p, int64_t i, int dtype) {
    if (dtype == E_F16) return __half2float(static_cast<const __half *>(p)[i]);
    return __bfloat162float(static_cast<const __nv_bfloat16 *>(p)[i]);
}
__device__ __forceinline__ void store16(void *p, int64_t i, int dtype, float v) {
    if (dtype == E_F16)
        static_cast<__half *>(p)[i] = __float2half_rn(v);
    else
        static_cast<__nv_bfloat16 *>(p)[i] = __float2bfloat16_rn(v);
}

int grid_for(int64_t total, int block) {
    const int64_t g = (total + block - 1) / block;
    const int64_t cap = (int64_t)num_sms() * 16;
    return (int)std::max<int64_t>(1, std::min<int64_t>(g, cap));
}

// Window value / observation at step i of row r: the context, then (with covariates) the known
// futures or blanks (timestral/model.zig:253-274).
struct Win {
    const TsStatsCall &c;
    __device__ float x(int64_t r, int64_t i) const {
        if (i < c.t) return c.ctx[r * c.t + i];
        return c.kf ? c.kf[r * c.kf_ld + (i - c.t)] : 0.0f;
    }
    __device__ bool o(int64_t r, int64_t i) const {
        if (i < c.t) return c.obs[r * c.t + i] != 0;
        return c.kfm ? c.kfm[r * c.kf_ld + (i - c.t)] != 0 : false;
    }
};

// One thread per row: causal per-patch Welford statistics (StatsJob.run,
// timestral/model.zig:712-750), whole-row statistics of known-future rows (model.zig:285-305),
// key validity and the group's first observed patch (model.zig:344-362).
__global__ void ts_stats_kernel(TsStatsCall c) {
    const int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= c.rows) return;
    const Win W{c};
    const int64_t w = c.cov ? c.t + c.hl : c.t, n = w / c.ps;
    const bool known = c.cov && c.roles[r % c.vall] == 2;
    double cum_w = 0, cum_x = 0, m2 = 0, prev = 0;
    bool started = false;
    int first = INT_MAX;
    for (int64_t p = 0; p < n; ++p) {
        bool any = false;
        for (int k = 0; k < c.ps; ++k) {
            const int64_t i = p * c.ps + k;
            const bool ob = W.o(r, i);
            const double wg = ob ? 1.0 : 0.0, x = (double)W.x(r, i);
            cum_w += wg;
            cum_x += wg * x;
            const double den = fmax(cum_w, 1.0);
            const double mean = cum_x / den;
            m2 += (x - prev) * (x - mean) * wg;
            prev = mean;
            any = any || ob;
        }
        const double den = fmax(cum_w, 1.0);
        const double var = m2 / fmax(den - 1.0, 1.0);
        c.loc[r * n + p] = (float)prev;
        c.scale[r * n + p] = (float)fmax(sqrt(var), c.min_scale);
        if (any && first == INT_MAX) first = (int)p;
        started = started || any;
        c.key_valid[r * n + p] = c.attend_missing ? (any || started) : any;
    }
    if (first != INT_MAX) atomicMin(&c.first_obs[r / c.vall], first);
    float kl = 0.0f, ks = 1.0f;
    uint8_t bin = 0;
    if (known) {
        float cnt = 0.0f, sum = 0.0f;
        bool zero_one = true, anyo = false;
        for (int64_t i = 0; i < w; ++i)
            if (W.o(r, i)) {
                const float x = W.x(r, i);
                cnt += 1.0f;
                sum += x;
                zero_one = zero_one && (x == 0.0f || x == 1.0f);
                anyo = true;
            }
        kl = sum / fmaxf(cnt, 1.0f);
        float ss = 0.0f;
        for (int64_t i = 0; i < w; ++i)
            if (W.o(r, i)) {
                const float dv = W.x(r, i) - kl;
                ss += dv * dv;
            }
        ks = fmaxf(sqrtf(ss / fmaxf(cnt, 1.0f)), (float)c.min_scale);
        bin = zero_one && anyo;
        if (bin) {
            kl = 0.0f;
            ks = 1.0f;
        }
    }
    c.kloc[r] = kl;
    c.kscale[r] = ks;
    c.binary[r] = bin;
}

// Patch features [asinh((x - loc_p) / scale_p), missing] per step (timestral/model.zig:306-327).
__global__ void ts_feat_kernel(TsStatsCall c, float *feats) {
    const Win W{c};
    const int64_t w = c.cov ? c.t + c.hl : c.t, n = w / c.ps;
    const int64_t total = c.rows * w;
    for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total; idx += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = idx / w, j = idx % w, p = j / c.ps;
        const int i = (int)(j % c.ps);
        const bool known = c.cov && c.roles[r % c.vall] == 2;
        const float lo = known ? c.kloc[r] : c.loc[r * n + p];
        const float sc = fmaxf(known ? c.kscale[r] : c.scale[r * n + p], FLT_EPSILON);
        const bool ob = W.o(r, j);
        float v = 0.0f;
        if (ob) {
            v = (W.x(r, j) - lo) / sc;
            if (c.use_asinh && !(known && c.binary[r])) v = asinhf(v);
        }
        float *dst = feats + (r * n + p) * 2 * c.ps;
        dst[i] = c.raw_feats ? v : to_tf32(v);
        dst[c.ps + i] = ob ? 0.0f : 1.0f;
    }
}

// cos / sin of rotate-half RoPE per (group, token): encoder token p sits at time p, decoder
// token j at l + j, both relative to the group's first observed patch (model.zig:449-463).
__global__ void ts_rope_kernel(const int *first_obs, int64_t groups, int64_t sl, int64_t ne, int64_t l,
                               const float *inv_freq, int half, float *cs, float *sn) {
    const int64_t total = groups * sl * half;
    for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total; idx += (int64_t)gridDim.x * blockDim.x) {
        const int i = (int)(idx % half);
        const int64_t tok = (idx / half) % sl, g = idx / (half * sl);
        int64_t fo = first_obs[g];
        if (fo >= ne) fo = 0;
        const int64_t time = tok < ne ? tok : l + tok - ne;
        const float ang = inv_freq[i] * (float)(time - fo);
        cs[idx] = cosf(ang);
        sn[idx] = sinf(ang);
    }
}

// One warp per output row, 32 steps per iteration: the forward fill takes, for each lane, the
// value of the last observed step at or before it in this chunk (a ballot), else the carry from
// the previous chunks.
__global__ void __launch_bounds__(256) ts_prepare_kernel(TsPrepareCall c) {
    const int lane = threadIdx.x & 31;
    const int64_t vall = c.v + c.n_past + c.n_known, per_pass = c.b * vall;
    const int64_t r = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    if (r >= per_pass * c.passes) return;
    const bool neg = r >= per_pass;
    const int64_t rr = r % per_pass, s = rr / vall, i = rr % vall;
    const int64_t first = c.t0 - c.keep, pad = c.t - c.keep;
    float *row = c.rows + r * c.t;
    uint8_t *msk = c.mask + r * c.t;
    float *row2 = c.rows2 ? c.rows2 + r * c.t : nullptr;
    uint8_t *msk2 = c.mask2 ? c.mask2 + r * c.t : nullptr;
    for (int64_t j = lane; j < pad; j += 32) {
        row[j] = 0.0f;
        msk[j] = 0;
        if (row2) row2[j] = 0.0f, msk2[j] = 0;
    }
    if (i < c.v) {
        const float *x = c.inputs + (s * c.v + i) * c.t0;
        const uint8_t *ob = c.observed + (s * c.v + i) * c.t0;
        float carry = 0.0f;
        bool seen = false, any = false, nonneg = true;
        for (int64_t j0 = 0; j0 < c.t0; j0 += 32) {
            const int64_t j = j0 + lane;
            const bool in = j < c.t0;
            const bool o = in && ob[j] != 0;
            const float raw = in ? x[j] : 0.0f;
            const float val = neg ? -raw : raw;
            if (o && isfinite(raw)) {
                any = true;
                nonneg = nonneg && raw >= 0.0f;
            }
            const unsigned m = __ballot_sync(0xffffffffu, o);
            const unsigned upto = m & (0xffffffffu >> (31 - lane));
            const float from = __shfl_sync(0xffffffffu, val, upto ? 31 - __clz(upto) : 0);
            const float filled = upto ? from : (seen ? carry : 0.0f);
            if (in && j >= first) {
                row[pad + j - first] = filled;
                msk[pad + j - first] = o ? 1 : 0;
                if (row2) row2[pad + j - first] = filled, msk2[pad + j - first] = o ? 1 : 0;
            }
            if (m) {
                carry = __shfl_sync(0xffffffffu, val, 31 - __clz(m));
                seen = true;
            }
        }
        if (c.clip && !neg) {
            const bool a = __any_sync(0xffffffffu, any), nn = __all_sync(0xffffffffu, nonneg);
            if (lane == 0) c.clip[s * c.v + i] = a && nn;
        }
    } else {
        const bool is_past = i < c.v + c.n_past;
        const float *x = is_past ? c.past + (s * c.n_past + (i - c.v)) * c.t0
                                 : c.known + (s * c.n_known + (i - c.v - c.n_past)) * (c.t0 + c.horizon);
        for (int64_t j = first + lane; j < c.t0; j += 32) {
            const float raw = x[j], val = neg ? -raw : raw;
            const bool o = !isnan(val);
            row[pad + j - first] = o ? val : 0.0f;
            msk[pad + j - first] = o ? 1 : 0;
            if (row2) row2[pad + j - first] = o ? val : 0.0f, msk2[pad + j - first] = o ? 1 : 0;
        }
    }
    // Known futures (zeros for the other rows and past the horizon).
    const bool known_row = i >= c.v + c.n_past;
    const float *xf = known_row ? c.known + (s * c.n_known + (i - c.v - c.n_past)) * (c.t0 + c.horizon) + c.t0 : nullptr;
    for (int64_t j = lane; j < c.hpad; j += 32) {
        float val = 0.0f;
        uint8_t o = 0;
        if (known_row && j < c.horizon) {
            const float raw = xf[j], x = neg ? -raw : raw;
            o = !isnan(x);
            val = o ? x : 0.0f;
        }
        c.kf[r * c.hpad + j] = val;
        c.kfm[r * c.hpad + j] = o;
    }
}

// One warp per series: the forward-filled target of the encoding (values as f64).
__global__ void __launch_bounds__(256) ts_target_kernel(const float *inputs, const uint8_t *observed, int64_t b,
                                                       int64_t t0, int64_t max_context, double *target) {
    const int lane = threadIdx.x & 31;
    const int64_t s = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    if (s >= b) return;
    const float *x = inputs + s * t0;
    const uint8_t *ob = observed + s * t0;
    float carry = 0.0f;
    bool seen = false;
    for (int64_t j0 = 0; j0 < t0; j0 += 32) {
        const int64_t j = j0 + lane;
        const bool o = j < t0 && ob[j] != 0;
        const float val = j < t0 ? x[j] : 0.0f;
        const unsigned m = __ballot_sync(0xffffffffu, o);
        const unsigned upto = m & (0xffffffffu >> (31 - lane));
        const float from = __shfl_sync(0xffffffffu, val, upto ? 31 - __clz(upto) : 0);
        const bool started = upto != 0 || seen;
        const float last = upto ? from : carry;
        if (j < t0) {
            const bool in_window = t0 <= max_context || j >= t0 - max_context;
            target[s * t0 + j] = started && in_window ? (double)last : (double)NAN;
        }
        if (m) {
            carry = __shfl_sync(0xffffffffu, val, 31 - __clz(m));
            seen = true;
        }
    }
}

// One block per (series, categorical channel).
__global__ void __launch_bounds__(256) ts_cat_encode_kernel(const double *codes, int64_t ncat, int64_t len, int64_t t0,
                                                           const double *target, float *out, int64_t chan_total,
                                                           int64_t chan0) {
    const int64_t s = blockIdx.x, ch = blockIdx.y;
    const double *row = codes + (s * ncat + ch) * len;
    float *dst = out + (s * chan_total + chan0 + ch) * len;
    if (target == nullptr) {
        for (int64_t i = threadIdx.x; i < len; i += blockDim.x) dst[i] = (float)row[i];
        return;
    }
    const double *tg = target + s * t0;
    __shared__ double s_mean;
    if (threadIdx.x == 0) {
        double count = 0.0, sum = 0.0;
        for (int64_t k = 0; k < t0; ++k)
            if (isfinite(tg[k])) {
                count += 1.0;
                sum += tg[k];
            }
        s_mean = count > 0.0 ? sum / count : 0.0;
    }
    __syncthreads();
    const double mean = s_mean;
    for (int64_t i = threadIdx.x; i < len; i += blockDim.x) {
        const double c = row[i];
        const bool other = i < t0 ? !isfinite(c) : isnan(c);
        double sum = 0.0, count = 0.0;
        bool known = other;
        for (int64_t k = 0; k < t0; ++k) {
            const double ck = row[k];
            const bool same = other ? !isfinite(ck) : (isfinite(ck) && ck == c);
            known |= same;
            const double tk = tg[k];
            if (same && isfinite(tk)) {
                sum += tk;
                count += 1.0;
            }
        }
        float v;
        if (i < t0) {
            v = (isnan(tg[i]) && isnan(c)) ? NAN : (float)((mean + sum) / (1.0 + count));
        } else {
            v = (float)(known ? (mean + sum) / (1.0 + count) : mean);
        }
        dst[i] = v;
    }
}

// Per-block row maps (model.zig:379-410, 600): the bidirectional flag of every row (known-future
// rows of a covariate window), and for each target row (the first v rows of each group, in order)
// its index and the indices of its h decoder tokens in the (rows * sl) token matrix.
__global__ void ts_rows_kernel(const int8_t *roles, int64_t rows, int vall, int v, int64_t sl, int64_t ne, int h,
                               bool cov, uint8_t *bidir, int64_t *head_rows, int64_t *target_row) {
    for (int64_t row = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; row < rows; row += (int64_t)gridDim.x * blockDim.x) {
        const int j = (int)(row % vall);
        const int role = roles[j];
        bidir[row] = cov && role == 2;
        if (j >= v) continue;
        const int64_t oi = row / vall * v + j;
        target_row[oi] = row;
        for (int jj = 0; jj < h; ++jj) head_rows[oi * h + jj] = row * sl + ne + jj;
    }
}

// o = o * sigmoid(g) (nn.mulSigmoid, core/nn.zig:423-433).
__global__ void ts_gate_kernel(void *o, int64_t ldo, const void *g, int64_t ldg, int64_t rows, int64_t d, int dtype) {
    const int64_t total = rows * d;
    for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total; idx += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = idx / d, j = idx % d;
        const float x = load16(o, r * ldo + j, dtype), gv = load16(g, r * ldg + j, dtype);
        store16(o, r * ldo + j, dtype, x / (1.0f + expf(-gv)));
    }
}

// a = gate * silu(up) with [gate | up] per row (MlpAct.run, timestral/model.zig:159-165).
__global__ void ts_swiglu_kernel(const void *h, void *a, int64_t rows, int64_t hid, int dtype) {
    const int64_t total = rows * hid;
    for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total; idx += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = idx / hid, j = idx % hid;
        const float gt = load16(h, r * 2 * hid + j, dtype), up = load16(h, r * 2 * hid + hid + j, dtype);
        store16(a, idx, dtype, gt * (up / (1.0f + expf(-up))));
    }
}

// 8 consecutive 16-bit values <-> floats.
template <bool F16>
__device__ __forceinline__ void unpack8(const uint4 &u, float (&f)[8]) {
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        if constexpr (F16) {
            const float2 t = __half22float2(*reinterpret_cast<const __half2 *>(&w[i]));
            f[2 * i] = t.x;
            f[2 * i + 1] = t.y;
        } else {
            const float2 t = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&w[i]));
            f[2 * i] = t.x;
            f[2 * i + 1] = t.y;
        }
    }
}
template <bool F16>
__device__ __forceinline__ uint4 pack8(const float (&f)[8]) {
    uint32_t w[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        if constexpr (F16) {
            const __half2 t = __floats2half2_rn(f[2 * i], f[2 * i + 1]);
            w[i] = *reinterpret_cast<const uint32_t *>(&t);
        } else {
            const __nv_bfloat162 t = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
            w[i] = *reinterpret_cast<const uint32_t *>(&t);
        }
    }
    return make_uint4(w[0], w[1], w[2], w[3]);
}

// The gate and SwiGLU above with 16-byte accesses (columns and strides multiples of 8, 16-byte
// aligned bases): blocks stride over rows, threads over 8-column chunks of a row. The logistic
// uses the fast exponential intrinsic (a few ulp; the result is rounded to 16 bits).
template <bool F16>
__global__ void ts_gate_vec_kernel(uint16_t *o, int64_t ldo, const uint16_t *g, int64_t ldg, int64_t rows, int d) {
    for (int64_t r = blockIdx.x; r < rows; r += gridDim.x)
        for (int c = threadIdx.x * 8; c < d; c += blockDim.x * 8) {
            uint4 *po = reinterpret_cast<uint4 *>(o + r * ldo + c);
            float x[8], gv[8];
            unpack8<F16>(*po, x);
            unpack8<F16>(*reinterpret_cast<const uint4 *>(g + r * ldg + c), gv);
#pragma unroll
            for (int i = 0; i < 8; ++i) x[i] = x[i] / (1.0f + __expf(-gv[i]));
            *po = pack8<F16>(x);
        }
}

// v = o32 * sigmoid(g) (or o32) in FP32, then its FP16 value and FP8 companion; 8 columns per
// thread (two float4 loads, one 16-byte FP16 store, 8-byte stores of each companion part).
__global__ void ts_gate_x8_kernel(const float *o32, int64_t ld32, const uint16_t *g, int64_t ldg, int64_t rows, int d,
                                  __half *o16, int64_t ldo, uint8_t *o8, int64_t ld8) {
    for (int64_t r = blockIdx.x; r < rows; r += gridDim.x)
        for (int c = threadIdx.x * 8; c < d; c += blockDim.x * 8) {
            const float4 a = *reinterpret_cast<const float4 *>(o32 + r * ld32 + c);
            const float4 b = *reinterpret_cast<const float4 *>(o32 + r * ld32 + c + 4);
            float x[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
            if (g != nullptr) {
                float gv[8];
                unpack8<true>(*reinterpret_cast<const uint4 *>(g + r * ldg + c), gv);
#pragma unroll
                for (int i = 0; i < 8; ++i) x[i] = x[i] / (1.0f + expf(-gv[i]));
            }
            uint32_t hw[4], hi[2] = {0u, 0u}, lo[2] = {0u, 0u};
#pragma unroll
            for (int i = 0; i < 8; i += 2) {
                const __half2 h2 = __floats2half2_rn(x[i], x[i + 1]);
                hw[i / 2] = *reinterpret_cast<const uint32_t *>(&h2);
                const float2 f = __half22float2(h2);
                hi[i / 4] |= e4m3x2(f.x * kX8HiScale, f.y * kX8HiScale) << (16 * ((i / 2) & 1));
                lo[i / 4] |= e4m3x2((x[i] - f.x) * kX8LoScale, (x[i + 1] - f.y) * kX8LoScale) << (16 * ((i / 2) & 1));
            }
            *reinterpret_cast<uint4 *>(o16 + r * ldo + c) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
            *reinterpret_cast<uint2 *>(o8 + r * ld8 + c) = make_uint2(hi[0], hi[1]);
            *reinterpret_cast<uint2 *>(o8 + r * ld8 + d + c) = make_uint2(lo[0], lo[1]);
        }
}

template <bool F16>
__global__ void ts_swiglu_vec_kernel(const uint16_t *h, uint16_t *a, int64_t rows, int hid) {
    for (int64_t r = blockIdx.x; r < rows; r += gridDim.x)
        for (int c = threadIdx.x * 8; c < hid; c += blockDim.x * 8) {
            float gt[8], up[8];
            unpack8<F16>(*reinterpret_cast<const uint4 *>(h + r * 2 * hid + c), gt);
            unpack8<F16>(*reinterpret_cast<const uint4 *>(h + r * 2 * hid + hid + c), up);
#pragma unroll
            for (int i = 0; i < 8; ++i) gt[i] = gt[i] * (up[i] / (1.0f + __expf(-up[i])));
            *reinterpret_cast<uint4 *>(a + r * hid + c) = pack8<F16>(gt);
        }
}

// Variate attention (VariateJob.run, timestral/model.zig:648-709): at each (group, token) the
// group's rows attend to each other per head. One warp per (group, token, head); each lane owns
// head dims (2 lane, 2 lane + 1).
constexpr int kMaxRows = 16;
__global__ void ts_variate_kernel(TsVariateCall c) {
    const int64_t wid = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    const int64_t total = c.groups * c.sl * c.heads;
    if (wid >= total) return;
    const int h = (int)(wid % c.heads);
    const int64_t tok = (wid / c.heads) % c.sl, g = wid / (c.heads * c.sl);
    const int64_t r0 = g * c.vall;
    float q0[kMaxRows], q1[kMaxRows], k0[kMaxRows], k1[kMaxRows];
    for (int i = 0; i < c.vall; ++i) {
        const int64_t row = (r0 + i) * c.sl + tok;
        const int64_t base = row * c.ld + h * 64 + 2 * lane;
        q0[i] = load16(c.qkv, base, c.dtype);
        q1[i] = load16(c.qkv, base + 1, c.dtype);
        k0[i] = load16(c.qkv, base + c.d, c.dtype);
        k1[i] = load16(c.qkv, base + c.d + 1, c.dtype);
    }
    for (int iq = 0; iq < c.vall; ++iq) {
        float s[kMaxRows];
        float mx = -INFINITY;
        for (int ik = 0; ik < c.vall; ++ik) {
            bool ok = ik == iq;
            if (!ok) {
                const bool valid = tok >= c.ne || c.key_valid[(r0 + ik) * c.ne + tok] != 0;
                bool forbidden = false;
                if (c.cov) {
                    const int rq = c.roles[iq], rk = c.roles[ik];
                    forbidden = (rq != 0 && rk == 0) || (rq == 2 && rk != 2);
                }
                ok = valid && !forbidden;
            }
            float dot = q0[iq] * k0[ik] + q1[iq] * k1[ik];
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
            s[ik] = ok ? dot * c.scale : -INFINITY;
            mx = fmaxf(mx, s[ik]);
        }
        float sum = 0.0f;
        for (int ik = 0; ik < c.vall; ++ik) {
            s[ik] = s[ik] == -INFINITY ? 0.0f : expf(s[ik] - mx);
            sum += s[ik];
        }
        const float inv = 1.0f / sum;
        float o0 = 0.0f, o1 = 0.0f;
        for (int ik = 0; ik < c.vall; ++ik) {
            const float p = s[ik] * inv;
            if (p == 0.0f) continue;
            const int64_t base = ((r0 + ik) * c.sl + tok) * c.ld + 2 * c.d + h * 64 + 2 * lane;
            o0 += p * load16(c.qkv, base, c.dtype);
            o1 += p * load16(c.qkv, base + 1, c.dtype);
        }
        const int64_t ob = ((r0 + iq) * c.sl + tok) * c.ldo + h * 64 + 2 * lane;
        store16(c.o, ob, c.dtype, o0);
        store16(c.o, ob + 1, c.dtype, o1);
    }
}

// The same for V rows per group, known at compile time: 16 lanes per (group, token, head), lane l
// owning head dims 4l .. 4l + 3, so q / k / v of all rows stay in registers (as 16-bit pairs),
// every dot product needs 4 shuffles, and the key masks are read once per instance.
template <int V, bool F16>
__global__ void __launch_bounds__(256, V <= 11 ? 2 : 1) ts_variate_vec_kernel(TsVariateCall c) {
    using H2 = typename std::conditional<F16, __half2, __nv_bfloat162>::type;
    const int64_t inst = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 4;
    const int hl = threadIdx.x & 15;
    const int64_t total = c.groups * c.sl * c.heads;
    // Both halves of a warp take part in the shuffles; an idle half computes instance 0.
    const bool active = inst < total;
    const int64_t id = active ? inst : 0;
    const int h = (int)(id % c.heads);
    const int64_t tok = (id / c.heads) % c.sl, g = id / (c.heads * c.sl);
    const int64_t r0 = g * V;
    auto to_f2 = [](uint32_t w) -> float2 {
        if constexpr (F16)
            return __half22float2(*reinterpret_cast<const __half2 *>(&w));
        else
            return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&w));
    };
    uint2 k[V], v[V];
    uint32_t valid = 0;
    const uint16_t *qrow = static_cast<const uint16_t *>(c.qkv) + (r0 * c.sl + tok) * c.ld + h * 64 + 4 * hl;
    const int64_t row_step = c.sl * c.ld;
#pragma unroll
    for (int i = 0; i < V; ++i) {
        const uint16_t *row = qrow + i * row_step;
        k[i] = *reinterpret_cast<const uint2 *>(row + c.d);
        v[i] = *reinterpret_cast<const uint2 *>(row + 2 * c.d);
        if (tok >= c.ne || c.key_valid[(r0 + i) * c.ne + tok] != 0) valid |= 1u << i;
    }
    int8_t role[V];
#pragma unroll
    for (int i = 0; i < V; ++i) role[i] = c.cov ? c.roles[i] : (int8_t)0;
    auto role_of = [&](int i) -> int { return c.cov ? c.roles[i] : 0; };
    float4 kf[V], vf[V];
#pragma unroll
    for (int i = 0; i < V; ++i) {
        const float2 a = to_f2(k[i].x), b = to_f2(k[i].y);
        kf[i] = make_float4(a.x, a.y, b.x, b.y);
        const float2 c2 = to_f2(v[i].x), d2 = to_f2(v[i].y);
        vf[i] = make_float4(c2.x, c2.y, d2.x, d2.y);
    }
#pragma unroll 1
    for (int iq = 0; iq < V; ++iq) {
        const uint2 qv = *reinterpret_cast<const uint2 *>(qrow + iq * row_step);
        const float2 qa = to_f2(qv.x), qb = to_f2(qv.y);
        float s[V];
        float mx = -INFINITY;
#pragma unroll
        for (int ik = 0; ik < V; ++ik) {
            float dot = qa.x * kf[ik].x + qa.y * kf[ik].y + qb.x * kf[ik].z + qb.y * kf[ik].w;
#pragma unroll
            for (int o = 8; o > 0; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
            const int rq = role_of(iq), rk = role[ik];
            const bool forbidden = (rq != 0 && rk == 0) || (rq == 2 && rk != 2);
            const bool ok = ik == iq || (((valid >> ik) & 1u) && !forbidden);
            s[ik] = ok ? dot * c.scale : -INFINITY;
            mx = fmaxf(mx, s[ik]);
        }
        float sum = 0.0f;
#pragma unroll
        for (int ik = 0; ik < V; ++ik) {
            s[ik] = s[ik] == -INFINITY ? 0.0f : expf(s[ik] - mx);
            sum += s[ik];
        }
        const float inv = 1.0f / sum;
        float o0 = 0.0f, o1 = 0.0f, o2 = 0.0f, o3 = 0.0f;
#pragma unroll
        for (int ik = 0; ik < V; ++ik) {
            const float p = s[ik] * inv;
            if (p == 0.0f) continue;  // masked rows contribute nothing, whatever their values
            o0 += p * vf[ik].x;
            o1 += p * vf[ik].y;
            o2 += p * vf[ik].z;
            o3 += p * vf[ik].w;
        }
        if (active) {
            uint16_t *dst = static_cast<uint16_t *>(c.o) + ((r0 + iq) * c.sl + tok) * c.ldo + h * 64 + 4 * hl;
            H2 lo, hi;
            if constexpr (F16) {
                lo = __floats2half2_rn(o0, o1);
                hi = __floats2half2_rn(o2, o3);
            } else {
                lo = __floats2bfloat162_rn(o0, o1);
                hi = __floats2bfloat162_rn(o2, o3);
            }
            *reinterpret_cast<uint2 *>(dst) = make_uint2(*reinterpret_cast<uint32_t *>(&lo), *reinterpret_cast<uint32_t *>(&hi));
        }
    }
}

// The same attention on the tensor cores, one block per (group, token, half of the heads): the
// q / k / v slices of the group's V rows for those heads are staged in shared memory by
// asynchronous 16-byte copies (rows padded to 16, row stride + 8 elements so ldmatrix rows fall in
// different banks; ≈ 50 KB at 8 heads, four blocks per SM); one warp per head computes S = Q K^T
// (16 x 16, k = 64: eight m16n8k16 MMAs), the masked softmax in registers (rows spread over lane
// quads), and O = P V (16 x 64, k = 16: eight MMAs); the output rows go back through shared
// memory (over the q slices) to coalesced 16-byte stores. The output gate's rows are loaded into
// registers while the copies land, so the gated store phase waits on no global load.
template <int V, bool F16>
__global__ void __launch_bounds__(256, 2) ts_variate_mma_kernel(TsVariateCall c, int nsplit) {
    static_assert(V <= 16, "at most 16 rows per group");
    extern __shared__ __align__(16) unsigned char vsm[];
    const int64_t dw = c.d / nsplit;  // columns of this block's heads
    const int rs = (int)dw + 8;       // row stride (elements)
    uint16_t *qs = reinterpret_cast<uint16_t *>(vsm);
    uint16_t *ks = qs + 16 * rs;
    uint16_t *vs = ks + 16 * rs;
    __shared__ uint32_t s_valid;
    const int64_t gt = blockIdx.x / nsplit;
    const int hs = (int)(blockIdx.x - gt * nsplit);
    const int64_t g = gt / c.sl, tok = gt % c.sl;
    const int64_t r0 = g * V;
    const int64_t hc0 = hs * dw;  // first column of this block's heads
    const int chunks = (int)(dw / 8);
    const int nt = (int)blockDim.x;
    const uint16_t *src = static_cast<const uint16_t *>(c.qkv);
    // chunks is a power of two (checked on the host): the copy index splits by shifts.
    const int csh = __ffs(chunks) - 1;
    for (int idx = threadIdx.x; idx < V * 3 * chunks; idx += nt) {
        const int seg = idx >> csh, ch = idx & (chunks - 1), i = seg / 3, sec = seg - 3 * i;
        const uint16_t *g16 = src + ((r0 + i) * c.sl + tok) * c.ld + sec * c.d + hc0 + ch * 8;
        const uint32_t s16 = smem_u32(qs + sec * 16 * rs + i * rs + ch * 8);
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(s16), "l"(g16) : "memory");
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
    // This thread's gate chunks for the store phase (output chunk idx = threadIdx.x + nt k).
    const uint16_t *gate = static_cast<const uint16_t *>(c.gate);
    constexpr int kPre = 6;
    uint4 gpre[kPre];
    if (gate != nullptr) {
#pragma unroll
        for (int k = 0; k < kPre; ++k) {
            const int idx = threadIdx.x + nt * k;
            if (idx < V * chunks) {
                const int i = idx >> csh, ch = idx & (chunks - 1);
                gpre[k] = __ldg(reinterpret_cast<const uint4 *>(gate + ((r0 + i) * c.sl + tok) * c.ldg + hc0 + ch * 8));
            }
        }
    }
    // Padding rows of K and V are zero (their P is 0; a zero row keeps 0 * row finite).
    if constexpr (V < 16) {
        for (int idx = threadIdx.x; idx < 2 * (16 - V) * chunks; idx += blockDim.x) {
            const int half = idx / ((16 - V) * chunks), rem = idx - half * (16 - V) * chunks;
            const int i = V + rem / chunks, ch = rem % chunks;
            *reinterpret_cast<uint4 *>((half ? vs : ks) + i * rs + ch * 8) = make_uint4(0u, 0u, 0u, 0u);
        }
    }
    if (threadIdx.x == 0) {
        uint32_t vb = 0;
        for (int i = 0; i < V; ++i)
            if (tok >= c.ne || c.key_valid[(r0 + i) * c.ne + tok] != 0) vb |= 1u << i;
        s_valid = vb;
    }
    asm volatile("cp.async.wait_all;" ::: "memory");
    __syncthreads();
    const uint32_t valid = s_valid;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int i0 = lane >> 2, i1 = i0 + 8;  // this thread's two query rows
    const int rq0 = (c.cov && i0 < V) ? c.roles[i0] : 0, rq1 = (c.cov && i1 < V) ? c.roles[i1] : 0;
    const int lheads = c.heads / nsplit;
    for (int h = warp; h < lheads; h += (int)(blockDim.x >> 5)) {
        float sacc[2][4];
#pragma unroll
        for (int nt = 0; nt < 2; ++nt) sacc[nt][0] = sacc[nt][1] = sacc[nt][2] = sacc[nt][3] = 0.0f;
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
            uint32_t a[4], b0, b1, b2, b3;
            const int ar = (lane & 7) + ((lane >> 3) & 1) * 8, ac = h * 64 + kk * 16 + (lane >> 4) * 8;
            ldsm_x4(qs + ar * rs + ac, a[0], a[1], a[2], a[3]);
            const int key = (lane & 7) + (lane >> 4) * 8, dim = h * 64 + kk * 16 + ((lane >> 3) & 1) * 8;
            ldsm_x4(ks + key * rs + dim, b0, b1, b2, b3);
            mma16816<F16>(sacc[0], a, b0, b1);
            mma16816<F16>(sacc[1], a, b2, b3);
        }
        // Mask, scale, softmax per row (the four values of a row per thread, then the lane quad).
        float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
        for (int nt = 0; nt < 2; ++nt)
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int iq = e < 2 ? i0 : i1, ik = nt * 8 + (lane & 3) * 2 + (e & 1);
                const int rq = e < 2 ? rq0 : rq1, rk = (c.cov && ik < V) ? c.roles[ik] : 0;
                const bool forbidden = (rq != 0 && rk == 0) || (rq == 2 && rk != 2);
                const bool ok = iq < V && ik < V && (ik == iq || (((valid >> ik) & 1u) && !forbidden));
                const float x = ok ? sacc[nt][e] * c.scale : -INFINITY;
                sacc[nt][e] = x;
                if (e < 2) mx0 = fmaxf(mx0, x); else mx1 = fmaxf(mx1, x);
            }
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
        const float m0 = mx0 == -INFINITY ? 0.0f : mx0, m1 = mx1 == -INFINITY ? 0.0f : mx1;
        float l0 = 0.0f, l1 = 0.0f;
#pragma unroll
        for (int nt = 0; nt < 2; ++nt)
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const float ev = sacc[nt][e] == -INFINITY ? 0.0f : expf(sacc[nt][e] - (e < 2 ? m0 : m1));
                sacc[nt][e] = ev;
                if (e < 2) l0 += ev; else l1 += ev;
            }
        l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
        l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
        l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
        l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
        const uint32_t pa[4] = {pack16<F16>(sacc[0][0], sacc[0][1]), pack16<F16>(sacc[0][2], sacc[0][3]),
                                pack16<F16>(sacc[1][0], sacc[1][1]), pack16<F16>(sacc[1][2], sacc[1][3])};
        float o[8][4];
#pragma unroll
        for (int nt = 0; nt < 8; ++nt) o[nt][0] = o[nt][1] = o[nt][2] = o[nt][3] = 0.0f;
#pragma unroll
        for (int dp = 0; dp < 4; ++dp) {
            uint32_t b0, b1, b2, b3;
            const int key = (lane & 7) + ((lane >> 3) & 1) * 8, dim = h * 64 + dp * 16 + (lane >> 4) * 8;
            ldsm_x4_t(vs + key * rs + dim, b0, b1, b2, b3);
            mma16816<F16>(o[2 * dp], pa, b0, b1);
            mma16816<F16>(o[2 * dp + 1], pa, b2, b3);
        }
        const float inv0 = l0 > 0.0f ? 1.0f / l0 : 0.0f, inv1 = l1 > 0.0f ? 1.0f / l1 : 0.0f;
        if (c.o32 != nullptr) {  // FP32 rows straight from the accumulators (no gate, no staging)
#pragma unroll
            for (int nt = 0; nt < 8; ++nt) {
                const int col = (int)hc0 + h * 64 + nt * 8 + (lane & 3) * 2;
                if (i0 < V)
                    *reinterpret_cast<float2 *>(c.o32 + ((r0 + i0) * c.sl + tok) * c.ld_o32 + col) =
                        make_float2(o[nt][0] * inv0, o[nt][1] * inv0);
                if (i1 < V)
                    *reinterpret_cast<float2 *>(c.o32 + ((r0 + i1) * c.sl + tok) * c.ld_o32 + col) =
                        make_float2(o[nt][2] * inv1, o[nt][3] * inv1);
            }
            continue;
        }
        // Only this warp reads head h's q columns: its output rows replace them.
        __syncwarp();
#pragma unroll
        for (int nt = 0; nt < 8; ++nt) {
            const int col = h * 64 + nt * 8 + (lane & 3) * 2;
            if (i0 < V) *reinterpret_cast<uint32_t *>(qs + i0 * rs + col) = pack16<F16>(o[nt][0] * inv0, o[nt][1] * inv0);
            if (i1 < V) *reinterpret_cast<uint32_t *>(qs + i1 * rs + col) = pack16<F16>(o[nt][2] * inv1, o[nt][3] * inv1);
        }
    }
    if (c.o32 != nullptr) return;  // every thread: the FP32 rows are written
    __syncthreads();
    uint16_t *dst = static_cast<uint16_t *>(c.o);
    auto store = [&](int idx, bool pre, uint4 gp) {
        const int i = idx >> csh, ch = idx & (chunks - 1);
        const int64_t row = (r0 + i) * c.sl + tok;
        uint4 v = *reinterpret_cast<const uint4 *>(qs + i * rs + ch * 8);
        if (gate != nullptr) {  // the gate kernel's arithmetic on the rounded output
            float x[8], gv[8];
            unpack8<F16>(v, x);
            unpack8<F16>(pre ? gp : __ldg(reinterpret_cast<const uint4 *>(gate + row * c.ldg + hc0 + ch * 8)), gv);
#pragma unroll
            for (int e = 0; e < 8; ++e) x[e] = x[e] / (1.0f + __expf(-gv[e]));
            v = pack8<F16>(x);
        }
        *reinterpret_cast<uint4 *>(dst + row * c.ldo + hc0 + ch * 8) = v;
    };
#pragma unroll
    for (int k = 0; k < kPre; ++k) {
        const int idx = threadIdx.x + nt * k;
        if (idx < V * chunks) store(idx, true, gpre[k]);
    }
    for (int idx = threadIdx.x + nt * kPre; idx < V * chunks; idx += nt)
        store(idx, false, make_uint4(0u, 0u, 0u, 0u));
}


__device__ __forceinline__ float softplus(float x) { return x > 20.0f ? x : log1pf(expf(x)); }

// nn.clampNonfinite (core/nn.zig:522-563) over q values.
__device__ void clamp_nonfinite(float *v, int q) {
    float hi = -INFINITY, lo = INFINITY;
    bool any_inf = false;
    for (int i = 0; i < q; ++i) {
        if (isfinite(v[i])) {
            hi = fmaxf(hi, v[i]);
            lo = fminf(lo, v[i]);
        } else if (isinf(v[i])) {
            any_inf = true;
        }
    }
    if (!any_inf) return;
    for (int i = 0; i < q; ++i) {
        if (v[i] == INFINITY) v[i] = hi;
        if (v[i] == -INFINITY) v[i] = lo;
        if (isinf(v[i])) v[i] = 0.0f;
    }
}

// Monotone quantile head and back-transform (timestral/model.zig:379-431): median free, the
// others at cumulative softplus offsets, then sinh(.) * scale + loc of the anchor frame (the
// last context patch), then clampNonfinite. One thread per (target row, step).
constexpr int kMaxQ = 32;
__global__ void ts_head_kernel(TsHeadCall c) {
    const int64_t total = c.nt * c.hl;
    for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total; idx += (int64_t)gridDim.x * blockDim.x) {
        const int64_t oi = idx / c.hl;
        const int64_t r = c.target_row[oi];
        const float lo = c.loc[r * c.n + c.l - 1], sc = c.scale[r * c.n + c.l - 1];
        const float *rv = c.raw + idx * c.q;
        float ov[kMaxQ];
        const float med = rv[c.m];
        float acc = 0.0f;
        for (int i = c.m + 1; i < c.q; ++i) {
            acc += c.wf * c.widths[i] * softplus(rv[i]);
            ov[i] = fmaxf(-FLT_MAX, fminf(med + acc, FLT_MAX));  // std.math.clamp
        }
        acc = 0.0f;
        for (int i = c.m - 1; i >= 0; --i) {
            acc += c.wf * c.widths[i] * softplus(rv[i]);
            ov[i] = fmaxf(-FLT_MAX, fminf(med - acc, FLT_MAX));
        }
        ov[c.m] = med;
        for (int i = 0; i < c.q; ++i) {
            const float y = c.use_asinh ? sinhf(ov[i]) : ov[i];
            ov[i] = y * sc + lo;
        }
        clamp_nonfinite(ov, c.q);
        for (int i = 0; i < c.q; ++i) c.out[idx * c.q + i] = ov[i];
    }
}

struct Welford {
    double w, mean, m2;
};
__device__ Welford combine(Welford a, Welford b) {  // timestral/forecaster.zig:567-577
    const double w = a.w + b.w;
    if (w == 0) return {0, 0, 0};
    const double w_safe = fmax(w, DBL_MIN);
    const double delta = b.mean - a.mean;
    return {w, a.mean + delta * b.w / w_safe, a.m2 + b.m2 + delta * delta * a.w * b.w / w_safe};
}

// refineBlock (timestral/forecaster.zig:582-662): one thread per target row moves the block
// from the anchor frame to the advancing refine frame.
constexpr int kMaxBlock = 64;
__global__ void ts_refine_kernel(TsRefineCall c) {
    const int64_t tr = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (tr >= c.groups * c.v) return;
    const int64_t g = tr / c.v, i = tr % c.v, r = g * c.vall + i;
    const float *row = c.ctx + r * c.t;
    const uint8_t *msk = c.mask + r * c.t;
    const int64_t l = c.t / c.ps;
    // Causal statistics at the last context patch (the anchor frame).
    double cum_w = 0, cum_x = 0, m2 = 0, prev = 0;
    for (int64_t j = 0; j < c.t; ++j) {
        const double wg = msk[j] ? 1.0 : 0.0, x = (double)row[j];
        cum_w += wg;
        cum_x += wg * x;
        const double mean = cum_x / fmax(cum_w, 1.0);
        m2 += (x - prev) * (x - mean) * wg;
        prev = mean;
    }
    const float loc0 = (float)prev;
    const float scale0 = (float)fmax(sqrt(m2 / fmax(fmax(cum_w, 1.0) - 1.0, 1.0)), c.min_scale);
    float *block = c.qs + tr * c.h * c.ps * c.q;
    Welford st{0, 0, 0};
    for (int64_t p = 0; p < l; ++p) {
        double cnt = 0, sum = 0;
        for (int k = 0; k < c.ps; ++k)
            if (msk[p * c.ps + k]) {
                cnt += 1;
                sum += row[p * c.ps + k];
            }
        Welford pm{cnt, 0, 0};
        if (cnt > 0) {
            pm.mean = sum / fmax(cnt, 1.0);
            for (int k = 0; k < c.ps; ++k)
                if (msk[p * c.ps + k]) {
                    const double dv = (double)row[p * c.ps + k] - pm.mean;
                    pm.m2 += dv * dv;
                }
        }
        st = combine(st, pm);
    }
    const double clip = sqrt((double)FLT_MAX) / 1e3;
    const double offset = st.mean;
    float loc_j[kMaxBlock], scale_j[kMaxBlock];
    for (int j = 0; j < c.h; ++j) {
        const double var = fmax(st.m2 / fmax(st.w - 1.0, 1.0), 0.0);
        const double sc = fmax(sqrt(var), c.min_scale);
        loc_j[j] = (float)st.mean;
        scale_j[j] = (float)sc;
        double bsum = 0;
        for (int k = 0; k < c.ps; ++k) {
            const double sm = ((double)block[(j * c.ps + k) * c.q + c.med] - (double)loc0) / (double)scale0;
            bsum += fmax(-clip, fmin(sm * sc + st.mean - offset, clip)) + offset;  // std.math.clamp
        }
        const double bmean = bsum / (double)c.ps;
        double bm2 = 0;
        for (int k = 0; k < c.ps; ++k) {
            const double sm = ((double)block[(j * c.ps + k) * c.q + c.med] - (double)loc0) / (double)scale0;
            const double f = fmax(-clip, fmin(sm * sc + st.mean - offset, clip)) + offset;
            bm2 += (f - bmean) * (f - bmean);
        }
        st = combine(st, {(double)c.ps, bmean, bm2});
    }
    loc_j[0] = loc0;
    scale_j[0] = scale0;
    for (int64_t s = 0; s < (int64_t)c.h * c.ps; ++s) {
        float *rowq = block + s * c.q;
        const float lj = loc_j[s / c.ps], sj = scale_j[s / c.ps];
        for (int k = 0; k < c.q; ++k) rowq[k] = (rowq[k] - loc0) / scale0 * sj + lj;
        clamp_nonfinite(rowq, c.q);
    }
}

// Store a decoded block into the (targets, horizon, q) output and build the next context
// (timestral/forecaster.zig:502-560).
__global__ void ts_store_kernel(const float *qs, float *out, int64_t nt, int64_t blen, int q, int64_t horizon,
                                int64_t done) {
    const int64_t total = nt * blen * q;
    for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total; idx += (int64_t)gridDim.x * blockDim.x) {
        const int64_t rt = idx / (blen * q), s = (idx / q) % blen;
        if (done + s < horizon) out[(rt * horizon + done + s) * q + idx % q] = qs[idx];
    }
}

__global__ void ts_feedback_kernel(TsFeedbackCall c) {
    const int64_t total = c.rows * c.keep_t;
    for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total; idx += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = idx / c.keep_t, j = idx % c.keep_t;
        const int64_t nt_len = c.t + c.blen, start = nt_len - c.keep_t;
        const int64_t ncopy = start < c.t ? c.t - start : 0;
        float val;
        uint8_t ob;
        if (j < ncopy) {
            val = c.ctx[r * c.t + start + j];
            ob = c.mask[r * c.t + start + j];
        } else {
            const int64_t s = (start < c.t ? 0 : start - c.t) + (j - ncopy);
            const int role = c.roles[r % c.vall];
            if (role == 0) {
                const int64_t trow = (r / c.vall) * c.v + (r % c.vall);
                float m = c.qs[(trow * c.blen + s) * c.q + c.med];
                if (!isfinite(m) || fabsf(m) >= c.extreme) m = 0.0f;
                val = m;
                ob = 1;
            } else if (role == 2) {
                val = c.kf[r * c.hpad + c.done + s];
                ob = c.kfm[r * c.hpad + c.done + s];
            } else {
                val = 0.0f;
                ob = 0;
            }
        }
        c.nctx[idx] = val;
        c.nmask[idx] = ob;
    }
}

// Quantile cap (timestral/forecaster.zig:396-418) and the NaN check (:419): one thread per target
// row computes the statistics of its initial context, then clamps its (horizon, q) block.
__global__ void ts_cap_kernel(TsCapCall c) {
    const int64_t tr = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (tr >= c.groups * c.v) return;
    const int64_t r = (tr / c.v) * c.vall + tr % c.v;
    const float *row = c.rows_ctx + r * c.t;
    const uint8_t *msk = c.mask + r * c.t;
    float *o = c.out + tr * c.horizon * c.q;
    if (c.cap_k > 0.0f) {
        double cum_w = 0, cum_x = 0, m2 = 0, prev = 0;
        float mx = -INFINITY, mn = INFINITY;
        for (int64_t j = 0; j < c.t; ++j) {
            const double wg = msk[j] ? 1.0 : 0.0, x = (double)row[j];
            cum_w += wg;
            cum_x += wg * x;
            const double mean = cum_x / fmax(cum_w, 1.0);
            m2 += (x - prev) * (x - mean) * wg;
            prev = mean;
            if (msk[j]) {
                mx = fmaxf(mx, row[j]);
                mn = fminf(mn, row[j]);
            }
        }
        const float scale_last = (float)fmax(sqrt(m2 / fmax(fmax(cum_w, 1.0) - 1.0, 1.0)), c.min_scale);
        if (isinf(mx)) mx = 0.0f;
        if (isinf(mn)) mn = 0.0f;
        const float a = scale_last * c.cap_k;
        for (int64_t k = 0; k < c.horizon * c.q; ++k) o[k] = fmaxf(mn - a, fminf(o[k], mx + a));  // std.math.clamp
    }
    for (int64_t k = 0; k < c.horizon * c.q; ++k)
        if (isnan(o[k])) atomicOr(c.nan_flag, 1);
}

// Symmetric averaging 0.5 * (a_j - m_{q-1-j}) and the non-negative clip
// (timestral/forecaster.zig:132-136, 163-180).
__global__ void ts_finish_kernel(const float *fwd, const float *mir, const uint8_t *clip_row, float *out, int64_t rows,
                                 int64_t horizon, int q) {
    const int64_t total = rows * horizon * q;
    for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total; idx += (int64_t)gridDim.x * blockDim.x) {
        const int j = (int)(idx % q);
        const int64_t base = idx - j, r = idx / (horizon * q);
        float v = fwd[idx];
        if (mir) v = 0.5f * (v + -mir[base + (q - 1 - j)]);
        if (clip_row && clip_row[r]) v = fmaxf(v, 0.0f);
        out[idx] = v;
    }
}

}  // namespace

Status launch_ts_stats(const TsStatsCall &c, float *feats, cudaStream_t s) {
    if (c.rows <= 0) return Status::ok();
    ts_stats_kernel<<<(unsigned)((c.rows + 127) / 128), 128, 0, s>>>(c);
    TSFM_CUDA(cudaGetLastError(), "timestral stats: launch");
    const int64_t w = c.cov ? c.t + c.hl : c.t;
    ts_feat_kernel<<<grid_for(c.rows * w, 256), 256, 0, s>>>(c, feats);
    TSFM_CUDA(cudaGetLastError(), "timestral features: launch");
    return Status::ok();
}

Status launch_ts_rope(const int *first_obs, int64_t groups, int64_t sl, int64_t ne, int64_t l, const float *inv_freq,
                      int half, float *cs, float *sn, cudaStream_t s) {
    ts_rope_kernel<<<grid_for(groups * sl * half, 256), 256, 0, s>>>(first_obs, groups, sl, ne, l, inv_freq, half, cs, sn);
    TSFM_CUDA(cudaGetLastError(), "timestral rope: launch");
    return Status::ok();
}

Status launch_ts_prepare(const TsPrepareCall &c, cudaStream_t s) {
    const int64_t rows = (c.v + c.n_past + c.n_known) * c.b * c.passes;
    if (rows <= 0) return Status::ok();
    if (c.keep > c.t0 || c.keep > c.t) return Status::fail(TSFM_ERR_INVALID_ARGUMENT, "timestral prepare: keep");
    ts_prepare_kernel<<<(unsigned)((rows + 7) / 8), 256, 0, s>>>(c);
    TSFM_CUDA(cudaGetLastError(), "timestral prepare: launch");
    return Status::ok();
}

Status launch_ts_target(const float *inputs, const uint8_t *observed, int64_t b, int64_t t0, int64_t max_context,
                        double *target, cudaStream_t s) {
    if (b <= 0 || t0 <= 0) return Status::ok();
    ts_target_kernel<<<(unsigned)((b + 7) / 8), 256, 0, s>>>(inputs, observed, b, t0, max_context, target);
    TSFM_CUDA(cudaGetLastError(), "timestral target: launch");
    return Status::ok();
}

Status launch_ts_cat_encode(const double *codes, int64_t b, int64_t ncat, int64_t len, int64_t t0, const double *target,
                            float *out, int64_t chan_total, int64_t chan0, cudaStream_t s) {
    if (b <= 0 || ncat <= 0 || len <= 0) return Status::ok();
    if (b > INT_MAX || ncat > 65535) return Status::fail(TSFM_ERR_INVALID_ARGUMENT, "timestral categorical: too many rows");
    ts_cat_encode_kernel<<<dim3((unsigned)b, (unsigned)ncat), 256, 0, s>>>(codes, ncat, len, t0, target, out, chan_total,
                                                                          chan0);
    TSFM_CUDA(cudaGetLastError(), "timestral categorical: launch");
    return Status::ok();
}

Status launch_ts_rows(const int8_t *roles, int64_t rows, int vall, int v, int64_t sl, int64_t ne, int h, bool cov,
                      uint8_t *bidir, int64_t *head_rows, int64_t *target_row, cudaStream_t s) {
    if (rows <= 0) return Status::ok();
    ts_rows_kernel<<<grid_for(rows, 256), 256, 0, s>>>(roles, rows, vall, v, sl, ne, h, cov, bidir, head_rows, target_row);
    TSFM_CUDA(cudaGetLastError(), "timestral rows: launch");
    return Status::ok();
}

bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

Status launch_ts_gate(void *o, int64_t ldo, const void *g, int64_t ldg, int64_t rows, int64_t d, int dtype, cudaStream_t s) {
    if (aligned16(o) && aligned16(g) && d % 8 == 0 && ldo % 8 == 0 && ldg % 8 == 0 && d <= INT_MAX && rows > 0) {
        const int grid = (int)std::min<int64_t>(rows, (int64_t)num_sms() * 16);
        if (dtype == E_F16)
            ts_gate_vec_kernel<true><<<grid, 128, 0, s>>>(static_cast<uint16_t *>(o), ldo,
                                                          static_cast<const uint16_t *>(g), ldg, rows, (int)d);
        else
            ts_gate_vec_kernel<false><<<grid, 128, 0, s>>>(static_cast<uint16_t *>(o), ldo,
                                                           static_cast<const uint16_t *>(g), ldg, rows, (int)d);
    } else {
        ts_gate_kernel<<<grid_for(rows * d, 256), 256, 0, s>>>(o, ldo, g, ldg, rows, d, dtype);
    }
    TSFM_CUDA(cudaGetLastError(), "timestral gate: launch");
    return Status::ok();
}

Status launch_ts_gate_x8(const float *o32, int64_t ld32, const void *g, int64_t ldg, int64_t rows, int64_t d, void *o16,
                         int64_t ldo, void *o8, int64_t ld8, cudaStream_t s) {
    if (rows <= 0) return Status::ok();
    if (!aligned16(o32) || !aligned16(o16) || !aligned16(o8) || (g && (!aligned16(g) || ldg % 8)) || d % 8 ||
        ld32 % 4 || ldo % 8 || ld8 % 16 || ld8 < 2 * d || d > INT_MAX)
        return Status::fail(TSFM_ERR_INVALID_ARGUMENT, "timestral gate (corrected): alignment");
    const int grid = (int)std::min<int64_t>(rows, (int64_t)num_sms() * 16);
    ts_gate_x8_kernel<<<grid, 128, 0, s>>>(o32, ld32, static_cast<const uint16_t *>(g), ldg, rows, (int)d,
                                           static_cast<__half *>(o16), ldo, static_cast<uint8_t *>(o8), ld8);
    TSFM_CUDA(cudaGetLastError(), "timestral gate (corrected): launch");
    return Status::ok();
}

Status launch_ts_swiglu(const void *h, void *a, int64_t rows, int64_t hid, int dtype, cudaStream_t s) {
    if (aligned16(h) && aligned16(a) && hid % 8 == 0 && hid <= INT_MAX / 2 && rows > 0) {
        const int grid = (int)std::min<int64_t>(rows, (int64_t)num_sms() * 16);
        if (dtype == E_F16)
            ts_swiglu_vec_kernel<true><<<grid, 256, 0, s>>>(static_cast<const uint16_t *>(h), static_cast<uint16_t *>(a),
                                                            rows, (int)hid);
        else
            ts_swiglu_vec_kernel<false><<<grid, 256, 0, s>>>(static_cast<const uint16_t *>(h), static_cast<uint16_t *>(a),
                                                             rows, (int)hid);
    } else {
        ts_swiglu_kernel<<<grid_for(rows * hid, 256), 256, 0, s>>>(h, a, rows, hid, dtype);
    }
    TSFM_CUDA(cudaGetLastError(), "timestral swiglu: launch");
    return Status::ok();
}

template <int V>
bool variate_vec(const TsVariateCall &c, cudaStream_t s) {  // true: gate applied
    // Block per (group, token) on the tensor cores when the rows are 16-byte aligned and the group's
    // slices (16 padded rows of q, k and v) fit.
    // Heads split over two blocks of 128 threads when their count is even (four blocks per SM,
    // each with half the copies, so one block's copies overlap another's arithmetic).
    const int nsplit = c.heads % 2 == 0 ? 2 : 1;
    const unsigned nthr = nsplit == 2 ? 128u : 256u;
    const int64_t chunks = c.d / nsplit / 8;
    const size_t smem = (size_t)3 * 16 * (c.d / nsplit + 8) * 2;
    const bool a16 = (reinterpret_cast<uintptr_t>(c.qkv) & 15) == 0 && (reinterpret_cast<uintptr_t>(c.o) & 15) == 0 &&
                     c.ld % 8 == 0 && c.d % 8 == 0 && c.ldo % 8 == 0 && c.d == (int64_t)c.heads * 64 &&
                     (c.gate == nullptr || ((reinterpret_cast<uintptr_t>(c.gate) & 15) == 0 && c.ldg % 8 == 0)) &&
                     chunks > 0 && (chunks & (chunks - 1)) == 0;
    if (a16 && smem <= 200 * 1024 && c.groups * c.sl * nsplit <= INT_MAX) {
        const void *fn = c.dtype == E_F16 ? reinterpret_cast<const void *>(&ts_variate_mma_kernel<V, true>)
                                          : reinterpret_cast<const void *>(&ts_variate_mma_kernel<V, false>);
        if (ensure_smem_attr(fn, (int)smem)) {
            const unsigned grid = (unsigned)(c.groups * c.sl * nsplit);
            if (c.dtype == E_F16)
                ts_variate_mma_kernel<V, true><<<grid, nthr, smem, s>>>(c, nsplit);
            else
                ts_variate_mma_kernel<V, false><<<grid, nthr, smem, s>>>(c, nsplit);
            return true;
        }
    }
    if (c.o32 != nullptr) return false;  // FP32 output: tensor-core path only (the caller reports it)
    const int64_t threads = c.groups * c.sl * c.heads * 16;
    const unsigned grid = (unsigned)((threads + 255) / 256);
    if (c.dtype == E_F16)
        ts_variate_vec_kernel<V, true><<<grid, 256, 0, s>>>(c);
    else
        ts_variate_vec_kernel<V, false><<<grid, 256, 0, s>>>(c);
    return false;
}

Status launch_ts_variate(const TsVariateCall &c, cudaStream_t s) {
    if (c.vall > kMaxRows) return Status::fail(TSFM_ERR_UNSUPPORTED, "Timestral: more than 16 rows per series");
    if (c.o32 && (c.gate || c.ld_o32 % 2 || (reinterpret_cast<uintptr_t>(c.o32) & 7)))
        return Status::fail(TSFM_ERR_INVALID_ARGUMENT, "timestral variate attention: FP32 output is ungated, 8-byte aligned");
    // 8-byte accesses per lane: row strides, the k / v offset and the base even in 4-element units.
    if ((c.ld % 4) == 0 && (c.d % 4) == 0 && (c.ldo % 4) == 0 && (reinterpret_cast<uintptr_t>(c.qkv) & 7) == 0 &&
        (reinterpret_cast<uintptr_t>(c.o) & 7) == 0 && c.groups * c.sl * c.heads * 16 < (int64_t)UINT_MAX * 256 / 2) {
        bool gated = false;
        switch (c.vall) {
        case 1: gated = variate_vec<1>(c, s); break;
        case 2: gated = variate_vec<2>(c, s); break;
        case 3: gated = variate_vec<3>(c, s); break;
        case 4: gated = variate_vec<4>(c, s); break;
        case 5: gated = variate_vec<5>(c, s); break;
        case 6: gated = variate_vec<6>(c, s); break;
        case 7: gated = variate_vec<7>(c, s); break;
        case 8: gated = variate_vec<8>(c, s); break;
        case 9: gated = variate_vec<9>(c, s); break;
        case 10: gated = variate_vec<10>(c, s); break;
        case 11: gated = variate_vec<11>(c, s); break;
        case 12: gated = variate_vec<12>(c, s); break;
        case 13: gated = variate_vec<13>(c, s); break;
        case 14: gated = variate_vec<14>(c, s); break;
        case 15: gated = variate_vec<15>(c, s); break;
        default: gated = variate_vec<16>(c, s); break;
        }
        TSFM_CUDA(cudaGetLastError(), "timestral variate attention: launch");
        if (c.o32 && !gated)
            return Status::fail(TSFM_ERR_UNSUPPORTED, "timestral variate attention: FP32 output needs the tensor-core path");
        if (c.gate && !gated)
            return launch_ts_gate(c.o, c.ldo, c.gate, c.ldg, c.groups * c.vall * c.sl, c.d, c.dtype, s);
        return Status::ok();
    }
    if (c.o32) return Status::fail(TSFM_ERR_UNSUPPORTED, "timestral variate attention: FP32 output needs the tensor-core path");
    const int64_t warps = c.groups * c.sl * c.heads;
    ts_variate_kernel<<<(unsigned)((warps * 32 + 255) / 256), 256, 0, s>>>(c);
    TSFM_CUDA(cudaGetLastError(), "timestral variate attention: launch");
    if (c.gate) return launch_ts_gate(c.o, c.ldo, c.gate, c.ldg, c.groups * c.vall * c.sl, c.d, c.dtype, s);
    return Status::ok();
}

Status launch_ts_head(const TsHeadCall &c, cudaStream_t s) {
    if (c.q > kMaxQ) return Status::fail(TSFM_ERR_UNSUPPORTED, "Timestral: more than 32 quantiles");
    ts_head_kernel<<<grid_for(c.nt * c.hl, 128), 128, 0, s>>>(c);
    TSFM_CUDA(cudaGetLastError(), "timestral head: launch");
    return Status::ok();
}

Status launch_ts_refine(const TsRefineCall &c, cudaStream_t s) {
    if (c.h > kMaxBlock) return Status::fail(TSFM_ERR_UNSUPPORTED, "Timestral: block longer than 64 patches");
    const int64_t n = c.groups * c.v;
    ts_refine_kernel<<<(unsigned)((n + 63) / 64), 64, 0, s>>>(c);
    TSFM_CUDA(cudaGetLastError(), "timestral refine: launch");
    return Status::ok();
}

Status launch_ts_store(const float *qs, float *out, int64_t nt, int64_t blen, int q, int64_t horizon, int64_t done,
                       cudaStream_t s) {
    ts_store_kernel<<<grid_for(nt * blen * q, 256), 256, 0, s>>>(qs, out, nt, blen, q, horizon, done);
    TSFM_CUDA(cudaGetLastError(), "timestral store: launch");
    return Status::ok();
}

Status launch_ts_feedback(const TsFeedbackCall &c, cudaStream_t s) {
    ts_feedback_kernel<<<grid_for(c.rows * c.keep_t, 256), 256, 0, s>>>(c);
    TSFM_CUDA(cudaGetLastError(), "timestral feedback: launch");
    return Status::ok();
}

Status launch_ts_cap(const TsCapCall &c, cudaStream_t s) {
    const int64_t n = c.groups * c.v;
    ts_cap_kernel<<<(unsigned)((n + 63) / 64), 64, 0, s>>>(c);
    TSFM_CUDA(cudaGetLastError(), "timestral cap: launch");
    return Status::ok();
}

Status launch_ts_finish(const float *fwd, const float *mir, const uint8_t *clip_row, float *out, int64_t rows,
                        int64_t horizon, int q, cudaStream_t s) {
    ts_finish_kernel<<<grid_for(rows * horizon * q, 256), 256, 0, s>>>(fwd, mir, clip_row, out, rows, horizon, q);
    TSFM_CUDA(cudaGetLastError(), "timestral finish: launch");
    return Status::ok();
}

}  // namespace tsfm
