// Fused flash attention for the patched encoders and the Timestral decoder: one CTA per
// (64-query block, head, group), K/V streamed in 64-key tiles through a double-buffered
// cp.async ring into XOR-swizzled shared memory, S = Q K^T and O += P V on BF16 tensor cores
// with FP32 accumulation, online softmax in registers; the n x n score matrix is never
// materialised (the reference builds it per (series, head): core/attn.zig:72-96).
//
// Masks, applied in-tile per (query i, key j):
//   mode 0 (T5, chronos2/model.zig:283-308, chronos_bolt/model.zig:343-357): invalid keys are
//     excluded, which equals the reference's additive -floatMax for any row that has a valid key;
//     a group with no valid key at all averages V uniformly, as -floatMax + s rounds every score
//     to the same value. Optional relative-position bias rel[h][j - i + n - 1] (positionBias,
//     chronos_bolt/model.zig:195-205), added before the mask; scale 1 (T5 convention).
//   mode 1 (Timestral, timestral/model.zig:558-635): encoder queries i < ne read encoder keys
//     j < ne with j == i or (valid(j) and j <= i) — or any valid j for bidirectional (known
//     covariate) groups; decoder queries i >= ne read valid keys j < l plus their causal decoder
//     chain ne <= j <= i.
#include "kernels.h"
#include "ptx.cuh"

#include <cuda_fp16.h>

namespace tsfm {

namespace {

constexpr int BQ = 64, BKV = 64, HD = 64;
constexpr float kLog2e = 1.4426950408889634f;

struct AttnP {
    const uint16_t *q, *k, *v;  // 16-bit elements (BF16 or FP16)
    int64_t ld;
    uint16_t *o;
    int64_t ldo;
    float *o32;  // FP32 output instead of o when set
    int64_t ldo32;
    const uint8_t *key_valid;
    int64_t kvs;
    const float *rel;
    int64_t rel_stride, rel_center;
    int n, heads;
    float scale_log2;
    int ne, l;
    const uint8_t *bidir;
    int bidir_all;
};

__device__ __forceinline__ int swz(int r, int c) { return r * HD + ((((c >> 3) ^ (r & 7))) << 3) + (c & 7); }

__device__ __forceinline__ void cp_async16(void *smem, const void *gmem, bool pred) {
    const int sz = pred ? 16 : 0;
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(smem)), "l"(gmem), "r"(sz) : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

template <int MODE, bool F16>
__global__ void __launch_bounds__(128) attn_kernel(AttnP p) {
    __shared__ __align__(128) uint16_t sQ[BQ * HD];
    __shared__ __align__(128) uint16_t sK[2][BKV * HD];
    __shared__ __align__(128) uint16_t sV[2][BKV * HD];
    __shared__ uint8_t sValid[2][BKV];

    const int qb = blockIdx.x, h = blockIdx.y, g = blockIdx.z;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int n = p.n;
    const int64_t row0 = (int64_t)g * n;
    const int q0 = qb * BQ;
    const uint8_t *kv_g = p.key_valid ? p.key_valid + (int64_t)g * p.kvs : nullptr;

    bool uniform = false;
    if (MODE == 0 && kv_g) {
        int any = 0;
        for (int j = tid; j < n && j < p.kvs; j += 128) any |= kv_g[j];
        if (n > p.kvs) any = 1;
        uniform = __syncthreads_or(any) == 0;
    }
    const bool bidir = MODE == 1 && (p.bidir_all || (p.bidir && p.bidir[g]));
    const int qhi = min(n, q0 + BQ);
    int kv_end = n;
    if (MODE == 1) kv_end = bidir ? max(p.ne, qhi) : qhi;
    const int ntiles = (kv_end + BKV - 1) / BKV;

    // Q tile (64 rows x 64 dims, 8 x 16-byte chunks per row).
    for (int c = tid; c < BQ * 8; c += 128) {
        const int r = c >> 3, ch = c & 7;
        const int tok = q0 + r;
        const uint16_t *src = p.q + (row0 + min(tok, n - 1)) * p.ld + h * HD + ch * 8;
        cp_async16(&sQ[swz(r, ch * 8)], src, tok < n);
    }
    auto load_kv = [&](int kt, int buf) {
        const int j0 = kt * BKV;
        for (int c = tid; c < BKV * 8; c += 128) {
            const int r = c >> 3, ch = c & 7;
            const int tok = j0 + r;
            const int64_t off = (row0 + min(tok, n - 1)) * p.ld + h * HD + ch * 8;
            cp_async16(&sK[buf][swz(r, ch * 8)], p.k + off, tok < n);
            cp_async16(&sV[buf][swz(r, ch * 8)], p.v + off, tok < n);
        }
        if (tid < BKV) {
            const int j = j0 + tid;
            uint8_t ok = j < n;
            if (ok && kv_g && j < p.kvs) ok = kv_g[j] != 0;
            sValid[buf][tid] = ok;
        }
    };
    load_kv(0, 0);
    cp_commit();

    float m_run[2] = {-INFINITY, -INFINITY};
    float l_run[2] = {0.0f, 0.0f};
    float o[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.0f;
    uint32_t qf[4][4];
    const int qi0 = q0 + warp * 16 + (lane >> 2), qi1 = qi0 + 8;

    for (int kt = 0; kt < ntiles; ++kt) {
        const int buf = kt & 1;
        if (kt + 1 < ntiles) {
            load_kv(kt + 1, buf ^ 1);
            cp_commit();
            cp_wait<1>();
        } else {
            cp_wait<0>();
        }
        __syncthreads();
        if (kt == 0) {
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
                const int r = warp * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
                const int c = kk * 16 + (lane >> 4) * 8;
                ldsm_x4(&sQ[swz(r, c)], qf[kk][0], qf[kk][1], qf[kk][2], qf[kk][3]);
            }
        }
        // S = Q K^T for the warp's 16 queries x 64 keys.
        float s[8][4];
#pragma unroll
        for (int i = 0; i < 8; ++i) s[i][0] = s[i][1] = s[i][2] = s[i][3] = 0.0f;
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
#pragma unroll
            for (int np = 0; np < 4; ++np) {
                const int key = np * 16 + (lane & 7) + (lane >> 4) * 8;
                const int dim = kk * 16 + ((lane >> 3) & 1) * 8;
                uint32_t b0, b1, b2, b3;
                ldsm_x4(&sK[buf][swz(key, dim)], b0, b1, b2, b3);
                mma16816<F16>(s[2 * np], qf[kk], b0, b1);
                mma16816<F16>(s[2 * np + 1], qf[kk], b2, b3);
            }
        }
        // Scale, bias, mask.
        const int j_base = kt * BKV;
#pragma unroll
        for (int nt = 0; nt < 8; ++nt) {
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int jl = nt * 8 + (lane & 3) * 2 + (e & 1);
                const int j = j_base + jl;
                const int i = e < 2 ? qi0 : qi1;
                const bool valid = sValid[buf][jl] != 0;
                float x = s[nt][e] * p.scale_log2;
                bool allowed;
                if (MODE == 0) {
                    if (uniform) {
                        allowed = j < n;
                        x = 0.0f;
                    } else {
                        allowed = valid;
                        if (p.rel && allowed && i < n) x += __ldg(p.rel + (int64_t)h * p.rel_stride + (j - i) + p.rel_center) * kLog2e;
                    }
                } else {
                    if (i < p.ne)
                        allowed = j < p.ne && (j == i || (valid && (bidir || j <= i)));
                    else
                        allowed = j < n && ((j < p.l && valid) || (j >= p.ne && j <= i));
                }
                s[nt][e] = allowed ? x : -INFINITY;
            }
        }
        // Online softmax per query row (two rows per thread, reduced across the quad).
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            float mx = -INFINITY;
#pragma unroll
            for (int nt = 0; nt < 8; ++nt) mx = fmaxf(mx, fmaxf(s[nt][2 * r], s[nt][2 * r + 1]));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
            const float m_new = fmaxf(m_run[r], mx);
            const float m_use = m_new == -INFINITY ? 0.0f : m_new;
            const float corr = exp2f(m_run[r] - m_use);
            float sum = 0.0f;
#pragma unroll
            for (int nt = 0; nt < 8; ++nt) {
                s[nt][2 * r] = exp2f(s[nt][2 * r] - m_use);
                s[nt][2 * r + 1] = exp2f(s[nt][2 * r + 1] - m_use);
                sum += s[nt][2 * r] + s[nt][2 * r + 1];
            }
            l_run[r] = l_run[r] * corr + sum;
#pragma unroll
            for (int nt = 0; nt < 8; ++nt) {
                o[nt][2 * r] *= corr;
                o[nt][2 * r + 1] *= corr;
            }
            m_run[r] = m_new;
        }
        // O += P V.
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
            uint32_t a[4];
            a[0] = pack16<F16>(s[2 * kk][0], s[2 * kk][1]);
            a[1] = pack16<F16>(s[2 * kk][2], s[2 * kk][3]);
            a[2] = pack16<F16>(s[2 * kk + 1][0], s[2 * kk + 1][1]);
            a[3] = pack16<F16>(s[2 * kk + 1][2], s[2 * kk + 1][3]);
#pragma unroll
            for (int dp = 0; dp < 4; ++dp) {
                const int key = kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
                const int dim = dp * 16 + (lane >> 4) * 8;
                uint32_t b0, b1, b2, b3;
                ldsm_x4_t(&sV[buf][swz(key, dim)], b0, b1, b2, b3);
                mma16816<F16>(o[2 * dp], a, b0, b1);
                mma16816<F16>(o[2 * dp + 1], a, b2, b3);
            }
        }
        __syncthreads();
    }

#pragma unroll
    for (int r = 0; r < 2; ++r) {
        l_run[r] += __shfl_xor_sync(0xffffffffu, l_run[r], 1);
        l_run[r] += __shfl_xor_sync(0xffffffffu, l_run[r], 2);
    }
    const float inv0 = l_run[0] > 0.0f ? 1.0f / l_run[0] : 0.0f;
    const float inv1 = l_run[1] > 0.0f ? 1.0f / l_run[1] : 0.0f;
    if (p.o32 != nullptr) {
#pragma unroll
        for (int nt = 0; nt < 8; ++nt) {
            const int col = h * HD + nt * 8 + (lane & 3) * 2;
            if (qi0 < n)
                *reinterpret_cast<float2 *>(p.o32 + (row0 + qi0) * p.ldo32 + col) = make_float2(o[nt][0] * inv0, o[nt][1] * inv0);
            if (qi1 < n)
                *reinterpret_cast<float2 *>(p.o32 + (row0 + qi1) * p.ldo32 + col) = make_float2(o[nt][2] * inv1, o[nt][3] * inv1);
        }
        return;
    }
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
        const int col = h * HD + nt * 8 + (lane & 3) * 2;
        if (qi0 < n)
            *reinterpret_cast<uint32_t *>(p.o + (row0 + qi0) * p.ldo + col) = pack16<F16>(o[nt][0] * inv0, o[nt][1] * inv0);
        if (qi1 < n)
            *reinterpret_cast<uint32_t *>(p.o + (row0 + qi1) * p.ldo + col) = pack16<F16>(o[nt][2] * inv1, o[nt][3] * inv1);
    }
}

}  // namespace

Status launch_attention(const AttentionCall &c, cudaStream_t stream) {
    if (c.groups <= 0 || c.heads <= 0 || c.n <= 0) return Status::fail(TSFM_ERR_INVALID_ARGUMENT, "attention: empty");
    // The tcgen05 kernel takes every call it supports, except the causal / decoder masks of short
    // sequences (n <= 256: at Timestral's 160 tokens the mma.sync kernel is ≈ 20 % faster, the
    // tcgen05 kernel's per-item cost dominating; at 577 tokens the tcgen05 kernel is 1.8x faster).
    const bool tc_pref = c.mask_mode == 0 || c.n > 256 || c.o8 != nullptr;
    if (c.force_path == 1 || c.force_path == 3 || (c.force_path == 0 && tc_pref && attention_tc_supported(c)))
        return launch_attention_tc(c, stream);
    if (c.o32 && (c.ld_o32 % 2 || (reinterpret_cast<uintptr_t>(c.o32) & 7)))
        return Status::fail(TSFM_ERR_INVALID_ARGUMENT, "attention: FP32 output needs 8-byte alignment");
    if (c.o8) return Status::fail(TSFM_ERR_UNSUPPORTED, "attention: FP8 companion output on the tcgen05 path only");
    if ((c.ld_qkv % 8) || (c.ld_o % 2) || (reinterpret_cast<uintptr_t>(c.q) & 15) ||
        (reinterpret_cast<uintptr_t>(c.k) & 15) || (reinterpret_cast<uintptr_t>(c.v) & 15))
        return Status::fail(TSFM_ERR_INVALID_ARGUMENT, "attention: q/k/v must be 16-byte aligned with ld % 8 == 0");
    if (c.groups > 65535 || c.heads > 65535)
        return Status::fail(TSFM_ERR_INVALID_ARGUMENT, "attention: too many groups for one launch");
    AttnP p;
    p.q = static_cast<const uint16_t *>(c.q);
    p.k = static_cast<const uint16_t *>(c.k);
    p.v = static_cast<const uint16_t *>(c.v);
    p.ld = c.ld_qkv;
    p.o = static_cast<uint16_t *>(c.o);
    p.ldo = c.ld_o;
    p.o32 = c.o32;
    p.ldo32 = c.ld_o32;
    p.key_valid = c.key_valid;
    p.kvs = c.kv_stride > 0 ? c.kv_stride : c.n;
    p.rel = c.rel_bias;
    p.rel_stride = c.rel_stride > 0 ? c.rel_stride : 2 * (int64_t)c.n - 1;
    p.rel_center = c.rel_center >= 0 ? c.rel_center : (int64_t)c.n - 1;
    p.n = c.n;
    p.heads = c.heads;
    p.scale_log2 = c.scale * kLog2e;
    p.ne = c.mask_mode == 0 ? c.n : c.ne;
    p.l = c.l;
    p.bidir = c.group_bidir;
    p.bidir_all = c.mask_mode == 2;
    const bool f16 = c.dtype == E_F16;
    if (c.dtype != E_F16 && c.dtype != E_BF16) return Status::fail(TSFM_ERR_UNSUPPORTED_DTYPE, "attention: dtype");
    dim3 grid((c.n + BQ - 1) / BQ, c.heads, c.groups);
    if (c.mask_mode == 0)
        f16 ? attn_kernel<0, true><<<grid, 128, 0, stream>>>(p) : attn_kernel<0, false><<<grid, 128, 0, stream>>>(p);
    else
        f16 ? attn_kernel<1, true><<<grid, 128, 0, stream>>>(p) : attn_kernel<1, false><<<grid, 128, 0, stream>>>(p);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return Status::cuda(e, "attention: launch");
    return Status::ok();
}

}  // namespace tsfm
