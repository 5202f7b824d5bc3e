// Flash attention on the 5th-generation tensor cores (sm_100a) for 64-wide heads.
//
// One CTA = one (group, head) and two 128-query tiles A and B that share every K / V tile.
// Roles (352 threads):
//   warps 0-3   softmax of tile A (thread = query row; warp w reads TMEM lanes 32 (w % 4) ...)
//   warps 4-7   softmax of tile B
//   warp 8      TMA: Q tiles, then the K tiles into a 2-stage ring
//   warp 9      TMEM allocation and the single MMA-issuing thread
//   warp 10     TMA: V tiles into a 2-stage ring
// Per key tile j the MMA thread issues S_A = Q_A K_j^T and S_B = Q_B K_j^T (M 128, N 128, K 64,
// accumulators in TMEM), then O_A += P_A(j-1) V_(j-1) and O_B += P_B(j-1) V_(j-1) (M 128, N 64,
// K 128; P from shared memory, V as an MN-major operand straight from its TMA tile). While the
// tensor cores work on one tile, the other tile's softmax warps read S with tcgen05.ld, apply the
// key mask, update the running max with the lazy rescale (O and the row sum are rescaled only
// when the max grows by more than 2^8, so P stays below 256), write P as 16-bit values into the
// 128-byte-swizzled K-major layout the MMA reads, and arrive on p_ready.
//
// Masks: the key-validity mask of chronos2/model.zig:208-233 and chronos_bolt/model.zig (mode 0:
// key j is visible when it is valid; a group without any valid key attends uniformly to all its
// keys, the reference's additive -floatMax mask). Every wait is bounded (ptx.cuh).
#include <algorithm>

#include "kernels.h"
#include "ptx.cuh"

#include <cuda_fp16.h>

namespace tsfm {

namespace {

constexpr int kTileRows = 128;                   // queries per tile, keys per tile
constexpr int kTileBytes = kTileRows * 64 * 2;   // 16 KB: 128 rows of 64 16-bit values (128 B)
constexpr int kPBytes = 2 * kTileBytes;          // 128 x 128 16-bit P: two 64-key swizzle columns
constexpr int kMaxKeys = 8192;
constexpr int kMaskWords = kMaxKeys / 32;
constexpr int kThreadsTc = 352;
constexpr int kSoftmaxThreads = 256;
constexpr float kRescaleThreshold = 8.0f;  // log2 units

// Shared memory map (offsets from the 1024-aligned base).
constexpr int OFF_Q = 0;                          // 2 tiles
constexpr int OFF_K = OFF_Q + 2 * kTileBytes;     // 2 stages
constexpr int OFF_V = OFF_K + 2 * kTileBytes;     // 2 stages
constexpr int OFF_P = OFF_V + 2 * kTileBytes;     // 2 tiles x 32 KB
constexpr int OFF_MASK = OFF_P + 2 * kPBytes;
constexpr int OFF_BAR = OFF_MASK + kMaskWords * 4;
constexpr int kNumBars = 20;
constexpr int OFF_MISC = OFF_BAR + kNumBars * 8;
constexpr int kSmemTc = OFF_MISC + 64 + 1024;     // + alignment slack

// TMEM columns: S_A, S_B (128 each), O_A, O_B (64 each).
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t TM_S = 0, TM_O = 256;

struct TcParams {
    const uint8_t *key_valid;
    int64_t kvs;
    void *o;
    int64_t ldo;
    int n, heads;
    float scale_log2;
    int *err;
};

template <bool F16>
__device__ __forceinline__ uint32_t pack_p(float a, float b) {
    if constexpr (F16) {
        __half2 h = __floats2half2_rn(a, b);
        return *reinterpret_cast<uint32_t *>(&h);
    } else {
        __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
        return *reinterpret_cast<uint32_t *>(&h);
    }
}

template <bool F16>
__global__ void __launch_bounds__(kThreadsTc, 1)
    attn_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                   const __grid_constant__ CUtensorMap tmV, TcParams p) {
    constexpr uint32_t FMT = F16 ? 0u : 1u;
    constexpr uint32_t IDESC_S = idesc_f32acc(FMT, 128, 128);
    constexpr uint32_t IDESC_PV = idesc_f32acc(FMT, 128, 64) | (1u << 16);  // B (V) is MN-major

    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint32_t *kmask = reinterpret_cast<uint32_t *>(smem + OFF_MASK);
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + OFF_BAR);
    uint64_t *q_full = bars + 0;
    uint64_t *k_full = bars + 1;   // [2]
    uint64_t *k_empty = bars + 3;  // [2]
    uint64_t *v_full = bars + 5;   // [2]
    uint64_t *v_empty = bars + 7;  // [2]
    uint64_t *s_full = bars + 9;   // [2] per tile
    uint64_t *s_free = bars + 11;  // [2]
    uint64_t *p_ready = bars + 13; // [2]
    uint64_t *o_done = bars + 15;  // [2]
    uint64_t *drain = bars + 17;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + OFF_MISC);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(smem + OFF_MISC + 4);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int h = blockIdx.y, g = blockIdx.z;
    const int n = p.n;
    const int q0 = blockIdx.x * 2 * kTileRows;
    const bool hasB = q0 + kTileRows < n;
    const int ntile = hasB ? 2 : 1;
    const int T = (n + kTileRows - 1) / kTileRows;  // key tiles
    const int32_t row0 = g * n;                     // first token row of this group
    const int32_t col = h * 64;

    if (threadIdx.x == 0) {
        mbar_init(q_full, 1);
        for (int i = 0; i < 2; ++i) {
            mbar_init(&k_full[i], 1);
            mbar_init(&k_empty[i], 1);
            mbar_init(&v_full[i], 1);
            mbar_init(&v_empty[i], 1);
            mbar_init(&s_full[i], 1);
            mbar_init(&s_free[i], 128);
            mbar_init(&p_ready[i], 128);
            mbar_init(&o_done[i], 1);
        }
        mbar_init(drain, 1);
        *abort_flag = 0;
        fence_barrier_init();
        tma_prefetch_desc(&tmQ);
        tma_prefetch_desc(&tmK);
        tma_prefetch_desc(&tmV);
    }
    if (warp == 9) {
        tmem_alloc(tmem_slot, kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 8) {
        // ---- Q and K producer ----
        if (lane == 0) {
            uint32_t issued = 0, issued_ph = 0;
            bool ok = true;
            mbar_arrive_expect_tx(q_full, ntile * kTileBytes);
            tma_load_2d(smem + OFF_Q, &tmQ, q_full, col, row0 + q0);
            if (hasB) tma_load_2d(smem + OFF_Q + kTileBytes, &tmQ, q_full, col, row0 + q0 + kTileRows);
            for (int j = 0; j < T && ok; ++j) {
                const int st = j & 1;
                if (j >= 2 && !mbar_wait(&k_empty[st], ((j - 2) >> 1) & 1, abort_flag, p.err, ERR_SITE_ATTN_PRODUCER)) {
                    ok = false;
                    break;
                }
                mbar_arrive_expect_tx(&k_full[st], kTileBytes);
                tma_load_2d(smem + OFF_K + st * kTileBytes, &tmK, &k_full[st], col, row0 + j * kTileRows);
                issued |= 1u << st;
                issued_ph = (issued_ph & ~(1u << st)) | ((uint32_t)((j >> 1) & 1) << st);
            }
            if (!ok) {
                // Let the loads in flight land before the CTA can exit (bounded grace period).
                const unsigned long long t0 = globaltimer_ns();
                while (!mbar_try_wait(q_full, 0) && globaltimer_ns() - t0 < 100000000ull) {
                }
                for (int i = 0; i < 2; ++i) {
                    if (!((issued >> i) & 1u)) continue;
                    while (!mbar_try_wait(&k_full[i], (issued_ph >> i) & 1u) && globaltimer_ns() - t0 < 100000000ull) {
                    }
                }
            }
        }
    } else if (warp == 10) {
        // ---- V producer ----
        if (lane == 0) {
            uint32_t issued = 0, issued_ph = 0;
            bool ok = true;
            for (int j = 0; j < T && ok; ++j) {
                const int st = j & 1;
                if (j >= 2 && !mbar_wait(&v_empty[st], ((j - 2) >> 1) & 1, abort_flag, p.err, ERR_SITE_ATTN_PRODUCER)) {
                    ok = false;
                    break;
                }
                mbar_arrive_expect_tx(&v_full[st], kTileBytes);
                tma_load_2d(smem + OFF_V + st * kTileBytes, &tmV, &v_full[st], col, row0 + j * kTileRows);
                issued |= 1u << st;
                issued_ph = (issued_ph & ~(1u << st)) | ((uint32_t)((j >> 1) & 1) << st);
            }
            if (!ok) {
                const unsigned long long t0 = globaltimer_ns();
                for (int i = 0; i < 2; ++i) {
                    if (!((issued >> i) & 1u)) continue;
                    while (!mbar_try_wait(&v_full[i], (issued_ph >> i) & 1u) && globaltimer_ns() - t0 < 100000000ull) {
                    }
                }
            }
        }
    } else if (warp == 9) {
        // ---- MMA issuer ----
        if (lane == 0) {
            bool ok = mbar_wait(q_full, 0, abort_flag, p.err, ERR_SITE_ATTN_MMA);
            const uint64_t qd0 = sdesc_k128(smem + OFF_Q), qd1 = sdesc_k128(smem + OFF_Q + kTileBytes);
            auto pv = [&](int i) -> bool {
                const int st = i & 1;
                if (!mbar_wait(&v_full[st], (i >> 1) & 1, abort_flag, p.err, ERR_SITE_ATTN_MMA)) return false;
                const uint64_t vd = sdesc_k128(smem + OFF_V + st * kTileBytes);
                for (int x = 0; x < ntile; ++x) {
                    if (!mbar_wait(&p_ready[x], i & 1, abort_flag, p.err, ERR_SITE_ATTN_MMA)) return false;
                    tc_fence_after();
                    const uint64_t pd = sdesc_k128(smem + OFF_P + x * kPBytes);
#pragma unroll
                    for (int kk = 0; kk < 8; ++kk) {
                        // A: 16 keys = 32 bytes inside a 64-key swizzle column; B: 16 key rows = 2048 bytes.
                        const uint64_t a = pd + (uint64_t)((kk >> 2) * (kTileBytes >> 4) + 2 * (kk & 3));
                        const uint64_t b = vd + (uint64_t)(kk * (2048 >> 4));
                        mma_f16kind(tmem_base + TM_O + 64 * x, a, b, IDESC_PV, (i > 0 || kk > 0) ? 1u : 0u);
                    }
                    mma_commit(&o_done[x]);
                }
                mma_commit(&v_empty[st]);
                return true;
            };
            for (int j = 0; j < T && ok; ++j) {
                const int st = j & 1;
                if (!mbar_wait(&k_full[st], (j >> 1) & 1, abort_flag, p.err, ERR_SITE_ATTN_MMA)) {
                    ok = false;
                    break;
                }
                const uint64_t kd = sdesc_k128(smem + OFF_K + st * kTileBytes);
                for (int x = 0; x < ntile && ok; ++x) {
                    if (j > 0 && !mbar_wait(&s_free[x], (j - 1) & 1, abort_flag, p.err, ERR_SITE_ATTN_MMA)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint64_t qd = x ? qd1 : qd0;
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk)
                        mma_f16kind(tmem_base + TM_S + 128 * x, qd + 2 * kk, kd + 2 * kk, IDESC_S, kk > 0 ? 1u : 0u);
                    mma_commit(&s_full[x]);
                }
                if (!ok) break;
                mma_commit(&k_empty[st]);
                if (j > 0 && !pv(j - 1)) ok = false;
            }
            if (ok) pv(T - 1);
            mma_commit(drain);
            const unsigned long long t0 = globaltimer_ns();
            while (!mbar_try_wait(drain, 0)) {
                if (globaltimer_ns() - t0 > kWaitTimeoutNs) {
                    if (p.err) atomicCAS(p.err, 0, ERR_SITE_ATTN_DRAIN);
                    break;
                }
            }
        }
    } else {
        // ---- softmax warps 0-7 ----
        const int x = warp >> 2;          // query tile
        const int quarter = warp & 3;     // TMEM lane quarter
        const int r = quarter * 32 + lane;
        const int sid = threadIdx.x;      // 0..255

        // Key mask words for the whole group (bits of keys >= n stay 0; keys at or past the mask
        // stride count as valid); a group with no valid key attends uniformly to its n keys.
        const int words = T * 4;
        const uint8_t *kv = p.key_valid ? p.key_valid + (int64_t)g * p.kvs : nullptr;
        bool any = false;
        for (int w = sid; w < words; w += kSoftmaxThreads) {
            uint32_t bits = 0;
            for (int b = 0; b < 32; ++b) {
                const int key = w * 32 + b;
                const bool v = key < n && (kv == nullptr || key >= p.kvs || kv[key] != 0);
                bits |= (uint32_t)v << b;
            }
            kmask[w] = bits;
            any = any || bits != 0;
        }
        // Uniform groups: every key below n gets score 0 (equal weights).
        const bool uniform = !named_bar_or(1, kSoftmaxThreads, any);
        const float sl2 = p.scale_log2;
        if (uniform) {
            for (int w = sid; w < words; w += kSoftmaxThreads) {
                const int rem = n - w * 32;
                kmask[w] = rem >= 32 ? 0xffffffffu : rem <= 0 ? 0u : ((1u << rem) - 1u);
            }
        }
        named_bar_sync(1, kSoftmaxThreads);

        if (x < ntile) {
            const uint32_t t_s = tmem_base + ((uint32_t)(quarter * 32) << 16) + TM_S + 128 * x;
            const uint32_t t_o = tmem_base + ((uint32_t)(quarter * 32) << 16) + TM_O + 64 * x;
            uint8_t *sp = smem + OFF_P + x * kPBytes;
            float m_run = -INFINITY, l_run = 0.0f;
            bool ok = true;
            for (int j = 0; j < T; ++j) {
                const bool got = mbar_wait(&s_full[x], j & 1, abort_flag, p.err, ERR_SITE_ATTN_SOFTMAX);
                if (!__all_sync(0xffffffffu, got)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                float s[128];
                {
                    float c0[32], c1[32], c2[32], c3[32];
                    tmem_ld32(t_s + 0, c0);
                    tmem_ld32(t_s + 32, c1);
                    tmem_ld32(t_s + 64, c2);
                    tmem_ld32(t_s + 96, c3);
                    tmem_wait_ld();
#pragma unroll
                    for (int i = 0; i < 32; ++i) {
                        s[i] = c0[i];
                        s[32 + i] = c1[i];
                        s[64 + i] = c2[i];
                        s[96 + i] = c3[i];
                    }
                }
                tc_fence_before();
                mbar_arrive(&s_free[x]);

                const uint32_t w0 = kmask[4 * j], w1 = kmask[4 * j + 1], w2 = kmask[4 * j + 2], w3 = kmask[4 * j + 3];
                // Four partial maxima / sums keep the dependency chains short.
                float mxp[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
                if (!uniform && (w0 & w1 & w2 & w3) == 0xffffffffu) {
#pragma unroll
                    for (int i = 0; i < 128; ++i) mxp[i & 3] = fmaxf(mxp[i & 3], s[i]);
                } else {
                    const uint32_t wd[4] = {w0, w1, w2, w3};
                    const float keep = uniform ? 0.0f : 1.0f;
#pragma unroll
                    for (int i = 0; i < 128; ++i) {
                        s[i] = ((wd[i >> 5] >> (i & 31)) & 1u) ? s[i] * keep : -INFINITY;
                        mxp[i & 3] = fmaxf(mxp[i & 3], s[i]);
                    }
                }
                const float mx = fmaxf(fmaxf(mxp[0], mxp[1]), fmaxf(mxp[2], mxp[3]));
                // Lazy rescale: keep the stale max unless the new one exceeds it by 2^8.
                const float m_new = fmaxf(m_run, mx);
                float alpha = 1.0f;
                bool rescale = false;
                if (m_new > m_run && (m_run == -INFINITY || (m_new - m_run) * sl2 > kRescaleThreshold)) {
                    alpha = m_run == -INFINITY ? 0.0f : ex2_approx((m_run - m_new) * sl2);
                    m_run = m_new;
                    rescale = true;
                }
                const float mb = m_run == -INFINITY ? 0.0f : m_run * sl2;

                // P(j) overwrites P(j-1), and O is rescaled below: both need PV(j-1) complete.
                if (j > 0) {
                    const bool done = mbar_wait(&o_done[x], (j - 1) & 1, abort_flag, p.err, ERR_SITE_ATTN_SOFTMAX);
                    if (!__all_sync(0xffffffffu, done)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                }
                // P row r into the K-major, 128-byte-swizzled layout: 16-byte chunk c of the row
                // (keys 8c .. 8c + 7) sits in swizzle column c / 8 at chunk (c % 8) ^ (r % 8).
                float sp4[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
                for (int c = 0; c < 16; ++c) {
                    uint32_t pk[4];
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const float a = ex2_approx(fmaf(s[8 * c + 2 * e], sl2, -mb));
                        const float b = ex2_approx(fmaf(s[8 * c + 2 * e + 1], sl2, -mb));
                        sp4[e] += a + b;
                        pk[e] = pack_p<F16>(a, b);
                    }
                    uint8_t *dst = sp + (c >> 3) * kTileBytes + r * 128 + ((((c & 7) ^ (r & 7))) << 4);
                    *reinterpret_cast<uint4 *>(dst) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
                }
                l_run = l_run * alpha + ((sp4[0] + sp4[1]) + (sp4[2] + sp4[3]));
                if (j > 0 && __any_sync(0xffffffffu, rescale)) {
#pragma unroll
                    for (int hcol = 0; hcol < 64; hcol += 32) {
                        float ov[32];
                        tmem_ld32(t_o + hcol, ov);
                        tmem_wait_ld();
#pragma unroll
                        for (int i = 0; i < 32; ++i) ov[i] *= alpha;
                        tmem_st32(t_o + hcol, ov);
                    }
                    tmem_wait_st();
                }
                fence_proxy_async_smem();
                tc_fence_before();
                mbar_arrive(&p_ready[x]);
            }
            if (ok) {
                const bool done = mbar_wait(&o_done[x], (T - 1) & 1, abort_flag, p.err, ERR_SITE_ATTN_SOFTMAX);
                if (__all_sync(0xffffffffu, done)) {
                    tc_fence_after();
                    float o0[32], o1[32];
                    tmem_ld32(t_o, o0);
                    tmem_ld32(t_o + 32, o1);
                    tmem_wait_ld();
                    const int tok = q0 + x * kTileRows + r;
                    if (tok < n) {
                        const float inv = l_run > 0.0f ? 1.0f / l_run : 0.0f;
                        uint16_t *dst = static_cast<uint16_t *>(p.o) + (int64_t)(row0 + tok) * p.ldo + col;
#pragma unroll
                        for (int c = 0; c < 4; ++c) {
                            const float *src = c < 2 ? o0 + 16 * c : o1 + 16 * (c - 2);
                            uint4 a, b;
                            a.x = pack_p<F16>(src[0] * inv, src[1] * inv);
                            a.y = pack_p<F16>(src[2] * inv, src[3] * inv);
                            a.z = pack_p<F16>(src[4] * inv, src[5] * inv);
                            a.w = pack_p<F16>(src[6] * inv, src[7] * inv);
                            b.x = pack_p<F16>(src[8] * inv, src[9] * inv);
                            b.y = pack_p<F16>(src[10] * inv, src[11] * inv);
                            b.z = pack_p<F16>(src[12] * inv, src[13] * inv);
                            b.w = pack_p<F16>(src[14] * inv, src[15] * inv);
                            reinterpret_cast<uint4 *>(dst)[2 * c] = a;
                            reinterpret_cast<uint4 *>(dst)[2 * c + 1] = b;
                        }
                    }
                }
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 9) {
        tc_fence_after();
        tmem_dealloc(tmem_base, kTmemCols);
    }
}

}  // namespace

bool attention_tc_supported(const AttentionCall &c) {
    if (c.force_path == 2) return false;
    if (c.mask_mode != 0 || c.rel_bias != nullptr) return false;
    if (c.dtype != E_F16 && c.dtype != E_BF16) return false;
    if (c.n <= 0 || c.n > kMaxKeys || c.heads <= 0 || c.groups <= 0) return false;
    if ((int64_t)c.groups * c.n > INT32_MAX - 2 * kTileRows) return false;
    // TMA: 16-byte aligned bases and row strides; 16-byte aligned output rows.
    const auto a16 = [](const void *q) { return (reinterpret_cast<uintptr_t>(q) & 15) == 0; };
    if (!a16(c.q) || !a16(c.k) || !a16(c.v) || !a16(c.o) || (c.ld_qkv % 8) || (c.ld_o % 8)) return false;
    if (c.groups > 65535 || c.heads > 65535) return false;
    return true;
}

Status launch_attention_tc(const AttentionCall &c, cudaStream_t stream) {
    if (!attention_tc_supported(c)) return Status::fail(TSFM_ERR_UNSUPPORTED, "attention: the tcgen05 path does not take this call");
    const int64_t rows = (int64_t)c.groups * c.n;
    const int64_t width = (int64_t)c.heads * 64;
    alignas(64) CUtensorMap mq, mk, mv;
    TSFM_TRY(make_tmap_2d(&mq, c.q, c.dtype, width, rows, c.ld_qkv, 64, kTileRows));
    TSFM_TRY(make_tmap_2d(&mk, c.k, c.dtype, width, rows, c.ld_qkv, 64, kTileRows));
    TSFM_TRY(make_tmap_2d(&mv, c.v, c.dtype, width, rows, c.ld_qkv, 64, kTileRows));
    TcParams p;
    p.key_valid = c.key_valid;
    p.kvs = c.kv_stride > 0 ? c.kv_stride : c.n;
    p.o = c.o;
    p.ldo = c.ld_o;
    p.n = c.n;
    p.heads = c.heads;
    p.scale_log2 = c.scale * 1.4426950408889634f;
    p.err = c.err;
    const dim3 grid((unsigned)((c.n + 2 * kTileRows - 1) / (2 * kTileRows)), (unsigned)c.heads, (unsigned)c.groups);
    cudaError_t e;
    if (c.dtype == E_F16) {
        e = cudaFuncSetAttribute(attn_tc_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemTc);
        if (e == cudaSuccess) attn_tc_kernel<true><<<grid, kThreadsTc, kSmemTc, stream>>>(mq, mk, mv, p);
    } else {
        e = cudaFuncSetAttribute(attn_tc_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemTc);
        if (e == cudaSuccess) attn_tc_kernel<false><<<grid, kThreadsTc, kSmemTc, stream>>>(mq, mk, mv, p);
    }
    if (e != cudaSuccess) return Status::cuda(e, "attention (tcgen05): set shared memory");
    e = cudaGetLastError();
    if (e != cudaSuccess) return Status::cuda(e, "attention (tcgen05): launch");
    return Status::ok();
}

}  // namespace tsfm
