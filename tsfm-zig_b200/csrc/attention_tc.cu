// Flash attention on the 5th-generation tensor cores (sm_100a) for 64-wide heads.
//
// Persistent: one CTA per SM walks a contiguous range of work items; an item is one
// (group, head) and two 128-query tiles A and B that share every K / V tile.
// Roles (352 threads):
//   warps 0-3   softmax of tile A (thread = query row; warp w reads TMEM lanes 32 (w % 4) ...)
//   warps 4-7   softmax of tile B
//   warp 8      lane 0: TMA of the Q tiles and the K ring; lane 1: TMA of the V ring
//   warp 9      TMEM allocation and the single MMA-issuing thread
//   warp 10     key mask of the next item: per-key additive biases (0 / -inf) in shared memory
// Per key tile j the MMA thread issues S_A = Q_A K_j^T and S_B = Q_B K_j^T (M 128, N 128, K 64,
// accumulators in TMEM), then O_A += P_A(j-1) V_(j-1) and O_B += P_B(j-1) V_(j-1) (M 128, N 64,
// K 128; P from shared memory, V as an MN-major operand straight from its TMA tile). While the
// tensor cores work, the softmax warps read S with tcgen05.ld, add the key biases (tiles with
// a masked key only), update the running max with the lazy rescale (O and the row sum are
// rescaled only when the max grows by more than 2^8, so P stays below 256), write P as 16-bit
// values into the 128-byte-swizzled K-major layout the MMA reads, and arrive on p_ready. The K
// and V rings and all barrier phases run on across items, so the next item's Q, K and mask
// loads overlap the current item's last tiles and its output stores.
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
constexpr int kMaxKeys = 4096;
constexpr int kThreadsTc = 352;
constexpr int kSoftmaxThreads = 256;
constexpr float kRescaleThreshold = 8.0f;  // log2 units

// Shared memory map (offsets from the 1024-aligned base).
constexpr int OFF_Q = 0;                          // 2 tiles
constexpr int OFF_K = OFF_Q + 2 * kTileBytes;     // 2 stages
constexpr int OFF_V = OFF_K + 2 * kTileBytes;     // 2 stages
constexpr int OFF_P = OFF_V + 2 * kTileBytes;     // 2 tiles x 32 KB
constexpr int OFF_BIAS = OFF_P + 2 * kPBytes;     // 2 slots x kMaxKeys floats
constexpr int OFF_BIAS_INFO = OFF_BIAS + 2 * kMaxKeys * 4;  // per slot: uniform flag, full-tile bits
constexpr int OFF_BAR = OFF_BIAS_INFO + 64;
constexpr int kNumBars = 24;
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
    int n, heads, groups;
    int pairs;     // query-tile pairs per (group, head)
    int64_t items;
    float scale_log2;
    int *err;
};

struct BiasInfo {
    uint32_t uniform;
    uint32_t pad;
    uint64_t full;  // bit t: key tile t has no masked key
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

// The item range [first, last) of this CTA: contiguous, so consecutive items share a group
// (and its K / V rows in L2).
__device__ __forceinline__ void item_range(const TcParams &p, int64_t &first, int64_t &last) {
    first = p.items * blockIdx.x / gridDim.x;
    last = p.items * (blockIdx.x + 1) / gridDim.x;
}

struct Item {
    int g, h, q0;
    bool hasB;
};
__device__ __forceinline__ Item decode_item(const TcParams &p, int64_t it) {
    Item r;
    const int pair = (int)(it % p.pairs);
    const int64_t gh = it / p.pairs;
    r.h = (int)(gh % p.heads);
    r.g = (int)(gh / p.heads);
    r.q0 = pair * 2 * kTileRows;
    r.hasB = r.q0 + kTileRows < p.n;
    return r;
}

// Registers are allocated for warps in groups of four: the 11 warps take 12 warps' worth, so
// 168 per thread (12 x 32 x 168 = 64,512 of the SM's 65,536). One CTA per SM (the shared memory
// allows no second one either).
template <bool F16>
__global__ void __maxnreg__(168)
    attn_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                   const __grid_constant__ CUtensorMap tmV, TcParams p) {
    constexpr uint32_t FMT = F16 ? 0u : 1u;
    constexpr uint32_t IDESC_S = idesc_f32acc(FMT, 128, 128);
    constexpr uint32_t IDESC_PV = idesc_f32acc(FMT, 128, 64) | (1u << 16);  // B (V) is MN-major

    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    float *kbias = reinterpret_cast<float *>(smem + OFF_BIAS);
    BiasInfo *binfo = reinterpret_cast<BiasInfo *>(smem + OFF_BIAS_INFO);
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + OFF_BAR);
    uint64_t *q_full = bars + 0;
    uint64_t *q_empty = bars + 1;
    uint64_t *k_full = bars + 2;     // [2]
    uint64_t *k_empty = bars + 4;    // [2]
    uint64_t *v_full = bars + 6;     // [2]
    uint64_t *v_empty = bars + 8;    // [2]
    uint64_t *s_full = bars + 10;    // [2] per query tile
    uint64_t *s_free = bars + 12;    // [2]
    uint64_t *p_ready = bars + 14;   // [2]
    uint64_t *o_done = bars + 16;    // [2]
    uint64_t *bias_full = bars + 18;   // [2] per bias slot
    uint64_t *bias_empty = bars + 20;  // [2]
    uint64_t *drain = bars + 22;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + OFF_MISC);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(smem + OFF_MISC + 4);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n = p.n;
    const int T = (n + kTileRows - 1) / kTileRows;  // key tiles per item
    int64_t first, last;
    item_range(p, first, last);

    if (threadIdx.x == 0) {
        mbar_init(q_full, 1);
        mbar_init(q_empty, 1);
        for (int i = 0; i < 2; ++i) {
            mbar_init(&k_full[i], 1);
            mbar_init(&k_empty[i], 1);
            mbar_init(&v_full[i], 1);
            mbar_init(&v_empty[i], 1);
            mbar_init(&s_full[i], 1);
            mbar_init(&s_free[i], 128);
            mbar_init(&p_ready[i], 128);
            mbar_init(&o_done[i], 1);
            mbar_init(&bias_full[i], 32);
            mbar_init(&bias_empty[i], kSoftmaxThreads);
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
        if (lane == 0) {
            // ---- Q tiles and the K ring ----
            uint32_t kt = 0;  // K tiles issued so far
            uint32_t issued = 0, issued_ph = 0;
            bool ok = true, q_issued = false;
            uint32_t q_ph = 0;
            for (int64_t it = first; it < last && ok; ++it) {
                const Item im = decode_item(p, it);
                const int32_t row0 = im.g * n, col = im.h * 64;
                const uint32_t wi = (uint32_t)(it - first);
                if (wi > 0 && !mbar_wait(q_empty, (wi - 1) & 1, abort_flag, p.err, ERR_SITE_ATTN_PRODUCER)) {
                    ok = false;
                    break;
                }
                mbar_arrive_expect_tx(q_full, (im.hasB ? 2 : 1) * kTileBytes);
                tma_load_2d(smem + OFF_Q, &tmQ, q_full, col, row0 + im.q0);
                if (im.hasB) tma_load_2d(smem + OFF_Q + kTileBytes, &tmQ, q_full, col, row0 + im.q0 + kTileRows);
                q_issued = true;
                q_ph = wi & 1;
                for (int j = 0; j < T; ++j, ++kt) {
                    const int st = kt & 1;
                    if (kt >= 2 && !mbar_wait(&k_empty[st], ((kt - 2) >> 1) & 1, abort_flag, p.err, ERR_SITE_ATTN_PRODUCER)) {
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx(&k_full[st], kTileBytes);
                    tma_load_2d(smem + OFF_K + st * kTileBytes, &tmK, &k_full[st], col, row0 + j * kTileRows);
                    issued |= 1u << st;
                    issued_ph = (issued_ph & ~(1u << st)) | (((kt >> 1) & 1u) << st);
                }
            }
            if (!ok) {
                // Let the loads in flight land before the CTA can exit (bounded grace period).
                const unsigned long long t0 = globaltimer_ns();
                if (q_issued)
                    while (!mbar_try_wait(q_full, q_ph) && globaltimer_ns() - t0 < 100000000ull) {
                    }
                for (int i = 0; i < 2; ++i) {
                    if (!((issued >> i) & 1u)) continue;
                    while (!mbar_try_wait(&k_full[i], (issued_ph >> i) & 1u) && globaltimer_ns() - t0 < 100000000ull) {
                    }
                }
            }
        } else if (lane == 1) {
            // ---- the V ring ----
            uint32_t vt = 0;
            uint32_t issued = 0, issued_ph = 0;
            bool ok = true;
            for (int64_t it = first; it < last && ok; ++it) {
                const Item im = decode_item(p, it);
                const int32_t row0 = im.g * n, col = im.h * 64;
                for (int j = 0; j < T; ++j, ++vt) {
                    const int st = vt & 1;
                    if (vt >= 2 && !mbar_wait(&v_empty[st], ((vt - 2) >> 1) & 1, abort_flag, p.err, ERR_SITE_ATTN_PRODUCER)) {
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx(&v_full[st], kTileBytes);
                    tma_load_2d(smem + OFF_V + st * kTileBytes, &tmV, &v_full[st], col, row0 + j * kTileRows);
                    issued |= 1u << st;
                    issued_ph = (issued_ph & ~(1u << st)) | (((vt >> 1) & 1u) << st);
                }
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
    } else if (warp == 10) {
        // ---- key biases of each item, one slot ahead ----
        for (int64_t it = first; it < last; ++it) {
            const uint32_t wi = (uint32_t)(it - first), slot = wi & 1;
            if (wi >= 2) {
                const bool got = mbar_wait(&bias_empty[slot], ((wi >> 1) - 1) & 1, abort_flag, p.err, ERR_SITE_ATTN_PRODUCER);
                if (!__all_sync(0xffffffffu, got)) break;
            }
            const Item im = decode_item(p, it);
            const uint8_t *kv = p.key_valid ? p.key_valid + (int64_t)im.g * p.kvs : nullptr;
            float *b = kbias + slot * kMaxKeys;
            uint64_t full = 0;
            bool any = false;
            for (int t = 0; t < T; ++t) {
                bool tile_ok = true;
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    const int key = t * kTileRows + q * 32 + lane;
                    const bool v = key < n && (kv == nullptr || key >= p.kvs || kv[key] != 0);
                    b[key] = v ? 0.0f : -INFINITY;
                    tile_ok = tile_ok && v;
                    any = any || v;
                }
                if (__all_sync(0xffffffffu, tile_ok)) full |= 1ull << t;
            }
            const bool uniform = !__any_sync(0xffffffffu, any);
            if (uniform) {
                // No valid key: every key below n gets bias 0 and score 0 (equal weights).
                for (int key = lane; key < T * kTileRows; key += 32) b[key] = key < n ? 0.0f : -INFINITY;
                full = 0;
            }
            if (lane == 0) {
                binfo[slot].uniform = uniform ? 1u : 0u;
                binfo[slot].full = full;
            }
            __syncwarp();
            mbar_arrive(&bias_full[slot]);
        }
    } else if (warp == 9) {
        // ---- MMA issuer ----
        if (lane == 0) {
            bool ok = true;
            uint32_t kt = 0, vt = 0;     // K / V ring positions
            uint32_t ns[2] = {0, 0};     // S tiles issued per query tile
            uint32_t np[2] = {0, 0};     // PV issued per query tile
            const uint64_t qd0 = sdesc_k128(smem + OFF_Q), qd1 = sdesc_k128(smem + OFF_Q + kTileBytes);
            // PV of one query tile for the V tile at ring position vt.
            auto pv_one = [&](int x, bool first_tile) -> bool {
                if (!mbar_wait(&p_ready[x], np[x] & 1, abort_flag, p.err, ERR_SITE_ATTN_MMA)) return false;
                tc_fence_after();
                const uint64_t vd = sdesc_k128(smem + OFF_V + (vt & 1) * kTileBytes);
                const uint64_t pd = sdesc_k128(smem + OFF_P + x * kPBytes);
#pragma unroll
                for (int kk = 0; kk < 8; ++kk) {
                    // A: 16 keys = 32 bytes inside a 64-key swizzle column; B: 16 key rows = 2048 bytes.
                    const uint64_t a = pd + (uint64_t)((kk >> 2) * (kTileBytes >> 4) + 2 * (kk & 3));
                    const uint64_t b = vd + (uint64_t)(kk * (2048 >> 4));
                    mma_f16kind(tmem_base + TM_O + 64 * x, a, b, IDESC_PV, (!first_tile || kk > 0) ? 1u : 0u);
                }
                mma_commit(&o_done[x]);
                ++np[x];
                return true;
            };
            // Issue order per key tile j: S_A(j), PV_A(j-1), S_B(j), PV_B(j-1). Each PV then waits
            // in the in-order tensor pipe behind at most its own tile's S, so o_done follows
            // p_ready closely, and the two query tiles settle into alternating phases.
            for (int64_t it = first; it < last && ok; ++it) {
                const Item im = decode_item(p, it);
                const int ntile = im.hasB ? 2 : 1;
                const uint32_t wi = (uint32_t)(it - first);
                if (!mbar_wait(q_full, wi & 1, abort_flag, p.err, ERR_SITE_ATTN_MMA)) {
                    ok = false;
                    break;
                }
                for (int j = 0; j < T && ok; ++j, ++kt) {
                    const int st = kt & 1;
                    if (!mbar_wait(&k_full[st], (kt >> 1) & 1, abort_flag, p.err, ERR_SITE_ATTN_MMA)) {
                        ok = false;
                        break;
                    }
                    if (j > 0 && !mbar_wait(&v_full[vt & 1], (vt >> 1) & 1, abort_flag, p.err, ERR_SITE_ATTN_MMA)) {
                        ok = false;
                        break;
                    }
                    const uint64_t kd = sdesc_k128(smem + OFF_K + st * kTileBytes);
                    for (int x = 0; x < ntile && ok; ++x) {
                        if (ns[x] > 0 && !mbar_wait(&s_free[x], (ns[x] - 1) & 1, abort_flag, p.err, ERR_SITE_ATTN_MMA)) {
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        const uint64_t qd = x ? qd1 : qd0;
#pragma unroll
                        for (int kk = 0; kk < 4; ++kk)
                            mma_f16kind(tmem_base + TM_S + 128 * x, qd + 2 * kk, kd + 2 * kk, IDESC_S, kk > 0 ? 1u : 0u);
                        mma_commit(&s_full[x]);
                        ++ns[x];
                        if (j > 0 && !pv_one(x, j == 1)) ok = false;
                    }
                    if (!ok) break;
                    mma_commit(&k_empty[st]);
                    if (j == T - 1) mma_commit(q_empty);  // the Q tiles are free once these S complete
                    if (j > 0) {
                        mma_commit(&v_empty[vt & 1]);
                        ++vt;
                    }
                }
                if (!ok) break;
                // The last key tile's PV.
                if (!mbar_wait(&v_full[vt & 1], (vt >> 1) & 1, abort_flag, p.err, ERR_SITE_ATTN_MMA)) {
                    ok = false;
                    break;
                }
                for (int x = 0; x < ntile && ok; ++x)
                    if (!pv_one(x, T == 1)) ok = false;
                if (!ok) break;
                mma_commit(&v_empty[vt & 1]);
                ++vt;
            }
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
        const uint32_t t_s = tmem_base + ((uint32_t)(quarter * 32) << 16) + TM_S + 128 * x;
        const uint32_t t_o = tmem_base + ((uint32_t)(quarter * 32) << 16) + TM_O + 64 * x;
        uint8_t *sp = smem + OFF_P + x * kPBytes;
        const float sl2 = p.scale_log2;
        uint32_t cx = 0;  // tiles processed by this query tile so far
        bool ok = true;
        for (int64_t it = first; it < last && ok; ++it) {
            const Item im = decode_item(p, it);
            const uint32_t wi = (uint32_t)(it - first), slot = wi & 1;
            {
                const bool got = mbar_wait(&bias_full[slot], (wi >> 1) & 1, abort_flag, p.err, ERR_SITE_ATTN_SOFTMAX);
                if (!__all_sync(0xffffffffu, got)) break;
            }
            if (x == 0 || im.hasB) {
                const float *bias = kbias + slot * kMaxKeys;
                const bool uniform = binfo[slot].uniform != 0;
                const uint64_t full = binfo[slot].full;
                float m_run = -INFINITY, l_run = 0.0f;
                for (int j = 0; j < T; ++j, ++cx) {
                    const bool got = mbar_wait(&s_full[x], cx & 1, abort_flag, p.err, ERR_SITE_ATTN_SOFTMAX);
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

                    // Key biases (0 / -inf), broadcast from shared memory; uniform groups replace
                    // the scores by the biases.
                    if (!((full >> j) & 1ull)) {
                        const float4 *b4 = reinterpret_cast<const float4 *>(bias + j * kTileRows);
                        if (uniform) {
#pragma unroll
                            for (int q = 0; q < 32; ++q) {
                                const float4 bb = b4[q];
                                s[4 * q] = bb.x;
                                s[4 * q + 1] = bb.y;
                                s[4 * q + 2] = bb.z;
                                s[4 * q + 3] = bb.w;
                            }
                        } else {
#pragma unroll
                            for (int q = 0; q < 32; ++q) {
                                const float4 bb = b4[q];
                                s[4 * q] += bb.x;
                                s[4 * q + 1] += bb.y;
                                s[4 * q + 2] += bb.z;
                                s[4 * q + 3] += bb.w;
                            }
                        }
                    }
                    // Four partial maxima / sums keep the dependency chains short.
                    float mxp[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
                    for (int i = 0; i < 128; ++i) mxp[i & 3] = fmaxf(mxp[i & 3], s[i]);
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

                    // P overwrites the previous tile's P, and O is rescaled below: both need the
                    // previous PV of this query tile complete.
                    if (cx > 0) {
                        const bool done = mbar_wait(&o_done[x], (cx - 1) & 1, abort_flag, p.err, ERR_SITE_ATTN_SOFTMAX);
                        if (!__all_sync(0xffffffffu, done)) {
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                    }
                    // P row r into the K-major, 128-byte-swizzled layout: 16-byte chunk c of the
                    // row (keys 8c .. 8c + 7) sits in swizzle column c / 8 at chunk (c % 8) ^ (r % 8).
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
                if (!ok) break;
                // Output rows of this query tile.
                const bool done = mbar_wait(&o_done[x], (cx - 1) & 1, abort_flag, p.err, ERR_SITE_ATTN_SOFTMAX);
                if (!__all_sync(0xffffffffu, done)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                float o0[32], o1[32];
                tmem_ld32(t_o, o0);
                tmem_ld32(t_o + 32, o1);
                tmem_wait_ld();
                const int tok = im.q0 + x * kTileRows + r;
                if (tok < n) {
                    const float inv = l_run > 0.0f ? 1.0f / l_run : 0.0f;
                    uint16_t *dst = static_cast<uint16_t *>(p.o) + (int64_t)(im.g * n + tok) * p.ldo + im.h * 64;
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
            // The bias slot is free once both query tiles are done with this item. The O tile is
            // in registers: the next item's first PV (accumulate = 0) may overwrite it once this
            // thread's next p_ready arrives.
            mbar_arrive(&bias_empty[slot]);
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
    p.groups = c.groups;
    p.pairs = (c.n + 2 * kTileRows - 1) / (2 * kTileRows);
    p.items = (int64_t)c.groups * c.heads * p.pairs;
    p.scale_log2 = c.scale * 1.4426950408889634f;
    p.err = c.err;
    const int64_t grid = std::min<int64_t>(p.items, num_sms());
    cudaError_t e;
    if (c.dtype == E_F16) {
        e = cudaFuncSetAttribute(attn_tc_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemTc);
        if (e == cudaSuccess) attn_tc_kernel<true><<<(unsigned)grid, kThreadsTc, kSmemTc, stream>>>(mq, mk, mv, p);
    } else {
        e = cudaFuncSetAttribute(attn_tc_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemTc);
        if (e == cudaSuccess) attn_tc_kernel<false><<<(unsigned)grid, kThreadsTc, kSmemTc, stream>>>(mq, mk, mv, p);
    }
    if (e != cudaSuccess) return Status::cuda(e, "attention (tcgen05): set shared memory");
    e = cudaGetLastError();
    if (e != cudaSuccess) return Status::cuda(e, "attention (tcgen05): launch");
    return Status::ok();
}

}  // namespace tsfm
