// Flash attention on the 5th-generation tensor cores (sm_100a) for 64-wide heads.
//
// Persistent: one CTA per SM walks a contiguous range of work items; an item is one
// (group, head, 128-query tile). The CTA runs two independent pipelines; pipeline p takes every
// other item of the range, so the softmax of one pipeline overlaps the other's loads, MMAs and
// bookkeeping and the SFU (exp2) stays busy.
// Roles (352 threads; the split-row instance doubles the softmax warps to 16, 608 threads):
//   warps 0-3, 4-7   softmax of pipeline 0 / 1 (thread = query row; warp w reads TMEM lanes
//                    32 (w % 4) .. + 31)
//   warps 8, 9       lane 0: the tensor-core thread of pipeline 0 / 1. It issues the MMAs and
//                    also every TMA transfer of its pipeline (Q, K and V loads, the output
//                    store), each at the point of its own loop where the buffer has just been
//                    released, so the loads run one or two key tiles ahead without a producer
//                    that could fall behind (V(j) right after S(j), K(j + 2) once S(j) is done).
//                    Warp 8 also allocates TMEM.
//   warp 10          key masks of the coming items (bit words per key tile, tile classes)
// Per key tile j a pipeline issues S = Q K_j^T (M 128, N 128, K 64, FP32 in TMEM), then
// O += P_(j-1) V_(j-1) (M 128, N 64, K 128) with P read from TMEM (16-bit, written by the
// softmax threads with tcgen05.st) and V as an MN-major operand straight from its TMA tile. The
// first S of an item follows the last S of the previous one directly (before that item's last
// PV), so the softmax finds it computed.
// The softmax threads read S with tcgen05.ld, mask it (tile classes: all keys valid, valid
// prefix, per-key bits), update the running max with the lazy rescale (O and the row sum are
// rescaled only when the max grows by more than 2^8, so P stays below 256) and write P.
// Output: Q is double-buffered per pipeline. An item's O is read from TMEM during the next item's
// first tile (before that tile's P is handed over, which lets the next PV overwrite O),
// normalised and written into the item's own Q buffer (free once its MMAs are done) in the
// 128-byte-swizzled layout; the tensor-core thread stores it with one TMA store, which clips the
// rows past n, and then loads the Q of the item after next into the buffer.
//
// Masks: the key-validity mask of chronos2/model.zig:208-233 and chronos_bolt/model.zig (mode 0:
// key j is visible when it is valid; a group without any valid key attends uniformly to all its
// keys, the reference's additive -floatMax mask), and Timestral's time-attention masks
// (timestral/model.zig:558-635, modes 1-2): encoder queries i < ne see the valid keys j <= i (any
// valid j < ne in a bidirectional group) and always j == i; decoder queries i >= ne see the valid
// keys below l and their chain ne <= j <= i. An item then reads only the key tiles up to the last
// key one of its rows can see, and tiles where the rows differ are masked per row from the
// validity bits (TILE_ROWS). The output is 16-bit (TMA store) or FP32 (written by the softmax
// threads, for corrected products). Relative-position bias (Chronos-Bolt's T5
// encoder, chronos_bolt/model.zig:195-205: score(i, j) += bias_h(j - i)) for n <= 512: the mask warp
// copies the item's window of the per-head offset table into its mask slot, and each softmax thread
// adds the 128 entries of its row to S before the row maximum. Every wait is bounded (ptx.cuh).
#include <algorithm>

#include "kernels.h"
#include "ptx.cuh"
#include "x8.cuh"

#include <cuda_fp16.h>

namespace tsfm {

namespace {

constexpr int kTileRows = 128;                   // queries per tile, keys per tile
constexpr int kTileBytes = kTileRows * 64 * 2;   // 16 KB: 128 rows of 64 16-bit values (128 B)
constexpr int kMaxKeys = 4096;
constexpr int kMaxKeyTiles = kMaxKeys / kTileRows;
constexpr int kMaxKeysRel = 512;                     // longest sequence with relative-position bias
constexpr int kRelWin = kMaxKeysRel + kTileRows;     // offsets one item's 128 query rows can see
constexpr int kThreadsTc = 352;
constexpr float kRescaleThreshold = 8.0f;  // log2 units
constexpr int kTailMax = 1;                // longest key tail folded into the softmax (mode 0; one key:
                                           // Chronos-Bolt's 129 tokens; longer tails spilled more)

// Tile classes of a key tile. TILE_ROWS (Timestral's causal / decoder masks): the visible keys
// depend on the query row; each softmax thread builds its row's bits from the validity bits.
enum : uint8_t { TILE_FULL = 0, TILE_PREFIX = 1, TILE_BITS = 2, TILE_ROWS = 3 };

// Mask of one item: per key tile its class and, for TILE_BITS, 128 validity bits; `uniform`:
// no valid key (every key below n gets score 0).
// `rel`: relative-position bias of the item's head, rel[i] = bias(i - 127 - q0) for
// i < T * 128 + 127 (0 outside the table), so query row r of the tile at key c of key tile j reads
// rel[128 j + c - r + 127].
// `ntiles`: key tiles the item reads (all of them in mode 0; up to the last visible key in modes
// 1-2); `bidir`: the item's group is bidirectional (mode 1-2).
struct MaskSlot {
    uint32_t bits[kMaxKeys / 32];
    uint8_t cls[kMaxKeyTiles];
    uint32_t uniform;
    int32_t ntiles;
    int32_t bidir;
    uint32_t pad[5];
    float rel[kRelWin];
};

// Shared memory map (offsets from the 1024-aligned base), per pipeline p.
constexpr int PIPE_BYTES = 6 * kTileBytes;       // Q[2] (then the item's output), K[2], V[2]
constexpr int OFF_Q = 0;
constexpr int OFF_K = 2 * kTileBytes;
constexpr int OFF_V = 4 * kTileBytes;
constexpr int OFF_MASK = 2 * PIPE_BYTES;         // [pipeline][slot]
constexpr int OFF_BAR = OFF_MASK + 4 * (int)sizeof(MaskSlot);
constexpr int kBarsPerPipe = 18;
constexpr int OFF_LSUM = OFF_BAR + (2 * kBarsPerPipe + 2) * 8;  // [pipeline][row] row sums
constexpr int OFF_MISC = OFF_LSUM + 2 * kTileRows * 4;
// Split rows (SPLIT instances): the two threads of a row exchange partial row maxima and sums through
// double-buffered slots [slot][pipeline][quarter][half][lane], one mbarrier per (pipeline, quarter).
constexpr int OFF_XBAR = OFF_MISC + 64;
constexpr int OFF_XBUF = OFF_XBAR + 8 * 8;
constexpr int kSmemTc = OFF_XBUF + 2 * 2 * 4 * 2 * 32 * 4 + 1024;  // + alignment slack
constexpr int kThreadsSplit = (16 + 3) * 32;

// TMEM columns of pipeline p (base p * 256): S (128 FP32), P (64 columns = 128 16-bit), O (64).
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t TM_S = 0, TM_P = 128, TM_O = 192;

struct TcParams {
    const uint8_t *key_valid;
    int64_t kvs;
    const float *rel;  // per head, indexed by key - query + rel_center; or null
    int64_t rel_stride, rel_center;
    int n, heads, groups;
    int qtiles;    // query tiles per (group, head)
    int64_t items;
    float scale_log2;
    int *err;
    // FP8 companion of the FP16 output (corrected products): row (g * n + i) at o8 + row * ld_o8,
    // head h's 64 values at byte h * 64, their low parts o8_half bytes further. o8_v8: o8 and
    // ld_o8 are 32-byte aligned, so each row's 32-byte runs leave in one 256-bit store.
    uint8_t *o8;
    int64_t ld_o8, o8_half;
    int o8_v8;
    // Masks of modes 1-2 (AttentionCall): encoder queries i < ne, decoder queries i >= ne reading
    // valid keys below l and their chain [ne, i]; per-group bidirectional flags.
    int mode, ne, l, bidir_all;
    const uint8_t *bidir;
    // FP32 output instead of the 16-bit one (row (g * n + i) at o32 + row * ld_o32, head h at h * 64).
    float *o32;
    int64_t ld_o32;
    // Key tail (mode 0, n = 128 (T - 1) + tail with 1 <= tail <= kTailMax, i.e. Chronos-Bolt's 129
    // tokens): the tensor cores cover the first T - 1 key tiles and the softmax threads the last
    // `tail` keys (scores from the Q tile in shared memory and the key rows, their P V added to the
    // output row when it is staged), so an item costs one key tile instead of two. tiles0: key
    // tiles of a mode-0 item; k / v (16-bit, row stride ld): the tail keys' rows.
    int tail, tiles0;
    const uint16_t *kraw, *vraw;
    int64_t ldraw;
};

// Key tiles an item reads: every tile in mode 0; in modes 1-2 the tiles up to the last key any of
// its rows can see (the causal bound, or the encoder for a bidirectional group), as the mma.sync
// kernel bounds its key loop.
__device__ __forceinline__ bool item_bidir(const TcParams &p, int g) {
    return p.mode != 0 && (p.bidir_all || (p.bidir != nullptr && p.bidir[g] != 0));
}
__device__ __forceinline__ int item_tiles(const TcParams &p, int g, int q0) {
    if (p.mode == 0) return p.tiles0;
    const int qhi = min(p.n, q0 + kTileRows);
    const int kv_end = item_bidir(p, g) ? max(p.ne, qhi) : qhi;
    return (kv_end + kTileRows - 1) / kTileRows;
}

// Lanes [0, x) of a 32-bit word (x clamped to [0, 32]).
__device__ __forceinline__ uint32_t low_bits(int x) {
    return x <= 0 ? 0u : x >= 32 ? 0xffffffffu : ((1u << x) - 1u);
}

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
__device__ __forceinline__ float2 unpack2(uint32_t u) {
    if constexpr (F16)
        return __half22float2(*reinterpret_cast<const __half2 *>(&u));
    else
        return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&u));
}

struct Item {
    int g, h, q0;
};
// Items fit in 31 bits (checked on the host), so the decode uses 32-bit division.
__device__ __forceinline__ Item decode_item(const TcParams &p, int64_t it64) {
    Item r;
    const uint32_t it = (uint32_t)it64, qtiles = (uint32_t)p.qtiles, heads = (uint32_t)p.heads;
    const uint32_t gh = it / qtiles;
    r.q0 = (int)(it - gh * qtiles) * kTileRows;
    r.g = (int)(gh / heads);
    r.h = (int)(gh - (uint32_t)r.g * heads);
    return r;
}

// Barriers of one pipeline.
struct PipeBars {
    uint64_t q_full[2], k_full[2], k_empty[2], v_full[2], v_empty[2];
    uint64_t s_full, s_free, p_ready, o_done, m_full[2], m_empty[2];
};
static_assert(sizeof(PipeBars) == kBarsPerPipe * 8, "barrier block");

// The item range [first, last) of this CTA (contiguous: neighbouring items share K / V rows in
// L2); pipeline p takes items first + p, first + p + 2, ...
__device__ __forceinline__ void item_range(const TcParams &p, int64_t &first, int64_t &last) {
    first = p.items * blockIdx.x / gridDim.x;
    last = p.items * (blockIdx.x + 1) / gridDim.x;
}

// The kernel body. O8: also writes the FP8 companion of the FP16 output (corrected products; a
// separate instance, so the plain kernel keeps its registers). TAIL: the key-tail instance
// (TcParams::tail > 0). SPLIT: two softmax threads per query row (16 softmax warps: warp w of a
// pipeline reads TMEM lanes 32 (w % 4) and keys 64 (w / 4) .. + 63 of each tile; the pair
// exchanges its partial row maximum every tile and its partial row sum every item), so twice the
// warps share the exponentials and every chain is half as long.
template <bool F16, bool O8, bool TAIL, bool SPLIT>
__device__ __forceinline__ void attn_tc_body(const CUtensorMap &tmQ, const CUtensorMap &tmK, const CUtensorMap &tmV,
                                             const CUtensorMap &tmO, const TcParams &p) {
    static_assert(!(TAIL && SPLIT), "the key tail runs on whole rows");
    constexpr int NSW = SPLIT ? 16 : 8;       // softmax warps (warps 0 .. NSW - 1)
    constexpr int W_MMA = NSW;                // warps NSW, NSW + 1: tensor-core threads of pipelines 0, 1
    constexpr int W_MASK = NSW + 2;           // the mask warp
    constexpr int PIPE_W = NSW / 2;           // softmax warps per pipeline
    constexpr uint32_t SM_ARRIVALS = PIPE_W * 32;
    constexpr uint32_t FMT = F16 ? 0u : 1u;
    constexpr uint32_t IDESC_S = idesc_f32acc(FMT, 128, 128);
    constexpr uint32_t IDESC_PV = idesc_f32acc(FMT, 128, 64) | (1u << 16);  // B (V) is MN-major

    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    MaskSlot *mslots = reinterpret_cast<MaskSlot *>(smem + OFF_MASK);  // [pipe * 2 + slot]
    PipeBars *pb = reinterpret_cast<PipeBars *>(smem + OFF_BAR);       // [2]
    uint64_t *drain = reinterpret_cast<uint64_t *>(smem + OFF_BAR + 2 * kBarsPerPipe * 8);  // [2]
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + OFF_MISC);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(smem + OFF_MISC + 4);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n = p.n;
    const int T = (n + kTileRows - 1) / kTileRows;  // key tiles per item
    int64_t first, last;
    item_range(p, first, last);

    if (threadIdx.x == 0) {
        for (int q = 0; q < 2; ++q) {
            PipeBars &b = pb[q];
            for (int i = 0; i < 2; ++i) {
                mbar_init(&b.q_full[i], 1);
                mbar_init(&b.k_full[i], 1);
                mbar_init(&b.k_empty[i], 1);
                mbar_init(&b.v_full[i], 1);
                mbar_init(&b.v_empty[i], 1);
                mbar_init(&b.m_full[i], 32);
                mbar_init(&b.m_empty[i], SM_ARRIVALS);
            }
            mbar_init(&b.s_full, 1);
            mbar_init(&b.s_free, SM_ARRIVALS);
            mbar_init(&b.p_ready, SM_ARRIVALS);
            mbar_init(&b.o_done, 1);
            mbar_init(&drain[q], 1);
        }
        if constexpr (SPLIT) {
            uint64_t *xbar = reinterpret_cast<uint64_t *>(smem + OFF_XBAR);
            for (int i = 0; i < 8; ++i) mbar_init(&xbar[i], 64);
        }
        *abort_flag = 0;
        fence_barrier_init();
        tma_prefetch_desc(&tmQ);
        tma_prefetch_desc(&tmK);
        tma_prefetch_desc(&tmV);
        tma_prefetch_desc(&tmO);
    }
    if (warp == W_MMA) {
        tmem_alloc(tmem_slot, kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == W_MASK) {
        // ---- key masks of the coming items, in item order ----
        uint32_t wi[2] = {0, 0};
        for (int64_t it = first; it < last; ++it) {
            const int q = (int)((it - first) & 1);
            PipeBars &b = pb[q];
            const uint32_t i = wi[q]++, slot = i & 1;
            if (i >= 2) {
                const bool got = mbar_wait(&b.m_empty[slot], ((i >> 1) - 1) & 1, abort_flag, p.err, ERR_SITE_ATTN_PRODUCER);
                if (!__all_sync(0xffffffffu, got)) break;
            }
            const Item im = decode_item(p, it);
            const uint8_t *kv = p.key_valid ? p.key_valid + (int64_t)im.g * p.kvs : nullptr;
            MaskSlot &m = mslots[q * 2 + slot];
            bool any = false;
            const int Ti = item_tiles(p, im.g, im.q0);
            const bool bid = item_bidir(p, im.g);
            // Modes 1-2: rows [i0, i1] of the item; a tile whose keys all lie below every row (or,
            // for a bidirectional group, hold no diagonal key) shows each row exactly the valid keys.
            const int i0 = im.q0, i1 = min(n, im.q0 + kTileRows) - 1;
            const int Tb = p.mode == 0 ? T : Ti;  // mode 0: the tail tile's bits too
            for (int t = 0; t < Tb; ++t) {
                bool all_valid = true, prefix = true;
#pragma unroll
                for (int w = 0; w < 4; ++w) {
                    const int key = t * kTileRows + w * 32 + lane;
                    const bool inside = key < n;
                    const bool v = inside && (kv == nullptr || key >= p.kvs || kv[key] != 0);
                    const uint32_t bits = __ballot_sync(0xffffffffu, v);
                    if (lane == 0) m.bits[t * 4 + w] = bits;
                    all_valid = all_valid && v;
                    prefix = prefix && (v == inside);
                    any = any || v;
                }
                all_valid = __all_sync(0xffffffffu, all_valid);
                prefix = __all_sync(0xffffffffu, prefix);
                bool per_row = false;
                if (p.mode != 0) {
                    const int k0 = t * kTileRows, k1 = min(n, k0 + kTileRows) - 1;
                    const bool below = i1 < p.ne && k1 < i0;
                    const bool bidir_clear = bid && i1 < p.ne && k1 < p.ne && (k1 < i0 || k0 > i1);
                    per_row = !(below || bidir_clear);
                }
                if (lane == 0) m.cls[t] = per_row ? TILE_ROWS : all_valid ? TILE_FULL : prefix ? TILE_PREFIX : TILE_BITS;
            }
            // Modes 1-2 never leave a row without a visible key (the diagonal, or the decoder
            // chain's own position), so no group attends uniformly.
            const bool uniform = p.mode == 0 && !__any_sync(0xffffffffu, any);
            if (lane == 0) {
                m.uniform = uniform ? 1u : 0u;
                m.ntiles = Ti;
                m.bidir = bid ? 1 : 0;
            }
            if (p.rel) {
                const float *tab = p.rel + (int64_t)im.h * p.rel_stride;
                const int64_t base = p.rel_center - im.q0 - (kTileRows - 1);
                for (int i = lane; i < T * kTileRows + kTileRows - 1; i += 32) {
                    const int64_t idx = base + i;
                    m.rel[i] = idx >= 0 && idx < p.rel_stride ? __ldg(tab + idx) : 0.0f;
                }
            }
            __syncwarp();
            mbar_arrive(&b.m_full[slot]);
        }
    } else if (warp == W_MMA || warp == W_MMA + 1) {
        // ---- tensor-core thread of pipeline warp - W_MMA: MMAs and TMA transfers ----
        if (lane == 0) {
            const int q = warp - W_MMA;
            PipeBars &b = pb[q];
            uint8_t *base = smem + q * PIPE_BYTES;
            const uint32_t t_s = tmem_base + q * 256 + TM_S, t_p = tmem_base + q * 256 + TM_P;
            const uint32_t t_o = tmem_base + q * 256 + TM_O;
            const uint32_t nq = last - first > q ? (uint32_t)((last - first - q + 1) / 2) : 0u;  // items
            auto item_of = [&](uint32_t wi) { return decode_item(p, first + q + 2 * (int64_t)wi); };
            auto tiles_of = [&](uint32_t wi) {
                const Item im = item_of(wi);
                return (uint32_t)item_tiles(p, im.g, im.q0);
            };
            // The pipeline's key tiles in order (item by item; items may read different numbers of
            // tiles in modes 1-2). A cursor walks them: item, tile within the item, and the item's
            // tile count.
            struct Cursor {
                uint32_t wi, j, n;
            };
            auto cursor_start = [&]() { return Cursor{0u, 0u, nq > 0 ? tiles_of(0) : 0u}; };
            auto advance = [&](Cursor &c) {
                if (++c.j == c.n) {
                    ++c.wi;
                    c.j = 0;
                    c.n = c.wi < nq ? tiles_of(c.wi) : 0u;
                }
            };
            uint32_t loads[3] = {0, 0, 0};  // Q, K, V loads issued (in ring order)
            auto load_q = [&](uint32_t wi) {
                ++loads[0];
                const Item im = item_of(wi);
                const uint32_t s = wi & 1;
                mbar_arrive_expect_tx(&b.q_full[s], kTileBytes);
                tma_load_2d(base + OFF_Q + s * kTileBytes, &tmQ, &b.q_full[s], im.h * 64, im.g * n + im.q0);
            };
            // Key tile g of this pipeline (the tile under the K or V cursor) into ring slot g % 2.
            Cursor kc = cursor_start(), vc = cursor_start(), pc = cursor_start();
            auto load_k = [&](uint32_t g) {
                ++loads[1];
                const Item im = item_of(kc.wi);
                const uint32_t s = g & 1;
                mbar_arrive_expect_tx(&b.k_full[s], kTileBytes);
                tma_load_2d(base + OFF_K + s * kTileBytes, &tmK, &b.k_full[s], im.h * 64,
                            im.g * n + (int32_t)kc.j * kTileRows);
                advance(kc);
            };
            auto load_v = [&](uint32_t g) {
                ++loads[2];
                const Item im = item_of(vc.wi);
                const uint32_t s = g & 1;
                mbar_arrive_expect_tx(&b.v_full[s], kTileBytes);
                tma_load_2d(base + OFF_V + s * kTileBytes, &tmV, &b.v_full[s], im.h * 64,
                            im.g * n + (int32_t)vc.j * kTileRows);
                advance(vc);
            };
            bool ok = true;
            // O += P V for key tile gg (the tile under the PV cursor). When gg opens an item, the
            // softmax threads have staged the previous item's output in its Q buffer before this
            // p_ready: store it (16-bit outputs; an FP32 output was written by the softmax threads),
            // then reuse the buffer for the Q two items ahead.
            auto pv = [&](uint32_t gg) -> bool {
                const uint32_t s = gg & 1;
                if (!mbar_wait(&b.v_full[s], (gg >> 1) & 1, abort_flag, p.err, ERR_SITE_ATTN_MMA)) return false;
                if (!mbar_wait(&b.p_ready, gg & 1, abort_flag, p.err, ERR_SITE_ATTN_MMA)) return false;
                tc_fence_after();
                const uint32_t wi = pc.wi, j = pc.j;
                advance(pc);
                const uint64_t vd = sdesc_k128(base + OFF_V + s * kTileBytes);
#pragma unroll
                for (int kk = 0; kk < 8; ++kk)  // A: 16 keys = 8 TMEM columns; B: 16 key rows = 2048 bytes
                    mma_f16kind_ts(t_o, t_p + 8 * kk, vd + (uint64_t)(kk * (2048 >> 4)), IDESC_PV,
                                   (j != 0 || kk > 0) ? 1u : 0u);
                mma_commit(&b.o_done);
                mma_commit(&b.v_empty[s]);
                if (j == 0 && wi >= 1) {
                    if (p.o32 == nullptr) {
                        const uint32_t ps = (wi - 1) & 1;
                        const Item im = item_of(wi - 1);
                        tma_store_3d(&tmO, base + OFF_Q + ps * kTileBytes, im.h * 64, im.q0, im.g);
                        bulk_commit();
                    }
                    if (wi + 1 < nq) {
                        bulk_wait_read_0();
                        load_q(wi + 1);
                    }
                }
                return true;
            };
            if (nq > 0) load_q(0);
            if (nq > 1) load_q(1);
            for (uint32_t g = 0; g < 2 && kc.wi < nq; ++g) {
                load_k(g);
                load_v(g);
            }
            uint32_t g = 0, next_pv = 0;
            for (uint32_t wi = 0; wi < nq && ok; ++wi) {
                const uint32_t qs = wi & 1;
                // When the pending PV opens the previous item (an item of one key tile), it stores
                // the output before it and loads this item's Q: issue it before waiting for that Q.
                if (next_pv < g && pc.j == 0 && !pv(next_pv++)) {
                    ok = false;
                    break;
                }
                if (!mbar_wait(&b.q_full[qs], (wi >> 1) & 1, abort_flag, p.err, ERR_SITE_ATTN_MMA)) {
                    ok = false;
                    break;
                }
                const uint64_t qd = sdesc_k128(base + OFF_Q + qs * kTileBytes);
                const uint32_t Ti = tiles_of(wi);
                for (uint32_t j = 0; j < Ti; ++j, ++g) {
                    const uint32_t s = g & 1;
                    if (!mbar_wait(&b.k_full[s], (g >> 1) & 1, abort_flag, p.err, ERR_SITE_ATTN_MMA) ||
                        (g > 0 && !mbar_wait(&b.s_free, (g - 1) & 1, abort_flag, p.err, ERR_SITE_ATTN_MMA))) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint64_t kd = sdesc_k128(base + OFF_K + s * kTileBytes);
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk)
                        mma_f16kind(t_s, qd + 2 * kk, kd + 2 * kk, IDESC_S, kk > 0 ? 1u : 0u);
                    mma_commit(&b.s_full);
                    mma_commit(&b.k_empty[s]);
                    // V of this tile into the slot PV(g - 2) read (long done by now), a period before
                    // PV(g) needs it; refilling here rather than after PV(g - 1) completes lets the
                    // next S follow the softmax's s_free without waiting for that PV.
                    if (g >= 2 && vc.wi < nq) {
                        if (!mbar_wait(&b.v_empty[s], ((g - 2) >> 1) & 1, abort_flag, p.err, ERR_SITE_ATTN_MMA)) {
                            ok = false;
                            break;
                        }
                        load_v(g);
                    }
                    if (next_pv < g && !pv(next_pv++)) {
                        ok = false;
                        break;
                    }
                    // K two tiles ahead once this S is done with its slot.
                    if (kc.wi < nq) {  // tile g + 2 exists
                        if (!mbar_wait(&b.k_empty[s], (g >> 1) & 1, abort_flag, p.err, ERR_SITE_ATTN_MMA)) {
                            ok = false;
                            break;
                        }
                        load_k(g + 2);
                    }
                }
            }
            while (ok && pc.wi < nq) ok = pv(next_pv++);
            // The last item's output: staged by the softmax threads after the last PV, signalled
            // by one more p_ready phase (g = the pipeline's key tiles).
            if (ok && g > 0 && mbar_wait(&b.p_ready, g & 1, abort_flag, p.err, ERR_SITE_ATTN_MMA) && p.o32 == nullptr) {
                const Item im = item_of(nq - 1);
                tma_store_3d(&tmO, base + OFF_Q + ((nq - 1) & 1) * kTileBytes, im.h * 64, im.q0, im.g);
                bulk_commit();
            }
            bulk_wait_all();
            if (!ok) {
                // Let the loads in flight land before the CTA can exit (bounded grace period):
                // the last load of every ring slot.
                const unsigned long long t0 = globaltimer_ns();
                for (int r = 0; r < 3; ++r) {
                    uint64_t *ful = r == 0 ? b.q_full : r == 1 ? b.k_full : b.v_full;
                    for (uint32_t back = 1; back <= 2 && back <= loads[r]; ++back) {
                        const uint32_t i = loads[r] - back;
                        while (!mbar_try_wait(&ful[i & 1], (i >> 1) & 1) && globaltimer_ns() - t0 < 100000000ull) {
                        }
                    }
                }
            }
            mma_commit(&drain[q]);
            const unsigned long long t0 = globaltimer_ns();
            while (!mbar_try_wait(&drain[q], 0)) {
                if (globaltimer_ns() - t0 > kWaitTimeoutNs) {
                    if (p.err) atomicCAS(p.err, 0, ERR_SITE_ATTN_DRAIN);
                    break;
                }
            }
        }
    } else if (warp < NSW) {
        // ---- softmax of pipeline warp / PIPE_W ----
        constexpr int SC = SPLIT ? 64 : 128;  // keys of a tile per thread
        constexpr int OC = SPLIT ? 32 : 64;   // output columns per thread
        const int q = warp / PIPE_W;
        const int wp = warp % PIPE_W;
        const int quarter = wp & 3;  // TMEM lane quarter
        const int half = SPLIT ? (wp >> 2) : 0;
        const int kofs = half * SC;  // this thread's first key of a tile
        const int r = quarter * 32 + lane;
        PipeBars &b = pb[q];
        const uint32_t lanes = (uint32_t)(quarter * 32) << 16;
        const uint32_t t_s = tmem_base + lanes + q * 256 + TM_S + kofs;
        const uint32_t t_p = tmem_base + lanes + q * 256 + TM_P + kofs / 2;
        const uint32_t t_o = tmem_base + lanes + q * 256 + TM_O + half * OC;
        const float sl2 = p.scale_log2;
        float *l_save = reinterpret_cast<float *>(smem + OFF_LSUM) + q * kTileRows + r;
        float prev_ltot = 0.0f;  // SPLIT: the previous item's full row sum
        // SPLIT: exchange a value with the row's other thread (bounded wait; false on abort).
        uint32_t xph = 0;
        float *xb = reinterpret_cast<float *>(smem + OFF_XBUF);
        uint64_t *xbar = reinterpret_cast<uint64_t *>(smem + OFF_XBAR) + q * 4 + quarter;
        auto xchg = [&](float v, float &other) -> bool {
            const int sl = (int)(xph & 1u);
            xb[(((sl * 2 + q) * 4 + quarter) * 2 + half) * 32 + lane] = v;
            mbar_arrive(xbar);
            const bool got = mbar_wait(xbar, xph & 1u, abort_flag, p.err, ERR_SITE_ATTN_SOFTMAX);
            other = xb[(((sl * 2 + q) * 4 + quarter) * 2 + (half ^ 1)) * 32 + lane];
            ++xph;
            return __all_sync(0xffffffffu, got);
        };
        uint32_t cx = 0, wi = 0;  // tiles / items processed by this pipeline
        bool ok = true;
        // This warp's rows of the previous item still wait in TMEM (not past n).
        bool prev_live = false;
        Item prev_im{0, 0, 0};
        float prev_pt[kTailMax];  // the previous item's tail probabilities (key tail)
#pragma unroll
        for (int t = 0; t < kTailMax; ++t) prev_pt[t] = 0.0f;
        // Reads this thread's row of the previous item's O, normalises it by the row sum and writes
        // it as 16-bit values into that item's Q buffer in the 128-byte-swizzled layout of a TMA
        // box (16-byte chunk c of row r at chunk c ^ (r % 8)).
        auto stage_prev_row = [&](uint32_t prev_slot) {
            const float l = SPLIT ? prev_ltot : *l_save;
            const float inv = l > 0.0f ? __frcp_rn(l) : 0.0f;
            uint8_t *row = smem + q * PIPE_BYTES + OFF_Q + prev_slot * kTileBytes + r * 128;
            // The FP8 companion goes straight to global memory (rows past n are not written).
            uint8_t *row8 = nullptr;
            if (O8 && prev_im.q0 + r < n)
                row8 = p.o8 + ((int64_t)prev_im.g * n + prev_im.q0 + r) * p.ld_o8;
            // An FP32 output goes straight to global memory as well (no TMA store follows).
            float *row32 = nullptr;
            if (p.o32 != nullptr && prev_im.q0 + r < n)
                row32 = p.o32 + ((int64_t)prev_im.g * n + prev_im.q0 + r) * p.ld_o32 + (int64_t)prev_im.h * 64 +
                        half * OC;
#pragma unroll
            for (int h = 0; h < OC / 32; ++h) {
                float v[32];
                tmem_ld32(t_o + 32 * h, v);
                tmem_wait_ld();
                if constexpr (TAIL) {
                    // O += P V over the key tail (rows of the previous item's group and head).
#pragma unroll
                    for (int t = 0; t < kTailMax; ++t) {
                        if (t >= p.tail) break;
                        const uint4 *vr = reinterpret_cast<const uint4 *>(
                            p.vraw + ((int64_t)prev_im.g * n + (int64_t)(p.tiles0 * kTileRows + t)) * p.ldraw +
                            prev_im.h * 64 + 32 * h);
                        const float pt = prev_pt[t];
#pragma unroll
                        for (int c = 0; c < 4; ++c) {
                            const uint4 u = __ldg(vr + c);
                            const float2 a = unpack2<F16>(u.x), b2 = unpack2<F16>(u.y), c2 = unpack2<F16>(u.z),
                                         d = unpack2<F16>(u.w);
                            v[8 * c + 0] = fmaf(pt, a.x, v[8 * c + 0]);
                            v[8 * c + 1] = fmaf(pt, a.y, v[8 * c + 1]);
                            v[8 * c + 2] = fmaf(pt, b2.x, v[8 * c + 2]);
                            v[8 * c + 3] = fmaf(pt, b2.y, v[8 * c + 3]);
                            v[8 * c + 4] = fmaf(pt, c2.x, v[8 * c + 4]);
                            v[8 * c + 5] = fmaf(pt, c2.y, v[8 * c + 5]);
                            v[8 * c + 6] = fmaf(pt, d.x, v[8 * c + 6]);
                            v[8 * c + 7] = fmaf(pt, d.y, v[8 * c + 7]);
                        }
                    }
                }
                if (O8) {
                    // The FP16 pairs serve the staged output and the companion's high parts.
                    float x[32];
                    uint32_t hp[16];
#pragma unroll
                    for (int i = 0; i < 32; ++i) x[i] = v[i] * inv;
#pragma unroll
                    for (int e = 0; e < 16; ++e) hp[e] = pack_p<true>(x[2 * e], x[2 * e + 1]);
                    if (row8 != nullptr) {
                        uint32_t hi[8], lo[8];
                        pack_x8_f16x2_32(x, hp, hi, lo);
                        const int64_t col0 = (int64_t)prev_im.h * 64 + half * OC + 32 * h;
                        if (p.o8_v8) {
                            st_global_v8(row8 + col0, hi[0], hi[1], hi[2], hi[3], hi[4], hi[5], hi[6], hi[7]);
                            st_global_v8(row8 + p.o8_half + col0, lo[0], lo[1], lo[2], lo[3], lo[4], lo[5], lo[6],
                                         lo[7]);
                        } else {
                            uint4 *ph = reinterpret_cast<uint4 *>(row8 + col0);
                            uint4 *pl = reinterpret_cast<uint4 *>(row8 + p.o8_half + col0);
                            ph[0] = make_uint4(hi[0], hi[1], hi[2], hi[3]);
                            ph[1] = make_uint4(hi[4], hi[5], hi[6], hi[7]);
                            pl[0] = make_uint4(lo[0], lo[1], lo[2], lo[3]);
                            pl[1] = make_uint4(lo[4], lo[5], lo[6], lo[7]);
                        }
                    }
#pragma unroll
                    for (int c = 0; c < 4; ++c) {
                        const int chunk = (half * (OC / 8) + 4 * h + c) ^ (r & 7);
                        *reinterpret_cast<uint4 *>(row + chunk * 16) =
                            make_uint4(hp[4 * c], hp[4 * c + 1], hp[4 * c + 2], hp[4 * c + 3]);
                    }
                    continue;
                }
                if (p.o32 != nullptr) {
                    if (row32 != nullptr) {
#pragma unroll
                        for (int c = 0; c < 8; ++c)
                            *reinterpret_cast<float4 *>(row32 + 32 * h + 4 * c) =
                                make_float4(v[4 * c] * inv, v[4 * c + 1] * inv, v[4 * c + 2] * inv, v[4 * c + 3] * inv);
                    }
                    continue;
                }
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    const int chunk = (half * (OC / 8) + 4 * h + c) ^ (r & 7);
                    *reinterpret_cast<uint4 *>(row + chunk * 16) =
                        make_uint4(pack_p<F16>(v[8 * c + 0] * inv, v[8 * c + 1] * inv),
                                   pack_p<F16>(v[8 * c + 2] * inv, v[8 * c + 3] * inv),
                                   pack_p<F16>(v[8 * c + 4] * inv, v[8 * c + 5] * inv),
                                   pack_p<F16>(v[8 * c + 6] * inv, v[8 * c + 7] * inv));
                }
            }
            fence_proxy_async_smem();  // visible to the TMA store
        };
        for (int32_t it = (int32_t)first + q, it_end = (int32_t)last; it < it_end && ok; it += 2, ++wi) {
            const Item im = decode_item(p, it);
            const uint32_t slot = wi & 1;
            {
                const bool got = mbar_wait(&b.m_full[slot], (wi >> 1) & 1, abort_flag, p.err, ERR_SITE_ATTN_SOFTMAX);
                if (!__all_sync(0xffffffffu, got)) break;
            }
            const MaskSlot &m = mslots[q * 2 + slot];
            const bool uniform = m.uniform != 0;
            // A warp whose 32 query rows all lie past n has no output: it only keeps the barrier
            // protocol (its P and O rows are never read back).
            const bool dead = im.q0 + quarter * 32 >= n;
            float m_run = -INFINITY, l_run = 0.0f;
            const int Ti = m.ntiles;
            float pt[kTailMax];  // this item's tail probabilities (key tail)
#pragma unroll
            for (int t = 0; t < kTailMax; ++t) pt[t] = 0.0f;
            // Modes 1-2, this thread's row i: the visible keys of a TILE_ROWS tile are the valid keys
            // below A plus the keys in [B, C] (encoder row: A = i + 1, or ne for a bidirectional
            // group, and B = C = i, the diagonal; decoder row: A = l, B = ne, C = i).
            int rA = 0, rB = 0, rC = -1;
            if (p.mode != 0) {
                const int i = im.q0 + r;
                if (i < p.ne) {
                    rA = m.bidir ? p.ne : i + 1;
                    rB = rC = i;
                } else {
                    rA = min(p.l, n);
                    rB = p.ne;
                    rC = i;
                }
            }
            for (int j = 0; j < Ti; ++j, ++cx) {
                // Key tail: this row's scores of the tail keys (raw units, like S), computed from the
                // item's Q tile in shared memory before waiting for the last S; -inf when masked.
                float st[kTailMax];
                const bool tail_here = TAIL && j == Ti - 1 && !dead;
                if constexpr (TAIL) {
                    bool q_ok = true;
                    if (tail_here) {
                        // The item's Q tile has landed (its load's barrier phase, observed here so the
                        // TMA-written bytes are visible to these loads).
                        q_ok = mbar_wait(&b.q_full[slot], (wi >> 1) & 1, abort_flag, p.err, ERR_SITE_ATTN_SOFTMAX);
                    }
                    if (!__all_sync(0xffffffffu, q_ok)) {
                        ok = false;
                        break;
                    }
                }
                if (tail_here) {
#pragma unroll
                    for (int t = 0; t < kTailMax; ++t) st[t] = 0.0f;
                    const uint8_t *qrow = smem + q * PIPE_BYTES + OFF_Q + slot * kTileBytes + r * 128;
#pragma unroll
                    for (int c = 0; c < 8; ++c) {
                        const uint4 qa = *reinterpret_cast<const uint4 *>(qrow + ((c ^ (r & 7)) << 4));
                        const float2 q0 = unpack2<F16>(qa.x), q1 = unpack2<F16>(qa.y), q2 = unpack2<F16>(qa.z),
                                     q3 = unpack2<F16>(qa.w);
#pragma unroll
                        for (int t = 0; t < kTailMax; ++t) {
                            if (t >= p.tail) break;
                            const uint4 ka = __ldg(reinterpret_cast<const uint4 *>(
                                                       p.kraw + ((int64_t)im.g * n + (int64_t)(p.tiles0 * kTileRows + t)) * p.ldraw +
                                                       im.h * 64) + c);
                            const float2 k0 = unpack2<F16>(ka.x), k1 = unpack2<F16>(ka.y), k2 = unpack2<F16>(ka.z),
                                         k3 = unpack2<F16>(ka.w);
                            float a = st[t];
                            a = fmaf(q0.x, k0.x, a);
                            a = fmaf(q0.y, k0.y, a);
                            a = fmaf(q1.x, k1.x, a);
                            a = fmaf(q1.y, k1.y, a);
                            a = fmaf(q2.x, k2.x, a);
                            a = fmaf(q2.y, k2.y, a);
                            a = fmaf(q3.x, k3.x, a);
                            a = fmaf(q3.y, k3.y, a);
                            st[t] = a;
                        }
                    }
                    const uint32_t tb = m.bits[4 * p.tiles0];
#pragma unroll
                    for (int t = 0; t < kTailMax; ++t) {
                        float x = st[t];
                        if (p.rel) x += m.rel[p.tiles0 * kTileRows + t - r + (kTileRows - 1)];
                        st[t] = t >= p.tail ? -INFINITY : uniform ? 0.0f : ((tb >> t) & 1u) ? x : -INFINITY;
                    }
                }
                const bool got = mbar_wait(&b.s_full, cx & 1, abort_flag, p.err, ERR_SITE_ATTN_SOFTMAX);
                if (!__all_sync(0xffffffffu, got)) {
                    ok = false;
                    break;
                }
                // In the first tile of an item the previous item's O is staged once the previous
                // PV is done and before this tile's p_ready lets the first PV overwrite it.
                const bool stage = j == 0 && prev_live;
                if (dead) {
                    // p_ready of this tile may only count once the previous phase completed:
                    // wait for the previous PV like the live warps.
                    tc_fence_before();
                    mbar_arrive(&b.s_free);
                    if (cx > 0) {
                        const bool done = mbar_wait(&b.o_done, (cx - 1) & 1, abort_flag, p.err, ERR_SITE_ATTN_SOFTMAX);
                        if (!__all_sync(0xffffffffu, done)) {
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                    }
                    if (stage) stage_prev_row(slot ^ 1u);
                    tc_fence_before();
                    mbar_arrive(&b.p_ready);
                    continue;
                }
                tc_fence_after();
                float s[SC];
                if constexpr (SPLIT) {
                    float c0[32], c1[32];
                    tmem_ld32(t_s + 0, c0);
                    tmem_ld32(t_s + 32, c1);
                    tmem_wait_ld();
#pragma unroll
                    for (int i = 0; i < 32; ++i) {
                        s[i] = c0[i];
                        s[32 + i] = c1[i];
                    }
                } else {
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
                mbar_arrive(&b.s_free);
                if (p.rel) {
                    const float *rw = m.rel + j * kTileRows + kofs - r + (kTileRows - 1);
#pragma unroll
                    for (int i = 0; i < SC; ++i) s[i] += rw[i];
                }

                // Mask: valid prefix of the tile (keys below n), or per-key bits; uniform groups
                // give every key below n the score 0.
                const int cls = m.cls[j];
                if (uniform || cls == TILE_PREFIX) {
                    const int cnt = n - j * kTileRows - kofs;
                    const float keep = uniform ? 0.0f : 1.0f;
#pragma unroll
                    for (int i = 0; i < SC; ++i) s[i] = i < cnt ? s[i] * keep : -INFINITY;
                } else if (cls == TILE_BITS || cls == TILE_ROWS) {
                    uint32_t wd[SC / 32];
#pragma unroll
                    for (int w = 0; w < SC / 32; ++w) wd[w] = m.bits[4 * j + kofs / 32 + w];
                    if (cls == TILE_ROWS) {
#pragma unroll
                        for (int w = 0; w < SC / 32; ++w) {
                            const int k0 = j * kTileRows + kofs + 32 * w;
                            wd[w] = (wd[w] & low_bits(rA - k0)) | (low_bits(rC + 1 - k0) & ~low_bits(rB - k0));
                        }
                    }
#pragma unroll
                    for (int i = 0; i < SC; ++i) s[i] = ((wd[i >> 5] >> (i & 31)) & 1u) ? s[i] : -INFINITY;
                }
                // Three-input maxima on four partial chains keep the dependency chains short.
                float mxp[4] = {s[0], s[1], s[2], s[3]};
#pragma unroll
                for (int i = 4; i + 1 < SC - 4; i += 2) mxp[(i >> 1) & 3] = max3(mxp[(i >> 1) & 3], s[i], s[i + 1]);
                float mx = max3(max3(mxp[0], mxp[1], mxp[2]), max3(mxp[3], s[SC - 4], s[SC - 3]),
                                fmaxf(s[SC - 2], s[SC - 1]));
                if (tail_here) {
#pragma unroll
                    for (int t = 0; t < kTailMax; ++t) mx = fmaxf(mx, st[t]);
                }
                if constexpr (SPLIT) {
                    // The row maximum over both halves (the pair takes the same rescale decision).
                    float other;
                    if (!xchg(mx, other)) {
                        ok = false;
                        break;
                    }
                    mx = fmaxf(mx, other);
                }
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

                // P overwrites the previous tile's P in TMEM, and O is rescaled below: both need
                // this pipeline's previous PV complete.
                if (cx > 0) {
                    const bool done = mbar_wait(&b.o_done, (cx - 1) & 1, abort_flag, p.err, ERR_SITE_ATTN_SOFTMAX);
                    if (!__all_sync(0xffffffffu, done)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                }
                float sp4[4] = {0.0f, 0.0f, 0.0f, 0.0f};
                // Quarters of a prefix tile past the last valid key hold only zeros.
                const int live = (uniform || cls == TILE_PREFIX) ? n - j * kTileRows : kTileRows;
#pragma unroll
                for (int qc = 0; qc < SC / 32; ++qc) {
                    uint32_t pk[16];  // 32 keys as 16 packed 16-bit pairs
                    if (kofs + 32 * qc >= live) {
#pragma unroll
                        for (int e = 0; e < 16; ++e) pk[e] = 0u;
                        tmem_st16(t_p + 16 * qc, pk);
                        continue;
                    }
#pragma unroll
                    for (int e = 0; e < 16; ++e) {
                        const float a = ex2_approx(fmaf(s[32 * qc + 2 * e], sl2, -mb));
                        const float c = ex2_approx(fmaf(s[32 * qc + 2 * e + 1], sl2, -mb));
                        sp4[e & 3] += a + c;
                        pk[e] = pack_p<F16>(a, c);
                    }
                    tmem_st16(t_p + 16 * qc, pk);
                }
                if (tail_here) {
#pragma unroll
                    for (int t = 0; t < kTailMax; ++t) {
                        pt[t] = ex2_approx(fmaf(st[t], sl2, -mb));
                        sp4[t & 3] += pt[t];
                    }
                }
                l_run = l_run * alpha + ((sp4[0] + sp4[1]) + (sp4[2] + sp4[3]));
                if (j > 0 && __any_sync(0xffffffffu, rescale)) {
#pragma unroll
                    for (int hcol = 0; hcol < OC; hcol += 32) {
                        float ov[32];
                        tmem_ld32(t_o + hcol, ov);
                        tmem_wait_ld();
#pragma unroll
                        for (int i = 0; i < 32; ++i) ov[i] *= alpha;
                        tmem_st32(t_o + hcol, ov);
                    }
                }
                if (stage) stage_prev_row(slot ^ 1u);
                tmem_wait_st();
                tc_fence_before();
                mbar_arrive(&b.p_ready);
            }
            if (!ok) break;
            if constexpr (SPLIT) {
                // The full row sum for the output staging (both halves of a live row).
                if (!dead) {
                    float other;
                    if (!xchg(l_run, other)) {
                        ok = false;
                        break;
                    }
                    prev_ltot = l_run + other;
                }
            }
            mbar_arrive(&b.m_empty[slot]);
            prev_live = !dead;
            prev_im = im;
#pragma unroll
            for (int t = 0; t < kTailMax; ++t) prev_pt[t] = pt[t];
            if constexpr (!SPLIT) *l_save = l_run;
        }
        // The last item's output, once its last PV is done; one more p_ready phase tells the
        // tensor-core thread that it is staged.
        if (ok && cx > 0) {
            const bool done = mbar_wait(&b.o_done, (cx - 1) & 1, abort_flag, p.err, ERR_SITE_ATTN_SOFTMAX);
            if (__all_sync(0xffffffffu, done)) {
                tc_fence_after();
                if (prev_live) stage_prev_row((wi - 1) & 1);
                mbar_arrive(&b.p_ready);
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == W_MMA) {
        tc_fence_after();
        tmem_dealloc(tmem_base, kTmemCols);
    }
}

// Registers are allocated for warps in groups of four: 12 warps x 32 x 168 = 64,512 of the SM's
// 65,536; the split instance, 19 warps (20 x 32 x 96 = 61,440). One CTA per SM (the shared memory
// and the 512 TMEM columns allow no second one).
template <bool F16, bool O8 = false, bool TAIL = false>
__global__ void __maxnreg__(168)
    attn_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                   const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmO, TcParams p) {
    attn_tc_body<F16, O8, TAIL, false>(tmQ, tmK, tmV, tmO, p);
}

template <bool F16, bool O8 = false>
__global__ void __maxnreg__(96)
    attn_tc_split_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                         const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmO,
                         TcParams p) {
    attn_tc_body<F16, O8, false, true>(tmQ, tmK, tmV, tmO, p);
}

}  // namespace

bool attention_tc_supported(const AttentionCall &c) {
    if (c.force_path == 2) return false;
    if (c.mask_mode < 0 || c.mask_mode > 2) return false;
    if (c.rel_bias != nullptr && (c.mask_mode != 0 || c.n > kMaxKeysRel)) return false;
    if (c.mask_mode != 0 && (c.ne < 0 || c.ne > c.n || c.l < 0)) return false;
    if (c.o32 != nullptr && (c.o8 != nullptr || (reinterpret_cast<uintptr_t>(c.o32) & 15) || (c.ld_o32 % 4))) return false;
    if (c.dtype != E_F16 && c.dtype != E_BF16) return false;
    if (c.n <= 0 || c.n > kMaxKeys || c.heads <= 0 || c.groups <= 0) return false;
    if ((int64_t)c.groups * c.n > INT32_MAX - 2 * kTileRows) return false;
    if ((int64_t)c.groups * c.heads * ((c.n + kTileRows - 1) / kTileRows) > INT32_MAX) return false;
    // TMA: 16-byte aligned bases and row strides.
    const auto a16 = [](const void *q) { return (reinterpret_cast<uintptr_t>(q) & 15) == 0; };
    if (!a16(c.q) || !a16(c.k) || !a16(c.v) || !a16(c.o) || (c.ld_qkv % 8) || (c.ld_o % 8)) return false;
    return true;
}

Status launch_attention_tc(const AttentionCall &c, cudaStream_t stream) {
    if (!attention_tc_supported(c)) return Status::fail(TSFM_ERR_UNSUPPORTED, "attention: the tcgen05 path does not take this call");
    const int64_t rows = (int64_t)c.groups * c.n;
    const int64_t width = (int64_t)c.heads * 64;
    alignas(64) CUtensorMap mq, mk, mv, mo;
    TSFM_TRY(make_tmap_2d(&mq, c.q, c.dtype, width, rows, c.ld_qkv, 64, kTileRows));
    TSFM_TRY(make_tmap_2d(&mk, c.k, c.dtype, width, rows, c.ld_qkv, 64, kTileRows));
    TSFM_TRY(make_tmap_2d(&mv, c.v, c.dtype, width, rows, c.ld_qkv, 64, kTileRows));
    // Output rows per group: a query tile that runs past n is clipped at the group's end. (An FP32
    // output is written by the softmax threads; the map is then never used.)
    if (c.o32 == nullptr)
        TSFM_TRY(make_tmap_grouped_rows(&mo, c.o, c.dtype, width, c.n, c.groups, c.ld_o, 64, kTileRows));
    else
        mo = mq;
    TcParams p;
    p.key_valid = c.key_valid;
    p.kvs = c.kv_stride > 0 ? c.kv_stride : c.n;
    p.rel = c.rel_bias;
    p.rel_stride = c.rel_stride > 0 ? c.rel_stride : 2 * (int64_t)c.n - 1;
    p.rel_center = c.rel_center >= 0 ? c.rel_center : (int64_t)c.n - 1;
    p.n = c.n;
    p.heads = c.heads;
    p.groups = c.groups;
    p.qtiles = (c.n + kTileRows - 1) / kTileRows;
    p.items = (int64_t)c.groups * c.heads * p.qtiles;
    p.scale_log2 = c.scale * 1.4426950408889634f;
    p.err = c.err;
    p.o8 = static_cast<uint8_t *>(c.o8);
    p.ld_o8 = c.ld_o8;
    p.o8_half = width;
    p.o8_v8 = ((reinterpret_cast<uintptr_t>(c.o8) | (uintptr_t)c.ld_o8) & 31) == 0;
    p.mode = c.mask_mode;
    p.ne = c.mask_mode == 0 ? c.n : c.ne;
    p.l = c.l;
    p.bidir = c.group_bidir;
    p.bidir_all = c.mask_mode == 2 ? 1 : 0;
    p.o32 = c.o32;
    p.ld_o32 = c.ld_o32;
    const int T = (c.n + kTileRows - 1) / kTileRows;
    const int rem = c.n - (T - 1) * kTileRows;
    p.tail = c.mask_mode == 0 && T >= 2 && rem <= kTailMax && c.o8 == nullptr && c.o32 == nullptr ? rem : 0;
    p.tiles0 = T - (p.tail > 0 ? 1 : 0);
    p.kraw = static_cast<const uint16_t *>(c.k);
    p.vraw = static_cast<const uint16_t *>(c.v);
    p.ldraw = c.ld_qkv;
    if (c.o8 && (c.dtype != E_F16 || c.ld_o8 % 16 || c.ld_o8 < 2 * width || (reinterpret_cast<uintptr_t>(c.o8) & 15)))
        return Status::fail(TSFM_ERR_INVALID_ARGUMENT, "attention: an FP8 companion needs an FP16 output");
    const int64_t grid = std::min<int64_t>((p.items + 1) / 2, num_sms());
    // Split rows (two softmax threads per query row) on request only (force_path 3): alone, with the
    // L2 flushed and fixed clocks, it ran Chronos-2's 577 tokens 8-9 % faster (0.889 -> 0.814 ms per
    // layer), but inside the corrected forward (power-capped clocks, operands warm in L2) the
    // attention class took 15.9-16.4 ms against 14.5-14.8 ms for whole rows (A/B on one box).
    const bool split = c.force_path == 3;
    if (split) p.tail = 0, p.tiles0 = p.mode == 0 ? (c.n + kTileRows - 1) / kTileRows : p.tiles0;
    if (split && c.dtype == E_F16 && c.o8) {
        TSFM_TRY(ensure_smem_attr(reinterpret_cast<const void *>(&attn_tc_split_kernel<true, true>), kSmemTc));
        attn_tc_split_kernel<true, true><<<(unsigned)grid, kThreadsSplit, kSmemTc, stream>>>(mq, mk, mv, mo, p);
    } else if (split && c.dtype == E_F16) {
        TSFM_TRY(ensure_smem_attr(reinterpret_cast<const void *>(&attn_tc_split_kernel<true>), kSmemTc));
        attn_tc_split_kernel<true><<<(unsigned)grid, kThreadsSplit, kSmemTc, stream>>>(mq, mk, mv, mo, p);
    } else if (split) {
        TSFM_TRY(ensure_smem_attr(reinterpret_cast<const void *>(&attn_tc_split_kernel<false>), kSmemTc));
        attn_tc_split_kernel<false><<<(unsigned)grid, kThreadsSplit, kSmemTc, stream>>>(mq, mk, mv, mo, p);
    } else if (c.dtype == E_F16 && c.o8) {
        TSFM_TRY(ensure_smem_attr(reinterpret_cast<const void *>(&attn_tc_kernel<true, true>), kSmemTc));
        attn_tc_kernel<true, true><<<(unsigned)grid, kThreadsTc, kSmemTc, stream>>>(mq, mk, mv, mo, p);
    } else if (c.dtype == E_F16 && p.tail > 0) {
        TSFM_TRY(ensure_smem_attr(reinterpret_cast<const void *>(&attn_tc_kernel<true, false, true>), kSmemTc));
        attn_tc_kernel<true, false, true><<<(unsigned)grid, kThreadsTc, kSmemTc, stream>>>(mq, mk, mv, mo, p);
    } else if (c.dtype == E_F16) {
        TSFM_TRY(ensure_smem_attr(reinterpret_cast<const void *>(&attn_tc_kernel<true>), kSmemTc));
        attn_tc_kernel<true><<<(unsigned)grid, kThreadsTc, kSmemTc, stream>>>(mq, mk, mv, mo, p);
    } else if (p.tail > 0) {
        TSFM_TRY(ensure_smem_attr(reinterpret_cast<const void *>(&attn_tc_kernel<false, false, true>), kSmemTc));
        attn_tc_kernel<false, false, true><<<(unsigned)grid, kThreadsTc, kSmemTc, stream>>>(mq, mk, mv, mo, p);
    } else {
        TSFM_TRY(ensure_smem_attr(reinterpret_cast<const void *>(&attn_tc_kernel<false>), kSmemTc));
        attn_tc_kernel<false><<<(unsigned)grid, kThreadsTc, kSmemTc, stream>>>(mq, mk, mv, mo, p);
    }
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return Status::cuda(e, "attention (tcgen05): launch");
    return Status::ok();
}

}  // namespace tsfm
