// The linear-layer kernel: y = epilogue(x[M, K] · W[N, K]^T) on the sm_100a tensor cores.
//
// Replaces nn.linear / gemmNTFallback (core/nn.zig:68-162, 270-293) and the cuBLAS SGEMM the
// reference offloads to (platform/cuda/gemm.c:252-314).
//
// Design (one persistent CTA per SM, 6 warps):
//   warp 0       TMA producer: 128-byte-swizzled K-major tiles of x (128 rows) and W (BN rows)
//                into a STAGES-deep shared-memory ring, one mbarrier pair per stage.
//   warp 1       tensor-memory allocator + MMA issuer (one elected thread): tcgen05.mma
//                M=128 x N=BN x K=16 (BF16, kind::f16) or K=8 (TF32, kind::tf32), FP32
//                accumulators in TMEM, double-buffered so the epilogue of tile i overlaps the
//                main loop of tile i+1.
//   warps 2..5   epilogue: tcgen05.ld 32 lanes x 32 columns, fused bias / ReLU / rotate-half RoPE
//                / residual accumulation, vectorised stores (BF16 or FP32), optional row remap
//                so embeddings land directly in their sequence slots.
// Tiles are walked m-major with the BN-wide column tiles of one row block adjacent, so CTAs
// working on the same 128 rows of x run together and share them through L2; W stays L2-resident.
// Every output element is reduced over K by one CTA in a fixed order (no split-K, no atomics),
// so results do not depend on the grid size or the number of GPUs.
#include "kernels.h"
#include "ptx.cuh"
#include "x8.cuh"

#include <cuda_fp16.h>
#include <cudaTypedefs.h>

#include <cstdlib>
#include <mutex>
#include <utility>
#include <vector>
#include <type_traits>

namespace tsfm {

namespace {

constexpr int kBM = 128;
constexpr int kThreads = 192;

// PAIR: the tile is 256 x BN, computed by a cluster of two CTAs with the 2-SM MMA; each CTA holds
// 128 rows of x and BN / 2 rows of W per stage and 128 x BN accumulators.
// NORM: the residual epilogue of a fused RMSNorm (see Epi) needs a 2 KB staging box per epilogue
// warp for the 16-bit row copy, paid for with one pipeline stage.
template <int BN, bool PAIR = false, bool NORM = false>
struct TileCfg {
    static constexpr int STAGES = (PAIR ? 6 : BN >= 256 ? 4 : 6) - (NORM ? 1 : 0);
    static constexpr int A_BYTES = kBM * 128;
    static constexpr int B_ROWS = PAIR ? BN / 2 : BN;
    static constexpr int B_BYTES = B_ROWS * 128;
    static constexpr int TMEM_COLS = 2 * BN <= 32 ? 32 : 2 * BN <= 64 ? 64 : 2 * BN <= 128 ? 128 : 2 * BN <= 256 ? 256 : 512;
    // Epilogue staging for the TMA stores: per epilogue warp two 4 KB boxes (32 rows x 128 B).
    static constexpr int STAGE_OFF = STAGES * (A_BYTES + B_BYTES);
    static constexpr int STAGE_BYTES = 4 * 2 * 4096 + (NORM ? 4 * 2048 : 0);
    static constexpr int SMEM = 1024 + STAGE_OFF + STAGE_BYTES + 256;
};

struct Epi {
    int64_t M, N, K;
    void *out;
    int64_t ldo;
    const float *bias;
    int act;           // 0 none, 1 relu, 2 silu
    int out_mode;      // OutMode
    int64_t rm_g, rm_G, rm_off;  // output row = (r / rm_g) * rm_G + r % rm_g + rm_off (rm_g > 0)
    const float *rope_cos;       // [positions, 32]; null = no rotation
    const float *rope_sin;
    int rope_cols;               // columns [0, rope_cols) are rotated per 64-wide head
    int64_t rope_p1, rope_p2;    // position index = (r / p1) * p2 + r % p2 (p1 == 0: r % p2)
    int tma_mode;                // 0: per-thread stores; 1: TMA store of staged boxes; 2: TMA reduce-add (f32)
    int *err;
    // Fused RMSNorm (LinearCall::norm_*). Reader side: rows scaled by rs / ns_in[r] with
    // rs = 1 / sqrt(sum_p nin[p * M + r] / ndim + neps); rs written to ns_out[r] by column tile 0.
    const float *nin;
    int nparts;
    float ndim, neps;
    const float *ns_in;
    float *ns_out;
    // Residual side (NORM kernels): y += result, then nx16[r, c] = y[r, c] * xs * ngamma[c] in 16
    // bits (xs = rs when nin is set, else ns_in[r]) and nout[tile * M + r] = sum over the tile of y^2.
    float *nout;
    void *nx16;
    int64_t ldx16;
    const float *ngamma;
    // Corrected products: K8 companion columns per row take part (2K: both correction terms; K:
    // the weight term only); the accumulator is multiplied by acc_scale before the epilogue; y8 /
    // nx8 (bytes, row strides ldy8 / ldnx8) receive the FP8 companions of the 16-bit outputs, the
    // low-part block `y8_half` / `nx8_half` bytes after the high part.
    int64_t K8;
    float acc_scale;
    uint8_t *y8;
    int64_t ldy8, y8_half;
    int y8_tma;  // y8 written by TMA stores of staged boxes (tmY8: bytes [rows, 2 y8_half], 64-byte boxes)
    uint8_t *nx8;
    int64_t ldnx8, nx8_half;
};

// Activation over n values: 1 relu, 2 silu (nn.siluInPlace, core/nn.zig:399-407). The branch is
// uniform and taken outside the element loops, so act == 0 costs nothing. ACT_GLU (gated pairs,
// handled in the epilogue loop) never reaches here.
template <int N>
__device__ __forceinline__ void apply_act(int act, float *v) {
    if (act == 1) {
#pragma unroll
        for (int j = 0; j < N; ++j) v[j] = fmaxf(v[j], 0.0f);
    } else if (act == 2) {
#pragma unroll
        for (int j = 0; j < N; ++j) v[j] = v[j] / (1.0f + expf(-v[j]));
    }
}

template <typename H>
__device__ __forceinline__ uint32_t pack2(float a, float b);
template <>
__device__ __forceinline__ uint32_t pack2<__nv_bfloat16>(float a, float b) {
    __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t *>(&v);
}
template <>
__device__ __forceinline__ uint32_t pack2<__half>(float a, float b) {
    __half2 v = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t *>(&v);
}

template <typename H>
__device__ __forceinline__ void store16(const Epi &e, int64_t orow, int64_t col0, int nvalid, const float (&v)[32]) {
    H *o = reinterpret_cast<H *>(e.out) + orow * e.ldo + col0;
    if (nvalid == 32 && ((reinterpret_cast<uintptr_t>(o) & 15) == 0)) {
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            uint4 pk;
            pk.x = pack2<H>(v[q * 8 + 0], v[q * 8 + 1]);
            pk.y = pack2<H>(v[q * 8 + 2], v[q * 8 + 3]);
            pk.z = pack2<H>(v[q * 8 + 4], v[q * 8 + 5]);
            pk.w = pack2<H>(v[q * 8 + 6], v[q * 8 + 7]);
            reinterpret_cast<uint4 *>(o)[q] = pk;
        }
    } else {
#pragma unroll
        for (int j = 0; j < 32; ++j)
            if (j < nvalid) {
                const uint32_t w = pack2<H>(v[j], 0.0f);
                *reinterpret_cast<uint16_t *>(o + j) = (uint16_t)(w & 0xffffu);
            }
    }
}

__device__ __forceinline__ void store_chunk(const Epi &e, int64_t orow, int64_t col0, int nvalid, float (&v)[32]) {
    if (e.out_mode == OUT_BF16) {
        store16<__nv_bfloat16>(e, orow, col0, nvalid, v);
    } else if (e.out_mode == OUT_F16) {
        store16<__half>(e, orow, col0, nvalid, v);
    } else {
        float *o = reinterpret_cast<float *>(e.out) + orow * e.ldo + col0;
        if (e.out_mode == OUT_TF32) {
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = to_tf32(v[j]);
        }
        const bool vec = nvalid == 32 && ((reinterpret_cast<uintptr_t>(o) & 15) == 0);
        if (e.out_mode == OUT_F32_ACC) {
            // Read the whole chunk first (eight loads in flight), add, activate, write back.
            float a[32];
            if (vec) {
#pragma unroll
                for (int q = 0; q < 8; ++q) {
                    const float4 t = reinterpret_cast<const float4 *>(o)[q];
                    a[4 * q] = t.x;
                    a[4 * q + 1] = t.y;
                    a[4 * q + 2] = t.z;
                    a[4 * q + 3] = t.w;
                }
            } else {
#pragma unroll
                for (int j = 0; j < 32; ++j) a[j] = j < nvalid ? o[j] : 0.0f;
            }
#pragma unroll
            for (int j = 0; j < 32; ++j) a[j] += v[j];
            apply_act<32>(e.act, a);
            if (vec) {
#pragma unroll
                for (int q = 0; q < 8; ++q)
                    reinterpret_cast<float4 *>(o)[q] = make_float4(a[4 * q], a[4 * q + 1], a[4 * q + 2], a[4 * q + 3]);
            } else {
#pragma unroll
                for (int j = 0; j < 32; ++j)
                    if (j < nvalid) o[j] = a[j];
            }
        } else {
            if (vec) {
#pragma unroll
                for (int q = 0; q < 8; ++q)
                    reinterpret_cast<float4 *>(o)[q] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
            } else {
#pragma unroll
                for (int j = 0; j < 32; ++j)
                    if (j < nvalid) o[j] = v[j];
            }
        }
    }
}

__device__ __forceinline__ void bias_act(const Epi &e, int64_t col0, int nvalid, float (&v)[32]) {
    if (e.bias) {
#pragma unroll
        for (int j = 0; j < 32; ++j)
            if (j < nvalid) v[j] += __ldg(e.bias + col0 + j);
    }
    // In accumulate mode the activation applies to the accumulated sum (store_chunk).
    if (e.out_mode != OUT_F32_ACC) apply_act<32>(e.act, v);
}

// CORR: corrected product; tmA8 / tmB8 map the FP8 companions of x and W ([rows, 2K] bytes).
// The K loop runs ceil(2K / 128) FP8 stages (kind::f8f6f4, the small correction terms first),
// then ceil(K / BK) FP16 stages (kind::f16), all into one FP32 accumulator.
template <typename T, int BN, bool PAIR, bool NORM, bool CORR>
__global__ void __launch_bounds__(kThreads, 1)
    linear_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                     const __grid_constant__ CUtensorMap tmY, const __grid_constant__ CUtensorMap tmA8,
                     const __grid_constant__ CUtensorMap tmB8, const __grid_constant__ CUtensorMap tmY8, Epi e) {
    using C = TileCfg<BN, PAIR, NORM>;
    constexpr int STAGES = C::STAGES;
    constexpr int BK = 128 / (int)sizeof(T);
    // FP8 companions of FP16 outputs are written by the FP16 and TF32 instances (BF16 never
    // feeds a corrected product).
    constexpr bool CORR_OUT = !std::is_same<T, __nv_bfloat16>::value;
    // operand format: BF16 = 1, F16 = 0 (kind::f16); TF32 = 2 (kind::tf32)
    constexpr uint32_t FMT = std::is_same<T, float>::value ? 2u : std::is_same<T, __half>::value ? 0u : 1u;
    static_assert(!PAIR || FMT != 2u, "the 2-SM path takes 16-bit operands");
    static_assert(!CORR || FMT == 0u, "corrected products take FP16 operands");
    constexpr uint32_t IDESC = idesc_f32acc(FMT, PAIR ? 2 * kBM : kBM, BN);
    // CTA pairs: rank 0 issues the MMAs for both; the tile's rows split by rank.
    const uint32_t rank = PAIR ? cluster_ctarank() : 0u;
    const bool leader = rank == 0;
    constexpr int kRows = PAIR ? 2 * kBM : kBM;  // rows of x per tile
    const int64_t unit = PAIR ? (int64_t)(blockIdx.x >> 1) : (int64_t)blockIdx.x;
    const int64_t units = PAIR ? (int64_t)(gridDim.x >> 1) : (int64_t)gridDim.x;

    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *sA = smem;
    uint8_t *sB = smem + STAGES * C::A_BYTES;
    uint8_t *sStage = smem + C::STAGE_OFF;
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + C::STAGE_OFF + C::STAGE_BYTES);
    uint64_t *empty = full + STAGES;
    uint64_t *tfull = empty + STAGES;
    uint64_t *tempty = tfull + 2;
    uint64_t *drain = tempty + 2;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(drain + 1);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t m_tiles = (e.M + kRows - 1) / kRows, n_tiles = (e.N + BN - 1) / BN;
    const int64_t tiles = m_tiles * n_tiles;
    const int num_k8 = CORR ? (int)((e.K8 + 127) / 128) : 0;  // FP8 correction stages
    const int num_k = num_k8 + (int)((e.K + BK - 1) / BK);

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&tfull[i], 1);
            mbar_init(&tempty[i], (PAIR ? 2 : 1) * 4 * 32);  // the epilogue threads of every CTA of the tile
        }
        mbar_init(drain, 1);
        *abort_flag = 0;
        fence_barrier_init();
        tma_prefetch_desc(&tmA);
        tma_prefetch_desc(&tmB);
        if constexpr (CORR) {
            tma_prefetch_desc(&tmA8);
            tma_prefetch_desc(&tmB8);
        }
    }
    if (warp == 1) {
        if constexpr (PAIR) {
            tmem_alloc_pair(tmem_slot, C::TMEM_COLS);
            tmem_relinquish_pair();
        } else {
            tmem_alloc(tmem_slot, C::TMEM_COLS);
            tmem_relinquish();
        }
    }
    tc_fence_before();
    __syncthreads();
    // Both CTAs of a pair have initialised their barriers before either signals the other's.
    if constexpr (PAIR) cluster_sync_all();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 0) {
        if (lane == 0) {
            int s = 0;
            uint32_t ph = 0;
            bool ok = true;
            uint32_t issued = 0, issued_ph = 0;  // per-stage bit: loaded at least once / parity of last load
            // Stages [kb0, kb1) of one operand kind: FP8 stages load 128 bytes of the companions'
            // rows (boxes of the same byte size as the 16-bit ones). One loop per kind, so no
            // stage branches on it.
            auto load_stages = [&](auto kind, int32_t m0, int32_t n0, int kb0, int kb1) -> bool {
                constexpr bool F8 = decltype(kind)::value;
                const CUtensorMap *ma = F8 ? &tmA8 : &tmA;
                const CUtensorMap *mb = F8 ? &tmB8 : &tmB;
                for (int kb = kb0; kb < kb1; ++kb) {
                    const bool got = PAIR ? mbar_wait_cl(&empty[s], ph ^ 1u, abort_flag, e.err, ERR_SITE_GEMM_PRODUCER)
                                          : mbar_wait(&empty[s], ph ^ 1u, abort_flag, e.err, ERR_SITE_GEMM_PRODUCER);
                    if (!got) return false;
                    const int32_t kc = F8 ? kb * 128 : (kb - kb0) * BK;
                    if constexpr (PAIR) {
                        // The pair's first CTA expects the bytes of both CTAs' boxes on its barrier.
                        if (leader) mbar_arrive_expect_tx(&full[s], 2 * (C::A_BYTES + C::B_BYTES));
                        const uint32_t fb = mapa_shared(&full[s], 0);
                        tma_load_2d_pair(sA + s * C::A_BYTES, ma, fb, kc, m0);
                        tma_load_2d_pair(sB + s * C::B_BYTES, mb, fb, kc, n0);
                    } else {
                        mbar_arrive_expect_tx(&full[s], C::A_BYTES + C::B_BYTES);
                        tma_load_2d(sA + s * C::A_BYTES, ma, &full[s], kc, m0);
                        tma_load_2d(sB + s * C::B_BYTES, mb, &full[s], kc, n0);
                    }
                    issued |= 1u << s;
                    issued_ph = (issued_ph & ~(1u << s)) | (ph << s);
                    if (++s == STAGES) {
                        s = 0;
                        ph ^= 1u;
                    }
                }
                return true;
            };
            for (int64_t t = unit; t < tiles && ok; t += units) {
                const int32_t m0 = (int32_t)((t / n_tiles) * kRows + rank * kBM);
                const int32_t n0 = (int32_t)((t % n_tiles) * BN + rank * C::B_ROWS);
                if constexpr (CORR) ok = load_stages(std::true_type{}, m0, n0, 0, num_k8);
                ok = ok && load_stages(std::false_type{}, m0, n0, num_k8, num_k);
            }
            if (!ok) {
                // Let loads already in flight land before the CTA can exit: the last load issued
                // into stage i completes phase issued_ph[i] of full[i]; bounded grace period. (A
                // pair's second CTA signals its loads on the first CTA's barriers; it waits out
                // the same grace period by the clock.)
                const unsigned long long t0 = globaltimer_ns();
                if (PAIR && !leader) {
                    while (globaltimer_ns() - t0 < 1000000ull) {
                    }
                } else {
                    for (int i = 0; i < STAGES; ++i) {
                        if (!((issued >> i) & 1u)) continue;
                        while (!mbar_try_wait_cl(&full[i], (issued_ph >> i) & 1u) && globaltimer_ns() - t0 < 100000000ull) {
                        }
                    }
                }
            }
        }
    } else if (warp == 1) {
        // In a pair only the first CTA issues MMAs (for both CTAs' tensor memory).
        if (lane == 0 && leader) {
            int s = 0;
            uint32_t ph = 0;
            int acc = 0;
            uint32_t aph = 0;
            bool ok = true;
            for (int64_t t = unit; t < tiles && ok; t += units) {
                const bool freed = PAIR ? mbar_wait_cl(&tempty[acc], aph ^ 1u, abort_flag, e.err, ERR_SITE_GEMM_MMA_EMPTY)
                                        : mbar_wait(&tempty[acc], aph ^ 1u, abort_flag, e.err, ERR_SITE_GEMM_MMA_EMPTY);
                if (!freed) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + (uint32_t)(acc * BN);
                // Stages [kb0, kb1) of one operand kind (one loop per kind, no per-stage branch).
                auto mma_stages = [&](auto kind, int kb0, int kb1) -> bool {
                  constexpr bool F8 = decltype(kind)::value;
                  for (int kb = kb0; kb < kb1; ++kb) {
                    const bool got = PAIR ? mbar_wait_cl(&full[s], ph, abort_flag, e.err, ERR_SITE_GEMM_MMA_FULL)
                                          : mbar_wait(&full[s], ph, abort_flag, e.err, ERR_SITE_GEMM_MMA_FULL);
                    if (!got) return false;
                    tc_fence_after();
                    const uint64_t ad = sdesc_k128(sA + s * C::A_BYTES);
                    const uint64_t bd = sdesc_k128(sB + s * C::B_BYTES);
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk) {
                        // advance 32 bytes along K inside the 128-byte swizzle atom
                        if constexpr (F8) {
                            if constexpr (PAIR)
                                mma_f8kind_pair(d_tmem, ad + 2 * kk, bd + 2 * kk, IDESC, (kb | kk) != 0);
                            else
                                mma_f8kind(d_tmem, ad + 2 * kk, bd + 2 * kk, IDESC, (kb | kk) != 0);
                        } else if constexpr (PAIR) {
                            mma_f16kind_pair(d_tmem, ad + 2 * kk, bd + 2 * kk, IDESC, (kb | kk) != 0);
                        } else if constexpr (sizeof(T) == 2) {
                            mma_f16kind(d_tmem, ad + 2 * kk, bd + 2 * kk, IDESC, (kb | kk) != 0);
                        } else {
                            mma_tf32(d_tmem, ad + 2 * kk, bd + 2 * kk, IDESC, (kb | kk) != 0);
                        }
                    }
                    if constexpr (PAIR) {
                        mma_commit_pair(mapa_shared(&empty[s], 0));
                        mma_commit_pair(mapa_shared(&empty[s], 1));
                    } else {
                        mma_commit(&empty[s]);
                    }
                    if (++s == STAGES) {
                        s = 0;
                        ph ^= 1u;
                    }
                  }
                  return true;
                };
                if constexpr (CORR) ok = mma_stages(std::true_type{}, 0, num_k8);
                ok = ok && mma_stages(std::false_type{}, num_k8, num_k);
                if (!ok) break;
                if constexpr (PAIR) {
                    mma_commit_pair(mapa_shared(&tfull[acc], 0));
                    mma_commit_pair(mapa_shared(&tfull[acc], 1));
                } else {
                    mma_commit(&tfull[acc]);
                }
                if (++acc == 2) {
                    acc = 0;
                    aph ^= 1u;
                }
            }
            // All MMAs issued by this thread have completed once `drain` fires; the tensor
            // memory can then be released safely even on the abort path.
            if constexpr (PAIR)
                mma_commit_pair(mapa_shared(drain, 0));
            else
                mma_commit(drain);
            const unsigned long long t0 = globaltimer_ns();
            while (!mbar_try_wait(drain, 0)) {
                if (globaltimer_ns() - t0 > kWaitTimeoutNs) {
                    if (e.err) atomicCAS(e.err, 0, ERR_SITE_GEMM_DRAIN);
                    break;
                }
            }
        }
    } else {
        // Epilogue warps 2..5 own TMEM lane groups (warp % 4) * 32.
        const int eg = warp & 3;
        const int r_in_tile = eg * 32 + lane;
        const bool f32_out = e.out_mode == OUT_F32 || e.out_mode == OUT_F32_ACC || e.out_mode == OUT_TF32;
        // TMA epilogue: each warp stages a box of its 32 rows (128 bytes per row: 32 f32 or 64
        // 16-bit values, 128-byte swizzle) and one lane stores or reduce-adds it; two boxes per
        // warp alternate so staging overlaps the previous box's transfer.
        uint8_t *wstage = sStage + eg * 8192;
        int sbuf = 0;
        auto stage_box = [&]() -> uint8_t * {
            if (lane == 0) bulk_wait_read_1();
            __syncwarp();
            uint8_t *b = wstage + sbuf * 4096;
            sbuf ^= 1;
            return b;
        };
        auto put16 = [&](uint8_t *b, int q, uint4 v) {  // 16-byte chunk q of this lane's row
            *reinterpret_cast<uint4 *>(b + lane * 128 + ((q ^ (lane & 7)) << 4)) = v;
        };
        auto issue_box = [&](const uint8_t *b, int64_t col0, int64_t row0) {
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
                if (e.tma_mode == 2)
                    tma_reduce_add_2d(&tmY, b, (int32_t)col0, (int32_t)row0);
                else
                    tma_store_2d(&tmY, b, (int32_t)col0, (int32_t)row0);
                bulk_commit();
            }
        };
        auto tma_f32 = [&](int64_t col0, int64_t row0, float (&v)[32]) {
            if (e.out_mode == OUT_TF32) {
#pragma unroll
                for (int j = 0; j < 32; ++j) v[j] = to_tf32(v[j]);
            }
            uint8_t *b = stage_box();
#pragma unroll
            for (int q = 0; q < 8; ++q) put16(b, q, make_uint4(__float_as_uint(v[4 * q]), __float_as_uint(v[4 * q + 1]),
                                                                __float_as_uint(v[4 * q + 2]), __float_as_uint(v[4 * q + 3])));
            issue_box(b, col0, row0);
        };
        auto tma_16 = [&](int64_t col0, int64_t row0, const float (&lo)[32], const float (&hi)[32]) {
            uint8_t *b = stage_box();
            const bool f16 = e.out_mode == OUT_F16;
#pragma unroll
            for (int q = 0; q < 8; ++q) {
                const float *src = q < 4 ? lo + 8 * q : hi + 8 * (q - 4);
                uint4 pk;
                pk.x = f16 ? pack2<__half>(src[0], src[1]) : pack2<__nv_bfloat16>(src[0], src[1]);
                pk.y = f16 ? pack2<__half>(src[2], src[3]) : pack2<__nv_bfloat16>(src[2], src[3]);
                pk.z = f16 ? pack2<__half>(src[4], src[5]) : pack2<__nv_bfloat16>(src[4], src[5]);
                pk.w = f16 ? pack2<__half>(src[6], src[7]) : pack2<__nv_bfloat16>(src[6], src[7]);
                put16(b, q, pk);
            }
            issue_box(b, col0, row0);
        };
        // The FP8 companion of this warp's 32 rows x 64 columns (col0 in output columns): staged as
        // 64 hi and 64 lo bytes per row in a 64-byte-swizzled box and stored with two TMA stores.
        auto stage_issue_x8 = [&](int64_t col0, int64_t row0, const uint32_t (&xh)[2][8], const uint32_t (&xl)[2][8]) {
            uint8_t *b = stage_box();
            stage_x8_32(b, lane, 0, xh[0], xl[0]);
            stage_x8_32(b, lane, 1, xh[1], xl[1]);
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
                tma_store_2d(&tmY8, b, (int32_t)col0, (int32_t)row0);
                tma_store_2d(&tmY8, b + 2048, (int32_t)(e.y8_half + col0), (int32_t)row0);
                bulk_commit();
            }
        };
        int acc = 0;
        uint32_t aph = 0;
        // NORM: the old residual of this warp's 32 rows of a tile, prefetched into L2 one tile
        // ahead (the epilogue then reads it from L2 instead of waiting on DRAM box by box).
        auto prefetch_tile = [&](int64_t tt) {
            if (!NORM || lane != 0 || tt >= tiles) return;
            const int64_t r0 = (tt / n_tiles) * kRows + rank * kBM + eg * 32;
            if (r0 >= e.M) return;
            const int64_t c0 = (tt % n_tiles) * BN;
#pragma unroll 1
            for (int c = 0; c < BN; c += 32) tma_prefetch_l2_2d(&tmY, (int32_t)(c0 + c), (int32_t)r0);
        };
        prefetch_tile(unit);
        for (int64_t t = unit; t < tiles; t += units) {
            prefetch_tile(t + units);
            const int64_t mrow0 = (t / n_tiles) * kRows + rank * kBM;  // this CTA's first row of the tile
            const int64_t row = mrow0 + r_in_tile;
            const int64_t wrow0 = mrow0 + eg * 32;  // first row of this warp's box
            const int64_t ncol0 = (t % n_tiles) * BN;
            const bool row_ok = row < e.M;
            // RoPE: the row's cos / sin (same for every head) load once per tile, before the wait
            // for the accumulator, so their latency hides behind the main loop.
            const bool rope_tile = e.rope_cos != nullptr && ncol0 < e.rope_cols && row_ok;
            float rc[32], rs[32];
            if (rope_tile) {
                const int64_t pidx = e.rope_p1 > 0 ? (row / e.rope_p1) * e.rope_p2 + row % e.rope_p2 : row % e.rope_p2;
                const float4 *cs = reinterpret_cast<const float4 *>(e.rope_cos + pidx * 32);
                const float4 *sn = reinterpret_cast<const float4 *>(e.rope_sin + pidx * 32);
#pragma unroll
                for (int q = 0; q < 8; ++q) {
                    const float4 c4 = __ldg(cs + q), s4 = __ldg(sn + q);
                    rc[4 * q] = c4.x;
                    rc[4 * q + 1] = c4.y;
                    rc[4 * q + 2] = c4.z;
                    rc[4 * q + 3] = c4.w;
                    rs[4 * q] = s4.x;
                    rs[4 * q + 1] = s4.y;
                    rs[4 * q + 2] = s4.z;
                    rs[4 * q + 3] = s4.w;
                }
            }
            // Fused RMSNorm factors of this thread's row (loads issued before the accumulator wait).
            // rsc: the row's factor applied to the accumulator (corrected products: times 2^-s).
            float rsc = e.acc_scale, xs = 1.0f;
            if (e.nin != nullptr) {
                if (row_ok) {
                    float sum = 0.0f;
                    for (int p = 0; p < e.nparts; ++p) sum += e.nin[(int64_t)p * e.M + row];
                    const float rs = 1.0f / sqrtf(sum / e.ndim + e.neps);
                    rsc = (e.ns_in ? rs / e.ns_in[row] : rs) * e.acc_scale;
                    xs = rs;
                    if (e.ns_out && ncol0 == 0) e.ns_out[row] = rs;
                }
            } else if (NORM && e.ns_in != nullptr && row_ok) {
                xs = e.ns_in[row];
            }
            // NORM: the old residual of the tile's first 32-column box, read in row-contiguous
            // order (lane -> row wrow0 + 4 i + lane / 8, columns 4 (lane % 8) .. + 3).
            float4 old_nxt[8];
            auto load_old = [&](int64_t col0) {
                const float *yb = reinterpret_cast<const float *>(e.out);
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    const int64_t gr = wrow0 + 4 * i + (lane >> 3);
                    old_nxt[i] = gr < e.M ? *reinterpret_cast<const float4 *>(yb + gr * e.ldo + col0 + 4 * (lane & 7))
                                          : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
                }
            };
            if constexpr (NORM) load_old(ncol0);
            // Warp-uniform wait: every lane polls the barrier, and the warp leaves together if any
            // lane gave up, so the .sync.aligned TMEM loads below always run converged.
            const bool got = PAIR ? mbar_wait_cl(&tfull[acc], aph, abort_flag, e.err, ERR_SITE_GEMM_EPILOGUE)
                                  : mbar_wait(&tfull[acc], aph, abort_flag, e.err, ERR_SITE_GEMM_EPILOGUE);
            if (!__all_sync(0xffffffffu, got)) break;
            tc_fence_after();
            const int64_t orow = e.rm_g > 0 ? (row / e.rm_g) * e.rm_G + row % e.rm_g + e.rm_off : row;
            const uint32_t tbase = tmem_base + ((uint32_t)(eg * 32) << 16) + (uint32_t)(acc * BN);
            if constexpr (NORM) {
                // Residual with the next RMSNorm's inputs: per 32-column box, the old values pass
                // through the staging box (row-contiguous global reads -> one row per thread), the
                // new values leave by TMA store, and the scaled 16-bit copy passes through this
                // warp's 2 KB box (64-byte rows, 16-byte chunks swizzled by (row / 2) % 4) to
                // row-contiguous global stores.
                uint8_t *xst = sStage + 4 * 2 * 4096 + eg * 2048;
                float ss = 0.0f;
#pragma unroll 1
                for (int c = 0; c < BN; c += 32) {
                    const int64_t col0 = ncol0 + c;
                    float4 cur[8];
#pragma unroll
                    for (int i = 0; i < 8; ++i) cur[i] = old_nxt[i];
                    if (c + 32 < BN) load_old(col0 + 32);
                    float v[32];
                    tmem_ld32(tbase + c, v);
                    uint8_t *b = stage_box();
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        const int rr = 4 * i + (lane >> 3), q = lane & 7;
                        *reinterpret_cast<float4 *>(b + rr * 128 + ((q ^ (rr & 7)) << 4)) = cur[i];
                    }
                    tmem_wait_ld();
                    __syncwarp();
#pragma unroll
                    for (int q = 0; q < 8; ++q) {
                        const float4 o = *reinterpret_cast<const float4 *>(b + lane * 128 + ((q ^ (lane & 7)) << 4));
                        v[4 * q] = v[4 * q] * rsc;
                        v[4 * q + 1] = v[4 * q + 1] * rsc;
                        v[4 * q + 2] = v[4 * q + 2] * rsc;
                        v[4 * q + 3] = v[4 * q + 3] * rsc;
                        if (e.bias) {
                            v[4 * q] += __ldg(e.bias + col0 + 4 * q);
                            v[4 * q + 1] += __ldg(e.bias + col0 + 4 * q + 1);
                            v[4 * q + 2] += __ldg(e.bias + col0 + 4 * q + 2);
                            v[4 * q + 3] += __ldg(e.bias + col0 + 4 * q + 3);
                        }
                        v[4 * q] += o.x;
                        v[4 * q + 1] += o.y;
                        v[4 * q + 2] += o.z;
                        v[4 * q + 3] += o.w;
                    }
                    __syncwarp();
#pragma unroll
                    for (int j = 0; j < 32; ++j) ss = fmaf(v[j], v[j], ss);
#pragma unroll
                    for (int q = 0; q < 8; ++q) put16(b, q, make_uint4(__float_as_uint(v[4 * q]), __float_as_uint(v[4 * q + 1]),
                                                                        __float_as_uint(v[4 * q + 2]), __float_as_uint(v[4 * q + 3])));
                    issue_box(b, col0, wrow0);
                    // 16-bit copy for the next GEMM: y * xs * gamma (and its FP8 companion).
                    float nv[32];
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        const float4 g0 = __ldg(reinterpret_cast<const float4 *>(e.ngamma + col0 + 8 * q));
                        const float4 g1 = __ldg(reinterpret_cast<const float4 *>(e.ngamma + col0 + 8 * q + 4));
                        const float *src = v + 8 * q;
                        const float a0 = src[0] * xs * g0.x, a1 = src[1] * xs * g0.y, a2 = src[2] * xs * g0.z,
                                    a3 = src[3] * xs * g0.w, a4 = src[4] * xs * g1.x, a5 = src[5] * xs * g1.y,
                                    a6 = src[6] * xs * g1.z, a7 = src[7] * xs * g1.w;
                        nv[8 * q] = a0;
                        nv[8 * q + 1] = a1;
                        nv[8 * q + 2] = a2;
                        nv[8 * q + 3] = a3;
                        nv[8 * q + 4] = a4;
                        nv[8 * q + 5] = a5;
                        nv[8 * q + 6] = a6;
                        nv[8 * q + 7] = a7;
                        uint4 pk;
                        pk.x = pack2<T>(a0, a1);
                        pk.y = pack2<T>(a2, a3);
                        pk.z = pack2<T>(a4, a5);
                        pk.w = pack2<T>(a6, a7);
                        *reinterpret_cast<uint4 *>(xst + lane * 64 + ((q ^ ((lane >> 1) & 3)) << 4)) = pk;
                    }
                    if (CORR_OUT && e.nx8 != nullptr && row_ok) store_x8_32(e.nx8 + row * e.ldnx8, e.nx8_half, col0, nv);
                    __syncwarp();
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        const int rr = 8 * i + (lane >> 2), q = lane & 3;
                        const uint4 pk = *reinterpret_cast<const uint4 *>(xst + rr * 64 + ((q ^ ((rr >> 1) & 3)) << 4));
                        const int64_t gr = wrow0 + rr;
                        if (gr < e.M)
                            *reinterpret_cast<uint4 *>(reinterpret_cast<T *>(e.nx16) + gr * e.ldx16 + col0 + 8 * q) = pk;
                    }
                    __syncwarp();
                }
                if (row_ok) e.nout[(ncol0 / BN) * e.M + row] = ss;
            } else if (BN == 256 && e.act == ACT_GLU) {
                // Gated pairs: the tile's columns are [g (128) | u (128)]; output column
                // (tile * 128 + c) = g[c] * silu(u[c]), staged and stored in 64-column boxes. The
                // logistic uses the fast exponential and division intrinsics (a few ulp; the result
                // is rounded to 16 bits), so the epilogue keeps pace with the main loop.
#pragma unroll 1
                for (int c = 0; c < 128; c += 64) {
                    uint8_t *b = stage_box();
                    const bool f16 = e.out_mode == OUT_F16;
                    uint32_t x8h[2][8], x8l[2][8];  // companion bytes of the 64 columns (y8_tma)
#pragma unroll
                    for (int h = 0; h < 64; h += 32) {
                        float g[32], u[32];
                        tmem_ld32(tbase + c + h, g);
                        tmem_ld32(tbase + 128 + c + h, u);
                        tmem_wait_ld();
                        if (rsc != 1.0f) {
#pragma unroll
                            for (int j = 0; j < 32; ++j) {
                                g[j] *= rsc;
                                u[j] *= rsc;
                            }
                        }
#pragma unroll
                        for (int j = 0; j < 32; ++j) g[j] = g[j] * __fdividef(u[j], 1.0f + __expf(-u[j]));
                        if (CORR_OUT && e.y8 != nullptr) {
                            if (e.y8_tma)
                                pack_x8_32(g, x8h[h / 32], x8l[h / 32]);
                            else if (row_ok)
                                store_x8_32(e.y8 + orow * e.ldy8, e.y8_half, ncol0 / 2 + c + h, g);
                        }
#pragma unroll
                        for (int q = 0; q < 4; ++q) {
                            const float *src = g + 8 * q;
                            uint4 pk;
                            pk.x = f16 ? pack2<__half>(src[0], src[1]) : pack2<__nv_bfloat16>(src[0], src[1]);
                            pk.y = f16 ? pack2<__half>(src[2], src[3]) : pack2<__nv_bfloat16>(src[2], src[3]);
                            pk.z = f16 ? pack2<__half>(src[4], src[5]) : pack2<__nv_bfloat16>(src[4], src[5]);
                            pk.w = f16 ? pack2<__half>(src[6], src[7]) : pack2<__nv_bfloat16>(src[6], src[7]);
                            put16(b, h / 8 + q, pk);
                        }
                    }
                    issue_box(b, ncol0 / 2 + c, wrow0);
                    if (CORR_OUT && e.y8 != nullptr && e.y8_tma) stage_issue_x8(ncol0 / 2 + c, wrow0, x8h, x8l);
                }
            } else if (e.rope_cos != nullptr || (e.tma_mode != 0 && !f32_out)) {
                // 64-column chunks (one head for RoPE): rotate-half pairs (i, i + 32) of columns
                // < rope_cols.
#pragma unroll 1
                for (int c = 0; c < BN; c += 64) {
                    const int64_t col0 = ncol0 + c;
                    if (col0 >= e.N) break;
                    float lo[32], hi[32];
                    tmem_ld32(tbase + c, lo);
                    tmem_ld32(tbase + c + 32, hi);
                    tmem_wait_ld();
                    if (rsc != 1.0f) {
#pragma unroll
                        for (int j = 0; j < 32; ++j) {
                            lo[j] *= rsc;
                            hi[j] *= rsc;
                        }
                    }
                    if (rope_tile && col0 < e.rope_cols) {
#pragma unroll
                        for (int j = 0; j < 32; ++j) {
                            const float x1 = lo[j], x2 = hi[j];
                            lo[j] = x1 * rc[j] - x2 * rs[j];
                            hi[j] = x2 * rc[j] + x1 * rs[j];
                        }
                    }
                    const int64_t rem0 = e.N - col0;
                    const int nv0 = rem0 < 32 ? (int)rem0 : 32;
                    const int64_t rem1 = e.N - col0 - 32;
                    const int nv1 = rem1 <= 0 ? 0 : (rem1 < 32 ? (int)rem1 : 32);
                    bias_act(e, col0, nv0, lo);
                    if (nv1 > 0) bias_act(e, col0 + 32, nv1, hi);
                    const bool x8_direct = CORR_OUT && e.y8 != nullptr && !e.y8_tma;
                    if (x8_direct && row_ok) {  // 16-bit output, N % 64 == 0
                        uint8_t *r8 = e.y8 + orow * e.ldy8;
                        store_x8_32(r8, e.y8_half, col0, lo);
                        store_x8_32(r8, e.y8_half, col0 + 32, hi);
                    }
                    if (e.tma_mode != 0) {
                        if (f32_out) {
                            tma_f32(col0, wrow0, lo);
                            if (nv1 > 0) tma_f32(col0 + 32, wrow0, hi);
                        } else {
                            tma_16(col0, wrow0, lo, hi);
                            if (CORR_OUT && e.y8 != nullptr && e.y8_tma) {
                                uint32_t x8h[2][8], x8l[2][8];
                                pack_x8_32(lo, x8h[0], x8l[0]);
                                pack_x8_32(hi, x8h[1], x8l[1]);
                                stage_issue_x8(col0, wrow0, x8h, x8l);
                            }
                        }
                    } else if (row_ok) {
                        store_chunk(e, orow, col0, nv0, lo);
                        if (nv1 > 0) store_chunk(e, orow, col0 + 32, nv1, hi);
                    }
                }
            } else {
#pragma unroll 1
                for (int c = 0; c < BN; c += 32) {
                    const int64_t col0 = ncol0 + c;
                    if (col0 >= e.N) break;
                    float v[32];
                    tmem_ld32(tbase + c, v);
                    tmem_wait_ld();
                    if (rsc != 1.0f) {
#pragma unroll
                        for (int j = 0; j < 32; ++j) v[j] *= rsc;
                    }
                    const int64_t rem = e.N - col0;
                    const int nv = rem < 32 ? (int)rem : 32;
                    bias_act(e, col0, nv, v);
                    if (CORR_OUT && e.y8 != nullptr && row_ok && !f32_out)
                        store_x8_32(e.y8 + orow * e.ldy8, e.y8_half, col0, v);
                    if (e.tma_mode != 0)
                        tma_f32(col0, wrow0, v);
                    else if (row_ok)
                        store_chunk(e, orow, col0, nv, v);
                }
            }
            tc_fence_before();
            if constexpr (PAIR)
                mbar_arrive_cluster(mapa_shared(&tempty[acc], 0));  // the MMA-issuing CTA's barrier
            else
                mbar_arrive(&tempty[acc]);
            if (++acc == 2) {
                acc = 0;
                aph ^= 1u;
            }
        }
        // Every staged box has been written (or reduced) before the CTA exits.
        if (e.tma_mode != 0 && lane == 0) bulk_wait_all();
    }

    __syncthreads();
    // A pair frees its tensor memory once both CTAs are done with it (the first CTA's MMAs have
    // drained and both epilogues have read their accumulators), and neither CTA exits while the
    // other could still reach its shared memory.
    if constexpr (PAIR) cluster_sync_all();
    if (warp == 1) {
        __syncwarp();
        tc_fence_after();
        if constexpr (PAIR)
            tmem_dealloc_pair(tmem_base, C::TMEM_COLS);
        else
            tmem_dealloc(tmem_base, C::TMEM_COLS);
    }
    if constexpr (PAIR) cluster_sync_all();
}

// ---- host side ------------------------------------------------------------------------------

PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::once_flag g_encode_once;
int g_num_sms[64] = {0};

bool load_encode() {
    std::call_once(g_encode_once, [] {
        void *fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    });
    return g_encode != nullptr;
}

Status make_tmap(CUtensorMap *map, const void *base, int dtype, int64_t inner, int64_t outer, int64_t ld,
                 uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_128B) {
    if (!load_encode()) return Status::fail(TSFM_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
    const bool f32 = dtype == E_F32;
    const int esz = f32 ? 4 : dtype == E_U8 ? 1 : 2;
    const CUtensorMapDataType dt = f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                   : dtype == E_U8 ? CU_TENSOR_MAP_DATA_TYPE_UINT8
                                   : dtype == E_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
    if ((reinterpret_cast<uintptr_t>(base) & 15) || ((ld * esz) & 15))
        return Status::fail(TSFM_ERR_INVALID_ARGUMENT, "linear: operand base and row stride must be 16-byte aligned");
    cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)outer};
    cuuint64_t strides[1] = {(cuuint64_t)(ld * esz)};
    cuuint32_t box[2] = {box_inner, box_outer};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = g_encode(map, dt, 2,
                          const_cast<void *>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                          swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return Status::fail(TSFM_ERR_CUDA, "cuTensorMapEncodeTiled failed (" + std::to_string((int)r) + ")");
    return Status::ok();
}

int sm_count() {
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return 148;
    if (g_num_sms[dev] == 0) {
        int n = 0;
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        g_num_sms[dev] = n > 0 ? n : 148;
    }
    return g_num_sms[dev];
}

}  // namespace

Status ensure_smem_attr(const void *func, int bytes) {
    // The attribute is a ceiling on the dynamic shared memory of every later launch of `func`, so
    // it only ever rises: a launch with more bytes than an earlier one raises it, one with fewer
    // leaves it.
    int dev = 0;
    cudaGetDevice(&dev);
    struct Entry {
        int dev;
        const void *func;
        int bytes;
    };
    static std::mutex mu;
    static std::vector<Entry> done;
    std::lock_guard<std::mutex> lk(mu);
    Entry *hit = nullptr;
    for (auto &d : done)
        if (d.dev == dev && d.func == func) hit = &d;
    if (hit && hit->bytes >= bytes) return Status::ok();
    const cudaError_t e = cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (e != cudaSuccess) return Status::cuda(e, "set dynamic shared memory");
    if (hit)
        hit->bytes = bytes;
    else
        done.push_back({dev, func, bytes});
    return Status::ok();
}

namespace {

template <typename T, int BN, bool PAIR, bool NORM = false, bool CORR = false>
Status launch_t(const LinearCall &c, cudaStream_t stream) {
    using C = TileCfg<BN, PAIR, NORM>;
    constexpr int BK = 128 / (int)sizeof(T);
    CUtensorMap ta, tb;
    Status s = make_tmap(&ta, c.x, c.dtype, c.K, c.M, c.ldx, BK, kBM);
    if (!s) return s;
    s = make_tmap(&tb, c.w, c.dtype, c.K, c.N, c.ldw, BK, C::B_ROWS);
    if (!s) return s;
    CUtensorMap ta8 = ta, tb8 = tb;  // unused unless CORR
    if constexpr (CORR) {
        const int64_t k8 = c.x8_cols > 0 ? c.x8_cols : 2 * c.K;
        TSFM_TRY(make_tmap(&ta8, c.x8, E_U8, k8, c.M, c.ldx8, 128, kBM));
        TSFM_TRY(make_tmap(&tb8, c.w8, E_U8, k8, c.N, c.ldw8, 128, C::B_ROWS));
    }
    TSFM_TRY(ensure_smem_attr(reinterpret_cast<const void *>(&linear_tc_kernel<T, BN, PAIR, NORM, CORR>), C::SMEM));
    cudaError_t ce;
    Epi e;
    e.M = c.M;
    e.N = c.N;
    e.K = c.K;
    e.out = c.y;
    e.ldo = c.ldy;
    e.bias = c.bias;
    e.act = c.act;
    e.out_mode = c.out_mode;
    e.rm_g = c.rm_g;
    e.rm_G = c.rm_G;
    e.rm_off = c.rm_off;
    e.rope_cos = c.rope_cos;
    e.rope_sin = c.rope_sin;
    e.rope_cols = c.rope_cols;
    e.rope_p1 = c.rope_p1;
    e.rope_p2 = c.rope_p2;
    e.err = c.err;
    e.nin = c.norm_in;
    e.nparts = c.norm_parts;
    e.ndim = (float)c.norm_dim;
    e.neps = c.norm_eps;
    e.ns_in = c.norm_s_in;
    e.ns_out = c.norm_s_out;
    e.nout = c.norm_out;
    e.nx16 = c.norm_x16;
    e.ldx16 = c.ld_x16;
    e.ngamma = c.norm_gamma;
    e.acc_scale = CORR ? c.acc_scale : 1.0f;
    e.K8 = c.x8_cols > 0 ? c.x8_cols : 2 * c.K;
    e.y8 = static_cast<uint8_t *>(c.y8);
    e.ldy8 = c.ldy8;
    e.y8_half = c.act == ACT_GLU ? c.N / 2 : c.N;
    e.nx8 = static_cast<uint8_t *>(c.norm_x8);
    e.ldnx8 = c.ld_nx8;
    e.nx8_half = c.N;
    // TMA epilogue unless rows are remapped or an activation follows the accumulation; the
    // output base and row stride must suit a tensor map (16-byte alignment).
    const bool f32_out = c.out_mode == OUT_F32 || c.out_mode == OUT_F32_ACC || c.out_mode == OUT_TF32;
    e.tma_mode = 0;
    CUtensorMap ty = tb;
    if (c.rm_g <= 0 && !(c.out_mode == OUT_F32_ACC && c.act != 0)) {
        const int ydt = f32_out ? E_F32 : c.out_mode == OUT_F16 ? E_F16 : E_BF16;
        const int64_t ycols = c.act == ACT_GLU ? c.N / 2 : c.N;
        if (make_tmap(&ty, c.y, ydt, ycols, c.M, c.ldy, f32_out ? 32 : 64, 32).code == 0)
            e.tma_mode = c.out_mode == OUT_F32_ACC ? 2 : 1;
    }
    if constexpr (NORM) {
        // The residual side reads the old rows itself and stores the new ones.
        if (e.tma_mode != 2) return Status::fail(TSFM_ERR_INVALID_ARGUMENT, "linear: fused norm needs an aligned f32 residual");
        e.tma_mode = 1;
    }
    if (c.act == ACT_GLU && e.tma_mode != 1)
        return Status::fail(TSFM_ERR_INVALID_ARGUMENT, "linear: gated pairs need a 16-byte-aligned 16-bit output");
    // The FP8 companion of a 16-bit output stored by TMA leaves by TMA too: bytes [M, 2 ycols] at
    // row stride ldy8, 64-byte x 32-row boxes in the 64-byte swizzle.
    CUtensorMap ty8 = tb;
    e.y8_tma = 0;
    if (c.y8 && e.tma_mode == 1 && !f32_out) {
        if (make_tmap(&ty8, c.y8, E_U8, 2 * e.y8_half, c.M, c.ldy8, 64, 32, CU_TENSOR_MAP_SWIZZLE_64B).code == 0)
            e.y8_tma = 1;
    }
    if constexpr (PAIR) {
        // Clusters of two CTAs, one per SM pair, persistent over 256-row tiles.
        const int64_t tiles = ((c.M + 2 * kBM - 1) / (2 * kBM)) * ((c.N + BN - 1) / BN);
        const int grid = 2 * (int)std::min<int64_t>(tiles, sm_count() / 2);
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3((unsigned)grid);
        cfg.blockDim = dim3(kThreads);
        cfg.dynamicSmemBytes = C::SMEM;
        cfg.stream = stream;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = 2;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        ce = cudaLaunchKernelEx(&cfg, linear_tc_kernel<T, BN, true, NORM, CORR>, ta, tb, ty, ta8, tb8, ty8, e);
        if (ce != cudaSuccess) return Status::cuda(ce, "linear: launch (CTA pairs)");
    } else {
        const int64_t tiles = ((c.M + kBM - 1) / kBM) * ((c.N + BN - 1) / BN);
        const int grid = (int)std::min<int64_t>(tiles, sm_count());
        linear_tc_kernel<T, BN, false, NORM, CORR><<<grid, kThreads, C::SMEM, stream>>>(ta, tb, ty, ta8, tb8, ty8, e);
    }
    ce = cudaGetLastError();
    if (ce != cudaSuccess) return Status::cuda(ce, "linear: launch");
    return Status::ok();
}

}  // namespace

int num_sms() { return sm_count(); }

Status make_tmap_2d(void *map, const void *base, int dtype, int64_t inner, int64_t outer, int64_t ld,
                    uint32_t box_inner, uint32_t box_outer) {
    return make_tmap(static_cast<CUtensorMap *>(map), base, dtype, inner, outer, ld, box_inner, box_outer);
}

Status make_tmap_grouped_rows(void *map, const void *base, int dtype, int64_t width, int64_t rows, int64_t groups,
                              int64_t ld, uint32_t box_inner, uint32_t box_rows) {
    if (!load_encode()) return Status::fail(TSFM_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
    const bool f32 = dtype == E_F32;
    const int esz = f32 ? 4 : 2;
    const CUtensorMapDataType dt = f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                       : dtype == E_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
    if ((reinterpret_cast<uintptr_t>(base) & 15) || ((ld * esz) & 15))
        return Status::fail(TSFM_ERR_INVALID_ARGUMENT, "tensor map: base and row stride must be 16-byte aligned");
    cuuint64_t dims[3] = {(cuuint64_t)width, (cuuint64_t)rows, (cuuint64_t)groups};
    cuuint64_t strides[2] = {(cuuint64_t)(ld * esz), (cuuint64_t)(rows * ld * esz)};
    cuuint32_t box[3] = {box_inner, box_rows, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = g_encode(static_cast<CUtensorMap *>(map), dt, 3, const_cast<void *>(base), dims, strides, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return Status::fail(TSFM_ERR_CUDA, "cuTensorMapEncodeTiled failed (" + std::to_string((int)r) + ")");
    return Status::ok();
}

// TSFM_GEMM_PAIRS=0 keeps every product on single-CTA tiles.
static bool gemm_pairs_enabled() {
    static const bool on = [] {
        const char *v = std::getenv("TSFM_GEMM_PAIRS");
        return !(v && v[0] == '0');
    }();
    return on;
}

Status launch_linear(const LinearCall &c, cudaStream_t stream) {
    if (c.M <= 0 || c.N <= 0 || c.K <= 0) return Status::fail(TSFM_ERR_INVALID_ARGUMENT, "linear: empty product");
    if (c.M > INT32_MAX || c.N > INT32_MAX || c.K > INT32_MAX)
        return Status::fail(TSFM_ERR_INVALID_ARGUMENT, "linear: dimension exceeds the TMA coordinate range");
    if (c.out_mode < OUT_BF16 || c.out_mode > OUT_F16) return Status::fail(TSFM_ERR_INVALID_ARGUMENT, "linear: bad out_mode");
    if (c.rope_cos && (c.out_mode == OUT_F32_ACC || c.rope_cols % 64))
        return Status::fail(TSFM_ERR_INVALID_ARGUMENT, "linear: bad rope");
    if (c.act == ACT_GLU && (c.N % 256 || (c.out_mode != OUT_F16 && c.out_mode != OUT_BF16) || c.bias || c.rm_g > 0 ||
                             c.rope_cos || c.dtype == E_F32))
        return Status::fail(TSFM_ERR_INVALID_ARGUMENT, "linear: gated pairs need N % 256 == 0, 16-bit operands and output");
    if (c.norm_in && (c.norm_parts <= 0 || c.norm_dim <= 0 || c.act == ACT_GLU || c.norm_s_in == c.norm_s_out))
        return Status::fail(TSFM_ERR_INVALID_ARGUMENT, "linear: bad fused-norm reader arguments");
    const auto a16 = [](const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
    const bool corr = c.x8 != nullptr;
    if (corr && (c.dtype != E_F16 || !c.w8 || c.K % 8 || c.ldx8 % 16 || c.ldw8 % 16 || c.ldx8 < 2 * c.K ||
                 c.ldw8 < 2 * c.K || !a16(c.x8) || !a16(c.w8) || !(c.acc_scale > 0.0f) ||
                 (c.x8_cols != 0 && c.x8_cols != c.K && c.x8_cols != 2 * c.K)))
        return Status::fail(TSFM_ERR_INVALID_ARGUMENT,
                            "linear: corrected products need FP16 operands, K % 8 == 0 and 16-byte-aligned FP8 companions");
    if (c.y8) {
        const int64_t ycols = c.act == ACT_GLU ? c.N / 2 : c.N;
        if (c.out_mode != OUT_F16 || ycols % 64 || c.ldy8 % 16 || c.ldy8 < 2 * ycols || !a16(c.y8) ||
            c.dtype == E_BF16)
            return Status::fail(TSFM_ERR_INVALID_ARGUMENT,
                                "linear: an FP8 companion output needs an FP16 output of a multiple of 64 columns");
    }
    if (c.norm_x8 && (!c.norm_out || c.dtype != E_F16 || c.ld_nx8 % 16 || c.ld_nx8 < 2 * c.N || !a16(c.norm_x8)))
        return Status::fail(TSFM_ERR_INVALID_ARGUMENT, "linear: bad FP8 companion of the fused norm");
    if (c.norm_out) {
        const bool ok = (c.dtype == E_F16 || c.dtype == E_BF16) && c.out_mode == OUT_F32_ACC && c.N % 256 == 0 &&
                        c.act == 0 && c.rm_g <= 0 && !c.rope_cos && c.norm_x16 && c.norm_gamma && c.ld_x16 >= c.N &&
                        c.ld_x16 % 8 == 0 && (reinterpret_cast<uintptr_t>(c.norm_x16) & 15) == 0 &&
                        (reinterpret_cast<uintptr_t>(c.norm_gamma) & 15) == 0 && c.norm_x16 != c.x &&
                        (c.norm_in || c.norm_s_in);
        if (!ok) return Status::fail(TSFM_ERR_INVALID_ARGUMENT, "linear: bad fused-norm residual arguments");
        const bool pair = c.M >= 4096 && gemm_pairs_enabled();
        if (corr)
            return pair ? launch_t<__half, 256, true, true, true>(c, stream)
                        : launch_t<__half, 256, false, true, true>(c, stream);
        if (c.dtype == E_F16)
            return pair ? launch_t<__half, 256, true, true>(c, stream) : launch_t<__half, 256, false, true>(c, stream);
        return pair ? launch_t<__nv_bfloat16, 256, true, true>(c, stream)
                    : launch_t<__nv_bfloat16, 256, false, true>(c, stream);
    }
    const bool small_n = c.N <= 128;
    // Large 16-bit products run on CTA pairs (2-SM MMA, 256 x 256 tiles): each SM then streams half
    // of W's tile instead of all of it.
    const bool pair = !small_n && c.M >= 4096 && gemm_pairs_enabled();
    if (corr)
        return small_n ? launch_t<__half, 128, false, false, true>(c, stream)
                       : pair ? launch_t<__half, 256, true, false, true>(c, stream)
                              : launch_t<__half, 256, false, false, true>(c, stream);
    switch (c.dtype) {
        case E_F32: return small_n ? launch_t<float, 128, false>(c, stream) : launch_t<float, 256, false>(c, stream);
        case E_F16:
            return small_n ? launch_t<__half, 128, false>(c, stream)
                           : pair ? launch_t<__half, 256, true>(c, stream) : launch_t<__half, 256, false>(c, stream);
        case E_BF16:
            return small_n ? launch_t<__nv_bfloat16, 128, false>(c, stream)
                           : pair ? launch_t<__nv_bfloat16, 256, true>(c, stream)
                                  : launch_t<__nv_bfloat16, 256, false>(c, stream);
        default: return Status::fail(TSFM_ERR_UNSUPPORTED_DTYPE, "linear: operand type");
    }
}

}  // namespace tsfm
