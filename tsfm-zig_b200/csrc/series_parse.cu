// Series CSV input on the GPU: the reference reader's parseBlocks (core/series.zig:21-68) and
// toF32 (core/series.zig:78-82).
//
// The text is split at '\n'; each line is trimmed of " \t\r"; lines starting with '#' are
// skipped; an empty line closes the current block; a data line holds comma-separated tokens
// when it contains a comma (empty tokens allowed), else tokens separated by runs of spaces /
// tabs. Every token is trimmed and parsed as f64 (NaN when empty or not a number). All data
// lines hold the same token count (error.RaggedInput) and all blocks the same line count
// (error.RaggedBlocks); no data at all is error.EmptyInput. Values come out as
// (blocks, rows, len) in line order.
//
// Device work is per byte, per line and per token: (1) newline positions by a count / scan /
// compaction over 4 KiB tiles; (2) one warp per line finds its trimmed bounds, its kind (empty,
// comment, data), whether it has a comma and its token count; (3) the host walks the lines'
// kinds and counts in order (O(lines), the reference's control flow and error order) and
// assigns each data line its output row; (4) one warp per data line writes its tokens' bounds;
// (5) one thread per token parses it (parse_number.cuh).
#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/tsfm_b200.h"
#include "kernels.h"
#include "parse_number.cuh"

namespace tsfm {
int32_t set_last_error(const Status &s);

namespace {

constexpr int kTile = 4096;  // bytes per block of the newline kernels (256 threads x 16 bytes)

__device__ __forceinline__ bool is_trim(char c) { return c == ' ' || c == '\t' || c == '\r'; }
__device__ __forceinline__ bool is_sep(char c) { return c == ' ' || c == '\t'; }

// Lines are read 16 bytes per lane (one aligned 16-byte chunk each, 512 bytes per warp step).
// Chunk k covers text positions [16k - mis, 16k - mis + 16), mis = the text pointer's offset in
// its 16-byte granule; a chunk inside [0, n) is one vector load, an edge chunk is read byte by
// byte (only its in-range bytes).
struct Chunk {
    uint32_t w[4];
    __device__ __forceinline__ char at(int j) const { return (char)((w[j >> 2] >> (8 * (j & 3))) & 0xff); }
};

__device__ __forceinline__ Chunk load_chunk(const char *text, int64_t n, int mis, int64_t k) {
    Chunk c;
    const int64_t q0 = k * 16 - mis;
    if (q0 >= 0 && q0 + 16 <= n) {
        const uint4 v = *reinterpret_cast<const uint4 *>(text + q0);
        c.w[0] = v.x, c.w[1] = v.y, c.w[2] = v.z, c.w[3] = v.w;
    } else {
        c.w[0] = c.w[1] = c.w[2] = c.w[3] = 0x20202020u;  // spaces
#pragma unroll
        for (int j = 0; j < 16; ++j)
            if (q0 + j >= 0 && q0 + j < n) c.w[j >> 2] = (c.w[j >> 2] & ~(0xffu << (8 * (j & 3)))) |
                                                         ((uint32_t)(uint8_t)text[q0 + j] << (8 * (j & 3)));
    }
    return c;
}

__device__ __forceinline__ uint32_t newline_mask(const Chunk &c, int64_t q0, int64_t n) {
    uint32_t m = 0;
#pragma unroll
    for (int j = 0; j < 16; ++j) m |= (q0 + j >= 0 && q0 + j < n && c.at(j) == '\n') ? (1u << j) : 0u;
    return m;
}

// (1a) newlines per tile (tile t = aligned chunks [256 t, 256 t + 256)).
__global__ void __launch_bounds__(256) nl_count_kernel(const char *text, int64_t n, uint32_t *tile_count) {
    const int mis = (int)(reinterpret_cast<uintptr_t>(text) & 15);
    const int64_t k = (int64_t)blockIdx.x * 256 + threadIdx.x;
    uint32_t c = __popc(newline_mask(load_chunk(text, n, mis, k), k * 16 - mis, n));
    for (int o = 16; o > 0; o >>= 1) c += __shfl_xor_sync(0xffffffffu, c, o);
    __shared__ uint32_t ws[8];
    if ((threadIdx.x & 31) == 0) ws[threadIdx.x >> 5] = c;
    __syncthreads();
    if (threadIdx.x == 0) {
        uint32_t t = 0;
        for (int w = 0; w < 8; ++w) t += ws[w];
        tile_count[blockIdx.x] = t;
    }
}

// (1b) exclusive scan of the tile counts (one block of 1024 threads); total into *total.
__global__ void __launch_bounds__(1024) scan_u32_kernel(const uint32_t *in, int64_t n, uint64_t *excl, uint64_t *total) {
    __shared__ uint64_t wtot[32];
    __shared__ uint64_t carry;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (threadIdx.x == 0) carry = 0;
    __syncthreads();
    for (int64_t base = 0; base < n; base += 1024) {
        const int64_t i = base + threadIdx.x;
        const uint64_t v = i < n ? in[i] : 0;
        uint64_t x = v;
        for (int o = 1; o < 32; o <<= 1) {
            const uint64_t y = __shfl_up_sync(0xffffffffu, x, o);
            if (lane >= o) x += y;
        }
        if (lane == 31) wtot[warp] = x;
        __syncthreads();
        if (warp == 0) {
            uint64_t w = wtot[lane];
            for (int o = 1; o < 32; o <<= 1) {
                const uint64_t y = __shfl_up_sync(0xffffffffu, w, o);
                if (lane >= o) w += y;
            }
            wtot[lane] = w;
        }
        __syncthreads();
        const uint64_t before = carry + (warp ? wtot[warp - 1] : 0);
        if (i < n) excl[i] = before + x - v;
        __syncthreads();
        if (threadIdx.x == 1023) carry = before + x;
        __syncthreads();
    }
    if (threadIdx.x == 0) *total = carry;
}

// (1c) newline positions, in order.
__global__ void __launch_bounds__(256) nl_pos_kernel(const char *text, int64_t n, const uint64_t *tile_off,
                                                    uint64_t *pos) {
    const int mis = (int)(reinterpret_cast<uintptr_t>(text) & 15);
    const int64_t k = (int64_t)blockIdx.x * 256 + threadIdx.x, q0 = k * 16 - mis;
    uint32_t m = newline_mask(load_chunk(text, n, mis, k), q0, n);
    const uint32_t c = __popc(m);
    // exclusive block scan of c
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    uint32_t x = c;
    for (int o = 1; o < 32; o <<= 1) {
        const uint32_t y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
    }
    __shared__ uint32_t ws[8];
    if (lane == 31) ws[warp] = x;
    __syncthreads();
    uint32_t before = 0;
    for (int w = 0; w < warp; ++w) before += ws[w];
    uint64_t at = tile_off[blockIdx.x] + before + x - c;
    while (m) {
        const int j = __ffs(m) - 1;
        m &= m - 1;
        pos[at++] = (uint64_t)(q0 + j);
    }
}

struct LineInfo {
    uint64_t a, b;     // trimmed bounds
    uint32_t tokens;   // data lines: token count
    uint8_t kind;      // 0 empty, 1 comment, 2 data
    uint8_t comma;     // data lines: comma-separated
};

__device__ __forceinline__ void line_span(const uint64_t *nl, int64_t n_nl, int64_t total, int64_t line, uint64_t *s,
                                          uint64_t *e) {
    *s = line == 0 ? 0 : nl[line - 1] + 1;
    *e = line < n_nl ? nl[line] : (uint64_t)total;
}

template <class T>
__device__ __forceinline__ T warp_excl_scan(T v, T *total) {
    const int lane = threadIdx.x & 31;
    T x = v;
    for (int o = 1; o < 32; o <<= 1) {
        const T y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
    }
    *total = __shfl_sync(0xffffffffu, x, 31);
    return x - v;
}

// (2) one warp per line: trimmed bounds, kind, separator, token count.
__global__ void __launch_bounds__(256) line_kernel(const char *text, int64_t total, const uint64_t *nl, int64_t n_nl,
                                                  LineInfo *info, uint32_t *meta) {
    const int lane = threadIdx.x & 31;
    const int64_t line = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    if (line > n_nl) return;
    const int mis = (int)(reinterpret_cast<uintptr_t>(text) & 15);
    uint64_t s, e;
    line_span(nl, n_nl, total, line, &s, &e);
    const int64_t k_first = ((int64_t)s + mis) >> 4, k_last = ((int64_t)e - 1 + mis) >> 4;
    // First byte that is not " \t\r".
    int64_t a = (int64_t)e;
    for (int64_t w = k_first; s < e && w <= k_last; w += 32) {
        const int64_t k = w + lane;
        int64_t mine = INT64_MAX;
        if (k <= k_last) {
            const Chunk c = load_chunk(text, total, mis, k);
#pragma unroll
            for (int j = 15; j >= 0; --j) {
                const int64_t q = k * 16 + j - mis;
                if (q >= (int64_t)s && q < (int64_t)e && !is_trim(c.at(j))) mine = q;
            }
        }
        for (int o = 16; o > 0; o >>= 1) mine = min(mine, (int64_t)__shfl_xor_sync(0xffffffffu, (long long)mine, o));
        if (mine != INT64_MAX) {
            a = mine;
            break;
        }
    }
    // Last such byte (scanning back from the end).
    int64_t b = a;
    if (a < (int64_t)e) {
        const int64_t k_a = (a + mis) >> 4;
        for (int64_t w = k_last; w >= k_a; w -= 32) {
            const int64_t k = w - lane;
            int64_t mine = -1;
            if (k >= k_a) {
                const Chunk c = load_chunk(text, total, mis, k);
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                    const int64_t q = k * 16 + j - mis;
                    if (q >= a && q < (int64_t)e && !is_trim(c.at(j))) mine = q;
                }
            }
            for (int o = 16; o > 0; o >>= 1) mine = max(mine, (int64_t)__shfl_xor_sync(0xffffffffu, (long long)mine, o));
            if (mine >= 0) {
                b = mine + 1;
                break;
            }
        }
    }
    LineInfo li{};
    li.a = (uint64_t)a;
    li.b = (uint64_t)b;
    if (a >= (int64_t)e) {
        li.kind = 0;
    } else if (text[a] == '#') {
        li.kind = 1;
    } else {
        li.kind = 2;
        // Commas, and starts of space / tab separated tokens, over [a, b).
        uint32_t commas = 0, starts = 0;
        char carry_last = ' ';  // byte before this step's first chunk
        const int64_t ka = (a + mis) >> 4, kb = (b - 1 + mis) >> 4;
        for (int64_t w = ka; w <= kb; w += 32) {
            const int64_t k = w + lane;
            Chunk c;
            if (k <= kb) {
                c = load_chunk(text, total, mis, k);
            } else {
                c.w[0] = c.w[1] = c.w[2] = c.w[3] = 0x20202020u;
            }
            const char last = c.at(15);
            char prev = __shfl_up_sync(0xffffffffu, last, 1);
            if (lane == 0) prev = carry_last;
            uint32_t cm = 0, st = 0;
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                const int64_t q = k * 16 + j - mis;
                const char ch = c.at(j);
                const bool in = q >= a && q < b;
                cm += (in && ch == ',') ? 1u : 0u;
                st += (in && !is_sep(ch) && (q == a || is_sep(prev))) ? 1u : 0u;
                prev = in ? ch : ' ';
            }
            for (int o = 16; o > 0; o >>= 1) {
                cm += __shfl_xor_sync(0xffffffffu, cm, o);
                st += __shfl_xor_sync(0xffffffffu, st, o);
            }
            commas += cm;
            starts += st;
            carry_last = __shfl_sync(0xffffffffu, last, 31);
        }
        li.comma = commas > 0;
        li.tokens = commas > 0 ? commas + 1 : starts;
    }
    if (lane == 0) {
        info[line] = li;
        // 2^30 - 1 tokens or more on one line saturate the count (the host reports it).
        meta[line] = ((uint32_t)li.kind << 30) | min(li.tokens, 0x3fffffffu);
    }
}

// (4) one warp per data line: each token's [start, end) (before trimming).
__global__ void __launch_bounds__(256) token_kernel(const char *text, int64_t total, const LineInfo *info,
                                                   const int64_t *data_lines, int64_t n_data, int64_t len,
                                                   uint64_t *tok_s, uint64_t *tok_e) {
    const int lane = threadIdx.x & 31;
    const int64_t d = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    if (d >= n_data) return;
    const int mis = (int)(reinterpret_cast<uintptr_t>(text) & 15);
    const LineInfo li = info[data_lines[d]];
    const int64_t a = (int64_t)li.a, b = (int64_t)li.b, base = d * len;
    const int64_t ka = (a + mis) >> 4, kb = (b - 1 + mis) >> 4;
    uint64_t k_tok = 0;  // tokens (comma mode: commas; space mode: starts) before this step
    char carry_last = ' ';
    if (li.comma && lane == 0) {
        tok_s[base] = (uint64_t)a;
        tok_e[base + len - 1] = (uint64_t)b;
    }
    for (int64_t w = ka; w <= kb; w += 32) {
        const int64_t k = w + lane;
        Chunk c;
        if (k <= kb) {
            c = load_chunk(text, total, mis, k);
        } else {
            c.w[0] = c.w[1] = c.w[2] = c.w[3] = 0x20202020u;
        }
        const char last = c.at(15);
        char prev = __shfl_up_sync(0xffffffffu, last, 1);
        if (lane == 0) prev = carry_last;
        char next = __shfl_down_sync(0xffffffffu, c.at(0), 1);
        if (lane == 31) next = (k + 1) * 16 - mis < b ? text[(k + 1) * 16 - mis] : ' ';
        uint32_t mine = 0;
        {
            char p = prev;
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                const int64_t q = k * 16 + j - mis;
                const char ch = c.at(j);
                const bool in = q >= a && q < b;
                if (li.comma) mine += (in && ch == ',') ? 1u : 0u;
                else mine += (in && !is_sep(ch) && (q == a || is_sep(p))) ? 1u : 0u;
                p = in ? ch : ' ';
            }
        }
        uint32_t step_total;
        const uint32_t before = warp_excl_scan(mine, &step_total);
        uint64_t idx = k_tok + before;
        char p = prev;
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            const int64_t q = k * 16 + j - mis;
            const char ch = c.at(j);
            const bool in = q >= a && q < b;
            if (li.comma) {
                if (in && ch == ',') {
                    tok_e[base + idx] = (uint64_t)q;
                    tok_s[base + idx + 1] = (uint64_t)q + 1;
                    ++idx;
                }
            } else if (in && !is_sep(ch)) {
                if (q == a || is_sep(p)) tok_s[base + idx++] = (uint64_t)q;
                const char nx = j < 15 ? c.at(j + 1) : next;
                if (q + 1 == b || is_sep(nx)) tok_e[base + idx - 1] = (uint64_t)q + 1;
            }
            p = in ? ch : ' ';
        }
        k_tok += step_total;
        carry_last = __shfl_sync(0xffffffffu, last, 31);
    }
}

__constant__ numparse::Recip10 c_recip;

constexpr int kStage = 16384;  // bytes of token text a block stages in shared memory

// (5) one thread per token: trim, parse, store f64 (and f32 when asked: @floatCast, nearest).
// A block's 256 tokens are consecutive in the text: their span is staged in shared memory with
// 16-byte loads when it fits, so each thread reads its token from there.
__global__ void __launch_bounds__(256) parse_kernel(const char *text, int64_t total, const uint64_t *tok_s,
                                                   const uint64_t *tok_e, int64_t n, double *out, float *out32) {
    __shared__ __align__(16) char stage[kStage + 32];
    __shared__ numparse::Recip10 recip;
    __shared__ int64_t span_lo, span_hi;
    const int64_t t0 = (int64_t)blockIdx.x * blockDim.x, t = t0 + threadIdx.x;
    const int64_t last = min(n, t0 + (int64_t)blockDim.x) - 1;
    for (int i = threadIdx.x; i < (int)(sizeof(recip) / 16); i += blockDim.x)
        reinterpret_cast<uint4 *>(&recip)[i] = reinterpret_cast<const uint4 *>(&c_recip)[i];
    if (threadIdx.x == 0) {
        span_lo = (int64_t)tok_s[t0];
        span_hi = (int64_t)tok_e[last];
    }
    __syncthreads();
    const int mis = (int)(reinterpret_cast<uintptr_t>(text) & 15);
    const int64_t lo = span_lo, hi = span_hi;
    // Aligned chunks covering [lo, hi): stage[0] holds text position (k_lo * 16 - mis).
    const int64_t k_lo = (lo + mis) >> 4, k_hi = (hi - 1 + mis) >> 4;
    const bool staged = hi > lo && (k_hi - k_lo + 1) * 16 <= kStage;
    if (staged) {
        for (int64_t k = k_lo + threadIdx.x; k <= k_hi; k += blockDim.x) {
            const Chunk c = load_chunk(text, total, mis, k);
            *reinterpret_cast<uint4 *>(stage + (k - k_lo) * 16) = make_uint4(c.w[0], c.w[1], c.w[2], c.w[3]);
        }
    }
    __syncthreads();
    if (t >= n) return;
    const int64_t origin = k_lo * 16 - mis;
    const char *src = staged ? stage - origin : text;  // src[q] is text position q
    int64_t a = (int64_t)tok_s[t], b = (int64_t)tok_e[t];
    while (a < b && is_trim(src[a])) ++a;
    while (b > a && is_trim(src[b - 1])) --b;
    double v;
    if (a == b || b - a > (1 << 20)) {
        v = numparse::quiet_nan(false);  // empty, or over a MiB (never a number the reader accepts)
    } else {
        v = numparse::parse_number(src + a, (int)(b - a), &recip);
    }
    if (out) out[t] = v;
    if (out32) out32[t] = (float)v;
}

// ---------------------------------------------------------------------------------------------
// Host side.

struct PCtx {
    std::mutex mu;
    bool ready = false;
    cudaStream_t stream = nullptr, copy = nullptr;
    cudaEvent_t ev[16] = {};
    char *d_text = nullptr;
    size_t text_cap = 0;
    uint32_t *d_tile = nullptr;
    size_t tile_cap = 0;
    uint64_t *d_tile_off = nullptr;
    size_t tile_off_cap = 0;
    uint64_t *d_total = nullptr;
    size_t total_cap = 0;
    uint64_t *h_total = nullptr;
    uint64_t *d_nl = nullptr;
    size_t nl_cap = 0;
    LineInfo *d_info = nullptr;
    size_t info_cap = 0;
    uint32_t *d_meta = nullptr;
    size_t meta_cap = 0;
    int64_t *d_data = nullptr;
    size_t data_cap = 0;
    uint64_t *d_ts = nullptr, *d_te = nullptr;
    size_t ts_cap = 0, te_cap = 0;
    double *d_vals = nullptr;
    size_t vals_cap = 0;
};

constexpr int kMaxDevices = 64;
PCtx g_pctx[kMaxDevices];

template <class T>
Status grow(T **p, size_t *cap, size_t bytes, const char *what) {
    bytes = std::max<size_t>(bytes, 16);
    if (*cap >= bytes) return Status::ok();
    if (*p) cudaFree(*p);
    *p = nullptr;
    *cap = 0;
    TSFM_CUDA(cudaMalloc(reinterpret_cast<void **>(p), bytes), what);
    *cap = bytes;
    return Status::ok();
}

Status pctx_init(PCtx &x, int device) {
    TSFM_CUDA(cudaSetDevice(device), "series: cudaSetDevice");
    if (x.ready) return Status::ok();
    TSFM_CUDA(cudaStreamCreateWithFlags(&x.stream, cudaStreamNonBlocking), "series: stream");
    TSFM_CUDA(cudaStreamCreateWithFlags(&x.copy, cudaStreamNonBlocking), "series: stream");
    for (cudaEvent_t &e : x.ev) TSFM_CUDA(cudaEventCreateWithFlags(&e, cudaEventDisableTiming), "series: event");
    TSFM_CUDA(cudaMallocHost(reinterpret_cast<void **>(&x.h_total), 16), "series: pinned total");
    const numparse::Recip10 r = numparse::make_recip10();
    TSFM_CUDA(cudaMemcpyToSymbol(c_recip, &r, sizeof r), "series: reciprocals");
    x.ready = true;
    return Status::ok();
}

struct Shape {
    size_t blocks = 0, rows = 0, len = 0;
    std::vector<int64_t> data_lines;
};

// Steps (1)-(3) over text[0, n) on the device: the shape and each data line's index, or the
// reference's error.
Status structure(PCtx &x, const char *text, int64_t n, cudaStream_t s, Shape &sh) {
    const int mis = (int)(reinterpret_cast<uintptr_t>(text) & 15);
    const int64_t tiles = std::max<int64_t>(1, (n + mis + kTile - 1) / kTile);
    TSFM_TRY(grow(&x.d_tile, &x.tile_cap, tiles * 4, "series: tiles"));
    TSFM_TRY(grow(&x.d_tile_off, &x.tile_off_cap, tiles * 8, "series: tiles"));
    TSFM_TRY(grow(&x.d_total, &x.total_cap, 16, "series: total"));
    nl_count_kernel<<<(unsigned)tiles, 256, 0, s>>>(text, n, x.d_tile);
    TSFM_CUDA(cudaGetLastError(), "series: newline count");
    scan_u32_kernel<<<1, 1024, 0, s>>>(x.d_tile, tiles, x.d_tile_off, x.d_total);
    TSFM_CUDA(cudaGetLastError(), "series: scan");
    TSFM_CUDA(cudaMemcpyAsync(x.h_total, x.d_total, 8, cudaMemcpyDeviceToHost, s), "series: total");
    TSFM_CUDA(cudaStreamSynchronize(s), "series: newline count");
    const int64_t n_nl = (int64_t)*x.h_total, lines = n_nl + 1;
    TSFM_TRY(grow(&x.d_nl, &x.nl_cap, (size_t)n_nl * 8, "series: newlines"));
    nl_pos_kernel<<<(unsigned)tiles, 256, 0, s>>>(text, n, x.d_tile_off, x.d_nl);
    TSFM_CUDA(cudaGetLastError(), "series: newline positions");
    TSFM_TRY(grow(&x.d_info, &x.info_cap, (size_t)lines * sizeof(LineInfo), "series: lines"));
    TSFM_TRY(grow(&x.d_meta, &x.meta_cap, (size_t)lines * 4, "series: lines"));
    const int64_t warps_per_block = 8;
    line_kernel<<<(unsigned)((lines + warps_per_block - 1) / warps_per_block), 256, 0, s>>>(text, n, x.d_nl, n_nl,
                                                                                         x.d_info, x.d_meta);
    TSFM_CUDA(cudaGetLastError(), "series: lines");
    std::vector<uint32_t> meta((size_t)lines);
    TSFM_CUDA(cudaMemcpyAsync(meta.data(), x.d_meta, (size_t)lines * 4, cudaMemcpyDeviceToHost, s), "series: lines");
    TSFM_CUDA(cudaStreamSynchronize(s), "series: lines");
    // parseBlocks' control flow (core/series.zig:32-66), on the lines' kinds and token counts.
    size_t blocks = 0, rows_in_block = 0, rows = 0, len = 0;
    bool have_len = false;
    auto close_block = [&]() -> Status {
        if (rows_in_block > 0) {
            if (blocks == 0) {
                rows = rows_in_block;
            } else if (rows_in_block != rows) {
                return Status::fail(TSFM_ERR_RAGGED_BLOCKS, "RaggedBlocks");
            }
            ++blocks;
            rows_in_block = 0;
        }
        return Status::ok();
    };
    sh.data_lines.clear();
    for (int64_t l = 0; l < lines; ++l) {
        const uint32_t kind = meta[(size_t)l] >> 30, tokens = meta[(size_t)l] & 0x3fffffffu;
        if (kind == 1) continue;
        if (kind == 0) {
            TSFM_TRY(close_block());
            continue;
        }
        if (tokens == 0x3fffffffu)
            return Status::fail(TSFM_ERR_UNSUPPORTED, "series: a line holds 2^30 - 1 or more values");
        if (!have_len) {
            len = tokens;
            have_len = true;
        } else if (tokens != len) {
            return Status::fail(TSFM_ERR_RAGGED_INPUT, "RaggedInput");
        }
        ++rows_in_block;
        sh.data_lines.push_back(l);
    }
    TSFM_TRY(close_block());
    if (blocks == 0 || len == 0) return Status::fail(TSFM_ERR_EMPTY_INPUT, "EmptyInput");
    sh.blocks = blocks;
    sh.rows = rows;
    sh.len = len;
    return Status::ok();
}

// Steps (4)-(5): values (f64 and / or f32, device) of the data lines.
// Steps (4)-(5). With host_out, the values are parsed in chunks and each chunk is copied to
// host_out on the copy stream while the next one is parsed.
Status tokens_and_values(PCtx &x, const char *text, int64_t total_bytes, const Shape &sh, double *out, float *out32,
                         cudaStream_t s, double *host_out = nullptr) {
    const int64_t n_data = (int64_t)sh.data_lines.size(), len = (int64_t)sh.len, n = n_data * len;
    TSFM_TRY(grow(&x.d_data, &x.data_cap, (size_t)n_data * 8, "series: data lines"));
    TSFM_TRY(grow(&x.d_ts, &x.ts_cap, (size_t)n * 8, "series: tokens"));
    TSFM_TRY(grow(&x.d_te, &x.te_cap, (size_t)n * 8, "series: tokens"));
    TSFM_CUDA(cudaMemcpyAsync(x.d_data, sh.data_lines.data(), (size_t)n_data * 8, cudaMemcpyHostToDevice, s),
              "series: data lines");
    token_kernel<<<(unsigned)((n_data + 7) / 8), 256, 0, s>>>(text, total_bytes, x.d_info, x.d_data, n_data, len,
                                                               x.d_ts, x.d_te);
    TSFM_CUDA(cudaGetLastError(), "series: tokens");
    if (host_out == nullptr) {
        parse_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(text, total_bytes, x.d_ts, x.d_te, n, out, out32);
        TSFM_CUDA(cudaGetLastError(), "series: parse");
        TSFM_CUDA(cudaStreamSynchronize(s), "series: parse");
        return Status::ok();
    }
    constexpr int kChunks = 16;
    const int64_t per = std::max<int64_t>(256, ((n + kChunks - 1) / kChunks + 255) / 256 * 256);
    int k = 0;
    for (int64_t t0 = 0; t0 < n; t0 += per, ++k) {
        const int64_t cnt = std::min(per, n - t0);
        parse_kernel<<<(unsigned)((cnt + 255) / 256), 256, 0, s>>>(text, total_bytes, x.d_ts + t0, x.d_te + t0, cnt,
                                                                   out + t0, nullptr);
        TSFM_CUDA(cudaGetLastError(), "series: parse");
        TSFM_CUDA(cudaEventRecord(x.ev[k], s), "series: event");
        TSFM_CUDA(cudaStreamWaitEvent(x.copy, x.ev[k], 0), "series: wait");
        TSFM_CUDA(cudaMemcpyAsync(host_out + t0, out + t0, (size_t)cnt * 8, cudaMemcpyDeviceToHost, x.copy),
                  "series: values out");
    }
    TSFM_CUDA(cudaStreamSynchronize(x.copy), "series: values out");
    TSFM_CUDA(cudaStreamSynchronize(s), "series: parse");
    return Status::ok();
}

Status check_out(size_t *blocks, size_t *rows, size_t *len) {
    if (!blocks || !rows || !len) return Status::fail(TSFM_ERR_INVALID_ARGUMENT, "series: null shape pointer");
    return Status::ok();
}

Status parse_host(int device, const char *text, size_t length, double *values, size_t capacity, size_t *blocks,
                  size_t *rows, size_t *len) {
    TSFM_TRY(check_out(blocks, rows, len));
    if (text == nullptr && length > 0) return Status::fail(TSFM_ERR_INVALID_ARGUMENT, "series: text is null");
    if (device < 0 || device >= kMaxDevices) return Status::fail(TSFM_ERR_NO_DEVICE, "series: device ordinal");
    PCtx &x = g_pctx[device];
    std::lock_guard<std::mutex> lock(x.mu);
    TSFM_TRY(pctx_init(x, device));
    TSFM_TRY(grow(&x.d_text, &x.text_cap, length + 16, "series: text"));
    if (length > 0)
        TSFM_CUDA(cudaMemcpyAsync(x.d_text, text, length, cudaMemcpyHostToDevice, x.stream), "series: text in");
    Shape sh;
    TSFM_TRY(structure(x, x.d_text, (int64_t)length, x.stream, sh));
    *blocks = sh.blocks;
    *rows = sh.rows;
    *len = sh.len;
    const size_t need = sh.blocks * sh.rows * sh.len;
    if (values == nullptr) return Status::ok();
    if (capacity < need)
        return Status::fail(TSFM_ERR_BUFFER_TOO_SMALL,
                            "series: " + std::to_string(need) + " values, capacity " + std::to_string(capacity));
    TSFM_TRY(grow(&x.d_vals, &x.vals_cap, need * 8, "series: values"));
    return tokens_and_values(x, x.d_text, (int64_t)length, sh, x.d_vals, nullptr, x.stream, values);
}

Status parse_device(const char *text, size_t length, double *values, float *values32, size_t capacity, size_t *blocks,
                    size_t *rows, size_t *len, cudaStream_t s) {
    TSFM_TRY(check_out(blocks, rows, len));
    if (text == nullptr && length > 0) return Status::fail(TSFM_ERR_INVALID_ARGUMENT, "series: text is null");
    int device = 0;
    TSFM_CUDA(cudaGetDevice(&device), "series: device");
    if (device >= kMaxDevices) return Status::fail(TSFM_ERR_NO_DEVICE, "series: device ordinal");
    PCtx &x = g_pctx[device];
    std::lock_guard<std::mutex> lock(x.mu);
    TSFM_TRY(pctx_init(x, device));
    Shape sh;
    TSFM_TRY(structure(x, text, (int64_t)length, s, sh));
    *blocks = sh.blocks;
    *rows = sh.rows;
    *len = sh.len;
    const size_t need = sh.blocks * sh.rows * sh.len;
    if (values == nullptr && values32 == nullptr) return Status::ok();
    if (capacity < need)
        return Status::fail(TSFM_ERR_BUFFER_TOO_SMALL,
                            "series: " + std::to_string(need) + " values, capacity " + std::to_string(capacity));
    return tokens_and_values(x, text, (int64_t)length, sh, values, values32, s);
}

template <class F>
int32_t guarded(F &&f) {
    try {
        return set_last_error(f());
    } catch (const std::bad_alloc &) {
        return set_last_error(Status::fail(TSFM_ERR_OUT_OF_MEMORY, "host allocation failed"));
    } catch (const std::exception &e) {
        return set_last_error(Status::fail(TSFM_ERR_INVALID_ARGUMENT, e.what()));
    }
}

}  // namespace
}  // namespace tsfm

extern "C" {

int32_t tsfm_parse_blocks(const char *text, size_t length, int32_t device, double *values, size_t capacity,
                          size_t *blocks, size_t *rows, size_t *len) {
    return tsfm::guarded([&] { return tsfm::parse_host(device, text, length, values, capacity, blocks, rows, len); });
}

int32_t tsfm_parse_blocks_device(const char *text, size_t length, double *values, float *values_f32, size_t capacity,
                                 size_t *blocks, size_t *rows, size_t *len, void *stream) {
    return tsfm::guarded([&] {
        return tsfm::parse_device(text, length, values, values_f32, capacity, blocks, rows, len,
                                  static_cast<cudaStream_t>(stream));
    });
}

}  // extern "C"
