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

// (1a) newlines per tile.
__global__ void __launch_bounds__(256) nl_count_kernel(const char *text, int64_t n, uint32_t *tile_count) {
    const int64_t base = (int64_t)blockIdx.x * kTile + threadIdx.x * 16;
    uint32_t c = 0;
    for (int i = 0; i < 16; ++i) c += (base + i < n && text[base + i] == '\n') ? 1u : 0u;
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
    const int64_t base = (int64_t)blockIdx.x * kTile + threadIdx.x * 16;
    uint32_t c = 0;
    for (int i = 0; i < 16; ++i) c += (base + i < n && text[base + i] == '\n') ? 1u : 0u;
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
    uint64_t k = tile_off[blockIdx.x] + before + x - c;
    for (int i = 0; i < 16; ++i)
        if (base + i < n && text[base + i] == '\n') pos[k++] = (uint64_t)(base + i);
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

// (2) one warp per line: trimmed bounds, kind, separator, token count.
__global__ void __launch_bounds__(256) line_kernel(const char *text, int64_t total, const uint64_t *nl, int64_t n_nl,
                                                  LineInfo *info, uint32_t *meta) {
    const int lane = threadIdx.x & 31;
    const int64_t line = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    if (line > n_nl) return;
    uint64_t s, e;
    line_span(nl, n_nl, total, line, &s, &e);
    // First and last bytes that are not " \t\r".
    uint64_t a = e, b = s;
    for (uint64_t p = s; p < e; p += 32) {
        const uint64_t q = p + lane;
        const unsigned m = __ballot_sync(0xffffffffu, q < e && !is_trim(text[q]));
        if (m) {
            a = p + (__ffs(m) - 1);
            break;
        }
    }
    if (a < e) {
        for (uint64_t p = e; p > a;) {
            const uint64_t step = p - a < 32 ? p - a : 32, lo = p - step;
            const uint64_t q = lo + lane;
            const unsigned m = __ballot_sync(0xffffffffu, q < p && !is_trim(text[q]));
            if (m) {
                b = lo + (31 - __clz(m)) + 1;
                break;
            }
            p = lo;
        }
    }
    LineInfo li{};
    li.a = a;
    li.b = a < e ? b : a;
    if (a >= e) {
        li.kind = 0;
    } else if (text[a] == '#') {
        li.kind = 1;
    } else {
        li.kind = 2;
        uint32_t commas = 0, starts = 0;
        for (uint64_t p = a; p < li.b; p += 32) {
            const uint64_t q = p + lane;
            const bool in = q < li.b;
            const char c = in ? text[q] : ' ';
            const char prev = (in && q > a) ? text[q - 1] : ' ';
            commas += __popc(__ballot_sync(0xffffffffu, in && c == ','));
            starts += __popc(__ballot_sync(0xffffffffu, in && !is_sep(c) && is_sep(prev)));
        }
        li.comma = commas > 0;
        li.tokens = commas > 0 ? commas + 1 : starts;
    }
    if (lane == 0) {
        info[line] = li;
        meta[line] = ((uint32_t)li.kind << 30) | (li.tokens & 0x3fffffffu);
    }
}

// (4) one warp per data line: each token's [start, end) (before trimming).
__global__ void __launch_bounds__(256) token_kernel(const char *text, const LineInfo *info, const int64_t *data_lines,
                                                   int64_t n_data, int64_t len, uint64_t *tok_s, uint64_t *tok_e) {
    const int lane = threadIdx.x & 31;
    const int64_t d = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    if (d >= n_data) return;
    const LineInfo li = info[data_lines[d]];
    const int64_t base = d * len;
    uint32_t k = 0;  // tokens seen so far
    if (li.comma) {
        if (lane == 0) tok_s[base] = li.a;
        for (uint64_t p = li.a; p < li.b; p += 32) {
            const uint64_t q = p + lane;
            const bool hit = q < li.b && text[q] == ',';
            const unsigned m = __ballot_sync(0xffffffffu, hit);
            if (hit) {
                const uint32_t r = k + __popc(m & ((1u << lane) - 1));
                tok_e[base + r] = q;
                tok_s[base + r + 1] = q + 1;
            }
            k += __popc(m);
        }
        if (lane == 0) tok_e[base + k] = li.b;
    } else {
        for (uint64_t p = li.a; p < li.b; p += 32) {
            const uint64_t q = p + lane;
            const bool in = q < li.b;
            const char c = in ? text[q] : ' ';
            const bool start = in && !is_sep(c) && (q == li.a || is_sep(text[q - 1]));
            const bool end = in && !is_sep(c) && (q + 1 == li.b || is_sep(text[q + 1]));
            const unsigned ms = __ballot_sync(0xffffffffu, start), me = __ballot_sync(0xffffffffu, end);
            if (start) tok_s[base + k + __popc(ms & ((1u << lane) - 1))] = q;
            // An end closes the token of the latest start at or before it (possibly in an earlier
            // window): index k - 1 + (starts in this window up to and including this lane).
            if (end) tok_e[base + k - 1 + __popc(ms & ((2u << lane) - 1))] = q + 1;
            (void)me;
            k += __popc(ms);
        }
    }
}

// (5) one thread per token: trim, parse, store f64 (and f32 when asked: @floatCast, nearest).
__global__ void __launch_bounds__(256) parse_kernel(const char *text, const uint64_t *tok_s, const uint64_t *tok_e,
                                                   int64_t n, double *out, float *out32) {
    const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= n) return;
    uint64_t a = tok_s[t], b = tok_e[t];
    while (a < b && is_trim(text[a])) ++a;
    while (b > a && is_trim(text[b - 1])) --b;
    double v;
    if (a == b) {
        v = numparse::quiet_nan(false);
    } else if (b - a > (1u << 20)) {
        v = numparse::quiet_nan(false);  // over a MiB is never a number the reader accepts
    } else {
        v = numparse::parse_number(text + a, (int)(b - a));
    }
    if (out) out[t] = v;
    if (out32) out32[t] = (float)v;
}

// ---------------------------------------------------------------------------------------------
// Host side.

struct PCtx {
    std::mutex mu;
    bool ready = false;
    cudaStream_t stream = nullptr;
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
    TSFM_CUDA(cudaMallocHost(reinterpret_cast<void **>(&x.h_total), 16), "series: pinned total");
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
    const int64_t tiles = std::max<int64_t>(1, (n + kTile - 1) / kTile);
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
Status tokens_and_values(PCtx &x, const char *text, const Shape &sh, double *out, float *out32, cudaStream_t s) {
    const int64_t n_data = (int64_t)sh.data_lines.size(), len = (int64_t)sh.len, n = n_data * len;
    TSFM_TRY(grow(&x.d_data, &x.data_cap, (size_t)n_data * 8, "series: data lines"));
    TSFM_TRY(grow(&x.d_ts, &x.ts_cap, (size_t)n * 8, "series: tokens"));
    TSFM_TRY(grow(&x.d_te, &x.te_cap, (size_t)n * 8, "series: tokens"));
    TSFM_CUDA(cudaMemcpyAsync(x.d_data, sh.data_lines.data(), (size_t)n_data * 8, cudaMemcpyHostToDevice, s),
              "series: data lines");
    token_kernel<<<(unsigned)((n_data + 7) / 8), 256, 0, s>>>(text, x.d_info, x.d_data, n_data, len, x.d_ts, x.d_te);
    TSFM_CUDA(cudaGetLastError(), "series: tokens");
    parse_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(text, x.d_ts, x.d_te, n, out, out32);
    TSFM_CUDA(cudaGetLastError(), "series: parse");
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
    TSFM_TRY(tokens_and_values(x, x.d_text, sh, x.d_vals, nullptr, x.stream));
    TSFM_CUDA(cudaMemcpyAsync(values, x.d_vals, need * 8, cudaMemcpyDeviceToHost, x.stream), "series: values out");
    TSFM_CUDA(cudaStreamSynchronize(x.stream), "series: values out");
    return Status::ok();
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
    return tokens_and_values(x, text, sh, values, values32, s);
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
