// CSV output of a forecast on the GPU: the reference CLI's writeCsv (src/main.zig:181-198).
//
// Text layout: a header "series,variate,step" + ",q<level>" per quantile level, then one line
// per (series, variate, step) in row-major order: "s,v,step+1" + ",<value>" per level, each
// line ended by '\n'. Levels are f64 and values f32, both printed as Zig's "{d}" (decimal
// notation, shortest round-trip digits; csv_digits.cuh).
//
// Three kernels per chunk of lines, each block owning `lpb` consecutive lines:
//   describe  the shortest digits of every value (Ryu), packed in 8 bytes per value, and the
//             block's text length;
//   scan      one block turns the block lengths into byte offsets (and the chunk's total);
//   text      the block renders its lines into shared memory (each thread a contiguous run of
//             prefixes, values and newlines, placed by a block-wide scan of their lengths) and
//             copies them out with 16-byte stores aligned to the destination.
// The host entry points stream chunks through three CUDA streams: host-to-device copies of
// the next chunk's values, the kernels, and device-to-host copies of the previous chunk's text
// overlap one another.
#include <cuda_runtime.h>
#include <errno.h>
#include <unistd.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>

#include "../../include/tsfm_b200.h"
#include "csv_digits.cuh"
#include "kernels.h"

namespace tsfm {
int32_t set_last_error(const Status &s);

namespace {

__constant__ csv::Pow5Tables c_pow5;

constexpr int kThreads = 256;
constexpr int kPrefixMax = 3 * 20 + 2;  // "s,v,step" with 20-digit integers
constexpr int kValueMax = 50;           // ',' + at most 49 bytes of f32 text ("-0.000...0ddddddddd")
constexpr int kMaxLevels = 1000;

// Lines per block: about 768 numbers per block, at most 32 lines.
inline int lines_per_block(int q) { return std::min(32, std::max(1, 768 / (q + 2))); }

struct Lines {
    const float *values;  // (lines, q) f32 of this chunk
    int64_t first;        // global index of the chunk's first line
    int64_t lines;
    int64_t variates, horizon;
    int q, lpb;
};

// A value's text description in 8 bytes: digits (30 bits) | exponent + 64 (7) | digit count (4)
// | text length (6) | kind (2) | sign (1).
__device__ __forceinline__ uint64_t pack(const csv::F32Text &f) {
    return (uint64_t)f.digits | ((uint64_t)(f.exponent + 64) << 30) | ((uint64_t)f.ndigits << 37) |
           ((uint64_t)f.len << 41) | ((uint64_t)f.kind << 47) | ((uint64_t)(f.neg ? 1 : 0) << 49);
}

__device__ __forceinline__ csv::F32Text unpack(uint64_t p) {
    csv::F32Text f;
    f.digits = (uint32_t)(p & 0x3fffffffu);
    f.exponent = (int32_t)((p >> 30) & 0x7f) - 64;
    f.ndigits = (int8_t)((p >> 37) & 0xf);
    f.len = (int16_t)((p >> 41) & 0x3f);
    f.kind = (int8_t)((p >> 47) & 0x3);
    f.neg = ((p >> 49) & 1) != 0;
    return f;
}

// Digit count of v (1..20) by comparison with powers of ten.
__device__ __forceinline__ int u64_digits(uint64_t v) {
    int n = 1;
    uint64_t p = 10;
    while (n < 20 && v >= p) {
        ++n;
        p *= 10;
    }
    return n;
}

__device__ __forceinline__ void emit_uint(uint64_t v, int len, char *o) {
    if (v < (1ull << 32)) {
        uint32_t w = (uint32_t)v;
        for (int i = len - 1; i >= 0; --i) {
            o[i] = (char)('0' + w % 10);
            w /= 10;
        }
    } else {
        csv::emit_u64(v, len, o);
    }
}

// The (series, variate, step) of a block's lines, one line per thread of the first warp; 32-bit
// divisions when the indices fit (the usual case), 64-bit ones otherwise.
struct LineIds {
    uint64_t s[32], v[32], step[32];
    uint8_t ls[32], lv[32], lst[32];
};

__device__ __forceinline__ void line_ids(const Lines &c, int64_t l0, int li, LineIds &ids) {
    const int64_t line = c.first + l0 + li, per_series = c.variates * c.horizon;
    uint64_t s, v, step;
    if (c.first + c.lines <= (int64_t)UINT32_MAX && per_series <= (int64_t)UINT32_MAX) {
        const uint32_t l = (uint32_t)line, ps = (uint32_t)per_series, h = (uint32_t)c.horizon;
        const uint32_t s32 = l / ps, rem = l - s32 * ps, v32 = rem / h;
        s = s32;
        v = v32;
        step = rem - v32 * h + 1;
    } else {
        s = (uint64_t)(line / per_series);
        const int64_t rem = line - (int64_t)s * per_series;
        v = (uint64_t)(rem / c.horizon);
        step = (uint64_t)(rem - (int64_t)v * c.horizon) + 1;
    }
    ids.s[li] = s;
    ids.v[li] = v;
    ids.step[li] = step;
    ids.ls[li] = (uint8_t)u64_digits(s);
    ids.lv[li] = (uint8_t)u64_digits(v);
    ids.lst[li] = (uint8_t)u64_digits(step);
}

__device__ __forceinline__ int prefix_len(const LineIds &ids, int li) {
    return ids.ls[li] + ids.lv[li] + ids.lst[li] + 2;  // "s,v,step"
}

__device__ __forceinline__ void emit_prefix(const LineIds &ids, int li, char *o) {
    const int ls = ids.ls[li], lv = ids.lv[li];
    emit_uint(ids.s[li], ls, o);
    o[ls] = ',';
    emit_uint(ids.v[li], lv, o + ls + 1);
    o[ls + 1 + lv] = ',';
    emit_uint(ids.step[li], ids.lst[li], o + ls + lv + 2);
}

// Block-wide exclusive scan of one value per thread; *total receives the block's sum.
__device__ __forceinline__ uint32_t block_scan(uint32_t v, uint32_t *wsum, uint32_t *total) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    uint32_t x = v;
    for (int o = 1; o < 32; o <<= 1) {
        const uint32_t y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
    }
    if (lane == 31) wsum[warp] = x;
    __syncthreads();
    if (warp == 0) {
        uint32_t w = lane < kThreads / 32 ? wsum[lane] : 0;
        for (int o = 1; o < 32; o <<= 1) {
            const uint32_t y = __shfl_up_sync(0xffffffffu, w, o);
            if (lane >= o) w += y;
        }
        if (lane < kThreads / 32) wsum[lane] = w;
    }
    __syncthreads();
    *total = wsum[kThreads / 32 - 1];
    return x - v + (warp ? wsum[warp - 1] : 0);
}

// (1) digits of every value, packed; the text length of each block of lines.
__global__ void __launch_bounds__(kThreads) csv_describe_kernel(Lines c, uint64_t *packed, uint32_t *block_sum) {
    __shared__ csv::Pow5Tables tab;
    __shared__ uint32_t wsum[kThreads / 32];
    __shared__ LineIds ids;
    {
        const uint64_t *src = reinterpret_cast<const uint64_t *>(&c_pow5);
        uint64_t *dst = reinterpret_cast<uint64_t *>(&tab);
        for (int i = threadIdx.x; i < (int)(sizeof(csv::Pow5Tables) / 8); i += kThreads) dst[i] = src[i];
    }
    __syncthreads();
    const int64_t l0 = (int64_t)blockIdx.x * c.lpb;
    const int nl = (int)min((int64_t)c.lpb, c.lines - l0);
    const int n = nl * c.q;
    const int64_t base = l0 * c.q;
    const uint32_t *bits = reinterpret_cast<const uint32_t *>(c.values);
    uint32_t acc = 0;
    for (int i = threadIdx.x; i < n; i += kThreads) {
        const csv::F32Text f = csv::describe(bits[base + i], tab);
        packed[base + i] = pack(f);
        acc += 1 + (uint32_t)f.len;
    }
    if (threadIdx.x < nl) {  // each thread reads back only its own line's entries
        line_ids(c, l0, threadIdx.x, ids);
        acc += (uint32_t)prefix_len(ids, threadIdx.x) + 1;
    }
    uint32_t total;
    block_scan(acc, wsum, &total);
    if (threadIdx.x == 0) block_sum[blockIdx.x] = total;
}

// (2) exclusive scan of the block lengths (one block of 1024 threads) and the chunk's total.
__global__ void __launch_bounds__(1024) csv_scan_kernel(const uint32_t *in, int64_t n, uint64_t *excl, uint64_t *total) {
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

// Dynamic shared memory of the text kernel: packed values, then the text (16-byte aligned).
__host__ __device__ inline size_t packed_smem(int q, int lpb) { return ((size_t)lpb * q * 8 + 15) / 16 * 16; }
__host__ __device__ inline size_t text_smem(int q, int lpb) {
    return (size_t)lpb * (kPrefixMax + 1 + (size_t)kValueMax * q) + 16;
}

// (3) the text of each block of lines at its offset.
__global__ void __launch_bounds__(kThreads) csv_text_kernel(Lines c, const uint64_t *packed, const uint64_t *block_off,
                                                           char *out) {
    extern __shared__ __align__(16) unsigned char smem[];
    __shared__ uint32_t wsum[kThreads / 32];
    __shared__ LineIds ids;
    uint64_t *pk = reinterpret_cast<uint64_t *>(smem);
    char *text = reinterpret_cast<char *>(smem + packed_smem(c.q, c.lpb));
    const int64_t l0 = (int64_t)blockIdx.x * c.lpb;
    const int nl = (int)min((int64_t)c.lpb, c.lines - l0);
    const int n = nl * c.q;
    const int64_t base = l0 * c.q;
    if (threadIdx.x < nl) line_ids(c, l0, threadIdx.x, ids);
    for (int i = threadIdx.x; i < n; i += kThreads) pk[i] = packed[base + i];
    __syncthreads();

    // Items of a line: its prefix, its q values, its newline. Each thread owns a contiguous run.
    const int per = c.q + 2, items = nl * per;
    const int ipt = (items + kThreads - 1) / kThreads;
    const int k0 = min(items, (int)threadIdx.x * ipt), k1 = min(items, k0 + ipt);
    uint32_t mine = 0;
    {
        int li = k0 / per, r = k0 - li * per;
        for (int k = k0; k < k1; ++k) {
            mine += r == 0 ? (uint32_t)prefix_len(ids, li)
                           : (r <= c.q ? 1 + (uint32_t)((pk[li * c.q + r - 1] >> 41) & 0x3f) : 1);
            if (++r == per) r = 0, ++li;
        }
    }
    uint32_t total;
    const uint32_t off = block_scan(mine, wsum, &total);
    char *dst = out + block_off[blockIdx.x];
    const int pad = (int)(reinterpret_cast<uintptr_t>(dst) & 15);
    {
        int li = k0 / per, r = k0 - li * per;
        uint32_t o = (uint32_t)pad + off;
        for (int k = k0; k < k1; ++k) {
            if (r == 0) {
                emit_prefix(ids, li, text + o);
                o += (uint32_t)prefix_len(ids, li);
            } else if (r <= c.q) {
                const csv::F32Text f = unpack(pk[li * c.q + r - 1]);
                text[o] = ',';
                csv::emit(f, text + o + 1);
                o += 1 + (uint32_t)f.len;
            } else {
                text[o++] = '\n';
            }
            if (++r == per) r = 0, ++li;
        }
    }
    __syncthreads();
    // text[pad, pad + total) -> dst[0, total), in 16-byte chunks aligned to the destination.
    char *abase = dst - pad;
    const int end = pad + (int)total;
    for (int i = threadIdx.x * 16; i < end; i += kThreads * 16) {
        if (i >= pad && i + 16 <= end) {
            *reinterpret_cast<uint4 *>(abase + i) = *reinterpret_cast<const uint4 *>(text + i);
        } else {
            for (int b = max(i, pad); b < min(i + 16, end); ++b) abase[b] = text[b];
        }
    }
}

// ---------------------------------------------------------------------------------------------
// Host side.

typedef unsigned __int128 u128;

// floor(2^n / d) by binary long division (the remainder stays below d < 2^110).
uint64_t floor_pow2_div(int n, u128 d) {
    u128 rem = 0;
    uint64_t q = 0;
    for (int b = n; b >= 0; --b) {
        rem = (rem << 1) | (b == n ? 1u : 0u);
        q <<= 1;
        if (rem >= d) {
            rem -= d;
            q |= 1;
        }
    }
    return q;
}

csv::Pow5Tables make_tables() {
    csv::Pow5Tables t{};
    u128 p = 1;
    for (int q = 0; q < csv::kPow5InvCount; ++q, p *= 5)
        t.inv[q] = floor_pow2_div(csv::pow5bits(q) - 1 + csv::kPow5InvBits, p) + 1;
    p = 1;
    for (int i = 0; i < csv::kPow5Count; ++i, p *= 5) {
        const int sh = csv::pow5bits(i) - csv::kPow5Bits;
        t.pos[i] = (uint64_t)(sh >= 0 ? (p >> sh) : (p << -sh));
    }
    return t;
}

// Zig "{d}" of an f64 (the quantile levels of the header): the shortest digit string that reads
// back to the same double (closest to the exact value among the shortest), in decimal notation.
std::string f64_text(double x) {
    if (std::isnan(x)) return "nan";
    const bool neg = std::signbit(x);
    if (std::isinf(x)) return neg ? "-inf" : "inf";
    if (x == 0) return neg ? "-0" : "0";
    char buf[64];
    std::string digits;
    int exponent = 0;  // value = digits * 10^exponent
    for (int len = 1; len <= 17 && digits.empty(); ++len) {
        snprintf(buf, sizeof buf, "%.*e", len - 1, std::fabs(x));
        const char *e = std::strchr(buf, 'e');
        std::string d;
        for (const char *c = buf; c < e; ++c)
            if (*c >= '0' && *c <= '9') d += *c;
        const int ex = std::atoi(e + 1) - (len - 1);
        if (std::strtod(buf, nullptr) == std::fabs(x)) {
            digits = d;
            exponent = ex;
            break;
        }
        // The correctly rounded candidate misses the interval: try its neighbour on the other
        // side of x.
        unsigned long long v = std::strtoull(d.c_str(), nullptr, 10);
        const double r = std::strtod(buf, nullptr);
        v = r < std::fabs(x) ? v + 1 : v - 1;
        snprintf(buf, sizeof buf, "%llue%d", v, ex);
        if (v > 0 && std::strtod(buf, nullptr) == std::fabs(x)) {
            digits = std::to_string(v);
            exponent = ex;
        }
    }
    while (digits.size() > 1 && digits.back() == '0') {
        digits.pop_back();
        ++exponent;
    }
    const int nd = (int)digits.size(), dp = exponent + nd;
    std::string s = neg ? "-" : "";
    if (dp <= 0) {
        s += "0." + std::string(-dp, '0') + digits;
    } else if (dp >= nd) {
        s += digits + std::string(dp - nd, '0');
    } else {
        s += digits.substr(0, dp) + "." + digits.substr(dp);
    }
    return s;
}

std::string header_text(const double *levels, size_t nq) {
    std::string h = "series,variate,step";
    for (size_t i = 0; i < nq; ++i) h += ",q" + f64_text(levels[i]);
    h += '\n';
    return h;
}

// Per-device state: streams, events, scratch and staging buffers (grown on demand). Two slots
// of values and text let consecutive chunks overlap.
struct Ctx {
    std::mutex mu;
    bool ready = false;
    cudaStream_t comp = nullptr, h2d = nullptr, d2h = nullptr;
    cudaEvent_t ev_in[2] = {}, ev_text[2] = {}, ev_out[2] = {}, ev_total[2] = {};
    float *d_values[2] = {nullptr, nullptr};
    size_t values_cap[2] = {0, 0};
    char *d_text[2] = {nullptr, nullptr};
    size_t text_cap[2] = {0, 0};
    uint64_t *d_packed = nullptr;
    size_t packed_cap = 0;
    uint32_t *d_block_sum = nullptr;
    uint64_t *d_block_off = nullptr, *d_total = nullptr;
    size_t blocks_cap = 0;
    char *h_text[2] = {nullptr, nullptr};
    size_t h_text_cap[2] = {0, 0};
    uint64_t *h_total = nullptr;  // pinned, one per slot
    // Optional per-kernel device time (CUDA events around each launch; read after each sync).
    bool prof = false;
    cudaEvent_t ev[6] = {};
    bool recorded[3] = {false, false, false};
    uint64_t launches[3] = {0, 0, 0};
    double ms[3] = {0, 0, 0};
};

enum { K_DESCRIBE = 0, K_SCAN = 1, K_TEXT = 2 };

void prof_mark(Ctx &x, int k, bool end, cudaStream_t s) {
    if (!x.prof) return;
    cudaEventRecord(x.ev[2 * k + (end ? 1 : 0)], s);
    if (end) x.recorded[k] = true;
}

// After a synchronisation that covers the recorded launches: adds their times.
void prof_collect(Ctx &x) {
    for (int k = 0; k < 3; ++k) {
        if (!x.recorded[k]) continue;
        float f = 0.0f;
        if (cudaEventElapsedTime(&f, x.ev[2 * k], x.ev[2 * k + 1]) == cudaSuccess) {
            x.ms[k] += f;
            x.launches[k] += 1;
        }
        x.recorded[k] = false;
    }
}

constexpr int kMaxDevices = 64;
Ctx g_ctx[kMaxDevices];

template <class T>
Status grow_dev(T **p, size_t *cap, size_t bytes, const char *what) {
    if (*cap >= bytes) return Status::ok();
    if (*p) cudaFree(*p);
    *p = nullptr;
    *cap = 0;
    TSFM_CUDA(cudaMalloc(reinterpret_cast<void **>(p), bytes), what);
    *cap = bytes;
    return Status::ok();
}

size_t max_text_smem() {
    size_t m = 0;
    for (int q = 0; q <= kMaxLevels; ++q) {
        const int l = lines_per_block(q);
        m = std::max(m, packed_smem(q, l) + text_smem(q, l));
    }
    return m;
}

Status ctx_init(Ctx &x, int device) {
    TSFM_CUDA(cudaSetDevice(device), "csv: cudaSetDevice");
    if (x.ready) return Status::ok();
    const csv::Pow5Tables t = make_tables();
    TSFM_CUDA(cudaMemcpyToSymbol(c_pow5, &t, sizeof t), "csv: tables");
    TSFM_CUDA(cudaFuncSetAttribute(csv_text_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)max_text_smem()),
              "csv: shared memory attribute");
    for (cudaStream_t *s : {&x.comp, &x.h2d, &x.d2h})
        TSFM_CUDA(cudaStreamCreateWithFlags(s, cudaStreamNonBlocking), "csv: stream");
    for (int i = 0; i < 2; ++i)
        for (cudaEvent_t *e : {&x.ev_in[i], &x.ev_text[i], &x.ev_out[i], &x.ev_total[i]})
            TSFM_CUDA(cudaEventCreateWithFlags(e, cudaEventDisableTiming), "csv: event");
    TSFM_CUDA(cudaMallocHost(reinterpret_cast<void **>(&x.h_total), 16), "csv: pinned total");
    x.ready = true;
    return Status::ok();
}

Status ensure_scratch(Ctx &x, int64_t lines, int q) {
    const int lpb = lines_per_block(q);
    const size_t blocks = (size_t)((lines + lpb - 1) / lpb) + 1;
    if (x.blocks_cap < blocks) {
        size_t c1 = 0, c2 = 0;
        TSFM_TRY(grow_dev(&x.d_block_sum, &c1, blocks * 4, "csv: block lengths"));
        TSFM_TRY(grow_dev(&x.d_block_off, &c2, blocks * 8, "csv: block offsets"));
        x.blocks_cap = blocks;
    }
    size_t ct = x.d_total ? 16 : 0;
    TSFM_TRY(grow_dev(&x.d_total, &ct, 16, "csv: total"));
    TSFM_TRY(grow_dev(&x.d_packed, &x.packed_cap, (size_t)lines * q * 8 + 16, "csv: packed digits"));
    return Status::ok();
}

// describe + scan for one chunk on stream s; the byte total lands in x.d_total.
Status run_lengths(Ctx &x, const Lines &c, cudaStream_t s) {
    const int64_t blocks = (c.lines + c.lpb - 1) / c.lpb;
    if (blocks == 0) {
        TSFM_CUDA(cudaMemsetAsync(x.d_total, 0, 8, s), "csv: total");
        return Status::ok();
    }
    prof_mark(x, K_DESCRIBE, false, s);
    csv_describe_kernel<<<(unsigned)blocks, kThreads, 0, s>>>(c, x.d_packed, x.d_block_sum);
    TSFM_CUDA(cudaGetLastError(), "csv: describe kernel");
    prof_mark(x, K_DESCRIBE, true, s);
    prof_mark(x, K_SCAN, false, s);
    csv_scan_kernel<<<1, 1024, 0, s>>>(x.d_block_sum, blocks, x.d_block_off, x.d_total);
    TSFM_CUDA(cudaGetLastError(), "csv: scan kernel");
    prof_mark(x, K_SCAN, true, s);
    return Status::ok();
}

Status run_text(Ctx &x, const Lines &c, char *out, cudaStream_t s) {
    const int64_t blocks = (c.lines + c.lpb - 1) / c.lpb;
    if (blocks == 0) return Status::ok();
    const size_t smem = packed_smem(c.q, c.lpb) + text_smem(c.q, c.lpb);
    prof_mark(x, K_TEXT, false, s);
    csv_text_kernel<<<(unsigned)blocks, kThreads, smem, s>>>(c, x.d_packed, x.d_block_off, out);
    TSFM_CUDA(cudaGetLastError(), "csv: text kernel");
    prof_mark(x, K_TEXT, true, s);
    return Status::ok();
}

Status check_shape(const float *values, size_t series, size_t variates, size_t horizon, const double *levels,
                   size_t nq, size_t *length) {
    if (length == nullptr) return Status::fail(TSFM_ERR_INVALID_ARGUMENT, "csv: length pointer is null");
    if (nq > 0 && levels == nullptr) return Status::fail(TSFM_ERR_INVALID_ARGUMENT, "csv: levels pointer is null");
    if (nq > (size_t)kMaxLevels)
        return Status::fail(TSFM_ERR_UNSUPPORTED, "csv: more than " + std::to_string(kMaxLevels) + " quantile levels");
    const double lines = (double)series * (double)variates * (double)horizon;
    if (lines > 9.0e15) return Status::fail(TSFM_ERR_INVALID_ARGUMENT, "csv: too many lines");
    if (lines > 0 && nq > 0 && values == nullptr)
        return Status::fail(TSFM_ERR_INVALID_ARGUMENT, "csv: values pointer is null");
    return Status::ok();
}

// Lines per chunk of the host entry points: 32 MiB of values, whole blocks.
int64_t chunk_lines(int q) {
    const int lpb = lines_per_block(q);
    const int64_t per = std::max<int64_t>(1, (int64_t)q) * 4;
    return std::max<int64_t>(lpb, ((int64_t)32 << 20) / per / lpb * lpb);
}

// The host entry points' pipeline. Per chunk c (slot c % 2): values in on the copy-in stream;
// describe + scan + the total back on the compute stream; the host reads the total, then the
// text kernel and the copy-out (stream d2h) of `sink.dest`. The next chunk's values go in
// while the host waits for this chunk's total; sink.done(c) runs once chunk c's copy-out ended.
struct Sink {
    virtual ~Sink() = default;
    // Where chunk c's text goes (host memory), or nullptr to skip rendering it.
    virtual Status dest(int64_t c, int slot, size_t bytes, char **p) = 0;
    virtual Status done(int64_t c, int slot, size_t bytes) = 0;
};

Status pipeline(Ctx &x, const float *values, int64_t lines, int64_t variates, int64_t horizon, int q, Sink &sink) {
    const int lpb = lines_per_block(q);
    const int64_t chunk = chunk_lines(q), nchunks = (lines + chunk - 1) / chunk;
    const int64_t cl = std::min<int64_t>(chunk, lines);
    TSFM_TRY(ensure_scratch(x, cl, q));
    for (int i = 0; i < 2; ++i) {
        TSFM_TRY(grow_dev(&x.d_values[i], &x.values_cap[i], (size_t)cl * q * 4 + 16, "csv: values"));
        TSFM_TRY(grow_dev(&x.d_text[i], &x.text_cap[i], (size_t)cl * (kPrefixMax + 1 + (size_t)kValueMax * q) + 16,
                          "csv: text"));
    }
    auto copy_in = [&](int64_t c) -> Status {
        const int slot = (int)(c & 1);
        const int64_t n = std::min<int64_t>(chunk, lines - c * chunk);
        TSFM_CUDA(cudaStreamWaitEvent(x.h2d, x.ev_text[slot], 0), "csv: wait");
        if (q > 0)
            TSFM_CUDA(cudaMemcpyAsync(x.d_values[slot], values + c * chunk * q, (size_t)n * q * 4,
                                      cudaMemcpyHostToDevice, x.h2d),
                      "csv: values in");
        TSFM_CUDA(cudaEventRecord(x.ev_in[slot], x.h2d), "csv: event");
        return Status::ok();
    };
    size_t sizes[2] = {0, 0};
    bool pending[2] = {false, false};
    if (nchunks > 0) TSFM_TRY(copy_in(0));
    for (int64_t c = 0; c < nchunks; ++c) {
        const int slot = (int)(c & 1);
        const int64_t n = std::min<int64_t>(chunk, lines - c * chunk);
        Lines lc{x.d_values[slot], c * chunk, n, variates, horizon, q, lpb};
        TSFM_CUDA(cudaStreamWaitEvent(x.comp, x.ev_in[slot], 0), "csv: wait");
        TSFM_TRY(run_lengths(x, lc, x.comp));
        TSFM_CUDA(cudaMemcpyAsync(x.h_total + slot, x.d_total, 8, cudaMemcpyDeviceToHost, x.comp), "csv: total out");
        TSFM_CUDA(cudaEventRecord(x.ev_total[slot], x.comp), "csv: event");
        if (c + 1 < nchunks) TSFM_TRY(copy_in(c + 1));
        TSFM_CUDA(cudaEventSynchronize(x.ev_total[slot]), "csv: lengths");
        const size_t bytes = (size_t)x.h_total[slot];
        char *p = nullptr;
        TSFM_TRY(sink.dest(c, slot, bytes, &p));
        if (p != nullptr) {
            TSFM_CUDA(cudaStreamWaitEvent(x.comp, x.ev_out[slot], 0), "csv: wait");
            TSFM_TRY(run_text(x, lc, x.d_text[slot], x.comp));
            TSFM_CUDA(cudaEventRecord(x.ev_text[slot], x.comp), "csv: event");
            TSFM_CUDA(cudaStreamWaitEvent(x.d2h, x.ev_text[slot], 0), "csv: wait");
            TSFM_CUDA(cudaMemcpyAsync(p, x.d_text[slot], bytes, cudaMemcpyDeviceToHost, x.d2h), "csv: text out");
            TSFM_CUDA(cudaEventRecord(x.ev_out[slot], x.d2h), "csv: event");
        } else {
            TSFM_CUDA(cudaEventRecord(x.ev_text[slot], x.comp), "csv: event");
        }
        // Chunk c - 1 has had its copy-out issued: finish it while this one renders.
        const int prev = 1 - slot;
        if (pending[prev]) {
            TSFM_CUDA(cudaEventSynchronize(x.ev_out[prev]), "csv: text");
            TSFM_TRY(sink.done(c - 1, prev, sizes[prev]));
            pending[prev] = false;
        }
        sizes[slot] = bytes;
        pending[slot] = p != nullptr;
        if (x.prof) {
            TSFM_CUDA(cudaStreamSynchronize(x.comp), "csv: profile");
            prof_collect(x);
        }
    }
    for (int i = 0; i < 2; ++i)
        if (pending[i]) {
            TSFM_CUDA(cudaEventSynchronize(x.ev_out[i]), "csv: text");
            TSFM_TRY(sink.done(nchunks - 1, i, sizes[i]));
        }
    TSFM_CUDA(cudaStreamSynchronize(x.d2h), "csv: text");
    TSFM_CUDA(cudaStreamSynchronize(x.comp), "csv: kernels");
    return Status::ok();
}

struct BufferSink : Sink {
    char *out;
    size_t capacity, pos;
    bool fits;
    Status dest(int64_t, int, size_t bytes, char **p) override {
        if (fits && pos + bytes <= capacity) {
            *p = out + pos;
        } else {
            fits = false;
            *p = nullptr;
        }
        pos += bytes;
        return Status::ok();
    }
    Status done(int64_t, int, size_t) override { return Status::ok(); }
};

Status write_all(int fd, const char *p, size_t n) {
    while (n > 0) {
        const ssize_t w = ::write(fd, p, n);
        if (w < 0) {
            if (errno == EINTR) continue;
            return Status::fail(TSFM_ERR_IO, std::string("csv: write failed: ") + std::strerror(errno));
        }
        p += w;
        n -= (size_t)w;
    }
    return Status::ok();
}

// Text copied into pinned staging (one buffer per slot) and written to fd.
struct FdSink : Sink {
    Ctx *x;
    int fd;
    size_t pos = 0;
    Status dest(int64_t, int slot, size_t bytes, char **p) override {
        if (x->h_text_cap[slot] < bytes) {
            if (x->h_text[slot]) cudaFreeHost(x->h_text[slot]);
            x->h_text[slot] = nullptr;
            x->h_text_cap[slot] = 0;
            TSFM_CUDA(cudaMallocHost(reinterpret_cast<void **>(&x->h_text[slot]), std::max<size_t>(bytes, 1)),
                      "csv: pinned text");
            x->h_text_cap[slot] = std::max<size_t>(bytes, 1);
        }
        *p = x->h_text[slot];
        return Status::ok();
    }
    Status done(int64_t, int slot, size_t bytes) override {
        TSFM_TRY(write_all(fd, x->h_text[slot], bytes));
        pos += bytes;
        return Status::ok();
    }
};

Status format_host(int device, const float *values, size_t series, size_t variates, size_t horizon,
                   const double *levels, size_t nq, char *out, size_t capacity, size_t *length) {
    TSFM_TRY(check_shape(values, series, variates, horizon, levels, nq, length));
    if (out == nullptr && capacity > 0) return Status::fail(TSFM_ERR_INVALID_ARGUMENT, "csv: out is null");
    if (device < 0 || device >= kMaxDevices) return Status::fail(TSFM_ERR_NO_DEVICE, "csv: device ordinal");
    Ctx &x = g_ctx[device];
    std::lock_guard<std::mutex> lock(x.mu);
    TSFM_TRY(ctx_init(x, device));
    const std::string head = header_text(levels, nq);
    BufferSink sink;
    sink.out = out;
    sink.capacity = capacity;
    sink.pos = head.size();
    sink.fits = head.size() <= capacity;
    if (sink.fits) std::memcpy(out, head.data(), head.size());
    TSFM_TRY(pipeline(x, values, (int64_t)(series * variates * horizon), (int64_t)variates, (int64_t)horizon, (int)nq,
                      sink));
    *length = sink.pos;
    if (!sink.fits)
        return Status::fail(TSFM_ERR_BUFFER_TOO_SMALL, "csv: the text needs " + std::to_string(sink.pos) +
                                                           " bytes, capacity " + std::to_string(capacity));
    return Status::ok();
}

Status write_fd(int device, const float *values, size_t series, size_t variates, size_t horizon, const double *levels,
                size_t nq, int fd, size_t *length) {
    TSFM_TRY(check_shape(values, series, variates, horizon, levels, nq, length));
    if (fd < 0) return Status::fail(TSFM_ERR_INVALID_ARGUMENT, "csv: bad file descriptor");
    if (device < 0 || device >= kMaxDevices) return Status::fail(TSFM_ERR_NO_DEVICE, "csv: device ordinal");
    Ctx &x = g_ctx[device];
    std::lock_guard<std::mutex> lock(x.mu);
    TSFM_TRY(ctx_init(x, device));
    const std::string head = header_text(levels, nq);
    TSFM_TRY(write_all(fd, head.data(), head.size()));
    FdSink sink;
    sink.x = &x;
    sink.fd = fd;
    sink.pos = head.size();
    TSFM_TRY(pipeline(x, values, (int64_t)(series * variates * horizon), (int64_t)variates, (int64_t)horizon, (int)nq,
                      sink));
    *length = sink.pos;
    return Status::ok();
}

Status format_device(const float *values, size_t series, size_t variates, size_t horizon, const double *levels,
                     size_t nq, char *out, size_t capacity, size_t *length, cudaStream_t s) {
    TSFM_TRY(check_shape(values, series, variates, horizon, levels, nq, length));
    if (out == nullptr && capacity > 0) return Status::fail(TSFM_ERR_INVALID_ARGUMENT, "csv: out is null");
    int device = 0;
    TSFM_CUDA(cudaGetDevice(&device), "csv: device");
    if (device >= kMaxDevices) return Status::fail(TSFM_ERR_NO_DEVICE, "csv: device ordinal");
    Ctx &x = g_ctx[device];
    std::lock_guard<std::mutex> lock(x.mu);
    TSFM_TRY(ctx_init(x, device));
    const std::string head = header_text(levels, nq);
    const int64_t lines = (int64_t)(series * variates * horizon);
    TSFM_TRY(ensure_scratch(x, lines, (int)nq));
    Lines c{values, 0, lines, (int64_t)variates, (int64_t)horizon, (int)nq, lines_per_block((int)nq)};
    TSFM_TRY(run_lengths(x, c, s));
    TSFM_CUDA(cudaMemcpyAsync(x.h_total, x.d_total, 8, cudaMemcpyDeviceToHost, s), "csv: total out");
    TSFM_CUDA(cudaStreamSynchronize(s), "csv: lengths");
    prof_collect(x);
    const size_t total = head.size() + (size_t)x.h_total[0];
    *length = total;
    if (total > capacity)
        return Status::fail(TSFM_ERR_BUFFER_TOO_SMALL,
                            "csv: the text needs " + std::to_string(total) + " bytes, capacity " + std::to_string(capacity));
    TSFM_CUDA(cudaMemcpyAsync(out, head.data(), head.size(), cudaMemcpyHostToDevice, s), "csv: header");
    TSFM_TRY(run_text(x, c, out + head.size(), s));
    TSFM_CUDA(cudaStreamSynchronize(s), "csv: text");
    prof_collect(x);
    return Status::ok();
}

Status profile_enable(int device, bool on) {
    if (device < 0 || device >= kMaxDevices) return Status::fail(TSFM_ERR_NO_DEVICE, "csv: device ordinal");
    Ctx &x = g_ctx[device];
    std::lock_guard<std::mutex> lock(x.mu);
    TSFM_TRY(ctx_init(x, device));
    if (on && x.ev[0] == nullptr)
        for (cudaEvent_t &e : x.ev) TSFM_CUDA(cudaEventCreate(&e), "csv: profile events");
    x.prof = on;
    for (int k = 0; k < 3; ++k) {
        x.recorded[k] = false;
        x.launches[k] = 0;
        x.ms[k] = 0.0;
    }
    return Status::ok();
}

Status profile_read(int device, const char *kernel, uint64_t *launches, double *ms) {
    if (device < 0 || device >= kMaxDevices) return Status::fail(TSFM_ERR_NO_DEVICE, "csv: device ordinal");
    if (kernel == nullptr || launches == nullptr || ms == nullptr)
        return Status::fail(TSFM_ERR_INVALID_ARGUMENT, "csv: null profile argument");
    const std::string k = kernel;
    const int id = k == "describe" ? K_DESCRIBE : k == "scan" ? K_SCAN : k == "text" ? K_TEXT : -1;
    if (id < 0) return Status::fail(TSFM_ERR_INVALID_ARGUMENT, "csv: kernel is one of describe, scan, text");
    Ctx &x = g_ctx[device];
    std::lock_guard<std::mutex> lock(x.mu);
    *launches = x.launches[id];
    *ms = x.ms[id];
    return Status::ok();
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

int32_t tsfm_csv_format(const float *values, size_t series, size_t variates, size_t horizon, const double *levels,
                        size_t num_levels, int32_t device, char *out, size_t capacity, size_t *length) {
    return tsfm::guarded([&] {
        return tsfm::format_host(device, values, series, variates, horizon, levels, num_levels, out, capacity, length);
    });
}

int32_t tsfm_csv_write(const float *values, size_t series, size_t variates, size_t horizon, const double *levels,
                       size_t num_levels, int32_t device, int32_t fd, size_t *length) {
    return tsfm::guarded([&] {
        return tsfm::write_fd(device, values, series, variates, horizon, levels, num_levels, fd, length);
    });
}

int32_t tsfm_csv_format_device(const float *values, size_t series, size_t variates, size_t horizon,
                               const double *levels, size_t num_levels, char *out, size_t capacity, size_t *length,
                               void *stream) {
    return tsfm::guarded([&] {
        return tsfm::format_device(values, series, variates, horizon, levels, num_levels, out, capacity, length,
                                   static_cast<cudaStream_t>(stream));
    });
}

int32_t tsfm_csv_profile_enable(int32_t device, int32_t enable) {
    return tsfm::guarded([&] { return tsfm::profile_enable(device, enable != 0); });
}

int32_t tsfm_csv_profile_read(int32_t device, const char *kernel, uint64_t *launches, double *ms) {
    return tsfm::guarded([&] { return tsfm::profile_read(device, kernel, launches, ms); });
}

}  // extern "C"
