// CSV output of a forecast on the GPU: the reference CLI's writeCsv (src/main.zig:181-198).
//
// Text layout: a header "series,variate,step" + ",q<level>" per quantile level, then one line
// per (series, variate, step) in row-major order: "s,v,step+1" + ",<value>" per level, each
// line ended by '\n'. Levels are f64 and values f32, both printed as Zig's "{d}" (decimal
// notation, shortest round-trip digits; csv_digits.cuh).
//
// Three kernels per chunk of lines: (1) one warp per line sums the text lengths of the line's
// numbers (block sums of 32 lines); (2) one block scans the block sums into byte offsets; (3) one
// warp per line renders the line into a shared-memory buffer and copies it to its offset with
// consecutive byte stores. The digit generation runs twice (lengths, then text) instead of
// keeping 8 bytes per value between the passes: it is cheaper than the HBM round trip.
#include <cuda_runtime.h>
#include <errno.h>
#include <unistd.h>

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

constexpr int kWarps = 8, kLinesPerWarp = 4, kLinesPerBlock = kWarps * kLinesPerWarp;
constexpr int kPrefixMax = 3 * 20 + 3;  // "s,v,step\n" with 20-digit integers
constexpr int kValueMax = 50;           // ',' + at most 49 bytes of f32 text ("-0.000...0ddddddddd")

struct Lines {
    const float *values;  // (lines, q) f32 of this chunk
    int64_t first;        // global index of the chunk's first line
    int64_t lines;
    int64_t variates, horizon;
    int q;
};

struct Prefix {
    uint64_t s, v, step;
    int ls, lv, lst, len;
};

__device__ __forceinline__ Prefix prefix_of(int64_t line, int64_t variates, int64_t horizon) {
    Prefix p;
    p.s = (uint64_t)(line / (variates * horizon));
    p.v = (uint64_t)((line / horizon) % variates);
    p.step = (uint64_t)(line % horizon) + 1;
    p.ls = csv::u64_length(p.s);
    p.lv = csv::u64_length(p.v);
    p.lst = csv::u64_length(p.step);
    p.len = p.ls + p.lv + p.lst + 3;  // two commas and the newline
    return p;
}

__device__ __forceinline__ void load_tables(csv::Pow5Tables *t) {
    const uint64_t *src = reinterpret_cast<const uint64_t *>(&c_pow5);
    uint64_t *dst = reinterpret_cast<uint64_t *>(t);
    for (int i = threadIdx.x; i < (int)(sizeof(csv::Pow5Tables) / 8); i += blockDim.x) dst[i] = src[i];
}

// (1) line lengths and per-block sums.
__global__ void __launch_bounds__(kWarps * 32) csv_len_kernel(Lines c, uint32_t *line_len, uint32_t *block_sum) {
    __shared__ csv::Pow5Tables tab;
    __shared__ uint32_t wsum[kWarps];
    load_tables(&tab);
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t base = (int64_t)blockIdx.x * kLinesPerBlock + warp * kLinesPerWarp;
    const uint32_t *bits = reinterpret_cast<const uint32_t *>(c.values);
    uint32_t mine = 0;
    for (int li = 0; li < kLinesPerWarp; ++li) {
        const int64_t line = base + li;
        if (line >= c.lines) break;
        uint32_t len = 0;
        for (int j = lane; j < c.q; j += 32) len += 1 + (uint32_t)csv::describe(bits[line * c.q + j], tab).len;
        for (int o = 16; o > 0; o >>= 1) len += __shfl_xor_sync(0xffffffffu, len, o);
        if (lane == 0) {
            len += (uint32_t)prefix_of(c.first + line, c.variates, c.horizon).len;
            line_len[line] = len;
            mine += len;
        }
    }
    if (lane == 0) wsum[warp] = mine;
    __syncthreads();
    if (threadIdx.x == 0) {
        uint32_t t = 0;
        for (int w = 0; w < kWarps; ++w) t += wsum[w];
        block_sum[blockIdx.x] = t;
    }
}

// (2) exclusive scan of the block sums (one block of 1024 threads) and the chunk's byte total.
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

// (3) text. Dynamic shared memory: the tables, 32 line offsets, one line buffer per warp.
__global__ void __launch_bounds__(kWarps * 32) csv_write_kernel(Lines c, const uint32_t *line_len,
                                                               const uint64_t *block_off, char *out, int buf_bytes) {
    extern __shared__ __align__(16) unsigned char smem[];
    csv::Pow5Tables &tab = *reinterpret_cast<csv::Pow5Tables *>(smem);
    uint64_t *line_off = reinterpret_cast<uint64_t *>(smem + sizeof(csv::Pow5Tables));
    char *bufs = reinterpret_cast<char *>(line_off + kLinesPerBlock);
    load_tables(&tab);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t first = (int64_t)blockIdx.x * kLinesPerBlock;
    if (warp == 0) {
        const int64_t line = first + lane;
        const uint64_t v = line < c.lines ? line_len[line] : 0;
        uint64_t x = v;
        for (int o = 1; o < 32; o <<= 1) {
            const uint64_t y = __shfl_up_sync(0xffffffffu, x, o);
            if (lane >= o) x += y;
        }
        line_off[lane] = block_off[blockIdx.x] + x - v;
    }
    __syncthreads();
    char *buf = bufs + (size_t)warp * buf_bytes;
    const uint32_t *bits = reinterpret_cast<const uint32_t *>(c.values);
    for (int li = 0; li < kLinesPerWarp; ++li) {
        const int lb = warp * kLinesPerWarp + li;
        const int64_t line = first + lb;
        if (line >= c.lines) break;
        const Prefix p = prefix_of(c.first + line, c.variates, c.horizon);
        if (lane == 0) {
            csv::emit_u64(p.s, p.ls, buf);
            buf[p.ls] = ',';
            csv::emit_u64(p.v, p.lv, buf + p.ls + 1);
            buf[p.ls + 1 + p.lv] = ',';
            csv::emit_u64(p.step, p.lst, buf + p.ls + p.lv + 2);
        }
        int pos = p.len - 1;
        for (int j0 = 0; j0 < c.q; j0 += 32) {
            const int j = j0 + lane;
            csv::F32Text f{};
            int n = 0;
            if (j < c.q) {
                f = csv::describe(bits[line * c.q + j], tab);
                n = 1 + f.len;
            }
            int x = n;
            for (int o = 1; o < 32; o <<= 1) {
                const int y = __shfl_up_sync(0xffffffffu, x, o);
                if (lane >= o) x += y;
            }
            if (j < c.q) {
                char *at = buf + pos + x - n;
                at[0] = ',';
                csv::emit(f, at + 1);
            }
            pos += __shfl_sync(0xffffffffu, x, 31);
        }
        if (lane == 0) buf[pos] = '\n';
        const int len = pos + 1;
        __syncwarp();
        char *dst = out + line_off[lb];
        for (int i = lane; i < len; i += 32) dst[i] = buf[i];
        __syncwarp();
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

// Per-device state: a stream, the tables, scratch and staging buffers (grown on demand).
struct Ctx {
    std::mutex mu;
    bool ready = false;
    cudaStream_t stream = nullptr;
    float *d_values = nullptr;
    size_t values_cap = 0;
    uint32_t *d_line_len = nullptr, *d_block_sum = nullptr;
    uint64_t *d_block_off = nullptr, *d_total = nullptr;
    size_t lines_cap = 0;
    char *d_text = nullptr;
    size_t text_cap = 0;
    char *h_text[2] = {nullptr, nullptr};
    size_t h_text_cap = 0;
    uint64_t *h_total = nullptr;
    // Optional per-kernel device time (CUDA events around each launch; read after each sync).
    bool prof = false;
    cudaEvent_t ev[6] = {};
    bool recorded[3] = {false, false, false};
    uint64_t launches[3] = {0, 0, 0};
    double ms[3] = {0, 0, 0};
};

enum { K_LENGTH = 0, K_SCAN = 1, K_TEXT = 2 };

void prof_mark(Ctx &x, int k, bool end, cudaStream_t s) {
    if (!x.prof) return;
    cudaEventRecord(x.ev[2 * k + (end ? 1 : 0)], s);
    if (end) x.recorded[k] = true;
}

// After a stream synchronisation: adds the recorded launches' times.
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

Status ctx_init(Ctx &x, int device) {
    TSFM_CUDA(cudaSetDevice(device), "csv: cudaSetDevice");
    if (x.ready) return Status::ok();
    const csv::Pow5Tables t = make_tables();
    TSFM_CUDA(cudaMemcpyToSymbol(c_pow5, &t, sizeof t), "csv: tables");
    TSFM_CUDA(cudaStreamCreateWithFlags(&x.stream, cudaStreamNonBlocking), "csv: stream");
    TSFM_CUDA(cudaMallocHost(reinterpret_cast<void **>(&x.h_total), 16), "csv: pinned total");
    x.ready = true;
    return Status::ok();
}

Status ensure_lines(Ctx &x, int64_t lines) {
    const size_t cap = (size_t)lines + kLinesPerBlock;
    if (x.lines_cap >= cap) return Status::ok();
    size_t dummy = 0;
    const size_t blocks = cap / kLinesPerBlock + 1;
    TSFM_TRY(grow_dev(&x.d_line_len, &dummy, cap * 4, "csv: line lengths"));
    dummy = 0;
    TSFM_TRY(grow_dev(&x.d_block_sum, &dummy, blocks * 4, "csv: block sums"));
    dummy = 0;
    TSFM_TRY(grow_dev(&x.d_block_off, &dummy, blocks * 8, "csv: block offsets"));
    dummy = 0;
    TSFM_TRY(grow_dev(&x.d_total, &dummy, 16, "csv: total"));
    x.lines_cap = cap;
    return Status::ok();
}

int line_buffer_bytes(int q) { return (kPrefixMax + kValueMax * q + 1 + 15) / 16 * 16; }

size_t write_smem_bytes(int q) {
    return sizeof(csv::Pow5Tables) + kLinesPerBlock * 8 + (size_t)kWarps * line_buffer_bytes(q);
}

// Largest level count whose line buffers fit in shared memory.
constexpr int kMaxLevels = 500;

// Lengths, offsets and total of `lines` lines at values (device); then the text into out
// (device) unless out is null. The total lands in x.d_total.
Status run_lengths(Ctx &x, const Lines &c, cudaStream_t s) {
    const int64_t blocks = (c.lines + kLinesPerBlock - 1) / kLinesPerBlock;
    if (blocks == 0) {
        TSFM_CUDA(cudaMemsetAsync(x.d_total, 0, 8, s), "csv: total");
        return Status::ok();
    }
    prof_mark(x, K_LENGTH, false, s);
    csv_len_kernel<<<(unsigned)blocks, kWarps * 32, 0, s>>>(c, x.d_line_len, x.d_block_sum);
    TSFM_CUDA(cudaGetLastError(), "csv: length kernel");
    prof_mark(x, K_LENGTH, true, s);
    prof_mark(x, K_SCAN, false, s);
    csv_scan_kernel<<<1, 1024, 0, s>>>(x.d_block_sum, blocks, x.d_block_off, x.d_total);
    TSFM_CUDA(cudaGetLastError(), "csv: scan kernel");
    prof_mark(x, K_SCAN, true, s);
    return Status::ok();
}

Status run_text(Ctx &x, const Lines &c, char *out, cudaStream_t s) {
    const int64_t blocks = (c.lines + kLinesPerBlock - 1) / kLinesPerBlock;
    if (blocks == 0) return Status::ok();
    const size_t smem = write_smem_bytes(c.q);
    static std::once_flag once[kMaxDevices];
    int dev = 0;
    TSFM_CUDA(cudaGetDevice(&dev), "csv: device");
    cudaError_t attr = cudaSuccess;
    std::call_once(once[dev % kMaxDevices], [&] {
        attr = cudaFuncSetAttribute(csv_write_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    (int)write_smem_bytes(kMaxLevels));
    });
    TSFM_CUDA(attr, "csv: shared memory attribute");
    prof_mark(x, K_TEXT, false, s);
    csv_write_kernel<<<(unsigned)blocks, kWarps * 32, smem, s>>>(c, x.d_line_len, x.d_block_off, out,
                                                                  line_buffer_bytes(c.q));
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

// Lines per chunk of the host entry points: 64 MiB of values (and at least one block).
int64_t chunk_lines(int q) {
    const int64_t per = std::max<int64_t>(1, (int64_t)q) * 4;
    return std::max<int64_t>(kLinesPerBlock, ((int64_t)64 << 20) / per / kLinesPerBlock * kLinesPerBlock);
}

// The host entry points' loop: per chunk, values in, lengths, total back; then `sink` gets the
// chunk's byte count and renders / delivers the text.
template <class Sink>
Status for_chunks(Ctx &x, const float *values, int64_t lines, int64_t variates, int64_t horizon, int q, Sink &&sink) {
    const int64_t chunk = chunk_lines(q);
    const size_t text_max = (size_t)std::min<int64_t>(chunk, lines) * (size_t)line_buffer_bytes(q);
    TSFM_TRY(ensure_lines(x, std::min<int64_t>(chunk, lines)));
    TSFM_TRY(grow_dev(&x.d_values, &x.values_cap, (size_t)std::min<int64_t>(chunk, lines) * q * 4 + 16, "csv: values"));
    TSFM_TRY(grow_dev(&x.d_text, &x.text_cap, text_max + 16, "csv: text"));
    cudaStream_t s = x.stream;
    for (int64_t l0 = 0; l0 < lines; l0 += chunk) {
        const int64_t n = std::min<int64_t>(chunk, lines - l0);
        if (q > 0)
            TSFM_CUDA(cudaMemcpyAsync(x.d_values, values + l0 * q, (size_t)n * q * 4, cudaMemcpyHostToDevice, s),
                      "csv: values in");
        Lines c{x.d_values, l0, n, variates, horizon, q};
        TSFM_TRY(run_lengths(x, c, s));
        TSFM_CUDA(cudaMemcpyAsync(x.h_total, x.d_total, 8, cudaMemcpyDeviceToHost, s), "csv: total out");
        TSFM_CUDA(cudaStreamSynchronize(s), "csv: lengths");
        prof_collect(x);
        TSFM_TRY(sink(c, (size_t)*x.h_total));
    }
    return Status::ok();
}

Status format_host(int device, const float *values, size_t series, size_t variates, size_t horizon,
                   const double *levels, size_t nq, char *out, size_t capacity, size_t *length) {
    TSFM_TRY(check_shape(values, series, variates, horizon, levels, nq, length));
    if (out == nullptr && capacity > 0) return Status::fail(TSFM_ERR_INVALID_ARGUMENT, "csv: out is null");
    if (device < 0 || device >= kMaxDevices) return Status::fail(TSFM_ERR_NO_DEVICE, "csv: device ordinal");
    Ctx &x = g_ctx[device];
    std::lock_guard<std::mutex> lock(x.mu);
    TSFM_TRY(ctx_init(x, device));
    const std::string head = header_text(levels, nq);
    size_t pos = head.size();
    bool fits = pos <= capacity;
    if (fits) std::memcpy(out, head.data(), head.size());
    const int64_t lines = (int64_t)(series * variates * horizon);
    TSFM_TRY(for_chunks(x, values, lines, (int64_t)variates, (int64_t)horizon, (int)nq,
                        [&](const Lines &c, size_t bytes) -> Status {
                            if (fits && pos + bytes <= capacity) {
                                TSFM_TRY(run_text(x, c, x.d_text, x.stream));
                                TSFM_CUDA(cudaMemcpyAsync(out + pos, x.d_text, bytes, cudaMemcpyDeviceToHost, x.stream),
                                          "csv: text out");
                                TSFM_CUDA(cudaStreamSynchronize(x.stream), "csv: text");
                                prof_collect(x);
                            } else {
                                fits = false;
                            }
                            pos += bytes;
                            return Status::ok();
                        }));
    *length = pos;
    if (!fits)
        return Status::fail(TSFM_ERR_BUFFER_TOO_SMALL,
                            "csv: the text needs " + std::to_string(pos) + " bytes, capacity " + std::to_string(capacity));
    return Status::ok();
}

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
    size_t pos = head.size();
    const int64_t lines = (int64_t)(series * variates * horizon);
    TSFM_TRY(for_chunks(x, values, lines, (int64_t)variates, (int64_t)horizon, (int)nq,
                        [&](const Lines &c, size_t bytes) -> Status {
                            if (x.h_text_cap < bytes) {
                                if (x.h_text[0]) cudaFreeHost(x.h_text[0]);
                                x.h_text[0] = nullptr;
                                x.h_text_cap = 0;
                                TSFM_CUDA(cudaMallocHost(reinterpret_cast<void **>(&x.h_text[0]), bytes),
                                          "csv: pinned text");
                                x.h_text_cap = bytes;
                            }
                            TSFM_TRY(run_text(x, c, x.d_text, x.stream));
                            TSFM_CUDA(cudaMemcpyAsync(x.h_text[0], x.d_text, bytes, cudaMemcpyDeviceToHost, x.stream),
                                      "csv: text out");
                            TSFM_CUDA(cudaStreamSynchronize(x.stream), "csv: text");
                            prof_collect(x);
                            TSFM_TRY(write_all(fd, x.h_text[0], bytes));
                            pos += bytes;
                            return Status::ok();
                        }));
    *length = pos;
    return Status::ok();
}

Status format_device(const float *values, size_t series, size_t variates, size_t horizon, const double *levels,
                     size_t nq, char *out, size_t capacity, size_t *length, cudaStream_t user_stream) {
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
    TSFM_TRY(ensure_lines(x, lines));
    Lines c{values, 0, lines, (int64_t)variates, (int64_t)horizon, (int)nq};
    TSFM_TRY(run_lengths(x, c, user_stream));
    TSFM_CUDA(cudaMemcpyAsync(x.h_total, x.d_total, 8, cudaMemcpyDeviceToHost, user_stream), "csv: total out");
    TSFM_CUDA(cudaStreamSynchronize(user_stream), "csv: lengths");
    prof_collect(x);
    const size_t total = head.size() + (size_t)*x.h_total;
    *length = total;
    if (total > capacity)
        return Status::fail(TSFM_ERR_BUFFER_TOO_SMALL,
                            "csv: the text needs " + std::to_string(total) + " bytes, capacity " + std::to_string(capacity));
    TSFM_CUDA(cudaMemcpyAsync(out, head.data(), head.size(), cudaMemcpyHostToDevice, user_stream), "csv: header");
    TSFM_TRY(run_text(x, c, out + head.size(), user_stream));
    TSFM_CUDA(cudaStreamSynchronize(user_stream), "csv: text");
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
    const int id = k == "length" ? K_LENGTH : k == "scan" ? K_SCAN : k == "text" ? K_TEXT : -1;
    if (id < 0) return Status::fail(TSFM_ERR_INVALID_ARGUMENT, "csv: kernel is one of length, scan, text");
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
