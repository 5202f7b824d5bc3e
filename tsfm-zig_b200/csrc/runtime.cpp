#include "runtime.h"

#include <cstdlib>

#include <algorithm>
#include <cmath>
#include <cstdarg>
#include <cstring>

#include <cuda_fp16.h>

namespace tsfm {

std::string strf(const char *fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    return buf;
}

Status DevBuf::alloc(size_t n) {
    reset();
    if (n == 0) return Status::ok();
    cudaError_t e = cudaMalloc(&p, n);
    if (e != cudaSuccess) {
        p = nullptr;
        return Status::cuda(e, strf("cudaMalloc(%zu)", n));
    }
    bytes = n;
    return Status::ok();
}

Status PinnedBuf::ensure(size_t n) {
    if (n <= bytes) return Status::ok();
    if (p) cudaFreeHost(p);
    p = nullptr;
    bytes = 0;
    cudaError_t e = cudaMallocHost(&p, n);
    if (e != cudaSuccess) {
        p = nullptr;
        return Status::cuda(e, strf("cudaMallocHost(%zu)", n));
    }
    bytes = n;
    return Status::ok();
}

Status Arena::reserve(size_t bytes) {
    used = 0;
    if (bytes <= buf.bytes) return Status::ok();
    return buf.alloc(bytes);
}

const char *kclass_name(int c) {
    static const char *names[6] = {"gemm", "attention", "rmsnorm", "patch", "head", "other"};
    return c >= 0 && c < 6 ? names[c] : "other";
}

Profiler::~Profiler() {
    for (auto &r : pending) {
        cudaEventDestroy(r.a);
        cudaEventDestroy(r.b);
    }
    for (auto e : pool) cudaEventDestroy(e);
}

cudaEvent_t Profiler::take() {
    if (!pool.empty()) {
        cudaEvent_t e = pool.back();
        pool.pop_back();
        return e;
    }
    cudaEvent_t e = nullptr;
    cudaEventCreate(&e);
    return e;
}

void Profiler::collect() {
    for (auto &r : pending) {
        float t = 0.0f;
        if (cudaEventElapsedTime(&t, r.a, r.b) == cudaSuccess) ms[r.cls] += t;
        pool.push_back(r.a);
        pool.push_back(r.b);
    }
    pending.clear();
}

LaunchScope::LaunchScope(Replica &rep, cudaStream_t st, int c, double w) : r(rep), cls(c), work(w), s(st) {
    r.prof.launches[cls] += 1;
    r.prof.work[cls] += w;
    r.prof.cur_launches += 1;
    if (r.prof.enabled) {
        a = r.prof.take();
        b = r.prof.take();
        cudaEventRecord(a, s);
    }
}

LaunchScope::~LaunchScope() {
    if (a) {
        cudaEventRecord(b, s);
        r.prof.pending.push_back({cls, work, a, b});
    }
}

GraphCache::Entry *GraphCache::find(const std::vector<uint64_t> &key) {
    for (auto &e : entries)
        if (e.key == key) return &e;
    return nullptr;
}

GraphCache::Entry *GraphCache::insert(const std::vector<uint64_t> &key) {
    if (entries.size() >= kMax) {
        size_t lru = 0;
        for (size_t i = 1; i < entries.size(); ++i)
            if (entries[i].used < entries[lru].used) lru = i;
        if (entries[lru].exec) cudaGraphExecDestroy(entries[lru].exec);
        entries.erase(entries.begin() + (std::ptrdiff_t)lru);
    }
    entries.push_back(Entry{});
    entries.back().key = key;
    entries.back().used = ++clock;
    return &entries.back();
}

GraphCache::~GraphCache() {
    for (auto &e : entries)
        if (e.exec) cudaGraphExecDestroy(e.exec);
}

bool graphs_enabled() {
    static const bool on = [] {
        const char *v = std::getenv("TSFM_CUDA_GRAPHS");
        return !(v && v[0] == '0');
    }();
    return on;
}

Replica::~Replica() {
    cudaSetDevice(device);
    for (cudaEvent_t e : events) cudaEventDestroy(e);
    if (copy) cudaStreamDestroy(copy);
    if (stream) cudaStreamDestroy(stream);
}

TensorTable::TensorTable(const tsfm_tensor *t, size_t n) {
    for (size_t i = 0; i < n; ++i)
        if (t[i].name) by_name[t[i].name] = &t[i];
}

static float half_bits_to_float(uint16_t h) {
    const uint32_t sign = (uint32_t)(h & 0x8000) << 16;
    uint32_t exp = (h >> 10) & 0x1f, mant = h & 0x3ff, bits;
    if (exp == 0) {
        if (mant == 0) {
            bits = sign;
        } else {
            int e = -1;
            do {
                ++e;
                mant <<= 1;
            } while ((mant & 0x400) == 0);
            mant &= 0x3ff;
            bits = sign | ((uint32_t)(127 - 15 - e) << 23) | (mant << 13);
        }
    } else if (exp == 31) {
        bits = sign | 0x7f800000u | (mant << 13);
    } else {
        bits = sign | ((exp + 112) << 23) | (mant << 13);
    }
    float f;
    std::memcpy(&f, &bits, 4);
    return f;
}

Status TensorTable::check(const std::string &name, size_t numel) const {
    auto it = by_name.find(name);
    if (it == by_name.end()) return Status::fail(TSFM_ERR_MISSING_TENSOR, "missing tensor: " + name);
    const tsfm_tensor *t = it->second;
    if (t->dtype != TSFM_DTYPE_F32 && t->dtype != TSFM_DTYPE_F16 && t->dtype != TSFM_DTYPE_BF16)
        return Status::fail(TSFM_ERR_UNSUPPORTED_DTYPE, "tensor " + name + " has unsupported dtype");
    if (t->numel != numel)
        return Status::fail(TSFM_ERR_SHAPE_MISMATCH, strf("tensor %s: expected %zu elements, file has %llu",
                                                          name.c_str(), numel, (unsigned long long)t->numel));
    if (!t->data && numel) return Status::fail(TSFM_ERR_INVALID_ARGUMENT, "tensor " + name + " has no data");
    return Status::ok();
}

Status TensorTable::get(const std::string &name, size_t numel, std::vector<float> &out) const {
    auto it = by_name.find(name);
    if (it == by_name.end()) return Status::fail(TSFM_ERR_MISSING_TENSOR, "missing tensor: " + name);
    const tsfm_tensor *t = it->second;
    if (t->dtype != TSFM_DTYPE_F32 && t->dtype != TSFM_DTYPE_F16 && t->dtype != TSFM_DTYPE_BF16)
        return Status::fail(TSFM_ERR_UNSUPPORTED_DTYPE, "tensor " + name + " has unsupported dtype");
    if (t->numel != numel)
        return Status::fail(TSFM_ERR_SHAPE_MISMATCH, strf("tensor %s: expected %zu elements, file has %llu",
                                                          name.c_str(), numel, (unsigned long long)t->numel));
    if (!t->data && numel) return Status::fail(TSFM_ERR_INVALID_ARGUMENT, "tensor " + name + " has no data");
    out.resize(numel);
    if (t->dtype == TSFM_DTYPE_F32) {
        std::memcpy(out.data(), t->data, numel * 4);
    } else {
        const uint16_t *s = static_cast<const uint16_t *>(t->data);
        for (size_t i = 0; i < numel; ++i) {
            if (t->dtype == TSFM_DTYPE_BF16) {
                const uint32_t bits = (uint32_t)s[i] << 16;
                std::memcpy(&out[i], &bits, 4);
            } else {
                out[i] = half_bits_to_float(s[i]);
            }
        }
    }
    return Status::ok();
}

Status TensorTable::raw(const std::string &name, size_t numel, const tsfm_tensor **out) const {
    auto it = by_name.find(name);
    if (it == by_name.end()) return Status::fail(TSFM_ERR_MISSING_TENSOR, "missing tensor: " + name);
    const tsfm_tensor *t = it->second;
    if (t->dtype != TSFM_DTYPE_F32 && t->dtype != TSFM_DTYPE_F16 && t->dtype != TSFM_DTYPE_BF16)
        return Status::fail(TSFM_ERR_UNSUPPORTED_DTYPE, "tensor " + name + " has unsupported dtype");
    if (t->numel != numel)
        return Status::fail(TSFM_ERR_SHAPE_MISMATCH, strf("tensor %s: expected %zu elements, file has %llu",
                                                          name.c_str(), numel, (unsigned long long)t->numel));
    if (!t->data && numel) return Status::fail(TSFM_ERR_INVALID_ARGUMENT, "tensor " + name + " has no data");
    *out = t;
    return Status::ok();
}

static int elem_of(const tsfm_tensor *t) {
    return t->dtype == TSFM_DTYPE_F32 ? E_F32 : t->dtype == TSFM_DTYPE_F16 ? E_F16 : E_BF16;
}

// Copies the tensors as stored, back to back, into the replica's staging buffer after `extra`
// leading bytes left free; returns where the first one starts.
static Status stage_tensors(Replica &r, const std::vector<const tsfm_tensor *> &parts, size_t extra, char **first) {
    const size_t esz = elem_of(parts[0]) == E_F32 ? 4 : 2;
    size_t bytes = extra;
    for (const tsfm_tensor *t : parts) bytes += Arena::span((size_t)t->numel * esz);
    if (r.stage.bytes < bytes) TSFM_TRY(r.stage.alloc(bytes));
    char *dst = static_cast<char *>(r.stage.p) + extra;
    *first = dst;
    for (const tsfm_tensor *t : parts) {
        const size_t n = (size_t)t->numel * esz;
        TSFM_CUDA(cudaMemcpyAsync(dst, t->data, n, cudaMemcpyHostToDevice, r.stream), "stage weight");
        dst += n;
    }
    return Status::ok();
}

Status upload_lin_raw(Replica &r, const std::vector<const tsfm_tensor *> &parts, const std::vector<int32_t> *map,
                      int64_t out, int64_t in, int dtype, DLin &dst) {
    if (parts.empty()) return Status::fail(TSFM_ERR_INVALID_ARGUMENT, "weight upload: no tensors");
    int64_t rows = 0;
    bool same = true;
    for (const tsfm_tensor *t : parts) {
        if ((int64_t)t->numel % in) return Status::fail(TSFM_ERR_SHAPE_MISMATCH, "weight upload: ragged rows");
        rows += (int64_t)t->numel / in;
        same = same && elem_of(t) == elem_of(parts[0]);
    }
    if (map ? (int64_t)map->size() != out : rows != out)
        return Status::fail(TSFM_ERR_SHAPE_MISMATCH, "weight upload: row count");
    if (!same) {
        // Mixed storage types: convert on the host (rare).
        std::vector<float> all((size_t)(rows * in));
        size_t off = 0;
        for (const tsfm_tensor *t : parts) {
            for (size_t i = 0; i < (size_t)t->numel; ++i) {
                const int dt = elem_of(t);
                if (dt == E_F32) {
                    all[off + i] = static_cast<const float *>(t->data)[i];
                } else {
                    const uint16_t u = static_cast<const uint16_t *>(t->data)[i];
                    if (dt == E_BF16) {
                        const uint32_t bits = (uint32_t)u << 16;
                        std::memcpy(&all[off + i], &bits, 4);
                    } else {
                        all[off + i] = half_bits_to_float(u);
                    }
                }
            }
            off += (size_t)t->numel;
        }
        if (!map) return upload_lin(r, all, out, in, dtype, dst);
        std::vector<float> perm((size_t)(out * in));
        for (int64_t i = 0; i < out; ++i)
            std::memcpy(&perm[(size_t)(i * in)], &all[(size_t)((*map)[(size_t)i] * in)], (size_t)in * 4);
        return upload_lin(r, perm, out, in, dtype, dst);
    }
    const size_t map_bytes = map ? Arena::span(map->size() * 4) : 0;
    char *src = nullptr;
    TSFM_TRY(stage_tensors(r, parts, map_bytes, &src));
    const int32_t *dmap = nullptr;
    if (map) {
        for (int32_t v : *map)
            if (v < 0 || v >= rows) return Status::fail(TSFM_ERR_INVALID_ARGUMENT, "weight upload: row map");
        TSFM_CUDA(cudaMemcpyAsync(r.stage.p, map->data(), map->size() * 4, cudaMemcpyHostToDevice, r.stream),
                  "stage row map");
        dmap = static_cast<const int32_t *>(r.stage.p);
    }
    DevBuf b;
    const bool corr = dtype == E_F16C;
    TSFM_TRY(b.alloc((size_t)(out * in) * (dtype == E_F32 || corr ? 4 : 2)));
    TSFM_TRY(launch_convert_rows(src, elem_of(parts[0]), dmap, b.p, corr ? E_F32X : dtype, out, in, r.stream));
    if (corr) {
        TSFM_TRY(upload_corrected(r, static_cast<const float *>(b.p), out, in, dst));
        TSFM_CUDA(cudaStreamSynchronize(r.stream), "weight upload");
        return Status::ok();
    }
    TSFM_CUDA(cudaStreamSynchronize(r.stream), "weight upload");
    dst.out = out;
    dst.in = in;
    dst.dtype = dtype;
    dst.w = b.p;
    r.weights.push_back(std::move(b));
    return Status::ok();
}

Status upload_fold_raw(Replica &r, const tsfm_tensor *a, const tsfm_tensor *b, int64_t m, int64_t k, int64_t n,
                       int dtype, DLin &dst) {
    if ((int64_t)a->numel != m * k || (int64_t)b->numel != k * n)
        return Status::fail(TSFM_ERR_SHAPE_MISMATCH, "weight fold: shapes");
    const size_t esz_a = elem_of(a) == E_F32 ? 4 : 2, esz_b = elem_of(b) == E_F32 ? 4 : 2;
    const size_t sa = Arena::span((size_t)a->numel * esz_a), sb = Arena::span((size_t)b->numel * esz_b);
    if (r.stage.bytes < sa + sb) TSFM_TRY(r.stage.alloc(sa + sb));
    char *pa = static_cast<char *>(r.stage.p), *pb = pa + sa;
    TSFM_CUDA(cudaMemcpyAsync(pa, a->data, (size_t)a->numel * esz_a, cudaMemcpyHostToDevice, r.stream), "stage weight");
    TSFM_CUDA(cudaMemcpyAsync(pb, b->data, (size_t)b->numel * esz_b, cudaMemcpyHostToDevice, r.stream), "stage weight");
    DevBuf w;
    const bool corr = dtype == E_F16C;
    TSFM_TRY(w.alloc((size_t)(m * n) * (dtype == E_F32 || corr ? 4 : 2)));
    TSFM_TRY(launch_fold_f64(pa, elem_of(a), pb, elem_of(b), w.p, corr ? E_F32X : dtype, m, k, n, r.stream));
    if (corr) {
        TSFM_TRY(upload_corrected(r, static_cast<const float *>(w.p), m, n, dst));
        TSFM_CUDA(cudaStreamSynchronize(r.stream), "weight fold");
        return Status::ok();
    }
    TSFM_CUDA(cudaStreamSynchronize(r.stream), "weight fold");
    dst.out = m;
    dst.in = n;
    dst.dtype = dtype;
    dst.w = w.p;
    r.weights.push_back(std::move(w));
    return Status::ok();
}

static uint16_t f32_to_bf16_rne(float f) {
    uint32_t u;
    std::memcpy(&u, &f, 4);
    if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40);  // quiet NaN
    u += 0x7fffu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}

static float f32_to_tf32_rna(float f) {
    uint32_t u;
    std::memcpy(&u, &f, 4);
    if ((u & 0x7f800000u) != 0x7f800000u) {
        u += 0x1000u;
        u &= ~0x1fffu;
    }
    float r;
    std::memcpy(&r, &u, 4);
    return r;
}

Status upload_f32(Replica &r, const std::vector<float> &h, float **out) {
    DevBuf b;
    TSFM_TRY(b.alloc(h.size() * 4));
    TSFM_CUDA(cudaMemcpy(b.p, h.data(), h.size() * 4, cudaMemcpyHostToDevice), "upload");
    *out = static_cast<float *>(b.p);
    r.weights.push_back(std::move(b));
    return Status::ok();
}

Status upload_corrected(Replica &r, const float *w32, int64_t out, int64_t in, DLin &dst) {
    if (in % 8) return Status::fail(TSFM_ERR_UNSUPPORTED, "corrected weights need in % 8 == 0");
    DevBuf w16, w8;
    TSFM_TRY(w16.alloc((size_t)(out * in) * 2));
    TSFM_TRY(w8.alloc((size_t)(out * in) * 2));
    int sh = 0;
    TSFM_TRY(build_corrected_weight(w32, out, in, w16.p, w8.p, &sh, r.stream));
    dst.out = out;
    dst.in = in;
    dst.dtype = E_F16;
    dst.w = w16.p;
    dst.w8 = w8.p;
    dst.acc_scale = std::ldexp(1.0f, -sh);
    r.weights.push_back(std::move(w16));
    r.weights.push_back(std::move(w8));
    return Status::ok();
}

Status upload_lin(Replica &r, const std::vector<float> &w, int64_t out, int64_t in, int dtype, DLin &dst) {
    DevBuf b;
    dst.out = out;
    dst.in = in;
    dst.dtype = dtype;
    if (dtype == E_F16C) {
        TSFM_TRY(b.alloc(w.size() * 4));
        TSFM_CUDA(cudaMemcpyAsync(b.p, w.data(), w.size() * 4, cudaMemcpyHostToDevice, r.stream), "upload weight");
        TSFM_TRY(upload_corrected(r, static_cast<const float *>(b.p), out, in, dst));
        TSFM_CUDA(cudaStreamSynchronize(r.stream), "upload weight");
        return Status::ok();
    }
    if (dtype == E_F16) {
        std::vector<__half> t(w.size());
        for (size_t i = 0; i < w.size(); ++i) t[i] = __float2half_rn(w[i]);
        TSFM_TRY(b.alloc(t.size() * 2));
        TSFM_CUDA(cudaMemcpy(b.p, t.data(), t.size() * 2, cudaMemcpyHostToDevice), "upload weight");
    } else if (dtype == E_F32) {
        std::vector<float> t(w.size());
        for (size_t i = 0; i < w.size(); ++i) t[i] = f32_to_tf32_rna(w[i]);
        TSFM_TRY(b.alloc(t.size() * 4));
        TSFM_CUDA(cudaMemcpy(b.p, t.data(), t.size() * 4, cudaMemcpyHostToDevice), "upload weight");
    } else {
        std::vector<uint16_t> t(w.size());
        for (size_t i = 0; i < w.size(); ++i) t[i] = f32_to_bf16_rne(w[i]);
        TSFM_TRY(b.alloc(t.size() * 2));
        TSFM_CUDA(cudaMemcpy(b.p, t.data(), t.size() * 2, cudaMemcpyHostToDevice), "upload weight");
    }
    dst.w = b.p;
    r.weights.push_back(std::move(b));
    return Status::ok();
}

Status upload_bias(Replica &r, const std::vector<float> &b, DLin &dst) { return upload_f32(r, b, &dst.b); }

Status upload_lin3(Replica &r, const std::vector<float> &w, int64_t out, int64_t in, DLin3 &dst) {
    std::vector<float> hi(w.size()), lo(w.size());
    for (size_t i = 0; i < w.size(); ++i) {
        hi[i] = f32_to_tf32_rna(w[i]);
        lo[i] = f32_to_tf32_rna(w[i] - hi[i]);
    }
    // upload_lin with E_F32 rounds to TF32 again, which leaves these values unchanged.
    TSFM_TRY(upload_lin(r, hi, out, in, E_F32, dst.hi));
    TSFM_TRY(upload_lin(r, lo, out, in, E_F32, dst.lo));
    return Status::ok();
}

Status check_device_error(Replica &r) {
    int code = 0;
    TSFM_CUDA(cudaMemcpy(&code, r.err.p, sizeof(int), cudaMemcpyDeviceToHost), "read device error word");
    if (code != 0) {
        const int zero = 0;
        cudaMemcpy(r.err.p, &zero, sizeof(int), cudaMemcpyHostToDevice);
        return Status::fail(TSFM_ERR_DEVICE_TIMEOUT,
                            strf("a kernel's bounded wait gave up (site 0x%04x) on device %d", code, r.device));
    }
    return Status::ok();
}

}  // namespace tsfm
