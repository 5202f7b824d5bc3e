// Host runtime shared by the family forwards: device buffers, per-device replicas, workspace
// arena, launch accounting and the checkpoint tensor table.
#pragma once

#include <cuda_runtime.h>

#include <map>
#include <memory>
#include <mutex>
#include <string>
#include <vector>

#include "kernels.h"

namespace tsfm {

// Owning device allocation.
struct DevBuf {
    void *p = nullptr;
    size_t bytes = 0;
    DevBuf() = default;
    DevBuf(const DevBuf &) = delete;
    DevBuf &operator=(const DevBuf &) = delete;
    DevBuf(DevBuf &&o) noexcept : p(o.p), bytes(o.bytes) {
        o.p = nullptr;
        o.bytes = 0;
    }
    DevBuf &operator=(DevBuf &&o) noexcept {
        if (this != &o) {
            reset();
            p = o.p;
            bytes = o.bytes;
            o.p = nullptr;
            o.bytes = 0;
        }
        return *this;
    }
    ~DevBuf() { reset(); }
    void reset() {
        if (p) cudaFree(p);
        p = nullptr;
        bytes = 0;
    }
    Status alloc(size_t n);
};

// Owning pinned host allocation (staging for host-pointer forecasts).
struct PinnedBuf {
    void *p = nullptr;
    size_t bytes = 0;
    ~PinnedBuf() {
        if (p) cudaFreeHost(p);
    }
    Status ensure(size_t n);
};

// A linear layer's device weight: W [out, in] in the operand type of its GEMM, FP32 bias.
struct DLin {
    void *w = nullptr;
    int dtype = E_BF16;  // E_BF16, E_F16, or E_F32 (stored TF32-rounded, read as TF32)
    int64_t out = 0, in = 0;
    float *b = nullptr;
    // Corrected product (uploaded as E_F16C): w holds f16(W) * 2^s, w8 [out, 2 in] its FP8
    // companion (kernels.h), acc_scale = 2^-s. Null for plain weights.
    void *w8 = nullptr;
    float acc_scale = 1.0f;
};

struct DResBlock {
    DLin hidden, output, residual;
};

// A weight split into two TF32 parts, w = hi + lo (hi = tf32(w), lo = tf32(w - hi)), for products
// that must keep FP32 accuracy: x w^T ~= x_hi w_hi + x_hi w_lo + x_lo w_hi. The bias rides on hi.
struct DLin3 {
    DLin hi, lo;
};

// Per-kernel-class launch accounting (optionally timed with CUDA events).
struct Profiler {
    bool enabled = false;
    struct Rec {
        int cls;
        double work;
        cudaEvent_t a, b;
    };
    std::vector<Rec> pending;
    std::vector<cudaEvent_t> pool;
    uint64_t launches[6] = {0};
    double ms[6] = {0};
    double work[6] = {0};
    uint64_t last_forecast_launches = 0;
    uint64_t cur_launches = 0;
    ~Profiler();
    cudaEvent_t take();
    void collect();  // after a stream sync
};

enum KClass { K_GEMM = 0, K_ATTN = 1, K_NORM = 2, K_PATCH = 3, K_HEAD = 4, K_OTHER = 5 };
const char *kclass_name(int c);

struct Replica;

// Records one launch of class `cls` doing `work` (FLOPs or bytes); brackets it with events when
// profiling is enabled.
struct LaunchScope {
    Replica &r;
    int cls;
    double work;
    cudaEvent_t a = nullptr, b = nullptr;
    cudaStream_t s;
    LaunchScope(Replica &rep, cudaStream_t st, int c, double w);
    ~LaunchScope();
};

// Grow-only workspace arena, 256-byte sub-allocations.
struct Arena {
    DevBuf buf;
    size_t used = 0;
    Status reserve(size_t bytes);
    void reset() { used = 0; }
    template <class T>
    T *take(size_t count) {
        const size_t bytes = (count * sizeof(T) + 255) & ~size_t(255);
        T *p = reinterpret_cast<T *>(static_cast<char *>(buf.p) + used);
        used += bytes;
        return p;
    }
    static size_t span(size_t bytes) { return (bytes + 255) & ~size_t(255); }
};

// Captured forwards. A forward's launch sequence depends only on its shapes and on the addresses of
// the buffers it touches, so after one plain run under a key (those shapes and addresses) the
// sequence is captured into a CUDA graph and later calls with the key replay it: one launch instead
// of ~126 per forward, which is what small batches pay for. TSFM_CUDA_GRAPHS=0 turns this off.
struct GraphCache {
    struct Entry {
        std::vector<uint64_t> key;
        cudaGraphExec_t exec = nullptr;
        uint64_t launches = 0;  // kernels in the graph
        uint64_t used = 0;      // LRU clock
        bool failed = false;    // capture not possible: always run plainly
    };
    std::vector<Entry> entries;
    uint64_t clock = 0;
    static constexpr size_t kMax = 16;
    Entry *find(const std::vector<uint64_t> &key);
    Entry *insert(const std::vector<uint64_t> &key);  // evicts the least recently used entry when full
    ~GraphCache();
};
bool graphs_enabled();

struct Replica {
    int device = 0;
    cudaStream_t stream = nullptr;
    cudaStream_t copy = nullptr;      // host<->device copies that overlap the forward on `stream`
    std::vector<cudaEvent_t> events;  // chunk hand-offs between the two streams
    DevBuf err;  // device error word(s)
    std::vector<DevBuf> weights;
    DevBuf stage;  // raw checkpoint bytes on their way to a device weight (load time only)
    Arena ws;   // per-chunk model workspace
    Arena fc;   // forecaster buffers that live across chunks (Bolt quantile paths)
    DevBuf io;  // device copies of host inputs / outputs
    PinnedBuf pin_in, pin_out;
    Profiler prof;
    GraphCache graphs;
    std::mutex mu;
    ~Replica();
};

// Runs `fwd(stream)` (a forward that enqueues kernels only: no allocation, copy or synchronisation)
// on `s`, through the replica's graph cache under `key` (see GraphCache). The capture itself runs
// on the replica's own stream, so `s` may be the legacy default stream.
template <class Fwd>
Status run_captured(Replica &r, cudaStream_t s, const std::vector<uint64_t> &key, Fwd &&fwd) {
    if (r.prof.enabled || !graphs_enabled()) return fwd(s);
    GraphCache::Entry *e = r.graphs.find(key);
    if (!e) {
        r.graphs.insert(key);
        return fwd(s);  // first sight: the plain run sizes the workspace and sets kernel attributes
    }
    if (e->failed) return fwd(s);
    if (!e->exec) {
        const uint64_t before = r.prof.cur_launches;
        cudaGraph_t g = nullptr;
        bool ok = cudaStreamBeginCapture(r.stream, cudaStreamCaptureModeThreadLocal) == cudaSuccess;
        if (ok) {
            const Status st = fwd(r.stream);
            ok = cudaStreamEndCapture(r.stream, &g) == cudaSuccess && st && g != nullptr;
        }
        if (ok) ok = cudaGraphInstantiate(&e->exec, g, 0) == cudaSuccess;
        if (g) cudaGraphDestroy(g);
        e->launches = r.prof.cur_launches - before;
        r.prof.cur_launches = before;
        if (!ok) {
            (void)cudaGetLastError();
            e->exec = nullptr;
            e->failed = true;
            return fwd(s);
        }
    }
    e->used = ++r.graphs.clock;
    r.prof.cur_launches += e->launches;
    TSFM_CUDA(cudaGraphLaunch(e->exec, s), "cudaGraphLaunch");
    return Status::ok();
}

// Checkpoint tensor table (core/safetensors.zig:59-97 semantics).
struct TensorTable {
    std::map<std::string, const tsfm_tensor *> by_name;
    TensorTable(const tsfm_tensor *t, size_t n);
    Status get(const std::string &name, size_t numel, std::vector<float> &out) const;
    // Presence, dtype and element count only (no conversion): lets a model be checked before
    // any device is touched.
    Status check(const std::string &name, size_t numel) const;
    // The tensor as stored, after the checks of get().
    Status raw(const std::string &name, size_t numel, const tsfm_tensor **out) const;
};

// Upload helpers (run with the replica's device current).
Status upload_f32(Replica &r, const std::vector<float> &h, float **out);
Status upload_lin(Replica &r, const std::vector<float> &w, int64_t out, int64_t in, int dtype, DLin &dst);
Status upload_bias(Replica &r, const std::vector<float> &b, DLin &dst);
// A device weight [out, in] from checkpoint tensors stacked by rows (each `in` columns wide), copied
// as stored and converted on the device to `dtype` (E_F16 / E_BF16; E_F32 = TF32-rounded; E_F16C =
// the corrected-product form). With `map`, output row r is stacked row (*map)[r]; without, out
// must equal the stacked row count.
Status upload_lin_raw(Replica &r, const std::vector<const tsfm_tensor *> &parts, const std::vector<int32_t> *map,
                      int64_t out, int64_t in, int dtype, DLin &dst);
// A device weight = a (m x k) b (k x n) formed in float64 on the device and rounded once (to
// float, then to `dtype`).
Status upload_fold_raw(Replica &r, const tsfm_tensor *a, const tsfm_tensor *b, int64_t m, int64_t k, int64_t n,
                       int dtype, DLin &dst);
Status upload_lin3(Replica &r, const std::vector<float> &w, int64_t out, int64_t in, DLin3 &dst);
// The corrected-product form (E_F16C) of an exact FP32 device weight [out, in]; `w32` stays the
// caller's.
Status upload_corrected(Replica &r, const float *w32, int64_t out, int64_t in, DLin &dst);

// Checks the device error word after a stream sync.
Status check_device_error(Replica &r);

std::string strf(const char *fmt, ...);

// Records `s` as the calling thread's last error (read by tsfm_last_error) and returns its code.
int32_t set_last_error(const Status &s);

}  // namespace tsfm
