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

struct Replica {
    int device = 0;
    cudaStream_t stream = nullptr;
    cudaStream_t copy = nullptr;      // host<->device copies that overlap the forward on `stream`
    std::vector<cudaEvent_t> events;  // chunk hand-offs between the two streams
    DevBuf err;  // device error word(s)
    std::vector<DevBuf> weights;
    Arena ws;   // per-chunk model workspace
    Arena fc;   // forecaster buffers that live across chunks (Bolt quantile paths)
    DevBuf io;  // device copies of host inputs / outputs
    PinnedBuf pin_in, pin_out;
    Profiler prof;
    std::mutex mu;
    ~Replica();
};

// Checkpoint tensor table (core/safetensors.zig:59-97 semantics).
struct TensorTable {
    std::map<std::string, const tsfm_tensor *> by_name;
    TensorTable(const tsfm_tensor *t, size_t n);
    Status get(const std::string &name, size_t numel, std::vector<float> &out) const;
    // Presence, dtype and element count only (no conversion): lets a model be checked before
    // any device is touched.
    Status check(const std::string &name, size_t numel) const;
};

// Upload helpers (run with the replica's device current).
Status upload_f32(Replica &r, const std::vector<float> &h, float **out);
Status upload_lin(Replica &r, const std::vector<float> &w, int64_t out, int64_t in, int dtype, DLin &dst);
// a (m, k) times b (k, n), row-major, accumulated in float64 and rounded to float32 once per
// element; rows split across host threads.
std::vector<float> matmul_f64(const std::vector<float> &a, const std::vector<float> &b, int64_t m, int64_t k, int64_t n);
Status upload_bias(Replica &r, const std::vector<float> &b, DLin &dst);
Status upload_lin3(Replica &r, const std::vector<float> &w, int64_t out, int64_t in, DLin3 &dst);

// Checks the device error word after a stream sync.
Status check_device_error(Replica &r);

std::string strf(const char *fmt, ...);

// Records `s` as the calling thread's last error (read by tsfm_last_error) and returns its code.
int32_t set_last_error(const Status &s);

}  // namespace tsfm
