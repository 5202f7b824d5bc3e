// The C ABI (include/tsfm_b200.h): argument checks, error reporting, model creation with one
// replica per device, series sharding across replicas (one host thread per device, no
// collective), host<->device staging, and the reference's GEMM seam.
#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <new>
#include <thread>

#include "model.h"
#include "ptx.cuh"
#include "timestral_kernels.h"

using namespace tsfm;

namespace {

thread_local std::string g_last_error;

int32_t report(const Status &s) {
    g_last_error = s.code ? s.msg : std::string();
    return s.code;
}

}  // namespace

namespace tsfm {
int32_t set_last_error(const Status &s) { return report(s); }
}  // namespace tsfm

namespace {

template <class F>
int32_t guarded(F &&f) {
    try {
        return report(f());
    } catch (const std::bad_alloc &) {
        return report(Status::fail(TSFM_ERR_OUT_OF_MEMORY, "host allocation failed"));
    } catch (const std::exception &e) {
        return report(Status::fail(TSFM_ERR_INVALID_ARGUMENT, e.what()));
    } catch (...) {
        return report(Status::fail(TSFM_ERR_INVALID_ARGUMENT, "unknown exception"));
    }
}

Status device_count(int *n) {
    *n = 0;
    cudaError_t e = cudaGetDeviceCount(n);
    if (e == cudaErrorNoDevice || e == cudaErrorInsufficientDriver) {
        cudaGetLastError();
        *n = 0;
        return Status::fail(TSFM_ERR_NO_DEVICE, std::string("no CUDA device: ") + cudaGetErrorString(e));
    }
    if (e != cudaSuccess) return Status::cuda(e, "cudaGetDeviceCount");
    if (*n == 0) return Status::fail(TSFM_ERR_NO_DEVICE, "no CUDA device");
    return Status::ok();
}

// Device error words for the kernel-level entry points (one per device, allocated once).
int *kernel_err_word() {
    static std::mutex mu;
    static int *words[64] = {nullptr};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return nullptr;
    std::lock_guard<std::mutex> lk(mu);
    if (!words[dev]) {
        void *p = nullptr;
        if (cudaMalloc(&p, 16) == cudaSuccess) {
            cudaMemset(p, 0, 16);
            words[dev] = static_cast<int *>(p);
        }
    }
    return words[dev];
}

bool is_pinned(const void *p) {
    cudaPointerAttributes a;
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    return a.type == cudaMemoryTypeHost;
}

// Runs fn(i) for every replica, one host thread per replica beyond the first; returns the first
// failure in replica order after all threads joined.
// Host-side failure injection for the tests of the sharded forecasts: with TSFM_FAIL_REPLICA=<i>
// the forecast worker of replica i fails before it touches its device, while the other workers
// run and are joined as usual (read on every call; unset in normal use).
Status injected_failure(size_t i) {
    const char *v = std::getenv("TSFM_FAIL_REPLICA");
    if (v && *v && std::strtoul(v, nullptr, 10) == i)
        return Status::fail(TSFM_ERR_INVALID_ARGUMENT, strf("injected failure in the worker of replica %zu", i));
    return Status::ok();
}

template <class F>
Status for_replicas(size_t n, F &&fn) {
    if (n == 1) return fn(0);
    std::vector<Status> st(n);
    std::vector<std::thread> th;
    for (size_t i = 1; i < n; ++i) th.emplace_back([&, i] {
        try {
            st[i] = fn(i);
        } catch (const std::bad_alloc &) {
            st[i] = Status::fail(TSFM_ERR_OUT_OF_MEMORY, "host allocation failed");
        } catch (...) {
            st[i] = Status::fail(TSFM_ERR_INVALID_ARGUMENT, "worker thread failed");
        }
    });
    st[0] = fn(0);
    for (auto &t : th) t.join();
    for (auto &s : st)
        if (!s) return s;
    return Status::ok();
}

// Forecast `nb` series of one replica from host memory. Inputs are staged through pinned memory
// unless the caller's buffer is pinned already. Large batches run as chunks: every chunk's inputs
// go up on the copy stream first, the forwards run in order on the compute stream, and each
// chunk's results come back on the copy stream while the next chunk computes.
template <class Fwd>
Status replica_forecast(Replica &r, const void *in, int64_t nb, size_t in_row, size_t out_row, void *out, Fwd &&fwd) {
    std::lock_guard<std::mutex> lk(r.mu);
    TSFM_CUDA(cudaSetDevice(r.device), "cudaSetDevice");
    r.prof.cur_launches = 0;
    const size_t in_bytes = (size_t)nb * in_row, out_bytes = (size_t)nb * out_row;
    const size_t in_span = Arena::span(in_bytes);
    if (r.io.bytes < in_span + out_bytes) TSFM_TRY(r.io.alloc(in_span + out_bytes));
    char *d_in = static_cast<char *>(r.io.p);
    char *d_out = static_cast<char *>(r.io.p) + in_span;
    const bool pin_in = is_pinned(in), pin_out = is_pinned(out);
    const char *src = static_cast<const char *>(in);
    if (!pin_in) {
        TSFM_TRY(r.pin_in.ensure(in_bytes));
        std::memcpy(r.pin_in.p, in, in_bytes);
        src = static_cast<const char *>(r.pin_in.p);
    }
    char *dst = static_cast<char *>(out);
    if (!pin_out) {
        TSFM_TRY(r.pin_out.ensure(out_bytes));
        dst = static_cast<char *>(r.pin_out.p);
    }
    // Chunks overlap the copies with the forwards, but every chunk repeats the forward's ~126 kernel
    // launches (about 1 ms of launch latency and tail per chunk): split only when the copies are
    // large enough to pay for it (at ~50 GB/s, 64 MB of copies take ~1.3 ms).
    const size_t copy_bytes = in_bytes + out_bytes;
    const int64_t chunks = std::min<int64_t>(nb, copy_bytes >= (size_t)256 << 20 ? 4 : copy_bytes >= (size_t)64 << 20 ? 2 : 1);
    while ((int64_t)r.events.size() < 2 * chunks) {
        cudaEvent_t e;
        TSFM_CUDA(cudaEventCreateWithFlags(&e, cudaEventDisableTiming), "cudaEventCreate");
        r.events.push_back(e);
    }
    for (int64_t c = 0; c < chunks; ++c) {
        const int64_t s0 = nb * c / chunks, s1 = nb * (c + 1) / chunks;
        TSFM_CUDA(cudaMemcpyAsync(d_in + s0 * in_row, src + s0 * in_row, (s1 - s0) * in_row, cudaMemcpyHostToDevice,
                                  r.copy),
                  "copy inputs");
        TSFM_CUDA(cudaEventRecord(r.events[2 * c], r.copy), "cudaEventRecord");
    }
    for (int64_t c = 0; c < chunks; ++c) {
        const int64_t s0 = nb * c / chunks, s1 = nb * (c + 1) / chunks;
        TSFM_CUDA(cudaStreamWaitEvent(r.stream, r.events[2 * c], 0), "cudaStreamWaitEvent");
        TSFM_TRY(fwd(reinterpret_cast<const float *>(d_in + s0 * in_row), reinterpret_cast<float *>(d_out + s0 * out_row),
                     s1 - s0, r.stream));
        TSFM_CUDA(cudaEventRecord(r.events[2 * c + 1], r.stream), "cudaEventRecord");
        TSFM_CUDA(cudaStreamWaitEvent(r.copy, r.events[2 * c + 1], 0), "cudaStreamWaitEvent");
        TSFM_CUDA(cudaMemcpyAsync(dst + s0 * out_row, d_out + s0 * out_row, (s1 - s0) * out_row, cudaMemcpyDeviceToHost,
                                  r.copy),
                  "copy results");
    }
    TSFM_CUDA(cudaStreamSynchronize(r.stream), "forecast");
    TSFM_CUDA(cudaStreamSynchronize(r.copy), "copy results");
    if (!pin_out) std::memcpy(out, r.pin_out.p, out_bytes);
    TSFM_TRY(check_device_error(r));
    r.prof.collect();
    r.prof.last_forecast_launches = r.prof.cur_launches;
    return Status::ok();
}

// Graph-cache key of one forward: family, shapes, and every buffer address it reads or writes
// (inputs, outputs, workspace, forecaster buffers); weights and the error word are fixed per replica.
std::vector<uint64_t> fwd_key(const Replica &r, int family, int64_t nb, size_t t, size_t horizon, const void *in,
                              const void *out) {
    return {(uint64_t)family,
            (uint64_t)nb,
            (uint64_t)t,
            (uint64_t)horizon,
            (uint64_t)reinterpret_cast<uintptr_t>(in),
            (uint64_t)reinterpret_cast<uintptr_t>(out),
            (uint64_t)reinterpret_cast<uintptr_t>(r.ws.buf.p),
            (uint64_t)r.ws.buf.bytes,
            (uint64_t)reinterpret_cast<uintptr_t>(r.fc.buf.p),
            (uint64_t)r.fc.buf.bytes};
}

// The same on device pointers (first replica, caller's stream).
template <class Fwd>
Status replica_forecast_device(Replica &r, cudaStream_t stream, Fwd &&fwd) {
    std::lock_guard<std::mutex> lk(r.mu);
    TSFM_CUDA(cudaSetDevice(r.device), "cudaSetDevice");
    cudaStream_t s = stream ? stream : r.stream;
    r.prof.cur_launches = 0;
    TSFM_TRY(fwd(s));
    TSFM_CUDA(cudaStreamSynchronize(s), "forecast");
    TSFM_TRY(check_device_error(r));
    r.prof.collect();
    r.prof.last_forecast_launches = r.prof.cur_launches;
    return Status::ok();
}

Status check_model(tsfm_model *m, int family) {
    if (!m) return Status::fail(TSFM_ERR_INVALID_ARGUMENT, "null model");
    if (m->cfg.family != family) return Status::fail(TSFM_ERR_INVALID_ARGUMENT, "model is of another family");
    return Status::ok();
}

Status c2_args(const tsfm_model *m, const void *in, size_t b, size_t t, size_t horizon, const void *out) {
    if (!in || !out) return Status::fail(TSFM_ERR_INVALID_ARGUMENT, "null inputs or outputs");
    if (b == 0 || t == 0) return Status::fail(TSFM_ERR_EMPTY_INPUT, "EmptyInput");
    if (horizon == 0 || horizon > (size_t)m->cfg.max_output_patches * m->cfg.patch_size)
        return Status::fail(TSFM_ERR_HORIZON_TOO_LONG, strf("HorizonTooLong: Chronos-2 supports horizons up to %d steps",
                                                            m->cfg.max_output_patches * m->cfg.patch_size));
    return Status::ok();
}

}  // namespace

extern "C" {

const char *tsfm_last_error(void) { return g_last_error.c_str(); }

const char *tsfm_version(void) { return "tsfm-b200 0.1.0 (sm_100a)"; }

const char *tsfm_status_string(int32_t s) {
    switch (s) {
        case TSFM_OK: return "ok";
        case TSFM_ERR_INVALID_ARGUMENT: return "invalid argument";
        case TSFM_ERR_INVALID_CONFIG: return "invalid config";
        case TSFM_ERR_MISSING_TENSOR: return "missing tensor";
        case TSFM_ERR_SHAPE_MISMATCH: return "shape mismatch";
        case TSFM_ERR_UNSUPPORTED_DTYPE: return "unsupported dtype";
        case TSFM_ERR_CUDA: return "CUDA error";
        case TSFM_ERR_OUT_OF_MEMORY: return "out of memory";
        case TSFM_ERR_DEVICE_TIMEOUT: return "device wait timed out";
        case TSFM_ERR_EMPTY_INPUT: return "empty input";
        case TSFM_ERR_HORIZON_TOO_LONG: return "horizon too long";
        case TSFM_ERR_UNSUPPORTED: return "unsupported";
        case TSFM_ERR_DEGENERATE_INPUT: return "degenerate input";
        case TSFM_ERR_ASYMMETRIC_QUANTILES: return "asymmetric quantiles";
        case TSFM_ERR_COVARIATES_UNSUPPORTED: return "covariates unsupported";
        case TSFM_ERR_NO_DEVICE: return "no device";
        case TSFM_ERR_BUFFER_TOO_SMALL: return "buffer too small";
        case TSFM_ERR_IO: return "I/O error";
        case TSFM_ERR_RAGGED_INPUT: return "ragged input";
        case TSFM_ERR_RAGGED_BLOCKS: return "ragged blocks";
        default: return "unknown status";
    }
}

int32_t tsfm_device_count(int32_t *count) {
    return guarded([&] {
        if (!count) return Status::fail(TSFM_ERR_INVALID_ARGUMENT, "null count");
        int n = 0;
        Status s = device_count(&n);
        *count = n;
        return s;
    });
}

int32_t tsfm_model_create(const tsfm_config *config, const tsfm_tensor *tensors, size_t n_tensors, int32_t compute,
                          const int32_t *devices, int32_t n_devices, tsfm_model **out) {
    return guarded([&]() -> Status {
        if (!config || !out || (!tensors && n_tensors)) return Status::fail(TSFM_ERR_INVALID_ARGUMENT, "null argument");
        *out = nullptr;
        if (compute != TSFM_COMPUTE_BF16 && compute != TSFM_COMPUTE_F16 && compute != TSFM_COMPUTE_F16C)
            return Status::fail(TSFM_ERR_UNSUPPORTED,
                                "compute type: TSFM_COMPUTE_BF16, TSFM_COMPUTE_F16 and TSFM_COMPUTE_F16C are implemented");
        if (compute == TSFM_COMPUTE_F16C && config->family == TSFM_CHRONOS_BOLT)
            return Status::fail(TSFM_ERR_UNSUPPORTED, "TSFM_COMPUTE_F16C: Chronos-2 and Timestral only in this build");
        // act: the weights' upload type (E_F16C: FP16 operands with FP8 correction companions).
        const int act = compute == TSFM_COMPUTE_F16C ? E_F16C : compute == TSFM_COMPUTE_F16 ? E_F16 : E_BF16;
        std::unique_ptr<tsfm_model> m(new tsfm_model());
        m->cfg = *config;
        if (config->num_quantiles > 0 && config->quantiles)
            m->quantiles.assign(config->quantiles, config->quantiles + config->num_quantiles);
        m->cfg.quantiles = m->quantiles.data();
        if (config->n_layer_kinds > 0 && config->layer_kinds)
            m->kinds.assign(config->layer_kinds, config->layer_kinds + config->n_layer_kinds);
        m->cfg.layer_kinds = m->kinds.data();
        m->compute = compute;
        const tsfm_config &c = m->cfg;
        TensorTable table(tensors, n_tensors);
        if (c.family == TSFM_CHRONOS2) {
            TSFM_TRY(c2_validate(c));
            TSFM_TRY(c2_check_tensors(c, table));
        } else if (c.family == TSFM_CHRONOS_BOLT) {
            TSFM_TRY(bolt_validate(c));
            TSFM_TRY(bolt_check_tensors(c, table));
        } else if (c.family == TSFM_TIMESTRAL) {
            TSFM_TRY(ts_validate(c));
            TSFM_TRY(ts_check_tensors(c, table));
        } else {
            return Status::fail(TSFM_ERR_UNSUPPORTED, "family not implemented in this build");
        }
        int ndev = 0;
        TSFM_TRY(device_count(&ndev));
        std::vector<int> devs;
        if (!devices || n_devices <= 0) {
            devs.push_back(0);
        } else {
            for (int i = 0; i < n_devices; ++i) {
                if (devices[i] < 0 || devices[i] >= ndev)
                    return Status::fail(TSFM_ERR_NO_DEVICE, strf("device %d out of range (%d visible)", devices[i], ndev));
                devs.push_back(devices[i]);
            }
        }
        // Replicas load in parallel, one host thread per device (each uploads over its own link).
        const size_t nrep = devs.size();
        std::vector<std::unique_ptr<Replica>> reps(nrep);
        std::vector<std::unique_ptr<C2Dev>> c2w(nrep);
        std::vector<std::unique_ptr<BoltDev>> boltw(nrep);
        std::vector<std::unique_ptr<TsDev>> tsw(nrep);
        TSFM_TRY(for_replicas(nrep, [&](size_t i) -> Status {
            auto r = std::make_unique<Replica>();
            r->device = devs[i];
            TSFM_CUDA(cudaSetDevice(r->device), "cudaSetDevice");
            TSFM_CUDA(cudaStreamCreateWithFlags(&r->stream, cudaStreamNonBlocking), "cudaStreamCreate");
            TSFM_CUDA(cudaStreamCreateWithFlags(&r->copy, cudaStreamNonBlocking), "cudaStreamCreate");
            TSFM_TRY(r->err.alloc(16));
            TSFM_CUDA(cudaMemset(r->err.p, 0, 16), "clear error word");
            Status st;
            if (c.family == TSFM_CHRONOS2) {
                c2w[i] = std::make_unique<C2Dev>();
                st = c2_load(*r, c, table, act, *c2w[i]);
            } else if (c.family == TSFM_CHRONOS_BOLT) {
                boltw[i] = std::make_unique<BoltDev>();
                st = bolt_load(*r, c, table, act, *boltw[i]);
            } else {
                tsw[i] = std::make_unique<TsDev>();
                st = ts_load(*r, c, table, act, *tsw[i]);
            }
            r->stage.reset();  // staging is needed at load time only
            reps[i] = std::move(r);
            return st;
        }));
        for (auto &b : reps[0]->weights) m->weight_bytes += b.bytes;
        for (size_t i = 0; i < nrep; ++i) {
            if (c2w[i]) m->c2.push_back(std::move(c2w[i]));
            if (boltw[i]) m->bolt.push_back(std::move(boltw[i]));
            if (tsw[i]) m->ts.push_back(std::move(tsw[i]));
            m->reps.push_back(std::move(reps[i]));
        }
        *out = m.release();
        return Status::ok();
    });
}

void tsfm_model_destroy(tsfm_model *model) {
    if (!model) return;
    for (auto &r : model->reps) {
        cudaSetDevice(r->device);
        if (r->stream) cudaStreamSynchronize(r->stream);
    }
    delete model;
}

int32_t tsfm_model_weight_bytes(const tsfm_model *model, uint64_t *bytes) {
    return guarded([&] {
        if (!model || !bytes) return Status::fail(TSFM_ERR_INVALID_ARGUMENT, "null argument");
        *bytes = model->weight_bytes;
        return Status::ok();
    });
}

int32_t tsfm_forecast_chronos2(tsfm_model *model, const float *inputs, size_t b, size_t t, size_t horizon, float *out) {
    return guarded([&]() -> Status {
        TSFM_TRY(check_model(model, TSFM_CHRONOS2));
        TSFM_TRY(c2_args(model, inputs, b, t, horizon, out));
        const size_t n = model->reps.size();
        const int64_t q = model->cfg.num_quantiles;
        return for_replicas(n, [&](size_t i) -> Status {
            TSFM_TRY(injected_failure(i));
            const int64_t s0 = (int64_t)(b * i / n), s1 = (int64_t)(b * (i + 1) / n);
            if (s1 <= s0) return Status::ok();
            Replica &r = *model->reps[i];
            const C2Dev &w = *model->c2[i];
            const int64_t nb = s1 - s0;
            return replica_forecast(r, inputs + s0 * t, nb, t * 4, horizon * q * 4, out + s0 * horizon * q,
                                    [&](const float *d_in, float *d_out, int64_t nc, cudaStream_t s) {
                                        return run_captured(r, s, fwd_key(r, TSFM_CHRONOS2, nc, t, horizon, d_in, d_out),
                                                            [&](cudaStream_t cs) {
                                                                return c2_forecast(r, model->cfg, w, d_in, nc, (int64_t)t,
                                                                                   (int64_t)horizon, d_out, cs);
                                                            });
                                    });
        });
    });
}

int32_t tsfm_forecast_chronos2_device(tsfm_model *model, const float *inputs, size_t b, size_t t, size_t horizon,
                                      float *out, void *stream) {
    return guarded([&]() -> Status {
        TSFM_TRY(check_model(model, TSFM_CHRONOS2));
        TSFM_TRY(c2_args(model, inputs, b, t, horizon, out));
        Replica &r = *model->reps[0];
        return replica_forecast_device(r, static_cast<cudaStream_t>(stream), [&](cudaStream_t s) {
            return run_captured(r, s, fwd_key(r, TSFM_CHRONOS2, (int64_t)b, t, horizon, inputs, out), [&](cudaStream_t cs) {
                return c2_forecast(r, model->cfg, *model->c2[0], inputs, (int64_t)b, (int64_t)t, (int64_t)horizon, out, cs);
            });
        });
    });
}

static Status bolt_args(const void *in, size_t b, size_t t, size_t horizon, const void *out) {
    if (!in || !out) return Status::fail(TSFM_ERR_INVALID_ARGUMENT, "null inputs or outputs");
    if (b == 0 || t == 0 || horizon == 0) return Status::fail(TSFM_ERR_EMPTY_INPUT, "EmptyInput");
    return Status::ok();
}

int32_t tsfm_forecast_bolt(tsfm_model *model, const float *inputs, size_t b, size_t t, size_t horizon, float *out) {
    return guarded([&]() -> Status {
        TSFM_TRY(check_model(model, TSFM_CHRONOS_BOLT));
        TSFM_TRY(bolt_args(inputs, b, t, horizon, out));
        const size_t n = model->reps.size();
        const int64_t q = model->cfg.num_quantiles;
        return for_replicas(n, [&](size_t i) -> Status {
            TSFM_TRY(injected_failure(i));
            const int64_t s0 = (int64_t)(b * i / n), s1 = (int64_t)(b * (i + 1) / n);
            if (s1 <= s0) return Status::ok();
            Replica &r = *model->reps[i];
            const BoltDev &w = *model->bolt[i];
            const int64_t nb = s1 - s0;
            return replica_forecast(r, inputs + s0 * t, nb, t * 4, horizon * q * 4, out + s0 * horizon * q,
                                    [&](const float *d_in, float *d_out, int64_t nc, cudaStream_t s) {
                                        return run_captured(r, s, fwd_key(r, TSFM_CHRONOS_BOLT, nc, t, horizon, d_in, d_out),
                                                            [&](cudaStream_t cs) {
                                                                return bolt_forecast(r, model->cfg, w, d_in, nc, (int64_t)t,
                                                                                     (int64_t)horizon, d_out, cs);
                                                            });
                                    });
        });
    });
}

int32_t tsfm_forecast_bolt_device(tsfm_model *model, const float *inputs, size_t b, size_t t, size_t horizon, float *out,
                                  void *stream) {
    return guarded([&]() -> Status {
        TSFM_TRY(check_model(model, TSFM_CHRONOS_BOLT));
        TSFM_TRY(bolt_args(inputs, b, t, horizon, out));
        Replica &r = *model->reps[0];
        return replica_forecast_device(r, static_cast<cudaStream_t>(stream), [&](cudaStream_t s) {
            return run_captured(r, s, fwd_key(r, TSFM_CHRONOS_BOLT, (int64_t)b, t, horizon, inputs, out), [&](cudaStream_t cs) {
                return bolt_forecast(r, model->cfg, *model->bolt[0], inputs, (int64_t)b, (int64_t)t, (int64_t)horizon, out, cs);
            });
        });
    });
}

void tsfm_timestral_default_options(tsfm_timestral_options *o) {
    if (!o) return;
    o->max_context = 0;
    o->per_shot_horizon_patches = 32;
    o->quantile_real_cap_k = 1e4f;
    o->extreme_value_threshold = 1e30f;
    o->symmetric_averaging = 1;
    o->clip_nonnegative = 1;
}

int32_t tsfm_forecast_timestral(tsfm_model *model, const float *inputs, const uint8_t *observed, size_t b, size_t v,
                                size_t t, size_t horizon, const tsfm_covariates *cov, const tsfm_timestral_options *opts,
                                float *out) {
    return guarded([&]() -> Status {
        TSFM_TRY(check_model(model, TSFM_TIMESTRAL));
        if (!inputs || !observed || !out) return Status::fail(TSFM_ERR_INVALID_ARGUMENT, "null inputs or outputs");
        if (b == 0 || v == 0 || t == 0 || horizon == 0) return Status::fail(TSFM_ERR_EMPTY_INPUT, "EmptyInput");
        tsfm_timestral_options o;
        tsfm_timestral_default_options(&o);
        if (opts) o = *opts;
        tsfm_covariates cv{};
        if (cov) cv = *cov;
        if ((cv.past && !cv.n_past) || (cv.known && !cv.n_known) || (cv.cat_past && !cv.n_cat_past) ||
            (cv.cat_known && !cv.n_cat_known))
            return Status::fail(TSFM_ERR_INVALID_ARGUMENT, "covariate array without channels");
        const size_t n = model->reps.size();
        const size_t q = (size_t)model->cfg.num_quantiles;
        // Series shard across replicas; every array is (b, channels, len), so a shard is a
        // contiguous slice of each.
        return for_replicas(n, [&](size_t i) -> Status {
            TSFM_TRY(injected_failure(i));
            const size_t s0 = b * i / n, s1 = b * (i + 1) / n;
            if (s1 <= s0) return Status::ok();
            Replica &r = *model->reps[i];
            std::lock_guard<std::mutex> lk(r.mu);
            TSFM_CUDA(cudaSetDevice(r.device), "cudaSetDevice");
            r.prof.cur_launches = 0;
            tsfm_covariates sh = cv;
            if (cv.past) sh.past = cv.past + s0 * cv.n_past * t;
            if (cv.known) sh.known = cv.known + s0 * cv.n_known * (t + horizon);
            if (cv.cat_past) sh.cat_past = cv.cat_past + s0 * cv.n_cat_past * t;
            if (cv.cat_known) sh.cat_known = cv.cat_known + s0 * cv.n_cat_known * (t + horizon);
            TSFM_TRY(ts_forecast(r, model->cfg, *model->ts[i], inputs + s0 * v * t, observed + s0 * v * t, s1 - s0, v, t,
                                 horizon, cov ? &sh : nullptr, o, out + s0 * v * horizon * q));
            TSFM_TRY(check_device_error(r));
            r.prof.collect();
            r.prof.last_forecast_launches = r.prof.cur_launches;
            return Status::ok();
        });
    });
}

int32_t tsfm_profile_enable(tsfm_model *model, int32_t enable) {
    return guarded([&] {
        if (!model) return Status::fail(TSFM_ERR_INVALID_ARGUMENT, "null model");
        for (auto &r : model->reps) r->prof.enabled = enable != 0;
        return Status::ok();
    });
}

int32_t tsfm_profile_reset(tsfm_model *model) {
    return guarded([&] {
        if (!model) return Status::fail(TSFM_ERR_INVALID_ARGUMENT, "null model");
        for (auto &r : model->reps) {
            std::fill(std::begin(r->prof.launches), std::end(r->prof.launches), 0);
            std::fill(std::begin(r->prof.ms), std::end(r->prof.ms), 0.0);
            std::fill(std::begin(r->prof.work), std::end(r->prof.work), 0.0);
        }
        return Status::ok();
    });
}

int32_t tsfm_profile_read(tsfm_model *model, const char *kernel_class, uint64_t *launches, double *ms, double *work) {
    return guarded([&] {
        if (!model || !kernel_class) return Status::fail(TSFM_ERR_INVALID_ARGUMENT, "null argument");
        int cls = -1;
        for (int i = 0; i < 6; ++i)
            if (std::strcmp(kernel_class, kclass_name(i)) == 0) cls = i;
        if (cls < 0) return Status::fail(TSFM_ERR_INVALID_ARGUMENT, std::string("unknown kernel class ") + kernel_class);
        uint64_t l = 0;
        double t = 0, wk = 0;
        for (auto &r : model->reps) {
            l += r->prof.launches[cls];
            t += r->prof.ms[cls];
            wk += r->prof.work[cls];
        }
        if (launches) *launches = l;
        if (ms) *ms = t;
        if (work) *work = wk;
        return Status::ok();
    });
}

int32_t tsfm_last_launch_count(tsfm_model *model, uint64_t *launches) {
    return guarded([&] {
        if (!model || !launches) return Status::fail(TSFM_ERR_INVALID_ARGUMENT, "null argument");
        *launches = model->reps[0]->prof.last_forecast_launches;
        return Status::ok();
    });
}

// ---- kernel-level entry points ------------------------------------------------------------

int32_t tsfm_kernel_linear(const void *x, int32_t x_dtype, const void *w, int32_t w_dtype, const float *bias, void *y,
                           int32_t out_mode, int32_t act, int64_t M, int64_t N, int64_t K, int64_t ldx, int64_t ldw,
                           int64_t ldy, void *stream) {
    return guarded([&]() -> Status {
        if (!x || !w || !y) return Status::fail(TSFM_ERR_INVALID_ARGUMENT, "null pointer");
        if (x_dtype != w_dtype ||
            (x_dtype != TSFM_DTYPE_BF16 && x_dtype != TSFM_DTYPE_F16 && x_dtype != TSFM_DTYPE_F32))
            return Status::fail(TSFM_ERR_UNSUPPORTED_DTYPE, "linear: x and w must both be BF16, F16 or F32");
        const int elem = x_dtype == TSFM_DTYPE_F32 ? E_F32 : x_dtype == TSFM_DTYPE_F16 ? E_F16 : E_BF16;
        if (out_mode == 0 && elem == E_F32)
            return Status::fail(TSFM_ERR_INVALID_ARGUMENT, "linear: out_mode 0 stores the 16-bit operand type");
        if (out_mode < 0 || out_mode > 2 || (act != 0 && act != 1 && act != ACT_GLU))
            return Status::fail(TSFM_ERR_INVALID_ARGUMENT, "linear: bad out_mode / act");
        LinearCall c;
        c.x = x;
        c.w = w;
        c.dtype = elem;
        c.M = M;
        c.N = N;
        c.K = K;
        c.ldx = ldx;
        c.ldw = ldw;
        c.y = y;
        c.ldy = ldy;
        c.out_mode = out_mode == 0 ? out_mode_for(elem) : out_mode == 1 ? OUT_F32 : OUT_F32_ACC;
        c.bias = bias;
        c.act = act;
        c.err = kernel_err_word();
        return launch_linear(c, static_cast<cudaStream_t>(stream));
    });
}

int32_t tsfm_kernel_linear_corrected(const float *x, const float *w, const float *bias, void *y, void *y8,
                                     int32_t out_mode, int32_t act, int64_t M, int64_t N, int64_t K, int32_t terms,
                                     void *stream) {
    return guarded([&]() -> Status {
        if (!x || !w || !y) return Status::fail(TSFM_ERR_INVALID_ARGUMENT, "null pointer");
        if (M <= 0 || N <= 0 || K <= 0 || K % 8) return Status::fail(TSFM_ERR_INVALID_ARGUMENT, "linear: bad shape");
        if (out_mode < 0 || out_mode > 2 || (act != 0 && act != 1) || (y8 && out_mode != 0) || (terms != 1 && terms != 2))
            return Status::fail(TSFM_ERR_INVALID_ARGUMENT, "linear: bad out_mode / act / y8 / terms");
        cudaStream_t st = static_cast<cudaStream_t>(stream);
        // Temporaries: the FP16 operands and their FP8 companions, as a corrected model holds them.
        void *buf = nullptr;
        const size_t xb = Arena::span((size_t)(M * K) * 2), wb = Arena::span((size_t)(N * K) * 2);
        TSFM_CUDA(cudaMallocAsync(&buf, 2 * xb + 2 * wb, st), "linear (corrected): temporaries");
        char *x16 = static_cast<char *>(buf), *x8 = x16 + xb, *w16 = x8 + xb, *w8 = w16 + wb;
        int sh = 0;
        Status res = launch_split_x8(x, M, K, K, x16, K, x8, 2 * K, st);
        if (res) res = build_corrected_weight(w, N, K, w16, w8, &sh, st);
        if (res) {
            LinearCall c;
            c.x = x16;
            c.w = w16;
            c.dtype = E_F16;
            c.M = M;
            c.N = N;
            c.K = K;
            c.ldx = K;
            c.ldw = K;
            c.y = y;
            c.ldy = N;
            c.out_mode = out_mode == 0 ? OUT_F16 : out_mode == 1 ? OUT_F32 : OUT_F32_ACC;
            c.bias = bias;
            c.act = act;
            c.err = kernel_err_word();
            c.x8 = x8;
            c.ldx8 = 2 * K;
            c.w8 = w8;
            c.ldw8 = 2 * K;
            c.acc_scale = std::ldexp(1.0f, -sh);
            c.x8_cols = terms == 1 ? K : 2 * K;
            c.y8 = y8;
            c.ldy8 = 2 * N;
            res = launch_linear(c, st);
        }
        cudaFreeAsync(buf, st);
        return res;
    });
}

int32_t tsfm_kernel_split_f16c(const float *x, int64_t rows, int64_t cols, void *x16, void *x8, void *stream) {
    return guarded([&]() -> Status {
        if (!x || !x16 || !x8 || rows <= 0 || cols <= 0) return Status::fail(TSFM_ERR_INVALID_ARGUMENT, "split: bad arguments");
        return launch_split_x8(x, rows, cols, cols, x16, cols, x8, 2 * cols, static_cast<cudaStream_t>(stream));
    });
}

int32_t tsfm_kernel_weight_f16c(const float *w, int64_t rows, int64_t cols, void *w16, void *w8, float *acc_scale,
                                void *stream) {
    return guarded([&]() -> Status {
        if (!w || !w16 || !w8 || !acc_scale || rows <= 0 || cols <= 0 || cols % 8)
            return Status::fail(TSFM_ERR_INVALID_ARGUMENT, "weight split: bad arguments");
        int sh = 0;
        TSFM_TRY(build_corrected_weight(w, rows, cols, w16, w8, &sh, static_cast<cudaStream_t>(stream)));
        *acc_scale = std::ldexp(1.0f, -sh);
        return Status::ok();
    });
}

int32_t tsfm_kernel_linear_f16c(const void *x16, const void *x8, const void *w16, const void *w8, float acc_scale,
                                const float *bias, void *y, void *y8, int32_t out_mode, int32_t act, int64_t M,
                                int64_t N, int64_t K, int32_t terms, void *stream) {
    return guarded([&]() -> Status {
        if (!x16 || !x8 || !w16 || !w8 || !y) return Status::fail(TSFM_ERR_INVALID_ARGUMENT, "null pointer");
        if (out_mode < 0 || out_mode > 2 || (act != 0 && act != 1) || (y8 && out_mode != 0) || (terms != 1 && terms != 2))
            return Status::fail(TSFM_ERR_INVALID_ARGUMENT, "linear: bad out_mode / act / y8 / terms");
        LinearCall c;
        c.x = x16;
        c.w = w16;
        c.dtype = E_F16;
        c.M = M;
        c.N = N;
        c.K = K;
        c.ldx = K;
        c.ldw = K;
        c.y = y;
        c.ldy = N;
        c.out_mode = out_mode == 0 ? OUT_F16 : out_mode == 1 ? OUT_F32 : OUT_F32_ACC;
        c.bias = bias;
        c.act = act;
        c.err = kernel_err_word();
        c.x8 = x8;
        c.ldx8 = 2 * K;
        c.w8 = w8;
        c.ldw8 = 2 * K;
        c.acc_scale = acc_scale;
        c.x8_cols = terms == 1 ? K : 2 * K;
        c.y8 = y8;
        c.ldy8 = 2 * N;
        return launch_linear(c, static_cast<cudaStream_t>(stream));
    });
}

int32_t tsfm_test_bounded_wait(int64_t limit_ns, void *stream) {
    return guarded([&]() -> Status {
        if (limit_ns < 1000 || limit_ns > (int64_t)kWaitTimeoutNs)
            return Status::fail(TSFM_ERR_INVALID_ARGUMENT, "bounded wait: limit outside [1 us, 2 s]");
        int *err = kernel_err_word();
        if (!err) return Status::fail(TSFM_ERR_CUDA, "bounded wait: no error word");
        cudaStream_t st = static_cast<cudaStream_t>(stream);
        int code = 0;
        TSFM_CUDA(cudaMemsetAsync(err, 0, sizeof(int), st), "bounded wait: clear error word");
        TSFM_TRY(launch_bounded_wait(err, (unsigned long long)limit_ns, st));
        TSFM_CUDA(cudaMemcpyAsync(&code, err, sizeof(int), cudaMemcpyDeviceToHost, st), "bounded wait: error word");
        TSFM_CUDA(cudaStreamSynchronize(st), "bounded wait");
        TSFM_CUDA(cudaMemsetAsync(err, 0, sizeof(int), st), "bounded wait: clear error word");
        TSFM_CUDA(cudaStreamSynchronize(st), "bounded wait");
        if (code) return Status::fail(TSFM_ERR_DEVICE_TIMEOUT, strf("a kernel's bounded wait gave up (site 0x%04x)", code));
        return Status::ok();
    });
}

int32_t tsfm_relative_bucket(int64_t rel, int32_t num_buckets, int32_t max_distance) {
    if (num_buckets < 2 || max_distance < 1) return -1;
    return (int32_t)relative_bucket(rel, (uint32_t)num_buckets, (uint32_t)max_distance);
}

int32_t tsfm_kernel_patch(int32_t family, const float *inputs, int64_t b, int64_t t_in, int64_t context_length,
                          int32_t patch, float time_encoding_scale, int32_t use_arcsinh, int32_t use_reg_token,
                          float *loc, float *scale, float *feats, uint8_t *key_valid, void *stream) {
    return guarded([&]() -> Status {
        if (!inputs || !loc || !scale || !feats || !key_valid) return Status::fail(TSFM_ERR_INVALID_ARGUMENT, "null pointer");
        if (family != TSFM_CHRONOS2 && family != TSFM_CHRONOS_BOLT)
            return Status::fail(TSFM_ERR_INVALID_ARGUMENT, "patch: family must be Chronos-2 or Chronos-Bolt");
        if (b <= 0 || t_in <= 0 || context_length <= 0 || patch <= 0)
            return Status::fail(TSFM_ERR_INVALID_ARGUMENT, "patch: empty");
        const bool bolt = family == TSFM_CHRONOS_BOLT;
        const int64_t t = std::min(t_in, context_length), pad = (patch - t % patch) % patch;
        const int64_t n_ctx = (t + pad) / patch;
        PatchCall pc;
        pc.inputs = inputs;
        pc.stride = t_in;
        pc.start = t_in - t;
        pc.t = t;
        pc.b = b;
        pc.ps = patch;
        pc.pad = (int)pad;
        pc.n_ctx = (int)n_ctx;
        pc.feat_kind = bolt ? 1 : 0;
        pc.tscale = time_encoding_scale;
        pc.arcsinh = bolt ? 0 : use_arcsinh;
        pc.feat_mode = OUT_F32;
        pc.feats = feats;
        pc.loc = loc;
        pc.scale = scale;
        pc.key_valid = key_valid;
        pc.seq = n_ctx + (bolt && use_reg_token ? 1 : 0);
        pc.extra_valid = bolt && use_reg_token ? 1 : 0;
        return launch_patch(pc, static_cast<cudaStream_t>(stream));
    });
}

int32_t tsfm_kernel_timestral_block_inputs(const float *ctx, const uint8_t *observed, int64_t rows, int64_t t,
                                           const float *known_future, const uint8_t *known_future_observed,
                                           int64_t hl, int32_t patch, int32_t vall, const int8_t *roles,
                                           int32_t covariates, double minimum_scale, int32_t use_asinh,
                                           int32_t attend_missing, float *loc, float *scale, float *feats,
                                           uint8_t *key_valid, int32_t *first_obs, void *stream) {
    return guarded([&]() -> Status {
        if (!ctx || !observed || !roles || !loc || !scale || !feats || !key_valid || !first_obs)
            return Status::fail(TSFM_ERR_INVALID_ARGUMENT, "null pointer");
        if (rows <= 0 || t <= 0 || patch <= 0 || vall <= 0 || rows % vall || t % patch || (covariates && hl % patch) ||
            hl < 0)
            return Status::fail(TSFM_ERR_INVALID_ARGUMENT, "timestral block inputs: bad geometry");
        cudaStream_t st = static_cast<cudaStream_t>(stream);
        void *buf = nullptr;
        TSFM_CUDA(cudaMallocAsync(&buf, (size_t)rows * 9, st), "timestral block inputs: temporaries");
        float *kloc = static_cast<float *>(buf), *kscale = kloc + rows;
        uint8_t *binary = reinterpret_cast<uint8_t *>(kscale + rows);
        Status res = Status::ok();
        const cudaError_t e = cudaMemsetAsync(first_obs, 0x7f, (size_t)(rows / vall) * sizeof(int32_t), st);
        if (e != cudaSuccess) res = Status::cuda(e, "timestral block inputs: first_obs");
        if (res) {
            TsStatsCall sc;
            sc.ctx = ctx;
            sc.obs = observed;
            sc.t = t;
            sc.kf = covariates ? known_future : nullptr;
            sc.kfm = covariates ? known_future_observed : nullptr;
            sc.kf_ld = hl;
            sc.hl = covariates ? hl : 0;
            sc.cov = covariates != 0;
            sc.rows = rows;
            sc.ps = patch;
            sc.vall = vall;
            sc.roles = roles;
            sc.min_scale = minimum_scale;
            sc.use_asinh = use_asinh;
            sc.attend_missing = attend_missing;
            sc.loc = loc;
            sc.scale = scale;
            sc.kloc = kloc;
            sc.kscale = kscale;
            sc.binary = binary;
            sc.key_valid = key_valid;
            sc.first_obs = first_obs;
            sc.raw_feats = 1;
            res = launch_ts_stats(sc, feats, st);
        }
        cudaFreeAsync(buf, st);
        return res;
    });
}

int32_t tsfm_kernel_attention_ex(const void *q, const void *k, const void *v, int64_t ld_qkv, void *o, int64_t ld_o,
                                 float *o32, int64_t ld_o32, uint8_t *o8, int64_t ld_o8, const uint8_t *key_valid,
                                 int64_t kv_stride, const float *rel_bias, const uint8_t *group_bidir, int32_t groups, int32_t heads, int32_t n, float scale,
                                 int32_t mask_mode, int32_t ne, int32_t l, int32_t dtype, int32_t force_path,
                                 void *stream) {
    return guarded([&]() -> Status {
        if (!q || !k || !v || (!o && !o32)) return Status::fail(TSFM_ERR_INVALID_ARGUMENT, "null pointer");
        if (mask_mode < 0 || mask_mode > 2) return Status::fail(TSFM_ERR_INVALID_ARGUMENT, "bad mask_mode");
        if (force_path < 0 || force_path > 3) return Status::fail(TSFM_ERR_INVALID_ARGUMENT, "bad force_path");
        if (mask_mode != 0 && (ne < 0 || ne > n || l < 0 || l > ne))
            return Status::fail(TSFM_ERR_INVALID_ARGUMENT, "attention: need 0 <= l <= ne <= n");
        if (dtype != TSFM_DTYPE_BF16 && dtype != TSFM_DTYPE_F16)
            return Status::fail(TSFM_ERR_UNSUPPORTED_DTYPE, "attention: q/k/v must be BF16 or F16");
        AttentionCall c;
        c.q = q;
        c.k = k;
        c.v = v;
        c.ld_qkv = ld_qkv;
        c.o = o;
        c.ld_o = ld_o;
        c.o32 = o32;
        c.ld_o32 = ld_o32;
        c.o8 = o8;
        c.ld_o8 = ld_o8;
        c.key_valid = key_valid;
        c.kv_stride = kv_stride > 0 ? kv_stride : n;
        c.rel_bias = rel_bias;
        c.group_bidir = group_bidir;
        c.groups = groups;
        c.heads = heads;
        c.n = n;
        c.scale = scale;
        c.mask_mode = mask_mode;
        c.dtype = dtype == TSFM_DTYPE_F16 ? E_F16 : E_BF16;
        c.ne = mask_mode == 0 ? n : ne;
        c.l = mask_mode == 0 ? n : l;
        c.force_path = force_path;
        c.err = kernel_err_word();
        if ((force_path == 1 || force_path == 3) && !attention_tc_supported(c))
            return Status::fail(TSFM_ERR_UNSUPPORTED, "attention: the tcgen05 path does not take this call");
        return launch_attention(c, static_cast<cudaStream_t>(stream));
    });
}

int32_t tsfm_kernel_attention(const void *q, const void *k, const void *v, int64_t ld_qkv, void *o, int64_t ld_o,
                              const uint8_t *key_valid, const float *rel_bias, int32_t groups, int32_t heads, int32_t n,
                              float scale, int32_t mask_mode, int32_t dtype, void *stream) {
    return guarded([&]() -> Status {
        if (!q || !k || !v || !o) return Status::fail(TSFM_ERR_INVALID_ARGUMENT, "null pointer");
        if (mask_mode < 0 || mask_mode > 2) return Status::fail(TSFM_ERR_INVALID_ARGUMENT, "bad mask_mode");
        AttentionCall c;
        c.q = q;
        c.k = k;
        c.v = v;
        c.ld_qkv = ld_qkv;
        c.o = o;
        c.ld_o = ld_o;
        c.key_valid = key_valid;
        c.kv_stride = n;
        c.rel_bias = rel_bias;
        c.groups = groups;
        c.heads = heads;
        c.n = n;
        c.scale = scale;
        c.mask_mode = mask_mode;
        if (dtype != TSFM_DTYPE_BF16 && dtype != TSFM_DTYPE_F16)
            return Status::fail(TSFM_ERR_UNSUPPORTED_DTYPE, "attention: q/k/v must be BF16 or F16");
        c.dtype = dtype == TSFM_DTYPE_F16 ? E_F16 : E_BF16;
        c.ne = n;
        c.l = n;
        c.err = kernel_err_word();
        return launch_attention(c, static_cast<cudaStream_t>(stream));
    });
}

int32_t tsfm_kernel_target_encode(const float *inputs, const uint8_t *observed, int64_t b, int64_t t,
                                  int64_t max_context, const double *codes, int64_t nc, int64_t len,
                                  int32_t have_target, float *out, void *stream) {
    return guarded([&]() -> Status {
        if (!codes || !out || (have_target && (!inputs || !observed)))
            return Status::fail(TSFM_ERR_INVALID_ARGUMENT, "null pointer");
        if (b <= 0 || t <= 0 || nc <= 0 || len < t) return Status::fail(TSFM_ERR_INVALID_ARGUMENT, "target encode: shape");
        cudaStream_t s = static_cast<cudaStream_t>(stream);
        double *target = nullptr;
        if (have_target) {
            TSFM_CUDA(cudaMallocAsync(reinterpret_cast<void **>(&target), (size_t)(b * t) * 8, s), "target encode: scratch");
            const Status st = launch_ts_target(inputs, observed, b, t, max_context, target, s);
            if (!st) {
                cudaFreeAsync(target, s);
                return st;
            }
        }
        const Status st = launch_ts_cat_encode(codes, b, nc, len, t, target, out, nc, 0, s);
        if (target) TSFM_CUDA(cudaFreeAsync(target, s), "target encode: scratch");
        return st;
    });
}

int32_t tsfm_kernel_rmsnorm(const float *x, const float *scale, void *out, int32_t out_dtype, int64_t rows, int64_t dim,
                            float eps, void *stream) {
    return guarded([&]() -> Status {
        if (!x || !scale || !out) return Status::fail(TSFM_ERR_INVALID_ARGUMENT, "null pointer");
        RmsNormCall c;
        c.x = x;
        c.scale = scale;
        c.out = out;
        c.out_mode = out_dtype == TSFM_DTYPE_BF16 ? OUT_BF16 : out_dtype == TSFM_DTYPE_F16 ? OUT_F16 : OUT_F32;
        c.rows = rows;
        c.dim = dim;
        c.eps = eps;
        return launch_rmsnorm(c, static_cast<cudaStream_t>(stream));
    });
}

int32_t tsfm_kernel_rmsnorm_ex(const float *x, const float *scale, void *out, int32_t out_dtype, void *out8,
                               int64_t ld8, int64_t rows, int64_t dim, float eps, void *stream) {
    return guarded([&]() -> Status {
        if (!x || !scale || !out) return Status::fail(TSFM_ERR_INVALID_ARGUMENT, "null pointer");
        RmsNormCall c;
        c.x = x;
        c.scale = scale;
        c.out = out;
        c.out_mode = out_dtype == TSFM_DTYPE_BF16 ? OUT_BF16 : out_dtype == TSFM_DTYPE_F16 ? OUT_F16 : OUT_F32;
        c.out8 = out8;
        c.ld8 = ld8;
        c.rows = rows;
        c.dim = dim;
        c.eps = eps;
        return launch_rmsnorm(c, static_cast<cudaStream_t>(stream));
    });
}

}  // extern "C"
