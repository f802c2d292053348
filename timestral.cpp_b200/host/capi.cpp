// Flat C ABI (include/timestral_capi.h) and the device-seam entries (include/timestral_b200.h).
// Error behaviour follows the reference (src/timestral_capi.cpp:8-92): no exception crosses
// the ABI, load and NULL-handle errors go to a thread-local string, every other error to
// the handle, and a successful call clears the handle's error. All sizes are validated
// before any caller buffer is read.
#include "timestral_capi.h"
#include "timestral_b200.h"

#include "engine.cuh"
#include "forecaster.hpp"
#include "gguf.hpp"
#include "model.hpp"

#include <algorithm>
#include <climits>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <limits>
#include <memory>
#include <new>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include <cuda_runtime.h>

namespace {

struct ErrorText {
    std::string text;
    bool fallback = false;
    void clear() noexcept { text.clear(); fallback = false; }
    void set(const char* m) noexcept {
        try { text = m ? m : "unknown C ABI error"; fallback = false; }
        catch (...) { fallback = true; }
    }
    const char* get() const noexcept { return fallback ? "C ABI error (diagnostic allocation failed)" : text.c_str(); }
};
thread_local ErrorText tls_error;
thread_local int tls_device = -1;

void require(bool ok, const char* msg) { if (!ok) throw ts::Error(msg); }
void pointer_count(const void* p, int32_t n) {
    require(n >= 0, "negative covariate count");
    require((n != 0) == (p != nullptr), "covariate pointer/count mismatch");
}
size_t mul(size_t a, size_t b) {
    if (b && a > std::numeric_limits<size_t>::max() / b) throw ts::Error("C ABI dimensions overflow");
    return a * b;
}
template <class T> size_t count(size_t a, size_t b, size_t c) {
    const size_t n = mul(mul(a, b), c);
    mul(n, sizeof(T));
    return n;
}

}  // namespace

// A handle: one model mapping and one Forecaster per GPU it forecasts on. With several GPUs
// (tsb_load_devices, or TIMESTRAL_DEVICES for timestral_capi_load) a request's series are
// split into contiguous shards, one per GPU, forecast concurrently by one host thread each,
// and every shard's result lands in its own slice of the one output buffer: no collective,
// a series never leaves its GPU, and a series' result does not depend on the shard it is in.
struct timestral_ctx {
    ts::Model model;
    ts::Forecaster forecaster;                                   // the first GPU
    std::vector<std::unique_ptr<ts::Forecaster>> more;           // the other GPUs, in list order
    int threads;
    ErrorText error;
    timestral_ctx(ts::Model&& m, int n, const std::vector<int>& devices)
        : model(std::move(m)), forecaster(model, devices.at(0)), threads(n) {
        for (size_t i = 1; i < devices.size(); ++i) more.push_back(std::make_unique<ts::Forecaster>(model, devices[i]));
    }
    size_t gpus() const { return 1 + more.size(); }
    ts::Forecaster& gpu(size_t k) { return k ? *more[k - 1] : forecaster; }
};

namespace {
ErrorText& error(timestral_ctx* c) noexcept { return c ? c->error : tls_error; }
void caught(timestral_ctx* c) noexcept {
    try { throw; }
    catch (const std::exception& e) { error(c).set(e.what()); }
    catch (...) { error(c).set("unknown C ABI exception"); }
}
}  // namespace

extern "C" {

TIMESTRAL_API int timestral_capi_abi_version(void) { return 1; }

namespace {
int device_count() {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0) throw ts::Error("no CUDA device available");
    return n;
}

// GPUs of a handle loaded with timestral_capi_load: TIMESTRAL_DEVICES ("all", or a comma-separated
// list of device ordinals), else the device chosen with tsb_set_device, else the current one.
std::vector<int> default_devices() {
    const int n = device_count();
    if (const char* env = std::getenv("TIMESTRAL_DEVICES")) {
        std::vector<int> list;
        const std::string v(env);
        if (v == "all") {
            for (int d = 0; d < n; ++d) list.push_back(d);
            return list;
        }
        size_t i = 0;
        while (i < v.size()) {
            size_t j = v.find(',', i);
            if (j == std::string::npos) j = v.size();
            const std::string item = v.substr(i, j - i);
            char* end = nullptr;
            const long d = std::strtol(item.c_str(), &end, 10);
            require(!item.empty() && end && *end == 0 && d >= 0 && d < n, "TIMESTRAL_DEVICES: invalid device list");
            list.push_back(int(d));
            i = j + 1;
        }
        require(!list.empty(), "TIMESTRAL_DEVICES: invalid device list");
        return list;
    }
    int dev = tls_device;
    if (dev < 0 && cudaGetDevice(&dev) != cudaSuccess) throw ts::Error("no CUDA device available");
    return {dev};
}

// The model file is checked before any GPU is touched (its errors come first, as in the
// reference); `devices` null: default_devices().
timestral_ctx* load_on(const char* path, int threads, const std::vector<int>* devices) {
    require(path && *path, "model path is required");
    require(threads >= 1 && threads <= 1024, "invalid CPU thread count");
    ts::Model model = ts::Model::load(path);
    auto p = std::make_unique<timestral_ctx>(std::move(model), threads, devices ? *devices : default_devices());
    tls_error.clear();
    return p.release();
}
}  // namespace

TIMESTRAL_API timestral_ctx* timestral_capi_load(const char* path, int threads) {
    try {
        require(path && *path, "model path is required");
        require(threads >= 1 && threads <= 1024, "invalid CPU thread count");
        return load_on(path, threads, nullptr);
    } catch (...) {
        caught(nullptr);
        return nullptr;
    }
}

TIMESTRAL_API timestral_ctx* tsb_load_devices(const char* path, int threads, const int32_t* devices, int32_t n_devices) {
    try {
        require(path && *path, "model path is required");
        require(devices && n_devices >= 1 && n_devices <= 64, "invalid device list");
        const int n = device_count();
        std::vector<int> list(devices, devices + n_devices);
        for (int d : list) require(d >= 0 && d < n, "invalid device ordinal");
        return load_on(path, threads, &list);
    } catch (...) {
        caught(nullptr);
        return nullptr;
    }
}

TIMESTRAL_API int32_t tsb_device_count(timestral_ctx* c) { return c ? int32_t(c->gpus()) : 0; }

TIMESTRAL_API void timestral_capi_free(timestral_ctx* c) {
    try { delete c; } catch (...) { caught(nullptr); }
}

TIMESTRAL_API const char* timestral_capi_last_error(timestral_ctx* c) { return error(c).get(); }

TIMESTRAL_API int timestral_capi_num_quantiles(timestral_ctx* c) {
    try {
        require(c, "null handle");
        const auto n = c->model.config().num_quantiles();
        require(n <= INT_MAX, "quantile count overflow");
        c->error.clear();
        return int(n);
    } catch (...) {
        caught(c);
        return 0;
    }
}

TIMESTRAL_API double timestral_capi_quantile_level(timestral_ctx* c, int i) {
    try {
        require(c, "null handle");
        const auto& q = c->model.config().quantile_knots;
        require(i >= 0 && size_t(i) < q.size(), "quantile index out of range");
        const double v = q[size_t(i)];
        c->error.clear();
        return v;
    } catch (...) {
        caught(c);
        return std::numeric_limits<double>::quiet_NaN();
    }
}

namespace {
// Result buffers of timestral_capi_forecast. The reference's contract is that the caller
// frees them only with timestral_capi_free_buffer (include/timestral_capi.h:42-44), so they
// come from page-locked host memory recycled through a small pool: the device writes the
// forecast straight into the caller's buffer, with no staging copy and no first-touch page
// faults. A 64-byte header before the data records how the block was obtained.
struct OutHeader {
    uint64_t magic;
    uint64_t capacity;     // data bytes
    uint32_t pinned;
    uint32_t pad;
    uint64_t reserved[5];
};
static_assert(sizeof(OutHeader) == 64, "header keeps the data 64-byte aligned");
constexpr uint64_t kOutMagic = 0x74736230'6f757462ull;
constexpr size_t kPoolMaxBuffers = 16;
constexpr size_t kPoolMaxBytes = size_t(4) << 30;

// A pooled buffer and its capacity, kept beside it: a device reset (cudaDeviceReset) frees
// the page-locked memory of the context it replaces, so a pooled buffer is checked with the
// runtime before it is reused and dropped, untouched, when it is no longer page-locked.
struct PoolEntry {
    OutHeader* h;
    size_t capacity;
};
std::mutex& pool_mutex() { static std::mutex m; return m; }
std::vector<PoolEntry>& pool() { static auto* v = new std::vector<PoolEntry>(); return *v; }   // never destroyed
size_t pool_bytes = 0;

bool still_page_locked(const void* p) {
    cudaPointerAttributes a;
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    return a.type == cudaMemoryTypeHost;
}

float* out_alloc(size_t bytes, bool* pinned) {
    {
        std::lock_guard<std::mutex> lock(pool_mutex());
        auto& v = pool();
        while (true) {
            size_t best = v.size();
            for (size_t i = 0; i < v.size(); ++i)
                if (v[i].capacity >= bytes && v[i].capacity <= 2 * bytes + (size_t(1) << 20) &&
                    (best == v.size() || v[i].capacity < v[best].capacity))
                    best = i;
            if (best == v.size()) break;
            const PoolEntry e = v[best];
            v.erase(v.begin() + std::ptrdiff_t(best));
            pool_bytes -= e.capacity;
            if (!still_page_locked(e.h)) continue;     // freed by a device reset
            *pinned = true;
            return reinterpret_cast<float*>(e.h + 1);
        }
    }
    void* p = nullptr;
    OutHeader* h = nullptr;
    if (cudaHostAlloc(&p, bytes + sizeof(OutHeader), cudaHostAllocPortable) == cudaSuccess) {
        h = static_cast<OutHeader*>(p);
        h->pinned = 1;
    } else {
        cudaGetLastError();
        p = std::malloc(bytes + sizeof(OutHeader));
        if (!p) throw std::bad_alloc();
        h = static_cast<OutHeader*>(p);
        h->pinned = 0;
    }
    h->magic = kOutMagic;
    h->capacity = bytes;
    *pinned = h->pinned != 0;
    return reinterpret_cast<float*>(h + 1);
}

void out_free(void* data) {
    if (!data) return;
    OutHeader* h = reinterpret_cast<OutHeader*>(data) - 1;
    if (h->magic != kOutMagic) return;      // not a buffer of this library: leave it alone
    if (!h->pinned) {
        h->magic = 0;
        std::free(h);
        return;
    }
    {
        std::lock_guard<std::mutex> lock(pool_mutex());
        auto& v = pool();
        if (v.size() < kPoolMaxBuffers && pool_bytes + h->capacity <= kPoolMaxBytes) {
            v.push_back(PoolEntry{h, size_t(h->capacity)});
            pool_bytes += h->capacity;
            return;
        }
    }
    h->magic = 0;
    cudaFreeHost(h);
}
}  // namespace

TIMESTRAL_API float* timestral_capi_forecast(timestral_ctx* c, const timestral_forecast_request* a, int32_t* out_q) {
    if (out_q) *out_q = 0;
    float* result = nullptr;
    try {
        require(c, "null handle");
        require(a, "null request");
        require(out_q, "out_q is required");
        require(a->context, "context is required");
        require(a->B > 0 && a->V > 0 && a->T > 0 && a->prediction_length > 0, "invalid forecast dimensions");
        require(a->max_context >= 0, "negative max_context");
        require(a->symmetric_averaging >= -1 && a->symmetric_averaging <= 1 && a->clip_nonnegative >= -1 &&
                    a->clip_nonnegative <= 1,
                "invalid forecast flag");
        pointer_count(a->past_cov, a->c_past);
        pointer_count(a->known_cov, a->c_known);
        pointer_count(a->cat_past, a->cc_past);
        pointer_count(a->cat_known, a->cc_known);
        const size_t B = size_t(a->B), V = size_t(a->V), T = size_t(a->T), H = size_t(a->prediction_length);
        require(T <= std::numeric_limits<size_t>::max() - H, "forecast length overflow");
        const size_t TH = T + H;
        const size_t nx = count<float>(B, V, T), np = count<float>(B, size_t(a->c_past), T);
        const size_t nk = count<float>(B, size_t(a->c_known), TH), ncp = count<double>(B, size_t(a->cc_past), T);
        const size_t nck = count<double>(B, size_t(a->cc_known), TH);
        (void)np; (void)nk; (void)ncp; (void)nck;      // overflow checks of the covariate sizes
        const ts::Config& cfg = c->model.config();
        const size_t Q = cfg.num_quantiles();
        require(Q <= INT32_MAX, "quantile count overflow");
        const size_t no = mul(count<float>(B, V, H), Q);
        mul(no, sizeof(float));
        const bool any = a->c_past || a->c_known || a->cc_past || a->cc_known;
        if (any && !cfg.covariate_enabled) throw ts::Error("this checkpoint was not trained with covariates");
        if ((a->c_known || a->cc_known) && !ts::supports_known_covariates(cfg))
            throw ts::Error("this checkpoint cannot condition on known-future covariates");
        if (size_t(a->max_context) > size_t(cfg.context_length)) throw ts::Error("max_context exceeds stored position range");
        if (a->observation_mask)
            for (size_t i = 0; i < nx; ++i) require(a->observation_mask[i] <= 1, "observation mask must be boolean");
        const bool sym = a->symmetric_averaging == -1 ? cfg.symmetric_averaging : a->symmetric_averaging != 0;
        const bool clip = a->clip_nonnegative == -1 ? cfg.clip_nonnegative : a->clip_nonnegative != 0;
        bool pinned = false;
        result = out_alloc(no * sizeof(float), &pinned);
        if (!any && sym)
            for (size_t i = 0; i < Q; ++i)
                if (std::abs(cfg.quantile_knots[i] + cfg.quantile_knots[Q - 1 - i] - 1) >= 1e-9)
                    throw ts::Error("symmetric averaging needs quantile levels symmetric about 0.5");
        // Series shard k of n: [k * B / n, (k + 1) * B / n), on the handle's k-th GPU.
        const size_t shards = std::min(c->gpus(), B);
        auto run_shard = [&](size_t k) {
            const size_t b0 = k * B / shards, b1 = (k + 1) * B / shards, Bk = b1 - b0;
            float* out_k = result + b0 * V * H * Q;
            ts::Forecaster& f = c->gpu(k);
            if (!any) {
                f.forecast_targets(a->context + b0 * V * T, a->observation_mask ? a->observation_mask + b0 * V * T : nullptr,
                                   Bk, V, T, H, sym, clip, size_t(a->max_context), out_k, pinned);
                return;
            }
            ts::ForecastRequest r;
            r.batch = Bk; r.targets = V; r.length = T; r.horizon = H; r.max_context = size_t(a->max_context);
            r.past_count = size_t(a->c_past); r.known_count = size_t(a->c_known);
            r.categorical_past_count = size_t(a->cc_past); r.categorical_known_count = size_t(a->cc_known);
            auto take = [&](auto* src, size_t per_series, auto& dst) {
                if (src && per_series) dst.assign(src + b0 * per_series, src + b1 * per_series);
            };
            if (a->observation_mask) r.observation_mask.assign(a->observation_mask + b0 * V * T, a->observation_mask + b1 * V * T);
            take(a->context, V * T, r.context);
            take(a->past_cov, size_t(a->c_past) * T, r.past);
            take(a->known_cov, size_t(a->c_known) * TH, r.known);
            take(a->cat_past, size_t(a->cc_past) * T, r.categorical_past);
            take(a->cat_known, size_t(a->cc_known) * TH, r.categorical_known);
            r.symmetric_averaging = sym;
            r.clip_nonnegative = clip;
            f.forecast_into(r, out_k);
        };
        if (shards == 1) {
            run_shard(0);
        } else {
            std::vector<std::exception_ptr> failed(shards);
            std::vector<std::thread> pool;
            pool.reserve(shards);
            for (size_t k = 0; k < shards; ++k)
                pool.emplace_back([&, k] {
                    try { run_shard(k); } catch (...) { failed[k] = std::current_exception(); }
                });
            for (auto& t : pool) t.join();
            for (auto& e : failed)
                if (e) std::rethrow_exception(e);
        }
        *out_q = int32_t(Q);
        c->error.clear();
        return result;
    } catch (...) {
        out_free(result);
        caught(c);
        return nullptr;
    }
}

TIMESTRAL_API void timestral_capi_free_buffer(void* p) { out_free(p); }

}  // extern "C"

namespace tsb {
// Thread-local error text of entry points that take no handle (read with
// timestral_capi_last_error(NULL)).
void set_thread_error(const char* message) { tls_error.set(message); }
}  // namespace tsb

extern "C" {

// ---- device seam --------------------------------------------------------------------

TIMESTRAL_API int tsb_set_device(int32_t device) {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || device < 0 || device >= n) {
        tls_error.set("invalid CUDA device");
        return TSB_ERR_ARG;
    }
    tls_device = device;
    return TSB_OK;
}

TIMESTRAL_API int tsb_forecast_device(timestral_ctx* c, const float* d_context, const uint8_t* d_mask, int32_t B,
                                      int32_t V, int32_t T, int32_t H, int32_t symmetric, int32_t clip,
                                      int32_t max_context, float* d_out, int32_t async) {
    try {
        require(c, "null handle");
        require(d_context && d_out, "device buffers are required");
        require(B > 0 && V > 0 && T > 0 && H > 0, "invalid forecast dimensions");
        require(symmetric >= -1 && symmetric <= 1 && clip >= -1 && clip <= 1, "invalid forecast flag");
        require(max_context >= 0, "negative max_context");
        const ts::Config& cfg = c->model.config();
        const bool sym = symmetric == -1 ? cfg.symmetric_averaging : symmetric != 0;
        const bool cl = clip == -1 ? cfg.clip_nonnegative : clip != 0;
        const size_t Q = cfg.num_quantiles();
        if (sym)
            for (size_t i = 0; i < Q; ++i)
                if (std::abs(cfg.quantile_knots[i] + cfg.quantile_knots[Q - 1 - i] - 1) >= 1e-9)
                    throw ts::Error("symmetric averaging needs quantile levels symmetric about 0.5");
        c->forecaster.engine().forecast_targets(d_context, d_mask, B, V, T, H, sym, cl, max_context, d_out, !async);
        c->error.clear();
        return TSB_OK;
    } catch (const std::exception& e) {
        error(c).set(e.what());
        return TSB_ERR_DEVICE;
    } catch (...) {
        caught(c);
        return TSB_ERR_DEVICE;
    }
}

TIMESTRAL_API int tsb_sync(timestral_ctx* c) {
    try {
        require(c, "null handle");
        c->forecaster.engine().check_errors();
        c->error.clear();
        return TSB_OK;
    } catch (...) {
        caught(c);
        return TSB_ERR_DEVICE;
    }
}

TIMESTRAL_API void* tsb_stream(timestral_ctx* c) { return c ? static_cast<void*>(c->forecaster.engine().stream()) : nullptr; }

TIMESTRAL_API int tsb_timing_enable(timestral_ctx* c, int32_t enable) {
    if (!c) return TSB_ERR_ARG;
    // 1: every kernel class; 2: attention launches alone (two events per launch).
    c->forecaster.engine().timing_enable(enable != 0, enable == 2 ? "attention" : nullptr);
    return TSB_OK;
}

TIMESTRAL_API int tsb_fused_norm(timestral_ctx* c, int32_t mode) {
    if (!c || mode < 0 || mode > 2) return TSB_ERR_ARG;
    try {
        for (size_t k = 0; k < c->gpus(); ++k) c->gpu(k).engine().fused_norm(mode);
    } catch (...) {
        caught(c);
        return TSB_ERR_CUDA;
    }
    return TSB_OK;
}

TIMESTRAL_API int tsb_attention_kernels(timestral_ctx* c, int32_t mode) {
    if (!c || mode < 0 || mode > 1) return TSB_ERR_ARG;
    try {
        for (size_t k = 0; k < c->gpus(); ++k) c->gpu(k).engine().attention_kernels(mode);
    } catch (...) {
        caught(c);
        return TSB_ERR_CUDA;
    }
    return TSB_OK;
}

TIMESTRAL_API int tsb_dequant_prologue(timestral_ctx* c, int32_t on) {
    if (!c) return TSB_ERR_ARG;
    try {
        bool ok = true;
        for (size_t k = 0; k < c->gpus(); ++k) ok &= c->gpu(k).engine().dequant_prologue(on != 0);
        if (!ok) {
            c->error.set("tsb_dequant_prologue: the model has no block-quantised weights");
            return TSB_ERR_MODEL;
        }
    } catch (...) {
        caught(c);
        return TSB_ERR_CUDA;
    }
    return TSB_OK;
}

TIMESTRAL_API int tsb_decoder_tail(timestral_ctx* c, int32_t on) {
    if (!c) return TSB_ERR_ARG;
    try {
        for (size_t k = 0; k < c->gpus(); ++k) c->gpu(k).engine().decoder_tail(on != 0);
    } catch (...) {
        caught(c);
        return TSB_ERR_CUDA;
    }
    return TSB_OK;
}

TIMESTRAL_API int tsb_graph_replay(timestral_ctx* c, int32_t on) {
    if (!c) return TSB_ERR_ARG;
    try {
        for (size_t k = 0; k < c->gpus(); ++k) c->gpu(k).engine().graph_replay(on != 0);
    } catch (...) {
        caught(c);
        return TSB_ERR_CUDA;
    }
    return TSB_OK;
}

TIMESTRAL_API int tsb_covariate_assembly(timestral_ctx* c, int32_t on_device) {
    if (!c) return TSB_ERR_ARG;
    for (size_t k = 0; k < c->gpus(); ++k) c->gpu(k).set_device_assembly(on_device != 0);
    return TSB_OK;
}

TIMESTRAL_API int tsb_timing_read(timestral_ctx* c, const char* cls, double* ms, int64_t* launches) {
    if (!c || !cls || !ms || !launches) return TSB_ERR_ARG;
    c->forecaster.engine().timing_read(cls, ms, launches);
    return TSB_OK;
}

TIMESTRAL_API void tsb_timing_reset(timestral_ctx* c) {
    if (c) c->forecaster.engine().timing_reset();
}

TIMESTRAL_API int64_t tsb_last_launch_count(timestral_ctx* c) { return c ? c->forecaster.engine().last_launches() : 0; }

TIMESTRAL_API int tsb_last_geometry(timestral_ctx* c, int64_t* rows, int32_t* S, int32_t* L, int32_t* blocks) {
    if (!c || !rows || !S || !L || !blocks) return TSB_ERR_ARG;
    const auto g = c->forecaster.engine().last_geometry();
    *rows = g.rows; *S = g.S; *L = g.L; *blocks = g.blocks;
    return TSB_OK;
}

TIMESTRAL_API int tsb_dequantize_rows(uint32_t type, const void* src, int64_t rows, int64_t ne0, float* dst) {
    if (!src || !dst || rows < 0 || ne0 <= 0) return TSB_ERR_ARG;
    const size_t row = ts::ggml_row_bytes(type, ne0);
    if (!row) return TSB_ERR_ARG;
    for (int64_t r = 0; r < rows; ++r)
        if (!ts::dequantize_row(type, static_cast<const uint8_t*>(src) + size_t(r) * row, ne0, dst + r * ne0))
            return TSB_ERR_ARG;
    return TSB_OK;
}

TIMESTRAL_API int tsb_scaled_int8_rows(uint32_t type, const void* src, int64_t rows, int64_t ne0, int8_t* q, float* a,
                                       float* b) {
    if (!src || !q || !a || !b || rows < 0 || ne0 <= 0 || ne0 % 16) return TSB_ERR_ARG;
    const size_t row = ts::ggml_row_bytes(type, ne0);
    if (!row) return TSB_ERR_ARG;
    for (int64_t r = 0; r < rows; ++r)
        if (!ts::scaled_int8_row(type, static_cast<const uint8_t*>(src) + size_t(r) * row, ne0, q + r * ne0,
                                 a + r * (ne0 / 16), b + r * (ne0 / 16)))
            return TSB_ERR_ARG;
    return TSB_OK;
}

TIMESTRAL_API int tsb_model_path(timestral_ctx* c) { return c && c->forecaster.engine().tensor_cores() ? 1 : 0; }

}  // extern "C"
