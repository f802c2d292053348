#include "forecaster.hpp"

#include "engine.cuh"

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <limits>
#include <thread>
#include <vector>

#include <cuda_runtime.h>
#ifdef __linux__
#include <sys/mman.h>
#include <unistd.h>
#endif

namespace ts {

namespace {

size_t mul(size_t a, size_t b) {
    if (b && a > SIZE_MAX / b) throw Error("row dimensions overflow");
    return a * b;
}
size_t add(size_t a, size_t b) {
    if (a > SIZE_MAX - b) throw Error("row dimensions overflow");
    return a + b;
}
float finite_value(float v) {
    return std::isnan(v) ? 0.f : std::isinf(v) ? std::copysign(std::numeric_limits<float>::max(), v) : v;
}
void codes_valid(const std::vector<double>& x) {
    for (double v : x)
        if (std::isinf(v)) throw Error("categorical covariates must hold finite codes or NaN; got an infinite value");
}

// NumPy pairwise float64 sum (reference src/numpy_sum.hpp:6-14).
double pairwise_sum(const double* x, size_t n) {
    if (n < 8) {
        double r = -0.0;
        for (size_t i = 0; i < n; ++i) r += x[i];
        return r;
    }
    if (n <= 128) {
        double r[8];
        for (size_t j = 0; j < 8; ++j) r[j] = x[j];
        size_t i = 8;
        for (; i < n - (n % 8); i += 8)
            for (size_t j = 0; j < 8; ++j) r[j] += x[i + j];
        double out = ((r[0] + r[1]) + (r[2] + r[3])) + ((r[4] + r[5]) + (r[6] + r[7]));
        for (; i < n; ++i) out += x[i];
        return out;
    }
    size_t half = n / 2;
    half -= half % 8;
    return pairwise_sum(x, half) + pairwise_sum(x + half, n - half);
}

// Smoothed mean target encoding of one categorical row, float64
// (reference src/covariates.cpp:14-25).
void target_encode(const std::vector<double>& target, const std::vector<double>& past, const std::vector<double>& future,
                   double smooth, std::vector<float>& out_past, std::vector<float>& out_future) {
    codes_valid(past);
    codes_valid(future);
    std::vector<double> cats;
    for (double x : past) if (std::isfinite(x)) cats.push_back(x);
    std::sort(cats.begin(), cats.end());
    cats.erase(std::unique(cats.begin(), cats.end()), cats.end());
    const size_t nan_slot = cats.size();
    auto slot = [&](double code) -> size_t {
        if (std::isnan(code)) return nan_slot;
        auto it = std::lower_bound(cats.begin(), cats.end(), code);
        return it != cats.end() && *it == code ? size_t(it - cats.begin()) : nan_slot + 1;
    };
    std::vector<double> values(target.size(), 0.0), sums(nan_slot + 1, 0.0), counts(nan_slot + 1, 0.0);
    double count = 0;
    for (size_t i = 0; i < target.size(); ++i)
        if (std::isfinite(target[i])) { values[i] = target[i]; ++count; }
    const double mean = count ? pairwise_sum(values.data(), values.size()) / count : 0;
    for (size_t i = 0; i < past.size(); ++i) {
        const size_t sl = slot(past[i]);
        sums[sl] += values[i];
        counts[sl] += std::isfinite(target[i]) ? 1 : 0;
    }
    std::vector<double> lookup(nan_slot + 2, mean);
    for (size_t i = 0; i <= nan_slot; ++i) lookup[i] = (smooth * mean + sums[i]) / (smooth + counts[i]);
    out_past.clear();
    out_future.clear();
    for (double v : past) out_past.push_back(float(lookup[slot(v)]));
    for (double v : future) out_future.push_back(float(lookup[slot(v)]));
}

tsb::ModelView make_view(const Model& m) {
    const Config& c = m.config();
    tsb::ModelView v;
    v.ps = int(c.patch_size); v.D = int(c.d_model); v.H = int(c.num_heads); v.F = int(c.mlp_hidden_dim);
    for (auto k : c.block_schedule)
        v.schedule.push_back(k == LayerKind::Time ? 0 : k == LayerKind::Variate ? 1 : k == LayerKind::TimeVariate ? 2 : 3);
    v.knots = c.quantile_knots;
    v.median = int(c.median_index());
    v.block_size = int(c.block_size); v.context_length = int(c.context_length);
    v.rope_dim = int(c.rope_dim); v.pos_min = c.rope_table_pos_min;
    v.eps = c.norm_eps;
    v.attn_bias = c.attn_bias; v.mlp_bias = c.mlp_bias;
    v.time_gate = c.time_gate == Gate::SdpaSigmoid; v.variate_gate = c.variate_gate == Gate::SdpaSigmoid;
    v.minimum_scale = c.minimum_scale; v.use_asinh = c.use_asinh;
    v.covariate_enabled = c.covariate_enabled; v.attend_missing = c.attend_missing_patches;
    v.width_factor = c.quantile_width_factor;
    v.per_shot = int(c.per_shot_horizon_patches);
    v.cap_k = c.quantile_real_cap_k; v.extreme = c.extreme_value_threshold;
    v.symmetric = c.symmetric_averaging; v.clip = c.clip_nonnegative;
    const Model* mp = &m;
    v.tensor = [mp](const std::string& n) {
        const TensorRef& t = mp->tensor(n);
        tsb::HostTensor h;
        h.type = int(t.type);
        h.ne0 = t.ne[0];
        h.ne1 = t.ne[1] * t.ne[2] * t.ne[3];
        h.data = t.data;
        return h;
    };
    v.has = [mp](const std::string& n) { return mp->has(n); };
    return v;
}

void cuda_check(cudaError_t e, const char* what) {
    if (e != cudaSuccess) throw Error(std::string(what) + ": " + cudaGetErrorString(e));
}

}  // namespace

bool supports_known_covariates(const Config& c) {  // reference src/covariates.cpp:27-31
    if (!c.covariate_enabled) return false;
    std::vector<bool> ops;
    for (auto k : c.block_schedule) for (bool t : layer_axes(k)) ops.push_back(t);
    for (size_t i = 0; i < ops.size(); ++i) {
        if (!ops[i]) continue;
        bool time = false, var = false;
        for (size_t j = i + 1; j < ops.size(); ++j) { time |= ops[j]; var |= !ops[j]; }
        if (time && var) return true;
    }
    return false;
}

namespace {
struct RowGeometry { size_t kept, pad, len, hor; };

// The checks and the kept/padded lengths of an assembled covariate request (reference
// src/covariates.cpp:32-47), shared by the host and the device assembly.
RowGeometry check_rows(const Config& c, const std::vector<float>& context, const std::vector<int8_t>& user, size_t B,
                       size_t V, size_t T, size_t H, const std::vector<float>& past, size_t P,
                       const std::vector<float>& known, size_t K, size_t cap, const std::vector<double>& cp, size_t CP,
                       const std::vector<double>& ck, size_t CK) {
    if (!B || !V || !T || !H || !c.patch_size || !c.context_length) throw Error("invalid row dimensions");
    const size_t TH = add(T, H), BV = mul(B, V);
    if (context.size() != mul(BV, T) || (!user.empty() && user.size() != context.size()) || past.size() != mul(mul(B, P), T) ||
        known.size() != mul(mul(B, K), TH) || cp.size() != mul(mul(B, CP), T) || ck.size() != mul(mul(B, CK), TH))
        throw Error("row input shape mismatch");
    for (auto v : user) if (v != 0 && v != 1) throw Error("observation mask must be boolean");
    if ((P || K || CP || CK) && !c.covariate_enabled) throw Error("this checkpoint was not trained with covariates");
    if ((K || CK) && !supports_known_covariates(c)) throw Error("this checkpoint cannot condition on known-future covariates");
    codes_valid(cp);
    codes_valid(ck);
    cap = cap ? cap : c.context_length;
    if (cap > c.context_length) throw Error("max_context exceeds stored position range");
    RowGeometry g;
    const size_t ps = c.patch_size;
    g.kept = std::min(T, cap);
    g.pad = (ps - g.kept % ps) % ps;
    g.len = add(g.kept, g.pad);
    g.hor = mul(add(H, ps - 1) / ps, ps);
    return g;
}
}  // namespace

AssembledRows assemble_rows(const Config& c, const std::vector<float>& context, const std::vector<int8_t>& user,
                            size_t B, size_t V, size_t T, size_t H, const std::vector<float>& past, size_t P,
                            const std::vector<float>& known, size_t K, size_t cap, const std::vector<double>& cp, size_t CP,
                            const std::vector<double>& ck, size_t CK) {
    const RowGeometry geo = check_rows(c, context, user, B, V, T, H, past, P, known, K, cap, cp, CP, ck, CK);
    const size_t TH = add(T, H), BV = mul(B, V);
    const size_t kept = geo.kept, pad = geo.pad, len = geo.len, hor = geo.hor;
    const size_t all = add(add(V, add(P, CP)), add(K, CK)), R = mul(B, all);
    AssembledRows a;
    a.rows_count = R; a.length = len; a.horizon = hor;
    a.rows.assign(mul(R, len), 0.f);
    a.mask.assign(a.rows.size(), 0);
    a.groups.resize(R);
    if (P || CP || K || CK) a.roles.resize(R);
    if (K || CK) { a.future.assign(mul(R, hor), 0.f); a.future_mask.assign(a.future.size(), 0); }
    // Targets: observed = finite and not masked out; forward fill from the first observation.
    std::vector<float> filled(context.size());
    std::vector<int8_t> obs(context.size());
    for (size_t r = 0; r < BV; ++r) {
        float prev = 0;
        for (size_t t = 0; t < T; ++t) {
            const size_t i = r * T + t;
            obs[i] = std::isfinite(context[i]) && (user.empty() || user[i]);
            if (obs[i]) prev = context[i];
            filled[i] = prev;
        }
    }
    auto encode = [&](const std::vector<double>& codes, size_t C, size_t width) {
        std::vector<float> out(codes.size());
        std::vector<float> ep, ef;
        for (size_t b = 0; b < B; ++b)
            for (size_t j = 0; j < C; ++j) {
                const size_t off = (b * C + j) * width;
                if (V != 1) {
                    for (size_t t = 0; t < width; ++t) out[off + t] = float(codes[off + t]);
                    continue;
                }
                std::vector<double> target(T);
                bool started = false;
                for (size_t t = 0; t < T; ++t) {
                    started |= obs[b * T + t] != 0;
                    target[t] = started && t >= T - kept ? double(filled[b * T + t]) : std::nan("");
                }
                std::vector<double> p(codes.begin() + off, codes.begin() + off + T);
                std::vector<double> f(codes.begin() + off + T, codes.begin() + off + width);
                target_encode(target, p, f, c.target_encoding_smooth, ep, ef);
                for (size_t t = 0; t < T; ++t) out[off + t] = std::isnan(target[t]) && std::isnan(p[t]) ? NAN : ep[t];
                std::copy(ef.begin(), ef.end(), out.begin() + off + T);
            }
        return out;
    };
    const auto enc_p = encode(cp, CP, T), enc_k = encode(ck, CK, TH);
    for (size_t b = 0; b < B; ++b)
        for (size_t j = 0; j < all; ++j) {
            const size_t r = b * all + j;
            const int role = j < V ? 0 : j < V + P + CP ? 1 : 2;
            a.groups[r] = int64_t(b);
            if (!a.roles.empty()) a.roles[r] = role;
            const std::vector<float>* src;
            size_t off;
            if (j < V) { src = &filled; off = (b * V + j) * T; }
            else if (j < V + P) { src = &past; off = (b * P + j - V) * T; }
            else if (j < V + P + CP) { src = &enc_p; off = (b * CP + j - V - P) * T; }
            else if (j < V + P + CP + K) { src = &known; off = (b * K + j - V - P - CP) * TH; }
            else { src = &enc_k; off = (b * CK + j - V - P - CP - K) * TH; }
            for (size_t t = 0; t < kept; ++t) {
                const size_t from = off + T - kept + t, to = r * len + pad + t;
                const float v = (*src)[from];
                a.rows[to] = role ? finite_value(v) : v;
                a.mask[to] = role ? !std::isnan(v) : obs[(b * V + j) * T + T - kept + t];
            }
            if (role == 2)
                for (size_t t = 0; t < H; ++t) {
                    const float v = (*src)[off + T + t];
                    a.future[r * hor + t] = finite_value(v);
                    a.future_mask[r * hor + t] = !std::isnan(v);
                }
        }
    return a;
}

struct Forecaster::Staging {
    void* ctx = nullptr; size_t ctx_bytes = 0;
    void* mask = nullptr; size_t mask_bytes = 0;
    void* out = nullptr; size_t out_bytes = 0;
    void* host_out = nullptr; size_t host_out_bytes = 0;   // pinned: the download lands here
    static void grow(void*& p, size_t& have, size_t need) {
        if (need <= have) return;
        if (p) cudaFree(p);
        p = nullptr;
        have = 0;
        cuda_check(cudaMalloc(&p, need), "cudaMalloc staging");
        have = need;
    }
    static void grow_host(void*& p, size_t& have, size_t need) {
        if (need <= have) return;
        if (p) cudaFreeHost(p);
        p = nullptr;
        have = 0;
        cuda_check(cudaMallocHost(&p, need), "cudaMallocHost staging");
        have = need;
    }
    ~Staging() {
        if (ctx) cudaFree(ctx);
        if (mask) cudaFree(mask);
        if (out) cudaFree(out);
        if (host_out) cudaFreeHost(host_out);
    }
};

namespace {
// Copy a large result from pinned staging into the caller's (typically freshly allocated,
// not yet faulted-in) buffer: large buffers are asked for transparent huge pages and are
// written by several threads, so first-touch page faults run in parallel.
void copy_out(float* dst, const float* src, size_t n) {
    const size_t bytes = n * sizeof(float);
    constexpr size_t kParallelBytes = size_t(8) << 20;
    if (bytes < kParallelBytes) {
        std::memcpy(dst, src, bytes);
        return;
    }
#ifdef __linux__
    {
        const uintptr_t page = uintptr_t(sysconf(_SC_PAGESIZE));
        const uintptr_t lo = (reinterpret_cast<uintptr_t>(dst) + page - 1) & ~(page - 1);
        const uintptr_t hi = (reinterpret_cast<uintptr_t>(dst) + bytes) & ~(page - 1);
        if (hi > lo) madvise(reinterpret_cast<void*>(lo), hi - lo, MADV_HUGEPAGE);
    }
#endif
    const unsigned hw = std::max(1u, std::thread::hardware_concurrency());
    const size_t threads = std::min<size_t>(std::min<size_t>(hw, 16), bytes / (size_t(4) << 20));
    const size_t per = (n + threads - 1) / threads;
    std::vector<std::thread> pool;
    pool.reserve(threads);
    for (size_t t = 0; t < threads; ++t) {
        const size_t b = t * per, e = std::min(n, b + per);
        if (b >= e) break;
        pool.emplace_back([=] { std::memcpy(dst + b, src + b, (e - b) * sizeof(float)); });
    }
    for (auto& th : pool) th.join();
}
}  // namespace

Forecaster::Forecaster(const Model& model, int device) : model_(model), staging_(new Staging) {
    int dev = device;
    if (dev < 0) cuda_check(cudaGetDevice(&dev), "cudaGetDevice");
    try {
        engine_ = std::make_unique<tsb::Engine>(make_view(model), dev);
    } catch (const std::exception& e) {
        throw Error(e.what());
    }
}

Forecaster::~Forecaster() {
    if (engine_) cudaSetDevice(engine_->device());
    staging_.reset();
}

void Forecaster::forecast_targets(const float* context, const uint8_t* mask, size_t B, size_t V, size_t T, size_t H,
                                  bool sym, bool clip, size_t max_context, float* out, bool out_pinned) {
    const Config& c = model_.config();
    const size_t Q = c.num_quantiles();
    const size_t cap = max_context ? max_context : c.context_length;
    if (cap > c.context_length) throw Error("max_context exceeds stored position range");
    if (T > size_t(INT32_MAX) || H > size_t(INT32_MAX) || mul(B, V) > size_t(INT32_MAX))
        throw Error("forecast dimensions exceed the device path limits");
    tsb::Engine& eng = *engine_;
    cuda_check(cudaSetDevice(eng.device()), "cudaSetDevice");
    const size_t BV = mul(B, V), n = mul(BV, T), no = mul(mul(BV, H), Q);
    Staging& st = *staging_;
    Staging::grow(st.ctx, st.ctx_bytes, n * 4);
    if (mask) Staging::grow(st.mask, st.mask_bytes, n);
    Staging::grow(st.out, st.out_bytes, no * 4);
    cudaStream_t s = eng.stream();
    cuda_check(cudaMemcpyAsync(st.ctx, context, n * 4, cudaMemcpyHostToDevice, s), "upload context");
    if (mask) cuda_check(cudaMemcpyAsync(st.mask, mask, n, cudaMemcpyHostToDevice, s), "upload mask");
    try {
        eng.forecast_targets(static_cast<float*>(st.ctx), mask ? static_cast<uint8_t*>(st.mask) : nullptr, int(B), int(V),
                             int(T), int(H), sym, clip, int(max_context), static_cast<float*>(st.out), false);
        // Completes the forecast (including a fallback run, which rewrites st.out) before the
        // download.
        eng.check_errors();
        if (out_pinned) {
            cuda_check(cudaMemcpyAsync(out, st.out, no * 4, cudaMemcpyDeviceToHost, s), "download forecast");
            cuda_check(cudaStreamSynchronize(s), "download forecast");
        } else {
            Staging::grow_host(st.host_out, st.host_out_bytes, no * 4);
            cuda_check(cudaMemcpyAsync(st.host_out, st.out, no * 4, cudaMemcpyDeviceToHost, s), "download forecast");
            cuda_check(cudaStreamSynchronize(s), "download forecast");
            copy_out(out, static_cast<const float*>(st.host_out), no);
        }
    } catch (const Error&) {
        throw;
    } catch (const std::exception& e) {
        throw Error(e.what());
    }
}

namespace {

// Per-call engine settings (request overrides, block observer), undone when the call ends.
struct CallScope {
    tsb::Engine& eng;
    CallScope(tsb::Engine& e, int per_shot, double cap_k, const tsb::BlockObserver* observer) : eng(e) {
        eng.set_overrides(per_shot, cap_k);
        eng.set_observer(observer);
    }
    ~CallScope() {
        eng.set_observer(nullptr);
        eng.set_overrides(0, -1);
    }
};

// Rows [r0, r0 + n) of a [rows][stride] device matrix of `width` used columns, to the host.
template <class T>
std::vector<T> download_rows(const T* d, int64_t stride, size_t r0, size_t n, size_t width) {
    std::vector<T> out(n * width);
    if (!n || !width) return out;
    cuda_check(cudaMemcpy2D(out.data(), width * sizeof(T), d + int64_t(r0) * stride, size_t(stride) * sizeof(T),
                            width * sizeof(T), n, cudaMemcpyDeviceToHost),
               "download trace");
    return out;
}

// One pass's rows of an observed block as the reference's DecodeBlock.
DecodeBlock block_of(const tsb::BlockView& v, size_t r0, size_t rows, size_t ps, size_t Q) {
    DecodeBlock b;
    const size_t n = size_t(v.patches) * ps;
    b.offset = size_t(v.offset); b.patches = size_t(v.patches); b.length = size_t(v.length);
    b.context = download_rows(v.context, v.context_stride, r0, rows, size_t(v.length));
    b.mask = download_rows(v.mask, v.context_stride, r0, rows, size_t(v.length));
    if (v.future) {
        b.future = download_rows(v.future, v.future_stride, r0, rows, n);
        b.future_mask = download_rows(v.future_mask, v.future_stride, r0, rows, n);
    }
    b.predicted = download_rows(v.predicted, int64_t(n * Q), r0, rows, n * Q);
    b.refined = download_rows(v.refined, int64_t(n * Q), r0, rows, n * Q);
    return b;
}

}  // namespace

Forecast Forecaster::forecast(const ForecastRequest& r, ForecastTrace* trace) {
    const Config& c = model_.config();
    Forecast f;
    f.batch = r.batch; f.targets = r.targets; f.horizon = r.horizon;
    f.quantile_levels = c.quantile_knots;
    f.quantiles.resize(mul(mul(mul(r.batch, r.targets), r.horizon), c.num_quantiles()));
    forecast_into(r, f.quantiles.data(), trace);
    return f;
}

std::vector<float> Forecaster::decode(const AssembledRows& a, size_t H, size_t cap, size_t shot,
                                      std::vector<DecodeBlock>* trace, const DecodeProgress& progress) {
    const Config& c = model_.config();
    const size_t ps = c.patch_size, Q = c.num_quantiles(), R = a.rows_count, T = a.length;
    const size_t cap_eff = cap ? cap : c.context_length;
    const size_t shot_eff = std::min<size_t>(shot ? shot : c.per_shot_horizon_patches, c.block_size);
    // The reference's checks (src/forecaster.cpp:21-27).
    if (!H || !R || !T || T % ps || !shot_eff || !cap_eff || cap_eff > c.context_length || H > SIZE_MAX - (ps - 1))
        throw Error("invalid decode dimensions");
    if (a.rows.size() != mul(R, T) || a.mask.size() != a.rows.size() || a.groups.size() != R ||
        (!a.roles.empty() && a.roles.size() != R))
        throw Error("invalid decode rows");
    const size_t patches = (H + ps - 1) / ps, full = mul(patches, ps);
    if (a.horizon != full || a.future.size() != a.future_mask.size() || (!a.future.empty() && a.future.size() != mul(R, full)))
        throw Error("invalid decode future");
    for (int64_t role : a.roles)
        if (role < 0 || role > 2) throw Error("invalid decode role");
    // The device keeps the rows of a group contiguous and of one size (as assemble_rows lays
    // them out: group b holds rows [b * all, (b + 1) * all)).
    size_t group_rows = 1;
    while (group_rows < R && a.groups[group_rows] == a.groups[0]) ++group_rows;
    if (R % group_rows) throw Error("decode rows: groups must be contiguous runs of equal size");
    for (size_t r = 0; r < R; ++r)
        if (a.groups[r] != a.groups[(r / group_rows) * group_rows] ||
            (r % group_rows == 0 && r && a.groups[r] == a.groups[r - 1]))
            throw Error("decode rows: groups must be contiguous runs of equal size");
    if (R > size_t(INT32_MAX) / 2 || T > size_t(INT32_MAX) || full > size_t(INT32_MAX) || H > size_t(INT32_MAX))
        throw Error("forecast dimensions exceed the device path limits");
    if (trace) trace->clear();
    tsb::HostRows h;
    h.R = int(R); h.T = int(T); h.Hh = int(full);
    h.rows = a.rows.data(); h.mask = a.mask.data();
    h.roles = a.roles.empty() ? nullptr : a.roles.data();
    h.future = a.future.empty() ? nullptr : a.future.data();
    h.future_mask = a.future_mask.empty() ? nullptr : a.future_mask.data();
    h.group_rows = int(group_rows);
    h.cap = int(cap_eff);
    tsb::BlockObserver obs;
    if (progress) obs.before = [&](int offset, int block, int length) {
        if (offset == 0 && trace) trace->clear();      // a fallback run starts again
        progress(size_t(offset), size_t(block), size_t(length));
    };
    else if (trace) obs.before = [&](int offset, int, int) { if (offset == 0) trace->clear(); };
    if (trace) obs.after = [&](const tsb::BlockView& v) { trace->push_back(block_of(v, 0, R, ps, Q)); };
    std::vector<float> out(mul(mul(R, H), Q));
    tsb::Engine& eng = *engine_;
    try {
        CallScope scope(eng, int(shot_eff), -1, (trace || progress) ? &obs : nullptr);
        eng.decode_host_rows(h, int(H), out.data());
    } catch (const Error&) {
        throw;
    } catch (const std::exception& e) {
        throw Error(e.what());
    }
    return out;
}

void Forecaster::forecast_into(const ForecastRequest& r, float* out, ForecastTrace* trace) {
    const Config& c = model_.config();
    const size_t Q = c.num_quantiles();
    if (trace) { trace->initial_anchors.reset(); trace->positive.clear(); trace->negative.clear(); }
    const bool sym = r.symmetric_averaging.value_or(c.symmetric_averaging);
    const bool clip = r.clip_nonnegative.value_or(c.clip_nonnegative);
    const double cap_k = r.quantile_real_cap_k.value_or(c.quantile_real_cap_k);
    if (!std::isfinite(cap_k)) throw Error("invalid quantile cap");
    if (!r.batch || !r.targets || !r.length || !r.horizon) throw Error("invalid row dimensions");
    const size_t shot = std::min<size_t>(r.per_shot_horizon_patches ? r.per_shot_horizon_patches : c.per_shot_horizon_patches,
                                 c.block_size);
    if (!shot) throw Error("invalid decode dimensions");
    // Trace: the observer splits each block's rows into the two passes (positive first).
    const size_t all = r.targets + r.past_count + r.categorical_past_count + r.known_count + r.categorical_known_count;
    std::optional<ForecastAnchors> anchors;
    tsb::BlockObserver obs;
    if (trace) {
        if (trace->capture_initial_anchors) anchors = ForecastAnchors{r.batch, r.targets, {}, {}};
        obs.before = [&, trace](int offset, int block, int length) {
            if (offset == 0) { trace->positive.clear(); trace->negative.clear(); }   // a fallback run starts again
            if (trace->before_block) {
                trace->before_block(size_t(offset), size_t(block), size_t(length));
                if (sym) trace->before_block(size_t(offset), size_t(block), size_t(length));
            }
        };
        obs.after = [&, trace](const tsb::BlockView& v) {
            const size_t rows = size_t(v.rows) / (sym ? 2 : 1), ps = c.patch_size;
            if (trace->capture_blocks) {
                trace->positive.push_back(block_of(v, 0, rows, ps, Q));
                if (sym) trace->negative.push_back(block_of(v, rows, rows, ps, Q));
            }
            if (anchors && v.offset == 0) {
                const std::vector<float> loc = download_rows(v.loc, 1, 0, rows, 1);
                const std::vector<float> scale = download_rows(v.scale, 1, 0, rows, 1);
                anchors->loc.resize(mul(r.batch, r.targets));
                anchors->scale.resize(anchors->loc.size());
                for (size_t b = 0; b < r.batch; ++b)
                    for (size_t v2 = 0; v2 < r.targets; ++v2) {
                        const float l = loc[b * all + v2], sc = scale[b * all + v2];
                        if (!std::isfinite(l) || !std::isfinite(sc) || sc <= 0) throw Error("invalid initial anchor");
                        anchors->loc[b * r.targets + v2] = l;
                        anchors->scale[b * r.targets + v2] = sc;
                    }
            }
        };
    }
    CallScope scope(*engine_, int(shot), cap_k, trace ? &obs : nullptr);
    forecast_request(r, out, sym, clip);
    if (trace && anchors) trace->initial_anchors = std::move(anchors);
}

void Forecaster::forecast_request(const ForecastRequest& r, float* out, bool sym, bool clip) {
    const Config& c = model_.config();
    const size_t Q = c.num_quantiles();
    if (sym)
        for (size_t i = 0; i < Q; ++i)
            if (std::abs(c.quantile_knots[i] + c.quantile_knots[Q - 1 - i] - 1) >= 1e-9)
                throw Error("symmetric averaging needs quantile levels symmetric about 0.5");
    if (r.length > size_t(INT32_MAX) || r.horizon > size_t(INT32_MAX) || r.batch * r.targets > size_t(INT32_MAX))
        throw Error("forecast dimensions exceed the device path limits");
    const bool any_cov = r.past_count || r.known_count || r.categorical_past_count || r.categorical_known_count;
    tsb::Engine& eng = *engine_;
    cuda_check(cudaSetDevice(eng.device()), "cudaSetDevice");
    if (!any_cov) {
        const size_t n = mul(mul(r.batch, r.targets), r.length);
        if (r.context.size() != n || (!r.observation_mask.empty() && r.observation_mask.size() != n))
            throw Error("row input shape mismatch");
        for (auto v : r.observation_mask) if (v != 0 && v != 1) throw Error("observation mask must be boolean");
        forecast_targets(r.context.data(),
                         r.observation_mask.empty() ? nullptr : reinterpret_cast<const uint8_t*>(r.observation_mask.data()),
                         r.batch, r.targets, r.length, r.horizon, sym, clip, r.max_context, out);
        return;
    }
    if (device_assembly_) {
        const RowGeometry g = check_rows(c, r.context, r.observation_mask, r.batch, r.targets, r.length, r.horizon, r.past,
                                         r.past_count, r.known, r.known_count, r.max_context, r.categorical_past,
                                         r.categorical_past_count, r.categorical_known, r.categorical_known_count);
        const size_t all = r.targets + r.past_count + r.categorical_past_count + r.known_count + r.categorical_known_count;
        if (mul(r.batch, all) > size_t(INT32_MAX) / 2 || g.len > size_t(INT32_MAX) || g.hor > size_t(INT32_MAX))
            throw Error("forecast dimensions exceed the device path limits");
        tsb::CovRequest q;
        q.B = int(r.batch); q.V = int(r.targets); q.T = int(r.length); q.H = int(r.horizon);
        q.P = int(r.past_count); q.K = int(r.known_count);
        q.CP = int(r.categorical_past_count); q.CK = int(r.categorical_known_count);
        q.ctx = r.context.data();
        q.umask = r.observation_mask.empty() ? nullptr : reinterpret_cast<const uint8_t*>(r.observation_mask.data());
        q.past = r.past.data(); q.known = r.known.data();
        q.cat_past = r.categorical_past.data(); q.cat_known = r.categorical_known.data();
        q.kept = int(g.kept); q.len = int(g.len); q.hor = int(g.hor);
        q.smooth = c.target_encoding_smooth;
        q.cap = int(r.max_context ? r.max_context : c.context_length);
        try {
            eng.forecast_covariates(q, sym, clip, out);
        } catch (const Error&) {
            throw;
        } catch (const std::exception& e) {
            throw Error(e.what());
        }
        return;
    }
    const AssembledRows a = assemble_rows(c, r.context, r.observation_mask, r.batch, r.targets, r.length, r.horizon, r.past,
                                          r.past_count, r.known, r.known_count, r.max_context, r.categorical_past,
                                          r.categorical_past_count, r.categorical_known, r.categorical_known_count);
    tsb::HostRows h;
    h.R = int(a.rows_count); h.T = int(a.length); h.Hh = int(a.horizon);
    h.rows = a.rows.data(); h.mask = a.mask.data();
    h.roles = a.roles.empty() ? nullptr : a.roles.data();
    h.future = a.future.empty() ? nullptr : a.future.data();
    h.future_mask = a.future_mask.empty() ? nullptr : a.future_mask.data();
    h.group_rows = int(a.rows_count / r.batch);
    h.cap = int(r.max_context ? r.max_context : c.context_length);
    std::vector<uint8_t> um(r.observation_mask.begin(), r.observation_mask.end());
    try {
        eng.forecast_rows(h, int(r.batch), int(r.targets), int(r.horizon), sym, clip, r.context.data(),
                          um.empty() ? nullptr : um.data(), int(r.length), out);
    } catch (const Error&) {
        throw;
    } catch (const std::exception& e) {
        throw Error(e.what());
    }
}

}  // namespace ts
