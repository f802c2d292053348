// C entry points into the reference's own sources, compiled from the reference's src/ by
// oracle/ref/Makefile into oracle/_ref/libtsref.so — TEST INFRASTRUCTURE ONLY: the tests use
// it to pin the CPU oracle (oracle/oracle.cpp) against the reference's real code.
//
// Besides the wrappers, this file defines the small part of ggml those sources call:
// tensor metadata helpers, and ggml_custom_4d evaluated eagerly (the reference's F32 ops
// are ggml custom nodes whose callbacks are the reference's own functions, so a custom node
// evaluated at construction computes exactly what the reference computes). Graph runtime
// entry points that the wrapped functions never reach abort.
#include "../oracle.h"

#include "config.hpp"
#include "covariates.hpp"
#include "head.hpp"
#include "layers.hpp"
#include "masks.hpp"
#include "refine.hpp"
#include "scaler.hpp"

#include <cmath>
#include <cstdlib>
#include <cstring>
#include <memory>
#include <string>
#include <vector>

struct ggml_context {
    std::vector<std::unique_ptr<ggml_tensor>> tensors;
    std::vector<std::vector<float>> buffers;
};

namespace {

[[noreturn]] void unreachable(const char* what) {
    std::fprintf(stderr, "oracle/_ref: %s is not available in the reference oracle\n", what);
    std::abort();
}

ggml_tensor* make_tensor(ggml_context* ctx, ggml_type type, int64_t a, int64_t b, int64_t c, int64_t d, float* data) {
    auto t = std::make_unique<ggml_tensor>();
    std::memset(t.get(), 0, sizeof(ggml_tensor));
    t->type = type;
    t->ne[0] = a; t->ne[1] = b; t->ne[2] = c; t->ne[3] = d;
    t->nb[0] = 4;
    for (int i = 1; i < 4; ++i) t->nb[i] = t->nb[i - 1] * size_t(t->ne[i - 1]);
    if (!data && ctx) {
        ctx->buffers.emplace_back(size_t(a * b * c * d));
        data = ctx->buffers.back().data();
    }
    t->data = data;
    ggml_tensor* p = t.get();
    if (ctx) ctx->tensors.push_back(std::move(t));
    else t.release();
    return p;
}

ts::Config to_config(const oracle_config* c) {
    ts::Config r;
    r.patch_size = uint32_t(c->patch_size); r.d_model = uint32_t(c->d_model); r.num_heads = uint32_t(c->num_heads);
    r.mlp_hidden_dim = uint32_t(c->mlp_hidden_dim); r.n_layers = uint32_t(c->n_layers);
    for (int i = 0; i < c->n_layers; ++i)
        r.block_schedule.push_back(c->schedule[i] == 0 ? ts::LayerKind::Time : c->schedule[i] == 1 ? ts::LayerKind::Variate
                                   : c->schedule[i] == 2 ? ts::LayerKind::TimeVariate : ts::LayerKind::VariateTime);
    r.quantile_knots.assign(c->knots, c->knots + c->num_quantiles);
    r.block_size = uint32_t(c->block_size); r.context_length = uint32_t(c->context_length);
    r.rope_dim = uint32_t(c->rope_dim); r.rope_table_pos_min = c->rope_table_pos_min;
    r.norm_eps = c->norm_eps; r.attn_bias = c->attn_bias; r.mlp_bias = c->mlp_bias;
    r.minimum_scale = c->minimum_scale; r.use_asinh = c->use_asinh; r.covariate_enabled = c->covariate_enabled;
    r.attend_missing_patches = c->attend_missing_patches; r.quantile_width_factor = c->quantile_width_factor;
    r.per_shot_horizon_patches = uint32_t(c->per_shot_horizon_patches); r.quantile_real_cap_k = c->quantile_real_cap_k;
    r.extreme_value_threshold = c->extreme_value_threshold; r.symmetric_averaging = c->symmetric_averaging;
    r.clip_nonnegative = c->clip_nonnegative; r.target_encoding_smooth = c->target_encoding_smooth;
    return r;
}

thread_local std::string g_error;
template <class F> int guarded(F f) {
    try { f(); g_error.clear(); return 0; }
    catch (const std::exception& e) { g_error = e.what(); return 1; }
}

}  // namespace

// ---- the part of ggml the compiled reference sources call -----------------------------
extern "C" {
int64_t ggml_nelements(const ggml_tensor* t) { return t->ne[0] * t->ne[1] * t->ne[2] * t->ne[3]; }
size_t ggml_nbytes(const ggml_tensor* t) { return size_t(ggml_nelements(t)) * 4; }
bool ggml_is_contiguous(const ggml_tensor* t) {
    size_t b = 4;
    for (int i = 0; i < 4; ++i) { if (t->ne[i] != 1 && t->nb[i] != b) return false; b *= size_t(t->ne[i]); }
    return true;
}
bool ggml_are_same_shape(const ggml_tensor* a, const ggml_tensor* b) {
    for (int i = 0; i < 4; ++i) if (a->ne[i] != b->ne[i]) return false;
    return true;
}
int64_t ggml_blck_size(ggml_type t) { return t == GGML_TYPE_Q8_0 ? 32 : t >= GGML_TYPE_Q4_K && t <= GGML_TYPE_Q6_K ? 256 : 1; }
const char* ggml_type_name(ggml_type) { return "type"; }
ggml_tensor* ggml_new_tensor_1d(ggml_context* c, ggml_type t, int64_t a) { return make_tensor(c, t, a, 1, 1, 1, nullptr); }
ggml_tensor* ggml_new_tensor_2d(ggml_context* c, ggml_type t, int64_t a, int64_t b) { return make_tensor(c, t, a, b, 1, 1, nullptr); }
ggml_tensor* ggml_new_tensor_3d(ggml_context* c, ggml_type t, int64_t a, int64_t b, int64_t d) { return make_tensor(c, t, a, b, d, 1, nullptr); }
ggml_tensor* ggml_new_tensor_4d(ggml_context* c, ggml_type t, int64_t a, int64_t b, int64_t d, int64_t e) { return make_tensor(c, t, a, b, d, e, nullptr); }
ggml_tensor* ggml_dup_tensor(ggml_context*, const ggml_tensor*) { unreachable("ggml_dup_tensor"); }
void ggml_set_input(ggml_tensor* t) { t->flags |= GGML_TENSOR_FLAG_INPUT; }
ggml_tensor* ggml_view_3d(ggml_context*, ggml_tensor*, int64_t, int64_t, int64_t, size_t, size_t, size_t) { unreachable("ggml_view_3d"); }
ggml_tensor* ggml_view_4d(ggml_context*, ggml_tensor*, int64_t, int64_t, int64_t, int64_t, size_t, size_t, size_t, size_t) { unreachable("ggml_view_4d"); }
ggml_tensor* ggml_permute(ggml_context*, ggml_tensor*, int, int, int, int) { unreachable("ggml_permute"); }
ggml_tensor* ggml_cont(ggml_context*, ggml_tensor*) { unreachable("ggml_cont"); }
ggml_tensor* ggml_concat(ggml_context*, ggml_tensor*, ggml_tensor*, int) { unreachable("ggml_concat"); }
ggml_tensor* ggml_neg(ggml_context*, ggml_tensor*) { unreachable("ggml_neg"); }
ggml_tensor* ggml_add(ggml_context*, ggml_tensor*, ggml_tensor*) { unreachable("ggml_add"); }
ggml_tensor* ggml_mul(ggml_context*, ggml_tensor*, ggml_tensor*) { unreachable("ggml_mul"); }
ggml_tensor* ggml_silu(ggml_context*, ggml_tensor*) { unreachable("ggml_silu"); }
ggml_tensor* ggml_mul_mat(ggml_context*, ggml_tensor*, ggml_tensor*) { unreachable("ggml_mul_mat"); }
// Custom node: allocate the output and run the reference callback on one thread now.
ggml_tensor* ggml_custom_4d(ggml_context* ctx, ggml_type type, int64_t a, int64_t b, int64_t c, int64_t d, ggml_tensor** args,
                            int n_args, ggml_custom_op_t fun, int, void* userdata) {
    ggml_tensor* t = make_tensor(ctx, type, a, b, c, d, nullptr);
    t->op = GGML_OP_CUSTOM;
    for (int i = 0; i < n_args && i < GGML_MAX_SRC; ++i) t->src[i] = args[i];
    fun(t, 0, 1, userdata);
    return t;
}
}

namespace ts {
GraphRunner::GraphRunner(size_t) { unreachable("GraphRunner"); }
GraphRunner::~GraphRunner() {}
ggml_context* GraphRunner::begin() { unreachable("GraphRunner::begin"); }
void GraphRunner::allocate(const std::vector<ggml_tensor*>&) { unreachable("GraphRunner::allocate"); }
void GraphRunner::upload(ggml_tensor*, const std::vector<float>&) { unreachable("GraphRunner::upload"); }
void GraphRunner::compute() { unreachable("GraphRunner::compute"); }
std::vector<float> GraphRunner::read(ggml_tensor*) const { unreachable("GraphRunner::read"); }
ggml_tensor* Model::tensor(const std::string&) const { unreachable("Model::tensor"); }
}  // namespace ts

// ---- wrappers -----------------------------------------------------------------------------
extern "C" {

const char* ref_last_error(void) { return g_error.c_str(); }

int ref_scale_rows(const oracle_config* c, const float* x, const int8_t* mask, int64_t rows, int64_t length, float* scaled,
                   float* loc, float* scale) {
    return guarded([&] {
        auto r = ts::scale_rows(to_config(c), std::vector<float>(x, x + rows * length),
                                std::vector<int8_t>(mask, mask + rows * length), size_t(rows), size_t(length));
        std::memcpy(scaled, r.scaled.data(), r.scaled.size() * 4);
        std::memcpy(loc, r.loc.data(), r.loc.size() * 4);
        std::memcpy(scale, r.scale.data(), r.scale.size() * 4);
    });
}

int ref_instance_norm_stats(const oracle_config* c, const float* x, const int8_t* mask, int64_t rows, int64_t length,
                            float* loc, float* scale, int8_t* is_binary) {
    return guarded([&] {
        auto r = ts::instance_norm_stats(to_config(c), std::vector<float>(x, x + rows * length),
                                         std::vector<int8_t>(mask, mask + rows * length), size_t(rows), size_t(length));
        std::memcpy(loc, r.loc.data(), rows * 4);
        std::memcpy(scale, r.scale.data(), rows * 4);
        std::memcpy(is_binary, r.is_binary.data(), rows);
    });
}

int ref_build_masks(const oracle_config* c, const int8_t* observed, int64_t R, int64_t T, int64_t h, const int64_t* groups,
                    const int64_t* roles, int8_t* obs, int8_t* key_valid, int64_t* first_group, int64_t* positions,
                    int8_t* time_allowed, int8_t* variate, int8_t* active, int64_t* anchor) {
    return guarded([&] {
        std::vector<int64_t> ro;
        if (roles) ro.assign(roles, roles + R);
        auto a = ts::build_masks(to_config(c), std::vector<int8_t>(observed, observed + R * T), size_t(R), size_t(T),
                                 size_t(h), std::vector<int64_t>(groups, groups + R), ro);
        std::memcpy(obs, a.obs.data(), a.obs.size());
        std::memcpy(key_valid, a.key_valid.data(), a.key_valid.size());
        std::memcpy(first_group, a.first_group.data(), a.first_group.size() * 8);
        std::memcpy(positions, a.positions.data(), a.positions.size() * 8);
        std::memcpy(time_allowed, a.time.allowed.data(), a.time.allowed.size());
        if (variate && !a.variate.empty()) std::memcpy(variate, a.variate.data(), a.variate.size());
        if (active && !a.active.empty()) std::memcpy(active, a.active.data(), a.active.size());
        if (anchor && !a.anchor.empty()) std::memcpy(anchor, a.anchor.data(), a.anchor.size() * 8);
    });
}

// The reference SDPA callback (src/layers.cpp:619-627) on q/k/v [R][S][H*hd], additive mask [R][S][S].
int ref_sdpa(const float* q, const float* k, const float* v, const float* mask, int64_t hd, int64_t H, int64_t S, int64_t R,
             int64_t split, float* out, int32_t threads) {
    return guarded([&] {
        ggml_tensor qt{}, kt{}, vt{}, mt{}, dst{};
        qt.ne[0] = hd; qt.ne[1] = H; qt.ne[2] = S; qt.ne[3] = R;
        qt.data = const_cast<float*>(q); kt.data = const_cast<float*>(k); vt.data = const_cast<float*>(v);
        mt.data = const_cast<float*>(mask);
        dst.src[0] = &qt; dst.src[1] = &kt; dst.src[2] = &vt; dst.src[3] = &mt;
        dst.data = out;
        for (int ith = 0; ith < threads; ++ith)
            ts::detail::sdpa_f32(&dst, ith, threads, reinterpret_cast<void*>(uintptr_t(split)));
    });
}

// The reference F32 linear callback (src/layers.cpp:187-222).
int ref_linear_f32(const float* w, const float* x, const float* b, int64_t K, int64_t N, int64_t rows, float* y) {
    return guarded([&] {
        ggml_tensor wt{}, xt{}, bt{}, dst{};
        wt.ne[0] = K; wt.ne[1] = N; wt.ne[2] = 1; wt.ne[3] = 1; wt.data = const_cast<float*>(w);
        xt.ne[0] = K; xt.ne[1] = rows; xt.ne[2] = 1; xt.ne[3] = 1; xt.data = const_cast<float*>(x);
        bt.ne[0] = N; bt.ne[1] = 1; bt.ne[2] = 1; bt.ne[3] = 1; bt.data = const_cast<float*>(b);
        dst.ne[0] = N; dst.ne[1] = rows; dst.ne[2] = 1; dst.ne[3] = 1; dst.data = y;
        dst.src[0] = &wt; dst.src[1] = &xt; dst.src[2] = b ? &bt : nullptr;
        ts::detail::linear_f32(&dst, 0, 1, nullptr);
    });
}

// The reference float64-accumulated head projection (src/head.cpp:269-274).
int ref_head_linear_f64(const float* w, const float* x, int64_t K, int64_t N, int64_t rows, float* y) {
    return guarded([&] {
        ggml_tensor wt{}, xt{}, dst{};
        wt.ne[0] = K; wt.ne[1] = N; wt.ne[2] = 1; wt.ne[3] = 1; wt.data = const_cast<float*>(w);
        xt.ne[0] = K; xt.ne[1] = rows; xt.ne[2] = 1; xt.ne[3] = 1; xt.data = const_cast<float*>(x);
        dst.ne[0] = N; dst.ne[1] = rows; dst.ne[2] = 1; dst.ne[3] = 1; dst.data = y;
        dst.src[0] = &wt; dst.src[1] = &xt; dst.src[2] = nullptr;
        ts::detail::head_linear_f64(&dst, 0, 1, nullptr);
    });
}

// The reference RMSNorm node (src/layers.cpp:279-292), evaluated eagerly.
int ref_rms_norm(const float* x, const float* w, int64_t rows, int64_t D, float eps, float* out) {
    return guarded([&] {
        ggml_context ctx;
        ggml_tensor* xt = make_tensor(&ctx, GGML_TYPE_F32, D, rows, 1, 1, const_cast<float*>(x));
        ggml_tensor* wt = make_tensor(&ctx, GGML_TYPE_F32, D, 1, 1, 1, const_cast<float*>(w));
        ggml_tensor* y = ts::rms_norm(&ctx, xt, wt, eps);
        std::memcpy(out, y->data, size_t(rows * D) * 4);
    });
}

// The reference sigmoid node (src/layers.cpp:668-674), evaluated eagerly.
int ref_sigmoid(const float* x, int64_t n, float* out) {
    return guarded([&] {
        ggml_context ctx;
        ggml_tensor* xt = make_tensor(&ctx, GGML_TYPE_F32, n, 1, 1, 1, const_cast<float*>(x));
        ggml_tensor* y = ts::sigmoid(&ctx, xt);
        std::memcpy(out, y->data, size_t(n) * 4);
    });
}

int ref_monotone_quantiles(const oracle_config* c, const float* raw, int64_t n, float* out) {
    return guarded([&] {
        auto v = ts::monotone_quantiles(to_config(c), std::vector<float>(raw, raw + n));
        std::memcpy(out, v.data(), size_t(n) * 4);
    });
}

int ref_denormalize(const float* x, const float* loc, const float* scale, int64_t rows, int64_t stride, int64_t Q,
                    int32_t use_asinh, float* out) {
    return guarded([&] {
        auto v = ts::denormalize_quantiles(std::vector<float>(x, x + rows * stride), std::vector<float>(loc, loc + rows),
                                           std::vector<float>(scale, scale + rows), size_t(Q), use_asinh != 0);
        std::memcpy(out, v.data(), v.size() * 4);
    });
}

int ref_refine_block(const oracle_config* c, const float* q, const float* x, const int8_t* mask, int64_t rows,
                     int64_t length, int64_t patches, const int8_t* targets, float* out) {
    return guarded([&] {
        const size_t n = size_t(rows) * patches * c->patch_size * c->num_quantiles;
        std::vector<int8_t> tg;
        if (targets) tg.assign(targets, targets + rows);
        auto v = ts::refine_block(to_config(c), std::vector<float>(q, q + n), std::vector<float>(x, x + rows * length),
                                  std::vector<int8_t>(mask, mask + rows * length), size_t(rows), size_t(length),
                                  size_t(patches), tg);
        std::memcpy(out, v.data(), n * 4);
    });
}

int ref_block_frames(const oracle_config* c, const float* x, const int8_t* mask, const double* median, int64_t rows,
                     int64_t length, int64_t patches, double* loc, double* scale) {
    return guarded([&] {
        auto f = ts::advancing_block_frames(to_config(c), std::vector<float>(x, x + rows * length),
                                            std::vector<int8_t>(mask, mask + rows * length),
                                            std::vector<double>(median, median + rows * patches * c->patch_size),
                                            size_t(rows), size_t(length), size_t(patches));
        std::memcpy(loc, f.loc.data(), f.loc.size() * 8);
        std::memcpy(scale, f.scale.data(), f.scale.size() * 8);
    });
}

// Row assembly (src/covariates.cpp:32-72). Outputs sized by the caller: rows/mask [R][len],
// groups [R], roles [R] (if any covariate), future/future_mask [R][hor] (if known covariates).
int ref_assemble_rows(const oracle_config* c, const oracle_request* r, int64_t* R, int64_t* len, int64_t* hor, float* rows,
                      int8_t* mask, int64_t* groups, int64_t* roles, float* future, int8_t* future_mask) {
    return guarded([&] {
        const size_t B = r->B, V = r->V, T = r->T, H = r->prediction_length, TH = T + H;
        std::vector<float> ctx(r->context, r->context + B * V * T);
        std::vector<int8_t> um;
        if (r->observation_mask) um.assign(r->observation_mask, r->observation_mask + B * V * T);
        auto vec = [](const float* p, size_t n) { return p ? std::vector<float>(p, p + n) : std::vector<float>(); };
        auto vecd = [](const double* p, size_t n) { return p ? std::vector<double>(p, p + n) : std::vector<double>(); };
        auto a = ts::assemble_rows(to_config(c), ctx, um, B, V, T, H, vec(r->past_cov, B * r->c_past * T), size_t(r->c_past),
                                   vec(r->known_cov, B * r->c_known * TH), size_t(r->c_known), size_t(r->max_context),
                                   vecd(r->cat_past, B * r->cc_past * T), size_t(r->cc_past),
                                   vecd(r->cat_known, B * r->cc_known * TH), size_t(r->cc_known));
        *R = int64_t(a.rows_count); *len = int64_t(a.length); *hor = int64_t(a.horizon);
        if (rows) std::memcpy(rows, a.rows.data(), a.rows.size() * 4);
        if (mask) std::memcpy(mask, a.mask.data(), a.mask.size());
        if (groups) std::memcpy(groups, a.groups.data(), a.groups.size() * 8);
        if (roles && !a.roles.empty()) std::memcpy(roles, a.roles.data(), a.roles.size() * 8);
        if (future && !a.future.empty()) std::memcpy(future, a.future.data(), a.future.size() * 4);
        if (future_mask && !a.future_mask.empty()) std::memcpy(future_mask, a.future_mask.data(), a.future_mask.size());
    });
}

}  // extern "C"
