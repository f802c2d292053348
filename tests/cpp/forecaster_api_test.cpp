// The C++ API of the library (ts::Model::load, ts::Forecaster::forecast with its trace, and
// ts::Forecaster::decode) against the C ABI and against itself, on a GPU. Built and run by
// tests/test_cpp_api.py: forecaster_api_test <model.gguf>. Prints "OK <checks>" on success.
//
// What it checks (after the reference's tests/test_capi.cpp transport check and
// tests/test_forecast_anchors.cpp trace checks):
//  * Forecaster::forecast and timestral_capi_forecast give the same bytes, with and without
//    covariates;
//  * a trace leaves the quantiles unchanged; full and anchor-only traces agree on blocks,
//    anchors and progress calls; the first block holds the assembled rows; anchors are
//    published only when the forecast succeeds;
//  * decode() of the assembled rows equals the forecast without symmetric averaging, clip and
//    cap, and its first block equals the forecast trace's first positive block;
//  * each decode block's context follows from the previous block (the reference's feedback
//    contract), at the model's cap and at a cap that slides every block;
//  * the per-request overrides (per-shot patches, cap factor) change the result as requested.
#include "forecaster.hpp"
#include "timestral_capi.h"

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <random>
#include <string>
#include <vector>

namespace {

int checks = 0;

void check(bool ok, const char* what) {
    ++checks;
    if (!ok) {
        std::fprintf(stderr, "FAILED: %s\n", what);
        std::exit(1);
    }
}

template <class T>
bool same_bytes(const std::vector<T>& a, const std::vector<T>& b) {
    return a.size() == b.size() && (a.empty() || !std::memcmp(a.data(), b.data(), a.size() * sizeof(T)));
}

void same_blocks(const std::vector<ts::DecodeBlock>& a, const std::vector<ts::DecodeBlock>& b) {
    check(a.size() == b.size(), "block counts");
    for (size_t i = 0; i < a.size(); ++i) {
        check(a[i].offset == b[i].offset && a[i].patches == b[i].patches && a[i].length == b[i].length, "block metadata");
        check(same_bytes(a[i].context, b[i].context) && same_bytes(a[i].mask, b[i].mask), "block context bytes");
        check(same_bytes(a[i].future, b[i].future) && same_bytes(a[i].future_mask, b[i].future_mask), "block future bytes");
        check(same_bytes(a[i].predicted, b[i].predicted) && same_bytes(a[i].refined, b[i].refined), "block quantile bytes");
    }
}

// Each block's context is the previous block's context followed by that block's refined
// medians, slid to the cap in whole patches (reference tests/test_forecast.cpp
// feedback_contract, src/forecaster.cpp decode_impl): a median that is not finite or at
// least the extreme-value threshold feeds back as 0, past-covariate rows (role 1) feed back
// 0 unobserved, known-covariate rows (role 2) their known future; bytes and masks exact.
void feedback_contract(const ts::Config& c, const std::vector<ts::DecodeBlock>& blocks,
                       const std::vector<int64_t>& roles, size_t R, size_t cap) {
    const size_t Q = c.num_quantiles(), ps = c.patch_size, med = c.median_index();
    for (size_t k = 1; k < blocks.size(); ++k) {
        const ts::DecodeBlock& b = blocks[k - 1];
        const ts::DecodeBlock& a = blocks[k];
        const size_t n = b.patches * ps, joined = b.length + n;
        const size_t keep = joined > cap ? std::max(ps, cap / ps * ps) : joined, start = joined - keep;
        check(a.offset == b.offset + n && a.length == keep && a.context.size() == R * keep && a.mask.size() == R * keep &&
                  b.refined.size() == R * n * Q,
              "feedback: block offsets and context length");
        bool ok = true;
        for (size_t row = 0; row < R && ok; ++row)
            for (size_t t = 0; t < keep && ok; ++t) {
                const size_t from = start + t;
                float v;
                int8_t observed;
                if (from < b.length) {
                    v = b.context[row * b.length + from];
                    observed = b.mask[row * b.length + from];
                } else {
                    const size_t j = from - b.length;
                    v = b.refined[(row * n + j) * Q + med];
                    observed = 1;
                    if (!std::isfinite(v) || std::abs(v) >= c.extreme_value_threshold) v = 0;
                    const int64_t role = roles.empty() ? 0 : roles[row];
                    if (role == 1) { v = 0; observed = 0; }
                    if (role == 2) { v = b.future[row * n + j]; observed = b.future_mask[row * n + j]; }
                }
                ok = !std::memcmp(&v, &a.context[row * keep + t], sizeof(float)) && observed == a.mask[row * keep + t];
            }
        check(ok, "feedback: context values and masks");
    }
}

ts::ForecastRequest make_request(bool covariates, unsigned seed) {
    std::mt19937 rng(seed);
    std::normal_distribution<float> n01(0.f, 1.f);
    ts::ForecastRequest r;
    r.batch = 2; r.targets = covariates ? 1 : 2; r.length = 200; r.horizon = 160;
    r.context.resize(r.batch * r.targets * r.length);
    float level = 5.f;
    for (size_t i = 0; i < r.context.size(); ++i) {
        level += n01(rng);
        r.context[i] = (i % 17 == 3) ? NAN : level;
    }
    if (covariates) {
        r.past_count = 2; r.known_count = 1; r.categorical_known_count = 1;
        r.past.resize(r.batch * 2 * r.length);
        for (auto& v : r.past) v = n01(rng);
        r.known.resize(r.batch * 1 * (r.length + r.horizon));
        for (auto& v : r.known) v = n01(rng);
        r.categorical_known.resize(r.batch * 1 * (r.length + r.horizon));
        for (auto& v : r.categorical_known) v = double(rng() % 5);
    }
    r.per_shot_horizon_patches = 2;          // 5 horizon patches: three decode blocks
    return r;
}

std::vector<float> capi_forecast(timestral_ctx* h, const ts::ForecastRequest& r) {
    timestral_forecast_request q{};
    q.context = r.context.data();
    q.B = int32_t(r.batch); q.V = int32_t(r.targets); q.T = int32_t(r.length); q.prediction_length = int32_t(r.horizon);
    q.past_cov = r.past.empty() ? nullptr : r.past.data(); q.c_past = int32_t(r.past_count);
    q.known_cov = r.known.empty() ? nullptr : r.known.data(); q.c_known = int32_t(r.known_count);
    q.cat_known = r.categorical_known.empty() ? nullptr : r.categorical_known.data();
    q.cc_known = int32_t(r.categorical_known_count);
    q.symmetric_averaging = q.clip_nonnegative = -1;
    int32_t Q = 0;
    float* out = timestral_capi_forecast(h, &q, &Q);
    check(out != nullptr, "C ABI forecast");
    std::vector<float> v(out, out + r.batch * r.targets * r.horizon * size_t(Q));
    timestral_capi_free_buffer(out);
    return v;
}

ts::AssembledRows assemble(const ts::Model& m, const ts::ForecastRequest& r) {
    return ts::assemble_rows(m.config(), r.context, r.observation_mask, r.batch, r.targets, r.length, r.horizon, r.past,
                             r.past_count, r.known, r.known_count, r.max_context, r.categorical_past,
                             r.categorical_past_count, r.categorical_known, r.categorical_known_count);
}

void run(const ts::Model& m, ts::Forecaster& fc, timestral_ctx* h, bool covariates) {
    const auto& c = m.config();
    const size_t Q = c.num_quantiles();
    ts::ForecastRequest r = make_request(covariates, covariates ? 11u : 7u);

    // Transport: the C++ API and the C ABI give the same bytes (the C ABI has no per-shot
    // field, so this request uses the model's).
    ts::ForecastRequest t = r;
    t.per_shot_horizon_patches = 0;
    check(same_bytes(fc.forecast(t).quantiles, capi_forecast(h, t)), "C++ forecast bytes == C ABI bytes");

    // Traces (reference tests/test_forecast_anchors.cpp).
    const auto plain = fc.forecast(r);
    ts::ForecastTrace original;
    size_t progress = 0;
    original.before_block = [&](size_t, size_t, size_t) { ++progress; };
    const auto full = fc.forecast(r, &original);
    check(same_bytes(plain.quantiles, full.quantiles), "default trace output");
    check(!original.initial_anchors, "default has no anchors");
    check(original.positive.size() == 3 && original.negative.size() == 3, "three blocks per pass");
    check(progress == 6, "one progress call per block and pass");
    ts::ForecastTrace captured;
    captured.capture_initial_anchors = true;
    const auto with = fc.forecast(r, &captured);
    check(same_bytes(plain.quantiles, with.quantiles), "capture output");
    same_blocks(original.positive, captured.positive);
    same_blocks(original.negative, captured.negative);
    ts::ForecastTrace only;
    only.capture_initial_anchors = true;
    only.capture_blocks = false;
    size_t count = 0;
    only.before_block = [&](size_t, size_t, size_t) { ++count; };
    const auto light = fc.forecast(r, &only);
    check(same_bytes(plain.quantiles, light.quantiles), "anchor-only output");
    check(only.positive.empty() && only.negative.empty() && count == progress, "anchor-only blocks and progress");
    check(only.initial_anchors && captured.initial_anchors, "anchor presence");
    const ts::ForecastAnchors anchor = *only.initial_anchors;   // a copy: `only` is reused below
    check(anchor.batch == r.batch && anchor.targets == r.targets, "anchor dimensions");
    check(same_bytes(anchor.loc, captured.initial_anchors->loc) && same_bytes(anchor.scale, captured.initial_anchors->scale),
          "anchor modes");
    for (size_t i = 0; i < anchor.loc.size(); ++i)
        check(std::isfinite(anchor.loc[i]) && anchor.scale[i] > 0, "anchor values");

    const ts::AssembledRows a = assemble(m, r);
    const auto& first = captured.positive.at(0);
    check(first.offset == 0 && first.patches == 2 && first.length == a.length, "first positive block");
    check(same_bytes(first.context, a.rows) && same_bytes(first.mask, a.mask), "assembled context and mask");
    if (!a.future.empty()) {
        const size_t n = first.patches * c.patch_size;
        std::vector<float> fut;
        std::vector<int8_t> fm;
        for (size_t row = 0; row < a.rows_count; ++row) {
            fut.insert(fut.end(), a.future.begin() + row * a.horizon, a.future.begin() + row * a.horizon + n);
            fm.insert(fm.end(), a.future_mask.begin() + row * a.horizon, a.future_mask.begin() + row * a.horizon + n);
        }
        check(same_bytes(first.future, fut) && same_bytes(first.future_mask, fm), "assembled first future");
    }
    const auto& neg = captured.negative.at(0);
    bool mirrored = neg.context.size() == first.context.size();
    for (size_t i = 0; mirrored && i < neg.context.size(); ++i) mirrored = neg.context[i] == -first.context[i];
    check(mirrored, "the mirrored pass holds the negated rows");

    // Block feedback on the device, both passes: at the model's cap (no slide here) and at a
    // cap of four patches (every later block slides).
    feedback_contract(c, captured.positive, a.roles, a.rows_count, c.context_length);
    feedback_contract(c, captured.negative, a.roles, a.rows_count, c.context_length);
    ts::ForecastRequest capped = r;
    capped.max_context = 4 * c.patch_size;
    ts::ForecastTrace slid;
    fc.forecast(capped, &slid);
    const ts::AssembledRows ac = assemble(m, capped);
    check(slid.positive.size() == 3 && slid.positive[0].length == capped.max_context, "capped blocks");
    feedback_contract(c, slid.positive, ac.roles, ac.rows_count, capped.max_context);
    feedback_contract(c, slid.negative, ac.roles, ac.rows_count, capped.max_context);

    // Transactional anchors: a failing forecast leaves none.
    only.capture_initial_anchors = false;
    fc.forecast(r, &only);
    check(!only.initial_anchors, "disabled capture clears");
    only.capture_initial_anchors = true;
    ts::ForecastRequest bad = r;
    bad.context.clear();
    bool failed = false;
    try { fc.forecast(bad, &only); } catch (const ts::Error&) { failed = true; }
    check(failed && !only.initial_anchors, "assembly failure clears");
    bad = r;
    bad.quantile_real_cap_k = NAN;
    failed = false;
    try { fc.forecast(bad, &only); } catch (const ts::Error&) { failed = true; }
    check(failed && !only.initial_anchors, "invalid cap leaves no anchors");
    ts::ForecastRequest positive_only = r;
    positive_only.symmetric_averaging = false;
    ts::ForecastTrace pos;
    pos.capture_initial_anchors = true;
    pos.capture_blocks = false;
    fc.forecast(positive_only, &pos);
    check(pos.initial_anchors && same_bytes(pos.initial_anchors->loc, anchor.loc) &&
              same_bytes(pos.initial_anchors->scale, anchor.scale),
          "symmetry leaves the initial anchors");

    // decode(): one pass without cap, symmetric average or clip.
    std::vector<ts::DecodeBlock> blocks;
    size_t calls = 0;
    const auto dec = fc.decode(a, r.horizon, 0, 2, &blocks, [&](size_t, size_t, size_t) { ++calls; });
    check(dec.size() == a.rows_count * r.horizon * Q && blocks.size() == 3 && calls == 3, "decode shape, blocks, progress");
    same_blocks(std::vector<ts::DecodeBlock>(blocks.begin(), blocks.begin() + 1),
                std::vector<ts::DecodeBlock>(captured.positive.begin(), captured.positive.begin() + 1));
    ts::ForecastRequest raw = r;
    raw.symmetric_averaging = false;
    raw.clip_nonnegative = false;
    raw.quantile_real_cap_k = 0.0;
    const auto out = fc.forecast(raw).quantiles;
    const size_t all = a.rows_count / r.batch, HQ = r.horizon * Q;
    bool equal = true;
    for (size_t b = 0; b < r.batch; ++b)
        for (size_t v = 0; v < r.targets; ++v)
            equal &= !std::memcmp(dec.data() + (b * all + v) * HQ, out.data() + (b * r.targets + v) * HQ, HQ * 4);
    check(equal, "decode equals the forecast without symmetric average, clip and cap");
    bool threw = false;
    ts::AssembledRows broken = a;
    broken.groups[0] = 99;
    try { fc.decode(broken, r.horizon); } catch (const ts::Error&) { threw = true; }
    check(threw, "decode rejects non-contiguous groups");

    // Overrides: one patch per block differs from two; cap factor 0 equals the uncapped decode.
    ts::ForecastRequest one = r;
    one.per_shot_horizon_patches = 1;
    check(!same_bytes(fc.forecast(one).quantiles, plain.quantiles), "per-shot override changes the forecast");
    ts::ForecastTrace one_trace;
    fc.forecast(one, &one_trace);
    check(one_trace.positive.size() == 5, "per-shot override: five blocks");
}

}  // namespace

int main(int argc, char** argv) {
    if (argc < 2) {
        std::fprintf(stderr, "usage: forecaster_api_test <model.gguf>\n");
        return 2;
    }
    try {
        ts::Model m = ts::Model::load(argv[1]);
        ts::Forecaster fc(m);
        timestral_ctx* h = timestral_capi_load(argv[1], 1);
        check(h != nullptr, "C ABI load");
        run(m, fc, h, false);
        run(m, fc, h, true);
        // A moved model keeps working for a new forecaster (reference src/model_loader.hpp:
        // movable; a forecaster needs its model to outlive it, so the first is not used again).
        const ts::ForecastRequest r = make_request(false, 7u);
        const auto before = fc.forecast(r).quantiles;
        ts::Model moved = std::move(m);
        ts::Forecaster fc2(moved);
        check(same_bytes(fc2.forecast(r).quantiles, before), "moved model, second forecaster");
        timestral_capi_free(h);
    } catch (const ts::Error& e) {
        std::fprintf(stderr, "FAILED with ts::Error: %s\n", e.what());
        return 1;
    }
    std::printf("OK %d checks\n", checks);
    return 0;
}
