// ts::Forecaster: the reference's forecast entry (reference src/forecaster.hpp:9-56) on a
// B200. Every request runs on the GPU from row assembly to the final quantiles: requests
// without covariates from the raw context, requests with covariates from their raw arrays
// (forward fill, casts and categorical target encoding on the device; the host assembly,
// assemble_rows, stays available for comparison and for decode()).
#pragma once
#include "model.hpp"

#include <cstdint>
#include <functional>
#include <memory>
#include <optional>
#include <vector>

namespace tsb { class Engine; }

namespace ts {

// Canonical packed inputs (B,V,T), (B,C,T), (B,C,T+H); NaN = missing.
struct ForecastRequest {
    size_t batch = 0, targets = 0, length = 0, horizon = 0;
    std::vector<float> context, past, known;
    std::vector<int8_t> observation_mask;
    std::vector<double> categorical_past, categorical_known;
    size_t past_count = 0, known_count = 0, categorical_past_count = 0, categorical_known_count = 0;
    size_t max_context = 0, per_shot_horizon_patches = 0;
    std::optional<bool> symmetric_averaging, clip_nonnegative;
    std::optional<double> quantile_real_cap_k;
};

struct Forecast {
    size_t batch = 0, targets = 0, horizon = 0;
    std::vector<double> quantile_levels;
    std::vector<float> quantiles;  // (B,V,H,Q)
};

// Host row assembly (reference src/covariates.cpp:32-72).
struct AssembledRows {
    size_t rows_count = 0, length = 0, horizon = 0;
    std::vector<float> rows, future;
    std::vector<int8_t> mask, future_mask;
    std::vector<int64_t> roles, groups;
};

// Audit types of the reference (src/forecaster.hpp:24-38), same fields and meaning.
// One decode block: its first step, patches and context length; the context rows and masks
// it was predicted from, its slice of the known future, its quantiles before (predicted)
// and after (refined) the advancing-frame refinement, all rows of one pass.
struct DecodeBlock {
    size_t offset = 0, patches = 0, length = 0;
    std::vector<float> context, future, predicted, refined;
    std::vector<int8_t> mask, future_mask;
};
using DecodeProgress = std::function<void(size_t offset, size_t patches, size_t context_length)>;
// loc/scale [B,V] of the first positive block's prediction (target rows only).
struct ForecastAnchors {
    size_t batch = 0, targets = 0;
    std::vector<float> loc, scale;
};
struct ForecastTrace {
    std::vector<DecodeBlock> positive, negative;
    // Called before each block's prediction. The device predicts the positive and the mirrored
    // pass of a block in one batch, so the observer is called for both passes of a block
    // before that batch runs (the reference runs every positive block, then every mirrored
    // one); the number of calls and their arguments are the reference's.
    DecodeProgress before_block;
    bool capture_initial_anchors = false;
    bool capture_blocks = true;
    std::optional<ForecastAnchors> initial_anchors;   // published only when the forecast succeeds
};
TS_API bool supports_known_covariates(const Config& c);
TS_API AssembledRows assemble_rows(const Config& c, const std::vector<float>& context, const std::vector<int8_t>& user_mask,
                            size_t B, size_t V, size_t T, size_t H, const std::vector<float>& past, size_t P,
                            const std::vector<float>& known, size_t K, size_t max_context,
                            const std::vector<double>& cat_past, size_t CP, const std::vector<double>& cat_known,
                            size_t CK);

class TS_API Forecaster {
public:
    // Uploads the model to `device` (-1: the current CUDA device). The Model must outlive
    // the Forecaster. Not reentrant; independent instances may run on independent threads.
    explicit Forecaster(const Model& model, int device = -1);
    ~Forecaster();
    Forecaster(const Forecaster&) = delete;
    Forecaster& operator=(const Forecaster&) = delete;

    // The reference's forecast (src/forecaster.cpp:87-108). With a trace, every decode block
    // is observed on the host (the stream synchronises per block, and the forecast is not
    // replayed from a CUDA graph); the quantiles are the same bits either way.
    Forecast forecast(const ForecastRequest& r, ForecastTrace* trace = nullptr);
    // Same result written to a caller buffer of B*V*H*Q floats.
    void forecast_into(const ForecastRequest& r, float* out, ForecastTrace* trace = nullptr);
    // The reference's packed decode (src/forecaster.cpp:15-67): assembled rows of one pass
    // decoded block by block with median feedback and refinement, no cap, symmetric average
    // or clip; returns [rows, horizon, Q]. max_context / per_shot 0: the model's.
    std::vector<float> decode(const AssembledRows& a, size_t horizon, size_t max_context = 0, size_t per_shot = 0,
                              std::vector<DecodeBlock>* trace = nullptr, const DecodeProgress& progress = {});
    // Requests without covariates from caller host buffers: context [B,V,T] (NaN = missing),
    // mask [B,V,T] bytes 0/1 or null; out [B,V,H,Q]. Flags already resolved.
    // out_pinned: `out` is page-locked host memory, so the forecast is downloaded into it
    // directly instead of through the staging buffer.
    void forecast_targets(const float* context, const uint8_t* mask, size_t B, size_t V, size_t T, size_t H,
                          bool symmetric, bool clip, size_t max_context, float* out, bool out_pinned = false);

    tsb::Engine& engine() { return *engine_; }
    // Covariate requests are assembled on the device (default) or, for comparison, on the
    // host (assemble_rows) and uploaded; both give identical forecasts.
    void set_device_assembly(bool on) { device_assembly_ = on; }
    bool device_assembly() const { return device_assembly_; }

private:
    void forecast_request(const ForecastRequest& r, float* out, bool symmetric, bool clip);
    const Model& model_;
    bool device_assembly_ = true;
    std::unique_ptr<tsb::Engine> engine_;
    struct Staging;
    std::unique_ptr<Staging> staging_;
};

}  // namespace ts
