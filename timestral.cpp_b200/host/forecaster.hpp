// ts::Forecaster: the reference's forecast entry (reference src/forecaster.hpp:9-56) on a
// B200. Requests without covariates run end to end on the GPU (row assembly included);
// requests with covariates are assembled on the host (categorical target encoding in
// float64) and predicted on the GPU.
#pragma once
#include "model.hpp"

#include <cstdint>
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
bool supports_known_covariates(const Config& c);
AssembledRows assemble_rows(const Config& c, const std::vector<float>& context, const std::vector<int8_t>& user_mask,
                            size_t B, size_t V, size_t T, size_t H, const std::vector<float>& past, size_t P,
                            const std::vector<float>& known, size_t K, size_t max_context,
                            const std::vector<double>& cat_past, size_t CP, const std::vector<double>& cat_known,
                            size_t CK);

class Forecaster {
public:
    // Uploads the model to `device` (-1: the current CUDA device). The Model must outlive
    // the Forecaster. Not reentrant; independent instances may run on independent threads.
    explicit Forecaster(const Model& model, int device = -1);
    ~Forecaster();
    Forecaster(const Forecaster&) = delete;
    Forecaster& operator=(const Forecaster&) = delete;

    Forecast forecast(const ForecastRequest& r);
    // Same result written to a caller buffer of B*V*H*Q floats.
    void forecast_into(const ForecastRequest& r, float* out);
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
    const Model& model_;
    bool device_assembly_ = true;
    std::unique_ptr<tsb::Engine> engine_;
    struct Staging;
    std::unique_ptr<Staging> staging_;
};

}  // namespace ts
