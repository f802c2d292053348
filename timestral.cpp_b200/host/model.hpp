// ts::Config and ts::Model: the reference's model surface (reference src/config.hpp:25-71,
// src/model_loader.hpp:33-65), loading a GGUF into a read-only mapping with the same
// KV/schema/storage-policy checks. The weights are uploaded to the GPU by ts::Forecaster.
#pragma once
#include "common.hpp"
#include "gguf.hpp"

#include <cstdint>
#include <map>
#include <memory>
#include <string>
#include <vector>

namespace ts {

enum class LayerKind { Time, Variate, TimeVariate, VariateTime };
enum class Gate { None, SdpaSigmoid };

// Ordered attention axes of a layer kind; true = time axis.
std::vector<bool> layer_axes(LayerKind k);

struct Config {
    std::string name, license, license_name, license_link, source_url;
    std::string hf_revision, code_sha, weights_sha256;
    uint32_t converter_version = 0;
    uint32_t patch_size = 0, d_model = 0, num_heads = 0, mlp_hidden_dim = 0, n_layers = 0;
    std::vector<std::string> block_schedule_names;
    std::vector<LayerKind> block_schedule;
    std::vector<double> quantile_knots;
    uint32_t block_size = 0, context_length = 0;
    double rope_theta = 0, rope_partial_factor = 0;
    uint32_t rope_dim = 0;
    int32_t rope_table_pos_min = 0;
    float norm_eps = 0;
    bool attn_bias = false, mlp_bias = false;
    Gate time_gate = Gate::None, variate_gate = Gate::None;
    bool split_context_horizon = false, qkv_head_major = false;
    double minimum_scale = 0;
    bool use_asinh = false, stabilize_with_global = false;
    bool covariate_enabled = false, attend_missing_patches = false;
    double quantile_width_factor = 0;
    uint32_t per_shot_horizon_patches = 0;
    double quantile_real_cap_k = 0, extreme_value_threshold = 0;
    bool symmetric_averaging = false, clip_nonnegative = false;
    double target_encoding_smooth = 0;

    uint32_t head_dim() const { return d_model / num_heads; }
    uint32_t num_quantiles() const { return uint32_t(quantile_knots.size()); }
    uint32_t median_index() const {
        for (size_t i = 0; i < quantile_knots.size(); ++i) if (quantile_knots[i] == 0.5) return uint32_t(i);
        return 0;
    }
    int64_t rope_table_len() const { return 2 * (-int64_t(rope_table_pos_min)) + 1; }
};

struct TensorSpec {
    std::string name;
    int64_t ne[4] = {1, 1, 1, 1};
    int n_dims = 1;
};

// The config of a parsed GGUF (reference src/model_loader.cpp:72-160). Throws ts::Error.
TS_API Config read_config(const GgufFile& g);
// The tensors a file with this config must contain, in file order
// (reference src/model_loader.cpp:166-207).
TS_API std::vector<TensorSpec> expected_schema(const Config& c);
// Storage policy (reference src/weight_policy.hpp:8-22): F32 everywhere, F16/Q8_0/K-quants
// only on the projection weights of the allowlist.
bool reduced_weight_name(const std::string& name);
bool weight_type_allowed(const std::string& name, uint32_t type, int64_t ne0);

struct TensorRef {
    uint32_t type = 0;
    int64_t ne[4] = {1, 1, 1, 1};
    const void* data = nullptr;
    size_t bytes = 0;
};

class TS_API Model {
public:
    // Load `path`; weights stay in the read-only mapping. Throws ts::Error.
    static Model load(const std::string& path);
    Model(Model&&) noexcept;
    Model& operator=(Model&&) noexcept;
    Model(const Model&) = delete;
    Model& operator=(const Model&) = delete;
    ~Model();

    const Config& config() const { return cfg_; }
    bool has(const std::string& name) const { return tensors_.count(name) != 0; }
    const TensorRef& tensor(const std::string& name) const;   // throws ts::Error when absent
    const std::vector<std::string>& tensor_names() const { return names_; }
    size_t mapped_bytes() const;
    const std::string& path() const { return path_; }

private:
    Model() = default;
    Config cfg_;
    std::unique_ptr<GgufFile> file_;
    std::map<std::string, TensorRef> tensors_;
    std::vector<std::string> names_;
    std::string path_;
};

}  // namespace ts
