#include "model.hpp"

#include <algorithm>
#include <cmath>
#include <cstring>
#include <regex>
#include <set>

namespace ts {

namespace {

constexpr int64_t kMaxRopePatches = int64_t(1) << 20;

[[noreturn]] void fail(const std::string& m) { throw Error(m); }

// Typed KV access: a missing key or a wrong type is a load error.
struct Kv {
    const GgufFile& g;
    const GgufValue& get(const char* key, GgufType want) const {
        auto it = g.kv().find(key);
        if (it == g.kv().end()) fail(std::string("missing KV: ") + key);
        if (it->second.type != want)
            fail(std::string("KV ") + key + " has type " + gguf_type_name(it->second.type) + ", expected " +
                 gguf_type_name(want));
        return it->second;
    }
    std::string str(const char* k) const { return get(k, GgufType::STRING).s; }
    uint32_t u32(const char* k) const { return uint32_t(get(k, GgufType::U32).u); }
    int32_t i32(const char* k) const { return int32_t(get(k, GgufType::I32).i); }
    float f32(const char* k) const { return float(get(k, GgufType::F32).f); }
    double f64(const char* k) const { return get(k, GgufType::F64).f; }
    bool boolean(const char* k) const { return get(k, GgufType::BOOL).u != 0; }
    std::vector<std::string> strs(const char* k) const {
        const auto& v = get(k, GgufType::ARRAY);
        if (v.array_type != GgufType::STRING) fail(std::string("KV ") + k + " is not an array of strings");
        return v.strings;
    }
    std::vector<double> f64s(const char* k) const {
        const auto& v = get(k, GgufType::ARRAY);
        if (v.array_type != GgufType::F64) fail(std::string("KV ") + k + " is not an array of float64");
        return v.numbers;
    }
};

LayerKind parse_kind(const std::string& s) {
    if (s == "time") return LayerKind::Time;
    if (s == "variate") return LayerKind::Variate;
    if (s == "time_variate") return LayerKind::TimeVariate;
    if (s == "variate_time") return LayerKind::VariateTime;
    fail("unknown layer kind '" + s + "'");
}

Gate parse_gate(const std::string& s) {
    if (s == "none") return Gate::None;
    if (s == "sdpa_sigmoid") return Gate::SdpaSigmoid;
    fail("unknown attention gate '" + s + "'");
}

TensorSpec spec(const std::string& n, int64_t a, int64_t b = -1) {
    TensorSpec s;
    s.name = n;
    s.ne[0] = a;
    if (b >= 0) { s.ne[1] = b; s.n_dims = 2; }
    return s;
}

}  // namespace

std::vector<bool> layer_axes(LayerKind k) {
    switch (k) {
        case LayerKind::Time: return {true};
        case LayerKind::Variate: return {false};
        case LayerKind::TimeVariate: return {true, false};
        case LayerKind::VariateTime: return {false, true};
    }
    return {};
}

Config read_config(const GgufFile& g) {
    Kv kv{g};
    Config c;
    const std::string arch = kv.str("general.architecture");
    if (arch != "timestral") fail("general.architecture is '" + arch + "', expected 'timestral'");
    c.name = kv.str("general.name");
    c.license = kv.str("general.license");
    c.license_name = kv.str("general.license.name");
    c.license_link = kv.str("general.license.link");
    c.source_url = kv.str("general.source.url");
    c.hf_revision = kv.str("timestral.source.hf_revision");
    c.code_sha = kv.str("timestral.source.code_sha");
    c.weights_sha256 = kv.str("timestral.source.weights_sha256");
    c.converter_version = kv.u32("timestral.converter_version");
    if (c.converter_version != 1)
        fail("converter_version " + std::to_string(c.converter_version) + " is not supported (expected 1)");
    c.patch_size = kv.u32("timestral.patch_size");
    c.d_model = kv.u32("timestral.embedding_length");
    c.num_heads = kv.u32("timestral.attention.head_count");
    c.mlp_hidden_dim = kv.u32("timestral.feed_forward_length");
    c.n_layers = kv.u32("timestral.block_count");
    c.block_schedule_names = kv.strs("timestral.block_schedule");
    for (const auto& s : c.block_schedule_names) c.block_schedule.push_back(parse_kind(s));
    c.quantile_knots = kv.f64s("timestral.quantile_knots");
    c.block_size = kv.u32("timestral.block_size");
    c.context_length = kv.u32("timestral.context_length");
    c.rope_theta = kv.f64("timestral.rope.freq_base");
    c.rope_partial_factor = kv.f64("timestral.rope.partial_factor");
    c.rope_dim = kv.u32("timestral.rope.dimension_count");
    c.rope_table_pos_min = kv.i32("timestral.rope.table_pos_min");
    c.norm_eps = kv.f32("timestral.attention.layer_norm_rms_epsilon");
    c.attn_bias = kv.boolean("timestral.attention.bias");
    c.mlp_bias = kv.boolean("timestral.mlp.bias");
    c.time_gate = parse_gate(kv.str("timestral.attention.time_gate"));
    c.variate_gate = parse_gate(kv.str("timestral.attention.variate_gate"));
    c.split_context_horizon = kv.boolean("timestral.attention.split_context_horizon");
    c.qkv_head_major = kv.boolean("timestral.attention.qkv_head_major");
    c.minimum_scale = kv.f64("timestral.scaler.minimum_scale");
    c.use_asinh = kv.boolean("timestral.scaler.use_asinh");
    c.stabilize_with_global = kv.boolean("timestral.scaler.stabilize_with_global");
    c.covariate_enabled = kv.boolean("timestral.covariate_enabled");
    c.attend_missing_patches = kv.boolean("timestral.attend_missing_patches");
    c.quantile_width_factor = kv.f64("timestral.quantile_width_factor");
    c.per_shot_horizon_patches = kv.u32("timestral.forecaster.per_shot_horizon_patches");
    c.quantile_real_cap_k = kv.f64("timestral.forecaster.quantile_real_cap_k");
    c.extreme_value_threshold = kv.f64("timestral.forecaster.extreme_value_threshold");
    c.symmetric_averaging = kv.boolean("timestral.forecaster.symmetric_averaging");
    c.clip_nonnegative = kv.boolean("timestral.forecaster.clip_nonnegative");
    c.target_encoding_smooth = kv.f64("timestral.target_encoding.smooth");

    if (!std::isfinite(c.target_encoding_smooth) || c.target_encoding_smooth <= 0)
        fail("target_encoding.smooth must be finite and positive");
    if (!c.qkv_head_major) fail("qkv_head_major is false: the file has torch row order, which this loader does not read");
    if (c.stabilize_with_global) fail("stabilize_with_global=true is not supported");
    if (!c.patch_size || !c.d_model || !c.num_heads || !c.mlp_hidden_dim || !c.block_size || !c.context_length)
        fail("a dimension is zero");
    if (c.d_model % c.num_heads) fail("d_model is not divisible by num_heads");
    if (c.n_layers != c.block_schedule.size()) fail("block_count does not match the length of block_schedule");
    if (!c.n_layers) fail("block_schedule is empty");
    if (!c.rope_dim || c.rope_dim % 2) fail("rope dimension_count must be positive and even");
    if (c.rope_partial_factor < 0.0 || c.rope_partial_factor > 1.0) fail("rope partial_factor out of range");
    if (c.rope_dim != uint32_t(int64_t(double(c.head_dim()) * c.rope_partial_factor)))
        fail("rope.dimension_count does not equal int(head_dim * partial_factor)");
    if (c.rope_dim > c.head_dim()) fail("rope dimension_count exceeds head_dim");
    if (c.quantile_knots.empty()) fail("quantile_knots is empty");
    if (std::find(c.quantile_knots.begin(), c.quantile_knots.end(), 0.5) == c.quantile_knots.end())
        fail("quantile_knots must contain 0.5");
    for (size_t i = 1; i < c.quantile_knots.size(); ++i)
        if (!(c.quantile_knots[i - 1] < c.quantile_knots[i])) fail("quantile_knots must be increasing");
    if (c.context_length % c.patch_size) fail("context_length is not a multiple of patch_size");
    const int64_t patches = int64_t(c.context_length / c.patch_size) + int64_t(c.block_size);
    if (patches > kMaxRopePatches)
        fail("context_length / patch_size + block_size = " + std::to_string(patches) +
             " exceeds the supported maximum of " + std::to_string(kMaxRopePatches) + " rope table positions per side");
    if (int64_t(c.rope_table_pos_min) != -patches)
        fail("rope.table_pos_min " + std::to_string(c.rope_table_pos_min) + " does not equal " + std::to_string(-patches));
    if (!(c.norm_eps > 0.f)) fail("norm eps must be positive");
    return c;
}

std::vector<TensorSpec> expected_schema(const Config& c) {
    const int64_t D = c.d_model, F = c.mlp_hidden_dim, ps = c.patch_size, Q = c.num_quantiles();
    const int64_t hd = c.head_dim(), P = c.rope_table_len();
    std::vector<TensorSpec> v;
    v.push_back(spec("patch.hidden.weight", 2 * ps, 4 * D));
    v.push_back(spec("patch.hidden.bias", 4 * D));
    v.push_back(spec("patch.out.weight", 4 * D, D));
    v.push_back(spec("patch.out.bias", D));
    v.push_back(spec("patch.res.weight", 2 * ps, D));
    v.push_back(spec("patch.res.bias", D));
    v.push_back(spec("patch.forecast_query", D));
    for (uint32_t i = 0; i < c.n_layers; ++i) {
        const std::string b = "blk." + std::to_string(i) + ".";
        const auto axes = layer_axes(c.block_schedule[i]);
        for (size_t j = 0; j < axes.size(); ++j) {
            const std::string a = b + "attn." + std::to_string(j) + ".";
            v.push_back(spec(b + "attn_norm." + std::to_string(j) + ".weight", D));
            v.push_back(spec(a + "qkv.weight", D, 3 * D));
            if (c.attn_bias) v.push_back(spec(a + "qkv.bias", 3 * D));
            if ((axes[j] ? c.time_gate : c.variate_gate) == Gate::SdpaSigmoid) {
                v.push_back(spec(a + "gate.weight", D, D));
                if (c.attn_bias) v.push_back(spec(a + "gate.bias", D));
            }
            v.push_back(spec(a + "out.weight", D, D));
            if (c.attn_bias) v.push_back(spec(a + "out.bias", D));
        }
        v.push_back(spec(b + "ffn_norm.weight", D));
        v.push_back(spec(b + "ffn_w12.weight", D, 2 * F));
        if (c.mlp_bias) v.push_back(spec(b + "ffn_w12.bias", 2 * F));
        v.push_back(spec(b + "ffn_w3.weight", F, D));
        if (c.mlp_bias) v.push_back(spec(b + "ffn_w3.bias", D));
    }
    v.push_back(spec("out_norm.weight", D));
    v.push_back(spec("head.hidden.weight", D, 4 * D));
    v.push_back(spec("head.out.weight", 4 * D, ps * Q));
    v.push_back(spec("head.res.weight", D, ps * Q));
    v.push_back(spec("rope.inv_freq", hd / 2));
    v.push_back(spec("rope.cos", hd, P));
    v.push_back(spec("rope.sin", hd, P));
    return v;
}

bool reduced_weight_name(const std::string& name) {
    static const std::regex block(R"(^blk\.[0-9]+\.(attn\.[0-9]+\.(qkv|gate|out)|ffn_w12|ffn_w3)\.weight$)");
    return name == "patch.out.weight" || name == "head.hidden.weight" || name == "head.out.weight" ||
           name == "head.res.weight" || std::regex_match(name, block);
}

bool weight_type_allowed(const std::string& name, uint32_t type, int64_t ne0) {
    if (ne0 <= 0) return false;
    if (type == 0) return true;
    const bool reduced = type == 1 || type == 8 || type == 12 || type == 13 || type == 14;
    const int64_t block = type == 1 ? 1 : type == 8 ? 32 : 256;
    return reduced && reduced_weight_name(name) && ne0 % block == 0;
}

Model::Model(Model&& o) noexcept { *this = std::move(o); }
Model& Model::operator=(Model&& o) noexcept {
    if (this != &o) {
        cfg_ = std::move(o.cfg_);
        file_ = std::move(o.file_);
        tensors_ = std::move(o.tensors_);
        names_ = std::move(o.names_);
        path_ = std::move(o.path_);
    }
    return *this;
}
Model::~Model() = default;

const TensorRef& Model::tensor(const std::string& name) const {
    auto it = tensors_.find(name);
    if (it == tensors_.end()) fail("tensor not found: " + name);
    return it->second;
}

size_t Model::mapped_bytes() const { return file_ ? file_->file().size() : 0; }

Model Model::load(const std::string& path) {
    Model m;
    m.path_ = path;
    m.file_ = std::make_unique<GgufFile>(path);
    const GgufFile& g = *m.file_;
    m.cfg_ = read_config(g);
    const Config& c = m.cfg_;
    // Schema: exactly the tensors the config implies, with the allowed types and shapes.
    const auto schema = expected_schema(c);
    std::set<std::string> want, have;
    for (const auto& s : schema) want.insert(s.name);
    std::map<std::string, const GgufTensorInfo*> infos;
    for (const auto& t : g.tensors()) {
        if (!have.insert(t.name).second) fail("duplicate tensor in file: " + t.name);
        if (!want.count(t.name)) fail("unexpected tensor in file (not in the schema of this config): " + t.name);
        infos[t.name] = &t;
    }
    for (const auto& s : schema) {
        auto it = infos.find(s.name);
        if (it == infos.end()) fail("missing tensor: " + s.name);
        const GgufTensorInfo& t = *it->second;
        if (!weight_type_allowed(s.name, t.type, t.ne[0]))
            fail("tensor " + s.name + " has type " + ggml_type_name(t.type) + ", forbidden by the storage policy");
        for (int d = 0; d < 4; ++d)
            if (t.ne[d] != s.ne[d])
                fail("tensor " + s.name + " has shape [" + std::to_string(t.ne[0]) + ", " + std::to_string(t.ne[1]) +
                     ", " + std::to_string(t.ne[2]) + ", " + std::to_string(t.ne[3]) + "], expected [" +
                     std::to_string(s.ne[0]) + ", " + std::to_string(s.ne[1]) + ", " + std::to_string(s.ne[2]) + ", " +
                     std::to_string(s.ne[3]) + "]");
    }
    // Place every tensor in the mapping, with bounds and alignment checked against the file.
    const size_t fsize = g.file().size();
    for (const auto& t : g.tensors()) {
        TensorRef r;
        r.type = t.type;
        std::copy(t.ne, t.ne + 4, r.ne);
        const size_t row = ggml_row_bytes(t.type, t.ne[0]);
        if (!row) fail("tensor " + t.name + " has type " + ggml_type_name(t.type) + ", which the B200 path does not read");
        r.bytes = row * size_t(t.ne[1]) * size_t(t.ne[2]) * size_t(t.ne[3]);
        const size_t off = g.data_offset() + size_t(t.offset);
        if (off > fsize || r.bytes > fsize - off) fail("tensor data out of file bounds: " + t.name);
        if (t.offset % g.alignment()) fail("tensor data not aligned: " + t.name);
        r.data = g.file().data() + off;
        m.tensors_[t.name] = r;
        m.names_.push_back(t.name);
    }
    // rope.inv_freq: recompute and warn on a difference; the stored table is used.
    const float* stored = static_cast<const float*>(m.tensor("rope.inv_freq").data);
    int diff = 0;
    for (uint32_t i = 0; i < c.head_dim() / 2; ++i) {
        float want_v = 0.f;
        if (i < c.rope_dim / 2) want_v = 1.0f / std::pow(float(c.rope_theta), float(2 * i) / float(c.rope_dim));
        if (std::memcmp(&want_v, &stored[i], 4) != 0) ++diff;
    }
    if (diff) TS_LOG("warning: rope.inv_freq differs from the recomputed table in %d entries; the stored table is used", diff);
    return m;
}

}  // namespace ts
