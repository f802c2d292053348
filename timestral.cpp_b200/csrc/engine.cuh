// Device engine: one model resident on one GPU and the forecast pipeline that replaces the
// reference's per-block ggml graphs (reference src/predict_block.cpp:6-56 via
// src/backend.cpp GraphRunner) and its host decode loop (src/forecaster.cpp:19-108).
#pragma once
#include <cstdint>
#include <functional>
#include <map>
#include <memory>
#include <string>
#include <vector>

#include <cuda_runtime.h>

namespace tsb {

enum TensorType : int { TT_F32 = 0, TT_F16 = 1, TT_Q8_0 = 8, TT_Q4_K = 12, TT_Q5_K = 13, TT_Q6_K = 14 };

struct HostTensor {
    int type = TT_F32;
    int64_t ne0 = 0, ne1 = 1;   // ne0 = contiguous (input) dimension
    const void* data = nullptr;
};

// Everything the device needs from a loaded model (config KVs + tensors by GGUF name).
struct ModelView {
    int ps = 0, D = 0, H = 0, F = 0;
    std::vector<int> schedule;        // 0 time, 1 variate, 2 time_variate, 3 variate_time
    std::vector<double> knots;
    int median = 0;
    int block_size = 0, context_length = 0;
    int rope_dim = 0, pos_min = 0;
    float eps = 0;
    bool attn_bias = false, mlp_bias = false, time_gate = false, variate_gate = false;
    double minimum_scale = 0;
    bool use_asinh = false, covariate_enabled = false, attend_missing = false;
    double width_factor = 0;
    int per_shot = 0;
    double cap_k = 0, extreme = 0;
    bool symmetric = false, clip = false;
    std::function<HostTensor(const std::string&)> tensor;
    std::function<bool(const std::string&)> has;
};

// Rows prepared on the host (covariate requests), reference AssembledRows
// (src/covariates.hpp:12-17).
struct HostRows {
    int R = 0, T = 0, Hh = 0;                 // rows, context length, padded horizon
    const float* rows = nullptr;              // [R][T]
    const int8_t* mask = nullptr;             // [R][T]
    const int64_t* roles = nullptr;           // [R] or null
    const float* future = nullptr;            // [R][Hh] or null
    const int8_t* future_mask = nullptr;
    int group_rows = 1;                       // rows per series (contiguous)
    int cap = 0;                              // context cap of the decode slide (0: the model's)
};

// A covariate request as the caller holds it (reference ForecastRequest fields), assembled
// on the device: context [B][V][T] (+ optional 0/1 mask), past [B][P][T], known [B][K][T+H],
// categorical past [B][CP][T] and known [B][CK][T+H] f64 codes (validated by the caller:
// finite or NaN). kept/len/hor: kept context steps, padded row length, padded horizon.
struct CovRequest {
    int B = 0, V = 0, T = 0, H = 0, P = 0, K = 0, CP = 0, CK = 0;
    const float* ctx = nullptr;
    const uint8_t* umask = nullptr;
    const float* past = nullptr;
    const float* known = nullptr;
    const double* cat_past = nullptr;
    const double* cat_known = nullptr;
    int kept = 0, len = 0, hor = 0;
    double smooth = 0;
    int cap = 0;                              // context cap of the decode slide (0: the model's)
};

// One decode block as the device holds it right after its prediction and refinement, for
// callers that trace a forecast (reference ForecastTrace / DecodeBlock,
// src/forecaster.hpp:24-38). Device pointers, valid until the next block starts; rows are
// both symmetric passes when the forecast is mirrored (positive pass first).
struct BlockView {
    int offset = 0, patches = 0, length = 0;     // first step, patches, context steps of the block
    int rows = 0;
    const float* context = nullptr;              // [rows][context_stride], first `length` steps used
    const int8_t* mask = nullptr;                // same layout
    int64_t context_stride = 0;
    const float* future = nullptr;               // [rows][future_stride] from the block's first step, or null
    const int8_t* future_mask = nullptr;
    int64_t future_stride = 0;
    const float* predicted = nullptr;            // [rows][patches * patch_size][Q] before refinement
    const float* refined = nullptr;              // [rows][patches * patch_size][Q]
    const float* loc = nullptr;                  // [rows] frame of the block's last context step
    const float* scale = nullptr;
};
struct BlockObserver {
    // Called before each block's prediction with (first step, patches, context steps).
    std::function<void(int, int, int)> before;
    // Called after each block's refinement, with the engine stream synchronised.
    std::function<void(const BlockView&)> after;
};

class Engine {
public:
    Engine(const ModelView& mv, int device);
    ~Engine();
    Engine(const Engine&) = delete;
    Engine& operator=(const Engine&) = delete;

    int device() const { return device_; }
    cudaStream_t stream() const { return stream_; }
    bool tensor_cores() const { return tc_; }

    // Requests without covariates, context and output in device memory.
    // Throws std::runtime_error (message) on invalid input or device failure.
    void forecast_targets(const float* d_ctx, const uint8_t* d_umask, int B, int V, int T, int H, bool symmetric,
                          bool clip, int max_context, float* d_out, bool sync);
    // Requests with covariates: rows assembled on the host (one pass; the mirrored pass is
    // formed on the device). ctx/umask: the original request context (clip eligibility).
    void forecast_rows(const HostRows& a, int B, int V, int H, bool symmetric, bool clip, const float* ctx,
                       const uint8_t* umask, int T_req, float* h_out);
    // Requests with covariates assembled on the device (host buffers in and out).
    void forecast_covariates(const CovRequest& q, bool symmetric, bool clip, float* h_out);
    // Decode of assembled rows of one pass (reference Forecaster::decode): every block with
    // median feedback and refinement, no cap, symmetric average or clip; h_decoded [R][H][Q].
    void decode_host_rows(const HostRows& a, int H, float* h_decoded);

    // CUDA-graph replay of single-block forecasts without covariates (on by default): the
    // second call with the same shapes, flags and device buffers is captured into a graph,
    // later identical calls launch the graph.
    void graph_replay(bool on);
    // RMSNorm carried by the tensor-core GEMMs (default, mode 1): the residual-add epilogues
    // leave an f16 copy of the residual and its row sums of squares for the next GEMM, which
    // applies 1/rms itself; a forecast that meets a row outside the f16 copy's range runs
    // again with the RMSNorm kernel. Mode 0: always the RMSNorm kernel. Mode 2: carried, and
    // every forecast also takes the fallback run (a test of that path).
    void fused_norm(int mode);
    // Attention kernels of the tensor-core path: 0 (default) the tensor-core kernels; 1 the
    // CUDA-core kernels with the reference's operation order (float64 q.k dots, f32 softmax
    // and value sums) on the same f16 q/k/v, for time rows of up to kSimtMaxKeys tokens and
    // the variate axis. Mode 1 isolates the tensor-core attention's share of the deviation
    // from the reference's f32 attention.
    void attention_kernels(int mode);
    // Decoder-token tail (on by default): when the last layer starts with a time sublayer and
    // the rest of it is per token, its out projection, one-row variate sublayer and MLP run on
    // the decoder tokens alone, the only tokens the head reads. Off: every token, same bits.
    void decoder_tail(bool on);
    // Block-quantised weights (Q8_0, Q4_K, Q5_K, Q6_K) dequantised in the GEMM prologue (on)
    // instead of read as the f16 copies made at load (off, the default): the int8 tiles and
    // their block scales (and offsets) travel to shared memory and converter warps write the
    // f16 tiles the tensor cores read; the same f16 values, so the same forecast bits. Weights
    // whose norm gain is folded into them keep the f16 copy unless the gain is 1. Returns
    // false when the model has no block-quantised weights (and `on` was asked).
    bool dequant_prologue(bool on);
    // Observe every decode block of the following forecasts (nullptr: none). While an
    // observer is set, forecasts are not captured into or replayed from CUDA graphs.
    void set_observer(const BlockObserver* observer);
    // Per-request overrides (reference ForecastRequest::per_shot_horizon_patches and
    // quantile_real_cap_k): patches per decode block (0: the model's) and the cap factor
    // (negative: the model's; 0 disables the cap).
    void set_overrides(int per_shot, double cap_k);

    // Synchronise the stream and turn a device error word into an exception.
    void check_errors();

    // Per-kernel-class timing (CUDA events on the engine stream).
    // `only`: time launches of that class alone (nullptr: every class).
    void timing_enable(bool on, const char* only = nullptr);
    void timing_reset();
    bool timing_read(const std::string& cls, double* ms, int64_t* launches);
    int64_t last_launches() const { return last_launches_; }
    // Geometry of the last decode block of the last forecast: rows (both passes, every row
    // role), tokens per row S, context patches L, decode blocks.
    struct Geometry { int64_t rows = 0; int S = 0, L = 0, blocks = 0; };
    Geometry last_geometry() const;

private:
    void finish_targets();
    void targets_body(const float* d_ctx, const uint8_t* d_umask, int B, int V, int T, int H, bool symmetric, bool clip,
                      float* d_out, int kept, int len, int patches, int shot, int R, int R2, int cap);
    // The decode blocks of an assembled covariate request (rows, masks, roles, futures in
    // device memory) through the final download.
    void decode_rows(int B, int V, int H, int R, int T, int Hh, bool symmetric, bool clip, bool cov, bool has_future,
                     int group_rows, int cap, float* h_out, float* h_decoded);
    struct Impl;
    std::unique_ptr<Impl> impl_;
    int device_ = 0;
    bool tc_ = false;
    cudaStream_t stream_ = nullptr;
    int64_t last_launches_ = 0;
};

// Test hook: the next n workspace allocations (any engine of the process) fail with
// cudaErrorMemoryAllocation; 0 clears it.
void inject_workspace_failures(int n);

}  // namespace tsb
