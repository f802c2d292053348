/* CPU oracle for the Timestral forecast hot path — TEST INFRASTRUCTURE ONLY.
 *
 * A C++17 restatement of the reference CPU path (mudler/timestral.cpp) that the
 * parity tests, __graft_entry__.smoke() and bench.py's cpu_baseline leg use as the
 * checker. The product library never links or calls it.
 *
 * F32 weights follow the reference's own F32 callbacks operation by operation
 * (src/layers.cpp, src/head.cpp, src/scaler.cpp, ...). F16 and Q8_0 weights follow
 * ggml's CPU mul_mat semantics (activations rounded to F16, or quantised to Q8_0 per
 * 32-block) as documented by the reference (docs/quantization.md:86,101); ggml is not
 * vendored in the reference, so the F16/Q8_0 accumulation order is not pinned.
 */
#ifndef TSB200_ORACLE_H
#define TSB200_ORACLE_H
#include <stdint.h>
#ifdef __cplusplus
extern "C" {
#endif

enum { ORACLE_F32 = 0, ORACLE_F16 = 1, ORACLE_Q8_0 = 8 };

typedef struct oracle_config {
    int32_t patch_size, d_model, num_heads, mlp_hidden_dim, n_layers;
    int32_t schedule[256];          /* 0 time, 1 variate, 2 time_variate, 3 variate_time */
    int32_t num_quantiles;
    double knots[64];
    int32_t block_size, context_length;
    int32_t rope_dim, rope_table_pos_min;
    float norm_eps;
    int32_t attn_bias, mlp_bias, time_gate, variate_gate; /* gate: 1 = sdpa_sigmoid */
    double minimum_scale;
    int32_t use_asinh, covariate_enabled, attend_missing_patches;
    double quantile_width_factor;
    int32_t per_shot_horizon_patches;
    double quantile_real_cap_k, extreme_value_threshold;
    int32_t symmetric_averaging, clip_nonnegative;
    double target_encoding_smooth;
} oracle_config;

typedef struct oracle_model oracle_model;

oracle_model* oracle_model_new(const oracle_config* cfg);
void oracle_model_free(oracle_model* m);
/* Register one tensor by GGUF name. data is copied. type: ORACLE_F32/F16/Q8_0;
   ne0 = contiguous (input) dimension, ne1 = rows. */
int oracle_model_set(oracle_model* m, const char* name, const void* data, int32_t type,
                     int64_t ne0, int64_t ne1);
const char* oracle_last_error(void);
/* Test override of the request's per_shot_horizon_patches (0 = model default). */
void oracle_model_set_per_shot(oracle_model* m, int32_t n);
/* Test knob: round q/k/v (after RoPE) and sigmoid(gate) to f16 before attention, as the
 * device's tensor-core path stores them, to separate that rounding from other deviations. */
void oracle_model_set_round_attention(oracle_model* m, int32_t on);

/* Same fields and meaning as timestral_forecast_request (include/timestral_capi.h). */
typedef struct oracle_request {
    const float* context; const uint8_t* observation_mask;
    int32_t B, V, T, prediction_length;
    const float* past_cov; int32_t c_past;
    const float* known_cov; int32_t c_known;
    const double* cat_past; int32_t cc_past;
    const double* cat_known; int32_t cc_known;
    int32_t symmetric_averaging, clip_nonnegative, max_context;
} oracle_request;

/* Full forecast (reference src/forecaster.cpp:87-108). out: [B,V,H,Q]. 0 on success. */
int oracle_forecast(oracle_model* m, const oracle_request* r, float* out, int32_t threads);

/* One block prediction on prepared rows (reference src/predict_block.cpp:26-56).
   out/normalized: [R, h*ps, Q]; loc/scale: [R]. roles/future may be NULL. */
int oracle_predict_block(oracle_model* m, const float* rows, const int8_t* observed, int64_t R,
                         int64_t T, int64_t h, const int64_t* groups, const int64_t* roles,
                         const float* future, const int8_t* future_mask, float* out,
                         float* normalized, float* loc, float* scale, int32_t threads);

/* ---- component entry points, for the known-answer tests ---- */
int oracle_scale_rows(const oracle_config* c, const float* x, const int8_t* mask, int64_t rows,
                      int64_t length, float* scaled, float* loc, float* scale);
int oracle_instance_norm_stats(const oracle_config* c, const float* x, const int8_t* mask,
                               int64_t rows, int64_t length, float* loc, float* scale,
                               int8_t* is_binary);
/* Outputs sized by the caller from oracle_mask_sizes. */
int oracle_mask_sizes(const oracle_config* c, int64_t R, int64_t T, int64_t h, int32_t cov,
                      int64_t* N, int64_t* S, int64_t* L);
int oracle_build_masks(const oracle_config* c, const int8_t* observed, int64_t R, int64_t T,
                       int64_t h, const int64_t* groups, const int64_t* roles, int8_t* obs,
                       int8_t* key_valid, int64_t* first_group, int64_t* positions,
                       int8_t* time_allowed, int8_t* variate, int8_t* active, int64_t* anchor);
int oracle_sdpa(const float* q, const float* k, const float* v, const float* mask, int64_t hd,
                int64_t H, int64_t S, int64_t R, int64_t split, float* out, int32_t threads);
int oracle_rms_norm(const float* x, const float* w, int64_t rows, int64_t D, float eps, float* out);
int oracle_linear_f32(const float* w, const float* x, const float* b, int64_t K, int64_t N,
                      int64_t rows, float* y);
int oracle_monotone_quantiles(const oracle_config* c, const float* raw, int64_t n, float* out);
int oracle_denormalize(const float* x, const float* loc, const float* scale, int64_t rows,
                       int64_t stride, int64_t Q, int32_t use_asinh, float* out);
int oracle_refine_block(const oracle_config* c, const float* q, const float* x, const int8_t* mask,
                        int64_t rows, int64_t length, int64_t patches, const int8_t* targets,
                        float* out);
int oracle_block_frames(const oracle_config* c, const float* x, const int8_t* mask,
                        const double* median, int64_t rows, int64_t length, int64_t patches,
                        double* loc, double* scale);
int oracle_head_linear_f64(const float* w, const float* x, int64_t K, int64_t N, int64_t rows, float* y);
int oracle_sigmoid(const float* x, int64_t n, float* out);
/* Row assembly (reference src/covariates.cpp:32-72); outputs sized by the caller. */
int oracle_assemble_rows(const oracle_config* c, const oracle_request* r, int64_t* R, int64_t* len, int64_t* hor,
                         float* rows, int8_t* mask, int64_t* groups, int64_t* roles, float* future, int8_t* future_mask);
float oracle_activation_exp(float x);
float oracle_attention_exp(float x);
double oracle_numpy_sum(const double* x, int64_t n);
float oracle_torch_sum_f32(const float* x, int64_t n);

#ifdef __cplusplus
}
#endif
#endif
