// Per-row and per-token kernels of the forecast path (scaler, masks metadata, norms,
// quantile head, refine, final combine) and the CUDA-core GEMM of the F32 path.
#pragma once
#include <cstdint>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

namespace tsb {

struct RowConfig {
    int ps = 0;                 // patch size
    double minimum_scale = 0;
    int use_asinh = 0;
    int attend_missing = 0;
    int Q = 0, median = 0;      // quantiles, median index
    float widths[64];           // monotone widths (float(width_factor) * float(knot gap))
    int pos_min = 0, rope_len = 0;
    double cap_k = 0;
    double extreme = 0;
};

// --- assembly of context-only requests (reference src/covariates.cpp:32-72, V rows only):
// forward fill, observed mask, cap to the last `kept` steps, left pad to `len`; the mirrored
// pass rows (if any) are the exact negation. ctx [BV][T]; umask [BV][T] or null.
cudaError_t assemble_targets(const float* ctx, const uint8_t* umask, int BV, int T, int kept, int len, int mirrored,
                             float* rows, int8_t* mask, cudaStream_t s);

// --- covariate requests assembled on the device (reference src/covariates.cpp:32-72):
// per series b the rows b * all + j are its V targets (forward filled), P past, CP
// categorical past, K known and CK categorical known covariates (codes cast to float, or
// smoothed-mean target encoded when V == 1), the kept context left-padded to len, roles, the
// known rows' future steps padded to hor, and the negated mirrored pass at rows R..2R-1.
struct CovShape {
    int B = 0, V = 0, P = 0, CP = 0, K = 0, CK = 0;
    int T = 0, H = 0;               // request context length and horizon
    int kept = 0, len = 0, hor = 0; // kept context steps, padded row length, padded horizon
    int mirrored = 0;
    double smooth = 0;              // target-encoding smoothing
};
size_t covariate_scratch_bytes(const CovShape& c);
// ctx/umask [B][V][T] (umask may be null); past [B][P][T]; known [B][K][T+H]; cat_past
// [B][CP][T] and cat_known [B][CK][T+H] f64 codes (finite or NaN); rows/mask [R2][len],
// role [R2], future/fmask [R2][hor]; first_obs [B * V] scratch; scratch of
// covariate_scratch_bytes(c) bytes (null when that is 0).
cudaError_t assemble_covariates(const CovShape& c, const float* ctx, const uint8_t* umask, const float* past,
                                const float* known, const double* cat_past, const double* cat_known, float* rows,
                                int8_t* mask, int8_t* role, float* future, int8_t* fmask, int* first_obs, void* scratch,
                                cudaStream_t s);

// --- causal scaler + patch features (reference src/scaler.cpp:27-58, src/encoder.cpp:12-23).
// rows/mask [R][W]; features [R][W/ps][2ps] f32; anchor frame of step `anchor_step`;
// key-valid bits [R][kv_words]; first observed patch per row (-1 if none) among the first
// `enc_patches` patches; optional cap statistics over the first `ctx_len` steps.
cudaError_t scale_rows(const RowConfig& c, const float* rows, const int8_t* mask, int R, int W, int anchor_step,
                       int enc_patches, int kv_words, float* features, float* loc, float* scale, uint32_t* key_valid,
                       int* first_obs, int ctx_len, float* cap_lo, float* cap_hi, float* cap_scale, cudaStream_t s,
                       int kernel = -1);
// kernel: -1 the block-per-row form when the patch size allows it, 0 one thread per row,
// 1 one block per row (identical results).

// --- instance-norm statistics of known covariate rows, overwriting their features and
// anchors (reference src/scaler.cpp:60-107).
cudaError_t known_rows(const RowConfig& c, const float* rows, const int8_t* mask, const int8_t* role, int R, int W,
                       int anchor_step, float* features, float* loc, float* scale, cudaStream_t s);

// --- positions -> rope table rows, and series group ranges (reference src/masks.cpp:13-18).
// Groups are contiguous runs of `group_rows` rows.
cudaError_t positions(const RowConfig& c, const int* first_obs, int R, int group_rows, int N, int S, int cov,
                      int* rope_row, int* group_begin, int* group_size, int* err, cudaStream_t s);

// --- token embedding of the decoder tokens: x[r][p] = query for p in [first, S).
cudaError_t fill_query(const float* query, float* x, int R, int S, int first, int D, cudaStream_t s);

// --- RMSNorm with the reference's float sum cascade (reference src/layers.cpp:257-287).
// out[i] = norm(x[tok(i)]) with tok(i) = (i / sub) * S + off + i % sub (sub = 0: identity).
cudaError_t rms_norm(const float* x, const float* w, int tokens, int D, float eps, void* out, int out_f16, int sub,
                     int S, int off, cudaStream_t s);

// --- F32-path element kernels.
// fused [M][3D] (+ gate [M][D]) -> head-major q,k (RoPE), v, sigmoid(gate) [rows][H][S][hd].
cudaError_t qkv_scatter(const float* fused, const float* gate, int M, int S, int H, int hd, int rope,
                        const float* cos_tab, const float* sin_tab, const int* rope_row, float* q, float* k, float* v,
                        float* g, cudaStream_t s);
// z [M][2F] -> h [M][F] = z[:F] * silu(z[F:])
cudaError_t swiglu(const float* z, int M, int F, float* h, cudaStream_t s);
// x[M][D] += y  (f32, order x + y)
cudaError_t add_inplace(float* x, const float* y, int64_t n, cudaStream_t s);

// --- quantile head tail: monotone quantiles, denormalisation, clamp (reference
// src/head.cpp:61-80, src/scaler.cpp:109-137). raw [R*P_all][ps*Q] f32 for P_all decoder
// tokens per row, of which patches [p0, p0+h) are kept. out/normalized [R][h*ps][Q].
cudaError_t quantile_head(const RowConfig& c, const float* raw, int R, int P_all, int p0, int h, const float* loc,
                          const float* scale, float* out, float* normalized, int* err, cudaStream_t s);

// --- refine (reference src/refine.cpp:32-106), h > 1 patches; scratch: [R][T/ps + h] x 3 doubles.
// rows/mask: context rows with row stride `stride` (>= T).
cudaError_t refine(const RowConfig& c, const float* q, const float* rows, const int8_t* mask, int stride, const int8_t* role,
                   const float* loc0, const float* scale0, int R, int T, int h, double clip, double* scratch,
                   float* out, cudaStream_t s);

// --- final combine (reference src/forecaster.cpp:68-86 cap, :95-104 symmetric + clip).
// decoded [R2][H][Q] where rows [0,Rp) are the positive pass and [Rp,2Rp) the mirrored pass
// (if mirrored). Target row of (b,v) = b*all + v. clip_src: original context [BV][T] + mask.
cudaError_t finalize(const RowConfig& c, const float* decoded, int Rp, int mirrored, int B, int V, int all, int H,
                     int Hfull, const float* cap_lo, const float* cap_hi, const float* cap_scale, int cap_on,
                     const int8_t* clip_ok, float* out, int* err, cudaStream_t s);
// Rows whose observed request context is all >= 0 with at least one observation.
cudaError_t clip_eligibility(const float* ctx, const uint8_t* umask, int BV, int T, int8_t* ok, cudaStream_t s);

// --- next decode block context (reference src/forecaster.cpp:52-64).
cudaError_t feedback(const RowConfig& c, const float* rows, const int8_t* mask, int R, int T, const float* q, int n,
                     const int8_t* role, const float* future, const int8_t* fmask, int keep, float* next_rows,
                     int8_t* next_mask, cudaStream_t s);

// --- CUDA-core GEMM: y[M][N] = A[M][K] . W[N][K]^T with the reference's F32 orders.
enum SimtOrder : int { ORDER_PANEL192 = 0, ORDER_CHAIN = 1, ORDER_F64 = 2 };
enum SimtEpi : int { SEPI_F32 = 0, SEPI_F16 = 1, SEPI_RESID = 2, SEPI_SILU_F32 = 3, SEPI_SILU_F16 = 4 };
struct SimtGemm {
    const float* A = nullptr; int64_t lda = 0;
    const float* W = nullptr;           // [N][K] f32 (F16/Q8_0 weights are expanded to f32 exactly)
    int M = 0, N = 0, K = 0;
    int round_a_f16 = 0;                // activations rounded to f16 first (F16-weight semantics)
    int order = ORDER_PANEL192;
    int epi = SEPI_F32;
    const float* bias = nullptr;
    void* out = nullptr; int64_t ldo = 0;
    int row_group = 0, row_stride = 0, row_offset = 0;  // output row remap (as in GemmEpilogue)
    const int* only_if = nullptr;       // when set, the launch does nothing unless *only_if != 0
    const int8_t* row_mask = nullptr;   // when set, only rows m with row_mask[m] != 0 are written
    // ORDER_PANEL192 with few rows: the 192-wide K panels run as separate blocks into this
    // scratch ([panels][M][N] f32) and are summed in order by a second kernel (same result).
    float* panel_scratch = nullptr;
    size_t panel_scratch_bytes = 0;
    // ORDER_PANEL192 launches of at least 64 rows without only_if / row_mask, K % 16 == 0 and
    // 16-byte aligned rows run a larger-tile kernel (same bits); 0 keeps the 64 x 64 kernel.
    int tiled = 1;
};
// Bytes of panel scratch that simt_gemm uses for `g` (0: one pass, no scratch).
size_t simt_panel_scratch_bytes(const SimtGemm& g);
cudaError_t simt_gemm(const SimtGemm& g, cudaStream_t s);

// Two-term f16 split of an f32 matrix for tensor-core products at near-f32 accuracy:
// out[m] = [hi(a[m]) | hi(a[m]) | lo(a[m])] (3K f16 per row), hi = f16(a), lo = f16(a - hi).
// With weights split as [hi(w) | lo(w) | hi(w)], a K = 3K f16 product sums
// hi*hi + hi*lo + lo*hi (relative error ~2^-22). Any |a| > 30000 (outside the range where
// the split is exact enough in f16) sets *overflow and, when given, row_overflow[row].
cudaError_t split_f16(const float* a, int64_t rows, int K, __half* out, int* overflow, int8_t* row_overflow,
                      cudaStream_t s);

// Read a device error word and reset it.
int read_error(int* d_err, cudaStream_t s);

}  // namespace tsb
