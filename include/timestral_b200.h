/* timestral-b200: device seam of the B200 forecast path.
 *
 * The public surface of the reference stays in timestral_capi.h (unchanged). This header
 * is the thin internal C ABI that replaces the reference's ggml graph runtime
 * (GraphRunner, reference src/backend.hpp:40-75) and the graph bodies built by
 * PredictBlock::predict (reference src/predict_block.cpp:6-56): plain pointers and sizes,
 * integer status codes, a per-handle error string, no C++ or torch types.
 *
 * Handles are not reentrant; one handle per device per host thread. Calls are synchronous
 * unless stated otherwise (work is stream-ordered inside).
 */
#ifndef TIMESTRAL_B200_H
#define TIMESTRAL_B200_H
#include <stddef.h>
#include <stdint.h>
#include "timestral_capi.h"
#ifdef __cplusplus
extern "C" {
#endif

/* Status codes. */
enum {
    TSB_OK = 0,
    TSB_ERR_ARG = 1,       /* invalid argument or shape */
    TSB_ERR_CUDA = 2,      /* CUDA runtime error */
    TSB_ERR_DEVICE = 3,    /* a kernel reported an error word (bounded wait expired) */
    TSB_ERR_MODEL = 4,     /* model not supported by the device path */
    TSB_ERR_NAN = 5,       /* forecast produced NaN (reference: degenerate input) */
};

/* ---- device-resident forecast (throughput path) ----------------------------------
 * Equivalent of timestral_capi_forecast for requests without covariates, with the
 * context and the output already in device memory of the handle's GPU.
 * d_context: [B,V,T] f32 (NaN = missing); d_mask: [B,V,T] u8 or NULL;
 * d_out: [B,V,H,Q] f32. Flags: -1 = model default, 0, 1. Runs on the handle's stream
 * and returns after enqueueing when `async` is nonzero, else after completion. */
TIMESTRAL_API int tsb_forecast_device(timestral_ctx* ctx, const float* d_context, const uint8_t* d_mask,
                                      int32_t B, int32_t V, int32_t T, int32_t H, int32_t symmetric,
                                      int32_t clip, int32_t max_context, float* d_out, int32_t async);

/* ---- several GPUs per handle ---------------------------------------------------------
 * A handle that forecasts on several GPUs of this machine through the unchanged
 * timestral_capi_forecast (reference src/timestral_capi.cpp:60-90): the model is uploaded
 * to every listed device; each request's series are split into contiguous shards, one per
 * device (shard k of n holds series [k*B/n, (k+1)*B/n)), forecast concurrently by one host
 * thread and CUDA stream per device, and each shard's result is copied from its device
 * straight into its slice of the one result buffer. There is no collective: a series never
 * leaves its device, and its forecast is the same bits as on one GPU. A device listed more
 * than once takes that many shards (each with its own stream). Returns NULL (error in
 * timestral_capi_last_error(NULL)) for an invalid device ordinal.
 * timestral_capi_load does the same when the environment variable TIMESTRAL_DEVICES holds a
 * comma-separated list of device ordinals or "all". The device-resident entries below
 * (tsb_forecast_device, tsb_stream, ...) act on the handle's first device. */
TIMESTRAL_API timestral_ctx* tsb_load_devices(const char* path, int threads, const int32_t* devices, int32_t n_devices);
/* Number of GPUs the handle forecasts on. */
TIMESTRAL_API int32_t tsb_device_count(timestral_ctx* ctx);

/* Wait for the handle's stream; returns TSB_ERR_DEVICE (with last_error set) when a kernel
 * of an asynchronous tsb_forecast_device call reported an error. */
TIMESTRAL_API int tsb_sync(timestral_ctx* ctx);
/* Select the GPU used by handles loaded afterwards on this thread (default: current device). */
TIMESTRAL_API int tsb_set_device(int32_t device);
/* cudaStream_t of the handle (as an opaque pointer), for callers that time with events. */
TIMESTRAL_API void* tsb_stream(timestral_ctx* ctx);
/* RMSNorm carried by the tensor-core GEMMs (mode 1, the default): each residual-add GEMM
 * also leaves an f16 copy of the residual (scaled by 1/16) and its row sums of squares, and
 * the next GEMM, whose weights hold the norm weight, scales each row by 1/rms itself, so the
 * RMSNorm kernel runs once per decode block instead of once per sublayer. A forecast that
 * meets a residual value the f16 copy cannot hold (|x| > 2^20) or a row whose RMS is below
 * 2^-8 is run again with the RMSNorm kernel, so results never depend on that range. Mode 0:
 * always the RMSNorm kernel. Mode 2: mode 1, and every forecast also takes the fallback run
 * (tests that path). Replaces the reference's per-sublayer rms_f32 node (src/layers.cpp:262-287)
 * on the tensor-core path. */
TIMESTRAL_API int tsb_fused_norm(timestral_ctx* ctx, int32_t mode);
/* Attention kernels of the tensor-core path: mode 0 (default) the tensor-core kernels (f16
 * probabilities, f32 accumulation in tensor memory); mode 1 the CUDA-core kernels that keep
 * the reference's attention arithmetic (float64 q.k dots, f32 softmax, f32 value sums;
 * reference src/layers.cpp:578-617) on the same f16 q/k/v, for time rows of up to 2176 tokens
 * and the variate axis. Mode 1 is slower; it shows how much of a forecast's deviation from the
 * reference comes from the tensor-core attention. */
TIMESTRAL_API int tsb_attention_kernels(timestral_ctx* ctx, int32_t mode);
/* Block-quantised weights dequantised in the GEMM prologue (on = 1) instead of read as the
 * f16 copies made at load (on = 0, the default): the GEMM streams the int8 weight tiles with
 * their block scales (Q8_0: the f16 scale of every 32 values, reference src/weight_policy.hpp:23-30)
 * or scales and offsets (Q4_K/Q5_K/Q6_K, src/weight_policy.hpp:13-16: one f32 scale and
 * offset per 16 values, unpacked from the super-blocks at load), and converter warps write the
 * f16 tiles the tensor cores read, each value rounded once to f16 as at load, so the forecast
 * is the same bits. Weights that carry a folded RMSNorm gain other than 1 keep their f16 copy.
 * Returns TSB_ERR_MODEL when the model has no block-quantised weights. */
TIMESTRAL_API int tsb_dequant_prologue(timestral_ctx* ctx, int32_t on);
/* Decoder-token tail (on = 1, the default): the last layer of the 209M schedule starts with a
 * time sublayer and continues with per-token work (a one-row series' variate sublayer and
 * the MLP), and the head reads only the decoder tokens, so after that layer's time attention
 * the remaining GEMMs run on the decoder tokens of every row alone (8 of 72 tokens at T = 2048,
 * H = 256). The forecast is the same bits either way; on = 0 computes every token as the
 * reference does (src/encoder.cpp:45-106 then src/predict_block.cpp:15-16 slices). */
TIMESTRAL_API int tsb_decoder_tail(timestral_ctx* ctx, int32_t on);
/* CUDA-graph replay (on by default): a forecast without covariates that fits one decode
 * block (H <= 32 patches of the 209M geometry) is captured into a CUDA graph on its second
 * call with the same sizes, flags and device buffers (tsb_forecast_device pointers, or the
 * handle's staging buffers for timestral_capi_forecast), and later identical calls launch
 * that graph, which removes the per-kernel launch cost. The graph is dropped when any
 * workspace of the library is reallocated. on = 0 disables it. Replaces nothing in the
 * reference (its graphs are ggml's per-block graphs, src/backend.cpp GraphRunner). */
TIMESTRAL_API int tsb_graph_replay(timestral_ctx* ctx, int32_t on);
/* Covariate requests: assemble the rows on the device (on_device != 0, the default) or on
 * the host (the host path of the reference's assemble_rows, kept for comparison); the two
 * give identical forecasts. Replaces nothing in the reference (its assembly is host-only,
 * src/covariates.cpp:32-72). */
TIMESTRAL_API int tsb_covariate_assembly(timestral_ctx* ctx, int32_t on_device);
/* Per-kernel timing: when enabled, kernel launches are bracketed by CUDA events on the
 * handle's stream and read back per class ("attention", "gemm", "rms", "scale", "all", ...).
 * enable: 0 off, 1 every launch, 2 attention launches alone. */
TIMESTRAL_API int tsb_timing_enable(timestral_ctx* ctx, int32_t enable);
/* Total milliseconds and launch count recorded for a kernel class since the last reset. */
TIMESTRAL_API int tsb_timing_read(timestral_ctx* ctx, const char* cls, double* ms, int64_t* launches);
TIMESTRAL_API void tsb_timing_reset(timestral_ctx* ctx);
/* Kernels launched by the last forecast call (all classes). */
TIMESTRAL_API int64_t tsb_last_launch_count(timestral_ctx* ctx);
/* Compute path chosen for the loaded model: 1 = tensor cores (F16/Q8_0 weights),
 * 0 = F32 CUDA-core path. */
TIMESTRAL_API int tsb_model_path(timestral_ctx* ctx);
/* Host-side dequantisation of `rows` rows of ne0 elements of a block-quantised GGUF type
 * (8 Q8_0, 12 Q4_K, 13 Q5_K, 14 Q6_K) into float, as the loader expands such weights.
 * No GPU is used. */
TIMESTRAL_API int tsb_dequantize_rows(uint32_t type, const void* src, int64_t rows, int64_t ne0, float* dst);
/* Host-side unpacking of `rows` rows of ne0 elements of a block-quantised GGUF type (8 Q8_0,
 * 12 Q4_K, 13 Q5_K, 14 Q6_K) into the form the GEMM's dequantising prologue reads: integer
 * values q [rows][ne0] and, per 16 consecutive values, a scale a and an offset b
 * ([rows][ne0 / 16] each), with tsb_dequantize_rows' value = (a * q) - b exactly in single
 * precision. No GPU is used. */
TIMESTRAL_API int tsb_scaled_int8_rows(uint32_t type, const void* src, int64_t rows, int64_t ne0, int8_t* q, float* a,
                                       float* b);
/* Geometry of the last decode block of the handle's last forecast: model rows (both
 * symmetric passes, every row role), tokens per row, context patches, decode blocks. */
TIMESTRAL_API int tsb_last_geometry(timestral_ctx* ctx, int64_t* rows, int32_t* S, int32_t* L, int32_t* blocks);

/* ---- refine without device allocation --------------------------------------------
 * No counterpart in the reference. The refine step of one decode block (re-normalising a
 * block's quantiles into advancing per-patch frames) on caller device buffers, for callers
 * that may not allocate GPU memory: an application that owns every allocation on the
 * device and hands this library fixed buffers, or a loop that must never enter the CUDA
 * allocator. The float64 scan scratch comes from a 4 MiB array compiled into the library
 * instead of cudaMalloc. CUDA loads a library's device code lazily, so the array is reserved
 * on a GPU when the library's code first runs there (this entry point's first call, or any
 * forecast) and is held until the process exits; make a first call at set-up (a one-row
 * request is enough) and every later call allocates nothing.
 * d_q/d_out: [rows][patches*patch_size][num_quantiles] f32; d_rows: [rows][length] f32
 * context; d_mask: [rows][length] bytes 0/1; d_role: [rows] (0 = target row; others keep
 * their quantiles) or NULL for all targets; d_loc0/d_scale0: [rows] frame of the last
 * context step. Requests needing more than the reserved scratch, rows * (3 * (length /
 * patch_size + patches) + 2 * patch_size + 2 * patches) float64 values above 524,288, are
 * rejected with TSB_ERR_ARG before any device work (split the rows across calls). The first
 * call on a device looks up the array's device address (cudaGetSymbolAddress), and so does
 * the first call after that device's context was reset (cudaDeviceReset); make those calls
 * before any stream capture. All calls share the one array, which keeps the last call's
 * values (every value a call reads it first writes): calls that overlap on the GPU (other
 * streams, other threads) race on it. Enqueued on `stream` (cudaStream_t, NULL = legacy
 * default stream); errors go to timestral_capi_last_error(NULL). */
TIMESTRAL_API int tsb_refine_static(const float* d_q, const float* d_rows, const int8_t* d_mask, const int8_t* d_role,
                                    const float* d_loc0, const float* d_scale0, int32_t rows, int32_t length,
                                    int32_t patches, int32_t patch_size, int32_t num_quantiles, int32_t median_index,
                                    double minimum_scale, float* d_out, void* stream);

/* ---- kernel-level test entries (device pointers) ---------------------------------- */
typedef struct tsb_gemm_test {
    int32_t kind;                 /* 0 f32, 1 f16, 2 resid, 3 silu, 4 swiglu, 5 vgate, 6 qkvg */
    const void* A; int64_t lda;   /* f16 [M][lda] */
    const void* B; int64_t ldb;   /* f16 [N][ldb] */
    int32_t M, N, K;
    void* out; int64_t ldo;
    const float* bias; const float* resid;
    int32_t row_group, row_stride, row_offset;
    void* qkvg[4]; int32_t S, H, D, rope;
    const float* cos_tab; const float* sin_tab; const int32_t* rope_row; int32_t rope_half;
    int32_t rope_dup;             /* tables have equal halves (cos[d] == cos[d + 32]) */
    int32_t a_group, a_stride, a_offset;  /* A row of accumulator row m: (m / a_group) * a_stride
                                             + a_offset + m % a_group (a_group 0: m) */
    const int8_t* Bq; const void* Bd; int64_t ldd;  /* Q8_0 B: int8 [N][ldb bytes], f16 scales
                                                       [K/32][ldd]; used instead of B when Bq is set */
    const float* Bs; int64_t lds;                   /* scaled int8 B: (scale, offset) per 16 values,
                                                       [K/16][lds][2]; used instead of Bd when set */
} tsb_gemm_test;
/* Runs one tensor-core GEMM on the current device and synchronizes. Returns a TSB_ code;
 * on TSB_ERR_DEVICE the kernel's error word is written to *dev_error. */
TIMESTRAL_API int tsb_test_gemm(const tsb_gemm_test* t, int32_t* dev_error);
/* RMSNorm of `tokens` rows of width D (device pointers) on the current device, synchronized:
 * out = x * (1 / sqrt(mean(x^2) + eps)) * w, f32 or (out_f16 != 0) f16. */
/* Tensor-core time attention of `rows` rows without covariates (S <= 128, head_dim 64):
 * q/k/v/gate f16 head-major [rows][H][S][64] (gate may be NULL), key_valid [rows][ceil(N/32)]
 * bit p = patch p observed, out f16 token-major [rows * S][H * 64]; synchronized. */
TIMESTRAL_API int tsb_test_attention_time(const void* q, const void* k, const void* v, const void* gate, void* out,
                                          const uint32_t* key_valid, int32_t rows, int32_t H, int32_t S, int32_t N,
                                          int32_t* dev_error);
/* Time attention with the full mask description: N encoder tokens, L context patches,
 * covariate layout (cov != 0: S = 2N, role [rows] 0 target / 1 past / 2 known, decode blocks
 * of block_size patches). kernel: 0 the engine's choice, 1 the S <= 128 tensor-core kernel
 * (two problems per score tile when S <= 64), 2 the tiled tensor-core kernel (any S), 3 the
 * CUDA-core kernel (the tiled one for S > 128), 4 the S <= 128 tensor-core kernel with one
 * problem per tile, 5 the CUDA-core kernel with one warp per query, 6 the tiled CUDA-core
 * kernel (kernels 3, 5 and 6 give the same bits). Same layouts as above.
 * repeat > 0 with ms non-NULL: after the checked launch, *ms = the average device time of
 * `repeat` more launches. */
TIMESTRAL_API int tsb_test_attention_time_ex(const void* q, const void* k, const void* v, const void* gate, void* out,
                                             const uint32_t* key_valid, const int8_t* role, int32_t rows, int32_t H,
                                             int32_t S, int32_t N, int32_t L, int32_t cov, int32_t block_size,
                                             int32_t kernel, int32_t repeat, float* ms, int32_t* dev_error);
/* Causal scaler and patch features of R rows of W steps (device pointers, synchronized):
 * rows f32 / mask int8 [R][W]; features [R][W/ps][2ps]; loc/scale [R] (frame of step
 * anchor_step); key_valid [R][ceil(enc_patches/32)]; first_obs [R]; cap_lo/cap_hi/cap_scale
 * [R] or NULL (statistics over the first ctx_len steps). kernel 0: one thread per row,
 * 1: one block per row (the two give identical results). */
TIMESTRAL_API int tsb_test_scale_rows(const float* rows, const int8_t* mask, int32_t R, int32_t W, int32_t ps,
                                      double minimum_scale, int32_t use_asinh, int32_t attend_missing,
                                      int32_t anchor_step, int32_t enc_patches, int32_t ctx_len, int32_t kernel,
                                      float* features, float* loc, float* scale, uint32_t* key_valid, int32_t* first_obs,
                                      float* cap_lo, float* cap_hi, float* cap_scale);
/* f16 hi/lo split used by the tensor-core patch projections: out [rows][3K] f16 =
 * [hi | hi | lo] of each f32 row of a; sets *d_overflow (device int) when any |a| > 30000. */
TIMESTRAL_API int tsb_test_split_f16(const float* a, int64_t rows, int32_t K, void* out, int32_t* d_overflow);
/* Variate-axis attention of the tensor-core path over groups of G consecutive rows (one
 * series each): q/k/v/gate f16 head-major [rows][H][S][64] (gate may be NULL), key_valid
 * [rows][ceil(N/32)] bits, role [rows] (0 target, 1 past, 2 known) or NULL without
 * covariates, out f16 token-major [rows * S][H * 64]; synchronized. kernel: 0 the engine's
 * choice, 1 the CUDA-core kernel (G <= 64), 2 the tensor-core kernel (G <= 32, four
 * (series, head, slot) problems per score tile). On TSB_ERR_DEVICE *dev_error (may be NULL)
 * holds the kernel's error word. */
TIMESTRAL_API int tsb_test_attention_variate_ex(const void* q, const void* k, const void* v, const void* gate, void* out,
                                                const uint32_t* key_valid, const int8_t* role, int32_t rows, int32_t H,
                                                int32_t S, int32_t N, int32_t G, int32_t kernel, int32_t* dev_error);
/* The same with kernel 1. */
TIMESTRAL_API int tsb_test_attention_variate(const void* q, const void* k, const void* v, const void* gate, void* out,
                                             const uint32_t* key_valid, const int8_t* role, int32_t rows, int32_t H,
                                             int32_t S, int32_t N, int32_t G);
/* CUDA-core GEMM of the F32 path, out[M][N] f32 = A[M][K] W[N][K]^T (device pointers,
 * synchronized), with the per-output order `order` (0: 192-wide K panels in K order, 1: one
 * FMA chain, 2: float64); tiled bit 0 lets large panel-order launches run the 64 x 128 tile
 * kernel (same bits as the 64 x 64 one); bit 1 gives launches of at most 512 rows with
 * K >= 384 panel scratch (allocated here), so that they run the panel-split path (one block
 * per 192-wide panel, the partials summed in panel order; same bits as one pass). */
TIMESTRAL_API int tsb_test_simt_gemm(const float* A, const float* W, int32_t M, int32_t N, int32_t K, int32_t order,
                                     int32_t tiled, float* out);
/* The refine step of one decode block with its float64 scratch from cudaMalloc (as the
 * forecast's workspace provides it), on the current device, synchronized; arguments as
 * tsb_refine_static (patches >= 2, d_role may be NULL). */
TIMESTRAL_API int tsb_test_refine(const float* d_q, const float* d_rows, const int8_t* d_mask, const int8_t* d_role,
                                  const float* d_loc0, const float* d_scale0, int32_t rows, int32_t length, int32_t patches,
                                  int32_t patch_size, int32_t num_quantiles, int32_t median_index, double minimum_scale,
                                  float* d_out);
TIMESTRAL_API int tsb_test_rms(const float* x, const float* w, int32_t tokens, int32_t D, float eps, void* out,
                               int32_t out_f16);
/* Failure detection without a GPU fault: one CTA whose bounded barrier wait runs out (a
 * barrier nothing arrives on) while a second role leaves through the abort flag; kernel 0
 * uses the GEMM roles' wait, 1 the attention kernels'. Takes one wait limit (about 2 s at
 * full clock), synchronizes, and returns TSB_ERR_DEVICE with the expired wait's error word
 * in *dev_error (the GEMM's stage-fill or the attention barrier code) and 1 in
 * *left_by_abort when the second role left through the flag; the context stays usable. */
TIMESTRAL_API int tsb_test_wait_expiry(int32_t kernel, int32_t* dev_error, int32_t* left_by_abort);
/* Failure injection on the host: the next n workspace allocations of any forecast in the
 * process fail as an exhausted device would (cudaErrorMemoryAllocation); 0 clears it. */
TIMESTRAL_API int tsb_test_fail_workspace_allocations(int32_t n);
/* cudaDeviceReset of the current device (ends this process's context there; every handle
 * and result buffer of that device must have been freed first). Later handles set their
 * kernels' launch attributes again and take no pooled result buffer the reset freed. */
TIMESTRAL_API int tsb_test_device_reset(void);

#ifdef __cplusplus
}
#endif
#endif
