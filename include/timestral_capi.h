/* Flat C ABI of the forecaster — the drop-in surface.
 *
 * Same symbols, argument meaning, request layout and error behaviour as the reference
 * (reference include/timestral_capi.h:20-46, src/timestral_capi.cpp:60-92), so a binding
 * written for the reference (ctypes, cgo, purego) loads this library unchanged. The
 * forecast runs on a B200 instead of the CPU; `n_threads` keeps its validation (1..1024)
 * and sizes the host-side thread pool of the covariate assembly.
 *
 * Handles are not reentrant (callers serialise calls on one handle, free included);
 * independent handles may run concurrently. ABI version 1.
 */
#ifndef TIMESTRAL_CAPI_H
#define TIMESTRAL_CAPI_H
#include <stdint.h>
#if defined(__GNUC__)
#define TIMESTRAL_API __attribute__((visibility("default")))
#else
#define TIMESTRAL_API
#endif
#ifdef __cplusplus
extern "C" {
#endif

typedef struct timestral_ctx timestral_ctx;

/* Always 1. */
TIMESTRAL_API int timestral_capi_abi_version(void);
/* Load a GGUF model and upload it to the current GPU. NULL on error
   (timestral_capi_last_error(NULL) explains). */
TIMESTRAL_API timestral_ctx* timestral_capi_load(const char* gguf_path, int n_threads);
TIMESTRAL_API void timestral_capi_free(timestral_ctx* ctx);
/* Error text of the last failed call on `ctx`, or of the calling thread's last load or
   NULL-handle error when ctx is NULL. Valid until the next modifying call. These queries
   do not clear errors. */
TIMESTRAL_API const char* timestral_capi_last_error(timestral_ctx* ctx);
TIMESTRAL_API int timestral_capi_num_quantiles(timestral_ctx* ctx);
TIMESTRAL_API double timestral_capi_quantile_level(timestral_ctx* ctx, int i);

/* Field order and types are part of the ABI. */
typedef struct timestral_forecast_request {
    const float* context;            /* B*V*T, NaN = missing */
    const uint8_t* observation_mask; /* B*V*T or NULL; bytes 0/1 */
    int32_t B, V, T, prediction_length;
    const float* past_cov; int32_t c_past;     /* B*c_past*T */
    const float* known_cov; int32_t c_known;   /* B*c_known*(T+H) */
    const double* cat_past; int32_t cc_past;   /* B*cc_past*T */
    const double* cat_known; int32_t cc_known; /* B*cc_known*(T+H) */
    int32_t symmetric_averaging; /* -1 model default, 0, 1 */
    int32_t clip_nonnegative;    /* -1 model default, 0, 1 */
    int32_t max_context;         /* 0 model default */
} timestral_forecast_request;

/* Returns an owned F32 buffer [B,V,H,Q] (free it only with timestral_capi_free_buffer),
   or NULL on error. out_q is required and set to Q on success, 0 on failure. All sizes
   are validated before any caller buffer is read. */
TIMESTRAL_API float* timestral_capi_forecast(timestral_ctx* ctx, const timestral_forecast_request* req,
                                             int32_t* out_q);
TIMESTRAL_API void timestral_capi_free_buffer(void* p);

#ifdef __cplusplus
}
#endif
#endif
