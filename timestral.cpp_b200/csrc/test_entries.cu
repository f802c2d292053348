// Kernel-level test entries of the C ABI (include/timestral_b200.h): run one kernel on
// caller-owned device buffers so the GPU tests can compare it with a reference op.
#include "common.cuh"
#include "attention.cuh"
#include "engine.cuh"
#include "gemm_tc.cuh"
#include "rows.cuh"
#include "timestral_b200.h"

#include <cfloat>
#include <cmath>
#include <cstring>

extern "C" TIMESTRAL_API int tsb_test_gemm(const tsb_gemm_test* t, int32_t* dev_error) {
    using namespace tsb;
    if (!t) return TSB_ERR_ARG;
    GemmArgs a;
    a.A = static_cast<const __half*>(t->A); a.lda = t->lda;
    a.B = static_cast<const __half*>(t->B); a.ldb = t->ldb;
    a.M = t->M; a.N = t->N; a.K = t->K;
    a.a_group = t->a_group; a.a_stride = t->a_stride; a.a_offset = t->a_offset;
    a.Bq = t->Bq; a.Bd = static_cast<const __half*>(t->Bd); a.ldd = t->ldd;
    a.Bs = t->Bs; a.lds = t->lds;
    GemmEpilogue& e = a.epi;
    e.out = t->out; e.ldo = t->ldo; e.bias = t->bias; e.resid = t->resid;
    e.row_group = t->row_group; e.row_stride = t->row_stride; e.row_offset = t->row_offset;
    for (int i = 0; i < 4; ++i) e.qkvg[i] = static_cast<__half*>(t->qkvg[i]);
    e.S = t->S; e.H = t->H; e.D = t->D; e.rope = t->rope;
    e.cos_tab = t->cos_tab; e.sin_tab = t->sin_tab; e.rope_row = t->rope_row; e.rope_half = t->rope_half;
    e.rope_dup = t->rope_dup;
    int* derr = nullptr;
    if (cudaMalloc(&derr, sizeof(int)) != cudaSuccess) return TSB_ERR_CUDA;
    cudaMemset(derr, 0, sizeof(int));
    cudaError_t ce = tc_gemm(static_cast<EpiKind>(t->kind), a, 0, derr);
    if (ce == cudaErrorInvalidValue) { cudaFree(derr); return TSB_ERR_ARG; }
    if (ce == cudaSuccess) ce = cudaDeviceSynchronize();
    int h = 0;
    cudaMemcpy(&h, derr, sizeof(int), cudaMemcpyDeviceToHost);
    cudaFree(derr);
    if (dev_error) *dev_error = h;
    if (ce != cudaSuccess) return TSB_ERR_CUDA;
    return h ? TSB_ERR_DEVICE : TSB_OK;
}

extern "C" TIMESTRAL_API int tsb_test_simt_gemm(const float* A, const float* W, int32_t M, int32_t N, int32_t K,
                                                int32_t order, int32_t tiled, float* out) {
    if (!A || !W || !out || M <= 0 || N <= 0 || K <= 0 || order < 0 || order > 2) return TSB_ERR_ARG;
    tsb::SimtGemm g;
    g.A = A; g.lda = K; g.W = W; g.M = M; g.N = N; g.K = K;
    g.order = order; g.epi = tsb::SEPI_F32; g.out = out; g.ldo = N; g.tiled = tiled & 1;
    // bit 1: give the launch panel scratch, as the engine does, so that few-row launches run
    // the panel-split path
    float* scratch = nullptr;
    const size_t need = (tiled & 2) ? tsb::simt_panel_scratch_bytes(g) : 0;
    if (need) {
        if (cudaMalloc(&scratch, need) != cudaSuccess) return TSB_ERR_CUDA;
        g.panel_scratch = scratch;
        g.panel_scratch_bytes = need;
    }
    cudaError_t e = tsb::simt_gemm(g, 0);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (scratch) cudaFree(scratch);
    return e == cudaSuccess ? TSB_OK : TSB_ERR_CUDA;
}

extern "C" TIMESTRAL_API int tsb_test_rms(const float* x, const float* w, int32_t tokens, int32_t D, float eps, void* out,
                                          int32_t out_f16) {
    if (!x || !w || !out || tokens < 0 || D <= 0) return TSB_ERR_ARG;
    cudaError_t e = tsb::rms_norm(x, w, tokens, D, eps, out, out_f16, 0, 0, 0, 0);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    return e == cudaSuccess ? TSB_OK : TSB_ERR_CUDA;
}

extern "C" TIMESTRAL_API int tsb_test_attention_time(const void* q, const void* k, const void* v, const void* gate, void* out,
                                                     const uint32_t* key_valid, int32_t rows, int32_t H, int32_t S,
                                                     int32_t N, int32_t* dev_error) {
    using namespace tsb;
    if (!q || !k || !v || !out || !key_valid || rows <= 0 || H <= 0 || S <= 0 || S > 128 || N <= 0 || N > S)
        return TSB_ERR_ARG;
    MaskMeta mm;
    mm.key_valid = key_valid; mm.kv_words = (N + 31) / 32; mm.N = N; mm.L = N; mm.S = S;
    int* derr = nullptr;
    if (cudaMalloc(&derr, sizeof(int)) != cudaSuccess) return TSB_ERR_CUDA;
    cudaMemset(derr, 0, sizeof(int));
    cudaError_t ce = attention_time_tc(static_cast<const __half*>(q), static_cast<const __half*>(k),
                                       static_cast<const __half*>(v), static_cast<const __half*>(gate),
                                       static_cast<__half*>(out), rows, H, mm, 0, derr);
    if (ce == cudaSuccess) ce = cudaDeviceSynchronize();
    int h = 0;
    cudaMemcpy(&h, derr, sizeof(int), cudaMemcpyDeviceToHost);
    cudaFree(derr);
    if (dev_error) *dev_error = h;
    if (ce != cudaSuccess) return ce == cudaErrorInvalidValue ? TSB_ERR_ARG : TSB_ERR_CUDA;
    return h ? TSB_ERR_DEVICE : TSB_OK;
}

extern "C" TIMESTRAL_API int tsb_test_attention_time_ex(const void* q, const void* k, const void* v, const void* gate,
                                                        void* out, const uint32_t* key_valid, const int8_t* role,
                                                        int32_t rows, int32_t H, int32_t S, int32_t N, int32_t L,
                                                        int32_t cov, int32_t block_size, int32_t kernel,
                                                        int32_t repeat, float* ms, int32_t* dev_error) {
    using namespace tsb;
    if (!q || !k || !v || !out || !key_valid || rows <= 0 || H <= 0 || S <= 0 || N <= 0 || N > S || L <= 0 || L > N ||
        (cov && (!role || block_size <= 0 || S != 2 * N)) || kernel < 0 || kernel > 6 || ((kernel == 1 || kernel == 4) && S > 128))
        return TSB_ERR_ARG;
    MaskMeta mm;
    mm.key_valid = key_valid; mm.kv_words = (N + 31) / 32; mm.N = N; mm.L = L; mm.S = S;
    mm.cov = cov ? 1 : 0; mm.block_size = block_size; mm.role = role;
    if (kernel == 0) kernel = S <= 128 ? 1 : 2;
    int* derr = nullptr;
    if (cudaMalloc(&derr, sizeof(int)) != cudaSuccess) return TSB_ERR_CUDA;
    cudaMemset(derr, 0, sizeof(int));
    const __half *hq = static_cast<const __half*>(q), *hk = static_cast<const __half*>(k), *hv = static_cast<const __half*>(v);
    const __half* hg = static_cast<const __half*>(gate);
    __half* ho = static_cast<__half*>(out);
    auto launch = [&]() {
        return kernel == 1   ? attention_time_tc(hq, hk, hv, hg, ho, rows, H, mm, 0, derr)
               : kernel == 4 ? attention_time_tc(hq, hk, hv, hg, ho, rows, H, mm, 0, derr, 0)
               : kernel == 2 ? attention_time_tc_long(hq, hk, hv, hg, ho, rows, H, mm, 0, derr)
               : kernel == 5 ? attention_time_simt<__half>(hq, hk, hv, hg, ho, rows, H, 64, mm, 0, 0)
               : kernel == 6 ? attention_time_simt<__half>(hq, hk, hv, hg, ho, rows, H, 64, mm, 0, 1)
                             : attention_time_simt<__half>(hq, hk, hv, hg, ho, rows, H, 64, mm, 0);
    };
    cudaError_t ce = launch();
    if (ce == cudaSuccess) ce = cudaDeviceSynchronize();
    if (ce == cudaSuccess && repeat > 0 && ms) {
        // average device time of `repeat` further launches (CUDA events on the launch stream)
        cudaEvent_t e0, e1;
        cudaEventCreate(&e0);
        cudaEventCreate(&e1);
        cudaEventRecord(e0, 0);
        for (int it = 0; it < repeat && ce == cudaSuccess; ++it) ce = launch();
        cudaEventRecord(e1, 0);
        if (ce == cudaSuccess) ce = cudaEventSynchronize(e1);
        float t = 0.f;
        cudaEventElapsedTime(&t, e0, e1);
        *ms = t / float(repeat);
        cudaEventDestroy(e0);
        cudaEventDestroy(e1);
    }
    int h = 0;
    cudaMemcpy(&h, derr, sizeof(int), cudaMemcpyDeviceToHost);
    cudaFree(derr);
    if (dev_error) *dev_error = h;
    if (ce != cudaSuccess) return ce == cudaErrorInvalidValue ? TSB_ERR_ARG : TSB_ERR_CUDA;
    return h ? TSB_ERR_DEVICE : TSB_OK;
}

extern "C" TIMESTRAL_API int tsb_test_scale_rows(const float* rows, const int8_t* mask, int32_t R, int32_t W, int32_t ps,
                                                double minimum_scale, int32_t use_asinh, int32_t attend_missing,
                                                int32_t anchor_step, int32_t enc_patches, int32_t ctx_len, int32_t kernel,
                                                float* features, float* loc, float* scale, uint32_t* key_valid,
                                                int32_t* first_obs, float* cap_lo, float* cap_hi, float* cap_scale) {
    if (!rows || !mask || !features || !loc || !scale || !key_valid || !first_obs || R <= 0 || ps <= 0 || W <= 0 ||
        W % ps || enc_patches <= 0 || enc_patches > W / ps || kernel < 0 || kernel > 1)
        return TSB_ERR_ARG;
    tsb::RowConfig c;
    c.ps = ps; c.minimum_scale = minimum_scale; c.use_asinh = use_asinh; c.attend_missing = attend_missing;
    cudaError_t e = tsb::scale_rows(c, rows, mask, R, W, anchor_step, enc_patches, (enc_patches + 31) / 32, features, loc,
                                    scale, key_valid, first_obs, ctx_len, cap_lo, cap_hi, cap_scale, 0, kernel);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    return e == cudaSuccess ? TSB_OK : (e == cudaErrorInvalidValue ? TSB_ERR_ARG : TSB_ERR_CUDA);
}

extern "C" TIMESTRAL_API int tsb_test_split_f16(const float* a, int64_t rows, int32_t K, void* out, int32_t* d_overflow) {
    if (!a || !out || !d_overflow || rows < 0 || K <= 0) return TSB_ERR_ARG;
    cudaError_t e = tsb::split_f16(a, rows, K, static_cast<__half*>(out), d_overflow, nullptr, 0);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    return e == cudaSuccess ? TSB_OK : TSB_ERR_CUDA;
}

extern "C" TIMESTRAL_API int tsb_test_attention_variate_ex(const void* q, const void* k, const void* v, const void* gate,
                                                           void* out, const uint32_t* key_valid, const int8_t* role,
                                                           int32_t rows, int32_t H, int32_t S, int32_t N, int32_t G,
                                                           int32_t kernel, int32_t* dev_error) {
    using namespace tsb;
    if (!q || !k || !v || !out || !key_valid || rows <= 0 || H <= 0 || S <= 0 || N <= 0 || N > S || G <= 0 ||
        rows % G || kernel < 0 || kernel > 2)
        return TSB_ERR_ARG;
    MaskMeta mm;
    mm.key_valid = key_valid; mm.kv_words = (N + 31) / 32; mm.N = N; mm.L = N; mm.S = S;
    mm.cov = role != nullptr; mm.role = role;
    if (kernel == 0) kernel = G <= 32 ? 2 : 1;
    int* derr = nullptr;
    if (cudaMalloc(&derr, sizeof(int)) != cudaSuccess) return TSB_ERR_CUDA;
    cudaMemset(derr, 0, sizeof(int));
    const __half *hq = static_cast<const __half*>(q), *hk = static_cast<const __half*>(k), *hv = static_cast<const __half*>(v);
    const __half* hg = static_cast<const __half*>(gate);
    __half* ho = static_cast<__half*>(out);
    cudaError_t ce = kernel == 2 ? attention_variate_tc(hq, hk, hv, hg, ho, rows, H, G, mm, 0, derr)
                                 : attention_variate_fast(hq, hk, hv, hg, ho, rows, H, G, mm, 0);
    if (ce == cudaSuccess) ce = cudaDeviceSynchronize();
    int h = 0;
    cudaMemcpy(&h, derr, sizeof(int), cudaMemcpyDeviceToHost);
    cudaFree(derr);
    if (dev_error) *dev_error = h;
    if (ce != cudaSuccess) return ce == cudaErrorInvalidValue ? TSB_ERR_ARG : TSB_ERR_CUDA;
    return h ? TSB_ERR_DEVICE : TSB_OK;
}

extern "C" TIMESTRAL_API int tsb_test_attention_variate(const void* q, const void* k, const void* v, const void* gate,
                                                        void* out, const uint32_t* key_valid, const int8_t* role,
                                                        int32_t rows, int32_t H, int32_t S, int32_t N, int32_t G) {
    return tsb_test_attention_variate_ex(q, k, v, gate, out, key_valid, role, rows, H, S, N, G, 1, nullptr);
}

// The refine kernel as the forecast runs it: float64 scan scratch taken from the allocator
// (the forecast's workspace), then freed. Same arguments as tsb_refine_static.
extern "C" TIMESTRAL_API int tsb_test_refine(const float* d_q, const float* d_rows, const int8_t* d_mask, const int8_t* d_role,
                                             const float* d_loc0, const float* d_scale0, int32_t rows, int32_t length,
                                             int32_t patches, int32_t patch_size, int32_t num_quantiles,
                                             int32_t median_index, double minimum_scale, float* d_out) {
    if (!d_q || !d_out || !d_rows || !d_mask || !d_loc0 || !d_scale0 || rows <= 0 || patches <= 1 || patch_size <= 0 ||
        length <= 0 || length % patch_size || num_quantiles <= 0 || num_quantiles > 64 || median_index < 0 ||
        median_index >= num_quantiles || !(minimum_scale > 0))
        return TSB_ERR_ARG;
    const size_t per_row = 3 * (size_t(length / patch_size) + size_t(patches)) + 2 * size_t(patch_size) + 2 * size_t(patches);
    double* scratch = nullptr;
    if (cudaMalloc(&scratch, per_row * size_t(rows) * sizeof(double)) != cudaSuccess) return TSB_ERR_CUDA;
    tsb::RowConfig rc;
    std::memset(&rc, 0, sizeof(rc));
    rc.ps = patch_size;
    rc.minimum_scale = minimum_scale;
    rc.Q = num_quantiles;
    rc.median = median_index;
    const double clip = std::pow(double(FLT_MAX), 0.5) / 1e3;
    cudaError_t e = tsb::refine(rc, d_q, d_rows, d_mask, length, d_role, d_loc0, d_scale0, rows, length, patches, clip,
                                scratch, d_out, 0);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    cudaFree(scratch);
    return e == cudaSuccess ? TSB_OK : TSB_ERR_CUDA;
}

extern "C" TIMESTRAL_API int tsb_test_wait_expiry(int32_t kernel, int32_t* dev_error, int32_t* left_by_abort) {
    using namespace tsb;
    if (kernel != 0 && kernel != 1) return TSB_ERR_ARG;
    int* d = nullptr;
    if (cudaMalloc(&d, 2 * sizeof(int)) != cudaSuccess) return TSB_ERR_CUDA;
    cudaError_t ce = cudaMemset(d, 0, 2 * sizeof(int));
    if (ce == cudaSuccess) ce = kernel == 0 ? gemm_wait_expiry_selftest(d, 0) : attention_wait_expiry_selftest(d, 0);
    if (ce == cudaSuccess) ce = cudaDeviceSynchronize();
    int h[2] = {0, 0};
    if (ce == cudaSuccess) ce = cudaMemcpy(h, d, sizeof(h), cudaMemcpyDeviceToHost);
    cudaFree(d);
    if (dev_error) *dev_error = h[0];
    if (left_by_abort) *left_by_abort = h[1];
    if (ce != cudaSuccess) return TSB_ERR_CUDA;
    return h[0] ? TSB_ERR_DEVICE : TSB_OK;
}

extern "C" TIMESTRAL_API int tsb_test_fail_workspace_allocations(int32_t n) {
    if (n < 0) return TSB_ERR_ARG;
    tsb::inject_workspace_failures(n);
    return TSB_OK;
}

extern "C" TIMESTRAL_API int tsb_test_device_reset(void) {
    return cudaDeviceReset() == cudaSuccess ? TSB_OK : TSB_ERR_CUDA;
}
