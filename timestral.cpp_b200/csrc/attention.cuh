// Attention kernels of the forecast path: time axis (per row, over patch tokens) and
// variate axis (per patch slot, over the rows of one series).
#pragma once
#include <cstdint>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

namespace tsb {

// Mask description shared by the kernels, computed in-register from compact metadata
// instead of the reference's dense [R,S,S] / [S,R,R] masks (reference src/masks.cpp:8-34).
struct MaskMeta {
    const uint32_t* key_valid = nullptr;  // [rows][kv_words] bit p = key_valid of patch p
    int kv_words = 0;
    int N = 0;            // encoder tokens (patches) per row
    int L = 0;            // context patches (== N on the context-only path)
    int S = 0;            // tokens per row
    int cov = 0;          // two-stream covariate layout (S = 2N)
    int block_size = 0;   // decoder block size (covariate anchors)
    const int8_t* role = nullptr;  // [rows] 0 target, 1 past, 2 known (covariate path)
    const int32_t* group_begin = nullptr;  // [rows] first row of the row's series (variate)
    const int32_t* group_size = nullptr;   // [rows] rows in the row's series
    int pass_rows = 0;    // rows of one forecast pass (variate lane/tail order)
};

// q/k/v/gate: head-major [rows][H][S][hd]; out: token-major [rows*S][H*hd] (gated).
// f16 tensor-core kernel, hd = 64, S <= 128. pack != 0: rows of S <= 64 tokens run two
// (row, head) problems per 128-query tile (same results as one per tile).
cudaError_t attention_time_tc(const __half* q, const __half* k, const __half* v, const __half* gate, __half* out,
                              int rows, int H, const MaskMeta& mm, cudaStream_t stream, int* err, int pack = 1);

// Same for S > 128 (any S): key/value tiles of 64 tokens, queries in tiles of 128.
cudaError_t attention_time_tc_long(const __half* q, const __half* k, const __half* v, const __half* gate, __half* out,
                                   int rows, int H, const MaskMeta& mm, cudaStream_t stream, int* err);

// Longest time row (tokens) the CUDA-core time-attention kernel takes.
constexpr int kSimtMaxKeys = 2176;

// CUDA-core kernels with the reference's operation order (float64 q.k dots, ATen exp for
// full eight-lane chunks, libm exp for the tail, eight-lane sums, value FMA chain, one
// reciprocal multiply). T = float (F32 path) or __half (tensor-core path inputs).
// gate may be null (no sdpa_sigmoid gate); out is T-typed token-major. tiled: -1 the tiled
// kernel for rows of more than 128 tokens at head_dim 64, 1 always at head_dim 64, 0 never
// (the two kernels give the same bits).
template <class T>
cudaError_t attention_time_simt(const T* q, const T* k, const T* v, const T* gate, T* out, int rows, int H, int hd,
                                const MaskMeta& mm, cudaStream_t stream, int tiled = -1);
// Variate-axis attention on tensor cores for series of G <= 32 consecutive rows (f16
// head-major q/k/v/gate, head_dim 64, out token-major f16): four (series, head, slot)
// problems per score tile. err: device error word (expired waits).
cudaError_t attention_variate_tc(const __half* q, const __half* k, const __half* v, const __half* gate, __half* out,
                                 int rows, int H, int G, const MaskMeta& mm, cudaStream_t stream, int* err);
// Variate-axis attention of the tensor-core path: groups of G <= 64 consecutive rows (one
// series), f16 head-major q/k/v/gate, head_dim 64, out token-major f16.
cudaError_t attention_variate_fast(const __half* q, const __half* k, const __half* v, const __half* gate, __half* out,
                                   int rows, int H, int G, const MaskMeta& mm, cudaStream_t stream);
template <class T>
cudaError_t attention_variate_simt(const T* q, const T* k, const T* v, const T* gate, T* out, int rows, int H,
                                   int hd, const MaskMeta& mm, cudaStream_t stream);

// Test of the attention kernels' bounded waits (no fault): one CTA in which one wait expires
// and records kDevTimeoutAttn in err[0], and a second warp leaves through the abort flag
// (err[1] = 1). Takes about one wait limit (kWaitCycles SM cycles).
cudaError_t attention_wait_expiry_selftest(int* err, cudaStream_t stream);

}  // namespace tsb
