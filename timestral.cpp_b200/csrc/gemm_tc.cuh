// Tensor-core GEMM interface: C = A * B^T with A [M,K] f16 activations (K contiguous) and
// B [N,K] f16 weights (the GGUF row layout), f32 accumulation in tensor memory, and the
// epilogue fused into the store.
#pragma once
#include <cstdint>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

namespace tsb {

enum EpiKind : int {
    EPI_F32 = 0,     // out f32 = acc + bias
    EPI_F16 = 1,     // out f16 = acc + bias
    EPI_RESID = 2,   // out f32 = resid + (acc + bias)            (resid may alias out)
    EPI_SILU = 3,    // out f16 = silu(acc + bias)
    EPI_SWIGLU = 4,  // tile halves (g | u): out f16 = g * silu(u) (weights interleaved per tile)
    EPI_VGATE = 5,   // tile halves (v | gate): out f16 = v * sigmoid(gate)
    EPI_QKVG = 6,    // columns q | k | v | gate: RoPE on q,k (optional), sigmoid on gate,
                     // scattered head-major to [rows][heads][tokens][64] f16
};

struct GemmEpilogue {
    void* out = nullptr;
    int64_t ldo = 0;                  // output row stride (elements)
    const float* bias = nullptr;      // [N] (in the weight's row order)
    const float* resid = nullptr;     // EPI_RESID input, same row mapping and stride as out
    // Output row of accumulator row m: (m / row_group) * row_stride + row_offset + m % row_group.
    int row_group = 0, row_stride = 0, row_offset = 0;
    // EPI_QKVG
    __half* qkvg[4] = {nullptr, nullptr, nullptr, nullptr};
    int S = 0, H = 0, D = 0;          // tokens per row, heads, model width
    int rope = 0;                     // apply RoPE to q and k
    const float* cos_tab = nullptr;   // [P][64]
    const float* sin_tab = nullptr;
    const int* rope_row = nullptr;    // [M] table row of each token
    int rope_half = 32;               // rotated dims per half head (rope_dim / 2)
    int rope_dup = 0;                 // tables satisfy cos[p][d] == cos[p][d + 32] (same for sin)
    // RMSNorm carried by the GEMMs (the norm weight folded into the consuming weights).
    // EPI_RESID: also write x16 = f16(x / 16) and, per row, the sum of squares of x over
    // each 128-column slot into ssq[m * ssq_slots + slot]; a value of x16 that would
    // overflow sets *norm_flag.
    __half* x16 = nullptr;
    int64_t ldx16 = 0;
    float* ssq = nullptr;
    int ssq_slots = 0;
    int* norm_flag = nullptr;
    // Consumers (EPI_F16, EPI_SWIGLU, EPI_VGATE, EPI_QKVG): with ssq_in set, the accumulator
    // of row m (A = x16) is scaled by 16 / sqrt(sum_j ssq_in[m * ssq_slots + j] / rms_D + rms_eps)
    // before the bias; a row whose RMS is below 2^-8 (where x / 16 loses precision in f16)
    // sets *norm_flag.
    const float* ssq_in = nullptr;
    int rms_D = 0;
    float rms_eps = 0.f;
};

struct GemmArgs {
    const __half* A = nullptr;
    int64_t lda = 0;
    // Row gather of A: with a_group > 0, accumulator row m reads A row
    // (m / a_group) * a_stride + a_offset + m % a_group (a_group divides 128), and so does its
    // ssq_in row (norm carried by the GEMM). Used to run a GEMM on the decoder tokens of every
    // row alone; 0: A rows are the accumulator rows.
    int a_group = 0, a_stride = 0, a_offset = 0;
    const __half* B = nullptr;
    int64_t ldb = 0;
    // Q8_0 weights dequantised in the GEMM prologue (used instead of B when Bq is set): int8
    // values Bq [N][K] (row pitch ldb bytes) and the f16 scale of every 32-value block,
    // Bd [K / 32][ldd] (scale of row n, block j at Bd[j * ldd + n]). In shared memory each
    // int8 tile becomes the f16 tile the tensor cores read, value q * d rounded once to f16:
    // the same f16 weights as dequantising at load.
    const int8_t* Bq = nullptr;
    const __half* Bd = nullptr;
    int64_t ldd = 0;
    // K-quant weights (and Q8_0) in scaled-int8 form, used with Bq instead of Bd when set: per
    // 16 values of row n, block g, a scale and an offset Bs[2 * (g * lds + n)], Bs[... + 1];
    // value (scale * q) - offset rounded once to f16, the loader's dequantisation.
    const float* Bs = nullptr;
    int64_t lds = 0;
    int M = 0, N = 0, K = 0;
    GemmEpilogue epi;
};

// Launch on `stream`. err: device error word (may be null). Returns a CUDA error code.
cudaError_t tc_gemm(EpiKind kind, const GemmArgs& args, cudaStream_t stream, int* err);
// Test of the GEMM roles' bounded waits (no fault): one CTA in which one wait expires and
// records kDevTimeoutFull in err[0], and a second role leaves through the abort flag
// (err[1] = 1). Takes about one wait limit (kWaitCycles SM cycles).
cudaError_t gemm_wait_expiry_selftest(int* err, cudaStream_t stream);

// Number of SMs of the current device (cached per device).
int device_sm_count();

}  // namespace tsb
