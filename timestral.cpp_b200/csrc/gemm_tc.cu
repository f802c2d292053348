// Persistent tcgen05 GEMM for sm_100a with fused epilogues.
//
// Replaces the reference's projection nodes (src/layers.cpp:250-256 affine, 682-687 swiglu,
// src/head.cpp:275-286 head/patch projections, src/weight_policy.hpp:23-30 reduced
// projection), which on the reference's F16/Q8_0 path round activations to F16 and
// accumulate F16 products in F32 — the same arithmetic as kind::f16 with f32 accumulators.
//
// Tile 128 x BN x 64 (f16, 128-byte swizzle), STAGES-deep TMA ring, two TMEM accumulators
// so the epilogue of tile i overlaps the MMAs of tile i+1. Warp roles (320 threads):
//   warp 0: TMA producer (one lane)      warp 1: TMEM owner + MMA issuer (one lane)
//   warps 2..9: epilogue, one accumulator row per thread (TMEM lane quarter = warp % 4),
//   warps 2..5 take the first half of the tile's columns and warps 6..9 the second.
// Every mbarrier wait is bounded; a timeout records a device error and unwinds.
#include "common.cuh"
#include "gemm_tc.cuh"

#include <cstdio>
#include <mutex>

namespace tsb {

namespace {

constexpr int BM = 128;
constexpr int BK = 64;
constexpr int BN = 256;
constexpr int STAGES = 4;
constexpr int A_BYTES = BM * BK * 2;          // 16 KB
constexpr int B_BYTES = BN * BK * 2;          // 32 KB
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int TMEM_COLS = 2 * BN;             // 512: two accumulators
constexpr int EPI_WARPS = 8;                 // two warps per TMEM lane quarter, one per column half
constexpr int THREADS = 64 + 32 * EPI_WARPS;
constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 /*align*/ + 256 /*barriers*/;

struct Smem {
    uint64_t full[STAGES];
    uint64_t empty[STAGES];
    uint64_t acc_full[2];
    uint64_t acc_empty[2];
    uint32_t tmem_base;
    int abort;
};

__device__ __forceinline__ bool wait_or_abort(uint64_t* bar, uint32_t parity, volatile int* abort, int* err, int code) {
    if (mbar_try_wait(bar, parity)) return true;
    const long long start = clock64();
    while (true) {
        if (*abort) return false;
        if (mbar_try_wait(bar, parity)) return true;
        if (clock64() - start > kWaitCycles) {
            *abort = 1;
            record_error(err, code);
            return false;
        }
    }
}

__device__ __forceinline__ int64_t out_row(const GemmEpilogue& e, int m) {
    if (e.row_group <= 0) return m;
    return int64_t(m / e.row_group) * e.row_stride + e.row_offset + (m % e.row_group);
}

__device__ __forceinline__ void store_f32x32(float* dst, const float* v, int valid) {
    if (valid >= 32) {
#pragma unroll
        for (int i = 0; i < 32; i += 4) *reinterpret_cast<float4*>(dst + i) = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
    } else {
        for (int i = 0; i < valid; ++i) dst[i] = v[i];
    }
}
__device__ __forceinline__ void store_f16x32(__half* dst, const float* v, int valid) {
    if (valid >= 32) {
#pragma unroll
        for (int i = 0; i < 32; i += 8) {
            uint4 u;
            u.x = pack_half2(v[i], v[i + 1]); u.y = pack_half2(v[i + 2], v[i + 3]);
            u.z = pack_half2(v[i + 4], v[i + 5]); u.w = pack_half2(v[i + 6], v[i + 7]);
            *reinterpret_cast<uint4*>(dst + i) = u;
        }
    } else {
        for (int i = 0; i < valid; ++i) dst[i] = __float2half_rn(v[i]);
    }
}

// Activations of the tensor-core path. Their results are rounded to f16 for the next
// GEMM, so they use the hardware exp2 and approximate divide (a few ulp in f32, far below
// the f16 rounding) instead of the reference's exact float sequence used on the F32 path.
__device__ __forceinline__ float fast_sigmoid(float x) { return __fdividef(1.0f, 1.0f + __expf(-x)); }
__device__ __forceinline__ float fast_silu(float x) { return __fdividef(x, 1.0f + __expf(-x)); }

// Epilogue of columns [half*BN/2, (half+1)*BN/2) of one 128 x BN accumulator: the thread owns
// accumulator row `row_in_tile` (its TMEM lane).
template <int KIND>
__device__ __forceinline__ void epilogue_tile(const GemmArgs& g, uint32_t tacc, int m0, int n0, int row_in_tile, int half) {
    const GemmEpilogue& e = g.epi;
    const int m = m0 + row_in_tile;
    const bool row_ok = m < g.M;
    uint32_t r[32];
    if constexpr (KIND == EPI_SWIGLU || KIND == EPI_VGATE) {
        // The first half of the tile holds the first operand, the second half the second.
        float a[32];
        for (int c = half * (BN / 128); c < (half + 1) * (BN / 128); ++c) {
            tmem_ld32(tacc + c * 32, r);
            tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < 32; ++i) a[i] = __uint_as_float(r[i]);
            tmem_ld32(tacc + BN / 2 + c * 32, r);
            tmem_ld_wait();
            if (!row_ok) continue;
            const int wn = n0 + c * 32;             // weight row of the first operand column 0
            const int on = n0 / 2 + c * 32;         // output column
            float o[32];
#pragma unroll
            for (int i = 0; i < 32; ++i) {
                float x = a[i], y = __uint_as_float(r[i]);
                if (e.bias) { x = __fadd_rn(x, e.bias[wn + i]); y = __fadd_rn(y, e.bias[wn + BN / 2 + i]); }
                o[i] = KIND == EPI_SWIGLU ? __fmul_rn(x, fast_silu(y)) : __fmul_rn(x, fast_sigmoid(y));
            }
            store_f16x32(static_cast<__half*>(e.out) + out_row(e, m) * e.ldo + on, o, 32);
        }
    } else if constexpr (KIND == EPI_QKVG) {
        float v[64];
        for (int c = half * (BN / 128); c < (half + 1) * (BN / 128); ++c) {
            const int col = n0 + c * 64;
            const int which = col / e.D, h = (col % e.D) >> 6;
            const bool rope = row_ok && col < g.N && which < 2 && e.rope;
            // RoPE table entries of this token's position, requested before the TMEM reads.
            float4 tc[8], ts[8];
            const bool rope16 = rope && e.rope_half <= 16;
            if (rope16) {
                const float4* ct = reinterpret_cast<const float4*>(e.cos_tab + int64_t(e.rope_row[m]) * 64);
                const float4* st = reinterpret_cast<const float4*>(e.sin_tab + int64_t(e.rope_row[m]) * 64);
#pragma unroll
                for (int j = 0; j < 4; ++j) { tc[j] = ct[j]; tc[4 + j] = ct[8 + j]; ts[j] = st[j]; ts[4 + j] = st[8 + j]; }
            }
            tmem_ld32(tacc + c * 64, r);
            tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
            tmem_ld32(tacc + c * 64 + 32, r);
            tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < 32; ++i) v[32 + i] = __uint_as_float(r[i]);
            if (!row_ok || col >= g.N) continue;
            if (e.bias) {
#pragma unroll
                for (int i = 0; i < 64; ++i) v[i] = __fadd_rn(v[i], e.bias[col + i]);
            }
            if (rope) {
                // x*cos + rotate_half(x)*sin with separately rounded products and sum
                // (reference src/layers.cpp:238-246). Dims whose inverse frequency is zero
                // have cos 1 and sin 0 in every table row and are left unchanged.
                if (rope16) {
                    const float* c0 = reinterpret_cast<const float*>(tc);       // dims 0..15
                    const float* c1 = reinterpret_cast<const float*>(tc + 4);   // dims 32..47
                    const float* s0 = reinterpret_cast<const float*>(ts);
                    const float* s1 = reinterpret_cast<const float*>(ts + 4);
#pragma unroll
                    for (int i = 0; i < 16; ++i) {
                        if (i >= e.rope_half) break;
                        const float x0 = v[i], x1 = v[i + 32];
                        v[i] = __fadd_rn(__fmul_rn(x0, c0[i]), __fmul_rn(-x1, s0[i]));
                        v[i + 32] = __fadd_rn(__fmul_rn(x1, c1[i]), __fmul_rn(x0, s1[i]));
                    }
                } else {
                    const float* ct = e.cos_tab + int64_t(e.rope_row[m]) * 64;
                    const float* st = e.sin_tab + int64_t(e.rope_row[m]) * 64;
                    for (int i = 0; i < e.rope_half; ++i) {
                        const float x0 = v[i], x1 = v[i + 32];
                        v[i] = __fadd_rn(__fmul_rn(x0, ct[i]), __fmul_rn(-x1, st[i]));
                        v[i + 32] = __fadd_rn(__fmul_rn(x1, ct[i + 32]), __fmul_rn(x0, st[i + 32]));
                    }
                }
            } else if (which == 3) {
#pragma unroll
                for (int i = 0; i < 64; ++i) v[i] = fast_sigmoid(v[i]);
            }
            const int rr = m / e.S, s = m % e.S;
            __half* dst = e.qkvg[which] + ((int64_t(rr) * e.H + h) * e.S + s) * 64;
            store_f16x32(dst, v, 32);
            store_f16x32(dst + 32, v + 32, 32);
        }
    } else {
        float v[32];
        const int c0 = half * (BN / 64), c1 = (half + 1) * (BN / 64);
        const int64_t orow = row_ok ? out_row(e, m) : 0;
        // Residual rows of the next chunk are requested while the current chunk is stored.
        float4 rnext[8];
        auto load_resid = [&](int c, float4 (&dst)[8]) {
            const int col = n0 + c * 32;
            if (KIND == EPI_RESID && row_ok && col + 32 <= g.N) {
                const float4* rs = reinterpret_cast<const float4*>(e.resid + orow * e.ldo + col);
#pragma unroll
                for (int j = 0; j < 8; ++j) dst[j] = rs[j];
            }
        };
        if (KIND == EPI_RESID) load_resid(c0, rnext);
        for (int c = c0; c < c1; ++c) {
            float4 rcur[8];
            if (KIND == EPI_RESID) {
#pragma unroll
                for (int j = 0; j < 8; ++j) rcur[j] = rnext[j];
                if (c + 1 < c1) load_resid(c + 1, rnext);
            }
            tmem_ld32(tacc + c * 32, r);
            tmem_ld_wait();
            const int col = n0 + c * 32;
            if (!row_ok || col >= g.N) continue;
            const int valid = min(32, g.N - col);
#pragma unroll
            for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
            if (e.bias) {
                for (int i = 0; i < valid; ++i) v[i] = __fadd_rn(v[i], e.bias[col + i]);
            }
            if constexpr (KIND == EPI_F32) {
                store_f32x32(static_cast<float*>(e.out) + orow * e.ldo + col, v, valid);
            } else if constexpr (KIND == EPI_F16) {
                store_f16x32(static_cast<__half*>(e.out) + orow * e.ldo + col, v, valid);
            } else if constexpr (KIND == EPI_SILU) {
#pragma unroll
                for (int i = 0; i < 32; ++i) v[i] = fast_silu(v[i]);
                store_f16x32(static_cast<__half*>(e.out) + orow * e.ldo + col, v, valid);
            } else if constexpr (KIND == EPI_RESID) {
                float o[32];
                if (valid >= 32) {
                    const float* rc = reinterpret_cast<const float*>(rcur);
#pragma unroll
                    for (int i = 0; i < 32; ++i) o[i] = __fadd_rn(rc[i], v[i]);
                } else {
                    const float* rs = e.resid + orow * e.ldo + col;
                    for (int i = 0; i < valid; ++i) o[i] = __fadd_rn(rs[i], v[i]);
                }
                store_f32x32(static_cast<float*>(e.out) + orow * e.ldo + col, o, valid);
            }
        }
    }
}

template <int KIND>
__global__ void __launch_bounds__(THREADS, 1)
    tc_gemm_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                   const GemmArgs g, int* err) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* tiles = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    Smem* sm = reinterpret_cast<Smem*>(tiles + STAGES * STAGE_BYTES);
    volatile int* abort = &sm->abort;

    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    const int m_tiles = (g.M + BM - 1) / BM, n_tiles = (g.N + BN - 1) / BN;
    const int num_tiles = m_tiles * n_tiles;
    const int k_blocks = (g.K + BK - 1) / BK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) { mbar_init(&sm->full[s], 1); mbar_init(&sm->empty[s], 1); }
        for (int b = 0; b < 2; ++b) { mbar_init(&sm->acc_full[b], 1); mbar_init(&sm->acc_empty[b], EPI_WARPS); }
        sm->abort = 0;
        mbar_fence_init();
        fence_proxy_async();
    }
    if (warp == 0 && lane == 0) { tma_prefetch_desc(&map_a); tma_prefetch_desc(&map_b); }
    if (warp == 1) { tmem_alloc(&sm->tmem_base, TMEM_COLS); tmem_relinquish(); }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = sm->tmem_base;

    if (warp == 0) {
        if (lane == 0) {
            uint32_t it = 0;
            for (int tile = blockIdx.x; tile < num_tiles && !*abort; tile += gridDim.x) {
                const int m0 = (tile / n_tiles) * BM, n0 = (tile % n_tiles) * BN;
                for (int kb = 0; kb < k_blocks; ++kb, ++it) {
                    const int s = it % STAGES;
                    const uint32_t ph = (it / STAGES) & 1;
                    if (!wait_or_abort(&sm->empty[s], ph ^ 1, abort, err, kDevTimeoutEmpty)) break;
                    uint8_t* a = tiles + s * STAGE_BYTES;
                    mbar_arrive_expect_tx(&sm->full[s], STAGE_BYTES);
                    tma_load_2d(a, &map_a, &sm->full[s], kb * BK, m0);
                    tma_load_2d(a + A_BYTES, &map_b, &sm->full[s], kb * BK, n0);
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            uint32_t it = 0, acc = 0;
            const uint32_t idesc = idesc_f16(BM, BN);
            for (int tile = blockIdx.x; tile < num_tiles && !*abort; tile += gridDim.x, ++acc) {
                const int b = acc & 1;
                const uint32_t aph = (acc >> 1) & 1;
                if (!wait_or_abort(&sm->acc_empty[b], aph ^ 1, abort, err, kDevTimeoutAccEmpty)) break;
                tc_fence_after();
                const uint32_t d = tmem + b * BN;
                bool ok = true;
                for (int kb = 0; kb < k_blocks; ++kb, ++it) {
                    const int s = it % STAGES;
                    const uint32_t ph = (it / STAGES) & 1;
                    if (!wait_or_abort(&sm->full[s], ph, abort, err, kDevTimeoutFull)) { ok = false; break; }
                    tc_fence_after();
                    const uint32_t a_addr = smem_u32(tiles + s * STAGE_BYTES);
                    const uint64_t adesc = smem_desc_sw128(a_addr), bdesc = smem_desc_sw128(a_addr + A_BYTES);
#pragma unroll
                    for (int k = 0; k < BK / 16; ++k)
                        mma_f16(d, adesc + uint64_t(2 * k), bdesc + uint64_t(2 * k), idesc, (kb | k) != 0);
                    mma_commit(&sm->empty[s]);
                }
                if (!ok) break;
                mma_commit(&sm->acc_full[b]);
            }
        }
    } else {
        const int quarter = warp & 3;         // TMEM lanes this warp may read
        const int half = (warp - 2) / 4;      // column half of the tile
        uint32_t acc = 0;
        for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++acc) {
            const int b = acc & 1;
            const uint32_t aph = (acc >> 1) & 1;
            bool ok = true;
            if (lane == 0) ok = wait_or_abort(&sm->acc_full[b], aph, abort, err, kDevTimeoutAccFull);
            ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
            if (!ok) break;
            __syncwarp();
            tc_fence_after();
            const int m0 = (tile / n_tiles) * BM, n0 = (tile % n_tiles) * BN;
            const uint32_t tacc = tmem + (uint32_t(quarter * 32) << 16) + b * BN;
            epilogue_tile<KIND>(g, tacc, m0, n0, quarter * 32 + lane, half);
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&sm->acc_empty[b]);
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) tmem_dealloc(tmem, TMEM_COLS);
}

// --- host side ---------------------------------------------------------------------------
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    });
    return fn;
}

}  // namespace

// 2D f16 tensor map over a row-major [rows][cols] matrix with row pitch `ld` elements,
// box {64 columns, box_rows rows}, 128-byte swizzle, zero fill out of bounds.
bool make_map_2d_f16(CUtensorMap* map, const void* base, int64_t rows, int64_t cols, int64_t ld, int box_rows) {
    auto fn = encode_fn();
    if (!fn) return false;
    cuuint64_t dims[2] = {cuuint64_t(cols), cuuint64_t(rows)};
    cuuint64_t strides[1] = {cuuint64_t(ld) * 2};
    cuuint32_t box[2] = {64, cuuint32_t(box_rows)};
    cuuint32_t estr[2] = {1, 1};
    return fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// 3D f16 tensor map over [planes][rows][64] (head-major q/k/v), box {64, box_rows, 1}.
bool make_map_3d_f16(CUtensorMap* map, const void* base, int64_t planes, int64_t rows, int box_rows) {
    auto fn = encode_fn();
    if (!fn) return false;
    cuuint64_t dims[3] = {64, cuuint64_t(rows), cuuint64_t(planes)};
    cuuint64_t strides[2] = {64 * 2, cuuint64_t(rows) * 64 * 2};
    cuuint32_t box[3] = {64, cuuint32_t(box_rows), 1};
    cuuint32_t estr[3] = {1, 1, 1};
    return fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int device_sm_count() {
    static int counts[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return 148;
    if (!counts[dev]) {
        int n = 0;
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        counts[dev] = n > 0 ? n : 148;
    }
    return counts[dev];
}

template <int KIND>
static cudaError_t launch(const GemmArgs& a, cudaStream_t stream, int* err) {
    static bool configured[64] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && !configured[dev]) {
        cudaError_t e = cudaFuncSetAttribute(tc_gemm_kernel<KIND>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
        if (e != cudaSuccess) return e;
        configured[dev] = true;
    }
    CUtensorMap ma, mb;
    if (!make_map_2d_f16(&ma, a.A, a.M, a.K, a.lda, BM) || !make_map_2d_f16(&mb, a.B, a.N, a.K, a.ldb, BN))
        return cudaErrorInvalidValue;
    const int tiles = ((a.M + BM - 1) / BM) * ((a.N + BN - 1) / BN);
    const int grid = tiles < device_sm_count() ? tiles : device_sm_count();
    tc_gemm_kernel<KIND><<<grid, THREADS, SMEM_BYTES, stream>>>(ma, mb, a, err);
    return cudaGetLastError();
}

cudaError_t tc_gemm(EpiKind kind, const GemmArgs& a, cudaStream_t stream, int* err) {
    if (a.M <= 0 || a.N <= 0 || a.K <= 0) return cudaSuccess;
    // TMA: 16-byte aligned base and row pitch.
    if ((reinterpret_cast<uintptr_t>(a.A) & 15) || (reinterpret_cast<uintptr_t>(a.B) & 15) || (a.lda * 2) % 16 ||
        (a.ldb * 2) % 16 || a.N % 16)
        return cudaErrorInvalidValue;
    if ((kind == EPI_SWIGLU || kind == EPI_VGATE) && a.N % BN) return cudaErrorInvalidValue;
    if (kind == EPI_QKVG && (a.epi.D % 64 || a.N % 64 || a.epi.S <= 0)) return cudaErrorInvalidValue;
    switch (kind) {
        case EPI_F32: return launch<EPI_F32>(a, stream, err);
        case EPI_F16: return launch<EPI_F16>(a, stream, err);
        case EPI_RESID: return launch<EPI_RESID>(a, stream, err);
        case EPI_SILU: return launch<EPI_SILU>(a, stream, err);
        case EPI_SWIGLU: return launch<EPI_SWIGLU>(a, stream, err);
        case EPI_VGATE: return launch<EPI_VGATE>(a, stream, err);
        case EPI_QKVG: return launch<EPI_QKVG>(a, stream, err);
    }
    return cudaErrorInvalidValue;
}

}  // namespace tsb
