// Persistent tcgen05 GEMM for sm_100a with fused epilogues, on CTA pairs.
//
// Replaces the reference's projection nodes (src/layers.cpp:250-256 affine, 682-687 swiglu,
// src/head.cpp:275-286 head/patch projections, src/weight_policy.hpp:23-30 reduced
// projection), which on the reference's F16/Q8_0 path round activations to F16 and
// accumulate F16 products in F32 — the same arithmetic as kind::f16 with f32 accumulators.
//
// Two CTAs of a cluster compute one 256 x 256 tile with tcgen05.mma.cta_group::2: CTA r holds
// rows [128 r, 128 r + 128) of the A tile and rows [128 r, 128 r + 128) of the B tile (the
// tile's columns) in its shared memory, and its TMEM receives the accumulator rows of its A
// half over all 256 columns. Each SM thus streams 32 KB per 64-deep K step instead of the
// 48 KB a single-CTA 128 x 256 tile needs, which is what lets the tensor pipe run near its
// peak on shared-memory bandwidth. No load uses multicast.
//
// Per CTA: warp 0 lane 0 loads both operand halves (CTA 0 also expects the pair's
// transaction bytes on its full barrier); warp 1 owns the TMEM (two 256-column accumulators)
// and, in CTA 0, issues the MMAs and commits to both CTAs' barriers; warps 2.. are the
// epilogue (TMEM lane quarter = warp % 4, column group = (warp - 2) / 4), and release an
// accumulator by arriving on CTA 0's accumulator-empty barrier.
// Every mbarrier wait is bounded; a timeout records a device error and unwinds.
#include "common.cuh"
#include "gemm_tc.cuh"

#include <cstdio>
#include <mutex>

namespace tsb {

namespace {

constexpr int BM = 128;                       // accumulator rows per CTA (256 per pair)
constexpr int BK = 64;
constexpr int BN = 256;                       // tile columns
constexpr int BN_HALF = BN / 2;               // B rows held by each CTA
constexpr int A_BYTES = BM * BK * 2;          // 16 KB
constexpr int B_BYTES = BN_HALF * BK * 2;     // 16 KB
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int TMEM_COLS = 2 * BN;             // 512: two accumulators
// Q8_0 prologue: each stage also holds the CTA's int8 weight tile (128 rows x 64) and the
// f16 scales of its two 32-value blocks (2 x 128), which the converter warps turn into the
// f16 B tile of the same stage.
constexpr int BQ_BYTES = BN_HALF * BK;        // 8 KB
constexpr int BD_BYTES = 2 * BN_HALF * 2;     // 512 B
constexpr int Q8_STAGE_BYTES = STAGE_BYTES + BQ_BYTES + 1024;   // scales padded: stages stay 1 KB aligned
// K-quant prologue (scaled int8): the same int8 tile plus, per 16 values, an f32 scale and
// offset for each of the 128 rows: 4 groups x 128 float2 = 4 KB.
constexpr int BS_BYTES = (BK / 16) * BN_HALF * 8;
constexpr int KQ_STAGE_BYTES = STAGE_BYTES + BQ_BYTES + BS_BYTES;
// Weight formats of the B operand: f16, Q8_0 (int8 + f16 scale per 32 values), scaled int8
// (int8 + f32 scale and offset per 16 values: the K-quants, and Q8_0 as well).
enum WeightFmt : int { FMT_F16 = 0, FMT_Q8 = 1, FMT_KQ = 2 };
constexpr int CONV_WARPS = 2;                 // 384 threads with the 8 epilogue warps: no spills

// Per epilogue kind: PARTS column groups per TMEM lane quarter (epilogue warps = 4 * PARTS).
// The q/k/v/gate epilogue (RoPE tables in registers) and the residual add (residual rows in
// registers; bound by its residual traffic or by a long K) run two groups of 128 columns;
// the activation and plain-store epilogues run four groups of 64, which doubles the warps
// that hide the epilogue's latency at 96 registers a thread; their staging blocks leave room
// for five operand stages instead of six.
// FMT != FMT_F16: the dequantising-prologue variants, which add CONV_WARPS converter warps
// after the epilogue warps, use two column groups for every epilogue kind (register budget)
// and four stages.
template <int KIND, int FMT = FMT_F16, bool RING_OK = true>
struct Cfg {
    static constexpr bool Q8 = FMT != FMT_F16;
    static constexpr int PARTS = (Q8 || KIND == EPI_QKVG || KIND == EPI_RESID) ? 2 : 4;
    static constexpr int EPI_WARPS = 4 * PARTS;
    static constexpr int THREADS = 64 + 32 * EPI_WARPS + (Q8 ? 32 * CONV_WARPS : 0);
    static constexpr int STAGE = FMT == FMT_Q8 ? Q8_STAGE_BYTES : FMT == FMT_KQ ? KQ_STAGE_BYTES : STAGE_BYTES;
    // The residual add (F16 weights) prefetches its residual rows into a ring of two
    // transposition blocks per warp (see resid_prefetch), for one operand stage less.
    static constexpr bool RING = RING_OK && KIND == EPI_RESID && !Q8;
    static constexpr int STAGES = Q8 ? 4 : RING ? 5 : PARTS == 2 ? 6 : 5;
    static constexpr int EPI_STAGE_BYTES = EPI_WARPS * 32 * 128 * (RING ? 2 : 1);   // per-warp transposition blocks
    static constexpr int SMEM_BYTES = STAGES * STAGE + EPI_STAGE_BYTES + 1024 /*align*/ + 512 /*barriers*/;
    static_assert(SMEM_BYTES <= 227 * 1024, "shared memory");
    static_assert(!RING || PARTS == 2, "the residual ring holds two column groups");
};

template <int STAGES>
struct Smem {
    uint64_t full[STAGES];
    uint64_t empty[STAGES];
    uint64_t acc_full[2];
    uint64_t acc_empty[2];
    uint64_t bfull[STAGES];   // Q8: this CTA's int8 tile and scales arrived
    uint64_t conv[STAGES];    // Q8 (CTA 0): both CTAs' f16 tiles written
    uint32_t tmem_base;
    int abort;
};
static_assert(sizeof(Smem<6>) <= 512, "barrier block");

// Four signed int8 values (one word, value k in byte k) times the f16 scale pair d2: two
// half2 words (values 0,1 and 2,3). Each byte b becomes the f16 1024 + (b + 128) by placing it
// under the exponent 0x64, so subtracting 1152 gives b exactly; one f16 multiply then rounds
// b * d once, as rounding the exact product at load does.
__device__ __forceinline__ void dequant4(uint32_t w, __half2 d2, uint32_t& lo, uint32_t& hi) {
    const uint32_t u = w ^ 0x80808080u;
    const uint32_t p0 = __byte_perm(u, 0x64646464u, 0x5140);
    const uint32_t p1 = __byte_perm(u, 0x64646464u, 0x5342);
    const __half2 bias = __halves2half2(__ushort_as_half(0x6480), __ushort_as_half(0x6480));   // 1152
    __half2 a = __hmul2(__hsub2(*reinterpret_cast<const __half2*>(&p0), bias), d2);
    __half2 b = __hmul2(__hsub2(*reinterpret_cast<const __half2*>(&p1), bias), d2);
    lo = *reinterpret_cast<uint32_t*>(&a);
    hi = *reinterpret_cast<uint32_t*>(&b);
}

template <bool CLUSTER = false>
__device__ __forceinline__ bool try_wait_scoped(uint64_t* bar, uint32_t parity) {
    return CLUSTER ? mbar_try_wait_cluster(bar, parity) : mbar_try_wait(bar, parity);
}

template <bool CLUSTER = false>
__device__ __forceinline__ bool wait_or_abort(uint64_t* bar, uint32_t parity, volatile int* abort, int* err, int code) {
    if (try_wait_scoped<CLUSTER>(bar, parity)) return true;
    const long long start = clock64();
    while (true) {
        if (*abort) return false;
        if (try_wait_scoped<CLUSTER>(bar, parity)) return true;
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

// Activations of the tensor-core path. Their results are rounded to f16 for the next
// GEMM, so they use the hardware exp2 and approximate divide (a few ulp in f32, far below
// the f16 rounding) instead of the reference's exact float sequence used on the F32 path.
__device__ __forceinline__ float fast_sigmoid(float x) { return __fdividef(1.0f, 1.0f + __expf(-x)); }
__device__ __forceinline__ float fast_silu(float x) { return __fdividef(x, 1.0f + __expf(-x)); }

// A row read by accumulator row m (GemmArgs::a_group).
__device__ __forceinline__ int64_t a_row(const GemmArgs& g, int m) {
    if (g.a_group <= 0) return m;
    return int64_t(m / g.a_group) * g.a_stride + g.a_offset + (m % g.a_group);
}

// 1/rms of A row `row` when the A operand is x / 16 and the norm is carried by the GEMM (see
// GemmEpilogue::ssq_in); 1 otherwise. The slot sums are added in slot order.
__device__ __forceinline__ float row_scale(const GemmEpilogue& e, int64_t row, bool row_ok) {
    if (!e.ssq_in || !row_ok) return 1.0f;
    const float* p = e.ssq_in + row * e.ssq_slots;
    float sum = 0.f;
    for (int j = 0; j < e.ssq_slots; ++j) sum = __fadd_rn(sum, p[j]);
    const float mean = __fdiv_rn(sum, float(e.rms_D));
    const float rms = __fsqrt_rn(__fadd_rn(mean, e.rms_eps));
    if (!(rms >= 0.00390625f) && e.norm_flag) atomicOr(e.norm_flag, 1);
    return __fdiv_rn(16.0f, rms);
}

// Per-warp staging block of the epilogue: 32 accumulator rows x 128 bytes. A thread writes
// its own row (the TMEM lane it read) and the warp then reads the block back so that eight
// threads cover one 128-byte row, four rows per instruction: every global load and store of
// the epilogue touches 4 full cache lines per instruction instead of 32 partial ones. The
// 16-byte chunk index is XORed with the row's low three bits, which keeps both the row
// writes and the transposed reads free of bank conflicts.
constexpr int STAGE_ROW_BYTES = 128;

__device__ __forceinline__ void stage_row(uint8_t* buf, int lane, const uint32_t (&w)[32]) {
#pragma unroll
    for (int j = 0; j < 8; ++j)
        *reinterpret_cast<uint4*>(buf + lane * STAGE_ROW_BYTES + ((j ^ (lane & 7)) << 4)) =
            make_uint4(w[4 * j], w[4 * j + 1], w[4 * j + 2], w[4 * j + 3]);
}
// Chunk (lane % 8) of staged row i * 4 + lane / 8.
__device__ __forceinline__ uint4 unstage(const uint8_t* buf, int i, int lane) {
    const int row = i * 4 + (lane >> 3), chunk = lane & 7;
    return *reinterpret_cast<const uint4*>(buf + row * STAGE_ROW_BYTES + ((chunk ^ (row & 7)) << 4));
}
__device__ __forceinline__ float4 f4(uint4 u) {
    return make_float4(__uint_as_float(u.x), __uint_as_float(u.y), __uint_as_float(u.z), __uint_as_float(u.w));
}
__device__ __forceinline__ float4 add4(float4 a, float4 b) {
    return make_float4(__fadd_rn(a.x, b.x), __fadd_rn(a.y, b.y), __fadd_rn(a.z, b.z), __fadd_rn(a.w, b.w));
}
__device__ __forceinline__ void pack32(const float* v, uint32_t* w) {
#pragma unroll
    for (int i = 0; i < 16; ++i) w[i] = pack_half2(v[2 * i], v[2 * i + 1]);
}

// Epilogue of one 128 x BN accumulator for one warp: accumulator rows [mw, mw + 32) (its
// TMEM lane quarter) and column group `part` of PARTS.
// RoPE table entries of the q/k/v/gate epilogue for the row this lane reads from TMEM:
// with rope_half <= 16 and tables whose two halves are equal (cos[d] == cos[d + 32], as for
// emb = [freqs, freqs]) only dims 0..15 of cos and sin are needed, fetched once for both
// heads of the column group. Loaded before the accumulator is ready (two dependent global
// loads: the row's table index, then its entries).
struct RopeRow {
    bool on = false;
    float4 tcs[8];
};
__device__ __forceinline__ void load_rope_row(const GemmArgs& g, int m, int first, RopeRow& rr) {
    const GemmEpilogue& e = g.epi;
    rr.on = e.rope && e.rope_dup && e.rope_half <= 16 && m < g.M && first / e.D < 2;
    if (!rr.on) return;
    const int64_t row = e.rope_row[m];
    const float4* ct = reinterpret_cast<const float4*>(e.cos_tab + row * 64);
    const float4* st = reinterpret_cast<const float4*>(e.sin_tab + row * 64);
#pragma unroll
    for (int j = 0; j < 4; ++j) { rr.tcs[j] = ct[j]; rr.tcs[4 + j] = st[j]; }
}

// Residual-add epilogue, norm carried by the GEMMs: the per-row sums of squares of one
// 128-column slot (each row's eight column quads are held by the eight lanes sharing
// lane / 8) into ssq; every |x| <= 2^20 (x / 16 fits f16) whenever a slot's sum of squares
// is at most 2^40, and a larger sum (rarely a false alarm) sends the forecast to the fallback.
__device__ __forceinline__ void store_ssq(const GemmEpilogue& e, const int (&orow)[8], const bool (&rok)[8], float (&sq)[8],
                                          int lane, int slot) {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
#pragma unroll
        for (int o = 1; o < 8; o <<= 1) sq[i] = __fadd_rn(sq[i], __shfl_xor_sync(0xffffffffu, sq[i], o));
    }
    bool over = false;
#pragma unroll
    for (int i = 0; i < 8; ++i) over |= !(sq[i] <= 1099511627776.0f);
    if ((lane & 7) == 0) {
#pragma unroll
        for (int i = 0; i < 8; ++i)
            if (rok[i]) e.ssq[int64_t(orow[i]) * e.ssq_slots + slot] = sq[i];
    }
    if (__any_sync(0xffffffffu, over && (lane & 7) == 0) && lane == 0 && e.norm_flag) atomicOr(e.norm_flag, 1);
}

template <int KIND, int PARTS>
__device__ __forceinline__ void epilogue_tile(const GemmArgs& g, uint32_t tacc, int m0, int n0, int quarter, int lane,
                                              int part, uint8_t* buf, float rsc, const RopeRow& rr) {
    const int half = part;
    const GemmEpilogue& e = g.epi;
    const int mw = m0 + quarter * 32;
    // Rows this thread stores after the transpose: mw + i * 4 + lane / 8, i = 0..7.
    int orow[8];
    bool rok[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int m = mw + i * 4 + (lane >> 3);
        rok[i] = m < g.M;
        orow[i] = rok[i] ? int(out_row(e, m)) : 0;
    }
    uint32_t w[32];
    if constexpr (KIND == EPI_F32 || KIND == EPI_RESID) {
        // 32 f32 columns per staging pass; the thread stores columns col .. col + 3.
        constexpr int C = BN / PARTS / 32;
        // Residual rows: with two column groups the next chunk's rows are requested while the
        // current chunk is stored; with four, each chunk's rows are requested ahead of its
        // TMEM read (the doubled warp count covers the latency, and registers are fewer).
        constexpr int RB = PARTS == 2 ? 2 : 1;
        float4 rs[RB][8];
        auto load_resid = [&](int c, float4 (&dst)[8]) {
            const int col = n0 + (half * C + c) * 32 + (lane & 7) * 4;
#pragma unroll
            for (int i = 0; i < 8; ++i)
                if (rok[i] && col < g.N) dst[i] = *reinterpret_cast<const float4*>(e.resid + int64_t(orow[i]) * e.ldo + col);
        };
        if constexpr (KIND == EPI_RESID && RB == 2) load_resid(0, rs[0]);
        float sq[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) sq[i] = 0.f;
#pragma unroll
        for (int c = 0; c < C; ++c) {
            if constexpr (KIND == EPI_RESID) {
                if constexpr (RB == 2) {
                    if (c + 1 < C) load_resid(c + 1, rs[(c + 1) & 1]);
                } else {
                    load_resid(c, rs[0]);
                }
            }
            tmem_ld32(tacc + (half * C + c) * 32, w);
            tmem_ld_wait();
            stage_row(buf, lane, w);
            __syncwarp();
            const int col = n0 + (half * C + c) * 32 + (lane & 7) * 4;
            if (col < g.N) {
                const float4 b = e.bias ? *reinterpret_cast<const float4*>(e.bias + col) : make_float4(0, 0, 0, 0);
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    if (!rok[i]) continue;
                    float4 v = f4(unstage(buf, i, lane));
                    if (e.bias) v = add4(v, b);
                    if constexpr (KIND == EPI_RESID) v = add4(rs[c % RB][i], v);
                    *reinterpret_cast<float4*>(static_cast<float*>(e.out) + int64_t(orow[i]) * e.ldo + col) = v;
                    if constexpr (KIND == EPI_RESID) {
                        if (e.x16) {
                            sq[i] = fmaf(v.w, v.w, fmaf(v.z, v.z, fmaf(v.y, v.y, fmaf(v.x, v.x, sq[i]))));
                            uint2 h;
                            h.x = pack_half2(v.x * 0.0625f, v.y * 0.0625f);
                            h.y = pack_half2(v.z * 0.0625f, v.w * 0.0625f);
                            *reinterpret_cast<uint2*>(e.x16 + int64_t(orow[i]) * e.ldx16 + col) = h;
                        }
                    }
                }
            }
            __syncwarp();
        }
        if constexpr (KIND == EPI_RESID) {
            // a column group past N (N = 128 in a 256-column tile) has no slot of its own
            if (e.x16 && n0 + half * C * 32 < g.N) store_ssq(e, orow, rok, sq, lane, (n0 + half * C * 32) / 128);
        }
    } else if constexpr (KIND == EPI_F16 || KIND == EPI_SILU) {
        // 64 columns (two TMEM reads) per staging pass; the thread stores 8 f16 columns.
        constexpr int C = BN / PARTS / 64;
#pragma unroll
        for (int c = 0; c < C; ++c) {
            const int cb = n0 + (half * C + c) * 64;
            float v[64];
            tmem_ld32(tacc + (half * C + c) * 64, w);
            tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(w[i]);
            tmem_ld32(tacc + (half * C + c) * 64 + 32, w);
            tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < 32; ++i) v[32 + i] = __uint_as_float(w[i]);
            if (e.ssq_in) {
#pragma unroll
                for (int i = 0; i < 64; ++i) v[i] = __fmul_rn(v[i], rsc);
            }
            if (e.bias) {
#pragma unroll
                for (int i = 0; i < 64; ++i)
                    if (cb + i < g.N) v[i] = __fadd_rn(v[i], e.bias[cb + i]);
            }
            if constexpr (KIND == EPI_SILU) {
#pragma unroll
                for (int i = 0; i < 64; ++i) v[i] = fast_silu(v[i]);
            }
            pack32(v, w);
            pack32(v + 32, w + 16);
            stage_row(buf, lane, w);
            __syncwarp();
            const int col = cb + (lane & 7) * 8;
            if (col < g.N) {
#pragma unroll
                for (int i = 0; i < 8; ++i)
                    if (rok[i]) *reinterpret_cast<uint4*>(static_cast<__half*>(e.out) + int64_t(orow[i]) * e.ldo + col) = unstage(buf, i, lane);
            }
            __syncwarp();
        }
    } else if constexpr (KIND == EPI_SWIGLU || KIND == EPI_VGATE) {
        // The first half of the tile holds the first operand, the second half the second:
        // each 32-column pair gives 32 outputs (64 bytes of a staging row); a group holds C pairs.
        constexpr int C = BN / 2 / PARTS / 32;
#pragma unroll
        for (int c = 0; c < C; ++c) {
            const int cc = half * C + c;
            const int wn = n0 + cc * 32;              // weight row of the first operand's column 0
            uint32_t y[32];
            tmem_ld32(tacc + cc * 32, w);
            tmem_ld32(tacc + BN / 2 + cc * 32, y);
            tmem_ld_wait();
            float o[32];
#pragma unroll
            for (int i = 0; i < 32; ++i) {
                float a = __uint_as_float(w[i]), b = __uint_as_float(y[i]);
                if (e.ssq_in) { a = __fmul_rn(a, rsc); b = __fmul_rn(b, rsc); }
                if (e.bias) { a = __fadd_rn(a, e.bias[wn + i]); b = __fadd_rn(b, e.bias[wn + BN / 2 + i]); }
                o[i] = KIND == EPI_SWIGLU ? __fmul_rn(a, fast_silu(b)) : __fmul_rn(a, fast_sigmoid(b));
            }
            // Row chunk c of the staging row: 16-byte chunks 4c .. 4c + 3.
            uint32_t pk[16];
            pack32(o, pk);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int jj = 4 * c + j;
                *reinterpret_cast<uint4*>(buf + lane * STAGE_ROW_BYTES + ((jj ^ (lane & 7)) << 4)) =
                    make_uint4(pk[4 * j], pk[4 * j + 1], pk[4 * j + 2], pk[4 * j + 3]);
            }
        }
        __syncwarp();
        if constexpr (C == 2) {
            const int col = n0 / 2 + half * 64 + (lane & 7) * 8;
#pragma unroll
            for (int i = 0; i < 8; ++i)
                if (rok[i]) *reinterpret_cast<uint4*>(static_cast<__half*>(e.out) + int64_t(orow[i]) * e.ldo + col) = unstage(buf, i, lane);
        } else {
            // 64-byte rows: four threads per row, eight rows per instruction.
            const int col = n0 / 2 + half * 32 + (lane & 3) * 8;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int row = i * 8 + (lane >> 2), chunk = lane & 3, m = mw + row;
                if (m < g.M)
                    *reinterpret_cast<uint4*>(static_cast<__half*>(e.out) + out_row(e, m) * e.ldo + col) =
                        *reinterpret_cast<const uint4*>(buf + row * STAGE_ROW_BYTES + ((chunk ^ (row & 7)) << 4));
            }
        }
        __syncwarp();
    } else if constexpr (KIND == EPI_QKVG) {
        static_assert(PARTS == 2, "q/k/v/gate groups are 128 columns");
        constexpr int C = BN / 128;
        const int m = mw + lane;                      // the TMEM row of this thread
        const bool row_ok = m < g.M;
        // Head-major row (row * H * S + token) of the rows stored after the transpose.
        int hm[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int mi = mw + i * 4 + (lane >> 3);
            hm[i] = (mi / e.S) * e.H * e.S + mi % e.S;
        }
        // RoPE table entries of this token's position, fetched once for both heads of the
        // half (load_rope_row, done before the accumulator was ready).
        const bool rope16 = rr.on;
        const float4* tcs = rr.tcs;
#pragma unroll 1
        for (int c = 0; c < C; ++c) {
            const int col = n0 + (half * C + c) * 64;
            const int which = col / e.D, h = (col % e.D) >> 6;
            const bool rope = row_ok && col < g.N && which < 2 && e.rope;
            float v[64];
            tmem_ld32(tacc + (half * C + c) * 64, w);
            tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(w[i]);
            tmem_ld32(tacc + (half * C + c) * 64 + 32, w);
            tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < 32; ++i) v[32 + i] = __uint_as_float(w[i]);
            if (col >= g.N) continue;                 // uniform across the warp
            if (e.ssq_in) {
#pragma unroll
                for (int i = 0; i < 64; ++i) v[i] = __fmul_rn(v[i], rsc);
            }
            if (e.bias) {
#pragma unroll
                for (int i = 0; i < 64; ++i) v[i] = __fadd_rn(v[i], e.bias[col + i]);
            }
            if (rope) {
                // x*cos + rotate_half(x)*sin with separately rounded products and sum
                // (reference src/layers.cpp:238-246). Dims whose inverse frequency is zero
                // have cos 1 and sin 0 in every table row and are left unchanged.
                if (rope16) {
                    const float* c0 = reinterpret_cast<const float*>(tcs);       // cos, dims 0..15
                    const float* s0 = reinterpret_cast<const float*>(tcs + 4);   // sin, dims 0..15
#pragma unroll
                    for (int i = 0; i < 16; ++i) {
                        if (i >= e.rope_half) break;
                        const float x0 = v[i], x1 = v[i + 32];
                        v[i] = __fadd_rn(__fmul_rn(x0, c0[i]), __fmul_rn(-x1, s0[i]));
                        v[i + 32] = __fadd_rn(__fmul_rn(x1, c0[i]), __fmul_rn(x0, s0[i]));
                    }
                } else {
                    const float* ct = e.cos_tab + int64_t(e.rope_row[m]) * 64;
                    const float* st = e.sin_tab + int64_t(e.rope_row[m]) * 64;
#pragma unroll
                    for (int i = 0; i < 32; ++i) {
                        if (i >= e.rope_half) break;
                        const float x0 = v[i], x1 = v[i + 32];
                        v[i] = __fadd_rn(__fmul_rn(x0, ct[i]), __fmul_rn(-x1, st[i]));
                        v[i + 32] = __fadd_rn(__fmul_rn(x1, ct[i + 32]), __fmul_rn(x0, st[i + 32]));
                    }
                }
            } else if (which == 3) {
#pragma unroll
                for (int i = 0; i < 64; ++i) v[i] = fast_sigmoid(v[i]);
            }
            pack32(v, w);
            pack32(v + 32, w + 16);
            stage_row(buf, lane, w);
            __syncwarp();
            __half* base = e.qkvg[which] + int64_t(h) * e.S * 64 + (lane & 7) * 8;
#pragma unroll
            for (int i = 0; i < 8; ++i)
                if (rok[i]) *reinterpret_cast<uint4*>(base + int64_t(hm[i]) * 64) = unstage(buf, i, lane);
            __syncwarp();
        }
    }
}

// Sixteen signed int8 values of one row (q) and their group's scale and offset: the f16
// values (a * q) - b, each operation rounded in single precision, then once to f16 (the
// loader's dequantisation). A byte b becomes the float 2^23 + (b + 128) under the exponent
// 0x4B, so subtracting 2^23 + 128 gives b exactly.
__device__ __forceinline__ void dequant16_scaled(const uint4 q, float2 ab, uint32_t (&h)[8]) {
    const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const uint32_t u = w[i] ^ 0x80808080u;
        float v[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const float f = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7540u + uint32_t(k)));
            v[k] = __fsub_rn(__fmul_rn(ab.x, __fsub_rn(f, 8388736.0f)), ab.y);
        }
        h[2 * i] = pack_half2(v[0], v[1]);
        h[2 * i + 1] = pack_half2(v[2], v[3]);
    }
}

// Residual-add epilogue with its residual rows prefetched (F16 weights). An epilogue warp
// works through a fixed sequence of 32-column chunks: for its k-th tile (tile pair + k * pairs
// of the persistent schedule) chunks 4k .. 4k + 3. Chunk q is copied with 16-byte cp.async into
// slot q % 2 of the warp's two transposition blocks, in the transposed layout the stores use
// (thread lane holds rows i * 4 + lane / 8, columns (lane % 8) * 4 .. + 3), two chunks before
// its use and across tile boundaries, so that a chunk's residual latency is covered by the two
// chunks before it without residual registers held across chunks. Every chunk commits one
// copy group (empty past the last tile), so a thread's chunk q has landed once at most one
// younger group is in flight.
struct ResidRing {
    int pair, pairs, num_tiles, n_tiles, rank, quarter, part;
};
constexpr int RING_CHUNKS = BN / 2 / 32;        // chunks per tile and warp (two column groups)
constexpr int RING_SLOT = 32 * STAGE_ROW_BYTES;
// The ring (which costs one of the six operand stages) is used where the epilogue bounds the
// GEMM: short K (the attention out projection, K = D). Long-K residual adds (the MLP down,
// K = 2048) keep six stages and the register prefetch of epilogue_tile.
constexpr int RING_K_MAX = 1024;

__device__ __forceinline__ void resid_prefetch(const GemmArgs& g, const ResidRing& r, int lane, uint32_t q, uint8_t* slot) {
    const GemmEpilogue& e = g.epi;
    const int tile = r.pair + int(q / RING_CHUNKS) * r.pairs, c = int(q % RING_CHUNKS);
    if (tile < r.num_tiles) {
        const int m0 = (tile / r.n_tiles) * 2 * BM + r.rank * BM, n0 = (tile % r.n_tiles) * BN;
        const int col = n0 + (r.part * RING_CHUNKS + c) * 32 + (lane & 7) * 4;
        if (col < g.N) {
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const int row = i * 4 + (lane >> 3), m = m0 + r.quarter * 32 + row;
                if (m < g.M)
                    cp_async16(slot + row * STAGE_ROW_BYTES + (((lane & 7) ^ (row & 7)) << 4),
                               e.resid + out_row(e, m) * e.ldo + col);
            }
        }
    }
    cp_async_commit();
}

// The residual-add epilogue of one tile for one warp (two column groups), chunks q0 .. q0 + 3
// of the warp's sequence; same operations and order as epilogue_tile's.
__device__ __forceinline__ void epilogue_resid_ring(const GemmArgs& g, uint32_t tacc, int m0, int n0, int lane,
                                                    const ResidRing& r, uint8_t* ring, uint32_t q0) {
    const GemmEpilogue& e = g.epi;
    constexpr int C = RING_CHUNKS;
    const int mw = m0 + r.quarter * 32;
    int orow[8];
    bool rok[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int m = mw + i * 4 + (lane >> 3);
        rok[i] = m < g.M;
        orow[i] = rok[i] ? int(out_row(e, m)) : 0;
    }
    float sq[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) sq[i] = 0.f;
    uint32_t w[32];
#pragma unroll
    for (int c = 0; c < C; ++c) {
        uint8_t* slot = ring + ((q0 + c) & 1) * RING_SLOT;
        tmem_ld32(tacc + (r.part * C + c) * 32, w);
        cp_async_wait<1>();
        float4 rs[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) rs[i] = f4(unstage(slot, i, lane));
        tmem_ld_wait();
        __syncwarp();
        stage_row(slot, lane, w);
        __syncwarp();
        const int col = n0 + (r.part * C + c) * 32 + (lane & 7) * 4;
        if (col < g.N) {
            const float4 b = e.bias ? *reinterpret_cast<const float4*>(e.bias + col) : make_float4(0, 0, 0, 0);
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                if (!rok[i]) continue;
                float4 v = f4(unstage(slot, i, lane));
                if (e.bias) v = add4(v, b);
                v = add4(rs[i], v);
                *reinterpret_cast<float4*>(static_cast<float*>(e.out) + int64_t(orow[i]) * e.ldo + col) = v;
                if (e.x16) {
                    sq[i] = fmaf(v.w, v.w, fmaf(v.z, v.z, fmaf(v.y, v.y, fmaf(v.x, v.x, sq[i]))));
                    uint2 h;
                    h.x = pack_half2(v.x * 0.0625f, v.y * 0.0625f);
                    h.y = pack_half2(v.z * 0.0625f, v.w * 0.0625f);
                    *reinterpret_cast<uint2*>(e.x16 + int64_t(orow[i]) * e.ldx16 + col) = h;
                }
            }
        }
        __syncwarp();
        resid_prefetch(g, r, lane, q0 + c + 2, slot);
    }
    if (e.x16 && n0 + r.part * C * 32 < g.N) store_ssq(e, orow, rok, sq, lane, (n0 + r.part * C * 32) / 128);
}

template <int KIND, int FMT, bool RING_OK>
__global__ void __launch_bounds__(Cfg<KIND, FMT, RING_OK>::THREADS, 1)
    tc_gemm_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                   const __grid_constant__ CUtensorMap map_bq, const __grid_constant__ CUtensorMap map_bd,
                   const GemmArgs g, int* err) {
    using CF = Cfg<KIND, FMT, RING_OK>;
    constexpr bool Q8 = CF::Q8;
    constexpr int STAGES = CF::STAGES, EPI_WARPS = CF::EPI_WARPS, PARTS = CF::PARTS, SB = CF::STAGE;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* tiles = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* stage = tiles + STAGES * SB;
    Smem<STAGES>* sm = reinterpret_cast<Smem<STAGES>*>(stage + CF::EPI_STAGE_BYTES);
    volatile int* abort = &sm->abort;

    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    const uint32_t rank = cluster_ctarank();          // 0: issues the MMAs
    const int pair = blockIdx.x / 2, pairs = gridDim.x / 2;
    const int m_tiles = (g.M + 2 * BM - 1) / (2 * BM), n_tiles = (g.N + BN - 1) / BN;
    const int num_tiles = m_tiles * n_tiles;
    const int k_blocks = (g.K + BK - 1) / BK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&sm->full[s], 1); mbar_init(&sm->empty[s], 1);
            mbar_init(&sm->bfull[s], 1); mbar_init(&sm->conv[s], 2 * CONV_WARPS);
        }
        for (int b = 0; b < 2; ++b) { mbar_init(&sm->acc_full[b], 1); mbar_init(&sm->acc_empty[b], 2 * EPI_WARPS); }
        sm->abort = 0;
        mbar_fence_init();
        fence_proxy_async();
    }
    if (warp == 0 && lane == 0) {
        tma_prefetch_desc(&map_a);
        if constexpr (Q8) { tma_prefetch_desc(&map_bq); tma_prefetch_desc(&map_bd); }
        else tma_prefetch_desc(&map_b);
    }
    if (warp == 1) { tmem_alloc_pair(&sm->tmem_base, TMEM_COLS); tmem_relinquish_pair(); }
    tc_fence_before();
    cluster_sync();                                   // barriers of both CTAs initialised
    tc_fence_after();
    const uint32_t tmem = sm->tmem_base;

    if (warp == 0) {
        if (lane == 0) {
            uint32_t it = 0;
            for (int tile = pair; tile < num_tiles && !*abort; tile += pairs) {
                const int m0 = (tile / n_tiles) * 2 * BM + int(rank) * BM;
                const int n0 = (tile % n_tiles) * BN + int(rank) * BN_HALF;
                for (int kb = 0; kb < k_blocks; ++kb, ++it) {
                    const int s = it % STAGES;
                    const uint32_t ph = (it / STAGES) & 1;
                    if (!wait_or_abort(&sm->empty[s], ph ^ 1, abort, err, kDevTimeoutEmpty)) break;
                    uint8_t* a = tiles + s * SB;
                    if (rank == 0) mbar_arrive_expect_tx(&sm->full[s], Q8 ? 2 * A_BYTES : 2 * STAGE_BYTES);
                    const uint32_t full0 = mapa_shared(smem_u32(&sm->full[s]), 0);
                    if (g.a_group > 0) tma_load_3d_pair(a, &map_a, full0, kb * BK, 0, m0 / g.a_group);
                    else tma_load_2d_pair(a, &map_a, full0, kb * BK, m0);
                    if constexpr (Q8) {
                        // This CTA's int8 rows and their scales, on its own barrier (its converter
                        // warps wait for them); the f16 tile is written by those warps.
                        uint8_t* bq = a + STAGE_BYTES;
                        mbar_arrive_expect_tx(&sm->bfull[s], BQ_BYTES + (FMT == FMT_Q8 ? BD_BYTES : BS_BYTES));
                        tma_load_2d(bq, &map_bq, &sm->bfull[s], kb * BK, n0);
                        if constexpr (FMT == FMT_Q8) tma_load_2d(bq + BQ_BYTES, &map_bd, &sm->bfull[s], n0, kb * (BK / 32));
                        else tma_load_2d(bq + BQ_BYTES, &map_bd, &sm->bfull[s], 2 * n0, kb * (BK / 16));
                    } else {
                        tma_load_2d_pair(a + A_BYTES, &map_b, full0, kb * BK, n0);
                    }
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0 && rank == 0) {
            uint32_t it = 0, acc = 0;
            const uint32_t idesc = idesc_f16(2 * BM, BN);
            for (int tile = pair; tile < num_tiles && !*abort; tile += pairs, ++acc) {
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
                    if constexpr (Q8) {
                        if (!wait_or_abort<true>(&sm->conv[s], ph, abort, err, kDevTimeoutConv)) { ok = false; break; }
                    }
                    tc_fence_after();
                    const uint32_t a_addr = smem_u32(tiles + s * SB);
                    const uint64_t adesc = smem_desc_sw128(a_addr), bdesc = smem_desc_sw128(a_addr + A_BYTES);
#pragma unroll
                    for (int k = 0; k < BK / 16; ++k)
                        mma_f16_pair(d, adesc + uint64_t(2 * k), bdesc + uint64_t(2 * k), idesc, (kb | k) != 0);
                    mma_commit_pair(&sm->empty[s]);
                }
                if (!ok) break;
                mma_commit_pair(&sm->acc_full[b]);
            }
        }
    } else if (Q8 && warp >= 2 + EPI_WARPS) {
        // Converter warps: warp c writes rows [64 c, 64 c + 64) of this CTA's f16 B tile of each
        // stage from its int8 tile. A lane takes 16 values (16 bytes) of one row per step, eight
        // rows per warp step: the int8 reads cover 512 contiguous bytes, and the two 16-byte f16
        // chunks a lane writes land in distinct banks (128-byte swizzle of the tile).
        const int cw = warp - 2 - EPI_WARPS;
        const int c = lane & 3;
        uint32_t it = 0;
        bool ok = true;
        for (int tile = pair; ok && tile < num_tiles; tile += pairs) {
            for (int kb = 0; kb < k_blocks; ++kb, ++it) {
                const int s = it % STAGES;
                const uint32_t ph = (it / STAGES) & 1;
                ok = __all_sync(0xffffffffu, wait_or_abort(&sm->bfull[s], ph, abort, err, kDevTimeoutConv));
                if (!ok) break;
                uint8_t* base = tiles + s * SB;
                const uint8_t* bq = base + STAGE_BYTES;
                const __half* bd = reinterpret_cast<const __half*>(bq + BQ_BYTES);
                uint8_t* bf = base + A_BYTES;
                constexpr int ROWS = BN_HALF / CONV_WARPS;
#pragma unroll 4
                for (int i = 0; i < ROWS / 8; ++i) {
                    const int r = cw * ROWS + i * 8 + (lane >> 2);
                    const uint4 q = *reinterpret_cast<const uint4*>(bq + r * BK + c * 16);
                    uint32_t h[8];
                    if constexpr (FMT == FMT_Q8) {
                        const __half d = bd[(c >> 1) * BN_HALF + r];
                        const __half2 d2 = __halves2half2(d, d);
                        dequant4(q.x, d2, h[0], h[1]);
                        dequant4(q.y, d2, h[2], h[3]);
                        dequant4(q.z, d2, h[4], h[5]);
                        dequant4(q.w, d2, h[6], h[7]);
                    } else {
                        // group c of this K step: row r's scale and offset
                        const float2 ab = reinterpret_cast<const float2*>(bq + BQ_BYTES)[c * BN_HALF + r];
                        dequant16_scaled(q, ab, h);
                    }
                    *reinterpret_cast<uint4*>(bf + r * 128 + (((2 * c) ^ (r & 7)) << 4)) = make_uint4(h[0], h[1], h[2], h[3]);
                    *reinterpret_cast<uint4*>(bf + r * 128 + (((2 * c + 1) ^ (r & 7)) << 4)) = make_uint4(h[4], h[5], h[6], h[7]);
                }
                fence_proxy_async();                  // generic-proxy writes -> tensor-core reads
                __syncwarp();
                if (lane == 0) mbar_arrive_cluster(mapa_shared(smem_u32(&sm->conv[s]), 0));
            }
        }
    } else {
        const int quarter = warp & 3;         // TMEM lanes this warp may read
        const int part = (warp - 2) / 4;      // column group of the tile
        const uint32_t acc_empty0 = mapa_shared(smem_u32(&sm->acc_empty[0]), 0);
        const uint32_t acc_empty1 = mapa_shared(smem_u32(&sm->acc_empty[1]), 0);
        uint32_t acc = 0;
        const ResidRing ring{pair, pairs, num_tiles, n_tiles, int(rank), quarter, part};
        uint8_t* const ring_buf = stage + (warp - 2) * 2 * RING_SLOT;
        if constexpr (CF::RING) {
            resid_prefetch(g, ring, lane, 0, ring_buf);
            resid_prefetch(g, ring, lane, 1, ring_buf + RING_SLOT);
        }
        for (int tile = pair; tile < num_tiles; tile += pairs, ++acc) {
            const int b = acc & 1;
            const uint32_t aph = (acc >> 1) & 1;
            const int m0 = (tile / n_tiles) * 2 * BM + int(rank) * BM, n0 = (tile % n_tiles) * BN;
            // The row's 1/rms (norm carried by the GEMM) and RoPE table entries are read before
            // the accumulator is ready.
            float rsc = 1.0f;
            RopeRow rr;
            if constexpr (KIND != EPI_F32 && KIND != EPI_RESID) {
                const int m = m0 + quarter * 32 + lane;
                rsc = row_scale(g.epi, a_row(g, m), m < g.M);
            }
            if constexpr (KIND == EPI_QKVG) load_rope_row(g, m0 + quarter * 32 + lane, n0 + part * 128, rr);
            bool ok = true;
            if (lane == 0) ok = wait_or_abort(&sm->acc_full[b], aph, abort, err, kDevTimeoutAccFull);
            ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
            if (!ok) break;
            __syncwarp();
            tc_fence_after();
            const uint32_t tacc = tmem + (uint32_t(quarter * 32) << 16) + b * BN;
            if constexpr (CF::RING)
                epilogue_resid_ring(g, tacc, m0, n0, lane, ring, ring_buf, acc * RING_CHUNKS);
            else
                epilogue_tile<KIND, PARTS>(g, tacc, m0, n0, quarter, lane, part, stage + (warp - 2) * 32 * 128, rsc, rr);
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster_relaxed(b ? acc_empty1 : acc_empty0);
        }
        if constexpr (CF::RING) cp_async_wait_all();   // the prefetches past the last tile (or an abort)
    }
    tc_fence_before();
    cluster_sync();                                   // no CTA leaves while its pair may touch it
    tc_fence_after();
    if (warp == 1) tmem_dealloc_pair(tmem, TMEM_COLS);
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

// The bounded waits of the GEMM roles, made to expire without a fault: warp 0 waits on a
// barrier that nothing arrives on, so its wait runs out (it records kDevTimeoutFull and raises
// the abort flag); warp 1 starts waiting on another such barrier half a limit later and
// leaves through the abort flag (err[1] = 1), as the other roles of a GEMM leave when one
// role's wait expires. The kernel then returns; nothing faults and the context stays usable.
__global__ void wait_expiry_kernel(int* err) {
    __shared__ uint64_t bars[2];
    __shared__ int abort_flag;
    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    if (threadIdx.x == 0) {
        mbar_init(&bars[0], 1);
        mbar_init(&bars[1], 1);
        abort_flag = 0;
        mbar_fence_init();
    }
    __syncthreads();
    volatile int* abort = &abort_flag;
    if (lane != 0 || warp > 1) return;
    if (warp == 0) {
        wait_or_abort(&bars[0], 0, abort, err, kDevTimeoutFull);
    } else {
        const long long t0 = clock64();
        while (clock64() - t0 < kWaitCycles / 2) __nanosleep(100000);
        if (!wait_or_abort(&bars[1], 0, abort, nullptr, kDevTimeoutEmpty) && *abort) err[1] = 1;
    }
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

// 3D f16 tensor map of a row gather: groups of `group` consecutive rows, one group every
// `stride` rows of a row-major matrix with pitch `ld` elements; `groups` groups, `cols`
// columns; box {64 columns, group rows, box_groups groups}, 128-byte swizzle (the same
// shared-memory image as the 2D map's box of group * box_groups rows).
bool make_map_gather_f16(CUtensorMap* map, const void* base, int64_t groups, int group, int64_t stride, int64_t cols,
                         int64_t ld, int box_groups) {
    auto fn = encode_fn();
    if (!fn) return false;
    cuuint64_t dims[3] = {cuuint64_t(cols), cuuint64_t(group), cuuint64_t(groups)};
    cuuint64_t strides[2] = {cuuint64_t(ld) * 2, cuuint64_t(stride) * cuuint64_t(ld) * 2};
    cuuint32_t box[3] = {64, cuuint32_t(group), cuuint32_t(box_groups)};
    cuuint32_t estr[3] = {1, 1, 1};
    return fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// 2D tensor map without swizzle over a row-major [rows][cols] matrix of 1- or 2-byte
// elements (pitch `ld_bytes`), box {box_cols, box_rows}: the Q8_0 int8 weight tiles and their
// scale blocks.
bool make_map_2d_plain(CUtensorMap* map, const void* base, CUtensorMapDataType type, int64_t rows, int64_t cols,
                       int64_t ld_bytes, int box_cols, int box_rows) {
    auto fn = encode_fn();
    if (!fn) return false;
    cuuint64_t dims[2] = {cuuint64_t(cols), cuuint64_t(rows)};
    cuuint64_t strides[1] = {cuuint64_t(ld_bytes)};
    cuuint32_t box[2] = {cuuint32_t(box_cols), cuuint32_t(box_rows)};
    cuuint32_t estr[2] = {1, 1};
    return fn(map, type, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
              CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) ==
           CUDA_SUCCESS;
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

// 3D f16 tensor map over head-major [rows][slots][64] (slots = heads x tokens of a row), box
// {64, 1 slot, box_rows rows}: the same (head, token) slot of box_rows consecutive rows, laid
// out in shared memory as box_rows 128-byte rows (the image of a 2D box of box_rows rows).
bool make_map_slot_rows_f16(CUtensorMap* map, const void* base, int64_t rows, int64_t slots, int box_rows) {
    auto fn = encode_fn();
    if (!fn) return false;
    cuuint64_t dims[3] = {64, cuuint64_t(slots), cuuint64_t(rows)};
    cuuint64_t strides[2] = {64 * 2, cuuint64_t(slots) * 64 * 2};
    cuuint32_t box[3] = {64, 1, cuuint32_t(box_rows)};
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

template <int KIND, int FMT, bool RING_OK = true>
static cudaError_t launch(const GemmArgs& a, cudaStream_t stream, int* err) {
    using CF = Cfg<KIND, FMT, RING_OK>;
    static KernelSetup configured;
    int dev = 0;
    cudaGetDevice(&dev);
    unsigned long long ctx_key = 0;
    if (configured.needed(dev, &ctx_key)) {
        cudaError_t e = cudaFuncSetAttribute(tc_gemm_kernel<KIND, FMT, RING_OK>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, CF::SMEM_BYTES);
        if (e != cudaSuccess) return e;
        configured.done(dev, ctx_key);
    }
    CUtensorMap ma, mb, mq, md;
    const bool map_a = a.a_group > 0
        ? make_map_gather_f16(&ma, a.A + int64_t(a.a_offset) * a.lda, (a.M + a.a_group - 1) / a.a_group, a.a_group,
                              a.a_stride, a.K, a.lda, BM / a.a_group)
        : make_map_2d_f16(&ma, a.A, a.M, a.K, a.lda, BM);
    if (!map_a) return cudaErrorInvalidValue;
    if constexpr (FMT == FMT_Q8) {
        if (!make_map_2d_plain(&mq, a.Bq, CU_TENSOR_MAP_DATA_TYPE_UINT8, a.N, a.K, a.ldb, BK, BN_HALF) ||
            !make_map_2d_plain(&md, a.Bd, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, (a.K + 31) / 32, a.N, a.ldd * 2, BN_HALF, BK / 32))
            return cudaErrorInvalidValue;
        mb = mq;                                      // unused by this variant
    } else if constexpr (FMT == FMT_KQ) {
        // scales as f32 [K / 16][2 * lds] (scale, offset of row n at columns 2n, 2n + 1)
        if (!make_map_2d_plain(&mq, a.Bq, CU_TENSOR_MAP_DATA_TYPE_UINT8, a.N, a.K, a.ldb, BK, BN_HALF) ||
            !make_map_2d_plain(&md, a.Bs, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, (a.K + 15) / 16, 2 * a.N, a.lds * 8,
                               2 * BN_HALF, BK / 16))
            return cudaErrorInvalidValue;
        mb = mq;
    } else {
        if (!make_map_2d_f16(&mb, a.B, a.N, a.K, a.ldb, BN_HALF)) return cudaErrorInvalidValue;
        mq = mb; md = mb;                             // unused by this variant
    }
    // One CTA pair (cluster of two) per two SMs, persistent over the 256 x 256 tiles.
    const int tiles = ((a.M + 2 * BM - 1) / (2 * BM)) * ((a.N + BN - 1) / BN);
    const int max_pairs = device_sm_count() / 2;
    const int pairs = tiles < max_pairs ? tiles : max_pairs;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * pairs);
    cfg.blockDim = dim3(CF::THREADS);
    cfg.dynamicSmemBytes = CF::SMEM_BYTES;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, tc_gemm_kernel<KIND, FMT, RING_OK>, ma, mb, mq, md, a, err);
}

template <int KIND>
static cudaError_t launch_kind(const GemmArgs& a, cudaStream_t stream, int* err) {
    if (a.Bq && a.Bs) return launch<KIND, FMT_KQ>(a, stream, err);
    if (a.Bq) return launch<KIND, FMT_Q8>(a, stream, err);
    if constexpr (KIND == EPI_RESID)
        if (a.K > RING_K_MAX) return launch<KIND, FMT_F16, false>(a, stream, err);
    return launch<KIND, FMT_F16>(a, stream, err);
}

cudaError_t tc_gemm(EpiKind kind, const GemmArgs& a, cudaStream_t stream, int* err) {
    if (a.M <= 0 || a.N <= 0 || a.K <= 0) return cudaSuccess;
    // TMA: 16-byte aligned bases and row pitches (f16 B: ldb elements; int8 Bq: ldb bytes;
    // scales Bd: ldd f16 per block row, at least N).
    if ((reinterpret_cast<uintptr_t>(a.A) & 15) || (a.lda * 2) % 16 || a.N % 16) return cudaErrorInvalidValue;
    if (a.Bq && a.Bs) {
        if ((reinterpret_cast<uintptr_t>(a.Bq) & 15) || (reinterpret_cast<uintptr_t>(a.Bs) & 15) || a.ldb % 16 ||
            (a.lds * 8) % 16 || a.lds < a.N || a.K % 16)
            return cudaErrorInvalidValue;
    } else if (a.Bq) {
        if ((reinterpret_cast<uintptr_t>(a.Bq) & 15) || (reinterpret_cast<uintptr_t>(a.Bd) & 15) || a.ldb % 16 ||
            (a.ldd * 2) % 16 || a.ldd < a.N || a.K % 32)
            return cudaErrorInvalidValue;
    } else if ((reinterpret_cast<uintptr_t>(a.B) & 15) || (a.ldb * 2) % 16) {
        return cudaErrorInvalidValue;
    }
    if ((kind == EPI_SWIGLU || kind == EPI_VGATE) && a.N % BN) return cudaErrorInvalidValue;
    // Row gather: whole groups per 128-row box, groups inside the strided rows, 16-byte base.
    if (a.a_group < 0 || (a.a_group > 0 && (BM % a.a_group || a.M % a.a_group || a.a_offset < 0 ||
                                           a.a_offset + a.a_group > a.a_stride ||
                                           (reinterpret_cast<uintptr_t>(a.A + int64_t(a.a_offset) * a.lda) & 15))))
        return cudaErrorInvalidValue;
    if (kind == EPI_QKVG && (a.epi.D % 64 || a.N % 64 || a.epi.S <= 0)) return cudaErrorInvalidValue;
    // The epilogue moves 16-byte vectors: outputs, residuals and f32 biases must be 16-byte
    // aligned with row pitches that keep every row aligned.
    auto misaligned = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) != 0; };
    if (kind == EPI_QKVG) {
        for (int i = 0; i < 4; ++i)
            if (misaligned(a.epi.qkvg[i])) return cudaErrorInvalidValue;
    } else {
        const int64_t elem = (kind == EPI_F32 || kind == EPI_RESID) ? 4 : 2;
        if (misaligned(a.epi.out) || (a.epi.ldo * elem) % 16 || (a.epi.row_group > 0 && (a.epi.row_offset * elem) % 16))
            return cudaErrorInvalidValue;
        if ((kind == EPI_F32 || kind == EPI_RESID) && (misaligned(a.epi.bias) || misaligned(a.epi.resid)))
            return cudaErrorInvalidValue;
    }
    switch (kind) {
        case EPI_F32: return launch_kind<EPI_F32>(a, stream, err);
        case EPI_F16: return launch_kind<EPI_F16>(a, stream, err);
        case EPI_RESID: return launch_kind<EPI_RESID>(a, stream, err);
        case EPI_SILU: return launch_kind<EPI_SILU>(a, stream, err);
        case EPI_SWIGLU: return launch_kind<EPI_SWIGLU>(a, stream, err);
        case EPI_VGATE: return launch_kind<EPI_VGATE>(a, stream, err);
        case EPI_QKVG: return launch_kind<EPI_QKVG>(a, stream, err);
    }
    return cudaErrorInvalidValue;
}

cudaError_t gemm_wait_expiry_selftest(int* err, cudaStream_t stream) {
    wait_expiry_kernel<<<1, 64, 0, stream>>>(err);
    return cudaGetLastError();
}

}  // namespace tsb
