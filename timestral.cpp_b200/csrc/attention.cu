// Attention of the forecast path (reference src/layers.cpp:578-617 sdpa, applied on the time
// axis per row and on the variate axis per patch slot, src/encoder.cpp:125-139).
#include "attention.cuh"
#include "common.cuh"

#include <cstdio>

namespace tsb {

bool make_map_3d_f16(CUtensorMap* map, const void* base, int64_t planes, int64_t rows, int box_rows);
int device_sm_count();

namespace {

__device__ __forceinline__ bool kv_bit(const MaskMeta& mm, int row, int p) {
    return (mm.key_valid[int64_t(row) * mm.kv_words + (p >> 5)] >> (p & 31)) & 1u;
}

__device__ __forceinline__ int anchor_of(const MaskMeta& mm, int p) {
    return p >= mm.L ? mm.L + mm.block_size * ((p - mm.L) / mm.block_size) : 0;
}

// Time-axis mask for query q and key k of row r (reference src/masks.cpp:21-26).
__device__ __forceinline__ bool time_allowed(const MaskMeta& mm, int r, int q, int k) {
    const int N = mm.N;
    if (!mm.cov) {
        if (q < N) return k < N && ((kv_bit(mm, r, k) && k <= q) || q == k);
        if (k < N) return kv_bit(mm, r, k);
        return k <= q;
    }
    if (q < N) return k < N && ((kv_bit(mm, r, k) && (mm.role[r] == 2 || k <= q)) || q == k);
    const int qp = q - N;
    const bool qa = qp >= mm.L;
    if (k < N) return kv_bit(mm, r, k) && qa && k < anchor_of(mm, qp);
    const int kp = k - N;
    return q == k || (k <= q && qa && kp >= mm.L && anchor_of(mm, qp) == anchor_of(mm, kp));
}

// Bits [lo, hi] of a 128-bit set that fall in 32-bit word w.
__device__ __forceinline__ uint32_t bits_in(int w, int lo, int hi) {
    const int a = max(lo, w * 32), b = min(hi, w * 32 + 31);
    if (a > b) return 0u;
    const int la = a - w * 32, lb = b - w * 32;
    const uint32_t upper = lb == 31 ? 0xffffffffu : ((1u << (lb + 1)) - 1u);
    return upper & ~((1u << la) - 1u);
}

// The set of keys (bit k) that query q of row r attends on the time axis, for S <= 128:
// time_allowed() restricted to the keys the reference computes (the encoder split),
// built with word operations from the row's key-valid bits.
__device__ __forceinline__ void key_set(const MaskMeta& mm, int r, int q, bool live, uint32_t (&m)[4]) {
    uint32_t kv[4];
#pragma unroll
    for (int w = 0; w < 4; ++w) {
        kv[w] = w < mm.kv_words ? mm.key_valid[int64_t(r) * mm.kv_words + w] : 0u;
        m[w] = 0u;
    }
    if (!live) return;
    const int N = mm.N;
    if (q < N) {
        const bool full = mm.cov && mm.role[r] == 2;
#pragma unroll
        for (int w = 0; w < 4; ++w) m[w] = (full ? kv[w] : (kv[w] & bits_in(w, 0, q))) | bits_in(w, q, q);
        return;
    }
    if (!mm.cov) {
#pragma unroll
        for (int w = 0; w < 4; ++w) m[w] = kv[w] | bits_in(w, N, q);
        return;
    }
    const int qp = q - N;
    if (qp < mm.L) {
#pragma unroll
        for (int w = 0; w < 4; ++w) m[w] = bits_in(w, q, q);
        return;
    }
    const int a = anchor_of(mm, qp);
#pragma unroll
    for (int w = 0; w < 4; ++w) m[w] = (kv[w] & bits_in(w, 0, a - 1)) | bits_in(w, N + a, q);
}

// Keys the reference computes for query t: the encoder split (src/layers.cpp:591).
__device__ __forceinline__ int time_keys(const MaskMeta& mm, int t) { return t < mm.N ? mm.N : mm.S; }

// Variate-axis mask at slot p for query row q and key row k (reference src/masks.cpp:27).
__device__ __forceinline__ bool variate_allowed(const MaskMeta& mm, int p, int q, int k) {
    if (q == k) return true;
    if (p < mm.N && !kv_bit(mm, k, p)) return false;
    if (mm.cov) {
        const int rq = mm.role[q], rk = mm.role[k];
        if ((rq != 0 && rk == 0) || (rq == 2 && rk != 2)) return false;
    }
    return true;  // same group is guaranteed by the caller's key range
}

// ---------------------------------------------------------------------------------------
// Tensor-core time attention: one (row, head) problem at a time per CTA, four CTAs per SM.
//
// 128 threads, one query row per thread (TMEM lane = query). Thread 0 also issues the TMA
// loads and the two MMAs, so every warp computes. TMEM (128 columns per CTA):
//   S = Q K^T in columns [0, NK); the softmax writes P (f16, two keys per column) over
//   columns [0, NK/2) behind its reads of S; O = P V (P read from TMEM) in columns [64, 128).
// Shared memory: Q [S rounded to 8 rows][64] f16 (the score MMA reads 128 rows from Q; rows
// past S fall in the K region and only give scores of queries that do not exist), K and V
// [NK = S rounded to 16 rows][64] f16 (rows past S zero-filled by TMA), and a 16 KB block in
// which the epilogue turns its rows into full 128-byte stores.
// Per problem: S = Q K^T -> Q/K of the next problem load -> softmax -> O = P V -> V of the
// next problem loads -> epilogue (the TMEM is released before the stores).
constexpr int AT_THREADS = 128;
constexpr uint32_t AT_TMEM_COLS = 128;
constexpr uint32_t AT_O_COL = 64;

struct AttnBars {
    uint64_t full_qk, full_v, s_full, p_ready, o_full, tm_free;
    uint32_t tmem;
    int abort;
};

template <int NK, int PK>
struct AttnLayout {
    static constexpr int KV_BYTES = PK * NK * 128;       // the keys (or values) of the tile's problems
    static constexpr int STAGE_BYTES = 128 * 128;
    __host__ __device__ static constexpr int q_rows(int S) { return (S + 7) / 8 * 8; }
    // Problem p's queries at row 64 p (the score MMA reads 128 rows; those past the last
    // problem's fall in the K region).
    __host__ __device__ static constexpr int q_bytes(int S) { return ((PK - 1) * 64 + q_rows(S)) * 128; }
    __host__ __device__ static constexpr int smem(int S) { return q_bytes(S) + 2 * KV_BYTES + STAGE_BYTES + 1024 + 256; }
};

// Keys of the second problem of a packed tile sit NK positions up: the key set moves up by NK
// bits (NK a multiple of 16, at most 64).
template <int NK>
__device__ __forceinline__ void shift_keys(uint32_t (&m)[4]) {
    constexpr int WS = NK / 32, BS = NK % 32;
    uint32_t o[4];
#pragma unroll
    for (int w = 0; w < 4; ++w) {
        const uint32_t a = w - WS >= 0 ? m[w - WS] : 0u;
        if constexpr (BS == 0) {
            o[w] = a;
        } else {
            const uint32_t b = w - WS - 1 >= 0 ? m[w - WS - 1] : 0u;
            o[w] = (a << BS) | (b >> (32 - BS));
        }
    }
#pragma unroll
    for (int w = 0; w < 4; ++w) m[w] = o[w];
}

__device__ __forceinline__ bool at_wait(uint64_t* bar, uint32_t parity, volatile int* abort, int* err) {
    if (mbar_try_wait(bar, parity)) return true;
    const long long start = clock64();
    while (true) {
        if (*abort) return false;
        if (mbar_try_wait(bar, parity)) return true;
        if (clock64() - start > kWaitCycles) { *abort = 1; record_error(err, kDevTimeoutAttn); return false; }
    }
}
// Lane 0 waits and the warp follows its verdict, so a warp never splits on an abort.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, volatile int* abort, int* err) {
    int ok = 1;
    if ((threadIdx.x & 31) == 0) ok = at_wait(bar, parity, abort, err);
    return __shfl_sync(0xffffffffu, ok, 0) != 0;
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
}
// Eight consecutive 32-bit columns of this thread's TMEM lane.
__device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint32_t (&r)[8]) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"r"(taddr), "r"(r[0]),
                 "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7])
                 : "memory");
}
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
// D (TMEM) (+)= A (TMEM, K-major f16) * B (shared memory descriptor).
__device__ __forceinline__ void mma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc, bool accumulate) {
    const uint32_t z = 0;
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, {%5, %6, %7, %8}, p;\n}\n"
        ::"r"(d_tmem), "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(uint32_t(accumulate)), "r"(z), "r"(z), "r"(z), "r"(z));
}

// 2^x with subnormal results flushed to zero (probabilities are relative to the row maximum
// and rounded to f16, whose smallest subnormal is 2^-24).
__device__ __forceinline__ float exp2_ftz(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// logit scale 1/sqrt(64) folded with log2(e) for exp2
constexpr float kScaleLog2e = 0.125f * 1.4426950408889634f;

// Softmax of the query row in this thread's TMEM lane (`row` = the score tile's address at
// this warp's lanes) over the keys in `allowed`, which all lie in the 16-key chunks
// [kmin / 16, kmax / 16] (warp-uniform bounds, kmax >= 0). Pass 1: the maximum (eight
// partial maxima). Pass 2: the probabilities exp2(s * scale - max * scale) rounded to f16,
// written two keys per TMEM column over the score columns already read (P columns
// [8c, 8c + 8) <= S columns [16c, 16c + 16)), zeros in the chunks outside the bounds; returns
// their sum (eight partial sums). NCH: the tile's 16-key chunks.
template <int NCH>
__device__ __forceinline__ float softmax_to_p(uint32_t row, const uint32_t (&allowed)[4], int kmin, int kmax, bool live) {
    float mxj[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) mxj[j] = -INFINITY;
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
        if (c * 16 > kmax) break;
        if (c * 16 + 15 < kmin) continue;
        uint32_t sc[16];
        tmem_ld16(row + c * 16, sc);
        tmem_ld_wait();
        const uint32_t bits = allowed[(c * 16) >> 5] >> ((c * 16) & 31);
#pragma unroll
        for (int j = 0; j < 16; ++j)
            if ((bits >> j) & 1u) mxj[j & 7] = fmaxf(mxj[j & 7], __uint_as_float(sc[j]));
    }
    const float mx = fmaxf(fmaxf(fmaxf(mxj[0], mxj[1]), fmaxf(mxj[2], mxj[3])),
                           fmaxf(fmaxf(mxj[4], mxj[5]), fmaxf(mxj[6], mxj[7])));
    const float off = live ? mx * kScaleLog2e : 0.f;
    float sj[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) sj[j] = 0.f;
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
        uint32_t pk[8];
        if (c * 16 <= kmax && c * 16 + 15 >= kmin) {
            uint32_t sc[16];
            tmem_ld16(row + c * 16, sc);
            tmem_ld_wait();
            const uint32_t bits = allowed[(c * 16) >> 5] >> ((c * 16) & 31);
            float p[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                p[j] = (bits >> j) & 1u ? exp2_ftz(__fmaf_rn(__uint_as_float(sc[j]), kScaleLog2e, -off)) : 0.f;
                sj[j & 7] += p[j];
            }
#pragma unroll
            for (int j = 0; j < 8; ++j) pk[j] = pack_half2(p[2 * j], p[2 * j + 1]);
        } else {
#pragma unroll
            for (int j = 0; j < 8; ++j) pk[j] = 0u;
        }
        tmem_st8(row + c * 8, pk);
    }
    tmem_st_wait();
    return ((sj[0] + sj[1]) + (sj[2] + sj[3])) + ((sj[4] + sj[5]) + (sj[6] + sj[7]));
}

template <int NK, int PK>
__global__ void __launch_bounds__(AT_THREADS, 4)
    attn_time_tc_kernel(const __grid_constant__ CUtensorMap map_q, const __grid_constant__ CUtensorMap map_k,
                        const __grid_constant__ CUtensorMap map_v, const __half* __restrict__ gate,
                        __half* __restrict__ out, int rows, int H, const MaskMeta mm, int* err) {
    static_assert(PK == 1 || (PK == 2 && NK <= 64), "two problems per tile need NK <= 64");
    using Lay = AttnLayout<NK, PK>;
    extern __shared__ uint8_t smem_raw[];
    const int S = mm.S, D = H * 64;
    const int QR = Lay::q_rows(S);
    uint8_t* qbuf = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* kbuf = qbuf + Lay::q_bytes(S);
    uint8_t* vbuf = kbuf + Lay::KV_BYTES;
    uint8_t* obuf = vbuf + Lay::KV_BYTES;
    AttnBars* bars = reinterpret_cast<AttnBars*>(obuf + Lay::STAGE_BYTES);
    volatile int* abort = &bars->abort;
    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32, t = threadIdx.x;
    const int num = rows * H;
    const int units = (num + PK - 1) / PK;               // tiles of PK problems
    const bool ctl = threadIdx.x == 0;
    // This thread's problem of the tile (queries of problem p at TMEM lanes 64 p ..) and query.
    const int pb = PK == 2 ? t >> 6 : 0;
    const int qi = t - 64 * pb;

    if (ctl) {
        mbar_init(&bars->full_qk, 1); mbar_init(&bars->full_v, 1); mbar_init(&bars->s_full, 1);
        mbar_init(&bars->p_ready, 4); mbar_init(&bars->o_full, 1); mbar_init(&bars->tm_free, 4);
        bars->abort = 0;
        mbar_fence_init();
        fence_proxy_async();
    }
    if (warp == 0) { tmem_alloc(&bars->tmem, AT_TMEM_COLS); tmem_relinquish(); }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tS = bars->tmem;                       // S, then P over its first NK/2 columns
    const uint32_t tO = tS + AT_O_COL;
    const uint32_t lane_base = uint32_t(warp * 32) << 16;

    // A tile's second problem past the last one loads the first one's tiles again (finite
    // values for the P V product, whose probabilities there are zero); its rows store nothing.
    auto tile_prob = [&](int unit, int p) { const int pr = unit * PK + p; return pr < num ? pr : unit * PK; };
    auto issue_qk = [&](int unit) {
        mbar_arrive_expect_tx(&bars->full_qk, PK * (QR * 128 + NK * 128));
#pragma unroll
        for (int p = 0; p < PK; ++p) {
            tma_load_3d(qbuf + p * 64 * 128, &map_q, &bars->full_qk, 0, 0, tile_prob(unit, p));
            tma_load_3d(kbuf + p * NK * 128, &map_k, &bars->full_qk, 0, 0, tile_prob(unit, p));
        }
    };
    auto issue_v = [&](int unit) {
        mbar_arrive_expect_tx(&bars->full_v, PK * NK * 128);
#pragma unroll
        for (int p = 0; p < PK; ++p) tma_load_3d(vbuf + p * NK * 128, &map_v, &bars->full_v, 0, 0, tile_prob(unit, p));
    };
    if (ctl && int(blockIdx.x) < units) { issue_qk(blockIdx.x); issue_v(blockIdx.x); }

    int i = 0;
    for (int unit = blockIdx.x; unit < units; unit += gridDim.x, ++i) {
        const uint32_t ph = i & 1;
        const int next = unit + gridDim.x;
        const int prob = unit * PK + pb;                // this thread's problem
        const bool has = prob < num;
        const int r = has ? prob / H : 0, h = has ? prob % H : 0;
        if (warp == 0) {
            // S = Q K^T once Q and K are resident and every warp has read the previous O.
            int ok = 1;
            if (lane == 0) {
                ok = at_wait(&bars->full_qk, ph, abort, err);
                if (ok && i > 0) ok = at_wait(&bars->tm_free, ph ^ 1, abort, err);
                if (ok) {
                    tc_fence_after();
                    const uint64_t dq = smem_desc_sw128(smem_u32(qbuf)), dk = smem_desc_sw128(smem_u32(kbuf));
                    const uint32_t id1 = idesc_f16(128, PK * NK);
#pragma unroll
                    for (int k = 0; k < 4; ++k) mma_f16(tS, dq + uint64_t(2 * k), dk + uint64_t(2 * k), id1, k > 0);
                    mma_commit(&bars->s_full);
                }
            }
            if (!__shfl_sync(0xffffffffu, ok, 0)) break;
        }
        const bool live = has && qi < S;
        uint32_t allowed[4];
        key_set(mm, r, qi, live, allowed);
        if constexpr (PK == 2) {
            if (pb) shift_keys<NK>(allowed);
        }
        // Highest key any query of this warp attends: key chunks above it are skipped
        // (written as zero probabilities), which halves the work of causal rows. In a packed
        // tile the chunks below the warp's lowest key (the other problem's) are skipped too.
        int hi = -1;
#pragma unroll
        for (int w = 3; w >= 0; --w)
            if (hi < 0 && allowed[w]) hi = w * 32 + 31 - __clz(allowed[w]);
        const int kmax = __reduce_max_sync(0xffffffffu, hi + 1) - 1;   // -1: no live query in this warp
        int kmin = 0;
        if constexpr (PK == 2) {
            int lo = 128;
#pragma unroll
            for (int w = 0; w < 4; ++w)
                if (lo == 128 && allowed[w]) lo = w * 32 + __ffs(int(allowed[w])) - 1;
            kmin = int(__reduce_min_sync(0xffffffffu, unsigned(lo)));
        }
        if (!warp_wait(&bars->s_full, ph, abort, err)) break;
        tc_fence_after();
        if (ctl && next < units) issue_qk(next);       // Q and K are free once S is complete
        const float sum = kmax >= 0 ? softmax_to_p<PK * NK / 16>(tS + lane_base, allowed, kmin, kmax, live) : 0.f;
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars->p_ready);
        if (warp == 0) {
            // O = P V once every warp's P rows are in TMEM and this problem's V is resident.
            int ok = 1;
            if (lane == 0) {
                ok = at_wait(&bars->p_ready, ph, abort, err) && at_wait(&bars->full_v, ph, abort, err);
                if (ok) {
                    tc_fence_after();
                    const uint32_t sv = smem_u32(vbuf);
                    const uint32_t id2 = idesc_f16_bmn(128, 64);
#pragma unroll
                    for (int kk = 0; kk < PK * NK / 16; ++kk)
                        mma_f16_ts(tO, tS + kk * 8, smem_desc_sw128(sv + kk * 16 * 128), id2, kk > 0);
                    mma_commit(&bars->o_full);
                }
            }
            if (!__shfl_sync(0xffffffffu, ok, 0)) break;
        }
        // gate row of this query, fetched while O = P V runs
        uint4 gv[8];
        const __half* g = (gate && live) ? gate + ((int64_t(r) * H + h) * S + qi) * 64 : nullptr;
        if (g) {
#pragma unroll
            for (int c = 0; c < 8; ++c) gv[c] = *reinterpret_cast<const uint4*>(g + c * 8);
        }
        if (!warp_wait(&bars->o_full, ph, abort, err)) break;
        tc_fence_after();
        if (ctl && next < units) issue_v(next);        // V is free once O is complete
        // O * (1/sum) * gate in f16, staged row-wise and stored eight threads per 128-byte
        // output row. The TMEM is released as soon as O's second half is in registers.
        const float inv = live ? 1.0f / sum : 0.f;
        auto stage = [&](const uint32_t (&o)[32], int half32) {
#pragma unroll
            for (int c4 = 0; c4 < 4; ++c4) {
                const int c = half32 * 4 + c4;
                float y[8];
#pragma unroll
                for (int j = 0; j < 8; ++j) y[j] = __uint_as_float(o[c4 * 8 + j]) * inv;
                if (g) {
                    const __half2* gh = reinterpret_cast<const __half2*>(&gv[c]);
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        const float2 f = __half22float2(gh[j]);
                        y[2 * j] = __fmul_rn(y[2 * j], f.x);
                        y[2 * j + 1] = __fmul_rn(y[2 * j + 1], f.y);
                    }
                }
                uint4 u;
                u.x = pack_half2(y[0], y[1]); u.y = pack_half2(y[2], y[3]);
                u.z = pack_half2(y[4], y[5]); u.w = pack_half2(y[6], y[7]);
                *reinterpret_cast<uint4*>(obuf + t * 128 + ((c ^ (t & 7)) << 4)) = u;
            }
        };
        uint32_t o[32];
        if (kmax >= 0) {
            tmem_ld32(tO + lane_base, o);
            tmem_ld_wait();
            stage(o, 0);
            tmem_ld32(tO + lane_base + 32, o);
            tmem_ld_wait();
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars->tm_free);    // the next S may overwrite P and O
        if (kmax < 0) continue;
        stage(o, 1);
        __syncwarp();
        // A warp's rows all belong to one problem of the tile (64 lanes per problem).
        const int wpb = PK == 2 ? warp >> 1 : 0;
        const int wprob = unit * PK + wpb;
        const int wr = wprob / H, wh = wprob % H;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int row = warp * 32 + j * 4 + (lane >> 3), chunk = lane & 7;
            const int rq = row - 64 * wpb;
            if (rq < S && wprob < num)
                *reinterpret_cast<uint4*>(out + (int64_t(wr) * S + rq) * D + wh * 64 + chunk * 8) =
                    *reinterpret_cast<const uint4*>(obuf + row * 128 + ((chunk ^ (row & 7)) << 4));
        }
        __syncwarp();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 0) tmem_dealloc(bars->tmem, AT_TMEM_COLS);
}

template <int NK, int PK>
cudaError_t launch_attn_tc(const __half* q, const __half* k, const __half* v, const __half* gate, __half* out,
                           int rows, int H, const MaskMeta& mm, cudaStream_t stream, int* err) {
    using Lay = AttnLayout<NK, PK>;
    const int smem = Lay::smem(mm.S);
    static KernelSetup configured;
    int dev = 0;
    cudaGetDevice(&dev);
    unsigned long long ctx_key = 0;
    if (configured.needed(dev, &ctx_key)) {
        // The largest request of this key count (S = NK) so later calls need no update.
        cudaError_t e = cudaFuncSetAttribute(attn_time_tc_kernel<NK, PK>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             Lay::smem(NK));
        if (e != cudaSuccess) return e;
        configured.done(dev, ctx_key);
    }
    CUtensorMap mq, mk, mv;
    const int64_t planes = int64_t(rows) * H;
    if (!make_map_3d_f16(&mq, q, planes, mm.S, Lay::q_rows(mm.S)) || !make_map_3d_f16(&mk, k, planes, mm.S, NK) ||
        !make_map_3d_f16(&mv, v, planes, mm.S, NK))
        return cudaErrorInvalidValue;
    // CTAs per SM: shared memory (227 KB), TMEM (512 columns, 128 per CTA) and the launch bounds.
    int per_sm = (227 * 1024) / smem;
    if (per_sm > 4) per_sm = 4;
    if (per_sm < 1) per_sm = 1;
    int grid = device_sm_count() * per_sm;
    const int64_t units = (planes + PK - 1) / PK;
    if (int64_t(grid) > units) grid = int(units);
    attn_time_tc_kernel<NK, PK><<<grid, AT_THREADS, smem, stream>>>(mq, mk, mv, gate, out, rows, H, mm, err);
    return cudaGetLastError();
}

// ---------------------------------------------------------------------------------------
// Tensor-core variate attention for series of at most 32 rows (reference src/encoder.cpp:80,
// 86, 88: sdpa over the rows of one series at each patch slot; mask src/masks.cpp:27). A tile
// holds four problems (series, head, patch slots p0 .. p0 + 3), one per warp: slot p0 + w's
// query rows at TMEM lanes 32 w .. 32 w + G - 1 and its keys and values at rows 32 w .. of the
// K and V tiles (one TMA box per slot: that slot of 32 consecutive rows), so the score tile
// S = Q K^T (M = N = 128) is block-diagonal and each warp's softmax reads its own two 16-key
// chunks; P in TMEM, O = P V and the epilogue as in the time kernel. Box rows past the series
// (G < 32) are other series' rows or zero fill, outside every key set. The key set of query
// row i at slot p: itself, and the series' rows whose patch p is observed (every row at decoder
// slots), under the covariate role firewall; lane j supplies key j's part through ballots.
constexpr int AV_SLOTS = 4;
constexpr int AV_TILE = 128 * 128;                  // one operand tile: 4 slots x 32 rows x 128 B
constexpr int AV_SMEM = 1024 + 4 * AV_TILE + 256;   // Q, K, V, output staging, barriers

__global__ void __launch_bounds__(AT_THREADS, 3)
    attn_variate_tc_kernel(const __grid_constant__ CUtensorMap map_q, const __grid_constant__ CUtensorMap map_k,
                           const __grid_constant__ CUtensorMap map_v, const __half* __restrict__ gate,
                           __half* __restrict__ out, int rows, int H, int G, const MaskMeta mm, int* err) {
    extern __shared__ uint8_t smem_raw[];
    const int S = mm.S, D = H * 64;
    uint8_t* qbuf = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* kbuf = qbuf + AV_TILE;
    uint8_t* vbuf = kbuf + AV_TILE;
    uint8_t* obuf = vbuf + AV_TILE;
    AttnBars* bars = reinterpret_cast<AttnBars*>(obuf + AV_TILE);
    volatile int* abort = &bars->abort;
    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32, t = threadIdx.x;
    const int SQ = (S + AV_SLOTS - 1) / AV_SLOTS;
    const int units = (rows / G) * H * SQ;
    const bool ctl = threadIdx.x == 0;

    if (ctl) {
        mbar_init(&bars->full_qk, 1); mbar_init(&bars->full_v, 1); mbar_init(&bars->s_full, 1);
        mbar_init(&bars->p_ready, 4); mbar_init(&bars->o_full, 1); mbar_init(&bars->tm_free, 4);
        bars->abort = 0;
        mbar_fence_init();
        fence_proxy_async();
    }
    if (warp == 0) { tmem_alloc(&bars->tmem, AT_TMEM_COLS); tmem_relinquish(); }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tS = bars->tmem;                       // S, then P over its first 64 columns
    const uint32_t tO = tS + AT_O_COL;
    const uint32_t lane_base = uint32_t(warp * 32) << 16;

    auto issue_qk = [&](int unit) {
        const int r0 = (unit / (H * SQ)) * G, h = (unit / SQ) % H, p0 = (unit % SQ) * AV_SLOTS;
        mbar_arrive_expect_tx(&bars->full_qk, 2 * AV_TILE);
#pragma unroll
        for (int w = 0; w < AV_SLOTS; ++w) {
            tma_load_3d(qbuf + w * 32 * 128, &map_q, &bars->full_qk, 0, h * S + p0 + w, r0);
            tma_load_3d(kbuf + w * 32 * 128, &map_k, &bars->full_qk, 0, h * S + p0 + w, r0);
        }
    };
    auto issue_v = [&](int unit) {
        const int r0 = (unit / (H * SQ)) * G, h = (unit / SQ) % H, p0 = (unit % SQ) * AV_SLOTS;
        mbar_arrive_expect_tx(&bars->full_v, AV_TILE);
#pragma unroll
        for (int w = 0; w < AV_SLOTS; ++w) tma_load_3d(vbuf + w * 32 * 128, &map_v, &bars->full_v, 0, h * S + p0 + w, r0);
    };
    if (ctl && int(blockIdx.x) < units) { issue_qk(blockIdx.x); issue_v(blockIdx.x); }

    int i = 0;
    for (int unit = blockIdx.x; unit < units; unit += gridDim.x, ++i) {
        const uint32_t ph = i & 1;
        const int next = unit + gridDim.x;
        const int r0 = (unit / (H * SQ)) * G, h = (unit / SQ) % H, p = (unit % SQ) * AV_SLOTS + warp;
        const int row = r0 + lane;                      // this thread's query row (and key row)
        const bool in_series = lane < G && p < S;
        const bool live = in_series;
        if (warp == 0) {
            int ok = 1;
            if (lane == 0) {
                ok = at_wait(&bars->full_qk, ph, abort, err);
                if (ok && i > 0) ok = at_wait(&bars->tm_free, ph ^ 1, abort, err);
                if (ok) {
                    tc_fence_after();
                    const uint64_t dq = smem_desc_sw128(smem_u32(qbuf)), dk = smem_desc_sw128(smem_u32(kbuf));
                    const uint32_t id1 = idesc_f16(128, 128);
#pragma unroll
                    for (int k = 0; k < 4; ++k) mma_f16(tS, dq + uint64_t(2 * k), dk + uint64_t(2 * k), id1, k > 0);
                    mma_commit(&bars->s_full);
                }
            }
            if (!__shfl_sync(0xffffffffu, ok, 0)) break;
        }
        const bool usable = in_series && (p >= mm.N || kv_bit(mm, row, p));
        const int role = (mm.cov && in_series) ? mm.role[row] : 0;
        uint32_t bits = __ballot_sync(0xffffffffu, usable);
        if (mm.cov) {
            const uint32_t b0 = __ballot_sync(0xffffffffu, in_series && role == 0);
            const uint32_t b2 = __ballot_sync(0xffffffffu, in_series && role == 2);
            if (role != 0) bits &= ~b0;
            if (role == 2) bits &= b2;
        }
        bits = live ? (bits | (1u << lane)) : 0u;
        uint32_t allowed[4];
#pragma unroll
        for (int w = 0; w < 4; ++w) allowed[w] = w == warp ? bits : 0u;
        const int hi = bits ? warp * 32 + 31 - __clz(bits) : -1;
        const int lo = bits ? warp * 32 + __ffs(int(bits)) - 1 : 128;
        const int kmax = __reduce_max_sync(0xffffffffu, hi + 1) - 1;   // -1: no live query in this warp
        const int kmin = int(__reduce_min_sync(0xffffffffu, unsigned(lo)));
        if (!warp_wait(&bars->s_full, ph, abort, err)) break;
        tc_fence_after();
        if (ctl && next < units) issue_qk(next);       // Q and K are free once S is complete
        const float sum = kmax >= 0 ? softmax_to_p<8>(tS + lane_base, allowed, kmin, kmax, live) : 0.f;
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars->p_ready);
        if (warp == 0) {
            int ok = 1;
            if (lane == 0) {
                ok = at_wait(&bars->p_ready, ph, abort, err) && at_wait(&bars->full_v, ph, abort, err);
                if (ok) {
                    tc_fence_after();
                    const uint32_t sv = smem_u32(vbuf);
                    const uint32_t id2 = idesc_f16_bmn(128, 64);
#pragma unroll
                    for (int kk = 0; kk < 8; ++kk)
                        mma_f16_ts(tO, tS + kk * 8, smem_desc_sw128(sv + kk * 16 * 128), id2, kk > 0);
                    mma_commit(&bars->o_full);
                }
            }
            if (!__shfl_sync(0xffffffffu, ok, 0)) break;
        }
        uint4 gv[8];
        const __half* g = (gate && live) ? gate + ((int64_t(row) * H + h) * S + p) * 64 : nullptr;
        if (g) {
#pragma unroll
            for (int c = 0; c < 8; ++c) gv[c] = *reinterpret_cast<const uint4*>(g + c * 8);
        }
        if (!warp_wait(&bars->o_full, ph, abort, err)) break;
        tc_fence_after();
        if (ctl && next < units) issue_v(next);        // V is free once O is complete
        const float inv = live ? 1.0f / sum : 0.f;
        auto stage = [&](const uint32_t (&o)[32], int half32) {
#pragma unroll
            for (int c4 = 0; c4 < 4; ++c4) {
                const int c = half32 * 4 + c4;
                float y[8];
#pragma unroll
                for (int j = 0; j < 8; ++j) y[j] = __uint_as_float(o[c4 * 8 + j]) * inv;
                if (g) {
                    const __half2* gh = reinterpret_cast<const __half2*>(&gv[c]);
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        const float2 f = __half22float2(gh[j]);
                        y[2 * j] = __fmul_rn(y[2 * j], f.x);
                        y[2 * j + 1] = __fmul_rn(y[2 * j + 1], f.y);
                    }
                }
                uint4 u;
                u.x = pack_half2(y[0], y[1]); u.y = pack_half2(y[2], y[3]);
                u.z = pack_half2(y[4], y[5]); u.w = pack_half2(y[6], y[7]);
                *reinterpret_cast<uint4*>(obuf + t * 128 + ((c ^ (t & 7)) << 4)) = u;
            }
        };
        uint32_t o[32];
        if (kmax >= 0) {
            tmem_ld32(tO + lane_base, o);
            tmem_ld_wait();
            stage(o, 0);
            tmem_ld32(tO + lane_base + 32, o);
            tmem_ld_wait();
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars->tm_free);    // the next S may overwrite P and O
        if (kmax < 0) continue;
        stage(o, 1);
        __syncwarp();
        // The warp's 32 staged rows: rows r0 + ri of slot p, eight threads per 128-byte row.
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int ri = j * 4 + (lane >> 3), chunk = lane & 7, srow = warp * 32 + ri;
            if (ri < G)
                *reinterpret_cast<uint4*>(out + (int64_t(r0 + ri) * S + p) * D + h * 64 + chunk * 8) =
                    *reinterpret_cast<const uint4*>(obuf + srow * 128 + ((chunk ^ (srow & 7)) << 4));
        }
        __syncwarp();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 0) tmem_dealloc(bars->tmem, AT_TMEM_COLS);
}

// The attention kernels' bounded waits (lane 0 waits, its warp follows), made to expire
// without a fault: warp 0 waits on a barrier that nothing arrives on (kDevTimeoutAttn, abort
// flag raised); warp 1, waiting on another from half a limit later, leaves through the abort
// flag (err[1] = 1). The kernel then returns.
__global__ void attention_wait_expiry_kernel(int* err) {
    __shared__ uint64_t bars[2];
    __shared__ int abort_flag;
    const int warp = threadIdx.x / 32;
    if (threadIdx.x == 0) {
        mbar_init(&bars[0], 1);
        mbar_init(&bars[1], 1);
        abort_flag = 0;
        mbar_fence_init();
    }
    __syncthreads();
    volatile int* abort = &abort_flag;
    if (warp == 0) {
        warp_wait(&bars[0], 0, abort, err);
    } else if (warp == 1) {
        const long long t0 = clock64();
        while (clock64() - t0 < kWaitCycles / 2) __nanosleep(100000);
        const bool ok = warp_wait(&bars[1], 0, abort, nullptr);
        if (!ok && (threadIdx.x & 31) == 0 && *abort) err[1] = 1;
    }
}

}  // namespace

cudaError_t attention_wait_expiry_selftest(int* err, cudaStream_t stream) {
    attention_wait_expiry_kernel<<<1, 64, 0, stream>>>(err);
    return cudaGetLastError();
}

bool make_map_slot_rows_f16(CUtensorMap* map, const void* base, int64_t rows, int64_t slots, int box_rows);

cudaError_t attention_variate_tc(const __half* q, const __half* k, const __half* v, const __half* gate, __half* out,
                                 int rows, int H, int G, const MaskMeta& mm, cudaStream_t stream, int* err) {
    if (rows <= 0) return cudaSuccess;
    if (G <= 0 || G > 32 || rows % G || mm.S <= 0 || H <= 0) return cudaErrorInvalidValue;
    static KernelSetup configured;
    int dev = 0;
    cudaGetDevice(&dev);
    unsigned long long ctx_key = 0;
    if (configured.needed(dev, &ctx_key)) {
        cudaError_t e = cudaFuncSetAttribute(attn_variate_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, AV_SMEM);
        if (e != cudaSuccess) return e;
        configured.done(dev, ctx_key);
    }
    CUtensorMap mq, mk, mv;
    const int64_t slots = int64_t(H) * mm.S;
    if (!make_map_slot_rows_f16(&mq, q, rows, slots, 32) || !make_map_slot_rows_f16(&mk, k, rows, slots, 32) ||
        !make_map_slot_rows_f16(&mv, v, rows, slots, 32))
        return cudaErrorInvalidValue;
    const int64_t units = int64_t(rows / G) * H * ((mm.S + AV_SLOTS - 1) / AV_SLOTS);
    if (units > INT32_MAX) return cudaErrorInvalidValue;
    int grid = device_sm_count() * 3;                 // shared memory: three CTAs per SM
    if (int64_t(grid) > units) grid = int(units);
    attn_variate_tc_kernel<<<grid, AT_THREADS, AV_SMEM, stream>>>(mq, mk, mv, gate, out, rows, H, G, mm, err);
    return cudaGetLastError();
}

namespace {

// ---------------------------------------------------------------------------------------
// Tensor-core time attention for long rows (S > 128: context_length / patch_size up to
// 1024 context patches plus a decode block, twice that on the covariate layout).
//
// One problem = (tile of 128 query tokens, row, head). Query tiles are aligned to the end of
// the row, so the partial tile is the first one, whose causal keys fit in one key tile;
// problems with the most key tiles run first. Keys and values stream through separate
// four-stage shared-memory rings in tiles of 64 tokens: a key stage is free once its score
// product completes, a value stage once its P V product does.
// Warps 0-3 own the queries (TMEM lane = query token of the tile), warp 4 issues the TMA
// loads (polling the query, key and value rings so that none waits behind another), warp 5
// issues the MMAs. TMEM (256 columns, two CTAs per SM): two score buffers of 64 columns,
// each overwritten by its f16 probabilities (two keys per column), and O in columns
// [128, 192). Per key tile g: S[g&1] = Q K_g^T, softmax, O += P V_g; the score product of
// tile g+1 runs while the softmax of tile g does. The epilogue stages its output rows in
// the problem's own query buffer, which the next-but-one problem reloads afterwards.
// Each query keeps a reference maximum m: a tile whose maximum exceeds m by more than
// 2^8 (in exp2 units) moves m and rescales the query's O row and running sum first, so
// every probability exp2(s - m) lies in (0, 256] and rescaling is rare.
constexpr int AL_THREADS = 192;
constexpr int AL_KT = 64;                 // keys per tile
constexpr int AL_QT = 128;                // queries per problem
constexpr int AL_NST = 4;                 // key stages, and value stages
constexpr uint32_t AL_TMEM_COLS = 256;
constexpr uint32_t AL_O_COL = 128;
constexpr float AL_RESCALE = 8.f;         // log2 of the largest probability kept unscaled
constexpr int AL_Q_BYTES = AL_QT * 128;   // 128 query rows of 64 f16
constexpr int AL_KV_BYTES = AL_KT * 128;  // 64 key (or value) rows of 64 f16

struct AlBars {
    uint64_t q_full[2], q_empty[2], k_full[AL_NST], k_empty[AL_NST], v_full[AL_NST], v_empty[AL_NST];
    uint64_t s_full[2], p_ready[2], pv_done, o_full, tm_free;
    uint32_t tmem;
    int abort;
};
constexpr int AL_SMEM = 1024 + 2 * AL_Q_BYTES + 2 * AL_NST * AL_KV_BYTES + int(sizeof(AlBars));

// Keys of query q as two parts: key-valid patches k <= A, and the contiguous range [lo, q]
// (empty for a query outside the row: lo > q). Equal to time_allowed() restricted to the
// keys the reference computes (src/masks.cpp:21-26, the encoder split of src/layers.cpp:591).
struct QKeys { int A, lo, q; };
__device__ __forceinline__ QKeys query_keys(const MaskMeta& mm, int r, int q, bool live) {
    QKeys m{-1, 1, 0};
    if (!live) return m;
    const int N = mm.N;
    m.q = q;
    if (q < N) {
        m.A = (mm.cov && mm.role[r] == 2) ? N - 1 : q;   // known covariates see the whole context
        m.lo = q;
    } else if (!mm.cov) {
        m.A = N - 1; m.lo = N;
    } else if (q - N < mm.L) {
        m.lo = q;                                         // second-stream context: itself only
    } else {
        const int a = anchor_of(mm, q - N);
        m.A = min(a - 1, N - 1); m.lo = N + a;
    }
    return m;
}
// Bits [lo, hi] of a 64-bit set, clipped to [0, 63].
__device__ __forceinline__ uint64_t range64(int lo, int hi) {
    lo = max(lo, 0); hi = min(hi, 63);
    if (lo > hi) return 0ull;
    const uint64_t upper = hi == 63 ? ~0ull : ((1ull << (hi + 1)) - 1ull);
    return upper & ~((1ull << lo) - 1ull);
}
// The keys [k0, k0 + 64) of query m, k0 a multiple of 64.
__device__ __forceinline__ uint64_t tile_keys(const MaskMeta& mm, int r, const QKeys& m, int k0) {
    uint64_t kv = 0;
    if (m.A >= k0) {
        const int w = k0 >> 5;
        const uint32_t* row = mm.key_valid + int64_t(r) * mm.kv_words;
        const uint64_t lo = w < mm.kv_words ? row[w] : 0u, hi = w + 1 < mm.kv_words ? row[w + 1] : 0u;
        kv = (hi << 32 | lo) & range64(0, m.A - k0);
    }
    return kv | range64(m.lo - k0, m.q - k0);
}
// Problem p: query tile qt (of QT, heaviest first) of plane rh = row * H + head. The tile's
// first query token q0 = S - (QT - qt) * 128 is negative for the partial first tile.
struct AlProblem { int q0, rh, r, n; };
__device__ __forceinline__ AlProblem al_problem(const MaskMeta& mm, int p, int RH, int QT, int H) {
    AlProblem a;
    const int qt = QT - 1 - p / RH;
    a.rh = p % RH;
    a.r = a.rh / H;
    a.q0 = mm.S - (QT - qt) * AL_QT;
    // key tiles: up to the tile's last query, or the whole context for the context queries
    // of a known-covariate row
    int kb = a.q0 + AL_QT - 1;
    if (mm.cov && a.q0 < mm.N && mm.role[a.r] == 2) kb = max(kb, mm.N - 1);
    a.n = kb / AL_KT + 1;
    return a;
}

__device__ __forceinline__ bool mbar_test(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
        "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
        "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]),
        "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]),
        "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
        : "memory");
}

// Walks the key (or value) tiles of this CTA's problems in order.
struct TileCursor {
    int p = 0, i = 0, j = 0, n = 0, g = 0, rh = 0;
};

__global__ void __launch_bounds__(AL_THREADS, 2)
    attn_time_long_kernel(const __grid_constant__ CUtensorMap map_q, const __grid_constant__ CUtensorMap map_k,
                          const __grid_constant__ CUtensorMap map_v, const __half* __restrict__ gate,
                          __half* __restrict__ out, int rows, int H, const MaskMeta mm, int* err) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* qbuf = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* kbuf = qbuf + 2 * AL_Q_BYTES;
    uint8_t* vbuf = kbuf + AL_NST * AL_KV_BYTES;
    AlBars* bars = reinterpret_cast<AlBars*>(vbuf + AL_NST * AL_KV_BYTES);
    volatile int* abort = &bars->abort;
    const int S = mm.S, D = H * 64, RH = rows * H, QT = (S + AL_QT - 1) / AL_QT;
    const int num = RH * QT;
    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;

    if (threadIdx.x == 0) {
        for (int b = 0; b < 2; ++b) {
            mbar_init(&bars->q_full[b], 1); mbar_init(&bars->q_empty[b], 4);
            mbar_init(&bars->s_full[b], 1); mbar_init(&bars->p_ready[b], 4);
        }
        for (int s = 0; s < AL_NST; ++s) {
            mbar_init(&bars->k_full[s], 1); mbar_init(&bars->k_empty[s], 1);
            mbar_init(&bars->v_full[s], 1); mbar_init(&bars->v_empty[s], 1);
        }
        mbar_init(&bars->pv_done, 1); mbar_init(&bars->o_full, 1); mbar_init(&bars->tm_free, 4);
        bars->abort = 0;
        mbar_fence_init();
        fence_proxy_async();
    }
    if (warp == 0) { tmem_alloc(&bars->tmem, AL_TMEM_COLS); tmem_relinquish(); }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tbase = bars->tmem;
    const uint32_t tO = tbase + AL_O_COL;

    if (warp == 4) {
        // TMA producer: three independent streams (query tiles per problem, key tiles and
        // value tiles), each issued as soon as its ring slot is free.
        if (lane == 0) {
            int qp = blockIdx.x, qi = 0;                  // next query tile: problem, local index
            TileCursor kc, vc;
            kc.p = vc.p = blockIdx.x;
            auto enter = [&](TileCursor& c) {
                if (c.p < num) { const AlProblem a = al_problem(mm, c.p, RH, QT, H); c.n = a.n; c.rh = a.rh; c.j = 0; }
            };
            auto advance = [&](TileCursor& c) {
                ++c.g;
                if (++c.j == c.n) { c.p += gridDim.x; ++c.i; enter(c); }
            };
            enter(kc);
            enter(vc);
            long long idle_since = clock64();
            while (qp < num || kc.p < num || vc.p < num) {
                bool moved = false;
                if (qp < num && (qi < 2 || mbar_test(&bars->q_empty[qi & 1], ((qi >> 1) - 1) & 1))) {
                    const AlProblem a = al_problem(mm, qp, RH, QT, H);
                    mbar_arrive_expect_tx(&bars->q_full[qi & 1], AL_Q_BYTES);
                    tma_load_3d(qbuf + (qi & 1) * AL_Q_BYTES, &map_q, &bars->q_full[qi & 1], 0, a.q0, a.rh);
                    qp += gridDim.x; ++qi;
                    moved = true;
                }
                if (kc.p < num) {
                    const int st = kc.g % AL_NST;
                    if (kc.g < AL_NST || mbar_test(&bars->k_empty[st], ((kc.g / AL_NST) - 1) & 1)) {
                        mbar_arrive_expect_tx(&bars->k_full[st], AL_KV_BYTES);
                        tma_load_3d(kbuf + st * AL_KV_BYTES, &map_k, &bars->k_full[st], 0, kc.j * AL_KT, kc.rh);
                        advance(kc);
                        moved = true;
                    }
                }
                if (vc.p < num) {
                    const int st = vc.g % AL_NST;
                    if (vc.g < AL_NST || mbar_test(&bars->v_empty[st], ((vc.g / AL_NST) - 1) & 1)) {
                        mbar_arrive_expect_tx(&bars->v_full[st], AL_KV_BYTES);
                        tma_load_3d(vbuf + st * AL_KV_BYTES, &map_v, &bars->v_full[st], 0, vc.j * AL_KT, vc.rh);
                        advance(vc);
                        moved = true;
                    }
                }
                if (moved) {
                    idle_since = clock64();
                } else {
                    if (*abort) break;
                    if (clock64() - idle_since > kWaitCycles) { *abort = 1; record_error(err, kDevTimeoutAttn); break; }
                    __nanosleep(64);
                }
            }
        }
        __syncwarp();
    } else if (warp == 5) {
        // MMA issuer. Order per key tile g: S[g&1] = Q K_g^T, then O += P_{g-1} V_{g-1}, so the
        // score product of the next tile overlaps the softmax of the current one.
        if (lane == 0) {
            const uint32_t id_qk = idesc_f16(128, AL_KT), id_pv = idesc_f16_bmn(128, 64);
            int pg = -1, pi = 0;            // pending P V: global tile and problem index
            bool pfirst = false, plast = false;
            auto issue_pv = [&]() -> bool {
                const int st = pg % AL_NST;
                if (!at_wait(&bars->p_ready[pg & 1], (pg >> 1) & 1, abort, err) ||
                    !at_wait(&bars->v_full[st], (pg / AL_NST) & 1, abort, err))
                    return false;
                // the first tile of a problem overwrites O: the previous problem's O must be read
                if (pfirst && pi >= 1 && !at_wait(&bars->tm_free, (pi - 1) & 1, abort, err)) return false;
                tc_fence_after();
                const uint32_t tp = tbase + uint32_t(pg & 1) * AL_KT;
                const uint32_t sv = smem_u32(vbuf + st * AL_KV_BYTES);
#pragma unroll
                for (int kk = 0; kk < AL_KT / 16; ++kk)
                    mma_f16_ts(tO, tp + kk * 8, smem_desc_sw128(sv + kk * 16 * 128), id_pv, kk > 0 || !pfirst);
                mma_commit(&bars->pv_done);
                mma_commit(&bars->v_empty[st]);
                if (plast) mma_commit(&bars->o_full);
                return true;
            };
            int i = 0, g = 0;
            bool ok = true;
            for (int p = blockIdx.x; p < num && ok; p += gridDim.x, ++i) {
                const int n = al_problem(mm, p, RH, QT, H).n;
                const int qb = i & 1;
                if (!at_wait(&bars->q_full[qb], (i >> 1) & 1, abort, err)) { ok = false; break; }
                const uint64_t dq = smem_desc_sw128(smem_u32(qbuf + qb * AL_Q_BYTES));
                for (int j = 0; j < n; ++j, ++g) {
                    const int st = g % AL_NST;
                    // S[g&1] is free once P_{g-2}, written over it, has been multiplied.
                    if (!at_wait(&bars->k_full[st], (g / AL_NST) & 1, abort, err) ||
                        (g >= 2 && !at_wait(&bars->pv_done, (g - 2) & 1, abort, err))) { ok = false; break; }
                    tc_fence_after();
                    const uint64_t dk = smem_desc_sw128(smem_u32(kbuf + st * AL_KV_BYTES));
#pragma unroll
                    for (int k = 0; k < 4; ++k)
                        mma_f16(tbase + uint32_t(g & 1) * AL_KT, dq + uint64_t(2 * k), dk + uint64_t(2 * k), id_qk, k > 0);
                    mma_commit(&bars->s_full[g & 1]);
                    mma_commit(&bars->k_empty[st]);
                    if (pg >= 0 && !issue_pv()) { ok = false; break; }
                    pg = g; pi = i; pfirst = j == 0; plast = j == n - 1;
                }
            }
            if (ok && pg >= 0) issue_pv();
        }
        __syncwarp();
    } else {
        // Softmax and epilogue: thread t = query token q0 + t, TMEM lane t.
        const int t = threadIdx.x;
        const uint32_t lane_base = uint32_t(warp * 32) << 16;
        int i = 0, g = 0;
        for (int p = blockIdx.x; p < num; p += gridDim.x, ++i) {
            const AlProblem a = al_problem(mm, p, RH, QT, H);
            const int r = a.r, h = a.rh % H, n = a.n;
            const int q = a.q0 + t;
            const bool live = q >= 0;
            const QKeys qk = query_keys(mm, r, q, live);
            float mref = -INFINITY, sum = 0.f;
            bool ok = true;
            for (int j = 0; j < n; ++j, ++g) {
                const int b = g & 1;
                const uint64_t bits = tile_keys(mm, r, qk, j * AL_KT);
                if (!warp_wait(&bars->s_full[b], (g >> 1) & 1, abort, err)) { ok = false; break; }
                tc_fence_after();
                const uint32_t ts = tbase + lane_base + uint32_t(b) * AL_KT;
                uint32_t pk[32];
                if (__any_sync(0xffffffffu, bits != 0ull)) {
                    uint32_t s0[32], s1[32];
                    tmem_ld32(ts, s0);
                    tmem_ld32(ts + 32, s1);
                    tmem_ld_wait();
                    const uint32_t b0 = uint32_t(bits), b1 = uint32_t(bits >> 32);
                    // every lane of the warp attends every key of the tile: no per-key masking
                    const bool full = __all_sync(0xffffffffu, bits == ~0ull);
                    float mxj[8];
#pragma unroll
                    for (int c = 0; c < 8; ++c) mxj[c] = -INFINITY;
                    if (full) {
#pragma unroll
                        for (int c = 0; c < 32; ++c)
                            mxj[c & 7] = fmaxf(mxj[c & 7], fmaxf(__uint_as_float(s0[c]), __uint_as_float(s1[c])));
                    } else {
#pragma unroll
                        for (int c = 0; c < 32; ++c) {
                            if ((b0 >> c) & 1u) mxj[c & 7] = fmaxf(mxj[c & 7], __uint_as_float(s0[c]));
                            if ((b1 >> c) & 1u) mxj[c & 7] = fmaxf(mxj[c & 7], __uint_as_float(s1[c]));
                        }
                    }
                    const float mt = fmaxf(fmaxf(fmaxf(mxj[0], mxj[1]), fmaxf(mxj[2], mxj[3])),
                                           fmaxf(fmaxf(mxj[4], mxj[5]), fmaxf(mxj[6], mxj[7]))) * kScaleLog2e;
                    // Move the reference maximum; with earlier keys, rescale O and the sum.
                    const bool first = mref == -INFINITY && bits != 0ull;
                    const bool need = mref != -INFINITY && mt > mref + AL_RESCALE;
                    float factor = 1.f;
                    if (need) { factor = exp2_ftz(mref - mt); sum *= factor; }
                    if (first || need) mref = mt;
                    if (__any_sync(0xffffffffu, need)) {
                        // O holds the tiles before this one once the last P V completed.
                        if (!warp_wait(&bars->pv_done, (g - 1) & 1, abort, err)) { ok = false; break; }
                        tc_fence_after();
#pragma unroll 1
                        for (int c0 = 0; c0 < 64; c0 += 16) {
                            uint32_t o[16];
                            tmem_ld16(tO + lane_base + c0, o);
                            tmem_ld_wait();
                            uint32_t w[8];
#pragma unroll
                            for (int c = 0; c < 8; ++c) w[c] = __float_as_uint(__uint_as_float(o[c]) * factor);
                            tmem_st8(tO + lane_base + c0, w);
#pragma unroll
                            for (int c = 0; c < 8; ++c) w[c] = __float_as_uint(__uint_as_float(o[8 + c]) * factor);
                            tmem_st8(tO + lane_base + c0 + 8, w);
                        }
                        tmem_st_wait();
                    }
                    const float off = bits ? mref : 0.f;
                    float sj[8];
#pragma unroll
                    for (int c = 0; c < 8; ++c) sj[c] = 0.f;
                    if (full) {
#pragma unroll
                        for (int c = 0; c < 16; ++c) {
                            const float e0 = exp2_ftz(__fmaf_rn(__uint_as_float(s0[2 * c]), kScaleLog2e, -off));
                            const float e1 = exp2_ftz(__fmaf_rn(__uint_as_float(s0[2 * c + 1]), kScaleLog2e, -off));
                            const float e2 = exp2_ftz(__fmaf_rn(__uint_as_float(s1[2 * c]), kScaleLog2e, -off));
                            const float e3 = exp2_ftz(__fmaf_rn(__uint_as_float(s1[2 * c + 1]), kScaleLog2e, -off));
                            sj[(2 * c) & 7] += e0; sj[(2 * c + 1) & 7] += e1;
                            sj[(2 * c) & 7] += e2; sj[(2 * c + 1) & 7] += e3;
                            pk[c] = pack_half2(e0, e1);
                            pk[16 + c] = pack_half2(e2, e3);
                        }
                    } else {
#pragma unroll
                        for (int c = 0; c < 16; ++c) {
                            const float e0 = (b0 >> (2 * c)) & 1u ? exp2_ftz(__fmaf_rn(__uint_as_float(s0[2 * c]), kScaleLog2e, -off)) : 0.f;
                            const float e1 = (b0 >> (2 * c + 1)) & 1u ? exp2_ftz(__fmaf_rn(__uint_as_float(s0[2 * c + 1]), kScaleLog2e, -off)) : 0.f;
                            const float e2 = (b1 >> (2 * c)) & 1u ? exp2_ftz(__fmaf_rn(__uint_as_float(s1[2 * c]), kScaleLog2e, -off)) : 0.f;
                            const float e3 = (b1 >> (2 * c + 1)) & 1u ? exp2_ftz(__fmaf_rn(__uint_as_float(s1[2 * c + 1]), kScaleLog2e, -off)) : 0.f;
                            sj[(2 * c) & 7] += e0; sj[(2 * c + 1) & 7] += e1;
                            sj[(2 * c) & 7] += e2; sj[(2 * c + 1) & 7] += e3;
                            pk[c] = pack_half2(e0, e1);
                            pk[16 + c] = pack_half2(e2, e3);
                        }
                    }
                    sum += ((sj[0] + sj[1]) + (sj[2] + sj[3])) + ((sj[4] + sj[5]) + (sj[6] + sj[7]));
                } else {
#pragma unroll
                    for (int c = 0; c < 32; ++c) pk[c] = 0u;
                }
                tmem_st32(ts, pk);
                tmem_st_wait();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&bars->p_ready[b]);
            }
            if (!ok) break;
            // Epilogue: O * (1/sum) * gate in f16, staged per warp in this problem's query
            // buffer (every score product of the problem has completed) and stored as full rows.
            uint8_t* obuf = qbuf + (i & 1) * AL_Q_BYTES;
            uint4 gv[8];
            const __half* gp = (gate && live) ? gate + ((int64_t(r) * H + h) * S + q) * 64 : nullptr;
            if (gp) {
#pragma unroll
                for (int c = 0; c < 8; ++c) gv[c] = *reinterpret_cast<const uint4*>(gp + c * 8);
            }
            if (!warp_wait(&bars->o_full, i & 1, abort, err)) break;
            tc_fence_after();
            const float inv = live ? 1.0f / sum : 0.f;
            uint32_t o[32];
#pragma unroll
            for (int c = 0; c < 8; ++c) {
                if ((c & 3) == 0) {
                    tmem_ld32(tO + lane_base + c * 8, o);
                    tmem_ld_wait();
                    if (c == 4) {                   // O is in registers: the next problem may overwrite it
                        tc_fence_before();
                        __syncwarp();
                        if (lane == 0) mbar_arrive(&bars->tm_free);
                    }
                }
                float y[8];
#pragma unroll
                for (int e = 0; e < 8; ++e) y[e] = __uint_as_float(o[(c & 3) * 8 + e]) * inv;
                if (gp) {
                    const __half2* gh = reinterpret_cast<const __half2*>(&gv[c]);
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const float2 f = __half22float2(gh[e]);
                        y[2 * e] = __fmul_rn(y[2 * e], f.x);
                        y[2 * e + 1] = __fmul_rn(y[2 * e + 1], f.y);
                    }
                }
                uint4 u;
                u.x = pack_half2(y[0], y[1]); u.y = pack_half2(y[2], y[3]);
                u.z = pack_half2(y[4], y[5]); u.w = pack_half2(y[6], y[7]);
                *reinterpret_cast<uint4*>(obuf + t * 128 + ((c ^ (t & 7)) << 4)) = u;
            }
            __syncwarp();
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const int row = warp * 32 + j * 4 + (lane >> 3), chunk = lane & 7;
                const int tok = a.q0 + row;
                if (tok >= 0)
                    *reinterpret_cast<uint4*>(out + (int64_t(r) * S + tok) * D + h * 64 + chunk * 8) =
                        *reinterpret_cast<const uint4*>(obuf + row * 128 + ((chunk ^ (row & 7)) << 4));
            }
            // the query buffer may be reloaded (async proxy) once every warp's rows are out
            fence_proxy_async();
            __syncwarp();
            if (lane == 0) mbar_arrive(&bars->q_empty[i & 1]);
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 0) tmem_dealloc(tbase, AL_TMEM_COLS);
}

}  // namespace

cudaError_t attention_time_tc_long(const __half* q, const __half* k, const __half* v, const __half* gate, __half* out,
                                   int rows, int H, const MaskMeta& mm, cudaStream_t stream, int* err) {
    if (rows <= 0) return cudaSuccess;
    if (mm.S <= 0 || H <= 0) return cudaErrorInvalidValue;
    static KernelSetup configured;
    int dev = 0;
    cudaGetDevice(&dev);
    unsigned long long ctx_key = 0;
    if (configured.needed(dev, &ctx_key)) {
        cudaError_t e = cudaFuncSetAttribute(attn_time_long_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, AL_SMEM);
        if (e != cudaSuccess) return e;
        configured.done(dev, ctx_key);
    }
    CUtensorMap mq, mk, mv;
    const int64_t planes = int64_t(rows) * H;
    if (!make_map_3d_f16(&mq, q, planes, mm.S, AL_QT) || !make_map_3d_f16(&mk, k, planes, mm.S, AL_KT) ||
        !make_map_3d_f16(&mv, v, planes, mm.S, AL_KT))
        return cudaErrorInvalidValue;
    const int64_t problems = planes * ((mm.S + AL_QT - 1) / AL_QT);
    if (problems > INT32_MAX) return cudaErrorInvalidValue;
    int grid = device_sm_count() * 2;
    if (int64_t(grid) > problems) grid = int(problems);
    attn_time_long_kernel<<<grid, AL_THREADS, AL_SMEM, stream>>>(mq, mk, mv, gate, out, rows, H, mm, err);
    return cudaGetLastError();
}

namespace {

// ---------------------------------------------------------------------------------------
// CUDA-core kernels with the reference's operation order. One warp per query.
template <class T>
__device__ __forceinline__ float ld(const T* p) { return float(*p); }
template <>
__device__ __forceinline__ float ld<__half>(const __half* p) { return __half2float(*p); }
template <class T>
__device__ __forceinline__ void st(T* p, float v) { *p = v; }
template <>
__device__ __forceinline__ void st<__half>(__half* p, float v) { *p = __float2half_rn(v); }

// Softmax-weighted value sum of one query over `count` candidate keys given by key(j) with
// sequence index seq(j) (the index the reference's lane/tail split uses), logits already in
// `lg` (-inf where masked), as the reference does it (src/layers.cpp:600-614).
template <class T, class KeyPtr>
__device__ void softmax_values(float* lg, int count, const int* seqidx, int keys_total, KeyPtr vrow, int hd, float* y_out) {
    const int lane = threadIdx.x & 31;
    float mx = -INFINITY;
    for (int j = lane; j < count; j += 32) mx = fmaxf(mx, lg[j]);
    for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    const int end = keys_total / 8 * 8;
    for (int j = lane; j < count; j += 32) {
        const float x = __fsub_rn(lg[j], mx);
        lg[j] = seqidx[j] < end ? attention_exp(x) : float(exp(double(x)));
    }
    __syncwarp();
    // Eight lane sums over full chunks in sequence order, then the fixed tree, then the tail.
    float part = 0.f;
    if (lane < 8)
        for (int j = 0; j < count; ++j)
            if (seqidx[j] < end && (seqidx[j] & 7) == lane) part = __fadd_rn(part, lg[j]);
    float s[8];
#pragma unroll
    for (int l = 0; l < 8; ++l) s[l] = __shfl_sync(0xffffffffu, part, l);
    const float a0 = __fadd_rn(s[0], s[4]), a1 = __fadd_rn(s[1], s[5]), a2 = __fadd_rn(s[2], s[6]), a3 = __fadd_rn(s[3], s[7]);
    float sum = __fadd_rn(__fadd_rn(a0, a2), __fadd_rn(a1, a3));
    for (int j = 0; j < count; ++j)
        if (seqidx[j] >= end) sum = __fadd_rn(sum, lg[j]);
    const float reciprocal = __fdiv_rn(1.0f, sum);
    for (int d = lane; d < hd; d += 32) {
        float acc = 0.f;
        for (int j = 0; j < count; ++j) {
            const float vv = ld(vrow(j) + d);
            acc = hd < 16 ? __fadd_rn(acc, __fmul_rn(lg[j], vv)) : __fmaf_rn(lg[j], vv, acc);
        }
        y_out[d] = __fmul_rn(acc, reciprocal);
    }
}

constexpr int SIMT_WARPS = 4;
constexpr int SIMT_MAX_KEYS = kSimtMaxKeys;

// Time axis: block = (row, head, 4 queries). Logits in shared memory.
template <class T>
__global__ void __launch_bounds__(SIMT_WARPS * 32)
    attn_time_simt_kernel(const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v,
                          const T* __restrict__ gate, T* __restrict__ out, int rows, int H, int hd, const MaskMeta mm) {
    extern __shared__ float sh[];
    const int warp = threadIdx.x / 32, lane = threadIdx.x & 31;
    const int S = mm.S;
    float* lg = sh + warp * (2 * SIMT_MAX_KEYS);
    int* seq = reinterpret_cast<int*>(lg + SIMT_MAX_KEYS);
    float* y = sh + SIMT_WARPS * 2 * SIMT_MAX_KEYS + warp * 256;
    const int qblocks = (S + SIMT_WARPS - 1) / SIMT_WARPS;
    const int64_t b = blockIdx.x;
    const int r = int(b / (int64_t(H) * qblocks)), h = int((b / qblocks) % H), t = int(b % qblocks) * SIMT_WARPS + warp;
    if (r >= rows || t >= S) return;
    const int keys = time_keys(mm, t);
    const T* qp = q + ((int64_t(r) * H + h) * S + t) * hd;
    const T* kb = k + (int64_t(r) * H + h) * S * hd;
    for (int j = lane; j < keys; j += 32) {
        seq[j] = j;
        if (!time_allowed(mm, r, t, j)) { lg[j] = -INFINITY; continue; }
        double s = 0;
        for (int d = 0; d < hd; ++d) s = __fma_rn(double(ld(qp + d)), double(ld(kb + int64_t(j) * hd + d)), s);
        lg[j] = __fmul_rn(float(s), float(1.0 / sqrt(double(hd))));
    }
    __syncwarp();
    const T* vb = v + (int64_t(r) * H + h) * S * hd;
    softmax_values<T>(lg, keys, seq, keys, [&](int j) { return vb + int64_t(j) * hd; }, hd, y);
    __syncwarp();
    const int D = H * hd;
    const T* g = gate ? gate + ((int64_t(r) * H + h) * S + t) * hd : nullptr;
    for (int d = lane; d < hd; d += 32) {
        float val = y[d];
        if (g) val = __fmul_rn(val, ld(g + d));
        st(out + (int64_t(r) * S + t) * D + h * hd + d, val);
    }
}

// The same computation for long rows (head_dim 64), tiled through shared memory: block =
// (row, head, TS_Q consecutive queries), 256 threads. The per-query warp kernel above reads
// every key row with per-lane strided loads and sums each value column behind a global load
// per key; here key and value tiles of TS_KT rows are staged once per block (keys as float64,
// values as float) and shared by its queries, and each thread runs four independent chains.
// Every operation and its order per query is the reference's, as above: float64 q.k dots over
// d = 0..63, the logit as float(s) * float(1/8), the maximum over the query's computed keys,
// ATen exp for keys below the last full eight-key chunk and libm exp after it, eight strided
// lane sums in key order + the fixed tree + the tail, one reciprocal, and per output column a
// float FMA chain over the keys in order (masked keys contribute p = 0, as there).
constexpr int TS_Q = 16;
constexpr int TS_KT = 64;
constexpr int TS_THREADS = 256;
constexpr int TS_KPAD = 65;                // float64 key rows padded: conflict-free column reads

constexpr size_t simt_tiled_smem(int S) {
    return size_t(TS_Q) * 64 * sizeof(double) + size_t(TS_KT) * TS_KPAD * sizeof(double) +
           size_t(TS_Q) * S * sizeof(float) + TS_Q * sizeof(float);
}

template <class T>
__global__ void __launch_bounds__(TS_THREADS)
    attn_time_simt_tiled_kernel(const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v,
                                const T* __restrict__ gate, T* __restrict__ out, int rows, int H, const MaskMeta mm) {
    extern __shared__ double ts_sh[];
    constexpr int HD = 64;
    double* qs = ts_sh;                                   // [TS_Q][64]
    double* ks = qs + TS_Q * HD;                          // [TS_KT][TS_KPAD]; values as float [TS_KT][64]
    float* vs = reinterpret_cast<float*>(ks);
    const int S = mm.S;
    float* lg = reinterpret_cast<float*>(ks + TS_KT * TS_KPAD);   // [TS_Q][S]: logits, then probabilities
    float* recip = lg + TS_Q * S;                                 // [TS_Q]
    const int tid = threadIdx.x;
    const int qblocks = (S + TS_Q - 1) / TS_Q;
    const int64_t b = blockIdx.x;
    const int r = int(b / (int64_t(H) * qblocks)), h = int((b / qblocks) % H), t0 = int(b % qblocks) * TS_Q;
    if (r >= rows) return;                                        // uniform across the block
    const int64_t plane = (int64_t(r) * H + h) * S;
    // Keys the block's queries can attend: causal encoder queries (no covariates) see keys up
    // to themselves, others all their computed keys. Tiles past the block's bound hold only
    // masked keys, whose probabilities are exactly 0: their logits are written as -inf and
    // their products are skipped (an FMA with p = 0 leaves the chain unchanged).
    int kend = 0;
    for (int qi = 0; qi < TS_Q && t0 + qi < S; ++qi) {
        const int t = t0 + qi;
        kend = max(kend, (!mm.cov && t < mm.N) ? t + 1 : time_keys(mm, t));
    }
    const int kdone = (kend + TS_KT - 1) / TS_KT * TS_KT;       // keys covered by the tiles

    for (int i = tid; i < TS_Q * HD; i += TS_THREADS) {
        const int qi = i / HD, d = i % HD;
        qs[i] = t0 + qi < S ? double(ld(q + (plane + t0 + qi) * HD + d)) : 0.0;
    }
    // Logits: thread (kj = tid % 64, queries 4 g .. 4 g + 3 with g = tid / 64).
    const int kj = tid & (TS_KT - 1), g = tid >> 6;
    int kq[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) kq[u] = t0 + 4 * g + u < S ? time_keys(mm, t0 + 4 * g + u) : 0;
    for (int k0 = 0; k0 < kend; k0 += TS_KT) {
        __syncthreads();                                          // the previous tile is consumed
        for (int i = tid; i < TS_KT * HD; i += TS_THREADS) {
            const int jj = i / HD, d = i % HD;
            ks[jj * TS_KPAD + d] = k0 + jj < S ? double(ld(k + (plane + k0 + jj) * HD + d)) : 0.0;
        }
        __syncthreads();
        const int j = k0 + kj;
        double acc[4] = {0.0, 0.0, 0.0, 0.0};
        const double* kr = ks + kj * TS_KPAD;
        const double* q0 = qs + (4 * g) * HD;
#pragma unroll 8
        for (int d = 0; d < HD; ++d) {
            const double kd = kr[d];
#pragma unroll
            for (int u = 0; u < 4; ++u) acc[u] = __fma_rn(q0[u * HD + d], kd, acc[u]);
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int t = t0 + 4 * g + u;
            if (j < kq[u])
                lg[(4 * g + u) * S + j] = time_allowed(mm, r, t, j) ? __fmul_rn(float(acc[u]), float(1.0 / sqrt(double(HD))))
                                                                    : -INFINITY;
        }
    }
    for (int i = tid; i < TS_Q * S; i += TS_THREADS) {
        const int qi = i / S, j = i % S;
        if (j >= kdone && t0 + qi < S && j < time_keys(mm, t0 + qi)) lg[i] = -INFINITY;
    }
    __syncthreads();
    // Softmax of each query: 16 threads per query for the maximum and the exponentials.
    {
        const int qi = tid >> 4, sub = tid & 15;
        const int t = t0 + qi, kt = t < S ? time_keys(mm, t) : 0;
        float* row = lg + qi * S;
        float mx = -INFINITY;
        for (int j = sub; j < kt; j += 16) mx = fmaxf(mx, row[j]);
#pragma unroll
        for (int o = 8; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        const int end = kt / 8 * 8;
        for (int j = sub; j < kt; j += 16) {
            const float x = __fsub_rn(row[j], mx);
            row[j] = j < end ? attention_exp(x) : float(exp(double(x)));
        }
    }
    __syncthreads();
    // Sums: eight lane chains per query (keys j = l mod 8 below the last full chunk, in key
    // order), the fixed tree, then the tail in order.
    if (tid < TS_Q * 8) {
        const int qi = tid >> 3, l = tid & 7;
        const int t = t0 + qi, kt = t < S ? time_keys(mm, t) : 0;
        const int end = kt / 8 * 8;
        const float* row = lg + qi * S;
        float part = 0.f;
        for (int j = l; j < end; j += 8) part = __fadd_rn(part, row[j]);
        const int base = (tid & 31) & ~7;
        float sv[8];
#pragma unroll
        for (int m = 0; m < 8; ++m) sv[m] = __shfl_sync(0xffffffffu, part, base + m);
        if (l == 0 && t < S) {
            const float a0 = __fadd_rn(sv[0], sv[4]), a1 = __fadd_rn(sv[1], sv[5]);
            const float a2 = __fadd_rn(sv[2], sv[6]), a3 = __fadd_rn(sv[3], sv[7]);
            float sum = __fadd_rn(__fadd_rn(a0, a2), __fadd_rn(a1, a3));
            for (int j = end; j < kt; ++j) sum = __fadd_rn(sum, row[j]);
            recip[qi] = __fdiv_rn(1.0f, sum);
        }
    }
    // Values: thread (query tid / 16, columns 4 (tid % 16) .. + 3): float FMA chains over the
    // keys in order, value tiles staged as float.
    const int vq = tid >> 4, d4 = (tid & 15) * 4;
    const int vt = t0 + vq, vkeys = vt < S ? min(time_keys(mm, vt), kend) : 0;
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    for (int k0 = 0; k0 < kend; k0 += TS_KT) {
        __syncthreads();                                          // logits / sums / previous tile done
        for (int i = tid; i < TS_KT * HD; i += TS_THREADS) {
            const int jj = i / HD, dd = i % HD;
            vs[i] = k0 + jj < S ? ld(v + (plane + k0 + jj) * HD + dd) : 0.f;
        }
        __syncthreads();
        const int n = min(TS_KT, vkeys - k0);
        const float* pr = lg + vq * S + k0;
        for (int jj = 0; jj < n; ++jj) {
            const float p = pr[jj];
            const float4 vv = *reinterpret_cast<const float4*>(vs + jj * HD + d4);
            acc[0] = __fmaf_rn(p, vv.x, acc[0]);
            acc[1] = __fmaf_rn(p, vv.y, acc[1]);
            acc[2] = __fmaf_rn(p, vv.z, acc[2]);
            acc[3] = __fmaf_rn(p, vv.w, acc[3]);
        }
    }
    if (vt >= S) return;
    const int D = H * HD;
    const float rc = recip[vq];
#pragma unroll
    for (int c = 0; c < 4; ++c) {
        float val = __fmul_rn(acc[c], rc);
        if (gate) val = __fmul_rn(val, ld(gate + (plane + vt) * HD + d4 + c));
        st(out + (int64_t(r) * S + vt) * D + h * HD + d4 + c, val);
    }
}

// Variate axis: block = (row, slot, head) with 4 warps over heads; keys are the rows of the
// query row's series. Sequence index of a key = its row index within the forecast pass.
template <class T>
__global__ void __launch_bounds__(SIMT_WARPS * 32)
    attn_variate_simt_kernel(const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v,
                             const T* __restrict__ gate, T* __restrict__ out, int rows, int H, int hd, const MaskMeta mm) {
    extern __shared__ float sh[];
    const int warp = threadIdx.x / 32, lane = threadIdx.x & 31;
    const int S = mm.S;
    float* lg = sh + warp * (2 * SIMT_MAX_KEYS);
    int* seq = reinterpret_cast<int*>(lg + SIMT_MAX_KEYS);
    float* y = sh + SIMT_WARPS * 2 * SIMT_MAX_KEYS + warp * 256;
    const int hblocks = (H + SIMT_WARPS - 1) / SIMT_WARPS;
    const int64_t b = blockIdx.x;
    const int r = int(b / (int64_t(S) * hblocks)), p = int((b / hblocks) % S), h = int(b % hblocks) * SIMT_WARPS + warp;
    if (r >= rows || h >= H) return;
    const int g0 = mm.group_begin[r], gs = mm.group_size[r];
    const int pass0 = (r / mm.pass_rows) * mm.pass_rows;
    const T* qp = q + ((int64_t(r) * H + h) * S + p) * hd;
    for (int j = lane; j < gs; j += 32) {
        const int kr = g0 + j;
        seq[j] = kr - pass0;
        if (!variate_allowed(mm, p, r, kr)) { lg[j] = -INFINITY; continue; }
        const T* kp = k + ((int64_t(kr) * H + h) * S + p) * hd;
        double s = 0;
        for (int d = 0; d < hd; ++d) s = __fma_rn(double(ld(qp + d)), double(ld(kp + d)), s);
        lg[j] = __fmul_rn(float(s), float(1.0 / sqrt(double(hd))));
    }
    __syncwarp();
    softmax_values<T>(lg, gs, seq, mm.pass_rows,
                      [&](int j) { return v + ((int64_t(g0 + j) * H + h) * S + p) * hd; }, hd, y);
    __syncwarp();
    const int D = H * hd;
    const T* g = gate ? gate + ((int64_t(r) * H + h) * S + p) * hd : nullptr;
    for (int d = lane; d < hd; d += 32) {
        float val = y[d];
        if (g) val = __fmul_rn(val, ld(g + d));
        st(out + (int64_t(r) * S + p) * D + h * hd + d, val);
    }
}

// Variate-axis attention on the tensor-core path (f16 q/k/v/gate, head_dim 64): one warp per
// (series group, patch slot, head) problem, the group's K and V rows converted to f32 in
// shared memory once and read as broadcasts, QPL query rows per lane (group size <= 32 QPL).
// Scores, softmax and the weighted sum in f32; the keys and mask are the reference's
// (src/masks.cpp:27: same series, key patch observed or a decoder slot, role firewall, or the
// query itself); the operation order is not the reference's float order (f16 path).
constexpr int VF_WARPS = 4;

template <int QPL>
__global__ void __launch_bounds__(VF_WARPS * 32)
    attn_variate_fast_kernel(const __half* __restrict__ q, const __half* __restrict__ k, const __half* __restrict__ v,
                             const __half* __restrict__ gate, __half* __restrict__ out, int rows, int H, int G,
                             const MaskMeta mm) {
    constexpr int GM = 32 * QPL;
    extern __shared__ float vf_sh[];
    const int warp = threadIdx.x / 32, lane = threadIdx.x & 31;
    float* Ks = vf_sh + warp * (2 * GM * 64 + GM);
    float* Vs = Ks + GM * 64;
    uint32_t* meta = reinterpret_cast<uint32_t*>(Vs + GM * 64);   // bit 0: key usable, bits 1..: role
    const int S = mm.S, D = H * 64;
    const int64_t pid = int64_t(blockIdx.x) * VF_WARPS + warp;
    const int64_t total = int64_t(rows / G) * H * S;
    if (pid >= total) return;                                     // uniform across the warp
    const int p = int(pid % S), h = int((pid / S) % H);
    const int r0 = int(pid / (int64_t(S) * H)) * G;
    // K and V rows of the group at (head, slot): eight lanes per 128-byte row.
    for (int j = lane >> 3; j < G; j += 4) {
        const int64_t off = ((int64_t(r0 + j) * H + h) * S + p) * 64 + (lane & 7) * 8;
        const uint4 kk = *reinterpret_cast<const uint4*>(k + off);
        const uint4 vv = *reinterpret_cast<const uint4*>(v + off);
        const __half2* kh = reinterpret_cast<const __half2*>(&kk);
        const __half2* vh = reinterpret_cast<const __half2*>(&vv);
        float* kd = Ks + j * 64 + (lane & 7) * 8;
        float* vd = Vs + j * 64 + (lane & 7) * 8;
#pragma unroll
        for (int t = 0; t < 4; ++t) {
            const float2 a = __half22float2(kh[t]), b = __half22float2(vh[t]);
            kd[2 * t] = a.x; kd[2 * t + 1] = a.y;
            vd[2 * t] = b.x; vd[2 * t + 1] = b.y;
        }
    }
    for (int j = lane; j < G; j += 32) {
        const int kr = r0 + j;
        const bool usable = p >= mm.N || kv_bit(mm, kr, p);
        meta[j] = (usable ? 1u : 0u) | (uint32_t(mm.cov ? mm.role[kr] : 0) << 1);
    }
    __syncwarp();
#pragma unroll 1
    for (int qi = 0; qi < QPL; ++qi) {
        const int i = lane + 32 * qi;
        const bool live = i < G;
        const int r = r0 + (live ? i : 0);
        const int64_t qoff = ((int64_t(r) * H + h) * S + p) * 64;
        float qv[64];
#pragma unroll
        for (int c = 0; c < 8; ++c) {
            const uint4 u = *reinterpret_cast<const uint4*>(q + qoff + c * 8);
            const __half2* hh = reinterpret_cast<const __half2*>(&u);
#pragma unroll
            for (int t = 0; t < 4; ++t) {
                const float2 f = __half22float2(hh[t]);
                qv[c * 8 + 2 * t] = f.x; qv[c * 8 + 2 * t + 1] = f.y;
            }
        }
        const int rq = mm.cov ? mm.role[r] : 0;
        float sc[GM];
        float mx = -INFINITY;
#pragma unroll
        for (int j = 0; j < GM; ++j) {
            sc[j] = -INFINITY;
            if (j < G) {
                const uint32_t mj = meta[j];
                const int rk = int(mj >> 1);
                const bool allowed = j == i || ((mj & 1u) && !(mm.cov && ((rq != 0 && rk == 0) || (rq == 2 && rk != 2))));
                if (allowed) {
                    const float4* kr4 = reinterpret_cast<const float4*>(Ks + j * 64);
                    float a0 = 0.f, a1 = 0.f;
#pragma unroll
                    for (int d = 0; d < 16; d += 2) {
                        const float4 x = kr4[d], y = kr4[d + 1];
                        a0 = fmaf(qv[4 * d], x.x, a0); a0 = fmaf(qv[4 * d + 1], x.y, a0);
                        a0 = fmaf(qv[4 * d + 2], x.z, a0); a0 = fmaf(qv[4 * d + 3], x.w, a0);
                        a1 = fmaf(qv[4 * d + 4], y.x, a1); a1 = fmaf(qv[4 * d + 5], y.y, a1);
                        a1 = fmaf(qv[4 * d + 6], y.z, a1); a1 = fmaf(qv[4 * d + 7], y.w, a1);
                    }
                    sc[j] = (a0 + a1) * 0.125f;
                    mx = fmaxf(mx, sc[j]);
                }
            }
        }
        float acc[64];
#pragma unroll
        for (int d = 0; d < 64; ++d) acc[d] = 0.f;
        float sum = 0.f;
#pragma unroll
        for (int j = 0; j < GM; ++j) {
            if (j < G && sc[j] != -INFINITY) {
                const float pj = __expf(sc[j] - mx);
                sum += pj;
                const float4* vr4 = reinterpret_cast<const float4*>(Vs + j * 64);
#pragma unroll
                for (int d = 0; d < 16; ++d) {
                    const float4 x = vr4[d];
                    acc[4 * d] = fmaf(pj, x.x, acc[4 * d]); acc[4 * d + 1] = fmaf(pj, x.y, acc[4 * d + 1]);
                    acc[4 * d + 2] = fmaf(pj, x.z, acc[4 * d + 2]); acc[4 * d + 3] = fmaf(pj, x.w, acc[4 * d + 3]);
                }
            }
        }
        if (!live) continue;
        const float inv = 1.0f / sum;
        const __half* gp = gate ? gate + qoff : nullptr;
        __half* dst = out + (int64_t(r) * S + p) * D + h * 64;
#pragma unroll
        for (int c = 0; c < 8; ++c) {
            float y[8];
#pragma unroll
            for (int t = 0; t < 8; ++t) y[t] = acc[c * 8 + t] * inv;
            if (gp) {
                const uint4 gu = *reinterpret_cast<const uint4*>(gp + c * 8);
                const __half2* gh = reinterpret_cast<const __half2*>(&gu);
#pragma unroll
                for (int t = 0; t < 4; ++t) {
                    const float2 f = __half22float2(gh[t]);
                    y[2 * t] = __fmul_rn(y[2 * t], f.x);
                    y[2 * t + 1] = __fmul_rn(y[2 * t + 1], f.y);
                }
            }
            uint4 u;
            u.x = pack_half2(y[0], y[1]); u.y = pack_half2(y[2], y[3]);
            u.z = pack_half2(y[4], y[5]); u.w = pack_half2(y[6], y[7]);
            *reinterpret_cast<uint4*>(dst + c * 8) = u;
        }
    }
}

constexpr size_t simt_smem() { return (SIMT_WARPS * 2 * SIMT_MAX_KEYS + SIMT_WARPS * 256) * sizeof(float); }

}  // namespace

cudaError_t attention_time_tc(const __half* q, const __half* k, const __half* v, const __half* gate, __half* out,
                              int rows, int H, const MaskMeta& mm, cudaStream_t stream, int* err, int pack) {
    if (rows <= 0) return cudaSuccess;
    if (mm.S <= 0 || mm.S > 128) return cudaErrorInvalidValue;
    const int nk = (mm.S + 15) / 16 * 16;
    const bool two = pack && mm.S <= 64;
    switch (nk) {
        case 16: return two ? launch_attn_tc<16, 2>(q, k, v, gate, out, rows, H, mm, stream, err)
                            : launch_attn_tc<16, 1>(q, k, v, gate, out, rows, H, mm, stream, err);
        case 32: return two ? launch_attn_tc<32, 2>(q, k, v, gate, out, rows, H, mm, stream, err)
                            : launch_attn_tc<32, 1>(q, k, v, gate, out, rows, H, mm, stream, err);
        case 48: return two ? launch_attn_tc<48, 2>(q, k, v, gate, out, rows, H, mm, stream, err)
                            : launch_attn_tc<48, 1>(q, k, v, gate, out, rows, H, mm, stream, err);
        case 64: return two ? launch_attn_tc<64, 2>(q, k, v, gate, out, rows, H, mm, stream, err)
                            : launch_attn_tc<64, 1>(q, k, v, gate, out, rows, H, mm, stream, err);
        case 80: return launch_attn_tc<80, 1>(q, k, v, gate, out, rows, H, mm, stream, err);
        case 96: return launch_attn_tc<96, 1>(q, k, v, gate, out, rows, H, mm, stream, err);
        case 112: return launch_attn_tc<112, 1>(q, k, v, gate, out, rows, H, mm, stream, err);
        case 128: return launch_attn_tc<128, 1>(q, k, v, gate, out, rows, H, mm, stream, err);
    }
    return cudaErrorInvalidValue;
}

template <class T>
cudaError_t attention_time_simt_tiled(const T* q, const T* k, const T* v, const T* gate, T* out, int rows, int H,
                                      const MaskMeta& mm, cudaStream_t stream) {
    const size_t smem = simt_tiled_smem(mm.S);
    if (smem > 227 * 1024) return cudaErrorInvalidValue;
    static KernelSetup configured;
    int dev = 0;
    cudaGetDevice(&dev);
    unsigned long long ctx_key = 0;
    if (configured.needed(dev, &ctx_key)) {
        // the largest row this kernel takes, so later calls need no update
        cudaError_t e = cudaFuncSetAttribute(attn_time_simt_tiled_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             int(simt_tiled_smem(SIMT_MAX_KEYS)));
        if (e != cudaSuccess) return e;
        configured.done(dev, ctx_key);
    }
    const int64_t blocks = int64_t(rows) * H * ((mm.S + TS_Q - 1) / TS_Q);
    attn_time_simt_tiled_kernel<T><<<unsigned(blocks), TS_THREADS, smem, stream>>>(q, k, v, gate, out, rows, H, mm);
    return cudaGetLastError();
}

template <class T>
cudaError_t attention_time_simt(const T* q, const T* k, const T* v, const T* gate, T* out, int rows, int H, int hd,
                                const MaskMeta& mm, cudaStream_t stream, int tiled) {
    if (rows <= 0) return cudaSuccess;
    if (mm.S > SIMT_MAX_KEYS || hd > 256) return cudaErrorInvalidValue;
    // Long rows of head_dim 64: the tiled kernel (same bits).
    if (hd == 64 && (tiled > 0 || (tiled < 0 && mm.S > 128)))
        return attention_time_simt_tiled(q, k, v, gate, out, rows, H, mm, stream);
    static KernelSetup configured;
    int dev = 0;
    cudaGetDevice(&dev);
    unsigned long long ctx_key = 0;
    if (configured.needed(dev, &ctx_key)) {
        cudaError_t e = cudaFuncSetAttribute(attn_time_simt_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(simt_smem()));
        if (e != cudaSuccess) return e;
        configured.done(dev, ctx_key);
    }
    const int64_t blocks = int64_t(rows) * H * ((mm.S + SIMT_WARPS - 1) / SIMT_WARPS);
    attn_time_simt_kernel<T><<<unsigned(blocks), SIMT_WARPS * 32, simt_smem(), stream>>>(q, k, v, gate, out, rows, H, hd, mm);
    return cudaGetLastError();
}

template <class T>
cudaError_t attention_variate_simt(const T* q, const T* k, const T* v, const T* gate, T* out, int rows, int H, int hd,
                                   const MaskMeta& mm, cudaStream_t stream) {
    if (rows <= 0) return cudaSuccess;
    if (hd > 256) return cudaErrorInvalidValue;
    static KernelSetup configured;
    int dev = 0;
    cudaGetDevice(&dev);
    unsigned long long ctx_key = 0;
    if (configured.needed(dev, &ctx_key)) {
        cudaError_t e = cudaFuncSetAttribute(attn_variate_simt_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(simt_smem()));
        if (e != cudaSuccess) return e;
        configured.done(dev, ctx_key);
    }
    const int64_t blocks = int64_t(rows) * mm.S * ((H + SIMT_WARPS - 1) / SIMT_WARPS);
    attn_variate_simt_kernel<T><<<unsigned(blocks), SIMT_WARPS * 32, simt_smem(), stream>>>(q, k, v, gate, out, rows, H, hd, mm);
    return cudaGetLastError();
}

cudaError_t attention_variate_fast(const __half* q, const __half* k, const __half* v, const __half* gate, __half* out,
                                   int rows, int H, int G, const MaskMeta& mm, cudaStream_t stream) {
    if (rows <= 0) return cudaSuccess;
    if (G <= 0 || G > 64 || rows % G || mm.S <= 0) return cudaErrorInvalidValue;
    const int64_t problems = int64_t(rows / G) * H * mm.S;
    const unsigned blocks = unsigned((problems + VF_WARPS - 1) / VF_WARPS);
    // Both variants use more than the default 48 KB of dynamic shared memory.
    static KernelSetup configured;
    const size_t smem1 = VF_WARPS * (2 * 32 * 64 + 32) * sizeof(float);
    const size_t smem2 = VF_WARPS * (2 * 64 * 64 + 64) * sizeof(float);
    int dev = 0;
    cudaGetDevice(&dev);
    unsigned long long ctx_key = 0;
    if (configured.needed(dev, &ctx_key)) {
        cudaError_t e = cudaFuncSetAttribute(attn_variate_fast_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem1));
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(attn_variate_fast_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem2));
        if (e != cudaSuccess) return e;
        configured.done(dev, ctx_key);
    }
    if (G <= 32)
        attn_variate_fast_kernel<1><<<blocks, VF_WARPS * 32, smem1, stream>>>(q, k, v, gate, out, rows, H, G, mm);
    else
        attn_variate_fast_kernel<2><<<blocks, VF_WARPS * 32, smem2, stream>>>(q, k, v, gate, out, rows, H, G, mm);
    return cudaGetLastError();
}

template cudaError_t attention_time_simt<float>(const float*, const float*, const float*, const float*, float*, int, int, int,
                                                const MaskMeta&, cudaStream_t, int);
template cudaError_t attention_time_simt<__half>(const __half*, const __half*, const __half*, const __half*, __half*, int,
                                                 int, int, const MaskMeta&, cudaStream_t, int);
template cudaError_t attention_variate_simt<float>(const float*, const float*, const float*, const float*, float*, int, int,
                                                   int, const MaskMeta&, cudaStream_t);
template cudaError_t attention_variate_simt<__half>(const __half*, const __half*, const __half*, const __half*, __half*,
                                                    int, int, int, const MaskMeta&, cudaStream_t);

}  // namespace tsb
