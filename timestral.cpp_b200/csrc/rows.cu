// Per-row / per-token kernels of the forecast path. Built with -fmad=false: like the
// reference's F32 path (built with -ffp-contract=off), no multiply-add is fused unless an
// explicit fma appears in the source.
#include "common.cuh"
#include "rows.cuh"

#include <cfloat>
#include <cmath>

namespace tsb {

namespace {

constexpr int TPB = 256;

inline unsigned blocks_for(int64_t n, int tpb = TPB) { return unsigned((n + tpb - 1) / tpb); }

// ---------------------------------------------------------------------------------------
// Assembly of target rows (reference src/covariates.cpp:48-50,69-70).
// Target row i = b * V + v of the request goes to row (i / V) * all + i % V (all = rows per
// series: V when there are no covariates), its negation to row `mirror_rows` + that row.
// first_obs (optional): first observed step of each target row, T if none.
__global__ void assemble_kernel(const float* __restrict__ ctx, const uint8_t* __restrict__ umask, int BV, int T,
                                int kept, int len, int mirrored, int V, int all, int64_t mirror_rows,
                                float* __restrict__ rows, int8_t* __restrict__ mask, int* __restrict__ first_obs) {
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) / 32, lane = threadIdx.x & 31;
    if (warp >= BV) return;
    const int r = warp, pad = len - kept, start = T - kept;
    const int64_t orow = int64_t(r / V) * all + r % V;
    const float* x = ctx + int64_t(r) * T;
    const uint8_t* um = umask ? umask + int64_t(r) * T : nullptr;
    float* out = rows + orow * len;
    int8_t* om = mask + orow * len;
    float* out2 = mirrored ? rows + (mirror_rows + orow) * len : nullptr;
    int8_t* om2 = mirrored ? mask + (mirror_rows + orow) * len : nullptr;
    int first = T;
    for (int t = lane; t < pad; t += 32) {
        out[t] = 0.f; om[t] = 0;
        if (out2) { out2[t] = -0.f; om2[t] = 0; }
    }
    float carry = 0.f;  // value of the last observed step before the chunk
    for (int c0 = 0; c0 < T; c0 += 32) {
        const int t = c0 + lane;
        float v = 0.f;
        bool obs = false;
        if (t < T) { v = x[t]; obs = isfinite(v) && (!um || um[t]); }
        int idx = obs ? lane : -1;
        // inclusive max-scan of the last observed lane
        for (int o = 1; o < 32; o <<= 1) {
            const int other = __shfl_up_sync(0xffffffffu, idx, o);
            if (lane >= o) idx = max(idx, other);
        }
        const float src = __shfl_sync(0xffffffffu, v, idx < 0 ? 0 : idx);
        const float filled = idx < 0 ? carry : src;
        const int last = __shfl_sync(0xffffffffu, idx, 31);
        const float last_val = __shfl_sync(0xffffffffu, v, last < 0 ? 0 : last);
        if (last >= 0) carry = last_val;
        const unsigned seen = __ballot_sync(0xffffffffu, obs);
        if (first == T && seen) first = c0 + __ffs(seen) - 1;
        if (t < T && t >= start) {
            const int o = pad + t - start;
            out[o] = filled; om[o] = obs;
            if (out2) { out2[o] = -filled; om2[o] = obs; }
        }
    }
    if (first_obs && lane == 0) first_obs[r] = first;
}

// ---------------------------------------------------------------------------------------
// Covariate rows (reference src/covariates.cpp:32-72): per series b the rows are the V
// targets, P past, CP categorical past, K known, CK categorical known covariates.
__device__ __forceinline__ float finite_value(float v) {
    return isnan(v) ? 0.f : isinf(v) ? copysignf(FLT_MAX, v) : v;
}

// One warp per covariate row (and per target row for its zero future): the kept context
// window (left-padded to len) as finite values with the not-NaN mask, the known rows' future
// steps, roles, and the negated copies of the mirrored pass.
__global__ void cov_rows_kernel(const CovShape c, const float* __restrict__ past, const float* __restrict__ known,
                                const double* __restrict__ cat_past, const double* __restrict__ cat_known,
                                const float* __restrict__ enc_past, const float* __restrict__ enc_known,
                                float* __restrict__ rows, int8_t* __restrict__ mask, int8_t* __restrict__ role,
                                float* __restrict__ future, int8_t* __restrict__ fmask) {
    const int all = c.V + c.P + c.CP + c.K + c.CK;
    const int64_t R = int64_t(c.B) * all;
    const int64_t warp = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) / 32;
    const int lane = threadIdx.x & 31;
    if (warp >= R) return;
    const int b = int(warp / all), j = int(warp % all);
    const int TH = c.T + c.H, pad = c.len - c.kept, start = c.T - c.kept;
    int kind;                 // 0 target, 1 past, 2 categorical past, 3 known, 4 categorical known
    int64_t off = 0;
    int jj = j;
    if (jj < c.V) kind = 0;
    else if ((jj -= c.V) < c.P) { kind = 1; off = (int64_t(b) * c.P + jj) * c.T; }
    else if ((jj -= c.P) < c.CP) { kind = 2; off = (int64_t(b) * c.CP + jj) * c.T; }
    else if ((jj -= c.CP) < c.K) { kind = 3; off = (int64_t(b) * c.K + jj) * TH; }
    else { jj -= c.K; kind = 4; off = (int64_t(b) * c.CK + jj) * TH; }
    const int rl = kind == 0 ? 0 : kind <= 2 ? 1 : 2;
    const bool encoded = c.V == 1;
    auto value = [&](int t) -> float {        // step t of the row's source (t < T + H)
        switch (kind) {
            case 1: return past[off + t];
            case 2: return encoded ? enc_past[off + t] : float(cat_past[off + t]);
            case 3: return known[off + t];
            default: return encoded ? enc_known[off + t] : float(cat_known[off + t]);
        }
    };
    if (lane == 0) {
        if (role) role[warp] = int8_t(rl);
        if (role && c.mirrored) role[R + warp] = int8_t(rl);
    }
    if (kind != 0) {
        float* out = rows + warp * c.len;
        int8_t* om = mask + warp * c.len;
        for (int t = lane; t < c.len; t += 32) {
            float y = 0.f;
            int8_t m = 0;
            if (t >= pad) {
                const float v = value(start + t - pad);
                y = finite_value(v);
                m = !isnan(v);
            }
            out[t] = y; om[t] = m;
            if (c.mirrored) { rows[(R + warp) * c.len + t] = -y; mask[(R + warp) * c.len + t] = m; }
        }
    }
    if (future) {
        for (int t = lane; t < c.hor; t += 32) {
            float y = 0.f;
            int8_t m = 0;
            if (rl == 2 && t < c.H) {
                const float v = value(c.T + t);
                y = finite_value(v);
                m = !isnan(v);
            }
            future[warp * c.hor + t] = y; fmask[warp * c.hor + t] = m;
            if (c.mirrored) { future[(R + warp) * c.hor + t] = -y; fmask[(R + warp) * c.hor + t] = m; }
        }
    }
}

// Smoothed mean target encoding of one categorical row of a one-target series (reference
// src/covariates.cpp:14-25), one block per (series, categorical row). The categories are the
// distinct non-NaN codes of the context part; each category's sum of target values runs in
// step order (the codes are sorted with their step as the tie-break), the target mean is the
// NumPy pairwise sum over the context divided by the count of finite targets. Context steps
// whose target and code are both NaN stay NaN; future codes absent from the context take the
// mean. Scratch per block: values [Tp] f64, order [Tp] i32, lookups [T] f32.
constexpr int ENC_THREADS = 256;
__device__ double numpy_sum_dev(const double* x, int n);   // NumPy pairwise sum, defined with refine

__device__ __forceinline__ bool code_before(const double* code, int a, int b) {
    if (a < 0) return false;                  // padding sorts last
    if (b < 0) return true;
    const double ca = code[a], cb = code[b];
    const bool na = isnan(ca), nb = isnan(cb);
    if (na != nb) return nb;                  // NaN codes after the categories
    if (!na && ca != cb) return ca < cb;
    return a < b;
}
__device__ __forceinline__ bool same_code(double a, double b) { return (isnan(a) && isnan(b)) || a == b; }

__global__ void __launch_bounds__(ENC_THREADS)
    target_encode_kernel(const CovShape c, const float* __restrict__ rows, const int* __restrict__ first_obs,
                         const double* __restrict__ cat_past, const double* __restrict__ cat_known,
                         float* __restrict__ enc_past, float* __restrict__ enc_known, double* __restrict__ scratch,
                         int Tp) {
    const int per = c.CP + c.CK;
    const int b = blockIdx.x / per, k = blockIdx.x % per, tid = threadIdx.x;
    const int all = c.V + c.P + c.CP + c.K + c.CK, T = c.T, TH = c.T + c.H;
    const bool is_known = k >= c.CP;
    const int width = is_known ? TH : T;
    const double* code = is_known ? cat_known + (int64_t(b) * c.CK + (k - c.CP)) * TH : cat_past + (int64_t(b) * c.CP + k) * T;
    float* enc = is_known ? enc_known + (int64_t(b) * c.CK + (k - c.CP)) * TH : enc_past + (int64_t(b) * c.CP + k) * T;
    double* values = scratch + int64_t(blockIdx.x) * Tp * 2;
    int* order = reinterpret_cast<int*>(values + Tp);
    float* lookup = reinterpret_cast<float*>(order + Tp);
    const float* filled = rows + int64_t(b) * all * c.len + (c.len - c.kept);   // the series' target row
    const int start = T - c.kept, first = first_obs[b];
    __shared__ int count_sh;
    __shared__ double mean_sh, nan_lookup_sh;
    __shared__ int has_nan_sh;
    if (tid == 0) { count_sh = 0; has_nan_sh = 0; }
    __syncthreads();
    // target values: the forward-filled target from its first observation, inside the kept window
    int cnt = 0;
    for (int i = tid; i < Tp; i += ENC_THREADS) {
        double v = 0.0;
        if (i < T && i >= start && i >= first) { v = double(filled[i - start]); cnt += isfinite(v) ? 1 : 0; }
        if (i < T && !isfinite(v)) v = 0.0;
        values[i] = v;
        order[i] = i < T ? i : -1;
    }
    atomicAdd(&count_sh, cnt);
    __syncthreads();
    if (tid == 0) mean_sh = count_sh ? __ddiv_rn(numpy_sum_dev(values, T), double(count_sh)) : 0.0;
    // bitonic sort of the steps by (code, step)
    for (int size = 2; size <= Tp; size <<= 1)
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            __syncthreads();
            for (int i = tid; i < Tp; i += ENC_THREADS) {
                const int jx = i ^ stride;
                if (jx > i) {
                    const int a = order[i], bb = order[jx];
                    const bool up = (i & size) == 0;
                    if (up ? code_before(code, bb, a) : code_before(code, a, bb)) { order[i] = bb; order[jx] = a; }
                }
            }
        }
    __syncthreads();
    const double mean = mean_sh, smooth = c.smooth;
    // one thread per category: its sum in step order, its count, its lookup value
    for (int kk = tid; kk < T; kk += ENC_THREADS) {
        const int i0 = order[kk];
        if (kk > 0 && same_code(code[order[kk - 1]], code[i0])) continue;
        double sum = 0.0, n = 0.0;
        int e = kk;
        for (; e < T && same_code(code[order[e]], code[i0]); ++e) {
            const int i = order[e];
            sum = __dadd_rn(sum, values[i]);
            const bool fin = i >= start && i >= first && isfinite(filled[i - start]);
            n = __dadd_rn(n, fin ? 1.0 : 0.0);
        }
        const double lk = __ddiv_rn(__dadd_rn(__dmul_rn(smooth, mean), sum), __dadd_rn(smooth, n));
        for (int e2 = kk; e2 < e; ++e2) lookup[order[e2]] = float(lk);
        if (isnan(code[i0])) { nan_lookup_sh = lk; has_nan_sh = 1; }
    }
    __syncthreads();
    if (tid == 0 && !has_nan_sh)
        nan_lookup_sh = __ddiv_rn(__dadd_rn(__dmul_rn(smooth, mean), 0.0), __dadd_rn(smooth, 0.0));
    __syncthreads();
    // number of non-NaN codes in the context part (they sort first)
    __shared__ int finite_sh;
    if (tid == 0) {
        int lo = 0, hi = T;
        while (lo < hi) { const int mid = (lo + hi) >> 1; if (isnan(code[order[mid]])) hi = mid; else lo = mid + 1; }
        finite_sh = lo;
    }
    __syncthreads();
    const int nf = finite_sh;
    for (int i = tid; i < width; i += ENC_THREADS) {
        if (i < T) {
            const bool tgt_nan = !(i >= start && i >= first) || !isfinite(filled[i - start]);
            enc[i] = (tgt_nan && isnan(code[i])) ? NAN : lookup[i];
        } else {
            const double f = code[i];
            float v;
            if (isnan(f)) {
                v = float(nan_lookup_sh);
            } else {
                int lo = 0, hi = nf;
                while (lo < hi) { const int mid = (lo + hi) >> 1; if (code[order[mid]] < f) lo = mid + 1; else hi = mid; }
                v = (lo < nf && code[order[lo]] == f) ? lookup[order[lo]] : float(mean);
            }
            enc[i] = v;
        }
    }
}

__global__ void clip_ok_kernel(const float* __restrict__ ctx, const uint8_t* __restrict__ umask, int BV, int T,
                               int8_t* __restrict__ ok) {
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) / 32, lane = threadIdx.x & 31;
    if (warp >= BV) return;
    bool any = false, eligible = true;
    for (int t = lane; t < T; t += 32) {
        const int64_t i = int64_t(warp) * T + t;
        const float v = ctx[i];
        const bool observed = isfinite(v) && (!umask || umask[i]);
        if (observed) { any = true; eligible &= v >= 0.f; }
    }
    any = __any_sync(0xffffffffu, any);
    eligible = __all_sync(0xffffffffu, eligible);
    if (lane == 0) ok[warp] = any && eligible;
}

// ---------------------------------------------------------------------------------------
// Causal scaler (reference src/scaler.cpp:27-58) and patch features (src/encoder.cpp:12-23).
__device__ __forceinline__ float affine_value(float x, float loc, float scale, bool observed, bool squash) {
    const float y = __fdiv_rn(__fsub_rn(x, loc), fmaxf(scale, FLT_EPSILON));
    if (!observed) return 0.0f;
    return squash ? asinhf(y) : y;
}

__global__ void scale_kernel(const RowConfig c, const float* __restrict__ rows, const int8_t* __restrict__ mask, int R,
                             int W, int anchor_step, int enc_patches, int kv_words, float* __restrict__ features,
                             float* __restrict__ aloc, float* __restrict__ ascale, uint32_t* __restrict__ key_valid,
                             int* __restrict__ first_obs, int ctx_len, float* __restrict__ cap_lo,
                             float* __restrict__ cap_hi, float* __restrict__ cap_scale) {
    const int r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= R) return;
    const int ps = c.ps;
    const float* x = rows + int64_t(r) * W;
    const int8_t* m = mask + int64_t(r) * W;
    float* feat = features + int64_t(r) * (W / ps) * 2 * ps;
    double cum_w = 0, cum_x = 0, prev_mean = 0, m2 = 0;
    bool started = false;
    int first = -1;
    uint32_t word = 0;
    float lo = INFINITY, hi = -INFINITY;
    for (int t = 0; t < W; ++t) {
        const double v = x[t], w = m[t];
        cum_w = __dadd_rn(cum_w, w);
        cum_x = __dadd_rn(cum_x, __dmul_rn(w, v));
        const double den = fmax(cum_w, 1.0);
        const double mean = __ddiv_rn(cum_x, den);
        const double inc = __dmul_rn(__dmul_rn(__dsub_rn(v, prev_mean), __dsub_rn(v, mean)), w);
        m2 = __dadd_rn(m2, inc);
        prev_mean = mean;
        if (t < ctx_len && m[t]) { lo = fminf(lo, x[t]); hi = fmaxf(hi, x[t]); }
        if ((t + 1) % ps == 0) {
            const int p = t / ps;
            const float loc = float(mean);
            const float scale = float(fmax(sqrt(__ddiv_rn(m2, fmax(__dsub_rn(den, 1.0), 1.0))), c.minimum_scale));
            bool obs = false;
            float* f = feat + int64_t(p) * 2 * ps;
            for (int j = 0; j < ps; ++j) {
                const int tj = t + 1 - ps + j;
                const bool o = m[tj] != 0;
                obs |= o;
                f[j] = affine_value(x[tj], loc, scale, o, c.use_asinh);
                f[ps + j] = o ? 0.f : 1.f;
            }
            if (p < enc_patches) {
                started |= obs;
                if (obs && first < 0) first = p;
                if (obs || (c.attend_missing && started)) word |= 1u << (p & 31);
                if ((p & 31) == 31 || p == enc_patches - 1) {
                    key_valid[int64_t(r) * kv_words + (p >> 5)] = word;
                    word = 0;
                }
            }
            if (anchor_step >= t + 1 - ps && anchor_step <= t) { aloc[r] = loc; ascale[r] = scale; }
            if (cap_scale && ctx_len - 1 >= t + 1 - ps && ctx_len - 1 <= t) cap_scale[r] = scale;
        }
    }
    first_obs[r] = first;
    if (cap_lo) {
        cap_lo[r] = isfinite(lo) ? lo : 0.f;
        cap_hi[r] = isfinite(hi) ? hi : 0.f;
    }
}

// The same scaler with one block per row, for long rows: thread 0 runs the reference's two
// float64 recurrences (the masked running sum, then the running sum of deviation terms) in
// their order, and nothing else; the products, the running weight (an integer count, so its
// prefix sums are exact in any order), the divisions, deviation terms, patch statistics,
// features and key-valid words are computed by all threads, over chunks of the row staged
// in shared memory. Every value is produced by the same operations as in scale_kernel, so
// the results are identical (the cap minimum and maximum are order-independent).
constexpr int SC_THREADS = 128;
constexpr int SC_CHUNK = 1024;
constexpr int SC_PER = SC_CHUNK / SC_THREADS;   // consecutive steps per thread in the count scan

__global__ void __launch_bounds__(SC_THREADS)
    scale_block_kernel(const RowConfig c, const float* __restrict__ rows, const int8_t* __restrict__ mask, int W,
                       int anchor_step, int enc_patches, int kv_words, float* __restrict__ features,
                       float* __restrict__ aloc, float* __restrict__ ascale, uint32_t* __restrict__ key_valid,
                       int* __restrict__ first_obs, int ctx_len, float* __restrict__ cap_lo,
                       float* __restrict__ cap_hi, float* __restrict__ cap_scale) {
    __shared__ float xs[SC_CHUNK];
    __shared__ int8_t mk[SC_CHUNK];
    __shared__ double cx[SC_CHUNK];      // w * x, then the running sum, then the running mean
    __shared__ double dn[SC_CHUNK];      // max(running weight, 1)
    __shared__ double dv[SC_CHUNK];      // deviation terms, then the running m2 at patch ends
    __shared__ float ploc[SC_CHUNK], pscale[SC_CHUNK];
    __shared__ int8_t pobs[SC_CHUNK];
    __shared__ int wsum[SC_THREADS / 32];
    __shared__ float wlo[SC_THREADS / 32], whi[SC_THREADS / 32];
    __shared__ double prev_mean_sh;
    __shared__ long long weight_sh;
    const int r = blockIdx.x, tid = threadIdx.x, lane = tid & 31, wid = tid >> 5, ps = c.ps;
    const int chunk = (SC_CHUNK / ps) * ps;
    const float* x = rows + int64_t(r) * W;
    const int8_t* m = mask + int64_t(r) * W;
    float* feat = features + int64_t(r) * (W / ps) * 2 * ps;
    // thread 0's sequential state
    double cum_x = 0, m2 = 0;
    bool started = false;
    int first = -1;
    uint32_t word = 0;
    float lo = INFINITY, hi = -INFINITY;    // this thread's share of the cap statistics
    if (tid == 0) { prev_mean_sh = 0.0; weight_sh = 0; }
    for (int c0 = 0; c0 < W; c0 += chunk) {
        const int n = min(chunk, W - c0);
        for (int i = tid; i < n; i += SC_THREADS) {
            const float v = x[c0 + i];
            const int8_t w = m[c0 + i];
            xs[i] = v;
            mk[i] = w;
            cx[i] = __dmul_rn(double(w), double(v));
            if (c0 + i < ctx_len && w) { lo = fminf(lo, v); hi = fmaxf(hi, v); }
        }
        __syncthreads();
        // running weight: block-wide inclusive scan of the mask over steps [tid*8, tid*8+8)
        {
            int part[SC_PER], run = 0;
#pragma unroll
            for (int k = 0; k < SC_PER; ++k) {
                const int i = tid * SC_PER + k;
                run += i < n ? int(mk[i]) : 0;
                part[k] = run;
            }
            int incl = run;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int y = __shfl_up_sync(0xffffffffu, incl, o);
                if (lane >= o) incl += y;
            }
            if (lane == 31) wsum[wid] = incl;
            __syncthreads();
            long long base = weight_sh;
            for (int w = 0; w < wid; ++w) base += wsum[w];
            base += incl - run;
#pragma unroll
            for (int k = 0; k < SC_PER; ++k) {
                const int i = tid * SC_PER + k;
                if (i < n) dn[i] = fmax(double(base + part[k]), 1.0);
            }
        }
        __syncthreads();
        if (tid == 0) {
            long long total = weight_sh;
            for (int w = 0; w < SC_THREADS / 32; ++w) total += wsum[w];
            weight_sh = total;
            // the running sum, eight products loaded ahead
            int i = 0;
            for (; i + 8 <= n; i += 8) {
                double a[8];
#pragma unroll
                for (int k = 0; k < 8; ++k) a[k] = cx[i + k];
#pragma unroll
                for (int k = 0; k < 8; ++k) { cum_x = __dadd_rn(cum_x, a[k]); cx[i + k] = cum_x; }
            }
            for (; i < n; ++i) { cum_x = __dadd_rn(cum_x, cx[i]); cx[i] = cum_x; }
        }
        __syncthreads();
        for (int i = tid; i < n; i += SC_THREADS) cx[i] = __ddiv_rn(cx[i], dn[i]);
        __syncthreads();
        for (int i = tid; i < n; i += SC_THREADS) {
            const double v = xs[i], w = mk[i];
            const double pm = i == 0 ? prev_mean_sh : cx[i - 1];
            dv[i] = __dmul_rn(__dmul_rn(__dsub_rn(v, pm), __dsub_rn(v, cx[i])), w);
        }
        __syncthreads();
        const int np = n / ps;
        if (tid == 0) {
            // the m2 chain, eight terms loaded ahead; m2 is kept at each patch end
            int i = 0;
            if ((ps & 7) == 0) {
                for (int pp = 0; pp < np; ++pp) {
                    for (int j = 0; j < ps; j += 8, i += 8) {
                        double d[8];
#pragma unroll
                        for (int k = 0; k < 8; ++k) d[k] = dv[i + k];
#pragma unroll
                        for (int k = 0; k < 8; ++k) m2 = __dadd_rn(m2, d[k]);
                    }
                    dv[i - 1] = m2;
                }
            } else {
                for (int pp = 0; pp < np; ++pp) {
                    for (int j = 0; j < ps; ++j, ++i) m2 = __dadd_rn(m2, dv[i]);
                    dv[i - 1] = m2;
                }
            }
            for (; i < n; ++i) m2 = __dadd_rn(m2, dv[i]);
            prev_mean_sh = cx[n - 1];
        }
        __syncthreads();
        for (int pp = tid; pp < np; pp += SC_THREADS) {
            const int te = (pp + 1) * ps - 1, t0 = c0 + pp * ps;
            const float loc = float(cx[te]);
            const float scale = float(fmax(sqrt(__ddiv_rn(dv[te], fmax(__dsub_rn(dn[te], 1.0), 1.0))), c.minimum_scale));
            ploc[pp] = loc;
            pscale[pp] = scale;
            bool obs = false;
            for (int j = 0; j < ps; ++j) obs |= mk[pp * ps + j] != 0;
            pobs[pp] = obs;
            if (anchor_step >= t0 && anchor_step <= t0 + ps - 1) { aloc[r] = loc; ascale[r] = scale; }
            if (cap_scale && ctx_len - 1 >= t0 && ctx_len - 1 <= t0 + ps - 1) cap_scale[r] = scale;
        }
        __syncthreads();
        float* f = feat + int64_t(c0 / ps) * 2 * ps;
        for (int e = tid; e < np * ps; e += SC_THREADS) {
            const int pp = e / ps, j = e - pp * ps;
            const bool o = mk[e] != 0;
            f[int64_t(pp) * 2 * ps + j] = affine_value(xs[e], ploc[pp], pscale[pp], o, c.use_asinh);
            f[int64_t(pp) * 2 * ps + ps + j] = o ? 0.f : 1.f;
        }
        if (tid == 0) {
            for (int pp = 0; pp < np; ++pp) {
                const int p = c0 / ps + pp;
                if (p >= enc_patches) break;
                const bool obs = pobs[pp];
                started |= obs;
                if (obs && first < 0) first = p;
                if (obs || (c.attend_missing && started)) word |= 1u << (p & 31);
                if ((p & 31) == 31 || p == enc_patches - 1) {
                    key_valid[int64_t(r) * kv_words + (p >> 5)] = word;
                    word = 0;
                }
            }
        }
        __syncthreads();
    }
    // cap statistics: minimum and maximum over the observed steps of the context
#pragma unroll
    for (int o = 16; o; o >>= 1) {
        lo = fminf(lo, __shfl_xor_sync(0xffffffffu, lo, o));
        hi = fmaxf(hi, __shfl_xor_sync(0xffffffffu, hi, o));
    }
    if (lane == 0) { wlo[wid] = lo; whi[wid] = hi; }
    __syncthreads();
    if (tid == 0) {
        first_obs[r] = first;
        if (cap_lo) {
            for (int w = 1; w < SC_THREADS / 32; ++w) { lo = fminf(lo, wlo[w]); hi = fmaxf(hi, whi[w]); }
            cap_lo[r] = isfinite(lo) ? lo : 0.f;
            cap_hi[r] = isfinite(hi) ? hi : 0.f;
        }
    }
}

// ---------------------------------------------------------------------------------------
// Float sum cascade of ATen's contiguous reduction, one warp per sequence: lane j holds the
// accumulators of lane slot (k, l) = (j / 8, j % 8) (reference src/torch_sum.hpp:9-23,
// src/layers.cpp:262-278). `sq` squares each element; `small` enables the four-partial
// path for length < 8 of the plain sum.
template <class F>
__device__ float warp_cascade(F val, int length, bool small_path) {
    const int lane = threadIdx.x & 31;
    if (small_path && length < 8) {
        float total = 0.f;
        if (lane == 0) {
            float partial[4] = {0.f, 0.f, 0.f, 0.f};
            int i = 0;
            for (; i + 4 <= length; i += 4) for (int j = 0; j < 4; ++j) partial[j] = __fadd_rn(partial[j], val(i + j));
            for (; i < length; ++i) partial[0] = __fadd_rn(partial[0], val(i));
            for (int j = 1; j < 4; ++j) partial[0] = __fadd_rn(partial[0], partial[j]);
            total = partial[0];
        }
        return __shfl_sync(0xffffffffu, total, 0);
    }
    float acc0 = 0.f, acc1 = 0.f, acc2 = 0.f, acc3 = 0.f;
    const int groups = length / 32;
    int log = 0;
    for (int n = groups ? groups - 1 : 0; n; n >>= 1) ++log;
    const int power = max(4, log / 4);
    const int step = 1 << power, msk = step - 1;
    int i = 0;
    for (; i + step <= groups;) {
        for (int j = 0; j < step; ++j, ++i) acc0 = __fadd_rn(acc0, val(i * 32 + lane));
        // level 1..3 promotions, with the early break of the reference
        acc1 = __fadd_rn(acc1, acc0); acc0 = 0.f;
        if (i & (msk << power)) continue;
        acc2 = __fadd_rn(acc2, acc1); acc1 = 0.f;
        if (i & (msk << (2 * power))) continue;
        acc3 = __fadd_rn(acc3, acc2); acc2 = 0.f;
    }
    for (; i < groups; ++i) acc0 = __fadd_rn(acc0, val(i * 32 + lane));
    acc0 = __fadd_rn(acc0, acc1);
    acc0 = __fadd_rn(acc0, acc2);
    acc0 = __fadd_rn(acc0, acc3);
    int v = groups * 4;
    if (lane < 8) for (int vv = v; vv < length / 8; ++vv) acc0 = __fadd_rn(acc0, val(vv * 8 + lane));
    v = max(v, length / 8);
    // acc[0][0][l] += acc[0][k][l] for k = 1, 2, 3
    const float k1 = __shfl_sync(0xffffffffu, acc0, (lane & 7) + 8);
    const float k2 = __shfl_sync(0xffffffffu, acc0, (lane & 7) + 16);
    const float k3 = __shfl_sync(0xffffffffu, acc0, (lane & 7) + 24);
    float a = __fadd_rn(__fadd_rn(__fadd_rn(acc0, k1), k2), k3);
    float sum = 0.f;
    float lanes[8];
#pragma unroll
    for (int l = 0; l < 8; ++l) lanes[l] = __shfl_sync(0xffffffffu, a, l);
    if (lane == 0) {
        for (int d = v * 8; d < length; ++d) sum = __fadd_rn(sum, val(d));
        for (int l = 0; l < 8; ++l) sum = __fadd_rn(sum, lanes[l]);
    }
    return __shfl_sync(0xffffffffu, sum, 0);
}

__global__ void rms_kernel(const float* __restrict__ x, const float* __restrict__ w, int tokens, int D, float eps,
                           void* __restrict__ out, int out_f16, int sub, int S, int off) {
    const int i = (blockIdx.x * blockDim.x + threadIdx.x) / 32, lane = threadIdx.x & 31;
    if (i >= tokens) return;
    const int64_t tok = sub ? int64_t(i / sub) * S + off + i % sub : i;
    const float* xr = x + tok * D;
    const float ssq = warp_cascade([&](int d) { const float a = xr[d]; return __fmul_rn(a, a); }, D, false);
    const float mean = __fdiv_rn(ssq, float(D));
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, eps)));
    if (out_f16) {
        __half* o = static_cast<__half*>(out) + int64_t(i) * D;
        for (int d = lane; d < D; d += 32) o[d] = __float2half_rn(__fmul_rn(__fmul_rn(xr[d], inv), w[d]));
    } else {
        float* o = static_cast<float*>(out) + int64_t(i) * D;
        for (int d = lane; d < D; d += 32) o[d] = __fmul_rn(__fmul_rn(xr[d], inv), w[d]);
    }
}

// RMSNorm for widths D = 32 * G: the token's row is loaded into registers with all G loads of
// a lane in flight at once, then summed in exactly warp_cascade's order (no tail terms exist
// when D is a multiple of 32) and normalised from the registers.
__host__ __device__ constexpr int bit_length(int n) { return n ? 1 + bit_length(n >> 1) : 0; }

template <int G>
__global__ void rms_regs_kernel(const float* __restrict__ x, const float* __restrict__ w, int tokens, float eps,
                                void* __restrict__ out, int out_f16, int sub, int S, int off) {
    constexpr int D = 32 * G;
    const int i = (blockIdx.x * blockDim.x + threadIdx.x) / 32, lane = threadIdx.x & 31;
    if (i >= tokens) return;
    const int64_t tok = sub ? int64_t(i / sub) * S + off + i % sub : i;
    const float* xr = x + tok * D;
    float v[G];
#pragma unroll
    for (int g = 0; g < G; ++g) v[g] = __ldcs(xr + g * 32 + lane);
    // warp_cascade with groups = G: blocks of STEP terms promoted through acc1..acc3.
    constexpr int POWER = bit_length(G - 1) / 4 > 4 ? bit_length(G - 1) / 4 : 4;
    constexpr int STEP = 1 << POWER, MSK = STEP - 1;
    float acc0 = 0.f, acc1 = 0.f, acc2 = 0.f, acc3 = 0.f;
#pragma unroll
    for (int b = 0; b < G / STEP; ++b) {
#pragma unroll
        for (int j = 0; j < STEP; ++j) acc0 = __fadd_rn(acc0, __fmul_rn(v[b * STEP + j], v[b * STEP + j]));
        const int done = (b + 1) * STEP;
        acc1 = __fadd_rn(acc1, acc0); acc0 = 0.f;
        if (done & (MSK << POWER)) continue;
        acc2 = __fadd_rn(acc2, acc1); acc1 = 0.f;
        if (done & (MSK << (2 * POWER))) continue;
        acc3 = __fadd_rn(acc3, acc2); acc2 = 0.f;
    }
#pragma unroll
    for (int g = (G / STEP) * STEP; g < G; ++g) acc0 = __fadd_rn(acc0, __fmul_rn(v[g], v[g]));
    acc0 = __fadd_rn(acc0, acc1);
    acc0 = __fadd_rn(acc0, acc2);
    acc0 = __fadd_rn(acc0, acc3);
    const float k1 = __shfl_sync(0xffffffffu, acc0, (lane & 7) + 8);
    const float k2 = __shfl_sync(0xffffffffu, acc0, (lane & 7) + 16);
    const float k3 = __shfl_sync(0xffffffffu, acc0, (lane & 7) + 24);
    const float a = __fadd_rn(__fadd_rn(__fadd_rn(acc0, k1), k2), k3);
    float ssq = 0.f;
#pragma unroll
    for (int l = 0; l < 8; ++l) ssq = __fadd_rn(ssq, __shfl_sync(0xffffffffu, a, l));
    const float mean = __fdiv_rn(ssq, float(D));
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, eps)));
    if (out_f16) {
        __half* o = static_cast<__half*>(out) + int64_t(i) * D;
#pragma unroll
        for (int g = 0; g < G; ++g) o[g * 32 + lane] = __float2half_rn(__fmul_rn(__fmul_rn(v[g], inv), w[g * 32 + lane]));
    } else {
        float* o = static_cast<float*>(out) + int64_t(i) * D;
#pragma unroll
        for (int g = 0; g < G; ++g) o[g * 32 + lane] = __fmul_rn(__fmul_rn(v[g], inv), w[g * 32 + lane]);
    }
}

// Known covariate rows: non-causal float statistics (reference src/scaler.cpp:60-107).
__global__ void known_kernel(const RowConfig c, const float* __restrict__ rows, const int8_t* __restrict__ mask,
                             const int8_t* __restrict__ role, int R, int W, int anchor_step, float* __restrict__ features,
                             float* __restrict__ aloc, float* __restrict__ ascale) {
    const int r = (blockIdx.x * blockDim.x + threadIdx.x) / 32, lane = threadIdx.x & 31;
    if (r >= R || role[r] != 2) return;
    const float* x = rows + int64_t(r) * W;
    const int8_t* m = mask + int64_t(r) * W;
    bool binary = true, any = false;
    for (int t = lane; t < W; t += 32) {
        any |= m[t] != 0;
        binary &= !m[t] || x[t] == 0.f || x[t] == 1.f;
    }
    any = __any_sync(0xffffffffu, any);
    binary = __all_sync(0xffffffffu, binary);
    const float n = fmaxf(warp_cascade([&](int t) { return float(m[t]); }, W, true), 1.0f);
    const float loc = __fdiv_rn(warp_cascade([&](int t) { return __fmul_rn(x[t], float(m[t])); }, W, true), n);
    const float var = __fdiv_rn(warp_cascade([&](int t) {
                                    const float cen = __fmul_rn(__fsub_rn(x[t], loc), float(m[t]));
                                    return __fmul_rn(cen, cen);
                                }, W, true), n);
    const float scale = fmaxf(__fsqrt_rn(var), float(c.minimum_scale));
    const bool is_bin = binary && any;
    const float L = is_bin ? 0.0f : loc, Sc = is_bin ? 1.0f : scale;
    const int ps = c.ps;
    float* feat = features + int64_t(r) * (W / ps) * 2 * ps;
    for (int t = lane; t < W; t += 32) {
        const int p = t / ps, j = t % ps;
        feat[int64_t(p) * 2 * ps + j] = affine_value(x[t], L, Sc, m[t] != 0, c.use_asinh && !is_bin);
    }
    if (lane == 0) { aloc[r] = L; ascale[r] = Sc; }
    (void)anchor_step;
}

// Positions and groups (reference src/masks.cpp:13-18).
__global__ void positions_kernel(const RowConfig c, const int* __restrict__ first_obs, int R, int group_rows, int N,
                                 int S, int cov, int* __restrict__ rope_row, int* __restrict__ gbegin,
                                 int* __restrict__ gsize, int* err) {
    const int r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= R) return;
    const int g0 = (r / group_rows) * group_rows;
    int first = N;
    for (int j = 0; j < group_rows; ++j) {
        const int f = first_obs[g0 + j];
        if (f >= 0 && f < first) first = f;
    }
    if (first == N) first = 0;
    for (int p = 0; p < S; ++p) {
        const int pos = (cov ? p % N : p) - first;
        const int idx = pos - c.pos_min;
        if (idx < 0 || idx >= c.rope_len) { record_error(err, kDevBadShape); rope_row[int64_t(r) * S + p] = 0; }
        else rope_row[int64_t(r) * S + p] = idx;
    }
    gbegin[r] = g0;
    gsize[r] = group_rows;
}

__global__ void fill_query_kernel(const float* __restrict__ q, float* __restrict__ x, int R, int S, int first, int D) {
    const int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    const int per = (S - first) * D;
    if (i >= int64_t(R) * per) return;
    const int r = int(i / per), rem = int(i % per), p = first + rem / D, d = rem % D;
    x[(int64_t(r) * S + p) * D + d] = q[d];
}

// ---------------------------------------------------------------------------------------
// F32-path element kernels.
__global__ void qkv_scatter_kernel(const float* __restrict__ fused, const float* __restrict__ gate, int M, int S, int H,
                                   int hd, int rope, const float* __restrict__ ct, const float* __restrict__ st,
                                   const int* __restrict__ rope_row, float* __restrict__ q, float* __restrict__ k,
                                   float* __restrict__ v, float* __restrict__ g) {
    const int D = H * hd;
    const int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= int64_t(M) * D) return;
    const int m = int(i / D), col = int(i % D), h = col / hd, d = col % hd, half = hd / 2;
    const float* z = fused + int64_t(m) * 3 * D;
    const int r = m / S, s = m % S;
    const int64_t o = ((int64_t(r) * H + h) * S + s) * hd + d;
    float qv = z[col], kv = z[D + col];
    if (rope) {
        const float* c = ct + int64_t(rope_row[m]) * hd;
        const float* sn = st + int64_t(rope_row[m]) * hd;
        const int base = h * hd;
        const float qr = d < half ? -z[base + d + half] : z[base + d - half];
        const float kr = d < half ? -z[D + base + d + half] : z[D + base + d - half];
        qv = __fadd_rn(__fmul_rn(qv, c[d]), __fmul_rn(qr, sn[d]));
        kv = __fadd_rn(__fmul_rn(kv, c[d]), __fmul_rn(kr, sn[d]));
    }
    q[o] = qv; k[o] = kv; v[o] = z[2 * D + col];
    if (g) g[o] = ref_sigmoid(gate[int64_t(m) * D + col]);
}

__global__ void swiglu_kernel(const float* __restrict__ z, int M, int F, float* __restrict__ h) {
    const int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= int64_t(M) * F) return;
    const int m = int(i / F), j = int(i % F);
    const float u = z[int64_t(m) * 2 * F + F + j];
    h[i] = __fmul_rn(z[int64_t(m) * 2 * F + j], ref_silu(u));
}

__global__ void add_kernel(float* __restrict__ x, const float* __restrict__ y, int64_t n) {
    const int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i < n) x[i] = __fadd_rn(x[i], y[i]);
}

// ---------------------------------------------------------------------------------------
// Quantile head tail (reference src/head.cpp:61-80, src/scaler.cpp:109-137).
__global__ void quantile_kernel(const RowConfig c, const float* __restrict__ raw, int R, int P_all, int p0, int h,
                                const float* __restrict__ loc, const float* __restrict__ scale, float* __restrict__ out,
                                float* __restrict__ normalized, int* err) {
    const int ps = c.ps, Q = c.Q, mi = c.median;
    const int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= int64_t(R) * h * ps) return;
    const int r = int(i / (int64_t(h) * ps)), j = int((i / ps) % h), kstep = int(i % ps);
    const float* x = raw + (int64_t(r) * P_all + p0 + j) * ps * Q + kstep * Q;
    const int64_t o = (int64_t(r) * h * ps + int64_t(j) * ps + kstep) * Q;
    float q[64];
    for (int t = 0; t < Q; ++t) if (isnan(x[t])) { record_error(err, kDevBadShape); }
    const float limit = FLT_MAX;
    auto clampv = [&](float v) { return fmaxf(-limit, fminf(limit, v)); };
    auto inc = [&](int t) {
        const float v = x[t];
        return __fmul_rn(c.widths[t], v > 20.f ? v : log1pf(activation_exp(v)));
    };
    const float median = x[mi];
    q[mi] = clampv(median);
    double sum = 0;
    for (int t = mi + 1; t < Q; ++t) { sum = __dadd_rn(sum, double(inc(t))); q[t] = clampv(__fadd_rn(median, float(sum))); }
    sum = 0;
    for (int t = mi - 1; t >= 0; --t) { sum = __dadd_rn(sum, double(inc(t))); q[t] = clampv(__fsub_rn(median, float(sum))); }
    const float L = loc[r], Sc = scale[r];
    float lo = INFINITY, hi = -INFINITY;
    for (int t = 0; t < Q; ++t) {
        if (normalized) normalized[o + t] = q[t];
        const float v = c.use_asinh ? sinhf(q[t]) : q[t];
        q[t] = __fadd_rn(__fmul_rn(v, Sc), L);
        if (isfinite(q[t])) { lo = fminf(lo, q[t]); hi = fmaxf(hi, q[t]); }
    }
    for (int t = 0; t < Q; ++t) {
        float v = q[t];
        if (v == INFINITY) v = isfinite(hi) ? hi : 0.f;
        else if (v == -INFINITY) v = isfinite(lo) ? lo : 0.f;
        out[o + t] = v;
    }
}

// ---------------------------------------------------------------------------------------
// Refine (reference src/refine.cpp).
// NumPy pairwise float64 sum (reference src/numpy_sum.hpp:6-14): leaves of at most 128 values
// summed with eight partial sums, each larger range split at half rounded down to a multiple
// of 8 and its two halves added. Walked iteratively (post-order over an explicit stack of at
// most 32 ranges) instead of recursively, so the per-thread stack stays fixed.
__device__ double numpy_leaf(const double* x, int n) {
    if (n < 8) { double r = -0.0; for (int i = 0; i < n; ++i) r = __dadd_rn(r, x[i]); return r; }
    double r[8];
    for (int j = 0; j < 8; ++j) r[j] = x[j];
    int i = 8;
    for (; i < n - (n % 8); i += 8) for (int j = 0; j < 8; ++j) r[j] = __dadd_rn(r[j], x[i + j]);
    double out = __dadd_rn(__dadd_rn(__dadd_rn(r[0], r[1]), __dadd_rn(r[2], r[3])),
                           __dadd_rn(__dadd_rn(r[4], r[5]), __dadd_rn(r[6], r[7])));
    for (; i < n; ++i) out = __dadd_rn(out, x[i]);
    return out;
}
__device__ double numpy_sum_dev(const double* x, int n) {
    if (n <= 128) return numpy_leaf(x, n);
    int off[32], len[32], state[32];   // state 0: unvisited, 1: left half pending, 2: right half pending
    double acc[32];
    int top = 0;
    off[0] = 0; len[0] = n; state[0] = 0;
    for (;;) {
        if (len[top] > 128 && state[top] == 0) {
            state[top] = 1;
            const int half = len[top] / 2 - (len[top] / 2) % 8;
            off[top + 1] = off[top]; len[top + 1] = half; state[top + 1] = 0;
            ++top;
            continue;
        }
        double v = numpy_leaf(x + off[top], len[top]);
        for (;;) {
            if (top == 0) return v;
            --top;
            if (state[top] == 1) {
                acc[top] = v; state[top] = 2;
                const int half = len[top] / 2 - (len[top] / 2) % 8;
                off[top + 1] = off[top] + half; len[top + 1] = len[top] - half; state[top + 1] = 0;
                ++top;
                break;
            }
            v = __dadd_rn(acc[top], v);
        }
    }
}

struct WS { double w, mean, m2; };
__device__ __forceinline__ WS combine(WS a, WS b) {
    const double w = __dadd_rn(a.w, b.w), safe = fmax(w, DBL_MIN);
    const double delta = __dsub_rn(b.mean, a.mean);
    const double mean = __dadd_rn(a.mean, __ddiv_rn(__dmul_rn(delta, b.w), safe));
    const double m2 = __dadd_rn(__dadd_rn(a.m2, b.m2), __ddiv_rn(__dmul_rn(__dmul_rn(__dmul_rn(delta, delta), a.w), b.w), safe));
    return {w, w == 0 ? 0.0 : mean, w == 0 ? 0.0 : m2};
}

__global__ void refine_kernel(const RowConfig c, const float* __restrict__ q, const float* __restrict__ rows,
                              const int8_t* __restrict__ mask, int stride, const int8_t* __restrict__ role,
                              const float* __restrict__ loc0a, const float* __restrict__ scale0a, int R, int T, int h,
                              double clip, double* __restrict__ scratch, float* __restrict__ out) {
    const int r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= R) return;
    const int ps = c.ps, Q = c.Q, mi = c.median, cp = T / ps, n = cp + h, steps = h * ps;
    const float* qr = q + int64_t(r) * steps * Q;
    float* outr = out + int64_t(r) * steps * Q;
    if (role && role[r] != 0) {
        for (int i = 0; i < steps * Q; ++i) outr[i] = qr[i];
        return;
    }
    double* st = scratch + int64_t(r) * (3 * int64_t(n) + 2 * ps + 2 * h);
    double* terms = st + 3 * int64_t(n);
    double* folded = terms + ps;
    double* floc = folded + ps;
    double* fscale = floc + h;
    const float* x = rows + int64_t(r) * stride;
    const int8_t* m = mask + int64_t(r) * stride;
    for (int p = 0; p < cp; ++p) {
        const int s0 = p * ps;
        for (int k = 0; k < ps; ++k) terms[k] = m[s0 + k];
        const double w = numpy_sum_dev(terms, ps);
        for (int k = 0; k < ps; ++k) terms[k] = __dmul_rn(double(x[s0 + k]), double(m[s0 + k]));
        const double mean = __ddiv_rn(numpy_sum_dev(terms, ps), fmax(w, 1.0));
        for (int k = 0; k < ps; ++k) { const double d = __dsub_rn(double(x[s0 + k]), mean); terms[k] = __dmul_rn(double(m[s0 + k]), __dmul_rn(d, d)); }
        const double m2 = numpy_sum_dev(terms, ps);
        st[3 * p] = w; st[3 * p + 1] = w == 0 ? 0.0 : mean; st[3 * p + 2] = w == 0 ? 0.0 : m2;
    }
    for (int p = cp; p < n; ++p) { st[3 * p] = 0; st[3 * p + 1] = 0; st[3 * p + 2] = 0; }
    // Inclusive Hillis-Steele rounds, in place from the top so each round reads the previous one.
    for (int d = 1; d < n;) {
        for (int i = n - 1; i >= 0; --i) {
            const WS prev = i >= d ? WS{st[3 * (i - d)], st[3 * (i - d) + 1], st[3 * (i - d) + 2]} : WS{0, 0, 0};
            const WS cur{st[3 * i], st[3 * i + 1], st[3 * i + 2]};
            const WS nw = combine(prev, cur);
            st[3 * i] = nw.w; st[3 * i + 1] = nw.mean; st[3 * i + 2] = nw.m2;
        }
        if (d > n / 2) break;
        d *= 2;
    }
    const float loc0 = loc0a[r], scale0 = scale0a[r];
    WS state{st[3 * (cp - 1)], st[3 * (cp - 1) + 1], st[3 * (cp - 1) + 2]};
    const double offset = state.mean;
    for (int j = 0; j < h; ++j) {
        const double var = fmax(__ddiv_rn(state.m2, fmax(__dsub_rn(state.w, 1.0), 1.0)), 0.0);
        const double sc = fmax(sqrt(var), c.minimum_scale);
        floc[j] = state.mean; fscale[j] = sc;
        for (int k = 0; k < ps; ++k) {
            const double med = __ddiv_rn(__dsub_rn(double(qr[(j * ps + k) * Q + mi]), double(loc0)), double(scale0));
            const double v = __dsub_rn(__dadd_rn(__dmul_rn(med, sc), state.mean), offset);
            folded[k] = __dadd_rn(fmin(fmax(v, -clip), clip), offset);
        }
        const double mean = __ddiv_rn(numpy_sum_dev(folded, ps), double(ps));
        for (int k = 0; k < ps; ++k) { const double d = __dsub_rn(folded[k], mean); terms[k] = __dmul_rn(d, d); }
        state = combine(state, WS{double(ps), mean, numpy_sum_dev(terms, ps)});
    }
    for (int t = 0; t < steps; ++t) {
        const int j = t / ps;
        const float loc = j ? float(floc[j]) : loc0, sc = j ? float(fscale[j]) : scale0;
        float lo = INFINITY, hi = -INFINITY;
        float vals[64];
        for (int k = 0; k < Q; ++k) {
            const float nrm = __fdiv_rn(__fsub_rn(qr[t * Q + k], loc0), scale0);
            const float v = __fadd_rn(__fmul_rn(nrm, sc), loc);
            vals[k] = v;
            if (isfinite(v)) { lo = fminf(lo, v); hi = fmaxf(hi, v); }
        }
        for (int k = 0; k < Q; ++k) {
            float v = vals[k];
            if (v == INFINITY) v = isfinite(hi) ? hi : 0.f;
            else if (v == -INFINITY) v = isfinite(lo) ? lo : 0.f;
            outr[t * Q + k] = v;
        }
    }
}

// ---------------------------------------------------------------------------------------
// Final combine (reference src/forecaster.cpp:72-104).
__global__ void finalize_kernel(const RowConfig c, const float* __restrict__ dec, int Rp, int mirrored, int B, int V,
                                int all, int H, int Hfull, const float* __restrict__ lo_a, const float* __restrict__ hi_a,
                                const float* __restrict__ sc_a, int cap_on, const int8_t* __restrict__ clip_ok,
                                float* __restrict__ out, int* err) {
    const int Q = c.Q;
    const int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= int64_t(B) * V * H * Q) return;
    const int q = int(i % Q), t = int((i / Q) % H), bv = int(i / (int64_t(H) * Q));
    const int b = bv / V, v = bv % V, row = b * all + v;
    auto capped = [&](int rr, int qq) {
        float val = dec[(int64_t(rr) * Hfull + t) * Q + qq];
        if (cap_on) {
            // std::min(std::max(v, lo), hi): a NaN value stays NaN
            const float width = __fmul_rn(sc_a[rr], float(c.cap_k));
            const float lo = __fsub_rn(lo_a[rr], width), hi = __fadd_rn(hi_a[rr], width);
            val = (val < lo) ? lo : val;
            val = (hi < val) ? hi : val;
        }
        if (isnan(val)) record_error(err, kDevNaN);
        return val;
    };
    float val = capped(row, q);
    if (mirrored) {
        const float mv = capped(Rp + row, Q - 1 - q);
        val = __fmul_rn(0.5f, __fadd_rn(val, -mv));
    }
    if (clip_ok && clip_ok[bv]) val = fmaxf(val, 0.f);
    if (!isfinite(val)) record_error(err, kDevNonFinite);
    out[i] = val;
}

// Next decode block (reference src/forecaster.cpp:52-64).
__global__ void feedback_kernel(const RowConfig c, const float* __restrict__ rows, const int8_t* __restrict__ mask, int R,
                                int T, const float* __restrict__ q, int n, const int8_t* __restrict__ role,
                                const float* __restrict__ future, const int8_t* __restrict__ fmask, int keep,
                                float* __restrict__ nrows, int8_t* __restrict__ nmask) {
    const int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= int64_t(R) * keep) return;
    const int r = int(i / keep), j = int(i % keep);
    const int start = T + n - keep, t = start + j;
    float value;
    int8_t observed;
    if (t < T) { value = rows[int64_t(r) * T + t]; observed = mask[int64_t(r) * T + t]; }
    else {
        const int k = t - T;
        value = q[(int64_t(r) * n + k) * c.Q + c.median];
        observed = 1;
        if (!isfinite(value) || fabsf(value) >= c.extreme) value = 0.f;
        if (role) {
            if (role[r] == 2 && future) { value = future[int64_t(r) * n + k]; observed = fmask[int64_t(r) * n + k]; }
            if (role[r] == 1) { value = 0.f; observed = 0; }
        }
    }
    nrows[i] = value;
    nmask[i] = observed;
}

// ---------------------------------------------------------------------------------------
// CUDA-core GEMM with per-output reference order. Block tile 64x64, 256 threads, 4x4 each.
constexpr int SB = 64, SK = 16;

template <int ORDER>
__global__ void __launch_bounds__(256) simt_gemm_kernel(const SimtGemm g) {
    if (g.only_if && *g.only_if == 0) return;
    using Acc = typename std::conditional<ORDER == ORDER_F64, double, float>::type;
    __shared__ float As[SK][SB + 1];
    __shared__ float Ws[SK][SB + 1];
    const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
    const int tiles_n = (g.N + SB - 1) / SB;
    const int64_t tiles = int64_t((g.M + SB - 1) / SB) * tiles_n;
    const int K = g.K;
    const bool panels = ORDER == ORDER_PANEL192 && K >= 192;
    for (int64_t tile = blockIdx.x + int64_t(blockIdx.y) * gridDim.x; tile < tiles; tile += int64_t(gridDim.x) * gridDim.y) {
        const int m0 = int(tile / tiles_n) * SB, n0 = int(tile % tiles_n) * SB;
        if (g.row_mask) {
            const int m = m0 + int(threadIdx.x);
            const bool mine = threadIdx.x < SB && m < g.M && g.row_mask[m] != 0;
            if (!__syncthreads_or(mine)) continue;
        }
        Acc sum[4][4], pan[4][4];
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int j = 0; j < 4; ++j) { sum[i][j] = 0; pan[i][j] = 0; }
        for (int k0 = 0; k0 < K; k0 += SK) {
            for (int e = threadIdx.x; e < SK * SB; e += 256) {
                const int kk = e % SK, rr = e / SK;
                const int m = m0 + rr, n = n0 + rr, k = k0 + kk;
                float a = (m < g.M && k < K) ? g.A[int64_t(m) * g.lda + k] : 0.f;
                if (g.round_a_f16) a = __half2float(__float2half_rn(a));
                As[kk][rr] = a;
                Ws[kk][rr] = (n < g.N && k < K) ? g.W[int64_t(n) * K + k] : 0.f;
            }
            __syncthreads();
            const int kend = min(SK, K - k0);
            for (int kk = 0; kk < kend; ++kk) {
                float a[4], w[4];
#pragma unroll
                for (int i = 0; i < 4; ++i) { a[i] = As[kk][ty * 4 + i]; w[i] = Ws[kk][tx * 4 + i]; }
#pragma unroll
                for (int i = 0; i < 4; ++i)
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        if constexpr (ORDER == ORDER_F64) pan[i][j] = __dadd_rn(pan[i][j], __dmul_rn(double(w[j]), double(a[i])));
                        else pan[i][j] = __fmaf_rn(w[j], a[i], pan[i][j]);
                    }
                const int k = k0 + kk + 1;
                if (panels && (k % 192 == 0 || k == K)) {
#pragma unroll
                    for (int i = 0; i < 4; ++i)
#pragma unroll
                        for (int j = 0; j < 4; ++j) { sum[i][j] = sum[i][j] + pan[i][j]; pan[i][j] = 0; }
                }
            }
            __syncthreads();
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int m = m0 + ty * 4 + i;
            if (m >= g.M || (g.row_mask && g.row_mask[m] == 0)) continue;
            const int64_t orow = g.row_group > 0 ? int64_t(m / g.row_group) * g.row_stride + g.row_offset + m % g.row_group : m;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int n = n0 + tx * 4 + j;
                if (n >= g.N) continue;
                float v = panels ? float(sum[i][j]) : float(pan[i][j]);
                if (g.bias) v = __fadd_rn(v, g.bias[n]);
                const int64_t o = orow * g.ldo + n;
                switch (g.epi) {
                    case SEPI_F32: static_cast<float*>(g.out)[o] = v; break;
                    case SEPI_F16: static_cast<__half*>(g.out)[o] = __float2half_rn(v); break;
                    case SEPI_RESID: static_cast<float*>(g.out)[o] = __fadd_rn(static_cast<float*>(g.out)[o], v); break;
                    case SEPI_SILU_F32: static_cast<float*>(g.out)[o] = ref_silu(v); break;
                    case SEPI_SILU_F16: static_cast<__half*>(g.out)[o] = __float2half_rn(ref_silu(v)); break;
                }
            }
        }
    }
}

// The same per-output order (ORDER_PANEL192) for large unconditional launches: a 64 x 128
// block tile, 256 threads of 4 x 8 outputs each (columns 4 tx .. + 3 and 64 + 4 tx .. + 3, so
// that a warp's 16-byte weight reads are conflict-free), 16-byte tile loads, and the 16-deep
// K steps unrolled (panel boundaries, every 192 = 12 x 16 of K, fall between steps). Each output
// still accumulates each 192-wide panel in K order with single-rounding FMAs and adds the
// panel sums in order, so the result is simt_gemm_kernel<ORDER_PANEL192>'s bit for bit.
// Requires K % 16 == 0 and 16-byte aligned A and W rows.
constexpr int GB_M = 64, GB_N = 128, GB_K = 16;

__global__ void __launch_bounds__(256, 2) simt_gemm_tiled_kernel(const SimtGemm g) {
    // Two shared-memory stages: the next K step's tiles are read into registers while the
    // current one is multiplied, then stored into the other stage (one barrier per step).
    __shared__ __align__(16) float As[2][GB_K][GB_M + 4];
    __shared__ __align__(16) float Ws[2][GB_K][GB_N + 4];
    const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
    const int m0 = int(blockIdx.y) * GB_M, n0 = int(blockIdx.x) * GB_N;
    const int K = g.K;
    const bool panels = K >= 192;
    float sum[4][8], pan[4][8];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) { sum[i][j] = 0.f; pan[i][j] = 0.f; }
    const float4 zero = make_float4(0.f, 0.f, 0.f, 0.f);
    const int ar = threadIdx.x >> 2, kq = (threadIdx.x & 3) * 4;
    const bool a_ok = m0 + ar < g.M;
    const float* a_src = g.A + int64_t(m0 + ar) * g.lda + kq;
    const float* w_src[2];
    bool w_ok[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        const int wr = (threadIdx.x + h * 256) >> 2;
        w_ok[h] = n0 + wr < g.N;
        w_src[h] = g.W + int64_t(n0 + wr) * K + kq;
    }
    float4 ra, rw[2];
    auto fetch = [&](int k0) {
        ra = a_ok ? *reinterpret_cast<const float4*>(a_src + k0) : zero;
        if (g.round_a_f16) {
            ra.x = __half2float(__float2half_rn(ra.x)); ra.y = __half2float(__float2half_rn(ra.y));
            ra.z = __half2float(__float2half_rn(ra.z)); ra.w = __half2float(__float2half_rn(ra.w));
        }
#pragma unroll
        for (int h = 0; h < 2; ++h) rw[h] = w_ok[h] ? *reinterpret_cast<const float4*>(w_src[h] + k0) : zero;
    };
    auto store = [&](int st) {
        As[st][kq][ar] = ra.x; As[st][kq + 1][ar] = ra.y; As[st][kq + 2][ar] = ra.z; As[st][kq + 3][ar] = ra.w;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int wr = (threadIdx.x + h * 256) >> 2;
            Ws[st][kq][wr] = rw[h].x; Ws[st][kq + 1][wr] = rw[h].y; Ws[st][kq + 2][wr] = rw[h].z; Ws[st][kq + 3][wr] = rw[h].w;
        }
    };
    fetch(0);
    store(0);
    __syncthreads();
    int st = 0;
    for (int k0 = 0; k0 < K; k0 += GB_K) {
        const bool more = k0 + GB_K < K;
        if (more) fetch(k0 + GB_K);
#pragma unroll
        for (int kk = 0; kk < GB_K; ++kk) {
            const float4 a4 = *reinterpret_cast<const float4*>(&As[st][kk][ty * 4]);
            const float4 w0 = *reinterpret_cast<const float4*>(&Ws[st][kk][tx * 4]);
            const float4 w1 = *reinterpret_cast<const float4*>(&Ws[st][kk][GB_N / 2 + tx * 4]);
            const float a[4] = {a4.x, a4.y, a4.z, a4.w};
            const float w[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 8; ++j) pan[i][j] = __fmaf_rn(w[j], a[i], pan[i][j]);
        }
        if (panels && ((k0 + GB_K) % 192 == 0 || k0 + GB_K >= K)) {
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 8; ++j) { sum[i][j] = __fadd_rn(sum[i][j], pan[i][j]); pan[i][j] = 0.f; }
        }
        if (more) store(st ^ 1);        // the other stage was last read before the previous barrier
        __syncthreads();
        st ^= 1;
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int m = m0 + ty * 4 + i;
        if (m >= g.M) continue;
        const int64_t orow = g.row_group > 0 ? int64_t(m / g.row_group) * g.row_stride + g.row_offset + m % g.row_group : m;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int n = n0 + (j < 4 ? tx * 4 + j : GB_N / 2 + tx * 4 + j - 4);
            if (n >= g.N) continue;
            float v = panels ? sum[i][j] : pan[i][j];
            if (g.bias) v = __fadd_rn(v, g.bias[n]);
            const int64_t o = orow * g.ldo + n;
            switch (g.epi) {
                case SEPI_F32: static_cast<float*>(g.out)[o] = v; break;
                case SEPI_F16: static_cast<__half*>(g.out)[o] = __float2half_rn(v); break;
                case SEPI_RESID: static_cast<float*>(g.out)[o] = __fadd_rn(static_cast<float*>(g.out)[o], v); break;
                case SEPI_SILU_F32: static_cast<float*>(g.out)[o] = ref_silu(v); break;
                case SEPI_SILU_F16: static_cast<__half*>(g.out)[o] = __float2half_rn(ref_silu(v)); break;
            }
        }
    }
}

}  // namespace

cudaError_t assemble_targets(const float* ctx, const uint8_t* umask, int BV, int T, int kept, int len, int mirrored,
                             float* rows, int8_t* mask, cudaStream_t s) {
    assemble_kernel<<<blocks_for(int64_t(BV) * 32), TPB, 0, s>>>(ctx, umask, BV, T, kept, len, mirrored, BV, BV, BV,
                                                                   rows, mask, nullptr);
    return cudaGetLastError();
}

static int pow2_at_least(int n) { int p = 1; while (p < n) p <<= 1; return p; }

size_t covariate_scratch_bytes(const CovShape& c) {
    if (c.V != 1 || c.CP + c.CK == 0) return 0;
    const int Tp = pow2_at_least(c.T);
    const int64_t blocks = int64_t(c.B) * (c.CP + c.CK);
    const int64_t th = int64_t(c.T) + c.H;
    // per block: values f64 + order i32 + lookups f32 over Tp; encoded rows f32
    return size_t(blocks) * size_t(Tp) * 16 + size_t(c.B) * (size_t(c.CP) * c.T + size_t(c.CK) * th) * 4 + 256;
}

cudaError_t assemble_covariates(const CovShape& c, const float* ctx, const uint8_t* umask, const float* past,
                                const float* known, const double* cat_past, const double* cat_known, float* rows,
                                int8_t* mask, int8_t* role, float* future, int8_t* fmask, int* first_obs, void* scratch,
                                cudaStream_t s) {
    const int all = c.V + c.P + c.CP + c.K + c.CK;
    const int64_t R = int64_t(c.B) * all, BV = int64_t(c.B) * c.V;
    if (c.B <= 0 || c.V <= 0 || c.T <= 0 || c.kept <= 0 || c.kept > c.T || c.len < c.kept || R > INT32_MAX)
        return cudaErrorInvalidValue;
    assemble_kernel<<<blocks_for(BV * 32), TPB, 0, s>>>(ctx, umask, int(BV), c.T, c.kept, c.len, c.mirrored, c.V, all, R,
                                                        rows, mask, first_obs);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    float *enc_p = nullptr, *enc_k = nullptr;
    if (c.V == 1 && c.CP + c.CK > 0) {
        if (!scratch) return cudaErrorInvalidValue;
        const int Tp = pow2_at_least(c.T);
        const int64_t blocks = int64_t(c.B) * (c.CP + c.CK);
        enc_p = reinterpret_cast<float*>(static_cast<char*>(scratch) + size_t(blocks) * Tp * 16);
        enc_k = enc_p + size_t(c.B) * c.CP * c.T;
        target_encode_kernel<<<unsigned(blocks), ENC_THREADS, 0, s>>>(c, rows, first_obs, cat_past, cat_known, enc_p, enc_k,
                                                                      static_cast<double*>(scratch), Tp);
        if ((e = cudaGetLastError()) != cudaSuccess) return e;
    }
    cov_rows_kernel<<<blocks_for(R * 32), TPB, 0, s>>>(c, past, known, cat_past, cat_known, enc_p, enc_k, rows, mask,
                                                       role, future, fmask);
    return cudaGetLastError();
}

cudaError_t clip_eligibility(const float* ctx, const uint8_t* umask, int BV, int T, int8_t* ok, cudaStream_t s) {
    clip_ok_kernel<<<blocks_for(int64_t(BV) * 32), TPB, 0, s>>>(ctx, umask, BV, T, ok);
    return cudaGetLastError();
}

cudaError_t scale_rows(const RowConfig& c, const float* rows, const int8_t* mask, int R, int W, int anchor_step,
                       int enc_patches, int kv_words, float* features, float* loc, float* scale, uint32_t* key_valid,
                       int* first_obs, int ctx_len, float* cap_lo, float* cap_hi, float* cap_scale, cudaStream_t s,
                       int kernel) {
    if (R <= 0) return cudaSuccess;
    const bool block_ok = c.ps > 0 && c.ps <= SC_CHUNK && (W % c.ps) == 0;
    if (kernel == 1 && !block_ok) return cudaErrorInvalidValue;
    if (kernel != 0 && block_ok)
        scale_block_kernel<<<R, SC_THREADS, 0, s>>>(c, rows, mask, W, anchor_step, enc_patches, kv_words, features, loc,
                                                    scale, key_valid, first_obs, ctx_len, cap_lo, cap_hi, cap_scale);
    else
        scale_kernel<<<blocks_for(R, 64), 64, 0, s>>>(c, rows, mask, R, W, anchor_step, enc_patches, kv_words, features,
                                                     loc, scale, key_valid, first_obs, ctx_len, cap_lo, cap_hi, cap_scale);
    return cudaGetLastError();
}

cudaError_t known_rows(const RowConfig& c, const float* rows, const int8_t* mask, const int8_t* role, int R, int W,
                       int anchor_step, float* features, float* loc, float* scale, cudaStream_t s) {
    known_kernel<<<blocks_for(int64_t(R) * 32), TPB, 0, s>>>(c, rows, mask, role, R, W, anchor_step, features, loc, scale);
    return cudaGetLastError();
}

cudaError_t positions(const RowConfig& c, const int* first_obs, int R, int group_rows, int N, int S, int cov,
                      int* rope_row, int* group_begin, int* group_size, int* err, cudaStream_t s) {
    positions_kernel<<<blocks_for(R), TPB, 0, s>>>(c, first_obs, R, group_rows, N, S, cov, rope_row, group_begin, group_size, err);
    return cudaGetLastError();
}

cudaError_t fill_query(const float* query, float* x, int R, int S, int first, int D, cudaStream_t s) {
    const int64_t n = int64_t(R) * (S - first) * D;
    if (n <= 0) return cudaSuccess;
    fill_query_kernel<<<blocks_for(n), TPB, 0, s>>>(query, x, R, S, first, D);
    return cudaGetLastError();
}

cudaError_t rms_norm(const float* x, const float* w, int tokens, int D, float eps, void* out, int out_f16, int sub,
                     int S, int off, cudaStream_t s) {
    if (tokens <= 0) return cudaSuccess;
    const unsigned grid = blocks_for(int64_t(tokens) * 32);
    switch (D) {
        case 128: rms_regs_kernel<4><<<grid, TPB, 0, s>>>(x, w, tokens, eps, out, out_f16, sub, S, off); break;
        case 256: rms_regs_kernel<8><<<grid, TPB, 0, s>>>(x, w, tokens, eps, out, out_f16, sub, S, off); break;
        case 512: rms_regs_kernel<16><<<grid, TPB, 0, s>>>(x, w, tokens, eps, out, out_f16, sub, S, off); break;
        case 768: rms_regs_kernel<24><<<grid, TPB, 0, s>>>(x, w, tokens, eps, out, out_f16, sub, S, off); break;
        case 1024: rms_regs_kernel<32><<<grid, TPB, 0, s>>>(x, w, tokens, eps, out, out_f16, sub, S, off); break;
        default: rms_kernel<<<grid, TPB, 0, s>>>(x, w, tokens, D, eps, out, out_f16, sub, S, off); break;
    }
    return cudaGetLastError();
}

cudaError_t qkv_scatter(const float* fused, const float* gate, int M, int S, int H, int hd, int rope, const float* cos_tab,
                        const float* sin_tab, const int* rope_row, float* q, float* k, float* v, float* g, cudaStream_t s) {
    const int64_t n = int64_t(M) * H * hd;
    qkv_scatter_kernel<<<blocks_for(n), TPB, 0, s>>>(fused, gate, M, S, H, hd, rope, cos_tab, sin_tab, rope_row, q, k, v, g);
    return cudaGetLastError();
}

cudaError_t swiglu(const float* z, int M, int F, float* h, cudaStream_t s) {
    swiglu_kernel<<<blocks_for(int64_t(M) * F), TPB, 0, s>>>(z, M, F, h);
    return cudaGetLastError();
}

cudaError_t add_inplace(float* x, const float* y, int64_t n, cudaStream_t s) {
    add_kernel<<<blocks_for(n), TPB, 0, s>>>(x, y, n);
    return cudaGetLastError();
}

cudaError_t quantile_head(const RowConfig& c, const float* raw, int R, int P_all, int p0, int h, const float* loc,
                          const float* scale, float* out, float* normalized, int* err, cudaStream_t s) {
    if (c.Q > 64) return cudaErrorInvalidValue;
    quantile_kernel<<<blocks_for(int64_t(R) * h * c.ps, 128), 128, 0, s>>>(c, raw, R, P_all, p0, h, loc, scale, out, normalized, err);
    return cudaGetLastError();
}

// NumPy pairwise float64 sum of val(0) .. val(n - 1) for n <= 128 (the same leaves and order
// as numpy_sum_dev on an array of those values).
template <class F>
__device__ __forceinline__ double numpy_sum_small(F val, int n) {
    if (n < 8) { double r = -0.0; for (int i = 0; i < n; ++i) r = __dadd_rn(r, val(i)); return r; }
    double r[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) r[j] = val(j);
    int i = 8;
    for (; i < n - (n % 8); i += 8)
#pragma unroll
        for (int j = 0; j < 8; ++j) r[j] = __dadd_rn(r[j], val(i + j));
    double out = __dadd_rn(__dadd_rn(__dadd_rn(r[0], r[1]), __dadd_rn(r[2], r[3])),
                           __dadd_rn(__dadd_rn(r[4], r[5]), __dadd_rn(r[6], r[7])));
    for (; i < n; ++i) out = __dadd_rn(out, val(i));
    return out;
}

// refine_kernel with one warp per row (patch_size <= 128): the per-patch statistics one patch
// per lane, the Hillis-Steele rounds over chunks of 32 elements from the top (each chunk read
// before it is written, as the in-place top-down loop), the block frames with one step per
// lane, the output one step per lane. Every value is computed by the same operations in the
// same order as refine_kernel; the scratch layout is the same.
__global__ void __launch_bounds__(128) refine_warp_kernel(const RowConfig c, const float* __restrict__ q,
                                                          const float* __restrict__ rows, const int8_t* __restrict__ mask,
                                                          int stride, const int8_t* __restrict__ role,
                                                          const float* __restrict__ loc0a, const float* __restrict__ scale0a,
                                                          int R, int T, int h, double clip, double* __restrict__ scratch,
                                                          float* __restrict__ out) {
    const int r = blockIdx.x * 4 + threadIdx.x / 32, lane = threadIdx.x & 31;
    if (r >= R) return;                                       // uniform across the warp
    const int ps = c.ps, Q = c.Q, mi = c.median, cp = T / ps, n = cp + h, steps = h * ps;
    const float* qr = q + int64_t(r) * steps * Q;
    float* outr = out + int64_t(r) * steps * Q;
    if (role && role[r] != 0) {
        for (int i = lane; i < steps * Q; i += 32) outr[i] = qr[i];
        return;
    }
    double* st = scratch + int64_t(r) * (3 * int64_t(n) + 2 * ps + 2 * h);
    double* terms = st + 3 * int64_t(n);
    double* folded = terms + ps;
    double* floc = folded + ps;
    double* fscale = floc + h;
    const float* x = rows + int64_t(r) * stride;
    const int8_t* m = mask + int64_t(r) * stride;
    for (int p = lane; p < cp; p += 32) {
        const int s0 = p * ps;
        const double w = numpy_sum_small([&](int k) { return double(m[s0 + k]); }, ps);
        const double mean = __ddiv_rn(numpy_sum_small([&](int k) { return __dmul_rn(double(x[s0 + k]), double(m[s0 + k])); }, ps),
                                      fmax(w, 1.0));
        const double m2 = numpy_sum_small([&](int k) {
            const double d = __dsub_rn(double(x[s0 + k]), mean);
            return __dmul_rn(double(m[s0 + k]), __dmul_rn(d, d));
        }, ps);
        st[3 * p] = w; st[3 * p + 1] = w == 0 ? 0.0 : mean; st[3 * p + 2] = w == 0 ? 0.0 : m2;
    }
    for (int p = cp + lane; p < n; p += 32) { st[3 * p] = 0; st[3 * p + 1] = 0; st[3 * p + 2] = 0; }
    __syncwarp();
    for (int d = 1; d < n;) {
        for (int c0 = ((n - 1) / 32) * 32; c0 >= 0; c0 -= 32) {
            const int i = c0 + lane;
            WS nw{0, 0, 0};
            if (i < n) {
                const WS prev = i >= d ? WS{st[3 * (i - d)], st[3 * (i - d) + 1], st[3 * (i - d) + 2]} : WS{0, 0, 0};
                const WS cur{st[3 * i], st[3 * i + 1], st[3 * i + 2]};
                nw = combine(prev, cur);
            }
            __syncwarp();
            if (i < n) { st[3 * i] = nw.w; st[3 * i + 1] = nw.mean; st[3 * i + 2] = nw.m2; }
            __syncwarp();
        }
        if (d > n / 2) break;
        d *= 2;
    }
    const float loc0 = loc0a[r], scale0 = scale0a[r];
    WS state{st[3 * (cp - 1)], st[3 * (cp - 1) + 1], st[3 * (cp - 1) + 2]};
    const double offset = state.mean;
    for (int j = 0; j < h; ++j) {
        const double var = fmax(__ddiv_rn(state.m2, fmax(__dsub_rn(state.w, 1.0), 1.0)), 0.0);
        const double sc = fmax(sqrt(var), c.minimum_scale);
        if (lane == 0) { floc[j] = state.mean; fscale[j] = sc; }
        for (int k = lane; k < ps; k += 32) {
            const double med = __ddiv_rn(__dsub_rn(double(qr[(j * ps + k) * Q + mi]), double(loc0)), double(scale0));
            const double v = __dsub_rn(__dadd_rn(__dmul_rn(med, sc), state.mean), offset);
            folded[k] = __dadd_rn(fmin(fmax(v, -clip), clip), offset);
        }
        __syncwarp();
        const double mean = __ddiv_rn(numpy_sum_small([&](int k) { return folded[k]; }, ps), double(ps));
        for (int k = lane; k < ps; k += 32) { const double dd = __dsub_rn(folded[k], mean); terms[k] = __dmul_rn(dd, dd); }
        __syncwarp();
        state = combine(state, WS{double(ps), mean, numpy_sum_small([&](int k) { return terms[k]; }, ps)});
        __syncwarp();
    }
    for (int t = lane; t < steps; t += 32) {
        const int j = t / ps;
        const float loc = j ? float(floc[j]) : loc0, sc = j ? float(fscale[j]) : scale0;
        float lo = INFINITY, hi = -INFINITY;
        float vals[64];
        for (int k = 0; k < Q; ++k) {
            const float nrm = __fdiv_rn(__fsub_rn(qr[t * Q + k], loc0), scale0);
            const float v = __fadd_rn(__fmul_rn(nrm, sc), loc);
            vals[k] = v;
            if (isfinite(v)) { lo = fminf(lo, v); hi = fmaxf(hi, v); }
        }
        for (int k = 0; k < Q; ++k) {
            float v = vals[k];
            if (v == INFINITY) v = isfinite(hi) ? hi : 0.f;
            else if (v == -INFINITY) v = isfinite(lo) ? lo : 0.f;
            outr[t * Q + k] = v;
        }
    }
}

cudaError_t refine(const RowConfig& c, const float* q, const float* rows, const int8_t* mask, int stride, const int8_t* role,
                   const float* loc0, const float* scale0, int R, int T, int h, double clip, double* scratch, float* out,
                   cudaStream_t s) {
    if (c.Q > 64) return cudaErrorInvalidValue;
    if (c.ps <= 128)
        refine_warp_kernel<<<unsigned((R + 3) / 4), 128, 0, s>>>(c, q, rows, mask, stride, role, loc0, scale0, R, T, h, clip,
                                                                 scratch, out);
    else
        refine_kernel<<<blocks_for(R, 64), 64, 0, s>>>(c, q, rows, mask, stride, role, loc0, scale0, R, T, h, clip, scratch,
                                                       out);
    return cudaGetLastError();
}

cudaError_t finalize(const RowConfig& c, const float* decoded, int Rp, int mirrored, int B, int V, int all, int H,
                     int Hfull, const float* cap_lo, const float* cap_hi, const float* cap_scale, int cap_on,
                     const int8_t* clip_ok, float* out, int* err, cudaStream_t s) {
    const int64_t n = int64_t(B) * V * H * c.Q;
    finalize_kernel<<<blocks_for(n), TPB, 0, s>>>(c, decoded, Rp, mirrored, B, V, all, H, Hfull, cap_lo, cap_hi, cap_scale,
                                                 cap_on, clip_ok, out, err);
    return cudaGetLastError();
}

cudaError_t feedback(const RowConfig& c, const float* rows, const int8_t* mask, int R, int T, const float* q, int n,
                     const int8_t* role, const float* future, const int8_t* fmask, int keep, float* next_rows,
                     int8_t* next_mask, cudaStream_t s) {
    feedback_kernel<<<blocks_for(int64_t(R) * keep), TPB, 0, s>>>(c, rows, mask, R, T, q, n, role, future, fmask, keep,
                                                                 next_rows, next_mask);
    return cudaGetLastError();
}

// Split-panel form of ORDER_PANEL192 for few rows: block (x, y, p) computes the 32 x 32 tile's
// FMA chain over panel p's 192 K values (ascending k, as the one-pass kernel), and the combine
// kernel adds the panels to 0 in order and applies the epilogue: the same operations on every
// output as simt_gemm_kernel<ORDER_PANEL192>.
constexpr int PT = 32, PK = 32, PANEL = 192;
__global__ void __launch_bounds__(256) simt_panel_kernel(const SimtGemm g) {
    __shared__ float As[PK][PT + 1];
    __shared__ float Ws[PK][PT + 1];
    const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
    const int m0 = blockIdx.y * PT, n0 = blockIdx.x * PT, p = blockIdx.z;
    const int k_lo = p * PANEL, k_hi = min(g.K, k_lo + PANEL);
    float pan[2][2] = {{0.f, 0.f}, {0.f, 0.f}};
    for (int k0 = k_lo; k0 < k_hi; k0 += PK) {
        for (int e = threadIdx.x; e < PK * PT; e += 256) {
            const int kk = e % PK, rr = e / PK;
            const int m = m0 + rr, n = n0 + rr, k = k0 + kk;
            float a = (m < g.M && k < k_hi) ? g.A[int64_t(m) * g.lda + k] : 0.f;
            if (g.round_a_f16) a = __half2float(__float2half_rn(a));
            As[kk][rr] = a;
            Ws[kk][rr] = (n < g.N && k < k_hi) ? g.W[int64_t(n) * g.K + k] : 0.f;
        }
        __syncthreads();
        const int kend = min(PK, k_hi - k0);
        for (int kk = 0; kk < kend; ++kk) {
            const float a0 = As[kk][ty * 2], a1 = As[kk][ty * 2 + 1];
            const float w0 = Ws[kk][tx * 2], w1 = Ws[kk][tx * 2 + 1];
            pan[0][0] = __fmaf_rn(w0, a0, pan[0][0]); pan[0][1] = __fmaf_rn(w1, a0, pan[0][1]);
            pan[1][0] = __fmaf_rn(w0, a1, pan[1][0]); pan[1][1] = __fmaf_rn(w1, a1, pan[1][1]);
        }
        __syncthreads();
    }
    float* part = g.panel_scratch + int64_t(p) * g.M * g.N;
#pragma unroll
    for (int i = 0; i < 2; ++i) {
        const int m = m0 + ty * 2 + i;
        if (m >= g.M) continue;
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            const int n = n0 + tx * 2 + j;
            if (n < g.N) part[int64_t(m) * g.N + n] = pan[i][j];
        }
    }
}

// The same partials with the whole 192-wide panel staged at once: every thread issues its
// 16-byte loads of the A and W panel tiles together (one memory latency per block instead of
// one per 32-deep step), then runs its 2 x 2 K-ordered FMA chains over the panel. Requires
// K % 4 == 0 and 16-byte aligned A and W rows.
constexpr int PF_STRIDE = PT + 4;                    // [k][row] tiles, padded
constexpr size_t panel_full_smem() { return size_t(2) * PANEL * PF_STRIDE * sizeof(float); }

__global__ void __launch_bounds__(256) simt_panel_full_kernel(const SimtGemm g) {
    extern __shared__ __align__(16) float pf_sh[];
    float* As = pf_sh;                               // [PANEL][PF_STRIDE]
    float* Ws = pf_sh + PANEL * PF_STRIDE;
    const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
    const int m0 = blockIdx.y * PT, n0 = blockIdx.x * PT, p = blockIdx.z;
    const int k_lo = p * PANEL, kn = min(g.K, k_lo + PANEL) - k_lo;
    const float4 zero = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int e = threadIdx.x; e < PT * (PANEL / 4); e += 256) {
        const int rr = e % PT, k4 = (e / PT) * 4;     // a warp stores one k-quad of 32 rows: no conflicts
        const int m = m0 + rr, n = n0 + rr;
        float4 a = (m < g.M && k4 < kn) ? *reinterpret_cast<const float4*>(g.A + int64_t(m) * g.lda + k_lo + k4) : zero;
        if (g.round_a_f16) {
            a.x = __half2float(__float2half_rn(a.x)); a.y = __half2float(__float2half_rn(a.y));
            a.z = __half2float(__float2half_rn(a.z)); a.w = __half2float(__float2half_rn(a.w));
        }
        const float4 w = (n < g.N && k4 < kn) ? *reinterpret_cast<const float4*>(g.W + int64_t(n) * g.K + k_lo + k4) : zero;
        As[(k4 + 0) * PF_STRIDE + rr] = a.x; As[(k4 + 1) * PF_STRIDE + rr] = a.y;
        As[(k4 + 2) * PF_STRIDE + rr] = a.z; As[(k4 + 3) * PF_STRIDE + rr] = a.w;
        Ws[(k4 + 0) * PF_STRIDE + rr] = w.x; Ws[(k4 + 1) * PF_STRIDE + rr] = w.y;
        Ws[(k4 + 2) * PF_STRIDE + rr] = w.z; Ws[(k4 + 3) * PF_STRIDE + rr] = w.w;
    }
    __syncthreads();
    float pan[2][2] = {{0.f, 0.f}, {0.f, 0.f}};
    for (int kk = 0; kk < kn; ++kk) {
        const float2 a = *reinterpret_cast<const float2*>(As + kk * PF_STRIDE + ty * 2);
        const float2 w = *reinterpret_cast<const float2*>(Ws + kk * PF_STRIDE + tx * 2);
        pan[0][0] = __fmaf_rn(w.x, a.x, pan[0][0]); pan[0][1] = __fmaf_rn(w.y, a.x, pan[0][1]);
        pan[1][0] = __fmaf_rn(w.x, a.y, pan[1][0]); pan[1][1] = __fmaf_rn(w.y, a.y, pan[1][1]);
    }
    float* part = g.panel_scratch + int64_t(p) * g.M * g.N;
#pragma unroll
    for (int i = 0; i < 2; ++i) {
        const int m = m0 + ty * 2 + i;
        if (m >= g.M) continue;
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            const int n = n0 + tx * 2 + j;
            if (n < g.N) part[int64_t(m) * g.N + n] = pan[i][j];
        }
    }
}

__global__ void simt_panel_combine_kernel(const SimtGemm g, int panels) {
    const int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= int64_t(g.M) * g.N) return;
    const int m = int(i / g.N), n = int(i % g.N);
    float v = 0.f;
    for (int p = 0; p < panels; ++p) v = v + g.panel_scratch[int64_t(p) * g.M * g.N + i];
    if (g.bias) v = __fadd_rn(v, g.bias[n]);
    const int64_t orow = g.row_group > 0 ? int64_t(m / g.row_group) * g.row_stride + g.row_offset + m % g.row_group : m;
    const int64_t o = orow * g.ldo + n;
    switch (g.epi) {
        case SEPI_F32: static_cast<float*>(g.out)[o] = v; break;
        case SEPI_F16: static_cast<__half*>(g.out)[o] = __float2half_rn(v); break;
        case SEPI_RESID: static_cast<float*>(g.out)[o] = __fadd_rn(static_cast<float*>(g.out)[o], v); break;
        case SEPI_SILU_F32: static_cast<float*>(g.out)[o] = ref_silu(v); break;
        case SEPI_SILU_F16: static_cast<__half*>(g.out)[o] = __float2half_rn(ref_silu(v)); break;
    }
}

size_t simt_panel_scratch_bytes(const SimtGemm& g) {
    if (g.order != ORDER_PANEL192 || g.K < 2 * PANEL || g.M > 512 || g.only_if || g.row_mask) return 0;
    const int panels = (g.K + PANEL - 1) / PANEL;
    return size_t(panels) * size_t(g.M) * size_t(g.N) * sizeof(float);
}

cudaError_t simt_gemm(const SimtGemm& g, cudaStream_t s) {
    if (g.M <= 0 || g.N <= 0) return cudaSuccess;
    const size_t need = simt_panel_scratch_bytes(g);
    if (need && g.panel_scratch && g.panel_scratch_bytes >= need) {
        const int panels = (g.K + PANEL - 1) / PANEL;
        const dim3 grid((g.N + PT - 1) / PT, (g.M + PT - 1) / PT, panels);
        auto aligned16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
        if (g.tiled != 0 && g.K % 4 == 0 && g.lda % 4 == 0 && aligned16(g.A) && aligned16(g.W)) {
            static KernelSetup configured;
            int dev = 0;
            cudaGetDevice(&dev);
            unsigned long long ctx_key = 0;
            if (configured.needed(dev, &ctx_key)) {
                cudaError_t e = cudaFuncSetAttribute(simt_panel_full_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                     int(panel_full_smem()));
                if (e != cudaSuccess) return e;
                configured.done(dev, ctx_key);
            }
            simt_panel_full_kernel<<<grid, 256, panel_full_smem(), s>>>(g);
        } else {
            simt_panel_kernel<<<grid, 256, 0, s>>>(g);
        }
        const int64_t n = int64_t(g.M) * g.N;
        simt_panel_combine_kernel<<<blocks_for(n), TPB, 0, s>>>(g, panels);
        return cudaGetLastError();
    }
    auto aligned = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
    if (g.order == ORDER_PANEL192 && g.tiled != 0 && !g.only_if && !g.row_mask && g.K % GB_K == 0 && g.lda % 4 == 0 &&
        aligned(g.A) && aligned(g.W) && g.M >= GB_M && (g.M + GB_M - 1) / GB_M <= 65535) {
        const dim3 grid((g.N + GB_N - 1) / GB_N, (g.M + GB_M - 1) / GB_M);
        simt_gemm_tiled_kernel<<<grid, 256, 0, s>>>(g);
        return cudaGetLastError();
    }
    // One tile per block; launches that are conditional on a device flag (only_if) or whose
    // tile rows exceed the grid's y limit use a bounded grid that strides over the tiles.
    const int64_t tm = (g.M + SB - 1) / SB;
    dim3 grid((g.N + SB - 1) / SB, unsigned(tm));
    if (g.only_if || tm > 65535) {
        grid.x = 148 * 8;
        grid.y = 1;
    }
    switch (g.order) {
        case ORDER_PANEL192: simt_gemm_kernel<ORDER_PANEL192><<<grid, 256, 0, s>>>(g); break;
        case ORDER_CHAIN: simt_gemm_kernel<ORDER_CHAIN><<<grid, 256, 0, s>>>(g); break;
        default: simt_gemm_kernel<ORDER_F64><<<grid, 256, 0, s>>>(g); break;
    }
    return cudaGetLastError();
}

__global__ void split_f16_kernel(const float* __restrict__ a, int64_t n, int K, __half* __restrict__ out,
                                 int* __restrict__ overflow, int8_t* __restrict__ row_overflow) {
    const int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const int64_t m = i / K;
    const int k = int(i % K);
    const float v = a[i];
    const __half hi = __float2half_rn(v);
    const __half lo = __float2half_rn(__fsub_rn(v, __half2float(hi)));
    __half* o = out + m * 3 * K;
    o[k] = hi;
    o[K + k] = hi;
    o[2 * K + k] = lo;
    if (!(fabsf(v) <= 30000.f)) {
        *overflow = 1;
        if (row_overflow) row_overflow[m] = 1;
    }
}

cudaError_t split_f16(const float* a, int64_t rows, int K, __half* out, int* overflow, int8_t* row_overflow,
                      cudaStream_t s) {
    const int64_t n = rows * K;
    if (n <= 0) return cudaSuccess;
    split_f16_kernel<<<blocks_for(n), TPB, 0, s>>>(a, n, K, out, overflow, row_overflow);
    return cudaGetLastError();
}

int read_error(int* d_err, cudaStream_t s) {
    int h = 0;
    cudaMemcpyAsync(&h, d_err, sizeof(int), cudaMemcpyDeviceToHost, s);
    cudaStreamSynchronize(s);
    if (h) cudaMemsetAsync(d_err, 0, sizeof(int), s);
    return h;
}

}  // namespace tsb
