// CPU oracle for the Timestral forecast hot path — TEST INFRASTRUCTURE ONLY (see oracle.h).
//
// Every function restates one reference function; the citation (reference file:line) is on
// each. Floating-point operation order follows the reference's F32 path, which is built with
// -ffp-contract=off (reference CMakeLists.txt:71-73); this file is built the same way and
// uses std::fma exactly where the reference does.
#include "oracle.h"

#include <algorithm>
#include <cmath>
#include <cstring>
#include <limits>
#include <map>
#include <stdexcept>
#include <string>
#include <vector>
#include <immintrin.h>
#ifdef _OPENMP
#include <omp.h>
#endif

namespace {

struct Error : std::runtime_error {
    explicit Error(const std::string& s) : std::runtime_error(s) {}
};
thread_local std::string g_error;

// ------------------------------------------------------------------------------------
// fp16 conversion (IEEE binary16, round to nearest even) — ggml's FP32->FP16 conversion.
uint16_t f32_to_f16(float f) {
    uint32_t x; std::memcpy(&x, &f, 4);
    uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t mant = x & 0x7fffffu;
    int32_t exp = int32_t((x >> 23) & 0xff);
    if (exp == 0xff) return uint16_t(sign | 0x7c00u | (mant ? 0x200u : 0));
    int32_t e = exp - 127 + 15;
    if (e >= 0x1f) return uint16_t(sign | 0x7c00u);
    if (e <= 0) {
        if (e < -10) return uint16_t(sign);
        mant |= 0x800000u;
        int shift = 14 - e;
        uint32_t h = mant >> shift, rem = mant & ((1u << shift) - 1), half = 1u << (shift - 1);
        if (rem > half || (rem == half && (h & 1))) ++h;
        return uint16_t(sign | h);
    }
    uint32_t h = (uint32_t(e) << 10) | (mant >> 13), rem = mant & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1))) ++h;
    return uint16_t(sign | h);
}
float f16_to_f32(uint16_t h) {
    uint32_t sign = uint32_t(h & 0x8000u) << 16, exp = (h >> 10) & 0x1f, mant = h & 0x3ffu, x;
    if (exp == 0) {
        if (!mant) x = sign;
        else { int e = -1; do { ++e; mant <<= 1; } while (!(mant & 0x400u)); x = sign | uint32_t(127 - 15 - e) << 23 | (mant & 0x3ffu) << 13; }
    } else if (exp == 0x1f) x = sign | 0x7f800000u | (mant << 13);
    else x = sign | (exp + 127 - 15) << 23 | (mant << 13);
    float f; std::memcpy(&f, &x, 4); return f;
}
float round_f16(float f) { return f16_to_f32(f32_to_f16(f)); }

// ------------------------------------------------------------------------------------
// Reductions.

// NumPy pairwise float64 sum (reference src/numpy_sum.hpp:6-14).
double numpy_sum(const double* x, size_t n) {
    if (n < 8) { double r = -0.0; for (size_t i = 0; i < n; ++i) r += x[i]; return r; }
    if (n <= 128) {
        double r[8]; for (size_t j = 0; j < 8; ++j) r[j] = x[j];
        size_t i = 8;
        for (; i < n - (n % 8); i += 8) for (size_t j = 0; j < 8; ++j) r[j] += x[i + j];
        double out = ((r[0] + r[1]) + (r[2] + r[3])) + ((r[4] + r[5]) + (r[6] + r[7]));
        for (; i < n; ++i) out += x[i];
        return out;
    }
    size_t half = n / 2; half -= half % 8;
    return numpy_sum(x, half) + numpy_sum(x + half, n - half);
}

// The four-level eight-lane cascade of the ATen contiguous float sum, used by the
// reference for torch_sum_f32 (src/torch_sum.hpp:9-23) and, on squares, for the RMSNorm
// mean (src/layers.cpp:262-278). `sq` selects x*x.
float cascade_sum(const float* x, size_t length, bool sq) {
    auto val = [&](size_t i) { float a = x[i]; return sq ? a * a : a; };
    if (!sq && length < 8) {
        float partial[4] = {}; size_t i = 0;
        for (; i + 4 <= length; i += 4) for (int j = 0; j < 4; ++j) partial[j] += x[i + j];
        for (; i < length; ++i) partial[0] += x[i];
        for (int j = 1; j < 4; ++j) partial[0] += partial[j];
        return partial[0];
    }
    float acc[4][4][8] = {};
    size_t groups = length / 32, log = 0;
    for (size_t n = groups ? groups - 1 : 0; n; n >>= 1) ++log;
    size_t power = std::max(size_t(4), log / 4), step = size_t(1) << power, mask = step - 1, i = 0;
    auto add = [&](size_t g) { for (int k = 0; k < 4; ++k) for (int l = 0; l < 8; ++l) acc[0][k][l] += val(g * 32 + k * 8 + l); };
    for (; i + step <= groups;) {
        for (size_t j = 0; j < step; ++j, ++i) add(i);
        for (size_t level = 1; level < 4; ++level) {
            for (int k = 0; k < 4; ++k) for (int l = 0; l < 8; ++l) { acc[level][k][l] += acc[level - 1][k][l]; acc[level - 1][k][l] = 0; }
            if (i & (mask << (level * power))) break;
        }
    }
    for (; i < groups; ++i) add(i);
    for (int level = 1; level < 4; ++level) for (int k = 0; k < 4; ++k) for (int l = 0; l < 8; ++l) acc[0][k][l] += acc[level][k][l];
    size_t v = groups * 4;
    for (; v < length / 8; ++v) for (int l = 0; l < 8; ++l) acc[0][0][l] += val(v * 8 + l);
    for (int k = 1; k < 4; ++k) for (int l = 0; l < 8; ++l) acc[0][0][l] += acc[0][k][l];
    float sum = 0;
    for (size_t d = v * 8; d < length; ++d) sum += val(d);
    for (int l = 0; l < 8; ++l) sum += acc[0][0][l];
    return sum;
}

// ------------------------------------------------------------------------------------
// Exponentials of the reference (restated algorithms, not libm's).

// SLEEF-style float exp used by the reference's sigmoid/SiLU/softplus
// (src/layers.cpp:658-667, src/head.cpp:252-261).
float activation_exp(float x) {
    if (!std::isfinite(x) || x < -87 || x > 88) return std::exp(x);
    float q = std::nearbyint(x * 1.4426950408889634f);
    float r = std::fma(q, -.693145751953125f, x);
    r = std::fma(q, -1.428606765330187045e-6f, r);
    float u = .000198527617612853646f;
    for (float c : {.00139304355252534151f, .00833336077630519867f, .0416664853692054749f,
                    .166666671633720398f, .5f}) u = std::fma(u, r, c);
    return std::ldexp(1.f + std::fma(r * r, u, r), int(q));
}

// ATen exp_u20 polynomial used for full eight-lane chunks of the softmax
// (src/layers.cpp:297-305).
float attention_exp(float x) {
    if (x < -87.3365478515625f) return 0;
    if (!std::isfinite(x) || x > 88) return std::exp(x);
    float n = std::floor(std::fma(x, 1.4426950216293335f, .5f));
    float r = std::fma(-n, .6931471824645996f, x);
    float y = std::fma(r, .00828929059f, .0418978221f);
    for (float a : {.166676521f, .499991506f, .999999701f, 1.f}) y = std::fma(r, y, a);
    return (y * std::ldexp(1.f, int(n) - 1)) * 2;
}

// ------------------------------------------------------------------------------------
// Config helpers.
const int kTime = 0, kVariate = 1, kTimeVariate = 2, kVariateTime = 3;
std::vector<bool> layer_axes(int k) {  // reference src/config.hpp:14-22
    switch (k) { case kTime: return {true}; case kVariate: return {false};
                 case kTimeVariate: return {true, false}; case kVariateTime: return {false, true}; }
    throw Error("bad layer kind");
}
size_t median_index(const oracle_config& c) {
    for (int i = 0; i < c.num_quantiles; ++i) if (c.knots[i] == 0.5) return size_t(i);
    return 0;
}
int64_t rope_table_len(const oracle_config& c) { return 2 * (-(int64_t)c.rope_table_pos_min) + 1; }

// reference src/covariates.cpp:27-32
bool supports_known_covariates(const oracle_config& c) {
    if (!c.covariate_enabled) return false;
    std::vector<bool> ops;
    for (int i = 0; i < c.n_layers; ++i) for (bool t : layer_axes(c.schedule[i])) ops.push_back(t);
    for (size_t i = 0; i < ops.size(); ++i) if (ops[i]) {
        bool time = false, var = false;
        for (size_t j = i + 1; j < ops.size(); ++j) { time |= ops[j]; var |= !ops[j]; }
        if (time && var) return true;
    }
    return false;
}

size_t mul(size_t a, size_t b) { if (b && a > SIZE_MAX / b) throw Error("dimensions overflow"); return a * b; }

// ------------------------------------------------------------------------------------
// Scaler (reference src/scaler.cpp).
struct ScaleResult { std::vector<float> scaled, loc, scale; };
struct InstanceStats { std::vector<float> loc, scale; std::vector<int8_t> is_binary; };

float affine_value(float x, float loc, float scale, bool observed, bool squash) {  // scaler.cpp:20-25
    float y = (x - loc) / std::max(scale, std::numeric_limits<float>::epsilon());
    if (!observed) return 0.0f;
    return squash ? std::asinh(y) : y;
}

ScaleResult scale_rows(const oracle_config& c, const float* x, const int8_t* mask, size_t rows, size_t length) {  // scaler.cpp:27-58
    if (!rows || !length || length % c.patch_size) throw Error("scaler: invalid packed row shape");
    for (size_t i = 0; i < rows * length; ++i) if (mask[i] != 0 && mask[i] != 1) throw Error("scaler: mask must be boolean");
    ScaleResult out;
    out.loc.resize(rows * length); out.scale.resize(rows * length); out.scaled.resize(rows * length);
    for (size_t r = 0; r < rows; ++r) {
        double cum_w = 0, cum_x = 0, prev_mean = 0, m2 = 0;
        for (size_t t = 0; t < length; ++t) {
            size_t i = r * length + t;
            double v = x[i], w = mask[i];
            cum_w += w;
            cum_x += w * v;
            double den = std::max(cum_w, 1.0);
            double mean = cum_x / den;
            double increment = (v - prev_mean) * (v - mean) * w;
            m2 += increment;
            prev_mean = mean;
            if ((t + 1) % c.patch_size == 0) {
                float loc = static_cast<float>(mean);
                float scale = static_cast<float>(std::max(std::sqrt(m2 / std::max(den - 1, 1.0)), c.minimum_scale));
                for (size_t j = i + 1 - c.patch_size; j <= i; ++j) {
                    out.loc[j] = loc; out.scale[j] = scale;
                    out.scaled[j] = affine_value(x[j], loc, scale, mask[j], c.use_asinh);
                }
            }
        }
    }
    return out;
}

InstanceStats instance_norm_stats(const oracle_config& c, const float* x, const int8_t* mask, size_t rows, size_t length) {  // scaler.cpp:60-90
    InstanceStats out;
    out.loc.resize(rows); out.scale.resize(rows); out.is_binary.resize(rows);
    std::vector<float> weighted(length), weights(length), squares(length);
    for (size_t r = 0; r < rows; ++r) {
        bool binary = true, any = false;
        for (size_t t = 0; t < length; ++t) {
            size_t i = r * length + t;
            weighted[t] = x[i] * static_cast<float>(mask[i]);
            weights[t] = static_cast<float>(mask[i]);
            any |= mask[i] != 0;
            binary &= !mask[i] || x[i] == 0 || x[i] == 1;
        }
        float n = std::max(cascade_sum(weights.data(), length, false), 1.0f);
        float loc = cascade_sum(weighted.data(), length, false) / n;
        for (size_t t = 0; t < length; ++t) {
            size_t i = r * length + t;
            float centered = (x[i] - loc) * static_cast<float>(mask[i]);
            squares[t] = centered * centered;
        }
        float var = cascade_sum(squares.data(), length, false) / n;
        float scale = std::max(std::sqrt(var), static_cast<float>(c.minimum_scale));
        out.is_binary[r] = binary && any;
        out.loc[r] = out.is_binary[r] ? 0.0f : loc;
        out.scale[r] = out.is_binary[r] ? 1.0f : scale;
    }
    return out;
}

void overwrite_known_rows(const oracle_config& c, const float* x, const int8_t* mask, const std::vector<int8_t>& known,
                          size_t length, ScaleResult& out) {  // scaler.cpp:92-107
    if (std::none_of(known.begin(), known.end(), [](int8_t k) { return k != 0; })) return;
    auto st = instance_norm_stats(c, x, mask, known.size(), length);
    for (size_t r = 0; r < known.size(); ++r) if (known[r]) {
        for (size_t t = 0; t < length; ++t) {
            size_t i = r * length + t;
            out.loc[i] = st.loc[r]; out.scale[i] = st.scale[r];
            out.scaled[i] = affine_value(x[i], st.loc[r], st.scale[r], mask[i], c.use_asinh && !st.is_binary[r]);
        }
    }
}

std::vector<float> clamp_nonfinite(const std::vector<float>& x, size_t last) {  // scaler.cpp:109-123
    std::vector<float> out = x;
    for (size_t i = 0; i < x.size(); i += last) {
        float lo = INFINITY, hi = -INFINITY;
        for (size_t j = i; j < i + last; ++j) if (std::isfinite(x[j])) { lo = std::min(lo, x[j]); hi = std::max(hi, x[j]); }
        for (size_t j = i; j < i + last; ++j) {
            if (x[j] == INFINITY) out[j] = std::isfinite(hi) ? hi : 0.0f;
            else if (x[j] == -INFINITY) out[j] = std::isfinite(lo) ? lo : 0.0f;
        }
    }
    return out;
}

std::vector<float> denormalize_quantiles(const std::vector<float>& x, const std::vector<float>& loc,
                                         const std::vector<float>& scale, size_t Q, bool use_asinh) {  // scaler.cpp:125-137
    size_t stride = x.size() / loc.size();
    std::vector<float> out(x.size());
    for (size_t i = 0; i < x.size(); ++i) {
        float v = use_asinh ? std::sinh(x[i]) : x[i];
        float product = v * scale[i / stride];
        out[i] = product + loc[i / stride];
    }
    return clamp_nonfinite(out, Q);
}

// ------------------------------------------------------------------------------------
// Masks (reference src/masks.cpp:8-34).
struct Masks {
    std::vector<int8_t> obs, key_valid, time, variate, active;
    std::vector<int64_t> first_group, inverse, positions, anchor;
    size_t enc_len = 0, N = 0, S = 0, L = 0;
};

Masks build_masks(const oracle_config& c, const int8_t* observed, size_t R, size_t T, size_t h,
                  const int64_t* groups, const int64_t* roles) {
    if (!R || !T || !h || T % c.patch_size) throw Error("invalid mask dimensions");
    for (size_t i = 0; i < R * T; ++i) if (observed[i] != 0 && observed[i] != 1) throw Error("observation mask must be boolean");
    bool cov = false;
    if (c.covariate_enabled && roles) for (size_t r = 0; r < R; ++r) { if (roles[r] < 0 || roles[r] > 2) throw Error("invalid row role"); cov |= roles[r] != 0; }
    size_t N = T / c.patch_size;
    if (cov && N <= h) throw Error("invalid mask horizon");
    size_t L = cov ? N - h : N, S = cov ? 2 * N : N + h, ndec = cov ? N : h;
    Masks a; a.N = N; a.S = S; a.L = L;
    a.obs.assign(R * N, 0); a.key_valid.resize(R * N);
    for (size_t r = 0; r < R; ++r) {
        bool started = false;
        for (size_t p = 0; p < N; ++p) {
            bool o = false;
            for (size_t j = 0; j < size_t(c.patch_size); ++j) o |= observed[r * T + p * c.patch_size + j] != 0;
            a.obs[r * N + p] = o; started |= o;
            a.key_valid[r * N + p] = o || (c.attend_missing_patches && started);
        }
    }
    std::vector<int64_t> unique(groups, groups + R);
    std::sort(unique.begin(), unique.end()); unique.erase(std::unique(unique.begin(), unique.end()), unique.end());
    a.inverse.resize(R); a.first_group.assign(unique.size(), int64_t(N));
    for (size_t r = 0; r < R; ++r) {
        size_t g = std::lower_bound(unique.begin(), unique.end(), groups[r]) - unique.begin();
        a.inverse[r] = g;
        for (size_t p = 0; p < N; ++p) if (a.obs[r * N + p]) { a.first_group[g] = std::min<int64_t>(a.first_group[g], p); break; }
    }
    for (auto& v : a.first_group) if (v == int64_t(N)) v = 0;
    a.positions.resize(R * S);
    for (size_t r = 0; r < R; ++r) for (size_t p = 0; p < S; ++p) a.positions[r * S + p] = int64_t(cov ? p % N : p) - a.first_group[a.inverse[r]];
    a.enc_len = N;
    a.time.assign(mul(mul(R, S), S), 0);
    if (cov) {
        a.anchor.resize(R * N); a.active.resize(R * N);
        for (size_t r = 0; r < R; ++r) for (size_t p = 0; p < N; ++p) {
            a.active[r * N + p] = p >= L;
            a.anchor[r * N + p] = p >= L ? int64_t(L + c.block_size * ((p - L) / c.block_size)) : 0;
        }
    }
    for (size_t r = 0; r < R; ++r) for (size_t q = 0; q < S; ++q) for (size_t k = 0; k < S; ++k) {
        bool yes = false;
        if (q < N && k < N) yes = (a.key_valid[r * N + k] && ((cov && roles[r] == 2) || k <= q)) || q == k;
        else if (q >= N && k < N) yes = a.key_valid[r * N + k] && (!cov || (a.active[r * N + q - N] && int64_t(k) < a.anchor[r * N + q - N]));
        else if (q >= N && k >= N) yes = q == k || (!cov ? k <= q : (k <= q && a.active[r * N + q - N] && a.active[r * N + k - N] && a.anchor[r * N + q - N] == a.anchor[r * N + k - N]));
        a.time[(r * S + q) * S + k] = yes;
    }
    if (R > 1) {
        a.variate.resize(mul(mul(S, R), R));
        for (size_t p = 0; p < N + ndec; ++p) for (size_t q = 0; q < R; ++q) for (size_t k = 0; k < R; ++k) {
            bool forbid = cov && ((roles[q] != 0 && roles[k] == 0) || (roles[q] == 2 && roles[k] != 2));
            a.variate[(p * R + q) * R + k] = q == k || (groups[q] == groups[k] && (p >= N || a.key_valid[k * N + p]) && !forbid);
        }
    }
    return a;
}

// ------------------------------------------------------------------------------------
// Weights.
struct Tensor {
    int type = ORACLE_F32;
    int64_t ne0 = 0, ne1 = 1;
    std::vector<float> f;         // F32 data, or the exact F32 value of F16 data
    std::vector<float> ft;        // f transposed to [ne0][ne1] for column-lane GEMM tiles
    std::vector<uint8_t> q8;      // Q8_0 blocks (34 bytes per 32 values)
};

}  // namespace

struct oracle_model {
    oracle_config c;
    int per_shot = 0;   // test override of ForecastRequest::per_shot_horizon_patches
    bool round_attention = false;   // test knob: f16-rounded q/k/v and sigmoid(gate), as the device stores them
    std::map<std::string, Tensor> t;
    const Tensor& get(const std::string& n) const {
        auto it = t.find(n); if (it == t.end()) throw Error("tensor not found: " + n); return it->second;
    }
    bool has(const std::string& n) const { return t.count(n) != 0; }
};

namespace {

int g_threads = 1;

// Register-tiled GEMM core: y[r,n] = (b ? s + b[n] : s) where s is, per output, the FMA
// chain over K split into panels of `panel` values (each panel chain starts at +0 and the
// panel sums are added in order to +0), or one chain when panel >= K. The tiling changes
// only which outputs are computed together, never the operation order of one output.
void gemm_core(const float* wt, const float* x, const float* b, size_t K, size_t N, size_t rows, float* y, size_t panel) {
    const bool single = panel >= K;
    const size_t step = single ? K : panel;
    const int64_t strips = int64_t((N + 15) / 16);
    // Column strips outermost: each thread keeps its 16-column weight strip in cache while
    // it streams the activation rows.
#pragma omp parallel for schedule(dynamic, 1) num_threads(g_threads)
    for (int64_t sidx = 0; sidx < strips; ++sidx) {
        const size_t c = size_t(sidx) * 16;
        for (size_t r0 = 0; r0 < rows; r0 += 4) {
            const size_t rc = std::min<size_t>(4, rows - r0);
            const float* xr[4];
            for (size_t i = 0; i < 4; ++i) xr[i] = x + (r0 + std::min(i, rc - 1)) * K;
            if (c + 16 <= N) {
                __m256 s[8], p[8];
                for (int i = 0; i < 8; ++i) s[i] = _mm256_setzero_ps();
                for (size_t start = 0; start < K; start += step) {
                    const size_t stop = std::min(K, start + step);
                    for (int i = 0; i < 8; ++i) p[i] = _mm256_setzero_ps();
                    for (size_t j = start; j < stop; ++j) {
                        const __m256 w0 = _mm256_loadu_ps(wt + j * N + c), w1 = _mm256_loadu_ps(wt + j * N + c + 8);
                        for (int i = 0; i < 4; ++i) {
                            const __m256 xb = _mm256_set1_ps(xr[i][j]);
                            p[2 * i] = _mm256_fmadd_ps(w0, xb, p[2 * i]);
                            p[2 * i + 1] = _mm256_fmadd_ps(w1, xb, p[2 * i + 1]);
                        }
                    }
                    if (single) for (int i = 0; i < 8; ++i) s[i] = p[i];
                    else for (int i = 0; i < 8; ++i) s[i] = _mm256_add_ps(s[i], p[i]);
                }
                for (size_t i = 0; i < rc; ++i) {
                    __m256 a = s[2 * i], bb = s[2 * i + 1];
                    if (b) { a = _mm256_add_ps(a, _mm256_loadu_ps(b + c)); bb = _mm256_add_ps(bb, _mm256_loadu_ps(b + c + 8)); }
                    _mm256_storeu_ps(y + (r0 + i) * N + c, a);
                    _mm256_storeu_ps(y + (r0 + i) * N + c + 8, bb);
                }
            } else {
                for (size_t i = 0; i < rc; ++i) for (size_t cc = c; cc < N; ++cc) {
                    float sum = 0;
                    for (size_t start = 0; start < K; start += step) {
                        const size_t stop = std::min(K, start + step);
                        float pp = 0;
                        for (size_t j = start; j < stop; ++j) pp = std::fma(wt[j * N + cc], xr[i][j], pp);
                        sum = single ? pp : sum + pp;
                    }
                    y[(r0 + i) * N + cc] = b ? sum + b[cc] : sum;
                }
            }
        }
    }
}

std::vector<float> transpose(const float* w, size_t K, size_t N) {
    std::vector<float> wt(K * N);
    for (size_t n = 0; n < N; ++n) for (size_t k = 0; k < K; ++k) wt[k * N + n] = w[n * K + k];
    return wt;
}

// F32 linear (reference src/layers.cpp:187-222): per output, 192-wide K panels of
// sequential FMA, panel sums added to +0 in order; K < 192 is one FMA chain; bias after.
void linear_f32(const float* wt, const float* x, const float* b, size_t K, size_t N, size_t rows, float* y) {
    gemm_core(wt, x, b, K, N, rows, y, K < 192 ? K : 192);
}

// Small-input F32 projection: one sequential FMA chain over all of K, bias after
// (reference src/head.cpp:264-268, head_linear_f32).
void head_linear_f32(const float* wt, const float* x, const float* b, size_t K, size_t N, size_t rows, float* y) {
    gemm_core(wt, x, b, K, N, rows, y, K);
}

// F32 head projection with float64 accumulation (reference src/head.cpp:269-274).
void head_linear_f64(const float* w, const float* x, size_t K, size_t N, size_t rows, float* y) {
#pragma omp parallel for schedule(static) num_threads(g_threads)
    for (int64_t r = 0; r < int64_t(rows); ++r)
        for (size_t n = 0; n < N; ++n) {
            double sum = 0;
            for (size_t k = 0; k < K; ++k) sum += double(w[n * K + k]) * double(x[r * K + k]);
            y[r * N + n] = float(sum);
        }
}

// ggml CPU mul_mat with an F16 weight: activations rounded to F16, products of F16 values
// accumulated in F32 (one FMA chain; ggml's own lane order is not pinned here).
void mulmat_f16(const float* wt16, const float* x, size_t K, size_t N, size_t rows, float* y) {
    std::vector<float> xr(rows * K);
    for (size_t i = 0; i < xr.size(); ++i) xr[i] = round_f16(x[i]);
    gemm_core(wt16, xr.data(), nullptr, K, N, rows, y, K);
}

// ggml CPU mul_mat with a Q8_0 weight: activations quantised to Q8_0 per 32-block
// (d = amax/127 stored as F16, q = round(x/d)), integer block dots scaled by d_w*d_x and
// accumulated in F32.
void mulmat_q8(const uint8_t* wq, const float* x, size_t K, size_t N, size_t rows, float* y) {
    const size_t nb = K / 32;
#pragma omp parallel for schedule(static) num_threads(g_threads)
    for (int64_t r = 0; r < int64_t(rows); ++r) {
        std::vector<int8_t> xq(K); std::vector<float> xd(nb);
        for (size_t b = 0; b < nb; ++b) {
            float amax = 0;
            for (size_t j = 0; j < 32; ++j) amax = std::max(amax, std::fabs(x[r * K + b * 32 + j]));
            float d = amax / 127.f, id = d ? 1.0f / d : 0.0f;
            xd[b] = f16_to_f32(f32_to_f16(d));
            for (size_t j = 0; j < 32; ++j) xq[b * 32 + j] = int8_t(std::lround(x[r * K + b * 32 + j] * id));
        }
        for (size_t n = 0; n < N; ++n) {
            const uint8_t* row = wq + n * nb * 34;
            float sum = 0;
            for (size_t b = 0; b < nb; ++b) {
                uint16_t dh; std::memcpy(&dh, row + b * 34, 2);
                const int8_t* qs = reinterpret_cast<const int8_t*>(row + b * 34 + 2);
                int isum = 0;
                for (size_t j = 0; j < 32; ++j) isum += int(qs[j]) * int(xq[b * 32 + j]);
                sum += (f16_to_f32(dh) * xd[b]) * float(isum);
            }
            y[r * N + n] = sum;
        }
    }
}

// Dispatch of one projection by weight type: F32 weights use linear_f32 or, when `small`
// is set and K < 192, head_linear_f32 (reference src/layers.cpp:250-256, src/head.cpp:279-286);
// reduced weights use ggml mul_mat plus the bias (src/weight_policy.hpp:23-30).
void project(const oracle_model& m, const std::string& base, const float* x, size_t rows, bool bias, bool small, std::vector<float>& y, bool precise = false) {
    const Tensor& w = m.get(base + ".weight");
    const float* b = bias ? m.get(base + ".bias").f.data() : nullptr;
    size_t K = w.ne0, N = w.ne1;
    y.assign(rows * N, 0.f);
    if (w.type == ORACLE_F32) {
        if (precise) { head_linear_f64(w.f.data(), x, K, N, rows, y.data()); if (b) for (size_t i = 0; i < y.size(); ++i) y[i] += b[i % N]; return; }
        if (small && K < 192) head_linear_f32(w.ft.data(), x, b, K, N, rows, y.data());
        else linear_f32(w.ft.data(), x, b, K, N, rows, y.data());
        return;
    }
    if (w.type == ORACLE_F16) mulmat_f16(w.ft.data(), x, K, N, rows, y.data());
    else mulmat_q8(w.q8.data(), x, K, N, rows, y.data());
    if (b) for (size_t i = 0; i < y.size(); ++i) y[i] = y[i] + b[i % N];
}

// RMSNorm (reference src/layers.cpp:279-287).
void rms_norm(const float* x, const float* w, size_t rows, size_t D, float eps, float* y) {
#pragma omp parallel for schedule(static) num_threads(g_threads)
    for (int64_t r = 0; r < int64_t(rows); ++r) {
        float mean = cascade_sum(x + r * D, D, true) / float(D);
        float inv = 1.0f / std::sqrt(mean + eps);
        for (size_t d = 0; d < D; ++d) y[r * D + d] = (x[r * D + d] * inv) * w[d];
    }
}

// SDPA over sequences addressed by an index function (reference src/layers.cpp:578-617,
// the path every AVX2 host takes: float64 q.k dots in ascending d, float scale and additive
// mask, ATen exp for full eight-lane chunks and libm exp for the tail, eight-lane sums,
// value contraction then one reciprocal multiply).
// tok(b, i) gives the token index of sequence position i in batch b; rows of q/k/v/out are
// D = H*hd floats per token. mask(b, t, j) is the additive mask.
template <class Tok, class Mask>
void sdpa_generic(const float* Q, const float* K, const float* V, float* Y, size_t hd, size_t H, size_t S,
                  size_t batches, size_t split, Tok tok, Mask mask) {
    const size_t D = H * hd;
    const float scale = float(1 / std::sqrt(double(hd)));
#pragma omp parallel num_threads(g_threads)
    {
        std::vector<float> lg(S), p(S);
#pragma omp for schedule(dynamic, 4)
        for (int64_t job = 0; job < int64_t(batches * H * S); ++job) {
            size_t h = job % H, t = job / H % S, b = job / (H * S);
            size_t keys = (split && t < split) ? split : S;
            const float* q = Q + tok(b, t) * D + h * hd;
            float mx = -INFINITY;
            for (size_t j = 0; j < keys; ++j) {
                const float* k = K + tok(b, j) * D + h * hd;
                double sum = 0;
                for (size_t d = 0; d < hd; ++d) sum += double(q[d]) * double(k[d]);
                lg[j] = float(sum) * scale + mask(b, t, j);
                mx = std::max(mx, lg[j]);
            }
            float sums[8] = {}; size_t end = keys / 8 * 8;
            for (size_t j = 0; j < keys; ++j) { p[j] = j < end ? attention_exp(lg[j] - mx) : float(std::exp(double(lg[j] - mx))); if (j < end) sums[j % 8] += p[j]; }
            float a0 = sums[0] + sums[4], a1 = sums[1] + sums[5], a2 = sums[2] + sums[6], a3 = sums[3] + sums[7];
            float sum = (a0 + a2) + (a1 + a3);
            for (size_t j = end; j < keys; ++j) sum += p[j];
            float reciprocal = 1.0f / float(sum);
            float* y = Y + tok(b, t) * D + h * hd;
            for (size_t d = 0; d < hd; ++d) {
                float acc = 0;
                for (size_t j = 0; j < keys; ++j) {
                    float vv = V[tok(b, j) * D + h * hd + d];
                    if (hd < 16) acc += p[j] * vv; else acc = std::fma(p[j], vv, acc);
                }
                y[d] = float(acc) * reciprocal;
            }
        }
    }
}

// RoPE: x*cos + rotate_half(x)*sin, each op rounded (reference src/layers.cpp:238-246).
void apply_rope(float* x, const float* cos, const float* sin, size_t tokens, size_t H, size_t hd) {
    const size_t half = hd / 2;
    for (size_t t = 0; t < tokens; ++t) for (size_t h = 0; h < H; ++h) {
        float* v = x + (t * H + h) * hd;
        std::vector<float> orig(v, v + hd);
        for (size_t d = 0; d < hd; ++d) {
            float rot = d < half ? -orig[d + half] : orig[d - half];
            float a = orig[d] * cos[t * hd + d];
            float b = rot * sin[t * hd + d];
            v[d] = a + b;
        }
    }
}

// Transformer (reference src/encoder.cpp:93-154, full-graph mode).
std::vector<float> run_encoder(const oracle_model& m, std::vector<float> x, size_t R, size_t S, const Masks& mk) {
    const auto& c = m.c;
    const size_t D = c.d_model, H = c.num_heads, hd = D / H, M = R * S;
    // Additive masks (encoder.cpp:100-114).
    std::vector<float> tadd(R * S * S), vadd(S * R * R);
    for (size_t i = 0; i < tadd.size(); ++i) tadd[i] = mk.time[i] ? 0.f : -INFINITY;
    for (size_t i = 0; i < vadd.size(); ++i) vadd[i] = mk.variate.empty() ? 0.f : (mk.variate[i] ? 0.f : -INFINITY);
    // RoPE tables gathered by position (reference src/rope.cpp:8-22).
    std::vector<float> cosg(M * hd), sing(M * hd);
    const Tensor& tc = m.get("rope.cos"); const Tensor& ts = m.get("rope.sin");
    for (size_t i = 0; i < M; ++i) {
        int64_t idx = mk.positions[i] - c.rope_table_pos_min;
        if (idx < 0 || idx >= tc.ne1) throw Error("position outside stored RoPE table");
        std::memcpy(&cosg[i * hd], &tc.f[idx * hd], hd * 4); std::memcpy(&sing[i * hd], &ts.f[idx * hd], hd * 4);
    }
    std::vector<float> norm(M * D), fused, q(M * D), k(M * D), v(M * D), att(M * D), gate, outp, z, hid;
    for (int li = 0; li < c.n_layers; ++li) {
        std::string b = "blk." + std::to_string(li) + ".";
        auto axes = layer_axes(c.schedule[li]);
        for (size_t j = 0; j < axes.size(); ++j) {
            bool time = axes[j];
            std::string a = b + "attn." + std::to_string(j) + ".";
            rms_norm(x.data(), m.get(b + "attn_norm." + std::to_string(j) + ".weight").f.data(), M, D, c.norm_eps, norm.data());
            project(m, a + "qkv", norm.data(), M, c.attn_bias, false, fused);
            for (size_t t = 0; t < M; ++t) for (size_t i = 0; i < D; ++i) {
                q[t * D + i] = fused[t * 3 * D + i]; k[t * D + i] = fused[t * 3 * D + D + i]; v[t * D + i] = fused[t * 3 * D + 2 * D + i];
            }
            if (time) {
                apply_rope(q.data(), cosg.data(), sing.data(), M, H, hd);
                apply_rope(k.data(), cosg.data(), sing.data(), M, H, hd);
            }
            if (m.round_attention)
                for (size_t i = 0; i < M * D; ++i) { q[i] = round_f16(q[i]); k[i] = round_f16(k[i]); v[i] = round_f16(v[i]); }
            if (time) {
                sdpa_generic(q.data(), k.data(), v.data(), att.data(), hd, H, S, R, mk.enc_len,
                             [S](size_t bb, size_t i) { return bb * S + i; },
                             [&](size_t bb, size_t t, size_t jj) { return tadd[(bb * S + t) * S + jj]; });
            } else {
                // Variate axis: sequence = rows, batch = slots (encoder.cpp:128,134).
                sdpa_generic(q.data(), k.data(), v.data(), att.data(), hd, H, R, S, 0,
                             [S](size_t bb, size_t i) { return i * S + bb; },
                             [&](size_t bb, size_t t, size_t jj) { return vadd[(bb * R + t) * R + jj]; });
            }
            bool gated = (time ? c.time_gate : c.variate_gate) == 1;
            if (gated) {
                project(m, a + "gate", norm.data(), M, c.attn_bias, false, gate);
                for (size_t i = 0; i < M * D; ++i) {
                    float sg = 1.0f / (1.0f + activation_exp(-gate[i]));
                    att[i] = att[i] * (m.round_attention ? round_f16(sg) : sg);
                }
            }
            project(m, a + "out", att.data(), M, c.attn_bias, false, outp);
            for (size_t i = 0; i < M * D; ++i) x[i] = x[i] + outp[i];
        }
        rms_norm(x.data(), m.get(b + "ffn_norm.weight").f.data(), M, D, c.norm_eps, norm.data());
        project(m, b + "ffn_w12", norm.data(), M, c.mlp_bias, false, z);
        const size_t F = c.mlp_hidden_dim;
        hid.resize(M * F);
        for (size_t t = 0; t < M; ++t) for (size_t i = 0; i < F; ++i) {
            float u = z[t * 2 * F + F + i];
            float s = u / (1.0f + activation_exp(-u));
            hid[t * F + i] = z[t * 2 * F + i] * s;
        }
        project(m, b + "ffn_w3", hid.data(), M, c.mlp_bias, false, outp);
        for (size_t i = 0; i < M * D; ++i) x[i] = x[i] + outp[i];
    }
    rms_norm(x.data(), m.get("out_norm.weight").f.data(), M, D, c.norm_eps, norm.data());
    return norm;
}

// Patch-embedding projection actually used by prediction (reference src/head.cpp:329-340).
std::vector<float> context_patch_projection(const oracle_model& m, const std::vector<float>& features, size_t rows) {
    std::vector<float> h, o, r;
    project(m, "patch.hidden", features.data(), rows, true, true, h);
    for (auto& v : h) v = v / (1.f + activation_exp(-v));
    project(m, "patch.out", h.data(), rows, true, true, o);
    project(m, "patch.res", features.data(), rows, true, true, r);
    for (size_t i = 0; i < o.size(); ++i) o[i] = o[i] + r[i];
    return o;
}

// Patch features [values(ps), 1-observed(ps)] per patch (reference src/encoder.cpp:12-23).
std::vector<float> patch_features(const oracle_config& c, const std::vector<float>& scaled, const int8_t* observed, size_t rows, size_t length) {
    size_t ps = c.patch_size;
    std::vector<float> f(2 * rows * length);
    for (size_t r = 0; r < rows; ++r) for (size_t t = 0; t < length; ++t) {
        size_t i = r * length + t, j = (r * (length / ps) + t / ps) * 2 * ps + t % ps;
        f[j] = scaled[i]; f[j + ps] = 1 - observed[i];
    }
    return f;
}

// Quantile head (reference src/head.cpp:314-323, precise path).
std::vector<float> head_project(const oracle_model& m, const std::vector<float>& dec, size_t rows) {
    std::vector<float> hid, out, res;
    project(m, "head.hidden", dec.data(), rows, false, false, hid, true);
    for (auto& v : hid) v = v / (1.f + activation_exp(-v));
    project(m, "head.out", hid.data(), rows, false, false, out, true);
    project(m, "head.res", dec.data(), rows, false, false, res, true);
    for (size_t i = 0; i < out.size(); ++i) out[i] = out[i] + res[i];
    return out;
}

// reference src/head.cpp:294-313
std::vector<float> monotone_quantiles(const oracle_config& c, const std::vector<float>& raw) {
    const size_t Q = c.num_quantiles, mi = median_index(c);
    if (!Q || raw.empty() || raw.size() % Q) throw Error("invalid raw quantile layout");
    for (float x : raw) if (std::isnan(x)) throw Error("NaN raw quantile");
    std::vector<float> widths(Q), out(raw.size());
    for (size_t q = 0; q < Q; ++q) {
        double w = q < mi ? c.knots[q + 1] - c.knots[q] : q > mi ? c.knots[q] - c.knots[q - 1] : 0;
        widths[q] = float(c.quantile_width_factor) * float(w);
    }
    const float limit = std::numeric_limits<float>::max();
    auto clamp = [&](float x) { if (std::isnan(x)) throw Error("NaN monotone quantile"); return std::max(-limit, std::min(limit, x)); };
    for (size_t i = 0; i < raw.size(); i += Q) {
        auto inc = [&](size_t q) { float x = raw[i + q]; return widths[q] * (x > 20 ? x : std::log1p(activation_exp(x))); };
        float median = raw[i + mi]; double sum = 0; out[i + mi] = clamp(median);
        for (size_t q = mi + 1; q < Q; ++q) { sum += inc(q); out[i + q] = clamp(median + float(sum)); }
        sum = 0;
        for (size_t q = mi; q-- > 0;) { sum += inc(q); out[i + q] = clamp(median - float(sum)); }
    }
    return out;
}

struct BlockPrediction { std::vector<float> output, normalized, loc, scale; };

// reference src/predict_block.cpp:6-20 (context-only) and :26-56 (covariate window).
BlockPrediction predict_block(const oracle_model& m, const std::vector<float>& inputs, const std::vector<int8_t>& observed,
                              size_t R, size_t T, size_t h, const std::vector<int64_t>& groups, const std::vector<int64_t>& roles,
                              const std::vector<float>& future, const std::vector<int8_t>& fm) {
    const auto& c = m.c;
    size_t ps = c.patch_size, D = c.d_model, Q = c.num_quantiles;
    if (!R || !T || !h || T % ps || h > size_t(c.block_size) || inputs.size() != R * T || observed.size() != inputs.size() || groups.size() != R || (!roles.empty() && roles.size() != R))
        throw Error("invalid prediction dimensions");
    if (T > size_t(c.context_length) + ps - 1) throw Error("context exceeds stored position range");
    for (float v : inputs) if (!std::isfinite(v)) throw Error("prediction inputs must be prepared finite values");
    for (float v : future) if (!std::isfinite(v)) throw Error("known future must be prepared finite values");
    bool cov = c.covariate_enabled && !roles.empty() && std::any_of(roles.begin(), roles.end(), [](int64_t v) { return v != 0; });
    const float* query = m.get("patch.forecast_query").f.data();
    BlockPrediction out;
    if (!cov) {
        auto a = build_masks(c, observed.data(), R, T, h, groups.data(), nullptr);
        size_t L = T / ps, S = L + h;
        auto scaled = scale_rows(c, inputs.data(), observed.data(), R, T);
        auto feats = patch_features(c, scaled.scaled, observed.data(), R, T);
        auto emb = context_patch_projection(m, feats, R * L);
        std::vector<float> x(R * S * D);
        for (size_t r = 0; r < R; ++r) {
            std::copy_n(emb.begin() + r * L * D, L * D, x.begin() + r * S * D);
            for (size_t j = L; j < S; ++j) std::copy_n(query, D, x.begin() + (r * S + j) * D);
        }
        auto norm = run_encoder(m, std::move(x), R, S, a);
        std::vector<float> dec(R * h * D);
        for (size_t r = 0; r < R; ++r) std::copy_n(norm.begin() + (r * S + L) * D, h * D, dec.begin() + r * h * D);
        out.normalized = monotone_quantiles(c, head_project(m, dec, R * h));
        for (size_t r = 0; r < R; ++r) { out.loc.push_back(scaled.loc[r * T + T - 1]); out.scale.push_back(scaled.scale[r * T + T - 1]); }
        out.output = denormalize_quantiles(out.normalized, out.loc, out.scale, Q, c.use_asinh);
        return out;
    }
    if (std::find(roles.begin(), roles.end(), 2) != roles.end() && !supports_known_covariates(c)) throw Error("this checkpoint cannot condition on known-future covariates");
    size_t Hs = h * ps, W = T + Hs, N = W / ps, L = T / ps, S = 2 * N;
    std::vector<float> full(R * W, 0); std::vector<int8_t> obs(full.size(), 0), known(R);
    for (size_t r = 0; r < R; ++r) {
        std::copy_n(inputs.begin() + r * T, T, full.begin() + r * W);
        std::copy_n(observed.begin() + r * T, T, obs.begin() + r * W);
        known[r] = roles[r] == 2;
        if (!future.empty()) { std::copy_n(future.begin() + r * Hs, Hs, full.begin() + r * W + T); std::copy_n(fm.begin() + r * Hs, Hs, obs.begin() + r * W + T); }
    }
    auto a = build_masks(c, obs.data(), R, W, h, groups.data(), roles.data());
    auto scaled = scale_rows(c, full.data(), obs.data(), R, W);
    overwrite_known_rows(c, full.data(), obs.data(), known, W, scaled);
    auto feats = patch_features(c, scaled.scaled, obs.data(), R, W);
    auto emb = context_patch_projection(m, feats, R * N);
    std::vector<float> x(R * S * D);
    for (size_t r = 0; r < R; ++r) {
        std::copy_n(emb.begin() + r * N * D, N * D, x.begin() + r * S * D);
        for (size_t p = N; p < S; ++p) std::copy_n(query, D, x.begin() + (r * S + p) * D);
    }
    auto norm = run_encoder(m, std::move(x), R, S, a);
    std::vector<float> dec(R * N * D);
    for (size_t r = 0; r < R; ++r) std::copy_n(norm.begin() + (r * S + N) * D, N * D, dec.begin() + r * N * D);
    auto quantiles = monotone_quantiles(c, head_project(m, dec, R * N));
    out.normalized.resize(R * Hs * Q);
    for (size_t r = 0; r < R; ++r) {
        std::copy_n(quantiles.begin() + (r * N + L) * ps * Q, Hs * Q, out.normalized.begin() + r * Hs * Q);
        out.loc.push_back(scaled.loc[r * W + (L - 1) * ps]); out.scale.push_back(scaled.scale[r * W + (L - 1) * ps]);
    }
    out.output = denormalize_quantiles(out.normalized, out.loc, out.scale, Q, c.use_asinh);
    return out;
}

// ------------------------------------------------------------------------------------
// Refine (reference src/refine.cpp).
struct WState { double w = 0, mean = 0, m2 = 0; };
WState combine(WState a, WState b) {  // refine.cpp:24-31
    double w = a.w + b.w, safe = std::max(w, std::numeric_limits<double>::min());
    double delta = b.mean - a.mean;
    double mean = a.mean + delta * b.w / safe;
    double m2 = a.m2 + b.m2 + delta * delta * a.w * b.w / safe;
    return {w, w == 0 ? 0 : mean, w == 0 ? 0 : m2};
}

void block_frames(const oracle_config& c, const float* x, const int8_t* mask, const double* median, size_t rows,
                  size_t length, size_t patches, double* oloc, double* oscale) {  // refine.cpp:32-75
    size_t ps = c.patch_size, cp = length / ps;
    const double clip = std::pow(double(std::numeric_limits<float>::max()), 0.5) / 1e3;
    std::vector<double> terms(ps), folded(ps);
    for (size_t r = 0; r < rows; ++r) {
        std::vector<WState> states(cp + patches);
        for (size_t p = 0; p < cp; ++p) {
            size_t start = r * length + p * ps;
            for (size_t k = 0; k < ps; ++k) terms[k] = mask[start + k];
            double w = numpy_sum(terms.data(), ps);
            for (size_t k = 0; k < ps; ++k) terms[k] = double(x[start + k]) * mask[start + k];
            double mean = numpy_sum(terms.data(), ps) / std::max(w, 1.0);
            for (size_t k = 0; k < ps; ++k) { double d = double(x[start + k]) - mean; terms[k] = mask[start + k] * (d * d); }
            double m2 = numpy_sum(terms.data(), ps);
            states[p] = {w, w == 0 ? 0 : mean, w == 0 ? 0 : m2};
        }
        for (size_t d = 1; d < states.size();) {
            auto previous = states;
            for (size_t i = 0; i < states.size(); ++i) states[i] = combine(i >= d ? previous[i - d] : WState{}, previous[i]);
            if (d > states.size() / 2) break;
            d *= 2;
        }
        WState state = states[cp - 1]; double offset = state.mean;
        for (size_t j = 0; j < patches; ++j) {
            double var = std::max(state.m2 / std::max(state.w - 1, 1.0), 0.0);
            double scale = std::max(std::sqrt(var), c.minimum_scale);
            oloc[r * patches + j] = state.mean; oscale[r * patches + j] = scale;
            for (size_t k = 0; k < ps; ++k) {
                double v = median[(r * patches + j) * ps + k] * scale + state.mean - offset;
                folded[k] = std::clamp(v, -clip, clip) + offset;
            }
            double mean = numpy_sum(folded.data(), ps) / double(ps);
            for (size_t k = 0; k < ps; ++k) { double d = folded[k] - mean; terms[k] = d * d; }
            state = combine(state, {double(ps), mean, numpy_sum(terms.data(), ps)});
        }
    }
}

std::vector<float> refine_block(const oracle_config& c, const std::vector<float>& q, const float* x, const int8_t* mask,
                                size_t rows, size_t length, size_t patches, const std::vector<int8_t>& targets) {  // refine.cpp:77-106
    size_t steps = patches * c.patch_size, Q = c.num_quantiles, mi = median_index(c);
    if (q.size() != rows * steps * Q) throw Error("refine: invalid quantile shape");
    if (patches <= 1) return q;
    auto anchor = scale_rows(c, x, mask, rows, length);
    std::vector<double> median(rows * steps);
    for (size_t r = 0; r < rows; ++r) for (size_t t = 0; t < steps; ++t)
        median[r * steps + t] = (double(q[(r * steps + t) * Q + mi]) - anchor.loc[r * length + length - 1]) / anchor.scale[r * length + length - 1];
    std::vector<double> floc(rows * patches), fscale(rows * patches);
    block_frames(c, x, mask, median.data(), rows, length, patches, floc.data(), fscale.data());
    std::vector<float> out(q.size());
    for (size_t r = 0; r < rows; ++r) {
        float loc0 = anchor.loc[r * length + length - 1], scale0 = anchor.scale[r * length + length - 1];
        for (size_t t = 0; t < steps; ++t) {
            size_t j = t / c.patch_size;
            float loc = j ? float(floc[r * patches + j]) : loc0, scale = j ? float(fscale[r * patches + j]) : scale0;
            for (size_t k = 0; k < Q; ++k) { size_t i = (r * steps + t) * Q + k; float norm = (q[i] - loc0) / scale0; float v = norm * scale; out[i] = v + loc; }
        }
    }
    out = clamp_nonfinite(out, Q);
    for (size_t r = 0; r < rows; ++r) if (!targets.empty() && !targets[r]) std::copy_n(q.begin() + r * steps * Q, steps * Q, out.begin() + r * steps * Q);
    return out;
}

// ------------------------------------------------------------------------------------
// Covariate assembly (reference src/covariates.cpp).
struct Assembled {
    size_t rows_count = 0, length = 0, horizon = 0;
    std::vector<float> rows, future; std::vector<int8_t> mask, future_mask; std::vector<int64_t> roles, groups;
};
float finite_value(float v) { return std::isnan(v) ? 0 : std::isinf(v) ? std::copysign(std::numeric_limits<float>::max(), v) : v; }
void codes_valid(const std::vector<double>& x) { for (double v : x) if (std::isinf(v)) throw Error("categorical covariates must hold finite codes or NaN; got an infinite value"); }

struct TargetEncoding { std::vector<float> past, future; };
TargetEncoding target_encode(const std::vector<double>& target, const std::vector<double>& past, const std::vector<double>& future, double smooth) {  // covariates.cpp:14-25
    codes_valid(past); codes_valid(future);
    auto cats = past;
    cats.erase(std::remove_if(cats.begin(), cats.end(), [](double x) { return !std::isfinite(x); }), cats.end());
    std::sort(cats.begin(), cats.end()); cats.erase(std::unique(cats.begin(), cats.end()), cats.end());
    size_t nan = cats.size();
    std::vector<double> values(target.size()), sums(nan + 1), counts(nan + 1); double count = 0;
    auto slot = [&](double code) { if (std::isnan(code)) return nan; auto it = std::lower_bound(cats.begin(), cats.end(), code); return it != cats.end() && *it == code ? size_t(it - cats.begin()) : nan + 1; };
    for (size_t i = 0; i < target.size(); ++i) if (std::isfinite(target[i])) { values[i] = target[i]; ++count; }
    double mean = count ? numpy_sum(values.data(), values.size()) / count : 0;
    for (size_t i = 0; i < past.size(); ++i) { size_t s = slot(past[i]); sums[s] += values[i]; counts[s] += std::isfinite(target[i]) ? 1 : 0; }
    std::vector<double> lookup(nan + 2, mean);
    for (size_t i = 0; i <= nan; ++i) lookup[i] = (smooth * mean + sums[i]) / (smooth + counts[i]);
    TargetEncoding e;
    for (double v : past) e.past.push_back(float(lookup[slot(v)]));
    for (double v : future) e.future.push_back(float(lookup[slot(v)]));
    return e;
}

Assembled assemble_rows(const oracle_config& c, const oracle_request& rq) {  // covariates.cpp:32-72
    size_t B = rq.B, V = rq.V, T = rq.T, H = rq.prediction_length, P = rq.c_past, K = rq.c_known, CP = rq.cc_past, CK = rq.cc_known;
    if (!B || !V || !T || !H) throw Error("invalid row dimensions");
    size_t TH = T + H, BV = B * V;
    std::vector<float> context(rq.context, rq.context + BV * T);
    std::vector<int8_t> user;
    if (rq.observation_mask) { user.resize(BV * T); for (size_t i = 0; i < user.size(); ++i) { if (rq.observation_mask[i] > 1) throw Error("observation mask must be boolean"); user[i] = rq.observation_mask[i]; } }
    std::vector<float> past(rq.past_cov ? rq.past_cov : nullptr, rq.past_cov ? rq.past_cov + B * P * T : nullptr);
    std::vector<float> known(rq.known_cov ? rq.known_cov : nullptr, rq.known_cov ? rq.known_cov + B * K * TH : nullptr);
    std::vector<double> cp(rq.cat_past ? rq.cat_past : nullptr, rq.cat_past ? rq.cat_past + B * CP * T : nullptr);
    std::vector<double> ck(rq.cat_known ? rq.cat_known : nullptr, rq.cat_known ? rq.cat_known + B * CK * TH : nullptr);
    if ((P || K || CP || CK) && !c.covariate_enabled) throw Error("this checkpoint was not trained with covariates");
    if ((K || CK) && !supports_known_covariates(c)) throw Error("this checkpoint cannot condition on known-future covariates");
    codes_valid(cp); codes_valid(ck);
    size_t cap = rq.max_context ? size_t(rq.max_context) : size_t(c.context_length);
    if (cap > size_t(c.context_length)) throw Error("max_context exceeds stored position range");
    size_t kept = std::min(T, cap), ps = c.patch_size, pad = (ps - kept % ps) % ps, len = kept + pad, hor = (H + ps - 1) / ps * ps;
    size_t all = V + P + CP + K + CK, R = B * all;
    Assembled a; a.rows_count = R; a.length = len; a.horizon = hor;
    a.rows.assign(R * len, 0); a.mask.assign(a.rows.size(), 0); a.groups.resize(R);
    if (P || CP || K || CK) a.roles.resize(R);
    if (K || CK) { a.future.assign(R * hor, 0); a.future_mask.assign(a.future.size(), 0); }
    std::vector<float> filled(context.size()); std::vector<int8_t> obs(context.size());
    for (size_t r = 0; r < BV; ++r) { float prev = 0; for (size_t t = 0; t < T; ++t) { size_t i = r * T + t; obs[i] = std::isfinite(context[i]) && (user.empty() || user[i]); if (obs[i]) prev = context[i]; filled[i] = prev; } }
    auto encode = [&](const std::vector<double>& codes, size_t C, size_t width) {
        std::vector<float> out(codes.size());
        for (size_t b = 0; b < B; ++b) for (size_t j = 0; j < C; ++j) {
            size_t off = (b * C + j) * width;
            if (V != 1) { for (size_t t = 0; t < width; ++t) out[off + t] = float(codes[off + t]); continue; }
            std::vector<double> target(T); bool started = false;
            for (size_t t = 0; t < T; ++t) { started |= obs[b * T + t]; target[t] = started && t >= T - kept ? double(filled[b * T + t]) : NAN; }
            std::vector<double> p(codes.begin() + off, codes.begin() + off + T), f(codes.begin() + off + T, codes.begin() + off + width);
            auto e = target_encode(target, p, f, c.target_encoding_smooth);
            for (size_t t = 0; t < T; ++t) out[off + t] = std::isnan(target[t]) && std::isnan(p[t]) ? NAN : e.past[t];
            std::copy(e.future.begin(), e.future.end(), out.begin() + off + T);
        }
        return out;
    };
    auto ep = encode(cp, CP, T), ek = encode(ck, CK, TH);
    for (size_t b = 0; b < B; ++b) for (size_t j = 0; j < all; ++j) {
        size_t r = b * all + j; int role = j < V ? 0 : j < V + P + CP ? 1 : 2;
        a.groups[r] = b; if (!a.roles.empty()) a.roles[r] = role;
        const std::vector<float>* src; size_t off;
        if (j < V) { src = &filled; off = (b * V + j) * T; }
        else if (j < V + P) { src = &past; off = (b * P + j - V) * T; }
        else if (j < V + P + CP) { src = &ep; off = (b * CP + j - V - P) * T; }
        else if (j < V + P + CP + K) { src = &known; off = (b * K + j - V - P - CP) * TH; }
        else { src = &ek; off = (b * CK + j - V - P - CP - K) * TH; }
        for (size_t t = 0; t < kept; ++t) {
            size_t from = off + T - kept + t, to = r * len + pad + t; float v = (*src)[from];
            a.rows[to] = role ? finite_value(v) : v;
            a.mask[to] = role ? !std::isnan(v) : obs[(b * V + j) * T + T - kept + t];
        }
        if (role == 2) for (size_t t = 0; t < H; ++t) { float v = (*src)[off + T + t]; a.future[r * hor + t] = finite_value(v); a.future_mask[r * hor + t] = !std::isnan(v); }
    }
    return a;
}

// ------------------------------------------------------------------------------------
// Forecaster (reference src/forecaster.cpp).
template <class T>
std::vector<T> slice(const std::vector<T>& x, size_t rows, size_t width, size_t start, size_t n) {
    if (x.empty()) return {};
    std::vector<T> out(rows * n);
    for (size_t r = 0; r < rows; ++r) std::copy_n(x.begin() + r * width + start, n, out.begin() + r * n);
    return out;
}

std::vector<float> decode(const oracle_model& m, const Assembled& a, size_t H, size_t cap, size_t shot) {  // forecaster.cpp:19-67
    const auto& c = m.c; size_t ps = c.patch_size, Q = c.num_quantiles, R = a.rows_count, T = a.length;
    cap = cap ? cap : c.context_length; shot = shot ? shot : c.per_shot_horizon_patches; shot = std::min(shot, size_t(c.block_size));
    if (!H || !R || !T || T % ps || !shot || !cap || cap > size_t(c.context_length)) throw Error("invalid decode dimensions");
    const size_t patches = (H + ps - 1) / ps, full = patches * ps;
    auto context = a.rows; auto mask = a.mask; std::vector<int8_t> targets;
    if (!a.roles.empty()) { targets.resize(R); for (size_t r = 0; r < R; ++r) targets[r] = a.roles[r] == 0; }
    std::vector<float> output(R * H * Q);
    size_t remaining = patches, done = 0;
    while (remaining) {
        size_t block = std::min(shot, remaining), n = block * ps, offset = done * ps;
        auto future = slice(a.future, R, full, offset, n); auto fm = slice(a.future_mask, R, full, offset, n);
        auto pred = predict_block(m, context, mask, R, T, block, a.groups, a.roles, future, fm);
        auto q = refine_block(c, pred.output, context.data(), mask.data(), R, T, block, targets);
        size_t used = std::min(n, H - offset);
        for (size_t r = 0; r < R; ++r) std::copy_n(q.begin() + r * n * Q, used * Q, output.begin() + (r * H + offset) * Q);
        remaining -= block; done += block;
        if (!remaining) break;
        size_t joined = T + n, keep = joined > cap ? std::max(ps, (cap / ps) * ps) : joined, start = joined - keep;
        std::vector<float> next(R * keep); std::vector<int8_t> nm(next.size());
        for (size_t r = 0; r < R; ++r) for (size_t j = 0; j < keep; ++j) {
            size_t t = start + j, i = r * keep + j;
            if (t < T) { next[i] = context[r * T + t]; nm[i] = mask[r * T + t]; continue; }
            size_t k = t - T; float value = q[(r * n + k) * Q + median_index(c)]; int8_t observed = 1;
            if (!std::isfinite(value) || std::abs(value) >= c.extreme_value_threshold) value = 0;
            if (!a.roles.empty()) {
                if (a.roles[r] == 2 && !future.empty()) { value = future[r * n + k]; observed = fm[r * n + k]; }
                if (a.roles[r] == 1) { value = 0; observed = 0; }
            }
            next[i] = value; nm[i] = observed;
        }
        context = std::move(next); mask = std::move(nm); T = keep;
    }
    return output;
}

std::vector<float> raw(const oracle_model& m, const Assembled& a, const oracle_request& r) {  // forecaster.cpp:68-86
    const auto& c = m.c; size_t Q = c.num_quantiles, all = a.rows_count / r.B;
    auto decoded = decode(m, a, r.prediction_length, r.max_context, size_t(m.per_shot));
    size_t B = r.B, V = r.V, H = r.prediction_length;
    std::vector<float> out(B * V * H * Q);
    double cap = c.quantile_real_cap_k;
    ScaleResult frames; if (cap > 0) frames = scale_rows(c, a.rows.data(), a.mask.data(), a.rows_count, a.length);
    size_t nan = 0;
    for (size_t b = 0; b < B; ++b) for (size_t v = 0; v < V; ++v) {
        size_t row = b * all + v;
        float lo = std::numeric_limits<float>::infinity(), hi = -lo;
        if (cap > 0) {
            for (size_t t = 0; t < a.length; ++t) if (a.mask[row * a.length + t]) { lo = std::min(lo, a.rows[row * a.length + t]); hi = std::max(hi, a.rows[row * a.length + t]); }
            if (!std::isfinite(lo)) lo = 0;
            if (!std::isfinite(hi)) hi = 0;
            float width = frames.scale[row * a.length + a.length - 1] * float(cap); lo = lo - width; hi = hi + width;
        }
        for (size_t t = 0; t < H * Q; ++t) { float value = decoded[row * H * Q + t]; if (cap > 0) value = std::min(std::max(value, lo), hi); nan += std::isnan(value); out[(b * V + v) * H * Q + t] = value; }
    }
    if (nan) throw Error("forecast produced " + std::to_string(nan) + " NaN values; the input is degenerate");
    return out;
}

std::vector<float> forecast(const oracle_model& m, const oracle_request& r) {  // forecaster.cpp:87-108
    const auto& c = m.c;
    auto a = assemble_rows(c, r);
    auto out = raw(m, a, r);
    size_t Q = c.num_quantiles;
    bool sym = r.symmetric_averaging == -1 ? c.symmetric_averaging != 0 : r.symmetric_averaging != 0;
    bool clip = r.clip_nonnegative == -1 ? c.clip_nonnegative != 0 : r.clip_nonnegative != 0;
    if (sym) {
        for (size_t i = 0; i < Q; ++i) if (std::abs(c.knots[i] + c.knots[Q - 1 - i] - 1) >= 1e-9) throw Error("symmetric averaging needs quantile levels symmetric about 0.5");
        for (auto& x : a.rows) x = -x;
        for (auto& x : a.future) x = -x;
        auto mirrored = raw(m, a, r);
        for (size_t i = 0; i < out.size(); ++i) out[i] = 0.5f * (out[i] + (-mirrored[(i / Q) * Q + Q - 1 - i % Q]));
    }
    if (clip) {
        size_t BV = size_t(r.B) * r.V, T = r.T, HQ = size_t(r.prediction_length) * Q;
        for (size_t row = 0; row < BV; ++row) {
            bool any = false, eligible = true;
            for (size_t t = 0; t < T; ++t) {
                size_t i = row * T + t;
                bool observed = std::isfinite(r.context[i]) && (!r.observation_mask || r.observation_mask[i]);
                if (observed) { any = true; eligible &= r.context[i] >= 0; }
            }
            if (any && eligible) for (size_t i = row * HQ; i < (row + 1) * HQ; ++i) out[i] = std::max(out[i], 0.f);
        }
    }
    return out;
}

template <class F> int guarded(F f) {
    try { f(); g_error.clear(); return 0; }
    catch (const std::exception& e) { g_error = e.what(); return 1; }
    catch (...) { g_error = "unknown oracle error"; return 1; }
}

}  // namespace

extern "C" {

const char* oracle_last_error(void) { return g_error.c_str(); }

oracle_model* oracle_model_new(const oracle_config* cfg) { auto* m = new oracle_model; m->c = *cfg; return m; }
void oracle_model_set_per_shot(oracle_model* m, int32_t n) { m->per_shot = n; }
void oracle_model_set_round_attention(oracle_model* m, int32_t on) { m->round_attention = on != 0; }
void oracle_model_free(oracle_model* m) { delete m; }

int oracle_model_set(oracle_model* m, const char* name, const void* data, int32_t type, int64_t ne0, int64_t ne1) {
    return guarded([&] {
        Tensor t; t.type = type; t.ne0 = ne0; t.ne1 = ne1;
        size_t n = size_t(ne0) * size_t(ne1);
        if (type == ORACLE_F32) { t.f.resize(n); std::memcpy(t.f.data(), data, n * 4); }
        else if (type == ORACLE_F16) { t.f.resize(n); auto p = static_cast<const uint16_t*>(data); for (size_t i = 0; i < n; ++i) t.f[i] = f16_to_f32(p[i]); }
        else if (type == ORACLE_Q8_0) { if (ne0 % 32) throw Error("Q8_0 row not a multiple of 32"); t.q8.resize(n / 32 * 34); std::memcpy(t.q8.data(), data, t.q8.size()); }
        else throw Error("unsupported tensor type");
        if (type != ORACLE_Q8_0 && ne1 > 1) t.ft = transpose(t.f.data(), size_t(ne0), size_t(ne1));
        m->t[name] = std::move(t);
    });
}

int oracle_forecast(oracle_model* m, const oracle_request* r, float* out, int32_t threads) {
    return guarded([&] {
        g_threads = std::max(1, int(threads));
        auto v = forecast(*m, *r);
        std::memcpy(out, v.data(), v.size() * 4);
    });
}

int oracle_predict_block(oracle_model* m, const float* rows, const int8_t* observed, int64_t R, int64_t T, int64_t h,
                         const int64_t* groups, const int64_t* roles, const float* future, const int8_t* future_mask,
                         float* out, float* normalized, float* loc, float* scale, int32_t threads) {
    return guarded([&] {
        g_threads = std::max(1, int(threads));
        size_t n = size_t(R) * T, hs = size_t(h) * m->c.patch_size;
        std::vector<float> x(rows, rows + n); std::vector<int8_t> o(observed, observed + n);
        std::vector<int64_t> g(groups, groups + R), ro; if (roles) ro.assign(roles, roles + R);
        std::vector<float> f; std::vector<int8_t> fm;
        if (future) { f.assign(future, future + R * hs); fm.assign(future_mask, future_mask + R * hs); }
        auto p = predict_block(*m, x, o, R, T, h, g, ro, f, fm);
        std::memcpy(out, p.output.data(), p.output.size() * 4);
        if (normalized) std::memcpy(normalized, p.normalized.data(), p.normalized.size() * 4);
        if (loc) std::memcpy(loc, p.loc.data(), p.loc.size() * 4);
        if (scale) std::memcpy(scale, p.scale.data(), p.scale.size() * 4);
    });
}

int oracle_scale_rows(const oracle_config* c, const float* x, const int8_t* mask, int64_t rows, int64_t length, float* scaled, float* loc, float* scale) {
    return guarded([&] {
        auto r = scale_rows(*c, x, mask, rows, length);
        std::memcpy(scaled, r.scaled.data(), r.scaled.size() * 4); std::memcpy(loc, r.loc.data(), r.loc.size() * 4); std::memcpy(scale, r.scale.data(), r.scale.size() * 4);
    });
}

int oracle_instance_norm_stats(const oracle_config* c, const float* x, const int8_t* mask, int64_t rows, int64_t length, float* loc, float* scale, int8_t* is_binary) {
    return guarded([&] {
        auto r = instance_norm_stats(*c, x, mask, rows, length);
        std::memcpy(loc, r.loc.data(), rows * 4); std::memcpy(scale, r.scale.data(), rows * 4); std::memcpy(is_binary, r.is_binary.data(), rows);
    });
}

int oracle_mask_sizes(const oracle_config* c, int64_t R, int64_t T, int64_t h, int32_t cov, int64_t* N, int64_t* S, int64_t* L) {
    (void)R;
    int64_t n = T / c->patch_size; *N = n; *L = cov ? n - h : n; *S = cov ? 2 * n : n + h; return 0;
}

int oracle_build_masks(const oracle_config* c, const int8_t* observed, int64_t R, int64_t T, int64_t h, const int64_t* groups,
                       const int64_t* roles, int8_t* obs, int8_t* key_valid, int64_t* first_group, int64_t* positions,
                       int8_t* time_allowed, int8_t* variate, int8_t* active, int64_t* anchor) {
    return guarded([&] {
        auto a = build_masks(*c, observed, R, T, h, groups, roles);
        std::memcpy(obs, a.obs.data(), a.obs.size()); std::memcpy(key_valid, a.key_valid.data(), a.key_valid.size());
        std::memcpy(first_group, a.first_group.data(), a.first_group.size() * 8);
        std::memcpy(positions, a.positions.data(), a.positions.size() * 8);
        std::memcpy(time_allowed, a.time.data(), a.time.size());
        if (variate && !a.variate.empty()) std::memcpy(variate, a.variate.data(), a.variate.size());
        if (active && !a.active.empty()) std::memcpy(active, a.active.data(), a.active.size());
        if (anchor && !a.anchor.empty()) std::memcpy(anchor, a.anchor.data(), a.anchor.size() * 8);
    });
}

int oracle_sdpa(const float* q, const float* k, const float* v, const float* mask, int64_t hd, int64_t H, int64_t S, int64_t R,
                int64_t split, float* out, int32_t threads) {
    return guarded([&] {
        g_threads = std::max(1, int(threads));
        sdpa_generic(q, k, v, out, hd, H, S, R, split, [S](size_t b, size_t i) { return b * S + i; },
                     [&](size_t b, size_t t, size_t j) { return mask[(b * S + t) * S + j]; });
    });
}

int oracle_rms_norm(const float* x, const float* w, int64_t rows, int64_t D, float eps, float* out) {
    return guarded([&] { g_threads = 1; rms_norm(x, w, rows, D, eps, out); });
}

int oracle_linear_f32(const float* w, const float* x, const float* b, int64_t K, int64_t N, int64_t rows, float* y) {
    return guarded([&] { g_threads = 1; auto wt = transpose(w, K, N); linear_f32(wt.data(), x, b, K, N, rows, y); });
}

int oracle_monotone_quantiles(const oracle_config* c, const float* raw, int64_t n, float* out) {
    return guarded([&] { auto v = monotone_quantiles(*c, std::vector<float>(raw, raw + n)); std::memcpy(out, v.data(), n * 4); });
}

int oracle_denormalize(const float* x, const float* loc, const float* scale, int64_t rows, int64_t stride, int64_t Q, int32_t use_asinh, float* out) {
    return guarded([&] {
        auto v = denormalize_quantiles(std::vector<float>(x, x + rows * stride), std::vector<float>(loc, loc + rows), std::vector<float>(scale, scale + rows), Q, use_asinh);
        std::memcpy(out, v.data(), v.size() * 4);
    });
}

int oracle_refine_block(const oracle_config* c, const float* q, const float* x, const int8_t* mask, int64_t rows, int64_t length,
                        int64_t patches, const int8_t* targets, float* out) {
    return guarded([&] {
        size_t n = size_t(rows) * patches * c->patch_size * c->num_quantiles;
        std::vector<int8_t> tg; if (targets) tg.assign(targets, targets + rows);
        auto v = refine_block(*c, std::vector<float>(q, q + n), x, mask, rows, length, patches, tg);
        std::memcpy(out, v.data(), n * 4);
    });
}

int oracle_block_frames(const oracle_config* c, const float* x, const int8_t* mask, const double* median, int64_t rows, int64_t length,
                        int64_t patches, double* loc, double* scale) {
    return guarded([&] { block_frames(*c, x, mask, median, rows, length, patches, loc, scale); });
}

int oracle_head_linear_f64(const float* w, const float* x, int64_t K, int64_t N, int64_t rows, float* y) {
    return guarded([&] { g_threads = 1; head_linear_f64(w, x, K, N, rows, y); });
}

int oracle_sigmoid(const float* x, int64_t n, float* out) {
    for (int64_t i = 0; i < n; ++i) out[i] = 1.0f / (1.0f + activation_exp(-x[i]));
    return 0;
}

int oracle_assemble_rows(const oracle_config* c, const oracle_request* r, int64_t* R, int64_t* len, int64_t* hor,
                         float* rows, int8_t* mask, int64_t* groups, int64_t* roles, float* future, int8_t* future_mask) {
    return guarded([&] {
        auto a = assemble_rows(*c, *r);
        *R = int64_t(a.rows_count); *len = int64_t(a.length); *hor = int64_t(a.horizon);
        if (rows) std::memcpy(rows, a.rows.data(), a.rows.size() * 4);
        if (mask) std::memcpy(mask, a.mask.data(), a.mask.size());
        if (groups) std::memcpy(groups, a.groups.data(), a.groups.size() * 8);
        if (roles && !a.roles.empty()) std::memcpy(roles, a.roles.data(), a.roles.size() * 8);
        if (future && !a.future.empty()) std::memcpy(future, a.future.data(), a.future.size() * 4);
        if (future_mask && !a.future_mask.empty()) std::memcpy(future_mask, a.future_mask.data(), a.future_mask.size());
    });
}

float oracle_activation_exp(float x) { return activation_exp(x); }
float oracle_attention_exp(float x) { return attention_exp(x); }
double oracle_numpy_sum(const double* x, int64_t n) { return numpy_sum(x, n); }
float oracle_torch_sum_f32(const float* x, int64_t n) { return cascade_sum(x, n, false); }

}  // extern "C"
