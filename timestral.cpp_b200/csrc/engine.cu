// Device engine: weights in device layouts, workspace, and the forecast pipeline.
//
// One forecast runs both symmetric passes as one batch of 2R rows (positive rows, then the
// exact negation), so every kernel sees twice the rows and the passes cost one launch each.
// Per decode block (reference src/forecaster.cpp:19-67):
//   scale_rows -> patch projection -> 24 transformer layers -> out_norm (decoder tokens)
//   -> head GEMMs -> monotone/denormalise -> refine
// then cap, symmetric average and clip (src/forecaster.cpp:68-108) in one kernel.
#include "attention.cuh"
#include "common.cuh"
#include "engine.cuh"
#include "gguf.hpp"
#include "gemm_tc.cuh"
#include "rows.cuh"

#include <algorithm>
#include <atomic>
#include <cfloat>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <memory>
#include <stdexcept>

#include <nvtx3/nvToolsExt.h>

namespace tsb {

namespace {

// NVTX range of one forecast stage on the calling host thread (visible in Nsight Systems
// timelines beside the kernels it enqueues; a no-op when no profiler is attached).
struct Range {
    explicit Range(const char* name) { nvtxRangePushA(name); }
    Range(const char* fmt, int i) {
        char buf[48];
        std::snprintf(buf, sizeof(buf), fmt, i);
        nvtxRangePushA(buf);
    }
    ~Range() { nvtxRangePop(); }
    Range(const Range&) = delete;
    Range& operator=(const Range&) = delete;
};

void check(cudaError_t e, const char* what) {
    if (e != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}

float half_bits_to_float(uint16_t h) {
    __half_raw r;
    r.x = h;
    return __half2float(__half(r));
}
uint16_t float_to_half_bits(float f) {
    __half h = __float2half_rn(f);
    return reinterpret_cast<__half_raw&>(h).x;
}
// W[n][k] *= norm[k] over f16 rows of width K, rounded to f16: the RMSNorm weight folded into
// the weights of the GEMM that consumes the normalised rows (tensor-core path).
void fold_norm(std::vector<uint16_t>& W, size_t K, const float* norm) {
    for (size_t i = 0; i < W.size(); ++i) W[i] = float_to_half_bits(half_bits_to_float(W[i]) * norm[i % K]);
}

// Counts workspace reallocations in the process: a captured forecast graph holds the
// workspace addresses of its capture and is replayed only while this count is unchanged.
std::atomic<uint64_t> g_workspace_generation{0};

// Test hook: the next n workspace allocations in the process fail as an exhausted device
// would (cudaErrorMemoryAllocation), so that the error path of a forecast can be exercised
// without a GPU fault.
std::atomic<int> g_injected_alloc_failures{0};
bool take_injected_failure() {
    int n = g_injected_alloc_failures.load();
    while (n > 0)
        if (g_injected_alloc_failures.compare_exchange_weak(n, n - 1)) return true;
    return false;
}

struct DevBuf {
    void* p = nullptr;
    size_t bytes = 0;
    DevBuf() = default;
    DevBuf(const DevBuf&) = delete;
    DevBuf& operator=(const DevBuf&) = delete;
    ~DevBuf() { if (p) cudaFree(p); }
    void ensure(size_t n) {
        if (n <= bytes) return;
        g_workspace_generation.fetch_add(1);
        if (p) { cudaFree(p); p = nullptr; bytes = 0; }
        check(take_injected_failure() ? cudaErrorMemoryAllocation : cudaMalloc(&p, std::max<size_t>(n, 256)),
              "cudaMalloc workspace");
        bytes = std::max<size_t>(n, 256);
    }
    template <class T> T* as() const { return static_cast<T*>(p); }
};

// Block-quantised weights in the device format of the GEMM's dequantising prologue: int8
// values [N][K] and either (Q8_0) the f16 scale of every 32-value block, transposed to
// [K / 32][N], or (K-quants) an f32 scale and offset per 16 values, [K / 16][N][2]; ldd = N.
struct BlockW {
    const int8_t* q = nullptr;
    const __half* d = nullptr;
    const float* s = nullptr;
    int64_t ldd = 0;
};
// The same on the host while the weights are rearranged, in row order: d [N][K / 32] (Q8_0)
// or ab [N][K / 16][2] (scaled: K-quants).
struct BlockHost {
    std::vector<int8_t> q;
    std::vector<uint16_t> d;
    std::vector<float> ab;
    bool scaled = false;
    size_t N = 0, K = 0;
};

struct AttnW {
    bool time = true, gate = false;
    BlockW qkvg_blk, vg_blk, out_blk;   // block-quantised twins of qkvg, vg, out (null when not block-quantised)
    const float* norm = nullptr;
    // tensor-core path
    __half* qkvg = nullptr; float* b_qkvg = nullptr; int n_qkvg = 0;   // [3D or 4D][D]
    __half* vg = nullptr; float* b_vg = nullptr;                        // variate, group size 1: [v|gate] per tile
    __half* out = nullptr; float* b_out = nullptr;
    // CUDA-core path
    float* f_qkv = nullptr; float* fb_qkv = nullptr; float* f_gate = nullptr; float* fb_gate = nullptr;
    float* f_out = nullptr; float* fb_out = nullptr;
};
struct MlpW {
    const float* norm = nullptr;
    BlockW w12_blk, w3_blk;
    __half* w12 = nullptr; float* b12 = nullptr;    // tensor cores: [g|u] per tile
    __half* w3 = nullptr; float* b3 = nullptr;
    float* f12 = nullptr; float* fb12 = nullptr; float* f3 = nullptr; float* fb3 = nullptr;
};

constexpr int kTile = 256;  // tensor-core GEMM tile width (gemm_tc.cu BN)

}  // namespace

struct Engine::Impl {
    ModelView mv;
    int D = 0, H = 0, hd = 0, F = 0, ps = 0, Q = 0, P = 0;
    bool tc = false, round_a = false;
    RowConfig rc;
    std::vector<void*> allocs;
    // weights
    float* query = nullptr;
    float* cos_tab = nullptr; float* sin_tab = nullptr;
    int rope_half = 32;
    int rope_dup = 0;
    float* p_hid = nullptr; float* pb_hid = nullptr; float* p_res = nullptr; float* pb_res = nullptr;
    __half* p_out = nullptr; float* f_pout = nullptr; float* pb_out = nullptr;
    __half* p_hid_split = nullptr; __half* p_res_split = nullptr;   // [N][3K] = [hi | lo | hi]
    bool patch_tc = false;
    std::vector<std::vector<AttnW>> attn;
    std::vector<MlpW> mlp;
    const float* out_norm = nullptr;
    __half* h_hid = nullptr; __half* h_out = nullptr; __half* h_res = nullptr;
    BlockW p_out_blk, h_hid_blk, h_out_blk, h_res_blk;
    bool dq_prologue = false;    // block-quantised weights dequantised in the GEMM prologue (else the f16 copies)
    float* fh_hid = nullptr; float* fh_out = nullptr; float* fh_res = nullptr;
    // workspace
    DevBuf rows, mask, win, wmask, role, future, fmask, feat, aloc, ascale, caplo, caphi, capsc, first_obs, kv, rope_row,
        gbeg, gsize, clip_ok, x, xn, qb, kb, vb, gb, att, hb, zb, fused, gtmp, ph, dec, hh, hraw, qout, refined, scratch,
        decoded, err, next_rows, next_mask, feat16, pflag, panel_scratch;
    // RMSNorm carried by the GEMMs (tensor-core path): x16 = f16(x / 16) and per-row sums of
    // squares per 128-column slot, written by the residual-add epilogues; unit norm weights for
    // the sublayers that normalise with the RMSNorm kernel (the norm weights are folded into
    // the consuming weights); a flag that sends a forecast back through the unfused path.
    DevBuf x16, ssq, nflag, ones;
    struct Pending {            // the last forecast without covariates, for its fallback run
        bool valid = false;
        const void* ctx = nullptr; const void* umask = nullptr;
        int B = 0, V = 0, T = 0, H = 0;
        bool sym = false, clip = false;
        void* out = nullptr;
        int kept = 0, len = 0, patches = 0, shot = 0, R = 0, R2 = 0, cap = 0;
    } pending;
    bool fuse = true;            // allowed
    bool fuse_now = true;        // used by the running forecast
    bool force_fallback = false; // test hook: treat every fused forecast as flagged
    bool attn_simt = false;      // tensor-core path: attention on the CUDA-core kernels
    bool tail_enabled = true;    // decoder-token tail of the last layer (see RowMap tail)
    const BlockObserver* observer = nullptr;
    int shot_override = 0;       // patches per decode block (0: the model's)
    double cap_override = -1;    // cap factor (negative: the model's)
    int shot() const { return std::min(shot_override ? shot_override : (mv.per_shot ? mv.per_shot : 32), mv.block_size); }
    double cap_k() const { return cap_override >= 0 ? cap_override : mv.cap_k; }
    // Hands one finished decode block to the observer (device pointers, stream synchronised).
    void observe(int offset, int block, int Tc, int R2, int64_t ctx_stride, const float* fut, const int8_t* fmask,
                 int64_t fut_stride) {
        if (!observer || !observer->after) return;
        check(cudaStreamSynchronize(s), "sync");
        BlockView v;
        v.offset = offset; v.patches = block; v.length = Tc; v.rows = R2;
        v.context = win.as<float>(); v.mask = wmask.as<int8_t>(); v.context_stride = ctx_stride;
        v.future = fut; v.future_mask = fmask; v.future_stride = fut_stride;
        v.predicted = qout.as<float>(); v.refined = refined.as<float>();
        v.loc = aloc.as<float>(); v.scale = ascale.as<float>();
        observer->after(v);
    }
    const __half* a_in = nullptr;
    const float* ssq_in = nullptr;
    bool produce16 = false;
    // Decoder-token tail of the last layer: after its time attention every later op of the
    // layer is per token, and only the decoder tokens reach the head, so the out projection,
    // the one-row variate sublayer and the MLP run on those tokens alone (rows r * S + N + j,
    // j < h; the other tokens' results were never used). Same bits for the tokens kept.
    struct RowMap { int group = 0, stride = 0, offset = 0; };
    RowMap a_map, tail;
    int tail_rows = 0;
    // raw covariate request inputs and assembly scratch
    DevBuf cov_ctx, cov_umask, cov_past, cov_known, cov_cpast, cov_cknown, cov_first, cov_scratch;
    // request-sized buffers kept across calls (no allocation on the forecast path once warm)
    DevBuf req_ctx, req_umask, fut_slice, fmask_slice, out_rows;
    // CUDA-graph replay of single-block forecasts without covariates: the second call with
    // the same shapes, flags and device buffers is captured, later ones replay the graph.
    struct GraphKey {
        const void* ctx = nullptr; const void* umask = nullptr; void* out = nullptr;
        int B = 0, V = 0, T = 0, H = 0, max_context = 0, shot = 0;
        double cap_k = 0;
        bool sym = false, clip = false;
        bool operator==(const GraphKey& o) const {
            return ctx == o.ctx && umask == o.umask && out == o.out && B == o.B && V == o.V && T == o.T && H == o.H &&
                   max_context == o.max_context && sym == o.sym && clip == o.clip && shot == o.shot && cap_k == o.cap_k;
        }
    };
    bool graphs = true;
    bool have_last = false;
    GraphKey last_key, graph_key;
    cudaGraphExec_t graph_exec = nullptr;
    uint64_t graph_generation = 0;
    int64_t graph_launches = 0;
    void drop_graph() {
        if (graph_exec) cudaGraphExecDestroy(graph_exec);
        graph_exec = nullptr;
    }
    // timing
    bool timing = false;
    std::string timing_only;   // empty: every class
    struct Ev { cudaEvent_t a, b; std::string cls; };
    std::vector<Ev> events;
    size_t ev_used = 0;
    int64_t launches = 0;
    cudaStream_t s = nullptr;

    template <class T> T* dalloc(size_t n) {
        void* p = nullptr;
        check(cudaMalloc(&p, std::max<size_t>(n * sizeof(T), 16)), "cudaMalloc weights");
        allocs.push_back(p);
        return static_cast<T*>(p);
    }
    template <class T> T* upload(const T* h, size_t n) {
        T* d = dalloc<T>(n);
        check(cudaMemcpy(d, h, n * sizeof(T), cudaMemcpyHostToDevice), "upload");
        return d;
    }

    HostTensor t(const std::string& n) const { return mv.tensor(n); }

    // Row values of a weight as float (exact for F32/F16; block-quantised types dequantised).
    std::vector<float> rows_f32(const HostTensor& w) const {
        const size_t K = size_t(w.ne0), N = size_t(w.ne1);
        std::vector<float> out(K * N);
        if (w.type == TT_F32) std::memcpy(out.data(), w.data, out.size() * 4);
        else if (w.type == TT_F16) {
            const uint16_t* p = static_cast<const uint16_t*>(w.data);
            for (size_t i = 0; i < out.size(); ++i) out[i] = half_bits_to_float(p[i]);
        } else {
            // Block-quantised rows (Q8_0, Q4_K, Q5_K, Q6_K), dequantised as ggml publishes.
            const uint8_t* p = static_cast<const uint8_t*>(w.data);
            const size_t row = ts::ggml_row_bytes(uint32_t(w.type), int64_t(K));
            if (!row) throw std::runtime_error("unsupported weight type " + std::to_string(w.type));
            for (size_t n = 0; n < N; ++n)
                if (!ts::dequantize_row(uint32_t(w.type), p + n * row, int64_t(K), out.data() + n * K))
                    throw std::runtime_error("unsupported weight type " + std::to_string(w.type));
        }
        return out;
    }
    // Row values as f16 bits (F16 as stored; Q8_0 dequantised then rounded to f16).
    std::vector<uint16_t> rows_f16(const HostTensor& w) const {
        const size_t n = size_t(w.ne0) * size_t(w.ne1);
        std::vector<uint16_t> out(n);
        if (w.type == TT_F16) std::memcpy(out.data(), w.data, n * 2);
        else {
            auto f = rows_f32(w);
            for (size_t i = 0; i < n; ++i) out[i] = float_to_half_bits(f[i]);
        }
        return out;
    }
    const float* f32_tensor(const std::string& n) {
        auto w = t(n);
        if (w.type != TT_F32) throw std::runtime_error("tensor " + n + " must be F32");
        return upload(static_cast<const float*>(w.data), size_t(w.ne0) * size_t(w.ne1));
    }
    float* bias_or_null(const std::string& n) {
        if (!mv.has(n)) return nullptr;
        return const_cast<float*>(f32_tensor(n));
    }
    // --- block-quantised twins (the dequantising GEMM prologue's weight formats) -------
    static bool block_type(const HostTensor& w) {
        return (w.type == TT_Q8_0 && w.ne0 % 32 == 0) ||
               ((w.type == TT_Q4_K || w.type == TT_Q5_K || w.type == TT_Q6_K) && w.ne0 % 256 == 0);
    }
    // GGUF Q8_0 rows (blocks of 34 bytes: f16 d, then 32 int8 values) as values and scales;
    // K-quant rows as values with a scale and an offset per 16 values (ts::scaled_int8_row).
    static BlockHost block_rows(const HostTensor& w) {
        BlockHost h;
        h.K = size_t(w.ne0); h.N = size_t(w.ne1);
        if (w.type != TT_Q8_0) {
            h.scaled = true;
            h.q.resize(h.N * h.K);
            h.ab.resize(h.N * (h.K / 16) * 2);
            std::vector<float> a(h.K / 16), b(h.K / 16);
            const size_t row = ts::ggml_row_bytes(uint32_t(w.type), int64_t(h.K));
            for (size_t n = 0; n < h.N; ++n) {
                if (!ts::scaled_int8_row(uint32_t(w.type), static_cast<const uint8_t*>(w.data) + n * row, int64_t(h.K),
                                         h.q.data() + n * h.K, a.data(), b.data()))
                    throw std::runtime_error("unsupported weight type " + std::to_string(w.type));
                for (size_t g = 0; g < h.K / 16; ++g) {
                    h.ab[(n * (h.K / 16) + g) * 2] = a[g];
                    h.ab[(n * (h.K / 16) + g) * 2 + 1] = b[g];
                }
            }
            return h;
        }
        const size_t nb = h.K / 32;
        h.q.resize(h.N * h.K);
        h.d.resize(h.N * nb);
        const uint8_t* p = static_cast<const uint8_t*>(w.data);
        for (size_t n = 0; n < h.N; ++n)
            for (size_t b = 0; b < nb; ++b) {
                const uint8_t* blk = p + (n * nb + b) * 34;
                std::memcpy(&h.d[n * nb + b], blk, 2);
                std::memcpy(&h.q[n * h.K + b * 32], blk + 2, 32);
            }
        return h;
    }
    static void block_append(BlockHost& a, const BlockHost& b) {
        if (a.scaled != b.scaled) throw std::runtime_error("mixed block formats in one projection");
        a.q.insert(a.q.end(), b.q.begin(), b.q.end());
        a.d.insert(a.d.end(), b.d.begin(), b.d.end());
        a.ab.insert(a.ab.end(), b.ab.begin(), b.ab.end());
        a.N += b.N;
    }
    // Scale entries per row (f16 scales or f32 scale/offset values).
    static size_t d_per_row(const BlockHost& h) { return h.scaled ? 0 : h.K / 32; }
    static size_t ab_per_row(const BlockHost& h) { return h.scaled ? (h.K / 16) * 2 : 0; }
    // Rows [r0, r0 + n) of a twin.
    static BlockHost block_slice(const BlockHost& a, size_t r0, size_t n) {
        BlockHost h;
        h.K = a.K; h.N = n; h.scaled = a.scaled;
        const size_t nb = d_per_row(a), na = ab_per_row(a);
        h.q.assign(a.q.begin() + r0 * a.K, a.q.begin() + (r0 + n) * a.K);
        h.d.assign(a.d.begin() + r0 * nb, a.d.begin() + (r0 + n) * nb);
        h.ab.assign(a.ab.begin() + r0 * na, a.ab.begin() + (r0 + n) * na);
        return h;
    }
    // Two twins of `rows` rows each interleaved per tile, as interleave() does for f16 rows.
    static BlockHost block_interleave(const BlockHost& a, const BlockHost& b, size_t rows) {
        if (a.scaled != b.scaled) throw std::runtime_error("mixed block formats in one projection");
        BlockHost h;
        h.K = a.K; h.N = 2 * rows; h.scaled = a.scaled;
        const size_t nb = d_per_row(a), na = ab_per_row(a), half = kTile / 2;
        for (size_t tile = 0; tile < rows / half; ++tile)
            for (const BlockHost* src : {&a, &b}) {
                h.q.insert(h.q.end(), src->q.begin() + tile * half * a.K, src->q.begin() + (tile + 1) * half * a.K);
                h.d.insert(h.d.end(), src->d.begin() + tile * half * nb, src->d.begin() + (tile + 1) * half * nb);
                h.ab.insert(h.ab.end(), src->ab.begin() + tile * half * na, src->ab.begin() + (tile + 1) * half * na);
            }
        return h;
    }
    BlockW block_upload(const BlockHost& h) {
        BlockW w;
        w.q = upload(h.q.data(), h.q.size());
        w.ldd = int64_t(h.N);
        if (h.scaled) {
            const size_t ng = h.K / 16;
            std::vector<float> st(ng * h.N * 2);
            for (size_t n = 0; n < h.N; ++n)
                for (size_t g = 0; g < ng; ++g) {
                    st[(g * h.N + n) * 2] = h.ab[(n * ng + g) * 2];
                    st[(g * h.N + n) * 2 + 1] = h.ab[(n * ng + g) * 2 + 1];
                }
            w.s = upload(st.data(), st.size());
            return w;
        }
        const size_t nb = h.K / 32;
        std::vector<uint16_t> dt(nb * h.N);
        for (size_t n = 0; n < h.N; ++n)
            for (size_t b = 0; b < nb; ++b) dt[b * h.N + n] = h.d[n * nb + b];
        w.d = reinterpret_cast<const __half*>(upload(dt.data(), dt.size()));
        return w;
    }
    static bool unit_gains(const float* w, size_t n) {
        for (size_t i = 0; i < n; ++i)
            if (w[i] != 1.0f) return false;
        return true;
    }
    // B operand of a GEMM from a twin when the prologue mode is on (row offset into it).
    void block_b(GemmArgs& g, const BlockW& w, int64_t row0 = 0) const {
        if (!dq_prologue || !w.q) return;
        g.Bq = w.q + row0 * g.K;
        g.ldb = g.K;
        if (w.s) { g.Bs = w.s + 2 * row0; g.lds = w.ldd; }
        else { g.Bd = w.d + row0; g.ldd = w.ldd; }
    }

    // Two [rows][K] blocks interleaved per tile: [a rows t*128.. | b rows t*128..].
    static std::vector<uint16_t> interleave(const uint16_t* a, const uint16_t* b, size_t rows, size_t K) {
        std::vector<uint16_t> out(2 * rows * K);
        const size_t half = kTile / 2;
        for (size_t tile = 0; tile < rows / half; ++tile) {
            std::memcpy(&out[(2 * tile) * half * K], a + tile * half * K, half * K * 2);
            std::memcpy(&out[(2 * tile + 1) * half * K], b + tile * half * K, half * K * 2);
        }
        return out;
    }
    static std::vector<float> interleave_bias(const float* a, const float* b, size_t rows) {
        std::vector<float> out(2 * rows);
        const size_t half = kTile / 2;
        for (size_t tile = 0; tile < rows / half; ++tile)
            for (size_t i = 0; i < half; ++i) {
                out[2 * tile * half + i] = a ? a[tile * half + i] : 0.f;
                out[(2 * tile + 1) * half + i] = b ? b[tile * half + i] : 0.f;
            }
        return out;
    }

    void load() {
        const auto& m = mv;
        D = m.D; H = m.H; hd = D / H; F = m.F; ps = m.ps; Q = int(m.knots.size());
        // Tensor cores when every projection weight is reduced (F16/Q8_0) and the shapes
        // tile (head_dim 64, widths multiple of the 128-row pairing half tile).
        bool reduced = true;
        auto is_reduced = [&](const std::string& n) { return t(n).type != TT_F32; };
        reduced &= is_reduced("patch.out.weight") && is_reduced("head.hidden.weight") && is_reduced("head.out.weight") &&
                   is_reduced("head.res.weight");
        for (size_t i = 0; i < m.schedule.size(); ++i) {
            const std::string b = "blk." + std::to_string(i) + ".";
            reduced &= is_reduced(b + "ffn_w12.weight") && is_reduced(b + "ffn_w3.weight");
        }
        tc = reduced && hd == 64 && D % 128 == 0 && F % 128 == 0 && (ps * Q) % 16 == 0;
        round_a = reduced && !tc;
        // row config
        rc.ps = ps; rc.minimum_scale = m.minimum_scale; rc.use_asinh = m.use_asinh; rc.attend_missing = m.attend_missing;
        rc.Q = Q; rc.median = m.median; rc.pos_min = m.pos_min; rc.cap_k = m.cap_k; rc.extreme = m.extreme;
        if (Q > 64) throw std::runtime_error("more than 64 quantile levels are not supported");
        for (int q = 0; q < Q; ++q) {
            const double w = q < m.median ? m.knots[q + 1] - m.knots[q] : q > m.median ? m.knots[q] - m.knots[q - 1] : 0;
            rc.widths[q] = float(m.width_factor) * float(w);
        }
        // tables
        auto tc_ = t("rope.cos");
        P = int(tc_.ne1);
        rc.rope_len = P;
        cos_tab = upload(static_cast<const float*>(tc_.data), size_t(tc_.ne0) * P);
        sin_tab = upload(static_cast<const float*>(t("rope.sin").data), size_t(tc_.ne0) * P);
        {   // dims whose table entries are exactly cos 1, sin 0 at every position
            const float* c = static_cast<const float*>(tc_.data);
            const float* s = static_cast<const float*>(t("rope.sin").data);
            const int half = hd / 2;
            auto identity = [&](int d) {
                for (int p = 0; p < P; ++p)
                    if (c[size_t(p) * hd + d] != 1.f || s[size_t(p) * hd + d] != 0.f) return false;
                return true;
            };
            int active = half;
            while (active > 0 && identity(active - 1) && identity(active - 1 + half)) --active;
            for (int d = 0; d < active; ++d) if (identity(d) && identity(d + half)) { active = half; break; }
            rope_half = active;
            rope_dup = 1;
            for (int p = 0; p < P && rope_dup; ++p)
                for (int d = 0; d < half; ++d)
                    if (c[size_t(p) * hd + d] != c[size_t(p) * hd + d + half] || s[size_t(p) * hd + d] != s[size_t(p) * hd + d + half]) {
                        rope_dup = 0;
                        break;
                    }
        }
        query = const_cast<float*>(f32_tensor("patch.forecast_query"));
        p_hid = const_cast<float*>(f32_tensor("patch.hidden.weight")); pb_hid = bias_or_null("patch.hidden.bias");
        p_res = const_cast<float*>(f32_tensor("patch.res.weight")); pb_res = bias_or_null("patch.res.bias");
        pb_out = bias_or_null("patch.out.bias");
        if (tc) {
            auto v = rows_f16(t("patch.out.weight")); p_out = reinterpret_cast<__half*>(upload(v.data(), v.size()));
            if (block_type(t("patch.out.weight"))) p_out_blk = block_upload(block_rows(t("patch.out.weight")));
        }
        else { auto v = rows_f32(t("patch.out.weight")); f_pout = upload(v.data(), v.size()); }
        // Tensor-core patch projections (K = 2 * patch_size, F32 weights): the weights split into
        // f16 hi/lo terms, rows of 3K f16 that stay 16-byte aligned.
        patch_tc = tc && (3 * 2 * ps * 2) % 16 == 0;
        if (patch_tc) {
            auto split = [&](const std::string& name) {
                auto w = t(name);
                const size_t n = size_t(w.ne1), k = size_t(w.ne0);
                const float* f = static_cast<const float*>(w.data);
                std::vector<uint16_t> out(n * 3 * k);
                for (size_t r = 0; r < n; ++r)
                    for (size_t c = 0; c < k; ++c) {
                        const float v = f[r * k + c];
                        const uint16_t hi = float_to_half_bits(v);
                        const uint16_t lo = float_to_half_bits(v - half_bits_to_float(hi));
                        out[r * 3 * k + c] = hi;
                        out[r * 3 * k + k + c] = lo;
                        out[r * 3 * k + 2 * k + c] = hi;
                    }
                return reinterpret_cast<__half*>(upload(out.data(), out.size()));
            };
            p_hid_split = split("patch.hidden.weight");
            p_res_split = split("patch.res.weight");
        }
        attn.resize(m.schedule.size());
        mlp.resize(m.schedule.size());
        for (size_t i = 0; i < m.schedule.size(); ++i) {
            const std::string b = "blk." + std::to_string(i) + ".";
            const int kind = m.schedule[i];
            std::vector<bool> axes = kind == 0 ? std::vector<bool>{true} : kind == 1 ? std::vector<bool>{false}
                                   : kind == 2 ? std::vector<bool>{true, false} : std::vector<bool>{false, true};
            for (size_t j = 0; j < axes.size(); ++j) {
                AttnW a;
                a.time = axes[j];
                a.gate = axes[j] ? m.time_gate : m.variate_gate;
                const std::string p = b + "attn." + std::to_string(j) + ".";
                a.norm = f32_tensor(b + "attn_norm." + std::to_string(j) + ".weight");
                std::vector<float> bq, bg;
                if (mv.has(p + "qkv.bias")) { auto w = t(p + "qkv.bias"); bq.assign(static_cast<const float*>(w.data), static_cast<const float*>(w.data) + 3 * D); }
                if (a.gate && mv.has(p + "gate.bias")) { auto w = t(p + "gate.bias"); bg.assign(static_cast<const float*>(w.data), static_cast<const float*>(w.data) + D); }
                if (tc) {
                    const float* nw = static_cast<const float*>(t(b + "attn_norm." + std::to_string(j) + ".weight").data);
                    auto q = rows_f16(t(p + "qkv.weight"));
                    fold_norm(q, size_t(D), nw);
                    std::vector<uint16_t> g;
                    if (a.gate) { g = rows_f16(t(p + "gate.weight")); fold_norm(g, size_t(D), nw); }
                    std::vector<uint16_t> cat(q);
                    cat.insert(cat.end(), g.begin(), g.end());
                    a.qkvg = reinterpret_cast<__half*>(upload(cat.data(), cat.size()));
                    a.n_qkvg = a.gate ? 4 * D : 3 * D;
                    if (!bq.empty() || !bg.empty()) {
                        std::vector<float> bc(size_t(a.n_qkvg), 0.f);
                        if (!bq.empty()) std::copy(bq.begin(), bq.end(), bc.begin());
                        if (!bg.empty()) std::copy(bg.begin(), bg.end(), bc.begin() + 3 * D);
                        a.b_qkvg = upload(bc.data(), bc.size());
                    }
                    if (!a.time && a.gate) {
                        auto vg = interleave(q.data() + size_t(2) * D * D, g.data(), size_t(D), size_t(D));
                        a.vg = reinterpret_cast<__half*>(upload(vg.data(), vg.size()));
                        if (!bq.empty() || !bg.empty()) {
                            auto bvg = interleave_bias(bq.empty() ? nullptr : bq.data() + 2 * D, bg.empty() ? nullptr : bg.data(), size_t(D));
                            a.b_vg = upload(bvg.data(), bvg.size());
                        }
                    }
                    auto o = rows_f16(t(p + "out.weight"));
                    a.out = reinterpret_cast<__half*>(upload(o.data(), o.size()));
                    // Block-quantised twins; the norm gain folded into q/k/v/gate must be a no-op for them.
                    if (block_type(t(p + "out.weight"))) a.out_blk = block_upload(block_rows(t(p + "out.weight")));
                    if (block_type(t(p + "qkv.weight")) && (!a.gate || block_type(t(p + "gate.weight"))) &&
                        unit_gains(nw, size_t(D))) {
                        BlockHost qk = block_rows(t(p + "qkv.weight"));
                        BlockHost gt;
                        if (a.gate) { gt = block_rows(t(p + "gate.weight")); block_append(qk, gt); }
                        a.qkvg_blk = block_upload(qk);
                        if (!a.time && a.gate)
                            a.vg_blk = block_upload(block_interleave(block_slice(qk, size_t(2) * D, size_t(D)), gt, size_t(D)));
                    }
                } else {
                    auto q = rows_f32(t(p + "qkv.weight"));
                    a.f_qkv = upload(q.data(), q.size());
                    if (!bq.empty()) a.fb_qkv = upload(bq.data(), bq.size());
                    if (a.gate) {
                        auto g = rows_f32(t(p + "gate.weight"));
                        a.f_gate = upload(g.data(), g.size());
                        if (!bg.empty()) a.fb_gate = upload(bg.data(), bg.size());
                    }
                    auto o = rows_f32(t(p + "out.weight"));
                    a.f_out = upload(o.data(), o.size());
                }
                a.b_out = bias_or_null(p + "out.bias");
                a.fb_out = a.b_out;
                attn[i].push_back(a);
            }
            MlpW w;
            w.norm = f32_tensor(b + "ffn_norm.weight");
            w.b3 = bias_or_null(b + "ffn_w3.bias");
            w.fb3 = w.b3;
            if (tc) {
                auto z = rows_f16(t(b + "ffn_w12.weight"));
                fold_norm(z, size_t(D), static_cast<const float*>(t(b + "ffn_norm.weight").data));
                auto zi = interleave(z.data(), z.data() + size_t(F) * D, size_t(F), size_t(D));
                w.w12 = reinterpret_cast<__half*>(upload(zi.data(), zi.size()));
                if (mv.has(b + "ffn_w12.bias")) {
                    const float* bb = static_cast<const float*>(t(b + "ffn_w12.bias").data);
                    auto bi = interleave_bias(bb, bb + F, size_t(F));
                    w.b12 = upload(bi.data(), bi.size());
                }
                auto w3 = rows_f16(t(b + "ffn_w3.weight"));
                w.w3 = reinterpret_cast<__half*>(upload(w3.data(), w3.size()));
                if (block_type(t(b + "ffn_w3.weight"))) w.w3_blk = block_upload(block_rows(t(b + "ffn_w3.weight")));
                if (block_type(t(b + "ffn_w12.weight")) &&
                    unit_gains(static_cast<const float*>(t(b + "ffn_norm.weight").data), size_t(D))) {
                    BlockHost z12 = block_rows(t(b + "ffn_w12.weight"));
                    w.w12_blk = block_upload(block_interleave(block_slice(z12, 0, size_t(F)), block_slice(z12, size_t(F), size_t(F)), size_t(F)));
                }
            } else {
                auto z = rows_f32(t(b + "ffn_w12.weight"));
                w.f12 = upload(z.data(), z.size());
                w.fb12 = bias_or_null(b + "ffn_w12.bias");
                auto w3 = rows_f32(t(b + "ffn_w3.weight"));
                w.f3 = upload(w3.data(), w3.size());
            }
            mlp[i] = w;
        }
        out_norm = f32_tensor("out_norm.weight");
        if (tc) {
            auto a = rows_f16(t("head.hidden.weight")); h_hid = reinterpret_cast<__half*>(upload(a.data(), a.size()));
            auto b = rows_f16(t("head.out.weight")); h_out = reinterpret_cast<__half*>(upload(b.data(), b.size()));
            auto c = rows_f16(t("head.res.weight")); h_res = reinterpret_cast<__half*>(upload(c.data(), c.size()));
            if (block_type(t("head.hidden.weight"))) h_hid_blk = block_upload(block_rows(t("head.hidden.weight")));
            if (block_type(t("head.out.weight"))) h_out_blk = block_upload(block_rows(t("head.out.weight")));
            if (block_type(t("head.res.weight"))) h_res_blk = block_upload(block_rows(t("head.res.weight")));
        } else {
            auto a = rows_f32(t("head.hidden.weight")); fh_hid = upload(a.data(), a.size());
            auto b = rows_f32(t("head.out.weight")); fh_out = upload(b.data(), b.size());
            auto c = rows_f32(t("head.res.weight")); fh_res = upload(c.data(), c.size());
        }
        err.ensure(sizeof(int));
        check(cudaMemset(err.p, 0, sizeof(int)), "memset");
        nflag.ensure(sizeof(int));
        check(cudaMemset(nflag.p, 0, sizeof(int)), "memset");
        if (tc) {
            std::vector<float> one(size_t(D), 1.0f);
            ones.ensure(size_t(D) * 4);
            check(cudaMemcpy(ones.p, one.data(), size_t(D) * 4, cudaMemcpyHostToDevice), "upload");
        }
    }

    bool fuse_allowed() const { return fuse && tc && D % 128 == 0; }
    // Reads and clears the flag of the forecast just run (synchronises the stream).
    bool take_norm_flag() {
        const int h = read_error(nflag.as<int>(), s);
        return h != 0 || force_fallback;
    }
    // The normalised input of the next consuming GEMM: x16 and the row sums of squares left by
    // the last residual-add epilogue, or the RMSNorm kernel (unit weights) into xn.
    void norm_input(bool have16, int64_t M) {
        a_map = RowMap{};
        if (fuse_now && have16) { a_in = x16.as<__half>(); ssq_in = ssq.as<float>(); return; }
        run("rms", [&] { return rms_norm(x.as<float>(), ones.as<float>(), int(M), D, mv.eps, xn.p, 1, 0, 0, 0, s); });
        a_in = xn.as<__half>();
        ssq_in = nullptr;
    }
    // The same for the decoder tokens alone (`tail` rows): the carried x16 read through the
    // row gather, or the RMSNorm kernel writing those tokens' normalised rows compactly.
    void norm_input_tail(bool have16) {
        if (fuse_now && have16) { a_in = x16.as<__half>(); ssq_in = ssq.as<float>(); a_map = tail; return; }
        run("rms", [&] {
            return rms_norm(x.as<float>(), ones.as<float>(), tail_rows, D, mv.eps, xn.p, 1, tail.group, tail.stride,
                            tail.offset, s);
        });
        a_in = xn.as<__half>();
        ssq_in = nullptr;
        a_map = RowMap{};
    }
    // A-operand rows of the next GEMM (see GemmArgs::a_group).
    void gather_a(GemmArgs& g) const { g.a_group = a_map.group; g.a_stride = a_map.stride; g.a_offset = a_map.offset; }
    // Output rows of a tail GEMM that writes the residual stream: the decoder tokens' rows.
    void scatter_out(GemmEpilogue& e) const { e.row_group = tail.group; e.row_stride = tail.stride; e.row_offset = tail.offset; }
    void consume(GemmEpilogue& e) const {
        e.ssq_in = ssq_in; e.ssq_slots = D / 128; e.rms_D = D; e.rms_eps = mv.eps; e.norm_flag = nflag.as<int>();
    }
    void produce(GemmEpilogue& e) const {
        if (!produce16) return;
        e.x16 = x16.as<__half>(); e.ldx16 = D; e.ssq = ssq.as<float>(); e.ssq_slots = D / 128;
        e.norm_flag = nflag.as<int>();
    }

    ~Impl() {
        for (auto p : allocs) cudaFree(p);
        for (auto& e : events) { cudaEventDestroy(e.a); cudaEventDestroy(e.b); }
    }

    // --- launch bookkeeping -------------------------------------------------------------
    template <class Fn> void run(const char* cls, Fn fn) {
        Ev* ev = nullptr;
        if (timing && (timing_only.empty() || timing_only == cls)) {
            if (ev_used == events.size()) {
                Ev e;
                check(cudaEventCreate(&e.a), "event");
                check(cudaEventCreate(&e.b), "event");
                events.push_back(e);
            }
            ev = &events[ev_used++];
            ev->cls = cls;
            cudaEventRecord(ev->a, s);
        }
        cudaError_t e = fn();
        if (e != cudaSuccess) throw std::runtime_error(std::string("launch ") + cls + ": " + cudaGetErrorString(e));
        if (ev) cudaEventRecord(ev->b, s);
        ++launches;
    }

    void gemm(EpiKind k, const GemmArgs& a, const char* cls = "gemm") {
        run(cls, [&] { return tc_gemm(k, a, s, err.as<int>()); });
    }
    void sgemm(SimtGemm g, const char* cls = "gemm_simt") {
        const size_t need = simt_panel_scratch_bytes(g);
        if (need) {
            panel_scratch.ensure(need);
            g.panel_scratch = panel_scratch.as<float>();
            g.panel_scratch_bytes = panel_scratch.bytes;
        }
        run(cls, [&] { return simt_gemm(g, s); });
    }

    // --- one decode block ---------------------------------------------------------------
    // Inputs: win/wmask [R2][W] (W = T on the context path, T + h*ps with covariates),
    // role [R2] (covariate path). Output: refined [R2][h*ps][Q]. first: compute cap stats.
    Engine::Geometry geo;
    void predict_block(int R2, int T, int h, bool cov, int group_rows, int pass_rows, bool first, int cap_ctx) {
        Range block_range("predict_block");
        const int W = cov ? T + h * ps : T;
        const int N = W / ps, L = T / ps;
        const int S = cov ? 2 * N : N + h;
        geo.rows = R2; geo.S = S; geo.L = L; geo.blocks = first ? 1 : geo.blocks + 1;
        const int P_all = cov ? N : h;
        const int kvw = (N + 31) / 32;
        const int64_t M = int64_t(R2) * S;
        if (M > INT32_MAX / 4) throw std::runtime_error("batch too large");
        const float* rows_p = win.as<float>();
        const int8_t* mask_p = wmask.as<int8_t>();
        feat.ensure(size_t(R2) * N * 2 * ps * 4);
        aloc.ensure(R2 * 4); ascale.ensure(R2 * 4); first_obs.ensure(R2 * 4);
        kv.ensure(size_t(R2) * kvw * 4);
        rope_row.ensure(size_t(M) * 4); gbeg.ensure(R2 * 4); gsize.ensure(R2 * 4);
        if (first) { caplo.ensure(R2 * 4); caphi.ensure(R2 * 4); capsc.ensure(R2 * 4); }
        auto embed_range = std::make_unique<Range>("scale_rows + patch embedding");
        run("scale", [&] {
            return scale_rows(rc, rows_p, mask_p, R2, W, cov ? (L - 1) * ps : T - 1, N, kvw, feat.as<float>(),
                              aloc.as<float>(), ascale.as<float>(), kv.as<uint32_t>(), first_obs.as<int>(),
                              first ? cap_ctx : 0, first ? caplo.as<float>() : nullptr,
                              first ? caphi.as<float>() : nullptr, first ? capsc.as<float>() : nullptr, s);
        });
        if (cov)
            run("scale", [&] {
                return known_rows(rc, rows_p, mask_p, role.as<int8_t>(), R2, W, (L - 1) * ps, feat.as<float>(),
                                  aloc.as<float>(), ascale.as<float>(), s);
            });
        run("positions", [&] {
            return positions(rc, first_obs.as<int>(), R2, group_rows, N, S, cov, rope_row.as<int>(), gbeg.as<int>(),
                             gsize.as<int>(), err.as<int>(), s);
        });
        // Patch projection (reference src/head.cpp:329-340) into token rows r*S + p, p < N.
        x.ensure(size_t(M) * D * 4);
        const int64_t PR = int64_t(R2) * N;
        ph.ensure(size_t(PR) * 4 * D * (tc ? 2 : 4));
        {
            SimtGemm g;
            g.A = feat.as<float>(); g.lda = 2 * ps; g.W = p_hid; g.M = int(PR); g.N = 4 * D; g.K = 2 * ps;
            g.order = ORDER_CHAIN; g.epi = tc ? SEPI_SILU_F16 : SEPI_SILU_F32; g.bias = pb_hid; g.out = ph.p; g.ldo = 4 * D;
            SimtGemm r;
            r.A = feat.as<float>(); r.lda = 2 * ps; r.W = p_res; r.M = int(PR); r.N = D; r.K = 2 * ps;
            r.order = ORDER_CHAIN; r.epi = SEPI_F32; r.bias = pb_res; r.out = x.p; r.ldo = D;
            r.row_group = N; r.row_stride = S;
            if (patch_tc) {
                // Tensor cores on the f16 hi/lo split of the features; rows with a feature
                // outside the split's range are recomputed by the CUDA-core kernels.
                const int K3 = 3 * 2 * ps;
                feat16.ensure(size_t(PR) * K3 * 2);
                pflag.ensure(sizeof(int) + size_t(PR));
                check(cudaMemsetAsync(pflag.p, 0, sizeof(int) + size_t(PR), s), "memset");
                int8_t* row_flags = pflag.as<int8_t>() + sizeof(int);
                run("patch_split", [&] {
                    return split_f16(feat.as<float>(), PR, 2 * ps, feat16.as<__half>(), pflag.as<int>(), row_flags, s);
                });
                GemmArgs h;
                h.A = feat16.as<__half>(); h.lda = K3; h.B = p_hid_split; h.ldb = K3; h.M = int(PR); h.N = 4 * D; h.K = K3;
                h.epi.out = ph.p; h.epi.ldo = 4 * D; h.epi.bias = pb_hid;
                gemm(EPI_SILU, h);
                GemmArgs o;
                o.A = feat16.as<__half>(); o.lda = K3; o.B = p_res_split; o.ldb = K3; o.M = int(PR); o.N = D; o.K = K3;
                o.epi.out = x.p; o.epi.ldo = D; o.epi.bias = pb_res; o.epi.row_group = N; o.epi.row_stride = S;
                gemm(EPI_F32, o);
                // Only the rows with such a feature are rewritten, so every row's result is
                // the same whatever else is in the batch.
                g.only_if = pflag.as<int>(); g.row_mask = row_flags;
                r.only_if = pflag.as<int>(); r.row_mask = row_flags;
            }
            sgemm(g);
            sgemm(r);
        }
        if (tc) {
            GemmArgs a;
            a.A = ph.as<__half>(); a.lda = 4 * D; a.B = p_out; a.ldb = 4 * D; a.M = int(PR); a.N = D; a.K = 4 * D;
            a.epi.out = x.p; a.epi.ldo = D; a.epi.bias = pb_out; a.epi.resid = x.as<float>();
            a.epi.row_group = N; a.epi.row_stride = S;
            block_b(a, p_out_blk);
            gemm(EPI_RESID, a);
        } else {
            SimtGemm g;
            g.A = ph.as<float>(); g.lda = 4 * D; g.W = f_pout; g.M = int(PR); g.N = D; g.K = 4 * D;
            g.order = ORDER_PANEL192; g.round_a_f16 = round_a; g.epi = SEPI_RESID; g.bias = pb_out; g.out = x.p; g.ldo = D;
            g.row_group = N; g.row_stride = S;
            sgemm(g);
        }
        run("fill", [&] { return fill_query(query, x.as<float>(), R2, S, N, D, s); });

        MaskMeta mm;
        mm.key_valid = kv.as<uint32_t>(); mm.kv_words = kvw; mm.N = N; mm.L = L; mm.S = S; mm.cov = cov;
        mm.block_size = mv.block_size; mm.role = cov ? role.as<int8_t>() : nullptr;
        mm.group_begin = gbeg.as<int>(); mm.group_size = gsize.as<int>(); mm.pass_rows = pass_rows;

        const size_t eb = tc ? 2 : 4;
        xn.ensure(size_t(M) * D * eb);
        qb.ensure(size_t(M) * D * eb); kb.ensure(size_t(M) * D * eb); vb.ensure(size_t(M) * D * eb);
        gb.ensure(size_t(M) * D * eb); att.ensure(size_t(M) * D * eb);
        hb.ensure(size_t(M) * F * eb);
        if (!tc) { fused.ensure(size_t(M) * 3 * D * 4); gtmp.ensure(size_t(M) * D * 4); zb.ensure(size_t(M) * 2 * F * 4); }

        if (tc && fuse_now) { x16.ensure(size_t(M) * D * 2); ssq.ensure(size_t(M) * (D / 128) * 4); }
        bool have16 = false;   // x16 and ssq hold the current x
        embed_range.reset();
        // The decoder-token tail applies when the last layer starts with a time sublayer and
        // the rest of it is per token (one-row series on the variate axis), on the context
        // path with h dividing the GEMM's 128-row box.
        const size_t last = attn.size() - 1;
        bool tail_ok = tc && tail_enabled && !cov && group_rows == 1 && h > 0 && 128 % h == 0 && !attn[last].empty() &&
                       attn[last][0].time;
        for (size_t j = 1; tail_ok && j < attn[last].size(); ++j) tail_ok = !attn[last][j].time;
        tail = RowMap{h, S, N};
        tail_rows = R2 * h;
        for (size_t li = 0; li < attn.size(); ++li) {
            Range layer_range("layer %d", int(li));
            const bool in_tail = tail_ok && li == last;
            for (size_t j = 0; j < attn[li].size(); ++j) {
                const AttnW& a = attn[li][j];
                if (tc) {
                    if (in_tail && j > 0) norm_input_tail(have16);
                    else norm_input(have16, M);
                    produce16 = fuse_now;
                    attention_sublayer_tc(a, int(M), R2, S, group_rows, mm, in_tail ? (j == 0 ? 1 : 2) : 0);
                    have16 = fuse_now;
                } else {
                    run("rms", [&] { return rms_norm(x.as<float>(), a.norm, int(M), D, mv.eps, xn.p, 0, 0, 0, 0, s); });
                    attention_sublayer_simt(a, int(M), R2, S, mm);
                }
            }
            const MlpW& w = mlp[li];
            if (tc) {
                const bool in_tail = tail_ok && li == last;
                const int Mm = in_tail ? tail_rows : int(M);
                if (in_tail) norm_input_tail(have16);
                else norm_input(have16, M);
                produce16 = fuse_now;
                GemmArgs a;
                a.A = a_in; a.lda = D; a.B = w.w12; a.ldb = D; a.M = Mm; a.N = 2 * F; a.K = D;
                a.epi.out = hb.p; a.epi.ldo = F; a.epi.bias = w.b12;
                block_b(a, w.w12_blk);
                gather_a(a);
                consume(a.epi);
                gemm(EPI_SWIGLU, a);
                GemmArgs o;
                o.A = hb.as<__half>(); o.lda = F; o.B = w.w3; o.ldb = F; o.M = Mm; o.N = D; o.K = F;
                o.epi.out = x.p; o.epi.ldo = D; o.epi.bias = w.b3; o.epi.resid = x.as<float>();
                block_b(o, w.w3_blk);
                if (in_tail) scatter_out(o.epi);
                produce(o.epi);
                gemm(EPI_RESID, o);
                have16 = fuse_now;
            } else {
                run("rms", [&] { return rms_norm(x.as<float>(), w.norm, int(M), D, mv.eps, xn.p, 0, 0, 0, 0, s); });
                SimtGemm g;
                g.A = xn.as<float>(); g.lda = D; g.W = w.f12; g.M = int(M); g.N = 2 * F; g.K = D;
                g.order = round_a ? ORDER_CHAIN : ORDER_PANEL192; g.round_a_f16 = round_a; g.epi = SEPI_F32;
                g.bias = w.fb12; g.out = zb.p; g.ldo = 2 * F;
                sgemm(g);
                run("swiglu", [&] { return swiglu(zb.as<float>(), int(M), F, hb.as<float>(), s); });
                SimtGemm o;
                o.A = hb.as<float>(); o.lda = F; o.W = w.f3; o.M = int(M); o.N = D; o.K = F;
                o.order = round_a ? ORDER_CHAIN : ORDER_PANEL192; o.round_a_f16 = round_a; o.epi = SEPI_RESID;
                o.bias = w.fb3; o.out = x.p; o.ldo = D;
                sgemm(o);
            }
        }
        // out_norm on the decoder tokens only (per-token op; reference src/encoder.cpp:146 +
        // src/predict_block.cpp:15-16 slice).
        Range head_range("out_norm + quantile head + refine");
        const int DR = R2 * P_all;
        dec.ensure(size_t(DR) * D * eb);
        run("rms", [&] { return rms_norm(x.as<float>(), out_norm, DR, D, mv.eps, dec.p, tc, P_all, S, N, s); });
        const int NQ = ps * Q;
        hh.ensure(size_t(DR) * 4 * D * eb);
        hraw.ensure(size_t(DR) * NQ * 4);
        if (tc) {
            GemmArgs a;
            a.A = dec.as<__half>(); a.lda = D; a.B = h_hid; a.ldb = D; a.M = DR; a.N = 4 * D; a.K = D;
            a.epi.out = hh.p; a.epi.ldo = 4 * D;
            block_b(a, h_hid_blk);
            gemm(EPI_SILU, a);
            GemmArgs b;
            b.A = hh.as<__half>(); b.lda = 4 * D; b.B = h_out; b.ldb = 4 * D; b.M = DR; b.N = NQ; b.K = 4 * D;
            b.epi.out = hraw.p; b.epi.ldo = NQ;
            block_b(b, h_out_blk);
            gemm(EPI_F32, b);
            GemmArgs c;
            c.A = dec.as<__half>(); c.lda = D; c.B = h_res; c.ldb = D; c.M = DR; c.N = NQ; c.K = D;
            c.epi.out = hraw.p; c.epi.ldo = NQ; c.epi.resid = hraw.as<float>();
            block_b(c, h_res_blk);
            gemm(EPI_RESID, c);
        } else {
            const int order = round_a ? ORDER_CHAIN : ORDER_F64;
            SimtGemm a;
            a.A = dec.as<float>(); a.lda = D; a.W = fh_hid; a.M = DR; a.N = 4 * D; a.K = D; a.order = order;
            a.round_a_f16 = round_a; a.epi = SEPI_SILU_F32; a.out = hh.p; a.ldo = 4 * D;
            sgemm(a);
            SimtGemm b;
            b.A = hh.as<float>(); b.lda = 4 * D; b.W = fh_out; b.M = DR; b.N = NQ; b.K = 4 * D; b.order = order;
            b.round_a_f16 = round_a; b.epi = SEPI_F32; b.out = hraw.p; b.ldo = NQ;
            sgemm(b);
            SimtGemm c;
            c.A = dec.as<float>(); c.lda = D; c.W = fh_res; c.M = DR; c.N = NQ; c.K = D; c.order = order;
            c.round_a_f16 = round_a; c.epi = SEPI_RESID; c.out = hraw.p; c.ldo = NQ;
            sgemm(c);
        }
        const int steps = h * ps;
        qout.ensure(size_t(R2) * steps * Q * 4);
        run("head", [&] {
            return quantile_head(rc, hraw.as<float>(), R2, P_all, cov ? L : 0, h, aloc.as<float>(), ascale.as<float>(),
                                 qout.as<float>(), nullptr, err.as<int>(), s);
        });
        refined.ensure(size_t(R2) * steps * Q * 4);
        if (h > 1) {
            const int n = T / ps + h;
            scratch.ensure(size_t(R2) * (3 * size_t(n) + 2 * ps + 2 * h) * 8);
            const double clip = std::pow(double(FLT_MAX), 0.5) / 1e3;
            run("refine", [&] {
                return refine(rc, qout.as<float>(), rows_p, mask_p, W, cov ? role.as<int8_t>() : nullptr, aloc.as<float>(),
                              ascale.as<float>(), R2, T, h, clip, scratch.as<double>(), refined.as<float>(), s);
            });
        } else {
            check(cudaMemcpyAsync(refined.p, qout.p, size_t(R2) * steps * Q * 4, cudaMemcpyDeviceToDevice, s), "copy");
        }
    }

    // tail_stage: 0 every token; 1 the last layer's time sublayer, whose out projection runs on
    // the decoder tokens alone; 2 a later one-row variate sublayer of that layer, wholly on them.
    void attention_sublayer_tc(const AttnW& a, int M, int R2, int S, int group_rows, const MaskMeta& mm, int tail_stage) {
        __half* att16 = att.as<__half>();
        GemmArgs o;                                  // the out projection (input: att16 rows)
        o.M = M;
        if (tail_stage == 2) {
            if (a.time || group_rows != 1) throw std::runtime_error("decoder tail: unexpected sublayer");
            M = tail_rows;
            o.M = tail_rows;                         // att16 holds the tail rows compactly
        } else if (tail_stage == 1) {
            o.M = tail_rows;                         // att16 holds every token: gather the tail rows
            o.a_group = tail.group; o.a_stride = tail.stride; o.a_offset = tail.offset;
        }
        if (!a.time && group_rows == 1) {
            // One row per series: attention over a single key returns v exactly
            // (reference tests/layer_kind_test.hpp:31-33), so the sublayer is
            // out(v * sigmoid(gate)) and only the v and gate projections are computed.
            GemmArgs g;
            g.A = a_in; g.lda = D; g.M = M; g.K = D; g.epi.out = att16; g.epi.ldo = D;
            if (tail_stage == 2) gather_a(g);
            consume(g.epi);
            if (a.gate) { g.B = a.vg; g.ldb = D; g.N = 2 * D; g.epi.bias = a.b_vg; block_b(g, a.vg_blk); gemm(EPI_VGATE, g); }
            else {
                g.B = a.qkvg + size_t(2) * D * D; g.ldb = D; g.N = D;
                g.epi.bias = a.b_qkvg ? a.b_qkvg + 2 * D : nullptr;
                block_b(g, a.qkvg_blk, int64_t(2) * D);
                gemm(EPI_F16, g);
            }
        } else {
            GemmArgs g;
            g.A = a_in; g.lda = D; g.B = a.qkvg; g.ldb = D; g.M = M; g.N = a.n_qkvg; g.K = D;
            g.epi.bias = a.b_qkvg;
            block_b(g, a.qkvg_blk);
            consume(g.epi);
            g.epi.qkvg[0] = qb.as<__half>(); g.epi.qkvg[1] = kb.as<__half>(); g.epi.qkvg[2] = vb.as<__half>();
            g.epi.qkvg[3] = gb.as<__half>();
            g.epi.S = S; g.epi.H = H; g.epi.D = D; g.epi.rope = a.time;
            g.epi.cos_tab = cos_tab; g.epi.sin_tab = sin_tab; g.epi.rope_row = rope_row.as<int>(); g.epi.rope_half = rope_half;
            g.epi.rope_dup = rope_dup;
            gemm(EPI_QKVG, g);
            const __half* gate = a.gate ? gb.as<__half>() : nullptr;
            if (attn_simt && a.time && S <= kSimtMaxKeys) {
                run("attention", [&] { return attention_time_simt<__half>(qb.as<__half>(), kb.as<__half>(), vb.as<__half>(), gate, att16, R2, H, hd, mm, s); });
            } else if (attn_simt && !a.time) {
                run("attention_variate", [&] { return attention_variate_simt<__half>(qb.as<__half>(), kb.as<__half>(), vb.as<__half>(), gate, att16, R2, H, hd, mm, s); });
            } else if (a.time) {
                if (S <= 128)
                    run("attention", [&] { return attention_time_tc(qb.as<__half>(), kb.as<__half>(), vb.as<__half>(), gate, att16, R2, H, mm, s, err.as<int>()); });
                else
                    run("attention", [&] { return attention_time_tc_long(qb.as<__half>(), kb.as<__half>(), vb.as<__half>(), gate, att16, R2, H, mm, s, err.as<int>()); });
            } else {
                if (group_rows <= 32)
                    run("attention_variate", [&] { return attention_variate_tc(qb.as<__half>(), kb.as<__half>(), vb.as<__half>(), gate, att16, R2, H, group_rows, mm, s, err.as<int>()); });
                else if (group_rows <= 64)
                    run("attention_variate", [&] { return attention_variate_fast(qb.as<__half>(), kb.as<__half>(), vb.as<__half>(), gate, att16, R2, H, group_rows, mm, s); });
                else
                    run("attention_variate", [&] { return attention_variate_simt<__half>(qb.as<__half>(), kb.as<__half>(), vb.as<__half>(), gate, att16, R2, H, hd, mm, s); });
            }
        }
        o.A = att16; o.lda = D; o.B = a.out; o.ldb = D; o.N = D; o.K = D;
        o.epi.out = x.p; o.epi.ldo = D; o.epi.bias = a.b_out; o.epi.resid = x.as<float>();
        block_b(o, a.out_blk);
        if (tail_stage) scatter_out(o.epi);
        produce(o.epi);
        gemm(EPI_RESID, o);
    }

    void attention_sublayer_simt(const AttnW& a, int M, int R2, int S, const MaskMeta& mm) {
        const int order = round_a ? ORDER_CHAIN : ORDER_PANEL192;
        SimtGemm g;
        g.A = xn.as<float>(); g.lda = D; g.W = a.f_qkv; g.M = M; g.N = 3 * D; g.K = D; g.order = order;
        g.round_a_f16 = round_a; g.epi = SEPI_F32; g.bias = a.fb_qkv; g.out = fused.p; g.ldo = 3 * D;
        sgemm(g);
        if (a.gate) {
            SimtGemm q;
            q.A = xn.as<float>(); q.lda = D; q.W = a.f_gate; q.M = M; q.N = D; q.K = D; q.order = order;
            q.round_a_f16 = round_a; q.epi = SEPI_F32; q.bias = a.fb_gate; q.out = gtmp.p; q.ldo = D;
            sgemm(q);
        }
        run("scatter", [&] {
            return qkv_scatter(fused.as<float>(), a.gate ? gtmp.as<float>() : nullptr, M, S, H, hd, a.time, cos_tab,
                               sin_tab, rope_row.as<int>(), qb.as<float>(), kb.as<float>(), vb.as<float>(),
                               a.gate ? gb.as<float>() : nullptr, s);
        });
        const float* gate = a.gate ? gb.as<float>() : nullptr;
        if (a.time)
            run("attention", [&] { return attention_time_simt<float>(qb.as<float>(), kb.as<float>(), vb.as<float>(), gate, att.as<float>(), R2, H, hd, mm, s); });
        else
            run("attention_variate", [&] { return attention_variate_simt<float>(qb.as<float>(), kb.as<float>(), vb.as<float>(), gate, att.as<float>(), R2, H, hd, mm, s); });
        SimtGemm o;
        o.A = att.as<float>(); o.lda = D; o.W = a.f_out; o.M = M; o.N = D; o.K = D; o.order = order;
        o.round_a_f16 = round_a; o.epi = SEPI_RESID; o.bias = a.fb_out; o.out = x.p; o.ldo = D;
        sgemm(o);
    }

    void check_device_error(const char* where) {
        const int e = read_error(err.as<int>(), s);
        if (!e) return;
        if (e == kDevBadShape) throw std::runtime_error("NaN raw quantile or position outside the stored RoPE table");
        if (e == kDevNaN) throw std::runtime_error("forecast produced NaN values; the input is degenerate");
        if (e == kDevNonFinite) throw std::runtime_error("C ABI nonfinite forecast output");
        throw std::runtime_error(std::string(where) + ": device wait expired (error word " + std::to_string(e) + ")");
    }
};

Engine::Engine(const ModelView& mv, int device) : impl_(new Impl), device_(device) {
    check(cudaSetDevice(device), "cudaSetDevice");
    check(cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking), "stream");
    impl_->s = stream_;
    impl_->mv = mv;
    impl_->load();
    tc_ = impl_->tc;
}

Engine::~Engine() {
    cudaSetDevice(device_);
    if (stream_) cudaStreamSynchronize(stream_);
    if (impl_) impl_->drop_graph();
    impl_.reset();
    if (stream_) cudaStreamDestroy(stream_);
}

void Engine::check_errors() {
    check(cudaSetDevice(device_), "cudaSetDevice");
    check(cudaStreamSynchronize(stream_), "forecast");
    finish_targets();
}

void Engine::timing_enable(bool on, const char* only) {
    impl_->timing = on;
    impl_->timing_only = only ? only : "";
}
void Engine::timing_reset() { impl_->ev_used = 0; }
Engine::Geometry Engine::last_geometry() const { return impl_->geo; }
bool Engine::timing_read(const std::string& cls, double* ms, int64_t* launches) {
    cudaStreamSynchronize(stream_);
    double total = 0;
    int64_t n = 0;
    for (size_t i = 0; i < impl_->ev_used; ++i) {
        const auto& e = impl_->events[i];
        if (cls != "all" && e.cls != cls) continue;
        float t = 0;
        if (cudaEventElapsedTime(&t, e.a, e.b) == cudaSuccess) { total += t; ++n; }
    }
    *ms = total;
    *launches = n;
    return true;
}

void Engine::forecast_targets(const float* d_ctx, const uint8_t* d_umask, int B, int V, int T, int H, bool symmetric,
                              bool clip, int max_context, float* d_out, bool sync) {
    Range range("tsb forecast");
    check(cudaSetDevice(device_), "cudaSetDevice");
    Impl& im = *impl_;
    im.launches = 0;
    const ModelView& mv = im.mv;
    const int ps = im.ps;
    if (B <= 0 || V <= 0 || T <= 0 || H <= 0) throw std::runtime_error("invalid forecast dimensions");
    const int cap = max_context ? max_context : mv.context_length;
    if (cap > mv.context_length) throw std::runtime_error("max_context exceeds stored position range");
    const int kept = std::min(T, cap), pad = (ps - kept % ps) % ps, len = kept + pad;
    const int patches = (H + ps - 1) / ps;
    const int shot = im.shot();
    const int R = B * V, R2 = symmetric ? 2 * R : R;
    const cudaStream_t s = stream_;
    const bool single = patches <= shot;
    Impl::GraphKey key;
    key.ctx = d_ctx; key.umask = d_umask; key.out = d_out;
    key.B = B; key.V = V; key.T = T; key.H = H; key.max_context = max_context; key.sym = symmetric; key.clip = clip;
    key.shot = shot; key.cap_k = im.cap_k();
    const bool graphable = im.graphs && single && !im.timing && !im.observer;
    // An earlier asynchronous forecast that carried the norm in the GEMMs is completed and
    // checked (and run again if flagged) before this one shares the flag.
    if (im.pending.valid && im.fuse_now) {
        check(cudaStreamSynchronize(s), "forecast");
        finish_targets();
        im.launches = 0;
    }
    im.fuse_now = im.fuse_allowed();
    im.pending = Impl::Pending{true, d_ctx, d_umask, B, V, T, H, symmetric, clip, d_out, kept, len, patches, shot, R, R2, cap};
    if (graphable && im.graph_exec && key == im.graph_key && im.graph_generation == g_workspace_generation.load()) {
        check(cudaGraphLaunch(im.graph_exec, s), "graph launch");
        im.launches = im.graph_launches;
        last_launches_ = im.launches;
        if (sync) finish_targets();
        return;
    }
    const bool capture = graphable && im.have_last && key == im.last_key;
    im.last_key = key;
    im.have_last = true;
    if (capture) {
        im.drop_graph();
        check(cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal), "begin capture");
    }
    try {
        targets_body(d_ctx, d_umask, B, V, T, H, symmetric, clip, d_out, kept, len, patches, shot, R, R2, cap);
    } catch (...) {
        if (capture) {
            cudaGraph_t g = nullptr;
            cudaStreamEndCapture(s, &g);
            if (g) cudaGraphDestroy(g);
            cudaGetLastError();
        }
        // The next identical call runs uncaptured: a failed call may have left workspace to
        // allocate, which a capture cannot do.
        im.have_last = false;
        throw;
    }
    if (capture) {
        cudaGraph_t g = nullptr;
        check(cudaStreamEndCapture(s, &g), "end capture");
        const cudaError_t e = cudaGraphInstantiate(&im.graph_exec, g, 0);
        cudaGraphDestroy(g);
        check(e, "graph instantiate");
        im.graph_key = key;
        im.graph_generation = g_workspace_generation.load();
        im.graph_launches = im.launches;
        check(cudaGraphLaunch(im.graph_exec, s), "graph launch");
    }
    last_launches_ = im.launches;
    if (sync) finish_targets();
}

// Errors of the last forecast without covariates; when the norm carried by the GEMMs flagged a
// row (an f16 overflow of the residual copy, or a row too small for it), the forecast is run
// again with the RMSNorm kernel, into the same output.
void Engine::finish_targets() {
    Impl& im = *impl_;
    im.check_device_error("forecast");
    if (!im.pending.valid || !im.fuse_now) return;
    im.pending.valid = false;
    if (!im.take_norm_flag()) return;
    const Impl::Pending p = im.pending;
    im.fuse_now = false;
    try {
        targets_body(static_cast<const float*>(p.ctx), static_cast<const uint8_t*>(p.umask), p.B, p.V, p.T, p.H, p.sym,
                     p.clip, static_cast<float*>(p.out), p.kept, p.len, p.patches, p.shot, p.R, p.R2, p.cap);
    } catch (...) {
        im.fuse_now = true;
        throw;
    }
    im.fuse_now = true;
    im.check_device_error("forecast");
}

void Engine::targets_body(const float* d_ctx, const uint8_t* d_umask, int B, int V, int T, int H, bool symmetric,
                          bool clip, float* d_out, int kept, int len, int patches, int shot, int R, int R2, int cap) {
    Impl& im = *impl_;
    const ModelView& mv = im.mv;
    const int ps = im.ps, Q = im.Q;
    const cudaStream_t s = stream_;
    if (clip) {
        im.clip_ok.ensure(size_t(R));
        im.run("clip", [&] { return clip_eligibility(d_ctx, d_umask, R, T, im.clip_ok.as<int8_t>(), s); });
    }
    im.win.ensure(size_t(R2) * len * 4);
    im.wmask.ensure(size_t(R2) * len);
    im.run("assemble", [&] { return assemble_targets(d_ctx, d_umask, R, T, kept, len, symmetric, im.win.as<float>(), im.wmask.as<int8_t>(), s); });
    int Tc = len, done = 0;
    const bool single = patches <= shot;
    if (!single) im.decoded.ensure(size_t(R2) * H * Q * 4);
    (void)T;
    while (done < patches) {
        const int block = std::min(shot, patches - done), n = block * ps, offset = done * ps;
        if (im.observer && im.observer->before) im.observer->before(offset, block, Tc);
        // The V target rows of one series form one group (reference src/covariates.cpp:63).
        im.predict_block(R2, Tc, block, false, V, R, done == 0, len);
        im.observe(offset, block, Tc, R2, Tc, nullptr, nullptr, 0);
        if (single) break;
        const int used = std::min(n, H - offset);
        check(cudaMemcpy2DAsync(im.decoded.as<float>() + size_t(offset) * Q, size_t(H) * Q * 4, im.refined.p,
                                size_t(n) * Q * 4, size_t(used) * Q * 4, R2, cudaMemcpyDeviceToDevice, s), "copy");
        done += block;
        if (done >= patches) break;
        // Slide to the request's context cap, whole patches (reference src/forecaster.cpp decode_impl).
        const int joined = Tc + n, keep = joined > cap ? std::max(ps, (cap / ps) * ps) : joined;
        im.next_rows.ensure(size_t(R2) * keep * 4);
        im.next_mask.ensure(size_t(R2) * keep);
        im.run("feedback", [&] {
            return feedback(im.rc, im.win.as<float>(), im.wmask.as<int8_t>(), R2, Tc, im.refined.as<float>(), n, nullptr,
                            nullptr, nullptr, keep, im.next_rows.as<float>(), im.next_mask.as<int8_t>(), s);
        });
        std::swap(im.win.p, im.next_rows.p); std::swap(im.win.bytes, im.next_rows.bytes);
        std::swap(im.wmask.p, im.next_mask.p); std::swap(im.wmask.bytes, im.next_mask.bytes);
        Tc = keep;
    }
    const float* dec = single ? im.refined.as<float>() : im.decoded.as<float>();
    const int Hfull = single ? patches * ps : H;
    im.run("finalize", [&] {
        RowConfig rc = im.rc;
        rc.cap_k = im.cap_k();
        return finalize(rc, dec, R, symmetric, B, V, V, H, Hfull, im.caplo.as<float>(), im.caphi.as<float>(),
                        im.capsc.as<float>(), rc.cap_k > 0, clip ? im.clip_ok.as<int8_t>() : nullptr, d_out,
                        im.err.as<int>(), s);
    });
}

void Engine::fused_norm(int mode) {
    impl_->fuse = mode != 0;
    impl_->force_fallback = mode == 2;
    impl_->drop_graph();
    impl_->have_last = false;
}

void Engine::attention_kernels(int mode) {
    impl_->attn_simt = mode == 1;
    impl_->drop_graph();
    impl_->have_last = false;
}

bool Engine::dequant_prologue(bool on) {
    const bool any = impl_->p_out_blk.q || impl_->h_hid_blk.q || (!impl_->mlp.empty() && impl_->mlp[0].w3_blk.q);
    impl_->dq_prologue = on && any;
    impl_->drop_graph();
    impl_->have_last = false;
    return impl_->dq_prologue == on;
}

void Engine::decoder_tail(bool on) {
    impl_->tail_enabled = on;
    impl_->drop_graph();
    impl_->have_last = false;
}

void Engine::set_observer(const BlockObserver* observer) {
    impl_->observer = observer;
    if (observer) impl_->have_last = false;
}

void Engine::set_overrides(int per_shot, double cap_k) {
    impl_->shot_override = per_shot > 0 ? per_shot : 0;
    impl_->cap_override = cap_k;
}

void Engine::graph_replay(bool on) {
    impl_->graphs = on;
    if (!on) { impl_->drop_graph(); impl_->have_last = false; }
}

void Engine::decode_host_rows(const HostRows& a, int H, float* h_decoded) {
    Range range("tsb decode");
    check(cudaSetDevice(device_), "cudaSetDevice");
    Impl& im = *impl_;
    if (im.pending.valid && im.fuse_now) {       // an earlier asynchronous forecast: complete it
        check(cudaStreamSynchronize(stream_), "forecast");
        finish_targets();
    }
    im.launches = 0;
    im.pending.valid = false;
    im.fuse_now = im.fuse_allowed();
    const ModelView& mv = im.mv;
    const int R = a.R, T = a.T;
    const bool cov = a.roles != nullptr && mv.covariate_enabled;
    const cudaStream_t s = stream_;
    if (cov) {
        std::vector<int8_t> role(R);
        for (int r = 0; r < R; ++r) role[r] = int8_t(a.roles[r]);
        im.role.ensure(R);
        check(cudaMemcpyAsync(im.role.p, role.data(), R, cudaMemcpyHostToDevice, s), "upload roles");
        check(cudaStreamSynchronize(s), "sync");
    }
    if (a.future) {
        im.future.ensure(size_t(R) * a.Hh * 4); im.fmask.ensure(size_t(R) * a.Hh);
        check(cudaMemcpyAsync(im.future.p, a.future, size_t(R) * a.Hh * 4, cudaMemcpyHostToDevice, s), "upload");
        check(cudaMemcpyAsync(im.fmask.p, a.future_mask, size_t(R) * a.Hh, cudaMemcpyHostToDevice, s), "upload");
    }
    im.rows.ensure(size_t(R) * T * 4); im.mask.ensure(size_t(R) * T);
    check(cudaMemcpyAsync(im.rows.p, a.rows, size_t(R) * T * 4, cudaMemcpyHostToDevice, s), "upload");
    check(cudaMemcpyAsync(im.mask.p, a.mask, size_t(R) * T, cudaMemcpyHostToDevice, s), "upload");
    decode_rows(0, 0, H, R, T, a.Hh, false, false, cov, a.future != nullptr, a.group_rows,
                a.cap ? a.cap : mv.context_length, nullptr, h_decoded);
    if (im.fuse_now && im.take_norm_flag()) {
        const bool saved = im.fuse;
        im.fuse = false;
        try { decode_host_rows(a, H, h_decoded); } catch (...) { im.fuse = saved; throw; }
        im.fuse = saved;
    }
}

void Engine::forecast_rows(const HostRows& a, int B, int V, int H, bool symmetric, bool clip, const float* ctx,
                           const uint8_t* umask, int T_req, float* h_out) {
    Range range("tsb forecast (host rows)");
    check(cudaSetDevice(device_), "cudaSetDevice");
    Impl& im = *impl_;
    if (im.pending.valid && im.fuse_now) {       // an earlier asynchronous forecast: complete it
        check(cudaStreamSynchronize(stream_), "forecast");
        finish_targets();
    }
    im.launches = 0;
    im.pending.valid = false;
    im.fuse_now = im.fuse_allowed();
    const ModelView& mv = im.mv;
    const int R = a.R, T = a.T, R2 = symmetric ? 2 * R : R;
    const bool cov = a.roles != nullptr && mv.covariate_enabled;
    const cudaStream_t s = stream_;
    // Upload context rows (+ negation), roles, known future (+ negation).
    std::vector<float> rows2(size_t(R2) * T);
    std::vector<int8_t> mask2(size_t(R2) * T);
    for (size_t i = 0; i < size_t(R) * T; ++i) {
        rows2[i] = a.rows[i]; mask2[i] = a.mask[i];
        if (symmetric) { rows2[size_t(R) * T + i] = -a.rows[i]; mask2[size_t(R) * T + i] = a.mask[i]; }
    }
    std::vector<int8_t> role2;
    if (cov) {
        role2.resize(R2);
        for (int r = 0; r < R2; ++r) role2[r] = int8_t(a.roles[r % R]);
        im.role.ensure(R2);
        check(cudaMemcpyAsync(im.role.p, role2.data(), R2, cudaMemcpyHostToDevice, s), "upload roles");
    }
    const int Hh = a.Hh;
    std::vector<float> fut2;
    std::vector<int8_t> fm2;
    if (a.future) {
        fut2.resize(size_t(R2) * Hh);
        fm2.resize(size_t(R2) * Hh);
        for (size_t i = 0; i < size_t(R) * Hh; ++i) {
            fut2[i] = a.future[i]; fm2[i] = a.future_mask[i];
            if (symmetric) { fut2[size_t(R) * Hh + i] = -a.future[i]; fm2[size_t(R) * Hh + i] = a.future_mask[i]; }
        }
        im.future.ensure(fut2.size() * 4); im.fmask.ensure(fm2.size());
        check(cudaMemcpyAsync(im.future.p, fut2.data(), fut2.size() * 4, cudaMemcpyHostToDevice, s), "upload");
        check(cudaMemcpyAsync(im.fmask.p, fm2.data(), fm2.size(), cudaMemcpyHostToDevice, s), "upload");
    }
    im.rows.ensure(rows2.size() * 4); im.mask.ensure(mask2.size());
    check(cudaMemcpyAsync(im.rows.p, rows2.data(), rows2.size() * 4, cudaMemcpyHostToDevice, s), "upload");
    check(cudaMemcpyAsync(im.mask.p, mask2.data(), mask2.size(), cudaMemcpyHostToDevice, s), "upload");
    // clip eligibility from the request context
    if (clip) {
        DevBuf& dctx = im.req_ctx;
        DevBuf& dum = im.req_umask;
        dctx.ensure(size_t(B) * V * T_req * 4);
        check(cudaMemcpyAsync(dctx.p, ctx, size_t(B) * V * T_req * 4, cudaMemcpyHostToDevice, s), "upload");
        if (umask) { dum.ensure(size_t(B) * V * T_req); check(cudaMemcpyAsync(dum.p, umask, size_t(B) * V * T_req, cudaMemcpyHostToDevice, s), "upload"); }
        im.clip_ok.ensure(size_t(B) * V);
        im.run("clip", [&] { return clip_eligibility(dctx.as<float>(), umask ? dum.as<uint8_t>() : nullptr, B * V, T_req, im.clip_ok.as<int8_t>(), s); });
        check(cudaStreamSynchronize(s), "sync");
    }
    decode_rows(B, V, H, R, T, Hh, symmetric, clip, cov, a.future != nullptr, a.group_rows, a.cap ? a.cap : mv.context_length, h_out, nullptr);
    if (im.fuse_now && im.take_norm_flag()) {
        const bool saved = im.fuse;
        im.fuse = false;
        try { forecast_rows(a, B, V, H, symmetric, clip, ctx, umask, T_req, h_out); } catch (...) { im.fuse = saved; throw; }
        im.fuse = saved;
    }
}

void Engine::forecast_covariates(const CovRequest& q, bool symmetric, bool clip, float* h_out) {
    Range range("tsb forecast (covariates)");
    check(cudaSetDevice(device_), "cudaSetDevice");
    Impl& im = *impl_;
    if (im.pending.valid && im.fuse_now) {       // an earlier asynchronous forecast: complete it
        check(cudaStreamSynchronize(stream_), "forecast");
        finish_targets();
    }
    im.launches = 0;
    im.pending.valid = false;
    im.fuse_now = im.fuse_allowed();
    const ModelView& mv = im.mv;
    const int all = q.V + q.P + q.CP + q.K + q.CK;
    const int64_t R64 = int64_t(q.B) * all;
    if (q.B <= 0 || q.V <= 0 || q.T <= 0 || q.H <= 0 || R64 * (symmetric ? 2 : 1) > INT32_MAX)
        throw std::runtime_error("invalid covariate request dimensions");
    const int R = int(R64), R2 = symmetric ? 2 * R : R;
    const cudaStream_t s = stream_;
    const size_t TH = size_t(q.T) + q.H;
    auto upload = [&](DevBuf& d, const void* src, size_t bytes) {
        if (!bytes) return;
        d.ensure(bytes);
        check(cudaMemcpyAsync(d.p, src, bytes, cudaMemcpyHostToDevice, s), "upload");
    };
    upload(im.cov_ctx, q.ctx, size_t(q.B) * q.V * q.T * 4);
    if (q.umask) upload(im.cov_umask, q.umask, size_t(q.B) * q.V * q.T);
    upload(im.cov_past, q.past, size_t(q.B) * q.P * q.T * 4);
    upload(im.cov_known, q.known, size_t(q.B) * q.K * TH * 4);
    upload(im.cov_cpast, q.cat_past, size_t(q.B) * q.CP * q.T * 8);
    upload(im.cov_cknown, q.cat_known, size_t(q.B) * q.CK * TH * 8);
    CovShape c;
    c.B = q.B; c.V = q.V; c.P = q.P; c.CP = q.CP; c.K = q.K; c.CK = q.CK;
    c.T = q.T; c.H = q.H; c.kept = q.kept; c.len = q.len; c.hor = q.hor;
    c.mirrored = symmetric ? 1 : 0;
    c.smooth = q.smooth;
    const bool cov = mv.covariate_enabled && (q.P || q.K || q.CP || q.CK);
    const bool has_future = q.K || q.CK;
    im.rows.ensure(size_t(R2) * q.len * 4);
    im.mask.ensure(size_t(R2) * q.len);
    im.role.ensure(R2);
    if (has_future) { im.future.ensure(size_t(R2) * q.hor * 4); im.fmask.ensure(size_t(R2) * q.hor); }
    im.cov_first.ensure(size_t(q.B) * q.V * 4);
    const size_t scratch = covariate_scratch_bytes(c);
    if (scratch) im.cov_scratch.ensure(scratch);
    im.run("assemble", [&] {
        return assemble_covariates(c, im.cov_ctx.as<float>(), q.umask ? im.cov_umask.as<uint8_t>() : nullptr,
                                   im.cov_past.as<float>(), im.cov_known.as<float>(), im.cov_cpast.as<double>(),
                                   im.cov_cknown.as<double>(), im.rows.as<float>(), im.mask.as<int8_t>(),
                                   cov ? im.role.as<int8_t>() : nullptr, has_future ? im.future.as<float>() : nullptr,
                                   has_future ? im.fmask.as<int8_t>() : nullptr, im.cov_first.as<int>(),
                                   scratch ? im.cov_scratch.p : nullptr, s);
    });
    if (clip) {
        im.clip_ok.ensure(size_t(q.B) * q.V);
        im.run("clip", [&] {
            return clip_eligibility(im.cov_ctx.as<float>(), q.umask ? im.cov_umask.as<uint8_t>() : nullptr, q.B * q.V,
                                    q.T, im.clip_ok.as<int8_t>(), s);
        });
    }
    decode_rows(q.B, q.V, q.H, R, q.len, q.hor, symmetric, clip, cov, has_future, all, q.cap ? q.cap : mv.context_length, h_out, nullptr);
    if (im.fuse_now && im.take_norm_flag()) {      // fallback: the whole request with RMSNorm kernels
        const bool saved = im.fuse;
        im.fuse = false;
        try { forecast_covariates(q, symmetric, clip, h_out); } catch (...) { im.fuse = saved; throw; }
        im.fuse = saved;
    }
}

void Engine::decode_rows(int B, int V, int H, int R, int T, int Hh, bool symmetric, bool clip, bool cov,
                         bool has_future, int group_rows, int cap, float* h_out, float* h_decoded) {
    Impl& im = *impl_;
    const ModelView& mv = im.mv;
    const int ps = im.ps, Q = im.Q;
    const int R2 = symmetric ? 2 * R : R;
    const int patches = (H + ps - 1) / ps;
    const int shot = im.shot();
    const cudaStream_t s = stream_;
    im.decoded.ensure(size_t(R2) * H * Q * 4);
    int Tc = T, done = 0;
    while (done < patches) {
        const int block = std::min(shot, patches - done), n = block * ps, offset = done * ps;
        const int W = cov ? Tc + n : Tc;
        im.win.ensure(size_t(R2) * W * 4);
        im.wmask.ensure(size_t(R2) * W);
        check(cudaMemsetAsync(im.win.p, 0, size_t(R2) * W * 4, s), "memset");
        check(cudaMemsetAsync(im.wmask.p, 0, size_t(R2) * W, s), "memset");
        check(cudaMemcpy2DAsync(im.win.p, size_t(W) * 4, im.rows.p, size_t(Tc) * 4, size_t(Tc) * 4, R2, cudaMemcpyDeviceToDevice, s), "copy");
        check(cudaMemcpy2DAsync(im.wmask.p, W, im.mask.p, Tc, Tc, R2, cudaMemcpyDeviceToDevice, s), "copy");
        if (cov && has_future) {
            check(cudaMemcpy2DAsync(im.win.as<float>() + Tc, size_t(W) * 4, im.future.as<float>() + offset, size_t(Hh) * 4, size_t(n) * 4, R2, cudaMemcpyDeviceToDevice, s), "copy");
            check(cudaMemcpy2DAsync(im.wmask.as<int8_t>() + Tc, W, im.fmask.as<int8_t>() + offset, Hh, n, R2, cudaMemcpyDeviceToDevice, s), "copy");
        }
        if (im.observer && im.observer->before) im.observer->before(offset, block, Tc);
        im.predict_block(R2, Tc, block, cov, group_rows, R, done == 0, Tc);
        im.observe(offset, block, Tc, R2, W, has_future ? im.future.as<float>() + offset : nullptr,
                   has_future ? im.fmask.as<int8_t>() + offset : nullptr, Hh);
        const int used = std::min(n, H - offset);
        check(cudaMemcpy2DAsync(im.decoded.as<float>() + size_t(offset) * Q, size_t(H) * Q * 4, im.refined.p,
                                size_t(n) * Q * 4, size_t(used) * Q * 4, R2, cudaMemcpyDeviceToDevice, s), "copy");
        done += block;
        if (done >= patches) break;
        const int joined = Tc + n, keep = joined > cap ? std::max(ps, (cap / ps) * ps) : joined;
        im.next_rows.ensure(size_t(R2) * keep * 4);
        im.next_mask.ensure(size_t(R2) * keep);
        // future slice of this block, row stride n
        DevBuf& fs = im.fut_slice;
        DevBuf& fms = im.fmask_slice;
        if (has_future) {
            fs.ensure(size_t(R2) * n * 4); fms.ensure(size_t(R2) * n);
            check(cudaMemcpy2DAsync(fs.p, size_t(n) * 4, im.future.as<float>() + offset, size_t(Hh) * 4, size_t(n) * 4, R2, cudaMemcpyDeviceToDevice, s), "copy");
            check(cudaMemcpy2DAsync(fms.p, n, im.fmask.as<int8_t>() + offset, Hh, n, R2, cudaMemcpyDeviceToDevice, s), "copy");
        }
        im.run("feedback", [&] {
            return feedback(im.rc, im.rows.as<float>(), im.mask.as<int8_t>(), R2, Tc, im.refined.as<float>(), n,
                            cov ? im.role.as<int8_t>() : nullptr, has_future ? fs.as<float>() : nullptr,
                            has_future ? fms.as<int8_t>() : nullptr, keep, im.next_rows.as<float>(), im.next_mask.as<int8_t>(), s);
        });
        check(cudaStreamSynchronize(s), "sync");
        std::swap(im.rows.p, im.next_rows.p); std::swap(im.rows.bytes, im.next_rows.bytes);
        std::swap(im.mask.p, im.next_mask.p); std::swap(im.mask.bytes, im.next_mask.bytes);
        Tc = keep;
    }
    if (h_decoded) {                             // decode only: [R2][H][Q] before cap and combine
        check(cudaMemcpyAsync(h_decoded, im.decoded.p, size_t(R2) * H * Q * 4, cudaMemcpyDeviceToHost, s), "download");
        check(cudaStreamSynchronize(s), "sync");
        last_launches_ = im.launches;
        im.check_device_error("decode");
        return;
    }
    DevBuf& dout = im.out_rows;
    dout.ensure(size_t(B) * V * H * Q * 4);
    const int all = R / B;
    // Cap statistics come from the first block's scale pass over the assembled context.
    im.run("finalize", [&] {
        RowConfig rc = im.rc;
        rc.cap_k = im.cap_k();
        return finalize(rc, im.decoded.as<float>(), R, symmetric, B, V, all, H, H, im.caplo.as<float>(),
                        im.caphi.as<float>(), im.capsc.as<float>(), rc.cap_k > 0, clip ? im.clip_ok.as<int8_t>() : nullptr,
                        dout.as<float>(), im.err.as<int>(), s);
    });
    check(cudaMemcpyAsync(h_out, dout.p, size_t(B) * V * H * Q * 4, cudaMemcpyDeviceToHost, s), "download");
    check(cudaStreamSynchronize(s), "sync");
    last_launches_ = im.launches;
    im.check_device_error("forecast");
}

void inject_workspace_failures(int n) { g_injected_alloc_failures.store(n > 0 ? n : 0); }

}  // namespace tsb
