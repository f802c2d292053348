// Shared device helpers for the sm_100a kernels: error words, bounded mbarrier waits,
// TMA and tcgen05 PTX wrappers, and the reference's float arithmetic restated for the GPU.
#pragma once
#include <atomic>
#include <cstdint>
#include <mutex>
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

namespace tsb {

// Unique id (for the life of the process) of the calling thread's current CUDA context, or
// false when the driver does not offer it or no context is current yet.
inline bool current_context_id(unsigned long long* id) {
    using GetCurrentFn = CUresult (*)(CUcontext*);
    using GetIdFn = CUresult (*)(CUcontext, unsigned long long*);
    static GetCurrentFn get_current = nullptr;
    static GetIdFn get_id = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            get_current = reinterpret_cast<GetCurrentFn>(p);
        if (cudaGetDriverEntryPoint("cuCtxGetId", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            get_id = reinterpret_cast<GetIdFn>(p);
    });
    CUcontext ctx = nullptr;
    if (!get_current || !get_id || get_current(&ctx) != CUDA_SUCCESS || !ctx) return false;
    return get_id(ctx, id) == CUDA_SUCCESS;
}

// Per device, the context in which a kernel's launch attributes (its dynamic shared-memory
// limit) were last set, so that they are set once per context: again after a device reset
// (cudaDeviceReset replaces the context and drops them), and on every launch when the
// context cannot be identified. Safe to use from several host threads.
struct KernelSetup {
    std::atomic<unsigned long long> ctx[64] = {};   // context id + 1; 0: not set yet
    bool needed(int dev, unsigned long long* key) {
        unsigned long long id = 0;
        *key = current_context_id(&id) ? id + 1 : 0;
        return dev < 0 || dev >= 64 || *key == 0 || ctx[dev].load(std::memory_order_acquire) != *key;
    }
    void done(int dev, unsigned long long key) {
        if (dev >= 0 && dev < 64) ctx[dev].store(key, std::memory_order_release);
    }
};

// ---------------------------------------------------------------------------------------
// Device error word. Kernels that wait on barriers never spin forever: a wait that runs
// past its limit records a code here and the kernel unwinds; the host reads the word after
// the launch sequence and turns it into an error status.
enum DeviceError : int {
    kDevOk = 0,
    kDevTimeoutFull = 1,      // MMA warp: smem stage never filled
    kDevTimeoutEmpty = 2,     // producer: smem stage never released
    kDevTimeoutAccFull = 3,   // epilogue: accumulator never committed
    kDevTimeoutAccEmpty = 4,  // MMA warp: accumulator never drained
    kDevTimeoutAttn = 5,      // attention kernel barrier
    kDevBadShape = 6,         // position outside the RoPE table, or a NaN raw quantile
    kDevNaN = 7,              // a capped forecast value is NaN (reference: degenerate input)
    kDevNonFinite = 8,        // a final forecast value is not finite
    kDevTimeoutConv = 9,      // Q8_0 GEMM: weights never converted / int8 stage never filled
};

__device__ __forceinline__ void record_error(int* err, int code) {
    if (err) atomicCAS(err, 0, code);
}

// Wait limit for one mbarrier wait, in SM clock cycles (about 2 s at 1.9 GHz).
constexpr long long kWaitCycles = 4000000000LL;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------------------------------
// mbarrier
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
__device__ __forceinline__ void mbar_fence_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
// The waiting thread may be suspended until the phase completes or `kSuspendNs` passes, so
// waiting warps take no issue slots from the warps that compute; callers loop with their
// own overall bound.
constexpr uint32_t kSuspendNs = 200000;
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity), "n"(kSuspendNs)
        : "memory");
    return ok != 0;
}
// The same with acquire semantics at cluster scope: for barriers that threads of the peer
// CTA arrive on after writing shared memory that this CTA's tensor-core operations read.
__device__ __forceinline__ bool mbar_try_wait_cluster(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2, %3;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity), "n"(kSuspendNs)
        : "memory");
    return ok != 0;
}
// Bounded wait: true when the phase completed, false after the cycle limit.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
    if (mbar_try_wait(bar, parity)) return true;
    const long long start = clock64();
    while (true) {
        if (mbar_try_wait(bar, parity)) return true;
        if (clock64() - start > kWaitCycles) return false;
    }
}

// ---------------------------------------------------------------------------------------
// TMA (tiled bulk tensor copies, global -> shared), no multicast.
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
            smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y)
        : "memory");
}
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y, int z) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(
            smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z)
        : "memory");
}
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}
__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// 16-byte asynchronous global -> shared copy (L2 only), grouped per thread.
__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
// Wait until at most N of this thread's most recent groups are still in flight.
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// ---------------------------------------------------------------------------------------
// tcgen05 (5th-generation tensor cores, accumulators in tensor memory)
__device__ __forceinline__ void tmem_alloc(uint32_t* slot, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)), "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D[tmem] (+)= A[smem] * B[smem]^T, kind::f16 (f16 operands, f32 accumulation).
__device__ __forceinline__ void mma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                        uint32_t accumulate) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// Arrive on an mbarrier once every previously issued tcgen05.mma of this thread completes.
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}
// ---- CTA pairs (cluster of two CTAs sharing one tcgen05.mma.cta_group::2) ----
__device__ __forceinline__ uint32_t cluster_ctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
// Address of the same shared-memory object in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t smem_addr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_addr), "r"(rank));
    return r;
}
// Arrive on an mbarrier given by its shared::cluster address (possibly in the peer CTA),
// without release semantics: the arrival orders no memory writes of the caller, so it does
// not wait for the caller's outstanding global stores (used to hand back TMEM whose reads
// have completed, tcgen05.wait::ld).
__device__ __forceinline__ void mbar_arrive_cluster_relaxed(uint32_t cluster_addr) {
    asm volatile("mbarrier.arrive.relaxed.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
// Arrive with release semantics (cluster scope) on an mbarrier given by its shared::cluster
// address: the caller's earlier shared-memory writes are visible to whoever waits on it.
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
// Every thread of both CTAs of the cluster.
__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\nbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* slot, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)), "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
// 2D tile load of this CTA's half of a pair operand; the transaction bytes count on the
// mbarrier at `leader_bar` (shared::cluster address in CTA 0). No multicast.
__device__ __forceinline__ void tma_load_2d_pair(void* dst, const CUtensorMap* map, uint32_t leader_bar, int x, int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];"
        ::"r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(leader_bar), "r"(x), "r"(y)
        : "memory");
}
__device__ __forceinline__ void tma_load_3d_pair(void* dst, const CUtensorMap* map, uint32_t leader_bar, int x, int y,
                                                 int z) {
    asm volatile(
        "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];"
        ::"r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(leader_bar), "r"(x), "r"(y), "r"(z)
        : "memory");
}
// D (both CTAs' TMEM, M = 256 split by rows) (+)= A (both CTAs' smem) * B^T (both CTAs' smem,
// N split by rows of B); issued by CTA 0 only.
__device__ __forceinline__ void mma_f16_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                             uint32_t accumulate) {
    const uint32_t z = 0;
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8, %9, %10, %11, %12}, p;\n}\n"
        ::"r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(z), "r"(z), "r"(z), "r"(z), "r"(z),
        "r"(z), "r"(z), "r"(z)
        : "memory");
}
// Arrive on the mbarrier at the same offset in both CTAs of the pair once the pair MMAs
// issued so far complete.
__device__ __forceinline__ void mma_commit_pair(uint64_t* bar) {
    const uint16_t mask = 0x3;
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;"
                 ::"r"(smem_u32(bar)), "h"(mask)
                 : "memory");
}

// 32 lanes x 32 consecutive 32-bit columns: thread i of the warp receives lane (base+i).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Shared-memory matrix descriptor for a K-major operand tile stored with the 128-byte
// swizzle: rows of 64 f16 (128 B), 8-row atoms of 1024 B (stride byte offset), layout
// type SWIZZLE_128B (2) in bits 61-63, descriptor version 1 in bits 46-47.
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t smem_addr) {
    uint64_t d = 0;
    d |= uint64_t((smem_addr >> 4) & 0x3FFF);
    d |= uint64_t(1) << 16;                 // leading byte offset (unused for swizzled K-major)
    d |= uint64_t(1024 >> 4) << 32;         // stride byte offset: 8 rows x 128 B
    d |= uint64_t(1) << 46;                 // version
    d |= uint64_t(2) << 61;                 // SWIZZLE_128B
    return d;
}
// Instruction descriptor, kind::f16: f16 A and B (K-major), f32 accumulator, M x N.
__host__ __device__ constexpr uint32_t idesc_f16(int M, int N) {
    return (1u << 4) | (0u << 7) | (0u << 10) | (uint32_t(N >> 3) << 17) | (uint32_t(M >> 4) << 24);
}
// Same with B given N-major (MN-major; used for P*V where V is [keys][hd]).
__host__ __device__ constexpr uint32_t idesc_f16_bmn(int M, int N) {
    return idesc_f16(M, N) | (1u << 16);
}

// ---------------------------------------------------------------------------------------
// Reference float arithmetic, restated for the GPU.

// SLEEF-style float exp of the reference's sigmoid, SiLU and softplus
// (reference src/layers.cpp:658-667). Outside the polynomial range it calls expf.
__device__ __forceinline__ float activation_exp(float x) {
    if (!isfinite(x) || x < -87.f || x > 88.f) return expf(x);
    const float q = nearbyintf(__fmul_rn(x, 1.4426950408889634f));
    float r = __fmaf_rn(q, -.693145751953125f, x);
    r = __fmaf_rn(q, -1.428606765330187045e-6f, r);
    float u = .000198527617612853646f;
    u = __fmaf_rn(u, r, .00139304355252534151f);
    u = __fmaf_rn(u, r, .00833336077630519867f);
    u = __fmaf_rn(u, r, .0416664853692054749f);
    u = __fmaf_rn(u, r, .166666671633720398f);
    u = __fmaf_rn(u, r, .5f);
    return ldexpf(__fadd_rn(1.f, __fmaf_rn(__fmul_rn(r, r), u, r)), int(q));
}
// ATen exp_u20 polynomial of the reference softmax (reference src/layers.cpp:297-305).
__device__ __forceinline__ float attention_exp(float x) {
    if (x < -87.3365478515625f) return 0.f;
    if (!isfinite(x) || x > 88.f) return expf(x);
    const float n = floorf(__fmaf_rn(x, 1.4426950216293335f, .5f));
    const float r = __fmaf_rn(-n, .6931471824645996f, x);
    float y = __fmaf_rn(r, .00828929059f, .0418978221f);
    y = __fmaf_rn(r, y, .166676521f);
    y = __fmaf_rn(r, y, .499991506f);
    y = __fmaf_rn(r, y, .999999701f);
    y = __fmaf_rn(r, y, 1.f);
    return __fmul_rn(__fmul_rn(y, ldexpf(1.f, int(n) - 1)), 2.f);
}
__device__ __forceinline__ float ref_sigmoid(float x) { return __fdiv_rn(1.0f, __fadd_rn(1.0f, activation_exp(-x))); }
__device__ __forceinline__ float ref_silu(float x) { return __fdiv_rn(x, __fadd_rn(1.0f, activation_exp(-x))); }

__device__ __forceinline__ uint32_t pack_half2(float a, float b) {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
}

}  // namespace tsb
