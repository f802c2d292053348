// Refine of one decode block with no device allocation (see tsb_refine_static in
// include/timestral_b200.h).
//
// The forecast path sizes the refine kernel's float64 scan scratch per request and takes it
// from the engine's workspace. Callers that may not allocate device memory at all — code
// running inside a host that owns every device allocation (a plugin given a fixed memory
// budget, a real-time loop that must not enter the CUDA allocator) — use this entry point
// instead: the scratch lives in a fixed array compiled into the library.
#include "common.cuh"
#include "rows.cuh"
#include "timestral_b200.h"

#include <cuda.h>

#include <cfloat>
#include <cmath>
#include <cstring>
#include <mutex>
#include <string>

namespace tsb {
void set_thread_error(const char* message);
}

namespace {

// Fixed scratch: 4 MiB of float64 on every GPU where the library's device code is loaded
// (with CUDA's lazy module loading, from the first call of this entry point or of another
// kernel of the library on that device), held until the process exits. One call needs rows * (3 * (length / patch_size + patches) + 2 * patch_size +
// 2 * patches) values (e.g. 1,700 rows of a 2048-step context with 8 horizon patches).
constexpr size_t kScratchDoubles = size_t(1) << 19;
static __device__ __align__(256) double g_refine_scratch[kScratchDoubles];

constexpr int kMaxDevices = 64;
double* g_scratch_ptr[kMaxDevices] = {};
unsigned long long g_scratch_ctx[kMaxDevices] = {};   // context id the address belongs to
std::mutex g_setup_mutex;

// Device address of the scratch array on the current device. In host code
// `g_refine_scratch` names a host-side stand-in, not device memory, so the address is looked
// up with cudaGetSymbolAddress: on a device's first call (which also loads the library's
// device code there and reserves the array, CUDA loading modules lazily), and again after
// the device's context was replaced (cudaDeviceReset), which invalidates the old address.
cudaError_t scratch_address(int dev, double** out) {
    std::lock_guard<std::mutex> lock(g_setup_mutex);
    unsigned long long id = 0;
    const bool known = tsb::current_context_id(&id);
    if (!g_scratch_ptr[dev] || !known || id != g_scratch_ctx[dev]) {
        void* p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_refine_scratch);
        if (e != cudaSuccess) return e;
        g_scratch_ptr[dev] = static_cast<double*>(p);
        g_scratch_ctx[dev] = tsb::current_context_id(&id) ? id : 0;
    }
    *out = g_scratch_ptr[dev];
    return cudaSuccess;
}

int fail(int code, const std::string& message) {
    tsb::set_thread_error(message.c_str());
    return code;
}

}  // namespace

extern "C" TIMESTRAL_API int tsb_refine_static(const float* d_q, const float* d_rows, const int8_t* d_mask,
                                               const int8_t* d_role, const float* d_loc0, const float* d_scale0,
                                               int32_t rows, int32_t length, int32_t patches, int32_t patch_size,
                                               int32_t num_quantiles, int32_t median_index, double minimum_scale,
                                               float* d_out, void* stream) {
    if (!d_q || !d_out || rows <= 0 || patches <= 0 || patch_size <= 0 || num_quantiles <= 0 || num_quantiles > 64 ||
        median_index < 0 || median_index >= num_quantiles)
        return fail(TSB_ERR_ARG, "tsb_refine_static: invalid arguments");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const size_t n = size_t(rows) * size_t(patches) * size_t(patch_size) * size_t(num_quantiles);
    if (patches == 1) {
        // One patch: the reference returns the block unchanged (src/refine.cpp:82).
        const cudaError_t e = cudaMemcpyAsync(d_out, d_q, n * sizeof(float), cudaMemcpyDeviceToDevice, s);
        return e == cudaSuccess ? TSB_OK : fail(TSB_ERR_CUDA, cudaGetErrorString(e));
    }
    if (!d_rows || !d_mask || !d_loc0 || !d_scale0 || length <= 0 || length % patch_size ||
        !(minimum_scale > 0) || !std::isfinite(minimum_scale))
        return fail(TSB_ERR_ARG, "tsb_refine_static: invalid context arguments");
    const size_t per_row = 3 * (size_t(length / patch_size) + size_t(patches)) + 2 * size_t(patch_size) + 2 * size_t(patches);
    const size_t need = per_row * size_t(rows);
    if (need > kScratchDoubles)
        return fail(TSB_ERR_ARG, "tsb_refine_static: needs " + std::to_string(need) + " float64 scratch values, above the " +
                                     std::to_string(kScratchDoubles) + " the library reserves; split the rows into smaller calls");
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess || dev < 0 || dev >= kMaxDevices) return fail(TSB_ERR_CUDA, "tsb_refine_static: no usable CUDA device");
    double* scratch = nullptr;
    e = scratch_address(dev, &scratch);
    if (e != cudaSuccess) return fail(TSB_ERR_CUDA, std::string("cudaGetSymbolAddress: ") + cudaGetErrorString(e));
    tsb::RowConfig rc;
    std::memset(&rc, 0, sizeof(rc));
    rc.ps = patch_size;
    rc.minimum_scale = minimum_scale;
    rc.Q = num_quantiles;
    rc.median = median_index;
    // Every scratch value the kernel reads it writes first in the same call, so nothing is
    // cleared between calls.
    const double clip = std::pow(double(FLT_MAX), 0.5) / 1e3;
    e = tsb::refine(rc, d_q, d_rows, d_mask, length, d_role, d_loc0, d_scale0, rows, length, patches, clip, scratch, d_out, s);
    return e == cudaSuccess ? TSB_OK : fail(TSB_ERR_CUDA, cudaGetErrorString(e));
}
