// SPDX-License-Identifier: Apache-2.0
//
// Column scaling of B without any device allocation.
//
// oztt_ii_scale_cols needs n*8 bytes of scratch for the column maxima and takes them from the CUDA
// stream-ordered allocator. Some callers cannot let a library allocate device memory at call time:
// applications that hand all device memory to their own allocator or to a fixed budget reserved up
// front, and code on latency-critical paths where a driver allocation (which may synchronise or fail
// under memory pressure) is not acceptable. oztt_ii_scale_cols_noalloc serves them: its scratch is
// the file-scope array below, of a fixed size, which every GPU that loads the library holds until the
// process exits.
//
// Rules of use, for callers:
//   * At most OZTT_NOALLOC_MAX_COLS columns per call; larger n is rejected with OZTT_EINVAL.
//   * The first call on a device looks up the array's device address (cudaGetSymbolAddress) with that
//     device current and caches it; make that first call before any stream capture on that device. The
//     cache is keyed on the device's current CUDA context, so after cudaDeviceReset (which unloads the
//     library's module with the context) the next call looks the address up again: make that call
//     before any stream capture too.
//   * Every call on a device uses the same array and leaves the last call's column maxima in it; the
//     call clears the part it uses (on `stream`) before the maxima are reduced into it. Calls that
//     overlap on the GPU (on different streams without ordering between them) race on the array.
//   * No cudaMalloc, cudaFree or allocating library routine is called.
#include <cuda.h>

#include <mutex>

#include "oztt_common.cuh"

namespace oztt {

void launch_scale_cols(const double* b, uint64_t k, uint64_t n, uint64_t ldb, int32_t shift, int32_t* delta,
                       uint16_t* bfmax, uint32_t* flags, unsigned long long* colmax, cudaStream_t st);

namespace {

constexpr uint64_t kMaxCols = OZTT_NOALLOC_MAX_COLS;

// Column maxima of the no-allocation variant (host code must not use this name as an address; it
// uses the device address looked up below).
static __device__ __align__(256) unsigned long long g_colmax_scratch[kMaxCols];

constexpr int kMaxDevices = 64;
std::mutex g_setup_mu;
unsigned long long* g_scratch_ptr[kMaxDevices] = {};
CUcontext g_scratch_ctx[kMaxDevices] = {};  // the context each cached address belongs to

using CtxGetCurrentFn = CUresult (*)(CUcontext*);

// The calling thread's current CUDA context (the device's primary context once the runtime has set it
// up), or nullptr when there is none yet.
CUcontext current_context() {
    static CtxGetCurrentFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<CtxGetCurrentFn>(p);
    });
    if (!fn) throw Error(OZTT_ERUNTIME, "cuCtxGetCurrent is not available from the CUDA driver");
    CUcontext ctx = nullptr;
    if (fn(&ctx) != CUDA_SUCCESS) return nullptr;
    return ctx;
}

// Device address of the scratch array on the current device, looked up once per device and context.
unsigned long long* scratch_on_current_device() {
    int dev = 0;
    OZTT_CUDA(cudaGetDevice(&dev));
    if (dev < 0 || dev >= kMaxDevices) throw Error(OZTT_ERUNTIME, "device ordinal out of the supported range");
    std::lock_guard<std::mutex> lock(g_setup_mu);
    const CUcontext ctx = current_context();
    if (!g_scratch_ptr[dev] || ctx == nullptr || ctx != g_scratch_ctx[dev]) {
        void* ptr = nullptr;
        const cudaError_t rc = cudaGetSymbolAddress(&ptr, g_colmax_scratch);
        if (rc != cudaSuccess || ptr == nullptr)
            throw Error(OZTT_ERUNTIME, std::string("cannot obtain the device address of the column scratch: ") +
                                           cudaGetErrorString(rc));
        g_scratch_ptr[dev] = static_cast<unsigned long long*>(ptr);
        g_scratch_ctx[dev] = current_context();  // set up by the lookup if there was none before
    }
    return g_scratch_ptr[dev];
}

}  // namespace
}  // namespace oztt

extern "C" int oztt_ii_scale_cols_noalloc(const double* b, uint64_t k, uint64_t n, uint64_t ldb, int32_t shift,
                                          int32_t* delta, uint16_t* bf16max, uint32_t* flags, void* stream, char* err,
                                          size_t errlen) {
    return oztt::guarded(err, errlen, [&] {
        if (!b || !delta || !flags || ldb < n) throw oztt::Error(OZTT_EINVAL, "scale_cols_noalloc: bad arguments");
        if (n > oztt::kMaxCols)
            throw oztt::Error(OZTT_EINVAL, "scale_cols_noalloc: n = " + std::to_string(n) + " exceeds the limit of " +
                                               std::to_string(oztt::kMaxCols) +
                                               " columns of the preallocated scratch; use oztt_ii_scale_cols");
        unsigned long long* colmax = oztt::scratch_on_current_device();
        oztt::launch_scale_cols(b, k, n, ldb, shift, delta, bf16max, flags, colmax,
                                reinterpret_cast<cudaStream_t>(stream));
    });
}
