// mhcPreRunNoAlloc: the operator for callers that cannot allocate device memory.
//
// The workspace that mhcPreRun takes from its caller (prepared weights plus the
// split-K partial records) lives here in one fixed device array instead.  Host
// code cannot use the array's name as a device address (it is a host-side
// stand-in), so each device's address is looked up once with
// cudaGetSymbolAddress while that device is current, and passed to the kernels.
#include <atomic>

#include "mhc_pre_internal.h"

namespace mhc {

static __device__ __align__(256) uint8_t g_noalloc_scratch[MHC_PRE_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
static std::atomic<void*> g_scratch_addr[kMaxDevices];

// Device address of the scratch array on the current device (looked up on the
// first call per device; concurrent first calls look up the same address).
static int scratch_for_current_device(void** out) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return MHC_STATUS_CUDA_ERROR;
    if (dev < 0 || dev >= kMaxDevices) return MHC_STATUS_UNSUPPORTED_DEVICE;
    void* p = g_scratch_addr[dev].load(std::memory_order_acquire);
    if (p == nullptr) {
        if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || p == nullptr) return MHC_STATUS_CUDA_ERROR;
        g_scratch_addr[dev].store(p, std::memory_order_release);
    }
    *out = p;
    return MHC_STATUS_SUCCESS;
}

}  // namespace mhc

using namespace mhc;

extern "C" int mhcPreRunNoAlloc(const mhcPreDesc_t* desc, const void* x, const float* phi, const float* alpha,
                                const float* bias, const float* gamma, void* hIn, float* hPost, float* hRes,
                                void* stream) {
    Problem p;
    Plan plan;
    int rc = plan_for(desc, &p, &plan);
    if (rc != 0) return rc;
    if (plan.totalBytes > MHC_PRE_NOALLOC_SCRATCH_BYTES) return MHC_STATUS_TOO_LARGE;
    void* scratch = nullptr;
    rc = scratch_for_current_device(&scratch);
    if (rc != 0) return rc;
    // The weight preparation clears the part of the scratch that must start at
    // zero (its header); every other byte the kernels read is written first.
    return prepare_and_run(p, plan, x, phi, alpha, bias, gamma, hIn, hPost, hRes, scratch,
                           static_cast<cudaStream_t>(stream));
}
