// no_alloc.cu -- MoeExpertFFNNoAlloc: the expert FFN for callers that cannot
// allocate device memory.
//
// Some callers of this library are not allowed to call cudaMalloc at all: code
// running inside a host framework that owns every device allocation through its
// own pool, a runtime that forbids allocation after start-up, or a service whose
// memory budget is fixed when it loads.  MoeExpertFFN needs a caller-provided
// workspace; this entry point instead uses one scratch array that lives in the
// library itself, a file-scope __device__ array of MOE_NO_ALLOC_SCRATCH_BYTES.
// Every GPU that loads the library holds that array until the process exits.
//
// In host code `g_moe_scratch` names a host-side stand-in, not a device address,
// so it is never passed to a kernel.  The device address is looked up with
// cudaGetSymbolAddress once per device, with that device current, the first time
// the entry point is called on it; make that first call before any stream
// capture begins.  The entry point then runs the ordinary MoeExpertFFN path on
// that address.  It calls no cudaMalloc, cudaFree or allocating library routine.
//
// All calls share the one array and it keeps the last call's contents; the path
// clears what must start at zero (the device error word) at the start of each
// call and overwrites everything else before reading it.  Calls that overlap on
// the GPU (on different streams, or from several host threads) race on the
// array and must be serialised by the caller.
//
// Device-side failures (an expert id outside [0,E), a bounded wait that gave up)
// land in the error word at the start of the array, as they land in word 0 of a
// caller's workspace on the ordinary path; MoeNoAllocGetDeviceError reads it.
//
// The cached address belongs to the device's primary context: do not keep using
// the entry point across cudaDeviceReset (the module is reloaded and the array
// may move).
#include <mutex>

#include "../../include/moe_ops.h"
#include "moe_common.cuh"

static __device__ __align__(256) uint8_t g_moe_scratch[MOE_NO_ALLOC_SCRATCH_BYTES];

namespace {

constexpr int kMaxDevices = 64;
void* g_scratch_ptr[kMaxDevices] = {nullptr};
std::mutex g_scratch_mu;

// Device address of g_moe_scratch on the current device (set up once per device).
int scratch_address(void** out)
{
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return MOE_ERR_CUDA;
    if (dev < 0 || dev >= kMaxDevices) return MOE_ERR_UNSUPPORTED;
    std::lock_guard<std::mutex> lock(g_scratch_mu);
    if (!g_scratch_ptr[dev]) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_moe_scratch);
        if (e != cudaSuccess || p == nullptr) return MOE_ERR_CUDA;
        g_scratch_ptr[dev] = p;
    }
    *out = g_scratch_ptr[dev];
    return MOE_OK;
}

}  // namespace

extern "C" int MoeExpertFFNNoAlloc(const void* x, const int32_t* expert_ids, const void* weights,
                                   const void* expert_weights, void* expert_out, int64_t T,
                                   int64_t H, int64_t E, int64_t K, int64_t I, void* stream)
{
    const size_t need = MoeExpertFFNWorkspaceSize(T, H, E, K, I);
    if (need == 0) return MOE_ERR_BAD_SHAPE;
    if (need > (size_t)MOE_NO_ALLOC_SCRATCH_BYTES) return MOE_ERR_WORKSPACE_TOO_SMALL;
    void* scratch = nullptr;
    int rc = scratch_address(&scratch);
    if (rc != MOE_OK) return rc;
    return MoeExpertFFN(x, expert_ids, weights, expert_weights, expert_out, T, H, E, K, I, scratch,
                        (size_t)MOE_NO_ALLOC_SCRATCH_BYTES, stream);
}

extern "C" int MoeNoAllocGetDeviceError(int* code, void* stream)
{
    if (!code) return MOE_ERR_NULL_POINTER;
    void* scratch = nullptr;
    int rc = scratch_address(&scratch);
    if (rc != MOE_OK) return rc;
    return MoeGetDeviceError(scratch, code, stream);
}
