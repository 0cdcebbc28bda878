// moe_noalloc.cu -- fmcuda_moe_block_noalloc: the MoE block with a scratch
// area that is part of the library image, for callers that cannot allocate
// device memory.
//
// Who needs it: a host whose device memory is fully committed before decoding
// starts -- FreeMoe's residency manager sizes its pool of HBM expert slots from
// the whole free budget (compute_budget) -- or a plug-in living inside a host
// framework that owns the device allocator and gives plug-ins no way to call
// cudaMalloc.  Both can still run the routed-expert block through this entry
// point: its scratch is a fixed array in the library's device image, so the
// call allocates nothing and frees nothing.
#include <cuda.h>

#include <mutex>
#include <string>

#include "common.cuh"

namespace fmb {

int moe_block_run(const fmcuda_moe_args *a, void *workspace, uint64_t workspace_bytes, cudaStream_t s);
uint64_t moe_workspace_size(uint32_t tokens, uint32_t experts, uint32_t top_k, uint32_t d, uint32_t ffn);

namespace {

// The scratch itself.  Every GPU that loads the library holds these bytes
// until the process exits.  In host code `g_noalloc_scratch` only names the
// symbol; its device address comes from cudaGetSymbolAddress below.
static __device__ __align__(256) uint8_t g_noalloc_scratch[FM_MOE_NOALLOC_SCRATCH_BYTES];

std::mutex g_scratch_mutex;
struct ScratchEntry {
    CUcontext ctx = nullptr; // the context the address belongs to
    void *addr = nullptr;
};
ScratchEntry g_scratch_addr[64];

// The current driver context (looked up through the runtime, so the library
// needs no link against the driver library); NULL if none is current yet.
CUcontext current_context() {
    using GetCurrent = CUresult (*)(CUcontext *);
    static GetCurrent fn = [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            p = nullptr;
        return reinterpret_cast<GetCurrent>(p);
    }();
    CUcontext ctx = nullptr;
    if (!fn || fn(&ctx) != CUDA_SUCCESS) return nullptr;
    return ctx;
}

// Device address of the scratch on the current device, looked up with that
// device current and cached per device and context: a context that was torn
// down and created again (cudaDeviceReset) gets its own lookup.
int scratch_address(void **out) {
    int dev = 0;
    cudaError_t err = cudaGetDevice(&dev);
    if (err != cudaSuccess) return cuda_status(err, "cudaGetDevice");
    if (dev < 0 || dev >= 64)
        return set_error(FM_STATUS_INVALID_ARGUMENT, "device ordinal out of range for the scratch table");
    std::lock_guard<std::mutex> lock(g_scratch_mutex);
    ScratchEntry &e = g_scratch_addr[dev];
    const CUcontext ctx = current_context();
    if (!e.addr || !ctx || ctx != e.ctx) {
        void *p = nullptr;
        err = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (err != cudaSuccess) {
            (void)cudaGetLastError();
            return cuda_status(err, "scratch symbol lookup");
        }
        e.addr = p;
        e.ctx = current_context(); // the lookup made the device's context current
    }
    *out = e.addr;
    return FM_STATUS_OK;
}

} // namespace
} // namespace fmb

using namespace fmb;

extern "C" int fmcuda_moe_block_noalloc(const fmcuda_moe_args *args, void *stream) {
    if (!args) return set_error(FM_STATUS_INVALID_ARGUMENT, "null MoE arguments");
    const uint64_t need = moe_workspace_size(args->tokens, args->experts, args->top_k, args->d_model, args->ffn);
    if (need > FM_MOE_NOALLOC_SCRATCH_BYTES)
        return set_error(FM_STATUS_INVALID_ARGUMENT,
                         "fmcuda_moe_block_noalloc: this block needs " + std::to_string(need) +
                             " bytes of scratch but the built-in scratch holds " +
                             std::to_string(static_cast<uint64_t>(FM_MOE_NOALLOC_SCRATCH_BYTES)) +
                             "; split the tokens into smaller calls or use fmcuda_moe_block");
    void *scratch = nullptr;
    int rc = scratch_address(&scratch);
    if (rc) return rc;
    // Nothing in the scratch has to start at zero: each call writes every
    // section before it reads it, so the previous call's contents do no harm.
    return moe_block_run(args, scratch, FM_MOE_NOALLOC_SCRATCH_BYTES, static_cast<cudaStream_t>(stream));
}
