// cuda_backend.hpp -- the physical-GPU fm::Backend for B200 (sm_100a).
//
// Drop-in replacement for the GpuBackend placeholder of the reference
// (src/backend.cpp:528-571).  It implements the fm::Backend interface
// (include/fm/backend.hpp:145-177) over the C ABI of libfreemoe_b200.so
// (include/freemoe_b200.h); every status the ABI returns becomes
// fm::fail(ErrorCode(status), message), so the engine, the residency manager
// and the CLI see the same typed errors as from the CPU backends.
//
// Memory placement:
//   ExpertCache            plain HBM (cudaMalloc): the residency manager's
//                          expert slots.  Only the device reads them; the
//                          slot read-back for checksums goes through
//                          download(), the quantised expert GEMVs through
//                          matvec_quant() (engine_hooks.cpp routes the
//                          unchanged engine's calls there).
//   Weights                HBM (managed, preferred location = the device):
//                          the GEMVs read them on the device; the unchanged
//                          engine also reads some on the host (token embedding
//                          rows, norm scales).
//   KV, Workspace, Staging,
//   Other                  pinned host memory: the parts of forward_token that
//                          stay on the CPU (attention, norms) use them.
// Uploads copy into a pinned staging ring and go to the device with
// cudaMemcpyAsync on a side stream; the fence is a CUDA event polled against
// the caller's deadline.  Injected faults are honoured on the host, before
// any CUDA call, exactly where CpuBackend honours them.
#pragma once

#include <cstdint>
#include <map>
#include <memory>
#include <set>
#include <string>
#include <vector>

#include "fm/backend.hpp"

namespace fmcuda {

struct Runtime; // device, streams, staging; shared with every DeviceBuffer cleanup

class CudaBackend final : public fm::Backend {
public:
    CudaBackend(fm::BackendConfig config, fm::TraceWriter *trace, int device = 0);
    ~CudaBackend() override;

    std::string name() const override { return "cuda-sm100a"; }
    fm::DeviceInfo info() const override;
    std::unique_ptr<fm::DeviceBuffer> allocate(uint64_t bytes, fm::AllocationTag tag) override;
    fm::Fence upload(fm::DeviceBuffer &buffer, const void *src, uint64_t bytes) override;
    bool fence_complete(const fm::Fence &fence) const override;
    void wait_fence(const fm::Fence &fence, uint32_t timeout_ms) override;
    void advance_fences() override;
    void matvec(const float *weights, const float *x, float *y, uint32_t out_dim, uint32_t in_dim,
                const std::string &op_name) override;
    void inject_fault(fm::BackendFault fault) override { fault_ = fault; }
    void clear_faults() override;

    // Quantised product on the device, the GEMV that Engine::matvec_view runs
    // on the CPU for block types (src/engine.cpp:360-367): W lives in a
    // buffer of this backend, x and y are host vectors.  An empty op_name
    // records nothing (the caller records the operation itself).
    void matvec_quant(uint32_t type_id, const uint8_t *weights, const float *x, float *y,
                      uint32_t out_dim, uint32_t in_dim, const std::string &op_name);
    // Copies device bytes back to the host (the slot read-back of
    // src/residency.cpp:703-714 without touching managed pages on the host).
    void download(const fm::DeviceBuffer &buffer, void *dst, uint64_t bytes);
    // The same for any range inside one of this backend's device buffers.
    void download_range(void *dst, const void *src, uint64_t bytes);
    // Synchronous host -> device copy into one of this backend's device buffers.
    void upload_range(void *dst, const void *src, uint64_t bytes);
    // True when `p` points into memory this backend allocated on the device;
    // *host_readable says whether the host may also read it (managed memory).
    bool owns_device_pointer(const void *p, bool *host_readable = nullptr) const;
    // The live CUDA backend whose device memory holds `p` (NULL if none).
    static CudaBackend *owner_of(const void *p, bool *host_readable = nullptr);

private:
    std::shared_ptr<Runtime> rt_;
    fm::BackendFault fault_ = fm::BackendFault::None;
    uint64_t next_fence_ = 1;
    std::map<uint64_t, void *> fence_events_; // fence id -> cudaEvent_t
    std::set<uint64_t> deferred_fences_;
    std::set<uint64_t> ready_fences_;
    int matvec_order_ = 0;
};

// Factory used by Backend::create for BackendKind::PhysicalGPU.
std::unique_ptr<fm::Backend> make_cuda_backend(const fm::BackendConfig &config,
                                               fm::TraceWriter *trace);

} // namespace fmcuda
