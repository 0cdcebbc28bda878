// cuda_backend.cpp -- fm::Backend over libfreemoe_b200.so (see cuda_backend.hpp).
#include "cuda_backend.hpp"

#include <algorithm>
#include <atomic>
#include <cstring>
#include <mutex>
#include <thread>

#include "freemoe_b200.h"

namespace fmcuda {

namespace {

[[noreturn]] void fail_status(int status, const std::string &what) {
    const char *msg = fmcuda_last_error();
    fm::fail(static_cast<fm::ErrorCode>(status), what + ": " + (msg ? msg : ""));
}

void check(int status, const std::string &what) {
    if (status != FM_STATUS_OK) fail_status(status, what);
}

bool device_tag(fm::AllocationTag tag) {
    return tag == fm::AllocationTag::Weights || tag == fm::AllocationTag::ExpertCache;
}

// Every live CudaBackend, for the link-time engine hooks that map a raw
// pointer back to the backend that owns it.
std::mutex g_registry_mutex;
std::vector<CudaBackend *> g_registry;
std::atomic<int> g_registry_size{0};

} // namespace

struct StagingSlot {
    void *host = nullptr;   // pinned
    uint64_t bytes = 0;
    void *event = nullptr;  // last copy out of this slot
    bool busy = false;
};

struct Runtime {
    int device = 0;
    void *upload_stream = nullptr;
    void *compute_stream = nullptr;
    std::vector<StagingSlot> staging = std::vector<StagingSlot>(4);
    size_t next_staging = 0;
    // matvec bounce buffers
    void *host_io = nullptr;
    uint64_t host_io_bytes = 0;
    void *dev_io = nullptr;
    uint64_t dev_io_bytes = 0;
    std::vector<void *> free_events;
    mutable std::mutex mutex;
    struct Range {
        uint64_t bytes;
        bool host_readable; // managed (Weights) vs plain HBM (ExpertCache)
    };
    std::map<uintptr_t, Range> device_ranges;
    fmcuda_device_info dev_info{};

    ~Runtime() {
        if (upload_stream) fmcuda_stream_sync(upload_stream);
        if (compute_stream) fmcuda_stream_sync(compute_stream);
        for (auto &s : staging) {
            if (s.event) fmcuda_event_destroy(s.event);
            if (s.host) fmcuda_host_free(s.host);
        }
        for (void *e : free_events) fmcuda_event_destroy(e);
        if (host_io) fmcuda_host_free(host_io);
        if (dev_io) fmcuda_free(dev_io);
        if (upload_stream) fmcuda_stream_destroy(upload_stream);
        if (compute_stream) fmcuda_stream_destroy(compute_stream);
    }

    void *take_event() {
        if (!free_events.empty()) {
            void *e = free_events.back();
            free_events.pop_back();
            return e;
        }
        void *e = nullptr;
        check(fmcuda_event_create(&e), "fence event");
        return e;
    }

    void ensure_io(uint64_t bytes) {
        if (host_io_bytes < bytes) {
            if (host_io) fmcuda_host_free(host_io);
            host_io = nullptr;
            host_io_bytes = 0;
            check(fmcuda_host_alloc(bytes, &host_io), "matvec host bounce buffer");
            host_io_bytes = bytes;
        }
        if (dev_io_bytes < bytes) {
            if (dev_io) fmcuda_free(dev_io);
            dev_io = nullptr;
            dev_io_bytes = 0;
            check(fmcuda_malloc(bytes, &dev_io), "matvec device bounce buffer");
            dev_io_bytes = bytes;
        }
    }
};

CudaBackend::CudaBackend(fm::BackendConfig config, fm::TraceWriter *trace, int device)
    : fm::Backend(std::move(config), trace), rt_(std::make_shared<Runtime>()) {
    rt_->device = device;
    check(fmcuda_init(device), "CUDA backend initialisation");
    check(fmcuda_device_info_get(device, &rt_->dev_info), "device query");
    check(fmcuda_stream_create(&rt_->upload_stream), "upload stream");
    check(fmcuda_stream_create(&rt_->compute_stream), "compute stream");
    // Backend::matvec must agree with CpuBackend::matvec bit for bit: pick the
    // summation order of the ISA the CPU backend would resolve to
    // (src/kernels.cpp:108-127: scalar on request, else AVX2, never AVX-512
    // in `auto`).
    const fm::KernelIsa isa = fm::resolve_kernel_isa(config_.kernel_isa);
    matvec_order_ = isa == fm::KernelIsa::Scalar ? FM_ORDER_SCALAR
                    : isa == fm::KernelIsa::Avx2Fma ? FM_ORDER_AVX2 : FM_ORDER_ANY;
    if (trace_) {
        fm::Json fields = fm::Json::object();
        fields.set("backend", name());
        fields.set("device", std::string(rt_->dev_info.name));
        fields.set("matvec_order", static_cast<int64_t>(matvec_order_));
        trace_->event("backend_init", std::move(fields));
    }
    std::lock_guard<std::mutex> lock(g_registry_mutex);
    g_registry.push_back(this);
    g_registry_size.store(static_cast<int>(g_registry.size()));
}

CudaBackend::~CudaBackend() {
    {
        std::lock_guard<std::mutex> lock(g_registry_mutex);
        g_registry.erase(std::remove(g_registry.begin(), g_registry.end(), this), g_registry.end());
        g_registry_size.store(static_cast<int>(g_registry.size()));
    }
    for (auto &kv : fence_events_) fmcuda_event_destroy(kv.second);
}

CudaBackend *CudaBackend::owner_of(const void *p, bool *host_readable) {
    if (g_registry_size.load(std::memory_order_relaxed) == 0 || !p) return nullptr;
    std::lock_guard<std::mutex> lock(g_registry_mutex);
    for (CudaBackend *b : g_registry)
        if (b->owns_device_pointer(p, host_readable)) return b;
    return nullptr;
}

fm::DeviceInfo CudaBackend::info() const {
    fm::DeviceInfo info;
    fmcuda_device_info d{};
    if (fmcuda_device_info_get(rt_->device, &d) != FM_STATUS_OK) d = rt_->dev_info;
    info.name = d.name;
    info.backend = "CUDA sm_" + std::to_string(d.cc_major) + std::to_string(d.cc_minor) +
                   "a, " + std::to_string(d.sm_count) + " SMs (freemoe_b200)";
    info.memory_type = "hbm3e";
    info.api_version = "CUDA runtime " + std::to_string(d.runtime_version);
    info.driver_version = "CUDA driver " + std::to_string(d.driver_version);
    info.total_memory_bytes = d.total_memory_bytes;
    info.free_memory_bytes = d.free_memory_bytes;
    info.dedicated_vram_bytes = d.total_memory_bytes;
    info.threads = static_cast<uint32_t>(d.sm_count);
    info.notes = "Weights and expert slots in HBM; attention and norms stay on the CPU. "
                 "No CPU fallback on the device path.";
    return info;
}

std::unique_ptr<fm::DeviceBuffer> CudaBackend::allocate(uint64_t bytes, fm::AllocationTag tag) {
    if (bytes == 0) fm::fail(fm::ErrorCode::INVALID_ARGUMENT, "zero-byte allocation");
    void *ptr = nullptr;
    const bool on_device = device_tag(tag);
    const bool host_readable = tag != fm::AllocationTag::ExpertCache;
    if (on_device) {
        if (host_readable) check(fmcuda_malloc_managed(bytes, &ptr), "HBM allocation");
        else check(fmcuda_malloc(bytes, &ptr), "HBM expert slot allocation");
    } else {
        check(fmcuda_host_alloc(bytes, &ptr), "pinned host allocation");
        std::memset(ptr, 0, static_cast<size_t>(bytes));
    }
    auto buffer = std::make_unique<fm::DeviceBuffer>();
    buffer->data = ptr;
    buffer->bytes = bytes;
    buffer->tag = tag;
    auto tracker = tracker_;
    buffer->allocation_id = tracker->allocate(tag, bytes);
    auto rt = rt_;
    if (on_device) {
        std::lock_guard<std::mutex> lock(rt->mutex);
        rt->device_ranges[reinterpret_cast<uintptr_t>(ptr)] = Runtime::Range{bytes, host_readable};
    }
    buffer->cleanup = [tracker, rt, id = buffer->allocation_id, ptr, on_device]() {
        // The runtime (streams, staging) outlives every buffer it served.
        if (on_device) {
            fmcuda_stream_sync(rt->upload_stream);
            fmcuda_stream_sync(rt->compute_stream);
            {
                std::lock_guard<std::mutex> lock(rt->mutex);
                rt->device_ranges.erase(reinterpret_cast<uintptr_t>(ptr));
            }
            fmcuda_free(ptr);
        } else {
            fmcuda_host_free(ptr);
        }
        tracker->free(id);
    };
    return buffer;
}

bool CudaBackend::owns_device_pointer(const void *p, bool *host_readable) const {
    const uintptr_t a = reinterpret_cast<uintptr_t>(p);
    std::lock_guard<std::mutex> lock(rt_->mutex);
    auto it = rt_->device_ranges.upper_bound(a);
    if (it == rt_->device_ranges.begin()) return false;
    --it;
    if (a >= it->first + it->second.bytes) return false;
    if (host_readable) *host_readable = it->second.host_readable;
    return true;
}

fm::Fence CudaBackend::upload(fm::DeviceBuffer &buffer, const void *src, uint64_t bytes) {
    if (fault_ == fm::BackendFault::TransferFailure)
        fm::fail(fm::ErrorCode::TRANSFER_FAILED, "injected CUDA transfer failure");
    if (fault_ == fm::BackendFault::DeviceLoss)
        fm::fail(fm::ErrorCode::DEVICE_LOSS, "injected CUDA device loss");
    if (!buffer.data || !src || bytes > buffer.bytes)
        fm::fail(fm::ErrorCode::INVALID_ARGUMENT, "bad CUDA upload");
    fm::Fence f;
    f.id = next_fence_++;
    f.ready_at_ms = fm::now_ms();
    void *event = rt_->take_event();
    if (!device_tag(buffer.tag)) {
        // host-resident buffer: a plain copy is the whole transfer
        std::memcpy(buffer.data, src, static_cast<size_t>(bytes));
        check(fmcuda_event_record(event, rt_->upload_stream), "fence record");
    } else {
        // pinned staging ring -> HBM on the upload stream, in chunks
        const uint64_t chunk = 64ull << 20;
        uint64_t done = 0;
        while (done < bytes) {
            StagingSlot &slot = rt_->staging[rt_->next_staging];
            rt_->next_staging = (rt_->next_staging + 1) % rt_->staging.size();
            if (slot.busy) {
                // the previous copy out of this slot must finish before reuse
                check(fmcuda_event_wait(slot.event, 60000), "staging slot reuse");
                slot.busy = false;
            }
            const uint64_t n = std::min(chunk, bytes - done);
            if (slot.bytes < n) {
                if (slot.host) fmcuda_host_free(slot.host);
                slot.host = nullptr;
                slot.bytes = 0;
                check(fmcuda_host_alloc(std::max<uint64_t>(n, 1ull << 20), &slot.host), "staging buffer");
                slot.bytes = std::max<uint64_t>(n, 1ull << 20);
            }
            if (!slot.event) slot.event = rt_->take_event();
            std::memcpy(slot.host, static_cast<const uint8_t *>(src) + done, static_cast<size_t>(n));
            check(fmcuda_upload_async(static_cast<uint8_t *>(buffer.data) + done, slot.host, n,
                                      rt_->upload_stream, slot.event),
                  "host-to-device upload");
            slot.busy = true;
            done += n;
        }
        check(fmcuda_event_record(event, rt_->upload_stream), "fence record");
    }
    fence_events_[f.id] = event;
    if (fault_ == fm::BackendFault::FenceDeferred) {
        f.deferred = true;
        f.ready_at_ms = fm::now_ms() + 3600000ull;
        deferred_fences_.insert(f.id);
        fault_ = fm::BackendFault::None;
    }
    record_operation({"upload", name(), bytes, bytes});
    return f;
}

bool CudaBackend::fence_complete(const fm::Fence &fence) const {
    if (fence.deferred && !ready_fences_.count(fence.id) && fm::now_ms() < fence.ready_at_ms)
        return false;
    auto it = fence_events_.find(fence.id);
    if (it == fence_events_.end()) return true; // retired
    int32_t done = 0;
    check(fmcuda_event_query(it->second, &done), "fence query");
    return done != 0;
}

void CudaBackend::wait_fence(const fm::Fence &fence, uint32_t timeout_ms) {
    if (fault_ == fm::BackendFault::FenceTimeout) {
        fault_ = fm::BackendFault::None;
        fm::fail(fm::ErrorCode::FENCE_TIMEOUT, "injected CUDA fence timeout");
    }
    const uint64_t start = fm::now_ms();
    if (fence.deferred) {
        // an injected deferral completes only after advance_fences()
        while (!ready_fences_.count(fence.id) && fm::now_ms() < fence.ready_at_ms) {
            if (fm::now_ms() - start >= timeout_ms)
                fm::fail(fm::ErrorCode::FENCE_TIMEOUT, "fence " + std::to_string(fence.id) + " timed out");
            std::this_thread::sleep_for(std::chrono::milliseconds(1));
        }
    }
    auto it = fence_events_.find(fence.id);
    if (it == fence_events_.end()) return;
    const uint64_t spent = fm::now_ms() - start;
    const uint32_t left = spent >= timeout_ms ? 0u : static_cast<uint32_t>(timeout_ms - spent);
    int status = fmcuda_event_wait(it->second, left);
    if (status == FM_STATUS_FENCE_TIMEOUT)
        fm::fail(fm::ErrorCode::FENCE_TIMEOUT, "fence " + std::to_string(fence.id) + " timed out");
    check(status, "fence wait");
    rt_->free_events.push_back(it->second);
    fence_events_.erase(it);
}

void CudaBackend::advance_fences() {
    for (uint64_t id : deferred_fences_) ready_fences_.insert(id);
}

void CudaBackend::clear_faults() {
    fault_ = fm::BackendFault::None;
    ready_fences_.clear();
    deferred_fences_.clear();
}

void CudaBackend::matvec(const float *weights, const float *x, float *y, uint32_t out_dim,
                         uint32_t in_dim, const std::string &op_name) {
    if (fault_ == fm::BackendFault::DeviceLoss)
        fm::fail(fm::ErrorCode::DEVICE_LOSS, "injected CUDA device loss");
    if (!weights || !x || !y || out_dim == 0 || in_dim == 0)
        fm::fail(fm::ErrorCode::INVALID_ARGUMENT, "invalid matvec arguments");
    if (!owns_device_pointer(weights))
        fm::fail(fm::ErrorCode::INVALID_ARGUMENT,
                 "matvec weights are not in a buffer of this backend: " + op_name);
    const uint64_t xb = static_cast<uint64_t>(in_dim) * 4, yb = static_cast<uint64_t>(out_dim) * 4;
    const uint64_t xoff = 0, yoff = (xb + 255) & ~uint64_t(255);
    rt_->ensure_io(yoff + yb);
    uint8_t *hio = static_cast<uint8_t *>(rt_->host_io);
    uint8_t *dio = static_cast<uint8_t *>(rt_->dev_io);
    std::memcpy(hio + xoff, x, static_cast<size_t>(xb));
    void *s = rt_->compute_stream;
    // weights may still be in flight on the upload stream
    check(fmcuda_stream_sync(rt_->upload_stream), "upload drain");
    check(fmcuda_upload_async(dio + xoff, hio + xoff, xb, s, nullptr), "matvec input");
    check(fmcuda_matvec_f32(weights, reinterpret_cast<const float *>(dio + xoff),
                            reinterpret_cast<float *>(dio + yoff), out_dim, in_dim, matvec_order_, s),
          "matvec " + op_name);
    check(fmcuda_download(y, dio + yoff, yb, s), "matvec output");
    record_operation({op_name, name(), (static_cast<uint64_t>(out_dim) * in_dim + in_dim) * 4, yb});
}

void CudaBackend::matvec_quant(uint32_t type_id, const uint8_t *weights, const float *x, float *y,
                               uint32_t out_dim, uint32_t in_dim, const std::string &op_name) {
    if (fault_ == fm::BackendFault::DeviceLoss)
        fm::fail(fm::ErrorCode::DEVICE_LOSS, "injected CUDA device loss");
    if (!owns_device_pointer(weights))
        fm::fail(fm::ErrorCode::INVALID_ARGUMENT,
                 "quantised weights are not in a buffer of this backend: " + op_name);
    const uint64_t xb = static_cast<uint64_t>(in_dim) * 4, yb = static_cast<uint64_t>(out_dim) * 4;
    const uint64_t yoff = (xb + 255) & ~uint64_t(255);
    rt_->ensure_io(yoff + yb);
    uint8_t *hio = static_cast<uint8_t *>(rt_->host_io);
    uint8_t *dio = static_cast<uint8_t *>(rt_->dev_io);
    std::memcpy(hio, x, static_cast<size_t>(xb));
    void *s = rt_->compute_stream;
    check(fmcuda_stream_sync(rt_->upload_stream), "upload drain");
    check(fmcuda_upload_async(dio, hio, xb, s, nullptr), "quantised matvec input");
    check(fmcuda_gemv(type_id, weights, dio, FM_X_F32, reinterpret_cast<float *>(dio + yoff), 1,
                      out_dim, in_dim, s),
          "quantised matvec " + op_name);
    check(fmcuda_download(y, dio + yoff, yb, s), "quantised matvec output");
    if (!op_name.empty()) record_operation({op_name, name(), fmcuda_row_bytes(type_id, in_dim) * out_dim + xb, yb});
}

void CudaBackend::download(const fm::DeviceBuffer &buffer, void *dst, uint64_t bytes) {
    if (bytes > buffer.bytes) fm::fail(fm::ErrorCode::INVALID_ARGUMENT, "download past the buffer");
    download_range(dst, buffer.data, bytes);
}

void CudaBackend::download_range(void *dst, const void *src, uint64_t bytes) {
    if (fault_ == fm::BackendFault::DeviceLoss) fm::fail(fm::ErrorCode::DEVICE_LOSS, "injected CUDA device loss");
    check(fmcuda_stream_sync(rt_->upload_stream), "upload drain");
    check(fmcuda_download(dst, src, bytes, rt_->compute_stream), "slot read-back");
    record_control("slot_readback", bytes, bytes, name());
}

void CudaBackend::upload_range(void *dst, const void *src, uint64_t bytes) {
    if (fault_ == fm::BackendFault::DeviceLoss) fm::fail(fm::ErrorCode::DEVICE_LOSS, "injected CUDA device loss");
    check(fmcuda_stream_sync(rt_->upload_stream), "upload drain");
    check(fmcuda_upload_async(dst, src, bytes, rt_->compute_stream, nullptr), "host-to-device copy");
    check(fmcuda_stream_sync(rt_->compute_stream), "host-to-device copy");
}

std::unique_ptr<fm::Backend> make_cuda_backend(const fm::BackendConfig &config, fm::TraceWriter *trace) {
    return std::make_unique<CudaBackend>(config, trace, 0);
}

} // namespace fmcuda
