// runtime.cu -- device plumbing behind fm::Backend: allocation, pinned
// staging, streams, fences and the device status word.
//
// Replaces the host-memory behaviour of CpuBackend / VnpuBackend
// (src/backend.cpp:233-299, :405-526) and the GpuBackend placeholder
// (src/backend.cpp:528-571) with real HBM and CUDA events.
#include <chrono>
#include <cstdio>
#include <cstring>
#include <string>
#include <thread>

#include "common.cuh"

namespace fmb {

__device__ int g_device_status = 0;

int *device_status_word() {
    static int *addr[64] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
    if (!addr[dev]) {
        void *p = nullptr;
        if (cudaGetSymbolAddress(&p, g_device_status) != cudaSuccess) return nullptr;
        addr[dev] = static_cast<int *>(p);
    }
    return addr[dev];
}

namespace {
thread_local std::string g_last_error;
}

int set_error(int code, const std::string &msg) {
    g_last_error = msg;
    return code;
}

const char *last_error_cstr() { return g_last_error.c_str(); }

int cuda_status(cudaError_t err, const char *what) {
    std::string msg = std::string(what) + ": " + cudaGetErrorName(err) + " (" +
                      cudaGetErrorString(err) + ")";
    switch (err) {
    case cudaErrorMemoryAllocation:
        return set_error(FM_STATUS_ALLOCATION_FAILED, msg);
    case cudaErrorIllegalAddress:
    case cudaErrorLaunchFailure:
    case cudaErrorIllegalInstruction:
    case cudaErrorMisalignedAddress:
    case cudaErrorHardwareStackError:
    case cudaErrorNoDevice:
    case cudaErrorInvalidDevice:
    case cudaErrorDevicesUnavailable:
    case cudaErrorECCUncorrectable:
    case cudaErrorLaunchTimeout:
        return set_error(FM_STATUS_DEVICE_LOSS, msg);
    default:
        return set_error(FM_STATUS_INTERNAL_ERROR, msg);
    }
}

} // namespace fmb

using namespace fmb;

#define FM_CUDA(call, what)                                                                   \
    do {                                                                                      \
        cudaError_t err__ = (call);                                                           \
        if (err__ != cudaSuccess) return cuda_status(err__, what);                            \
    } while (0)

extern "C" {

const char *fmcuda_last_error(void) { return last_error_cstr(); }

int fmcuda_init(int32_t device) {
    int count = 0;
    cudaError_t err = cudaGetDeviceCount(&count);
    if (err != cudaSuccess || count == 0)
        return set_error(FM_STATUS_DEVICE_LOSS, "no CUDA device is visible");
    if (device < 0 || device >= count)
        return set_error(FM_STATUS_INVALID_ARGUMENT,
                         "device ordinal " + std::to_string(device) + " out of range");
    FM_CUDA(cudaSetDevice(device), "cudaSetDevice");
    cudaDeviceProp prop;
    FM_CUDA(cudaGetDeviceProperties(&prop, device), "cudaGetDeviceProperties");
    if (prop.major != 10)
        return set_error(FM_STATUS_DEVICE_LOSS,
                         std::string("device ") + prop.name +
                             " is not sm_100; this library is built for sm_100a only");
    FM_CUDA(cudaFree(nullptr), "context creation");
    return FM_STATUS_OK;
}

int fmcuda_device_info_get(int32_t device, fmcuda_device_info *out) {
    if (!out) return set_error(FM_STATUS_INVALID_ARGUMENT, "null device info");
    std::memset(out, 0, sizeof(*out));
    cudaDeviceProp prop;
    FM_CUDA(cudaGetDeviceProperties(&prop, device), "cudaGetDeviceProperties");
    std::snprintf(out->name, sizeof(out->name), "%s", prop.name);
    out->sm_count = prop.multiProcessorCount;
    out->cc_major = prop.major;
    out->cc_minor = prop.minor;
    out->l2_bytes = prop.l2CacheSize;
    int prev = 0;
    FM_CUDA(cudaGetDevice(&prev), "cudaGetDevice");
    FM_CUDA(cudaSetDevice(device), "cudaSetDevice");
    size_t free_b = 0, total_b = 0;
    cudaError_t err = cudaMemGetInfo(&free_b, &total_b);
    cudaSetDevice(prev);
    if (err != cudaSuccess) return cuda_status(err, "cudaMemGetInfo");
    out->total_memory_bytes = total_b;
    out->free_memory_bytes = free_b;
    FM_CUDA(cudaDriverGetVersion(&out->driver_version), "cudaDriverGetVersion");
    FM_CUDA(cudaRuntimeGetVersion(&out->runtime_version), "cudaRuntimeGetVersion");
    return FM_STATUS_OK;
}

int fmcuda_malloc(uint64_t bytes, void **ptr) {
    if (!ptr) return set_error(FM_STATUS_INVALID_ARGUMENT, "null output pointer");
    *ptr = nullptr;
    if (bytes == 0) return set_error(FM_STATUS_INVALID_ARGUMENT, "zero-byte allocation");
    void *p = nullptr;
    cudaError_t err = cudaMalloc(&p, bytes);
    if (err != cudaSuccess) {
        (void)cudaGetLastError();
        return cuda_status(err, "cudaMalloc");
    }
    err = cudaMemset(p, 0, bytes);
    if (err != cudaSuccess) {
        cudaFree(p);
        return cuda_status(err, "cudaMemset");
    }
    *ptr = p;
    return FM_STATUS_OK;
}

int fmcuda_malloc_managed(uint64_t bytes, void **ptr) {
    if (!ptr) return set_error(FM_STATUS_INVALID_ARGUMENT, "null output pointer");
    *ptr = nullptr;
    if (bytes == 0) return set_error(FM_STATUS_INVALID_ARGUMENT, "zero-byte allocation");
    int dev = 0;
    FM_CUDA(cudaGetDevice(&dev), "cudaGetDevice");
    void *p = nullptr;
    cudaError_t err = cudaMallocManaged(&p, bytes, cudaMemAttachGlobal);
    if (err != cudaSuccess) {
        (void)cudaGetLastError();
        return cuda_status(err, "cudaMallocManaged");
    }
    cudaMemLocation loc{};
    loc.type = cudaMemLocationTypeDevice;
    loc.id = dev;
    // Advice is a placement hint; a device that declines it still works.
    if (cudaMemAdvise(p, bytes, cudaMemAdviseSetPreferredLocation, loc) != cudaSuccess)
        (void)cudaGetLastError();
    err = cudaMemset(p, 0, bytes);
    if (err == cudaSuccess) err = cudaDeviceSynchronize();
    if (err != cudaSuccess) {
        cudaFree(p);
        return cuda_status(err, "managed zero-fill");
    }
    *ptr = p;
    return FM_STATUS_OK;
}

int fmcuda_free(void *ptr) {
    if (!ptr) return FM_STATUS_OK;
    FM_CUDA(cudaFree(ptr), "cudaFree");
    return FM_STATUS_OK;
}

int fmcuda_host_alloc(uint64_t bytes, void **ptr) {
    if (!ptr || bytes == 0) return set_error(FM_STATUS_INVALID_ARGUMENT, "bad pinned allocation");
    *ptr = nullptr;
    cudaError_t err = cudaHostAlloc(ptr, bytes, cudaHostAllocPortable);
    if (err != cudaSuccess) {
        (void)cudaGetLastError();
        return cuda_status(err, "cudaHostAlloc");
    }
    return FM_STATUS_OK;
}

int fmcuda_host_free(void *ptr) {
    if (!ptr) return FM_STATUS_OK;
    FM_CUDA(cudaFreeHost(ptr), "cudaFreeHost");
    return FM_STATUS_OK;
}

int fmcuda_stream_create(void **stream) {
    if (!stream) return set_error(FM_STATUS_INVALID_ARGUMENT, "null stream pointer");
    cudaStream_t s;
    FM_CUDA(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking), "cudaStreamCreate");
    *stream = s;
    return FM_STATUS_OK;
}

int fmcuda_stream_destroy(void *stream) {
    if (!stream) return FM_STATUS_OK;
    FM_CUDA(cudaStreamDestroy(static_cast<cudaStream_t>(stream)), "cudaStreamDestroy");
    return FM_STATUS_OK;
}

int fmcuda_stream_sync(void *stream) {
    FM_CUDA(cudaStreamSynchronize(static_cast<cudaStream_t>(stream)), "cudaStreamSynchronize");
    return FM_STATUS_OK;
}

int fmcuda_event_create(void **event) {
    if (!event) return set_error(FM_STATUS_INVALID_ARGUMENT, "null event pointer");
    cudaEvent_t e;
    FM_CUDA(cudaEventCreateWithFlags(&e, cudaEventDisableTiming), "cudaEventCreate");
    *event = e;
    return FM_STATUS_OK;
}

int fmcuda_event_create_timing(void **event) {
    if (!event) return set_error(FM_STATUS_INVALID_ARGUMENT, "null event pointer");
    cudaEvent_t e;
    FM_CUDA(cudaEventCreate(&e), "cudaEventCreate");
    *event = e;
    return FM_STATUS_OK;
}

int fmcuda_event_elapsed_ms(void *start, void *end, float *ms) {
    if (!start || !end || !ms) return set_error(FM_STATUS_INVALID_ARGUMENT, "bad elapsed-time query");
    FM_CUDA(cudaEventElapsedTime(ms, static_cast<cudaEvent_t>(start), static_cast<cudaEvent_t>(end)),
            "cudaEventElapsedTime");
    return FM_STATUS_OK;
}

int fmcuda_event_destroy(void *event) {
    if (!event) return FM_STATUS_OK;
    FM_CUDA(cudaEventDestroy(static_cast<cudaEvent_t>(event)), "cudaEventDestroy");
    return FM_STATUS_OK;
}

int fmcuda_event_record(void *event, void *stream) {
    if (!event) return set_error(FM_STATUS_INVALID_ARGUMENT, "null event");
    FM_CUDA(cudaEventRecord(static_cast<cudaEvent_t>(event), static_cast<cudaStream_t>(stream)),
            "cudaEventRecord");
    return FM_STATUS_OK;
}

int fmcuda_upload_async(void *dst, const void *src, uint64_t bytes, void *stream, void *event) {
    if (!dst || !src) return set_error(FM_STATUS_INVALID_ARGUMENT, "bad upload pointers");
    cudaError_t err = cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice,
                                      static_cast<cudaStream_t>(stream));
    if (err != cudaSuccess) {
        (void)cudaGetLastError();
        int code = cuda_status(err, "host-to-device upload");
        return code == FM_STATUS_DEVICE_LOSS ? code : set_error(FM_STATUS_TRANSFER_FAILED,
                                                                fmcuda_last_error());
    }
    if (event) {
        FM_CUDA(cudaEventRecord(static_cast<cudaEvent_t>(event),
                                static_cast<cudaStream_t>(stream)),
                "fence record");
    }
    return FM_STATUS_OK;
}

int fmcuda_event_query(void *event, int32_t *complete) {
    if (!event || !complete) return set_error(FM_STATUS_INVALID_ARGUMENT, "bad fence query");
    cudaError_t err = cudaEventQuery(static_cast<cudaEvent_t>(event));
    if (err == cudaSuccess) {
        *complete = 1;
        return FM_STATUS_OK;
    }
    if (err == cudaErrorNotReady) {
        (void)cudaGetLastError();
        *complete = 0;
        return FM_STATUS_OK;
    }
    return cuda_status(err, "fence query");
}

int fmcuda_event_wait(void *event, uint32_t timeout_ms) {
    // Polled, like Backend::wait_fence (src/backend.cpp:128-135): a fence that
    // does not complete within the deadline is a typed FENCE_TIMEOUT, never an
    // unbounded synchronisation.
    if (!event) return set_error(FM_STATUS_INVALID_ARGUMENT, "null fence");
    const auto start = std::chrono::steady_clock::now();
    for (;;) {
        cudaError_t err = cudaEventQuery(static_cast<cudaEvent_t>(event));
        if (err == cudaSuccess) return FM_STATUS_OK;
        if (err != cudaErrorNotReady) return cuda_status(err, "fence wait");
        (void)cudaGetLastError();
        const auto waited = std::chrono::duration_cast<std::chrono::milliseconds>(
                                std::chrono::steady_clock::now() - start)
                                .count();
        if (static_cast<uint64_t>(waited) >= timeout_ms)
            return set_error(FM_STATUS_FENCE_TIMEOUT,
                             "fence timed out after " + std::to_string(timeout_ms) + " ms");
        std::this_thread::sleep_for(std::chrono::microseconds(50));
    }
}

int fmcuda_download(void *dst, const void *src, uint64_t bytes, void *stream) {
    if (!dst || !src) return set_error(FM_STATUS_INVALID_ARGUMENT, "bad download pointers");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    FM_CUDA(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, s), "device-to-host copy");
    FM_CUDA(cudaStreamSynchronize(s), "device-to-host sync");
    return FM_STATUS_OK;
}

int fmcuda_memset_async(void *dst, int32_t value, uint64_t bytes, void *stream) {
    if (!dst) return set_error(FM_STATUS_INVALID_ARGUMENT, "null memset target");
    FM_CUDA(cudaMemsetAsync(dst, value, bytes, static_cast<cudaStream_t>(stream)), "memset");
    return FM_STATUS_OK;
}

int fmcuda_device_status(int32_t clear, int32_t *status) {
    if (!status) return set_error(FM_STATUS_INVALID_ARGUMENT, "null status pointer");
    FM_CUDA(cudaDeviceSynchronize(), "device synchronise");
    int v = 0;
    FM_CUDA(cudaMemcpyFromSymbol(&v, g_device_status, sizeof(int)), "status read");
    if (clear) {
        int zero = 0;
        FM_CUDA(cudaMemcpyToSymbol(g_device_status, &zero, sizeof(int)), "status clear");
    }
    *status = v;
    return FM_STATUS_OK;
}

uint64_t fmcuda_row_bytes(uint32_t type_id, uint32_t in_dim) { return row_bytes(type_id, in_dim); }

} // extern "C"
