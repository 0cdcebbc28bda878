// engine_hooks.cpp -- link-time stand-in for the engine change that moves the
// quantised expert path and the slot read-back onto the device.
//
// FreeMoe's unchanged engine runs every quantised GEMV on the CPU, straight on
// the slot pointer (Engine::matvec_view, src/engine.cpp:358-367, then labels
// the operation "cpu-quant"), and reads expert slots back with a host memcpy
// for the checksum (ResidencyManager::load_slot, src/residency.cpp:703-714).
// With expert slots in plain HBM neither can run on the host.  A maintainer
// makes the two-line engine change shown in the integration notes
// (Backend::matvec_quant / Backend::download virtuals).  Without editing the
// reference's sources, the same routing is done here at link time
// (-Wl,--wrap on three symbols of the reference objects):
//   fm::gemv_quant        weights in a CudaBackend buffer -> the device GEMV
//                         (CudaBackend::matvec_quant); any other pointer -> the
//                         reference's own CPU kernel, unchanged;
//   fm::Backend::record_control
//                         the "cpu-quant" record of a GEMV that ran on the
//                         device is logged as an operation of the CUDA backend;
//   memcpy                a copy out of (or into) plain-HBM slot memory is a
//                         device copy (CudaBackend::download_range /
//                         upload_range); every other copy is the C library's.
#include <cstddef>
#include <cstdint>
#include <string>

#include "cuda_backend.hpp"
#include "fm/kernels.hpp"

namespace {
// set by the GEMV hook, consumed by the record that Engine::matvec_view
// writes right after the GEMV returns (same thread)
thread_local bool t_quant_ran_on_device = false;
} // namespace

extern "C" {

void __real__ZN2fm10gemv_quantERKNS_12KernelConfigEjPKhPKfPfjj(const fm::KernelConfig &config, uint32_t type_id,
                                                               const uint8_t *weights, const float *x, float *y,
                                                               uint32_t out_dim, uint32_t in_dim);

void __wrap__ZN2fm10gemv_quantERKNS_12KernelConfigEjPKhPKfPfjj(const fm::KernelConfig &config, uint32_t type_id,
                                                               const uint8_t *weights, const float *x, float *y,
                                                               uint32_t out_dim, uint32_t in_dim) {
    if (fmcuda::CudaBackend *b = fmcuda::CudaBackend::owner_of(weights)) {
        b->matvec_quant(type_id, weights, x, y, out_dim, in_dim, std::string());
        t_quant_ran_on_device = true;
        return;
    }
    __real__ZN2fm10gemv_quantERKNS_12KernelConfigEjPKhPKfPfjj(config, type_id, weights, x, y, out_dim, in_dim);
}

void __real__ZN2fm7Backend14record_controlERKNSt7__cxx1112basic_stringIcSt11char_traitsIcESaIcEEEmmS8_(
    fm::Backend *self, const std::string &name, uint64_t input_bytes, uint64_t output_bytes,
    const std::string &backend);

void __wrap__ZN2fm7Backend14record_controlERKNSt7__cxx1112basic_stringIcSt11char_traitsIcESaIcEEEmmS8_(
    fm::Backend *self, const std::string &name, uint64_t input_bytes, uint64_t output_bytes,
    const std::string &backend) {
    if (t_quant_ran_on_device && backend == "cpu-quant") {
        t_quant_ran_on_device = false;
        self->record_operation({name, self->name(), input_bytes, output_bytes});
        return;
    }
    __real__ZN2fm7Backend14record_controlERKNSt7__cxx1112basic_stringIcSt11char_traitsIcESaIcEEEmmS8_(
        self, name, input_bytes, output_bytes, backend);
}

void *__real_memcpy(void *dst, const void *src, size_t n);

void *__wrap_memcpy(void *dst, const void *src, size_t n) {
    bool host_readable = true;
    if (fmcuda::CudaBackend *b = fmcuda::CudaBackend::owner_of(src, &host_readable); b && !host_readable) {
        b->download_range(dst, src, n);
        return dst;
    }
    host_readable = true;
    if (fmcuda::CudaBackend *b = fmcuda::CudaBackend::owner_of(dst, &host_readable); b && !host_readable) {
        b->upload_range(dst, src, n);
        return dst;
    }
    return __real_memcpy(dst, src, n);
}

} // extern "C"
