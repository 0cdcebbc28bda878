// common.cuh -- shared definitions for the freemoe_b200 sm_100a kernels.
//
// Status codes returned across the C ABI are the ordinal values of the
// reference's fm::ErrorCode (include/fm/common.hpp:27-57), so the C++ backend
// adapter turns a non-zero status straight into fm::fail(code, message).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

#include "freemoe_b200.h"

namespace fmb {

// Records `msg` as this thread's last error and returns `code`.
int set_error(int code, const std::string &msg);
// Maps a CUDA error to a status: allocation failures to ALLOCATION_FAILED,
// sticky context errors to DEVICE_LOSS, everything else to INTERNAL_ERROR.
int cuda_status(cudaError_t err, const char *what);

// Checks the launch that just happened on the current thread.
inline int check_launch(const char *what) {
    cudaError_t err = cudaPeekAtLastError();
    if (err != cudaSuccess) {
        (void)cudaGetLastError();
        return cuda_status(err, what);
    }
    return FM_STATUS_OK;
}

// Geometry of the GGUF block types on the path (src/gguf.cpp:58-106).
inline bool block_geometry(uint32_t type_id, uint32_t *bs, uint32_t *bb) {
    switch (type_id) {
    case FM_TYPE_F32: *bs = 1; *bb = 4; return true;
    case FM_TYPE_Q8_0: *bs = 32; *bb = 34; return true;
    case FM_TYPE_Q4_K: *bs = 256; *bb = 144; return true;
    case FM_TYPE_Q6_K: *bs = 256; *bb = 210; return true;
    default: return false;
    }
}

inline uint64_t row_bytes(uint32_t type_id, uint32_t in_dim) {
    uint32_t bs, bb;
    if (!block_geometry(type_id, &bs, &bb) || in_dim % bs) return 0;
    return static_cast<uint64_t>(in_dim / bs) * bb;
}

// Device-side status word (one per device, defined in runtime.cu): kernels
// that detect a data error (a non-finite router logit, an unresident expert)
// record the first error code there instead of trapping; fmcuda_device_status()
// reads and clears it.  Kernels receive its address as an argument.
int *device_status_word();

__device__ __forceinline__ void raise_device_status(int *status, int code) {
    if (status) atomicCAS(status, 0, code);
}

// ---------------------------------------------------------------------------
// Block decoding helpers (bit-exact with src/quant.cpp).
// ---------------------------------------------------------------------------

// binary16 -> binary32; the hardware conversion is exact, subnormals included.
__device__ __forceinline__ float fp16_bits_to_f32(uint16_t h) {
    return __half2float(__ushort_as_half(h));
}

// Six-bit scale and min of sub-block j of a Q4_K block (src/quant.cpp:63-71).
__device__ __forceinline__ void q4k_scale_min(int j, const uint8_t *s, uint32_t &sc,
                                              uint32_t &mn) {
    if (j < 4) {
        sc = s[j] & 63u;
        mn = s[j + 4] & 63u;
    } else {
        sc = (s[j + 4] & 0x0Fu) | ((s[j - 4] >> 6) << 4);
        mn = (s[j + 4] >> 4) | ((s[j] >> 6) << 4);
    }
}

// Same unpacking from the 12 scale bytes held as three little-endian words.
__device__ __forceinline__ void q4k_scale_min_w(int j, uint32_t s0, uint32_t s1, uint32_t s2,
                                                uint32_t &sc, uint32_t &mn) {
    // s0 = bytes 0..3, s1 = bytes 4..7, s2 = bytes 8..11
    if (j < 4) {
        sc = (s0 >> (8 * j)) & 63u;
        mn = (s1 >> (8 * j)) & 63u;
    } else {
        const int i = j - 4;
        const uint32_t b_hi = (s2 >> (8 * i)) & 0xFFu;  // byte j+4
        const uint32_t b_lo = (s0 >> (8 * i)) & 0xFFu;  // byte j-4
        const uint32_t b_mid = (s1 >> (8 * i)) & 0xFFu; // byte j
        sc = (b_hi & 0x0Fu) | ((b_lo >> 6) << 4);
        mn = (b_hi >> 4) | ((b_mid >> 6) << 4);
    }
}

__device__ __forceinline__ float bf16_bits_to_f32(uint16_t h) {
    return __uint_as_float(static_cast<uint32_t>(h) << 16);
}

// Activation element load for either input dtype.
template <typename XT> __device__ __forceinline__ float load_x(const XT *p);
template <> __device__ __forceinline__ float load_x<float>(const float *p) { return __ldg(p); }
template <> __device__ __forceinline__ float load_x<__nv_bfloat16>(const __nv_bfloat16 *p) {
    return __bfloat162float(*p);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
    return v;
}

} // namespace fmb
