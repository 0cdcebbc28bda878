// dequant.cu -- K1: block decoding (bit-exact) and the synthetic-weight encoder.
//
// K1 is dequantize_tensor_region (src/quant.cpp:723-732) on the device: Q8_0
// (src/quant.cpp:223-228) and Q4_K (src/quant.cpp:297-318).  The decoded
// values are bit-identical to the reference: the fp16 scale conversion is
// exact, d*sc and dmin*m are exact products (11-bit x 6-bit significands), and
// d1*q is exact (17-bit x 4-bit), so `d1*q - m1` rounds once exactly as the
// reference's mul-then-sub does.  The explicit __fmul_rn/__fsub_rn keep nvcc
// from contracting anyway.
#include "common.cuh"

namespace fmb {

// 8 threads per Q8_0 block, 4 values each: a warp writes 4 whole blocks.
__global__ void dequant_q8_0_kernel(const uint8_t *__restrict__ src, float *__restrict__ dst,
                                    uint64_t n_blocks) {
    const uint64_t tid = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x;
    const uint64_t blk = tid >> 3;
    if (blk >= n_blocks) return;
    const int part = tid & 7;
    const uint8_t *b = src + blk * 34;
    const uint16_t dh = static_cast<uint16_t>(b[0] | (b[1] << 8));
    const float d = fp16_bits_to_f32(dh);
    const int8_t *q = reinterpret_cast<const int8_t *>(b + 2 + 4 * part);
    float4 out;
    out.x = __fmul_rn(d, static_cast<float>(q[0]));
    out.y = __fmul_rn(d, static_cast<float>(q[1]));
    out.z = __fmul_rn(d, static_cast<float>(q[2]));
    out.w = __fmul_rn(d, static_cast<float>(q[3]));
    reinterpret_cast<float4 *>(dst + blk * 32)[part] = out;
}

// 32 threads per Q4_K block, 8 values each.
__global__ void dequant_q4_k_kernel(const uint8_t *__restrict__ src, float *__restrict__ dst,
                                    uint64_t n_blocks) {
    const uint64_t tid = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x;
    const uint64_t blk = tid >> 5;
    if (blk >= n_blocks) return;
    const int l = tid & 31;
    const uint8_t *b = src + blk * 144;
    const float d = fp16_bits_to_f32(static_cast<uint16_t>(b[0] | (b[1] << 8)));
    const float dmin = fp16_bits_to_f32(static_cast<uint16_t>(b[2] | (b[3] << 8)));
    const int g = l >> 3;          // 64-value group
    const int p = (l & 7) * 8;     // position inside the group
    const bool hi = p >= 32;
    const int j = 2 * g + (hi ? 1 : 0);
    uint32_t sc, mn;
    q4k_scale_min(j, b + 4, sc, mn);
    const float d1 = __fmul_rn(d, static_cast<float>(sc));
    const float m1 = __fmul_rn(dmin, static_cast<float>(mn));
    const uint8_t *qs = b + 16 + 32 * g + (hi ? p - 32 : p);
    float v[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const uint32_t q = hi ? (qs[i] >> 4) : (qs[i] & 0x0Fu);
        v[i] = __fsub_rn(__fmul_rn(d1, static_cast<float>(q)), m1);
    }
    float4 *o = reinterpret_cast<float4 *>(dst + blk * 256 + 64 * g + p);
    o[0] = make_float4(v[0], v[1], v[2], v[3]);
    o[1] = make_float4(v[4], v[5], v[6], v[7]);
}

// ---------------------------------------------------------------------------
// Synthetic weights: counter-based Gaussian draws, encoded on the device.
// ---------------------------------------------------------------------------

__device__ __forceinline__ uint64_t mix64(uint64_t z) {
    // splitmix64 finaliser
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

__device__ __forceinline__ float gauss(uint64_t seed, uint64_t i) {
    const uint64_t h = mix64(seed ^ mix64(i));
    const float u1 = (static_cast<float>(h >> 40) + 0.5f) * (1.0f / 16777216.0f);
    const float u2 = static_cast<float>((h >> 8) & 0xFFFFFFu) * (1.0f / 16777216.0f);
    return sqrtf(-2.0f * logf(u1)) * cospif(2.0f * u2);
}

__device__ __forceinline__ uint16_t f32_to_fp16_bits(float f) {
    return __half_as_ushort(__float2half_rn(f));
}

__global__ void synth_f32_kernel(float *dst, uint64_t n, uint64_t seed, float std) {
    for (uint64_t i = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<uint64_t>(gridDim.x) * blockDim.x)
        dst[i] = std * gauss(seed, i);
}

// One thread per Q8_0 block: amax/127 scale, round-to-nearest codes.
__global__ void synth_q8_0_kernel(uint8_t *dst, uint64_t n_blocks, uint64_t seed, float std) {
    for (uint64_t blk = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x;
         blk < n_blocks; blk += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
        float v[32];
        float amax = 0.0f;
#pragma unroll
        for (int j = 0; j < 32; ++j) {
            v[j] = std * gauss(seed, blk * 32 + j);
            amax = fmaxf(amax, fabsf(v[j]));
        }
        const uint16_t dh = f32_to_fp16_bits(amax / 127.0f);
        const float dd = fp16_bits_to_f32(dh);
        const float id = dd != 0.0f ? 1.0f / dd : 0.0f;
        uint8_t *b = dst + blk * 34;
        b[0] = static_cast<uint8_t>(dh & 0xFF);
        b[1] = static_cast<uint8_t>(dh >> 8);
#pragma unroll
        for (int j = 0; j < 32; ++j) {
            const float q = fminf(127.0f, fmaxf(-127.0f, rintf(v[j] * id)));
            b[2 + j] = static_cast<uint8_t>(static_cast<int8_t>(q));
        }
    }
}

// One thread per Q6_K block: a scale per 16 values (int8, relative to the fp16
// block scale d), codes q + 32 in six bits packed as src/quant.cpp:347-372 reads them.
__global__ void synth_q6_k_kernel(uint8_t *dst, uint64_t n_blocks, uint64_t seed, float std) {
    for (uint64_t blk = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x;
         blk < n_blocks; blk += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
        float gs[16];
        float smax = 0.0f;
        for (int g = 0; g < 16; ++g) {
            float amax = 0.0f;
            for (int j = 0; j < 16; ++j) amax = fmaxf(amax, fabsf(std * gauss(seed, blk * 256 + 16 * g + j)));
            gs[g] = amax / 31.0f;
            smax = fmaxf(smax, gs[g]);
        }
        const uint16_t dh = f32_to_fp16_bits(smax / 127.0f);
        const float d = fp16_bits_to_f32(dh);
        uint8_t *b = dst + blk * 210;
        int8_t sc[16];
        for (int g = 0; g < 16; ++g) {
            const float r = d != 0.0f ? rintf(gs[g] / d) : 0.0f;
            sc[g] = static_cast<int8_t>(fminf(127.0f, fmaxf(1.0f, r)));
            b[192 + g] = static_cast<uint8_t>(sc[g]);
        }
        b[208] = static_cast<uint8_t>(dh & 0xFF);
        b[209] = static_cast<uint8_t>(dh >> 8);
        for (int h = 0; h < 2; ++h)
            for (int l = 0; l < 32; ++l) {
                int q[4];
                for (int i = 0; i < 4; ++i) {
                    const int v = 128 * h + l + 32 * i;
                    const float step = d * static_cast<float>(sc[v / 16]);
                    const float x = std * gauss(seed, blk * 256 + v);
                    q[i] = static_cast<int>(fminf(31.0f, fmaxf(-32.0f, step != 0.0f ? rintf(x / step) : 0.0f))) + 32;
                }
                b[64 * h + l] = static_cast<uint8_t>((q[0] & 0x0F) | ((q[2] & 0x0F) << 4));
                b[64 * h + l + 32] = static_cast<uint8_t>((q[1] & 0x0F) | ((q[3] & 0x0F) << 4));
                b[128 + 32 * h + l] =
                    static_cast<uint8_t>((q[0] >> 4) | ((q[1] >> 4) << 2) | ((q[2] >> 4) << 4) | ((q[3] >> 4) << 6));
            }
    }
}

// One thread per Q4_K block: per-sub-block affine fit, 6-bit scales and mins
// relative to the fp16 super-block scale and min.
__global__ void synth_q4_k_kernel(uint8_t *dst, uint64_t n_blocks, uint64_t seed, float std) {
    for (uint64_t blk = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x;
         blk < n_blocks; blk += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
        float scale[8], minv[8], max_scale = 0.0f, max_min = 0.0f;
        for (int j = 0; j < 8; ++j) {
            float lo = 3.0e38f, hi = -3.0e38f;
            for (int l = 0; l < 32; ++l) {
                const float x = std * gauss(seed, blk * 256 + 32 * j + l);
                lo = fminf(lo, x);
                hi = fmaxf(hi, x);
            }
            lo = fminf(lo, 0.0f);
            scale[j] = (hi - lo) / 15.0f;
            minv[j] = -lo;
            max_scale = fmaxf(max_scale, scale[j]);
            max_min = fmaxf(max_min, minv[j]);
        }
        const uint16_t dh = f32_to_fp16_bits(max_scale / 63.0f);
        const uint16_t mh = f32_to_fp16_bits(max_min / 63.0f);
        const float d = fp16_bits_to_f32(dh), dmin = fp16_bits_to_f32(mh);
        uint32_t sc[8], mn[8];
        for (int j = 0; j < 8; ++j) {
            const float s = d > 0.0f ? rintf(scale[j] / d) : 0.0f;
            const float m = dmin > 0.0f ? rintf(minv[j] / dmin) : 0.0f;
            sc[j] = static_cast<uint32_t>(fminf(63.0f, fmaxf(0.0f, s)));
            mn[j] = static_cast<uint32_t>(fminf(63.0f, fmaxf(0.0f, m)));
        }
        uint8_t *b = dst + blk * 144;
        b[0] = static_cast<uint8_t>(dh & 0xFF);
        b[1] = static_cast<uint8_t>(dh >> 8);
        b[2] = static_cast<uint8_t>(mh & 0xFF);
        b[3] = static_cast<uint8_t>(mh >> 8);
        for (int j = 0; j < 4; ++j) {
            b[4 + j] = static_cast<uint8_t>((sc[j] & 63) | ((sc[j + 4] >> 4) << 6));
            b[8 + j] = static_cast<uint8_t>((mn[j] & 63) | ((mn[j + 4] >> 4) << 6));
            b[12 + j] = static_cast<uint8_t>((sc[j + 4] & 0x0F) | ((mn[j + 4] & 0x0F) << 4));
        }
        for (int g = 0; g < 4; ++g) {
            uint8_t q[32];
            for (int half = 0; half < 2; ++half) {
                const int j = 2 * g + half;
                const float D = d * static_cast<float>(sc[j]);
                const float M = dmin * static_cast<float>(mn[j]);
                for (int l = 0; l < 32; ++l) {
                    const float x = std * gauss(seed, blk * 256 + 32 * j + l);
                    const float qf = D > 0.0f ? rintf((x + M) / D) : 0.0f;
                    const uint32_t qi = static_cast<uint32_t>(fminf(15.0f, fmaxf(0.0f, qf)));
                    if (half == 0) q[l] = static_cast<uint8_t>(qi);
                    else q[l] = static_cast<uint8_t>(q[l] | (qi << 4));
                }
            }
            for (int l = 0; l < 32; ++l) b[16 + 32 * g + l] = q[l];
        }
    }
}

} // namespace fmb

using namespace fmb;

// 32 threads per Q6_K block (src/quant.cpp:347-372): thread l of the block
// writes y[l], y[l+32], y[l+64], y[l+96] of both 128-value halves,
// y = (d * scale) * q with q = 6-bit code - 32, two float roundings as there.
__global__ void dequant_q6_k_kernel(const uint8_t *__restrict__ src, float *__restrict__ dst,
                                    uint64_t n_blocks) {
    const uint64_t tid = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x;
    const uint64_t blk = tid >> 5;
    if (blk >= n_blocks) return;
    const int l = tid & 31;
    const uint8_t *b = src + blk * 210;
    const float d = fp16_bits_to_f32(static_cast<uint16_t>(b[208] | (b[209] << 8)));
    const int is = l / 16;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        const uint8_t *ql = b + 64 * h, *qh = b + 128 + 32 * h;
        const int8_t *sc = reinterpret_cast<const int8_t *>(b + 192 + 8 * h);
        const int q1 = static_cast<int>((ql[l] & 0x0F) | (((qh[l] >> 0) & 3) << 4)) - 32;
        const int q2 = static_cast<int>((ql[l + 32] & 0x0F) | (((qh[l] >> 2) & 3) << 4)) - 32;
        const int q3 = static_cast<int>((ql[l] >> 4) | (((qh[l] >> 4) & 3) << 4)) - 32;
        const int q4 = static_cast<int>((ql[l + 32] >> 4) | (((qh[l] >> 6) & 3) << 4)) - 32;
        float *y = dst + blk * 256 + 128 * h;
        y[l] = __fmul_rn(__fmul_rn(d, static_cast<float>(sc[is])), static_cast<float>(q1));
        y[l + 32] = __fmul_rn(__fmul_rn(d, static_cast<float>(sc[is + 2])), static_cast<float>(q2));
        y[l + 64] = __fmul_rn(__fmul_rn(d, static_cast<float>(sc[is + 4])), static_cast<float>(q3));
        y[l + 96] = __fmul_rn(__fmul_rn(d, static_cast<float>(sc[is + 6])), static_cast<float>(q4));
    }
}

extern "C" int fmcuda_dequant(uint32_t type_id, const void *src, float *dst, uint64_t n_elems,
                              void *stream) {
    uint32_t bs, bb;
    if (!block_geometry(type_id, &bs, &bb))
        return set_error(FM_STATUS_UNSUPPORTED_QUANTISATION,
                         "no block decoder for tensor type " + std::to_string(type_id));
    if (n_elems % bs)
        return set_error(FM_STATUS_SHAPE_MISMATCH,
                         "region is not a whole number of quantisation blocks");
    if (n_elems == 0) return FM_STATUS_OK;
    if (!src || !dst) return set_error(FM_STATUS_INVALID_ARGUMENT, "null dequant pointer");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const uint64_t n_blocks = n_elems / bs;
    if (type_id == FM_TYPE_F32) {
        cudaError_t err = cudaMemcpyAsync(dst, src, n_elems * 4, cudaMemcpyDeviceToDevice, s);
        if (err != cudaSuccess) return cuda_status(err, "f32 copy");
        return FM_STATUS_OK;
    }
    const int threads = 256;
    if (type_id == FM_TYPE_Q8_0) {
        const uint64_t total = n_blocks * 8;
        dequant_q8_0_kernel<<<static_cast<unsigned>((total + threads - 1) / threads), threads, 0,
                              s>>>(static_cast<const uint8_t *>(src), dst, n_blocks);
    } else if (type_id == FM_TYPE_Q6_K) {
        const uint64_t total = n_blocks * 32;
        dequant_q6_k_kernel<<<static_cast<unsigned>((total + threads - 1) / threads), threads, 0,
                              s>>>(static_cast<const uint8_t *>(src), dst, n_blocks);
    } else {
        const uint64_t total = n_blocks * 32;
        dequant_q4_k_kernel<<<static_cast<unsigned>((total + threads - 1) / threads), threads, 0,
                              s>>>(static_cast<const uint8_t *>(src), dst, n_blocks);
    }
    return check_launch("dequant launch");
}

extern "C" int fmcuda_synth_weights(uint32_t type_id, void *dst, uint64_t rows, uint32_t cols,
                                    uint64_t seed, float std, void *stream) {
    uint32_t bs, bb;
    if (!block_geometry(type_id, &bs, &bb))
        return set_error(FM_STATUS_UNSUPPORTED_QUANTISATION, "unsupported synthetic type");
    if (cols % bs) return set_error(FM_STATUS_SHAPE_MISMATCH, "columns not whole blocks");
    if (!dst) return set_error(FM_STATUS_INVALID_ARGUMENT, "null synthetic target");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const uint64_t n = rows * static_cast<uint64_t>(cols);
    int sms = 148;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, 0);
    const unsigned grid = static_cast<unsigned>(sms) * 8;
    if (type_id == FM_TYPE_F32)
        synth_f32_kernel<<<grid, 256, 0, s>>>(static_cast<float *>(dst), n, seed, std);
    else if (type_id == FM_TYPE_Q8_0)
        synth_q8_0_kernel<<<grid, 128, 0, s>>>(static_cast<uint8_t *>(dst), n / 32, seed, std);
    else if (type_id == FM_TYPE_Q6_K)
        synth_q6_k_kernel<<<grid, 128, 0, s>>>(static_cast<uint8_t *>(dst), n / 256, seed, std);
    else
        synth_q4_k_kernel<<<grid, 128, 0, s>>>(static_cast<uint8_t *>(dst), n / 256, seed, std);
    return check_launch("synthetic weights launch");
}
