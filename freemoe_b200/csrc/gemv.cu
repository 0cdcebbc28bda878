// gemv.cu -- K2 entry points: quantised GEMV (gemv_quant / gemm_quant,
// src/kernels.cpp:846-878, :316-345) and the F32 matvec behind
// Backend::matvec (src/backend.cpp:277-290 -> gemv, src/kernels.cpp:470-508).
#include <algorithm>
#include <mutex>
#include <string>
#include <vector>

#include "gemv_kernels.cuh"
#include "gemv_async.cuh"

// Tile shape of the streamed GEMV: MT m-tiles of 16 rows per tile, NW warps
// per CTA splitting K, ring depth P (two matrices: gate/up) or P1 (one).
#ifndef FMB_GEMV_MT
#define FMB_GEMV_MT 2
#endif
#ifndef FMB_GEMV_NW
#define FMB_GEMV_NW 2
#endif
#ifndef FMB_GEMV_P2
#define FMB_GEMV_P2 2
#endif
#ifndef FMB_GEMV_P1
#define FMB_GEMV_P1 4
#endif

namespace fmb {

// ---------------------------------------------------------------------------
// F32 weights: CUDA cores, one warp per row (tolerance-level order).
// ---------------------------------------------------------------------------
template <typename XT>
__global__ void gemv_f32_kernel(const float *__restrict__ w, const XT *__restrict__ x,
                                float *__restrict__ y, uint32_t tokens, uint32_t out_dim,
                                uint32_t in_dim) {
    const uint32_t lane = threadIdx.x & 31;
    const uint32_t warps = gridDim.x * (blockDim.x >> 5);
    for (uint32_t row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); row < out_dim;
         row += warps) {
        const float *wr = w + static_cast<uint64_t>(row) * in_dim;
        for (uint32_t t0 = 0; t0 < tokens; t0 += 8) {
            const uint32_t nt = min(8u, tokens - t0);
            float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
            for (uint32_t k = lane; k < in_dim; k += 32) {
                const float wv = __ldg(wr + k);
#pragma unroll
                for (int t = 0; t < 8; ++t)
                    if (static_cast<uint32_t>(t) < nt)
                        acc[t] = fmaf(wv, load_x<XT>(x + static_cast<uint64_t>(t0 + t) * in_dim + k),
                                      acc[t]);
            }
#pragma unroll
            for (int t = 0; t < 8; ++t) {
                const float s = warp_sum(acc[t]);
                if (lane == 0 && static_cast<uint32_t>(t) < nt)
                    y[static_cast<uint64_t>(t0 + t) * out_dim + row] = s;
            }
        }
    }
}

// Bit-identical to gemv_scalar (src/kernels.cpp:132-140): ascending k, float
// accumulator, multiply then add.  One thread per row.
__global__ void matvec_scalar_order_kernel(const float *__restrict__ w,
                                           const float *__restrict__ x, float *__restrict__ y,
                                           uint32_t out_dim, uint32_t in_dim) {
    const uint32_t row = blockIdx.x * blockDim.x + threadIdx.x;
    if (row >= out_dim) return;
    const float *wr = w + static_cast<uint64_t>(row) * in_dim;
    float acc = 0.0f;
    for (uint32_t k = 0; k < in_dim; ++k) acc = __fadd_rn(acc, __fmul_rn(wr[k], x[k]));
    y[row] = acc;
}

// Bit-identical to gemv_avx2_row (src/kernels.cpp:147-166): lanes 0..7 are
// acc0's chain over k = 16i + l, lanes 8..15 acc1's over k = 16i + 8 + l; a
// trailing group of 8 goes to acc0; then acc0 + acc1, the 4+4 fold, the two
// horizontal adds, and an FMA tail.  Half a warp per row.
__global__ void matvec_avx2_order_kernel(const float *__restrict__ w, const float *__restrict__ x,
                                         float *__restrict__ y, uint32_t out_dim,
                                         uint32_t in_dim) {
    const uint32_t lane = threadIdx.x & 31, hl = lane & 15;
    const uint32_t row = (blockIdx.x * blockDim.x + threadIdx.x) >> 4;
    const bool active = row < out_dim;
    const float *wr = w + static_cast<uint64_t>(active ? row : 0) * in_dim;
    float acc = 0.0f;
    uint32_t k = 0;
    for (; k + 16 <= in_dim; k += 16) acc = __fmaf_rn(wr[k + hl], x[k + hl], acc);
    if (k + 8 <= in_dim) {
        if (hl < 8) acc = __fmaf_rn(wr[k + hl], x[k + hl], acc);
        k += 8;
    }
    // a[l] = acc0[l] + acc1[l]
    const float other = __shfl_down_sync(0xFFFFFFFFu, acc, 8, 16);
    const float a = __fadd_rn(acc, other);
    // s[l] = a[l] + a[l+4], l < 4
    const float a4 = __shfl_down_sync(0xFFFFFFFFu, a, 4, 16);
    const float s = __fadd_rn(a, a4);
    const float s1 = __shfl_down_sync(0xFFFFFFFFu, s, 1, 16);
    const float s2 = __shfl_down_sync(0xFFFFFFFFu, s, 2, 16);
    const float s3 = __shfl_down_sync(0xFFFFFFFFu, s, 3, 16);
    if (active && hl == 0) {
        float total = __fadd_rn(__fadd_rn(s, s1), __fadd_rn(s2, s3));
        for (; k < in_dim; ++k) total = __fmaf_rn(wr[k], x[k], total);
        y[row] = total;
    }
}

// ---------------------------------------------------------------------------
// Internal cached workspace for the x planes of the plain GEMV entry point.
// ---------------------------------------------------------------------------
struct PlaneCache {
    std::mutex mutex;
    void *ptr[64] = {};
    uint64_t bytes[64] = {};
};
PlaneCache g_planes;

int plane_workspace(uint64_t need, void **out) {
    int dev = 0;
    cudaError_t err = cudaGetDevice(&dev);
    if (err != cudaSuccess) return cuda_status(err, "cudaGetDevice");
    if (dev < 0 || dev >= 64) return set_error(FM_STATUS_INVALID_ARGUMENT, "device ordinal too large");
    std::lock_guard<std::mutex> lock(g_planes.mutex);
    if (g_planes.bytes[dev] < need) {
        if (g_planes.ptr[dev]) {
            cudaDeviceSynchronize();
            cudaFree(g_planes.ptr[dev]);
            g_planes.ptr[dev] = nullptr;
            g_planes.bytes[dev] = 0;
        }
        err = cudaMalloc(&g_planes.ptr[dev], need);
        if (err != cudaSuccess) {
            (void)cudaGetLastError();
            return cuda_status(err, "x-plane workspace");
        }
        g_planes.bytes[dev] = need;
    }
    *out = g_planes.ptr[dev];
    return FM_STATUS_OK;
}

inline uint64_t align256(uint64_t v) { return (v + 255) & ~uint64_t(255); }

// Launches the x-plane preparation for `rows` x `k_dim` values.
// fp16 hi (and lo) planes of x in natural element order, for the Q6_K kernel.
template <typename XT>
__global__ void xplanes_natural_kernel(const XT *__restrict__ x, uint64_t n, __half *__restrict__ xh,
                                       __half *__restrict__ xl) {
    const uint64_t i = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x;
    if (i >= n) return;
    const float v = load_x<XT>(x + i);
    const __half h = __float2half_rn(v);
    xh[i] = h;
    if (xl) xl[i] = __float2half_rn(v - __half2float(h));
}

int launch_xplanes_natural(const void *x, int32_t x_dtype, uint32_t rows, uint32_t k_dim, __half *xh, __half *xl,
                           cudaStream_t s) {
    const uint64_t n = static_cast<uint64_t>(rows) * k_dim;
    if (n == 0) return FM_STATUS_OK;
    const unsigned grid = static_cast<unsigned>((n + 255) / 256);
    if (x_dtype == FM_X_BF16)
        xplanes_natural_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>(static_cast<const __nv_bfloat16 *>(x), n, xh, xl);
    else
        xplanes_natural_kernel<float><<<grid, 256, 0, s>>>(static_cast<const float *>(x), n, xh, xl);
    return check_launch("x-plane launch");
}

int launch_xplanes(const void *x, int32_t x_dtype, uint32_t rows, uint32_t k_dim, __half *xh,
                   __half *xl, float *xs, cudaStream_t s);

// The x planes the register-fed kernel of `type_id` reads.
int launch_xplanes_for(uint32_t type_id, const void *x, int32_t x_dtype, uint32_t rows, uint32_t k_dim,
                       __half *xh, __half *xl, float *xs, cudaStream_t s) {
    if (type_id == FM_TYPE_Q6_K) return launch_xplanes_natural(x, x_dtype, rows, k_dim, xh, xl, s);
    return launch_xplanes(x, x_dtype, rows, k_dim, xh, xl, xs, s);
}

int launch_xplanes(const void *x, int32_t x_dtype, uint32_t rows, uint32_t k_dim, __half *xh,
                   __half *xl, float *xs, cudaStream_t s) {
    const uint64_t n = static_cast<uint64_t>(rows) * (k_dim / 32);
    if (n == 0) return FM_STATUS_OK;
    const unsigned grid = static_cast<unsigned>((n + 127) / 128);
    if (x_dtype == FM_X_BF16)
        xplanes_kernel<__nv_bfloat16><<<grid, 128, 0, s>>>(
            static_cast<const __nv_bfloat16 *>(x), rows, k_dim, xh, xl, xs);
    else
        xplanes_kernel<float><<<grid, 128, 0, s>>>(static_cast<const float *>(x), rows, k_dim, xh,
                                                   xl, xs);
    return check_launch("x-plane launch");
}

// Picks the tile shape for a quantised GEMV and launches it.
template <int MODE>
int launch_qgemv(const QGemvParams &prm, int planes, uint32_t grid_y, uint32_t grid_z,
                 cudaStream_t s) {
    const uint32_t rows16 = (prm.out_dim + 15) / 16;
    // Two m-tiles per warp when that still leaves >= 2 CTAs per SM, else one.
    const bool mt2 = rows16 / 2 * grid_z >= 2 * 148;
    dim3 grid;
    grid.y = grid_y;
    grid.z = grid_z;
#define FM_LAUNCH(TYPE, MT, NW, PL)                                                              \
    do {                                                                                         \
        grid.x = (prm.out_dim + 16 * MT - 1) / (16 * MT);                                        \
        qgemv_kernel<TYPE, MT, NW, PL, MODE><<<grid, NW * 32, 0, s>>>(prm);                      \
    } while (0)
    if (prm.type_id == FM_TYPE_Q4_K) {
        if (planes == 1) {
            if (mt2) FM_LAUNCH(FM_TYPE_Q4_K, 2, 4, 1);
            else FM_LAUNCH(FM_TYPE_Q4_K, 1, 8, 1);
        } else {
            if (mt2) FM_LAUNCH(FM_TYPE_Q4_K, 2, 4, 2);
            else FM_LAUNCH(FM_TYPE_Q4_K, 1, 8, 2);
        }
    } else if (prm.type_id == FM_TYPE_Q6_K) {
        if (planes == 1) {
            if (mt2) FM_LAUNCH(FM_TYPE_Q6_K, 2, 4, 1);
            else FM_LAUNCH(FM_TYPE_Q6_K, 1, 8, 1);
        } else {
            if (mt2) FM_LAUNCH(FM_TYPE_Q6_K, 2, 4, 2);
            else FM_LAUNCH(FM_TYPE_Q6_K, 1, 8, 2);
        }
    } else {
        if (planes == 1) {
            if (mt2) FM_LAUNCH(FM_TYPE_Q8_0, 2, 4, 1);
            else FM_LAUNCH(FM_TYPE_Q8_0, 1, 8, 1);
        } else {
            if (mt2) FM_LAUNCH(FM_TYPE_Q8_0, 2, 4, 2);
            else FM_LAUNCH(FM_TYPE_Q8_0, 1, 8, 2);
        }
    }
#undef FM_LAUNCH
    return check_launch("quantised GEMV launch");
}

template int launch_qgemv<GEMV_PLAIN>(const QGemvParams &, int, uint32_t, uint32_t, cudaStream_t);
template int launch_qgemv<GEMV_GATE_UP>(const QGemvParams &, int, uint32_t, uint32_t, cudaStream_t);
template int launch_qgemv<GEMV_DOWN>(const QGemvParams &, int, uint32_t, uint32_t, cudaStream_t);

// Shape checks shared with the MoE block (gemv_quant's own rules,
// src/kernels.cpp:850-858: whole blocks per row).  The register-fed kernel
// additionally needs Q8_0 rows of a multiple of 32 values (whole blocks).
int check_quant_shape(uint32_t type_id, uint32_t in_dim, const char *what) {
    uint32_t bs, bb;
    if (!block_geometry(type_id, &bs, &bb))
        return set_error(FM_STATUS_UNSUPPORTED_QUANTISATION,
                         std::string(what) + ": no GEMV kernel for tensor type " +
                             std::to_string(type_id));
    if (in_dim % bs)
        return set_error(FM_STATUS_SHAPE_MISMATCH,
                         std::string(what) + ": quantised row length is not a whole number of blocks");
    return FM_STATUS_OK;
}

// Quantised rows are read with loads as wide as the type allows: Q4_K with
// 16-byte loads (144-byte blocks keep every row 16-byte aligned), Q8_0 and
// Q6_K with 2- and 4-byte loads (34- and 210-byte blocks).  A matrix whose first
// byte breaks that alignment is refused instead of read misaligned.
int check_quant_alignment(uint32_t type_id, uint64_t byte_offset, const char *what) {
    const uint64_t need = type_id == FM_TYPE_Q4_K ? 16 : (type_id == FM_TYPE_F32 ? 4 : 2);
    if (byte_offset % need)
        return set_error(FM_STATUS_INVALID_ARGUMENT, std::string(what) + ": quantised matrix must start on a " +
                                                          std::to_string(need) + "-byte boundary");
    return FM_STATUS_OK;
}

// The TMA-staged kernel takes rows of whole 256-value K steps whose byte
// length keeps every row 16-byte aligned (bulk copies need 16-byte aligned
// sources); everything on the BASELINE shapes qualifies.
bool staged_shape(uint32_t type_id, uint32_t in_dim) {
    return (type_id == FM_TYPE_Q8_0 || type_id == FM_TYPE_Q4_K) && in_dim % 256 == 0 &&
           row_bytes(type_id, in_dim) % 16 == 0;
}

int xplane_layout(uint32_t type_id) { return type_id == FM_TYPE_Q4_K ? XL_Q4K : XL_Q8; }

int launch_xplanes_staged(const void *x, int32_t x_dtype, uint32_t rows, uint32_t k_dim, int layout,
                          __half *xh, __half *xl, float *xs, cudaStream_t s) {
    const uint64_t n = static_cast<uint64_t>(rows) * (k_dim / 32);
    if (n == 0) return FM_STATUS_OK;
    const unsigned grid = static_cast<unsigned>((n + 127) / 128);
    if (x_dtype == FM_X_BF16)
        xplanes_staged_kernel<__nv_bfloat16><<<grid, 128, 0, s>>>(
            static_cast<const __nv_bfloat16 *>(x), rows, k_dim, layout, xh, xl, xs);
    else
        xplanes_staged_kernel<float><<<grid, 128, 0, s>>>(static_cast<const float *>(x), rows, k_dim,
                                                          layout, xh, xl, xs);
    return check_launch("staged x-plane launch");
}

namespace {
int sm_count() {
    static int n[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return 148;
    if (!n[dev]) {
        if (cudaDeviceGetAttribute(&n[dev], cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || !n[dev])
            n[dev] = 148;
    }
    return n[dev];
}

template <int TYPE, int PL, int MODE, int P>
int launch_async_inst(const QGemvParams &prm, uint32_t tok_tiles, uint32_t experts, cudaStream_t s) {
    constexpr int MT = FMB_GEMV_MT, NW = FMB_GEMV_NW;
    constexpr int NMAT = MODE == GEMV_GATE_UP ? 2 : 1;
    using G = StageGeom<TYPE, MT, NMAT>;
    // rings, then (MoE modes) the per-expert prefix of token tiles
    constexpr size_t ring = static_cast<size_t>(NW) * P * G::BYTES;
    constexpr size_t smem_max = ring + (kMaxGroupExperts + 4) * 4;
    const size_t smem = ring + (MODE == GEMV_PLAIN ? 0 : (static_cast<size_t>(experts) + 4) / 4 * 16);
    auto kern = qgemv_async_kernel<TYPE, MT, NW, PL, MODE, P>;
    static bool configured[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && !configured[dev]) {
        cudaError_t err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               static_cast<int>(smem_max));
        if (err != cudaSuccess) return cuda_status(err, "streamed GEMV shared-memory limit");
        configured[dev] = true;
    }
    int per_sm = 0;
    cudaError_t err = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, NW * 32, smem);
    if (err != cudaSuccess || per_sm < 1) per_sm = 1;
    if (prm.out_dim < static_cast<uint32_t>(G::TILE)) // too few rows for one staged tile
        return launch_qgemv<MODE>(prm, PL, tok_tiles, experts, s);
    const uint32_t row_tiles = (prm.out_dim + G::TILE - 1) / G::TILE;
    uint32_t grid = static_cast<uint32_t>(per_sm * sm_count());
    if (MODE == GEMV_PLAIN) grid = std::min<uint32_t>(grid, row_tiles * tok_tiles);
    if (grid == 0) return FM_STATUS_OK;
    kern<<<grid, NW * 32, smem, s>>>(prm, row_tiles, tok_tiles, experts);
    return check_launch("streamed GEMV launch");
}
} // namespace

// Ring depth P per warp (K steps in flight per warp).
template <int MODE>
int launch_qgemv_stream(const QGemvParams &prm, int planes, uint32_t tok_tiles, uint32_t experts,
                        cudaStream_t s) {
    constexpr int PQ4 = MODE == GEMV_GATE_UP ? FMB_GEMV_P2 : FMB_GEMV_P1;
    if (prm.type_id == FM_TYPE_Q4_K)
        return planes == 1 ? launch_async_inst<FM_TYPE_Q4_K, 1, MODE, PQ4>(prm, tok_tiles, experts, s)
                           : launch_async_inst<FM_TYPE_Q4_K, 2, MODE, PQ4>(prm, tok_tiles, experts, s);
    return planes == 1 ? launch_async_inst<FM_TYPE_Q8_0, 1, MODE, 2>(prm, tok_tiles, experts, s)
                       : launch_async_inst<FM_TYPE_Q8_0, 2, MODE, 2>(prm, tok_tiles, experts, s);
}

template int launch_qgemv_stream<GEMV_PLAIN>(const QGemvParams &, int, uint32_t, uint32_t, cudaStream_t);
template int launch_qgemv_stream<GEMV_GATE_UP>(const QGemvParams &, int, uint32_t, uint32_t, cudaStream_t);
template int launch_qgemv_stream<GEMV_DOWN>(const QGemvParams &, int, uint32_t, uint32_t, cudaStream_t);

} // namespace fmb

using namespace fmb;

extern "C" int fmcuda_gemv(uint32_t type_id, const void *w, const void *x, int32_t x_dtype,
                           float *y, uint32_t tokens, uint32_t out_dim, uint32_t in_dim,
                           void *stream) {
    if (out_dim == 0 || in_dim == 0 || tokens == 0) return FM_STATUS_OK;
    if (!w || !x || !y) return set_error(FM_STATUS_INVALID_ARGUMENT, "invalid quantised GEMV arguments");
    if (x_dtype != FM_X_F32 && x_dtype != FM_X_BF16)
        return set_error(FM_STATUS_INVALID_ARGUMENT, "unknown activation dtype");
    int rc = check_quant_shape(type_id, in_dim, "gemv");
    if (rc) return rc;
    if ((rc = check_quant_alignment(type_id, reinterpret_cast<uintptr_t>(w), "gemv"))) return rc;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (type_id == FM_TYPE_F32) {
        const unsigned grid = min(65535u, (out_dim + 7) / 8);
        if (x_dtype == FM_X_BF16)
            gemv_f32_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>(
                static_cast<const float *>(w), static_cast<const __nv_bfloat16 *>(x), y, tokens,
                out_dim, in_dim);
        else
            gemv_f32_kernel<float><<<grid, 256, 0, s>>>(static_cast<const float *>(w),
                                                        static_cast<const float *>(x), y, tokens,
                                                        out_dim, in_dim);
        return check_launch("f32 GEMV launch");
    }
    const int planes = x_dtype == FM_X_F32 ? 2 : 1;
    const bool staged = staged_shape(type_id, in_dim) && (reinterpret_cast<uintptr_t>(w) & 15u) == 0;
    const uint64_t plane_bytes = align256(static_cast<uint64_t>(tokens) * in_dim * 2);
    const uint64_t sum_bytes = align256(static_cast<uint64_t>(tokens) * (in_dim / 32) * 4);
    void *ws = nullptr;
    rc = plane_workspace(plane_bytes * planes + sum_bytes, &ws);
    if (rc) return rc;
    __half *xh = static_cast<__half *>(ws);
    __half *xl = planes > 1 ? reinterpret_cast<__half *>(static_cast<uint8_t *>(ws) + plane_bytes)
                            : nullptr;
    float *xs = reinterpret_cast<float *>(static_cast<uint8_t *>(ws) + plane_bytes * planes);
    rc = staged ? launch_xplanes_staged(x, x_dtype, tokens, in_dim, xplane_layout(type_id), xh, xl, xs, s)
                : launch_xplanes_for(type_id, x, x_dtype, tokens, in_dim, xh, xl, xs, s);
    if (rc) return rc;
    QGemvParams prm{};
    prm.w = static_cast<const uint8_t *>(w);
    prm.type_id = type_id;
    prm.out_dim = out_dim;
    prm.in_dim = in_dim;
    prm.row_bytes = row_bytes(type_id, in_dim);
    prm.tokens = tokens;
    prm.xh = xh;
    prm.xl = xl;
    prm.xs = xs;
    prm.y = y;
    prm.status = device_status_word();
    if (staged) return launch_qgemv_stream<GEMV_PLAIN>(prm, planes, (tokens + 7) / 8, 1, s);
    return launch_qgemv<GEMV_PLAIN>(prm, planes, (tokens + 7) / 8, 1, s);
}

extern "C" int fmcuda_matvec_f32(const float *w, const float *x, float *y, uint32_t out_dim,
                                 uint32_t in_dim, int32_t order, void *stream) {
    if (!w || !x || !y || out_dim == 0 || in_dim == 0)
        return set_error(FM_STATUS_INVALID_ARGUMENT, "invalid matvec arguments");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (order == FM_ORDER_SCALAR) {
        matvec_scalar_order_kernel<<<(out_dim + 127) / 128, 128, 0, s>>>(w, x, y, out_dim, in_dim);
    } else if (order == FM_ORDER_AVX2) {
        const uint64_t threads = static_cast<uint64_t>(out_dim) * 16;
        matvec_avx2_order_kernel<<<static_cast<unsigned>((threads + 255) / 256), 256, 0, s>>>(
            w, x, y, out_dim, in_dim);
    } else if (order == FM_ORDER_ANY) {
        const unsigned grid = min(65535u, (out_dim + 7) / 8);
        gemv_f32_kernel<float><<<grid, 256, 0, s>>>(w, x, y, 1, out_dim, in_dim);
    } else {
        return set_error(FM_STATUS_INVALID_ARGUMENT, "unknown matvec order");
    }
    return check_launch("f32 matvec launch");
}
