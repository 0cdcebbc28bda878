// gemv_core.cuh -- fused dequant + tensor-core GEMV tiles for GGUF Q4_K / Q8_0.
//
// Replaces the per-row CPU kernels row_dot_q4_k_avx2 / row_dot_q8_0_avx2
// (src/kernels.cpp:720-771, :639-653) and the fused scalar path (:574-590).
//
// Data flow per warp: a tile of 16*MT weight rows x 8 tokens, over the
// quantisation blocks of the warp's K slice.  Weights stay in their stored
// GGUF bytes (the residency slot holds the file's bytes, checksummed); the
// codes are unpacked in registers straight into mma.sync m16n8k16 A
// fragments, and x comes from "x planes" prepared once per call:
//
//   xh   fp16 copy of x, each group of 4 stored as (x0, x2, x1, x3) so that a
//        thread's 8-byte load is exactly its B fragment (the k order inside a
//        fragment is free as long as A and B use the same one);
//   xl   fp16 residual x - xh (only for f32 inputs: x = xh + xl to 2^-22);
//   xs   f32 sums of x over each 32-value sub-block.
//
// Exactness of the unpacking.  A code q masked in place is read as the fp16
// bit pattern q, i.e. the subnormal q * 2^-24: exact, and one AND with a single
// immediate mask per pair of codes (no magic-exponent OR, so no second constant
// has to live in a register).  The tensor cores take subnormal fp16 operands
// exactly.
//   Q4_K  one HMUL2 by (sc, sc) gives sc*q * 2^-24 exactly (sc*q <= 945 stays
//         on the subnormal grid), so the sub-block scale is applied before the
//         MMA and one accumulator spans the whole 256-value block; high
//         nibbles are masked in place (16 q * 2^-24) and use (sc/16, sc/16).
//         The mins enter through one more MMA of the 6-bit mins against the
//         sub-block sums (split into two fp16 planes).  Per block:
//         y += (2^24 d) * acc - dmin * acc_min, the same algebra as
//         row_dot_q4_k_avx2 (src/kernels.cpp:759-762).
//   Q8_0  (q ^ 0x80) is 128 + q; PRMT with zero bytes makes it the subnormal
//         (128 + q) * 2^-24; per block y += (2^24 d) * acc - 128 d * X.
// All products are exact in the tensor core's fp32 accumulation; the result
// differs from the reference only by summation order.
#pragma once

#include "common.cuh"

namespace fmb {

// ---- PTX wrappers ---------------------------------------------------------

// Not volatile: the MMA has no side effects, and leaving the compiler free to
// interleave independent accumulator chains hides the MMA latency.
__device__ __forceinline__ void mma_f16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                        uint32_t a3, uint32_t b0, uint32_t b1) {
    asm(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%0,%1,%2,%3};\n"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// D = A * B (accumulator starts from zero, no C registers to clear).
__device__ __forceinline__ void mma_f16_zc(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                           uint32_t b0, uint32_t b1) {
    asm(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%10,%10,%10,%10};\n"
        : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "f"(0.0f));
}

__device__ __forceinline__ uint32_t hfma2_u32(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t d;
    asm("fma.rn.f16x2 %0, %1, %2, %3;\n" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

__device__ __forceinline__ uint32_t hsub2_u32(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("sub.rn.f16x2 %0, %1, %2;\n" : "=r"(d) : "r"(a), "r"(b));
    return d;
}

__device__ __forceinline__ uint32_t hmul2_u32(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("mul.rn.f16x2 %0, %1, %2;\n" : "=r"(d) : "r"(a), "r"(b));
    return d;
}

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
    uint32_t d;
    asm("prmt.b32 %0, %1, %2, %3;\n" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
    return d;
}

__device__ __forceinline__ uint32_t lop_and_or(uint32_t a, uint32_t mask, uint32_t orv) {
    return (a & mask) | orv;
}

__device__ __forceinline__ uint4 ldg_nc_v4(const void *p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

__device__ __forceinline__ uint32_t ldg_nc_u32(const void *p) {
    uint32_t v;
    asm volatile("ld.global.nc.L1::no_allocate.u32 %0, [%1];\n" : "=r"(v) : "l"(p));
    return v;
}

__device__ __forceinline__ uint32_t ldg_nc_u16(const void *p) {
    unsigned short v;
    asm volatile("ld.global.nc.L1::no_allocate.u16 %0, [%1];\n" : "=h"(v) : "l"(p));
    return v;
}

__device__ __forceinline__ uint32_t pack_half2(float lo, float hi) {
    __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t *>(&h);
}

__device__ __forceinline__ float half_lo_f(uint32_t v) {
    return __half2float(__ushort_as_half(static_cast<unsigned short>(v & 0xFFFFu)));
}
__device__ __forceinline__ float half_hi_f(uint32_t v) {
    return __half2float(__ushort_as_half(static_cast<unsigned short>(v >> 16)));
}

// ---- x planes -------------------------------------------------------------

// Position of logical element k inside its group of 4 in the xh/xl planes.
__host__ __device__ __forceinline__ uint32_t xplane_pos(uint32_t k) {
    const uint32_t r = k & 3u;
    return (k & ~3u) | (r == 1u ? 2u : r == 2u ? 1u : r);
}

// One thread per 32-value sub-block of one row of x: writes the permuted fp16
// plane(s) and the sub-block sum.  `row_of` maps plane rows to source rows
// (NULL = identity).
template <typename XT>
__global__ void xplanes_kernel(const XT *__restrict__ x, uint32_t rows, uint32_t k_dim,
                               __half *__restrict__ xh, __half *__restrict__ xl,
                               float *__restrict__ xs) {
    const uint32_t subs = k_dim / 32;
    const uint64_t id = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x;
    if (id >= static_cast<uint64_t>(rows) * subs) return;
    const uint32_t row = static_cast<uint32_t>(id / subs), s = static_cast<uint32_t>(id % subs);
    const XT *src = x + static_cast<uint64_t>(row) * k_dim + 32 * s;
    __half *dh = xh + static_cast<uint64_t>(row) * k_dim + 32 * s;
    float sum = 0.0f;
    __align__(16) __half hv[32];
    __align__(16) __half lv[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) {
        const float v = load_x<XT>(src + i);
        sum += v;
        const __half h = __float2half_rn(v);
        hv[xplane_pos(i)] = h;
        lv[xplane_pos(i)] = __float2half_rn(v - __half2float(h));
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) reinterpret_cast<uint4 *>(dh)[i] = reinterpret_cast<uint4 *>(hv)[i];
    if (xl) {
        __half *dl = xl + static_cast<uint64_t>(row) * k_dim + 32 * s;
#pragma unroll
        for (int i = 0; i < 4; ++i)
            reinterpret_cast<uint4 *>(dl)[i] = reinterpret_cast<uint4 *>(lv)[i];
    }
    xs[static_cast<uint64_t>(row) * subs + s] = sum;
}

// ---- tile job description -------------------------------------------------

// Which weight rows, which x rows and where the outputs go for one CTA.
struct QTile {
    const uint8_t *w[2];   // up to two matrices over the same rows (gate, up)
    uint32_t row0;         // first output row of the tile
    uint32_t out_dim;
    uint32_t in_dim;
    uint64_t row_bytes;
    uint32_t ncol;         // valid token columns (<= 8)
    uint32_t xrow[8];      // x plane row of each column
    uint32_t orow[8];      // output row of each column
};

// ---- Q4_K -----------------------------------------------------------------

struct Q4kRowConsts {
    uint32_t hs_lo, hs_hi; // half2 (sc, sc) and (sc/16, sc/16)
    uint32_t mins;         // half2 (m_2c, m_2c+1)
    float d, dmin;         // d carries the 2^24 of the subnormal codes
};

__device__ __forceinline__ Q4kRowConsts q4k_row_consts(const uint4 &h, int c) {
    Q4kRowConsts r;
    r.d = half_lo_f(h.x) * 16777216.0f;
    r.dmin = half_hi_f(h.x);
    const uint32_t s0 = h.y, s1 = h.z, s2 = h.w;
    // The lane's two sub-blocks j = 2c, 2c + 1 (src/quant.cpp:63-71): bytes
    // k = 2 (c & 1), k + 1 of each scale word.  R = (sc_2c, sc_2c+1, m_2c, m_2c+1).
    const uint32_t sel = (c & 1) ? 0x7632u : 0x5410u;
    const uint32_t y = prmt(s0, s1, sel);                              // low 6 bits (j < 4), top 2 (j >= 4)
    uint32_t R;
    if (c < 2) {
        R = y & 0x3F3F3F3Fu;
    } else {
        const uint32_t x = prmt(s2, s2 >> 4, sel) & 0x0F0F0F0Fu;      // low 4 bits (j >= 4)
        R = x | ((y >> 2) & 0x30303030u);
    }
    // bytes -> exact fp16 via 1024 + b
    r.hs_lo = hsub2_u32(prmt(R, 0x64646464u, 0x4040u), 0x64006400u);  // (sc_2c, sc_2c)
    r.hs_hi = hfma2_u32(prmt(R, 0x64646464u, 0x4141u), 0x2C002C00u, 0xD400D400u); // (sc_2c+1 / 16) x 2
    r.mins = hsub2_u32(prmt(R, 0x64646464u, 0x4342u), 0x64006400u);   // (m_2c, m_2c+1)
    return r;
}

// One m-tile (rows g and g+8 of the tile) over one Q4_K block.
// xb: the thread's 32 B-fragment registers of x plane(s) for this block.
template <int PLANES>
__device__ __forceinline__ void q4k_mtile_block(const uint4 &h0, const uint4 &h1,
                                                const uint4 (&q0)[2], const uint4 (&q1)[2], int c,
                                                const uint32_t (&xb)[PLANES][32],
                                                const uint32_t (&xm)[2], float (&tot)[4]) {
    const Q4kRowConsts r0 = q4k_row_consts(h0, c);
    const Q4kRowConsts r1 = q4k_row_consts(h1, c);
    // four independent accumulator chains (low / high nibbles x even / odd words)
    float acc[4][4];
    const uint32_t w0[8] = {q0[0].x, q0[0].y, q0[0].z, q0[0].w, q0[1].x, q0[1].y, q0[1].z, q0[1].w};
    const uint32_t w1[8] = {q1[0].x, q1[0].y, q1[0].z, q1[0].w, q1[1].x, q1[1].y, q1[1].z, q1[1].w};
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const uint32_t s0 = w0[i] >> 8, s1 = w1[i] >> 8;
        // low nibbles: sub-block 2c
        const uint32_t a0 = hmul2_u32(w0[i] & 0x000F000Fu, r0.hs_lo);
        const uint32_t a1 = hmul2_u32(w1[i] & 0x000F000Fu, r1.hs_lo);
        const uint32_t a2 = hmul2_u32(s0 & 0x000F000Fu, r0.hs_lo);
        const uint32_t a3 = hmul2_u32(s1 & 0x000F000Fu, r1.hs_lo);
#pragma unroll
        for (int p = 0; p < PLANES; ++p) {
            if (i < 2 && p == 0) mma_f16_zc(acc[i & 1], a0, a1, a2, a3, xb[p][2 * i], xb[p][2 * i + 1]);
            else mma_f16(acc[i & 1], a0, a1, a2, a3, xb[p][2 * i], xb[p][2 * i + 1]);
        }
        // high nibbles: sub-block 2c+1
        const uint32_t e0 = hmul2_u32(w0[i] & 0x00F000F0u, r0.hs_hi);
        const uint32_t e1 = hmul2_u32(w1[i] & 0x00F000F0u, r1.hs_hi);
        const uint32_t e2 = hmul2_u32(s0 & 0x00F000F0u, r0.hs_hi);
        const uint32_t e3 = hmul2_u32(s1 & 0x00F000F0u, r1.hs_hi);
#pragma unroll
        for (int p = 0; p < PLANES; ++p) {
            if (i < 2 && p == 0) mma_f16_zc(acc[2 + (i & 1)], e0, e1, e2, e3, xb[p][16 + 2 * i], xb[p][16 + 2 * i + 1]);
            else mma_f16(acc[2 + (i & 1)], e0, e1, e2, e3, xb[p][16 + 2 * i], xb[p][16 + 2 * i + 1]);
        }
    }
    float accm[4];
    mma_f16_zc(accm, r0.mins, r1.mins, 0u, 0u, xm[0], 0u);
    mma_f16(accm, r0.mins, r1.mins, 0u, 0u, xm[1], 0u);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
        const float a = (acc[0][e] + acc[1][e]) + (acc[2][e] + acc[3][e]);
        const float d = e < 2 ? r0.d : r1.d, dm = e < 2 ? r0.dmin : r1.dmin;
        tot[e] = fmaf(d, a, fmaf(-dm, accm[e], tot[e]));
    }
}

// ---- Q8_0 -----------------------------------------------------------------

// Loads the thread's 8 codes (bytes 8c..8c+7 of the block's qs) of one row.
__device__ __forceinline__ void q8_load(const uint8_t *row, uint32_t blk, int c, uint32_t &wa,
                                        uint32_t &wb, uint32_t &dbits) {
    const uint8_t *s = row + 34ull * blk;
    dbits = ldg_nc_u16(s);
    if ((reinterpret_cast<uintptr_t>(s) & 2u) == 0u) {
        // block start is 4-byte aligned: codes start 2 bytes into a word
        const uint32_t W0 = ldg_nc_u32(s + 8 * c);
        const uint32_t W1 = ldg_nc_u32(s + 8 * c + 4);
        const uint32_t W2 = ldg_nc_u32(s + 8 * c + 8);
        wa = __funnelshift_r(W0, W1, 16);
        wb = __funnelshift_r(W1, W2, 16);
    } else {
        wa = ldg_nc_u32(s + 2 + 8 * c);
        wb = ldg_nc_u32(s + 6 + 8 * c);
    }
}

} // namespace fmb
