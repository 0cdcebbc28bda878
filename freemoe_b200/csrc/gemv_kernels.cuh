// gemv_kernels.cuh -- the CTA-level quantised GEMV kernel shared by the plain
// GEMV entry point and the MoE block (gate/up + SwiGLU, down).
//
// CTA = NW warps on one tile of 16*MT rows (of NMAT matrices over the same
// rows) x 8 token columns; the warps split the quantisation blocks of the
// row (K) and their partial sums are reduced in shared memory in a fixed
// order, so results are deterministic run to run.
#pragma once

#include "gemv_core.cuh"

namespace fmb {

enum { GEMV_PLAIN = 0, GEMV_GATE_UP = 1, GEMV_DOWN = 2 };

struct QGemvParams {
    // matrices
    const uint8_t *w;                 // plain mode
    const void *const *slots;         // MoE modes: per-expert payload base
    uint64_t w_off0, w_off1;          // byte offsets of matrix 0 / 1 within a slot
    uint32_t type_id;
    uint32_t out_dim, in_dim;
    uint64_t row_bytes;
    // tokens
    uint32_t tokens;                  // plain mode: number of x rows
    const uint32_t *offsets;          // MoE: [E+1] grouped pair ranges
    const uint32_t *pairs;            // MoE: flat pair index of each grouped slot
    uint32_t top_k;
    // x planes
    const __half *xh, *xl;            // [rows][in_dim]
    const float *xs;                  // [rows][in_dim/32]
    // output
    float *y;                         // [rows][out_dim]
    int *status;                      // device status word
    // gate/up of the streamed kernel only: when act_h is set, the SwiGLU output
    // goes straight into the down projection's x planes (hi, lo fp16 in the
    // staged order `act_layout`, f32 sums per 32 values) instead of y
    __half *act_h, *act_l;
    float *act_s;
    int act_layout;
};

// SwiGLU of include/fm/activation.hpp:62-84 (plain form): float(silu(double(g))) * u.
__device__ __forceinline__ float swiglu_ref(float g, float u) {
    const double gd = static_cast<double>(g);
    const float act = static_cast<float>(gd / (1.0 + exp(-gd)));
    return __fmul_rn(act, u);
}

template <int TYPE, int MT, int NW, int PLANES, int MODE>
__global__ void __launch_bounds__(NW * 32)
    qgemv_kernel(const QGemvParams p) {
    constexpr int NMAT = (MODE == GEMV_GATE_UP) ? 2 : 1;
    constexpr int TILE = 16 * MT;
    __shared__ uint32_t s_xrow[8], s_orow[8];
    __shared__ const uint8_t *s_w[2];
    __shared__ uint32_t s_ncol;
    __shared__ float s_red[NW][NMAT][TILE][8];

    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int g = lane >> 2, c = lane & 3;
    const uint32_t row0 = blockIdx.x * TILE;

    if (threadIdx.x == 0) {
        uint32_t ncol = 0;
        const uint8_t *base = nullptr;
        if (MODE == GEMV_PLAIN) {
            const uint32_t t0 = blockIdx.y * 8;
            ncol = p.tokens > t0 ? min(8u, p.tokens - t0) : 0u;
            for (uint32_t n = 0; n < 8; ++n) s_xrow[n] = s_orow[n] = t0 + (n < ncol ? n : 0);
            base = p.w;
        } else {
            const uint32_t e = blockIdx.z;
            const uint32_t start = p.offsets[e], end = p.offsets[e + 1];
            const uint32_t s0 = start + blockIdx.y * 8;
            ncol = end > s0 ? min(8u, end - s0) : 0u;
            for (uint32_t n = 0; n < 8; ++n) {
                const uint32_t slot = s0 + (n < ncol ? n : 0);
                s_orow[n] = slot;
                s_xrow[n] = (MODE == GEMV_GATE_UP) ? (ncol ? p.pairs[slot] / p.top_k : 0u) : slot;
            }
            base = ncol ? static_cast<const uint8_t *>(p.slots[e]) : nullptr;
            if (ncol && !base) {
                raise_device_status(p.status, FM_STATUS_EXPERT_EXECUTION_MISMATCH);
                ncol = 0;
            }
        }
        s_ncol = ncol;
        s_w[0] = base ? base + p.w_off0 : nullptr;
        s_w[1] = base ? base + p.w_off1 : nullptr;
    }
    __syncthreads();
    const uint32_t ncol = s_ncol;
    if (ncol == 0 || row0 >= p.out_dim) return;

    // rows of this thread: r(mt, h) = row0 + 16 mt + g + 8 h, clamped for loads
    const uint8_t *rowp[NMAT][MT][2];
#pragma unroll
    for (int m = 0; m < NMAT; ++m)
#pragma unroll
        for (int mt = 0; mt < MT; ++mt)
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const uint32_t r = min(row0 + 16 * mt + g + 8 * h, p.out_dim - 1);
                rowp[m][mt][h] = s_w[m] + static_cast<uint64_t>(r) * p.row_bytes;
            }

    float tot[NMAT][MT][4];
#pragma unroll
    for (int m = 0; m < NMAT; ++m)
#pragma unroll
        for (int mt = 0; mt < MT; ++mt)
#pragma unroll
            for (int e = 0; e < 4; ++e) tot[m][mt][e] = 0.0f;

    const bool col_ok = static_cast<uint32_t>(g) < ncol;
    const uint32_t xrow = s_xrow[g];
    const uint32_t nsub = p.in_dim / 32;
    const __half *xh_row = p.xh + static_cast<uint64_t>(xrow) * p.in_dim;
    const __half *xl_row = PLANES > 1 ? p.xl + static_cast<uint64_t>(xrow) * p.in_dim : nullptr;
    const float *xs_row = p.xs + static_cast<uint64_t>(xrow) * nsub;

    if (TYPE == FM_TYPE_Q4_K) {
        const uint32_t nblk = p.in_dim / 256;
        for (uint32_t b = warp; b < nblk; b += NW) {
            uint32_t xb[PLANES][32];
            uint32_t xm[2];
            if (col_ok) {
#pragma unroll
                for (int pl = 0; pl < PLANES; ++pl) {
                    const uint4 *src = reinterpret_cast<const uint4 *>(
                        (pl == 0 ? xh_row : xl_row) + b * 256 + 64 * c);
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        const uint4 v = src[i];
                        xb[pl][4 * i + 0] = v.x;
                        xb[pl][4 * i + 1] = v.y;
                        xb[pl][4 * i + 2] = v.z;
                        xb[pl][4 * i + 3] = v.w;
                    }
                }
                const float2 X = *reinterpret_cast<const float2 *>(xs_row + b * 8 + 2 * c);
                xm[0] = pack_half2(X.x, X.y);
                xm[1] = pack_half2(X.x - half_lo_f(xm[0]), X.y - half_hi_f(xm[0]));
            } else {
#pragma unroll
                for (int pl = 0; pl < PLANES; ++pl)
#pragma unroll
                    for (int i = 0; i < 32; ++i) xb[pl][i] = 0u;
                xm[0] = xm[1] = 0u;
            }
#pragma unroll
            for (int m = 0; m < NMAT; ++m)
#pragma unroll
                for (int mt = 0; mt < MT; ++mt) {
                    const uint8_t *b0 = rowp[m][mt][0] + 144ull * b;
                    const uint8_t *b1 = rowp[m][mt][1] + 144ull * b;
                    const uint4 h0 = ldg_nc_v4(b0), h1 = ldg_nc_v4(b1);
                    uint4 q0[2], q1[2];
                    q0[0] = ldg_nc_v4(b0 + 16 + 32 * c);
                    q0[1] = ldg_nc_v4(b0 + 32 + 32 * c);
                    q1[0] = ldg_nc_v4(b1 + 16 + 32 * c);
                    q1[1] = ldg_nc_v4(b1 + 32 + 32 * c);
                    q4k_mtile_block<PLANES>(h0, h1, q0, q1, c, xb, xm, tot[m][mt]);
                }
        }
    } else if (TYPE == FM_TYPE_Q6_K) {
        // Q6_K (src/quant.cpp:347-372): one MMA per 16-value scale group j of a
        // block; lane (g, c) takes values 16j + 4c .. 16j + 4c + 3 of rows g and
        // g+8, so x is read in its natural order (4 consecutive fp16 per lane).
        // The 6-bit code c6 placed in a zero fp16 is the subnormal c6 * 2^-24;
        // subtracting 32 * 2^-24 is exact, so A holds (c6 - 32) * 2^-24; the
        // accumulator of each group is scaled by 2^24 d * scale in f32.
        const uint32_t nblk = p.in_dim / 256;
        for (uint32_t b = warp; b < nblk; b += NW) {
#pragma unroll 2
            for (uint32_t j = 0; j < 16; ++j) {
                uint32_t xb[PLANES][2];
#pragma unroll
                for (int pl = 0; pl < PLANES; ++pl) {
                    if (col_ok) {
                        const uint2 v = *reinterpret_cast<const uint2 *>((pl == 0 ? xh_row : xl_row) + b * 256 + 16 * j +
                                                                         4 * c);
                        xb[pl][0] = v.x;
                        xb[pl][1] = v.y;
                    } else {
                        xb[pl][0] = xb[pl][1] = 0u;
                    }
                }
                const uint32_t u = 16 * (j & 7) + 4 * c;          // value index inside the 128-value half
                const uint32_t h = j >> 3, grp = u >> 5, l = u & 31;
                const uint32_t ql_off = 64 * h + (grp & 1) * 32 + l, qh_off = 128 + 32 * h + l;
                const uint32_t nib = (grp >> 1) * 4, qsh = 2 * grp;
#pragma unroll
                for (int m = 0; m < NMAT; ++m)
#pragma unroll
                    for (int mt = 0; mt < MT; ++mt) {
                        uint32_t a[2][2];
                        float ds[2];
#pragma unroll
                        for (int hr = 0; hr < 2; ++hr) {
                            const uint8_t *bp = rowp[m][mt][hr] + 210ull * b;
                            const uint32_t ql = ldg_nc_u16(bp + ql_off) | (ldg_nc_u16(bp + ql_off + 2) << 16);
                            const uint32_t qh = ldg_nc_u16(bp + qh_off) | (ldg_nc_u16(bp + qh_off + 2) << 16);
                            const uint32_t c6 = ((ql >> nib) & 0x0F0F0F0Fu) | (((qh >> qsh) & 0x03030303u) << 4);
                            a[hr][0] = hsub2_u32(prmt(c6, 0u, 0x5140u), 0x00200020u);
                            a[hr][1] = hsub2_u32(prmt(c6, 0u, 0x7362u), 0x00200020u);
                            const float d = fp16_bits_to_f32(static_cast<uint16_t>(ldg_nc_u16(bp + 208)));
                            const int8_t sc = static_cast<int8_t>(ldg_nc_u16(bp + 192 + (j & ~1u)) >> (8 * (j & 1)));
                            ds[hr] = __fmul_rn(d, static_cast<float>(sc)) * 16777216.0f; // codes carry 2^-24
                        }
                        float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
                        for (int pl = 0; pl < PLANES; ++pl)
                            mma_f16(acc, a[0][0], a[1][0], a[0][1], a[1][1], xb[pl][0], xb[pl][1]);
                        float *t = tot[m][mt];
                        t[0] = fmaf(ds[0], acc[0], t[0]);
                        t[1] = fmaf(ds[0], acc[1], t[1]);
                        t[2] = fmaf(ds[1], acc[2], t[2]);
                        t[3] = fmaf(ds[1], acc[3], t[3]);
                    }
            }
        }
    } else { // Q8_0
        const uint32_t nblk = p.in_dim / 32;
        const uint32_t xr_a = s_xrow[2 * c], xr_b = s_xrow[2 * c + 1];
        const bool ok_a = static_cast<uint32_t>(2 * c) < ncol, ok_b = static_cast<uint32_t>(2 * c + 1) < ncol;
        for (uint32_t blk = warp; blk < nblk; blk += NW) {
            uint32_t xb[PLANES][4];
            if (col_ok) {
#pragma unroll
                for (int pl = 0; pl < PLANES; ++pl) {
                    const uint4 v = *reinterpret_cast<const uint4 *>(
                        (pl == 0 ? xh_row : xl_row) + blk * 32 + 8 * c);
                    xb[pl][0] = v.x;
                    xb[pl][1] = v.y;
                    xb[pl][2] = v.z;
                    xb[pl][3] = v.w;
                }
            } else {
#pragma unroll
                for (int pl = 0; pl < PLANES; ++pl) xb[pl][0] = xb[pl][1] = xb[pl][2] = xb[pl][3] = 0u;
            }
            const float Xa = ok_a ? p.xs[static_cast<uint64_t>(xr_a) * nsub + blk] : 0.0f;
            const float Xb = ok_b ? p.xs[static_cast<uint64_t>(xr_b) * nsub + blk] : 0.0f;
#pragma unroll
            for (int m = 0; m < NMAT; ++m)
#pragma unroll
                for (int mt = 0; mt < MT; ++mt) {
                    uint32_t wa0, wb0, d0, wa1, wb1, d1;
                    q8_load(rowp[m][mt][0], blk, c, wa0, wb0, d0);
                    q8_load(rowp[m][mt][1], blk, c, wa1, wb1, d1);
                    const uint32_t va0 = wa0 ^ 0x80808080u, vb0 = wb0 ^ 0x80808080u;
                    const uint32_t va1 = wa1 ^ 0x80808080u, vb1 = wb1 ^ 0x80808080u;
                    float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
                    for (int pl = 0; pl < PLANES; ++pl) {
                        mma_f16(acc, prmt(va0, 0u, 0x4240u), prmt(va1, 0u, 0x4240u),
                                prmt(va0, 0u, 0x4341u), prmt(va1, 0u, 0x4341u),
                                xb[pl][0], xb[pl][1]);
                        mma_f16(acc, prmt(vb0, 0u, 0x4240u), prmt(vb1, 0u, 0x4240u),
                                prmt(vb0, 0u, 0x4341u), prmt(vb1, 0u, 0x4341u),
                                xb[pl][2], xb[pl][3]);
                    }
                    const float dr0 = fp16_bits_to_f32(static_cast<uint16_t>(d0));
                    const float dr1 = fp16_bits_to_f32(static_cast<uint16_t>(d1));
                    const float dr0s = dr0 * 16777216.0f, dr1s = dr1 * 16777216.0f; // codes carry 2^-24
                    float *t = tot[m][mt];
                    t[0] = fmaf(dr0s, acc[0], fmaf(-128.0f * dr0, Xa, t[0]));
                    t[1] = fmaf(dr0s, acc[1], fmaf(-128.0f * dr0, Xb, t[1]));
                    t[2] = fmaf(dr1s, acc[2], fmaf(-128.0f * dr1, Xa, t[2]));
                    t[3] = fmaf(dr1s, acc[3], fmaf(-128.0f * dr1, Xb, t[3]));
                }
        }
    }

    // deterministic cross-warp reduction
#pragma unroll
    for (int m = 0; m < NMAT; ++m)
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
            s_red[warp][m][16 * mt + g][2 * c] = tot[m][mt][0];
            s_red[warp][m][16 * mt + g][2 * c + 1] = tot[m][mt][1];
            s_red[warp][m][16 * mt + g + 8][2 * c] = tot[m][mt][2];
            s_red[warp][m][16 * mt + g + 8][2 * c + 1] = tot[m][mt][3];
        }
    __syncthreads();
    for (int idx = threadIdx.x; idx < TILE * 8; idx += NW * 32) {
        const int r = idx >> 3, n = idx & 7;
        const uint32_t row = row0 + r;
        if (static_cast<uint32_t>(n) >= ncol || row >= p.out_dim) continue;
        float v[NMAT];
#pragma unroll
        for (int m = 0; m < NMAT; ++m) {
            float s = 0.0f;
#pragma unroll
            for (int w = 0; w < NW; ++w) s += s_red[w][m][r][n];
            v[m] = s;
        }
        float out;
        if (MODE == GEMV_GATE_UP) out = swiglu_ref(v[0], v[NMAT - 1]);
        else out = v[0];
        p.y[static_cast<uint64_t>(s_orow[n]) * p.out_dim + row] = out;
    }
}

} // namespace fmb
