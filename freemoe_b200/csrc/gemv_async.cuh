// gemv_async.cuh -- the decode GEMV: quantised rows streamed with 16-byte
// cp.async copies into per-warp shared-memory rings, dequantised in
// registers into mma.sync tensor-core fragments.
//
// Replaces the per-row CPU kernels row_dot_q4_k_avx2 / row_dot_q8_0_avx2
// (src/kernels.cpp:720-771, :639-653) for rows of a multiple of 256 values.
//
// Structure: persistent CTAs of NW warps; a tile is 16*MT rows (of NMAT
// matrices over the same rows: gate and up) x 8 token columns.  Warp w takes
// the 256-value K steps w, w + NW, ... of each tile.  Each warp keeps P of its
// K steps in flight: for step j it issues 16-byte cp.async copies of every
// tile row's quant bytes (each warp instruction moves 512 contiguous-ish
// bytes; 9 or 17 chunks per row) into ring slot j % P, P steps ahead,
// crossing tile boundaries, so the HBM stream never drains between tiles.
// The weight bytes never pass through registers until they are unpacked; x
// fragments (L2/L1 resident, read by every tile) are loaded directly before
// the ring wait.  Per tile the warps' partial sums are reduced in shared
// memory in a fixed order (deterministic) and written (with SwiGLU for
// gate/up).  Only tiles that hold tokens are visited: the CTA first builds
// the prefix of token tiles per expert from the grouping offsets.
#pragma once

#include "gemv_core.cuh"
#include "gemv_kernels.cuh"
#include "ptx.cuh"

namespace fmb {

// ---- x-plane layouts for the staged kernel -----------------------------------
//
// Position of logical element k of a 256-value K step inside its staged row,
// chosen so that a warp's 16-byte fragment loads read 64 contiguous bytes per
// token:
//   Q4_K: lane (g, c) reads, for i = 0..7, the 8 values 64c + 8i + [0, 8) as
//         chunk 4i + c;
//   Q8_0: lane (g, c) reads, for sub-block s = 0..7, the 4 + 4 values
//         32s + 4c + [0, 4) and 32s + 16 + 4c + [0, 4) as chunk 4s + c.
// Inside a chunk each group of 4 is stored (0, 2, 1, 3) (xplane_pos).
enum { XL_Q4K = 0, XL_Q8 = 1 };

__host__ __device__ __forceinline__ uint32_t staged_pos(uint32_t k, int layout) {
    const uint32_t base = k & ~255u, r = k & 255u;
    uint32_t chunk, j;
    if (layout == XL_Q4K) {
        const uint32_t c = r >> 6, i = (r >> 3) & 7u;
        chunk = 4 * i + c;
        j = r & 7u;
    } else {
        const uint32_t s = r >> 5, w = r & 31u;       // sub-block, position in it
        const uint32_t half = w >> 4, c = (w >> 2) & 3u; // [0,16) or [16,32); lane c
        chunk = 4 * s + c;
        j = half * 4 + (w & 3u);
    }
    return base + chunk * 8 + (j & 4u) + xplane_pos(j & 3u);
}

// One 32-value sub-block s of x row `row`: staged fp16 plane(s) and the sum.
// Each group of 4 values lands on 4 consecutive positions (xplane_pos order),
// so the planes are written 8 bytes at a time; x is read 16 bytes at a time
// when the row is 16-byte aligned.
template <typename XT>
__device__ __forceinline__ void xplanes_staged_item(const XT *__restrict__ x, uint32_t row, uint32_t s,
                                                    uint32_t k_dim, int layout, __half *__restrict__ xh,
                                                    __half *__restrict__ xl, float *__restrict__ xs) {
    const uint32_t subs = k_dim / 32;
    const XT *src = x + static_cast<uint64_t>(row) * k_dim + 32 * s;
    __half *dh = xh + static_cast<uint64_t>(row) * k_dim;
    __half *dl = xl ? xl + static_cast<uint64_t>(row) * k_dim : nullptr;
    float v[32];
    if ((reinterpret_cast<uintptr_t>(src) & 15u) == 0) {
        if constexpr (sizeof(XT) == 2) {
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const uint4 w = __ldg(reinterpret_cast<const uint4 *>(src) + q);
                const uint32_t u[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    v[8 * q + 2 * i] = __uint_as_float(u[i] << 16);
                    v[8 * q + 2 * i + 1] = __uint_as_float(u[i] & 0xFFFF0000u);
                }
            }
        } else {
#pragma unroll
            for (int q = 0; q < 8; ++q) {
                const float4 w = __ldg(reinterpret_cast<const float4 *>(src) + q);
                v[4 * q] = w.x;
                v[4 * q + 1] = w.y;
                v[4 * q + 2] = w.z;
                v[4 * q + 3] = w.w;
            }
        }
    } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] = load_x<XT>(src + i);
    }
    float sum = 0.0f;
#pragma unroll
    for (int i = 0; i < 32; ++i) sum += v[i];
#pragma unroll
    for (int g4 = 0; g4 < 8; ++g4) {
        const uint32_t pos = staged_pos(32 * s + 4 * g4, layout); // the group's first position
        __half h[4], l[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            h[i] = __float2half_rn(v[4 * g4 + i]);
            l[i] = __float2half_rn(v[4 * g4 + i] - __half2float(h[i]));
        }
        const uint2 hv = make_uint2(__half_as_ushort(h[0]) | (static_cast<uint32_t>(__half_as_ushort(h[2])) << 16),
                                    __half_as_ushort(h[1]) | (static_cast<uint32_t>(__half_as_ushort(h[3])) << 16));
        *reinterpret_cast<uint2 *>(dh + pos) = hv;
        if (dl) {
            const uint2 lv = make_uint2(__half_as_ushort(l[0]) | (static_cast<uint32_t>(__half_as_ushort(l[2])) << 16),
                                        __half_as_ushort(l[1]) | (static_cast<uint32_t>(__half_as_ushort(l[3])) << 16));
            *reinterpret_cast<uint2 *>(dl + pos) = lv;
        }
    }
    xs[static_cast<uint64_t>(row) * subs + s] = sum;
}

template <typename XT>
__global__ void xplanes_staged_kernel(const XT *__restrict__ x, uint32_t rows, uint32_t k_dim,
                                      int layout, __half *__restrict__ xh, __half *__restrict__ xl,
                                      float *__restrict__ xs) {
    const uint32_t subs = k_dim / 32;
    const uint64_t id = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x;
    if (id >= static_cast<uint64_t>(rows) * subs) return;
    xplanes_staged_item(x, static_cast<uint32_t>(id / subs), static_cast<uint32_t>(id % subs), k_dim, layout, xh, xl,
                        xs);
}

template <int TYPE, int MT, int NMAT>
struct StageGeom {
    static constexpr int TILE = 16 * MT;
    static constexpr int RB = TYPE == FM_TYPE_Q4_K ? 144 : 272; // quant bytes per row per K step
    static constexpr int CHUNKS = RB / 16;                       // 16-byte copies per row
    static constexpr int BYTES = NMAT * TILE * RB;               // one ring slot
};

constexpr int kMaxGroupExperts = 1024;

// x operands of one 256-value K step b for one warp: the B fragments of the
// token planes (lane (g, c) holds column g) and the sub-block sums (Q4_K: the
// pair of sub-blocks 2c, 2c+1 of column g; Q8_0: the 8 sums of columns 2c and
// 2c + 1).  Lanes of columns past the tile's tokens load a valid row (the
// caller points them at x row 0): their MMA columns are never written out.
template <int TYPE, int PLANES>
struct ItemX {
    uint32_t xb[PLANES][32];
    float2 X;
    float Xa[8], Xb[8];
};

template <int TYPE, int PLANES>
__device__ __forceinline__ void load_item_x(ItemX<TYPE, PLANES> &ix, const uint8_t *xh_row, const uint8_t *xl_row,
                                            const float *xs_row, const float *xs_a, const float *xs_b,
                                            bool ok_a, bool ok_b, uint32_t b, int c) {
#pragma unroll
    for (int pl = 0; pl < PLANES; ++pl) {
        const uint8_t *row = (pl ? xl_row : xh_row) + static_cast<uint64_t>(b) * 512;
#pragma unroll
        for (int q = 0; q < 8; ++q) {
            const uint4 v = __ldg(reinterpret_cast<const uint4 *>(row + (4 * q + c) * 16));
            ix.xb[pl][4 * q + 0] = v.x;
            ix.xb[pl][4 * q + 1] = v.y;
            ix.xb[pl][4 * q + 2] = v.z;
            ix.xb[pl][4 * q + 3] = v.w;
        }
    }
    ix.X = make_float2(0.f, 0.f);
    if (TYPE == FM_TYPE_Q4_K) {
        ix.X = __ldg(reinterpret_cast<const float2 *>(xs_row + b * 8 + 2 * c));
    } else {
#pragma unroll
        for (int q = 0; q < 8; ++q) {
            ix.Xa[q] = ok_a ? __ldg(xs_a + b * 8 + q) : 0.0f;
            ix.Xb[q] = ok_b ? __ldg(xs_b + b * 8 + q) : 0.0f;
        }
    }
}

// One K step of one tile from its staged ring slot `st` (the tile's NMAT x
// 16*MT rows back to back, RB bytes each): tot[m][mt] += this step's partial
// dot products of rows (g, g + 8) of m-tile mt with columns (2c, 2c + 1).
template <int TYPE, int MT, int NMAT, int PLANES, int RB>
__device__ __forceinline__ void qgemv_item(const uint8_t *st, const ItemX<TYPE, PLANES> &ix, int g, int c,
                                           float (&tot)[NMAT][MT][4]) {
    constexpr int TILE = 16 * MT;
    if (TYPE == FM_TYPE_Q4_K) {
        uint32_t xm[2];
        xm[0] = pack_half2(ix.X.x, ix.X.y);
        xm[1] = pack_half2(ix.X.x - half_lo_f(xm[0]), ix.X.y - half_hi_f(xm[0]));
#pragma unroll
        for (int m = 0; m < NMAT; ++m)
#pragma unroll
            for (int mt = 0; mt < MT; ++mt) {
                const uint8_t *r0 = st + (m * TILE + 16 * mt + g) * RB;
                const uint8_t *r1 = r0 + 8 * RB;
                const uint4 h0 = *reinterpret_cast<const uint4 *>(r0);
                const uint4 h1 = *reinterpret_cast<const uint4 *>(r1);
                uint4 q0[2], q1[2];
                q0[0] = *reinterpret_cast<const uint4 *>(r0 + 16 + 32 * c);
                q0[1] = *reinterpret_cast<const uint4 *>(r0 + 32 + 32 * c);
                q1[0] = *reinterpret_cast<const uint4 *>(r1 + 16 + 32 * c);
                q1[1] = *reinterpret_cast<const uint4 *>(r1 + 32 + 32 * c);
                q4k_mtile_block<PLANES>(h0, h1, q0, q1, c, ix.xb, xm, tot[m][mt]);
            }
    } else { // Q8_0: 8 blocks of 32 per K step; block sb uses registers 4sb..4sb+3
#pragma unroll
        for (int sb = 0; sb < 8; ++sb) {
            const uint32_t off = 34 * sb;
#pragma unroll
            for (int m = 0; m < NMAT; ++m)
#pragma unroll
                for (int mt = 0; mt < MT; ++mt) {
                    uint32_t wa[2], wb[2], dr[2];
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        const uint8_t *r = st + (m * TILE + 16 * mt + g + 8 * h) * RB + off;
                        dr[h] = *reinterpret_cast<const uint16_t *>(r);
                        if ((sb & 1) == 0) { // codes start 2 bytes into an aligned word
                            const uint32_t *wp = reinterpret_cast<const uint32_t *>(r + 4 * c);
                            const uint32_t *wq = reinterpret_cast<const uint32_t *>(r + 16 + 4 * c);
                            wa[h] = __funnelshift_r(wp[0], wp[1], 16);
                            wb[h] = __funnelshift_r(wq[0], wq[1], 16);
                        } else {
                            wa[h] = *reinterpret_cast<const uint32_t *>(r + 2 + 4 * c);
                            wb[h] = *reinterpret_cast<const uint32_t *>(r + 18 + 4 * c);
                        }
                    }
                    const uint32_t va0 = wa[0] ^ 0x80808080u, vb0 = wb[0] ^ 0x80808080u;
                    const uint32_t va1 = wa[1] ^ 0x80808080u, vb1 = wb[1] ^ 0x80808080u;
                    float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
                    for (int pl = 0; pl < PLANES; ++pl) {
                        mma_f16(acc, prmt(va0, 0u, 0x4240u), prmt(va1, 0u, 0x4240u),
                                prmt(va0, 0u, 0x4341u), prmt(va1, 0u, 0x4341u),
                                ix.xb[pl][4 * sb + 0], ix.xb[pl][4 * sb + 1]);
                        mma_f16(acc, prmt(vb0, 0u, 0x4240u), prmt(vb1, 0u, 0x4240u),
                                prmt(vb0, 0u, 0x4341u), prmt(vb1, 0u, 0x4341u),
                                ix.xb[pl][4 * sb + 2], ix.xb[pl][4 * sb + 3]);
                    }
                    const float d0 = fp16_bits_to_f32(static_cast<uint16_t>(dr[0]));
                    const float d1 = fp16_bits_to_f32(static_cast<uint16_t>(dr[1]));
                    const float d0s = d0 * 16777216.0f, d1s = d1 * 16777216.0f; // codes carry 2^-24
                    float *tt = tot[m][mt];
                    tt[0] = fmaf(d0s, acc[0], fmaf(-128.0f * d0, ix.Xa[sb], tt[0]));
                    tt[1] = fmaf(d0s, acc[1], fmaf(-128.0f * d0, ix.Xb[sb], tt[1]));
                    tt[2] = fmaf(d1s, acc[2], fmaf(-128.0f * d1, ix.Xa[sb], tt[2]));
                    tt[3] = fmaf(d1s, acc[3], fmaf(-128.0f * d1, ix.Xb[sb], tt[3]));
                }
        }
    }
}

#ifndef FMB_GEMV_MINB
#define FMB_GEMV_MINB 1
#endif

template <int TYPE, int MT, int NW, int PLANES, int MODE, int P>
__global__ void __launch_bounds__(NW * 32, FMB_GEMV_MINB)
    qgemv_async_kernel(const QGemvParams p, uint32_t row_tiles, uint32_t tok_tiles, uint32_t experts) {
    constexpr int NMAT = (MODE == GEMV_GATE_UP) ? 2 : 1;
    using G = StageGeom<TYPE, MT, NMAT>;
    constexpr int TILE = G::TILE;
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ float s_red[NW][NMAT][TILE][8];
    __shared__ float s_act[MODE == GEMV_GATE_UP ? TILE : 1][8]; // SwiGLU outputs of a tile (planes epilogue)
    // token tiles before expert e, in the dynamic shared memory after the rings
    uint32_t *s_prefix = reinterpret_cast<uint32_t *>(smem + static_cast<size_t>(NW) * P * G::BYTES);

    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int g = lane >> 2, c = lane & 3;
    const uint32_t nsteps = p.in_dim / 256;
    const uint32_t nsub = p.in_dim / 32;
    uint8_t *ring = smem + static_cast<size_t>(warp) * P * G::BYTES;

    // ---- active tiles: (expert, token tile, row tile), empty experts skipped
    uint32_t total_tok_tiles;
    if (MODE == GEMV_PLAIN) {
        total_tok_tiles = tok_tiles;
    } else {
        if (warp == 0) {
            uint32_t carry = 0;
            for (uint32_t e0 = 0; e0 < experts; e0 += 32) {
                const uint32_t e = e0 + lane;
                uint32_t v = 0;
                if (e < experts) v = (__ldg(p.offsets + e + 1) - __ldg(p.offsets + e) + 7) / 8;
                uint32_t incl = v;
#pragma unroll
                for (int o = 1; o < 32; o <<= 1) {
                    const uint32_t n = __shfl_up_sync(0xFFFFFFFFu, incl, o);
                    if (lane >= o) incl += n;
                }
                if (e < experts) s_prefix[e] = carry + incl - v;
                carry += __shfl_sync(0xFFFFFFFFu, incl, 31);
            }
            if (lane == 0) s_prefix[experts] = carry;
        }
        __syncthreads();
        total_tok_tiles = s_prefix[experts];
    }
    const uint32_t n_tiles = total_tok_tiles * row_tiles;
    const uint32_t my_tiles = n_tiles > blockIdx.x ? (n_tiles - blockIdx.x + gridDim.x - 1) / gridDim.x : 0u;
    const uint32_t nw = nsteps > static_cast<uint32_t>(warp) ? (nsteps - warp + NW - 1) / NW : 0u;

    // tile i of this CTA -> rows, expert, columns
    struct Tile {
        uint32_t row0, e, start, ncol;
        const uint8_t *base;
    };
    auto tile_of = [&](uint32_t i) -> Tile {
        Tile tl;
        const uint32_t a = blockIdx.x + i * gridDim.x;
        tl.row0 = min((a % row_tiles) * TILE, p.out_dim - TILE); // last tile overlaps the previous one
        const uint32_t q = a / row_tiles;
        if (MODE == GEMV_PLAIN) {
            tl.e = 0;
            tl.start = q * 8;
            tl.ncol = min(8u, p.tokens - tl.start);
            tl.base = p.w;
        } else {
            uint32_t lo = 0, hi = experts; // last e with s_prefix[e] <= q
            while (hi - lo > 1) {
                const uint32_t mid = (lo + hi) >> 1;
                if (s_prefix[mid] <= q) lo = mid;
                else hi = mid;
            }
            tl.e = lo;
            const uint32_t off = __ldg(p.offsets + lo), end = __ldg(p.offsets + lo + 1);
            tl.start = off + (q - s_prefix[lo]) * 8;
            tl.ncol = min(8u, end - tl.start);
            tl.base = static_cast<const uint8_t *>(p.slots[lo]);
        }
        return tl;
    };

    // ---- copy issue.  A ring slot holds the tile rows back to back (RB bytes
    // each), so chunk q of a slot is 16 bytes at q * 16 and lane l copies
    // chunks l, l + 32, ...: every cp.async warp instruction moves 512
    // contiguous slot bytes, drawn from 3-4 consecutive row pieces.  The
    // global offset of each of the lane's chunks relative to the tile's first
    // row is fixed for the whole kernel (row_bytes and the matrix offsets do
    // not change), so it is computed once; a cursor walks this warp's items
    // (tile, K step) without divisions.
    constexpr int ROWS = NMAT * TILE, NCH = ROWS * G::CHUNKS, NU = (NCH + 31) / 32;
    uint32_t gofs[NU];
#pragma unroll
    for (int u = 0; u < NU; ++u) {
        const int q = lane + 32 * u;
        const int r = q / G::CHUNKS, part = q % G::CHUNKS;
        const int m = r / TILE, rr = r % TILE;
        gofs[u] = static_cast<uint32_t>((m ? p.w_off1 : p.w_off0) + static_cast<uint64_t>(rr) * p.row_bytes) +
                  part * 16;
    }
    const uint8_t *cur_base = nullptr; // first row of the current tile (matrix 0)
    uint32_t cur_tile = 0xFFFFFFFFu, cur_jj = 0, issued = 0;
    const uint32_t my_items = my_tiles * nw;

    auto issue = [&]() {
        if (issued < my_items) {
            if (cur_jj == 0) {
                cur_tile = cur_tile == 0xFFFFFFFFu ? 0u : cur_tile + 1;
                const Tile tl = tile_of(cur_tile);
                const bool ok = tl.base && (reinterpret_cast<uintptr_t>(tl.base) & 15u) == 0;
                cur_base = ok ? tl.base + static_cast<uint64_t>(tl.row0) * p.row_bytes : nullptr;
            }
            if (cur_base) {
                const uint8_t *src = cur_base + static_cast<uint64_t>(warp + NW * cur_jj) * G::RB;
                uint8_t *dst = ring + (issued % P) * G::BYTES + lane * 16;
#pragma unroll
                for (int u = 0; u < NU; ++u)
                    if (lane + 32 * u < NCH) cp_async16(dst + 512 * u, src + gofs[u]);
            }
            if (++cur_jj == nw) cur_jj = 0;
            ++issued;
        }
        cp_async_commit(); // one group per item, even an empty one
    };

    for (int j = 0; j < P; ++j) issue();

    for (uint32_t i = 0; i < my_tiles; ++i) {
        const Tile tl = tile_of(i);
        if (threadIdx.x == 0 && MODE != GEMV_PLAIN && !tl.base)
            raise_device_status(p.status, FM_STATUS_EXPERT_EXECUTION_MISMATCH);
        if (threadIdx.x == 0 && tl.base && (reinterpret_cast<uintptr_t>(tl.base) & 15u))
            raise_device_status(p.status, FM_STATUS_INVALID_ARGUMENT);
        const bool tile_ok = tl.base && (reinterpret_cast<uintptr_t>(tl.base) & 15u) == 0;
        const bool col_ok = static_cast<uint32_t>(g) < tl.ncol;
        auto xrow_of = [&](uint32_t col) -> uint32_t {
            const uint32_t o = tl.start + col;
            return MODE == GEMV_GATE_UP ? __ldg(p.pairs + o) / p.top_k : o;
        };
        const uint32_t xr = col_ok ? xrow_of(g) : 0u;
        const uint8_t *xh_row = reinterpret_cast<const uint8_t *>(p.xh + static_cast<uint64_t>(xr) * p.in_dim);
        const uint8_t *xl_row =
            PLANES > 1 ? reinterpret_cast<const uint8_t *>(p.xl + static_cast<uint64_t>(xr) * p.in_dim) : nullptr;
        const float *xs_row = p.xs + static_cast<uint64_t>(xr) * nsub;
        const bool ok_a = static_cast<uint32_t>(2 * c) < tl.ncol, ok_b = static_cast<uint32_t>(2 * c + 1) < tl.ncol;
        const float *xs_a = (TYPE == FM_TYPE_Q8_0 && ok_a) ? p.xs + static_cast<uint64_t>(xrow_of(2 * c)) * nsub : nullptr;
        const float *xs_b = (TYPE == FM_TYPE_Q8_0 && ok_b) ? p.xs + static_cast<uint64_t>(xrow_of(2 * c + 1)) * nsub : nullptr;

        float tot[NMAT][MT][4];
#pragma unroll
        for (int m = 0; m < NMAT; ++m)
#pragma unroll
            for (int mt = 0; mt < MT; ++mt)
#pragma unroll
                for (int e = 0; e < 4; ++e) tot[m][mt][e] = 0.0f;

        for (uint32_t jj = 0; jj < nw; ++jj) {
            const uint32_t j = i * nw + jj;
            const uint32_t b = warp + NW * jj;
            // x operands for this K step, loaded before the ring wait
            ItemX<TYPE, PLANES> ix;
            load_item_x<TYPE, PLANES>(ix, xh_row, xl_row, xs_row, xs_a, xs_b, ok_a, ok_b, b, c);
            cp_async_wait<P - 1>(); // item j landed (this lane's copies)
            __syncwarp();           // ... and every other lane's
            if (tile_ok) qgemv_item<TYPE, MT, NMAT, PLANES, G::RB>(ring + (j % P) * G::BYTES, ix, g, c, tot);
            __syncwarp(); // every lane is done with the slot before it is refilled
            issue();
        }
        // ---- per-tile epilogue: fixed-order reduction over the NW warps
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
        if (MODE == GEMV_GATE_UP && p.act_h) {
            // The down projection's x planes, as xplanes_staged_kernel writes them:
            // four consecutive rows of one column land on four consecutive staged
            // positions in (0, 2, 1, 3) order, one 8-byte store per plane.
            for (int idx = threadIdx.x; idx < (TILE / 4) * 8; idx += NW * 32) {
                const int g4 = idx >> 3, col = idx & 7;
                if (!tile_ok || static_cast<uint32_t>(col) >= tl.ncol) continue;
                __half h[4], l[4];
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const int r = 4 * g4 + i;
                    float v[NMAT];
#pragma unroll
                    for (int m = 0; m < NMAT; ++m) {
                        float sum = 0.0f;
#pragma unroll
                        for (int w = 0; w < NW; ++w) sum += s_red[w][m][r][col];
                        v[m] = sum;
                    }
                    const float out = swiglu_ref(v[0], v[NMAT - 1]);
                    h[i] = __float2half_rn(out);
                    l[i] = __float2half_rn(out - __half2float(h[i]));
                    s_act[MODE == GEMV_GATE_UP ? r : 0][col] = out;
                }
                const uint64_t at =
                    static_cast<uint64_t>(tl.start + col) * p.out_dim + staged_pos(tl.row0 + 4 * g4, p.act_layout);
                *reinterpret_cast<uint2 *>(p.act_h + at) =
                    make_uint2(__half_as_ushort(h[0]) | (static_cast<uint32_t>(__half_as_ushort(h[2])) << 16),
                               __half_as_ushort(h[1]) | (static_cast<uint32_t>(__half_as_ushort(h[3])) << 16));
                *reinterpret_cast<uint2 *>(p.act_l + at) =
                    make_uint2(__half_as_ushort(l[0]) | (static_cast<uint32_t>(__half_as_ushort(l[2])) << 16),
                               __half_as_ushort(l[1]) | (static_cast<uint32_t>(__half_as_ushort(l[3])) << 16));
            }
        } else {
            for (int idx = threadIdx.x; idx < TILE * 8; idx += NW * 32) {
                const int r = idx >> 3, col = idx & 7;
                const uint32_t row = tl.row0 + r;
                if (!tile_ok || static_cast<uint32_t>(col) >= tl.ncol || row >= p.out_dim) continue;
                float v[NMAT];
#pragma unroll
                for (int m = 0; m < NMAT; ++m) {
                    float sum = 0.0f;
#pragma unroll
                    for (int w = 0; w < NW; ++w) sum += s_red[w][m][r][col];
                    v[m] = sum;
                }
                const float out = (MODE == GEMV_GATE_UP) ? swiglu_ref(v[0], v[NMAT - 1]) : v[0];
                p.y[static_cast<uint64_t>(tl.start + col) * p.out_dim + row] = out;
            }
        }
        if (MODE == GEMV_GATE_UP && p.act_h) {
            // sums over each 32-value sub-block, in ascending order (tile rows are
            // whole sub-blocks: the fused epilogue needs out_dim % 32 == 0)
            __syncthreads();
            for (int t = threadIdx.x; t < 8 * (TILE / 32); t += NW * 32) {
                const int col = t & 7, sb = t >> 3;
                if (!tile_ok || static_cast<uint32_t>(col) >= tl.ncol) continue;
                float sum = 0.0f;
#pragma unroll 8
                for (int i = 0; i < 32; ++i) sum += s_act[MODE == GEMV_GATE_UP ? 32 * sb + i : 0][col];
                p.act_s[static_cast<uint64_t>(tl.start + col) * (p.out_dim / 32) + (tl.row0 / 32 + sb)] = sum;
            }
        }
        __syncthreads();
    }
    cp_async_wait<0>();
}

} // namespace fmb
