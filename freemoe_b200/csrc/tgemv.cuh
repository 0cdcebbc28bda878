// tgemv.cuh -- decode GEMVs of the MoE block on the sm_100a tensor cores
// (tcgen05.mma, A operand and accumulators in TMEM) for GGUF Q4_K experts.
//
// Replaces, for the routed experts of a decode batch, the per-row CPU kernels
// row_dot_q4_k_avx2 (src/kernels.cpp:720-771) inside the engine's per-token
// expert loop (src/engine.cpp:1711-1772):
//   gate/up  act[pair, f] = swiglu(Wg[f] . x[tok], Wu[f] . x[tok])   f < ffn
//   down     part[pair, j] = Wd[j] . act[pair]                        j < d
// Every weight row is streamed from HBM once per tile of up to 8 of its
// expert's tokens.
//
// Exact decoding, as in the mma.sync kernel (gemv_core.cuh): a 4-bit code q
// masked in place is the fp16 subnormal q * 2^-24 (high nibbles: 16 q * 2^-24),
// and one HMUL2 by the 6-bit sub-block scale (sc, or sc / 16) gives
// sc * q * 2^-24 exactly.  x is fp16 (bf16 converts exactly in range).  The
// tensor core sums the exact products of one 256-value block in f32; the block
// scale is applied in f32 when the block's accumulator is read back:
//   y += (2^24 d) * acc_codes - dmin * acc_mins,
// where acc_mins = sum over the 8 sub-blocks of m_j * X_j (X_j = f32 sum of the
// sub-block's x, split into two fp16 planes; m_j exact in fp16) is one more MMA
// per block.  This is the algebra of row_dot_q4_k_avx2 (src/kernels.cpp:
// 759-762); results differ from the reference only in summation order.
//
// Layout of one step (one 256-value block of 128 weight rows x one token tile):
//   raw    the rows' 144 stored bytes of the block, one 2-D TMA box (144 B x
//          128 rows) per matrix through a per-expert tensor map (the maps are
//          written on the device from a host-encoded template, since only the
//          device holds the slot table).
//   A      per thread (= weight row = TMEM lane) 4 chunks of 64 values, each
//          32 TMEM columns of fp16 pairs, written with tcgen05.st; inside a
//          chunk column 2i holds codes (4i, 4i+2) and column 2i+1 codes
//          (4i+1, 4i+3) of the low nibbles (sub-block 2c), columns 16.. the
//          high nibbles (sub-block 2c+1): the MMA's k order is the logical
//          order with every group of four stored (0, 2, 1, 3).
//   B      a 10 KB "image" per (tile, block) built in global memory in the
//          exact shared-memory form the MMA reads (K-major, 128-byte swizzle,
//          16 rows): 4 chunks x 2 KB of x in the same k order, then 2 KB of
//          sub-block sums; one bulk copy per step.
//   gate/up (one x plane): accumulator columns 0-7 = codes x tokens (image rows
//          0-7; rows 8-15 are zero), columns 8-15 = mins x sums (sums image
//          rows 8-15; rows 0-7 are zero), one 16-column accumulator per matrix.
//   down   (act in two fp16 planes hi + lo): a step takes two 128-row tiles of
//          the down matrix (two rows per thread, as gate/up), 16 columns per
//          tile (0-7 hi, 8-15 lo), then one 16-column mins accumulator for both
//          tiles: the sums image holds X in rows 0-7 at K 0-15 and in rows 8-15
//          at K 16-31 (zeros elsewhere), so tile 0's mins MMA (K 0-15) fills
//          columns 0-7 and tile 1's (K 16-31) columns 8-15, both issued in order
//          by one thread.
//
// CTA = 13 warps, one per SM, two pipelines (p = 2 x CTA + w):
//   warp 0        producer of both pipelines: per step one bulk copy of the B
//                 image and one TMA box per matrix, polled without blocking;
//   warps 1-4     MMA issuers, two per pipeline (warp 1 + 2w + i; one thread
//                 each: M = 128, N = 16, K = 16): one per matrix (gate/up) or
//                 row tile (down), each into its own accumulator (fixed
//                 summation order);
//   warps 5-12    converters, four per pipeline (warp v reaches TMEM lanes
//                 32 (v % 4) ..): decode their 32 rows of both matrices (row
//                 tiles) into TMEM,
//                 read the accumulators back and run the epilogue.
// Work split ("stream-K"): the (unit, block) steps of all units are divided
// into equal contiguous ranges, one per pipeline.  A unit split between
// pipelines leaves f32 partial sums in global memory; the last pipeline to
// finish the unit (atomic counter) adds the parts in pipeline order (the same
// result whatever the arrival order) and runs the epilogue.
// Epilogues: gate/up applies the reference SwiGLU and writes the down GEMV's B
// images (act hi/lo planes and sub-block sums); down writes part[pair][j].
// Every wait is bounded; a timeout sets an abort flag, the status word, and
// every role leaves its loop.
#pragma once

#include <cuda.h>

#include <type_traits>

#include "common.cuh"
#include "gemv_core.cuh"
#include "gemv_kernels.cuh"
#include "p2p_flags.cuh"
#include "router_core.cuh"
#include "tcgen05.cuh"

namespace fmb {

constexpr uint32_t TG_ROWS = 128;          // weight rows per unit (TMEM lanes)
constexpr uint32_t TG_NT = 8;              // tokens per tile
constexpr uint32_t TG_IMG = 10240;         // one step's B image: 4 x 2 KB of x + 2 KB of sums
constexpr uint32_t TG_MINS_OFF = 8192;     // sums part of an image
constexpr uint32_t TG_THREADS = 416;       // 13 warps
constexpr uint32_t TG_CONV0 = 5;           // first converter warp
constexpr uint32_t TG_MAX_EXPERTS = 1024;
constexpr uint32_t TG_MAX_CTAS = 160;      // bounds the partial-sum buffer
constexpr uint32_t TG_XS = 3;              // B-image stages per pipeline
constexpr uint32_t TG_RB = 144;            // Q4_K bytes per 256 values
constexpr uint32_t TG_BOX = TG_RB * TG_ROWS; // one matrix's raw box of one step
constexpr uint32_t TG_RAW = 73728;         // raw-ring bytes per pipeline

struct TgParams {
    const uint8_t *const *slots; // per-expert slot base (device array), for the residency check
    uint64_t w_off0, w_off1;     // byte offsets of the kernel's matrices inside a slot
    const CUtensorMap *maps;     // [expert][3] (gate, up, down) raw-weight maps
    uint32_t map0;               // map index of matrix 0 (0: gate/up, 2: down)
    uint32_t out_dim;            // rows of each matrix (multiple of 128)
    uint32_t in_dim;             // K (multiple of 256)
    uint32_t experts;
    const uint32_t *counts;      // tokens per expert
    const uint32_t *offsets;     // first grouped pair of each expert
    const uint8_t *img;          // B images [tile][in_dim / 256][TG_IMG]
    uint8_t *out_img;            // gate/up: the down GEMV's images [tile][out_dim / 256][TG_IMG]
    float *part;                 // down: [pair][out_dim]
    const uint32_t *out_rows;    // down: part row of grouped pair g (NULL: g)
    float *partial;              // stream-K parts [pipeline][2][2][TG_NT][128]
    uint32_t *unit_cnt;          // stream-K arrivals per unit (zero on entry, left zero)
    int *status;
};

enum { TG_GATE_UP = 0, TG_DOWN = 1 };

template <int MODE> struct TgLayout {
    static constexpr uint32_t NMAT = 2;                    // matrices (gate/up) or row tiles (down) per step
    static constexpr uint32_t STAGE = NMAT * TG_BOX;      // one step's raw boxes
    static constexpr uint32_t P = TG_RAW / STAGE;          // raw stages per pipeline
    static constexpr uint32_t OFF_RAW = 2 * TG_XS * TG_IMG;
    static constexpr uint32_t OFF_BAR = OFF_RAW + 2 * TG_RAW;
    static constexpr uint32_t BARS_WG = 24;
    static constexpr uint32_t OFF_MISC = OFF_BAR + 2 * BARS_WG * 8;
    static constexpr uint32_t OFF_TILES = OFF_MISC + 64;
    // token-tile prefix, then (wide mode) tile-pair prefix, experts + 1 words each
    static constexpr uint32_t smem_bytes(uint32_t experts) { return 1024 + OFF_TILES + 8 * (experts + 1); }
    // TMEM columns inside a pipeline's 256
    static constexpr uint32_t ACC_COLS = MODE == TG_GATE_UP ? 32 : 48;  // one buffer's accumulators
    static constexpr uint32_t ACC = 0;                         // [2 buffers][ACC_COLS]
    static constexpr uint32_t ASTG = 2 * ACC_COLS;             // [2 stages][NMAT * 32]
    static constexpr uint32_t MINS = ASTG + 2 * NMAT * 32;     // [2 buffers][NMAT * 8]
    static_assert(MINS + 2 * NMAT * 8 <= 256, "TMEM columns of one pipeline");
    // wide mode (one step stream per CTA, two token tiles per step): half h
    // converts chunks 2h, 2h + 1 into its own two A stages (each stage then takes
    // one chunk per step, so every wait sees every phase); mins shared; one
    // N = 32 MMA covers both tiles (B rows 0-15 tile 0, 16-31 tile 1), so the
    // accumulators hold per matrix (row tile) 32 columns, tile h's at 16 h
    // (gate/up: codes 0-7, mins 8-15; down: hi 0-7, lo 8-15, then the mins
    // accumulator at 64: tile h's row-tile-0 mins at 16 h, row tile 1's at 16 h + 8);
    // x stages of 20 KB (chunk c of tile h at 4096 c + 2048 h, sums of tile h at
    // 16384 + 2048 h); raw ring of both pipelines' space
    static constexpr uint32_t W_ASTG = 0;                  // [half][2 stages][NMAT * 32]
    static constexpr uint32_t W_MINS = 4 * NMAT * 32;
    static constexpr uint32_t W_ACC_COLS = MODE == TG_GATE_UP ? 64 : 96;
    static constexpr uint32_t W_ACC = W_MINS + 2 * NMAT * 8;  // [2 buffers][W_ACC_COLS]
    static_assert(W_ACC + 2 * W_ACC_COLS <= 512, "TMEM columns of a wide CTA");
    static constexpr uint32_t W_XIMG = 2 * TG_IMG;         // one wide x stage
    static_assert(TG_XS * W_XIMG <= OFF_RAW, "wide x stages");
    static constexpr uint32_t PW = 2 * TG_RAW / STAGE;
    static_assert(P == 2 && P * STAGE == TG_RAW, "raw ring");
    static_assert(1024 + OFF_TILES + 8 * (TG_MAX_EXPERTS + 1) <= 227u * 1024u, "shared memory per CTA");
};

// Barriers of one pipeline, in its 24-slot block.
struct TgBars {
    uint64_t *x_full, *x_free, *raw_full, *raw_free, *a_full, *a_free, *acc_full, *acc_free, *drain;
};
__device__ __forceinline__ TgBars tg_bars(uint64_t *base) {
    TgBars b;
    b.x_full = base;
    b.x_free = base + TG_XS;
    b.raw_full = base + 2 * TG_XS;
    b.raw_free = b.raw_full + 4;
    b.a_full = b.raw_free + 4;
    b.a_free = b.a_full + 2;
    b.acc_full = b.a_free + 2;
    b.acc_free = b.acc_full + 2;
    b.drain = b.acc_free + 2;  // one per MMA issuer
    return b;
}

struct TgUnit {
    uint32_t e, rho, tile, pair0, ntok;
};

// Unit u -> (expert, row tile, token tile).  s_tile[e] is the first tile of
// expert e (exclusive prefix of ceil(count / 8)); an expert's units are
// ordered (row tile, token tile) with token tiles fastest, so the tiles that
// read the same weight rows run next to each other (L2 reuse).
__device__ __forceinline__ TgUnit tg_unit(const uint32_t *s_tile, uint32_t experts, uint32_t row_tiles, uint32_t u,
                                          const uint32_t *counts, const uint32_t *offsets) {
    uint32_t lo = 0, hi = experts;
    while (hi - lo > 1) {
        const uint32_t mid = (lo + hi) >> 1;
        if (s_tile[mid] * row_tiles <= u) lo = mid;
        else hi = mid;
    }
    TgUnit g;
    g.e = lo;
    const uint32_t tiles = s_tile[lo + 1] - s_tile[lo];
    const uint32_t local = u - s_tile[lo] * row_tiles;
    g.rho = local / tiles;
    const uint32_t tau = local - g.rho * tiles;
    g.tile = s_tile[lo] + tau;
    g.pair0 = __ldg(offsets + lo) + TG_NT * tau;
    g.ntok = min(TG_NT, __ldg(counts + lo) - TG_NT * tau);
    return g;
}

// Exclusive prefix of token tiles over the experts (one warp); s_tile[E] = total.
__device__ __forceinline__ void tg_tile_prefix(uint32_t *s_tile, const uint32_t *counts, uint32_t experts,
                                               uint32_t lane) {
    uint32_t carry = 0;
    for (uint32_t base = 0; base < experts; base += 32) {
        const uint32_t e = base + lane;
        const uint32_t v = e < experts ? (__ldg(counts + e) + TG_NT - 1) / TG_NT : 0u;
        uint32_t incl = v;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const uint32_t t = __shfl_up_sync(0xFFFFFFFFu, incl, o);
            if (lane >= static_cast<uint32_t>(o)) incl += t;
        }
        if (e < experts) s_tile[e] = carry + incl - v;
        carry += __shfl_sync(0xFFFFFFFFu, incl, 31);
    }
    if (lane == 0) s_tile[experts] = carry;
}

// Wide mode: units are (expert, row tile, pair of token tiles), the pairs of
// expert e numbered from s_pair[e] (exclusive prefix of ceil(tiles / 2)); half
// h of the CTA takes tile 2 tp + h of the pair.  A pair's missing second tile
// reads the first one's image and has no tokens (ntok 0).
__device__ __forceinline__ TgUnit tg_unit_wide(const uint32_t *s_tile, const uint32_t *s_pair, uint32_t experts,
                                               uint32_t row_tiles, uint32_t u, uint32_t half,
                                               const uint32_t *counts, const uint32_t *offsets) {
    uint32_t lo = 0, hi = experts;
    while (hi - lo > 1) {
        const uint32_t mid = (lo + hi) >> 1;
        if (s_pair[mid] * row_tiles <= u) lo = mid;
        else hi = mid;
    }
    TgUnit g;
    g.e = lo;
    const uint32_t npairs = s_pair[lo + 1] - s_pair[lo];
    const uint32_t local = u - s_pair[lo] * row_tiles;
    g.rho = local / npairs;
    const uint32_t tp = local - g.rho * npairs;
    const uint32_t tau = 2 * tp + half, ntiles = s_tile[lo + 1] - s_tile[lo];
    const bool exists = tau < ntiles;
    g.tile = s_tile[lo] + (exists ? tau : 2 * tp);
    g.pair0 = __ldg(offsets + lo) + TG_NT * tau;
    g.ntok = exists ? min(TG_NT, __ldg(counts + lo) - TG_NT * tau) : 0u;
    return g;
}

// Exclusive prefix of ceil(tiles / 2) over the experts (one warp, after
// tg_tile_prefix); s_pair[E] = total.
__device__ __forceinline__ void tg_pair_prefix(uint32_t *s_pair, const uint32_t *s_tile, uint32_t experts,
                                               uint32_t lane) {
    uint32_t carry = 0;
    for (uint32_t base = 0; base < experts; base += 32) {
        const uint32_t e = base + lane;
        const uint32_t v = e < experts ? (s_tile[e + 1] - s_tile[e] + 1) / 2 : 0u;
        uint32_t incl = v;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const uint32_t t = __shfl_up_sync(0xFFFFFFFFu, incl, o);
            if (lane >= static_cast<uint32_t>(o)) incl += t;
        }
        if (e < experts) s_pair[e] = carry + incl - v;
        carry += __shfl_sync(0xFFFFFFFFu, incl, 31);
    }
    if (lane == 0) s_pair[experts] = carry;
}

// Pipeline p's steps are [tg_start(p), tg_start(p + 1)); the pipeline holding step s.
__device__ __forceinline__ uint64_t tg_start(uint64_t p, uint64_t W, uint64_t NP) { return p * W / NP; }
__device__ __forceinline__ uint32_t tg_pipe_of(uint64_t s, uint64_t W, uint64_t NP) {
    return static_cast<uint32_t>(((s + 1) * NP - 1) / W);
}

__device__ __forceinline__ void tma_fence_acquire(const CUtensorMap *map) {
    asm volatile("fence.proxy.tensormap::generic.acquire.gpu [%0], 128;\n" ::"l"(map) : "memory");
}


// Bounded mbarrier wait that also gives up once another role has aborted.
__device__ __forceinline__ bool tg_wait(uint64_t *bar, uint32_t parity, volatile uint32_t *abort_flag, int *status) {
    if (mbar_try_wait(bar, parity)) return true;
    const long long start = clock64();
    for (uint32_t it = 1;; ++it) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((it & 63u) == 0) {
            if (*abort_flag) return false;
            if (clock64() - start > (1ll << 31)) {
                *abort_flag = 1;
                raise_device_status(status, FM_STATUS_INTERNAL_ERROR);
                return false;
            }
        }
    }
}

// The 16-byte Q4_K header of one row: 6-bit scales and mins of the 8
// sub-blocks packed one per byte (src/quant.cpp:63-71), 2^24 d and dmin.
struct TgHdr {
    uint32_t sc_lo, sc_hi, m_lo, m_hi;
    float d, dmin;
};
__device__ __forceinline__ TgHdr tg_hdr(const uint4 h) {
    TgHdr r;
    r.d = fp16_bits_to_f32(static_cast<uint16_t>(h.x & 0xFFFFu)) * 16777216.0f;
    r.dmin = fp16_bits_to_f32(static_cast<uint16_t>(h.x >> 16));
    r.sc_lo = h.y & 0x3F3F3F3Fu;                                           // sc 0..3
    r.m_lo = h.z & 0x3F3F3F3Fu;                                            // m 0..3
    r.sc_hi = (h.w & 0x0F0F0F0Fu) | ((h.y >> 2) & 0x30303030u);            // sc 4..7
    r.m_hi = ((h.w >> 4) & 0x0F0F0F0Fu) | ((h.z >> 2) & 0x30303030u);     // m 4..7
    return r;
}

// A operand of the mins MMA: K 0-7 and 8-15 both m_0..m_7 (fp16, exact).
__device__ __forceinline__ void tg_mins_a(const TgHdr &h, uint32_t (&v)[8]) {
    v[0] = hsub2_u32(prmt(h.m_lo, 0x64646464u, 0x4140u), 0x64006400u);
    v[1] = hsub2_u32(prmt(h.m_lo, 0x64646464u, 0x4342u), 0x64006400u);
    v[2] = hsub2_u32(prmt(h.m_hi, 0x64646464u, 0x4140u), 0x64006400u);
    v[3] = hsub2_u32(prmt(h.m_hi, 0x64646464u, 0x4342u), 0x64006400u);
    v[4] = v[0];
    v[5] = v[1];
    v[6] = v[2];
    v[7] = v[3];
}

// Chunk C (values 64C .. 64C+63 of the block) of one row into 32 fp16x2 words.
template <int C>
__device__ __forceinline__ void tg_unpack(const uint8_t *row, const TgHdr &h, uint32_t (&v)[32]) {
    const uint32_t scw = C < 2 ? h.sc_lo : h.sc_hi;
    constexpr uint32_t SEL0 = (C & 1) ? 0x4242u : 0x4040u, SEL1 = (C & 1) ? 0x4343u : 0x4141u;
    const uint32_t hs_lo = hsub2_u32(prmt(scw, 0x64646464u, SEL0), 0x64006400u);            // (sc, sc)
    const uint32_t hs_hi = hfma2_u32(prmt(scw, 0x64646464u, SEL1), 0x2C002C00u, 0xD400D400u); // (sc/16, sc/16)
    const uint4 qa = *reinterpret_cast<const uint4 *>(row + 16 + 32 * C);
    const uint4 qb = *reinterpret_cast<const uint4 *>(row + 32 + 32 * C);
    const uint32_t w[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const uint32_t s = w[i] >> 8;
        v[2 * i] = hmul2_u32(w[i] & 0x000F000Fu, hs_lo);
        v[2 * i + 1] = hmul2_u32(s & 0x000F000Fu, hs_lo);
        v[16 + 2 * i] = hmul2_u32(w[i] & 0x00F000F0u, hs_hi);
        v[16 + 2 * i + 1] = hmul2_u32(s & 0x00F000F0u, hs_hi);
    }
}

// Byte offset of fp16 element k (0..63) of row n (0..15) inside a 2 KB
// K-major 128-byte-swizzled chunk image.
__host__ __device__ __forceinline__ uint32_t tg_sw_off(uint32_t n, uint32_t k) {
    return (n >> 3) * 1024u + (n & 7u) * 128u + ((((k >> 3) ^ (n & 7u)) & 7u) << 4) + (k & 7u) * 2u;
}


template <int MODE, bool WIDE>
__global__ void __launch_bounds__(TG_THREADS, 1) tgemv_kernel(const TgParams p) {
    using L = TgLayout<MODE>;
    constexpr int NMAT = 2;
    constexpr bool DN = MODE == TG_DOWN;
    extern __shared__ uint8_t tg_smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(tg_smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + L::OFF_BAR);
    uint32_t *misc = reinterpret_cast<uint32_t *>(smem + L::OFF_MISC); // [0] TMEM base [1] abort [2] bad slot [3,4] last
    uint32_t *s_tile = reinterpret_cast<uint32_t *>(smem + L::OFF_TILES);
    uint32_t *s_pair = s_tile + p.experts + 1;
    volatile uint32_t *abort_flag = misc + 1;
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
    const uint32_t E = p.experts;

    if (threadIdx.x == 0) {
        misc[1] = 0;
        misc[2] = 0;
    }
    __syncthreads();
    if (warp == 1) {
        tg_tile_prefix(s_tile, p.counts, E, lane);
        if (WIDE) {
            __syncwarp();
            tg_pair_prefix(s_pair, s_tile, E, lane);
        }
    } else if (warp == 3) {
        // every expert with tokens needs a resident slot with 16-byte aligned matrices
        for (uint32_t e = lane; e < E; e += 32) {
            if (__ldg(p.counts + e) == 0) continue;
            const uintptr_t base = reinterpret_cast<uintptr_t>(p.slots[e]);
            if (!base) atomicCAS(misc + 2, 0u, static_cast<uint32_t>(FM_STATUS_EXPERT_EXECUTION_MISMATCH));
            else if ((base + p.w_off0) % 16 || (base + p.w_off1) % 16)
                atomicCAS(misc + 2, 0u, static_cast<uint32_t>(FM_STATUS_INVALID_ARGUMENT));
        }
    } else if (warp == 2 && lane == 0) {
        for (uint32_t w = 0; w < 2; ++w) {
            const TgBars b = tg_bars(bars + w * L::BARS_WG);
            for (uint32_t q = 0; q < TG_XS; ++q) {
                mbar_init(&b.x_full[q], 1);
                mbar_init(&b.x_free[q], 2); // both issuers
            }
            // wide: the raw ring, x stages and accumulators of block 0 serve both
            // halves; block h's two A stages are half h's
            for (uint32_t q = 0; q < 4; ++q) {
                mbar_init(&b.raw_full[q], 1);
                mbar_init(&b.raw_free[q], WIDE ? 8 : 4); // the converter warps reading the stage
            }
            for (uint32_t q = 0; q < 2; ++q) {
                mbar_init(&b.a_full[q], 4);                // the warps converting the chunk
                mbar_init(&b.a_free[q], 2);                // both issuers read every chunk
                mbar_init(&b.acc_full[q], 2);
                mbar_init(&b.acc_free[q], WIDE ? 8 : 4);   // the warps reading the accumulators back
                mbar_init(&b.drain[q], 1);
            }
        }
        fence_barrier_init();
    }
    __syncthreads();
    if (misc[2]) {
        if (threadIdx.x == 0) raise_device_status(p.status, static_cast<int>(misc[2]));
        return;
    }
    const uint32_t row_tiles = p.out_dim / (DN ? 2 * TG_ROWS : TG_ROWS), nb = p.in_dim / 256;
    const uint64_t W = static_cast<uint64_t>(WIDE ? s_pair[E] : s_tile[E]) * row_tiles * nb;
    if (W == 0) return;

    if (warp == 0) {
        tmem_alloc(misc, 512);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = misc[0];
    const uint64_t NP = WIDE ? gridDim.x : 2ull * gridDim.x;

    if (WIDE && warp == 0) {
        // ---- wide producer: one step stream, both halves' images, one raw box set
        if (lane == 0) {
            const uint64_t s0 = tg_start(blockIdx.x, W, NP), s1 = tg_start(blockIdx.x + 1ull, W, NP);
            const TgBars b0 = tg_bars(bars);
            uint32_t j = 0, cur_u = 0xFFFFFFFFu;
            TgUnit g0{}, g1{};
            long long last_progress = clock64();
            while (s0 + j < s1 && !*abort_flag) {
                const uint32_t xs = j % TG_XS, rs = j % L::PW;
                if (!mbar_test_wait(&b0.x_free[xs], ((j / TG_XS) & 1u) ^ 1u) ||
                    !mbar_test_wait(&b0.raw_free[rs], ((j / L::PW) & 1u) ^ 1u)) {
                    __nanosleep(64);
                    if (clock64() - last_progress > (1ll << 31)) {
                        *abort_flag = 1;
                        raise_device_status(p.status, FM_STATUS_INTERNAL_ERROR);
                    }
                    continue;
                }
                const uint64_t s = s0 + j;
                const uint32_t u = static_cast<uint32_t>(s / nb), b = static_cast<uint32_t>(s - static_cast<uint64_t>(u) * nb);
                if (u != cur_u) {
                    const uint32_t old_e = cur_u == 0xFFFFFFFFu ? 0xFFFFFFFFu : g0.e;
                    g0 = tg_unit_wide(s_tile, s_pair, E, row_tiles, u, 0, p.counts, p.offsets);
                    g1 = tg_unit_wide(s_tile, s_pair, E, row_tiles, u, 1, p.counts, p.offsets);
                    if (g0.e != old_e)
#pragma unroll
                        for (int m = 0; m < (DN ? 1 : NMAT); ++m) tma_fence_acquire(p.maps + 3 * g0.e + p.map0 + m);
                    cur_u = u;
                }
                // both tiles' images interleaved chunk by chunk (one N = 32 B operand)
                uint8_t *xdst = smem + xs * L::W_XIMG;
                mbar_expect_tx(&b0.x_full[xs], L::W_XIMG);
#pragma unroll
                for (uint32_t w = 0; w < 2; ++w) {
                    const uint8_t *src = p.img + (static_cast<uint64_t>(w ? g1.tile : g0.tile) * nb + b) * TG_IMG;
#pragma unroll
                    for (uint32_t c = 0; c < 5; ++c)
                        bulk_g2s(xdst + c * 4096u + w * 2048u, src + c * 2048u, 2048u, &b0.x_full[xs]);
                }
                uint8_t *rdst = smem + L::OFF_RAW + rs * L::STAGE;
                mbar_expect_tx(&b0.raw_full[rs], L::STAGE);
#pragma unroll
                for (int m = 0; m < NMAT; ++m)
                    tma_load_2d(rdst + m * TG_BOX, p.maps + 3 * g0.e + p.map0 + (DN ? 0 : m),
                                static_cast<int32_t>(b * TG_RB),
                                static_cast<int32_t>((DN ? 2 * g0.rho + m : g0.rho) * TG_ROWS), &b0.raw_full[rs]);
                ++j;
                last_progress = clock64();
            }
            // copies still in flight must land before the CTA's shared memory goes away
            for (uint32_t q = j > TG_XS ? j - TG_XS : 0; q < j; ++q)
                (void)mbar_wait(&b0.x_full[q % TG_XS], (q / TG_XS) & 1u);
            for (uint32_t q = j > L::PW ? j - L::PW : 0; q < j; ++q)
                (void)mbar_wait(&b0.raw_full[q % L::PW], (q / L::PW) & 1u);
        }
    } else if (warp == 0) {
        // ---- producer of both pipelines ----------------------------------------
        if (lane == 0) {
            uint64_t s0[2], s1[2];
            uint32_t j[2] = {0, 0}, cur_u[2] = {0xFFFFFFFFu, 0xFFFFFFFFu};
            TgUnit g[2];
            TgBars bw[2];
            for (uint32_t w = 0; w < 2; ++w) {
                s0[w] = tg_start(2ull * blockIdx.x + w, W, NP);
                s1[w] = tg_start(2ull * blockIdx.x + w + 1, W, NP);
                bw[w] = tg_bars(bars + w * L::BARS_WG);
            }
            long long last_progress = clock64();
            while ((s0[0] + j[0] < s1[0] || s0[1] + j[1] < s1[1]) && !*abort_flag) {
                bool progress = false;
#pragma unroll
                for (uint32_t w = 0; w < 2; ++w) {
                    if (s0[w] + j[w] >= s1[w]) continue;
                    const uint32_t xs = j[w] % TG_XS, rs = j[w] % L::P;
                    if (!mbar_test_wait(&bw[w].x_free[xs], ((j[w] / TG_XS) & 1u) ^ 1u) ||
                        !mbar_test_wait(&bw[w].raw_free[rs], ((j[w] / L::P) & 1u) ^ 1u))
                        continue;
                    const uint64_t s = s0[w] + j[w];
                    const uint32_t u = static_cast<uint32_t>(s / nb), b = static_cast<uint32_t>(s - static_cast<uint64_t>(u) * nb);
                    if (u != cur_u[w]) {
                        const uint32_t old_e = cur_u[w] == 0xFFFFFFFFu ? 0xFFFFFFFFu : g[w].e;
                        g[w] = tg_unit(s_tile, E, row_tiles, u, p.counts, p.offsets);
                        if (g[w].e != old_e)
#pragma unroll
                            for (int m = 0; m < (DN ? 1 : NMAT); ++m)
                                tma_fence_acquire(p.maps + 3 * g[w].e + p.map0 + m);
                        cur_u[w] = u;
                    }
                    uint8_t *xdst = smem + (w * TG_XS + xs) * TG_IMG;
                    mbar_expect_tx(&bw[w].x_full[xs], TG_IMG);
                    bulk_g2s(xdst, p.img + (static_cast<uint64_t>(g[w].tile) * nb + b) * TG_IMG, TG_IMG,
                             &bw[w].x_full[xs]);
                    uint8_t *rdst = smem + L::OFF_RAW + w * TG_RAW + rs * L::STAGE;
                    mbar_expect_tx(&bw[w].raw_full[rs], L::STAGE);
#pragma unroll
                    for (int m = 0; m < NMAT; ++m)
                        tma_load_2d(rdst + m * TG_BOX, p.maps + 3 * g[w].e + p.map0 + (DN ? 0 : m),
                                    static_cast<int32_t>(b * TG_RB),
                                    static_cast<int32_t>((DN ? 2 * g[w].rho + m : g[w].rho) * TG_ROWS),
                                    &bw[w].raw_full[rs]);
                    ++j[w];
                    progress = true;
                }
                if (progress) {
                    last_progress = clock64();
                } else {
                    __nanosleep(64);
                    if (clock64() - last_progress > (1ll << 31)) {
                        *abort_flag = 1;
                        raise_device_status(p.status, FM_STATUS_INTERNAL_ERROR);
                    }
                }
            }
            // copies still in flight must land before the CTA's shared memory goes away
            for (uint32_t w = 0; w < 2; ++w) {
                for (uint32_t q = j[w] > TG_XS ? j[w] - TG_XS : 0; q < j[w]; ++q)
                    (void)mbar_wait(&bw[w].x_full[q % TG_XS], (q / TG_XS) & 1u);
                for (uint32_t q = j[w] > L::P ? j[w] - L::P : 0; q < j[w]; ++q)
                    (void)mbar_wait(&bw[w].raw_full[q % L::P], (q / L::P) & 1u);
            }
        }
    } else if (warp < TG_CONV0) {
        // ---- MMA issuers: warp 1 + 2w + i = issuer i of pipeline w --------------
        // (wide: warp 1 + 2w + i = issuer i of half w, both halves on the shared A)
        // (wide: warps 1 + i, one per matrix or row tile, N = 32 over both tiles)
        const uint32_t wg = WIDE ? 0u : (warp - 1) >> 1, iss = WIDE ? warp - 1 : (warp - 1) & 1u;
        if (lane == 0 && (!WIDE || warp < 3)) {
            const uint64_t pipe = WIDE ? blockIdx.x : 2ull * blockIdx.x + wg;
            const uint64_t s0 = tg_start(pipe, W, NP), s1 = tg_start(pipe + 1, W, NP);
            const TgBars bw = tg_bars(bars + wg * L::BARS_WG);       // x images, accumulators
            const TgBars ba = bw;                                      // A stages (narrow)
            const uint32_t idesc = idesc_f16_m128(WIDE ? 32 : 16);
            constexpr uint32_t ACW = WIDE ? L::W_ACC_COLS : L::ACC_COLS;  // one accumulator buffer
            constexpr uint32_t MW = WIDE ? 32u : 16u;                     // columns per matrix / row tile
            const uint32_t t_acc = WIDE ? tmem + L::W_ACC : tmem + wg * 256u + L::ACC;
            const uint32_t t_a = WIDE ? tmem + L::W_ASTG : tmem + wg * 256u + L::ASTG;
            const uint32_t t_m = WIDE ? tmem + L::W_MINS : tmem + wg * 256u + L::MINS;
            uint32_t j = 0;
            bool issued = false;
            for (uint64_t s = s0; s < s1; ++s, ++j) {
                const uint32_t st = j % TG_XS, ab = j & 1u;
                if (!tg_wait(&bw.x_full[st], (j / TG_XS) & 1u, abort_flag, p.status)) break;
                if (!tg_wait(&bw.acc_free[ab], ((j >> 1) & 1u) ^ 1u, abort_flag, p.status)) break;
                tc_fence_after();
                const uint32_t xbase = smem_u32(smem + (WIDE ? st * L::W_XIMG : (wg * TG_XS + st) * TG_IMG));
                const uint64_t bd0 = smem_desc_sw128(xbase);
                const uint32_t acc = t_acc + ab * ACW + iss * MW; // matrix / row tile iss
                bool ok = true;
#pragma unroll
                for (uint32_t c = 0; c < 4; ++c) {
                    // the chunk's A stage: narrow, stage cc % 2 of the pipeline's ring;
                    // wide, stage c % 2 of the converting half c / 2 (one use per step)
                    const uint32_t cc = 4 * j + c, as = WIDE ? (c & 1u) : (cc & 1u);
                    const uint32_t aph = WIDE ? (j & 1u) : ((cc >> 1) & 1u);
                    const TgBars bh = WIDE ? tg_bars(bars + (c >> 1) * L::BARS_WG) : ba;
                    if (!tg_wait(&bh.a_full[as], aph, abort_flag, p.status)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t astg = t_a + (WIDE ? 2 * (c >> 1) + as : as) * (NMAT * 32u) + iss * 32u;
                    constexpr uint32_t CHUNK_B = WIDE ? 4096u : 2048u; // bytes of one chunk's B rows
#pragma unroll
                    for (uint32_t kk = 0; kk < 4; ++kk)
                        mma_f16_ts(acc, astg + kk * 8u, bd0 + ((c * CHUNK_B + kk * 32u) >> 4), idesc, (c | kk) != 0u);
                    if (c == 0) {
                        // the block's mins (their A was stored before chunk 0's arrival)
                        const uint64_t bm = bd0 + ((4 * CHUNK_B) >> 4);
                        const uint32_t ma = t_m + ab * (NMAT * 8u);
                        if (!DN) {
                            mma_f16_ts(acc, ma + iss * 8u, bm, idesc, 1u);
                        } else if (iss == 0) {
                            // both row tiles into one accumulator, in order: tile 0 from
                            // K 0-15 of the sums image (columns 0-7), tile 1 from K 16-31
                            // (columns 8-15)
                            const uint32_t am = t_acc + ab * ACW + 2 * MW;
                            mma_f16_ts(am, ma, bm, idesc, 0u);
                            mma_f16_ts(am, ma + 8u, bm + (32u >> 4), idesc, 1u);
                        }
                    }
                    issued = true;
                    tc_commit(&bh.a_free[as]);
                }
                if (!ok) break;
                tc_commit(&bw.acc_full[ab]);
                tc_commit(&bw.x_free[st]);
            }
            if (issued) {
                // every MMA issued must finish before TMEM is released
                tc_commit(&bw.drain[iss]);
                (void)mbar_wait(&bw.drain[iss], 0);
            }
        }
    } else {
        // ---- converters, read-back and epilogue ---------------------------------
        // (wide: warps of half w convert chunks 2w, 2w + 1 of the shared step and
        // read back half w's accumulators)
        const uint32_t wg = (warp - TG_CONV0) >> 2, wq = warp & 3u;
        const uint32_t r = wq * 32u + lane; // weight row inside the unit = TMEM lane
        const uint64_t pipe = WIDE ? blockIdx.x : 2ull * blockIdx.x + wg; // stream-K range
        const uint64_t s0 = tg_start(pipe, W, NP), s1 = tg_start(pipe + 1, W, NP);
        const uint32_t my = static_cast<uint32_t>(s1 - s0);
        const TgBars bw = tg_bars(bars + wg * L::BARS_WG);            // A stages (wide: this half's)
        const TgBars ba = WIDE ? tg_bars(bars) : bw;                   // raw ring, accumulators
        const uint32_t lq = (wq * 32u) << 16;                          // this warp's TMEM lanes
        const uint32_t t_acc = (WIDE ? tmem + L::W_ACC : tmem + wg * 256u + L::ACC) + lq;
        constexpr uint32_t ACW = WIDE ? L::W_ACC_COLS : L::ACC_COLS;  // one accumulator buffer
        const uint32_t t_a = (WIDE ? tmem + L::W_ASTG : tmem + wg * 256u + L::ASTG) + lq;
        const uint32_t t_m = (WIDE ? tmem + L::W_MINS : tmem + wg * 256u + L::MINS) + lq;
        const uint8_t *raw = smem + L::OFF_RAW + (WIDE ? 0u : wg * TG_RAW) + r * TG_RB;
        constexpr uint32_t NRAW = WIDE ? L::PW : L::P;                 // raw stages
        // stream-K parts of this warp's accumulators: pipeline q's at q (wide: 2 q + half)
        auto part_of = [&](uint64_t q) -> uint64_t { return WIDE ? 2 * q + wg : q; };
        const uint32_t first_u = static_cast<uint32_t>(s0 / nb);
        const int bar_sk = 1 + wg;
        // (unit, block) of the next step to read back, advanced by one per read-back
        uint32_t rb_u = first_u, rb_b = static_cast<uint32_t>(s0 - static_cast<uint64_t>(first_u) * nb);

        float tot[NMAT][TG_NT];
#pragma unroll
        for (int m = 0; m < NMAT; ++m)
#pragma unroll
            for (uint32_t n = 0; n < TG_NT; ++n) tot[m][n] = 0.0f;
        float pd[2] = {0.f, 0.f}, pdm[2] = {0.f, 0.f}; // scales of the step waiting for read-back

        // Read-back of step j (its accumulators) into tot, then the unit's
        // epilogue when j is the unit's last step in this pipeline.
        auto readback = [&](uint32_t j) -> bool {
            const uint32_t ab = j & 1u;
            if (!tg_wait(&ba.acc_full[ab], (j >> 1) & 1u, abort_flag, p.status)) return false;
            tc_fence_after();
            uint32_t a[32];
            if (WIDE) {
                // this tile's 16 columns of each matrix (row tile)
                uint32_t a0[16], a1[16];
                tmem_ld16(t_acc + ab * ACW + wg * 16u, a0);
                tmem_ld16(t_acc + ab * ACW + 32u + wg * 16u, a1);
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    a[i] = a0[i];
                    a[16 + i] = a1[i];
                }
            } else {
                tmem_ld32(t_acc + ab * ACW, a);
            }
            if (!DN) {
                tmem_wait_ld();
#pragma unroll
                for (int m = 0; m < NMAT; ++m)
#pragma unroll
                    for (uint32_t n = 0; n < TG_NT; ++n)
                        tot[m][n] = fmaf(pd[m], __uint_as_float(a[16 * m + n]),
                                         fmaf(-pdm[m], __uint_as_float(a[16 * m + 8 + n]), tot[m][n]));
            } else {
                uint32_t mn[8], mn1[8];
                const uint32_t mcol = WIDE ? 64u + wg * 16u : 32u;
                tmem_ld8(t_acc + ab * ACW + mcol, mn);
                tmem_ld8(t_acc + ab * ACW + mcol + 8u, mn1);
                tmem_wait_ld();
#pragma unroll
                for (uint32_t n = 0; n < TG_NT; ++n) {
                    tot[0][n] = fmaf(pd[0], __uint_as_float(a[n]) + __uint_as_float(a[8 + n]),
                                     fmaf(-pdm[0], __uint_as_float(mn[n]), tot[0][n]));
                    tot[1][n] = fmaf(pd[1], __uint_as_float(a[16 + n]) + __uint_as_float(a[24 + n]),
                                     fmaf(-pdm[1], __uint_as_float(mn1[n]), tot[1][n]));
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&ba.acc_free[ab]);

            const uint32_t u = rb_u, b = rb_b;
            if (++rb_b == nb) {
                rb_b = 0;
                ++rb_u;
            }
            if (b != nb - 1 && j != my - 1) return true;
            // ---- the unit's epilogue --------------------------------------------
            const TgUnit g = WIDE ? tg_unit_wide(s_tile, s_pair, E, row_tiles, u, wg, p.counts, p.offsets)
                                  : tg_unit(s_tile, E, row_tiles, u, p.counts, p.offsets);
            const uint64_t us = static_cast<uint64_t>(u) * nb;
            const bool whole = (s0 <= us) && (us + nb <= s1);
            float val[NMAT][TG_NT];
#pragma unroll
            for (int m = 0; m < NMAT; ++m)
#pragma unroll
                for (uint32_t n = 0; n < TG_NT; ++n) {
                    val[m][n] = tot[m][n];
                    tot[m][n] = 0.0f;
                }
            // wide: the missing second tile of a pair (every pipeline holding the
            // unit skips it alike: no parts, no counter, no output)
            if (WIDE && g.ntok == 0) return true;
            if (!whole) {
                // the pipelines holding the unit's steps, in order (pipelines with
                // empty ranges are skipped): pf, then the holder of the next step
                // after each one's range; with at least one step per pipeline
                // (dense) simply pf .. the holder of the unit's last step
                const uint32_t pf = tg_pipe_of(us, W, NP);
                const bool dense = W >= NP;
                uint32_t nparts = 1;
                if (dense) {
                    nparts = tg_pipe_of(us + nb - 1, W, NP) - pf + 1;
                } else {
                    for (uint32_t q = pf;; ++nparts) {
                        const uint64_t e = tg_start(q + 1ull, W, NP);
                        if (e >= us + nb) break;
                        q = tg_pipe_of(e, W, NP);
                    }
                }
                const uint32_t slot = (u == first_u) ? 0u : 1u;
                float *mine = p.partial + (part_of(pipe) * 2 + slot) * (NMAT * TG_NT * TG_ROWS);
#pragma unroll
                for (int m = 0; m < NMAT; ++m)
#pragma unroll
                    for (uint32_t n = 0; n < TG_NT; ++n)
                        if (n < g.ntok) __stcg(mine + (m * TG_NT + n) * TG_ROWS + r, val[m][n]);
                __threadfence();
                named_bar_sync(bar_sk, 128);
                if (wq == 1 && lane == 0) {
                    const uint32_t ci = WIDE ? 2 * u + wg : u;
                    const uint32_t old = atomicAdd(p.unit_cnt + ci, 1u);
                    const uint32_t last = old == nparts - 1 ? 1u : 0u;
                    if (last) p.unit_cnt[ci] = 0; // every part has arrived: ready for the next call
                    misc[3 + wg] = last;
                }
                named_bar_sync(bar_sk, 128);
                if (misc[3 + wg] == 0) return true;
                __threadfence();
                // every part, this pipeline's included, from the buffer in pipeline order
#pragma unroll
                for (int m = 0; m < NMAT; ++m)
#pragma unroll
                    for (uint32_t n = 0; n < TG_NT; ++n) val[m][n] = 0.0f;
                // slot 0 holds a pipeline's first unit: every holder after pf starts
                // inside this unit
                const uint32_t slot_pf = (u == static_cast<uint32_t>(tg_start(pf, W, NP) / nb)) ? 0u : 1u;
                for (uint32_t q = pf, i = 0; i < nparts;
                     ++i, q = dense ? q + 1 : tg_pipe_of(tg_start(q + 1ull, W, NP), W, NP)) {
                    const uint32_t qslot = i == 0 ? slot_pf : 0u;
                    const float *src = p.partial + (part_of(q) * 2 + qslot) * (NMAT * TG_NT * TG_ROWS);
#pragma unroll
                    for (int m = 0; m < NMAT; ++m)
#pragma unroll
                        for (uint32_t n = 0; n < TG_NT; ++n)
                            if (n < g.ntok) val[m][n] += __ldcg(src + (m * TG_NT + n) * TG_ROWS + r);
                }
            }
            if (!DN) {
                const uint32_t f = g.rho * TG_ROWS + r; // output feature
                // SwiGLU (include/fm/activation.hpp:62-84), then the down GEMV's B image:
                // act hi plane in rows 0-7, lo plane in rows 8-15, at the staged k
                // position of feature f; sub-block sums of 32 features (one warp)
                const uint32_t nbd = p.out_dim / 256, bd = f >> 8, cd = (f & 255u) >> 6;
                const uint32_t kpos = xplane_pos(f & 63u);
                uint8_t *img = p.out_img + (static_cast<uint64_t>(g.tile) * nbd + bd) * TG_IMG;
                uint8_t *chunk = img + cd * 2048u;
                float act[TG_NT];
#pragma unroll
                for (uint32_t n = 0; n < TG_NT; ++n) {
                    act[n] = n < g.ntok ? swiglu_ref(val[0][n], val[NMAT - 1][n]) : 0.0f;
                    const __half h = __float2half_rn(act[n]);
                    const __half l = __float2half_rn(act[n] - __half2float(h));
                    *reinterpret_cast<__half *>(chunk + tg_sw_off(n, kpos)) = h;
                    *reinterpret_cast<__half *>(chunk + tg_sw_off(8 + n, kpos)) = l;
                }
                // sums image of the down GEMV: X (hi at K j, lo at K 8 + j) in rows 0-7 for
                // its first row tile and (K 16 + j, 24 + j) in rows 8-15 for its second,
                // zeros in the other half of each row
                const uint32_t jsub = (f & 255u) >> 5;
                const __half z = __float2half_rn(0.0f);
#pragma unroll
                for (uint32_t n = 0; n < TG_NT; ++n) {
                    const float X = warp_sum(act[n]);
                    if (lane == 0) {
                        const __half h = __float2half_rn(X);
                        const __half l = __float2half_rn(X - __half2float(h));
                        uint8_t *mi = img + TG_MINS_OFF;
                        *reinterpret_cast<__half *>(mi + tg_sw_off(n, jsub)) = h;
                        *reinterpret_cast<__half *>(mi + tg_sw_off(n, 8 + jsub)) = l;
                        *reinterpret_cast<__half *>(mi + tg_sw_off(n, 16 + jsub)) = z;
                        *reinterpret_cast<__half *>(mi + tg_sw_off(n, 24 + jsub)) = z;
                        *reinterpret_cast<__half *>(mi + tg_sw_off(8 + n, jsub)) = z;
                        *reinterpret_cast<__half *>(mi + tg_sw_off(8 + n, 8 + jsub)) = z;
                        *reinterpret_cast<__half *>(mi + tg_sw_off(8 + n, 16 + jsub)) = h;
                        *reinterpret_cast<__half *>(mi + tg_sw_off(8 + n, 24 + jsub)) = l;
                    }
                }
            } else {
#pragma unroll
                for (uint32_t n = 0; n < TG_NT; ++n)
                    if (n < g.ntok) {
                        const uint32_t row = p.out_rows ? __ldg(p.out_rows + g.pair0 + n) : g.pair0 + n;
#pragma unroll
                        for (int m = 0; m < NMAT; ++m)
                            p.part[static_cast<uint64_t>(row) * p.out_dim + (2 * g.rho + m) * TG_ROWS + r] = val[m][n];
                    }
            }
            return true;
        };

        // step j is converted in iteration j and read back in iteration j + 1
        for (uint32_t j = 0; j <= my; ++j) {
            if (j == my) {
                if (my > 0) (void)readback(j - 1);
                break;
            }
            const uint32_t rs = j % NRAW;
            if (!tg_wait(&ba.raw_full[rs], (j / NRAW) & 1u, abort_flag, p.status)) break;
            const uint8_t *rows[2];
            TgHdr hd[2];
#pragma unroll
            for (int m = 0; m < 2; ++m) {
                rows[m] = raw + rs * L::STAGE + m * TG_BOX;
                hd[m] = tg_hdr(*reinterpret_cast<const uint4 *>(rows[m]));
            }
            if (!WIDE) {
                // mins A of this step (its buffer was last read by step j - 2's MMAs,
                // whose accumulators have been read back)
#pragma unroll
                for (int m = 0; m < NMAT; ++m) {
                    uint32_t mv[8];
                    tg_mins_a(hd[m], mv);
                    tmem_st8(t_m + (j & 1u) * (NMAT * 8u) + m * 8u, mv);
                }
            }
            bool ok = true;
#pragma unroll
            for (uint32_t c = 0; c < 4; ++c) {
                if (WIDE && (c >> 1) != wg) continue; // the other half's chunk
                // A stage (as the issuers): wide, this half's own pair of stages
                const uint32_t cc = 4 * j + c, as = WIDE ? (c & 1u) : (cc & 1u);
                const uint32_t aph = WIDE ? (j & 1u) : ((cc >> 1) & 1u);
                const TgBars &bh = WIDE ? bw : ba;
                if (!tg_wait(&bh.a_free[as], aph ^ 1u, abort_flag, p.status)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                if (WIDE && c == 0) {
                    // mins A of this step: its buffer was last read by step j - 2's mins
                    // MMAs, issued before chunk 0 of step j - 1, whose stage this wait freed
#pragma unroll
                    for (int m = 0; m < NMAT; ++m) {
                        uint32_t mv[8];
                        tg_mins_a(hd[m], mv);
                        tmem_st8(t_m + (j & 1u) * (NMAT * 8u) + m * 8u, mv);
                    }
                }
                const uint32_t astg = t_a + (WIDE ? 2 * wg + as : as) * (NMAT * 32u);
#pragma unroll
                for (int m = 0; m < NMAT; ++m) {
                    uint32_t v[32];
                    if (c == 0) tg_unpack<0>(rows[m], hd[m], v);
                    else if (c == 1) tg_unpack<1>(rows[m], hd[m], v);
                    else if (c == 2) tg_unpack<2>(rows[m], hd[m], v);
                    else tg_unpack<3>(rows[m], hd[m], v);
                    tmem_st32(astg + 32u * m, v);
                }
                tmem_wait_st();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&bh.a_full[as]);
            }
            if (!ok) break;
            __syncwarp(); // every lane has read the raw stage
            if (lane == 0) mbar_arrive(&ba.raw_free[rs]);
            if (j > 0 && !readback(j - 1)) break;
#pragma unroll
            for (int m = 0; m < NMAT; ++m) {
                pd[m] = hd[m].d;
                pdm[m] = hd[m].dmin;
            }
        }
    }

    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, 512);
    }
}

struct TgMapArgs {
    CUtensorMap tmpl_gu, tmpl_dn;  // host-encoded templates of the gate/up and down matrices
    const uint8_t *const *slots;
    uint64_t up_off, down_off;
    CUtensorMap *maps;             // [expert][gate, up, down]
    uint32_t *cnt;                 // stream-K counters to clear
    uint32_t n_cnt;
};

// Grid-wide part of the image launch: the per-expert raw-weight tensor maps (a
// copy of the template with its global address replaced by the expert's
// matrix through tensormap.replace; experts without tokens or without a usable
// slot are skipped, the GEMV kernels report those) and the cleared stream-K
// counters.  `counts` may point to shared memory.
__device__ __forceinline__ void tg_maps_and_counters(const TgMapArgs &ma, const uint32_t *counts, uint32_t experts) {
    const uint32_t gid = blockIdx.x * blockDim.x + threadIdx.x, gsz = gridDim.x * blockDim.x;
    for (uint32_t i = gid; i < ma.n_cnt; i += gsz) ma.cnt[i] = 0;
    for (uint32_t id = gid; id < 3 * experts; id += gsz) {
        const uint32_t e = id / 3, m = id - 3 * e;
        const uint8_t *base = ma.slots[e];
        const uint64_t off = m == 0 ? 0 : (m == 1 ? ma.up_off : ma.down_off);
        if (counts[e] == 0 || !base || (reinterpret_cast<uintptr_t>(base) + off) % 16) continue;
        CUtensorMap *dst = ma.maps + id;
        const uint4 *src = reinterpret_cast<const uint4 *>(m == 2 ? &ma.tmpl_dn : &ma.tmpl_gu);
#pragma unroll
        for (int i = 0; i < 8; ++i) reinterpret_cast<uint4 *>(dst)[i] = src[i];
        asm volatile("tensormap.replace.tile.global_address.global.b1024.b64 [%0], %1;\n" ::"l"(dst),
                     "l"(reinterpret_cast<uint64_t>(base + off))
                     : "memory");
        asm volatile("fence.proxy.tensormap::generic.release.gpu;\n" ::: "memory");
    }
}

struct TgImageSmem {
    float x[TG_NT][256];
    float sum[TG_NT][8];
};

// CTA (tile, block) of the image launch writes the 16 x 256 staged x values of
// its tile's tokens (rows >= the tile's tokens and rows 8-15 zero) and the
// sub-block sums (rows 8-15 of the sums part, as hi and lo fp16 planes; rows
// 0-7 zero).  s_tile holds the exclusive tile prefix over the experts;
// counts / offsets / pairs may point to shared memory.
template <typename XT>
__device__ __forceinline__ void tg_image_block(const XT *__restrict__ x, uint32_t d, const uint32_t *counts,
                                               const uint32_t *offsets, const uint32_t *pairs, uint32_t top_k,
                                               uint32_t experts, uint32_t max_tiles, const uint32_t *s_tile,
                                               uint8_t *__restrict__ img, TgImageSmem &sm) {
    const uint32_t nb = d / 256;
    const uint32_t tile = blockIdx.x / nb, b = blockIdx.x - tile * nb;
    if (tile >= s_tile[experts] || tile >= max_tiles) return;
    uint32_t lo = 0, hi = experts;
    while (hi - lo > 1) {
        const uint32_t mid = (lo + hi) >> 1;
        if (s_tile[mid] <= tile) lo = mid;
        else hi = mid;
    }
    const uint32_t tau = tile - s_tile[lo];
    const uint32_t pair0 = offsets[lo] + TG_NT * tau, ntok = min(TG_NT, counts[lo] - TG_NT * tau);
    // the tile's x values of this block, as floats
    for (uint32_t i = threadIdx.x; i < TG_NT * 256; i += blockDim.x) {
        const uint32_t n = i >> 8, k = i & 255u;
        float v = 0.0f;
        if (n < ntok) {
            const uint32_t tok = pairs[pair0 + n] / top_k;
            const XT xv = x[static_cast<uint64_t>(tok) * d + 256u * b + k];
            if constexpr (sizeof(XT) == 2 && std::is_same<XT, __half>::value) v = __half2float(xv);
            else v = __bfloat162float(xv);
        }
        sm.x[n][k] = v;
    }
    __syncthreads();
    uint8_t *out = img + (static_cast<uint64_t>(tile) * nb + b) * TG_IMG;
    // 4 chunks x 16 rows x 8 pieces of 16 bytes
    for (uint32_t i = threadIdx.x; i < 4 * 16 * 8; i += blockDim.x) {
        const uint32_t c = i >> 7, n = (i >> 3) & 15u, q = i & 7u;
        uint32_t w[4] = {0u, 0u, 0u, 0u};
        if (n < TG_NT) {
#pragma unroll
            for (uint32_t e = 0; e < 8; e += 2) {
                const uint32_t k0 = 64u * c + xplane_pos(8u * q + e), k1 = 64u * c + xplane_pos(8u * q + e + 1);
                const __half2 h = __floats2half2_rn(sm.x[n][k0], sm.x[n][k1]);
                w[e >> 1] = *reinterpret_cast<const uint32_t *>(&h);
            }
        }
        *reinterpret_cast<uint4 *>(out + c * 2048u + tg_sw_off(n, 8u * q)) = make_uint4(w[0], w[1], w[2], w[3]);
    }
    // sums: rows 8-15 = tokens 0-7, K 0-7 hi and 8-15 lo of the 8 sub-blocks
    // (each sum in ascending order by one thread)
    if (threadIdx.x < TG_NT * 8) {
        const uint32_t t = threadIdx.x >> 3, jj = threadIdx.x & 7u;
        float sum = 0.0f;
#pragma unroll 8
        for (uint32_t k = 0; k < 32; ++k) sum += sm.x[t][32 * jj + k];
        sm.sum[t][jj] = sum;
    }
    __syncthreads();
    for (uint32_t i = threadIdx.x; i < 16 * 8; i += blockDim.x) {
        const uint32_t n = i >> 3, q = i & 7u;
        uint32_t w[4] = {0u, 0u, 0u, 0u};
        if (n >= TG_NT && q < 2) {
            const uint32_t t = n - TG_NT;
            __half hv[8];
#pragma unroll
            for (uint32_t jj = 0; jj < 8; ++jj) {
                const float sum = sm.sum[t][jj];
                const __half h = __float2half_rn(sum);
                hv[jj] = q == 0 ? h : __float2half_rn(sum - __half2float(h));
            }
#pragma unroll
            for (uint32_t e = 0; e < 4; ++e)
                w[e] = static_cast<uint32_t>(__half_as_ushort(hv[2 * e])) |
                       (static_cast<uint32_t>(__half_as_ushort(hv[2 * e + 1])) << 16);
        }
        *reinterpret_cast<uint4 *>(out + TG_MINS_OFF + tg_sw_off(n, 8u * q)) = make_uint4(w[0], w[1], w[2], w[3]);
    }
}

// B images of the gate/up GEMV from the grouping in global memory: grid =
// (upper bound of tiles) x (d / 256) CTAs.
template <typename XT>
__global__ void __launch_bounds__(256)
    tg_ximage_kernel(const __grid_constant__ TgMapArgs ma, const XT *__restrict__ x, uint32_t d,
                     const uint32_t *__restrict__ counts, const uint32_t *__restrict__ offsets,
                     const uint32_t *__restrict__ pairs, uint32_t top_k, uint32_t experts, uint32_t max_tiles,
                     uint8_t *__restrict__ img) {
    __shared__ uint32_t s_tile[TG_MAX_EXPERTS + 1];
    __shared__ TgImageSmem sm;
    tg_maps_and_counters(ma, counts, experts);
    if ((threadIdx.x >> 5) == 0) tg_tile_prefix(s_tile, counts, experts, threadIdx.x & 31u);
    __syncthreads();
    tg_image_block(x, d, counts, offsets, pairs, top_k, experts, max_tiles, s_tile, img, sm);
}

// Router, grouping and the gate/up B images in one launch, for short batches:
// every CTA routes all tokens and groups the pairs in its own shared memory
// (the same device code and inputs, so the same result in every CTA), CTA 0
// writes the routing and grouping to global memory, and CTA (tile, block)
// writes its image from its shared copy.  Replaces the router + grouping
// kernels and tg_ximage_kernel (one launch and one dependency instead of two).
constexpr uint32_t TG_FRONT_MAX_TOKENS = 64, TG_FRONT_MAX_EXPERTS = 64, TG_FRONT_MAX_PAIRS = 1024;

template <typename XT>
__global__ void __launch_bounds__(256)
    tg_front_kernel(const __grid_constant__ TgMapArgs ma, const float *__restrict__ logits, const XT *__restrict__ x,
                    uint32_t tokens, uint32_t experts, uint32_t top_k, int normalise, double epsilon, double scale,
                    uint32_t d, uint32_t max_tiles, uint32_t *ids, float *weights, uint32_t *counts,
                    uint32_t *offsets, uint32_t *pairs, uint32_t *slot_of, uint8_t *__restrict__ img, int *status) {
    __shared__ double s_ex[8][TG_FRONT_MAX_EXPERTS];
    __shared__ float s_pr[8][TG_FRONT_MAX_EXPERTS];
    __shared__ uint32_t s_ids[TG_FRONT_MAX_PAIRS], s_pairs[TG_FRONT_MAX_PAIRS], s_slot[TG_FRONT_MAX_PAIRS];
    __shared__ float s_w[TG_FRONT_MAX_PAIRS];
    __shared__ uint32_t s_cnt[TG_FRONT_MAX_EXPERTS], s_offs[TG_FRONT_MAX_EXPERTS + 1];
    __shared__ uint32_t s_count[TG_FRONT_MAX_EXPERTS], s_off[TG_FRONT_MAX_EXPERTS], s_warp_tot[32];
    __shared__ uint32_t s_tile[TG_FRONT_MAX_EXPERTS + 1];
    __shared__ TgImageSmem sm;
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u, nwarps = blockDim.x >> 5;
    const uint32_t P = tokens * top_k;
    if (threadIdx.x < 32) s_warp_tot[threadIdx.x] = 0;
    for (uint32_t t = warp; t < tokens; t += nwarps)
        route_token(logits, t, experts, top_k, normalise, epsilon, scale, s_ids, s_w, nullptr, status, s_ex[warp],
                    s_pr[warp], static_cast<int>(lane));
    __syncthreads();
    group_block(s_ids, P, experts, s_cnt, s_offs, s_pairs, s_slot, status, s_count, s_off, s_warp_tot);
    __syncthreads();
    if (blockIdx.x == 0) {
        for (uint32_t i = threadIdx.x; i < P; i += blockDim.x) {
            ids[i] = s_ids[i];
            weights[i] = s_w[i];
            pairs[i] = s_pairs[i];
            slot_of[i] = s_slot[i];
        }
        for (uint32_t e = threadIdx.x; e <= experts; e += blockDim.x) {
            if (e < experts) counts[e] = s_cnt[e];
            offsets[e] = s_offs[e];
        }
    }
    tg_maps_and_counters(ma, s_cnt, experts);
    if (warp == 0) {
        // exclusive prefix of token tiles over the experts (experts <= 64)
        uint32_t carry = 0;
        for (uint32_t base = 0; base < experts; base += 32) {
            const uint32_t e = base + lane;
            const uint32_t v = e < experts ? (s_cnt[e] + TG_NT - 1) / TG_NT : 0u;
            uint32_t incl = v;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const uint32_t t = __shfl_up_sync(0xFFFFFFFFu, incl, o);
                if (lane >= static_cast<uint32_t>(o)) incl += t;
            }
            if (e < experts) s_tile[e] = carry + incl - v;
            carry += __shfl_sync(0xFFFFFFFFu, incl, 31);
        }
        if (lane == 0) s_tile[experts] = carry;
    }
    __syncthreads();
    tg_image_block(x, d, s_cnt, s_offs, s_pairs, top_k, experts, max_tiles, s_tile, img, sm);
}

// The expert-parallel receive side in one launch: every CTA waits for every
// source's rows (epoch flags of the peer exchange), groups the received
// (row, slot) pairs by local expert in shared memory (keys: the local expert
// id of each slot, absent for other ranks' slots and rows past the received
// count), CTA 0 publishes the grouping, and CTA (tile, block) writes its gate/up
// B image from the fp16 receive rows.  Replaces the wait, key, grouping and
// image kernels of the receive side.
__global__ void __launch_bounds__(256)
    tg_recv_front_kernel(const __grid_constant__ TgMapArgs ma, const uint32_t *flags, uint32_t world, uint32_t epoch,
                         const uint32_t *ectr, uint64_t timeout_ns, const uint32_t *n_rows,
                         const int32_t *__restrict__ meta_e, const __half *__restrict__ x, uint32_t rows,
                         uint32_t top_k, uint32_t experts, uint32_t d, uint32_t max_tiles, uint32_t *counts,
                         uint32_t *offsets, uint32_t *pairs, uint8_t *__restrict__ img, int *status) {
    __shared__ uint32_t s_keys[TG_FRONT_MAX_PAIRS], s_pairs[TG_FRONT_MAX_PAIRS];
    __shared__ uint32_t s_cnt[TG_FRONT_MAX_EXPERTS], s_offs[TG_FRONT_MAX_EXPERTS + 1];
    __shared__ uint32_t s_count[TG_FRONT_MAX_EXPERTS], s_off[TG_FRONT_MAX_EXPERTS], s_warp_tot[32];
    __shared__ uint32_t s_tile[TG_FRONT_MAX_EXPERTS + 1];
    __shared__ TgImageSmem sm;
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
    wait_flags_cta(flags, world, call_epoch(epoch, ectr), timeout_ns, status);
    const uint32_t live = *reinterpret_cast<const volatile uint32_t *>(n_rows);
    const uint32_t P = rows * top_k;
    for (uint32_t i = threadIdx.x; i < P; i += blockDim.x) {
        const int32_t e = i / top_k < live ? meta_e[i] : -1;
        s_keys[i] = e >= 0 ? static_cast<uint32_t>(e) : 0xFFFFFFFFu;
    }
    if (threadIdx.x < 32) s_warp_tot[threadIdx.x] = 0;
    __syncthreads();
    group_block(s_keys, P, experts, s_cnt, s_offs, s_pairs, nullptr, status, s_count, s_off, s_warp_tot);
    __syncthreads();
    if (blockIdx.x == 0) {
        for (uint32_t i = threadIdx.x; i < P; i += blockDim.x) pairs[i] = s_pairs[i];
        for (uint32_t e = threadIdx.x; e <= experts; e += blockDim.x) {
            if (e < experts) counts[e] = s_cnt[e];
            offsets[e] = s_offs[e];
        }
    }
    tg_maps_and_counters(ma, s_cnt, experts);
    if (warp == 0) {
        uint32_t carry = 0;
        for (uint32_t base = 0; base < experts; base += 32) {
            const uint32_t e = base + lane;
            const uint32_t v = e < experts ? (s_cnt[e] + TG_NT - 1) / TG_NT : 0u;
            uint32_t incl = v;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const uint32_t t = __shfl_up_sync(0xFFFFFFFFu, incl, o);
                if (lane >= static_cast<uint32_t>(o)) incl += t;
            }
            if (e < experts) s_tile[e] = carry + incl - v;
            carry += __shfl_sync(0xFFFFFFFFu, incl, 31);
        }
        if (lane == 0) s_tile[experts] = carry;
    }
    __syncthreads();
    tg_image_block(x, d, s_cnt, s_offs, s_pairs, top_k, experts, max_tiles, s_tile, img, sm);
}

} // namespace fmb
