// grouped_gemm.cuh -- fused dequant + grouped GEMM for MoE prefill on the
// sm_100a tensor cores (tcgen05.mma, accumulators and A operand in TMEM, B
// operand staged by TMA).
//
// Replaces, for batches of tokens, the per-token expert loop of the reference
// (src/engine.cpp:1711-1772): for every expert e with n_e routed tokens,
//   GEMM1  act[n_e, ffn] = silu(X_e Wg_e^T) * (X_e Wu_e^T)     (gate/up + SwiGLU)
//   GEMM2  part[n_e, d]  = act_e Wd_e^T                        (down)
// where X_e are the expert's token rows gathered into one contiguous fp16
// matrix (grouped order, see router.cu) and W are the expert's GGUF rows in
// their stored Q8_0 / Q4_K bytes (src/quant.cpp:223-228, :297-318).
//
// Work unit = (expert e, tile of 128 weight rows, tile of <= 192 tokens for
// gate/up, <= 256 tokens for down; more tokens per unit = fewer conversions of
// the same weights per FLOP, bounded by the 512 TMEM columns); the
// persistent CTAs (one per SM) take units round-robin.  Inside a CTA:
//   warp 0      TMA producer: 192-token (gate/up) or 256-token (down) x 64-value
//               fp16 tiles of X (or act), 128-byte swizzled, into a 3- or 2-stage
//               ring (B operand);
//   warp 1      MMA issuer: one thread issues tcgen05.mma kind::f16,
//               M = 128 weight rows, N = tokens of the tile (rounded to 16),
//               K = 16 per instruction, A from TMEM, B from shared memory;
//   warp 2      TMEM allocation (512 columns) and release;
//   warps 4-11  two converter warpgroups.  Thread t of a warpgroup owns weight
//               row t of the tile = TMEM lane t.  Each warp streams its 32
//               rows' raw bytes (256 values per row per chunk) into its own
//               cp.async ring, decodes 64 values per step to fp16 in registers
//               and writes them into an A stage in TMEM with tcgen05.st.  For
//               gate/up, warpgroup 0 converts the gate rows and warpgroup 1
//               the up rows of the same output features, and the two
//               accumulators (gate, up) sit in TMEM side by side, so the
//               SwiGLU epilogue needs no exchange.  For down, the warpgroups
//               take alternate 256-value chunks.  After the K loop the same
//               threads read the accumulators back (tcgen05.ld) and write
//               act (fp16) or part (f32) rows.
//
// Numerics: weights become fp16 within one fp16 rounding of the dequantised
// value (Q8_0: exactly RN(d*q); Q4_K: RN(d*sc*q - RN(dmin*m))); X is fp16
// (bf16 inputs convert exactly in fp16 range); products accumulate in f32.
// The SwiGLU uses float silu.  Results therefore match the reference within a
// relative tolerance, not bit for bit.
#pragma once

#include "common.cuh"
#include "gemv_core.cuh"
#include "tcgen05.cuh"

namespace fmb {

constexpr uint32_t GG_BM = 128;     // weight rows per tile (TMEM lanes)
#ifndef FMB_GG_BN2
#define FMB_GG_BN2 192
#endif
#ifndef FMB_GG_SA2
#define FMB_GG_SA2 2
#endif
#ifndef FMB_GG_SB2
#define FMB_GG_SB2 3
#endif
#ifndef FMB_GG_BN1
#define FMB_GG_BN1 256
#endif
constexpr uint32_t GG_BN = FMB_GG_BN2;  // tokens per tile of the gate/up GEMM (two accumulators)
constexpr uint32_t GG_BN1 = FMB_GG_BN1; // tokens per tile of the one-matrix GEMM (one accumulator)
constexpr uint32_t GG_BK = 64;      // K values per MMA stage (one 128-byte fp16 row)
constexpr uint32_t GG_CHUNK = 256;  // K values per raw chunk (one Q4_K block, eight Q8_0 blocks)
constexpr uint32_t GG_THREADS = 384;
constexpr uint32_t GG_TMEM_COLS = 512;
constexpr uint32_t GG_MAX_EXPERTS = 1024;

enum { GG_EPI_SWIGLU = 0, GG_EPI_F32 = 1 };

struct GGemmParams {
    const uint8_t *const *slots; // per-expert slab base (device array)
    uint64_t w_off0, w_off1;     // byte offset of matrix 0 / 1 inside a slab
    uint32_t out_dim;            // rows of each weight matrix (multiple of 128)
    uint32_t in_dim;             // K (multiple of 64)
    uint32_t row_bytes;          // stored bytes per weight row
    uint32_t experts;
    const uint32_t *counts;      // tokens per expert
    const uint32_t *offsets;     // first grouped row of each expert
    void *out;                   // GEMM1: __half [rows][out_dim]; GEMM2: float [rows][out_dim]
    const uint32_t *out_rows;    // optional: output row of grouped row g is out_rows[g] (else g)
    int *status;
};

template <int TYPE> struct GGeom;
template <> struct GGeom<FM_TYPE_Q8_0> {
    static constexpr uint32_t CB = 272; // bytes of one 256-value chunk of a row
    static constexpr uint32_t RS = 2;   // raw chunks in flight per warp
};
template <> struct GGeom<FM_TYPE_Q4_K> {
    static constexpr uint32_t CB = 144;
    static constexpr uint32_t RS = 3;
};
// Q6_K: one 210-byte block per chunk; block starts are only 2-byte aligned, so
// the converter copies the 16-byte aligned window around the block (at most
// 15 pieces = 240 bytes) and decodes from the block's offset in the window.
template <> struct GGeom<FM_TYPE_Q6_K> {
    static constexpr uint32_t CB = 210;
    static constexpr uint32_t RS = 2;
    static constexpr uint32_t WINDOW = 240;
};
template <int TYPE> constexpr uint32_t gg_pitch() {
    if constexpr (TYPE == FM_TYPE_Q6_K) return GGeom<TYPE>::WINDOW;
    else return GGeom<TYPE>::CB;
}

// Token (B) stages of the one-matrix GEMM: three where shared memory holds
// them next to the raw rings (Q4_K, Q6_K; measured on the Qwen3 shape: down
// -11% against two), else two (Q8_0's 272-byte chunks leave no room).
template <int TYPE> constexpr uint32_t gg_sb1() {
    constexpr uint32_t raw = 8 * GGeom<TYPE>::RS * 32 * gg_pitch<TYPE>();
    constexpr uint32_t stage = GG_BN1 * GG_BK * 2;
    constexpr uint32_t fixed = 1024 + 512 + 4 * (GG_MAX_EXPERTS + 1); // alignment, barriers, unit table
    return raw + 3 * stage + fixed <= 227u * 1024u ? 3u : 2u;
}

template <int TYPE, int NMAT> struct GGLayout {
    static constexpr uint32_t BN = NMAT == 2 ? GG_BN : GG_BN1;  // tokens per unit
    static constexpr uint32_t SB = NMAT == 2 ? FMB_GG_SB2 : gg_sb1<TYPE>(); // B ring stages
    static constexpr uint32_t SA = NMAT == 2 ? FMB_GG_SA2 : 8;          // A stages in TMEM
    static constexpr uint32_t A_COL0 = NMAT * BN;               // accumulators first
    static constexpr uint32_t A_STAGE_COLS = NMAT * (GG_BK / 2); // fp16 pairs per column
    static constexpr uint32_t PITCH = gg_pitch<TYPE>();         // raw row pitch (odd multiple of 16)
    static constexpr uint32_t RS = GGeom<TYPE>::RS;
    static constexpr uint32_t B_STAGE = BN * GG_BK * 2;
    static constexpr uint32_t RAW_SLOT = 32 * PITCH;
    static constexpr uint32_t RAW_WARP = RS * RAW_SLOT;
    static constexpr uint32_t OFF_RAW = SB * B_STAGE;
    static constexpr uint32_t OFF_BAR = OFF_RAW + 8 * RAW_WARP;
    static constexpr uint32_t NBAR = 2 * SB + 2 * SA + 3;
    static constexpr uint32_t OFF_MISC = OFF_BAR + NBAR * 8;
    static constexpr uint32_t OFF_UNITS = OFF_MISC + 16;
    static_assert(A_COL0 + SA * A_STAGE_COLS <= GG_TMEM_COLS, "TMEM budget");
    static_assert(BN % 64 == 0 && BN <= 256, "token tile: two warpgroups x 32-column loads");
    static_assert((SB * B_STAGE) % 1024 == 0, "1024-byte aligned raw rings");
    static_assert(PITCH % 16 == 0 && (PITCH / 16) % 2 == 1, "conflict-free 16-byte row reads");
    static constexpr uint32_t smem_bytes(uint32_t experts) { return 1024 + OFF_UNITS + 4 * (experts + 1); }
    static_assert(1024 + OFF_UNITS + 4 * (GG_MAX_EXPERTS + 1) <= 227u * 1024u, "shared memory per CTA");
};

struct GUnit {
    uint32_t e, rt, n_tok, row_b0;
};

// Unit u -> (expert, row tile, token tile).  s_units[e] is the first unit of
// expert e (exclusive prefix over experts of token_tiles * row_tiles); token
// tiles vary fastest, so CTAs running side by side share a weight tile in L2.
template <uint32_t BN>
__device__ __forceinline__ GUnit gg_unit(const uint32_t *s_units, uint32_t experts, uint32_t u,
                                         const uint32_t *counts, const uint32_t *offsets) {
    uint32_t lo = 0, hi = experts;
    while (hi - lo > 1) {
        const uint32_t mid = (lo + hi) >> 1;
        if (s_units[mid] <= u) lo = mid;
        else hi = mid;
    }
    GUnit g;
    g.e = lo;
    const uint32_t cnt = __ldg(counts + lo);
    const uint32_t tiles = (cnt + BN - 1) / BN;
    const uint32_t local = u - s_units[lo];
    g.rt = local / tiles;
    const uint32_t tt = local - g.rt * tiles;
    g.n_tok = min(BN, cnt - tt * BN);
    g.row_b0 = __ldg(offsets + lo) + tt * BN;
    return g;
}

// Bounded mbarrier wait that also gives up once another role has aborted.
__device__ __forceinline__ bool gg_wait(uint64_t *bar, uint32_t parity, volatile uint32_t *abort_flag,
                                        int *status) {
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

// ---- decoding one 64-value step of one row into 32 fp16x2 words (k order) ----

// The fast paths below read a code placed in a zero fp16 as the subnormal
// code * 2^-24 (exact; PRMT with zero bytes, no magic-exponent constant), and
// fold the scale powers of two into the block factor; each produces the same
// bits as the generic path, which stays for blocks whose scaled factor would
// not fit fp16.

// Q8_0: blocks 2*ST and 2*ST+1 of the chunk, bytes [68*ST, 68*ST + 68).
// Generic: (q ^ 0x80) | 0x6400 is the fp16 1152 + q; subtracting 1152 is exact
// and the multiply by d rounds once, giving RN(d * q).  Fast (d < 2^-8): one
// FMA of the subnormal (128 + q) * 2^-24 with 2^24 d and -128 d, the same
// single rounding of d * q.
template <int ST>
__device__ __forceinline__ void gg_decode_q8_0(const uint8_t *row, uint32_t (&v)[32]) {
    constexpr int BASE = (68 * ST) / 16 * 16;
    constexpr int M0 = 68 * ST - BASE;
    uint32_t w[20];
#pragma unroll
    for (int i = 0; i < 5; ++i) {
        const uint4 t = *reinterpret_cast<const uint4 *>(row + BASE + 16 * i);
        w[4 * i] = t.x;
        w[4 * i + 1] = t.y;
        w[4 * i + 2] = t.z;
        w[4 * i + 3] = t.w;
    }
#pragma unroll
    for (int b = 0; b < 2; ++b) {
        const int o = M0 + 34 * b;
        const uint32_t dbits = (o % 4 == 0) ? (w[o / 4] & 0xFFFFu) : (w[o / 4] >> 16);
        const int qo = o + 2;
        const int qi = qo / 4;
        const int sh = (qo % 4) * 8;
        const float df = fp16_bits_to_f32(static_cast<uint16_t>(dbits));
        if (fabsf(df) < 0.00390625f) {
            const __half2 dd = __float2half2_rn(df * 16777216.0f), nb = __float2half2_rn(-128.0f * df);
            const uint32_t udd = *reinterpret_cast<const uint32_t *>(&dd), unb = *reinterpret_cast<const uint32_t *>(&nb);
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                uint32_t q = sh ? __funnelshift_r(w[qi + j], w[qi + j + 1], sh) : w[qi + j];
                q ^= 0x80808080u;
                v[16 * b + 2 * j] = hfma2_u32(prmt(q, 0u, 0x5140u), udd, unb);
                v[16 * b + 2 * j + 1] = hfma2_u32(prmt(q, 0u, 0x7362u), udd, unb);
            }
        } else {
            const uint32_t d2 = dbits | (dbits << 16);
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                uint32_t q = sh ? __funnelshift_r(w[qi + j], w[qi + j + 1], sh) : w[qi + j];
                q ^= 0x80808080u;
                const uint32_t lo = prmt(q, 0x64646464u, 0x5140u);
                const uint32_t hi = prmt(q, 0x64646464u, 0x7362u);
                v[16 * b + 2 * j] = hmul2_u32(hsub2_u32(lo, 0x64806480u), d2);
                v[16 * b + 2 * j + 1] = hmul2_u32(hsub2_u32(hi, 0x64806480u), d2);
            }
        }
    }
}

// Q4_K: group G4 (values 64*G4 .. 64*G4+63) of the 256-value block: low
// nibbles of qs[32*G4 .. +32) are sub-block 2*G4, high nibbles 2*G4+1.
// Generic: (1024 + q) * sc - 1024 * sc = sc * q exactly; then one rounding of
// d * (sc * q) - RN(dmin * m).  Fast (|d| < 4): the subnormal q * 2^-24 (high
// nibbles masked in place: 16 q * 2^-24) times 2^10 sc (2^6 sc) is
// sc * q * 2^-14 exactly, and one FMA with 2^14 d and -RN(dmin * m) rounds
// d * (sc * q) - RN(dmin * m) once, as the generic path does.
template <int G4>
__device__ __forceinline__ void gg_decode_q4_k(const uint8_t *row, uint32_t (&v)[32]) {
    const uint4 h = *reinterpret_cast<const uint4 *>(row);
    const uint4 qa = *reinterpret_cast<const uint4 *>(row + 16 + 32 * G4);
    const uint4 qb = *reinterpret_cast<const uint4 *>(row + 32 + 32 * G4);
    const uint32_t dbits = h.x & 0xFFFFu;
    const float df = fp16_bits_to_f32(static_cast<uint16_t>(dbits));
    const float dmin = fp16_bits_to_f32(static_cast<uint16_t>(h.x >> 16));
    uint32_t sc0, mn0, sc1, mn1;
    q4k_scale_min_w(2 * G4, h.y, h.z, h.w, sc0, mn0);
    q4k_scale_min_w(2 * G4 + 1, h.y, h.z, h.w, sc1, mn1);
    const float m0f = -(dmin * static_cast<float>(mn0)), m1f = -(dmin * static_cast<float>(mn1));
    const __half2 mm0 = __floats2half2_rn(m0f, m0f), mm1 = __floats2half2_rn(m1f, m1f);
    const uint32_t um0 = *reinterpret_cast<const uint32_t *>(&mm0), um1 = *reinterpret_cast<const uint32_t *>(&mm1);
    const uint32_t qw[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
    if (fabsf(df) < 4.0f) {
        const __half2 s0 = __float2half2_rn(1024.0f * sc0), s1 = __float2half2_rn(64.0f * sc1);
        const __half2 dd = __float2half2_rn(16384.0f * df);
        const uint32_t us0 = *reinterpret_cast<const uint32_t *>(&s0), us1 = *reinterpret_cast<const uint32_t *>(&s1);
        const uint32_t udd = *reinterpret_cast<const uint32_t *>(&dd);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const uint32_t lo = qw[j] & 0x0F0F0F0Fu;
            const uint32_t hi = qw[j] & 0xF0F0F0F0u;
            v[2 * j] = hfma2_u32(hmul2_u32(prmt(lo, 0u, 0x5140u), us0), udd, um0);
            v[2 * j + 1] = hfma2_u32(hmul2_u32(prmt(lo, 0u, 0x7362u), us0), udd, um0);
            v[16 + 2 * j] = hfma2_u32(hmul2_u32(prmt(hi, 0u, 0x5140u), us1), udd, um1);
            v[16 + 2 * j + 1] = hfma2_u32(hmul2_u32(prmt(hi, 0u, 0x7362u), us1), udd, um1);
        }
    } else {
        const uint32_t d2 = dbits | (dbits << 16);
        const __half2 s0 = __floats2half2_rn(static_cast<float>(sc0), static_cast<float>(sc0));
        const __half2 n0 = __floats2half2_rn(-1024.0f * sc0, -1024.0f * sc0);
        const __half2 s1 = __floats2half2_rn(static_cast<float>(sc1), static_cast<float>(sc1));
        const __half2 n1 = __floats2half2_rn(-1024.0f * sc1, -1024.0f * sc1);
        const uint32_t us0 = *reinterpret_cast<const uint32_t *>(&s0), un0 = *reinterpret_cast<const uint32_t *>(&n0);
        const uint32_t us1 = *reinterpret_cast<const uint32_t *>(&s1), un1 = *reinterpret_cast<const uint32_t *>(&n1);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const uint32_t lo = qw[j] & 0x0F0F0F0Fu;
            const uint32_t hi = (qw[j] >> 4) & 0x0F0F0F0Fu;
            const uint32_t l01 = prmt(lo, 0x64646464u, 0x5140u), l23 = prmt(lo, 0x64646464u, 0x7362u);
            const uint32_t h01 = prmt(hi, 0x64646464u, 0x5140u), h23 = prmt(hi, 0x64646464u, 0x7362u);
            v[2 * j] = hfma2_u32(hfma2_u32(l01, us0, un0), d2, um0);
            v[2 * j + 1] = hfma2_u32(hfma2_u32(l23, us0, un0), d2, um0);
            v[16 + 2 * j] = hfma2_u32(hfma2_u32(h01, us1, un1), d2, um1);
            v[16 + 2 * j + 1] = hfma2_u32(hfma2_u32(h23, us1, un1), d2, um1);
        }
    }
}

// Q6_K (src/quant.cpp:347-372): step ST covers values 64*ST .. 64*ST+63 of
// the block, i.e. half h = ST/2 and the two 32-value groups 2*(ST&1) and
// 2*(ST&1)+1: low bits from the nibble (ST&1) of ql[64h + l] and ql[64h + 32
// + l], high bits from qh[32h + l] >> 2*group, scale group 4*ST + k/16.  `o`
// is the block's (even) byte offset inside its copied window; words are read
// aligned and shifted.  Each value is RN_f32(RN_f32(d * sc) * (c6 - 32)), the
// reference's dequantised value bit for bit (one FMA: c6 * ds - 32 * ds),
// then rounded once to fp16.
template <int ST>
__device__ __forceinline__ void gg_decode_q6_k(const uint8_t *win, uint32_t o, uint32_t (&v)[32]) {
    constexpr uint32_t H = ST >> 1, NIB = 4 * (ST & 1), G0 = 2 * (ST & 1);
    const uint32_t sh = (o & 3u) * 8u;
    const uint32_t *w = reinterpret_cast<const uint32_t *>(win + (o & ~3u));
    auto word = [&](uint32_t byte_off) -> uint32_t { // 4 bytes at o + byte_off (byte_off % 4 == 0)
        const uint32_t i = byte_off >> 2;
        return sh ? __funnelshift_r(w[i], w[i + 1], sh) : w[i];
    };
    const float d = fp16_bits_to_f32(*reinterpret_cast<const uint16_t *>(win + o + 208));
    const uint32_t scw = word(192 + 4 * ST);
    float ds[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) ds[q] = __fmul_rn(d, static_cast<float>(static_cast<int8_t>(scw >> (8 * q))));
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const uint32_t qh = word(128 + 32 * H + 4 * i);
        const uint32_t lo = word(64 * H + 4 * i), hi = word(64 * H + 32 + 4 * i);
        const uint32_t c0 = ((lo >> NIB) & 0x0F0F0F0Fu) | (((qh >> (2 * G0)) & 0x03030303u) << 4);
        const uint32_t c1 = ((hi >> NIB) & 0x0F0F0F0Fu) | (((qh >> (2 * G0 + 2)) & 0x03030303u) << 4);
        float y0[4], y1[4];
#pragma unroll
        for (int b = 0; b < 4; ++b) {
            const float f0 = static_cast<float>((c0 >> (8 * b)) & 0xFFu);
            const float f1 = static_cast<float>((c1 >> (8 * b)) & 0xFFu);
            const float s0 = ds[(4 * i + b) >> 4], s1 = ds[2 + ((4 * i + b) >> 4)];
            y0[b] = fmaf(f0, s0, -32.0f * s0);
            y1[b] = fmaf(f1, s1, -32.0f * s1);
        }
        const __half2 a0 = __floats2half2_rn(y0[0], y0[1]), a1 = __floats2half2_rn(y0[2], y0[3]);
        const __half2 b0 = __floats2half2_rn(y1[0], y1[1]), b1 = __floats2half2_rn(y1[2], y1[3]);
        v[2 * i] = *reinterpret_cast<const uint32_t *>(&a0);
        v[2 * i + 1] = *reinterpret_cast<const uint32_t *>(&a1);
        v[16 + 2 * i] = *reinterpret_cast<const uint32_t *>(&b0);
        v[16 + 2 * i + 1] = *reinterpret_cast<const uint32_t *>(&b1);
    }
}

template <int TYPE, int ST>
__device__ __forceinline__ void gg_decode(const uint8_t *row, uint32_t o, uint32_t (&v)[32]) {
    if constexpr (TYPE == FM_TYPE_Q8_0) gg_decode_q8_0<ST>(row, v);
    else if constexpr (TYPE == FM_TYPE_Q4_K) gg_decode_q4_k<ST>(row, v);
    else gg_decode_q6_k<ST>(row, o, v);
}

template <int TYPE, int NMAT, int EPI, int G>
__global__ void __launch_bounds__(GG_THREADS, 1)
    grouped_gemm_kernel(const __grid_constant__ CUtensorMap tmap_b, const GGemmParams p) {
    using L = GGLayout<TYPE, NMAT>;
    constexpr uint32_t SB = L::SB, SA = L::SA, RS = L::RS, CB = GGeom<TYPE>::CB, BN = L::BN;
    extern __shared__ uint8_t gg_smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(gg_smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *sB = smem;
    uint8_t *sRaw = smem + L::OFF_RAW;
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + L::OFF_BAR);
    uint64_t *b_full = bars, *b_empty = bars + SB;
    uint64_t *a_full = bars + 2 * SB, *a_empty = a_full + SA;
    uint64_t *acc_full = a_empty + SA, *acc_empty = acc_full + 1, *drain = acc_full + 2;
    // with equal A and B ring depths one commit per K step releases both stages
    uint64_t *b_release = (SA == SB) ? a_empty : b_empty;
    uint32_t *misc = reinterpret_cast<uint32_t *>(smem + L::OFF_MISC); // [0] TMEM base, [1] abort, [2] bad
    volatile uint32_t *abort_flag = misc + 1;
    uint32_t *s_units = reinterpret_cast<uint32_t *>(smem + L::OFF_UNITS);

    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
    const uint32_t E = p.experts;
    const uint32_t row_tiles = p.out_dim / GG_BM;
    const uint32_t ksteps = p.in_dim / GG_BK;
    const uint32_t nchunks = (p.in_dim + GG_CHUNK - 1) / GG_CHUNK;

    if (threadIdx.x == 0) {
        misc[1] = 0;
        misc[2] = 0;
    }
    __syncthreads();
    if (warp == 0) {
        // exclusive prefix of units over experts
        uint32_t carry = 0;
        for (uint32_t base = 0; base < E; base += 32) {
            const uint32_t e = base + lane;
            uint32_t v = 0;
            if (e < E) v = ((__ldg(p.counts + e) + BN - 1) / BN) * row_tiles;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const uint32_t t = __shfl_up_sync(0xFFFFFFFFu, v, o);
                if (lane >= static_cast<uint32_t>(o)) v += t;
            }
            if (e < E) s_units[e + 1] = carry + v;
            carry += __shfl_sync(0xFFFFFFFFu, v, 31);
        }
        if (lane == 0) s_units[0] = 0;
    } else if (warp == 3) {
        // every expert with tokens needs a resident slab at a G-aligned address
        for (uint32_t e = lane; e < E; e += 32) {
            if (__ldg(p.counts + e) == 0) continue;
            const uintptr_t base = reinterpret_cast<uintptr_t>(p.slots[e]);
            if (!base) atomicCAS(misc + 2, 0u, static_cast<uint32_t>(FM_STATUS_EXPERT_EXECUTION_MISMATCH));
            else if ((base + p.w_off0) % G || (base + p.w_off1) % G)
                atomicCAS(misc + 2, 0u, static_cast<uint32_t>(FM_STATUS_INVALID_ARGUMENT));
        }
    } else if (threadIdx.x == 32) {
        for (uint32_t i = 0; i < SB; ++i) {
            mbar_init(&b_full[i], 1);
            mbar_init(&b_empty[i], 1);
        }
        for (uint32_t i = 0; i < SA; ++i) {
            mbar_init(&a_full[i], NMAT == 2 ? 8 : 4);
            mbar_init(&a_empty[i], 1);
        }
        mbar_init(acc_full, 1);
        mbar_init(acc_empty, 8);
        mbar_init(drain, 1);
        fence_barrier_init();
    }
    __syncthreads();
    const uint32_t U = s_units[E];
    if (misc[2]) {
        if (threadIdx.x == 0) raise_device_status(p.status, static_cast<int>(misc[2]));
        return;
    }
    if (blockIdx.x >= U) return;

    if (warp == 2) {
        tmem_alloc(misc, GG_TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = misc[0];

    if (warp == 0) {
        // ---- TMA producer: B tiles --------------------------------------------
        if (lane == 0) {
            uint32_t it = 0;
            for (uint32_t u = blockIdx.x; u < U && !*abort_flag; u += gridDim.x) {
                const GUnit g = gg_unit<BN>(s_units, E, u, p.counts, p.offsets);
                for (uint32_t s = 0; s < ksteps; ++s, ++it) {
                    const uint32_t st = it % SB;
                    if (!gg_wait(&b_release[st], ((it / SB) & 1u) ^ 1u, abort_flag, p.status)) goto producer_done;
                    mbar_expect_tx(&b_full[st], L::B_STAGE);
                    tma_load_2d(sB + st * L::B_STAGE, &tmap_b, static_cast<int32_t>(s * GG_BK),
                                static_cast<int32_t>(g.row_b0), &b_full[st]);
                }
            }
        producer_done:
            // loads still in flight must land before the CTA's shared memory goes away
            for (uint32_t j = it > SB ? it - SB : 0; j < it; ++j) (void)mbar_wait(&b_full[j % SB], (j / SB) & 1u);
        }
    } else if (warp == 1) {
        // ---- MMA issuer -------------------------------------------------------
        if (lane == 0) {
            uint32_t it = 0, acc_it = 0;
            bool issued = false;
            for (uint32_t u = blockIdx.x; u < U; u += gridDim.x, ++acc_it) {
                const GUnit g = gg_unit<BN>(s_units, E, u, p.counts, p.offsets);
                const uint32_t idesc = idesc_f16_m128((g.n_tok + 15u) & ~15u);
                if (!gg_wait(acc_empty, (acc_it & 1u) ^ 1u, abort_flag, p.status)) break;
                tc_fence_after();
                for (uint32_t s = 0; s < ksteps; ++s, ++it) {
                    const uint32_t bst = it % SB, ast = it % SA;
                    if (!gg_wait(&b_full[bst], (it / SB) & 1u, abort_flag, p.status)) goto mma_done;
                    if (!gg_wait(&a_full[ast], (it / SA) & 1u, abort_flag, p.status)) goto mma_done;
                    tc_fence_after();
                    const uint32_t bsa = smem_u32(sB + bst * L::B_STAGE);
#pragma unroll
                    for (uint32_t kk = 0; kk < GG_BK / 16; ++kk) {
                        const uint64_t bd = smem_desc_sw128(bsa + kk * 32u);
#pragma unroll
                        for (uint32_t m = 0; m < static_cast<uint32_t>(NMAT); ++m)
                            mma_f16_ts(tmem + m * BN, tmem + L::A_COL0 + ast * L::A_STAGE_COLS + m * 32u + kk * 8u,
                                       bd, idesc, (s | kk) != 0u);
                    }
                    issued = true;
                    if (SA != SB) tc_commit(&b_empty[bst]);
                    tc_commit(&a_empty[ast]);
                }
                tc_commit(acc_full);
            }
        mma_done:
            if (issued) {
                // every MMA issued must finish before TMEM is released
                tc_commit(drain);
                (void)mbar_wait(drain, 0);
            }
        }
    } else if (warp >= 4) {
        // ---- converters + epilogue -------------------------------------------
        const uint32_t wg = (warp - 4) >> 2;
        const uint32_t wq = warp & 3u; // TMEM lane quarter reachable by this warp
        const uint32_t row_in_tile = wq * 32 + lane;
        const uint32_t m = NMAT == 2 ? wg : 0;
        const uint64_t w_off = m == 0 ? p.w_off0 : p.w_off1;
        const uint32_t c0 = NMAT == 2 ? 0 : wg, cstep = NMAT == 2 ? 1 : 2;
        const uint32_t J = NMAT == 2 ? nchunks : (nchunks > c0 ? (nchunks - c0 + 1) / 2 : 0);
        uint8_t *ring = sRaw + (warp - 4) * L::RAW_WARP;
        const uint32_t my_units = (U - blockIdx.x + gridDim.x - 1) / gridDim.x;
        const uint32_t njobs = my_units * J;
        const uint32_t lane_addr = (wq * 32u) << 16;

        // The prefetch cursor runs up to RS chunks ahead, possibly into the next
        // unit; the unit's row address is worked out once per unit.  The warp
        // copies its 32 rows' chunk as one block: lane l moves pieces l, l+32, ...
        // in row-major order, so each copy instruction covers ~512 contiguous
        // bytes of two or three rows instead of 32 scattered rows.
        uint32_t iss_nord = 0xFFFFFFFFu;
        const uint8_t *iss_row0 = nullptr, *iss_end = nullptr;
        auto issue = [&](uint32_t j) {
            if (j < njobs) {
                const uint32_t n_ord = j / J, ch = c0 + (j - n_ord * J) * cstep;
                if (n_ord != iss_nord) {
                    const GUnit g = gg_unit<BN>(s_units, E, blockIdx.x + n_ord * gridDim.x, p.counts, p.offsets);
                    iss_row0 = p.slots[g.e] + w_off + static_cast<uint64_t>(g.rt * GG_BM + wq * 32u) * p.row_bytes;
                    iss_end = p.slots[g.e] + w_off + static_cast<uint64_t>(p.out_dim) * p.row_bytes;
                    iss_nord = n_ord;
                }
                const uint8_t *src = iss_row0 + static_cast<uint64_t>(ch) * CB;
                uint8_t *dst = ring + (j % RS) * L::RAW_SLOT;
                const uint32_t bytes = min(CB, p.row_bytes - ch * CB);
                if constexpr (TYPE == FM_TYPE_Q6_K) {
                    // 14 aligned 16-byte pieces hold the block: the window starts at
                    // the block rounded down to 16 bytes and the block ends at most
                    // 14 + 210 = 224 bytes in; a piece is clipped at the matrix end.
#pragma unroll
                    for (uint32_t u = 0; u < 14; ++u) {
                        const uint32_t q = lane + 32u * u, r = q / 14, k = q - r * 14;
                        const uint8_t *a = src + static_cast<uint64_t>(r) * p.row_bytes;
                        const uint8_t *piece =
                            reinterpret_cast<const uint8_t *>(reinterpret_cast<uintptr_t>(a) & ~uintptr_t(15)) + 16 * k;
                        const uint64_t left = static_cast<uint64_t>(iss_end - piece);
                        cp_async16_zfill(dst + r * L::PITCH + 16 * k, piece, left < 16 ? static_cast<uint32_t>(left) : 16u);
                    }
                } else if (bytes == CB) {
                    constexpr uint32_t PPR = CB / G; // pieces per row
#pragma unroll
                    for (uint32_t u = 0; u < PPR; ++u) {
                        const uint32_t q = lane + 32u * u, r = q / PPR, c = q - r * PPR;
                        cp_async_g<G>(dst + r * L::PITCH + c * G, src + static_cast<uint64_t>(r) * p.row_bytes + c * G);
                    }
                } else {
                    const uint32_t ppr = bytes / G;
                    for (uint32_t q = lane; q < 32u * ppr; q += 32u) {
                        const uint32_t r = q / ppr, c = q - r * ppr;
                        cp_async_g<G>(dst + r * L::PITCH + c * G, src + static_cast<uint64_t>(r) * p.row_bytes + c * G);
                    }
                }
            }
            cp_async_commit();
        };

        for (uint32_t j = 0; j < RS; ++j) issue(j);
        uint32_t j = 0;
        for (uint32_t n_ord = 0; n_ord < my_units; ++n_ord) {
            const GUnit g = gg_unit<BN>(s_units, E, blockIdx.x + n_ord * gridDim.x, p.counts, p.offsets);
            for (uint32_t jj = 0; jj < J; ++jj, ++j) {
                const uint32_t ch = c0 + jj * cstep;
                cp_async_wait<RS - 1>();
                __syncwarp();
                const uint8_t *row = ring + (j % RS) * L::RAW_SLOT + lane * L::PITCH;
                const uint32_t steps = min(GG_CHUNK / GG_BK, ksteps - ch * (GG_CHUNK / GG_BK));
                // Q6_K: the block's byte offset inside its 16-byte aligned window
                // (slot bases and matrix offsets are 16-byte aligned)
                const uint32_t win_off =
                    TYPE == FM_TYPE_Q6_K ? static_cast<uint32_t>((static_cast<uint64_t>(g.rt * GG_BM + row_in_tile) *
                                                                      p.row_bytes + static_cast<uint64_t>(ch) * CB) & 15u)
                                         : 0u;
#pragma unroll
                for (uint32_t st = 0; st < GG_CHUNK / GG_BK; ++st) {
                    if (st < steps) {
                        const uint32_t gs = n_ord * ksteps + ch * (GG_CHUNK / GG_BK) + st;
                        const uint32_t ast = gs % SA;
                        if (!gg_wait(&a_empty[ast], ((gs / SA) & 1u) ^ 1u, abort_flag, p.status)) goto conv_done;
                        tc_fence_after();
                        uint32_t v[32];
                        if (st == 0) gg_decode<TYPE, 0>(row, win_off, v);
                        else if (st == 1) gg_decode<TYPE, 1>(row, win_off, v);
                        else if (st == 2) gg_decode<TYPE, 2>(row, win_off, v);
                        else gg_decode<TYPE, 3>(row, win_off, v);
                        tmem_st32(tmem + lane_addr + L::A_COL0 + ast * L::A_STAGE_COLS + m * 32u, v);
                        tmem_wait_st();
                        tc_fence_before();
                        __syncwarp();
                        if (lane == 0) mbar_arrive(&a_full[ast]);
                    }
                }
                __syncwarp();
                issue(j + RS);
            }

            // epilogue: accumulators -> act (SwiGLU, fp16) or part (f32)
            if (!gg_wait(acc_full, n_ord & 1u, abort_flag, p.status)) goto conv_done;
            tc_fence_after();
#pragma unroll 1
            for (uint32_t h = 0; h < BN / 64; ++h) {
                const uint32_t j0 = wg * (BN / 2) + h * 32u;
                if (j0 >= g.n_tok) break;
                uint32_t a[32];
                tmem_ld32(tmem + lane_addr + j0, a);
                const uint32_t orow0 = g.rt * GG_BM + row_in_tile;
                if constexpr (EPI == GG_EPI_SWIGLU) {
                    uint32_t b[32];
                    tmem_ld32(tmem + lane_addr + BN + j0, b);
                    tmem_wait_ld();
                    __half *out = static_cast<__half *>(p.out);
#pragma unroll
                    for (uint32_t t = 0; t < 32; ++t) {
                        if (j0 + t < g.n_tok) {
                            const float gv = __uint_as_float(a[t]), uv = __uint_as_float(b[t]);
                            const float act = gv / (1.0f + __expf(-gv)) * uv;
                            out[static_cast<uint64_t>(g.row_b0 + j0 + t) * p.out_dim + orow0] = __float2half_rn(act);
                        }
                    }
                } else {
                    tmem_wait_ld();
                    float *out = static_cast<float *>(p.out);
#pragma unroll
                    for (uint32_t t = 0; t < 32; ++t) {
                        if (j0 + t < g.n_tok) {
                            const uint32_t r = p.out_rows ? __ldg(p.out_rows + g.row_b0 + j0 + t) : g.row_b0 + j0 + t;
                            out[static_cast<uint64_t>(r) * p.out_dim + orow0] = __uint_as_float(a[t]);
                        }
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(acc_empty);
        }
    conv_done:
        cp_async_wait<0>();
    }

    __syncthreads();
    if (warp == 2) {
        tc_fence_after();
        tmem_dealloc(tmem, GG_TMEM_COLS);
    }
}

} // namespace fmb
