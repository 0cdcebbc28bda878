// fnv.cu -- FNV-1a 64 of a device byte range, computed in parallel and
// bit-identical to the reference's sequential checksum fm::fnv1a64
// (include/fm/common.hpp:73-81), which the residency manager evaluates over
// every expert payload and again over the slot copy after the upload
// (src/residency.cpp:656-667, :700-720).
//
// Why a byte-serial hash parallelises.  One step is h' = (h ^ b) * P mod 2^64
// with b < 256 and P = 0x100000001B3.
//  * The low byte s = h mod 256 evolves on its own, s' = (s ^ b) * P mod 256
//    (the low bits of a product depend only on the low bits of the operands).
//    Because P is odd, bit k of s' is bit k of (s ^ b) XOR a function of the
//    bits below k of (s ^ b).  So once the bits below k of a chunk's starting
//    state are known, running the chunk from bit k = 0 yields bit k at its end
//    up to an XOR with the true starting bit k, and the true starting bits are
//    an exclusive prefix XOR over the chunks before.  Eight rounds, one bit
//    each, give every chunk its exact starting low byte.
//  * XOR with b changes only the low byte, so h ^ b = h + d with
//    d = (s ^ b) - s.  With the low-byte trajectory fixed, a chunk is affine in
//    its starting hash: h_end = P^L h_start + A, where A = F - P^L s_start and
//    F is the chunk's FNV run from the start value s_start.  Hence
//    h_N = P^N h_0 + sum_c (P^(N-end_c) F_c - P^(N-start_c) s_c), a sum mod 2^64.
// Every operation is integer arithmetic mod 2^64, so the result is exact.
//
// Launches: one init kernel, eight round kernels (bit k of every chunk's start
// state), one final kernel (bit 7, then the chunk terms, summed with 64-bit
// atomics into the result word).  Each thread owns one 512-byte chunk.
#include "common.cuh"

namespace fmb {
namespace {

constexpr uint64_t kFnvBasis = 0xCBF29CE484222325ull;
constexpr uint64_t kFnvPrime = 0x100000001B3ull;
constexpr uint32_t kFnvPrimeLow = 0xB3u; // P mod 256
constexpr uint32_t kChunk = 512;         // bytes per thread
constexpr uint32_t kThreads = 256;       // threads per CTA

struct FnvWork {
    uint8_t *start;    // [chunks] known low bits of each chunk's starting state
    uint8_t *t;        // [chunks] end bit of the current round
    const uint8_t *blk_prev; // [blocks] per-CTA XOR of t, previous round
    uint8_t *blk_cur;        // [blocks] the same, this round (the two alternate)
};

__host__ __device__ inline uint64_t pow_p(uint64_t e) {
    uint64_t r = 1, b = kFnvPrime;
    while (e) {
        if (e & 1) r *= b;
        b *= b;
        e >>= 1;
    }
    return r;
}

__device__ __forceinline__ uint32_t low_step4(uint32_t s, uint32_t w) {
    // only bits 0..7 of s are meaningful; higher bits carry harmless garbage
    s = (s ^ w) * kFnvPrimeLow;
    s = (s ^ (w >> 8)) * kFnvPrimeLow;
    s = (s ^ (w >> 16)) * kFnvPrimeLow;
    return (s ^ (w >> 24)) * kFnvPrimeLow;
}

__device__ __forceinline__ uint64_t full_step4(uint64_t h, uint32_t w) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        h ^= (w >> (8 * j)) & 0xFFu;
        h *= kFnvPrime;
    }
    return h;
}

// Runs one chunk: the low byte only (FULL = false) or the whole 64-bit hash.
template <bool FULL, bool ALIGNED, typename S>
__device__ __forceinline__ S run_chunk(const uint8_t *p, uint32_t len, S s) {
    uint32_t i = 0;
    if (ALIGNED) {
        const uint4 *v = reinterpret_cast<const uint4 *>(p);
        for (; i + 16 <= len; i += 16) {
            const uint4 q = __ldg(v + i / 16);
            if constexpr (FULL) {
                s = full_step4(full_step4(full_step4(full_step4(s, q.x), q.y), q.z), q.w);
            } else {
                s = low_step4(low_step4(low_step4(low_step4(static_cast<uint32_t>(s), q.x), q.y), q.z), q.w);
            }
        }
    }
    for (; i < len; ++i) {
        const uint32_t b = __ldg(p + i);
        if constexpr (FULL) {
            s = (s ^ b) * kFnvPrime;
        } else {
            s = (static_cast<uint32_t>(s) ^ b) * kFnvPrimeLow;
        }
    }
    return s;
}

// Exclusive prefix XOR of the previous round's end bits: every chunk's true
// starting bit (k - 1), folded into w.start.  Called by all threads of a CTA.
__device__ __forceinline__ uint32_t finish_bit(const FnvWork &w, uint32_t k, uint64_t c,
                                               bool valid, uint32_t nblk_prev) {
    const uint32_t lane = threadIdx.x & 31u, warp = threadIdx.x >> 5;
    __shared__ uint32_t s_warp[kThreads / 32];
    const uint32_t t = valid ? w.t[c] : 0u;
    // CTAs before this one
    uint32_t x = 0;
    for (uint32_t j = threadIdx.x; j < blockIdx.x && j < nblk_prev; j += kThreads) x ^= w.blk_prev[j];
    const uint32_t before = static_cast<uint32_t>(__syncthreads_count(x & 1u)) & 1u;
    // threads before this one in the CTA
    const uint32_t bal = __ballot_sync(0xFFFFFFFFu, t);
    uint32_t pre = static_cast<uint32_t>(__popc(bal & ((1u << lane) - 1u))) & 1u;
    if (lane == 0) s_warp[warp] = static_cast<uint32_t>(__popc(bal)) & 1u;
    __syncthreads();
    for (uint32_t j = 0; j < warp; ++j) pre ^= s_warp[j];
    const uint32_t bit = (static_cast<uint32_t>(kFnvBasis >> (k - 1)) ^ before ^ pre) & 1u;
    // round 1 sets bit 0 of a fresh value; later rounds add to what is stored
    uint32_t s0 = valid && k > 1 ? w.start[c] : 0u;
    s0 |= bit << (k - 1);
    if (valid) w.start[c] = static_cast<uint8_t>(s0);
    return s0;
}

__global__ void fnv_init_kernel(uint64_t *out, uint64_t n) { *out = pow_p(n) * kFnvBasis; }

template <bool ALIGNED>
__global__ void __launch_bounds__(kThreads) fnv_round_kernel(const uint8_t *data, uint64_t n,
                                                             uint64_t chunks, FnvWork w, uint32_t k) {
    const uint64_t c = static_cast<uint64_t>(blockIdx.x) * kThreads + threadIdx.x;
    const bool valid = c < chunks;
    uint32_t s0 = 0;
    if (k > 0) s0 = finish_bit(w, k, c, valid, gridDim.x);
    uint32_t t = 0;
    if (valid) {
        const uint64_t off = c * kChunk;
        const uint32_t len = static_cast<uint32_t>(n - off < kChunk ? n - off : kChunk);
        const uint32_t s = run_chunk<false, ALIGNED>(data + off, len, s0);
        t = (s >> k) & 1u;
        w.t[c] = static_cast<uint8_t>(t);
    }
    const uint32_t odd = static_cast<uint32_t>(__syncthreads_count(t)) & 1u;
    if (threadIdx.x == 0) w.blk_cur[blockIdx.x] = static_cast<uint8_t>(odd);
}

template <bool ALIGNED>
__global__ void __launch_bounds__(kThreads) fnv_final_kernel(const uint8_t *data, uint64_t n,
                                                             uint64_t chunks, FnvWork w, uint64_t *out) {
    const uint64_t c = static_cast<uint64_t>(blockIdx.x) * kThreads + threadIdx.x;
    const bool valid = c < chunks;
    const uint32_t s0 = finish_bit(w, 8, c, valid, gridDim.x);
    uint64_t term = 0;
    if (valid) {
        const uint64_t off = c * kChunk;
        const uint32_t len = static_cast<uint32_t>(n - off < kChunk ? n - off : kChunk);
        const uint64_t f = run_chunk<true, ALIGNED>(data + off, len, static_cast<uint64_t>(s0));
        term = pow_p(n - off - len) * f - pow_p(n - off) * static_cast<uint64_t>(s0);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) term += __shfl_xor_sync(0xFFFFFFFFu, term, o);
    if ((threadIdx.x & 31u) == 0 && term != 0) atomicAdd(reinterpret_cast<unsigned long long *>(out), term);
}

uint64_t fnv_chunks(uint64_t n) { return (n + kChunk - 1) / kChunk; }

uint64_t fnv_blocks(uint64_t n) { return (fnv_chunks(n) + kThreads - 1) / kThreads; }

} // namespace

uint64_t fnv1a64_workspace_bytes(uint64_t n) {
    const uint64_t c = fnv_chunks(n), b = fnv_blocks(n);
    return ((2 * c + 255) & ~uint64_t(255)) + ((2 * b + 255) & ~uint64_t(255));
}

int fnv1a64_launch(const void *data, uint64_t n, uint64_t *out, void *workspace, uint64_t ws_bytes,
                   cudaStream_t stream) {
    if (!out || (n && !data)) return set_error(FM_STATUS_INVALID_ARGUMENT, "fnv1a64: null pointer");
    if (reinterpret_cast<uintptr_t>(out) & 7u)
        return set_error(FM_STATUS_INVALID_ARGUMENT, "fnv1a64: result word is not 8-byte aligned");
    const uint64_t chunks = fnv_chunks(n), blocks = fnv_blocks(n);
    if (blocks > 0x7FFFFFFFull) return set_error(FM_STATUS_INVALID_ARGUMENT, "fnv1a64: range too large");
    if (n && (!workspace || ws_bytes < fnv1a64_workspace_bytes(n)))
        return set_error(FM_STATUS_INVALID_ARGUMENT, "fnv1a64: workspace too small");
    fnv_init_kernel<<<1, 1, 0, stream>>>(out, n);
    int rc = check_launch("fnv1a64 init");
    if (rc || n == 0) return rc;
    uint8_t *ws = static_cast<uint8_t *>(workspace);
    FnvWork w;
    w.start = ws;
    w.t = ws + chunks;
    uint8_t *blk[2] = {ws + ((2 * chunks + 255) & ~uint64_t(255)), nullptr};
    blk[1] = blk[0] + blocks;
    const bool aligned = (reinterpret_cast<uintptr_t>(data) & 15u) == 0;
    const uint8_t *p = static_cast<const uint8_t *>(data);
    const dim3 grid(static_cast<uint32_t>(blocks));
    for (uint32_t k = 0; k < 8; ++k) {
        w.blk_prev = blk[(k + 1) & 1u];
        w.blk_cur = blk[k & 1u];
        if (aligned)
            fnv_round_kernel<true><<<grid, kThreads, 0, stream>>>(p, n, chunks, w, k);
        else
            fnv_round_kernel<false><<<grid, kThreads, 0, stream>>>(p, n, chunks, w, k);
        if ((rc = check_launch("fnv1a64 round"))) return rc;
    }
    w.blk_prev = blk[1];
    w.blk_cur = nullptr;
    if (aligned)
        fnv_final_kernel<true><<<grid, kThreads, 0, stream>>>(p, n, chunks, w, out);
    else
        fnv_final_kernel<false><<<grid, kThreads, 0, stream>>>(p, n, chunks, w, out);
    return check_launch("fnv1a64 final");
}

} // namespace fmb

extern "C" uint64_t fmcuda_fnv1a64_workspace_bytes(uint64_t bytes) { return fmb::fnv1a64_workspace_bytes(bytes); }

extern "C" int fmcuda_fnv1a64(const void *data, uint64_t bytes, uint64_t *out, void *workspace,
                              uint64_t workspace_bytes, void *stream) {
    return fmb::fnv1a64_launch(data, bytes, out, workspace, workspace_bytes,
                               static_cast<cudaStream_t>(stream));
}
