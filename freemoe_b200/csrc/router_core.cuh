// router_core.cuh -- device bodies of the native router (one warp per token)
// and of the one-CTA grouping by expert, shared by the standalone kernels
// (router.cu) and the fused decode front kernel (moe.cu).
//
// Router (linear-topk-softmax-v1):
//   softmax  Engine::softmax, src/engine.cpp:378-393: max in float, exp of
//            (double)v - max in double, sum in double in index order, float(e/sum);
//            a non-finite logit is INTERNAL_ERROR.
//   top-k    Engine::topk, src/engine.cpp:395-411: the first k of a stable
//            descending sort, ties to the lower id.
//   renorm   src/engine.cpp:1680-1702: float total in top-k order,
//            w = float(w / max(double(total), eps)), then float(w * scale).
#pragma once

#include "common.cuh"

namespace fmb {

constexpr int kMaxExperts = 1024;

// One token by one warp; ex / pr are the warp's `experts` doubles / floats of
// shared memory.
__device__ __forceinline__ void route_token(const float *__restrict__ logits, uint32_t t, uint32_t experts,
                                            uint32_t top_k, int normalise, double epsilon, double scale,
                                            uint32_t *__restrict__ ids, float *__restrict__ weights,
                                            float *__restrict__ probs_out, int *status, double *ex, float *pr,
                                            int lane) {
    const float *v = logits + static_cast<uint64_t>(t) * experts;

    // max over the logits (float), finiteness check
    float mx = -INFINITY;
    bool bad = false;
    for (uint32_t e = lane; e < experts; e += 32) {
        const float x = v[e];
        bad |= !isfinite(x);
        mx = fmaxf(mx, x);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, o));
    bad = __any_sync(0xFFFFFFFFu, bad);
    if (bad) {
        if (lane == 0) raise_device_status(status, FM_STATUS_INTERNAL_ERROR);
        for (uint32_t r = lane; r < top_k; r += 32) {
            ids[static_cast<uint64_t>(t) * top_k + r] = 0xFFFFFFFFu;
            weights[static_cast<uint64_t>(t) * top_k + r] = 0.0f;
        }
        return;
    }
    for (uint32_t e = lane; e < experts; e += 32)
        ex[e] = exp(static_cast<double>(v[e]) - static_cast<double>(mx));
    __syncwarp();
    double sum = 0.0;
    if (lane == 0)
        for (uint32_t e = 0; e < experts; ++e) sum += ex[e];
    sum = __shfl_sync(0xFFFFFFFFu, sum, 0);
    for (uint32_t e = lane; e < experts; e += 32) {
        const float p = static_cast<float>(ex[e] / sum);
        pr[e] = p;
        if (probs_out) probs_out[static_cast<uint64_t>(t) * experts + e] = p;
    }
    __syncwarp();

    // top-k: k rounds of a warp arg-max (value descending, id ascending)
    uint32_t my_id = 0xFFFFFFFFu;
    float my_w = 0.0f;
    for (uint32_t r = 0; r < top_k; ++r) {
        float bv = -INFINITY;
        uint32_t bi = 0xFFFFFFFFu;
        for (uint32_t e = lane; e < experts; e += 32) {
            const float p = pr[e];
            if (p > bv || (bi == 0xFFFFFFFFu && p == bv)) {
                bv = p;
                bi = e;
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xFFFFFFFFu, bv, o);
            const uint32_t oi = __shfl_xor_sync(0xFFFFFFFFu, bi, o);
            if (ov > bv || (ov == bv && oi < bi)) {
                bv = ov;
                bi = oi;
            }
        }
        if (lane == r) {
            my_id = bi;
            my_w = bv;
        }
        __syncwarp();
        if (lane == 0) pr[bi] = -INFINITY; // taken (probabilities are >= 0)
        __syncwarp();
    }
    // renormalisation: the float total in top-k order
    float total = 0.0f;
    for (uint32_t r = 0; r < top_k; ++r) total = __fadd_rn(total, __shfl_sync(0xFFFFFFFFu, my_w, r));
    if (static_cast<uint32_t>(lane) < top_k) {
        float w = my_w;
        if (normalise) {
            const double denom = static_cast<double>(total) > epsilon ? static_cast<double>(total)
                                                                      : epsilon;
            w = static_cast<float>(static_cast<double>(w) / denom);
        }
        w = static_cast<float>(static_cast<double>(w) * scale);
        ids[static_cast<uint64_t>(t) * top_k + lane] = my_id;
        weights[static_cast<uint64_t>(t) * top_k + lane] = w;
    }
}

// Grouping by expert in one CTA: histogram, exclusive scan, then a stable
// rank of each pair within its expert.  Key 0xFFFFFFFF is an absent pair (no
// slot, no error), any other key >= experts raises INVALID_EXPERT_ID.  The ranking walks the pairs in flat
// order 32 at a time with __match_any_sync, so the result is the ascending
// token order of the host grouping, independent of scheduling.
// The whole CTA (1024 threads) groups; s_count / s_off hold `experts` words,
// s_warp_tot 32.
__device__ __forceinline__ void group_block(const uint32_t *__restrict__ ids, uint32_t n_pairs, uint32_t experts,
                                            uint32_t *__restrict__ counts, uint32_t *__restrict__ offsets,
                                            uint32_t *__restrict__ pairs, uint32_t *__restrict__ slot_of,
                                            int *status, uint32_t *s_count, uint32_t *s_off, uint32_t *s_warp_tot) {
    for (uint32_t e = threadIdx.x; e < experts; e += blockDim.x) s_count[e] = 0;
    __syncthreads();
    for (uint32_t i = threadIdx.x; i < n_pairs; i += blockDim.x) {
        const uint32_t e = ids[i];
        if (e < experts) atomicAdd(&s_count[e], 1u);
        else if (e != 0xFFFFFFFFu) raise_device_status(status, FM_STATUS_INVALID_EXPERT_ID);
    }
    __syncthreads();
    // exclusive scan over experts (blockDim.x == 1024 >= experts)
    const uint32_t tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const uint32_t mine = tid < experts ? s_count[tid] : 0u;
    uint32_t incl = mine;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const uint32_t n = __shfl_up_sync(0xFFFFFFFFu, incl, o);
        if (lane >= static_cast<uint32_t>(o)) incl += n;
    }
    if (lane == 31) s_warp_tot[warp] = incl;
    __syncthreads();
    if (warp == 0) {
        uint32_t wt = s_warp_tot[lane];
        uint32_t wincl = wt;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const uint32_t n = __shfl_up_sync(0xFFFFFFFFu, wincl, o);
            if (lane >= static_cast<uint32_t>(o)) wincl += n;
        }
        s_warp_tot[lane] = wincl - wt;
    }
    __syncthreads();
    const uint32_t excl = incl - mine + s_warp_tot[warp];
    if (tid < experts) {
        s_off[tid] = excl;
        counts[tid] = mine;
        offsets[tid] = excl;
        if (tid == experts - 1) offsets[experts] = excl + mine;
    }
    __syncthreads();
    // stable ranking by warp 0; s_off[e] becomes the running cursor
    if (warp == 0) {
        for (uint32_t base = 0; base < n_pairs; base += 32) {
            const uint32_t i = base + lane;
            const bool valid = i < n_pairs;
            const uint32_t e = valid ? ids[i] : 0xFFFFFFFFu;
            const bool ok = valid && e < experts;
            const uint32_t key = ok ? e : 0xFFFFFFFEu - (valid ? 0u : 1u);
            const uint32_t peers = __match_any_sync(0xFFFFFFFFu, key);
            const uint32_t rank = __popc(peers & ((1u << lane) - 1u));
            const uint32_t cur = ok ? s_off[e] : 0u;
            __syncwarp();
            if (ok) {
                const uint32_t pos = cur + rank;
                pairs[pos] = i;
                if (slot_of) slot_of[i] = pos;
                if (rank == 0) s_off[e] = cur + __popc(peers);
            } else if (valid && slot_of) {
                slot_of[i] = 0xFFFFFFFFu;
            }
            __syncwarp();
        }
    }
}

} // namespace fmb
