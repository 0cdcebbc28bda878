// router.cu -- K4: the native router and the grouping of tokens by expert.
//
// Router (linear-topk-softmax-v1), one warp per token:
//   softmax  Engine::softmax, src/engine.cpp:378-393: max in float, exp of
//            (double)v - max in double, sum in double in index order, float(e/sum);
//            a non-finite logit is INTERNAL_ERROR.
//   top-k    Engine::topk, src/engine.cpp:395-411: the first k of a stable
//            descending sort, ties to the lower id.
//   renorm   src/engine.cpp:1680-1702: float total in top-k order,
//            w = float(w / max(double(total), eps)), then float(w * scale).
// The double sum runs in index order on one lane so that it rounds exactly as
// the reference's loop does.
#include <algorithm>

#include "common.cuh"
#include "router_core.cuh"

namespace fmb {

int launch_route(const float *logits, uint32_t tokens, uint32_t experts, uint32_t top_k,
                 int32_t normalise, double epsilon, double scale, uint32_t *ids, float *weights,
                 float *probs, cudaStream_t s);

__global__ void route_kernel(const float *__restrict__ logits, uint32_t tokens, uint32_t experts,
                             uint32_t top_k, int normalise, double epsilon, double scale,
                             uint32_t *__restrict__ ids, float *__restrict__ weights,
                             float *__restrict__ probs_out, int *status) {
    extern __shared__ unsigned char smem_raw[];
    const int warps = blockDim.x >> 5;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    double *ex = reinterpret_cast<double *>(smem_raw) + static_cast<size_t>(warp) * experts;
    float *pr = reinterpret_cast<float *>(reinterpret_cast<double *>(smem_raw) +
                                          static_cast<size_t>(warps) * experts) +
                static_cast<size_t>(warp) * experts;
    const uint32_t t = blockIdx.x * warps + warp;
    if (t >= tokens) return;
    route_token(logits, t, experts, top_k, normalise, epsilon, scale, ids, weights, probs_out, status, ex, pr, lane);
}

__global__ void group_kernel(const uint32_t *__restrict__ ids, uint32_t n_pairs, uint32_t experts,
                             uint32_t *__restrict__ counts, uint32_t *__restrict__ offsets,
                             uint32_t *__restrict__ pairs, uint32_t *__restrict__ slot_of,
                             int *status) {
    __shared__ uint32_t s_count[kMaxExperts];
    __shared__ uint32_t s_off[kMaxExperts];
    __shared__ uint32_t s_warp_tot[32];
    group_block(ids, n_pairs, experts, counts, offsets, pairs, slot_of, status, s_count, s_off, s_warp_tot);
}

} // namespace fmb

using namespace fmb;

namespace fmb {
// ---- the router's model-family variants (src/engine.cpp:1603-1702) ---------
//
//   logit bias      scores[e] += bias[e] (float)                     :1608-1613
//   gating          softmax (Engine::softmax), sigmoid float(1/(1+exp(-(double)s))),
//                   sqrt-softplus float(sqrt(log1p(exp((double)s)))), or
//                   softmax-weight (probabilities = the logits)      :1618-1633
//   selection bias  selection[e] = probs[e] + bias[e] (float), picks only :1637-1643
//   groups          keep the groups_used groups whose two best selection values
//                   sum highest (float; stable, ties to the lower group), mask
//                   the others to -inf                               :1644-1675
//   top-k           Engine::topk on the selection; NaN or +inf is INTERNAL_ERROR,
//                   -inf (masked) is allowed                         :1676, :395-411
//   weights         probs of the picked experts; total = float sum in top-k order;
//                   softmax-weight softmaxes the picked weights; renormalise by
//                   max(double(total), eps) or double(total) + eps; float(w*scale)
//                                                                    :1677-1702
// One warp per token, as route_kernel.

__device__ __forceinline__ void warp_top2(float &a, float &b) {
    // merge each lane's (a >= b) pair across the warp
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float oa = __shfl_xor_sync(0xFFFFFFFFu, a, o), ob = __shfl_xor_sync(0xFFFFFFFFu, b, o);
        const float hi = fmaxf(a, oa), lo = fmaxf(fminf(a, oa), fmaxf(b, ob));
        a = hi;
        b = lo;
    }
}

__global__ void route_ex_kernel(const float *__restrict__ logits, uint32_t tokens, uint32_t experts,
                                uint32_t top_k, fmcuda_router_config cfg, uint32_t *__restrict__ ids,
                                float *__restrict__ weights, float *__restrict__ probs_out, int *status) {
    extern __shared__ unsigned char smem_raw[];
    const int warps = blockDim.x >> 5;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const size_t per_warp = static_cast<size_t>(experts) * 20; // double ex + float pr, sel, gsum
    unsigned char *base = smem_raw + static_cast<size_t>(warp) * per_warp;
    double *ex = reinterpret_cast<double *>(base);
    float *pr = reinterpret_cast<float *>(base + static_cast<size_t>(experts) * 8);
    float *sel = pr + experts;
    float *gsum = sel + experts;
    const uint32_t t = blockIdx.x * warps + warp;
    if (t >= tokens) return;
    const float *v = logits + static_cast<uint64_t>(t) * experts;
    auto fail_token = [&]() {
        if (lane == 0) raise_device_status(status, FM_STATUS_INTERNAL_ERROR);
        for (uint32_t r = lane; r < top_k; r += 32) {
            ids[static_cast<uint64_t>(t) * top_k + r] = 0xFFFFFFFFu;
            weights[static_cast<uint64_t>(t) * top_k + r] = 0.0f;
        }
    };

    // scores (+ logit bias) and the gating function
    float mx = -INFINITY;
    bool bad = false;
    for (uint32_t e = lane; e < experts; e += 32) {
        float x = v[e];
        if (cfg.logit_bias) x = __fadd_rn(x, cfg.logit_bias[e]);
        pr[e] = x;
        bad |= !isfinite(x);
        mx = fmaxf(mx, x);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, o));
    if (cfg.gating == FM_GATING_SOFTMAX && __any_sync(0xFFFFFFFFu, bad)) { // Engine::softmax's check
        fail_token();
        return;
    }
    __syncwarp();
    if (cfg.gating == FM_GATING_SOFTMAX) {
        for (uint32_t e = lane; e < experts; e += 32)
            ex[e] = exp(static_cast<double>(pr[e]) - static_cast<double>(mx));
        __syncwarp();
        double sum = 0.0;
        if (lane == 0)
            for (uint32_t e = 0; e < experts; ++e) sum += ex[e];
        sum = __shfl_sync(0xFFFFFFFFu, sum, 0);
        for (uint32_t e = lane; e < experts; e += 32) pr[e] = static_cast<float>(ex[e] / sum);
    } else if (cfg.gating == FM_GATING_SIGMOID) {
        for (uint32_t e = lane; e < experts; e += 32)
            pr[e] = static_cast<float>(1.0 / (1.0 + exp(-static_cast<double>(pr[e]))));
    } else if (cfg.gating == FM_GATING_SQRT_SOFTPLUS) {
        for (uint32_t e = lane; e < experts; e += 32)
            pr[e] = static_cast<float>(sqrt(log1p(exp(static_cast<double>(pr[e])))));
    } // FM_GATING_SOFTMAX_WEIGHT: the probabilities are the scores
    __syncwarp();
    bad = false;
    for (uint32_t e = lane; e < experts; e += 32) {
        if (probs_out) probs_out[static_cast<uint64_t>(t) * experts + e] = pr[e];
        float s = pr[e];
        if (cfg.selection_bias) s = __fadd_rn(s, cfg.selection_bias[e]);
        sel[e] = s;
        bad |= isnan(s) || s == INFINITY;
    }
    if (__any_sync(0xFFFFFFFFu, bad)) { // Engine::topk's check
        fail_token();
        return;
    }
    __syncwarp();

    // group-limited selection
    if (cfg.groups > 1) {
        const uint32_t per = experts / cfg.groups;
        for (uint32_t g = 0; g < cfg.groups; ++g) {
            float a = -INFINITY, b = -INFINITY;
            for (uint32_t e = lane; e < per; e += 32) {
                const float x = sel[g * per + e];
                if (x > a) {
                    b = a;
                    a = x;
                } else if (x > b) {
                    b = x;
                }
            }
            warp_top2(a, b);
            if (lane == 0) gsum[g] = per >= 2 ? __fadd_rn(__fadd_rn(0.0f, a), b) : __fadd_rn(0.0f, a);
        }
        __syncwarp();
        for (uint32_t g = lane; g < cfg.groups; g += 32) {
            uint32_t rank = 0;
            for (uint32_t h = 0; h < cfg.groups; ++h)
                rank += (gsum[h] > gsum[g]) || (gsum[h] == gsum[g] && h < g);
            if (rank >= cfg.groups_used)
                for (uint32_t e = 0; e < per; ++e) sel[g * per + e] = -INFINITY;
        }
        __syncwarp();
    }

    // top-k over the selection: value descending, id ascending; taken = NaN
    uint32_t my_id = 0xFFFFFFFFu;
    float my_w = 0.0f;
    for (uint32_t r = 0; r < top_k; ++r) {
        float bv = -INFINITY;
        uint32_t bi = 0xFFFFFFFFu;
        for (uint32_t e = lane; e < experts; e += 32) {
            const float p = sel[e];
            if (p > bv || (bi == 0xFFFFFFFFu && p == bv)) {
                bv = p;
                bi = e;
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xFFFFFFFFu, bv, o);
            const uint32_t oi = __shfl_xor_sync(0xFFFFFFFFu, bi, o);
            if (oi != 0xFFFFFFFFu && (bi == 0xFFFFFFFFu || ov > bv || (ov == bv && oi < bi))) {
                bv = ov;
                bi = oi;
            }
        }
        if (lane == static_cast<int>(r)) {
            my_id = bi;
            my_w = pr[bi];
        }
        __syncwarp();
        if (lane == 0) sel[bi] = __int_as_float(0x7FC00000); // NaN: never picked again
        __syncwarp();
    }
    float total = 0.0f;
    for (uint32_t r = 0; r < top_k; ++r) total = __fadd_rn(total, __shfl_sync(0xFFFFFFFFu, my_w, r));
    float w = my_w;
    if (cfg.gating == FM_GATING_SOFTMAX_WEIGHT &&
        __any_sync(0xFFFFFFFFu, static_cast<uint32_t>(lane) < top_k && !isfinite(w))) { // Engine::softmax's check
        fail_token();
        return;
    }
    if (cfg.gating == FM_GATING_SOFTMAX_WEIGHT) {
        // Engine::softmax over the k picked values (lane r holds value r)
        float m = static_cast<uint32_t>(lane) < top_k ? w : -INFINITY;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xFFFFFFFFu, m, o));
        const double e_r = static_cast<uint32_t>(lane) < top_k ? exp(static_cast<double>(w) - static_cast<double>(m)) : 0.0;
        double sum = 0.0;
        for (uint32_t r = 0; r < top_k; ++r) sum += __shfl_sync(0xFFFFFFFFu, e_r, r);
        w = static_cast<float>(e_r / sum);
    }
    if (static_cast<uint32_t>(lane) < top_k) {
        if (cfg.normalise) {
            const double tot = static_cast<double>(total);
            const double denom = cfg.epsilon_additive ? tot + cfg.epsilon : (tot > cfg.epsilon ? tot : cfg.epsilon);
            w = static_cast<float>(static_cast<double>(w) / denom);
        }
        w = static_cast<float>(static_cast<double>(w) * cfg.scale);
        ids[static_cast<uint64_t>(t) * top_k + lane] = my_id;
        weights[static_cast<uint64_t>(t) * top_k + lane] = w;
    }
}

int launch_route_ex(const float *logits, uint32_t tokens, uint32_t experts, uint32_t top_k,
                    const fmcuda_router_config &cfg, uint32_t *ids, float *weights, float *probs, cudaStream_t s) {
    if (cfg.gating < FM_GATING_SOFTMAX || cfg.gating > FM_GATING_SOFTMAX_WEIGHT)
        return set_error(FM_STATUS_INVALID_ARGUMENT, "unknown gating function");
    if (cfg.groups > 1 && (experts % cfg.groups || cfg.groups_used == 0 || cfg.groups_used > cfg.groups))
        return set_error(FM_STATUS_SHAPE_MISMATCH, "group-limited routing needs E % groups == 0 and 1 <= used <= groups");
    const size_t per_warp = static_cast<size_t>(experts) * 20;
    const int warps = static_cast<int>(std::max<size_t>(1, std::min<size_t>(4, (48u * 1024u) / per_warp)));
    route_ex_kernel<<<(tokens + warps - 1) / warps, warps * 32, per_warp * warps, s>>>(
        logits, tokens, experts, top_k, cfg, ids, weights, probs, device_status_word());
    return check_launch("router launch");
}

// The default configuration (softmax, no biases, no groups) goes to the
// original kernel; any other to route_ex_kernel.
int launch_route_cfg(const float *logits, uint32_t tokens, uint32_t experts, uint32_t top_k,
                     const fmcuda_router_config *cfg, int32_t normalise, double epsilon, double scale,
                     uint32_t *ids, float *weights, float *probs, cudaStream_t s) {
    if (!cfg || (cfg->gating == FM_GATING_SOFTMAX && !cfg->logit_bias && !cfg->selection_bias && cfg->groups <= 1 &&
                 !cfg->epsilon_additive))
        return launch_route(logits, tokens, experts, top_k, cfg ? cfg->normalise : normalise,
                            cfg ? cfg->epsilon : epsilon, cfg ? cfg->scale : scale, ids, weights, probs, s);
    return launch_route_ex(logits, tokens, experts, top_k, *cfg, ids, weights, probs, s);
}

int launch_route(const float *logits, uint32_t tokens, uint32_t experts, uint32_t top_k,
                 int32_t normalise, double epsilon, double scale, uint32_t *ids, float *weights,
                 float *probs, cudaStream_t s) {
    const int warps = 4;
    const size_t smem = static_cast<size_t>(warps) * experts * (sizeof(double) + sizeof(float));
    route_kernel<<<(tokens + warps - 1) / warps, warps * 32, smem, s>>>(
        logits, tokens, experts, top_k, normalise, epsilon, scale, ids, weights, probs,
        device_status_word());
    return check_launch("router launch");
}

// ---- grouping for large batches (prefill): the same outputs as group_kernel
// (a key of 0xFFFFFFFF is an absent item: no group, no error),
// computed by many warps.  Each warp owns 256 consecutive pairs; a pair's
// place is offsets[e] + (pairs of expert e in earlier warps) + (earlier pairs
// of expert e in its own warp), so the order inside an expert's group is
// ascending pair index, exactly as in group_kernel.

constexpr uint32_t kGroupWarpPairs = 256;

__global__ void group_count_kernel(const uint32_t *__restrict__ ids, uint32_t n_pairs, uint32_t experts,
                                   uint32_t *__restrict__ warp_counts, int *status) {
    extern __shared__ uint32_t s_hist[];
    const uint32_t lane = threadIdx.x & 31u, wl = threadIdx.x >> 5;
    const uint32_t w = blockIdx.x * (blockDim.x >> 5) + wl;
    const uint32_t nw = (n_pairs + kGroupWarpPairs - 1) / kGroupWarpPairs;
    if (w >= nw) return;
    uint32_t *h = s_hist + wl * experts;
    for (uint32_t e = lane; e < experts; e += 32) h[e] = 0;
    __syncwarp();
    for (uint32_t base = w * kGroupWarpPairs; base < min(n_pairs, (w + 1) * kGroupWarpPairs); base += 32) {
        const uint32_t i = base + lane;
        const bool valid = i < n_pairs;
        const uint32_t e = valid ? ids[i] : 0xFFFFFFFFu;
        const bool ok = valid && e < experts;
        // key 0xFFFFFFFF marks "no item" (skipped silently); any other key >= experts is an error
        if (valid && !ok && e != 0xFFFFFFFFu) raise_device_status(status, FM_STATUS_INVALID_EXPERT_ID);
        const uint32_t key = ok ? e : 0xFFFFFFFEu - (valid ? 0u : 1u);
        const uint32_t peers = __match_any_sync(0xFFFFFFFFu, key);
        if (ok && __popc(peers & ((1u << lane) - 1u)) == 0) h[e] += __popc(peers);
        __syncwarp();
    }
    for (uint32_t e = lane; e < experts; e += 32) warp_counts[static_cast<uint64_t>(w) * experts + e] = h[e];
}

// warp_counts[w][e] -> pairs of expert e in warps before w; counts, offsets.
__global__ void group_scan_kernel(uint32_t *__restrict__ warp_counts, uint32_t n_warps, uint32_t experts,
                                  uint32_t *__restrict__ counts, uint32_t *__restrict__ offsets) {
    __shared__ uint32_t s_warp_tot[32];
    const uint32_t tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    uint32_t mine = 0;
    if (tid < experts) {
        for (uint32_t w = 0; w < n_warps; ++w) {
            uint32_t *c = warp_counts + static_cast<uint64_t>(w) * experts + tid;
            const uint32_t v = *c;
            *c = mine;
            mine += v;
        }
    }
    uint32_t incl = mine;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const uint32_t n = __shfl_up_sync(0xFFFFFFFFu, incl, o);
        if (lane >= static_cast<uint32_t>(o)) incl += n;
    }
    if (lane == 31) s_warp_tot[warp] = incl;
    __syncthreads();
    if (warp == 0) {
        const uint32_t wt = s_warp_tot[lane];
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
        counts[tid] = mine;
        offsets[tid] = excl;
        if (tid == experts - 1) offsets[experts] = excl + mine;
    }
}

__global__ void group_place_kernel(const uint32_t *__restrict__ ids, uint32_t n_pairs, uint32_t experts,
                                   const uint32_t *__restrict__ warp_base, const uint32_t *__restrict__ offsets,
                                   uint32_t *__restrict__ pairs, uint32_t *__restrict__ slot_of) {
    extern __shared__ uint32_t s_run[];
    const uint32_t lane = threadIdx.x & 31u, wl = threadIdx.x >> 5;
    const uint32_t w = blockIdx.x * (blockDim.x >> 5) + wl;
    const uint32_t nw = (n_pairs + kGroupWarpPairs - 1) / kGroupWarpPairs;
    if (w >= nw) return;
    uint32_t *run = s_run + wl * experts;
    for (uint32_t e = lane; e < experts; e += 32)
        run[e] = offsets[e] + warp_base[static_cast<uint64_t>(w) * experts + e];
    __syncwarp();
    for (uint32_t base = w * kGroupWarpPairs; base < min(n_pairs, (w + 1) * kGroupWarpPairs); base += 32) {
        const uint32_t i = base + lane;
        const bool valid = i < n_pairs;
        const uint32_t e = valid ? ids[i] : 0xFFFFFFFFu;
        const bool ok = valid && e < experts;
        const uint32_t key = ok ? e : 0xFFFFFFFEu - (valid ? 0u : 1u);
        const uint32_t peers = __match_any_sync(0xFFFFFFFFu, key);
        const uint32_t rank = __popc(peers & ((1u << lane) - 1u));
        const uint32_t cur = ok ? run[e] : 0u;
        __syncwarp();
        if (ok) {
            const uint32_t pos = cur + rank;
            pairs[pos] = i;
            if (slot_of) slot_of[i] = pos;
            if (rank == 0) run[e] = cur + __popc(peers);
        } else if (valid && slot_of) {
            slot_of[i] = 0xFFFFFFFFu;
        }
        __syncwarp();
    }
}

uint64_t group_scratch_bytes(uint32_t n_pairs, uint32_t experts) {
    const uint64_t nw = (static_cast<uint64_t>(n_pairs) + kGroupWarpPairs - 1) / kGroupWarpPairs;
    return nw * experts * 4;
}

int launch_group_large(const uint32_t *ids, uint32_t n_pairs, uint32_t experts, uint32_t *counts,
                       uint32_t *offsets, uint32_t *pairs, uint32_t *slot_of, uint32_t *scratch,
                       cudaStream_t s) {
    if (experts == 0 || experts > kMaxExperts)
        return set_error(FM_STATUS_INVALID_ARGUMENT, "grouping takes 1..1024 experts");
    const uint32_t nw = (n_pairs + kGroupWarpPairs - 1) / kGroupWarpPairs;
    constexpr uint32_t kWarps = 4;
    const uint32_t blocks = (nw + kWarps - 1) / kWarps;
    const size_t smem = static_cast<size_t>(kWarps) * experts * 4;
    if (nw) {
        group_count_kernel<<<blocks, kWarps * 32, smem, s>>>(ids, n_pairs, experts, scratch, device_status_word());
        int rc = check_launch("grouping count launch");
        if (rc) return rc;
    }
    group_scan_kernel<<<1, 1024, 0, s>>>(scratch, nw, experts, counts, offsets);
    int rc = check_launch("grouping scan launch");
    if (rc || !nw) return rc;
    group_place_kernel<<<blocks, kWarps * 32, smem, s>>>(ids, n_pairs, experts, scratch, offsets, pairs, slot_of);
    return check_launch("grouping place launch");
}

int launch_group(const uint32_t *ids, uint32_t n_pairs, uint32_t experts, uint32_t *counts,
                 uint32_t *offsets, uint32_t *pairs, uint32_t *slot_of, cudaStream_t s) {
    group_kernel<<<1, 1024, 0, s>>>(ids, n_pairs, experts, counts, offsets, pairs, slot_of,
                                    device_status_word());
    return check_launch("grouping launch");
}

int check_route_args(uint32_t experts, uint32_t top_k) {
    if (experts == 0 || experts > static_cast<uint32_t>(kMaxExperts))
        return set_error(FM_STATUS_INVALID_ARGUMENT,
                         "expert count must be in 1..1024, got " + std::to_string(experts));
    if (top_k > experts) return set_error(FM_STATUS_INVALID_ARGUMENT, "top-k exceeds expert count");
    if (top_k == 0 || top_k > 32)
        return set_error(FM_STATUS_INVALID_ARGUMENT, "top-k must be in 1..32");
    return FM_STATUS_OK;
}
} // namespace fmb

extern "C" int fmcuda_route(const float *logits, uint32_t tokens, uint32_t experts,
                            uint32_t top_k, int32_t normalise, double epsilon, double scale,
                            uint32_t *ids, float *weights, float *probs, void *stream) {
    int rc = check_route_args(experts, top_k);
    if (rc) return rc;
    if (tokens == 0) return FM_STATUS_OK;
    if (!logits || !ids || !weights) return set_error(FM_STATUS_INVALID_ARGUMENT, "null router pointer");
    return launch_route(logits, tokens, experts, top_k, normalise, epsilon, scale, ids, weights,
                        probs, static_cast<cudaStream_t>(stream));
}

extern "C" int fmcuda_group(const uint32_t *ids, uint32_t tokens, uint32_t top_k,
                            uint32_t experts, uint32_t *counts, uint32_t *offsets, uint32_t *pairs,
                            uint32_t *slot_of, void *stream) {
    if (experts == 0 || experts > static_cast<uint32_t>(kMaxExperts))
        return set_error(FM_STATUS_INVALID_ARGUMENT, "expert count must be in 1..1024");
    if (!ids || !counts || !offsets || !pairs)
        return set_error(FM_STATUS_INVALID_ARGUMENT, "null grouping pointer");
    const uint64_t n = static_cast<uint64_t>(tokens) * top_k;
    if (n > 0xFFFFFFF0ull) return set_error(FM_STATUS_INVALID_ARGUMENT, "too many pairs");
    return launch_group(ids, static_cast<uint32_t>(n), experts, counts, offsets, pairs, slot_of,
                        static_cast<cudaStream_t>(stream));
}

extern "C" uint64_t fmcuda_group_scratch_bytes(uint32_t n_pairs, uint32_t experts) {
    return group_scratch_bytes(n_pairs, experts);
}

extern "C" int fmcuda_group_batched(const uint32_t *ids, uint32_t tokens, uint32_t top_k, uint32_t experts,
                                    uint32_t *counts, uint32_t *offsets, uint32_t *pairs, uint32_t *slot_of,
                                    void *scratch, void *stream) {
    if (!ids || !counts || !offsets || !pairs || !scratch)
        return set_error(FM_STATUS_INVALID_ARGUMENT, "null grouping pointer");
    const uint64_t n = static_cast<uint64_t>(tokens) * top_k;
    if (n > 0xFFFFFFF0ull) return set_error(FM_STATUS_INVALID_ARGUMENT, "too many pairs");
    return launch_group_large(ids, static_cast<uint32_t>(n), experts, counts, offsets, pairs, slot_of,
                              static_cast<uint32_t *>(scratch), static_cast<cudaStream_t>(stream));
}

extern "C" int fmcuda_route_ex(const float *logits, uint32_t tokens, uint32_t experts, uint32_t top_k,
                               const fmcuda_router_config *config, uint32_t *ids, float *weights, float *probs,
                               void *stream) {
    if (!config) return set_error(FM_STATUS_INVALID_ARGUMENT, "null router configuration");
    int rc = check_route_args(experts, top_k);
    if (rc) return rc;
    if (tokens == 0) return FM_STATUS_OK;
    if (!logits || !ids || !weights) return set_error(FM_STATUS_INVALID_ARGUMENT, "null router pointer");
    return launch_route_cfg(logits, tokens, experts, top_k, config, 1, 0.0, 1.0, ids, weights, probs,
                            static_cast<cudaStream_t>(stream));
}
