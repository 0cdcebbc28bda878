// moe.cu -- one routed-expert MoE block on the device (src/engine.cpp:1603-1772).
//
// Launch sequence on one stream (no host synchronisation):
//   1. router        logits -> ids, weights                (router.cu)
//   2. grouping      ids -> counts, offsets, pairs, slot_of (router.cu)
//   3. x planes      x -> fp16 plane(s) + sub-block sums    (gemv_core.cuh)
//      (1-3 are one CTA-sized launch, moe_front_kernel, for short batches)
//   4. gate/up       per expert, fused gate and up GEMV with SwiGLU -> act[slot]
//   5. act planes    act -> fp16 planes + sums (written by the gate/up epilogue
//                    when both GEMVs are the streamed kernel)
//   6. down          per expert, down GEMV -> part[slot]
//   7. combine       y[t] = sum over r of w[t,r] * part[slot_of(t,r)], in top-k
//                    order, multiply then add (src/engine.cpp:1770)
// Each expert's weight rows are read once per 8 of its tokens.
// Q4_K experts with bf16 activations take the tcgen05 expert stage (tgemv.cu)
// instead of 3-6: for short batches with the plain router one launch
// (tg_front_kernel) routes, groups and writes the gate/up B images, then the
// gate/up and down GEMVs and the combine: four launches per block.
#include <string>

#include "gemv_async.cuh"
#include "gemv_kernels.cuh"
#include "router_core.cuh"
#include "tgemv_host.h"

namespace fmb {

int launch_route_cfg(const float *logits, uint32_t tokens, uint32_t experts, uint32_t top_k,
                     const fmcuda_router_config *cfg, int32_t normalise, double epsilon, double scale,
                     uint32_t *ids, float *weights, float *probs, cudaStream_t s);
int launch_group(const uint32_t *ids, uint32_t n_pairs, uint32_t experts, uint32_t *counts,
                 uint32_t *offsets, uint32_t *pairs, uint32_t *slot_of, cudaStream_t s);
int check_route_args(uint32_t experts, uint32_t top_k);
int launch_xplanes_for(uint32_t type_id, const void *x, int32_t x_dtype, uint32_t rows, uint32_t k_dim,
                       __half *xh, __half *xl, float *xs, cudaStream_t s);
template <int MODE>
int launch_qgemv(const QGemvParams &prm, int planes, uint32_t grid_y, uint32_t grid_z,
                 cudaStream_t s);
int check_quant_shape(uint32_t type_id, uint32_t in_dim, const char *what);
int check_quant_alignment(uint32_t type_id, uint64_t byte_offset, const char *what);
bool staged_shape(uint32_t type_id, uint32_t in_dim);
int xplane_layout(uint32_t type_id);
int launch_xplanes_staged(const void *x, int32_t x_dtype, uint32_t rows, uint32_t k_dim, int layout,
                          __half *xh, __half *xl, float *xs, cudaStream_t s);
template <int MODE>
int launch_qgemv_stream(const QGemvParams &prm, int planes, uint32_t tok_tiles, uint32_t experts,
                     cudaStream_t s);

namespace {

inline uint64_t a256(uint64_t v) { return (v + 255) & ~uint64_t(255); }

// Steps 1-3 for a short batch in one launch: CTA 0 runs the router (warp w
// takes tokens w, w + 32, ...) and, once the ids are visible to the CTA, the
// grouping (the whole CTA); CTAs 1.. write the x planes.  Same device code and
// results as the three separate kernels, two launches fewer.
constexpr uint32_t kFrontMaxTokens = 64, kFrontMaxExperts = 64;

template <typename XT>
__global__ void __launch_bounds__(1024)
    moe_front_kernel(const float *__restrict__ logits, const XT *__restrict__ x, uint32_t tokens, uint32_t experts,
                     uint32_t top_k, int normalise, double epsilon, double scale, uint32_t d, int layout,
                     uint32_t *ids, float *weights, uint32_t *counts, uint32_t *offsets, uint32_t *pairs,
                     uint32_t *slot_of, __half *xh, __half *xl, float *xs, int *status) {
    __shared__ double s_ex[32][kFrontMaxExperts];
    __shared__ float s_pr[32][kFrontMaxExperts];
    __shared__ uint32_t s_count[kFrontMaxExperts], s_off[kFrontMaxExperts], s_warp_tot[32];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (blockIdx.x > 0) {
        const uint32_t subs = d / 32;
        for (uint32_t i = (blockIdx.x - 1) * blockDim.x + threadIdx.x; i < tokens * subs;
             i += (gridDim.x - 1) * blockDim.x)
            xplanes_staged_item(x, i / subs, i % subs, d, layout, xh, xl, xs);
        return;
    }
    for (uint32_t t = warp; t < tokens; t += 32)
        route_token(logits, t, experts, top_k, normalise, epsilon, scale, ids, weights, nullptr, status, s_ex[warp],
                    s_pr[warp], lane);
    __syncthreads();
    group_block(ids, tokens * top_k, experts, counts, offsets, pairs, slot_of, status, s_count, s_off, s_warp_tot);
}

// Byte layout of the MoE workspace.
struct MoeLayout {
    uint64_t ids, weights, counts, offsets, pairs, slot_of;
    uint64_t xh, xl, xs;
    uint64_t act, ah, al, as;
    uint64_t part;
    uint64_t tg_img_gu, tg_img_dn, tg_partial, tg_cnt, tg_maps; // tcgen05 expert stage (tgemv.cu)
    uint64_t total;
};

MoeLayout moe_layout(uint32_t tokens, uint32_t experts, uint32_t top_k, uint32_t d,
                     uint32_t ffn) {
    MoeLayout L{};
    const uint64_t P = static_cast<uint64_t>(tokens) * top_k;
    uint64_t o = 0;
    auto take = [&](uint64_t bytes) {
        const uint64_t at = o;
        o += a256(bytes);
        return at;
    };
    L.ids = take(P * 4);
    L.weights = take(P * 4);
    L.counts = take(static_cast<uint64_t>(experts) * 4);
    L.offsets = take((static_cast<uint64_t>(experts) + 1) * 4);
    L.pairs = take(P * 4);
    L.slot_of = take(P * 4);
    L.xh = take(static_cast<uint64_t>(tokens) * d * 2);
    L.xl = take(static_cast<uint64_t>(tokens) * d * 2);
    L.xs = take(static_cast<uint64_t>(tokens) * (d / 32) * 4);
    L.act = take(P * ffn * 4);
    L.ah = take(P * ffn * 2);
    L.al = take(P * ffn * 2);
    L.as = take(P * (ffn / 32) * 4);
    L.part = take(P * d * 4);
    const TgSections tg = tg_sections(static_cast<uint32_t>(P), experts, d, ffn);
    L.tg_img_gu = take(tg.img_gu);
    L.tg_img_dn = take(tg.img_dn);
    L.tg_partial = take(tg.partial);
    L.tg_cnt = take(tg.cnt);
    L.tg_maps = take(tg.maps);
    L.total = o;
    return L;
}

__global__ void combine_kernel(const float *__restrict__ part, const float *__restrict__ weights,
                               const uint32_t *__restrict__ slot_of, uint32_t tokens,
                               uint32_t top_k, uint32_t d, float *__restrict__ y) {
    const uint64_t id = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x;
    if (id >= static_cast<uint64_t>(tokens) * d) return;
    const uint32_t t = static_cast<uint32_t>(id / d), j = static_cast<uint32_t>(id % d);
    float acc = 0.0f;
    for (uint32_t r = 0; r < top_k; ++r) {
        const uint32_t slot = slot_of[static_cast<uint64_t>(t) * top_k + r];
        if (slot == 0xFFFFFFFFu) continue;
        acc = __fadd_rn(acc, __fmul_rn(weights[static_cast<uint64_t>(t) * top_k + r],
                                       part[static_cast<uint64_t>(slot) * d + j]));
    }
    y[id] = acc;
}

// The same combine, four consecutive outputs per thread (16-byte loads and
// stores); the arithmetic per element is unchanged.
__global__ void combine4_kernel(const float *__restrict__ part, const float *__restrict__ weights,
                                const uint32_t *__restrict__ slot_of, uint32_t tokens, uint32_t top_k, uint32_t d,
                                float *__restrict__ y) {
    const uint64_t id = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x;
    const uint32_t d4 = d / 4;
    if (id >= static_cast<uint64_t>(tokens) * d4) return;
    const uint32_t t = static_cast<uint32_t>(id / d4), j = static_cast<uint32_t>(id % d4);
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (uint32_t r = 0; r < top_k; ++r) {
        const uint32_t slot = slot_of[static_cast<uint64_t>(t) * top_k + r];
        if (slot == 0xFFFFFFFFu) continue;
        const float w = weights[static_cast<uint64_t>(t) * top_k + r];
        const float4 v = __ldg(reinterpret_cast<const float4 *>(part + static_cast<uint64_t>(slot) * d) + j);
        acc.x = __fadd_rn(acc.x, __fmul_rn(w, v.x));
        acc.y = __fadd_rn(acc.y, __fmul_rn(w, v.y));
        acc.z = __fadd_rn(acc.z, __fmul_rn(w, v.z));
        acc.w = __fadd_rn(acc.w, __fmul_rn(w, v.w));
    }
    reinterpret_cast<float4 *>(y)[id] = acc;
}

} // namespace

// y[t] = sum over r of w[t,r] * part[slot_of(t,r)]; also used by the prefill path.
int launch_combine(const float *part, const float *weights, const uint32_t *slot_of, uint32_t tokens,
                   uint32_t top_k, uint32_t d, float *y, cudaStream_t s) {
    const uint64_t n = static_cast<uint64_t>(tokens) * d;
    if (d % 4 == 0 && reinterpret_cast<uintptr_t>(part) % 16 == 0 && reinterpret_cast<uintptr_t>(y) % 16 == 0)
        combine4_kernel<<<static_cast<unsigned>((n / 4 + 255) / 256), 256, 0, s>>>(part, weights, slot_of, tokens,
                                                                                  top_k, d, y);
    else
        combine_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0, s>>>(part, weights, slot_of, tokens, top_k,
                                                                              d, y);
    return check_launch("combine launch");
}


// Shared by the allocating entry point and any variant that brings its own scratch.
int moe_block_run(const fmcuda_moe_args *a, void *workspace, uint64_t workspace_bytes,
                  cudaStream_t s) {
    if (!a) return set_error(FM_STATUS_INVALID_ARGUMENT, "null MoE arguments");
    if (a->tokens == 0) return FM_STATUS_OK;
    int rc = check_route_args(a->experts, a->top_k);
    if (rc) return rc;
    if (!a->x || !a->logits || !a->expert_slots || !a->y)
        return set_error(FM_STATUS_INVALID_ARGUMENT, "null MoE pointer");
    if (a->x_dtype != FM_X_F32 && a->x_dtype != FM_X_BF16)
        return set_error(FM_STATUS_INVALID_ARGUMENT, "unknown activation dtype");
    if ((rc = check_quant_shape(a->gate_type, a->d_model, "expert gate"))) return rc;
    if ((rc = check_quant_shape(a->up_type, a->d_model, "expert up"))) return rc;
    if ((rc = check_quant_shape(a->down_type, a->ffn, "expert down"))) return rc;
    // slot bases are device-checked; the offsets inside a slot are checked here
    if ((rc = check_quant_alignment(a->up_type, a->up_offset, "expert up offset"))) return rc;
    if ((rc = check_quant_alignment(a->down_type, a->down_offset, "expert down offset"))) return rc;
    if (a->gate_type != a->up_type)
        return set_error(FM_STATUS_UNSUPPORTED_QUANTISATION,
                         "fused gate/up needs one block type for both projections");
    if (a->gate_type == FM_TYPE_F32 || a->down_type == FM_TYPE_F32)
        return set_error(FM_STATUS_UNSUPPORTED_QUANTISATION,
                         "F32 experts run through fmcuda_matvec_f32 (Backend::matvec)");
    const MoeLayout L = moe_layout(a->tokens, a->experts, a->top_k, a->d_model, a->ffn);
    if (!workspace || workspace_bytes < L.total)
        return set_error(FM_STATUS_INVALID_ARGUMENT,
                         "MoE workspace too small: need " + std::to_string(L.total) + " bytes");
    uint8_t *ws = static_cast<uint8_t *>(workspace);
    uint32_t *ids = reinterpret_cast<uint32_t *>(ws + L.ids);
    float *weights = reinterpret_cast<float *>(ws + L.weights);
    uint32_t *counts = reinterpret_cast<uint32_t *>(ws + L.counts);
    uint32_t *offsets = reinterpret_cast<uint32_t *>(ws + L.offsets);
    uint32_t *pairs = reinterpret_cast<uint32_t *>(ws + L.pairs);
    uint32_t *slot_of = reinterpret_cast<uint32_t *>(ws + L.slot_of);
    __half *xh = reinterpret_cast<__half *>(ws + L.xh);
    __half *xl = reinterpret_cast<__half *>(ws + L.xl);
    float *xs = reinterpret_cast<float *>(ws + L.xs);
    float *act = reinterpret_cast<float *>(ws + L.act);
    __half *ah = reinterpret_cast<__half *>(ws + L.ah);
    __half *al = reinterpret_cast<__half *>(ws + L.al);
    float *as = reinterpret_cast<float *>(ws + L.as);
    float *part = reinterpret_cast<float *>(ws + L.part);
    const uint32_t P = a->tokens * a->top_k;
    int mark_rc = FM_STATUS_OK;
    auto mark = [&](int i) {
        if (a->stage_events && a->stage_events[i] && mark_rc == FM_STATUS_OK) {
            const cudaError_t err = cudaEventRecord(static_cast<cudaEvent_t>(a->stage_events[i]), s);
            if (err != cudaSuccess) mark_rc = cuda_status(err, "stage event record");
        }
    };

    const int xplanes = a->x_dtype == FM_X_F32 ? 2 : 1;
    // Expert slots come from cudaMalloc-class allocations (256-byte aligned);
    // the staged kernels also re-check each slot base on the device.
    const bool gu_staged = staged_shape(a->gate_type, a->d_model) && a->up_offset % 16 == 0;
    const bool dn_staged = staged_shape(a->down_type, a->ffn) && a->down_offset % 16 == 0;
    const fmcuda_router_config *cfg = a->router;
    const bool plain_router = !cfg || (cfg->gating == FM_GATING_SOFTMAX && !cfg->logit_bias && !cfg->selection_bias &&
                                       cfg->groups <= 1 && !cfg->epsilon_additive);
    mark(0);
    if (tg_eligible(a)) {
        // Q4_K experts, bf16 activations: the tcgen05 expert stage (tgemv.cu)
        struct MarkCtx {
            decltype(mark) *fn;
        } mctx{&mark};
        auto mark_fn = [](void *ctx, int i) { (*static_cast<MarkCtx *>(ctx)->fn)(i); };
        TgStage ts{};
        ts.x = a->x;
        ts.x_f16 = false;
        ts.pairs_max = P;
        ts.top_k = a->top_k;
        ts.experts = a->experts;
        ts.d = a->d_model;
        ts.ffn = a->ffn;
        ts.slots = a->expert_slots;
        ts.up_offset = a->up_offset;
        ts.down_offset = a->down_offset;
        ts.counts = counts;
        ts.offsets = offsets;
        ts.pairs = pairs;
        ts.out_rows = nullptr;
        if (plain_router && tg_front_eligible(a->tokens, a->experts, a->top_k)) {
            // router, grouping and B images in one launch
            TgFront f{};
            f.logits = a->logits;
            f.tokens = a->tokens;
            f.normalise = cfg ? cfg->normalise : a->normalise;
            f.epsilon = cfg ? cfg->epsilon : a->epsilon;
            f.scale = cfg ? cfg->scale : a->scale;
            f.ids = ids;
            f.weights = weights;
            f.slot_of = slot_of;
            rc = tg_block_stage(ts, f, ws + L.tg_img_gu, ws + L.tg_img_dn, reinterpret_cast<float *>(ws + L.tg_partial),
                                reinterpret_cast<uint32_t *>(ws + L.tg_cnt), ws + L.tg_maps, part, mark_fn, &mctx, s);
        } else {
            if ((rc = launch_route_cfg(a->logits, a->tokens, a->experts, a->top_k, a->router, a->normalise,
                                       a->epsilon, a->scale, ids, weights, nullptr, s)))
                return rc;
            mark(1);
            if ((rc = launch_group(ids, P, a->experts, counts, offsets, pairs, slot_of, s))) return rc;
            mark(2);
            rc = tg_expert_stage(ts, ws + L.tg_img_gu, ws + L.tg_img_dn, reinterpret_cast<float *>(ws + L.tg_partial),
                                 reinterpret_cast<uint32_t *>(ws + L.tg_cnt), ws + L.tg_maps, part, mark_fn, &mctx, s);
        }
        if (rc) return rc;
        if ((rc = launch_combine(part, weights, slot_of, a->tokens, a->top_k, a->d_model, a->y, s))) return rc;
        mark(7);
        if (a->ids_out)
            cudaMemcpyAsync(a->ids_out, ids, static_cast<uint64_t>(P) * 4, cudaMemcpyDeviceToDevice, s);
        if (a->weights_out)
            cudaMemcpyAsync(a->weights_out, weights, static_cast<uint64_t>(P) * 4, cudaMemcpyDeviceToDevice, s);
        if (mark_rc) return mark_rc;
        return check_launch("MoE output copies");
    }
    if (plain_router && gu_staged && a->tokens <= kFrontMaxTokens && a->experts <= kFrontMaxExperts) {
        const int norm = cfg ? cfg->normalise : a->normalise;
        const double eps = cfg ? cfg->epsilon : a->epsilon, scl = cfg ? cfg->scale : a->scale;
        const int layout = xplane_layout(a->gate_type);
        __half *xl_or_null = xplanes > 1 ? xl : nullptr;
        const unsigned front_grid = 1 + (a->tokens * (a->d_model / 32) + 1023) / 1024;
        if (a->x_dtype == FM_X_BF16)
            moe_front_kernel<__nv_bfloat16><<<front_grid, 1024, 0, s>>>(
                a->logits, static_cast<const __nv_bfloat16 *>(a->x), a->tokens, a->experts, a->top_k, norm, eps, scl,
                a->d_model, layout, ids, weights, counts, offsets, pairs, slot_of, xh, xl_or_null, xs,
                device_status_word());
        else
            moe_front_kernel<float><<<front_grid, 1024, 0, s>>>(
                a->logits, static_cast<const float *>(a->x), a->tokens, a->experts, a->top_k, norm, eps, scl,
                a->d_model, layout, ids, weights, counts, offsets, pairs, slot_of, xh, xl_or_null, xs,
                device_status_word());
        if ((rc = check_launch("MoE front launch"))) return rc;
        mark(1);
        mark(2);
    } else {
        if ((rc = launch_route_cfg(a->logits, a->tokens, a->experts, a->top_k, a->router, a->normalise, a->epsilon,
                                   a->scale, ids, weights, nullptr, s)))
            return rc;
        mark(1);
        if ((rc = launch_group(ids, P, a->experts, counts, offsets, pairs, slot_of, s))) return rc;
        mark(2);
        rc = gu_staged ? launch_xplanes_staged(a->x, a->x_dtype, a->tokens, a->d_model,
                                               xplane_layout(a->gate_type), xh, xplanes > 1 ? xl : nullptr, xs, s)
                       : launch_xplanes_for(a->gate_type, a->x, a->x_dtype, a->tokens, a->d_model, xh,
                                            xplanes > 1 ? xl : nullptr, xs, s);
        if (rc) return rc;
    }
    mark(3);

    const uint32_t tok_tiles = (a->tokens + 7) / 8; // an expert holds at most `tokens` pairs
    QGemvParams gu{};
    gu.slots = a->expert_slots;
    gu.w_off0 = 0;
    gu.w_off1 = a->up_offset;
    gu.type_id = a->gate_type;
    gu.out_dim = a->ffn;
    gu.in_dim = a->d_model;
    gu.row_bytes = row_bytes(a->gate_type, a->d_model);
    gu.offsets = offsets;
    gu.pairs = pairs;
    gu.top_k = a->top_k;
    gu.xh = xh;
    gu.xl = xplanes > 1 ? xl : nullptr;
    gu.xs = xs;
    gu.y = act;
    gu.status = device_status_word();
    // both GEMVs streamed: the gate/up epilogue writes the down projection's x
    // planes directly (same values and order as the separate plane kernel)
    const bool fused_planes = gu_staged && dn_staged && a->ffn % 32 == 0;
    if (fused_planes) {
        gu.act_h = ah;
        gu.act_l = al;
        gu.act_s = as;
        gu.act_layout = xplane_layout(a->down_type);
    }
    rc = gu_staged ? launch_qgemv_stream<GEMV_GATE_UP>(gu, xplanes, tok_tiles, a->experts, s)
                   : launch_qgemv<GEMV_GATE_UP>(gu, xplanes, tok_tiles, a->experts, s);
    if (rc) return rc;
    mark(4);

    rc = fused_planes ? FM_STATUS_OK
         : dn_staged  ? launch_xplanes_staged(act, FM_X_F32, P, a->ffn, xplane_layout(a->down_type), ah, al, as, s)
                      : launch_xplanes_for(a->down_type, act, FM_X_F32, P, a->ffn, ah, al, as, s);
    if (rc) return rc;
    mark(5);

    QGemvParams dn{};
    dn.slots = a->expert_slots;
    dn.w_off0 = a->down_offset;
    dn.w_off1 = a->down_offset;
    dn.type_id = a->down_type;
    dn.out_dim = a->d_model;
    dn.in_dim = a->ffn;
    dn.row_bytes = row_bytes(a->down_type, a->ffn);
    dn.offsets = offsets;
    dn.pairs = pairs;
    dn.top_k = a->top_k;
    dn.xh = ah;
    dn.xl = al;
    dn.xs = as;
    dn.y = part;
    dn.status = device_status_word();
    rc = dn_staged ? launch_qgemv_stream<GEMV_DOWN>(dn, 2, tok_tiles, a->experts, s)
                   : launch_qgemv<GEMV_DOWN>(dn, 2, tok_tiles, a->experts, s);
    if (rc) return rc;
    mark(6);

    if ((rc = launch_combine(part, weights, slot_of, a->tokens, a->top_k, a->d_model, a->y, s))) return rc;
    mark(7);
    if (a->ids_out)
        cudaMemcpyAsync(a->ids_out, ids, static_cast<uint64_t>(P) * 4, cudaMemcpyDeviceToDevice, s);
    if (a->weights_out)
        cudaMemcpyAsync(a->weights_out, weights, static_cast<uint64_t>(P) * 4,
                        cudaMemcpyDeviceToDevice, s);
    if (mark_rc) return mark_rc;
    return check_launch("MoE output copies");
}

uint64_t moe_workspace_size(uint32_t tokens, uint32_t experts, uint32_t top_k, uint32_t d,
                            uint32_t ffn) {
    return moe_layout(tokens, experts, top_k, d, ffn).total;
}

} // namespace fmb

using namespace fmb;

extern "C" int fmcuda_moe_workspace_bytes(uint32_t tokens, uint32_t experts, uint32_t top_k,
                                          uint32_t d_model, uint32_t ffn, uint64_t *bytes) {
    if (!bytes) return set_error(FM_STATUS_INVALID_ARGUMENT, "null size pointer");
    *bytes = moe_workspace_size(tokens, experts, top_k, d_model, ffn);
    return FM_STATUS_OK;
}

extern "C" int fmcuda_moe_block(const fmcuda_moe_args *args, void *workspace,
                                uint64_t workspace_bytes, void *stream) {
    return moe_block_run(args, workspace, workspace_bytes, static_cast<cudaStream_t>(stream));
}
