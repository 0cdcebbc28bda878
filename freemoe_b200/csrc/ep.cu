// ep.cu -- device pieces of the expert-parallel MoE layer (no reference
// counterpart: FreeMoe runs every expert in one process).  Experts are sharded
// contiguously over `world` ranks (expert e lives on rank e / experts_per_rank);
// every rank routes its own tokens.  The exchange itself (token rows out, expert
// outputs back) is done by the host's collective library between these calls:
//
//   fmcuda_route          ids, weights of the local tokens        (router.cu)
//   fmcuda_ep_dispatch    pairs grouped by destination rank, fp16 token rows
//                         and local expert ids packed in that order
//   -- all-to-all of the packed rows and expert ids (counts first) --
//   fmcuda_moe_experts    the received rows through the local experts: grouped
//                         by local expert, gate/up + SwiGLU and down on the
//                         tcgen05 grouped GEMM, outputs in received order
//   -- all-to-all of the outputs back to the owners of the tokens --
//   fmcuda_moe_combine    y[t] = sum over r of w[t,r] * out[slot_of(t,r)], in
//                         top-k order (src/engine.cpp:1770)
//
// Each pair's expert output is the same number whichever rank computes it (a
// grouped-GEMM column depends only on its own token row), so the layer's result
// equals fmcuda_moe_prefill's on one GPU bit for bit.
#include <functional>
#include <string>

#include "common.cuh"
#include "tgemv_host.h"

namespace fmb {

uint64_t group_scratch_bytes(uint32_t n_pairs, uint32_t experts);
int launch_group_large(const uint32_t *ids, uint32_t n_pairs, uint32_t experts, uint32_t *counts,
                       uint32_t *offsets, uint32_t *pairs, uint32_t *slot_of, uint32_t *scratch, cudaStream_t s);
int launch_combine(const float *part, const float *weights, const uint32_t *slot_of, uint32_t tokens,
                   uint32_t top_k, uint32_t d, float *y, cudaStream_t s);
int run_expert_gemms(uint32_t experts, const void *const *slots, uint64_t up_offset, uint64_t down_offset,
                     uint32_t gu_type, uint32_t dn_type, uint32_t d, uint32_t ffn, const uint32_t *counts,
                     const uint32_t *offsets, uint32_t rows, const __half *xg, __half *act, float *part,
                     const uint32_t *part_rows, const std::function<void(int)> *mark, cudaStream_t s);

namespace {

inline uint64_t a256(uint64_t v) { return (v + 255) & ~uint64_t(255); }

__global__ void ep_dest_kernel(const uint32_t *__restrict__ ids, uint32_t n, uint32_t per_rank,
                               uint32_t *__restrict__ dest) {
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) dest[i] = ids[i] / per_rank; // >= world for a bad id: the grouping flags it
}

// send row i <- pair send_pairs[i]: fp16 copy of its token row and its local expert id.
template <typename XT>
__global__ void ep_pack_kernel(const XT *__restrict__ x, const uint32_t *__restrict__ ids,
                               const uint32_t *__restrict__ send_pairs, const uint32_t *__restrict__ n_send,
                               uint32_t top_k, uint32_t per_rank, uint32_t d, __half *__restrict__ send_x,
                               uint32_t *__restrict__ send_expert) {
    const uint32_t i = blockIdx.x;
    if (i >= *n_send) return;
    const uint32_t p = send_pairs[i];
    const XT *src = x + static_cast<uint64_t>(p / top_k) * d;
    __half *dst = send_x + static_cast<uint64_t>(i) * d;
    for (uint32_t c = threadIdx.x * 2; c < d; c += blockDim.x * 2)
        *reinterpret_cast<__half2 *>(dst + c) = __floats2half2_rn(load_x(src + c), load_x(src + c + 1));
    if (threadIdx.x == 0) send_expert[i] = ids[p] % per_rank;
}

// xg[g] = x[pairs[g]] (fp16 rows, 16 bytes per thread step).
__global__ void gather_f16_rows_kernel(const __half *__restrict__ x, const uint32_t *__restrict__ pairs,
                                       const uint32_t *__restrict__ n_rows, uint32_t d, __half *__restrict__ xg) {
    const uint32_t g = blockIdx.x;
    if (g >= *n_rows) return;
    const uint4 *src = reinterpret_cast<const uint4 *>(x + static_cast<uint64_t>(pairs[g]) * d);
    uint4 *dst = reinterpret_cast<uint4 *>(xg + static_cast<uint64_t>(g) * d);
    for (uint32_t c = threadIdx.x; c < d / 8; c += blockDim.x) dst[c] = src[c];
}

// key of item t*world + dest: dest when token t has at least one pair on that
// rank, else 0xFFFFFFFF (absent).
__global__ void ep_row_keys_kernel(const uint32_t *__restrict__ ids, uint32_t tokens, uint32_t top_k,
                                   uint32_t per_rank, uint32_t world, uint32_t *__restrict__ keys) {
    const uint64_t i = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x;
    if (i >= static_cast<uint64_t>(tokens) * world) return;
    const uint32_t t = static_cast<uint32_t>(i / world), dest = static_cast<uint32_t>(i % world);
    bool any = false;
    for (uint32_t r = 0; r < top_k; ++r) any |= ids[static_cast<uint64_t>(t) * top_k + r] / per_rank == dest;
    keys[i] = any ? dest : 0xFFFFFFFFu;
}

// send row j <- item rows[j] = t*world + dest: the fp16 token row once, and for
// each top-k slot r the local expert (or -1 when that pair goes elsewhere) and
// its routing weight.
template <typename XT>
__global__ void ep_pack_rows_kernel(const XT *__restrict__ x, const uint32_t *__restrict__ ids,
                                    const float *__restrict__ w, const uint32_t *__restrict__ rows,
                                    const uint32_t *__restrict__ n_rows, uint32_t top_k, uint32_t per_rank,
                                    uint32_t world, uint32_t d, __half *__restrict__ send_x,
                                    int32_t *__restrict__ meta_e, float *__restrict__ meta_w) {
    const uint32_t j = blockIdx.x;
    if (j >= *n_rows) return;
    const uint32_t item = rows[j], t = item / world, dest = item % world;
    const XT *src = x + static_cast<uint64_t>(t) * d;
    __half *dst = send_x + static_cast<uint64_t>(j) * d;
    for (uint32_t c = threadIdx.x * 2; c < d; c += blockDim.x * 2)
        *reinterpret_cast<__half2 *>(dst + c) = __floats2half2_rn(load_x(src + c), load_x(src + c + 1));
    for (uint32_t r = threadIdx.x; r < top_k; r += blockDim.x) {
        const uint32_t e = ids[static_cast<uint64_t>(t) * top_k + r];
        const bool mine = e / per_rank == dest;
        meta_e[static_cast<uint64_t>(j) * top_k + r] = mine ? static_cast<int32_t>(e % per_rank) : -1;
        meta_w[static_cast<uint64_t>(j) * top_k + r] = mine ? w[static_cast<uint64_t>(t) * top_k + r] : 0.0f;
    }
}

// partial[row] = sum over the row's slots r (top-k order) of w_r * out[row*k + r]
__global__ void ep_partial_kernel(const float *__restrict__ out, const int32_t *__restrict__ meta_e,
                                  const float *__restrict__ meta_w, uint32_t rows, uint32_t top_k, uint32_t d,
                                  float *__restrict__ partial) {
    const uint64_t id = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x;
    if (id >= static_cast<uint64_t>(rows) * d) return;
    const uint32_t row = static_cast<uint32_t>(id / d), c = static_cast<uint32_t>(id % d);
    float acc = 0.0f;
    for (uint32_t r = 0; r < top_k; ++r) {
        const uint64_t slot = static_cast<uint64_t>(row) * top_k + r;
        if (meta_e[slot] >= 0) acc = __fadd_rn(acc, __fmul_rn(meta_w[slot], out[slot * d + c]));
    }
    partial[id] = acc;
}

// y[t] = sum over destination ranks (ascending) of the returned partial rows.
__global__ void ep_combine_rows_kernel(const float *__restrict__ back, const uint32_t *__restrict__ row_of,
                                       uint32_t tokens, uint32_t world, uint32_t d, float *__restrict__ y) {
    const uint64_t id = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x;
    if (id >= static_cast<uint64_t>(tokens) * d) return;
    const uint32_t t = static_cast<uint32_t>(id / d), c = static_cast<uint32_t>(id % d);
    float acc = 0.0f;
    for (uint32_t r = 0; r < world; ++r) {
        const uint32_t row = row_of[static_cast<uint64_t>(t) * world + r];
        if (row != 0xFFFFFFFFu) acc = __fadd_rn(acc, back[static_cast<uint64_t>(row) * d + c]);
    }
    y[id] = acc;
}

struct ExpertsLayout {
    uint64_t counts, offsets, pairs, gscratch, xg, act, total;
};

ExpertsLayout experts_layout(uint32_t rows, uint32_t experts, uint32_t d, uint32_t ffn) {
    ExpertsLayout L{};
    uint64_t o = 0;
    auto take = [&](uint64_t bytes) {
        const uint64_t at = o;
        o += a256(bytes);
        return at;
    };
    L.counts = take(static_cast<uint64_t>(experts) * 4);
    L.offsets = take((static_cast<uint64_t>(experts) + 1) * 4);
    L.pairs = take(static_cast<uint64_t>(rows) * 4);
    L.gscratch = take(group_scratch_bytes(rows, experts));
    L.xg = take(static_cast<uint64_t>(rows) * d * 2);
    L.act = take(static_cast<uint64_t>(rows) * ffn * 2);
    L.total = o;
    return L;
}

struct PartialLayout {
    uint64_t keys, counts, offsets, pairs, gscratch, xg, act, tg, out, total;
};

// Routed pairs at most: a row holds one slot per local expert it was sent for.
inline uint32_t partial_pairs_max(uint32_t rows, uint32_t top_k, uint32_t experts) {
    return rows * (top_k < experts ? top_k : experts);
}

// The tcgen05 decode stage (tgemv.cu) takes the experts' GEMMs when the weights
// are Q4_K and the experts hold one 8-token tile each on average (decode-sized
// batches: pairs <= 8 x experts); larger batches go to the grouped GEMM, which
// converts each weight tile once for up to 192 tokens.
inline bool partial_uses_tg(uint32_t rows, uint32_t top_k, uint32_t experts, uint32_t d, uint32_t ffn) {
    return tg_shape(d, ffn) && experts <= 1024 &&
           static_cast<uint64_t>(partial_pairs_max(rows, top_k, experts)) <= 8ull * experts;
}

PartialLayout partial_layout(uint32_t rows, uint32_t top_k, uint32_t experts, uint32_t d, uint32_t ffn) {
    PartialLayout L{};
    const uint64_t n = static_cast<uint64_t>(rows) * top_k;
    uint64_t o = 0;
    auto take = [&](uint64_t bytes) {
        const uint64_t at = o;
        o += a256(bytes);
        return at;
    };
    L.keys = take(n * 4);
    L.counts = take(static_cast<uint64_t>(experts) * 4);
    L.offsets = take((static_cast<uint64_t>(experts) + 1) * 4);
    L.pairs = take(n * 4);
    L.gscratch = take(group_scratch_bytes(static_cast<uint32_t>(n), experts));
    L.xg = take(n * d * 2);
    L.act = take(n * ffn * 2);
    L.tg = partial_uses_tg(rows, top_k, experts, d, ffn)
               ? take(tg_sections(partial_pairs_max(rows, top_k, experts), experts, d, ffn).total())
               : o;
    L.out = take(n * d * 4);
    L.total = o;
    return L;
}

// key of pair slot i = local expert, or absent for other ranks' slots and for
// rows at or past *rows_dev (when the row count lives on the device)
__global__ void ep_meta_keys_kernel(const int32_t *__restrict__ meta_e, uint64_t n, uint32_t top_k,
                                    const uint32_t *__restrict__ rows_dev, uint32_t *__restrict__ keys) {
    const uint64_t i = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x;
    if (i >= n) return;
    const bool live = !rows_dev || i / top_k < *rows_dev;
    keys[i] = live && meta_e[i] >= 0 ? static_cast<uint32_t>(meta_e[i]) : 0xFFFFFFFFu;
}

// xg[g] = x[pairs[g] / k]
__global__ void gather_pair_rows_kernel(const __half *__restrict__ x, const uint32_t *__restrict__ pairs,
                                        const uint32_t *__restrict__ n_rows, uint32_t top_k, uint32_t d,
                                        __half *__restrict__ xg) {
    const uint32_t g = blockIdx.x;
    if (g >= *n_rows) return;
    const uint4 *src = reinterpret_cast<const uint4 *>(x + static_cast<uint64_t>(pairs[g] / top_k) * d);
    uint4 *dst = reinterpret_cast<uint4 *>(xg + static_cast<uint64_t>(g) * d);
    for (uint32_t c = threadIdx.x; c < d / 8; c += blockDim.x) dst[c] = src[c];
}

} // namespace
} // namespace fmb

using namespace fmb;

extern "C" uint64_t fmcuda_ep_dispatch_rows_scratch_bytes(uint32_t tokens, uint32_t world) {
    const uint64_t n = static_cast<uint64_t>(tokens) * world;
    return a256(n * 4) + group_scratch_bytes(static_cast<uint32_t>(n), world);
}

extern "C" int fmcuda_ep_dispatch_rows(const uint32_t *ids, const float *weights, uint32_t tokens, uint32_t top_k,
                                       uint32_t experts_per_rank, uint32_t world, const void *x, int32_t x_dtype,
                                       uint32_t d_model, uint32_t *send_counts, uint32_t *send_offsets,
                                       uint32_t *send_items, uint32_t *row_of, void *send_x, int32_t *meta_expert,
                                       float *meta_weight, void *scratch, void *stream) {
    if (!ids || !weights || !x || !send_counts || !send_offsets || !send_items || !row_of || !send_x ||
        !meta_expert || !meta_weight || !scratch)
        return set_error(FM_STATUS_INVALID_ARGUMENT, "null dispatch pointer");
    if (world == 0 || world > 1024 || experts_per_rank == 0)
        return set_error(FM_STATUS_INVALID_ARGUMENT, "dispatch needs 1..1024 ranks and >= 1 expert per rank");
    if (x_dtype != FM_X_F32 && x_dtype != FM_X_BF16)
        return set_error(FM_STATUS_INVALID_ARGUMENT, "unknown activation dtype");
    if (d_model == 0 || d_model % 2) return set_error(FM_STATUS_SHAPE_MISMATCH, "d_model must be even");
    const uint64_t n64 = static_cast<uint64_t>(tokens) * world;
    if (n64 > 0x7FFFFFFFull) return set_error(FM_STATUS_INVALID_ARGUMENT, "too many token-rank items");
    const uint32_t n = static_cast<uint32_t>(n64);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    uint32_t *keys = static_cast<uint32_t *>(scratch);
    uint32_t *gscratch = reinterpret_cast<uint32_t *>(static_cast<uint8_t *>(scratch) + a256(n64 * 4));
    if (n) {
        ep_row_keys_kernel<<<(n + 255) / 256, 256, 0, s>>>(ids, tokens, top_k, experts_per_rank, world, keys);
        int rc = check_launch("dispatch row keys launch");
        if (rc) return rc;
    }
    int rc = launch_group_large(keys, n, world, send_counts, send_offsets, send_items, row_of, gscratch, s);
    if (rc || !n) return rc;
    if (x_dtype == FM_X_F32)
        ep_pack_rows_kernel<float><<<n, 128, 0, s>>>(static_cast<const float *>(x), ids, weights, send_items,
                                                     send_offsets + world, top_k, experts_per_rank, world, d_model,
                                                     static_cast<__half *>(send_x), meta_expert, meta_weight);
    else
        ep_pack_rows_kernel<__nv_bfloat16><<<n, 128, 0, s>>>(
            static_cast<const __nv_bfloat16 *>(x), ids, weights, send_items, send_offsets + world, top_k,
            experts_per_rank, world, d_model, static_cast<__half *>(send_x), meta_expert, meta_weight);
    return check_launch("dispatch row pack launch");
}

extern "C" uint64_t fmcuda_moe_experts_partial_workspace_bytes(uint32_t rows, uint32_t top_k, uint32_t experts,
                                                               uint32_t d_model, uint32_t ffn) {
    return partial_layout(rows, top_k, experts, d_model, ffn).total;
}

namespace fmb {
// The expert GEMMs of fmcuda_moe_experts_partial up to the per-pair outputs
// out_pairs[row * k + r] (rows = capacity when rows_dev holds the live count).
// Whether experts_partial_run takes the fused receive front of the tcgen05
// stage (then it also waits for the rows: the caller launches no wait).
bool partial_fused_recv(uint32_t rows, uint32_t top_k, uint32_t experts, uint32_t d_model, uint32_t ffn,
                        uint32_t gate_type, uint32_t up_type, uint32_t down_type, uint64_t up_offset,
                        uint64_t down_offset) {
    return rows > 0 && gate_type == FM_TYPE_Q4_K && up_type == FM_TYPE_Q4_K && down_type == FM_TYPE_Q4_K &&
           up_offset % 16 == 0 && down_offset % 16 == 0 && partial_uses_tg(rows, top_k, experts, d_model, ffn) &&
           tg_recv_eligible(rows, top_k, experts);
}

// recv: the peer exchange's receive wait, taken by the fused receive front
// (partial_fused_recv true), else NULL.
int experts_partial_run(const void *x, const int32_t *meta_expert, const float *meta_weight, uint32_t rows,
                        const uint32_t *rows_dev, uint32_t top_k, uint32_t experts, const void *const *expert_slots,
                        uint64_t up_offset, uint64_t down_offset, uint32_t gate_type, uint32_t up_type,
                        uint32_t down_type, uint32_t d_model, uint32_t ffn, float *out_pairs, void *workspace,
                        uint64_t workspace_bytes, cudaStream_t s, const TgRecvWait *recv) {
    if (rows == 0) return FM_STATUS_OK;
    if (!x || !meta_expert || !meta_weight || !expert_slots || !out_pairs)
        return set_error(FM_STATUS_INVALID_ARGUMENT, "null expert-compute pointer");
    if (experts == 0 || experts > 1024) return set_error(FM_STATUS_INVALID_ARGUMENT, "1..1024 local experts");
    if (gate_type != up_type)
        return set_error(FM_STATUS_UNSUPPORTED_QUANTISATION, "fused gate/up needs one block type for both projections");
    for (uint32_t t : {gate_type, down_type})
        if (t != FM_TYPE_Q8_0 && t != FM_TYPE_Q4_K && t != FM_TYPE_Q6_K)
            return set_error(FM_STATUS_UNSUPPORTED_QUANTISATION, "the grouped GEMM takes Q8_0, Q4_K or Q6_K weights");
    const uint32_t kq = gate_type != FM_TYPE_Q8_0 || down_type != FM_TYPE_Q8_0 ? 256 : 64;
    if (reinterpret_cast<uintptr_t>(x) % 16 || d_model % 128 || ffn % 128 || d_model % kq || ffn % kq)
        return set_error(FM_STATUS_SHAPE_MISMATCH,
                         "expert rows must be 16-byte aligned fp16; d_model and ffn multiples of 128 (256 for "
                         "Q4_K / Q6_K)");
    const uint64_t n64 = static_cast<uint64_t>(rows) * top_k;
    if (n64 > 0x7FFFFFFFull) return set_error(FM_STATUS_INVALID_ARGUMENT, "too many pairs");
    const uint32_t n = static_cast<uint32_t>(n64);
    const PartialLayout L = partial_layout(rows, top_k, experts, d_model, ffn);
    if (!workspace || workspace_bytes < L.out)
        return set_error(FM_STATUS_INVALID_ARGUMENT,
                         "expert workspace too small: need " + std::to_string(L.out) + " bytes");
    uint8_t *ws = static_cast<uint8_t *>(workspace);
    uint32_t *keys = reinterpret_cast<uint32_t *>(ws + L.keys);
    uint32_t *counts = reinterpret_cast<uint32_t *>(ws + L.counts);
    uint32_t *offsets = reinterpret_cast<uint32_t *>(ws + L.offsets);
    uint32_t *pairs = reinterpret_cast<uint32_t *>(ws + L.pairs);
    __half *xg = reinterpret_cast<__half *>(ws + L.xg);
    __half *act = reinterpret_cast<__half *>(ws + L.act);
    auto tg_stage = [&]() {
        const uint32_t pmax = partial_pairs_max(rows, top_k, experts);
        TgStage t{};
        t.x = x;
        t.x_f16 = true;
        t.pairs_max = pmax;
        t.top_k = top_k;
        t.experts = experts;
        t.d = d_model;
        t.ffn = ffn;
        t.slots = expert_slots;
        t.up_offset = up_offset;
        t.down_offset = down_offset;
        t.counts = counts;
        t.offsets = offsets;
        t.pairs = pairs;
        t.out_rows = pairs;
        return t;
    };
    if (recv) {
        if (!partial_fused_recv(rows, top_k, experts, d_model, ffn, gate_type, up_type, down_type, up_offset,
                                down_offset))
            return set_error(FM_STATUS_INTERNAL_ERROR, "receive wait passed to a batch without the fused front");
        // wait, grouping and images in one launch, then the decode GEMVs; the
        // output of grouped pair g goes to slot pairs[g]
        const TgStage t = tg_stage();
        const TgSections ts = tg_sections(t.pairs_max, experts, d_model, ffn);
        uint8_t *tg = ws + L.tg;
        return tg_recv_stage(t, *recv, tg, tg + ts.img_gu, reinterpret_cast<float *>(tg + ts.img_gu + ts.img_dn),
                             reinterpret_cast<uint32_t *>(tg + ts.img_gu + ts.img_dn + ts.partial),
                             tg + ts.img_gu + ts.img_dn + ts.partial + ts.cnt, out_pairs, s);
    }
    ep_meta_keys_kernel<<<static_cast<unsigned>((n64 + 255) / 256), 256, 0, s>>>(meta_expert, n64, top_k, rows_dev,
                                                                                 keys);
    int rc = check_launch("expert keys launch");
    if (rc) return rc;
    if ((rc = launch_group_large(keys, n, experts, counts, offsets, pairs, nullptr,
                                 reinterpret_cast<uint32_t *>(ws + L.gscratch), s)))
        return rc;
    if (gate_type == FM_TYPE_Q4_K && down_type == FM_TYPE_Q4_K && partial_uses_tg(rows, top_k, experts, d_model, ffn) &&
        up_offset % 16 == 0 && down_offset % 16 == 0) {
        // decode-sized batch: the tcgen05 decode stage reads the received rows in
        // place and writes the output of grouped pair g to slot pairs[g]
        const TgStage t = tg_stage();
        const TgSections ts = tg_sections(t.pairs_max, experts, d_model, ffn);
        uint8_t *tg = ws + L.tg;
        return tg_expert_stage(t, tg, tg + ts.img_gu, reinterpret_cast<float *>(tg + ts.img_gu + ts.img_dn),
                               reinterpret_cast<uint32_t *>(tg + ts.img_gu + ts.img_dn + ts.partial),
                               tg + ts.img_gu + ts.img_dn + ts.partial + ts.cnt, out_pairs,
                               [](void *, int) {}, nullptr, s);
    }
    gather_pair_rows_kernel<<<n, 128, 0, s>>>(static_cast<const __half *>(x), pairs, offsets + experts, top_k,
                                              d_model, xg);
    if ((rc = check_launch("expert gather launch"))) return rc;
    // GEMM2 writes the output of grouped pair g to slot pairs[g] = row * k + r
    return run_expert_gemms(experts, expert_slots, up_offset, down_offset, gate_type, down_type, d_model, ffn, counts,
                            offsets, n, xg, act, out_pairs, pairs, nullptr, s);
}

// workspace of experts_partial_run: everything but the per-pair outputs
uint64_t experts_pairs_workspace_bytes(uint32_t rows, uint32_t top_k, uint32_t experts, uint32_t d, uint32_t ffn) {
    return partial_layout(rows, top_k, experts, d, ffn).out;
}
} // namespace fmb

extern "C" int fmcuda_moe_experts_partial(const void *x, const int32_t *meta_expert, const float *meta_weight,
                                          uint32_t rows, uint32_t top_k, uint32_t experts,
                                          const void *const *expert_slots, uint64_t up_offset,
                                          uint64_t down_offset, uint32_t gate_type, uint32_t up_type,
                                          uint32_t down_type, uint32_t d_model, uint32_t ffn, float *partial,
                                          void *workspace, uint64_t workspace_bytes, void *stream) {
    if (rows == 0) return FM_STATUS_OK;
    if (!partial) return set_error(FM_STATUS_INVALID_ARGUMENT, "null expert-compute pointer");
    const PartialLayout L = partial_layout(rows, top_k, experts, d_model, ffn);
    if (!workspace || workspace_bytes < L.total)
        return set_error(FM_STATUS_INVALID_ARGUMENT,
                         "expert workspace too small: need " + std::to_string(L.total) + " bytes");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    float *out = reinterpret_cast<float *>(static_cast<uint8_t *>(workspace) + L.out);
    int rc = experts_partial_run(x, meta_expert, meta_weight, rows, nullptr, top_k, experts, expert_slots, up_offset,
                                 down_offset, gate_type, up_type, down_type, d_model, ffn, out, workspace,
                                 workspace_bytes, s, nullptr);
    if (rc) return rc;
    const uint64_t m = static_cast<uint64_t>(rows) * d_model;
    ep_partial_kernel<<<static_cast<unsigned>((m + 255) / 256), 256, 0, s>>>(out, meta_expert, meta_weight, rows,
                                                                              top_k, d_model, partial);
    return check_launch("expert partial-sum launch");
}

extern "C" int fmcuda_ep_combine_rows(const float *back, const uint32_t *row_of, uint32_t tokens, uint32_t world,
                                      uint32_t d_model, float *y, void *stream) {
    if (!back || !row_of || !y) return set_error(FM_STATUS_INVALID_ARGUMENT, "null combine pointer");
    if (tokens == 0) return FM_STATUS_OK;
    const uint64_t m = static_cast<uint64_t>(tokens) * d_model;
    ep_combine_rows_kernel<<<static_cast<unsigned>((m + 255) / 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
        back, row_of, tokens, world, d_model, y);
    return check_launch("combine rows launch");
}

extern "C" uint64_t fmcuda_ep_dispatch_scratch_bytes(uint32_t tokens, uint32_t top_k, uint32_t world) {
    const uint64_t P = static_cast<uint64_t>(tokens) * top_k;
    return a256(P * 4) + group_scratch_bytes(static_cast<uint32_t>(P), world);
}

extern "C" int fmcuda_ep_dispatch(const uint32_t *ids, uint32_t tokens, uint32_t top_k, uint32_t experts_per_rank,
                                  uint32_t world, const void *x, int32_t x_dtype, uint32_t d_model,
                                  uint32_t *send_counts, uint32_t *send_offsets, uint32_t *send_pairs,
                                  uint32_t *slot_of, void *send_x, uint32_t *send_expert, void *scratch,
                                  void *stream) {
    if (!ids || !x || !send_counts || !send_offsets || !send_pairs || !slot_of || !send_x || !send_expert || !scratch)
        return set_error(FM_STATUS_INVALID_ARGUMENT, "null dispatch pointer");
    if (world == 0 || world > 1024 || experts_per_rank == 0)
        return set_error(FM_STATUS_INVALID_ARGUMENT, "dispatch needs 1..1024 ranks and >= 1 expert per rank");
    if (x_dtype != FM_X_F32 && x_dtype != FM_X_BF16)
        return set_error(FM_STATUS_INVALID_ARGUMENT, "unknown activation dtype");
    if (d_model == 0 || d_model % 2) return set_error(FM_STATUS_SHAPE_MISMATCH, "d_model must be even");
    const uint64_t P64 = static_cast<uint64_t>(tokens) * top_k;
    if (P64 > 0x7FFFFFFFull) return set_error(FM_STATUS_INVALID_ARGUMENT, "too many pairs");
    const uint32_t P = static_cast<uint32_t>(P64);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    uint32_t *dest = static_cast<uint32_t *>(scratch);
    uint32_t *gscratch = reinterpret_cast<uint32_t *>(static_cast<uint8_t *>(scratch) + a256(P64 * 4));
    if (P) {
        ep_dest_kernel<<<(P + 255) / 256, 256, 0, s>>>(ids, P, experts_per_rank, dest);
        int rc = check_launch("dispatch destination launch");
        if (rc) return rc;
    }
    int rc = launch_group_large(dest, P, world, send_counts, send_offsets, send_pairs, slot_of, gscratch, s);
    if (rc || !P) return rc;
    if (x_dtype == FM_X_F32)
        ep_pack_kernel<float><<<P, 128, 0, s>>>(static_cast<const float *>(x), ids, send_pairs, send_offsets + world,
                                                top_k, experts_per_rank, d_model, static_cast<__half *>(send_x),
                                                send_expert);
    else
        ep_pack_kernel<__nv_bfloat16><<<P, 128, 0, s>>>(static_cast<const __nv_bfloat16 *>(x), ids, send_pairs,
                                                        send_offsets + world, top_k, experts_per_rank, d_model,
                                                        static_cast<__half *>(send_x), send_expert);
    return check_launch("dispatch pack launch");
}

extern "C" uint64_t fmcuda_moe_experts_workspace_bytes(uint32_t rows, uint32_t experts, uint32_t d_model,
                                                       uint32_t ffn) {
    return experts_layout(rows, experts, d_model, ffn).total;
}

extern "C" int fmcuda_moe_experts(const void *x, const uint32_t *expert_of_row, uint32_t rows, uint32_t experts,
                                  const void *const *expert_slots, uint64_t up_offset, uint64_t down_offset,
                                  uint32_t gate_type, uint32_t up_type, uint32_t down_type, uint32_t d_model,
                                  uint32_t ffn, float *out, void *workspace, uint64_t workspace_bytes,
                                  void *stream) {
    if (rows == 0) return FM_STATUS_OK;
    if (!x || !expert_of_row || !expert_slots || !out)
        return set_error(FM_STATUS_INVALID_ARGUMENT, "null expert-compute pointer");
    if (experts == 0 || experts > 1024) return set_error(FM_STATUS_INVALID_ARGUMENT, "1..1024 local experts");
    if (gate_type != up_type)
        return set_error(FM_STATUS_UNSUPPORTED_QUANTISATION, "fused gate/up needs one block type for both projections");
    for (uint32_t t : {gate_type, down_type})
        if (t != FM_TYPE_Q8_0 && t != FM_TYPE_Q4_K && t != FM_TYPE_Q6_K)
            return set_error(FM_STATUS_UNSUPPORTED_QUANTISATION, "the grouped GEMM takes Q8_0, Q4_K or Q6_K weights");
    const uint32_t kq = gate_type != FM_TYPE_Q8_0 || down_type != FM_TYPE_Q8_0 ? 256 : 64;
    if (reinterpret_cast<uintptr_t>(x) % 16 || d_model % 128 || ffn % 128 || d_model % kq || ffn % kq)
        return set_error(FM_STATUS_SHAPE_MISMATCH,
                         "expert rows must be 16-byte aligned fp16; d_model and ffn multiples of 128 (256 for "
                         "Q4_K / Q6_K)");
    const ExpertsLayout L = experts_layout(rows, experts, d_model, ffn);
    if (!workspace || workspace_bytes < L.total)
        return set_error(FM_STATUS_INVALID_ARGUMENT,
                         "expert workspace too small: need " + std::to_string(L.total) + " bytes");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    uint8_t *ws = static_cast<uint8_t *>(workspace);
    uint32_t *counts = reinterpret_cast<uint32_t *>(ws + L.counts);
    uint32_t *offsets = reinterpret_cast<uint32_t *>(ws + L.offsets);
    uint32_t *pairs = reinterpret_cast<uint32_t *>(ws + L.pairs);
    __half *xg = reinterpret_cast<__half *>(ws + L.xg);
    __half *act = reinterpret_cast<__half *>(ws + L.act);
    int rc = launch_group_large(expert_of_row, rows, experts, counts, offsets, pairs, nullptr,
                                reinterpret_cast<uint32_t *>(ws + L.gscratch), s);
    if (rc) return rc;
    gather_f16_rows_kernel<<<rows, 128, 0, s>>>(static_cast<const __half *>(x), pairs, offsets + experts, d_model, xg);
    if ((rc = check_launch("expert gather launch"))) return rc;
    // GEMM2 writes output row pairs[g] for grouped row g: the received order.
    return run_expert_gemms(experts, expert_slots, up_offset, down_offset, gate_type, down_type, d_model, ffn, counts,
                            offsets, rows, xg, act, out, pairs, nullptr, s);
}

extern "C" int fmcuda_moe_combine(const float *rows_out, const float *weights, const uint32_t *slot_of,
                                  uint32_t tokens, uint32_t top_k, uint32_t d_model, float *y, void *stream) {
    if (!rows_out || !weights || !slot_of || !y) return set_error(FM_STATUS_INVALID_ARGUMENT, "null combine pointer");
    if (tokens == 0) return FM_STATUS_OK;
    return launch_combine(rows_out, weights, slot_of, tokens, top_k, d_model, y, static_cast<cudaStream_t>(stream));
}
