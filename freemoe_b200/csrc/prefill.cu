// prefill.cu -- the routed-expert MoE block for batches of tokens on the
// tcgen05 grouped GEMM (grouped_gemm.cuh).
//
// Launch sequence on one stream:
//   1. router        logits -> ids, weights                   (router.cu)
//   2. grouping      ids -> counts, offsets, pairs, slot_of    (router.cu)
//   3. gather        xg[i] = fp16(x[token of pair i]), grouped order
//   4. GEMM1         per expert act = silu(xg Wg^T) * (xg Wu^T)   (fp16 out)
//   5. (no stage)    kept so the stage numbering matches fmcuda_moe_block
//   6. GEMM2         per expert part = act Wd^T                   (f32 out)
//   7. combine       y[t] = sum over r of w[t,r] * part[slot_of(t,r)] in top-k
//                    order (src/engine.cpp:1770), then + the shared expert
// The same block as the reference's per-token loop (src/engine.cpp:1711-1811),
// computed with fp16 tensor-core operands and f32 accumulation.
#include <cudaTypedefs.h>

#include <functional>
#include <mutex>
#include <string>

#include "grouped_gemm.cuh"

namespace fmb {

int launch_route_cfg(const float *logits, uint32_t tokens, uint32_t experts, uint32_t top_k,
                     const fmcuda_router_config *cfg, int32_t normalise, double epsilon, double scale,
                     uint32_t *ids, float *weights, float *probs, cudaStream_t s);
int launch_group(const uint32_t *ids, uint32_t n_pairs, uint32_t experts, uint32_t *counts,
                 uint32_t *offsets, uint32_t *pairs, uint32_t *slot_of, cudaStream_t s);
int check_route_args(uint32_t experts, uint32_t top_k);
uint64_t group_scratch_bytes(uint32_t n_pairs, uint32_t experts);
int launch_group_large(const uint32_t *ids, uint32_t n_pairs, uint32_t experts, uint32_t *counts,
                       uint32_t *offsets, uint32_t *pairs, uint32_t *slot_of, uint32_t *scratch,
                       cudaStream_t s);
int launch_combine(const float *part, const float *weights, const uint32_t *slot_of, uint32_t tokens,
                   uint32_t top_k, uint32_t d, float *y, cudaStream_t s);

namespace {

inline uint64_t a256(uint64_t v) { return (v + 255) & ~uint64_t(255); }

struct PrefillLayout {
    uint64_t ids, weights, counts, offsets, pairs, slot_of, gscratch;
    uint64_t xg, act, part;
    uint64_t sh_counts, sh_offsets, sh_slot, sh_act, sh_part;
    uint64_t total;
};

PrefillLayout prefill_layout(uint32_t tokens, uint32_t experts, uint32_t top_k, uint32_t d, uint32_t ffn,
                             uint32_t shared_ffn) {
    PrefillLayout L{};
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
    L.gscratch = take(group_scratch_bytes(static_cast<uint32_t>(P), experts));
    // rows [0, P) grouped pairs; rows [P, P + tokens) the tokens in order (shared expert)
    L.xg = take((P + (shared_ffn ? tokens : 0)) * d * 2);
    L.act = take(P * ffn * 2);
    L.part = take(P * d * 4);
    if (shared_ffn) {
        L.sh_counts = take(4);
        L.sh_offsets = take(8);
        L.sh_slot = take(8);
        L.sh_act = take(static_cast<uint64_t>(tokens) * shared_ffn * 2);
        L.sh_part = take(static_cast<uint64_t>(tokens) * d * 4);
    }
    L.total = o;
    return L;
}

// xg[i, :] = fp16(x[pairs[i] / top_k, :]) for i < P; xg[P + t, :] = fp16(x[t, :])
// when the shared expert needs the tokens in order.
template <typename XT>
__global__ void gather_rows_kernel(const XT *__restrict__ x, const uint32_t *__restrict__ pairs, uint32_t top_k,
                                   uint32_t n_pairs, uint32_t n_rows, uint32_t d, __half *__restrict__ xg) {
    const uint32_t i = blockIdx.x;
    if (i >= n_rows) return;
    const uint32_t tok = i < n_pairs ? pairs[i] / top_k : i - n_pairs;
    const XT *src = x + static_cast<uint64_t>(tok) * d;
    __half *dst = xg + static_cast<uint64_t>(i) * d;
    for (uint32_t c = threadIdx.x * 2; c < d; c += blockDim.x * 2) {
        const __half2 h = __floats2half2_rn(load_x(src + c), load_x(src + c + 1));
        *reinterpret_cast<__half2 *>(dst + c) = h;
    }
}

// The same gather, 8 values per thread step (16-byte fp16 stores); x rows
// 16-byte aligned.
template <typename XT>
__global__ void gather_rows8_kernel(const XT *__restrict__ x, const uint32_t *__restrict__ pairs, uint32_t top_k,
                                    uint32_t n_pairs, uint32_t n_rows, uint32_t d, __half *__restrict__ xg) {
    const uint32_t i = blockIdx.x;
    if (i >= n_rows) return;
    const uint32_t tok = i < n_pairs ? pairs[i] / top_k : i - n_pairs;
    const XT *src = x + static_cast<uint64_t>(tok) * d;
    uint4 *dst = reinterpret_cast<uint4 *>(xg + static_cast<uint64_t>(i) * d);
    for (uint32_t c = threadIdx.x; c < d / 8; c += blockDim.x) {
        float v[8];
        if constexpr (sizeof(XT) == 2) {
            const uint4 raw = __ldg(reinterpret_cast<const uint4 *>(src) + c);
            const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                v[2 * q] = bf16_bits_to_f32(static_cast<uint16_t>(w[q] & 0xFFFFu));
                v[2 * q + 1] = bf16_bits_to_f32(static_cast<uint16_t>(w[q] >> 16));
            }
        } else {
            const float4 a = __ldg(reinterpret_cast<const float4 *>(src) + 2 * c);
            const float4 b = __ldg(reinterpret_cast<const float4 *>(src) + 2 * c + 1);
            v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
            v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
        }
        uint4 o;
        o.x = pack_half2(v[0], v[1]);
        o.y = pack_half2(v[2], v[3]);
        o.z = pack_half2(v[4], v[5]);
        o.w = pack_half2(v[6], v[7]);
        dst[c] = o;
    }
}

// One-expert group for the shared expert: all tokens, in order.
__global__ void shared_group_kernel(uint32_t *counts, uint32_t *offsets, const void **slot_tab, const void *slot,
                                    uint32_t tokens) {
    counts[0] = tokens;
    offsets[0] = 0;
    offsets[1] = tokens;
    slot_tab[0] = slot;
}

// y[t, j] += s[t] * sh[t, j] (s = 1 when absent), after the routed combine --
// the order of src/engine.cpp:1808-1809.
__global__ void add_shared_kernel(float *__restrict__ y, const float *__restrict__ sh,
                                  const float *__restrict__ scalar, uint32_t tokens, uint32_t d) {
    const uint64_t id = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x;
    if (id >= static_cast<uint64_t>(tokens) * d) return;
    const float s = scalar ? scalar[id / d] : 1.0f;
    y[id] = __fadd_rn(y[id], __fmul_rn(s, sh[id]));
}

// ---- TMA descriptors ---------------------------------------------------------

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
    static std::once_flag once;
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    std::call_once(once, [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
        else
            (void)cudaGetLastError();
    });
    return fn;
}

// fp16 matrix [rows][cols], row-major, as 64-value x box_rows boxes with 128-byte swizzle.
int make_b_map(CUtensorMap *map, const __half *base, uint32_t rows, uint32_t cols, uint32_t box_rows) {
    auto enc = tensor_map_encoder();
    if (!enc) return set_error(FM_STATUS_INTERNAL_ERROR, "cuTensorMapEncodeTiled is unavailable");
    const cuuint64_t dims[2] = {cols, rows};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(cols) * 2};
    const cuuint32_t box[2] = {GG_BK, box_rows};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<__half *>(base), dims, strides, box,
                           estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS)
        return set_error(FM_STATUS_INTERNAL_ERROR, "cuTensorMapEncodeTiled failed (" + std::to_string(r) + ")");
    return FM_STATUS_OK;
}

// ---- grouped GEMM launch ------------------------------------------------------

int sm_count() {
    static int n = 0;
    if (!n) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        if (n <= 0) n = 148;
    }
    return n;
}

template <int TYPE, int NMAT, int EPI, int G>
int launch_gg_inst(const GGemmParams &p, const CUtensorMap &map, uint32_t max_units, cudaStream_t s) {
    auto kfn = grouped_gemm_kernel<TYPE, NMAT, EPI, G>;
    const uint32_t smem = GGLayout<TYPE, NMAT>::smem_bytes(p.experts);
    cudaError_t err = cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (err != cudaSuccess) {
        (void)cudaGetLastError();
        return cuda_status(err, "grouped GEMM shared-memory attribute");
    }
    const uint32_t grid = max_units < static_cast<uint32_t>(sm_count()) ? max_units : static_cast<uint32_t>(sm_count());
    if (grid == 0) return FM_STATUS_OK;
    kfn<<<grid, GG_THREADS, smem, s>>>(map, p);
    return check_launch("grouped GEMM launch");
}

// Widest async-copy size that every row start and chunk start is aligned to.
int copy_granule(uint32_t type_id, uint64_t row_bytes, uint64_t off0, uint64_t off1) {
    // Q6_K blocks are copied as 16-byte aligned windows: only the matrix starts matter
    if (type_id == FM_TYPE_Q6_K) return (off0 % 16 == 0 && off1 % 16 == 0) ? 16 : 0;
    const uint64_t chunk = type_id == FM_TYPE_Q8_0 ? 272 : 144;
    const uint64_t tail = row_bytes % chunk;
    for (int g = 16; g >= 4; g /= 2)
        if (row_bytes % g == 0 && chunk % g == 0 && tail % g == 0 && off0 % g == 0 && off1 % g == 0) return g;
    return 0;
}

template <int NMAT, int EPI>
int launch_gg(uint32_t type_id, const GGemmParams &p, const CUtensorMap &map, uint32_t max_units, int g,
              cudaStream_t s) {
    if (type_id == FM_TYPE_Q4_K) {
        if (g != 16) return set_error(FM_STATUS_INVALID_ARGUMENT, "Q4_K rows must be 16-byte aligned");
        return launch_gg_inst<FM_TYPE_Q4_K, NMAT, EPI, 16>(p, map, max_units, s);
    }
    if (type_id == FM_TYPE_Q6_K) {
        if (g != 16) return set_error(FM_STATUS_INVALID_ARGUMENT, "Q6_K matrices must start 16-byte aligned");
        return launch_gg_inst<FM_TYPE_Q6_K, NMAT, EPI, 16>(p, map, max_units, s);
    }
    switch (g) {
    case 16: return launch_gg_inst<FM_TYPE_Q8_0, NMAT, EPI, 16>(p, map, max_units, s);
    case 8: return launch_gg_inst<FM_TYPE_Q8_0, NMAT, EPI, 8>(p, map, max_units, s);
    case 4: return launch_gg_inst<FM_TYPE_Q8_0, NMAT, EPI, 4>(p, map, max_units, s);
    default: return set_error(FM_STATUS_INVALID_ARGUMENT, "Q8_0 rows must be 4-byte aligned");
    }
}

int check_prefill_shape(uint32_t type_id, uint32_t in_dim, uint32_t out_dim, const char *what) {
    if (type_id != FM_TYPE_Q8_0 && type_id != FM_TYPE_Q4_K && type_id != FM_TYPE_Q6_K)
        return set_error(FM_STATUS_UNSUPPORTED_QUANTISATION,
                         std::string(what) + ": the grouped GEMM takes Q8_0, Q4_K or Q6_K weights");
    const uint32_t kq = type_id == FM_TYPE_Q8_0 ? 64 : 256;
    if (in_dim == 0 || in_dim % kq || out_dim == 0 || out_dim % GG_BM)
        return set_error(FM_STATUS_SHAPE_MISMATCH,
                         std::string(what) + ": the grouped GEMM needs K a multiple of " + std::to_string(kq) +
                             " and output rows a multiple of 128 (got " + std::to_string(out_dim) + " x " +
                             std::to_string(in_dim) + ")");
    return FM_STATUS_OK;
}

} // namespace

// Gate/up + SwiGLU then down for one set of experts whose token rows are
// grouped in xg (rows = pairs); act and part use the same row numbering.
int run_expert_gemms(uint32_t experts, const void *const *slots, uint64_t up_offset, uint64_t down_offset,
                     uint32_t gu_type, uint32_t dn_type, uint32_t d, uint32_t ffn, const uint32_t *counts,
                     const uint32_t *offsets, uint32_t rows, const __half *xg, __half *act, float *part,
                     const uint32_t *part_rows, const std::function<void(int)> *mark, cudaStream_t s) {
    int rc;
    const uint64_t gu_rb = row_bytes(gu_type, d), dn_rb = row_bytes(dn_type, ffn);
    const int g1 = copy_granule(gu_type, gu_rb, 0, up_offset);
    const int g2 = copy_granule(dn_type, dn_rb, down_offset, down_offset);
    const uint32_t tiles_max1 = rows / GG_BN + experts, tiles_max2 = rows / GG_BN1 + experts;

    CUtensorMap map1, map2;
    if ((rc = make_b_map(&map1, xg, rows, d, GG_BN))) return rc;
    if ((rc = make_b_map(&map2, act, rows, ffn, GG_BN1))) return rc;
    GGemmParams p1{};
    p1.slots = reinterpret_cast<const uint8_t *const *>(slots);
    p1.w_off0 = 0;
    p1.w_off1 = up_offset;
    p1.out_dim = ffn;
    p1.in_dim = d;
    p1.row_bytes = static_cast<uint32_t>(gu_rb);
    p1.experts = experts;
    p1.counts = counts;
    p1.offsets = offsets;
    p1.out = act;
    p1.status = device_status_word();
    if ((rc = launch_gg<2, GG_EPI_SWIGLU>(gu_type, p1, map1, tiles_max1 * (ffn / GG_BM), g1, s))) return rc;
    if (mark) {
        (*mark)(4);
        (*mark)(5);
    }

    GGemmParams p2 = p1;
    p2.w_off0 = down_offset;
    p2.w_off1 = down_offset;
    p2.out_dim = d;
    p2.in_dim = ffn;
    p2.row_bytes = static_cast<uint32_t>(dn_rb);
    p2.out = part;
    p2.out_rows = part_rows;
    return launch_gg<1, GG_EPI_F32>(dn_type, p2, map2, tiles_max2 * (d / GG_BM), g2, s);
}

int moe_prefill_run(const fmcuda_moe_args *a, const fmcuda_shared_expert *sh, void *workspace,
                    uint64_t workspace_bytes, cudaStream_t s) {
    if (!a) return set_error(FM_STATUS_INVALID_ARGUMENT, "null MoE arguments");
    if (a->tokens == 0) return FM_STATUS_OK;
    int rc = check_route_args(a->experts, a->top_k);
    if (rc) return rc;
    if (a->experts > GG_MAX_EXPERTS)
        return set_error(FM_STATUS_INVALID_ARGUMENT, "the grouped GEMM takes at most 1024 experts");
    if (!a->x || !a->logits || !a->expert_slots || !a->y)
        return set_error(FM_STATUS_INVALID_ARGUMENT, "null MoE pointer");
    if (a->x_dtype != FM_X_F32 && a->x_dtype != FM_X_BF16)
        return set_error(FM_STATUS_INVALID_ARGUMENT, "unknown activation dtype");
    if (a->gate_type != a->up_type)
        return set_error(FM_STATUS_UNSUPPORTED_QUANTISATION, "fused gate/up needs one block type for both projections");
    if ((rc = check_prefill_shape(a->gate_type, a->d_model, a->ffn, "expert gate/up"))) return rc;
    if ((rc = check_prefill_shape(a->down_type, a->ffn, a->d_model, "expert down"))) return rc;
    const uint32_t sh_ffn = sh ? sh->ffn : 0;
    if (sh) {
        if (!sh->slot) return set_error(FM_STATUS_INVALID_ARGUMENT, "null shared-expert slot");
        if (sh->gate_type != sh->up_type)
            return set_error(FM_STATUS_UNSUPPORTED_QUANTISATION, "shared expert: one block type for gate and up");
        if ((rc = check_prefill_shape(sh->gate_type, a->d_model, sh->ffn, "shared gate/up"))) return rc;
        if ((rc = check_prefill_shape(sh->down_type, sh->ffn, a->d_model, "shared down"))) return rc;
    }
    const uint64_t P64 = static_cast<uint64_t>(a->tokens) * a->top_k;
    if (P64 + a->tokens > 0x7FFFFFFFull)
        return set_error(FM_STATUS_INVALID_ARGUMENT, "too many token-expert pairs for one call");
    const PrefillLayout L = prefill_layout(a->tokens, a->experts, a->top_k, a->d_model, a->ffn, sh_ffn);
    if (!workspace || workspace_bytes < L.total)
        return set_error(FM_STATUS_INVALID_ARGUMENT,
                         "prefill workspace too small: need " + std::to_string(L.total) + " bytes");
    uint8_t *ws = static_cast<uint8_t *>(workspace);
    uint32_t *ids = reinterpret_cast<uint32_t *>(ws + L.ids);
    float *weights = reinterpret_cast<float *>(ws + L.weights);
    uint32_t *counts = reinterpret_cast<uint32_t *>(ws + L.counts);
    uint32_t *offsets = reinterpret_cast<uint32_t *>(ws + L.offsets);
    uint32_t *pairs = reinterpret_cast<uint32_t *>(ws + L.pairs);
    uint32_t *slot_of = reinterpret_cast<uint32_t *>(ws + L.slot_of);
    __half *xg = reinterpret_cast<__half *>(ws + L.xg);
    __half *act = reinterpret_cast<__half *>(ws + L.act);
    float *part = reinterpret_cast<float *>(ws + L.part);
    const uint32_t P = static_cast<uint32_t>(P64);
    int mark_rc = FM_STATUS_OK;
    const std::function<void(int)> mark = [&](int i) {
        if (a->stage_events && a->stage_events[i] && mark_rc == FM_STATUS_OK) {
            const cudaError_t err = cudaEventRecord(static_cast<cudaEvent_t>(a->stage_events[i]), s);
            if (err != cudaSuccess) mark_rc = cuda_status(err, "stage event record");
        }
    };

    mark(0);
    if ((rc = launch_route_cfg(a->logits, a->tokens, a->experts, a->top_k, a->router, a->normalise, a->epsilon, a->scale, ids,
                           weights, nullptr, s)))
        return rc;
    mark(1);
    if ((rc = launch_group_large(ids, P, a->experts, counts, offsets, pairs, slot_of,
                                 reinterpret_cast<uint32_t *>(ws + L.gscratch), s)))
        return rc;
    mark(2);
    const uint32_t n_rows = P + (sh ? a->tokens : 0);
    const bool x16 = reinterpret_cast<uintptr_t>(a->x) % 16 == 0; // rows then aligned too (d % 128 == 0)
    if (a->x_dtype == FM_X_F32) {
        if (x16)
            gather_rows8_kernel<float><<<n_rows, 128, 0, s>>>(static_cast<const float *>(a->x), pairs, a->top_k, P,
                                                               n_rows, a->d_model, xg);
        else
            gather_rows_kernel<float><<<n_rows, 128, 0, s>>>(static_cast<const float *>(a->x), pairs, a->top_k, P,
                                                              n_rows, a->d_model, xg);
    } else {
        if (x16)
            gather_rows8_kernel<__nv_bfloat16><<<n_rows, 128, 0, s>>>(static_cast<const __nv_bfloat16 *>(a->x),
                                                                       pairs, a->top_k, P, n_rows, a->d_model, xg);
        else
            gather_rows_kernel<__nv_bfloat16><<<n_rows, 128, 0, s>>>(static_cast<const __nv_bfloat16 *>(a->x),
                                                                      pairs, a->top_k, P, n_rows, a->d_model, xg);
    }
    if ((rc = check_launch("gather launch"))) return rc;
    mark(3);
    if ((rc = run_expert_gemms(a->experts, a->expert_slots, a->up_offset, a->down_offset, a->gate_type,
                               a->down_type, a->d_model, a->ffn, counts, offsets, P, xg, act, part, nullptr, &mark, s)))
        return rc;
    mark(6);
    if ((rc = launch_combine(part, weights, slot_of, a->tokens, a->top_k, a->d_model, a->y, s))) return rc;
    if (sh) {
        uint32_t *sc = reinterpret_cast<uint32_t *>(ws + L.sh_counts);
        uint32_t *so = reinterpret_cast<uint32_t *>(ws + L.sh_offsets);
        const void **stab = reinterpret_cast<const void **>(ws + L.sh_slot);
        __half *sact = reinterpret_cast<__half *>(ws + L.sh_act);
        float *spart = reinterpret_cast<float *>(ws + L.sh_part);
        shared_group_kernel<<<1, 1, 0, s>>>(sc, so, stab, sh->slot, a->tokens);
        if ((rc = check_launch("shared expert group"))) return rc;
        if ((rc = run_expert_gemms(1, stab, sh->up_offset, sh->down_offset, sh->gate_type, sh->down_type,
                                   a->d_model, sh->ffn, sc, so, a->tokens,
                                   xg + static_cast<uint64_t>(P) * a->d_model, sact, spart, nullptr, nullptr, s)))
            return rc;
        const uint64_t n = static_cast<uint64_t>(a->tokens) * a->d_model;
        add_shared_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0, s>>>(a->y, spart, sh->gate_scalar,
                                                                                 a->tokens, a->d_model);
        if ((rc = check_launch("shared expert add"))) return rc;
    }
    mark(7);
    if (a->ids_out)
        cudaMemcpyAsync(a->ids_out, ids, static_cast<uint64_t>(P) * 4, cudaMemcpyDeviceToDevice, s);
    if (a->weights_out)
        cudaMemcpyAsync(a->weights_out, weights, static_cast<uint64_t>(P) * 4, cudaMemcpyDeviceToDevice, s);
    if (mark_rc) return mark_rc;
    return check_launch("prefill output copies");
}

} // namespace fmb

using namespace fmb;

extern "C" int fmcuda_moe_prefill_workspace_bytes(uint32_t tokens, uint32_t experts, uint32_t top_k,
                                                  uint32_t d_model, uint32_t ffn, uint32_t shared_ffn,
                                                  uint64_t *bytes) {
    if (!bytes) return set_error(FM_STATUS_INVALID_ARGUMENT, "null size pointer");
    *bytes = prefill_layout(tokens, experts, top_k, d_model, ffn, shared_ffn).total;
    return FM_STATUS_OK;
}

extern "C" int fmcuda_moe_prefill(const fmcuda_moe_args *args, const fmcuda_shared_expert *shared,
                                  void *workspace, uint64_t workspace_bytes, void *stream) {
    return moe_prefill_run(args, shared, workspace, workspace_bytes, static_cast<cudaStream_t>(stream));
}
