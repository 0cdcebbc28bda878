// tgemv.cu -- host side of the tcgen05 decode GEMVs (tgemv.cuh): workspace
// sections, eligibility and the launch sequence of the MoE block's expert
// stage for Q4_K experts and bf16 activations.
#include <cudaTypedefs.h>

#include <mutex>
#include <string>

#include "tgemv.cuh"
#include "tgemv_host.h"

namespace fmb {

namespace {

inline uint64_t a256(uint64_t v) { return (v + 255) & ~uint64_t(255); }

int tg_sm_count() {
    static int n = 0;
    if (!n) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        if (n <= 0) n = 148;
    }
    return n;
}

template <int MODE, bool WIDE> int tg_configure() {
    static int done = 0;
    if (!done) {
        const cudaError_t err = cudaFuncSetAttribute(tgemv_kernel<MODE, WIDE>,
                                                     cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                     TgLayout<MODE>::smem_bytes(TG_MAX_EXPERTS));
        if (err != cudaSuccess) return cuda_status(err, "tgemv shared-memory attribute");
        done = 1;
    }
    return FM_STATUS_OK;
}

PFN_cuTensorMapEncodeTiled_v12000 tg_encoder() {
    static std::once_flag once;
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    std::call_once(once, [] {
        void *ptr = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
        else
            (void)cudaGetLastError();
    });
    return fn;
}

// Template map of one Q4_K matrix [rows][row_bytes] (uint8), 144-byte x 128-row
// boxes, no swizzle; the device writes a copy per expert with its own address.
int tg_template(CUtensorMap *map, const void *any_base, uint32_t row_bytes, uint32_t rows) {
    auto enc = tg_encoder();
    if (!enc) return set_error(FM_STATUS_INTERNAL_ERROR, "cuTensorMapEncodeTiled is unavailable");
    const cuuint64_t dims[2] = {row_bytes, rows};
    const cuuint64_t strides[1] = {row_bytes};
    const cuuint32_t box[2] = {TG_RB, TG_ROWS};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void *>(any_base), dims, strides, box,
                           estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS)
        return set_error(FM_STATUS_INTERNAL_ERROR, "cuTensorMapEncodeTiled failed (" + std::to_string(r) + ")");
    return FM_STATUS_OK;
}

} // namespace

// Upper bound of token tiles: every expert's last tile may be partial.
uint32_t tg_max_tiles(uint32_t pairs_max, uint32_t experts) {
    return pairs_max / TG_NT + (pairs_max < experts ? pairs_max : experts);
}

// Wide mode (one weight conversion for two token tiles) pays when the experts
// hold two or more tiles on average: at least 16 routed pairs per expert.
bool tg_wide(uint32_t pairs_max, uint32_t experts) { return pairs_max >= 16ull * experts; }

bool tg_shape(uint32_t d, uint32_t ffn) { return d % 256 == 0 && ffn % 256 == 0 && d > 0 && ffn > 0; }

TgSections tg_sections(uint32_t pairs_max, uint32_t experts, uint32_t d, uint32_t ffn) {
    TgSections t{};
    if (!tg_shape(d, ffn)) return t;
    const uint64_t tiles = tg_max_tiles(pairs_max, experts);
    t.img_gu = a256(tiles * (d / 256) * TG_IMG);
    t.img_dn = a256(tiles * (ffn / 256) * TG_IMG);
    t.partial = a256(2ull * TG_MAX_CTAS * 2 * 2 * TG_NT * TG_ROWS * 4);
    // stream-K arrivals per unit (wide mode: per unit and half, 2 x pairs <= tiles + experts)
    t.cnt = a256((tiles + experts) * (ffn / TG_ROWS + d / TG_ROWS) * 4);
    t.maps = a256(static_cast<uint64_t>(experts) * 3 * sizeof(CUtensorMap) + 256);
    return t;
}

bool tg_eligible(const fmcuda_moe_args *a) {
    return a->gate_type == FM_TYPE_Q4_K && a->up_type == FM_TYPE_Q4_K && a->down_type == FM_TYPE_Q4_K &&
           a->x_dtype == FM_X_BF16 && tg_shape(a->d_model, a->ffn) && a->experts <= TG_MAX_EXPERTS &&
           a->up_offset % 16 == 0 && a->down_offset % 16 == 0;
}

namespace {

// Stream-K counters and the raw-weight map templates of one expert stage.
int tg_map_args(const TgStage &t, uint32_t *cnt, uint8_t *maps_area, TgMapArgs &ma) {
    int rc;
    if ((rc = tg_configure<TG_GATE_UP, false>())) return rc;
    if ((rc = tg_configure<TG_DOWN, false>())) return rc;
    if ((rc = tg_configure<TG_GATE_UP, true>())) return rc;
    if ((rc = tg_configure<TG_DOWN, true>())) return rc;
    const uint32_t tiles = tg_max_tiles(t.pairs_max, t.experts);
    ma = TgMapArgs{};
    ma.maps = reinterpret_cast<CUtensorMap *>(maps_area + 256);
    ma.slots = reinterpret_cast<const uint8_t *const *>(t.slots);
    ma.up_off = t.up_offset;
    ma.down_off = t.down_offset;
    ma.cnt = cnt;
    ma.n_cnt = (tiles + t.experts) * (t.ffn / TG_ROWS + t.d / TG_ROWS);
    const uint32_t rb_gu = static_cast<uint32_t>(row_bytes(FM_TYPE_Q4_K, t.d));
    const uint32_t rb_dn = static_cast<uint32_t>(row_bytes(FM_TYPE_Q4_K, t.ffn));
    if ((rc = tg_template(&ma.tmpl_gu, ma.maps, rb_gu, t.ffn))) return rc;
    return tg_template(&ma.tmpl_dn, ma.maps, rb_dn, t.d);
}

// gate/up + SwiGLU (writing the down images), then down.
int tg_gemvs(const TgStage &t, const TgMapArgs &ma, uint8_t *img_gu, uint8_t *img_dn, float *partial, uint32_t *cnt,
             float *part, void (*mark)(void *, int), void *mark_ctx, cudaStream_t s) {
    const uint32_t tiles = tg_max_tiles(t.pairs_max, t.experts);
    const uint32_t grid = static_cast<uint32_t>(tg_sm_count() < static_cast<int>(TG_MAX_CTAS) ? tg_sm_count()
                                                                                              : TG_MAX_CTAS);
    const bool wide = tg_wide(t.pairs_max, t.experts);
    TgParams gu{};
    gu.slots = ma.slots;
    gu.w_off0 = 0;
    gu.w_off1 = t.up_offset;
    gu.maps = ma.maps;
    gu.map0 = 0;
    gu.out_dim = t.ffn;
    gu.in_dim = t.d;
    gu.experts = t.experts;
    gu.counts = t.counts;
    gu.offsets = t.offsets;
    gu.img = img_gu;
    gu.out_img = img_dn;
    gu.partial = partial;
    gu.unit_cnt = cnt;
    gu.status = device_status_word();
    int rc;
    if (wide)
        tgemv_kernel<TG_GATE_UP, true><<<grid, TG_THREADS, TgLayout<TG_GATE_UP>::smem_bytes(t.experts), s>>>(gu);
    else
        tgemv_kernel<TG_GATE_UP, false><<<grid, TG_THREADS, TgLayout<TG_GATE_UP>::smem_bytes(t.experts), s>>>(gu);
    if ((rc = check_launch("tgemv gate/up"))) return rc;
    mark(mark_ctx, 4);
    mark(mark_ctx, 5);

    TgParams dn = gu;
    dn.w_off0 = t.down_offset;
    dn.w_off1 = t.down_offset;
    dn.map0 = 2;
    dn.out_dim = t.d;
    dn.in_dim = t.ffn;
    dn.img = img_dn;
    dn.out_img = nullptr;
    dn.part = part;
    dn.out_rows = t.out_rows;
    dn.unit_cnt = cnt + (tiles + t.experts) * (t.ffn / TG_ROWS);
    if (wide)
        tgemv_kernel<TG_DOWN, true><<<grid, TG_THREADS, TgLayout<TG_DOWN>::smem_bytes(t.experts), s>>>(dn);
    else
        tgemv_kernel<TG_DOWN, false><<<grid, TG_THREADS, TgLayout<TG_DOWN>::smem_bytes(t.experts), s>>>(dn);
    if ((rc = check_launch("tgemv down"))) return rc;
    mark(mark_ctx, 6);
    return FM_STATUS_OK;
}

} // namespace

// Steps after routing and grouping: x images, gate/up + SwiGLU (writing the
// down images), down.
int tg_expert_stage(const TgStage &t, uint8_t *img_gu, uint8_t *img_dn, float *partial, uint32_t *cnt,
                    uint8_t *maps_area, float *part, void (*mark)(void *, int), void *mark_ctx, cudaStream_t s) {
    TgMapArgs ma;
    int rc = tg_map_args(t, cnt, maps_area, ma);
    if (rc) return rc;
    const uint32_t tiles = tg_max_tiles(t.pairs_max, t.experts);
    if (t.x_f16)
        tg_ximage_kernel<__half><<<tiles * (t.d / 256), 256, 0, s>>>(
            ma, static_cast<const __half *>(t.x), t.d, t.counts, t.offsets, t.pairs, t.top_k, t.experts, tiles,
            img_gu);
    else
        tg_ximage_kernel<__nv_bfloat16><<<tiles * (t.d / 256), 256, 0, s>>>(
            ma, static_cast<const __nv_bfloat16 *>(t.x), t.d, t.counts, t.offsets, t.pairs, t.top_k, t.experts,
            tiles, img_gu);
    if ((rc = check_launch("tgemv x images"))) return rc;
    mark(mark_ctx, 3);
    return tg_gemvs(t, ma, img_gu, img_dn, partial, cnt, part, mark, mark_ctx, s);
}

bool tg_recv_eligible(uint32_t rows, uint32_t top_k, uint32_t experts) {
    return experts <= TG_FRONT_MAX_EXPERTS && static_cast<uint64_t>(rows) * top_k <= TG_FRONT_MAX_PAIRS;
}

// The expert-parallel receive side: wait, grouping and B images in one launch
// (tg_recv_front_kernel, writing the grouping named in `t`), then the GEMVs.
int tg_recv_stage(const TgStage &t, const TgRecvWait &r, uint8_t *img_gu, uint8_t *img_dn, float *partial,
                  uint32_t *cnt, uint8_t *maps_area, float *part, cudaStream_t s) {
    if (!tg_recv_eligible(r.rows, t.top_k, t.experts) || !t.x_f16)
        return set_error(FM_STATUS_INTERNAL_ERROR, "tg_recv_stage: batch too large for the fused receive front");
    TgMapArgs ma;
    int rc = tg_map_args(t, cnt, maps_area, ma);
    if (rc) return rc;
    const uint32_t tiles = tg_max_tiles(t.pairs_max, t.experts);
    tg_recv_front_kernel<<<tiles * (t.d / 256), 256, 0, s>>>(
        ma, r.flags, r.world, r.epoch, r.ectr, r.timeout_ns, r.n_rows, r.meta_e, static_cast<const __half *>(t.x),
        r.rows, t.top_k, t.experts, t.d, tiles, const_cast<uint32_t *>(t.counts), const_cast<uint32_t *>(t.offsets),
        const_cast<uint32_t *>(t.pairs), img_gu, device_status_word());
    if ((rc = check_launch("tgemv receive front"))) return rc;
    return tg_gemvs(t, ma, img_gu, img_dn, partial, cnt, part, [](void *, int) {}, nullptr, s);
}

bool tg_front_eligible(uint32_t tokens, uint32_t experts, uint32_t top_k) {
    return tokens <= TG_FRONT_MAX_TOKENS && experts <= TG_FRONT_MAX_EXPERTS &&
           static_cast<uint64_t>(tokens) * top_k <= TG_FRONT_MAX_PAIRS;
}

// The whole block after the router logits: router, grouping and B images in one
// launch (tg_front_kernel, which writes ids / weights / slot_of and the grouping
// named in `t`), then the GEMVs.
int tg_block_stage(const TgStage &t, const TgFront &f, uint8_t *img_gu, uint8_t *img_dn, float *partial,
                   uint32_t *cnt, uint8_t *maps_area, float *part, void (*mark)(void *, int), void *mark_ctx,
                   cudaStream_t s) {
    if (!tg_front_eligible(f.tokens, t.experts, t.top_k) || t.x_f16)
        return set_error(FM_STATUS_INTERNAL_ERROR, "tg_block_stage: batch too large for the fused front");
    TgMapArgs ma;
    int rc = tg_map_args(t, cnt, maps_area, ma);
    if (rc) return rc;
    const uint32_t tiles = tg_max_tiles(t.pairs_max, t.experts);
    tg_front_kernel<__nv_bfloat16><<<tiles * (t.d / 256), 256, 0, s>>>(
        ma, f.logits, static_cast<const __nv_bfloat16 *>(t.x), f.tokens, t.experts, t.top_k, f.normalise, f.epsilon,
        f.scale, t.d, tiles, f.ids, f.weights, const_cast<uint32_t *>(t.counts), const_cast<uint32_t *>(t.offsets),
        const_cast<uint32_t *>(t.pairs), f.slot_of, img_gu, device_status_word());
    if ((rc = check_launch("tgemv front"))) return rc;
    mark(mark_ctx, 1);
    mark(mark_ctx, 2);
    mark(mark_ctx, 3);
    return tg_gemvs(t, ma, img_gu, img_dn, partial, cnt, part, mark, mark_ctx, s);
}

} // namespace fmb
