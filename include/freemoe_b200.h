/*
 * freemoe_b200.h -- C ABI of the B200 (sm_100a) backend for FreeMoe's
 * routed-expert MoE hot path.
 *
 * Plain pointers and sizes only.  Every entry point returns a status: 0 on
 * success, otherwise the ordinal of the reference's fm::ErrorCode
 * (include/fm/common.hpp:27-57) with a message readable through
 * fmcuda_last_error().  Nothing throws, traps or aborts.  Device pointers are
 * ordinary CUDA device addresses of the current device; `stream` is a
 * cudaStream_t (NULL = the legacy default stream).  Kernels are asynchronous
 * on `stream` unless documented otherwise.
 *
 * The reference interface each entry point replaces is cited as
 * path:line of the reference tree (StrangeFrostMax/FreeMoe).
 */
#ifndef FREEMOE_B200_H
#define FREEMOE_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes: fm::ErrorCode ordinals (include/fm/common.hpp:27-57) ---- */
enum {
    FM_STATUS_OK = 0,
    FM_STATUS_UNSUPPORTED_QUANTISATION = 3,
    FM_STATUS_SHAPE_MISMATCH = 8,
    FM_STATUS_SOURCE_CHANGED = 10,
    FM_STATUS_IO_ERROR = 11,
    FM_STATUS_SHORT_READ = 12,
    FM_STATUS_ALLOCATION_FAILED = 14,
    FM_STATUS_INVALID_EXPERT_ID = 16,
    FM_STATUS_EXPERT_CHECKSUM_MISMATCH = 17,
    FM_STATUS_EXPERT_EXECUTION_MISMATCH = 18,
    FM_STATUS_TRANSFER_FAILED = 21,
    FM_STATUS_FENCE_TIMEOUT = 22,
    FM_STATUS_DEVICE_LOSS = 23,
    FM_STATUS_INVALID_ARGUMENT = 26,
    FM_STATUS_INTERNAL_ERROR = 28
};

/* ---- GGUF tensor types on the path (src/gguf.cpp:58-106) ---- */
enum { FM_TYPE_F32 = 0, FM_TYPE_Q8_0 = 8, FM_TYPE_Q4_K = 12, FM_TYPE_Q6_K = 14 };
/* Q6_K (src/quant.cpp:347-372) is decoded and multiplied on the device too: it is
 * the down projection of mixed-type expert records (Q4_K gate/up + Q6_K down);
 * its GEMV is the register-fed kernel, not the streamed one. */

/* ---- activation dtypes ---- */
enum { FM_X_F32 = 0, FM_X_BF16 = 1 };

/* ---- summation order of the F32 matvec (fmcuda_matvec_f32) ---- */
enum {
    FM_ORDER_ANY = 0,    /* fastest; tolerance-level agreement */
    FM_ORDER_SCALAR = 1, /* bit-identical to gemv_scalar, src/kernels.cpp:132-140 */
    FM_ORDER_AVX2 = 2    /* bit-identical to gemv_avx2_row, src/kernels.cpp:147-166 */
};

/* Last error message of the calling thread ("" when none). */
const char *fmcuda_last_error(void);

/* ======================= runtime (Backend plumbing) ======================= */

/* Device facts for fm::DeviceInfo (include/fm/backend.hpp:22-36). */
typedef struct fmcuda_device_info {
    char name[256];
    uint64_t total_memory_bytes;
    uint64_t free_memory_bytes;
    int32_t sm_count;
    int32_t cc_major;
    int32_t cc_minor;
    int32_t driver_version;
    int32_t runtime_version;
    int32_t l2_bytes;
} fmcuda_device_info;

/* Selects `device` for the calling thread and creates the library's per-device
 * state.  Replaces the GpuBackend placeholder constructor (src/backend.cpp:528-531).
 * Fails with DEVICE_LOSS when no usable sm_100 device is present. */
int fmcuda_init(int32_t device);
/* Backend::info (include/fm/backend.hpp:151). */
int fmcuda_device_info_get(int32_t device, fmcuda_device_info *out);

/* Backend::allocate (include/fm/backend.hpp:152): HBM, 256-byte aligned,
 * zero-filled like CpuBackend::allocate (src/backend.cpp:240-256). */
int fmcuda_malloc(uint64_t bytes, void **ptr);
/* Backend::allocate for buffers that the unchanged engine also reads on the
 * host (fixed weights read by Engine::weights, src/engine.cpp:306-346; expert
 * slots read back for checksums, src/residency.cpp:703-714): managed memory
 * whose preferred location is this device's HBM, zero-filled.  Freed with
 * fmcuda_free. */
int fmcuda_malloc_managed(uint64_t bytes, void **ptr);
/* DeviceBuffer::cleanup (include/fm/backend.hpp:70-110). */
int fmcuda_free(void *ptr);
/* Pinned host staging for uploads (host side of Backend::upload). */
int fmcuda_host_alloc(uint64_t bytes, void **ptr);
int fmcuda_host_free(void *ptr);

int fmcuda_stream_create(void **stream);
int fmcuda_stream_destroy(void *stream);
int fmcuda_stream_sync(void *stream);
int fmcuda_event_create(void **event);
int fmcuda_event_destroy(void *event);
int fmcuda_event_record(void *event, void *stream);
/* Events with timing enabled, and the milliseconds between two recorded ones
 * (cudaEventElapsedTime), for live per-kernel timing. */
int fmcuda_event_create_timing(void **event);
int fmcuda_event_elapsed_ms(void *start, void *end, float *ms);

/* Backend::upload (include/fm/backend.hpp:153): enqueue a host->device copy on
 * `stream` and record `event` after it (the fence).  `src` should be pinned
 * (fmcuda_host_alloc) for the copy to be asynchronous. */
int fmcuda_upload_async(void *dst, const void *src, uint64_t bytes, void *stream, void *event);
/* Backend::fence_complete (include/fm/backend.hpp:154): *complete = 1 when
 * the event's work has finished, 0 while pending. */
int fmcuda_event_query(void *event, int32_t *complete);
/* Backend::wait_fence (include/fm/backend.hpp:155, src/backend.cpp:128-135):
 * polls the event and returns FENCE_TIMEOUT after `timeout_ms`; never an
 * unbounded wait. */
int fmcuda_event_wait(void *event, uint32_t timeout_ms);
/* Synchronous device->host copy: the slot read-back that the residency
 * manager checksums (src/residency.cpp:703-704, :713-714). */
int fmcuda_download(void *dst, const void *src, uint64_t bytes, void *stream);
int fmcuda_memset_async(void *dst, int32_t value, uint64_t bytes, void *stream);

/* Reads (and with clear != 0 resets) the device-side status word that kernels
 * set instead of trapping (non-finite router logit, unresident expert).
 * Synchronises the device first. */
int fmcuda_device_status(int32_t clear, int32_t *status);

/* ============================ hot-path kernels ============================ */

/* Row bytes of `in_dim` values of `type_id` (0 on bad geometry). */
uint64_t fmcuda_row_bytes(uint32_t type_id, uint32_t in_dim);

/* K1, dequantize_tensor_region (src/quant.cpp:723-732) over `n_elems` values
 * (whole blocks): F32, Q8_0 (:223-228), Q4_K (:297-318).  Bit-exact. */
int fmcuda_dequant(uint32_t type_id, const void *src, float *dst, uint64_t n_elems,
                   void *stream);

/* K2, gemv_quant / gemm_quant (src/kernels.cpp:846-878, :316-345):
 * y[t*out_dim + o] = sum_k W[o,k] x[t*in_dim + k] for t < tokens, with W in
 * GGUF row-major blocks of `type_id` and x in `x_dtype`.  Dequantisation is
 * fused into the contraction.  Any number of tokens; the weight rows are read
 * once per 8 tokens.  Validation and error codes as gemv_quant. */
int fmcuda_gemv(uint32_t type_id, const void *w, const void *x, int32_t x_dtype, float *y,
                uint32_t tokens, uint32_t out_dim, uint32_t in_dim, void *stream);

/* Backend::matvec (include/fm/backend.hpp:157; CpuBackend::matvec
 * src/backend.cpp:277-290): one F32 product, y = W x, in the requested
 * summation order (FM_ORDER_*). */
int fmcuda_matvec_f32(const float *w, const float *x, float *y, uint32_t out_dim,
                      uint32_t in_dim, int32_t order, void *stream);

/* K4, the native router (Engine::softmax src/engine.cpp:378-393, Engine::topk
 * :395-411, renormalisation :1680-1702), one warp per token:
 *   logits [T*E] f32 -> ids [T*k] (stable descending, ties to the lower id),
 *   weights [T*k] f32, probs [T*E] f32 (optional, may be NULL).
 * A non-finite logit sets the device status to INTERNAL_ERROR (read it with
 * fmcuda_device_status).  E <= 1024, k <= min(E, 32). */
int fmcuda_route(const float *logits, uint32_t tokens, uint32_t experts, uint32_t top_k,
                 int32_t normalise, double epsilon, double scale, uint32_t *ids, float *weights,
                 float *probs, void *stream);

/* The router's model-family variants (src/engine.cpp:1603-1702; parsed from
 * GGUF metadata at src/gguf.cpp:1445-1480, :1531-1535, :1946).  A NULL config,
 * or the default below, is the native router of fmcuda_route. */
enum {
    FM_GATING_SOFTMAX = 0,        /* Engine::softmax over all experts */
    FM_GATING_SIGMOID = 1,        /* float(1 / (1 + exp(-(double)s))) */
    FM_GATING_SQRT_SOFTPLUS = 2,  /* float(sqrt(log1p(exp((double)s)))) */
    FM_GATING_SOFTMAX_WEIGHT = 3  /* probabilities = logits; softmax over the picked k */
};
typedef struct fmcuda_router_config {
    int32_t gating;               /* FM_GATING_* (expert_gating) */
    const float *logit_bias;      /* optional device [E] (ffn_gate_inp.bias), added before gating */
    const float *selection_bias;  /* optional device [E] (ffn_exp_probs_b.bias), picks only */
    uint32_t groups;              /* expert_groups (<= 1: no group limit) */
    uint32_t groups_used;         /* expert_groups_used */
    int32_t normalise;            /* expert_weights_norm */
    int32_t epsilon_additive;     /* expert_weights_epsilon_additive: total + eps, else max(total, eps) */
    double epsilon;               /* expert_weights_epsilon */
    double scale;                 /* expert_weights_scale */
} fmcuda_router_config;

/* fmcuda_route with a router configuration: logits -> ids, weights, probs (the
 * gated probabilities, before any selection bias; optional).  NaN or +inf in the
 * selection, or a non-finite logit under softmax gating, sets INTERNAL_ERROR. */
int fmcuda_route_ex(const float *logits, uint32_t tokens, uint32_t experts, uint32_t top_k,
                    const fmcuda_router_config *config, uint32_t *ids, float *weights, float *probs,
                    void *stream);

/* Grouping of the T*k (token, rank) pairs by expert:
 *   counts [E], offsets [E+1] (exclusive scan), pairs [T*k] (for each expert,
 *   its flat pair indices t*k + r in ascending token order), slot_of [T*k]
 *   (inverse permutation; may be NULL).  Single kernel, bit-exact with the
 *   deterministic host grouping.  E <= 1024. */
int fmcuda_group(const uint32_t *ids, uint32_t tokens, uint32_t top_k, uint32_t experts,
                 uint32_t *counts, uint32_t *offsets, uint32_t *pairs, uint32_t *slot_of,
                 void *stream);

/* The same grouping computed by many warps, for large batches (prefill): the
 * same outputs as fmcuda_group, bit for bit.  `scratch` is device memory of
 * fmcuda_group_scratch_bytes() bytes. */
uint64_t fmcuda_group_scratch_bytes(uint32_t n_pairs, uint32_t experts);
int fmcuda_group_batched(const uint32_t *ids, uint32_t tokens, uint32_t top_k, uint32_t experts,
                         uint32_t *counts, uint32_t *offsets, uint32_t *pairs, uint32_t *slot_of,
                         void *scratch, void *stream);

/* One routed-expert MoE block (src/engine.cpp:1603-1772) for `tokens` tokens:
 * router (softmax, top-k, renormalisation) on the given logits, grouping by
 * expert, per expert a fused gate/up GEMV with SwiGLU
 * (include/fm/activation.hpp:62-84), the down GEMV, and the weighted combine
 * ffn[j] += w * down[j] in top-k order (src/engine.cpp:1770).
 *
 * expert_slots: device array [E] of expert payload base pointers laid out as
 * an ExpertRecord (include/fm/gguf.hpp:737-758): gate rows, then up rows at
 * `up_offset`, then down rows at `down_offset`.  A NULL entry is an expert
 * that is not resident; routing to it sets the device status to
 * EXPERT_EXECUTION_MISMATCH and leaves that expert's contribution out.
 *
 * workspace: device scratch of fmcuda_moe_workspace_bytes() bytes. */
typedef struct fmcuda_moe_args {
    const void *x;            /* [tokens * d_model], x_dtype */
    int32_t x_dtype;          /* FM_X_F32 or FM_X_BF16 */
    const float *logits;      /* [tokens * experts] router logits */
    uint32_t tokens;
    uint32_t experts;
    uint32_t top_k;
    uint32_t d_model;
    uint32_t ffn;
    const void *const *expert_slots; /* device array [experts] */
    uint64_t up_offset;       /* bytes from slot base to the up rows */
    uint64_t down_offset;     /* bytes from slot base to the down rows */
    uint32_t gate_type;
    uint32_t up_type;
    uint32_t down_type;
    int32_t normalise;        /* expert_weights_norm */
    double epsilon;           /* expert_weights_epsilon (6.103515625e-5) */
    double scale;             /* expert_weights_scale (1.0) */
    float *y;                 /* [tokens * d_model] f32 output */
    uint32_t *ids_out;        /* optional [tokens * top_k] */
    float *weights_out;       /* optional [tokens * top_k] */
    /* optional: FM_MOE_STAGES + 1 cudaEvent_t handles recorded on `stream`
     * before the first stage and after each stage (router, grouping, x
     * planes, gate/up, act planes, down, combine), for live per-kernel timing;
     * NULL disables.  Entries may be NULL. */
    void *const *stage_events;
    /* optional router variant; NULL = softmax with normalise/epsilon/scale above */
    const fmcuda_router_config *router;
} fmcuda_moe_args;

enum { FM_MOE_STAGES = 7 };

int fmcuda_moe_workspace_bytes(uint32_t tokens, uint32_t experts, uint32_t top_k,
                               uint32_t d_model, uint32_t ffn, uint64_t *bytes);
int fmcuda_moe_block(const fmcuda_moe_args *args, void *workspace, uint64_t workspace_bytes,
                     void *stream);

/* ========================= MoE prefill (grouped GEMM) ========================= */

/* A dense SwiGLU FFN run beside the routed experts for every token
 * (src/engine.cpp:1778-1811): y[t] += gate_scalar[t] * down(silu(gate x) * up x),
 * added after the routed combine.  `slot` holds gate rows, up rows at
 * `up_offset`, down rows at `down_offset` (the ffn_*_shexp tensors, one record). */
typedef struct fmcuda_shared_expert {
    const void *slot;          /* device pointer */
    uint32_t ffn;              /* shared_expert_intermediate (multiple of 128) */
    uint64_t up_offset;
    uint64_t down_offset;
    uint32_t gate_type;
    uint32_t up_type;
    uint32_t down_type;
    const float *gate_scalar;  /* optional device [tokens]: the per-token branch scalar
                                  (sigmoid of ffn_gate_inp_shexp); NULL = 1.0 (ungated) */
} fmcuda_shared_expert;

/* The routed MoE block of fmcuda_moe_block for a batch of tokens (prompt
 * prefill), on the sm_100a tensor cores: router and grouping as in
 * fmcuda_moe_block, the token rows gathered per expert, then per expert one
 * grouped GEMM for gate/up with SwiGLU and one for down (tcgen05.mma, fp16
 * operands dequantised from the stored Q8_0 / Q4_K bytes in the kernel, f32
 * accumulation), then the weighted combine in top-k order and the optional
 * shared expert.  Reference: the per-token expert loop of src/engine.cpp:1711-1811
 * applied to every prompt token.  Outputs match fmcuda_moe_block / the
 * reference within a relative tolerance (fp16 operands), not bit for bit.
 *
 * Shapes: Q8_0 or Q4_K experts (gate and up of one type), d_model and ffn
 * multiples of 128 (and of 256 for Q4_K rows), at most 1024 experts; other
 * shapes return SHAPE_MISMATCH / UNSUPPORTED_QUANTISATION.  `shared` may be
 * NULL.  stage_events: 0 start, 1 router, 2 grouping, 3 gather, 4 gate/up,
 * 5 (same as 4), 6 down, 7 combine and shared expert. */
int fmcuda_moe_prefill_workspace_bytes(uint32_t tokens, uint32_t experts, uint32_t top_k,
                                       uint32_t d_model, uint32_t ffn, uint32_t shared_ffn,
                                       uint64_t *bytes);
int fmcuda_moe_prefill(const fmcuda_moe_args *args, const fmcuda_shared_expert *shared,
                       void *workspace, uint64_t workspace_bytes, void *stream);

/* ===================== expert parallelism (device pieces) ===================== */

/* No counterpart in the reference (FreeMoe runs all experts in one process).
 * Experts are sharded contiguously over `world` ranks: expert e lives on rank
 * e / experts_per_rank as local expert e % experts_per_rank.  Each rank routes
 * its own tokens with fmcuda_route, then:
 *
 * fmcuda_ep_dispatch: groups the T*k pairs by destination rank (ascending pair
 * order inside each rank's block) and packs, in that order, the fp16 token row
 * [d_model] and the local expert id of every pair:
 *   send_counts [world], send_offsets [world+1], send_pairs [T*k] (pair index
 *   t*k + r of send row i), slot_of [T*k] (send row of pair p), send_x
 *   [T*k * d_model] fp16, send_expert [T*k].
 * `scratch`: fmcuda_ep_dispatch_scratch_bytes() bytes of device memory.
 * The caller then exchanges rows and expert ids with its collective library
 * (an all-to-all with send_counts / the peers' counts). */
uint64_t fmcuda_ep_dispatch_scratch_bytes(uint32_t tokens, uint32_t top_k, uint32_t world);
int fmcuda_ep_dispatch(const uint32_t *ids, uint32_t tokens, uint32_t top_k, uint32_t experts_per_rank,
                       uint32_t world, const void *x, int32_t x_dtype, uint32_t d_model,
                       uint32_t *send_counts, uint32_t *send_offsets, uint32_t *send_pairs,
                       uint32_t *slot_of, void *send_x, uint32_t *send_expert, void *scratch,
                       void *stream);

/* The routed experts of this rank applied to `rows` received token rows:
 * x [rows * d_model] fp16 (16-byte aligned), expert_of_row [rows] local ids;
 * out [rows * d_model] f32 = down(silu(gate x) * up x) of each row's expert,
 * in the received order.  The rows are grouped by expert and run on the
 * tcgen05 grouped GEMM, as in fmcuda_moe_prefill.  Shapes as
 * fmcuda_moe_prefill; `workspace` of fmcuda_moe_experts_workspace_bytes(). */
uint64_t fmcuda_moe_experts_workspace_bytes(uint32_t rows, uint32_t experts, uint32_t d_model,
                                            uint32_t ffn);
int fmcuda_moe_experts(const void *x, const uint32_t *expert_of_row, uint32_t rows, uint32_t experts,
                       const void *const *expert_slots, uint64_t up_offset, uint64_t down_offset,
                       uint32_t gate_type, uint32_t up_type, uint32_t down_type, uint32_t d_model,
                       uint32_t ffn, float *out, void *workspace, uint64_t workspace_bytes,
                       void *stream);

/* y[t] = sum over r < top_k of weights[t*k + r] * rows_out[slot_of[t*k + r]]
 * (multiply then add, in top-k order: src/engine.cpp:1770); rows_out are the
 * expert outputs back at the token's owner, in its send order. */
int fmcuda_moe_combine(const float *rows_out, const float *weights, const uint32_t *slot_of,
                       uint32_t tokens, uint32_t top_k, uint32_t d_model, float *y, void *stream);

/* The de-duplicated exchange: a token goes once to each rank that owns at
 * least one of its experts, and comes back as one partial sum per rank.
 *
 * fmcuda_ep_dispatch_rows: items t*world + dest (token t has a pair on rank
 * dest) grouped by destination, ascending token order inside each block:
 *   send_counts [world], send_offsets [world+1], send_items [T*world] (item of
 *   send row j), row_of [T*world] (send row of item t*world + dest, or
 *   0xFFFFFFFF), send_x [T*world * d_model] fp16, meta_expert [T*world * k]
 *   (local expert of top-k slot r of send row j, -1 when that pair goes to
 *   another rank), meta_weight [T*world * k] (its routing weight, else 0).
 * `scratch`: fmcuda_ep_dispatch_rows_scratch_bytes() bytes.
 *
 * fmcuda_moe_experts_partial: for each received row, the outputs of its
 * slots' experts combined in top-k order: partial[row] = sum over r of
 * meta_weight[row*k + r] * down(silu(gate x) * up x) of expert meta_expert[...]
 * (multiply then add, src/engine.cpp:1770).  Shapes as fmcuda_moe_prefill.
 *
 * fmcuda_ep_combine_rows: y[t] = sum over ranks (ascending) of the returned
 * partial rows back[row_of[t*world + rank]].  The sum of each token's pairs is
 * therefore grouped by rank: equal to the reference's top-k-order sum within
 * the f32 rounding of the regrouping. */
uint64_t fmcuda_ep_dispatch_rows_scratch_bytes(uint32_t tokens, uint32_t world);
int fmcuda_ep_dispatch_rows(const uint32_t *ids, const float *weights, uint32_t tokens, uint32_t top_k,
                            uint32_t experts_per_rank, uint32_t world, const void *x, int32_t x_dtype,
                            uint32_t d_model, uint32_t *send_counts, uint32_t *send_offsets,
                            uint32_t *send_items, uint32_t *row_of, void *send_x, int32_t *meta_expert,
                            float *meta_weight, void *scratch, void *stream);
uint64_t fmcuda_moe_experts_partial_workspace_bytes(uint32_t rows, uint32_t top_k, uint32_t experts,
                                                    uint32_t d_model, uint32_t ffn);
int fmcuda_moe_experts_partial(const void *x, const int32_t *meta_expert, const float *meta_weight,
                               uint32_t rows, uint32_t top_k, uint32_t experts,
                               const void *const *expert_slots, uint64_t up_offset, uint64_t down_offset,
                               uint32_t gate_type, uint32_t up_type, uint32_t down_type, uint32_t d_model,
                               uint32_t ffn, float *partial, void *workspace, uint64_t workspace_bytes,
                               void *stream);
int fmcuda_ep_combine_rows(const float *back, const uint32_t *row_of, uint32_t tokens, uint32_t world,
                           uint32_t d_model, float *y, void *stream);

/* ============ expert parallelism over NCCL, driven from C ============ *
 * No reference counterpart (FreeMoe runs every expert in one process); this is
 * the SURVEY-listed fmcuda_ep_init(nccl_uid, rank, G) boundary for hosts that
 * are not Python.  NCCL is loaded at run time (libnccl.so.2: the copy the
 * process already holds, else the system's).
 *
 * fmcuda_ep_nccl_unique_id: rank 0 creates the group's id (FM_EP_NCCL_ID_BYTES
 * bytes) and shares it with the other ranks out of band (a store, a file, MPI).
 * fmcuda_ep_init: every rank, with its device current, joins the group
 * (ncclCommInitRank; collective); fmcuda_ep_destroy leaves it.
 * fmcuda_ep_layer: one routed-expert MoE layer for this rank's `tokens` tokens,
 * experts sharded over the group (expert e on rank e / (experts / world),
 * `local_slots` = this rank's experts in order): route, one fp16 row per
 * (token, destination rank) with its slots' local experts and weights, NCCL
 * send/recv of the counts (read on the host: one stream synchronisation per
 * call), of the rows, this rank's experts (fmcuda_moe_experts_partial), the
 * f32 partial rows back, combine -- the de-duplicated ("rows") exchange of
 * freemoe_b200/ep.py, with the same result bit for bit.  Every rank calls it
 * once per layer, in the same order; `tokens_max` >= every rank's token count
 * (sizes the workspace: fmcuda_ep_layer_workspace_bytes).  NCCL failures come
 * back as TRANSFER_FAILED with NCCL's message. */
#define FM_EP_NCCL_ID_BYTES 128
typedef struct fmcuda_ep_layer_args {
    const void *x;                    /* [tokens][d_model] bf16 or f32 */
    int32_t x_dtype;                  /* FM_X_F32 or FM_X_BF16 */
    const float *logits;              /* [tokens][experts] router logits */
    uint32_t tokens, experts, top_k;  /* experts = all experts of the layer */
    uint32_t d_model, ffn;
    const void *const *local_slots;   /* device array: this rank's expert records */
    uint64_t up_offset, down_offset;  /* inside a record */
    uint32_t gate_type, up_type, down_type;
    int32_t normalise;                /* renormalise the selected weights */
    double epsilon, scale;            /* src/engine.cpp:1680-1702 */
    float *y;                         /* [tokens][d_model] f32 */
} fmcuda_ep_layer_args;
int fmcuda_ep_nccl_unique_id(void *uid);
int fmcuda_ep_init(const void *nccl_uid, uint32_t rank, uint32_t world, void **comm);
int fmcuda_ep_destroy(void *comm);
int fmcuda_ep_layer_workspace_bytes(uint32_t tokens_max, uint32_t world, uint32_t experts_local, uint32_t top_k,
                                    uint32_t d_model, uint32_t ffn, uint64_t *bytes);
int fmcuda_ep_layer(void *comm, const fmcuda_ep_layer_args *args, uint32_t tokens_max, void *workspace,
                    uint64_t workspace_bytes, void *stream);

/* ============ expert parallelism over peer memory (one node) ============ *
 * The same de-duplicated exchange with no collective library call and no host
 * read of the split sizes: each rank owns a mailbox (device memory shared with
 * the other processes of the node by CUDA IPC); the dispatch kernel writes
 * every token row straight into its destination's mailbox over NVLink, and
 * the kernel that sums a received row's expert outputs writes the partial sum
 * straight back into the source's mailbox.  Per layer call and rank:
 *   fmcuda_ep_p2p_dispatch   route already done: group this rank's tokens by
 *                            destination, publish the counts, send the rows
 *   fmcuda_ep_p2p_experts    wait for the rows, run the local experts, return
 *                            one f32 partial sum per received row
 *   fmcuda_ep_p2p_combine    wait for the partial sums, y[t] = their sum over
 *                            ranks (ascending): the result of mode "rows"
 * `epoch` numbers the calls 1, 2, ... (the same on every rank), or is 0 in
 * all three calls: then the kernels of the call take one past a counter in
 * this rank's own mailbox as their epoch and fmcuda_ep_p2p_combine advances
 * the counter when it has finished (every device-epoch call runs all three),
 * so the calls can be captured in a CUDA graph once and replayed (one layer
 * uses one of the two forms).  `capacity`
 * (the same on every rank) bounds the rows a mailbox receives: at least the
 * largest tokens-per-rank times world.  `peers` is a device array of the
 * world mailbox addresses as this process sees them (its own included);
 * `mailbox` is this rank's own.  Waits give up after `timeout_ms` (0 = 2000)
 * with FENCE_TIMEOUT in the device status word; a row that would land past a
 * mailbox's capacity is dropped with INVALID_ARGUMENT there. */
uint64_t fmcuda_ep_mailbox_bytes(uint32_t world, uint32_t capacity, uint32_t top_k, uint32_t d_model);
/* allocates (zeroed) and returns the 64-byte cudaIpcMemHandle_t in ipc_handle */
int fmcuda_ep_mailbox_alloc(uint64_t bytes, void **mailbox, void *ipc_handle);
int fmcuda_ep_mailbox_open(const void *ipc_handle, void **mailbox);
int fmcuda_ep_mailbox_close(void *mailbox);
int fmcuda_ep_mailbox_free(void *mailbox);
uint64_t fmcuda_ep_p2p_dispatch_scratch_bytes(uint32_t tokens, uint32_t world);
int fmcuda_ep_p2p_dispatch(const uint32_t *ids, const float *weights, uint32_t tokens, uint32_t top_k,
                           uint32_t experts_per_rank, uint32_t world, uint32_t rank, const void *x, int32_t x_dtype,
                           uint32_t d_model, void *mailbox, void *const *peers, uint32_t capacity, uint32_t epoch,
                           uint32_t *row_of, void *scratch, uint32_t timeout_ms, void *stream);
uint64_t fmcuda_ep_p2p_experts_workspace_bytes(uint32_t capacity, uint32_t top_k, uint32_t experts,
                                               uint32_t d_model, uint32_t ffn);
int fmcuda_ep_p2p_experts(void *mailbox, void *const *peers, uint32_t world, uint32_t rank, uint32_t capacity,
                          uint32_t epoch, uint32_t top_k, uint32_t experts, const void *const *expert_slots,
                          uint64_t up_offset, uint64_t down_offset, uint32_t gate_type, uint32_t up_type,
                          uint32_t down_type, uint32_t d_model, uint32_t ffn, void *workspace,
                          uint64_t workspace_bytes, uint32_t timeout_ms, void *stream);
int fmcuda_ep_p2p_combine(void *mailbox, uint32_t world, uint32_t rank, uint32_t capacity, uint32_t epoch,
                          uint32_t top_k, const uint32_t *row_of, uint32_t tokens, uint32_t d_model, float *y,
                          uint32_t timeout_ms, void *stream);

/* Size of the scratch built into the library for fmcuda_moe_block_noalloc. */
#define FM_MOE_NOALLOC_SCRATCH_BYTES (16u * 1024u * 1024u)

/* The same MoE block as fmcuda_moe_block, for callers that cannot allocate
 * device memory -- for example a host whose HBM is fully committed to expert
 * slots before decoding starts, or a plug-in whose host framework owns the
 * device allocator.  No counterpart in the reference: FreeMoe has no GPU path.
 *
 * It allocates and frees nothing: its scratch is a fixed array of
 * FM_MOE_NOALLOC_SCRATCH_BYTES inside the library's device image, held by
 * every GPU that loads the library until the process exits.  A block whose
 * fmcuda_moe_workspace_bytes() exceeds that size is refused with
 * INVALID_ARGUMENT.  The first call on each device (and the first after that
 * device's context was destroyed and created again) looks up the scratch's
 * device address with that device current.  With CUDA's lazy module loading
 * that lookup is also when the device maps the scratch, so it can fail with
 * ALLOCATION_FAILED once HBM is full: make the first call on each device --
 * a call with tokens = 0 does the lookup and nothing else -- before the
 * device memory is committed (to expert slots, say) and before capturing the
 * stream.  All calls share the one array and the next call overwrites it, so
 * calls that overlap on the GPU (other streams, other host threads on the
 * same device) race: keep them ordered on one stream. */
int fmcuda_moe_block_noalloc(const fmcuda_moe_args *args, void *stream);

/* ==================== cold -> warm expert loads (record_loader.cu) ==================== */

/* FNV-1a 64 of `bytes` device bytes at `data` -- the reference's expert
 * checksum fm::fnv1a64 (include/fm/common.hpp:73-81), bit for bit -- computed
 * in parallel on the device and written to the device word *out (8-byte
 * aligned) on `stream`.  `workspace` holds
 * fmcuda_fnv1a64_workspace_bytes(bytes) device bytes.  Replaces the host-side
 * fnv1a64 of a slot read-back (src/residency.cpp:700-720). */
uint64_t fmcuda_fnv1a64_workspace_bytes(uint64_t bytes);
int fmcuda_fnv1a64(const void *data, uint64_t bytes, uint64_t *out, void *workspace,
                   uint64_t workspace_bytes, void *stream);

/* fm::Extent (include/fm/io.hpp:24-27): one byte range of the model file. */
typedef struct fmcuda_extent {
    uint64_t offset;
    uint64_t size;
} fmcuda_extent;

/* fm::FileIdentity (include/fm/common.hpp:144-160): stat fields plus a sparse
 * FNV-1a content probe over the first, middle and last 64 bytes. */
typedef struct fmcuda_file_identity {
    uint64_t size;
    uint64_t dev;
    uint64_t ino;
    int64_t mtime_ns;
    int64_t ctime_ns;
    uint64_t content_probe;
} fmcuda_file_identity;
int fmcuda_file_identity_get(const char *path, fmcuda_file_identity *id);

/* coalesce_extents (src/io.cpp:46-78): extents sorted by (offset, size) merge
 * into one read when they start at most `max_gap` bytes past the group's end.
 * Writes *n_groups and, when the arrays are given, each group's
 * [offset, end) and the group of every extent.  Host only; a zero-sized or
 * overflowing extent is INVALID_ARGUMENT. */
int fmcuda_coalesce_extents(const fmcuda_extent *extents, uint32_t n, uint64_t max_gap,
                            uint64_t *group_offset, uint64_t *group_end, uint32_t *group_of,
                            uint32_t *n_groups);

/* fm::ReaderMode ordinals (include/fm/io.hpp:19): the loader reads with
 * pread (Buffered) or O_DIRECT aligned spans (Direct). */
enum { FM_READER_BUFFERED = 1, FM_READER_DIRECT = 3 };

typedef struct fmcuda_record_loader fmcuda_record_loader;

/* Opens `path` for expert loads by `reader_threads` reader threads, each with
 * a copy stream and a ring of `ring_depth` pinned chunks of `chunk_bytes`
 * (rounded up to the direct-I/O alignment); the reader mode, the coalescing
 * gap and force_direct_fallback of fm::SchedulerConfig (include/fm/io.hpp:
 * 100-107).  `expected` is the identity the manifest was built against (NULL:
 * the file as it is now); every load verifies it first and fails
 * SOURCE_CHANGED (src/io.cpp:262-278) when the file differs.  One loader
 * serves one caller thread at a time. */
int fmcuda_record_loader_create(const char *path, int reader_mode, uint64_t coalesce_gap,
                                uint64_t chunk_bytes, uint32_t ring_depth, uint32_t reader_threads,
                                int force_direct_fallback, const fmcuda_file_identity *expected,
                                fmcuda_record_loader **out);
int fmcuda_record_loader_destroy(fmcuda_record_loader *loader);

typedef struct fmcuda_record_load_stats {
    uint64_t payload_bytes;      /* bytes written to the slot (sum of the extents) */
    uint64_t physical_bytes;     /* bytes read from the file (aligned spans in Direct mode) */
    uint64_t read_requests;      /* coalesced groups read */
    uint64_t coalesced_requests; /* extents merged into another extent's read */
    uint64_t direct_fallbacks;   /* groups read buffered in Direct mode */
    uint64_t checksum;           /* FNV-1a 64 of the slot bytes after the copy */
    double elapsed_ms;           /* host wall time of the call */
} fmcuda_record_load_stats;

/* Device bytes of `workspace` for a record of `payload_bytes` (256-byte aligned). */
uint64_t fmcuda_record_load_workspace_bytes(uint64_t payload_bytes);

/* One expert record from the file into the HBM slot: the demand path of
 * ResidencyManager::load_slot (src/residency.cpp:624-724) from
 * ReadScheduler::read_record (src/io.cpp:392-400) through the upload and the
 * slot checksum.  The extents are copied to the slot in record (role) order,
 * as read_record concatenates them; the coalesced groups are cut into chunks
 * that the reader threads read straight into their pinned rings and copy to
 * the slot with cudaMemcpyAsync on their own streams, which first wait for
 * the work already queued on `stream`.  Then `stream` waits for every copy
 * and FNV-1a 64 of the slot runs on the device; stats->checksum holds it.  With checksum_known, a value other than
 * expected_checksum is EXPERT_CHECKSUM_MISMATCH -- one test covering the
 * source check and the slot check of load_slot.  Without it (vendor files
 * publish no checksum) the value is returned for the caller to keep.
 * Errors: SOURCE_CHANGED, SHORT_READ (an extent past the end of the file,
 * before any byte moves; or a short read), IO_ERROR, INVALID_ARGUMENT
 * (zero-sized extent, payload larger than `slot_bytes`, small workspace),
 * TRANSFER_FAILED / DEVICE_LOSS, FENCE_TIMEOUT (a copy not done within
 * `timeout_ms`).  The call returns once the checksum is on the host; after an
 * error, copies already issued may still be in flight on `stream`. */
int fmcuda_record_load(fmcuda_record_loader *loader, const fmcuda_extent *extents, uint32_t n_extents,
                       void *slot, uint64_t slot_bytes, int checksum_known, uint64_t expected_checksum,
                       void *workspace, uint64_t workspace_bytes, void *stream, uint32_t timeout_ms,
                       fmcuda_record_load_stats *stats);

/* ====================== synthetic weights (bench/test) ====================== */

/* Fills `dst` with `rows` rows of `cols` values of `type_id` (Q8_0 / Q4_K /
 * F32) encoding seeded Gaussian weights N(0, std^2): value i of the tensor is
 * a Box-Muller draw from a counter-based hash of (seed, i).  Any valid
 * encoding is acceptable to the path; only the decode is graded. */
int fmcuda_synth_weights(uint32_t type_id, void *dst, uint64_t rows, uint32_t cols,
                         uint64_t seed, float std, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* FREEMOE_B200_H */
