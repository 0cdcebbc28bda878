/*
 * fm_oracle.h -- CPU restatement of FreeMoe's routed-expert MoE hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the checker that the sm_100a
 * kernels in freemoe_b200/csrc are compared against.  It is never linked into,
 * loaded by, or called from the product path; only tests/, the smoke check in
 * __graft_entry__.py and the cpu_baseline / reference legs of bench.py use it.
 *
 * Every function restates the arithmetic of a named routine of the reference
 * (StrangeFrostMax/FreeMoe, C++17) in plain C, in the same operation order, so
 * that byte/integer/index results are bit-identical and float results are
 * produced by the same sequence of IEEE operations.  Pinned against the
 * reference's own golden vectors (tests/fixtures/quant_reference.bin, copied as
 * an extract under tests/golden/) and against outputs of the reference itself
 * compiled from source (oracle/_ref, built by oracle/Makefile).
 *
 * Build with -ffp-contract=off: the reference is built for baseline x86-64
 * (no FMA), so a*b+c is two roundings there and must be two roundings here.
 */
#ifndef FM_ORACLE_H
#define FM_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes: the ordinal values of fm::ErrorCode (include/fm/common.hpp:27-57). */
enum {
    FMO_OK = 0,
    FMO_UNSUPPORTED_QUANTISATION = 3,
    FMO_SHAPE_MISMATCH = 8,
    FMO_INVALID_ARGUMENT = 26,
    FMO_INTERNAL_ERROR = 28,
};

/* GGUF tensor type ids covered by the hot path (src/gguf.cpp:58-106). */
enum { FMO_TYPE_F32 = 0, FMO_TYPE_Q8_0 = 8, FMO_TYPE_Q4_K = 12, FMO_TYPE_Q6_K = 14 };

/* {block_size, block_bytes} from the quantisation table (src/gguf.cpp:58-106). */
int fmo_block_geometry(uint32_t type_id, uint32_t *block_size, uint32_t *block_bytes);
/* Bytes of one row of `in_dim` values, or 0 when in_dim is not whole blocks. */
uint64_t fmo_row_bytes(uint32_t type_id, uint32_t in_dim);

/* binary16 -> binary32, exact including subnormals (src/quant.cpp:23-48). */
float fmo_fp16_to_f32(uint16_t h);
/* binary32 -> binary16, round to nearest even (used only by the encoders). */
uint16_t fmo_f32_to_fp16(float f);
/* bfloat16 -> binary32 (exact widening). */
float fmo_bf16_to_f32(uint16_t h);

/* One block -> block_size floats (src/quant.cpp:163-167 F32, :223-228 Q8_0,
 * :297-318 Q4_K with get_scale_min_k4 :63-71). */
int fmo_dequant_block(uint32_t type_id, const uint8_t *src, float *dst);
/* `n_elems` values (whole blocks) (src/quant.cpp:723-732). */
int fmo_dequant_region(uint32_t type_id, const uint8_t *src, float *dst, uint64_t n_elems);

/* y[o] = sum_k W[o,k] x[k], ascending k, float accumulator, mul then add
 * (gemv_scalar, src/kernels.cpp:132-140). */
void fmo_gemv_f32_scalar(const float *w, const float *x, float *y, uint32_t out_dim,
                         uint32_t in_dim);
/* The lane order of gemv_avx2_row (src/kernels.cpp:147-166): two 8-lane FMA
 * chains over k%16, lane-wise add, 4+4 fold, two horizontal adds, FMA tail. */
void fmo_gemv_f32_avx2_order(const float *w, const float *x, float *y, uint32_t out_dim,
                             uint32_t in_dim);

/* Quantised GEMV over `tokens` inputs, x[t*in_dim + k], y[t*out_dim + o].
 * Dequantises each block exactly and accumulates the row dot in double: the
 * order-neutral reference that every float path is compared against. */
int fmo_gemv_quant_f64(uint32_t type_id, const uint8_t *w, const float *x, double *y,
                       uint32_t tokens, uint32_t out_dim, uint32_t in_dim);
/* The same product in the order of row_dot_fused_scalar (src/kernels.cpp:574-590)
 * with the scalar dot_isa (:256-259): per block a sequential float dot, added
 * to the row total. */
int fmo_gemv_quant_fused_scalar(uint32_t type_id, const uint8_t *w, const float *x, float *y,
                                uint32_t tokens, uint32_t out_dim, uint32_t in_dim);

/* Router for the native adapter (linear-topk-softmax-v1):
 *   softmax  src/engine.cpp:378-393   (float max, double exp/sum, float out)
 *   top-k    src/engine.cpp:395-411   (stable, descending, ties -> lower id;
 *                                      NaN/+inf -> INTERNAL_ERROR, k>E -> INVALID_ARGUMENT)
 *   renorm   src/engine.cpp:1680-1702 (float total in top-k order, w/max(total,eps),
 *                                      then w*scale; gguf.cpp:3027-3028 sets norm=1, scale=1)
 * logits [T*E]; ids/weights [T*k]; probs [T*E] (may be NULL). */
/* Router variants (src/engine.cpp:1603-1702): gating 0 softmax, 1 sigmoid,
 * 2 sqrt-softplus, 3 softmax-weight; optional logit / selection biases [E];
 * groups > 1 enables group-limited routing. */
int fmo_route_ex(const float *logits, uint32_t tokens, uint32_t experts, uint32_t top_k, int gating,
                 const float *logit_bias, const float *selection_bias, uint32_t groups, uint32_t groups_used,
                 int normalise, int epsilon_additive, double epsilon, double scale, uint32_t *ids,
                 float *weights, float *probs_out);

int fmo_route(const float *logits, uint32_t tokens, uint32_t experts, uint32_t top_k,
              int normalise, double epsilon, double scale, uint32_t *ids, float *weights,
              float *probs);

/* Grouping of (token, rank) pairs by expert.  counts[E], offsets[E+1];
 * pairs[T*k] lists for each expert, in ascending token order, the flat pair
 * index t*k + r routed to it; slot_of[t*k + r] is the pair's position in
 * `pairs`.  Deterministic, so the device grouping must match it exactly. */
int fmo_group_by_expert(const uint32_t *ids, uint32_t tokens, uint32_t top_k, uint32_t experts,
                        uint32_t *counts, uint32_t *offsets, uint32_t *pairs,
                        uint32_t *slot_of);

/* Plain SwiGLU: float(silu((double)gate)) * up (include/fm/activation.hpp:33, :62-84). */
float fmo_swiglu(float gate, float up);

/* One routed-expert MoE block for `tokens` tokens, as engine.cpp:1711-1772
 * runs it per token: for each selected expert in top-k order, gate/up GEMV,
 * SwiGLU, down GEMV, ffn[j] += w * down[j].  GEMVs use the double-accumulated
 * reference above (rounded to float), so the result is the order-neutral
 * value of the reference's arithmetic.
 *   x [T*d] float, ids/weights [T*k] from fmo_route,
 *   expert_base[e] -> gate||up||down payload of expert e (GGUF row-major
 *   extents, each `ffn` or `d` rows), y [T*d]. */
int fmo_moe_block(const float *x, uint32_t tokens, uint32_t d, uint32_t ffn, uint32_t top_k,
                  const uint32_t *ids, const float *weights, const uint8_t *const *expert_base,
                  uint32_t gate_type, uint32_t up_type, uint32_t down_type, float *y);

/* Encoders for synthetic weights (any valid encoding is acceptable; only the
 * decode is graded).  Q8_0 follows the amax/127 rounding encoder of the
 * reference's fixture tool; Q4_K fits per-sub-block 6-bit scales and mins so
 * that the min path is exercised. */
void fmo_quantize_q8_0(const float *x, uint8_t *dst, uint64_t n_elems);
void fmo_quantize_q4_k(const float *x, uint8_t *dst, uint64_t n_elems);
/* Q6_K: one int8 scale per 16 values relative to an fp16 block scale, 6-bit
 * codes q + 32 packed as src/quant.cpp:347-372 reads them. */
void fmo_quantize_q6_k(const float *x, uint8_t *dst, uint64_t n_elems);

/* FNV-1a 64 over a byte range (include/fm/common.hpp:73-85). */
uint64_t fmo_fnv1a64(const uint8_t *data, uint64_t size);

#ifdef __cplusplus
}
#endif

#endif /* FM_ORACLE_H */
