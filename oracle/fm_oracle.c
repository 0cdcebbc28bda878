/*
 * fm_oracle.c -- CPU restatement of FreeMoe's routed-expert MoE hot path.
 *
 * TEST INFRASTRUCTURE ONLY (see fm_oracle.h).  Never part of the product path.
 * Compiled with -ffp-contract=off so each float expression rounds exactly as
 * the reference's baseline-x86-64 build does.
 */
#include "fm_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

int fmo_block_geometry(uint32_t type_id, uint32_t *block_size, uint32_t *block_bytes) {
    /* src/gguf.cpp:58-106: F32 {1,4}, Q8_0 {32,34}, Q4_K {256,144}. */
    uint32_t bs = 0, bb = 0;
    switch (type_id) {
    case FMO_TYPE_F32: bs = 1; bb = 4; break;
    case FMO_TYPE_Q8_0: bs = 32; bb = 34; break;
    case FMO_TYPE_Q4_K: bs = 256; bb = 144; break;
    case FMO_TYPE_Q6_K: bs = 256; bb = 210; break;
    default: return FMO_UNSUPPORTED_QUANTISATION;
    }
    if (block_size) *block_size = bs;
    if (block_bytes) *block_bytes = bb;
    return FMO_OK;
}

uint64_t fmo_row_bytes(uint32_t type_id, uint32_t in_dim) {
    uint32_t bs, bb;
    if (fmo_block_geometry(type_id, &bs, &bb) != FMO_OK) return 0;
    if (in_dim % bs) return 0;
    return (uint64_t)(in_dim / bs) * bb;
}

static uint16_t rd16(const uint8_t *p) { return (uint16_t)(p[0] | ((uint16_t)p[1] << 8)); }

float fmo_fp16_to_f32(uint16_t h) {
    /* src/quant.cpp:23-48.  A subnormal half is man * 2^-24, which a float
     * holds exactly, so the scaled product is the exact value. */
    const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    const uint32_t ex = (h >> 10) & 0x1Fu;
    const uint32_t man = h & 0x3FFu;
    uint32_t bits;
    if (ex == 0) {
        if (man == 0) {
            bits = sign;
        } else {
            float v = (float)man * 5.9604644775390625e-08f;
            memcpy(&bits, &v, 4);
            bits |= sign;
        }
    } else if (ex == 0x1F) {
        bits = sign | 0x7F800000u | (man << 13);
    } else {
        bits = sign | ((ex + 112u) << 23) | (man << 13);
    }
    float out;
    memcpy(&out, &bits, 4);
    return out;
}

uint16_t fmo_f32_to_fp16(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    const uint16_t sign = (uint16_t)((x >> 16) & 0x8000u);
    const uint32_t ax = x & 0x7FFFFFFFu;
    if (ax >= 0x7F800000u) return (uint16_t)(sign | 0x7C00u | (ax > 0x7F800000u ? 0x200u : 0));
    if (ax >= 0x477FF000u) return (uint16_t)(sign | 0x7C00u); /* rounds to >= 65520 -> inf */
    if (ax < 0x33000001u) return sign;                          /* < 2^-25 (ties to 0) */
    int e = (int)(ax >> 23) - 127;
    uint32_t m = (ax & 0x7FFFFFu) | 0x800000u;
    if (e < -14) {
        /* subnormal half: value = m * 2^(e-23), unit 2^-24 -> shift = -e - 1 */
        int shift = -e - 1; /* 14..24 */
        uint32_t q = m >> shift, rem = m & ((1u << shift) - 1), half = 1u << (shift - 1);
        if (rem > half || (rem == half && (q & 1))) ++q;
        return (uint16_t)(sign | q);
    }
    uint32_t q = m >> 13, rem = m & 0x1FFFu;
    if (rem > 0x1000u || (rem == 0x1000u && (q & 1))) ++q;
    uint32_t out = ((uint32_t)(e + 15) << 10) + (q - 0x400u);
    if (q == 0x800u) out = ((uint32_t)(e + 16) << 10);
    return (uint16_t)(sign | out);
}

float fmo_bf16_to_f32(uint16_t h) {
    uint32_t bits = (uint32_t)h << 16;
    float out;
    memcpy(&out, &bits, 4);
    return out;
}

/* Six-bit scale/min pair j of a Q4_K block (src/quant.cpp:63-71). */
static void q4k_scale_min(int j, const uint8_t *s, uint8_t *sc, uint8_t *mn) {
    if (j < 4) {
        *sc = (uint8_t)(s[j] & 63);
        *mn = (uint8_t)(s[j + 4] & 63);
    } else {
        *sc = (uint8_t)((s[j + 4] & 0x0F) | ((s[j - 4] >> 6) << 4));
        *mn = (uint8_t)((s[j + 4] >> 4) | ((s[j] >> 6) << 4));
    }
}

int fmo_dequant_block(uint32_t type_id, const uint8_t *src, float *dst) {
    switch (type_id) {
    case FMO_TYPE_F32: /* src/quant.cpp:165-167 */
        memcpy(dst, src, 4);
        return FMO_OK;
    case FMO_TYPE_Q8_0: { /* src/quant.cpp:223-228: d * (float)q */
        const float d = fmo_fp16_to_f32(rd16(src));
        for (int j = 0; j < 32; ++j) dst[j] = d * (float)(int8_t)src[2 + j];
        return FMO_OK;
    }
    case FMO_TYPE_Q4_K: { /* src/quant.cpp:297-318 */
        const float d = fmo_fp16_to_f32(rd16(src));
        const float dmin = fmo_fp16_to_f32(rd16(src + 2));
        const uint8_t *scales = src + 4;
        const uint8_t *qs = src + 16;
        for (int g = 0; g < 4; ++g) {
            uint8_t sc, mn;
            q4k_scale_min(2 * g, scales, &sc, &mn);
            const float d1 = d * (float)sc, m1 = dmin * (float)mn;
            q4k_scale_min(2 * g + 1, scales, &sc, &mn);
            const float d2 = d * (float)sc, m2 = dmin * (float)mn;
            float *y = dst + 64 * g;
            for (int l = 0; l < 32; ++l) y[l] = d1 * (float)(qs[l] & 0x0F) - m1;
            for (int l = 0; l < 32; ++l) y[32 + l] = d2 * (float)(qs[l] >> 4) - m2;
            qs += 32;
        }
        return FMO_OK;
    }
    case FMO_TYPE_Q6_K: { /* src/quant.cpp:347-372: (d * scale) * q, q = 6-bit code - 32 */
        const uint8_t *ql = src;
        const uint8_t *qh = src + 128;
        const int8_t *scales = (const int8_t *)(src + 192);
        const float d = fmo_fp16_to_f32(rd16(src + 208));
        float *y = dst;
        for (int n = 0; n < 256; n += 128) {
            for (int l = 0; l < 32; ++l) {
                const int is = l / 16;
                const int q1 = (int)((ql[l] & 0x0F) | (((qh[l] >> 0) & 3) << 4)) - 32;
                const int q2 = (int)((ql[l + 32] & 0x0F) | (((qh[l] >> 2) & 3) << 4)) - 32;
                const int q3 = (int)((ql[l] >> 4) | (((qh[l] >> 4) & 3) << 4)) - 32;
                const int q4 = (int)((ql[l + 32] >> 4) | (((qh[l] >> 6) & 3) << 4)) - 32;
                y[l] = d * (float)scales[is + 0] * (float)q1;
                y[l + 32] = d * (float)scales[is + 2] * (float)q2;
                y[l + 64] = d * (float)scales[is + 4] * (float)q3;
                y[l + 96] = d * (float)scales[is + 6] * (float)q4;
            }
            y += 128;
            ql += 64;
            qh += 32;
            scales += 8;
        }
        return FMO_OK;
    }
    default:
        return FMO_UNSUPPORTED_QUANTISATION;
    }
}

int fmo_dequant_region(uint32_t type_id, const uint8_t *src, float *dst, uint64_t n_elems) {
    uint32_t bs, bb;
    int rc = fmo_block_geometry(type_id, &bs, &bb);
    if (rc) return rc;
    if (n_elems % bs) return FMO_SHAPE_MISMATCH;
    for (uint64_t b = 0; b < n_elems / bs; ++b) fmo_dequant_block(type_id, src + b * bb, dst + b * bs);
    return FMO_OK;
}

void fmo_gemv_f32_scalar(const float *w, const float *x, float *y, uint32_t out_dim,
                         uint32_t in_dim) {
    /* src/kernels.cpp:132-140 */
    for (uint32_t o = 0; o < out_dim; ++o) {
        const float *row = w + (uint64_t)o * in_dim;
        float acc = 0.0f;
        for (uint32_t k = 0; k < in_dim; ++k) acc += row[k] * x[k];
        y[o] = acc;
    }
}

void fmo_gemv_f32_avx2_order(const float *w, const float *x, float *y, uint32_t out_dim,
                             uint32_t in_dim) {
    /* src/kernels.cpp:147-166: lanes l of acc0 see k = 16i + l, lanes of acc1
     * k = 16i + 8 + l; a trailing group of 8 goes to acc0. */
    for (uint32_t o = 0; o < out_dim; ++o) {
        const float *row = w + (uint64_t)o * in_dim;
        float a0[8] = {0}, a1[8] = {0};
        uint32_t k = 0;
        for (; k + 16 <= in_dim; k += 16)
            for (int l = 0; l < 8; ++l) {
                a0[l] = fmaf(row[k + l], x[k + l], a0[l]);
                a1[l] = fmaf(row[k + 8 + l], x[k + 8 + l], a1[l]);
            }
        for (; k + 8 <= in_dim; k += 8)
            for (int l = 0; l < 8; ++l) a0[l] = fmaf(row[k + l], x[k + l], a0[l]);
        float a[8], s[4];
        for (int l = 0; l < 8; ++l) a[l] = a0[l] + a1[l];
        for (int l = 0; l < 4; ++l) s[l] = a[l] + a[l + 4];
        float total = (s[0] + s[1]) + (s[2] + s[3]);
        for (; k < in_dim; ++k) total = fmaf(row[k], x[k], total);
        y[o] = total;
    }
}

static int check_gemv_args(uint32_t type_id, uint32_t in_dim, uint32_t *bs, uint32_t *bb) {
    int rc = fmo_block_geometry(type_id, bs, bb);
    if (rc) return rc;
    if (in_dim % *bs) return FMO_SHAPE_MISMATCH;
    return FMO_OK;
}

int fmo_gemv_quant_f64(uint32_t type_id, const uint8_t *w, const float *x, double *y,
                       uint32_t tokens, uint32_t out_dim, uint32_t in_dim) {
    uint32_t bs, bb;
    int rc = check_gemv_args(type_id, in_dim, &bs, &bb);
    if (rc) return rc;
    const uint64_t row_bytes = (uint64_t)(in_dim / bs) * bb;
    float *row = (float *)malloc(sizeof(float) * in_dim);
    if (!row) return FMO_INTERNAL_ERROR;
    for (uint32_t o = 0; o < out_dim; ++o) {
        fmo_dequant_region(type_id, w + o * row_bytes, row, in_dim);
        for (uint32_t t = 0; t < tokens; ++t) {
            const float *xt = x + (uint64_t)t * in_dim;
            double acc = 0.0;
            for (uint32_t k = 0; k < in_dim; ++k) acc += (double)row[k] * (double)xt[k];
            y[(uint64_t)t * out_dim + o] = acc;
        }
    }
    free(row);
    return FMO_OK;
}

int fmo_gemv_quant_fused_scalar(uint32_t type_id, const uint8_t *w, const float *x, float *y,
                                uint32_t tokens, uint32_t out_dim, uint32_t in_dim) {
    /* src/kernels.cpp:574-590 with the scalar dot of :256-259. */
    uint32_t bs, bb;
    int rc = check_gemv_args(type_id, in_dim, &bs, &bb);
    if (rc) return rc;
    const uint64_t row_bytes = (uint64_t)(in_dim / bs) * bb;
    float decoded[256];
    for (uint32_t t = 0; t < tokens; ++t) {
        const float *xt = x + (uint64_t)t * in_dim;
        for (uint32_t o = 0; o < out_dim; ++o) {
            const uint8_t *r = w + o * row_bytes;
            float total = 0.0f;
            for (uint32_t b = 0; b < in_dim / bs; ++b) {
                const float *xb = xt + (uint64_t)b * bs;
                if (bs == 1) {
                    float v;
                    fmo_dequant_block(type_id, r + (uint64_t)b * bb, &v);
                    total += v * xb[0];
                    continue;
                }
                fmo_dequant_block(type_id, r + (uint64_t)b * bb, decoded);
                float dot = 0.0f;
                for (uint32_t k = 0; k < bs; ++k) dot += decoded[k] * xb[k];
                total += dot;
            }
            y[(uint64_t)t * out_dim + o] = total;
        }
    }
    return FMO_OK;
}

int fmo_route(const float *logits, uint32_t tokens, uint32_t experts, uint32_t top_k,
              int normalise, double epsilon, double scale, uint32_t *ids, float *weights,
              float *probs_out) {
    if (experts == 0) return FMO_INVALID_ARGUMENT;
    float *probs = (float *)malloc(sizeof(float) * experts);
    double *ex = (double *)malloc(sizeof(double) * experts);
    unsigned char *taken = (unsigned char *)malloc(experts);
    int rc = FMO_OK;
    if (!probs || !ex || !taken) { rc = FMO_INTERNAL_ERROR; goto done; }
    for (uint32_t t = 0; t < tokens; ++t) {
        const float *v = logits + (uint64_t)t * experts;
        /* softmax, src/engine.cpp:378-393 */
        float mx = v[0];
        for (uint32_t e = 1; e < experts; ++e)
            if (v[e] > mx) mx = v[e];
        double sum = 0.0;
        for (uint32_t e = 0; e < experts; ++e) {
            if (!isfinite(v[e])) { rc = FMO_INTERNAL_ERROR; goto done; }
            ex[e] = exp((double)v[e] - (double)mx);
            sum += ex[e];
        }
        for (uint32_t e = 0; e < experts; ++e) probs[e] = (float)(ex[e] / sum);
        if (probs_out) memcpy(probs_out + (uint64_t)t * experts, probs, sizeof(float) * experts);
        /* top-k, src/engine.cpp:395-411: the first k of a stable descending
         * sort with ties broken toward the lower id. */
        if (experts > 1)
            for (uint32_t e = 0; e < experts; ++e)
                if (isnan(probs[e]) || probs[e] == INFINITY) { rc = FMO_INTERNAL_ERROR; goto done; }
        if (top_k > experts) { rc = FMO_INVALID_ARGUMENT; goto done; }
        memset(taken, 0, experts);
        for (uint32_t r = 0; r < top_k; ++r) {
            uint32_t best = UINT32_MAX;
            for (uint32_t e = 0; e < experts; ++e) {
                if (taken[e]) continue;
                if (best == UINT32_MAX || probs[e] > probs[best]) best = e;
            }
            taken[best] = 1;
            ids[(uint64_t)t * top_k + r] = best;
        }
        /* renormalisation, src/engine.cpp:1680-1702 */
        float *w = weights + (uint64_t)t * top_k;
        float total = 0.0f;
        for (uint32_t r = 0; r < top_k; ++r) {
            w[r] = probs[ids[(uint64_t)t * top_k + r]];
            total += w[r];
        }
        if (normalise) {
            const double denom = (double)total > epsilon ? (double)total : epsilon;
            for (uint32_t r = 0; r < top_k; ++r) w[r] = (float)((double)w[r] / denom);
        }
        for (uint32_t r = 0; r < top_k; ++r) w[r] = (float)((double)w[r] * scale);
    }
done:
    free(probs);
    free(ex);
    free(taken);
    return rc;
}

/* Engine::softmax (src/engine.cpp:378-393) over n values; 0 or INTERNAL_ERROR. */
static int softmax_ref(const float *v, uint32_t n, float *out, double *ex) {
    float mx = v[0];
    for (uint32_t i = 1; i < n; ++i)
        if (v[i] > mx) mx = v[i];
    double sum = 0.0;
    for (uint32_t i = 0; i < n; ++i) {
        if (!isfinite(v[i])) return FMO_INTERNAL_ERROR;
        ex[i] = exp((double)v[i] - (double)mx);
        sum += ex[i];
    }
    for (uint32_t i = 0; i < n; ++i) out[i] = (float)(ex[i] / sum);
    return FMO_OK;
}

/* The router's model-family variants, src/engine.cpp:1603-1702: optional logit
 * bias (:1608-1613), gating (:1618-1633), selection bias (:1637-1643), group-
 * limited routing (:1644-1675), Engine::topk on the selection (:395-411, -inf
 * allowed), weights = probs of the picked experts with the float total taken
 * before softmax-weight re-softmaxes them (:1677-1684), renormalisation with
 * the clamped or additive epsilon and the scale (:1685-1702). */
int fmo_route_ex(const float *logits, uint32_t tokens, uint32_t experts, uint32_t top_k, int gating,
                 const float *logit_bias, const float *selection_bias, uint32_t groups, uint32_t groups_used,
                 int normalise, int epsilon_additive, double epsilon, double scale, uint32_t *ids,
                 float *weights, float *probs_out) {
    if (experts == 0 || top_k > experts) return FMO_INVALID_ARGUMENT;
    if (groups > 1 && (experts % groups || groups_used == 0 || groups_used > groups)) return FMO_INVALID_ARGUMENT;
    float *scores = (float *)malloc(sizeof(float) * experts);
    float *probs = (float *)malloc(sizeof(float) * experts);
    float *sel = (float *)malloc(sizeof(float) * experts);
    double *ex = (double *)malloc(sizeof(double) * (experts > top_k ? experts : top_k));
    unsigned char *taken = (unsigned char *)malloc(experts);
    float *gsum = (float *)malloc(sizeof(float) * (groups > 1 ? groups : 1));
    unsigned char *keep = (unsigned char *)malloc(groups > 1 ? groups : 1);
    float *sw = (float *)malloc(sizeof(float) * (top_k ? top_k : 1));
    int rc = FMO_OK;
    if (!scores || !probs || !sel || !ex || !taken || !gsum || !keep || !sw) { rc = FMO_INTERNAL_ERROR; goto done; }
    for (uint32_t t = 0; t < tokens; ++t) {
        const float *v = logits + (uint64_t)t * experts;
        for (uint32_t e = 0; e < experts; ++e) scores[e] = logit_bias ? v[e] + logit_bias[e] : v[e];
        if (gating == 1) {
            for (uint32_t e = 0; e < experts; ++e) probs[e] = (float)(1.0 / (1.0 + exp(-(double)scores[e])));
        } else if (gating == 2) {
            for (uint32_t e = 0; e < experts; ++e) probs[e] = (float)sqrt(log1p(exp((double)scores[e])));
        } else if (gating == 3) {
            memcpy(probs, scores, sizeof(float) * experts);
        } else {
            if ((rc = softmax_ref(scores, experts, probs, ex))) goto done;
        }
        if (probs_out) memcpy(probs_out + (uint64_t)t * experts, probs, sizeof(float) * experts);
        for (uint32_t e = 0; e < experts; ++e) sel[e] = selection_bias ? probs[e] + selection_bias[e] : probs[e];
        for (uint32_t e = 0; e < experts; ++e)
            if (isnan(sel[e]) || sel[e] == INFINITY) { rc = FMO_INTERNAL_ERROR; goto done; }
        if (groups > 1) {
            const uint32_t per = experts / groups;
            for (uint32_t g = 0; g < groups; ++g) {
                float b0 = -INFINITY, b1 = -INFINITY; /* the two largest of the group */
                for (uint32_t e = 0; e < per; ++e) {
                    const float x = sel[g * per + e];
                    if (x > b0) { b1 = b0; b0 = x; }
                    else if (x > b1) b1 = x;
                }
                float sum = 0.0f;
                sum += b0;
                if (per >= 2) sum += b1;
                gsum[g] = sum;
            }
            for (uint32_t g = 0; g < groups; ++g) {
                uint32_t rank = 0;
                for (uint32_t h = 0; h < groups; ++h)
                    rank += (gsum[h] > gsum[g]) || (gsum[h] == gsum[g] && h < g);
                keep[g] = rank < groups_used;
            }
            for (uint32_t g = 0; g < groups; ++g)
                if (!keep[g])
                    for (uint32_t e = 0; e < per; ++e) sel[g * per + e] = -INFINITY;
        }
        memset(taken, 0, experts);
        for (uint32_t r = 0; r < top_k; ++r) {
            uint32_t best = UINT32_MAX;
            for (uint32_t e = 0; e < experts; ++e) {
                if (taken[e]) continue;
                if (best == UINT32_MAX || sel[e] > sel[best]) best = e;
            }
            taken[best] = 1;
            ids[(uint64_t)t * top_k + r] = best;
        }
        float *w = weights + (uint64_t)t * top_k;
        float total = 0.0f;
        for (uint32_t r = 0; r < top_k; ++r) {
            w[r] = probs[ids[(uint64_t)t * top_k + r]];
            total += w[r];
        }
        if (gating == 3) {
            if ((rc = softmax_ref(w, top_k, sw, ex))) goto done;
            memcpy(w, sw, sizeof(float) * top_k);
        }
        if (normalise) {
            const double denom = epsilon_additive ? (double)total + epsilon
                                                  : ((double)total > epsilon ? (double)total : epsilon);
            for (uint32_t r = 0; r < top_k; ++r) w[r] = (float)((double)w[r] / denom);
        }
        for (uint32_t r = 0; r < top_k; ++r) w[r] = (float)((double)w[r] * scale);
    }
done:
    free(scores); free(probs); free(sel); free(ex); free(taken); free(gsum); free(keep); free(sw);
    return rc;
}

int fmo_group_by_expert(const uint32_t *ids, uint32_t tokens, uint32_t top_k, uint32_t experts,
                        uint32_t *counts, uint32_t *offsets, uint32_t *pairs,
                        uint32_t *slot_of) {
    const uint64_t n = (uint64_t)tokens * top_k;
    memset(counts, 0, sizeof(uint32_t) * experts);
    for (uint64_t p = 0; p < n; ++p) {
        if (ids[p] >= experts) return FMO_INVALID_ARGUMENT;
        counts[ids[p]]++;
    }
    offsets[0] = 0;
    for (uint32_t e = 0; e < experts; ++e) offsets[e + 1] = offsets[e] + counts[e];
    uint32_t *cursor = (uint32_t *)calloc(experts ? experts : 1, sizeof(uint32_t));
    if (!cursor) return FMO_INTERNAL_ERROR;
    for (uint64_t p = 0; p < n; ++p) {
        const uint32_t e = ids[p];
        const uint32_t pos = offsets[e] + cursor[e]++;
        pairs[pos] = (uint32_t)p;
        if (slot_of) slot_of[p] = pos;
    }
    free(cursor);
    return FMO_OK;
}

float fmo_swiglu(float gate, float up) {
    /* include/fm/activation.hpp:33 and :62-84 (plain form). */
    const double g = (double)gate;
    const float act = (float)(g / (1.0 + exp(-g)));
    return act * up;
}

int fmo_moe_block(const float *x, uint32_t tokens, uint32_t d, uint32_t ffn, uint32_t top_k,
                  const uint32_t *ids, const float *weights, const uint8_t *const *expert_base,
                  uint32_t gate_type, uint32_t up_type, uint32_t down_type, float *y) {
    const uint64_t gate_bytes = fmo_row_bytes(gate_type, d) * ffn;
    const uint64_t up_bytes = fmo_row_bytes(up_type, d) * ffn;
    if (!gate_bytes || !up_bytes || !fmo_row_bytes(down_type, ffn)) return FMO_SHAPE_MISMATCH;
    double *g = (double *)malloc(sizeof(double) * ffn);
    double *u = (double *)malloc(sizeof(double) * ffn);
    double *dn = (double *)malloc(sizeof(double) * d);
    float *act = (float *)malloc(sizeof(float) * ffn);
    int rc = FMO_OK;
    if (!g || !u || !dn || !act) { rc = FMO_INTERNAL_ERROR; goto done; }
    for (uint32_t t = 0; t < tokens; ++t) {
        const float *xt = x + (uint64_t)t * d;
        float *ffn_out = y + (uint64_t)t * d;
        for (uint32_t j = 0; j < d; ++j) ffn_out[j] = 0.0f;
        for (uint32_t r = 0; r < top_k; ++r) {
            const uint32_t e = ids[(uint64_t)t * top_k + r];
            const float w = weights[(uint64_t)t * top_k + r];
            const uint8_t *base = expert_base[e];
            if ((rc = fmo_gemv_quant_f64(gate_type, base, xt, g, 1, ffn, d))) goto done;
            if ((rc = fmo_gemv_quant_f64(up_type, base + gate_bytes, xt, u, 1, ffn, d))) goto done;
            for (uint32_t j = 0; j < ffn; ++j) act[j] = fmo_swiglu((float)g[j], (float)u[j]);
            if ((rc = fmo_gemv_quant_f64(down_type, base + gate_bytes + up_bytes, act, dn, 1, d,
                                         ffn)))
                goto done;
            /* src/engine.cpp:1770 */
            for (uint32_t j = 0; j < d; ++j) ffn_out[j] += w * (float)dn[j];
        }
    }
done:
    free(g);
    free(u);
    free(dn);
    free(act);
    return rc;
}

void fmo_quantize_q8_0(const float *x, uint8_t *dst, uint64_t n_elems) {
    for (uint64_t b = 0; b < n_elems / 32; ++b) {
        const float *v = x + b * 32;
        uint8_t *blk = dst + b * 34;
        float amax = 0.0f;
        for (int j = 0; j < 32; ++j) amax = fabsf(v[j]) > amax ? fabsf(v[j]) : amax;
        const float d = amax / 127.0f;
        const uint16_t dh = fmo_f32_to_fp16(d);
        const float dd = fmo_fp16_to_f32(dh);
        const float id = dd != 0.0f ? 1.0f / dd : 0.0f;
        blk[0] = (uint8_t)(dh & 0xFF);
        blk[1] = (uint8_t)(dh >> 8);
        for (int j = 0; j < 32; ++j) {
            float q = roundf(v[j] * id);
            if (q > 127.0f) q = 127.0f;
            if (q < -127.0f) q = -127.0f;
            blk[2 + j] = (uint8_t)(int8_t)q;
        }
    }
}

void fmo_quantize_q4_k(const float *x, uint8_t *dst, uint64_t n_elems) {
    for (uint64_t b = 0; b < n_elems / 256; ++b) {
        const float *v = x + b * 256;
        uint8_t *blk = dst + b * 144;
        float scale[8], minv[8], max_scale = 0.0f, max_min = 0.0f;
        for (int j = 0; j < 8; ++j) {
            float lo = v[32 * j], hi = v[32 * j];
            for (int l = 1; l < 32; ++l) {
                lo = v[32 * j + l] < lo ? v[32 * j + l] : lo;
                hi = v[32 * j + l] > hi ? v[32 * j + l] : hi;
            }
            if (lo > 0.0f) lo = 0.0f;
            scale[j] = (hi - lo) / 15.0f;
            minv[j] = -lo;
            max_scale = scale[j] > max_scale ? scale[j] : max_scale;
            max_min = minv[j] > max_min ? minv[j] : max_min;
        }
        const uint16_t dh = fmo_f32_to_fp16(max_scale / 63.0f);
        const uint16_t mh = fmo_f32_to_fp16(max_min / 63.0f);
        const float d = fmo_fp16_to_f32(dh), dmin = fmo_fp16_to_f32(mh);
        uint8_t sc[8], mn[8];
        for (int j = 0; j < 8; ++j) {
            float s = d > 0.0f ? roundf(scale[j] / d) : 0.0f;
            float m = dmin > 0.0f ? roundf(minv[j] / dmin) : 0.0f;
            sc[j] = (uint8_t)(s < 0 ? 0 : s > 63 ? 63 : s);
            mn[j] = (uint8_t)(m < 0 ? 0 : m > 63 ? 63 : m);
        }
        blk[0] = (uint8_t)(dh & 0xFF);
        blk[1] = (uint8_t)(dh >> 8);
        blk[2] = (uint8_t)(mh & 0xFF);
        blk[3] = (uint8_t)(mh >> 8);
        uint8_t *s = blk + 4;
        for (int j = 0; j < 4; ++j) {
            s[j] = (uint8_t)((sc[j] & 63) | ((sc[j + 4] >> 4) << 6));
            s[j + 4] = (uint8_t)((mn[j] & 63) | ((mn[j + 4] >> 4) << 6));
            s[j + 8] = (uint8_t)((sc[j + 4] & 0x0F) | ((mn[j + 4] & 0x0F) << 4));
        }
        uint8_t *qs = blk + 16;
        for (int g = 0; g < 4; ++g) {
            for (int half = 0; half < 2; ++half) {
                const int j = 2 * g + half;
                const float D = d * (float)sc[j], M = dmin * (float)mn[j];
                for (int l = 0; l < 32; ++l) {
                    float q = D > 0.0f ? roundf((v[32 * j + l] + M) / D) : 0.0f;
                    int qi = q < 0 ? 0 : q > 15 ? 15 : (int)q;
                    if (half == 0) qs[32 * g + l] = (uint8_t)qi;
                    else qs[32 * g + l] |= (uint8_t)(qi << 4);
                }
            }
        }
    }
}

uint64_t fmo_fnv1a64(const uint8_t *data, uint64_t size) {
    uint64_t h = 0xCBF29CE484222325ull;
    for (uint64_t i = 0; i < size; ++i) {
        h ^= data[i];
        h *= 0x100000001B3ull;
    }
    return h;
}

void fmo_quantize_q6_k(const float *x, uint8_t *dst, uint64_t n_elems) {
    for (uint64_t blk = 0; blk < n_elems / 256; ++blk) {
        const float *v = x + blk * 256;
        uint8_t *b = dst + blk * 210;
        float gs[16], smax = 0.0f;
        for (int g = 0; g < 16; ++g) {
            float amax = 0.0f;
            for (int j = 0; j < 16; ++j) amax = fmaxf(amax, fabsf(v[16 * g + j]));
            gs[g] = amax / 31.0f;
            if (gs[g] > smax) smax = gs[g];
        }
        const uint16_t dh = fmo_f32_to_fp16(smax / 127.0f);
        const float d = fmo_fp16_to_f32(dh);
        int8_t sc[16];
        for (int g = 0; g < 16; ++g) {
            float r = d != 0.0f ? rintf(gs[g] / d) : 0.0f;
            if (r < 1.0f) r = 1.0f;
            if (r > 127.0f) r = 127.0f;
            sc[g] = (int8_t)r;
            b[192 + g] = (uint8_t)sc[g];
        }
        b[208] = (uint8_t)(dh & 0xFF);
        b[209] = (uint8_t)(dh >> 8);
        for (int h = 0; h < 2; ++h)
            for (int l = 0; l < 32; ++l) {
                int q[4];
                for (int i = 0; i < 4; ++i) {
                    const int idx = 128 * h + l + 32 * i;
                    const float step = d * (float)sc[idx / 16];
                    float r = step != 0.0f ? rintf(v[idx] / step) : 0.0f;
                    if (r < -32.0f) r = -32.0f;
                    if (r > 31.0f) r = 31.0f;
                    q[i] = (int)r + 32;
                }
                b[64 * h + l] = (uint8_t)((q[0] & 0x0F) | ((q[2] & 0x0F) << 4));
                b[64 * h + l + 32] = (uint8_t)((q[1] & 0x0F) | ((q[3] & 0x0F) << 4));
                b[128 + 32 * h + l] = (uint8_t)((q[0] >> 4) | ((q[1] >> 4) << 2) | ((q[2] >> 4) << 4) | ((q[3] >> 4) << 6));
            }
    }
}
