// tgemv_host.h -- host interface of the tcgen05 decode GEMVs (tgemv.cu) for
// the MoE block (moe.cu) and the expert-parallel expert compute (ep.cu):
// workspace sections, eligibility, the expert stage.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "freemoe_b200.h"

namespace fmb {

// Workspace bytes of the tcgen05 expert stage (zero where the shape has no such path).
struct TgSections {
    uint64_t img_gu, img_dn, partial, cnt, maps;
    uint64_t total() const { return img_gu + img_dn + partial + cnt + maps; }
};

// One expert stage: grouped pairs (router.cu's grouping) in, one f32 output row
// per pair out.  x rows are bf16 or fp16; pair g reads x row pairs[g] / top_k.
struct TgStage {
    const void *x;
    bool x_f16;                   // fp16 rows (the expert-parallel receive buffer), else bf16
    uint32_t pairs_max;           // upper bound of the routed pairs (sizes the token tiles)
    uint32_t top_k, experts, d, ffn;
    const void *const *slots;
    uint64_t up_offset, down_offset;
    const uint32_t *counts, *offsets, *pairs;
    const uint32_t *out_rows;     // output row of grouped pair g (NULL: g)
};

// pairs_max = routed pairs of one call, at most
TgSections tg_sections(uint32_t pairs_max, uint32_t experts, uint32_t d, uint32_t ffn);
bool tg_shape(uint32_t d, uint32_t ffn);
// Whether the GEMVs take the wide mode (two token tiles per weight conversion).
bool tg_wide(uint32_t pairs_max, uint32_t experts);
// Q4_K gate/up/down, bf16 activations, d and ffn multiples of 256, <= 1024 experts.
bool tg_eligible(const fmcuda_moe_args *a);
// B images, gate/up + SwiGLU, down; `mark(ctx, i)` records stage event i (3 after
// the images, 4 and 5 after gate/up, 6 after down).
int tg_expert_stage(const TgStage &t, uint8_t *img_gu, uint8_t *img_dn, float *partial, uint32_t *cnt,
                    uint8_t *maps_area, float *part, void (*mark)(void *, int), void *mark_ctx, cudaStream_t s);

// Router inputs and outputs of tg_block_stage (the plain softmax top-k router).
struct TgFront {
    const float *logits;
    uint32_t tokens;
    int normalise;
    double epsilon, scale;
    uint32_t *ids;
    float *weights;
    uint32_t *slot_of;
};
// A batch the fused front takes: <= 64 tokens, <= 64 experts, <= 1024 pairs.
bool tg_front_eligible(uint32_t tokens, uint32_t experts, uint32_t top_k);
// Router, grouping (into t.counts / t.offsets / t.pairs) and B images in one
// launch, then gate/up + SwiGLU and down; marks 1-3 after the first launch.
int tg_block_stage(const TgStage &t, const TgFront &f, uint8_t *img_gu, uint8_t *img_dn, float *partial,
                   uint32_t *cnt, uint8_t *maps_area, float *part, void (*mark)(void *, int), void *mark_ctx,
                   cudaStream_t s);

// The peer exchange's receive side for tg_recv_stage: wait until flags[0 ..
// world) reach the call's epoch (explicit, else one past *ectr), then take the
// first *n_rows of `rows` receive rows, meta_e the local expert of each
// (row, top-k slot) or -1.
struct TgRecvWait {
    const uint32_t *flags;
    uint32_t world, epoch;
    const uint32_t *ectr;
    uint64_t timeout_ns;
    const uint32_t *n_rows;
    const int32_t *meta_e;
    uint32_t rows;
};
// A receive batch the fused receive front takes: <= 64 local experts, <= 1024 (row, slot) pairs.
bool tg_recv_eligible(uint32_t rows, uint32_t top_k, uint32_t experts);
// Wait, grouping (into t.counts / t.offsets / t.pairs) and B images in one launch,
// then gate/up + SwiGLU and down; t.x are the fp16 receive rows.
int tg_recv_stage(const TgStage &t, const TgRecvWait &r, uint8_t *img_gu, uint8_t *img_dn, float *partial,
                  uint32_t *cnt, uint8_t *maps_area, float *part, cudaStream_t s);

} // namespace fmb
