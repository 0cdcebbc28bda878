// tgemv_host.h -- host interface of the tcgen05 decode GEMVs (tgemv.cu) for
// the MoE block (moe.cu): workspace sections, eligibility, the expert stage.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "freemoe_b200.h"

namespace fmb {

// Workspace bytes of the tcgen05 expert stage (zero where the shape has no such path).
struct TgSections {
    uint64_t img_gu, img_dn, partial, cnt, maps;
};

TgSections tg_sections(uint32_t tokens, uint32_t experts, uint32_t top_k, uint32_t d, uint32_t ffn);
// Q4_K gate/up/down, bf16 activations, d and ffn multiples of 256, <= 1024 experts.
bool tg_eligible(const fmcuda_moe_args *a);
// x images, gate/up + SwiGLU, down; `mark(ctx, i)` records stage event i.
int tg_expert_stage(const fmcuda_moe_args *a, const uint32_t *counts, const uint32_t *offsets, const uint32_t *pairs,
                    uint8_t *img_gu, uint8_t *img_dn, float *partial, uint32_t *cnt, uint8_t *maps_area, float *part,
                    void (*mark)(void *, int), void *mark_ctx, cudaStream_t s);

} // namespace fmb
