// Attention dispatch: tensor-core flash attention for f16 plans (attn_tc.cu), the CUDA-core
// kernel (kernels.cu) for f32 plans.
#pragma once

#include "kernels.h"

namespace kh {

// Query rows per attention work tile (the sequence table's tiles are cut at this size).
int attention_tile_q(bool f16);

void launch_attention(bool f16, const AttnArgs& a, const SeqTable& seq, cudaStream_t st);

// Code of the first tensor-core attention wait that gave up (0: none); read after a sync.
int attn_error_code();

}  // namespace kh
