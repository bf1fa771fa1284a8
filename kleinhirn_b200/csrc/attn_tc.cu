// Attention dispatch (first version: CUDA-core flash attention for every plan).
#include "attn_tc.h"

namespace kh {

int attention_tile_q(bool) { return 64; }

void launch_attention(bool f16, const AttnArgs& a, const SeqTable& seq, cudaStream_t st) {
  launch_attention_simt(f16, a, seq, st);
}

int attn_error_code() { return 0; }

}  // namespace kh
