// Attention dispatch: tensor-core flash attention for f16 plans (attn_tc.cu), the CUDA-core
// kernel (kernels.cu) for f32 plans.
#pragma once

#include "kernels.h"

namespace kh {

// Query rows per attention work tile (the sequence table's tiles are cut at this size).
int attention_tile_q(bool f16);

void launch_attention(bool f16, const AttnArgs& a, const SeqTable& seq, cudaStream_t st);

// Whether the tensor-core kernel takes this attention (the relative form needs AttnArgs::np and,
// at launch, AttnArgs::rel_tables of attention_rel_table_floats_per_row floats per packed row).
bool attention_tc_supported(bool f16, const AttnArgs& a);
int64_t attention_rel_table_floats_per_row(int H, int np);

// Code of the first tensor-core attention wait that gave up on the current device (0: none), read
// after a sync and cleared, so the next call starts clean.
int attn_error_code();

// Failure-path self-test: one CTA waits, with a limit of limit_us microseconds, on an mbarrier
// that nothing arrives on, so the wait gives up and records its code in the attention kernels'
// error word, as a pipeline wait that timed out does. No copy or MMA is in flight.
void launch_wait_limit_selftest(int limit_us, cudaStream_t st);

// Synchronizes `st` and returns the attention error word of the current device (cleared).
int attention_status(cudaStream_t st);

// Packed f16 attention over caller-owned device buffers with the sequence table in static device
// memory (kh_attention_f16_noalloc): qkv [T, 3 H D], mask [T] f32, ctx [T, H D]; seq_lens on the
// host, T = their sum. Throws ArgError beyond its limits, and when `st` belongs to another device
// than the current one.
void attention_f16_noalloc(const void* qkv, const float* mask, void* ctx, const int32_t* seq_lens, int n_seqs,
                           int H, int D, float scale, int window, cudaStream_t st);

}  // namespace kh
