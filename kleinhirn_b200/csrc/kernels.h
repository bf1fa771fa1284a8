// Launchers of the plan kernels (kernels.cu: bandwidth-bound row kernels and the SIMT
// fallbacks; gemm_tc.cu: tcgen05 GEMM; attn_tc.cu: tensor-core attention).
// Every launcher takes the storage type of the plan (f16: __half storage, f32: float) and
// accumulates in f32, as the reference kernels do (src/kernels/index.ts:1-3).
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <cstdint>

namespace kh {

// Sequence table of one launch: sequence s owns packed rows [start[s], start[s] + len[s]).
// row_pos[r] is the local position of packed row r inside its sequence.
struct SeqTable {
  const int32_t* start = nullptr;
  const int32_t* len = nullptr;
  const int32_t* row_pos = nullptr;
  int count = 0;     // sequences
  int max_len = 0;   // longest sequence
  const int32_t* tiles = nullptr;  // attention work tiles: (seq, q0) pairs
  int ntiles = 0;
  const int32_t* row_seq = nullptr;  // sequence of every packed row
  // Packed attention tiles of the tensor-core kernel: 128 consecutive packed rows (q0) and the
  // packed key rows [kstart, kend) of every sequence those rows belong to.
  const int32_t* ptiles = nullptr;   // (q0, kstart, kend) triples
  int nptiles = 0;
};

constexpr int PACKED_TILE = 128;

// embln.wgsl / src/wasm/plan.ts:434-447: word + position + type, two-pass LN, optional x mask.
void launch_embln(bool f16, const void* word, const void* pos, const void* typ, const uint32_t* tt,
                  const void* w, const void* b, const float* mask, void* out, int N, int rows,
                  const int32_t* row_pos, int offset, int maxpos, float eps, int maskmul, int posids,
                  cudaStream_t st);

// layernorm.wgsl / src/wasm/plan.ts:414-431: MODE 0 LN(a), 1 LN(a) * mask, 2 LN(a + b).
void launch_layernorm(bool f16, const void* a, const void* b, const void* w, const void* bias, const float* mask,
                      void* out, int N, int rows, int mode, float eps, cudaStream_t st);

// add.wgsl MODE 0: dst += src over count elements (storage rounding).
void launch_add(bool f16, void* dst, const void* src, int64_t count, cudaStream_t st);

// add.wgsl MODE 1: dst[r, :] += src[sequence of r, :] (one source row per sequence).
void launch_add_rows(bool f16, void* dst, const void* src, int N, int rows, const int32_t* row_seq, cudaStream_t st);

// geglu.wgsl: gate[r, j] = gelu(mid[r, j]) * mid[r, I + j].
void launch_geglu(bool f16, const void* mid, void* gate, int I, int rows, cudaStream_t st);

// rope.wgsl: rotate-half RoPE on the q and k parts of qkv, table row = local position.
void launch_rope(bool f16, void* qkv, const float* cossin, const int32_t* row_pos, int H, int D, int rows,
                 cudaStream_t st);

// pool.wgsl: MODE 0 masked mean (floor 1e-9), MODE 1 masked max, one output row per sequence.
void launch_pool(bool f16, const void* x, const float* mask, void* out, int N, int mode, const SeqTable& seq,
                 cudaStream_t st);

// gather.wgsl with the zero marker buffer: out[s] = x[start[s] + marker[s]] (CLS row: marker 0).
void launch_gather(bool f16, const void* x, void* out, int D, const SeqTable& seq, const uint32_t* markers,
                   int K, cudaStream_t st);
// GLiNER2 / Julia logits: raw / temp where the marker is valid, -1e4 elsewhere (f32 out).
void launch_masklogits(bool f16, const void* raw, const uint32_t* packed, float* logits, int K, float temp,
                       int n_seqs, cudaStream_t st);

// im2col.wgsl (DeBERTa-v2 convolution input).
void launch_im2col(bool f16, const void* x, const float* mask, void* out, int N, int KS, int rows,
                   const SeqTable& seq, const int32_t* row_seq, cudaStream_t st);

// matmul.wgsl / mmtile.wgsl semantics on CUDA cores: C = act(A W^T + bias), f32 accumulation.
void launch_gemm_simt(bool f16, const void* A, const void* W, const void* bias, void* C, int M, int N, int K,
                      int act, cudaStream_t st);

// Attention over packed sequences on CUDA cores (mbattention.wgsl / attention.wgsl semantics):
// scores in f32, masked keys and keys outside the window get probability 0, a masked query row
// gets a zero context row. rel != null: DeBERTa c2p + p2c terms through relidx (L x L).
struct AttnArgs {
  const void* qkv = nullptr;
  const float* mask = nullptr;
  void* ctx = nullptr;
  int H = 0, D = 0;
  float scale = 1.f;   // standard: multiplies q.k; relative: 1 / sqrt(3 D) multiplies the sum
  int window = 0;
  bool rel = false;
  const void* pos_key = nullptr;
  const void* pos_query = nullptr;
  const uint32_t* relidx = nullptr;
  // the same index as one row over i - j when it depends on i - j only (DeBERTa's relBucketIndex,
  // src/plan/build.ts:22-45): rel1d[i - j + L - 1] == relidx[i][j]; null otherwise
  const int32_t* rel1d = nullptr;
  int L = 0;           // bucket length: relidx is L x L
  int rows = 0;        // packed rows of the launch
  int np = 0;          // rows of pos_key / pos_query (relative positions)
  float* rel_tables = nullptr;  // tensor-core relative attention: [rows][2][H][np] f32 scratch
};
void launch_attention_simt(bool f16, const AttnArgs& a, const SeqTable& seq, cudaStream_t st);

// f32 -> f16 storage conversion of a weight on the device.
void launch_f32_to_f16(const float* src, __half* dst, int64_t n, cudaStream_t st);
void launch_f16_to_f32(const __half* src, float* dst, int64_t n, cudaStream_t st);

// out[i] = table[ids[i]] for n rows of E elements (f16 or f32): the word rows of packed token ids
// (wordRows, src/encoder.ts:273-314) gathered on the device. An id outside [0, vocab) writes a
// zero row and records the failure for gather_error_code().
void launch_gather_rows(bool f16, const void* table, int64_t vocab, const int32_t* ids, int64_t n, int E, void* out,
                        cudaStream_t st);
// Number of out-of-range ids seen since the last call (0: none); resets the count. Syncs.
int gather_error_code();

// Sequence tables of a bulk run's chunks, built on the device from the sequence lengths. Chunk c
// covers sequences [seq0, seq0 + S) and packed rows [tok0, tok0 + T); its table starts at word
// word0 of `table` in the build_seq_table layout: start[S], len[S], row_pos[T], row_seq[T],
// tiles[2 ntiles] (attention work tiles of tile_q rows), ptiles[3 ceil(T / 128)].
struct ChunkDesc {
  int64_t tok0, word0;
  int32_t seq0, S, T, ntiles;
};
void launch_build_seq_tables(const int32_t* lens, const ChunkDesc* chunks, int n_chunks, int64_t total_rows,
                             int tile_q, int32_t* table, cudaStream_t st);

}  // namespace kh
