// Host runtime of the CUDA backend: context, weights, compiled plans, executions.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <functional>
#include <map>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

#include "json.hpp"
#include "kernels.h"

namespace kh {

struct CudaError : std::runtime_error {
  using std::runtime_error::runtime_error;
};
struct ArgError : std::runtime_error {
  using std::runtime_error::runtime_error;
};
struct PlanError : std::runtime_error {
  using std::runtime_error::runtime_error;
};

void cuda_check(cudaError_t e, const char* what);
#define KH_CUDA(x) ::kh::cuda_check((x), #x)

struct DevTensor {
  std::string name;
  int dtype = 0;  // 0 f32, 1 f16
  std::vector<int64_t> shape;
  void* ptr = nullptr;
  size_t bytes = 0;
  int64_t numel() const {
    int64_t n = 1;
    for (auto s : shape) n *= s;
    return n;
  }
};

struct Ctx {
  int device = 0;
  int sms = 0;
  cudaStream_t stream = nullptr;
  std::map<std::string, DevTensor> tensors;  // as added
  std::map<std::string, DevTensor> derived;  // dtype conversions and repacked layouts
  int64_t weight_bytes = 0;
  std::string broken;  // first CUDA error of a run: latched (src/device.ts:79-81)
  std::string inject;  // a failure the next latching call reports (kh_inject_cuda_error)
  ~Ctx();
  // The tensor in storage type f16 (true) or f32, converted once on the device and cached.
  const DevTensor& weight(const std::string& name, bool f16);
  // A derived tensor built by `make` once and cached under `key`.
  const DevTensor& derive(const std::string& key, const std::function<DevTensor()>& make);
};

// One launch group of a compiled plan.
struct Exec;
struct Step {
  std::string label;               // kernel family, e.g. "gemm_tc", "layernorm"
  std::vector<std::string> ops;    // plan op names covered
  int launches = 1;
  std::function<void(Exec&, cudaStream_t)> run;
};

// Buffer of a plan: row buffers scale with the packed rows, sequence buffers with the
// sequences of a launch, fixed buffers (init tables) keep their plan size.
struct BufInfo {
  std::string id;
  enum Kind { Rows, Seqs, Fixed } kind = Rows;
  size_t elem = 2;       // bytes per element
  int64_t cols = 0;      // elements per row (Rows, Seqs)
  size_t fixed_bytes = 0;
  size_t decl_bytes = 0;  // the plan's declared size (plan-mode executions allocate at least this)
  std::vector<unsigned char> init;
};

struct CompiledPlan {
  bool f16 = true;
  int length = 0, batch = 1, emb_size = 0;
  std::vector<BufInfo> bufs;
  std::map<std::string, int> buf_index;
  std::vector<Step> steps;
  std::string in_emb, in_mask, in_type;  // input buffer ids ("" when absent)
  std::string in_markers;                // marker payload of GLiNER2 / Julia plans ("" when absent)
  // Julia type rows (src/plan/ir.ts:52, src/plan/executor.ts:236-246): before the first op,
  // row qtype[b] of the table (in the plan's precision) is copied to row b of rs_dst.
  const void* rs_table = nullptr;
  int64_t rs_table_rows = 0;
  int rs_row_bytes = 0;
  std::string rs_dst;
  std::string out_buf;
  int out_rows = 0, out_cols = 0;
  bool out_f32 = false;     // output dtype 'f32' (marker logits), else the plan's storage type
  // Capture runs (src/plan/executor.ts:178-186, :267-281): f32 plans of batch 1 only. The
  // capture launch list interleaves the plan steps with the launches of each segment's
  // captureOps; after an entry, its copies put buffer prefixes into their slots.
  struct CaptureEntry {
    int step = -1;   // index into steps, or
    int extra = -1;  // index into capture_steps
    std::vector<std::pair<int, int>> copies;  // (buffer index, slot)
  };
  bool capturable = false;
  std::string capture_refusal;  // why not, in the reference's words
  std::vector<Step> capture_steps;
  std::vector<CaptureEntry> capture_order;
  int capture_slots = 0;
  int64_t capture_slot_bytes = 0;
  bool out_per_seq = true;  // pooled head: one output row per sequence
  int tile_q = 64;          // attention query tile of the launch list
};

// Device memory of one execution: plan buffers sized for `cap_rows` packed rows and
// `cap_seqs` sequences, the sequence table and the f32 output.
struct Exec {
  Ctx* ctx = nullptr;
  const CompiledPlan* cp = nullptr;
  int64_t cap_rows = 0;
  int cap_seqs = 0;
  std::vector<void*> ptr;       // by buffer index (inputs may point into bulk storage)
  std::vector<size_t> sizes;    // allocated bytes, by buffer index
  std::vector<void*> owned;     // allocations to free
  bool bulk = false;            // ragged bulk execution (fixed-dispatch ops run once per sequence)
  // current launch
  int T = 0;                    // packed rows
  SeqTable seq;                 // device pointers
  int32_t* row_seq = nullptr;   // per packed row: sequence
  // device sequence-table storage of this exec (plan mode)
  int32_t* d_table = nullptr;
  int64_t table_cap = 0;
  float* d_out = nullptr;       // f32 output staging
  int64_t out_cap = 0;
  int64_t bytes = 0;
  ~Exec();
  void* buf(int i) const { return ptr[i]; }
};

void exec_alloc(Exec& ex, Ctx* ctx, const CompiledPlan* cp, int64_t cap_rows, int cap_seqs, bool bulk);
void plan_compile(Ctx* ctx, const Json& plan, CompiledPlan& cp);
void plan_check(Ctx* ctx, const Json& plan);
// Builds the host sequence table: start, len, row_pos, row_seq, tiles for the given lengths.
void build_seq_table(const std::vector<int32_t>& lens, int tile_q, std::vector<int32_t>& out, SeqTable& offsets,
                     int64_t& total_rows);
void exec_steps(Exec& ex, cudaStream_t st);
// A capture run (f32 plans of batch 1): the launches of exec_steps with each segment's
// captureOps in place, and after each segment its capture buffers' first captureSlotBytes
// copied into slot * captureSlotBytes of `dst` (device memory of captureSlots slots).
void exec_capture(Exec& ex, void* dst, cudaStream_t st);
void exec_output(Exec& ex, int rows_out, float* dst, cudaStream_t st);

}  // namespace kh
