// C ABI of libkhcuda.so (include/kh_cuda.h). Each entry point catches every exception of the
// runtime and turns it into a status code and a thread-local message.

#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <map>
#include <memory>
#include <set>
#include <sstream>
#include <string>
#include <vector>

#include "../../include/kh_cuda.h"
#include "attn_tc.h"
#include "gemm_tc.h"
#include "gemm_tf32.h"
#include "runtime.h"
#include "tmap.h"

using kh::Ctx;

struct kh_ctx {
  std::unique_ptr<Ctx> c;
  std::set<kh_plan*> plans;  // plans not yet destroyed: kh_destroy frees them
};

// The launch list of a plan-mode run (kh_run) replayed as one CUDA graph: captured on the second
// run with a row count (the first runs eagerly and sets every per-device kernel attribute), keyed
// by the row count and the sequence-table allocation its launches read. Everything else a launch
// reads on the host (grids, tensor maps, buffer addresses) follows from those two and the plan.
struct RunGraph {
  int rows = 0;
  const void* table = nullptr;
  cudaGraphExec_t exec = nullptr;
};

struct kh_plan {
  kh_ctx* owner = nullptr;
  std::set<kh_bulk*> bulks;  // bulk handles not yet destroyed: kh_plan_destroy frees them
  kh::CompiledPlan cp;
  kh::Exec ex;
  std::vector<int32_t> htable;
  bool markers_ready = false;   // kh_upload_markers since creation (plans with a markers input)
  void* d_capture = nullptr;    // capture slots (owned by ex once allocated)
  std::vector<int32_t> qtypes;  // Julia type of each sequence of the batch
  std::vector<RunGraph> graphs;
  std::map<int, int> eager_runs;  // eager runs per row count (a graph is captured on the second)
  bool graphs_off = false;        // KH_NO_GRAPHS set, or a capture of this plan failed
  ~kh_plan() {
    for (RunGraph& g : graphs)
      if (g.exec) cudaGraphExecDestroy(g.exec);
  }
};

struct kh_bulk {
  kh_plan* plan = nullptr;
  kh::Exec ex;               // chunk workspace
  void* d_emb = nullptr;     // resident packed inputs
  uint32_t* d_type = nullptr;
  float* d_mask = nullptr;   // ones
  float* d_out = nullptr;    // f32 outputs of every sequence (or row)
  int64_t max_tokens = 0, chunk_tokens = 0;
  int max_seqs = 0;
  int32_t* d_table = nullptr;
  int64_t table_cap = 0;
  struct Chunk {
    int64_t tok0 = 0, T = 0;
    int seq0 = 0, S = 0;
    int64_t word0 = 0;  // offset of the chunk's sequence table in d_table
    kh::SeqTable seq;   // offsets inside the chunk table
  };
  std::vector<Chunk> chunks;
  int n_seqs = 0;
  int64_t n_tokens = 0;
  cudaEvent_t ev0 = nullptr, ev1 = nullptr;
  int64_t last_launches = 0;
  const void* d_words = nullptr;  // device word table (kh_bulk_set_word_table)
  int64_t vocab = 0;
  int32_t* d_ids = nullptr;       // packed token ids of kh_bulk_upload_ids
  bool ids_used = false;          // the last upload gathered rows on the device
  // kh_bulk_run replayed as one CUDA graph when its chunks have the shapes of the previous run
  // (the same lengths uploaded again): captured on the second such run, keyed by every launch
  // parameter the chunks give (offsets, rows, sequences, tile counts, table address)
  std::vector<int64_t> graph_key, eager_key;
  cudaGraphExec_t graph = nullptr;
  bool graphs_off = false;
  ~kh_bulk();
};

namespace {

thread_local std::string g_err;

enum class Latch { No, Yes };

template <class F>
int guard(Ctx* c, Latch latch, F&& f) {
  try {
    if (c && !c->broken.empty()) {
      g_err = "device error latched earlier: " + c->broken;
      return KH_ERR_STATE;
    }
    if (c) KH_CUDA(cudaSetDevice(c->device));
    if (c && latch == Latch::Yes && !c->inject.empty()) {
      // a failure injected by kh_inject_cuda_error stands for a CUDA call of this entry point
      // that failed: reported here, latched like a real one
      const std::string what = "injected CUDA failure: " + c->inject;
      c->inject.clear();
      throw kh::CudaError(what);
    }
    f();
    return KH_OK;
  } catch (const kh::CudaError& e) {
    g_err = e.what();
    if (c && latch == Latch::Yes) c->broken = g_err;
    return KH_ERR_CUDA;
  } catch (const kh::PlanError& e) {
    g_err = e.what();
    return KH_ERR_PLAN;
  } catch (const kh::ArgError& e) {
    g_err = e.what();
    return KH_ERR_ARG;
  } catch (const std::exception& e) {
    g_err = e.what();
    return KH_ERR_ARG;
  }
}

size_t put_string(const std::string& s, char* buf, size_t cap) {
  if (buf && cap) {
    const size_t n = std::min(cap - 1, s.size());
    std::memcpy(buf, s.data(), n);
    buf[n] = 0;
  }
  return s.size() + 1;
}

// Rebases the word offsets of a host sequence table onto its device copy.
kh::SeqTable rebase(const kh::SeqTable& o, const int32_t* base) {
  kh::SeqTable s = o;
  s.start = base + (intptr_t)o.start;
  s.len = base + (intptr_t)o.len;
  s.row_pos = base + (intptr_t)o.row_pos;
  s.row_seq = base + (intptr_t)o.row_seq;
  s.tiles = base + (intptr_t)o.tiles;
  s.ptiles = base + (intptr_t)o.ptiles;
  return s;
}

// A tensor-core pipeline wait that gave up leaves a code on the device; after a sync it becomes
// a CUDA error of the call (and latches like one). Reading clears the device's error words, so
// the call that reads a code reports it and later contexts on the device start clean.
void check_pipelines() {
  const int g = kh::tc_error_code();
  const int a = kh::attn_error_code();
  const int f = kh::tf32_error_code();
  if (g || a || f)
    throw kh::CudaError("tensor-core pipeline wait timed out (gemm code " + std::to_string(g) + ", attention code " +
                        std::to_string(a) + ", f32 gemm code " + std::to_string(f) + ")");
}

std::string json_escape(const std::string& s) {
  std::string o;
  for (char c : s) {
    if (c == '"' || c == '\\') o += '\\';
    o += c;
  }
  return o;
}

}  // namespace

kh_bulk::~kh_bulk() {
  if (plan) cudaSetDevice(plan->owner->c->device);
  cudaFree(d_emb);
  cudaFree(d_type);
  cudaFree(d_mask);
  cudaFree(d_out);
  cudaFree(d_table);
  cudaFree(d_ids);
  if (graph) cudaGraphExecDestroy(graph);
  if (ev0) cudaEventDestroy(ev0);
  if (ev1) cudaEventDestroy(ev1);
}

extern "C" {

const char* kh_last_error(void) { return g_err.c_str(); }

int kh_init(const int* devices, int n_devices, kh_ctx** out) {
  if (!out || !devices || n_devices < 1) {
    g_err = "kh_init: devices and out are required";
    return KH_ERR_ARG;
  }
  *out = nullptr;
  if (n_devices > 1) {
    g_err = "kh_init: a context drives one device; open one context per device (" + std::to_string(n_devices) +
            " given)";
    return KH_ERR_ARG;
  }
  auto h = std::make_unique<kh_ctx>();
  h->c = std::make_unique<Ctx>();
  Ctx* c = h->c.get();
  c->device = devices[0];
  const int st = guard(nullptr, Latch::No, [&] {
    int count = 0;
    KH_CUDA(cudaGetDeviceCount(&count));
    if (c->device < 0 || c->device >= count) throw kh::ArgError("kh_init: device " + std::to_string(c->device) +
                                                                " outside the " + std::to_string(count) + " devices");
    KH_CUDA(cudaSetDevice(c->device));
    cudaDeviceProp prop;
    KH_CUDA(cudaGetDeviceProperties(&prop, c->device));
    if (prop.major != 10) throw kh::PlanError(std::string("kh_init: ") + prop.name + " is not an sm_100 device");
    c->sms = prop.multiProcessorCount;
    KH_CUDA(cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking));
  });
  if (st != KH_OK) return st;
  *out = h.release();
  return KH_OK;
}

int kh_add_tensor(kh_ctx* ctx, const char* name, int dtype, const int64_t* shape, int ndim, const void* bytes,
                  size_t len) {
  if (!ctx || !name || (ndim > 0 && !shape) || (len && !bytes)) {
    g_err = "kh_add_tensor: null argument";
    return KH_ERR_ARG;
  }
  Ctx* c = ctx->c.get();
  return guard(c, Latch::No, [&] {
    if (dtype != KH_F32 && dtype != KH_F16) throw kh::ArgError(std::string("tensor ") + name + ": dtype " +
                                                               std::to_string(dtype) + " is neither f32 nor f16");
    if (c->tensors.count(name)) throw kh::ArgError(std::string("weight ") + name + " loaded twice");
    kh::DevTensor t;
    t.name = name;
    t.dtype = dtype;
    t.shape.assign(shape, shape + ndim);
    const int64_t n = t.numel();
    if (n < 0 || size_t(n) * (dtype == KH_F16 ? 2 : 4) != len)
      throw kh::ArgError(std::string("tensor ") + name + ": " + std::to_string(len) + " bytes for " +
                         std::to_string(n) + " elements");
    t.bytes = len;
    KH_CUDA(cudaMalloc(&t.ptr, std::max<size_t>(len, 16)));
    KH_CUDA(cudaMemcpy(t.ptr, bytes, len, cudaMemcpyHostToDevice));
    c->weight_bytes += int64_t(len);
    c->tensors.emplace(t.name, t);
  });
}

int kh_add_words(kh_ctx* ctx, const char* name, int dtype, int64_t rows, int64_t width, int64_t row_bytes,
                 const void* bytes, size_t len) {
  if (!ctx || !name || (len && !bytes)) {
    g_err = "kh_add_words: null argument";
    return KH_ERR_ARG;
  }
  Ctx* c = ctx->c.get();
  return guard(c, Latch::No, [&] {
    if (dtype != KH_F32 && dtype != KH_F16) throw kh::ArgError("kh_add_words: dtype is neither f32 nor f16");
    if (c->tensors.count(name)) throw kh::ArgError(std::string("weight ") + name + " loaded twice");
    const int64_t esz = dtype == KH_F16 ? 2 : 4;
    if (rows < 1 || width < 1 || row_bytes < width * esz + 4 || row_bytes % 4)
      throw kh::ArgError("kh_add_words: rows of " + std::to_string(row_bytes) + " bytes cannot hold " +
                         std::to_string(width) + " values and a checksum word");
    if (int64_t(len) != rows * row_bytes)  // wordsView, src/words.ts
      throw kh::ArgError("kh_add_words: " + std::to_string(len) + " bytes, " + std::to_string(rows) + " rows of " +
                         std::to_string(row_bytes) + " need " + std::to_string(rows * row_bytes));
    kh::DevTensor t;
    t.name = name;
    t.dtype = dtype;
    t.shape = {rows, width};
    t.bytes = size_t(rows * width * esz);
    KH_CUDA(cudaMalloc(&t.ptr, std::max<size_t>(t.bytes, 16)));
    // the row values without the checksum word after each of them
    KH_CUDA(cudaMemcpy2D(t.ptr, size_t(width * esz), bytes, size_t(row_bytes), size_t(width * esz), size_t(rows),
                         cudaMemcpyHostToDevice));
    c->weight_bytes += int64_t(t.bytes);
    c->tensors.emplace(t.name, t);
  });
}

int64_t kh_weight_bytes(const kh_ctx* ctx) { return ctx ? ctx->c->weight_bytes : 0; }

int kh_check(kh_ctx* ctx, const char* plan_json, size_t len) {
  if (!ctx || !plan_json) {
    g_err = "kh_check: null argument";
    return KH_ERR_ARG;
  }
  Ctx* c = ctx->c.get();
  return guard(c, Latch::No, [&] {
    kh::Json plan;
    try {
      plan = kh::parse_json(plan_json, len);
    } catch (const std::exception& e) {
      throw kh::PlanError(e.what());
    }
    kh::plan_check(c, plan);
  });
}

int kh_plan_create(kh_ctx* ctx, const char* plan_json, size_t len, kh_plan** out) {
  if (!ctx || !plan_json || !out) {
    g_err = "kh_plan_create: null argument";
    return KH_ERR_ARG;
  }
  *out = nullptr;
  Ctx* c = ctx->c.get();
  auto p = std::make_unique<kh_plan>();
  p->owner = ctx;
  p->graphs_off = std::getenv("KH_NO_GRAPHS") != nullptr;  // every run eager (measurement, debugging)
  const int st = guard(c, Latch::No, [&] {
    kh::Json plan;
    try {
      plan = kh::parse_json(plan_json, len);
    } catch (const std::exception& e) {
      throw kh::PlanError(e.what());
    }
    kh::plan_compile(c, plan, p->cp);
    const int64_t rows = int64_t(p->cp.length) * p->cp.batch;
    kh::exec_alloc(p->ex, c, &p->cp, rows, p->cp.batch, false);
  });
  if (st != KH_OK) return st;
  ctx->plans.insert(p.get());
  *out = p.release();
  return KH_OK;
}

int kh_plan_info(const kh_plan* plan, int* length, int* batch, int* out_rows, int* out_cols, int64_t* bytes) {
  if (!plan) {
    g_err = "kh_plan_info: null plan";
    return KH_ERR_ARG;
  }
  if (length) *length = plan->cp.length;
  if (batch) *batch = plan->cp.batch;
  if (out_rows) *out_rows = plan->cp.out_rows;
  if (out_cols) *out_cols = plan->cp.out_cols;
  if (bytes) *bytes = plan->ex.bytes;
  return KH_OK;
}

int kh_upload(kh_plan* plan, const void* emb, size_t emb_bytes, const float* mask, size_t mask_len,
              const uint32_t* type_ids, size_t type_len) {
  if (!plan || !emb || !mask) {
    g_err = "kh_upload: plan, embeddings and mask are required";
    return KH_ERR_ARG;
  }
  Ctx* c = plan->owner->c.get();
  return guard(c, Latch::Yes, [&] {
    const kh::CompiledPlan& cp = plan->cp;
    const int64_t rows = int64_t(cp.length) * cp.batch;
    const size_t esz = cp.f16 ? 2 : 4;
    if (emb_bytes > size_t(rows) * cp.emb_size * esz)
      throw kh::ArgError("kh_upload: embeddings of " + std::to_string(emb_bytes) + " B exceed the plan's " +
                         std::to_string(size_t(rows) * cp.emb_size * esz) + " B");
    if (mask_len > size_t(rows)) throw kh::ArgError("kh_upload: mask longer than the plan rows");
    KH_CUDA(cudaMemcpyAsync(plan->ex.buf(cp.buf_index.at(cp.in_emb)), emb, emb_bytes, cudaMemcpyHostToDevice,
                            c->stream));
    KH_CUDA(cudaMemcpyAsync(plan->ex.buf(cp.buf_index.at(cp.in_mask)), mask, mask_len * 4, cudaMemcpyHostToDevice,
                            c->stream));
    if (!cp.in_type.empty()) {
      if (!type_ids) throw kh::ArgError("plan needs typeIds");
      if (type_len > size_t(rows)) throw kh::ArgError("kh_upload: typeIds longer than the plan rows");
      KH_CUDA(cudaMemcpyAsync(plan->ex.buf(cp.buf_index.at(cp.in_type)), type_ids, type_len * 4,
                              cudaMemcpyHostToDevice, c->stream));
    }
    KH_CUDA(cudaStreamSynchronize(c->stream));  // the caller may reuse its arrays at once
  });
}

static void plan_prepare(kh_plan* plan, int rows) {
  const kh::CompiledPlan& cp = plan->cp;
  const int L = cp.length, B = cp.batch;
  if (rows < 1 || rows > L * B)
    throw kh::ArgError("kh_run: " + std::to_string(rows) + " rows, the plan has " + std::to_string(L * B));
  std::vector<int32_t> lens;
  if (B == 1) lens.push_back(rows);
  else
    for (int b = 0; b < B; ++b) lens.push_back(std::max(0, std::min(L, rows - b * L)));
  kh::SeqTable offs;
  int64_t T = 0;
  kh::build_seq_table(lens, cp.tile_q, plan->htable, offs, T);
  kh::Exec& ex = plan->ex;
  const int64_t words = int64_t(plan->htable.size());
  if (words > ex.table_cap) {
    if (ex.d_table) cudaFree(ex.d_table);
    ex.d_table = nullptr;
    KH_CUDA(cudaMalloc((void**)&ex.d_table, size_t(std::max<int64_t>(words, 1024)) * 4));
    ex.table_cap = std::max<int64_t>(words, 1024);
  }
  KH_CUDA(cudaMemcpyAsync(ex.d_table, plan->htable.data(), size_t(words) * 4, cudaMemcpyHostToDevice,
                          plan->owner->c->stream));
  ex.seq = rebase(offs, ex.d_table);
  ex.row_seq = ex.d_table + (intptr_t)offs.row_pos + T;
  ex.T = int(T);
  if (!cp.in_markers.empty() && !plan->markers_ready) throw kh::ArgError("plan needs packedMarkers");
  if (cp.rs_table) {
    // the type row of each sequence, copied before the first op (src/plan/executor.ts:236-246)
    char* dst = (char*)ex.buf(cp.buf_index.at(cp.rs_dst));
    for (int b = 0; b < B; ++b) {
      const int q = b < int(plan->qtypes.size()) ? plan->qtypes[size_t(b)] : 0;
      KH_CUDA(cudaMemcpyAsync(dst + int64_t(b) * cp.rs_row_bytes, (const char*)cp.rs_table + int64_t(q) * cp.rs_row_bytes,
                              size_t(cp.rs_row_bytes), cudaMemcpyDeviceToDevice, plan->owner->c->stream));
    }
  }
}

int kh_upload_markers(kh_plan* plan, const uint32_t* packed, size_t packed_len, const int32_t* qtypes,
                      size_t n_qtypes) {
  if (!plan || (packed_len && !packed) || (n_qtypes && !qtypes)) {
    g_err = "kh_upload_markers: null argument";
    return KH_ERR_ARG;
  }
  Ctx* c = plan->owner->c.get();
  return guard(c, Latch::Yes, [&] {
    const kh::CompiledPlan& cp = plan->cp;
    if (cp.in_markers.empty()) throw kh::ArgError("kh_upload_markers: the plan has no markers input");
    const int ib = cp.buf_index.at(cp.in_markers);
    const size_t room = cp.bufs[size_t(ib)].fixed_bytes / 4;
    if (packed_len > room)
      throw kh::ArgError("kh_upload_markers: " + std::to_string(packed_len) + " words, the plan's payload holds " +
                         std::to_string(room));
    std::vector<int32_t> q(size_t(cp.batch), 0);
    // (a plan without type rows ignores qtype, as the reference does)
    for (size_t b = 0; cp.rs_table && b < n_qtypes && b < q.size(); ++b) {
      if (qtypes[b] < 0 || qtypes[b] >= cp.rs_table_rows)
        throw kh::ArgError("kh_upload_markers: qtype " + std::to_string(qtypes[b]) + " outside the " +
                           std::to_string(cp.rs_table_rows) + " rows of the type table");
      q[b] = qtypes[b];
    }
    if (packed_len)
      KH_CUDA(cudaMemcpyAsync(plan->ex.buf(ib), packed, packed_len * 4, cudaMemcpyHostToDevice, c->stream));
    KH_CUDA(cudaStreamSynchronize(c->stream));  // the caller may reuse its arrays at once
    plan->qtypes = std::move(q);
    plan->markers_ready = true;
  });
}

// The steps and the f32 output staging of a prepared plan-mode run: a replay of the graph of
// this row count when one exists, else eagerly (and captured for the next run on the second).
static void run_graphed(kh_plan* plan, int rows, cudaStream_t st) {
  kh::Exec& ex = plan->ex;
  auto eager = [&] {
    kh::exec_steps(ex, st);
    kh::exec_output(ex, plan->cp.out_rows, ex.d_out, st);
  };
  for (const RunGraph& g : plan->graphs)
    if (g.rows == rows && g.table == ex.d_table) {
      KH_CUDA(cudaGraphLaunch(g.exec, st));
      return;
    }
  if (plan->graphs_off || ++plan->eager_runs[rows] < 2) {
    eager();
    return;
  }
  cudaGraph_t graph = nullptr;
  KH_CUDA(cudaStreamBeginCapture(st, cudaStreamCaptureModeRelaxed));
  try {
    eager();
  } catch (...) {
    cudaStreamEndCapture(st, &graph);
    if (graph) cudaGraphDestroy(graph);
    cudaGetLastError();
    plan->graphs_off = true;
    throw;
  }
  KH_CUDA(cudaStreamEndCapture(st, &graph));
  cudaGraphExec_t exec = nullptr;
  const cudaError_t e = cudaGraphInstantiate(&exec, graph, 0);
  cudaGraphDestroy(graph);
  if (e != cudaSuccess) {  // not replayable here: this plan runs eagerly from now on
    cudaGetLastError();
    plan->graphs_off = true;
    eager();
    return;
  }
  if (plan->graphs.size() >= 8) {  // a few row counts at a time (B = 1 callers vary the length)
    cudaGraphExecDestroy(plan->graphs.front().exec);
    plan->graphs.erase(plan->graphs.begin());
  }
  plan->graphs.push_back({rows, ex.d_table, exec});
  KH_CUDA(cudaGraphLaunch(exec, st));
}

int kh_run(kh_plan* plan, int rows) {
  if (!plan) {
    g_err = "kh_run: null plan";
    return KH_ERR_ARG;
  }
  Ctx* c = plan->owner->c.get();
  return guard(c, Latch::Yes, [&] {
    plan_prepare(plan, rows);
    run_graphed(plan, rows, c->stream);
    KH_CUDA(cudaGetLastError());
  });
}

int kh_read_output(kh_plan* plan, float* out, size_t n) {
  if (!plan || !out) {
    g_err = "kh_read_output: null argument";
    return KH_ERR_ARG;
  }
  Ctx* c = plan->owner->c.get();
  return guard(c, Latch::Yes, [&] {
    const size_t need = size_t(plan->cp.out_rows) * plan->cp.out_cols;
    if (n < need) throw kh::ArgError("kh_read_output: room for " + std::to_string(n) + " values, the output has " +
                                     std::to_string(need));
    KH_CUDA(cudaMemcpyAsync(out, plan->ex.d_out, need * 4, cudaMemcpyDeviceToHost, c->stream));
    KH_CUDA(cudaStreamSynchronize(c->stream));
    check_pipelines();
  });
}

int kh_capture_check(const kh_plan* plan) {
  if (!plan) {
    g_err = "kh_capture_check: null plan";
    return KH_ERR_ARG;
  }
  if (plan->cp.capturable) return KH_OK;
  g_err = plan->cp.capture_refusal;
  return KH_ERR_ARG;
}

int kh_run_capture(kh_plan* plan) {
  if (!plan) {
    g_err = "kh_run_capture: null plan";
    return KH_ERR_ARG;
  }
  Ctx* c = plan->owner->c.get();
  return guard(c, Latch::Yes, [&] {
    const kh::CompiledPlan& cp = plan->cp;
    if (!cp.capturable) throw kh::ArgError(cp.capture_refusal);
    const size_t bytes = size_t(cp.capture_slots) * size_t(cp.capture_slot_bytes);
    if (!plan->d_capture && bytes) {
      KH_CUDA(cudaMalloc(&plan->d_capture, bytes));
      plan->ex.owned.push_back(plan->d_capture);
      KH_CUDA(cudaMemsetAsync(plan->d_capture, 0, bytes, c->stream));
    }
    plan_prepare(plan, cp.length);  // capture keeps the full bucket (src/plan/executor.ts:232)
    kh::exec_capture(plan->ex, plan->d_capture, c->stream);
    kh::exec_output(plan->ex, cp.out_rows, plan->ex.d_out, c->stream);
    KH_CUDA(cudaGetLastError());
  });
}

int kh_read_capture(kh_plan* plan, float* out, size_t n) {
  if (!plan || !out) {
    g_err = "kh_read_capture: null argument";
    return KH_ERR_ARG;
  }
  Ctx* c = plan->owner->c.get();
  return guard(c, Latch::Yes, [&] {
    const kh::CompiledPlan& cp = plan->cp;
    if (!cp.capturable) throw kh::ArgError(cp.capture_refusal);
    const size_t need = size_t(cp.capture_slots) * size_t(cp.capture_slot_bytes) / 4;
    if (n < need)
      throw kh::ArgError("kh_read_capture: room for " + std::to_string(n) + " values, the capture has " +
                         std::to_string(need));
    if (!plan->d_capture) throw kh::ArgError("kh_read_capture: no capture run yet");
    KH_CUDA(cudaMemcpyAsync(out, plan->d_capture, need * 4, cudaMemcpyDeviceToHost, c->stream));
    KH_CUDA(cudaStreamSynchronize(c->stream));
    check_pipelines();
  });
}

void kh_plan_destroy(kh_plan* plan) {
  if (!plan) return;
  cudaSetDevice(plan->owner->c->device);
  cudaStreamSynchronize(plan->owner->c->stream);
  for (kh_bulk* b : plan->bulks) delete b;  // the plan's bulk handles end with it
  plan->owner->plans.erase(plan);
  delete plan;
}

void kh_destroy(kh_ctx* ctx) {
  if (!ctx) return;
  cudaSetDevice(ctx->c->device);
  cudaStreamSynchronize(ctx->c->stream);
  // plans and bulk handles still open end with the context (Backend.dispose, src/backend.ts:45)
  for (kh_plan* p : ctx->plans) {
    for (kh_bulk* b : p->bulks) delete b;
    delete p;
  }
  delete ctx;
}

size_t kh_info(const kh_ctx* ctx, char* buf, size_t cap) {
  std::ostringstream o;
  if (!ctx) return put_string("{}", buf, cap);
  cudaDeviceProp prop;
  std::string name = "?";
  size_t total = 0;
  if (cudaGetDeviceProperties(&prop, ctx->c->device) == cudaSuccess) {
    name = prop.name;
    total = prop.totalGlobalMem;
  }
  o << "{\"backend\":\"cuda\",\"device\":" << ctx->c->device << ",\"name\":\"" << json_escape(name)
    << "\",\"sms\":" << ctx->c->sms << ",\"memoryBytes\":" << total << ",\"weightBytes\":" << ctx->c->weight_bytes
    << ",\"broken\":\"" << json_escape(ctx->c->broken) << "\"}";
  return put_string(o.str(), buf, cap);
}

size_t kh_plan_launches(const kh_plan* plan, char* buf, size_t cap) {
  std::ostringstream o;
  o << "[";
  if (plan) {
    bool first = true;
    for (const kh::Step& s : plan->cp.steps) {
      if (!first) o << ",";
      first = false;
      o << "{\"label\":\"" << json_escape(s.label) << "\",\"launches\":" << s.launches << ",\"ops\":[";
      for (size_t i = 0; i < s.ops.size(); ++i) o << (i ? "," : "") << "\"" << json_escape(s.ops[i]) << "\"";
      o << "]}";
    }
    o << (first ? "" : ",") << "{\"label\":\"output\",\"launches\":1,\"ops\":[]}";
  }
  o << "]";
  return put_string(o.str(), buf, cap);
}

int kh_plan_buffer_write(kh_plan* plan, const char* id, const void* bytes, size_t len) {
  if (!plan || !id || (len && !bytes)) {
    g_err = "kh_plan_buffer_write: null argument";
    return KH_ERR_ARG;
  }
  Ctx* c = plan->owner->c.get();
  return guard(c, Latch::Yes, [&] {
    auto it = plan->cp.buf_index.find(id);
    if (it == plan->cp.buf_index.end()) throw kh::ArgError(std::string("plan buffer ") + id + " has no memory");
    KH_CUDA(cudaMemcpy(plan->ex.buf(it->second), bytes, len, cudaMemcpyHostToDevice));
  });
}

int kh_plan_buffer_read(kh_plan* plan, const char* id, void* out, size_t len) {
  if (!plan || !id || (len && !out)) {
    g_err = "kh_plan_buffer_read: null argument";
    return KH_ERR_ARG;
  }
  Ctx* c = plan->owner->c.get();
  return guard(c, Latch::Yes, [&] {
    auto it = plan->cp.buf_index.find(id);
    if (it == plan->cp.buf_index.end()) throw kh::ArgError(std::string("plan buffer ") + id + " has no memory");
    KH_CUDA(cudaStreamSynchronize(c->stream));
    KH_CUDA(cudaMemcpy(out, plan->ex.buf(it->second), len, cudaMemcpyDeviceToHost));
  });
}

int kh_profile(kh_plan* plan, int rows, float* ms, size_t n) {
  if (!plan || (n && !ms)) {
    g_err = "kh_profile: null argument";
    return KH_ERR_ARG;
  }
  Ctx* c = plan->owner->c.get();
  return guard(c, Latch::Yes, [&] {
    plan_prepare(plan, rows);
    const auto& steps = plan->cp.steps;
    std::vector<cudaEvent_t> ev(steps.size() + 2);
    for (auto& e : ev) KH_CUDA(cudaEventCreate(&e));
    KH_CUDA(cudaEventRecord(ev[0], c->stream));
    for (size_t i = 0; i < steps.size(); ++i) {
      steps[i].run(plan->ex, c->stream);
      KH_CUDA(cudaEventRecord(ev[i + 1], c->stream));
    }
    kh::exec_output(plan->ex, plan->cp.out_rows, plan->ex.d_out, c->stream);
    KH_CUDA(cudaEventRecord(ev[steps.size() + 1], c->stream));
    KH_CUDA(cudaGetLastError());
    KH_CUDA(cudaEventSynchronize(ev.back()));
    for (size_t i = 0; i + 1 < ev.size() && i < n; ++i) KH_CUDA(cudaEventElapsedTime(&ms[i], ev[i], ev[i + 1]));
    for (auto& e : ev) cudaEventDestroy(e);
  });
}

int kh_bulk_create(kh_plan* plan, int64_t max_tokens, int max_seqs, int64_t chunk_tokens, kh_bulk** out) {
  if (!plan || !out) {
    g_err = "kh_bulk_create: null argument";
    return KH_ERR_ARG;
  }
  *out = nullptr;
  Ctx* c = plan->owner->c.get();
  auto b = std::make_unique<kh_bulk>();
  b->plan = plan;
  b->graphs_off = std::getenv("KH_NO_GRAPHS") != nullptr;
  const int st = guard(c, Latch::No, [&] {
    const kh::CompiledPlan& cp = plan->cp;
    if (max_tokens < 1 || max_seqs < 1) throw kh::ArgError("kh_bulk_create: max_tokens and max_seqs must be >= 1");
    if (!cp.in_markers.empty() || cp.rs_table)
      throw kh::ArgError("kh_bulk_create: marker plans (GLiNER2, Julia) run through kh_upload_markers / kh_run");
    if (chunk_tokens < cp.length)
      throw kh::ArgError("kh_bulk_create: chunk_tokens " + std::to_string(chunk_tokens) +
                         " below the plan length " + std::to_string(cp.length));
    chunk_tokens = std::min(chunk_tokens, std::max<int64_t>(max_tokens, cp.length));
    b->max_tokens = max_tokens;
    b->max_seqs = max_seqs;
    b->chunk_tokens = chunk_tokens;
    const int cap_seqs = int(std::min<int64_t>(max_seqs, chunk_tokens));
    kh::exec_alloc(b->ex, c, &cp, chunk_tokens, cap_seqs, true);
    const size_t esz = cp.f16 ? 2 : 4;
    KH_CUDA(cudaMalloc(&b->d_emb, size_t(max_tokens) * cp.emb_size * esz + 256));
    if (!cp.in_type.empty()) KH_CUDA(cudaMalloc((void**)&b->d_type, size_t(max_tokens) * 4 + 256));
    KH_CUDA(cudaMalloc((void**)&b->d_mask, size_t(max_tokens) * 4 + 256));
    std::vector<float> ones(size_t(max_tokens), 1.0f);
    KH_CUDA(cudaMemcpy(b->d_mask, ones.data(), size_t(max_tokens) * 4, cudaMemcpyHostToDevice));
    const int64_t out_rows = cp.out_per_seq ? max_seqs : max_tokens;
    KH_CUDA(cudaMalloc((void**)&b->d_out, size_t(out_rows) * cp.out_cols * 4 + 256));
    KH_CUDA(cudaEventCreate(&b->ev0));
    KH_CUDA(cudaEventCreate(&b->ev1));
  });
  if (st != KH_OK) return st;
  plan->bulks.insert(b.get());
  *out = b.release();
  return KH_OK;
}

int kh_bulk_set_lengths(kh_bulk* bulk, const int32_t* seq_lens, int n) {
  if (!bulk || (n > 0 && !seq_lens)) {
    g_err = "kh_bulk_set_lengths: null argument";
    return KH_ERR_ARG;
  }
  Ctx* c = bulk->plan->owner->c.get();
  return guard(c, Latch::Yes, [&] {
    const kh::CompiledPlan& cp = bulk->plan->cp;
    if (n < 1 || n > bulk->max_seqs)
      throw kh::ArgError("kh_bulk_set_lengths: " + std::to_string(n) + " sequences, room for " +
                         std::to_string(bulk->max_seqs));
    int64_t total = 0;
    for (int i = 0; i < n; ++i) {
      if (seq_lens[i] < 1 || seq_lens[i] > cp.length)
        throw kh::ArgError("kh_bulk_set_lengths: sequence " + std::to_string(i) + " has " +
                           std::to_string(seq_lens[i]) + " rows, the plan takes 1 to " + std::to_string(cp.length));
      total += seq_lens[i];
    }
    if (total > bulk->max_tokens)
      throw kh::ArgError("kh_bulk_set_lengths: " + std::to_string(total) + " rows, room for " +
                         std::to_string(bulk->max_tokens));
    // chunks on the host (O(sequences)); their tables are built on the device
    bulk->chunks.clear();
    std::vector<kh::ChunkDesc> descs;
    int s = 0;
    int64_t tok = 0, words = 0;
    const int cap_seqs = std::min(bulk->ex.cap_seqs, 1024 * 64);
    while (s < n) {
      kh_bulk::Chunk ch;
      ch.seq0 = s;
      ch.tok0 = tok;
      int64_t T = 0;
      int S = 0, ntiles = 0, max_len = 0;
      while (s < n && T + seq_lens[s] <= bulk->chunk_tokens && S < cap_seqs) {
        T += seq_lens[s];
        ntiles += (seq_lens[s] + cp.tile_q - 1) / cp.tile_q;
        max_len = std::max(max_len, int(seq_lens[s]));
        ++S;
        ++s;
      }
      const int nptiles = int((T + kh::PACKED_TILE - 1) / kh::PACKED_TILE);
      ch.T = T;
      ch.S = S;
      ch.word0 = words;
      kh::SeqTable& o = ch.seq;  // word offsets, rebased on d_table at run time
      o.start = (const int32_t*)(intptr_t)0;
      o.len = (const int32_t*)(intptr_t)S;
      o.row_pos = (const int32_t*)(intptr_t)(2 * S);
      o.row_seq = (const int32_t*)(intptr_t)(2 * S + T);
      o.tiles = (const int32_t*)(intptr_t)(2 * S + 2 * T);
      o.ptiles = (const int32_t*)(intptr_t)(2 * S + 2 * T + 2 * ntiles);
      o.count = S;
      o.max_len = max_len;
      o.ntiles = ntiles;
      o.nptiles = nptiles;
      descs.push_back({tok, words, ch.seq0, S, int32_t(T), ntiles});
      words += 2 * int64_t(S) + 2 * T + 2 * int64_t(ntiles) + 3 * int64_t(nptiles);
      bulk->chunks.push_back(ch);
      tok += T;
    }
    // device room: the tables, the lengths and the chunk descriptors (grown, never shrunk)
    const int64_t desc_words = int64_t(descs.size() * sizeof(kh::ChunkDesc) + 3) / 4;
    const int64_t need = words + n + desc_words + 64;
    if (need > bulk->table_cap) {
      cudaFree(bulk->d_table);
      bulk->d_table = nullptr;
      KH_CUDA(cudaMalloc((void**)&bulk->d_table, size_t(need) * 4));
      bulk->table_cap = need;
    }
    int32_t* d_lens = bulk->d_table + words;
    kh::ChunkDesc* d_descs = reinterpret_cast<kh::ChunkDesc*>(bulk->d_table + ((words + n + 3) & ~int64_t(3)));
    KH_CUDA(cudaMemcpyAsync(d_lens, seq_lens, size_t(n) * 4, cudaMemcpyHostToDevice, c->stream));
    KH_CUDA(cudaMemcpyAsync(d_descs, descs.data(), descs.size() * sizeof(kh::ChunkDesc), cudaMemcpyHostToDevice,
                            c->stream));
    // (copies from pageable host memory have read the host arrays when they return)
    kh::launch_build_seq_tables(d_lens, d_descs, int(descs.size()), total, cp.tile_q, bulk->d_table, c->stream);
    bulk->n_seqs = n;
    bulk->n_tokens = total;
  });
}

int kh_bulk_upload(kh_bulk* bulk, const void* emb, size_t emb_bytes, const uint32_t* type_ids, size_t type_len) {
  if (!bulk || !emb) {
    g_err = "kh_bulk_upload: bulk and embeddings are required";
    return KH_ERR_ARG;
  }
  Ctx* c = bulk->plan->owner->c.get();
  return guard(c, Latch::Yes, [&] {
    const kh::CompiledPlan& cp = bulk->plan->cp;
    const size_t need = size_t(bulk->n_tokens) * cp.emb_size * (cp.f16 ? 2 : 4);
    if (emb_bytes != need)
      throw kh::ArgError("kh_bulk_upload: embeddings of " + std::to_string(emb_bytes) + " B, the sequences need " +
                         std::to_string(need));
    KH_CUDA(cudaMemcpyAsync(bulk->d_emb, emb, need, cudaMemcpyHostToDevice, c->stream));
    if (!cp.in_type.empty()) {
      if (!type_ids || type_len != size_t(bulk->n_tokens)) throw kh::ArgError("plan needs typeIds for every row");
      KH_CUDA(cudaMemcpyAsync(bulk->d_type, type_ids, type_len * 4, cudaMemcpyHostToDevice, c->stream));
    }
  });
}

int kh_bulk_set_word_table(kh_bulk* bulk, const char* name) {
  if (!bulk || !name) {
    g_err = "kh_bulk_set_word_table: bulk and name are required";
    return KH_ERR_ARG;
  }
  Ctx* c = bulk->plan->owner->c.get();
  return guard(c, Latch::No, [&] {
    const kh::CompiledPlan& cp = bulk->plan->cp;
    if (!c->tensors.count(name)) throw kh::ArgError(std::string("kh_bulk_set_word_table: no tensor ") + name);
    const kh::DevTensor& t = c->weight(name, cp.f16);
    if (t.shape.size() != 2 || t.shape[1] != cp.emb_size)
      throw kh::ArgError(std::string("kh_bulk_set_word_table: ") + name + " is not [vocab, " +
                         std::to_string(cp.emb_size) + "]");
    if (!bulk->d_ids) KH_CUDA(cudaMalloc((void**)&bulk->d_ids, size_t(bulk->max_tokens) * 4 + 256));
    bulk->d_words = t.ptr;
    bulk->vocab = t.shape[0];
  });
}

int kh_bulk_upload_ids(kh_bulk* bulk, const int32_t* ids, size_t n, const uint32_t* type_ids, size_t type_len) {
  if (!bulk || !ids) {
    g_err = "kh_bulk_upload_ids: bulk and ids are required";
    return KH_ERR_ARG;
  }
  Ctx* c = bulk->plan->owner->c.get();
  return guard(c, Latch::Yes, [&] {
    const kh::CompiledPlan& cp = bulk->plan->cp;
    if (!bulk->d_words) throw kh::ArgError("kh_bulk_upload_ids: no word table (kh_bulk_set_word_table)");
    if (n != size_t(bulk->n_tokens))
      throw kh::ArgError("kh_bulk_upload_ids: " + std::to_string(n) + " ids, the sequences have " +
                         std::to_string(bulk->n_tokens) + " rows");
    KH_CUDA(cudaMemcpyAsync(bulk->d_ids, ids, n * 4, cudaMemcpyHostToDevice, c->stream));
    if (!cp.in_type.empty()) {
      if (!type_ids || type_len != size_t(bulk->n_tokens)) throw kh::ArgError("plan needs typeIds for every row");
      KH_CUDA(cudaMemcpyAsync(bulk->d_type, type_ids, type_len * 4, cudaMemcpyHostToDevice, c->stream));
    }
    kh::launch_gather_rows(cp.f16, bulk->d_words, bulk->vocab, bulk->d_ids, int64_t(n), cp.emb_size, bulk->d_emb,
                           c->stream);
    bulk->ids_used = true;
  });
}

int kh_bulk_run(kh_bulk* bulk) {
  if (!bulk) {
    g_err = "kh_bulk_run: null bulk";
    return KH_ERR_ARG;
  }
  Ctx* c = bulk->plan->owner->c.get();
  return guard(c, Latch::Yes, [&] {
    const kh::CompiledPlan& cp = bulk->plan->cp;
    kh::Exec& ex = bulk->ex;
    const size_t esz = cp.f16 ? 2 : 4;
    const int ie = cp.buf_index.at(cp.in_emb), im = cp.buf_index.at(cp.in_mask);
    const int it = cp.in_type.empty() ? -1 : cp.buf_index.at(cp.in_type);
    int64_t per_chunk = 1;
    for (const kh::Step& s : cp.steps) per_chunk += s.launches;
    const int64_t launches = per_chunk * int64_t(bulk->chunks.size());
    auto run_chunks = [&] {
      for (const kh_bulk::Chunk& ch : bulk->chunks) {
        ex.ptr[ie] = (char*)bulk->d_emb + size_t(ch.tok0) * cp.emb_size * esz;
        ex.ptr[im] = bulk->d_mask + ch.tok0;
        if (it >= 0) ex.ptr[it] = bulk->d_type + ch.tok0;
        const int32_t* base = bulk->d_table + ch.word0;
        ex.seq = rebase(ch.seq, base);
        ex.row_seq = const_cast<int32_t*>(base) + (intptr_t)ch.seq.row_pos + ch.T;
        ex.T = int(ch.T);
        kh::exec_steps(ex, c->stream);
        float* dst = bulk->d_out + (cp.out_per_seq ? int64_t(ch.seq0) : ch.tok0) * cp.out_cols;
        kh::exec_output(ex, cp.out_per_seq ? ch.S : int(ch.T), dst, c->stream);
      }
    };
    std::vector<int64_t> key{int64_t(reinterpret_cast<intptr_t>(bulk->d_table)), int64_t(bulk->chunks.size())};
    for (const kh_bulk::Chunk& ch : bulk->chunks) {
      const kh::SeqTable& q = ch.seq;
      for (int64_t v : {ch.tok0, ch.T, int64_t(ch.seq0), int64_t(ch.S), ch.word0, int64_t(q.count),
                        int64_t(q.max_len), int64_t(q.ntiles), int64_t(q.nptiles),
                        int64_t(reinterpret_cast<intptr_t>(q.start)), int64_t(reinterpret_cast<intptr_t>(q.len)),
                        int64_t(reinterpret_cast<intptr_t>(q.row_pos)), int64_t(reinterpret_cast<intptr_t>(q.tiles)),
                        int64_t(reinterpret_cast<intptr_t>(q.ptiles))})
        key.push_back(v);
    }
    KH_CUDA(cudaEventRecord(bulk->ev0, c->stream));
    if (bulk->graph && key == bulk->graph_key) {
      KH_CUDA(cudaGraphLaunch(bulk->graph, c->stream));
    } else if (!bulk->graphs_off && key == bulk->eager_key) {
      cudaGraph_t g = nullptr;
      KH_CUDA(cudaStreamBeginCapture(c->stream, cudaStreamCaptureModeRelaxed));
      try {
        run_chunks();
      } catch (...) {
        cudaStreamEndCapture(c->stream, &g);
        if (g) cudaGraphDestroy(g);
        cudaGetLastError();
        bulk->graphs_off = true;
        throw;
      }
      KH_CUDA(cudaStreamEndCapture(c->stream, &g));
      cudaGraphExec_t e = nullptr;
      const cudaError_t r = cudaGraphInstantiate(&e, g, 0);
      cudaGraphDestroy(g);
      if (r != cudaSuccess) {  // not replayable here: eager from now on
        cudaGetLastError();
        bulk->graphs_off = true;
        run_chunks();
      } else {
        if (bulk->graph) cudaGraphExecDestroy(bulk->graph);
        bulk->graph = e;
        bulk->graph_key = key;
        KH_CUDA(cudaGraphLaunch(e, c->stream));
      }
    } else {
      run_chunks();
      bulk->eager_key = std::move(key);
    }
    KH_CUDA(cudaEventRecord(bulk->ev1, c->stream));
    KH_CUDA(cudaGetLastError());
    bulk->last_launches = launches;
  });
}

int kh_bulk_read(kh_bulk* bulk, float* out, size_t n) {
  if (!bulk || !out) {
    g_err = "kh_bulk_read: null argument";
    return KH_ERR_ARG;
  }
  Ctx* c = bulk->plan->owner->c.get();
  return guard(c, Latch::Yes, [&] {
    const kh::CompiledPlan& cp = bulk->plan->cp;
    const size_t need = size_t(cp.out_per_seq ? bulk->n_seqs : bulk->n_tokens) * cp.out_cols;
    if (n < need) throw kh::ArgError("kh_bulk_read: room for " + std::to_string(n) + " values, the output has " +
                                     std::to_string(need));
    KH_CUDA(cudaMemcpyAsync(out, bulk->d_out, need * 4, cudaMemcpyDeviceToHost, c->stream));
    KH_CUDA(cudaStreamSynchronize(c->stream));
    check_pipelines();
    if (bulk->ids_used) {
      bulk->ids_used = false;
      const int bad = kh::gather_error_code();
      if (bad)
        throw kh::ArgError("kh_bulk_read: " + std::to_string(bad) +
                           " token ids outside the word table (their rows were zeros)");
    }
  });
}

int kh_run_batch(kh_bulk* bulk, const int32_t* seq_lens, int n, const void* emb, size_t emb_bytes,
                 const uint32_t* type_ids, size_t type_len, float* out, size_t out_len) {
  int st = kh_bulk_set_lengths(bulk, seq_lens, n);
  if (st == KH_OK) st = kh_bulk_upload(bulk, emb, emb_bytes, type_ids, type_len);
  if (st == KH_OK) st = kh_bulk_run(bulk);
  if (st == KH_OK) st = kh_bulk_read(bulk, out, out_len);
  return st;
}

int kh_bulk_last_timing(const kh_bulk* bulk, float* ms, int64_t* launches) {
  if (!bulk) {
    g_err = "kh_bulk_last_timing: null bulk";
    return KH_ERR_ARG;
  }
  Ctx* c = bulk->plan->owner->c.get();
  return guard(c, Latch::Yes, [&] {
    KH_CUDA(cudaEventSynchronize(bulk->ev1));
    if (ms) KH_CUDA(cudaEventElapsedTime(ms, bulk->ev0, bulk->ev1));
    if (launches) *launches = bulk->last_launches;
  });
}

int kh_bulk_profile(kh_bulk* bulk, float* ms, size_t n) {
  if (!bulk || (n && !ms)) {
    g_err = "kh_bulk_profile: null argument";
    return KH_ERR_ARG;
  }
  Ctx* c = bulk->plan->owner->c.get();
  return guard(c, Latch::Yes, [&] {
    const kh::CompiledPlan& cp = bulk->plan->cp;
    kh::Exec& ex = bulk->ex;
    const size_t esz = cp.f16 ? 2 : 4;
    const int ie = cp.buf_index.at(cp.in_emb), im = cp.buf_index.at(cp.in_mask);
    const int it = cp.in_type.empty() ? -1 : cp.buf_index.at(cp.in_type);
    const size_t ns = cp.steps.size() + 1;
    std::vector<double> acc(ns, 0.0);
    std::vector<cudaEvent_t> ev(ns + 1);
    for (auto& e : ev) KH_CUDA(cudaEventCreate(&e));
    for (const kh_bulk::Chunk& ch : bulk->chunks) {
      ex.ptr[ie] = (char*)bulk->d_emb + size_t(ch.tok0) * cp.emb_size * esz;
      ex.ptr[im] = bulk->d_mask + ch.tok0;
      if (it >= 0) ex.ptr[it] = bulk->d_type + ch.tok0;
      const int32_t* base = bulk->d_table + ch.word0;
      ex.seq = rebase(ch.seq, base);
      ex.row_seq = const_cast<int32_t*>(base) + (intptr_t)ch.seq.row_pos + ch.T;
      ex.T = int(ch.T);
      KH_CUDA(cudaEventRecord(ev[0], c->stream));
      for (size_t i = 0; i < cp.steps.size(); ++i) {
        cp.steps[i].run(ex, c->stream);
        KH_CUDA(cudaEventRecord(ev[i + 1], c->stream));
      }
      float* dst = bulk->d_out + (cp.out_per_seq ? int64_t(ch.seq0) : ch.tok0) * cp.out_cols;
      kh::exec_output(ex, cp.out_per_seq ? ch.S : int(ch.T), dst, c->stream);
      KH_CUDA(cudaEventRecord(ev[ns], c->stream));
      KH_CUDA(cudaGetLastError());
      KH_CUDA(cudaEventSynchronize(ev[ns]));
      for (size_t i = 0; i < ns; ++i) {
        float t = 0;
        KH_CUDA(cudaEventElapsedTime(&t, ev[i], ev[i + 1]));
        acc[i] += t;
      }
    }
    for (auto& e : ev) cudaEventDestroy(e);
    for (size_t i = 0; i < ns && i < n; ++i) ms[i] = float(acc[i]);
  });
}

void* kh_ctx_stream(const kh_ctx* ctx) { return ctx ? (void*)ctx->c->stream : nullptr; }

void kh_bulk_destroy(kh_bulk* bulk) {
  if (!bulk) return;
  cudaSetDevice(bulk->plan->owner->c->device);
  cudaStreamSynchronize(bulk->plan->owner->c->stream);
  bulk->plan->bulks.erase(bulk);
  delete bulk;
}

int kh_attention_f16_noalloc(const void* qkv, const float* mask, void* ctx, const int32_t* seq_lens, int n_seqs,
                             int heads, int head_dim, float scale, int window, void* stream) {
  return guard(nullptr, Latch::No, [&] {
    kh::attention_f16_noalloc(qkv, mask, ctx, seq_lens, n_seqs, heads, head_dim, scale, window,
                              static_cast<cudaStream_t>(stream));
  });
}

int kh_attention_f16_noalloc_status(void* stream) {
  return guard(nullptr, Latch::No, [&] {
    const int code = kh::attention_status(static_cast<cudaStream_t>(stream));
    if (code)
      throw kh::CudaError("attention pipeline wait timed out (attention code " + std::to_string(code) + ")");
  });
}

int kh_inject_cuda_error(kh_ctx* ctx, const char* what) {
  if (!ctx || !what) {
    g_err = "kh_inject_cuda_error: null argument";
    return KH_ERR_ARG;
  }
  ctx->c->inject = *what ? what : "(unnamed)";
  return KH_OK;
}

int kh_selftest_wait_limit(kh_ctx* ctx, int limit_us) {
  if (!ctx) {
    g_err = "kh_selftest_wait_limit: null context";
    return KH_ERR_ARG;
  }
  Ctx* c = ctx->c.get();
  return guard(c, Latch::Yes, [&] {
    kh::launch_wait_limit_selftest(limit_us, c->stream);
    KH_CUDA(cudaStreamSynchronize(c->stream));
    check_pipelines();
  });
}

int64_t kh_selftest_tensor_maps(int threads, int iters) {
  int64_t bad = -1;
  const int st = guard(nullptr, Latch::No, [&] { bad = kh::selftest_tensor_maps(threads, iters); });
  return st == KH_OK ? bad : -1;
}

}  // extern "C"
