// Host runtime of the CUDA backend: weights on the device, Plan JSON -> launch list, plan-mode
// runs (PlanRunner.upload / run / readOutput, src/backend.ts:14-28) and ragged bulk runs.
//
// Compilation of a Plan (src/plan/ir.ts:41-60):
// - the op list of every segment in order (capture ops are a WebGPU parity tool and skipped);
// - attention groups become one attention launch, as the WASM host fuses them
//   (fuseAttention, src/plan/wasm.ts:58-82): attscore + attsoftmax + attpv and
//   attrel(c2p) + attrel(p2c) + attscore + attsoftrel + attpv, and the fused kernels
//   mbattention / mbflash / attention of the plan itself;
// - a buffer no launch touches after the fusion (scores, c2p, p2c, kinfo) gets no memory;
// - GEMM epilogues take the residual add, GeGLU and RoPE ops that follow their GEMM
//   (gemm_tc.cu), when the f16 tensor-core path runs the GEMM.
// Rows: every row op runs over the packed rows of the launch; ops with a fixed dispatch in
// the plan (pooled heads) run over one row per sequence (src/plan/wasm.ts:338 fixed rows).

#include <cuda.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <mutex>
#include <sstream>

#include "gemm_tc.h"
#include "gemm_tf32.h"
#include "attn_tc.h"
#include "runtime.h"

namespace kh {

void cuda_check(cudaError_t e, const char* what) {
  if (e != cudaSuccess) throw CudaError(std::string(what) + ": " + cudaGetErrorString(e));
}

Ctx::~Ctx() {
  cudaSetDevice(device);
  for (auto& kv : tensors) cudaFree(kv.second.ptr);
  for (auto& kv : derived) cudaFree(kv.second.ptr);
  if (stream) cudaStreamDestroy(stream);
}

const DevTensor& Ctx::weight(const std::string& name, bool f16) {
  auto it = tensors.find(name);
  if (it == tensors.end()) throw PlanError("weight " + name + " missing");
  const DevTensor& t = it->second;
  if ((t.dtype == 1) == f16) return t;
  const std::string key = name + (f16 ? "#f16" : "#f32");
  return derive(key, [&]() {
    DevTensor d;
    d.name = key;
    d.dtype = f16 ? 1 : 0;
    d.shape = t.shape;
    d.bytes = size_t(t.numel()) * (f16 ? 2 : 4);
    KH_CUDA(cudaMalloc(&d.ptr, std::max<size_t>(d.bytes, 16)));
    if (f16) launch_f32_to_f16((const float*)t.ptr, (__half*)d.ptr, t.numel(), stream);
    else launch_f16_to_f32((const __half*)t.ptr, (float*)d.ptr, t.numel(), stream);
    KH_CUDA(cudaGetLastError());
    KH_CUDA(cudaStreamSynchronize(stream));
    return d;
  });
}

const DevTensor& Ctx::derive(const std::string& key, const std::function<DevTensor()>& make) {
  auto it = derived.find(key);
  if (it != derived.end()) return it->second;
  DevTensor d = make();
  weight_bytes += int64_t(d.bytes);
  return derived.emplace(key, d).first->second;
}

Exec::~Exec() {
  if (ctx) cudaSetDevice(ctx->device);
  for (void* p : owned) cudaFree(p);
}

namespace {

bool is_matmul(const std::string& k) { return k == "matmul" || k == "mmtile" || k == "mmtile8" || k == "mmtile16"; }

int64_t elements_written(const Json& op) {
  const std::string& k = op["kernel"].as_str();
  const Json& c = op["constants"];
  if (is_matmul(k) || k == "layernorm" || k == "embln" || k == "pool") return c["N"].as_int();
  if (k == "geglu") return c["I"].as_int();
  if (k == "attention" || k == "mbattention" || k == "mbflash" || k == "attpv") return c["H"].as_int() * c["D"].as_int();
  if (k == "gather") return c["D"].as_int();
  if (k == "im2col") return c["N"].as_int() * c["KS"].as_int();
  return 0;
}

// Ops that run once per sequence (a fixed dispatch in the plan).
bool seq_level(const Json& op) {
  const std::string& k = op["kernel"].as_str();
  const Json& d = op["dispatch"];
  if (is_matmul(k)) return d[1].is_num();
  if (k == "layernorm") return d[0].is_num();
  return k == "gather" || k == "pool" || k == "masklogits";
}

int writable_binding(const Json& op) {
  const std::string& k = op["kernel"].as_str();
  return (k == "add" || k == "rope") ? 0 : int(op["bind"].size()) - 1;
}

const std::string& bind(const Json& op, size_t i) { return op["bind"][i].as_str(); }
bool is_weight(const std::string& id) { return id.rfind("w:", 0) == 0; }
double cnum(const Json& op, const char* k) { return op["constants"][k].as_num(); }
int cint(const Json& op, const char* k) { return int(op["constants"][k].as_int()); }

// A group of plan ops that compiles to one attention launch.
struct AttnGroup {
  bool rel = false;
  std::string qkv, mask, ctx, pos_key, pos_query, relidx;
  int L = 0, H = 0, D = 0, window = 0;
  float scale = 1.f;  // multiplies q.k (standard) or the relative sum
  std::vector<std::string> names;
  size_t span = 1;    // plan ops covered
};

// src/plan/wasm.ts:58-82 plus the plan's own fused kernels.
bool match_attention(const std::vector<const Json*>& ops, size_t i, AttnGroup& g) {
  auto kern = [&](size_t j) -> std::string { return j < ops.size() ? (*ops[j])["kernel"].as_str() : ""; };
  const Json& o = *ops[i];
  const std::string k = kern(i);
  if (k == "attscore" && kern(i + 1) == "attsoftmax" && kern(i + 2) == "attpv" &&
      bind(*ops[i + 1], 1) == bind(o, 2) && bind(*ops[i + 2], 0) == bind(o, 2)) {
    g.rel = false;
    g.qkv = bind(o, 0);
    g.mask = bind(*ops[i + 1], 0);
    g.ctx = bind(*ops[i + 2], 4);
    g.L = cint(o, "L"); g.H = cint(o, "H"); g.D = cint(o, "D");
    g.scale = float(cnum(o, "SCALE"));
    g.window = cint(*ops[i + 1], "WINDOW");
    g.span = 3;
  } else if (k == "attrel" && cint(o, "PART") == 0 && kern(i + 1) == "attrel" && cint(*ops[i + 1], "PART") == 1 &&
             kern(i + 2) == "attscore" && kern(i + 3) == "attsoftrel" && kern(i + 4) == "attpv") {
    const Json& s = *ops[i + 2];
    g.rel = true;
    g.qkv = bind(o, 0);
    g.pos_key = bind(o, 1);
    g.pos_query = bind(*ops[i + 1], 1);
    g.relidx = bind(o, 3);
    g.mask = bind(*ops[i + 3], 0);
    g.ctx = bind(*ops[i + 4], 4);
    g.L = cint(s, "L"); g.H = cint(s, "H"); g.D = cint(s, "D");
    g.scale = float(cnum(*ops[i + 3], "INVSCALE"));
    g.span = 5;
  } else if (k == "mbattention" || k == "mbflash") {
    g.rel = false;
    g.qkv = bind(o, 0); g.mask = bind(o, 1); g.ctx = bind(o, 2);
    g.L = cint(o, "L"); g.H = cint(o, "H"); g.D = cint(o, "D");
    g.scale = float(cnum(o, "SCALE"));
    g.window = cint(o, "WINDOW");
    g.span = 1;
  } else if (k == "attention") {
    g.rel = true;
    g.qkv = bind(o, 0); g.pos_key = bind(o, 1); g.pos_query = bind(o, 2); g.relidx = bind(o, 3);
    g.mask = bind(o, 4); g.ctx = bind(o, 5);
    g.L = cint(o, "L"); g.H = cint(o, "H"); g.D = cint(o, "D");
    g.scale = float(1.0 / cnum(o, "SCALE"));
    g.span = 1;
  } else {
    return false;
  }
  for (size_t j = i; j < i + g.span; ++j) g.names.push_back((*ops[j])["name"].as_str());
  return true;
}

const char* SUPPORTED[] = {"matmul", "mmtile", "mmtile8", "mmtile16", "layernorm", "embln", "add", "gather",
                           "pool", "geglu", "rope", "im2col", "attscore", "attsoftmax", "attpv", "attrel",
                           "attsoftrel", "mbattention", "mbflash", "attention", "masklogits"};

}  // namespace

void plan_check(Ctx* ctx, const Json& plan) {
  (void)ctx;
  const bool f16 = plan["f16"].as_bool();
  (void)f16;
  for (const Json& seg : plan["segments"].arr) {
    for (const Json& op : seg["ops"].arr) {
      const std::string& k = op["kernel"].as_str();
      bool ok = false;
      for (const char* s : SUPPORTED) ok = ok || k == s;
      if (!ok) throw PlanError("plan op " + op["name"].as_str() + ": kernel " + k + " has no CUDA computation");
      if ((k == "layernorm" || k == "embln") && cint(op, "N") > 1024)
        throw PlanError("plan op " + op["name"].as_str() + ": norm width above 1024");
      if ((k == "attention" || k == "mbattention" || k == "mbflash" || k == "attscore") && cint(op, "D") > 64)
        throw PlanError("plan op " + op["name"].as_str() + ": head dimension above 64");
    }
  }
  if (plan.has("rowSelect") && plan["rowSelect"].kind != Json::Null) {
    const Json& rs = plan["rowSelect"];
    if (!is_weight(rs["table"].as_str())) throw PlanError("rowSelect: the table is not a weight");
  }
}

void plan_compile(Ctx* ctx, const Json& plan, CompiledPlan& cp) {
  plan_check(ctx, plan);
  cp.f16 = plan["f16"].as_bool();
  cp.length = int(plan["length"].as_int());
  cp.batch = int(plan["batch"].as_int());
  cp.emb_size = int(plan["embeddingSize"].as_int());
  const bool f16 = cp.f16;
  const size_t esz = f16 ? 2 : 4;

  // The ops in order, with their segment; the captureOps of capturable plans are compiled too,
  // into launches only capture runs make.
  if (f16) cp.capture_refusal = "capture needs an f32 plan: the capture copies and readCapture are f32";
  else if (cp.batch != 1)
    cp.capture_refusal = "capture needs a plan of batch 1, this one has " + std::to_string(cp.batch);
  cp.capturable = cp.capture_refusal.empty();
  std::vector<const Json*> ops;
  std::vector<int> op_seg;
  std::vector<bool> op_cap;
  {
    int sgi = 0;
    for (const Json& seg : plan["segments"].arr) {
      if (cp.capturable && seg.has("captureOps"))
        for (const Json& op : seg["captureOps"].arr) {
          ops.push_back(&op);
          op_seg.push_back(sgi);
          op_cap.push_back(true);
        }
      for (const Json& op : seg["ops"].arr) {
        ops.push_back(&op);
        op_seg.push_back(sgi);
        op_cap.push_back(false);
      }
      ++sgi;
    }
  }

  // Buffers: declared ones, with their init blobs.
  std::map<std::string, const Json*> decl;
  for (const Json& d : plan["buffers"].arr) decl[d["id"].as_str()] = &d;
  const Json& inputs = plan["inputs"];
  cp.in_emb = inputs["embeddings"].as_str();
  cp.in_mask = inputs["mask"].as_str();
  cp.in_type = inputs.has("typeIds") ? inputs["typeIds"].as_str() : "";
  cp.in_markers = inputs.has("markers") ? inputs["markers"].as_str() : "";
  const Json& out = plan["output"];
  cp.out_buf = out["buffer"].as_str();
  cp.out_rows = int(out["rows"].as_int());
  cp.out_cols = int(out["cols"].as_int());
  cp.out_f32 = out.has("dtype") && out["dtype"].as_str() == "f32";
  if (plan.has("rowSelect") && plan["rowSelect"].kind != Json::Null) {
    const Json& rs = plan["rowSelect"];
    const DevTensor& t = ctx->weight(rs["table"].as_str().substr(2), f16);
    cp.rs_table = t.ptr;
    cp.rs_row_bytes = int(rs["rowBytes"].as_int());
    cp.rs_table_rows = int64_t(t.bytes / size_t(cp.rs_row_bytes));
    cp.rs_dst = rs["dst"].as_str();
  }

  std::map<std::string, BufInfo> info;
  auto touch = [&](const std::string& id) -> BufInfo& {
    auto it = info.find(id);
    if (it != info.end()) return it->second;
    BufInfo b;
    b.id = id;
    b.elem = esz;
    if (id[0] == '#') return info.emplace(id, b).first->second;  // scratch of this runtime, not in the plan
    auto dit = decl.find(id);
    if (dit == decl.end()) throw PlanError("plan: buffer " + id + " is not declared");
    const Json& d = *dit->second;
    b.decl_bytes = size_t(d["bytes"].as_int());
    if (d.has("init_b64")) {
      b.kind = BufInfo::Fixed;
      b.init = base64_decode(d["init_b64"].as_str());
      b.fixed_bytes = size_t(d["bytes"].as_int());
    } else if (id == "dummy") {
      b.kind = BufInfo::Fixed;
      b.fixed_bytes = size_t(d["bytes"].as_int());
    }
    return info.emplace(id, b).first->second;
  };
  {
    BufInfo& e = touch(cp.in_emb);
    e.kind = BufInfo::Rows; e.cols = cp.emb_size; e.elem = esz;
    BufInfo& m = touch(cp.in_mask);
    m.kind = BufInfo::Rows; m.cols = 1; m.elem = 4;
    if (!cp.in_type.empty()) {
      BufInfo& t = touch(cp.in_type);
      t.kind = BufInfo::Rows; t.cols = 1; t.elem = 4;
    }
  }
  auto written = [&](const Json& op) {
    const std::string& id = bind(op, size_t(writable_binding(op)));
    BufInfo& b = touch(id);
    if (b.kind == BufInfo::Fixed) return;
    b.cols = std::max<int64_t>(b.cols, elements_written(op));
    if (seq_level(op)) b.kind = BufInfo::Seqs;
  };
  auto use = [&](const std::string& id) {
    if (!is_weight(id)) touch(id);
  };

  // Launch list.
  std::vector<std::function<void(CompiledPlan&)>> pending;  // index resolution after buffers exist
  struct Proto {
    std::string label;
    std::vector<std::string> names;
    std::function<Step(const CompiledPlan&)> make;
    int seg = 0;
    bool cap = false;
  };
  std::vector<Proto> protos;
  size_t tagged = 0;  // protos whose segment is recorded
  auto tag = [&](size_t op_index) {
    for (; tagged < protos.size(); ++tagged) {
      protos[tagged].seg = op_seg[op_index];
      protos[tagged].cap = op_cap[op_index];
    }
  };
  auto bi = [](const CompiledPlan& c, const std::string& id) -> int {
    auto it = c.buf_index.find(id);
    if (it == c.buf_index.end()) throw PlanError("plan: buffer " + id + " has no memory");
    return it->second;
  };
  auto wptr = [ctx, f16](const std::string& id) -> const void* {
    if (id == "zero") return nullptr;
    return ctx->weight(id.substr(2), f16).ptr;
  };
  // A bias or norm-bias binding: a weight, or the plan's zero buffer (read as zeros).
  struct Ref {
    bool weight = false;
    const void* w = nullptr;
    std::string buf;
  };
  auto ref = [&](const std::string& id) -> Ref {
    Ref r;
    if (is_weight(id)) {
      r.weight = true;
      r.w = ctx->weight(id.substr(2), f16).ptr;
    } else {
      r.buf = id;
      use(id);
    }
    return r;
  };
  auto resolve = [bi](const CompiledPlan& c, const Ref& r) -> std::function<const void*(Exec&)> {
    if (r.weight) {
      const void* w = r.w;
      return [w](Exec&) { return w; };
    }
    const int i = bi(c, r.buf);
    return [i](Exec& ex) -> const void* { return ex.buf(i); };
  };

  std::vector<bool> consumed(ops.size(), false);
  size_t last_op = 0;
  for (size_t i = 0; i < ops.size(); ++i) {
    if (consumed[i]) continue;
    tag(last_op);
    last_op = i;
    const Json& op = *ops[i];
    const std::string k = op["kernel"].as_str();
    const std::string name = op["name"].as_str();
    AttnGroup g;
    if (match_attention(ops, i, g)) {
      for (size_t j = i; j < i + g.span; ++j) consumed[j] = true;
      use(g.qkv); use(g.mask);
      BufInfo& cb = touch(g.ctx);
      cb.cols = std::max<int64_t>(cb.cols, int64_t(g.H) * g.D);
      const void* pk = nullptr;
      const void* pq = nullptr;
      int np = 0;
      bool rel_tables = false;
      std::string rel1d_id;
      if (g.rel) {
        const DevTensor& tk = ctx->weight(g.pos_key.substr(2), f16);
        pk = tk.ptr;
        pq = ctx->weight(g.pos_query.substr(2), f16).ptr;
        np = tk.shape.empty() ? 0 : int(tk.shape[0]);
        use(g.relidx);
        {
          // relidx as one row over i - j, when the plan's L x L table depends on i - j only
          const BufInfo& rb = touch(g.relidx);
          const int L = g.L;
          if (L > 0 && rb.init.size() >= size_t(L) * L * 4) {
            const uint32_t* t = reinterpret_cast<const uint32_t*>(rb.init.data());
            std::vector<int32_t> r1(size_t(2 * L - 1));
            for (int d = 0; d < L; ++d) r1[size_t(d + L - 1)] = int32_t(t[size_t(d) * L]);    // i - j = d >= 0
            for (int d = 1; d < L; ++d) r1[size_t(L - 1 - d)] = int32_t(t[size_t(d)]);        // i - j = -d
            bool toeplitz = true;
            for (int i = 0; i < L && toeplitz; ++i)
              for (int j = 0; j < L; ++j)
                if (int32_t(t[size_t(i) * L + j]) != r1[size_t(i - j + L - 1)]) { toeplitz = false; break; }
            if (toeplitz) {
              rel1d_id = "#rel1d:" + g.relidx;
              BufInfo& b1 = touch(rel1d_id);
              b1.kind = BufInfo::Fixed;
              b1.elem = 4;
              b1.init.resize(r1.size() * 4);
              std::memcpy(b1.init.data(), r1.data(), b1.init.size());
              b1.fixed_bytes = b1.init.size();
            }
          }
        }
        AttnArgs probe;
        probe.rel = true; probe.D = g.D; probe.L = g.L; probe.np = np;
        if (attention_tc_supported(f16, probe)) {
          // c2p / p2c tables of the tensor-core path: f32 scratch rows shared by every layer
          rel_tables = true;
          BufInfo& tb = touch("#reltables");
          tb.kind = BufInfo::Rows;
          tb.elem = 4;
          tb.cols = std::max<int64_t>(tb.cols, attention_rel_table_floats_per_row(g.H, np));
        }
      }
      protos.push_back({"attention", g.names, [=](const CompiledPlan& c) {
        const int iq = bi(c, g.qkv), im = bi(c, g.mask), ic = bi(c, g.ctx);
        const int ir = g.rel ? bi(c, g.relidx) : -1;
        const int i1 = rel1d_id.empty() ? -1 : bi(c, rel1d_id);
        const int it = rel_tables ? bi(c, "#reltables") : -1;
        Step s;
        s.run = [=](Exec& ex, cudaStream_t st) {
          AttnArgs a;
          a.qkv = ex.buf(iq); a.mask = (const float*)ex.buf(im); a.ctx = ex.buf(ic);
          a.H = g.H; a.D = g.D; a.scale = g.scale; a.window = g.window; a.rel = g.rel;
          a.pos_key = pk; a.pos_query = pq; a.relidx = ir >= 0 ? (const uint32_t*)ex.buf(ir) : nullptr;
          a.rel1d = i1 >= 0 ? (const int32_t*)ex.buf(i1) : nullptr;
          a.L = g.L;
          a.np = np;
          a.rel_tables = it >= 0 ? (float*)ex.buf(it) : nullptr;
          a.rows = ex.T;
          launch_attention(f16, a, ex.seq, st);
        };
        return s;
      }});
      continue;
    }
    consumed[i] = true;
    for (size_t b = 0; b < op["bind"].size(); ++b) {
      const std::string& id = bind(op, b);
      if (!is_weight(id) && int(b) != writable_binding(op)) use(id);
    }
    if (!is_matmul(k)) written(op);
    const bool fixed_rows = seq_level(op);
    if (is_matmul(k)) {
      const int N = cint(op, "N"), K = cint(op, "K"), act = cint(op, "ACT");
      const int fixed_m = cint(op, "M");
      const std::string a_id = bind(op, 0), c_id = bind(op, 3);
      const void* W = wptr(bind(op, 1));
      Ref bias = ref(bind(op, 2));
      // Epilogue fusion with the op that follows (tensor-core path only).
      GemmEpilogue epi;
      std::vector<std::string> names{name};
      std::string res_id, out_id = c_id;
      int out_cols = N;
      const std::string wname = bind(op, 1).substr(2);
      // matmul + layernorm mode 2 over (residual, matmul output): one kernel (post-norm layers)
      bool addln = false;
      std::string ln_res, ln_out;
      Ref ln_w, ln_b;
      float ln_eps = 0.f;
      if (f16 && !fixed_rows && act == 0 && i + 1 < ops.size() && gemm_tc_supported_addln(N, K)) {
        const Json& nx = *ops[i + 1];
        if (nx["kernel"].as_str() == "layernorm" && cint(nx, "MODE") == 2 && cint(nx, "N") == N &&
            !seq_level(nx) && bind(nx, 1) == c_id && bind(nx, 0) != c_id) {
          addln = true;
          ln_res = bind(nx, 0);
          ln_out = bind(nx, 5);
          ln_w = ref(bind(nx, 2));
          ln_b = ref(bind(nx, 3));
          ln_eps = float(cnum(nx, "EPS"));
          use(ln_res);
          consumed[i + 1] = true;
          names.push_back(nx["name"].as_str());
          written(nx);
        }
      }
      if (!f16 && gemm_tf32_supported(N, K)) {
        // f32 plans on the tensor cores: the weight's TF32 split derived once, the activations
        // split stage by stage inside the GEMM, three TF32 products per K step
        const float* wsplit = static_cast<const float*>(gemm_tf32_weight(ctx, wname).ptr);
        const int64_t wn = int64_t(N) * K;
        written(op);
        protos.push_back({"gemm", names, [=](const CompiledPlan& c) {
          const int ia = bi(c, a_id), io = bi(c, out_id);
          auto fb = resolve(c, bias);
          const bool bias_zero = !bias.weight;
          Step s;
          s.run = [=](Exec& ex, cudaStream_t st) {
            const int M = fixed_rows ? (ex.bulk ? ex.seq.count : fixed_m) : ex.T;
            launch_gemm_tf32x3(static_cast<const float*>(ex.buf(ia)), wsplit, wsplit + wn,
                               bias_zero ? nullptr : static_cast<const float*>(fb(ex)),
                               static_cast<float*>(ex.buf(io)), M, N, K, act, st);
          };
          return s;
        }});
        continue;
      }
      if (addln) {
        protos.push_back({"gemm", names, [=](const CompiledPlan& c) {
          const int ia = bi(c, a_id), ir = bi(c, ln_res), io = bi(c, ln_out);
          auto fb = resolve(c, bias);
          auto fw = resolve(c, ln_w), fnb = resolve(c, ln_b);
          const bool bias_zero = !bias.weight, lnb_zero = !ln_b.weight;
          Step s;
          s.run = [=](Exec& ex, cudaStream_t st) {
            launch_gemm_addln(ex.buf(ia), W, bias_zero ? nullptr : fb(ex), ex.buf(ir), fw(ex),
                              lnb_zero ? nullptr : fnb(ex), ln_eps, ex.buf(io), ex.T, N, K, st);
          };
          return s;
        }});
        continue;
      }
      if (f16 && !fixed_rows && act == 0 && i + 1 < ops.size() && gemm_tc_supported(N, K)) {
        const Json& nx = *ops[i + 1];
        const std::string nk = nx["kernel"].as_str();
        if (nk == "add" && cint(nx, "MODE") == 0 && bind(nx, 1) == c_id) {
          epi.kind = GemmEpilogue::Residual;  // dst = dst + round(acc + bias)
          res_id = bind(nx, 0);
          out_id = res_id;
          consumed[i + 1] = true;
          names.push_back(nx["name"].as_str());
        } else if (nk == "geglu" && bind(nx, 0) == c_id && cint(nx, "I") * 2 == N && gemm_tc_supported_geglu(N, K)) {
          epi.kind = GemmEpilogue::GeGLU;  // gate = gelu(round(a)) * round(b)
          out_id = bind(nx, 1);
          out_cols = N / 2;
          consumed[i + 1] = true;
          names.push_back(nx["name"].as_str());
          BufInfo& gb = touch(out_id);
          gb.cols = std::max<int64_t>(gb.cols, out_cols);
          W = ctx->derive(wname + "#geglu-interleave", [&]() { return gemm_geglu_weight(ctx, wname, N, K); }).ptr;
          if (!bias.weight) {
            // zero bias: none
          } else {
            const std::string bname = bind(op, 2).substr(2);
            bias.w = ctx->derive(bname + "#geglu-interleave", [&]() { return gemm_geglu_bias(ctx, bname, N); }).ptr;
          }
        } else if (nk == "rope" && bind(nx, 0) == c_id && gemm_tc_supported_rope(cint(nx, "D"))) {
          epi.kind = GemmEpilogue::Rope;
          epi.H = cint(nx, "H");
          epi.D = cint(nx, "D");
          epi.table_id = bind(nx, 1);
          use(epi.table_id);
          consumed[i + 1] = true;
          names.push_back(nx["name"].as_str());
        }
      }
      if (epi.kind == GemmEpilogue::None || epi.kind == GemmEpilogue::Rope) written(op);
      protos.push_back({"gemm", names, [=](const CompiledPlan& c) {
        const int ia = bi(c, a_id), io = bi(c, out_id);
        auto fb = resolve(c, bias);
        const int itab = epi.kind == GemmEpilogue::Rope ? bi(c, epi.table_id) : -1;
        const bool bias_zero = !bias.weight;
        Step s;
        s.run = [=](Exec& ex, cudaStream_t st) {
          const int M = fixed_rows ? (ex.bulk ? ex.seq.count : fixed_m) : ex.T;
          const void* bp = bias_zero ? nullptr : fb(ex);
          GemmEpilogue e = epi;
          if (itab >= 0) { e.table = (const float*)ex.buf(itab); e.row_pos = ex.seq.row_pos; }
          launch_gemm(ex.ctx, f16, ex.buf(ia), W, bp, ex.buf(io), M, N, K, act, e, st);
        };
        return s;
      }});
      (void)out_cols;
      continue;
    }
    if (k == "layernorm") {
      const int N = cint(op, "N"), mode = cint(op, "MODE");
      const int fixed_n = fixed_rows ? int(op["dispatch"][0].as_int()) : 0;
      const float eps = float(cnum(op, "EPS"));
      const std::string a = bind(op, 0), b2 = bind(op, 1), m = bind(op, 4), o = bind(op, 5);
      Ref w = ref(bind(op, 2)), bb = ref(bind(op, 3));
      protos.push_back({"layernorm", {name}, [=](const CompiledPlan& c) {
        const int ia = bi(c, a), ib = bi(c, b2), im = bi(c, m), io = bi(c, o);
        auto fw = resolve(c, w);
        auto fbb = resolve(c, bb);
        Step s;
        s.run = [=](Exec& ex, cudaStream_t st) {
          const int rows = fixed_rows ? (ex.bulk ? ex.seq.count : fixed_n) : ex.T;
          launch_layernorm(f16, ex.buf(ia), ex.buf(ib), fw(ex), fbb(ex), (const float*)ex.buf(im), ex.buf(io), N,
                           rows, mode, eps, st);
        };
        return s;
      }});
      continue;
    }
    if (k == "embln") {
      const int N = cint(op, "N"), offset = cint(op, "OFFSET"), maxpos = cint(op, "MAXPOS");
      const int maskmul = cint(op, "MASKMUL"), posids = cint(op, "POSIDS");
      const float eps = float(cnum(op, "EPS"));
      const std::string e = bind(op, 0), tt = bind(op, 3), m = bind(op, 6), o = bind(op, 7);
      Ref pos = ref(bind(op, 1)), typ = ref(bind(op, 2)), w = ref(bind(op, 4)), bb = ref(bind(op, 5));
      protos.push_back({"embln", {name}, [=](const CompiledPlan& c) {
        const int ie = bi(c, e), it = bi(c, tt), im = bi(c, m), io = bi(c, o);
        auto fp = resolve(c, pos), ft = resolve(c, typ), fw = resolve(c, w), fbb = resolve(c, bb);
        Step s;
        s.run = [=](Exec& ex, cudaStream_t st) {
          launch_embln(f16, ex.buf(ie), fp(ex), ft(ex), (const uint32_t*)ex.buf(it), fw(ex), fbb(ex),
                       (const float*)ex.buf(im), ex.buf(io), N, ex.T, ex.seq.row_pos, offset, maxpos, eps, maskmul,
                       posids, st);
        };
        return s;
      }});
      continue;
    }
    if (k == "add") {
      const int N = cint(op, "N"), mode = cint(op, "MODE");
      const std::string d = bind(op, 0), sname = bind(op, 1);
      protos.push_back({"add", {name}, [=](const CompiledPlan& c) {
        const int id = bi(c, d), is = bi(c, sname);
        Step s;
        s.run = [=](Exec& ex, cudaStream_t st) {
          if (mode == 0) launch_add(f16, ex.buf(id), ex.buf(is), int64_t(ex.T) * N, st);
          else launch_add_rows(f16, ex.buf(id), ex.buf(is), N, ex.T, ex.row_seq, st);
        };
        return s;
      }});
      continue;
    }
    if (k == "geglu") {
      const int I = cint(op, "I");
      const std::string m = bind(op, 0), g2 = bind(op, 1);
      protos.push_back({"geglu", {name}, [=](const CompiledPlan& c) {
        const int im = bi(c, m), ig = bi(c, g2);
        Step s;
        s.run = [=](Exec& ex, cudaStream_t st) { launch_geglu(f16, ex.buf(im), ex.buf(ig), I, ex.T, st); };
        return s;
      }});
      continue;
    }
    if (k == "rope") {
      const int H = cint(op, "H"), D = cint(op, "D");
      const std::string q = bind(op, 0), t = bind(op, 1);
      protos.push_back({"rope", {name}, [=](const CompiledPlan& c) {
        const int iq = bi(c, q), itb = bi(c, t);
        Step s;
        s.run = [=](Exec& ex, cudaStream_t st) {
          launch_rope(f16, ex.buf(iq), (const float*)ex.buf(itb), ex.seq.row_pos, H, D, ex.T, st);
        };
        return s;
      }});
      continue;
    }
    if (k == "pool") {
      const int N = cint(op, "N"), mode = cint(op, "MODE");
      const std::string x = bind(op, 0), m = bind(op, 1), o = bind(op, 2);
      protos.push_back({"pool", {name}, [=](const CompiledPlan& c) {
        const int ix = bi(c, x), im = bi(c, m), io = bi(c, o);
        Step s;
        s.run = [=](Exec& ex, cudaStream_t st) {
          launch_pool(f16, ex.buf(ix), (const float*)ex.buf(im), ex.buf(io), N, mode, ex.seq, st);
        };
        return s;
      }});
      continue;
    }
    if (k == "gather") {
      const int D = cint(op, "D"), K = cint(op, "K");
      const std::string mk = bind(op, 0), x = bind(op, 1), o = bind(op, 2);
      protos.push_back({"gather", {name}, [=](const CompiledPlan& c) {
        const int imk = bi(c, mk), ix = bi(c, x), io = bi(c, o);
        // The pooled heads bind an all-zero marker buffer sized for the plan's batch ('first',
        // src/plan/build.ts:304-310,482): marker 0 of every sequence, the CLS row. It is not read,
        // so a launch with more sequences than the plan's batch (bulk runs) stays in bounds.
        const BufInfo& mb = c.bufs[imk];
        const bool zero_markers =
            !mb.init.empty() && std::all_of(mb.init.begin(), mb.init.end(), [](unsigned char v) { return v == 0; });
        Step s;
        s.run = [=](Exec& ex, cudaStream_t st) {
          if (!zero_markers && ex.bulk) throw PlanError("gather with marker indices has no bulk form");
          launch_gather(f16, ex.buf(ix), ex.buf(io), D, ex.seq,
                        zero_markers ? nullptr : (const uint32_t*)ex.buf(imk), K, st);
        };
        return s;
      }});
      continue;
    }
    if (k == "masklogits") {
      const int K = cint(op, "K");
      const float temp = float(cnum(op, "TEMP"));
      const std::string raw = bind(op, 0), pk = bind(op, 1), o = bind(op, 2);
      touch(o).elem = 4;  // f32 logits whatever the plan's storage type
      protos.push_back({"masklogits", {name}, [=](const CompiledPlan& c) {
        const int ir = bi(c, raw), ip = bi(c, pk), io = bi(c, o);
        Step s;
        s.run = [=](Exec& ex, cudaStream_t st) {
          if (ex.bulk) throw PlanError("marker logits have no bulk form");
          launch_masklogits(f16, ex.buf(ir), (const uint32_t*)ex.buf(ip), (float*)ex.buf(io), K, temp, ex.seq.count,
                            st);
        };
        return s;
      }});
      continue;
    }
    if (k == "im2col") {
      const int N = cint(op, "N"), KS = cint(op, "KS");
      const std::string x = bind(op, 0), m = bind(op, 1), o = bind(op, 2);
      protos.push_back({"im2col", {name}, [=](const CompiledPlan& c) {
        const int ix = bi(c, x), im = bi(c, m), io = bi(c, o);
        Step s;
        s.run = [=](Exec& ex, cudaStream_t st) {
          launch_im2col(f16, ex.buf(ix), (const float*)ex.buf(im), ex.buf(io), N, KS, ex.T, ex.seq, ex.row_seq, st);
        };
        return s;
      }});
      continue;
    }
    throw PlanError("plan op " + name + ": kernel " + k + " outside an attention group has no CUDA computation");
  }

  if (!ops.empty()) tag(last_op);
  // Capture buffers (only read by the copies).
  std::vector<std::vector<std::pair<std::string, int>>> seg_caps;
  if (cp.capturable) {
    for (const Json& seg : plan["segments"].arr) {
      seg_caps.emplace_back();
      if (!seg.has("capture")) continue;
      for (const Json& c : seg["capture"].arr) {
        use(c["buffer"].as_str());
        seg_caps.back().emplace_back(c["buffer"].as_str(), int(c["slot"].as_int()));
      }
    }
    cp.capture_slots = plan.has("captureSlots") ? int(plan["captureSlots"].as_int()) : 0;
    cp.capture_slot_bytes = plan.has("captureSlotBytes") ? plan["captureSlotBytes"].as_int() : 0;
  }
  // Output buffer must exist.
  touch(cp.out_buf);
  // Order buffers deterministically: declaration order.
  for (const Json& d : plan["buffers"].arr) {
    const std::string& id = d["id"].as_str();
    auto it = info.find(id);
    if (it == info.end()) continue;
    BufInfo b = it->second;
    if (b.kind != BufInfo::Fixed && b.cols == 0) {
      // a buffer that is only read: keep the declared size as a fixed buffer
      b.kind = BufInfo::Fixed;
      b.fixed_bytes = size_t(d["bytes"].as_int());
    }
    cp.buf_index[id] = int(cp.bufs.size());
    cp.bufs.push_back(b);
  }
  // scratch of this runtime (not declared by the plan), after the plan's buffers
  for (const auto& kv : info)
    if (kv.first[0] == '#') {
      cp.buf_index[kv.first] = int(cp.bufs.size());
      cp.bufs.push_back(kv.second);
    }
  if (!cp.in_markers.empty() && !cp.buf_index.count(cp.in_markers))
    throw PlanError("plan: the marker input " + cp.in_markers + " is not read");
  if (!cp.rs_dst.empty() && !cp.buf_index.count(cp.rs_dst)) throw PlanError("rowSelect: buffer " + cp.rs_dst + " is not used");
  const BufInfo& ob = cp.bufs[cp.buf_index.at(cp.out_buf)];
  cp.out_per_seq = ob.kind == BufInfo::Seqs;
  cp.tile_q = attention_tile_q(cp.f16);
  // capture_order[0] launches nothing (copies of segments before any launch); entry k + 1 is
  // proto k
  if (cp.capturable) cp.capture_order.emplace_back();
  for (auto& p : protos) {
    Step s = p.make(cp);
    s.label = p.label;
    s.ops = p.names;
    CompiledPlan::CaptureEntry e;
    if (p.cap) {
      e.extra = int(cp.capture_steps.size());
      cp.capture_steps.push_back(std::move(s));
    } else {
      e.step = int(cp.steps.size());
      cp.steps.push_back(std::move(s));
    }
    if (cp.capturable) cp.capture_order.push_back(e);
  }
  if (cp.capturable) {
    // a segment's copies follow its last launch (or the last launch before it)
    for (size_t sgi = 0; sgi < seg_caps.size(); ++sgi) {
      if (seg_caps[sgi].empty()) continue;
      int at = 0;
      for (size_t k = 0; k < protos.size(); ++k)
        if (protos[k].seg <= int(sgi)) at = int(k) + 1;
      for (const auto& bc : seg_caps[sgi]) {
        if (bc.second < 0 || bc.second >= cp.capture_slots) throw PlanError("capture slot outside captureSlots");
        cp.capture_order[size_t(at)].copies.emplace_back(cp.buf_index.at(bc.first), bc.second);
      }
    }
  }
}

void exec_alloc(Exec& ex, Ctx* ctx, const CompiledPlan* cp, int64_t cap_rows, int cap_seqs, bool bulk) {
  ex.ctx = ctx;
  ex.bulk = bulk;
  ex.cp = cp;
  ex.cap_rows = cap_rows;
  ex.cap_seqs = cap_seqs;
  ex.ptr.assign(cp->bufs.size(), nullptr);
  for (size_t i = 0; i < cp->bufs.size(); ++i) {
    const BufInfo& b = cp->bufs[i];
    size_t bytes = 0;
    if (b.kind == BufInfo::Fixed) bytes = std::max(b.fixed_bytes, b.init.size());
    else if (b.kind == BufInfo::Rows) bytes = size_t(cap_rows) * size_t(b.cols) * b.elem;
    else bytes = size_t(cap_seqs) * size_t(b.cols) * b.elem;
    if (!bulk) bytes = std::max(bytes, b.decl_bytes);
    bytes = (bytes + 255) / 256 * 256 + 256;
    void* p = nullptr;
    KH_CUDA(cudaMalloc(&p, bytes));
    KH_CUDA(cudaMemsetAsync(p, 0, bytes, ctx->stream));
    if (!b.init.empty()) KH_CUDA(cudaMemcpyAsync(p, b.init.data(), b.init.size(), cudaMemcpyHostToDevice, ctx->stream));
    ex.owned.push_back(p);
    ex.ptr[i] = p;
    ex.sizes.push_back(bytes);
    ex.bytes += int64_t(bytes);
  }
  const int64_t out_rows = std::max<int64_t>(cp->out_per_seq ? cap_seqs : cap_rows, bulk ? 0 : cp->out_rows);
  ex.out_cap = out_rows * cp->out_cols;
  KH_CUDA(cudaMalloc((void**)&ex.d_out, size_t(ex.out_cap) * 4 + 256));
  ex.owned.push_back(ex.d_out);
  ex.bytes += ex.out_cap * 4;
  KH_CUDA(cudaStreamSynchronize(ctx->stream));
}

// Host sequence table, int32 words: start[S] | len[S] | row_pos[T] | row_seq[T] | tiles[2 ntiles].
void build_seq_table(const std::vector<int32_t>& lens, int tile_q, std::vector<int32_t>& out, SeqTable& offs,
                     int64_t& total_rows) {
  const int S = int(lens.size());
  int64_t T = 0;
  int ntiles = 0, max_len = 0;
  for (int32_t l : lens) {
    T += l;
    ntiles += (l + tile_q - 1) / tile_q;
    max_len = std::max(max_len, int(l));
  }
  const int nptiles = int((T + PACKED_TILE - 1) / PACKED_TILE);
  out.assign(size_t(2 * S + 2 * T + 2 * ntiles + 3 * nptiles), 0);
  int32_t* start = out.data();
  int32_t* len = start + S;
  int32_t* pos = len + S;
  int32_t* rseq = pos + T;
  int32_t* tiles = rseq + T;
  int32_t* ptiles = tiles + 2 * ntiles;
  int64_t r = 0;
  int t = 0;
  for (int s = 0; s < S; ++s) {
    start[s] = int32_t(r);
    len[s] = lens[s];
    for (int i = 0; i < lens[s]; ++i) {
      pos[r + i] = i;
      rseq[r + i] = s;
    }
    for (int q = 0; q < lens[s]; q += tile_q) {
      tiles[2 * t] = s;
      tiles[2 * t + 1] = q;
      ++t;
    }
    r += lens[s];
  }
  // packed tiles: keys of every sequence the tile's 128 rows belong to
  for (int p = 0; p < nptiles; ++p) {
    const int64_t q0 = int64_t(p) * PACKED_TILE;
    const int64_t q1 = std::min<int64_t>(q0 + PACKED_TILE, T) - 1;
    const int s0 = rseq[q0], s1 = rseq[q1];
    ptiles[3 * p] = int32_t(q0);
    ptiles[3 * p + 1] = start[s0];
    ptiles[3 * p + 2] = start[s1] + len[s1];
  }
  // offsets (in words) stored in the pointer fields, rebased by the caller
  offs.start = (const int32_t*)(intptr_t)0;
  offs.len = (const int32_t*)(intptr_t)S;
  offs.row_pos = (const int32_t*)(intptr_t)(2 * S);
  offs.row_seq = (const int32_t*)(intptr_t)(2 * S + T);
  offs.tiles = (const int32_t*)(intptr_t)(2 * S + 2 * T);
  offs.ptiles = (const int32_t*)(intptr_t)(2 * S + 2 * T + 2 * ntiles);
  offs.count = S;
  offs.max_len = max_len;
  offs.ntiles = ntiles;
  offs.nptiles = nptiles;
  total_rows = T;
}

void exec_steps(Exec& ex, cudaStream_t st) {
  for (const Step& s : ex.cp->steps) s.run(ex, st);
}

void exec_capture(Exec& ex, void* dst, cudaStream_t st) {
  const CompiledPlan& cp = *ex.cp;
  if (!cp.capturable) throw PlanError(cp.capture_refusal);
  const size_t slot_bytes = size_t(cp.capture_slot_bytes);
  for (const auto& e : cp.capture_order) {
    if (e.step >= 0) cp.steps[size_t(e.step)].run(ex, st);
    else if (e.extra >= 0) cp.capture_steps[size_t(e.extra)].run(ex, st);
    for (const auto& c : e.copies) {
      // copyBufferToBuffer(buffer, 0, capture, slot * slotBytes, slotBytes)
      const size_t n = std::min(slot_bytes, ex.sizes[size_t(c.first)]);
      KH_CUDA(cudaMemcpyAsync((char*)dst + size_t(c.second) * slot_bytes, ex.buf(c.first), n,
                              cudaMemcpyDeviceToDevice, st));
    }
  }
}

namespace {
template <typename T>
__global__ void to_f32_kernel(const T* src, float* dst, int64_t n);
template <>
__global__ void to_f32_kernel<__half>(const __half* src, float* dst, int64_t n) {
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x)
    dst[i] = __half2float(src[i]);
}
template <>
__global__ void to_f32_kernel<float>(const float* src, float* dst, int64_t n) {
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x)
    dst[i] = src[i];
}
}  // namespace

// Output rows of the last launch -> f32 staging (f16 storage converted, src/half.ts:14-26).
void exec_output(Exec& ex, int rows_out, float* dst, cudaStream_t st) {
  const int64_t n = int64_t(rows_out) * ex.cp->out_cols;
  if (n <= 0) return;
  const void* src = ex.buf(ex.cp->buf_index.at(ex.cp->out_buf));
  int grid = int(std::min<int64_t>((n + 255) / 256, 4096));
  if (ex.cp->f16 && !ex.cp->out_f32) to_f32_kernel<__half><<<grid, 256, 0, st>>>((const __half*)src, dst, n);
  else to_f32_kernel<float><<<grid, 256, 0, st>>>((const float*)src, dst, n);
}

}  // namespace kh
