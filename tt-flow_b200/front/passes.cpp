// Passes of the tensixflow front end on the B200 backend, and the pipeline
// driver shared by the `tfb200-opt` tool and the C ABI (tfb200_opt).
//
//   --tensixflow-fuse-rmsnorm-matmul   FuseMlpPattern (benefit 2) then
//       FuseRmsnormMatmulPattern (benefit 1), single-use guards, eliminated
//       tensors / bytes on each fused op, module tensixflow.fusion_report
//       (tensixflow lib/tensixflow/FuseRmsnormMatmulPass.cpp:60-234)
//   --tensixflow-plan-noc-sharding     B200 plan -> module attributes
//       tensixflow.schedule and tensixflow.emission (PlanNocShardingPass.cpp:135-304)
//   --tensixflow-allocate-circular-buffers   fills the schedule's buffer list
//       (shared-memory rings and TMEM accumulators; AllocateCircularBuffersPass.cpp:63-104)
//   --canonicalize, --tensixflow-canonicalize   identity-add removal: add %x, zero-splat
//       constant (either operand) -> %x, then dead constants dropped
//       (TensixflowOps.cpp hasCanonicalizer pattern, test/Tensixflow/canonicalize.mlir)
//   --tensixflow-to-json               plan JSON instead of IR (tensixflow-translate.cpp:75-222)
//   --tensixflow-device=<name>         device selection (DeviceSelection.cpp:26-49); b200 only
//   --tensixflow-import-ttir           bare-tensor TTIR in (ttir_import.cpp)
//   --tensixflow-emit-cuda=output-dir=<dir>   standalone CUDA project (emit_cuda.cpp;
//       --tensixflow-emit-metalium=output-dir=<dir> is read the same way for the B200)
#include "passes.hpp"

#include <cstdlib>
#include <sstream>

#include "ir.hpp"
#include "emit_cuda.hpp"
#include "plan.hpp"
#include "ttir_import.hpp"

namespace tfb200::front {

namespace {

bool one_use(const Value* v) { return v->users.size() == 1; }

int64_t bytes_of(const Value* v) {
  const int64_t n = v->type.elements();
  const int b = v->type.bytes_per_element();
  return n > 0 ? n * b : 0;
}

Op* insert_before(Module& m, Func& f, Op* anchor, const std::string& name) {
  Op* op = m.new_op(name);
  for (size_t i = 0; i < f.body.size(); ++i)
    if (f.body[i] == anchor) {
      f.body.insert(f.body.begin() + static_cast<long>(i), op);
      return op;
    }
  f.body.push_back(op);
  return op;
}

void set_operands(Op* op, std::initializer_list<Value*> vs) {
  for (Value* v : vs) {
    op->operands.push_back(v);
    v->users.push_back(op);
  }
}

std::string eps_of(const Op* rms) {
  auto it = rms->attrs.find("epsilon");
  return it == rms->attrs.end() ? "" : it->second;
}

bool try_fuse_mlp(Module& m, Func& f, Op* rms) {
  Value* n = rms->result;
  if (!one_use(n)) return false;
  Op* mm1 = n->users[0];
  if (mm1->name != "tensixflow.matmul" || mm1->operands[0] != n) return false;
  Value* m1 = mm1->result;
  if (!one_use(m1)) return false;
  Op* add1 = m1->users[0];
  if (add1->name != "tensixflow.add" || (add1->operands[0] != m1 && add1->operands[1] != m1)) return false;
  Value* b1 = add1->operands[0] == m1 ? add1->operands[1] : add1->operands[0];
  Value* bb = add1->result;
  if (!one_use(bb)) return false;
  Op* gelu = bb->users[0];
  if (gelu->name != "tensixflow.gelu" || gelu->operands[0] != bb) return false;
  Value* g = gelu->result;
  if (!one_use(g)) return false;
  Op* mm2 = g->users[0];
  if (mm2->name != "tensixflow.matmul" || mm2->operands[0] != g) return false;
  Value* m2 = mm2->result;
  if (!one_use(m2)) return false;
  Op* add2 = m2->users[0];
  if (add2->name != "tensixflow.add" || (add2->operands[0] != m2 && add2->operands[1] != m2)) return false;
  Value* res = add2->operands[0] == m2 ? add2->operands[1] : add2->operands[0];
  const int64_t eliminated = bytes_of(n) + bytes_of(m1) + bytes_of(bb) + bytes_of(g) + bytes_of(m2);
  Op* fused = insert_before(m, f, add2, "tensixflow.fused_mlp");
  set_operands(fused, {rms->operands[0], rms->operands[1], mm1->operands[1], b1, mm2->operands[1], res});
  fused->result = m.new_value(add2->result->type);
  fused->result->def = fused;
  if (!eps_of(rms).empty()) fused->attrs["epsilon"] = eps_of(rms);
  fused->attrs["tensixflow.eliminated_tensors"] = i64_attr(5);
  fused->attrs["tensixflow.eliminated_bytes"] = i64_attr(eliminated);
  replace_all_uses(add2->result, fused->result);
  for (Op* dead : {add2, mm2, gelu, add1, mm1, rms}) erase_op(dead);
  return true;
}

bool try_fuse_rms_mm(Module& m, Func& f, Op* rms) {
  Value* n = rms->result;
  if (!one_use(n)) return false;
  Op* mm = n->users[0];
  if (mm->name != "tensixflow.matmul" || mm->operands[0] != n) return false;
  const int64_t eliminated = bytes_of(n);
  Op* fused = insert_before(m, f, mm, "tensixflow.fused_rmsnorm_matmul");
  set_operands(fused, {rms->operands[0], rms->operands[1], mm->operands[1]});
  fused->result = m.new_value(mm->result->type);
  fused->result->def = fused;
  if (!eps_of(rms).empty()) fused->attrs["epsilon"] = eps_of(rms);
  fused->attrs["tensixflow.eliminated_tensors"] = i64_attr(1);
  fused->attrs["tensixflow.eliminated_bytes"] = i64_attr(eliminated);
  replace_all_uses(mm->result, fused->result);
  erase_op(mm);
  erase_op(rms);
  return true;
}

// A splat constant whose value is +0 or -0 ("dense<0.000000e+00> : tensor<...>").
bool zero_splat(const Op* op) {
  if (!op || op->name != "tensixflow.constant") return false;
  const auto it = op->attrs.find("value");
  if (it == op->attrs.end() || it->second.rfind("dense<", 0) != 0) return false;
  const size_t close = it->second.find('>');
  const std::string lit = it->second.substr(6, close == std::string::npos ? std::string::npos : close - 6);
  if (lit.empty() || lit[0] == '[' || lit[0] == '"') return false;  // not a scalar splat
  char* end = nullptr;
  const double v = std::strtod(lit.c_str(), &end);
  return end && *end == '\0' && v == 0.0;
}

// add %x, %zero and add %zero, %x become %x; constants left without users go.
void canonicalize_pass(Module& m) {
  for (Func& f : m.funcs) {
    for (Op* op : f.body) {
      if (op->erased || op->name != "tensixflow.add" || op->operands.size() != 2) continue;
      for (int z = 0; z < 2; ++z) {
        Value* zero = op->operands[z];
        Value* keep = op->operands[1 - z];
        if (zero_splat(zero->def) && keep->type == op->result->type) {
          replace_all_uses(op->result, keep);
          erase_op(op);
          break;
        }
      }
    }
    for (Op* op : f.body)
      if (!op->erased && op->name == "tensixflow.constant" && op->result->users.empty()) erase_op(op);
  }
}

void fuse_pass(Module& m) {
  for (Func& f : m.funcs) {
    // Higher benefit first: a full MLP chain collapses before its head can be
    // taken by the rmsnorm+matmul pattern. Iterate to a fixed point.
    bool changed = true;
    while (changed) {
      changed = false;
      std::vector<Op*> body = f.body;
      for (Op* op : body)
        if (!op->erased && op->name == "tensixflow.rmsnorm" && try_fuse_mlp(m, f, op)) changed = true;
      body = f.body;
      for (Op* op : body)
        if (!op->erased && op->name == "tensixflow.rmsnorm" && try_fuse_rms_mm(m, f, op)) changed = true;
    }
  }
  int64_t fused = 0;
  for (const Func& f : m.funcs)
    for (const Op* op : f.body)
      if (!op->erased && (op->name == "tensixflow.fused_rmsnorm_matmul" || op->name == "tensixflow.fused_mlp")) ++fused;
  m.attrs["tensixflow.fusion_report"] = i64_attr(fused);
}

int64_t rows_of(const TensorType& t) {
  int64_t r = 1;
  for (size_t i = 0; i + 1 < t.shape.size(); ++i) r *= t.shape[i];
  return r;
}

std::string dtype_name(const std::string& e) { return e == "f32" ? "fp32" : e; }

PlanTensor tensor(const std::string& name, const TensorType& t, const std::string& placement) {
  return {name, t.shape, dtype_name(t.elem), placement};
}

// Find the graph to plan in the first function (PlanNocShardingPass.cpp:168-236).
bool discover(const Module& m, PlanRequest* r, std::string* err) {
  if (m.funcs.empty()) {
    *err = "no tensixflow.func to plan";
    return false;
  }
  const Func& f = m.funcs[0];
  r->graph_id = f.name;
  const Op *fmlp = nullptr, *frm = nullptr, *rms = nullptr, *mm = nullptr;
  for (const Op* op : f.body) {
    if (op->erased) continue;
    if (op->name == "tensixflow.fused_mlp" && !fmlp) fmlp = op;
    if (op->name == "tensixflow.fused_rmsnorm_matmul" && !frm) frm = op;
    if (op->name == "tensixflow.rmsnorm" && !rms) rms = op;
    if (op->name == "tensixflow.matmul" && !mm) mm = op;
  }
  auto T = [](const Op* op, size_t k) -> const TensorType& { return op->operands[k]->type; };
  if (fmlp) {
    r->fusion = "fused_mlp";
    r->already_fused = true;
    r->M = rows_of(T(fmlp, 0));
    r->K = T(fmlp, 0).shape.back();
    r->H = T(fmlp, 2).shape.back();
    r->N = T(fmlp, 4).shape.back();
    r->bpe = T(fmlp, 0).bytes_per_element();
    r->tensors = {tensor("input", T(fmlp, 0), "DRAM"), tensor("gamma", T(fmlp, 1), "DRAM"),
                  tensor("w1", T(fmlp, 2), "DRAM"),    tensor("b1", T(fmlp, 3), "DRAM"),
                  tensor("w2", T(fmlp, 4), "DRAM"),    tensor("residual", T(fmlp, 5), "DRAM"),
                  tensor("output", fmlp->result->type, "DRAM")};
    return true;
  }
  const Op* chain_rms = nullptr;
  if (frm) {
    r->fusion = "fused_rmsnorm_matmul";
    r->already_fused = true;
    r->M = rows_of(T(frm, 0));
    r->K = T(frm, 0).shape.back();
    r->N = T(frm, 2).shape.back();
    r->bpe = T(frm, 0).bytes_per_element();
    r->tensors = {tensor("input", T(frm, 0), "DRAM"), tensor("gamma", T(frm, 1), "DRAM"),
                  tensor("weight", T(frm, 2), "DRAM"), tensor("output", frm->result->type, "DRAM")};
    return true;
  }
  if (rms && rms->result->users.size() == 1 && rms->result->users[0]->name == "tensixflow.matmul" &&
      rms->result->users[0]->operands[0] == rms->result)
    chain_rms = rms;
  if (chain_rms) {
    // The planner decides fusion: an rmsnorm -> matmul pair is planned fused.
    const Op* m1 = chain_rms->result->users[0];
    r->fusion = "fused_rmsnorm_matmul";
    r->M = rows_of(T(chain_rms, 0));
    r->K = T(chain_rms, 0).shape.back();
    r->N = T(m1, 1).shape.back();
    r->bpe = T(chain_rms, 0).bytes_per_element();
    r->tensors = {tensor("input", T(chain_rms, 0), "DRAM"), tensor("gamma", T(chain_rms, 1), "DRAM"),
                  tensor("weight", T(m1, 1), "DRAM"), tensor("normalized", chain_rms->result->type, "L1"),
                  tensor("output", m1->result->type, "DRAM")};
    return true;
  }
  if (mm) {
    r->fusion = "none";
    r->M = rows_of(T(mm, 0));
    r->K = T(mm, 0).shape.back();
    r->N = T(mm, 1).shape.back();
    r->bpe = T(mm, 0).bytes_per_element();
    r->tensors = {tensor("lhs", T(mm, 0), "DRAM"), tensor("rhs", T(mm, 1), "DRAM"),
                  tensor("output", mm->result->type, "DRAM")};
    return true;
  }
  *err = "no matmul, fused_rmsnorm_matmul or fused_mlp to plan in @" + f.name;
  return false;
}

std::vector<std::string> split_args(const std::string& s) {
  std::vector<std::string> out;
  std::istringstream is(s);
  std::string a;
  while (is >> a) out.push_back(a);
  return out;
}

}  // namespace

// -verify-diagnostics: the file's "expected-error" annotations must match the
// verifier's diagnostic (line and text), as in mlir-opt.
PipelineResult verify_diagnostics(const std::string& text) {
  PipelineResult res;
  struct Expect {
    int line;
    std::string msg;
  };
  std::vector<Expect> want;
  std::vector<std::string> lines;
  {
    std::istringstream is(text);
    std::string l;
    while (std::getline(is, l)) lines.push_back(l);
  }
  for (size_t i = 0; i < lines.size(); ++i) {
    const std::string& l = lines[i];
    const size_t at = l.find("expected-error");
    if (at == std::string::npos) continue;
    const size_t b = l.find("{{", at), e = l.rfind("}}");
    if (b == std::string::npos || e == std::string::npos || e < b) continue;
    int target = static_cast<int>(i) + 1;
    const size_t sel = l.find('@', at);
    if (sel != std::string::npos && sel < b) {
      const std::string spec = l.substr(sel + 1, b - sel - 1);
      if (spec.rfind("below", 0) == 0) {
        size_t j = i + 1;
        while (j < lines.size() && (lines[j].find_first_not_of(" \t") == std::string::npos ||
                                    lines[j].find("//") == lines[j].find_first_not_of(" \t")))
          ++j;
        target = static_cast<int>(j) + 1;
      } else if (spec.rfind("above", 0) == 0) {
        target = static_cast<int>(i);
      } else {
        target = static_cast<int>(i) + 1 + std::atoi(spec.c_str());
      }
    }
    want.push_back({target, l.substr(b + 2, e - b - 2)});
  }
  std::string err;
  auto m = parse_module(text, &err);
  std::string got;
  int line = 0;
  if (!m) {
    got = err;
    line = std::atoi(err.c_str());
  } else {
    got = verify_module(*m, &line);
  }
  if (want.empty()) {
    res.ok = got.empty();
    res.diag = got.empty() ? "" : "unexpected error: " + got;
    return res;
  }
  if (got.empty()) {
    res.diag = "expected error \"" + want[0].msg + "\" was not produced";
    return res;
  }
  for (const Expect& w : want)
    if (w.line == line && got.find(w.msg) != std::string::npos) {
      res.ok = true;
      return res;
    }
  res.diag = "line " + std::to_string(line) + ": unexpected error: " + got;
  return res;
}

PipelineResult run_pipeline(const std::string& text, const std::vector<std::string>& args) {
  PipelineResult res;
  std::string device = "b200";
  std::vector<std::string> passes;
  bool to_json = false, import_ttir_text = false, emit = false;
  std::string emit_dir;
  for (const std::string& a : args)
    if (a == "-verify-diagnostics" || a == "--verify-diagnostics") return verify_diagnostics(text);
  for (const std::string& a : args) {
    if (a.rfind("--tensixflow-device=", 0) == 0) {
      device = a.substr(20);
    } else if (a == "--tensixflow-import-ttir") {
      import_ttir_text = true;
    } else if (a == "--allow-unregistered-dialect") {
      // the TTIR source parses as generic operations either way
    } else if (a.rfind("--tensixflow-emit-cuda=", 0) == 0 || a.rfind("--tensixflow-emit-metalium=", 0) == 0) {
      // The project of the selected device; for the B200 that is a CUDA project, so the reference's
      // emission flag names it too.
      const std::string opt = a.substr(a.find('=') + 1);
      if (opt.rfind("output-dir=", 0) != 0) {
        res.diag = "error: " + a.substr(0, a.find('=')) + " expects output-dir=<directory>";
        return res;
      }
      emit_dir = opt.substr(11);
      emit = true;
    } else if (a == "--tensixflow-to-json") {
      to_json = true;
    } else if (a == "--tensixflow-fuse-rmsnorm-matmul" || a == "--tensixflow-plan-noc-sharding" ||
               a == "--tensixflow-allocate-circular-buffers" || a == "--canonicalize" ||
               a == "--tensixflow-canonicalize") {
      passes.push_back(a);
    } else {
      res.diag = "unknown option '" + a + "'";
      return res;
    }
  }
  if (device != "b200") {
    res.diag = "unknown device '" + device + "'; valid devices: b200";  // the reference's wording (Scheduler/DeviceSelection.cpp:35)
    return res;
  }
  std::string err;
  auto m = import_ttir_text ? import_ttir(text, &err) : parse_module(text, &err);
  if (!m) {
    res.diag = err;
    return res;
  }
  err = verify_module(*m);
  if (!err.empty()) {
    res.diag = "error: " + err;
    return res;
  }
  B200Plan plan;
  bool planned = false;
  for (const std::string& p : passes) {
    if (p == "--canonicalize" || p == "--tensixflow-canonicalize") {
      canonicalize_pass(*m);
    } else if (p == "--tensixflow-fuse-rmsnorm-matmul") {
      fuse_pass(*m);
    } else if (p == "--tensixflow-plan-noc-sharding") {
      PlanRequest req;
      if (!discover(*m, &req, &err)) {
        res.diag = "error: " + err;
        return res;
      }
      plan = plan_b200(req);
      planned = true;
      m->attrs["tensixflow.schedule"] = schedule_attr(plan, false);
      m->attrs["tensixflow.emission"] = emission_attr(plan);
      m->attrs["tensixflow.device"] = "\"" + device + "\"";
      res.diag += plan_report(plan);
    } else if (p == "--tensixflow-allocate-circular-buffers") {
      if (!planned) {
        res.diag = "error: --tensixflow-allocate-circular-buffers needs a tensixflow.schedule "
                   "(run --tensixflow-plan-noc-sharding first)";
        return res;
      }
      m->attrs["tensixflow.schedule"] = schedule_attr(plan, true);
    }
  }
  err = verify_module(*m);
  if (!err.empty()) {
    res.diag = "error: " + err;
    return res;
  }
  if (emit) {
    if (!planned) {
      res.diag = "error: the module has no tensixflow.emission block; run --tensixflow-plan-noc-sharding before "
                 "--tensixflow-emit-cuda";
      return res;
    }
    if (!emit_cuda_project(*m, plan, emit_dir, &err)) {
      res.diag += "error: " + err;
      return res;
    }
  }
  if (to_json) {
    if (!planned) {
      PlanRequest req;
      if (!discover(*m, &req, &err)) {
        res.diag = "error: " + err;
        return res;
      }
      plan = plan_b200(req);
    }
    res.output = plan_json(plan);
  } else {
    res.output = print_module(*m);
  }
  res.ok = true;
  return res;
}

PipelineResult run_pipeline(const std::string& text, const std::string& args) {
  return run_pipeline(text, split_args(args));
}

}  // namespace tfb200::front
