// Plan report for the B200: validate a plan document against the planner, then
// render it (see report.hpp).
#include "report.hpp"

#include <cstdio>
#include <sstream>
#include <vector>

#include "plan.hpp"
#include "plan_in.hpp"

namespace tfb200::front {

namespace {

const char* const kMappings[] = {"persistent-cta-pair-tiles", "persistent-cta-tiles", "stream-k-swap-ab", "none"};

std::string esc(const std::string& s) {
  std::string o;
  for (char c : s) {
    switch (c) {
      case '&': o += "&amp;"; break;
      case '<': o += "&lt;"; break;
      case '>': o += "&gt;"; break;
      case '"': o += "&quot;"; break;
      default: o += c;
    }
  }
  return o;
}

std::string num(double v) {
  char b[64];
  std::snprintf(b, sizeof(b), "%.4g", v);
  return b;
}

bool read_int(const JVal& v, long long* out) {
  if (v.kind != JVal::kNum) return false;
  try {
    size_t used = 0;
    *out = std::stoll(v.text, &used);
    return used == v.text.size();
  } catch (...) {
    return false;
  }
}

// One emission field of the document against the projection; appends a line
// naming the field when they differ (or the field is missing or mistyped).
void check_int(const JVal& em, const char* key, long long want, std::vector<std::string>* bad) {
  const JVal* v = em.get(key);
  long long got = 0;
  if (!v || !read_int(*v, &got)) {
    bad->push_back(std::string("emission.") + key + ": missing or not an integer (the projection gives " +
                   std::to_string(want) + ")");
  } else if (got != want) {
    bad->push_back(std::string("emission.") + key + ": the plan says " + std::to_string(got) +
                   ", the projection from its tensors gives " + std::to_string(want));
  }
}

std::string item(const std::string& label, const std::string& value) {
  return "      <li class=\"emitted-path item\"><span class=\"k\">" + esc(label) + "</span> <span class=\"v\">" +
         esc(value) + "</span></li>\n";
}

std::string render(const B200Plan& p) {
  const B200Device& d = b200();
  std::ostringstream h;
  h << "<!DOCTYPE html>\n<html lang=\"en\">\n<head>\n<meta charset=\"utf-8\">\n<title>tt-flow plan "
    << esc(p.req.graph_id) << " (b200)</title>\n<style>\n"
    << "body{font-family:system-ui,sans-serif;margin:2em;max-width:60em;color:#222}\n"
    << "h1{font-size:1.4em}h2{font-size:1.1em;border-bottom:1px solid #ccc;margin-top:1.6em}\n"
    << "table{border-collapse:collapse}td,th{border:1px solid #ccc;padding:.2em .6em;text-align:left}\n"
    << "ul.emitted-path{list-style:none;padding:0}.k{display:inline-block;min-width:16em;color:#555}\n"
    << ".bad{color:#a00}\n</style>\n</head>\n<body>\n";
  h << "<h1>Plan " << esc(p.req.graph_id) << " on " << esc(d.name) << " (" << esc(d.arch) << ")</h1>\n";
  h << "<p>Fusion <b>" << esc(p.req.fusion) << "</b>; activation sharding " << esc(p.act) << ", weight strategy "
    << esc(p.weight) << ", intermediates in " << esc(p.storage) << ". Every figure below is a projection of the "
    << "planner, checked against the plan's own emission block.</p>\n";
  h << "<h2>Tensors</h2>\n<table>\n<tr><th>name</th><th>shape</th><th>dtype</th><th>placement</th></tr>\n";
  for (const PlanTensor& t : p.req.tensors) {
    std::string shape;
    for (size_t i = 0; i < t.shape.size(); ++i) shape += (i ? " x " : "") + std::to_string(t.shape[i]);
    h << "<tr><td>" << esc(t.name) << "</td><td>" << esc(shape) << "</td><td>" << esc(t.dtype) << "</td><td>"
      << esc(t.placement) << "</td></tr>\n";
  }
  h << "</table>\n";
  h << "<h2>Projected Emitted Path</h2>\n<ul class=\"emitted-path\">\n";
  h << item("kernel mapping", p.mapping);
  h << item("persistent CTAs", std::to_string(p.ctas) + " of " + std::to_string(d.sms()) + " SMs");
  h << item("work units", std::to_string(p.tiles) + " of " + std::to_string(p.tile_m) + " x " +
                              std::to_string(p.tile_n) + " x " + std::to_string(p.tile_k) + ", at most " +
                              std::to_string(p.max_tiles_per_cta) + " per CTA");
  h << item("shared-memory stages", std::to_string(p.stages) + " (" + std::to_string(p.smem_bytes) + " of " +
                                        std::to_string(d.smem_per_cta) + " bytes)");
  h << item("TMEM columns", std::to_string(p.tmem_columns) + " of " + std::to_string(d.tmem_columns));
  h << item("HBM read bytes", std::to_string(p.dram_read));
  h << item("HBM write bytes", std::to_string(p.dram_write));
  h << item("fused stage tiles", std::to_string(p.fused_stage_tiles));
  h << item("fused_feasible", p.fused_feasible ? "true" : "false (" + p.infeasible_reason + ")");
  h << item("launches", std::to_string(p.launches));
  h << "</ul>\n";
  h << "<h2>Roofline</h2>\n<table>\n";
  h << "<tr><td>FLOPs</td><td>" << p.flops << "</td></tr>\n";
  h << "<tr><td>estimated time</td><td>" << num(p.est_seconds * 1e6) << " us (" << esc(p.bottleneck)
    << "-bound)</td></tr>\n";
  h << "<tr><td>estimated cycles at " << num(d.sm_clock_hz / 1e9) << " GHz</td><td>" << p.est_cycles << "</td></tr>\n";
  h << "<tr><td>tensor-core share of the estimate</td><td>" << num(p.compute_util * 100) << " %</td></tr>\n";
  h << "<tr><td>peaks used</td><td>" << num(d.measured_bf16_flops_per_s / 1e12) << " TFLOP/s bf16, "
    << num(d.measured_hbm_bytes_per_s / 1e9) << " GB/s HBM (measured on B200)</td></tr>\n</table>\n";
  h << "<h2>Shared-memory and TMEM buffers</h2>\n<table>\n<tr><th>index</th><th>depth</th><th>bytes each</th></tr>\n";
  for (const CbSpec& c : p.cbs)
    h << "<tr><td>" << c.index << "</td><td>" << c.depth << "</td><td>" << c.tile_bytes << "</td></tr>\n";
  h << "</table>\n";
  if (!p.suggestions.empty()) {
    h << "<h2>Suggestions</h2>\n<ul>\n";
    for (const std::string& s : p.suggestions) h << "<li>" << esc(s) << "</li>\n";
    h << "</ul>\n";
  }
  h << "</body>\n</html>\n";
  return h.str();
}

}  // namespace

ReportResult report_plan(const std::string& text) {
  ReportResult r;
  JVal root;
  std::string err;
  if (!parse_json(text, &root, &err)) {
    r.diag = err;
    return r;
  }
  if (root.kind != JVal::kObj) {
    r.diag = "plan JSON: the document is not an object";
    return r;
  }
  const JVal* dev = root.get("device");
  const JVal* dname = dev && dev->kind == JVal::kObj ? dev->get("name") : nullptr;
  if (dname && dname->kind == JVal::kStr && dname->text != b200().name) {
    r.diag = "device \"" + dname->text + "\": this report checks plans for b200; re-plan the document for b200 "
             "first (tfb200_plan)";
    return r;
  }
  const JVal* em = root.get("emission");
  if (!em || em->kind != JVal::kObj) {
    r.diag = "plan JSON: no \"emission\" block (plan the module before translating it to JSON)";
    return r;
  }
  const JVal* mp = em->get("mapping");
  if (!mp || mp->kind != JVal::kStr) {
    r.diag = "emission.mapping: missing or not a string";
    return r;
  }
  bool known = false;
  for (const char* m : kMappings) known = known || mp->text == m;
  if (!known) {
    r.diag = "emission.mapping \"" + mp->text +
             "\" is not a kernel mapping of this backend (persistent-cta-pair-tiles, persistent-cta-tiles, "
             "stream-k-swap-ab, none)";
    return r;
  }
  PlanRequest req;
  if (!request_from_plan_json(text, &req, &err)) {
    r.diag = err;
    return r;
  }
  const B200Plan p = plan_b200(req);
  std::vector<std::string> bad;
  if (mp->text != p.mapping)
    bad.push_back("emission.mapping: the plan says \"" + mp->text + "\", the projection from its tensors gives \"" +
                  p.mapping + "\"");
  check_int(*em, "cores_used", p.ctas, &bad);
  check_int(*em, "max_tiles_per_core", p.max_tiles_per_cta, &bad);
  check_int(*em, "dram_read_bytes", p.dram_read, &bad);
  check_int(*em, "dram_write_bytes", p.dram_write, &bad);
  check_int(*em, "fused_stage_tiles", p.fused_stage_tiles, &bad);
  const JVal* ff = em->get("fused_feasible");
  if (!ff || ff->kind != JVal::kBool)
    bad.push_back("emission.fused_feasible: missing or not a boolean");
  else if (ff->b != p.fused_feasible)
    bad.push_back(std::string("emission.fused_feasible: the plan says ") + (ff->b ? "true" : "false") +
                  ", the projection gives " + (p.fused_feasible ? "true" : "false"));
  if (!bad.empty()) {
    r.diag = "the plan's emission block disagrees with the projection (a stale or edited plan):";
    for (const std::string& b : bad) r.diag += "\n  " + b;
    return r;
  }
  r.html = render(p);
  r.ok = true;
  return r;
}

}  // namespace tfb200::front
