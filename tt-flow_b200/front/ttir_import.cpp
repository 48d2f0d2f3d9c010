// --tensixflow-import-ttir: bare-tensor TTIR (one func.func of generic
// "ttir.*" operations, as tt-mlir writes it) to the tensixflow dialect, so the
// fusion and planning passes run unchanged on it (tensixflow
// lib/tensixflow/Import/ImportTTIR.cpp and its lit tests
// test/Tensixflow/import_ttir.mlir, import_ttir_negative.mlir).
//
// Import subset: ttir.matmul (no transposes) -> tensixflow.matmul,
// ttir.add -> tensixflow.add, ttir.gelu -> tensixflow.gelu, ttir.rms_norm
// (input and weight, normalized_shape = the last dimension) ->
// tensixflow.rmsnorm {epsilon}. Static shapes, bf16 or f32, no layout
// encodings, no ttcore / ttnn module attributes, exactly one function, rank-1
// arguments only as the rms_norm weight. Every rejection names the construct;
// the diagnostic texts are the reference's (its lit tests check them).
#include "ttir_import.hpp"

#include <cctype>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <set>

namespace tfb200::front {

namespace {

const char* kAccepts =
    "; the importer accepts ttir.matmul, ttir.add, ttir.gelu, and ttir.rms_norm (docs/ttir.md)";

struct Src {
  const std::string& s;
  size_t i = 0;
  std::string err;
  explicit Src(const std::string& t) : s(t) {}

  int line_at(size_t pos) const {
    int line = 1;
    for (size_t k = 0; k < pos && k < s.size(); ++k) line += s[k] == '\n';
    return line;
  }
  bool fail(const std::string& msg, size_t pos) {
    if (err.empty()) {
      int col = 1;
      for (size_t k = pos; k > 0 && s[k - 1] != '\n'; --k) ++col;
      err = std::to_string(line_at(pos)) + ":" + std::to_string(col) + ": error: " + msg;
    }
    return false;
  }
  bool fail(const std::string& msg) { return fail(msg, i); }
  void skip() {
    while (i < s.size()) {
      if (std::isspace(static_cast<unsigned char>(s[i]))) {
        ++i;
      } else if (s.compare(i, 2, "//") == 0) {
        while (i < s.size() && s[i] != '\n') ++i;
      } else {
        break;
      }
    }
  }
  bool peek(const char* t) {
    skip();
    return s.compare(i, std::char_traits<char>::length(t), t) == 0;
  }
  bool accept(const char* t) {
    if (!peek(t)) return false;
    i += std::char_traits<char>::length(t);
    return true;
  }
  bool expect(const char* t) { return accept(t) || fail(std::string("expected '") + t + "'"); }
  std::string ident() {
    skip();
    const size_t b = i;
    while (i < s.size() && (std::isalnum(static_cast<unsigned char>(s[i])) || s[i] == '_' || s[i] == '.' ||
                            s[i] == '$' || s[i] == '-'))
      ++i;
    return s.substr(b, i - b);
  }
  // Balanced text from the current position up to the matching `close` (the
  // opener already consumed); returns the inner text and moves past `close`.
  std::string balanced(char open, char close) {
    const size_t b = i;
    int depth = 1;
    while (i < s.size()) {
      const char c = s[i];
      if (c == '"') {
        ++i;
        while (i < s.size() && s[i] != '"') i += s[i] == '\\' ? 2 : 1;
        ++i;
        continue;
      }
      if (c == open) {
        ++depth;
      } else if (c == close && --depth == 0) {
        ++i;
        return s.substr(b, i - 1 - b);
      }
      ++i;
    }
    fail("unbalanced '" + std::string(1, open) + "'", b);
    return s.substr(b);
  }
};

// A tensor type as written, with attribute aliases (#name) expanded.
struct RawType {
  std::string text;   // printed form
  TensorType t;
  bool encoded = false;
  size_t pos = 0;
};

std::string expand_aliases(const std::string& text, const std::map<std::string, std::string>& aliases) {
  std::string out;
  for (size_t k = 0; k < text.size();) {
    if (text[k] == '#') {
      size_t e = k + 1;
      while (e < text.size() && (std::isalnum(static_cast<unsigned char>(text[e])) || text[e] == '_' ||
                                 text[e] == '.'))
        ++e;
      auto it = aliases.find(text.substr(k + 1, e - k - 1));
      if (it != aliases.end() && (e >= text.size() || text[e] != '<')) {
        out += it->second;
        k = e;
        continue;
      }
    }
    out += text[k++];
  }
  return out;
}

bool parse_raw_type(Src& c, const std::map<std::string, std::string>& aliases, RawType* r) {
  c.skip();
  r->pos = c.i;
  if (!c.accept("tensor<")) return c.fail("expected a tensor type");
  const std::string inner = c.balanced('<', '>');
  if (!c.err.empty()) return false;
  r->text = "tensor<" + expand_aliases(inner, aliases) + ">";
  // shape x ... x elem [, encoding]
  size_t k = 0;
  r->t = TensorType{};
  while (k < inner.size()) {
    size_t b = k;
    if (inner[k] == '?') {
      ++k;
      if (k < inner.size() && inner[k] == 'x') {
        r->t.shape.push_back(-1);
        ++k;
        continue;
      }
      k = b;
      break;
    }
    while (k < inner.size() && std::isdigit(static_cast<unsigned char>(inner[k]))) ++k;
    if (k > b && k < inner.size() && inner[k] == 'x') {
      r->t.shape.push_back(std::stoll(inner.substr(b, k - b)));
      ++k;
      continue;
    }
    k = b;
    break;
  }
  size_t e = k;
  while (e < inner.size() && inner[e] != ',' && inner[e] != '>') ++e;
  r->t.elem = inner.substr(k, e - k);
  while (!r->t.elem.empty() && std::isspace(static_cast<unsigned char>(r->t.elem.back()))) r->t.elem.pop_back();
  r->encoded = e < inner.size() && inner[e] == ',';
  return true;
}

// An f32 attribute value in the form the reference prints for an imported
// epsilon: the 7-digit scientific form when it reads back as the same value
// (widened to double), else nine significant digits, truncated, as d.ddddddddE-x.
std::string f32_attr_text(float v) {
  char buf[64];
  std::snprintf(buf, sizeof(buf), "%.6e", static_cast<double>(v));
  if (std::strtod(buf, nullptr) == static_cast<double>(v)) return buf;
  if (v == 0.0f || !std::isfinite(v)) return buf;
  // 21 significant digits of |v| (exact enough to truncate nine from), d.ddd...e[+-]xx.
  std::snprintf(buf, sizeof(buf), "%.20e", std::fabs(static_cast<double>(v)));
  const char* ep = std::strchr(buf, 'e');
  const int e10 = std::atoi(ep + 1);
  std::string digits;
  for (const char* p = buf; p < ep && digits.size() < 9; ++p)
    if (std::isdigit(static_cast<unsigned char>(*p))) digits.push_back(*p);
  while (digits.size() > 1 && digits.back() == '0') digits.pop_back();
  std::string out = v < 0 ? "-" : "";
  out += digits.substr(0, 1) + "." + (digits.size() > 1 ? digits.substr(1) : "0") + "E" + std::to_string(e10);
  return out;
}

struct GenericOp {
  std::string result;  // without '%'
  std::string name;
  std::vector<std::string> operands;
  std::string props;  // inside <{ ... }>
  std::string attrs;  // inside { ... }
  std::vector<RawType> in_types, out_types;
  size_t pos = 0;
};

// key = value pairs of a properties / attribute dictionary (top-level commas).
std::map<std::string, std::string> dict_entries(const std::string& d) {
  std::map<std::string, std::string> out;
  size_t k = 0;
  while (k < d.size()) {
    while (k < d.size() && (std::isspace(static_cast<unsigned char>(d[k])) || d[k] == ',')) ++k;
    size_t b = k;
    while (k < d.size() && d[k] != '=' && d[k] != ',') ++k;
    std::string key = d.substr(b, k - b);
    while (!key.empty() && std::isspace(static_cast<unsigned char>(key.back()))) key.pop_back();
    std::string val = "unit";
    if (k < d.size() && d[k] == '=') {
      ++k;
      int depth = 0;
      b = k;
      while (k < d.size()) {
        const char c = d[k];
        if (c == '<' || c == '[' || c == '(' || c == '{') ++depth;
        if (c == '>' || c == ']' || c == ')' || c == '}') --depth;
        if (c == ',' && depth == 0) break;
        ++k;
      }
      val = d.substr(b, k - b);
      while (!val.empty() && std::isspace(static_cast<unsigned char>(val.front()))) val.erase(val.begin());
      while (!val.empty() && std::isspace(static_cast<unsigned char>(val.back()))) val.pop_back();
    }
    if (!key.empty()) out[key] = val;
  }
  return out;
}

std::vector<int64_t> i64_array(const std::string& v, bool* ok) {
  // array<i64: 4, 8>
  std::vector<int64_t> out;
  *ok = false;
  const size_t c = v.find(':');
  if (v.rfind("array<i64", 0) != 0 || c == std::string::npos) return out;
  std::string body = v.substr(c + 1);
  if (!body.empty() && body.back() == '>') body.pop_back();
  size_t k = 0;
  while (k < body.size()) {
    while (k < body.size() && (body[k] == ',' || std::isspace(static_cast<unsigned char>(body[k])))) ++k;
    if (k >= body.size()) break;
    char* end = nullptr;
    out.push_back(std::strtoll(body.c_str() + k, &end, 10));
    if (end == body.c_str() + k) return out;
    k = static_cast<size_t>(end - body.c_str());
  }
  *ok = true;
  return out;
}

bool check_type(Src& c, const RawType& r, const std::string& what) {
  if (r.encoded)
    return c.fail(what + " is layout-encoded: '" + r.text +
                      "'; layout-encoded tensors are outside the import subset because this build does not link "
                      "the ttcore or ttnn dialects (docs/ttir.md)",
                  r.pos);
  for (int64_t d : r.t.shape)
    if (d < 0)
      return c.fail(what + " has a dynamic shape: '" + r.text +
                        "'; the import subset requires static shapes (docs/ttir.md)",
                    r.pos);
  if (r.t.elem != "bf16" && r.t.elem != "f32")
    return c.fail(what + " has element type '" + r.t.elem +
                      "'; the import subset accepts bf16 and f32 only (docs/ttir.md)",
                  r.pos);
  return true;
}

}  // namespace

std::unique_ptr<Module> import_ttir(const std::string& text, std::string* err) {
  Src c(text);
  std::map<std::string, std::string> aliases;
  auto m = std::make_unique<Module>();

  // Top level: attribute aliases, an optional module wrapper, func.func bodies.
  int nfuncs = 0;
  for (size_t k = text.find("func.func"); k != std::string::npos; k = text.find("func.func", k + 9)) {
    size_t ls = text.rfind('\n', k);
    ls = ls == std::string::npos ? 0 : ls + 1;
    const size_t cm = text.find("//", ls);
    if (cm == std::string::npos || cm > k) ++nfuncs;
  }
  bool wrapped = false;
  while (true) {
    c.skip();
    if (c.i >= text.size()) break;
    if (text[c.i] == '#') {
      ++c.i;
      const std::string name = c.ident();
      if (!c.expect("=")) break;
      c.skip();
      const size_t b = c.i;
      while (c.i < text.size() && text[c.i] != '\n') ++c.i;
      std::string v = text.substr(b, c.i - b);
      while (!v.empty() && std::isspace(static_cast<unsigned char>(v.back()))) v.pop_back();
      aliases[name] = v;
      continue;
    }
    break;
  }
  if (c.err.empty() && c.accept("module")) {
    wrapped = true;
    if (c.accept("attributes")) {
      if (!c.expect("{")) goto done;
      const size_t at = c.i;
      const std::string body = c.balanced('{', '}');
      for (const auto& kv : dict_entries(body)) {
        std::string key = kv.first;
        if (!key.empty() && key.front() == '"') key = key.substr(1, key.size() - 2);
        if (key.rfind("ttcore.", 0) == 0 || key.rfind("ttnn.", 0) == 0) {
          c.fail("module attribute '" + key +
                     "' is outside the import subset; device and layout attributes from the ttcore or ttnn "
                     "dialects are rejected because this build does not link them (docs/ttir.md)",
                 at);
          goto done;
        }
        m->attrs[key] = kv.second;
      }
    }
    if (!c.expect("{")) goto done;
  }
  if (nfuncs != 1) {
    c.fail("expected exactly one func.func in the module, found " + std::to_string(nfuncs) +
               "; multiple functions are outside the import subset (docs/ttir.md)",
           c.i);
    goto done;
  }
  {
    if (!c.expect("func.func")) goto done;
    c.skip();
    if (!c.expect("@")) goto done;
    Func f;
    f.name = c.ident();
    if (!c.expect("(")) goto done;
    std::map<std::string, Value*> names;
    std::vector<RawType> arg_types;
    if (!c.accept(")")) {
      while (true) {
        if (!c.expect("%")) goto done;
        const std::string an = c.ident();
        if (!c.expect(":")) goto done;
        RawType rt;
        if (!parse_raw_type(c, aliases, &rt)) goto done;
        if (c.peek("{")) {
          ++c.i;
          c.balanced('{', '}');
        }
        Value* v = m->new_value(rt.t);
        v->arg_index = static_cast<int>(f.args.size());
        v->src_name = an;
        f.args.push_back(v);
        names[an] = v;
        arg_types.push_back(rt);
        if (c.accept(",")) continue;
        if (!c.expect(")")) goto done;
        break;
      }
    }
    for (size_t a = 0; a < arg_types.size(); ++a)
      if (!check_type(c, arg_types[a], "function argument " + std::to_string(a))) goto done;
    if (c.accept("->")) {
      const bool paren = c.accept("(");
      while (true) {
        RawType rt;
        if (!parse_raw_type(c, aliases, &rt)) goto done;
        if (!check_type(c, rt, "function result " + std::to_string(f.results.size()))) goto done;
        f.results.push_back(rt.t);
        if (paren && c.accept(",")) continue;
        if (paren && !c.expect(")")) goto done;
        break;
      }
    }
    if (c.accept("attributes")) {
      if (!c.expect("{")) goto done;
      c.balanced('{', '}');
    }
    if (!c.expect("{")) goto done;
    std::set<const Value*> rms_weights;
    std::map<const Value*, int> uses;
    while (true) {
      c.skip();
      if (c.accept("}")) break;
      const size_t op_pos = c.i;
      if (c.accept("return") || c.accept("func.return")) {
        Op* ret = m->new_op("tensixflow.return");
        ret->line = c.line_at(op_pos);
        c.skip();
        if (c.peek("%")) {
          while (true) {
            if (!c.expect("%")) goto done;
            const std::string n = c.ident();
            auto it = names.find(n);
            if (it == names.end()) {
              c.fail("use of undefined value '%" + n + "'");
              goto done;
            }
            ret->operands.push_back(it->second);
            it->second->users.push_back(ret);
            ++uses[it->second];
            if (!c.accept(",")) break;
          }
          if (!c.expect(":")) goto done;
          for (size_t k = 0; k < ret->operands.size(); ++k) {
            RawType rt;
            if (!parse_raw_type(c, aliases, &rt)) goto done;
            if (k + 1 < ret->operands.size() && !c.expect(",")) goto done;
          }
        }
        f.body.push_back(ret);
        continue;
      }
      GenericOp g;
      g.pos = op_pos;
      if (c.accept("%")) {
        g.result = c.ident();
        if (!c.expect("=")) goto done;
      }
      c.skip();
      if (!c.accept("\"")) {
        const std::string nm = c.ident();
        c.fail("operation '" + nm + "' is outside the import subset" + kAccepts, op_pos);
        goto done;
      }
      {
        const size_t b = c.i;
        while (c.i < text.size() && text[c.i] != '"') ++c.i;
        g.name = text.substr(b, c.i - b);
        ++c.i;
      }
      static const std::set<std::string> subset = {"ttir.matmul", "ttir.add", "ttir.gelu", "ttir.rms_norm"};
      if (!subset.count(g.name)) {
        c.fail("operation '" + g.name + "' is outside the import subset" + kAccepts, op_pos);
        goto done;
      }
      if (!c.expect("(")) goto done;
      if (!c.accept(")")) {
        while (true) {
          if (!c.expect("%")) goto done;
          g.operands.push_back(c.ident());
          if (c.accept(",")) continue;
          if (!c.expect(")")) goto done;
          break;
        }
      }
      if (c.accept("<{")) {
        g.props = c.balanced('{', '}');
        if (!c.expect(">")) goto done;
      }
      if (c.accept("{")) g.attrs = c.balanced('{', '}');
      if (!c.expect(":") || !c.expect("(")) goto done;
      if (!c.accept(")")) {
        while (true) {
          RawType rt;
          if (!parse_raw_type(c, aliases, &rt)) goto done;
          g.in_types.push_back(rt);
          if (c.accept(",")) continue;
          if (!c.expect(")")) goto done;
          break;
        }
      }
      if (!c.expect("->")) goto done;
      {
        RawType rt;
        if (!parse_raw_type(c, aliases, &rt)) goto done;
        if (!check_type(c, rt, "'" + g.name + "' result")) goto done;
        g.out_types.push_back(rt);
      }
      std::map<std::string, std::string> props = dict_entries(g.props);
      for (const auto& kv : dict_entries(g.attrs)) props[kv.first] = kv.second;
      std::string tname;
      size_t want = 2;
      if (g.name == "ttir.matmul") {
        tname = "tensixflow.matmul";
        for (const char* tr : {"transpose_a", "transpose_b"}) {
          auto it = props.find(tr);
          if (it != props.end() && it->second != "false") {
            c.fail("'ttir.matmul' attribute '" + std::string(tr) + " = " + it->second +
                       "' is outside the import subset; only untransposed operands are imported (docs/ttir.md)",
                   op_pos);
            goto done;
          }
        }
      } else if (g.name == "ttir.add") {
        tname = "tensixflow.add";
      } else if (g.name == "ttir.gelu") {
        tname = "tensixflow.gelu";
        want = 1;
      } else {
        tname = "tensixflow.rmsnorm";
        if (g.operands.size() == 3) {
          c.fail("'ttir.rms_norm' with a bias operand is outside the import subset; only the input and weight "
                 "operands are imported (docs/ttir.md)",
                 op_pos);
          goto done;
        }
      }
      if (g.operands.size() != want) {
        c.fail("'" + g.name + "' expects " + std::to_string(want) + " operands, found " +
                   std::to_string(g.operands.size()),
               op_pos);
        goto done;
      }
      Op* op = m->new_op(tname);
      op->line = c.line_at(op_pos);
      for (const std::string& on : g.operands) {
        auto it = names.find(on);
        if (it == names.end()) {
          c.fail("use of undefined value '%" + on + "'", op_pos);
          goto done;
        }
        op->operands.push_back(it->second);
        it->second->users.push_back(op);
        ++uses[it->second];
      }
      if (tname == "tensixflow.rmsnorm") {
        const TensorType& xt = op->operands[0]->type;
        auto ns = props.find("normalized_shape");
        if (ns != props.end()) {
          bool ok = false;
          const std::vector<int64_t> dims = i64_array(ns->second, &ok);
          const int64_t last = xt.shape.empty() ? -1 : xt.shape.back();
          if (!ok || dims.size() != 1 || dims[0] != last) {
            c.fail("'ttir.rms_norm' normalized_shape " + ns->second +
                       " is outside the import subset; tensixflow normalizes the last dimension (" +
                       std::to_string(last) + ") only (docs/ttir.md)",
                   op_pos);
            goto done;
          }
        }
        auto ep = props.find("epsilon");
        if (ep != props.end()) {
          const float eps = std::strtof(ep->second.c_str(), nullptr);
          op->attrs["epsilon"] = f32_attr_text(eps) + " : f32";
        }
        rms_weights.insert(op->operands[1]);
      }
      op->result = m->new_value(g.out_types[0].t);
      op->result->def = op;
      op->result->src_name = g.result;
      names[g.result] = op->result;
      f.body.push_back(op);
    }
    // Rank-1 arguments only as the rms_norm weight.
    for (size_t a = 0; a < f.args.size(); ++a) {
      const Value* v = f.args[a];
      if (v->type.shape.size() == 1) {
        bool only_weight = !v->users.empty();
        for (const Op* u : v->users)
          if (u->name != "tensixflow.rmsnorm" || u->operands.size() < 2 || u->operands[1] != v ||
              u->operands[0] == v)
            only_weight = false;
        if (!only_weight) {
          c.fail("function argument " + std::to_string(a) + " has rank 1: '" + arg_types[a].text +
                     "'; rank-1 tensors are outside the import subset except the ttir.rms_norm weight "
                     "(docs/ttir.md)",
                 arg_types[a].pos);
          goto done;
        }
      }
    }
    if (f.body.empty() || f.body.back()->name != "tensixflow.return") {
      c.fail("the function has no return");
      goto done;
    }
    m->funcs.push_back(std::move(f));
    if (wrapped) c.expect("}");
  }
done:
  if (!c.err.empty()) {
    *err = c.err;
    return nullptr;
  }
  return m;
}

}  // namespace tfb200::front
