// Parser, printer and verifier of the tensixflow dialect subset (see ir.hpp).
#include "ir.hpp"

#include <algorithm>
#include <cctype>
#include <cstdio>
#include <cstdlib>
#include <sstream>

namespace tfb200::front {

int64_t TensorType::elements() const {
  int64_t n = 1;
  for (int64_t d : shape) {
    if (d < 0) return -1;
    n *= d;
  }
  return n;
}

int TensorType::bytes_per_element() const {
  if (elem == "bf16" || elem == "f16") return 2;
  if (elem == "f32" || elem == "i32") return 4;
  if (elem == "f64" || elem == "i64") return 8;
  if (elem == "i8" || elem == "f8E4M3FN" || elem == "f8E5M2") return 1;
  return 0;
}

std::string TensorType::str() const {
  if (!ranked) return "tensor<*x" + elem + ">";
  std::string s = "tensor<";
  for (int64_t d : shape) s += (d < 0 ? std::string("?") : std::to_string(d)) + "x";
  return s + elem + ">";
}

Value* Module::new_value(const TensorType& t) {
  values.push_back(std::make_unique<Value>());
  values.back()->type = t;
  return values.back().get();
}

Op* Module::new_op(const std::string& name) {
  ops.push_back(std::make_unique<Op>());
  ops.back()->name = name;
  return ops.back().get();
}

std::string i64_attr(int64_t v) { return std::to_string(v) + " : i64"; }

void erase_op(Op* op) {
  op->erased = true;
  for (Value* v : op->operands) {
    auto& u = v->users;
    auto it = std::find(u.begin(), u.end(), op);
    if (it != u.end()) u.erase(it);
  }
}

void replace_all_uses(Value* from, Value* to) {
  for (Op* u : from->users) {
    for (Value*& o : u->operands)
      if (o == from) o = to;
    to->users.push_back(u);
  }
  from->users.clear();
}

// ------------------------------------------------------------------- parsing

namespace {

struct Cursor {
  const std::string& s;
  size_t i = 0;
  std::string err;

  explicit Cursor(const std::string& text) : s(text) {}

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
  bool eof() {
    skip();
    return i >= s.size();
  }
  bool peek(const std::string& t) {
    skip();
    return s.compare(i, t.size(), t) == 0;
  }
  bool accept(const std::string& t) {
    if (peek(t)) {
      i += t.size();
      return true;
    }
    return false;
  }
  bool expect(const std::string& t) {
    if (accept(t)) return true;
    fail("expected '" + t + "'");
    return false;
  }
  void fail(const std::string& msg) {
    if (!err.empty()) return;
    size_t line = 1, col = 1;
    for (size_t k = 0; k < i && k < s.size(); ++k) {
      if (s[k] == '\n') {
        ++line;
        col = 1;
      } else {
        ++col;
      }
    }
    err = std::to_string(line) + ":" + std::to_string(col) + ": error: " + msg;
  }
  std::string ident() {
    skip();
    size_t b = i;
    while (i < s.size() && (std::isalnum(static_cast<unsigned char>(s[i])) || s[i] == '_' || s[i] == '.' ||
                            s[i] == '$' || s[i] == '-'))
      ++i;
    return s.substr(b, i - b);
  }
  // Raw text of one attribute value: up to a top-level ',' or '}' / ')'.
  std::string raw_value() {
    skip();
    size_t b = i;
    int depth = 0;
    while (i < s.size()) {
      const char c = s[i];
      if (c == '"') {
        ++i;
        while (i < s.size() && s[i] != '"') i += (s[i] == '\\') ? 2 : 1;
        ++i;
        continue;
      }
      if (c == '<' || c == '(' || c == '[' || c == '{') ++depth;
      if (c == '>' || c == ')' || c == ']' || c == '}') {
        if (depth == 0) break;
        --depth;
      }
      if (c == ',' && depth == 0) break;
      if (c == '-' && i + 1 < s.size() && s[i + 1] == '>' && depth > 0) {  // '->' inside a nested type
        i += 2;
        continue;
      }
      ++i;
    }
    std::string v = s.substr(b, i - b);
    while (!v.empty() && std::isspace(static_cast<unsigned char>(v.back()))) v.pop_back();
    return v;
  }
};

// A splat float literal prints the way MLIR's printer writes it ("%.6e" when
// that round-trips), e.g. dense<1.0> -> dense<1.000000e+00>.
std::string normalize_dense(const std::string& value, const TensorType& t) {
  if (value.rfind("dense<", 0) != 0 || (t.elem != "f32" && t.elem != "f16" && t.elem != "bf16" && t.elem != "f64"))
    return value;
  const size_t close = value.find('>');
  if (close == std::string::npos) return value;
  const std::string lit = value.substr(6, close - 6);
  char* end = nullptr;
  const double v = std::strtod(lit.c_str(), &end);
  if (lit.empty() || end != lit.c_str() + lit.size()) return value;
  char buf[64];
  std::snprintf(buf, sizeof(buf), "%.6e", v);
  if (std::strtod(buf, nullptr) != v) std::snprintf(buf, sizeof(buf), "%.17g", v);
  return "dense<" + std::string(buf) + value.substr(close);
}

bool parse_type(Cursor& c, TensorType* t) {
  if (!c.expect("tensor<")) return false;
  c.skip();
  t->shape.clear();
  if (c.accept("*x")) {
    t->ranked = false;
  }
  while (true) {
    c.skip();
    size_t b = c.i;
    if (c.i < c.s.size() && c.s[c.i] == '?') {
      ++c.i;
      if (c.i < c.s.size() && c.s[c.i] == 'x') {
        ++c.i;
        t->shape.push_back(-1);
        continue;
      }
      c.fail("bad dimension");
      return false;
    }
    while (c.i < c.s.size() && std::isdigit(static_cast<unsigned char>(c.s[c.i]))) ++c.i;
    if (c.i > b && c.i < c.s.size() && c.s[c.i] == 'x') {
      t->shape.push_back(std::stoll(c.s.substr(b, c.i - b)));
      ++c.i;
      continue;
    }
    c.i = b;
    break;
  }
  size_t b = c.i;
  while (c.i < c.s.size() && c.s[c.i] != '>' && c.s[c.i] != ',') ++c.i;
  t->elem = c.s.substr(b, c.i - b);
  if (c.accept(",")) {  // encoding attribute: skip it
    int depth = 0;
    while (c.i < c.s.size() && !(c.s[c.i] == '>' && depth == 0)) {
      if (c.s[c.i] == '<') ++depth;
      if (c.s[c.i] == '>') --depth;
      ++c.i;
    }
  }
  if (t->elem.empty()) {
    c.fail("missing element type");
    return false;
  }
  return c.expect(">");
}

bool parse_attr_dict(Cursor& c, std::map<std::string, std::string>* attrs) {
  if (!c.accept("{")) return true;
  if (c.accept("}")) return true;
  while (true) {
    std::string key;
    c.skip();
    if (c.peek("\"")) {
      ++c.i;
      size_t b = c.i;
      while (c.i < c.s.size() && c.s[c.i] != '"') ++c.i;
      key = c.s.substr(b, c.i - b);
      ++c.i;
    } else {
      key = c.ident();
    }
    if (key.empty()) {
      c.fail("expected attribute name");
      return false;
    }
    std::string val = "unit";
    if (c.accept("=")) val = c.raw_value();
    (*attrs)[key] = val;
    if (c.accept(",")) continue;
    return c.expect("}");
  }
}

struct Scope {
  std::map<std::string, Value*> names;
};

Value* use(Cursor& c, Scope& sc) {
  c.skip();
  if (!c.accept("%")) {
    c.fail("expected an SSA value");
    return nullptr;
  }
  std::string n = c.ident();
  auto it = sc.names.find(n);
  if (it == sc.names.end()) {
    c.fail("use of undefined value '%" + n + "'");
    return nullptr;
  }
  return it->second;
}

bool parse_op(Cursor& c, Module& m, Func& f, Scope& sc) {
  std::string res_name;
  if (c.accept("%")) {
    res_name = c.ident();
    if (!c.expect("=")) return false;
  }
  c.skip();
  if (c.peek("\"")) {
    c.fail("generic operation form is not supported");
    return false;
  }
  size_t line = 1;
  for (size_t k = 0; k < c.i && k < c.s.size(); ++k) line += c.s[k] == '\n';
  std::string name = c.ident();
  static const char* known[] = {"tensixflow.return",  "tensixflow.constant", "tensixflow.add",
                                "tensixflow.gelu",    "tensixflow.matmul",   "tensixflow.rmsnorm",
                                "tensixflow.fused_rmsnorm_matmul", "tensixflow.fused_mlp"};
  if (std::find(std::begin(known), std::end(known), name) == std::end(known)) {
    c.fail("unsupported operation '" + name + "'");
    return false;
  }
  Op* op = m.new_op(name);
  op->line = static_cast<int>(line);
  if (name == "tensixflow.return") {
    if (!c.peek("}") && c.peek("%")) {
      while (true) {
        Value* v = use(c, sc);
        if (!v) return false;
        op->operands.push_back(v);
        if (!c.accept(",")) break;
      }
      if (!parse_attr_dict(c, &op->attrs)) return false;
      if (!c.expect(":")) return false;
      for (size_t k = 0; k < op->operands.size(); ++k) {
        TensorType t;
        if (!parse_type(c, &t)) return false;
        if (k + 1 < op->operands.size() && !c.expect(",")) return false;
      }
    }
    for (Value* v : op->operands) v->users.push_back(op);
    f.body.push_back(op);
    return true;
  }
  if (name == "tensixflow.constant") {
    // The value attribute carries its type: "dense<...> : tensor<...>".
    c.skip();
    const size_t b = c.i;
    int depth = 0;
    while (c.i < c.s.size()) {
      const char ch = c.s[c.i];
      if (ch == '<' || ch == '[' || ch == '(') ++depth;
      if (ch == '>' || ch == ']' || ch == ')') {
        --depth;
        if (depth == 0) {
          ++c.i;
          break;
        }
      }
      ++c.i;
    }
    const std::string literal = c.s.substr(b, c.i - b);
    if (!c.expect(":")) return false;
    TensorType t;
    if (!parse_type(c, &t)) return false;
    const std::string value = literal + " : " + t.str();
    op->attrs["value"] = normalize_dense(value, t);
    if (!parse_attr_dict(c, &op->attrs)) return false;
    op->result = m.new_value(t);
    op->result->def = op;
    op->result->src_name = res_name;
    sc.names[res_name] = op->result;
    f.body.push_back(op);
    return true;
  }
  size_t nin = name == "tensixflow.gelu" ? 1
               : name == "tensixflow.fused_rmsnorm_matmul" ? 3
               : name == "tensixflow.fused_mlp"            ? 6
                                                           : 2;
  for (size_t k = 0; k < nin; ++k) {
    Value* v = use(c, sc);
    if (!v) return false;
    op->operands.push_back(v);
    if (k + 1 < nin && !c.expect(",")) return false;
  }
  if (!parse_attr_dict(c, &op->attrs)) return false;
  if (!c.expect(":")) return false;
  std::vector<TensorType> tys;
  TensorType t;
  TensorType rt;
  if (name == "tensixflow.add" || name == "tensixflow.gelu") {
    if (!parse_type(c, &t)) return false;
    tys.assign(nin, t);
    rt = t;
  } else if (name == "tensixflow.matmul") {
    TensorType a, b;
    if (!parse_type(c, &a) || !c.expect("x") || !parse_type(c, &b) || !c.expect("->") || !parse_type(c, &rt))
      return false;
    tys = {a, b};
  } else {
    for (size_t k = 0; k < nin; ++k) {
      if (!parse_type(c, &t)) return false;
      tys.push_back(t);
      if (k + 1 < nin && !c.expect(",")) return false;
    }
    if (!c.expect("->") || !parse_type(c, &rt)) return false;
  }
  for (size_t k = 0; k < nin; ++k) {
    if (op->operands[k]->type != tys[k]) {
      c.fail("operand #" + std::to_string(k) + " of '" + name + "' has type " + op->operands[k]->type.str() +
             " but the op declares " + tys[k].str());
      return false;
    }
    op->operands[k]->users.push_back(op);
  }
  op->result = m.new_value(rt);
  op->result->def = op;
  op->result->src_name = res_name;
  if (res_name.empty()) {
    c.fail("'" + name + "' must name its result");
    return false;
  }
  sc.names[res_name] = op->result;
  f.body.push_back(op);
  return true;
}

bool parse_func(Cursor& c, Module& m) {
  Func f;
  if (!c.expect("@")) return false;
  f.name = c.ident();
  if (!c.expect("(")) return false;
  Scope sc;
  if (!c.accept(")")) {
    while (true) {
      if (!c.expect("%")) return false;
      std::string an = c.ident();
      if (!c.expect(":")) return false;
      TensorType t;
      if (!parse_type(c, &t)) return false;
      std::map<std::string, std::string> argattrs;
      if (!parse_attr_dict(c, &argattrs)) return false;
      Value* v = m.new_value(t);
      v->arg_index = static_cast<int>(f.args.size());
      v->src_name = an;
      f.args.push_back(v);
      sc.names[an] = v;
      if (c.accept(",")) continue;
      if (!c.expect(")")) return false;
      break;
    }
  }
  if (c.accept("->")) {
    if (c.accept("(")) {
      if (!c.accept(")")) {
        while (true) {
          TensorType t;
          if (!parse_type(c, &t)) return false;
          f.results.push_back(t);
          if (c.accept(",")) continue;
          if (!c.expect(")")) return false;
          break;
        }
      }
    } else {
      TensorType t;
      if (!parse_type(c, &t)) return false;
      f.results.push_back(t);
    }
  }
  if (c.accept("attributes")) {
    std::map<std::string, std::string> fa;
    if (!parse_attr_dict(c, &fa)) return false;
  }
  if (!c.expect("{")) return false;
  while (!c.accept("}")) {
    if (c.eof()) {
      c.fail("unterminated function body");
      return false;
    }
    if (!parse_op(c, m, f, sc)) return false;
  }
  m.funcs.push_back(std::move(f));
  return true;
}

}  // namespace

std::unique_ptr<Module> parse_module(const std::string& text, std::string* err) {
  auto m = std::make_unique<Module>();
  Cursor c(text);
  bool wrapped = false;
  if (c.accept("module")) {
    wrapped = true;
    if (c.peek("@")) {
      c.accept("@");
      c.ident();
    }
    if (c.accept("attributes") && !parse_attr_dict(c, &m->attrs)) {
      *err = c.err;
      return nullptr;
    }
    if (!c.expect("{")) {
      *err = c.err;
      return nullptr;
    }
  }
  while (true) {
    if (wrapped && c.accept("}")) break;
    if (c.eof()) {
      if (wrapped) c.fail("unterminated module");
      break;
    }
    if (!c.accept("tensixflow.func")) {
      c.fail("expected 'tensixflow.func'");
      break;
    }
    if (!parse_func(c, *m)) break;
  }
  if (!c.err.empty()) {
    *err = c.err;
    return nullptr;
  }
  return m;
}

// ------------------------------------------------------------------ printing

std::string print_module(const Module& m) {
  std::ostringstream os;
  os << "module ";
  if (!m.attrs.empty()) {
    os << "attributes {";
    bool first = true;
    for (const auto& [k, v] : m.attrs) {
      os << (first ? "" : ", ") << k << " = " << v;
      first = false;
    }
    os << "} ";
  }
  os << "{\n";
  for (const Func& f : m.funcs) {
    std::map<const Value*, std::string> names;
    os << "  tensixflow.func @" << f.name << "(";
    for (size_t k = 0; k < f.args.size(); ++k) {
      names[f.args[k]] = "%arg" + std::to_string(k);
      os << (k ? ", " : "") << names[f.args[k]] << ": " << f.args[k]->type.str();
    }
    os << ")";
    if (f.results.size() == 1) {
      os << " -> " << f.results[0].str();
    } else if (f.results.size() > 1) {
      os << " -> (";
      for (size_t k = 0; k < f.results.size(); ++k) os << (k ? ", " : "") << f.results[k].str();
      os << ")";
    }
    os << " {\n";
    int next = 0;
    auto nm = [&](const Value* v) { return names.count(v) ? names[v] : std::string("%<dead>"); };
    for (const Op* op : f.body) {
      if (op->erased) continue;
      os << "    ";
      if (op->result) {
        names[op->result] = "%" + std::to_string(next++);
        os << names[op->result] << " = ";
      }
      os << op->name;
      if (op->name == "tensixflow.constant") {
        os << " " << op->attrs.at("value");
        std::map<std::string, std::string> rest = op->attrs;
        rest.erase("value");
        if (!rest.empty()) {
          os << " {";
          bool first = true;
          for (const auto& [k, v] : rest) {
            os << (first ? "" : ", ") << k << " = " << v;
            first = false;
          }
          os << "}";
        }
        os << "\n";
        continue;
      }
      for (size_t k = 0; k < op->operands.size(); ++k) os << (k ? ", " : " ") << nm(op->operands[k]);
      if (!op->attrs.empty()) {
        os << " {";
        bool first = true;
        for (const auto& [k, v] : op->attrs) {
          os << (first ? "" : ", ") << k;
          if (v != "unit") os << " = " << v;
          first = false;
        }
        os << "}";
      }
      if (op->name == "tensixflow.return") {
        if (!op->operands.empty()) {
          os << " :";
          for (size_t k = 0; k < op->operands.size(); ++k) os << (k ? ", " : " ") << op->operands[k]->type.str();
        }
      } else if (op->name == "tensixflow.add" || op->name == "tensixflow.gelu") {
        os << " : " << op->operands[0]->type.str();
      } else if (op->name == "tensixflow.matmul") {
        os << " : " << op->operands[0]->type.str() << " x " << op->operands[1]->type.str() << " -> "
           << op->result->type.str();
      } else {
        os << " :";
        for (size_t k = 0; k < op->operands.size(); ++k) os << (k ? ", " : " ") << op->operands[k]->type.str();
        os << " -> " << op->result->type.str();
      }
      os << "\n";
    }
    os << "  }\n";
  }
  os << "}\n";
  return os.str();
}

// ----------------------------------------------------------------- verifying

namespace {

std::string op_error(const Op* op, const std::string& msg) { return "'" + op->name + "' op " + msg; }

bool dyn(int64_t d) { return d < 0; }

std::string verify_op(const Op* op) {
  auto T = [&](size_t k) -> const TensorType& { return op->operands[k]->type; };
  const std::string& n = op->name;
  if (n == "tensixflow.add") {
    if (T(0) != T(1) || T(0) != op->result->type) return op_error(op, "requires the same type for all operands and results");
    return "";
  }
  if (n == "tensixflow.gelu") {
    if (T(0) != op->result->type) return op_error(op, "requires the same type for all operands and results");
    return "";
  }
  if (n == "tensixflow.matmul") {
    const TensorType &a = T(0), &b = T(1);
    if (a.shape.size() < 2 || b.shape.size() < 2) return op_error(op, "expected operands of rank >= 2");
    if (a.elem != b.elem) return op_error(op, "expected lhs and rhs element types to match");
    const int64_t ka = a.shape.back(), kb = b.shape[b.shape.size() - 2];
    if (!dyn(ka) && !dyn(kb) && ka != kb)
      return op_error(op, "mismatched contracting dimensions: lhs K = " + std::to_string(ka) + " but rhs K = " +
                              std::to_string(kb));
    std::vector<int64_t> want(a.shape.begin(), a.shape.end() - 1);
    want.push_back(b.shape.back());
    if (op->result->type.shape != want) return op_error(op, "result shape does not match [..., M, N]");
    return "";
  }
  if (n == "tensixflow.rmsnorm") {
    const TensorType &x = T(0), &g = T(1);
    if (x.shape.empty()) return op_error(op, "expected input of rank >= 1");
    if (g.shape.size() != 1) return op_error(op, "gamma must be a 1-D tensor, got rank " + std::to_string(g.shape.size()));
    if (!dyn(g.shape[0]) && !dyn(x.shape.back()) && g.shape[0] != x.shape.back())
      return op_error(op, "gamma size (" + std::to_string(g.shape[0]) + ") must match the input's last dimension (" +
                              std::to_string(x.shape.back()) + ")");
    if (op->result->type != x) return op_error(op, "result type must equal the input type");
    return "";
  }
  if (n == "tensixflow.fused_rmsnorm_matmul") {
    const TensorType &x = T(0), &g = T(1), &w = T(2);
    if (x.shape.size() < 2) return op_error(op, "expected input to have rank >= 2, got " + std::to_string(x.shape.size()));
    if (w.shape.size() < 2) return op_error(op, "expected weight to have rank >= 2, got " + std::to_string(w.shape.size()));
    if (g.shape.size() != 1) return op_error(op, "gamma must be a 1-D tensor, got rank " + std::to_string(g.shape.size()));
    if (x.elem != g.elem || x.elem != w.elem)
      return op_error(op, "expected input, gamma, and weight element types to match, got " + x.elem + ", " + g.elem +
                              ", and " + w.elem);
    const int64_t k = x.shape.back();
    if (!dyn(k) && !dyn(g.shape[0]) && g.shape[0] != k)
      return op_error(op, "gamma size (" + std::to_string(g.shape[0]) + ") must match the input's last dimension (" +
                              std::to_string(k) + ")");
    const int64_t wk = w.shape[w.shape.size() - 2];
    if (!dyn(k) && !dyn(wk) && k != wk)
      return op_error(op, "mismatched contracting dimensions: input K = " + std::to_string(k) + " but weight K = " +
                              std::to_string(wk));
    std::vector<int64_t> want(x.shape.begin(), x.shape.end() - 1);
    want.push_back(w.shape.back());
    if (op->result->type.shape != want) return op_error(op, "result shape must be the input's leading dimensions and the weight's last");
    return "";
  }
  if (n == "tensixflow.fused_mlp") {
    const TensorType &x = T(0), &g = T(1), &w1 = T(2), &b1 = T(3), &w2 = T(4), &r = T(5);
    if (x.shape.size() < 2) return op_error(op, "expected input to have rank >= 2, got " + std::to_string(x.shape.size()));
    if (g.shape.size() != 1) return op_error(op, "gamma must be a 1-D tensor, got rank " + std::to_string(g.shape.size()));
    if (w1.shape.size() < 2) return op_error(op, "expected w1 to have rank >= 2, got " + std::to_string(w1.shape.size()));
    if (w2.shape.size() < 2) return op_error(op, "expected w2 to have rank >= 2, got " + std::to_string(w2.shape.size()));
    if (b1.shape.empty()) return op_error(op, "b1 must have rank >= 1, got rank 0");
    for (const TensorType* t : {&g, &w1, &b1, &w2, &r})
      if (t->elem != x.elem)
        return op_error(op, "expected input, gamma, w1, b1, w2, and residual element types to match");
    const int64_t k = x.shape.back();
    if (!dyn(k) && !dyn(g.shape[0]) && g.shape[0] != k)
      return op_error(op, "gamma size (" + std::to_string(g.shape[0]) + ") must match the input's last dimension (" +
                              std::to_string(k) + ")");
    const int64_t w1k = w1.shape[w1.shape.size() - 2], h = w1.shape.back();
    if (!dyn(k) && !dyn(w1k) && k != w1k)
      return op_error(op, "mismatched contracting dimensions: input K = " + std::to_string(k) + " but w1 K = " +
                              std::to_string(w1k));
    if (!dyn(h) && !dyn(b1.shape.back()) && b1.shape.back() != h)
      return op_error(op, "b1 last dimension (" + std::to_string(b1.shape.back()) + ") must match w1's hidden dimension (" +
                              std::to_string(h) + ")");
    if (b1.shape.size() > 1) {
      std::vector<int64_t> want(x.shape.begin(), x.shape.end() - 1);
      want.push_back(h);
      if (b1.shape != want) return op_error(op, "a full-rank b1 must have shape [..., H]");
    }
    const int64_t w2h = w2.shape[w2.shape.size() - 2];
    if (!dyn(h) && !dyn(w2h) && h != w2h)
      return op_error(op, "mismatched hidden dimensions: w1 H = " + std::to_string(h) + " but w2 H = " +
                              std::to_string(w2h));
    std::vector<int64_t> out(x.shape.begin(), x.shape.end() - 1);
    out.push_back(w2.shape.back());
    if (r.shape != out) return op_error(op, "residual shape must equal the output shape");
    if (op->result->type != r) return op_error(op, "result type must equal the residual type");
    return "";
  }
  return "";
}

}  // namespace

std::string verify_module(const Module& m, int* line) {
  for (const Func& f : m.funcs) {
    const Op* ret = nullptr;
    for (const Op* op : f.body) {
      if (op->erased) continue;
      std::string e = verify_op(op);
      if (!e.empty()) {
        if (line) *line = op->line;
        return e;
      }
      if (op->name == "tensixflow.return") ret = op;
    }
    if (!ret) return "'tensixflow.func' op @" + f.name + " has no tensixflow.return";
    if (ret->operands.size() != f.results.size())
      return "'tensixflow.return' op has " + std::to_string(ret->operands.size()) + " operands, but the function returns " +
             std::to_string(f.results.size());
    for (size_t k = 0; k < f.results.size(); ++k)
      if (ret->operands[k]->type != f.results[k])
        return "'tensixflow.return' op type of operand #" + std::to_string(k) + " (" + ret->operands[k]->type.str() +
               ") does not match the function result type (" + f.results[k].str() + ")";
  }
  return "";
}

}  // namespace tfb200::front
