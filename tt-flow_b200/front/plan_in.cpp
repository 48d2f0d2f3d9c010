// Plan JSON in: re-plans a graph described by a plan document (schema/plan.schema.json,
// as tensixflow-translate --tensixflow-to-json writes it for any device,
// tools/tensixflow-translate/tensixflow-translate.cpp:75-222) for the B200. The
// document's `tensors` give the problem; its device block and numbers are ignored.
// Tensor roles are taken from the names this front end writes (input, gamma,
// weight / w1, b1, w2, residual, lhs, rhs, output) or, for the reference's
// argument names (arg0, arg1, ...), from the shapes: X is the first tensor of rank
// >= 2, then the weights chain on the inner dimension (W[K, N] or W1[K, H],
// W2[H, N]).
#include "plan_in.hpp"

#include <cctype>
#include <cstdlib>
#include <map>

namespace tfb200::front {

namespace {

struct Parser {
  const std::string& s;
  size_t i = 0;
  std::string err;

  explicit Parser(const std::string& t) : s(t) {}

  void ws() {
    while (i < s.size() && std::isspace(static_cast<unsigned char>(s[i]))) ++i;
  }
  bool fail(const std::string& what) {
    if (err.empty()) {
      size_t line = 1, col = 1;
      for (size_t k = 0; k < i && k < s.size(); ++k) {
        if (s[k] == '\n') {
          ++line;
          col = 1;
        } else {
          ++col;
        }
      }
      err = "plan JSON " + std::to_string(line) + ":" + std::to_string(col) + ": " + what;
    }
    return false;
  }
  bool lit(const char* w) {
    size_t n = 0;
    while (w[n]) ++n;
    if (s.compare(i, n, w) != 0) return false;
    i += n;
    return true;
  }
  bool str(std::string* out) {
    if (i >= s.size() || s[i] != '"') return fail("expected a string");
    ++i;
    out->clear();
    while (i < s.size() && s[i] != '"') {
      char c = s[i++];
      if (c == '\\') {
        if (i >= s.size()) return fail("unterminated escape");
        const char e = s[i++];
        switch (e) {
          case '"': c = '"'; break;
          case '\\': c = '\\'; break;
          case '/': c = '/'; break;
          case 'b': c = '\b'; break;
          case 'f': c = '\f'; break;
          case 'n': c = '\n'; break;
          case 'r': c = '\r'; break;
          case 't': c = '\t'; break;
          case 'u': {
            if (i + 4 > s.size()) return fail("short \\u escape");
            const unsigned long cp = std::strtoul(s.substr(i, 4).c_str(), nullptr, 16);
            i += 4;
            c = cp < 0x80 ? static_cast<char>(cp) : '?';  // names and enums here are ASCII
            break;
          }
          default:
            return fail("bad escape");
        }
      }
      out->push_back(c);
    }
    if (i >= s.size()) return fail("unterminated string");
    ++i;
    return true;
  }
  bool value(JVal* v) {
    ws();
    if (i >= s.size()) return fail("unexpected end of input");
    const char c = s[i];
    if (c == '{') {
      v->kind = JVal::kObj;
      ++i;
      ws();
      if (i < s.size() && s[i] == '}') {
        ++i;
        return true;
      }
      for (;;) {
        ws();
        std::string key;
        if (!str(&key)) return false;
        ws();
        if (i >= s.size() || s[i] != ':') return fail("expected ':'");
        ++i;
        JVal member;
        if (!value(&member)) return false;
        v->obj.emplace_back(std::move(key), std::move(member));
        ws();
        if (i < s.size() && s[i] == ',') {
          ++i;
          continue;
        }
        if (i < s.size() && s[i] == '}') {
          ++i;
          return true;
        }
        return fail("expected ',' or '}'");
      }
    }
    if (c == '[') {
      v->kind = JVal::kArr;
      ++i;
      ws();
      if (i < s.size() && s[i] == ']') {
        ++i;
        return true;
      }
      for (;;) {
        JVal item;
        if (!value(&item)) return false;
        v->arr.push_back(std::move(item));
        ws();
        if (i < s.size() && s[i] == ',') {
          ++i;
          continue;
        }
        if (i < s.size() && s[i] == ']') {
          ++i;
          return true;
        }
        return fail("expected ',' or ']'");
      }
    }
    if (c == '"') {
      v->kind = JVal::kStr;
      return str(&v->text);
    }
    if (lit("true")) {
      v->kind = JVal::kBool;
      v->b = true;
      return true;
    }
    if (lit("false")) {
      v->kind = JVal::kBool;
      v->b = false;
      return true;
    }
    if (lit("null")) {
      v->kind = JVal::kNull;
      return true;
    }
    if (c == '-' || std::isdigit(static_cast<unsigned char>(c))) {
      const size_t b = i;
      if (s[i] == '-') ++i;
      while (i < s.size() && (std::isdigit(static_cast<unsigned char>(s[i])) || s[i] == '.' || s[i] == 'e' ||
                              s[i] == 'E' || s[i] == '+' || s[i] == '-'))
        ++i;
      v->kind = JVal::kNum;
      v->text = s.substr(b, i - b);
      return true;
    }
    return fail(std::string("unexpected character '") + c + "'");
  }
};

bool as_int(const JVal& v, int64_t* out) {
  if (v.kind != JVal::kNum) return false;
  char* end = nullptr;
  const long long x = std::strtoll(v.text.c_str(), &end, 10);
  if (!end || *end != '\0') return false;  // integers only
  *out = x;
  return true;
}

int bytes_of(const std::string& dtype) { return dtype == "fp32" || dtype == "f32" ? 4 : 2; }

int64_t rows_of(const std::vector<int64_t>& shape) {
  int64_t r = 1;
  for (size_t k = 0; k + 1 < shape.size(); ++k) r *= shape[k];
  return r;
}

}  // namespace

const JVal* JVal::get(const std::string& key) const {
  for (const auto& kv : obj)
    if (kv.first == key) return &kv.second;
  return nullptr;
}

bool parse_json(const std::string& text, JVal* out, std::string* err) {
  Parser p(text);
  if (!p.value(out)) {
    *err = p.err;
    return false;
  }
  p.ws();
  if (p.i != text.size()) {
    p.fail("trailing characters after the document");
    *err = p.err;
    return false;
  }
  return true;
}

bool request_from_plan_json(const std::string& text, PlanRequest* r, std::string* err) {
  JVal root;
  if (!parse_json(text, &root, err)) return false;
  if (root.kind != JVal::kObj) {
    *err = "plan JSON: the document is not an object";
    return false;
  }
  const JVal* gid = root.get("graph_id");
  r->graph_id = gid && gid->kind == JVal::kStr ? gid->text : "graph";
  const JVal* tens = root.get("tensors");
  if (!tens || tens->kind != JVal::kArr) {
    *err = "plan JSON: no \"tensors\" array";
    return false;
  }
  r->tensors.clear();
  for (const JVal& t : tens->arr) {
    if (t.kind != JVal::kObj) {
      *err = "plan JSON: a tensor is not an object";
      return false;
    }
    PlanTensor pt;
    const JVal* nm = t.get("name");
    const JVal* sh = t.get("shape");
    const JVal* dt = t.get("dtype");
    const JVal* pl = t.get("placement");
    if (!nm || nm->kind != JVal::kStr || !sh || sh->kind != JVal::kArr) {
      *err = "plan JSON: a tensor needs \"name\" and \"shape\"";
      return false;
    }
    pt.name = nm->text;
    for (const JVal& d : sh->arr) {
      int64_t x = 0;
      if (!as_int(d, &x) || x < 0) {
        *err = "plan JSON: tensor " + pt.name + " has a shape entry that is not a non-negative integer";
        return false;
      }
      pt.shape.push_back(x);
    }
    pt.dtype = dt && dt->kind == JVal::kStr ? dt->text : "bf16";
    pt.placement = pl && pl->kind == JVal::kStr ? pl->text : "DRAM";
    r->tensors.push_back(pt);
  }
  const JVal* fu = root.get("fusion");
  std::string fusion = fu && fu->kind == JVal::kStr ? fu->text : "";

  // Roles by the names this front end writes.
  std::map<std::string, const PlanTensor*> by;
  for (const PlanTensor& t : r->tensors) by[t.name] = &t;
  const PlanTensor* x = by.count("input") ? by["input"] : (by.count("lhs") ? by["lhs"] : nullptr);
  const PlanTensor* w = by.count("weight") ? by["weight"] : (by.count("rhs") ? by["rhs"] : nullptr);
  const PlanTensor* w1 = by.count("w1") ? by["w1"] : nullptr;
  const PlanTensor* w2 = by.count("w2") ? by["w2"] : nullptr;
  const PlanTensor* gamma = by.count("gamma") ? by["gamma"] : nullptr;
  if (!x) {
    // The reference's argument names: roles from the shapes.
    for (const PlanTensor& t : r->tensors)
      if (t.shape.size() >= 2) {
        x = &t;
        break;
      }
    if (!x) {
      *err = "plan JSON: no tensor of rank >= 2 to take as the input";
      return false;
    }
    const int64_t K = x->shape.back();
    for (const PlanTensor& t : r->tensors)
      if (&t != x && t.shape.size() == 2 && t.shape[0] == K) {
        w1 = &t;
        break;
      }
    if (w1)
      for (const PlanTensor& t : r->tensors)
        if (&t != x && &t != w1 && t.shape.size() == 2 && t.shape[0] == w1->shape[1]) {
          w2 = &t;
          break;
        }
    for (const PlanTensor& t : r->tensors)
      if (t.shape.size() == 1 && t.shape[0] == K) {
        gamma = &t;
        break;
      }
    if (fusion.empty()) fusion = w2 ? "fused_mlp" : (gamma ? "fused_rmsnorm_matmul" : "none");
    if (fusion != "fused_mlp") {
      w = w1;
      w1 = w2 = nullptr;
    }
  }
  if (fusion.empty()) fusion = w1 && w2 ? "fused_mlp" : (gamma ? "fused_rmsnorm_matmul" : "none");
  r->fusion = fusion;
  r->already_fused = fusion != "none";
  r->M = rows_of(x->shape);
  r->K = x->shape.back();
  r->bpe = bytes_of(x->dtype);
  if (fusion == "fused_mlp") {
    if (!w1 || !w2 || w1->shape.size() != 2 || w2->shape.size() != 2 || w1->shape[0] != r->K ||
        w2->shape[0] != w1->shape[1]) {
      *err = "plan JSON: fused_mlp needs weights W1[K, H] and W2[H, N] that chain on the input's K";
      return false;
    }
    r->H = w1->shape[1];
    r->N = w2->shape[1];
    return true;
  }
  if (fusion != "fused_rmsnorm_matmul" && fusion != "none") {
    *err = "plan JSON: unknown fusion \"" + fusion + "\"";
    return false;
  }
  if (!w || w->shape.size() != 2 || w->shape[0] != r->K) {
    *err = "plan JSON: " + fusion + " needs a weight W[K, N] that chains on the input's K";
    return false;
  }
  r->N = w->shape[1];
  return true;
}

}  // namespace tfb200::front
