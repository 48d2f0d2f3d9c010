// Minimal IR for the tensixflow dialect subset that reaches the fused hot path:
// tensixflow.func / return / constant / add / gelu / matmul / rmsnorm /
// fused_rmsnorm_matmul / fused_mlp (tensixflow include/tensixflow/
// TensixflowOps.td:30-288), parsed from and printed to the dialect's textual
// form so that `tfb200-opt` can stand in for `tensixflow-opt` on the passes this
// backend implements. Host-only C++ (no MLIR dependency).
#pragma once

#include <cstdint>
#include <map>
#include <memory>
#include <optional>
#include <string>
#include <vector>

namespace tfb200::front {

struct TensorType {
  std::vector<int64_t> shape;  // -1 for a dynamic extent ('?')
  std::string elem;            // "bf16", "f32", "f16", ...
  bool ranked = true;
  int64_t elements() const;
  int bytes_per_element() const;
  std::string str() const;
  bool operator==(const TensorType& o) const { return shape == o.shape && elem == o.elem; }
  bool operator!=(const TensorType& o) const { return !(*this == o); }
};

struct Op;

struct Value {
  TensorType type;
  Op* def = nullptr;   // nullptr for a function argument
  int arg_index = -1;  // function argument index
  std::vector<Op*> users;
  std::string src_name;  // name in the parsed text (without '%')
};

struct Op {
  std::string name;  // e.g. "tensixflow.matmul"
  std::vector<Value*> operands;
  Value* result = nullptr;
  std::map<std::string, std::string> attrs;  // name -> printed value (sorted)
  bool erased = false;
  int line = 0;  // 1-based source line (0 for ops created by passes)
};

struct Func {
  std::string name;
  std::vector<Value*> args;
  std::vector<TensorType> results;
  std::vector<Op*> body;  // in order; the last op is tensixflow.return
};

struct Module {
  std::map<std::string, std::string> attrs;
  std::vector<Func> funcs;
  std::vector<std::unique_ptr<Value>> values;
  std::vector<std::unique_ptr<Op>> ops;

  Value* new_value(const TensorType& t);
  Op* new_op(const std::string& name);
};

// Parse the textual form. Returns nullopt and sets *err on failure.
std::unique_ptr<Module> parse_module(const std::string& text, std::string* err);
// Print in the dialect's generic-printer layout (module attributes sorted,
// SSA values renumbered %argN / %N as MLIR's printer does).
std::string print_module(const Module& m);
// Structural and shape verification of every op (the dialect's verifiers,
// TensixflowOps.cpp:197-413). Returns an error message or "" and, on error,
// the source line of the offending op in *line.
std::string verify_module(const Module& m, int* line = nullptr);

// Helpers shared by the passes.
void erase_op(Op* op);
void replace_all_uses(Value* from, Value* to);
std::string i64_attr(int64_t v);

}  // namespace tfb200::front
