// --tensixflow-import-ttir: bare-tensor TTIR to the tensixflow dialect subset.
#pragma once

#include <memory>
#include <string>

#include "ir.hpp"

namespace tfb200::front {

// Import one func.func of generic ttir.{matmul, add, gelu, rms_norm} ops.
// Returns nullptr and sets *err ("line:col: error: ...") outside the subset.
std::unique_ptr<Module> import_ttir(const std::string& text, std::string* err);

}  // namespace tfb200::front
