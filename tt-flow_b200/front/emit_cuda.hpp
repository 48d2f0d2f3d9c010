// --tensixflow-emit-cuda=output-dir=<dir>: standalone CUDA project of a planned graph.
#pragma once

#include <string>

#include "ir.hpp"
#include "plan.hpp"

namespace tfb200::front {

// Writes host.cpp, Makefile, run.sh, README.md and plan.json into `dir`.
// Refuses (nothing written) when the plan is not fused_feasible.
bool emit_cuda_project(const Module& m, const B200Plan& plan, const std::string& dir, std::string* err);

}  // namespace tfb200::front
