// Pipeline driver of the tensixflow front end on the B200 backend.
#pragma once

#include <string>
#include <vector>

namespace tfb200::front {

struct PipelineResult {
  bool ok = false;
  std::string output;  // printed IR, or plan JSON with --tensixflow-to-json
  std::string diag;    // errors, and the planner's report lines
};

// Parse `text`, apply the flags in order (tensixflow-opt style) and print.
PipelineResult run_pipeline(const std::string& text, const std::vector<std::string>& args);
PipelineResult run_pipeline(const std::string& text, const std::string& args);

}  // namespace tfb200::front
