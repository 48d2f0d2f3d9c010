// tfb200-opt: the tensixflow-opt / tensixflow-translate entry points of the B200
// backend for the fused path (tensixflow tools/tensixflow-opt/tensixflow-opt.cpp,
// tools/tensixflow-translate/tensixflow-translate.cpp:291-297).
//
//   tfb200-opt [--tensixflow-device=b200] [--tensixflow-fuse-rmsnorm-matmul]
//              [--tensixflow-plan-noc-sharding] [--tensixflow-allocate-circular-buffers]
//              [--tensixflow-to-json] [-o out] [input.mlir | -]
//
// Exit status 0 on success; diagnostics and the planner report go to stderr.
#include <fstream>
#include <iostream>
#include <iterator>
#include <sstream>
#include <string>
#include <vector>

#include "passes.hpp"

int main(int argc, char** argv) {
  std::vector<std::string> flags;
  std::string input = "-", output;
  for (int i = 1; i < argc; ++i) {
    std::string a = argv[i];
    if (a == "-o" && i + 1 < argc) {
      output = argv[++i];
    } else if (a.rfind("--", 0) == 0 || a == "-verify-diagnostics") {
      flags.push_back(a);
    } else {
      input = a;
    }
  }
  std::string text;
  if (input == "-") {
    text.assign(std::istreambuf_iterator<char>(std::cin), std::istreambuf_iterator<char>());
  } else {
    std::ifstream f(input);
    if (!f) {
      std::cerr << "could not open input file '" << input << "'\n";
      return 1;
    }
    text.assign(std::istreambuf_iterator<char>(f), std::istreambuf_iterator<char>());
  }
  const auto r = tfb200::front::run_pipeline(text, flags);
  if (!r.diag.empty()) std::cerr << r.diag << (r.diag.back() == '\n' ? "" : "\n");
  if (!r.ok) return 1;
  if (output.empty()) {
    std::cout << r.output;
  } else {
    std::ofstream o(output);
    o << r.output;
  }
  return 0;
}
