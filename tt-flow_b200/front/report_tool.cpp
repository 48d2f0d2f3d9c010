// tfb200-report: the plan report of the B200 backend, with the command line of
// the reference's report tool (tensixflow tools/tensixflow-report).
//
//   tfb200-report --in plan.json --out report.html
//
// Exit status 0 with the page written. Exit status 1 with the reason on stderr
// and nothing written when the plan is refused (no emission block, an unknown
// mapping, or emission numbers that disagree with the planner's projection).
#include <fstream>
#include <iostream>
#include <iterator>
#include <string>

#include "report.hpp"

int main(int argc, char** argv) {
  std::string in, out;
  for (int i = 1; i < argc; ++i) {
    const std::string a = argv[i];
    if (a == "--in" && i + 1 < argc) {
      in = argv[++i];
    } else if (a == "--out" && i + 1 < argc) {
      out = argv[++i];
    } else if (a.rfind("--in=", 0) == 0) {
      in = a.substr(5);
    } else if (a.rfind("--out=", 0) == 0) {
      out = a.substr(6);
    } else {
      std::cerr << "usage: tfb200-report --in plan.json --out report.html\n";
      return 2;
    }
  }
  if (in.empty() || out.empty()) {
    std::cerr << "usage: tfb200-report --in plan.json --out report.html\n";
    return 2;
  }
  std::ifstream f(in);
  if (!f) {
    std::cerr << "could not open plan '" << in << "'\n";
    return 1;
  }
  const std::string text((std::istreambuf_iterator<char>(f)), std::istreambuf_iterator<char>());
  const auto r = tfb200::front::report_plan(text);
  if (!r.ok) {
    std::cerr << "tfb200-report: " << in << ": " << r.diag << "\n";
    return 1;
  }
  std::ofstream o(out);
  if (!(o << r.html)) {
    std::cerr << "could not write '" << out << "'\n";
    return 1;
  }
  return 0;
}
